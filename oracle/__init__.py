"""CPU oracle of the NVFP4 path (test infrastructure only; see nvfp4_oracle.h)."""
