// abi_util.h -- error reporting helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stddef.h>

namespace nvfp4 {

// Records a printf-style message as the thread's last error; returns `code`.
int fail(int code, const char *fmt, ...);
// NVFP4_OK, or NVFP4_ERR_CUDA with the CUDA error text recorded.
int check_launch(cudaError_t e, const char *what);
bool aligned(const void *p, size_t a);

// An NVTX range named after the C-ABI call it wraps, so that Nsight tools
// (ncu --nvtx, nsys) attribute the kernels to the entry point that launched
// them.  Header-only NVTX: without a tool attached each push/pop is a few
// nanoseconds and nothing is loaded.
struct AbiRange {
  explicit AbiRange(const char *name) { nvtxRangePushA(name); }
  ~AbiRange() { nvtxRangePop(); }
  AbiRange(const AbiRange &) = delete;
  AbiRange &operator=(const AbiRange &) = delete;
};
#define NVFP4_ABI_RANGE() ::nvfp4::AbiRange nvfp4_abi_range_(__func__)

}  // namespace nvfp4
