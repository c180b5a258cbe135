"""Regenerate the golden fixtures in this folder.

reference_kats.json -- the known-answer tests of the reference, read as text
  from its test sources (the reference is Mojo and cannot be run here):
    tests/test_nvfp4.mojo:44-62   FP4_E2M1_LUT entries
    tests/test_nvfp4.mojo:65-75   pack_fp4_pair / unpack_fp4_pair
    tests/test_nvfp4.mojo:78-90   dequant_fp4 at scales 1.0 and 2.0
    tests/test_nvfp4.mojo:93-115  NvFp4Config defaults, group size, pack factor
    tests/test_deltanet.mojo:65-76 sigmoid / silu
    tests/helpers.mojo:4-28       tolerance of expect_close (abs or rel 1e-4)
e4m3_table.json -- float8_e4m3fn -> float32 for all 256 codes from ml_dtypes
  (an implementation independent of the oracle), NaN written as "nan".

Usage: python tests/golden/make_golden.py <path-to-reference-checkout>
"""
from __future__ import annotations

import json
import math
import re
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _num(s: str) -> float:
    return float(s)


def parse_reference(ref: Path) -> dict:
    t_nvfp4 = (ref / "tests" / "test_nvfp4.mojo").read_text()
    t_dn = (ref / "tests" / "test_deltanet.mojo").read_text()
    helpers = (ref / "tests" / "helpers.mojo").read_text()

    lut = {}
    for m in re.finditer(r"expect_close\(FP4_E2M1_LUT\[(\d+)\],\s*([-0-9.e]+)", t_nvfp4):
        lut[int(m.group(1))] = m.group(2)
    assert sorted(lut) == list(range(16)), lut

    m = re.search(r"pack_fp4_pair\(UInt8\((\d+)\),\s*UInt8\((\d+)\)\)", t_nvfp4)
    lo, hi = int(m.group(1)), int(m.group(2))
    m2 = re.search(r"packed,\s*UInt8\((\d+)\)", t_nvfp4)
    packed = int(m2.group(1))

    # dequant_fp4 KATs: walk the test body in order, tracking `scale = ...`.
    body = t_nvfp4[t_nvfp4.index("def test_dequant"):t_nvfp4.index("def test_config")]
    dequant = []
    scale = None
    for line in body.splitlines():
        ms = re.search(r"scale(?::\s*Float32)?\s*=\s*([-0-9.e]+)", line)
        if ms and "expect_close" not in line:
            scale = float(ms.group(1))
        md = re.search(r"dequant_fp4\(UInt8\((\d+)\),\s*scale\),\s*([-0-9.e]+)", line)
        if md:
            dequant.append({"code": int(md.group(1)), "scale": scale,
                             "expected": float(md.group(2))})

    cfg = {
        "pack_factor": int(re.search(r"assert_equal\(NVFP4_PACK_FACTOR,\s*(\d+)", t_nvfp4).group(1)),
        "weight_dtype": re.search(r"config\.weight_dtype,\s*DType\.(\w+)", t_nvfp4).group(1),
        "scale_dtype": re.search(r"config\.scale_dtype,\s*DType\.(\w+)", t_nvfp4, re.S).group(1),
        "output_dtype": re.search(r"config\.output_dtype,\s*DType\.(\w+)", t_nvfp4, re.S).group(1),
    }
    cfg_src = (ref / "nvfp4" / "config.mojo").read_text()
    cfg["group_size"] = int(re.search(r"NVFP4_GROUP_SIZE: Int = (\d+)", cfg_src).group(1))

    act = {"sigmoid": [], "silu": []}
    for fn in ("sigmoid", "silu"):
        for m in re.finditer(rf"expect_close\({fn}\(([-0-9.e]+)\),\s*([-0-9.e]+)", t_dn):
            act[fn].append({"x": float(m.group(1)), "expected": float(m.group(2))})

    tol = float(re.search(r"tol: Float32 = ([0-9.e-]+)", helpers).group(1))

    return {
        "_source": "read as text from the reference's tests; see make_golden.py",
        "lut": {"citation": "tests/test_nvfp4.mojo:44-62",
                "values": [lut[i] for i in range(16)]},
        "pack_unpack": {"citation": "tests/test_nvfp4.mojo:65-75",
                        "lo": lo, "hi": hi, "packed": packed},
        "dequant": {"citation": "tests/test_nvfp4.mojo:78-90", "cases": dequant},
        "config": {"citation": "tests/test_nvfp4.mojo:93-115, nvfp4/config.mojo:13-14",
                   **cfg},
        "activations": {"citation": "tests/test_deltanet.mojo:65-76", **act},
        "tolerance": {"citation": "tests/helpers.mojo:4-28", "abs_or_rel": tol},
    }


def e4m3_table() -> dict:
    import ml_dtypes
    import numpy as np

    codes = np.arange(256, dtype=np.uint8)
    vals = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    out = []
    for v in vals:
        if math.isnan(v):
            out.append("nan")
        elif v == 0.0 and math.copysign(1.0, v) < 0:
            out.append("-0.0")
        else:
            out.append(repr(float(v)))
    return {"_source": f"ml_dtypes {ml_dtypes.__version__} float8_e4m3fn -> float32",
            "values": out}


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    ref = Path(sys.argv[1])
    (HERE / "reference_kats.json").write_text(json.dumps(parse_reference(ref), indent=1) + "\n")
    (HERE / "e4m3_table.json").write_text(json.dumps(e4m3_table(), indent=0) + "\n")
    print("wrote", HERE / "reference_kats.json", HERE / "e4m3_table.json")


if __name__ == "__main__":
    main()
