"""The C ABI library loads, exports every symbol include/nvfp4.h declares, and
its host-side validation rejects bad calls before any CUDA work (CPU only)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        src = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(nvfp4_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ("nvfp4_linear_forward", "nvfp4_gemm_kernel", "nvfp4_matvec",
                 "nvfp4_dequant_tile", "nvfp4_dequant", "nvfp4_last_error_string"):
        assert must in syms


def test_library_exports_every_declared_symbol():
    from nvfp4 import _lib

    L = _lib.load()
    for name in declared_symbols():
        assert hasattr(L, name), f"libnvfp4.so does not export {name}"
        assert name in _lib.SIGNATURES, f"ctypes signature missing for {name}"
    assert L.nvfp4_abi_version() == 1


def test_validation_errors_without_gpu():
    from nvfp4 import _lib

    L = _lib.load()
    desc = _lib.LinearDesc(2048, 1536, 1.0, 1.0, None)
    rc = L.nvfp4_linear_forward(ctypes.byref(desc), None, None, None, 1, None, 1, 4, 0, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG
    assert b"null" in L.nvfp4_last_error_string()
    bad = _lib.LinearDesc(2050, 1536, 1.0, 1.0, None)  # K not a multiple of 16
    rc = L.nvfp4_linear_forward(ctypes.byref(bad), 16, 16, 16, 1, 16, 1, 4, 0, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG
    assert b"multiple of 16" in L.nvfp4_last_error_string()
    rc = L.nvfp4_linear_forward(None, 16, 16, 16, 1, 16, 1, 4, 0, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG
    rc = L.nvfp4_linear_forward(ctypes.byref(desc), 16, 16, 16, 7, 16, 1, 4, 0, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG and b"dtype" in L.nvfp4_last_error_string()
    rc = L.nvfp4_dequant_tile(16, 16, 16, 1024, 128, 0, 1, 4, 64, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG  # odd start_col
    with pytest.raises(_lib.Nvfp4Error):
        _lib.check(_lib.NVFP4_ERR_INVALID_ARG)


def test_shared_expert_and_stack_validation_without_gpu():
    from nvfp4 import _lib

    L = _lib.load()
    desc = _lib.MoEDesc(128, 8, 2048, 768, 1)
    w = _lib.MoEWeightPtrs(16, 16, 16, None, None, 16, 16, None, None)
    # The shared expert's workspace adds its rows to the routed layer's.
    for T in (1, 16, 4096):
        routed = L.nvfp4_moe_workspace_size(ctypes.byref(desc), T)
        assert L.nvfp4_moe_shared_workspace_size(ctypes.byref(desc), 1024, T) > routed
    assert L.nvfp4_moe_shared_workspace_size(ctypes.byref(desc), 1000, 16) == 0  # I % 128
    rc = L.nvfp4_moe_forward_shared(ctypes.byref(desc), ctypes.byref(w), None, 1024, 16, None,
                                    16, 1, 4, None, None, 256, 1 << 30, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG and b"shared" in L.nvfp4_last_error_string()
    bad = _lib.MoEWeightPtrs(None, None, 16, None, None, 16, 16, None, None)
    rc = L.nvfp4_moe_forward_shared(ctypes.byref(desc), ctypes.byref(w), ctypes.byref(bad), 1024,
                                    16, None, 16, 1, 4, None, None, 256, 1 << 30, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG
    rc = L.nvfp4_moe_forward_shared(ctypes.byref(desc), ctypes.byref(w), ctypes.byref(w), 1024,
                                    16, None, 16, 1, 4, None, None, 256, 1024, None)
    assert rc == _lib.NVFP4_ERR_WORKSPACE
    assert L.nvfp4_stack_rows(None, None, 0, 16, None, None) == _lib.NVFP4_OK
    rows = (ctypes.c_int64 * 1)(-1)
    srcs = (ctypes.c_void_p * 1)(16)
    assert L.nvfp4_stack_rows(srcs, rows, 1, 16, 16, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_stack_rows(srcs, rows, 1, 0, 16, None) == _lib.NVFP4_ERR_INVALID_ARG


def test_token_counts_that_would_wrap_are_refused():
    """T * top_k is bounded by 2^24 slots without forming the product, so a
    count near 2^61 cannot wrap into a small, accepted layer."""
    from nvfp4 import _lib

    L = _lib.load()
    desc = _lib.MoEDesc(128, 8, 2048, 768, 1)
    huge = (1 << 61) + 1
    assert L.nvfp4_moe_workspace_size(ctypes.byref(desc), huge) == 0
    assert L.nvfp4_moe_workspace_size(ctypes.byref(desc), (1 << 21) + 1) == 0
    assert L.nvfp4_moe_workspace_size(ctypes.byref(desc), 1 << 21) > 0
    assert L.nvfp4_moe_shared_workspace_size(ctypes.byref(desc), 1024, huge) == 0
    assert L.nvfp4_moe_experts_workspace_size(ctypes.byref(desc), huge) == 0
    w = _lib.MoEWeightPtrs(16, 16, 16, None, None, 16, 16, None, None)
    rc = L.nvfp4_moe_forward_noalloc(ctypes.byref(desc), ctypes.byref(w), 16, None, 16, 1, huge,
                                     None, None, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG and b"token count" in L.nvfp4_last_error_string()
    rc = L.nvfp4_moe_forward(ctypes.byref(desc), ctypes.byref(w), 16, None, 16, 1, huge, None,
                             None, 256, 1 << 40, None)
    assert rc == _lib.NVFP4_ERR_INVALID_ARG and b"token count" in L.nvfp4_last_error_string()
    for fn, args in (("nvfp4_ep_dispatch_plan", (16, huge, 8, 16, 8, 16, 16, 16, 16, None)),):
        assert getattr(L, fn)(*args) == _lib.NVFP4_ERR_INVALID_ARG
    p = _lib.EpPeers()
    p.rank, p.world, p.max_rows, p.hidden, p.timeout_ms = 0, 1, 64, 2048, 0
    p.windows[0] = 1 << 20
    assert L.nvfp4_ep_p2p_dispatch(ctypes.byref(p), 16, 16, huge, 8, 16, None) == \
        _lib.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_ep_p2p_workspace_size(ctypes.byref(desc), ctypes.byref(p), huge) == 0


def test_peer_exchange_validation_without_gpu():
    """include/nvfp4_ep.h host side: window sizes and layout, and the checks
    that refuse a bad peer table before any CUDA work."""
    from nvfp4 import _lib

    L = _lib.load()
    H, k = 2048, 8
    up = lambda v: (v + 255) // 256 * 256
    for world, rows in ((1, 8), (2, 64), (8, 512)):
        n = world * rows
        want = up(up(256 + 4 * n) + 2 * n * H) + 4 * n * H
        assert L.nvfp4_ep_window_size(world, rows, H) == want
    assert L.nvfp4_ep_window_size(9, 8, H) == 0
    assert L.nvfp4_ep_window_size(2, 8, 1000) == 0
    assert L.nvfp4_ep_window_size(2, 0, H) == 0

    def peers(rank=1, world=2, rows=64, wins=(1 << 20, 1 << 30)):
        p = _lib.EpPeers()
        p.rank, p.world, p.max_rows, p.hidden, p.timeout_ms = rank, world, rows, H, 0
        for i, w in enumerate(wins):
            p.windows[i] = w
        return p

    x, e, o = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    p = peers()
    assert L.nvfp4_ep_p2p_rows(ctypes.byref(p), 8, k, ctypes.byref(x), ctypes.byref(e),
                               ctypes.byref(o)) == 0
    base = 1 << 30  # rank 1's own window
    assert e.value == base + 256
    assert x.value == base + up(256 + 4 * 128)
    assert o.value == x.value + up(2 * 128 * H)
    # 9 tokens x 8 slots exceed the 64 rows per rank.
    assert L.nvfp4_ep_p2p_dispatch(ctypes.byref(p), 16, 16, 9, k, 16, None) == \
        _lib.NVFP4_ERR_INVALID_ARG
    assert b"exceed" in L.nvfp4_last_error_string()
    for bad in (peers(rank=2), peers(world=9), peers(wins=(1 << 20, 0)),
                peers(wins=(1 << 20, (1 << 30) + 16))):
        assert L.nvfp4_ep_p2p_dispatch(ctypes.byref(bad), 16, 16, 1, k, 16, None) == \
            _lib.NVFP4_ERR_INVALID_ARG
        assert L.nvfp4_ep_p2p_wait_dispatch(ctypes.byref(bad), None) == _lib.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_ep_p2p_combine(ctypes.byref(p), 16, 16, 1, k, 16, None, 16, 7, None) == \
        _lib.NVFP4_ERR_INVALID_ARG  # output dtype
    desc = _lib.MoEDesc(128, k, H, 768, 1)
    assert L.nvfp4_ep_p2p_workspace_size(ctypes.byref(desc), ctypes.byref(p), 8) > 0
    assert L.nvfp4_ep_p2p_workspace_size(ctypes.byref(_lib.MoEDesc(127, k, H, 768, 1)),
                                         ctypes.byref(p), 8) == 0  # E % world
    assert L.nvfp4_ep_p2p_workspace_size(ctypes.byref(_lib.MoEDesc(128, k, 1024, 768, 1)),
                                         ctypes.byref(p), 8) == 0  # hidden mismatch
    w = _lib.MoEWeightPtrs(16, 16, 16, None, None, 16, 16, None, None)
    rc = L.nvfp4_ep_p2p_forward(ctypes.byref(desc), ctypes.byref(w), ctypes.byref(p), 16, None,
                                16, 1, 8, 256, 1024, None)
    assert rc == _lib.NVFP4_ERR_WORKSPACE


def test_python_api_refuses_host_tensors():
    import torch
    import nvfp4

    lin = nvfp4.NvFp4Linear(64, 32)
    w = torch.zeros((32, 32), dtype=torch.uint8)
    sf = torch.zeros((32, 4), dtype=torch.uint8)
    x = torch.zeros((2, 64), dtype=torch.bfloat16)
    y = torch.zeros((2, 32), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        nvfp4.nvfp4_linear_forward(lin, w, sf, x, y, 2)


def test_moe_descriptor_rules_without_gpu():
    """nvfp4_moe_workspace_size is 0 exactly for the layers nvfp4.h rules
    out, over generated descriptors (host-side check)."""
    from hypothesis import given, settings
    from hypothesis import strategies as st
    from nvfp4 import _lib

    L = _lib.load()

    def ok(E, k, H, I):
        return (1 <= E <= 256 and 1 <= k <= min(32, E) and H > 0 and H % 128 == 0
                and H <= 6144 and I > 0 and I % 128 == 0)

    @settings(max_examples=300, deadline=None)
    @given(st.integers(-1, 300), st.integers(-1, 40),
           st.sampled_from([-128, 0, 64, 128, 256, 2048, 6144, 6272, 8192]),
           st.sampled_from([-128, 0, 96, 128, 768, 1024]), st.integers(0, 64))
    def check(E, k, H, I, T):
        desc = _lib.MoEDesc(E, k, H, I, 1)
        size = L.nvfp4_moe_workspace_size(ctypes.byref(desc), T)
        assert (size > 0) == ok(E, k, H, I), (E, k, H, I, T)

    check()


def test_headers_compile_as_c():
    """Every header of the drop-in boundary is plain C (C99 and C11, no C++ or
    torch types), so any FFI (Mojo external_call, cgo, ctypes, JNI) can bind
    it; each also compiles on its own."""
    import shutil
    import subprocess
    import tempfile

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    headers = sorted((ROOT / "include").glob("*.h"))
    assert headers
    with tempfile.TemporaryDirectory() as d:
        for std in ("c99", "c11"):
            for hs in [[h] for h in headers] + [headers]:
                src = Path(d) / "t.c"
                src.write_text("".join(f'#include "{h.name}"\n' for h in hs) +
                               "int main(void) { return 0; }\n")
                out = subprocess.run([cc, f"-std={std}", "-Wall", "-Wextra", "-Werror",
                                      "-pedantic", "-fsyntax-only", "-I", str(ROOT / "include"),
                                      str(src)], capture_output=True, text=True)
                assert out.returncode == 0, (std, [h.name for h in hs], out.stderr)


def test_plain_c_program_links_and_calls_the_library():
    """A C program (no Python, no torch) links libnvfp4.so and gets the
    library's answers and error strings through the C ABI alone."""
    import shutil
    import subprocess
    import tempfile

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = ROOT / "nvfp4-mojo_b200" / "nvfp4"
    with tempfile.TemporaryDirectory() as d:
        src, exe = Path(d) / "abi.c", Path(d) / "abi"
        src.write_text(
            '#include <stdio.h>\n#include "nvfp4.h"\n#include "nvfp4_ep.h"\n'
            "int main(void) {\n"
            "  nvfp4_linear_desc d = {2048, 1536, 1.0f, 1.0f, 0};\n"
            '  printf("%d %zu\\n", nvfp4_abi_version(), nvfp4_ep_window_size(2, 64, 2048));\n'
            "  int rc = nvfp4_linear_forward(&d, 0, 0, 0, 1, 0, 1, 4, 0, 0);\n"
            '  printf("%d %s\\n", rc, nvfp4_last_error_string());\n'
            "  return 0;\n}\n")
        out = subprocess.run([cc, "-std=c11", "-I", str(ROOT / "include"), str(src), "-L",
                              str(libdir), "-lnvfp4", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                             capture_output=True, text=True)
        assert out.returncode == 0, out.stderr
        run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
        assert run.returncode == 0, run.stderr
        lines = run.stdout.splitlines()
        assert lines[0] == "1 1573632"
        assert lines[1].startswith("-1 ") and "null" in lines[1]


def test_compute_calls_fail_loudly_without_a_gpu():
    """On a host without a usable GPU every compute entry point returns
    NVFP4_ERR_CUDA with the failing step named (no CPU fallback, no crash).
    Fake device addresses are passed, so this runs only where no GPU is
    visible: on a GPU host the same calls would launch kernels on them."""
    import torch

    from nvfp4 import _lib

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible: the fake device pointers must not reach a kernel")
    L = _lib.load()
    A = 1 << 20  # 256-byte aligned, never dereferenced on the host
    lin = _lib.LinearDesc(2048, 1536, 1.0, 1.0, None)
    moe = _lib.MoEDesc(16, 4, 256, 256, 1)
    w = _lib.MoEWeightPtrs(A, A, A, None, None, A, A, None, None)
    peers = _lib.EpPeers()
    peers.rank, peers.world, peers.max_rows, peers.hidden = 0, 1, 64, 256
    peers.windows[0] = A
    calls = {
        "linear_forward": lambda: L.nvfp4_linear_forward(ctypes.byref(lin), A, A, A, 1, A, 1, 4,
                                                         0, None),
        "dequant": lambda: L.nvfp4_dequant(A, A, 16, 256, A, 0, None),
        "quantize_act": lambda: L.nvfp4_quantize_act(A, 1, 4, 256, 256, 1.0, A, A, None),
        "moe_forward": lambda: L.nvfp4_moe_forward(ctypes.byref(moe), ctypes.byref(w), A, None, A,
                                                   1, 4, None, None, A, 1 << 30, None),
        "ep_p2p_dispatch": lambda: L.nvfp4_ep_p2p_dispatch(ctypes.byref(peers), A, A, 4, 4, 16,
                                                           None),
    }
    for name, call in calls.items():
        rc = call()
        assert rc == _lib.NVFP4_ERR_CUDA, (name, rc, L.nvfp4_last_error_string())
        assert L.nvfp4_last_error_string(), name
