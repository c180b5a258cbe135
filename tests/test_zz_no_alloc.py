"""nvfp4_moe_forward_noalloc: the MoE layer for callers that cannot allocate
device memory (a caller with no device allocator of its own, such as
foreign-function host code holding only the pointers it was given, or a
serving loop that must not call cudaMalloc once it runs).  Its workspace is
a static 16 MiB array inside the library instead of caller memory.

Checked through the C ABI: two calls in a row (the second one finds the
first one's leftovers in the shared scratch) against the existing entry
point nvfp4_moe_forward with a caller workspace, within the MoE tests'
tolerance (max|err| <= 2e-2 * RMS); and a layer too large for the scratch is
rejected with NVFP4_ERR_WORKSPACE.  Kept in a file of its own, collected
last, and independent of earlier tests (it passes alone in a fresh process).
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.sqrt(np.mean(ref * ref)))


def _layer(T):
    from nvfp4 import synthetic
    from nvfp4.moe import MoELayer, MoEWeights

    wd = synthetic.moe_weights(128, 2048, 768, seed=41)
    x = synthetic.bf16_round(synthetic.activations(T, 2048, seed=42))
    layer = MoELayer(MoEWeights.from_dict(wd), top_k=8)
    return layer, torch.from_numpy(x).cuda().to(torch.bfloat16)


def test_noalloc_matches_workspace_entry_point(cuda):
    from nvfp4 import _lib

    L = _lib.load()
    T = 24
    layer, X = _layer(T)
    ref = layer(X).float().cpu().numpy()  # nvfp4_moe_forward, caller workspace
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        y = torch.full_like(X, float("nan"))
        rc = L.nvfp4_moe_forward_noalloc(ctypes.byref(layer.desc), ctypes.byref(layer.ptrs),
                                         X.data_ptr(), None, y.data_ptr(), _lib.DTYPE_BF16, T,
                                         None, None, stream)
        assert rc == 0, L.nvfp4_last_error_string()
        torch.cuda.synchronize()
        got = y.float().cpu().numpy()
        assert not np.isnan(got).any(), call
        assert rel_err(got, ref) <= TOL, call


def test_noalloc_largest_layer_that_fits(cuda):
    """The largest token count whose workspace fits the scratch runs (and uses
    its top end); one more token is rejected before anything is launched."""
    from nvfp4 import _lib

    L = _lib.load()
    cap = 16 * 1024 * 1024
    layer, _ = _layer(1)
    T = 1
    while L.nvfp4_moe_workspace_size(ctypes.byref(layer.desc), T + 1) <= cap:
        T += 1
    assert L.nvfp4_moe_workspace_size(ctypes.byref(layer.desc), T) <= cap
    layer, X = _layer(T)
    ref = layer(X).float().cpu().numpy()
    y = torch.full_like(X, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.nvfp4_moe_forward_noalloc(ctypes.byref(layer.desc), ctypes.byref(layer.ptrs),
                                     X.data_ptr(), None, y.data_ptr(), _lib.DTYPE_BF16, T,
                                     None, None, stream)
    assert rc == 0, L.nvfp4_last_error_string()
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    assert not np.isnan(got).any() and rel_err(got, ref) <= TOL
    X2 = torch.zeros((T + 1, X.shape[1]), dtype=X.dtype, device=X.device)
    rc = L.nvfp4_moe_forward_noalloc(ctypes.byref(layer.desc), ctypes.byref(layer.ptrs),
                                     X2.data_ptr(), None, X2.data_ptr(), _lib.DTYPE_BF16, T + 1,
                                     None, None, stream)
    assert rc == _lib.NVFP4_ERR_WORKSPACE


def test_noalloc_rejects_layers_beyond_the_scratch(cuda):
    from nvfp4 import _lib

    L = _lib.load()
    T = 4096  # needs ~187 MB of workspace, more than the 16 MiB scratch
    layer, _ = _layer(1)
    assert L.nvfp4_moe_workspace_size(ctypes.byref(layer.desc), T) > 16 * 1024 * 1024
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    rc = L.nvfp4_moe_forward_noalloc(ctypes.byref(layer.desc), ctypes.byref(layer.ptrs),
                                     dummy.data_ptr(), None, dummy.data_ptr(), _lib.DTYPE_BF16,
                                     T, None, None, None)
    assert rc == _lib.NVFP4_ERR_WORKSPACE
    assert b"static scratch" in L.nvfp4_last_error_string()
