"""exl3_matmul_noalloc -- the matmul entry point for hosts that cannot let a library allocate device memory --
against exl3_matmul, through the C ABI.

Such a host (a server that reserves its device memory up front and admits nothing beyond its memory bill, or a
runtime whose allocator owns every device byte) fills the weight struct itself and passes its own input and output;
the entry point keeps its scratch in a static device array instead of the per-device workspace exl3_matmul uses.
This file is named to be collected last, so that if it fails a run that stops at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REL_L2_BAR = 2e-3  # the bar the other GEMV parity tests use


def _raw_weight(tr, suh, svh):
    """The weight struct filled by hand: no library call, and so no allocation, is needed to make it."""
    from plugins_b200 import _lib as L
    w = L.Weight()
    w.size = ctypes.sizeof(L.Weight)
    w.flags = 0
    w.trellis, w.suh, w.svh = tr.data_ptr(), suh.data_ptr(), svh.data_ptr()
    w.groups = 1
    w.in_features, w.out_features, w.n = tr.shape[0] * 16, tr.shape[1] * 16, tr.shape[2]
    w.device = tr.device.index
    w.nseg = 1
    w.seg_cols[0], w.seg_cols[1] = 0, w.out_features
    return w


def _noalloc(w, x, out):
    from plugins_b200 import _lib as L
    from plugins_b200 import quant as Q
    xt, ot = Q._tensor(x), Q._tensor(out)
    return L.lib().exl3_matmul_noalloc(ctypes.byref(w), ctypes.byref(xt), torch.cuda.current_stream().cuda_stream,
                                       ctypes.byref(ot))


def _rel(a, b):
    a = a.double()
    b = b.double()
    return float(((a - b).norm() / b.norm().clamp_min(1e-30)).item())


@pytest.mark.parametrize("in_f,out_f,n,rows", [(4096, 12288, 64, 1), (2048, 3072, 48, 5), (1024, 2048, 64, 16)])
def test_noalloc_matches_matmul_on_two_calls(in_f, out_f, n, rows):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=in_f + rows)
    raw = _raw_weight(tr, suh, svh)
    ref_w = Q.weight_from_tensors(tr, suh, svh)
    for call in range(2):  # two calls in a row: the shared static scratch must come back clean
        x = torch.randn((rows, in_f), device="cuda", dtype=torch.float16, generator=torch.Generator(device="cuda").manual_seed(call))
        out = torch.full((rows, out_f), float("nan"), device="cuda", dtype=torch.float16)
        v = _noalloc(raw, x, out)
        assert v.code == 0, v.message()
        ref = Q.matmul(ref_w, x)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert _rel(out, ref) < REL_L2_BAR, (call, _rel(out, ref))


def test_noalloc_refuses_a_layer_beyond_its_static_scratch():
    from plugins_b200 import _lib as L
    from plugins_b200 import encoder as E
    tr, suh, svh = E.random_linear(16384, 8192, 64, seed=3)
    raw = _raw_weight(tr, suh, svh)
    x = torch.zeros((16, 16384), device="cuda", dtype=torch.float16)
    out = torch.zeros((16, 8192), device="cuda", dtype=torch.float16)
    v = _noalloc(raw, x, out)
    assert v.code == L.EXL3_TOO_LARGE and b"static scratch" in v.why
