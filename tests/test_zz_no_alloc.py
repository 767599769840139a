"""exl3_matmul_noalloc -- the matmul entry point for hosts that cannot let a library allocate device memory --
through the C ABI, against the CPU oracle's f32 truth and against exl3_matmul.

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

REL_L2_BAR = 2e-3  # the bar the other GEMV parity tests use


def _raw_weight(tr, suh, svh, seg_cols=None):
    """The weight struct filled by hand: no library call, and so no allocation, is needed to make it.  seg_cols:
    stacked segments' column bounds (suh then holds one row per segment)."""
    from plugins_b200 import _lib as L
    w = L.Weight()
    w.size = ctypes.sizeof(L.Weight)
    w.flags = 0
    w.trellis, w.suh, w.svh = tr.data_ptr(), suh.data_ptr(), svh.data_ptr()
    w.groups = 1
    w.in_features, w.out_features, w.n = tr.shape[0] * 16, tr.shape[1] * 16, tr.shape[2]
    w.device = tr.device.index if tr.is_cuda else 0
    bounds = list(seg_cols) if seg_cols is not None else [0, w.out_features]
    w.nseg = len(bounds) - 1
    for i, c in enumerate(bounds):
        w.seg_cols[i] = c
    return w


def _noalloc(w, x, out, stream=0):
    from plugins_b200 import _lib as L
    from plugins_b200 import quant as Q
    xt, ot = Q._tensor(x), Q._tensor(out)
    return L.lib().exl3_matmul_noalloc(ctypes.byref(w), ctypes.byref(xt), stream, ctypes.byref(ot))


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / max((b ** 2).sum(), 1e-30)))


def _np16(t):
    return t.detach().cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("in_f,out_f,n,rows,dtype", [
    (4096, 12288, 64, 1, "float16"),
    (2048, 3072, 48, 5, "bfloat16"),
    (1024, 2048, 64, 16, "float32"),
    (1024, 1536, 40, 40, "float16"),   # 40 rows: three chunked launches back to back on the shared array
])
def test_noalloc_against_the_oracle_on_two_calls(in_f, out_f, n, rows, dtype):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from oracle import oracle as O
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    dt = getattr(torch, dtype)
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=in_f + rows)
    raw = _raw_weight(tr, suh, svh)
    ref_w = Q.weight_from_tensors(tr, suh, svh)
    Q.device_error(tr.device.index, clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row: the shared static scratch must come back clean
        g = torch.Generator(device="cuda").manual_seed(call)
        x = torch.randn((rows, in_f), device="cuda", generator=g).to(dt)
        out = torch.full((rows, out_f), float("nan"), device="cuda", dtype=dt)
        v = _noalloc(raw, x, out, stream)
        assert v.code == 0, v.why
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        want = O.host_project(x.float().cpu().numpy(), _np16(tr), _np16(suh), _np16(svh), in_f, out_f, n, threads=8)
        assert _rel(out.float().cpu().numpy(), want) < REL_L2_BAR, call
        ref = Q.matmul(ref_w, x)  # exl3_matmul: the same decode, other kernels (not bit-identical)
        assert _rel(out.float().cpu().numpy(), ref.float().cpu().numpy()) < REL_L2_BAR, call
    assert Q.device_error(tr.device.index) == 0


@pytest.mark.gpu
def test_noalloc_stacked_segments_filled_by_hand():
    # two linears that read one input, stacked by the caller: trellis columns side by side, one suh row each,
    # outputs back to back ([rows, 640] then [rows, 384])
    from oracle import oracle as O
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    in_f, widths, n, rows = 1024, (640, 384), 48, 11
    parts = [E.random_linear(in_f, wd, n, seed=50 + i) for i, wd in enumerate(widths)]
    tr = torch.cat([p[0] for p in parts], dim=1).contiguous()
    suh = torch.stack([p[1] for p in parts]).contiguous()
    svh = torch.cat([p[2] for p in parts]).contiguous()
    raw = _raw_weight(tr, suh, svh, seg_cols=[0, widths[0], sum(widths)])
    Q.device_error(tr.device.index, clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.randn((rows, in_f), device="cuda", generator=torch.Generator(device="cuda").manual_seed(7 + call))
        x = x.to(torch.float16)
        out = torch.full((rows, sum(widths)), float("nan"), device="cuda", dtype=torch.float16)
        v = _noalloc(raw, x, out, stream)
        assert v.code == 0, v.why
        torch.cuda.synchronize()
        flat = out.reshape(-1)
        c0 = 0
        for (t, s, h), wd in zip(parts, widths):
            got = flat[rows * c0: rows * (c0 + wd)].view(rows, wd).float().cpu().numpy()
            want = O.host_project(x.float().cpu().numpy(), _np16(t), _np16(s), _np16(h), in_f, wd, n, threads=8)
            assert _rel(got, want) < REL_L2_BAR, (call, wd)
            c0 += wd
    assert Q.device_error(tr.device.index) == 0


@pytest.mark.gpu
def test_noalloc_refuses_a_layer_beyond_its_static_scratch():
    from plugins_b200 import _lib as L
    from plugins_b200 import encoder as E
    tr, suh, svh = E.random_linear(16384, 8192, 64, seed=3)
    raw = _raw_weight(tr, suh, svh)
    x = torch.zeros((16, 16384), device="cuda", dtype=torch.float16)
    out = torch.zeros((16, 8192), device="cuda", dtype=torch.float16)
    v = _noalloc(raw, x, out, torch.cuda.current_stream().cuda_stream)
    assert v.code == L.EXL3_TOO_LARGE and b"static scratch" in v.why


class _Fake:
    """Stands in for a device tensor in checks that refuse before any CUDA call (no GPU needed)."""

    is_cuda = False

    def __init__(self, shape, dtype=torch.float16, ptr=256):
        self.shape, self.dtype, self.ptr = tuple(shape), dtype, ptr

    def data_ptr(self):
        return self.ptr


def _fake_tensor(shape, dt):
    from plugins_b200 import _lib as L
    t = L.Tensor()
    t.data = 4096
    t.dtype = dt
    t.ndim = len(shape)
    for i, s in enumerate(shape):
        t.shape[i] = s
    return t


@pytest.mark.parametrize("bounds,why", [
    ([0, 0, 1024], b"rise"),          # a zero-width segment
    ([0, 512, 896], b"from 0 to"),    # the last bound is not out_features
    ([128, 512, 1024], b"from 0 to"), # the first bound is not 0
    ([0, 600, 1024], b"rise"),        # a bound off the 128-column grid
    ([0, 768, 512, 1024], b"rise"),   # bounds that go backwards
])
def test_noalloc_refuses_bad_segment_bounds_before_any_launch(bounds, why):
    from plugins_b200 import _lib as L
    in_f, out_f = 512, 1024
    raw = _raw_weight(_Fake((in_f // 16, out_f // 16, 64)), _Fake((len(bounds) - 1, in_f)), _Fake((out_f,)), bounds)
    xt, ot = _fake_tensor((3, in_f), L.F16), _fake_tensor((3, out_f), L.F16)
    v = L.lib().exl3_matmul_noalloc(ctypes.byref(raw), ctypes.byref(xt), 0, ctypes.byref(ot))
    assert v.code == L.EXL3_UNSUPPORTED and why in v.why, v.why
