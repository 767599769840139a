"""The tensor-core prefill GEMM (matmul at 64 rows and more) against the CPU oracle, through the C ABI.

The reference takes many rows through prepare + GEMM + finish (plugins/sushi_ds41/src/sushi/linear.zig:77-100), with the
trellis tiles decoded ahead of the MMA (kernels/header_dig_mul1h_k3.metal:1090-1166).  The bars are the GEMV's:
  * decoded weights bit-exact: one-hot prepared rows with the inner product reproduce W_hat's rows word for word
    (selfcheck.zig:861-907 does the same through its GEMM);
  * outputs within relative L2 2e-3 of the f32-accumulated truth, and within sqrt(LINEAR_BAR^2 + floor^2)
    (linear.zig:252-321);
Every tile shape of the GEMM (EXL3_GEMM_SHAPE 0..3: 128x128, 128x256, 256x128, 256x256) is run, including ragged
rows and a column count that leaves a half-empty last tile.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REL_L2_BAR = 2e-3
LINEAR_BAR = 1.5e-3
PREPARED, INNER, GEMV, GEMM = 1, 2, 8, 16


@pytest.fixture(scope="module")
def Q():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import quant
    return quant


@pytest.fixture(scope="module")
def E():
    from plugins_b200 import encoder
    return encoder


@pytest.fixture(params=["0", "1", "2", "3"])
def shape(request, monkeypatch):
    monkeypatch.setenv("EXL3_GEMM_SHAPE", request.param)
    return int(request.param)


def _rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / max((want ** 2).sum(), 1e-30)))


def _round(dt, v):
    return torch.from_numpy(np.asarray(v, np.float32)).to(dt).float().numpy()


def _np(t):
    return t.detach().cpu().numpy()


def _truth(oracle, x, tr, suh, svh, in_f, out_f, n):
    return oracle.host_project(x.float().cpu().numpy(), _np(tr).view(np.uint16), _np(suh).view(np.uint16),
                               _np(svh).view(np.uint16), in_f, out_f, n, threads=os.cpu_count() or 8)


@pytest.mark.parametrize("n", [16, 40, 48, 64, 88, 96])
def test_one_hot_rows_reproduce_w_hat(Q, E, oracle, shape, n):
    # prepared x = the identity, inner product: every output row is a row of W_hat, exactly (1.0 * w + 0s in f32)
    in_f, out_f = 256, 640  # 640 columns: a ragged last tile for the 256-wide shapes
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=n + 17)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.eye(in_f, dtype=torch.float16, device="cuda")
    y = Q.matmul_ex(w, x, flags=PREPARED | INNER | GEMM)
    got = y.to(torch.float16).view(torch.uint16).cpu().numpy()
    want = oracle.reconstruct_inner(_np(tr).view(np.uint16), in_f, out_f, n)
    assert y.dtype == torch.float32 and np.array_equal(got, want)
    assert torch.equal(y, y.to(torch.float16).float())  # nothing but the weights themselves


CASES = [
    # (in, out, n, rows)
    (512, 768, 64, 64), (1024, 640, 48, 200), (256, 1280, 32, 333), (768, 384, 96, 130), (384, 512, 80, 257),
    (5120, 2304, 48, 128),  # the DeepSeek-V4.1 prefill shape (dsv41_prefill_dig_gemm_5120x2304)
    (512, 768, 56, 96), (768, 512, 24, 300),  # half-bit rates: 3.5 and 1.5 bits per weight
]


@pytest.mark.parametrize("in_f,out_f,n,rows", CASES)
@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_gemm_against_f32_truth(Q, E, oracle, shape, in_f, out_f, n, rows, dtype):
    dt = getattr(torch, dtype)
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=in_f + out_f + n + rows)
    w = Q.weight_from_tensors(tr, suh, svh)
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = ((torch.rand((rows, in_f), generator=g, device="cuda") * 2 - 1) * 30).to(dt)
    y = Q.matmul(w, x)  # rows >= 64: the GEMM by default
    assert y.dtype == dt and y.shape == (rows, out_f)
    got = y.float().cpu().numpy()
    want = _truth(oracle, x, tr, suh, svh, in_f, out_f, n)
    assert np.isfinite(got).all()
    err = _rel(got, want)
    floor = _rel(_round(dt, want), want)
    assert err < REL_L2_BAR, err
    assert err < np.sqrt(LINEAR_BAR ** 2 + floor ** 2), (err, floor)
    assert Q.device_error(0, clear=True) == 0


@pytest.mark.parametrize("in_f,out_f,n,rows", [
    (4096, 12288, 64, 64),    # config 3's layer at the crossover's smallest width: 128-column tiles, one 128-row block
    (1024, 640, 48, 200),     # two 128-row blocks in one tile, a ragged last row block
    (512, 768, 88, 256),
    (768, 512, 24, 100),      # a half-bit rate
])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_decode_in_the_gemm_gives_the_image_paths_bytes(Q, E, monkeypatch, in_f, out_f, n, rows, dtype):
    # the GEMM that decodes W_hat^T into shared memory itself (no B image; EXL3_GEMM_FUSED=1): the same tiles, the
    # same MMA k order and the same output Hadamard make it byte-for-byte the decode-into-an-image path
    dt = getattr(torch, dtype)
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=in_f + rows + n)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = (torch.randn((rows, in_f), generator=torch.Generator().manual_seed(rows)) * 3).to(dt).cuda()
    monkeypatch.setenv("EXL3_GEMM_FUSED", "1")
    fused = Q.matmul(w, x)
    monkeypatch.delenv("EXL3_GEMM_FUSED")
    image = Q.matmul(w, x)
    torch.cuda.synchronize()
    assert Q.device_error(0, clear=True) == 0
    assert torch.equal(fused.view(-1).view(torch.uint8), image.view(-1).view(torch.uint8))


def test_decode_in_the_gemm_stacked_and_forced_past_256_rows(Q, E, oracle, monkeypatch):
    # a stacked q|k|v-like weight (three segments, each its own svh slice) through the fused form, and 300 rows forced
    # through it (two 256-row tiles, each decoding its B blocks again), against the truth
    segs = [E.random_linear(512, o, 64, seed=90 + o) for o in (512, 256, 256)]
    w = Q.stack([Q.weight_from_tensors(*s_) for s_ in segs])
    x = (torch.randn((300, 512), generator=torch.Generator().manual_seed(5)) * 2).half().cuda()
    monkeypatch.setenv("EXL3_GEMM_FUSED", "1")
    y = Q.matmul(w, x)
    monkeypatch.delenv("EXL3_GEMM_FUSED")
    y0 = Q.matmul(w, x)
    assert torch.equal(y.view(torch.int16), y0.view(torch.int16))
    for s_, want_y in zip(segs, Q.segment_outputs(w, y, 300)):
        want = _truth(oracle, x, s_[0], s_[1], s_[2], 512, s_[0].shape[1] * 16, 64)
        assert _rel(want_y.float().cpu().numpy(), want) < REL_L2_BAR
    assert Q.device_error(0, clear=True) == 0


def test_gemm_and_gemv_agree(Q, E, oracle):
    # the same rows forced through either path land within the bar of each other and of the truth
    in_f, out_f, n, rows = 1024, 1536, 48, 96
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=77)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.randn((rows, in_f), device="cuda", dtype=torch.float16)
    a = Q.matmul_ex(w, x, flags=GEMM).float().cpu().numpy()
    b = Q.matmul_ex(w, x, flags=GEMV).float().cpu().numpy()
    want = _truth(oracle, x, tr, suh, svh, in_f, out_f, n)
    assert _rel(a, want) < REL_L2_BAR and _rel(b, want) < REL_L2_BAR
    assert _rel(a, b) < REL_L2_BAR


def test_gemm_is_deterministic_and_capturable(Q, E):
    in_f, out_f, n, rows = 512, 1024, 64, 192
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=5)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.randn((rows, in_f), device="cuda", dtype=torch.bfloat16)
    eager = Q.matmul(w, x)
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        Q.matmul(w, x, out=out)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        Q.matmul(w, x, out=out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), eager.view(torch.int16))
    assert torch.equal(Q.matmul(w, x).view(torch.int16), eager.view(torch.int16))


def test_stacked_linears_through_the_gemm(Q, E, oracle):
    in_f, widths, rows = 512, (640, 256, 384), 100
    parts, raw = [], []
    for i, wd in enumerate(widths):
        tr, suh, svh = E.random_linear(in_f, wd, 48, seed=200 + i)
        raw.append((tr, suh, svh))
        parts.append(Q.weight_from_tensors(tr, suh, svh))
    st = Q.stack(parts)
    x = ((torch.rand((rows, in_f), device="cuda") * 2 - 1) * 30).to(torch.float16)
    outs = Q.segment_outputs(st, Q.matmul(st, x), rows)
    for (tr, suh, svh), yo, wd in zip(raw, outs, widths):
        want = _truth(oracle, x, tr, suh, svh, in_f, wd, 48)
        assert _rel(yo.float().cpu().numpy(), want) < REL_L2_BAR


def test_grouped_linear_through_the_gemm(Q, E, oracle):
    from plugins_b200 import _lib as L
    groups, in_f, out_f, n, rows = 3, 256, 384, 64, 70
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=21, groups=groups)
    w = Q.weight_from_tensors(tr, suh, svh)
    w.raw.flags |= L.WEIGHT_GROUPED
    x = torch.randn((rows, groups, in_f), device="cuda", dtype=torch.float16)
    y = Q.matmul(w, x)
    for g in range(groups):
        want = _truth(oracle, x[:, g], tr[g], suh[g], svh[g], in_f, out_f, n)
        assert _rel(y[:, g].float().cpu().numpy(), want) < REL_L2_BAR


def test_prefill_layer_at_full_size(Q, E, oracle):
    # the prefill config's layer: X [2048, 4096] bf16, W 4096 x 12288 at 4 bpw.  Sampled rows against the f32 truth,
    # and every row against the decode GEMV's answer (itself held to the truth by the GEMV tests).
    in_f, out_f, n, rows = 4096, 12288, 64, 2048
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=2)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.randn((rows, in_f), device="cuda", generator=torch.Generator(device="cuda").manual_seed(2)).to(torch.bfloat16)
    y = Q.matmul(w, x)
    pick = torch.tensor([0, 1, 777, 1024, 1500, 2047], device="cuda")
    want = _truth(oracle, x[pick], tr, suh, svh, in_f, out_f, n)
    assert _rel(y[pick].float().cpu().numpy(), want) < REL_L2_BAR
    ref = Q.matmul_ex(w, x, flags=GEMV)
    assert float(((y.float() - ref.float()).norm() / ref.float().norm()).item()) < REL_L2_BAR
    assert Q.device_error(0) == 0


def test_unaligned_rows_take_the_gemv(Q, E, oracle):
    # rows that start off an 8-byte boundary cannot feed the prepare's vector loads: the decode GEMV serves them
    in_f, out_f, n, rows = 512, 384, 64, 80
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=31)
    w = Q.weight_from_tensors(tr, suh, svh)
    buf = torch.randn(rows * in_f + 1, device="cuda").to(torch.float16)
    x = buf[1:].view(rows, in_f)
    assert x.data_ptr() % 8 != 0
    y = Q.matmul(w, x)
    want = _truth(oracle, x, tr, suh, svh, in_f, out_f, n)
    assert _rel(y.float().cpu().numpy(), want) < REL_L2_BAR


def test_kept_matrices_give_the_decoding_calls_bytes(Q, E):
    # quant.zig:96-101 resident / resident_pending: the first prefill call after exl3_resident fills the kept matrix,
    # later calls read it instead of decoding; every call gives the bytes of the decoding path, for a plain linear
    # (640 columns: a ragged last tile), a stacked one and a grouped one
    from plugins_b200 import _lib as L
    plain = Q.weight_from_tensors(*E.random_linear(512, 640, 48, seed=31))
    stacked = Q.stack([Q.weight_from_tensors(*E.random_linear(512, o, 64, seed=40 + i))
                       for i, o in enumerate((384, 128, 128))])
    grouped = Q.weight_from_tensors(*E.random_linear(256, 384, 64, seed=50, groups=3))
    grouped.raw.flags |= L.WEIGHT_GROUPED
    xs = {id(plain): torch.randn((100, 512), device="cuda", dtype=torch.float16),
          id(stacked): torch.randn((300, 512), device="cuda", dtype=torch.bfloat16),
          id(grouped): torch.randn((70, 3, 256), device="cuda", dtype=torch.float16)}
    ws = (plain, stacked, grouped)
    want = {id(w): Q.matmul(w, xs[id(w)]) for w in ws}
    try:
        kept = Q.resident(list(ws))
        assert kept == (640 // 128 + 2) * 512 * 256 + (640 // 128 + 2) * 512 * 256 + 3 * (384 // 128 + 2) * 256 * 256
        assert Q.resident_pending() == kept
        assert Q.resident([plain]) == kept  # kept once
        for rep in range(2):
            for w in ws:
                y = Q.matmul(w, xs[id(w)])
                assert torch.equal(y.view(torch.int16), want[id(w)].view(torch.int16)), (rep, w.out_features)
            assert Q.resident_pending() == 0
        with pytest.raises(Q.Exl3Error, match="room"):
            Q.resident([Q.weight_from_tensors(*E.random_linear(256, 256, 32, seed=60))], room=kept + 1)
        assert Q.resident([]) == 0 and Q.resident_pending() == 0
        y = Q.matmul(plain, xs[id(plain)])
        assert torch.equal(y.view(torch.int16), want[id(plain)].view(torch.int16))
    finally:
        Q.resident([])
    assert Q.device_error(0) == 0
