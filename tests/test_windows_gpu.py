"""Narrowed codeword windows (expert_exl3.zig Window: the codeword is the low w bits of each 16-bit window, w = 8..16;
packs searched at a narrowed window, plugins/turboexl3_qwen38/config.zig:86-104 accepting 8..16) through the C ABI,
against the CPU oracle at the same window: decoded weights bit-exact, layer outputs within the GEMV bars."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REL_L2_BAR = 2e-3


@pytest.fixture(scope="module")
def Q():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import quant
    return quant


@pytest.fixture(scope="module")
def E():
    from plugins_b200 import encoder
    return encoder


def _np(t):
    return t.detach().cpu().numpy()


def _u16(t):
    return _np(t).view(np.uint16)


def _rel(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / max((want ** 2).sum(), 1e-30)))


@pytest.mark.parametrize("n", [32, 40, 48, 64, 88])
@pytest.mark.parametrize("window", [8, 12, 15])
@pytest.mark.parametrize("dp4a", [False, True])
def test_decode_dense_at_a_narrowed_window(Q, E, oracle, n, window, dp4a):
    in_f, out_f = 256, 384
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=n + window)
    w = Q.weight_from_tensors(tr, suh, svh, window=window)
    assert w.window == window
    got = Q.decode_dense(w, dp4a=dp4a).view(torch.uint16).cpu().numpy()
    assert np.array_equal(got, oracle.reconstruct_inner(_u16(tr), in_f, out_f, n, window=window))


@pytest.mark.parametrize("in_f,out_f,n,window", [
    (512, 640, 64, 12), (1024, 768, 48, 10), (768, 512, 40, 8),
    (12288, 4096, 48, 14),  # a shape the persistent GEMV would take at 16 bits: a narrowed window takes the cluster split
])
def test_gemv_and_gemm_at_a_narrowed_window(Q, E, oracle, in_f, out_f, n, window):
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=in_f + window)
    w = Q.weight_from_tensors(tr, suh, svh, window=window)
    x = torch.randn((100, in_f), device="cuda", dtype=torch.float16)
    want = oracle.host_project(x.float().cpu().numpy(), _u16(tr), _u16(suh), _u16(svh), in_f, out_f, n,
                               threads=os.cpu_count() or 8, window=window)
    ys = {}
    for rows in (1, 9, 16):
        ys[rows] = Q.matmul(w, x[:rows].contiguous())
        assert _rel(ys[rows].float().cpu().numpy(), want[:rows]) < REL_L2_BAR, rows
    for rows in (1, 9):  # a row's bytes do not depend on the rows batched with it
        assert torch.equal(ys[rows].view(torch.int16), ys[16][:rows].view(torch.int16)), rows
    y = Q.matmul(w, x)  # 100 rows: the tensor-core GEMM
    assert _rel(y.float().cpu().numpy(), want) < REL_L2_BAR
    assert Q.device_error(0) == 0


def test_routed_experts_at_narrowed_windows(Q, E, oracle):
    experts, hidden, inter, topk, rows, n = 16, 512, 256, 4, 12, 48
    banks = [E.random_linear(a, b, n, seed=70 + i, groups=experts)
             for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden)))]
    windows = (12, 12, 10)
    wg, wu, wd = (Q.weight_from_tensors(*b, window=wn) for b, wn in zip(banks, windows))
    g = torch.Generator().manual_seed(3)
    sc, ind = torch.topk(torch.softmax(torch.randn((rows, experts), generator=g), -1), topk, -1)
    ind, sc = ind.to(torch.int32), sc.float()
    x = (torch.randn((1, rows, hidden), generator=g) * 2).to(torch.float16)
    y = Q.swiglu(wg, wu, wd, x.cuda(), ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda())
    want = oracle.moe_truth(x.float().numpy().reshape(rows, hidden), ind.numpy(), sc.numpy(),
                            *[(_u16(b[0]), _u16(b[1]), _u16(b[2]), n) for b in banks], hidden, inter,
                            threads=os.cpu_count() or 8, windows=(12, 10))
    got = y.float().cpu().numpy().reshape(rows, hidden)
    floor = _rel(torch.from_numpy(want).half().float().numpy(), want)
    assert _rel(got, want) < np.sqrt(REL_L2_BAR ** 2 + floor ** 2)
    wu2 = Q.weight_from_tensors(*banks[1], window=11)
    with pytest.raises(Q.Exl3Error, match="different codeword windows"):
        Q.swiglu(wg, wu2, wd, x.cuda(), ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda())


def test_narrowed_windows_refused_by_name(Q, E):
    tr, suh, svh = E.random_linear(256, 256, 48, seed=9)
    w12 = Q.weight_from_tensors(tr, suh, svh, window=12)
    x = torch.randn((2, 256), device="cuda", dtype=torch.float16)
    with pytest.raises(Q.Exl3Error, match="no dp4a"):
        Q.matmul_ex(w12, x, flags=4)
    with pytest.raises(Q.Exl3Error, match="Exl3WindowUnsupported"):
        Q.weight_from_tensors(tr, suh, svh, window=7)
    w16 = Q.weight_from_tensors(*E.random_linear(256, 128, 48, seed=10))
    with pytest.raises(Q.Exl3Error, match="codeword window"):
        Q.stack([w12, w16])
    st = Q.stack([w12, Q.weight_from_tensors(*E.random_linear(256, 128, 48, seed=11), window=12)])
    assert st.window == 12


# ---------------------------------------------------------------- the mcg codebook (expert_exl3.zig:267-273)

@pytest.mark.parametrize("n", [32, 40, 48, 64, 96])
@pytest.mark.parametrize("window", [16, 12])
@pytest.mark.parametrize("dp4a", [False, True])
def test_decode_dense_mcg(Q, E, oracle, n, window, dp4a):
    # both operand orders: the natural one (dp4a flag) and the tensor-pipe one, where each lane reads its two
    # neighbours' windows
    in_f, out_f = 256, 384
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=3 * n + window)
    w = Q.weight_from_tensors(tr, suh, svh, window=window, codebook="mcg")
    assert w.codebook == "mcg"
    got = Q.decode_dense(w, dp4a=dp4a).view(torch.uint16).cpu().numpy()
    assert np.array_equal(got, oracle.reconstruct_inner(_u16(tr), in_f, out_f, n, window=window, codebook="mcg"))


@pytest.mark.parametrize("in_f,out_f,n,window", [(512, 640, 48, 16), (1024, 768, 40, 12), (4096, 12288, 64, 16)])
def test_gemv_and_gemm_mcg(Q, E, oracle, in_f, out_f, n, window):
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=in_f + n)
    w = Q.weight_from_tensors(tr, suh, svh, window=window, codebook="mcg")
    x = torch.randn((100, in_f), device="cuda", dtype=torch.float16)
    want = oracle.host_project(x.float().cpu().numpy(), _u16(tr), _u16(suh), _u16(svh), in_f, out_f, n,
                               threads=os.cpu_count() or 8, window=window, codebook="mcg")
    ys = {rows: Q.matmul(w, x[:rows].contiguous()) for rows in (1, 9, 16)}
    for rows, y in ys.items():
        assert _rel(y.float().cpu().numpy(), want[:rows]) < REL_L2_BAR, rows
        assert torch.equal(y.view(torch.int16), ys[16][:rows].view(torch.int16)), rows
    assert _rel(Q.matmul(w, x).float().cpu().numpy(), want) < REL_L2_BAR  # the GEMM
    assert Q.device_error(0) == 0


def test_routed_experts_mcg(Q, E, oracle):
    experts, hidden, inter, topk, rows, n = 16, 512, 256, 4, 12, 40
    banks = [E.random_linear(a, b, n, seed=90 + i, groups=experts)
             for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden)))]
    specs = ((16, "mcg"), (16, "mcg"), (12, "mul1"))  # gate|up mcg, down mul1 at a narrowed window
    wg, wu, wd = (Q.weight_from_tensors(*b, window=wn, codebook=cb) for b, (wn, cb) in zip(banks, specs))
    g = torch.Generator().manual_seed(5)
    sc, ind = torch.topk(torch.softmax(torch.randn((rows, experts), generator=g), -1), topk, -1)
    ind, sc = ind.to(torch.int32), sc.float()
    x = (torch.randn((1, rows, hidden), generator=g) * 2).to(torch.float16)
    y = Q.swiglu(wg, wu, wd, x.cuda(), ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda())
    want = oracle.moe_truth(x.float().numpy().reshape(rows, hidden), ind.numpy(), sc.numpy(),
                            *[(_u16(b[0]), _u16(b[1]), _u16(b[2]), n) for b in banks], hidden, inter,
                            threads=os.cpu_count() or 8, windows=(16, 12), codebooks=("mcg", "mul1"))
    got = y.float().cpu().numpy().reshape(rows, hidden)
    floor = _rel(torch.from_numpy(want).half().float().numpy(), want)
    assert _rel(got, want) < np.sqrt(REL_L2_BAR ** 2 + floor ** 2)
    with pytest.raises(Q.Exl3Error, match="codebooks"):
        Q.swiglu(wg, Q.weight_from_tensors(*banks[1]), wd, x.cuda(), ind.view(1, rows, topk).cuda(),
                 sc.view(1, rows, topk).cuda())
