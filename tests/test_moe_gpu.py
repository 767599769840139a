"""Routed SwiGLU experts (the swiglu seam, plugins/turboexl3_ds41/plugin.zig:267-283; SX/root.zig:32-167) against
the oracle's f32 truth, through the C ABI.  Bar: relative L2 2e-3 (north star); the chain's own f16 roundings (the
prepared inputs of the gate/up and down linears) sit well inside it."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REL_L2_BAR = 2e-3


def _bank(E, experts, in_f, out_f, n, seed):
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=seed, groups=experts)
    return tr, suh, svh


def _np16(t):
    return t.detach().cpu().numpy().view(np.uint16)


def _route(rows, experts, topk, seed):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn((rows, experts), generator=g)
    probs = torch.softmax(logits, dim=-1)
    sc, ind = torch.topk(probs, topk, dim=-1)
    return ind.to(torch.int32), sc.float()


@pytest.mark.parametrize("experts,hidden,inter,topk,rows,ng,nd,limit,dtype", [
    (8, 256, 384, 2, 1, 48, 48, 0, "float16"),
    (8, 256, 384, 8, 3, 64, 48, 0, "bfloat16"),
    (16, 384, 256, 4, 20, 32, 64, 0, "float32"),
    (8, 256, 256, 8, 16, 48, 48, 7, "float16"),
    (64, 512, 256, 6, 5, 48, 32, 0, "float16"),
    (16, 256, 384, 4, 7, 40, 56, 0, "bfloat16"),  # half-bit banks: 2.5 and 3.5 bits per weight
])
def test_swiglu_against_f32_truth(oracle, experts, hidden, inter, topk, rows, ng, nd, limit, dtype):
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    dt = getattr(torch, dtype)
    gate = _bank(E, experts, hidden, inter, ng, 10 + rows)
    up = _bank(E, experts, hidden, inter, ng, 20 + rows)
    down = _bank(E, experts, inter, hidden, nd, 30 + rows)
    wg, wu, wd = (Q.weight_from_tensors(*b) for b in (gate, up, down))
    ind, sc = _route(rows, experts, topk, rows)
    x = (torch.randn((1, rows, hidden), generator=torch.Generator().manual_seed(rows)) * 2).to(dt)
    y = Q.swiglu(wg, wu, wd, x.cuda(), ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda(), limit=limit)
    assert y.shape == x.shape and y.dtype == dt
    want = oracle.moe_truth(x.float().numpy().reshape(rows, hidden), ind.numpy(), sc.numpy(),
                            (_np16(gate[0]), _np16(gate[1]), _np16(gate[2]), ng),
                            (_np16(up[0]), _np16(up[1]), _np16(up[2]), ng),
                            (_np16(down[0]), _np16(down[1]), _np16(down[2]), nd),
                            hidden, inter, limit=float(limit), threads=8)
    got = y.float().cpu().numpy().reshape(rows, hidden)
    assert np.isfinite(got).all()
    err = float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))
    floor = float(np.sqrt(((torch.from_numpy(want).to(dt).float().numpy() - want) ** 2).sum() / (want ** 2).sum()))
    assert err < np.sqrt(REL_L2_BAR ** 2 + floor ** 2), (err, floor)


def test_swiglu_is_deterministic_and_refuses_bad_shapes():
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    experts, hidden, inter, topk, rows = 8, 256, 256, 4, 6
    wg, wu, wd = (Q.weight_from_tensors(*_bank(E, experts, i, o, 48, s))
                  for i, o, s in ((hidden, inter, 1), (hidden, inter, 2), (inter, hidden, 3)))
    ind, sc = _route(rows, experts, topk, 5)
    x = torch.randn((2, 3, hidden), device="cuda", dtype=torch.float16)
    a = Q.swiglu(wg, wu, wd, x, ind.view(2, 3, topk).cuda(), sc.view(2, 3, topk).cuda())
    b = Q.swiglu(wg, wu, wd, x, ind.view(2, 3, topk).cuda(), sc.view(2, 3, topk).cuda())
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    with pytest.raises(Q.Exl3Error, match="InvalidExl3Clamp"):
        Q.swiglu(wg, wu, wd, x, ind.view(2, 3, topk).cuda(), sc.view(2, 3, topk).cuda(), limit=200)
    with pytest.raises(Q.Exl3Error, match="BadExl3Dtype"):
        Q.swiglu(wg, wu, wd, x, ind.view(2, 3, topk).cuda(), sc.view(2, 3, topk).cuda().half())
    with pytest.raises(Q.Exl3Error, match="swiglu"):
        Q.moe(wg, x)


def test_absent_experts_contribute_nothing_after_a_full_call(oracle):
    # slots whose expert is outside the bank (-1, E) are dropped; a previous call with every slot present leaves its
    # sorted slot list in the workspace, which must not leak into this one
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    experts, hidden, inter, topk, rows, n = 8, 256, 256, 3, 7, 48
    raw = [_bank(E, experts, i, o, n, s) for i, o, s in ((hidden, inter, 11), (hidden, inter, 12), (inter, hidden, 13))]
    wg, wu, wd = (Q.weight_from_tensors(*b) for b in raw)
    ind, sc = _route(rows, experts, topk, 8)
    x = torch.randn((1, rows, hidden), device="cuda", dtype=torch.float16)
    Q.swiglu(wg, wu, wd, x, ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda())  # every slot present
    ind2 = ind.clone()
    ind2[0, 0], ind2[3, 2], ind2[6, 1] = -1, experts, -1
    y = Q.swiglu(wg, wu, wd, x, ind2.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda(), out=torch.empty(
        (1, rows, hidden), device="cuda", dtype=torch.float32))
    keep_i, keep_s = ind2.clone(), sc.clone()
    absent = (keep_i < 0) | (keep_i >= experts)
    keep_s[absent], keep_i[absent] = 0.0, 0
    bank = lambda b: (_np16(b[0]), _np16(b[1]), _np16(b[2]), n)
    want = oracle.moe_truth(x.float().cpu().numpy(), keep_i.numpy(), keep_s.numpy(), *[bank(b) for b in raw],
                            hidden, inter, 0.0, threads=8)
    got = y.view(rows, hidden).cpu().numpy()
    for r in range(rows):  # row by row: a leaked slot shows in its own row
        rel = np.linalg.norm(got[r] - want[r]) / np.linalg.norm(want[r])
        assert rel < REL_L2_BAR, (r, rel)


def test_config4_call_at_full_size(oracle):
    # config 4 as the bench runs it -- 256 routed experts + the shared one (bank entry 256, score 1), 4096 <-> 2048 at
    # 3 bpw, 32 tokens, top-8 -- in one call; a token's output needs only its own experts, so sampled tokens are held
    # to the f32 truth on the banks' slices of just those experts
    import os
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    experts, hidden, inter, topk, tokens, n = 256, 4096, 2048, 8, 32, 48
    raw = [E.random_linear(a, b, n, seed=3 + i, groups=experts + 1)
           for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden)))]
    banks = [Q.weight_from_tensors(*r) for r in raw]
    g = torch.Generator(device="cuda").manual_seed(4)
    logits = torch.randn((tokens, experts), device="cuda", generator=g)
    sc, ind = torch.topk(torch.softmax(logits, -1), topk, -1)
    ind = torch.cat([ind.to(torch.int32), torch.full((tokens, 1), experts, dtype=torch.int32, device="cuda")], 1)
    sc = torch.cat([sc.float(), torch.ones((tokens, 1), device="cuda")], 1)
    ind, sc = ind.view(1, tokens, topk + 1).contiguous(), sc.view(1, tokens, topk + 1).contiguous()
    x = torch.randn((1, tokens, hidden), device="cuda", dtype=torch.float16, generator=g)
    y = Q.swiglu(*banks, x, ind, sc).float().cpu().numpy().reshape(tokens, hidden)
    picked = [0, 13, 31]
    sub = ind[0, picked]
    used = torch.unique(sub)
    local = torch.searchsorted(used, sub.contiguous()).to(torch.int32)
    sl = [tuple(_np16(t.index_select(0, used.long()).contiguous()) for t in r) + (n,) for r in raw]
    want = oracle.moe_truth(x[0, picked].float().cpu().numpy(), local.cpu().numpy(), sc[0, picked].cpu().numpy(),
                            sl[0], sl[1], sl[2], hidden, inter, threads=os.cpu_count() or 8)
    got = y[picked]
    err = float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))
    floor = float(np.sqrt(((torch.from_numpy(want).half().float().numpy() - want) ** 2).sum() / (want ** 2).sum()))
    assert err < np.sqrt(REL_L2_BAR ** 2 + floor ** 2), (err, floor)
    assert Q.device_error(0) == 0


@pytest.mark.parametrize("experts,hidden,inter,topk,n", [
    (64, 2048, 1024, 8, 48),  # 32 rows: whole units and shared ones; 1-16 rows: shared only
    (16, 1024, 512, 4, 64),
    (256, 4096, 2048, 8, 48),  # config 4's widths
])
def test_rows_share_a_call_without_changing_bytes(experts, hidden, inter, topk, n):
    # the reference's row invariance on its expert kernels (plugins/turboexl3_ds41/src/exl3/selfcheck.zig:755-851):
    # rows slot .. slot + m - 1 computed alone have the bytes they have in the full call, whichever other rows and
    # experts share it (exl3_moe.cu cuts every unit's k range into the same runs in every call)
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    wg, wu, wd = (Q.weight_from_tensors(*_bank(E, experts, i, o, n, s))
                  for i, o, s in ((hidden, inter, 1), (hidden, inter, 2), (inter, hidden, 3)))
    rows = 32
    ind, sc = _route(rows, experts, topk, 7)
    ind, sc = ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda()
    x = (torch.randn((1, rows, hidden), generator=torch.Generator().manual_seed(8)) * 2).to(torch.float16).cuda()
    full = Q.swiglu(wg, wu, wd, x, ind, sc)
    for m, slot in ((1, 0), (1, 17), (2, 30), (3, 5), (8, 24), (16, 0), (31, 1)):
        y = Q.swiglu(wg, wu, wd, x[:, slot:slot + m].contiguous(), ind[:, slot:slot + m].contiguous(),
                     sc[:, slot:slot + m].contiguous())
        assert torch.equal(y.view(torch.int16), full[:, slot:slot + m].view(torch.int16)), (m, slot)


def _shared_setup(E, Q, experts, hidden, inter, inter_s, rows, topk, dt, seed):
    gate = _bank(E, experts, hidden, inter, 48, seed)
    up = _bank(E, experts, hidden, inter, 48, seed + 1)
    down = _bank(E, experts, inter, hidden, 48, seed + 2)
    sh = [E.random_linear(i, o, 64, seed=seed + 3 + j) for j, (i, o) in
          enumerate(((hidden, inter_s), (hidden, inter_s), (inter_s, hidden)))]
    banks = [Q.weight_from_tensors(*b) for b in (gate, up, down)]
    shw = [Q.weight_from_tensors(*b) for b in sh]
    ind, sc = _route(rows, experts, topk, seed)
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn((1, rows, hidden), generator=g) * 2).to(dt).cuda()
    return (gate, up, down), sh, banks, shw, ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda(), x


def _sigtab(dt):
    # the host's table: sigmoid of every 16-bit pattern, in the activations' dtype
    pats = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(dt)
    return torch.sigmoid(pats.float()).to(dt).cuda()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_swiglu_shared_gated_is_the_composition_bit_for_bit(dt):
    # SX/root.zig:50-68 moeWithGatedShared: bit-identical to the sigmoid, multiply and add it replaces; the shared
    # expert through its own linears (quant.zig:95 swiglu_shared) is the routed kernels' one-expert call
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    rows, topk, hidden = 5, 4, 256
    _, _, banks, shw, ind, sc, x = _shared_setup(E, Q, 8, hidden, 384, 256, rows, topk, dt, 40)
    logit = (torch.randn((1, rows), generator=torch.Generator().manual_seed(3)) * 3).to(dt).cuda()
    tab = _sigtab(dt)
    got = Q.swiglu_shared(*banks, x, ind, sc, shared_linears=tuple(shw), logit=logit, sigtab=tab)
    routed = Q.swiglu(*banks, x, ind, sc)
    one_i = torch.zeros((1, rows, 1), dtype=torch.int32, device="cuda")
    one_s = torch.ones((1, rows, 1), dtype=torch.float32, device="cuda")
    shared = Q.swiglu(*shw, x, one_i, one_s)
    sig = tab[logit.view(torch.int16).long() & 0xFFFF]
    want = routed + sig[..., None] * shared
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # the shared expert's output given instead of its linears: the same bytes
    got2 = Q.swiglu_shared(*banks, x, ind, sc, shared=shared, logit=logit, sigtab=tab)
    assert torch.equal(got2.view(torch.int16), want.view(torch.int16))
    # ungated (moeWithShared, SX/root.zig:38-48): the routed output's rounding, then the add
    got3 = Q.swiglu_shared(*banks, x, ind, sc, shared=shared)
    assert torch.equal(got3.view(torch.int16), (routed + shared).view(torch.int16))
    assert Q.device_error(0) == 0


def test_swiglu_shared_against_f32_truth(oracle):
    # the gate's logit from its vector inside the combine, sigmoid without a table, clamped routed experts, 40 rows
    # (the routed call's passes take 512 / 6 = 85 rows each), a shared expert wider than the routed ones
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    rows, topk, hidden, inter, inter_s, limit = 40, 6, 384, 256, 512, 7
    (gate, up, down), sh, banks, shw, ind, sc, x = _shared_setup(E, Q, 16, hidden, inter, inter_s, rows, topk,
                                                                 torch.float16, 60)
    gv = (torch.randn(hidden, generator=torch.Generator().manual_seed(9)) * 0.05).half().cuda()
    got = Q.swiglu_shared(*banks, x, ind, sc, shared_linears=tuple(shw), gate_vec=gv, limit=limit)
    xf = x.float().cpu().numpy().reshape(rows, hidden)
    routed = oracle.moe_truth(xf, ind.cpu().numpy().reshape(rows, topk), sc.cpu().numpy().reshape(rows, topk),
                              (_np16(gate[0]), _np16(gate[1]), _np16(gate[2]), 48),
                              (_np16(up[0]), _np16(up[1]), _np16(up[2]), 48),
                              (_np16(down[0]), _np16(down[1]), _np16(down[2]), 48),
                              hidden, inter, limit=float(limit), threads=8)
    shared = oracle.moe_truth(xf, np.zeros((rows, 1), np.int32), np.ones((rows, 1), np.float32),
                              *[(_np16(t[0])[None], _np16(t[1])[None], _np16(t[2])[None], 64) for t in sh],
                              hidden, inter_s, threads=8)
    logit = xf @ gv.float().cpu().numpy()
    want = routed + (1.0 / (1.0 + np.exp(-logit)))[:, None] * shared
    out = got.float().cpu().numpy().reshape(rows, hidden)
    err = float(np.sqrt(((out - want) ** 2).sum() / (want ** 2).sum()))
    assert err < 2 * REL_L2_BAR, err
    assert Q.device_error(0) == 0


def test_swiglu_shared_refuses_by_name():
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    _, _, banks, shw, ind, sc, x = _shared_setup(E, Q, 8, 256, 256, 256, 3, 2, torch.float16, 80)
    with pytest.raises(Q.Exl3Error, match="one of the two"):
        Q.swiglu_shared(*banks, x, ind, sc)
    with pytest.raises(Q.Exl3Error, match="one of the two"):
        Q.swiglu_shared(*banks, x, ind, sc, shared_linears=tuple(shw), shared=torch.zeros_like(x))
    logit = torch.zeros((1, 3), dtype=torch.float16, device="cuda")
    with pytest.raises(Q.Exl3Error, match="not both"):
        Q.swiglu_shared(*banks, x, ind, sc, shared=torch.zeros_like(x), logit=logit,
                        gate_vec=torch.zeros(256, dtype=torch.float16, device="cuda"))


def _sub_truth(oracle, x, ind, sc, banks, hidden, inter, ns, rows_idx, limit=0.0):
    """moe_truth of some tokens only (a token's output depends on its own row alone)."""
    xs = x.float().cpu().numpy().reshape(-1, hidden)[rows_idx]
    k = ind.shape[-1]
    return oracle.moe_truth(xs, ind.cpu().numpy().reshape(-1, k)[rows_idx], sc.cpu().numpy().reshape(-1, k)[rows_idx],
                            *[(_np16(b[0]), _np16(b[1]), _np16(b[2]), n) for b, n in zip(banks, ns)],
                            hidden, inter, limit=float(limit), threads=8)


@pytest.mark.parametrize("experts,hidden,inter,topk,rows,ng,nd,limit,dtype", [
    (16, 256, 384, 4, 300, 48, 40, 0, "float16"),    # 1200 slots; 384-wide gate/up take 128-column tiles
    (8, 384, 256, 8, 160, 64, 48, 7, "bfloat16"),    # clamped, every expert with many rows
])
def test_moe_prefill_against_truth_and_the_decode_chain(oracle, experts, hidden, inter, topk, rows, ng, nd, limit,
                                                        dtype):
    # SX/expert_exl3_kernels.zig:2955-3029 moePrefill: prompt-width calls through expert-sorted GEMMs
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    dt = getattr(torch, dtype)
    banks = [_bank(E, experts, hidden, inter, ng, 300 + rows), _bank(E, experts, hidden, inter, ng, 301 + rows),
             _bank(E, experts, inter, hidden, nd, 302 + rows)]
    wg, wu, wd = (Q.weight_from_tensors(*b) for b in banks)
    assert Q.moe_prefill_reserve(experts, hidden, inter, rows * topk) > 0
    try:
        ind, sc = _route(rows, experts, topk, rows)
        x = (torch.randn((1, rows, hidden), generator=torch.Generator().manual_seed(rows)) * 2).to(dt).cuda()
        i3, s3 = ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda()
        Q.device_error(0, clear=True)
        y = Q.swiglu(wg, wu, wd, x, i3, s3, limit=limit)
        chain = Q.swiglu(wg, wu, wd, x, i3, s3, limit=limit, verify_rows=True)  # the decode chain, in passes
        torch.cuda.synchronize()
        assert Q.device_error(0) == 0
        want = _sub_truth(oracle, x, ind, sc, banks, hidden, inter, (ng, ng, nd), np.arange(rows), limit)
        got = y.float().cpu().numpy().reshape(rows, hidden)
        assert np.isfinite(got).all()
        err = float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))
        floor = float(np.sqrt(((torch.from_numpy(want).to(dt).float().numpy() - want) ** 2).sum() / (want ** 2).sum()))
        assert err < np.sqrt(REL_L2_BAR ** 2 + floor ** 2), (err, floor)
        c = chain.float().cpu().numpy().reshape(rows, hidden)
        assert float(np.sqrt(((got - c) ** 2).sum() / (c ** 2).sum())) < 2 * REL_L2_BAR
        # every row's bytes are its own: a call of the first half of the rows gives the same bytes for them
        half = rows // 2
        if half * topk >= 1024:
            yh = Q.swiglu(wg, wu, wd, x[:, :half].contiguous(), i3[:, :half].contiguous(), s3[:, :half].contiguous(),
                          limit=limit)
            assert torch.equal(yh.view(torch.int16), y[:, :half].contiguous().view(torch.int16))
    finally:
        Q.moe_prefill_reserve(experts, hidden, inter, 0)


def test_moe_prefill_decode_in_the_gemm_gives_the_image_paths_bytes(monkeypatch):
    # the routed experts' prefill decodes every expert's W_hat^T inside its grouped GEMMs (one pass over all experts);
    # the per-group image form (EXL3_GEMM_FUSED=0) gives the same bytes
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    experts, hidden, inter, topk, rows = 12, 512, 768, 4, 400
    banks = [_bank(E, experts, hidden, inter, 48, 500), _bank(E, experts, hidden, inter, 48, 501),
             _bank(E, experts, inter, hidden, 40, 502)]
    wg, wu, wd = (Q.weight_from_tensors(*b) for b in banks)
    Q.moe_prefill_reserve(experts, hidden, inter, rows * topk)
    try:
        ind, sc = _route(rows, experts, topk, 11)
        x = torch.randn((1, rows, hidden), generator=torch.Generator().manual_seed(11)).half().cuda()
        i3, s3 = ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda()
        monkeypatch.delenv("EXL3_GEMM_FUSED", raising=False)
        y = Q.swiglu(wg, wu, wd, x, i3, s3, limit=5)
        monkeypatch.setenv("EXL3_GEMM_FUSED", "0")
        y0 = Q.swiglu(wg, wu, wd, x, i3, s3, limit=5)
        monkeypatch.delenv("EXL3_GEMM_FUSED")
        torch.cuda.synchronize()
        assert Q.device_error(0, clear=True) == 0
        assert torch.equal(y.view(torch.int16), y0.view(torch.int16))
    finally:
        Q.moe_prefill_reserve(experts, hidden, inter, 0)


def test_moe_prefill_config4_widths_2048_tokens_top8(oracle):
    # config 4's expert widths (4096 <-> 2048 at 3 bpw) at a 2048-token prompt, top-8 of 64 experts; 24 tokens checked
    # against the truth on their own rows
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    experts, hidden, inter, topk, rows = 64, 4096, 2048, 8, 2048
    banks = [_bank(E, experts, hidden, inter, 48, 40), _bank(E, experts, hidden, inter, 48, 41),
             _bank(E, experts, inter, hidden, 48, 42)]
    wg, wu, wd = (Q.weight_from_tensors(*b) for b in banks)
    Q.moe_prefill_reserve(experts, hidden, inter, rows * topk)
    try:
        ind, sc = _route(rows, experts, topk, 9)
        x = torch.randn((1, rows, hidden), generator=torch.Generator().manual_seed(9)).half().cuda()
        Q.device_error(0, clear=True)
        y = Q.swiglu(wg, wu, wd, x, ind.view(1, rows, topk).cuda(), sc.view(1, rows, topk).cuda())
        torch.cuda.synchronize()
        assert Q.device_error(0) == 0
        pick = np.random.default_rng(3).choice(rows, 24, replace=False)
        want = _sub_truth(oracle, x, ind, sc, banks, hidden, inter, (48, 48, 48), pick)
        got = y.float().cpu().numpy().reshape(rows, hidden)[pick]
        err = float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))
        assert err < 2 * REL_L2_BAR, err
    finally:
        Q.moe_prefill_reserve(experts, hidden, inter, 0)
