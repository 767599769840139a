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
