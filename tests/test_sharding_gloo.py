"""The multi-GPU drivers' host logic on gloo ranks (CPU, world size 2), and the column-parallel experts' split.

plugins_b200/sharding.py splits the path the two ways it shards: linears column-parallel with an all-gather of y, and
routed experts expert-parallel with a dispatch all-to-all and a combine all-to-all.  Here the drivers run unchanged
over gloo with the oracle as their compute (tests/sharding_cpu_ops.py), so the shard bounds, buffer layouts, slot
bookkeeping and the sequence of collectives are checked against the single-process f32 truth.
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _rand_linear(rng, in_f, out_f, n, lead=()):
    tr = rng.integers(0, 65536, lead + (in_f // 16, out_f // 16, n), dtype=np.uint16)
    suh = (rng.choice([-1.0, 1.0], lead + (in_f,)) * (0.002 + 0.02 * rng.random(lead + (in_f,)))).astype(np.float16)
    svh = (rng.choice([-1.0, 1.0], lead + (out_f,)) * (0.5 + rng.random(lead + (out_f,)))).astype(np.float16)
    return tr, suh, svh


def _tp_rank(rank, world, port, out_f):
    _init(rank, world, port)
    try:
        from oracle import oracle as O
        import sharding_cpu_ops as C
        from plugins_b200 import sharding as S
        rng = np.random.default_rng(7)
        in_f, n = 256, 48
        tr, suh, svh = _rand_linear(rng, in_f, out_f, n)
        x = rng.standard_normal((3, in_f)).astype(np.float32)
        lin = S.ColumnParallelLinear(torch.from_numpy(tr.view(np.int16)), torch.from_numpy(suh),
                                     torch.from_numpy(svh), rank, world, ops=C.OracleLinearOps(O))
        y = lin.forward(torch.from_numpy(x))
        want = O.host_project(x, tr, suh.view(np.uint16), svh.view(np.uint16), in_f, out_f, n, threads=2)
        assert y.shape == (3, out_f)
        assert np.array_equal(y.numpy(), want)  # columns are independent: the shards reassemble bit for bit
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("out_f", [512, 640])  # 640 = 5 column blocks: shards of 3 and 2 blocks
def test_column_parallel_linear_on_two_gloo_ranks(oracle, out_f):
    mp.spawn(_tp_rank, args=(2, _free_port(), out_f), nprocs=2)


def test_column_ranges_cover_the_output_once():
    from plugins_b200 import sharding as S
    for out_f in (128, 640, 4096, 53248):
        for world in (1, 2, 4, 8):
            if out_f // 128 < world:
                with pytest.raises(ValueError):
                    S.column_range(out_f, 0, world)
                continue
            ranges = [S.column_range(out_f, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == out_f
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            widths = [b - a for a, b in ranges]
            assert all(w % 128 == 0 for w in widths) and max(widths) - min(widths) <= 128


def _ep_rank(rank, world, port, tokens, topk, experts, shared, limit):
    _init(rank, world, port)
    try:
        from oracle import oracle as O
        import sharding_cpu_ops as C
        from plugins_b200 import sharding as S
        rng = np.random.default_rng(11)  # every rank draws the same model and the same tokens
        hidden, inter, n = 256, 128, 48
        banks = [_rand_linear(rng, a, b, n, (experts,)) for a, b in ((hidden, inter), (hidden, inter), (inter, hidden))]
        sbanks = [_rand_linear(rng, a, b, n, (1,)) for a, b in ((hidden, inter), (hidden, inter), (inter, hidden))]
        total = world * tokens
        x = rng.standard_normal((total, hidden)).astype(np.float16).astype(np.float32)
        inds = np.stack([rng.permutation(experts)[:topk] for _ in range(total)]).astype(np.int32)
        inds[0, -1] = -1  # an absent slot
        scores = rng.random((total, topk)).astype(np.float32)

        def as_oracle(b, e0=0, e1=None):
            tr, su, sv = b
            return (tr[e0:e1], su[e0:e1].view(np.uint16), sv[e0:e1].view(np.uint16), n)

        e0, e1 = S.expert_range(experts, rank, world)
        sh = [as_oracle(b) for b in sbanks] if shared else None
        if shared:  # this rank's experts, then the shared expert (every rank holds it)
            local = [(np.concatenate([tr[e0:e1], str_]), np.concatenate([su[e0:e1], ssu]).view(np.uint16),
                      np.concatenate([sv[e0:e1], ssv]).view(np.uint16), n)
                     for (tr, su, sv), (str_, ssu, ssv) in zip(banks, sbanks)]
        else:
            local = [as_oracle(b, e0, e1) for b in banks]
        ep = S.ExpertParallelSwiglu(*local, experts=experts, tokens=tokens, topk=topk, hidden=hidden, rank=rank,
                                    world=world, dtype=torch.float32, device=torch.device("cpu"), shared=shared,
                                    limit=limit, ops=C.OracleExpertOps(O))
        sl = slice(rank * tokens, (rank + 1) * tokens)
        out = ep.forward(torch.from_numpy(x[sl]), torch.from_numpy(inds[sl]), torch.from_numpy(scores[sl]))
        # the truth: every token's routed experts on the whole banks (absent slots dropped), plus the shared expert
        ii, ss = inds[sl].copy(), scores[sl].copy()
        ss[ii < 0] = 0.0
        ii[ii < 0] = 0
        full = [as_oracle(b) for b in banks]
        want = O.moe_truth(x[sl], ii, ss, *full, hidden, inter, float(limit), threads=2)
        if shared:
            want = want + O.moe_truth(x[sl], np.zeros((tokens, 1), np.int32), np.ones((tokens, 1), np.float32),
                                      *sh, hidden, inter, float(limit), threads=2)
        got = out.numpy()
        rel = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
        assert rel < 1e-6, rel
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,topk,experts,shared,limit", [(3, 4, 8, False, 0), (2, 3, 6, True, 7)])
def test_expert_parallel_swiglu_on_two_gloo_ranks(oracle, tokens, topk, experts, shared, limit):
    mp.spawn(_ep_rank, args=(2, _free_port(), tokens, topk, experts, shared, limit), nprocs=2)


def test_dispatch_layout_and_overflow():
    import sharding_cpu_ops as C
    tokens, topk, experts, world, hidden = 3, 2, 4, 2, 128
    x = torch.arange(tokens * hidden, dtype=torch.float32).view(tokens, hidden)
    # the shared expert (id `experts`) stays on the calling rank, at local index experts / world
    sh_inds = torch.tensor([[0, 4], [3, 4], [2, 4]], dtype=torch.int32)
    sh_send = torch.zeros((world, 6, hidden))  # capacity 5
    sh_back = torch.empty((tokens, topk), dtype=torch.int32)
    assert not C.ep_dispatch_ref(x, sh_inds, experts, world, sh_send, sh_back, rank=1, shared=True)
    # rank 0 block: slot (0,0); rank 1 block (row 6 on): (0,1) shared, (1,0), (1,1) shared, (2,0), (2,1) shared
    assert sh_back.tolist() == [[0, 6], [7, 8], [9, 10]]
    assert sh_send[1, 5].view(torch.int32)[:5].tolist() == [2, 1, 2, 0, 2]
    assert torch.equal(sh_send[1, 0], x[0]) and torch.equal(sh_send[1, 4], x[2])
    inds = torch.tensor([[0, 3], [2, -1], [1, 4]], dtype=torch.int32)  # -1 and 4 are outside the bank
    send = torch.full((world, 3, hidden), 7.0)
    back = torch.empty((tokens, topk), dtype=torch.int32)
    assert not C.ep_dispatch_ref(x, inds, experts, world, send, back)
    # rank 0 owns experts 0, 1: slots (0,0) and (2,0); rank 1 owns 2, 3: slots (0,1) and (1,0)
    assert back.tolist() == [[0, 3], [4, -1], [1, -1]]
    assert torch.equal(send[0, 0], x[0]) and torch.equal(send[0, 1], x[2])
    assert torch.equal(send[1, 0], x[0]) and torch.equal(send[1, 1], x[1])
    assert send[0, 2].view(torch.int32)[:2].tolist() == [0, 1]
    assert send[1, 2].view(torch.int32)[:2].tolist() == [1, 0]
    small = torch.zeros((world, 2, hidden))  # capacity 1: the second slot for each peer is dropped
    assert C.ep_dispatch_ref(x, inds, experts, world, small, back)
    assert back.tolist() == [[0, 2], [-1, -1], [-1, -1]]


def test_column_parallel_experts_decompose_exactly(oracle):
    """The column-parallel experts' split (exl3_swiglu_cp): with every rank's expert_columns slices -- gate/up output
    columns [r I/W, (r+1) I/W), down output columns [r D/W, (r+1) D/W) -- the slices' gate/up columns are the whole
    expert's columns bit for bit (output blocks are independent), the down input gathered from all ranks is the whole
    intermediate, and the ranks' output columns reassemble the f32 truth."""
    from plugins_b200 import sharding as S
    O = oracle
    rng = np.random.default_rng(21)
    experts, hidden, inter, n, world, rows, topk = 3, 256, 256, 48, 2, 4, 2
    banks = [_rand_linear(rng, a, b, n, (experts,)) for a, b in ((hidden, inter), (hidden, inter), (inter, hidden))]
    x = rng.standard_normal((rows, hidden)).astype(np.float16).astype(np.float32)
    inds = np.stack([rng.permutation(experts)[:topk] for _ in range(rows)]).astype(np.int32)
    scores = rng.random((rows, topk)).astype(np.float32)

    def sliced(b, c0, c1):
        tr, su, sv = (torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a) for a in b)
        t2, s2, v2 = S.expert_columns(tr, su, sv, c0, c1)
        return t2.numpy().view(np.uint16), s2.numpy(), v2.numpy()

    def proj(b, e, xin, in_f, out_f):
        tr, su, sv = b
        return O.host_project(xin, tr[e], su[e].view(np.uint16), sv[e].view(np.uint16), in_f, out_f, n, threads=2)

    want = O.moe_truth(x, inds, scores, *[(tr, su.view(np.uint16), sv.view(np.uint16), n) for tr, su, sv in banks],
                       hidden, inter, 0.0, threads=2)
    y = np.zeros((rows, hidden), np.float32)
    for t in range(rows):
        for k in range(topk):
            e = int(inds[t, k])
            hs = []
            for r in range(world):  # every rank's slice of the intermediate
                c0, c1 = r * inter // world, (r + 1) * inter // world
                g = proj(sliced(banks[0], c0, c1), e, x[t:t + 1], hidden, c1 - c0)
                u = proj(sliced(banks[1], c0, c1), e, x[t:t + 1], hidden, c1 - c0)
                assert np.array_equal(g, proj(banks[0], e, x[t:t + 1], hidden, inter)[:, c0:c1])
                hs.append(g / (1.0 + np.exp(-g)) * u)
            h = np.concatenate(hs, 1)  # the gathered down input
            outs = []
            for r in range(world):  # every rank's output columns
                d0, d1 = r * hidden // world, (r + 1) * hidden // world
                outs.append(proj(sliced(banks[2], d0, d1), e, h, inter, d1 - d0))
            y[t] += scores[t, k] * np.concatenate(outs, 1)[0]
    rel = np.sqrt(((y - want) ** 2).sum() / (want ** 2).sum())
    assert rel < 1e-5, rel
    with pytest.raises(ValueError):
        S.expert_columns(torch.zeros((1, 1, 16, 48), dtype=torch.int16), torch.zeros((1, 16)), torch.zeros((1, 256)),
                         64, 192)
