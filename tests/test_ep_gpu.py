"""Expert parallelism on the GPU: exl3_ep_dispatch / exl3_ep_unpack / exl3_ep_combine against their host restatement
(tests/sharding_cpu_ops.py), the expert-parallel driver against the single-GPU swiglu and the f32 truth, its
peer-memory exchange (exl3_epx_*) against the all-to-all one, the column-parallel experts (exl3_swiglu_cp) against the
single-GPU swiglu, and -- when the box has two GPUs -- both drivers on two ranks, with a rank that stops taking steps.
"""
import datetime
import os
import socket

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


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / max((b ** 2).sum(), 1e-30)))


def _routing(tokens, topk, experts, seed):
    g = torch.Generator().manual_seed(seed)
    inds = torch.stack([torch.randperm(experts, generator=g)[:topk] for _ in range(tokens)]).to(torch.int32)
    scores = torch.rand((tokens, topk), generator=g)
    return inds, scores


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_dispatch_unpack_combine_match_the_host_restatement(Q, dtype):
    import sharding_cpu_ops as C
    from plugins_b200 import _lib as L
    from plugins_b200 import sharding as S
    torch.manual_seed(0)
    tokens, topk, experts, world, hidden = 5, 3, 6, 3, 256
    inds, scores = _routing(tokens, topk, experts, 1)
    inds[1, 2] = -1
    inds[3, 0] = experts  # absent: outside the bank
    x = torch.randn((tokens, hidden)).to(dtype)
    cap = S.ep_capacity(tokens, topk, experts, world)
    send_ref = torch.zeros((world, cap + 1, hidden), dtype=dtype)
    back_ref = torch.empty((tokens, topk), dtype=torch.int32)
    C.ep_dispatch_ref(x, inds, experts, world, send_ref, back_ref)
    send = torch.empty((world, cap + 1, hidden), dtype=dtype, device="cuda")
    back = torch.empty((tokens, topk), dtype=torch.int32, device="cuda")
    Q.ep_dispatch(x.cuda(), inds.cuda(), experts, world, send, back)
    torch.cuda.synchronize()
    assert torch.equal(back.cpu(), back_ref)
    got = send.cpu()
    for d in range(world):
        meta = got[d, cap].view(torch.int32)[:cap]
        assert torch.equal(meta, send_ref[d, cap].view(torch.int32)[:cap])
        rows = int((meta >= 0).sum())
        assert torch.equal(got[d, :rows].view(torch.int16), send_ref[d, :rows].view(torch.int16)) if dtype == torch.float16 \
            else torch.equal(got[d, :rows], send_ref[d, :rows])
    # unpack: the received blocks (here: the sent ones) -> swiglu's indices
    ui = torch.empty((world, cap + 1, 1), dtype=torch.int32, device="cuda")
    us = torch.empty((world, cap + 1, 1), dtype=torch.float32, device="cuda")
    Q.ep_unpack(send, ui, us)
    ui_ref, us_ref = torch.empty_like(ui.cpu()), torch.empty_like(us.cpu())
    C.ep_unpack_ref(got, ui_ref, us_ref)
    assert torch.equal(ui.cpu(), ui_ref) and torch.equal(us.cpu(), us_ref)
    # combine
    rows_back = torch.randn((world, cap + 1, hidden))
    shared = torch.randn((tokens, hidden))
    out = torch.empty((tokens, hidden), dtype=dtype, device="cuda")
    Q.ep_combine(rows_back.cuda(), back, scores.cuda(), shared.cuda(), out)
    out_ref = torch.empty((tokens, hidden), dtype=dtype)
    C.ep_combine_ref(rows_back, back_ref, scores, shared, out_ref)
    # same sums in the same order; the kernel fuses score * row + acc, the restatement rounds the product first, so
    # an f16 output can differ by one unit in the last place
    assert _rel(out.float().cpu(), out_ref.float()) < (1e-6 if dtype == torch.float32 else 2e-4)
    # the shared expert (id `experts`) stays on the calling rank, at local index experts / world
    sh_inds = torch.cat([inds, torch.full((tokens, 1), experts, dtype=torch.int32)], 1)
    cap2 = S.ep_capacity(tokens, topk, experts, world, shared=True)
    send2 = torch.empty((world, cap2 + 1, hidden), dtype=dtype, device="cuda")
    back2 = torch.empty((tokens, topk + 1), dtype=torch.int32, device="cuda")
    Q.ep_dispatch(x.cuda(), sh_inds.cuda(), experts, world, send2, back2, rank=2, shared=True)
    send2_ref = torch.zeros((world, cap2 + 1, hidden), dtype=dtype)
    back2_ref = torch.empty((tokens, topk + 1), dtype=torch.int32)
    C.ep_dispatch_ref(x, sh_inds, experts, world, send2_ref, back2_ref, rank=2, shared=True)
    torch.cuda.synchronize()
    assert torch.equal(back2.cpu(), back2_ref)
    for d in range(world):
        assert torch.equal(send2.cpu()[d, cap2].view(torch.int32)[:cap2], send2_ref[d, cap2].view(torch.int32)[:cap2])
    assert Q.device_error(0) & L.ERR_EP_OVERFLOW == 0


def test_dispatch_overflow_is_flagged(Q):
    from plugins_b200 import _lib as L
    tokens, topk, experts, world, hidden = 4, 2, 4, 2, 128
    inds = torch.tensor([[0, 1], [0, 1], [2, 3], [0, 2]], dtype=torch.int32, device="cuda")
    x = torch.randn((tokens, hidden), device="cuda", dtype=torch.float16)
    send = torch.empty((world, 3, hidden), dtype=torch.float16, device="cuda")  # capacity 2: rank 0 gets 5 slots
    back = torch.empty((tokens, topk), dtype=torch.int32, device="cuda")
    Q.device_error(0, clear=True)
    Q.ep_dispatch(x, inds, experts, world, send, back)
    torch.cuda.synchronize()
    assert Q.device_error(0, clear=True) & L.ERR_EP_OVERFLOW
    assert back.cpu().tolist() == [[0, 1], [-1, -1], [3, 4], [-1, -1]]


def _banks(E, experts, hidden, inter, n, seed, device="cuda"):
    out = []
    for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden))):
        out.append(E.random_linear(a, b, n, seed=seed + i, groups=experts, device=device))
    return out


def _np(t):
    return t.detach().cpu().numpy()


def test_expert_parallel_on_one_rank_matches_swiglu_and_truth(Q, oracle):
    from plugins_b200 import encoder as E
    from plugins_b200 import sharding as S
    experts, hidden, inter, n, tokens, topk = 16, 512, 256, 48, 12, 4
    raw = _banks(E, experts, hidden, inter, n, 40)
    sraw = _banks(E, 1, hidden, inter, n, 50)
    inds, scores = _routing(tokens, topk, experts, 2)
    inds, scores = inds.cuda(), scores.cuda()
    x = torch.randn((tokens, hidden), device="cuda", dtype=torch.float16)
    # the bank with the shared expert appended (local index experts / world = experts at one rank)
    ext = [Q.weight_from_tensors(torch.cat([r[0], s[0]]), torch.cat([r[1], s[1]]), torch.cat([r[2], s[2]]))
           for r, s in zip(raw, sraw)]
    ep = S.ExpertParallelSwiglu(*ext, experts=experts, tokens=tokens, topk=topk, hidden=hidden, rank=0, world=1,
                                shared=True)
    got = ep.forward(x, inds, scores)
    # the single-GPU path: the shared expert as one more slot of score 1
    inds2 = torch.cat([inds, torch.full((tokens, 1), experts, dtype=torch.int32, device="cuda")], 1)
    sc2 = torch.cat([scores, torch.ones((tokens, 1), device="cuda")], 1)
    single = Q.swiglu(*ext, x.view(1, tokens, hidden), inds2.view(1, tokens, topk + 1).contiguous(),
                      sc2.view(1, tokens, topk + 1).contiguous()).view(tokens, hidden)
    assert _rel(_np(got.float()), _np(single.float())) < 1e-5  # the same sums in the same order
    bank = lambda b: (_np(b[0]).view(np.uint16), _np(b[1]).view(np.uint16), _np(b[2]).view(np.uint16), n)
    want = oracle.moe_truth(_np(x.float()), _np(inds2), _np(sc2), *[bank(
        (torch.cat([r[0], s[0]]), torch.cat([r[1], s[1]]), torch.cat([r[2], s[2]]))) for r, s in zip(raw, sraw)],
        hidden, inter, 0.0, threads=os.cpu_count() or 8)
    assert _rel(_np(got.float()), want) < REL_L2_BAR


def test_peer_exchange_on_one_rank_matches_the_all_to_all_and_replays(Q):
    """world 1: the peer exchange's kernels (dispatch into the receive region, receive copy, return, combine) give the
    same bits as the all-to-all path; a captured step replayed on new inputs alternates the two copies of the
    regions and stays equal."""
    from plugins_b200 import encoder as E
    from plugins_b200 import sharding as S
    experts, hidden, inter, n, tokens, topk = 8, 256, 256, 48, 10, 3
    raw = _banks(E, experts + 1, hidden, inter, n, 70)  # 8 routed experts and the shared one last
    banks = [Q.weight_from_tensors(*b) for b in raw]
    kw = dict(experts=experts, tokens=tokens, topk=topk, hidden=hidden, rank=0, world=1, shared=True)
    a2a = S.ExpertParallelSwiglu(*banks, **kw)
    peer = S.ExpertParallelSwiglu(*banks, exchange="peer", **kw)
    x = torch.empty((tokens, hidden), device="cuda", dtype=torch.float16)
    inds = torch.empty((tokens, topk), device="cuda", dtype=torch.int32)
    sc = torch.empty((tokens, topk), device="cuda")
    out = torch.empty((tokens, hidden), device="cuda", dtype=torch.float16)

    def draw(seed):
        g = torch.Generator(device="cuda").manual_seed(seed)
        x.copy_(torch.randn((tokens, hidden), device="cuda", generator=g).half())
        i, s_ = _routing(tokens, topk, experts, seed)
        i[1, 2] = -1  # an absent slot
        inds.copy_(i)
        sc.copy_(s_)

    for seed in (1, 2, 3):
        draw(seed)
        assert torch.equal(peer.forward(x, inds, sc), a2a.forward(x, inds, sc))
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st), torch.cuda.graph(graph, stream=st):
        peer.forward(x, inds, sc, out=out)
    torch.cuda.current_stream().wait_stream(st)
    for seed in (4, 5, 6, 7):
        draw(seed)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, a2a.forward(x, inds, sc)), seed
    del graph
    assert Q.device_error(0) == 0
    peer.peer.close()


def test_column_parallel_experts_on_one_rank_match_swiglu_and_replay(Q):
    """world 1: the column-parallel call (gather, route, gate|up storing the down input through the exchange, down,
    combine, return) gives swiglu's bits; a captured call replayed on new inputs stays equal."""
    from plugins_b200 import encoder as E
    from plugins_b200 import sharding as S
    experts, hidden, inter, n, tokens, topk = 8, 256, 384, 48, 10, 3
    raw = _banks(E, experts + 1, hidden, inter, n, 80)  # 8 routed experts and the shared one last
    banks = [Q.weight_from_tensors(*b) for b in raw]
    cp = S.ColumnParallelExperts(*banks, experts=experts, tokens=tokens, topk=topk, hidden=hidden, inter=inter, rank=0,
                                 world=1, shared=True)
    x = torch.empty((tokens, hidden), device="cuda", dtype=torch.float16)
    inds = torch.empty((tokens, topk), device="cuda", dtype=torch.int32)
    sc = torch.empty((tokens, topk), device="cuda")
    out = torch.empty((tokens, hidden), device="cuda", dtype=torch.float16)

    def draw(seed):
        g = torch.Generator(device="cuda").manual_seed(seed)
        x.copy_(torch.randn((tokens, hidden), device="cuda", generator=g).half())
        i, s_ = _routing(tokens, topk, experts, seed)
        i[2, 1] = -1  # an absent slot
        inds.copy_(i)
        sc.copy_(s_)

    def single():
        i2 = torch.cat([inds, torch.full((tokens, 1), experts, dtype=torch.int32, device="cuda")], 1)
        s2 = torch.cat([sc, torch.ones((tokens, 1), device="cuda")], 1)
        return Q.swiglu(*banks, x.view(1, tokens, hidden), i2.view(1, tokens, topk + 1).contiguous(),
                        s2.view(1, tokens, topk + 1).contiguous()).view(tokens, hidden)

    for seed in (1, 2):
        draw(seed)
        assert torch.equal(cp.forward(x, inds, sc), single())
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st), torch.cuda.graph(graph, stream=st):
        cp.forward(x, inds, sc, out=out)
    torch.cuda.current_stream().wait_stream(st)
    for seed in (3, 4, 5):
        draw(seed)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, single()), seed
    del graph
    assert Q.device_error(0) == 0
    cp.close()


def test_peer_and_column_exchange_timelines_on_one_rank(monkeypatch):
    """EXL3_TRACE=1 at create: the expert-parallel and column-parallel exchanges stamp their eight phases of every
    step in order (dispatch / copies / waits / the caller's swiglu / return / combine; tokens / gate|up / down /
    out), oldest step first."""
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    from plugins_b200 import sharding as S
    experts, hidden, inter, n, tokens, topk = 8, 256, 256, 48, 6, 2
    banks = [Q.weight_from_tensors(*b) for b in _banks(E, experts + 1, hidden, inter, n, 90)]
    monkeypatch.setenv("EXL3_TRACE", "1")
    peer = S.ExpertParallelSwiglu(*banks, experts=experts, tokens=tokens, topk=topk, hidden=hidden, rank=0, world=1,
                                  shared=True, exchange="peer")
    cp = S.ColumnParallelExperts(*banks, experts=experts, tokens=tokens, topk=topk, hidden=hidden, inter=inter, rank=0,
                                 world=1, shared=True)
    monkeypatch.delenv("EXL3_TRACE")
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((tokens, hidden), device="cuda", generator=g).half()
    inds, sc = [t.cuda() for t in _routing(tokens, topk, experts, 5)]
    for _ in range(4):
        peer.forward(x, inds, sc)
        cp.forward(x, inds, sc)
    for got in (peer.peer.trace(), cp.trace()):
        assert len(got) == 4
        for st in got:
            assert all(st) and all(a <= b for a, b in zip(st, st[1:])), st
        assert all(a[7] <= b[0] for a, b in zip(got, got[1:]))
    assert Q.device_error(0) == 0
    peer.peer.close()
    cp.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_two_gpu_rank(rank, world, port, exchange="nccl"):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from plugins_b200 import encoder as E
        from plugins_b200 import quant as Q
        from plugins_b200 import sharding as S
        experts, hidden, inter, n, tokens, topk = 8, 512, 256, 48, 6, 3
        raw = _banks(E, experts, hidden, inter, n, 60, device=dev)  # seeded: identical on both GPUs
        e0, e1 = S.expert_range(experts, rank, world)
        local = [Q.weight_from_tensors(b[0][e0:e1].contiguous(), b[1][e0:e1].contiguous(), b[2][e0:e1].contiguous())
                 for b in raw]
        g = torch.Generator(device=dev).manual_seed(3)
        x_all = torch.randn((world * tokens, hidden), device=dev, generator=g).half()
        inds_all, sc_all = _routing(world * tokens, topk, experts, 4)
        inds_all, sc_all = inds_all.to(dev), sc_all.to(dev)
        sl = slice(rank * tokens, (rank + 1) * tokens)
        ep = S.ExpertParallelSwiglu(*local, experts=experts, tokens=tokens, topk=topk, hidden=hidden, rank=rank,
                                    world=world, device=dev, exchange=exchange)
        full = [Q.weight_from_tensors(*b) for b in raw]
        want = Q.swiglu(*full, x_all[sl].contiguous().view(1, tokens, hidden),
                        inds_all[sl].contiguous().view(1, tokens, topk), sc_all[sl].contiguous().view(1, tokens, topk))
        for _ in range(3):  # (the peer exchange alternates its two copies of the regions)
            got = ep.forward(x_all[sl].contiguous(), inds_all[sl].contiguous(), sc_all[sl].contiguous())
            rel = float(((got.float() - want.view(tokens, hidden).float()).norm() / want.float().norm()).item())
            assert rel < 1e-3, rel
        torch.cuda.synchronize()
        assert Q.device_error(rank) == 0
        if exchange == "peer":
            # a rank that stops taking steps (between steps: none of its kernels in flight): the other's receive and
            # combine wait for flags nothing sets, give up after about a second each with EXL3_ERR_EP_TIMEOUT, and
            # its context runs on
            from plugins_b200 import _lib as L
            dist.barrier()
            if rank == 0:
                ep.forward(x_all[sl].contiguous(), inds_all[sl].contiguous(), sc_all[sl].contiguous())
                torch.cuda.synchronize()
                assert Q.device_error(0, clear=True) & L.ERR_EP_TIMEOUT
                assert torch.isfinite(Q.swiglu(*full, x_all[sl].contiguous().view(1, tokens, hidden),
                                               inds_all[sl].contiguous().view(1, tokens, topk),
                                               sc_all[sl].contiguous().view(1, tokens, topk)).float()).all()
            dist.barrier()  # rank 1 keeps its regions mapped until rank 0's kernels are done
            ep.peer.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _cp_two_gpu_rank(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from plugins_b200 import encoder as E
        from plugins_b200 import quant as Q
        from plugins_b200 import sharding as S
        experts, hidden, inter, n, tokens, topk = 8, 512, 512, 48, 6, 3
        raw = _banks(E, experts + 1, hidden, inter, n, 90, device=dev)  # seeded: identical on both GPUs; shared last
        c0, c1 = rank * inter // world, (rank + 1) * inter // world
        h0, h1 = rank * hidden // world, (rank + 1) * hidden // world
        local = [Q.weight_from_tensors(*S.expert_columns(*raw[0], c0, c1)),
                 Q.weight_from_tensors(*S.expert_columns(*raw[1], c0, c1)),
                 Q.weight_from_tensors(*S.expert_columns(*raw[2], h0, h1))]
        g = torch.Generator(device=dev).manual_seed(3)
        x_all = torch.randn((world * tokens, hidden), device=dev, generator=g).half()
        inds_all, sc_all = _routing(world * tokens, topk, experts, 4)
        inds_all, sc_all = inds_all.to(dev), sc_all.to(dev)
        sl = slice(rank * tokens, (rank + 1) * tokens)
        cp = S.ColumnParallelExperts(*local, experts=experts, tokens=tokens, topk=topk, hidden=hidden, inter=inter,
                                     rank=rank, world=world, device=dev, shared=True)
        full = [Q.weight_from_tensors(*b) for b in raw]
        i2 = torch.cat([inds_all[sl], torch.full((tokens, 1), experts, dtype=torch.int32, device=dev)], 1).contiguous()
        s2 = torch.cat([sc_all[sl], torch.ones((tokens, 1), device=dev)], 1).contiguous()
        want = Q.swiglu(*full, x_all[sl].contiguous().view(1, tokens, hidden), i2.view(1, tokens, topk + 1),
                        s2.view(1, tokens, topk + 1)).view(tokens, hidden)
        for _ in range(3):
            got = cp.forward(x_all[sl].contiguous(), inds_all[sl].contiguous(), sc_all[sl].contiguous())
            rel = float(((got.float() - want.float()).norm() / want.float().norm()).item())
            assert rel < 1e-3, rel
        torch.cuda.synchronize()
        assert Q.device_error(rank) == 0
        # a rank that stops taking calls (between calls: none of its kernels in flight): the other's waits give up
        # after about a second each with EXL3_ERR_EP_TIMEOUT, and its context runs on
        from plugins_b200 import _lib as L
        dist.barrier()
        if rank == 0:
            cp.forward(x_all[sl].contiguous(), inds_all[sl].contiguous(), sc_all[sl].contiguous())
            torch.cuda.synchronize()
            assert Q.device_error(0, clear=True) & L.ERR_EP_TIMEOUT
            assert torch.isfinite(Q.swiglu(*full, x_all[sl].contiguous().view(1, tokens, hidden),
                                           i2.view(1, tokens, topk + 1), s2.view(1, tokens, topk + 1)).float()).all()
        dist.barrier()  # rank 1 keeps its exchange mapped until rank 0's kernels are done
        cp.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_column_parallel_experts_on_two_gpus(Q):
    import torch.multiprocessing as mp
    mp.spawn(_cp_two_gpu_rank, args=(2, _free_port()), nprocs=2)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_expert_parallel_on_two_gpus(Q, exchange):
    import torch.multiprocessing as mp
    mp.spawn(_ep_two_gpu_rank, args=(2, _free_port(), exchange), nprocs=2)
