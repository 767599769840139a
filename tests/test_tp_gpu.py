"""Column-parallel linears with the all-gather fused into the decode GEMV (exl3_tp_*, plugins_b200/sharding.py
TpExchange): the gathered rows against the single-GPU matmul of the whole layer, stacked shards, graph replay across
the double-buffered steps -- and, when the box has two GPUs, two ranks over NVLink, including the bounded wait's
timeout status when one rank stops taking steps.
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REL_L2_BAR = 2e-3


def _rel(a, b):
    a, b = a.double(), b.double()
    return float(((a - b).norm() / b.norm().clamp_min(1e-30)).item())


def _shard(tr, suh, svh, c0, c1):
    return tr[:, c0 // 16:c1 // 16].contiguous(), suh, svh[c0:c1].contiguous()


def test_one_rank_exchange_matches_matmul_and_replays():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    from plugins_b200 import sharding as S
    in_f, widths, n = 512, (640, 256, 384), 48
    raws = [E.random_linear(in_f, o, n, seed=300 + i) for i, o in enumerate(widths)]
    stacked = Q.stack([Q.weight_from_tensors(*r) for r in raws])
    plain = Q.weight_from_tensors(*E.random_linear(in_f, 1024, 64, seed=310))
    ex = S.TpExchange(0, 1, slots=2, slot_bytes=16 * 1280 * 4, max_cb=16)
    for rows, dt in ((1, torch.float16), (5, torch.bfloat16), (16, torch.float32)):
        x = torch.randn((rows, in_f), device="cuda").to(dt)
        out = torch.empty(2 * ex.slot_bytes, dtype=torch.uint8, device="cuda")
        for _ in range(3):  # parities flip every step
            ex.begin()
            ex.matmul(stacked, x, 0, [0, 0, 0], list(widths))
            ex.matmul(plain, x, 1, [0], [1024])
            ex.gather(0, 2, out)
            torch.cuda.synchronize()
            esize = torch.finfo(dt).bits // 8
            got0 = out[:rows * sum(widths) * esize].view(dt)
            want0 = Q.segment_outputs(stacked, Q.matmul(stacked, x), rows)
            off = 0
            for wd, wo in zip(widths, want0):
                assert _rel(got0[off:off + rows * wd].view(rows, wd).float(), wo.float()) < 1e-6
                off += rows * wd
            got1 = out[ex.slot_bytes:ex.slot_bytes + rows * 1024 * esize].view(dt).view(rows, 1024)
            assert _rel(got1.float(), Q.matmul(plain, x).float()) < 1e-6
    # a captured step replays (the step counter and parity advance on the device)
    x = torch.randn((2, in_f), device="cuda", dtype=torch.float16)
    out = torch.zeros(2 * ex.slot_bytes, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ex.begin(stream=s)
        ex.matmul(plain, x, 1, [0], [1024], stream=s)
        ex.gather(1, 1, out, stream=s)
    want = Q.matmul(plain, x)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out[:2 * 1024 * 2].view(torch.float16).view(2, 1024), want)
    g.reset()
    assert Q.device_error(0) == 0
    ex.close()


def test_one_rank_exchange_on_the_persistent_gemv():
    """Shards whose shape the persistent GEMV serves (a deep narrow one and a wide one) gather through its epilogue:
    the same bytes as exl3_matmul of the shard at 1, 3 and 8 rows (in-CTA rotation, then the prepare launch)."""
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    from plugins_b200 import sharding as S
    for in_f, out_f, n in ((12288, 2048, 48), (4096, 24576, 48)):
        w = Q.weight_from_tensors(*E.random_linear(in_f, out_f, n, seed=320 + out_f))
        ex = S.TpExchange(0, 1, slots=1, slot_bytes=8 * out_f * 2, max_cb=out_f // 128)
        out = torch.empty(ex.slot_bytes, dtype=torch.uint8, device="cuda")
        for rows in (1, 3, 8):
            x = torch.randn((rows, in_f), device="cuda", dtype=torch.float16)
            for _ in range(2):  # both parities
                ex.begin()
                ex.matmul(w, x, 0, [0], [out_f])
                ex.gather(0, 1, out)
                torch.cuda.synchronize()
                got = out[:rows * out_f * 2].view(torch.float16).view(rows, out_f)
                assert torch.equal(got, Q.matmul(w, x)), (in_f, out_f, rows)
        assert Q.device_error(0) == 0
        ex.close()


def test_one_rank_timeline_stamps_each_phase_in_order(monkeypatch):
    """EXL3_TRACE=1 at create: each step's four stamps (begin, publish, every rank seen, gathered) come back oldest
    step first and in order; an exchange made without it refuses the read by name."""
    from plugins_b200 import encoder as E
    from plugins_b200 import quant as Q
    from plugins_b200 import sharding as S
    w = Q.weight_from_tensors(*E.random_linear(512, 1024, 64, seed=311))
    x = torch.randn((1, 512), device="cuda", dtype=torch.float16)
    out = torch.empty(1024 * 2, dtype=torch.uint8, device="cuda")
    plain = S.TpExchange(0, 1, slots=1, slot_bytes=1024 * 2, max_cb=8)
    with pytest.raises(Q.Exl3Error, match="without EXL3_TRACE=1"):
        plain.trace()
    plain.close()
    monkeypatch.setenv("EXL3_TRACE", "1")
    ex = S.TpExchange(0, 1, slots=1, slot_bytes=1024 * 2, max_cb=8)
    monkeypatch.delenv("EXL3_TRACE")
    for steps in (3, 20):  # 20 steps wrap the 16-step ring
        for _ in range(steps - (3 if steps == 20 else 0)):
            ex.begin()
            ex.matmul(w, x, 0, [0], [1024])
            ex.gather(0, 1, out)
        got = ex.trace()
        assert len(got) == min(steps, 16)
        for st in got:
            assert all(st[:4]) and st[0] <= st[1] <= st[2] <= st[3] and not any(st[4:]), st
        assert all(a[0] <= b[0] for a, b in zip(got, got[1:]))
    assert Q.device_error(0) == 0
    ex.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        from plugins_b200 import encoder as E
        from plugins_b200 import quant as Q
        from plugins_b200 import sharding as S
        in_f, n = 1024, 64
        widths = (1280, 512, 512)  # q|k|v-like: the 1280 = 10 blocks split 5 / 5, 512 = 4 blocks split 2 / 2
        raws = [E.random_linear(in_f, o, n, seed=400 + i, device=dev) for i, o in enumerate(widths)]
        shards, col0 = [], []
        for (tr, suh, svh), wd in zip(raws, widths):
            c0, c1 = S.column_range(wd, rank, world)
            shards.append(Q.weight_from_tensors(*_shard(tr, suh, svh, c0, c1)))
            col0.append(c0)
        stacked = Q.stack(shards)
        full = [Q.weight_from_tensors(*r) for r in raws]
        ex = S.TpExchange(rank, world, slots=1, slot_bytes=16 * sum(widths) * 2, max_cb=64)
        g = torch.Generator(device=dev).manual_seed(7)
        out = torch.empty(ex.slot_bytes, dtype=torch.uint8, device=dev)
        for rows in (1, 8, 16):
            x = torch.randn((rows, in_f), device=dev, generator=g).half()  # the same x on both ranks
            for _ in range(3):
                ex.begin()
                ex.matmul(stacked, x, 0, col0, list(widths))
                ex.gather(0, 1, out)
                torch.cuda.synchronize()
                got = out[:rows * sum(widths) * 2].view(torch.float16)
                off = 0
                for w, wd in zip(full, widths):
                    want = Q.matmul(w, x)
                    rel = _rel(got[off:off + rows * wd].view(rows, wd).float(), want.float())
                    assert rel < 1e-3, (rank, rows, wd, rel)
                    off += rows * wd
        assert Q.device_error(rank) == 0
        # a rank that stops taking steps (between steps: none of its kernels in flight): the other's gather waits
        # for a flag nothing sets, gives up after about a second with EXL3_ERR_TP_TIMEOUT, and its context runs on
        from plugins_b200 import _lib as L
        dist.barrier()
        if rank == 0:
            x = torch.randn((1, in_f), device=dev).half()
            ex.begin()
            ex.matmul(stacked, x, 0, col0, list(widths))
            ex.gather(0, 1, out)
            torch.cuda.synchronize()
            assert Q.device_error(0, clear=True) & L.ERR_TP_TIMEOUT
            assert torch.isfinite(Q.matmul(full[0], x).float()).all()
        dist.barrier()  # rank 1 keeps its exchange mapped until rank 0's kernels are done
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_gather_inside_the_gemv():
    import torch.multiprocessing as mp
    mp.spawn(_tp_rank, args=(2, _free_port()), nprocs=2)
