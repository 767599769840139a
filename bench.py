"""Benchmark of the EXL3 decode path on B200: the Qwen3-8B-shaped 36-layer linear stack.

Metric: "EXL3 GEMV HBM GB/s (% of peak) and decode tok/s at 1/2/4/8 B200 vs host CPU".  One step = every linear of
one decode token through the library: per layer q|k|v (4096 -> 4096+1024+1024, 4 bpw, one stacked launch), o
(4096 -> 4096, 4 bpw), gate|up (4096 -> 12288+12288, 3 bpw, one stacked launch) and down (12288 -> 4096, 3 bpw).
Weights are random-init N(0, 0.02) (seed 1 + linear index) encoded by the library's encoder; activations N(0, 1) f16,
each linear reading its own resident input.  `value` is algorithmic bytes (trellis + suh + svh + activations, each
distinct weight once) per second over CUDA-graph replays of whole steps; `e2e` adds the pinned host->device copy of a
step's inputs and the device->host copy of its outputs.  At N > 1 GPUs each linear is column-parallel (output rows
split over ranks, 128-aligned) and every launch's output is all-gathered over NCCL (strong scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, HEADS_Q, KV = 4096, 4096, 1024
INTER, LAYERS = 12288, 36
METRIC = "EXL3 GEMV HBM GB/s (% of peak) and decode tok/s at 1/2/4/8 B200 vs host CPU"
WORKLOAD = "qwen3-8b-shaped EXL3 decode linear stack (36 layers; q/k/v/o 4 bpw, gate/up/down 3 bpw)"

# (name, in, out, bits) per layer, in launch order; q|k|v and gate|up are stacked launches
LINEARS = [("q", HIDDEN, HEADS_Q, 4), ("k", HIDDEN, KV, 4), ("v", HIDDEN, KV, 4), ("o", HIDDEN, HIDDEN, 4),
           ("gate", HIDDEN, INTER, 3), ("up", HIDDEN, INTER, 3), ("down", INTER, HIDDEN, 3)]
GROUPS = [("qkv", ["q", "k", "v"]), ("o", ["o"]), ("gate_up", ["gate", "up"]), ("down", ["down"])]
GEMV6_MIN_SLABS, GEMV6_MIN_SLABS_DEEP = 49152, 16384  # the library's kGemv6MinSlabs / kGemv6MinSlabsDeep
GEMV6_NARROW_CB, GEMV6_NARROW_SLABS = 64, 8192  # the library's kGemv6NarrowCb / kGemv6NarrowSlabs
CTA_ROTATE_ROWS = 1  # the library's kCtaRotateRows: more rows take the cluster-split GEMV's prepare launch
XI_TAKE = 1  # the library's kXiTake: more rows take the persistent GEMV's prepare launch


def gemv_kernels(in_f: int, out_f: int, exchange: bool, rows: int = 1, sms: int = 148) -> int:
    """Kernels one decode-GEMV call launches (the selection in plugins_b200/csrc/exl3_abi.cu and exl3_gemv6.cu): the
    persistent GEMV for large and for narrow launches -- one kernel when its CTAs rotate the input themselves (XI_TAKE
    rows, runs of at most 128 slabs), else a prepare launch and the GEMV -- and the cluster-split GEMV otherwise: one
    launch at one row (its CTAs rotate their slabs' input), a prepare launch and the GEMV from CTA_ROTATE_ROWS + 1
    rows; the column-parallel exchange (`exchange`) takes the same kernels as its shard's shape."""
    cb, kt = out_f // 128, in_f // 16
    if not gemv6_serves(in_f, out_f):
        return 1 if rows <= CTA_ROTATE_ROWS else 2
    v = sms * 3
    dp = cb // v * v
    run = -(-(cb - dp) * kt // v)
    run = (32 if run < 32 else run + 3) & ~3
    return 1 if rows <= XI_TAKE and dp == 0 and run <= 128 else 2


def gemv6_serves(in_f: int, out_f: int) -> bool:
    """The library's gemv6_prefers: the shapes the persistent GEMV takes."""
    cb, kt = out_f // 128, in_f // 16
    slabs = cb * kt
    return (slabs >= GEMV6_MIN_SLABS or (in_f >= 8192 and slabs >= GEMV6_MIN_SLABS_DEEP)
            or (cb <= GEMV6_NARROW_CB and slabs >= GEMV6_NARROW_SLABS))


def gemv6_mode(in_f: int, out_f: int, exchange: bool, rows: int = 1) -> int:
    """0: the cluster-split GEMV; 1: the persistent one rotating its input in-CTA; 2: prepare launch + persistent.
    The column-parallel exchange takes the same kernel as its shard's shape."""
    if not gemv6_serves(in_f, out_f):
        return 0
    return gemv_kernels(in_f, out_f, exchange, rows)


def linear_bytes(i: int, o: int, bits: int, rows: int) -> int:
    """Algorithmic bytes of one linear: trellis + suh + svh + x + y (f16)."""
    return i * o * bits // 8 + 2 * i + 2 * o + 2 * rows * (i + o)


def step_bytes(rows: int) -> int:
    return LAYERS * sum(linear_bytes(i, o, b, rows) for _, i, o, b in LINEARS)


def load_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ------------------------------------------------------------------ the other configs (N = 1, rank 0)

def _graph_ms(torch, fn, reps: int, inner: int = 4) -> float:
    """Milliseconds per call of fn, replayed as a CUDA graph of `inner` calls after warm-up (device time, events)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(inner):
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    g.reset()
    return e0.elapsed_time(e1) / (reps * inner)


def measure_layer(Q, E, torch, peaks: dict, in_f: int, out_f: int, bits: int, seed: int, label: str,
                  copies: int = 36, reps: int = 20) -> dict:
    """One decode-GEMV layer at batch 1: W N(0, 0.02) (seed) encoded at `bits` by the library's encoder, held as
    `copies` distinct device copies (so consecutive launches stream distinct bytes, >> 126 MB L2), the copies' launches
    captured back to back in one CUDA graph; each replay is timed with events on its stream, and the median and the
    fastest replay give microseconds per launch (the reference's chainNs statistics, SX/bench_util.zig:41-74)."""
    n = 16 * bits
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn((out_f, in_f), generator=g, device="cuda") * 0.02
    tr, suh, svh = E.quantize(w, bits, seed)
    del w
    trs = [tr.clone() for _ in range(copies)]
    ws = [Q.weight_from_tensors(t, suh, svh) for t in trs]
    x = torch.randn((1, in_f), generator=g, device="cuda").half()
    y = torch.empty((1, out_f), device="cuda", dtype=torch.float16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for wi in ws[:3]:
            Q.matmul(wi, x, out=y)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=s):
        for wi in ws:
            Q.matmul(wi, x, out=y)
    for _ in range(5):
        gr.replay()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    with torch.cuda.stream(s):
        ev[0].record(s)
        for i in range(reps):
            gr.replay()
            ev[i + 1].record(s)
    torch.cuda.synchronize()
    per = sorted(ev[i].elapsed_time(ev[i + 1]) * 1000.0 / copies for i in range(reps))
    gr.reset()
    nbytes = linear_bytes(in_f, out_f, bits, 1)
    med, fast = statistics.median(per), per[0]
    gbs = nbytes / (med * 1e-6) / 1e9
    del ws, trs
    return {"workload": label, "us_per_launch": round(med, 3), "us_fastest": round(fast, 3),
            "value": round(gbs, 1), "unit": "GB/s", "bytes_per_launch": nbytes,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "frac_fastest": round(nbytes / (fast * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)"},
            "timing": f"{copies} distinct copies per CUDA-graph replay, {reps} replays timed one by one with events; "
                      "median (value) and fastest",
            "l2": "no flush: a replay streams %.2f GB of distinct weights (> 126 MB L2)" % (copies * nbytes / 1e9)}


def measure_prefill(Q, E, torch, peaks: dict, reps: int = 10) -> dict:
    """Config 3: X [M, 4096] bf16 through the 4096 x 12288 4-bpw layer (seed 2), M = 2048 headline plus 64, 256 and
    8192 for the GEMV/GEMM crossover.  Whole-path time per call (operand images + tensor-core GEMM) and the GEMM
    kernel alone, from events recorded between the launches (exl3_matmul_timed); medians of `reps` calls.  At 64
    and 256 rows the same rows forced through the decode GEMV are timed too."""
    in_f, out_f, n = 4096, 12288, 64
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=2)
    w = Q.weight_from_tensors(tr, suh, svh)
    rows_list, out = (2048, 64, 256, 8192), {}
    for m in rows_list:
        g = torch.Generator(device="cuda").manual_seed(m)
        x = torch.randn((m, in_f), device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty((m, out_f), device="cuda", dtype=torch.bfloat16)
        rec = {}
        for label, flags in (("gemm", 16), ("gemv", 8)):
            if label == "gemv" and m > 256:
                continue
            for _ in range(3):
                Q.matmul_ex(w, x, flags, out=y)
            tot, img, mm = [], [], []
            for _ in range(reps):
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
                for e in ev:
                    e.record()
                Q.matmul_timed(w, x, ev, flags=flags, out=y)
                torch.cuda.synchronize()
                tot.append(ev[0].elapsed_time(ev[3]))
                if label == "gemm":
                    img.append(ev[0].elapsed_time(ev[1]))
                    mm.append(ev[1].elapsed_time(ev[2]))
            rec[label + "_ms"] = round(statistics.median(tot), 4)
            if label == "gemm":
                rec["images_ms"] = round(statistics.median(img), 4)
                rec["gemm_kernel_ms"] = round(statistics.median(mm), 4)
        out[m] = rec
    # resident (quant.zig:96-101): the decoded matrix kept from the first prefill call on, so later calls only prepare
    # the rows (no decode); the same 2048-row call
    x = torch.randn((2048, in_f), device="cuda", generator=torch.Generator(device="cuda").manual_seed(2048)).to(
        torch.bfloat16)
    y = torch.empty((2048, out_f), device="cuda", dtype=torch.bfloat16)
    kept = Q.resident([w])
    try:
        for _ in range(3):
            Q.matmul_ex(w, x, 16, out=y)
        tot = []
        for _ in range(reps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            for e in ev:
                e.record()
            Q.matmul_timed(w, x, ev, flags=16, out=y)
            torch.cuda.synchronize()
            tot.append(ev[0].elapsed_time(ev[3]))
        res_ms = statistics.median(tot)
    finally:
        Q.resident([])
    del w
    flops = 2.0 * 2048 * in_f * out_f
    h = out[2048]
    tf_total = flops / (h["gemm_ms"] * 1e-3) / 1e12
    tf_kernel = flops / (h["gemm_kernel_ms"] * 1e-3) / 1e12
    return {
        "workload": "config 3: X [2048, 4096] bf16 x EXL3 4 bpw 4096 x 12288 (random trellis, seed 2), bf16 out",
        "value": round(tf_total, 1), "unit": "TFLOP/s", "ms": h["gemm_ms"],
        "frac_of_bf16_peak": round(tf_total / peaks["bf16_tflops"], 4),
        "phases_ms": {"operand_images": h["images_ms"], "gemm_kernel": h["gemm_kernel_ms"]},
        "roofline": {"bound": "tensor", "achieved": round(tf_kernel, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(tf_kernel / peaks["bf16_tflops"], 4), "traffic": None,
                     "kernel": "gemm_image_kernel (tcgen05.mma kind::f16, TMEM accumulators)",
                     "flops_per_launch": flops,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json bf16_tflops, burst)"},
        "crossover": [{"rows": m, **out[m]} for m in sorted(out)],
        "resident": {"ms": round(res_ms, 4), "value": round(flops / (res_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                     "kept_bytes": kept,
                     "note": "exl3_resident: W_hat^T's operand image kept from the first call; later calls prepare "
                             "only the rows (no decode) before the GEMM"},
        "l2": "no flush: each call writes and reads a 100.7 MB B image and reads 25 MB of trellis (> 126 MB L2)",
    }


def measure_moe(Q, E, torch, peaks: dict, reps: int = 10) -> dict:
    """Config 4: 256 routed experts + 1 shared, hidden 4096, intermediate 2048, 3 bpw (random trellis, seed 3), 32
    tokens, top-8 of a softmax over N(0, 1) router logits (seed 4).  The shared expert is bank entry 256, routed to
    every token with score 1 (the reference's moeSwigluFusedWithShared sums it in the same way); one swiglu call."""
    experts, hidden, inter, topk, tokens = 256, 4096, 2048, 8, 32
    banks = []
    for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden))):
        tr, suh, svh = E.random_linear(a, b, 48, seed=3 + i, groups=experts + 1)
        banks.append(Q.weight_from_tensors(tr, suh, svh))
    g = torch.Generator(device="cuda").manual_seed(4)
    logits = torch.randn((tokens, experts), device="cuda", generator=g)
    sc, ind = torch.topk(torch.softmax(logits, -1), topk, -1)
    ind = torch.cat([ind.to(torch.int32), torch.full((tokens, 1), experts, dtype=torch.int32, device="cuda")], 1)
    sc = torch.cat([sc.float(), torch.ones((tokens, 1), device="cuda")], 1)
    ind, sc = ind.view(1, tokens, topk + 1).contiguous(), sc.view(1, tokens, topk + 1).contiguous()
    x = torch.randn((1, tokens, hidden), device="cuda", dtype=torch.float16, generator=g)
    y = torch.empty_like(x)
    ms = _graph_ms(torch, lambda: Q.swiglu(*banks, x, ind, sc, out=y), reps)
    distinct = int(torch.unique(ind).numel())
    per_expert = 3 * (hidden * inter * 3 // 8 + 2 * hidden + 2 * inter)
    nbytes = distinct * per_expert + 2 * 2 * tokens * hidden
    gbs = nbytes / (ms * 1e-3) / 1e9
    del banks
    return {"workload": "config 4: routed SwiGLU, 256 + 1 shared experts, 4096 <-> 2048 @ 3 bpw, 32 tokens, top-8",
            "value": round(gbs, 1), "unit": "GB/s", "ms": round(ms, 4), "distinct_experts": distinct,
            "bytes_per_call": nbytes, "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4),
            "l2": "no flush: a call streams %.2f GB of distinct experts (> 126 MB L2)" % (nbytes / 1e9)}


def measure_moe_prefill(Q, E, torch, peaks: dict, tokens: int = 2048, reps: int = 5) -> dict:
    """Config 4's banks (256 routed + 1 shared expert, 4096 <-> 2048 @ 3 bpw) at a prompt of `tokens` rows, top-8 of a
    softmax over N(0, 1) router logits plus the shared expert's slot: one swiglu call on the tensor-core prefill path
    (exl3_moe_prefill_reserve), replayed in a CUDA graph; TFLOP/s of the routed and shared experts' three GEMMs."""
    experts, hidden, inter, topk = 256, 4096, 2048, 8
    banks = []
    for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden))):
        tr, suh, svh = E.random_linear(a, b, 48, seed=3 + i, groups=experts + 1)
        banks.append(Q.weight_from_tensors(tr, suh, svh))
    g = torch.Generator(device="cuda").manual_seed(4)
    logits = torch.randn((tokens, experts), device="cuda", generator=g)
    sc, ind = torch.topk(torch.softmax(logits, -1), topk, -1)
    ind = torch.cat([ind.to(torch.int32), torch.full((tokens, 1), experts, dtype=torch.int32, device="cuda")], 1)
    sc = torch.cat([sc.float(), torch.ones((tokens, 1), device="cuda")], 1)
    ind, sc = ind.view(1, tokens, topk + 1).contiguous(), sc.view(1, tokens, topk + 1).contiguous()
    x = torch.randn((1, tokens, hidden), device="cuda", dtype=torch.bfloat16, generator=g)
    y = torch.empty_like(x)
    ws = Q.moe_prefill_reserve(experts + 1, hidden, inter, tokens * (topk + 1))
    try:
        ms = _graph_ms(torch, lambda: Q.swiglu(*banks, x, ind, sc, out=y), reps, inner=1)
    finally:
        Q.moe_prefill_reserve(experts + 1, hidden, inter, 0)
    flops = 2.0 * 3 * hidden * inter * tokens * (topk + 1)
    tf = flops / (ms * 1e-3) / 1e12
    del banks
    return {"workload": f"config 4 banks at a {tokens}-token prompt: 256 routed + 1 shared experts, 4096 <-> 2048 "
                        "@ 3 bpw, top-8 + the shared slot, bf16",
            "value": round(tf, 1), "unit": "TFLOP/s", "ms": round(ms, 4), "flops_per_call": flops,
            "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4), "workspace_bytes": ws,
            "path": "slots sorted into per-expert 128-row blocks; grouped tcgen05 GEMMs for gate, up and down with "
                    "each block's expert W_hat^T decoded inside the GEMM (no operand image); SwiGLU between "
                    "(exl3_moe_prefill.cu, exl3_gemm_fused.cu)"}


def measure_moe_ep(Q, E, torch, dist, rank: int, world: int, device, peaks: dict, steps: int = 20) -> dict:
    """Config 4 expert-parallel over the ranks (plugins_b200/sharding.py): rank r holds experts [32 r', ...) of the 256
    (256/world each) plus the shared expert, brings 32/world of the 32 tokens, and a step is dispatch, exchange, its
    experts' SwiGLU, exchange back and the combine -- captured in one CUDA graph and timed as the max over ranks, once
    with the peer-memory exchange (exl3_epx_*, the headline) and once with NCCL all-to-alls.  Bytes are the distinct
    routed experts each rank streams plus its shared expert, summed over the ranks."""
    from plugins_b200 import sharding as S
    experts, hidden, inter, topk, total = 256, 4096, 2048, 8, 32
    tokens = total // world
    e0, e1 = S.expert_range(experts, rank, world)
    local, cols = [], []
    for i, (a, b) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden))):
        tr, suh, svh = E.random_linear(a, b, 48, seed=3 + i, groups=experts, device=device)
        st, ssu, ssv = E.random_linear(a, b, 48, seed=13 + i, groups=1, device=device)
        # expert parallel: this rank's experts, then the shared expert (its slots stay on the token's rank)
        local.append(Q.weight_from_tensors(torch.cat([tr[e0:e1], st]), torch.cat([suh[e0:e1], ssu]),
                                           torch.cat([svh[e0:e1], ssv])))
        # column parallel: this rank's output columns of every expert, the shared one last
        c0, c1 = rank * b // world, (rank + 1) * b // world
        cols.append(Q.weight_from_tensors(*S.expert_columns(torch.cat([tr, st]), torch.cat([suh, ssu]),
                                                            torch.cat([svh, ssv]), c0, c1)))
        del tr, suh, svh
    g = torch.Generator(device=device).manual_seed(4)
    logits = torch.randn((total, experts), device=device, generator=g)
    sc, ind = torch.topk(torch.softmax(logits, -1), topk, -1)
    x_all = torch.randn((total, hidden), device=device, generator=g).half()
    sl = slice(rank * tokens, (rank + 1) * tokens)
    # the slot lists with the shared expert as the last column (id 256, score 1)
    ind = torch.cat([ind[sl].to(torch.int32), torch.full((tokens, 1), experts, dtype=torch.int32, device=device)], 1)
    sc = torch.cat([sc[sl].float(), torch.ones((tokens, 1), device=device)], 1)
    x, ind, sc = x_all[sl].contiguous(), ind.contiguous(), sc.contiguous()
    per_expert = 3 * (hidden * inter * 3 // 8 + 2 * hidden + 2 * inter)
    all_ind = torch.unique(torch.topk(torch.softmax(logits, -1), topk, -1)[1])
    mine = int(((all_ind >= e0) & (all_ind < e1)).sum().item())

    def timed(exchange, trace: bool = False):
        # trace: a second exchange built with EXL3_TRACE=1 records the kernels' %globaltimer stamps per step
        if trace:
            os.environ["EXL3_TRACE"] = "1"
        if exchange == "columns":
            ep = S.ColumnParallelExperts(*cols, experts=experts, tokens=tokens, topk=topk, hidden=hidden, inter=inter,
                                         rank=rank, world=world, device=device, shared=True)
        else:
            ep = S.ExpertParallelSwiglu(*local, experts=experts, tokens=tokens, topk=topk, hidden=hidden, rank=rank,
                                        world=world, device=device, shared=True, exchange=exchange)
        os.environ.pop("EXL3_TRACE", None)
        y = torch.empty_like(x)
        st = torch.cuda.Stream(device=device)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for _ in range(3):
                ep.forward(x, ind, sc, out=y)
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            ep.forward(x, ind, sc, out=y)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
        t = torch.tensor([ev0.elapsed_time(ev1) / steps], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        graph.reset()
        closer = ep if exchange == "columns" else ep.peer
        stamps = closer.trace() if trace else None
        if closer is not None:
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()  # every rank's kernels are done before any exchange region is unmapped
            closer.close()
        return (float(t[0]), stamps) if trace else float(t[0])

    b = torch.tensor([float((mine + 1) * per_expert)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
    nbytes = float(b[0])
    ms = timed("peer")
    ms_nccl = timed("nccl")
    ms_cols = timed("columns")
    phases = phases_cols = None
    if world > 1:
        _, st_peer = timed("peer", trace=True)
        _, st_cols = timed("columns", trace=True)
        phases = phase_table(dist, world, st_peer, EPX_PHASES)
        phases_cols = phase_table(dist, world, st_cols, CPX_PHASES)
    cp_bytes = (int(all_ind.numel()) + 1) * per_expert  # every distinct expert once, the shared one once
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "config 4 expert-parallel: 256 routed (256/N per GPU) + 1 shared expert, 4096 <-> 2048 "
                        "@ 3 bpw, 32 tokens (32/N per GPU), top-8; dispatch and combine over NVLink peer memory",
            "n_gpus": world, "ms_per_step": round(ms, 4), "tokens_per_s": round(total / (ms * 1e-3), 1),
            "value": round(gbs, 1), "unit": "GB/s (whole box)", "bytes_per_step": int(nbytes),
            "frac_of_hbm_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4),
            "nccl_all_to_all": {"ms_per_step": round(ms_nccl, 4),
                                "value": round(nbytes / (ms_nccl * 1e-3) / 1e9, 1)},
            "column_parallel": {"ms_per_step": round(ms_cols, 4), "tokens_per_s": round(total / (ms_cols * 1e-3), 1),
                                "value": round(cp_bytes / (ms_cols * 1e-3) / 1e9, 1), "unit": "GB/s (whole box)",
                                "bytes_per_step": int(cp_bytes),
                                "note": "every rank holds 1/N of every expert's columns and streams 1/N of the "
                                        "distinct experts' bytes; tokens, the down input and the outputs move over "
                                        "NVLink peer memory inside one call (exl3_swiglu_cp)"},
            **({"phases_us": phases, "column_parallel_phases_us": phases_cols} if phases else {})}


# the stamps an exchange's kernels record per step (include/exl3_b200.h, exchange timelines) and the phases between
# them: (name, from stamp, to stamp); "next" is the stretch from a step's last stamp to the next step's first
EPX_PHASES = [("dispatch_copies", 0, 1), ("wait_peers_dispatch", 1, 2), ("receive_copy", 2, 3), ("swiglu", 3, 4),
              ("return_copies", 4, 5), ("wait_peers_return", 5, 6), ("combine", 6, 7), ("step", 0, 7)]
CPX_PHASES = [("token_copies", 0, 1), ("wait_peers_tokens", 1, 2), ("route_prep_gate_up", 2, 3),
              ("wait_peers_gate_up", 3, 4), ("down_combine", 4, 5), ("out_copies_wait_peers", 5, 6),
              ("copy_out", 6, 7), ("step", 0, 7)]
TP_PHASES = [("gemvs", 0, 1), ("wait_peers", 1, 2), ("gather_copy", 2, 3), ("step", 0, 3)]


def phase_table(dist, world: int, steps: list, phases: list) -> dict:
    """Per phase, the median over the traced steps (us) on each rank, then the max and the mean over the ranks; the
    phase whose max is largest bounds the step, a wait shows how long a rank idled for its slowest peer."""
    mine = {}
    for name, a, b in phases:
        d = [(st[b] - st[a]) / 1e3 for st in steps if st[a] and st[b] and st[b] >= st[a]]
        mine[name] = statistics.median(d) if d else None
    every = [None] * world
    dist.all_gather_object(every, mine)
    out = {}
    for name, _, _ in phases:
        vals = [r[name] for r in every if r[name] is not None]
        if vals:
            out[name] = {"max": round(max(vals), 2), "mean": round(sum(vals) / len(vals), 2),
                         "rank_of_max": max(range(len(every)), key=lambda i: every[i][name] or -1)}
    return out


def measure_c5(Q, E, torch, peaks: dict, reps: int = 5) -> dict:
    """Config 5: K = 16384, N = 53248 at 2, 3, 4 and 5 bpw (random trellis, seed 5), batch-1 f16, one GPU."""
    in_f, out_f = 16384, 53248
    res = {}
    for bits in (2, 3, 4, 5):
        tr, suh, svh = E.random_linear(in_f, out_f, 16 * bits, seed=5)
        w = Q.weight_from_tensors(tr, suh, svh)
        x = torch.randn((1, in_f), device="cuda", dtype=torch.float16)
        y = torch.empty((1, out_f), device="cuda", dtype=torch.float16)
        ms = _graph_ms(torch, lambda: Q.matmul(w, x, out=y), reps)
        nbytes = linear_bytes(in_f, out_f, bits, 1)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[f"{bits}bpw"] = {"ms": round(ms, 4), "value": round(gbs, 1), "unit": "GB/s",
                             "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "bytes": nbytes}
        del w, tr
    return {"workload": "config 5: 16384 x 53248 decode GEMV, batch 1", **res}


def measure_c5_tp(Q, E, torch, dist, rank: int, world: int, device, peaks: dict, reps: int = 5) -> dict:
    """Config 5 column-parallel (N > 1): rank r keeps its 128-aligned range of the 53248 output columns
    (sharding.column_range) of the same seeded layer, and its decode GEMV stores those columns into every rank's
    exchange over NVLink (exl3_matmul_tp); a call is begin, the GEMV and the gather of the whole y [1, 53248] on every
    rank, replayed as a CUDA graph and timed as the max over ranks.  Bytes are the whole layer's (every rank streams
    its share once)."""
    from plugins_b200 import sharding as S
    in_f, out_f = 16384, 53248
    c0, c1 = S.column_range(out_f, rank, world)
    res = {}
    for bits in (2, 3, 4, 5):
        tr, suh, svh = E.random_linear(in_f, out_f, 16 * bits, seed=5, device=device)
        w = Q.weight_from_tensors(tr[:, c0 // 16:c1 // 16].contiguous(), suh, svh[c0:c1].contiguous())
        del tr, svh
        g = torch.Generator(device=device).manual_seed(6)
        x = torch.randn((1, in_f), device=device, generator=g).half()
        y = torch.empty(out_f, dtype=torch.float16, device=device)
        ex = S.TpExchange(rank, world, slots=1, slot_bytes=out_f * 2, max_cb=out_f // 128)

        def call():
            ex.begin()
            ex.matmul(w, x, 0, [c0], [out_f])
            ex.gather(0, 1, y)

        dist.barrier()
        ms = _graph_ms(torch, call, reps)
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        torch.cuda.synchronize()
        dist.barrier()
        ex.close()
        nbytes = linear_bytes(in_f, out_f, bits, 1)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[f"{bits}bpw"] = {"ms": round(ms, 4), "value": round(gbs, 1), "unit": "GB/s (whole box)",
                             "per_gpu": round(gbs / world, 1), "frac_of_hbm_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4),
                             "bytes": nbytes}
        del w
    return {"workload": f"config 5 column-parallel over {world} GPUs: 16384 x 53248 decode GEMV, batch 1, each rank "
                        "1/N of the 128-column blocks, y gathered inside the GEMV over NVLink", **res}


# ------------------------------------------------------------------ clocks during the timed region

class ClockSampler:
    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._idx = device_index
        self._t = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self._idx)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            names = {
                "hw_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwSlowdown", 0x8),
                "hw_thermal_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwThermalSlowdown", 0x40),
                "sw_thermal_slowdown": getattr(nv, "nvmlClocksThrottleReasonSwThermalSlowdown", 0x20),
                "sw_power_cap": getattr(nv, "nvmlClocksThrottleReasonSwPowerCap", 0x4),
                "hw_power_brake_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwPowerBrakeSlowdown", 0x80),
            }

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h) if hasattr(
                            nv, "nvmlDeviceGetCurrentClocksEventReasons") else nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                        for k, bit in names.items():
                            if r & bit:
                                self.reasons.add(k)
                    except Exception:
                        pass
                    self._stop.wait(0.02)

            self._t = threading.Thread(target=run, daemon=True)
            self._t.start()
        except Exception:
            self._t = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=1)

    def summary(self) -> dict:
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ the reference arm: the CPU port of project()

def cpu_sample(rows: int, budget_s: float, threads: int, seed: int = 1):
    """Times the oracle's restatement of the reference's scalar project() (expert_exl3.zig:546-566) over the layer's
    linears (layer 0 of the stack, random trellis of the same shapes), `rows` rows each, for about `budget_s`."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    lin = []
    for name, i, o, b in LINEARS:
        tr = rng.integers(0, 65536, (i // 16, o // 16, 16 * b), dtype=np.uint16)
        suh = rng.standard_normal(i).astype(np.float16).view(np.uint16)
        svh = rng.standard_normal(o).astype(np.float16).view(np.uint16)
        x = rng.standard_normal((rows, i)).astype(np.float32)
        lin.append((name, i, o, b, tr, suh, svh, x))
    done_bytes, t0, reps = 0, time.perf_counter(), 0
    while True:
        for name, i, o, b, tr, suh, svh, x in lin:
            for r in range(rows):
                O.project(x[r], tr, suh, svh, i, o, 16 * b, threads=threads)
            done_bytes += linear_bytes(i, o, b, rows)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return done_bytes / el / 1e9, el, reps


def zig_probe() -> str:
    """`zig version` on this host: the reference's own build (Zig ReleaseFast) needs it."""
    import shutil
    import subprocess
    z = shutil.which("zig")
    if z is None:
        return "absent (no zig on PATH): the C restatement of project() is timed instead"
    try:
        return "zig " + subprocess.run([z, "version"], capture_output=True, text=True, timeout=20).stdout.strip()
    except Exception as e:  # noqa: BLE001
        return f"zig present but `zig version` failed: {e}"


def host_cpu() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip() + f", {os.cpu_count()} threads"
    except OSError:
        pass
    return f"{os.cpu_count()} threads"


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sample(args.batch, 0.0, threads)
    times, gbs = [], []
    for _ in range(args.steps):
        g, el, reps = cpu_sample(args.batch, 0.0, threads)
        times.append(el)
        gbs.append(g)
    total_bytes = args.steps * sum(linear_bytes(i, o, b, args.batch) for _, i, o, b in LINEARS)
    value = total_bytes / sum(times) / 1e9
    layer_s = sum(times) / args.steps
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * layer_s, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u16 trellis -> f16/f32",
        "data": "synthetic (random trellis of the stack's shapes)",
        "config": {"workload": WORKLOAD, "batch": args.batch, "step": "one layer's 7 linears (bounded sample)"},
        "decode_tok_s": round(args.batch / (layer_s * LAYERS), 4),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"layer 0's 7 linears at batch {args.batch} per step (1/36 of a decode step); "
                                   "C restatement of expert_exl3.zig project(), OpenMP over output tiles",
                         "host_cpu": host_cpu(), "zig": zig_probe()},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ the B200 arm

def build_stack(Q, E, torch, rank: int, world: int, device):
    """Encodes every linear (seeded, identical on all ranks), keeps this rank's column shard, stacks launch groups."""
    layers = []
    for l in range(LAYERS):
        parts = {}
        for idx, (name, i, o, b) in enumerate(LINEARS):
            seed = 1 + l * len(LINEARS) + idx
            g = torch.Generator(device=device)
            g.manual_seed(seed)
            w = torch.randn((o, i), generator=g, device=device) * 0.02
            tr, suh, svh = E.quantize(w, b, seed)
            del w
            if world > 1:
                cols = o // world
                tr = tr[:, rank * cols // 16:(rank + 1) * cols // 16, :].contiguous()
                svh = svh[rank * cols:(rank + 1) * cols].contiguous()
            parts[name] = Q.weight_from_tensors(tr, suh, svh)
        groups = {}
        for gname, members in GROUPS:
            groups[gname] = Q.stack([parts[m] for m in members]) if len(members) > 1 else parts[members[0]]
        layers.append(groups)
    torch.cuda.synchronize()
    return layers


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline sampling (rank 0, N=1)")
    ap.add_argument("--no-batch8", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip configs 3-5 (prefill, MoE, large layer)")
    ap.add_argument("--tp-nccl", action="store_true",
                    help="N > 1: gather the column shards with NCCL all-gathers instead of inside the GEMV")
    args = ap.parse_args()
    if args.impl == "reference":
        if args.steps > 20:
            args.steps = 20  # each reference step is a full layer on the CPU; keep the run within minutes
        run_reference(args)
        return

    import torch
    import torch.distributed as dist
    from plugins_b200 import quant as Q
    from plugins_b200 import encoder as E

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    layers = build_stack(Q, E, torch, rank, world, device)

    def make_io(rows: int):
        g = torch.Generator(device=device)
        g.manual_seed(1234 + rows)
        ins, outs = [], []
        for l in range(LAYERS):
            x = torch.randn((rows, HIDDEN), generator=g, device=device).half()
            a = torch.randn((rows, HIDDEN), generator=g, device=device).half()
            m = torch.randn((rows, INTER), generator=g, device=device).half()
            ins.append({"qkv": x, "o": a, "gate_up": x, "down": m})
            outs.append({k: torch.empty((rows, layers[l][k].out_features), dtype=torch.float16, device=device)
                         for k, _ in GROUPS})
        return ins, outs

    def flat_views(tensors):
        total = sum(t.numel() for t in tensors)
        buf = torch.empty(total, dtype=torch.float16, device=device)
        views, off = [], 0
        for t in tensors:
            v = buf[off:off + t.numel()].view(t.shape)
            v.copy_(t)
            views.append(v)
            off += t.numel()
        return buf, views

    fused = world > 1 and not args.tp_nccl
    seg = {"qkv": ([rank * HEADS_Q // world, rank * KV // world, rank * KV // world], [HEADS_Q, KV, KV]),
           "o": ([rank * HIDDEN // world], [HIDDEN]),
           "gate_up": ([rank * INTER // world] * 2, [INTER, INTER]),
           "down": ([rank * HIDDEN // world], [HIDDEN])}

    def run_config(rows: int, steps: int, warmup: int):
        ins, outs = make_io(rows)
        ex = None
        from plugins_b200 import sharding as S
        if fused:
            # every launch writes its columns into a slot of every rank's exchange; one gather per step
            ex = S.TpExchange(rank, world, slots=LAYERS * len(GROUPS), slot_bytes=rows * 2 * INTER * 2,
                              max_cb=2 * INTER // 128)
            tp_out = torch.empty(LAYERS * len(GROUPS) * ex.slot_bytes, dtype=torch.uint8, device=device)
        # inputs live in one contiguous device buffer (one H2D per step); outputs likewise (one D2H)
        uniq_in = []
        for l in range(LAYERS):
            uniq_in += [ins[l]["qkv"], ins[l]["o"], ins[l]["down"]]
        in_buf, in_views = flat_views(uniq_in)
        for l in range(LAYERS):
            x, a, m = in_views[3 * l: 3 * l + 3]
            ins[l] = {"qkv": x, "o": a, "gate_up": x, "down": m}
        gathered = []
        if world > 1 and not fused:
            for l in range(LAYERS):
                gathered.append({k: torch.empty((world,) + tuple(outs[l][k].shape), dtype=torch.float16,
                                                device=device) for k, _ in GROUPS})
        if fused:
            out_buf = tp_out
        else:
            out_list = [outs[l][k] for l in range(LAYERS) for k, _ in GROUPS] if world == 1 else \
                [gathered[l][k] for l in range(LAYERS) for k, _ in GROUPS]
            out_buf, out_views = flat_views(out_list)
            j = 0
            for l in range(LAYERS):
                for k, _ in GROUPS:
                    if world == 1:
                        outs[l][k] = out_views[j]
                    else:
                        gathered[l][k] = out_views[j]
                    j += 1

        def step():
            if fused:
                ex.begin()
                for l in range(LAYERS):
                    for j, (k, _) in enumerate(GROUPS):
                        ex.matmul(layers[l][k], ins[l][k], l * len(GROUPS) + j, *seg[k])
                ex.gather(0, LAYERS * len(GROUPS), tp_out)
                return
            for l in range(LAYERS):
                for k, _ in GROUPS:
                    Q.matmul(layers[l][k], ins[l][k], out=outs[l][k])
                    if world > 1:
                        dist.all_gather_into_tensor(gathered[l][k], outs[l][k])

        s = torch.cuda.Stream(device=device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
        torch.cuda.synchronize()
        # the decode-GEMV kernels of each launch group (+ the step begin and the gather when the exchange is fused)
        lin = {n: (i, o) for n, i, o, _ in LINEARS}
        group_dims = {g: (lin[names[0]][0], sum(lin[n][1] for n in names) // world) for g, names in GROUPS}
        launches_per_step = (LAYERS * sum(gemv_kernels(i, o, fused, rows) for i, o in group_dims.values())
                             + (2 if fused else 0))

        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        with ClockSampler(local) as clk:
            evs[0].record(st)
            for i in range(steps):
                graph.replay()
                evs[i + 1].record(st)
            torch.cuda.synchronize()
        ms = evs[0].elapsed_time(evs[steps]) / steps
        per_step = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(steps))
        ms_med, ms_fast = statistics.median(per_step), per_step[0]
        if world > 1:
            t = torch.tensor([ms_med, ms_fast], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_med, ms_fast = float(t[0].item()), float(t[1].item())
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())

        # e2e: pinned host inputs -> device, the step, device -> pinned host outputs
        h_in = torch.empty(in_buf.shape, dtype=in_buf.dtype, pin_memory=True)
        h_in.copy_(in_buf)
        h_out = torch.empty(out_buf.shape, dtype=out_buf.dtype, pin_memory=True)
        for _ in range(3):
            in_buf.copy_(h_in, non_blocking=True)
            graph.replay()
            h_out.copy_(out_buf, non_blocking=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(st)
        for _ in range(steps):
            in_buf.copy_(h_in, non_blocking=True)
            graph.replay()
            h_out.copy_(out_buf, non_blocking=True)
        e3.record(st)
        torch.cuda.synchronize()
        ms_e2e = e2.elapsed_time(e3) / steps
        if world > 1:
            t = torch.tensor([ms_e2e], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e2e = float(t.item())

        # the dominant launch (gate|up, 37.7 MB at 3 bpw) and the 4-bpw q|k|v: the group's 36 launches (one per layer,
        # distinct weights) captured back to back in one CUDA graph and timed with events on its stream, so the
        # average is the kernels' own duration in a dense sequence, without host launch gaps
        def time_group(k: str) -> float:
            gs = torch.cuda.Stream(device=device)
            gs.wait_stream(torch.cuda.current_stream())
            gg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gg, stream=gs):
                for l in range(LAYERS):
                    Q.matmul(layers[l][k], ins[l][k], out=outs[l][k])
            for _ in range(3):
                gg.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 10
            a.record(st)
            for _ in range(reps):
                gg.replay()
            b.record(st)
            torch.cuda.synchronize()
            gg.reset()
            return a.elapsed_time(b) / (reps * LAYERS)

        dom_ms = time_group("gate_up")
        qkv_ms = time_group("qkv")
        graph.reset()
        phases = None
        if ex is not None:
            # the step's phases: the same step on a second exchange built with EXL3_TRACE=1 (its kernels stamp
            # %globaltimer per step), replayed apart from the timed runs
            torch.cuda.synchronize()
            timed_ex = ex
            os.environ["EXL3_TRACE"] = "1"
            ex = S.TpExchange(rank, world, slots=LAYERS * len(GROUPS), slot_bytes=timed_ex.slot_bytes,
                              max_cb=2 * INTER // 128)
            os.environ.pop("EXL3_TRACE", None)
            with torch.cuda.stream(s):
                for _ in range(3):
                    step()
            torch.cuda.synchronize()
            tg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(tg, stream=s):
                step()
            for _ in range(20):
                tg.replay()
            torch.cuda.synchronize()
            phases = phase_table(dist, world, ex.trace(), TP_PHASES)
            tg.reset()
            dist.barrier()  # no rank unmaps its exchange while another still writes into it
            ex.close()
            ex = timed_ex
        if ex is not None:
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()  # no rank unmaps its exchange while another still writes into it
            ex.close()
        return {"ms": ms, "ms_med": ms_med, "ms_fast": ms_fast, "ms_e2e": ms_e2e, "clk": clk.summary(),
                "launches": launches_per_step * steps,
                "h2d": in_buf.numel() * in_buf.element_size(), "d2h": out_buf.numel() * out_buf.element_size(),
                "dom_ms": dom_ms, "qkv_ms": qkv_ms, "phases": phases}

    peaks = load_peaks()
    r1 = run_config(args.batch, args.steps, args.warmup)
    moe_ep = None if args.no_extras else measure_moe_ep(Q, E, torch, dist, rank, world, device, peaks)
    c5_tp = None if (args.no_extras or world == 1) else measure_c5_tp(Q, E, torch, dist, rank, world, device, peaks)
    r8 = None if (args.no_batch8 or args.batch == 8) else run_config(8, args.steps, args.warmup)
    total = step_bytes(args.batch)
    value = total / (r1["ms"] * 1e-3) / 1e9
    e2e = total / (r1["ms_e2e"] * 1e-3) / 1e9
    # dominant kernel: the stacked gate|up launch of this rank (its shard's algorithmic bytes)
    gu_bytes = sum(linear_bytes(HIDDEN, INTER // world, 3, args.batch) for _ in range(2))
    achieved = gu_bytes / (r1["dom_ms"] * 1e-3) / 1e9
    qkv_bytes = sum(linear_bytes(HIDDEN, o // world, 4, args.batch) for o in (HEADS_Q, KV, KV))

    cpu = None
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        threads = os.cpu_count() or 1
        gbs, el, reps = cpu_sample(args.batch, args.cpu_budget, threads)
        gbs1, el1, reps1 = cpu_sample(args.batch, args.cpu_budget, 1)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"layer 0's 7 linears at batch {args.batch}, {reps} pass(es) in {el:.1f} s; C restatement "
                         "of expert_exl3.zig project() (scalar decode+GEMV), OpenMP over output tiles",
               "single_core": {"value": round(gbs1, 4), "unit": "GB/s", "cores": 1,
                               "sample": f"the same linears, {reps1} pass(es) in {el1:.1f} s on one thread (the "
                                         "reference's project() is single-threaded)"},
               "host_cpu": host_cpu(), "zig": zig_probe()}
    if rank == 0:
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
                tj = json.load(f)
            traffic = tj.get("gate_up_k3_batch%d" % args.batch)
        except Exception:
            pass
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(r1["ms"], 4),
            "ms_per_step_median": round(r1["ms_med"], 4), "ms_per_step_fastest": round(r1["ms_fast"], 4),
            "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u16 trellis -> f16 (f32 accumulate)",
            "data": "synthetic: random-init N(0,0.02) weights (seeded) encoded to EXL3 mul1 by the library; "
                    "N(0,1) f16 activations",
            "config": {"workload": WORKLOAD, "batch": args.batch, "layers": LAYERS,
                       "parallelism": ("single GPU" if world == 1 else
                                       f"tp{world} column-parallel, NCCL all-gather per launch" if args.tp_nccl else
                                       f"tp{world} column-parallel, all-gather inside the GEMV (NVLink peer stores)"),
                       "bytes_per_step": total,
                       "l2": "no flush: a step streams %.2f GB of distinct weights, >> 126 MB L2" % (total / 1e9)},
            "decode_tok_s": round(args.batch / (r1["ms"] * 1e-3), 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                         "kernel": ("gate|up decode GEMV (4096 -> 2x12288 @ 3 bpw): "
                                    + {0: "gemv5_kernel (cluster split)",
                                       1: "gemv6_kernel (persistent, balanced; input rotated in-CTA)",
                                       2: "gemv6_prep_kernel + gemv6_kernel (persistent, balanced)"}[
                                        gemv6_mode(HIDDEN, 2 * INTER // world, world > 1 and not args.tp_nccl,
                                                   args.batch)]),
                         "bytes_per_launch": gu_bytes, "ms_per_launch": round(r1["dom_ms"], 5),
                         "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)"},
            "roofline_4bpw_qkv": {"achieved": round(qkv_bytes / (r1["qkv_ms"] * 1e-3) / 1e9, 1),
                                  "frac": round(qkv_bytes / (r1["qkv_ms"] * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                                  "ms_per_launch": round(r1["qkv_ms"], 5), "bytes_per_launch": qkv_bytes},
            "step_frac_of_hbm": round(value / peaks["hbm_gbs"], 4),
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": r1["h2d"],
                    "d2h_bytes_per_step": r1["d2h"], "ms_per_step": round(r1["ms_e2e"], 4),
                    "decode_tok_s": round(args.batch / (r1["ms_e2e"] * 1e-3), 2)},
            "gpu_launches": r1["launches"],
            "clocks": r1["clk"],
            "cpu_baseline": cpu,
        }
        if moe_ep is not None:
            line["moe_ep"] = moe_ep
        if c5_tp is not None:
            line["large_layer_tp"] = c5_tp
        if r1.get("phases"):
            line["tp_phases_us"] = r1["phases"]
        if world == 1 and not args.no_extras:
            line["north_star"] = measure_layer(Q, E, torch, peaks, 4096, 12288, 4, 0,
                                               "north-star layer: 4096 x 12288 @ 4 bpw decode GEMV, batch 1 "
                                               "(W N(0,0.02) seed 0, 36 distinct copies)")
            line["config1"] = measure_layer(Q, E, torch, peaks, 4096, 4096, 4, 0,
                                            "config 1: 4096 x 4096 @ 4 bpw decode GEMV, batch 1 "
                                            "(W N(0,0.02) seed 0, 36 distinct copies)")
            line["prefill"] = measure_prefill(Q, E, torch, peaks)
            line["moe"] = measure_moe(Q, E, torch, peaks)
            line["moe_prefill"] = measure_moe_prefill(Q, E, torch, peaks)
            line["large_layer"] = measure_c5(Q, E, torch, peaks)
        if r8 is not None:
            v8 = step_bytes(8) / (r8["ms"] * 1e-3) / 1e9
            line["batch8"] = {"value": round(v8, 2), "unit": "GB/s", "ms_per_step": round(r8["ms"], 4),
                              "decode_tok_s": round(8 / (r8["ms"] * 1e-3), 2),
                              "e2e_value": round(step_bytes(8) / (r8["ms_e2e"] * 1e-3) / 1e9, 2)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
