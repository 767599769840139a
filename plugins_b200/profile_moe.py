"""GPU time of one routed-expert call (exl3_swiglu), replayed in a CUDA graph; also the capture target for kernel
profiles of the grouped expert GEMV.

    python -m plugins_b200.profile_moe EXPERTS TOKENS TOPK [--hidden 4096] [--inter 2048] [--n 48] [--ep-share WORLD]
                                   [--prefill]

Random-trellis banks (seeded) of EXPERTS experts, TOKENS rows routed top-TOPK by softmax of seeded logits.  With
--ep-share WORLD the call is instead one rank's share of an expert-parallel step over WORLD ranks: the receive layout
of plugins_b200/sharding.py ([WORLD][C + 1] rows, one slot each, most of them empty) over a bank of EXPERTS / WORLD
routed experts plus a shared one, TOKENS being the tokens of the whole step.  Prints microseconds per call, the
distinct experts read and the bank bytes they hold per second.  A few eager calls run before the graph, so
`ncu -k regex:moe_ -s 5` skips the first call's five launches.
"""
from __future__ import annotations

import argparse

import torch

from . import encoder as E
from . import quant as Q


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("experts", type=int)
    ap.add_argument("tokens", type=int)
    ap.add_argument("topk", type=int)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--n", type=int, default=48, help="halfwords per tile (16 x bits per weight)")
    ap.add_argument("--ep-share", type=int, default=0, metavar="WORLD")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--prefill", action="store_true",
                    help="reserve the prefill workspace (calls of 1024+ slots then run on the tensor cores)")
    a = ap.parse_args()
    h, m, n = a.hidden, a.inter, a.n
    g = torch.Generator(device="cuda").manual_seed(4)
    logits = torch.randn((a.tokens, a.experts), device="cuda", generator=g)
    _, top = torch.topk(torch.softmax(logits, -1), a.topk, -1)
    if a.ep_share:
        world = a.ep_share
        per = a.experts // world
        bank_e = per + 1  # this rank's experts, then the shared one
        cap = (a.tokens // world) * (min(a.topk, per) + 1)
        rows = world * (cap + 1)
        inds = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        fill = [0] * world  # rank 0's share: the slots every source rank routes to experts [0, per)
        for t in range(a.tokens):
            src = t // (a.tokens // world)
            for e in top[t].tolist():
                if e < per:
                    inds[src * (cap + 1) + fill[src]] = e
                    fill[src] += 1
            if src == 0:  # the shared expert's slot stays on the token's own rank
                inds[fill[0]] = per
                fill[0] += 1
        x = torch.randn((1, rows, h), device="cuda", dtype=torch.float16)
        ii = inds.view(1, rows, 1)
        sc = torch.ones((1, rows, 1), device="cuda")
        y = torch.empty((1, rows, h), device="cuda", dtype=torch.float32)
        distinct = int(torch.unique(inds[inds >= 0]).numel())
    else:
        bank_e = a.experts
        x = torch.randn((1, a.tokens, h), device="cuda", dtype=torch.float16)
        ii = top.to(torch.int32).view(1, a.tokens, a.topk).contiguous()
        sc = torch.rand((1, a.tokens, a.topk), device="cuda", generator=g)
        y = torch.empty_like(x)
        distinct = int(torch.unique(ii).numel())
    banks = [Q.weight_from_tensors(*E.random_linear(i, o, n, seed=7 + k, groups=bank_e))
             for k, (i, o) in enumerate(((h, m), (h, m), (m, h)))]
    if a.prefill:
        Q.moe_prefill_reserve(bank_e, h, m, x.shape[1] * ii.shape[2])
    for _ in range(3):
        Q.swiglu(*banks, x, ii, sc, out=y)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for _ in range(4):
            Q.swiglu(*banks, x, ii, sc, out=y)
    for _ in range(10):
        graph.replay()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(a.reps):
        graph.replay()
    ev[1].record()
    torch.cuda.synchronize()
    us = ev[0].elapsed_time(ev[1]) * 1000 / (4 * a.reps)
    nbytes = distinct * 3 * h * m * n // 128
    flops = 2.0 * 3 * h * m * int((ii >= 0).sum().item())
    print(f"{'ep-share ' + str(a.ep_share) if a.ep_share else 'call'} experts {a.experts} tokens {a.tokens} "
          f"top-{a.topk}: {us:.1f} us, {distinct} distinct experts, {nbytes / us / 1e3:.1f} GB/s, "
          f"{flops / us / 1e6:.1f} TFLOP/s", flush=True)


if __name__ == "__main__":
    main()
