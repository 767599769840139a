"""Per-launch GPU time of one decode-GEMV shape, replayed in a CUDA graph (no host launch cost in the number).

    python -m plugins_b200.profile_gemv IN OUT N [ROWS] [--dp4a] [--reps R]

Builds `reps` distinct random-trellis weights of the shape (so consecutive launches stream distinct bytes, and more
than L2 holds when the shape is large), captures `loops x reps` launches in one graph and reports microseconds per
launch and trellis GB/s.  Under `ncu -k regex:gemv_kernel` it is also the capture target for kernel profiles.
"""
from __future__ import annotations

import argparse
import time

import torch

from . import encoder as E
from . import quant as Q


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("in_features", type=int)
    ap.add_argument("out_features", type=int)
    ap.add_argument("n", type=int, help="halfwords per tile (16 x bits per weight)")
    ap.add_argument("rows", type=int, nargs="?", default=1)
    ap.add_argument("--dp4a", action="store_true", help="byte sums on dp4a instead of the tensor pipe")
    ap.add_argument("--reps", type=int, default=0, help="distinct weights (0: enough to exceed 300 MB, 2..16)")
    ap.add_argument("--loops", type=int, default=8)
    a = ap.parse_args()
    nbytes = a.in_features * a.out_features * a.n // 128
    reps = a.reps or max(2, min(16, (300 << 20) // nbytes))
    ws = []
    for i in range(reps):
        tr, suh, svh = E.random_linear(a.in_features, a.out_features, a.n, seed=i)
        ws.append(Q.weight_from_tensors(tr, suh, svh))
    x = torch.randn((a.rows, a.in_features), device="cuda", dtype=torch.float16)
    y = torch.empty((a.rows, a.out_features), device="cuda", dtype=torch.float16)
    flags = 4 if a.dp4a else 0
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for w in ws:
            Q.matmul_ex(w, x, flags, out=y)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(a.loops):
            for w in ws:
                Q.matmul_ex(w, x, flags, out=y)
    t0 = time.time()
    while time.time() - t0 < 0.3:  # clocks up from idle before the timed replays
        g.replay()
        torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(5):
        g.replay()
    ev[1].record()
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / (5 * a.loops * reps)
    print(f"{'dp4a' if a.dp4a else 'imma'} {a.in_features}x{a.out_features} n{a.n} rows{a.rows}: "
          f"{ms * 1000:.2f} us/launch, {nbytes / ms / 1e6:.1f} GB/s trellis", flush=True)


if __name__ == "__main__":
    main()
