"""GPU time of the prefill path (prepare, decode to the B image, tensor-core GEMM) for one layer at several row counts.

    python -m plugins_b200.profile_gemm [--in 4096] [--out 12288] [--n 64] [--rows 64,256,2048,8192] [--reps 10]
                                        [--gemv-up-to 256] [--shape S] [--keep]

For each row count: the whole matmul and its two launches (the operand images: prepare + decode; the GEMM), timed
with CUDA events recorded between the launches (exl3_matmul_timed) over `reps` calls after warm-up, medians
reported; the GEMM kernel's TFLOP/s (2 M in out flops) and the images' bytes (x read, trellis read, A and B images
written); and, up to --gemv-up-to rows, the same rows forced through
the decode GEMV, for the crossover.  One JSON line per row count.  With --shape the GEMM's tile shape is fixed
(EXL3_GEMM_SHAPE).  With --keep the weight's decoded matrix is kept (exl3_resident: the first call fills it, the
timed calls read it instead of decoding; the images launch then only prepares x).  Under `ncu -k
regex:gemm_image_kernel` it is also the capture target for kernel profiles.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from . import encoder as E
from . import quant as Q

GEMV, GEMM = 8, 16


def _events():
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for e in ev:
        e.record()  # creates the CUDA event
    return ev


def time_call(w, x, out, flags, reps, warmup=3):
    for _ in range(warmup):
        Q.matmul_timed(w, x, [None] * 4, flags=flags, out=out)
    phases = {"total": [], "images": [], "gemm": []}
    for _ in range(reps):
        ev = _events()
        Q.matmul_timed(w, x, ev, flags=flags, out=out)
        torch.cuda.synchronize()
        phases["total"].append(ev[0].elapsed_time(ev[3]))
        if flags & GEMM:
            phases["images"].append(ev[0].elapsed_time(ev[1]))
            phases["gemm"].append(ev[1].elapsed_time(ev[2]))
    return {k: statistics.median(v) for k, v in phases.items() if v}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--in", dest="in_f", type=int, default=4096)
    ap.add_argument("--out", dest="out_f", type=int, default=12288)
    ap.add_argument("--n", type=int, default=64)
    ap.add_argument("--rows", default="64,256,2048,8192")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--gemv-up-to", type=int, default=256)
    ap.add_argument("--shape", type=int, default=-1)
    ap.add_argument("--keep", action="store_true", help="keep the decoded matrix (exl3_resident)")
    a = ap.parse_args()
    if a.shape >= 0:
        os.environ["EXL3_GEMM_SHAPE"] = str(a.shape)
    tr, suh, svh = E.random_linear(a.in_f, a.out_f, a.n, seed=2)
    w = Q.weight_from_tensors(tr, suh, svh)
    if a.keep:
        print(json.dumps({"kept_bytes": Q.resident([w])}), flush=True)
    for m in [int(v) for v in a.rows.split(",")]:
        x = torch.randn((m, a.in_f), device="cuda", generator=torch.Generator(device="cuda").manual_seed(m))
        x = x.to(torch.bfloat16)
        out = torch.empty((m, a.out_f), device="cuda", dtype=torch.bfloat16)
        t = time_call(w, x, out, GEMM, a.reps)
        flops = 2.0 * m * a.in_f * a.out_f
        img_bytes = (0 if a.keep else a.in_f * a.out_f * (a.n / 128 + 2)) + m * a.in_f * 4
        rec = {"rows": m, "in": a.in_f, "out": a.out_f, "n": a.n, "ms": {k: round(v, 4) for k, v in t.items()},
               "gemm_tflops": round(flops / (t["gemm"] * 1e-3) / 1e12, 1),
               "total_tflops": round(flops / (t["total"] * 1e-3) / 1e12, 1),
               "images_gbs": round(img_bytes / (t["images"] * 1e-3) / 1e9, 1)}
        if m <= a.gemv_up_to:
            g = time_call(w, x, out, GEMV, a.reps)
            rec["gemv_ms"] = round(g["total"], 4)
        print(json.dumps(rec), flush=True)
    if a.keep:
        Q.resident([])
    assert Q.device_error(0) == 0


if __name__ == "__main__":
    main()
