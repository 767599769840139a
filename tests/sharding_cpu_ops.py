"""CPU stand-ins for the sharding drivers' compute (test infrastructure).

The drivers in plugins_b200/sharding.py take their compute as an ``ops`` object; these run it on the host so the
drivers' collectives, buffer layouts and index bookkeeping can be exercised over gloo ranks without a GPU:
  * the linear and the experts' SwiGLU are the oracle's f32 truth (oracle/exl3_oracle.c: host_project, moe_truth);
  * dispatch / unpack / combine restate exl3_ep_dispatch / exl3_ep_unpack / exl3_ep_combine (exl3_ep.cu) in Python:
    the same buffer layout ([world, C + 1, D] blocks, metadata row of 32-bit expert words), slot order, capacity and
    absent-slot rules, so the GPU tests can also hold the kernels to them word for word.
"""
from __future__ import annotations

import numpy as np
import torch


def _u16(t):
    return t.detach().cpu().contiguous().numpy().view(np.uint16)


class OracleLinearOps:
    def __init__(self, oracle):
        self.O = oracle

    def load(self, tr, suh, svh):
        return (_u16(tr), _u16(suh), _u16(svh), suh.shape[-1], svh.shape[-1], tr.shape[-1])

    def matmul(self, w, x, out=None):
        tr, suh, svh, i, o, n = w
        y = self.O.host_project(x.float().numpy(), tr, suh, svh, i, o, n, threads=2)
        y = torch.from_numpy(y).to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y


def ep_dispatch_ref(x, inds, experts, world, send, back_slot, rank=0, shared=False):
    """exl3_ep_dispatch on the host: fills send [world, C + 1, D] (x's dtype) and back_slot [T, K]."""
    tokens, topk = inds.shape
    cap = send.shape[1] - 1
    per = experts // world
    flat = inds.reshape(-1).tolist()
    bs = back_slot.view(-1)
    overflow = False
    for d in range(world):
        meta = send[d, cap].view(torch.int32)
        j = 0
        for s, e in enumerate(flat):
            if 0 <= e < experts:
                dest, local = e // per, e % per
            elif shared and e == experts:
                dest, local = rank, per
            else:
                if d == 0:
                    bs[s] = -1
                continue
            if dest != d:
                continue
            if j < cap:
                send[d, j] = x[s // topk]
                meta[j] = local
                bs[s] = d * (cap + 1) + j
                j += 1
            else:
                bs[s] = -1
                overflow = True
        meta[j:cap] = -1
    return overflow


def ep_unpack_ref(recv, inds, scores):
    world, rows, _ = recv.shape
    cap = rows - 1
    for d in range(world):
        inds[d, :cap, 0] = recv[d, cap].view(torch.int32)[:cap]
        inds[d, cap, 0] = -1
    scores.fill_(1.0)


def ep_combine_ref(back, back_slot, scores, shared, out):
    hidden = back.shape[-1]
    rows = back.reshape(-1, hidden)
    tokens, topk = back_slot.shape
    acc = torch.zeros((tokens, hidden), dtype=torch.float32)
    for t in range(tokens):
        for k in range(topk):
            pos = int(back_slot[t, k])
            if pos >= 0:
                acc[t] += scores[t, k] * rows[pos]
    if shared is not None:
        acc += shared
    out.copy_(acc.to(out.dtype))


class OracleExpertOps:
    """Banks are (trellis [E, ...], suh [E, in], svh [E, out], n) numpy tuples, as oracle.moe_truth takes them."""

    def __init__(self, oracle):
        self.O = oracle

    def dispatch(self, x, inds, experts, world, rank, shared, send, back_slot):
        ep_dispatch_ref(x, inds, experts, world, send, back_slot, rank, shared)

    def unpack(self, recv, inds, scores):
        ep_unpack_ref(recv, inds, scores)

    def swiglu(self, gate, up, down, x, inds, scores, out, limit):
        hidden = x.shape[-1]
        inter = gate[2].shape[-1]
        experts = gate[0].shape[0]
        xr = x.reshape(-1, hidden).float().numpy()
        ir = inds.reshape(xr.shape[0], -1).numpy()
        sr = scores.reshape(xr.shape[0], -1).numpy()
        y = np.zeros_like(xr)
        keep = [r for r in range(xr.shape[0]) if all(0 <= e < experts for e in ir[r])]
        if keep:
            y[keep] = self.O.moe_truth(xr[keep], ir[keep], sr[keep], gate, up, down, hidden, inter, float(limit),
                                       threads=2)
        out.copy_(torch.from_numpy(y).view(out.shape).to(out.dtype))

    def combine(self, back, back_slot, scores, out):
        ep_combine_ref(back, back_slot, scores, None, out)
