"""EXL3 encoding of dense weights on the GPU (the reference ships no encoder: plugins/turboexl3_ds41/NOTICE:30-32).

A dense weight W [out, in] (torch Linear layout; y = x @ W^T) is stored as the reference decodes it
(plugins/sushi_ds41/src/sushi/exl3/linear.zig:119-148):  W^T = diag(suh) H M H diag(svh), H the block-diagonal
orthonormal 128-wide Hadamard.  The encoder draws seeded +-1 signs for suh and svh, rotates
M = H diag(suh) W^T diag(svh)^-1 H with a per-column scale folded into svh so M has the mul1 codebook's unit
variance, and searches a trellis for M with the library's greedy encoder (exl3_encode_trellis).
"""
from __future__ import annotations

import ctypes
import functools

import torch

from . import _lib as L
from ._lib import check


@functools.lru_cache(maxsize=8)
def _h128(device: str) -> torch.Tensor:
    idx = torch.arange(128)
    bits = (idx[:, None] & idx[None, :]).to(torch.int64)
    pop = torch.zeros_like(bits)
    for b in range(7):
        pop += (bits >> b) & 1
    h = torch.where(pop % 2 == 0, 1.0, -1.0) / (128 ** 0.5)
    return h.to(device=device, dtype=torch.float32)


def rotate_rows(m: torch.Tensor) -> torch.Tensor:
    """H (block-diagonal, 128) applied along dim 0 of m [k, c]."""
    k, c = m.shape
    h = _h128(str(m.device))
    return torch.matmul(h, m.reshape(k // 128, 128, c)).reshape(k, c)


def rotate_cols(m: torch.Tensor) -> torch.Tensor:
    """m [k, c] times H (block-diagonal, 128) on the right."""
    k, c = m.shape
    h = _h128(str(m.device))
    return torch.matmul(m.reshape(k, c // 128, 128), h).reshape(k, c)


def encode_trellis(target: torch.Tensor, n: int, stream=None) -> torch.Tensor:
    """target [in, out] f32 (rotated, unit variance) -> trellis int16 [in/16, out/16, n] on the same device."""
    target = target.contiguous().float()
    k, c = target.shape
    tr = torch.empty((k // 16, c // 16, n), dtype=torch.int16, device=target.device)
    st = torch.cuda.current_stream(target.device) if stream is None else stream
    check(L.lib().exl3_encode_trellis(target.data_ptr(), k, c, n, tr.data_ptr(), int(st.cuda_stream)))
    return tr


def quantize(w: torch.Tensor, bits: int, seed: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Dense W [out, in] -> (trellis int16 [in/16, out/16, 16 bits], suh f16 [in], svh f16 [out]) on W's device."""
    out_f, in_f = w.shape
    dev = w.device
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    suh = torch.where(torch.rand(in_f, generator=g, device=dev) < 0.5, -1.0, 1.0)
    sv = torch.where(torch.rand(out_f, generator=g, device=dev) < 0.5, -1.0, 1.0)
    a = rotate_rows(suh[:, None] * w.t().float() * sv[None, :])
    scale = a.pow(2).mean(dim=0).sqrt().clamp_min(1e-8)
    svh = (sv * scale).to(torch.float16)
    m = rotate_cols(a / svh.float().abs()[None, :])
    trellis = encode_trellis(m, 16 * bits)
    return trellis, suh.to(torch.float16), svh


def synthetic_linear(in_f: int, out_f: int, bits: int, seed: int, std: float = 0.02, device="cuda"):
    """A random-init dense weight W ~ N(0, std) of shape [out, in] (seeded) and its EXL3 encoding."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randn((out_f, in_f), generator=g, device=device) * std
    tr, suh, svh = quantize(w, bits, seed)
    return w, tr, suh, svh


def random_linear(in_f: int, out_f: int, n: int, seed: int, device="cuda", groups: int | None = None):
    """Uniformly random trellis words with the reference test's scales (SX/linear.zig:160-176): suh = +-(0.002 + U
    0.02), svh = +-(0.5 + U).  Decoding is defined for any bitstream, so these exercise every state."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    lead = () if groups is None else (groups,)
    tr = torch.randint(-32768, 32768, lead + (in_f // 16, out_f // 16, n), generator=g, device=device,
                       dtype=torch.int32).to(torch.int16)

    def signed(shape, lo, span):
        s = torch.where(torch.rand(shape, generator=g, device=device) < 0.5, -1.0, 1.0)
        return (s * (lo + torch.rand(shape, generator=g, device=device) * span)).to(torch.float16)

    suh = signed(lead + (in_f,), 0.002, 0.02)
    svh = signed(lead + (out_f,), 0.5, 1.0)
    return tr, suh, svh
