"""The reference plugin's quant seam, in Python over libexl3b200.so.

Mirrors the QuantTable entries the turboexl3 plugins implement (plugins/turboexl3_ds41/plugin.zig:28-43;
plugins/turboexl3_qwen38/overlay/mlx_serve/abi/quant.zig:24-108): ``claims``, ``validate``, ``bill``, ``open`` /
``close`` (a :class:`LoadContext`), ``load_tensor``, ``load_bank``, ``release``, ``matmul``, ``moe`` and ``swiglu``,
with torch CUDA tensors in place of MLX arrays and the current torch stream in place of the MLX stream.  Every call
goes through the C ABI; refusals raise :class:`Exl3Error` with the library's message.
"""
from __future__ import annotations

import ctypes
import json
from typing import Callable, Mapping

import numpy as np
import torch

from . import _lib as L
from ._lib import Exl3Error, check

__all__ = ["Exl3Error", "Weight", "LoadContext", "claims", "validate", "bill", "matmul", "matmul_ex", "moe", "swiglu",
           "ep_dispatch", "ep_unpack", "ep_combine",
           "release", "weight_from_tensors", "stack", "decode_dense", "device_error", "CLAIM_NO", "CLAIM_BY_MARKER"]

CLAIM_NO, CLAIM_BY_MODE, CLAIM_BY_MARKER = L.CLAIM_NO, L.CLAIM_BY_MODE, L.CLAIM_BY_MARKER

_TORCH_DT = {torch.float16: L.F16, torch.bfloat16: L.BF16, torch.float32: L.F32, torch.int32: L.I32,
             torch.uint16: L.U16, torch.int16: L.I16}
_NP_DT = {np.dtype(np.float16): L.F16, np.dtype(np.float32): L.F32, np.dtype(np.int32): L.I32,
          np.dtype(np.uint32): L.U32, np.dtype(np.uint16): L.U16, np.dtype(np.int16): L.I16}


def _s(x) -> L.Str:
    if isinstance(x, (dict, list)):
        x = json.dumps(x)
    return L.Str.of(x if x is not None else "")


def _tensor(t: torch.Tensor) -> L.Tensor:
    if not t.is_cuda:
        raise Exl3Error(L.EXL3_FAILED, "exl3_b200: tensors must live on the GPU")
    if not t.is_contiguous():
        raise Exl3Error(L.EXL3_FAILED, "exl3_b200: tensors must be contiguous")
    if t.dim() < 1 or t.dim() > 4:
        raise Exl3Error(L.EXL3_FAILED, "exl3_b200: tensors have 1..4 dims")
    dt = _TORCH_DT.get(t.dtype)
    if dt is None:
        raise Exl3Error(L.EXL3_UNSUPPORTED, f"exl3_b200: dtype {t.dtype} is not served")
    out = L.Tensor()
    out.data = t.data_ptr()
    out.dtype = dt
    out.ndim = t.dim()
    for i, s in enumerate(t.shape):
        out.shape[i] = s
    return out


def _stream(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


class Weight:
    """A loaded (library-owned) or borrowed weight: the ABI's ``Weight`` (w = trellis, scales = suh, biases = svh)."""

    def __init__(self, raw: L.Weight, keep=()):
        self.raw = raw
        self._keep = tuple(keep)  # torch tensors a borrowed view points into

    @property
    def in_features(self) -> int:
        return self.raw.in_features

    @property
    def out_features(self) -> int:
        return self.raw.out_features

    @property
    def groups(self) -> int:
        return self.raw.groups

    @property
    def n(self) -> int:
        return self.raw.n

    @property
    def codebook(self) -> str:
        return "mcg" if self.raw.flags & L.WEIGHT_MCG else "mul1"

    @property
    def window(self) -> int:
        """The codeword window in bits (16 unless the pack narrowed it)."""
        return 16 - ((self.raw.flags & L.WEIGHT_WINDOW_MASK) >> L.WEIGHT_WINDOW_SHIFT)

    @property
    def bits(self) -> float:
        return self.raw.n / 16.0

    @property
    def device(self) -> int:
        return self.raw.device

    @property
    def trellis_bytes(self) -> int:
        return self.groups * (self.in_features // 16) * (self.out_features // 16) * self.n * 2

    def release(self) -> None:
        L.lib().exl3_release(ctypes.byref(self.raw))
        self._keep = ()

    def __del__(self):
        # an owned weight frees its memory; a borrowed one drops its kept matrices (exl3_resident), whose key -- the
        # device pointers -- a later weight may reuse once the tensors go
        try:
            if self.raw.size:
                self.release()
        except Exception:
            pass


# ------------------------------------------------------------------ claims / validate / bill (no GPU)

def claims(block_json, config_json="{}") -> int:
    """plugins/turboexl3_ds41/config.zig:43-47"""
    return L.lib().exl3_claims(_s(block_json), _s(config_json))


def validate(block_json, config_json="{}") -> None:
    """plugins/turboexl3_ds41/config.zig:49-54: raises Exl3Error naming what is refused."""
    check(L.lib().exl3_validate(_s(block_json), _s(config_json)))


def bill(block_json, model_dir: str, stored: int) -> int:
    """plugins/turboexl3_ds41/config.zig:57-61"""
    return int(L.lib().exl3_bill(_s(block_json), _s(model_dir), stored))


# ------------------------------------------------------------------ the load sequence

class LoadContext:
    """open -> load_tensor / load_bank* -> close (quant.zig:23), reading host tensors from ``source``.

    ``source`` maps a tensor name to a numpy array (or is a callable name -> array | None), e.g. a
    :class:`plugins_b200.pack.PackSource` over a pack's safetensors.
    """

    def __init__(self, block_json, config_json="{}", source: Mapping | Callable | None = None, model_dir: str = "",
                 device: int | None = None, stream=None):
        self.device = torch.cuda.current_device() if device is None else device
        self._get = source if callable(source) else (lambda name, s=source or {}: s.get(name))
        self._held: list = []
        self._cb = L.TensorFn(self._tensor_cb)
        self.ctx = L.LoadCtx()
        self.ctx.size = ctypes.sizeof(L.LoadCtx)
        self._strs = (_s(block_json), _s(config_json), _s(model_dir))
        self.ctx.block_json, self.ctx.config_json, self.ctx.model_dir = self._strs
        self.ctx.source = L.Source(None, self._cb)
        self.ctx.device = self.device
        with torch.cuda.device(self.device):
            self.ctx.stream = _stream(stream)
        self.opened = False

    def _tensor_cb(self, _ctx, name: L.Str, out) -> int:
        key = ctypes.string_at(name.ptr, name.len).decode()
        a = self._get(key)
        if a is None:
            return 1
        a = np.ascontiguousarray(a)
        dt = _NP_DT.get(a.dtype)
        if dt is None or a.ndim > 4:
            return 1
        self._held.append(a)
        out.contents.data = a.ctypes.data
        out.contents.dtype = dt
        out.contents.ndim = a.ndim
        for i, s in enumerate(a.shape):
            out.contents.shape[i] = s
        return 0

    def open(self) -> "LoadContext":
        check(L.lib().exl3_open(ctypes.byref(self.ctx)))
        self.opened = True
        return self

    def close(self) -> None:
        L.lib().exl3_close(ctypes.byref(self.ctx))
        self._held.clear()
        self.opened = False

    def __enter__(self):
        return self.open()

    def __exit__(self, *exc):
        self.close()

    def load_tensor(self, name: str, in_dim: int = 0) -> Weight:
        """plugins/turboexl3_ds41/plugin.zig:86-103"""
        w = L.Weight()
        try:
            check(L.lib().exl3_load_tensor(ctypes.byref(self.ctx), _s(name), in_dim, ctypes.byref(w)))
        finally:
            self._held.clear()
        return Weight(w)

    def load_bank(self, name: str, in_dim: int = 0) -> Weight:
        """plugins/turboexl3_ds41/plugin.zig:127-185"""
        w = L.Weight()
        try:
            check(L.lib().exl3_load_bank(ctypes.byref(self.ctx), _s(name), in_dim, ctypes.byref(w)))
        finally:
            self._held.clear()
        return Weight(w)


def release(w: Weight) -> None:
    """plugins/turboexl3_ds41/plugin.zig:231-237"""
    w.release()


# ------------------------------------------------------------------ forward calls

def matmul_ex(w: Weight, x: torch.Tensor, flags: int = 0, stream=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ W^T`` with EXL3_MATMUL_* flags (PREPARED: x already prepared f16; INNER: f32 inner product)."""
    shape = list(x.shape[:-1]) + [w.out_features]
    if out is None:
        dt = torch.float32 if flags & L.MATMUL_INNER else (torch.float16 if flags & L.MATMUL_PREPARED else x.dtype)
        out = torch.empty(shape, dtype=dt, device=x.device)
    xt, ot = _tensor(x), _tensor(out)
    check(L.lib().exl3_matmul_ex(ctypes.byref(w.raw), ctypes.byref(xt), flags, _stream(stream), ctypes.byref(ot)))
    return out


def matmul_timed(w: Weight, x: torch.Tensor, events, flags: int = 0, stream=None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """matmul_ex recording four torch.cuda.Event (or None) between its launches: [0] before the first and [3] after
    the last; on the GEMM path [1] after the operand images (prepare + decode) and [2] after the first GEMM."""
    shape = list(x.shape[:-1]) + [w.out_features]
    if out is None:
        dt = torch.float32 if flags & L.MATMUL_INNER else (torch.float16 if flags & L.MATMUL_PREPARED else x.dtype)
        out = torch.empty(shape, dtype=dt, device=x.device)
    ev = (ctypes.c_void_p * 4)(*[(e.cuda_event if e is not None else 0) for e in events])
    xt, ot = _tensor(x), _tensor(out)
    check(L.lib().exl3_matmul_timed(ctypes.byref(w.raw), ctypes.byref(xt), flags, _stream(stream), ctypes.byref(ot),
                                    ev))
    return out


def matmul(w: Weight, x: torch.Tensor, stream=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """plugins/turboexl3_ds41/plugin.zig:243-248: ``x @ W^T`` in x's dtype."""
    return matmul_ex(w, x, 0, stream, out)


def moe(bank: Weight, x: torch.Tensor, lhs=None, rhs=None, sorted_: bool = False, stream=None) -> torch.Tensor:
    """plugins/turboexl3_ds41/plugin.zig:263-265: refused by name (routed experts run through swiglu)."""
    empty = L.Tensor()
    xt = _tensor(x)
    out = L.Tensor()
    check(L.lib().exl3_moe(ctypes.byref(bank.raw), ctypes.byref(xt), ctypes.byref(empty), ctypes.byref(empty), int(sorted_),
                           _stream(stream), ctypes.byref(out)))
    raise AssertionError("unreachable")


def swiglu(gate: Weight, up: Weight, down: Weight, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor,
           limit: int = 0, verify_rows: bool = False, stream=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """plugins/turboexl3_ds41/plugin.zig:267-283: routed SwiGLU experts, x [B, S, D] -> [B, S, D] in x's dtype."""
    if out is None:
        out = torch.empty_like(x)
    opts = L.SwigluOpts(ctypes.sizeof(L.SwigluOpts), int(limit), int(bool(verify_rows)))
    xt, it, st, ot = _tensor(x), _tensor(inds), _tensor(scores), _tensor(out)
    check(L.lib().exl3_swiglu(ctypes.byref(gate.raw), ctypes.byref(up.raw), ctypes.byref(down.raw), ctypes.byref(xt),
                              ctypes.byref(it), ctypes.byref(st), ctypes.byref(opts), _stream(stream), ctypes.byref(ot)))
    return out


def moe_prefill_reserve(experts: int, hidden: int, inter: int, max_slots: int, device: int | None = None) -> int:
    """Reserves the workspace with which swiglu runs prompt-width calls (>= 1024 slots) on the tensor cores; returns its
    bytes (max_slots 0 frees it)."""
    b = ctypes.c_uint64(0)
    dev = torch.cuda.current_device() if device is None else device
    check(L.lib().exl3_moe_prefill_reserve(dev, int(experts), int(hidden), int(inter), int(max_slots), ctypes.byref(b)))
    return int(b.value)


def swiglu_shared(gate: Weight, up: Weight, down: Weight, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor,
                  shared_linears: tuple[Weight, Weight, Weight] | None = None, shared: torch.Tensor | None = None,
                  logit: torch.Tensor | None = None, gate_vec: torch.Tensor | None = None,
                  sigtab: torch.Tensor | None = None, limit: int = 0, stream=None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """quant.zig:95 swiglu_shared / SX/root.zig:38-68: the routed experts plus the shared expert (its three linears,
    or its output `shared`), gated by sigmoid(logit) when `logit` [B, S] or `gate_vec` [D] is given:
    out = RN(RN(routed) + RN(RN(sigmoid(logit)) * shared)), everything in x's dtype."""
    if out is None:
        out = torch.empty_like(x)
    for t in (shared, logit, gate_vec, sigtab):
        if t is not None and (not t.is_cuda or not t.is_contiguous() or t.dtype != x.dtype):
            raise Exl3Error(L.EXL3_UNSUPPORTED, "exl3_b200: shared-expert arrays are contiguous, on the GPU, in x's dtype")
    ptr = (lambda t: t.data_ptr() if t is not None else None)
    opts = L.SharedSwiglu(ctypes.sizeof(L.SharedSwiglu), int(limit),
                          *(ctypes.addressof(w.raw) if w is not None else None for w in (shared_linears or (None,) * 3)),
                          ptr(shared), ptr(logit), ptr(gate_vec), ptr(sigtab))
    xt, it, st, ot = _tensor(x), _tensor(inds), _tensor(scores), _tensor(out)
    check(L.lib().exl3_swiglu_shared(ctypes.byref(gate.raw), ctypes.byref(up.raw), ctypes.byref(down.raw),
                                     ctypes.byref(xt), ctypes.byref(it), ctypes.byref(st), ctypes.byref(opts),
                                     _stream(stream), ctypes.byref(ot)))
    return out


# ------------------------------------------------------------------ weights already on the device

def weight_from_tensors(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, window: int = 16,
                        codebook: str = "mul1") -> Weight:
    """A borrowed view of device tensors in the pack layout: trellis [(G,) in/16, out/16, n] (int16/uint16),
    suh [(G,) in] f16, svh [(G,) out] f16; ``window`` the block's codeword window (8..16 bits), ``codebook`` its
    codebook (mul1 or mcg)."""
    if trellis.dim() == 3:
        g = 1
        kt, ot, n = trellis.shape
    else:
        g, kt, ot, n = trellis.shape
    for t in (trellis, suh, svh):
        if not t.is_cuda or not t.is_contiguous():
            raise Exl3Error(L.EXL3_FAILED, "exl3_b200: weight tensors must be contiguous CUDA tensors")
    if suh.dtype != torch.float16 or svh.dtype != torch.float16:
        raise Exl3Error(L.EXL3_UNSUPPORTED, "exl3_b200: suh and svh are f16")
    if suh.numel() != g * kt * 16 or svh.numel() != g * ot * 16:
        raise Exl3Error(L.EXL3_UNSUPPORTED, "exl3_b200: suh/svh do not match the trellis")
    w = L.Weight()
    check(L.lib().exl3_weight_view(trellis.data_ptr(), suh.data_ptr(), svh.data_ptr(), g, kt * 16, ot * 16, n,
                                   trellis.device.index, ctypes.byref(w)))
    if not 8 <= int(window) <= 16:
        raise Exl3Error(L.EXL3_UNSUPPORTED, "exl3_b200: Exl3WindowUnsupported")
    if codebook not in ("mul1", "mcg"):
        raise Exl3Error(L.EXL3_UNSUPPORTED, "exl3_b200: Exl3CodebookUnsupported")
    w.flags |= L.weight_window(window) | (L.WEIGHT_MCG if codebook == "mcg" else 0)
    return Weight(w, keep=(trellis, suh, svh))


def stack(parts: list[Weight], stream=None) -> Weight:
    """Linears that read the same input, stacked along the output into one launch (SX/linear.zig:39-72)."""
    arr = (L.Weight * len(parts))(*[p.raw for p in parts])
    w = L.Weight()
    check(L.lib().exl3_weight_stack(arr, len(parts), _stream(stream), ctypes.byref(w)))
    return Weight(w)


def segment_outputs(w: Weight, y: torch.Tensor, rows: int) -> list[torch.Tensor]:
    """Splits a stacked weight's output (segments back to back, each [rows, width]) into per-linear views."""
    outs, flat = [], y.reshape(-1)
    for s in range(w.raw.nseg):
        c0, c1 = w.raw.seg_cols[s], w.raw.seg_cols[s + 1]
        outs.append(flat[rows * c0: rows * c1].view(rows, c1 - c0))
    return outs


def decode_dense(w: Weight, group: int = 0, dp4a: bool = False, stream=None) -> torch.Tensor:
    """W_hat (f16 bits as int16 -> viewed f16), row-major [in, out], decoded on the GPU."""
    dev = torch.device("cuda", w.device)
    out = torch.empty((w.in_features, w.out_features), dtype=torch.float16, device=dev)
    check(L.lib().exl3_decode_dense(ctypes.byref(w.raw), group, out.data_ptr(), L.MATMUL_DP4A if dp4a else 0,
                                    _stream(stream)))
    return out


def reconstruct_public(w: Weight, group: int = 0, stream=None) -> torch.Tensor:
    """The dense effective W (f16, row-major [in, out]; x @ W_eff = the linear's output), built on the GPU
    (SX/expert_exl3.zig:440-488 reconstructPublic)."""
    dev = torch.device("cuda", w.device)
    out = torch.empty((w.in_features, w.out_features), dtype=torch.float16, device=dev)
    check(L.lib().exl3_reconstruct_public(ctypes.byref(w.raw), group, out.data_ptr(), _stream(stream)))
    return out


def ep_dispatch(x: torch.Tensor, inds: torch.Tensor, experts: int, world: int, send: torch.Tensor,
                back_slot: torch.Tensor, rank: int = 0, shared: bool = False, stream=None) -> None:
    """Expert-parallel dispatch: x [T, D], inds [T, K] -> send [world, C + 1, D] (x's dtype), back_slot [T, K] i32.
    With `shared`, expert id `experts` is the shared expert every rank holds (local index experts / world)."""
    check(L.lib().exl3_ep_dispatch(ctypes.byref(_tensor(x)), ctypes.byref(_tensor(inds)), int(experts), int(world),
                                   int(rank), int(bool(shared)), _stream(stream), ctypes.byref(_tensor(send)),
                                   ctypes.byref(_tensor(back_slot))))


def ep_unpack(recv: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor, stream=None) -> None:
    """Received blocks [world, C + 1, D] -> swiglu's inds [world, C + 1, 1] i32 and scores (all 1) f32."""
    check(L.lib().exl3_ep_unpack(ctypes.byref(_tensor(recv)), _stream(stream), ctypes.byref(_tensor(inds)),
                                 ctypes.byref(_tensor(scores))))


def ep_combine(back: torch.Tensor, back_slot: torch.Tensor, scores: torch.Tensor, shared: torch.Tensor | None,
               out: torch.Tensor, stream=None) -> None:
    """out [T, D] = sum_k scores[t, k] * back[back_slot[t, k]] (k order, f32) + shared [T, D] f32 (optional)."""
    sh = _tensor(shared) if shared is not None else L.Tensor()
    check(L.lib().exl3_ep_combine(ctypes.byref(_tensor(back)), ctypes.byref(_tensor(back_slot)),
                                  ctypes.byref(_tensor(scores)), ctypes.byref(sh), _stream(stream),
                                  ctypes.byref(_tensor(out))))


def resident(ws: list[Weight], room: int = 0, stream=None) -> int:
    """quant.zig:96-99 ``resident``: keep the weights' decoded matrices from their first prefill call on (memory for
    speed), if everything kept fits in ``room`` bytes (0: no bound); returns the bytes kept.  An empty list drops every
    kept matrix."""
    arr = (L.Weight * max(len(ws), 1))(*[w.raw for w in ws])
    got = ctypes.c_uint64(0)
    check(L.lib().exl3_resident(arr, len(ws), int(room), _stream(stream), ctypes.byref(got)))
    return got.value


def resident_pending() -> int:
    """quant.zig:100-101 ``resident_pending``: the bytes ``resident`` admitted that no prefill call has filled yet."""
    return int(L.lib().exl3_resident_pending())


def device_error(device: int = 0, clear: bool = False) -> int:
    bits = ctypes.c_uint32(0)
    check(L.lib().exl3_device_error(device, ctypes.byref(bits), int(clear)))
    return bits.value
