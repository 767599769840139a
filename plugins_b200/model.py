"""The reference's model seam, narrowed to the EXL3 linears: claims, parse, bill, load and the forward over the linears.

The reference's model plugin (plugins/turboexl3_qwen38/plugin.zig:38-53, ``ModelTable``) serves a whole
Qwen3.8-Flash-Next EXL3 pack: attention, caches, a drafter.  On this path only four of its entries matter, and this
module is them, over this library's quant seam (:mod:`plugins_b200.quant`):

* ``claims(model_type, config_json)`` -- config.zig:19-33: a ``qwen4_exp`` pack whose config names a ``trunk_quant``
  block is claimed by marker (the library's ``exl3_model_claims``);
* ``parse(config_json)`` -- config.zig:35-119 ``parse`` / ``checkPack`` and src/direct/config.zig:301-420
  ``parseJson``, in the library (``exl3_model_parse``, C++): MLX-free and bounds-checked; the pack's EXL3 blocks are
  checked with the reference's refusal names (``NotExl3``, ``Exl3CodebookUnsupported``, ``Exl3WindowUnsupported``,
  ``Exl3RateUnsupported``, ``Exl3TopKExceedsReduceBank``), narrowed to what this library decodes (the mul1 codebook,
  windows 8..16, whole and half bits per weight 1..6);
* ``bill(cfg, source)`` -- the resident bytes: EXL3 weights stay resident as the pack stores them
  (plugins/turboexl3_ds41/config.zig:57-61);
* :class:`ModelLinears` -- the load (every EXL3 linear and routed bank of the pack uploaded once, the linears that
  read one input stacked into one launch) and the forward over the linears: single and stacked projections, the dense
  SwiGLU MLP and the routed experts (plus the shared expert).

The compute goes through an ``ops`` object (:class:`CudaModelOps` by default), so the host logic runs unchanged on
the CPU oracle in the tests.
"""
from __future__ import annotations

import dataclasses
import json
import re

from ._lib import CLAIM_BY_MARKER, CLAIM_NO, EXL3_UNSUPPORTED, Exl3Error

_NAME = "turboexl3_qwen38"


def _refuse(name: str):
    raise Exl3Error(EXL3_UNSUPPORTED, f"{_NAME}: {name}")


@dataclasses.dataclass
class ModelConfig:
    """The parsed pack: the keys the linears need (src/direct/config.zig:24-78 names and defaults)."""
    model_type: str = "qwen4_exp"
    weight_prefix: str = "language_model.model"
    hidden_size: int = 3840
    intermediate_size: int = 15360
    num_hidden_layers: int = 48
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 256
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    expert_rate_n: int = 0  # the expert bank's halfwords per tile (16 k), 0 without experts
    trunk_quant: dict = dataclasses.field(default_factory=dict)
    expert_quant: dict | None = None


def claims(model_type: str, config_json: str) -> int:
    """A qwen4_exp pack whose config names a ``trunk_quant`` block (config.zig:19-29): by marker (exl3_model_claims)."""
    from . import _lib as L
    return int(L.lib().exl3_model_claims(L.Str.of(model_type), L.Str.of(config_json)))


def parse(config_json: str) -> ModelConfig:
    """config.json -> :class:`ModelConfig` through the library's parse (exl3_model_parse: MLX-free, bounds-checked,
    refusals by the reference's names); the EXL3 blocks ride along for the load."""
    import ctypes
    from . import _lib as L
    raw = L.ModelConfig()
    raw.size = ctypes.sizeof(L.ModelConfig)
    L.check(L.lib().exl3_model_parse(L.Str.of(config_json), ctypes.byref(raw)))
    root = json.loads(config_json)  # (parsed by the library above: a JSON object)
    c = ModelConfig(model_type=str(root.get("model_type", "qwen4_exp")), weight_prefix=raw.weight_prefix.decode(),
                    trunk_quant=root["trunk_quant"], expert_quant=root.get("expert_quant"))
    for f in ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
              "head_dim", "num_experts", "num_experts_per_tok", "moe_intermediate_size",
              "shared_expert_intermediate_size", "expert_rate_n"):
        setattr(c, f, int(getattr(raw, f)))
    return c


# ------------------------------------------------------------------ load and forward

_LAYER = re.compile(r"\.layers\.(\d+)\.(.+)$")
_EXPERT = re.compile(r"^(.*)\.experts\.(\d+)\.([^.]+)$")
STACKS = (("q_proj", "k_proj", "v_proj"), ("gate_proj", "up_proj"))  # linears that read one input (linear.zig:39-72)


def linear_names(cfg: ModelConfig, names) -> tuple[dict, dict]:
    """The pack's EXL3 linears by layer: ({layer: [module, ...]}, {layer: {bank: [proj, ...]}}), from the tensors
    named ``<prefix>.layers.<i>.<module>.trellis``; a routed bank is ``<bank>.experts.<e>.<proj>``."""
    linears, banks = {}, {}
    prefix = cfg.weight_prefix + ".layers."
    for n in sorted(names):
        if not n.endswith(".trellis") or not n.startswith(prefix):
            continue
        m = _LAYER.search(n[:-len(".trellis")])
        if not m:
            continue
        layer, module = int(m.group(1)), m.group(2)
        if layer >= cfg.num_hidden_layers:
            _refuse("InvalidConfigField")
        x = _EXPERT.match(module)
        if x:
            projs = banks.setdefault(layer, {}).setdefault(x.group(1), [])
            if x.group(3) not in projs:
                projs.append(x.group(3))
        else:
            linears.setdefault(layer, []).append(module)
    return linears, banks


def bill(cfg: ModelConfig, source) -> int:
    """Resident bytes: every EXL3 tensor the load uploads (trellis, suh, svh), as the pack stores it."""
    total = 0
    for n in source.names():
        if n.startswith(cfg.weight_prefix + ".layers.") and n.endswith((".trellis", ".suh", ".svh")):
            total += int(source(n).nbytes)
    return total


class CudaModelOps:
    """The library's quant seam on the GPU."""

    def __init__(self):
        import torch
        from . import quant as Q
        self.Q, self.torch = Q, torch
        self.ctx = None

    def open(self, block_json: str, config_json: str, source):
        self.ctx = self.Q.LoadContext(block_json, config_json, source=source).open()

    def close(self):
        if self.ctx is not None:
            self.ctx.close()
            self.ctx = None

    def load_tensor(self, name, in_dim):
        return self.ctx.load_tensor(name, in_dim=in_dim)

    def load_bank(self, name, in_dim):
        return self.ctx.load_bank(name, in_dim=in_dim)

    def stack(self, parts):
        return self.Q.stack(parts)

    def matmul(self, w, x):
        return self.Q.matmul(w, x)

    def split(self, w, y, rows):
        return self.Q.segment_outputs(w, y, rows)

    def silu_mul(self, g, u):
        t = self.torch
        return (t.nn.functional.silu(g.float()) * u.float()).to(g.dtype)

    def swiglu(self, gate, up, down, x, inds, scores):
        rows, hidden = x.shape
        k = inds.shape[1]
        return self.Q.swiglu(gate, up, down, x.reshape(1, rows, hidden).contiguous(),
                             inds.reshape(1, rows, k).contiguous(), scores.reshape(1, rows, k).contiguous()
                             ).reshape(rows, hidden)

    def add(self, a, b):
        return (a.float() + b.float()).to(a.dtype)

    def release(self, w):
        self.Q.release(w)


class ModelLinears:
    """The load and the forward over a pack's EXL3 linears.

    ``source`` is the pack (``source(name)`` -> host array or None, ``source.names()``; e.g.
    :class:`plugins_b200.pack.PackSource`).  Every EXL3 linear of every layer is uploaded once; the linears of a layer
    that read one input (q|k|v, gate|up) are also stacked into one launch; routed banks (``<bank>.experts.<e>.<proj>``)
    are loaded as banks.
    """

    def __init__(self, cfg: ModelConfig, source, config_json: str = "{}", ops=None):
        self.cfg, self.ops = cfg, ops or CudaModelOps()
        self.linears_by_layer, self.banks_by_layer = linear_names(cfg, source.names())
        self.w = {}       # (layer, module) -> weight
        self.stacked = {}  # (layer, (module, ...)) -> stacked weight
        self.banks = {}   # (layer, bank) -> {proj: weight}
        ops = self.ops
        ops.open(json.dumps(cfg.trunk_quant), config_json, source)
        try:
            for layer, modules in self.linears_by_layer.items():
                for m in modules:
                    name = f"{cfg.weight_prefix}.layers.{layer}.{m}"
                    self.w[(layer, m)] = ops.load_tensor(name, int(source(name + ".trellis").shape[0]) * 16)
                for group in STACKS:
                    for base in {m.rsplit(".", 1)[0] for m in modules if "." in m}:
                        full = tuple(f"{base}.{g}" for g in group)
                        if all((layer, f) in self.w for f in full):
                            self.stacked[(layer, full)] = ops.stack([self.w[(layer, f)] for f in full])
            if self.banks_by_layer:
                ops.close()
                ops.open(json.dumps(cfg.expert_quant or cfg.trunk_quant), config_json, source)
            for layer, banks in self.banks_by_layer.items():
                for bank, projs in banks.items():
                    d = {}
                    for p in projs:
                        first = f"{cfg.weight_prefix}.layers.{layer}.{bank}.experts.0.{p}.trellis"
                        arr = source(first)
                        if arr is None:
                            _refuse("MissingTensor")
                        d[p] = ops.load_bank(f"{cfg.weight_prefix}.layers.{layer}.{bank}.experts.{p}",
                                             int(arr.shape[0]) * 16)
                    self.banks[(layer, bank)] = d
        finally:
            ops.close()

    def linear(self, layer: int, module: str, x):
        """One linear: x [rows, in] -> [rows, out]."""
        w = self.w.get((layer, module))
        if w is None:
            _refuse(f"MissingLinear {layer}.{module}")
        return self.ops.matmul(w, x)

    def linears(self, layer: int, modules, x):
        """Linears that read the same x: one stacked launch when the load stacked them, else one each."""
        key = (layer, tuple(modules))
        if key in self.stacked:
            w = self.stacked[key]
            return list(self.ops.split(w, self.ops.matmul(w, x), x.shape[0]))
        return [self.linear(layer, m, x) for m in modules]

    def mlp(self, layer: int, x, module: str = "mlp"):
        """The dense SwiGLU MLP: down(silu(gate x) * up x)."""
        g, u = self.linears(layer, (f"{module}.gate_proj", f"{module}.up_proj"), x)
        return self.linear(layer, f"{module}.down_proj", self.ops.silu_mul(g, u))

    def experts(self, layer: int, x, inds, scores, bank: str = "mlp", shared: str | None = "mlp.shared_expert"):
        """The routed experts (sum_k score * expert_k(x), the library's routed SwiGLU), plus the shared expert's
        dense MLP when the layer has one."""
        b = self.banks.get((layer, bank))
        if b is None or not all(p in b for p in ("gate_proj", "up_proj", "down_proj")):
            _refuse(f"MissingBank {layer}.{bank}")
        y = self.ops.swiglu(b["gate_proj"], b["up_proj"], b["down_proj"], x, inds, scores)
        if shared and (layer, f"{shared}.down_proj") in self.w:
            y = self.ops.add(y, self.mlp(layer, x, module=shared))
        return y

    def release(self):
        for w in list(self.stacked.values()) + list(self.w.values()) + \
                [w for d in self.banks.values() for w in d.values()]:
            self.ops.release(w)
        self.w.clear()
        self.stacked.clear()
        self.banks.clear()


# ------------------------------------------------------------------ the same seam inside the library (C ABI)

def _native_names(source):
    from . import _lib as L
    names = [L.Str.of(n) for n in source.names()]
    arr = (L.Str * max(1, len(names)))(*names)
    return names, arr


def bill_native(config_json: str, source) -> int:
    """The bill through the library (exl3_model_bill): what a C or Zig host calls; no GPU."""
    import ctypes
    from . import _lib as L
    held = []
    cb = L.TensorFn(_host_tensor_cb(source, held))
    src = L.Source(None, cb)
    keep, arr = _native_names(source)
    return int(L.lib().exl3_model_bill(L.Str.of(config_json), ctypes.byref(src), arr, len(keep)))


def _host_tensor_cb(source, held: list):
    import numpy as np
    from .quant import _NP_DT

    def cb(_ctx, name, out) -> int:
        import ctypes
        a = source(ctypes.string_at(name.ptr, name.len).decode())
        if a is None:
            return 1
        a = np.ascontiguousarray(a)
        dt = _NP_DT.get(a.dtype)
        if dt is None or a.ndim > 4:
            return 1
        held.append(a)
        out.contents.data = a.ctypes.data
        out.contents.dtype = dt
        out.contents.ndim = a.ndim
        for i, s in enumerate(a.shape):
            out.contents.shape[i] = s
        return 0

    return cb


class NativeModel:
    """The model seam's load and forward over the linears inside the library (exl3_model_load / _linear / _linears /
    _mlp / _experts / _unload): the entries a C or Zig host binds in place of the reference's ModelTable
    (plugins/turboexl3_qwen38/plugin.zig:38-53).  ``source``: the pack (``source(name)`` and ``source.names()``)."""

    def __init__(self, config_json: str, source, device: int | None = None, max_rows: int = 64, stream=None):
        import ctypes
        import torch
        from . import _lib as L
        from .quant import _stream
        self.L, self.torch = L, torch
        self.device = torch.cuda.current_device() if device is None else device
        held: list = []
        self._cb = L.TensorFn(_host_tensor_cb(source, held))
        src = L.Source(None, self._cb)
        keep, arr = _native_names(source)
        self.m = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.check(L.lib().exl3_model_load(L.Str.of(config_json), ctypes.byref(src), arr, len(keep), self.device,
                                            int(max_rows), _stream(stream), ctypes.byref(self.m)))
        held.clear()

    def _out(self, x, width):
        return self.torch.empty(tuple(x.shape[:-1]) + (width,), dtype=x.dtype, device=x.device)

    def weight(self, layer: int, module: str):
        import ctypes
        w = self.L.Weight()
        if not self.L.lib().exl3_model_weight(self.m, layer, self.L.Str.of(module), ctypes.byref(w)):
            _refuse(f"MissingLinear {layer}.{module}")
        return w

    def linear(self, layer: int, module: str, x, stream=None):
        import ctypes
        from .quant import _stream, _tensor
        out = self._out(x, self.weight(layer, module).out_features)
        self.L.check(self.L.lib().exl3_model_linear(self.m, layer, self.L.Str.of(module), ctypes.byref(_tensor(x)),
                                                    _stream(stream), ctypes.byref(_tensor(out))))
        return out

    def linears(self, layer: int, modules, x, stream=None):
        import ctypes
        from .quant import _stream, _tensor
        widths = [self.weight(layer, m).out_features for m in modules]
        rows = x.numel() // x.shape[-1]
        flat = self.torch.empty(rows * sum(widths), dtype=x.dtype, device=x.device)
        mods = (self.L.Str * len(modules))(*[self.L.Str.of(m) for m in modules])
        self.L.check(self.L.lib().exl3_model_linears(self.m, layer, mods, len(modules), ctypes.byref(_tensor(x)),
                                                     _stream(stream), ctypes.byref(_tensor(flat))))
        outs, c0 = [], 0
        for wd in widths:
            outs.append(flat[rows * c0: rows * (c0 + wd)].view(tuple(x.shape[:-1]) + (wd,)))
            c0 += wd
        return outs

    def mlp(self, layer: int, x, module: str = "mlp", stream=None):
        import ctypes
        from .quant import _stream, _tensor
        out = self._out(x, self.weight(layer, module + ".down_proj").out_features)
        self.L.check(self.L.lib().exl3_model_mlp(self.m, layer, self.L.Str.of(module), ctypes.byref(_tensor(x)),
                                                 _stream(stream), ctypes.byref(_tensor(out))))
        return out

    def experts(self, layer: int, x, inds, scores, bank: str = "mlp", shared: str | None = "mlp.shared_expert",
                logit=None, stream=None):
        """x [B, S, D], inds / scores [B, S, K] -> [B, S, D]: the routed bank plus the shared expert (gated by
        sigmoid(logit) when `logit` [B, S] is given)."""
        import ctypes
        from .quant import _stream, _tensor
        out = self.torch.empty_like(x)
        self.L.check(self.L.lib().exl3_model_experts(
            self.m, layer, self.L.Str.of(bank), self.L.Str.of(shared or ""), ctypes.byref(_tensor(x)),
            ctypes.byref(_tensor(inds)), ctypes.byref(_tensor(scores)),
            None if logit is None else logit.data_ptr(), _stream(stream), ctypes.byref(_tensor(out))))
        return out

    def unload(self):
        if self.m:
            self.L.lib().exl3_model_unload(self.m)
            self.m = None
