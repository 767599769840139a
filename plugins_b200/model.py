"""The reference's model seam, narrowed to the EXL3 linears: claims, parse, bill, load and the forward over the linears.

The reference's model plugin (plugins/turboexl3_qwen38/plugin.zig:38-53, ``ModelTable``) serves a whole
Qwen3.8-Flash-Next EXL3 pack: attention, caches, a drafter.  On this path only four of its entries matter, and this
module is them, over this library's quant seam (:mod:`plugins_b200.quant`):

* ``claims(model_type, config_json)`` -- config.zig:19-33: a ``qwen4_exp`` pack whose config names a ``trunk_quant``
  block is claimed by marker;
* ``parse(config_json)`` -- config.zig:35-119 ``parse`` / ``checkPack`` and src/direct/config.zig:301-420
  ``parseJson``: MLX-free and bounds-checked; the pack's EXL3 blocks are checked with the reference's refusal names
  (``NotExl3``, ``Exl3CodebookUnsupported``, ``Exl3WindowUnsupported``, ``Exl3RateUnsupported``,
  ``Exl3TopKExceedsReduceBank``), narrowed to what this library decodes (the mul1 codebook, 16-bit windows, whole
  bits per weight 1..6);
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
import math
import re

from ._lib import CLAIM_BY_MARKER, CLAIM_NO, EXL3_UNSUPPORTED, Exl3Error

MODEL_TYPES = ("qwen4_exp", "qwen4_exp_text")  # plugins/turboexl3_qwen38/src/direct/config.zig:11
MAX_TOPK = 32  # the widest top-k the routed reduction holds (plugins/turboexl3_qwen38/config.zig:16)
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
    trunk_quant: dict = dataclasses.field(default_factory=dict)
    expert_quant: dict | None = None


def claims(model_type: str, config_json: str) -> int:
    """A qwen4_exp pack whose config names a ``trunk_quant`` block (config.zig:19-29); everything else is not ours."""
    if model_type not in MODEL_TYPES:
        return CLAIM_NO
    try:
        doc = json.loads(config_json)
    except (ValueError, TypeError):
        return CLAIM_NO
    if not isinstance(doc, dict):
        return CLAIM_NO
    t = doc.get("trunk_quant")
    return CLAIM_NO if t is None else CLAIM_BY_MARKER


def _check_block(o: dict, bank: bool) -> None:
    """config.zig:101-119 checkBlock, narrowed to this library's decode."""
    if o.get("format") != "exl3":
        _refuse("NotExl3")
    if o.get("codebook") != "mul1":
        # the reference also decodes mcg, and lets a trunk block leave its codebook unnamed; this library decodes
        # mul1 only and needs the block to say so
        _refuse("Exl3CodebookUnsupported")
    w = o.get("window")
    if w is not None and (not isinstance(w, int) or isinstance(w, bool) or w != 16):
        _refuse("Exl3WindowUnsupported")  # the reference admits 8..16; narrowed windows are not decoded here
    if bank:
        k = o.get("k")
        if isinstance(k, bool) or not isinstance(k, (int, float)):
            _refuse("Exl3RateUnsupported")
        scaled = float(k) * 16.0
        n = round(scaled)
        if not math.isfinite(scaled) or abs(scaled - n) > 1e-6 or n < 16 or n > 96 or n % 16:
            _refuse("Exl3RateUnsupported")  # the reference admits even n in 16..128; here whole bits per weight


def _u32(obj: dict, key: str, default: int, required: bool = False) -> int:
    v = obj.get(key)
    if v is None:
        if required:
            _refuse("InvalidConfigField")
        return default
    if isinstance(v, bool) or not isinstance(v, int) or v < 0 or v > 0xFFFFFFFF:
        _refuse("InvalidConfigField")
    return v


def parse(config_json: str) -> ModelConfig:
    """config.json -> :class:`ModelConfig`, refusing by name what the reference refuses and what this library does
    not decode."""
    try:
        root = json.loads(config_json)
    except (ValueError, TypeError):
        _refuse("InvalidConfig")
    if not isinstance(root, dict):
        _refuse("InvalidConfig")
    # the pack's EXL3 blocks first (config.zig:35-41: checkPack runs before the model's parse)
    t = root.get("trunk_quant")
    if t is not None:
        if not isinstance(t, dict):
            _refuse("TrunkQuantNotAnObject")
        _check_block(t, False)
    e = root.get("expert_quant")
    text = root.get("text_config", root)
    if not isinstance(text, dict):
        _refuse("InvalidConfigField")
    if e is not None:
        if not isinstance(e, dict):
            _refuse("NotExl3")
        _check_block(e, True)
        k = text.get("num_experts_per_tok")
        if isinstance(k, int) and not isinstance(k, bool) and k > MAX_TOPK:
            _refuse("Exl3TopKExceedsReduceBank")
    if t is None:
        _refuse("Unsupported")  # a K pack is fully EXL3 (src/direct/config.zig:372-374)
    c = ModelConfig(model_type=str(root.get("model_type", "qwen4_exp")), trunk_quant=t, expert_quant=e)
    if isinstance(root.get("weight_prefix"), str):
        c.weight_prefix = root["weight_prefix"]
    c.hidden_size = _u32(text, "hidden_size", c.hidden_size)
    c.intermediate_size = _u32(text, "intermediate_size", c.intermediate_size)
    c.num_hidden_layers = _u32(text, "num_hidden_layers", c.num_hidden_layers)
    c.num_attention_heads = _u32(text, "num_attention_heads", c.num_attention_heads)
    c.num_key_value_heads = _u32(text, "num_key_value_heads", c.num_key_value_heads)
    c.head_dim = _u32(text, "head_dim", c.head_dim)
    c.num_experts = _u32(text, "num_experts", 0)
    c.num_experts_per_tok = _u32(text, "num_experts_per_tok", 0)
    c.moe_intermediate_size = _u32(text, "moe_intermediate_size", 0)
    c.shared_expert_intermediate_size = _u32(text, "shared_expert_intermediate_size", 0)
    # bounds the linears need: every width a whole number of 128-column blocks, heads that divide
    if c.hidden_size == 0 or c.hidden_size % 128 or c.num_hidden_layers == 0:
        _refuse("InvalidConfigField")
    if c.num_key_value_heads == 0 or c.num_attention_heads % c.num_key_value_heads:
        _refuse("InvalidConfigField")
    for width in (c.intermediate_size, c.moe_intermediate_size, c.shared_expert_intermediate_size):
        if width % 128:
            _refuse("InvalidConfigField")
    if c.num_experts:
        if e is None or c.num_experts_per_tok == 0 or c.num_experts_per_tok > c.num_experts or \
                c.num_experts > 1024 or c.moe_intermediate_size == 0:
            _refuse("InvalidConfigField")
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
