"""The model seam narrowed to the EXL3 linears (plugins_b200/model.py): claims and parse with the reference's named
refusals (plugins/turboexl3_qwen38/config.zig:19-119 and its tests), the bill, and the load and forward over a written
two-layer pack -- on the CPU oracle (the same host logic with oracle compute), and on the GPU through the library.
"""
import json

import numpy as np
import pytest

HIDDEN, INTER, MOE_INTER, SHARED_INTER, EXPERTS, TOPK = 256, 384, 256, 256, 4, 2
PREFIX = "model"


def _config(**over):
    text = {"hidden_size": HIDDEN, "intermediate_size": INTER, "num_hidden_layers": 2, "num_attention_heads": 4,
            "num_key_value_heads": 2, "head_dim": 64, "num_experts": EXPERTS, "num_experts_per_tok": TOPK,
            "moe_intermediate_size": MOE_INTER, "shared_expert_intermediate_size": SHARED_INTER}
    cfg = {"model_type": "qwen4_exp", "weight_prefix": PREFIX, "text_config": text,
           "trunk_quant": {"format": "exl3", "codebook": "mul1", "window": 16},
           "expert_quant": {"format": "exl3", "codebook": "mul1", "window": 16, "k": 3}}
    for k, v in over.items():
        if k in text:
            text[k] = v
        else:
            cfg[k] = v
    return cfg


def test_claims_by_marker_only_a_qwen38_pack_with_a_trunk_block():
    from plugins_b200 import model as M
    cfg = json.dumps(_config())
    assert M.claims("qwen4_exp", cfg) == M.CLAIM_BY_MARKER
    assert M.claims("qwen4_exp_text", cfg) == M.CLAIM_BY_MARKER
    assert M.claims("deepseek_v41", cfg) == M.CLAIM_NO
    assert M.claims("qwen4_exp", json.dumps({"trunk_quant": None})) == M.CLAIM_NO
    assert M.claims("qwen4_exp", json.dumps({})) == M.CLAIM_NO
    assert M.claims("qwen4_exp", "{") == M.CLAIM_NO


@pytest.mark.parametrize("edit,name", [
    ({"trunk_quant": {"format": "awq"}}, "NotExl3"),
    ({"trunk_quant": "exl3"}, "TrunkQuantNotAnObject"),
    ({"trunk_quant": {"format": "exl3", "codebook": "3inst"}}, "Exl3CodebookUnsupported"),
    ({"trunk_quant": {"format": "exl3", "codebook": "mul1", "window": 7}}, "Exl3WindowUnsupported"),
    ({"expert_quant": {"format": "exl3", "codebook": "mul1", "k": 3, "window": 17}}, "Exl3WindowUnsupported"),
    ({"expert_quant": {"format": "exl3", "codebook": "mul1"}}, "Exl3RateUnsupported"),
    ({"expert_quant": {"format": "exl3", "codebook": "mul1", "k": 2.25}}, "Exl3RateUnsupported"),
    ({"expert_quant": {"format": "exl3", "codebook": "mul1", "k": 8}}, "Exl3RateUnsupported"),
    ({"expert_quant": {"format": "exl3", "k": 3}}, "Exl3CodebookUnsupported"),
    ({"num_experts_per_tok": 33}, "Exl3TopKExceedsReduceBank"),
    ({"trunk_quant": None}, "Unsupported"),
    ({"hidden_size": 300}, "InvalidConfigField"),
    ({"num_attention_heads": 3}, "InvalidConfigField"),
    ({"hidden_size": -1}, "InvalidConfigField"),
    ({"num_experts_per_tok": 5}, "InvalidConfigField"),
])
def test_parse_refuses_by_name(edit, name):
    from plugins_b200 import model as M
    from plugins_b200._lib import Exl3Error
    with pytest.raises(Exl3Error) as e:
        M.parse(json.dumps(_config(**edit)))
    assert str(e.value).endswith("turboexl3_qwen38: " + name), str(e.value)


def test_parse_reads_the_linears_keys():
    from plugins_b200 import model as M
    c = M.parse(json.dumps(_config()))
    assert (c.hidden_size, c.intermediate_size, c.num_hidden_layers, c.num_experts, c.num_experts_per_tok) == \
        (HIDDEN, INTER, 2, EXPERTS, TOPK)
    assert c.weight_prefix == PREFIX and c.expert_quant["k"] == 3
    flat = _config()
    flat.update(flat.pop("text_config"))  # keys at the root read the same
    assert M.parse(json.dumps(flat)).moe_intermediate_size == MOE_INTER
    half = _config(expert_quant={"format": "exl3", "codebook": "mul1", "k": 2.5})
    assert M.parse(json.dumps(half)).expert_rate_n == 40  # the half-bit rates are served: n = 16 k halfwords
    narrow = _config(trunk_quant={"format": "exl3", "codebook": "mul1", "window": 12},
                     expert_quant={"format": "exl3", "codebook": "mul1", "k": 3, "window": 8})
    assert M.parse(json.dumps(narrow)).expert_rate_n == 48  # narrowed codeword windows 8..15 are served
    mcg = _config(trunk_quant={"format": "exl3", "codebook": "mcg"},
                  expert_quant={"format": "exl3", "codebook": "mcg", "k": 2.5, "window": 12})
    assert M.parse(json.dumps(mcg)).expert_rate_n == 40  # the mcg codebook too (config.zig:86-104)


def _linear(rng, i, o, n):
    return {"trellis": rng.integers(-32768, 32768, (i // 16, o // 16, n), dtype=np.int16),
            "suh": (rng.choice([-1.0, 1.0], i) * (0.002 + 0.02 * rng.random(i))).astype(np.float16),
            "svh": (rng.choice([-1.0, 1.0], o) * (0.5 + rng.random(o))).astype(np.float16)}


def _write_pack(d):
    from plugins_b200 import pack as P
    rng = np.random.default_rng(17)
    t = {}

    def put(name, i, o, n):
        for k, v in _linear(rng, i, o, n).items():
            t[f"{name}.{k}"] = v

    for layer in (0, 1):
        base = f"{PREFIX}.layers.{layer}"
        for proj, o in (("q_proj", 256), ("k_proj", 128), ("v_proj", 128)):
            put(f"{base}.self_attn.{proj}", HIDDEN, o, 64)
        put(f"{base}.self_attn.o_proj", 256, HIDDEN, 64)
    put(f"{PREFIX}.layers.0.mlp.gate_proj", HIDDEN, INTER, 48)
    put(f"{PREFIX}.layers.0.mlp.up_proj", HIDDEN, INTER, 48)
    put(f"{PREFIX}.layers.0.mlp.down_proj", INTER, HIDDEN, 48)
    for e in range(EXPERTS):
        for proj, (i, o) in (("gate_proj", (HIDDEN, MOE_INTER)), ("up_proj", (HIDDEN, MOE_INTER)),
                             ("down_proj", (MOE_INTER, HIDDEN))):
            put(f"{PREFIX}.layers.1.mlp.experts.{e}.{proj}", i, o, 48)
    t[f"{PREFIX}.layers.1.mlp.gate.weight"] = rng.standard_normal((EXPERTS, HIDDEN)).astype(np.float16)
    for proj, (i, o) in (("gate_proj", (HIDDEN, SHARED_INTER)), ("up_proj", (HIDDEN, SHARED_INTER)),
                         ("down_proj", (SHARED_INTER, HIDDEN))):
        put(f"{PREFIX}.layers.1.mlp.shared_expert.{proj}", i, o, 48)
    P.write_pack(str(d), t, _config(), shards=2)
    return t


class OracleModelOps:
    """The model's compute on the CPU oracle (f32 truths): linears are (trellis, suh, svh, in, out, n) tuples."""

    def __init__(self, O):
        self.O, self.src = O, None

    def open(self, block_json, config_json, source):
        self.src = source

    def close(self):
        self.src = None

    def _lin(self, name):
        tr, su, sv = (self.src(f"{name}.{k}") for k in ("trellis", "suh", "svh"))
        kt, ot, n = tr.shape
        return (tr.view(np.uint16), su.view(np.uint16), sv.view(np.uint16), kt * 16, ot * 16, n)

    def load_tensor(self, name, in_dim):
        w = self._lin(name)
        assert w[3] == in_dim
        return [w]

    def load_bank(self, name, in_dim):
        prefix, proj = name.rsplit(".experts.", 1)
        count = self.src(prefix + ".gate.weight").shape[0]
        parts = [self._lin(f"{prefix}.experts.{e}.{proj}") for e in range(count)]
        assert parts[0][3] == in_dim
        return tuple(np.stack([p[k] for p in parts]) for k in range(3)) + (parts[0][5],)

    def stack(self, parts):
        return [p for w in parts for p in w]

    def matmul(self, w, x):
        ys = [self.O.host_project(x, tr, su, sv, i, o, n, threads=2) for tr, su, sv, i, o, n in w]
        return ys[0] if len(ys) == 1 else ys

    def split(self, w, y, rows):
        return y

    def silu_mul(self, g, u):
        return g / (1.0 + np.exp(-g)) * u

    def swiglu(self, gate, up, down, x, inds, scores):
        return self.O.moe_truth(x, inds, scores, gate, up, down, x.shape[1], gate[0].shape[2] * 16, 0.0, threads=2)

    def add(self, a, b):
        return a + b

    def release(self, w):
        pass


def test_load_and_forward_over_the_linears_on_the_oracle(tmp_path, oracle):
    from plugins_b200 import model as M
    from plugins_b200 import pack as P
    O = oracle
    t = _write_pack(tmp_path)
    pk = P.PackSource(str(tmp_path))
    assert M.claims(pk.config["model_type"], pk.config_json) == M.CLAIM_BY_MARKER
    cfg = M.parse(pk.config_json)
    # the bill: every EXL3 tensor of the layers, as stored (the router weight is not an EXL3 tensor)
    assert M.bill(cfg, pk) == sum(v.nbytes for k, v in t.items() if k.endswith((".trellis", ".suh", ".svh")))
    ml = M.ModelLinears(cfg, pk, pk.config_json, ops=OracleModelOps(O))
    assert sorted(ml.linears_by_layer[0]) == ["mlp.down_proj", "mlp.gate_proj", "mlp.up_proj", "self_attn.k_proj",
                                              "self_attn.o_proj", "self_attn.q_proj", "self_attn.v_proj"]
    assert ml.banks_by_layer == {1: {"mlp": ["down_proj", "gate_proj", "up_proj"]}}
    assert (0, ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")) in ml.stacked
    assert (0, ("mlp.gate_proj", "mlp.up_proj")) in ml.stacked
    assert (1, ("mlp.shared_expert.gate_proj", "mlp.shared_expert.up_proj")) in ml.stacked

    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, HIDDEN)).astype(np.float16).astype(np.float32)

    def truth(name, xin):
        tr, su, sv = (t[f"{PREFIX}.layers.{name}.{k}"] for k in ("trellis", "suh", "svh"))
        return O.host_project(xin, tr.view(np.uint16), su.view(np.uint16), sv.view(np.uint16), tr.shape[0] * 16,
                              tr.shape[1] * 16, tr.shape[2], threads=2)

    q, k, v = ml.linears(0, ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), x)
    assert np.array_equal(q, truth("0.self_attn.q_proj", x)) and np.array_equal(v, truth("0.self_attn.v_proj", x))
    assert np.array_equal(ml.linear(1, "self_attn.o_proj", x), truth("1.self_attn.o_proj", x))
    g, u = truth("0.mlp.gate_proj", x), truth("0.mlp.up_proj", x)
    assert np.array_equal(ml.mlp(0, x), truth("0.mlp.down_proj", g / (1.0 + np.exp(-g)) * u))
    inds = np.array([[0, 3], [2, 1], [1, 0]], dtype=np.int32)
    sc = rng.random((3, TOPK)).astype(np.float32)
    bank = [tuple(np.stack([t[f"{PREFIX}.layers.1.mlp.experts.{e}.{p}.{kk}"] for e in range(EXPERTS)]).view(np.uint16)
                  for kk in ("trellis", "suh", "svh")) + (48,) for p in ("gate_proj", "up_proj", "down_proj")]
    gs, us = truth("1.mlp.shared_expert.gate_proj", x), truth("1.mlp.shared_expert.up_proj", x)
    want = O.moe_truth(x, inds, sc, *bank, HIDDEN, MOE_INTER, 0.0, threads=2) + \
        truth("1.mlp.shared_expert.down_proj", gs / (1.0 + np.exp(-gs)) * us)
    got = ml.experts(1, x, inds, sc)
    assert np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()) < 1e-6
    from plugins_b200._lib import Exl3Error
    with pytest.raises(Exl3Error):
        ml.linear(0, "self_attn.nope", x)
    with pytest.raises(Exl3Error):
        ml.experts(0, x, inds, sc)
    ml.release()
    pk.close()


@pytest.mark.gpu
def test_load_and_forward_over_the_linears_on_the_gpu(tmp_path, oracle):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import model as M
    from plugins_b200 import pack as P
    t = _write_pack(tmp_path)
    pk = P.PackSource(str(tmp_path))
    cfg = M.parse(pk.config_json)
    gpu = M.ModelLinears(cfg, pk, pk.config_json)
    cpu = M.ModelLinears(cfg, pk, pk.config_json, ops=OracleModelOps(oracle))
    rng = np.random.default_rng(6)
    x = rng.standard_normal((3, HIDDEN)).astype(np.float16)
    xg = torch.from_numpy(x).cuda()
    xf = x.astype(np.float32)

    def rel(a, b):
        a = a.float().cpu().numpy() if hasattr(a, "cpu") else a
        return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))

    for got, want in zip(gpu.linears(0, ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), xg),
                         cpu.linears(0, ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), xf)):
        assert rel(got, want) < 2e-3
    assert rel(gpu.linear(1, "self_attn.o_proj", xg), cpu.linear(1, "self_attn.o_proj", xf)) < 2e-3
    assert rel(gpu.mlp(0, xg), cpu.mlp(0, xf)) < 2e-3
    inds = np.array([[0, 3], [2, 1], [1, 0]], dtype=np.int32)
    sc = rng.random((3, TOPK)).astype(np.float32)
    got = gpu.experts(1, xg, torch.from_numpy(inds).cuda(), torch.from_numpy(sc).cuda())
    assert rel(got, cpu.experts(1, xf, inds, sc)) < 2e-3
    gpu.release()
    pk.close()


def test_native_bill_matches_the_stored_bytes(tmp_path):
    # exl3_model_bill: the bill a C or Zig host calls (no GPU)
    from plugins_b200 import model as M
    from plugins_b200 import pack as P
    t = _write_pack(tmp_path)
    pk = P.PackSource(str(tmp_path))
    want = sum(v.nbytes for k, v in t.items() if k.endswith((".trellis", ".suh", ".svh")))
    assert M.bill_native(pk.config_json, pk) == want == M.bill(M.parse(pk.config_json), pk)
    assert M.bill_native(json.dumps(_config(trunk_quant={"format": "awq"})), pk) == 0  # a refused pack bills nothing
    pk.close()


def test_native_load_refuses_a_pack_before_any_upload(tmp_path):
    import ctypes
    from plugins_b200 import _lib as L
    from plugins_b200 import model as M
    from plugins_b200 import pack as P
    _write_pack(tmp_path)
    pk = P.PackSource(str(tmp_path))
    keep, arr = M._native_names(pk)
    held = []
    src = L.Source(None, L.TensorFn(M._host_tensor_cb(pk, held)))
    m = ctypes.c_void_p()
    v = L.lib().exl3_model_load(L.Str.of(json.dumps(_config(trunk_quant={"format": "exl3", "codebook": "3inst"}))),
                                ctypes.byref(src), arr, len(keep), 0, 8, None, ctypes.byref(m))
    assert v.code == L.EXL3_UNSUPPORTED and v.message().endswith("Exl3CodebookUnsupported") and not m
    v = L.lib().exl3_model_load(L.Str.of(json.dumps(_config())), ctypes.byref(src), arr, len(keep), 0, 0, None,
                                ctypes.byref(m))
    assert v.code == L.EXL3_FAILED and not m  # max_rows 0
    pk.close()


@pytest.mark.gpu
def test_native_model_against_the_mirror_and_the_oracle(tmp_path, oracle):
    # the library's own load and forward (exl3_model_*) against the Python mirror on the same kernels (bit for bit
    # where both take the same launches) and against the oracle's f32 truth
    torch = pytest.importorskip("torch")
    from plugins_b200 import model as M
    from plugins_b200 import pack as P
    t = _write_pack(tmp_path)
    pk = P.PackSource(str(tmp_path))
    cfg = M.parse(pk.config_json)
    nat = M.NativeModel(pk.config_json, pk, max_rows=8)
    mir = M.ModelLinears(cfg, pk, pk.config_json)
    cpu = M.ModelLinears(cfg, pk, pk.config_json, ops=OracleModelOps(oracle))
    rng = np.random.default_rng(8)
    x = rng.standard_normal((3, HIDDEN)).astype(np.float16)
    xg = torch.from_numpy(x).cuda()
    xf = x.astype(np.float32)

    def rel(a, b):
        a = a.float().cpu().numpy() if hasattr(a, "cpu") else a
        return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))

    qkv = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")
    for a, b in zip(nat.linears(0, qkv, xg), mir.linears(0, qkv, xg)):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    for a, b in zip(nat.linears(1, ("self_attn.k_proj", "self_attn.o_proj"), xg),
                    (mir.linear(1, "self_attn.k_proj", xg), mir.linear(1, "self_attn.o_proj", xg))):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))  # not stacked at load: one launch each
    assert torch.equal(nat.linear(1, "self_attn.o_proj", xg).view(torch.int16),
                       mir.linear(1, "self_attn.o_proj", xg).view(torch.int16))
    assert rel(nat.mlp(0, xg), cpu.mlp(0, xf)) < 4e-3
    inds = np.array([[0, 3], [2, 1], [1, 0]], dtype=np.int32)
    sc = rng.random((3, TOPK)).astype(np.float32)
    y = nat.experts(1, xg.view(1, 3, HIDDEN), torch.from_numpy(inds).cuda().view(1, 3, TOPK),
                    torch.from_numpy(sc).cuda().view(1, 3, TOPK))
    assert rel(y.view(3, HIDDEN), cpu.experts(1, xf, inds, sc)) < 4e-3
    from plugins_b200._lib import Exl3Error
    with pytest.raises(Exl3Error, match="MissingLinear"):
        nat.linear(0, "self_attn.nope", xg)
    with pytest.raises(Exl3Error, match="max_rows"):
        nat.mlp(0, torch.zeros((9, HIDDEN), dtype=torch.float16, device="cuda"))
    nat.unload()
    mir.release()
    pk.close()
