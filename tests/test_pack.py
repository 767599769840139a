"""Packs on disk (plugins_b200/pack.py): the safetensors reader/writer, the pack index, the claim of a pack's
quantization block, and -- on the GPU -- a pack uploaded through the seam's load sequence (exl3_open /
exl3_load_tensor / exl3_load_bank, plugins/turboexl3_ds41/plugin.zig:84-185) computing the same bytes as the same
tensors registered directly.
"""
import json
import os
import struct

import numpy as np
import pytest


def test_safetensors_round_trip(tmp_path):
    from plugins_b200 import pack as P
    rng = np.random.default_rng(0)
    t = {
        "a.trellis": rng.integers(-32768, 32768, (4, 6, 48), dtype=np.int16),
        "a.suh": rng.standard_normal(64).astype(np.float16),
        "a.svh": rng.standard_normal(96).astype(np.float16),
        "f32": rng.standard_normal((3, 5)).astype(np.float32),
        "u16": rng.integers(0, 65536, (7,), dtype=np.uint16),
        "flag": np.array([True, False, True]),
        "scalar": np.array(3.5, dtype=np.float32),
    }
    path = str(tmp_path / "x.safetensors")
    P.write_safetensors(path, t, metadata={"format": "pt"})
    st = P.SafetensorsFile(path)
    assert set(st.names()) == set(t) and st.metadata == {"format": "pt"}
    for k, v in t.items():
        got = st.get(k)
        assert got.dtype == v.dtype and got.shape == v.shape and np.array_equal(got, v)
    assert st.get("missing") is None
    st.close()


def test_truncated_and_inconsistent_files_are_refused(tmp_path):
    from plugins_b200 import pack as P
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(ValueError):
        P.SafetensorsFile(str(bad))
    h = json.dumps({"w": {"dtype": "F16", "shape": [4], "data_offsets": [0, 6]}}).encode()
    wrong = tmp_path / "wrong.safetensors"
    wrong.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(ValueError):
        P.SafetensorsFile(str(wrong))


def _linear(rng, i, o, n):
    return {"trellis": rng.integers(-32768, 32768, (i // 16, o // 16, n), dtype=np.int16),
            "suh": (rng.choice([-1.0, 1.0], i) * (0.002 + 0.02 * rng.random(i))).astype(np.float16),
            "svh": (rng.choice([-1.0, 1.0], o) * (0.5 + rng.random(o))).astype(np.float16)}


def _make_pack(d, shards):
    from plugins_b200 import pack as P
    rng = np.random.default_rng(3)
    hidden, inter, experts = 256, 384, 4
    t = {}
    for name, (i, o, n) in {"model.layers.0.self_attn.q_proj": (hidden, 512, 64),
                            "model.layers.0.self_attn.o_proj": (512, hidden, 48)}.items():
        for k, v in _linear(rng, i, o, n).items():
            t[f"{name}.{k}"] = v
    for e in range(experts):
        for proj, (i, o) in (("gate_proj", (hidden, inter)), ("up_proj", (hidden, inter)), ("down_proj", (inter, hidden))):
            for k, v in _linear(rng, i, o, 48).items():
                t[f"model.layers.0.mlp.experts.{e}.{proj}.{k}"] = v
    t["model.layers.0.mlp.gate.weight"] = rng.standard_normal((experts, hidden)).astype(np.float16)
    config = {"model_type": "deepseek_v41", "hidden_size": hidden,
              "quantization_config": {"quant_method": "exl3", "bits": 3.0, "codebook": "mul1"}}
    P.write_pack(str(d), t, config, shards=shards)
    return t


@pytest.mark.parametrize("shards", [1, 3])
def test_pack_index_and_claim(tmp_path, shards):
    from plugins_b200 import pack as P
    from plugins_b200 import quant as Q
    t = _make_pack(tmp_path, shards)
    pk = P.PackSource(str(tmp_path))
    assert set(pk.names()) == set(t)
    for k, v in t.items():
        assert np.array_equal(pk(k), v)
    assert pk("model.layers.0.self_attn.k_proj.trellis") is None
    assert pk.stored_bytes == sum(v.nbytes for v in t.values())
    assert Q.claims(pk.block_json, pk.config_json) == Q.CLAIM_BY_MARKER
    Q.validate(pk.block_json, pk.config_json)
    assert Q.bill(pk.block_json, str(tmp_path), pk.stored_bytes) == pk.stored_bytes
    pk.close()


@pytest.mark.gpu
def test_pack_uploads_through_the_seam(tmp_path):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import pack as P
    from plugins_b200 import quant as Q
    t = _make_pack(tmp_path, 2)
    pk = P.PackSource(str(tmp_path))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    with Q.LoadContext(pk.block_json, pk.config_json, source=pk, model_dir=str(tmp_path)) as ctx:
        q = ctx.load_tensor("model.layers.0.self_attn.q_proj", in_dim=256)
        o = ctx.load_tensor("model.layers.0.self_attn.o_proj", in_dim=512)
        banks = [ctx.load_bank(f"model.layers.0.mlp.experts.{p}", in_dim=256 if p != "down_proj" else 384)
                 for p in ("gate_proj", "up_proj", "down_proj")]
    x = torch.randn((3, 256), device="cuda", dtype=torch.float16)
    for w, name in ((q, "model.layers.0.self_attn.q_proj"),):
        ref = Q.weight_from_tensors(dev(t[f"{name}.trellis"]), dev(t[f"{name}.suh"]), dev(t[f"{name}.svh"]))
        assert torch.equal(Q.matmul(w, x), Q.matmul(ref, x))
    xo = torch.randn((2, 512), device="cuda", dtype=torch.float16)
    ref_o = Q.weight_from_tensors(*(dev(t[f"model.layers.0.self_attn.o_proj.{k}"]) for k in ("trellis", "suh", "svh")))
    assert torch.equal(Q.matmul(o, xo), Q.matmul(ref_o, xo))
    ref_banks = []
    for p in ("gate_proj", "up_proj", "down_proj"):
        parts = [[dev(t[f"model.layers.0.mlp.experts.{e}.{p}.{k}"]) for e in range(4)] for k in ("trellis", "suh", "svh")]
        ref_banks.append(Q.weight_from_tensors(*(torch.stack(v) for v in parts)))
    xs = torch.randn((1, 5, 256), device="cuda", dtype=torch.float16)
    inds = torch.tensor([[[0, 2], [1, 3], [2, 0], [3, 1], [0, 1]]], dtype=torch.int32, device="cuda")
    sc = torch.rand((1, 5, 2), device="cuda")
    assert torch.equal(Q.swiglu(*banks, xs, inds, sc), Q.swiglu(*ref_banks, xs, inds, sc))
    for w in (q, o, *banks):
        Q.release(w)
    pk.close()
