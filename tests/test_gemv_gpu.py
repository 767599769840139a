"""The CUDA decode GEMV and decoder against the CPU oracle, through the C ABI.

Bars (from the reference and the north star):
  * decoded weights bit-exact (plugins/turboexl3_ds41/src/exl3/selfcheck.zig:861-930: decode_table, golden_tiles);
  * layer outputs within relative L2 2e-3 of the f32-accumulated truth (north star), and within the reference's own
    bar sqrt(LINEAR_BAR^2 + floor^2), LINEAR_BAR = 1.5e-3, floor = the output dtype's rounding of the truth
    (plugins/sushi_ds41/src/sushi/exl3/linear.zig:252-321);
  * a row's output bytes do not depend on how many rows share the launch (linear.zig:450-491).
"""
import hashlib
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REL_L2_BAR = 2e-3
LINEAR_BAR = 1.5e-3


@pytest.fixture(scope="module")
def Q():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from plugins_b200 import quant
    return quant


@pytest.fixture(scope="module")
def E():
    from plugins_b200 import encoder
    return encoder


def _rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / max((want ** 2).sum(), 1e-30)))


def _round(dt, v):
    t = torch.from_numpy(np.asarray(v, np.float32))
    return t.to(dt).float().numpy()


def _linear(E, in_f, out_f, n, seed):
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed)
    return tr, suh, svh


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("n", list(range(16, 97, 8)))  # whole and half bits per weight, 1..6
@pytest.mark.parametrize("dp4a", [False, True])
def test_decode_dense_bit_exact(Q, E, oracle, n, dp4a):
    in_f, out_f = 256, 384
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=n)
    w = Q.weight_from_tensors(tr, suh, svh)
    got = Q.decode_dense(w, dp4a=dp4a).view(torch.uint16).cpu().numpy()
    want = oracle.reconstruct_inner(_np(tr).view(np.uint16), in_f, out_f, n)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("in_f,out_f,n", [(256, 384, 64), (512, 256, 48), (384, 640, 40), (128, 128, 96)])
def test_reconstruct_public_against_oracle(Q, E, oracle, in_f, out_f, n):
    # reconstructPublic (SX/expert_exl3.zig:440-488): the dense effective W.  The oracle sums each Hadamard directly
    # and the GPU in butterflies, both in f32, so an f16 result may differ by one unit in the last place where the f32
    # value sits at a rounding boundary; and x @ W_eff is the linear (SX/linear.zig:200-224, the dense twin).
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=in_f + n)
    w = Q.weight_from_tensors(tr, suh, svh)
    got = Q.reconstruct_public(w).view(torch.int16).cpu().numpy().astype(np.int32)
    want = oracle.reconstruct_public(_np(tr).view(np.uint16), _np(suh).view(np.uint16), _np(svh).view(np.uint16),
                                     in_f, out_f, n).view(np.int16).astype(np.int32)
    ulp = np.abs(got - want)
    assert ulp.max() <= 1 and (ulp == 0).mean() > 0.99, (ulp.max(), (ulp == 0).mean())
    x = np.random.default_rng(n).standard_normal((3, in_f)).astype(np.float32)
    dense = x @ torch.from_numpy(got.astype(np.int16)).view(torch.float16).float().numpy()
    truth = oracle.host_project(x, _np(tr).view(np.uint16), _np(suh).view(np.uint16), _np(svh).view(np.uint16),
                                in_f, out_f, n, threads=8)
    assert _rel(dense, truth) < REL_L2_BAR


def test_reconstruct_public_group_of_a_bank(Q, E, oracle):
    groups, in_f, out_f, n = 3, 256, 128, 48
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=77, groups=groups)
    w = Q.weight_from_tensors(tr, suh, svh)
    for gi in range(groups):
        got = Q.reconstruct_public(w, gi).view(torch.int16).cpu().numpy().astype(np.int32)
        want = oracle.reconstruct_public(_np(tr[gi]).view(np.uint16), _np(suh[gi]).view(np.uint16),
                                         _np(svh[gi]).view(np.uint16), in_f, out_f, n).view(np.int16).astype(np.int32)
        assert np.abs(got - want).max() <= 1, gi


@pytest.mark.parametrize("n", [24, 32, 40, 48])
@pytest.mark.parametrize("dp4a", [False, True])
def test_frac_tiles_decode_on_gpu(Q, oracle, n, dp4a):
    # the real exllamav3 tiles at 1.5-3 bits (plugins/turboexl3_ds41/src/frac_tiles.json, frac_test.zig:23-57) laid
    # into a 128 x 128 layer (random words elsewhere) decode on the GPU to their pinned f16 bits, tile for tile
    tiles = [t for t in json.load(open(os.path.join(GOLD, "frac_tiles.json")))["tiles"] if t["n"] == n]
    assert 14 <= len(tiles) <= 64
    rng = np.random.default_rng(n)
    words = rng.integers(0, 65536, (8, 8, n), dtype=np.uint16)
    for i, t in enumerate(tiles):
        words[i // 8, i % 8] = t["words"]
    tr = torch.from_numpy(words.view(np.int16)).cuda()
    suh = torch.ones(128, dtype=torch.float16, device="cuda")
    svh = torch.ones(128, dtype=torch.float16, device="cuda")
    w = Q.weight_from_tensors(tr, suh, svh)
    got = Q.decode_dense(w, dp4a=dp4a).view(torch.uint16).cpu().numpy()
    for i, t in enumerate(tiles):
        ti, tj = i // 8, i % 8
        assert got[16 * ti:16 * ti + 16, 16 * tj:16 * tj + 16].reshape(-1).tolist() == t["expect"], t["src"]
    assert np.array_equal(got, oracle.reconstruct_inner(words, 128, 128, n))


@pytest.mark.parametrize("name", ["down_k2", "gate_up_k2", "down", "gate_up"])
def test_golden_planes_on_gpu(Q, oracle, name):
    # the manifest's splitmix64 planes decode on the GPU to the pinned W_hat digest, and the one-hot rows through
    # the GEMV (prepared x = e_r, inner product) reproduce W_hat's rows word for word (selfcheck.zig:861-907)
    p = json.load(open(os.path.join(GOLD, "manifest_golden.json")))["golden"]["planes"][name]
    i, o = p["projection"]
    k = p["K"]
    code = oracle.synth_plane(p["seed"], i, o, k)
    tr = torch.from_numpy(code.view(np.int16)).cuda()
    suh = torch.ones(i, dtype=torch.float16, device="cuda")
    svh = torch.ones(o, dtype=torch.float16, device="cuda")
    w = Q.weight_from_tensors(tr, suh, svh)
    for dp4a in (False, True):
        what = Q.decode_dense(w, dp4a=dp4a).view(torch.uint16).cpu().numpy()
        assert hashlib.sha256(what.astype("<u2").tobytes()).hexdigest() == p["w_hat_sha256"]
    rows = p["onehot_rows"]
    got = []
    for r0 in range(0, rows, 16):
        rc = min(16, rows - r0)
        x = torch.zeros((rc, i), dtype=torch.float16, device="cuda")
        x[torch.arange(rc), torch.arange(r0, r0 + rc)] = 1.0
        got.append(Q.matmul_ex(w, x, flags=1 | 2))  # PREPARED | INNER
    got = torch.cat(got).to(torch.float16).view(torch.uint16).cpu().numpy()
    assert hashlib.sha256(got.astype("<u2").tobytes()).hexdigest() == p["onehot_rows_sha256"]


CASES = [
    # (in, out, n, rows)
    (384, 256, 64, 1), (384, 256, 48, 3), (256, 384, 32, 8), (256, 384, 80, 5),
    (512, 640, 64, 9), (512, 256, 48, 16), (384, 512, 64, 17), (1024, 1024, 96, 2), (640, 384, 16, 4),
    # DeepSeek-V4.1 widths (the ds41 kernels' 5120 / 2304, TK/dsv41_exl3_mul1h_k{2,3}_*.metal)
    (5120, 2304, 32, 1), (2304, 5120, 48, 4),
    # half-bit rates (n = 16 k halfwords, k = 1.5 .. 5.5): the lane windows straddle word boundaries
    (384, 256, 24, 1), (256, 384, 40, 8), (512, 640, 56, 9), (512, 256, 72, 16), (1024, 1024, 88, 3),
]


@pytest.mark.parametrize("in_f,out_f,n,rows", CASES)
@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_matmul_against_f32_truth(Q, E, oracle, in_f, out_f, n, rows, dtype):
    dt = getattr(torch, dtype)
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=in_f * 7 + out_f + n + rows)
    w = Q.weight_from_tensors(tr, suh, svh)
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = ((torch.rand((rows, in_f), generator=g, device="cuda") * 2 - 1) * 30).to(dt)
    for dp4a in (False, True):
        y = Q.matmul_ex(w, x, flags=4 if dp4a else 0)
        assert y.dtype == dt and y.shape == (rows, out_f)
        got = y.float().cpu().numpy()
        want = oracle.host_project(x.float().cpu().numpy(), _np(tr).view(np.uint16), _np(suh).view(np.uint16),
                                   _np(svh).view(np.uint16), in_f, out_f, n, threads=8)
        assert np.isfinite(got).all()
        err = _rel(got, want)
        floor = _rel(_round(dt, want), want)
        assert err < REL_L2_BAR, (err, dp4a)
        assert err < np.sqrt(LINEAR_BAR ** 2 + floor ** 2), (err, floor, dp4a)


def test_imma_and_dp4a_paths_agree_bitwise(Q, E):
    tr, suh, svh = _linear(E, 1024, 2048, 64, seed=11)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.randn((8, 1024), device="cuda", dtype=torch.float16)
    a = Q.matmul_ex(w, x, flags=0)
    b = Q.matmul_ex(w, x, flags=4)
    # same weights and the same f32 sum order: identical bytes
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("in_f,out_f,n", [
    (2048, 3072, 48),
    # config 2's layer at 3 and 4 bpw: the cluster split's shared memory grows with the rows, and a split chosen per
    # width would change at 9 and 13 rows (exl3_gemv5.cu chooses it for every width at once)
    (4096, 12288, 48), (4096, 12288, 64),
])
def test_rows_share_a_launch_without_changing_bytes(Q, E, in_f, out_f, n):
    # linear.zig:450-491: row r has the same bytes at widths 1..16
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=5)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = (torch.rand((16, in_f), device="cuda") * 8 - 4).to(torch.bfloat16)
    solo = [Q.matmul(w, x[r:r + 1].contiguous()) for r in range(16)]
    for width in (2, 3, 5, 8, 9, 12, 13, 16):
        y = Q.matmul(w, x[:width].contiguous())
        for r in range(width):
            assert torch.equal(y[r].view(torch.int16), solo[r][0].view(torch.int16)), (width, r)


def test_past_f16_range_stays_finite(Q, E, oracle):
    # linear.zig:329-376: bf16/f32 rows whose outputs pass 65504
    for in_f, out_f in ((512, 256), (256, 4096)):
        tr, suh, svh = _linear(E, in_f, out_f, 64, seed=in_f + out_f)
        w = Q.weight_from_tensors(tr, suh, svh)
        for dt in (torch.bfloat16, torch.float32):
            x = ((torch.rand((5, in_f), device="cuda") * 2 - 1) * 3e5).to(dt)
            y = Q.matmul(w, x).float().cpu().numpy()
            want = oracle.host_project(x.float().cpu().numpy(), _np(tr).view(np.uint16), _np(suh).view(np.uint16),
                                       _np(svh).view(np.uint16), in_f, out_f, 64, threads=8)
            assert np.abs(want).max() > 65504
            assert np.isfinite(y).all()
            assert _rel(y, want) < np.sqrt(LINEAR_BAR ** 2 + _rel(_round(dt, want), want) ** 2)


def test_stacked_linears_each_hold_their_own_bar(Q, E, oracle):
    # SX/linear.zig:48-72 linearShared: linears that read one input in one launch
    in_f = 512
    widths = (640, 256, 256)
    parts, raw = [], []
    for i, wd in enumerate(widths):
        tr, suh, svh = _linear(E, in_f, wd, 64, seed=100 + i)
        raw.append((tr, suh, svh))
        parts.append(Q.weight_from_tensors(tr, suh, svh))
    st = Q.stack(parts)
    for rows in (1, 5, 8, 12):
        x = ((torch.rand((rows, in_f), device="cuda") * 2 - 1) * 30).to(torch.float16)
        y = Q.matmul(st, x)
        outs = Q.segment_outputs(st, y, rows)
        for (tr, suh, svh), yo, wd in zip(raw, outs, widths):
            want = oracle.host_project(x.float().cpu().numpy(), _np(tr).view(np.uint16), _np(suh).view(np.uint16),
                                       _np(svh).view(np.uint16), in_f, wd, 64, threads=8)
            assert _rel(yo.float().cpu().numpy(), want) < REL_L2_BAR


def test_grouped_linear(Q, E, oracle):
    # x [rows, groups, in] through each group's own linear (plugin.zig:107-124, linear.zig:24-36)
    groups, in_f, out_f, n = 3, 256, 384, 48
    tr, suh, svh = E.random_linear(in_f, out_f, n, seed=9, groups=groups)
    from plugins_b200 import _lib as L
    import ctypes
    w = Q.weight_from_tensors(tr, suh, svh)
    w.raw.flags |= L.WEIGHT_GROUPED
    x = torch.randn((4, groups, in_f), device="cuda", dtype=torch.float16)
    y = Q.matmul(w, x)
    assert y.shape == (4, groups, out_f)
    for g in range(groups):
        want = oracle.host_project(x[:, g].float().cpu().numpy(), _np(tr[g]).view(np.uint16),
                                   _np(suh[g]).view(np.uint16), _np(svh[g]).view(np.uint16), in_f, out_f, n, threads=8)
        assert _rel(y[:, g].float().cpu().numpy(), want) < REL_L2_BAR


def test_north_star_layer_parity(Q, E, oracle):
    # the 4096 x 12288 4-bpw layer at batch 1 and 8, against the f32 truth
    in_f, out_f, n = 4096, 12288, 64
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=2)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.randn((8, in_f), device="cuda", dtype=torch.float16)
    want = oracle.host_project(x.float().cpu().numpy(), _np(tr).view(np.uint16), _np(suh).view(np.uint16),
                               _np(svh).view(np.uint16), in_f, out_f, n, threads=os.cpu_count() or 8)
    for rows in (1, 8):
        y = Q.matmul(w, x[:rows].contiguous()).float().cpu().numpy()
        assert _rel(y, want[:rows]) < REL_L2_BAR
    assert Q.device_error(0) == 0


@pytest.mark.parametrize("n", [48, 40])
def test_persistent_gemv_layer_against_truth_and_row_invariance(Q, E, oracle, n):
    # config 2's down layer, 12288 -> 4096 at 3 (and 2.5) bpw: large enough for the persistent GEMV (exl3_gemv6.cu:
    # 8192 inputs and 16384 slab-units or more), at 1-4 rows with the input rotated in-CTA, at 8 with the prepare
    # launch, at 12-16 with two row groups; against the f32 truth, and row r's bytes the same at every width
    in_f, out_f = 12288, 4096
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=12)
    w = Q.weight_from_tensors(tr, suh, svh)
    x = torch.randn((16, in_f), device="cuda", dtype=torch.float16)
    want = oracle.host_project(x.float().cpu().numpy(), _np(tr).view(np.uint16), _np(suh).view(np.uint16),
                               _np(svh).view(np.uint16), in_f, out_f, n, threads=os.cpu_count() or 8)
    ys = {}
    for rows in (1, 3, 4, 8, 12, 16):
        y = Q.matmul(w, x[:rows].contiguous())
        assert _rel(y.float().cpu().numpy(), want[:rows]) < REL_L2_BAR, rows
        ys[rows] = y
    for rows, y in ys.items():
        assert torch.equal(y.view(torch.int16), ys[16][:rows].view(torch.int16)), rows
    assert Q.device_error(0) == 0


@pytest.mark.parametrize("n", [32, 48, 64, 80])
def test_large_layer_at_full_size(Q, E, oracle, n):
    # config 5's layer, 16384 x 53248 at 2-5 bpw (the persistent GEMV), through two size-independent properties:
    # one-hot prepared rows with the inner product give W_hat's rows bit for bit (the oracle decodes those slabs), and
    # batch-1 outputs of sampled 128-column blocks hold the f32 truth's bar (the output rotation is per block, so a
    # block's truth needs only its own columns)
    in_f, out_f = 16384, 53248
    tr, suh, svh = _linear(E, in_f, out_f, n, seed=5 + n)
    w = Q.weight_from_tensors(tr, suh, svh)
    ks = (0, 9999, in_f - 1)
    x = torch.zeros((len(ks), in_f), device="cuda", dtype=torch.float16)
    for i, k in enumerate(ks):
        x[i, k] = 1.0
    got = Q.matmul_ex(w, x, flags=1 | 2).to(torch.float16).view(torch.uint16).cpu().numpy()  # PREPARED | INNER
    for i, k in enumerate(ks):
        slab = _np(tr[k // 16:k // 16 + 1]).view(np.uint16)
        want = oracle.reconstruct_inner(slab, 16, out_f, n)[k % 16]
        assert np.array_equal(got[i], want), k
    x = torch.randn((1, in_f), device="cuda", dtype=torch.float16)
    y = Q.matmul(w, x).float().cpu().numpy()
    got, want = [], []
    for cb in (0, 137, out_f // 128 - 1):
        cols = slice(cb * 128, cb * 128 + 128)
        want.append(oracle.host_project(x.float().cpu().numpy(), _np(tr[:, cb * 8:cb * 8 + 8].contiguous()).view(np.uint16),
                                        _np(suh).view(np.uint16), _np(svh[cols].contiguous()).view(np.uint16), in_f, 128, n,
                                        threads=os.cpu_count() or 8))
        got.append(y[:, cols])
    assert _rel(np.concatenate(got, 1), np.concatenate(want, 1)) < REL_L2_BAR
    assert Q.device_error(0) == 0


def test_encoder_round_trip(Q, E, oracle):
    # encode -> decode on the GPU is bit-identical to the oracle's decode of the same bitstream, and the decoded
    # layer approximates the dense weight it encoded
    for bits in (2, 3, 4):
        w_dense, tr, suh, svh = E.synthetic_linear(512, 768, bits, seed=bits)
        w = Q.weight_from_tensors(tr, suh, svh)
        got = Q.decode_dense(w).view(torch.uint16).cpu().numpy()
        want = oracle.reconstruct_inner(_np(tr).view(np.uint16), 512, 768, 16 * bits)
        assert np.array_equal(got, want)
        x = torch.randn((4, 512), device="cuda", dtype=torch.float32)
        y = Q.matmul(w, x)
        ref = x @ w_dense.t()
        err = float(((y - ref).norm() / ref.norm()).item())
        assert err < {2: 0.7, 3: 0.45, 4: 0.3}[bits], (bits, err)  # greedy search: a sanity bound, not parity


def test_shapes_are_refused_by_name(Q, E):
    tr, suh, svh = _linear(E, 256, 256, 64, seed=1)
    w = Q.weight_from_tensors(tr, suh, svh)
    with pytest.raises(Q.Exl3Error, match="input width"):
        Q.matmul(w, torch.zeros((1, 384), device="cuda", dtype=torch.float16))
    with pytest.raises(Q.Exl3Error, match="f16, bf16 or f32"):
        Q.matmul(w, torch.zeros((1, 256), device="cuda", dtype=torch.int32))
    tr36 = torch.zeros((16, 16, 36), dtype=torch.int16, device="cuda")  # 2.25 bits: off the half-bit grid
    with pytest.raises(Q.Exl3Error, match="half-bit grid"):
        Q.weight_from_tensors(tr36, suh, svh)
    y = Q.matmul(w, torch.zeros((0, 256), device="cuda", dtype=torch.float16))
    assert y.shape == (0, 256)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_second_device_in_one_process(Q, E):
    # a kernel's shared-memory opt-in and occupancy belong to each device's context: the cluster-split GEMV, the
    # persistent GEMV and the GEMM on the second GPU of a process that ran them on the first give the same bytes
    outs = {}
    for dev in (0, 1):
        with torch.cuda.device(dev):
            for in_f, out_f, n, rows in ((4096, 12288, 64, 1), (12288, 4096, 48, 1), (512, 768, 64, 128)):
                tr, suh, svh = _linear(E, in_f, out_f, n, seed=in_f + out_f)
                w = Q.weight_from_tensors(tr, suh, svh)
                g = torch.Generator(device="cuda").manual_seed(rows)
                x = torch.randn((rows, in_f), generator=g, device="cuda").to(torch.float16)
                outs[(dev, in_f, out_f)] = Q.matmul(w, x).cpu()
            assert Q.device_error(dev) == 0
    for key, y in outs.items():
        if key[0] == 1:
            assert torch.equal(y.view(torch.int16), outs[(0,) + key[1:]].view(torch.int16)), key
