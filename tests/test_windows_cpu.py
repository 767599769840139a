"""The lane-window rule the decode kernels use (plugins_b200/csrc/exl3_windows.h), compiled for the host, against the
oracle's unpacking of the bitstream (oracle/exl3_oracle.c exl3o_unpack_tile, SX/expert_exl3.zig:317-336): every
lane's eight windows of random tiles, at every rate the kernels serve -- whole and half bits per weight, n = 16..96.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RATES = tuple(range(16, 97, 8))  # n halfwords per tile: 1, 1.5, 2, ..., 6 bits per weight

SHIM = r"""
#include "exl3_windows.h"
extern "C" int lane_windows_host(const uint32_t* words, int n, uint32_t lane, uint32_t* out) {
  uint32_t w[8];
  switch (n) {
#define CASE(N) case N: { exl3::LaneWin<N> lw; lw.init(lane); exl3::lane_windows<N>(words, lw, w); break; }
    CASE(16) CASE(24) CASE(32) CASE(40) CASE(48) CASE(56) CASE(64) CASE(72) CASE(80) CASE(88) CASE(96)
    default: return 1;
  }
  for (int j = 0; j < 8; ++j) out[j] = w[j];
  return 0;
}
"""


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    d = tmp_path_factory.mktemp("windows")
    src, so = d / "shim.cpp", d / "shim.so"
    src.write_text(SHIM)
    subprocess.check_call(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I", os.path.join(ROOT, "plugins_b200", "csrc"),
                           str(src), "-o", str(so)])
    lib = ctypes.CDLL(str(so))
    lib.lane_windows_host.restype = ctypes.c_int
    lib.lane_windows_host.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p]
    return lib


@pytest.mark.parametrize("n", RATES)
def test_lane_windows_are_the_bitstreams_windows(shim, oracle, n):
    rng = np.random.default_rng(n)
    for _ in range(20):
        halves = rng.integers(0, 65536, n, dtype=np.uint16)
        words = halves.view(np.uint32).copy()  # u32 word m = hw[2m] | hw[2m+1] << 16
        want = oracle.unpack_tile(halves, n)
        out = np.empty(8, np.uint32)
        for lane in range(32):
            assert shim.lane_windows_host(words.ctypes.data, n, lane, out.ctypes.data) == 0
            assert np.array_equal(out, want[8 * lane:8 * lane + 8].astype(np.uint32)), (n, lane)


def test_narrowed_window_truth_is_the_masked_decode(oracle):
    # expert_exl3.zig Window: a narrowed window decodes the low w bits of each 16-bit window.  The oracle's W_hat at
    # window w is the tile decode of the masked codewords, differs from the 16-bit one, and its f32 truth is the
    # rotated product with that W_hat
    rng = np.random.default_rng(12)
    in_f, out_f, n = 256, 384, 40
    tr = rng.integers(0, 65536, (in_f // 16, out_f // 16, n), dtype=np.uint16)
    suh = (rng.choice([-1.0, 1.0], in_f) * (0.002 + 0.02 * rng.random(in_f))).astype(np.float16).view(np.uint16)
    svh = (rng.choice([-1.0, 1.0], out_f) * (0.5 + rng.random(out_f))).astype(np.float16).view(np.uint16)
    for w in (8, 12, 15):
        full = oracle.reconstruct_inner(tr, in_f, out_f, n)
        narrow = oracle.reconstruct_inner(tr, in_f, out_f, n, window=w)
        assert not np.array_equal(full, narrow)
        tile = oracle.decode_tile(tr[1, 2], n, window=w)
        assert np.array_equal(narrow[16:32, 32:48].reshape(-1), tile)
        x = rng.standard_normal((2, in_f)).astype(np.float32)
        got = oracle.host_project(x, tr, suh, svh, in_f, out_f, n, threads=2, window=w)
        s = x * suh.view(np.float16).astype(np.float32)
        s = np.concatenate([np.stack([oracle.hadamard128(r[b:b + 128]) for b in range(0, in_f, 128)]).reshape(-1)
                            for r in s]).reshape(2, in_f)
        inner = s @ narrow.view(np.float16).astype(np.float32)
        y = np.stack([np.concatenate([oracle.hadamard128(r[b:b + 128]) for b in range(0, out_f, 128)]) for r in inner])
        y *= svh.view(np.float16).astype(np.float32)
        assert np.allclose(got, y, rtol=1e-4, atol=1e-4 * np.abs(y).max())


IMMA_SHIM = r"""
#include "exl3_windows.h"
extern "C" int imma_windows_host(const uint32_t* words, int n, uint32_t lane, uint32_t mask, uint32_t* out) {
  uint32_t w[8];
  switch (n) {
#define CASE(N) case N: { exl3::ImmaWin<N> iw; iw.init(lane, mask); exl3::imma_windows<N>(words, iw, w); break; }
    CASE(16) CASE(24) CASE(32) CASE(40) CASE(48) CASE(56) CASE(64) CASE(72) CASE(80) CASE(88) CASE(96)
    default: return 1;
  }
  for (int j = 0; j < 8; ++j) out[j] = w[j];
  return 0;
}
"""


@pytest.fixture(scope="module")
def imma_shim(tmp_path_factory):
    d = tmp_path_factory.mktemp("imma_windows")
    src, so = d / "shim.cpp", d / "shim.so"
    src.write_text(IMMA_SHIM)
    subprocess.check_call(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I", os.path.join(ROOT, "plugins_b200", "csrc"),
                           str(src), "-o", str(so)])
    lib = ctypes.CDLL(str(so))
    lib.imma_windows_host.restype = ctypes.c_int
    lib.imma_windows_host.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p]
    return lib


@pytest.mark.parametrize("n", RATES)
@pytest.mark.parametrize("window", [16, 12])
def test_imma_order_windows_are_the_neighbours_windows(imma_shim, oracle, n, window):
    # lane (g, q) of the tensor-pipe order reads lanes (g, 2q mod 4) and (g, 2q + 1 mod 4)'s windows jb, jb+1, jb+4,
    # jb+5 (jb = 0 for q < 2, else 2): checked against the oracle's unpacking of the bitstream, masked to the window
    rng = np.random.default_rng(n + window)
    mask = (1 << window) - 1
    for _ in range(10):
        halves = rng.integers(0, 65536, n, dtype=np.uint16)
        words = halves.view(np.uint32).copy()
        cw = oracle.unpack_tile(halves, n).astype(np.uint32) & mask
        out = np.empty(8, np.uint32)
        for lane in range(32):
            g, q = lane >> 2, lane & 3
            jb = 0 if q < 2 else 2
            want = [cw[8 * (4 * g + ((2 * q + i) & 3)) + j] for i in (0, 1) for j in (jb, jb + 1, jb + 4, jb + 5)]
            assert imma_shim.imma_windows_host(words.ctypes.data, n, lane, mask, out.ctypes.data) == 0
            assert out.tolist() == want, (n, lane)


@pytest.mark.parametrize("n", [24, 48, 64, 88])
def test_imma_order_mcg_fragment_is_the_tiles_weights(imma_shim, oracle, n):
    # the tensor-pipe operand order (lane (g, q): column g's and g + 8's weights at k = 4q .. 4q + 3, pairs
    # (4q, 4q + 1) then (4q + 2, 4q + 3)): the neighbours' windows decoded by mcg in the order the kernels pack them
    # (a[0] = w0, w1; a[1] = w2, w3 (column g + 8); a[2] = w4, w5; a[3] = w6, w7) are the tile's weights there
    rng = np.random.default_rng(n)
    halves = rng.integers(0, 65536, n, dtype=np.uint16)
    words = halves.view(np.uint32).copy()
    tile = oracle.decode_tile(halves, n, codebook="mcg").reshape(16, 16)  # [k][column]
    out = np.empty(8, np.uint32)
    for lane in range(32):
        g, q = lane >> 2, lane & 3
        assert imma_shim.imma_windows_host(words.ctypes.data, n, lane, 0xFFFF, out.ctypes.data) == 0
        dec = [oracle.decode_mcg(int(c)) for c in out]
        k = 4 * q
        want = [tile[k, g], tile[k + 1, g], tile[k, g + 8], tile[k + 1, g + 8],
                tile[k + 2, g], tile[k + 3, g], tile[k + 2, g + 8], tile[k + 3, g + 8]]
        assert dec == [int(v) for v in want], (n, lane)
