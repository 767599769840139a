"""ctypes bindings for the CPU oracle (oracle/exl3_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker that tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs
compare the CUDA path against.  The product (plugins_b200/) never imports this module.

The C file restates the reference's scalar EXL3 path (plugins/sushi_ds41/src/sushi/exl3/expert_exl3.zig:259-566,
plugins/sushi_ds41/src/sushi/exl3/linear.zig:121-197, plugins/turboexl3_ds41/src/exl3/kernels.zig:964-1045); each C
function names the reference function it follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libexl3_oracle.so")
_lock = threading.Lock()
_lib = None

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u = ctypes.c_uint32


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no GPU needed); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_HERE, "exl3_oracle.c")):
                build()
            L = ctypes.CDLL(_SO)
            L.exl3o_f16_to_f32.restype = ctypes.c_float
            L.exl3o_f16_to_f32.argtypes = [ctypes.c_uint16]
            L.exl3o_f32_to_f16.restype = ctypes.c_uint16
            L.exl3o_f32_to_f16.argtypes = [ctypes.c_float]
            L.exl3o_f64_to_f16.restype = ctypes.c_uint16
            L.exl3o_f64_to_f16.argtypes = [ctypes.c_double]
            L.exl3o_bit_end.restype = _u
            L.exl3o_bit_end.argtypes = [_u, _u]
            L.exl3o_rate_admitted.restype = ctypes.c_int
            L.exl3o_rate_admitted.argtypes = [_u]
            for name in ("exl3o_decode_mul1", "exl3o_decode_mul1_f64", "exl3o_decode_mcg"):
                getattr(L, name).restype = ctypes.c_uint16
                getattr(L, name).argtypes = [ctypes.c_uint16]
            L.exl3o_mul1_table.argtypes = [_u16p]
            L.exl3o_unpack_tile.argtypes = [_u16p, _u, _u16p]
            L.exl3o_codeword_by_definition.restype = ctypes.c_uint16
            L.exl3o_codeword_by_definition.argtypes = [_u16p, _u, _u]
            L.exl3o_tensor_core_perm.argtypes = [_u32p]
            L.exl3o_decode_tile.argtypes = [_u16p, _u, _u, _u16p]
            L.exl3o_decode_tile_mcg.argtypes = [_u16p, _u, _u, _u16p]
            L.exl3o_hadamard128.argtypes = [_f32p]
            L.exl3o_reconstruct_inner.argtypes = [_u16p, _u, _u, _u, _u16p]
            L.exl3o_reconstruct_inner_w.argtypes = [_u16p, _u, _u, _u, _u, ctypes.c_int, _u16p]
            L.exl3o_reconstruct_states.argtypes = [_u16p, _u, _u, _u, _u16p, _u16p]
            L.exl3o_reconstruct_public.restype = ctypes.c_int
            L.exl3o_reconstruct_public.argtypes = [_u16p, _u16p, _u16p, _u, _u, _u, _u16p]
            L.exl3o_prepare_input.argtypes = [_f32p, _u16p, _u, _f32p]
            L.exl3o_inner_gemv.argtypes = [_u16p, _f32p, _u, _u, _u, _f32p]
            L.exl3o_finish_output.argtypes = [_f32p, _u16p, _u, _f32p]
            L.exl3o_project.restype = ctypes.c_int
            L.exl3o_project.argtypes = [_f32p, _u16p, _u16p, _u16p, _u, _u, _u, ctypes.c_int, _f32p]
            L.exl3o_host_project.restype = ctypes.c_int
            L.exl3o_host_project.argtypes = [_f32p, _u16p, _u16p, _u16p, _u, _u, _u, _u, ctypes.c_int, _f32p]
            L.exl3o_host_project_w.restype = ctypes.c_int
            L.exl3o_host_project_w.argtypes = [_f32p, _u16p, _u16p, _u16p, _u, _u, _u, _u, _u, ctypes.c_int, ctypes.c_int,
                                               _f32p]
            L.exl3o_moe_truth.restype = ctypes.c_int
            L.exl3o_moe_truth.argtypes = [_f32p, _i32p, _f32p, _u, _u,
                                          _u16p, _u16p, _u16p, _u, _u16p, _u16p, _u16p, _u, _u16p, _u16p, _u16p, _u,
                                          _u, _u, ctypes.c_float, ctypes.c_int, _f32p]
            L.exl3o_moe_truth_w.restype = ctypes.c_int
            L.exl3o_moe_truth_w.argtypes = [_f32p, _i32p, _f32p, _u, _u,
                                            _u16p, _u16p, _u16p, _u, _u16p, _u16p, _u16p, _u, _u16p, _u16p, _u16p, _u,
                                            _u, _u, ctypes.c_int, ctypes.c_int, _u, _u, ctypes.c_float, ctypes.c_int, _f32p]
            L.exl3o_splitmix64.restype = ctypes.c_uint64
            L.exl3o_splitmix64.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
            L.exl3o_synth_plane.argtypes = [ctypes.c_uint64, ctypes.c_size_t, _u16p]
            L.exl3o_init()
            _lib = L
    return _lib


def _cb(codebook: str) -> int:
    if codebook not in ("mul1", "mcg"):
        raise ValueError(codebook)
    return 1 if codebook == "mcg" else 0


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def f16_to_f32(h: int) -> float:
    return lib().exl3o_f16_to_f32(h)


def f32_to_f16(f: float) -> int:
    return lib().exl3o_f32_to_f16(f)


def decode_mul1(cw: int) -> int:
    return lib().exl3o_decode_mul1(cw)


def decode_mul1_f64(cw: int) -> int:
    return lib().exl3o_decode_mul1_f64(cw)


def decode_mcg(cw: int) -> int:
    return lib().exl3o_decode_mcg(cw)


def bit_end(n: int, t: int) -> int:
    return lib().exl3o_bit_end(n, t)


def rate_admitted(n: int) -> bool:
    return bool(lib().exl3o_rate_admitted(n))


def mul1_table() -> np.ndarray:
    out = np.empty(65536, np.uint16)
    lib().exl3o_mul1_table(out)
    return out


def tensor_core_perm() -> np.ndarray:
    out = np.empty(256, np.uint32)
    lib().exl3o_tensor_core_perm(out)
    return out


def unpack_tile(words, n: int) -> np.ndarray:
    out = np.empty(256, np.uint16)
    lib().exl3o_unpack_tile(_c(words, np.uint16), n, out)
    return out


def codeword_by_definition(words, n: int, slot: int) -> int:
    return lib().exl3o_codeword_by_definition(_c(words, np.uint16), n, slot)


def decode_tile(words, n: int, window: int = 16, codebook: str = "mul1") -> np.ndarray:
    out = np.empty(256, np.uint16)
    fn = lib().exl3o_decode_tile if codebook == "mul1" else lib().exl3o_decode_tile_mcg
    fn(_c(words, np.uint16), n, window, out)
    return out


def hadamard128(v) -> np.ndarray:
    a = _c(v, np.float32).copy()
    lib().exl3o_hadamard128(a)
    return a


def reconstruct_inner(trellis, in_features: int, out_features: int, n: int, window: int = 16,
                      codebook: str = "mul1") -> np.ndarray:
    """W_hat as f16 bits, row-major [in, out]; ``window`` the codeword window in bits (8..16), ``codebook`` mul1 or
    mcg."""
    out = np.empty(in_features * out_features, np.uint16)
    lib().exl3o_reconstruct_inner_w(_c(trellis, np.uint16).reshape(-1), in_features, out_features, n, window,
                                    _cb(codebook), out)
    return out.reshape(in_features, out_features)


def reconstruct_states(trellis, in_features: int, out_features: int, n: int):
    w = np.empty(in_features * out_features, np.uint16)
    st = np.empty(in_features * out_features, np.uint16)
    lib().exl3o_reconstruct_states(_c(trellis, np.uint16).reshape(-1), in_features, out_features, n, w, st)
    return w.reshape(in_features, out_features), st.reshape(in_features, out_features)


def reconstruct_public(trellis, suh, svh, in_features: int, out_features: int, n: int) -> np.ndarray:
    out = np.empty(in_features * out_features, np.uint16)
    rc = lib().exl3o_reconstruct_public(_c(trellis, np.uint16).reshape(-1), _c(suh, np.uint16), _c(svh, np.uint16),
                                        in_features, out_features, n, out)
    if rc != 0:
        raise MemoryError("exl3o_reconstruct_public")
    return out.reshape(in_features, out_features)


def project(x, trellis, suh, svh, in_features: int, out_features: int, n: int, threads: int = 1) -> np.ndarray:
    """The reference's scalar linear (project(), f16 roundings included) for one row x [in] -> y [out] f32."""
    out = np.empty(out_features, np.float32)
    rc = lib().exl3o_project(_c(x, np.float32).reshape(-1), _c(trellis, np.uint16).reshape(-1), _c(suh, np.uint16),
                             _c(svh, np.uint16), in_features, out_features, n, threads, out)
    if rc != 0:
        raise MemoryError("exl3o_project")
    return out


def host_project(x, trellis, suh, svh, in_features: int, out_features: int, n: int, threads: int = 1,
                 window: int = 16, codebook: str = "mul1") -> np.ndarray:
    """The f32 truth (Host.project): x [rows, in] -> y [rows, out] f32, no intermediate f16 rounding; ``window``
    the codeword window in bits (8..16)."""
    x2 = _c(x, np.float32).reshape(-1, in_features)
    rows = x2.shape[0]
    out = np.empty(rows * out_features, np.float32)
    rc = lib().exl3o_host_project_w(x2.reshape(-1), _c(trellis, np.uint16).reshape(-1), _c(suh, np.uint16).reshape(-1),
                                    _c(svh, np.uint16).reshape(-1), rows, in_features, out_features, n, window,
                                    _cb(codebook), threads, out)
    if rc != 0:
        raise MemoryError("exl3o_host_project")
    return out.reshape(rows, out_features)


def moe_truth(x, inds, scores, gate, up, down, hidden: int, inter: int, limit: float = 0.0, threads: int = 1,
              windows=(16, 16), codebooks=("mul1", "mul1")):
    """Routed SwiGLU f32 truth.  gate/up/down = (trellis [E, ...], suh [E, in], svh [E, out], n); ``windows`` the
    codeword windows of gate|up and of down (8..16 bits)."""
    x2 = _c(x, np.float32).reshape(-1, hidden)
    rows = x2.shape[0]
    inds2 = _c(inds, np.int32).reshape(rows, -1)
    topk = inds2.shape[1]
    sc = _c(scores, np.float32).reshape(rows, topk)
    y = np.empty(rows * hidden, np.float32)
    args = []
    for tr, su, sv, n in (gate, up, down):
        args += [_c(tr, np.uint16).reshape(-1), _c(su, np.uint16).reshape(-1), _c(sv, np.uint16).reshape(-1), n]
    rc = lib().exl3o_moe_truth_w(x2.reshape(-1), inds2.reshape(-1), sc.reshape(-1), rows, topk, *args,
                                 int(windows[0]), int(windows[1]), _cb(codebooks[0]), _cb(codebooks[1]), hidden, inter,
                                 float(limit), threads, y)
    if rc != 0:
        raise MemoryError("exl3o_moe_truth")
    return y.reshape(rows, hidden)


def splitmix64_seq(seed: int, count: int) -> list[int]:
    s = ctypes.c_uint64(seed)
    return [lib().exl3o_splitmix64(ctypes.byref(s)) for _ in range(count)]


def synth_plane(seed: int, in_dim: int, out_dim: int, k: int) -> np.ndarray:
    """A golden plane's seeded trellis (TX/kernels.zig:1035-1045): u16 [in/16, out/16, 16k]."""
    count = (in_dim // 16) * (out_dim // 16) * 16 * k
    out = np.empty(count, np.uint16)
    lib().exl3o_synth_plane(seed, count, out)
    return out.reshape(in_dim // 16, out_dim // 16, 16 * k)
