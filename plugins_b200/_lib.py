"""ctypes binding of libexl3b200.so (include/exl3_b200.h).

The library is built in-tree (``python -m plugins_b200.build``) and loaded from this package directory; there is no
other implementation to fall back to, so a missing library is an error.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libexl3b200.so")

EXL3_OK, EXL3_UNSUPPORTED, EXL3_FAILED, EXL3_TOO_LARGE = 0, 1, 2, 3
CLAIM_NO, CLAIM_BY_MODE, CLAIM_BY_MARKER = 0, 1, 2
F16, BF16, F32, I32, U32, U16, I16 = 0, 1, 2, 3, 4, 5, 6

WEIGHT_OWNED, WEIGHT_BANK, WEIGHT_GROUPED = 1, 2, 4
WEIGHT_WINDOW_SHIFT, WEIGHT_WINDOW_MASK = 8, 0xF00
WEIGHT_MCG = 16


def weight_window(bits: int) -> int:
    """EXL3_WEIGHT_WINDOW(bits): a narrowed codeword window (8..16 bits) as weight flags."""
    return ((16 - int(bits)) << WEIGHT_WINDOW_SHIFT) & WEIGHT_WINDOW_MASK
MATMUL_PREPARED, MATMUL_INNER, MATMUL_DP4A, MATMUL_GEMV, MATMUL_GEMM = 1, 2, 4, 8, 16
MAX_SEGMENTS = 4
ERR_WAIT_TIMEOUT, ERR_BAD_SHAPE, ERR_EP_OVERFLOW, ERR_TP_TIMEOUT, ERR_EP_TIMEOUT = 1, 2, 4, 8, 16

# every symbol include/exl3_b200.h declares
EXPORTS = (
    "exl3_claims", "exl3_validate", "exl3_bill", "exl3_open", "exl3_close", "exl3_load_tensor", "exl3_load_bank",
    "exl3_release", "exl3_matmul", "exl3_moe", "exl3_swiglu", "exl3_swiglu_shared", "exl3_moe_prefill_reserve", "exl3_matmul_ex", "exl3_matmul_timed",
    "exl3_ep_dispatch", "exl3_ep_unpack", "exl3_ep_combine", "exl3_epx_create", "exl3_epx_connect",
    "exl3_epx_destroy", "exl3_epx_dispatch", "exl3_epx_receive", "exl3_epx_return", "exl3_epx_combine",
    "exl3_cpx_create", "exl3_cpx_connect", "exl3_cpx_destroy", "exl3_swiglu_cp",
    "exl3_tp_create", "exl3_tp_connect", "exl3_tp_destroy", "exl3_tp_begin", "exl3_matmul_tp", "exl3_tp_gather",
    "exl3_tp_trace", "exl3_epx_trace", "exl3_cpx_trace",
    "exl3_weight_view", "exl3_weight_stack",
    "exl3_decode_dense", "exl3_reconstruct_public", "exl3_encode_trellis", "exl3_matmul_noalloc", "exl3_device_error", "exl3_version",
    "exl3_model_claims", "exl3_model_parse", "exl3_model_bill", "exl3_model_load", "exl3_model_unload",
    "exl3_model_weight", "exl3_model_linear", "exl3_model_linears", "exl3_model_mlp", "exl3_model_experts", "exl3_resident", "exl3_resident_pending",
)


class ModelConfig(ctypes.Structure):
    """exl3_model_config: the model seam's parsed keys (include/exl3_b200.h)."""
    _fields_ = [("size", ctypes.c_uint32), ("hidden_size", ctypes.c_uint32), ("intermediate_size", ctypes.c_uint32),
                ("num_hidden_layers", ctypes.c_uint32), ("num_attention_heads", ctypes.c_uint32),
                ("num_key_value_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("num_experts", ctypes.c_uint32), ("num_experts_per_tok", ctypes.c_uint32),
                ("moe_intermediate_size", ctypes.c_uint32), ("shared_expert_intermediate_size", ctypes.c_uint32),
                ("expert_rate_n", ctypes.c_uint32), ("weight_prefix", ctypes.c_char * 96)]


class Str(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_char_p), ("len", ctypes.c_size_t)]

    @classmethod
    def of(cls, s: str | bytes) -> "Str":
        b = s.encode() if isinstance(s, str) else bytes(s)
        o = cls(b, len(b))
        o._keep = b  # keep the bytes alive with the struct
        return o


class Verdict(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("why", ctypes.c_char_p)]

    @property
    def ok(self) -> bool:
        return self.code == EXL3_OK

    def message(self) -> str:
        return self.why.decode() if self.why else ""


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 4)]


class HostTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 4)]


TensorFn = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, Str, ctypes.POINTER(HostTensor))


class Source(ctypes.Structure):
    _fields_ = [("ctx", ctypes.c_void_p), ("tensor", TensorFn)]


class LoadCtx(ctypes.Structure):
    _fields_ = [("size", ctypes.c_uint32), ("block_json", Str), ("config_json", Str), ("model_dir", Str),
                ("source", Source), ("device", ctypes.c_int32), ("stream", ctypes.c_void_p)]


class Weight(ctypes.Structure):
    _fields_ = [("size", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("trellis", ctypes.c_void_p),
                ("suh", ctypes.c_void_p), ("svh", ctypes.c_void_p), ("groups", ctypes.c_int32),
                ("in_features", ctypes.c_int32), ("out_features", ctypes.c_int32), ("n", ctypes.c_int32),
                ("device", ctypes.c_int32), ("nseg", ctypes.c_int32), ("seg_cols", ctypes.c_int32 * (MAX_SEGMENTS + 1))]


class SwigluOpts(ctypes.Structure):
    _fields_ = [("size", ctypes.c_uint32), ("limit", ctypes.c_int32), ("verify_rows", ctypes.c_int32)]


class SharedSwiglu(ctypes.Structure):
    """exl3_shared_swiglu: the shared expert's linears (or its output), its gate and the sigmoid table."""
    _fields_ = [("size", ctypes.c_uint32), ("limit", ctypes.c_int32), ("gate", ctypes.c_void_p),
                ("up", ctypes.c_void_p), ("down", ctypes.c_void_p), ("shared", ctypes.c_void_p),
                ("logit", ctypes.c_void_p), ("gate_vec", ctypes.c_void_p), ("sigtab", ctypes.c_void_p)]


_lock = threading.Lock()
_lib = None


class Exl3Error(RuntimeError):
    """A refusal or failure verdict from the library: `.code` and the library's message."""

    def __init__(self, code: int, why: str):
        super().__init__(why)
        self.code = code
        self.why = why


def check(v: Verdict) -> None:
    if v.code != EXL3_OK:
        raise Exl3Error(v.code, v.message())


def lib() -> ctypes.CDLL:
    """The loaded libexl3b200.so.  Raises if it was not built -- there is no CPU or eager fallback."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m plugins_b200.build` "
                                   "(the EXL3 path has no fallback)")
            L = ctypes.CDLL(LIB_PATH)
            P = ctypes.POINTER
            L.exl3_claims.restype = ctypes.c_int32
            L.exl3_claims.argtypes = [Str, Str]
            L.exl3_validate.restype = Verdict
            L.exl3_validate.argtypes = [Str, Str]
            L.exl3_bill.restype = ctypes.c_uint64
            L.exl3_bill.argtypes = [Str, Str, ctypes.c_uint64]
            L.exl3_open.restype = Verdict
            L.exl3_open.argtypes = [P(LoadCtx)]
            L.exl3_close.restype = None
            L.exl3_close.argtypes = [P(LoadCtx)]
            for f in (L.exl3_load_tensor, L.exl3_load_bank):
                f.restype = Verdict
                f.argtypes = [P(LoadCtx), Str, ctypes.c_uint32, P(Weight)]
            L.exl3_release.restype = None
            L.exl3_release.argtypes = [P(Weight)]
            L.exl3_matmul.restype = Verdict
            L.exl3_matmul.argtypes = [P(Weight), P(Tensor), ctypes.c_void_p, P(Tensor)]
            L.exl3_matmul_ex.restype = Verdict
            L.exl3_matmul_ex.argtypes = [P(Weight), P(Tensor), ctypes.c_uint32, ctypes.c_void_p, P(Tensor)]
            L.exl3_tp_create.restype = Verdict
            L.exl3_tp_create.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                         ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
            L.exl3_tp_connect.restype = Verdict
            L.exl3_tp_connect.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
            L.exl3_tp_destroy.restype = None
            L.exl3_tp_destroy.argtypes = [ctypes.c_void_p]
            L.exl3_tp_begin.restype = Verdict
            L.exl3_tp_begin.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
            L.exl3_matmul_tp.restype = Verdict
            L.exl3_matmul_tp.argtypes = [P(Weight), P(Tensor), ctypes.c_void_p, ctypes.c_int32,
                                         ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p]
            L.exl3_tp_gather.restype = Verdict
            L.exl3_tp_gather.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
            for name in ("exl3_tp_trace", "exl3_epx_trace", "exl3_cpx_trace"):
                getattr(L, name).restype = Verdict
                getattr(L, name).argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]
            L.exl3_ep_dispatch.restype = Verdict
            L.exl3_ep_dispatch.argtypes = [P(Tensor), P(Tensor), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_void_p, P(Tensor), P(Tensor)]
            L.exl3_ep_unpack.restype = Verdict
            L.exl3_ep_unpack.argtypes = [P(Tensor), ctypes.c_void_p, P(Tensor), P(Tensor)]
            L.exl3_ep_combine.restype = Verdict
            L.exl3_ep_combine.argtypes = [P(Tensor), P(Tensor), P(Tensor), P(Tensor), ctypes.c_void_p, P(Tensor)]
            L.exl3_model_claims.restype = ctypes.c_int
            L.exl3_model_claims.argtypes = [Str, Str]
            L.exl3_model_parse.restype = Verdict
            L.exl3_model_parse.argtypes = [Str, P(ModelConfig)]
            L.exl3_epx_create.restype = Verdict
            L.exl3_epx_create.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p),
                                          ctypes.c_void_p]
            L.exl3_epx_connect.restype = Verdict
            L.exl3_epx_connect.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
            L.exl3_epx_destroy.restype = None
            L.exl3_epx_destroy.argtypes = [ctypes.c_void_p]
            L.exl3_epx_dispatch.restype = Verdict
            L.exl3_epx_dispatch.argtypes = [ctypes.c_void_p, P(Tensor), P(Tensor), ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_void_p, P(Tensor)]
            L.exl3_epx_receive.restype = Verdict
            L.exl3_epx_receive.argtypes = [ctypes.c_void_p, ctypes.c_void_p, P(Tensor), P(Tensor), P(Tensor)]
            L.exl3_epx_return.restype = Verdict
            L.exl3_epx_return.argtypes = [ctypes.c_void_p, P(Tensor), ctypes.c_void_p]
            L.exl3_epx_combine.restype = Verdict
            L.exl3_epx_combine.argtypes = [ctypes.c_void_p, P(Tensor), P(Tensor), ctypes.c_void_p, P(Tensor)]
            L.exl3_cpx_create.restype = Verdict
            L.exl3_cpx_create.argtypes = [ctypes.c_int32] * 8 + [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
            L.exl3_cpx_connect.restype = Verdict
            L.exl3_cpx_connect.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
            L.exl3_cpx_destroy.restype = None
            L.exl3_cpx_destroy.argtypes = [ctypes.c_void_p]
            L.exl3_swiglu_cp.restype = Verdict
            L.exl3_swiglu_cp.argtypes = [ctypes.c_void_p, P(Weight), P(Weight), P(Weight), P(Tensor), P(Tensor),
                                         P(Tensor), ctypes.c_void_p, ctypes.c_void_p, P(Tensor)]
            L.exl3_matmul_timed.restype = Verdict
            L.exl3_matmul_timed.argtypes = [P(Weight), P(Tensor), ctypes.c_uint32, ctypes.c_void_p, P(Tensor),
                                            ctypes.POINTER(ctypes.c_void_p)]
            L.exl3_moe.restype = Verdict
            L.exl3_moe.argtypes = [P(Weight), P(Tensor), P(Tensor), P(Tensor), ctypes.c_int32, ctypes.c_void_p,
                                   P(Tensor)]
            L.exl3_swiglu.restype = Verdict
            L.exl3_swiglu.argtypes = [P(Weight), P(Weight), P(Weight), P(Tensor), P(Tensor), P(Tensor),
                                      P(SwigluOpts), ctypes.c_void_p, P(Tensor)]
            L.exl3_model_bill.restype = ctypes.c_uint64
            L.exl3_model_bill.argtypes = [Str, P(Source), ctypes.c_void_p, ctypes.c_int32]
            L.exl3_model_load.restype = Verdict
            L.exl3_model_load.argtypes = [Str, P(Source), ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_void_p, P(ctypes.c_void_p)]
            L.exl3_model_unload.restype = None
            L.exl3_model_unload.argtypes = [ctypes.c_void_p]
            L.exl3_model_weight.restype = ctypes.c_int32
            L.exl3_model_weight.argtypes = [ctypes.c_void_p, ctypes.c_int32, Str, P(Weight)]
            L.exl3_model_linear.restype = Verdict
            L.exl3_model_linear.argtypes = [ctypes.c_void_p, ctypes.c_int32, Str, P(Tensor), ctypes.c_void_p,
                                            P(Tensor)]
            L.exl3_model_linears.restype = Verdict
            L.exl3_model_linears.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32,
                                             P(Tensor), ctypes.c_void_p, P(Tensor)]
            L.exl3_model_mlp.restype = Verdict
            L.exl3_model_mlp.argtypes = [ctypes.c_void_p, ctypes.c_int32, Str, P(Tensor), ctypes.c_void_p, P(Tensor)]
            L.exl3_model_experts.restype = Verdict
            L.exl3_model_experts.argtypes = [ctypes.c_void_p, ctypes.c_int32, Str, Str, P(Tensor), P(Tensor),
                                             P(Tensor), ctypes.c_void_p, ctypes.c_void_p, P(Tensor)]
            L.exl3_moe_prefill_reserve.restype = Verdict
            L.exl3_moe_prefill_reserve.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                   ctypes.c_int32, P(ctypes.c_uint64)]
            L.exl3_swiglu_shared.restype = Verdict
            L.exl3_swiglu_shared.argtypes = [P(Weight), P(Weight), P(Weight), P(Tensor), P(Tensor), P(Tensor),
                                             P(SharedSwiglu), ctypes.c_void_p, P(Tensor)]
            L.exl3_weight_view.restype = Verdict
            L.exl3_weight_view.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, P(Weight)]
            L.exl3_weight_stack.restype = Verdict
            L.exl3_weight_stack.argtypes = [P(Weight), ctypes.c_int32, ctypes.c_void_p, P(Weight)]
            L.exl3_decode_dense.restype = Verdict
            L.exl3_decode_dense.argtypes = [P(Weight), ctypes.c_int32, ctypes.c_void_p, ctypes.c_uint32,
                                            ctypes.c_void_p]
            L.exl3_reconstruct_public.restype = Verdict
            L.exl3_reconstruct_public.argtypes = [P(Weight), ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
            L.exl3_encode_trellis.restype = Verdict
            L.exl3_encode_trellis.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_void_p, ctypes.c_void_p]
            L.exl3_matmul_noalloc.restype = Verdict
            L.exl3_matmul_noalloc.argtypes = [P(Weight), P(Tensor), ctypes.c_void_p, P(Tensor)]
            L.exl3_device_error.restype = Verdict
            L.exl3_device_error.argtypes = [ctypes.c_int32, P(ctypes.c_uint32), ctypes.c_int32]
            L.exl3_resident.restype = Verdict
            L.exl3_resident.argtypes = [P(Weight), ctypes.c_int32, ctypes.c_uint64, ctypes.c_void_p, P(ctypes.c_uint64)]
            L.exl3_resident_pending.restype = ctypes.c_uint64
            L.exl3_resident_pending.argtypes = []
            L.exl3_version.restype = ctypes.c_char_p
            L.exl3_version.argtypes = []
            _lib = L
    return _lib
