"""The C-ABI library without a GPU: it loads, exports every entry point include/exl3_b200.h declares, and the
seam's GPU-free calls (claims / validate / bill, plugins/turboexl3_ds41/config.zig:43-61 and its tests :66-86;
plugins/turboexl3_qwen38/config.zig:84-104 and :151-176) behave as the reference's."""
import ctypes
import json
import os
import re

import pytest

from plugins_b200 import _lib as L
from plugins_b200 import quant as Q

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared() -> set[str]:
    text = open(os.path.join(ROOT, "include", "exl3_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(exl3_[a-z_0-9]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    declared = _declared()
    assert declared == set(L.EXPORTS), declared ^ set(L.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.exl3_version()


DS41_BLOCK = {"quant_method": "exl3", "bits": 2.81, "codebook": "mul1"}


def test_claims_exl3_blocks_by_marker():
    assert Q.claims(DS41_BLOCK, {"model_type": "deepseek_v41"}) == Q.CLAIM_BY_MARKER
    assert Q.claims({"format": "exl3", "k": 4, "codebook": "mul1"}) == Q.CLAIM_BY_MARKER
    assert Q.claims({"quant_method": "fp8"}) == Q.CLAIM_NO
    assert Q.claims("{") == Q.CLAIM_NO
    assert Q.claims("[]") == Q.CLAIM_NO
    assert Q.claims("") == Q.CLAIM_NO


def test_validate_refuses_by_name():
    Q.validate(DS41_BLOCK)
    Q.validate({"format": "exl3", "codebook": "mul1", "window": 16, "k": 3})
    for cb in ("mcg", "3inst"):
        with pytest.raises(Q.Exl3Error) as e:
            Q.validate({"quant_method": "exl3", "codebook": cb})
        assert e.value.code == L.EXL3_UNSUPPORTED and "codebook is not mul1" in e.value.why
    with pytest.raises(Q.Exl3Error, match="Exl3WindowUnsupported"):
        Q.validate({"format": "exl3", "codebook": "mul1", "window": 20})
    Q.validate({"format": "exl3", "codebook": "mul1", "window": 12})  # narrowed windows 8..15 are served
    with pytest.raises(Q.Exl3Error, match="Exl3WindowUnsupported"):
        Q.validate({"format": "exl3", "codebook": "mul1", "window": 7})
    with pytest.raises(Q.Exl3Error, match="Exl3RateUnsupported"):
        Q.validate({"format": "exl3", "codebook": "mul1", "k": 9.25})
    Q.validate({"format": "exl3", "codebook": "mul1", "k": 2.5})  # half-bit rates are served (n = 40)
    for k in (2.25, 6.5):  # n = 36 (a quarter bit) and n = 104 (above 6 bits): admitted rates, not served
        with pytest.raises(Q.Exl3Error, match="half-bit grid"):
            Q.validate({"format": "exl3", "codebook": "mul1", "k": k})
    with pytest.raises(Q.Exl3Error, match="not an exllamav3 block"):
        Q.validate({"format": "gptq", "codebook": "mul1"})
    with pytest.raises(Q.Exl3Error, match="not a JSON object"):
        Q.validate("{")


def test_validate_on_the_reference_pack_configs():
    # turboexl3_qwen38/tests/fixtures/k{2,3,4,5}.json carry these trunk/expert blocks (integer K)
    for k in (2, 3, 4, 5):
        Q.validate({"format": "exl3", "codebook": "mul1", "window": 16,
                    "source": f"turboderp/Qwen3.8-Flash-Next-exl3@{k}.05bpw"})
        Q.validate({"format": "exl3", "k": k, "codebook": "mul1"})


def test_bill_is_the_stored_bytes():
    assert Q.bill(DS41_BLOCK, "/nowhere", 123456789) == 123456789
    assert Q.bill(DS41_BLOCK, "", 0) == 0


def test_moe_entry_refuses_by_name_without_a_gpu_call():
    v = L.lib().exl3_moe(None, None, None, None, 0, None, None)
    assert v.code == L.EXL3_UNSUPPORTED and b"swiglu" in v.why


def test_matmul_rejects_a_null_weight_before_any_launch():
    v = L.lib().exl3_matmul(ctypes.POINTER(L.Weight)(), None, None, None)
    assert v.code == L.EXL3_FAILED


def test_resident_keeps_nothing_and_refuses_a_bad_weight_without_a_gpu_call():
    # quant.zig:96-101: an empty list drops every kept matrix; a weight that is not loaded is refused before any
    # allocation
    got = ctypes.c_uint64(7)
    v = L.lib().exl3_resident(ctypes.POINTER(L.Weight)(), 0, 0, None, ctypes.byref(got))
    assert v.code == L.EXL3_OK and got.value == 0 and L.lib().exl3_resident_pending() == 0
    bad = L.Weight()
    v = L.lib().exl3_resident(ctypes.byref(bad), 1, 0, None, ctypes.byref(got))
    assert v.code == L.EXL3_FAILED and b"not a loaded weight" in v.why


def test_bench_counts_launches_with_the_librarys_gemv_selection():
    """bench.py's gpu_launches claim mirrors the library's decode-GEMV selection (exl3_abi.cu run_linear,
    exl3_gemv6.cu launch_gemv6): the thresholds and the in-CTA rotation limits it restates are the library's."""
    import importlib.util
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    hdr = open(os.path.join(root, "plugins_b200", "csrc", "exl3_internal.h")).read()
    g6 = open(os.path.join(root, "plugins_b200", "csrc", "exl3_gemv6.cu")).read()
    val = lambda src, name: int(re.search(r"constexpr int(?:64_t)? %s = (\d+);" % name, src).group(1))
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(root, "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    assert b.GEMV6_MIN_SLABS == val(hdr, "kGemv6MinSlabs")
    assert b.GEMV6_MIN_SLABS_DEEP == val(hdr, "kGemv6MinSlabsDeep")
    assert b.GEMV6_NARROW_CB == val(hdr, "kGemv6NarrowCb") and b.GEMV6_NARROW_SLABS == val(hdr, "kGemv6NarrowSlabs")
    assert val(g6, "kVirt6") == 3 and val(g6, "kMinRun6") == 32 and val(g6, "kXiRows") == 4
    assert b.XI_TAKE == val(g6, "kXiTake")
    assert val(g6, "kXiSlabs") - 8 == 128  # the longest run rotated in-CTA
    # config 2's launches at batch 1 and 8, one GPU: q|k|v, o, gate|up and down on the persistent GEMV (in-CTA
    # rotation at one row), the north-star 4096 x 12288 on the cluster split
    assert [b.gemv6_mode(i, o, False, 1) for i, o in ((4096, 6144), (4096, 4096), (4096, 24576), (12288, 4096))] == \
        [1, 1, 1, 1]
    assert b.gemv6_mode(4096, 12288, False, 1) == 0
    assert [b.gemv_kernels(i, o, False, 8) for i, o in ((4096, 24576), (12288, 4096))] == [2, 2]
    assert [b.gemv_kernels(4096, 4096, False, r) for r in (1, 2)] == [1, 2]
    # the column-parallel exchange takes its shard's kernel: config 2's gate|up shard at two GPUs on the cluster split
    # (a prepare launch from two rows), config 5's shard on the persistent GEMV
    assert [b.gemv_kernels(4096, 12288, True, r) for r in (1, 8)] == [1, 2]
    assert b.gemv6_mode(16384, 26624, True, 1) == 2 and b.gemv6_mode(4096, 12288, True, 1) == 0
    # the cluster split rotates in-CTA at one row, else takes the prepare launch
    abi = open(os.path.join(root, "plugins_b200", "csrc", "exl3_abi.cu")).read()
    assert b.CTA_ROTATE_ROWS == val(abi, "kCtaRotateRows")
    assert [b.gemv_kernels(4096, 12288, False, r) for r in (1, 2, 8)] == [1, 2, 2]


def test_timeline_reads_refuse_a_missing_exchange_without_a_gpu_call():
    lib = L.lib()
    buf = (ctypes.c_uint64 * 128)()
    for fn in (lib.exl3_tp_trace, lib.exl3_epx_trace, lib.exl3_cpx_trace):
        v = fn(None, buf)
        assert v.code == L.EXL3_FAILED and b"bad arguments" in v.why


def test_exchanges_refuse_bad_shapes_before_touching_the_gpu():
    """The multi-GPU exchanges validate their arguments before any CUDA call: refusals come back by name on a box
    without a GPU (exl3_tp.cu, exl3_epx.cu, exl3_moe.cu exl3_cpx_create)."""
    lib = L.lib()
    handle = (ctypes.c_uint8 * 64)()
    out = ctypes.c_void_p()
    cases = [
        (lib.exl3_tp_create, (0, 9, 0, 1, 16, 1), "1..8 ranks"),
        (lib.exl3_tp_create, (0, 2, 2, 1, 16, 1), "1..8 ranks"),
        (lib.exl3_tp_create, (0, 2, 0, 1, 24, 1), "slot_bytes a multiple of 16"),
        (lib.exl3_epx_create, (0, 0, 0, 8, 256, L.F16), "1..8 ranks"),
        (lib.exl3_epx_create, (0, 2, 0, 4, 200, L.F16), "hidden a multiple of 128"),
        (lib.exl3_epx_create, (0, 2, 0, 4, 256, L.I32), "an activation dtype"),
        (lib.exl3_cpx_create, (0, 9, 0, 4, 9, 4096, 2048, L.F16), "1..8 ranks"),
        (lib.exl3_cpx_create, (0, 8, 0, 8, 9, 4096, 2048, L.F16), "at most 512"),
        (lib.exl3_cpx_create, (0, 8, 0, 4, 9, 4096, 1536, L.F16), "128-column blocks per rank"),
        (lib.exl3_cpx_create, (0, 2, 0, 4, 9, 4096, 2048, L.I32), "an activation dtype"),
    ]
    for fn, args, why in cases:
        v = fn(*args, ctypes.byref(out), handle)
        assert v.code == L.EXL3_UNSUPPORTED and why in v.message(), (fn.__name__, args, v.message())
        assert not out.value
