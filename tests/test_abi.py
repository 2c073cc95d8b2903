"""The C-ABI boundary (CPU only: nothing here launches a kernel).

* libmlkb200.so loads and exports every symbol include/mlkb200.h declares;
* the module wire format written by mlk2_b200.kir is the document the
  reference's KernelModule::toJson produces, and the shim classifies it the
  way the reference executor dispatches it;
* malformed or out-of-scope modules are rejected with the documented codes.
"""
import ctypes as C
import json
import os
import re

import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "mlkb200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:int|void|const char\s*\*)\s*(\w+)\s*\(", text, re.M)


def test_library_exports_every_declared_symbol():
    L = mb.lib()
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(L, s)]
    assert missing == []
    assert "sm_100a" in mb.version()


def test_library_is_sm100a_only():
    # every CUDA translation unit is compiled for sm_100a and nothing else
    mk = open(os.path.join(ROOT, "mlk2_b200", "csrc", "Makefile")).read()
    assert "arch=compute_100a,code=sm_100a" in mk
    assert re.search(r"sm_(?!100a)\d+", mk) is None


def _ref_json(kind, **kw):
    lib = oracle.ref().lib
    buf = C.create_string_buffer(1 << 16)
    if kind == mb.KIND_MAP:
        chains = kw["chains"]
        allx = np.ascontiguousarray(np.concatenate(chains), dtype=kir.EXPR_DTYPE)
        lens = (C.c_int32 * len(chains))(*[len(c) for c in chains])
        rc = lib.mlkref_module_json(kind, len(chains), lens, C.c_void_p(allx.ctypes.data),
                                    kw.get("n_inputs", 1), 0, C.c_int64(0), C.c_int64(0),
                                    C.c_int64(0), buf, C.c_int64(len(buf)))
    else:
        rc = lib.mlkref_module_json(kind, 0, None, None, 0, 0, C.c_int64(kw["m"]),
                                    C.c_int64(kw["k"]), C.c_int64(kw.get("n", 0)), buf,
                                    C.c_int64(len(buf)))
    assert rc == 0
    return json.loads(buf.value.decode())


@needs_ref
@pytest.mark.parametrize("case", ["sin", "sin_dsin", "two_input", "softmax", "matmul", "reducesum"])
def test_wire_format_matches_reference_tojson(case):
    if case == "sin":
        ref, ours = _ref_json(mb.KIND_MAP, chains=[kir.SIN_CHAIN]), kir.map_module([kir.SIN_CHAIN])
    elif case == "sin_dsin":
        chains = [kir.SIN_CHAIN, kir.DSIN_CHAIN]
        ref, ours = _ref_json(mb.KIND_MAP, chains=chains), kir.map_module(chains)
    elif case == "two_input":
        ch = [kir.chain(kir.E("mul", kir.A, kir.B), kir.E("exp", kir.T(0)))]
        ref, ours = _ref_json(mb.KIND_MAP, chains=ch, n_inputs=2), kir.map_module(ch, n_inputs=2)
    elif case == "softmax":
        ref, ours = _ref_json(mb.KIND_SOFTMAX, m=7, k=9), kir.call_module("softmax", 7, 9)
    elif case == "matmul":
        ref, ours = _ref_json(mb.KIND_MATMUL, m=4, k=5, n=6), kir.call_module("matmul", 4, 5, 6)
    else:
        ref, ours = _ref_json(mb.KIND_REDUCESUM, m=3, k=8), kir.call_module("reducesum", 3, 8)
    assert ours == ref


@pytest.mark.parametrize("module,kind", [
    (kir.map_module([kir.SIN_CHAIN]), mb.KIND_MAP),
    (kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]), mb.KIND_MAP),
    (kir.call_module("softmax", 65536, 4096), mb.KIND_SOFTMAX),
    (kir.call_module("matmul", 8192, 8192, 8192, ("f16", "f16", "f32")), mb.KIND_MATMUL),
    (kir.call_module("reducesum", 10, 20), mb.KIND_REDUCESUM),
    (kir.qk_softmax_module(2048, 128, 128 ** -0.5), mb.KIND_QK_SOFTMAX),
])
def test_module_classification(module, kind):
    m = api.Module(module)
    assert m.kind == kind
    assert m.num_buffers == sum(1 for b in module["buffers"] if b["input"] or b["output"])


@needs_ref
def test_reference_json_parses_to_same_kind():
    for kind, kw in [(mb.KIND_MAP, {"chains": [kir.SIN_CHAIN, kir.DSIN_CHAIN]}),
                     (mb.KIND_SOFTMAX, {"m": 5, "k": 3}),
                     (mb.KIND_MATMUL, {"m": 4, "k": 5, "n": 6}),
                     (mb.KIND_REDUCESUM, {"m": 4, "k": 5})]:
        assert api.Module(json.dumps(_ref_json(kind, **kw))).kind == kind


def _status_of_create(text):
    h = C.c_void_p()
    rc = mb.lib().mlkb_module_create(text.encode(), C.byref(h))
    if h:
        mb.lib().mlkb_module_destroy(h)
    return rc


def test_rejections():
    assert _status_of_create("{not json") == mb.ERR_INVALID
    assert _status_of_create('{"format":"other","buffers":[],"nodes":[]}') == mb.ERR_INVALID
    # accumulate stores belong to poly-scheduled multi-dim nests: not this path
    m = kir.map_module([kir.SIN_CHAIN])
    m["nodes"][2]["accumulate"] = True
    m["nodes"][2]["out_index_coeffs"] = [1]
    assert _status_of_create(kir.dumps(m)) == mb.ERR_UNSUPPORTED
    # a temp operand that is not an earlier expression
    bad = kir.map_module([kir.chain(kir.E("exp", kir.T(0)))])
    assert _status_of_create(kir.dumps(bad)) == mb.ERR_UNSUPPORTED
    # shape mismatch is the reference's InvalidGraph analogue
    mm = kir.call_module("matmul", 4, 5, 6)
    mm["buffers"][1]["dims"] = [7, 6]
    assert _status_of_create(kir.dumps(mm)) == mb.ERR_INVALID


def test_shape_limits():
    # empty or negative GEMM extents, an extent past 2^31 and a buffer past
    # 2^40 elements are rejected before any size is computed from them
    for m, k, n in [(0, 5, 6), (4, 0, 6), (4, 5, 0), (-4, 5, 6)]:
        mm = kir.call_module("matmul", 4, 5, 6)
        mm["buffers"][0]["dims"] = [m, k]
        mm["buffers"][1]["dims"] = [k, n]
        mm["buffers"][2]["dims"] = [m, n]
        assert _status_of_create(kir.dumps(mm)) == mb.ERR_INVALID, (m, k, n)
    big = kir.call_module("softmax", 4, 5)
    big["buffers"][0]["dims"] = [2**31, 5]
    assert _status_of_create(kir.dumps(big)) == mb.ERR_INVALID
    huge = kir.call_module("matmul", 2**21, 2**21, 2**21)
    assert _status_of_create(kir.dumps(huge)) == mb.ERR_INVALID   # 2^42 elements each
    qk = kir.qk_softmax_module(256, 64, 0.125)
    assert _status_of_create(kir.dumps(qk)) == mb.OK
    qk["buffers"][0]["dims"] = [0, 64]
    qk["buffers"][1]["dims"] = [64, 0]
    assert _status_of_create(kir.dumps(qk)) != mb.OK


def test_mlk_kernel_without_binding_reports_not_bound():
    L = mb.lib()
    assert L.mlk_bind_module(None) == 0
    x = np.zeros(4)
    L.mlk_kernel(*([x.ctypes.data, x.ctypes.data, 4, 0, 0] + [0] * 13))
    assert L.mlk_last_status() == mb.ERR_NOT_BOUND


@pytest.mark.skipif(mb.lib().mlkb_device_count() > 0, reason="host without a GPU only")
def test_no_device_is_reported_not_faked():
    # Without a GPU every compute entry fails loudly with code 4 (reference
    # ABI: "no CUDA device"); nothing falls back to the CPU.
    x = np.linspace(-1, 1, 16)
    y = np.zeros(16)
    status = api.legacy_call(kir.map_module([kir.SIN_CHAIN], dtype="f64"), [x, y], 16)
    assert status == mb.ERR_NO_DEVICE
    assert np.all(y == 0)
    with pytest.raises(mb.MLKBError):
        api.Module(kir.map_module([kir.SIN_CHAIN])).run_host(
            [x.astype(np.float32), y.astype(np.float32)], n=16)


def _run_host_status(module, bufs, n):
    ptrs = (C.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs])
    dts = (C.c_int32 * len(bufs))(*[api._dt_of(b) for b in bufs])
    sc = (C.c_double * 1)(0.0)
    return mb.lib().mlkb_module_run_host(module._h, ptrs, dts, len(bufs), n, sc, 0, 1)


def test_qk_composite_forms():
    # S and Sc outputs: the reference's three steps; temps: the fused kernel
    out = api.Module(kir.qk_softmax_module(256, 64, 0.125))
    assert out.kind == mb.KIND_QK_SOFTMAX and out.num_buffers == 5
    assert out.plan([mb.F16, mb.F16, mb.F32, mb.F32, mb.F32]) == \
        "gemm_f16_tcgen05,map_chain,softmax_f32"
    assert out.plan([mb.F64] * 5) == "gemm_f64,map_chain,softmax_f64"
    tmp = api.Module(kir.qk_softmax_module(256, 64, 0.125, temps=True))
    assert tmp.kind == mb.KIND_QK_SOFTMAX and tmp.num_buffers == 3
    assert tmp.plan([mb.F16, mb.F16, mb.F32]) == "qk_softmax_tcgen05_kt"
    # one temp and one output intermediate: not a form this path runs
    mixed = kir.qk_softmax_module(256, 64, 0.125)
    mixed["buffers"][2]["output"] = False
    mixed["buffers"][2]["temp"] = True
    assert _status_of_create(kir.dumps(mixed)) == mb.ERR_UNSUPPORTED


def test_qk_composite_run_requests_checked_before_any_device_work():
    # These statuses come from the host-side checks, so they hold on a host
    # without a GPU too: a run never returns OK for work it did not do.
    s, d = 128, 64
    q = np.zeros((s, d), np.float16)
    kt = np.zeros((d, s), np.float16)
    y = np.zeros((s, s), np.float32)
    tmp = api.Module(kir.qk_softmax_module(s, d, 0.125, temps=True))
    # temp scores need the scale map over all of S: n = s*s
    assert _run_host_status(tmp, [q, kt, y], s * s - 1) == mb.ERR_UNSUPPORTED
    # the fused form is f16 in, f32 out
    assert _run_host_status(tmp, [q.astype(np.float64), kt.astype(np.float64),
                                  y.astype(np.float64)], s * s) == mb.ERR_UNSUPPORTED
    out = api.Module(kir.qk_softmax_module(s, d, 0.125))
    sf = np.zeros((s, s), np.float32)
    assert _run_host_status(out, [q, kt, sf, sf.astype(np.float64), y], s * s) == mb.ERR_INVALID
    # a scale map running past S is the reference's out-of-range store
    assert _run_host_status(out, [q, kt, sf, sf.copy(), y], s * s + 1) == mb.ERR_INVALID


def test_failed_bind_leaves_nothing_bound():
    # mlk_kernel must never run the previously bound module after a bind fails
    L = mb.lib()
    assert L.mlk_bind_module(kir.dumps(kir.map_module([kir.SIN_CHAIN], dtype="f64")).encode()) == 0
    bad = kir.map_module([kir.SIN_CHAIN])
    bad["nodes"][2]["accumulate"] = True
    assert L.mlk_bind_module(kir.dumps(bad).encode()) == mb.ERR_UNSUPPORTED
    x = np.zeros(4)
    L.mlk_kernel(*([x.ctypes.data, x.ctypes.data, 4, 0, 0] + [0] * 13))
    assert L.mlk_last_status() == mb.ERR_UNSUPPORTED
    assert L.mlk_bind_module(None) == 0


def test_mlk_kernel_rejects_a_negative_scalar_count():
    # the reference reads any scalar index below the table size
    # (kernel_buffers.cpp:114-117): tables of any size are accepted, a
    # negative count is an error, and nothing is silently zeroed
    L = mb.lib()
    assert L.mlk_bind_module(kir.dumps(kir.map_module([kir.SIN_CHAIN], dtype="f64")).encode()) == 0
    x, y = np.zeros(4), np.zeros(4)
    sc = np.zeros(1)
    L.mlk_kernel(*([x.ctypes.data, y.ctypes.data, 4, sc.ctypes.data, -1] + [0] * 13))
    assert L.mlk_last_status() == mb.ERR_INVALID
    assert L.mlk_bind_module(None) == 0


def test_map_dtype_mismatch_checked_on_the_host():
    m = api.Module(kir.map_module([kir.SIN_CHAIN]))
    x = np.zeros(8, np.float32)
    assert _run_host_status(m, [x, np.zeros(8, np.float64)], 8) == mb.ERR_INVALID
