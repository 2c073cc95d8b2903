"""Modules the reference's OWN compiler produces, on the B200 path (CPU part).

tests/golden/pipeline.npz holds what the reference's Tier-1 pipeline emitted
for sin(x^2+3x) over a tensor x and for its derivative through the reference's
calculus passes (oracle/ref_modules.h), with the reference executor's results.
These tests check, without a GPU, that the B200 path reads those documents,
picks its dedicated kernels for them, and that the pipeline's derivative chain
is the same function as the hand-written one the fast kernel implements.
"""
import json

import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir

needs_ref = pytest.mark.skipif(not oracle.ref_available(),
                               reason="reference sources were not available to build oracle/_ref")


def modules(golden):
    g = golden("pipeline")
    return {k: json.loads(str(g[k + "_json"])) for k in ("sin", "dsin", "both", "scalar")}


def test_pipeline_modules_take_the_dedicated_kernels(golden):
    m = modules(golden)
    plans = {k: api.Module(v).plan([mb.F32] * api.Module(v).num_buffers) for k, v in m.items()}
    assert plans["sin"] == "map_sin_f32"
    assert plans["both"] == "map_sin_dsin_f32"
    assert plans["dsin"] == "map_chain"     # a derivative alone has no dedicated kernel
    assert plans["scalar"] == "map_chain"   # x as a ScalarParam: a one-element chain
    # the reference ABI is f64 end to end: the generic chain path, both roots
    # in one kernel (they read the same x over the same range)
    both = api.Module(m["both"])
    assert both.plan([mb.F64] * 3) == "map_chains2"


def test_pipeline_derivative_is_the_hand_chain(golden):
    # cos(3x + x*x) * ((x + x) + (0*x + 3)) equals cos(x*x + 3x) * (2x + 3)
    # for every f32 x, bit for bit up to the NaN payload: the argument the
    # fast path's matcher relies on, checked on the reference's own results.
    g = golden("pipeline")
    x = g["x"].astype(np.float64)
    pipe = kir.chains_of(modules(golden)["dsin"])[0]
    (a,) = oracle.port().chain([pipe], x)
    (b,) = oracle.port().chain([kir.DSIN_CHAIN], x)
    fin = ~np.isnan(b)
    assert np.array_equal(np.isnan(a), np.isnan(b))
    assert np.array_equal(a[fin].view(np.int64), b[fin].view(np.int64))
    assert np.array_equal(a[fin].view(np.int64), g["dy"][fin].view(np.int64))
    assert g["patched"] == 1   # the one constant the reference left untyped


def test_pipeline_goldens_reproduced_by_the_port(golden):
    g = golden("pipeline")
    m = modules(golden)
    y_chain = kir.chains_of(m["sin"])[0]
    (y,) = oracle.port().chain([y_chain], g["x"].astype(np.float64))
    assert np.array_equal(y.view(np.int64), g["y"].view(np.int64))
    s_chain = kir.chains_of(m["scalar"])[0]
    for v, want in zip(g["scalar_x"], g["scalar_y"]):
        (out,) = oracle.port().chain([s_chain], np.zeros(1), scalars=[v])
        assert out[0] == want


@needs_ref
def test_pipeline_is_deterministic():
    # the committed documents are what the reference's pipeline emits now
    got, _ = oracle.pipeline_json(1, 4096)
    want = kir.chains_of(got)[0]
    assert len(want) == 9 and want[-1]["op"] == kir.OP["mul"]


def test_tier2_output_is_not_on_this_path():
    # The reference's Tier-2 pipeline gives the same map an affine store
    # ("out_index_coeffs": [1]) over ElemA operands, which its own multi-dim
    # walker rejects (kernel_buffers.cpp:717-727); the B200 path reports it
    # unsupported rather than guessing.
    m = json.loads(kir.dumps(kir.map_module([kir.SIN_CHAIN])))
    m["nodes"][2]["out_index_coeffs"] = [1]
    m["nodes"][2]["out_index_offset"] = 0
    with pytest.raises(mb.MLKBError) as e:
        api.Module(m)
    assert e.value.status == mb.ERR_UNSUPPORTED
