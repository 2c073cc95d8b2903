"""libmlkb200 inside a PATCHED reference: the reference-side changes a
maintainer would make to plug this library in (oracle/ref_patches/*.patch,
applied to a copy of the reference by oracle/ref_patched.mk, driven by
oracle/ref_integration_check.cpp).

* 03-multi-output-lowering: the reference's own compiler emits config 2 --
  y = sin(x^2+3x) and its derivative -- as ONE module with two roots, each
  storing to its own buffer, and the B200 path runs it on its fused kernel.
* 01-backend-driver: sm_100a is an accepted arch; a legacy-form call's
  status is read back from mlk_last_status.
* 02-fastkernel: runFastKernelSearch certifies the NativeCuda candidate on
  the prebuilt library -- bit-exact for the f64 GEMM under the reference's own
  policy, within a declared ULP bound for the transcendental map (GPU part).
"""
import json
import os
import subprocess

import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir

CHECK = os.path.join(os.path.dirname(oracle.REF_PATH), "patched", "ref_integration_check")
needs_check = pytest.mark.skipif(not os.path.exists(CHECK),
                                 reason="patched reference not built (reference sources absent)")


def run(*args, timeout=600):
    out = subprocess.run([CHECK, *args], capture_output=True, text=True, timeout=timeout)
    assert out.returncode == 0, out.stdout + out.stderr
    return [json.loads(line) for line in out.stdout.strip().splitlines()]


@needs_check
def test_patched_lowering_emits_the_two_root_module(golden):
    (module,) = run("lowering")
    outs = [n["out"] for n in module["nodes"] if n["op"] == "store"]
    assert len(outs) == 2 and len(set(outs)) == 2          # one buffer per output
    m = api.Module(module)
    assert m.plan([mb.F32] * 3) == "map_sin_dsin_f32"
    # the reference executor on the module its own compiler emitted
    g = golden("pipeline")
    x = g["x"].astype(np.float64)
    y, dy = np.zeros_like(x), np.zeros_like(x)
    oracle.run_json(module, [x, y, dy], x.size)
    assert np.array_equal(y.view(np.int64), g["y"].view(np.int64))
    fin = ~np.isnan(g["dy"])
    assert np.array_equal(np.isnan(dy), ~fin)
    assert np.array_equal(dy[fin].view(np.int64), g["dy"][fin].view(np.int64))


@needs_check
def test_patched_arch_validation():
    rows = {r["arch"]: r for r in run("arch")}
    assert rows["sm_100a"]["built"] and rows["sm_90a"]["built"]
    assert not rows["sm_100x"]["built"] and not rows["sm_a"]["built"]


@needs_check
@pytest.mark.skipif(mb.lib().mlkb_device_count() > 0, reason="host without a GPU only")
def test_fastkernel_cuda_candidate_reports_no_device():
    rows = run("fastkernel", mb.LIB_PATH)
    cuda = [r for r in rows if r["exec"] == "native-cuda"]
    assert len(cuda) == 2
    for r in cuda:
        # the library's status 4 (no device) surfaces through mlk_last_status
        assert not r["admissible"] and "code 4" in r["detail"], r


@needs_check
@pytest.mark.gpu
def test_fastkernel_certifies_the_cuda_variant(cuda):
    rows = run("fastkernel", mb.LIB_PATH)
    by = {(r["graph"], r["exec"]): r for r in rows}
    gemm = by[("gemm_64x48x56", "native-cuda")]
    assert gemm["admissible"] and gemm["identity"], gemm
    assert gemm["policy"] == "bitexact-f64-cpu-v1" and gemm["max_abs_diff"] == 0
    assert gemm["library"] == mb.LIB_PATH
    sin = by[("map_sin_4096", "native-cuda")]
    assert sin["admissible"] and sin["identity"], sin
    assert sin["policy"] == "ulp-bounded-f64-cuda-v1" and sin["max_ulp"] <= 16
    for g in ("gemm_64x48x56", "map_sin_4096"):
        assert by[(g, "walker")]["identity"]
