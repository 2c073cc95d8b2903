"""Drop-in check: the REFERENCE's own artifact loader drives this library.

oracle/_ref/ref_loader_check is built from the reference sources
(oracle/ref.mk). It binds each module with mlk_bind_module(toJson(module)),
loads libmlkb200.so through mlk::loadKernelLibrary and runs it through
LoadedKernel::run -- the reference's exactly-typed legacy mlk_kernel call --
then compares with executeKernelOnBuffers. One JSON line per case.
"""
import json
import os
import subprocess

import pytest

import mlk2_b200 as mb
import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not os.path.exists(oracle.LOADER_CHECK_PATH),
                    reason="reference loader check not built (reference sources absent)")
def test_reference_loader_runs_the_shim(cuda):
    out = subprocess.run([oracle.LOADER_CHECK_PATH, mb.LIB_PATH], capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    rows = {r["case"]: r for r in map(json.loads, out.stdout.strip().splitlines())}
    assert set(rows) == {"map_sin", "map_sin_dsin", "softmax", "matmul", "map_poly7",
                         "qk_composite", "pipeline_sin", "pipeline_dsin", "pipeline_scalar"}
    for r in rows.values():
        assert r["ok"] and r["status"] == 0 and not r["multi_dim"], r
    assert rows["matmul"]["max_ulp_f64"] == 0          # bit-exact, as the reference demands
    assert rows["map_poly7"]["max_ulp_f64"] == 0       # the poly7 family is restated exactly
    assert rows["map_sin"]["max_ulp_f64"] <= 4
    assert rows["map_sin_dsin"]["max_ulp_f64"] <= 8
    assert rows["softmax"]["max_ulp_f64"] <= 8
    # S and Sc bit-exact (f64 GEMM in the reference's order, one multiply), Y
    # through the f64 softmax
    assert rows["qk_composite"]["max_ulp_f64"] <= 8
    # modules compiled by the reference's own Tier-1 pipeline
    assert rows["pipeline_sin"]["max_ulp_f64"] <= 4
    assert rows["pipeline_dsin"]["max_ulp_f64"] <= 8
    assert rows["pipeline_scalar"]["max_ulp_f64"] <= 4
