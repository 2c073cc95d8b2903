"""Row softmax and row sums on the GPU against the oracle."""
import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu
ULP_BOUND = 2  # BASELINE tolerance for f32 softmax


def test_golden_softmax_all_cases(cuda, golden):
    g = golden("softmax")
    for key in [k[:-2] for k in g.files if k.endswith("_x")]:
        x = dev(cuda, g[key + "_x"])
        y = empty(cuda, x.shape, cuda.float32)
        api.softmax(x, y)
        d = oracle.ulp_f32(host(y), g[key + "_y"])
        assert d.max() <= ULP_BOUND, (key, d.max())


def test_nan_row_semantics(cuda, golden):
    g = golden("softmax")
    x = dev(cuda, g["adv_x"])
    y = empty(cuda, x.shape, cuda.float32)
    api.softmax(x, y)
    yh = host(y)
    assert np.all(np.isnan(yh[9]))              # a NaN input poisons its row
    assert not np.any(np.isnan(np.delete(yh, 9, axis=0)))


@pytest.mark.parametrize("shape", [(1, 1), (7, 3), (33, 1000), (5, 4096), (3, 5000), (2, 8192),
                                   (2, 8196), (3, 20000), (129, 256)])
def test_shapes_register_and_streaming_paths(cuda, shape):
    rng = np.random.default_rng(sum(shape))
    xh = rng.normal(0, 4, shape).astype(np.float32)
    y = empty(cuda, shape, cuda.float32)
    api.softmax(dev(cuda, xh), y)
    ref = oracle.port().softmax(xh.astype(np.float64))
    assert oracle.ulp_f32(host(y), ref).max() <= ULP_BOUND


def test_full_size_config3_sampled(cuda):
    """BASELINE config 3 ([65536 x 4096], N(0, 4^2)) at full size; every 256th
    row is checked against the oracle, every row's sum against 1."""
    rows, cols = 65536, 4096
    x = cuda.empty((rows, cols), dtype=cuda.float32, device="cuda")
    api.fill(x, 0x4D4C4B2B, 3, "normal", 0.0, 4.0)
    y = cuda.empty_like(x)
    api.softmax(x, y)
    sums = y.double().sum(dim=1)
    assert float((sums - 1).abs().max()) < 1e-5
    xs = host(x[::256])
    ref = oracle.port().softmax(xs.astype(np.float64))
    assert oracle.ulp_f32(host(y[::256]), ref).max() <= ULP_BOUND


def test_softmax_f64_and_reducesum(cuda, golden):
    g = golden("softmax")
    x = dev(cuda, g["rand_x"].astype(np.float64))
    y = empty(cuda, x.shape, cuda.float64)
    api.softmax(x, y)
    assert oracle.ulp_f64(host(y), g["rand_y"]).max() <= 8   # only exp differs (same order)
    r = golden("reducesum")
    for dt, npdt in ((cuda.float32, np.float32), (cuda.float64, np.float64)):
        xr = dev(cuda, r["x"].astype(npdt))
        yr = empty(cuda, (xr.shape[0],), dt)
        api.reducesum(xr, yr)
        if npdt == np.float64:
            assert np.array_equal(host(yr), r["y"])          # same order: bit-exact
        else:
            assert oracle.ulp_f32(host(yr), r["y"]).max() == 0


def test_softmax_module_paths(cuda, golden):
    g = golden("softmax")
    xh = g["rand_x"]
    m = api.Module(kir.call_module("softmax", *xh.shape))
    assert m.kind == mb.KIND_SOFTMAX
    y = np.full(xh.shape, np.nan, np.float32)
    m.run_host([xh, y])
    assert oracle.ulp_f32(y, g["rand_y"]).max() <= ULP_BOUND
    # legacy reference ABI, host f64
    y64 = np.zeros(xh.shape, np.float64)
    assert api.legacy_call(kir.call_module("softmax", *xh.shape, dtypes=("f64", "f64")),
                           [xh.astype(np.float64), y64], xh.size) == mb.OK
    assert oracle.ulp_f64(y64, g["rand_y"]).max() <= 8
