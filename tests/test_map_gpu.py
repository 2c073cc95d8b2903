"""Fused maps on the GPU against the oracle (<= 2 ULP in f32)."""
import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu
ULP_BOUND = 2  # BASELINE tolerance for f32 maps


def test_golden_sin(cuda, golden):
    g = golden("map_sin")
    x = dev(cuda, g["x"])
    y = empty(cuda, x.shape, cuda.float32)
    api.map_sin(x, y)
    d = oracle.ulp_f32(host(y), g["y"])
    assert d.max() <= ULP_BOUND, d.max()


def test_golden_sin_dsin(cuda, golden):
    g = golden("map_sin_dsin")
    x = dev(cuda, g["x"])
    y = empty(cuda, x.shape, cuda.float32)
    dy = empty(cuda, x.shape, cuda.float32)
    api.map_sin_dsin(x, y, dy)
    assert oracle.ulp_f32(host(y), g["y"]).max() <= ULP_BOUND
    assert oracle.ulp_f32(host(dy), g["dy"]).max() <= ULP_BOUND
    # known answer of the reference's differential test
    assert abs(float(host(y)[0]) - (-0.5440211108893698)) < 1e-7


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 1023, 4097, 65536 + 7])
@pytest.mark.parametrize("offset", [0, 1])
def test_ragged_and_unaligned(cuda, n, offset):
    x_h = np.linspace(-8, 8, n + offset, dtype=np.float32)
    x = dev(cuda, x_h)[offset:]
    y = empty(cuda, (n + offset,), cuda.float32)[offset:]
    dy = empty(cuda, (n + offset,), cuda.float32)[offset:]
    api.map_sin_dsin(x, y, dy)
    if n == 0:
        return
    ry, rdy = oracle.port().chain([kir.SIN_CHAIN, kir.DSIN_CHAIN], x_h[offset:].astype(np.float64))
    assert oracle.ulp_f32(host(y), ry).max() <= ULP_BOUND
    assert oracle.ulp_f32(host(dy), rdy).max() <= ULP_BOUND


def test_special_values(cuda):
    xs = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e30, -1e30, 3e5, -3e5, 1e19],
                  dtype=np.float32)
    x = dev(cuda, xs)
    y = empty(cuda, xs.shape, cuda.float32)
    dy = empty(cuda, xs.shape, cuda.float32)
    api.map_sin_dsin(x, y, dy)
    ry, rdy = oracle.port().chain([kir.SIN_CHAIN, kir.DSIN_CHAIN], xs.astype(np.float64))
    assert oracle.ulp_f32(host(y), ry).max() <= ULP_BOUND
    assert oracle.ulp_f32(host(dy), rdy).max() <= ULP_BOUND


@pytest.mark.parametrize("cfg", [(1, 1 << 24, -4.0, 4.0), (2, 1 << 28, -8.0, 8.0)])
def test_full_size_configs_sampled(cuda, cfg):
    """BASELINE configs 1 and 2 at full size: inputs generated on the device
    (bit-identical to the host generator), every output checked for range and
    a strided sample of 2^18 elements checked against the oracle."""
    cfg_id, n, lo, hi = cfg
    seed = 0x4D4C4B2B
    x = cuda.empty(n, dtype=cuda.float32, device="cuda")
    api.fill(x, seed, cfg_id, "uniform", lo, hi)
    y = cuda.empty_like(x)
    dy = cuda.empty_like(x) if cfg_id == 2 else None
    if cfg_id == 2:
        api.map_sin_dsin(x, y, dy)
    else:
        api.map_sin(x, y)
    cuda.cuda.synchronize()
    assert bool(cuda.all(cuda.abs(y) <= 1.0))
    assert not bool(cuda.any(cuda.isnan(y)))
    stride = n // (1 << 18)
    idx = np.arange(0, n, stride)
    xs = host(x[::stride])
    assert np.array_equal(xs, oracle.fill_uniform_f32(n, seed, cfg_id, lo, hi)[idx])
    chains = [kir.SIN_CHAIN, kir.DSIN_CHAIN] if cfg_id == 2 else [kir.SIN_CHAIN]
    refs = oracle.port().chain(chains, xs.astype(np.float64))
    assert oracle.ulp_f32(host(y[::stride]), refs[0]).max() <= ULP_BOUND
    if cfg_id == 2:
        assert oracle.ulp_f32(host(dy[::stride]), refs[1]).max() <= ULP_BOUND


def test_fast_path_wide_sample(cuda):
    """2^21 inputs over the whole fast-path range |x| < 1000 (where
    |x^2 + 3x| reaches 10^6 and the reduction does real work) plus every
    binade of small |x|: both specialised kernels within the bound of the
    f64 oracle; the observed worst case and 1-ULP rate are printed."""
    rng = np.random.default_rng(77)
    n = 1 << 21
    parts = [rng.uniform(-1000.0, 1000.0, n // 2),
             rng.uniform(-8.0, 8.0, n // 4),
             np.sign(rng.uniform(-1, 1, n // 4)) * 2.0 ** rng.uniform(-40, 9.9, n // 4)]
    xh = np.concatenate(parts).astype(np.float32)
    x = dev(cuda, xh)
    y, dy, y1 = (empty(cuda, xh.shape, cuda.float32) for _ in range(3))
    api.map_sin_dsin(x, y, dy)
    api.map_sin(x, y1)
    ry, rdy = oracle.port().chain([kir.SIN_CHAIN, kir.DSIN_CHAIN], xh.astype(np.float64))
    for name, got, ref in (("sin_dsin.y", y, ry), ("sin_dsin.dy", dy, rdy), ("sin.y", y1, ry)):
        d = oracle.ulp_f32(host(got), ref)
        print(f"{name}: max {int(d.max())} ULP, {100.0 * np.mean(d > 0):.2f} % off by >= 1")
        assert d.max() <= ULP_BOUND, (name, int(d.max()))


def test_back_to_back_dependent_maps(cuda):
    """Map launches overlap through programmatic dependent launch; a map that
    reads the previous map's output must still see all of it (each kernel
    waits on the preceding grid before touching memory). 40 chained launches
    over 2^24 elements, each the next one's input, against the same chain run
    with a device synchronisation between launches."""
    n = 1 << 24
    x0 = dev(cuda, oracle.fill_uniform_f32(n, 11, 1, -4.0, 4.0))
    bufs = [x0.clone(), cuda.empty_like(x0)]
    for i in range(40):
        api.map_sin(bufs[i & 1], bufs[(i + 1) & 1])
    chained = host(bufs[0])
    ref = [x0.clone(), cuda.empty_like(x0)]
    for i in range(40):
        api.map_sin(ref[i & 1], ref[(i + 1) & 1])
        cuda.cuda.synchronize()
    assert np.array_equal(chained, host(ref[0]))


ARITH = {"add", "sub", "mul", "div", "neg", "pow22", "scalar", "poly", "sqrt", "rsqrt"}


@pytest.mark.parametrize("dtype", ["f32", "f64"])
def test_generic_chain_every_op(cuda, golden, dtype, chain_path):
    g = golden("chains")
    npdt = np.float32 if dtype == "f32" else np.float64
    xa = dev(cuda, g["xa"].astype(npdt))
    xb = dev(cuda, g["xb"].astype(npdt))
    names = [k[2:] for k in g.files if k.startswith("c_")]
    for name in names:
        ch = g["c_" + name]
        uses_b = any(int(e["a_kind"]) == 2 or int(e["b_kind"]) == 2 for e in ch)
        out = empty(cuda, xa.shape, xa.dtype)
        api.map_chain(ch, xa, out, b=xb if uses_b else None, scalars=list(g["scalars"]))
        got = host(out)
        if dtype == "f32":
            d = oracle.ulp_f32(got, g["y_" + name])
            assert d.max() <= ULP_BOUND, (name, d.max())
        else:
            ref = g["y_" + name]
            if name == "gelu":
                # 1 + tanh(.) cancels for negative inputs and amplifies the
                # libm-vs-CUDA tanh difference; checked relatively instead.
                err = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-300)
                assert np.nanmax(np.where(ref == 0, np.abs(got), err)) <= 1e-12, name
                continue
            d = oracle.ulp_f64(got, ref)
            # +,-,*,/,sqrt are correctly rounded on both sides: bit-exact.
            bound = 0 if name in ARITH else 4
            assert d.max() <= bound, (name, d.max())


def test_module_paths_match_direct(cuda):
    n = 100003
    x_h = oracle.fill_uniform_f32(n, 5, 2, -8.0, 8.0)
    x = dev(cuda, x_h)
    y0, dy0 = empty(cuda, (n,), cuda.float32), empty(cuda, (n,), cuda.float32)
    api.map_sin_dsin(x, y0, dy0)
    m = api.Module(kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]))
    y1, dy1 = empty(cuda, (n,), cuda.float32), empty(cuda, (n,), cuda.float32)
    m.run_dev([x, y1, dy1], n=n)
    assert np.array_equal(host(y0), host(y1)) and np.array_equal(host(dy0), host(dy1))
    # host buffers through the sharded host entry (all visible GPUs)
    y2 = np.full(n, np.nan, np.float32)
    dy2 = np.full(n, np.nan, np.float32)
    m.run_host([x_h, y2, dy2], n=n)
    assert np.array_equal(host(y0), y2) and np.array_equal(host(dy0), dy2)


def test_reference_legacy_abi_f64(cuda):
    """mlk_kernel in the legacy 1-D form over host f64 buffers, as
    LoadedKernel::run calls it, against the reference executor's f64 output."""
    x = np.concatenate([np.linspace(-8, 8, 5001), [2.0, 0.0, -0.0]])
    y = np.zeros_like(x)
    dy = np.zeros_like(x)
    mod = kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN], dtype="f64")
    assert api.legacy_call(mod, [x, y, dy], x.size) == mb.OK
    ry, rdy = oracle.best().chain([kir.SIN_CHAIN, kir.DSIN_CHAIN], x)
    assert oracle.ulp_f64(y, ry).max() <= 64
    assert oracle.ulp_f64(dy, rdy).max() <= 64
    assert api.take_device_error() == 0
