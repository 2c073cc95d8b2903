"""GEMM on the GPU against the oracle.

Bounds (fp32 accumulation of exact f16 products, order unspecified):
componentwise |C - C_ref| <= 2^-12 * sum_k |a_ik b_kj| (+ |C0| rounding for
accumulate), normwise ||C - C_ref||_F / ||C_ref||_F <= 1e-5. The f32-input
path uses 2^-14 componentwise (f32 FMA, no TF32). f64 is bit-exact.
"""
import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def check_bounds(c, a, b, c0=None, rel=2.0**-12):
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    ref = oracle.port().matmul(a64, b64, None if c0 is None else c0.astype(np.float64))
    scale = np.abs(a64) @ np.abs(b64) + (0 if c0 is None else np.abs(c0.astype(np.float64)))
    err = np.abs(c.astype(np.float64) - ref)
    assert np.all(err <= rel * scale + 1e-30), float((err / np.maximum(scale, 1e-30)).max())
    fro = np.linalg.norm(c - ref) / max(np.linalg.norm(ref), 1e-300)
    assert fro <= 1e-5, fro
    return ref


@pytest.mark.parametrize("mnk", [(128, 256, 64), (256, 512, 128), (200, 264, 72),
                                 (1, 8, 8), (384, 256, 1024), (129, 520, 136)])
def test_f16_tcgen05_shapes(cuda, mnk):
    m, n, k = mnk
    rng = np.random.default_rng(m + n + k)
    a = (rng.normal(0, 1, (m, k)) / np.sqrt(k)).astype(np.float16)
    b = (rng.normal(0, 1, (k, n)) / np.sqrt(k)).astype(np.float16)
    c = empty(cuda, (m, n), cuda.float32)
    api.gemm(dev(cuda, a), dev(cuda, b), c)
    check_bounds(host(c), a, b)
    assert api.take_device_error() == 0


def test_f16_exact_pattern_bit_exact(cuda):
    # The reference's own GEMM operands (unit_poly.cpp:5150-5157): every
    # product and partial sum is exact in f32, so the tensor-core result must
    # equal the f64 reference bit for bit.
    m, n, k = 128, 256, 64
    a = np.array([(i % 7) * 0.25 for i in range(m * k)]).reshape(m, k).astype(np.float16)
    b = np.array([(i % 5) * 0.5 for i in range(k * n)]).reshape(k, n).astype(np.float16)
    c = empty(cuda, (m, n), cuda.float32)
    api.gemm(dev(cuda, a), dev(cuda, b), c)
    ref = oracle.port().matmul(a.astype(np.float64), b.astype(np.float64))
    assert np.array_equal(host(c).astype(np.float64), ref)


def test_f16_golden_accumulate_and_fallback(cuda, golden):
    g = golden("gemm")
    a, b, c0 = g["h_a"], g["h_b"], g["h_c0"]       # K = 56, N = 48: TMA path
    c = dev(cuda, c0.copy())
    api.gemm(dev(cuda, a), dev(cuda, b), c, accumulate=True)
    ref = check_bounds(host(c), a, b, c0)          # componentwise, C0 included
    assert np.array_equal(ref, g["h_c"])           # the oracle is the golden itself
    # K = 14 and N = 12 are not multiples of 8: the SIMT fallback, exact here
    ea, eb = g["exact_a"].astype(np.float16), g["exact_b"].astype(np.float16)
    c = empty(cuda, (16, 12), cuda.float32)
    api.gemm(dev(cuda, ea), dev(cuda, eb), c)
    assert np.array_equal(host(c).astype(np.float64), g["exact_c"])


def test_f16_config4_full_size_sampled(cuda):
    """BASELINE config 4 (8192^3, N(0,1)/sqrt(K)): one 64-row block checked
    against the oracle componentwise, 8 more blocks against an f64 product."""
    n = 8192
    a = cuda.empty((n, n), dtype=cuda.float16, device="cuda")
    b = cuda.empty((n, n), dtype=cuda.float16, device="cuda")
    api.fill(a, 0x4D4C4B2B, 41, "normal", 0.0, 1.0 / np.sqrt(n))
    api.fill(b, 0x4D4C4B2B, 42, "normal", 0.0, 1.0 / np.sqrt(n))
    c = cuda.empty((n, n), dtype=cuda.float32, device="cuda")
    api.gemm(a, b, c)
    bh = host(b).astype(np.float64)
    ah_blk = host(a[8128:8192]).astype(np.float64)
    check_bounds(host(c[8128:8192]), ah_blk, bh)
    for r0 in np.linspace(0, n - 64, 8).astype(int):
        ab = host(a[r0:r0 + 64]).astype(np.float64)
        ref = ab @ bh
        got = host(c[r0:r0 + 64]).astype(np.float64)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5
    assert api.take_device_error() == 0


def test_f32_simt_1024(cuda):
    rng = np.random.default_rng(3)
    a = (rng.normal(0, 1, (1024, 1024)) / 32).astype(np.float32)
    b = (rng.normal(0, 1, (1024, 1024)) / 32).astype(np.float32)
    c = empty(cuda, (1024, 1024), cuda.float32)
    api.gemm(dev(cuda, a), dev(cuda, b), c)
    check_bounds(host(c), a, b, rel=2.0**-14)


def test_f64_bit_exact_and_module(cuda):
    rng = np.random.default_rng(4)
    a, b, c0 = rng.normal(size=(100, 70)), rng.normal(size=(70, 90)), rng.normal(size=(100, 90))
    a[5, :10] = 0.0
    c = dev(cuda, c0.copy())
    api.gemm(dev(cuda, a), dev(cuda, b), c, accumulate=True)
    assert np.array_equal(host(c), oracle.port().matmul(a, b, c0))
    # the reference-facing legacy ABI: C += A*B over host f64 buffers
    ch = c0.copy()
    mod = kir.call_module("matmul", 100, 70, 90, ("f64", "f64", "f64"))
    assert api.legacy_call(mod, [a, b, ch], ch.size) == mb.OK
    assert np.array_equal(ch, oracle.best().matmul(a, b, c0))
