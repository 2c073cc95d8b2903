"""Batched scaled-scores softmax against the oracle composition
Call(MatMul) -> scale map -> Call(Softmax) in f64.

Bound: |y - y_ref| <= 2^-16 * y_ref + 2^-30.
"""
import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def reference(q, k, scale):
    """Per batch: S = Q K^T (K^T materialised, as the reference requires),
    Sc = S * scale (the map), Y = softmax(Sc) -- all by the oracle."""
    o = oracle.port()
    mul = kir.chain(kir.E("mul", kir.A, kir.C(scale)))
    out = []
    for b in range(q.shape[0]):
        s = o.matmul(q[b].astype(np.float64), k[b].astype(np.float64).T.copy())
        (sc,) = o.chain([mul], s.ravel())
        out.append(o.softmax(sc.reshape(s.shape)))
    return np.stack(out)


def check(y, ref):
    assert np.all(np.abs(y.astype(np.float64) - ref) <= 2.0**-16 * ref + 2.0**-30), \
        float(np.max(np.abs(y - ref) / (ref + 2.0**-30)))


# s = 1024, 2048 and 4096 run kernels specialised on the row length, other
# multiples of 128 the runtime-length kernel. (2, 200, 64) and (1, 136, 96): s
# not a multiple of 128 or d not in {64, 128} take the two-step form
# (single-CTA batched tcgen05 GEMM with K-major B and the scale in its
# epilogue, then the row softmax in place).
@pytest.mark.parametrize("shape", [(2, 256, 128), (3, 384, 64), (2, 1024, 64), (1, 2048, 128),
                                   (1, 4096, 128), (2, 200, 64), (1, 136, 96)])
def test_qk_softmax(cuda, shape):
    batch, s, d = shape
    rng = np.random.default_rng(s + d)
    q = rng.normal(0, 1, (batch, s, d)).astype(np.float16)
    k = rng.normal(0, 1, (batch, s, d)).astype(np.float16)
    y = empty(cuda, (batch, s, s), cuda.float32)
    api.qk_softmax(dev(cuda, q), dev(cuda, k), y, d ** -0.5)
    check(host(y), reference(q, k, d ** -0.5))
    assert api.take_device_error() == 0


def test_config5_full_size_sampled(cuda):
    """BASELINE config 5 (256 x [2048 x 2048], d = 128) at full size: batches
    0, 1, 127 and 255 against the oracle, every row sum against 1."""
    batch, s, d = 256, 2048, 128
    q = cuda.empty((batch, s, d), dtype=cuda.float16, device="cuda")
    k = cuda.empty((batch, s, d), dtype=cuda.float16, device="cuda")
    api.fill(q, 0x4D4C4B2B, 51, "normal", 0.0, 1.0)
    api.fill(k, 0x4D4C4B2B, 52, "normal", 0.0, 1.0)
    y = cuda.empty((batch, s, s), dtype=cuda.float32, device="cuda")
    api.qk_softmax(q, k, y, d ** -0.5)
    sums = y.double().sum(dim=2)
    assert float((sums - 1).abs().max()) < 1e-4
    for b in (0, 255):
        ref = reference(host(q[b:b + 1]), host(k[b:b + 1]), d ** -0.5)
        check(host(y[b:b + 1]), ref)


def test_qk_module_composite_recognised():
    m = api.Module(kir.qk_softmax_module(2048, 128, 128 ** -0.5))
    assert m.kind == mb.KIND_QK_SOFTMAX
