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
# (74, 512, 64): 296 units over 148 CTAs, where runs of 2 bands fill the CTAs
# evenly (runs of 4 would leave half of them idle); single batches take runs
# of 1.
@pytest.mark.parametrize("shape", [(2, 256, 128), (3, 384, 64), (2, 1024, 64), (1, 2048, 128),
                                   (1, 4096, 128), (2, 200, 64), (1, 136, 96), (74, 512, 64)])
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


# K given as the reference's MatMul B operand, Kt [batch, d, s], read in place
# as the MN-major operand. (batch, m, s, d): m != s, the row-specialised
# lengths, and shapes that take the two-step form (m or s not a multiple of
# 128, d not in {64, 128}).
@pytest.mark.parametrize("shape", [(2, 256, 256, 128), (1, 384, 512, 64), (3, 128, 1024, 64),
                                   (1, 2048, 2048, 128), (2, 200, 136, 64), (1, 256, 200, 96)])
def test_qk_softmax_kt(cuda, shape):
    batch, m, s, d = shape
    rng = np.random.default_rng(m + s + d)
    q = rng.normal(0, 1, (batch, m, d)).astype(np.float16)
    k = rng.normal(0, 1, (batch, s, d)).astype(np.float16)
    kt = np.ascontiguousarray(k.transpose(0, 2, 1))
    y = empty(cuda, (batch, m, s), cuda.float32)
    api.qk_softmax_kt(dev(cuda, q), dev(cuda, kt), y, d ** -0.5)
    check(host(y), reference(q, k, d ** -0.5))
    assert api.take_device_error() == 0


def test_qk_module_temp_form(cuda, golden):
    # S and Sc temps: the fused kernel, Kt read in place. Its result is the
    # reference's output form with S starting at zero.
    g = golden("qk")
    s_, d_ = g["q"].shape
    mod = api.Module(kir.qk_softmax_module(s_, d_, float(g["scale"]), temps=True))
    assert mod.plan([mb.F16, mb.F16, mb.F32]) == "qk_softmax_tcgen05_kt"
    y = empty(cuda, (s_, s_), cuda.float32)
    mod.run_dev([dev(cuda, g["q"]), dev(cuda, g["kt"]), y], n=s_ * s_)
    check(host(y), g["Y_zero"])
    yh = np.full((s_, s_), np.nan, np.float32)
    mod.run_host([g["q"], g["kt"], yh], n=s_ * s_, n_gpus=1)
    check(yh, g["Y_zero"])
    assert api.take_device_error() == 0


def test_qk_module_temp_form_full_rows(cuda):
    # one config-5 batch through the module, every row sum 1, sampled rows
    # against the oracle; on several GPUs the rows are split in 128-row bands
    s_, d_ = 2048, 128
    rng = np.random.default_rng(9)
    q = rng.normal(0, 1, (s_, d_)).astype(np.float16)
    k = rng.normal(0, 1, (s_, d_)).astype(np.float16)
    kt = np.ascontiguousarray(k.T)
    mod = api.Module(kir.qk_softmax_module(s_, d_, d_ ** -0.5, temps=True))
    yh = np.full((s_, s_), np.nan, np.float32)
    mod.run_host([q, kt, yh], n=s_ * s_, n_gpus=0)
    assert np.abs(yh.astype(np.float64).sum(axis=1) - 1).max() < 1e-4
    rows = np.array([0, 1, 127, 128, 1023, 1024, 2047])
    o = oracle.port()
    sc = o.matmul(q[rows].astype(np.float64), kt.astype(np.float64)) * d_ ** -0.5
    check(yh[rows], o.softmax(sc))


@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_qk_module_output_form(cuda, golden, dtype):
    # S and Sc outputs: S += Q*Kt (S starts from the caller's values),
    # Sc = S*scale, Y = softmax(Sc) -- the reference's three steps on the GPU
    g = golden("qk")
    s_, d_ = g["q"].shape
    mod = api.Module(kir.qk_softmax_module(s_, d_, float(g["scale"]), dtype=dtype))
    npdt = np.float16 if dtype == "f16" else np.float32
    S = g["s0"].copy()
    Sc = np.full_like(S, np.nan)
    Y = np.full_like(S, np.nan)
    mod.run_host([g["q"].astype(npdt), g["kt"].astype(npdt), S, Sc, Y], n=s_ * s_, n_gpus=1)
    # f32 accumulation of f16 products onto S: componentwise bound
    q64, kt64 = g["q"].astype(np.float64), g["kt"].astype(np.float64)
    bound = 2.0**-12 * (np.abs(q64) @ np.abs(kt64) + np.abs(g["s0"]))
    assert np.all(np.abs(S - g["S"]) <= bound)
    assert np.all(Sc == (S.astype(np.float64) * float(g["scale"])).astype(np.float32))
    check(Y, g["Y"])


def test_qk_module_output_form_reference_abi(cuda, golden):
    # f64 through the reference's legacy mlk_kernel call: S and Sc bit-exact
    g = golden("qk")
    s_, d_ = g["q"].shape
    mod = kir.qk_softmax_module(s_, d_, float(g["scale"]), dtype="f64")
    S = g["s0"].astype(np.float64)
    Sc, Y = np.zeros_like(S), np.zeros_like(S)
    assert api.legacy_call(mod, [g["q"].astype(np.float64), g["kt"].astype(np.float64), S, Sc, Y],
                           s_ * s_) == 0
    assert np.array_equal(S, g["S"]) and np.array_equal(Sc, g["Sc"])
    assert oracle.ulp_f64(Y, g["Y"]).max() <= 8
