"""The oracle itself, pinned (CPU only).

The C restatement (oracle/mlk_oracle.c) must reproduce the reference's own
executor bit for bit: against the committed golden vectors (produced by the
compiled reference, tests/golden/make_golden.py) and, where the compiled
reference is present, against it directly on fresh inputs.
"""
import numpy as np
import pytest

import oracle
from mlk2_b200 import kir

port = oracle.port()
needs_ref = pytest.mark.skipif(not oracle.ref_available(),
                               reason="reference sources were not available to build oracle/_ref")


def same_bits(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return a.shape == b.shape and np.array_equal(a.view(np.int64), b.view(np.int64))


def test_known_answer_sin_graph():
    # reference tests/differential/differential_test.cpp:48 (tol 1e-13)
    (y,) = port.chain([kir.SIN_CHAIN], np.array([2.0]))
    assert abs(y[0] - (-0.5440211108893698)) <= 1e-13


def test_known_answer_derivative():
    # d/dx sin(x^2+3x) = cos(x^2+3x)(2x+3); at x = 3: cos(18) * 9
    (dy,) = port.chain([kir.DSIN_CHAIN], np.array([3.0]))
    assert abs(dy[0] - np.cos(18.0) * 9.0) <= 1e-13


def test_golden_maps(golden):
    g = golden("map_sin")
    (y,) = port.chain([kir.SIN_CHAIN], g["x"].astype(np.float64))
    assert same_bits(y, g["y"])
    g = golden("map_sin_dsin")
    y, dy = port.chain([kir.SIN_CHAIN, kir.DSIN_CHAIN], g["x"].astype(np.float64))
    assert same_bits(y, g["y"]) and same_bits(dy, g["dy"])


def test_golden_chains_every_op(golden):
    g = golden("chains")
    xa, xb = g["xa"].astype(np.float64), g["xb"].astype(np.float64)
    names = [k[2:] for k in g.files if k.startswith("c_")]
    assert len(names) >= 19
    for name in names:
        ch = g["c_" + name]
        uses_b = any(int(e["a_kind"]) == 2 or int(e["b_kind"]) == 2 for e in ch)
        (y,) = port.chain([ch], xa, xb if uses_b else None, scalars=g["scalars"])
        assert same_bits(y, g["y_" + name]), name


def test_golden_guards(golden):
    # Div by 0 -> 0, Log of <= 0 -> 0, Sqrt of < 0 -> 0, Rsqrt of <= 0 -> 0
    g = golden("chains")
    xa, xb = g["xa"], g["xb"]
    assert np.all(g["y_div"][xb == 0] == 0.0)
    assert np.all(g["y_log"][xa <= 0] == 0.0)
    assert np.all(g["y_sqrt"][xa < 0] == 0.0)
    assert np.all(g["y_rsqrt"][xa <= 0] == 0.0)


def test_golden_softmax(golden):
    g = golden("softmax")
    for key in [k[:-2] for k in g.files if k.endswith("_x")]:
        y = port.softmax(g[key + "_x"].astype(np.float64))
        assert same_bits(y, g[key + "_y"]), key
    adv = g["adv_y"]
    assert np.all(np.isnan(adv[9]))            # NaN poisons its row
    assert not np.any(np.isnan(adv[10:]))      # +-0 ties do not
    assert np.all(g["k_5x1_y"] == 1.0)         # K == 1 edge
    r = g["rand_y"]
    assert np.all(np.isnan(r[3])) and np.all(np.isnan(r[4]))


def test_golden_reducesum_gemm(golden):
    g = golden("reducesum")
    assert same_bits(port.reducesum(g["x"].astype(np.float64)), g["y"])
    g = golden("gemm")
    assert same_bits(port.matmul(g["exact_a"], g["exact_b"]), g["exact_c"])
    c = port.matmul(g["h_a"].astype(np.float64), g["h_b"].astype(np.float64),
                    g["h_c0"].astype(np.float64))
    assert same_bits(c, g["h_c"])


def test_generator_matches_documented_formula():
    # word = splitmix64(seed + stream*2^40 + (i+1)*golden); k = top 24 bits
    def word(seed, sid, i):
        m = (1 << 64) - 1
        z = (seed + (sid << 40) + (i + 1) * 0x9E3779B97F4A7C15) & m
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
        return z ^ (z >> 31)

    x = oracle.fill_uniform_f32(64, 123, 5, -8.0, 8.0)
    for i in range(64):
        k = word(123, 5, i) >> 40
        assert x[i] == np.float32(-8.0 + 16.0 * k * 2.0**-24)
    assert np.all((x >= -8) & (x < 8))


@needs_ref
def test_port_matches_reference_fresh_inputs():
    ref = oracle.ref()
    rng = np.random.default_rng(11)
    x = rng.uniform(-9, 9, 5000)
    for chains in ([kir.SIN_CHAIN], [kir.SIN_CHAIN, kir.DSIN_CHAIN]):
        for a, b in zip(port.chain(chains, x), ref.chain(chains, x, threads=3)):
            assert same_bits(a, b)
    a = rng.normal(0, 4, (37, 129))
    assert same_bits(port.softmax(a), ref.softmax(a))
    assert same_bits(port.reducesum(a), ref.reducesum(a))
    ma, mb, mc = rng.normal(size=(70, 33)), rng.normal(size=(33, 90)), rng.normal(size=(70, 90))
    ma[3, :5] = 0.0  # exercise the zero-a skip
    assert same_bits(port.matmul(ma, mb, mc), ref.matmul(ma, mb, mc, threads=4))


def test_ulp_distance_rules():
    # reference tools/mlk-poly/poly_bench.cpp:78-93 semantics
    assert oracle.ulp_f32(np.float32(np.nan), np.nan)[()] == 0
    assert np.isinf(oracle.ulp_f32(np.float32(1.0), np.nan)[()])
    assert oracle.ulp_f32(np.float32(-0.0), 0.0)[()] == 0
    one_up = np.nextafter(np.float32(1.0), np.float32(2.0))
    assert oracle.ulp_f32(one_up, 1.0)[()] == 1
    # across zero: smallest subnormals of opposite sign are 2 apart
    tiny = np.float32(1e-45)
    assert oracle.ulp_f32(tiny, -float(tiny))[()] == 2


def test_golden_poly7(golden):
    # the reference's "poly7" sine family (math_families.h:81-90), both on
    # f64 inputs and on f32 inputs widened exactly
    g = golden("map_poly7")
    (y,) = port.chain([g["chain_sin"]], g["x"], poly7=True)
    assert same_bits(y, g["sin"])
    (y,) = port.chain([g["chain_sin"]], g["xf"].astype(np.float64), poly7=True)
    assert same_bits(y, g["sin_f"])
    (y,) = port.chain([g["chain_u"]], g["xf"].astype(np.float64), poly7=True)
    assert same_bits(y, g["sin_u_f"])


def test_poly7_is_a_different_family_within_its_certificate(golden):
    # poly7 differs from libm somewhere on [-pi, pi], and by single-digit ULP
    # at most there (the reference's own accuracy claim, math_families.h:10-13)
    g = golden("map_poly7")
    x = g["x"]
    grid = (x >= -np.pi) & (x <= np.pi)
    (p7,) = port.chain([g["chain_sin"]], x[grid], poly7=True)
    (lm,) = port.chain([g["chain_sin"]], x[grid])
    d = oracle.ulp_f64(p7, lm)
    assert 0 < d.max() < 10
    assert np.all(np.isnan(g["sin"][~np.isfinite(x)]))


@needs_ref
def test_poly7_port_matches_reference_fresh_inputs():
    rng = np.random.default_rng(12)
    x = np.concatenate([rng.uniform(-20, 20, 4000), rng.uniform(-1e6, 1e6, 1000)])
    for chains in ([kir.chain(kir.E("sin", kir.A))], [kir.SIN_CHAIN, kir.DSIN_CHAIN]):
        for a, b in zip(port.chain(chains, x, poly7=True), oracle.ref().chain(chains, x, poly7=True)):
            assert same_bits(a, b)
