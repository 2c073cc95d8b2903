"""Generates the golden vectors in this directory by running the REFERENCE's
own CPU executor (executeKernelOnBuffers, compiled from the reference
sources into oracle/_ref/libmlkref.so by oracle/ref.mk).

    python tests/golden/make_golden.py

Inputs are f32 (or f16) values, widened exactly to f64 for the reference, the
way the B200 path's parity tests feed it. Outputs are the reference's f64
results. Cases follow the reference's own tests where they exist:
  * sin(x^2+3x) at x=2 = -0.5440211108893698 (reference
    tests/differential/differential_test.cpp:48, examples/scalar/README.md);
  * the softmax adversarial matrix of tests/unit/unit_poly.cpp:3812-3830
    (inputs ((i*13)%19)*0.25-2, a NaN in row 9, -0/+0 ties in rows 10-11);
  * the K == 1 softmax shapes of unit_poly.cpp:3612-3650;
  * the GEMM operands of unit_poly.cpp:5150-5157 (A=(i%7)*0.25, B=(i%5)*0.5),
    which the reference requires bit-exact;
  * the "poly7" sine family (compiler/include/mlk/support/math_families.h:
    81-90) at its quadrant edges, the points its own certificate samples
    (:113-137), and far outside them;
  * modules the reference's OWN compiler produces (its Tier-1 pipeline over
    sin(x^2+3x) and over its calculus passes' derivative of it), stored as
    the JSON it wrote, with the reference executor's results on them;
  * the scaled-scores composite Call(MatMul) -> scale map -> Call(Softmax) as
    a module, with a nonzero initial S (MatMul accumulates into it).

    python tests/golden/make_golden.py [section ...]   (default: all)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from mlk2_b200 import kir  # noqa: E402
from mlk2_b200.kir import A, B, C, E, S, T, chain  # noqa: E402

SEED = 0x4D4C4B2B

EDGE = np.array([2.0, 0.0, -0.0, -1.5, -3.0, 1e-20, -1e-20, 3.0, -4.0, 3.999999761581421,
                 0.5, -0.5, 1.0, -1.0, 7.9999995, -7.9999995, 1e-3, 2.5, -2.5, 1.25],
                dtype=np.float32)

# One chain per scalar-realisable op, with the reference's guarded semantics
# (runtime/src/execution/kernel_buffers.cpp:130-159).
OP_CHAINS = {
    "add": chain(E("add", A, B)),
    "sub": chain(E("sub", A, B)),
    "mul": chain(E("mul", A, B)),
    "div": chain(E("div", A, B)),
    "neg": chain(E("neg", A)),
    "pow22": chain(E("pow", C(2), C(2)), E("mul", T(0), A)),
    "pow": chain(E("mul", A, A), E("add", T(0), C(0.5)), E("pow", T(1), C(1.5))),
    "exp": chain(E("exp", A)),
    "log": chain(E("log", A)),
    "sin": chain(E("sin", A)),
    "cos": chain(E("cos", A)),
    "tan": chain(E("tan", A)),
    "tanh": chain(E("tanh", A)),
    "sqrt": chain(E("sqrt", A)),
    "rsqrt": chain(E("rsqrt", A)),
    "erf": chain(E("erf", A)),
    "gelu": chain(E("gelu", A)),
    "scalar": chain(E("mul", A, S(0)), E("add", T(0), S(1)), E("mul", T(1), S(7))),
    "poly": chain(E("mul", A, A), E("mul", T(0), C(0.25)), E("sub", T(1), B), E("div", T(2), C(3))),
}


def main(sections) -> None:
    ref = oracle.ref()
    if "base" in sections:
        base(ref)
    if "poly7" in sections:
        poly7(ref)
    if "pipeline" in sections:
        pipeline()
    if "qk" in sections:
        qk()
    print("golden vectors written to", HERE)


def poly7(ref) -> None:
    quarter = np.pi / 4
    edges = np.array([k * quarter for k in range(-16, 17)] +
                     [np.nextafter(k * quarter, np.inf) for k in range(-8, 9)] +
                     [1e5, -1e5, 123456.789, 1e10, -3e15, 1e300, np.inf, -np.inf, np.nan,
                      0.0, -0.0, 1e-300], np.float64)
    sample = -np.pi + 2 * np.pi * np.arange(4096) / 4096  # the certificate's grid
    x = np.concatenate([edges, sample, np.random.default_rng(11).uniform(-50, 50, 2048)])
    with np.errstate(over="ignore"):
        xf = x.astype(np.float32)  # the f32 path's inputs (out-of-range values become inf)
    sin1 = chain(E("sin", A))
    (y_sin,) = ref.chain([sin1], x, poly7=True)
    (y_u,) = ref.chain([kir.SIN_CHAIN], xf.astype(np.float64), poly7=True)
    (y_sinf,) = ref.chain([sin1], xf.astype(np.float64), poly7=True)
    np.savez_compressed(os.path.join(HERE, "map_poly7.npz"), x=x, xf=xf, sin=y_sin,
                        sin_u_f=y_u, sin_f=y_sinf, chain_sin=sin1, chain_u=kir.SIN_CHAIN)


def pipeline() -> None:
    import json

    n = 4096
    y_mod, _ = oracle.pipeline_json(0, n)
    d_mod, patched = oracle.pipeline_json(1, n)
    s_mod, _ = oracle.pipeline_json(2, 1)
    both = kir.merge_roots([y_mod, d_mod], ["y", "dy"])
    x = np.concatenate([EDGE, np.array([np.inf, -np.inf, np.nan, 1e30, -1e30], np.float32),
                        oracle.fill_uniform_f32(n - EDGE.size - 5, SEED, 2, -8.0, 8.0)])
    x64 = x.astype(np.float64)
    y, dy = np.zeros(n), np.zeros(n)
    oracle.run_json(both, [x64, y, dy], n)
    ys, dys = np.zeros(n), np.zeros(n)
    oracle.run_json(y_mod, [x64, ys], n)
    oracle.run_json(d_mod, [x64, dys], n)
    assert np.array_equal(ys.view(np.int64), y.view(np.int64))
    assert np.array_equal(dys.view(np.int64), dy.view(np.int64), equal_nan=False) or \
        np.array_equal(np.isnan(dys), np.isnan(dy))
    xs = np.array([2.0, 0.0, -1.5, 3.0, 1e-3, -4.0])
    s_out = []
    for v in xs:
        out = np.zeros(1)
        oracle.run_json(s_mod, [out], 1, scalars=[v])
        s_out.append(out[0])
    np.savez_compressed(os.path.join(HERE, "pipeline.npz"),
                        sin_json=json.dumps(y_mod), dsin_json=json.dumps(d_mod),
                        both_json=json.dumps(both), scalar_json=json.dumps(s_mod),
                        patched=patched, x=x, y=y, dy=dy, scalar_x=xs, scalar_y=np.array(s_out))


def qk() -> None:
    rng = np.random.default_rng(5)
    s_, d_ = 128, 64
    q = rng.normal(0, 1, (s_, d_)).astype(np.float16)
    kt = np.ascontiguousarray(rng.normal(0, 1, (s_, d_)).astype(np.float16).T)
    s0 = rng.normal(0, 2, (s_, s_)).astype(np.float32)  # MatMul accumulates into S
    scale = d_ ** -0.5
    mod = kir.qk_softmax_module(s_, d_, scale)
    S, Sc, Y = s0.astype(np.float64), np.zeros((s_, s_)), np.zeros((s_, s_))
    oracle.run_json(mod, [q.astype(np.float64), kt.astype(np.float64), S, Sc, Y], s_ * s_)
    S0, Sc0, Y0 = np.zeros((s_, s_)), np.zeros((s_, s_)), np.zeros((s_, s_))
    oracle.run_json(mod, [q.astype(np.float64), kt.astype(np.float64), S0, Sc0, Y0], s_ * s_)
    np.savez_compressed(os.path.join(HERE, "qk.npz"), q=q, kt=kt, s0=s0, scale=scale,
                        S=S, Sc=Sc, Y=Y, Y_zero=Y0)


def base(ref) -> None:
    out = {}

    # config-1 chain: sin(x^2 + 3x), x ~ U(-4, 4), plus edge values
    x1 = np.concatenate([EDGE, oracle.fill_uniform_f32(4096, SEED, 1, -4.0, 4.0)])
    (y1,) = ref.chain([kir.SIN_CHAIN], x1.astype(np.float64))
    np.savez_compressed(os.path.join(HERE, "map_sin.npz"), x=x1, y=y1)

    # config-2 chains: y and dy/dx, x ~ U(-8, 8)
    x2 = np.concatenate([EDGE, oracle.fill_uniform_f32(4096, SEED, 2, -8.0, 8.0)])
    y2, dy2 = ref.chain([kir.SIN_CHAIN, kir.DSIN_CHAIN], x2.astype(np.float64))
    np.savez_compressed(os.path.join(HERE, "map_sin_dsin.npz"), x=x2, y=y2, dy=dy2)

    # every scalar op, over edge values including the guard boundaries
    rng = np.random.default_rng(7)
    xa = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 2.0, 0.5, -0.5, 1e-30, -1e-30, 3.0, 10.0, -10.0, 100.0,
                  -100.0, 1e30, -1e30, np.inf, -np.inf, np.nan, 700.0, -700.0], np.float32),
        rng.uniform(-6, 6, 235).astype(np.float32)])
    xb = np.concatenate([
        np.array([0.0, 0.0, -0.0, 2.0, 0.0, 3.0, 0.0, 1.0, 0.0, -2.0, 0.0, 5.0, -0.5, 0.0, 1.0,
                  0.0, 1.0, 2.0, 0.0, 1.0, 1.0], np.float32),
        rng.uniform(-3, 3, 235).astype(np.float32)])
    scalars = np.array([1.5, -0.25, 0, 0, 0, 0, 0, 3.0])
    ops = {"xa": xa, "xb": xb, "scalars": scalars}
    for name, ch in OP_CHAINS.items():
        uses_b = any(int(e["a_kind"]) == 2 or int(e["b_kind"]) == 2 for e in ch)
        (y,) = ref.chain([ch], xa.astype(np.float64), xb.astype(np.float64) if uses_b else None,
                         scalars=scalars)
        ops["y_" + name] = y
        ops["c_" + name] = ch
    np.savez_compressed(os.path.join(HERE, "chains.npz"), **ops)

    # softmax: the reference's adversarial matrix, K == 1 shapes, random rows
    m, k = 12, 8
    adv = np.array([((i * 13) % 19) * 0.25 - 2.0 for i in range(m * k)], np.float64)
    adv[9 * k + 2] = np.nan
    for j in range(k):
        adv[10 * k + j] = -0.0 if j % 2 == 0 else 0.0
    adv[11 * k + 0], adv[11 * k + 1], adv[11 * k + 2], adv[11 * k + 3] = -1.0, -0.0, 0.0, -2.0
    adv = adv.reshape(m, k).astype(np.float32)
    sm = {"adv_x": adv, "adv_y": ref.softmax(adv.astype(np.float64))}
    for (mm, kk) in [(5, 1), (3, 7), (8, 4)]:
        xs = np.array([((i * 7) % 11) * 0.5 - 2.5 for i in range(mm * kk)], np.float32).reshape(mm, kk)
        sm[f"k_{mm}x{kk}_x"] = xs
        sm[f"k_{mm}x{kk}_y"] = ref.softmax(xs.astype(np.float64))
    xr = rng.normal(0.0, 4.0, (64, 256)).astype(np.float32)
    xr[3, 17] = np.inf            # +inf: (inf - inf) poisons the row
    xr[4, :] = -np.inf            # all -inf: NaN row
    xr[5, :] = 0.0                # flat row
    xr[6, 100] = 80.0             # one dominant entry, the rest underflow
    sm["rand_x"] = xr
    sm["rand_y"] = ref.softmax(xr.astype(np.float64))
    np.savez_compressed(os.path.join(HERE, "softmax.npz"), **sm)

    # reducesum
    xs = rng.normal(0.0, 1.0, (32, 100)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "reducesum.npz"), x=xs,
                        y=ref.reducesum(xs.astype(np.float64)))

    # GEMM: the bit-exact operands, and a random f16-valued problem
    ga = np.array([(i % 7) * 0.25 for i in range(16 * 14)]).reshape(16, 14)
    gb = np.array([(i % 5) * 0.5 for i in range(14 * 12)]).reshape(14, 12)
    ha = (rng.normal(0, 1, (64, 56)) / np.sqrt(56)).astype(np.float16)
    hb = (rng.normal(0, 1, (56, 48)) / np.sqrt(56)).astype(np.float16)
    hc = rng.normal(0, 1, (64, 48)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "gemm.npz"),
                        exact_a=ga, exact_b=gb, exact_c=ref.matmul(ga, gb),
                        h_a=ha, h_b=hb, h_c0=hc,
                        h_c=ref.matmul(ha.astype(np.float64), hb.astype(np.float64),
                                       hc.astype(np.float64)))


if __name__ == "__main__":
    main(sys.argv[1:] or ["base", "poly7", "pipeline", "qk"])
