"""Seeded random chains through mlkb_map_chain, compiled at run time and on the
interpreter. Random ops (all sixteen), operands (constants, ElemA, ElemB,
ScalarParams, earlier temps) and lengths exercise the code generator's
operand wiring, temp numbering and constant / scalar ordering:
  * for every chain, in f32 and f64, the compiled kernel's output is
    bit-identical to the interpreter's (the same device math);
  * chains of correctly rounded arithmetic only (Add, Sub, Mul, Div, Neg,
    Sqrt, Rsqrt with their guards) are bit-exact against the oracle's f64
    restatement of the reference executor.
"""
import numpy as np
import pytest

import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu

UNARY = {"neg", "exp", "log", "sin", "cos", "tan", "tanh", "sqrt", "rsqrt", "erf", "gelu"}
EXACT = {"add", "sub", "mul", "div", "neg", "sqrt", "rsqrt"}


def random_chain(rng, ops, length):
    ex = []
    for k in range(length):
        op = ops[rng.integers(len(ops))]

        def operand():
            r = rng.random()
            if k > 0 and r < 0.45:
                return kir.T(int(rng.integers(k)))
            if r < 0.65:
                return kir.A
            if r < 0.75:
                return kir.B
            if r < 0.85:
                return kir.S(int(rng.integers(6)))  # 4, 5: past a 4-entry table, read 0
            return kir.C(float(rng.choice([0.0, -0.0, 0.5, -2.0, 3.0, 1e-3, 7.25])))
        ex.append(kir.E(op, operand()) if op in UNARY else kir.E(op, operand(), operand()))
    return kir.chain(*ex)


def _same_bits(x, y):
    """Bit-identical, any NaN matching any NaN."""
    nx, ny = np.isnan(x), np.isnan(y)
    if not np.array_equal(nx, ny):
        return False
    it = np.int32 if x.dtype == np.float32 else np.int64
    return np.array_equal(x[~nx].view(it), y[~ny].view(it))


def _inputs(n, seed):
    rng = np.random.default_rng(seed)
    a = rng.uniform(-3.0, 3.0, n)
    b = rng.uniform(-3.0, 3.0, n)
    a[:6] = [0.0, -0.0, 1.0, -1.0, 2.0, 1e-300]
    b[:6] = [0.0, 2.0, -0.0, 0.5, 2.0, -1e-300]
    return a, b


@pytest.mark.parametrize("dtype", ["f32", "f64"])
def test_compiled_equals_interpreted_on_random_chains(cuda, dtype):
    rng = np.random.default_rng(1234 if dtype == "f32" else 4321)
    n = 4099                                        # ragged: vector body and tail
    a, b = _inputs(n, 7)
    npdt = np.float32 if dtype == "f32" else np.float64
    tdt = cuda.float32 if dtype == "f32" else cuda.float64
    xa, xb = dev(cuda, a.astype(npdt)), dev(cuda, b.astype(npdt))
    scalars = [0.75, -1.5, 2.0, 0.0, 3.25, -0.5]
    _, _, launched0 = api.chain_compile(-1)
    try:
        for i in range(24):
            ch = random_chain(rng, kir.OPS, int(rng.integers(1, 20)))
            got = {}
            for mode in (1, 0):
                api.chain_compile(mode)
                out = empty(cuda, (n,), tdt)
                api.map_chain(ch, xa, out, b=xb, scalars=scalars[:4])
                got[mode] = host(out)
            assert _same_bits(got[1], got[0]), (i, ch)
    finally:
        api.chain_compile(1)
    _, _, launched1 = api.chain_compile(-1)
    assert launched1 - launched0 == 24                # every compiled run really compiled


def test_arithmetic_chains_bit_exact_against_the_oracle(cuda):
    rng = np.random.default_rng(99)
    n = 2053
    a, b = _inputs(n, 11)
    xa, xb = dev(cuda, a), dev(cuda, b)
    scalars = [0.75, -1.5, 2.0, 0.0]
    api.chain_compile(1)
    for i in range(24):
        ch = random_chain(rng, sorted(EXACT), int(rng.integers(1, 24)))
        out = empty(cuda, (n,), cuda.float64)
        api.map_chain(ch, xa, out, b=xb, scalars=scalars)
        (want,) = oracle.port().chain([ch], a, b, scalars=scalars)
        assert _same_bits(host(out), want), (i, ch)
