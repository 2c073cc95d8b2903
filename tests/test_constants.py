"""The approximation constants shipped in the CUDA sources meet the error
bounds their comments state (evaluated here in long double on dense grids;
the f64 roundings the kernels add are ~1e-16 and do not matter at these
levels). The constants are read from the sources, so a change to a kernel's
polynomial is checked against the bound it claims."""
import math
import os
import re

import numpy as np

CSRC = os.path.join(os.path.dirname(__file__), "..", "mlk2_b200", "csrc")
NUM = r"(-?[0-9.]+(?:e-?[0-9]+)?)"


def _source(name):
    with open(os.path.join(CSRC, name)) as f:
        return f.read()


def _body(src, signature):
    start = src.index(signature)
    return src[start:src.index("\n}", start)]


def _horner_coeffs(body):
    """Coefficients of p(z) from `p = fma(z, c_hi, c_next); p = fma(z, p, c)...`
    (highest degree first), as the kernels write them."""
    first = re.search(r"double p = fma\(z, " + NUM + ", " + NUM + r"\);", body)
    rest = re.findall(r"p = fma\(z, p, " + NUM + r"\);", body)
    return [float(first.group(1)), float(first.group(2))] + [float(c) for c in rest]


def _poly(coeffs, z):
    p = np.zeros_like(z)
    for c in coeffs:
        p = p * z + np.longdouble(c)
    return p


def test_map_sin_cos_quadrant_polynomials():
    body_s = _body(_source("map.cu"), "double sin_r(double r, double z)")
    body_c = _body(_source("map.cu"), "double cos_r(double z)")
    r = np.linspace(-math.pi / 4 * 1.001, math.pi / 4 * 1.001, 400001).astype(np.longdouble)
    r = r[r != 0]
    z = r * r
    sin_err = np.max(np.abs((r + r * z * _poly(_horner_coeffs(body_s), z)) / np.sin(r) - 1))
    cos_err = np.max(np.abs((1 + z * _poly(_horner_coeffs(body_c), z)) / np.cos(r) - 1))
    # half an f32 ulp at worst is 2^-25 ~ 3e-8 (the comments claim 3.9e-9 / 3.9e-8)
    assert sin_err < 4e-9, sin_err
    assert cos_err < 4e-8, cos_err


def test_map_half_period_sine_polynomial():
    body = _body(_source("map.cu"), "double sin_half_period(double u, int& k)")
    r = np.linspace(-math.pi / 2 * 1.0005, math.pi / 2 * 1.0005, 400001).astype(np.longdouble)
    r = r[r != 0]
    z = r * r
    err = np.max(np.abs((r + r * z * _poly(_horner_coeffs(body), z)) / np.sin(r) - 1))
    assert err < 6.5e-9, err


def test_softmax_table_exponential():
    """exp(d) = 2^(k/256) (1 + r + r^2/2), r = d - k ln2/256: the shipped
    constants give relative error < 4.3e-10 over the softmax range."""
    body = _body(_source("softmax.cu"), "double exp_neg_tab(double d, const double* tab)")
    c_k = float(re.search(r"fma\(d, " + NUM + r", kMagic\)", body).group(1))
    c_ln = float(re.search(r"fma\(-kd, " + NUM + r", d\)", body).group(1))
    assert abs(c_k - 256 / math.log(2)) < 1e-12 and abs(c_ln - math.log(2) / 256) < 1e-18
    d = np.linspace(-120.0, 0.0, 2000001)
    k = np.rint(d * c_k)
    r = (d - k * c_ln).astype(np.longdouble)
    approx = np.exp2(k.astype(np.longdouble) / 256) * (1 + r + r * r / 2)
    err = np.max(np.abs(approx / np.exp(d.astype(np.longdouble)) - 1))
    assert err < 4.3e-10, err
