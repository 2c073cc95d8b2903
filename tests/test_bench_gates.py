"""The bench's parity gates (CPU): the ordered-bits ULP distance and the pass /
fail decisions that every bench line reports before it is timed."""
import math

import numpy as np
import torch

import bench


def _f32(vals):
    return torch.tensor(vals, dtype=torch.float32)


def _f64(vals):
    return torch.tensor(vals, dtype=torch.float64)


def test_ulp_distance_basics():
    one = np.float32(1.0)
    up = np.nextafter(one, np.float32(2.0))
    down = np.nextafter(one, np.float32(0.0))
    d = bench._ulp_f32(torch, _f32([1.0, float(up), float(down), 0.0, -0.0]),
                       _f64([1.0, 1.0, 1.0, -0.0, 0.0]))
    assert d.tolist() == [0, 1, 1, 0, 0]


def test_ulp_distance_across_zero_and_infinities():
    tiny = float(np.float32(1.4e-45))  # smallest positive subnormal
    d = bench._ulp_f32(torch, _f32([tiny, math.inf, -math.inf]), _f64([-tiny, math.inf, -math.inf]))
    assert d.tolist() == [2, 0, 0]


def test_ulp_distance_nan_pairs():
    d = bench._ulp_f32(torch, _f32([math.nan, math.nan, 1.0]), _f64([math.nan, 1.0, math.nan]))
    assert d[0].item() == 0
    assert d[1].item() > 1 << 20 and d[2].item() > 1 << 20  # a lone NaN never passes


def test_ulp_gate_decisions():
    ref = _f64([0.5, 2.0, -3.0])
    got = ref.float().clone()
    assert bench.parity_gate(torch, "same", got, ref, ulp_bound=2)["pass"]
    got[1] = float(np.nextafter(np.nextafter(np.nextafter(np.float32(2.0), np.float32(3.0)),
                                            np.float32(3.0)), np.float32(3.0)))
    g = bench.parity_gate(torch, "three ulp", got, ref, ulp_bound=2)
    assert g["worst_ulp"] == 3 and not g["pass"]


def test_relative_gate_decisions():
    ref = _f64([1e-3, 0.25, 0.0])
    got = (ref * (1 + 1e-6)).float()
    assert bench.parity_gate(torch, "rel", got, ref, rel_bound=2.0 ** -16, abs_floor=2.0 ** -14)["pass"]
    bad = got.clone()
    bad[0] = 2e-3
    assert not bench.parity_gate(torch, "rel", bad, ref, rel_bound=2.0 ** -16,
                                 abs_floor=2.0 ** -14)["pass"]
    nan = got.clone()
    nan[1] = math.nan
    assert not bench.parity_gate(torch, "rel", nan, ref, rel_bound=2.0 ** -16,
                                 abs_floor=2.0 ** -14)["pass"]
