"""Failure detection on the GPU without a fault: a device-side wait that can
never complete gives up after its bound, the status word reports
MLKB_ERR_TIMEOUT, and the context keeps working."""
import time

import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda):
    assert api.take_device_error() == 0
    t0 = time.perf_counter()
    mb.check(mb.lib().mlkb_selftest_bounded_wait(50_000_000, None))  # 50 ms
    status = api.take_device_error()                                  # synchronises
    elapsed = time.perf_counter() - t0
    assert status == mb.ERR_TIMEOUT
    assert 0.04 <= elapsed < 5.0
    assert api.take_device_error() == 0                               # cleared on read
    # the context is still healthy: a kernel runs and is correct afterwards
    x = oracle.fill_uniform_f32(4096, 3, 2, -8.0, 8.0)
    y = empty(cuda, (4096,), cuda.float32)
    api.map_sin(dev(cuda, x), y)
    (ref,) = oracle.port().chain([kir.SIN_CHAIN], x.astype(np.float64))
    assert oracle.ulp_f32(host(y), ref).max() <= 2


def test_selftest_rejects_unbounded_limits(cuda):
    assert mb.lib().mlkb_selftest_bounded_wait(0, None) == mb.ERR_INVALID
    assert mb.lib().mlkb_selftest_bounded_wait(10_000_000_000, None) == mb.ERR_INVALID
