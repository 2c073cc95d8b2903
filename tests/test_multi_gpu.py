"""In-process multi-GPU host runs: mlkb_module_run_host splits the work into
contiguous element / row shards over devices 0..n-1 (one host thread and
stream each). Results must be identical to the single-GPU run. Needs at
least two visible GPUs; skipped otherwise."""
import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir

pytestmark = pytest.mark.gpu


def _two_gpus():
    return mb.lib().mlkb_device_count() >= 2


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("n_gpus", [2, 0])
def test_sharded_host_runs_match_single_gpu(cuda, n_gpus):
    # maps: element shards
    n = 3 * 65536 + 5
    x = oracle.fill_uniform_f32(n, 9, 2, -8.0, 8.0)
    m = api.Module(kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]))
    one = [np.empty(n, np.float32) for _ in range(2)]
    many = [np.empty(n, np.float32) for _ in range(2)]
    m.run_host([x] + one, n=n, n_gpus=1)
    m.run_host([x] + many, n=n, n_gpus=n_gpus)
    assert all(np.array_equal(a, b) for a, b in zip(one, many))
    # softmax: row shards
    xs = np.random.default_rng(1).normal(0, 4, (1001, 4096)).astype(np.float32)
    sm = api.Module(kir.call_module("softmax", *xs.shape))
    y1, y2 = np.empty_like(xs), np.empty_like(xs)
    sm.run_host([xs, y1], n_gpus=1)
    sm.run_host([xs, y2], n_gpus=n_gpus)
    assert np.array_equal(y1, y2)
    # matmul: M-block shards, B replicated, C accumulated (reference C += A*B)
    rng = np.random.default_rng(2)
    a = rng.normal(size=(301, 77))
    b = rng.normal(size=(77, 129))
    c0 = rng.normal(size=(301, 129))
    mm = api.Module(kir.call_module("matmul", 301, 77, 129, ("f64", "f64", "f64")))
    c = c0.copy()
    mm.run_host([a, b, c], n_gpus=n_gpus)
    assert np.array_equal(c, oracle.port().matmul(a, b, c0))
