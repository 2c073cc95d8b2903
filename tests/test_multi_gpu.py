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


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_device_checks_and_current_device_kept(cuda):
    """A kernel never runs on one GPU against another GPU's buffers: run_dev
    refuses buffers (or a stream) of another device, and no entry point leaves
    the caller on a different current device."""
    import ctypes as C

    m = api.Module(kir.map_module([kir.SIN_CHAIN]))
    x1 = cuda.zeros(1024, device="cuda:1")
    y1 = cuda.zeros(1024, device="cuda:1")
    ptrs = (C.c_void_p * 2)(x1.data_ptr(), y1.data_ptr())
    dts = (C.c_int32 * 2)(mb.F32, mb.F32)
    sc = (C.c_double * 1)(0.0)
    cuda.cuda.set_device(0)
    st = mb.lib().mlkb_module_run_dev(m._h, ptrs, dts, 2, 1024, sc, 0, 0, None)
    assert st == mb.ERR_INVALID
    s1 = cuda.cuda.Stream(device=1)
    ptrs0 = (C.c_void_p * 2)(cuda.zeros(1024, device="cuda:0").data_ptr(),
                             cuda.zeros(1024, device="cuda:0").data_ptr())
    st = mb.lib().mlkb_module_run_dev(m._h, ptrs0, dts, 2, 1024, sc, 0, 0, s1.cuda_stream)
    assert st == mb.ERR_INVALID
    # the right device and stream run, and the caller's device is kept
    m.run_dev([x1, y1], n=1024, device=1)
    assert cuda.cuda.current_device() == 0
    xs = np.linspace(-8, 8, 4096).astype(np.float32)
    out = [cuda.zeros(4096, device="cuda:0"), cuda.zeros(4096, device="cuda:0")]
    two = api.Module(kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]))
    assert two.run_sharded([xs] + out, n=4096, n_gpus=2) == 0
    assert cuda.cuda.current_device() == 0
