"""Host-buffer runs from pageable memory. The reference's LoadedKernel::run
passes ordinary std::vector memory, which the library stages through its own
pinned buffers; the results must be exactly those of a run from pinned
buffers and of the device-resident run, across pipeline chunks (16 MB of the
widest staged buffer each for maps), partial static ranges and the piecewise (32 MB) copies of the
row-split kinds."""
import numpy as np
import pytest

import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def _pinned(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


@pytest.mark.parametrize("n_gpus", [1, 0])        # 0: every GPU, shards staging at once
def test_map_pageable_equals_pinned_and_device(cuda, n_gpus):
    n = 3 * (1 << 21) + 12345                      # two 2^22-element chunks, the last ragged
    xh = oracle.fill_uniform_f32(n, 5, 9, -8.0, 8.0)
    m = api.Module(kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]))
    y0, dy0 = empty(cuda, (n,), cuda.float32), empty(cuda, (n,), cuda.float32)
    m.run_dev([dev(cuda, xh), y0, dy0], n=n)
    want_y, want_dy = host(y0), host(dy0)
    for _ in range(2):                              # the second call reuses the staging
        y1, dy1 = np.full(n, np.nan, np.float32), np.full(n, np.nan, np.float32)
        m.run_host([xh, y1, dy1], n=n, n_gpus=n_gpus)
        assert np.array_equal(y1, want_y) and np.array_equal(dy1, want_dy)
    xp = _pinned(cuda, xh)
    yp, dyp = _pinned(cuda, np.full(n, np.nan, np.float32)), _pinned(cuda, np.full(n, np.nan, np.float32))
    m.run_host([xp, yp, dyp], n=n, n_gpus=n_gpus)
    assert np.array_equal(yp.numpy(), want_y) and np.array_equal(dyp.numpy(), want_dy)
    # a pageable input with pinned outputs, and the reverse
    y2, dy2 = _pinned(cuda, np.zeros(n, np.float32)), np.zeros(n, np.float32)
    m.run_host([xh, y2, dy2], n=n, n_gpus=n_gpus)
    assert np.array_equal(y2.numpy(), want_y) and np.array_equal(dy2, want_dy)


def test_reference_abi_static_range_across_chunks(cuda):
    # f64 buffers through mlk_kernel, as LoadedKernel::run passes them (2^21-
    # element chunks); root 0 stops at a static end inside the second chunk, root 1 runs to n, and the
    # rest of root 0's output keeps the caller's values
    n = (1 << 22) + 7
    stop = (1 << 21) + 1000
    mod = kir.map_module([kir.SIN_CHAIN, kir.chain(kir.E("mul", kir.A, kir.C(2.0)))], dtype="f64")
    mod["nodes"][0]["end"] = stop
    x = np.linspace(-6.0, 6.0, n)
    y0 = np.full(n, 7.0)
    y1 = np.zeros(n)
    assert api.legacy_call(mod, [x, y0, y1], n) == 0
    (want,) = oracle.port().chain([kir.SIN_CHAIN], x[:stop])
    assert oracle.ulp_f64(y0[:stop], want).max() <= 4
    assert np.all(y0[stop:] == 7.0)
    assert np.array_equal(y1, x * 2.0)


def test_row_kinds_pageable_pieces(cuda):
    # softmax over 4096 x 4096 f32 (64 MB: two 32 MB pieces each way) and a
    # MatMul whose C is both read and written (C += A B)
    rng = np.random.default_rng(3)
    xs = (rng.standard_normal((4096, 4096)) * 4).astype(np.float32)
    sm = api.Module(kir.call_module("softmax", 4096, 4096))
    ys = np.full_like(xs, np.nan)
    sm.run_host([xs, ys], n=0, n_gpus=0)           # row shards over every GPU
    yd = empty(cuda, xs.shape, cuda.float32)
    api.softmax(dev(cuda, xs), yd)
    assert np.array_equal(ys, host(yd))

    a = rng.standard_normal((512, 1024)).astype(np.float32) / 32
    b = rng.standard_normal((1024, 2048)).astype(np.float32) / 32
    c0 = rng.standard_normal((512, 2048)).astype(np.float32)
    mm = api.Module(kir.call_module("matmul", 512, 1024, 2048))
    c = c0.copy()
    mm.run_host([a, b, c], n=0, n_gpus=1)
    cd = dev(cuda, c0)
    api.gemm(dev(cuda, a), dev(cuda, b), cd, accumulate=True)
    assert np.array_equal(c, host(cd))
