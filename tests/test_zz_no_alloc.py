"""The allocation-free row softmax, mlkb_softmax_f32_noalloc.

Some callers cannot let a library call cudaMalloc: their device memory is
all handed out by their own pool allocator, or they run inside a host
callback that must not allocate. For them the library offers this entry: the
same row-softmax kernel as mlkb_softmax_f32, with the kernel's scratch (the
status word of its bounded waits) in a fixed array inside the library.

This test calls it through the C ABI and checks two calls in a row against
mlkb_softmax_f32 on the same input, to the tolerance of the softmax tests
(<= 2 ULP), and that the second call leaves the device's free memory as it
was. It lives in its own file, collected last, and passes both alone in a
fresh process and after the rest of the suite.
"""
import numpy as np
import pytest

import mlk2_b200 as mb
import oracle

pytestmark = pytest.mark.gpu


def free_bytes():
    import torch

    return torch.cuda.mem_get_info()[0]


@pytest.mark.parametrize("shape", [(4099, 4096), (300, 1000), (64, 8192)])
def test_noalloc_matches_allocating_entry(cuda, shape):
    rows, cols = shape
    rng = np.random.default_rng(rows + cols)
    xh = rng.normal(0.0, 4.0, shape).astype(np.float32)
    xh[1, 3] = np.inf          # a poisoned row
    x = cuda.from_numpy(xh).cuda()
    want = cuda.full(shape, np.nan, device="cuda")
    L = mb.lib()
    stream = cuda.cuda.current_stream().cuda_stream
    assert L.mlkb_softmax_f32(x.data_ptr(), want.data_ptr(), rows, cols, stream) == 0
    cuda.cuda.synchronize()
    ref = want.cpu().numpy()
    for call, wait in ((1, 1), (2, 0)):
        got = cuda.full(shape, np.nan, device="cuda")
        before = free_bytes() if call == 2 else None
        st = L.mlkb_softmax_f32_noalloc(x.data_ptr(), got.data_ptr(), rows, cols, wait, stream)
        assert st == 0, L.mlkb_last_error().decode()
        cuda.cuda.synchronize()
        if before is not None:
            assert free_bytes() == before          # nothing was allocated
        g = got.cpu().numpy()
        assert oracle.ulp_f32(g, ref.astype(np.float64)).max() <= 2, call
    # and against the f64 oracle, like the other softmax tests
    sample = slice(0, rows, max(1, rows // 64))
    r64 = oracle.port().softmax(xh[sample].astype(np.float64))
    assert oracle.ulp_f32(g[sample], r64).max() <= 2


def test_noalloc_rejects_rows_past_its_limit(cuda):
    x = cuda.zeros((4, 8196), device="cuda")
    y = cuda.zeros_like(x)
    st = mb.lib().mlkb_softmax_f32_noalloc(x.data_ptr(), y.data_ptr(), 4, 8196, 1, None)
    assert st == mb.ERR_INVALID
    assert "8192" in mb.lib().mlkb_last_error().decode()
