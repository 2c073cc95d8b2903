"""Sharded runs assembled on device 0 (mlkb_module_run_sharded): maps by the
shards' own peer stores into device 0's buffers, the other kinds (and maps
with MLKB_ASSEMBLE_VIA_NCCL) by NCCL.

CPU part: NCCL that cannot be loaded, or lacks its entry points, is reported
as MLKB_ERR_NCCL (code 5) before any device is touched. GPU part: an NCCL
whose communicator creation fails (a stand-in library built here) is
reported the same way with the outputs untouched; otherwise the assembled
outputs are bit-identical to the host-buffer run, on one GPU and on every
GPU of the box, by either transfer.
"""
import os
import subprocess

import numpy as np
import pytest

import mlk2_b200 as mb
from mlk2_b200 import api, kir

FAKE_NCCL = r"""
typedef void* ncclComm_t;
int ncclCommInitAll(ncclComm_t* c, int n, const int* d) { (void)c; (void)n; (void)d; return 2; }
int ncclGroupStart(void) { return 0; }
int ncclGroupEnd(void) { return 0; }
int ncclSend(const void* b, unsigned long n, int t, int p, ncclComm_t c, void* s) { return 0; }
int ncclRecv(void* b, unsigned long n, int t, int p, ncclComm_t c, void* s) { return 0; }
const char* ncclGetErrorString(int r) { (void)r; return "injected communicator failure"; }
"""


def build_so(tmp_path, name, source):
    src = tmp_path / (name + ".c")
    src.write_text(source)
    out = tmp_path / (name + ".so")
    subprocess.run(["gcc", "-shared", "-fPIC", "-w", str(src), "-o", str(out)], check=True)
    return str(out)


def map_case(n=4096):
    m = api.Module(kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]))
    x = np.linspace(-8, 8, n).astype(np.float32)
    return m, x


def test_missing_nccl_is_reported(monkeypatch, tmp_path):
    m, x = map_case()
    y, dy = np.zeros_like(x), np.zeros_like(x)
    monkeypatch.setenv("MLKB_NCCL_LIB", str(tmp_path / "no_such_libnccl.so"))
    assert m.run_sharded([x, y, dy], n=x.size) == mb.ERR_NCCL
    assert "cannot load" in mb.lib().mlkb_last_error().decode()
    empty = build_so(tmp_path, "libempty", "int unrelated(void) { return 0; }\n")
    monkeypatch.setenv("MLKB_NCCL_LIB", empty)
    assert m.run_sharded([x, y, dy], n=x.size) == mb.ERR_NCCL
    assert "lacks" in mb.lib().mlkb_last_error().decode()


def test_unknown_flag_rejected():
    m, x = map_case()
    y = np.zeros_like(x)
    ptrs, dts, nb, sc = m._args([x, y, y.copy()], [])
    assert mb.lib().mlkb_module_run_sharded(m._h, ptrs, dts, nb, x.size, sc, 0, 1, 6) == \
        mb.ERR_INVALID
    # the NCCL-only flag means nothing without assembly
    assert mb.lib().mlkb_module_run_sharded(m._h, ptrs, dts, nb, x.size, sc, 0, 1, 2) == \
        mb.ERR_INVALID


@pytest.mark.gpu
def test_injected_communicator_failure(cuda, monkeypatch, tmp_path):
    m, x = map_case()
    y = cuda.full((x.size,), 7.0, device="cuda")
    dy = cuda.full((x.size,), 7.0, device="cuda")
    monkeypatch.setenv("MLKB_NCCL_LIB", build_so(tmp_path, "libfakenccl", FAKE_NCCL))
    assert m.run_sharded([x, y, dy], n=x.size, n_gpus=1) == mb.ERR_NCCL
    assert "injected" in mb.lib().mlkb_last_error().decode()
    cuda.cuda.synchronize()
    assert bool((y == 7.0).all()) and bool((dy == 7.0).all())   # nothing was written


def _cases(cuda):
    rng = np.random.default_rng(3)
    # config-2 map, odd length
    x = rng.uniform(-8, 8, 100003).astype(np.float32)
    yield "map", kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]), [x], [(x.size,)] * 2, x.size, \
        np.float32
    # a root that writes only part of its output, next to a full one: the rest
    # of device 0's buffer keeps its values
    part = kir.map_module([kir.SIN_CHAIN, kir.chain(kir.E("mul", kir.A, kir.C(2.0)))])
    part["nodes"][0]["end"] = 60000
    yield "map_part", part, [x], [(x.size,)] * 2, x.size, np.float32
    # softmax rows
    a = rng.normal(0, 4, (1000, 512)).astype(np.float32)
    yield "softmax", kir.call_module("softmax", 1000, 512), [a], [(1000, 512)], 0, np.float32
    # GEMM accumulating into a C that starts on device 0
    ga = rng.normal(0, 1, (300, 256)).astype(np.float16)
    gb = rng.normal(0, 1, (256, 384)).astype(np.float16)
    yield "matmul", kir.call_module("matmul", 300, 256, 384, ("f16", "f16", "f32")), [ga, gb], \
        [(300, 384)], 0, np.float32
    # the fused scaled-scores composite, Kt in place
    q = rng.normal(0, 1, (512, 64)).astype(np.float16)
    kt = np.ascontiguousarray(rng.normal(0, 1, (64, 512)).astype(np.float16))
    yield "qk", kir.qk_softmax_module(512, 64, 0.125, temps=True), [q, kt], [(512, 512)], \
        512 * 512, np.float32


@pytest.mark.gpu
@pytest.mark.parametrize("via_nccl", [False, True])
@pytest.mark.parametrize("n_gpus", [1, 0])
def test_assembled_equals_host_run(cuda, monkeypatch, n_gpus, via_nccl):
    # maps assemble by the shards' peer stores into device 0 unless via_nccl;
    # the other kinds always by NCCL. Same bits either way.
    monkeypatch.delenv("MLKB_NCCL_LIB", raising=False)
    for name, doc, ins, out_shapes, n, odt in _cases(cuda):
        m = api.Module(doc)
        start = [np.random.default_rng(1).normal(0, 1, s).astype(odt) for s in out_shapes]
        host_outs = [o.copy() for o in start]
        m.run_host(ins + host_outs, n=n, n_gpus=1)
        dev_outs = [cuda.from_numpy(o.copy()).cuda() for o in start]
        st = m.run_sharded(ins + dev_outs, n=n, n_gpus=n_gpus, via_nccl=via_nccl)
        assert st == 0, (name, mb.lib().mlkb_last_error().decode())
        for h, d in zip(host_outs, dev_outs):
            got = d.cpu().numpy()
            assert np.array_equal(got.view(np.int32), h.view(np.int32)), name
    assert api.take_device_error() == 0


@pytest.mark.gpu
def test_outputs_must_live_on_device_0(cuda, monkeypatch):
    monkeypatch.delenv("MLKB_NCCL_LIB", raising=False)
    m, x = map_case()
    y, dy = np.zeros_like(x), np.zeros_like(x)   # host memory: not an assembled output
    assert m.run_sharded([x, y, dy], n=x.size, n_gpus=1) == mb.ERR_INVALID
