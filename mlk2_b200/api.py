"""Typed wrappers over the libmlkb200 C ABI.

Device buffers are passed as torch CUDA tensors (torch provides device memory
and streams only); every computation happens in libmlkb200.so. Host buffers
are numpy arrays or CPU tensors.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import F16, F32, F64, check, kir, lib

ASSEMBLE_DEVICE0 = 1  # MLKB_ASSEMBLE_DEVICE0
ASSEMBLE_VIA_NCCL = 2  # MLKB_ASSEMBLE_VIA_NCCL

_TORCH_DT = None


def _dt_of(x) -> int:
    global _TORCH_DT
    if isinstance(x, np.ndarray):
        return {np.dtype(np.float16): F16, np.dtype(np.float32): F32,
                np.dtype(np.float64): F64}[x.dtype]
    if _TORCH_DT is None:
        import torch

        _TORCH_DT = {torch.float16: F16, torch.float32: F32, torch.float64: F64}
    return _TORCH_DT[x.dtype]


def _ptr(x) -> int:
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("host buffers must be C-contiguous")
        return x.ctypes.data
    if not x.is_contiguous():
        raise ValueError("tensors must be contiguous")
    return x.data_ptr()


def _stream(stream=None) -> int:
    if stream is not None:
        return int(stream)
    import torch

    return torch.cuda.current_stream().cuda_stream


# ---- direct kernels (device tensors, asynchronous on the current stream) ----

def map_sin(x, y, stream=None):
    check(lib().mlkb_map_sin_f32(_ptr(x), _ptr(y), x.numel(), _stream(stream)))


def map_sin_dsin(x, y, dy, stream=None):
    check(lib().mlkb_map_sin_dsin_f32(_ptr(x), _ptr(y), _ptr(dy), x.numel(), _stream(stream)))


def map_chain(exprs: np.ndarray, a, out, b=None, scalars: Sequence[float] = (), poly7=False,
              stream=None):
    exprs = np.ascontiguousarray(exprs, dtype=kir.EXPR_DTYPE)
    sc = (C.c_double * max(1, len(scalars)))(*scalars)
    check(lib().mlkb_map_chain(exprs.ctypes.data, len(exprs), int(poly7), _ptr(a), _ptr(b),
                               _ptr(out), _dt_of(out), out.numel(), sc, len(scalars),
                               _stream(stream)))


def chain_compile(mode: int = -1):
    """Run-time chain compilation: mode 1 on, 0 off (interpreter), -1 query.
    Returns (active, compiled, launched): whether chains will be compiled and
    how many chain kernels this process has compiled and launched."""
    comp, launched = C.c_int64(0), C.c_int64(0)
    active = lib().mlkb_chain_compile(int(mode), C.byref(comp), C.byref(launched))
    return bool(active), comp.value, launched.value


def chain_build(exprs: np.ndarray, dtype: str = "f32", has_b: bool = False, poly7=False):
    """Compiles the kernel map_chain would use for this chain (no GPU needed)."""
    exprs = np.ascontiguousarray(exprs, dtype=kir.EXPR_DTYPE)
    check(lib().mlkb_chain_build(exprs.ctypes.data, len(exprs), int(poly7),
                                 F64 if dtype == "f64" else F32, int(has_b)))


def softmax(x, y, stream=None):
    rows, cols = x.shape
    fn = lib().mlkb_softmax_f32 if _dt_of(x) == F32 else lib().mlkb_softmax_f64
    check(fn(_ptr(x), _ptr(y), rows, cols, _stream(stream)))


def reducesum(x, y, stream=None):
    rows, cols = x.shape
    fn = lib().mlkb_reducesum_f32 if _dt_of(x) == F32 else lib().mlkb_reducesum_f64
    check(fn(_ptr(x), _ptr(y), rows, cols, _stream(stream)))


def gemm(a, b, c, accumulate=False, stream=None):
    m, k = a.shape
    k2, n = b.shape
    assert k == k2 and tuple(c.shape) == (m, n)
    dt = _dt_of(a)
    fn = {F16: lib().mlkb_gemm_f16_f32, F32: lib().mlkb_gemm_f32, F64: lib().mlkb_gemm_f64}[dt]
    check(fn(_ptr(a), _ptr(b), _ptr(c), m, n, k, int(accumulate), _stream(stream)))


def qk_softmax(q, k, y, scale: float, stream=None):
    batch, s, d = q.shape
    check(lib().mlkb_qk_softmax_f16(_ptr(q), _ptr(k), _ptr(y), batch, s, d, float(scale),
                                    _stream(stream)))


def qk_softmax_kt(q, kt, y, scale: float, stream=None):
    """Y[b] = softmax_rows(scale * Q[b] @ Kt[b]): Q [batch, m, d], Kt [batch, d, s]."""
    batch, m, d = q.shape
    s = kt.shape[2]
    assert tuple(kt.shape) == (batch, d, s) and tuple(y.shape) == (batch, m, s)
    check(lib().mlkb_qk_softmax_kt_f16(_ptr(q), _ptr(kt), _ptr(y), batch, m, s, d, float(scale),
                                       _stream(stream)))


def fill(out, seed: int, stream_id: int, dist: str, lo: float, hi: float, stream=None):
    d = {"uniform": 0, "normal": 1}[dist]
    fn = lib().mlkb_fill_f32 if _dt_of(out) == F32 else lib().mlkb_fill_f16
    check(fn(_ptr(out), out.numel(), seed, stream_id, d, lo, hi, _stream(stream)))


def take_device_error() -> int:
    return lib().mlkb_take_device_error()


# ---- module API ---------------------------------------------------------------

class Module:
    """A Kernel IR module bound from its `mlk-kernel` JSON (dict or str)."""

    def __init__(self, module):
        text = module if isinstance(module, str) else kir.dumps(module)
        h = C.c_void_p()
        check(lib().mlkb_module_create(text.encode(), C.byref(h)))
        self._h = h

    def close(self) -> None:
        """Releases the native module (also done when the object is collected)."""
        if getattr(self, "_h", None):
            lib().mlkb_module_destroy(self._h)
            self._h = None

    def __del__(self):
        # At interpreter shutdown the module globals this needs may already be
        # gone; the process is exiting and the handle dies with it.
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    @property
    def kind(self) -> int:
        return lib().mlkb_module_kind(self._h)

    @property
    def num_buffers(self) -> int:
        return lib().mlkb_module_num_buffers(self._h)

    def plan(self, dtypes) -> str:
        """Names of the kernels run_dev launches with these buffer dtypes
        (MLKB_F16 / F32 / F64 codes, or arrays / tensors to take them from)."""
        codes = [d if isinstance(d, int) else _dt_of(d) for d in dtypes]
        arr = (C.c_int32 * len(codes))(*codes)
        buf = C.create_string_buffer(512)
        check(lib().mlkb_module_plan(self._h, arr, len(codes), buf, 512))
        return buf.value.decode()

    def _args(self, bufs, scalars):
        n = len(bufs)
        ptrs = (C.c_void_p * n)(*[_ptr(b) for b in bufs])
        dts = (C.c_int32 * n)(*[_dt_of(b) for b in bufs])
        sc = (C.c_double * max(1, len(scalars)))(*scalars)
        return ptrs, dts, n, sc

    def run_dev(self, bufs, n: int = 0, scalars: Sequence[float] = (), device=None,
                stream=None):
        """Runs over device tensors on `device` (default: the tensors' own
        device) and `stream` (default: torch's current stream of it)."""
        if device is None:
            device = next((b.device.index for b in bufs if hasattr(b, "device")), 0)
        if stream is None:
            import torch

            stream = torch.cuda.current_stream(device).cuda_stream
        ptrs, dts, nb, sc = self._args(bufs, scalars)
        check(lib().mlkb_module_run_dev(self._h, ptrs, dts, nb, n, sc, len(scalars), device,
                                        _stream(stream)))

    def run_host(self, bufs, n: int = 0, scalars: Sequence[float] = (), n_gpus: int = 0):
        ptrs, dts, nb, sc = self._args(bufs, scalars)
        check(lib().mlkb_module_run_host(self._h, ptrs, dts, nb, n, sc, len(scalars), n_gpus))

    def run_sharded(self, bufs, n: int = 0, scalars: Sequence[float] = (), n_gpus: int = 0,
                    assemble: bool = True, via_nccl: bool = False) -> int:
        """Inputs from host buffers, sharded over n_gpus devices; with
        `assemble` the outputs are device-0 tensors, filled by the shards'
        peer stores (maps) or by NCCL (other kinds, or with `via_nccl`).
        Returns the status (0 = ok) rather than raising, for fault-injection
        tests."""
        ptrs, dts, nb, sc = self._args(bufs, scalars)
        flags = (ASSEMBLE_DEVICE0 | (ASSEMBLE_VIA_NCCL if via_nccl else 0)) if assemble else 0
        return lib().mlkb_module_run_sharded(self._h, ptrs, dts, nb, n, sc, len(scalars), n_gpus,
                                             flags)


def legacy_call(module: dict, host_f64: Sequence[np.ndarray], n: int,
                scalars: Sequence[float] = ()) -> int:
    """Bind `module` and call mlk_kernel in the reference's legacy 1-D form
    (buffers..., n, scalars, n_scalars) exactly as LoadedKernel::run does;
    returns mlk_last_status()."""
    L = lib()
    check(L.mlk_bind_module(kir.dumps(module).encode()))
    sc = (C.c_double * max(1, len(scalars)))(*scalars)
    args = [b.ctypes.data for b in host_f64] + [n, C.cast(sc, C.c_void_p).value, len(scalars)]
    args += [0] * (18 - len(args))
    L.mlk_kernel(*args)
    return L.mlk_last_status()
