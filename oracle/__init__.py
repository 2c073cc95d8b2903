"""Parity oracle for the B200 path. TEST INFRASTRUCTURE ONLY.

Two CPU implementations of the reference's buffer executor, both f64:
  * ``port``: oracle/mlk_oracle.c, a plain-C restatement (always built);
  * ``ref``:  oracle/_ref/libmlkref.so, the reference's OWN executor compiled
    from its sources by oracle/ref.mk (present where the reference sources
    were available at build time; the built file travels with the repo).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package, as the checker or the timed CPU baseline -- never the shipped path.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(_HERE, "libmlk_oracle.so")
REF_PATH = os.path.join(_HERE, "_ref", "libmlkref.so")
LOADER_CHECK_PATH = os.path.join(_HERE, "_ref", "ref_loader_check")

_vp, _i32, _i64 = C.c_void_p, C.c_int32, C.c_int64


def _p(a):
    return None if a is None else a.ctypes.data


class _Executor:
    """Common ctypes surface of the port and the compiled reference."""

    def __init__(self, path: str, prefix: str):
        self.path = path
        self.lib = C.CDLL(path)
        self.prefix = prefix
        f = self._fn
        if prefix == "mlkref_":
            f("chain").argtypes = [_i32, _vp, _vp, _i32, _vp, _vp, _vp, _i64, _vp, _i64, _i64]
        else:
            f("chain").argtypes = [_i32, _vp, _vp, _i32, _vp, _vp, _vp, _i64, _vp, _i64]
        for name in ("softmax", "reducesum"):
            f(name).argtypes = [_vp, _vp, _i64, _i64]
        if prefix == "mlkref_":
            f("matmul").argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64]
        else:
            f("matmul").argtypes = [_vp, _vp, _vp, _i64, _i64, _i64]
            f("matmul_rows").argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64]

    def _fn(self, name):
        return getattr(self.lib, self.prefix + name)

    def _check(self, rc):
        if rc != 0:
            msg = ""
            if self.prefix == "mlkref_":
                self.lib.mlkref_last_error.restype = C.c_char_p
                msg = self.lib.mlkref_last_error().decode()
            raise RuntimeError(f"{self.prefix} status {rc} {msg}")

    def chain(self, chains, a, b=None, scalars=(), poly7=False, threads=0):
        """Multi-root chain over f64 inputs: returns one f64 output per chain."""
        from mlk2_b200.kir import EXPR_DTYPE

        a = np.ascontiguousarray(a, dtype=np.float64)
        b = None if b is None else np.ascontiguousarray(b, dtype=np.float64)
        allx = np.ascontiguousarray(np.concatenate(chains), dtype=EXPR_DTYPE)
        lens = (C.c_int32 * len(chains))(*[len(c) for c in chains])
        outs = [np.zeros(a.size, np.float64) for _ in chains]
        optr = (C.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        sc = np.ascontiguousarray(scalars, dtype=np.float64)
        if self.prefix == "mlkref_":
            rc = self._fn("chain")(len(chains), lens, allx.ctypes.data, int(poly7), _p(a), _p(b),
                                   optr, a.size, sc.ctypes.data if sc.size else None, sc.size,
                                   threads)
        else:
            rc = self._fn("chain")(len(chains), lens, allx.ctypes.data, int(poly7), _p(a), _p(b),
                                   optr, a.size, sc.ctypes.data if sc.size else None, sc.size)
        self._check(rc)
        return outs

    def softmax(self, a):
        a = np.ascontiguousarray(a, dtype=np.float64)
        y = np.zeros_like(a)
        self._check(self._fn("softmax")(_p(a), _p(y), a.shape[0], a.shape[1]))
        return y

    def reducesum(self, a):
        a = np.ascontiguousarray(a, dtype=np.float64)
        y = np.zeros(a.shape[0], np.float64)
        self._check(self._fn("reducesum")(_p(a), _p(y), a.shape[0], a.shape[1]))
        return y

    def matmul(self, a, b, c=None, threads=0):
        """C + A*B in f64 (the reference accumulates into C)."""
        a = np.ascontiguousarray(a, dtype=np.float64)
        b = np.ascontiguousarray(b, dtype=np.float64)
        m, k = a.shape
        n = b.shape[1]
        c = np.zeros((m, n), np.float64) if c is None else np.array(c, dtype=np.float64)
        if self.prefix == "mlkref_":
            self._check(self._fn("matmul")(_p(a), _p(b), _p(c), m, n, k, threads))
        else:
            self._check(self._fn("matmul")(_p(a), _p(b), _p(c), m, n, k))
        return c


_port = None
_ref = None


def port() -> _Executor:
    global _port
    if _port is None:
        _port = _Executor(PORT_PATH, "mlko_")
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref() -> _Executor:
    global _ref
    if _ref is None:
        _ref = _Executor(REF_PATH, "mlkref_")
    return _ref


def run_json(module, bufs, n: int, scalars=(), threads: int = 0):
    """Runs an `mlk-kernel` module (dict or JSON text) through the compiled
    reference's executeKernelOnBuffers, in place over f64 numpy buffers given
    in table order (inputs, then outputs)."""
    import json as _json

    text = module if isinstance(module, str) else _json.dumps(module)
    r = ref()
    fn = r.lib.mlkref_run_json
    fn.argtypes = [C.c_char_p, _vp, _i32, _i64, _vp, _i64, _i64]
    for b in bufs:
        assert b.dtype == np.float64 and b.flags["C_CONTIGUOUS"]
    ptrs = (C.c_void_p * max(1, len(bufs)))(*[b.ctypes.data for b in bufs])
    sc = np.ascontiguousarray(scalars, dtype=np.float64)
    r._check(fn(text.encode(), ptrs, len(bufs), n, sc.ctypes.data if sc.size else None, sc.size,
                threads))


def pipeline_json(which: int, n: int, f32: bool = True):
    """(module dict, patched constants) of a module the reference's own Tier-1
    pipeline compiles: which 0 = sin(x*x + 3x) over a tensor x[n], 1 = its
    Derivative through the reference's calculus passes, 2 = the scalar form."""
    import json as _json

    r = ref()
    fn = r.lib.mlkref_pipeline_json
    fn.argtypes = [_i32, _i64, _i32, C.c_char_p, _i64, C.POINTER(_i32)]
    buf = C.create_string_buffer(1 << 16)
    patched = _i32(0)
    r._check(fn(which, n, int(f32), buf, 1 << 16, C.byref(patched)))
    return _json.loads(buf.value.decode()), patched.value


def best():
    """The compiled reference when present, else the C port."""
    return ref() if ref_available() else port()


def fill_uniform_f32(n: int, seed: int, stream_id: int, lo: float, hi: float, first: int = 0):
    """Host copy of the device uniform generator (bit-identical)."""
    lib = port().lib
    lib.mlko_fill_uniform_f32.argtypes = [_vp, _i64, C.c_uint64, C.c_uint32, C.c_double,
                                          C.c_double, _i64]
    out = np.empty(n, np.float32)
    lib.mlko_fill_uniform_f32(out.ctypes.data, n, seed, stream_id, lo, hi, first)
    return out


def _ulp(g, r, ibits, utype):
    def ordered(x):
        b = x.view(utype)
        sign = utype(1) << utype(ibits - 1)
        return np.where(b & sign, ~b, b | sign)

    og, orr = ordered(g), ordered(r)
    d = np.where(og > orr, og - orr, orr - og).astype(np.float64)
    # The reference maps -0 and +0 to the same point; the unsigned map above
    # keeps them one apart, so pairs straddling zero are one step closer.
    sign = utype(1) << utype(ibits - 1)
    d = np.where(((g.view(utype) ^ r.view(utype)) & sign) != 0, d - 1.0, d)
    gn, rn = np.isnan(g), np.isnan(r)
    d = np.where(gn & rn, 0.0, d)
    d = np.where(gn ^ rn, np.inf, d)
    d = np.where((g == r) & ~gn, 0.0, d)
    return d


def ulp_f32(got, ref_f64):
    """Ordered-bits ULP distance between f32 results and the f64 oracle
    rounded to f32 (the reference's ulpDistance, tools/mlk-poly/
    poly_bench.cpp:78-93, applied to float bits): NaN pairs count 0, a
    one-sided NaN is an infinite gap, +0 and -0 are equal."""
    g = np.ascontiguousarray(got, dtype=np.float32)
    r = np.ascontiguousarray(np.asarray(ref_f64, dtype=np.float64).astype(np.float32))
    return _ulp(g, r, 32, np.uint32)


def ulp_f64(got, ref):
    """The same ordered-bits distance on f64 values."""
    g = np.ascontiguousarray(got, dtype=np.float64)
    r = np.ascontiguousarray(ref, dtype=np.float64)
    return _ulp(g, r, 64, np.uint64)
