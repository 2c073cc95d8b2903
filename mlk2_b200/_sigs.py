"""ctypes signatures of every entry point in include/mlkb200.h."""
from __future__ import annotations

import ctypes as C

i32, i64, u32, u64, f64 = C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_double
vp, cp = C.c_void_p, C.c_char_p

# name -> (restype, argtypes)
SIGNATURES = {
    "mlk_bind_module": (i32, [cp]),
    "mlk_kernel": (i32, [C.c_ssize_t] * 18),
    "mlk_last_status": (i32, []),
    "mlkb_last_error": (cp, []),
    "mlkb_version": (cp, []),
    "mlkb_device_count": (i32, []),
    "mlkb_take_device_error": (i32, []),
    "mlkb_selftest_bounded_wait": (i32, [u64, vp]),
    "mlkb_module_create": (i32, [cp, C.POINTER(vp)]),
    "mlkb_module_destroy": (None, [vp]),
    "mlkb_module_kind": (i32, [vp]),
    "mlkb_module_num_buffers": (i32, [vp]),
    "mlkb_module_plan": (i32, [vp, C.POINTER(i32), i32, C.c_char_p, i64]),
    "mlkb_module_run_dev": (i32, [vp, C.POINTER(vp), C.POINTER(i32), i32, i64, C.POINTER(f64), i64, i32, vp]),
    "mlkb_module_run_host": (i32, [vp, C.POINTER(vp), C.POINTER(i32), i32, i64, C.POINTER(f64), i64, i32]),
    "mlkb_module_run_sharded": (i32, [vp, C.POINTER(vp), C.POINTER(i32), i32, i64, C.POINTER(f64), i64, i32, u32]),
    "mlkb_map_sin_f32": (i32, [vp, vp, i64, vp]),
    "mlkb_map_sin_dsin_f32": (i32, [vp, vp, vp, i64, vp]),
    "mlkb_map_chain": (i32, [vp, i32, i32, vp, vp, vp, i32, i64, C.POINTER(f64), i64, vp]),
    "mlkb_chain_compile": (i32, [i32, C.POINTER(i64), C.POINTER(i64)]),
    "mlkb_chain_build": (i32, [vp, i32, i32, i32, i32]),
    "mlkb_softmax_f32": (i32, [vp, vp, i64, i64, vp]),
    "mlkb_softmax_f64": (i32, [vp, vp, i64, i64, vp]),
    "mlkb_softmax_f32_noalloc": (i32, [vp, vp, i64, i64, i32, vp]),
    "mlkb_reducesum_f32": (i32, [vp, vp, i64, i64, vp]),
    "mlkb_reducesum_f64": (i32, [vp, vp, i64, i64, vp]),
    "mlkb_gemm_f16_f32": (i32, [vp, vp, vp, i64, i64, i64, i32, vp]),
    "mlkb_gemm_f32": (i32, [vp, vp, vp, i64, i64, i64, i32, vp]),
    "mlkb_gemm_f64": (i32, [vp, vp, vp, i64, i64, i64, i32, vp]),
    "mlkb_qk_softmax_f16": (i32, [vp, vp, vp, i64, i64, i64, f64, vp]),
    "mlkb_qk_softmax_kt_f16": (i32, [vp, vp, vp, i64, i64, i64, i64, f64, vp]),
    "mlkb_fill_f32": (i32, [vp, i64, u64, u32, i32, f64, f64, vp]),
    "mlkb_fill_f16": (i32, [vp, i64, u64, u32, i32, f64, f64, vp]),
}


def declare(lib: C.CDLL) -> None:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
