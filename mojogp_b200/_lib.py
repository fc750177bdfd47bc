"""ctypes binding of the gpb200 C ABI (include/gpb200.h).

The shared library is built in-tree (mojogp_b200/libgpb200.so) by
mojogp_b200/build.py. There is no fallback: if the library is missing or
fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libgpb200.so"
_lib = None

c_int, c_i32, c_i64, c_f32, c_f64 = C.c_int, C.c_int32, C.c_int64, C.c_float, C.c_double
P = C.c_void_p
PF = C.POINTER(C.c_float)
PD = C.POINTER(C.c_double)
PI32 = C.POINTER(C.c_int32)
PI64 = C.POINTER(C.c_int64)
PP = C.POINTER(C.c_void_p)

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "gpb_version": [],
    "gpb_last_error": [C.c_char_p, c_i64],
    "gpb_device_count": [PI32],
    "gpb_device_alloc": [c_i32, c_i64, PP],
    "gpb_device_free": [c_i32, P],
    "gpb_memcpy_h2d": [c_i32, P, P, c_i64],
    "gpb_memcpy_d2h": [c_i32, P, P, c_i64],
    "gpb_host_register": [P, c_i64],
    "gpb_host_unregister": [P],
    "gpb_memset_d": [c_i32, P, c_i32, c_i64],
    "gpb_provider_create": [P, c_i64, c_i32, P, c_i32, P, c_i32, c_f32, P, c_i32, PP],
    "gpb_provider_destroy": [P],
    "gpb_provider_synchronize": [P],
    "gpb_update_params": [P, P, c_i32],
    "gpb_update_noise": [P, c_f32],
    "gpb_get_noise": [P, PF],
    "gpb_get_noise_mode": [P, PI32],
    "gpb_get_num_params": [P, PI32],
    "gpb_get_params": [P, P, c_i32],
    "gpb_get_diagonal_value": [P, PF],
    "gpb_get_x_ptr": [P, PP],
    "gpb_forward_matvec": [P, P, P, c_i64],
    "gpb_matvec_layout": [P, c_i64, P],
    "gpb_forward_matvec_rows": [P, P, P, c_i64, c_i64, c_i64],
    "gpb_forward_matvec_host": [P, P, P, c_i64],
    "gpb_cross_matvec": [P, P, P, P, c_i64, c_i64],
    "gpb_extract_diagonal": [P, P],
    "gpb_extract_diagonal_test": [P, P, P, c_i64],
    "gpb_kernel_column": [P, P, c_i64],
    "gpb_gradient_matvec": [P, P, P, c_i64, c_i32],
    "gpb_fused_gradient_matvec": [P, P, P, c_i64],
    "gpb_gradient_bilinear": [P, P, P, c_i64, P, P],
    "gpb_benchmark_forward": [P, P, P, c_i64, c_i32, c_i32, c_i32, P, P, P],
    "gpb_measure_fp32_peak": [c_i32, PD, PD],
    "gpb_comm_unique_id": [P],
    "gpb_comm_init": [P, c_i32, c_i32, c_i32, PP],
    "gpb_comm_destroy": [P],
    "gpb_comm_allreduce_max_f64": [P, PD],
    "gpb_comm_allreduce_sum_f64": [P, P, c_i64],
    "gpb_comm_barrier": [P],
    "gpb_benchmark_forward_sharded": [P, P, P, c_i64, c_i32, c_i32, c_i32, P, P, P],
    "gpb_train": [P, P, P, c_i64, P, P],
    "gpb_bbmm": [P, P, P, c_i64, c_i32, c_i32, c_i32, c_f32, c_i32, c_i32, P, P, P, P, P],
    "gpb_precond_pivots": [P, P, c_i32, P, P, PI32],
    "gpb_matvec_sharded": [P, P, P, P, c_i64],
    "gpb_slq_logdet": [P, P, c_i32, c_i32, c_i64, P],
    "gpb_tridiag_eig": [P, P, c_i32, P, P],
    "gpb_hash_gaussian": [c_i32, P, c_i64, C.c_uint64],
    "gpb_compute_alpha": [P, P, P, c_i64, c_i32, c_f32, P, PI32],
    "gpb_prediction_cache_create": [P, P, P, c_f32, c_i32, P, PP],
    "gpb_prediction_cache_root": [P, P],
    "gpb_predict_with_cache": [P, P, c_i64, P, P],
    "gpb_prediction_cache_destroy": [P],
    "gpb_forward_matvec_noalloc": [P, P, P, c_i64],
    "gpb_device_mem_info": [c_i32, P, P],
    "gpb_tc_selftest": [c_i32, c_i32, P, P, P],
    "gpb_predict_exact_variance": [P, P, P, c_i64, c_i32, c_i32, c_f32, c_i32, P, PI32],
    "gpb_lmc_create": [P, c_i32, c_i32, PP],
    "gpb_lmc_create_sharded": [P, c_i32, c_i32, P, PP],
    "gpb_lmc_destroy": [P],
    "gpb_lmc_set_coregion": [P, P, P],
    "gpb_lmc_matvec": [P, P, P, c_i64],
    "gpb_lmc_bbmm": [P, P, c_i32, c_i32, c_i32, c_f32, c_i32, c_i32, P, P, P, P, P, P, PI32],
    "gpb_lmc_solve": [P, P, c_i32, c_f32, P, PI32],
    "gpb_lmc_build_precond": [P, c_i32, PI32, P],
    "gpb_lmc_precond_apply": [P, P, P, c_i64],
    "gpb_lmc_precond_sample": [P, P, c_i32, C.c_uint64],
    "gpb_lmc_predict_exact_variance": [P, P, c_i64, c_i32, c_i32, c_f32, P, PI32],
}
_RESTYPES = {"gpb_version": C.c_char_p}

ERR_INVALID = -1


class GPBError(RuntimeError):
    """Raised when a gpb200 call returns a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> C.CDLL:
    """Load (once) and return the CUDA library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("GPB200_LIBRARY", _LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"gpb200 CUDA library not found at {path}; build it with "
            "`python -m mojogp_b200.build` (there is no CPU fallback)"
        )
    handle = C.CDLL(str(path))
    for name, args in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, c_int)
    _lib = handle
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().gpb_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != 0:
        msg = last_error()
        if status == ERR_INVALID:
            raise ValueError(msg)
        raise GPBError(status, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def declared_symbols(header: Path) -> list[str]:
    """Function names declared in a C header (used by the ABI tests)."""
    import re

    text = header.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\*|int)\s+(gpb_\w+)\s*\(", text, re.M)))
