"""ctypes binding of libabra_b200.so (the C ABI in include/abra_b200.h).

The shared library is built in-tree by ``python -m abra_b200.build``.  There
is no fallback: if the library is missing or does not load, importing this
module raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libabra_b200.so"

ABRA_OK = 0
ABRA_E_INVALID = -1
ABRA_E_CUDA = -2
ABRA_E_UNSUPPORTED = -3
ABRA_MMVQ_PDL = 1

_vp, _i32, _i64, _u64, _f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float
_fp = C.c_void_p  # float* passed as an address

# name -> (restype, argtypes); every symbol declared in include/abra_b200.h
SIGNATURES: dict[str, tuple] = {
    "abra_version": (C.c_char_p, []),
    "abra_last_error": (C.c_char_p, []),
    "abra_device_error": (C.c_int, [C.POINTER(C.c_uint32), _i32]),
    "abra_test_flag_timeout": (C.c_int, [C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)]),
    "abra_q4k_mmvq": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _vp]),
    "abra_q4k_pack": (C.c_int, [_vp, _vp, _i64, _vp]),
    "abra_q4k_mmvq_packed": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i32, _vp]),
    "abra_q4k_mmvq_candidate": (C.c_int, [_i32, _vp, _vp, _fp, _i64, _i64, _i32, _vp]),
    "abra_q4k_mmvq_ex": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _i64, _i32, _i32, _vp]),
    "abra_q4k_mmvq_swiglu": (C.c_int, [_vp, _vp, _vp, _fp, _i64, _i64, _i32, _i64, _i32, _i32, _vp]),
    "abra_q4k_mmvq_partials": (C.c_int, [_vp, _vp, _fp, _vp, _vp, _i64, _i64, _i32, _i32, _vp]),
    "launch_pinned_upstream_mmvq": (None, [_vp, _vp, _fp, _i64, _i64, _vp]),
    "abra_quantize_q8_1": (C.c_int, [_fp, _vp, _i64, _i32, _vp]),
    "abra_q4k_mmvq_tc": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _i64, _i32, _fp, _i32, _vp]),
    "abra_q4k_mmvq_kshard": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _i64, _i32, _i32, _i32, _i32, _vp]),
    "abra_q4k_mmvq_combined": (C.c_int, [_i32, _vp, _fp, _vp, _fp, _i64, _i64, _i32, _vp]),
    "abra_q4k_mmvq_combined_static": (C.c_int, [_i32, _vp, _fp, _fp, _i64, _i64, _i32, _vp]),
    "launch_pinned_upstream_q8_1_quantize": (None, [_fp, _vp, _i64, _vp]),
    "quantize_row_q4_K_upstream_cpu": (None, [_vp, _vp, _i64]),
    "dequantize_row_q4_K_upstream_cpu": (None, [_vp, _vp, _i64]),
    "abra_rmsnorm_quantize_q8_1": (C.c_int, [_fp, _fp, _f32, _vp, _fp, _i64, _i32, _vp]),
    "abra_gen_q4k": (C.c_int, [_vp, _i64, _u64, _u64, _i64, _vp]),
    "abra_gen_uniform_f32": (C.c_int, [_fp, _i64, _u64, _u64, _i64, _f32, _f32, _vp]),
    "abra_candidate_count": (C.c_int, []),
    "abra_candidate_info": (C.c_int, [_i32] + [C.POINTER(C.c_int32)] * 6),
    "abra_tune_set": (C.c_int, [_i64, _i64, _i32, _i32, _i32]),
    "abra_tune_get": (C.c_int, [_i64, _i64, _i32, _i32]),
    "abra_tune_clear": (C.c_int, []),
    # Q6_K
    "abra_q6k_mmvq": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _vp]),
    "abra_q6k_mmvq_ex": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _i64, _i32, _i32, _vp]),
    "abra_q6k_mmvq_kshard": (C.c_int, [_vp, _vp, _fp, _i64, _i64, _i32, _i64, _i32, _i32, _i32, _i32, _vp]),
    "abra_q6k_mmvq_partials": (C.c_int, [_vp, _vp, _fp, _vp, _i64, _i64, _i32, _vp]),
    "abra_gen_q6k": (C.c_int, [_vp, _i64, _u64, _u64, _i64, _vp]),
    "abra_q6k_candidate_count": (C.c_int, []),
    "abra_q6k_candidate_info": (C.c_int, [_i32] + [C.POINTER(C.c_int32)] * 5),
    "abra_q6k_tune_set": (C.c_int, [_i64, _i64, _i32, _i32]),
    "abra_q6k_tune_get": (C.c_int, [_i64, _i64, _i32]),
    "abra_q4k_mmvq_rmsnorm": (C.c_int, [_vp, _vp, _fp, _fp, _f32, _fp, _vp, _i64, _i64, _i32, _i32,
                                        _vp]),
    "abra_mmvq_plan_info": (C.c_int, [_i32, _i32, _i64, _i64, _i32, _i32, _i32, _i64, _i32, _i32,
                                      _i32, _vp]),
    # decode model
    "abra_model_default_config": (C.c_int, [_vp]),
    "abra_model_create": (C.c_int, [_vp, C.POINTER(C.c_void_p)]),
    "abra_model_destroy": (C.c_int, [_vp]),
    "abra_model_reset": (C.c_int, [_vp, _vp, _i32]),
    "abra_model_step": (C.c_int, [_vp, _i32]),
    "abra_model_prefill": (C.c_int, [_vp, _i32]),
    "abra_lookup_draft": (C.c_int, [_vp, _i32, _i32, _i32, _vp]),
    "abra_model_verify": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "abra_model_generate_lookup": (C.c_int, [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp]),
    "abra_model_sync": (C.c_int, [_vp]),
    "abra_model_invalidate": (C.c_int, [_vp]),
    "abra_model_read": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "abra_model_generate": (C.c_int, [_vp, _vp, _i32, _i32, _vp]),
    "abra_model_decode_streaming": (C.c_int, [_vp, _i32, _vp]),
    "abra_model_info": (C.c_int, [_vp, C.POINTER(C.c_void_p), C.POINTER(C.c_uint64),
                                  C.POINTER(C.c_uint64)]),
    "abra_model_last_error": (C.c_char_p, []),
    "abra_model_create_batched": (C.c_int, [_vp, _i32, C.POINTER(C.c_void_p)]),
    "abra_model_create_batched_tp": (C.c_int, [_vp, _i32, _i32, _i32, C.POINTER(C.c_void_p)]),
    "abra_model_reset_batched": (C.c_int, [_vp, _vp, _i32]),
    "abra_model_read_batched": (C.c_int, [_vp, _vp, _i32, _vp]),
    "abra_tp_shard_info": (C.c_int, [_vp, _i32, _i32, _vp]),
    "abra_model_create_tp": (C.c_int, [_vp, _i32, _i32, C.POINTER(C.c_void_p)]),
    "abra_model_tp_handle": (C.c_int, [_vp, _vp, _i32]),
    "abra_model_tp_connect": (C.c_int, [_vp, _vp, _i32]),
    "abra_model_load_tensor": (C.c_int, [_vp, _i32, _i32, _i32, _vp, C.c_uint64]),
    "abra_tp_tensor_slice": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _vp]),
    "abra_model_path": (C.c_int, [_vp, C.POINTER(C.c_int32)]),
    "abra_persist_plan": (C.c_int, [_vp, _i32, _vp]),
}


class AbraError(RuntimeError):
    """A C-ABI call returned an error code."""

    def __init__(self, code: int, func: str, msg: str):
        super().__init__(f"{func} failed ({code}): {msg}")
        self.code = code


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python abra_b200/build.py` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    msg = lib.abra_last_error()
    return msg.decode() if msg else ""


def check(rc: int, func: str) -> None:
    if rc != ABRA_OK:
        msg = last_error()
        if rc == ABRA_E_INVALID:
            raise ValueError(f"{func}: {msg}")
        raise AbraError(rc, func, msg)


def call(name: str, *args) -> int:
    rc = getattr(lib, name)(*args)
    check(rc, name)
    return rc
