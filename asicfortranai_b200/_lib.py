"""ctypes binding of libq35.so (the C ABI declared in include/q35.h).

The library is the product: there is no Python or CPU fallback.  Importing this module
on a machine without the built library raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libq35.so")

Q35_OK = 0
Q35_FMT_3P5BIT = 0
Q35_FMT_INT4 = 1
Q35_LAYOUT_COLMAJOR = 0
Q35_LAYOUT_ROWMAJOR = 1

_vp, _i32, _i64, _sz = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t

# name -> (restype, argtypes); every symbol include/q35.h declares
SIGNATURES = {
    "q35_last_error": (C.c_char_p, []),
    "q35_status_string": (C.c_char_p, [C.c_int]),
    "q35_version": (C.c_int, []),
    "q35_ctx_create": (C.c_int, [C.c_int, _vp, C.POINTER(_vp)]),
    "q35_ctx_destroy": (C.c_int, [_vp]),
    "q35_ctx_synchronize": (C.c_int, [_vp]),
    "q35_ctx_set_gemm_path": (C.c_int, [_vp, C.c_int]),
    "q35_ctx_stream": (_vp, [_vp]),
    "q35_ctx_device_error": (C.c_int, [_vp]),
    "q35_ctx_capture_begin": (C.c_int, [_vp]),
    "q35_ctx_capture_end": (C.c_int, [_vp, C.POINTER(_vp)]),
    "q35_graph_launch": (C.c_int, [_vp, _vp]),
    "q35_graph_destroy": (C.c_int, [_vp]),
    "q35_weights_upload": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _i32, _i32, C.c_int, C.POINTER(_vp)]),
    "q35_weights_free": (C.c_int, [_vp]),
    "q35_weights_device_bytes": (_sz, [_vp]),
    "q35_weights_download_ref": (C.c_int, [_vp, _vp, _vp]),
    "q35_gemm_dev": (C.c_int, [_vp, _vp, _vp, _i32, C.c_int, _vp, _vp, C.c_int]),
    "q35_matmul_cached": (C.c_int, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "q35_gemm_dev_noalloc": (C.c_int, [_vp, _vp, _i32, C.c_int, _vp, _vp, C.c_int, _vp]),
    "q35_gemm_noalloc_device_error": (C.c_int, [_vp]),
    "matmul_3p5bit_awq": (None, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32]),
    "q35_dequantize_output_3p5bit": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32]),
    "q35_matmul_int4_awq": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32]),
    "q35_dequantize_output": (C.c_int, [_vp, _vp, _vp, _i32, _i32]),
    "q35_matmul_3p5bit_awq": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32]),
    "q35_matmul_int4_fused": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32]),
    "q35_dropin_cache_stats": (C.c_int, [_vp, _vp, _vp, _vp]),
    "q35_dropin_cache_clear": (C.c_int, []),
    "q35_rms_norm": (C.c_int, [_vp, _vp, _vp, _i32, _i32]),
    "q35_gen_int8_dev": (C.c_int, [_vp, _i64, C.c_uint64, C.c_uint64, _vp]),
    "q35_gen_normal_dev": (C.c_int, [_vp, _i64, C.c_uint64, C.c_uint64, C.c_double, _vp]),
    "q35_gen_tokens_dev": (C.c_int, [_vp, _i64, C.c_uint64, C.c_uint64, _i32, _vp]),
    "q35_quantize_dev": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _i32, _i32, _vp]),
    "q35_weights_generate": (C.c_int, [_vp, C.c_int, _i32, _i32, C.c_uint64, C.c_uint64, C.c_double,
                                       C.POINTER(_vp)]),
    "q35_tp_unique_id": (C.c_int, [_vp, _sz]),
    "q35_tp_create": (C.c_int, [_vp, _i32, _i32, _vp, _sz, C.c_double, C.POINTER(_vp)]),
    "q35_tp_destroy": (C.c_int, [_vp]),
    "q35_tp_abort": (C.c_int, [_vp]),
    "q35_tp_rank": (C.c_int, [_vp]),
    "q35_tp_world": (C.c_int, [_vp]),
    "q35_tp_allreduce_i32": (C.c_int, [_vp, _vp, _vp, _sz]),
    "q35_tp_allreduce_dequant": (C.c_int, [_vp, _vp, _vp, C.c_int64, C.c_int32, _vp, _vp, _vp]),
    "q35_tp_wait_selftest": (C.c_int, [_vp, _vp]),
    "q35_tp_norm_selftest": (C.c_int, [_vp, C.c_int32, C.c_uint64, _vp]),
    "q35_tp_norm_selftest_rows": (C.c_int, [_vp, _i32, _i32, C.c_uint64, _vp]),
    "q35_sample_greedy": (C.c_int, [_vp, _vp, _i32, _vp]),
    "q35_sample_temperature": (C.c_int, [_vp, _vp, _i32, C.c_float, C.c_float, _vp]),
    "q35_sample_top_k": (C.c_int, [_vp, _vp, _i32, _i32, C.c_float, _vp]),
    "q35_sample_top_p": (C.c_int, [_vp, _vp, _i32, C.c_float, C.c_float, _vp]),
    "q35_sample_dev": (C.c_int, [_vp, _i32, _vp, _i32, _i32, C.c_float, _i32, C.c_float, _vp, _vp]),
    "q35_model_set_sampling": (C.c_int, [_vp, _vp]),
    "q35_model_create": (C.c_int, [_vp, _vp, C.POINTER(_vp)]),
    "q35_model_create_tp": (C.c_int, [_vp, _vp, _vp, C.POINTER(_vp)]),
    "q35_model_destroy": (C.c_int, [_vp]),
    "q35_model_set_layer": (C.c_int, [_vp, _i32, _vp]),
    "q35_model_set_embeddings": (C.c_int, [_vp, _vp, _vp, _vp]),
    "q35_model_load_layer_file": (C.c_int, [_vp, _i32, C.c_char_p]),
    "q35_model_load_safetensors": (C.c_int, [_vp, _vp, _i32]),
    "q35_model_init_random": (C.c_int, [_vp, C.c_uint64, C.c_double]),
    "q35_model_reset": (C.c_int, [_vp]),
    "q35_model_forward": (C.c_int, [_vp, _i32, _vp, _i32, _vp]),
    "q35_model_last_tokens": (C.c_int, [_vp, _vp]),
    "q35_model_decode_step": (C.c_int, [_vp, _vp, _vp, _vp]),
    "q35_model_decode_steps_async": (C.c_int, [_vp, _i32]),
    "q35_model_generate": (C.c_int, [_vp, _vp, _i32, _i32, _i32, _vp, _vp]),
    "q35_model_layer_forward": (C.c_int, [_vp, _i32, _i32, _vp, _i32, _vp, _i32]),
    "q35_model_weight_bytes": (_sz, [_vp]),
    "q35_model_debug_buffer": (C.c_int, [_vp, C.c_char_p, _vp, _sz]),
}

_lib = None


class Q35Error(RuntimeError):
    pass


def load():
    """Load libq35.so (built in-tree by asicfortranai_b200/build.py); raise if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise Q35Error(f"libq35.so not built ({LIB_PATH}); run python -m asicfortranai_b200.build")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str = "") -> None:
    if status != Q35_OK:
        lib = load()
        msg = lib.q35_last_error().decode(errors="replace")
        kind = lib.q35_status_string(status).decode()
        raise Q35Error(f"{what}: {kind} ({status}): {msg}")


def last_error() -> str:
    return load().q35_last_error().decode(errors="replace")
