"""ctypes binding of libb2d.so (include/b2d_decode.h).

The structures below mirror b2d_gqa_args / b2d_mla_args field for field.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libb2d.so"

B2D_KV_STRIDED, B2D_KV_VLLM = 0, 1
B2D_BF16, B2D_FP16, B2D_FP8_E4M3, B2D_FP32 = 0, 1, 2, 3
B2D_FLAG_SKIP_COMBINE, B2D_FLAG_COMBINE_ONLY, B2D_FLAG_TEST_NO_LOADS = 1, 2, 4
B2D_WORKSPACE_HEADER_BYTES = 65792

EXPORTED = (
    "b2d_gqa_workspace_bytes",
    "b2d_decode_gqa",
    "b2d_decode_gqa_static_scratch",
    "b2d_mla_workspace_bytes",
    "b2d_decode_mla",
    "b2d_check_device_status",
    "b2d_append_kv",
    "b2d_gqa_plan",
    "b2d_error_string",
    "b2d_version",
)


class GqaArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("q_stride_b", C.c_int64), ("q_stride_h", C.c_int64),
        ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
        ("k_stride_page", C.c_int64), ("k_stride_tok", C.c_int64), ("k_stride_head", C.c_int64),
        ("v_stride_page", C.c_int64), ("v_stride_tok", C.c_int64), ("v_stride_head", C.c_int64),
        ("num_pages", C.c_int64),
        ("cache_seqlens", C.c_void_p), ("block_table", C.c_void_p),
        ("block_table_stride", C.c_int64),
        ("k_scale", C.c_void_p), ("v_scale", C.c_void_p),
        ("out", C.c_void_p), ("out_stride_b", C.c_int64), ("out_stride_h", C.c_int64),
        ("lse", C.c_void_p), ("lse_stride_b", C.c_int64),
        ("batch", C.c_int32), ("num_q_heads", C.c_int32), ("num_kv_heads", C.c_int32),
        ("head_dim", C.c_int32), ("page_size", C.c_int32), ("max_pages_per_seq", C.c_int32),
        ("q_dtype", C.c_int32), ("kv_dtype", C.c_int32),
        ("softmax_scale", C.c_float),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("num_ctas", C.c_int32), ("flags", C.c_int32), ("kv_layout", C.c_int32),
        ("wait_limit_us", C.c_int32),
    ]


class MlaArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("q_stride_b", C.c_int64), ("q_stride_h", C.c_int64),
        ("kv_cache", C.c_void_p), ("kv_stride_page", C.c_int64), ("kv_stride_tok", C.c_int64),
        ("num_pages", C.c_int64),
        ("cache_seqlens", C.c_void_p), ("block_table", C.c_void_p),
        ("block_table_stride", C.c_int64),
        ("out", C.c_void_p), ("out_stride_b", C.c_int64), ("out_stride_h", C.c_int64),
        ("lse", C.c_void_p), ("lse_stride_b", C.c_int64),
        ("batch", C.c_int32), ("num_heads", C.c_int32), ("head_dim_qk", C.c_int32),
        ("head_dim_v", C.c_int32), ("page_size", C.c_int32), ("max_pages_per_seq", C.c_int32),
        ("dtype", C.c_int32), ("softmax_scale", C.c_float),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("num_ctas", C.c_int32), ("flags", C.c_int32), ("wait_limit_us", C.c_int32),
        ("reserved", C.c_int32),
    ]


class AppendArgs(C.Structure):
    _fields_ = [
        ("key", C.c_void_p), ("value", C.c_void_p),
        ("src_stride_t", C.c_int64), ("src_stride_h", C.c_int64),
        ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
        ("k_stride_page", C.c_int64), ("k_stride_tok", C.c_int64), ("k_stride_head", C.c_int64),
        ("v_stride_page", C.c_int64), ("v_stride_tok", C.c_int64), ("v_stride_head", C.c_int64),
        ("num_pages", C.c_int64), ("slot_mapping", C.c_void_p),
        ("k_scale", C.c_void_p), ("v_scale", C.c_void_p), ("bad_slots", C.c_void_p),
        ("num_tokens", C.c_int32), ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32),
        ("page_size", C.c_int32), ("src_dtype", C.c_int32), ("cache_dtype", C.c_int32),
        ("kv_layout", C.c_int32), ("reserved", C.c_int32),
    ]


_lib = None


def load() -> C.CDLL:
    """Load libb2d.so once; raise (never fall back) when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("B2D_LIBRARY", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"libb2d.so not found at {path}; build it with "
            "`python roofline-analysis_b200/build.py` (there is no CPU fallback)")
    lib = C.CDLL(str(path))
    lib.b2d_gqa_workspace_bytes.argtypes = [C.POINTER(GqaArgs), C.POINTER(C.c_size_t)]
    lib.b2d_decode_gqa.argtypes = [C.POINTER(GqaArgs), C.c_void_p]
    lib.b2d_decode_gqa_static_scratch.argtypes = [C.POINTER(GqaArgs), C.c_void_p]
    lib.b2d_mla_workspace_bytes.argtypes = [C.POINTER(MlaArgs), C.POINTER(C.c_size_t)]
    lib.b2d_decode_mla.argtypes = [C.POINTER(MlaArgs), C.c_void_p]
    lib.b2d_append_kv.argtypes = [C.POINTER(AppendArgs), C.c_void_p]
    lib.b2d_check_device_status.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    lib.b2d_static_scratch_check_status.argtypes = [C.c_int, C.c_void_p]
    lib.b2d_gqa_launch_count.argtypes = [C.POINTER(GqaArgs), C.POINTER(C.c_int32)]
    lib.b2d_gqa_plan.argtypes = [C.POINTER(GqaArgs), C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                 C.POINTER(C.c_int32)]
    lib.b2d_error_string.restype = C.c_char_p
    lib.b2d_error_string.argtypes = [C.c_int]
    lib.b2d_version.restype = C.c_char_p
    _lib = lib
    return lib
