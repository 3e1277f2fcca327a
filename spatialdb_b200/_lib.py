"""ctypes binding of libslx.so (include/slx.h).

The library is built in-tree on first use (nvcc for sm_100a). There is no fallback: if the CUDA
library cannot be built or loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

I64P = ctypes.POINTER(ctypes.c_int64)
I32P = ctypes.POINTER(ctypes.c_int32)
U8P = ctypes.POINTER(ctypes.c_uint8)
F32P = ctypes.POINTER(ctypes.c_float)
U64P = ctypes.POINTER(ctypes.c_uint64)
VP = ctypes.c_void_p
i, i64, f32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float

# name -> (restype, argtypes); kept in the order of include/slx.h
SIGNATURES = {
    "slx_init": (i, [i, ctypes.POINTER(VP)]),
    "slx_destroy": (i, [VP]),
    "slx_last_error": (ctypes.c_char_p, [VP]),
    "slx_version": (ctypes.c_char_p, []),
    "slx_ctx_status": (i, [VP, VP]),
    "slx_ctx_set_option": (i, [VP, i, i64]),
    "slx_gguf_read_f32": (i, [VP, ctypes.c_char_p, ctypes.c_char_p, F32P, i64]),
    "slx_dequantize": (i, [VP, i, U8P, i64, F32P, i64]),
    "slx_model_load_gguf": (i, [VP, ctypes.c_char_p, i, i, ctypes.POINTER(VP)]),
    "slx_model_free": (i, [VP]),
    "slx_model_info": (i, [VP, I32P, i]),
    "slx_encode": (i, [VP, I32P, i, i, I64P, F32P]),
    "slx_encode_device": (i, [VP, VP, i, i, VP, VP]),
    "slx_trace_hidden": (i, [VP, I32P, i, i, i, I64P]),
    "slx_causal_forward_last": (i, [VP, I32P, i, I64P]),
    "slx_causal_next_token": (i, [VP, I32P, i, i, I32P]),
    "slx_causal_generate": (i, [VP, I32P, i, i, i, I32P, I32P]),
    "slx_causal_next_token_lattice": (i, [VP, I32P, i, i, i, I32P]),
    "slx_causal_generate_lattice": (i, [VP, I32P, i, i, i, i, I32P, I32P]),
    "slx_vocab_lattice_query": (i, [VP, F32P, i, i, I32P, U64P]),
    "slx_matmul_q30": (i, [VP, I64P, i, i, i, U8P, i64, i, i, i, i, I64P]),
    "slx_matmul_q30_device": (i, [VP, VP, i, i, i, VP, i64, i, i, i, i, VP, VP]),
    "slx_weight_prepare": (i, [VP, VP, i64, i, i, i, i, i, ctypes.POINTER(VP)]),
    "slx_weight_free": (i, [VP]),
    "slx_weight_info": (i, [VP, I32P, i]),
    "slx_matmul_q30_prepared": (i, [VP, VP, i, i, VP, VP]),
    "slx_matmul_q30_noalloc": (i, [VP, i, i, i, VP, i64, i, i, i, i, VP, VP]),
    "slx_attention": (i, [VP, I64P, I64P, I64P, i, i, i, i, i, i, i, i, I64P]),
    "slx_lattice_build": (i, [VP, F32P, i64, i, f32, i64, i64, ctypes.POINTER(VP)]),
    "slx_lattice_build_device": (i, [VP, VP, i64, i, f32, i64, i64, VP, ctypes.POINTER(VP)]),
    "slx_lattice_free": (i, [VP]),
    "slx_lattice_info": (i, [VP, I64P, i]),
    "slx_lattice_build_tree": (i, [VP, i]),
    "slx_lattice_tree_info": (i, [VP, I64P, i]),
    "slx_lattice_tree_export": (i, [VP, I32P, I32P, I32P, I64P, I64P, I64P, I32P]),
    "slx_lattice_save_slat": (i, [VP, ctypes.c_char_p]),
    "slx_lattice_save_slat_mem": (i, [VP, U8P, i64, I64P]),
    "slx_lattice_load_slat": (i, [VP, ctypes.c_char_p, f32, i64, ctypes.POINTER(VP)]),
    "slx_lattice_load_slat_mem": (i, [VP, U8P, i64, f32, i64, ctypes.POINTER(VP)]),
    "slx_lattice_query_knn_l2": (i, [VP, F32P, i, i, i, I64P, U64P, ctypes.POINTER(i)]),
    "slx_lattice_query_knn_l2_device": (i, [VP, VP, i, i, i, VP, VP, ctypes.POINTER(i), VP]),
    "slx_knn_merge_device": (i, [VP, VP, VP, i, i, i, VP, VP, VP]),
    "slx_profile_begin": (i, [VP]),
    "slx_profile_end": (i, [VP, VP, i, ctypes.POINTER(i)]),
    "slx_launch_count": (i, [VP, I64P]),
}


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 24), ("launches", ctypes.c_int64), ("ms", ctypes.c_double),
                ("macs", ctypes.c_double), ("bytes", ctypes.c_double), ("tc_macs", ctypes.c_double)]


def header_symbols() -> list[str]:
    """Function names declared in include/slx.h."""
    src = open(os.path.join(_build.INCLUDE, "slx.h")).read()
    return re.findall(r"^\s*(?:slx_status|const char\*)\s+(slx_\w+)\s*\(", src, re.M)


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            path = _build.build()
            cdll = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(cdll, name)
                fn.restype = res
                fn.argtypes = args
            _lib = cdll
    return _lib


def library_path() -> str:
    return _build.LIB
