"""ctypes binding of ``librv_b200.so`` (the sm_100a library); declarations mirror ``include/ripvec_b200.h``.

Loading fails loudly when the library has not been built: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "librv_b200.so"

RV_OK = 0
RV_E_INVALID = -1
RV_E_CUDA = -2
RV_E_NOT_READY = -3
RV_E_IO = -4
RV_E_DEVICE = -5
RV_E_NOMEM = -6
RV_E_COMM = -7
RV_COMM_ID_BYTES = 128

RV_ARCH_MODERNBERT = 1
RV_ARCH_CLASSICBERT = 2
RV_DTYPE_F32 = 0
RV_DTYPE_BF16 = 1
RV_DTYPE_F16 = 2
RV_POOL_MEAN = 0
RV_POOL_CLS = 1
RV_KIND_GEMM = 0
RV_KIND_ATTENTION = 1
RV_KIND_NORM = 2
RV_KIND_EMBED = 3
RV_KIND_POOL = 4
RV_KIND_COUNT = 5
KIND_NAMES = ["gemm_tc", "attention_varlen", "layernorm", "embed_ln", "pool_l2"]


class ModelDesc(C.Structure):
    _fields_ = [
        ("arch", C.c_int32),
        ("dtype", C.c_int32),
        ("hidden", C.c_int32),
        ("num_layers", C.c_int32),
        ("num_heads", C.c_int32),
        ("intermediate", C.c_int32),
        ("vocab", C.c_int32),
        ("max_position", C.c_int32),
        ("global_every_n", C.c_int32),
        ("local_window", C.c_int32),
        ("global_rope_theta", C.c_float),
        ("local_rope_theta", C.c_float),
        ("norm_eps", C.c_float),
        ("type_vocab", C.c_int32),
        ("pooling", C.c_int32),
        ("max_batch_tokens", C.c_int64),
    ]


vp = C.c_void_p
i32 = C.c_int32
i64 = C.c_int64
f32 = C.c_float

# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "rv_create": (C.c_int, [C.POINTER(ModelDesc), C.c_int, C.POINTER(vp)]),
    "rv_destroy": (None, [vp]),
    "rv_set_weight": (C.c_int, [vp, C.c_char_p, vp, i64]),
    "rv_load_safetensors": (C.c_int, [vp, C.c_char_p]),
    "rv_finalize": (C.c_int, [vp]),
    "rv_embed_varlen": (C.c_int, [vp, vp, vp, i32, vp]),
    "rv_embed_varlen_device": (C.c_int, [vp, vp, vp, i32, vp, i32, vp]),
    "rv_embed_submit": (C.c_int, [vp, vp, vp, i32, vp, C.POINTER(i64)]),
    "rv_embed_wait": (C.c_int, [vp, i64]),
    "rv_embed_varlen_multi": (C.c_int, [vp, i32, vp, vp, i32, vp]),
    "rv_max_tokens": (C.c_int, [vp]),
    "rv_hidden_dim": (C.c_int, [vp]),
    "rv_name": (C.c_char_p, [vp]),
    "rv_is_gpu": (C.c_int, [vp]),
    "rv_last_error": (C.c_char_p, [vp]),
    "rv_kernel_launches": (i64, [vp]),
    "rv_set_profiling": (C.c_int, [vp, C.c_int]),
    "rv_get_profile": (C.c_int, [vp, C.c_int, C.POINTER(C.c_double), C.POINTER(i64), C.POINTER(C.c_double)]),
    "rv_reset_profile": (C.c_int, [vp]),
    "rv_index_create": (C.c_int, [C.c_int, vp, i64, i32, i32, i32, C.POINTER(vp)]),
    "rv_index_destroy": (None, [vp]),
    "rv_index_last_error": (C.c_char_p, [vp]),
    "rv_index_size": (i64, [vp]),
    "rv_index_kernel_launches": (i64, [vp]),
    "rv_index_set_base": (C.c_int, [vp, i64]),
    "rv_index_topk": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_topk_device": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_topk_noalloc": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_rank": (C.c_int, [vp, vp, f32, i64, vp, vp, vp, C.POINTER(i64)]),
    "rv_comm_get_unique_id": (C.c_int, [vp]),
    "rv_comm_create": (C.c_int, [C.c_int, vp, i32, i32, i32, C.POINTER(vp)]),
    "rv_comm_destroy": (None, [vp]),
    "rv_comm_last_error": (C.c_char_p, [vp]),
    "rv_comm_rank": (C.c_int, [vp]),
    "rv_comm_world": (C.c_int, [vp]),
    "rv_index_topk_sharded": (C.c_int, [vp, vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_topk_merge_device": (C.c_int, [C.c_int, vp, vp, i32, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_build_polar": (C.c_int, [vp, vp, i32]),
    "rv_index_has_polar": (C.c_int, [vp]),
    "rv_index_polar_export": (C.c_int, [vp, vp, vp]),
    "rv_index_polar_scores": (C.c_int, [vp, vp, i32, vp]),
    "rv_index_rank_turboquant": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_rank_turboquant_device": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_build_cascade": (C.c_int, [vp, i32]),
    "rv_index_cascade_dim": (C.c_int, [vp]),
    "rv_index_cascade_rows": (C.c_int, [vp, vp]),
    "rv_index_rank_cascade": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp, vp]),
    "rv_index_find_duplicates": (C.c_int, [vp, f32, i64, vp, vp, vp, vp, vp]),
    "rv_cache_decode": (C.c_int, [vp, C.c_uint64, vp, i64, C.POINTER(i64), C.POINTER(i32)]),
    "rv_cache_last_error": (C.c_char_p, []),
    "rv_index_export": (C.c_int, [vp, i64, i64, i32, vp, i32]),
    "rv_op_gemm": (C.c_int, [i32, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "rv_op_attention": (C.c_int, [i32, vp, vp, vp, i32, i32, i32, i32, f32, vp]),
    "rv_debug_stall_attention": (C.c_int, [i32, i64]),
    "rv_debug_exp2_poly": (C.c_int, [vp, vp, i64, vp]),
    "rv_op_layernorm": (C.c_int, [i32, vp, vp, i32, i32, vp, vp, f32, vp]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the library once.  Raises when it is missing (build it with ``python -m ripvec_b200.build``)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the sm_100a library with `python -m ripvec_b200.build`"
                " (there is no CPU fallback)")
        l = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


class RvError(RuntimeError):
    """A non-zero status from the library, carrying the code and the handle's last message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ripvec_b200 error {code}: {msg}")
        self.code = code


def ptr(a) -> int | None:
    """Address of a numpy array's data, or of a torch tensor's storage."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data
