"""ctypes binding of libhtrc_flat.so (the C ABI declared in include/htrc_flat.h and include/htrc_tree.h).

The library is built in-tree (``python -m htrc_b200.build``) and loaded from this package directory.
There is no fallback: if the library is missing, every operator call raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libhtrc_flat.so")

HTRC_OK, HTRC_ERR_ARG, HTRC_ERR_UNSUPPORTED, HTRC_ERR_WORKSPACE, HTRC_ERR_CUDA, HTRC_ERR_DEVICE, HTRC_ERR_TOO_LARGE = range(7)
DTYPE_F32, DTYPE_BF16 = 0, 1
ORDER_SEQ, ORDER_KMEANS = 0, 1
CURV_LIN, CURV_ISO = 0, 1
STORE_INT8, STORE_FP8, STORE_BF16 = 0, 1, 2
STORES = {"int8": STORE_INT8, "fp8": STORE_FP8, "bf16": STORE_BF16}
PREC_FP32, PREC_TF32, PREC_TRITON_DIV = 0, 1, 2      # flags, OR-ed
PRECISIONS = {"fp32": PREC_FP32, "tf32": PREC_TF32}
DIVISIONS = {"ieee": 0, "triton": PREC_TRITON_DIV}
FQ_FORMATS = {"int8": 1, "int4": 2, "fp8": 3, "fp4": 4}
ROUND_HALF_EVEN, ROUND_HALF_AWAY = 0, 1
STATUS_BITS = {1: "bounded wait gave up", 2: "routed leaf index out of range", 4: "non-finite log-partition"}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class HtrcFlatArgs(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("q_dtype", _i32), ("k", _p), ("v", _p),
        ("n_queries", _i64), ("n_keys", _i64),
        ("dim", _i32), ("tile", _i32), ("leaf", _i32), ("exact_leaves", _i32), ("sink_leaves", _i32),
        ("tile_chunk", _i32), ("scale", _f32),
        ("tail_k", _p), ("tail_v", _p), ("n_tail", _i32),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
        ("out", _p), ("lse", _p),
        ("stage_events", ctypes.POINTER(_p)), ("n_stage_events", _i32),
        ("group", _i32), ("order", _i32), ("curvature", _i32), ("store", _i32), ("qk_scale_block", _i32),
        ("route_mask", _p), ("precision", _i32),
    ]


class HtrcTreeDims(ctypes.Structure):
    """Mirror of include/htrc_tree.h HtrcTreeDims."""
    _fields_ = [("n_keys", _i64), ("n_queries", _i64), ("n_centres", _i32), ("leaf_size", _i32), ("fanout", _i32),
                ("kv_dtype", _i32), ("q_dtype", _i32), ("scale", _f32), ("threshold", _f32)]


TREE_MAX_LEVELS, TREE_MAX_CENTRES, TREE_KMEANS_CENTRES = 16, 256, 32
TREE_STAGE_ACCEPT, TREE_STAGE_LEAVES, TREE_STAGE_FINAL, TREE_STAGE_ALL = 1, 2, 4, 7

# name -> (restype, argtypes); every symbol include/htrc_flat.h and include/htrc_tree.h declare
SIGNATURES = {
    "htrc_leaf_pitch": (_i64, [_i64]),
    "htrc_flat_workspace_size": (ctypes.c_int, [ctypes.POINTER(HtrcFlatArgs), ctypes.POINTER(ctypes.c_size_t)]),
    "htrc_flat_forward": (ctypes.c_int, [ctypes.POINTER(HtrcFlatArgs), _p]),
    "htrc_flat_status": (ctypes.c_int, [_p, ctypes.POINTER(_i32), _p]),
    "htrc_pack_int8": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _p, _p, _p, _p]),
    "htrc_tile_prep": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _p, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "htrc_kmeans_scratch_size": (ctypes.c_int, [_i64, ctypes.POINTER(ctypes.c_size_t)]),
    "htrc_kmeans_order": (ctypes.c_int, [_p, _i32, _i64, _i32, _p, _p, ctypes.c_size_t, _p]),
    "htrc_leaf_stats": (ctypes.c_int, [_p, _p, _i64, _i64, _i64, _p, _p, _i64, _i32, _i32, _f32, _p, _p, _p, _p, _p, _p,
                                       _i32, _p, _p]),
    "htrc_rowmax_select": (ctypes.c_int, [_p, _p, _p, _i64, _i64, _i32, _p, _p, _p, _p, _i64, _i32, _p, _p, _p]),
    "htrc_route": (ctypes.c_int, [_p, _i64, _i64, _i32, _i32, _i32, _p, _p, _p]),
    "htrc_tile_attention": (ctypes.c_int, [_p, _p, _p, _p, _i64, _i32, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _i32,
                                           _i64, _p, _p, _p, _i64, _i32, _i32, _f32, _p, _p, _p, _p, _p, _p, _p, _p]),
    "htrc_tail_partial": (ctypes.c_int, [_p, _i32, _i64, _i32, _p, _p, _i32, _f32, _p, _p]),
    "htrc_pack_int8_blocks": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _i32, _p, _p, _p, _p]),
    "htrc_tile_prep_ex": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _p, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _i32,
                                         _i32, _p]),
    "htrc_tile_prep_fp8": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _p, _i32, _p, _p, _p, _p, _p, _i32, _p]),
    "htrc_leaf_stats_fp8": (ctypes.c_int, [_p, _p, _i64, _i64, _i64, _p, _p, _i64, _i32, _i32, _f32, _p, _p, _p, _p, _p,
                                           _i32, _p, _p]),
    "htrc_rowmax_select_fp8": (ctypes.c_int, [_p, _i64, _i64, _i32, _p, _p, _p, _i64, _i32, _p, _p, _p]),
    "htrc_tile_attention_fp8": (ctypes.c_int, [_p, _p, _i64, _i32, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _p, _i32,
                                               _i64, _p, _p, _i64, _i32, _i32, _f32, _p, _p, _p, _p, _p, _p, _p]),
    # bf16 state (htrc_flat.h: qb, dqb / gb, vbb bf16; no scales)
    "htrc_tile_prep_bf16": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _p, _i32, _p, _p, _p, _p, _p, _i32, _p]),
    "htrc_leaf_stats_bf16": (ctypes.c_int, [_p, _p, _i64, _i64, _i64, _p, _p, _i64, _i32, _i32, _f32, _p, _p, _p,
                                            _i32, _p, _p]),
    "htrc_rowmax_select_bf16": (ctypes.c_int, [_p, _i64, _i64, _i32, _p, _p, _i64, _i32, _p, _p, _p]),
    "htrc_tile_attention_bf16": (ctypes.c_int, [_p, _p, _i64, _i32, _i64, _i64, _i32, _p, _p, _p, _p, _p, _i32, _i64,
                                                _p, _p, _i64, _i32, _i32, _f32, _p, _p, _p, _p, _p, _p, _p]),
    "htrc_flat_forward_static_ws": (ctypes.c_int, [ctypes.POINTER(HtrcFlatArgs), _p]),
    "htrc_flat_static_ws_status": (ctypes.c_int, [ctypes.POINTER(_i32), _p]),
    "htrc_fake_quant": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _i32, _p, _i32, _p]),
    "htrc_dequant_rows": (ctypes.c_int, [_p, _i64, _p, _i64, _i64, _i32, _p, _p]),
    "htrc_selftest_wait_timeout": (ctypes.c_int, [_p, _i64, _p]),
    "htrc_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    # hierarchical operator (include/htrc_tree.h)
    "htrc_tree_levels": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "htrc_tree_forest_size": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), ctypes.POINTER(ctypes.c_size_t)]),
    "htrc_tree_build": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), _p, _p, _p, _p, ctypes.c_size_t, _p]),
    "htrc_tree_forest_view": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), _p, _i32] + [ctypes.POINTER(_p)] * 6),
    "htrc_tree_walk_size": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), ctypes.POINTER(ctypes.c_size_t)]),
    "htrc_tree_walk": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), _p, _p, _p, _p, _p, ctypes.c_size_t, _p, _p,
                                      _p, ctypes.POINTER(_i64), _p]),
    "htrc_tree_records_size": (ctypes.c_int, [_i64, ctypes.POINTER(ctypes.c_size_t)]),
    "htrc_tree_values": (ctypes.c_int, [ctypes.POINTER(HtrcTreeDims), _p, _p, _p, _p, _p, _p, _p, _i64,
                                        ctypes.c_size_t, _p, _p, _p, _i32, _p]),
    "htrc_tree_centres_scratch_size": (ctypes.c_int, [_i64, ctypes.POINTER(ctypes.c_size_t)]),
    "htrc_tree_centres": (ctypes.c_int, [_p, _i32, _i64, _f32, _p, _p, _p, ctypes.c_size_t, _p]),
}

_lib = None


class HtrcError(RuntimeError):
    """A CUDA-side failure reported by libhtrc_flat (launch error, no sm_100 device, device status)."""


def lib():
    """The loaded library (loaded once)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run `python -m htrc_b200.build` (no CPU fallback)")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def check(rc: int, what: str) -> None:
    """Raise the Python exception matching a library return code."""
    if rc == HTRC_OK:
        return
    msg = f"{what}: {lib().htrc_strerror(rc).decode()}"
    if rc == HTRC_ERR_ARG:
        raise ValueError(msg)
    if rc == HTRC_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc in (HTRC_ERR_WORKSPACE, HTRC_ERR_TOO_LARGE):
        raise MemoryError(msg)
    raise HtrcError(msg)


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else int(t.data_ptr())


def stream_ptr(stream=None) -> int:
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)
