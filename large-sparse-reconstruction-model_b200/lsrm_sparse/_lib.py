"""ctypes binding of liblsrm_sparse.so (the C ABI declared in
include/lsrm_sparse.h).  The library is required: there is no fallback path;
importing an op without the built library raises."""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblsrm_sparse.so")

c_int = ctypes.c_int
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t
c_void_p = ctypes.c_void_p
c_uint64 = ctypes.c_uint64

LSRM_ERR_TIMEOUT = 0x1
LSRM_ERR_DUPLICATE_BLOCK = 0x2
LSRM_ERR_CAPACITY = 0x4
LSRM_ERR_BAD_INDEX = 0x8

DENSE_COMPRESSED = 0
DENSE_INTRA_BLOCK = 1
DENSE_SLIDING = 2


class Varlen(ctypes.Structure):
    _fields_ = [
        ("num_seqs", c_int32),
        ("total_q", c_int32),
        ("total_k", c_int32),
        ("num_blocks", c_int32),
        ("cu_seqlens_q", c_void_p),
        ("cu_seqlens_k", c_void_p),
        ("cu_seqblocks", c_void_p),
        ("cu_block_include_tokens", c_void_p),
    ]


class AttnShape(ctypes.Structure):
    _fields_ = [
        ("num_q_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("dtype", c_int32),
        ("q_token_stride", c_int64),
        ("kv_token_stride", c_int64),
        ("softmax_scale", c_float),
    ]


class QkvSegment(ctypes.Structure):
    _fields_ = [("cols", c_int32), ("reserved", c_int32), ("out", c_void_p), ("out_norm", c_void_p)]


class QkvGradSegment(ctypes.Structure):
    _fields_ = [("cols", c_int32), ("reserved", c_int32), ("out_norm", c_void_p), ("grad_out", c_void_p),
                ("grad_norm", c_void_p)]


# name -> (restype, argtypes)
_SIGS = {
    "lsrm_abi_version": (c_int, []),
    "lsrm_last_error": (ctypes.c_char_p, []),
    "lsrm_launch_count": (c_uint64, []),
    "lsrm_profile_enable": (None, [c_int]),
    "lsrm_profile_collect": (c_int, []),
    "lsrm_profile_get": (c_int, [c_int, ctypes.c_char_p, c_int, ctypes.POINTER(ctypes.c_double),
                                 ctypes.POINTER(c_uint64)]),
    "lsrm_select_workspace_bytes": (c_size_t, [c_void_p, c_void_p, c_int32, c_int32]),
    "lsrm_select_attn_fwd": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p,
         c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "lsrm_select_attn_bwd": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32,
         c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "lsrm_select_attn_fwd_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p,
         c_void_p, c_void_p, c_void_p],
    ),
    "lsrm_dense_workspace_bytes": (c_size_t, [c_void_p, c_void_p, c_int32]),
    "lsrm_dense_attn_fwd": (
        c_int,
        [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_size_t, c_void_p, c_void_p],
    ),
    "lsrm_dense_attn_bwd": (
        c_int,
        [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "lsrm_block_topk_workspace_bytes": (c_size_t, [c_void_p, c_void_p, c_int32, c_int32]),
    "lsrm_block_topk": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32, ctypes.c_double,
         c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "lsrm_block_mean_fwd": (c_int, [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "lsrm_block_mean_bwd": (c_int, [c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_void_p]),
    "lsrm_resnorm_mean_fwd": (
        c_int,
        [c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p],
    ),
    "lsrm_resnorm_mean_bwd": (
        c_int,
        [c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p],
    ),
    "lsrm_gate_merge_fwd": (
        c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]
    ),
    "lsrm_gate_merge_bwd": (
        c_int,
        [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p],
    ),
    "lsrm_volume_sort_keys": (c_int, [c_int64, c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "lsrm_block_separation_workspace_bytes": (c_size_t, [c_int32, c_void_p, c_void_p, c_int32]),
    "lsrm_block_separation": (
        c_int,
        [c_int64, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_size_t, c_void_p, c_void_p],
    ),
    "lsrm_ulysses_pack": (c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int64, c_void_p, c_void_p, c_void_p]),
    "lsrm_ulysses_unpack": (
        c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p]
    ),
    "lsrm_head_layernorm_pack": (
        c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int64, ctypes.c_float, c_void_p, c_void_p, c_void_p]
    ),
    "lsrm_head_layernorm_pack_bwd": (
        c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int64, ctypes.c_float, c_void_p, c_void_p, c_void_p,
                c_void_p]
    ),
    "lsrm_volume_block_topk": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, ctypes.c_float, c_int32, c_void_p, c_void_p,
                c_void_p, c_void_p]
    ),
    "lsrm_points_volume_block_topk": (
        c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, ctypes.c_float,
                c_int32, c_void_p, c_void_p, c_void_p, c_void_p]
    ),
    "lsrm_image_sort_keys": (c_int, [c_int64, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "lsrm_voxel_points": (c_int, [c_void_p, c_int64, c_int32, ctypes.c_float, c_void_p, c_void_p]),
    "lsrm_image_token_points": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                c_void_p]
    ),
    "lsrm_view_block_topk_workspace_bytes": (
        c_int64, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int64]
    ),
    "lsrm_view_block_topk": (
        c_int, [c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int64, c_int32, c_int32, c_void_p,
                c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32, ctypes.c_float,
                c_void_p, c_void_p, c_int64, c_void_p, c_void_p]
    ),
    "lsrm_prepare_volume_output": (
        c_int, [c_void_p, c_int32, c_void_p, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                c_void_p, c_void_p, c_void_p, c_void_p]
    ),
    "lsrm_qkv_norm_fwd": (
        c_int, [c_int64, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32,
                ctypes.c_float, c_void_p, c_void_p, c_void_p]
    ),
    "lsrm_qkv_norm_bwd": (c_int, [c_int64, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_void_p]),
    "lsrm_umma_selftest": (
        c_int, [c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    ),
}

EXPORTED = tuple(_SIGS)

_lib = None
_lock = threading.Lock()


def lib():
    """Load (once) and return the ctypes handle; raises if the library is
    missing or lacks a declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python large-sparse-reconstruction-model_b200/build.py`"
                )
            h = ctypes.CDLL(LIB_PATH)
            missing = [n for n in _SIGS if not hasattr(h, n)]
            if missing:
                raise RuntimeError(f"{LIB_PATH} lacks declared entry points: {missing}")
            for name, (res, args) in _SIGS.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


class LsrmError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().lsrm_last_error().decode(errors="replace")
        raise LsrmError(f"{what or 'lsrm call'} failed ({rc}): {msg}")


def launch_count() -> int:
    return int(lib().lsrm_launch_count())


def profile_enable(on: bool = True) -> None:
    lib().lsrm_profile_enable(1 if on else 0)


def profile_collect() -> dict:
    """Per-kernel totals {name: (total_ms, launches)} since profile_enable."""
    L = lib()
    n = L.lsrm_profile_collect()
    if n < 0:
        raise LsrmError(L.lsrm_last_error().decode())
    out = {}
    buf = ctypes.create_string_buffer(128)
    for i in range(n):
        ms = ctypes.c_double()
        cnt = c_uint64()
        check(L.lsrm_profile_get(i, buf, 128, ctypes.byref(ms), ctypes.byref(cnt)), "lsrm_profile_get")
        out[buf.value.decode()] = (ms.value, int(cnt.value))
    return out
