"""ctypes bindings of libp2pattn.so (the C ABI in include/p2p_attn.h).

Loading the library needs no GPU; every compute entry point needs one.  There is no CPU
fallback: if the shared library is missing this module raises at import time.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("P2P_ATTN_LIB", _PKG / "libp2pattn.so"))

P2P_OK = 0
P2P_ERR_INVALID_ARG = 1
P2P_ERR_OOM = 2
P2P_ERR_KV_FULL = 3
P2P_ERR_CUDA = 4
P2P_ERR_TIMEOUT = 5
P2P_ERR_NCCL = 6
P2P_ERR_UNSUPPORTED = 7

P2P_F16 = 0
P2P_F32 = 1
MAX_LAYERS = 16
P2P_IPC_HANDLE_BYTES = 64
P2P_COMM_ID_BYTES = 128


class P2PError(RuntimeError):
    """A non-OK p2p_status; `.status` holds the code, the message is p2p_last_error()."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[{status}] {msg}")
        self.status = status


class KvFullError(P2PError):
    """P2P_ERR_KV_FULL: the engine reports this as reason 'kv_full' (engine.js:418-421)."""


class OomError(P2PError):
    """P2P_ERR_OOM."""


class AttnParams(C.Structure):
    _fields_ = [
        ("num_heads", C.c_int32),
        ("num_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("scale", C.c_float),
        ("eps", C.c_float),
        ("dtype", C.c_int32),
    ]


class KvLayout(C.Structure):
    _fields_ = [
        ("format", C.c_int32),
        ("k_scale", C.c_void_p),
        ("v_scale", C.c_void_p),
        ("scale_count", C.c_int32),
        ("block_size", C.c_int32),
        ("block_table", C.c_void_p),
        ("max_blocks", C.c_int32),
    ]


class Q4Matrix(C.Structure):
    _fields_ = [
        ("qweight", C.c_void_p),
        ("scales", C.c_void_p),
        ("zero_points", C.c_void_p),
        ("n", C.c_int32),
        ("k", C.c_int32),
    ]


P2P_KV_F16 = 0
P2P_KV_I8 = 1


class DecodeLayer(C.Structure):
    _fields_ = [
        ("qkv", C.c_void_p),
        ("norm_w", C.c_void_p),
        ("k_cache", C.c_void_p),
        ("v_cache", C.c_void_p),
        ("out", C.c_void_p),
    ]


_v = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_u32 = C.c_uint32
_st = C.c_int
_pp = C.POINTER(AttnParams)

# name -> (restype, argtypes); every symbol include/p2p_attn.h declares.
PROTOTYPES = {
    "p2p_abi_version": (C.c_int, []),
    "p2p_status_string": (C.c_char_p, [_st]),
    "p2p_ctx_create": (_st, [C.c_int, C.POINTER(_v)]),
    "p2p_ctx_destroy": (_st, [_v]),
    "p2p_last_error": (C.c_char_p, [_v]),
    "p2p_ctx_stream": (_v, [_v]),
    "p2p_sync": (_st, [_v, _v]),
    "p2p_rope_table": (_st, [_v, _i32, _i32, C.c_double, _i32, C.POINTER(_v)]),
    "p2p_meta": (_st, [_v, C.POINTER(_v)]),
    "p2p_meta_write": (_st, [_v, _u32, _u32, _u32, _v]),
    "p2p_argmax_step": (_st, [_v, _v, _i32, _v, _v, _i64, _v, _v]),
    "p2p_kv_create": (_st, [_v, _i32, _i32, _i32, _i64, _i32, C.POINTER(_v)]),
    "p2p_kv_destroy": (_st, [_v]),
    "p2p_kv_ensure_capacity": (_st, [_v, _i64, _i64, _i64, _v]),
    "p2p_kv_capacity": (_i64, [_v]),
    "p2p_kv_k": (_v, [_v, _i32]),
    "p2p_kv_v": (_v, [_v, _i32]),
    "p2p_qk_prep": (_st, [_v, _pp, _v, _i64, _v, _v, _v, _i64, _v, _v, _i64, _v, _i32, _i32, _v]),
    "p2p_attn": (_st, [_v, _pp, _v, _i64, _v, _v, _i64, _v, _i64, _v, _i32, _i32, _v]),
    "p2p_decode_step": (_st, [_v, _pp, _i32, C.POINTER(DecodeLayer), _v, _i64, _v, _i32, _v]),
    "p2p_attn_decode_ragged": (
        _st, [_v, _pp, _v, _i64, _v, _v, _v, _v, _i64, _v, _v, _i32, _i32, _i32, _v, _i64, _v]),
    "p2p_attn_bidir": (_st, [_v, _pp, _v, _v, _v, _v, _i64, _i32, _i32, _v]),
    "p2p_attn_decode_ragged_noalloc": (
        _st, [_v, _pp, _v, _i64, _v, _v, _v, _v, _i64, _v, _v, _i32, _i32, _i32, _v, _i64, _v]),
    "p2p_attn_scatter": (
        _st, [_v, _pp, _v, _i64, _v, _v, _i64, C.POINTER(_v), _i32, _i64, _i32, _v, _i32, _i32, _v]),
    "p2p_attn_multicast": (
        _st, [_v, _pp, _v, _i64, _v, _v, _i64, _v, _i64, _i32, _v, _i32, _i32, _v]),
    "p2p_shared_alloc": (_st, [_v, C.c_size_t, C.POINTER(_v), C.c_char_p]),
    "p2p_shared_free": (_st, [_v, _v]),
    "p2p_shared_open": (_st, [_v, C.c_char_p, C.POINTER(_v)]),
    "p2p_shared_close": (_st, [_v, _v]),
    "p2p_attn_decode_kv": (
        _st, [_v, _pp, C.POINTER(KvLayout), _v, _i64, _v, _v, _v, _v, _i64, _v, _v, _i32, _i32,
              _i32, _v, _i64, _v]),
    "p2p_kv_quantize_q8": (_st, [_v, _v, _v, _i64, _i32, _v, _i32, _v]),
    "p2p_gemv_q4": (_st, [_v, C.POINTER(Q4Matrix), _v, _v, _i64, _v]),
    "p2p_qkv_gemv_prep": (
        _st, [_v, _pp, _v, C.POINTER(Q4Matrix), C.POINTER(Q4Matrix), C.POINTER(Q4Matrix), _v,
              _v, _v, _v, _v, _i64, _v, _i32, _v]),
    "p2p_gemm_q4": (_st, [_v, C.POINTER(Q4Matrix), _v, _i64, _i32, _v, _i64, _i64, _v]),
    "p2p_q4_to_f16": (_st, [_v, C.POINTER(Q4Matrix), _v, _v]),
    "p2p_gemm_f16w": (_st, [_v, _v, _i32, _i32, _v, _i64, _i32, _v, _i64, _i64, _v]),
    "p2p_qkv_gemm_prep_f16w": (
        _st, [_v, _pp, _v, _i64, _v, _i32, _v, _v, _v, _i64, _v, _v, _i64, _v, _i32, _i32, _v]),
    "p2p_qkv_gemm_prep": (
        _st, [_v, _pp, _v, _i64, C.POINTER(Q4Matrix), C.POINTER(Q4Matrix), C.POINTER(Q4Matrix),
              _v, _v, _v, _i64, _v, _v, _i64, _v, _i32, _i32, _v]),
    "p2p_comm_unique_id": (_st, [C.c_char_p]),
    "p2p_comm_create": (_st, [_v, _i32, _i32, C.c_char_p, _i32, C.POINTER(_v)]),
    "p2p_comm_destroy": (_st, [_v]),
    "p2p_comm_wait": (_st, [_v, _v]),
    "p2p_comm_barrier": (_st, [_v, _v]),
    "p2p_attn_prefill_sharded": (
        _st, [_v, _v, _pp, _v, _i64, _v, _v, _v, _v, _i64, _v, _i32, _i32, _v, _i64, _v]),
    "p2p_debug_set_alloc_limit": (_st, [_i64]),
    "p2p_debug_set_wait_deficit": (_st, [_i32]),
    "p2p_debug_stream_read": (_st, [_v, _v, _i64, _v, _v]),
}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python p2p_b200/build.py` "
            "(there is no CPU fallback for the attention kernels)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int, ctx=None) -> None:
    if status == P2P_OK:
        return
    msg = lib.p2p_last_error(ctx).decode() if ctx else lib.p2p_status_string(status).decode()
    cls = {P2P_ERR_KV_FULL: KvFullError, P2P_ERR_OOM: OomError}.get(status, P2PError)
    raise cls(status, msg)
