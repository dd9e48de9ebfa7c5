"""ctypes bindings for the CPU checker (TEST INFRASTRUCTURE ONLY).

Loads oracle/libp2poracle.so (the C++ restatement of the reference path) and, when it has
been built, oracle/_ref/libp2pref.so (the reference's own WGSL shaders translated to C++ by
oracle/wgsl2cpp.py).  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import
this module; the product library never does.

Arrays are numpy: float16 for f16 storage (passed as their binary16 bit patterns), float32
for the fp32 case, int64/int32 for offsets and lengths.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
_LIB = None
_REF = None

_p = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_f = C.c_float
_d = C.c_double


def _ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def lib():
    """The restatement library; builds it with make if it is missing."""
    global _LIB
    if _LIB is None:
        path = _DIR / "libp2poracle.so"
        if not path.exists():
            import subprocess

            subprocess.run(["make", "-C", str(_DIR), "libp2poracle.so"], check=True)
        L = C.CDLL(str(path))
        L.p2p_or_f32_to_f16.restype = C.c_uint16
        L.p2p_or_f32_to_f16.argtypes = [_f]
        L.p2p_or_f16_to_f32.restype = _f
        L.p2p_or_f16_to_f32.argtypes = [C.c_uint16]
        L.p2p_or_f32_to_f16_array.argtypes = [_p, _p, _i64]
        L.p2p_or_f16_to_f32_array.argtypes = [_p, _p, _i64]
        L.p2p_or_rope_table.argtypes = [_i, _i, _d, _p]
        L.p2p_or_rope_table_f32.argtypes = [_i, _i, _d, _p]
        L.p2p_or_qk_prep_h.argtypes = [_i, _i, _i, _f, _p, _i64, _p, _p, _p, _i64, _p, _p, _i, _i]
        L.p2p_or_qk_prep_f.argtypes = [_i, _i, _i, _f, _p, _i64, _p, _p, _p, _i64, _p, _p, _i, _i]
        L.p2p_or_attn_h.argtypes = [_i, _i, _i, _f, _p, _i64, _p, _p, _p, _i64, _i, _i]
        L.p2p_or_attn_f.argtypes = [_i, _i, _i, _f, _p, _i64, _p, _p, _p, _i64, _i, _i]
        L.p2p_or_attn_ragged_h.argtypes = [_i, _i, _i, _f, _p, _i64, _p, _p, _p, _p, _i, _p, _i64]
        L.p2p_or_vision_attn_h.argtypes = [_i, _i, _f, _i, _i, _p, _p, _p, _p, _i64]
        L.p2p_or_quantize_q8.argtypes = [_p, _p, _i64, _i, _i, _p, _i]
        L.p2p_or_gemv_q4.argtypes = [_i, _i, _p, _p, _p, _p, _p, _i64]
        L.p2p_or_gemm_q4.argtypes = [_i, _i, _i, _p, _p, _p, _p, _p, _i64, _i64]
        L.p2p_or_attn_ragged_q8.argtypes = [_i, _i, _i, _f, _p, _i64, _p, _p, _p, _p, _i, _p, _p,
                                            _i, _p, _i64]
        L.p2p_or_attn_exact.argtypes = [_i, _i, _i, _d, _p, _i64, _p, _p, _p, _i64, _i, _i]
        L.p2p_or_argmax_h.argtypes = [_p, C.c_uint32, _p, _p, _p]
        L.p2p_or_set_threads.restype = _i
        L.p2p_or_set_threads.argtypes = [_i]
        _LIB = L
    return _LIB


def ref_available() -> bool:
    return (_DIR / "_ref" / "libp2pref.so").exists()


def ref():
    """The translated reference shaders (oracle/_ref); raises if they were never built."""
    global _REF
    if _REF is None:
        path = _DIR / "_ref" / "libp2pref.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (needs the reference sources)")
        L = C.CDLL(str(path))
        for name in ("QK_PREP", "ATTN", "VISION_ATTN", "ARGMAX", "GEMV"):
            fn = getattr(L, f"ref_{name}")
            fn.restype = _i
            fn.argtypes = [_p, _p, C.c_uint32, C.c_uint32, C.c_uint32]
        _REF = L
    return _REF


def set_threads(n: int = 0) -> int:
    return lib().p2p_or_set_threads(int(n))


# ---- f16 helpers (engine.js:28-50, 331-345) ----------------------------------------------

def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.float16)
    lib().p2p_or_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
    return out


def f16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float16)
    out = np.empty(x.shape, np.float32)
    lib().p2p_or_f16_to_f32_array(_ptr(x), _ptr(out), x.size)
    return out


def rope_table(max_ctx: int, d: int = 64, theta: float = 1e6, f32: bool = False) -> np.ndarray:
    if f32:
        out = np.empty((max_ctx, d), np.float32)
        lib().p2p_or_rope_table_f32(max_ctx, d, theta, _ptr(out))
    else:
        out = np.empty((max_ctx, d), np.float16)
        lib().p2p_or_rope_table(max_ctx, d, theta, _ptr(out))
    return out


# ---- the three shaders, restated ----------------------------------------------------------

def qk_prep(hq, hkv, d, qkv, nw, rope, q_out, kc, vc, pos0, m_tokens, eps=1e-5):
    """kernels.js:216-266 in place on q_out / kc / vc (f16 or f32 storage)."""
    fn = lib().p2p_or_qk_prep_f if qkv.dtype == np.float32 else lib().p2p_or_qk_prep_h
    fn(hq, hkv, d, eps, _ptr(qkv), qkv.shape[-1], _ptr(nw), _ptr(rope), _ptr(q_out),
       q_out.shape[-1], _ptr(kc), _ptr(vc), pos0, m_tokens)


def attn(hq, hkv, d, q, kc, vc, out, pos0, m_tokens, scale=0.125):
    """kernels.js:268-319 (f16 or f32 storage)."""
    fn = lib().p2p_or_attn_f if q.dtype == np.float32 else lib().p2p_or_attn_h
    fn(hq, hkv, d, scale, _ptr(q), q.shape[-1], _ptr(kc), _ptr(vc), _ptr(out), out.shape[-1],
       pos0, m_tokens)


def attn_ragged(hq, hkv, d, q, kc, vc, offsets, past, out, scale=0.125):
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    past = np.ascontiguousarray(past, dtype=np.int32)
    lib().p2p_or_attn_ragged_h(hq, hkv, d, scale, _ptr(q), q.shape[-1], _ptr(kc), _ptr(vc),
                               _ptr(offsets), _ptr(past), len(past), _ptr(out), out.shape[-1])


def gemv_q4(x, wq, sc, zp, y=None, y_off=0):
    """kernels.js:22-68: y[y_off + n] = f16(x . W[n]) for the 4-bit matrix (wq u32 [N][K/8],
    sc f16 [N][K/32], zp u8 bytes packed in u32 words).  Returns y (float16)."""
    x = np.ascontiguousarray(x, dtype=np.float16).reshape(-1)
    n, wpr = wq.shape
    if y is None:
        y = np.zeros(y_off + n, np.float16)
    lib().p2p_or_gemv_q4(x.size, n, _ptr(x), _ptr(np.ascontiguousarray(wq, np.uint32)),
                         _ptr(np.ascontiguousarray(sc, np.float16)),
                         _ptr(np.ascontiguousarray(zp, np.uint32)), _ptr(y), y_off)
    return y


def ref_gemv(x, wq, sc, zp, y, y_off=0):
    """The reference's own GEMV shader (oracle/_ref), dispatched as engine.js does: N/8
    workgroups of 256."""
    n = wq.shape[0]
    ovr = (C.c_double * 3)(x.size, n, y_off)
    rc = ref().ref_GEMV(_bind(x, wq, sc, zp, y), ovr, (n + 7) // 8, 1, 1)
    if rc:
        raise RuntimeError(f"ref_GEMV failed ({rc})")


def gemm_q4(x, wq, sc, zp, y=None, y_stride=None, y_off=0):
    """kernels.js:70-145: Y[m][y_off + n] = f16(X[m] . W[n]) for an [M][K] f16 block X (rows of
    y_stride elements in y).  Returns y (float16, [M][y_stride])."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    m, k = x.shape
    n, wpr = wq.shape
    assert wpr * 8 == k
    if y_stride is None:
        y_stride = y_off + n
    if y is None:
        y = np.zeros((m, y_stride), np.float16)
    lib().p2p_or_gemm_q4(m, k, n, _ptr(x), _ptr(np.ascontiguousarray(wq, np.uint32)),
                         _ptr(np.ascontiguousarray(sc, np.float16)),
                         _ptr(np.ascontiguousarray(zp, np.uint32)), _ptr(y), y_stride, y_off)
    return y


def dequant_q4(wq, sc, zp):
    """W[n][k] = (q - zp) * scale in f32, the block rule of kernels.js:22-68 / :70-145 (value
    8w+i of a row is nibble i of word w; zero point of block b is nibble b&1 of byte b>>1 of the
    row's ceil(K/64) bytes).  For error bounds; the GEMV / GEMM restatements do not use it."""
    wq = np.ascontiguousarray(wq, np.uint32)
    n, wpr = wq.shape
    k = wpr * 8
    q = (wq[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15
    q = q.reshape(n, k).astype(np.float32)
    nb, zr = k // 32, (k // 32 + 1) // 2
    zb = np.ascontiguousarray(zp).view(np.uint8)[: n * zr].reshape(n, zr)
    blk = np.arange(nb)
    z = ((zb[:, blk // 2] >> ((blk & 1) * 4)) & 15).astype(np.float32)
    s = np.asarray(sc).astype(np.float32)
    return (q - np.repeat(z, 32, axis=1)) * np.repeat(s, 32, axis=1)


def ref_gemm(x, wq, sc, zp, y, y_stride, y_off=0):
    """The reference's own GEMM shader (oracle/_ref), dispatched as engine.js does: (N/64,
    M/64) workgroups of 256, M from the meta buffer's second word."""
    m, k = x.shape
    n = wq.shape[0]
    mt = np.array([0, m, 0, 0], np.uint32)
    ovr = (C.c_double * 4)(k, n, y_stride, y_off)
    rc = ref().ref_GEMM(_bind(x, wq, sc, zp, y, mt), ovr, (n + 63) // 64, (m + 63) // 64, 1)
    if rc:
        raise RuntimeError(f"ref_GEMM failed ({rc})")


def random_q4(rng, n, k):
    """A random 4-bit matrix in the reference layout: (wq, scales, zero-point words)."""
    wq = rng.integers(0, 2**32, (n, k // 8), dtype=np.uint64).astype(np.uint32)
    sc = (0.01 + 0.02 * rng.random((n, k // 32))).astype(np.float16)
    zr = (k // 32 + 1) // 2
    zbytes = rng.integers(0, 256, n * zr + (-(n * zr)) % 4, dtype=np.uint64).astype(np.uint8)
    return wq, sc, zbytes.view(np.uint32)


def quantize_q8(src, scale):
    """f16 cache rows [..., Hkv, D] -> int8 (the reference bundle's int8 cache rule)."""
    src = np.ascontiguousarray(src, dtype=np.float16)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    hkv, d = src.shape[-2], src.shape[-1]
    rows = src.size // (hkv * d)
    out = np.empty(src.shape, np.int8)
    lib().p2p_or_quantize_q8(_ptr(src), _ptr(out), rows, hkv, d, _ptr(scale),
                             int(scale.size > 1))
    return out


def attn_ragged_q8(hq, hkv, d, q, kc, vc, k_scale, v_scale, offsets, past, out, scale=0.125):
    """ATTN per sequence over int8 cache slices (dequantised f32(q) * scale)."""
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    past = np.ascontiguousarray(past, dtype=np.int32)
    ks = np.ascontiguousarray(k_scale, dtype=np.float32)
    vs = np.ascontiguousarray(v_scale, dtype=np.float32)
    lib().p2p_or_attn_ragged_q8(hq, hkv, d, scale, _ptr(q), q.shape[-1], _ptr(kc), _ptr(vc),
                                _ptr(ks), _ptr(vs), int(ks.size > 1), _ptr(offsets), _ptr(past),
                                len(past), _ptr(out), out.shape[-1])


def gather_pages(pages, block_table, n_tokens):
    """The rows of one paged sequence in token order: pages [P][B][Hkv][D], block_table [nb]."""
    bs = pages.shape[1]
    nb = (n_tokens + bs - 1) // bs
    rows = pages[np.asarray(block_table[:nb], np.int64)].reshape(nb * bs, *pages.shape[2:])
    return np.ascontiguousarray(rows[:n_tokens])


def vision_attn(nh, d, q, k, v, out, scale=0.125):
    """vision-kernels.js:176-258; q/k/v/out are [B][S][NH*D] float16."""
    b, s, ld = q.shape
    lib().p2p_or_vision_attn_h(nh, d, scale, b, s, _ptr(q), _ptr(k), _ptr(v), _ptr(out), ld)


def argmax(logits, tok, meta, out_tok):
    """kernels.js:362-399 in place on tok / meta / out_tok (uint32 arrays); logits float16."""
    logits = np.ascontiguousarray(logits, dtype=np.float16)
    lib().p2p_or_argmax_h(_ptr(logits), logits.size, _ptr(tok), _ptr(meta), _ptr(out_tok))


def attn_exact(hq, hkv, d, q, kc, vc, pos0, m_tokens, scale=0.125):
    out = np.empty((m_tokens, hq * d), np.float64)
    lib().p2p_or_attn_exact(hq, hkv, d, scale, _ptr(q), q.shape[-1], _ptr(kc), _ptr(vc),
                            _ptr(out), out.shape[-1], pos0, m_tokens)
    return out


# ---- the reference's own shaders (translated), fixed reference shapes ---------------------

def _bind(*arrays):
    ptrs = (C.c_void_p * len(arrays))(*[_ptr(a) for a in arrays])
    return ptrs


def ref_qk_prep(qkv, nwb, qout, kc, vc, meta, rope, m_tokens):
    """QK_PREP dispatched as engine.js:221 does: grid (32, M).  Reference shapes only:
    qkv [M][2048], qout [M][1024], caches [cap][8][64]."""
    b = _bind(qkv, nwb, qout, kc, vc, meta, rope)
    rc = ref().ref_QK_PREP(b, None, 32, m_tokens, 1)
    if rc != 0:
        raise RuntimeError("QK_PREP: non-uniform barrier")


def ref_attn(q, kc, vc, out, meta, m_tokens):
    """ATTN dispatched as engine.js:222 does: grid (16, M)."""
    b = _bind(q, kc, vc, out, meta)
    rc = ref().ref_ATTN(b, None, 16, m_tokens, 1)
    if rc != 0:
        raise RuntimeError("ATTN: non-uniform barrier")


def ref_vision_attn(q, k, v, out, s_tokens=1024, num_heads=12, scale=0.125):
    """VISION_ATTN dispatched as vision.js:271-276 does: grid (NUM_HEADS, S), one image."""
    b = _bind(q, k, v, out)
    ov = (C.c_double * 4)(float(s_tokens), float(num_heads), 64.0, float(scale))
    rc = ref().ref_VISION_ATTN(b, ov, num_heads, s_tokens, 1)
    if rc != 0:
        raise RuntimeError("VISION_ATTN: non-uniform barrier")


def ref_argmax(logits, tok, meta, out_tok):
    """ARGMAX dispatched as engine.js:265-266 does: one workgroup, V = len(logits)."""
    b = _bind(logits, tok, meta, out_tok)
    ov = (C.c_double * 1)(float(logits.size))
    rc = ref().ref_ARGMAX(b, ov, 1, 1, 1)
    if rc != 0:
        raise RuntimeError("ARGMAX: non-uniform barrier")


def threads_env() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
