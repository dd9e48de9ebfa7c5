"""Host-side mirror of the reference engine's attention plumbing, over the C ABI.

The reference engine (src/scripts/lfm-engine/engine.js, vision.js) builds, for each attention
layer, a QK_PREP op and an ATTN op bound to [qkv, norm weights, qrot, K cache, V cache, meta,
rope] and dispatches them per prefill chunk and per decode step; the vision encoder dispatches
VISION_ATTN on separate q/k/v buffers.  This module keeps those operators, their buffer
layouts, their argument meaning and their error behaviour (KV growth failure -> 'kv_full'),
with device memory held in torch tensors and every kernel in libp2pattn.so:

    Context.qk_prep        QK_PREP   kernels.js:216-266, dispatched engine.js:213-221
    Context.attn           ATTN      kernels.js:268-319, dispatched engine.js:214-222
    Context.decode_step    QK_PREP + ATTN at M=1 for all attention layers (engine.js:425-429)
    Context.attn_decode_ragged  ATTN at M=1 over many sequences sharing one cache
    Context.attn_bidir     VISION_ATTN vision-kernels.js:176-258, dispatched vision.js:271-276
    KVCache                K/V buffers engine.js:152-165 and ensureCapacity engine.js:274-304
    LfmAttention           the per-layer op pair + meta + rope + KV cache of createLfmEngine
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import AttnParams, DecodeLayer, check, lib

HEAD_DIM = 64


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream) -> C.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


@dataclass
class Params:
    """Uniform parameters of one attention layer (kernels.js:268: 16 q heads, 8 kv heads,
    head_dim 64, scale 0.125; vision-kernels.js:182-185: S, NUM_HEADS, HEAD_DIM, SCALE)."""

    num_heads: int
    num_kv_heads: int
    head_dim: int = HEAD_DIM
    scale: float = 0.0  # 0 -> 1/sqrt(head_dim)
    eps: float = 1e-5
    dtype: torch.dtype = torch.float16

    def c(self) -> AttnParams:
        dt = {torch.float16: _lib.P2P_F16, torch.float32: _lib.P2P_F32}[self.dtype]
        return AttnParams(self.num_heads, self.num_kv_heads, self.head_dim, self.scale,
                          self.eps, dt)

    @property
    def qkv_width(self) -> int:
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim


class Context:
    """One p2p_ctx: a CUDA device, its split-KV workspace and its meta buffer."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib.p2p_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device
        m = C.c_void_p()
        check(lib.p2p_meta(self.h, C.byref(m)), self.h)
        self.meta_ptr = m
        self._rope = {}

    def close(self):
        if self.h:
            lib.p2p_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _chk(self, status):
        check(status, self.h)

    # -- engine.js:60-71, :144-146 ----------------------------------------------------------
    def rope_table(self, max_ctx: int, head_dim: int = HEAD_DIM, theta: float = 1e6,
                   dtype: torch.dtype = torch.float16) -> C.c_void_p:
        dt = _lib.P2P_F16 if dtype == torch.float16 else _lib.P2P_F32
        p = C.c_void_p()
        self._chk(lib.p2p_rope_table(self.h, max_ctx, head_dim, theta, dt, C.byref(p)))
        return p

    def meta_write(self, pos0: int, m_tokens: int, step: int = 0, stream=None):
        self._chk(lib.p2p_meta_write(self.h, pos0, m_tokens, step, _stream(stream)))

    def argmax_step(self, logits: torch.Tensor, tok: torch.Tensor, out_tok: torch.Tensor,
                    meta: Optional[torch.Tensor] = None, stream=None):
        """kernels.js:362-399 (ARGMAX): greedy token of `logits` (f16, vocab elements) into
        tok[0] and out_tok[step]; then step and position advance in the meta buffer (the
        context's own unless `meta`, a uint32[4] device tensor, is given), on the device."""
        self._chk(lib.p2p_argmax_step(self.h, _ptr(logits), logits.numel(), _ptr(tok),
                                      _ptr(out_tok), out_tok.numel(),
                                      _ptr(meta) if meta is not None else None, _stream(stream)))

    def sync(self, stream=None):
        self._chk(lib.p2p_sync(self.h, _stream(stream)))

    def debug_stream_read(self, src: torch.Tensor, xor_out: torch.Tensor, nbytes=None,
                          stream=None):
        """Measurement reference: one launch streaming `nbytes` (default all) of `src` and
        XOR-folding its 32-bit words into xor_out[0] (an int32 device tensor, zeroed by the
        caller)."""
        n = src.numel() * src.element_size() if nbytes is None else nbytes
        self._chk(lib.p2p_debug_stream_read(self.h, _ptr(src), n, _ptr(xor_out),
                                            _stream(stream)))

    # -- the shader entry points ----------------------------------------------------------------
    def qk_prep(self, prm: Params, qkv: torch.Tensor, norm_w: Optional[torch.Tensor], rope,
                q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                pos0: int = 0, m_tokens: Optional[int] = None, use_meta: bool = False,
                stream=None):
        m = qkv.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_qk_prep(
            self.h, C.byref(prm.c()), _ptr(qkv), qkv.stride(0), _ptr(norm_w),
            rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(q_out), q_out.stride(0),
            _ptr(k_cache), _ptr(v_cache), k_cache.shape[0], self.meta_ptr if use_meta else None,
            pos0, m, _stream(stream)))

    def attn_scatter(self, prm: Params, q: torch.Tensor, k_cache: torch.Tensor,
                     v_cache: torch.Tensor, outs: Sequence[int], ld_o: int, out_head0: int, *,
                     pos0: int = 0, m_tokens: Optional[int] = None, use_meta: bool = False,
                     stream=None):
        """p2p_attn_scatter: causal prefill over this rank's heads, every output row written
        into each buffer of `outs` (device addresses: this rank's own first, then the other
        ranks' opened with shared_open) at column (out_head0 + h) * 64."""
        m = q.shape[0] if m_tokens is None else m_tokens
        arr = (C.c_void_p * len(outs))(*[int(o) for o in outs])
        self._chk(lib.p2p_attn_scatter(
            self.h, C.byref(prm.c()), _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache),
            k_cache.shape[0], arr, len(outs), ld_o, out_head0,
            self.meta_ptr if use_meta else None, pos0, m, _stream(stream)))

    def attn_multicast(self, prm: Params, q: torch.Tensor, k_cache: torch.Tensor,
                       v_cache: torch.Tensor, mc_out: int, ld_o: int, out_head0: int, *,
                       pos0: int = 0, m_tokens: Optional[int] = None, use_meta: bool = False,
                       stream=None):
        """p2p_attn_multicast: as attn_scatter, with the rows written once to the NVLink
        multicast address mc_out (NVSwitch replicates them into every rank's buffer)."""
        m = q.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_attn_multicast(
            self.h, C.byref(prm.c()), _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache),
            k_cache.shape[0], C.c_void_p(mc_out), ld_o, out_head0,
            self.meta_ptr if use_meta else None, pos0, m, _stream(stream)))

    def shared_alloc(self, nbytes: int):
        """p2p_shared_alloc: (device address, IPC handle bytes) of a new node-shared buffer."""
        ptr = C.c_void_p()
        handle = C.create_string_buffer(_lib.P2P_IPC_HANDLE_BYTES)
        self._chk(lib.p2p_shared_alloc(self.h, nbytes, C.byref(ptr), handle))
        return ptr.value, handle.raw

    def shared_open(self, handle: bytes) -> int:
        """p2p_shared_open: this process's address of another process's shared buffer."""
        ptr = C.c_void_p()
        self._chk(lib.p2p_shared_open(self.h, handle, C.byref(ptr)))
        return ptr.value

    def shared_close(self, ptr: int):
        self._chk(lib.p2p_shared_close(self.h, C.c_void_p(ptr)))

    def shared_free(self, ptr: int):
        self._chk(lib.p2p_shared_free(self.h, C.c_void_p(ptr)))

    def attn(self, prm: Params, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             out: torch.Tensor, *, pos0: int = 0, m_tokens: Optional[int] = None,
             use_meta: bool = False, stream=None):
        m = q.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_attn(
            self.h, C.byref(prm.c()), _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache),
            k_cache.shape[0], _ptr(out), out.stride(0), self.meta_ptr if use_meta else None,
            pos0, m, _stream(stream)))

    def decode_step(self, prm: Params, layers: Sequence[tuple], rope, kv_cap: int, *,
                    pos: int = 0, use_meta: bool = False, stream=None):
        """layers: (qkv_row, norm_w or None, k_cache, v_cache, out_row) per attention layer."""
        arr = (DecodeLayer * len(layers))()
        for i, (qkv, nw, kc, vc, out) in enumerate(layers):
            arr[i] = DecodeLayer(qkv.data_ptr(), nw.data_ptr() if nw is not None else None,
                                 kc.data_ptr(), vc.data_ptr(), out.data_ptr())
        self._chk(lib.p2p_decode_step(
            self.h, C.byref(prm.c()), len(layers), arr,
            rope if isinstance(rope, C.c_void_p) else _ptr(rope), kv_cap,
            self.meta_ptr if use_meta else None, pos, _stream(stream)))

    def plan_decode_step(self, prm: Params, layers: Sequence[tuple], rope, kv_cap: int, *,
                         pos: int = 0, use_meta: bool = False) -> "DecodeStepPlan":
        """Builds the C arguments of decode_step once; plan.run() is one ctypes call."""
        return DecodeStepPlan(self, prm, layers, rope, kv_cap, pos, use_meta)

    def attn_decode_ragged(self, prm: Params, qkv: torch.Tensor, norm_w, rope,
                           k_cache: torch.Tensor, v_cache: torch.Tensor, offsets: torch.Tensor,
                           past: torch.Tensor, out: torch.Tensor, *, max_past: int,
                           fused_prep: bool = True, kv_rows: Optional[int] = None, stream=None):
        """Sequence i owns cache rows offsets[i] .. offsets[i] + past[i]; kv_rows (default: the
        cache tensor's first dimension) bounds them.  A sequence outside the cache, or with
        past[i] > max_past, is skipped on the device and the next sync() raises KvFullError."""
        assert offsets.dtype == torch.int32 and past.dtype == torch.int32
        rows = k_cache.shape[0] if kv_rows is None else kv_rows
        self._chk(lib.p2p_attn_decode_ragged(
            self.h, C.byref(prm.c()), _ptr(qkv), qkv.stride(0), _ptr(norm_w),
            rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(k_cache), _ptr(v_cache),
            rows, _ptr(offsets), _ptr(past), past.shape[0], max_past, int(fused_prep),
            _ptr(out), out.stride(0), _stream(stream)))

    def attn_decode_ragged_noalloc(self, prm: Params, qkv: torch.Tensor, norm_w, rope,
                                   k_cache: torch.Tensor, v_cache: torch.Tensor,
                                   offsets: torch.Tensor, past: torch.Tensor, out: torch.Tensor,
                                   *, max_past: int, fused_prep: bool = True,
                                   kv_rows: Optional[int] = None, stream=None):
        """attn_decode_ragged without any device allocation: the split scratch is the
        library's fixed array of P2P_NOALLOC_SCRATCH_BYTES (see include/p2p_attn.h)."""
        assert offsets.dtype == torch.int32 and past.dtype == torch.int32
        rows = k_cache.shape[0] if kv_rows is None else kv_rows
        self._chk(lib.p2p_attn_decode_ragged_noalloc(
            self.h, C.byref(prm.c()), _ptr(qkv), qkv.stride(0), _ptr(norm_w),
            rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(k_cache), _ptr(v_cache),
            rows, _ptr(offsets), _ptr(past), past.shape[0], max_past, int(fused_prep),
            _ptr(out), out.stride(0), _stream(stream)))

    def attn_decode_kv(self, prm: Params, qkv: torch.Tensor, norm_w, rope,
                       k_cache: torch.Tensor, v_cache: torch.Tensor, past: torch.Tensor,
                       out: torch.Tensor, *, max_past: int, offsets: Optional[torch.Tensor] = None,
                       k_scale: Optional[torch.Tensor] = None,
                       v_scale: Optional[torch.Tensor] = None,
                       block_table: Optional[torch.Tensor] = None, fused_prep: bool = True,
                       kv_rows: Optional[int] = None, stream=None):
        """Batched decode over an int8 and/or paged KV cache (p2p_attn_decode_kv).

        int8 caches (k_cache.dtype == torch.int8) take k_scale / v_scale (f32, 1 or Hkv*64
        values).  Paged caches are [pages][block_size][Hkv][64] with block_table [nseq][max
        blocks] (int32); contiguous ones [rows][Hkv][64] with offsets (int32)."""
        assert past.dtype == torch.int32
        q8 = k_cache.dtype == torch.int8
        lay = _lib.KvLayout()
        lay.format = _lib.P2P_KV_I8 if q8 else _lib.P2P_KV_F16
        if q8:
            assert k_scale is not None and v_scale is not None
            assert k_scale.dtype == torch.float32 and v_scale.dtype == torch.float32
            lay.k_scale, lay.v_scale = k_scale.data_ptr(), v_scale.data_ptr()
            lay.scale_count = k_scale.numel()
        if block_table is not None:
            assert block_table.dtype == torch.int32 and k_cache.dim() == 4
            lay.block_size = k_cache.shape[1]
            lay.block_table = block_table.data_ptr()
            lay.max_blocks = block_table.shape[1]
        else:
            assert offsets is not None and offsets.dtype == torch.int32
        rows = k_cache.shape[0] if kv_rows is None else kv_rows
        self._chk(lib.p2p_attn_decode_kv(
            self.h, C.byref(prm.c()), C.byref(lay), _ptr(qkv), qkv.stride(0), _ptr(norm_w),
            rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(k_cache), _ptr(v_cache),
            rows, _ptr(offsets), _ptr(past), past.shape[0], max_past, int(fused_prep),
            _ptr(out), out.stride(0), _stream(stream)))

    def kv_quantize_q8(self, src: torch.Tensor, scale: torch.Tensor,
                       dst: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """f16 cache rows [..., Hkv, 64] -> int8 (the decode's int8 cache format)."""
        assert src.dtype == torch.float16 and scale.dtype == torch.float32
        hkv = src.shape[-2]
        rows = src.numel() // (hkv * HEAD_DIM)
        if dst is None:
            dst = torch.empty(src.shape, dtype=torch.int8, device=src.device)
        self._chk(lib.p2p_kv_quantize_q8(self.h, _ptr(src), _ptr(dst), rows, hkv, _ptr(scale),
                                         scale.numel(), _stream(stream)))
        return dst

    @staticmethod
    def q4(w) -> "_lib.Q4Matrix":
        """(qweight u32 [n][k/8], scales f16 [n][k/32], zero_points u32 words) -> the C view."""
        qw, sc, zp = w
        return _lib.Q4Matrix(qw.data_ptr(), sc.data_ptr(), zp.data_ptr(), qw.shape[0],
                             qw.shape[1] * 8)

    def gemv_q4(self, w, x: torch.Tensor, y: torch.Tensor, y_off: int = 0, stream=None):
        """kernels.js:22-68: y[y_off + n] = f16(x . W[n]) for one token (e.g. o_proj)."""
        m = self.q4(w)
        self._chk(lib.p2p_gemv_q4(self.h, C.byref(m), _ptr(x), _ptr(y), y_off, _stream(stream)))

    def qkv_gemv_prep(self, prm: Params, x: torch.Tensor, wq, wk, wv, norm_w, rope,
                      q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                      pos: int = 0, use_meta: bool = False, stream=None):
        """q/k/v projections of one token with QK_PREP in the epilogue (rotated q to q_out,
        k/v to cache row pos)."""
        mq, mk, mv = self.q4(wq), self.q4(wk), self.q4(wv)
        self._chk(lib.p2p_qkv_gemv_prep(
            self.h, C.byref(prm.c()), _ptr(x), C.byref(mq), C.byref(mk), C.byref(mv),
            _ptr(norm_w), rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(q_out),
            _ptr(k_cache), _ptr(v_cache), k_cache.shape[0], self.meta_ptr if use_meta else None,
            pos, _stream(stream)))

    def gemm_q4(self, w, x: torch.Tensor, y: torch.Tensor, y_off: int = 0,
                m_tokens: Optional[int] = None, stream=None):
        """kernels.js:70-145: y[m][y_off + n] = f16(x[m] . W[n]) for a prompt chunk."""
        mw = self.q4(w)
        m = x.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_gemm_q4(self.h, C.byref(mw), _ptr(x), x.stride(0), m, _ptr(y),
                                  y.stride(0), y_off, _stream(stream)))

    def qkv_gemm_prep(self, prm: Params, x: torch.Tensor, wq, wk, wv, norm_w, rope,
                      q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                      pos0: int = 0, m_tokens: Optional[int] = None, use_meta: bool = False,
                      stream=None):
        """q/k/v projections of a prompt chunk with QK_PREP in the epilogue (rotated q to
        q_out [M][Hq*64], k/v to cache rows pos0..pos0+M-1)."""
        mq, mk, mv = self.q4(wq), self.q4(wk), self.q4(wv)
        m = x.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_qkv_gemm_prep(
            self.h, C.byref(prm.c()), _ptr(x), x.stride(0), C.byref(mq), C.byref(mk),
            C.byref(mv), _ptr(norm_w), rope if isinstance(rope, C.c_void_p) else _ptr(rope),
            _ptr(q_out), q_out.stride(0), _ptr(k_cache), _ptr(v_cache), k_cache.shape[0],
            self.meta_ptr if use_meta else None, pos0, m, _stream(stream)))

    def q4_to_f16(self, w, dst: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """The resident f16 copy [n][k] of a 4-bit matrix (made once, reused by every call of
        gemm_f16w / qkv_gemm_prep_f16w)."""
        mw = self.q4(w)
        if dst is None:
            dst = torch.empty((mw.n, mw.k), dtype=torch.float16, device="cuda")
        self._chk(lib.p2p_q4_to_f16(self.h, C.byref(mw), _ptr(dst), _stream(stream)))
        return dst

    def gemm_f16w(self, w16: torch.Tensor, x: torch.Tensor, y: torch.Tensor, y_off: int = 0,
                  m_tokens: Optional[int] = None, stream=None):
        """gemm_q4 on resident f16 weights w16 [n][k]."""
        m = x.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_gemm_f16w(self.h, _ptr(w16), w16.shape[0], w16.shape[1], _ptr(x),
                                    x.stride(0), m, _ptr(y), y.stride(0), y_off,
                                    _stream(stream)))

    def qkv_gemm_prep_f16w(self, prm: Params, x: torch.Tensor, w16_qkv: torch.Tensor, norm_w,
                           rope, q_out: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor, *, pos0: int = 0,
                           m_tokens: Optional[int] = None, use_meta: bool = False, stream=None):
        """qkv_gemm_prep on resident f16 weights stacked [q rows | k rows | v rows][k]."""
        m = x.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_qkv_gemm_prep_f16w(
            self.h, C.byref(prm.c()), _ptr(x), x.stride(0), _ptr(w16_qkv), w16_qkv.shape[1],
            _ptr(norm_w), rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(q_out),
            q_out.stride(0), _ptr(k_cache), _ptr(v_cache), k_cache.shape[0],
            self.meta_ptr if use_meta else None, pos0, m, _stream(stream)))

    def attn_prefill_sharded(self, comm, prm: Params, qkv_local: torch.Tensor, norm_w, rope,
                             k_cache: torch.Tensor, v_cache: torch.Tensor, out: torch.Tensor, *,
                             pos0: int = 0, m_tokens: Optional[int] = None,
                             use_meta: bool = False, stream=None):
        """QK_PREP + ATTN of a causal chunk split by kv-head group over comm's ranks; prm
        counts the model's heads, qkv_local / the caches hold this rank's heads only, and every
        rank's out [M][Hq*64] receives all heads (one all-gather inside the library)."""
        m = qkv_local.shape[0] if m_tokens is None else m_tokens
        self._chk(lib.p2p_attn_prefill_sharded(
            self.h, comm.h, C.byref(prm.c()), _ptr(qkv_local), qkv_local.stride(0),
            _ptr(norm_w), rope if isinstance(rope, C.c_void_p) else _ptr(rope), _ptr(k_cache),
            _ptr(v_cache), k_cache.shape[0], self.meta_ptr if use_meta else None, pos0, m,
            _ptr(out), out.stride(0), _stream(stream)))

    def attn_bidir(self, prm: Params, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   out: torch.Tensor, stream=None):
        """q/k/v/out: [B][S][ld] (vision-kernels.js:198 layout)."""
        b, s, ld = q.shape
        self._chk(lib.p2p_attn_bidir(self.h, C.byref(prm.c()), _ptr(q), _ptr(k), _ptr(v),
                                     _ptr(out), ld, b, s, _stream(stream)))


class DecodeStepPlan:
    """Pre-marshalled arguments of p2p_decode_step (the per-token call of a decode loop)."""

    def __init__(self, ctx: Context, prm: Params, layers, rope, kv_cap, pos, use_meta):
        self.ctx = ctx
        self.keep = list(layers)  # keeps the tensors alive
        self.arr = (DecodeLayer * len(layers))()
        for i, (qkv, nw, kc, vc, out) in enumerate(layers):
            self.arr[i] = DecodeLayer(qkv.data_ptr(), nw.data_ptr() if nw is not None else None,
                                      kc.data_ptr(), vc.data_ptr(), out.data_ptr())
        self.prm = prm.c()
        self.rope = rope if isinstance(rope, C.c_void_p) else _ptr(rope)
        self.args = (ctx.h, C.byref(self.prm), len(layers), self.arr, self.rope, kv_cap,
                     ctx.meta_ptr if use_meta else None, pos)
        self.fn = lib.p2p_decode_step

    def run(self, stream=None):
        st = self.fn(*self.args, _stream(stream))
        if st:
            self.ctx._chk(st)


class KVCache:
    """engine.js:152-165: one K and one V buffer [cap][Hkv][D] per attention layer, grown by
    ensure_capacity as engine.js:274-304 does (allocate, copy, rebind, free)."""

    def __init__(self, ctx: Context, n_layers: int, num_kv_heads: int, cap_tokens: int,
                 dtype: torch.dtype = torch.float16):
        self.ctx = ctx
        self.n_layers = n_layers
        self.num_kv_heads = num_kv_heads
        self.dtype = dtype
        h = C.c_void_p()
        dt = _lib.P2P_F16 if dtype == torch.float16 else _lib.P2P_F32
        ctx._chk(lib.p2p_kv_create(ctx.h, n_layers, num_kv_heads, HEAD_DIM, cap_tokens, dt,
                                   C.byref(h)))
        self.h = h

    @property
    def capacity(self) -> int:
        return lib.p2p_kv_capacity(self.h)

    def ensure_capacity(self, need: int, grow: int, max_tokens: int, stream=None) -> bool:
        """True when the cache holds `need` tokens; False for 'kv_full' or OOM
        (engine.js:274-286 returns false in both cases)."""
        st = lib.p2p_kv_ensure_capacity(self.h, need, grow, max_tokens, _stream(stream))
        if st in (_lib.P2P_ERR_KV_FULL, _lib.P2P_ERR_OOM):
            return False
        self.ctx._chk(st)
        return True

    def _view(self, ptr: int) -> torch.Tensor:
        n = self.capacity * self.num_kv_heads * HEAD_DIM
        es = 2 if self.dtype == torch.float16 else 4
        # Wrap the library-owned buffer without copying (the KVCache keeps it alive).
        t = _from_device_ptr(ptr, n * es, self.ctx.device)
        return t.view(self.dtype).view(self.capacity, self.num_kv_heads, HEAD_DIM)

    def k(self, layer: int) -> torch.Tensor:
        return self._view(lib.p2p_kv_k(self.h, layer))

    def v(self, layer: int) -> torch.Tensor:
        return self._view(lib.p2p_kv_v(self.h, layer))

    def close(self):
        if self.h:
            lib.p2p_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _CudaArrayView:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
            "strides": None,
        }


def _from_device_ptr(ptr: int, nbytes: int, device: int) -> torch.Tensor:
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaArrayView(ptr, nbytes), device=f"cuda:{device}")


class LfmAttention:
    """The attention half of createLfmEngine (engine.js:73-304) for a decoder with
    `n_layers` attention layers: RoPE table, meta buffer, KV cache with growth, and the
    QK_PREP/ATTN pair per layer, dispatched per prefill chunk or per decode step."""

    KV_INIT_BYTES = 20 * 1024 * 1024  # engine.js:14
    KV_GROW_BYTES = 2 * 1024 * 1024   # engine.js:15

    def __init__(self, ctx: Context, prm: Params, n_layers: int, max_ctx: int = 4096,
                 rope_theta: float = 1e6, kv_init_bytes: int = KV_INIT_BYTES,
                 kv_grow_bytes: int = KV_GROW_BYTES):
        self.ctx, self.prm, self.n_layers, self.max_ctx = ctx, prm, n_layers, max_ctx
        self.kv_bytes_per_token = n_layers * 2 * prm.num_kv_heads * prm.head_dim * 2  # :24
        self.rope = ctx.rope_table(max_ctx, prm.head_dim, rope_theta)
        self.kv = KVCache(ctx, n_layers, prm.num_kv_heads,
                          max(1, kv_init_bytes // self.kv_bytes_per_token))  # :153
        self.grow_step = max(1, kv_grow_bytes // self.kv_bytes_per_token)   # :272

    def ensure_capacity(self, need: int) -> bool:
        if need > self.max_ctx:  # engine.js:276
            return False
        return self.kv.ensure_capacity(need, self.grow_step, self.max_ctx)

    def prefill_layer(self, layer: int, qkv: torch.Tensor, norm_w, q_rot: torch.Tensor,
                      out: torch.Tensor, pos0: int, stream=None):
        """QK_PREP then ATTN for one prefill chunk of M = qkv.shape[0] tokens at pos0
        (engine.js:384-401 writes meta = [s, mc, 0, 0] then dispatches the pair)."""
        m = qkv.shape[0]
        kc, vc = self.kv.k(layer), self.kv.v(layer)
        self.ctx.qk_prep(self.prm, qkv, norm_w, self.rope, q_rot, kc, vc, pos0=pos0,
                         m_tokens=m, stream=stream)
        self.ctx.attn(self.prm, q_rot, kc, vc, out, pos0=pos0, m_tokens=m, stream=stream)

    def decode_step(self, qkv_rows: Sequence[torch.Tensor], norm_ws, outs, pos: int,
                    use_meta: bool = False, stream=None):
        """All attention layers of one decode step at position `pos` in one launch."""
        layers = [(qkv_rows[l], norm_ws[l] if norm_ws else None, self.kv.k(l), self.kv.v(l),
                   outs[l]) for l in range(self.n_layers)]
        self.ctx.decode_step(self.prm, layers, self.rope, self.kv.capacity, pos=pos,
                             use_meta=use_meta, stream=stream)
