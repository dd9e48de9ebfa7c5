"""Generate the golden fixtures of tests/golden/ from the reference's own shaders.

Runs oracle/_ref (the reference's QK_PREP / ATTN / VISION_ATTN / GEMV WGSL, translated to C++ by
oracle/wgsl2cpp.py, which needs the reference sources) on seeded inputs at the reference's
hard-coded shapes (16 q heads, 8 kv heads, head_dim 64, qkv row 2048, q row 1024, vision row
768), dispatched exactly as engine.js:221-222 and vision.js:271-276 do, and stores inputs and
outputs as compressed .npz files.  The RoPE table is engine.js:60-71 as restated by the
oracle (the reference computes it in JavaScript).

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import pyoracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def decoder_case(name: str, seed: int, pos0: int, m: int, with_norm_scale: float):
    rng = np.random.default_rng(seed)
    cap = pos0 + m
    qkv = rng.standard_normal((m, 2048)).astype(np.float16)
    nwb = (1.0 + with_norm_scale * rng.standard_normal(128)).astype(np.float16)
    kc = rng.standard_normal((cap, 8, 64)).astype(np.float16)
    vc = rng.standard_normal((cap, 8, 64)).astype(np.float16)
    kc[pos0:] = 0
    vc[pos0:] = 0
    rope = O.rope_table(max(cap, 256))
    meta = np.array([pos0, m, 0, 0], np.uint32)
    qout = np.zeros((m, 1024), np.float16)
    kc_out, vc_out = kc.copy(), vc.copy()
    O.ref_qk_prep(qkv, nwb, qout, kc_out, vc_out, meta, rope, m)
    out = np.zeros((m, 1024), np.float16)
    O.ref_attn(qout, kc_out, vc_out, out, meta, m)
    assert np.array_equal(kc_out[:pos0], kc[:pos0]) and np.array_equal(vc_out[:pos0], vc[:pos0])
    # Rows before pos0 are unchanged by QK_PREP, so only the appended rows are stored.
    np.savez_compressed(OUT / f"{name}.npz", qkv=qkv, nwb=nwb, kc_in=kc[:pos0], vc_in=vc[:pos0],
                        rope=rope[:cap], meta=meta, qout=qout, k_new=kc_out[pos0:],
                        v_new=vc_out[pos0:], out=out)


def vision_case(name: str, seed: int, s_tokens: int):
    rng = np.random.default_rng(seed)
    q, k, v = ((0.5 * rng.standard_normal((s_tokens, 768))).astype(np.float16) for _ in range(3))
    out = np.zeros_like(q)
    O.ref_vision_attn(q, k, v, out, s_tokens=s_tokens, num_heads=12, scale=0.125)
    np.savez_compressed(OUT / f"{name}.npz", q=q, k=k, v=v, out=out,
                        s_tokens=np.int32(s_tokens))


def gemv_case(name: str, seed: int, k: int, n: int):
    """The GEMV shader (kernels.js:22-68) at the reference's q_proj shape class: one token's
    4-bit projection (x [k] -> y [n]), dispatched N/8 workgroups as engine.js does."""
    rng = np.random.default_rng(seed)
    wq, sc, zp = O.random_q4(rng, n, k)
    x = rng.standard_normal(k).astype(np.float16)
    y = np.zeros(n, np.float16)
    O.ref_gemv(x, wq, sc, zp, y)
    np.savez_compressed(OUT / f"{name}.npz", x=x, wq=wq, sc=sc, zp=zp, y=y)


def gemm_case(name: str, seed: int, m: int, k: int, n: int, y_off: int):
    """The GEMM shader (kernels.js:70-145): a prompt chunk's 4-bit projection (x [m][k] ->
    y [m][y_off + n] inside rows of y_off + n + 5), (N/64, M/64) workgroups as engine.js
    dispatches it."""
    rng = np.random.default_rng(seed)
    wq, sc, zp = O.random_q4(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float16)
    stride = y_off + n + 5
    y = np.zeros((m, stride), np.float16)
    O.ref_gemm(x, wq, sc, zp, y, stride, y_off)
    np.savez_compressed(OUT / f"{name}.npz", x=x, wq=wq, sc=sc, zp=zp, y=y,
                        y_off=np.int32(y_off))


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref not built: run `make -C oracle` where the reference exists")
    decoder_case("decoder_prefill_16x8", seed=101, pos0=60, m=4, with_norm_scale=0.1)
    decoder_case("decoder_decode_16x8", seed=202, pos0=130, m=1, with_norm_scale=0.1)
    vision_case("vision_s70_h12", seed=303, s_tokens=70)
    gemv_case("gemv_q4_k1024_n96", seed=404, k=1024, n=96)
    gemm_case("gemm_q4_m70_k256_n96", seed=505, m=70, k=256, n=96, y_off=7)
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
