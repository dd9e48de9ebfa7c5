"""Known-answer tests of the oracle at the LFM2.5-1.2B shape (32 q / 8 kv heads) and fp32.

These pin properties the reference has no tests for: uniform V, a single key, a dominant
score, RoPE at position 0, GQA reducing to MHA, and the causal mask at the first token; plus
the oracle's own rounding error against a float64 evaluation.
"""
import numpy as np

from conftest import assert_close

HQ, HKV, D = 32, 8, 64


def _rand(rng, shape, scale=1.0, dtype=np.float16):
    return (scale * rng.standard_normal(shape)).astype(dtype)


def test_uniform_v_gives_v(oracle):
    rng = np.random.default_rng(1)
    pos0, m = 200, 3
    q = _rand(rng, (m, HQ * D))
    kc = _rand(rng, (pos0 + m, HKV, D))
    vc = np.broadcast_to(_rand(rng, (1, HKV, D)), (pos0 + m, HKV, D)).copy()
    out = np.zeros((m, HQ * D), np.float16)
    oracle.attn(HQ, HKV, D, q, kc, vc, out, pos0, m)
    want = np.repeat(vc[0], HQ // HKV, axis=0).reshape(-1)
    assert_close(out, np.broadcast_to(want, out.shape), what="uniform V")


def test_single_key_gives_its_v(oracle):
    rng = np.random.default_rng(2)
    q = _rand(rng, (1, HQ * D))
    kc = _rand(rng, (1, HKV, D))
    vc = _rand(rng, (1, HKV, D))
    out = np.zeros((1, HQ * D), np.float16)
    oracle.attn(HQ, HKV, D, q, kc, vc, out, 0, 1)
    want = np.repeat(vc[0], HQ // HKV, axis=0).reshape(1, -1)
    assert np.array_equal(out.view(np.uint16), want.view(np.uint16))


def test_dominant_score_selects_row(oracle):
    rng = np.random.default_rng(3)
    pos = 300
    kc = _rand(rng, (pos + 1, HKV, D), 0.01)
    vc = _rand(rng, (pos + 1, HKV, D))
    q = np.zeros((1, HQ * D), np.float16)
    q[0, :] = 8.0
    kc[137] = 8.0  # scores 0.125 * 64 * 64 = 512 for key 137, ~0 elsewhere
    out = np.zeros((1, HQ * D), np.float16)
    oracle.attn(HQ, HKV, D, q, kc, vc, out, pos, 1)
    want = np.repeat(vc[137], HQ // HKV, axis=0).reshape(1, -1)
    assert_close(out, want, what="one-hot")


def test_rope_position_zero_is_identity(oracle):
    rng = np.random.default_rng(4)
    qkv = _rand(rng, (1, (HQ + 2 * HKV) * D))
    rope = oracle.rope_table(4)
    q = np.zeros((1, HQ * D), np.float16)
    kc = np.zeros((4, HKV, D), np.float16)
    vc = np.zeros((4, HKV, D), np.float16)
    oracle.qk_prep(HQ, HKV, D, qkv, None, rope, q, kc, vc, 0, 1)
    assert np.array_equal(q.view(np.uint16), qkv[:, :HQ * D].view(np.uint16))
    assert np.array_equal(kc[0].reshape(-1).view(np.uint16),
                          qkv[0, HQ * D:(HQ + HKV) * D].view(np.uint16))
    assert np.array_equal(vc[0].reshape(-1).view(np.uint16),
                          qkv[0, (HQ + HKV) * D:].view(np.uint16))


def test_gqa_equals_mha_with_repeated_kv(oracle):
    rng = np.random.default_rng(5)
    pos0, m = 150, 4
    q = _rand(rng, (m, HQ * D))
    kc = _rand(rng, (pos0 + m, HKV, D))
    vc = _rand(rng, (pos0 + m, HKV, D))
    a = np.zeros((m, HQ * D), np.float16)
    oracle.attn(HQ, HKV, D, q, kc, vc, a, pos0, m)
    kr = np.ascontiguousarray(np.repeat(kc, HQ // HKV, axis=1))
    vr = np.ascontiguousarray(np.repeat(vc, HQ // HKV, axis=1))
    b = np.zeros_like(a)
    oracle.attn(HQ, HQ, D, q, kr, vr, b, pos0, m)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def test_causal_first_token_sees_only_key_zero(oracle):
    rng = np.random.default_rng(6)
    m = 5
    q = _rand(rng, (m, HQ * D))
    kc = _rand(rng, (m, HKV, D))
    vc = _rand(rng, (m, HKV, D))
    out = np.zeros((m, HQ * D), np.float16)
    oracle.attn(HQ, HKV, D, q, kc, vc, out, 0, m)
    want = np.repeat(vc[0], HQ // HKV, axis=0).reshape(-1)
    assert np.array_equal(out[0].view(np.uint16), want.view(np.uint16))
    vc2 = vc.copy()
    vc2[1:] = 0  # later rows must not influence token 0
    out2 = np.zeros_like(out)
    oracle.attn(HQ, HKV, D, q, kc, vc2, out2, 0, m)
    assert np.array_equal(out2[0].view(np.uint16), out[0].view(np.uint16))


def test_oracle_error_against_float64(oracle):
    rng = np.random.default_rng(7)
    pos0, m = 4096, 1
    q = _rand(rng, (m, HQ * D))
    kc = _rand(rng, (pos0 + 1, HKV, D))
    vc = _rand(rng, (pos0 + 1, HKV, D))
    out = np.zeros((m, HQ * D), np.float16)
    oracle.attn(HQ, HKV, D, q, kc, vc, out, pos0, m)
    ex = oracle.attn_exact(HQ, HKV, D, q, kc, vc, pos0, m)
    # the f16 output rounding dominates: half an f16 ulp of |out| < 1
    assert np.abs(out.astype(np.float64) - ex).max() < 5e-4


def test_fp32_storage_decode_case(oracle):
    """The fp32 decode case (past 512 + 1 new, RoPE theta 1e6, no q/k norm)."""
    rng = np.random.default_rng(8)
    past = 512
    qkv = rng.standard_normal((1, (HQ + 2 * HKV) * D)).astype(np.float32)
    kc = np.zeros((past + 1, HKV, D), np.float32)
    vc = np.zeros((past + 1, HKV, D), np.float32)
    kc[:past] = rng.standard_normal((past, HKV, D))
    vc[:past] = rng.standard_normal((past, HKV, D))
    rope = oracle.rope_table(past + 1, D, 1e6, f32=True)
    q = np.zeros((1, HQ * D), np.float32)
    oracle.qk_prep(HQ, HKV, D, qkv, None, rope, q, kc, vc, past, 1)
    out = np.zeros((1, HQ * D), np.float32)
    oracle.attn(HQ, HKV, D, q, kc, vc, out, past, 1)
    # float64 reference of the same math
    qh = q.reshape(HQ, D).astype(np.float64)
    k64, v64 = kc.astype(np.float64), vc.astype(np.float64)
    want = np.empty((HQ, D))
    for h in range(HQ):
        s = k64[:, h // 4, :] @ qh[h] * 0.125
        p = np.exp(s - s.max())
        want[h] = p @ v64[:, h // 4, :] / p.sum()
    assert np.abs(out.reshape(HQ, D) - want).max() < 1e-5
