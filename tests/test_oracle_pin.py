"""Pins the CPU oracle (the C++ restatement) to the reference.

1. Bit-for-bit against the reference's own WGSL shaders (QK_PREP, ATTN, VISION_ATTN), run on
   the host through oracle/_ref (translated by oracle/wgsl2cpp.py; built only where the
   reference sources exist).
2. Bit-for-bit against the committed golden fixtures generated from those shaders
   (tests/golden/make_golden.py), which travel with the repository.
3. toHalfBits (engine.js:28-50) against IEEE round-to-nearest-even, ropeTable
   (engine.js:60-71) against double-precision trigonometry.
"""
import numpy as np
import pytest

from conftest import ROOT


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def test_f16_conversion_is_ieee_rne(oracle):
    rng = np.random.default_rng(0)
    x = rng.integers(0, 2**32, 1 << 22, dtype=np.uint64).astype(np.uint32).view(np.float32)
    # every binary16 rounding boundary: midpoints between neighbours and one f32 ulp either side
    h = np.arange(0, 0x7C00, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    mid = (h[:-1].astype(np.float64) + h[1:].astype(np.float64)) / 2
    mids = mid.astype(np.float32)
    edges = np.concatenate([mids, np.nextafter(mids, np.float32(np.inf)),
                            np.nextafter(mids, np.float32(0)), h])
    edges = np.concatenate([edges, -edges, np.float32([65504, 65519.99, 65520, 1e6, -1e6])])
    for arr in (x, edges.astype(np.float32)):
        got = oracle.f32_to_f16(arr)
        nan = np.isnan(arr)
        with np.errstate(over="ignore"):
            want = arr.astype(np.float16)
        assert np.array_equal(_bits(got)[~nan], _bits(want)[~nan])
        assert np.isnan(got[nan]).all()
    back = oracle.f16_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16))
    ref = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    fin = ~np.isnan(ref)
    assert np.array_equal(back[fin].view(np.uint32), ref[fin].view(np.uint32))


def test_rope_table_matches_double_trig(oracle):
    max_ctx, d, theta = 4097, 64, 1e6
    t = oracle.rope_table(max_ctx, d, theta)
    p = np.arange(max_ctx, dtype=np.float64)[:, None]
    i = np.arange(d // 2, dtype=np.float64)[None, :]
    ang = p * np.power(theta, -i / (d // 2))
    want = np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32).astype(np.float16)
    assert np.array_equal(_bits(t), _bits(want))
    assert np.all(t[0, :32] == 1) and np.all(t[0, 32:] == 0)  # position 0 is the identity


ref_only = pytest.mark.skipif(
    not (ROOT / "oracle" / "_ref" / "libp2pref.so").exists(),
    reason="oracle/_ref (the reference's shaders) not built here")


@ref_only
@pytest.mark.parametrize("pos0,m,seed", [(0, 1, 1), (0, 7, 2), (127, 1, 3), (128, 1, 4),
                                         (200, 37, 5), (5, 300, 6)])
def test_restatement_matches_reference_decoder_shaders(oracle, pos0, m, seed):
    rng = np.random.default_rng(seed)
    cap = pos0 + m
    qkv = rng.standard_normal((m, 2048)).astype(np.float16)
    nwb = (1 + 0.2 * rng.standard_normal(128)).astype(np.float16)
    rope = oracle.rope_table(max(cap, 1))
    kc0 = rng.standard_normal((cap, 8, 64)).astype(np.float16)
    vc0 = rng.standard_normal((cap, 8, 64)).astype(np.float16)
    meta = np.array([pos0, m, 0, 0], np.uint32)
    qa, ka, va = np.zeros((m, 1024), np.float16), kc0.copy(), vc0.copy()
    oracle.ref_qk_prep(qkv, nwb, qa, ka, va, meta, rope, m)
    qb, kb, vb = np.zeros((m, 1024), np.float16), kc0.copy(), vc0.copy()
    oracle.qk_prep(16, 8, 64, qkv, nwb, rope, qb, kb, vb, pos0, m)
    assert np.array_equal(_bits(qa), _bits(qb))
    assert np.array_equal(_bits(ka), _bits(kb)) and np.array_equal(_bits(va), _bits(vb))
    oa, ob = np.zeros((m, 1024), np.float16), np.zeros((m, 1024), np.float16)
    oracle.ref_attn(qa, ka, va, oa, meta, m)
    oracle.attn(16, 8, 64, qb, kb, vb, ob, pos0, m)
    assert np.array_equal(_bits(oa), _bits(ob))


@ref_only
@pytest.mark.parametrize("s_tokens,seed", [(1, 7), (64, 8), (130, 9)])
def test_restatement_matches_reference_vision_shader(oracle, s_tokens, seed):
    rng = np.random.default_rng(seed)
    q, k, v = ((0.5 * rng.standard_normal((1, s_tokens, 768))).astype(np.float16)
               for _ in range(3))
    oa, ob = np.zeros_like(q), np.zeros_like(q)
    oracle.ref_vision_attn(q[0], k[0], v[0], oa[0], s_tokens=s_tokens)
    oracle.vision_attn(12, 64, q, k, v, ob)
    assert np.array_equal(_bits(oa), _bits(ob))


def _argmax_cases():
    """Logits for ARGMAX: random, ties at the maximum, all -inf, NaNs mixed in; vocab sizes
    65536 (the model's), one that is not a multiple of 8, and 1."""
    rng = np.random.default_rng(31)
    out = []
    for v in (65536, 1001, 1):
        lg = rng.standard_normal(v).astype(np.float16)
        out.append(lg)
        t = lg.copy()
        t[rng.integers(0, v, 5)] = t.max()
        out.append(t)
        out.append(np.full(v, -np.inf, np.float16))
        t = lg.copy()
        t[::7] = np.nan
        out.append(t)
    return out


def argmax_rule(lg):
    """The shaders' result in closed form: the smallest index among the maxima of the values
    above -3e38 (NaN never wins), else 0."""
    x = lg.astype(np.float32)
    ok = ~np.isnan(x) & (x > -3e38)
    if not ok.any():
        return 0
    return int(np.flatnonzero(ok & (x == x[ok].max()))[0])


def test_argmax_restatement_rule(oracle):
    """kernels.js:362-399 restated: token, out_tok[step] and the advance of step and position."""
    for lg in _argmax_cases():
        tok = np.zeros(1, np.uint32)
        meta = np.array([100, 1, 3, 0], np.uint32)
        out_tok = np.zeros(8, np.uint32)
        oracle.argmax(lg, tok, meta, out_tok)
        assert tok[0] == argmax_rule(lg) and out_tok[3] == tok[0]
        assert list(meta) == [101, 1, 4, 0]


@ref_only
def test_argmax_restatement_matches_reference_shader(oracle):
    for lg in _argmax_cases():
        res = []
        for fn in (oracle.ref_argmax, oracle.argmax):
            tok = np.zeros(4, np.uint32)
            meta = np.array([4096, 1, 5, 0], np.uint32)
            out_tok = np.zeros(16, np.uint32)
            fn(lg, tok, meta, out_tok)
            res.append((tok.copy(), meta.copy(), out_tok.copy()))
        for a, b in zip(*res):
            assert np.array_equal(a, b)


def _load_decoder(golden_dir, name):
    z = np.load(golden_dir / f"{name}.npz")
    pos0, m = int(z["meta"][0]), int(z["meta"][1])
    kc = np.concatenate([z["kc_in"], np.zeros((m, 8, 64), np.float16)])
    vc = np.concatenate([z["vc_in"], np.zeros((m, 8, 64), np.float16)])
    return z, pos0, m, kc, vc


@pytest.mark.parametrize("name", ["decoder_prefill_16x8", "decoder_decode_16x8"])
def test_restatement_reproduces_golden_decoder(oracle, golden_dir, name):
    z, pos0, m, kc, vc = _load_decoder(golden_dir, name)
    q = np.zeros((m, 1024), np.float16)
    oracle.qk_prep(16, 8, 64, z["qkv"], z["nwb"], z["rope"], q, kc, vc, pos0, m)
    assert np.array_equal(_bits(q), _bits(z["qout"]))
    assert np.array_equal(_bits(kc[pos0:]), _bits(z["k_new"]))
    assert np.array_equal(_bits(vc[pos0:]), _bits(z["v_new"]))
    out = np.zeros((m, 1024), np.float16)
    oracle.attn(16, 8, 64, q, kc, vc, out, pos0, m)
    assert np.array_equal(_bits(out), _bits(z["out"]))


def test_restatement_reproduces_golden_vision(oracle, golden_dir):
    z = np.load(golden_dir / "vision_s70_h12.npz")
    out = np.zeros_like(z["q"])[None]
    oracle.vision_attn(12, 64, z["q"][None], z["k"][None], z["v"][None], out)
    assert np.array_equal(_bits(out[0]), _bits(z["out"]))


@ref_only
@pytest.mark.parametrize("k,n,seed", [(1024, 2048, 1), (2048, 3072, 2), (96, 40, 3), (4608, 16, 4)])
def test_gemv_restatement_matches_reference_shader(oracle, k, n, seed):
    """kernels.js:22-68 (GEMV): the restatement equals the translated shader bit for bit,
    including an odd block count (K = 96: the zero-point row ends mid-byte) and the largest K
    its workgroup array holds (4608)."""
    rng = np.random.default_rng(seed)
    wq, sc, zp = oracle.random_q4(rng, n, k)
    x = (2 * rng.standard_normal(k)).astype(np.float16)
    want = np.zeros(n + 5, np.float16)
    oracle.ref_gemv(x, wq, sc, zp, want, y_off=5)
    got = oracle.gemv_q4(x, wq, sc, zp, y=np.zeros(n + 5, np.float16), y_off=5)
    assert np.array_equal(_bits(got), _bits(want))


@ref_only
@pytest.mark.parametrize("m,k,n,seed", [(5, 64, 70, 1), (64, 256, 128, 2), (130, 96, 40, 3),
                                         (77, 1024, 200, 4)])
def test_gemm_restatement_matches_reference_shader(oracle, m, k, n, seed):
    """kernels.js:70-145 (GEMM): the restatement equals the translated shader bit for bit,
    with partial 64-row / 64-column tiles, an odd block count (K = 96) and the output written
    at an offset inside wider rows (Y_STRIDE, Y_OFF)."""
    rng = np.random.default_rng(100 + seed)
    wq, sc, zp = oracle.random_q4(rng, n, k)
    x = (2 * rng.standard_normal((m, k))).astype(np.float16)
    stride, off = n + 9, 3
    want = np.zeros((m, stride), np.float16)
    oracle.ref_gemm(x, wq, sc, zp, want, stride, off)
    got = oracle.gemm_q4(x, wq, sc, zp, y_stride=stride, y_off=off)
    assert np.array_equal(_bits(got), _bits(want))


def test_gemm_restatement_reproduces_golden(oracle, golden_dir):
    z = np.load(golden_dir / "gemm_q4_m70_k256_n96.npz")
    got = oracle.gemm_q4(z["x"], z["wq"], z["sc"], z["zp"], y_stride=int(z["y"].shape[1]),
                         y_off=int(z["y_off"]))
    assert np.array_equal(_bits(got), _bits(z["y"]))


def test_gemv_restatement_reproduces_golden(oracle, golden_dir):
    z = np.load(golden_dir / "gemv_q4_k1024_n96.npz")
    got = oracle.gemv_q4(z["x"], z["wq"], z["sc"], z["zp"])
    assert np.array_equal(_bits(got), _bits(z["y"]))
