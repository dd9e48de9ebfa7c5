"""GPU parity of the tcgen05 flash-attention kernel (prefill ATTN for M > 1 and VISION_ATTN)
against the oracle, through the C ABI; |x - r| <= 2e-3 + 1e-2 |r| on seeded inputs."""
import numpy as np
import pytest

from conftest import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

D = 64


@pytest.fixture(scope="module")
def ctx():
    import p2p_b200
    c = p2p_b200.Context(0)
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def test_golden_prefill_fixture(ctx, golden_dir):
    """The reference shaders' own output: 16 q / 8 kv heads, chunk of 4 tokens at pos0 60."""
    import p2p_b200
    z = np.load(golden_dir / "decoder_prefill_16x8.npz")
    pos0, m = int(z["meta"][0]), int(z["meta"][1])
    kc = np.concatenate([z["kc_in"], np.zeros((m, 8, D), np.float16)])
    vc = np.concatenate([z["vc_in"], np.zeros((m, 8, D), np.float16)])
    prm = p2p_b200.Params(16, 8, scale=0.125)
    q = torch.zeros((m, 1024), dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    ctx.meta_write(pos0, m)
    ctx.qk_prep(prm, dev(z["qkv"]), dev(z["nwb"]), dev(z["rope"]), q, kc_g, vc_g, m_tokens=m,
                use_meta=True)
    out = torch.zeros((m, 1024), dtype=torch.float16, device="cuda")
    ctx.attn(prm, q, kc_g, vc_g, out, m_tokens=m, use_meta=True)
    ctx.sync()
    assert np.array_equal(bits(host(q)), bits(z["qout"]))
    assert np.array_equal(bits(host(kc_g)[pos0:]), bits(z["k_new"]))
    assert np.array_equal(bits(host(vc_g)[pos0:]), bits(z["v_new"]))
    assert_close(host(out), z["out"], what="golden prefill")


def run_prefill(ctx, oracle, hq, hkv, pos0, m, seed, garbage_tail=False, cap_extra=0):
    import p2p_b200
    rng = np.random.default_rng(seed)
    cap = pos0 + m + cap_extra
    q = (0.5 * rng.standard_normal((m, hq * D))).astype(np.float16)
    kc = (0.5 * rng.standard_normal((cap, hkv, D))).astype(np.float16)
    vc = (0.5 * rng.standard_normal((cap, hkv, D))).astype(np.float16)
    if garbage_tail:  # rows past the last key are never read (NaN there must not leak)
        kc[pos0 + m:] = np.nan
        vc[pos0 + m:] = np.nan
    want = np.zeros((m, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q, kc, vc, want, pos0, m)
    out = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    ctx.attn(p2p_b200.Params(hq, hkv), dev(q), dev(kc), dev(vc), out, pos0=pos0, m_tokens=m)
    ctx.sync()
    return host(out), want


@pytest.mark.parametrize("pos0,m", [(0, 2), (0, 127), (0, 128), (0, 129), (0, 300),
                                    (57, 200), (300, 256), (1000, 77), (4096, 64)])
def test_prefill_causal_shapes(ctx, oracle, pos0, m):
    got, want = run_prefill(ctx, oracle, 32, 8, pos0, m, seed=pos0 * 7 + m)
    assert_close(got, want, what=f"prefill pos0={pos0} M={m}")


def test_prefill_lfm_1p2b_s2048(ctx, oracle):
    """Causal prefill of a 2048-token prompt, 32 q / 8 kv heads (the prefill benchmark shape)."""
    got, want = run_prefill(ctx, oracle, 32, 8, 0, 2048, seed=2048)
    assert_close(got, want, what="prefill S=2048")


@pytest.mark.parametrize("hq,hkv", [(16, 8), (8, 8), (32, 4), (64, 8)])
def test_prefill_group_sizes(ctx, oracle, hq, hkv):
    got, want = run_prefill(ctx, oracle, hq, hkv, 33, 190, seed=hq * hkv)
    assert_close(got, want, what=f"G={hq // hkv}")


def test_prefill_ignores_rows_past_the_last_key(ctx, oracle):
    got, want = run_prefill(ctx, oracle, 32, 8, 10, 100, seed=5, garbage_tail=True, cap_extra=90)
    assert np.isfinite(got.astype(np.float32)).all()
    assert_close(got, want, what="NaN tail")


def test_prefill_full_pipeline_writes_decode_cache(ctx, oracle):
    """QK_PREP over the prompt writes the cache that the next decode step reads."""
    import p2p_b200
    hq, hkv, m = 32, 8, 333
    rng = np.random.default_rng(11)
    qkv = (0.5 * rng.standard_normal((m + 1, (hq + 2 * hkv) * D))).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
    rope = oracle.rope_table(m + 1)
    cap = m + 1
    kc_o = np.zeros((cap, hkv, D), np.float16)
    vc_o = np.zeros_like(kc_o)
    q_o = np.zeros((m, hq * D), np.float16)
    oracle.qk_prep(hq, hkv, D, qkv[:m], nw, rope, q_o, kc_o, vc_o, 0, m)
    want = np.zeros((m, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q_o, kc_o, vc_o, want, 0, m)
    prm = p2p_b200.Params(hq, hkv)
    kc, vc = torch.zeros((cap, hkv, D), dtype=torch.float16, device="cuda"), \
        torch.zeros((cap, hkv, D), dtype=torch.float16, device="cuda")
    q = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    out = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    rg = dev(rope)
    ctx.qk_prep(prm, dev(qkv[:m]), dev(nw), rg, q, kc, vc, pos0=0, m_tokens=m)
    ctx.attn(prm, q, kc, vc, out, pos0=0, m_tokens=m)
    assert_close(host(out), want, what="prefill after qk_prep")
    assert np.array_equal(bits(host(kc)[:m]), bits(kc_o[:m]))
    # next token: fused decode step on the prefilled cache
    q1 = np.zeros((1, hq * D), np.float16)
    oracle.qk_prep(hq, hkv, D, qkv[m:], nw, rope, q1, kc_o, vc_o, m, 1)
    want1 = np.zeros((1, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q1, kc_o, vc_o, want1, m, 1)
    out1 = torch.zeros((hq * D,), dtype=torch.float16, device="cuda")
    ctx.decode_step(prm, [(dev(qkv[m]), dev(nw), kc, vc, out1)], rg, cap, pos=m)
    assert_close(host(out1)[None], want1, what="decode after prefill")


def test_golden_vision_fixture(ctx, golden_dir):
    import p2p_b200
    z = np.load(golden_dir / "vision_s70_h12.npz")
    out = torch.zeros((1, 70, 768), dtype=torch.float16, device="cuda")
    ctx.attn_bidir(p2p_b200.Params(12, 12, scale=0.125), dev(z["q"][None]), dev(z["k"][None]),
                   dev(z["v"][None]), out)
    ctx.sync()
    assert_close(host(out)[0], z["out"], what="golden vision")


@pytest.mark.parametrize("b,s", [(2, 1024), (3, 200), (1, 1), (2, 129)])
def test_vision_bidirectional(ctx, oracle, b, s):
    import p2p_b200
    rng = np.random.default_rng(b * 1000 + s)
    q, k, v = ((0.5 * rng.standard_normal((b, s, 768))).astype(np.float16) for _ in range(3))
    want = np.zeros_like(q)
    oracle.vision_attn(12, D, q, k, v, want)
    out = torch.zeros((b, s, 768), dtype=torch.float16, device="cuda")
    ctx.attn_bidir(p2p_b200.Params(12, 12), dev(q), dev(k), dev(v), out)
    ctx.sync()
    assert_close(host(out), want, what=f"vision B={b} S={s}")


def test_vision_siglip2_batch16_sampled(ctx, oracle):
    """The SigLIP2-base vision attention at full size (16 images x 1024 patches x 12 heads):
    GPU on all images, oracle on images 0 and 15."""
    import p2p_b200
    b, s = 16, 1024
    g = torch.Generator(device="cuda").manual_seed(9)
    q, k, v = ((0.5 * torch.randn((b, s, 768), generator=g, device="cuda")).half()
               for _ in range(3))
    out = torch.zeros_like(q)
    ctx.attn_bidir(p2p_b200.Params(12, 12), q, k, v, out)
    got = host(out)
    for i in (0, 15):
        want = np.zeros((1, s, 768), np.float16)
        oracle.vision_attn(12, D, host(q)[i:i + 1], host(k)[i:i + 1], host(v)[i:i + 1], want)
        assert_close(got[i:i + 1], want, what=f"vision image {i}")


def test_attn_scatter_two_outputs_head_halves(ctx, oracle):
    """p2p_attn_scatter on one GPU: the two halves of the heads (as two ranks of a head-sharded
    prefill would own them) each write their rows into two full-layout buffers at their head
    columns; both buffers must then equal attention over all heads."""
    import p2p_b200
    hq, hkv, m = 32, 8, 300
    rng = np.random.default_rng(515)
    q = (0.5 * rng.standard_normal((m, hq * D))).astype(np.float16)
    kc = (0.5 * rng.standard_normal((m, hkv, D))).astype(np.float16)
    vc = (0.5 * rng.standard_normal((m, hkv, D))).astype(np.float16)
    want = np.zeros((m, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q, kc, vc, want, 0, m)
    a = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    b = torch.zeros_like(a)
    half_q, half_kv = hq // 2, hkv // 2
    for part in (0, 1):
        q_p = dev(q[:, part * half_q * D:(part + 1) * half_q * D])
        kc_p = dev(kc[:, part * half_kv:(part + 1) * half_kv])
        vc_p = dev(vc[:, part * half_kv:(part + 1) * half_kv])
        ctx.attn_scatter(p2p_b200.Params(half_q, half_kv), q_p, kc_p, vc_p,
                         [a.data_ptr(), b.data_ptr()], hq * D, part * half_q, pos0=0,
                         m_tokens=m)
    ctx.sync()
    assert_close(host(a), want, what="scatter output 0")
    assert np.array_equal(bits(host(a)), bits(host(b)))


def test_prefill_device_position_beyond_cache_is_refused(ctx):
    """A prompt chunk whose device-side position runs past the cache rows: the q rows whose
    keys the cache does not hold (here the second pair of 128-row tiles) are not written, and
    p2p_sync reports P2P_ERR_KV_FULL (the reference's 'kv_full'); the context stays usable."""
    import p2p_b200
    hq, hkv, m, cap = 32, 8, 300, 400
    q = torch.ones((m, hq * D), dtype=torch.float16, device="cuda")
    kc = torch.zeros((cap, hkv, D), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.full((m, hq * D), 7.0, dtype=torch.float16, device="cuda")
    prm = p2p_b200.Params(hq, hkv)
    ctx.meta_write(cap - m + 1, m)  # rows 256.. need keys up to cap + 1
    ctx.attn(prm, q, kc, vc, out, m_tokens=m, use_meta=True)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.sync()
    assert bool((out[256:] == 7.0).all())
    ctx.meta_write(cap - m, m)
    ctx.attn(prm, q, kc, vc, out, m_tokens=m, use_meta=True)
    ctx.sync()
    assert bool(torch.isfinite(out.float()).all())


@pytest.mark.parametrize("scale_in", [1.0, 0.5])
def test_prefill_s2048_with_norm_weights_full_oracle(ctx, oracle, scale_in):
    """Config 3 through the engine's two dispatches (QK_PREP with learned norm weights, then
    ATTN) at S = 2048, 32 q / 8 kv heads, q/k/v N(0,1) unscaled and x0.5: every output row
    against the oracle; max-abs also held to the 2e-3 cap on its own."""
    import p2p_b200
    hq, hkv, m = 32, 8, 2048
    rng = np.random.default_rng(20480 + int(10 * scale_in))
    qkv = (scale_in * rng.standard_normal((m, (hq + 2 * hkv) * D))).astype(np.float16)
    nw = (1 + 0.2 * rng.standard_normal(2 * D)).astype(np.float16)
    rope = oracle.rope_table(m)
    kc_o = np.zeros((m, hkv, D), np.float16)
    vc_o = np.zeros_like(kc_o)
    q_o = np.zeros((m, hq * D), np.float16)
    oracle.qk_prep(hq, hkv, D, qkv, nw, rope, q_o, kc_o, vc_o, 0, m)
    want = np.zeros((m, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q_o, kc_o, vc_o, want, 0, m)
    prm = p2p_b200.Params(hq, hkv)
    kc = torch.zeros((m, hkv, D), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    ctx.qk_prep(prm, dev(qkv), dev(nw), dev(rope), q, kc, vc, pos0=0, m_tokens=m)
    ctx.attn(prm, q, kc, vc, out, pos0=0, m_tokens=m)
    assert np.array_equal(bits(host(q)), bits(q_o))
    assert np.array_equal(bits(host(kc)), bits(kc_o))
    max_abs, _ = assert_close(host(out), want, what=f"prefill S=2048 x{scale_in} with norm")
    assert max_abs <= 2e-3
