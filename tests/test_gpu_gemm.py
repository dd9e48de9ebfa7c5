"""The prompt-chunk 4-bit projection on the tensor cores (gemm_q4.cu) against the oracle's
restatement of the GEMM shader (kernels.js:70-145), which the CPU tests pin bit for bit to the
reference's own shader.

The kernel dequantises the weights to f16 once per call (the shader keeps them in f32), so its
result is not bit-identical.  The tolerance written here follows from that one rounding: each
weight moves by at most 2^-11 of itself, so the exact sums differ by at most
2^-11 * sum_k |x_k w_k|; the f32 accumulation (different order, K <= 4608) adds less than
2^-13 of the same sum; the final f16 rounding of each side adds at most one f16 ulp of the
result.  The test allows 2^-10 * sum_k |x_k w_k| + 1 ulp.

The fused q/k/v form (QK_PREP in the epilogue, engine.js:202-204 then kernels.js:216-266) is
checked bit for bit against the same GPU GEMM followed by the QK_PREP kernel (both bit-identical
per stage to what they restate), and to a tolerance against the oracle's GEMM + QK_PREP.
"""
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
    return t.detach().cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def dev_q4(m):
    wq, sc, zp = m
    return dev(wq.view(np.int32)), dev(sc), dev(zp.view(np.int32))


def gemm_tolerance(x, m):
    """2^-10 * sum_k |x_k w_k| + 1 f16 ulp of the reference result, per output element."""
    from oracle import pyoracle
    w = pyoracle.dequant_q4(*m).astype(np.float64)
    return 2.0 ** -10 * (np.abs(x.astype(np.float64)) @ np.abs(w).T)


def assert_gemm_close(got, want, tol, what):
    got = got.astype(np.float64)
    want16 = want.astype(np.float16)
    ulp = np.spacing(np.abs(want16)).astype(np.float64)
    err = np.abs(got - want.astype(np.float64))
    bad = err > tol + ulp
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} out of tolerance; worst "
                           f"err/bound {float((err / (tol + ulp)).max()):.3f}")
    return float((err / (tol + ulp)).max())


@pytest.mark.parametrize("m,k,n", [(70, 256, 128), (129, 96, 64), (300, 2048, 2048),
                                   (256, 2048, 3072), (128, 4608, 512), (1, 512, 256)])
def test_gemm_against_oracle(ctx, oracle, m, k, n):
    rng = np.random.default_rng(m * 31 + k + n)
    w = oracle.random_q4(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float16)
    want = oracle.gemm_q4(x, *w)
    y = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    ctx.gemm_q4(dev_q4(w), dev(x), y)
    ctx.sync()
    assert_gemm_close(host(y), want, gemm_tolerance(x, w), f"gemm {m}x{k}x{n}")


def test_gemm_writes_only_its_columns(ctx, oracle):
    """y_off / ld_y place the block inside a wider row (engine.js writes q, k and v into one
    qkv row); the columns around it and the rows past M stay untouched."""
    rng = np.random.default_rng(3)
    m, k, n, ld, off = 200, 512, 192, 448, 128
    w = oracle.random_q4(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float16)
    y0 = rng.standard_normal((m + 5, ld)).astype(np.float16)
    want = oracle.gemm_q4(x, *w, y=y0[:m].copy(), y_stride=ld, y_off=off)
    y = dev(y0)
    ctx.gemm_q4(dev_q4(w), dev(x), y, y_off=off, m_tokens=m)
    ctx.sync()
    got = host(y)
    assert np.array_equal(bits(got[:, :off]), bits(y0[:, :off]))
    assert np.array_equal(bits(got[:, off + n:]), bits(y0[:, off + n:]))
    assert np.array_equal(bits(got[m:]), bits(y0[m:]))
    assert_gemm_close(got[:m, off:off + n], want[:, off:off + n], gemm_tolerance(x, w), "placed")


def test_gemm_golden_fixture(ctx, golden_dir):
    """The committed GEMM vector (made by the reference's own shader): N = 96 is padded to the
    kernel's 64-column unit with zero rows, whose outputs are exactly 0."""
    z = np.load(golden_dir / "gemm_q4_m70_k256_n96.npz")
    wq, sc, zp, x, want = z["wq"], z["sc"], z["zp"], z["x"], z["y"]
    n, k = wq.shape[0], wq.shape[1] * 8
    npad = 128
    zr = (k // 32 + 1) // 2
    wq_p = np.zeros((npad, wq.shape[1]), np.uint32)
    wq_p[:n] = wq
    sc_p = np.zeros((npad, sc.shape[1]), np.float16)
    sc_p[:n] = sc
    zb = np.zeros(npad * zr + (-(npad * zr)) % 4, np.uint8)
    zb[: n * zr] = zp.view(np.uint8)[: n * zr]
    m = x.shape[0]
    y = torch.zeros((m, npad), dtype=torch.float16, device="cuda")
    ctx.gemm_q4(dev_q4((wq_p, sc_p, zb.view(np.uint32))), dev(x), y)
    ctx.sync()
    got = host(y)
    assert not got[:, n:].any()
    off = int(z["y_off"])
    want = want[:, off:off + n]
    assert_gemm_close(got[:, :n], want, gemm_tolerance(x, (wq, sc, zp)), "golden")


def qkv_case(oracle, rng, hq, hkv, k, m, cap, norm):
    mq, mk, mv = (oracle.random_q4(rng, h * D, k) for h in (hq, hkv, hkv))
    x = rng.standard_normal((m, k)).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16) if norm else None
    rope = oracle.rope_table(cap)
    kc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    return mq, mk, mv, x, nw, rope, kc, vc


@pytest.mark.parametrize("hq,hkv,k,m,norm,use_meta", [(32, 8, 2048, 300, True, False),
                                                      (16, 8, 1024, 129, True, True),
                                                      (32, 8, 2048, 64, False, False),
                                                      (12, 12, 768, 200, True, False)])
def test_qkv_gemm_prep_bit_exact_to_unfused(ctx, oracle, hq, hkv, k, m, norm, use_meta):
    """Fused projection + QK_PREP == the GPU GEMM into one qkv block, then the QK_PREP kernel:
    same f16 projection, same norm / rotation arithmetic, so every bit agrees."""
    import p2p_b200
    rng = np.random.default_rng(hq * 13 + m)
    pos0, cap = 500, 1000
    mq, mk, mv, x, nw, rope, kc, vc = qkv_case(oracle, rng, hq, hkv, k, m, cap, norm)
    prm = p2p_b200.Params(hq, hkv)
    wq, wk, wv = dev_q4(mq), dev_q4(mk), dev_q4(mv)
    g_x, g_nw, g_rope = dev(x), dev(nw) if norm else None, dev(rope)
    # unfused: three GEMMs into one qkv block (engine.js:202-204), then QK_PREP
    w_all = hq + 2 * hkv
    qkv = torch.zeros((m, w_all * D), dtype=torch.float16, device="cuda")
    ctx.gemm_q4(wq, g_x, qkv, y_off=0)
    ctx.gemm_q4(wk, g_x, qkv, y_off=hq * D)
    ctx.gemm_q4(wv, g_x, qkv, y_off=(hq + hkv) * D)
    q_u = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    kc_u, vc_u = dev(kc), dev(vc)
    ctx.qk_prep(prm, qkv, g_nw, g_rope, q_u, kc_u, vc_u, pos0=pos0)
    # fused
    q_f = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    kc_f, vc_f = dev(kc), dev(vc)
    if use_meta:
        ctx.meta_write(pos0, m, 0)
    ctx.qkv_gemm_prep(prm, g_x, wq, wk, wv, g_nw, g_rope, q_f, kc_f, vc_f,
                      pos0=0 if use_meta else pos0, use_meta=use_meta)
    ctx.sync()
    assert np.array_equal(bits(host(q_f)), bits(host(q_u)))
    assert np.array_equal(bits(host(kc_f)), bits(host(kc_u)))
    assert np.array_equal(bits(host(vc_f)), bits(host(vc_u)))
    # rows outside pos0 .. pos0+m-1 untouched
    untouched = np.r_[0:pos0, pos0 + m:cap]
    assert np.array_equal(bits(host(kc_f)[untouched]), bits(kc[untouched]))
    assert np.array_equal(bits(host(vc_f)[untouched]), bits(vc[untouched]))


def test_qkv_gemm_prep_against_oracle(ctx, oracle):
    """LFM2.5-1.2B shapes (32 q heads, 8 kv heads, hidden 2048) against the oracle's GEMM +
    QK_PREP: v rows within the GEMM bound; q / k after the norm and rotation within the
    attention tolerance (the f16 weight rounding is the only source of difference)."""
    import p2p_b200
    hq, hkv, k, m, pos0, cap = 32, 8, 2048, 256, 100, 512
    rng = np.random.default_rng(11)
    mq, mk, mv, x, nw, rope, kc, vc = qkv_case(oracle, rng, hq, hkv, k, m, cap, True)
    row = np.zeros((m, (hq + 2 * hkv) * D), np.float16)
    ld = row.shape[1]
    oracle.gemm_q4(x, *mq, y=row, y_stride=ld, y_off=0)
    oracle.gemm_q4(x, *mk, y=row, y_stride=ld, y_off=hq * D)
    oracle.gemm_q4(x, *mv, y=row, y_stride=ld, y_off=(hq + hkv) * D)
    q_o = np.zeros((m, hq * D), np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    oracle.qk_prep(hq, hkv, D, row, nw, rope, q_o, kc_o, vc_o, pos0, m)
    prm = p2p_b200.Params(hq, hkv)
    q = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    ctx.qkv_gemm_prep(prm, dev(x), dev_q4(mq), dev_q4(mk), dev_q4(mv), dev(nw), dev(rope), q,
                      kc_g, vc_g, pos0=pos0)
    ctx.sync()
    sl = slice(pos0, pos0 + m)
    assert_gemm_close(host(vc_g)[sl].reshape(m, -1), vc_o[sl].reshape(m, -1),
                      gemm_tolerance(x, mv), "v rows")
    # After the RMS norm the rotated values are O(1) (|v| < 4 here) and each is the difference
    # of two f16-rounded products: a one-ulp change of the projection can move an element by
    # two f16 ulps at magnitude 4 (2 * 2^-9), even where the result itself is near zero.
    atol = 2 * 2.0 ** -9
    assert_close(host(q), q_o, atol=atol, rtol=1e-2, what="rotated q")
    assert_close(host(kc_g)[sl], kc_o[sl], atol=atol, rtol=1e-2, what="rotated k")


def test_qkv_gemm_prep_refusals(ctx, oracle):
    """A chunk past the cache: refused on the host (host position) or by the kernel (device
    position, nothing written); f32 parameters: the projection path is f16 only."""
    import p2p_b200
    hq, hkv, k, m, cap = 16, 8, 512, 40, 64
    rng = np.random.default_rng(9)
    mq, mk, mv, x, _, rope, _, _ = qkv_case(oracle, rng, hq, hkv, k, m, cap, False)
    w3 = dev_q4(mq), dev_q4(mk), dev_q4(mv)
    prm = p2p_b200.Params(hq, hkv)
    q = torch.full((m, hq * D), 3.0, dtype=torch.float16, device="cuda")
    kc = torch.zeros((cap, hkv, D), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    g_x, g_rope = dev(x), dev(rope)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.qkv_gemm_prep(prm, g_x, *w3, None, g_rope, q, kc, vc, pos0=cap - m + 1)
    ctx.meta_write(cap, m, 0)
    ctx.qkv_gemm_prep(prm, g_x, *w3, None, g_rope, q, kc, vc, use_meta=True)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.sync()
    assert float(q.float().min()) == 3.0 and float(kc.abs().sum()) == 0
    assert float(vc.abs().sum()) == 0
    with pytest.raises(p2p_b200.P2PError):
        ctx.qkv_gemm_prep(p2p_b200.Params(hq, hkv, dtype=torch.float32), g_x, *w3, None,
                          g_rope, q, kc, vc, pos0=0)


def test_gemm_in_a_graph(ctx, oracle):
    """A prompt chunk's projections captured in a CUDA graph and replayed with new inputs."""
    rng = np.random.default_rng(21)
    m, k, n = 192, 1024, 512
    w = oracle.random_q4(rng, n, k)
    g_w = dev_q4(w)
    g_x = torch.zeros((m, k), dtype=torch.float16, device="cuda")
    y = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    ctx.gemm_q4(g_w, g_x, y)  # workspace sized before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(graph, stream=s):
        ctx.gemm_q4(g_w, g_x, y, stream=s)
    for it in range(2):
        x = rng.standard_normal((m, k)).astype(np.float16)
        g_x.copy_(dev(x))
        graph.replay()
        torch.cuda.synchronize()
        assert_gemm_close(host(y), oracle.gemm_q4(x, *w), gemm_tolerance(x, w), f"replay {it}")
    del graph


FORMS = [(bn, pair) for pair in ("0", "1") for bn in ("256", "192", "128")]


@pytest.mark.parametrize("m,k,n", [(2048, 256, 3072), (300, 512, 2048), (70, 96, 192)])
def test_gemm_tile_forms_agree(ctx, oracle, monkeypatch, m, k, n):
    """The output tile (128 x 256 / 192 / 128 on one CTA, or 256 x 256 / 192 / 128 on a pair of
    CTAs sharing one tcgen05.mma.cta_group::2 stream, chosen per shape) changes only which SM
    computes an element, not its K order: every form gives the same bits, within the bound."""
    rng = np.random.default_rng(m + 3 * n)
    w = oracle.random_q4(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float16)
    g_w, g_x = dev_q4(w), dev(x)
    outs = {}
    for bn, pair in FORMS:
        monkeypatch.setenv("P2P_GEMM_BN", bn)
        monkeypatch.setenv("P2P_GEMM_PAIR", pair)
        y = torch.zeros((m, n), dtype=torch.float16, device="cuda")
        ctx.gemm_q4(g_w, g_x, y)
        ctx.sync()
        outs[(bn, pair)] = host(y)
    monkeypatch.delenv("P2P_GEMM_BN")
    monkeypatch.delenv("P2P_GEMM_PAIR")
    ref = outs[("256", "0")]
    assert_gemm_close(ref, oracle.gemm_q4(x, *w), gemm_tolerance(x, w), "forms")
    for form, got in outs.items():
        assert np.array_equal(bits(got), bits(ref)), f"tile form {form}"


@pytest.mark.parametrize("pair", ["0", "1"])
def test_qkv_gemm_prep_forms_bit_exact(ctx, oracle, monkeypatch, pair):
    """The fused q/k/v + QK_PREP on either tile form equals the unfused GEMMs + QK_PREP."""
    import p2p_b200
    monkeypatch.setenv("P2P_GEMM_PAIR", pair)
    hq, hkv, k, m, pos0, cap = 32, 8, 1024, 700, 37, 800
    rng = np.random.default_rng(41)
    mq, mk, mv, x, nw, rope, kc, vc = qkv_case(oracle, rng, hq, hkv, k, m, cap, True)
    prm = p2p_b200.Params(hq, hkv)
    wq, wk, wv = dev_q4(mq), dev_q4(mk), dev_q4(mv)
    g_x, g_nw, g_rope = dev(x), dev(nw), dev(rope)
    qkv = torch.zeros((m, (hq + 2 * hkv) * D), dtype=torch.float16, device="cuda")
    ctx.gemm_q4(wq, g_x, qkv, y_off=0)
    ctx.gemm_q4(wk, g_x, qkv, y_off=hq * D)
    ctx.gemm_q4(wv, g_x, qkv, y_off=(hq + hkv) * D)
    q_u = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    kc_u, vc_u = dev(kc), dev(vc)
    ctx.qk_prep(prm, qkv, g_nw, g_rope, q_u, kc_u, vc_u, pos0=pos0)
    q_f = torch.zeros_like(q_u)
    kc_f, vc_f = dev(kc), dev(vc)
    ctx.qkv_gemm_prep(prm, g_x, wq, wk, wv, g_nw, g_rope, q_f, kc_f, vc_f, pos0=pos0)
    ctx.sync()
    assert np.array_equal(bits(host(q_f)), bits(host(q_u)))
    assert np.array_equal(bits(host(kc_f)), bits(host(kc_u)))
    assert np.array_equal(bits(host(vc_f)), bits(host(vc_u)))


def test_q4_to_f16_exact(ctx, oracle):
    """The resident f16 copy is (q - zp) * scale in f32, rounded once to f16 (RNE)."""
    rng = np.random.default_rng(12)
    w = oracle.random_q4(rng, 192, 96)
    got = host(ctx.q4_to_f16(dev_q4(w)))
    want = oracle.dequant_q4(*w).astype(np.float16)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("m", [256, 2048])
def test_f16_weight_entry_points_equal_q4(ctx, oracle, m):
    """gemm_f16w / qkv_gemm_prep_f16w on the resident copies give the 4-bit entry points'
    outputs bit for bit (the same dequantised values, the same GEMM)."""
    import p2p_b200
    hq, hkv, k, pos0, cap = 32, 8, 2048, 3, m + 16
    rng = np.random.default_rng(m)
    mq, mk, mv, x, nw, rope, kc, vc = qkv_case(oracle, rng, hq, hkv, k, m, cap, True)
    mo = oracle.random_q4(rng, k, hq * D)
    prm = p2p_b200.Params(hq, hkv)
    wq, wk, wv, wo = dev_q4(mq), dev_q4(mk), dev_q4(mv), dev_q4(mo)
    g_x, g_nw, g_rope = dev(x), dev(nw), dev(rope)
    w16_qkv = torch.cat([ctx.q4_to_f16(w) for w in (wq, wk, wv)])
    w16_o = ctx.q4_to_f16(wo)
    outs = []
    for resident in (False, True):
        q = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
        kc_g, vc_g = dev(kc), dev(vc)
        y = torch.zeros((m, k), dtype=torch.float16, device="cuda")
        if resident:
            ctx.qkv_gemm_prep_f16w(prm, g_x, w16_qkv, g_nw, g_rope, q, kc_g, vc_g, pos0=pos0)
            ctx.gemm_f16w(w16_o, q, y)
        else:
            ctx.qkv_gemm_prep(prm, g_x, wq, wk, wv, g_nw, g_rope, q, kc_g, vc_g, pos0=pos0)
            ctx.gemm_q4(wo, q, y)
        ctx.sync()
        outs.append([host(t) for t in (q, kc_g, vc_g, y)])
    for a, b in zip(*outs):
        assert np.array_equal(bits(a), bits(b))
    assert np.isfinite(outs[1][3].astype(np.float32)).all()


def test_f16_weight_entry_points_refuse_bad_buffers(ctx, oracle):
    """Refusals on the host, before any launch: a k that is not a multiple of 8 (the weight
    rows would not start on 16-byte boundaries), a misaligned weight pointer and a misaligned
    f16 copy destination; the output is left untouched."""
    import ctypes as C
    import p2p_b200
    lib, bad = p2p_b200.lib, p2p_b200.P2P_ERR_INVALID_ARG
    rng = np.random.default_rng(5)
    x = torch.zeros((64, 2048), dtype=torch.float16, device="cuda")
    y = torch.ones((64, 256), dtype=torch.float16, device="cuda")
    w16 = torch.zeros((256 * 2048 + 8,), dtype=torch.float16, device="cuda")
    assert lib.p2p_gemm_f16w(ctx.h, w16.data_ptr(), 256, 2044, x.data_ptr(), 2048, 64,
                             y.data_ptr(), 256, 0, None) == bad
    assert lib.p2p_gemm_f16w(ctx.h, w16.data_ptr() + 2, 256, 2048, x.data_ptr(), 2048, 64,
                             y.data_ptr(), 256, 0, None) == bad
    mw = ctx.q4(dev_q4(oracle.random_q4(rng, 64, 256)))
    assert lib.p2p_q4_to_f16(ctx.h, C.byref(mw), w16.data_ptr() + 2, None) == bad
    ctx.sync()
    assert float(y.float().min()) == 1.0  # nothing ran
