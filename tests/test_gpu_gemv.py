"""The 4-bit projections around the attention path on the GPU (gemv_q4.cu) against the oracle's
restatement of the GEMV shader (kernels.js:22-68), which the CPU tests pin bit for bit to the
reference's own shader:

  * p2p_gemv_q4 (the o_proj consumer, engine.js:224) -- bit-identical;
  * p2p_qkv_gemv_prep (q/k/v projections with QK_PREP in the epilogue, engine.js:202-204 then
    kernels.js:216-266) -- rotated q and the appended cache rows bit-identical to the oracle's
    three GEMVs followed by its QK_PREP;
  * one attention layer of a decode step (projection + prep, attention, o_proj) captured in a
    CUDA graph with the position read from the meta buffer.
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
    """A 4-bit matrix on the device; the u32 words travel as int32 tensors (same bytes)."""
    wq, sc, zp = m
    return dev(wq.view(np.int32)), dev(sc), dev(zp.view(np.int32))


@pytest.mark.parametrize("k,n", [(1024, 1024), (2048, 2048), (96, 40), (4608, 16), (2048, 3072)])
def test_gemv_bit_exact(ctx, oracle, k, n):
    rng = np.random.default_rng(k + n)
    m = oracle.random_q4(rng, n, k)
    x = (2 * rng.standard_normal(k)).astype(np.float16)
    want = oracle.gemv_q4(x, *m, y=np.zeros(n + 7, np.float16), y_off=7)
    y = torch.zeros(n + 7, dtype=torch.float16, device="cuda")
    ctx.gemv_q4(dev_q4(m), dev(x), y, y_off=7)
    ctx.sync()
    assert np.array_equal(bits(host(y)), bits(want))


def test_gemv_golden_fixture(ctx, golden_dir):
    z = np.load(golden_dir / "gemv_q4_k1024_n96.npz")
    y = torch.zeros(96, dtype=torch.float16, device="cuda")
    ctx.gemv_q4(dev_q4((z["wq"], z["sc"], z["zp"])), dev(z["x"]), y)
    ctx.sync()
    assert np.array_equal(bits(host(y)), bits(z["y"]))


def oracle_qkv_prep(oracle, hq, hkv, k, x, mq, mk, mv, nw, rope, kc, vc, pos):
    """The reference's order: three GEMVs into one qkv row, then QK_PREP."""
    row = np.zeros((1, (hq + 2 * hkv) * D), np.float16)
    oracle.gemv_q4(x, *mq, y=row[0], y_off=0)
    oracle.gemv_q4(x, *mk, y=row[0], y_off=hq * D)
    oracle.gemv_q4(x, *mv, y=row[0], y_off=(hq + hkv) * D)
    q = np.zeros((1, hq * D), np.float16)
    oracle.qk_prep(hq, hkv, D, row, nw, rope, q, kc, vc, pos, 1)
    return q


@pytest.mark.parametrize("hq,hkv,k,norm,use_meta", [(16, 8, 1024, True, False),
                                                    (32, 8, 2048, True, True),
                                                    (32, 8, 2048, False, False),
                                                    (12, 12, 768, True, True)])
def test_qkv_gemv_prep_bit_exact(ctx, oracle, hq, hkv, k, norm, use_meta):
    import p2p_b200
    rng = np.random.default_rng(hq * 7 + k)
    mq, mk, mv = (oracle.random_q4(rng, h * D, k) for h in (hq, hkv, hkv))
    x = rng.standard_normal(k).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16) if norm else None
    pos, cap = 777, 1000
    rope = oracle.rope_table(cap)
    kc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = oracle_qkv_prep(oracle, hq, hkv, k, x, mq, mk, mv, nw, rope, kc_o, vc_o, pos)
    q = torch.zeros(hq * D, dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    if use_meta:
        ctx.meta_write(pos, 1, 0)
    ctx.qkv_gemv_prep(p2p_b200.Params(hq, hkv), dev(x), dev_q4(mq), dev_q4(mk), dev_q4(mv),
                      dev(nw) if norm else None, dev(rope), q, kc_g, vc_g,
                      pos=0 if use_meta else pos, use_meta=use_meta)
    ctx.sync()
    assert np.array_equal(bits(host(q)), bits(q_o[0]))
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))  # only row pos changed, bit-exact
    assert np.array_equal(bits(host(vc_g)), bits(vc_o))


def test_qkv_gemv_prep_position_beyond_cache_is_refused(ctx, oracle):
    import p2p_b200
    rng = np.random.default_rng(5)
    hq, hkv, k, cap = 32, 8, 2048, 64
    mq, mk, mv = (oracle.random_q4(rng, h * D, k) for h in (hq, hkv, hkv))
    q = torch.full((hq * D,), 3.0, dtype=torch.float16, device="cuda")
    kc = torch.zeros((cap, hkv, D), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    rope = dev(oracle.rope_table(cap))
    prm = p2p_b200.Params(hq, hkv)
    x = dev(rng.standard_normal(k).astype(np.float16))
    with pytest.raises(p2p_b200.KvFullError):  # host-known position: refused on the host
        ctx.qkv_gemv_prep(prm, x, dev_q4(mq), dev_q4(mk), dev_q4(mv), None, rope, q, kc, vc,
                          pos=cap)
    ctx.meta_write(cap, 1, 0)  # device position: the kernel refuses and writes nothing
    ctx.qkv_gemv_prep(prm, x, dev_q4(mq), dev_q4(mk), dev_q4(mv), None, rope, q, kc, vc,
                      use_meta=True)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.sync()
    assert float(q.float().min()) == 3.0 and float(kc.abs().sum()) == 0


def test_attention_layer_in_one_graph(ctx, oracle):
    """One LFM2.5-1.2B attention layer of a decode step: qkv projection + QK_PREP, attention
    at M = 1 and the o_proj consumer, captured in one CUDA graph reading the position from the
    meta buffer; replayed at two positions."""
    import p2p_b200
    hq, hkv, k, cap = 32, 8, 2048, 3000
    rng = np.random.default_rng(17)
    mq, mk, mv = (oracle.random_q4(rng, h * D, k) for h in (hq, hkv, hkv))
    mo = oracle.random_q4(rng, k, hq * D)
    x = rng.standard_normal(k).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
    rope = oracle.rope_table(cap)
    kc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    prm = p2p_b200.Params(hq, hkv)
    g_x, g_nw, g_rope = dev(x), dev(nw), dev(rope)
    g_q = torch.zeros(hq * D, dtype=torch.float16, device="cuda")
    g_att = torch.zeros(hq * D, dtype=torch.float16, device="cuda")
    g_y = torch.zeros(k, dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    wq, wk, wv, wo = dev_q4(mq), dev_q4(mk), dev_q4(mv), dev_q4(mo)

    def layer():
        ctx.qkv_gemv_prep(prm, g_x, wq, wk, wv, g_nw, g_rope, g_q, kc_g, vc_g, use_meta=True)
        ctx.attn(prm, g_q[None], kc_g, vc_g, g_att[None], m_tokens=1, use_meta=True)
        ctx.gemv_q4(wo, g_att, g_y)

    ctx.meta_write(100, 1, 0)
    layer()  # warm-up (workspace, kernel configuration) before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer()
    for pos in (1500, 2999):
        ctx.meta_write(pos, 1, 0)
        graph.replay()
        ctx.sync()
        kc_o, vc_o = host(kc_g).copy(), host(vc_g).copy()
        q_o = oracle_qkv_prep(oracle, hq, hkv, k, x, mq, mk, mv, nw, rope, kc_o, vc_o, pos)
        assert np.array_equal(bits(host(g_q)), bits(q_o[0]))
        att_o = np.zeros((1, hq * D), np.float16)
        oracle.attn(hq, hkv, D, q_o, kc_o, vc_o, att_o, pos, 1)
        assert_close(host(g_att)[None], att_o, what=f"attention at {pos}")
        # o_proj of the GPU's attention row: bit-exact against the GEMV shader's restatement
        assert np.array_equal(bits(host(g_y)), bits(oracle.gemv_q4(host(g_att), *mo)))
    del graph
