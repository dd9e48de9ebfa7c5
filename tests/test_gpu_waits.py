"""Bounded device-side waits.  A wait that never completes ends after its 1 s limit: the
kernel writes no output for that work, p2p_sync reports P2P_ERR_TIMEOUT and the context stays
usable.  The wait is made to run out with a test hook (the waiting CTA expects 16 bytes more
than will ever arrive); nothing faults and no copy is left in flight."""
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


def expect_timeout(ctx, fn):
    import p2p_b200
    p2p_b200.lib.p2p_debug_set_wait_deficit(16)
    try:
        fn()
        with pytest.raises(p2p_b200.P2PError) as e:
            ctx.sync()
        assert e.value.status == p2p_b200.P2P_ERR_TIMEOUT
    finally:
        p2p_b200.lib.p2p_debug_set_wait_deficit(0)


def test_decode_combine_wait_times_out(ctx, oracle):
    """Decode step (cluster combine): the owners of every head give up, no output is written;
    the same step afterwards is correct."""
    import p2p_b200
    hq, hkv, past, cap = 32, 8, 3000, 4097
    rng = np.random.default_rng(77)
    qkv = rng.standard_normal((1, (hq + 2 * hkv) * D)).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
    kc = np.zeros((cap, hkv, D), np.float16)
    vc = np.zeros((cap, hkv, D), np.float16)
    kc[:past] = rng.standard_normal((past, hkv, D))
    vc[:past] = rng.standard_normal((past, hkv, D))
    rope = oracle.rope_table(cap)
    q_o = np.zeros((1, hq * D), np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    oracle.qk_prep(hq, hkv, D, qkv, nw, rope, q_o, kc_o, vc_o, past, 1)
    out_o = np.zeros((1, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q_o, kc_o, vc_o, out_o, past, 1)

    prm = p2p_b200.Params(hq, hkv)
    rope_g = dev(rope)
    layers = [(dev(qkv[0]), dev(nw), dev(kc), dev(vc),
               torch.full((hq * D,), 7.0, dtype=torch.float16, device="cuda"))
              for _ in range(6)]
    ctx.meta_write(past, 1)
    expect_timeout(ctx, lambda: ctx.decode_step(prm, layers, rope_g, cap, use_meta=True))
    for L in layers:
        assert bool((L[4] == 7.0).all())
    ctx.decode_step(prm, layers, rope_g, cap, use_meta=True)
    ctx.sync()
    for L in layers:
        assert_close(host(L[4])[None], out_o, what="decode after a timed-out launch")


def test_flash_q_wait_times_out(ctx, oracle):
    """Prefill (tcgen05 flash): the Q-tile wait gives up in every CTA, every role leaves its
    loop, TMEM is freed and no output row is written; the same call afterwards is correct."""
    import p2p_b200
    hq, hkv, m = 32, 8, 300
    rng = np.random.default_rng(78)
    q = rng.standard_normal((m, hq * D)).astype(np.float16)
    kc = rng.standard_normal((m, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((m, hkv, D)).astype(np.float16)
    want = np.zeros((m, hq * D), np.float16)
    oracle.attn(hq, hkv, D, q, kc, vc, want, 0, m)
    prm = p2p_b200.Params(hq, hkv)
    q_g, kc_g, vc_g = dev(q), dev(kc), dev(vc)
    out = torch.full((m, hq * D), 7.0, dtype=torch.float16, device="cuda")
    expect_timeout(ctx, lambda: ctx.attn(prm, q_g, kc_g, vc_g, out, pos0=0, m_tokens=m))
    assert bool((out == 7.0).all())
    ctx.attn(prm, q_g, kc_g, vc_g, out, pos0=0, m_tokens=m)
    ctx.sync()
    assert_close(host(out), want, what="flash after a timed-out launch")
