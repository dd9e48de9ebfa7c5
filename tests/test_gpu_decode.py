"""GPU parity of QK_PREP and the split-KV decode kernels against the oracle (C ABI calls).

QK_PREP outputs (rotated q, appended k/v cache rows) must be bit-identical to the oracle;
attention outputs must satisfy |x - r| <= 2e-3 + 1e-2 |r| on the same seeded inputs.
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
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16 if a.dtype == np.float16 else np.uint32)


def make_layer(rng, hq, hkv, past, cap, dtype=np.float16, norm=True):
    qkv = rng.standard_normal((1, (hq + 2 * hkv) * D)).astype(dtype)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(dtype) if norm else None
    kc = np.zeros((cap, hkv, D), dtype)
    vc = np.zeros((cap, hkv, D), dtype)
    kc[:past] = rng.standard_normal((past, hkv, D))
    vc[:past] = rng.standard_normal((past, hkv, D))
    return qkv, nw, kc, vc


def oracle_decode(oracle, hq, hkv, qkv, nw, rope, kc, vc, past):
    q = np.zeros((1, hq * D), qkv.dtype)
    kc, vc = kc.copy(), vc.copy()
    oracle.qk_prep(hq, hkv, D, qkv, nw, rope, q, kc, vc, past, 1)
    out = np.zeros((1, hq * D), qkv.dtype)
    oracle.attn(hq, hkv, D, q, kc, vc, out, past, 1)
    return q, kc, vc, out


@pytest.mark.parametrize("hq,hkv,pos0,m,norm", [(32, 8, 0, 5, True), (32, 8, 4000, 3, True),
                                                (16, 8, 77, 64, True), (32, 8, 9, 2, False),
                                                (12, 12, 3, 7, True),
                                                # whole prompt chunks (the token-tile kernel),
                                                # including the config's S = 2048 and a last
                                                # tile of 5 tokens
                                                (32, 8, 0, 2048, True), (32, 8, 0, 2048, False),
                                                (32, 8, 150, 333, True), (16, 8, 0, 8, True)])
def test_qk_prep_bit_exact(ctx, oracle, hq, hkv, pos0, m, norm):
    import p2p_b200
    rng = np.random.default_rng(hq * 1000 + pos0 + m)
    cap = pos0 + m
    qkv = rng.standard_normal((m, (hq + 2 * hkv) * D)).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16) if norm else None
    rope_np = oracle.rope_table(cap)
    kc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    q_o = np.zeros((m, hq * D), np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    oracle.qk_prep(hq, hkv, D, qkv, nw, rope_np, q_o, kc_o, vc_o, pos0, m)
    prm = p2p_b200.Params(hq, hkv)
    q_g = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    ctx.qk_prep(prm, dev(qkv), None if nw is None else dev(nw), dev(rope_np), q_g, kc_g, vc_g,
                pos0=pos0, m_tokens=m)
    assert np.array_equal(bits(host(q_g)), bits(q_o))
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))
    assert np.array_equal(bits(host(vc_g)), bits(vc_o))


@pytest.mark.parametrize("norm", [True, False])
def test_qk_prep_unaligned_rows_bit_exact(ctx, oracle, norm):
    """Row strides that are not a multiple of 16 bytes (qkv and q rows one element longer than
    their data) take the warp-per-row kernel instead of the thread-per-row one; same bits."""
    import p2p_b200
    hq, hkv, pos0, m = 32, 8, 21, 6
    rng = np.random.default_rng(4242 + norm)
    cap = pos0 + m
    w_in, w_q = (hq + 2 * hkv) * D, hq * D
    qkv = rng.standard_normal((m, w_in)).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16) if norm else None
    rope_np = oracle.rope_table(cap)
    kc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((cap, hkv, D)).astype(np.float16)
    q_o = np.zeros((m, w_q), np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    oracle.qk_prep(hq, hkv, D, qkv, nw, rope_np, q_o, kc_o, vc_o, pos0, m)
    qkv_pad = torch.zeros((m, w_in + 1), dtype=torch.float16, device="cuda")
    qkv_pad[:, :w_in] = dev(qkv)
    q_pad = torch.zeros((m, w_q + 1), dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    ctx.qk_prep(p2p_b200.Params(hq, hkv), qkv_pad[:, :w_in], None if nw is None else dev(nw),
                dev(rope_np), q_pad[:, :w_q], kc_g, vc_g, pos0=pos0, m_tokens=m)
    assert np.array_equal(bits(host(q_pad[:, :w_q].contiguous())), bits(q_o))
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))
    assert np.array_equal(bits(host(vc_g)), bits(vc_o))


@pytest.mark.parametrize("vocab,offset", [(65536, 0), (1001, 0), (65536, 1)])
def test_argmax_step_two_calls_match_oracle(ctx, oracle, vocab, offset):
    """p2p_argmax_step (kernels.js:362-399) twice in a row on the context's meta buffer: same
    tokens as the oracle (ties and NaNs included), out_tok filled at steps 7 and 8, position
    and step advanced on the device.  offset 1 makes the logits unaligned (element path)."""
    from p2p_b200.attention import _from_device_ptr
    rng = np.random.default_rng(vocab + offset)
    meta_o = np.array([300, 1, 7, 0], np.uint32)
    out_o = np.zeros(16, np.uint32)
    tok_o = np.zeros(1, np.uint32)
    ctx.meta_write(300, 1, 7)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_tok = torch.zeros(16, dtype=torch.int32, device="cuda")
    for call in range(2):
        lg = rng.standard_normal(vocab).astype(np.float16)
        lg[rng.integers(0, vocab, 3)] = lg.max()  # ties at the maximum
        lg[rng.integers(0, vocab, 3)] = np.nan
        buf = torch.zeros(vocab + offset, dtype=torch.float16, device="cuda")
        buf[offset:] = dev(lg)
        ctx.argmax_step(buf[offset:], tok, out_tok)
        ctx.sync()
        oracle.argmax(lg, tok_o, meta_o, out_o)
        assert int(host(tok)[0]) == int(tok_o[0])
    meta = _from_device_ptr(ctx.meta_ptr.value if hasattr(ctx.meta_ptr, "value") else ctx.meta_ptr,
                            16, 0).view(torch.int32)
    assert host(meta).astype(np.uint32).tolist() == meta_o.tolist() == [302, 1, 9, 0]
    assert np.array_equal(host(out_tok).astype(np.uint32), out_o)


def test_decode_loop_in_one_cuda_graph_advances_positions_on_device(ctx, oracle):
    """Three decode steps, each followed by p2p_argmax_step, captured in one CUDA graph and
    replayed once: every decode step reads its position from the meta buffer that the previous
    argmax advanced on the device (no host write between steps, as in the reference's
    multi-step decode), so the steps land at positions past, past+1, past+2."""
    import p2p_b200
    from p2p_b200.attention import _from_device_ptr
    hq, hkv, cap, past, n_steps, vocab = 32, 8, 600, 400, 3, 1024
    rope = oracle.rope_table(cap)
    prm = p2p_b200.Params(hq, hkv)
    rng = np.random.default_rng(2718)
    qkv, nw, kc, vc = make_layer(rng, hq, hkv, past, cap)
    steps = [rng.standard_normal((1, (hq + 2 * hkv) * D)).astype(np.float16)
             for _ in range(n_steps)]
    logits = [rng.standard_normal(vocab).astype(np.float16) for _ in range(n_steps)]
    rope_g, nw_g = dev(rope), dev(nw)
    kc_g, vc_g = dev(kc), dev(vc)
    q_rows = [dev(x[0]) for x in steps]
    outs = [torch.zeros((hq * D,), dtype=torch.float16, device="cuda") for _ in range(n_steps)]
    lg = [dev(x) for x in logits]
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_tok = torch.zeros(8, dtype=torch.int32, device="cuda")
    # first launches of each kernel outside the capture, on scratch buffers
    ctx.meta_write(past, 1, 0)
    scratch = (dev(steps[0][0]), nw_g, dev(kc), dev(vc), torch.zeros_like(outs[0]))
    ctx.decode_step(prm, [scratch], rope_g, cap, use_meta=True)
    ctx.argmax_step(lg[0], tok, out_tok)
    ctx.sync()
    ctx.meta_write(past, 1, 0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for s in range(n_steps):
            ctx.decode_step(prm, [(q_rows[s], nw_g, kc_g, vc_g, outs[s])], rope_g, cap,
                            use_meta=True)
            ctx.argmax_step(lg[s], tok, out_tok)
    g.replay()
    torch.cuda.synchronize()
    ctx.sync()
    kc_o, vc_o = kc.copy(), vc.copy()
    tok_o = np.zeros(1, np.uint32)
    meta_o = np.array([past, 1, 0, 0], np.uint32)
    out_o = np.zeros(8, np.uint32)
    for s in range(n_steps):
        _, kc_o, vc_o, want = oracle_decode(oracle, hq, hkv, steps[s], nw, rope, kc_o, vc_o,
                                            past + s)
        assert_close(host(outs[s])[None], want, what=f"graph step {s} at position {past + s}")
        oracle.argmax(logits[s], tok_o, meta_o, out_o)
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))
    assert np.array_equal(bits(host(vc_g)), bits(vc_o))
    assert np.array_equal(host(out_tok).astype(np.uint32), out_o)
    meta = _from_device_ptr(ctx.meta_ptr.value, 16, 0).view(torch.int32)
    assert host(meta).astype(np.uint32).tolist() == meta_o.tolist() == [past + 3, 1, 3, 0]
    del g


def test_argmax_step_full_token_buffer_is_reported(ctx):
    """The step index at out_tok's capacity: the token is not stored there, tok and the meta
    buffer still advance, and p2p_sync reports P2P_ERR_INVALID_ARG."""
    import p2p_b200
    ctx.meta_write(10, 1, 4)
    lg = torch.zeros(64, dtype=torch.float16, device="cuda")
    lg[9] = 1.0
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_tok = torch.full((4,), -1, dtype=torch.int32, device="cuda")
    ctx.argmax_step(lg, tok, out_tok)
    with pytest.raises(p2p_b200.P2PError) as e:
        ctx.sync()
    assert e.value.status == p2p_b200.P2P_ERR_INVALID_ARG
    assert int(host(tok)[0]) == 9 and host(out_tok).tolist() == [-1, -1, -1, -1]
    ctx.sync()  # the error bit was cleared by the previous sync


def test_library_rope_table_equals_oracle(ctx, oracle):
    import p2p_b200  # noqa: F401
    p = ctx.rope_table(40000, D, 1e6)
    from p2p_b200.attention import _from_device_ptr
    t = _from_device_ptr(p.value, 40000 * D * 2, 0).view(torch.float16).view(40000, D)
    assert np.array_equal(bits(host(t)), bits(oracle.rope_table(40000)))


def test_golden_decode_fixture(ctx, golden_dir):
    """The reference shaders' own output (16 q / 8 kv heads, position 130, 2 key chunks)."""
    import p2p_b200
    z = np.load(golden_dir / "decoder_decode_16x8.npz")
    pos0 = int(z["meta"][0])
    kc = np.concatenate([z["kc_in"], np.zeros((1, 8, D), np.float16)])
    vc = np.concatenate([z["vc_in"], np.zeros((1, 8, D), np.float16)])
    prm = p2p_b200.Params(16, 8, scale=0.125)
    # separate QK_PREP then ATTN (engine.js:213-222) through the meta buffer
    ctx.meta_write(pos0, 1)
    q = torch.zeros((1, 1024), dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    ctx.qk_prep(prm, dev(z["qkv"]), dev(z["nwb"]), dev(z["rope"]), q, kc_g, vc_g,
                m_tokens=1, use_meta=True)
    out = torch.zeros((1, 1024), dtype=torch.float16, device="cuda")
    ctx.attn(prm, q, kc_g, vc_g, out, m_tokens=1, use_meta=True)
    assert np.array_equal(bits(host(q)), bits(z["qout"]))
    assert np.array_equal(bits(host(kc_g)[pos0:]), bits(z["k_new"]))
    assert_close(host(out), z["out"], what="golden decode (separate ops)")
    # fused one-launch decode step
    kc_g, vc_g = dev(kc), dev(vc)
    out2 = torch.zeros((1024,), dtype=torch.float16, device="cuda")
    ctx.decode_step(prm, [(dev(z["qkv"][0]), dev(z["nwb"]), kc_g, vc_g, out2)], dev(z["rope"]),
                    kc.shape[0], pos=pos0)
    assert np.array_equal(bits(host(kc_g)[pos0:]), bits(z["k_new"]))
    assert np.array_equal(bits(host(vc_g)[pos0:]), bits(z["v_new"]))
    assert_close(host(out2)[None], z["out"], what="golden decode (fused)")


@pytest.mark.parametrize("past", [0, 1, 15, 16, 63, 64, 65, 127, 128, 1000, 4096, 20000])
def test_decode_positions(ctx, oracle, past):
    import p2p_b200
    hq, hkv = 32, 8
    rng = np.random.default_rng(past + 11)
    qkv, nw, kc, vc = make_layer(rng, hq, hkv, past, past + 1)
    rope = oracle.rope_table(past + 1)
    q_o, kc_o, vc_o, out_o = oracle_decode(oracle, hq, hkv, qkv, nw, rope, kc, vc, past)
    prm = p2p_b200.Params(hq, hkv)
    kc_g, vc_g = dev(kc), dev(vc)
    out = torch.zeros((hq * D,), dtype=torch.float16, device="cuda")
    ctx.decode_step(prm, [(dev(qkv[0]), dev(nw), kc_g, vc_g, out)], dev(rope), past + 1, pos=past)
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))
    assert np.array_equal(bits(host(vc_g)), bits(vc_o))
    assert_close(host(out)[None], out_o, what=f"fused decode past={past}")
    # unfused ATTN on the oracle's rotated q and cache
    out3 = torch.zeros((1, hq * D), dtype=torch.float16, device="cuda")
    ctx.attn(prm, dev(q_o), dev(kc_o), dev(vc_o), out3, pos0=past, m_tokens=1)
    assert_close(host(out3), out_o, what=f"attn M=1 past={past}")


@pytest.mark.parametrize("hq,hkv", [(16, 8), (8, 8), (64, 8), (32, 4)])
def test_decode_group_sizes(ctx, oracle, hq, hkv):
    import p2p_b200
    past = 777
    rng = np.random.default_rng(hq + hkv)
    qkv, nw, kc, vc = make_layer(rng, hq, hkv, past, past + 1)
    rope = oracle.rope_table(past + 1)
    _, kc_o, _, out_o = oracle_decode(oracle, hq, hkv, qkv, nw, rope, kc, vc, past)
    kc_g, vc_g = dev(kc), dev(vc)
    out = torch.zeros((hq * D,), dtype=torch.float16, device="cuda")
    ctx.decode_step(p2p_b200.Params(hq, hkv), [(dev(qkv[0]), dev(nw), kc_g, vc_g, out)],
                    dev(rope), past + 1, pos=past)
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))
    assert_close(host(out)[None], out_o, what=f"G={hq // hkv}")


def test_decode_step_six_layers_ctx4096(ctx, oracle):
    """LFM2.5-1.2B decode: 32 q / 8 kv heads, 4096 past tokens + 1 new, 6 independent layers,
    all in one launch; position from the device meta buffer."""
    import p2p_b200
    hq, hkv, past, n_layers = 32, 8, 4096, 6
    cap = past + 1
    rope = oracle.rope_table(cap)
    rope_g = dev(rope)
    prm = p2p_b200.Params(hq, hkv)
    layers, want = [], []
    for l in range(n_layers):
        rng = np.random.default_rng(1000 + l)
        qkv, nw, kc, vc = make_layer(rng, hq, hkv, past, cap)
        _, kc_o, vc_o, out_o = oracle_decode(oracle, hq, hkv, qkv, nw, rope, kc, vc, past)
        out = torch.zeros((hq * D,), dtype=torch.float16, device="cuda")
        layers.append((dev(qkv[0]), dev(nw), dev(kc), dev(vc), out))
        want.append((kc_o, vc_o, out_o))
    ctx.meta_write(past, 1)
    ctx.decode_step(prm, layers, rope_g, cap, use_meta=True)
    for l in range(n_layers):
        kc_o, vc_o, out_o = want[l]
        assert np.array_equal(bits(host(layers[l][2])[past]), bits(kc_o[past]))
        assert np.array_equal(bits(host(layers[l][3])[past]), bits(vc_o[past]))
        assert_close(host(layers[l][4])[None], out_o, what=f"layer {l}")


@pytest.mark.parametrize("hq,past", [(32, 0), (32, 5), (32, 100), (32, 3000), (64, 37)])
def test_decode_step_device_position_in_large_cache(ctx, oracle, hq, past):
    """Device-side position well inside a 4097-row cache: the split count follows the cache
    size, so most splits of a (layer, head) get an empty key range and must contribute
    nothing to the combine."""
    import p2p_b200
    hkv, cap, n_layers = 8, 4097, 2
    rope = oracle.rope_table(cap)
    prm = p2p_b200.Params(hq, hkv)
    layers, want = [], []
    for l in range(n_layers):
        rng = np.random.default_rng(7000 + 10 * past + l)
        qkv, nw, kc, vc = make_layer(rng, hq, hkv, past, cap)
        _, kc_o, vc_o, out_o = oracle_decode(oracle, hq, hkv, qkv, nw, rope, kc, vc, past)
        out = torch.zeros((hq * D,), dtype=torch.float16, device="cuda")
        layers.append((dev(qkv[0]), dev(nw), dev(kc), dev(vc), out))
        want.append((kc_o, vc_o, out_o))
    ctx.meta_write(past, 1)
    ctx.decode_step(prm, layers, dev(rope), cap, use_meta=True)
    for l in range(n_layers):
        kc_o, vc_o, out_o = want[l]
        assert np.array_equal(bits(host(layers[l][2])), bits(kc_o))
        assert np.array_equal(bits(host(layers[l][3])), bits(vc_o))
        assert_close(host(layers[l][4])[None], out_o, what=f"layer {l} past {past}")


def test_decode_step_host_rows(ctx, oracle):
    """qkv and out rows in page-locked host memory: the decode kernel reads the inputs and
    writes the outputs across the host link itself; two steps with different inputs and
    positions both match the oracle, and the caches get the new rows."""
    import p2p_b200
    hq, hkv, cap, n_layers = 32, 8, 700, 3
    rope = oracle.rope_table(cap)
    prm = p2p_b200.Params(hq, hkv)
    rng = np.random.default_rng(4242)
    row = (hq + 2 * hkv) * D
    kcs = [rng.standard_normal((cap, hkv, D)).astype(np.float16) for _ in range(n_layers)]
    vcs = [rng.standard_normal((cap, hkv, D)).astype(np.float16) for _ in range(n_layers)]
    nws = [(1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16) for _ in range(n_layers)]
    h_in = torch.zeros((n_layers, row), dtype=torch.float16).pin_memory()
    h_out = torch.zeros((n_layers, hq * D), dtype=torch.float16).pin_memory()
    layers = [(h_in[l], dev(nws[l]), dev(kcs[l]), dev(vcs[l]), h_out[l]) for l in range(n_layers)]
    plan = ctx.plan_decode_step(prm, layers, dev(rope), cap, use_meta=True)
    stream = torch.cuda.current_stream()
    for past in (500, 501):
        qkv = rng.standard_normal((n_layers, row)).astype(np.float16)
        h_in.copy_(torch.from_numpy(qkv))
        ctx.meta_write(past, 1, stream=stream)
        plan.run(stream)
        stream.synchronize()
        ctx.sync()
        for l in range(n_layers):
            _, kc_o, vc_o, out_o = oracle_decode(oracle, hq, hkv, qkv[l:l + 1], nws[l], rope,
                                                 kcs[l], vcs[l], past)
            kcs[l], vcs[l] = kc_o, vc_o  # the next step sees this step's k/v rows
            assert np.array_equal(bits(host(layers[l][2])[past]), bits(kc_o[past]))
            assert_close(h_out[l].numpy()[None], out_o, what=f"host rows layer {l} past {past}")


def test_decode_fp32_storage(ctx, oracle):
    """The fp32 case: past 512 + 1 new, RoPE theta 1e6 on positions 0..512, no q/k norm."""
    import p2p_b200
    hq, hkv, past = 32, 8, 512
    rng = np.random.default_rng(512)
    qkv, _, kc, vc = make_layer(rng, hq, hkv, past, past + 1, dtype=np.float32, norm=False)
    rope = oracle.rope_table(past + 1, D, 1e6, f32=True)
    _, kc_o, _, out_o = oracle_decode(oracle, hq, hkv, qkv, None, rope, kc, vc, past)
    prm = p2p_b200.Params(hq, hkv, dtype=torch.float32)
    kc_g, vc_g = dev(kc), dev(vc)
    out = torch.zeros((hq * D,), dtype=torch.float32, device="cuda")
    ctx.decode_step(prm, [(dev(qkv[0]), None, kc_g, vc_g, out)], dev(rope), past + 1, pos=past)
    assert np.array_equal(bits(host(kc_g)), bits(kc_o))
    np.testing.assert_allclose(host(out)[None], out_o, atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("fused", [True, False])
def test_ragged_decode(ctx, oracle, fused):
    import p2p_b200
    hq, hkv = 32, 8
    rng = np.random.default_rng(7 + fused)
    past = np.array([0, 1, 17, 64, 300, 1023, 1024, 1025, 2500, 5000, 7, 3333], np.int32)
    nseq = len(past)
    offsets = np.zeros(nseq, np.int32)
    offsets[1:] = np.cumsum(past[:-1] + 1 + 3)  # 3 spare rows between sequences
    rows = int(offsets[-1] + past[-1] + 1)
    kc = rng.standard_normal((rows, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((rows, hkv, D)).astype(np.float16)
    rope = oracle.rope_table(int(past.max()) + 1)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
    qkv = rng.standard_normal((nseq, (hq + 2 * hkv) * D)).astype(np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = np.zeros((nseq, hq * D), np.float16)
    for i in range(nseq):
        o = offsets[i]
        sl = slice(o, o + past[i] + 1)
        kk, vv = kc_o[sl], vc_o[sl]
        qq = np.zeros((1, hq * D), np.float16)
        oracle.qk_prep(hq, hkv, D, qkv[i:i + 1], nw, rope, qq, kk, vv, int(past[i]), 1)
        kc_o[sl], vc_o[sl], q_o[i] = kk, vv, qq[0]
    out_o = np.zeros((nseq, hq * D), np.float16)
    oracle.attn_ragged(hq, hkv, D, q_o, kc_o, vc_o, offsets.astype(np.int64), past, out_o)
    prm = p2p_b200.Params(hq, hkv)
    out = torch.zeros((nseq, hq * D), dtype=torch.float16, device="cuda")
    if fused:
        kc_g, vc_g = dev(kc), dev(vc)
        ctx.attn_decode_ragged(prm, dev(qkv), dev(nw), dev(rope), kc_g, vc_g, dev(offsets),
                               dev(past), out, max_past=int(past.max()), fused_prep=True)
        assert np.array_equal(bits(host(kc_g)), bits(kc_o))
        assert np.array_equal(bits(host(vc_g)), bits(vc_o))
    else:
        ctx.attn_decode_ragged(prm, dev(q_o), None, None, dev(kc_o), dev(vc_o), dev(offsets),
                               dev(past), out, max_past=int(past.max()), fused_prep=False)
    assert_close(host(out), out_o, what="ragged")


@pytest.mark.parametrize("fused", [True, False])
def test_ragged_entries_outside_the_cache_are_refused(ctx, oracle, fused):
    """Ragged sequences whose rows would leave the cache (offsets[i] + past[i] >= kv_rows), or
    with a negative entry, or with past[i] > max_past, are skipped on the device before any
    load: their output rows keep what they held, sync() reports KV_FULL, and every other
    sequence still matches the oracle."""
    import p2p_b200
    hq, hkv = 32, 8
    rng = np.random.default_rng(31 + fused)
    past = np.array([40, 700, 5, 2000, 90, 64, 300, 1500], np.int32)
    nseq = len(past)
    offsets = np.zeros(nseq, np.int32)
    offsets[1:] = np.cumsum(past[:-1] + 1)
    rows = int(offsets[-1] + past[-1] + 1)
    max_past = int(past.max())
    kc = rng.standard_normal((rows, hkv, D)).astype(np.float16)
    vc = rng.standard_normal((rows, hkv, D)).astype(np.float16)
    rope = oracle.rope_table(max_past + 1)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
    qkv = rng.standard_normal((nseq, (hq + 2 * hkv) * D)).astype(np.float16)
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = np.zeros((nseq, hq * D), np.float16)
    for i in range(nseq):
        sl = slice(offsets[i], offsets[i] + past[i] + 1)
        kk, vv = kc_o[sl], vc_o[sl]
        qq = np.zeros((1, hq * D), np.float16)
        oracle.qk_prep(hq, hkv, D, qkv[i:i + 1], nw, rope, qq, kk, vv, int(past[i]), 1)
        kc_o[sl], vc_o[sl], q_o[i] = kk, vv, qq[0]
    out_o = np.zeros((nseq, hq * D), np.float16)
    oracle.attn_ragged(hq, hkv, D, q_o, kc_o, vc_o, offsets.astype(np.int64), past, out_o)
    bad_off, bad_past = offsets.copy(), past.copy()
    bad_past[7] = rows - offsets[7]          # one row past the end of the cache
    bad_past[2] = -1                         # negative length
    bad_off[4] = -3                          # negative offset
    bad_past[5] = max_past + 1               # longer than the host-declared bound
    refused = [2, 4, 5, 7]
    prm = p2p_b200.Params(hq, hkv)
    out = torch.full((nseq, hq * D), 7.0, dtype=torch.float16, device="cuda")
    kc_g = dev(kc if fused else kc_o)
    vc_g = dev(vc if fused else vc_o)
    ctx.attn_decode_ragged(prm, dev(qkv if fused else q_o), dev(nw) if fused else None,
                           dev(rope) if fused else None, kc_g, vc_g, dev(bad_off),
                           dev(bad_past), out, max_past=max_past, fused_prep=fused)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.sync()
    got = host(out)
    ok = [i for i in range(nseq) if i not in refused]
    assert (got[refused] == 7.0).all()
    assert_close(got[ok], out_o[ok], what="sequences beside the refused ones")
    if fused:  # the refused sequences' cache rows were not written either
        for i in refused:
            sl = slice(offsets[i], offsets[i] + past[i] + 1)
            assert np.array_equal(bits(host(kc_g[sl])), bits(kc[sl]))
    # the context stays usable: a valid call afterwards syncs clean
    ctx.attn_decode_ragged(prm, dev(q_o), None, None, dev(kc_o), dev(vc_o), dev(offsets),
                           dev(past), out, max_past=max_past, fused_prep=False)
    ctx.sync()
    assert_close(host(out), out_o, what="after the refusal")


def test_repeated_calls_reuse_counters(ctx, oracle):
    """The split counters reset themselves: many back-to-back launches stay correct."""
    import p2p_b200
    hq, hkv, past = 32, 8, 3000
    rng = np.random.default_rng(99)
    qkv, nw, kc, vc = make_layer(rng, hq, hkv, past, past + 1)
    rope = oracle.rope_table(past + 1)
    _, _, _, out_o = oracle_decode(oracle, hq, hkv, qkv, nw, rope, kc, vc, past)
    kc_g, vc_g, rg, qg, ng = dev(kc), dev(vc), dev(rope), dev(qkv[0]), dev(nw)
    out = torch.zeros((hq * D,), dtype=torch.float16, device="cuda")
    for _ in range(50):
        ctx.decode_step(p2p_b200.Params(hq, hkv), [(qg, ng, kc_g, vc_g, out)], rg, past + 1,
                        pos=past)
    assert_close(host(out)[None], out_o, what="after 50 launches")


def test_errors_are_statuses(ctx):
    import p2p_b200
    prm = p2p_b200.Params(32, 8, head_dim=128)
    x = torch.zeros(16, dtype=torch.float16, device="cuda")
    with pytest.raises(p2p_b200.P2PError) as e:
        ctx.attn(prm, x.view(1, 16), x.view(1, 1, 16), x.view(1, 1, 16), x.view(1, 16))
    assert e.value.status == 7  # UNSUPPORTED
    with pytest.raises(p2p_b200.P2PError) as e:
        ctx.attn(p2p_b200.Params(30, 8), x.view(1, 16), x.view(1, 1, 16), x.view(1, 1, 16),
                 x.view(1, 16))
    assert e.value.status == 1
    # host-known position beyond the cache -> KV_FULL
    kc = torch.zeros((4, 8, D), dtype=torch.float16, device="cuda")
    q = torch.zeros((1, 32 * D), dtype=torch.float16, device="cuda")
    with pytest.raises(p2p_b200.KvFullError):
        ctx.attn(p2p_b200.Params(32, 8), q, kc, kc, q, pos0=4, m_tokens=1)


def test_kv_cache_growth_and_kv_full(ctx, oracle):
    import p2p_b200
    prm = p2p_b200.Params(16, 8)
    eng = p2p_b200.LfmAttention(ctx, prm, n_layers=2, max_ctx=600, kv_init_bytes=2 * 2 * 8 * 64
                                * 2 * 100, kv_grow_bytes=2 * 2 * 8 * 64 * 2 * 64)
    assert eng.kv.capacity == 100
    k0 = eng.kv.k(1)
    k0.copy_(torch.randn_like(k0))
    before = host(k0).copy()
    assert eng.ensure_capacity(250)
    assert eng.kv.capacity == 292  # 100 + 3 * 64
    assert np.array_equal(bits(host(eng.kv.k(1))[:100]), bits(before))
    assert not eng.ensure_capacity(601)  # beyond max_ctx -> 'kv_full'
    assert eng.ensure_capacity(600) and eng.kv.capacity == 600
    # allocation failure keeps the old cache and reports failure
    p2p_b200.lib.p2p_debug_set_alloc_limit(0)
    try:
        eng2 = p2p_b200.LfmAttention.__new__(p2p_b200.LfmAttention)
        with pytest.raises(p2p_b200.OomError):
            p2p_b200.KVCache(ctx, 1, 8, 10)
        del eng2
    finally:
        p2p_b200.lib.p2p_debug_set_alloc_limit(-1)


def test_device_position_beyond_cache_is_refused(ctx):
    """A meta position the cache cannot hold: the kernel touches nothing and p2p_sync reports
    P2P_ERR_KV_FULL (the reference's 'kv_full'), leaving the context usable."""
    import p2p_b200
    hq, hkv, cap = 32, 8, 64
    prm = p2p_b200.Params(hq, hkv)
    kc = torch.zeros((cap, hkv, D), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    qkv = torch.ones(((hq + 2 * hkv) * D,), dtype=torch.float16, device="cuda")
    out = torch.full((hq * D,), 7.0, dtype=torch.float16, device="cuda")
    rope = ctx.rope_table(cap + 8)
    ctx.meta_write(cap, 1)
    ctx.decode_step(prm, [(qkv, None, kc, vc, out)], rope, cap, use_meta=True)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.sync()
    assert float(kc.abs().sum()) == 0 and float(out[0]) == 7.0
    ctx.meta_write(cap - 1, 1)
    ctx.decode_step(prm, [(qkv, None, kc, vc, out)], rope, cap, use_meta=True)
    ctx.sync()


def test_ragged_decode_full_scale_sampled(ctx, oracle):
    """The 256-sequence ragged workload at full size (past ~ U[1024, 32768], ~9 GB of KV):
    run on the GPU, then check a sample of sequences (shortest, longest, a few others)
    against the oracle on their downloaded cache slices."""
    import p2p_b200
    hq, hkv = 32, 8
    rng = np.random.default_rng(4)
    past = rng.integers(1024, 32769, 256).astype(np.int32)
    offsets = np.zeros(256, np.int64)
    offsets[1:] = np.cumsum(past[:-1].astype(np.int64) + 1)
    rows = int(offsets[-1] + past[-1] + 1)
    g = torch.Generator(device="cuda").manual_seed(5)
    kc = torch.randn((rows, hkv, D), generator=g, device="cuda", dtype=torch.float16)
    vc = torch.randn((rows, hkv, D), generator=g, device="cuda", dtype=torch.float16)
    qkv = torch.randn((256, (hq + 2 * hkv) * D), generator=g, device="cuda", dtype=torch.float16)
    nw = (1 + 0.1 * torch.randn((2 * D,), generator=g, device="cuda")).half()
    rope = oracle.rope_table(int(past.max()) + 1)
    sample = sorted({int(np.argmin(past)), int(np.argmax(past)), 0, 77, 128, 255})
    before = {i: (host(kc[offsets[i]:offsets[i] + past[i] + 1]).copy(),
                  host(vc[offsets[i]:offsets[i] + past[i] + 1]).copy()) for i in sample}
    out = torch.zeros((256, hq * D), dtype=torch.float16, device="cuda")
    ctx.attn_decode_ragged(p2p_b200.Params(hq, hkv), qkv, nw, dev(rope), kc, vc,
                           dev(offsets.astype(np.int32)), dev(past), out,
                           max_past=int(past.max()), fused_prep=True)
    got = host(out)
    qkv_h, nw_h = host(qkv), host(nw)
    for i in sample:
        k_i, v_i = before[i]
        q_o = np.zeros((1, hq * D), np.float16)
        oracle.qk_prep(hq, hkv, D, qkv_h[i:i + 1], nw_h, rope, q_o, k_i, v_i, int(past[i]), 1)
        want = np.zeros((1, hq * D), np.float16)
        oracle.attn(hq, hkv, D, q_o, k_i, v_i, want, int(past[i]), 1)
        assert np.array_equal(bits(host(kc[offsets[i] + past[i]])), bits(k_i[past[i]]))
        assert_close(got[i:i + 1], want, what=f"ragged seq {i} (past {past[i]})")
    del kc, vc
    torch.cuda.empty_cache()
