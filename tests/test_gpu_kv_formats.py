"""The batched decode over the KV-cache formats beyond the engine's f16 rows
(p2p_attn_decode_kv): int8 caches with per-tensor / per-channel scales, paged caches with a
block table, and both together -- against the oracle, and paged against contiguous.

The int8 rule restates the reference bundle's GroupQueryAttention int8 cache
(public/kernels/megakernel.json): stored q = clamp(roundeven(x / scale), -128, 127), read
f32(q) * scale.  The paged layout is the bundle's PagedAttention one ([pages][block][Hkv][D]
plus a block table).
"""
import numpy as np
import pytest

from conftest import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 64


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


def scales(rng, per_channel):
    n = HKV * D if per_channel else 1
    ks = (0.02 + 0.04 * rng.random(n)).astype(np.float32)
    vs = (0.02 + 0.04 * rng.random(n)).astype(np.float32)
    return ks, vs


def problem(seed, past):
    rng = np.random.default_rng(seed)
    past = np.asarray(past, np.int32)
    nseq = len(past)
    offsets = np.zeros(nseq, np.int32)
    offsets[1:] = np.cumsum(past[:-1] + 1)
    rows = int(offsets[-1] + past[-1] + 1)
    kc = rng.standard_normal((rows, HKV, D)).astype(np.float16)
    vc = rng.standard_normal((rows, HKV, D)).astype(np.float16)
    qkv = rng.standard_normal((nseq, (HQ + 2 * HKV) * D)).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
    return rng, past, offsets, kc, vc, qkv, nw


def oracle_prep(oracle, past, offsets, kc, vc, qkv, nw, rope):
    """QK_PREP of every sequence's new token: rotated q rows and the caches with the new k/v."""
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = np.zeros((len(past), HQ * D), np.float16)
    for i in range(len(past)):
        sl = slice(int(offsets[i]), int(offsets[i]) + int(past[i]) + 1)
        kk, vv = kc_o[sl], vc_o[sl]
        qq = np.zeros((1, HQ * D), np.float16)
        oracle.qk_prep(HQ, HKV, D, qkv[i:i + 1], nw, rope, qq, kk, vv, int(past[i]), 1)
        kc_o[sl], vc_o[sl], q_o[i] = kk, vv, qq[0]
    return q_o, kc_o, vc_o


def fill_pages(pool_like, rows_per_seq, table, block):
    """A pool with the same page assignment as `table`, holding other rows (the V cache)."""
    pool = np.zeros_like(pool_like)
    for i, rows in enumerate(rows_per_seq):
        for b in range((len(rows) + block - 1) // block):
            chunk = rows[b * block:(b + 1) * block]
            pool[table[i, b], :len(chunk)] = chunk
    return pool


def to_pages(rows_per_seq, block, rng, n_spare=3):
    """A shuffled page pool holding each sequence's rows: (pages, block_table)."""
    nblk = [(len(r) + block - 1) // block for r in rows_per_seq]
    total = sum(nblk) + n_spare
    perm = rng.permutation(total).astype(np.int32)
    pool = np.zeros((total, block) + rows_per_seq[0].shape[1:], rows_per_seq[0].dtype)
    table = np.full((len(rows_per_seq), max(nblk) + 1), -1, np.int32)
    k = 0
    for i, r in enumerate(rows_per_seq):
        for b in range(nblk[i]):
            pg = perm[k]
            k += 1
            chunk = r[b * block:(b + 1) * block]
            pool[pg, :len(chunk)] = chunk
            table[i, b] = pg
    return pool, table


@pytest.mark.parametrize("per_channel", [False, True])
def test_quantize_equals_oracle(ctx, oracle, per_channel):
    rng = np.random.default_rng(3 + per_channel)
    x = (4 * rng.standard_normal((777, HKV, D))).astype(np.float16)
    x[0, 0, :6] = [0.5, -0.5, 1.5, -2.5, 1000, -1000]  # ties and clamps
    ks, _ = scales(rng, per_channel)
    ks[0] = 1.0
    got = host(ctx.kv_quantize_q8(dev(x), dev(ks)))
    assert np.array_equal(got, oracle.quantize_q8(x, ks))


@pytest.mark.parametrize("per_channel", [False, True])
@pytest.mark.parametrize("fused", [True, False])
def test_int8_decode_matches_oracle(ctx, oracle, per_channel, fused):
    past = [0, 1, 17, 64, 300, 1023, 1024, 1025, 2500, 5000, 7, 3333]
    rng, past, offsets, kc, vc, qkv, nw = problem(11 + 2 * fused + per_channel, past)
    rope = oracle.rope_table(int(past.max()) + 1)
    ks, vs = scales(rng, per_channel)
    q_o, kc_o, vc_o = oracle_prep(oracle, past, offsets, kc, vc, qkv, nw, rope)
    k8_o, v8_o = oracle.quantize_q8(kc_o, ks), oracle.quantize_q8(vc_o, vs)
    want = np.zeros((len(past), HQ * D), np.float16)
    oracle.attn_ragged_q8(HQ, HKV, D, q_o, k8_o, v8_o, ks, vs, offsets, past, want)
    import p2p_b200
    prm = p2p_b200.Params(HQ, HKV)
    out = torch.zeros((len(past), HQ * D), dtype=torch.float16, device="cuda")
    if fused:  # the int8 cache before the append, the new k/v quantised by the kernel
        k8, v8 = dev(oracle.quantize_q8(kc, ks)), dev(oracle.quantize_q8(vc, vs))
        ctx.attn_decode_kv(prm, dev(qkv), dev(nw), dev(rope), k8, v8, dev(past), out,
                           max_past=int(past.max()), offsets=dev(offsets), k_scale=dev(ks),
                           v_scale=dev(vs), fused_prep=True)
        ctx.sync()
        for i in range(len(past)):  # the appended rows equal the oracle's quantised QK_PREP
            r = int(offsets[i] + past[i])
            assert np.array_equal(host(k8[r]), k8_o[r]) and np.array_equal(host(v8[r]), v8_o[r])
    else:
        ctx.attn_decode_kv(prm, dev(q_o), None, None, dev(k8_o), dev(v8_o), dev(past), out,
                           max_past=int(past.max()), offsets=dev(offsets), k_scale=dev(ks),
                           v_scale=dev(vs), fused_prep=False)
        ctx.sync()
    assert_close(host(out), want, what=f"int8 decode (per_channel={per_channel})")


@pytest.mark.parametrize("block", [16, 64, 256])
@pytest.mark.parametrize("q8", [False, True])
def test_paged_decode_equals_contiguous_and_oracle(ctx, oracle, block, q8):
    past = [3, 100, 63, 64, 2049, 700, 15, 4000]
    rng, past, offsets, kc, vc, qkv, nw = problem(40 + block + q8, past)
    rope = oracle.rope_table(int(past.max()) + 1)
    ks, vs = scales(rng, True)
    if q8:
        kc, vc = oracle.quantize_q8(kc, ks), oracle.quantize_q8(vc, vs)
    seqs = [slice(int(offsets[i]), int(offsets[i]) + int(past[i]) + 1) for i in range(len(past))]
    kpool, table = to_pages([kc[s] for s in seqs], block, rng)
    vpool = fill_pages(kpool, [vc[s] for s in seqs], table, block)
    import p2p_b200
    prm = p2p_b200.Params(HQ, HKV)
    kw = dict(k_scale=dev(ks), v_scale=dev(vs)) if q8 else {}
    # contiguous and paged, fused, on copies of the same caches
    out_c = torch.zeros((len(past), HQ * D), dtype=torch.float16, device="cuda")
    kc_g, vc_g = dev(kc), dev(vc)
    ctx.attn_decode_kv(prm, dev(qkv), dev(nw), dev(rope), kc_g, vc_g, dev(past), out_c,
                       max_past=int(past.max()), offsets=dev(offsets), fused_prep=True, **kw)
    out_p = torch.zeros_like(out_c)
    kp_g, vp_g = dev(kpool), dev(vpool)
    ctx.attn_decode_kv(prm, dev(qkv), dev(nw), dev(rope), kp_g, vp_g, dev(past), out_p,
                       max_past=int(past.max()), block_table=dev(table), fused_prep=True, **kw)
    ctx.sync()
    assert torch.equal(out_p, out_c), "paged and contiguous differ"
    kp_h = host(kp_g)
    for i, s in enumerate(seqs):  # the new token's k row landed in its page
        r = int(past[i])
        assert np.array_equal(kp_h[table[i, r // block], r % block], host(kc_g[s.start + r]))
    # and against the oracle on the gathered rows (which must equal the contiguous cache)
    want = np.zeros((len(past), HQ * D), np.float16)
    kc_new, vc_new = host(kc_g), host(vc_g)
    q_rot = np.zeros((len(past), HQ * D), np.float16)
    k_scr = np.zeros((int(past.max()) + 1, HKV, D), np.float16)
    v_scr = np.zeros_like(k_scr)
    for i in range(len(past)):
        qq = np.zeros((1, HQ * D), np.float16)
        oracle.qk_prep(HQ, HKV, D, qkv[i:i + 1], nw, rope, qq, k_scr, v_scr, int(past[i]), 1)
        q_rot[i] = qq[0]
    gk = np.concatenate([oracle.gather_pages(kp_h, table[i], int(past[i]) + 1)
                         for i in range(len(past))])
    gv = np.concatenate([oracle.gather_pages(host(vp_g), table[i], int(past[i]) + 1)
                         for i in range(len(past))])
    assert np.array_equal(gk, kc_new) and np.array_equal(gv, vc_new)
    if q8:
        oracle.attn_ragged_q8(HQ, HKV, D, q_rot, gk, gv, ks, vs, offsets, past, want)
    else:
        oracle.attn_ragged(HQ, HKV, D, q_rot, gk, gv, offsets, past, want)
    assert_close(host(out_p), want, what=f"paged block {block} int8={q8}")


def test_paged_bad_block_table_entry_is_refused(ctx, oracle):
    """A block-table entry outside the page pool (or a sequence with more pages than its
    table row) is refused before any load; the other sequences are computed."""
    import p2p_b200
    past = [40, 300, 130, 90]
    rng, past, offsets, kc, vc, qkv, nw = problem(77, past)
    seqs = [slice(int(offsets[i]), int(offsets[i]) + int(past[i]) + 1) for i in range(len(past))]
    kpool, table = to_pages([kc[s] for s in seqs], 64, rng)
    vpool = fill_pages(kpool, [vc[s] for s in seqs], table, 64)
    rope = oracle.rope_table(int(past.max()) + 1)
    prm = p2p_b200.Params(HQ, HKV)
    good = torch.zeros((len(past), HQ * D), dtype=torch.float16, device="cuda")
    ctx.attn_decode_kv(prm, dev(qkv), dev(nw), dev(rope), dev(kpool), dev(vpool), dev(past),
                       good, max_past=int(past.max()), block_table=dev(table), fused_prep=True)
    ctx.sync()
    bad = table.copy()
    bad[1, 2] = kpool.shape[0]       # one page beyond the pool
    bad[3, 0] = -1                   # negative page
    out = torch.full_like(good, 7.0)
    kp = dev(kpool)
    ctx.attn_decode_kv(prm, dev(qkv), dev(nw), dev(rope), kp, dev(vpool), dev(past), out,
                       max_past=int(past.max()), block_table=dev(bad), fused_prep=True)
    with pytest.raises(p2p_b200.KvFullError):
        ctx.sync()
    got = host(out)
    assert (got[[1, 3]] == 7.0).all()
    assert np.array_equal(got[[0, 2]], host(good)[[0, 2]])
    # the refused sequences' pages were not written (their new-token rows keep the pool's)
    assert np.array_equal(host(kp)[table[1, 300 // 64], 300 % 64], kpool[table[1, 300 // 64], 300 % 64])
