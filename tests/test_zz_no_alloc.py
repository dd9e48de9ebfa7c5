"""The decode entry point that allocates nothing (p2p_attn_decode_ragged_noalloc).

Callers that cannot allocate device memory while serving (a process that gave its free HBM
to its own pool at start-up, or a host whose device memory belongs to another component) use
this variant: its split scratch is a fixed array inside the library, placed on the device when
the context is created.  These tests call it through the C ABI and compare it with
p2p_attn_decode_ragged, the allocating entry point, on two calls in a row, with the library's
own allocations forbidden during the calls, in both split regimes and close to the scratch
limit.  This file is collected last so that a failure here leaves every other test already run.
"""
import numpy as np
import pytest

from conftest import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 64
SCRATCH_BYTES = 32 << 20  # P2P_NOALLOC_SCRATCH_BYTES


def _problem(rng, past):
    past = np.asarray(past, np.int32)
    offsets = np.zeros(len(past), np.int32)
    offsets[1:] = np.cumsum(past[:-1] + 1)
    rows = int(offsets[-1] + past[-1] + 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    g = torch.Generator(device="cuda").manual_seed(int(rng.integers(1 << 30)))
    kc = torch.randn((rows, HKV, D), generator=g, device="cuda", dtype=torch.float16)
    vc = torch.randn((rows, HKV, D), generator=g, device="cuda", dtype=torch.float16)
    qkv = t(rng.standard_normal((len(past), (HQ + 2 * HKV) * D)).astype(np.float16))
    nw = t((1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16))
    return past, offsets, t(offsets), t(past), kc, vc, qkv, nw


def _check_against_oracle(oracle, seqs, past, offsets, kc_before, vc_before, qkv, nw, rope_h,
                          got, what):
    """Sequences `seqs` of a fused call against the oracle's QK_PREP + ATTN on their rows."""
    qkv_h = qkv.cpu().numpy()
    nw_h = nw.cpu().numpy()
    for i in seqs:
        sl = slice(int(offsets[i]), int(offsets[i]) + int(past[i]) + 1)
        k_i = kc_before[sl].cpu().numpy().copy()
        v_i = vc_before[sl].cpu().numpy().copy()
        q_o = np.zeros((1, HQ * D), np.float16)
        oracle.qk_prep(HQ, HKV, D, qkv_h[i:i + 1], nw_h, rope_h, q_o, k_i, v_i, int(past[i]), 1)
        want = np.zeros((1, HQ * D), np.float16)
        oracle.attn(HQ, HKV, D, q_o, k_i, v_i, want, int(past[i]), 1)
        assert_close(got[i:i + 1], want, what=f"{what}: seq {i} (past {past[i]}) vs oracle")


def _run_twice(ctx, oracle, past_list, seed, check_seqs):
    """Allocating call, then two no-alloc calls with library allocations forbidden, fused and
    unfused, all compared; a sample of sequences is also compared with the oracle."""
    import p2p_b200
    rng = np.random.default_rng(seed)
    past, offsets, off_d, past_d, kc, vc, qkv, nw = _problem(rng, past_list)
    max_past = int(past.max())
    rope_h = oracle.rope_table(max_past + 1)
    rope = torch.from_numpy(rope_h).cuda()
    prm = p2p_b200.Params(HQ, HKV)
    want = torch.zeros((len(past), HQ * D), dtype=torch.float16, device="cuda")
    kc_w, vc_w = kc.clone(), vc.clone()
    ctx.attn_decode_ragged(prm, qkv, nw, rope, kc_w, vc_w, off_d, past_d, want,
                           max_past=max_past, fused_prep=True)
    ctx.sync()
    for call in range(2):
        out = torch.full_like(want, float("nan"))
        kc_i, vc_i = kc.clone(), vc.clone()
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        p2p_b200.lib.p2p_debug_set_alloc_limit(0)  # any library allocation would now fail
        try:
            ctx.attn_decode_ragged_noalloc(prm, qkv, nw, rope, kc_i, vc_i, off_d, past_d, out,
                                           max_past=max_past, fused_prep=True)
            ctx.sync()
        finally:
            p2p_b200.lib.p2p_debug_set_alloc_limit(-1)
        free1 = torch.cuda.mem_get_info()[0]
        # the scratch array was placed when the context was created, not by this call
        assert free0 - free1 < SCRATCH_BYTES // 4, (free0, free1)
        got = out.cpu().numpy()
        assert_close(got, want.cpu().numpy(), what=f"no-alloc call {call}")
        assert torch.equal(kc_i, kc_w) and torch.equal(vc_i, vc_w)
    _check_against_oracle(oracle, check_seqs, past, offsets, kc, vc, qkv, nw, rope_h, got,
                          "no-alloc fused")
    # unfused form on the cache the fused call completed, against the allocating unfused call
    q_rot = torch.zeros((len(past), HQ * D), dtype=torch.float16, device="cuda")
    k_scr = torch.zeros((max_past + 1, HKV, D), dtype=torch.float16, device="cuda")
    v_scr = torch.zeros_like(k_scr)
    for i in range(len(past)):  # rotated q rows, as QK_PREP leaves them
        ctx.qk_prep(prm, qkv[i:i + 1], nw, rope, q_rot[i:i + 1], k_scr, v_scr,
                    pos0=int(past[i]), m_tokens=1)
    want_u = torch.zeros_like(want)
    ctx.attn_decode_ragged(prm, q_rot, None, None, kc_i, vc_i, off_d, past_d, want_u,
                           max_past=max_past, fused_prep=False)
    for call in range(2):
        out_u = torch.full_like(want, float("nan"))
        ctx.attn_decode_ragged_noalloc(prm, q_rot, None, None, kc_i, vc_i, off_d, past_d, out_u,
                                       max_past=max_past, fused_prep=False)
        ctx.sync()
        assert_close(out_u.cpu().numpy(), want_u.cpu().numpy(), what=f"unfused call {call}")
    # and the unfused outputs equal the fused ones (same q, same cache rows)
    assert_close(out_u.cpu().numpy(), got, what="unfused vs fused")
    return past


def test_noalloc_few_pairs_matches_allocating_entry_point_twice(oracle):
    """10 sequences x 8 kv heads: every sequence split to fill the SMs once."""
    import p2p_b200
    ctx = p2p_b200.Context(0)
    try:
        _run_twice(ctx, oracle, [0, 5, 63, 64, 700, 1023, 1024, 2049, 4000, 333], 2024,
                   [0, 3, 8])
    finally:
        ctx.close()


def test_noalloc_many_pairs_near_the_scratch_limit(oracle):
    """64 sequences x 8 kv heads (the fixed 1024-key split regime) with one sequence of 63487
    keys: 62 splits, whose partials and counters fill all but ~29 KB of the 32 MiB scratch."""
    import p2p_b200
    ctx = p2p_b200.Context(0)
    try:
        rng = np.random.default_rng(9)
        past = rng.integers(100, 3000, 64).astype(np.int32)
        past[17] = 63487
        past[40] = 2049
        _run_twice(ctx, oracle, past, 77, [0, 17, 40, 63])
    finally:
        ctx.close()


def test_noalloc_rejects_requests_beyond_its_scratch():
    import p2p_b200
    ctx = p2p_b200.Context(0)
    try:
        x = torch.zeros(4096 * HQ * D, dtype=torch.float16, device="cuda")
        idx = torch.zeros(64, dtype=torch.int32, device="cuda")
        # one 1024-key split more than the 64-sequence case above fits
        with pytest.raises(p2p_b200.P2PError) as e:
            ctx.attn_decode_ragged_noalloc(p2p_b200.Params(HQ, HKV), x.view(4096, HQ * D)[:64],
                                           None, None, x, x, idx, idx, x.view(4096, HQ * D),
                                           max_past=63488, fused_prep=False, kv_rows=1)
        assert e.value.status == 1 and "scratch" in str(e.value)
    finally:
        ctx.close()


def test_noalloc_refuses_sequences_outside_the_cache(oracle):
    """The same device-side check as the allocating entry point: a sequence reaching past the
    cache is skipped, the others are computed, and sync() reports KV_FULL."""
    import p2p_b200
    ctx = p2p_b200.Context(0)
    try:
        rng = np.random.default_rng(5)
        past, offsets, off_d, past_d, kc, vc, qkv, nw = _problem(rng, [50, 900, 20, 300])
        rope = ctx.rope_table(int(past.max()) + 1)
        prm = p2p_b200.Params(HQ, HKV)
        want = torch.zeros((4, HQ * D), dtype=torch.float16, device="cuda")
        ctx.attn_decode_ragged(prm, qkv, nw, rope, kc.clone(), vc.clone(), off_d, past_d, want,
                               max_past=int(past.max()), fused_prep=True)
        ctx.sync()
        # declare the cache one row shorter than sequence 3 needs (its new token's row)
        out = torch.full_like(want, 7.0)
        ctx.attn_decode_ragged_noalloc(prm, qkv, nw, rope, kc.clone(), vc.clone(), off_d,
                                       past_d, out, max_past=int(past.max()), fused_prep=True,
                                       kv_rows=int(offsets[3] + past[3]))
        with pytest.raises(p2p_b200.KvFullError):
            ctx.sync()
        got = out.cpu().numpy()
        assert (got[3] == 7.0).all()
        assert_close(got[:3], want.cpu().numpy()[:3], what="sequences beside the refused one")
    finally:
        ctx.close()
