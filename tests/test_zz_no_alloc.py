"""The decode entry point that allocates nothing (p2p_attn_decode_ragged_noalloc).

Callers that cannot allocate device memory while serving (a process that gave its free HBM
to its own pool at start-up, or a host whose device memory belongs to another component) use
this variant: its split scratch is a fixed array inside the library.  These tests call it
through the C ABI and compare it with p2p_attn_decode_ragged, the allocating entry point, on
two calls in a row, with the library's own allocations forbidden during the calls.  This file
is collected last so that a failure here leaves every other test already run.
"""
import numpy as np
import pytest

from conftest import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 64


def _problem(rng):
    past = np.array([0, 5, 63, 64, 700, 1023, 1024, 2049, 4000, 333], np.int32)
    offsets = np.zeros(len(past), np.int32)
    offsets[1:] = np.cumsum(past[:-1] + 1)
    rows = int(offsets[-1] + past[-1] + 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    kc = t(rng.standard_normal((rows, HKV, D)).astype(np.float16))
    vc = t(rng.standard_normal((rows, HKV, D)).astype(np.float16))
    qkv = t(rng.standard_normal((len(past), (HQ + 2 * HKV) * D)).astype(np.float16))
    nw = t((1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16))
    return past, t(offsets), t(past), kc, vc, qkv, nw


def test_noalloc_matches_allocating_entry_point_twice():
    import p2p_b200
    ctx = p2p_b200.Context(0)
    try:
        rng = np.random.default_rng(2024)
        past, off_d, past_d, kc, vc, qkv, nw = _problem(rng)
        rope = ctx.rope_table(int(past.max()) + 1)
        prm = p2p_b200.Params(HQ, HKV)
        want = torch.zeros((len(past), HQ * D), dtype=torch.float16, device="cuda")
        ctx.attn_decode_ragged(prm, qkv, nw, rope, kc.clone(), vc.clone(), off_d, past_d, want,
                               max_past=int(past.max()), fused_prep=True)
        torch.cuda.synchronize()
        for call in range(2):
            out = torch.full_like(want, float("nan"))
            kc_i, vc_i = kc.clone(), vc.clone()
            torch.cuda.synchronize()
            p2p_b200.lib.p2p_debug_set_alloc_limit(0)  # any library allocation would now fail
            try:
                ctx.attn_decode_ragged_noalloc(prm, qkv, nw, rope, kc_i, vc_i, off_d, past_d,
                                               out, max_past=int(past.max()), fused_prep=True)
                ctx.sync()
            finally:
                p2p_b200.lib.p2p_debug_set_alloc_limit(-1)
            assert_close(out.cpu().numpy(), want.cpu().numpy(), what=f"no-alloc call {call}")
        # unfused form as well, on the cache the fused call completed
        out_u = torch.zeros_like(want)
        ctx.attn_decode_ragged_noalloc(prm, qkv, None, None, kc_i, vc_i, off_d, past_d, out_u,
                                       max_past=int(past.max()), fused_prep=False)
        ctx.sync()
        assert np.isfinite(out_u.float().cpu().numpy()).all()
    finally:
        ctx.close()


def test_noalloc_rejects_requests_beyond_its_scratch():
    import p2p_b200
    ctx = p2p_b200.Context(0)
    try:
        x = torch.zeros(4096 * HQ * D, dtype=torch.float16, device="cuda")
        idx = torch.zeros(4096, dtype=torch.int32, device="cuda")
        with pytest.raises(p2p_b200.P2PError) as e:
            ctx.attn_decode_ragged_noalloc(p2p_b200.Params(HQ, HKV), x.view(4096, HQ * D), None,
                                           None, x, x, idx, idx, x.view(4096, HQ * D),
                                           max_past=100000, fused_prep=False)
        assert e.value.status == 1 and "scratch" in str(e.value)
    finally:
        ctx.close()
