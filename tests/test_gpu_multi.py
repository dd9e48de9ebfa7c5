"""Multi-GPU paths on real GPUs (skipped with fewer than 2 visible GPUs).

Two NCCL ranks, one process per GPU, rendezvous on 127.0.0.1:
  * causal prefill split by KV-head group + all-gather (p2p_attn_prefill_sharded: NCCL inside
    the library, through the C ABI) vs the oracle on the full heads, and
    the same with the flash kernel scattering its rows into every rank's output (CUDA IPC);
  * ragged decode split by sequence (LPT by tokens, no collective) vs the oracle.

And one process driving two GPUs through two contexts: the kernels whose launch sets
per-device attributes (flash attention, the prompt-chunk GEMM in both tile forms) give the same
bits on the second device as on the first.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

D = 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import p2p_b200
    from oracle import pyoracle as O
    from p2p_b200.sharding import HeadShardedPrefill, lpt_partition

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    ok = {}
    try:
        ctx = p2p_b200.Context(rank)
        hq, hkv, m = 32, 8, 300
        rng = np.random.default_rng(31)  # identical inputs on every rank
        qkv = (0.5 * rng.standard_normal((m, (hq + 2 * hkv) * D))).astype(np.float16)
        nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
        rope = O.rope_table(m)
        # the library's own communicator (NCCL inside libp2pattn.so), id shared over the group
        sp = HeadShardedPrefill(ctx, hq, hkv, world, rank)
        cols = sp.local_qkv_columns().numpy()
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
        qkv_l = dev(qkv[:, cols])
        kc = torch.zeros((m, sp.kvn, D), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        q_buf = torch.zeros((m, sp.qn * D), dtype=torch.float16, device="cuda")
        out = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
        sp(qkv_l, dev(nw), dev(rope), kc, vc, out, 0, m)
        sp.comm.wait()
        # oracle on the full heads
        qo = np.zeros((m, hq * D), np.float16)
        ko = np.zeros((m, hkv, D), np.float16)
        vo = np.zeros_like(ko)
        O.qk_prep(hq, hkv, D, qkv, nw, rope, qo, ko, vo, 0, m)
        want = np.zeros((m, hq * D), np.float16)
        O.attn(hq, hkv, D, qo, ko, vo, want, 0, m)
        got = out.cpu().numpy().astype(np.float64)
        err = np.abs(got - want)
        ok["prefill"] = bool((err <= 2e-3 + 1e-2 * np.abs(want.astype(np.float64))).all())
        ok["prefill_kv_slice"] = bool(np.array_equal(
            kc.cpu().numpy().view(np.uint16), ko[:, sp.kv0:sp.kv0 + sp.kvn].view(np.uint16)))
        # a second chunk through the same communicator, positions 0..m-1 again, same result
        out.zero_()
        sp(qkv_l, dev(nw), dev(rope), kc, vc, out, 0, m)
        sp.comm.wait()
        ok["prefill_again"] = bool(np.array_equal(out.cpu().numpy(), got.astype(np.float16)))
        comm = sp.comm
        # the same prefill with the flash kernel writing its rows into every rank's output
        # over NVLink (CUDA IPC mappings) instead of an all-gather; twice in a row
        from p2p_b200.sharding import ScatterHeadShardedPrefill
        ssp = ScatterHeadShardedPrefill(ctx, hq, hkv, world, rank, max_tokens=m, comm=comm)
        for it in range(2):
            kc.zero_()
            vc.zero_()
            full = ssp(qkv_l, dev(nw), dev(rope), kc, vc, q_buf, 0, m)
            torch.cuda.synchronize()
            g3 = full.cpu().numpy().astype(np.float64)
            ok[f"scatter_{it}"] = bool((np.abs(g3 - want) <= 2e-3 + 1e-2 * np.abs(want.astype(np.float64))).all())
        ssp.close()
        # the same with every row stored once to an NVLink multicast address (NVSwitch
        # writes it into both ranks' outputs), where the node supports multicast
        from p2p_b200.sharding import MulticastHeadShardedPrefill
        try:
            msp = MulticastHeadShardedPrefill(ctx, hq, hkv, world, rank, max_tokens=m,
                                              comm=comm)
        except RuntimeError:
            msp = None
        if msp is not None:
            for it in range(2):
                kc.zero_()
                vc.zero_()
                full = msp(qkv_l, dev(nw), dev(rope), kc, vc, q_buf, 0, m)
                torch.cuda.synchronize()
                g4 = full.cpu().numpy().astype(np.float64)
                ok[f"multicast_{it}"] = bool((np.abs(g4 - want) <= 2e-3 + 1e-2 * np.abs(want.astype(np.float64))).all())
            del msp
        # ragged decode split by sequence
        past = np.array([100, 2000, 37, 700, 1500, 9], np.int32)
        mine = lpt_partition(list(past + 1), world)[rank]
        pl = past[mine]
        offs = np.zeros(len(pl), np.int32)
        offs[1:] = np.cumsum(pl[:-1] + 1)
        rows = int(offs[-1] + pl[-1] + 1)
        r2 = np.random.default_rng(100 + rank)
        kc2 = r2.standard_normal((rows, hkv, D)).astype(np.float16)
        vc2 = r2.standard_normal((rows, hkv, D)).astype(np.float16)
        q2 = r2.standard_normal((len(pl), hq * D)).astype(np.float16)
        want2 = np.zeros((len(pl), hq * D), np.float16)
        O.attn_ragged(hq, hkv, D, q2, kc2, vc2, offs.astype(np.int64), pl, want2)
        out2 = torch.zeros((len(pl), hq * D), dtype=torch.float16, device="cuda")
        ctx.attn_decode_ragged(p2p_b200.Params(hq, hkv), dev(q2), None, None, dev(kc2), dev(vc2),
                               dev(offs), dev(pl), out2, max_past=int(past.max()),
                               fused_prep=False)
        sp.close()
        g2 = out2.cpu().numpy().astype(np.float64)
        ok["ragged"] = bool((np.abs(g2 - want2) <= 2e-3 + 1e-2 * np.abs(want2.astype(np.float64))).all())
        ctx.close()
    finally:
        dist.destroy_process_group()
    q.put((rank, ok))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_gpu_prefill_heads_and_ragged_sequences():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok in results.items():
        assert all(ok.values()), (rank, ok)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_devices_in_one_process(oracle):
    import p2p_b200
    rng = np.random.default_rng(8)
    hq, hkv, s_tok, k, n = 32, 8, 512, 1024, 3072
    q = (0.5 * rng.standard_normal((s_tok, hq * D))).astype(np.float16)
    kc = (0.5 * rng.standard_normal((s_tok, hkv, D))).astype(np.float16)
    vc = rng.standard_normal((s_tok, hkv, D)).astype(np.float16)
    wq, sc, zp = oracle.random_q4(rng, n, k)
    x = rng.standard_normal((s_tok, k)).astype(np.float16)
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            ctx = p2p_b200.Context(dev)
            try:
                t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{dev}")
                out = torch.zeros((s_tok, hq * D), dtype=torch.float16, device=f"cuda:{dev}")
                ctx.attn(p2p_b200.Params(hq, hkv), t(q), t(kc), t(vc), out, pos0=0,
                         m_tokens=s_tok)
                w = (t(wq.view(np.int32)), t(sc), t(zp.view(np.int32)))
                ys = []
                for pair in ("0", "1"):  # single-CTA and 2-CTA tiles
                    os.environ["P2P_GEMM_PAIR"] = pair
                    y = torch.zeros((s_tok, n), dtype=torch.float16, device=f"cuda:{dev}")
                    ctx.gemm_q4(w, t(x), y)
                    ys.append(y)
                os.environ.pop("P2P_GEMM_PAIR", None)
                ctx.sync()
                outs.append([o.cpu().numpy().view(np.uint16) for o in [out] + ys])
            finally:
                os.environ.pop("P2P_GEMM_PAIR", None)
                ctx.close()
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    assert np.isfinite(outs[0][0].view(np.float16).astype(np.float32)).all()
