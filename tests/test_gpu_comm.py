"""The library's own communicator on one GPU (two-GPU runs are in test_gpu_multi.py).

  * a one-rank communicator runs p2p_attn_prefill_sharded through the C ABI: the result equals
    QK_PREP + ATTN on all heads and the oracle;
  * a peer that never joins: p2p_comm_create returns P2P_ERR_TIMEOUT after its host-side limit
    (the failure is made on the host -- the second rank simply never starts -- and no GPU work
    is in flight; run in a child process with NVLink SHARP off).
"""
import os
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import numpy as np
import pytest

from conftest import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
D = 64


def test_one_rank_prefill_sharded_equals_attn_and_oracle(oracle):
    import p2p_b200
    from p2p_b200.comm import Comm, unique_id
    ctx = p2p_b200.Context(0)
    comm = Comm(ctx, 1, 0, unique_id(), timeout_ms=30000)
    try:
        hq, hkv, m = 32, 8, 257
        rng = np.random.default_rng(12)
        qkv = rng.standard_normal((m, (hq + 2 * hkv) * D)).astype(np.float16)
        nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
        rope = oracle.rope_table(m)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
        prm = p2p_b200.Params(hq, hkv)
        kc = torch.zeros((m, hkv, D), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        out = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
        for _ in range(2):
            ctx.attn_prefill_sharded(comm, prm, dev(qkv), dev(nw), dev(rope), kc, vc, out,
                                     pos0=0, m_tokens=m)
            comm.wait()
        q = torch.zeros((m, hq * D), dtype=torch.float16, device="cuda")
        kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
        want_dev = torch.zeros_like(out)
        ctx.qk_prep(prm, dev(qkv), dev(nw), dev(rope), q, kc2, vc2, pos0=0, m_tokens=m)
        ctx.attn(prm, q, kc2, vc2, want_dev, pos0=0, m_tokens=m)
        ctx.sync()
        assert torch.equal(out, want_dev) and torch.equal(kc, kc2) and torch.equal(vc, vc2)
        qo = np.zeros((m, hq * D), np.float16)
        ko = np.zeros((m, hkv, D), np.float16)
        vo = np.zeros_like(ko)
        oracle.qk_prep(hq, hkv, D, qkv, nw, rope, qo, ko, vo, 0, m)
        want = np.zeros((m, hq * D), np.float16)
        oracle.attn(hq, hkv, D, qo, ko, vo, want, 0, m)
        assert_close(out.cpu().numpy(), want, what="one-rank sharded prefill")
    finally:
        comm.close()
        ctx.close()


_NEVER_JOINS = textwrap.dedent("""
    import sys, time
    sys.path.insert(0, sys.argv[1])
    import p2p_b200
    from p2p_b200.comm import Comm, unique_id
    ctx = p2p_b200.Context(0)
    t0 = time.time()
    try:
        Comm(ctx, 2, 0, unique_id(), timeout_ms=3000)   # rank 1 is never started
        print("STATUS ok")
    except p2p_b200.P2PError as e:
        print("STATUS", e.status, round(time.time() - t0, 2), str(e)[:160])
    ctx.close()
""")


def test_peer_that_never_joins_times_out_on_the_host():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    t0 = time.time()
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS, str(ROOT)], capture_output=True,
                       text=True, timeout=180, env=env)
    line = [x for x in r.stdout.splitlines() if x.startswith("STATUS")]
    assert r.returncode == 0 and line, (r.returncode, r.stdout[-800:], r.stderr[-800:])
    parts = line[0].split()
    assert parts[1] == "5", line[0]           # P2P_ERR_TIMEOUT
    assert 2.5 <= float(parts[2]) < 60.0, line[0]
    assert time.time() - t0 < 170
