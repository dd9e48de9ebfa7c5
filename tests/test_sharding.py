"""Host-side multi-GPU logic on CPU: LPT sharding by tokens, KV-head groups, image splits,
and the all-gather assembly of head-sharded prefill outputs over a world-size-2 gloo group."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from p2p_b200.sharding import assemble_head_shards, head_groups, lpt_partition, split_images


def test_lpt_partition_balances_tokens():
    rng = np.random.default_rng(4)
    lengths = rng.integers(1024, 32769, 256)
    for world in (1, 2, 4, 8):
        bins = lpt_partition(lengths, world)
        assert sorted(i for b in bins for i in b) == list(range(256))
        loads = [int(lengths[b].sum()) for b in bins]
        # LPT guarantee: max load <= 4/3 of optimal; here within 1% of the mean
        assert max(loads) <= 1.01 * sum(loads) / world + lengths.max()
        assert max(loads) - min(loads) <= lengths.max()
    assert lpt_partition([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]


def test_head_groups_and_images():
    assert head_groups(32, 8, 4, 1) == (2, 2, 8, 8)
    assert head_groups(32, 8, 8, 7) == (7, 1, 28, 4)
    with pytest.raises(ValueError):
        head_groups(32, 8, 3, 0)
    parts = [split_images(16, 3, r) for r in range(3)]
    assert parts == [(0, 6), (6, 5), (11, 5)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    s, hq, hkv, d = 5, 32, 8, 64
    full = torch.arange(s * hq * d, dtype=torch.float32).reshape(s, hq * d)
    kv0, kvn, q0, qn = head_groups(hq, hkv, world, rank)
    mine = full[:, q0 * d:(q0 + qn) * d].contiguous()
    out = torch.empty((world * s, qn * d))  # ranks concatenated along dim 0
    dist.all_gather_into_tensor(out, mine)
    got = assemble_head_shards(out.view(world, s, qn * d), s, qn, d)
    q.put((rank, bool(torch.equal(got, full))))
    dist.destroy_process_group()


def test_allgather_assembles_head_shards_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok in results)
