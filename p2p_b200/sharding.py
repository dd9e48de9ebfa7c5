"""Multi-GPU partitioning of the attention path (one process per GPU).

Where the work shards naturally:
  * batched decode -- independent sequences: greedy LPT by token count (not by sequence
    count) gives every rank a near-equal share of KV bytes to stream; no collective on the
    data path.
  * long-context prefill -- KV-head groups: rank g owns kv heads [g*Hkv/G, (g+1)*Hkv/G) and
    their query heads, computes out[:, heads_g] and its KV-cache slice; either one NCCL
    all-gather inside the library assembles the [S][Hq*D] output (HeadShardedPrefill, the C
    ABI's p2p_attn_prefill_sharded over its own communicator), or the flash kernel writes
    its rows straight into every rank's full output over NVLink, either once per peer
    (ScatterHeadShardedPrefill) or once as NVLink multicast stores that NVSwitch replicates
    (MulticastHeadShardedPrefill).
  * vision -- independent images.
  * single-sequence decode does not shard (8.4 MB per layer is less than the cost of a
    cross-GPU exchange): replicas only.
"""
from __future__ import annotations

import heapq
from typing import List, Sequence, Tuple


def lpt_partition(costs: Sequence[int], world: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of items (by cost) to `world` bins.

    Returns, per rank, the item indices in ascending order.  Deterministic: ties go to the
    lower rank, items of equal cost in index order."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    heap = [(0, r) for r in range(world)]
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + int(costs[i]), r))
    return [sorted(b) for b in bins]


def head_groups(num_heads: int, num_kv_heads: int, world: int, rank: int) -> Tuple[int, int, int, int]:
    """KV-head group of `rank`: (kv_head0, kv_heads, q_head0, q_heads).  world must divide
    num_kv_heads so that every rank owns whole GQA groups."""
    if num_kv_heads % world:
        raise ValueError(f"{world} ranks do not divide {num_kv_heads} kv heads")
    g = num_heads // num_kv_heads
    kv_per = num_kv_heads // world
    return rank * kv_per, kv_per, rank * kv_per * g, kv_per * g


def split_images(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous image range [start, start+count) of `rank`."""
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def assemble_head_shards(gathered, s_tokens: int, q_heads_per_rank: int, head_dim: int = 64):
    """Turn the all-gathered per-rank outputs [world][S][q_heads_per_rank*D] into the
    reference layout [S][Hq*D] (head h at column h*D).  Works on torch tensors."""
    world = gathered.shape[0]
    x = gathered.reshape(world, s_tokens, q_heads_per_rank * head_dim)
    return x.permute(1, 0, 2).reshape(s_tokens, world * q_heads_per_rank * head_dim)


class HeadShardedPrefill:
    """Causal prefill over `world` GPUs split by KV-head group (one process per GPU).

    Rank g owns kv heads [g*Hkv/G, (g+1)*Hkv/G) and their query heads: its QK_PREP writes only
    its slice of the KV cache (dense [cap][Hkv/G][64] on this GPU, the layout a column-parallel
    QKV projection produces) and its flash attention produces out[:, heads_g].  One all-gather
    over NVLink exchanges the [M][Hq/G*64] slices and every rank assembles the reference's
    [M][Hq*64] layout -- all inside the library (p2p_attn_prefill_sharded, its own NCCL
    communicator), so a host calling the C ABI needs no collective library of its own.
    `comm` is a p2p_b200.Comm; without one it is created over the torch.distributed group.
    """

    def __init__(self, ctx, num_heads: int, num_kv_heads: int, world: int, rank: int,
                 group=None, comm=None):
        from .attention import Params
        from .comm import Comm
        self.ctx, self.world, self.rank, self.group = ctx, world, rank, group
        self.kv0, self.kvn, self.q0, self.qn = head_groups(num_heads, num_kv_heads, world, rank)
        self.prm = Params(self.qn, self.kvn)
        self.prm_full = Params(num_heads, num_kv_heads)
        self.num_heads = num_heads
        self.own_comm = comm is None
        self.comm = comm if comm is not None else Comm.from_process_group(ctx, world, rank,
                                                                          group)

    def local_qkv_columns(self, head_dim: int = 64):
        """Column indices of this rank's q, k and v heads inside a full qkv row."""
        import torch
        hq, d = self.num_heads, head_dim
        hkv = self.kvn * self.world
        cols = [torch.arange(self.q0 * d, (self.q0 + self.qn) * d),
                torch.arange(hq * d + self.kv0 * d, hq * d + (self.kv0 + self.kvn) * d),
                torch.arange((hq + hkv) * d + self.kv0 * d, (hq + hkv) * d + (self.kv0 + self.kvn) * d)]
        return torch.cat(cols)

    def __call__(self, qkv_local, norm_w, rope, k_cache, v_cache, out_full, pos0: int,
                 m_tokens: int, stream=None):
        self.ctx.attn_prefill_sharded(self.comm, self.prm_full, qkv_local, norm_w, rope,
                                      k_cache, v_cache, out_full, pos0=pos0, m_tokens=m_tokens,
                                      stream=stream)
        return out_full

    def close(self):
        if self.own_comm and self.comm is not None:
            self.comm.close()
        self.comm = None


class ScatterHeadShardedPrefill(HeadShardedPrefill):
    """HeadShardedPrefill without the all-gather: the flash kernel of every rank writes each of
    its output rows straight into the full [max_tokens][Hq*64] output buffer of every rank (its
    own, and the other ranks' through CUDA IPC mappings, so the rows cross NVLink as the
    kernel's own stores, overlapped with its compute).  One all-reduce of a single element then
    orders the ranks, after which every rank's buffer holds all heads.

    The buffers are reused by every call: a rank must be done reading one result before any
    rank starts the next call (in a model, the next layer's collective orders that)."""

    def __init__(self, ctx, num_heads: int, num_kv_heads: int, world: int, rank: int,
                 max_tokens: int, group=None, comm=None):
        import torch
        import torch.distributed as dist
        from .attention import _from_device_ptr
        super().__init__(ctx, num_heads, num_kv_heads, world, rank, group, comm)
        self.max_tokens = max_tokens
        self.ld_o = num_heads * 64
        nbytes = max_tokens * self.ld_o * 2
        self.own, handle = ctx.shared_alloc(nbytes)
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles[0] = handle
        self.peers = [ctx.shared_open(handles[r]) for r in range(world) if r != rank]
        self.outs = [self.own] + self.peers
        self.out_full = _from_device_ptr(self.own, nbytes, ctx.device).view(torch.float16).view(
            max_tokens, self.ld_o)

    def __call__(self, qkv_local, norm_w, rope, k_cache, v_cache, q_buf, pos0: int,
                 m_tokens: int, stream=None):
        if m_tokens > self.max_tokens:
            raise ValueError(f"{m_tokens} tokens > max_tokens {self.max_tokens}")
        self.ctx.qk_prep(self.prm, qkv_local, norm_w, rope, q_buf, k_cache, v_cache, pos0=pos0,
                         m_tokens=m_tokens, stream=stream)
        self.ctx.attn_scatter(self.prm, q_buf, k_cache, v_cache, self.outs, self.ld_o, self.q0,
                              pos0=pos0, m_tokens=m_tokens, stream=stream)
        if self.world > 1:
            self.comm.barrier(stream)  # every rank's rows have landed
        return self.out_full[:m_tokens]

    def close(self):
        import torch.distributed as dist
        for p in self.peers:
            self.ctx.shared_close(p)
        self.peers = []
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank still maps this rank's buffer
        if self.own:
            self.ctx.shared_free(self.own)
            self.own = None
        super().close()


class MulticastHeadShardedPrefill(HeadShardedPrefill):
    """HeadShardedPrefill whose flash epilogue stores every output row once, to the NVLink
    multicast address of a symmetric-memory buffer bound on all ranks: NVSwitch writes it into
    every rank's full [max_tokens][Hq*64] output, so a GPU sends its slice once instead of once
    per peer (the scatter variant's cost grows with the number of GPUs).  One all-reduce of a
    single element then orders the ranks.  Needs NVLink multicast (NVSwitch); raises if the
    node has none.  The same buffer reuse rule as ScatterHeadShardedPrefill applies."""

    def __init__(self, ctx, num_heads: int, num_kv_heads: int, world: int, rank: int,
                 max_tokens: int, group=None, comm=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        super().__init__(ctx, num_heads, num_kv_heads, world, rank, group, comm)
        self.max_tokens = max_tokens
        self.ld_o = num_heads * 64
        self.out_full = symm_mem.empty((max_tokens, self.ld_o), dtype=torch.float16,
                                       device=f"cuda:{ctx.device}")
        self.handle = symm_mem.rendezvous(self.out_full, group or dist.group.WORLD)
        self.mc = int(self.handle.multicast_ptr)
        if not self.mc:
            raise RuntimeError("no NVLink multicast support for this group")

    def __call__(self, qkv_local, norm_w, rope, k_cache, v_cache, q_buf, pos0: int,
                 m_tokens: int, stream=None):
        if m_tokens > self.max_tokens:
            raise ValueError(f"{m_tokens} tokens > max_tokens {self.max_tokens}")
        self.ctx.qk_prep(self.prm, qkv_local, norm_w, rope, q_buf, k_cache, v_cache, pos0=pos0,
                         m_tokens=m_tokens, stream=stream)
        self.ctx.attn_multicast(self.prm, q_buf, k_cache, v_cache, self.mc, self.ld_o, self.q0,
                                pos0=pos0, m_tokens=m_tokens, stream=stream)
        if self.world > 1:
            self.comm.barrier(stream)  # every rank's rows have landed
        return self.out_full[:m_tokens]
