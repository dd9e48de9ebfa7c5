"""Benchmark of the attention hot path on B200 (one JSON line on rank 0).

Headline (N GPUs, one process per GPU): LFM2.5-1.2B decode attention at context 4096 --
32 q / 8 kv heads, head_dim 64, fp16 KV cache of 4096 past tokens plus one new token per step,
6 independent attention layers with their own seeded N(0,1) q/k/v.  One step = QK_PREP (q/k
RMSNorm + RoPE + KV append) and ATTN for all 6 layers, one launch of the fused split-KV kernel.
The metric is achieved GB/s over the algorithmic bytes (K/V rows read + q/new-row/out
traffic, 8,400,896 B per layer) and us/step.  At N > 1 each GPU decodes its own sequences
(weak scaling: per-GPU work fixed; the ranks share nothing on the data path).

Side legs (reported inside the same line): causal prefill S=2048 (TFLOP/s), the SigLIP2
vision attention B=16 x S=1024 x 12 heads (TFLOP/s), and ragged batched decode over 256
sequences with contexts U[1024, 32768] sharded by sequence across the N GPUs (GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

L2 (126 MB) is defeated by rotating the decode step over 12 distinct copies of the 6-layer
KV cache (605 MB); prefill/vision/ragged inputs are larger than L2 or rotated likewise.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HQ, HKV, D = 32, 8, 64
PAST = 4096
N_LAYERS = 6
ROW_BYTES = HKV * D * 2  # one token's K (or V) row for all kv heads, fp16


def decode_layer_bytes(past: int = PAST) -> int:
    kv = (past + 1) * HKV * D * 2 * 2                    # K and V rows 0..past
    q = (HQ + 2 * HKV) * D * 2                           # the new token's qkv row
    new = 2 * HKV * D * 2                                # appended k/v row
    out = HQ * D * 2
    return kv + q + new + out


def prefill_flops(s: int, hq: int = HQ, d: int = D) -> float:
    return 4.0 * d * hq * s * (s + 1) / 2  # exact causal pairs


def vision_flops(b=16, s=1024, nh=12, d=D) -> float:
    return 4.0 * s * s * d * nh * b


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def load_traffic():
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/p2p_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3][1:5])
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded),
                "sm_max_mhz": max(r[1] for r in loaded), "reasons": reasons,
                "samples": len(loaded)}


# ---------------------------------------------------------------------------------------------
# distributed plumbing (barrier + max over ranks only; nothing on the data path)

def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------------------------
# the checker: outputs of each leg compared after its timed region (never inside it).  An
# element passes when |x - r| <= 2e-3 + 1e-2 |r|; max-abs and max-rel (over |r| > 1e-3, and
# over |r| > 1e-2) are reported separately as well; within_caps = max-abs <= 2e-3 and
# max-rel <= 1e-2 as two separate caps.

ATOL, RTOL = 2e-3, 1e-2


def parity_stats(got, want, what):
    import numpy as np
    x = np.asarray(got, np.float64)
    r = np.asarray(want, np.float64)
    err = np.abs(x - r)
    finite = bool(np.isfinite(x).all())
    bad = int((~(err <= ATOL + RTOL * np.abs(r))).sum())
    big = np.abs(r) > 1e-3
    big2 = np.abs(r) > 1e-2
    return {"max_abs": float(err.max()) if err.size else 0.0,
            "max_rel": float((err[big] / np.abs(r[big])).max()) if big.any() else 0.0,
            "max_rel_r_gt_1e-2": float((err[big2] / np.abs(r[big2])).max()) if big2.any() else 0.0,
            "bad": bad if finite else int(x.size), "n": int(x.size), "checked": what}


def reduce_parity(p, world):
    """Every rank's stats -> the job's (max of the maxima, sum of the counts); same collective
    steps on every rank."""
    out = dict(p)
    out["max_abs"] = max_over_ranks(p["max_abs"], world)
    out["max_rel"] = max_over_ranks(p["max_rel"], world)
    out["max_rel_r_gt_1e-2"] = max_over_ranks(p["max_rel_r_gt_1e-2"], world)
    out["bad"] = int(sum_over_ranks(float(p["bad"]), world))
    out["n"] = int(sum_over_ranks(float(p["n"]), world))
    out["ok"] = out["bad"] == 0
    out["within_caps"] = out["max_abs"] <= ATOL and out["max_rel"] <= RTOL
    for k in ("max_abs", "max_rel", "max_rel_r_gt_1e-2"):
        out[k] = float(f"{out[k]:.3e}")
    if world > 1:
        out["checked"] = f"every rank: {p['checked']}"
    return out


# ---------------------------------------------------------------------------------------------
# workloads

def warm_up_agreed(fn, warmup, world):
    """The untimed warm-up calls, then every rank learns whether any rank's failed (one
    all-reduce): a library error on one rank only becomes the same P2PError on every rank, so
    no rank is left waiting in a collective the others skipped."""
    import torch
    import p2p_b200
    err = None
    try:
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
    except p2p_b200.P2PError as e:
        err = e
    if world > 1 and max_over_ranks(1.0 if err is not None else 0.0, world) > 0 and err is None:
        err = p2p_b200.P2PError(-1, "the leg failed on another rank")
    if err is not None:
        raise err


def timed_loop(fn, steps, warmup, world, stream):
    import torch
    warm_up_agreed(fn, warmup, world)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        fn(warmup + i)
    end.record(stream)
    end.synchronize()
    barrier(world)
    return start.elapsed_time(end) / steps  # ms per step on this rank


def timed_graph(fn, steps, warmup, world, capture_error_mode="global"):
    """Warm up with direct calls, capture `steps` calls into one CUDA graph, then time one
    replay (the K steps back to back on the device, no host launch overhead).  Legs with NCCL
    calls capture in "relaxed" mode (NCCL may enqueue from its own thread)."""
    import torch
    warm_up_agreed(fn, warmup, world)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode=capture_error_mode):
        for i in range(steps):
            fn(warmup + i)
    g.replay()  # untimed: first replay uploads the graph
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    g.replay()
    end.record(stream)
    end.synchronize()
    barrier(world)
    del g
    return start.elapsed_time(end) / steps


def stream_reference(ctx, nbytes, steps, warmup, world, copies=12):
    """The speed of light of "read these bytes in one launch": p2p_debug_stream_read over the
    same number of bytes, one launch per graph node, rotating over `copies` windows of one
    buffer (> L2) exactly like the decode legs.  Returns (us per launch, bytes)."""
    import torch
    n = (int(nbytes) + 15) // 16 * 16
    buf = torch.empty((copies * n // 4,), dtype=torch.int32, device="cuda")
    buf.random_(generator=torch.Generator(device="cuda").manual_seed(7))
    sink = torch.zeros(1, dtype=torch.int32, device="cuda")
    views = [buf[i * n // 4:(i + 1) * n // 4] for i in range(copies)]

    def step(i):
        ctx.debug_stream_read(views[i % copies], sink, n)

    ms = max_over_ranks(timed_graph(step, steps, warmup, world), world)
    del buf, views
    return ms * 1e3, n


class DecodeWorkload:
    """6 independent LFM2.5-1.2B attention layers at context 4096 (+1), R rotating copies."""

    def __init__(self, ctx, rank, copies=12, past=PAST):
        import torch
        import p2p_b200
        self.torch = torch
        self.prm = p2p_b200.Params(HQ, HKV)
        self.ctx = ctx
        cap = past + 1
        self.cap = cap
        g = torch.Generator(device="cuda").manual_seed(1234 + rank)
        self.rope = ctx.rope_table(cap, D, 1e6)
        self.copies = []
        for c in range(copies):
            layers = []
            for l in range(N_LAYERS):
                kc = torch.randn((cap, HKV, D), generator=g, device="cuda", dtype=torch.float16)
                vc = torch.randn((cap, HKV, D), generator=g, device="cuda", dtype=torch.float16)
                layers.append((kc, vc))
            self.copies.append(layers)
        self.qkv = torch.randn((N_LAYERS, (HQ + 2 * HKV) * D), generator=g, device="cuda",
                               dtype=torch.float16)
        self.nw = (1 + 0.1 * torch.randn((N_LAYERS, 2 * D), generator=g, device="cuda")).half()
        self.out = torch.zeros((N_LAYERS, HQ * D), device="cuda", dtype=torch.float16)
        self.plans = [
            ctx.plan_decode_step(self.prm, [(self.qkv[l], self.nw[l], kc, vc, self.out[l])
                                            for l, (kc, vc) in enumerate(c)],
                                 self.rope, cap, use_meta=True)
            for c in self.copies]
        # the drop-in per-layer call (engine.js:245-259 runs QK_PREP/ATTN once per attention
        # layer, between that layer's GEMMs): every (copy, layer) cache as its own one-layer
        # step, rotating over all of them (605 MB > L2)
        self.layer_plans = [
            ctx.plan_decode_step(self.prm, [(self.qkv[l], self.nw[l], kc, vc, self.out[l])],
                                 self.rope, cap, use_meta=True)
            for c in self.copies for l, (kc, vc) in enumerate(c)]
        ctx.meta_write(past, 1, 0, stream=torch.cuda.current_stream())
        self.past = past
        self.bytes_per_step = N_LAYERS * decode_layer_bytes(past)

    def step(self, i):
        self.plans[i % len(self.plans)].run()

    def step_one_layer(self, i):
        self.layer_plans[i % len(self.layer_plans)].run()

    def check(self):
        """The checker, after the timed regions: copy 0's six layers against the oracle."""
        import numpy as np
        from oracle import pyoracle as O
        torch = self.torch
        self.plans[0].run()
        torch.cuda.synchronize()
        got = self.out.cpu().numpy()
        rope = self.rope_host()
        want = np.zeros((N_LAYERS, HQ * D), np.float16)
        for l, (kc, vc) in enumerate(self.copies[0]):
            k_h = kc.cpu().numpy()
            v_h = vc.cpu().numpy()
            q = np.zeros((1, HQ * D), np.float16)
            O.qk_prep(HQ, HKV, D, self.qkv[l:l + 1].cpu().numpy(), self.nw[l].cpu().numpy(),
                      rope, q, k_h, v_h, self.past, 1)
            o = np.zeros((1, HQ * D), np.float16)
            O.attn(HQ, HKV, D, q, k_h, v_h, o, self.past, 1)
            want[l] = o[0]
        return parity_stats(got, want, f"6 layers x {HQ} heads at past {self.past} vs the oracle")

    def rope_host(self):
        from oracle import pyoracle as O
        return O.rope_table(self.cap)


def q4_weights(g, n, k):
    """A random 4-bit MatMulNBits matrix (qweight words, f16 scales, zero-point words) on the
    device; int32 tensors carry the u32 words."""
    import torch
    qw = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=g, device="cuda",
                       dtype=torch.int32)
    sc = (0.01 + 0.02 * torch.rand((n, k // 32), generator=g, device="cuda")).half()
    zr = (k // 32 + 1) // 2
    zp = torch.randint(-2**31, 2**31 - 1, ((n * zr + 3) // 4,), generator=g, device="cuda",
                       dtype=torch.int32)
    return qw, sc, zp


def q4_bytes(n, k):
    return n * (k // 2 + (k // 32) * 2 + (k // 32 + 1) // 2)


def run_decode_block(ctx, wl, steps, warmup, fused=True, sets=4):
    """The six attention layers of one LFM2.5-1.2B decode step with their projections: per
    layer the q/k/v projection of the token's hidden row (4-bit weights), QK_PREP, attention
    over the ctx-4096 cache and the o_proj consumer.  fused: p2p_qkv_gemv_prep (QK_PREP in the
    projection's epilogue) + p2p_attn + p2p_gemv_q4, 3 launches per layer; unfused: the
    reference's order, three GEMVs into the qkv row, then QK_PREP + attention
    (p2p_decode_step, one layer) and o_proj, 5 launches.  Weights rotate over `sets` copies
    and the caches over the workload's 12 (L2 defeated).  Returns (ms per step, bytes)."""
    import torch
    import p2p_b200
    k = HQ * D  # the hidden size of LFM2.5-1.2B (2048)
    g = torch.Generator(device="cuda").manual_seed(91)
    weights = [[tuple(q4_weights(g, n, k) for n in (HQ * D, HKV * D, HKV * D, k))
                for _ in range(N_LAYERS)] for _ in range(sets)]
    x = (torch.randn((N_LAYERS, k), generator=g, device="cuda")).half()
    q = torch.zeros((N_LAYERS, HQ * D), device="cuda", dtype=torch.float16)
    att = torch.zeros_like(q)
    y = torch.zeros((N_LAYERS, k), device="cuda", dtype=torch.float16)
    qkv = torch.zeros((N_LAYERS, (HQ + 2 * HKV) * D), device="cuda", dtype=torch.float16)
    prm = p2p_b200.Params(HQ, HKV)
    plans = None
    if not fused:
        plans = [[ctx.plan_decode_step(prm, [(qkv[l], wl.nw[l], kc, vc, att[l])], wl.rope,
                                       wl.cap, use_meta=True)
                  for l, (kc, vc) in enumerate(c)] for c in wl.copies]

    def step(i):
        ws = weights[i % sets]
        caches = wl.copies[i % len(wl.copies)]
        for l in range(N_LAYERS):
            wq, wk, wv, wo = ws[l]
            kc, vc = caches[l]
            if fused:
                ctx.qkv_gemv_prep(prm, x[l], wq, wk, wv, wl.nw[l], wl.rope, q[l], kc, vc,
                                  use_meta=True)
                ctx.attn(prm, q[l:l + 1], kc, vc, att[l:l + 1], m_tokens=1, use_meta=True)
            else:
                ctx.gemv_q4(wq, x[l], qkv[l], 0)
                ctx.gemv_q4(wk, x[l], qkv[l], HQ * D)
                ctx.gemv_q4(wv, x[l], qkv[l], (HQ + HKV) * D)
                plans[i % len(plans)][l].run()
            ctx.gemv_q4(wo, att[l], y[l])

    ms = timed_graph(step, steps, warmup, 1)
    per_layer = (q4_bytes(HQ * D, k) + 2 * q4_bytes(HKV * D, k) + q4_bytes(k, HQ * D)
                 + decode_layer_bytes(wl.past) + k * 2 * 2)
    del weights
    return ms, N_LAYERS * per_layer


def gemm_flops(m, n, k):
    return 2.0 * m * n * k


def run_qkv_gemm_calls(ctx, s, calls, resident):
    """`calls` direct calls of one LFM2.5-1.2B layer's fused q/k/v projection + QK_PREP over an
    s-token chunk (4-bit weights dequantised per call, or resident f16 copies): the command the
    profiler wraps for the GEMM kernels."""
    import torch
    import p2p_b200
    k = HQ * D
    g = torch.Generator(device="cuda").manual_seed(77)
    ws = [q4_weights(g, n, k) for n in (HQ * D, HKV * D, HKV * D)]
    w16 = torch.cat([ctx.q4_to_f16(w) for w in ws]) if resident else None
    x = torch.randn((s, k), generator=g, device="cuda").half()
    nw = torch.ones((2 * D,), device="cuda", dtype=torch.float16)
    rope = ctx.rope_table(s, D, 1e6)
    prm = p2p_b200.Params(HQ, HKV)
    q = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)
    kc = torch.zeros((s, HKV, D), device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(calls):
        if resident:
            ctx.qkv_gemm_prep_f16w(prm, x, w16, nw, rope, q, kc, vc, pos0=0)
        else:
            ctx.qkv_gemm_prep(prm, x, *ws, nw, rope, q, kc, vc, pos0=0)
    end.record()
    ctx.sync()
    return {"chunk": s, "calls": calls, "resident_f16": bool(resident),
            "us_per_call_direct_launch": start.elapsed_time(end) * 1e3 / max(calls, 1)}


def run_prefill_projections(ctx, steps, warmup, s=2048, sets=12, check=True):
    """The 4-bit projections around the attention of an s-token prompt chunk of one LFM2.5-1.2B
    layer (hidden 2048, 32q/8kv): the q/k/v projections with QK_PREP in the GEMM's epilogue
    (p2p_qkv_gemm_prep: the qkv block never reaches memory), the reference's order (three GEMMs
    into the qkv block, then QK_PREP; engine.js:202-204, :221) and the o_proj GEMM
    (engine.js:224).  Hidden rows and weights rotate over `sets` copies (12 x 12.4 MB > L2).
    The 4-bit calls dequantise their weights to f16 first (inside the timed region); the
    resident calls use f16 copies made once beforehand (p2p_q4_to_f16, as at weight upload,
    engine.js:100), rotating alike (12 x 21 MB)."""
    import numpy as np
    import torch
    import p2p_b200
    k = HQ * D
    g = torch.Generator(device="cuda").manual_seed(77)
    weights = [tuple(q4_weights(g, n, k) for n in (HQ * D, HKV * D, HKV * D, k))
               for _ in range(sets)]
    xs = [torch.randn((s, k), generator=g, device="cuda").half() for _ in range(sets)]
    nw = (1 + 0.1 * torch.randn((2 * D,), generator=g, device="cuda")).half()
    rope = ctx.rope_table(s, D, 1e6)
    prm = p2p_b200.Params(HQ, HKV)
    q = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)
    kc = torch.zeros((s, HKV, D), device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    q_u, kc_u, vc_u = torch.zeros_like(q), torch.zeros_like(kc), torch.zeros_like(vc)
    q_r, kc_r, vc_r = torch.zeros_like(q), torch.zeros_like(kc), torch.zeros_like(vc)
    resident = [(torch.cat([ctx.q4_to_f16(w) for w in ws[:3]]), ctx.q4_to_f16(ws[3]))
                for ws in weights]
    qkv = torch.zeros((s, (HQ + 2 * HKV) * D), device="cuda", dtype=torch.float16)
    y = torch.zeros((s, k), device="cuda", dtype=torch.float16)

    def fused(i):
        wq, wk, wv, _ = weights[i % sets]
        ctx.qkv_gemm_prep(prm, xs[i % sets], wq, wk, wv, nw, rope, q, kc, vc, pos0=0)

    def unfused(i):
        wq, wk, wv, _ = weights[i % sets]
        x = xs[i % sets]
        ctx.gemm_q4(wq, x, qkv, y_off=0)
        ctx.gemm_q4(wk, x, qkv, y_off=HQ * D)
        ctx.gemm_q4(wv, x, qkv, y_off=(HQ + HKV) * D)
        ctx.qk_prep(prm, qkv, nw, rope, q_u, kc_u, vc_u, pos0=0)

    def oproj(i):
        ctx.gemm_q4(weights[i % sets][3], xs[(i + 1) % sets], y)

    def fused_resident(i):
        ctx.qkv_gemm_prep_f16w(prm, xs[i % sets], resident[i % sets][0], nw, rope, q_r, kc_r,
                               vc_r, pos0=0)

    def oproj_resident(i):
        ctx.gemm_f16w(resident[i % sets][1], xs[(i + 1) % sets], y)

    def gemm_only_resident(i):  # the same projection without the QK_PREP epilogue
        ctx.gemm_f16w(resident[i % sets][0], xs[i % sets], qkv)

    att = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)

    def layer_resident(i):  # the prompt chunk's whole attention layer, fused
        fused_resident(i)
        ctx.attn(prm, q_r, kc_r, vc_r, att, pos0=0, m_tokens=s)
        ctx.gemm_f16w(resident[i % sets][1], att, y)

    def layer_reference_order(i):  # three GEMMs, QK_PREP, attention, o_proj (engine.js:202-224)
        unfused(i)
        ctx.attn(prm, q_u, kc_u, vc_u, att, pos0=0, m_tokens=s)
        ctx.gemm_q4(weights[i % sets][3], att, y)

    res = {"ms_fused": timed_graph(fused, steps, warmup, 1),
           "ms_unfused": timed_graph(unfused, steps, warmup, 1),
           "ms_oproj": timed_graph(oproj, steps, warmup, 1),
           "ms_fused_resident": timed_graph(fused_resident, steps, warmup, 1),
           "ms_oproj_resident": timed_graph(oproj_resident, steps, warmup, 1),
           "ms_gemm_only_resident": timed_graph(gemm_only_resident, steps, warmup, 1),
           "ms_layer_resident": timed_graph(layer_resident, steps, warmup, 1),
           "ms_layer_reference_order": timed_graph(layer_reference_order, steps, warmup, 1)}
    if check:
        from oracle import pyoracle as O
        fused(0)
        unfused(0)
        fused_resident(0)
        torch.cuda.synchronize()
        same = all(torch.equal(a.view(torch.int16), b.view(torch.int16))
                   for a, b in ((q, q_u), (kc, kc_u), (vc, vc_u)))
        same_resident = all(torch.equal(a.view(torch.int16), b.view(torch.int16))
                            for a, b in ((q, q_r), (kc, kc_r), (vc, vc_r)))
        # GEMM rows against the oracle's restatement of the GEMM shader, within the bound of
        # the f16 weight rounding: |err| <= 2^-10 sum_k |x_k w_k| + 1 f16 ulp
        rows = sample_rows(s)
        wq, wk, wv, _ = weights[0]
        x_h = xs[0][rows].cpu().numpy()
        want = np.zeros((len(rows), (HQ + 2 * HKV) * D), np.float16)
        bound = np.zeros(want.shape, np.float64)
        off = 0
        for w in (wq, wk, wv):
            wq_h = w[0].cpu().numpy().view(np.uint32)
            sc_h = w[1].cpu().numpy()
            zp_h = w[2].cpu().numpy().view(np.uint32)
            n = wq_h.shape[0]
            O.gemm_q4(x_h, wq_h, sc_h, zp_h, y=want, y_stride=want.shape[1], y_off=off)
            wd = O.dequant_q4(wq_h, sc_h, zp_h).astype(np.float64)
            bound[:, off:off + n] = 2.0 ** -10 * (np.abs(x_h.astype(np.float64)) @ np.abs(wd).T)
            off += n
        got = qkv[rows].cpu().numpy().astype(np.float64)
        ulp = np.spacing(np.abs(want.astype(np.float16))).astype(np.float64)
        ratio = np.abs(got - want.astype(np.float64)) / (bound + ulp)
        res["parity"] = {
            "fused_equals_unfused_bits": bool(same),
            "resident_equals_q4_bits": bool(same_resident),
            "gemm_rows_max_err_over_bound": float(f"{float(ratio.max()):.3e}"),
            "ok": bool(same and same_resident and ratio.max() <= 1.0 and np.isfinite(got).all()),
            "checked": f"{len(rows)} qkv rows x 3072 against the oracle's GEMM (bound 2^-10 "
                       "sum|x w| + 1 ulp); fused q / k / v cache rows bit-equal to GEMM x3 + "
                       "QK_PREP on the GPU"}
    del weights, xs, resident
    return res


def e2e_decode(wl, steps, warmup):
    """The user-facing per-token call with host buffers: p2p_decode_step whose 6 qkv rows and 6
    output rows live in page-locked host memory, so the kernel itself reads the step's inputs
    from the host and writes its outputs back (no separate copy); the host then waits for the
    result."""
    import torch
    stream = torch.cuda.current_stream()
    h_in = torch.randn(wl.qkv.shape, dtype=torch.float16).pin_memory()
    h_out = torch.empty(wl.out.shape, dtype=torch.float16).pin_memory()
    plans = [wl.ctx.plan_decode_step(wl.prm, [(h_in[l], wl.nw[l], kc, vc, h_out[l])
                                              for l, (kc, vc) in enumerate(c)],
                                     wl.rope, wl.cap, use_meta=True)
             for c in wl.copies]

    def one(i):
        plans[i % len(plans)].run()
        stream.synchronize()

    for i in range(warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(steps):
        one(warmup + i)
    dt = (time.perf_counter() - t0) / steps
    return dt, h_in.numel() * 2, h_out.numel() * 2


def e2e_native(device, steps, warmup, world, graph=True):
    """The same per-token call from a plain C host (p2p_b200/host/p2p_decode_loop: the C ABI
    alone, no Python or torch, as a native engine binding calls it), one process per GPU, all
    ranks at once.  graph: the binding records each cache copy's p2p_decode_step once as a
    CUDA graph and replays it per token (the kernel reads the token's qkv rows from and writes
    its outputs to page-locked host memory on every replay); otherwise it calls the C ABI per
    token.  Returns (seconds per step, h2d bytes, d2h bytes, finite)."""
    exe = ROOT / "p2p_b200" / "host" / "p2p_decode_loop"
    if not exe.exists():
        raise RuntimeError(f"{exe} is missing: build with python p2p_b200/build.py")
    barrier(world)
    r = subprocess.run([str(exe), "--device", str(device), "--steps", str(steps),
                        "--warmup", str(warmup), "--copies", "12", "--past", str(PAST),
                        "--graph", "1" if graph else "0"],
                       capture_output=True, text=True, timeout=600)
    barrier(world)
    if r.returncode != 0:
        raise RuntimeError(f"p2p_decode_loop failed ({r.returncode}): {r.stderr[-300:]}")
    j = json.loads(r.stdout.strip().splitlines()[-1])
    return (j["us_per_step"] * 1e-6, j["h2d_bytes_per_step"], j["d2h_bytes_per_step"],
            j["outputs_finite"])


def ragged_lengths(nseq=256, lo=1024, hi=32768, seed=4):
    import numpy as np
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, nseq).astype(np.int64)


def lpt_shard(lengths, world):
    from p2p_b200.sharding import lpt_partition
    return lpt_partition([int(x) + 1 for x in lengths], world)


RAGGED_BLOCK = 64  # tokens per page of the paged leg


def run_ragged(ctx, rank, world, steps, warmup, check=True, fmt="f16", nseq_total=256):
    """The 256-sequence batched decode (this rank's LPT share) with the KV cache in format
    `fmt`: "f16" rows at per-sequence offsets (the engine's layout), "int8" rows with
    per-channel scales (half the bytes), or "paged" f16 pages of RAGGED_BLOCK tokens in a
    shuffled pool with a block table.  Returns (ms per step, algorithmic bytes, parity)."""
    import numpy as np
    import torch
    import p2p_b200
    past_all = ragged_lengths()[:nseq_total]
    mine = lpt_shard(past_all, world)[rank]
    past = past_all[mine].astype(np.int32)
    rows = past + 1
    offsets = np.zeros(len(past), np.int64)
    offsets[1:] = np.cumsum(rows[:-1])
    total_rows = int(rows.sum())
    if total_rows >= 2**31:
        raise RuntimeError("ragged cache too large for int32 offsets")
    nseq = len(past)
    max_past = int(past_all.max())
    g = torch.Generator(device="cuda").manual_seed(77 + rank)
    table = None
    ks = vs = None
    if fmt == "paged":
        nblk = (rows + RAGGED_BLOCK - 1) // RAGGED_BLOCK
        n_pages = int(nblk.sum())
        perm = np.random.default_rng(5 + rank).permutation(n_pages).astype(np.int32)
        # as wide as max_past needs (the entry point checks max_past against max_blocks); on
        # a rank whose longest sequence is shorter the extra entries stay -1 (never read)
        table = np.full((nseq, max_past // RAGGED_BLOCK + 1), -1, np.int32)
        start = np.concatenate([[0], np.cumsum(nblk)[:-1]])
        for i in range(nseq):
            table[i, :nblk[i]] = perm[start[i]:start[i] + nblk[i]]
        shape = (n_pages, RAGGED_BLOCK, HKV, D)
    else:
        shape = (total_rows, HKV, D)
    kc = torch.randn(shape, generator=g, device="cuda", dtype=torch.float16)
    vc = torch.randn(shape, generator=g, device="cuda", dtype=torch.float16)
    if fmt == "int8":
        ks = (0.02 + 0.02 * torch.rand((HKV * D,), generator=g, device="cuda")).float()
        vs = (0.02 + 0.02 * torch.rand((HKV * D,), generator=g, device="cuda")).float()
        kc, vc = ctx.kv_quantize_q8(kc, ks), ctx.kv_quantize_q8(vc, vs)
        torch.cuda.synchronize()
    qkv = torch.randn((nseq, (HQ + 2 * HKV) * D), generator=g, device="cuda",
                      dtype=torch.float16)
    nw = (1 + 0.1 * torch.randn((2 * D,), generator=g, device="cuda")).half()
    out = torch.zeros((nseq, HQ * D), device="cuda", dtype=torch.float16)
    rope = ctx.rope_table(max_past + 1, D, 1e6)
    off_d = torch.from_numpy(offsets.astype(np.int32)).cuda()
    past_d = torch.from_numpy(past).cuda()
    tbl_d = torch.from_numpy(table).cuda() if table is not None else None
    prm = p2p_b200.Params(HQ, HKV)

    def step(i):
        if fmt == "f16":
            ctx.attn_decode_ragged(prm, qkv, nw, rope, kc, vc, off_d, past_d, out,
                                   max_past=max_past, fused_prep=True)
        else:
            ctx.attn_decode_kv(prm, qkv, nw, rope, kc, vc, past_d, out, max_past=max_past,
                               offsets=off_d if fmt == "int8" else None, k_scale=ks,
                               v_scale=vs, block_table=tbl_d, fused_prep=True)

    ms = timed_graph(step, steps, warmup, world)
    row_bytes = HKV * D * (1 if fmt == "int8" else 2)
    my_bytes = float(rows.sum() * row_bytes * 2 + nseq * ((HQ + 2 * HKV) * D * 2
                                                          + 2 * row_bytes + HQ * D * 2))
    if not check:
        del kc, vc
        torch.cuda.empty_cache()
        return ms, my_bytes, None
    # the checker: this rank's shortest, longest and two more sequences against the oracle
    from oracle import pyoracle as O
    ctx.sync()
    got = out.cpu().numpy()
    rope_h = O.rope_table(max_past + 1)
    qkv_h, nw_h = qkv.cpu().numpy(), nw.cpu().numpy()
    sample = sorted({int(np.argmin(past)), int(np.argmax(past)), 0, nseq // 2})
    want = np.zeros((len(sample), HQ * D), np.float16)
    for j, i in enumerate(sample):
        n = int(past[i]) + 1
        if fmt == "paged":  # the sequence's pages, gathered (the new k/v included)
            k_i = O.gather_pages(kc[tbl_d[i].clamp(min=0).long()].cpu().numpy(),
                                 np.arange(table.shape[1], dtype=np.int32), n)
            v_i = O.gather_pages(vc[tbl_d[i].clamp(min=0).long()].cpu().numpy(),
                                 np.arange(table.shape[1], dtype=np.int32), n)
        else:
            sl = slice(int(offsets[i]), int(offsets[i]) + n)
            k_i, v_i = kc[sl].cpu().numpy(), vc[sl].cpu().numpy()
        q_o = np.zeros((1, HQ * D), np.float16)
        if fmt == "int8":  # q as QK_PREP rotates it; the int8 rows already hold the new k/v
            k_scr = np.zeros((n, HKV, D), np.float16)
            O.qk_prep(HQ, HKV, D, qkv_h[i:i + 1], nw_h, rope_h, q_o, k_scr, k_scr.copy(),
                      n - 1, 1)
            O.attn_ragged_q8(HQ, HKV, D, q_o, k_i, v_i, ks.cpu().numpy(), vs.cpu().numpy(),
                             np.zeros(1, np.int64), past[i:i + 1], want[j:j + 1])
        else:
            O.qk_prep(HQ, HKV, D, qkv_h[i:i + 1], nw_h, rope_h, q_o, k_i, v_i, n - 1, 1)
            O.attn(HQ, HKV, D, q_o, k_i, v_i, want[j:j + 1], n - 1, 1)
    par = parity_stats(got[sample], want, f"{len(sample)} sequences (shortest, longest, 2 more) "
                                          f"vs the oracle")
    del kc, vc
    torch.cuda.empty_cache()
    return ms, my_bytes, par


def prefill_inputs(s, seed=33, scale=0.5):
    """The config's prompt: qkv rows [s][3072] ~ scale * N(0,1) (same on every rank)."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (scale * torch.randn((s, (HQ + 2 * HKV) * D), generator=g, device="cuda")).half()


def prefill_oracle_rows(qkv, rows, what):
    """The checker's reference for query rows `rows` of a causal prefill of all heads from
    position 0: the oracle's QK_PREP on the whole prompt, then its ATTN on those rows."""
    import numpy as np
    from oracle import pyoracle as O
    qkv_h = qkv.cpu().numpy()
    s = qkv_h.shape[0]
    rope = O.rope_table(s)
    q = np.zeros((s, HQ * D), np.float16)
    kc = np.zeros((s, HKV, D), np.float16)
    vc = np.zeros_like(kc)
    O.qk_prep(HQ, HKV, D, qkv_h, None, rope, q, kc, vc, 0, s)
    want = np.zeros((len(rows), HQ * D), np.float16)
    for j, r in enumerate(rows):
        O.attn(HQ, HKV, D, q[r:r + 1], kc, vc, want[j:j + 1], int(r), 1)
    return want


def sample_rows(s):
    return sorted({0, 1, 2, 127, 128, s // 2, s - 129, s - 2, s - 1})


def run_prefill(ctx, steps, warmup, s=2048, copies=4, check=True):
    """Causal prefill of an s-token prompt on one GPU, all 32 q heads: attention alone (q and
    the cache rotated beforehand) and QK_PREP + attention (the config's step, cache write
    included); graph-timed and with direct launches."""
    import numpy as np
    import torch
    import p2p_b200
    prm = p2p_b200.Params(HQ, HKV)
    rope = ctx.rope_table(s, D, 1e6)
    qkv = [prefill_inputs(s, 33 + i) for i in range(copies)]
    q = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)
    kc = torch.zeros((s, HKV, D), device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    out = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)
    stream = torch.cuda.current_stream()
    for i in range(copies):  # QK_PREP writes the cache layout used by decode
        ctx.qk_prep(prm, qkv[i], None, rope, q, kc, vc, pos0=0, m_tokens=s)

    def attn_only(i):
        ctx.attn(prm, q, kc, vc, out, pos0=0, m_tokens=s)

    def prep_and_attn(i):
        ctx.qk_prep(prm, qkv[i % copies], None, rope, q, kc, vc, pos0=0, m_tokens=s)
        ctx.attn(prm, q, kc, vc, out, pos0=0, m_tokens=s)

    res = {"ms_attn": timed_graph(attn_only, steps, warmup, 1),
           "ms_both": timed_graph(prep_and_attn, steps, warmup, 1),
           "ms_both_direct": timed_loop(prep_and_attn, steps, warmup, 1, stream)}
    if check:
        prep_and_attn(0)
        torch.cuda.synchronize()
        rows = sample_rows(s)
        want = prefill_oracle_rows(qkv[0], rows, "")
        res["parity"] = parity_stats(out.cpu().numpy()[rows], want,
                                     f"{len(rows)} query rows x {HQ} heads vs the oracle")
    return res


def sharded_prefill_leg(ctx, comm, rank, world, s, variant, steps, warmup):
    """Causal prefill of an s-token prompt split by KV-head group over the ranks, one variant
    of the output assembly, inside the timed region (captured in one CUDA graph with its
    collectives).  Afterwards the checker compares this rank's full [s][2048] output with all
    heads computed on this one GPU, and a sample of rows with the oracle."""
    import numpy as np
    import torch
    import p2p_b200
    from p2p_b200.sharding import (HeadShardedPrefill, MulticastHeadShardedPrefill,
                                   ScatterHeadShardedPrefill)
    cls = {"allgather": HeadShardedPrefill, "scatter": ScatterHeadShardedPrefill,
           "multicast": MulticastHeadShardedPrefill}[variant]
    kw = {} if variant == "allgather" else {"max_tokens": s}
    sp = cls(ctx, HQ, HKV, world, rank, comm=comm, **kw)
    qkv_full = prefill_inputs(s)
    qkv_l = qkv_full[:, sp.local_qkv_columns().cuda()].contiguous()
    rope = ctx.rope_table(s, D, 1e6)
    kc = torch.zeros((s, sp.kvn, D), device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    q_buf = torch.zeros((s, sp.qn * D), device="cuda", dtype=torch.float16)
    out = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)

    def step(i):
        if variant == "allgather":
            sp(qkv_l, None, rope, kc, vc, out, 0, s)
        else:
            sp(qkv_l, None, rope, kc, vc, q_buf, 0, s)

    try:
        ms = timed_graph(step, steps, warmup, world, capture_error_mode="relaxed")
        timing = "graph"
    except RuntimeError:  # capture refused: the same steps as direct launches
        torch.cuda.synchronize()
        ms = timed_loop(step, steps, warmup, world, torch.cuda.current_stream())
        timing = "direct"
    step(0)
    comm.wait()
    got = (out if variant == "allgather" else sp.out_full[:s]).clone()
    # all heads on this GPU (the 1-GPU path the tests pin to the oracle)
    prm = p2p_b200.Params(HQ, HKV)
    q1 = torch.zeros((s, HQ * D), device="cuda", dtype=torch.float16)
    k1 = torch.zeros((s, HKV, D), device="cuda", dtype=torch.float16)
    v1 = torch.zeros_like(k1)
    want1 = torch.zeros_like(q1)
    ctx.qk_prep(prm, qkv_full, None, rope, q1, k1, v1, pos0=0, m_tokens=s)
    ctx.attn(prm, q1, k1, v1, want1, pos0=0, m_tokens=s)
    torch.cuda.synchronize()
    same = bool(torch.equal(got, want1))
    rows = sample_rows(s)
    par = parity_stats(got.cpu().numpy()[rows], prefill_oracle_rows(qkv_full, rows, ""),
                       f"{len(rows)} query rows x {HQ} heads vs the oracle, and the whole "
                       f"[{s}][{HQ * D}] output vs all heads on one GPU")
    sp.close()
    del sp
    return ms, timing, par, same


def vision_oracle_check(q, k, v, out, images, what):
    import numpy as np
    from oracle import pyoracle as O
    want, got = [], []
    for b in images:
        w = np.zeros((1, 1024, 12 * D), np.float16)
        O.vision_attn(12, D, q[b:b + 1].cpu().numpy(), k[b:b + 1].cpu().numpy(),
                      v[b:b + 1].cpu().numpy(), w)
        want.append(w[0])
        got.append(out[b].cpu().numpy())
    return parity_stats(np.stack(got), np.stack(want), what)


def run_vision_split(ctx, rank, world, steps, warmup):
    """The vision batch split by image over the ranks (no collective)."""
    import torch
    import p2p_b200
    from p2p_b200.sharding import split_images
    b0, nb = split_images(16, world, rank)
    g = torch.Generator(device="cuda").manual_seed(55 + rank)
    q, k, v = ((0.5 * torch.randn((max(nb, 1), 1024, 768), generator=g, device="cuda")).half()
               for _ in range(3))
    out = torch.zeros_like(q)
    prm = p2p_b200.Params(12, 12)

    def step(i):
        if nb:
            ctx.attn_bidir(prm, q, k, v, out)

    ms = timed_graph(step, steps, warmup, world)
    torch.cuda.synchronize()
    par = vision_oracle_check(q, k, v, out, sorted({0, max(nb, 1) - 1}),
                              "first and last image of each rank (all 12 heads) vs the oracle")
    return ms, par


def run_vision(ctx, steps, warmup, check=True):
    import torch
    import p2p_b200
    b, s, nh = 16, 1024, 12
    g = torch.Generator(device="cuda").manual_seed(55)
    prm = p2p_b200.Params(nh, nh)
    q, k, v = ((0.5 * torch.randn((b, s, nh * D), generator=g, device="cuda")).half()
               for _ in range(3))
    out = torch.zeros_like(q)

    def step(i):
        ctx.attn_bidir(prm, q, k, v, out)

    ms = timed_graph(step, steps, warmup, 1)
    torch.cuda.synchronize()
    if not check:
        return ms, None
    par = vision_oracle_check(q, k, v, out, [0, 7, 15], "images 0, 7, 15 (all 12 heads) vs "
                                                        "the oracle")
    return ms, par


# ---------------------------------------------------------------------------------------------
# CPU legs (the oracle only runs here, as the checker/baseline)

def cpu_reference_step_seconds(kind: str, n_steps: int = 0, warmup: int = 1,
                               n_layers: int = N_LAYERS, seconds: float = 3.0):
    """One decode step of the headline workload on host cores.  kind 'reference' runs the
    reference's own QK_PREP/ATTN shaders (oracle/_ref) dispatched as engine.js does: their
    16-head shape is applied to the 32/8 layer as two dispatches over the q-head pairs that
    share a kv head (h = 4k, 4k+1 and 4k+2, 4k+3), which is the same per-(head, token)
    arithmetic.  kind 'port' runs the oracle restatement at 32/8 directly."""
    import numpy as np
    from oracle import pyoracle as O
    threads = O.set_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    cap = PAST + 1
    rope = O.rope_table(cap)
    layers = []
    for _ in range(n_layers):
        kc = rng.standard_normal((cap, HKV, D)).astype(np.float16)
        vc = rng.standard_normal((cap, HKV, D)).astype(np.float16)
        qkv = rng.standard_normal((1, (HQ + 2 * HKV) * D)).astype(np.float16)
        nw = (1 + 0.1 * rng.standard_normal(2 * D)).astype(np.float16)
        layers.append((qkv, nw, kc, vc))
    meta = np.array([PAST, 1, 0, 0], np.uint32)
    halves = [np.array([4 * k + r for k in range(HKV) for r in (0, 1)]),
              np.array([4 * k + r for k in range(HKV) for r in (2, 3)])]

    def step():
        for qkv, nw, kc, vc in layers:
            if kind == "reference":
                q16 = qkv[0, :HQ * D].reshape(HQ, D)
                kv = qkv[0, HQ * D:]
                out32 = np.zeros((HQ, D), np.float16)
                for hs in halves:
                    row = np.ascontiguousarray(np.concatenate([q16[hs].reshape(-1), kv])[None])
                    qo = np.zeros((1, 1024), np.float16)
                    O.ref_qk_prep(row, nw, qo, kc, vc, meta, rope, 1)
                    oo = np.zeros((1, 1024), np.float16)
                    O.ref_attn(qo, kc, vc, oo, meta, 1)
                    out32[hs] = oo.reshape(16, D)
            else:
                q = np.zeros((1, HQ * D), np.float16)
                O.qk_prep(HQ, HKV, D, qkv, nw, rope, q, kc, vc, PAST, 1)
                out = np.zeros((1, HQ * D), np.float16)
                O.attn(HQ, HKV, D, q, kc, vc, out, PAST, 1)

    for _ in range(max(warmup, 0)):
        step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        if (n_steps and n >= n_steps) or (not n_steps and (time.perf_counter() - t0 > seconds
                                                           or n >= 50)):
            break
    return (time.perf_counter() - t0) / n, threads, n


def cpu_kind():
    from oracle import pyoracle as O
    return "reference" if O.ref_available() else "port"


def reference_arm(args):
    """The reference's own CPU implementation of the path (oracle/_ref when it was built from
    the reference sources, else the oracle restatement), all host threads, same metric and
    workload.  Each bench step is one whole decode step (6 layers); if K steps would take more
    than ~150 s the steps are cut to fewer layers and the bytes counted accordingly."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    kind = cpu_kind()
    sec1, threads, _ = cpu_reference_step_seconds(kind, n_steps=1)
    budget = 150.0
    layers = N_LAYERS
    if sec1 * (args.steps + min(args.warmup, 3)) > budget:
        layers = max(1, int(N_LAYERS * budget / (sec1 * (args.steps + min(args.warmup, 3)))))
    sec, threads, n = cpu_reference_step_seconds(kind, n_steps=args.steps,
                                                 warmup=min(args.warmup, 3), n_layers=layers)
    bytes_step = layers * decode_layer_bytes()
    gbs = bytes_step / sec / 1e9
    sample = (f"{n} timed steps of {layers} of the 6 layers (32 heads x 4097 keys each), "
              f"{min(args.warmup, 3)} untimed")
    line = {
        "impl": "reference", "metric": "decode_attn_gbs_ctx4096", "value": round(gbs, 4),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3 * N_LAYERS / layers, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "lfm2.5-1.2b decode attention, ctx 4096+1, 6 layers, 32q/8kv, d64",
                   "past": PAST, "layers": N_LAYERS},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_only(ctx, args):
    """One leg, one GPU, minimal setup: the commands the profiler wraps."""
    import torch
    if args.only == "decode":
        wl = DecodeWorkload(ctx, 0, copies=4, past=args.past)
        ms = timed_graph(wl.step, args.steps, args.warmup, 1)
        res = {"us_per_step": ms * 1e3, "gbs": wl.bytes_per_step / (ms * 1e-3) / 1e9,
               "stream_same_bytes_us": stream_reference(ctx, wl.bytes_per_step, args.steps,
                                                        args.warmup, 1, copies=4)[0]}
    elif args.only == "decode1":
        wl = DecodeWorkload(ctx, 0, copies=12, past=args.past)
        ms = timed_graph(wl.step_one_layer, args.steps, args.warmup, 1)
        b = wl.bytes_per_step / N_LAYERS
        res = {"us_per_step": ms * 1e3, "gbs": b / (ms * 1e-3) / 1e9,
               "stream_same_bytes_us": stream_reference(ctx, b, args.steps, args.warmup, 1)[0]}
    elif args.only == "ragged":
        ms, b, _ = run_ragged(ctx, 0, 1, args.steps, args.warmup, check=False, fmt=args.kv,
                              nseq_total=args.ragged_seqs)
        res = {"ms_per_step": ms, "gbs": b / (ms * 1e-3) / 1e9}
    elif args.only == "block":
        wl = DecodeWorkload(ctx, 0, copies=12, past=args.past)
        res = {}
        for fused in (True, False):
            ms, b = run_decode_block(ctx, wl, args.steps, args.warmup, fused=fused)
            res["fused" if fused else "unfused"] = {"us_per_layer": ms * 1e3 / N_LAYERS,
                                                    "gbs": b / (ms * 1e-3) / 1e9}
    elif args.only == "prefill":
        r = run_prefill(ctx, args.steps, args.warmup, s=args.prefill_s, check=False)
        fl = prefill_flops(args.prefill_s)
        res = {"us_attn": r["ms_attn"] * 1e3, "tflops_attn": fl / (r["ms_attn"] * 1e-3) / 1e12,
               "us_prep_plus_attn": r["ms_both"] * 1e3}
    elif args.only == "qkvgemm":
        res = run_qkv_gemm_calls(ctx, args.prefill_s, args.steps, args.resident)
    elif args.only == "projections":
        r = run_prefill_projections(ctx, args.steps, args.warmup, s=args.prefill_s,
                                    check=args.check)
        res = {"us_qkv_fused": r["ms_fused"] * 1e3, "us_qkv_unfused": r["ms_unfused"] * 1e3,
               "us_oproj": r["ms_oproj"] * 1e3,
               "us_qkv_fused_resident_f16": r["ms_fused_resident"] * 1e3,
               "us_oproj_resident_f16": r["ms_oproj_resident"] * 1e3,
               "us_qkv_gemm_only_resident_f16": r["ms_gemm_only_resident"] * 1e3,
               "us_attention_layer_resident_f16": r["ms_layer_resident"] * 1e3,
               "us_attention_layer_reference_order": r["ms_layer_reference_order"] * 1e3,
               "tflops_qkv_fused": gemm_flops(args.prefill_s, (HQ + 2 * HKV) * D, HQ * D)
               / (r["ms_fused"] * 1e-3) / 1e12, **({"parity": r["parity"]} if args.check else {})}
    else:
        va, _ = run_vision(ctx, args.steps, args.warmup, check=False)
        res = {"us": va * 1e3, "tflops": vision_flops() / (va * 1e-3) / 1e12}
    print(json.dumps({"only": args.only, **res}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-side", action="store_true", help="skip prefill/vision/ragged legs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--only", choices=["decode", "decode1", "ragged", "prefill", "vision", "block",
                                       "projections", "qkvgemm"],
                    help="run one leg on one GPU and print its timing (profiling commands)")
    ap.add_argument("--past", type=int, default=PAST, help="decode context for --only decode")
    ap.add_argument("--prefill-s", type=int, default=2048, help="prompt length for --only prefill")
    ap.add_argument("--resident", action="store_true",
                    help="with --only qkvgemm: resident f16 weights instead of 4-bit per call")
    ap.add_argument("--check", action="store_true",
                    help="with --only projections: also run the leg's output checks")
    ap.add_argument("--kv", default="f16", choices=["f16", "int8", "paged"],
                    help="KV-cache format for --only ragged")
    ap.add_argument("--ragged-seqs", type=int, default=256,
                    help="sequences of the batch for --only ragged (a smaller case to profile)")
    ap.add_argument("--quick", action="store_true",
                    help="headline kernel only (no e2e, side legs, CPU leg or clock tail); "
                         "the profiling command")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    rank, world, local = dist_setup(args.gpus)
    import p2p_b200
    ctx = p2p_b200.Context(local)
    if args.only:
        run_only(ctx, args)
        ctx.close()
        return
    stream = torch.cuda.current_stream()
    hbm_peak, tensor_peak, peak_kind = load_peaks()
    traffic = load_traffic()

    wl = DecodeWorkload(ctx, rank)
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    gpu_index = int(phys[local]) if phys and phys[0] not in ("",) and phys[local].isdigit() else local
    if args.quick:
        args.no_side = args.no_cpu = True
    with ClockSampler(gpu_index) as clk:
        ms = timed_graph(wl.step, args.steps, args.warmup, world)
        ms_direct = timed_loop(wl.step, args.steps, args.warmup, world, stream)
        # keep the same kernel under load ~1.5 s so the 200 ms clock sampler sees the timed state
        t_end = time.perf_counter() + (0.0 if args.quick else 1.5)
        i = 0
        while time.perf_counter() < t_end:
            for _ in range(200):
                wl.step(i)
                i += 1
            torch.cuda.synchronize()
    clocks = clk.summary()
    ms_max = max_over_ranks(ms, world)
    total_bytes = wl.bytes_per_step * world
    value_gbs = total_bytes / (ms_max * 1e-3) / 1e9
    per_gpu_gbs = wl.bytes_per_step / (ms_max * 1e-3) / 1e9

    e2e_note = ("plain C host over the C ABI (p2p_b200/host/p2p_decode_loop), wall clock; "
                "each cache copy's p2p_decode_step recorded once as a CUDA graph and replayed "
                "per token, the kernel reading and writing the host rows")
    direct_sec = float("nan")
    if args.quick:
        e2e_sec, h2d, d2h, py_sec = float("nan"), 0, 0, float("nan")
    else:
        try:
            e2e_sec, h2d, d2h, finite = e2e_native(local, max(50, args.steps), args.warmup,
                                                   world)
            direct_sec, _, _, finite_d = e2e_native(local, max(50, args.steps), args.warmup,
                                                    world, graph=False)
            if not (finite and finite_d):
                e2e_note += "; NON-FINITE OUTPUT"
        except (RuntimeError, subprocess.TimeoutExpired, ValueError) as e:
            e2e_sec, h2d, d2h = float("nan"), 0, 0
            e2e_note = f"native host program failed: {str(e)[:160]}"
        py_sec, _, _ = e2e_decode(wl, max(20, args.steps // 2), args.warmup)
    e2e_sec = max_over_ranks(e2e_sec, world)
    direct_sec = max_over_ranks(direct_sec, world)
    py_sec = max_over_ranks(py_sec, world)
    e2e_gbs = total_bytes / e2e_sec / 1e9

    # the headline's output against the oracle (after its timed region); every rank checks
    parity = reduce_parity(wl.check(), world) if not args.quick else None

    # speed of light of the same bytes read by one plain streaming launch, timed the same way
    sol_us, _ = stream_reference(ctx, wl.bytes_per_step, args.steps, args.warmup, world)

    side = {}
    if not args.no_side:
        # the drop-in per-layer call: one p2p_decode_step with one layer (8.4 MB)
        ms1 = max_over_ranks(timed_graph(wl.step_one_layer, args.steps, args.warmup, world),
                             world)
        b1 = wl.bytes_per_step / N_LAYERS
        sol1_us, _ = stream_reference(ctx, b1, args.steps, args.warmup, world)
        side["decode_one_layer"] = {
            "workload": "one attention layer per call (what engine.js:245-259 dispatches "
                        "between that layer's GEMMs), ctx 4096+1, 32q/8kv, rotating over 72 "
                        "layer caches (605 MB > L2)",
            "gbs_per_gpu": round(b1 / (ms1 * 1e-3) / 1e9, 1), "us_per_step": round(ms1 * 1e3, 3),
            "hbm_frac_of_measured": round(b1 / (ms1 * 1e-3) / 1e9 / hbm_peak, 4),
            "stream_same_bytes_us": round(sol1_us, 3),
            "frac_of_stream": round(sol1_us / (ms1 * 1e3), 4)}
        for fused in (True, False):
            key = "decode_layers_with_projections" + ("" if fused else "_unfused")
            try:
                b_ms, b_bytes = run_decode_block(ctx, wl, steps=20, warmup=3, fused=fused)
                b_ms = max_over_ranks(b_ms, world)
                side[key] = {
                    "workload": "6 LFM2.5-1.2B attention layers of a decode step at ctx 4096 "
                                "with their 4-bit q/k/v and o_proj GEMVs (hidden 2048): " +
                                ("QK_PREP fused into the q/k/v projection's epilogue, then "
                                 "attention and o_proj (3 launches per layer)" if fused else
                                 "three GEMVs into the qkv row, QK_PREP + attention, o_proj "
                                 "(5 launches per layer, the reference's order)"),
                    "us_per_step": round(b_ms * 1e3, 2),
                    "us_per_layer": round(b_ms * 1e3 / N_LAYERS, 2),
                    "gbs_per_gpu": round(b_bytes / (b_ms * 1e-3) / 1e9, 1),
                    "bytes_per_step": int(b_bytes)}
            except p2p_b200.P2PError as e:
                side[key] = {"error": str(e)}
        try:
            r_ms, r_bytes, r_par = run_ragged(ctx, rank, world, steps=10, warmup=3)
            r_ms = max_over_ranks(r_ms, world)
            r_bytes = sum_over_ranks(r_bytes, world)
            side["ragged_decode"] = {
                "workload": "256 seqs, past ~ U[1024, 32768] (seed 4), 32q/8kv, fused prep, "
                            "LPT-sharded by tokens across ranks",
                "gbs": round(r_bytes / (r_ms * 1e-3) / 1e9, 1), "ms_per_step": round(r_ms, 4),
                "bytes_per_step": int(r_bytes), "hbm_frac_per_gpu_of_measured":
                    round(r_bytes / world / (r_ms * 1e-3) / 1e9 / hbm_peak, 4),
                "parity": reduce_parity(r_par, world)}
        except p2p_b200.P2PError as e:
            side["ragged_decode"] = {"error": str(e)}
        f16_ms = side.get("ragged_decode", {}).get("ms_per_step")
        for fmt, what in (("int8", "int8 KV cache, per-channel f32 scales (half the bytes)"),
                          ("paged", f"paged f16 KV cache, {RAGGED_BLOCK}-token pages in a "
                                    f"shuffled pool + block table")):
            try:
                r_ms, r_bytes, r_par = run_ragged(ctx, rank, world, steps=10, warmup=3, fmt=fmt)
                r_ms = max_over_ranks(r_ms, world)
                r_bytes = sum_over_ranks(r_bytes, world)
                side[f"ragged_decode_{fmt}"] = {
                    "workload": f"the 256-sequence batched decode with an {what}",
                    "gbs": round(r_bytes / (r_ms * 1e-3) / 1e9, 1),
                    "ms_per_step": round(r_ms, 4), "bytes_per_step": int(r_bytes),
                    "hbm_frac_per_gpu_of_measured":
                        round(r_bytes / world / (r_ms * 1e-3) / 1e9 / hbm_peak, 4),
                    "speedup_vs_f16_rows": round(f16_ms / r_ms, 3) if f16_ms else None,
                    "parity": reduce_parity(r_par, world)}
            except p2p_b200.P2PError as e:
                side[f"ragged_decode_{fmt}"] = {"error": str(e)}
        if world > 1:
            from p2p_b200.comm import Comm
            comm = Comm.from_process_group(ctx, world, rank)
            what = {"allgather": "NCCL all-gather inside the library (p2p_attn_prefill_sharded) "
                                 "+ [S][2048] assembly",
                    "scatter": "flash epilogue writes every rank's [S][2048] output over NVLink "
                               "(CUDA IPC), then one ordering all-reduce",
                    "multicast": "flash epilogue stores every row once as NVLink multicast "
                                 "(NVSwitch writes every rank's output), then one ordering "
                                 "all-reduce"}
            for s_tok in (2048, 4096, 8192, 16384):
                fl = prefill_flops(s_tok)
                # the crossover sizes (4096, 8192) with the two assemblies that need no multicast
                variants = (("allgather", "scatter", "multicast") if s_tok in (2048, 16384)
                            else ("allgather", "scatter"))
                for variant in variants:
                    key = f"prefill_head_{variant}_s{s_tok}"
                    try:
                        ms, timing, par, same = sharded_prefill_leg(ctx, comm, rank, world,
                                                                    s_tok, variant, 10, 3)
                    except RuntimeError as e:  # same on every rank: no collective was entered
                        side[key] = {"unavailable": str(e).splitlines()[0][:200]}
                        continue
                    ms = max_over_ranks(ms, world)
                    par = reduce_parity(par, world)
                    par["equal_to_one_gpu"] = max_over_ranks(0.0 if same else 1.0, world) == 0
                    par["ok"] = par["ok"] and par["equal_to_one_gpu"]
                    side[key] = {
                        "workload": f"causal prefill S={s_tok} (QK_PREP + attention), 32q/8kv "
                                    f"split by kv-head group over {world} GPUs, {what[variant]}",
                        "tflops": round(fl / (ms * 1e-3) / 1e12, 1), "us": round(ms * 1e3, 2),
                        "timing": timing, "parity": par}
            comm.close()
            v_ms, v_par = run_vision_split(ctx, rank, world, 10, 3)
            ms = max_over_ranks(v_ms, world)
            side["vision_image_split"] = {
                "workload": f"vision B=16 S=1024 12 heads split by image over {world} GPUs",
                "tflops": round(vision_flops() / (ms * 1e-3) / 1e12, 1), "us": round(ms * 1e3, 2),
                "parity": reduce_parity(v_par, world)}
        if world == 1:
            # 4096 and 8192: the one-GPU side of the sharded prefill's crossover
            for s_tok, steps in ((2048, 20), (4096, 10), (8192, 10), (16384, 5)):
                key = "prefill" if s_tok == 2048 else f"prefill_s{s_tok}"
                try:
                    r = run_prefill(ctx, steps=steps, warmup=5 if s_tok == 2048 else 3,
                                    s=s_tok, copies=4 if s_tok <= 4096 else 1)
                    fl = prefill_flops(s_tok)
                    pa, pb = r["ms_attn"], r["ms_both"]
                    side[key] = {
                        "workload": f"causal prefill S={s_tok}, 32q/8kv, d64, fp16, one GPU",
                        "tflops_attn": round(fl / (pa * 1e-3) / 1e12, 1),
                        "us_attn": round(pa * 1e3, 2),
                        "tflops_prep_plus_attn": round(fl / (pb * 1e-3) / 1e12, 1),
                        "us_prep_plus_attn": round(pb * 1e3, 2),
                        "us_prep_plus_attn_direct_launch": round(r["ms_both_direct"] * 1e3, 2),
                        "tensor_frac_of_measured": round(fl / (pa * 1e-3) / 1e12 / tensor_peak,
                                                         4),
                        "parity": reduce_parity(r["parity"], 1)}
                except p2p_b200.P2PError as e:
                    side[key] = {"error": str(e)}
            # 2048: the whole prompt as one chunk; 256: the reference engine's chunk
            # (engine.js:80, :384-401)
            for s_tok in (2048, 256):
                key = "prefill_projections" + ("" if s_tok == 2048 else f"_chunk{s_tok}")
                try:
                    r = run_prefill_projections(ctx, steps=20, warmup=5, s=s_tok)
                    fl_qkv = gemm_flops(s_tok, (HQ + 2 * HKV) * D, HQ * D)
                    fl_o = gemm_flops(s_tok, HQ * D, HQ * D)
                    pf, pu, po = r["ms_fused"], r["ms_unfused"], r["ms_oproj"]
                    side[key] = {
                        "workload": f"4-bit q/k/v projections + QK_PREP and o_proj of a "
                                    f"{s_tok}-token prompt chunk, one LFM2.5-1.2B layer (hidden "
                                    "2048, 32q/8kv); 4-bit weights dequantised to f16 in every "
                                    "call, and resident f16 copies made once; 12 rotating sets "
                                    "of hidden rows and weights",
                        "us_qkv_fused": round(pf * 1e3, 2),
                        "us_qkv_unfused": round(pu * 1e3, 2),
                        "us_oproj": round(po * 1e3, 2),
                        "us_qkv_fused_resident_f16": round(r["ms_fused_resident"] * 1e3, 2),
                        "us_oproj_resident_f16": round(r["ms_oproj_resident"] * 1e3, 2),
                        "us_qkv_gemm_only_resident_f16": round(
                            r["ms_gemm_only_resident"] * 1e3, 2),
                        "us_attention_layer_resident_f16": round(
                            r["ms_layer_resident"] * 1e3, 2),
                        "us_attention_layer_reference_order": round(
                            r["ms_layer_reference_order"] * 1e3, 2),
                        "tflops_qkv_fused": round(fl_qkv / (pf * 1e-3) / 1e12, 1),
                        "tflops_qkv_fused_resident_f16": round(
                            fl_qkv / (r["ms_fused_resident"] * 1e-3) / 1e12, 1),
                        "tflops_oproj": round(fl_o / (po * 1e-3) / 1e12, 1),
                        "tensor_frac_of_measured_qkv": round(
                            fl_qkv / (pf * 1e-3) / 1e12 / tensor_peak, 4),
                        "tensor_frac_of_measured_qkv_resident_f16": round(
                            fl_qkv / (r["ms_fused_resident"] * 1e-3) / 1e12 / tensor_peak, 4),
                        "hbm_bytes_saved": s_tok * (HQ + 2 * HKV) * D * 2 * 2,
                        "parity": r["parity"]}
                except p2p_b200.P2PError as e:
                    side[key] = {"error": str(e)}
            try:
                va, v_par = run_vision(ctx, steps=20, warmup=5)
                fl = vision_flops()
                side["vision"] = {
                    "workload": "bidirectional MHA B=16 S=1024 12 heads d64 fp16",
                    "tflops": round(fl / (va * 1e-3) / 1e12, 1), "us": round(va * 1e3, 2),
                    "tensor_frac_of_measured": round(fl / (va * 1e-3) / 1e12 / tensor_peak, 4),
                    "parity": reduce_parity(v_par, 1)}
            except p2p_b200.P2PError as e:
                side["vision"] = {"error": str(e)}

    # every rank takes the same collective steps: reduce before rank 0 formats the line
    ms_direct_max = max_over_ranks(ms_direct, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        kind = cpu_kind()
        sec, threads, n = cpu_reference_step_seconds(kind)
        cpu = {"value": round(wl.bytes_per_step / sec / 1e9, 4), "unit": "GB/s",
               "cores": threads, "kind": kind,
               "sample": f"{n} whole decode steps (6 layers x 32 heads x 4097 keys)"}

    if rank == 0:
        tr = traffic.get("decode_kernel_per_step_bytes")
        line = {
            "metric": "decode_attn_gbs_ctx4096", "value": round(value_gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max, 5), "us_per_step": round(ms_max * 1e3, 3),
            "us_per_step_direct_launch": round(ms_direct_max * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1), torch CUDA generator)",
            "config": {"workload": "lfm2.5-1.2b decode attention, ctx 4096+1, 6 layers, 32q/8kv, "
                                   "d64, fused qk-prep + split-KV, one launch per step",
                       "past": PAST, "layers": N_LAYERS, "bytes_per_step_per_gpu": wl.bytes_per_step,
                       "l2": "inputs rotate over 12 KV copies (605 MB > L2)",
                       "timing": "K steps captured in one CUDA graph, one replay timed with "
                                 "CUDA events; us_per_step_direct_launch = K host calls",
                       "parallelism": f"replicas x{world} (independent sequences per GPU)"},
            "roofline": {"bound": "hbm", "achieved": round(per_gpu_gbs, 1),
                         "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(per_gpu_gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "frac_of_nominal_8tbs": round(per_gpu_gbs / 8000.0, 4),
                         "traffic": tr, "kernel": "decode_mma_kernel<G=4,fused,layers,cluster>",
                         "stream_same_bytes_us": round(sol_us, 3),
                         "frac_of_stream": round(sol_us / (ms_max * 1e3), 4),
                         "stream_note": "p2p_debug_stream_read: one plain streaming launch "
                                        "over the same bytes per graph node, same rotation"},
            "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_step": round(e2e_sec * 1e6, 2),
                    "host": e2e_note,
                    "c_abi_call_per_token_us_per_step": round(direct_sec * 1e6, 2),
                    "python_ctypes_us_per_step": round(py_sec * 1e6, 2)},
            "gpu_launches": args.steps,
            "parity": parity,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "side": side,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
