"""Decode-step benchmark of the paged KV-cache path on B200.

Workload (one "step"): one decode token for every sequence of the batch,
through all 32 layers: fused RoPE + slot-mapped append of the token's K/V
(and RoPE of q), then paged split-K GQA attention over the sequence's
blocks.  Shape: Llama-3-8B attention (32 query heads, 8 KV heads, head_dim
128), block_size 16, 64 sequences per GPU with context lengths uniform in
[128, 4096] (seed 1), blocks drawn from a randomly permuted pool sized at
1.25x need.  fp32 K/V storage is the headline (the reference's type); the
bf16-storage variant is measured in the same run.  Synthetic data (numpy /
torch seeded normal), no dataset.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun); sequences are sharded across
GPUs by balanced context sum, each GPU runs its own pool, no collective on
the data path ("weak" scaling: 64 sequences per GPU).  Rank 0 prints one
JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "s1-infer_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "paged decode-attn KV GB/s/GPU (% HBM peak); decode tok/s at 1/2/4/8 B200"
LAYERS, HQ, HKV, D, BS = 32, 32, 8, 128, 16  # LAYERS may be lowered by --layers for profiling cases
EVENT_STEPS = 5  # decode steps of the per-launch timing pass that follows the timed steps
# DRAM bytes (read + write) per decode launch over its algorithmic bytes, from
# one ncu capture of each kernel on the one- or two-layer case of this
# workload (same shapes, 1.08 GB / 0.54 GB per launch, above L2):
#   fp32 decode_tma_kernel: 1.082104 GB read + 6.259 MB written, 1.082991 GB algorithmic
#   bf16 decode_mma_kernel: 0.542419 GB read + 6.341 MB written, 0.542561 GB algorithmic
# Traffic grows with the context like the algorithmic bytes, so a launch of
# the full run is reported as this ratio times its algorithmic bytes.
DRAM_PER_ALGORITHMIC = {"f32": (1.082104e9 + 6.259e6) / 1.082991e9, "bf16": (0.542419e9 + 6.341e6) / 0.542561e9}
SEQS_PER_GPU = 64
CTX_LO, CTX_HI, CTX_SEED = 128, 4096, 1
WORKLOAD = "cfg2: batched ragged paged decode, Llama-3-8B attention shape"


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_tflops_peak():
    """Dense bf16 tensor peak for a kernel timed alone (the burst figure)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured bf16_tflops (burst, MEASURED_PEAKS.json)"
    except Exception:
        return 1590.0, "fallback 1590 TFLOP/s"


def contexts(n_gpus):
    """Per-rank context lengths.  Weak scaling with identical per-GPU work:
    every rank serves its own 64 sequences drawn from U[128, 4096] with the
    same seed, so the global batch is 64*N sequences and each GPU's work is
    exactly the 1-GPU workload at every N."""
    rng = np.random.default_rng(CTX_SEED)
    ctx = [int(c) for c in rng.integers(CTX_LO, CTX_HI + 1, size=SEQS_PER_GPU)]
    return [list(ctx) for _ in range(n_gpus)]


def balanced_shards(ctx, n_ranks):
    """Greedy split of a global batch over ranks by context sum (longest
    first, equal counts): how a server would shard one shared queue."""
    order = np.argsort(-np.asarray(ctx), kind="stable")
    per = len(ctx) // n_ranks
    loads = np.zeros(n_ranks)
    share = [[] for _ in range(n_ranks)]
    for i in order:
        r = min((r for r in range(n_ranks) if len(share[r]) < per), key=lambda x: loads[x])
        share[r].append(int(ctx[i]))
        loads[r] += ctx[i]
    return share


def decode_bytes(ctx_after, elem):
    """Algorithmic bytes of one decode-attention launch (one layer): K and V
    of every context token once per KV head, q in and out (fp32), and the
    block-table entries."""
    c = np.asarray(ctx_after, np.int64)
    return int((c * 2 * HKV * D * elem).sum() + len(c) * HQ * D * (4 + 4) + ((c + BS - 1) // BS * 4).sum())


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU,
    polled every 100 ms from a thread through NVML while the timed region
    runs (nvidia-smi as a fallback)."""

    PERIOD_S = 0.1
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        import torch
        self.samples = []
        self.stop_ev = threading.Event()
        self.nvml = None
        pr = torch.cuda.get_device_properties(device)
        self.bus = "%08X:%02X:%02X.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        try:
            import pynvml
            pynvml.nvmlInit()
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(self.bus.encode())
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _poll(self):
        n = self.nvml
        while not self.stop_ev.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
                try:
                    rs = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    rs = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((sm, rs))
            except Exception:
                pass
            self.stop_ev.wait(self.PERIOD_S)

    def start(self):
        if self.nvml:
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()

    def stop(self):
        if not self.nvml:
            return self._smi_once()
        self.stop_ev.set()
        self.t.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"], "samples": 0}
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm for sm, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}

    def _smi_once(self):
        try:
            out = subprocess.run(["nvidia-smi", f"--id={self.bus}", "--query-gpu=clocks.sm,clocks.max.sm",
                                  "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10).stdout
            sm, smax = (float(x) for x in out.strip().split(","))
            return {"sm_mhz": sm, "sm_max_mhz": smax, "reasons": [], "samples": 1, "source": "nvidia-smi after"}
        except Exception:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"], "samples": 0}


# ----------------------------------------------------------------- ours ---

def run_variant(s1kv, torch, dtype, ctx, steps, warmup, rank, world, timed_e2e, sample_clocks):
    elem = 4 if dtype == "f32" else 2
    B = len(ctx)
    total_steps = 2 * (steps + warmup) + min(steps, EVENT_STEPS) + 2
    need = sum((c + total_steps + BS - 1) // BS for c in ctx)
    max_blocks = int(need * 1.25)
    rng = np.random.default_rng(1000 + rank)
    order = rng.permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(LAYERS, HKV, D, max_blocks, BS, dtype=dtype, initial_free_list=order, max_seqs=max(256, B))
    seqs = list(range(B))
    gen = torch.Generator(device="cuda").manual_seed(17 + rank)
    # prefill: random post-RoPE K/V for every context token, layer by layer
    with pool.batch(seqs, ctx, [0] * B) as b:
        for layer in range(LAYERS):
            k = torch.randn((sum(ctx), HKV, D), device="cuda", generator=gen)
            v = torch.randn((sum(ctx), HKV, D), device="cuda", generator=gen)
            b.rope_append(layer, k, v)
            del k, v
    torch.cuda.synchronize()
    q = torch.randn((LAYERS, B, HQ, D), device="cuda", generator=gen)
    kn = torch.randn((LAYERS, B, HKV, D), device="cuda", generator=gen)
    vn = torch.randn((LAYERS, B, HKV, D), device="cuda", generator=gen)
    q_rot = torch.empty((LAYERS, B, HQ, D), device="cuda")
    out = torch.empty((LAYERS, B, HQ, D), device="cuda")

    # per-layer views made once: the timed loop issues the library's calls only
    views = [(kn[l], vn[l], q[l], q_rot[l], out[l]) for l in range(LAYERS)]
    ones = [1] * B

    def step(ev=None):
        with pool.batch(seqs, ones) as bt:
            for layer, (kl, vl, ql, qrl, ol) in enumerate(views):
                bt.rope_append(layer, kl, vl, q=ql, q_out=qrl)
                if ev is not None:
                    ev[layer][0].record()
                bt.attention(layer, qrl, out=ol)
                if ev is not None:
                    ev[layer][1].record()

    for _ in range(warmup):
        step()
    barrier(torch, world)
    torch.cuda.synchronize()
    ctx_timed = [pool.length(s) for s in seqs]
    clocks = ClockSampler(torch.cuda.current_device()) if sample_clocks else None
    if clocks:
        clocks.start()
    launches0 = s1kv.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push(f"timed_decode_{dtype}")  # ncu --nvtx-include filters the launch list on it
    t0.record()
    h0 = time.perf_counter()
    for i in range(steps):
        step()
    t1.record()
    host_ms = (time.perf_counter() - h0) * 1e3  # issuing the steps; below the device time: not host-bound
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    launches = s1kv.launch_count() - launches0
    clk = clocks.stop() if clocks else None
    elapsed_ms = t0.elapsed_time(t1)
    # Attention launch durations: the next steps again with an event pair
    # around every attention call.  An event recorded between two kernels
    # ends the programmatic overlap of their launches, so the timed steps
    # above carry no per-layer events.
    n_ev = min(steps, EVENT_STEPS)
    ctx_before = [pool.length(s) for s in seqs]
    evs = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(LAYERS)]
           for _ in range(n_ev)]
    for i in range(n_ev):
        step(evs[i])
    torch.cuda.synchronize()
    attn_ms = [evs[i][layer][0].elapsed_time(evs[i][layer][1]) for i in range(n_ev) for layer in range(LAYERS)]
    attn_bytes = sum(decode_bytes([c + i + 1 for c in ctx_before], elem) for i in range(n_ev)) * LAYERS
    res = {
        "elapsed_ms": elapsed_ms,
        "attn_ms_total": float(sum(attn_ms)),
        "attn_launches": len(attn_ms),
        "attn_bytes": attn_bytes,
        "bytes_per_launch": attn_bytes / len(attn_ms),
        "avg_launch_ms": float(np.mean(attn_ms)),
        "launches": launches,
        "clocks": clk,
        "tokens": B * steps,
        "kv_bytes_step": sum(decode_bytes([c + i + 1 for c in ctx_timed], elem) for i in range(steps)) * LAYERS / steps,
        "host_issue_ms_per_step": host_ms / steps,
    }
    if timed_e2e:
        hq = torch.empty((LAYERS, B, HQ, D), pin_memory=True)
        hk = torch.empty((LAYERS, B, HKV, D), pin_memory=True)
        hv = torch.empty((LAYERS, B, HKV, D), pin_memory=True)
        ho = torch.empty((LAYERS, B, HQ, D), pin_memory=True)
        hq.copy_(q)
        hk.copy_(kn)
        hv.copy_(vn)

        def step_host():
            with pool.batch(seqs, [1] * B) as bt:
                for layer in range(LAYERS):
                    bt.layer_host(layer, hq[layer], hk[layer], hv[layer], ho[layer], HQ)

        for _ in range(warmup):
            step_host()
        barrier(torch, world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step_host()
        e1.record()
        torch.cuda.synchronize()
        res["e2e_ms"] = e0.elapsed_time(e1)
        res["h2d_bytes_per_step"] = LAYERS * (hq[0].numel() + hk[0].numel() + hv[0].numel()) * 4
        res["d2h_bytes_per_step"] = LAYERS * ho[0].numel() * 4
    assert pool.check_device() == 0
    pool.close()
    del q, kn, vn, q_rot, out
    torch.cuda.empty_cache()
    return res


def barrier(torch, world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _reduce(torch, world, x, op):
    """All-reduce one number over the ranks (NCCL on GPU, gloo on CPU)."""
    if world == 1:
        return x
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(torch, world, x):
    import torch.distributed as dist
    return _reduce(torch, world, x, dist.ReduceOp.MAX) if world > 1 else x


def sum_over_ranks(torch, world, x):
    import torch.distributed as dist
    return _reduce(torch, world, x, dist.ReduceOp.SUM) if world > 1 else x


def cpu_reference_sample(ctx, n_threads, layers_sampled=1, repeats=2, seed=5):
    """Times the reference's GQA_attention_paged (oracle/_ref, compiled from
    the reference sources) on one decode step of `ctx` sequences over
    `layers_sampled` layer pools, fanned over (layer, sequence) tasks with
    the reference's ThreadPool.  Falls back to the C restatement
    (oracle/kvoracle.c, one thread) when the reference library is absent."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    B = len(ctx)
    need = sum((c + 1 + BS - 1) // BS for c in ctx) + 4
    kind = "reference" if O.ref_available() else "port"
    q = rng.standard_normal((layers_sampled, B, HQ, D), dtype=np.float32)
    if kind == "reference":
        pools = [O.RefPool(HKV, D, need, BS) for _ in range(layers_sampled)]
    else:
        pools = [O.Pool(HKV, D, need, BS) for _ in range(layers_sampled)]
        n_threads = 1
    for p in pools:
        for s, c in enumerate(ctx):
            k = rng.standard_normal((c + 1, HKV, D), dtype=np.float32)
            p.append(s, k, k)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        if kind == "reference":
            O.ref_decode_batch(pools, np.arange(B), q, HQ, HKV, D, n_threads)
        else:
            for li, p in enumerate(pools):
                for s in range(B):
                    p.attention(s, q[li, s:s + 1], HQ)
        times.append(time.perf_counter() - t0)
    t_layer = min(times) / layers_sampled
    tok_s = B / (LAYERS * t_layer)
    kv_bytes = decode_bytes([c + 1 for c in ctx], 4)
    return {
        "value": tok_s,
        "unit": "tok/s",
        "cores": n_threads,
        "kind": kind,
        "sample": f"{layers_sampled} of {LAYERS} layers x {B} sequences x 1 decode step (fp32), "
                  f"best of {repeats}; per-layer time scaled x{LAYERS}",
        "kv_gbs": kv_bytes / t_layer / 1e9,
        "layer_s": t_layer,
    }


def prefill_flops(prefix, suffixes, hq, d):
    """QK^T + PV FLOPs of a causal prefix-hit prefill: 4*Hq*D per visible
    (query, key) pair, query i of a suffix seeing prefix + i + 1 keys."""
    return sum(4 * hq * d * (L * prefix + L * (L + 1) // 2) for L in suffixes)


def run_cfg3(s1kv, torch, rank, reps=10, n=256):
    """cfg3: 256 sequences fork one 2050-token prefix (128 full blocks plus
    a 2-token tail, shared with refcounts); each appends a suffix of
    U[64, 512] tokens (seed 2), which first copies the shared tail block
    (copy-on-write), then runs the prefix-hit chunked prefill (tensor-core
    kernel), then 32 decode steps.  bf16 K/V, Hq 32 / Hkv 8 / D 128, block
    16; one layer (the workload names no layer count: figures are per
    layer).  `n` below 256 is a smaller profiling case of the same shape."""
    P, bs = 2050, 16
    # first launches (module loading, tensor maps) on a throwaway pool, so
    # the timed step measures the step's work
    warm = s1kv.Pool(1, HKV, D, 64, bs, dtype="bf16", max_seqs=8)
    with warm.batch([0], [40], [0]) as b:
        b.rope_append(0, torch.randn((40, HKV, D), device="cuda"), torch.randn((40, HKV, D), device="cuda"))
    warm.fork(0, 1, 40)
    with warm.batch([1], [300]) as b:
        q_w = b.rope_append(0, torch.randn((300, HKV, D), device="cuda"), torch.randn((300, HKV, D), device="cuda"),
                            q=torch.randn((300, HQ, D), device="cuda"))
        b.attention(0, q_w)
    torch.cuda.synchronize()
    warm.close()
    rng = np.random.default_rng(2)
    suff = [int(x) for x in rng.integers(64, 513, size=n)]
    dec_steps = 32
    blocks = (P + bs - 1) // bs + sum((L + dec_steps + bs) // bs + 1 for L in suff) + 8
    order = rng.permutation(blocks).astype(np.int32)
    pool = s1kv.Pool(1, HKV, D, blocks, bs, dtype="bf16", initial_free_list=order, max_seqs=n + 8)
    gen = torch.Generator(device="cuda").manual_seed(23 + rank)
    with pool.batch([0], [P], [0]) as b:
        b.rope_append(0, torch.randn((P, HKV, D), device="cuda", generator=gen),
                      torch.randn((P, HKV, D), device="cuda", generator=gen))
    seqs = list(range(1, n + 1))
    for s_ in seqs:
        pool.fork(0, s_, P)
    T = sum(suff)
    q = torch.randn((T, HQ, D), device="cuda", generator=gen)
    k = torch.randn((T, HKV, D), device="cuda", generator=gen)
    v = torch.randn((T, HKV, D), device="cuda", generator=gen)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    # outputs allocated before the timed step (torch's allocator is not the step)
    q_rot, out = torch.empty_like(q), torch.empty_like(q)
    torch.cuda.synchronize()
    e0.record()
    with pool.batch(seqs, suff) as b:  # COW of every tail, RoPE+append, prefill
        b.rope_append(0, k, v, q=q, q_out=q_rot)
        e1.record()
        b.attention(0, q_rot, out=out)
        e2.record()
        torch.cuda.synchronize()
        step_ms = e0.elapsed_time(e2)
        # the attention call is idempotent: time it alone, repeated
        for _ in range(3):
            b.attention(0, q_rot, out=out)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        for _ in range(reps):
            b.attention(0, q_rot, out=out)
        t1.record()
        torch.cuda.synchronize()
        # the same step's appends from raw projections: q/k RMSNorm + RoPE +
        # append in one kernel, against the RoPE + append kernel alone
        qw = torch.randn(D, device="cuda", generator=gen)
        kw = torch.randn(D, device="cuda", generator=gen)
        q_n = torch.empty_like(q)
        ap = []
        for fused in (True, False):
            for _ in range(2):
                if fused:
                    b.norm_rope_append(0, k, v, kw, q=q, q_norm_weight=qw, q_out=q_n)
                else:
                    b.rope_append(0, k, v, q=q, q_out=q_n)
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            for _ in range(reps):
                if fused:
                    b.norm_rope_append(0, k, v, kw, q=q, q_norm_weight=qw, q_out=q_n)
                else:
                    b.rope_append(0, k, v, q=q, q_out=q_n)
            a1.record()
            torch.cuda.synchronize()
            ap.append(a0.elapsed_time(a1) / reps)
    attn_ms = t0.elapsed_time(t1) / reps
    # fp32 q, k, v read; q_out fp32 and K, V (bf16) written
    ap_bytes = T * (HQ * D * 4 * 2 + 2 * HKV * D * 4 + 2 * HKV * D * 2)
    flops = prefill_flops(P, suff, HQ, D)
    cow = pool.stats()["cow_copies"]
    # 32 decode steps of all 256 sequences (split-K decode over shared blocks)
    qd = torch.randn((n, HQ, D), device="cuda", generator=gen)
    kd = torch.randn((n, HKV, D), device="cuda", generator=gen)
    vd = torch.randn((n, HKV, D), device="cuda", generator=gen)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(dec_steps):
        with pool.batch(seqs, [1] * n) as b:
            qr = b.rope_append(0, kd, vd, q=qd)
            b.attention(0, qr)
    d1.record()
    torch.cuda.synchronize()
    dec_ms = d0.elapsed_time(d1) / dec_steps
    assert pool.check_device() == 0
    pool.close()
    return {"prefill_attn_ms": attn_ms, "prefill_tflops": flops / (attn_ms * 1e-3) / 1e12, "prefill_flops": flops,
            "prefill_step_ms": step_ms, "cow_copies": cow, "decode_ms_per_step": dec_ms,
            "norm_rope_append_ms": ap[0], "norm_rope_append_gbs": ap_bytes / (ap[0] * 1e-3) / 1e9,
            "rope_append_ms": ap[1], "append_tokens": T,
            "decode_tok_s_per_layer": n / (dec_ms * 1e-3)}


CFG4_B, CFG4_CTX, CFG4_HQ, CFG4_HKV, CFG4_LAYERS = 4, 131072, 64, 8, 80


def run_cfg4(s1kv, torch, rank, world, steps=10, warmup=3, shard=None, max_layers=CFG4_LAYERS):
    """cfg4, KV-head-sharded long-context decode: 4 sequences at context
    131072, Hq 64 / Hkv 8 / D 128, bf16 K/V, 80 layers, blocks scattered over
    a pool of 1.1x need (permutation seed 3).  Rank r of N keeps only KV heads
    [8r/N, 8(r+1)/N) (s1kv.head_shard).  Each layer of a step: RoPE + append
    of the new token, paged decode of the local heads, one all-gather of the
    [4, 64/N, 128] outputs (NCCL over NVLink) and the head-major to
    token-major reorder.  The next layer's queries for this rank's heads are
    another rank's outputs, so the gather is on the critical path as it is in
    a model.  Where 80 layers of the pool do not fit in one GPU's memory
    (N = 1), fewer layers are timed and the step figures are scaled to 80.
    K/V are seeded normal values (synthetic post-RoPE keys)."""
    B, CTX, hq_all, hkv_all = CFG4_B, CFG4_CTX, CFG4_HQ, CFG4_HKV
    # shard (profiling case, one process): rank 0's share of a `shard`-GPU
    # run, timed alone on this GPU
    kv_lo, kv_hi, q_lo, q_hi = s1kv.head_shard(shard or world, rank, hkv_all, hq_all)
    hkv, hq = kv_hi - kv_lo, q_hi - q_lo
    need = B * ((CTX + 2 * (warmup + steps + 3) + BS - 1) // BS)  # two modes of warm-up, timed and breakdown steps
    max_blocks = int(need * 1.1)
    per_layer = max_blocks * BS * hkv * D * 2 * 2
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info()
    layers = int(min(max_layers, (free - 16e9) // per_layer))
    layers = int(-max_over_ranks(torch, world, -layers))  # every rank times the same layers
    order = np.random.default_rng(3).permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(layers, hkv, D, max_blocks, BS, dtype="bf16", initial_free_list=order, max_seqs=8)
    gen = torch.Generator(device="cuda").manual_seed(31 + rank)
    seqs = list(range(B))
    with pool.batch(seqs, [CTX] * B, [0] * B) as b:
        kbuf = torch.empty((B * CTX, hkv, D), device="cuda")
        vbuf = torch.empty_like(kbuf)
        for layer in range(layers):
            kbuf.normal_(generator=gen)
            vbuf.normal_(generator=gen)
            b.append(layer, kbuf, vbuf)
        del kbuf, vbuf
    torch.cuda.synchronize()
    q0 = torch.randn((B, hq, D), device="cuda", generator=gen)
    kn = torch.randn((layers, B, hkv, D), device="cuda", generator=gen)
    vn = torch.randn((layers, B, hkv, D), device="cuda", generator=gen)
    q_rot = torch.empty((B, hq, D), device="cuda")
    q_next = torch.empty((B, hq, D), device="cuda")
    out = torch.empty((B, hq, D), device="cuda")
    gbuf = torch.empty((world, B, hq, D), device="cuda")
    nxt = (rank + 1) % world

    # one process standing in for one rank of `shard`: no other rank writes
    # the other heads, so its exchange holds its own heads only (the wait
    # checks every word of the slot)
    ex_heads = hq if world == 1 and (shard or 1) > 1 else hq_all
    ex_h0, ex_nxt = (q_lo, nxt * hq) if ex_heads == hq_all else (0, 0)
    ex = s1kv.PeerExchange(rank, world, B, ex_heads, D)
    epoch = [0]

    def step(ev=None, fused=False):
        q = q0
        with pool.batch(seqs, [1] * B) as bt:
            for layer in range(layers):
                bt.rope_append(layer, kn[layer], vn[layer], q=q, q_out=q_rot)
                if ev is not None:
                    ev[layer][0].record()
                # the next layer's queries of this rank's heads are another
                # rank's outputs
                if fused:
                    # the decode kernels store every finished row into all
                    # ranks' token-major buffers over NVLink, then signal;
                    # one kernel waits for every rank and copies the next
                    # layer's query heads out
                    epoch[0] += 1
                    ex.attention(bt, layer, q_rot, ex_h0, epoch[0])
                    if ev is not None:
                        ev[layer][1].record()
                    q = ex.wait_copy(epoch[0], ex_nxt, hq, q_next)
                else:
                    bt.attention(layer, q_rot, out=out)
                    if ev is not None:
                        ev[layer][1].record()
                    full = s1kv.gather_heads(out, world, buf=gbuf)  # [B, 64, 128] token-major on every rank
                    q = q_next.copy_(full[:, nxt * hq:(nxt + 1) * hq])
                if ev is not None:
                    ev[layer][2].record()

    res = {}
    for mode in ("nccl", "fused"):
        fused = mode == "fused"
        for _ in range(warmup):
            step(fused=fused)
        barrier(torch, world)
        torch.cuda.synchronize()
        ctx_before = [pool.length(s) for s in seqs]
        # the timed steps carry no per-layer events (an event between two
        # kernels ends their programmatic launch overlap)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        h0 = time.perf_counter()
        for i in range(steps):
            step(fused=fused)
        issue_us = (time.perf_counter() - h0) * 1e6 / (steps * layers)  # host time to issue a layer
        t1.record()
        torch.cuda.synchronize()
        elapsed = max_over_ranks(torch, world, t0.elapsed_time(t1))
        # per-layer breakdown: a few more steps with an event pair around
        # each attention call and the exchange that follows it
        n_ev = min(steps, 3)
        evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(layers)] for _ in range(n_ev)]
        for i in range(n_ev):
            step(evs[i], fused=fused)
        torch.cuda.synchronize()
        attn_ms = float(np.mean([evs[i][l][0].elapsed_time(evs[i][l][1]) for i in range(n_ev) for l in range(layers)]))
        xchg_ms = float(np.mean([evs[i][l][1].elapsed_time(evs[i][l][2]) for i in range(n_ev) for l in range(layers)]))
        res[mode] = (elapsed, max_over_ranks(torch, world, attn_ms), max_over_ranks(torch, world, xchg_ms), ctx_before,
                     max_over_ranks(torch, world, issue_us))
    s1kv.device_check(torch.cuda.current_device())
    barrier(torch, world)  # no rank frees its exchange buffer while a peer may still hold it open
    ex.close()
    elapsed, attn_ms, gather_ms, ctx_before, issue_us = res["fused"]
    # algorithmic bytes of one layer's attention on this GPU: K and V of the
    # local heads once, q in and out (fp32), block ids
    ctx_mid = [c + (steps + 1) // 2 for c in ctx_before]
    attn_bytes = (sum(ctx_mid) * 2 * hkv * D * 2 + B * hq * D * (4 + 4) + sum((c + BS - 1) // BS for c in ctx_mid) * 4)
    assert pool.check_device() == 0
    pool.close()
    del q0, kn, vn, q_rot, out, gbuf
    torch.cuda.empty_cache()
    step_ms_80 = elapsed / steps * CFG4_LAYERS / layers
    nccl_step_80 = res["nccl"][0] / steps * CFG4_LAYERS / layers
    return {"workload": "cfg4: 4 seqs x ctx 131072, Hq64/Hkv8/D128, bf16, 80 layers, pool 1.1x scattered (seed 3)",
            "parallelism": f"kv-head-sharded x{world} ({hkv} KV heads per GPU); finished rows stored into every "
                           f"rank's buffer over NVLink by the decode kernels (fused exchange)",
            "nccl_allgather": {"ms_per_step_80_layers": nccl_step_80, "tok_s": B / (nccl_step_80 * 1e-3),
                               "allgather_reorder_ms_per_layer": res["nccl"][2]},
            "scaling": "strong", "layers_timed": layers, "steps": steps,
            "ms_per_step_80_layers": step_ms_80, "tok_s": B / (step_ms_80 * 1e-3),
            "ms_per_layer": elapsed / steps / layers, "attn_ms_per_layer": attn_ms,
            "exchange_wait_ms_per_layer": gather_ms, "host_issue_us_per_layer": issue_us,
            "attn_bytes_per_layer_per_gpu": attn_bytes, "kv_gbs_per_gpu": attn_bytes / (attn_ms * 1e-3) / 1e9}


def run_cfg5(s1kv, torch, rank, world, steps=100, warmup=20):
    """cfg5, pool churn, one GPU's share of a sequence-sharded 8-GPU node
    (512 running sequences, 8 arrivals per step, 55k blocks per layer):
    64 running sequences on a pool of 6875 blocks per layer (32 layers,
    Hq 32 / Hkv 8 / D 128, bf16), Poisson(1) arrivals per step, prompts
    log-normal (median 1024, sigma 0.8), outputs U[32, 512], 30% of the
    prompts starting with one of 16 prefixes of U[256, 4096] tokens, LRU
    eviction of zero-refcount prefix blocks (s1kv.churn; seed 4, and
    1000 * rank added per rank).  A step: retire finished requests, admit
    queued ones (prefix-cache match, reserve, prompt K/V appended),
    one-token RoPE + append for every running sequence and decode attention
    over its blocks, all 32 layers.  Timed on the wall clock (host
    bookkeeping included) and with CUDA events."""
    from s1kv.churn import ChurnDriver, ChurnWorkload
    layers, max_blocks, max_running = 32, 55000 // 8, 64
    order = np.random.default_rng(4 + rank).permutation(max_blocks).astype(np.int32)
    pool = s1kv.Pool(layers, HKV, D, max_blocks, BS, dtype="bf16", initial_free_list=order,
                     max_seqs=4 * max_running)
    wl = ChurnWorkload(seed=4 + 1000 * rank)
    drv = ChurnDriver(pool, wl, max_running=max_running)
    drv.queue.extend(wl.request() for _ in range(max_running))
    gen = torch.Generator(device="cuda").manual_seed(41 + rank)
    cap = 1 << 17
    kbuf = torch.randn((cap, HKV, D), device="cuda", generator=gen)
    vbuf = torch.randn((cap, HKV, D), device="cuda", generator=gen)
    qbuf = torch.randn((max_running, HQ, D), device="cuda", generator=gen)
    # host[0]: wall time of the bookkeeping calls (which includes waiting for
    # a staging buffer the GPU still reads when the host is ahead); host[1]:
    # the CPU time this thread spent in them; host[2]: CPU time of the whole
    # step's issue (bookkeeping and the 64 per-layer calls)
    host = [0.0, 0.0, 0.0]

    def step():
        h0, c0, s0 = time.perf_counter(), time.thread_time(), time.thread_time()
        plan = drv.plan()
        b = drv.open(plan)
        host[0] += time.perf_counter() - h0
        host[1] += time.thread_time() - c0
        assert plan.n_tokens <= cap
        for layer in range(layers):
            q = qbuf[:plan.n_rows] if plan.n_rows else None
            qr = b.rope_append(layer, kbuf[:plan.n_tokens], vbuf[:plan.n_tokens], q=q)
            if plan.n_rows:
                b.attention(layer, qr)
        h0, c0 = time.perf_counter(), time.thread_time()
        b.end()
        drv.close(plan)
        host[0] += time.perf_counter() - h0
        host[1] += time.thread_time() - c0
        host[2] += time.thread_time() - s0

    step()
    rng = np.random.default_rng(7 + rank)
    for s in drv.running:  # steady state: the first requests are somewhere inside their outputs
        drv.running[s] = int(rng.integers(1, drv.running[s] + 1))
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(torch, world)
    s0 = dict(drv.stats)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host[:] = [0.0, 0.0, 0.0]
    t0 = time.perf_counter()
    ev0.record()
    for _ in range(steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3
    gpu_ms = ev0.elapsed_time(ev1)
    d = {k: drv.stats[k] - s0.get(k, 0) for k in drv.stats}
    # The bookkeeping alone: further steps with the device drained before
    # each bookkeeping call, so that no wait for a staging buffer still in
    # use (the host running ahead of the GPU) is counted.
    idle = []
    for _ in range(20):
        torch.cuda.synchronize()
        c0 = time.perf_counter()
        plan = drv.plan()
        b = drv.open(plan)
        c1 = time.perf_counter()
        for layer in range(layers):
            qr = b.rope_append(layer, kbuf[:plan.n_tokens], vbuf[:plan.n_tokens],
                               q=qbuf[:plan.n_rows] if plan.n_rows else None)
            if plan.n_rows:
                b.attention(layer, qr)
        torch.cuda.synchronize()
        c2 = time.perf_counter()
        b.end()
        drv.close(plan)
        idle.append((c1 - c0) + (time.perf_counter() - c2))
    st = pool.stats()
    assert pool.check_device() == 0
    pool.close()
    del kbuf, vbuf, qbuf
    torch.cuda.empty_cache()
    wall_max = max_over_ranks(torch, world, wall_ms)
    dec = sum_over_ranks(torch, world, float(d.get("decode_tokens", 0)))
    app = sum_over_ranks(torch, world, float(d.get("appended_tokens", 0)))
    return {"workload": "cfg5 per GPU: 64 running seqs, Poisson(1) arrivals, prompts lognormal(1024, 0.8), outputs "
                        "U[32,512], 30% reuse of 16 prefixes U[256,4096], LRU eviction, pool 6875 blocks x 32 "
                        "layers bf16 Hq32/Hkv8/D128 (seed 4)",
            "parallelism": f"sequence-sharded x{world}, independent pools, no collective", "scaling": "weak",
            "steps": steps, "decode_tok_s": dec / (wall_max * 1e-3), "appended_tok_s": app / (wall_max * 1e-3),
            "ms_per_step": wall_max / steps, "gpu_ms_per_step": gpu_ms / steps,
            "host_bookkeeping_ms_per_step": host[0] * 1e3 / steps,
            "host_bookkeeping_cpu_ms_per_step": host[1] * 1e3 / steps,
            "host_issue_cpu_ms_per_step": host[2] * 1e3 / steps,
            "host_bookkeeping_idle_ms_per_step": float(np.median(idle)) * 1e3,
            "per_gpu_in_window": {k: d.get(k, 0) for k in ("admitted", "retired", "deferred", "preempted",
                                                             "prefix_hit_tokens", "decode_tokens", "appended_tokens")},
            "evictions_total": st["evictions"], "occupancy": 1.0 - st["num_free"] / max_blocks}


# int8 projections of one decode token through the reference's model shape
# (Qwen3-0.6B: hidden 1024, 16 query heads and 8 KV heads of 128, MLP 3072,
# 28 layers; src/nn/attention.cpp:253-254, tests/test_layer.cpp:20-27) with
# the Qwen3 vocabulary for the LM head (src/model/model.cpp:177).
INT8_LAYERS, INT8_VOCAB = 28, 151936
INT8_PROJ = [("q_proj", 1024, 2048), ("k_proj", 1024, 1024), ("v_proj", 1024, 1024), ("o_proj", 2048, 1024),
             ("gate_proj", 1024, 3072), ("up_proj", 1024, 3072), ("down_proj", 3072, 1024)]


def run_int8(s1kv, torch, rank, steps=20, warmup=3, cpu_sample=True):
    """The int8 projections either side of the KV path for one decode step:
    28 layers x 7 weights plus the LM head [1024, 151936], quantized with
    quantize_tensor (one scale per row), multiplied by M = 1 (the
    reference's single-sequence decode) and M = 8 rows.  596 MB of int8
    weights, far above L2: every step streams them from HBM.  A step's 197
    launches are captured once in a CUDA graph and replayed; the LM head is
    also timed alone (155.6 MB per launch).  Roofline: weight bytes (+ x and
    out) per step over the measured HBM copy bandwidth."""
    gen = torch.Generator(device="cuda").manual_seed(31 + rank)
    mats = []
    for _ in range(INT8_LAYERS):
        for _, K, N in INT8_PROJ:
            mats.append(s1kv.quantize_tensor(torch.randn((K, N), device="cuda", generator=gen) * 0.05))
    w = torch.randn((1024, INT8_VOCAB), device="cuda", generator=gen) * 0.05
    mats.append(s1kv.quantize_tensor(w))
    del w
    torch.cuda.synchronize()
    wbytes = sum(q.rows * q.cols + 4 * q.rows for q in mats)
    peak, _ = load_peaks()
    res = {}
    for M in (1, 8):
        xs = {K: torch.randn((M, K), device="cuda", generator=gen) for K in (1024, 2048, 3072)}
        outs = [torch.empty((M, q.cols), device="cuda") for q in mats]

        def step(sel=None):
            for qt, o in (zip(mats, outs) if sel is None else [sel]):
                s1kv.matmul_quantized(xs[qt.rows], qt, out=o)

        def step_grouped():
            # the products that share x in one launch each: q/k/v, gate/up
            n = len(INT8_PROJ)
            for li in range(INT8_LAYERS):
                m, o = mats[li * n:(li + 1) * n], outs[li * n:(li + 1) * n]
                s1kv.matmul_quantized_group(xs[1024], m[0:3], o[0:3])
                s1kv.matmul_quantized(xs[2048], m[3], out=o[3])
                s1kv.matmul_quantized_group(xs[1024], m[4:6], o[4:6])
                s1kv.matmul_quantized(xs[3072], m[6], out=o[6])
            s1kv.matmul_quantized(xs[1024], mats[-1], out=outs[-1])

        step()  # first launches (attributes, cluster query) outside the capture
        step_grouped()
        torch.cuda.synchronize()
        l0 = s1kv.launch_count()
        g, gl, gg = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        launches = s1kv.launch_count() - l0
        with torch.cuda.graph(gl):
            step((mats[-1], outs[-1]))
        l1 = s1kv.launch_count()
        with torch.cuda.graph(gg):
            step_grouped()
        launches_grouped = s1kv.launch_count() - l1
        io_bytes = sum(4 * M * (q.rows + q.cols) for q in mats)
        times = {}
        for name, gr in (("step", g), ("lm_head", gl), ("grouped", gg)):
            for _ in range(warmup):
                gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(steps):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            times[name] = e0.elapsed_time(e1) / steps
        # end to end: x from pinned host memory, the LM-head logits back
        hx = torch.randn((M, 1024), generator=torch.Generator().manual_seed(7)).pin_memory()
        hout = torch.empty((M, INT8_VOCAB)).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            xs[1024].copy_(hx, non_blocking=True)
            g.replay()
            hout.copy_(outs[-1], non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / steps
        lm = mats[-1]
        lm_bytes = lm.rows * lm.cols + 4 * lm.rows + 4 * M * (lm.rows + lm.cols)
        res[f"M{M}"] = {
            "ms_per_step": times["step"], "tok_s": M / (times["step"] * 1e-3),
            "weight_gbs": (wbytes + io_bytes) / (times["step"] * 1e-3) / 1e9,
            "frac_of_hbm": (wbytes + io_bytes) / (times["step"] * 1e-3) / 1e9 / peak,
            "launches_per_step": launches,
            "grouped_ms_per_step": times["grouped"], "grouped_tok_s": M / (times["grouped"] * 1e-3),
            "grouped_frac_of_hbm": (wbytes + io_bytes) / (times["grouped"] * 1e-3) / 1e9 / peak,
            "grouped_launches_per_step": launches_grouped,
            "lm_head_ms": times["lm_head"], "lm_head_gbs": lm_bytes / (times["lm_head"] * 1e-3) / 1e9,
            "lm_head_frac_of_hbm": lm_bytes / (times["lm_head"] * 1e-3) / 1e9 / peak,
            "e2e_ms_per_step": e2e_ms, "e2e_tok_s": M / (e2e_ms * 1e-3),
            "e2e_h2d_bytes_per_step": 4 * M * 1024, "e2e_d2h_bytes_per_step": 4 * M * INT8_VOCAB}
        del g, gl, gg
    out = {"workload": f"int8 projections of one decode step: {INT8_LAYERS} layers x (q 1024x2048, k/v 1024x1024, "
                       f"o 2048x1024, gate/up 1024x3072, down 3072x1024) + LM head 1024x{INT8_VOCAB}, one scale "
                       f"per row, seeded normal weights",
           "weight_bytes_per_step": wbytes, "l2": "weights 596 MB per step, above L2", **res}
    if cpu_sample and rank == 0:
        from oracle import oracle as O
        if O.ref_available():
            import time as _t
            layer = mats[:len(INT8_PROJ)]
            host = [(q.data.cpu().numpy(), q.scales.cpu().numpy()) for q in layer + [mats[-1]]]
            x1 = {K: np.random.default_rng(K).standard_normal((1, K)).astype(np.float32) for K in (1024, 2048, 3072)}
            best = {}
            for _ in range(2):
                t0 = _t.perf_counter()
                for q, sc in host[:-1]:
                    O.ref_matmul_int8(x1[q.shape[0]], q, sc, threaded=True)
                t1 = _t.perf_counter()
                O.ref_matmul_int8(x1[1024], host[-1][0], host[-1][1], threaded=True)
                t2 = _t.perf_counter()
                best["layer"] = min(best.get("layer", 1e9), t1 - t0)
                best["lm"] = min(best.get("lm", 1e9), t2 - t1)
            tok_ms = (best["layer"] * INT8_LAYERS + best["lm"]) * 1e3
            out["cpu_baseline"] = {"value": 1e3 / tok_ms, "unit": "tok/s (M = 1)", "cores": os.cpu_count() or 1,
                                   "kind": "reference",
                                   "sample": "matmul_quantized (thread pool) on layer 0's 7 weights (x28) and the LM "
                                             "head, M = 1, best of 2",
                                   "ms_per_step": tok_ms,
                                   "weight_gbs": wbytes / (tok_ms * 1e-3) / 1e9}
    return out


def run_ours(args):
    import torch
    import s1kv

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))  # each rank names its GPU
    share = contexts(world)[rank]
    peak, peak_kind = load_peaks()
    res = {}
    for dtype in ("f32", "bf16"):
        if args.only and dtype != args.only:
            continue
        res[dtype] = run_variant(s1kv, torch, dtype, share, args.steps, args.warmup, rank, world,
                                 timed_e2e=not args.no_e2e, sample_clocks=(dtype == "f32"))
    cfg3 = run_cfg3(s1kv, torch, rank, n=args.cfg3_seqs) if not args.only or args.only == "cfg3" else None
    cfg4 = run_cfg4(s1kv, torch, rank, world, shard=args.cfg4_shard, max_layers=args.cfg4_layers) \
        if not args.only or args.only == "cfg4" else None
    cfg5 = run_cfg5(s1kv, torch, rank, world) if not args.only or args.only == "cfg5" else None
    int8 = run_int8(s1kv, torch, rank, cpu_sample=(world == 1 and not args.no_cpu_baseline)) \
        if not args.only or args.only == "int8" else None
    if args.only:
        # profiling case: one variant, no summary line
        if rank == 0 and args.only in ("cfg3", "cfg4", "cfg5", "int8"):
            print(json.dumps({"profiling_case": args.only,
                              **{"cfg3": cfg3, "cfg4": cfg4, "cfg5": cfg5, "int8": int8}[args.only]}))
        elif rank == 0:
            r = res[args.only]
            print(json.dumps({"profiling_case": args.only, "layers": LAYERS, "ms_per_step": r["elapsed_ms"] / args.steps,
                              "avg_launch_ms": r["avg_launch_ms"], "bytes_per_launch": r["bytes_per_launch"],
                              "e2e_ms_per_step": r["e2e_ms"] / args.steps if "e2e_ms" in r else None}))
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    h = res["f32"]
    elapsed = max_over_ranks(torch, world, h["elapsed_ms"])
    tokens = sum_over_ranks(torch, world, h["tokens"])
    e2e_ms = max_over_ranks(torch, world, h["e2e_ms"])
    bf = res["bf16"]
    bf_elapsed = max_over_ranks(torch, world, bf["elapsed_ms"])
    bf_tokens = sum_over_ranks(torch, world, bf["tokens"])
    bf_e2e_ms = max_over_ranks(torch, world, bf["e2e_ms"])
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_sample(share, os.cpu_count() or 1)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    achieved = h["bytes_per_launch"] / (h["avg_launch_ms"] * 1e-3) / 1e9
    tflops_peak, _ = load_tflops_peak()
    bf_achieved = bf["bytes_per_launch"] / (bf["avg_launch_ms"] * 1e-3) / 1e9
    step_s, bf_step_s = elapsed / args.steps * 1e-3, bf_elapsed / args.steps * 1e-3

    def r(x, n=4):
        return None if x is None else float(f"{x:.{n}g}")

    # One compact line (numbers only; the workloads are described in DESIGN.md):
    # every figure must survive in the few-KB tail of stdout the driver keeps.
    line = {
        "metric": METRIC,
        "value": r(tokens / (elapsed * 1e-3), 6),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": r(elapsed / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "cfg2 batched ragged paged decode", "layers": LAYERS, "hq": HQ, "hkv": HKV, "d": D,
                   "bs": BS, "seqs_per_gpu": SEQS_PER_GPU, "global_batch": SEQS_PER_GPU * world,
                   "ctx": f"U[{CTX_LO},{CTX_HI}] seed {CTX_SEED}", "kv": "fp32",
                   "parallelism": f"seq-shard x{world}", "l2": "inputs > L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": r(achieved), "peak": peak, "unit": "GB/s",
                     "frac": r(achieved / peak), "traffic": r(DRAM_PER_ALGORITHMIC["f32"] * h["bytes_per_launch"]),
                     "peak_src": peak_kind, "launch_ms": r(h["avg_launch_ms"]), "bytes": r(h["bytes_per_launch"]),
                     "step_frac": r(h["kv_bytes_step"] / (h["elapsed_ms"] / args.steps * 1e-3) / 1e9 / peak)},
        "e2e": {"value": r(tokens / (e2e_ms * 1e-3), 6), "unit": "tok/s",
                "h2d_bytes_per_step": h["h2d_bytes_per_step"], "d2h_bytes_per_step": h["d2h_bytes_per_step"]},
        "gpu_launches": h["launches"],
        "host_issue_ms": r(h["host_issue_ms_per_step"], 3),
        "clocks": {k: h["clocks"].get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons", "samples")} if h["clocks"] else None,
        "cpu_baseline": None if cpu is None else {k: (r(cpu[k]) if k == "value" else cpu[k])
                                                  for k in ("value", "unit", "cores", "kind", "sample")},
        "variants": {
            "bf16": {"tok_s": r(bf_tokens / (bf_elapsed * 1e-3), 5), "e2e_tok_s": r(bf_tokens / (bf_e2e_ms * 1e-3), 5),
                     "ms_per_step": r(bf_elapsed / args.steps), "frac": r(bf_achieved / peak),
                     "step_frac": r(bf["kv_bytes_step"] / (bf["elapsed_ms"] / args.steps * 1e-3) / 1e9 / peak),
                     "launch_ms": r(bf["avg_launch_ms"])},
        },
    }
    v = line["variants"]
    if cfg3 is not None:
        v["cfg3"] = {"prefill_tflops": r(cfg3["prefill_tflops"]), "frac": r(cfg3["prefill_tflops"] / tflops_peak),
                     "prefill_ms": r(cfg3["prefill_attn_ms"]), "step_ms": r(cfg3["prefill_step_ms"]),
                     "cow": cfg3["cow_copies"], "decode_ms": r(cfg3["decode_ms_per_step"]),
                     "nra_ms": r(cfg3["norm_rope_append_ms"]), "nra_frac": r(cfg3["norm_rope_append_gbs"] / peak),
                     "ra_ms": r(cfg3["rope_append_ms"])}
    if cfg4 is not None:
        v["cfg4"] = {"tok_s": r(cfg4["tok_s"]), "ms_per_step": r(cfg4["ms_per_step_80_layers"]),
                     "layers_timed": cfg4["layers_timed"], "attn_ms": r(cfg4["attn_ms_per_layer"]),
                     "frac": r(cfg4["kv_gbs_per_gpu"] / peak), "wait_ms": r(cfg4["exchange_wait_ms_per_layer"]),
                     "issue_us": r(cfg4["host_issue_us_per_layer"]),
                     "nccl_tok_s": r(cfg4["nccl_allgather"]["tok_s"]), "scaling": "strong"}
    if cfg5 is not None:
        v["cfg5"] = {"decode_tok_s": r(cfg5["decode_tok_s"]), "ms_per_step": r(cfg5["ms_per_step"]),
                     "gpu_ms": r(cfg5["gpu_ms_per_step"]), "host_wall_ms": r(cfg5["host_bookkeeping_ms_per_step"]),
                     "host_cpu_ms": r(cfg5["host_bookkeeping_cpu_ms_per_step"]),
                     "host_idle_ms": r(cfg5["host_bookkeeping_idle_ms_per_step"]),
                     "issue_cpu_ms": r(cfg5["host_issue_cpu_ms_per_step"]),
                     "evictions": cfg5["evictions_total"]}
    if int8 is not None:
        m1, m8 = int8["M1"], int8["M8"]
        v["int8"] = {"m1_ms": r(m1["grouped_ms_per_step"]), "m1_frac": r(m1["grouped_frac_of_hbm"]),
                     "m1_launches": m1["grouped_launches_per_step"], "m1_ungrouped_frac": r(m1["frac_of_hbm"]),
                     "lm_head_frac": r(m1["lm_head_frac_of_hbm"]), "m8_ms": r(m8["grouped_ms_per_step"]),
                     "m8_frac": r(m8["grouped_frac_of_hbm"]), "m1_e2e_tok_s": r(m1["e2e_tok_s"]),
                     "cpu_tok_s": r(int8["cpu_baseline"]["value"]) if "cpu_baseline" in int8 else None}
    if args.detail:
        with open(args.detail, "w") as f:
            json.dump({"f32": h, "bf16": bf, "cfg3": cfg3, "cfg4": cfg4, "cfg5": cfg5, "int8": int8, "cpu": cpu}, f,
                      indent=1, default=str)
    print(json.dumps(line))


# ------------------------------------------------------------ reference ---

def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if rank != 0:
        return
    share = contexts(world)[0]
    from oracle import oracle as O
    n_threads = os.cpu_count() or 1
    rng = np.random.default_rng(5)
    B = len(share)
    need = sum((c + 1 + BS - 1) // BS for c in share) + 4
    kind = "reference" if O.ref_available() else "port"
    pool = O.RefPool(HKV, D, need, BS) if kind == "reference" else O.Pool(HKV, D, need, BS)
    for s, c in enumerate(share):
        k = rng.standard_normal((c + 1, HKV, D), dtype=np.float32)
        pool.append(s, k, k)
    q = rng.standard_normal((1, B, HQ, D), dtype=np.float32)

    def one_layer():
        if kind == "reference":
            O.ref_decode_batch([pool], np.arange(B), q, HQ, HKV, D, n_threads)
        else:
            for s in range(B):
                pool.attention(s, q[0, s:s + 1], HQ)

    for _ in range(args.warmup):
        one_layer()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_layer()
    dt = (time.perf_counter() - t0) / args.steps
    tok_s = B / (LAYERS * dt)
    # Each timed step is ONE of the 32 layers of a decode step (the bounded
    # sample); the per-step figures below are that layer's time scaled x32
    # and say so.
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * LAYERS * 1e3,
        "ms_per_step_kind": f"extrapolated: measured layer ms x {LAYERS}",
        "layers_timed": 1, "ms_per_layer_measured": dt * 1e3, "timed_region_s": dt * args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg2 batched ragged paged decode", "layers": LAYERS, "hq": HQ, "hkv": HKV, "d": D,
                   "bs": BS, "seqs_per_gpu": SEQS_PER_GPU, "global_batch": B,
                   "ctx": f"U[{CTX_LO},{CTX_HI}] seed {CTX_SEED}", "kv": "fp32",
                   "parallelism": "host CPU, rank 0 only (the sequences of one GPU)"},
        "kv_gbs": decode_bytes([c + 1 for c in share], 4) / dt / 1e9,
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": n_threads if kind == "reference" else 1,
                         "kind": kind,
                         "sample": f"each step = 1 of {LAYERS} layers x {B} sequences x 1 decode token "
                                   f"(GQA_attention_paged over the reference ThreadPool); scaled x{LAYERS}"},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS, help="profiling cases only (the bench line uses 32)")
    ap.add_argument("--only", choices=["f32", "bf16", "cfg3", "cfg4", "cfg5", "int8"],
                    help="profiling case: run one variant")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cfg3-seqs", type=int, default=256, help="profiling case: sequences of the cfg3 variant")
    ap.add_argument("--detail", help="also write every figure of the run, unrounded, to this JSON file")
    ap.add_argument("--cfg4-shard", type=int, default=None,
                    help="profiling case: the cfg4 variant as one GPU's KV-head shard of an N-GPU run")
    ap.add_argument("--cfg4-layers", type=int, default=CFG4_LAYERS, help="profiling case: layers of the cfg4 variant")
    args = ap.parse_args()
    globals()["LAYERS"] = args.layers
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
