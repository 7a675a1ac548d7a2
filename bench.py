#!/usr/bin/env python
"""Benchmark of the 4-bit KV-cache hot path on B200.

Metric (headline): int4-KV attention TFLOP/s on the single-layer workload
"Q [1, 4680, 40, 128] over a 4680-token int4 window (3 latent frames) with a
1560-token sink, non-causal", plus quantize GB/s and prefill ms/block at
windows 3/12/21 as extra keys.

  python bench.py [--gpus N --steps K --warmup W]        this implementation
  python bench.py --impl reference [...]                 the reference's CPU path
At N > 1 (one process per GPU under torch.distributed.run) the run is weakly
scaled: N streams, the 40 heads split over the ranks (40/N per GPU), so every
GPU does the single-GPU amount of work, then one NCCL all-gather of the
attention output per step. `value` is whole-job TFLOP/s (all ranks), timed on
the device with CUDA events, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "krea-realtime-bench_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "int4-KV attn TFLOP/s + quantize GB/s; prefill ms/block at window 3/12/21"
H_TOTAL, D, FRAME = 40, 128, 1560
LQ = LK = 3 * FRAME
SINK = FRAME
MODE = "bands4"
N_SETS = 4                      # rotating input sets: ~4 x 160 MB > 126 MB L2
DATA = ("synthetic, seeded: K ~ N(0,1) x log-normal per-channel scales + 3-axis RoPE, "
        "V ~ N(0,1), Q ~ N(0,1)/sqrt(128); bf16")


def attn_flops(B, H, Lq, Lk, d=D):
    return 4.0 * B * H * Lq * Lk * d


def quant_bytes_per_row(G, d=D):
    return 2 * d + d // 2 + 2 * G


# ----------------------------------------------------------------------------- clocks
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU (NVML, read-only) in a
    background thread, as fast as NVML answers. mark_start() / mark_end() bracket
    the timed region (host clock, right before the start event is recorded and
    right after the closing synchronize); the summary keeps the samples inside
    it, and when a short region holds fewer than 3 samples, also the ones
    within 50 ms of it (and says so)."""

    def __init__(self, device: int, period_s: float = 0.0005):
        self.period = period_s
        self.samples: list[tuple[float, int, int, float]] = []
        self.max_mhz = None
        self.t0 = self.t1 = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        n = 0
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except Exception:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                pw = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0 if n % 8 == 0 else float("nan")
                self.samples.append((time.perf_counter(), mhz, rs, pw))
                n += 1
            except Exception:
                pass
            time.sleep(self.period)

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __enter__(self):
        if self._h is not None:
            self._t.start()
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            time.sleep(0.05)
        self._stop.set()
        if self._h is not None:
            self._t.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml unavailable" if self._h is None else "nvml"}
        t0 = self.t0 if self.t0 is not None else -math.inf
        t1 = self.t1 if self.t1 is not None else math.inf
        sel = [x for x in self.samples if t0 <= x[0] <= t1]
        window = "timed region"
        if len(sel) < 3:
            sel = [x for x in self.samples if t0 - 0.05 <= x[0] <= t1 + 0.05]
            window = "timed region +- 50 ms (the region is shorter than 3 samples)"
        if not sel:
            sel = self.samples
            window = "whole run"
        mhz = [x[1] for x in sel]
        bits = 0
        for x in sel:
            bits |= int(x[2])
        reasons = sorted(n for b, n in _REASONS.items() if bits & b and n != "gpu_idle")
        pw = [x[3] for x in sel if x[3] == x[3]]
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz), "window": window, "power_w_max": round(max(pw), 1) if pw else None,
                "source": "nvml"}


def load_peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(name: str):
    """DRAM bytes per launch of a kernel from a committed ncu summary, or None."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(name)
    except Exception:
        return None


# ----------------------------------------------------------------------------- workload
def make_caches(B, S, Hl, sink, device, seed, h0=0):
    """Two QuantKVTensor caches [B, S, Hl, 128] filled by quantize-append of
    synthetic K and V (generated on the device)."""
    import quant_kv
    from kvq import synth
    tk = quant_kv.QuantKVTensor([B, S, Hl, D], device, torch.bfloat16, 4, MODE, sink)
    tv = quant_kv.QuantKVTensor([B, S, Hl, D], device, torch.bfloat16, 4, MODE, sink)
    k = torch.stack([synth.make_k(S, Hl, seed=seed + 101 * b + h0, device=device) for b in range(B)])
    v = torch.stack([synth.make_v(S, Hl, seed=seed + 101 * b + h0 + 1, device=device) for b in range(B)])
    tk[:, 0:S] = k
    tv[:, 0:S] = v
    return tk, tv, k, v


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU path
def cpu_attention_sample(n_heads: int, reps: int | None = None, min_seconds: float = 0.0, warmup: int = 0):
    """The reference's CPU path on a bounded sample of the workload: for
    `n_heads` of the 40 heads, quantize K and V of the 4680-token block (int4,
    bands4), read the window back (dequantize + bf16 sink overlay) and run
    fp32 softmax attention of 4680 queries. Oracle port (plain C, all host
    threads) + torch fp32 SDPA (all host threads). Returns per-rep seconds."""
    from kvq import synth
    from oracle import c_oracle
    from oracle import kvq_oracle as ko
    bands = ko.band_edges(D, MODE)
    k = synth.make_k(LK, n_heads, seed=1).view(torch.int16).numpy().view(np.uint16)
    v = synth.make_v(LK, n_heads, seed=2).view(torch.int16).numpy().view(np.uint16)
    q = synth.make_q(1, LQ, n_heads, seed=3).float()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def one():
        out = []
        for x in (k, v):
            c, s = c_oracle.quantize(x, bands, 4, threads)
            w = c_oracle.dequantize(c, s, bands, D, 4, threads)
            w[:SINK] = x[:SINK]
            out.append(torch.from_numpy(ko.bf16_to_f32(w)))
        kw, vw = out
        o = torch.nn.functional.scaled_dot_product_attention(
            q[0].transpose(0, 1), kw.transpose(0, 1), vw.transpose(0, 1))
        return o

    for _ in range(warmup):
        one()
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if reps is not None and len(times) >= reps:
            break
        if reps is None and time.perf_counter() - t_start >= min_seconds:
            break
    return times, threads


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    heads = 1
    times, threads = cpu_attention_sample(heads, reps=args.steps, warmup=args.warmup)
    per_step = sum(times) / len(times)
    v = attn_flops(1, heads, LQ, LK) / per_step / 1e12
    cfg = workload_config(world)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": DATA, "config": cfg,
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{heads} of 40 heads per step: int4 quantize of K and V (4680 tokens), "
                                   "window read with bf16 sink overlay, fp32 SDPA of 4680 queries"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(world, gather="fused"):
    return {"workload": "int4-KV attention, window 3 frames (4680 tokens, 1560-token bf16 sink), "
                        "Q 4680 tokens, non-causal; bands4 groups",
            "streams": world, "heads": H_TOTAL, "heads_per_gpu": H_TOTAL // world, "lq": LQ, "lk": LK,
            "sink": SINK, "head_dim": D, "group_mode": MODE,
            "l2": f"{N_SETS} rotating input sets (Q + packed K/V + sink + out, ~{N_SETS * 160} MB) > 126 MB L2",
            "parallelism": "single GPU" if world == 1 else (
                f"head-sharded x{world}; output all-gather fused into the attention epilogue (NVLink peer stores)"
                if gather == "fused" else f"head-sharded x{world} + NCCL all-gather")}


# ----------------------------------------------------------------------------- our path
def run_ours(args):
    import quant_kv
    from kvq import ops, shard, synth
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    if H_TOTAL % world:
        raise SystemExit(f"{H_TOTAL} heads do not split over {world} GPUs")
    B = world
    h0, h1 = shard.head_range(H_TOTAL, world, rank)
    Hl = h1 - h0
    peaks = load_peaks()

    # ---- inputs resident in HBM: N_SETS rotating sets
    fused = world > 1 and args.gather == "fused"
    sets, peers = [], []
    for i in range(N_SETS):
        tk, tv, _, _ = make_caches(B, LK, Hl, SINK, dev, seed=1000 * i, h0=h0)
        q = synth.make_q(B, LQ, Hl, seed=1000 * i + 7, device=dev)
        out = torch.empty_like(q)
        sets.append((q, tk, tv, out))
        if fused:
            # full-width output of the set on every rank, mapped into every peer, with
            # a completion counter per rank (device-side signal, no host barrier)
            peers.append(shard.PeerOutputs(torch.empty((B, LQ, H_TOTAL, D), dtype=torch.bfloat16, device=dev)))
    gbuf = shard.gather_buffer(sets[0][3], world) if world > 1 else None
    torch.cuda.synchronize()

    def step(i, kev=None):
        q, tk, tv, out = sets[i % N_SETS]
        if kev is not None:
            kev[0].record()
        if fused:
            po = peers[i % N_SETS]
            ops.attention_packed_gather(q, tk, tv, 0, LK, po.ptrs, h0, H_TOTAL)
        else:
            ops.attention_packed(q, tk, tv, 0, LK, out=out)
        if kev is not None:
            kev[1].record()
        if fused:
            # the step's consumer may read po.local once every rank's launch has
            # completed: a device-side barrier of the ranks (part of the timed step)
            po.barrier()
        elif world > 1:
            shard.gather_outputs(out, gbuf)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    kevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        clk.mark_start()
        e0.record()
        for i in range(args.steps):
            step(i, kevs[i])
        e1.record()
        torch.cuda.synchronize()
        clk.mark_end()
    if world > 1:
        dist.barrier()
    t_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    k_ms = [a.elapsed_time(b) for a, b in kevs]
    k_mean = sum(k_ms) / len(k_ms)
    # per-rank attention time at N > 1 (the step also waits for the slowest rank)
    k_max_ranks = max_over_ranks(k_mean, world, dev)
    k_min_ranks = -max_over_ranks(-k_mean, world, dev)
    status = ops.device_status()
    if status != 0:
        raise SystemExit(f"device status {status}: a kernel wait timed out; results invalid")
    gather_check = None
    if world > 1:
        gather_check = check_gather(sets, peers, fused, gbuf, step, args.warmup + args.steps, world, dev)
    flops_rank = attn_flops(B, Hl, LQ, LK)
    value = world * flops_rank * args.steps / (t_ms / 1e3) / 1e12
    achieved = flops_rank / (k_mean / 1e3) / 1e12

    # ---- end to end through the public API, host buffers, copies timed
    e2e = run_e2e(args, dev, world, B, Hl, h0, gbuf)

    extra = {}
    cpu = None
    if world == 1 and not args.no_extras:
        extra = run_extras(dev, peaks)
    if not args.no_config4:
        extra["config4"] = run_config4(args, dev, world, rank, peaks)
    if rank == 0 and world == 1 and not args.no_cpu:
        times, threads = cpu_attention_sample(2, min_seconds=args.cpu_seconds, warmup=1)
        per = sum(times) / len(times)
        cpu = {"value": attn_flops(1, 2, LQ, LK) / per / 1e12, "unit": "TFLOP/s", "cores": threads,
               "kind": "port",
               "sample": f"2 of 40 heads x {len(times)} reps ({sum(times):.1f} s): int4 quantize of K and V "
                         "(4680 tokens), window read with bf16 sink overlay, fp32 SDPA of 4680 queries; "
                         "C oracle + torch CPU"}

    traffic = load_traffic("attention_config1")
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": DATA, "config": workload_config(world, args.gather),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"],
                     "traffic": traffic,
                     "kernel": "attention_kernel (tcgen05, per-launch CUDA events, mean)",
                     "kernel_ms": k_mean,
                     "kernel_ms_over_ranks": {"min": k_min_ranks, "max": k_max_ranks},
                     "peak_source": f"{peaks['source']} bf16 dense (burst), of {peaks['source']}"},
        "e2e": e2e,
        "gpu_launches": args.steps * (2 if fused else 1),
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "extra": extra,
    }
    if gather_check is not None:
        line["gather_check"] = gather_check
    if rank == 0:
        print(json.dumps(line), flush=True)
    if gather_check is False:
        raise SystemExit("gather_check failed: a rank's gathered output differs from the NCCL-gathered outputs")
    if world > 1:
        dist.barrier()          # every rank is done storing into the peers' buffers
        for p in peers:
            p.close()
        dist.barrier()
        dist.destroy_process_group()


def check_gather(sets, peers, fused, gbuf, step, i, world, dev) -> bool:
    """Untimed step i (set i % N_SETS) after the timing; every rank then compares
    the full output it holds with the ranks' own attention outputs gathered by
    NCCL, bit for bit. The verdict is the AND over the ranks."""
    import torch.distributed as dist
    from kvq import ops, shard
    q, tk, tv, out = sets[i % N_SETS]
    full = peers[i % N_SETS].local if fused else None
    if fused:
        full.zero_()
        torch.cuda.synchronize()
        dist.barrier()
    step(i)
    if fused:
        got = full.clone()
    else:
        got = shard.assemble_heads(gbuf.view(world, *out.shape)).clone()
    ref = shard.assemble_heads(shard.gather_outputs(ops.attention_packed(q, tk, tv, 0, LK)))
    ok = torch.tensor([1 if torch.equal(got, ref) and ops.device_status() == 0 else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    torch.cuda.synchronize()
    dist.barrier()
    return bool(ok.item())


def run_e2e(args, dev, world, B, Hl, h0, gbuf):
    """Same metric through the public API, from host memory: per step, copy q, k,
    v of the block from pinned host memory, quantize-append K and V into the
    caches (QuantKVTensor slice writes), attention over the window
    (quant_kv.attention on one GPU; at N > 1 the head-sharded
    ops.attention_packed_gather into PeerOutputs with its device-side completion
    wait), and copy the step's result back to the host (N = 1: the output; N > 1:
    the full output of the stream this rank serves, all 40 heads). Three streams
    pipeline consecutive steps (upload of step i+1 and download of step i-1
    overlap the compute of step i); every step still moves all of its inputs and
    its output across PCIe inside the timed region."""
    import quant_kv
    from kvq import ops, shard, synth
    tk = quant_kv.QuantKVTensor([B, LK, Hl, D], dev, torch.bfloat16, 4, MODE, SINK)
    tv = quant_kv.QuantKVTensor([B, LK, Hl, D], dev, torch.bfloat16, 4, MODE, SINK)
    nb = 2          # input buffers
    no = 3          # output buffers: a peer may store into buffer i % 3 once this rank's
                    # download of step i - 3 is done (the compute of step i - 1 waited for it)
    qh = [synth.make_q(B, LQ, Hl, seed=11 + i).pin_memory() for i in range(nb)]
    kh = [torch.stack([synth.make_k(LK, Hl, seed=12 + b + i) for b in range(B)]).pin_memory() for i in range(nb)]
    vh = [torch.stack([synth.make_v(LK, Hl, seed=13 + b + i) for b in range(B)]).pin_memory() for i in range(nb)]
    qd = [torch.empty_like(qh[0], device=dev) for _ in range(nb)]
    kd = [torch.empty_like(kh[0], device=dev) for _ in range(nb)]
    vd = [torch.empty_like(vh[0], device=dev) for _ in range(nb)]
    if world == 1:
        od = [torch.empty((B, LQ, Hl, D), dtype=torch.bfloat16, device=dev) for _ in range(no)]
        res = od
        pos = None
    else:
        rank = int(os.environ.get("RANK", "0"))
        pos = [shard.PeerOutputs(torch.empty((B, LQ, H_TOTAL, D), dtype=torch.bfloat16, device=dev))
               for _ in range(no)]
        res = [p.local[rank] for p in pos]              # [LQ, 40, D]: the stream this rank serves
    oh = [torch.empty(res[0].shape, dtype=torch.bfloat16).pin_memory() for _ in range(no)]
    s_up, s_cmp, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    up_done, cmp_done, dn_done = {}, {}, {}

    def step(i):
        j, o = i % nb, i % no
        with torch.cuda.stream(s_up):
            if i - nb in cmp_done:
                s_up.wait_event(cmp_done[i - nb])      # step i-2 finished reading input buffer j
            qd[j].copy_(qh[j], non_blocking=True)
            kd[j].copy_(kh[j], non_blocking=True)
            vd[j].copy_(vh[j], non_blocking=True)
            up_done[i] = ev()
            up_done[i].record(s_up)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(up_done[i])
            if i - 2 in dn_done:
                s_cmp.wait_event(dn_done[i - 2])       # output buffer (i-2) % 3 downloaded
            tk[:, 0:LK] = kd[j]
            tv[:, 0:LK] = vd[j]
            if pos is None:
                quant_kv.attention(qd[j], tk[:, 0:LK], tv[:, 0:LK], out=od[o])
            else:
                po = pos[o]
                ops.attention_packed_gather(qd[j], tk, tv, 0, LK, po.ptrs, h0, H_TOTAL)
                po.barrier()
            cmp_done[i] = ev()
            cmp_done[i].record(s_cmp)
        with torch.cuda.stream(s_dn):
            s_dn.wait_event(cmp_done[i])
            oh[o].copy_(res[o], non_blocking=True)
            dn_done[i] = ev()
            dn_done[i].record(s_dn)

    n = max(3, min(args.steps, 20))
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    up_done.clear(); cmp_done.clear(); dn_done.clear()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_up)
    for i in range(n):
        step(i)
    s_up.wait_stream(s_dn)
    e1.record(s_up)
    torch.cuda.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1), world, dev)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()              # every rank is done storing into and reading the buffers
        for p in pos:
            p.close()
        dist.barrier()
    flops = world * attn_flops(B, Hl, LQ, LK) * n
    h2d = (qh[0].numel() + kh[0].numel() + vh[0].numel()) * 2
    return {"value": flops / (t / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": oh[0].numel() * 2, "steps": n, "ms_per_step": t / n,
            "path": ("pinned H2D of q,k,v -> QuantKVTensor slice writes (quantize-append) -> "
                     + ("quant_kv.attention" if world == 1 else
                        "ops.attention_packed_gather (all-gather in the epilogue) + device-side completion wait")
                     + " -> D2H of the step's output; upload, compute and download of consecutive steps on "
                       "three streams")}


def _time_events(fn, n, warm=2):
    for _ in range(warm):
        fn(0)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for i in range(n):
        ev[i][0].record()
        fn(i)
        ev[i][1].record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def _time_graph(fn, n, reps=5):
    """Per-call device time of fn(i) for i < n launched back to back: the n calls
    are captured in one CUDA graph, so host-side argument handling between the
    launches is not timed (a small kernel timed call by call measures the host).
    Returns per-call ms of each replay."""
    fn(0)                                    # warm-up (one-time set-up happens outside the capture)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1) / n)
    del g
    return out


def run_extras(dev, peaks):
    """Quantize/dequantize GB/s and prefill ms/block at windows 3/12/21."""
    import quant_kv
    import quant_kv_kernels
    from kvq import ops, synth
    bands = quant_kv._band_edges(D, MODE)
    G = len(bands)
    cb = quant_kv_kernels.host_chan_band(quant_kv_kernels.build_chan_band(bands, D, "cpu"))
    res = {}
    # quantize-append of one block (K and V, 4680 x 40 heads), and the window-21 rebuild size
    for name, L in (("append_block_4680", LK), ("rebuild_layer_32760", 21 * FRAME)):
        xs = [synth.make_k(L, H_TOTAL, seed=50 + i, device=dev) for i in range(4)]
        cs = [torch.empty((L, H_TOTAL, D // 2), dtype=torch.uint8, device=dev) for _ in range(4)]
        ss = [torch.empty((L, H_TOTAL, G), dtype=torch.bfloat16, device=dev) for _ in range(4)]

        def fq(i):
            for t in range(2):  # K and V of one layer
                j = (2 * i + t) % 4
                ops.quantize_into(xs[j], cs[j], ss[j], cb, G, 4)
        ms = _time_graph(fq, 20)
        byts = 2 * L * H_TOTAL * quant_bytes_per_row(G)
        gbs = byts / (statistics.median(ms) / 1e3) / 1e9
        res[f"quantize_{name}"] = {"gbs": gbs, "ms": statistics.median(ms), "bytes": byts,
                                   "frac_hbm": gbs / peaks["hbm_gbs"],
                                   "timing": "CUDA graph of 20 iterations (K and V: two launches each)"}
        outs = [torch.empty_like(x) for x in xs]

        def fd(i):
            for t in range(2):
                j = (2 * i + t) % 4
                ops.dequantize_into(cs[j], ss[j], outs[j], cb, G, 4)
        ms = _time_graph(fd, 20)
        res[f"dequantize_{name}"] = {"gbs": byts / (statistics.median(ms) / 1e3) / 1e9,
                                     "ms": statistics.median(ms)}
        del xs, cs, ss, outs
        torch.cuda.empty_cache()

    # the append of one block of keys before their rotary embedding (fused rotate + quantize)
    from kvq import rope
    fr = rope.freqs(1024, device=dev)
    pos = rope.grid_positions(0, LK, device=dev)
    xs = [synth.make_k(LK, H_TOTAL, seed=60 + i, device=dev) for i in range(4)]
    cs = [torch.empty((LK, H_TOTAL, D // 2), dtype=torch.uint8, device=dev) for _ in range(4)]
    ss = [torch.empty((LK, H_TOTAL, G), dtype=torch.bfloat16, device=dev) for _ in range(4)]

    def fr_q(i):
        j = i % 4
        ops.rope_quantize_into(xs[j], cs[j], ss[j], cb, G, 4, fr, pos)
    ms = _time_graph(fr_q, 20)
    byts = LK * H_TOTAL * quant_bytes_per_row(G)
    res["rope_quantize_append_block_4680_per_tensor"] = {
        "gbs": byts / (statistics.median(ms) / 1e3) / 1e9, "ms": statistics.median(ms), "bytes": byts,
        "frac_hbm": byts / (statistics.median(ms) / 1e3) / 1e9 / peaks["hbm_gbs"],
        "timing": "CUDA graph of 20 launches"}
    del xs, cs, ss
    torch.cuda.empty_cache()

    # the append of one layer's block (K and V, 4680 tokens x 40 heads) as ONE launch
    # (kvq_rebuild_layers with the two tensors): the runtime's per-layer pattern
    xs = [synth.make_k(LK, H_TOTAL, seed=650 + i, device=dev) for i in range(8)]
    cs = [torch.empty((LK, H_TOTAL, D // 2), dtype=torch.uint8, device=dev) for _ in range(8)]
    ss = [torch.empty((LK, H_TOTAL, G), dtype=torch.bfloat16, device=dev) for _ in range(8)]

    def fl(i):
        j = 2 * (i % 4)
        ops.quantize_layers_into(xs[j:j + 2], cs[j:j + 2], ss[j:j + 2], cb, G, 4)
    ms = _time_graph(fl, 20)
    byts = 2 * LK * H_TOTAL * quant_bytes_per_row(G)
    gbs = byts / (statistics.median(ms) / 1e3) / 1e9
    res["quantize_append_layer_kv_4680_one_launch"] = {
        "gbs": gbs, "ms": statistics.median(ms), "bytes": byts, "frac_hbm": gbs / peaks["hbm_gbs"],
        "note": "4 rotating input pairs (384 MB > L2); CUDA graph of 20 launches"}
    del xs, cs, ss
    torch.cuda.empty_cache()

    # the append of one block to all 40 layers x {K, V} in one launch (kvq_rebuild_layers),
    # 80 distinct inputs (3.8 GB), so no input is re-read from L2
    nt = 80
    xs = [synth.make_k(LK, H_TOTAL, seed=700 + i, device=dev) for i in range(nt)]
    cs = [torch.empty((LK, H_TOTAL, D // 2), dtype=torch.uint8, device=dev) for _ in range(nt)]
    ss = [torch.empty((LK, H_TOTAL, G), dtype=torch.bfloat16, device=dev) for _ in range(nt)]

    def fb(_i):
        ops.quantize_layers_into(xs, cs, ss, cb, G, 4)
    ms = _time_events(fb, 10)
    byts = nt * LK * H_TOTAL * quant_bytes_per_row(G)
    gbs = byts / (statistics.median(ms) / 1e3) / 1e9
    res["quantize_append_40layers_kv_4680_one_launch"] = {
        "gbs": gbs, "ms": statistics.median(ms), "bytes": byts, "frac_hbm": gbs / peaks["hbm_gbs"],
        "note": "80 distinct inputs (3.8 GB)"}
    del xs, cs, ss
    torch.cuda.empty_cache()

    res["window21_block"] = run_window21_block(dev, peaks)

    # eviction in a window-21 cache (one layer's K and V): the 2 oldest frames after the
    # sink leave, `kv[:, a:b] = kv[:, c:d].clone()` moves the rest down; the reference's
    # dequantize + requantize (default) against the lossless packed move
    L21 = 21 * FRAME
    ev = {}
    for lossless in (False, True):
        kvs = [quant_kv.QuantKVTensor([1, L21, H_TOTAL, D], dev, torch.bfloat16, 4, MODE, SINK, lossless)
               for _ in range(2)]
        for i, c in enumerate(kvs):
            c[:, 0:L21] = synth.make_k(L21, H_TOTAL, seed=80 + i, device=dev)
        a0, c0 = SINK, SINK + 2 * FRAME
        n = L21 - c0

        def fe(_i):
            for c in kvs:
                c[:, a0:a0 + n] = c[:, c0:c0 + n].clone()
        ms = _time_events(fe, 5)
        ev["lossless" if lossless else "requantize"] = {"ms": statistics.median(ms), "tokens_moved": n}
        del kvs
        torch.cuda.empty_cache()
    res["eviction_move_window21_layer_kv"] = ev

    # prefill (rebuild) per block, 40 layers: quantize the window's K and V into
    # the cache, then attention of the window's queries over the window; and the
    # 4 denoising steps' attention (4680 queries) over the same window
    layers = 40
    pre = {}
    for w in (3, 12, 21):
        L = w * FRAME
        ks, vs, qs, caches = [], [], [], []
        for layer in range(layers):
            ks.append(synth.make_k(L, H_TOTAL, seed=300 + layer, device=dev))
            vs.append(synth.make_v(L, H_TOTAL, seed=400 + layer, device=dev))
            qs.append(synth.make_q(1, L, H_TOTAL, seed=500 + layer, device=dev))
            caches.append((quant_kv.QuantKVTensor([1, L, H_TOTAL, D], dev, torch.bfloat16, 4, MODE, SINK),
                           quant_kv.QuantKVTensor([1, L, H_TOTAL, D], dev, torch.bfloat16, 4, MODE, SINK)))
        qd = synth.make_q(1, LQ, H_TOTAL, seed=600, device=dev)
        out = torch.empty((1, L, H_TOTAL, D), dtype=torch.bfloat16, device=dev)
        outd = torch.empty((1, LQ, H_TOTAL, D), dtype=torch.bfloat16, device=dev)

        def block(_i):
            for layer in range(layers):
                tk, tv = caches[layer]
                tk.write_(0, L, ks[layer])
                tv.write_(0, L, vs[layer])
                ops.attention_packed(qs[layer], tk, tv, 0, L, out=out)

        def denoise(_i):
            for _s in range(4):
                for layer in range(layers):
                    tk, tv = caches[layer]
                    ops.attention_packed(qd, tk, tv, 0, L, out=outd)
        ms = _time_events(block, 2, warm=1)
        msd = _time_events(denoise, 1, warm=1)
        fl = layers * attn_flops(1, H_TOTAL, L, L)
        fld = 4 * layers * attn_flops(1, H_TOTAL, LQ, L)
        pre[f"window_{w}"] = {"tokens": L, "prefill_ms_per_block": min(ms),
                              "prefill_attention_tflops": fl / (min(ms) / 1e3) / 1e12,
                              "denoise_4steps_ms_per_block": msd[0],
                              "denoise_attention_tflops": fld / (msd[0] / 1e3) / 1e12}
        del ks, vs, qs, caches, out, outd, qd
        torch.cuda.empty_cache()
    res["prefill"] = pre
    res["prefill_note"] = ("hot path only: per block 40 layers x (quantize-rebuild of the window's K and V + "
                           "attention of the window's queries over the window, non-causal); the reference's "
                           "published prefill times cover the whole 14B forward and are not comparable")
    return res


def run_window21_block(dev, peaks):
    """One block of the resident runtime at window 21 (32,760 tokens, a 1,560-token
    sink), 40 layers, one stream, 40 heads (quant_kv.py:12-14): per layer
      1. rolling eviction of the oldest block after the sink, K and V:
         kv[:, 1560:28080] = kv[:, 6240:32760].clone() (the reference's
         dequantize + requantize; lossless_moves copies packed rows instead)
      2. append of the new 4,680-token block: keys before their rotary embedding
         through the fused rotate + quantize (write_rope_), values by slice write
      3. attention of the block's 4,680 queries over the window.
    Reported per block, with the phases also timed alone."""
    import quant_kv
    from kvq import ops, rope, synth
    S, NB, layers = 21 * FRAME, 3 * FRAME, 40
    fr = rope.freqs(1024, device=dev)
    pos = rope.grid_positions(S, NB, device=dev)
    res = {}
    k_fill = synth.make_k(S, H_TOTAL, seed=800, device=dev)
    v_fill = synth.make_v(S, H_TOTAL, seed=801, device=dev)
    kpre = [synth.make_v(NB, H_TOTAL, seed=810 + i, device=dev) for i in range(layers)]   # keys before rotation
    vnew = [synth.make_v(NB, H_TOTAL, seed=860 + i, device=dev) for i in range(layers)]
    qs = [synth.make_q(1, NB, H_TOTAL, seed=910 + i, device=dev) for i in range(layers)]
    out = torch.empty((1, NB, H_TOTAL, D), dtype=torch.bfloat16, device=dev)
    for lossless in (False, True):
        caches = []
        for _ in range(layers):
            ck = quant_kv.QuantKVTensor([1, S, H_TOTAL, D], dev, torch.bfloat16, 4, MODE, SINK, lossless)
            cv = quant_kv.QuantKVTensor([1, S, H_TOTAL, D], dev, torch.bfloat16, 4, MODE, SINK, lossless)
            quant_kv.write_layers([ck, cv], [k_fill, v_fill], 0, S)
            caches.append((ck, cv))

        def evict(layer):
            for c in caches[layer]:
                c[:, SINK:S - NB] = c[:, SINK + NB:S].clone()

        def append(layer):
            ck, cv = caches[layer]
            ck.write_rope_(S - NB, S, kpre[layer], fr, pos)
            cv[:, S - NB:S] = vnew[layer]

        def attend(layer):
            ck, cv = caches[layer]
            quant_kv.attention(qs[layer], ck[:, 0:S], cv[:, 0:S], out=out)

        def block(_i, phases=(evict, append, attend)):
            for layer in range(layers):
                for f in phases:
                    f(layer)
        ms = min(_time_events(block, 2, warm=1))
        parts = {name: min(_time_events(lambda _i, f=f: block(_i, (f,)), 2, warm=1))
                 for name, f in (("evict", evict), ("append", append), ("attention", attend))}
        fl = layers * attn_flops(1, H_TOTAL, NB, S)
        res["lossless" if lossless else "requantize"] = {
            "ms_per_block": ms, "phase_ms": parts, "attention_tflops": fl / (parts["attention"] / 1e3) / 1e12}
        del caches
        torch.cuda.empty_cache()
    res["workload"] = ("window 21, 40 layers, 1 stream x 40 heads; per layer: eviction of 4680 tokens after the "
                       "1560-token sink (K and V), rotate+quantize append of the new block's keys, append of its "
                       "values, attention of its 4680 queries over the 32760-token window")
    return res


def run_config4(args, dev, world, rank, peaks):
    """The head-sharded workload, strong scaling: window 21 (32,760 tokens, a
    1,560-token sink), 40 layers, 4 independent streams, the 40 heads split
    40/20/10/5 over 1/2/4/8 GPUs. Per block and layer: append of the new
    4,680-token block of K and V at the ring's end (one launch for K and V of the
    4 streams), then attention of the block's 4 x 4,680 queries over the window;
    at N > 1 the attention's epilogue all-gathers the output into every rank
    (alternating two PeerOutputs), and the layer ends with the device-side wait
    for every rank's tiles (what the next layer's input needs). Timed with CUDA
    events, max over ranks; the total work is the same at every N."""
    import quant_kv
    from kvq import ops, shard, synth
    B, S, NB, layers = 4, 21 * FRAME, 3 * FRAME, 40
    h0, h1 = shard.head_range(H_TOTAL, world, rank)
    Hl = h1 - h0
    caches, ks, vs, qs = [], [], [], []
    # the window's contents: one synthetic K and V per stream, quantized into every layer
    k_fill = torch.stack([synth.make_k(S, Hl, seed=2000 + 101 * b + h0, device=dev) for b in range(B)])
    v_fill = torch.stack([synth.make_v(S, Hl, seed=2001 + 101 * b + h0, device=dev) for b in range(B)])
    for layer in range(layers):
        ck = quant_kv.QuantKVTensor([B, S, Hl, D], dev, torch.bfloat16, 4, MODE, SINK)
        cv = quant_kv.QuantKVTensor([B, S, Hl, D], dev, torch.bfloat16, 4, MODE, SINK)
        quant_kv.write_layers([ck, cv], [k_fill, v_fill], 0, S)
        caches.append((ck, cv))
        # the new block of every layer: distinct inputs (> L2 in total at every N)
        ks.append(torch.stack([synth.make_k(NB, Hl, seed=3000 + 7 * layer + b + h0, pos0=S, device=dev)
                               for b in range(B)]))
        vs.append(torch.stack([synth.make_v(NB, Hl, seed=4000 + 7 * layer + b + h0, device=dev) for b in range(B)]))
        qs.append(synth.make_q(B, NB, Hl, seed=5000 + layer + h0, device=dev))
    del k_fill, v_fill
    if world == 1:
        outs = [torch.empty((B, NB, H_TOTAL, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        pos = None
    else:
        pos = [shard.PeerOutputs(torch.empty((B, NB, H_TOTAL, D), dtype=torch.bfloat16, device=dev))
               for _ in range(2)]
    torch.cuda.synchronize()

    def block():
        for layer in range(layers):
            ck, cv = caches[layer]
            quant_kv.write_layers([ck, cv], [ks[layer], vs[layer]], S - NB, S)
            if pos is None:
                ops.attention_packed(qs[layer], ck, cv, 0, S, out=outs[layer % 2])
            else:
                po = pos[layer % 2]
                ops.attention_packed_gather(qs[layer], ck, cv, 0, S, po.ptrs, h0, H_TOTAL)
                po.barrier()

    n_blocks = 2
    block()                                   # warm-up
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_blocks):
        block()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / n_blocks
    status = ops.device_status()
    flops = layers * attn_flops(B, H_TOTAL, NB, S)
    abytes = layers * 2 * B * NB * H_TOTAL * quant_bytes_per_row(len(quant_kv._band_edges(D, MODE)))
    res = {"workload": "window 21 (32760 tokens, 1560-token sink), 40 layers, 4 streams; per layer: append of "
                       "a 4680-token block (K and V) + attention of 4x4680 queries over the window"
                       + ("" if world == 1 else ", output all-gathered in the attention epilogue + device-side "
                          "completion wait"),
           "scaling": "strong", "heads_per_gpu": Hl, "n_gpus": world, "ms_per_block": ms,
           "attention_tflops": flops / (ms / 1e3) / 1e12, "append_bytes_per_block": abytes,
           "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops_sustained"],
           "peak": "sustained bf16 (a block runs for a second and more), of " + peaks["source"],
           "device_status": status}
    if world > 1:
        # the last layer's gathered output against the ranks' own outputs gathered by NCCL
        import torch.distributed as dist
        last = layers - 1
        ck, cv = caches[last]
        ref = shard.assemble_heads(shard.gather_outputs(ops.attention_packed(qs[last], ck, cv, 0, S)))
        ok = torch.tensor([1 if torch.equal(pos[last % 2].local, ref) and status == 0 else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        res["gather_check"] = bool(ok.item())
        torch.cuda.synchronize()
        dist.barrier()
        for p in pos:
            p.close()
        dist.barrier()
    del caches, ks, vs, qs
    torch.cuda.empty_cache()
    return res


def run_profile_case(case: str, launches: int = 6):
    """A small single-GPU case for ncu captures: a few launches of one kernel on
    inputs larger than L2, nothing else."""
    import quant_kv
    import quant_kv_kernels
    from kvq import ops, synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if case in ("attention", "attention_gather", "attention_stats"):
        # window 3 (config 1); the gather instance stores into two local [1, 4680, 80, 128]
        # buffers at head offset 20, the statistics instance also writes the row statistics
        tk, tv, _, _ = make_caches(1, LK, H_TOTAL, SINK, dev, seed=1)
        q = synth.make_q(1, LQ, H_TOTAL, seed=2, device=dev)
        out = torch.empty_like(q)
        bufs = [torch.empty((1, LQ, 2 * H_TOTAL, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        st = torch.empty((1, LQ, H_TOTAL, 4), dtype=torch.float32, device=dev)
        for _ in range(launches):
            if case == "attention":
                ops.attention_packed(q, tk, tv, 0, LK, out=out)
            elif case == "attention_gather":
                ops.attention_packed_gather(q, tk, tv, 0, LK, [b.data_ptr() for b in bufs], 20, 2 * H_TOTAL)
            else:
                ops.attention_packed(q, tk, tv, 0, LK, out=out, stats=st)
    elif case in ("append", "rope"):
        # one block of 4680 tokens x 40 heads: K and V by two launches, by one launch,
        # the rotate + quantize of the keys, and the block's read back (dequantize)
        from kvq import rope
        bands = quant_kv._band_edges(D, MODE)
        G = len(bands)
        cb = quant_kv_kernels.host_chan_band(quant_kv_kernels.build_chan_band(bands, D, "cpu"))
        xs = [synth.make_k(LK, H_TOTAL, seed=70 + i, device=dev) for i in range(2)]
        cs = [torch.empty((LK, H_TOTAL, D // 2), dtype=torch.uint8, device=dev) for _ in range(2)]
        ss = [torch.empty((LK, H_TOTAL, G), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        fr = rope.freqs(1024, device=dev)
        pos = rope.grid_positions(0, LK, device=dev)
        for _ in range(launches):
            if case == "rope":
                ops.rope_quantize_into(xs[0], cs[0], ss[0], cb, G, 4, fr, pos)
                continue
            for t in range(2):
                ops.quantize_into(xs[t], cs[t], ss[t], cb, G, 4)
            ops.quantize_layers_into(xs, cs, ss, cb, G, 4)
            ops.rope_quantize_into(xs[0], cs[0], ss[0], cb, G, 4, fr, pos)
            ops.dequantize_into(cs[1], ss[1], xs[1], cb, G, 4)
    elif case == "requantize":
        # the window-21 eviction of one block after the 1560-token sink in one layer
        # tensor, through the public API: a packed snapshot copy + one kvq_requantize
        S = 21 * FRAME
        c = quant_kv.QuantKVTensor([1, S, H_TOTAL, D], dev, torch.bfloat16, 4, MODE, SINK)
        c[:, 0:S] = synth.make_k(S, H_TOTAL, seed=5, device=dev).unsqueeze(0)
        for _ in range(launches):
            c[:, SINK:S - FRAME * 3] = c[:, SINK + FRAME * 3:S].clone()
    else:
        bands = quant_kv._band_edges(D, MODE)
        G = len(bands)
        cb = quant_kv_kernels.host_chan_band(quant_kv_kernels.build_chan_band(bands, D, "cpu"))
        L = 21 * FRAME
        x = synth.make_k(L, H_TOTAL, seed=3, device=dev)
        codes = torch.empty((L, H_TOTAL, D // 2), dtype=torch.uint8, device=dev)
        scales = torch.empty((L, H_TOTAL, G), dtype=torch.bfloat16, device=dev)
        for _ in range(launches):
            ops.quantize_into(x, codes, scales, cb, G, 4)
            if case == "dequantize":
                ops.dequantize_into(codes, scales, x, cb, G, 4)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "launches": launches, "status": ops.device_status()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-extras", action="store_true", help="skip quantize / prefill extras")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the window-21 / 40-layer / 4-stream head-sharded block")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--gather", default="fused", choices=("fused", "nccl"),
                    help="N > 1: all-gather of the output in the attention epilogue, or by NCCL")
    ap.add_argument("--profile-case", choices=("attention", "attention_gather", "attention_stats", "quantize",
                                               "dequantize", "append", "rope", "requantize"),
                    help="run a few launches of one kernel for an ncu capture and exit")
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args.profile_case)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
