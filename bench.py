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
    background thread while the timed region runs."""

    def __init__(self, device: int, period_s: float = 0.02):
        self.period = period_s
        self.samples: list[tuple[int, int, float]] = []
        self.max_mhz = None
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
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except Exception:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                pw = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0
                self.samples.append((mhz, rs, pw))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml unavailable" if self._h is None else "nvml"}
        mhz = [s[0] for s in self.samples]
        bits = 0
        for s in self.samples:
            bits |= int(s[1])
        reasons = sorted(n for b, n in _REASONS.items() if bits & b and n != "gpu_idle")
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz), "power_w_max": round(max(s[2] for s in self.samples), 1),
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
            # full-width output of the set on every rank, mapped into every peer
            peers.append(shard.PeerOutputs(torch.empty((B, LQ, H_TOTAL, D), dtype=torch.bfloat16, device=dev)))
    gbuf = shard.gather_buffer(sets[0][3], world) if world > 1 else None
    torch.cuda.synchronize()

    def step(i, kev=None):
        q, tk, tv, out = sets[i % N_SETS]
        if kev is not None:
            kev[0].record()
        if fused:
            ops.attention_packed_gather(q, tk, tv, 0, LK, peers[i % N_SETS].ptrs, h0, H_TOTAL)
        else:
            ops.attention_packed(q, tk, tv, 0, LK, out=out)
        if kev is not None:
            kev[1].record()
        if world > 1 and not fused:
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
        e0.record()
        for i in range(args.steps):
            step(i, kevs[i])
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    k_ms = [a.elapsed_time(b) for a, b in kevs]
    k_mean = sum(k_ms) / len(k_ms)
    status = ops.device_status()
    if status != 0:
        raise SystemExit(f"device status {status}: a kernel wait timed out; results invalid")
    flops_rank = attn_flops(B, Hl, LQ, LK)
    value = world * flops_rank * args.steps / (t_ms / 1e3) / 1e12
    achieved = flops_rank / (k_mean / 1e3) / 1e12

    # ---- end to end through the public API, host buffers, copies timed
    e2e = run_e2e(args, dev, world, B, Hl, h0, gbuf)

    extra = {}
    cpu = None
    if world == 1 and not args.no_extras:
        extra = run_extras(dev, peaks)
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
                     "peak_source": f"{peaks['source']} bf16 dense (burst), of {peaks['source']}"},
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "extra": extra,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()          # every rank is done storing into the peers' buffers
        for p in peers:
            p.close()
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, dev, world, B, Hl, h0, gbuf):
    """Same metric through quant_kv (the drop-in API), from host memory: per step,
    copy q, k, v of the block from pinned host memory, quantize-append K and V
    into the caches (slice write), attention over the window, copy the output
    back to the host. Three streams pipeline consecutive steps (upload of step
    i+1 and download of step i-1 overlap the compute of step i); every step still
    moves all of its inputs and its output across PCIe inside the timed region."""
    import quant_kv
    from kvq import shard, synth
    tk = quant_kv.QuantKVTensor([B, LK, Hl, D], dev, torch.bfloat16, 4, MODE, SINK)
    tv = quant_kv.QuantKVTensor([B, LK, Hl, D], dev, torch.bfloat16, 4, MODE, SINK)
    nb = 2
    qh = [synth.make_q(B, LQ, Hl, seed=11 + i).pin_memory() for i in range(nb)]
    kh = [torch.stack([synth.make_k(LK, Hl, seed=12 + b + i) for b in range(B)]).pin_memory() for i in range(nb)]
    vh = [torch.stack([synth.make_v(LK, Hl, seed=13 + b + i) for b in range(B)]).pin_memory() for i in range(nb)]
    oh = [torch.empty((B, LQ, Hl, D), dtype=torch.bfloat16).pin_memory() for _ in range(nb)]
    qd = [torch.empty_like(qh[0], device=dev) for _ in range(nb)]
    kd = [torch.empty_like(kh[0], device=dev) for _ in range(nb)]
    vd = [torch.empty_like(vh[0], device=dev) for _ in range(nb)]
    od = [torch.empty_like(qd[0]) for _ in range(nb)]
    s_up, s_cmp, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    up_done, cmp_done, dn_done = {}, {}, {}

    def step(i):
        j = i % nb
        with torch.cuda.stream(s_up):
            if i - nb in cmp_done:
                s_up.wait_event(cmp_done[i - nb])      # step i-2 finished reading buffer j
            qd[j].copy_(qh[j], non_blocking=True)
            kd[j].copy_(kh[j], non_blocking=True)
            vd[j].copy_(vh[j], non_blocking=True)
            up_done[i] = ev()
            up_done[i].record(s_up)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(up_done[i])
            if i - nb in dn_done:
                s_cmp.wait_event(dn_done[i - nb])      # output buffer j downloaded
            tk[:, 0:LK] = kd[j]
            tv[:, 0:LK] = vd[j]
            quant_kv.attention(qd[j], tk[:, 0:LK], tv[:, 0:LK], out=od[j])
            if world > 1:
                shard.gather_outputs(od[j], gbuf)
            cmp_done[i] = ev()
            cmp_done[i].record(s_cmp)
        with torch.cuda.stream(s_dn):
            s_dn.wait_event(cmp_done[i])
            oh[j].copy_(od[j], non_blocking=True)
            dn_done[i] = ev()
            dn_done[i].record(s_dn)

    n = max(3, min(args.steps, 20))
    for i in range(max(2, args.warmup)):
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
    flops = world * attn_flops(B, Hl, LQ, LK) * n
    h2d = (qh[0].numel() + kh[0].numel() + vh[0].numel()) * 2
    return {"value": flops / (t / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": oh[0].numel() * 2, "steps": n, "ms_per_step": t / n,
            "path": "pinned H2D of q,k,v -> QuantKVTensor slice writes (quantize-append) -> "
                    "quant_kv.attention -> D2H of the output; upload, compute and download of "
                    "consecutive steps on three streams"}


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
        ms = _time_events(fq, 20)
        byts = 2 * L * H_TOTAL * quant_bytes_per_row(G)
        gbs = byts / (statistics.median(ms) / 1e3) / 1e9
        res[f"quantize_{name}"] = {"gbs": gbs, "ms": statistics.median(ms), "bytes": byts,
                                   "frac_hbm": gbs / peaks["hbm_gbs"]}
        outs = [torch.empty_like(x) for x in xs]

        def fd(i):
            for t in range(2):
                j = (2 * i + t) % 4
                ops.dequantize_into(cs[j], ss[j], outs[j], cb, G, 4)
        ms = _time_events(fd, 20)
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
    ms = _time_events(fr_q, 20)
    byts = LK * H_TOTAL * quant_bytes_per_row(G)
    res["rope_quantize_append_block_4680_per_tensor"] = {
        "gbs": byts / (statistics.median(ms) / 1e3) / 1e9, "ms": statistics.median(ms), "bytes": byts}
    del xs, cs, ss
    torch.cuda.empty_cache()

    # the append of one block to all 40 layers x {K, V} in one launch (kvq_rebuild_layers)
    nt = 80
    xs = [synth.make_k(LK, H_TOTAL, seed=700 + (i % 8), device=dev) for i in range(8)]
    cs = [torch.empty((LK, H_TOTAL, D // 2), dtype=torch.uint8, device=dev) for _ in range(nt)]
    ss = [torch.empty((LK, H_TOTAL, G), dtype=torch.bfloat16, device=dev) for _ in range(nt)]
    xin = [xs[i % 8] for i in range(nt)]

    def fb(_i):
        ops.quantize_layers_into(xin, cs, ss, cb, G, 4)
    ms = _time_events(fb, 10)
    byts = nt * LK * H_TOTAL * quant_bytes_per_row(G)
    gbs = byts / (statistics.median(ms) / 1e3) / 1e9
    res["quantize_append_40layers_kv_4680_one_launch"] = {
        "gbs": gbs, "ms": statistics.median(ms), "bytes": byts, "frac_hbm": gbs / peaks["hbm_gbs"],
        "note": "8 distinct inputs cycled over the 80 tensors (inputs 384 MB > L2)"}
    del xs, cs, ss, xin
    torch.cuda.empty_cache()

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


def run_profile_case(case: str, launches: int = 6):
    """A small single-GPU case for ncu captures: a few launches of one kernel on
    inputs larger than L2, nothing else."""
    import quant_kv
    import quant_kv_kernels
    from kvq import ops, synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if case == "attention":
        tk, tv, _, _ = make_caches(1, LK, H_TOTAL, SINK, dev, seed=1)
        q = synth.make_q(1, LQ, H_TOTAL, seed=2, device=dev)
        out = torch.empty_like(q)
        for _ in range(launches):
            ops.attention_packed(q, tk, tv, 0, LK, out=out)
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
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--gather", default="fused", choices=("fused", "nccl"),
                    help="N > 1: all-gather of the output in the attention epilogue, or by NCCL")
    ap.add_argument("--profile-case", choices=("attention", "quantize", "dequantize"),
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
