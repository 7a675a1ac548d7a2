"""Times the reference's own CPU path beside the oracle port, on the same
sample and the same host threads (test infrastructure; run where the
reference checkout exists, e.g. `python oracle/time_reference_cpu.py
/path/to/krea-realtime-bench`; the reference cannot travel to the GPU box,
so bench.py's CPU legs time the port).

Sample: 2 of 40 heads of the window-3 workload (4680 tokens, 1560-token sink,
bands4): int4 quantize of K and V, the window read (dequantize + bf16 sink
overlay), fp32 attention of 4680 queries. Reference: QuantKVTensor on the CPU
(torch path, quant_kv.py:142-176 and 189-215) and torch SDPA; port: the C
oracle (oracle/kvq_oracle.c) and the same SDPA. Prints one JSON line with
both rates and the attention flops per second they imply.
"""
from __future__ import annotations

import json
import os
import sys
import time

import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "krea-realtime-bench_b200")]
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KREA_REFERENCE", "")
if not REF or not os.path.isfile(os.path.join(REF, "quant_kv.py")):
    raise SystemExit("usage: time_reference_cpu.py /path/to/krea-realtime-bench (or set KREA_REFERENCE)")
sys.path.insert(0, REF)
import quant_kv as ref  # noqa: E402  (the reference module)

assert os.path.abspath(ref.__file__).startswith(os.path.abspath(REF)), ref.__file__

from kvq import synth  # noqa: E402
from oracle import c_oracle  # noqa: E402
from oracle import kvq_oracle as ko  # noqa: E402

L, SINK, H, MODE = 4680, 1560, 2, "bands4"


def sample_inputs():
    k = synth.make_k(L, H, seed=1)
    v = synth.make_v(L, H, seed=2)
    q = synth.make_q(1, L, H, seed=3).float()
    return k, v, q


def sdpa(q, kw, vw):
    return torch.nn.functional.scaled_dot_product_attention(q[0].transpose(0, 1), kw.transpose(0, 1),
                                                            vw.transpose(0, 1))


def run_reference(k, v, q):
    wins = []
    for x in (k, v):
        t = ref.QuantKVTensor([1, L, H, 128], "cpu", torch.bfloat16, 4, MODE, SINK)
        assert not t.use_kernels
        t[:, 0:L] = x.unsqueeze(0)
        wins.append(t[:, 0:L][0].float())
    return sdpa(q, *wins)


def run_port(k, v, q, threads):
    bands = ko.band_edges(128, MODE)
    wins = []
    for x in (k, v):
        xb = x.view(torch.int16).numpy().view("uint16")
        c, s = c_oracle.quantize(xb, bands, 4, threads)
        w = c_oracle.dequantize(c, s, bands, 128, 4, threads)
        w[:SINK] = xb[:SINK]
        wins.append(torch.from_numpy(ko.bf16_to_f32(w)))
    return sdpa(q, *wins)


def timed(fn, reps):
    fn()
    t0 = time.perf_counter()
    for _ in range(reps):
        out = fn()
    return (time.perf_counter() - t0) / reps, out


def main():
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    k, v, q = sample_inputs()
    t_ref, o_ref = timed(lambda: run_reference(k, v, q), 5)
    t_port, o_port = timed(lambda: run_port(k, v, q, threads), 5)
    flops = 4.0 * H * L * L * 128
    print(json.dumps({
        "sample": f"{H} of 40 heads: int4 quantize of K and V ({L} tokens, {MODE}), window read with a "
                  f"{SINK}-token bf16 sink, fp32 SDPA of {L} queries",
        "cores": threads, "cpu": torch.backends.cpu.get_cpu_capability(),
        "reference_torch_s": t_ref, "port_s": t_port,
        "reference_tflops": flops / t_ref / 1e12, "port_tflops": flops / t_port / 1e12,
        "same_output": bool(torch.equal(o_ref, o_port)),
    }))


if __name__ == "__main__":
    main()
