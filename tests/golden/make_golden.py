"""Generates the golden fixtures under tests/golden/ from the REFERENCE itself.

Run in a container where the reference checkout is present, naming it by
argument or by the environment variable KREA_REFERENCE:
    python tests/golden/make_golden.py /path/to/krea-realtime-bench
It imports the reference's quant_kv.py (torch path on CPU, use_kernels False)
and records, for seeded inputs, the reference's codes, scales, dequantized
windows (with the bf16 sink overlay) and the dequant-then-fp32-SDPA attention.
The inputs are stored in the fixtures too, so the tests never regenerate them.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KREA_REFERENCE", "")
if not REF or not os.path.isfile(os.path.join(REF, "quant_kv.py")):
    raise SystemExit("usage: make_golden.py /path/to/krea-realtime-bench (or set KREA_REFERENCE)")
sys.path.insert(0, REF)
import quant_kv as ref  # noqa: E402  (the reference module)

assert os.path.abspath(ref.__file__).startswith(os.path.abspath(REF)), ref.__file__
sys.path.insert(1, os.path.join(os.path.dirname(os.path.dirname(HERE)), "krea-realtime-bench_b200"))
from kvq import synth  # noqa: E402

MODES = ("bands", "bands2", "bands4", "blind32", "blind64", "bands3", "bands8", "blind16")


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def ref_tensor(S, H, D, bits, mode, sink):
    t = ref.QuantKVTensor([1, S, H, D], "cpu", torch.bfloat16, bits, mode, sink)
    assert not t.use_kernels
    return t


def edge_input() -> torch.Tensor:
    """Hand-built rows that hit the corners of the arithmetic."""
    H, D = 1, 128
    rows = []
    z = torch.zeros(D)
    rows.append(z.clone())                                     # all zero -> scale 1
    r = torch.zeros(D); r[5] = -0.0; r[50] = 3.0; rows.append(r)  # one nonzero band
    # exact ties: amax = 7 * 2^k so s is exact and x = (k + 0.5) * s is representable
    r = torch.zeros(D)
    for c in range(D):
        r[c] = ((c % 15) - 7 + 0.5) * 0.25 if c % 15 != 14 else 1.75
    rows.append(r)
    r = torch.zeros(D)
    for c in range(D):
        r[c] = ((c % 8) + 0.5) * (1.0 if c % 2 else -1.0)
    r[0::11] = 7.0
    rows.append(r)
    r = torch.full((D,), 3.0e38); r[1::2] = -1.0e38; rows.append(r)  # near bf16 max
    r = torch.full((D,), 2.0 ** -130); r[3::4] = -(2.0 ** -133); rows.append(r)  # subnormals
    r = torch.full((D,), 1.0e-35); r[::3] = 4.0e-36; rows.append(r)  # tiny normal scales
    r = torch.linspace(-5, 5, D); rows.append(r)
    r = torch.ones(D) * -2.5; rows.append(r)
    x = torch.stack(rows).reshape(len(rows), H, D).to(torch.bfloat16)
    return x


def quant_fixture():
    cases = {
        "outlier": synth.make_outlier(24, 8, seed=0),
        "rope_k": synth.make_k(40, 6, seed=3, pos0=1540),
        "v": synth.make_v(24, 5, seed=4),
        "edge": edge_input(),
    }
    out = {}
    for name, x in cases.items():
        L, H, D = x.shape
        out[f"{name}/x"] = bits16(x)
        for mode in MODES:
            for bits in (4, 8):
                if bits == 8 and mode not in ("bands", "bands4", "blind64"):
                    continue
                t = ref_tensor(L, H, D, bits, mode, 0)
                p, s = t._quantize(x)
                d = t._dequantize(p, s)
                out[f"{name}/{mode}/int{bits}/codes"] = p.numpy().copy()
                out[f"{name}/{mode}/int{bits}/scales"] = bits16(s)
                if mode in MODES[:5]:
                    out[f"{name}/{mode}/int{bits}/deq"] = bits16(d)
    np.savez_compressed(os.path.join(HERE, "quant_cases.npz"), **out)
    return out


def proxy_fixture():
    """Scripted slice writes/reads on the reference proxy with a bf16 sink."""
    S, H, D, sink = 96, 3, 128, 40
    out = {}
    for mode in ("bands", "bands4"):
        t = ref_tensor(S, H, D, 4, mode, sink)
        a = synth.make_k(40, H, seed=5, pos0=0)
        b = synth.make_k(56, H, seed=6, pos0=40)
        out[f"{mode}/w0"] = bits16(a)
        out[f"{mode}/w1"] = bits16(b)
        t[:, 0:40] = a.unsqueeze(0)
        t[:, 40:96] = b.unsqueeze(0)
        for lo, hi in ((0, 96), (20, 60), (50, 70), (39, 41), (0, 1)):
            out[f"{mode}/read_{lo}_{hi}"] = bits16(t[:, lo:hi][0])
        # the runtime's rolling eviction: kv[:, a:b] = kv[:, c:d].clone()
        t[:, 30:60] = t[:, 60:90].clone()
        out[f"{mode}/after_evict"] = bits16(t[:, 0:96][0])
        out[f"{mode}/packed"] = t.packed.numpy().copy()
        out[f"{mode}/scales"] = bits16(t.scales)
        out[f"{mode}/sink"] = bits16(t.sink)
        e = t[:, 10:10]
        out[f"{mode}/empty_shape"] = np.array(e.shape, dtype=np.int64)
        t.zero_()
        out[f"{mode}/after_zero"] = bits16(t[:, 0:12][0])
    np.savez_compressed(os.path.join(HERE, "proxy_semantics.npz"), **out)


def attention_fixture():
    """Reference window read (dequant + sink overlay) then fp32 SDPA."""
    H, D = 2, 128
    out = {}
    for name, (S, sink, Lq, lo, hi) in {"a": (80, 16, 24, 0, 80), "b": (80, 16, 17, 8, 72),
                                        "c": (70, 0, 33, 0, 70)}.items():
        k = synth.make_k(S, H, seed=21, pos0=0)
        v = synth.make_v(S, H, seed=22)
        q = synth.make_q(1, Lq, H, seed=23)
        tk = ref_tensor(S, H, D, 4, "bands4", sink)
        tv = ref_tensor(S, H, D, 4, "bands4", sink)
        tk[:, 0:S] = k.unsqueeze(0)
        tv[:, 0:S] = v.unsqueeze(0)
        kw, vw = tk[:, lo:hi], tv[:, lo:hi]
        o = torch.nn.functional.scaled_dot_product_attention(
            q.float().transpose(1, 2), kw.float().transpose(1, 2), vw.float().transpose(1, 2))
        o = o.transpose(1, 2).contiguous()
        out[f"{name}/k"] = bits16(k)
        out[f"{name}/v"] = bits16(v)
        out[f"{name}/q"] = bits16(q)
        out[f"{name}/meta"] = np.array([S, sink, Lq, lo, hi], dtype=np.int64)
        out[f"{name}/kwin"] = bits16(kw)
        out[f"{name}/vwin"] = bits16(vw)
        out[f"{name}/out_fp32"] = o.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "attention_small.npz"), **out)


if __name__ == "__main__":
    torch.set_num_threads(4)
    quant_fixture()
    proxy_fixture()
    attention_fixture()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
