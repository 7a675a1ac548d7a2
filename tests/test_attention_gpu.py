"""Fused int4-KV attention against the oracle: the reference's window read
(dequantize + bf16 sink overlay, quant_kv.py:189-199) followed by softmax
attention in fp32. Tolerance: max-abs <= 2e-2 and mean-abs <= 2e-3 of the
fp32 result, per call."""
import math

import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import kvq_oracle as ko

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _t(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def _u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_window(x_bits, bands, sink, lo, hi):
    """Reference read of tokens [lo, hi) of a cache holding x (bf16 bits [S,H,D])."""
    codes, scales = c_oracle.quantize(x_bits, bands)
    w = c_oracle.dequantize(codes[lo:hi], scales[lo:hi], bands, x_bits.shape[-1])
    if sink > lo:
        e = min(hi, sink)
        w[: e - lo] = x_bits[lo:e]
    return w


def _oracle_attention(q_bits, kw, vw, scale=None, chunk=2048):
    """fp32 softmax attention per (stream, head) with torch on the CPU; q [B,Lq,H,D].
    Queries go in chunks (fp32 logits, softmax and products), so that windows of
    32,760 tokens need neither the whole logit matrix in memory nor the slow path
    of the CPU's fused attention."""
    q = torch.from_numpy(ko.bf16_to_f32(q_bits))
    k = torch.from_numpy(ko.bf16_to_f32(kw))
    v = torch.from_numpy(ko.bf16_to_f32(vw))
    B, Lq, H, D = q.shape
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.empty((B, H, Lq, D), dtype=torch.float32)
    for b in range(B):
        kb, vb = k[b].transpose(0, 1), v[b].transpose(0, 1)          # [H, Lk, D]
        qb = q[b].transpose(0, 1)                                     # [H, Lq, D]
        for i in range(0, Lq, chunk):
            s = torch.matmul(qb[:, i:i + chunk], kb.transpose(1, 2)) * sc
            out[b, :, i:i + chunk] = torch.matmul(torch.softmax(s, dim=-1), vb)
    return out.transpose(1, 2).contiguous().numpy()


def _check(o_gpu, o_ref, what):
    err = np.abs(o_gpu.float().cpu().numpy() - o_ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, f"{what}: max {err.max():.3e} mean {err.mean():.3e}"
    return err


def _make_caches(B, S, H, mode, sink, seed=0):
    import quant_kv
    from kvq import synth
    tk = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, mode, sink)
    tv = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, mode, sink)
    ks = [synth.make_k(S, H, seed=seed + 10 * b) for b in range(B)]
    vs = [synth.make_v(S, H, seed=seed + 10 * b + 1) for b in range(B)]
    tk[:, 0:S] = torch.stack(ks).cuda()
    tv[:, 0:S] = torch.stack(vs).cuda()
    return tk, tv, [_u16(k) for k in ks], [_u16(v) for v in vs]


def _run_case(B, S, H, Lq, lo, hi, sink, mode="bands4", seed=0):
    import quant_kv
    from kvq import synth
    tk, tv, kb, vb = _make_caches(B, S, H, mode, sink, seed)
    q = synth.make_q(B, Lq, H, seed=seed + 5)
    o = quant_kv.attention(q.cuda(), tk[:, lo:hi], tv[:, lo:hi])
    bands = ko.band_edges(128, mode)
    kw = np.stack([_oracle_window(kb[b], bands, sink, lo, hi) for b in range(B)])
    vw = np.stack([_oracle_window(vb[b], bands, sink, lo, hi) for b in range(B)])
    ref = _oracle_attention(_u16(q), kw, vw)
    return _check(o, ref, f"B{B} S{S} H{H} Lq{Lq} [{lo},{hi}) sink{sink} {mode}")


def test_golden_reference_attention(golden):
    import quant_kv
    g = golden("attention_small.npz")
    for name in ("a", "b", "c"):
        S, sink, Lq, lo, hi = (int(v) for v in g[f"{name}/meta"])
        tk = quant_kv.QuantKVTensor([1, S, 2, 128], "cuda", torch.bfloat16, 4, "bands4", sink)
        tv = quant_kv.QuantKVTensor([1, S, 2, 128], "cuda", torch.bfloat16, 4, "bands4", sink)
        tk[:, 0:S] = _t(g[f"{name}/k"]).unsqueeze(0).cuda()
        tv[:, 0:S] = _t(g[f"{name}/v"]).unsqueeze(0).cuda()
        # the packed window is the reference's window, bit for bit
        np.testing.assert_array_equal(_u16(tk[:, lo:hi].materialize()), g[f"{name}/kwin"])
        o = quant_kv.attention(_t(g[f"{name}/q"]).cuda(), tk[:, lo:hi], tv[:, lo:hi])
        _check(o, g[f"{name}/out_fp32"], name)


def test_config1_full_size():
    """Q [1, 4680, 40, 128] over a 4680-token int4 window with a 1560-token sink."""
    err = _run_case(1, 4680, 40, 4680, 0, 4680, 1560)
    assert err.mean() < 5e-4


@pytest.mark.parametrize("B,S,H,Lq,sink", [
    (1, 18720, 2, 18720, 1560),   # window 12, prefill: the window's queries over the window
    (1, 32760, 2, 4680, 1560),    # window 21, denoise step: one block's queries over the window
    (1, 32760, 1, 32760, 1560),   # window 21, prefill
    (4, 32760, 1, 4680, 1560),    # window 21 with 4 streams (the head-sharded workload's shape)
])
def test_long_windows(B, S, H, Lq, sink):
    """The window lengths the prefill and denoise timings use: 293 and 512 KV
    tiles per row, where the online softmax's lazy rescale and the fp32 row sums
    run longest (reference window read quant_kv.py:189-199 at S = 32,760,
    quant_kv.py:238-241)."""
    err = _run_case(B, S, H, Lq, 0, S, sink, seed=S + Lq + B)
    assert err.mean() < 5e-4


@pytest.mark.parametrize("B,S,H,Lq,lo,hi,sink", [
    (1, 200, 3, 1, 0, 200, 0),          # one query row
    (1, 200, 3, 130, 0, 1, 0),          # one key
    (1, 300, 2, 129, 17, 283, 64),      # window crossing the sink border, ragged tiles
    (2, 256, 4, 64, 0, 256, 128),       # streams, window = sink + body
    (1, 512, 2, 200, 0, 100, 200),      # window entirely inside the sink
    (3, 700, 5, 300, 100, 700, 0),      # no sink, odd head count
])
def test_ragged_windows(B, S, H, Lq, lo, hi, sink):
    _run_case(B, S, H, Lq, lo, hi, sink, seed=B + S + H)


@pytest.mark.parametrize("mode", ["bands", "bands2", "blind32", "blind64"])
def test_group_layouts(mode):
    _run_case(1, 640, 4, 256, 0, 640, 128, mode=mode, seed=7)


def test_custom_scale_and_out_buffer():
    import quant_kv
    from kvq import synth
    tk, tv, kb, vb = _make_caches(1, 384, 2, "bands4", 0, seed=3)
    q = synth.make_q(1, 100, 2, seed=4).cuda()
    out = torch.full((1, 100, 2, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    o = quant_kv.attention(q, tk[:, 0:384], tv[:, 0:384], softmax_scale=0.05, out=out)
    assert o.data_ptr() == out.data_ptr()
    bands = ko.band_edges(128, "bands4")
    ref = _oracle_attention(_u16(q), _oracle_window(kb[0], bands, 0, 0, 384)[None],
                            _oracle_window(vb[0], bands, 0, 0, 384)[None], scale=0.05)
    _check(o, ref, "scale 0.05")


def test_padded_q_and_out_views():
    """q and out as views into wider buffers (a padding head on each side, so the
    token stride is (H + 2) * 128): the output tile is stored by TMA through a map
    that covers the H real heads and Lq rows of each stream, so the padding heads
    keep their contents and no stream's partial last tile spills into the next."""
    import quant_kv
    from kvq import synth
    B, S, H, Lq, sink = 2, 300, 3, 200, 64
    tk, tv, kb, vb = _make_caches(B, S, H, "bands4", sink, seed=11)
    q = synth.make_q(B, Lq, H, seed=12)
    qbuf = torch.zeros((B, Lq, H + 2, 128), dtype=torch.bfloat16, device="cuda")
    qbuf[:, :, 1:H + 1] = q.cuda()
    obuf = torch.full((B, Lq, H + 2, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    o = quant_kv.attention(qbuf[:, :, 1:H + 1], tk[:, 0:S], tv[:, 0:S], out=obuf[:, :, 1:H + 1])
    assert o.data_ptr() == obuf[:, :, 1:H + 1].data_ptr()
    bands = ko.band_edges(128, "bands4")
    kw = np.stack([_oracle_window(kb[b], bands, sink, 0, S) for b in range(B)])
    vw = np.stack([_oracle_window(vb[b], bands, sink, 0, S) for b in range(B)])
    _check(obuf[:, :, 1:H + 1], _oracle_attention(_u16(q), kw, vw), "padded q and out")
    assert torch.all(obuf[:, :, 0] == 7.0) and torch.all(obuf[:, :, H + 1] == 7.0), "padding heads written"


def test_plain_tensors_are_rejected_and_status_is_clean():
    import quant_kv
    from kvq import ops
    q = torch.zeros((1, 8, 2, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(TypeError):
        quant_kv.attention(q, q, q)
    assert ops.device_status() == 0


def _oracle_window_bits(x_bits, bands, sink, lo, hi, bits):
    codes, scales = c_oracle.quantize(x_bits, bands, bits=bits)
    w = c_oracle.dequantize(codes[lo:hi], scales[lo:hi], bands, x_bits.shape[-1], bits=bits)
    if sink > lo:
        e = min(hi, sink)
        w[: e - lo] = x_bits[lo:e]
    return w


@pytest.mark.parametrize("mode", ["bands4", "bands", "blind64"])
@pytest.mark.parametrize("B,S,H,Lq,lo,hi,sink", [(1, 4680, 40, 4680, 0, 4680, 1560),
                                                 (2, 900, 3, 333, 100, 877, 300)])
def test_attention_int8_k_int4_v(mode, B, S, H, Lq, lo, hi, sink):
    """K8V4 (bench_qkv.py:160): int8 K codes (+128 offset) and int4 V in one kernel."""
    import quant_kv
    from kvq import synth
    tk = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 8, mode, sink)
    tv = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, mode, sink)
    ks = [synth.make_k(S, H, seed=31 + 10 * b) for b in range(B)]
    vs = [synth.make_v(S, H, seed=32 + 10 * b) for b in range(B)]
    tk[:, 0:S] = torch.stack(ks).cuda()
    tv[:, 0:S] = torch.stack(vs).cuda()
    q = synth.make_q(B, Lq, H, seed=33)
    o = quant_kv.attention(q.cuda(), tk[:, lo:hi], tv[:, lo:hi])
    bands = ko.band_edges(128, mode)
    kw = np.stack([_oracle_window_bits(_u16(ks[b]), bands, sink, lo, hi, 8) for b in range(B)])
    vw = np.stack([_oracle_window_bits(_u16(vs[b]), bands, sink, lo, hi, 4) for b in range(B)])
    # the kernel reads exactly the reference's window: check the int8 K read itself bit-exact
    kread = tk[:, lo:hi].materialize()
    assert np.array_equal(_u16(kread), kw)
    _check(o, _oracle_attention(_u16(q), kw, vw), f"K8V4 {mode} B{B} S{S} [{lo},{hi})")
    assert quant_kv._ops.device_status() == 0


def test_attention_rejects_int8_v():
    import quant_kv
    from kvq import synth
    tk = quant_kv.QuantKVTensor([1, 256, 2, 128], "cuda", torch.bfloat16, 4, "bands4", 0)
    tv = quant_kv.QuantKVTensor([1, 256, 2, 128], "cuda", torch.bfloat16, 8, "bands4", 0)
    q = synth.make_q(1, 16, 2, seed=1).cuda()
    with pytest.raises(ValueError):
        quant_kv.attention(q, tk[:, 0:256], tv[:, 0:256])


@pytest.mark.parametrize("B,S,H,Lq,lo,hi,sink,mode", [(1, 4680, 8, 600, 0, 4680, 1560, "bands4"),
                                                      (2, 900, 3, 333, 100, 877, 300, "bands"),
                                                      (1, 700, 2, 129, 0, 700, 0, "blind64")])
def test_attention_stats_match_fp32_softmax(B, S, H, Lq, lo, hi, sink, mode):
    """The side output against the reference probe's fp32 arithmetic on the same
    (dequantized) window: entropy, max weight and sink mass (probe_attention.py:
    102-121, without the probe's 1e-9 in the log), plus the log-sum-exp."""
    import quant_kv
    from kvq import synth
    tk, tv, kb, vb = _make_caches(B, S, H, mode, sink, seed=41)
    q = synth.make_q(B, Lq, H, seed=43)
    out, st = quant_kv.attention_stats(q.cuda(), tk[:, lo:hi], tv[:, lo:hi])
    bands = ko.band_edges(128, mode)
    kw = np.stack([_oracle_window(kb[b], bands, sink, lo, hi) for b in range(B)])
    vw = np.stack([_oracle_window(vb[b], bands, sink, lo, hi) for b in range(B)])
    _check(out, _oracle_attention(_u16(q), kw, vw), "attention output of the statistics kernel")
    qf = torch.from_numpy(ko.bf16_to_f32(_u16(q))).double()
    kf = torch.from_numpy(ko.bf16_to_f32(kw)).double()
    logits = torch.einsum("bqhd,bkhd->bqhk", qf, kf) / math.sqrt(128)
    lse = torch.logsumexp(logits, -1)
    p = torch.softmax(logits, -1)
    ent = -(p * torch.log(p.clamp_min(1e-300))).sum(-1)
    pmax = p.max(-1).values
    ns = max(0, min(hi, sink) - lo)
    anchor = p[..., :ns].sum(-1)
    got = st.double().cpu()
    assert (got[..., 0] - lse).abs().max() < 2e-3
    assert (got[..., 1] - ent).abs().max() < 2e-3
    assert (got[..., 2] - pmax).abs().max() < 2e-3
    assert (got[..., 3] - anchor).abs().max() < 2e-3
    assert quant_kv._ops.device_status() == 0
