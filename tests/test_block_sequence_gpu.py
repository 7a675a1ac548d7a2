"""One block of the resident runtime at window 21 (32,760 tokens per stream, a
1,560-token bf16 sink), through the drop-in API, against the oracle's
QuantKVRef run through the same steps (quant_kv.py:12-14):

  1. rolling eviction   kv[:, sink:S-n] = kv[:, sink+n:S].clone()   (quant_kv.py:13,
                        dequantize + requantize as quant_kv.py:189-218 do it; or,
                        with lossless_moves, a copy of the packed rows)
  2. slice write        keys of the new block before their rotary embedding,
                        rotated and quantized in one kernel (write_rope_), and the
                        values, at [S-n, S)                        (quant_kv.py:12)
  3. slice read         attention(q, k[:, 0:S], v[:, 0:S])          (quant_kv.py:14)

for two layers of two heads. Codes, scales and sink rows are bit-exact; the
attention output is within max-abs 2e-2 / mean-abs 2e-3 of fp32 attention on
the oracle's window."""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as ko

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
S, SINK, N, H = 21 * 1560, 1560, 3 * 1560, 2


def _u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _attention_fp32(q_bits, kw, vw, chunk=2048):
    q = torch.from_numpy(ko.bf16_to_f32(q_bits))[0].transpose(0, 1)   # [H, Lq, D]
    k = torch.from_numpy(ko.bf16_to_f32(kw))[0].transpose(0, 1)
    v = torch.from_numpy(ko.bf16_to_f32(vw))[0].transpose(0, 1)
    out = torch.empty_like(q)
    for i in range(0, q.shape[1], chunk):
        s = torch.matmul(q[:, i:i + chunk], k.transpose(1, 2)) / np.sqrt(128.0)
        out[:, i:i + chunk] = torch.matmul(torch.softmax(s, dim=-1), v)
    return out.transpose(0, 1).numpy()[None]


@pytest.mark.parametrize("lossless", [False, True])
def test_window21_block(lossless):
    import quant_kv
    from kvq import rope, synth
    mode = "bands4"
    fr = rope.freqs(1024)
    t_new = 21 * 1560                      # global position of the block's first token
    pos = rope.grid_positions(t_new, N)
    for layer in range(2):
        seed = 900 + 10 * layer
        k0, v0 = synth.make_k(S, H, seed=seed), synth.make_v(S, H, seed=seed + 1)
        k_pre = (torch.randn(N, H, 128, generator=torch.Generator().manual_seed(seed + 2))
                 * torch.exp(torch.randn(H, 128, generator=torch.Generator().manual_seed(seed + 3)))).to(torch.bfloat16)
        v_new = synth.make_v(N, H, seed=seed + 4)
        q = synth.make_q(1, N, H, seed=seed + 5)

        ck = quant_kv.QuantKVTensor([1, S, H, 128], "cuda", torch.bfloat16, 4, mode, SINK, lossless)
        cv = quant_kv.QuantKVTensor([1, S, H, 128], "cuda", torch.bfloat16, 4, mode, SINK, lossless)
        ck[:, 0:S] = k0.unsqueeze(0).cuda()
        cv[:, 0:S] = v0.unsqueeze(0).cuda()
        rk = ko.QuantKVRef(S, H, 128, 4, mode, SINK)
        rv = ko.QuantKVRef(S, H, 128, 4, mode, SINK)
        rk.setitem(0, S, _u16(k0))
        rv.setitem(0, S, _u16(v0))

        # 1. eviction of the oldest block after the sink
        for c in (ck, cv):
            c[:, SINK:S - N] = c[:, SINK + N:S].clone()
        for r in (rk, rv):
            if lossless:
                r.packed[SINK:S - N] = r.packed[SINK + N:S].copy()
                r.scales[SINK:S - N] = r.scales[SINK + N:S].copy()
            else:
                r.setitem(SINK, S - N, r.getitem(SINK + N, S)[0])
        # 2. append of the new block: keys rotated in the quantize kernel
        ck.write_rope_(S - N, S, k_pre.unsqueeze(0).cuda(), fr.cuda(), pos.cuda())
        cv[:, S - N:S] = v_new.unsqueeze(0).cuda()
        rk.setitem(S - N, S, ko.rope_f64(_u16(k_pre), fr.numpy(), pos.numpy()))
        rv.setitem(S - N, S, _u16(v_new))
        for c, r in ((ck, rk), (cv, rv)):
            assert np.array_equal(c.packed.cpu().numpy(), r.packed), f"layer {layer}: codes differ"
            assert np.array_equal(_u16(c.scales), r.scales), f"layer {layer}: scales differ"
            assert np.array_equal(_u16(c.sink), r.sink), f"layer {layer}: sink differs"
        # 3. attention of the block's queries over the window
        o = quant_kv.attention(q.cuda(), ck[:, 0:S], cv[:, 0:S])
        ref = _attention_fp32(_u16(q), rk.getitem(0, S), rv.getitem(0, S))
        err = np.abs(o.float().cpu().numpy() - ref)
        assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, \
            f"layer {layer}: max {err.max():.3e} mean {err.mean():.3e}"
    assert quant_kv._ops.device_status() == 0
