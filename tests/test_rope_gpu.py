"""Fused rotary embedding + quantize-on-append (kvq_rope_quantize,
QuantKVTensor.write_rope_): codes, scales and sink rows bit-identical to the
oracle's rotation (complex128 product, fp32, bf16; pinned against torch in
test_oracle.py) followed by the reference quantization."""
import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import kvq_oracle as ko

pytestmark = pytest.mark.gpu


def _u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("mode,bits", [("bands4", 4), ("bands", 4), ("blind64", 8)])
@pytest.mark.parametrize("B,S,a,b,sink,t0,H", [(1, 4680, 0, 4680, 1560, 0, 5), (2, 3000, 1200, 2901, 1500, 9360, 5),
                                               (1, 500, 7, 8, 0, 77, 5),
                                               # 16-40 heads: a 128-row tile spans 4-9 tokens; 4680 x 40 rows
                                               # are 1463 tiles, several per CTA
                                               (1, 4680, 0, 4680, 1560, 0, 40), (2, 1000, 33, 901, 100, 3120, 40),
                                               (1, 700, 5, 690, 64, 1560, 16), (1, 300, 0, 300, 0, 0, 18)])
def test_rope_quantize_matches_oracle(mode, bits, B, S, a, b, sink, t0, H):
    import quant_kv
    from kvq import rope
    c = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, bits, mode, sink)
    g = torch.Generator().manual_seed(b + t0)
    x = (torch.randn(B, b - a, H, 128, generator=g) * torch.exp(torch.randn(H, 128, generator=g))).to(torch.bfloat16)
    fr = rope.freqs(1024)
    pos = rope.grid_positions(t0, b - a)
    c.write_rope_(a, b, x.cuda(), fr.cuda(), pos.cuda())
    bands = ko.band_edges(128, mode)
    for s in range(B):
        xr = ko.rope_f64(_u16(x[s]), fr.numpy(), pos.numpy())
        codes, scales = c_oracle.quantize(xr, bands, bits=bits)
        assert np.array_equal(c.packed[c._rows(s, a, b)].cpu().numpy(), codes)
        assert np.array_equal(_u16(c.scales[c._rows(s, a, b)]), scales)
        ns = max(0, min(b, sink) - a)
        if ns:
            assert np.array_equal(_u16(c.sink[c._sink_rows(s, a, a + ns)]), xr[:ns])


def test_rope_quantize_rejects_bad_arguments():
    from kvq import ops, rope
    x = torch.zeros(8, 2, 128, dtype=torch.bfloat16, device="cuda")
    codes = torch.zeros(8, 2, 64, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(8, 2, 12, dtype=torch.bfloat16, device="cuda")
    cb = ko.chan_band(ko.band_edges(128, "bands4"), 128)
    fr = rope.freqs(16, device="cuda")
    with pytest.raises(ValueError):   # positions of the wrong shape
        ops.rope_quantize_into(x, codes, scales, cb, 12, 4, fr, torch.zeros(8, 2, dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):   # float32 table
        ops.rope_quantize_into(x, codes, scales, cb, 12, 4, fr.float(), rope.grid_positions(0, 8, device="cuda"))


def test_rope_quantize_special_values():
    """Zeros (both signs), subnormals and values near 2^126 (finite after the rotation) in the
    keys before rotation: codes, scales and sink rows stay bit-identical to the
    oracle."""
    import quant_kv
    from kvq import rope
    S, H = 600, 40
    g = torch.Generator().manual_seed(5)
    x = torch.randn(S, H, 128, generator=g).to(torch.bfloat16)
    bits = x.view(torch.int16)
    specials = torch.tensor([0x0000, 0x8000, 0x0001, 0x807F, 0x0040, 0x7E7F, 0xFE7F, 0x0080, 0x8080],
                            dtype=torch.int32).to(torch.int16)
    idx = torch.randint(0, S * H * 128, (4000,), generator=g)
    bits.view(-1)[idx] = specials[torch.arange(4000) % len(specials)]
    x[17] = 0                                   # a whole row of zeros (scale 1 path)
    c = quant_kv.QuantKVTensor([1, S, H, 128], "cuda", torch.bfloat16, 4, "bands4", 200)
    fr = rope.freqs(1024)
    pos = rope.grid_positions(3000, S)
    c.write_rope_(0, S, x.unsqueeze(0).cuda(), fr.cuda(), pos.cuda())
    bands = ko.band_edges(128, "bands4")
    xr = ko.rope_f64(_u16(x), fr.numpy(), pos.numpy())
    codes, scales = c_oracle.quantize(xr, bands)
    assert np.array_equal(c.packed.cpu().numpy(), codes)
    assert np.array_equal(_u16(c.scales), scales)
    assert np.array_equal(_u16(c.sink), xr[:200])


def _near_decision_keys(S, H, t0, tries, seed):
    """bf16 keys [S, H, 128] whose rotated pairs lie close to a point where
    bf16(fp32(t)) changes: for each (token, head, pair) the best of `tries` random
    N(0,1) x log-normal candidates by the distance (in fp32 ulps) of the fp64
    rotation's real or imaginary part from that point."""
    from kvq import rope
    rng = np.random.default_rng(seed)
    fr = rope.freqs(1024).numpy()
    pos = rope.grid_positions(t0, S).numpy()
    axis = np.repeat(np.arange(3), ko.ROPE_SPLIT)
    cs = fr[np.clip(pos, 0, 1023)[:, axis], np.arange(64)[None, :]]
    scale = np.exp(rng.standard_normal((H, 64, 1)))

    def dist(t):
        r = t.astype(np.float32)
        m = ((r.view(np.uint32) & np.uint32(0xFFFF0000)) | np.uint32(0x8000)).view(np.float32)
        u = np.spacing(np.abs(m)).astype(np.float64)
        m = m.astype(np.float64)
        return np.minimum(np.abs(t - (m - u / 2)), np.abs(t - (m + u / 2))) / u

    out = np.empty((S, H, 128), np.uint16)
    best = np.empty((S, H, 64))
    for t in range(S):
        c, s = cs[t, :, 0][None, :, None], cs[t, :, 1][None, :, None]
        b0 = ko.f32_to_bf16((rng.standard_normal((H, 64, tries)) * scale).astype(np.float32))
        b1 = ko.f32_to_bf16((rng.standard_normal((H, 64, tries)) * scale).astype(np.float32))
        x0, x1 = ko.bf16_to_f32(b0).astype(np.float64), ko.bf16_to_f32(b1).astype(np.float64)
        d = np.minimum(dist(x0 * c - x1 * s), dist(x0 * s + x1 * c))
        k = d.argmin(-1)[..., None]
        best[t] = np.take_along_axis(d, k, -1)[..., 0]
        out[t, :, 0::2] = np.take_along_axis(b0, k, -1)[..., 0]
        out[t, :, 1::2] = np.take_along_axis(b1, k, -1)[..., 0]
    return out, best


def test_rope_near_rounding_decision_points():
    """Keys whose fp64 rotation lands within a few fp32 ulps of a point where
    bf16(fp32(t)) changes, so that the double rounding (fp64 -> fp32 -> bf16,
    ties to even on the fp32 value) decides the result: every rotated row, all
    of them kept in the sink, and the codes and scales stay bit-identical to the
    oracle."""
    import quant_kv
    from kvq import rope
    S, H, t0 = 32, 4, 4717
    xb, best = _near_decision_keys(S, H, t0, 1024, seed=11)
    assert np.mean(best < 8) > 0.25           # the search found hard pairs
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
    c = quant_kv.QuantKVTensor([1, S, H, 128], "cuda", torch.bfloat16, 4, "bands4", S)
    fr = rope.freqs(1024)
    pos = rope.grid_positions(t0, S)
    c.write_rope_(0, S, x.unsqueeze(0).cuda(), fr.cuda(), pos.cuda())
    xr = ko.rope_f64(xb, fr.numpy(), pos.numpy())
    assert np.array_equal(_u16(c.sink), xr)
    codes, scales = c_oracle.quantize(xr, ko.band_edges(128, "bands4"))
    assert np.array_equal(c.packed.cpu().numpy(), codes)
    assert np.array_equal(_u16(c.scales), scales)
