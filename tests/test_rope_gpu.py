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
@pytest.mark.parametrize("B,S,a,b,sink,t0", [(1, 4680, 0, 4680, 1560, 0), (2, 3000, 1200, 2901, 1500, 9360),
                                             (1, 500, 7, 8, 0, 77)])
def test_rope_quantize_matches_oracle(mode, bits, B, S, a, b, sink, t0):
    import quant_kv
    from kvq import rope
    H = 5
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
