"""Quantize / dequantize kernels against the reference (golden fixtures) and the
oracle at full workload sizes. Bit-exact: codes, scales and dequantized bf16."""
import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import kvq_oracle as ko

pytestmark = pytest.mark.gpu
MODES = ("bands", "bands2", "bands4", "blind32", "blind64", "bands3", "bands8", "blind16")


def _t(bits_u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits_u16.view(np.int16)).view(torch.bfloat16)


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _quant(x_cpu_bf16, mode, bits=4):
    import quant_kv_kernels as qk
    bands = ko.band_edges(x_cpu_bf16.shape[-1], mode)
    cb = qk.build_chan_band(bands, x_cpu_bf16.shape[-1], "cuda")
    p, s = qk.quantize(x_cpu_bf16.cuda(), cb, len(bands), 7 if bits == 4 else 127)
    torch.cuda.synchronize()
    return p, s, cb, bands


def test_golden_codes_scales_dequant(golden):
    import quant_kv_kernels as qk
    g = golden("quant_cases.npz")
    n = 0
    for name in ("outlier", "rope_k", "v", "edge"):
        x = _t(g[f"{name}/x"])
        for mode in MODES:
            for bits in (4, 8):
                key = f"{name}/{mode}/int{bits}"
                if f"{key}/codes" not in g.files:
                    continue
                p, s, cb, bands = _quant(x, mode, bits)
                np.testing.assert_array_equal(p.cpu().numpy(), g[f"{key}/codes"], err_msg=key)
                np.testing.assert_array_equal(_u16(s), g[f"{key}/scales"], err_msg=key)
                if f"{key}/deq" in g.files:
                    d = qk.dequantize(torch.from_numpy(g[f"{key}/codes"]).cuda(),
                                      _t(g[f"{key}/scales"]).cuda(), cb, x.shape[-1])
                    np.testing.assert_array_equal(_u16(d), g[f"{key}/deq"], err_msg=key)
                n += 1
    assert n >= 40


@pytest.mark.parametrize("mode", ["bands", "bands4", "blind64", "bands2", "blind32", "bands8"])
def test_config0_full_size_against_oracle(mode):
    """One layer's K and V at 4680 x 40 x 128 (the CPU-runnable round-trip workload)."""
    from kvq import synth
    import quant_kv_kernels as qk
    for x in (synth.make_k(4680, 40, seed=0), synth.make_v(4680, 40, seed=0)):
        p, s, cb, bands = _quant(x, mode)
        xb = _u16(x)
        rc, rs = c_oracle.quantize(xb, bands)
        np.testing.assert_array_equal(p.cpu().numpy(), rc)
        np.testing.assert_array_equal(_u16(s), rs)
        d = qk.dequantize(p, s, cb, 128)
        np.testing.assert_array_equal(_u16(d), c_oracle.dequantize(rc, rs, bands, 128))


def test_window21_size_against_oracle():
    """32760 tokens x 40 heads (one layer-tensor of the window-21 cache), bands4."""
    from kvq import synth
    x = synth.make_k(32760, 40, seed=9)
    p, s, cb, bands = _quant(x, "bands4")
    rc, rs = c_oracle.quantize(_u16(x), bands)
    np.testing.assert_array_equal(p.cpu().numpy(), rc)
    np.testing.assert_array_equal(_u16(s), rs)


@pytest.mark.parametrize("L,H", [(1, 1), (7, 5), (1559, 3), (1561, 2), (3, 40), (129, 1), (0, 4)])
def test_ragged_shapes(L, H):
    from kvq import synth
    x = synth.make_outlier(max(L, 1), H, seed=L + H)[:L]
    for mode in ("bands4", "blind16"):
        for bits in (4, 8):
            p, s, _, bands = _quant(x, mode, bits)
            rc, rs = c_oracle.quantize(_u16(x), bands, bits)
            np.testing.assert_array_equal(p.cpu().numpy(), rc)
            np.testing.assert_array_equal(_u16(s), rs)


def test_strided_input_and_in_place_slices():
    """x as the K slice of a fused [L, 3, H, D] buffer, written into a cache slice
    at a token offset whose scale rows are not 16-byte aligned."""
    from kvq import ops, synth
    L, H = 100, 3
    fused = torch.stack([synth.make_k(L, H, seed=s) for s in range(3)], dim=1).cuda()  # [L,3,H,D]
    x = fused[:, 1]                                        # token stride 3*H*D
    bands = ko.band_edges(128, "bands")
    S, a = 160, 37
    codes = torch.zeros((S, H, 64), dtype=torch.uint8, device="cuda")
    scales = torch.zeros((S, H, 3), dtype=torch.bfloat16, device="cuda")
    ops.quantize_into(x, codes[a:a + L], scales[a:a + L], ko.chan_band(bands, 128), 3, 4)
    rc, rs = c_oracle.quantize(_u16(fused[:, 1].contiguous()), bands)
    np.testing.assert_array_equal(codes[a:a + L].cpu().numpy(), rc)
    np.testing.assert_array_equal(_u16(scales[a:a + L]), rs)
    assert int(codes[:a].count_nonzero()) == 0 and int(codes[a + L:].count_nonzero()) == 0
    assert int(scales[:a].view(torch.int16).count_nonzero()) == 0
    # dequantize into a strided output
    out = torch.zeros((L, 2, H, 128), dtype=torch.bfloat16, device="cuda")
    ops.dequantize_into(codes[a:a + L], scales[a:a + L], out[:, 1], ko.chan_band(bands, 128), 3, 4)
    np.testing.assert_array_equal(_u16(out[:, 1]), c_oracle.dequantize(rc, rs, bands, 128))
    assert int(out[:, 0].view(torch.int16).count_nonzero()) == 0


def test_sink_copy_and_overlay():
    from kvq import ops, synth
    L, H, sink = 300, 4, 130
    x = synth.make_k(L, H, seed=2).cuda()
    bands = ko.band_edges(128, "bands4")
    cb = ko.chan_band(bands, 128)
    codes = torch.empty((L, H, 64), dtype=torch.uint8, device="cuda")
    scales = torch.empty((L, H, 12), dtype=torch.bfloat16, device="cuda")
    sbuf = torch.zeros((sink + 5, H, 128), dtype=torch.bfloat16, device="cuda")
    ops.quantize_into(x, codes, scales, cb, 12, 4, sink=sbuf, sink_tokens=sink)
    assert torch.equal(sbuf[:sink], x[:sink]) and int(sbuf[sink:].view(torch.int16).count_nonzero()) == 0
    out = torch.empty((L, H, 128), dtype=torch.bfloat16, device="cuda")
    ops.dequantize_into(codes, scales, out, cb, 12, 4, sink=sbuf, sink_tokens=sink)
    assert torch.equal(out[:sink], x[:sink])
    ref = c_oracle.dequantize(*c_oracle.quantize(_u16(x), bands), bands, 128)
    np.testing.assert_array_equal(_u16(out[sink:]), ref[sink:])


def test_errors_are_loud():
    import quant_kv_kernels as qk
    cb = qk.build_chan_band(ko.band_edges(128, "bands"), 128, "cuda")
    x = torch.zeros((4, 2, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        qk.quantize(x, cb, 4, 7)           # group 3 empty
    with pytest.raises(ValueError):
        qk.dequantize(torch.zeros((4, 2, 10), dtype=torch.uint8, device="cuda"),
                      torch.zeros((4, 2, 3), dtype=torch.bfloat16, device="cuda"), cb, 128)
