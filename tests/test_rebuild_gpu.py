"""Batched quantize of many tensors in one launch (kvq_rebuild_layers,
quant_kv.write_layers): bit-identical codes, scales and sink rows to one slice
write per cache, and to the oracle; ragged token counts, windows crossing the
sink border, several streams, more tensors than one launch takes, int8, strided
values and argument errors."""
import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import kvq_oracle as ko

pytestmark = pytest.mark.gpu


def _u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _caches(n, B, S, H, mode="bands4", sink=0, bits=4):
    import quant_kv
    return [quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, bits, mode, sink) for _ in range(n)]


def _values(n, B, L, H, seed):
    from kvq import synth
    return [torch.stack([synth.make_k(L, H, seed=seed + 7 * i + b, device="cuda") for b in range(B)])
            for i in range(n)]


def _same(c1, c2):
    assert torch.equal(c1.packed, c2.packed)
    assert torch.equal(c1.scales.view(torch.int16), c2.scales.view(torch.int16))
    if c1.sink is not None:
        assert torch.equal(c1.sink.view(torch.int16), c2.sink.view(torch.int16))


@pytest.mark.parametrize("mode,bits", [("bands4", 4), ("bands", 4), ("blind64", 8), ("bands3", 4)])
@pytest.mark.parametrize("B,S,L,a,sink", [(1, 700, 700, 0, 130), (2, 600, 129, 70, 100), (3, 300, 1, 299, 0)])
def test_write_layers_matches_slice_writes(mode, bits, B, S, L, a, sink):
    import quant_kv
    n, H = 5, 3
    vals = _values(n, B, L, H, seed=B * 100 + L)
    one = _caches(n, B, S, H, mode, sink, bits)
    many = _caches(n, B, S, H, mode, sink, bits)
    for c, v in zip(one, vals):
        c[:, a:a + L] = v
    quant_kv.write_layers(many, vals, a, a + L)
    torch.cuda.synchronize()
    for c1, c2 in zip(one, many):
        _same(c1, c2)


def test_write_layers_against_oracle_with_sink():
    import quant_kv
    n, B, S, H, sink = 4, 1, 2000, 5, 500
    a, b = 300, 1900            # crosses the sink border
    vals = _values(n, B, b - a, H, seed=11)
    caches = _caches(n, B, S, H, "bands4", sink)
    quant_kv.write_layers(caches, vals, a, b)
    bands = ko.band_edges(128, "bands4")
    for c, v in zip(caches, vals):
        xb = _u16(v[0])
        codes, scales = c_oracle.quantize(xb, bands)
        assert np.array_equal(c.packed[a:b].cpu().numpy(), codes)
        assert np.array_equal(_u16(c.scales[a:b]), scales)
        assert np.array_equal(_u16(c.sink[a:sink]), xb[: sink - a])


def test_write_layers_more_than_one_launch():
    import quant_kv
    n, B, S, H = 50, 2, 160, 2        # 100 (cache, stream) tensors: two launches
    vals = _values(n, B, S, H, seed=3)
    one = _caches(n, B, S, H)
    many = _caches(n, B, S, H)
    for c, v in zip(one, vals):
        c[:, 0:S] = v
    quant_kv.write_layers(many, vals, 0, S)
    for c1, c2 in zip(one, many):
        _same(c1, c2)


def test_write_layers_strided_values():
    import quant_kv
    n, S, H = 3, 257, 4
    big = _values(n, 1, S, 2 * H, seed=5)
    vals = [v[:, :, :H] for v in big]        # token stride 2*H*D, heads contiguous
    one = _caches(n, 1, S, H)
    many = _caches(n, 1, S, H)
    for c, v in zip(one, vals):
        c[:, 0:S] = v
    quant_kv.write_layers(many, vals, 0, S)
    for c1, c2 in zip(one, many):
        _same(c1, c2)


def test_write_layers_rejects_mismatched_caches():
    import quant_kv
    c = _caches(1, 1, 64, 2)[0]
    d = _caches(1, 1, 64, 2, mode="bands")[0]
    v = _values(2, 1, 64, 2, seed=1)
    with pytest.raises(ValueError):
        quant_kv.write_layers([c, d], v, 0, 64)
    with pytest.raises(ValueError):
        quant_kv.write_layers([c], v, 0, 64)


def test_rebuild_layers_rejects_bad_arguments(libkvq):
    import ctypes
    cb = np.zeros(128, np.int32)
    cb[44:86], cb[86:] = 1, 2
    p = (ctypes.c_void_p * 2)(16, 32)
    cbp = cb.ctypes.data_as(ctypes.c_void_p)
    assert libkvq.kvq_rebuild_layers(0, p, 5120, p, p, None, 0, 4, 40, 128, cbp, 3, 4, None) == -1
    assert libkvq.kvq_rebuild_layers(97, p, 5120, p, p, None, 0, 4, 40, 128, cbp, 3, 4, None) == -1
    assert libkvq.kvq_rebuild_layers(2, p, 5120, p, p, None, 0, 4, 40, 128, cbp, 3, 5, None) == -1
    odd = (ctypes.c_void_p * 2)(16, 40)   # second x not 16-byte aligned
    rc = libkvq.kvq_rebuild_layers(2, odd, 5120, p, p, None, 0, 4, 40, 128, cbp, 3, 4, None)
    assert rc == -4 and b"tensor 1" in libkvq.kvq_last_error()
