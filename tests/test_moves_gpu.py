"""Lossless packed eviction moves (QuantKVTensor(lossless_moves=True)): the
runtime's `kv[:, a:b] = kv[:, c:d].clone()` copies codes and scales unchanged,
so the destination reads back exactly what the source read before the move;
overlapping ranges behave like memmove; destination rows inside the sink get the
source's read values. The default keeps the reference's dequantize-requantize,
as one fused pass over the packed snapshot (kvq_requantize)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cache(B, S, H, sink, lossless, mode="bands4", bits=4):
    import quant_kv
    return quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, bits, mode, sink, lossless)


def _fill(c, seed):
    from kvq import synth
    S, H = c.n_tokens, c.n_heads
    c[:, 0:S] = torch.stack([synth.make_k(S, H, seed=seed + b, device="cuda") for b in range(c.n_streams)])


def _bits(t):
    return t.contiguous().view(torch.int16)


@pytest.mark.parametrize("B,S,sink,src,dst", [
    (1, 4000, 1000, (2000, 3500), (1000, 2500)),   # eviction after the sink, overlapping
    (2, 3000, 500, (1200, 1900), (1500, 2200)),    # overlapping, moving up
    (1, 2000, 600, (100, 400), (900, 1200)),       # sink rows to outside the sink
    (2, 2000, 600, (1300, 1700), (400, 800)),      # outside rows into the sink border
    (1, 1500, 0, (0, 1500), (0, 1500)),            # identity, no sink
])
def test_lossless_move_reads_back_exactly(B, S, sink, src, dst):
    import quant_kv
    c = _cache(B, S, 4, sink, True)
    _fill(c, seed=B * 10 + S)
    before = c[:, src[0]:src[1]].materialize()
    blk = c[:, src[0]:src[1]].clone()
    assert isinstance(blk, quant_kv.PackedBlock)
    codes_before = torch.cat([c.packed[c._rows(i, *src)] for i in range(B)]).clone()
    c[:, dst[0]:dst[1]] = blk
    after = c[:, dst[0]:dst[1]].materialize()
    codes_after = torch.cat([c.packed[c._rows(i, *dst)] for i in range(B)])
    assert torch.equal(codes_after, codes_before)
    # rows read exactly as before the move, except rows that leave the sink: only
    # their codes travel, and they read back dequantized, as the reference's
    # dequantize-requantize gives (the stored codes are the quantized sink rows)
    n = src[1] - src[0]
    leave = [i for i in range(n) if src[0] + i < sink and dst[0] + i >= sink]
    keep = [i for i in range(n) if i not in set(leave)]
    assert torch.equal(_bits(after[:, keep]), _bits(before[:, keep]))
    if leave:
        ref = _cache(B, S, 4, sink, False)
        _fill(ref, seed=B * 10 + S)
        ref[:, dst[0]:dst[1]] = ref[:, src[0]:src[1]].clone()
        want = ref[:, dst[0]:dst[1]].materialize()
        assert torch.equal(_bits(after[:, leave]), _bits(want[:, leave]))


def test_default_keeps_requantizing_semantics():
    """Without the flag the clone holds the bf16 read and the write requantizes it,
    exactly as writing that tensor would (the reference's path)."""
    import quant_kv
    c = _cache(1, 3000, 4, 500, False)
    _fill(c, seed=7)
    v = c[:, 1500:2500].clone()
    assert isinstance(v, quant_kv.PackedBlock)
    ref = _cache(1, 3000, 4, 500, False)
    _fill(ref, seed=7)
    c[:, 500:1500] = v
    ref[:, 500:1500] = v.materialize()
    assert torch.equal(c.packed, ref.packed)
    assert torch.equal(_bits(c.scales), _bits(ref.scales))
    assert torch.equal(_bits(c.sink), _bits(ref.sink))


@pytest.mark.parametrize("mode,bits", [("bands4", 4), ("bands", 4), ("blind64", 4), ("bands4", 8)])
@pytest.mark.parametrize("B,S,H,sink,src,dst", [
    (1, 4000, 4, 1000, (2000, 3500), (1000, 2500)),       # eviction after the sink, overlapping
    (2, 3000, 4, 500, (1200, 1900), (1500, 2200)),        # overlapping, moving up
    (1, 2000, 4, 600, (100, 400), (900, 1200)),           # sink rows (exact) to outside the sink
    (2, 2000, 4, 600, (1300, 1700), (400, 800)),          # outside rows into the sink border
    (1, 300, 3, 0, (77, 211), (0, 134)),                  # ragged, no sink
    (1, 32760, 40, 1560, (6240, 32760), (1560, 28080)),   # the window-21 eviction of one block
])
def test_requantizing_move_equals_two_pass(mode, bits, B, S, H, sink, src, dst):
    """The default eviction `kv[:, a:b] = kv[:, c:d].clone()`: the write of the
    packed snapshot (one fused kvq_requantize pass for int4; the dequantize +
    quantize pair otherwise) equals quantizing the window's bf16 read, codes,
    scales and sink rows bit for bit."""
    import quant_kv
    if S > 10000 and (mode, bits) != ("bands4", 4):
        pytest.skip("the window-21 shape runs for the default format only")
    c = _cache(B, S, H, sink, False, mode, bits)
    ref = _cache(B, S, H, sink, False, mode, bits)
    for t in (c, ref):
        _fill(t, seed=B * 100 + S + H)
    blk = c[:, src[0]:src[1]].clone()
    assert isinstance(blk, quant_kv.PackedBlock)
    values = ref[:, src[0]:src[1]].materialize()
    c[:, dst[0]:dst[1]] = blk
    ref.write_(dst[0], dst[1], values)
    assert torch.equal(c.packed, ref.packed)
    assert torch.equal(_bits(c.scales), _bits(ref.scales))
    if sink:
        assert torch.equal(_bits(c.sink), _bits(ref.sink))


def test_packed_block_behaves_like_its_read():
    import quant_kv
    c = _cache(2, 1200, 3, 300, True)
    _fill(c, seed=3)
    blk = c[:, 100:700].clone()
    want = c[:, 100:700].materialize()
    assert torch.equal(_bits(blk.materialize()), _bits(want))
    assert torch.equal(_bits(blk + 0), _bits(want + 0))
    assert blk.shape == want.shape
    # a snapshot: later writes to the cache do not change it
    c[:, 100:700] = torch.zeros_like(want)
    assert torch.equal(_bits(blk.materialize()), _bits(want))
    # into a cache of another format it is written as its bf16 read
    d = quant_kv.QuantKVTensor([2, 1200, 3, 128], "cuda", torch.bfloat16, 4, "bands", 300, True)
    d[:, 0:600] = blk
    e = quant_kv.QuantKVTensor([2, 1200, 3, 128], "cuda", torch.bfloat16, 4, "bands", 300, True)
    e[:, 0:600] = want
    assert torch.equal(d.packed, e.packed)
