"""Wave balance of the attention launch: with a workspace, the units of the last
wave are cut along the KV window into parts (two-tile units in halves, one-tile
units in up to four parts) and the part that finishes last merges them. The
merged output is within the attention tolerance of the oracle, agrees with the
launch that runs every unit whole, and is bit-identical from launch to launch
(the merge reads the parts in a fixed order; the counters are cleared by each
launch)."""
import ctypes

import numpy as np
import pytest
import torch

from test_attention_gpu import _check, _make_caches, _oracle_attention, _oracle_window, _u16
from oracle import kvq_oracle as ko

pytestmark = pytest.mark.gpu


def _ws_bytes(B, Lq, H, n_kv):
    from kvq import _lib
    n = ctypes.c_int64()
    assert _lib.load().kvq_attention_workspace_bytes(B, Lq, H, n_kv, ctypes.byref(n)) == 0
    return n.value


def _launch(q, tk, tv, lo, hi, workspace):
    """kvq_attention through the C ABI, with or without a workspace."""
    from kvq import _lib, ops
    B, Lq, H, D = q.shape
    out = torch.empty_like(q)
    cb = np.ascontiguousarray(tk.chan_band_host, dtype=np.int32)
    ws = ctypes.c_void_p(workspace.data_ptr()) if workspace is not None else None
    wsb = workspace.numel() if workspace is not None else 0
    rc = _lib.load().kvq_attention(
        ctypes.c_void_p(q.data_ptr()), q.stride(1), ctypes.c_void_p(tk.packed.data_ptr()),
        ctypes.c_void_p(tk.scales.data_ptr()), ctypes.c_void_p(tk.sink.data_ptr() if tk.sink is not None else 0),
        ctypes.c_void_p(tv.packed.data_ptr()), ctypes.c_void_p(tv.scales.data_ptr()),
        ctypes.c_void_p(tv.sink.data_ptr() if tv.sink is not None else 0), tk.n_tokens,
        tk.sink_tokens if tk.sink is not None else 0, lo, hi, ctypes.c_void_p(out.data_ptr()), out.stride(1),
        B, Lq, H, D, cb.ctypes.data_as(ctypes.c_void_p), len(tk.bands), 4, 4, 0.0, ws, wsb,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "kvq_attention")
    return out


@pytest.mark.parametrize("B,S,H,Lq,sink", [
    (1, 4680, 40, 4680, 1560),     # window 3: the forty one-tile units (72 queries) in parts
    (4, 32760, 5, 4680, 1560),     # 4 streams at window 21, 5 heads (a GPU of eight): two-tile units halved
    (2, 2000, 37, 700, 300),       # odd sizes: 3 pairs per (head, stream), the last with 188 queries
    (1, 256, 2, 100, 0),           # a launch far smaller than a wave: its two units run in parts on idle SMs
])
def test_split_launch_matches_oracle_and_whole_units(B, S, H, Lq, sink):
    from kvq import ops, synth
    need = _ws_bytes(B, Lq, H, S)
    assert need > 0, "this shape is expected to split its last wave"
    tk, tv, kb, vb = _make_caches(B, S, H, "bands4", sink, seed=B + S + H)
    q = synth.make_q(B, Lq, H, seed=7).cuda()
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    assert ws.data_ptr() % 256 == 0
    split1 = _launch(q, tk, tv, 0, S, ws)
    split2 = _launch(q, tk, tv, 0, S, ws)
    whole = _launch(q, tk, tv, 0, S, None)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(split1.view(torch.int16), split2.view(torch.int16))
    bands = ko.band_edges(128, "bands4")
    kw = np.stack([_oracle_window(kb[b], bands, sink, 0, S) for b in range(B)])
    vw = np.stack([_oracle_window(vb[b], bands, sink, 0, S) for b in range(B)])
    ref = _oracle_attention(_u16(q), kw, vw)
    _check(split1, ref, "split launch")
    _check(whole, ref, "whole-unit launch")
    d = (split1.float() - whole.float()).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-4


def test_split_gather_two_local_destinations():
    """The gather epilogue of a merged unit stores to every destination too."""
    from kvq import ops, synth
    B, S, H, Lq, sink = 1, 4680, 40, 4680, 1560
    assert _ws_bytes(B, Lq, H, S) > 0
    tk, tv, _, _ = _make_caches(B, S, H, "bands4", sink, seed=3)
    q = synth.make_q(B, Lq, H, seed=9).cuda()
    ref = ops.attention_packed(q, tk, tv, 0, S)            # the Python path uses the workspace as well
    bufs = [torch.full((B, Lq, 42, 128), 5.0, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ops.attention_packed_gather(q, tk, tv, 0, S, [b.data_ptr() for b in bufs], 1, 42)
    torch.cuda.synchronize()
    for b in bufs:
        assert torch.equal(b[:, :, 1:41], ref)
        assert bool((b[:, :, 0] == 5.0).all()) and bool((b[:, :, 41] == 5.0).all())
    assert ops.device_status() == 0


def test_workspace_bytes_is_zero_when_nothing_is_split():
    assert _ws_bytes(1, 4680, 40, 64) == 0         # one KV tile: nothing to cut
    assert _ws_bytes(1, 0, 40, 4680) == 0          # no queries


def test_statistics_kernel_equals_the_whole_unit_launch():
    """The statistics instance never splits: its output is the whole-unit launch's,
    bit for bit (same arithmetic)."""
    import quant_kv
    from kvq import synth
    B, S, H, Lq, sink = 1, 4680, 8, 600, 1560
    tk, tv, _, _ = _make_caches(B, S, H, "bands4", sink, seed=41)
    q = synth.make_q(B, Lq, H, seed=43).cuda()
    out, _ = quant_kv.attention_stats(q, tk[:, 0:S], tv[:, 0:S])
    whole = _launch(q, tk, tv, 0, S, None)
    assert torch.equal(out.view(torch.int16), whole.view(torch.int16))
