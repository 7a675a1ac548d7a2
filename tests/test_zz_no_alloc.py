"""kvq_attention_noalloc: kvq_attention with its wave-balance workspace in a
fixed array inside the library instead of caller memory. Its output agrees with
kvq_attention given a workspace of kvq_attention_workspace_bytes() bytes, within
the attention tolerance, on two calls in a row (the second reuses the scratch
and its counters); a call after the first takes no device memory; a shape whose
workspace would not fit the array is rejected without a launch. This file is
collected last so that it runs both alone and after every other test."""
import ctypes

import numpy as np
import pytest
import torch

from test_attention_gpu import _make_caches
from test_attention_split_gpu import _launch, _ws_bytes

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-4
SCRATCH_BYTES = 32 << 20          # KVQ_NOALLOC_SCRATCH_BYTES


def _noalloc(q, tk, tv, lo, hi, out):
    """kvq_attention_noalloc through the C ABI; returns its status code."""
    from kvq import _lib
    B, Lq, H, D = q.shape
    cb = np.ascontiguousarray(tk.chan_band_host, dtype=np.int32)
    return _lib.load().kvq_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), q.stride(1), ctypes.c_void_p(tk.packed.data_ptr()),
        ctypes.c_void_p(tk.scales.data_ptr()), ctypes.c_void_p(tk.sink.data_ptr() if tk.sink is not None else 0),
        ctypes.c_void_p(tv.packed.data_ptr()), ctypes.c_void_p(tv.scales.data_ptr()),
        ctypes.c_void_p(tv.sink.data_ptr() if tv.sink is not None else 0), tk.n_tokens,
        tk.sink_tokens if tk.sink is not None else 0, lo, hi, ctypes.c_void_p(out.data_ptr()), out.stride(1),
        B, Lq, H, D, cb.ctypes.data_as(ctypes.c_void_p), len(tk.bands), 4, 4, 0.0,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _close(a, b, what):
    d = (a.float() - b.float()).abs()
    assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, \
        f"{what}: max {d.max().item():.3e} mean {d.mean().item():.3e}"


@pytest.mark.parametrize("B,S,H,Lq,sink", [
    (1, 4680, 40, 4680, 1560),     # window 3, forty heads: the one-tile units run in parts
    (2, 2000, 37, 700, 300),       # odd sizes: two-tile units halved
    (1, 256, 2, 100, 0),           # a launch far smaller than a wave
])
def test_noalloc_matches_attention_with_workspace(B, S, H, Lq, sink):
    from kvq import _lib, ops, synth
    need = _ws_bytes(B, Lq, H, S)
    assert 0 < need <= SCRATCH_BYTES, f"expected a split launch that fits the scratch, needs {need}"
    tk, tv, _, _ = _make_caches(B, S, H, "bands4", sink, seed=3 * B + S + H)
    qs = [synth.make_q(B, Lq, H, seed=s).cuda() for s in (17, 29)]
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    refs = [_launch(q, tk, tv, 0, S, ws) for q in qs]
    outs = [torch.full_like(q, 3.0) for q in qs]
    _lib.check(_noalloc(qs[0], tk, tv, 0, S, outs[0]), "kvq_attention_noalloc")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    _lib.check(_noalloc(qs[1], tk, tv, 0, S, outs[1]), "kvq_attention_noalloc")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "the second call changed the device's free memory"
    assert ops.device_status() == 0
    for i in range(2):
        _close(outs[i], refs[i], f"call {i + 1}")


def test_noalloc_rejects_a_shape_beyond_the_scratch():
    """One-tile units of 160 (head, stream) pairs over 2,000 tokens run in four
    parts each: 640 partial slots, more than 32 MiB."""
    from kvq import _lib
    B, S, H, Lq = 1, 2000, 160, 100
    need = _ws_bytes(B, Lq, H, S)
    assert need > SCRATCH_BYTES
    tk, tv, _, _ = _make_caches(B, S, H, "bands4", 0, seed=5)
    q = torch.zeros((B, Lq, H, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(q, 3.0)
    rc = _noalloc(q, tk, tv, 0, S, out)
    assert rc == _lib.KVQ_ERR_UNSUPPORTED
    assert b"scratch" in _lib.load().kvq_last_error()
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())
