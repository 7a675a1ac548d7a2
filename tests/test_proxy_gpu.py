"""QuantKVTensor drop-in against the reference proxy (golden fixtures) and the
reference's own semantics test (test_quant_kv.py:29-58)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(b):
    return torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)


def _u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_proxy_matches_reference(golden):
    import quant_kv
    g = golden("proxy_semantics.npz")
    for mode in ("bands", "bands4"):
        t = quant_kv.QuantKVTensor([1, 96, 3, 128], "cuda", torch.bfloat16, 4, mode, 40)
        t[:, 0:40] = _t(g[f"{mode}/w0"]).unsqueeze(0).cuda()
        t[:, 40:96] = _t(g[f"{mode}/w1"]).unsqueeze(0).cuda()
        for lo, hi in ((0, 96), (20, 60), (50, 70), (39, 41), (0, 1)):
            w = t[:, lo:hi]
            assert isinstance(w, quant_kv.QuantKVWindow) and tuple(w.shape) == (1, hi - lo, 3, 128)
            np.testing.assert_array_equal(_u16(w.materialize()[0]), g[f"{mode}/read_{lo}_{hi}"])
        t[:, 30:60] = t[:, 60:90].clone()          # the runtime's eviction path
        np.testing.assert_array_equal(_u16(t[:, 0:96].materialize()[0]), g[f"{mode}/after_evict"])
        np.testing.assert_array_equal(t.packed.cpu().numpy(), g[f"{mode}/packed"])
        np.testing.assert_array_equal(_u16(t.scales), g[f"{mode}/scales"])
        np.testing.assert_array_equal(_u16(t.sink), g[f"{mode}/sink"])
        e = t[:, 10:10]
        assert tuple(e.shape) == tuple(g[f"{mode}/empty_shape"])
        t.zero_()
        np.testing.assert_array_equal(_u16(t[:, 0:12].materialize()[0]), g[f"{mode}/after_zero"])


def test_reference_semantics_check():
    """Restates test_quant_kv.py:29-58 on the drop-in (S=4680, H=8, sink 1560)."""
    import quant_kv
    S, H, D = 4680, 8, 128
    t = quant_kv.QuantKVTensor([1, S, H, D], "cuda", bits=4, group_mode="bands", sink_tokens=1560)
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(1, 1560, H, D, dtype=torch.bfloat16, device="cuda", generator=gen)
    t[:, 0:1560] = x
    back = t[:, 0:1560]
    assert torch.equal(back, x)                        # sink kept in bf16 (torch fn on a window)
    y = torch.randn(1, 3120, H, D, dtype=torch.bfloat16, device="cuda", generator=gen)
    t[:, 1560:4680] = y
    yb = t[:, 1560:4680]
    rel = ((yb.float() - y.float()).norm() / y.float().norm()).item()
    assert 0.05 < rel < 0.15                             # reference records 0.10155
    assert tuple(t.shape) == (1, S, H, D) and tuple(yb.shape) == (1, 3120, H, D)
    partial = t[:, 1000:2000]
    assert tuple(partial.shape) == (1, 1000, H, D)
    assert torch.equal(partial[:, :560], x[:, 1000:1560])
    t.zero_()
    assert float(t[:, 0:100].abs().max()) == 0.0
    assert abs(t.storage_bytes() / (S * H * D * 2) - 0.6068) < 1e-3


def test_batch_of_streams():
    """The leading dim generalised to independent streams (reference asserts 1)."""
    import quant_kv
    import quant_kv_kernels as qk
    from kvq import synth
    B, S, H = 3, 64, 2
    t = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", bits=4, group_mode="bands4", sink_tokens=20)
    xs = torch.stack([synth.make_k(S, H, seed=i) for i in range(B)]).cuda()
    t[:, 0:S] = xs
    for i in range(B):
        p, s = qk.quantize(xs[i], t.chan_band, 12, 7)
        assert torch.equal(t.packed[i * S:(i + 1) * S], p)
        assert torch.equal(t.scales[i * S:(i + 1) * S], s)
    w = t[:, 10:40].materialize()
    assert w.shape == (B, 30, H, 128)
    for i in range(B):
        assert torch.equal(w[i, :10], xs[i, 10:20])     # sink rows exact per stream


def test_window_behaves_like_tensor():
    import quant_kv
    from kvq import synth
    t = quant_kv.QuantKVTensor([1, 32, 2, 128], "cuda", group_mode="bands")
    x = synth.make_v(32, 2).cuda().unsqueeze(0)
    t[:, 0:32] = x
    w = t[:, 4:20]
    m = w.materialize()
    assert torch.equal(w.float(), m.float())
    assert torch.equal(torch.abs(w), m.abs())
    assert torch.equal(w - m, torch.zeros_like(m))
    assert w.shape == m.shape and w.dtype == torch.bfloat16 and w.device == m.device
    assert torch.equal(w[:, 3], m[:, 3])


def test_stale_window_refuses_use():
    """A window is read when used, so once its cache was written after the window
    was taken, using it raises instead of returning the newer data (the
    reference's __getitem__ returns a snapshot); a clone taken before the write
    keeps the old contents."""
    import quant_kv
    from kvq import synth
    t = quant_kv.QuantKVTensor([1, 64, 2, 128], "cuda", group_mode="bands4", sink_tokens=8)
    t[:, 0:64] = synth.make_v(64, 2, seed=1).cuda().unsqueeze(0)
    w = t[:, 0:32]
    snap = w.clone()
    t[:, 16:48] = synth.make_v(32, 2, seed=2).cuda().unsqueeze(0)
    with pytest.raises(RuntimeError, match="taken before a later write"):
        w.materialize()
    q = synth.make_q(1, 8, 2, seed=3).cuda()
    with pytest.raises(RuntimeError):
        quant_kv.attention(q, w, t[:, 0:32])
    assert not torch.equal(t[:, 0:32].materialize(), snap)       # the cache did change, the clone did not


def test_attention_accepts_neutral_upstream_arguments():
    """The upstream wrapper's optional arguments that do not change the result are
    accepted, positionally or by name; the others raise."""
    import quant_kv
    from kvq import synth
    S, H = 256, 2
    tk = quant_kv.QuantKVTensor([1, S, H, 128], "cuda", group_mode="bands4")
    tv = quant_kv.QuantKVTensor([1, S, H, 128], "cuda", group_mode="bands4")
    tk[:, 0:S] = synth.make_k(S, H, seed=4).cuda().unsqueeze(0)
    tv[:, 0:S] = synth.make_v(S, H, seed=5).cuda().unsqueeze(0)
    q = synth.make_q(1, 40, H, seed=6).cuda()
    ref = quant_kv.attention(q, tk[:, 0:S], tv[:, 0:S])
    same = [
        quant_kv.attention(q, tk[:, 0:S], tv[:, 0:S], None, torch.tensor([S]), 0.0),
        quant_kv.attention(q, tk[:, 0:S], tv[:, 0:S], q_lens=torch.tensor([40]), causal=False,
                           window_size=(-1, -1), deterministic=True, dtype=torch.bfloat16, fa_version=3),
    ]
    for o in same:
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))
    scaled = quant_kv.attention(q, tk[:, 0:S], tv[:, 0:S], softmax_scale=0.1)
    assert not torch.equal(scaled, ref)
    for bad in ({"causal": True}, {"dropout_p": 0.1}, {"window_size": (64, 64)}, {"k_lens": torch.tensor([S - 1])},
                {"q_scale": 2.0}, {"dtype": torch.float16}):
        with pytest.raises(NotImplementedError):
            quant_kv.attention(q, tk[:, 0:S], tv[:, 0:S], **bad)
    with pytest.raises(TypeError):
        quant_kv.attention(q, tk[:, 0:S], tv[:, 0:S], bogus=1)
