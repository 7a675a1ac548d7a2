"""Host-side logic of the drop-in modules (CPU): group maps, slicing rules and
the no-CPU-path contract."""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as ko


def test_band_edges_equal_oracle():
    import quant_kv
    for mode in ("bands", "bands2", "bands3", "bands4", "bands8", "blind16", "blind32", "blind64"):
        assert quant_kv._band_edges(128, mode) == ko.band_edges(128, mode)
    assert quant_kv._band_edges(96, "blind64") == ((0, 64), (64, 96))
    with pytest.raises(ValueError):
        quant_kv._band_edges(128, "x")


def test_build_chan_band_and_host_copy():
    import quant_kv_kernels as qk
    bands = ko.band_edges(128, "bands4")
    t = qk.build_chan_band(bands, 128, "cpu")
    assert t.dtype == torch.int32 and t.shape == (128,)
    np.testing.assert_array_equal(t.numpy(), ko.chan_band(bands, 128))
    np.testing.assert_array_equal(qk.host_chan_band(t), ko.chan_band(bands, 128))
    np.testing.assert_array_equal(qk.host_chan_band([0] * 64 + [1] * 64), [0] * 64 + [1] * 64)


def test_token_slice_rules():
    import quant_kv
    assert quant_kv._token_slice((slice(None), slice(3, 9))) == slice(3, 9)
    with pytest.raises(TypeError):
        quant_kv._token_slice(slice(0, 4))
    with pytest.raises(AssertionError):
        quant_kv._token_slice((slice(0, 1), slice(3, 9)))
    with pytest.raises(AssertionError):
        quant_kv._token_slice((slice(None), slice(0, 8, 2)))


def test_no_cpu_path():
    import quant_kv
    import quant_kv_kernels as qk
    with pytest.raises(RuntimeError, match="CUDA"):
        quant_kv.QuantKVTensor([1, 16, 2, 128], "cpu")
    cb = qk.build_chan_band(ko.band_edges(128, "bands"), 128, "cpu")
    x = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        qk.quantize(x, cb, 3, 7)
    with pytest.raises(ValueError):
        qk.quantize(x, cb, 3, 5)
    with pytest.raises(TypeError):
        qk.quantize(x.float(), cb, 3, 7)


def test_drop_in_surface():
    import quant_kv
    import quant_kv_kernels as qk
    for name in ("quantize", "dequantize", "build_chan_band", "HAVE_TRITON"):
        assert hasattr(qk, name)
    assert qk.HAVE_TRITON  # the library loads (no GPU needed to load it)
    for name in ("QuantKVTensor", "install", "_band_edges", "ROPE_BANDS", "FRAME_SEQ_LEN",
                 "HAVE_KERNELS", "USE_KERNELS"):
        assert hasattr(quant_kv, name)
    assert quant_kv.FRAME_SEQ_LEN == 1560


def test_install_patches_and_reuses(monkeypatch):
    """install() swaps _initialize_kv_cache (quant_kv.py:228-269); checked with a
    fake pipeline and a recording QuantKVTensor so no GPU is needed."""
    import quant_kv
    made = []

    class FakeQ:
        def __init__(self, shape, device, dtype, bits, mode, sink):
            self.shape = list(shape)
            self.args = (device, dtype, bits, mode, sink)
            self.zeroed = 0
            made.append(self)

        def zero_(self):
            self.zeroed += 1

        def storage_bytes(self):
            return 10

    monkeypatch.setattr(quant_kv, "QuantKVTensor", FakeQ)

    class Cfg:
        num_heads, dim = 40, 5120

    class P:
        local_attn_size = 3
        frame_seq_length = 1560
        num_transformer_blocks = 2

        def _initialize_kv_cache(self, batch_size, dtype, device):
            raise AssertionError("original must not run")

        class generator:
            class model:
                config = Cfg

    p = P()
    orig = quant_kv.install(p, k_bits=4, v_bits=8, group_mode="bands4", sink_frames=1, verbose=False)
    assert callable(orig)
    p._initialize_kv_cache(1, torch.bfloat16, "cuda")
    assert len(p.kv_cache1) == 2 and p.k_shape == [1, 4680, 40, 128]
    assert p.kv_cache1[0]["v"].args[2] == 8 and p.kv_cache1[0]["k"].args[4] == 1560
    n = len(made)
    p.kv_cache1[0]["global_end_index"] = 5
    p._initialize_kv_cache(1, torch.bfloat16, "cuda")   # same shape: reuse + zero
    assert len(made) == n and made[0].zeroed == 1 and p.kv_cache1[0]["global_end_index"] == 0
    p.local_attn_size = -1
    p._initialize_kv_cache(1, torch.bfloat16, "cuda")
    assert p.k_shape == [1, 32760, 40, 128]
