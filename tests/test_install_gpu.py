import pytest
import torch

pytestmark = pytest.mark.gpu


def test_install_allocates_quant_tensors():
    import quant_kv

    class Cfg:
        num_heads, dim = 40, 5120

    class P:
        local_attn_size = 3
        frame_seq_length = 1560
        num_transformer_blocks = 3

        def _initialize_kv_cache(self, batch_size, dtype, device):
            raise AssertionError

        class generator:
            class model:
                config = Cfg

    p = P()
    quant_kv.install(p, group_mode="bands4", sink_frames=1, verbose=True)
    p._initialize_kv_cache(1, torch.bfloat16, "cuda")
    k = p.kv_cache1[0]["k"]
    assert isinstance(k, quant_kv.QuantKVTensor) and k.shape == (1, 4680, 40, 128)
    assert k.packed.shape == (4680, 40, 64) and k.scales.shape == (4680, 40, 12)
    assert k.sink.shape == (1560, 40, 128)
