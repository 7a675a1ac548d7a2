"""The bounded waits of the attention kernel: a launch whose K tiles stop
arriving gives up instead of hanging, raises the library's device status word,
lets its in-flight copies and MMAs finish and frees its tensor memory, so the
next launch on the same context runs normally and gives the same bits as
before. The stall is made on purpose by the producer (a test hook of the
library), with every wait limited to 1e5 cycles; nothing faults or traps."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("stall_tile", [0, 3])
def test_stalled_launch_times_out_and_context_stays_usable(stall_tile):
    import quant_kv
    from kvq import ops, synth
    B, S, H, Lq, sink = 1, 640, 2, 300, 128
    tk = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, "bands4", sink)
    tv = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, "bands4", sink)
    tk[:, 0:S] = synth.make_k(S, H, seed=5, device="cuda").unsqueeze(0)
    tv[:, 0:S] = synth.make_v(S, H, seed=6, device="cuda").unsqueeze(0)
    q = synth.make_q(B, Lq, H, seed=7, device="cuda")
    assert ops.device_status(reset=True) == 0
    before = ops.attention_packed(q, tk, tv, 0, S).clone()
    torch.cuda.synchronize()

    ops.attention_timeout_test(q, tk, tv, 0, S, stall_tile=stall_tile, wait_cycles=100_000)
    torch.cuda.synchronize()                       # the launch returned: no hang, no fault
    assert ops.device_status(reset=False) == 1     # it reported the timeout
    assert ops.device_status(reset=True) == 1      # reading with reset returns it once ...
    assert ops.device_status(reset=False) == 0     # ... and clears it

    # tensor memory was released and the context works: same bits as before
    after = ops.attention_packed(q, tk, tv, 0, S)
    torch.cuda.synchronize()
    assert torch.equal(after.view(torch.int16), before.view(torch.int16))
    assert ops.device_status(reset=True) == 0


def test_timeout_hook_rejects_bad_limits():
    import quant_kv
    from kvq import ops, synth
    tk = quant_kv.QuantKVTensor([1, 128, 1, 128], "cuda", torch.bfloat16, 4, "bands4", 0)
    tv = quant_kv.QuantKVTensor([1, 128, 1, 128], "cuda", torch.bfloat16, 4, "bands4", 0)
    q = synth.make_q(1, 16, 1, seed=1, device="cuda")
    with pytest.raises(ValueError):
        ops.attention_timeout_test(q, tk, tv, 0, 128, stall_tile=0, wait_cycles=10)
    with pytest.raises(ValueError):
        ops.attention_timeout_test(q, tk, tv, 0, 128, stall_tile=-1, wait_cycles=100_000)
