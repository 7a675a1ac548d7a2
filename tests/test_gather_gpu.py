"""Head-sharded attention with the all-gather in its epilogue
(kvq_attention_gather): rows land at their head offset in every destination
buffer, bit-identical to kvq_attention, and nothing else is written; on two
GPUs every rank ends with the full output, equal to the per-rank outputs
gathered by NCCL."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _caches(B, S, H, sink, seed, h0=0):
    import quant_kv
    from kvq import synth
    tk = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, "bands4", sink)
    tv = quant_kv.QuantKVTensor([B, S, H, 128], "cuda", torch.bfloat16, 4, "bands4", sink)
    tk[:, 0:S] = torch.stack([synth.make_k(S, H, seed=seed + 101 * b + h0, device="cuda") for b in range(B)])
    tv[:, 0:S] = torch.stack([synth.make_v(S, H, seed=seed + 101 * b + h0 + 1, device="cuda") for b in range(B)])
    return tk, tv


def test_gather_two_local_destinations_match_attention():
    from kvq import ops, synth
    B, S, H, Lq, sink = 2, 700, 3, 300, 130
    tk, tv = _caches(B, S, H, sink, seed=1)
    q = synth.make_q(B, Lq, H, seed=5, device="cuda")
    ref = ops.attention_packed(q, tk, tv, 0, S)
    Ht, h0, fill = 7, 2, -7.0
    bufs = [torch.full((B, Lq, Ht, 128), fill, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ops.attention_packed_gather(q, tk, tv, 0, S, [b.data_ptr() for b in bufs], h0, Ht)
    torch.cuda.synchronize()
    for b in bufs:
        assert torch.equal(b[:, :, h0:h0 + H], ref)
        assert bool((b[:, :, :h0] == fill).all()) and bool((b[:, :, h0 + H:] == fill).all())
    assert ops.device_status() == 0


def test_gather_barrier_counts_and_is_bounded():
    """Two ranks emulated on one GPU, one stream, ordered so that no barrier waits
    for a later launch: "rank 1" adds 1 to both counters and finds its own target
    met, then "rank 0" adds 1 to both and finds its target met too; the gathered
    rows are all there afterwards. A barrier whose target is never reached gives
    up, raises the status word and returns."""
    from kvq import ops, synth
    B, S, H, Lq, sink = 2, 500, 3, 300, 100
    tk, tv = _caches(B, S, H, sink, seed=4)
    q = synth.make_q(B, Lq, H, seed=8, device="cuda")
    ref = ops.attention_packed(q, tk, tv, 0, S)
    bufs = [torch.zeros((B, Lq, H, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ctr = torch.zeros(2 * 64, dtype=torch.int32, device="cuda")
    ptrs = [ctr.data_ptr(), ctr.data_ptr() + 256]
    for step in (1, 2):
        ops.attention_packed_gather(q, tk, tv, 0, S, [b.data_ptr() for b in bufs], 0, H)
        # "rank 1" signals first (it never waits long: its own target is reached by
        # its own add plus rank 0's add of the previous step), then rank 0
        ops.gather_barrier(ptrs, 1, 2 * step - 1)
        ops.gather_barrier(ptrs, 0, 2 * step)
        torch.cuda.synchronize()
        assert int(ctr[0]) == 2 * step and int(ctr[64]) == 2 * step
        for b in bufs:
            assert torch.equal(b, ref)
    assert ops.device_status() == 0
    ops.gather_barrier(ptrs, 0, 2 * 2 + 2, wait_cycles=200_000)   # only one more add will come
    torch.cuda.synchronize()
    assert ops.device_status(reset=True) == 1
    assert ops.device_status() == 0


def test_gather_window_and_padded_token_stride():
    """A window [lo, hi) inside the sink border and an output token stride wider
    than heads * D."""
    from kvq import ops, synth
    B, S, H, Lq, sink = 1, 900, 2, 77, 200
    tk, tv = _caches(B, S, H, sink, seed=2)
    q = synth.make_q(B, Lq, H, seed=6, device="cuda")
    lo, hi = 150, 611
    ref = ops.attention_packed(q, tk, tv, lo, hi)
    Ht, h0, stride = 4, 1, 4 * 128 + 64
    raw = torch.zeros((B, Lq, stride), dtype=torch.bfloat16, device="cuda")
    ops.attention_packed_gather(q, tk, tv, lo, hi, [raw.data_ptr()], h0, Ht, out_token_stride=stride)
    torch.cuda.synchronize()
    got = raw[:, :, : Ht * 128].view(B, Lq, Ht, 128)[:, :, h0:h0 + H]
    assert torch.equal(got, ref)
    assert bool((raw[:, :, Ht * 128:] == 0).all())


def test_gather_rejects_bad_arguments():
    from kvq import ops, synth
    tk, tv = _caches(1, 256, 2, 0, seed=3)
    q = synth.make_q(1, 16, 2, seed=7, device="cuda")
    buf = torch.zeros((1, 16, 4, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.attention_packed_gather(q, tk, tv, 0, 256, [buf.data_ptr()], 3, 4)   # heads 3..4 of 4
    with pytest.raises(ValueError):
        ops.attention_packed_gather(q, tk, tv, 0, 256, [buf.data_ptr()] * 9, 0, 4)
    with pytest.raises(ValueError):
        ops.attention_packed_gather(q, tk, tv, 0, 256, [buf.data_ptr() + 2], 0, 4)  # misaligned


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_gpu_worker(rank, world, port, paths):
    import datetime
    import sys
    sys.path[:0] = paths
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from kvq import ops, shard, synth
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    B, S, H, Lq, sink = 2, 640, 8, 333, 128
    h0, h1 = shard.head_range(H, world, rank)
    tk, tv = _caches(B, S, h1 - h0, sink, seed=9, h0=h0)
    q = synth.make_q(B, Lq, h1 - h0, seed=11 + h0, device=dev)
    full = torch.zeros((B, Lq, H, 128), dtype=torch.bfloat16, device=dev)
    po = shard.PeerOutputs(full)
    ref = shard.assemble_heads(shard.gather_outputs(ops.attention_packed(q, tk, tv, 0, S)))
    ok = True
    for _step in range(3):
        # completion by the device-side signal: no synchronize, no barrier between
        # the launch and the read of the gathered rows
        full.zero_()
        torch.cuda.synchronize()
        dist.barrier()                      # every rank cleared its buffer before anyone stores
        ops.attention_packed_gather(q, tk, tv, 0, S, po.ptrs, h0, H)
        po.barrier(wait_cycles=200_000_000)
        ok = ok and torch.equal(full, ref)
        torch.cuda.synchronize()
        dist.barrier()                      # every rank compared before the next step clears
    ok = ok and ops.device_status() == 0
    dist.barrier()          # every peer is done with `full` before it is unmapped and freed
    po.close()
    dist.barrier()
    dist.destroy_process_group()
    if not ok:
        raise SystemExit(3)


def test_gather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import sys
    paths = [p for p in sys.path if p]
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, paths)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:                 # a stuck worker must not keep holding its GPU
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0, 0]
