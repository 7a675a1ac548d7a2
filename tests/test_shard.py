"""Head-parallel sharding host logic on CPU: 2 gloo ranks gather per-rank
attention outputs into the global head order; a rank failure surfaces as an
error on the other rank instead of a hang."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_head_range_partitions():
    from kvq import shard
    for world in (1, 2, 4, 8):
        rs = [shard.head_range(40, world, r) for r in range(world)]
        assert rs[0][0] == 0 and rs[-1][1] == 40
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
        assert len({h1 - h0 for h0, h1 in rs}) == 1
    assert shard.head_range(10, 3, 0) == (0, 4) and shard.head_range(10, 3, 2) == (7, 10)
    with pytest.raises(ValueError):
        shard.head_range(4, 8, 0)
    with pytest.raises(ValueError):
        shard.head_range(40, 2, 2)


def _gather_worker(rank, world, port, paths):
    import datetime
    import sys
    sys.path[:0] = paths
    import torch.distributed as dist
    from kvq import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    B, Lq, H, D = 2, 5, 8, 4
    h0, h1 = shard.head_range(H, world, rank)
    full = torch.arange(B * Lq * H * D, dtype=torch.float32).reshape(B, Lq, H, D)
    local = full[:, :, h0:h1].contiguous()
    g = shard.gather_outputs(local)
    out = shard.assemble_heads(g)
    ok = torch.equal(out, full)
    dist.destroy_process_group()
    if not ok:
        raise SystemExit(3)


def _run(target, world, paths):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = []
    for r in range(world):
        p = ctx.Process(target=target, args=(r, world, port, list(paths)))
        p.start()
        procs.append(p)
    for p in procs:
        p.join(timeout=120)
    return [p.exitcode for p in procs]


def test_gather_two_ranks():
    import sys
    assert _run(_gather_worker, 2, [p for p in sys.path if p]) == [0, 0]


def _failing_worker(rank, world, port, paths):
    import datetime
    import sys
    sys.path[:0] = paths
    import torch.distributed as dist
    from kvq import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(7)          # the rank dies between steps, with nothing in flight
    local = torch.zeros(1, 2, 1, 4)
    try:
        shard.gather_outputs(local)
    except Exception:
        os._exit(11)         # the survivor gets an error, not a hang
    os._exit(0)


def test_dead_rank_is_an_error_not_a_hang():
    import sys
    codes = _run(_failing_worker, 2, [p for p in sys.path if p])
    assert codes[1] == 7 and codes[0] == 11


class _FakeIpc:
    """Stands in for kvq.ops' CUDA IPC calls: a 'handle' names the exporting rank
    and the export's serial number (0 = output buffer, 1 = signal counter)."""

    def __init__(self, rank):
        self.rank = rank
        self.serial = 0
        self.opened, self.closed = [], []

    def ipc_export(self, t):
        h = (b"rank%d:%d" % (self.rank, self.serial)).ljust(64, b"\0")
        self.serial += 1
        return h, 16 * self.rank

    def ipc_import(self, handle, offset):
        peer, serial = (int(x) for x in handle.rstrip(b"\0")[4:].split(b":"))
        assert offset == 16 * peer
        base = 1000 * (peer + 1) + 100 * serial
        self.opened.append(base)
        return base, base + offset

    def ipc_close(self, base):
        self.closed.append(base)


def _peer_worker(rank, world, port, paths):
    import datetime
    import sys
    sys.path[:0] = paths
    import torch.distributed as dist
    from kvq import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    fake = _FakeIpc(rank)
    local = torch.zeros(4)
    po = shard.PeerOutputs(local, ops=fake)
    want = [local.data_ptr() if r == rank else 1000 * (r + 1) + 16 * r for r in range(world)]
    want_sig = [po.signal.data_ptr() if r == rank else 1000 * (r + 1) + 100 + 16 * r for r in range(world)]
    ok = po.ptrs == want and po.sig_ptrs == want_sig and len(fake.opened) == 2 * (world - 1)
    # the barrier target advances by one add per rank, modulo 2^32
    po.target = 0xFFFFFFFF - world + 2
    ok = ok and po.next_target() == 1 and po.next_target() == 1 + world
    po.close()
    po.close()  # idempotent
    ok = ok and sorted(fake.closed) == sorted(fake.opened)
    dist.destroy_process_group()
    if not ok:
        raise SystemExit(3)


def test_peer_outputs_exchange_three_ranks():
    """Every rank ends with the buffers of all ranks in rank order: its own
    pointer first-hand, the peers' through their exported handles and offsets."""
    import sys
    assert _run(_peer_worker, 3, [p for p in sys.path if p]) == [0, 0, 0]
