"""Slot sharding and the migration protocol, as world_size-2 gloo ranks on
CPU. The packer is a test stand-in over CPU tensors (the GPU packer uses the
slot snapshot/restore kernels, covered by the GPU tests); what is tested here
is the host protocol: allocation order, send/ack, free-after-ack, bounded
waits when a peer never answers."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wkvm_b200 import shard


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_packer(bank):
    def pack(ids):
        return bank[list(ids)].contiguous().view(-1)

    def unpack(ids, buf):
        bank[list(ids)] = buf.view(len(ids), *bank.shape[1:])

    def empty(n):
        return torch.empty(n * bank[0].numel(), dtype=bank.dtype)

    return pack, unpack, empty


def _worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=20))
    try:
        smap = shard.ShardMap(world, slots_per_rank=6)
        # identical bookkeeping on both ranks (it is replicated host state)
        for i in range(4):
            smap.place(f"req{i}", rank=0)
        bank = torch.zeros(7, 3, 5)
        if rank == 0:
            for s in range(1, 7):
                bank[s] = s + torch.arange(15.0).view(3, 5)
        pack, unpack, empty = _cpu_packer(bank)
        src, dst = smap.plan_move("req2", 1)
        if mode == "ok":
            if rank == 0:
                shard.send_slots([src.local], 1, pack, timeout=10)
                smap.commit_move("req2", src, dst)
                q.put(("r0", smap.arenas[0].is_live(src.local), smap.where["req2"].rank))
            else:
                shard.recv_slots([dst.local], 0, unpack, empty, timeout=10)
                expected = src.local + torch.arange(15.0).view(3, 5)
                q.put(("r1", bool(torch.equal(bank[dst.local], expected)), dst.local))
        else:  # the destination never answers
            if rank == 0:
                try:
                    shard.send_slots([src.local], 1, pack, timeout=2)
                    q.put(("r0", "no-timeout"))
                except shard.MigrationTimeout:
                    smap.abort_move(dst)
                    q.put(("r0", "timeout", smap.arenas[0].is_live(src.local)))
            else:
                q.put(("r1", "silent"))
    finally:
        if mode == "ok":
            dist.barrier()
        dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        item = q.get(timeout=60)
        out[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
    return out


def test_migration_moves_rows_and_frees_source_after_ack():
    out = _run("ok")
    assert out["r1"][0] is True           # destination rows equal the source's
    assert out["r0"] == (False, 1)        # source slot freed, request now on rank 1


def test_migration_timeout_keeps_source_slot():
    out = _run("silent")
    assert out["r0"][0] == "timeout"
    assert out["r0"][1] is True           # source slot still allocated: no state lost


def test_shard_arena_and_map():
    a = shard.ShardArena(3)
    assert a.allocate(2) == [1, 2]        # slot 0 is never handed out
    a.free([1])
    assert a.allocate(1) == [1]
    with pytest.raises(KeyError):
        a.free([3])
    with pytest.raises(RuntimeError, match="full"):
        a.allocate(2)
    m = shard.ShardMap(2, 2)
    g0 = m.place("a")
    g1 = m.place("b")
    assert {g0.rank, g1.rank} == {0, 1}   # placement balances free slots
    src, dst = m.plan_move("a", 1 - g0.rank)
    m.abort_move(dst)
    assert m.where["a"] == src
    src, dst = m.plan_move("a", 1 - g0.rank)
    m.commit_move("a", src, dst)
    assert m.where["a"] == dst and not m.arenas[src.rank].is_live(src.local)


def _ring_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=20))
    try:
        bank = torch.zeros(9, 3, 5)
        for s in range(1, 9):
            bank[s] = 100 * rank + s + torch.arange(15.0).view(3, 5)
        pack, unpack, empty = _cpu_packer(bank)
        arena = shard.ShardArena(8)
        live = arena.allocate(4)                       # slots 1..4 hold sessions
        mig = shard.RingMigrator(pack, unpack, empty, rank, world, timeout=10)
        incoming = arena.allocate(2)                   # step 1: destination allocates
        mig.start([live[0], live[1]], incoming)        # steps 2-4
        freed = mig.reap(block=True)                   # step 5: free after the ack
        arena.free(freed)
        src = (rank - 1) % world
        expected = torch.stack([100 * src + s + torch.arange(15.0).view(3, 5) for s in (1, 2)])
        q.put((rank, bool(torch.equal(bank[incoming], expected)), freed,
               [arena.is_live(s) for s in (1, 2, 3, 4)], mig.in_flight))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_ring_migration_three_ranks():
    """RingMigrator over three gloo ranks: every rank sends two sessions to
    the next and receives two from the previous; the acknowledgement flows
    back the other way and only then are the sent slots freed."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ring_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    out = dict((item[0], item[1:]) for item in (q.get(timeout=60) for _ in range(3)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(3):
        ok, freed, live, in_flight = out[r]
        assert ok, r
        assert freed == [1, 2] and live == [False, False, True, True] and in_flight == 0
