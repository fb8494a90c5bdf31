"""Cross-process slot migration over NCCL between two GPUs (one process per
GPU, as the serving deployment runs). Needs two GPUs; NVLS is switched off
and the processes only exchange between steps."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    import torch.distributed as dist
    from wkvm_b200 import shard
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
    lay = RWKV7StateLayout(n_layer=3, hidden_size=64, num_heads=2, head_dim=32, head_v_dim=32)
    bank = RWKV7StateBank(lay, num_slots=5, device=dev)
    if rank == 0:
        bank.wkv.normal_(generator=torch.Generator(device=dev).manual_seed(1))
        bank.shift.normal_(generator=torch.Generator(device=dev).manual_seed(2))
    pack, unpack, empty = shard.bank_packer(bank)
    if rank == 0:
        shard.send_slots([2, 4], 1, pack, timeout=60)
        q.put(("src", bank.wkv[:, [2, 4]].cpu(), bank.shift[:, :, [2, 4]].cpu()))
    else:
        shard.recv_slots([1, 3], 0, unpack, empty, timeout=60)
        q.put(("dst", bank.wkv[:, [1, 3]].cpu(), bank.shift[:, :, [1, 3]].cpu()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_migration_bit_exact():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((item[0], item[1:]) for item in (q.get(timeout=120), q.get(timeout=120)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert torch.equal(got["src"][0], got["dst"][0])
    assert torch.equal(got["src"][1], got["dst"][1])


def _ring_worker(rank, port, q):
    import torch.distributed as dist
    from wkvm_b200 import shard
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
    lay = RWKV7StateLayout(n_layer=3, hidden_size=64, num_heads=2, head_dim=32, head_v_dim=32)
    bank = RWKV7StateBank(lay, num_slots=8, device=dev)
    bank.wkv.normal_(generator=torch.Generator(device=dev).manual_seed(10 + rank))
    bank.shift.normal_(generator=torch.Generator(device=dev).manual_seed(20 + rank))
    sent = (bank.wkv[:, [1, 2, 3]].cpu(), bank.shift[:, :, [1, 2, 3]].cpu())
    mig = shard.RingMigrator(*shard.bank_packer(bank), rank, 2, device=dev, timeout=60)
    mig.start([1, 2, 3], [6, 7, 8])
    mig.fence()
    freed = mig.reap(block=True)
    got = (bank.wkv[:, [6, 7, 8]].cpu(), bank.shift[:, :, [6, 7, 8]].cpu())
    q.put((rank, sent, got, freed))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ring_migration_stream_ordered_bit_exact():
    """RingMigrator between two GPUs: each side sends three slots and
    receives the other's three, with no host wait until the reap."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ring_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((item[0], item[1:]) for item in (q.get(timeout=120), q.get(timeout=120)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        sent_by_peer = out[1 - r][0]
        got, freed = out[r][1], out[r][2]
        assert torch.equal(got[0], sent_by_peer[0]) and torch.equal(got[1], sent_by_peer[1])
        assert freed == [1, 2, 3]
