"""Slot sharding across GPUs and live slot migration.

Each GPU (one process per GPU, torch.distributed) owns one arena shard:
its own RWKV7StateBank with ``slots_per_rank`` usable slots (local slot 0
stays wkvm's reserved padding row). A request's state lives in exactly one
shard, so decode, prefill, fork and snapshot never communicate; the only
exchange is migrating a slot to another GPU:

  1. the destination rank allocates local slots,
  2. the source packs the slots' rows of every state family into one
     contiguous buffer (the slot snapshot kernel, device-to-device),
  3. the buffer crosses NVLink as one point-to-point send (NCCL),
  4. the destination scatters it into its slots (slot restore kernel) and
     sends an acknowledgement,
  5. the source frees its slots only after the acknowledgement arrived.

Every wait is bounded (``timeout``); a missing peer or message raises
MigrationTimeout on the host and leaves the source slots allocated, so no
state is lost. Within one process that drives two GPUs, RWKV7StateBank.
migrate_to copies with peer stores instead (wkvm_slot_migrate).

wkvm keeps the slot bookkeeping in StateArena (wkvm/core/arena.py:26-96) and
has no multi-GPU path; its README only plans migration (README.md:221).
"""

from __future__ import annotations

import datetime as _dt
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch
import torch.distributed as dist


class MigrationTimeout(RuntimeError):
    """A peer did not send or acknowledge within the timeout."""


@dataclass
class ShardArena:
    """Integer slot allocator of one shard (the behaviour of wkvm's
    StateArena.allocate/free: slot 0 reserved, LIFO reuse, double free is an
    error)."""

    num_slots: int
    _free: list[int] = field(default_factory=list)
    _live: set[int] = field(default_factory=set)

    def __post_init__(self):
        self._free = list(range(self.num_slots, 0, -1))

    def allocate(self, n: int = 1) -> list[int]:
        if n > len(self._free):
            raise RuntimeError(f"shard full: {n} slots requested, {len(self._free)} free")
        out = [self._free.pop() for _ in range(n)]
        self._live.update(out)
        return out

    def free(self, ids: Sequence[int]) -> None:
        for i in ids:
            if i not in self._live:
                raise KeyError(f"slot {i} is not allocated")
            self._live.remove(i)
            self._free.append(i)

    def claim(self, ids: Sequence[int]) -> None:
        """Marks the given free slots live (sessions placed by id)."""
        for i in ids:
            if i in self._live or not 0 < i <= self.num_slots:
                raise KeyError(f"slot {i} is not free")
        gone = set(ids)
        self._free = [i for i in self._free if i not in gone]
        self._live.update(gone)

    @property
    def num_free(self) -> int:
        return len(self._free)

    def is_live(self, i: int) -> bool:
        return i in self._live


@dataclass(frozen=True)
class GlobalSlot:
    rank: int
    local: int


class ShardMap:
    """Global view: which rank holds which request's slot."""

    def __init__(self, world_size: int, slots_per_rank: int):
        self.world_size = world_size
        self.arenas = [ShardArena(slots_per_rank) for _ in range(world_size)]
        self.where: dict[str, GlobalSlot] = {}

    def place(self, request: str, rank: int | None = None) -> GlobalSlot:
        """Allocates a slot for ``request`` on ``rank`` (default: the rank
        with the most free slots, which balances weak-scaled decode)."""
        if request in self.where:
            raise KeyError(f"{request} already placed")
        if rank is None:
            rank = max(range(self.world_size), key=lambda r: self.arenas[r].num_free)
        gs = GlobalSlot(rank, self.arenas[rank].allocate(1)[0])
        self.where[request] = gs
        return gs

    def release(self, request: str) -> None:
        gs = self.where.pop(request)
        self.arenas[gs.rank].free([gs.local])

    def plan_move(self, request: str, dst_rank: int) -> tuple[GlobalSlot, GlobalSlot]:
        """Reserves the destination slot (step 1); the source stays live
        until :meth:`commit_move`."""
        src = self.where[request]
        if src.rank == dst_rank:
            raise ValueError("request already lives on that rank")
        dst = GlobalSlot(dst_rank, self.arenas[dst_rank].allocate(1)[0])
        return src, dst

    def commit_move(self, request: str, src: GlobalSlot, dst: GlobalSlot) -> None:
        self.arenas[src.rank].free([src.local])
        self.where[request] = dst

    def abort_move(self, dst: GlobalSlot) -> None:
        self.arenas[dst.rank].free([dst.local])


Packer = Callable[[Sequence[int]], torch.Tensor]
Unpacker = Callable[[Sequence[int], torch.Tensor], None]


def bank_packer(bank) -> tuple[Packer, Unpacker, Callable[[int], torch.Tensor]]:
    """Pack / unpack / receive-buffer callables over an RWKV7StateBank: the
    rows of both state families for n slots as one flat byte tensor on the
    bank's GPU (slot snapshot / restore kernels, no host round trip)."""
    from . import ops

    lay = bank.layout
    wkv_row = lay.wkv_bytes_per_slot()
    shift_row = lay.shift_bytes_per_slot()
    per_slot = wkv_row + shift_row

    def empty(n: int) -> torch.Tensor:
        return torch.empty(n * per_slot, dtype=torch.uint8, device=bank.device)

    def pack(ids):
        n = len(ids)
        buf = empty(n)
        wkv = buf[: n * wkv_row].view(torch.float32).view(n, *bank.wkv.shape[:1], *bank.wkv.shape[2:])
        shift = buf[n * wkv_row:].view(bank.shift.dtype).view(n, *bank.shift.shape[:2], *bank.shift.shape[3:])
        ops.slot_snapshot(bank.wkv, 1, ids, out=wkv)
        ops.slot_snapshot(bank.shift, 2, ids, out=shift)
        return buf

    def unpack(ids, buf):
        n = len(ids)
        wkv = buf[: n * wkv_row].view(torch.float32).view(n, *bank.wkv.shape[:1], *bank.wkv.shape[2:])
        shift = buf[n * wkv_row:].view(bank.shift.dtype).view(n, *bank.shift.shape[:2], *bank.shift.shape[3:])
        ops.slot_restore(bank.wkv, 1, ids, wkv)
        ops.slot_restore(bank.shift, 2, ids, shift)

    return pack, unpack, empty


def _wait(work, timeout: float, what: str) -> None:
    try:
        ok = work.wait(timeout=_dt.timedelta(seconds=timeout))
    except RuntimeError as e:  # backends raise on timeout
        raise MigrationTimeout(f"{what}: {e}") from e
    if ok is False:
        raise MigrationTimeout(f"{what}: timed out after {timeout}s")


def send_slots(ids: Sequence[int], dst_rank: int, pack: Packer, *, group=None,
               timeout: float = 30.0, tag: int = 0) -> None:
    """Source side of a migration (steps 2, 3 and the wait for step 4's ack).
    The caller frees ``ids`` after this returns; on MigrationTimeout it keeps
    them."""
    buf = pack(ids)
    if buf.is_cuda:
        torch.cuda.current_stream(buf.device).synchronize()
    _wait(dist.isend(buf, dst_rank, group=group, tag=tag), timeout, "send")
    ack = torch.zeros(1, dtype=torch.int32, device=buf.device)
    _wait(dist.irecv(ack, dst_rank, group=group, tag=tag + 1), timeout, "acknowledgement")
    if int(ack.item()) != len(ids):
        raise RuntimeError(f"peer acknowledged {int(ack.item())} of {len(ids)} slots")


def recv_slots(ids: Sequence[int], src_rank: int, unpack: Unpacker,
               empty: Callable[[int], torch.Tensor], *, group=None, timeout: float = 30.0,
               tag: int = 0) -> None:
    """Destination side: receive into preallocated local slots ``ids``,
    restore them and acknowledge."""
    buf = empty(len(ids))
    _wait(dist.irecv(buf, src_rank, group=group, tag=tag), timeout, "receive")
    unpack(ids, buf)
    if buf.is_cuda:
        torch.cuda.current_stream(buf.device).synchronize()
    ack = torch.full((1,), len(ids), dtype=torch.int32, device=buf.device)
    _wait(dist.isend(ack, src_rank, group=group, tag=tag + 1), timeout, "acknowledge")


class RingMigrator:
    """Migration around the ring rank -> rank + 1 that never blocks the host
    (the steady-state form a serving loop uses between decode steps).

    :meth:`start` enqueues, on a side stream that first waits for the
    caller's current stream (so the outgoing rows are final): pack the
    outgoing slots, one NCCL send to rank + 1 paired with one receive from
    rank - 1, unpack into the caller's newly allocated slots, then the
    acknowledgement exchange (each rank tells its sender how many slots it
    restored). Nothing waits on the host. :meth:`fence` makes a stream wait
    for the restores before it reads the incoming slots. :meth:`reap` returns
    the outgoing slots whose acknowledgement has arrived, which the caller may
    now free (step 5 of the protocol above); a migration unacknowledged for
    ``timeout`` seconds raises MigrationTimeout and its slots stay allocated.

    With CPU buffers (gloo) the same calls run synchronously."""

    def __init__(self, pack: Packer, unpack: Unpacker, empty: Callable[[int], torch.Tensor],
                 rank: int, world: int, *, device=None, group=None, timeout: float = 30.0):
        if world < 2:
            raise ValueError("migration needs at least two ranks")
        self.pack, self.unpack, self.empty = pack, unpack, empty
        self.rank, self.world, self.group, self.timeout = rank, world, group, timeout
        self.dst, self.src = (rank + 1) % world, (rank - 1) % world
        self.device = torch.device(device) if device is not None else None
        cuda = self.device is not None and self.device.type == "cuda"
        self.stream = torch.cuda.Stream(self.device) if cuda else None
        self._pending: list = []
        self._last = None

    def _p2p(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        ops_ = [dist.P2POp(dist.isend, send, self.dst, group=self.group),
                dist.P2POp(dist.irecv, recv, self.src, group=self.group)]
        for w in dist.batch_isend_irecv(ops_):
            w.wait()  # NCCL: the side stream waits; gloo: the host does

    def start(self, out_ids: Sequence[int], in_ids: Sequence[int]) -> None:
        """Sends ``out_ids`` to rank + 1 and receives rank - 1's slots into
        ``in_ids`` (the same count on every rank)."""
        import contextlib
        import time

        out_ids, in_ids = list(out_ids), list(in_ids)
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            ctx = torch.cuda.stream(self.stream)
        else:
            ctx = contextlib.nullcontext()
        with ctx:
            sendbuf = self.pack(out_ids)
            recvbuf = self.empty(len(in_ids))
            self._p2p(sendbuf, recvbuf)
            self.unpack(in_ids, recvbuf)
            dev = sendbuf.device
            ack_out = torch.full((1,), len(in_ids), dtype=torch.int32, device=dev)
            ack_in = torch.full((1,), -1, dtype=torch.int32, device=dev)
            # the acknowledgement goes back to the sender (rank - 1) and ours
            # comes from rank + 1: the ring in the other direction
            ops_ = [dist.P2POp(dist.isend, ack_out, self.src, group=self.group),
                    dist.P2POp(dist.irecv, ack_in, self.dst, group=self.group)]
            for w in dist.batch_isend_irecv(ops_):
                w.wait()
            if self.stream is not None:
                host = torch.empty(1, dtype=torch.int32, pin_memory=True)
                host.copy_(ack_in, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
                for t in (sendbuf, recvbuf, ack_out, ack_in):
                    t.record_stream(self.stream)
            else:
                host, ev = ack_in, None
        self._last = ev
        self._pending.append((ev, host, out_ids, time.monotonic()))

    def fence(self, stream=None) -> None:
        """Makes ``stream`` (default: current) wait for the restores so far."""
        if self._last is not None:
            (stream or torch.cuda.current_stream(self.device)).wait_event(self._last)

    def reap(self, block: bool = False) -> list[int]:
        """Outgoing slot ids acknowledged since the last call (free them)."""
        import time

        done, keep = [], []
        for ev, host, ids, t0 in self._pending:
            if ev is not None and not ev.query():
                if block:
                    while not ev.query():
                        if time.monotonic() - t0 > self.timeout:
                            raise MigrationTimeout("acknowledgement: timed out")
                        time.sleep(1e-4)
                elif time.monotonic() - t0 > self.timeout:
                    raise MigrationTimeout(f"acknowledgement: none after {self.timeout}s")
                else:
                    keep.append((ev, host, ids, t0))
                    continue
            if int(host.item()) != len(ids):
                raise RuntimeError(f"peer acknowledged {int(host.item())} of {len(ids)} slots")
            done.extend(ids)
        self._pending = keep
        return done

    @property
    def in_flight(self) -> int:
        return len(self._pending)
