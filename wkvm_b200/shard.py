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
