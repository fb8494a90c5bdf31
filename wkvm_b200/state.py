"""The state arena on the GPU: wkvm's RWKV7StateBank with slot-indexed
kernels in place of gather/scatter copies.

Mirrors wkvm/runner/state.py:23-100 and wkvm/models/rwkv7.py:42-99:
  wkv   [L, S+1, H, K, V] fp32   (slot 0 = reserved padding row)
  shift [L, 2, S+1, D] model dtype ([:, 0] attn token-shift, [:, 1] ffn)
Tensors, dtypes and slot semantics are identical, so wkvm's StateStore files
and fingerprints stay compatible. The differences are in how state moves:
decode/prefill kernels read and write ``wkv[layer, slot]`` in place, and
zero / fork / snapshot / restore / migrate are single kernels over all
layers instead of per-layer strided copies.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Mapping, Sequence

import torch

from . import ops

WKV_DTYPE = torch.float32


@dataclass(frozen=True)
class RWKV7StateLayout:
    """Per-slot state shapes (wkvm/models/rwkv7.py:42-99)."""

    n_layer: int
    hidden_size: int
    num_heads: int
    head_dim: int
    head_v_dim: int
    dtype: torch.dtype = torch.bfloat16

    @property
    def wkv_shape(self) -> tuple[int, ...]:
        return (self.num_heads, self.head_dim, self.head_v_dim)

    @property
    def shift_shape(self) -> tuple[int, ...]:
        return (self.hidden_size,)

    def wkv_bytes_per_slot(self) -> int:
        return self.n_layer * self.num_heads * self.head_dim * self.head_v_dim * 4

    def shift_bytes_per_slot(self) -> int:
        return self.n_layer * 2 * self.hidden_size * torch.empty((), dtype=self.dtype).element_size()


SlotDict = Mapping[str, int]


def _ids(slot_batch: Sequence[SlotDict], family: str) -> list[int]:
    return [int(s[family]) for s in slot_batch]


class RWKV7StateBank:
    """Dense slot-indexed state tensors (wkvm/runner/state.py:23-48)."""

    def __init__(self, layout: RWKV7StateLayout, num_slots: int,
                 device: torch.device | str = "cuda") -> None:
        self.layout = layout
        self.num_slots = num_slots
        self.device = torch.device(device)
        self.wkv = torch.zeros((layout.n_layer, num_slots + 1, *layout.wkv_shape),
                               dtype=WKV_DTYPE, device=self.device)
        self.shift = torch.zeros((layout.n_layer, 2, num_slots + 1, *layout.shift_shape),
                                 dtype=layout.dtype, device=self.device)

    # -- slot lifecycle ---------------------------------------------------

    def zero_slots(self, slots: SlotDict) -> None:
        """wkvm RWKV7StateBank.zero_slots (state.py:50-54): one kernel per family."""
        ops.slot_zero(self.wkv, 1, [int(slots["wkv"])])
        ops.slot_zero(self.shift, 2, [int(slots["shift"])])

    def zero_many(self, slot_batch: Sequence[SlotDict]) -> None:
        ops.slot_zero(self.wkv, 1, _ids(slot_batch, "wkv"))
        ops.slot_zero(self.shift, 2, _ids(slot_batch, "shift"))

    def fork(self, parents: Sequence[SlotDict], children: Sequence[SlotDict]) -> None:
        """Device copy child <- parent for every family (the O(MB) copy wkvm's
        StateArena.fork leaves to the runner, wkvm/core/arena.py:82-92)."""
        ops.slot_copy(self.wkv, 1, _ids(parents, "wkv"), _ids(children, "wkv"))
        ops.slot_copy(self.shift, 2, _ids(parents, "shift"), _ids(children, "shift"))

    # -- mutation rules (wkvm/store.py:260-268, 298-305) on live slots --------

    def decay(self, slots: SlotDict, alpha: float = 0.9) -> None:
        """wkv <- wkv * alpha in place; token-shift untouched (wkvm's "decay")."""
        i = [int(slots["wkv"])]
        ops.slot_affine(self.wkv, 1, i, i, None, float(alpha))

    def merge(self, dst: SlotDict, a: SlotDict, b: SlotDict, weight: float = 0.5) -> None:
        """Every family: dst <- (1 - weight) * a + weight * b (wkvm's "merge")."""
        for fam, t, dim in (("wkv", self.wkv, 1), ("shift", self.shift, 2)):
            ops.slot_affine(t, dim, [int(dst[fam])], [int(a[fam])], [int(b[fam])],
                            1.0 - float(weight), float(weight))

    # -- decode -----------------------------------------------------------

    def wkv_decode(self, layer: int, slot_ids, r, w, k, v, kk, a) -> torch.Tensor:
        """One layer's WKV step for a batch, state updated in place."""
        return ops.wkv7_decode_slots(r, w, k, v, kk, a, self.wkv, layer, slot_ids)

    def device_ids(self, slot_batch: Sequence[SlotDict], family: str = "wkv") -> torch.Tensor:
        """Validated int32 device ids for a batch (reuse across layers/steps)."""
        return ops.slot_ids_tensor(_ids(slot_batch, family), self.num_slots + 1, self.device)

    # -- gather / scatter (wkvm/runner/state.py:63-97) ----------------------

    def gather_cache(self, slot_batch: Sequence[SlotDict], resident: bool | None = None):
        """wkvm's RWKV7StateBank.gather_cache: an fla ``Cache`` seeded with the
        batch's states (offset 0), for one model forward; commit it with
        :meth:`scatter_cache`. wkvm's RWKV7Runner calls the pair around every
        forward (wkvm/runner/runner.py:53-61, 79-87).

        ``resident`` (default: whether ``fla_compat.install()`` is in effect)
        picks what the cache holds. Resident: each layer's recurrent state is
        a :class:`~wkvm_b200.fla_compat.SlotState` that the installed ops
        update in place in ``wkv[layer, slot]``, and the token-shift rows are
        gathered by one kernel; nothing of the wkv family is copied. Not
        resident: plain tensor copies, as wkvm's bank gives them (one gather
        kernel per family for all layers), for fla's own ops or any caller
        that edits the states."""
        from fla.models.utils import Cache

        from . import fla_compat

        wkv_ids = _ids(slot_batch, "wkv")
        shift_ids = _ids(slot_batch, "shift")
        if resident is None:
            resident = fla_compat.installed()
        if resident:
            h = fla_compat.slot_cache(self, wkv_ids, shift_ids=shift_ids)
            h.cache._wkvm_slot_handle = h
            return h.cache
        wkv = ops.slot_gather_outer_major(self.wkv, 1, wkv_ids)      # [L, n, H, K, V]
        shift = ops.slot_gather_outer_major(self.shift, 2, shift_ids)  # [L, 2, n, D]
        cache = Cache()
        for i in range(self.layout.n_layer):
            cache.update(recurrent_state=wkv[i], conv_state=shift[i, 0], ffn_state=shift[i, 1],
                         layer_idx=i, offset=0)
        return cache

    def scatter_cache(self, slot_batch: Sequence[SlotDict], cache) -> None:
        """wkvm's RWKV7StateBank.scatter_cache: commits a forward's states
        back to the batch's rows. For a resident cache only the token-shift
        rows move (the wkv states were updated in place)."""
        handle = getattr(cache, "_wkvm_slot_handle", None)
        if handle is not None:
            handle.commit()
            return
        wkv_ids = _ids(slot_batch, "wkv")
        shift_ids = _ids(slot_batch, "shift")
        for i in range(self.layout.n_layer):
            st = cache[i]
            ops.slot_restore(self.wkv[i], 0, wkv_ids,
                             st["recurrent_state"].to(WKV_DTYPE).contiguous())
            ops.slot_restore(self.shift[i, 0], 0, shift_ids,
                             st["conv_state"].to(self.shift.dtype).contiguous())
            ops.slot_restore(self.shift[i, 1], 0, shift_ids,
                             st["ffn_state"].to(self.shift.dtype).contiguous())

    # -- snapshot / restore (wkvm/store.py:108-156) --------------------------

    def snapshot(self, slots: SlotDict) -> dict[str, torch.Tensor]:
        """Pinned host copies {"wkv": [L,H,K,V], "shift": [L,2,D]} — the
        tensors wkvm's StateStore.save keeps in its WARM tier. Synchronises."""
        wkv = ops.slot_snapshot(self.wkv, 1, [int(slots["wkv"])])
        shift = ops.slot_snapshot(self.shift, 2, [int(slots["shift"])])
        torch.cuda.current_stream(self.device).synchronize()
        return {"wkv": wkv[0], "shift": shift[0]}

    def snapshot_many(self, slot_batch: Sequence[SlotDict]) -> dict[str, torch.Tensor]:
        """Batched snapshot: {"wkv": [n,L,H,K,V], "shift": [n,L,2,D]} pinned."""
        wkv = ops.slot_snapshot(self.wkv, 1, _ids(slot_batch, "wkv"))
        shift = ops.slot_snapshot(self.shift, 2, _ids(slot_batch, "shift"))
        torch.cuda.current_stream(self.device).synchronize()
        return {"wkv": wkv, "shift": shift}

    def restore(self, slots: SlotDict, tensors: Mapping[str, torch.Tensor]) -> None:
        """Inverse of :meth:`snapshot` (wkvm StateStore.load). Synchronises."""
        wkv = tensors["wkv"].reshape(1, *tensors["wkv"].shape)
        shift = tensors["shift"].reshape(1, *tensors["shift"].shape)
        ops.slot_restore(self.wkv, 1, [int(slots["wkv"])], _pinned(wkv))
        ops.slot_restore(self.shift, 2, [int(slots["shift"])], _pinned(shift))
        torch.cuda.current_stream(self.device).synchronize()

    # -- migration --------------------------------------------------------

    def migrate_to(self, peer: "RWKV7StateBank", src: Sequence[SlotDict],
                   dst: Sequence[SlotDict]) -> torch.cuda.Event:
        """Copies slots to ``peer`` (another GPU's bank) with peer stores.
        Returns an event recorded after the copy on this GPU's stream; the
        source slots may be freed once it completes."""
        if peer.layout != self.layout:
            raise ValueError("peer bank has a different layout")
        ops.slot_migrate(self.wkv, peer.wkv, 1, _ids(src, "wkv"), _ids(dst, "wkv"))
        ops.slot_migrate(self.shift, peer.shift, 2, _ids(src, "shift"), _ids(dst, "shift"))
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        return ev

    def state_bytes(self) -> int:
        return (self.wkv.numel() * self.wkv.element_size()
                + self.shift.numel() * self.shift.element_size())


def _pinned(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t.contiguous()
    t = t.contiguous()
    return t if t.is_pinned() else t.pin_memory()
