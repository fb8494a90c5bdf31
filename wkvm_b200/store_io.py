"""WARM and COLD snapshot tiers of wkvm's StateStore on the slot arena.

WARM (pinned host): :class:`Hibernation` copies a whole batch of slots to
pinned host memory with one snapshot kernel per state family, on a side
stream, so decode of the other slots keeps running; each session's tensors
are views with wkvm's layout ({"wkv": [L,H,K,V] fp32, "shift": [L,2,D]}, the
tensors wkvm/store.py:130-131 keeps). :func:`wake` restores sessions into
slots (one restore kernel per family for a hibernated batch).

COLD (disk): one safetensors file per handle with the same two tensors,
named ``<name>_v<version>.safetensors``, and an ``index.json`` of records,
as wkvm's StateStore.persist / _write_index write them
(wkvm/store.py:200-218, 253-254, 275-295), so files move between wkvm and
this library unchanged. :func:`persist_many` writes a hibernated batch with
a thread pool. The layout fingerprint is wkvm's (wkvm/store.py:84-88).

The reference copies one session per call with a device synchronise per
family (wkvm/store.py:127-133, 248-252); its fleet demo snapshots 2,000
finished sessions that way (experiments/m3_demos.py:87-120).
"""

from __future__ import annotations

import hashlib
import json
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Iterable, Mapping, Sequence

import torch

from . import ops

_side_streams: dict[int, torch.cuda.Stream] = {}


def _side_stream(dev: torch.device) -> torch.cuda.Stream:
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    if i not in _side_streams:
        _side_streams[i] = torch.cuda.Stream(torch.device("cuda", i))
    return _side_streams[i]


def fingerprint(layout) -> str:
    """wkvm's model-compatibility key of a state layout (sha256 of
    "rwkv7:L<n_layer>:wkv<wkv_shape>:shift<shift_shape>:<dtype>", 16 hex)."""
    key = (f"rwkv7:L{layout.n_layer}:wkv{tuple(layout.wkv_shape)}:"
           f"shift{tuple(layout.shift_shape)}:{layout.dtype}")
    return hashlib.sha256(key.encode()).hexdigest()[:16]


class Hibernation:
    """Asynchronous batched snapshot of ``slots`` (arena slot ids, the same
    id in both families as wkvm's runner assigns them) into pinned host
    memory. The copy is ordered after the work already queued on the current
    stream and runs on a side stream; :meth:`fence` orders later writes to
    those slots after it. ``buffers`` (wkv, shift) are pinned tensors of at
    least the batch's shape to reuse (allocating pinned memory costs far more
    than the copy); by default new ones are allocated."""

    def __init__(self, bank, slots: Sequence[int], buffers=None):
        self.slots = [int(s) for s in slots]
        n = len(self.slots)
        lay = bank.layout
        self.device = bank.device
        wshape = (n, lay.n_layer, *lay.wkv_shape)
        sshape = (n, lay.n_layer, 2, *lay.shift_shape)
        if buffers is None:
            self.wkv = torch.empty(wshape, dtype=torch.float32, pin_memory=True)
            self.shift = torch.empty(sshape, dtype=bank.shift.dtype, pin_memory=True)
        else:
            w, sh = buffers
            if (not w.is_pinned() or not sh.is_pinned() or w.dtype != torch.float32
                    or sh.dtype != bank.shift.dtype or w.numel() < n * w[0].numel()
                    or tuple(w.shape[1:]) != wshape[1:] or tuple(sh.shape[1:]) != sshape[1:]
                    or sh.shape[0] < n or not w.is_contiguous() or not sh.is_contiguous()):
                raise ValueError(f"buffers must be pinned contiguous {wshape} float32 and "
                                 f"{sshape} {bank.shift.dtype} (or more rows)")
            self.wkv, self.shift = w[:n], sh[:n]
        cur = torch.cuda.current_stream(self.device)
        side = _side_stream(self.device)
        side.wait_stream(cur)
        self.event = torch.cuda.Event()
        with torch.cuda.stream(side):
            if n:
                ops.slot_snapshot(bank.wkv, 1, self.slots, out=self.wkv)
                ops.slot_snapshot(bank.shift, 2, self.slots, out=self.shift)
            self.event.record(side)

    @property
    def nbytes(self) -> int:
        return self.wkv.numel() * 4 + self.shift.numel() * self.shift.element_size()

    def ready(self) -> bool:
        return self.event.query()

    def wait(self) -> "Hibernation":
        self.event.synchronize()
        return self

    def fence(self, stream: torch.cuda.Stream | None = None) -> None:
        """Makes ``stream`` (default: current) wait for the copy on the GPU,
        so the slots can be reused or freed without a host synchronise."""
        (stream or torch.cuda.current_stream(self.device)).wait_event(self.event)

    def tensors(self, i: int) -> dict[str, torch.Tensor]:
        """Session i's WARM tensors in wkvm's layout (views; call wait() first)."""
        return {"wkv": self.wkv[i], "shift": self.shift[i]}


def hibernate(bank, slots: Sequence[int], buffers=None) -> Hibernation:
    return Hibernation(bank, slots, buffers)


def pinned_buffers(bank, n: int):
    """Reusable pinned (wkv, shift) buffers for hibernating up to n sessions."""
    lay = bank.layout
    return (torch.empty((n, lay.n_layer, *lay.wkv_shape), dtype=torch.float32, pin_memory=True),
            torch.empty((n, lay.n_layer, 2, *lay.shift_shape), dtype=bank.shift.dtype,
                        pin_memory=True))


def wake(bank, slots: Sequence[int], source) -> None:
    """Restores sessions into ``slots`` on the current stream: ``source`` is a
    :class:`Hibernation` of the same length (one kernel per family) or a
    sequence of {"wkv", "shift"} dicts in wkvm's layout (pinned host or
    device tensors; one kernel per family and session)."""
    slots = [int(s) for s in slots]
    if isinstance(source, Hibernation):
        if len(source.slots) != len(slots):
            raise ValueError("hibernated batch and slot list differ in length")
        source.fence()
        ops.slot_restore(bank.wkv, 1, slots, source.wkv)
        ops.slot_restore(bank.shift, 2, slots, source.shift)
        return
    source = list(source)
    if len(source) != len(slots):
        raise ValueError("sessions and slots differ in length")
    staged = []  # pinned copies of pageable sources, alive until the restores ran
    for s, t in zip(slots, source):
        wkv = _pinned_or_device(t["wkv"], staged)
        shift = _pinned_or_device(t["shift"], staged)
        ops.slot_restore(bank.wkv, 1, [s], wkv.reshape(1, *wkv.shape))
        ops.slot_restore(bank.shift, 2, [s], shift.reshape(1, *shift.shape))
    if staged:
        # the restore kernels read host memory directly, and torch's pinned
        # allocator does not know it: a staged copy freed now could be handed
        # out again while a restore still reads it
        torch.cuda.current_stream(bank.device).synchronize()


def _pinned_or_device(t: torch.Tensor, staged: list) -> torch.Tensor:
    t = t.contiguous()
    if t.is_cuda or t.is_pinned():
        return t
    p = t.pin_memory()
    staged.append(p)
    return p


# ---------------------------------------------------------------- COLD tier


def cold_path(store_dir: str | Path, handle: str) -> Path:
    """wkvm's file name for a handle "name@version"."""
    return Path(store_dir) / f"{handle.replace('@', '_v')}.safetensors"


def save_cold(path: str | Path, tensors: Mapping[str, torch.Tensor]) -> Path:
    """Writes {"wkv", "shift"} as wkvm's StateStore.persist does."""
    from safetensors.torch import save_file

    save_file({k: tensors[k].contiguous() for k in ("wkv", "shift")}, str(path))
    return Path(path)


def load_cold(path: str | Path, pin: bool | None = None) -> dict[str, torch.Tensor]:
    """Reads a COLD file into host tensors (pinned when CUDA is present)."""
    from safetensors.torch import load_file

    out = load_file(str(path))
    if pin is None:
        pin = torch.cuda.is_available()
    return {k: (v.pin_memory() if pin else v) for k, v in out.items()}


@dataclass(frozen=True)
class Record:
    """wkvm's StateRecord fields (wkvm/store.py:42-60)."""

    name: str
    version: int
    fingerprint: str
    num_computed_tokens: int
    token_ids: tuple[int, ...]
    parent: str | None = None
    rule: str | None = None
    rule_params: dict = field(default_factory=dict)

    @property
    def handle(self) -> str:
        return f"{self.name}@{self.version}"


def write_index(store_dir: str | Path, records: Iterable[Record], cold: set[str]) -> Path:
    """index.json in wkvm's format, replaced atomically."""
    data = {}
    for r in records:
        data[r.handle] = {"name": r.name, "version": r.version, "fingerprint": r.fingerprint,
                          "num_computed_tokens": r.num_computed_tokens,
                          "token_ids": list(r.token_ids), "parent": r.parent, "rule": r.rule,
                          "rule_params": r.rule_params, "cold": r.handle in cold}
    path = Path(store_dir) / "index.json"
    tmp = path.with_suffix(".tmp")
    tmp.write_text(json.dumps(data))
    os.replace(tmp, path)
    return path


def read_index(store_dir: str | Path) -> tuple[dict[str, Record], set[str]]:
    """Records and the set of COLD handles from an index.json (wkvm's or ours)."""
    path = Path(store_dir) / "index.json"
    if not path.exists():
        return {}, set()
    recs, cold = {}, set()
    for handle, e in json.loads(path.read_text()).items():
        r = Record(name=e["name"], version=int(e["version"]), fingerprint=e["fingerprint"],
                   num_computed_tokens=int(e["num_computed_tokens"]),
                   token_ids=tuple(e["token_ids"]), parent=e.get("parent"),
                   rule=e.get("rule"), rule_params=e.get("rule_params") or {})
        recs[handle] = r
        if e.get("cold", False):
            cold.add(handle)
    return recs, cold


def persist_many(store_dir: str | Path, records: Sequence[Record], batch: Hibernation,
                 threads: int = 8) -> list[Path]:
    """Writes session i of a hibernated batch as records[i]'s COLD file (a
    thread pool of safetensors writers) and adds them to index.json."""
    if len(records) != len(batch.slots):
        raise ValueError("one record per hibernated session")
    store = Path(store_dir)
    store.mkdir(parents=True, exist_ok=True)
    batch.wait()
    with ThreadPoolExecutor(max_workers=max(1, threads)) as pool:
        paths = list(pool.map(lambda i: save_cold(cold_path(store, records[i].handle),
                                                  batch.tensors(i)), range(len(records))))
    old, cold = read_index(store)
    old.update({r.handle: r for r in records})
    cold.update(r.handle for r in records)
    write_index(store, old.values(), cold)
    return paths
