"""Whole decode step as one CUDA graph over slot-resident state.

Counterpart of the reference engine's GraphedDecode
(wkvm experiments/m2_engine_bench.py:44-113). There, the graph captures only
the model forward on static state copies: every step still gathers each
layer's states into the static inputs (3 x L index_select) before the replay
and scatters them back (3 x L index_copy_) after it. Here the captured step
reads and writes the arena in place through slot ids held in static device
buffers, so a step is: copy the batch's slot ids and last tokens into the
static buffers, replay, read the logits. Nothing is gathered or scattered
outside the graph.

With ``fla_compat.install(fuse_time_mix=True)`` (the default here) the
captured step runs the fused time-mix core and the token-shift prologues on
the arena's shift rows; otherwise fla's forward with wkvm_b200's WKV ops, and
the token-shift rows are gathered and restored inside the graph.

Batches smaller than the captured size are padded with slot 0, wkvm's
reserved padding row (wkvm/core/arena.py:32-37): padded rows decode into
slot 0, whose contents are never read back.
"""

from __future__ import annotations

import torch

from . import fla_compat, ops


class GraphedDecode:
    """CUDA graph of one decode step of ``runner.model`` for up to
    ``batch_size`` slots of ``runner.bank`` (wkvm's GraphedDecode interface:
    construct once, then ``decode_step(slot_batch, last_tokens)``)."""

    def __init__(self, runner, batch_size: int, fuse_time_mix: bool = True,
                 overlap: bool = True) -> None:
        self.runner, self.batch_size = runner, batch_size
        self.fuse = fuse_time_mix
        self.overlap = overlap
        bank = runner.bank
        dev = bank.device
        self.tokens = torch.zeros(batch_size, 1, dtype=torch.long, device=dev)
        self.wkv_ids = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.shift_ids = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self._host = torch.zeros(3, batch_size, dtype=torch.int64, pin_memory=True)
        self._staged = None  # event: the last H2D copy out of _host finished
        ops.status_word(dev)
        fla_compat.install(fuse_time_mix=fuse_time_mix)
        prev = ops.set_decode_overlap(overlap)
        try:
            with torch.inference_mode():
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    for _ in range(2):  # every static id is slot 0 here
                        self._forward()
                torch.cuda.current_stream(dev).wait_stream(side)
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self.logits = self._forward()
        finally:
            ops.set_decode_overlap(prev)

    def _forward(self) -> torch.Tensor:
        h = fla_compat.slot_cache(self.runner.bank, self.wkv_ids, shift_in_bank=self.fuse,
                                  shift_ids=self.shift_ids)
        out = self.runner.model(input_ids=self.tokens, past_key_values=h.cache, use_cache=True,
                                logits_to_keep=1)
        h.commit()
        return out.logits

    @torch.inference_mode()
    def decode_step(self, slot_batch: list[dict[str, int]], last_tokens: list[int]) -> torch.Tensor:
        """Advances every slot of the batch by its last token; returns fp32
        next-token logits ``[len(slot_batch), vocab]``. The graph was captured
        with ``fla_compat`` installed as chosen at construction; it replays
        the same kernels whatever is installed now."""
        n = len(slot_batch)
        if n != len(last_tokens):
            raise ValueError("slot_batch and last_tokens length mismatch")
        if not 0 < n <= self.batch_size:
            raise ValueError(f"batch of {n} rows for a graph of {self.batch_size}")
        bank = self.runner.bank
        wkv = [int(s["wkv"]) for s in slot_batch]
        shift = [int(s["shift"]) for s in slot_batch]
        # range and duplicate checks on the host (the padding rows are slot 0)
        ops._validate_ids(torch.tensor(wkv), bank.num_slots + 1)
        ops._validate_ids(torch.tensor(shift), bank.num_slots + 1)
        h = self._host
        if self._staged is not None:
            self._staged.synchronize()  # the previous call's copy has read h
        h.zero_()
        h[0, :n] = torch.tensor(last_tokens)
        h[1, :n] = torch.tensor(wkv)
        h[2, :n] = torch.tensor(shift)
        dev = bank.device
        staged = h.to(dev, non_blocking=True)
        self.tokens.copy_(staged[0].unsqueeze(1))
        self.wkv_ids.copy_(staged[1])
        self.shift_ids.copy_(staged[2])
        self._staged = torch.cuda.Event()
        self._staged.record(torch.cuda.current_stream(dev))
        self.graph.replay()
        return self.logits[:n, -1].float()
