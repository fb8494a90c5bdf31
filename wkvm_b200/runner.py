"""Host driver for prefill and batched decode against arena slots, with the
interface of wkvm's RWKV7Runner (wkvm/runner/runner.py:21-89): the same
constructor, method names, arguments, return values and errors, so a caller
of wkvm's runner can switch to this one.

What changes is where the state lives during the forward. wkvm gathers each
layer's state out of the bank into an fla Cache, runs the model, and
scatters it back. Here, with ``fla_compat.install()`` in effect, the bank's
``gather_cache`` hands the model slot-resident states that the installed ops
update in place (``RWKV7StateBank.gather_cache``), so the per-call copies of
the wkv family disappear. Without the install, the bank returns plain
copies and fla's own ops run, exactly wkvm's flow.

Single-token decode can also keep the token-shift family in the bank
(``shift_in_bank``, needs ``install(fuse_time_mix=True)``): then nothing at
all is gathered or scattered.
"""

from __future__ import annotations

import torch

from . import fla_compat


class RWKV7Runner:
    """Prefill / decode over slots of an :class:`~wkvm_b200.state.RWKV7StateBank`."""

    def __init__(self, model, bank, prefill_chunk: int = 512) -> None:
        """``prefill_chunk``: tokens per model forward during prefill. Keep it a
        multiple of the chunk kernel's 64 so re-entry points fall on chunk
        boundaries (wkvm's default and advice, runner.py:30-36)."""
        if prefill_chunk < 1:
            raise ValueError("prefill_chunk must be >= 1")
        self.model = model
        self.bank = bank
        self.prefill_chunk = prefill_chunk
        self.device = bank.device

    @torch.inference_mode()
    def prefill(self, token_ids: list[int], slots: dict[str, int]) -> torch.Tensor:
        """Runs a prompt through the model in ``prefill_chunk``-token pieces,
        leaving its final state in ``slots``; returns the last position's
        logits as fp32 ``[vocab]``."""
        if not token_ids:
            raise ValueError("empty prompt")
        ids = torch.tensor(token_ids, dtype=torch.long, device=self.device)
        logits = None
        for start in range(0, len(token_ids), self.prefill_chunk):
            piece = ids[start:start + self.prefill_chunk].unsqueeze(0)
            cache = self.bank.gather_cache([slots])
            out = self.model(input_ids=piece, past_key_values=cache, use_cache=True,
                             logits_to_keep=1)
            self.bank.scatter_cache([slots], cache)
            logits = out.logits
        return logits[0, -1].float()

    @torch.inference_mode()
    def decode_step(self, slot_batch: list[dict[str, int]], last_tokens: list[int]) -> torch.Tensor:
        """Advances every slot of the batch by its last token; returns the
        next-token logits as fp32 ``[batch, vocab]``."""
        if len(slot_batch) != len(last_tokens):
            raise ValueError("slot_batch and last_tokens length mismatch")
        ids = torch.tensor(last_tokens, dtype=torch.long, device=self.device)
        if fla_compat.fused_installed():
            # shift family in the bank too: the fused prologues read and
            # write it in place, so there is nothing to commit afterwards
            h = fla_compat.slot_cache(self.bank, [int(s["wkv"]) for s in slot_batch],
                                      shift_in_bank=True,
                                      shift_ids=[int(s["shift"]) for s in slot_batch])
            out = self.model(input_ids=ids.unsqueeze(1), past_key_values=h.cache,
                             use_cache=True, logits_to_keep=1)
            h.commit()
            return out.logits[:, -1].float()
        cache = self.bank.gather_cache(slot_batch)
        out = self.model(input_ids=ids.unsqueeze(1), past_key_values=cache, use_cache=True,
                         logits_to_keep=1)
        self.bank.scatter_cache(slot_batch, cache)
        return out.logits[:, -1].float()
