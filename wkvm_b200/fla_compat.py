"""Running fla's RWKV-7 model (the model wkvm serves) on wkvm_b200.

Two levels of drop-in:

* :func:`install` swaps the two WKV ops fla's RWKV7Attention imports
  (fla/layers/rwkv7.py:23, called at :305-334) for wkvm_b200's. States passed
  as tensors behave exactly as before (fla signature, new final state).
* :class:`SlotState` / :func:`slot_cache` keep the recurrent state in the
  arena: a cache built with ``slot_cache(bank, slot_ids)`` hands each layer a
  SlotState instead of a gathered copy; the installed ops see it and update
  ``bank.wkv[layer, slot_ids]`` in place, so wkvm's gather_cache /
  scatter_cache copies of the wkv family (wkvm/runner/state.py:63-97)
  disappear. The token-shift family still travels through the cache, moved
  with one slot-snapshot kernel for all layers and one restore.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from . import prefill as _prefill
from . import _lib

_orig: dict = {}


@dataclass
class SlotState:
    """One layer's WKV state living in the arena: bank_wkv[layer, ids]."""

    bank_wkv: torch.Tensor
    layer: int
    ids: torch.Tensor  # int32, on the bank's device

    @property
    def device(self) -> torch.device:
        return self.bank_wkv.device


def fused_mul_recurrent_rwkv7(r, w, k, v, kk, a, scale: float = 1.0, initial_state=None,
                              output_final_state: bool = False, reverse: bool = False,
                              cu_seqlens=None, **kwargs):
    """fla signature; a SlotState initial state is updated in place."""
    if isinstance(initial_state, SlotState):
        if scale != 1.0 or reverse or cu_seqlens is not None:
            raise NotImplementedError("slot-resident decode takes scale=1, forward, no varlen")
        o = ops.wkv7_decode_slots(r, w, k, v, kk, a, initial_state.bank_wkv, initial_state.layer,
                                  initial_state.ids)
        return o, initial_state
    return ops.fused_mul_recurrent_rwkv7(r, w, k, v, kk, a, scale=scale,
                                         initial_state=initial_state,
                                         output_final_state=output_final_state, reverse=reverse,
                                         cu_seqlens=cu_seqlens, **kwargs)


def chunk_rwkv7(r, w, k, v, a, b, scale: float = 1.0, initial_state=None,
                output_final_state: bool = False, cu_seqlens=None, **kwargs):
    """fla signature; a SlotState initial state is read and written in place."""
    if isinstance(initial_state, SlotState):
        st = initial_state
        layer_t = ops._bank_layer(st.bank_wkv, st.layer)
        _ops = ops
        (r, w, k, v, a, b), dt = _ops._acts(r, w, k, v, a, b)
        B, T, H, K = r.shape
        nseq = B if cu_seqlens is None else len(cu_seqlens) - 1
        cu = _ops._cu(cu_seqlens, r.device)
        o = torch.empty_like(v)
        with torch.cuda.device(r.device):
            _lib.call("wkvm_dplr_prefill_slots", _ops._ptr(r), _ops._ptr(w), _ops._ptr(k),
                      _ops._ptr(v), _ops._ptr(a), _ops._ptr(b), _ops._ptr(o),
                      _ops._ptr(layer_t), layer_t.shape[0], _ops._ptr(st.ids), _ops._ptr(cu),
                      nseq, T, H, K, v.shape[-1], float(scale), dt,
                      _ops._ptr(_ops.status_word(r.device)), _ops._stream(r.device))
        return o, st
    return _prefill.chunk_dplr(r, w, k, v, a, b, scale, initial_state, output_final_state,
                               cu_seqlens)


def install() -> None:
    """Points fla's RWKV7Attention at wkvm_b200's WKV ops (idempotent)."""
    import fla.layers.rwkv7 as layer
    if not _orig:
        _orig["fused_mul_recurrent_rwkv7"] = layer.fused_mul_recurrent_rwkv7
        _orig["chunk_rwkv7"] = layer.chunk_rwkv7
    layer.fused_mul_recurrent_rwkv7 = fused_mul_recurrent_rwkv7
    layer.chunk_rwkv7 = chunk_rwkv7


def uninstall() -> None:
    """Restores fla's own ops."""
    import fla.layers.rwkv7 as layer
    for name, fn in _orig.items():
        setattr(layer, name, fn)
    _orig.clear()


class SlotCacheHandle:
    """An fla Cache whose wkv entries are SlotStates, plus the token-shift
    rows gathered for this batch; :meth:`commit` writes the updated
    token-shift rows back to the bank."""

    def __init__(self, bank, slot_ids):
        from fla.models.utils import Cache

        self.bank = bank
        dev = bank.device
        self.ids = ops.slot_ids_tensor(slot_ids, bank.num_slots + 1, dev)
        L = bank.layout.n_layer
        # [L, 2, n, D]: one kernel, and every (layer, family) view is contiguous
        self.shift = ops.slot_gather_outer_major(bank.shift, 2, self.ids)
        self.cache = Cache()
        for i in range(L):
            self.cache.update(recurrent_state=SlotState(bank.wkv, i, self.ids),
                              conv_state=self.shift[i, 0], ffn_state=self.shift[i, 1],
                              layer_idx=i, offset=0)

    def commit(self) -> None:
        """Writes each layer's new token-shift rows back to the bank."""
        L = self.bank.layout.n_layer
        for i in range(L):
            st = self.cache[i]
            for j, key in ((0, "conv_state"), (1, "ffn_state")):
                x = st[key]
                if x.data_ptr() == self.shift[i, j].data_ptr():
                    x = self.shift[i, j]
                ops.slot_restore(self.bank.shift[i, j], 0, self.ids,
                                 x.reshape(self.ids.numel(), -1).to(self.bank.shift.dtype))


def slot_cache(bank, slot_ids) -> SlotCacheHandle:
    return SlotCacheHandle(bank, slot_ids)
