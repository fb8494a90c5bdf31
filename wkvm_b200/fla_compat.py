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
  disappear. The token-shift family travels through the cache, moved with one
  gather kernel for all layers and one restore per layer, unless the cache is
  built with ``shift_in_bank=True`` (single-token decode with
  ``install(fuse_time_mix=True)``): then each layer gets :class:`SlotShift`
  markers and the token shift + lerp prologue of both the time-mix and the
  channel-mix block reads and writes ``bank.shift[layer, family, slot_ids]``
  in place (ops.wkv7_shift_mix_slots), so nothing is gathered or restored.
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


@dataclass
class SlotShift:
    """One layer's token-shift row family living in the arena:
    bank_shift[layer, family, ids] (family 0: time mix, 1: channel mix)."""

    bank_shift: torch.Tensor
    layer: int
    family: int
    ids: torch.Tensor  # int32, on the bank's device

    @property
    def device(self) -> torch.device:
        return self.bank_shift.device

    @property
    def rows(self) -> torch.Tensor:
        return self.bank_shift[self.layer, self.family]


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


def _fused_time_mix_forward(self, hidden_states, attention_mask=None, past_key_values=None,
                            use_cache=False, output_attentions=False, v_first=None,
                            cu_seqlens=None, **kwargs):
    """RWKV7Attention.forward with the part between the projections and o_proj
    in one kernel (wkv7_timemix_decode_slots), for single-token decode with
    slot-resident state; every other case runs fla's own forward."""
    import fla.layers.rwkv7 as layer
    orig = _orig["forward"]
    B, T, _ = hidden_states.shape
    last = layer.get_layer_cache(self, past_key_values)
    st = last["recurrent_state"] if last is not None else None
    if (not isinstance(st, SlotState) or T != 1 or attention_mask is not None
            or cu_seqlens is not None or self.training or not self.fuse_norm):
        return orig(self, hidden_states, attention_mask, past_key_values, use_cache,
                    output_attentions, v_first, cu_seqlens, **kwargs)
    shift = last["conv_state"]
    if isinstance(shift, SlotShift):  # token shift + lerp on the arena rows, in place
        xr, xw, xk, xv, xa, xg = ops.wkv7_shift_mix_slots(
            hidden_states, (self.x_r, self.x_w, self.x_k, self.x_v, self.x_a, self.x_g),
            shift.rows, shift.ids)
        conv_state = shift
    else:
        delta, conv_state = layer.token_shift(hidden_states, cu_seqlens, output_cache=True,
                                              cache=shift)
        xr, xw, xk, xv, xa, xg = layer.fused_addcmul_rwkv7(hidden_states, delta, self.x_r,
                                                           self.x_w, self.x_k, self.x_v,
                                                           self.x_a, self.x_g)
    r = self.r_proj(xr)
    w_raw = self.w_lora(xw)
    k = self.k_proj(xk)
    v = self.v_proj(xv)
    if self.layer_idx == 0:
        v_first, vf, vr = v, None, None
    else:
        vf, vr = v_first, self.v_lora(xv)
    a_raw = self.a_lora(xa)
    g = self.g_lora(xg)
    o = ops.wkv7_timemix_decode_slots(r, w_raw, k, v, vf, vr, a_raw, g, self.k_k, self.k_a,
                                      self.r_k, self.g_norm.weight, self.g_norm.bias,
                                      self.g_norm.eps, st.bank_wkv, st.layer, st.ids)
    layer.update_layer_cache(self, past_key_values, recurrent_state=st, conv_state=conv_state,
                             offset=T)
    return self.o_proj(o), None, past_key_values, v_first


def _ffn_forward(self, x, attention_mask=None, state=None, cu_seqlens=None, **kwargs):
    """RWKV7FeedForward.forward with the token shift + lerp on the arena rows
    when the cache carries a SlotShift (single-token decode); otherwise
    fla's own forward."""
    st = None
    if state is not None and len(state) > self.layer_idx:
        st = state[self.layer_idx].get("ffn_state")
    if (not isinstance(st, SlotShift) or x.shape[1] != 1 or attention_mask is not None
            or cu_seqlens is not None or self.training):
        return _orig["ffn_forward"](self, x, attention_mask, state, cu_seqlens, **kwargs)
    (xk,) = ops.wkv7_shift_mix_slots(x, (self.x_k,), st.rows, st.ids)
    return self.value(self.act_fn(self.key(xk))), state


def install(fuse_time_mix: bool = False) -> None:
    """Points fla's RWKV7Attention at wkvm_b200's WKV ops (idempotent). With
    ``fuse_time_mix`` single-token decode with slot-resident state also runs
    the gates, norms and output correction inside the decode kernel, and the
    token shift + lerp of both blocks on the arena rows when the cache was
    built with ``shift_in_bank=True``."""
    import fla.layers.rwkv7 as layer
    import fla.models.rwkv7.modeling_rwkv7 as modeling
    if not _orig:
        _orig["fused_mul_recurrent_rwkv7"] = layer.fused_mul_recurrent_rwkv7
        _orig["chunk_rwkv7"] = layer.chunk_rwkv7
        _orig["forward"] = layer.RWKV7Attention.forward
        _orig["ffn_forward"] = modeling.RWKV7FeedForward.forward
    layer.fused_mul_recurrent_rwkv7 = fused_mul_recurrent_rwkv7
    layer.chunk_rwkv7 = chunk_rwkv7
    layer.RWKV7Attention.forward = (_fused_time_mix_forward if fuse_time_mix
                                    else _orig["forward"])
    modeling.RWKV7FeedForward.forward = (_ffn_forward if fuse_time_mix
                                         else _orig["ffn_forward"])


def uninstall() -> None:
    """Restores fla's own ops and forward."""
    import fla.layers.rwkv7 as layer
    import fla.models.rwkv7.modeling_rwkv7 as modeling
    for name, fn in _orig.items():
        if name == "forward":
            layer.RWKV7Attention.forward = fn
        elif name == "ffn_forward":
            modeling.RWKV7FeedForward.forward = fn
        else:
            setattr(layer, name, fn)
    _orig.clear()


class SlotCacheHandle:
    """An fla Cache whose wkv entries are SlotStates, plus the token-shift
    rows gathered for this batch; :meth:`commit` writes the updated
    token-shift rows back to the bank."""

    def __init__(self, bank, slot_ids, shift_in_bank: bool = False, shift_ids=None):
        from fla.models.utils import Cache

        self.bank = bank
        dev = bank.device
        self.ids = ops.slot_ids_tensor(slot_ids, bank.num_slots + 1, dev)
        # the token-shift family's own slot ids (wkvm's slot dicts name one id
        # per family); the wkv ids when not given
        self.shift_ids = (self.ids if shift_ids is None
                          else ops.slot_ids_tensor(shift_ids, bank.num_slots + 1, dev))
        if self.shift_ids.numel() != self.ids.numel():
            raise ValueError("wkv and shift slot id lists differ in length")
        L = bank.layout.n_layer
        self.shift_in_bank = shift_in_bank
        if shift_in_bank:  # the fused prologues read and write bank.shift in place
            self.shift = None
            self.cache = Cache()
            for i in range(L):
                self.cache.update(recurrent_state=SlotState(bank.wkv, i, self.ids),
                                  conv_state=SlotShift(bank.shift, i, 0, self.shift_ids),
                                  ffn_state=SlotShift(bank.shift, i, 1, self.shift_ids),
                                  layer_idx=i, offset=0)
            return
        # [L, 2, n, D]: one kernel, and every (layer, family) view is contiguous
        self.shift = ops.slot_gather_outer_major(bank.shift, 2, self.shift_ids)
        self.cache = Cache()
        for i in range(L):
            self.cache.update(recurrent_state=SlotState(bank.wkv, i, self.ids),
                              conv_state=self.shift[i, 0], ffn_state=self.shift[i, 1],
                              layer_idx=i, offset=0)

    def commit(self) -> None:
        """Writes each layer's new token-shift rows back to the bank (nothing
        to do when they were updated in place)."""
        if self.shift_in_bank:
            return
        L = self.bank.layout.n_layer
        for i in range(L):
            st = self.cache[i]
            for j, key in ((0, "conv_state"), (1, "ffn_state")):
                x = st[key]
                if x.data_ptr() == self.shift[i, j].data_ptr():
                    x = self.shift[i, j]
                ops.slot_restore(self.bank.shift[i, j], 0, self.shift_ids,
                                 x.reshape(self.ids.numel(), -1).to(self.bank.shift.dtype))


def slot_cache(bank, slot_ids, shift_in_bank: bool = False, shift_ids=None) -> SlotCacheHandle:
    """fla Cache over the arena rows of ``slot_ids``; see the module docstring
    for ``shift_in_bank`` (single-token decode with install(fuse_time_mix=True)
    only: fla's own token shift cannot read a SlotShift and raises).
    ``shift_ids`` names the token-shift family's rows when they differ."""
    return SlotCacheHandle(bank, slot_ids, shift_in_bank, shift_ids)


def installed() -> bool:
    """True while fla's RWKV7Attention runs wkvm_b200's ops (after install())."""
    if not _orig:
        return False
    import fla.layers.rwkv7 as layer
    return layer.fused_mul_recurrent_rwkv7 is fused_mul_recurrent_rwkv7


def fused_installed() -> bool:
    """True after install(fuse_time_mix=True)."""
    if not installed():
        return False
    import fla.layers.rwkv7 as layer
    return layer.RWKV7Attention.forward is _fused_time_mix_forward
