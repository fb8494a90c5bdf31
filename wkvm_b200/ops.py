"""Operators with fla's signatures, backed by the sm_100a kernels of
libwkvm_b200.so, plus slot-native variants that read and write wkvm's state
arena in place.

Drop-in surface (fla 0.5.1, the package wkvm's RWKV-7 model calls):
  fused_mul_recurrent_rwkv7   fla/ops/rwkv7/fused_recurrent.py:240
  fused_recurrent_rwkv7       fla/ops/rwkv7/fused_recurrent.py:183
  chunk_rwkv7                 fla/ops/rwkv7/chunk.py:13
  fused_recurrent_gated_delta_rule  fla/ops/gated_delta_rule/fused_recurrent.py:291
  chunk_gated_delta_rule      fla/ops/gated_delta_rule/chunk.py:365
The call sites are fla/layers/rwkv7.py:305-334 (RWKV-7 time-mix) and
wkvm/runner/runner.py:42,66 (through the model forward).

Argument meaning and error behaviour follow fla: tensors are [B, T, H, D]
(head_first raises DeprecationWarning), varlen needs B == 1 (ValueError),
the initial-state count must match the sequence count (ValueError), the
output has v's dtype and the final state is fp32 [N, H, K, V] or None.

Every op runs on CUDA tensors only and enqueues on the current stream;
nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_status: dict[int, torch.Tensor] = {}


# ---------------------------------------------------------------------------
# plumbing
# ---------------------------------------------------------------------------

def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def status_word(device: torch.device | int | str | None = None) -> torch.Tensor:
    """The per-device int32 word kernels report device-side errors into
    (0 = ok). It is never cleared implicitly; see :func:`check_device_status`."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        # a normal tensor even when first requested under inference_mode, so
        # it can be reset anywhere
        with torch.inference_mode(False):
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_device_status(device=None, reset: bool = True) -> None:
    """Synchronises with the device's status word and raises the first
    recorded device-side error (e.g. an out-of-range slot id)."""
    t = status_word(device)
    code = int(t.item())
    if reset:
        t.zero_()
    if code != 0:
        raise _lib.WkvmError("device kernel", code)


_debug = False


def set_debug_checks(enable: bool) -> bool:
    """Debug mode (off by default; returns the previous setting). While on,
    every op synchronises after its launch and raises the first device-side
    error the kernels recorded (check_device_status on every device used so
    far), and slot ids given as CUDA tensors are checked for range and
    duplicates on the host before the launch. Not for use inside CUDA graph
    capture: it synchronises."""
    global _debug
    prev = _debug
    _debug = bool(enable)
    _lib.post_call = _check_after_call if _debug else None
    return prev


def _check_after_call(name: str) -> None:
    for idx in list(_status):
        code = int(_status[idx].item())
        if code != 0:
            _status[idx].zero_()
            raise _lib.WkvmError(f"{name} (device {idx})", code)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("wkvm_b200 ops take CUDA tensors only (no CPU path)")


def _acts(*ts):
    """Contiguous activations in one dtype; mixed dtypes are promoted to fp32
    (lossless), matching fla's per-pointer dtype loads."""
    dt = ts[0].dtype
    if any(t.dtype != dt for t in ts) or dt not in _DTYPES:
        ts = tuple(t.float() for t in ts)
        dt = torch.float32
    return tuple(t.contiguous() for t in ts), _DTYPES[dt]


GATES_F32 = 0x100  # WKVM_GATES_F32: g and beta fp32, q/k/v/o in the low byte's dtype


def _gdn_acts(q, k, v, g, beta):
    """Activations of the gated delta rule. q, k, v sharing a dtype keep it;
    gates of another dtype are widened to fp32 (lossless) and flagged, so a
    16-bit q/k/v with fp32 g/beta (what fla's GDN layers pass) stays on the
    16-bit paths. q, k, v of mixed dtypes are all promoted to fp32."""
    dt = q.dtype
    if k.dtype != dt or v.dtype != dt or dt not in _DTYPES:
        return _acts(q, k, v, g, beta)
    if g.dtype == dt and beta.dtype == dt:
        return tuple(t.contiguous() for t in (q, k, v, g, beta)), _DTYPES[dt]
    gates = tuple(t.to(torch.float32).contiguous() for t in (g, beta))
    return (q.contiguous(), k.contiguous(), v.contiguous(), *gates), _DTYPES[dt] | GATES_F32


def _state(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    if t.dtype != torch.float32:
        t = t.float()
    return t.contiguous()


def _check_varlen(x: torch.Tensor, initial_state, cu_seqlens, name0="r"):
    if cu_seqlens is not None:
        if x.shape[0] != 1:
            raise ValueError(
                f"The batch size is expected to be 1 rather than {x.shape[0]} when using "
                f"`cu_seqlens`. Please flatten variable-length inputs before processing.")
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(
                "The number of initial states is expected to be equal to the number of input "
                f"sequences, i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}.")


def _cu(cu_seqlens, device):
    if cu_seqlens is None:
        return None
    return cu_seqlens.to(device=device, dtype=torch.int64).contiguous()


def _no_head_first(kwargs):
    if "head_first" in kwargs:
        raise DeprecationWarning(
            "head_first has been removed. Inputs must be in `[B, T, H, ...]` format.")


# ---------------------------------------------------------------------------
# RWKV-7
# ---------------------------------------------------------------------------

def _rwkv7_recurrent(entry, r, w, k, v, p5, p6, scale, initial_state, output_final_state,
                     cu_seqlens):
    _require_cuda(r, w, k, v, p5, p6, initial_state)
    (r, w, k, v, p5, p6), dt = _acts(r, w, k, v, p5, p6)
    B, T, H, K = r.shape
    V = v.shape[-1]
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    cu = _cu(cu_seqlens, r.device)
    h0 = _state(initial_state)
    o = torch.empty_like(v)
    ht = torch.empty(N, H, K, V, dtype=torch.float32, device=r.device) if output_final_state else None
    if ht is not None and h0 is None:
        pass  # the kernel starts from zeros when h0 is NULL
    with torch.cuda.device(r.device):
        _lib.call(entry, _ptr(r), _ptr(w), _ptr(k), _ptr(v), _ptr(p5), _ptr(p6), _ptr(o),
                  _ptr(h0), _ptr(ht), _ptr(cu), N if cu is not None else B,
                  T if cu is None else r.shape[1], H, K, V, float(scale), dt,
                  _ptr(status_word(r.device)), _stream(r.device))
    return o, ht


def fused_mul_recurrent_rwkv7(r, w, k, v, kk, a, scale: float = 1.0, initial_state=None,
                              output_final_state: bool = False, reverse: bool = False,
                              cu_seqlens=None, **kwargs):
    """fla fused_mul_recurrent_rwkv7 (fla/ops/rwkv7/fused_recurrent.py:240):
    RWKV-7 recurrence with a = -kk, b = kk * a. Returns (o, final_state)."""
    _no_head_first(kwargs)
    _check_varlen(r, initial_state, cu_seqlens)
    if reverse:
        raise NotImplementedError("reverse=True is a training-only mode not on the wkvm path")
    if scale is None:
        scale = r.shape[-1] ** -0.5
    return _rwkv7_recurrent("wkvm_fused_mul_recurrent_rwkv7", r, w, k, v, kk, a, scale,
                            initial_state, output_final_state, cu_seqlens)


def fused_recurrent_rwkv7(r, w, k, v, a, b, scale=None, initial_state=None,
                          output_final_state: bool = True, cu_seqlens=None, **kwargs):
    """fla fused_recurrent_rwkv7 (fla/ops/rwkv7/fused_recurrent.py:183): the
    general DPLR recurrence with explicit a, b; scale defaults to K^-0.5."""
    _no_head_first(kwargs)
    _check_varlen(r, initial_state, cu_seqlens)
    if scale is None:
        scale = r.shape[-1] ** -0.5
    return _rwkv7_recurrent("wkvm_fused_recurrent_dplr", r, w, k, v, a, b, scale,
                            initial_state, output_final_state, cu_seqlens)


def chunk_rwkv7(r, w, k, v, a, b, scale: float = 1.0, initial_state=None,
                output_final_state: bool = False, cu_seqlens=None, cu_seqlens_cpu=None,
                safe_gate: bool = False, chunk_size: int | None = None, **kwargs):
    """fla chunk_rwkv7 (fla/ops/rwkv7/chunk.py:13): chunked DPLR prefill."""
    _no_head_first(kwargs)
    _check_varlen(r, initial_state, cu_seqlens)
    if scale is None:
        scale = r.shape[-1] ** -0.5
    from . import prefill
    return prefill.chunk_dplr(r, w, k, v, a, b, scale, initial_state, output_final_state,
                              cu_seqlens)


# ---------------------------------------------------------------------------
# Gated delta rule
# ---------------------------------------------------------------------------

def _gdn_common(q, k, v, g, beta, gk, gv, use_gate_in_kernel, transpose_state_layout):
    if gk is not None or gv is not None:
        raise NotImplementedError("per-key / per-value decays (gk, gv) are not on the wkvm path")
    if use_gate_in_kernel:
        raise NotImplementedError("use_gate_in_kernel is not supported")
    if transpose_state_layout:
        raise NotImplementedError("transpose_state_layout is not supported")
    if q.shape[2] != k.shape[2]:
        raise ValueError(
            f"q and k must have the same number of heads, but got q.shape[2]={q.shape[2]} "
            f"and k.shape[2]={k.shape[2]}")
    HV = v.shape[2]
    if HV % q.shape[2] != 0:
        raise ValueError("the number of value heads must be divisible by the number of q/k heads")
    if g is None:
        g = torch.zeros(v.shape[:3], dtype=v.dtype, device=v.device)
    if beta is None:
        beta = torch.ones(v.shape[:3], dtype=v.dtype, device=v.device)
    if beta.dim() != 3:
        raise NotImplementedError("per-value beta is not supported; beta must be [B, T, HV]")
    return g, beta


def fused_recurrent_gated_delta_rule(q, k, v, g=None, gk=None, gv=None, beta=None, scale=None,
                                     initial_state=None, output_final_state: bool = False,
                                     use_qk_l2norm_in_kernel: bool = False,
                                     use_gate_in_kernel: bool = False, A_log=None, dt_bias=None,
                                     cu_seqlens=None, transpose_state_layout: bool = False):
    """fla fused_recurrent_gated_delta_rule
    (fla/ops/gated_delta_rule/fused_recurrent.py:291). Returns (o, final_state)."""
    _check_varlen(q, initial_state, cu_seqlens)
    g, beta = _gdn_common(q, k, v, g, beta, gk, gv, use_gate_in_kernel, transpose_state_layout)
    if scale is None:
        scale = k.shape[-1] ** -0.5
    _require_cuda(q, k, v, g, beta, initial_state)
    (q, k, v, g, beta), dt = _gdn_acts(q, k, v, g, beta)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    cu = _cu(cu_seqlens, q.device)
    h0 = _state(initial_state)
    o = torch.empty_like(v)
    ht = torch.empty(N, HV, K, V, dtype=torch.float32, device=q.device) if output_final_state else None
    with torch.cuda.device(q.device):
        _lib.call("wkvm_fused_recurrent_gated_delta_rule", _ptr(q), _ptr(k), _ptr(v), _ptr(g),
                  _ptr(beta), _ptr(o), _ptr(h0), _ptr(ht), _ptr(cu),
                  N if cu is not None else B, T, H, HV, K, V, float(scale),
                  int(bool(use_qk_l2norm_in_kernel)), dt, _ptr(status_word(q.device)),
                  _stream(q.device))
    return o, ht


def chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None,
                           output_final_state: bool = False,
                           use_qk_l2norm_in_kernel: bool = False, cu_seqlens=None,
                           cu_seqlens_cpu=None, cp_context=None,
                           transpose_state_layout: bool = False, **kwargs):
    """fla chunk_gated_delta_rule (fla/ops/gated_delta_rule/chunk.py:365)."""
    if cp_context is not None:
        raise NotImplementedError("context parallelism is not on the wkvm path")
    _check_varlen(q, initial_state, cu_seqlens)
    g, beta = _gdn_common(q, k, v, g, beta, None, None, kwargs.get("use_gate_in_kernel", False),
                          transpose_state_layout)
    if scale is None:
        scale = k.shape[-1] ** -0.5
    from . import prefill
    return prefill.chunk_gdn(q, k, v, g, beta, scale, initial_state, output_final_state,
                             use_qk_l2norm_in_kernel, cu_seqlens)


# ---------------------------------------------------------------------------
# Slot-native ops (state read and written in place in the arena)
# ---------------------------------------------------------------------------

def slot_ids_tensor(slot_ids, num_slots: int, device, validate: bool = True) -> torch.Tensor:
    """int32 CUDA tensor of slot ids. Python lists and CPU tensors are checked
    on the host (range [0, num_slots), no duplicates) before the copy; CUDA
    tensors are trusted (kernels still skip and report out-of-range ids)."""
    if isinstance(slot_ids, torch.Tensor) and slot_ids.is_cuda:
        if slot_ids.dtype != torch.int32:
            slot_ids = slot_ids.to(torch.int32)
        if not (_debug and validate):
            return slot_ids.contiguous()
        dev_ids = slot_ids.contiguous()
        ids = dev_ids.reshape(-1).to("cpu", torch.int64)
        _validate_ids(ids, num_slots)
        return dev_ids
    ids = torch.as_tensor(slot_ids, dtype=torch.int64).reshape(-1)
    if validate:
        _validate_ids(ids, num_slots)
    return ids.to(torch.int32).to(device, non_blocking=True)


def _validate_ids(ids: torch.Tensor, num_slots: int) -> None:
    if ids.numel():
        lo, hi = int(ids.min()), int(ids.max())
        if lo < 0 or hi >= num_slots:
            raise _lib.WkvmError("slot id check", -4)
        if torch.unique(ids).numel() != ids.numel():
            raise _lib.WkvmError("slot id check", -5)


def _bank_layer(bank: torch.Tensor, layer: int) -> torch.Tensor:
    if bank.dtype != torch.float32 or not bank.is_contiguous():
        raise ValueError("the wkv bank must be a contiguous fp32 tensor [L, S+1, H, K, V]")
    if not 0 <= layer < bank.shape[0]:
        raise IndexError(f"layer {layer} out of range [0, {bank.shape[0]})")
    return bank[layer]


def set_decode_overlap(enable: bool) -> bool:
    """Opt-in overlap of consecutive wkv7_decode_slots launches (programmatic
    dependent launch). While enabled, the kernel launched right before a
    decode call on the same stream must not write that call's slot ids or
    those slots' state in that layer — true for a loop over layers. Returns
    the previous setting."""
    return bool(_lib.load().wkvm_set_decode_overlap(int(bool(enable))))


def wkv7_decode_slots(r, w, k, v, kk, a, bank_wkv: torch.Tensor, layer: int, slot_ids,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """RWKV-7 decode of B rows whose states live in bank_wkv[layer, slot_ids]
    ([L, S+1, H, K, V] fp32, updated in place); replaces wkvm's
    gather_cache -> fused_mul_recurrent_rwkv7 -> scatter_cache for one layer
    (wkvm/runner/state.py:63-97). Inputs [B, T, H, K] (T tokens applied in
    order); returns o [B, T, H, V]."""
    _require_cuda(r, w, k, v, kk, a, bank_wkv)
    layer_t = _bank_layer(bank_wkv, layer)
    (r, w, k, v, kk, a), dt = _acts(r, w, k, v, kk, a)
    B, T, H, K = r.shape
    V = v.shape[-1]
    if tuple(layer_t.shape[1:]) != (H, K, V):
        raise ValueError(f"bank layer shape {tuple(layer_t.shape)} does not match H,K,V={H},{K},{V}")
    ids = slot_ids_tensor(slot_ids, layer_t.shape[0], r.device)
    if ids.numel() != B:
        raise ValueError(f"{ids.numel()} slot ids for a batch of {B}")
    o = torch.empty_like(v) if out is None else out
    with torch.cuda.device(r.device):
        _lib.call("wkvm_wkv7_decode_slots", _ptr(r), _ptr(w), _ptr(k), _ptr(v), _ptr(kk),
                  _ptr(a), _ptr(o), _ptr(layer_t), layer_t.shape[0], _ptr(ids), B, T, H, K, V,
                  dt, _ptr(status_word(r.device)), _stream(r.device))
    return o


def gdn_decode_slots(q, k, v, g, beta, bank: torch.Tensor, layer: int, slot_ids, scale=None,
                     use_qk_l2norm_in_kernel: bool = False,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Gated-delta-rule decode with states in bank[layer, slot_ids]
    ([L, S+1, HV, K, V] fp32, in place). Returns o [B, T, HV, V]."""
    _require_cuda(q, k, v, g, beta, bank)
    layer_t = _bank_layer(bank, layer)
    (q, k, v, g, beta), dt = _gdn_acts(q, k, v, g, beta)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if tuple(layer_t.shape[1:]) != (HV, K, V):
        raise ValueError("bank layer shape does not match HV, K, V")
    if scale is None:
        scale = K ** -0.5
    ids = slot_ids_tensor(slot_ids, layer_t.shape[0], q.device)
    if ids.numel() != B:
        raise ValueError(f"{ids.numel()} slot ids for a batch of {B}")
    o = torch.empty_like(v) if out is None else out
    with torch.cuda.device(q.device):
        _lib.call("wkvm_gdn_decode_slots", _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                  _ptr(o), _ptr(layer_t), layer_t.shape[0], _ptr(ids), B, T, H, HV, K, V,
                  float(scale), int(bool(use_qk_l2norm_in_kernel)), dt,
                  _ptr(status_word(q.device)), _stream(q.device))
    return o


def wkv7_prefill_slots(r, w, k, v, kk, a, bank_wkv: torch.Tensor, layer: int, slot_ids,
                       cu_seqlens=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Chunked RWKV-7 prefill whose initial state is read from, and final
    state written to, bank_wkv[layer, slot_ids] (replaces wkvm's
    RWKV7Runner.prefill gather -> chunk_rwkv7 -> scatter, runner.py:52-62)."""
    from . import prefill
    return prefill.wkv7_prefill_slots(r, w, k, v, kk, a, bank_wkv, layer, slot_ids, cu_seqlens,
                                      out=out)


def gdn_prefill_slots(q, k, v, g, beta, bank, layer: int, slot_ids, scale=None,
                      use_qk_l2norm_in_kernel: bool = False, cu_seqlens=None) -> torch.Tensor:
    """Chunked GDN prefill with initial/final state in bank[layer, slot_ids]."""
    from . import prefill
    if scale is None:
        scale = k.shape[-1] ** -0.5
    return prefill.gdn_prefill_slots(q, k, v, g, beta, bank, layer, slot_ids, scale,
                                     use_qk_l2norm_in_kernel, cu_seqlens)


def _family_geometry(t: torch.Tensor, slot_dim: int):
    """(outer, outer_stride, slot_stride, row_bytes, num_slots) in bytes for a
    contiguous family tensor whose slot axis is ``slot_dim``."""
    if not t.is_contiguous():
        raise ValueError("state family tensors must be contiguous")
    es = t.element_size()
    outer = 1
    for s in t.shape[:slot_dim]:
        outer *= s
    num_slots = t.shape[slot_dim]
    row = es
    for s in t.shape[slot_dim + 1:]:
        row *= s
    return outer, num_slots * row, row, row, num_slots


def slot_copy(family: torch.Tensor, slot_dim: int, src_ids, dst_ids) -> None:
    """Bitwise fork: family[..., dst, ...] <- family[..., src, ...] for every
    outer index (e.g. bank.wkv with slot_dim=1, bank.shift with slot_dim=2)."""
    outer, ostr, sstr, row, ns = _family_geometry(family, slot_dim)
    s = slot_ids_tensor(src_ids, ns, family.device)
    d = slot_ids_tensor(dst_ids, ns, family.device)
    if s.numel() != d.numel():
        raise ValueError("src_ids and dst_ids differ in length")
    if not isinstance(src_ids, torch.Tensor) or not src_ids.is_cuda:
        if set(torch.as_tensor(src_ids).tolist()) & set(torch.as_tensor(dst_ids).tolist()):
            raise ValueError("fork source and destination slots overlap")
    with torch.cuda.device(family.device):
        _lib.call("wkvm_slot_copy", _ptr(family), outer, ostr, sstr, row, ns, _ptr(s), _ptr(d),
                  s.numel(), _ptr(status_word(family.device)), _stream(family.device))


def slot_zero(family: torch.Tensor, slot_dim: int, ids) -> None:
    """Zeroes the rows of ``ids`` (wkvm RWKV7StateBank.zero_slots)."""
    outer, ostr, sstr, row, ns = _family_geometry(family, slot_dim)
    i = slot_ids_tensor(ids, ns, family.device)
    with torch.cuda.device(family.device):
        _lib.call("wkvm_slot_zero", _ptr(family), outer, ostr, sstr, row, ns, _ptr(i), i.numel(),
                  _ptr(status_word(family.device)), _stream(family.device))


def slot_snapshot(family: torch.Tensor, slot_dim: int, ids,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Gathers the rows of ``ids`` into ``out`` [n, *outer_shape, *row_shape]
    (pinned host memory by default; device memory also works) with one
    kernel. out[i] has the layout of family[:, ids[i]] — wkvm StateStore.save's
    host copy (wkvm/store.py:130-131). Asynchronous: synchronise before
    reading a host buffer."""
    outer, ostr, sstr, row, ns = _family_geometry(family, slot_dim)
    i = slot_ids_tensor(ids, ns, family.device)
    n = i.numel()
    shape = (n, *family.shape[:slot_dim], *family.shape[slot_dim + 1:])
    if out is None:
        out = torch.empty(shape, dtype=family.dtype, pin_memory=True)
    if tuple(out.shape) != shape or out.dtype != family.dtype or not out.is_contiguous():
        raise ValueError(f"snapshot buffer must be contiguous {shape} {family.dtype}")
    if not out.is_cuda and not out.is_pinned():
        raise ValueError("a host snapshot buffer must be pinned")
    with torch.cuda.device(family.device):
        _lib.call("wkvm_slot_snapshot", _ptr(family), outer, ostr, sstr, row, ns, _ptr(i), n,
                  _ptr(out), _ptr(status_word(family.device)), _stream(family.device))
    return out


def slot_restore(family: torch.Tensor, slot_dim: int, ids, packed: torch.Tensor) -> None:
    """Scatters ``packed`` [n, ...] (pinned host or device) into the rows of
    ``ids`` (wkvm StateStore.load, wkvm/store.py:151-153)."""
    outer, ostr, sstr, row, ns = _family_geometry(family, slot_dim)
    i = slot_ids_tensor(ids, ns, family.device)
    n = i.numel()
    shape = (n, *family.shape[:slot_dim], *family.shape[slot_dim + 1:])
    if tuple(packed.shape) != shape or packed.dtype != family.dtype:
        raise ValueError(f"restore buffer must be {shape} {family.dtype}")
    packed = packed.contiguous()
    if not packed.is_cuda and not packed.is_pinned():
        raise ValueError("a host restore buffer must be pinned")
    with torch.cuda.device(family.device):
        _lib.call("wkvm_slot_restore", _ptr(family), outer, ostr, sstr, row, ns, _ptr(i), n,
                  _ptr(packed), _ptr(status_word(family.device)), _stream(family.device))


def slot_migrate(src: torch.Tensor, dst: torch.Tensor, slot_dim: int, src_ids, dst_ids) -> None:
    """Copies rows src[.., src_ids[i], ..] (this GPU) into dst[.., dst_ids[i], ..]
    on a peer GPU with peer stores over NVLink. Launches on the source GPU's
    current stream; the caller orders the destination's later use (event)."""
    if src.shape != dst.shape and src.shape[:slot_dim] != dst.shape[:slot_dim]:
        raise ValueError("src and dst families differ in layout")
    outer, ostr, sstr, row, ns_src = _family_geometry(src, slot_dim)
    outer_d, ostr_d, sstr_d, row_d, ns_dst = _family_geometry(dst, slot_dim)
    if (outer, sstr, row) != (outer_d, sstr_d, row_d) or ostr != ostr_d:
        raise ValueError("src and dst families must have identical geometry")
    s = slot_ids_tensor(src_ids, ns_src, src.device)
    d = slot_ids_tensor(dst_ids, ns_dst, src.device)
    if s.numel() != d.numel():
        raise ValueError("src_ids and dst_ids differ in length")
    if src.device != dst.device:
        enable_peer_access(src.device, dst.device)
    with torch.cuda.device(src.device):
        _lib.call("wkvm_slot_migrate", _ptr(src), _ptr(dst), outer, ostr, sstr, row, ns_src,
                  ns_dst, _ptr(s), _ptr(d), s.numel(), _ptr(status_word(src.device)),
                  _stream(src.device))


_peer_enabled: set[tuple[int, int]] = set()


def enable_peer_access(src: torch.device, dst: torch.device) -> None:
    """Enables src -> dst peer access once (cudaDeviceEnablePeerAccess)."""
    key = (src.index, dst.index)
    if key in _peer_enabled:
        return
    if not torch.cuda.can_device_access_peer(src.index, dst.index):
        raise RuntimeError(f"GPU {src.index} cannot access GPU {dst.index}'s memory")
    _lib.call("wkvm_enable_peer_access", src.index, dst.index)
    _peer_enabled.add(key)


def slot_affine(family: torch.Tensor, slot_dim: int, dst_ids, a_ids, b_ids, c1: float,
                c2: float = 0.0) -> None:
    """family[.., dst[i], ..] <- c1 * family[.., a[i], ..] + c2 * family[.., b[i], ..]
    (b_ids None: c1 * a), fp32 arithmetic rounded like torch's elementwise ops."""
    outer, ostr, sstr, row, ns = _family_geometry(family, slot_dim)
    d = slot_ids_tensor(dst_ids, ns, family.device)
    a = slot_ids_tensor(a_ids, ns, family.device, validate=False)
    b = None if b_ids is None else slot_ids_tensor(b_ids, ns, family.device, validate=False)
    if a.numel() != d.numel() or (b is not None and b.numel() != d.numel()):
        raise ValueError("id lists differ in length")
    host_lists = [x for x in (dst_ids, a_ids, b_ids)
                  if x is not None and not (isinstance(x, torch.Tensor) and x.is_cuda)]
    if len(host_lists) == (3 if b_ids is not None else 2):
        # pairs run concurrently: a destination may be its own pair's source
        # (in place) but no other pair's
        dl = torch.as_tensor(dst_ids).reshape(-1).tolist()
        srcs = [torch.as_tensor(x).reshape(-1).tolist() for x in (a_ids, b_ids) if x is not None]
        users: dict[int, set[int]] = {}
        for src in srcs:
            for j, sj in enumerate(src):
                users.setdefault(sj, set()).add(j)
        for i, di in enumerate(dl):
            if users.get(di, set()) - {i}:
                raise ValueError(f"slot {di} is a destination and another pair's source")
    dt = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[family.dtype]
    with torch.cuda.device(family.device):
        _lib.call("wkvm_slot_affine", _ptr(family), outer, ostr, sstr, row, ns, _ptr(d),
                  _ptr(a), _ptr(b), d.numel(), float(c1), float(c2), dt,
                  _ptr(status_word(family.device)), _stream(family.device))


def slot_gather_outer_major(family: torch.Tensor, slot_dim: int, ids,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Gathers the rows of ``ids`` into ``out`` [*outer_shape, n, *row_shape]:
    for every outer index a contiguous [n, row] block (one kernel)."""
    outer, ostr, sstr, row, ns = _family_geometry(family, slot_dim)
    i = slot_ids_tensor(ids, ns, family.device)
    n = i.numel()
    shape = (*family.shape[:slot_dim], n, *family.shape[slot_dim + 1:])
    if out is None:
        out = torch.empty(shape, dtype=family.dtype, device=family.device)
    if tuple(out.shape) != shape or not out.is_contiguous():
        raise ValueError(f"gather buffer must be contiguous {shape}")
    with torch.cuda.device(family.device):
        _lib.call("wkvm_slot_gather", _ptr(family), outer, ostr, sstr, row, ns, _ptr(i), n,
                  _ptr(out), n * row, row, _ptr(status_word(family.device)),
                  _stream(family.device))
    return out


def wkv7_shift_mix_slots(x: torch.Tensor, mixes, shift_rows: torch.Tensor, slot_ids,
                         out: torch.Tensor | None = None):
    """Token shift + lerp of RWKV-7 single-token decode with the token-shift
    state in the arena: delta = shift_rows[ids] - x (rounded to x's dtype),
    returns (x + delta * m for m in mixes) as [B, 1, D] views and sets
    shift_rows[ids] = x in place. shift_rows is a contiguous [S+1, D] view
    (bank.shift[layer, family]); mixes are up to six [D]-sized parameters."""
    _require_cuda(x, shift_rows)
    B, D = x.shape[0], x.shape[-1]
    if x.numel() != B * D:
        raise ValueError("x must hold one token per row: [B, 1, D] or [B, D]")
    if shift_rows.dim() != 2 or shift_rows.shape[1] != D or not shift_rows.is_contiguous():
        raise ValueError("shift_rows must be a contiguous [num_slots, D] view")
    if shift_rows.dtype != x.dtype:
        raise ValueError("shift_rows and x must share a dtype")
    if not 0 <= len(mixes) <= 6:
        raise ValueError("at most six mixes")
    x_ = x.contiguous()
    ms = [m if (m.dtype == x.dtype and m.is_contiguous()) else m.to(x.dtype).contiguous()
          for m in mixes]
    if any(m.numel() != D for m in ms):
        raise ValueError("each mix must have D elements")
    ids = slot_ids_tensor(slot_ids, shift_rows.shape[0], x.device)
    if ids.numel() != B:
        raise ValueError(f"{ids.numel()} slot ids for a batch of {B}")
    o = torch.empty(len(ms), B, 1, D, dtype=x.dtype, device=x.device) if out is None else out
    arr = (ctypes.c_void_p * max(len(ms), 1))(*[m.data_ptr() for m in ms])
    with torch.cuda.device(x.device):
        _lib.call("wkvm_wkv7_shift_mix_slots", _ptr(x_), _ptr(o), _ptr(shift_rows),
                  shift_rows.stride(0) * shift_rows.element_size(), shift_rows.shape[0],
                  _ptr(ids), arr, len(ms), B, D, _DTYPES[x.dtype],
                  _ptr(status_word(x.device)), _stream(x.device))
    return tuple(o[i] for i in range(len(ms)))


def wkv7_timemix_decode_slots(r, w_raw, k, v, v_first, v_raw, a_raw, g, k_k, k_a, r_k, gn_w,
                              gn_b, gn_eps: float, bank_wkv: torch.Tensor, layer: int, slot_ids,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused RWKV-7 time-mix decode core (fla RWKV7Attention between its
    projections and o_proj, one token): gates, v lerp, kk norm, k update, the
    in-place WKV step of bank_wkv[layer, slot_ids], GroupNorm, correction and
    output gate. Activations [B, 1, H*64] (or [B, H*64]); v_first / v_raw
    None for layer 0. Returns o [B, 1, H*64] (input to o_proj)."""
    _require_cuda(r, k, v, bank_wkv)
    layer_t = _bank_layer(bank_wkv, layer)
    Hn, K = layer_t.shape[1], layer_t.shape[2]
    B = r.shape[0]
    dt_t = r.dtype
    acts = [r, w_raw, k, v, a_raw, g] + ([v_first, v_raw] if v_first is not None else [])
    acts = [t.to(dt_t).contiguous() for t in acts]
    r_, w_, k_, v_, a_, g_ = acts[:6]
    vf_, vr_ = (acts[6], acts[7]) if v_first is not None else (None, None)
    params = [t.to(dt_t).contiguous() for t in (k_k, k_a, r_k, gn_w, gn_b)]
    ids = slot_ids_tensor(slot_ids, layer_t.shape[0], r.device)
    if ids.numel() != B:
        raise ValueError(f"{ids.numel()} slot ids for a batch of {B}")
    o = torch.empty_like(r_) if out is None else out
    with torch.cuda.device(r.device):
        _lib.call("wkvm_wkv7_timemix_decode_slots", _ptr(r_), _ptr(w_), _ptr(k_), _ptr(v_),
                  _ptr(vf_), _ptr(vr_), _ptr(a_), _ptr(g_), *(_ptr(t) for t in params), _ptr(o),
                  _ptr(layer_t), layer_t.shape[0], _ptr(ids), B, Hn, K, float(gn_eps),
                  _DTYPES[dt_t], _ptr(status_word(r.device)), _stream(r.device))
    return o
