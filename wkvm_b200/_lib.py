"""ctypes binding of libwkvm_b200.so (the C ABI declared in include/wkvm_b200.h).

The library is the only compute path of this package. If it is missing or
fails to load, every op raises: there is no CPU or eager fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libwkvm_b200.so"

P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
F32 = ctypes.c_float

# name -> argtypes, in the order of include/wkvm_b200.h
SIGNATURES: dict[str, list] = {
    "wkvm_version": [],
    "wkvm_strerror": [ctypes.c_int],
    "wkvm_fused_mul_recurrent_rwkv7": [P] * 7 + [P, P, P] + [I32] * 5 + [F32, I32, P, P],
    "wkvm_fused_recurrent_dplr": [P] * 7 + [P, P, P] + [I32] * 5 + [F32, I32, P, P],
    "wkvm_wkv7_decode_slots": [P] * 7 + [P, I64, P] + [I32] * 5 + [I32, P, P],
    "wkvm_wkv7_timemix_decode_slots": [P] * 14 + [P, I64, P, I32, I32, I32, F32, I32, P, P],
    "wkvm_fused_recurrent_gated_delta_rule": [P] * 6 + [P, P, P] + [I32] * 6 + [F32, I32, I32, P, P],
    "wkvm_gdn_decode_slots": [P] * 6 + [P, I64, P] + [I32] * 6 + [F32, I32, I32, P, P],
    "wkvm_slot_copy": [P, I64, I64, I64, I64, I64, P, P, I32, P, P],
    "wkvm_slot_zero": [P, I64, I64, I64, I64, I64, P, I32, P, P],
    "wkvm_slot_snapshot": [P, I64, I64, I64, I64, I64, P, I32, P, P, P],
    "wkvm_slot_restore": [P, I64, I64, I64, I64, I64, P, I32, P, P, P],
    "wkvm_slot_gather": [P, I64, I64, I64, I64, I64, P, I32, P, I64, I64, P, P],
    "wkvm_slot_scatter": [P, I64, I64, I64, I64, I64, P, I32, P, I64, I64, P, P],
    "wkvm_slot_migrate": [P, P, I64, I64, I64, I64, I64, I64, P, P, I32, P, P],
    "wkvm_enable_peer_access": [I32, I32],
    "wkvm_set_decode_overlap": [I32],
    "wkvm_slot_affine": [P, I64, I64, I64, I64, I64, P, P, P, I32, F32, F32, I32, P, P],
    "wkvm_selftest_tf32_mma": [P, P, P, I32, I32, P, P],
    "wkvm_chunk_dplr": [P] * 7 + [P, P, P] + [I32] * 5 + [F32, I32, P, P],
    "wkvm_wkv7_prefill_slots": [P] * 7 + [P, I64, P, P] + [I32] * 5 + [I32, P, P],
    "wkvm_dplr_prefill_slots": [P] * 7 + [P, I64, P, P] + [I32] * 5 + [F32, I32, P, P],
    "wkvm_chunk_gated_delta_rule": [P] * 6 + [P, P, P] + [I32] * 6 + [F32, I32, I32, P, I64, P, P],
    "wkvm_gdn_prefill_slots": [P] * 6 + [P, I64, P, P] + [I32] * 6 + [F32, I32, I32, P, I64, P, P],
    "wkvm_gdn_chunk_workspace_bytes": [I32] * 5,
    "wkvm_wkv7_shift_mix_slots": [P, P, P, I64, I64, P, P, I32, I32, I32, I32, P, P],
    "wkvm_chunk_gated_delta_rule_static": [P] * 6 + [P, P, P] + [I32] * 6 + [F32, I32, I32, P, P],
}

RESTYPES = {
    "wkvm_strerror": ctypes.c_char_p,
    "wkvm_gdn_chunk_workspace_bytes": ctypes.c_int64,
}

ERR_NAMES = {
    -1: "WKVM_ERR_INVALID_ARG", -2: "WKVM_ERR_SHAPE", -3: "WKVM_ERR_DTYPE",
    -4: "WKVM_ERR_SLOT_RANGE", -5: "WKVM_ERR_DUPLICATE", -6: "WKVM_ERR_CUDA",
    -7: "WKVM_ERR_ALIGN", -8: "WKVM_ERR_UNSUPPORTED", -9: "WKVM_ERR_TIMEOUT",
    -10: "WKVM_ERR_SCRATCH",
}

_lock = threading.Lock()
_lib = None


class WkvmError(RuntimeError):
    """A nonzero status from the C ABI."""

    def __init__(self, fn: str, code: int):
        self.code = code
        msg = ERR_NAMES.get(code, str(code))
        try:
            text = _lib.wkvm_strerror(code).decode() if _lib is not None else ""
        except Exception:  # pragma: no cover
            text = ""
        super().__init__(f"{fn} failed: {msg} ({text})")


def load(path: Path | str | None = None):
    """Loads the library once; raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python -m wkvm_b200.build` "
                "(nvcc, sm_100a). wkvm_b200 has no fallback path.")
        lib = ctypes.CDLL(str(p))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.argtypes = argtypes
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = lib
        return lib


# Called with the entry point's name after every successful call when set
# (wkvm_b200.ops.set_debug_checks installs a device-status check here).
post_call = None


def call(name: str, *args) -> None:
    """Calls an entry point and raises WkvmError on a nonzero return."""
    lib = load()
    fn = getattr(lib, name)
    rc = fn(*args)
    if rc != 0:
        raise WkvmError(name, rc)
    if post_call is not None:
        post_call(name)


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in SIGNATURES if hasattr(lib, n)]
