"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments on the host before any launch."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(wkvm_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from wkvm_b200 import _lib, build
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "wkvm_wkv7_decode_slots" in names and "wkvm_slot_copy" in names
    assert len(names) >= 12


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(lib):
    from wkvm_b200 import _lib
    missing = [n for n in declared_symbols() if n not in _lib.SIGNATURES]
    assert not missing, missing


def test_version_and_strerror(lib):
    assert lib.wkvm_version() >= 100
    assert lib.wkvm_strerror(-4) == b"slot id out of range"


def _buffers():
    """Two pointers the rejected calls below receive: zeroed 1 MiB device
    buffers when a GPU is present (a check that regressed then launches on
    real memory, larger than any of these calls would touch), else dummy
    addresses that no call here may dereference."""
    import torch
    if torch.cuda.is_available():
        bufs = [torch.zeros(1 << 20, dtype=torch.uint8, device="cuda") for _ in range(2)]
        return bufs, [ctypes.c_void_p(b.data_ptr()) for b in bufs]
    return [], [ctypes.c_void_p(4096), ctypes.c_void_p(1 << 20)]


def test_host_argument_checks(lib):
    from wkvm_b200 import _lib
    keep, (dummy, dummy2) = _buffers()
    # null bank / ids are rejected before anything reaches the device
    assert lib.wkvm_slot_copy(None, 1, 16, 16, 16, 4, None, None, 1, None, None) == -1
    # misaligned row size
    assert lib.wkvm_slot_zero(dummy, 1, 24, 24, 24, 4, dummy2, 1, None, None) == -7
    # unsupported head dim never launches
    rc = lib.wkvm_fused_mul_recurrent_rwkv7(*([dummy] * 7), None, None, None, 1, 1, 1, 48, 48,
                                            ctypes.c_float(1.0), 1, None, None)
    assert rc == -2
    # unknown dtype
    rc = lib.wkvm_fused_mul_recurrent_rwkv7(*([dummy] * 7), None, None, None, 1, 1, 1, 64, 64,
                                            ctypes.c_float(1.0), 7, None, None)
    assert rc == -3
    # empty batch is a no-op
    rc = lib.wkvm_wkv7_decode_slots(*([dummy] * 7), dummy, 5, dummy, 0, 1, 1, 64, 64, 1, None,
                                    None)
    assert rc == 0
    assert _lib.ERR_NAMES[-5] == "WKVM_ERR_DUPLICATE"
    if keep:
        import torch
        torch.cuda.synchronize()


def test_gdn_workspace_size(lib):
    # one 73,856-byte chunk record per (sequence, value head, 64-token chunk)
    assert lib.wkvm_gdn_chunk_workspace_bytes(4, 8192, 16, 128, 128) == 4 * 16 * 128 * 73856
    assert lib.wkvm_gdn_chunk_workspace_bytes(1, 65, 2, 128, 128) == 2 * 2 * 73856
    assert lib.wkvm_gdn_chunk_workspace_bytes(2, 0, 2, 128, 128) == 0
    # shapes without the two-launch path
    assert lib.wkvm_gdn_chunk_workspace_bytes(4, 64, 16, 64, 64) == 0
