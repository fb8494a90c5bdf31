"""wkvm_b200's runner and bank expose wkvm's interface: the same method
names and parameters as wkvm's RWKV7Runner and RWKV7StateBank (read from
the reference's source when it is present; CPU only, nothing runs)."""

import inspect
import sys
from pathlib import Path

import pytest

REF = Path("/root/reference")


@pytest.fixture(scope="module")
def ref_modules():
    if not (REF / "wkvm" / "runner" / "runner.py").exists():
        pytest.skip("the reference tree is not present")
    sys.path.insert(0, str(REF))
    try:
        from wkvm.runner import runner, state
    except Exception as e:  # pragma: no cover - depends on the reference's imports
        pytest.skip(f"reference not importable: {e}")
    finally:
        sys.path.remove(str(REF))
    return runner, state


def _params(fn):
    return [p for p in inspect.signature(fn).parameters if p != "self"]


def test_runner_interface(ref_modules):
    from wkvm_b200 import runner as ours
    ref = ref_modules[0].RWKV7Runner
    for name in ("__init__", "prefill", "decode_step"):
        assert _params(getattr(ours.RWKV7Runner, name)) == _params(getattr(ref, name)), name


def test_bank_interface(ref_modules):
    from wkvm_b200 import state as ours
    ref = ref_modules[1].RWKV7StateBank
    for name in ("__init__", "zero_slots", "gather_cache", "scatter_cache", "state_bytes"):
        mine = _params(getattr(ours.RWKV7StateBank, name))
        theirs = _params(getattr(ref, name))
        assert mine[:len(theirs)] == theirs, name  # extra keyword parameters only at the end
