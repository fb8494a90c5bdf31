"""COLD-tier format and fingerprints against files written by wkvm's own
StateStore (tests/golden/make_store_golden.py)."""

import json
import sys
from pathlib import Path

import torch

from wkvm_b200 import store_io
from wkvm_b200.state import RWKV7StateLayout

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
from make_store_golden import TINY, make_tensors  # noqa: E402


def test_fingerprint_matches_wkvm():
    for e in json.loads((GOLDEN / "store_fingerprints.json").read_text()):
        dtype = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16}[e["dtype"]]
        lay = RWKV7StateLayout(dtype=dtype, **e["layout"])
        assert store_io.fingerprint(lay) == e["fingerprint"]


def test_index_round_trip_matches_wkvm(tmp_path):
    recs, cold = store_io.read_index(GOLDEN / "store")
    assert set(recs) == {"s0@1", "s0@2", "fork@0"} and cold == {"s0@1"}
    assert recs["s0@2"].rule == "decay" and recs["s0@2"].rule_params == {"alpha": 0.5}
    assert recs["fork@0"].parent == "s0@1" and recs["s0@1"].token_ids == (11, 12, 13, 14, 15, 16)
    store_io.write_index(tmp_path, recs.values(), cold)
    ours = json.loads((tmp_path / "index.json").read_text())
    assert ours == json.loads((GOLDEN / "store" / "index.json").read_text())


def test_cold_file_is_byte_identical_to_wkvm(tmp_path):
    path = store_io.cold_path(tmp_path, "s0@1")
    assert path.name == "s0_v1.safetensors"
    store_io.save_cold(path, make_tensors(TINY))
    assert path.read_bytes() == (GOLDEN / "store" / "s0_v1.safetensors").read_bytes()
    back = store_io.load_cold(GOLDEN / "store" / "s0_v1.safetensors", pin=False)
    ref = make_tensors(TINY)
    assert back["wkv"].dtype == torch.float32 and back["shift"].dtype == torch.bfloat16
    assert torch.equal(back["wkv"], ref["wkv"]) and torch.equal(back["shift"], ref["shift"])
