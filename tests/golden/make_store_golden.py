"""Generates golden files that pin wkvm_b200.store_io to wkvm's own StateStore
(wkvm/store.py): layout fingerprints, an index.json and a COLD snapshot file,
all produced by wkvm's code.

Run once in a container where the reference checkout is importable, passing
its path:  python tests/golden/make_store_golden.py <path to the wkvm checkout>

It writes, next to this script:
  store_fingerprints.json  StateStore._fingerprint for a few layouts
  store/index.json         StateStore._write_index for three records (one COLD)
  store/s0_v1.safetensors  StateStore.persist of record s0@1 (tiny layout,
                           values from make_tensors below)
"""

from __future__ import annotations

import json
import shutil
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent

TINY = dict(n_layer=2, hidden_size=8, num_heads=2, head_dim=4, head_v_dim=4)


def make_tensors(layout_kw: dict) -> dict[str, torch.Tensor]:
    """Deterministic WARM tensors of a session for the tiny layout."""
    L, D = layout_kw["n_layer"], layout_kw["hidden_size"]
    H, K, V = layout_kw["num_heads"], layout_kw["head_dim"], layout_kw["head_v_dim"]
    n = L * H * K * V
    wkv = (torch.arange(n, dtype=torch.float32) * 0.37 - 3.1).reshape(L, H, K, V)
    shift = (torch.arange(L * 2 * D, dtype=torch.float32) * -0.11 + 0.5).to(torch.bfloat16)
    return {"wkv": wkv, "shift": shift.reshape(L, 2, D)}


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    from wkvm.models.rwkv7 import RWKV7StateLayout
    from wkvm.store import StateRecord, StateStore

    class _Bank:  # StateStore._fingerprint reads only bank.layout
        def __init__(self, layout):
            self.layout = layout

    layouts = [TINY, dict(n_layer=24, hidden_size=2048, num_heads=32, head_dim=64, head_v_dim=64),
               dict(n_layer=32, hidden_size=4096, num_heads=64, head_dim=64, head_v_dim=64)]
    fps = []
    for kw in layouts:
        for dt in (torch.bfloat16, torch.float16):
            lay = RWKV7StateLayout(dtype=dt, **kw)
            fps.append({"layout": kw, "dtype": str(dt),
                        "fingerprint": StateStore._fingerprint(_Bank(lay))})
    (HERE / "store_fingerprints.json").write_text(json.dumps(fps, indent=1))

    out = HERE / "store"
    if out.exists():
        shutil.rmtree(out)
    out.mkdir()
    store = StateStore.__new__(StateStore)  # no bank needed for the index / persist paths
    store.store_dir = out
    fp = StateStore._fingerprint(_Bank(RWKV7StateLayout(dtype=torch.bfloat16, **TINY)))
    recs = [StateRecord(name="s0", version=1, fingerprint=fp, num_computed_tokens=5,
                        token_ids=(11, 12, 13, 14, 15, 16)),
            StateRecord(name="s0", version=2, fingerprint=fp, num_computed_tokens=5,
                        token_ids=(11, 12, 13, 14, 15, 16), parent="s0@1", rule="decay",
                        rule_params={"alpha": 0.5}),
            StateRecord(name="fork", version=0, fingerprint=fp, num_computed_tokens=5,
                        token_ids=(11, 12, 13, 14, 15, 16), parent="s0@1")]
    store._meta = {r.handle: r for r in recs}
    store._warm = {"s0@1": make_tensors(TINY)}
    store._cold = set()
    store.persist("s0@1")  # writes s0_v1.safetensors and the index
    print("wrote", sorted(p.name for p in out.iterdir()), "and store_fingerprints.json")


if __name__ == "__main__":
    main(sys.argv[1])
