"""fla's RWKV-7 model (the model wkvm serves) run with wkvm_b200 installed
and slot-resident state, against the same model on fla's own Triton ops with
wkvm's gather -> forward -> scatter flow. Prefill (>= 64 tokens: chunk path)
then decode steps. Skipped where fla cannot run."""

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

fla_models = pytest.importorskip("fla.models.rwkv7")


def test_slot_resident_model_matches_fla_path(cuda):
    from fla.models.utils import Cache
    from wkvm_b200 import fla_compat
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    torch.manual_seed(0)
    L, D, N = 2, 256, 64
    cfg = fla_models.RWKV7Config(hidden_size=D, num_hidden_layers=L, head_dim=N, vocab_size=512)
    with torch.device(cuda):
        model = fla_models.RWKV7ForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
    lay = RWKV7StateLayout(n_layer=L, hidden_size=D, num_heads=D // N, head_dim=N, head_v_dim=N)
    ours = RWKV7StateBank(lay, num_slots=4, device=cuda)
    ref = RWKV7StateBank(lay, num_slots=4, device=cuda)
    slots = [3, 1]
    ids = torch.tensor(slots, device=cuda)
    prompt = torch.randint(0, 512, (2, 96), device=cuda)

    def ref_forward(tokens):
        cache = Cache()
        for i in range(L):
            cache.update(recurrent_state=ref.wkv[i].index_select(0, ids),
                         conv_state=ref.shift[i, 0].index_select(0, ids),
                         ffn_state=ref.shift[i, 1].index_select(0, ids), layer_idx=i, offset=0)
        out = model(input_ids=tokens, past_key_values=cache, use_cache=True, logits_to_keep=1)
        for i in range(L):
            ref.wkv[i].index_copy_(0, ids, cache[i]["recurrent_state"].float())
            ref.shift[i, 0].index_copy_(0, ids, cache[i]["conv_state"])
            ref.shift[i, 1].index_copy_(0, ids, cache[i]["ffn_state"])
        return out.logits.float()

    def our_forward(tokens):
        h = fla_compat.slot_cache(ours, slots)
        out = model(input_ids=tokens, past_key_values=h.cache, use_cache=True, logits_to_keep=1)
        h.commit()
        return out.logits.float()

    with torch.inference_mode():
        fla_compat.uninstall()
        ref_logits = [ref_forward(prompt)]
        fla_compat.install()
        try:
            our_logits = [our_forward(prompt)]
            tok = our_logits[0].argmax(-1)
            for _ in range(3):
                our_logits.append(our_forward(tok))
                fla_compat.uninstall()
                ref_logits.append(ref_forward(tok))
                fla_compat.install()
                tok = our_logits[-1].argmax(-1)
        finally:
            fla_compat.uninstall()
    # prefill: fla's chunk path rounds to bf16 inside its dots, ours keeps tf32
    assert rel_err(our_logits[0], ref_logits[0]) < 2e-2
    for o, r in zip(our_logits[1:], ref_logits[1:]):
        assert rel_err(o, r) < 2e-2
        assert (o.argmax(-1) == r.argmax(-1)).all()
    assert rel_err(ours.wkv[:, slots], ref.wkv[:, slots]) < 2e-2
    assert torch.equal(ours.wkv[:, [0, 2, 4]], ref.wkv[:, [0, 2, 4]])  # untouched slots stay zero
