"""Fused RWKV-7 time-mix decode core against the same chain of fla's
formulas (fla/layers/rwkv7.py:270-349) computed step by step in fp32."""

import pytest
import torch

from conftest import REL_TOL, assert_out_close, rel_err
from wkvm_b200 import ops

pytestmark = pytest.mark.gpu


def _reference_chain(r, w_raw, k, v, v_first, v_raw, a_raw, g, k_k, k_a, r_k, gn_w, gn_b, eps,
                     h0):
    B, D = r.shape
    H, N = D // 64, 64
    f = lambda t: t.float()
    w = -0.6065306597126334 * torch.sigmoid(f(w_raw))
    vv = f(v)
    if v_first is not None:
        vv = torch.lerp(vv, f(v_first), torch.sigmoid(f(v_raw)))
    a = torch.sigmoid(f(a_raw))
    kk = (f(k) * f(k_k)).view(B, H, N)
    kk = (kk / torch.sqrt((kk * kk).sum(-1, keepdim=True) + 1e-6)).view(B, D)
    ku = f(k) + f(k) * (a - 1) * f(k_a)
    sh = lambda t: t.view(B, 1, H, N).contiguous()
    o, ht = ops.fused_mul_recurrent_rwkv7(sh(f(r)), sh(w), sh(ku), sh(vv), sh(kk), sh(a),
                                          scale=1.0, initial_state=h0, output_final_state=True)
    o = o.view(B, H, N)
    mean = o.mean(-1, keepdim=True)
    var = ((o - mean) ** 2).mean(-1, keepdim=True)
    on = ((o - mean) / torch.sqrt(var + eps)).view(B, D) * f(gn_w) + f(gn_b)
    corr = (f(r) * ku * f(r_k).view(D)).view(B, H, N).sum(-1, keepdim=True)
    out = (on + (corr * vv.view(B, H, N)).view(B, D)) * f(g)
    return out, ht


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("first_layer", [True, False])
def test_timemix_matches_formula_chain(cuda, dtype, first_layer):
    torch.manual_seed(0)
    B, H, N, S = 6, 4, 64, 9
    D = H * N
    mk = lambda *s, sc=1.0: (torch.randn(*s, device=cuda) * sc).to(dtype)
    r, w_raw, k, v, a_raw = mk(B, D), mk(B, D), mk(B, D), mk(B, D), mk(B, D)
    g = torch.sigmoid(torch.randn(B, D, device=cuda)).to(dtype)
    v_first = None if first_layer else mk(B, D)
    v_raw = None if first_layer else mk(B, D)
    k_k, k_a, r_k = mk(D, sc=0.5), mk(D, sc=0.5), mk(H, N, sc=0.5)
    gn_w, gn_b = mk(D, sc=0.3), mk(D, sc=0.1)
    eps = 64e-5
    bank = (torch.randn(2, S, H, N, N, device=cuda) * 0.1)
    ids = [7, 2, 5, 1, 8, 3]
    h0 = bank[1, ids].clone()
    ref, ht = _reference_chain(r, w_raw, k, v, v_first, v_raw, a_raw, g, k_k, k_a, r_k, gn_w,
                               gn_b, eps, h0)
    o = ops.wkv7_timemix_decode_slots(r, w_raw, k, v, v_first, v_raw, a_raw, g, k_k, k_a, r_k,
                                      gn_w, gn_b, eps, bank, 1, ids)
    ops.check_device_status(cuda)
    assert rel_err(bank[1, ids], ht) < (1e-5 if dtype == torch.float32 else REL_TOL)
    if dtype == torch.float32:
        assert rel_err(o, ref) < 1e-4
    else:
        assert_out_close(o, ref)


@pytest.mark.parametrize("n_mix", [6, 1])
def test_shift_mix_matches_token_shift_addcmul(cuda, n_mix):
    # fla decode prologue: delta = token_shift(x, cache) stored as bf16, then
    # torch.addcmul(x, delta, mix) per mix; the new shift state is x
    torch.manual_seed(3)
    L, S, B, D = 2, 9, 5, 256
    shift = torch.randn(L, 2, S + 1, D, device=cuda).to(torch.bfloat16)
    before = shift.clone()
    x = torch.randn(B, 1, D, device=cuda).to(torch.bfloat16)
    mixes = [torch.rand(1, 1, D, device=cuda).to(torch.bfloat16) for _ in range(n_mix)]
    ids = [7, 2, 9, 0, 4]
    layer, fam = 1, n_mix == 1
    prev = shift[layer, int(fam), ids].view(B, 1, D)
    delta = (prev.float() - x.float()).to(torch.bfloat16)
    ref = [torch.addcmul(x, delta, m) for m in mixes]
    outs = ops.wkv7_shift_mix_slots(x, mixes, shift[layer, int(fam)], ids)
    ops.check_device_status(cuda)
    assert len(outs) == n_mix
    for o, r in zip(outs, ref):
        assert o.shape == (B, 1, D)
        # one bf16 rounding of the same fp32 value (at most one ulp apart)
        assert ((o.float() - r.float()).abs() <= r.float().abs() * 2.0 ** -7 + 1e-30).all()
    assert torch.equal(shift[layer, int(fam), ids], x.view(B, D))
    rest = [i for i in range(S + 1) if i not in ids]
    assert torch.equal(shift[layer, int(fam), rest], before[layer, int(fam), rest])
    assert torch.equal(shift[layer, 1 - int(fam)], before[layer, 1 - int(fam)])
    assert torch.equal(shift[0], before[0])


@pytest.mark.parametrize("shift_in_bank", [False, True])
def test_fused_time_mix_model_decode_close_to_fla(cuda, shift_in_bank):
    fla_models = pytest.importorskip("fla.models.rwkv7")
    from fla.models.utils import Cache
    from wkvm_b200 import fla_compat
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    torch.manual_seed(1)
    L, D, N = 3, 256, 64
    cfg = fla_models.RWKV7Config(hidden_size=D, num_hidden_layers=L, head_dim=N, vocab_size=512)
    with torch.device(cuda):
        model = fla_models.RWKV7ForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
    for p in model.parameters():  # non-trivial parameters (fla's init zeroes some)
        p.data.add_(torch.randn_like(p) * 0.05)
    lay = RWKV7StateLayout(n_layer=L, hidden_size=D, num_heads=D // N, head_dim=N, head_v_dim=N)
    ours = RWKV7StateBank(lay, num_slots=4, device=cuda)
    ref = RWKV7StateBank(lay, num_slots=4, device=cuda)
    for b in (ours, ref):
        b.wkv.copy_(torch.randn_like(b.wkv, generator=torch.Generator(device=cuda).manual_seed(3)) * 0.1)
        b.shift.copy_(torch.randn(b.shift.shape, device=cuda,
                                  generator=torch.Generator(device=cuda).manual_seed(4)))
    slots = [2, 4, 1]
    ids = torch.tensor(slots, device=cuda)
    tok = torch.randint(0, 512, (3, 1), device=cuda)

    def ref_step(t):
        cache = Cache()
        for i in range(L):
            cache.update(recurrent_state=ref.wkv[i].index_select(0, ids),
                         conv_state=ref.shift[i, 0].index_select(0, ids),
                         ffn_state=ref.shift[i, 1].index_select(0, ids), layer_idx=i, offset=0)
        out = model(input_ids=t, past_key_values=cache, use_cache=True, logits_to_keep=1)
        for i in range(L):
            ref.wkv[i].index_copy_(0, ids, cache[i]["recurrent_state"].float())
            ref.shift[i, 0].index_copy_(0, ids, cache[i]["conv_state"])
            ref.shift[i, 1].index_copy_(0, ids, cache[i]["ffn_state"])
        return out.logits.float()

    with torch.inference_mode():
        fla_compat.uninstall()
        ref_logits = [ref_step(tok) for _ in range(4)]
        fla_compat.install(fuse_time_mix=True)
        try:
            our_logits = []
            for _ in range(4):
                h = fla_compat.slot_cache(ours, slots, shift_in_bank=shift_in_bank)
                our_logits.append(model(input_ids=tok, past_key_values=h.cache, use_cache=True,
                                        logits_to_keep=1).logits.float())
                h.commit()
        finally:
            fla_compat.uninstall()
    # fla rounds every intermediate to bf16; the fused core keeps fp32
    for o, r in zip(our_logits, ref_logits):
        assert rel_err(o, r) < 3e-2
    assert rel_err(ours.wkv[:, slots], ref.wkv[:, slots]) < 3e-2
    assert rel_err(ours.shift[:, :, slots], ref.shift[:, :, slots]) < 3e-2
    rest = [i for i in range(5) if i not in slots]
    assert torch.equal(ours.shift[:, :, rest], ref.shift[:, :, rest])


@pytest.mark.parametrize("graph", [False, True])
def test_timemix_overlap_layer_loop(cuda, graph):
    """Overlapped (programmatic dependent launch) time-mix over a layer loop
    whose activations each come from the kernel launched just before (a
    stand-in for the projection GEMM): the same bits as without overlap,
    eagerly and inside a CUDA graph."""
    torch.manual_seed(3)
    L, S, H, N, B, steps = 4, 9, 4, 64, 5, 3
    D = H * N
    mk = lambda *s, sc=1.0: torch.randn(*s, device=cuda) * sc
    base = [[mk(B, D).to(torch.bfloat16) for _ in range(8)] for _ in range(L)]
    prm = [[mk(D, sc=0.5).to(torch.bfloat16), mk(D, sc=0.5).to(torch.bfloat16),
            mk(H, N, sc=0.5).to(torch.bfloat16), mk(D, sc=0.3).to(torch.bfloat16),
            mk(D, sc=0.1).to(torch.bfloat16)] for _ in range(L)]
    ids = ops.slot_ids_tensor([5, 1, 7, 3, 8], S, cuda)
    bank0 = mk(L, S, H, N, N, sc=0.1)
    acts = [[torch.empty_like(t) for t in base[layer]] for layer in range(L)]
    outs = [torch.empty(B, D, dtype=torch.bfloat16, device=cuda) for _ in range(L)]

    def run(bank):
        for s in range(steps):
            for layer in range(L):
                a = acts[layer]
                torch.mul(base[layer][0], 1.0 + s, out=a[0])  # written by the kernel just before
                for i in range(1, 8):
                    a[i].copy_(base[layer][i])
                r, w, k, v, vf, vr, aa, g = a
                ops.wkv7_timemix_decode_slots(r, w, k, v, vf if layer else None,
                                              vr if layer else None, aa, g, *prm[layer], 64e-5,
                                              bank, layer, ids, out=outs[layer])
        return [o.clone() for o in outs]

    bank_ref = bank0.clone()
    ref = run(bank_ref)
    torch.cuda.synchronize()
    bank = bank0.clone()
    prev = ops.set_decode_overlap(True)
    try:
        if graph:
            s = torch.cuda.Stream(cuda)
            s.wait_stream(torch.cuda.current_stream(cuda))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                got = run(bank)
            bank.copy_(bank0)
            g.replay()
        else:
            got = run(bank)
        torch.cuda.synchronize()
    finally:
        ops.set_decode_overlap(prev)
    ops.check_device_status(cuda)
    assert torch.equal(bank, bank_ref)
    for o, r in zip(got, ref):
        assert torch.equal(o, r)
