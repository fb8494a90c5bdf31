"""The bank and runner as wkvm's RWKV7Runner drives them
(wkvm/runner/runner.py:42-89, wkvm/runner/state.py:63-97).

* gather_cache / scatter_cache round trips and untouched neighbours, the
  checks of wkvm's own bank tests (tests/test_rwkv7_gpu.py:85-120), in both
  cache modes (copies, and slot-resident with wkvm_b200 installed in fla);
* the runner on a small random-init fla RWKV-7 model: prefill in 64-token
  pieces (chunk path, then a 36-token recurrent remainder) and batched
  decode, with wkvm_b200 installed (plain and with the fused time-mix core),
  against the same runner on a bank with wkvm's index_select / index_copy
  gather and scatter and fla's own Triton kernels."""

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

fla_models = pytest.importorskip("fla.models.rwkv7")


def _bank(cuda, n_layer=3, D=64, N=32, slots=4):
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout
    lay = RWKV7StateLayout(n_layer=n_layer, hidden_size=D, num_heads=D // N, head_dim=N,
                           head_v_dim=N, dtype=torch.bfloat16)
    return RWKV7StateBank(lay, num_slots=slots, device=cuda)


@pytest.mark.parametrize("resident", [False, True])
def test_gather_scatter_roundtrip(cuda, resident):
    bank = _bank(cuda)
    g = torch.Generator(device=cuda).manual_seed(1)
    bank.wkv.normal_(generator=g)
    bank.shift.copy_(torch.randn(bank.shift.shape, generator=g, device=cuda))
    before = (bank.wkv.clone(), bank.shift.clone())
    batch = [{"wkv": 2, "shift": 2}, {"wkv": 4, "shift": 4}]
    cache = bank.gather_cache(batch, resident=resident)
    expected = []
    for i in range(bank.layout.n_layer):
        st = cache[i]
        if not resident:
            assert torch.equal(st["recurrent_state"], before[0][i, [2, 4]])
            st["recurrent_state"].normal_(generator=g)
        st["conv_state"].normal_(generator=g)
        st["ffn_state"].normal_(generator=g)
        expected.append((None if resident else st["recurrent_state"].clone(),
                         st["conv_state"].clone(), st["ffn_state"].clone()))
    bank.scatter_cache(batch, cache)
    back = bank.gather_cache(batch, resident=False)
    for i, (wkv, conv, ffn) in enumerate(expected):
        ref_wkv = before[0][i, [2, 4]] if resident else wkv
        assert torch.equal(back[i]["recurrent_state"], ref_wkv)
        assert torch.equal(back[i]["conv_state"], conv)
        assert torch.equal(back[i]["ffn_state"], ffn)
    for s in (0, 1, 3):
        assert torch.equal(bank.wkv[:, s], before[0][:, s])
        assert torch.equal(bank.shift[:, :, s], before[1][:, :, s])


def test_scatter_leaves_other_slots_untouched(cuda):
    bank = _bank(cuda)
    cache = bank.gather_cache([{"wkv": 3, "shift": 3}], resident=False)
    for i in range(bank.layout.n_layer):
        for key in ("recurrent_state", "conv_state", "ffn_state"):
            cache[i][key].fill_(1.0)
    bank.scatter_cache([{"wkv": 3, "shift": 3}], cache)
    for s in (0, 1, 2, 4):
        assert bank.wkv[:, s].abs().sum().item() == 0.0
        assert bank.shift[:, :, s].abs().sum().item() == 0.0
    assert bank.wkv[:, 3].abs().sum().item() > 0.0


class StockBank:
    """wkvm's bank flow: index_select copies into an fla Cache and
    index_copy_ back (what wkvm/runner/state.py:63-97 does), for the
    reference side of the comparison."""

    def __init__(self, like):
        self.layout = like.layout
        self.device = like.device
        self.wkv = torch.zeros_like(like.wkv)
        self.shift = torch.zeros_like(like.shift)

    def gather_cache(self, batch):
        from fla.models.utils import Cache
        w = torch.tensor([s["wkv"] for s in batch], device=self.device)
        sh = torch.tensor([s["shift"] for s in batch], device=self.device)
        cache = Cache()
        for i in range(self.layout.n_layer):
            cache.update(recurrent_state=self.wkv[i].index_select(0, w),
                         conv_state=self.shift[i, 0].index_select(0, sh),
                         ffn_state=self.shift[i, 1].index_select(0, sh), layer_idx=i, offset=0)
        return cache

    def scatter_cache(self, batch, cache):
        w = torch.tensor([s["wkv"] for s in batch], device=self.device)
        sh = torch.tensor([s["shift"] for s in batch], device=self.device)
        for i in range(self.layout.n_layer):
            self.wkv[i].index_copy_(0, w, cache[i]["recurrent_state"].float())
            self.shift[i, 0].index_copy_(0, sh, cache[i]["conv_state"].to(self.shift.dtype))
            self.shift[i, 1].index_copy_(0, sh, cache[i]["ffn_state"].to(self.shift.dtype))


@pytest.mark.parametrize("fuse", [False, True])
def test_runner_matches_wkvm_flow(cuda, fuse):
    from wkvm_b200 import fla_compat
    from wkvm_b200.runner import RWKV7Runner

    torch.manual_seed(0)
    L, D, N, vocab = 2, 256, 64, 512
    cfg = fla_models.RWKV7Config(hidden_size=D, num_hidden_layers=L, head_dim=N,
                                 vocab_size=vocab)
    with torch.device(cuda):
        model = fla_models.RWKV7ForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
    ours = _bank(cuda, n_layer=L, D=D, N=N, slots=6)
    stock = StockBank(ours)
    batch = [{"wkv": 5, "shift": 2}, {"wkv": 1, "shift": 6}]
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, vocab, (100,), generator=g).tolist(),
               torch.randint(0, vocab, (70,), generator=g).tolist()]

    def run(runner, feed=None):
        # feed: the tokens to decode (the reference run's argmax), so that both
        # runs see the same inputs
        logits = [torch.stack([runner.prefill(p, s) for p, s in zip(prompts, batch)])]
        for step in range(4):
            tok = feed[step] if feed else logits[-1].argmax(-1).tolist()
            logits.append(runner.decode_step(batch, tok))
        return logits

    fla_compat.uninstall()
    ref = run(RWKV7Runner(model, stock, prefill_chunk=64))
    fla_compat.install(fuse_time_mix=fuse)
    try:
        got = run(RWKV7Runner(model, ours, prefill_chunk=64),
                  feed=[r.argmax(-1).tolist() for r in ref])
    finally:
        fla_compat.uninstall()
    # fla's chunk path rounds to bf16 inside its dots, ours keeps tf32; the
    # fused core computes the gates in fp32 where fla rounds to bf16
    for i, (o, r) in enumerate(zip(got, ref)):
        assert rel_err(o, r) < 2e-2, i
        assert (o.argmax(-1) == r.argmax(-1)).all(), i
    assert rel_err(ours.wkv[:, [5, 1]], stock.wkv[:, [5, 1]]) < 2e-2
    assert rel_err(ours.shift[:, :, [2, 6]].float(), stock.shift[:, :, [2, 6]].float()) < 2e-2
    for s in (0, 2, 3, 4, 6):
        assert ours.wkv[:, s].abs().sum().item() == 0.0
    for s in (0, 1, 3, 4, 5):
        assert ours.shift[:, :, s].abs().sum().item() == 0.0


@pytest.mark.parametrize("fuse", [True, False])
def test_graphed_decode_matches_wkvm_flow(cuda, fuse):
    """The whole decode step captured once (wkvm_b200.graph.GraphedDecode)
    and replayed for changing batches -- full, and smaller than the graph
    (padded with slot 0) -- against wkvm's gather -> fla Triton -> scatter
    flow on the same states."""
    from wkvm_b200 import fla_compat
    from wkvm_b200.graph import GraphedDecode
    from wkvm_b200.runner import RWKV7Runner

    torch.manual_seed(1)
    L, D, N, vocab = 2, 256, 64, 512
    cfg = fla_models.RWKV7Config(hidden_size=D, num_hidden_layers=L, head_dim=N,
                                 vocab_size=vocab)
    with torch.device(cuda):
        model = fla_models.RWKV7ForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
    ours = _bank(cuda, n_layer=L, D=D, N=N, slots=8)
    g = torch.Generator(device=cuda).manual_seed(2)
    ours.wkv.normal_(0.0, 0.1, generator=g)
    ours.shift.copy_(torch.randn(ours.shift.shape, generator=g, device=cuda) * 0.5)
    stock = StockBank(ours)
    stock.wkv.copy_(ours.wkv)
    stock.shift.copy_(ours.shift)
    batches = [[{"wkv": 3, "shift": 3}, {"wkv": 7, "shift": 5}, {"wkv": 1, "shift": 8}],
               [{"wkv": 7, "shift": 5}, {"wkv": 2, "shift": 2}],
               [{"wkv": 1, "shift": 8}, {"wkv": 3, "shift": 3}, {"wkv": 8, "shift": 1}]]
    gen = torch.Generator().manual_seed(5)
    toks = [torch.randint(0, vocab, (len(b),), generator=gen).tolist() for b in batches]
    fla_compat.uninstall()
    ref_runner = RWKV7Runner(model, stock)
    ref = [ref_runner.decode_step(b, t) for b, t in zip(batches, toks)]
    try:
        gd = GraphedDecode(RWKV7Runner(model, ours), batch_size=3, fuse_time_mix=fuse)
        got = [gd.decode_step(b, t) for b, t in zip(batches, toks)]
        torch.cuda.synchronize()
    finally:
        fla_compat.uninstall()
    for i, (o, r) in enumerate(zip(got, ref)):
        assert o.shape == r.shape, i
        assert rel_err(o, r) < 2e-2, i
        assert (o.argmax(-1) == r.argmax(-1)).all(), i
    used_wkv = [1, 2, 3, 7, 8]
    used_shift = [1, 2, 3, 5, 8]
    assert rel_err(ours.wkv[:, used_wkv], stock.wkv[:, used_wkv]) < 2e-2
    assert rel_err(ours.shift[:, :, used_shift].float(), stock.shift[:, :, used_shift].float()) < 2e-2
    for s in (4, 5, 6):  # never in a batch: untouched
        assert torch.equal(ours.wkv[:, s], stock.wkv[:, s])
