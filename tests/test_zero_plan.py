"""Host-side bookkeeping of the ZeRO-1 in-GEMM all-gather (no GPU needed)."""
import torch

from dtrain_b200.models.gpt import GPT, GPTConfig
from dtrain_b200.models.params import FlatParams
from dtrain_b200.parallel.zero import GS_GEN, GS_SITES, GatherPlan, keep_intervals


def test_keep_intervals_is_the_complement():
    assert keep_intervals(10, []) == [(0, 10)]
    assert keep_intervals(10, [(0, 10)]) == []
    assert keep_intervals(10, [(6, 8), (2, 4)]) == [(0, 2), (4, 6), (8, 10)]
    assert keep_intervals(10, [(0, 3), (3, 5)]) == [(5, 10)]


def test_gemm_weights_are_the_linear_weights_and_the_rest_is_kept():
    m = GPT(GPTConfig(vocab=65, ctx=16, dim=32, heads=2, layers=2))
    ws = m.gemm_weights()
    names = {id(p): n for n, p in m.named_parameters()}
    assert [names[id(w)] for w in ws] == [
        "blocks.0.qkv.w", "blocks.0.proj.w", "blocks.0.fc.w", "blocks.0.out.w",
        "blocks.1.qkv.w", "blocks.1.proj.w", "blocks.1.fc.w", "blocks.1.out.w", "head.w"]
    params = list(m.parameters())
    offs, off = {}, 0
    for p in params:
        offs[id(p)] = (off, off + p.numel())
        off += p.numel()
    keep = keep_intervals(off, [offs[id(w)] for w in ws])
    kept = sum(hi - lo for lo, hi in keep)
    assert kept + sum(w.numel() for w in ws) == off
    # every non-GEMM parameter lies entirely inside one kept interval
    for p in params:
        if any(p is w for w in ws):
            continue
        lo, hi = offs[id(p)]
        assert any(a <= lo and hi <= b for a, b in keep)


def test_gather_plan_sites_and_generation_bookkeeping():
    m = GPT(GPTConfig(vocab=65, ctx=16, dim=32, heads=2, layers=1))
    fp = FlatParams(list(m.parameters()), "cpu", with_work=False)
    ws = m.gemm_weights()
    bases = [1 << 20, 3 << 20]  # every rank's base address of the bf16 working copy
    plan = GatherPlan(fp, ws, bases, rank=1)
    assert plan.rank == 1 and plan.nflat == fp.n
    for s, w in enumerate(ws):
        site, off, peers = plan.sites[id(w)]
        assert site == s and off == fp.slot(fp.index[id(w)])[0]
        assert peers == [b + 2 * off for b in bases]  # bf16: 2 bytes per element
    keep = [tuple(r) for r in plan.keep.tolist()]
    assert keep == keep_intervals(fp.n, [(o, o + w.numel()) for w in ws for o in [fp.slot(fp.index[id(w)])[0]]])
    assert plan.state.dtype == torch.int32 and plan.state.numel() == GS_SITES + len(ws)
    plan.state[GS_GEN] = 7
    plan.mark_gathered()
    assert plan.state[GS_SITES:].tolist() == [7] * len(ws)


def test_train_flops_per_token_counts_gemm_weights_and_causal_attention():
    from dtrain_b200.models.gpt import train_flops_per_token
    c = GPTConfig(vocab=50304, ctx=1024, dim=768, heads=12, layers=12)
    gemm = 12 * (768 * 2304 + 768 * 768 + 2 * 768 * 3072) + 768 * 50304  # 123.57 M weights
    assert gemm == 123_568_128
    assert train_flops_per_token(c) == 6.0 * gemm + 6.0 * 12 * 1024 * 768
