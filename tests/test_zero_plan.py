"""Host-side bookkeeping of the ZeRO-1 in-GEMM all-gather (no GPU needed)."""
from dtrain_b200.models.gpt import GPT, GPTConfig
from dtrain_b200.parallel.zero import keep_intervals


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
