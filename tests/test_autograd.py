"""Gradient checks for every op and the full model (float64, CPU), and hook semantics.

Same coverage as the reference's finite-difference tests; differences are taken
by torch.autograd.gradcheck (central differences in float64).
"""
import numpy as np
import pytest
import torch

from dtrain_b200.autograd import (causal_attention, cross_entropy, embedding, gelu, layer_norm, linear,
                                  register_grad_ready_hook, relu)
from dtrain_b200.nn import GPT, GPTConfig

g = torch.Generator().manual_seed(0)


def _t(*shape):
    return torch.randn(*shape, generator=g, dtype=torch.float64, requires_grad=True)


def check(fn, *xs):
    assert torch.autograd.gradcheck(fn, xs, eps=1e-6, atol=1e-5, rtol=1e-5)


def test_elementwise_broadcast_and_matmul():
    check(lambda a, b: a + b, _t(3, 4), _t(4))
    check(lambda a, b: a * b, _t(2, 3, 4), _t(1, 4))
    check(lambda a, b: a @ b, _t(2, 3, 4), _t(4, 5))
    check(lambda a, b: a @ b, _t(2, 3, 4), _t(2, 4, 2))
    check(lambda x, w, b: linear(x, w, b), _t(2, 3, 4), _t(4, 5), _t(5))


def test_reductions_reshape_transpose():
    check(lambda a: a.sum(dim=1), _t(3, 4, 2))
    check(lambda a: a.mean(dim=-1, keepdim=True), _t(3, 4))
    check(lambda a: a.reshape(4, 6).transpose(1, 0), _t(2, 3, 4))


def test_activations():
    check(gelu, _t(4, 5))
    check(relu, _t(4, 5))


def test_layer_norm():
    check(lambda x, w, b: layer_norm(x, w, b), _t(2, 3, 6), _t(6), _t(6))


def test_attention():
    check(causal_attention, _t(1, 2, 4, 3), _t(1, 2, 4, 3), _t(1, 2, 4, 3))


def test_embedding_with_repeated_indices():
    idx = torch.tensor([[0, 2, 2], [1, 0, 2]])
    check(lambda w: embedding(w, idx), _t(3, 4))


def test_cross_entropy():
    t = torch.randint(0, 5, (2, 3), generator=g)
    check(lambda z: cross_entropy(z, t), _t(2, 3, 5))


def test_attention_matches_reference_formula():
    q, k, v = _t(2, 2, 5, 4), _t(2, 2, 5, 4), _t(2, 2, 5, 4)
    out = causal_attention(q, k, v)
    s = (q @ k.transpose(-1, -2)) / 2.0
    s = s.masked_fill(torch.triu(torch.ones(5, 5, dtype=torch.bool), 1), float("-inf"))
    s = s - s.max(-1, keepdim=True).values
    p = torch.exp(s)
    p = p / p.sum(-1, keepdim=True)
    torch.testing.assert_close(out, p @ v, rtol=1e-12, atol=1e-12)


def test_full_model_gradient_float64():
    cfg = GPTConfig(vocab=7, ctx=5, dim=8, heads=2, layers=2, dtype="float64")
    m = GPT(cfg, seed=1)
    rng = np.random.default_rng(0)
    x = torch.as_tensor(rng.integers(0, 7, size=(2, 5)))
    y = torch.as_tensor(rng.integers(0, 7, size=(2, 5)))
    _, loss = m(x, y)
    loss.backward()
    with torch.no_grad():
        for name, p in m.named_parameters():
            for _ in range(3):
                i = tuple(int(rng.integers(0, s)) for s in p.shape)
                old = p[i].item()
                p[i] = old + 1e-6
                fp = m(x, y)[1].item()
                p[i] = old - 1e-6
                fm = m(x, y)[1].item()
                p[i] = old
                assert abs(p.grad[i].item() - (fp - fm) / 2e-6) < 1e-6, name


def test_grad_ready_hook_fires_once_with_final_gradient():
    w = _t(3, 3)
    seen = []
    register_grad_ready_hook(w, lambda t: seen.append(t.grad.clone()))
    x = torch.randn(2, 3, generator=g, dtype=torch.float64)
    y = (x @ w) + (x @ w) * 2.0  # w used twice
    y.sum().backward()
    assert len(seen) == 1
    torch.testing.assert_close(seen[0], w.grad)


def test_parameter_names_and_order_match_reference():
    cfg = GPTConfig(vocab=7, ctx=5, dim=8, heads=2, layers=1, dtype="float64")
    names = [n for n, _ in GPT(cfg).named_parameters()]
    assert names == ["tok", "pos", "blocks.0.ln1.w", "blocks.0.ln1.b", "blocks.0.qkv.w", "blocks.0.qkv.b",
                     "blocks.0.proj.w", "blocks.0.proj.b", "blocks.0.ln2.w", "blocks.0.ln2.b", "blocks.0.fc.w",
                     "blocks.0.fc.b", "blocks.0.out.w", "blocks.0.out.b", "ln.w", "ln.b", "head.w"]


@pytest.mark.skipif(not __import__("os").path.isdir(
    __import__("os").path.join(__import__("os").path.dirname(__import__("os").path.dirname(__file__)),
                               "baseline", "_ref", "dtrain")), reason="reference not installed")
def test_init_and_loss_identical_to_reference_numpy_model():
    import os
    import sys
    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    sys.path.insert(0, ref)
    try:
        from dtrain.nn import GPT as RefGPT
        from dtrain.nn import GPTConfig as RefCfg
    finally:
        sys.path.remove(ref)
    cfg = dict(vocab=11, ctx=6, dim=8, heads=2, layers=2, dtype="float64")
    rm = RefGPT(RefCfg(**cfg), seed=3)
    om = GPT(GPTConfig(**cfg), seed=3)
    for (n1, p1), (n2, p2) in zip(rm.named_parameters(), om.named_parameters()):
        assert n1 == n2 and np.array_equal(p1.data, p2.detach().numpy())
    rng = np.random.default_rng(1)
    x, y = rng.integers(0, 11, (3, 6)), rng.integers(0, 11, (3, 6))
    _, rl = rm(x, y)
    _, ol = om(torch.as_tensor(x), torch.as_tensor(y))
    assert abs(float(rl.data) - ol.item()) < 1e-12
