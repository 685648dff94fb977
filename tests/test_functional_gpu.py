"""The reference-named functional ops on CUDA bf16 (kernel path) against fp32 torch math."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from dtrain_b200 import autograd as A  # noqa: E402


def _pair(*shape, scale=1.0):
    x = (torch.randn(*shape, device="cuda") * scale).bfloat16().requires_grad_()
    xf = x.detach().float().requires_grad_()
    return x, xf


def _rel(a, b):
    return (a.float() - b.float()).norm().item() / max(1e-12, b.float().norm().item())


def test_linear():
    x, xf = _pair(3, 100, 64)
    w, wf = _pair(64, 256, scale=0.1)
    b, bf = _pair(256)
    y = A.linear(x, w, b)
    yf = xf @ wf + bf
    assert _rel(y, yf) < 1e-2
    g = torch.randn_like(yf)
    y.backward(g.bfloat16())
    yf.backward(g)
    for a, r in ((x, xf), (w, wf), (b, bf)):
        assert a.grad.dtype == torch.bfloat16 and _rel(a.grad, r.grad) < 2e-2


def test_layer_norm_attention_cross_entropy():
    x, xf = _pair(4, 64, 768)
    w, wf = _pair(768)
    b, bf = _pair(768)
    y = A.layer_norm(x, w, b)
    yf = torch.nn.functional.layer_norm(xf, (768,), wf, bf, 1e-5)
    assert _rel(y, yf) < 1e-2
    y.backward(torch.ones_like(y))
    yf.backward(torch.ones_like(yf))
    assert _rel(x.grad, xf.grad) < 3e-2 and _rel(w.grad, wf.grad) < 2e-2

    q, qf = _pair(2, 3, 128, 64)
    k, kf = _pair(2, 3, 128, 64)
    v, vf = _pair(2, 3, 128, 64)
    o = A.causal_attention(q, k, v)
    mask = torch.triu(torch.ones(128, 128, dtype=torch.bool, device="cuda"), 1)
    of = torch.softmax(((qf @ kf.transpose(-1, -2)) / 8.0).masked_fill(mask, float("-inf")), -1) @ vf
    assert _rel(o, of) < 2e-2
    gg = torch.randn_like(of)
    o.backward(gg.bfloat16())
    of.backward(gg)
    for a, r in ((q, qf), (k, kf), (v, vf)):
        assert _rel(a.grad, r.grad) < 3e-2

    z, zf = _pair(4, 32, 1000, scale=3.0)
    t = torch.randint(0, 1000, (4, 32), device="cuda")
    loss = A.cross_entropy(z, t)
    lf = torch.nn.functional.cross_entropy(zf.reshape(-1, 1000), t.reshape(-1))
    assert abs(loss.item() - lf.item()) < 1e-2
    loss.backward()
    lf.backward()
    assert _rel(z.grad, zf.grad) < 2e-2
