"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op.

Shapes include odd sizes (rows not multiples of the tile, K tails, T not a
multiple of 64) so the edge handling of each kernel is exercised.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from dtrain_b200.ops import kernels as K  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.manual_seed(0)
    yield
    assert K.device_status() == 0


def _rel(a, b):
    return (a.float() - b.float()).abs().max().item() / max(1e-6, b.float().abs().max().item())


GEMM_SHAPES = [(128, 256, 64), (300, 264, 200), (1024, 768, 768), (513, 2304, 768), (64, 128, 1000),
               (4096, 3072, 768)]


@pytest.mark.parametrize("M,N,K_", GEMM_SHAPES)
@pytest.mark.parametrize("layout", ["nn", "nt", "tn"])
@pytest.mark.parametrize("bn", [0, 128, 256, 512])  # 0: the heuristic's choice; 512: 2-SM pair tiles
def test_gemm_layouts(M, N, K_, layout, bn):
    dev = "cuda"
    if layout == "tn":  # M is the contiguous dimension of the stored A: keep rows 16-byte aligned
        M = (M + 7) // 8 * 8
    x = torch.randn(M, K_, device=dev).bfloat16()
    w = torch.randn(K_, N, device=dev).bfloat16()
    ref = x.float() @ w.float()
    if layout == "nn":      # forward: A [M,K], B [K,N]
        out = K.gemm(x, w, force_bn=bn)
    elif layout == "nt":    # dX: A [M,K], B stored [N,K]
        out = K.gemm(x, w.t().contiguous(), b_trans=True, force_bn=bn)
    else:                   # dW: A stored [K,M], B [K,N]
        out = K.gemm(x.t().contiguous(), w, a_trans=True, epi=K.EPI_F32, force_bn=bn)
    torch.cuda.synchronize()
    assert _rel(out, ref) < 1e-2, layout


@pytest.mark.parametrize("splits", [2, 3])
def test_gemm_splitk_f32_accumulate(splits):
    M, N, K_ = 768, 768, 4096
    x = torch.randn(K_, M, device="cuda").bfloat16()
    g = torch.randn(K_, N, device="cuda").bfloat16()
    base = torch.randn(M, N, device="cuda")
    out = base.clone()
    K.gemm(x, g, out, a_trans=True, epi=K.EPI_F32, accumulate=True, force_splits=splits)
    ref = base + x.float().t() @ g.float()
    assert _rel(out, ref) < 1e-3
    out2 = base.clone()
    K.gemm(x, g, out2, a_trans=True, epi=K.EPI_F32, accumulate=True, force_splits=splits)
    assert torch.equal(out, out2), "split-K reduction must be deterministic"


def test_gemm_epilogues():
    M, N, K_ = 1000, 3072, 768
    x = torch.randn(M, K_, device="cuda").bfloat16()
    w = (torch.randn(K_, N, device="cuda") * 0.05).bfloat16()
    b = torch.randn(N, device="cuda").bfloat16()
    r = torch.randn(M, N, device="cuda").bfloat16()
    acc = x.float() @ w.float()
    y = K.gemm(x, w, bias=b, resid=r)
    assert _rel(y, acc + b.float() + r.float()) < 1e-2
    pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    act = K.gemm(x, w, epi=K.EPI_GELU, bias=b, aux=pre)
    pre_ref = acc + b.float()
    assert _rel(pre, pre_ref) < 1e-2
    assert _rel(act, torch.nn.functional.gelu(pre.float(), approximate="tanh")) < 1e-2
    dg = K.gemm(x, w, epi=K.EPI_DGELU, aux=pre)
    pf = pre.float().requires_grad_()
    torch.nn.functional.gelu(pf, approximate="tanh").backward(acc)
    assert _rel(dg, pf.grad) < 2e-2
    y2 = K.gemm(x, w, alpha=0.5)
    assert _rel(y2, 0.5 * acc) < 1e-2


def test_gemm_deterministic():
    x = torch.randn(2048, 768, device="cuda").bfloat16()
    w = torch.randn(768, 2304, device="cuda").bfloat16()
    a = K.gemm(x, w)
    b = K.gemm(x, w)
    assert torch.equal(a, b)


@pytest.mark.parametrize("rows,C", [(37, 64), (1024, 768), (300, 1024), (64, 2048), (129, 264), (70, 1288)])
def test_layernorm(rows, C):
    x = torch.randn(rows, C, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(C, device="cuda")).bfloat16()
    b = (0.1 * torch.randn(C, device="cuda")).bfloat16()
    y, mu, rs = K.layernorm_fwd(x, w, b)
    xf = x.float().requires_grad_()
    wf = w.float().requires_grad_()
    bf = b.float().requires_grad_()
    yr = torch.nn.functional.layer_norm(xf, (C,), wf, bf, 1e-5)
    assert _rel(y, yr) < 1e-2
    dy = torch.randn(rows, C, device="cuda").bfloat16()
    dres = torch.randn(rows, C, device="cuda").bfloat16()
    yr.backward(dy.float())
    dw = torch.empty(C, device="cuda")
    db = torch.empty(C, device="cuda")
    dsum = torch.empty(C, device="cuda")
    dx = K.layernorm_bwd(dy, x, w, mu, rs, dres, dw, db, dres_sum=dsum)
    assert _rel(dx, xf.grad + dres.float()) < 2e-2
    assert _rel(dw, wf.grad) < 1e-3
    assert _rel(db, bf.grad) < 1e-3
    assert _rel(dsum, dres.float().sum(0)) < 1e-4  # column sums of the residual gradient
    dx2 = K.layernorm_bwd(dy, x, w, mu, rs, dres, dw.clone(), db.clone(), dres_sum=dsum.clone())
    assert torch.equal(dx, dx2)


def test_bias_grad():
    g = torch.randn(3000, 2304, device="cuda").bfloat16()
    db = torch.empty(2304, device="cuda")
    K.bias_grad(g, db)
    assert _rel(db, g.float().sum(0)) < 1e-4


def _attn_ref(qkv, B, T, H, D):
    q, k, v = qkv.float().view(B, T, 3, H, D).permute(2, 0, 3, 1, 4)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(D)
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=qkv.device), 1)
    p = torch.softmax(s.masked_fill(mask, float("-inf")), -1)
    return (p @ v).transpose(1, 2).reshape(B * T, H * D)


@pytest.mark.parametrize("legacy", [False, True])
@pytest.mark.parametrize("B,T,H,D", [(2, 64, 2, 64), (1, 100, 3, 64), (2, 256, 4, 64), (1, 384, 2, 64),
                                     (1, 1024, 2, 64), (1, 192, 2, 128)])
def test_attention(B, T, H, D, legacy):
    qkv = torch.randn(B * T, 3 * H * D, device="cuda").bfloat16()
    out, lse = K.attn_fwd(qkv, B, T, H, D, legacy=legacy)
    qf = qkv.float().requires_grad_()
    ref = _attn_ref(qf, B, T, H, D)
    assert _rel(out, ref) < 2e-2
    dout = torch.randn(B * T, H * D, device="cuda").bfloat16()
    ref.backward(dout.float())
    dqkv = K.attn_bwd(qkv, out, dout, lse, B, T, H, D, legacy=legacy)
    g = qf.grad.view(B * T, 3, H * D)
    d = dqkv.view(B * T, 3, H * D)
    for i, name in enumerate("qkv"):
        assert _rel(d[:, i], g[:, i]) < 3e-2, name
    dqkv2 = K.attn_bwd(qkv, out, dout, lse, B, T, H, D, legacy=legacy)
    assert torch.equal(dqkv, dqkv2), "attention backward must be deterministic"


def test_kernels_from_a_fresh_host_thread():
    """Autograd runs every backward on its own worker thread, which starts with no
    CUDA context bound; TMA descriptor encoding (GEMM, tcgen05 attention) must work
    there and give the same bits as on the main thread."""
    import threading
    x = torch.randn(300, 64, device="cuda").bfloat16()
    w = torch.randn(256, 64, device="cuda").bfloat16()
    qkv = torch.randn(128, 3 * 2 * 64, device="cuda").bfloat16()
    main = (K.gemm(x, w, b_trans=True), K.attn_fwd(qkv, 1, 128, 2, 64)[0])
    got = {}

    def body():
        try:
            got["r"] = (K.gemm(x, w, b_trans=True), K.attn_fwd(qkv, 1, 128, 2, 64)[0])
            torch.cuda.synchronize()
        except BaseException as e:  # noqa: BLE001
            got["e"] = e

    t = threading.Thread(target=body)
    t.start()
    t.join()
    assert "e" not in got, got.get("e")
    for a, b in zip(main, got["r"]):
        assert torch.equal(a, b)


def test_embedding():
    B, T, V, C = 4, 64, 1000, 256
    idx = torch.randint(0, V, (B, T), device="cuda")
    idx[0, :10] = 7  # repeated ids
    tok = torch.randn(V, C, device="cuda").bfloat16()
    pos = torch.randn(T, C, device="cuda").bfloat16()
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = K.embed_fwd(idx, tok, pos, bad)
    assert _rel(x, tok.float()[idx] + pos.float()[None]) < 1e-2
    dx = torch.randn(B, T, C, device="cuda").bfloat16()
    dtok = torch.empty(V, C, device="cuda")
    dpos = torch.empty(T, C, device="cuda")
    K.embed_bwd(idx, dx, dtok, dpos)
    ref_tok = torch.zeros(V, C, device="cuda").index_add_(0, idx.reshape(-1), dx.float().reshape(-1, C))
    assert _rel(dtok, ref_tok) < 1e-4
    assert _rel(dpos, dx.float().sum(0)) < 1e-4
    assert bad.item() == 0
    again = torch.empty_like(dtok)
    K.embed_bwd(idx, dx, again, torch.empty_like(dpos))
    assert torch.equal(again, dtok)  # fixed summation order: the same bits every time


@pytest.mark.parametrize("n,V", [(1, 65), (1000, 65), (16384, 50304), (70001, 50304), (5000, 70000)])
def test_id_sort_is_stable_and_matches_torch(n, V):
    """The embedding backward's radix sort (2 passes below 65536 ids, 3 above) against
    torch's stable sort: same sorted ids and the same positions for equal ids."""
    g = torch.Generator(device="cuda").manual_seed(n)
    idx = torch.randint(0, V, (n,), device="cuda", generator=g)
    idx[: n // 3] = idx[0]  # a long run of one id
    ids, perm = K.sort_ids(idx, V)
    want_ids, want_perm = torch.sort(idx, stable=True)
    assert torch.equal(ids, want_ids)
    assert torch.equal(perm, want_perm)


@pytest.mark.parametrize("rows,V", [(64, 65), (256, 50304), (33, 1000)])
def test_cross_entropy(rows, V):
    z = (3 * torch.randn(rows, V, device="cuda")).bfloat16()
    t = torch.randint(0, V, (rows,), device="cuda")
    loss, lse = K.xent_fwd(z, t)
    zf = z.float().requires_grad_()
    ref = torch.nn.functional.cross_entropy(zf, t)
    assert abs(loss.item() - ref.item()) < 1e-3 * max(1.0, abs(ref.item()))
    ref.backward(torch.tensor(2.0, device="cuda"))
    zz = z.clone()
    K.xent_bwd(zz, t, lse, torch.tensor([2.0], device="cuda"))
    assert _rel(zz, zf.grad) < 2e-2


@pytest.mark.parametrize("rows,V,K_", [(16384, 50304, 768), (300, 50304, 256), (256, 512, 128), (200, 128, 64),
                                       (1000, 1000, 192)])
def test_head_gemm_with_fused_cross_entropy_statistics(rows, V, K_):
    """LM head GEMM whose epilogue emits the softmax partials (gemm_xent) vs the plain
    GEMM followed by the streaming cross-entropy kernel and an fp32 torch reference."""
    x = torch.randn(rows, K_, device="cuda").bfloat16()
    w = (torch.randn(K_, V, device="cuda") * (2.0 / K_ ** 0.5)).bfloat16()
    t = torch.randint(0, V, (rows,), device="cuda")
    logits, loss, lse = K.gemm_xent(x, w, t)
    plain = K.gemm(x, w)
    torch.cuda.synchronize()
    assert torch.equal(logits, plain), "the fused epilogue must store the same logits"
    loss2, lse2 = K.xent_fwd(plain, t)
    ref_lse = torch.logsumexp(plain.float(), -1)
    ref = torch.nn.functional.cross_entropy(plain.float(), t)
    assert (lse - ref_lse).abs().max().item() < 1e-4 * max(1.0, ref_lse.abs().max().item())
    assert (lse - lse2).abs().max().item() < 1e-4 * max(1.0, ref_lse.abs().max().item())
    assert abs(loss.item() - ref.item()) < 1e-4 * max(1.0, abs(ref.item()))
    # deterministic: a second call gives the same bits
    _, loss3, lse3 = K.gemm_xent(x, w, t)
    assert torch.equal(lse3, lse) and torch.equal(loss3, loss)


def test_adamw_and_norm():
    n = 100003
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    sq = K.grad_sqnorm(g)
    assert abs(sq.item() - (g.double() ** 2).sum().item()) < 1e-9 * sq.item()
    pr, mr, vr = p.double().clone(), torch.zeros(n, dtype=torch.float64, device="cuda"), torch.zeros(
        n, dtype=torch.float64, device="cuda")
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.95, 1e-8, 0.1
    max_norm = 1.0
    for t in (1, 2):
        K.adamw_step(p, g, m, v, p16, lr, b1, b2, eps, wd, t, sq, max_norm)
        cs = max_norm / (math.sqrt(sq.item()) + 1e-6)
        gg = g.double() * cs
        mr = b1 * mr + (1 - b1) * gg
        vr = b2 * vr + (1 - b2) * gg * gg
        pr -= lr * (wd * pr)
        pr -= lr * (mr / (1 - b1 ** t)) / (torch.sqrt(vr / (1 - b2 ** t)) + eps)
    assert (p.double() - pr).abs().max().item() < 1e-5
    assert torch.equal(p16, p.bfloat16())
    sq2 = K.grad_sqnorm(g)
    assert torch.equal(sq, sq2)
