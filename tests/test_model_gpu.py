"""The fused bf16 GPT (sm_100a kernels) against the fp32 reference math of the same model."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from dtrain_b200.models.gpt import GPT, GPTConfig  # noqa: E402
from dtrain_b200.ops import kernels as K  # noqa: E402
from dtrain_b200.ops.optim import AdamW  # noqa: E402

CFG = dict(vocab=512, ctx=128, dim=128, heads=2, layers=2)


def _batch(B=4, T=128, V=512, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(0, V, (B, T), generator=g).cuda(), torch.randint(0, V, (B, T), generator=g).cuda())


def test_fused_matches_fp32_reference():
    x, y = _batch()
    ref = GPT(GPTConfig(dtype="float32", **CFG), seed=3).cuda()
    _, lref = ref(x, y)
    lref.backward()
    fused = GPT(GPTConfig(dtype="bfloat16", **CFG), seed=3)
    fused.flatten("cuda")
    _, lf = fused(x, y)
    lf.backward()
    assert abs(lf.item() - lref.item()) < 2e-2
    for (n, pr), (_, pf) in zip(ref.named_parameters(), fused.named_parameters()):
        gr, gf = pr.grad.float(), pf.grad.float()
        err = (gr - gf).norm().item() / max(1e-12, gr.norm().item())
        assert err < 6e-2, f"{n}: relative grad error {err:.3g}"
        assert pf.grad.data_ptr() == fused.flat.grad_view(pf).data_ptr(), f"{n}: grad not in the flat buffer"
    assert K.device_status() == 0
    assert not fused.bad_token_ids_seen()


def _train(steps, seed=0):
    model = GPT(GPTConfig(dtype="bfloat16", **CFG), seed=seed)
    fp = model.flatten("cuda")
    opt = AdamW([fp.master], lr=3e-3, work=[fp.work])
    x, y = _batch(seed=1)
    losses = []
    for _ in range(steps):
        model.zero_grad()
        _, loss = model(x, y)
        loss.backward()
        sq = K.grad_sqnorm(fp.grad)
        opt.step([fp.grad], sq_norm=sq, max_norm=1.0)
        losses.append(loss.item())
    return losses, fp.master.clone()


def test_training_decreases_loss_and_is_deterministic():
    l1, p1 = _train(15)
    l2, p2 = _train(15)
    assert l1[-1] < l1[0] - 0.5, l1
    assert l1 == l2
    assert torch.equal(p1, p2), "bf16 training must be bit-reproducible"


def test_grad_accumulation_matches_single_batch():
    """Two half-batches accumulated == one full batch (up to bf16 rounding)."""
    x, y = _batch(B=8)
    m1 = GPT(GPTConfig(dtype="bfloat16", **CFG), seed=5)
    m1.flatten("cuda")
    _, l = m1(x, y)
    l.backward()
    full = torch.cat([p.grad.reshape(-1).float() for p in m1.parameters()])
    m2 = GPT(GPTConfig(dtype="bfloat16", **CFG), seed=5)
    m2.flatten("cuda")
    for sl in (slice(0, 4), slice(4, 8)):
        _, l = m2(x[sl], y[sl])
        (l * 0.5).backward()
    acc = torch.cat([p.grad.reshape(-1).float() for p in m2.parameters()])
    assert (acc - full).norm().item() / full.norm().item() < 2e-2


def test_init_matches_reference_initialiser():
    m = GPT(GPTConfig(dtype="bfloat16", **CFG), seed=7)
    rng = np.random.default_rng(7)
    tok = (rng.standard_normal((CFG["vocab"], CFG["dim"])) * 0.02).astype(np.float32)
    assert np.array_equal(m.tok.detach().numpy(), tok)


@pytest.mark.parametrize("accum", [1, 2])
def test_cuda_graph_step_matches_eager(accum):
    """--cuda-graph replays a captured forward+backward: parameters and losses must be
    bit-identical to launching every kernel eagerly (same kernels, same order)."""
    from dtrain_b200 import train as T
    from dtrain_b200.models.gpt import GPTConfig

    def run(graph):
        args = T.parse(["--mode", "single", "--dtype", "bfloat16", "--batch", "2", "--ctx", "128", "--dim", "128",
                        "--heads", "2", "--layers", "2", "--vocab", "512", "--data", "synthetic", "--lr", "3e-3",
                        "--accum", str(accum)] + (["--cuda-graph"] if graph else []))
        cfg = GPTConfig(vocab=512, ctx=128, dim=128, heads=2, layers=2, dtype="bfloat16")
        tr = T.Trainer(args, cfg, torch.device("cuda", 0), None)
        g = torch.Generator().manual_seed(3)
        losses = []
        for _ in range(4):
            batches = [[(torch.randint(0, 512, (2, 128), generator=g), torch.randint(0, 512, (2, 128), generator=g))]
                       for _ in range(accum)]
            losses.append(tr.step(batches))
        torch.cuda.synchronize()
        return losses, tr.model.flat.master.clone(), tr
    l_e, p_e, _ = run(False)
    l_g, p_g, tr = run(True)
    assert tr.graph_replays == 4 and tr.graph_launches > 0
    assert l_e == l_g
    assert torch.equal(p_e, p_g)
