"""This framework against torch.distributed on CPU ranks (gloo), float64.

Pinned behaviours (the reference's torch cross-check, tests/test_torch_crosscheck.py
there): the ring all-reduce stays within the error bound of a (W-1)-term sum and
matches gloo bit for bit at W=2; DDP with AdamW or SGD follows torch DDP step by
step (gradients ~1e-14 relative, parameters and loss ~1e-13); ZeRO-1 follows
ZeroRedundancyOptimizer and both keep one copy of the AdamW state in total;
checkpoint/exit/resume is bit-identical in both libraries; AdamW alone matches
torch.optim.AdamW.  Every rank runs both libraries side by side on the same
weights and batches (benchmarks/torch_crosscheck.py).
"""
import json

import numpy as np
import pytest
from harness import launch_script

torch = pytest.importorskip("torch")
if not torch.distributed.is_available() or not torch.distributed.is_gloo_available():
    pytest.skip("torch.distributed with gloo is not available", allow_module_level=True)

MODEL = ["--dim", "24", "--heads", "2", "--layers", "2", "--ctx", "12", "--batch", "3", "--dtype", "float64"]


@pytest.fixture
def crosscheck(tmp_path, corpus):
    """Runs torch_crosscheck.py and returns (per-step rows, meta, final parameters)."""

    def run(world, tag, *flags):
        prefix = tmp_path / tag
        launch_script(tmp_path, world, "torch_crosscheck.py",
                      ["--data", corpus, *MODEL, "--out", str(prefix), *flags], tag)
        rows = [json.loads(line) for line in open(f"{prefix}.jsonl")]
        meta = json.load(open(f"{prefix}.meta.json"))
        return rows, meta, np.load(f"{prefix}.npz")

    return run


@pytest.mark.parametrize("world", [2, 3])
def test_ring_allreduce_agrees_with_gloo(tmp_path, world):
    out = tmp_path / "check.json"
    launch_script(tmp_path, world, "torch_allreduce.py", ["--no-speed", "--n-check", "30000", "--out", str(out)],
                  "ar")
    check = json.load(open(out))["check"]
    for dt, eps in (("float32", 2.0 ** -23), ("float64", 2.0 ** -52)):
        c = check[dt]
        bound = 2 * (world - 1) * eps * c["max_abs_value"]
        assert c["max_abs_err_dtrain"] <= bound, (dt, c)
        assert c["max_abs_err_gloo"] <= bound, (dt, c)
        if world == 2:  # two addends: every order gives the same bits
            assert c["bit_identical_frac"] == 1.0


@pytest.mark.parametrize("opt", ["adamw", "sgd"])
def test_ddp_follows_torch_ddp_step_by_step(crosscheck, opt):
    rows, _, _ = crosscheck(2, f"ddp-{opt}", "--mode", "ddp", "--steps", "4", "--opt", opt)
    assert len(rows) == 4
    for r in rows:
        assert r["grad_maxabs_diff"] <= 1e-14 * max(1.0, r["grad_maxabs"]), r
        assert r["param_maxabs_diff"] <= 1e-13, r
        assert r["loss_abs_diff"] <= 1e-13, r


def test_zero1_follows_zero_redundancy_optimizer(crosscheck):
    rows, meta, _ = crosscheck(2, "zero", "--mode", "zero", "--steps", "4")
    assert all(r["param_maxabs_diff"] <= 1e-13 for r in rows), rows
    n = meta["n_params"]
    per_rank = meta["state_bytes_per_rank"]
    assert sum(s["torch_state_bytes"] for s in per_rank) == 16 * n  # two fp64 moments, sharded once
    assert sum(s["dtrain_state_bytes"] for s in per_rank) == 16 * n


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_resume_is_bit_identical_in_both_libraries(crosscheck, tmp_path, mode):
    flags = ["--mode", mode, "--steps", "6", "--k", "3"]
    _, _, whole = crosscheck(2, f"{mode}-whole", *flags, "--phase", "full")
    ck = str(tmp_path / f"ck-{mode}")
    crosscheck(2, f"{mode}-first", *flags, "--phase", "first", "--ckpt", ck)
    _, _, resumed = crosscheck(2, f"{mode}-resumed", *flags, "--phase", "resume", "--ckpt", ck)
    assert np.array_equal(whole["dtrain"], resumed["dtrain"])
    assert np.array_equal(whole["torch"], resumed["torch"])
    assert np.abs(resumed["dtrain"] - resumed["torch"]).max() <= 1e-13


def test_adamw_alone_matches_torch_adamw():
    from dtrain_b200.ops.optim import AdamW
    rng = np.random.default_rng(5)
    start = rng.standard_normal(3000)
    mine, ref = torch.from_numpy(start.copy()), torch.from_numpy(start.copy()).requires_grad_()
    hp = dict(lr=2e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    opt_mine, opt_ref = AdamW([mine], **hp), torch.optim.AdamW([ref], **hp)
    for _ in range(12):
        g = rng.standard_normal(start.size) * 10.0 ** rng.uniform(-7, 0, start.size)
        opt_mine.step([torch.from_numpy(g.copy())])
        ref.grad = torch.from_numpy(g.copy())
        opt_ref.step()
    assert float((mine - ref.detach()).abs().max()) <= 1e-14
