"""NVSwitch multicast (NVLS) collectives across real processes, one GPU per rank.

The group maps its buffers through a multicast object (``NVLinkGroup(nvls=True)``);
``method="nvls"`` all-reduces with multimem.ld_reduce (sums formed in the switch)
and multimem.st (one store reaches every rank), and the NVLS reduce-scatter reduces
only this rank's partition through the switch.  Oracles: fp64 sums of the same
inputs (the switch's addition order is its own, so the bound is an fp32 rounding
bound, not bit-equality with the ring order), bit-identity across ranks, the same
bits on a repeated call, and the sums of squares the DDP clip uses.

No rank leaves while its memory is bound: the harness closes every NVLS group
(barrier, then unbind) on success and on error alike.  Skipped with fewer than two
GPUs or when the GPUs do not support multicast.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
WORLD = min(4, NGPU)
needs2 = pytest.mark.skipif(NGPU < 2, reason="needs at least 2 GPUs")


def _mc_supported():
    if NGPU < 2:
        return False
    from dtrain_b200.ops._ext import lib
    with torch.cuda.device(0):
        return bool(lib().mc_supported())


needs_mc = pytest.mark.skipif(not _mc_supported(), reason="GPUs without NVSwitch multicast")


def _run(world, fn, *args):
    from harness import run_ranks
    return run_ranks(world, fn, *args, group="nvls", timeout=20.0, wait_s=240.0)


def _inputs(rank, n, seed):
    return np.random.default_rng([seed, rank]).standard_normal(n).astype(np.float32)


# lengths with and without a partial 16-byte vector at the end; one past 1 Mi
SIZES = [1, 5, 4096, 12347, (1 << 20) + 6]


def _allreduce_nvls(pg, dtype):
    out = []
    for i, n in enumerate(SIZES):
        if dtype == torch.bfloat16 and n % 8:
            continue
        x = torch.from_numpy(_inputs(pg.rank, n, i)).cuda().to(dtype)
        buf = pg.alloc(n, dtype)
        buf.copy_(x)
        pg.allreduce(buf, method="nvls", scale=0.5)
        first = buf.float().cpu().numpy()
        buf.copy_(x)
        pg.allreduce(buf, method="nvls", scale=0.5)  # the same input again
        again = buf.float().cpu().numpy()
        y = x.clone()
        pg.allreduce(y, method="nvls", scale=0.5)  # staged: y is not peer-mapped
        pg.synchronize()
        out.append((n, first, again, y.float().cpu().numpy()))
    return out


@needs2
@needs_mc
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_nvls_allreduce_matches_fp64_and_ranks_agree(dtype):
    dt = torch.float32 if dtype == "f32" else torch.bfloat16
    res = _run(WORLD, _allreduce_nvls, dt)
    for k, (n, first, again, staged) in enumerate(res[0]):
        i = SIZES.index(n)
        xs = [_inputs(r, n, i) for r in range(WORLD)]
        if dt == torch.bfloat16:
            xs = [torch.from_numpy(x).bfloat16().double().numpy() for x in xs]
        exp = 0.5 * np.sum(np.stack(xs).astype(np.float64), axis=0)
        # fp32 sums in some order: a few ulps of the partial sums; bf16 outputs round once more
        tol = 1e-5 * WORLD if dt == torch.float32 else 1e-2
        np.testing.assert_allclose(first, exp, rtol=tol, atol=tol)
        np.testing.assert_array_equal(again, first)
        np.testing.assert_array_equal(staged, first)
        for r in range(1, WORLD):
            np.testing.assert_array_equal(res[r][k][1], first)


def _allreduce_sq(pg):
    n = 3 * 65536 + 4
    x = torch.from_numpy(_inputs(pg.rank, n, 7)).cuda()
    buf = pg.alloc(n, torch.float32)
    buf.copy_(x)
    blocks = 8
    stride = 16
    pad = pg.alloc(pg.world * stride, torch.float64)
    pg.allreduce(buf, method="nvls", scale=1.0 / pg.world, blocks=blocks, sq=(pad, 0, stride))
    total = torch.zeros(1, dtype=torch.float64, device=buf.device)
    pg.sq_total(pad, total, stride, 0, blocks)
    pg.synchronize()
    return float(total.item()), float((buf.double() ** 2).sum().item())


@needs2
@needs_mc
def test_nvls_allreduce_publishes_the_sum_of_squares():
    res = _run(WORLD, _allreduce_sq)
    for fused, direct in res:
        assert fused == res[0][0]
        assert abs(fused - direct) <= 1e-9 * direct


def _rs_nvls(pg, n):
    from dtrain_b200.parallel.comm import partition
    x = torch.from_numpy(_inputs(pg.rank, n, 3)).cuda()
    flat = pg.alloc(n, torch.float32)
    flat.copy_(x)
    parts = torch.zeros(64, dtype=torch.float64, device=flat.device)
    mine = pg.reduce_scatter(flat, scale=2.0, sq_parts=parts, method="nvls").clone()
    pg.synchronize()
    b = partition(n, pg.world)
    assert mine.numel() == b[pg.rank + 1] - b[pg.rank]
    return mine.cpu().numpy(), float(parts.sum().item())


@needs2
@needs_mc
@pytest.mark.parametrize("n", [3, 1001, (1 << 20) + 5])
def test_nvls_reduce_scatter(n):
    from dtrain_b200.parallel.comm import partition
    res = _run(WORLD, _rs_nvls, n)
    exp = 2.0 * np.sum(np.stack([_inputs(r, n, 3) for r in range(WORLD)]).astype(np.float64), axis=0)
    b = partition(n, WORLD)
    for r, (mine, sq) in enumerate(res):
        np.testing.assert_allclose(mine, exp[b[r]:b[r + 1]], rtol=1e-5 * WORLD, atol=1e-5 * WORLD)
        direct = float(np.sum(mine.astype(np.float64) ** 2))
        assert abs(sq - direct) <= 1e-9 * max(direct, 1.0)


def _unaligned_and_lean(pg):
    n = 50001
    x = torch.from_numpy(_inputs(pg.rank, n + 3, 11)).cuda()
    buf = pg.alloc(n + 3, torch.float32)
    buf.copy_(x)
    pg.allreduce(buf[1:n + 1], method="nvls")             # starts 4 bytes past a 16-byte boundary
    pg.allreduce(buf[n + 1:], method="nvls", lean=True)   # two elements, 128-thread CTAs
    pg.synchronize()
    return buf.cpu().numpy()


@needs2
@needs_mc
def test_nvls_allreduce_unaligned_slices_and_lean_ctas():
    n = 50001
    res = _run(WORLD, _unaligned_and_lean)
    xs = np.stack([_inputs(r, n + 3, 11) for r in range(WORLD)]).astype(np.float64)
    exp = xs.sum(axis=0)
    exp[0] = xs[0, 0]  # element 0 was not part of either call
    tol = 1e-5 * WORLD
    for r in range(WORLD):
        np.testing.assert_allclose(res[r][1:], exp[1:], rtol=tol, atol=tol)
        assert res[r][0] == np.float32(_inputs(r, n + 3, 11)[0])
        np.testing.assert_array_equal(res[r][1:], res[0][1:])


def _ddp_steps(pg, method):
    from dtrain_b200.models.gpt import GPT, GPTConfig
    from dtrain_b200.ops.optim import AdamW
    from dtrain_b200.parallel.ddp import DDP
    cfg = GPTConfig(vocab=256, ctx=128, dim=128, heads=2, layers=2, dtype="bfloat16")
    g = torch.Generator().manual_seed(3)
    model = GPT(cfg, seed=0)
    ddp = DDP(model, pg, bucket_mb=0.02, method=method)
    fp = model.flat
    opt = AdamW([fp.master], lr=3e-3, work=[fp.work])
    for _ in range(3):
        x = torch.randint(0, 256, (2 * pg.world, 128), generator=g)[2 * pg.rank:2 * pg.rank + 2].cuda()
        y = torch.randint(0, 256, (2 * pg.world, 128), generator=g)[2 * pg.rank:2 * pg.rank + 2].cuda()
        model.zero_grad()
        _, loss = model(x, y)
        loss.backward()
        ddp.finish()
        opt.step([fp.grad], sq_norm=ddp.sq_norm, max_norm=1.0)
    pg.synchronize()
    return fp.master.cpu().numpy(), float(ddp.sq_norm.item())


@needs2
@needs_mc
def test_ddp_with_nvls_buckets_tracks_the_two_shot_path():
    nv = _run(WORLD, _ddp_steps, "nvls")
    ts = _run(WORLD, _ddp_steps, "twoshot")
    for r in range(WORLD):
        np.testing.assert_array_equal(nv[r][0], nv[0][0])  # ranks agree bit for bit
        np.testing.assert_allclose(nv[r][0], ts[r][0], rtol=1e-3, atol=1e-4)
        assert abs(nv[r][1] - ts[r][1]) <= 1e-3 * ts[r][1]
