"""NVLink collectives (csrc/comm.cu) across real processes, one GPU per rank.

Each test spawns W ranks (W = min(4, visible GPUs); skipped with fewer than 2),
bootstraps an NVLinkGroup through the rendezvous store and checks results
against fp64 sums, bit-identity across ranks, and bit-equality with the
reference's summation orders ("ring": chunk c summed from rank c cyclically;
"direct": rank order).  The failure test makes one rank skip a collective on
the host; its peer's device-side wait must time out into CommError with the
CUDA context still usable - no GPU fault or hang.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
WORLD = min(4, NGPU)
needs2 = pytest.mark.skipif(NGPU < 2, reason="needs at least 2 GPUs")


def _run(world, fn, *args, timeout=240):
    """Ranks as spawned processes, each with an NVLinkGroup on GPU ``rank`` (tests/harness.py)."""
    from harness import run_ranks
    return run_ranks(world, fn, *args, group="nvlink", timeout=20.0, wait_s=timeout)


def _inputs(rank, n, seed, dtype):
    return np.random.default_rng([seed, rank]).standard_normal(n).astype(np.float32 if dtype == "f32" else np.float32)


def _expected(world, n, seed, algo, dtype):
    from dtrain_b200.parallel.comm import partition
    xs = [_inputs(r, n, seed, dtype) for r in range(world)]
    if dtype == "bf16":
        xs = [torch.from_numpy(x).bfloat16().float().numpy() for x in xs]
    out = np.empty(n, np.float32)
    b = partition(n, world)
    for c in range(world):
        lo, hi = b[c], b[c + 1]
        first = c if algo == "ring" else 0
        acc = xs[first][lo:hi].copy()
        for k in range(1, world):
            acc = (acc + xs[(first + k) % world][lo:hi]).astype(np.float32)
        out[lo:hi] = acc
    return out


SIZES = [1, 7, 1000, 12345, (1 << 20) + 3]


def _allreduce_all(pg, algo, method, dtype):
    import torch
    res = []
    for i, n in enumerate(SIZES):
        x = torch.from_numpy(_inputs(pg.rank, n, i, dtype)).cuda()
        if dtype == "bf16":
            x = x.bfloat16()
        buf = pg.alloc(n, x.dtype)
        buf.copy_(x)
        pg.allreduce(buf, algo, method=method)
        y = x.clone()
        pg.allreduce(y, algo, method=method)  # staged path (tensor not peer-mapped)
        pg.synchronize()
        res.append((buf.float().cpu().numpy(), y.float().cpu().numpy()))
    return res


@needs2
@pytest.mark.parametrize("method", ["oneshot", "twoshot"])
@pytest.mark.parametrize("algo", ["ring", "direct"])
def test_allreduce_orders_and_bit_identity(method, algo):
    res = _run(WORLD, _allreduce_all, algo, method, "f32")
    for i, n in enumerate(SIZES):
        exp = _expected(WORLD, n, i, algo, "f32")
        for r in range(WORLD):
            inplace, staged = res[r][i]
            assert np.array_equal(inplace, exp), (r, n)
            assert np.array_equal(staged, exp), (r, n)


@needs2
def test_allreduce_bf16():
    res = _run(WORLD, _allreduce_all, "direct", "twoshot", "bf16")
    for i, n in enumerate(SIZES):
        exp = _expected(WORLD, n, i, "direct", "bf16")
        for r in range(WORLD):
            np.testing.assert_allclose(res[r][i][0], exp, rtol=1e-2, atol=1e-2)
            assert np.array_equal(res[r][i][0], res[0][i][0])


def _rs_ag_bcast(pg, n):
    import torch
    from dtrain_b200.parallel.comm import partition
    flat = pg.alloc(n, torch.float32)
    flat.copy_(torch.arange(n, dtype=torch.float32, device=flat.device) * (pg.rank + 1))
    mine = pg.reduce_scatter(flat).clone()
    b = partition(n, pg.world)
    full = pg.alloc(n, torch.float32)
    full[b[pg.rank]:b[pg.rank + 1]] = mine
    pg.all_gather(full)
    x = torch.full((1001,), float(pg.rank), device=flat.device)
    pg.broadcast(x, root=1)
    pg.barrier()
    pg.synchronize()
    return mine.cpu().numpy(), full.cpu().numpy(), x.cpu().numpy()


@needs2
@pytest.mark.parametrize("n", [3, 1001, 1 << 20])
def test_reduce_scatter_all_gather_broadcast(n):
    from dtrain_b200.parallel.comm import partition
    res = _run(WORLD, _rs_ag_bcast, n)
    total = np.arange(n, dtype=np.float32) * sum(range(1, WORLD + 1))
    b = partition(n, WORLD)
    for r, (mine, full, x) in enumerate(res):
        np.testing.assert_array_equal(mine, total[b[r]:b[r + 1]])
        np.testing.assert_array_equal(full, total)
        np.testing.assert_array_equal(x, np.ones(1001, np.float32))


def _skip_one(pg):
    import torch
    from dtrain_b200.utils.store import CommError
    x = pg.alloc(1 << 16, torch.float32)  # collective allocation, before the fault
    if pg.rank == 1:
        # never joins the collective (host-side fault); keeps its buffers mapped
        # until rank 0 has seen the timeout, then leaves
        pg._exchange("fault-test-done", b"")
        return "skipped"
    pg.timeout = 1.0
    pg.allreduce(x, "ring", method="twoshot")
    out = "no error"
    try:
        pg.synchronize()
    except CommError as e:
        # the context is still usable after the timed-out kernel returned
        y = torch.ones(10, device=x.device) * 2
        out = ("commerror", str(e)[:80], float(y.sum().item()))
    pg._exchange("fault-test-done", b"")
    return out


@needs2
def test_peer_that_never_arrives_gives_commerror_not_a_hang():
    res = _run(2, _skip_one)
    assert res[1] == "skipped"
    assert res[0][0] == "commerror" and res[0][2] == 20.0


def _abort_while_blocked(pg):
    import threading
    import time

    from dtrain_b200.utils.store import CommError
    x = pg.alloc(1 << 16, torch.float32)
    if pg.rank == 1:
        pg._exchange("abort-test-done", b"")  # never joins the collective
        return "skipped"
    pg.timeout = 60.0
    pg.allreduce(x, "ring", method="twoshot")
    t0 = time.monotonic()
    threading.Timer(1.0, pg.abort).start()  # e.g. the SIGTERM watcher of a stopping worker
    out = "no error"
    try:
        pg.synchronize()  # blocked on the waiting kernel until the abort lands
    except CommError as e:
        y = torch.ones(10, device=x.device) * 2
        out = ("commerror", "aborted" in str(e), time.monotonic() - t0, float(y.sum().item()))
    pg._exchange("abort-test-done", b"")
    return out


@needs2
def test_abort_ends_a_blocked_wait_long_before_the_timeout():
    res = _run(2, _abort_while_blocked)
    assert res[1] == "skipped"
    kind, aborted, waited, ysum = res[0]
    assert kind == "commerror" and aborted and ysum == 20.0
    assert waited < 20.0  # the kernel's own timeout is 60 s


def _desync(pg):
    import torch
    from dtrain_b200.utils.store import CommError
    x = pg.alloc(2048, torch.float32)
    x.fill_(1.0)
    pg.timeout = 5.0
    # same kernel shape (one CTA) but different sizes: a programming error on the host
    n = 1000 if pg.rank == 0 else 1008
    pg.allreduce(x[:n], "ring", method="twoshot")
    out = "no error"
    try:
        pg.synchronize()
    except CommError as e:
        y = torch.ones(4, device=x.device) * 3
        out = ("commerror", "desync" in str(e), float(y.sum().item()))
    pg._exchange("desync-test-done", b"")
    return out


@needs2
def test_desynchronised_collectives_give_commerror():
    """Ranks that issue different collectives at the same point are told so (the
    descriptor ring in the signal pads), without a hang and with a usable context."""
    res = _run(2, _desync)
    for r in res:
        assert r[0] == "commerror" and r[1] and r[2] == 12.0


def _zero_vs_ddp(pg):
    import torch
    from dtrain_b200.models.gpt import GPT, GPTConfig
    from dtrain_b200.ops import kernels as K
    from dtrain_b200.ops.optim import AdamW
    from dtrain_b200.parallel.ddp import DDP
    from dtrain_b200.parallel.zero import ZeroAdamW
    cfg = GPTConfig(vocab=512, ctx=128, dim=128, heads=2, layers=2, dtype="bfloat16")
    g = torch.Generator().manual_seed(1)
    batches = [(torch.randint(0, 512, (2 * pg.world, 128), generator=g),
                torch.randint(0, 512, (2 * pg.world, 128), generator=g)) for _ in range(3)]
    mine = [(x[2 * pg.rank:2 * pg.rank + 2].cuda(), y[2 * pg.rank:2 * pg.rank + 2].cuda()) for x, y in batches]
    # DDP + flat AdamW with on-device clipping
    md = GPT(cfg, seed=0)
    ddp = DDP(md, pg, bucket_mb=0.05)
    fp = md.flat
    opt = AdamW([fp.master], lr=3e-3, work=[fp.work])
    sq = torch.zeros(1, dtype=torch.float64, device=fp.master.device)
    for x, y in mine:
        md.zero_grad()
        _, loss = md(x, y)
        loss.backward()
        ddp.finish()
        K.grad_sqnorm(fp.grad, sq)
        opt.step([fp.grad], sq_norm=sq, max_norm=1.0)
    # ZeRO-1
    mz = GPT(cfg, seed=0)
    zero = ZeroAdamW(mz, pg, max_grad_norm=1.0, lr=3e-3)
    for x, y in mine:
        mz.zero_grad()
        _, loss = mz(x, y)
        loss.backward()
        zero.step()
    zero.gather_params()
    pg.synchronize()
    work_equal = bool(torch.equal(zero.fp.work, zero.fp.master.bfloat16()))
    return ((fp.master - zero.flat).abs().max().item(), fp.master.abs().max().item(),
            zero.state_bytes(), work_equal, zero.last_grad_norm)


@needs2
def test_zero1_matches_ddp_adamw_on_gpu():
    res = _run(2, _zero_vs_ddp)
    for diff, scale, state_bytes, work_equal, gnorm in res:
        assert diff <= 1e-5 * max(1.0, scale), diff
        assert work_equal, "bf16 working copy must equal the gathered fp32 masters"
        assert gnorm > 0
    from dtrain_b200.models.gpt import GPT, GPTConfig
    n = sum(p.numel() for p in GPT(GPTConfig(vocab=512, ctx=128, dim=128, heads=2, layers=2,
                                             dtype="bfloat16")).parameters())
    assert sum(r[2] for r in res) == 8 * n  # fp32 m and v, sharded exactly once across ranks


def _zero_variants(pg):
    import torch
    from dtrain_b200.models.gpt import GPT, GPTConfig
    from dtrain_b200.parallel.zero import ZeroAdamW
    cfg = GPTConfig(vocab=512, ctx=128, dim=256, heads=4, layers=2, dtype="bfloat16")
    g = torch.Generator().manual_seed(2)
    batches = [(torch.randint(0, 512, (2, 128), generator=g).cuda(), torch.randint(0, 512, (2, 128), generator=g).cuda())
               for _ in range(4 * pg.world)]
    mine = batches[pg.rank::pg.world]
    out = []
    # (weights gathered inside the forward GEMMs, reduce-scatter fused into the update kernel)
    for gather_gemm, fuse_rs in ((True, True), (False, True), (False, False)):
        m = GPT(cfg, seed=0)
        zero = ZeroAdamW(m, pg, max_grad_norm=1.0, gather_gemm=gather_gemm, fuse_rs=fuse_rs, lr=3e-3)
        assert (zero.plan is not None) == gather_gemm
        losses = []
        for i, (x, y) in enumerate(mine):
            if i % 2 == 0:
                m.zero_grad()
            _, loss = m(x, y)  # the second micro-step's forward finds the weights already gathered
            loss.backward()
            losses.append(float(loss.item()))
            if i % 2 == 1:
                zero.step()
        zero.gather_params()
        pg.synchronize()
        out.append((zero.flat.clone(), zero.fp.work.clone(), losses, zero.last_grad_norm))
    (f1, w1, l1, n1), (f2, w2, l2, n2), (f3, w3, l3, n3) = out
    return ((f1 - f2).abs().max().item(), f2.abs().max().item(), bool(torch.equal(w1, f1.bfloat16())),
            max(abs(a - b) for a, b in zip(l1, l2)), bool(torch.equal(f2, f3)), bool(torch.equal(w2, w3)),
            l2 == l3, n2 == n3)


@needs2
def test_zero1_gather_in_gemm_and_one_kernel_update_match_the_two_kernel_path():
    for diff, scale, work_ok, dloss, master_same, work_same, loss_same, norm_same in _run(2, _zero_variants):
        # all-gather inside the GEMMs vs inside the optimizer kernel (GEMM tiling differs: 1-SM vs 2-SM)
        assert diff <= 1e-5 * max(1.0, scale), diff
        assert work_ok
        assert dloss < 1e-3, dloss
        # reduce-scatter fused into the update kernel vs separate kernels: the same sums in the same order
        assert master_same and work_same and loss_same and norm_same


def _ddp_step(pg, bucket_mb, overlap=True):
    import torch
    from dtrain_b200.models.gpt import GPT, GPTConfig
    from dtrain_b200.parallel.ddp import DDP
    cfg = GPTConfig(vocab=512, ctx=128, dim=128, heads=2, layers=2, dtype="bfloat16")
    m = GPT(cfg, seed=0)
    ddp = DDP(m, pg, bucket_mb=bucket_mb, overlap=overlap)
    g = torch.Generator().manual_seed(0)
    xs = torch.randint(0, 512, (2 * pg.world, 128), generator=g)
    ys = torch.randint(0, 512, (2 * pg.world, 128), generator=g)
    x, y = xs[2 * pg.rank:2 * pg.rank + 2].cuda(), ys[2 * pg.rank:2 * pg.rank + 2].cuda()
    m.zero_grad()
    _, loss = m(x, y)
    loss.backward()
    ddp.finish()
    pg.synchronize()
    return torch.cat([p.grad.reshape(-1) for p in m.parameters()]).cpu().numpy()


@needs2
@pytest.mark.parametrize("bucket_mb,overlap", [(0.01, True), (25.0, True), (1.0, False)])
def test_ddp_gradients_match_single_process_and_agree_across_ranks(bucket_mb, overlap):
    from dtrain_b200.models.gpt import GPT, GPTConfig
    res = _run(2, _ddp_step, bucket_mb, overlap)
    assert np.array_equal(res[0], res[1]), "DDP gradients must be bit-identical across ranks"
    cfg = GPTConfig(vocab=512, ctx=128, dim=128, heads=2, layers=2, dtype="bfloat16")
    m = GPT(cfg, seed=0)
    m.flatten("cuda:0")
    g = torch.Generator().manual_seed(0)
    xs = torch.randint(0, 512, (4, 128), generator=g).cuda()
    ys = torch.randint(0, 512, (4, 128), generator=g).cuda()
    for sl in (slice(0, 2), slice(2, 4)):
        _, loss = m(xs[sl], ys[sl])
        (loss * 0.5).backward()
    ref = torch.cat([p.grad.reshape(-1) for p in m.parameters()]).cpu().numpy()
    err = np.linalg.norm(res[0] - ref) / np.linalg.norm(ref)
    assert err < 1e-2, err


def _ddp_trainer_runs(pg):
    """Three DDP training steps through the Trainer, for each way of synchronising
    the gradient: per-bucket all-reduces launched from the grad-ready hooks during
    backward (lean CTAs) or one flat all-reduce after it, each eager or captured
    in the CUDA graph with forward+backward."""
    import torch
    from dtrain_b200 import train as T
    from dtrain_b200.models.gpt import GPTConfig
    from dtrain_b200.utils.data import SyntheticData
    out = {}
    for algo, clip in (("direct", "0"), ("ring", "1.0")):
        for overlap in (True, False):
            for graph in (True, False):
                argv = ["--mode", "ddp", "--dtype", "bfloat16", "--batch", "2", "--ctx", "128", "--dim", "128",
                        "--heads", "2", "--layers", "2", "--vocab", "512", "--data", "synthetic", "--algo", algo,
                        "--clip", clip, "--bucket-mb", "0.05", "--lr", "3e-3"]
                argv += ([] if overlap else ["--no-overlap"]) + (["--cuda-graph"] if graph else [])
                a = T.parse(argv)
                cfg = GPTConfig(vocab=512, ctx=128, dim=128, heads=2, layers=2, dtype="bfloat16")
                tr = T.Trainer(a, cfg, pg.device, pg)
                data = SyntheticData(512)
                losses = [tr.step([[data.rank_batch(s, 0, 2, 128, 0, pg.rank, pg.world)]]) for s in range(3)]
                pg.synchronize()
                fp = tr.model.flat
                # numpy, not torch tensors: the queue would share CPU tensors by file descriptor
                out[(algo, overlap, graph)] = (fp.master.cpu().numpy().copy(), fp.grad.cpu().numpy().copy(),
                                               tr.grad_norm(), losses, len(tr.ddp.buckets))
                tr._graph = None
                torch.cuda.synchronize()
    return out


@needs2
def test_ddp_overlap_in_cuda_graph_matches_flat_allreduce_bit_for_bit():
    res = _run(2, _ddp_trainer_runs)
    for r in range(2):
        o = res[r]
        assert o[("direct", True, True)][4] > 4, "the test model must span several buckets"
        base = o[("direct", False, False)]
        # rank-order sums do not depend on how the gradient is cut into buckets
        for key in [("direct", True, True), ("direct", True, False), ("direct", False, True)]:
            assert np.array_equal(o[key][0], base[0]), key
            assert np.array_equal(o[key][1], base[1]), key
            assert o[key][3] == base[3], key
            assert abs(o[key][2] - base[2]) <= 1e-12 * base[2]
        # same buckets, same kernels: graph replay is bit-equal to eager launches, clip included
        for overlap in (True, False):
            a, b = o[("ring", overlap, True)], o[("ring", overlap, False)]
            assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2] and a[3] == b[3]
    for key in res[0]:
        assert np.array_equal(res[0][key][0], res[1][key][0]), ("ranks differ", key)
        assert np.array_equal(res[0][key][1], res[1][key][1]), ("ranks differ", key)
