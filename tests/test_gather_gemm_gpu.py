"""The forward GEMM with the ZeRO-1 weight all-gather fused in (``gemm_gather``).

One GPU emulates W ranks: every "rank" owns a separate bf16 copy of a flat
parameter buffer in which only its own partition (``partition(n, W)``) holds the
true values and the rest is stale.  The kernel, called as rank ``r``, must pull
the other partitions of the weight from the other copies (plain loads, no
cross-kernel waits: the other copies are already complete), leave the weight
complete in rank r's copy, and compute the same product as a plain PyTorch fp32
matmul of the true weight.  A second call in the same generation must not copy.
"""
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

from dtrain_b200.ops import kernels as K  # noqa: E402
from dtrain_b200.parallel.comm import partition  # noqa: E402
from dtrain_b200.parallel.zero import GS_GEN, GS_SITES  # noqa: E402

STALE = 7.0


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    yield
    assert K.device_status() == 0


def _rel(a, b):
    return (a.float() - b.float()).abs().max().item() / max(1e-6, b.float().abs().max().item())


def _setup(world, nflat, woff, K_, N, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    truth = torch.randn(nflat, device="cuda", generator=g).bfloat16()
    bounds = partition(nflat, world)
    copies = []
    for r in range(world):
        c = torch.full((nflat,), STALE, dtype=torch.bfloat16, device="cuda")
        c[bounds[r]:bounds[r + 1]] = truth[bounds[r]:bounds[r + 1]]
        copies.append(c)
    return truth, copies


def _plan(copies, rank, woff, nflat, state, site=0):
    peers = [c.data_ptr() + 2 * woff for c in copies]
    return SimpleNamespace(rank=rank, nflat=nflat, state=state, sites={"w": (site, woff, peers)})


# (world, rank, M, N, K, extra flat elements before / after the weight, epilogue)
CASES = [
    (2, 0, 512, 2304, 768, 1000, 333, "bias"),
    (2, 1, 300, 128, 200, 8, 7, "plain"),
    (4, 2, 1024, 3072, 768, 96, 5, "gelu"),
    (8, 5, 256, 768, 3072, 40, 13, "resid"),
    (2, 0, 256, 50304, 768, 768, 0, "plain"),
]


@pytest.mark.parametrize("world,rank,M,N,K_,pre,post,epi", CASES)
def test_gather_gemm_pulls_peer_partitions_and_matches_fp32(world, rank, M, N, K_, pre, post, epi):
    woff = pre  # flat offset of the weight (multiple of 8: 16-byte aligned rows)
    nflat = pre + K_ * N + post
    truth, copies = _setup(world, nflat, woff, K_, N, seed=world * 100 + rank)
    state = torch.zeros(GS_SITES + 1, dtype=torch.int32, device="cuda")
    state[GS_GEN] = 5
    plan = _plan(copies, rank, woff, nflat, state)
    w_true = truth[woff:woff + K_ * N].view(K_, N)
    w_local = copies[rank][woff:woff + K_ * N].view(K_, N)
    x = torch.randn(M, K_, device="cuda").bfloat16()
    bias = torch.randn(N, device="cuda").bfloat16()
    resid = torch.randn(M, N, device="cuda").bfloat16()
    kw = {}
    if epi == "bias":
        kw = dict(bias=bias)
    elif epi == "resid":
        kw = dict(bias=bias, resid=resid)
    elif epi == "gelu":
        kw = dict(epi=K.EPI_GELU, bias=bias, aux=torch.empty(M, N, dtype=torch.bfloat16, device="cuda"))

    def ref(w):
        y = x.float() @ w.float()
        if epi in ("bias", "gelu", "resid"):
            y = y + bias.float()
        if epi == "resid":
            y = y + resid.float()
        return torch.nn.functional.gelu(y, approximate="tanh") if epi == "gelu" else y

    before = [c.clone() for c in copies]
    out = K.gemm_gather(x, w_local, plan, "w", **kw)
    torch.cuda.synchronize()
    assert torch.equal(w_local, w_true), "the weight must be complete in this rank's copy"
    mine = copies[rank]
    assert torch.equal(mine[:woff], before[rank][:woff]) and torch.equal(mine[woff + K_ * N:],
                                                                          before[rank][woff + K_ * N:])
    assert all(torch.equal(copies[r], before[r]) for r in range(world) if r != rank), "peers are read-only"
    assert _rel(out, ref(w_true)) < 2e-2
    st = state.cpu()
    assert int(st[GS_SITES]) == 5, "the site must record the generation it gathered"
    assert int(st[:GS_GEN].abs().sum()) == 0, "counters, ticket and done count must be reset for the next launch"

    # same generation: no copy (stale peers are not read), same result bit for bit
    for r in range(world):
        if r != rank:
            copies[r].fill_(STALE)
    out2 = K.gemm_gather(x, w_local, plan, "w", **kw)
    torch.cuda.synchronize()
    assert torch.equal(out2, out)
    assert torch.equal(w_local, w_true)

    # next generation: new values in the owners' partitions are pulled again
    truth2, copies2 = _setup(world, nflat, woff, K_, N, seed=7 + rank)
    for r in range(world):
        copies[r].copy_(copies2[r])
    state[GS_GEN] = 6
    out3 = K.gemm_gather(x, w_local, plan, "w", **kw)
    torch.cuda.synchronize()
    w2 = truth2[woff:woff + K_ * N].view(K_, N)
    assert torch.equal(w_local, w2)
    assert _rel(out3, ref(w2)) < 2e-2
    assert int(state[GS_SITES].item()) == 6


def test_gather_gemm_equals_plain_gemm_when_nothing_to_pull():
    M, N, K_ = 384, 2304, 768
    nflat = K_ * N
    truth, copies = _setup(2, nflat, 0, K_, N, seed=3)
    copies[0].copy_(truth)
    state = torch.zeros(GS_SITES + 1, dtype=torch.int32, device="cuda")  # generation 0 == site 0
    plan = _plan(copies, 0, 0, nflat, state)
    x = torch.randn(M, K_, device="cuda").bfloat16()
    w = copies[0].view(K_, N)
    out = K.gemm_gather(x, w, plan, "w")
    ref = K.gemm(x, w)  # same tiling choice (2-SM pair tiles) as the gather kernel
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
