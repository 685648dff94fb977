"""Per-kernel timings of the sm_100a kernels on the GPT-2-small training shapes.

    python benchmarks/kernel_bench.py [--only gemm,gather,headxent,attn,ln,xent,adamw] [--iters 20]

Each kernel is timed with CUDA events on the current stream after warm-up, with
a synchronize on both sides and a cold L2 (see ``timeit``); the median over
``--iters`` launches is reported
with the achieved TFLOP/s (or GB/s) and the fraction of the measured peak from
MEASURED_PEAKS.json (bf16 burst GEMM, HBM copy) when that file exists.
"""
import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from dtrain_b200.ops import kernels as K  # noqa: E402


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["bf16_tflops"], d["hbm_gbs"], "of measured"
    return 1590.0, 6650.0, "of fallback"


_FLUSH = None


def timeit(fn, iters):
    """Median device time of one call, in microseconds, with a cold L2.

    Before every timed call a 256 MiB buffer is written (flushing the 126 MB L2);
    that kernel also keeps the GPU busy while the host enqueues the timed call, so
    the events bracket device work only, not host launch latency.
    """
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _FLUSH.fill_(1.0)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2] * 1e3  # us


def gather_cases(a, rep, N, C, V):
    """ZeRO-1 forward GEMM with the weight's all-gather fused in (``gemm_gather``).

    One GPU emulates ``--gather-world`` ranks: each rank's copy of the weight is a
    separate buffer on this GPU holding only its own partition, so the pulled
    bytes come from local HBM here, not over NVLink.  Reported per shape:
    ``gather_pull`` (the call that pulls (W-1)/W of the weight; every timed call
    uses a fresh call site so it pulls), ``gather_nopull`` (same kernel, weight
    already gathered), ``gemm_plain`` (the ordinary GEMM's own tiling choice) and
    ``copy_then_gemm`` (the unfused sequence: copy the other partitions, then GEMM).
    """
    from types import SimpleNamespace

    from dtrain_b200.parallel.comm import partition
    from dtrain_b200.parallel.zero import GS_GEN, GS_SITES

    W = a.gather_world
    shapes = {"qkv": (C, 3 * C), "proj": (C, C), "fc": (C, 4 * C), "out": (4 * C, C), "head": (C, V)}
    for name in a.gather_shapes.split(","):
        kin, kout = shapes[name]
        n = kin * kout
        bounds = partition(n, W)
        truth = (torch.randn(n, device="cuda") * 0.02).bfloat16()
        copies = [truth.clone() for _ in range(W)]
        x = torch.randn(N, kin, device="cuda").bfloat16()
        nsites = a.iters + 8
        state = torch.zeros(GS_SITES + nsites, dtype=torch.int32, device="cuda")
        state[GS_GEN] = 1
        peers = [c.data_ptr() for c in copies]
        plan = SimpleNamespace(rank=0, nflat=n, state=state, sites={i: (i, 0, peers) for i in range(nsites)})
        w = copies[0].view(kin, kout)
        f = 2.0 * N * kin * kout
        pulled = (n - (bounds[1] - bounds[0])) * 2
        it = iter(range(nsites))
        rep(f"gather_pull_{name}_w{W}", timeit(lambda: K.gemm_gather(x, w, plan, next(it)), a.iters), f, pulled)
        state[GS_SITES:] = 1
        rep(f"gather_nopull_{name}_w{W}", timeit(lambda: K.gemm_gather(x, w, plan, 0), a.iters), f)
        rep(f"gemm_plain_{name}", timeit(lambda: K.gemm(x, w), a.iters), f)
        flat0 = copies[0]

        def unfused():
            for r in range(1, W):
                flat0[bounds[r]:bounds[r + 1]].copy_(copies[r][bounds[r]:bounds[r + 1]])
            return K.gemm(x, w)
        rep(f"copy_then_gemm_{name}_w{W}", timeit(unfused, a.iters), f, pulled)
        del truth, copies, x


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,attn,ln,xent,adamw")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--gather-world", type=int, default=2,
                    help="ranks emulated on this GPU by the 'gather' case (fused all-gather -> GEMM)")
    ap.add_argument("--gather-shapes", default="qkv,fc,out,head")
    ap.add_argument("--head-rows", type=int, default=16384, help="token rows of the 'headxent' case")
    a = ap.parse_args()
    pk_tf, pk_bw, tag = peaks()
    only = set(a.only.split(","))
    N, C, V, B, T, H = 16384, 768, 50304, 16, 1024, 12
    rows = []

    def rep(name, us, flops=None, nbytes=None):
        r = {"kernel": name, "us": round(us, 2)}
        if flops:
            r["tflops"] = round(flops / us / 1e6, 1)
            r["frac_peak"] = f"{flops / us / 1e6 / pk_tf:.2f} {tag} bf16 {pk_tf:.0f} TF/s"
        if nbytes:
            r["gbs"] = round(nbytes / us / 1e3, 1)
            r["frac_hbm"] = f"{nbytes / us / 1e3 / pk_bw:.2f} {tag} HBM {pk_bw:.0f} GB/s"
        rows.append(r)
        print(json.dumps(r), flush=True)

    dev = "cuda"
    if "gemm" in only:
        shapes = {"qkv": (C, 3 * C), "proj": (C, C), "fc": (C, 4 * C), "out": (4 * C, C), "head": (C, V)}
        for name, (kin, kout) in shapes.items():
            x = torch.randn(N, kin, device=dev).bfloat16()
            w = (torch.randn(kin, kout, device=dev) * 0.02).bfloat16()
            dy = torch.randn(N, kout, device=dev).bfloat16()
            f = 2.0 * N * kin * kout
            if name == "fc":
                pre = torch.empty(N, kout, device=dev, dtype=torch.bfloat16)
                b = torch.zeros(kout, device=dev).bfloat16()
                rep(f"gemm_fwd_{name}_gelu", timeit(lambda: K.gemm(x, w, epi=K.EPI_GELU, bias=b, aux=pre), a.iters), f)
            else:
                rep(f"gemm_fwd_{name}", timeit(lambda: K.gemm(x, w), a.iters), f)
            rep(f"gemm_dx_{name}", timeit(lambda: K.gemm(dy, w, b_trans=True), a.iters), f)
            gw = torch.empty(kin, kout, device=dev)
            rep(f"gemm_dw_{name}", timeit(lambda: K.gemm(x, dy, gw, a_trans=True, epi=K.EPI_F32), a.iters), f)
            del x, w, dy, gw
    if "gather" in only:
        gather_cases(a, rep, N, C, V)
    if "headxent" in only:
        # LM head + cross-entropy forward: fused (softmax partials from the GEMM epilogue)
        # against the plain GEMM followed by the streaming cross-entropy kernel
        R = a.head_rows
        h = torch.randn(R, C, device=dev).bfloat16()
        w = (torch.randn(C, V, device=dev) * 0.05).bfloat16()
        t = torch.randint(0, V, (R,), device=dev)
        f = 2.0 * R * C * V
        rep("head_gemm_xent_fused", timeit(lambda: K.gemm_xent(h, w, t), a.iters), f)
        rep("head_gemm_then_xent", timeit(lambda: K.xent_fwd(K.gemm(h, w), t), a.iters), f)
        del h, w, t
    if "attn" in only:
        D = C // H
        qkv = torch.randn(B * T, 3 * C, device=dev).bfloat16()
        f_fwd = 4.0 * B * H * T * T * D / 2
        for legacy in (False, True):
            tagk = "mma_sync" if legacy else "tcgen05"
            rep(f"attn_fwd_{tagk}", timeit(lambda: K.attn_fwd(qkv, B, T, H, D, legacy=legacy), a.iters), f_fwd)
        out, lse = K.attn_fwd(qkv, B, T, H, D)
        dout = torch.randn_like(out)
        rep("attn_bwd", timeit(lambda: K.attn_bwd(qkv, out, dout, lse, B, T, H, D), a.iters), 2.5 * f_fwd)
    if "ln" in only:
        x = torch.randn(N, C, device=dev).bfloat16()
        w = torch.ones(C, device=dev).bfloat16()
        b = torch.zeros(C, device=dev).bfloat16()
        rep("ln_fwd", timeit(lambda: K.layernorm_fwd(x, w, b), a.iters), nbytes=2 * N * C * 2)
        y, mu, rs = K.layernorm_fwd(x, w, b)
        dw = torch.empty(C, device=dev)
        db = torch.empty(C, device=dev)
        dres = torch.randn_like(x)
        rep("ln_bwd", timeit(lambda: K.layernorm_bwd(y, x, w, mu, rs, dres, dw, db), a.iters), nbytes=4 * N * C * 2)
        rep("bias_grad_fc", timeit(lambda: K.bias_grad(torch.empty(N, 4 * C, device=dev, dtype=torch.bfloat16),
                                                       torch.empty(4 * C, device=dev)), a.iters),
            nbytes=N * 4 * C * 2)
    if "xent" in only:
        z = torch.randn(N, V, device=dev).bfloat16()
        t = torch.randint(0, V, (N,), device=dev)
        rep("xent_fwd", timeit(lambda: K.xent_fwd(z, t), a.iters), nbytes=N * V * 2)
        loss, lse = K.xent_fwd(z, t)
        g = torch.ones(1, device=dev)
        rep("xent_bwd", timeit(lambda: K.xent_bwd(z, t, lse, g), a.iters), nbytes=2 * N * V * 2)
    if "adamw" in only:
        n = 163_000_000
        p, g, m, v = (torch.zeros(n, device=dev) for _ in range(4))
        p16 = torch.empty(n, device=dev, dtype=torch.bfloat16)
        rep("adamw", timeit(lambda: K.adamw_step(p, g, m, v, p16, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1), a.iters),
            nbytes=n * (16 + 12 + 2))
        sq = torch.empty(1, device=dev, dtype=torch.float64)
        rep("grad_sqnorm", timeit(lambda: K.grad_sqnorm(g, sq), a.iters), nbytes=n * 4)


if __name__ == "__main__":
    main()
