"""Collective sweep: this package's NVLink kernels vs NCCL on one node.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P benchmarks/collectives_bench.py [--out results.jsonl] [--md table.md] [--max-mb 1024]

Ops: all-reduce (one-shot, two-shot, the size-based choice and, with ``--nvls``,
the NVSwitch multicast reduction), reduce-scatter (ring order; with ``--nvls`` also
through the switch, fp32), all-gather and broadcast, on fp32 and bf16 buffers of every power of two from
4 KB to 1 GB.  Each rank fills its buffer with N(0,1) values seeded by its rank.
Every measurement is CUDA-event timed after warm-up (the same buffer each call:
sizes below the 126 MB L2 are L2-warm, as in NCCL's own tests) and the reported
time is the max over ranks.  By default the timed calls are captured once in a
CUDA graph and replayed (both stacks' collectives are graph-capturable), so the
numbers are device time without the host's per-call cost; ``--eager`` times
back-to-back eager calls instead.  Bus bandwidth: all-reduce
2(W-1)/W * bytes / t; reduce-scatter and all-gather (W-1)/W * bytes / t (bytes =
full buffer); broadcast bytes / t.  ``frac_peer_copy`` divides it by the 770 GB/s
peer-copy bandwidth measured on this pool.  Bit identity across ranks is checked
for every op on fresh data: the all-reduce result, the buffer that reduce-scatter
followed by all-gather leaves on every rank, and the broadcast copy.
"""
import argparse
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from dtrain_b200.parallel.nvlink import NVLinkGroup, torch_exchange  # noqa: E402


PEER_COPY_GBS = 770.0  # measured peer-copy bandwidth per direction on this pool's B200s


def _fingerprint(t: torch.Tensor) -> int:
    """64-bit position-weighted sum of the buffer's 32-bit words, on the device (a
    difference in any word changes it)."""
    w = t.contiguous().view(torch.int32).reshape(-1).long()
    idx = torch.arange(w.numel(), device=w.device, dtype=torch.int64)
    return int((w * ((idx * 2654435761 + 40503) % 2147483647 * 2 + 1)).sum().item()) & ((1 << 64) - 1)


def same_on_all_ranks(t: torch.Tensor, world: int) -> bool:
    hs = [None] * world
    dist.all_gather_object(hs, _fingerprint(t))
    return len(set(hs)) == 1


GRAPH = True


def timed(fn, iters, world):
    """Mean device time of one call in us (max over ranks): ``iters`` calls captured in
    one CUDA graph and replayed (``GRAPH``), or issued eagerly back to back."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = None
    if GRAPH:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(iters):
                fn()
        graph.replay()
        torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    if graph is not None:
        graph.replay()
    else:
        for _ in range(iters):
            fn()
    b.record()
    torch.cuda.synchronize()
    del graph
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) * 1e3  # us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--max-mb", type=int, default=1024)
    ap.add_argument("--md", default=None, help="write a Markdown summary table here (rank 0)")
    ap.add_argument("--blocks", type=int, default=0, help="CTAs per collective kernel (0 = size-based default)")
    ap.add_argument("--memory", choices=["ipc", "vmm"], default="ipc",
                    help="peer memory: cudaMalloc + IPC handles, or CUDA VMM allocations shared by file descriptor")
    ap.add_argument("--eager", action="store_true", help="time eager back-to-back calls instead of graph replays")
    ap.add_argument("--nvls", action="store_true",
                    help="map the buffers through NVSwitch multicast (VMM memory) and add the NVLS methods")
    a = ap.parse_args()
    global GRAPH
    GRAPH = not a.eager
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    pg = NVLinkGroup(rank, world, dev, torch_exchange(), timeout=60.0, blocks=a.blocks,
                     memory="vmm" if a.nvls else a.memory, nvls=a.nvls)
    maxb = a.max_mb << 20
    big = {dt: pg.alloc(maxb // torch.tensor([], dtype=dt).element_size(), dt) for dt in (torch.float32, torch.bfloat16)}
    ref = {dt: torch.empty(maxb // torch.tensor([], dtype=dt).element_size(), dtype=dt, device=dev)
           for dt in (torch.float32, torch.bfloat16)}
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    for dt in big:
        big[dt].copy_(torch.randn(big[dt].numel(), generator=gen, device=dev).to(dt))
        ref[dt].copy_(big[dt])
    out = open(a.out, "a") if (a.out and rank == 0) else None
    rows = []
    fac_ar = 2 * (world - 1) / world
    fac_rs = (world - 1) / world

    def emit(rec):
        rec.update(world=world, frac_peer_copy=round(rec["busbw_GBs"] / PEER_COPY_GBS, 3))
        rows.append(rec)
        if rank == 0:
            print(json.dumps(rec), flush=True)
            if out:
                out.write(json.dumps(rec) + "\n")
                out.flush()

    def sizes(pow2):
        s, step = 4096, (2 if pow2 else 4)
        while s <= maxb:
            yield s
            s *= step

    for dt, name in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        esz = torch.tensor([], dtype=dt).element_size()
        for nbytes in sizes(pow2=True):
            n = nbytes // esz
            iters = max(5, min(100, (2 << 30) // nbytes))
            x = big[dt][:n]
            y = ref[dt][:n]
            res = {}
            for meth in ("oneshot", "twoshot", "auto") + (("nvls",) if a.nvls else ()):
                if meth == "oneshot" and nbytes > (64 << 20):
                    continue
                res[f"ours_{meth}"] = timed(lambda: pg.allreduce(x, "direct", method=meth), iters, world)
            if nbytes >= (1 << 20):  # a wider grid than the size-based default
                res["ours_twoshot_b128"] = timed(lambda: pg.allreduce(x, "direct", method="twoshot", blocks=128),
                                                 iters, world)
                if nbytes <= (16 << 20):
                    res["ours_oneshot_b128"] = timed(
                        lambda: pg.allreduce(x, "direct", method="oneshot", blocks=128), iters, world)
                if a.nvls:
                    res["ours_nvls_b128"] = timed(lambda: pg.allreduce(x, "direct", method="nvls", blocks=128),
                                                  iters, world)
            res["nccl"] = timed(lambda: dist.all_reduce(y), iters, world)
            pg.check()
            # bit-identity across ranks of one fresh all-reduce
            x.copy_(torch.randn(n, generator=torch.Generator(device=dev).manual_seed(7 + rank), device=dev).to(dt))
            pg.allreduce(x, "ring")
            torch.cuda.synchronize()
            same = {"ring": same_on_all_ranks(x, world)}
            if a.nvls:
                x.copy_(torch.randn(n, generator=torch.Generator(device=dev).manual_seed(9 + rank), device=dev).to(dt))
                pg.allreduce(x, method="nvls")
                torch.cuda.synchronize()
                same["nvls"] = same_on_all_ranks(x, world)
            for k, us in res.items():
                emit({"op": "allreduce", "impl": k, "dtype": name, "bytes": nbytes, "us": round(us, 2),
                      "busbw_GBs": round(fac_ar * nbytes / us / 1e3, 2),
                      "bit_identical": same["nvls" if "nvls" in k else "ring"]})
        for nbytes in sizes(pow2=True):
            n = nbytes // esz
            if n % world:
                continue
            iters = max(5, min(100, (2 << 30) // nbytes))
            x = big[dt][:n]
            y = ref[dt][:n]
            yo = torch.empty(n // world, dtype=dt, device=dev)
            t_rs = timed(lambda: pg.reduce_scatter(x), iters, world)
            t_rs_nv = timed(lambda: pg.reduce_scatter(x, method="nvls"), iters, world) \
                if (a.nvls and dt == torch.float32) else None
            t_rs_n = timed(lambda: dist.reduce_scatter_tensor(yo, y), iters, world)
            t_ag = timed(lambda: pg.all_gather(x), iters, world)
            t_ag_n = timed(lambda: dist.all_gather_into_tensor(y, yo), iters, world)
            t_bc = timed(lambda: pg.broadcast(x, root=0), iters, world)
            t_bc_n = timed(lambda: dist.broadcast(y, src=0), iters, world)
            pg.check()
            # bit identity on fresh data: reduce-scatter then all-gather, then a broadcast
            x.copy_(torch.randn(n, generator=torch.Generator(device=dev).manual_seed(11 + rank), device=dev).to(dt))
            pg.reduce_scatter(x)
            pg.all_gather(x)
            torch.cuda.synchronize()
            same_rsag = same_on_all_ranks(x, world)
            x.copy_(torch.randn(n, generator=torch.Generator(device=dev).manual_seed(13 + rank), device=dev).to(dt))
            pg.broadcast(x, root=0)
            torch.cuda.synchronize()
            same_bc = same_on_all_ranks(x, world)
            for op, us, fac, same in (("reduce_scatter", t_rs, fac_rs, same_rsag), ("all_gather", t_ag, fac_rs, same_rsag),
                                      ("broadcast", t_bc, 1.0, same_bc)):
                emit({"op": op, "impl": "ours", "dtype": name, "bytes": nbytes, "us": round(us, 2),
                      "busbw_GBs": round(fac * nbytes / us / 1e3, 2), "bit_identical": same})
            if t_rs_nv is not None:
                emit({"op": "reduce_scatter", "impl": "ours_nvls", "dtype": name, "bytes": nbytes,
                      "us": round(t_rs_nv, 2), "busbw_GBs": round(fac_rs * nbytes / t_rs_nv / 1e3, 2)})
            for op, us, fac in (("reduce_scatter", t_rs_n, fac_rs), ("all_gather", t_ag_n, fac_rs),
                                ("broadcast", t_bc_n, 1.0)):
                emit({"op": op, "impl": "nccl", "dtype": name, "bytes": nbytes, "us": round(us, 2),
                      "busbw_GBs": round(fac * nbytes / us / 1e3, 2)})
    if rank == 0 and a.md:
        with open(a.md, "w") as f:
            f.write(markdown(rows, world, "CUDA-graph replay" if GRAPH else "eager calls"))
    pg.close()
    dist.destroy_process_group()


def _fmt_size(b: int) -> str:
    return f"{b >> 30} GiB" if b >= 1 << 30 else f"{b >> 20} MiB" if b >= 1 << 20 else f"{b >> 10} KiB"


def markdown(rows: list, world: int, timing: str = "") -> str:
    """One table per op and dtype: ours (the fastest fixed-order method per size, and
    the NVLS method where it ran) vs NCCL."""
    out = [f"## W = {world}" + (f" ({timing})" if timing else ""), ""]
    for op in ("allreduce", "reduce_scatter", "all_gather", "broadcast"):
        for dt in ("fp32", "bf16"):
            sel = [r for r in rows if r["op"] == op and r["dtype"] == dt]
            if not sel:
                continue
            has_nv = any(r["impl"] == "ours_nvls" for r in sel)
            head = "| size | ours GB/s | method | NCCL GB/s | ours/NCCL | ours frac of 770 | bit-identical |"
            rule = "|---|---|---|---|---|---|---|"
            if has_nv:
                head += " NVLS GB/s | NVLS/NCCL |"
                rule += "---|---|"
            out += [f"### {op} {dt}", "", head, rule]
            for nb in sorted({r["bytes"] for r in sel}):
                mine = [r for r in sel if r["bytes"] == nb and r["impl"] != "nccl" and "nvls" not in r["impl"]]
                nv = sorted((r for r in sel if r["bytes"] == nb and "nvls" in r["impl"]),
                            key=lambda r: -r["busbw_GBs"])
                nccl = [r for r in sel if r["bytes"] == nb and r["impl"] == "nccl"]
                if op == "allreduce":  # the fastest fixed-order method at this size
                    best = max(mine, key=lambda r: r["busbw_GBs"])
                else:
                    best = mine[0]
                n = nccl[0]["busbw_GBs"] if nccl else float("nan")
                line = (f"| {_fmt_size(nb)} | {best['busbw_GBs']:.1f} | {best['impl']} | {n:.1f} | "
                        f"{best['busbw_GBs'] / n:.2f} | {best['frac_peer_copy']:.2f} | {best.get('bit_identical')} |")
                if has_nv:
                    line += (f" {nv[0]['busbw_GBs']:.1f} | {nv[0]['busbw_GBs'] / n:.2f} |" if nv else " - | - |")
                out.append(line)
            out.append("")
    return "\n".join(out)


if __name__ == "__main__":
    main()
