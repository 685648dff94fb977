"""Collective sweep: this package's NVLink kernels vs NCCL on one node.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P benchmarks/collectives_bench.py [--out results.jsonl] [--max-mb 1024]

Ops: all-reduce (one-shot, two-shot, auto), reduce-scatter, all-gather and
broadcast on fp32 and bf16 buffers from 4 KB to 1 GB (powers of 2 for the fp32
all-reduce, powers of 4 otherwise).  Each rank fills its buffer with N(0,1)
values seeded by its rank.  Every measurement is CUDA-event timed on the
launching stream after warm-up, and the reported time is the max over ranks.
Bus bandwidth: all-reduce 2(W-1)/W * bytes / t; reduce-scatter and all-gather
(W-1)/W * bytes / t (bytes = full buffer); broadcast bytes / t.  For the
all-reduce the result is checked to be bit-identical on every rank.
"""
import argparse
import datetime
import hashlib
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from dtrain_b200.parallel.nvlink import NVLinkGroup, torch_exchange  # noqa: E402


def timed(fn, iters, world):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) * 1e3  # us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--max-mb", type=int, default=1024)
    ap.add_argument("--blocks", type=int, default=0, help="CTAs per collective kernel (0 = size-based default)")
    ap.add_argument("--memory", choices=["ipc", "vmm"], default="ipc",
                    help="peer memory: cudaMalloc + IPC handles, or CUDA VMM allocations shared by file descriptor")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    pg = NVLinkGroup(rank, world, dev, torch_exchange(), timeout=60.0, blocks=a.blocks, memory=a.memory)
    maxb = a.max_mb << 20
    big = {dt: pg.alloc(maxb // torch.tensor([], dtype=dt).element_size(), dt) for dt in (torch.float32, torch.bfloat16)}
    ref = {dt: torch.empty(maxb // torch.tensor([], dtype=dt).element_size(), dtype=dt, device=dev)
           for dt in (torch.float32, torch.bfloat16)}
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    for dt in big:
        big[dt].copy_(torch.randn(big[dt].numel(), generator=gen, device=dev).to(dt))
        ref[dt].copy_(big[dt])
    out = open(a.out, "a") if (a.out and rank == 0) else None
    fac_ar = 2 * (world - 1) / world
    fac_rs = (world - 1) / world

    def emit(rec):
        rec.update(world=world)
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
        for nbytes in sizes(pow2=(dt == torch.float32)):
            n = nbytes // esz
            iters = max(5, min(200, (2 << 30) // nbytes))
            x = big[dt][:n]
            y = ref[dt][:n]
            res = {}
            for meth in ("oneshot", "twoshot", "auto"):
                if meth == "oneshot" and nbytes > (64 << 20):
                    continue
                res[f"ours_{meth}"] = timed(lambda: pg.allreduce(x, "direct", method=meth), iters, world)
            res["nccl"] = timed(lambda: dist.all_reduce(y), iters, world)
            pg.check()
            # bit-identity across ranks of one fresh all-reduce
            x.copy_(torch.randn(n, generator=torch.Generator(device=dev).manual_seed(7 + rank), device=dev).to(dt))
            pg.allreduce(x, "ring")
            torch.cuda.synchronize()
            h = hashlib.sha256(x.view(torch.uint8).cpu().numpy().tobytes()).hexdigest()[:16]
            hs = [None] * world
            dist.all_gather_object(hs, h)
            for k, us in res.items():
                emit({"op": "allreduce", "impl": k, "dtype": name, "bytes": nbytes, "us": round(us, 2),
                      "busbw_GBs": round(fac_ar * nbytes / us / 1e3, 2), "bit_identical": len(set(hs)) == 1})
        for nbytes in sizes(pow2=False):
            n = nbytes // esz
            if n % world:
                continue
            iters = max(5, min(200, (2 << 30) // nbytes))
            x = big[dt][:n]
            y = ref[dt][:n]
            yo = torch.empty(n // world, dtype=dt, device=dev)
            t_rs = timed(lambda: pg.reduce_scatter(x), iters, world)
            t_rs_n = timed(lambda: dist.reduce_scatter_tensor(yo, y), iters, world)
            t_ag = timed(lambda: pg.all_gather(x), iters, world)
            t_ag_n = timed(lambda: dist.all_gather_into_tensor(y, yo), iters, world)
            t_bc = timed(lambda: pg.broadcast(x, root=0), iters, world)
            t_bc_n = timed(lambda: dist.broadcast(y, src=0), iters, world)
            pg.check()
            for op, us, fac in (("reduce_scatter", t_rs, fac_rs), ("all_gather", t_ag, fac_rs),
                                ("broadcast", t_bc, 1.0)):
                emit({"op": op, "impl": "ours", "dtype": name, "bytes": nbytes, "us": round(us, 2),
                      "busbw_GBs": round(fac * nbytes / us / 1e3, 2)})
            for op, us, fac in (("reduce_scatter", t_rs_n, fac_rs), ("all_gather", t_ag_n, fac_rs),
                                ("broadcast", t_bc_n, 1.0)):
                emit({"op": op, "impl": "nccl", "dtype": name, "bytes": nbytes, "us": round(us, 2),
                      "busbw_GBs": round(fac * nbytes / us / 1e3, 2)})
    pg.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
