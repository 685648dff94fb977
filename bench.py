"""Flagship benchmark: GPT-2-small-shape DDP training throughput on N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--bucket-mb 25]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Config (GPT-2-small DDP): 12 layers, d_model 768, 12 heads,
context 1024, vocab 50304, 16 sequences per GPU of iid uniform random tokens,
bf16 compute with fp32 grads and master weights, AdamW with global-norm clip
1.0, 25 MiB gradient buckets (``--bucket-mb 1`` for the config's other size),
random init.  Weak scaling: per-GPU work is fixed.

Gradient sync (N > 1): each bucket's all-reduce is launched from the grad-ready
hooks while backward runs, inside the CUDA graph that replays forward + backward;
the same kernels publish the gradient's sum of squares for the clip.  After the
timed runs the line reports ``checks``: whether every rank holds bit-identical
masters and gradients, and whether bucket-by-bucket and flat all-reduces of one
local gradient agree bit for bit.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the training
stream; the reported time is the max over ranks.  ``value`` is the whole-job
tokens/s with inputs already on the device; ``e2e`` is the same metric through
the public per-step API (``Trainer.step``): each step copies its token ids from
pinned host memory and reads the loss back.  Inputs (weights, activations,
logits) are far larger than the 126 MB L2, so no flush is needed between steps.

``--impl reference`` runs the reference's own torch path from ``baseline/_ref``
(dtrain.torch_ref.TorchGPT + torch DistributedDataParallel over NCCL +
torch.optim.AdamW + clip_grad_norm_, bf16 autocast) on the same config and
prints the same JSON line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import contextlib
import csv
import datetime
import io
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "GPT tokens/s at 1/2/4/8 B200 (DDP, ZeRO-1) vs ref NCCL; all-reduce busbw GB/s"
MODEL = dict(vocab=50304, ctx=1024, dim=768, heads=12, layers=12)
SEQ_PER_GPU = 16
# benchmark configurations runnable with --config (the flagship is the default)
CONFIGS = {
    "gpt2-small-ddp": dict(model=MODEL, seq=SEQ_PER_GPU, mode="ddp", accum=1,
                           name="GPT-2-small (12L, d768, 12H, ctx 1024, vocab 50304)"),
    "gpt2-medium-zero": dict(model=dict(vocab=50304, ctx=1024, dim=1024, heads=16, layers=24), seq=8, mode="zero",
                             accum=4, name="GPT-2-medium (24L, d1024, 16H, ctx 1024, vocab 50304), no_sync accum 4"),
    "gpt-1.3b-zero": dict(model=dict(vocab=50304, ctx=2048, dim=2048, heads=16, layers=24), seq=4, mode="zero",
                          accum=1, name="1.3B (24L, d2048, 16H, ctx 2048, vocab 50304)"),
}
BASELINE_VALUE = None  # the reference publishes no GPU number for this config (its numbers are CPU-only)


def _env_rank():
    if "RANK" in os.environ and "WORLD_SIZE" in os.environ:
        return int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ.get("LOCAL_RANK", 0))
    return 0, 1, 0


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons every 50 ms.  Started before
    the warm-up (nvidia-smi needs a moment to start); ``window()`` brackets the timed
    region and only the samples whose timestamps fall inside it are summarised."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def window(self, t0: float, t1: float):
        self.t0, self.t1 = t0, t1

    @staticmethod
    def _ts(field: str):
        try:
            return datetime.datetime.strptime(field.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 10]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        where = "whole run"
        if self.t0 is not None:
            inside = [r for r in rows if (t := self._ts(r[0])) is not None and self.t0 <= t <= self.t1]
            if inside:
                rows, where = inside, "timed region"
        sm = [float(r[2]) for r in rows]
        smax = float(rows[0][3])
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[6:10]) if v.strip().lower() == "active"})
        pw = [float(r[4]) for r in rows if r[4].strip() not in ("", "[N/A]")]
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows),
                "samples_from": where, "power_w_max": max(pw) if pw else None}


def _model_rate(M: dict, tokens_per_step: float, ms_per_step: float) -> dict:
    """Model FLOP rate of a step against the measured bf16 GEMM peak (MEASURED_PEAKS.json
    when present, else the pool's fallback), per GPU."""
    from dtrain_b200.models.gpt import GPTConfig, train_flops_per_token
    flops = train_flops_per_token(GPTConfig(**M)) * tokens_per_step
    peak, tag = 1590.0, "of fallback"
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak, tag = float(json.load(f)["bf16_tflops"]), "of measured"
    tf = flops / (ms_per_step / 1e3) / 1e12
    return {"model_tflops_per_step": flops / 1e12, "model_tflops_per_s": tf,
            "frac_of_bf16_peak": f"{tf / peak:.3f} {tag} {peak:.0f} TFLOP/s burst"}


def _hash64(t: torch.Tensor) -> int:
    """A 64-bit fingerprint of a tensor's bits (position-weighted wrapping sum of its
    32-bit words, computed on the device; equal bits give equal fingerprints)."""
    w = t.reshape(-1).view(torch.int32).long()
    idx = torch.arange(w.numel(), device=w.device, dtype=torch.int64)
    coef = (idx * 2654435761 + 40503) % 2147483647 * 2 + 1
    return int((w * coef).sum().item()) & ((1 << 64) - 1)


def _all_rows(pg, row: list[int]) -> list[list[int]]:
    """Every rank's row of 64-bit integers, exchanged through the NVLink group: each
    value travels as four exact 16-bit pieces in fp32 in this rank's slot of a
    rank-order all-reduce (a sum with zeros everywhere else)."""
    k = len(row)
    buf = torch.zeros(pg.world, 4 * k, dtype=torch.float32, device=pg.device)
    buf[pg.rank] = torch.tensor([float((v >> (16 * j)) & 0xFFFF) for v in row for j in range(4)],
                                device=pg.device)
    pg.allreduce(buf.reshape(-1), "direct", method="twoshot")
    pg.check()
    out = buf.long().cpu().tolist()
    return [[sum(r[4 * i + j] << (16 * j) for j in range(4)) for i in range(k)] for r in out]


def _consistency(tr, pg, batch) -> dict:
    """Cross-rank checks after the timed runs (ranks in lockstep):
    ranks_bit_identical - every rank's fp32 masters and averaged gradient of the last
    step have the same bits; bucketed_equals_flat - one more backward without sync,
    then its local gradient all-reduced bucket by bucket (the lean kernels the
    overlapped step uses) and, from the same input, as one flat all-reduce, both in
    rank order: the two results have the same bits on every rank."""
    fp = tr.model.flat
    rows = _all_rows(pg, [_hash64(fp.master), _hash64(fp.grad)])
    ident = all(r == rows[0] for r in rows)
    ddp = tr.ddp
    tr.model.zero_grad()
    x, y = batch
    with ddp.no_sync():
        _, loss = tr.model(x, y)
        loss.backward()
    raw = fp.grad.clone()
    for b in ddp.buckets:
        pg.allreduce(fp.grad[b.lo:b.hi], "direct", scale=1.0 / pg.world, method="twoshot", blocks=b.blocks,
                     lean=b.lean)
    bucketed = fp.grad.clone()
    fp.grad.copy_(raw)
    pg.allreduce(fp.grad, "direct", scale=1.0 / pg.world, method="twoshot")
    same = bool(torch.equal(bucketed, fp.grad))
    votes = _all_rows(pg, [int(same)])
    pg.synchronize()
    return {"ranks_bit_identical": ident, "bucketed_equals_flat": all(v[0] == 1 for v in votes),
            "fingerprints_rank0": {"master": hex(rows[0][0]), "grad": hex(rows[0][1])}}


def _timed(fn, steps: int, world: int):
    """CUDA-event time of ``steps`` calls of fn, barrier + synchronize on both sides; max over ranks (ms)."""
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _grad_sync(tr, C, a, world) -> dict | str:
    """What the gradient synchronisation of the measured step actually ran."""
    if C["mode"] == "zero":
        if world == 1:
            return "one GPU: no collective (AdamW + norm kernels)"
        return ("one kernel: reduce-scatter + clip + AdamW (non-GEMM params gathered there); Linear weights "
                "all-gathered inside the forward GEMMs" if a.gather_gemm else
                "one kernel: reduce-scatter + clip + AdamW + all-gather")
    if world == 1:
        return "one GPU: no collective (gradient norm kernel + AdamW)"
    d = tr.ddp
    kind = "NVSwitch (multimem) reduction" if d.method == "nvls" else "two-shot"
    order = "the switch's" if d.method == "nvls" else a.algo
    if not d.overlap:
        return {"buckets": "unused", "method": f"one {kind} all-reduce of the flat gradient after backward",
                "order": order, "grad_norm": "fused into the all-reduce"}
    lean = sum(1 for b in d.buckets if b.lean)
    return {"buckets": len(d.buckets), "bucket_mb": a.bucket_mb,
            "method": f"{kind} per bucket, launched from the grad-ready hooks during backward",
            "lean_buckets": lean, "full_width_buckets": len(d.buckets) - lean, "order": order,
            "grad_norm": "fused into the all-reduce"}


# ------------------------------------------------------------------ our arm
def run_ours(a, rank, world, local):
    from dtrain_b200 import train as T
    from dtrain_b200.models.gpt import GPTConfig
    from dtrain_b200.ops import kernels as K
    from dtrain_b200.parallel.nvlink import NVLinkGroup, torch_exchange
    from dtrain_b200.utils.data import SyntheticData
    import torch.distributed as dist

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        pg = NVLinkGroup(rank, world, dev, torch_exchange(), timeout=120.0, blocks=a.comm_blocks,
                         comm_priority=a.comm_priority, nvls=(a.ar_method == "nvls"))
    else:
        pg = NVLinkGroup(0, 1, dev, lambda k, p: [p], timeout=120.0)
    C = CONFIGS[a.config]
    M, seq, accum = C["model"], C["seq"], C["accum"]
    args = T.parse(["--mode", C["mode"], "--dtype", "bfloat16", "--batch", str(seq), "--ctx", str(M["ctx"]),
                    "--dim", str(M["dim"]), "--heads", str(M["heads"]), "--layers", str(M["layers"]),
                    "--lr", "6e-4", "--clip", "1.0", "--bucket-mb", str(a.bucket_mb), "--data", "synthetic",
                    "--vocab", str(M["vocab"]), "--algo", a.algo, "--accum", str(accum), "--ar-method", a.ar_method]
                   + (["--no-overlap"] if a.no_overlap else []) + (["--cuda-graph"] if a.cuda_graph else [])
                   + (["--gather-gemm"] if a.gather_gemm else []))
    cfg = GPTConfig(dtype="bfloat16", **M)
    tr = T.Trainer(args, cfg, dev, pg)
    if a.trace and tr.ddp is not None:
        tr.ddp.enable_trace()
    data = SyntheticData(M["vocab"])
    nb = a.warmup + a.steps
    host = [[data.rank_batch(s, mi, seq, M["ctx"], 0, rank, world) for mi in range(accum)] for s in range(nb)]
    dev_batches = [[(torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)) for x, y in hs] for hs in host]

    def device_step(i):  # inputs already resident: the kernel-side number
        tr.step([[mb] for mb in dev_batches[i % nb]], return_loss=False)

    sampler = ClockSampler(local) if local == 0 else None
    if sampler:
        sampler.start()
    for i in range(a.warmup):
        device_step(i)
    torch.cuda.synchronize()
    pg.check()
    l0, r0 = K.launch_count(), tr.graph_replays
    t0 = time.time()
    ms = _timed(lambda i: device_step(a.warmup + i), a.steps, world)
    t1 = time.time()
    trace = tr.ddp.trace_report() if (a.trace and tr.ddp is not None) else None
    # eager launches counted on the host, plus the kernels each graph replay runs
    launches = K.launch_count() - l0 + (tr.graph_replays - r0) * tr.graph_launches
    if sampler:
        sampler.window(t0, t1)
    clocks = sampler.stop() if sampler else None
    pg.check()

    # end to end through the public per-step API: H2D of ids from pinned memory + loss D2H every step
    losses = []

    def e2e_step(i):
        s = a.warmup + i
        losses.append(tr.step([[mb] for mb in host[s % nb]]))

    ms_e2e = _timed(e2e_step, a.steps, world)
    pg.check()
    checks = _consistency(tr, pg, dev_batches[0][0]) if (world > 1 and tr.ddp is not None) else None
    tokens = seq * accum * M["ctx"] * world
    res = {
        "metric": METRIC, "value": tokens * a.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (iid uniform token ids, random-init weights)",
        "config": {"model": C["name"], "global_batch": seq * accum * world,
                   "seq_len": M["ctx"], "parallelism": f"{'dp' if C['mode'] == 'ddp' else 'zero1-dp'}{world}",
                   "grad_accum": accum, "grad_sync": _grad_sync(tr, C, a, world),
                   "optimizer": "AdamW, clip 1.0",
                   "cuda_graph": (("forward+backward" + (" + bucket all-reduces + gradient norm"
                                                         if tr.sync_in_graph and world > 1 else ""))
                                  + " captured once and replayed; optimizer eager" if a.cuda_graph else False),
                   "l2": "no flush: weights/activations/logits per step >> 126 MB L2"},
        "e2e": {"value": tokens * a.steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * seq * accum * M["ctx"] * 8, "d2h_bytes_per_step": 4,
                "ms_per_step": ms_e2e / a.steps, "final_loss": losses[-1] if losses else None},
        "checks": checks,
        **({"trace_last_step": trace} if trace is not None else {}),
        "gpu_launches": int(launches),
        "gpu_launches_per_step": launches / max(1, a.steps),
        "per_gpu": _model_rate(M, seq * accum * M["ctx"], ms / a.steps),
        "clocks": clocks,
    }
    tr._graph = None  # release the captured graph before the groups go away
    torch.cuda.synchronize()
    pg.close()
    if world > 1:
        dist.destroy_process_group()
    return res


# ------------------------------------------------------------ reference arm
def run_reference(a, rank, world, local):
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "dtrain")):
        return {"impl": "reference", "unavailable": "baseline/_ref is not installed (pip install --target baseline/_ref)"}
    sys.path.insert(0, ref_dir)
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel

    from dtrain.nn import GPTConfig as RefConfig
    from dtrain.torch_ref import TorchGPT

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    C = CONFIGS[a.config]
    M, seq, accum = C["model"], C["seq"], C["accum"]
    cfg = RefConfig(dtype="float32", **M)
    # random init with the reference's own initialiser (dtrain.nn.GPT), then its torch mirror
    from dtrain.nn import GPT as RefGPT
    model = TorchGPT.from_dtrain(RefGPT(cfg, seed=0)).to(dev)
    ddp = DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=a.bucket_mb) if world > 1 else model
    adam = dict(lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    if C["mode"] == "zero" and world > 1:
        from torch.distributed.optim import ZeroRedundancyOptimizer
        opt = ZeroRedundancyOptimizer(model.parameters(), optimizer_class=torch.optim.AdamW, **adam)
    else:
        opt = torch.optim.AdamW(model.parameters(), **adam)
    rng = np.random.default_rng([0, rank])
    nb = a.warmup + a.steps
    host = [[rng.integers(0, M["vocab"], size=(seq, M["ctx"] + 1), dtype=np.int64) for _ in range(accum)]
            for _ in range(nb)]
    pinned = [[torch.from_numpy(h).pin_memory() for h in hs] for hs in host]
    dev_tokens = [[p.to(dev) for p in ps] for ps in pinned]

    def step(toks, read_loss):
        opt.zero_grad(set_to_none=True)
        total = 0.0
        for mi, tok in enumerate(toks):
            last = mi == len(toks) - 1
            ctx = ddp.no_sync() if (world > 1 and not last) else contextlib.nullcontext()
            with ctx:
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    _, loss = ddp(tok[:, :-1], tok[:, 1:])
                (loss / len(toks)).backward()
            total = total + loss.detach() / len(toks)
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        return float(total.item()) if read_loss else None

    sampler = ClockSampler(local) if local == 0 else None
    if sampler:
        sampler.start()
    for i in range(a.warmup):
        step(dev_tokens[i], False)
    t0 = time.time()
    ms = _timed(lambda i: step(dev_tokens[a.warmup + i], False), a.steps, world)
    t1 = time.time()
    if sampler:
        sampler.window(t0, t1)
    clocks = sampler.stop() if sampler else None
    ms_e2e = _timed(lambda i: step([p.to(dev, non_blocking=True) for p in pinned[a.warmup + i]], True),
                    a.steps, world)
    tokens = seq * accum * M["ctx"] * world
    res = {
        "impl": "reference", "metric": METRIC, "value": tokens * a.steps / (ms / 1e3), "unit": "tokens/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (torch.autocast)",
        "data": "synthetic (iid uniform token ids, random-init weights)",
        "config": {"model": C["name"], "global_batch": seq * accum * world, "grad_accum": accum,
                   "seq_len": M["ctx"], "parallelism": f"{'dp' if C['mode'] == 'ddp' else 'zero1-dp'}{world}",
                   "bucket_mb": a.bucket_mb,
                   "stack": "dtrain.torch_ref.TorchGPT + torch DDP (NCCL) + torch.optim.AdamW"
                            + (" in ZeroRedundancyOptimizer" if C["mode"] == "zero" else "") + " + clip_grad_norm_",
                   "l2": "no flush: weights/activations/logits per step >> 126 MB L2"},
        "e2e": {"value": tokens * a.steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": seq * accum * (M["ctx"] + 1) * 8, "d2h_bytes_per_step": 4,
                "ms_per_step": ms_e2e / a.steps},
        "gpu_launches": 0,
        "per_gpu": _model_rate(M, seq * accum * M["ctx"], ms / a.steps),
        "clocks": clocks,
    }
    if world > 1:
        dist.destroy_process_group()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--bucket-mb", type=float, default=25.0,
                    help="DDP gradient bucket size in MiB, both arms (the configuration names 1 and 25; 25 is torch "
                         "DDP's default and measured faster here: fewer per-bucket cross-GPU barriers)")
    ap.add_argument("--algo", choices=["ring", "direct"], default="ring")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="gpt2-small-ddp")
    ap.add_argument("--ar-method", choices=["auto", "twoshot", "nvls"], default="auto",
                    help="bucket all-reduce: fixed-order two-shot (auto) or NVSwitch reduction (nvls)")
    ap.add_argument("--comm-blocks", type=int, default=0, help="CTAs per collective kernel (0: by size)")
    ap.add_argument("--comm-priority", type=int, default=0, help="CUDA priority of the collective stream")
    ap.add_argument("--no-cuda-graph", dest="cuda_graph", action="store_false",
                    help="launch every kernel from Python each step instead of replaying the captured "
                         "forward+backward graph")
    ap.add_argument("--gather-gemm", action="store_true",
                    help="ZeRO: all-gather the Linear weights inside the forward GEMMs instead of in the optimizer "
                         "kernel (measured 1.6%% slower on 2 GPUs, GPT-2-medium)")
    ap.add_argument("--trace", action="store_true",
                    help="DDP: record device timestamps of the buckets' ready points and all-reduces (adds ~3 tiny "
                         "kernels per bucket) and print the last timed step's timeline")
    ap.add_argument("--no-overlap", action="store_true",
                    help="one all-reduce of the flat gradient after backward instead of per-bucket all-reduces "
                         "launched from the grad-ready hooks during backward")
    a = ap.parse_args()
    if a.warmup < 3:
        a.warmup = 3
    rank, world, local = _env_rank()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    res = run_reference(a, rank, world, local) if a.impl == "reference" else run_ours(a, rank, world, local)
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
