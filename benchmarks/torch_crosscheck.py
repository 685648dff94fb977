"""Side-by-side check of this package's DDP / ZeRO-1 / AdamW / checkpoint-resume
against torch.distributed (gloo, CPU ranks).

Counterpart of the reference's benchmarks/torch_crosscheck.py (same flags and the
same output files, so its tests and reports read either).  Run one copy per rank
through the launcher:

    python -m dtrain_b200.launch --nproc 2 -- python benchmarks/torch_crosscheck.py \
        --mode ddp --steps 20 --dtype float64 --torch-init /tmp/gloo_x --out out/ddp_w2

Every rank holds two replicas that start from the same weights and see the same
per-rank batches (``utils.data.rank_batch``):
  ours   this package's GPT under its DDP (TCP collectives) + AdamW or SGD, or
         under ZeroAdamW;
  torch  ``TorchGPT`` (the same model, reference math) under torch
         DistributedDataParallel + torch.optim.AdamW / SGD, or
         ZeroRedundancyOptimizer(AdamW), over a gloo group.
Rank 0 writes ``<out>.jsonl`` (per-step loss, parameter and - DDP - averaged
gradient differences), ``<out>.npz`` (final flat parameters of both) and
``<out>.meta.json`` (arguments, parameter count, optimizer state bytes per rank).

Checkpoint/resume: ``--phase first`` stops after ``--k`` steps and saves both
replicas under ``--ckpt`` (ours in the sharded .npz layout, torch with
torch.save); ``--phase resume`` continues from there in fresh processes.
``--only ours|torch`` runs one side (timing); no differences are recorded then.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
from torch.distributed.optim import ZeroRedundancyOptimizer  # noqa: E402
from torch.nn.parallel import DistributedDataParallel  # noqa: E402

from dtrain_b200.models.gpt import GPT, GPTConfig  # noqa: E402
from dtrain_b200.ops.optim import AdamW  # noqa: E402
from dtrain_b200.parallel.comm import init_from_env  # noqa: E402
from dtrain_b200.parallel.ddp import DDP  # noqa: E402
from dtrain_b200.parallel.zero import ZeroAdamW  # noqa: E402
from dtrain_b200.torch_ref import TorchGPT  # noqa: E402
from dtrain_b200.utils import checkpoint  # noqa: E402
from dtrain_b200.utils.data import CharData, load_text, rank_batch  # noqa: E402

BETAS, EPS = (0.9, 0.95), 1e-8


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--mode", choices=["ddp", "zero"], default="ddp")
    ap.add_argument("--phase", choices=["full", "first", "resume"], default="full")
    ap.add_argument("--only", choices=["both", "ours", "dtrain", "torch"], default="both")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--k", type=int, default=10, help="checkpoint step of --phase first / resume")
    ap.add_argument("--ckpt", default=None)
    ap.add_argument("--dtype", default="float64")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--ctx", type=int, default=32)
    ap.add_argument("--dim", type=int, default=64)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--opt", choices=["adamw", "sgd"], default="adamw", help="sgd: DDP mode only")
    ap.add_argument("--wd", type=float, default=0.1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--torch-bucket-mb", type=float, default=25.0)
    ap.add_argument("--data", default=None)
    ap.add_argument("--torch-init", required=True, help="gloo FileStore path (must not exist yet)")
    ap.add_argument("--out", required=True, help="output prefix written by rank 0")
    a = ap.parse_args(argv)
    if a.only == "dtrain":
        a.only = "ours"
    if a.mode == "zero" and a.opt != "adamw":
        ap.error("--opt sgd is DDP-only")
    return a


class _Sgd:
    """p -= lr * g, the update torch.optim.SGD makes with default arguments."""

    def __init__(self, params, lr):
        self.params, self.lr = list(params), lr

    def step(self, grads):
        with torch.no_grad():
            for p, g in zip(self.params, grads):
                p.sub_(self.lr * g)

    def state_bytes(self):
        return 0


class Ours:
    """This package's replica: GPT + DDP (+ AdamW / SGD) or GPT + ZeroAdamW."""

    def __init__(self, a, model, pg):
        self.a, self.model, self.pg = a, model, pg
        self.params = list(model.parameters())
        self.ddp = self.zero = self.opt = None
        if a.mode == "ddp":
            self.ddp = DDP(model, pg, bucket_mb=1.0, overlap=True)
            self.opt = (AdamW(self.params, lr=a.lr, betas=BETAS, eps=EPS, weight_decay=a.wd)
                        if a.opt == "adamw" else _Sgd(self.params, a.lr))
        else:
            self.zero = ZeroAdamW(model, pg, max_grad_norm=None, lr=a.lr, betas=BETAS, eps=EPS, weight_decay=a.wd)

    def step(self, x, y):
        """One optimizer step; returns (mean loss over ranks, flat averaged grads or None)."""
        self.model.zero_grad()
        _, loss = self.model(torch.as_tensor(x).long(), torch.as_tensor(y).long())
        loss.backward()
        grads = None
        if self.ddp is not None:
            self.ddp.finish()
            grads = np.concatenate([p.grad.detach().numpy().reshape(-1) for p in self.params])
            self.opt.step([p.grad for p in self.params])
        else:
            self.zero.step()
        lv = np.array([float(loss.detach())])
        self.pg.allreduce(lv)
        return float(lv[0]) / self.pg.world, grads

    def flat(self):
        return np.concatenate([p.detach().numpy().reshape(-1) for p in self.params])

    def state_bytes(self):
        return (self.zero or self.opt).state_bytes()

    def state(self):
        """Checkpoint dict in the reference's key layout (params + t + moments)."""
        if self.zero is not None:
            sd = self.zero.state_dict()
            return {"params": self.zero.flat, "t": sd["t"], "m": sd["m"][0], "v": sd["v"][0]}
        st = {"params": self.flat()}
        if isinstance(self.opt, AdamW):
            sd = self.opt.state_dict()
            st["t"] = sd["t"]
            st.update({f"m{i}": m for i, m in enumerate(sd["m"])})
            st.update({f"v{i}": v for i, v in enumerate(sd["v"])})
        return st

    def load(self, st):
        flat = np.asarray(st["params"])
        off = 0
        with torch.no_grad():
            for p in self.params:
                p.copy_(torch.from_numpy(flat[off:off + p.numel()].reshape(tuple(p.shape))))
                off += p.numel()
        if self.zero is not None:
            self.zero.load_state_dict({"t": st["t"], "m": [st["m"]], "v": [st["v"]]})
        elif isinstance(self.opt, AdamW):
            n = len(self.params)
            self.opt.load_state_dict({"t": st["t"], "m": [st[f"m{i}"] for i in range(n)],
                                      "v": [st[f"v{i}"] for i in range(n)]})


class Torch:
    """The torch replica: TorchGPT under DistributedDataParallel (+ ZeroRedundancyOptimizer)."""

    def __init__(self, a, model):
        self.a, self.model = a, model
        self.ddp = DistributedDataParallel(model, bucket_cap_mb=a.torch_bucket_mb)
        if a.mode == "ddp":
            self.opt = (torch.optim.AdamW(model.parameters(), lr=a.lr, betas=BETAS, eps=EPS, weight_decay=a.wd)
                        if a.opt == "adamw" else torch.optim.SGD(model.parameters(), lr=a.lr))
        else:
            self.opt = ZeroRedundancyOptimizer(model.parameters(), optimizer_class=torch.optim.AdamW, lr=a.lr,
                                               betas=BETAS, eps=EPS, weight_decay=a.wd)

    def step(self, x, y):
        self.opt.zero_grad(set_to_none=True)
        _, loss = self.ddp(x, y)
        loss.backward()
        grads = self.model.flat_grads() if self.a.mode == "ddp" else None
        self.opt.step()
        lv = loss.detach().reshape(1).clone()
        dist.all_reduce(lv)
        return float(lv[0]) / dist.get_world_size(), grads

    def flat(self):
        return self.model.flat_params()

    def state_bytes(self):
        inner = self.opt.optim if isinstance(self.opt, ZeroRedundancyOptimizer) else self.opt
        return sum(v.numel() * v.element_size() for s in inner.state.values() for k, v in s.items()
                   if torch.is_tensor(v) and k != "step")


def main(argv=None):
    a = parse(argv)
    torch.set_num_threads(1)
    pg = init_from_env()
    rank, world = pg.rank, pg.world
    dist.init_process_group("gloo", init_method=f"file://{a.torch_init}", rank=rank, world_size=world)
    data = CharData(load_text(a.data))
    cfg = GPTConfig(vocab=data.vocab, ctx=a.ctx, dim=a.dim, heads=a.heads, layers=a.layers, dtype=a.dtype)
    use_o, use_t = a.only in ("both", "ours"), a.only in ("both", "torch")
    model = GPT(cfg, seed=a.seed)
    tmodel = TorchGPT.from_dtrain(model)  # identical initial weights
    ours = Ours(a, model, pg) if use_o else None
    theirs = Torch(a, tmodel) if use_t else None
    ck_ours = os.path.join(a.ckpt, "ours") if a.ckpt else None
    ck_torch = os.path.join(a.ckpt, "torch.pt") if a.ckpt else None
    start = 0
    if a.phase == "resume":
        if ours is not None:
            start, st = checkpoint.load(checkpoint.latest(ck_ours), rank, world)
            ours.load(st)
        if theirs is not None:
            saved = torch.load(ck_torch, weights_only=False)
            tmodel.load_state_dict(saved["model"])
            theirs.opt.load_state_dict(saved["opt"])
            start = saved["step"]

    end = a.k if a.phase == "first" else a.steps
    log = open(a.out + ".jsonl", "w") if rank == 0 else None
    for step in range(start, end):
        x, y = rank_batch(data.train, step, 0, a.batch, a.ctx, a.seed, rank, world)
        rec = {"step": step + 1}
        g_o = g_t = None
        if ours is not None:
            t0 = time.perf_counter()
            rec["dtrain_loss"], g_o = ours.step(x, y)
            rec["dtrain_s"] = time.perf_counter() - t0
        if theirs is not None:
            t0 = time.perf_counter()
            rec["torch_loss"], g_t = theirs.step(x, y)
            rec["torch_s"] = time.perf_counter() - t0
        if ours is not None and theirs is not None:
            po, pt = ours.flat(), theirs.flat()
            rec.update(param_maxabs_diff=float(np.max(np.abs(po - pt))), param_maxabs=float(np.max(np.abs(pt))),
                       param_bit_identical_frac=float(np.mean(po == pt)),
                       loss_abs_diff=abs(rec["dtrain_loss"] - rec["torch_loss"]))
            if g_o is not None:
                rec.update(grad_maxabs_diff=float(np.max(np.abs(g_o - g_t))), grad_maxabs=float(np.max(np.abs(g_t))),
                           grad_bit_identical_frac=float(np.mean(g_o == g_t)))
        if log:
            log.write(json.dumps(rec) + "\n")
            log.flush()

    # every replica must agree with rank 0's, in both implementations
    for side, name in ((ours, "ours"), (theirs, "torch")):
        if side is None:
            continue
        mine = side.flat()
        r0 = mine.copy()
        pg.broadcast(r0, root=0)
        if not np.array_equal(r0, mine):
            raise SystemExit(f"rank {rank}: {name} replica differs from rank 0")

    sb = {}
    if ours is not None:
        sb["dtrain_state_bytes"] = ours.state_bytes()
    if theirs is not None:
        sb["torch_state_bytes"] = theirs.state_bytes()
    allsb = [None] * world
    dist.all_gather_object(allsb, sb)

    if a.phase == "first":
        if ours is not None:
            checkpoint.save(ck_ours, end, rank, world, ours.state(), pg.barrier)
        if theirs is not None:
            if isinstance(theirs.opt, ZeroRedundancyOptimizer):
                theirs.opt.consolidate_state_dict(to=0)
            if rank == 0:
                torch.save({"model": tmodel.state_dict(), "opt": theirs.opt.state_dict(), "step": end},
                           ck_torch + ".tmp")
                os.replace(ck_torch + ".tmp", ck_torch)
            dist.barrier()

    if rank == 0:
        arrays = {}
        if ours is not None:
            arrays["dtrain"] = ours.flat()
        if theirs is not None:
            arrays["torch"] = theirs.flat()
        np.savez(a.out + ".npz", **arrays)
        with open(a.out + ".meta.json", "w") as f:
            json.dump({"args": vars(a), "world": world, "torch": torch.__version__, "numpy": np.__version__,
                       "n_params": int(sum(p.numel() for p in model.parameters())),
                       "state_bytes_per_rank": allsb}, f)
    dist.barrier()
    dist.destroy_process_group()
    pg.barrier()
    pg.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
