"""Train a GPT, single-process or distributed (CLI of dtrain/train.py:31-191).

    python -m dtrain_b200.train --mode single ...
    python -m dtrain_b200.launch --nproc 8 -- python -m dtrain_b200.train --mode ddp --dtype bfloat16 ...
    python -m dtrain_b200.launch --nproc 8 -- python -m dtrain_b200.train --mode zero ...

Every reference flag is kept; additions: ``--dtype bfloat16`` (bf16 compute with
fp32 masters/grads on the sm_100a kernels), ``--data synthetic`` with ``--vocab``,
``--device``, ``--algo {ring,direct}`` plus ``--ar-method {auto,oneshot,twoshot,nvls}``.

``--mode single --emulate-world W`` runs the exact global batch of a W-rank job
in one process (the reference for equivalence tests).  One JSON line per step
goes to --log: step, lr, loss, grad_norm, step_s, tokens_per_s, comm_wait_s
(plus step_ms_device on GPUs); ZeRO appends optimizer_state_bytes_per_rank.
stderr messages match the reference ("resumed from step N", "injected failure
at step N").
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import sys
import time

import numpy as np
import torch

from .models.gpt import GPT, GPTConfig, train_flops_per_token
from .ops.optim import AdamW, clip_scale
from .utils import checkpoint
from .utils.data import CharData, SyntheticData, load_text, lr_at, rank_batch


_PRECISION = {"fp64": "float64", "fp32": "float32", "bf16": "bfloat16"}


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["single", "ddp", "zero"], default="single")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--batch", type=int, default=8, help="sequences per rank per micro-step")
    ap.add_argument("--accum", type=int, default=1, help="gradient-accumulation micro-steps")
    ap.add_argument("--ctx", type=int, default=64)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--dtype", default="float32", help="float64 | float32 | bfloat16 (bf16 compute, fp32 masters)")
    ap.add_argument("--precision", choices=sorted(_PRECISION), default=None,
                    help="short form of --dtype: fp64 | fp32 | bf16")
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--warmup", type=int, default=0, help="linear warm-up steps, then cosine decay to lr/10")
    ap.add_argument("--wd", type=float, default=0.1)
    ap.add_argument("--clip", type=float, default=1.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--data", default=None, help="text file, or 'synthetic' (default: tiny shakespeare)")
    ap.add_argument("--vocab", type=int, default=50304, help="vocabulary for --data synthetic")
    ap.add_argument("--emulate-world", type=int, default=1)
    ap.add_argument("--bucket-mb", type=float, default=1.0)
    ap.add_argument("--no-overlap", action="store_true")
    ap.add_argument("--algo", choices=["ring", "direct"], default="ring")
    ap.add_argument("--ar-method", choices=["auto", "oneshot", "twoshot", "nvls"], default="auto",
                    help="GPU all-reduce data movement; nvls reduces in the NVSwitch (multicast memory)")
    ap.add_argument("--device", default=None, help="cpu | cuda (default: cuda for bfloat16, else cpu)")
    ap.add_argument("--gather-gemm", action="store_true",
                    help="ZeRO on GPUs: let the forward GEMMs pull their weights from the other ranks (all-gather "
                         "fused into the GEMM) instead of gathering every parameter in the optimizer kernel")
    ap.add_argument("--cuda-graph", action="store_true",
                    help="GPU: capture forward+backward of a step in a CUDA graph and replay it (removes the "
                         "per-kernel host launch cost); under DDP the bucket all-reduces launched from the "
                         "grad-ready hooks are captured with it; the optimizer runs eagerly")
    ap.add_argument("--ckpt-dir", default=None)
    ap.add_argument("--ckpt-every", type=int, default=0)
    ap.add_argument("--async-ckpt", action="store_true",
                    help="write checkpoint shards in a background thread; each checkpoint is committed "
                         "(barrier, manifest, LATEST) at the next checkpoint or at the end of the run")
    ap.add_argument("--resume", action="store_true", help="resume from the latest checkpoint if any")
    ap.add_argument("--stop-after", type=int, default=-1, help="stop cleanly after this many steps (preemption)")
    ap.add_argument("--fail-at-step", type=int, default=-1, help="fault injection: crash at this step")
    ap.add_argument("--fail-rank", type=int, default=1)
    ap.add_argument("--log", default=None)
    ap.add_argument("--save-params", default=None, help="write final parameters (.npz) from rank 0")
    a = ap.parse_args(argv)
    if a.precision is not None:
        a.dtype = _PRECISION[a.precision]
    return a


def _default_device(a) -> torch.device:
    if a.device:
        d = torch.device(a.device)
        if d.type == "cuda" and d.index is None:
            d = torch.device("cuda", int(os.environ.get("LOCAL_RANK", os.environ.get("RANK", "0"))))
        return d
    if a.dtype in ("bfloat16", "bf16"):
        return torch.device("cuda", int(os.environ.get("LOCAL_RANK", os.environ.get("RANK", "0"))))
    return torch.device("cpu")


@contextlib.contextmanager
def _nvtx(name: str):
    """NVTX range around a phase of the step (visible in Nsight timelines; no-op on CPU)."""
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class Trainer:
    """One training job: model, parallel wrapper, optimizer and the per-step loop body.

    ``step(step_idx, batches)`` runs one optimizer step over the given micro-batches
    (host arrays or tensors; copied to the device from pinned memory) and returns
    the step's mean loss as a Python float.
    """

    def __init__(self, a, cfg: GPTConfig, device: torch.device, pg=None):
        self.a, self.cfg, self.device, self.pg = a, cfg, device, pg
        self.rank, self.world = (pg.rank, pg.world) if pg is not None else (0, 1)
        self.gpu = device.type == "cuda"
        if self.gpu:
            torch.cuda.set_device(device)
        self.model = GPT(cfg, seed=a.seed)
        self.params = list(self.model.parameters())
        self.ddp = self.zero = self.opt = None
        if self.gpu and a.mode == "single":
            self.model.flatten(device)
        elif not self.gpu:
            pass
        if a.mode == "ddp":
            from .parallel.ddp import DDP
            self.ddp = DDP(self.model, pg, bucket_mb=a.bucket_mb, overlap=not a.no_overlap, algo=a.algo,
                           method=a.ar_method)
        elif a.mode == "zero":
            from .parallel.zero import ZeroAdamW
            self.zero = ZeroAdamW(self.model, pg, max_grad_norm=a.clip, lr=a.lr, weight_decay=a.wd,
                                  gather_gemm=getattr(a, "gather_gemm", False))
        if self.zero is None:
            fp = self.model.flat
            if fp is not None and self.gpu:
                # one flat AdamW over all parameters (fused kernel, also refreshes the bf16 copy)
                self.opt = AdamW([fp.master], lr=a.lr, weight_decay=a.wd, work=[fp.work])
            else:
                self.opt = AdamW([p.data for p in self.params], lr=a.lr, weight_decay=a.wd)
        self._sq = torch.zeros(1, dtype=torch.float64, device=device) if self.gpu else None
        self._pinned: dict = {}
        # CUDA-graph state (--cuda-graph): static inputs, the captured forward+backward,
        # its loss output, and how many of this extension's kernels one replay launches
        self.use_graph = bool(getattr(a, "cuda_graph", False)) and self.gpu
        # GPU DDP: the gradient sync (bucket all-reduces launched from the grad-ready
        # hooks, their join and the gradient norm) is captured with forward+backward
        self.sync_in_graph = self.use_graph and self.ddp is not None and self.ddp.gpu
        self._graph = None
        self._graph_key = None
        self._static_in: list = []
        self._static_loss = None
        self.graph_launches = 0
        self.graph_replays = 0
        self.last_grad_norm = 0.0
        self.comm_wait = 0.0

    # -------------------------------------------------------------- inputs
    def to_device(self, arr, key) -> torch.Tensor:
        if isinstance(arr, torch.Tensor) and arr.device == self.device:
            return arr if arr.dtype == torch.int64 else arr.long()
        t = torch.as_tensor(np.asarray(arr, dtype=np.int64))
        if not self.gpu:
            return t
        buf = self._pinned.get(key)
        if buf is None or buf.shape != t.shape:
            buf = torch.empty(t.shape, dtype=torch.int64, pin_memory=True)
            self._pinned[key] = buf
        buf.copy_(t)
        return buf.to(self.device, non_blocking=True)

    # ----------------------------------------------------------------- step
    def set_lr(self, lr: float):
        if self.zero is not None:
            self.zero.opt.lr = lr
        else:
            self.opt.lr = lr

    def _fwd_bwd(self, batches_dev, n_micro: int):
        """Forward and backward over all micro-batches (device tensors); returns the mean loss."""
        if self.ddp is not None and self.gpu:
            self.ddp.trace_begin()
        loss_acc = torch.zeros((), dtype=torch.float64, device=self.device)
        for mi, vrs in enumerate(batches_dev):
            last = mi == len(batches_dev) - 1
            for xt, yt in vrs:
                _, loss = self.model(xt, yt)
                scaled = loss * (1.0 / n_micro)
                if self.ddp is not None and not last:
                    with self.ddp.no_sync():
                        scaled.backward()
                else:
                    scaled.backward()
                loss_acc = loss_acc + loss.detach().double() / n_micro
        return loss_acc

    def _step_graph(self, batches):
        """Forward+backward by CUDA-graph replay.  The first call (and any change of
        batch shapes) warms up on a side stream and captures; every call copies its
        batch into the static input buffers first.  Gradients land in the flat
        gradient buffer, whose addresses the graph keeps."""
        key = tuple(tuple((tuple(np.shape(x)), tuple(np.shape(y))) for x, y in vrs) for vrs in batches)
        n_micro = sum(len(v) for v in batches)
        if self._graph is None or key != self._graph_key:
            from .ops import kernels as K
            self._static_in = [[(self.to_device(x, ("gx", mi, vi)).clone(), self.to_device(y, ("gy", mi, vi)).clone())
                                for vi, (x, y) in enumerate(vrs)] for mi, vrs in enumerate(batches)]
            side = torch.cuda.Stream(device=self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self.model.zero_grad()
                    self._fwd_bwd(self._static_in, n_micro)
                    if self.sync_in_graph:
                        self.ddp.finish()
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            if self.pg is not None and self.gpu:
                self.pg.check()
            self.model.zero_grad()
            g = torch.cuda.CUDAGraph()
            before = K.launch_count()
            with torch.cuda.graph(g):
                self._static_loss = self._fwd_bwd(self._static_in, n_micro)
                if self.sync_in_graph:
                    self.ddp.finish()
            self.graph_launches = K.launch_count() - before
            self._graph, self._graph_key = g, key
        for mi, vrs in enumerate(batches):
            for vi, (x, y) in enumerate(vrs):
                sx, sy = self._static_in[mi][vi]
                sx.copy_(self.to_device(x, ("x", mi, vi)), non_blocking=True)
                sy.copy_(self.to_device(y, ("y", mi, vi)), non_blocking=True)
        self._graph.replay()
        self.graph_replays += 1
        return self._static_loss

    def _eager_fwd_bwd(self, batches):
        """Forward and backward over host or device micro-batches, kernels launched eagerly."""
        if self.ddp is not None and self.gpu:
            self.ddp.trace_begin()
        n_micro = sum(len(v) for v in batches)
        loss_acc = torch.zeros((), dtype=torch.float64, device=self.device) if self.gpu else 0.0
        for mi, vrs in enumerate(batches):
            last = mi == len(batches) - 1
            for x, y in vrs:
                xt = self.to_device(x, ("x", mi))
                yt = self.to_device(y, ("y", mi))
                _, loss = self.model(xt, yt)
                scaled = loss * (1.0 / n_micro)
                if self.ddp is not None and not last:
                    with self.ddp.no_sync():
                        scaled.backward()
                else:
                    scaled.backward()
                if self.gpu:
                    loss_acc = loss_acc + loss.detach().double() / n_micro
                else:
                    loss_acc += float(loss.detach()) / n_micro
        return loss_acc

    def step(self, batches, return_loss: bool = True):
        """``batches``: list over micro-steps of lists over virtual ranks of (x, y)."""
        a = self.a
        if self.use_graph:
            with _nvtx("forward+backward+gradient sync (graph replay)" if self.sync_in_graph
                       else "forward+backward (graph replay)"):
                loss_acc = self._step_graph(batches)
            with _nvtx("gradient sync"):
                if self.ddp is not None and not self.sync_in_graph:
                    before = self.ddp.comm_wait_s
                    self.ddp.finish()
                    self.comm_wait = self.ddp.comm_wait_s - before
            with _nvtx("optimizer"):
                if self.zero is not None:
                    self.zero.step()
                else:
                    self._clip_and_update()
            return self._reduce_loss(loss_acc) if return_loss else None
        self.model.zero_grad()
        with _nvtx("forward+backward"):
            loss_acc = self._eager_fwd_bwd(batches)
        with _nvtx("gradient sync"):
            if self.ddp is not None:
                before = self.ddp.comm_wait_s
                self.ddp.finish()
                self.comm_wait = self.ddp.comm_wait_s - before
        with _nvtx("optimizer"):
            if self.zero is not None:
                self.zero.step()
            else:
                self._clip_and_update()
        if not return_loss:
            return None
        return self._reduce_loss(loss_acc)

    def _clip_and_update(self):
        a = self.a
        fp = self.model.flat
        if self.gpu and fp is not None and fp.work is not None:
            if self.ddp is not None and self.ddp.gpu and self.ddp.fused_norm:
                # the all-reduce kernels already summed the squares of the averaged gradient
                self._sq = self.ddp.sq_norm
            else:
                from .ops import kernels as K
                K.grad_sqnorm(fp.grad, self._sq)
            self.opt.step([fp.grad], sq_norm=self._sq, max_norm=a.clip if a.clip else 0.0)
            return
        grads = [p.grad for p in self.params]
        sq = sum(float(torch.dot(g.reshape(-1).double(), g.reshape(-1).double())) for g in grads if g is not None)
        self.last_grad_norm = math.sqrt(sq)
        s = clip_scale(sq, a.clip) if a.clip else 1.0
        self.opt.step([g * s if g is not None else None for g in grads])

    def grad_norm(self) -> float:
        if self.zero is not None:
            return self.zero.last_grad_norm
        if self.gpu and self.model.flat is not None and self.model.flat.work is not None:
            return math.sqrt(float(self._sq.item()))
        return self.last_grad_norm

    def max_over_ranks(self, value: float) -> float:
        """Max of a per-rank host value (the collectives sum, so each rank fills its own slot)."""
        if self.pg is None or self.world == 1:
            return float(value)
        if self.gpu:
            v = torch.zeros(self.world, dtype=torch.float32, device=self.device)
            v[self.rank] = float(value)
            self.pg.allreduce(v, "direct")
            out = float(v.max().item())
            self.pg.check()
            return out
        v = np.zeros(self.world)
        v[self.rank] = value
        self.pg.allreduce(v)
        return float(v.max())

    def _reduce_loss(self, loss_acc) -> float:
        pg = self.pg
        if pg is None:
            return float(loss_acc)
        if self.gpu:
            lt = loss_acc.reshape(1).float()
            pg.allreduce(lt, "direct")
            val = float(lt.item()) / self.world
            pg.check()
            return val
        l = np.array([loss_acc])
        pg.allreduce(l)
        return float(l[0]) / self.world

    # ---------------------------------------------------------- checkpoint
    def state(self) -> dict:
        if self.zero is not None:
            self.zero.gather_params()
            sd = self.zero.state_dict()
            return {"params": self.zero.flat, "t": sd["t"], "m": sd["m"][0], "v": sd["v"][0]}
        sd = self.opt.state_dict()
        st = {"params": torch.cat([p.detach().reshape(-1) for p in self.params]), "t": sd["t"]}
        if len(sd["m"]) == 1 and len(self.params) > 1:  # flat optimizer: split per parameter
            fp = self.model.flat
            for i, (o, k) in enumerate(zip(fp.offsets, fp.numels)):
                st[f"m{i}"] = sd["m"][0][o:o + k].reshape(self.params[i].shape)
                st[f"v{i}"] = sd["v"][0][o:o + k].reshape(self.params[i].shape)
        else:
            st.update({f"m{i}": m for i, m in enumerate(sd["m"])})
            st.update({f"v{i}": v for i, v in enumerate(sd["v"])})
        return st

    def load_state(self, st: dict):
        dev = self.device
        if self.zero is not None:
            with torch.no_grad():
                self.zero.flat.copy_(torch.from_numpy(st["params"]).to(dev, self.zero.flat.dtype))
            self.zero.load_state_dict({"t": st["t"], "m": [torch.from_numpy(st["m"]).to(dev)],
                                       "v": [torch.from_numpy(st["v"]).to(dev)]})
            return
        flat_params = torch.from_numpy(st["params"])
        with torch.no_grad():
            off = 0
            for p in self.params:
                p.copy_(flat_params[off:off + p.numel()].reshape(p.shape).to(dev, p.dtype))
                off += p.numel()
        n = len(self.params)
        fp = self.model.flat
        if len(self.opt.m) == 1 and n > 1:
            m = torch.cat([torch.from_numpy(st[f"m{i}"]).reshape(-1) for i in range(n)]).to(dev)
            v = torch.cat([torch.from_numpy(st[f"v{i}"]).reshape(-1) for i in range(n)]).to(dev)
            self.opt.load_state_dict({"t": st["t"], "m": [m], "v": [v]})
        else:
            self.opt.load_state_dict({"t": st["t"], "m": [torch.from_numpy(st[f"m{i}"]) for i in range(n)],
                                      "v": [torch.from_numpy(st[f"v{i}"]) for i in range(n)]})
        if fp is not None:
            fp.refresh_work()

    def barrier(self):
        if self.pg is None:
            return
        self.pg.barrier()
        if self.gpu:
            self.pg.synchronize()


def make_group(a, device):
    if a.mode == "single":
        return None
    if device.type == "cuda":
        from .parallel.nvlink import from_env
        if "STORE_ADDR" not in os.environ:
            import datetime

            import torch.distributed as dist
            if not dist.is_initialized():
                dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=float(
                    os.environ.get("DTRAIN_TIMEOUT", "60"))))
        return from_env(device, nvls=(a.ar_method == "nvls") or None)
    from .parallel.comm import init_from_env
    return init_from_env()


class _StopRequest:
    """SIGTERM (the launcher stopping an attempt) becomes a flag checked between
    steps.  Python runs a signal handler only once the current call returns, so a
    worker blocked on the GPU - e.g. in a collective waiting for a peer that is gone -
    would otherwise only stop after that wait timed out.  With a GPU process group the
    signal also reaches a watcher thread (through ``signal.set_wakeup_fd``, written by
    the C-level handler at once), which aborts the group: the waiting collective
    kernels give up immediately and the blocked call returns."""

    def __init__(self):
        self.requested = False
        self._pipe = None

    def install(self):
        import signal

        def handler(signum, frame):
            self.requested = True

        signal.signal(signal.SIGTERM, handler)
        return self

    def abort_on_signal(self, pg):
        """Once the GPU process group exists: SIGTERM also aborts it (watcher thread)."""
        import signal
        import threading

        if pg is not None and getattr(pg, "backend", "") == "nvlink":
            r, w = os.pipe()
            os.set_blocking(w, False)
            signal.set_wakeup_fd(w, warn_on_full_buffer=False)
            self._pipe = (r, w)

            def watch():
                while True:
                    try:
                        data = os.read(r, 64)
                    except OSError:
                        return
                    if not data:
                        return
                    if signal.SIGTERM in data:
                        self.requested = True
                        try:
                            pg.abort()
                        except Exception:  # noqa: BLE001 - stopping anyway
                            pass
                        return

            threading.Thread(target=watch, name="sigterm-abort", daemon=True).start()


def main(argv=None):
    a = parse(argv)
    stop = _StopRequest()
    device = _default_device(a)
    if device.type == "cuda":
        stop.install()  # CPU workers keep the default: nothing of theirs runs on a GPU
    if a.data == "synthetic":
        data = SyntheticData(a.vocab)
        vocab = a.vocab
        batch_fn = lambda step, micro, r, w: data.rank_batch(step, micro, a.batch, a.ctx, a.seed, r, w)  # noqa: E731
    else:
        cd = CharData(load_text(a.data))
        vocab = cd.vocab
        batch_fn = lambda step, micro, r, w: rank_batch(cd.train, step, micro, a.batch, a.ctx, a.seed, r, w)  # noqa: E731
    cfg = GPTConfig(vocab=vocab, ctx=a.ctx, dim=a.dim, heads=a.heads, layers=a.layers, dtype=a.dtype)
    pg = make_group(a, device)
    if device.type == "cuda":
        stop.abort_on_signal(pg)
    tr = Trainer(a, cfg, device, pg)
    rank, world = tr.rank, tr.world

    start = 0
    if a.resume and a.ckpt_dir and checkpoint.latest(a.ckpt_dir):
        step, st = checkpoint.load(checkpoint.latest(a.ckpt_dir), rank, world)
        tr.load_state(st)
        start = step
        print(f"[rank {rank}] resumed from step {step}", file=sys.stderr, flush=True)

    log = open(a.log, "a") if (a.log and rank == 0) else None
    restarts = int(os.environ.get("DTRAIN_RESTART_COUNT", "0"))
    tokens_per_step = a.batch * a.ctx * a.accum * max(world, a.emulate_world)
    saver = checkpoint.AsyncSaver() if (a.async_ckpt and a.ckpt_dir and a.ckpt_every) else None
    flops_per_token = train_flops_per_token(cfg)
    vworlds = a.emulate_world if a.mode == "single" else 1
    # GPU jobs that log also record the device time of each step (every rank takes
    # part in the max, so the decision depends only on the shared flags)
    timing = bool(tr.gpu and a.log)
    if timing:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    for step in range(start, a.steps):
        if stop.requested:
            if tr.gpu:
                torch.cuda.synchronize()  # every queued kernel is bounded: this returns
            print(f"[rank {rank}] stopping at step {step} (SIGTERM)", file=sys.stderr, flush=True)
            return 143
        if step == a.fail_at_step and rank == a.fail_rank and restarts == 0:
            if tr.gpu:
                torch.cuda.synchronize()  # leave between steps, nothing in flight
            print(f"[rank {rank}] injected failure at step {step}", file=sys.stderr, flush=True)
            os._exit(17)
        t0 = time.perf_counter()
        if timing:
            ev0.record()
        lr = lr_at(step, a)
        tr.set_lr(lr)
        batches = []
        for micro in range(a.accum):
            vr_batches = []
            for vr in range(vworlds):
                r = vr if a.mode == "single" else rank
                w = vworlds if a.mode == "single" else world
                vr_batches.append(batch_fn(step, micro, r, w))
            batches.append(vr_batches)
        loss = tr.step(batches)
        dt = time.perf_counter() - t0
        dev_ms = None
        if timing:
            ev1.record()
            ev1.synchronize()
            dev_ms = tr.max_over_ranks(ev0.elapsed_time(ev1))
        if log:
            rec = {"step": step + 1, "lr": lr, "loss": loss, "grad_norm": tr.grad_norm(), "step_s": dt,
                   "tokens_per_s": tokens_per_step / dt, "comm_wait_s": tr.comm_wait}
            if dev_ms is not None:  # device-timed (CUDA events on the training stream), max over ranks
                rec["step_ms_max_over_ranks"] = dev_ms
                rec["tokens_per_s_device"] = tokens_per_step / (dev_ms / 1e3)
                rec["model_tflops_per_s_per_gpu"] = flops_per_token * tokens_per_step / world / (dev_ms / 1e3) / 1e12
            log.write(json.dumps(rec) + "\n")
            log.flush()
        if a.ckpt_dir and a.ckpt_every and (step + 1) % a.ckpt_every == 0:
            if saver is not None:
                saver.commit(tr.barrier)
                saver.start(a.ckpt_dir, step + 1, rank, world, tr.state())
            else:
                checkpoint.save(a.ckpt_dir, step + 1, rank, world, tr.state(), tr.barrier)
        if a.stop_after >= 0 and step + 1 >= a.stop_after:
            break
    if saver is not None:
        saver.commit(tr.barrier)

    if a.save_params:
        if tr.zero is not None:
            tr.zero.gather_params()
        if rank == 0:
            np.savez(a.save_params, **{n: p.detach().float().cpu().numpy() if p.dtype == torch.bfloat16
                                        else p.detach().cpu().numpy() for n, p in tr.model.named_parameters()})
    if tr.zero is not None and rank == 0 and log:
        log.write(json.dumps({"optimizer_state_bytes_per_rank": tr.zero.state_bytes()}) + "\n")
    if pg is not None:
        tr.barrier()
        pg.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
