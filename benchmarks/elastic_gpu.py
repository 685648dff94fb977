"""Elastic ZeRO-1 run on GPUs: a job that crashes and restarts against the same job run
through without a crash (the reference's crash/restart/resume check,
tests/test_training.py:102-111 there, at the scale of its 1.3B configuration).

    python benchmarks/elastic_gpu.py --gpus 8 [--model 1.3b] [--steps 130] [--ckpt-every 50]
        [--fail-at-step 120] [--out result.json]

Both jobs go through the restart-all launcher (``dtrain_b200.launch``) with the same
flags: ZeRO-1, bf16 compute with fp32 masters, synthetic tokens, the forward+backward
CUDA graph.  The second job also checkpoints every ``--ckpt-every`` steps (sharded,
SHA-256 manifest, atomic LATEST) and its rank ``--fail-rank`` leaves at
``--fail-at-step`` (between steps, after synchronising its GPU); the launcher stops the
group (its SIGTERM aborts the survivors' waiting collectives) and starts a
second attempt that resumes from the latest checkpoint.  No NVLS / multicast memory is
used (a rank leaves on purpose).

Prints one JSON line: whether every logged loss of the restarted job equals the
uninterrupted job's bit for bit, the step it resumed from, and the uninterrupted
job's throughput (median of the per-step device tokens/s after ``--skip`` steps).
``--model tiny`` runs a small model, and ``--device cpu`` fp64 CPU ranks, for a quick
check of the script itself.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MODELS = {
    "1.3b": ["--dim", "2048", "--heads", "16", "--layers", "24", "--ctx", "2048", "--batch", "4", "--vocab", "50304"],
    "gpt2-small": ["--dim", "768", "--heads", "12", "--layers", "12", "--ctx", "1024", "--batch", "16",
                   "--vocab", "50304"],
    "tiny": ["--dim", "64", "--heads", "2", "--layers", "2", "--ctx", "32", "--batch", "2", "--vocab", "128"],
}


def run(world, flags, log, restarts, timeout, extra_env):
    cmd = [sys.executable, "-m", "dtrain_b200.launch", "--nproc", str(world), "--max-restarts", str(restarts),
           "--timeout", str(timeout), "--", sys.executable, "-m", "dtrain_b200.train", "--log", log, *flags]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), **extra_env)
    t0 = time.time()
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    recs = [json.loads(line) for line in open(log)] if os.path.exists(log) else []
    return r, recs, time.time() - t0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--model", choices=sorted(MODELS), default="1.3b")
    ap.add_argument("--mode", choices=["zero", "ddp"], default="zero")
    ap.add_argument("--steps", type=int, default=130)
    ap.add_argument("--ckpt-every", type=int, default=50)
    ap.add_argument("--fail-at-step", type=int, default=120)
    ap.add_argument("--fail-rank", type=int, default=1)
    ap.add_argument("--timeout", type=float, default=60.0,
                    help="collective timeout (s); a stopped worker aborts its waits at once, so this only bounds skew")
    ap.add_argument("--skip", type=int, default=5, help="steps left out of the throughput median")
    ap.add_argument("--device", choices=["cuda", "cpu"], default="cuda")
    ap.add_argument("--workdir", default=None)
    ap.add_argument("--out", default=None)
    a = ap.parse_args()

    work = a.workdir or tempfile.mkdtemp(prefix="dtb-elastic-")
    os.makedirs(work, exist_ok=True)
    common = ["--mode", a.mode, "--steps", str(a.steps), "--data", "synthetic", "--lr", "3e-4", "--warmup", "10",
              *MODELS[a.model]]
    if a.device == "cuda":
        common += ["--dtype", "bfloat16", "--cuda-graph"]
        env = {"NCCL_NVLS_ENABLE": "0", "DTB_NVLS": "0"}
    else:
        common += ["--dtype", "float64", "--device", "cpu"]
        env = {}
    ck = os.path.join(work, "ckpt")
    try:
        clean, clean_log, t_clean = run(a.gpus, common, os.path.join(work, "clean.jsonl"), 0, a.timeout, env)
        if clean.returncode != 0:
            sys.stderr.write(clean.stderr[-4000:])
            raise SystemExit(f"uninterrupted job failed with {clean.returncode}")
        crashed, crash_log, t_crash = run(
            a.gpus, [*common, "--ckpt-dir", ck, "--ckpt-every", str(a.ckpt_every), "--resume",
                     "--fail-at-step", str(a.fail_at_step), "--fail-rank", str(a.fail_rank)],
            os.path.join(work, "crashed.jsonl"), 1, a.timeout, env)
        if crashed.returncode != 0:
            sys.stderr.write(crashed.stderr[-4000:])
            raise SystemExit(f"restarted job failed with {crashed.returncode}")
    finally:
        if a.workdir is None:
            shutil.rmtree(work, ignore_errors=True)

    loss_clean = {r["step"]: r["loss"] for r in clean_log if "loss" in r}
    # the restarted job logs steps before the crash (attempt 0) and from the checkpoint
    # on (attempt 1); a step logged twice must give the same loss both times
    loss_crash: dict[int, list[float]] = {}
    for r in crash_log:
        if "loss" in r:
            loss_crash.setdefault(r["step"], []).append(r["loss"])
    resumed = [line for line in crashed.stderr.splitlines() if "resumed from step" in line]
    identical = (set(loss_crash) == set(loss_clean)
                 and all(all(v == loss_clean[s] for v in vs) for s, vs in loss_crash.items()))
    dev = [r.get("tokens_per_s_device", r.get("tokens_per_s")) for r in clean_log if "loss" in r][a.skip:]
    out = {
        "config": {"model": a.model, "mode": a.mode, "gpus": a.gpus, "steps": a.steps, "ckpt_every": a.ckpt_every,
                   "fail_at_step": a.fail_at_step, "fail_rank": a.fail_rank, "device": a.device,
                   "flags": " ".join(common)},
        "loss_trajectory_bit_identical": identical,
        "steps_compared": len(loss_clean),
        "steps_logged_twice": sorted(s for s, vs in loss_crash.items() if len(vs) > 1),
        "resumed": resumed[-1].strip() if resumed else None,
        "injected": any("injected failure" in line for line in crashed.stderr.splitlines()),
        "restarted": "restarting" in crashed.stderr,
        "tokens_per_s_median": statistics.median(dev) if dev else None,
        "final_loss": loss_clean.get(a.steps),
        "wall_s": {"uninterrupted": round(t_clean, 1), "crash_and_restart": round(t_crash, 1)},
    }
    line = json.dumps(out)
    print(line)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    if not identical:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
