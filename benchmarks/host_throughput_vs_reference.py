"""Host (CPU rank) training throughput of this stack against the reference's own CLI.

    python benchmarks/host_throughput_vs_reference.py [--steps 30] [--out results.json]

Runs the reference's published throughput benchmark (its benchmarks/scaling.sh: GPT
with 4 layers, d 128, 4 heads, ctx 64, 8 sequences per rank, fp32, one BLAS thread per
rank, ranks over TCP loopback through the launcher) twice on this machine: once with
``dtrain_b200`` and once with the reference installed in baseline/_ref.  Both read
the same generated character corpus (the reference would otherwise download
tiny-shakespeare).  Reports the median ``tokens_per_s`` of each run's JSONL log after
the first five steps.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODEL = ["--dim", "128", "--heads", "4", "--layers", "4", "--ctx", "64", "--batch", "8", "--lr", "1e-3",
         "--warmup", "10"]
RUNS = [("single", 1, []), ("ddp", 2, []), ("ddp", 2, ["--no-overlap"]), ("zero", 2, []),
        ("ddp", 4, []), ("ddp", 4, ["--no-overlap"]), ("zero", 4, [])]


def _corpus(path: str):
    rng = np.random.default_rng(0)
    words = ["the", "king", "and", "queen", "of", "rome", "said", "to", "thee", "now", "thou", "art"]
    with open(path, "w") as f:
        f.write(" ".join(rng.choice(words, 200_000)) + "\n")


def _run(pkg: str, mode: str, nproc: int, extra: list, steps: int, data: str, log: str) -> float:
    env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1", MKL_NUM_THREADS="1")
    if pkg == "dtrain":
        env["PYTHONPATH"] = os.path.join(ROOT, "baseline", "_ref")
        extra_pkg = []
    else:
        env["PYTHONPATH"] = ROOT
        extra_pkg = ["--dtype", "float32", "--device", "cpu"]
    train = [sys.executable, "-m", f"{pkg}.train", "--mode", mode, "--steps", str(steps), "--data", data,
             "--log", log] + MODEL + extra + extra_pkg
    cmd = train if nproc == 1 else [sys.executable, "-m", f"{pkg}.launch", "--nproc", str(nproc), "--"] + train
    subprocess.run(cmd, env=env, cwd=ROOT, check=True, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL,
                   timeout=1800)
    tps = [json.loads(line)["tokens_per_s"] for line in open(log) if '"tokens_per_s"' in line]
    return float(np.median(tps[5:] if len(tps) > 5 else tps))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    if not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "dtrain")):
        raise SystemExit("the reference is not installed in baseline/_ref")
    rows = []
    with tempfile.TemporaryDirectory() as tmp:
        data = os.path.join(tmp, "corpus.txt")
        _corpus(data)
        for mode, nproc, extra in RUNS:
            row = {"mode": mode + ("-nooverlap" if extra else ""), "world": nproc}
            for pkg in ("dtrain_b200", "dtrain"):
                log = os.path.join(tmp, f"{pkg}_{mode}_{nproc}_{len(extra)}.jsonl")
                row[pkg] = _run(pkg, mode, nproc, extra, a.steps, data, log)
            row["ratio"] = row["dtrain_b200"] / row["dtrain"]
            rows.append(row)
            print(json.dumps(row), flush=True)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rows, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
