"""Whole cross-check of this framework against PyTorch on host ranks, plus the
host throughput comparison, summarised in one JSON file.

    python benchmarks/run_torch_crosscheck.py --out benchmarks/results/xcheck [--quick] [--skip-bench]

Counterpart of the reference's benchmarks/run_torch_crosscheck.py (same
summary.json sections, so benchmarks/torch_report.py renders either):
  adamw_only   this AdamW vs torch.optim.AdamW on identical parameters/gradients
  collective   ring all-reduce vs gloo at W = 2, 3, 4 (torch_allreduce.py)
  equivalence  DDP (AdamW and SGD) and ZeRO-1 step by step vs torch DDP /
               ZeroRedundancyOptimizer, float64 and float32, several W
  resume       checkpoint in one set of processes, resume in another, vs an
               uninterrupted run, in both libraries
  throughput   host step time of each library alone (--only), and all-reduce speed
Everything runs through ``python -m dtrain_b200.launch`` on this machine (CPU, gloo
over loopback).
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

PY = sys.executable
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)


_DATA: list = []  # ["--data", path] for torch_crosscheck.py runs


def _launch(nproc: int, script: str, args: list, tmp: str, timeout: int = 1800):
    init = os.path.join(tmp, f"gloo_{os.getpid()}_{len(os.listdir(tmp))}")
    extra = _DATA if script == "torch_crosscheck.py" else []
    cmd = [PY, "-m", "dtrain_b200.launch", "--nproc", str(nproc), "--timeout", "120", "--",
           PY, os.path.join(HERE, script), "--torch-init", init, *extra, *args]
    env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1", MKL_NUM_THREADS="1",
               PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout, cwd=ROOT)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd)} failed:\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}")


def _jsonl(path: str) -> list:
    with open(path) as f:
        return [json.loads(line) for line in f]


def _load() -> list:
    with open("/proc/loadavg") as f:
        return f.read().split()[:3]


def adamw_only(steps: int) -> dict:
    import torch
    from dtrain_b200.ops.optim import AdamW
    out = {}
    for dt in ("float64", "float32"):
        rng = np.random.default_rng(1)
        p0 = rng.standard_normal(100_000).astype(dt)
        ours = torch.from_numpy(p0.copy())
        theirs = torch.from_numpy(p0.copy()).requires_grad_()
        od = AdamW([ours], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
        ot = torch.optim.AdamW([theirs], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
        diffs = []
        for _ in range(steps):
            # gradient magnitudes from 1e-12 to 1: some far below eps, some far above
            g = (rng.standard_normal(p0.size) * 10.0 ** rng.uniform(-12, 0, p0.size)).astype(dt)
            od.step([torch.from_numpy(g.copy())])
            theirs.grad = torch.from_numpy(g.copy())
            ot.step()
            diffs.append(float(torch.max(torch.abs(ours - theirs.detach()))))
        out[dt] = {"param_maxabs_diff_per_step": diffs, "param_maxabs_diff_max": max(diffs)}
    return out


def equivalence(out_dir: str, tmp: str, steps: int) -> list:
    res = []
    for mode, worlds in (("ddp", (1, 2, 4)), ("ddp-sgd", (1, 2, 4)), ("zero", (2, 4))):
        for dt in ("float64", "float32"):
            for w in worlds:
                name = os.path.join(out_dir, f"{mode}_w{w}_{dt}")
                extra = ["--mode", "ddp", "--opt", "sgd", "--lr", "0.1"] if mode == "ddp-sgd" else ["--mode", mode]
                _launch(w, "torch_crosscheck.py", [*extra, "--steps", str(steps), "--dtype", dt, "--out", name], tmp)
                rs = _jsonl(name + ".jsonl")
                with open(name + ".meta.json") as f:
                    meta = json.load(f)
                e = {"mode": mode, "world": w, "dtype": dt, "steps": len(rs), "n_params": meta["n_params"],
                     "param_maxabs_diff_per_step": [r["param_maxabs_diff"] for r in rs],
                     "param_maxabs_diff_max": max(r["param_maxabs_diff"] for r in rs),
                     "loss_abs_diff_max": max(r["loss_abs_diff"] for r in rs),
                     "final_loss_dtrain": rs[-1]["dtrain_loss"], "final_loss_torch": rs[-1]["torch_loss"],
                     "state_bytes_per_rank": meta["state_bytes_per_rank"]}
                if mode != "zero":
                    e.update(grad_maxabs_diff_per_step=[r["grad_maxabs_diff"] for r in rs],
                             grad_maxabs_diff_max=max(r["grad_maxabs_diff"] for r in rs),
                             grad_maxabs=max(r["grad_maxabs"] for r in rs),
                             grad_bit_identical_frac_step1=rs[0]["grad_bit_identical_frac"])
                res.append(e)
                os.remove(name + ".npz")
    return res


def resume(out_dir: str, tmp: str, quick: bool) -> list:
    res = []
    steps, k = (6, 3) if quick else (20, 10)
    w = 2 if quick else 4
    for mode in ("ddp", "zero"):
        for dt in ("float64", "float32"):
            base = os.path.join(out_dir, f"resume_{mode}_w{w}_{dt}")
            ck = os.path.join(tmp, f"ck_{mode}_{dt}")
            common = ["--mode", mode, "--steps", str(steps), "--k", str(k), "--dtype", dt]
            _launch(w, "torch_crosscheck.py", [*common, "--phase", "full", "--out", base + "_full"], tmp)
            _launch(w, "torch_crosscheck.py", [*common, "--phase", "first", "--ckpt", ck, "--out", base + "_first"], tmp)
            _launch(w, "torch_crosscheck.py", [*common, "--phase", "resume", "--ckpt", ck, "--out", base + "_resumed"],
                    tmp)
            full, done = np.load(base + "_full.npz"), np.load(base + "_resumed.npz")
            res.append({"mode": mode, "world": w, "dtype": dt, "steps": steps, "ckpt_step": k,
                        "dtrain_resumed_bit_identical": bool(np.array_equal(full["dtrain"], done["dtrain"])),
                        "torch_resumed_bit_identical": bool(np.array_equal(full["torch"], done["torch"])),
                        "dtrain_vs_torch_full_maxabs": float(np.max(np.abs(full["dtrain"] - full["torch"]))),
                        "dtrain_vs_torch_resumed_maxabs": float(np.max(np.abs(done["dtrain"] - done["torch"])))})
            for suffix in ("_full.npz", "_first.npz", "_resumed.npz"):
                os.remove(base + suffix)
    return res


def throughput(out_dir: str, tmp: str, repeats: int):
    tp, speed = [], []
    args = ["--mode", "ddp", "--steps", "30", "--dtype", "float32", "--dim", "128", "--layers", "4", "--heads", "4",
            "--ctx", "64", "--batch", "8"]
    for rep in range(repeats):
        for w in (1, 2, 4):
            for impl in ("dtrain", "torch"):
                name = os.path.join(out_dir, f"tp_{impl}_w{w}_r{rep}")
                before = _load()
                _launch(w, "torch_crosscheck.py", [*args, "--only", impl, "--out", name], tmp)
                rs = _jsonl(name + ".jsonl")[5:]
                s = float(np.median([r[f"{impl}_s"] for r in rs]))
                tp.append({"impl": impl, "world": w, "repeat": rep, "median_step_s": s,
                           "tokens_per_s": 8 * 64 * w / s, "load_before": before, "load_after": _load()})
                os.remove(name + ".npz")
        for w in (2, 4):
            f = os.path.join(out_dir, f"allreduce_speed_w{w}_r{rep}.json")
            before = _load()
            _launch(w, "torch_allreduce.py", ["--n-check", "1000", "--out", f], tmp)
            with open(f) as fh:
                speed += [{"world": w, "repeat": rep, "load_before": before, **r} for r in json.load(fh)["speed"]]
    return tp, speed


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--skip-bench", action="store_true")
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--data", default=None,
                    help="text corpus; default: a generated word corpus (no download needed)")
    a = ap.parse_args(argv)
    os.makedirs(a.out, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="xc_")
    if a.data is None:
        rng = np.random.default_rng(0)
        words = ["the", "king", "and", "queen", "of", "rome", "said", "to", "thee", "now"]
        a.data = os.path.join(tmp, "corpus.txt")
        with open(a.data, "w") as f:
            f.write(" ".join(rng.choice(words, 20000)) + "\n")
    _DATA[:] = ["--data", a.data]
    steps = 8 if a.quick else 50
    import torch
    summ = {"steps": steps, "load_before": _load(), "torch": torch.__version__, "numpy": np.__version__}
    summ["adamw_only"] = adamw_only(steps)
    summ["collective"] = []
    for w in (2, 3, 4):
        f = os.path.join(a.out, f"allreduce_check_w{w}.json")
        _launch(w, "torch_allreduce.py", ["--no-speed", "--out", f], tmp)
        with open(f) as fh:
            summ["collective"].append({"world": w, **json.load(fh)["check"]})
    summ["equivalence"] = equivalence(a.out, tmp, steps)
    summ["resume"] = resume(a.out, tmp, a.quick)
    summ["throughput"], summ["allreduce_speed"] = ([], []) if a.skip_bench else throughput(a.out, tmp, a.repeats)
    summ["load_after"] = _load()
    shutil.rmtree(tmp, ignore_errors=True)
    with open(os.path.join(a.out, "summary.json"), "w") as f:
        json.dump(summ, f, indent=1)
    print(json.dumps({k: summ[k] for k in ("collective", "resume")}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
