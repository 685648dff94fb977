"""This framework against PyTorch on host ranks, end to end, into one summary.json.

    python benchmarks/run_torch_crosscheck.py --out DIR [--quick] [--skip-bench] [--repeats 3] [--data FILE]

The work is a plan of launches (``Launch``: a script from this directory, a
world size and its flags) grouped into the sections of summary.json, which
``benchmarks/torch_report.py`` renders as Markdown:

  adamw_only    AdamW alone vs torch.optim.AdamW on identical gradients (in process)
  collective    ring all-reduce vs gloo exactness at W = 2, 3, 4 (torch_allreduce.py)
  equivalence   DDP (AdamW, SGD) and ZeRO-1 step by step vs torch DDP and
                ZeroRedundancyOptimizer, float64 and float32 (torch_crosscheck.py)
  resume        checkpoint, exit, resume in new processes vs an uninterrupted run
  throughput    host step time of each library alone, and all-reduce speed

Every launch goes through ``python -m dtrain_b200.launch`` (CPU ranks, gloo and
this framework's TCP group over loopback).  The section names and record keys
are the ones the reference's cross-check summary uses, so either stack's
summary.json renders with the same report.
"""
from __future__ import annotations

import argparse
import dataclasses
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


@dataclasses.dataclass
class Launch:
    script: str          # file in benchmarks/
    world: int
    args: list
    out: str             # output prefix (or JSON file for torch_allreduce.py)


class Runner:
    """Launches benchmark scripts on CPU ranks; each launch gets a fresh gloo rendezvous file."""

    def __init__(self, tmp: str, data_flags: list, timeout: int = 1800):
        self.tmp, self.data_flags, self.timeout = tmp, data_flags, timeout
        self.count = 0

    def __call__(self, job: Launch):
        self.count += 1
        init = os.path.join(self.tmp, f"rdv{self.count}")
        extra = self.data_flags if job.script == "torch_crosscheck.py" else []
        out_flag = ["--out", job.out]
        cmd = [PY, "-m", "dtrain_b200.launch", "--nproc", str(job.world), "--timeout", "120", "--",
               PY, os.path.join(HERE, job.script), "--torch-init", init, *extra, *job.args, *out_flag]
        env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1", MKL_NUM_THREADS="1",
                   PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=self.timeout, cwd=ROOT)
        if r.returncode:
            raise RuntimeError(f"launch {job} failed ({r.returncode}):\n{r.stdout[-2000:]}\n{r.stderr[-3000:]}")


def _rows(prefix: str) -> list:
    with open(prefix + ".jsonl") as f:
        return [json.loads(line) for line in f]


def _meta(prefix: str) -> dict:
    with open(prefix + ".meta.json") as f:
        return json.load(f)


def loadavg() -> list:
    with open("/proc/loadavg") as f:
        return f.read().split()[:3]


# ------------------------------------------------------------------ sections
def section_adamw(steps: int) -> dict:
    """This AdamW and torch.optim.AdamW from the same start, fed the same gradients
    whose magnitudes span 1e-12 .. 1 (below and above eps)."""
    import torch
    from dtrain_b200.ops.optim import AdamW
    res = {}
    for dt in ("float64", "float32"):
        rng = np.random.default_rng(11)
        start = rng.standard_normal(80_000).astype(dt)
        mine, ref = torch.from_numpy(start.copy()), torch.from_numpy(start.copy()).requires_grad_()
        hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
        opt_mine, opt_ref = AdamW([mine], **hp), torch.optim.AdamW([ref], **hp)
        per_step = []
        for _ in range(steps):
            g = (rng.standard_normal(start.size) * 10.0 ** rng.uniform(-12, 0, start.size)).astype(dt)
            opt_mine.step([torch.from_numpy(g.copy())])
            ref.grad = torch.from_numpy(g.copy())
            opt_ref.step()
            per_step.append(float((mine - ref.detach()).abs().max()))
        res[dt] = {"param_maxabs_diff_per_step": per_step, "param_maxabs_diff_max": max(per_step)}
    return res


def section_collective(run: Runner, out_dir: str) -> list:
    res = []
    for w in (2, 3, 4):
        f = os.path.join(out_dir, f"allreduce_check_w{w}.json")
        run(Launch("torch_allreduce.py", w, ["--no-speed"], f))
        with open(f) as fh:
            res.append({"world": w, **json.load(fh)["check"]})
    return res


EQUIVALENCE_PLAN = [  # (name in the summary, crosscheck flags, world sizes)
    ("ddp", ["--mode", "ddp"], (1, 2, 4)),
    ("ddp-sgd", ["--mode", "ddp", "--opt", "sgd", "--lr", "0.1"], (1, 2, 4)),
    ("zero", ["--mode", "zero"], (2, 4)),
]


def section_equivalence(run: Runner, out_dir: str, steps: int) -> list:
    res = []
    for name, flags, worlds in EQUIVALENCE_PLAN:
        for dt in ("float64", "float32"):
            for w in worlds:
                prefix = os.path.join(out_dir, f"{name}_w{w}_{dt}")
                run(Launch("torch_crosscheck.py", w, [*flags, "--steps", str(steps), "--dtype", dt], prefix))
                rows, meta = _rows(prefix), _meta(prefix)
                rec = {"mode": name, "world": w, "dtype": dt, "steps": len(rows), "n_params": meta["n_params"],
                       "state_bytes_per_rank": meta["state_bytes_per_rank"],
                       "param_maxabs_diff_per_step": [r["param_maxabs_diff"] for r in rows],
                       "final_loss_dtrain": rows[-1]["dtrain_loss"], "final_loss_torch": rows[-1]["torch_loss"]}
                rec["param_maxabs_diff_max"] = max(rec["param_maxabs_diff_per_step"])
                rec["loss_abs_diff_max"] = max(r["loss_abs_diff"] for r in rows)
                if name != "zero":
                    rec["grad_maxabs_diff_per_step"] = [r["grad_maxabs_diff"] for r in rows]
                    rec["grad_maxabs_diff_max"] = max(rec["grad_maxabs_diff_per_step"])
                    rec["grad_maxabs"] = max(r["grad_maxabs"] for r in rows)
                    rec["grad_bit_identical_frac_step1"] = rows[0]["grad_bit_identical_frac"]
                res.append(rec)
                os.remove(prefix + ".npz")
    return res


def section_resume(run: Runner, out_dir: str, tmp: str, quick: bool) -> list:
    """Each library: an uninterrupted run, and one that checkpoints at step k, exits and
    resumes in new processes; the two final parameter sets must be bit-identical."""
    steps, k, w = (6, 3, 2) if quick else (20, 10, 4)
    res = []
    for mode in ("ddp", "zero"):
        for dt in ("float64", "float32"):
            prefix = os.path.join(out_dir, f"resume_{mode}_w{w}_{dt}")
            ck = os.path.join(tmp, f"ck-{mode}-{dt}")
            flags = ["--mode", mode, "--steps", str(steps), "--k", str(k), "--dtype", dt]
            phases = {"full": [], "first": ["--ckpt", ck], "resumed": ["--ckpt", ck]}
            for phase, extra in phases.items():
                run(Launch("torch_crosscheck.py", w, [*flags, "--phase", "resume" if phase == "resumed" else phase,
                                                      *extra], f"{prefix}_{phase}"))
            full, resumed = np.load(prefix + "_full.npz"), np.load(prefix + "_resumed.npz")
            res.append({"mode": mode, "world": w, "dtype": dt, "steps": steps, "ckpt_step": k,
                        "dtrain_resumed_bit_identical": bool(np.array_equal(full["dtrain"], resumed["dtrain"])),
                        "torch_resumed_bit_identical": bool(np.array_equal(full["torch"], resumed["torch"])),
                        "dtrain_vs_torch_full_maxabs": float(np.abs(full["dtrain"] - full["torch"]).max()),
                        "dtrain_vs_torch_resumed_maxabs": float(np.abs(resumed["dtrain"] - resumed["torch"]).max())})
            for phase in phases:
                os.remove(f"{prefix}_{phase}.npz")
    return res


THROUGHPUT_MODEL = ["--mode", "ddp", "--steps", "30", "--dtype", "float32", "--dim", "128", "--layers", "4",
                    "--heads", "4", "--ctx", "64", "--batch", "8"]


def section_throughput(run: Runner, out_dir: str, repeats: int):
    steps_rec, speed_rec = [], []
    for rep in range(repeats):
        for w in (1, 2, 4):
            for impl in ("dtrain", "torch"):
                prefix = os.path.join(out_dir, f"tp_{impl}_w{w}_r{rep}")
                before = loadavg()
                run(Launch("torch_crosscheck.py", w, [*THROUGHPUT_MODEL, "--only", impl], prefix))
                step_s = float(np.median([r[f"{impl}_s"] for r in _rows(prefix)[5:]]))
                steps_rec.append({"impl": impl, "world": w, "repeat": rep, "median_step_s": step_s,
                                  "tokens_per_s": 8 * 64 * w / step_s, "load_before": before, "load_after": loadavg()})
                os.remove(prefix + ".npz")
        for w in (2, 4):
            f = os.path.join(out_dir, f"allreduce_speed_w{w}_r{rep}.json")
            before = loadavg()
            run(Launch("torch_allreduce.py", w, ["--n-check", "1000"], f))
            with open(f) as fh:
                speed_rec += [{"world": w, "repeat": rep, "load_before": before, **r} for r in json.load(fh)["speed"]]
    return steps_rec, speed_rec


def _corpus(path: str):
    """An offline corpus: pseudo-words from a fixed syllable set."""
    rng = np.random.default_rng(3)
    syl = ["ma", "ne", "ri", "so", "tu", "va", "ke", "lo", "pi", "da"]
    words = ["".join(rng.choice(syl, int(rng.integers(1, 4)))) for _ in range(60)]
    with open(path, "w") as f:
        f.write("\n".join(" ".join(rng.choice(words, 16)) for _ in range(1500)) + "\n")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", required=True)
    ap.add_argument("--quick", action="store_true", help="8 steps, W<=2 resume (minutes instead of an hour)")
    ap.add_argument("--skip-bench", action="store_true", help="no throughput section")
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--data", default=None, help="text corpus (default: a generated one)")
    a = ap.parse_args(argv)
    os.makedirs(a.out, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="xcheck_")
    try:
        if a.data is None:
            a.data = os.path.join(tmp, "corpus.txt")
            _corpus(a.data)
        run = Runner(tmp, ["--data", a.data])
        steps = 8 if a.quick else 50
        import torch
        summary = {"steps": steps, "load_before": loadavg(), "torch": torch.__version__, "numpy": np.__version__}
        summary["adamw_only"] = section_adamw(steps)
        summary["collective"] = section_collective(run, a.out)
        summary["equivalence"] = section_equivalence(run, a.out, steps)
        summary["resume"] = section_resume(run, a.out, tmp, a.quick)
        summary["throughput"], summary["allreduce_speed"] = ([], []) if a.skip_bench else \
            section_throughput(run, a.out, a.repeats)
        summary["load_after"] = loadavg()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    with open(os.path.join(a.out, "summary.json"), "w") as f:
        json.dump(summary, f, indent=1)
    print(json.dumps({k: summary[k] for k in ("collective", "resume")}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
