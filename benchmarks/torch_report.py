"""Markdown rendering of run_torch_crosscheck.py's summary.json.

    python benchmarks/torch_report.py benchmarks/results/xcheck/summary.json

Counterpart of the reference's benchmarks/torch_report.py: one table per
section (optimizer alone, collectives, step-by-step equivalence, resume,
throughput).
"""
from __future__ import annotations

import json
import statistics
import sys


def _g(x) -> str:
    return f"{x:.3g}" if isinstance(x, float) else str(x)


def render(s: dict) -> str:
    out = [f"# Cross-check vs PyTorch {s.get('torch', '')} ({s.get('steps')} steps)", ""]
    out += ["## AdamW alone", "", "| dtype | max param diff |", "|---|---|"]
    for dt, r in s.get("adamw_only", {}).items():
        out.append(f"| {dt} | {_g(r['param_maxabs_diff_max'])} |")
    out += ["", "## All-reduce exactness vs gloo", "",
            "| W | dtype | ours vs gloo max diff | bit-identical | ours err | gloo err |", "|---|---|---|---|---|---|"]
    for c in s.get("collective", []):
        for dt in ("float32", "float64"):
            if dt in c:
                r = c[dt]
                out.append(f"| {c['world']} | {dt} | {_g(r['max_abs_diff_dtrain_vs_gloo'])} | "
                           f"{r['bit_identical_frac']:.4f} | {_g(r['max_abs_err_dtrain'])} | {_g(r['max_abs_err_gloo'])} |")
    out += ["", "## Step-by-step equivalence", "",
            "| mode | W | dtype | max param diff | max loss diff | max grad diff | final loss ours / torch |",
            "|---|---|---|---|---|---|---|"]
    for e in s.get("equivalence", []):
        out.append(f"| {e['mode']} | {e['world']} | {e['dtype']} | {_g(e['param_maxabs_diff_max'])} | "
                   f"{_g(e['loss_abs_diff_max'])} | {_g(e.get('grad_maxabs_diff_max', ''))} | "
                   f"{e['final_loss_dtrain']:.6f} / {e['final_loss_torch']:.6f} |")
    out += ["", "## Checkpoint / resume", "",
            "| mode | W | dtype | ours bit-identical | torch bit-identical | ours vs torch |", "|---|---|---|---|---|---|"]
    for r in s.get("resume", []):
        out.append(f"| {r['mode']} | {r['world']} | {r['dtype']} | {r['dtrain_resumed_bit_identical']} | "
                   f"{r['torch_resumed_bit_identical']} | {_g(r['dtrain_vs_torch_resumed_maxabs'])} |")
    tp = s.get("throughput", [])
    if tp:
        out += ["", "## Host throughput (median over repeats)", "", "| W | ours tokens/s | torch tokens/s |",
                "|---|---|---|"]
        for w in sorted({r["world"] for r in tp}):
            med = {impl: statistics.median(r["tokens_per_s"] for r in tp if r["world"] == w and r["impl"] == impl)
                   for impl in ("dtrain", "torch") if any(r["world"] == w and r["impl"] == impl for r in tp)}
            out.append(f"| {w} | {med.get('dtrain', 0):,.0f} | {med.get('torch', 0):,.0f} |")
    return "\n".join(out) + "\n"


def main(argv=None):
    args = sys.argv[1:] if argv is None else argv
    with open(args[0]) as f:
        print(render(json.load(f)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
