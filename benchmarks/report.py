"""Markdown tables from benchmark results.

    python benchmarks/report.py <results dir or files...>

Understands, by content:
  * all-reduce sweeps (allreduce_bench.py / torch_allreduce.py "speed" /
    collectives_bench.py JSON lines): latency and bus bandwidth per size and impl;
  * training logs (train.py --log JSONL, e.g. from scaling.sh): median step time
    and tokens/s per run, skipping the first 5 steps;
  * bench.py lines (bench.jsonl): tokens/s, ms/step, e2e, impl and GPU count;
  * summary.json of run_torch_crosscheck.py (delegates to torch_report.py).
Counterpart of the reference's benchmarks/report.py.
"""
from __future__ import annotations

import glob
import json
import os
import statistics
import sys


def _records(path: str):
    with open(path) as f:
        text = f.read().strip()
    if not text:
        return []
    if text[0] == "[" or (text[0] == "{" and "\n" not in text):
        obj = json.loads(text)
        return obj if isinstance(obj, list) else [obj]
    if text[0] == "{":
        try:
            obj = json.loads(text)
            return obj.get("speed", [obj]) if isinstance(obj, dict) else obj
        except json.JSONDecodeError:
            pass
    out = []
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("{"):
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                continue
    return out


def _fmt_bytes(n: int) -> str:
    for unit in ("B", "KiB", "MiB", "GiB"):
        if n < 1024:
            return f"{n:g} {unit}"
        n /= 1024
    return f"{n:g} TiB"


def allreduce_table(rows) -> str:
    impls = sorted({r["impl"] + (f" W={r['world']}" if "world" in r else "") for r in rows})
    sizes = sorted({r["bytes"] for r in rows})
    key = {(r["impl"] + (f" W={r['world']}" if "world" in r else ""), r["bytes"]): r for r in rows}
    head = "| size | " + " | ".join(f"{i} us / GB/s" for i in impls) + " |"
    lines = [head, "|" + "---|" * (len(impls) + 1)]
    for s in sizes:
        cells = []
        for i in impls:
            r = key.get((i, s))
            cells.append(f"{r['latency_us']:.1f} / {r['bus_GBps']:.2f}" if r else "")
        lines.append(f"| {_fmt_bytes(s)} | " + " | ".join(cells) + " |")
    return "\n".join(lines)


def training_table(named_logs) -> str:
    lines = ["| run | steps | median step s | tokens/s | final loss |", "|---|---|---|---|---|"]
    for name, rows in named_logs:
        body = [r for r in rows if "step_s" in r][5:] or [r for r in rows if "step_s" in r]
        if not body:
            continue
        med = statistics.median(r["step_s"] for r in body)
        tps = statistics.median(r.get("tokens_per_s", 0.0) for r in body)
        lines.append(f"| {name} | {len(rows)} | {med:.4f} | {tps:,.0f} | {rows[-1].get('loss', float('nan')):.4f} |")
    return "\n".join(lines)


def bench_table(rows) -> str:
    lines = ["| impl | GPUs | config | tokens/s | ms/step | e2e tokens/s | clocks |", "|---|---|---|---|---|---|---|"]
    for r in rows:
        if r.get("unavailable"):
            lines.append(f"| {r.get('impl', '?')} | {r.get('n_gpus', '')} | | unavailable: {r['unavailable']} | | | |")
            continue
        e2e = r.get("e2e", {}).get("value")
        clk = r.get("clocks", {})
        lines.append(f"| {r.get('impl', 'ours')} | {r['n_gpus']} | {r['config'].get('model', '')} | "
                     f"{r['value']:,.0f} | {r['ms_per_step']:.2f} | {e2e:,.0f} | "
                     f"{clk.get('sm_mhz', '')} MHz {','.join(clk.get('reasons', []))} |" if e2e else
                     f"| {r.get('impl', 'ours')} | {r['n_gpus']} | | {r['value']:,.0f} | {r['ms_per_step']:.2f} | | |")
    return "\n".join(lines)


def main(argv=None):
    args = sys.argv[1:] if argv is None else argv
    files = []
    for a in args:
        files += sorted(glob.glob(os.path.join(a, "*.json*"))) if os.path.isdir(a) else [a]
    sweeps, logs, bench = [], [], []
    for f in files:
        if os.path.basename(f) == "summary.json":
            from torch_report import render  # noqa: PLC0415  (sibling script)
            with open(f) as fh:
                print(render(json.load(fh)))
            continue
        recs = _records(f)
        if not recs:
            continue
        if all("bus_GBps" in r for r in recs):
            sweeps += recs
        elif all("metric" in r or "unavailable" in r for r in recs):
            bench += recs
        elif any("step_s" in r for r in recs):
            logs.append((os.path.splitext(os.path.basename(f))[0], recs))
    if sweeps:
        print("## All-reduce\n\n" + allreduce_table(sweeps) + "\n")
    if logs:
        print("## Training runs\n\n" + training_table(logs) + "\n")
    if bench:
        print("## bench.py\n\n" + bench_table(bench) + "\n")
    return 0


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    sys.exit(main())
