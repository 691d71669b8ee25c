"""Summarise ``bench.py`` JSON lines (one run per GPU count) into a scaling table.

``python -m brain_b200.bench.report run1.json run2.json ...`` prints, per GPU count, the whole-job
throughput, the step time, the per-GPU throughput and the weak-scaling efficiency against the
smallest GPU count (per-GPU throughput at N / per-GPU throughput at the smallest N), as Markdown.
Lines that are not JSON objects with a ``value`` are skipped (logs can be passed as they are).
"""
from __future__ import annotations

import json
import sys


def load_runs(paths) -> list[dict]:
    runs = []
    for p in paths:
        with open(p) as f:
            for line in f:
                line = line.strip()
                if not line.startswith("{"):
                    continue
                try:
                    d = json.loads(line)
                except ValueError:
                    continue
                if isinstance(d, dict) and "value" in d and d.get("impl", "brain") != "reference":
                    runs.append(d)
    return runs


def scaling_table(runs: list[dict]) -> str:
    by_n = {}
    for r in runs:
        by_n[int(r.get("n_gpus", r.get("n_ranks", 1)))] = r  # the last run per GPU count wins
    if not by_n:
        return "no runs"
    n0 = min(by_n)
    base = by_n[n0]["value"] / n0
    unit = by_n[n0].get("unit", "")
    out = [f"| GPUs | {unit} | ms/step | per GPU | weak-scaling efficiency |", "|---|---|---|---|---|"]
    for n in sorted(by_n):
        r = by_n[n]
        per = r["value"] / n
        out.append(f"| {n} | {r['value']:,.0f} | {r.get('ms_per_step', float('nan')):.1f} | {per:,.0f} | "
                   f"{per / base:.3f} |")
    return "\n".join(out)


def main(argv=None) -> int:
    paths = sys.argv[1:] if argv is None else argv
    print(scaling_table(load_runs(paths)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
