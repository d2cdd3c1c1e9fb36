"""Throughput report over a directory of training runs (role of sae_lens/hooks_results_analysis.py
and scripts/analyze_hooks_results.py).

Each run directory (`saelens_runner_gpu_<timestamp>`) holds the trainer's `timing_history.jsonl`
(one record per timing step: `n_training_samples`, `elapsed_s`, ...) and usually `runner_cfg.json`.
Runs are grouped by how many hooks they trained (from the config's `hook_names`, a
`multi_sae_manifest.json`, or `blocks_*` subfolders; unknown counts borrow the nearest known run's
group), ordered by timestamp, labelled with a scenario template by position, and reported as
tokens/s, also normalised to the largest token budget of the group so runs with different budgets
compare.  A run is complete when it logged at least `min_steps` timing steps and reached
`min_completion_ratio` of its budget.

CLI: `python -m saelens_b200.analysis.results --results-dir DIR [--checkpoints-dir DIR]`.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass
from datetime import datetime
from pathlib import Path
from typing import Any

DEFAULT_COMMAND_TEMPLATE = [
    "baseline", "vDP+sDP(fsdp)", "sDP(fsdp)+bs8", "vTP+sDP(fsdp)+bs8", "vDP+sDP(ddp)", "sDP(ddp)+bs8",
    "vTP+sDP(ddp)+bs8", "vTP", "sTP", "vTP+sTP", "vDP", "vDP+sTP",
]
RUN_PREFIX = "saelens_runner_gpu_"


@dataclass
class RunRow:
    run_id: str
    timestamp: str
    hook_count: int
    slot: int
    scenario: str
    steps: int
    final_samples: int
    elapsed_s: float
    complete: bool
    local_completion_ratio: float | None
    local_tokens_per_s: float
    normalized_tokens_per_s: float
    training_tokens: int | None
    notes: tuple[str, ...]


@dataclass
class HookGroupReport:
    hook_count: int
    rows: list[RunRow]

    @property
    def best_complete(self) -> RunRow | None:
        done = [r for r in self.rows if r.complete]
        return max(done, key=lambda r: r.normalized_tokens_per_s) if done else None


@dataclass
class Report:
    groups: dict[int, HookGroupReport]
    rows: list[RunRow]


def _timestamp(run_id: str) -> str:
    return run_id[len(RUN_PREFIX):] if run_id.startswith(RUN_PREFIX) else run_id


def _sort_key(ts: str) -> tuple[int, str]:
    digits = ts.replace("_", "")
    return (int(digits), ts) if digits.isdigit() else (10**20, ts)


def _jsonl(path: Path) -> list[dict[str, Any]]:
    return [json.loads(line) for line in path.read_text().splitlines() if line.strip()]


def _nearest_ckpt(checkpoints: Path, ts: str) -> Path | None:
    try:
        t0 = datetime.strptime(ts, "%y%m%d_%H%M%S")
    except ValueError:
        return None
    best: tuple[float, Path] | None = None
    for c in checkpoints.glob(ts.split("_")[0] + "_*"):
        try:
            dt = abs((datetime.strptime(c.name, "%y%m%d_%H%M%S") - t0).total_seconds())
        except ValueError:
            continue
        if c.is_dir() and dt <= 2.0 and (best is None or dt < best[0]):
            best = (dt, c)
    return best[1] if best else None


def _runner_cfg(run_dir: Path, checkpoints: Path | None) -> dict[str, Any] | None:
    local = run_dir / "runner_cfg.json"
    if local.exists():
        return json.loads(local.read_text())
    if checkpoints is None:
        return None
    ts = _timestamp(run_dir.name)
    d = checkpoints / ts if (checkpoints / ts).exists() else _nearest_ckpt(checkpoints, ts)
    if d is None:
        return None
    found = sorted(d.glob("final_*/runner_cfg.json"))
    return json.loads(found[-1].read_text()) if found else None


def _hook_count(run_dir: Path, cfg: dict[str, Any] | None) -> int | None:
    counts = []
    if cfg:
        if isinstance(cfg.get("hook_names"), list) and cfg["hook_names"]:
            counts.append(len(cfg["hook_names"]))
        elif cfg.get("hook_name"):
            counts.append(1)
    man = run_dir / "multi_sae_manifest.json"
    if man.exists():
        names = json.loads(man.read_text()).get("hook_names")
        if isinstance(names, list) and names:
            counts.append(len(names))
    dirs = [c for c in run_dir.iterdir() if c.is_dir() and c.name.startswith("blocks_")]
    if dirs:
        counts.append(len(dirs))
    return max(counts) if counts else None


def _fill_hook_counts(runs: list[dict[str, Any]]) -> None:
    known = [i for i, r in enumerate(runs) if r["hook_count"] is not None]
    for i, r in enumerate(runs):
        if r["hook_count"] is not None:
            continue
        if not known:
            r["hook_count"] = 0
            continue
        prev = max((k for k in known if k < i), default=None)
        nxt = min((k for k in known if k > i), default=None)
        if prev is None or (nxt is not None and nxt - i <= i - prev):
            r["hook_count"] = runs[nxt]["hook_count"]  # ties go to the following group
        else:
            r["hook_count"] = runs[prev]["hook_count"]


def build_report(results_dir: Path | str, *, checkpoints_dir: Path | str | None = None,
                 command_template: list[str] | None = None, min_steps: int = 32,
                 min_completion_ratio: float = 0.98) -> Report:
    root = Path(results_dir)
    ckpt = Path(checkpoints_dir) if checkpoints_dir is not None else None
    template = command_template or DEFAULT_COMMAND_TEMPLATE
    runs: list[dict[str, Any]] = []
    for d in sorted(root.glob(RUN_PREFIX + "*")):
        tp = d / "timing_history.jsonl"
        recs = _jsonl(tp) if tp.exists() else []
        if not recs:
            continue
        cfg = _runner_cfg(d, ckpt)
        ts = _timestamp(d.name)
        runs.append({"run_id": d.name, "timestamp": ts, "steps": len(recs),
                     "final_samples": int(recs[-1].get("n_training_samples", 0)),
                     "elapsed_s": float(recs[-1].get("elapsed_s", 0.0)), "cfg": cfg,
                     "hook_count": _hook_count(d, cfg), "key": _sort_key(ts)})
    runs.sort(key=lambda r: r["key"])
    _fill_hook_counts(runs)
    groups: dict[int, HookGroupReport] = {}
    rows_all: list[RunRow] = []
    for hc in sorted({r["hook_count"] for r in runs}):
        members = [r for r in runs if r["hook_count"] == hc]
        budgets = [int(r["cfg"]["training_tokens"]) for r in members
                   if r["cfg"] and isinstance(r["cfg"].get("training_tokens"), int)]
        ref = max(budgets) if budgets else None
        rows = []
        for slot, r in enumerate(members, start=1):
            tt = (r["cfg"] or {}).get("training_tokens")
            tt = int(tt) if isinstance(tt, int) and tt > 0 else None
            ratio = r["final_samples"] / tt if tt else None
            notes = []
            complete = r["steps"] >= min_steps
            if not complete:
                notes.append("short_steps")
            if ratio is not None and ratio < min_completion_ratio:
                complete = False
                notes.append("under_target_tokens")
            if r["cfg"] is None:
                notes.append("missing_cfg")
            local = r["final_samples"] / r["elapsed_s"] if r["elapsed_s"] > 0 else 0.0
            norm = (r["final_samples"] * (ref / tt) / r["elapsed_s"]) if (r["elapsed_s"] > 0 and tt and ref) else local
            row = RunRow(r["run_id"], r["timestamp"], hc, slot,
                         template[slot - 1] if slot <= len(template) else f"extra#{slot}", r["steps"],
                         r["final_samples"], r["elapsed_s"], complete, ratio, local, norm, tt, tuple(notes))
            rows.append(row)
            rows_all.append(row)
        groups[hc] = HookGroupReport(hc, rows)
    return Report(groups, rows_all)


def format_report(report: Report) -> str:
    lines = []
    for hc, g in report.groups.items():
        lines.append(f"== {hc} hook(s) ==")
        lines.append(f"{'slot':>4} {'scenario':<22} {'steps':>6} {'tokens/s':>12} {'norm tok/s':>12} complete notes")
        for r in g.rows:
            lines.append(f"{r.slot:>4} {r.scenario:<22} {r.steps:>6} {r.local_tokens_per_s:>12.1f} "
                         f"{r.normalized_tokens_per_s:>12.1f} {str(r.complete):<8} {','.join(r.notes)}")
        best = g.best_complete
        if best:
            lines.append(f"best: {best.scenario} ({best.normalized_tokens_per_s:.1f} tokens/s)")
    return "\n".join(lines)


def main() -> None:
    p = argparse.ArgumentParser(description="Throughput report over saelens_runner_gpu_* run directories")
    p.add_argument("--results-dir", required=True)
    p.add_argument("--checkpoints-dir", default=None)
    p.add_argument("--min-steps", type=int, default=32)
    p.add_argument("--min-completion-ratio", type=float, default=0.98)
    a = p.parse_args()
    print(format_report(build_report(a.results_dir, checkpoints_dir=a.checkpoints_dir, min_steps=a.min_steps,
                                     min_completion_ratio=a.min_completion_ratio)))


if __name__ == "__main__":
    main()
