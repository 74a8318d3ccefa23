"""Training-log parsing and figures.

Reads step lines of this package's trainer (``python -m dion_b200.train``)
and of torchtitan-style logs (``[titan] <date> ... step: N loss: ...``),
keeps the first line per step (multi-rank logs repeat them), and draws the
comparison figures: loss vs step and vs tokens, throughput, memory, MFU, plus
a Markdown summary table. The fields are those of the reference's log parser
(ada_dion/scripts/generate_plots.py:55-68): step, loss, grad_norm, memory,
tps, tflops, mfu.

    python -m dion_b200.benchmarks.logparse logs/*.log --out plots/ [--tokens-per-step 65536]
"""
from __future__ import annotations

import argparse
import os
import re
from datetime import datetime
from typing import Dict, List, Optional

from ..utils.svgplot import Figure
from .plots import COLORS, LABELS

__all__ = ["parse_log", "parse_log_text", "generate_plots", "summary_table"]

_FIELDS = {
    "step": (re.compile(r"step:\s*(\d+)"), int),
    "loss": (re.compile(r"loss:\s*([-\d.eE+naif]+)"), float),
    "grad_norm": (re.compile(r"grad_norm:\s*([-\d.eE+naif]+)"), float),
    "memory_gib": (re.compile(r"memory:\s*([\d.]+)\s*GiB"), float),
    "tps": (re.compile(r"tps:\s*([\d,]+)"), lambda s: float(s.replace(",", ""))),
    "tflops": (re.compile(r"tflops:\s*([\d,.]+)"), lambda s: float(s.replace(",", ""))),
    "mfu": (re.compile(r"mfu:\s*([\d.]+)%"), float),
}
_TS = re.compile(r"(\d{4}-\d{2}-\d{2}[ T]\d{2}:\d{2}:\d{2})")
_OPT = re.compile(r"(?:Optimizer:\s*|--config\s+\S*?_)(adamw|muon|dion2|dion|adadion_v2|adadion)\b", re.I)


def parse_log_text(text: str, name: Optional[str] = None) -> dict:
    """{"optimizer", "step", "loss", ..., "time_s"} lists (one entry per logged
    step), plus "val_step" / "val_loss" from validation lines."""
    m = _OPT.search(text)
    out: Dict[str, list] = {k: [] for k in _FIELDS}
    out["time_s"] = []
    out["val_step"], out["val_loss"] = [], []
    seen = set()
    t0 = None
    for line in text.splitlines():
        if "step:" not in line or "loss:" not in line:
            continue
        if "validate" in line:  # validation pass: "validate step: N  loss: X"
            vm, lm = _FIELDS["step"][0].search(line), _FIELDS["loss"][0].search(line)
            if vm and lm and int(vm.group(1)) not in out["val_step"]:
                out["val_step"].append(int(vm.group(1)))
                out["val_loss"].append(float(lm.group(1)))
            continue
        sm = _FIELDS["step"][0].search(line)
        if not sm:
            continue
        step = int(sm.group(1))
        if step in seen:
            continue
        seen.add(step)
        for k, (rx, conv) in _FIELDS.items():
            fm = rx.search(line)
            out[k].append(conv(fm.group(1)) if fm else float("nan"))
        tm = _TS.search(line)
        if tm:
            ts = datetime.fromisoformat(tm.group(1).replace(" ", "T"))
            t0 = t0 or ts
            out["time_s"].append((ts - t0).total_seconds())
        else:
            out["time_s"].append(float("nan"))
    out["optimizer"] = (m.group(1).lower() if m else None) or name
    return out


def parse_log(path: str) -> dict:
    with open(path, errors="replace") as f:
        text = f.read()
    base = os.path.splitext(os.path.basename(path))[0]
    guess = next((o for o in ("adadion_v2", "adadion", "dion2", "dion", "muon", "adamw") if o in base.lower()), base)
    d = parse_log_text(text, guess)
    d["name"] = base
    return d


def generate_plots(paths: List[str], out_dir: str, tokens_per_step: Optional[int] = None) -> List[str]:
    os.makedirs(out_dir, exist_ok=True)
    runs = [parse_log(p) for p in paths]
    written = []
    panels = [("loss", "Training loss", "loss"), ("tps", "Throughput", "tokens/s"),
              ("memory_gib", "Peak memory", "GiB"), ("mfu", "MFU", "%"), ("grad_norm", "Gradient norm", "norm")]
    fig = Figure(ncols=3, nrows=2, title="Training runs")
    for ax, (key, title, ylab) in zip(fig.axes, panels):
        for r in runs:
            if r["step"]:
                ax.line(r["step"], r[key], label=r["name"], color=COLORS.get(r["optimizer"] or ""))
        ax.set(title=title, xlabel="step", ylabel=ylab)
    if tokens_per_step:
        ax = fig.axes[5]
        for r in runs:
            if r["step"]:
                ax.line([s * tokens_per_step for s in r["step"]], r["loss"], label=LABELS.get(r["optimizer"], r["name"]),
                        color=COLORS.get(r["optimizer"] or ""))
        ax.set(title="Loss vs tokens", xlabel="tokens", ylabel="loss")
    written.append(fig.save(os.path.join(out_dir, "training_runs.svg")))
    with open(os.path.join(out_dir, "summary.md"), "w") as f:
        f.write(summary_table(runs))
    written.append(os.path.join(out_dir, "summary.md"))
    return written


def summary_table(runs: List[dict]) -> str:
    def mean(xs):
        xs = [x for x in xs if x == x]
        return sum(xs) / len(xs) if xs else float("nan")

    lines = ["| run | optimizer | steps | final loss | mean tps | peak memory (GiB) | mean MFU (%) |",
             "|---|---|---|---|---|---|---|"]
    for r in runs:
        if not r["step"]:
            continue
        lines.append(f"| {r['name']} | {r['optimizer']} | {r['step'][-1]} | {r['loss'][-1]:.4f} | "
                     f"{mean(r['tps'][1:] or r['tps']):,.0f} | {max(r['memory_gib']):.2f} | {mean(r['mfu']):.2f} |")
    return "\n".join(lines) + "\n"


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("logs", nargs="+")
    p.add_argument("--out", default="plots")
    p.add_argument("--tokens-per-step", type=int, default=None)
    a = p.parse_args(argv)
    for w in generate_plots(a.logs, a.out, a.tokens_per_step):
        print(w)


if __name__ == "__main__":
    main()
