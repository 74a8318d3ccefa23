"""Measured report: loss parity, throughput and optimizer-step tables with
SVG figures, generated from this package's own benchmark outputs.

The reference ships its results as a paper (paper/main.tex: per-optimizer
final losses, throughput and scaling figures). This module produces the
counterpart from runs of this package:

* ``--parity``: JSON files written by ``python -m dion_b200.benchmarks.parity
  --out ...`` (both implementations from the same seed, data and init);
* ``--bench``: files holding the JSON lines printed by ``bench.py`` (either
  arm, any number of GPUs);
* ``--optimizer``: files holding the JSON lines of
  ``python -m dion_b200.benchmarks.optimizer_bench``.

    python -m dion_b200.benchmarks.report --parity muon.json dion.json \\
        --bench bench_lines.jsonl --optimizer ob_lines.jsonl --out docs/report

Writes ``report.md``, one SVG per figure and ``data.json`` (the numbers
behind every table and figure, so the report can be regenerated without the
raw run outputs).
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Dict, List, Optional

from ..utils.svgplot import Figure

__all__ = ["load_json_lines", "collect", "render", "main"]

ARM_COLORS = {"ours": "#d62728", "reference": "#1f77b4"}


def load_json_lines(path: str) -> List[dict]:
    """Every line of ``path`` that parses as a JSON object (log noise is skipped)."""
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line.startswith("{"):
                continue
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                continue
    return out


def _parity_entry(path: str) -> dict:
    """A parity run's output, or a committed golden file (``ours_losses`` /
    ``reference_losses``, written with ``parity --golden``)."""
    with open(path) as f:
        d = json.load(f)
    cfg = d.get("config", {})
    if "ours_losses" in d:
        arms = {"ours": {"losses": d["ours_losses"], "seconds": None},
                "reference": {"losses": d["reference_losses"][0], "seconds": None}}
    else:
        arms = {k: {"losses": d[k]["losses"], "seconds": d[k].get("seconds")} for k in ("ours", "reference") if k in d}
    name = f"{cfg.get('preset', '?')} {cfg.get('optimizer', '?')} ({cfg.get('device', '?')})"
    return {"name": name, "config": cfg, "arms": arms, "comparison": d.get("comparison", {})}


def collect(parity: List[str], bench: List[str], optimizer: List[str]) -> dict:
    """Gather the report's data from run outputs (see the module doc)."""
    data = {"parity": [_parity_entry(p) for p in parity], "bench": [], "optimizer": []}
    for p in bench:
        for d in load_json_lines(p):
            if "metric" in d and "value" in d:
                e2e = d.get("e2e") or {}
                data["bench"].append({
                    "impl": d.get("impl", "ours"), "n_gpus": d.get("n_gpus"), "value": d["value"],
                    "unit": d.get("unit"), "ms_per_step": d.get("ms_per_step"),
                    "optimizer_step_ms": d.get("optimizer_step_ms"), "e2e": e2e.get("value"),
                    "model": (d.get("config") or {}).get("model"),
                    "optimizer": (d.get("config") or {}).get("optimizer"),
                    "sm_mhz": (d.get("clocks") or {}).get("sm_mhz"), "source": os.path.basename(p)})
    for p in optimizer:
        for d in load_json_lines(p):
            if d.get("metric") == "optimizer_step_ms":
                data["optimizer"].append({k: d.get(k) for k in ("optimizer", "impl", "n_gpus", "ms", "p2p",
                                                                 "matrices", "rank_fraction")})
    return data


def _loss_figure(entry: dict) -> Figure:
    fig = Figure()
    ax = fig.axes[0]
    for arm, d in entry["arms"].items():
        ys = d["losses"]
        ax.line(list(range(1, len(ys) + 1)), ys, label=arm, color=ARM_COLORS.get(arm))
    ax.set(title=f"Training loss, {entry['name']}", xlabel="step", ylabel="loss")
    return fig


def _scaling_figure(bench: List[dict]) -> Optional[Figure]:
    series: Dict[str, Dict[int, float]] = {}
    for b in bench:
        if b.get("n_gpus") is None:
            continue
        key = f"{b['impl']} {b.get('model') or '?'} ({b.get('optimizer') or '?'})"
        series.setdefault(key, {})[int(b["n_gpus"])] = max(series.get(key, {}).get(int(b["n_gpus"]), 0.0),
                                                           float(b["value"]))
    if not series:
        return None
    fig = Figure()
    ax = fig.axes[0]
    for key, pts in sorted(series.items()):
        ns = sorted(pts)
        arm = key.split(" ")[0]
        ax.line(ns, [pts[n] for n in ns], label=key, color=ARM_COLORS.get(arm), markers=True)
    ax.set(title="Throughput vs GPUs (weak scaling)", xlabel="GPUs", ylabel="tokens/s")
    return fig


def _fmt(v, nd=1) -> str:
    if v is None:
        return "-"
    if isinstance(v, float):
        return f"{v:,.{nd}f}"
    return str(v)


def render(data: dict, out_dir: str, title: str = "dion_b200 measured report") -> str:
    """Write report.md, the SVG figures and data.json into ``out_dir``; returns the report path."""
    os.makedirs(out_dir, exist_ok=True)
    lines = [f"# {title}", "",
             "Generated by `python -m dion_b200.benchmarks.report` from this package's run outputs; "
             "`data.json` holds every number shown.", ""]
    if data["parity"]:
        lines += ["## Loss parity against the reference implementation", "",
                  "Both arms start from the same weights and see the same tokens, schedule and clipping.", "",
                  "| run | steps | final loss (ours) | final loss (reference) | mean abs. diff | tail-mean rel. diff "
                  "| wall s (ours / reference) |",
                  "|---|---|---|---|---|---|---|"]
        figs = []
        for i, e in enumerate(data["parity"]):
            c = e["comparison"]
            n = len(next(iter(e["arms"].values()))["losses"]) if e["arms"] else 0
            secs = " / ".join(_fmt(e["arms"].get(a, {}).get("seconds")) for a in ("ours", "reference"))
            lines.append(f"| {e['name']} | {n} | {_fmt(c.get('final_ours'), 4)} | {_fmt(c.get('final_ref'), 4)} | "
                         f"{_fmt(c.get('mean_abs_diff'), 4)} | {_fmt(c.get('tail_rel_diff'), 5)} | {secs} |")
            fn = f"loss_{i}.svg"
            _loss_figure(e).save(os.path.join(out_dir, fn))
            figs.append(f"![loss {e['name']}]({fn})")
        lines.append("")
        for f in figs:
            lines += [f, ""]
    if data["bench"]:
        lines += ["## Training throughput (bench.py)", "",
                  "| arm | GPUs | model | optimizer | tokens/s (device) | tokens/s (end to end) | ms / step "
                  "| optimizer ms | SM MHz | source |",
                  "|---|---|---|---|---|---|---|---|---|---|"]
        for b in sorted(data["bench"], key=lambda b: (b.get("model") or "", b.get("optimizer") or "",
                                                       b["n_gpus"] or 0, b["impl"])):
            lines.append(f"| {b['impl']} | {b['n_gpus']} | {b.get('model')} | {b.get('optimizer')} | "
                         f"{_fmt(b['value'], 0)} | {_fmt(b.get('e2e'), 0)} | {_fmt(b.get('ms_per_step'))} | "
                         f"{_fmt(b.get('optimizer_step_ms'))} | {_fmt(b.get('sm_mhz'), 0)} | {b['source']} |")
        fig = _scaling_figure(data["bench"])
        if fig is not None:
            fig.save(os.path.join(out_dir, "throughput.svg"))
            lines += ["", "![throughput](throughput.svg)", ""]
        lines.append("")
    if data["optimizer"]:
        lines += ["## Optimizer step (optimizer_bench)", "",
                  "| optimizer | arm | GPUs | peer-memory path | ms | matrices |", "|---|---|---|---|---|---|"]
        for o in sorted(data["optimizer"], key=lambda o: (o["optimizer"] or "", o["n_gpus"] or 0, str(o["p2p"]))):
            lines.append(f"| {o['optimizer']} | {o['impl']} | {o['n_gpus']} | {o['p2p']} | {_fmt(o['ms'])} | "
                         f"{o['matrices']} |")
        lines.append("")
    path = os.path.join(out_dir, "report.md")
    with open(path, "w") as f:
        f.write("\n".join(lines))
    with open(os.path.join(out_dir, "data.json"), "w") as f:
        json.dump(data, f, indent=1)
    return path


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--parity", nargs="*", default=[])
    p.add_argument("--bench", nargs="*", default=[])
    p.add_argument("--optimizer", nargs="*", default=[])
    p.add_argument("--data", default=None,
                   help="start from a data.json written by an earlier run (inputs given here are added)")
    p.add_argument("--out", required=True)
    a = p.parse_args(argv)
    data = collect(a.parity, a.bench, a.optimizer)
    if a.data:  # an earlier run's data, with this call's inputs added
        with open(a.data) as f:
            old = json.load(f)
        for k in ("parity", "bench", "optimizer"):
            data[k] = old.get(k, []) + data[k]
    print(render(data, a.out))


if __name__ == "__main__":
    main()
