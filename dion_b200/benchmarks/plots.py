"""Benchmark and diagnostics plots (SVG, no plotting library needed).

Same functions and input dictionaries as the reference's plot library
(ada_dion/benchmarks/plots.py:84-635) so its analysis notebooks' data feeds
straight in; each returns a :class:`dion_b200.utils.svgplot.Figure`.

    runs = {"dion": {"tokens": [...], "val_loss": [...]}, "muon": {...}}
    save_all_plots("plots/", runs=runs, dion_data=..., dion2_data=..., adadion_data=...)
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional

from ..utils.svgplot import Figure

__all__ = [
    "plot_val_loss_vs_tokens", "plot_val_loss_vs_wallclock", "plot_tokens_per_sec", "plot_scaling_tokens_per_sec",
    "plot_step_time_breakdown", "plot_communicated_bytes", "plot_collective_time", "plot_comm_compute_ratio",
    "plot_dion_rank_residual", "plot_dion2_alpha_sparsity", "plot_adadion_diagnostics", "plot_adadion_anchor_drift",
    "plot_adadion_tail_ratio", "plot_adadion_effective_rank", "plot_adadion_energy_captured", "load_metrics_jsonl",
    "save_all_plots",
]

COLORS = {"adamw": "#7f7f7f", "muon": "#1f77b4", "dion": "#d62728", "dion2": "#2ca02c", "adadion": "#ff7f0e",
          "adadion_v2": "#9467bd"}
LABELS = {"adamw": "AdamW", "muon": "Muon", "dion": "Dion", "dion2": "Dion2", "adadion": "AdaDion",
          "adadion_v2": "AdaDionV2"}


def _lines(runs: Dict[str, dict], xkey: str, ykey: str, title: str, xlabel: str, ylabel: str,
           markers: bool = False) -> Figure:
    fig = Figure()
    ax = fig.axes[0]
    for name, d in runs.items():
        ax.line(d[xkey], d[ykey], label=LABELS.get(name, name), color=COLORS.get(name), markers=markers)
    ax.set(title=title, xlabel=xlabel, ylabel=ylabel)
    return fig


def plot_val_loss_vs_tokens(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"tokens": [...], "val_loss": [...]}}"""
    return _lines(runs, "tokens", "val_loss", "Validation Loss vs Tokens", "Tokens", "Validation Loss")


def plot_val_loss_vs_wallclock(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"time_s": [...], "val_loss": [...]}}"""
    return _lines(runs, "time_s", "val_loss", "Validation Loss vs Wall-clock", "Time (s)", "Validation Loss")


def plot_tokens_per_sec(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"step": [...], "tokens_per_sec": [...]}}"""
    return _lines(runs, "step", "tokens_per_sec", "Throughput Stability", "Training Step", "Tokens/sec")


def plot_scaling_tokens_per_sec(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"num_gpus": [...], "tokens_per_sec": [...]}}; dashed = linear scaling of the first run."""
    fig = _lines(runs, "num_gpus", "tokens_per_sec", "Scaling Efficiency", "Number of GPUs", "Tokens/sec", True)
    if runs:
        first = next(iter(runs.values()))
        if first["num_gpus"]:
            g0, t0 = first["num_gpus"][0], first["tokens_per_sec"][0]
            fig.axes[0].line(first["num_gpus"], [t0 * g / g0 for g in first["num_gpus"]], label="ideal",
                             color="#999999", dashed=True)
    return fig


def _stacked(runs: Dict[str, dict], keys: List[str], title: str, ylabel: str, scale: float = 1.0,
             stacked: bool = True) -> Figure:
    fig = Figure()
    names = list(runs)
    vals = [[float(runs[n].get(k, 0.0)) * scale for n in names] for k in keys]
    fig.axes[0].bar([LABELS.get(n, n) for n in names], [k.replace("_ms", "").replace("_bytes", "") for k in keys],
                    vals, stacked=stacked)
    fig.axes[0].set(title=title, ylabel=ylabel)
    return fig


def plot_step_time_breakdown(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"fwd_ms", "bwd_ms", "opt_ms", "nccl_ms"}}"""
    return _stacked(runs, ["fwd_ms", "bwd_ms", "opt_ms", "nccl_ms"], "Step Time Breakdown", "Time (ms)")


def plot_communicated_bytes(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"allreduce_bytes", "allgather_bytes", "reducescatter_bytes"}} (bytes per step)"""
    return _stacked(runs, ["allreduce_bytes", "allgather_bytes", "reducescatter_bytes"],
                    "Communication Volume per Step", "Communicated (MB/step)", scale=1.0 / 2**20)


def plot_collective_time(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"allreduce_ms", "allgather_ms", "reducescatter_ms"}}"""
    return _stacked(runs, ["allreduce_ms", "allgather_ms", "reducescatter_ms"], "Collective Time per Step",
                    "Time (ms/step)")


def plot_comm_compute_ratio(runs: Dict[str, dict]) -> Figure:
    """runs: {optimizer: {"num_gpus": [...], "comm_compute_ratio": [...]}}"""
    return _lines(runs, "num_gpus", "comm_compute_ratio", "Communication Overhead vs Scale", "Number of GPUs",
                  "Comm / Compute Ratio", True)


def plot_dion_rank_residual(data: dict) -> Figure:
    """data: {"step": [...], "rank_mean": [...], "residual_norm_mean": [...]}"""
    fig = Figure(ncols=2)
    fig.axes[0].line(data["step"], data["rank_mean"], color=COLORS["dion"])
    fig.axes[0].set(title="Dion: Effective Rank", xlabel="Training Step", ylabel="Rank (mean across layers)")
    fig.axes[1].line(data["step"], data["residual_norm_mean"], color=COLORS["dion"])
    fig.axes[1].set(title="Dion: Residual Norm (after error feedback)", xlabel="Training Step",
                    ylabel="||M||_F (mean)")
    return fig


def plot_dion2_alpha_sparsity(data: dict) -> Figure:
    """data: {"step": [...], "alpha": [...], "sparsity": [...], "selected_frac_mean": [...]}"""
    fig = Figure(ncols=2)
    fig.axes[0].line(data["step"], data["selected_frac_mean"], color=COLORS["dion2"], label="selected")
    fig.axes[0].hline(data["alpha"][0] if data.get("alpha") else 0.25, label="target alpha")
    fig.axes[0].set(title="Dion2: Selected Row/Col Fraction", xlabel="Training Step", ylabel="Selected Fraction")
    fig.axes[1].line(data["step"], data["sparsity"], color=COLORS["dion2"])
    fig.axes[1].set(title="Dion2: Update Sparsity", xlabel="Training Step", ylabel="Sparsity (1 - fraction updated)")
    return fig


def plot_adadion_diagnostics(data: dict) -> Figure:
    """data: {"step": [...], plus any of "rank_mean", "erank_mean", "aerr_mean", "anchor_drift_mean",
    "tail_ratio_mean", "energy_captured_mean"} -- one panel per present key."""
    keys = [k for k in ("rank_mean", "erank_mean", "aerr_mean", "anchor_drift_mean", "tail_ratio_mean",
                        "energy_captured_mean") if k in data]
    ncols = min(3, max(1, len(keys)))
    fig = Figure(ncols=ncols, nrows=max(1, (len(keys) + ncols - 1) // ncols), title="AdaDion diagnostics")
    for ax, k in zip(fig.axes, keys):
        ax.line(data["step"], data[k], color=COLORS["adadion"])
        ax.set(title=k.replace("_mean", "").replace("_", " "), xlabel="Training Step", ylabel=k)
    return fig


def _single(data: dict, key: str, title: str, ylabel: str) -> Figure:
    fig = Figure()
    fig.axes[0].line(data["step"], data[key], color=COLORS["adadion"])
    fig.axes[0].set(title=title, xlabel="Training Step", ylabel=ylabel)
    return fig


def plot_adadion_anchor_drift(data: dict) -> Figure:
    return _single(data, "anchor_drift_mean", "AdaDion: Anchor Drift", "||Q - Q_anchor||_F")


def plot_adadion_tail_ratio(data: dict) -> Figure:
    return _single(data, "tail_ratio_mean", "AdaDion: Tail Energy Ratio", "||(I - QQ^T) M|| / ||M||")


def plot_adadion_effective_rank(data: dict) -> Figure:
    return _single(data, "erank_mean", "AdaDion: Effective Rank (EMA)", "effective rank")


def plot_adadion_energy_captured(data: dict) -> Figure:
    return _single(data, "energy_captured_mean", "AdaDion: Energy Captured", "fraction of ||M||^2")


def load_metrics_jsonl(path: str) -> List[dict]:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def save_all_plots(output_dir: str, runs: Optional[dict] = None, dion_data: Optional[dict] = None,
                   dion2_data: Optional[dict] = None, adadion_data: Optional[dict] = None) -> List[str]:
    """Write every plot whose inputs are present; returns the written paths."""
    os.makedirs(output_dir, exist_ok=True)
    written: List[str] = []

    def save(fig: Figure, name: str) -> None:
        written.append(fig.save(os.path.join(output_dir, name)))

    if runs:
        def has(*keys):
            return all(all(k in r for k in keys) for r in runs.values())

        if has("tokens", "val_loss"):
            save(plot_val_loss_vs_tokens(runs), "01_val_loss_vs_tokens.svg")
        if has("time_s", "val_loss"):
            save(plot_val_loss_vs_wallclock(runs), "02_val_loss_vs_wallclock.svg")
        if has("step", "tokens_per_sec"):
            save(plot_tokens_per_sec(runs), "03_tokens_per_sec.svg")
        if has("num_gpus", "tokens_per_sec"):
            save(plot_scaling_tokens_per_sec(runs), "04_scaling.svg")
        if has("fwd_ms"):
            save(plot_step_time_breakdown(runs), "05_step_time_breakdown.svg")
        if has("allreduce_bytes"):
            save(plot_communicated_bytes(runs), "06_communicated_bytes.svg")
        if has("allreduce_ms"):
            save(plot_collective_time(runs), "07_collective_time.svg")
        if has("num_gpus", "comm_compute_ratio"):
            save(plot_comm_compute_ratio(runs), "08_comm_compute_ratio.svg")
    if dion_data:
        save(plot_dion_rank_residual(dion_data), "09_dion_rank_residual.svg")
    if dion2_data:
        save(plot_dion2_alpha_sparsity(dion2_data), "10_dion2_alpha_sparsity.svg")
    if adadion_data:
        save(plot_adadion_diagnostics(adadion_data), "11_adadion_diagnostics.svg")
    return written
