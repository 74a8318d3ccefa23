"""Training entry point.

    python -m dion_b200.train --config llama3_160m_dion [--section.field value ...]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dion_b200.train --config llama3_1b_muon

Builds the model, FSDP2/HSDP mesh, hybrid optimizer and LR schedule from a
registered :class:`~dion_b200.integration.config.JobConfig`, trains on
synthetic uniform tokens or token files (``--dataloader.dataset``), logs
torchtitan-style lines (step, loss, grad_norm, memory, tps, tflops, mfu),
runs a validation pass every ``--validator.freq`` steps when enabled,
records profiler traces every ``--profiling.profile_freq`` steps when
enabled, and optionally writes JSONL metrics and DCP checkpoints (with the
data position).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from typing import List, Optional

import torch
import torch.distributed as dist

from .integration.config import JobConfig, apply_overrides
from .integration.config_registry import get_config
from .integration.trainer import Trainer, TrainerConfig

__all__ = ["trainer_config_from_job", "parse_job", "main"]

# default MFU denominator: B200 dense bf16 (--metrics.peak_tflops sets another, e.g. a measured rate)
PEAK_FLOPS = {"bfloat16": 2.25e15}


def trainer_config_from_job(job: JobConfig) -> TrainerConfig:
    par = job.parallelism
    return TrainerConfig(
        model=job.model.flavor,
        model_overrides=dict(job.model.overrides),
        seq_len=job.training.seq_len,
        local_batch_size=job.training.local_batch_size,
        steps=job.training.steps,
        warmup_steps=job.lr_scheduler.warmup_steps,
        min_lr_factor=job.lr_scheduler.min_lr_factor,
        decay_ratio=job.lr_scheduler.decay_ratio,
        decay_type=job.lr_scheduler.decay_type,
        max_norm=job.training.max_norm,
        seed=job.debug.seed or job.training.seed or job.dataloader.seed,
        init_mode=job.model.init,
        dp_replicate=par.data_parallel_replicate_degree,
        dp_shard=par.data_parallel_shard_degree,
        tp=par.tensor_parallel_degree,
        pp=par.pipeline_parallel_degree,
        pp_microbatches=par.pipeline_parallel_microbatches,
        pp_schedule=par.pipeline_parallel_schedule,
        optimizer=job.optimizer,
        log_freq=job.metrics.log_freq,
        ac_mode=job.activation_checkpoint.mode,
        ac_option=job.activation_checkpoint.selective_ac_option,
        dataset=job.dataloader.dataset,
        data_shuffle=job.dataloader.shuffle,
        data_prefetch=job.dataloader.prefetch,
        data_bytes_per_token=job.dataloader.bytes_per_token,
        data_tokenizer=job.dataloader.tokenizer,
        data_text_field=job.dataloader.text_field,
        val_dataset=job.validator.dataset if job.validator.enable else "",
        global_batch_size=job.training.global_batch_size,
        param_dtype=job.training.mixed_precision_param,
        reduce_dtype=job.training.mixed_precision_reduce,
    )


def _profiler(job: JobConfig, tr: Trainer):
    """torch.profiler over the training loop when ``--profiling.enable_profiling``:
    every ``profile_freq`` steps the last step is recorded (one warm-up step
    before it) and written as a Chrome trace to
    ``<save_traces_folder>/iteration_<step>/rank<r>_trace.json``, the layout
    torchtitan uses and ``benchmarks.tiers.parse_profiler_trace`` reads."""
    pc = job.profiling
    if not pc.enable_profiling:
        return None
    freq = max(2, int(pc.profile_freq))
    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)

    def on_ready(p):
        d = os.path.join(pc.save_traces_folder, f"iteration_{tr.step_idx}")
        os.makedirs(d, exist_ok=True)
        p.export_chrome_trace(os.path.join(d, f"rank{tr.rank}_trace.json"))

    prof = torch.profiler.profile(activities=acts, schedule=torch.profiler.schedule(wait=freq - 2, warmup=1, active=1),
                                  on_trace_ready=on_ready)
    prof.__enter__()
    return prof


def _load_config(module: Optional[str], name: str) -> JobConfig:
    """Config ``name`` from this package's registry, or from ``module``'s
    function of that name (so experiment modules can add configs)."""
    if module in (None, "", "dion_b200.integration.config_registry", "ada_dion.integration.config_registry"):
        return get_config(name)
    import importlib

    mod = importlib.import_module(module)
    fn = getattr(mod, name, None)
    if fn is None:
        raise SystemExit(f"config {name!r} not found in module {module!r}")
    return fn()


def _print_fields(argv: List[str]) -> None:
    """Every ``--section.field`` of the job configuration, with its value in
    ``--config NAME`` (or the defaults)."""
    import dataclasses

    job = JobConfig()
    if "--config" in argv:
        i = argv.index("--config")
        job = _load_config(None, argv[i + 1])
    for sec in dataclasses.fields(job):
        val = getattr(job, sec.name)
        if not dataclasses.is_dataclass(val):
            continue
        for f in dataclasses.fields(val):
            print(f"--{sec.name}.{f.name} {getattr(val, f.name)!r}")


def parse_job(argv: List[str]) -> JobConfig:
    """The job configuration a command line selects: ``--config`` (and
    ``--module``), then every ``--section.field value`` override. The
    reference's torchtitan command lines parse as they are: section and field
    names may use hyphens, ``--compile.*`` is accepted (torch.compile is not
    used: the hot ops are hand-written kernels) and ``--hf-assets-path``
    names the tokenizer assets (the data comes from token files here)."""
    if "--list-fields" in argv:
        _print_fields(argv)
        raise SystemExit(0)
    p = argparse.ArgumentParser(add_help=True, epilog="--list-fields [--config NAME]: every --section.field "
                                                      "override with its value in that config")
    p.add_argument("--config", required=True)
    p.add_argument("--module", default=None,
                   help="module whose config functions to use (torchtitan-style --module); "
                        "default: dion_b200.integration.config_registry")
    p.add_argument("--job.config_file", dest="unused", default=None)
    p.add_argument("--hf-assets-path", "--hf_assets_path", dest="hf_assets_path", default=None,
                   help="tokenizer assets; pass them to `python -m dion_b200.data.tokenize --tokenizer`")
    known, rest = p.parse_known_args(argv)
    job = _load_config(known.module, known.config)
    leftover = apply_overrides(job, rest)
    if leftover:
        raise SystemExit(f"unrecognised arguments: {leftover}")
    job.hf_assets_path = known.hf_assets_path
    return job


def main(argv: Optional[List[str]] = None) -> List[float]:
    argv = list(sys.argv[1:] if argv is None else argv)
    job = parse_job(argv)
    rank0 = int(os.environ.get("RANK", "0")) == 0
    if job.compile.enable and rank0:
        print("note: --compile.enable has no effect (the model's hot ops are hand-written sm_100a kernels)",
              flush=True)
    if getattr(job, "hf_assets_path", None) and job.dataloader.dataset == "synthetic" and rank0:
        print(f"note: --hf-assets-path {job.hf_assets_path}: tokenize the corpus with `python -m "
              "dion_b200.data.tokenize --tokenizer <that directory>` and pass --dataloader.dataset; "
              "training on synthetic tokens", flush=True)
    if job.validator.enable and not job.validator.dataset:
        raise SystemExit("--validator.enable needs held-out token files: --validator.dataset PATH")
    if job.debug.deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)
        torch.backends.cudnn.benchmark = False
    tc = trainer_config_from_job(job)
    tr = Trainer(tc)
    from .benchmarks.metrics_collector import OptimizerMetricsCollector

    collector = None
    tb = wb = None
    if tr.rank == 0:
        mc = job.metrics
        if mc.enable_tensorboard:
            try:
                from torch.utils.tensorboard import SummaryWriter

                tb = SummaryWriter(log_dir=mc.save_tb_folder)
            except Exception as e:  # a missing package must not stop the run
                print(f"warning: TensorBoard disabled ({type(e).__name__}: {e})", flush=True)
        if mc.enable_wandb:
            try:
                import wandb

                # without credentials (or with WANDB_MODE=offline) the run is recorded locally
                # for a later `wandb sync`: a node without network access never waits on W&B
                mode = os.environ.get("WANDB_MODE") or ("online" if os.environ.get("WANDB_API_KEY") else "offline")
                wb = wandb.init(project=mc.wandb_project or os.environ.get("WANDB_PROJECT", "dion_b200"),
                                name=mc.wandb_run_name or os.environ.get("WANDB_RUN_NAME"), config=job.to_dict(),
                                mode=mode)
            except Exception as e:
                print(f"warning: W&B disabled ({type(e).__name__}: {e})", flush=True)
                wb = None
        if mc.save_jsonl or tb is not None or wb is not None:
            collector = OptimizerMetricsCollector(tr.optimizers, output_dir=mc.save_jsonl or mc.save_tb_folder,
                                                  tb_writer=tb, wandb_run=wb)
    ckpt = None
    if job.checkpoint.enable:
        from .checkpoint import CheckpointManager

        ckpt = CheckpointManager(job.checkpoint.folder, tr.model, tr.optimizers, interval=job.checkpoint.interval,
                                 model_only_last=job.checkpoint.last_save_model_only,
                                 async_mode=job.checkpoint.async_mode,
                                 export_dtype=getattr(torch, job.checkpoint.export_dtype))
        cc = job.checkpoint
        ckpt.maybe_load(tr, load_step=cc.load_step, initial_load_path=cc.initial_load_path,
                        initial_load_model_only=cc.initial_load_model_only)
    prof = _profiler(job, tr)
    flops_tok = tr.model_cfg.flops_per_token(tc.seq_len)
    tokens_step = tc.local_batch_size * tr.grad_accum * tc.seq_len
    losses: List[float] = []
    t_last = time.perf_counter()
    for step in range(tr.step_idx, tc.steps):
        t, l = tr.data.next()
        loss = tr.train_step(t, l)
        s = step + 1
        if s % tc.log_freq == 0 or s == tc.steps:
            v = float(loss.item())
            losses.append(v)
            torch.cuda.synchronize() if torch.cuda.is_available() else None
            now = time.perf_counter()
            dt = (now - t_last) / max(1, tc.log_freq)
            t_last = now
            tps = tokens_step / dt
            tflops = flops_tok * tps / 1e12
            mem = torch.cuda.max_memory_allocated() / 2**30 if torch.cuda.is_available() else 0.0
            peak = job.metrics.peak_tflops * 1e12 if job.metrics.peak_tflops > 0 else PEAK_FLOPS["bfloat16"]
            mfu = 100.0 * flops_tok * tps / peak
            gn = tr.last_grad_norm
            if tr.rank == 0:
                print(f"step: {s:5d}  loss: {v:8.4f}  grad_norm: {gn:7.4f}  memory: {mem:5.2f}GiB  "
                      f"tps: {tps:,.0f}  tflops: {tflops:,.2f}  mfu: {mfu:.2f}%", flush=True)
            if collector is not None:
                collector.collect(s, loss=v, grad_norm=gn, tps=tps)
        if job.validator.enable and (s % job.validator.freq == 0 or s == tc.steps):
            vloss = tr.validate(job.validator.steps)
            if tr.rank == 0:
                print(f"validate step: {s:5d}  loss: {vloss:8.4f}", flush=True)
            if collector is not None:
                collector.collect(s, val_loss=vloss)
        if ckpt is not None:
            ckpt.maybe_save(tr, s, final=(s == tc.steps))
        if prof is not None:
            prof.step()
    if prof is not None:
        prof.__exit__(None, None, None)
    if ckpt is not None:
        ckpt.wait()
    if collector is not None:
        collector.close()
    if tb is not None:
        tb.close()
    if wb is not None:
        wb.finish()
    if dist.is_initialized():
        dist.barrier()
    return losses


if __name__ == "__main__":
    main()
