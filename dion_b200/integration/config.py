"""Job configuration: a dataclass tree plus a ``--section.field value`` CLI.

Section and field names follow the torchtitan-style config the reference
registers (ada_dion/integration/config_registry.py:161-184 for training, lr
scheduler and metrics; hybrid_optimizer.py:62-113 for the optimizer), so
the reference's command lines carry over, e.g.

    python -m dion_b200.train --config llama3_160m_dion --optimizer.lr 0.01 \\
        --training.steps 500 --parallelism.data_parallel_shard_degree 4

Booleans accept ``--section.use-x`` / ``--section.no-use-x`` as well as an
explicit value.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

from .hybrid_optimizer import HybridOptimizersContainer

__all__ = [
    "ModelConfig",
    "TrainingConfig",
    "LRSchedulerConfig",
    "ActivationCheckpointConfig",
    "ParallelismConfig",
    "CheckpointConfig",
    "MetricsConfig",
    "DataConfig",
    "ValidatorConfig",
    "ProfilingConfig",
    "DebugConfig",
    "CompileConfig",
    "JobConfig",
    "apply_overrides",
]


@dataclass
class ModelConfig:
    name: str = "llama3"
    flavor: str = "160M"
    overrides: Dict[str, Any] = field(default_factory=dict)
    init: str = "normal"


@dataclass
class TrainingConfig:
    local_batch_size: int = 8
    global_batch_size: int = -1  # > local x data-parallel degree: gradient accumulation
    seq_len: int = 2048
    steps: int = 10000
    dtype: str = "bfloat16"
    # FSDP mixed precision (torchtitan's names): compute dtype of the gathered
    # parameters, and dtype of the gradient reduction
    mixed_precision_param: str = "bfloat16"
    mixed_precision_reduce: str = "float32"
    max_norm: float = 1.0
    seed: int = 0


@dataclass
class ActivationCheckpointConfig:
    mode: str = "none"  # none | full | selective
    selective_ac_option: str = "op"  # "op" or an integer N (every N-th block)


@dataclass
class LRSchedulerConfig:
    warmup_steps: int = 200
    decay_type: str = "cosine"  # cosine | linear | sqrt
    decay_ratio: Optional[float] = None  # decay over this fraction of the steps (None: all after warm-up)
    min_lr_factor: float = 0.1


@dataclass
class ParallelismConfig:
    data_parallel_replicate_degree: int = 1
    data_parallel_shard_degree: int = -1
    tensor_parallel_degree: int = 1
    pipeline_parallel_degree: int = 1
    pipeline_parallel_microbatches: int = 0
    pipeline_parallel_schedule: str = "1F1B"


@dataclass
class CheckpointConfig:
    enable: bool = False
    folder: str = "checkpoint"
    interval: int = 1000
    last_save_model_only: bool = True
    # resume from step-<load_step> instead of the newest full checkpoint (-1: newest)
    load_step: int = -1
    # when `folder` holds no checkpoint yet: start from this checkpoint (e.g. a
    # model-only export); with initial_load_model_only only its weights are taken
    initial_load_path: Optional[str] = None
    initial_load_model_only: bool = True
    # "async": write checkpoints in the background once the state is staged in host memory
    async_mode: str = "disabled"
    # dtype of the model-only final export (torchtitan's export_dtype)
    export_dtype: str = "float32"


@dataclass
class MetricsConfig:
    log_freq: int = 10
    enable_tensorboard: bool = False
    save_tb_folder: str = "tb"
    # W&B: project / run name / mode from WANDB_PROJECT, WANDB_RUN_NAME, WANDB_MODE
    enable_wandb: bool = False
    wandb_project: Optional[str] = None
    wandb_run_name: Optional[str] = None
    save_jsonl: Optional[str] = None
    # denominator of the logged MFU, TFLOP/s per GPU (0: the B200's 2250 dense bf16 figure;
    # pass a measured rate to report against it)
    peak_tflops: float = 0.0


@dataclass
class DataConfig:
    # "synthetic" or token files: comma-separated files, directories of *.bin or
    # glob patterns (written by `python -m dion_b200.data.tokenize`)
    # "text:<files>" (jsonl / json / parquet / txt) tokenizes on the fly with `tokenizer`
    dataset: str = "synthetic"
    seed: int = 0
    tokenizer: str = "byte"  # for "text:" datasets: "byte" or a local HuggingFace tokenizer directory
    text_field: str = "text"
    shuffle: bool = True
    prefetch: int = 4
    bytes_per_token: int = 0  # raw token files without a header: 2 or 4


@dataclass
class ValidatorConfig:
    enable: bool = False
    freq: int = 100
    steps: int = 20
    dataset: str = ""  # held-out token files (same forms as dataloader.dataset)


@dataclass
class ProfilingConfig:
    enable_profiling: bool = False
    save_traces_folder: str = "profile_traces"
    profile_freq: int = 100


@dataclass
class CompileConfig:
    # torchtitan's [compile] section, accepted so its command lines carry over:
    # the model's hot ops are hand-written kernels here, so torch.compile is
    # not applied and ``enable`` only prints a note
    enable: bool = False
    components: str = "model,loss"


@dataclass
class DebugConfig:
    # torchtitan's [debug] section: ``--debug.seed`` (taking precedence over
    # training.seed) and ``--debug.deterministic``
    seed: int = 0
    deterministic: bool = False


@dataclass
class JobConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    optimizer: HybridOptimizersContainer.Config = field(default_factory=HybridOptimizersContainer.Config)
    lr_scheduler: LRSchedulerConfig = field(default_factory=LRSchedulerConfig)
    training: TrainingConfig = field(default_factory=TrainingConfig)
    activation_checkpoint: ActivationCheckpointConfig = field(default_factory=ActivationCheckpointConfig)
    parallelism: ParallelismConfig = field(default_factory=ParallelismConfig)
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    metrics: MetricsConfig = field(default_factory=MetricsConfig)
    dataloader: DataConfig = field(default_factory=DataConfig)
    validator: ValidatorConfig = field(default_factory=ValidatorConfig)
    profiling: ProfilingConfig = field(default_factory=ProfilingConfig)
    debug: DebugConfig = field(default_factory=DebugConfig)
    compile: CompileConfig = field(default_factory=CompileConfig)

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


def _coerce(cur: Any, text: str) -> Any:
    if isinstance(cur, bool):
        if text.lower() in ("1", "true", "yes", "on"):
            return True
        if text.lower() in ("0", "false", "no", "off"):
            return False
        raise ValueError(f"not a boolean: {text}")
    if isinstance(cur, int) and not isinstance(cur, bool):
        return int(text)
    if isinstance(cur, float):
        return float(text)
    if cur is None:
        for conv in (int, float):
            try:
                return conv(text)
            except ValueError:
                pass
        return None if text.lower() == "none" else text
    return text


def apply_overrides(cfg: JobConfig, argv: Sequence[str]) -> List[str]:
    """Apply ``--section.field value`` overrides in place; returns unknown args."""
    rest: List[str] = []
    i = 0
    args = list(argv)
    while i < len(args):
        a = args[i]
        if not a.startswith("--") or "." not in a:
            rest.append(a)
            i += 1
            continue
        key = a[2:]
        val: Optional[str] = None
        if "=" in key:
            key, val = key.split("=", 1)
        section, name = key.split(".", 1)
        section, name = section.replace("-", "_"), name.replace("-", "_")
        sec = getattr(cfg, section, None)
        if sec is None:
            rest.append(a)
            i += 1
            continue
        negate = False
        if not hasattr(sec, name) and name.startswith("no_") and hasattr(sec, name[3:]):
            name, negate = name[3:], True
        if not hasattr(sec, name):
            raise ValueError(f"unknown config field --{section}.{name}")
        cur = getattr(sec, name)
        if isinstance(cur, bool) and (val is None) and (i + 1 >= len(args) or args[i + 1].startswith("--")):
            setattr(sec, name, not negate)
            i += 1
            continue
        if val is None:
            val = args[i + 1]
            i += 1
        setattr(sec, name, _coerce(cur, val) if not negate else not _coerce(cur, val))
        i += 1
    return rest
