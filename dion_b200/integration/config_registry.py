"""Named training configurations.

Same function names and settings as the reference's registry
(ada_dion/integration/config_registry.py:191-656 and
ada_dion/optim/config_registry.py:102-237): Llama-3 160M / 320M / debug with
AdamW, Muon, Dion, Dion2 or AdaDion (SDion in baseline mode, as the
reference's container routes it), and the AdaDionV2 320M configurations;
plus the 1B / 8B flavours used by the B200 benchmarks.

    from dion_b200.integration.config_registry import get_config
    cfg = get_config("llama3_160m_dion")
"""
from __future__ import annotations

from typing import Callable, Dict

from .config import (
    CheckpointConfig,
    JobConfig,
    LRSchedulerConfig,
    MetricsConfig,
    ModelConfig,
    TrainingConfig,
    ValidatorConfig,
)
from .hybrid_optimizer import HybridOptimizersContainer

Opt = HybridOptimizersContainer.Config
REGISTRY: Dict[str, Callable[[], JobConfig]] = {}


def register(fn: Callable[[], JobConfig]) -> Callable[[], JobConfig]:
    REGISTRY[fn.__name__] = fn
    return fn


def get_config(name: str) -> JobConfig:
    if name not in REGISTRY:
        raise KeyError(f"unknown config {name!r}; known: {sorted(REGISTRY)}")
    return REGISTRY[name]()


def _base(flavor: str, opt: Opt, steps: int = 10000, warmup: int = 200, lbs: int = 8, seq: int = 2048,
          ckpt_interval: int = 1000, model_only: bool = True) -> JobConfig:
    return JobConfig(
        model=ModelConfig(flavor=flavor),
        optimizer=opt,
        lr_scheduler=LRSchedulerConfig(warmup_steps=warmup, decay_type="cosine", min_lr_factor=0.1),
        training=TrainingConfig(local_batch_size=lbs, seq_len=seq, steps=steps, dtype="bfloat16", max_norm=1.0),
        checkpoint=CheckpointConfig(interval=ckpt_interval, last_save_model_only=model_only),
        metrics=MetricsConfig(log_freq=10, enable_tensorboard=True, enable_wandb=True),
        validator=ValidatorConfig(freq=100, steps=20),
    )


def _adamw(lr: float) -> Opt:
    # plain AdamW everywhere: every group runs the scalar rule
    return Opt(name="AdamW", lr=lr, weight_decay=0.1, scalar_lr=lr, scalar_beta1=0.9, scalar_beta2=0.95,
               scalar_weight_decay=0.1)


def _muon() -> Opt:
    return Opt(name="Muon", lr=0.02, mu=0.95, weight_decay=0.0, scalar_lr=3e-4, scalar_weight_decay=0.01)


def _dion() -> Opt:
    return Opt(name="Dion", lr=0.02, rank_fraction=0.25, weight_decay=0.0, scalar_lr=3e-4, scalar_weight_decay=0.01)


def _dion2() -> Opt:
    return Opt(name="Dion2", lr=0.02, fraction=0.25, ef_decay=0.95, weight_decay=0.0, scalar_lr=3e-4,
               scalar_weight_decay=0.01)


def _adadion() -> Opt:
    return Opt(name="AdaDion", lr=0.02, mu=0.95, init_rank=64, rank_min=16, rank_max=256, weight_decay=0.0,
               scalar_lr=3e-4, scalar_weight_decay=0.01, sdion_mode="baseline")


# ---------------------------------------------------------------- 160M
@register
def llama3_160m_adamw() -> JobConfig:
    return _base("160M", _adamw(3e-4))


@register
def llama3_160m_muon() -> JobConfig:
    return _base("160M", _muon())


@register
def llama3_160m_dion() -> JobConfig:
    return _base("160M", _dion())


@register
def llama3_160m_dion2() -> JobConfig:
    return _base("160M", _dion2())


@register
def llama3_160m_adadion() -> JobConfig:
    return _base("160M", _adadion())


# ---------------------------------------------------------------- 320M (warmup 610, 6104 steps, cosine to 0)
def _320m(opt: Opt) -> JobConfig:
    cfg = _base("320M", opt, steps=6104, warmup=610)
    cfg.lr_scheduler.min_lr_factor = 0.0  # ada_dion/integration/config_registry.py:359-364
    return cfg


@register
def llama3_320m_adamw() -> JobConfig:
    opt = _adamw(0.008)
    opt.scalar_beta1 = 0.95  # betas (0.95, 0.95) for the 320M AdamW baseline
    return _320m(opt)


@register
def llama3_320m_muon() -> JobConfig:
    return _320m(_muon())


@register
def llama3_320m_dion() -> JobConfig:
    return _320m(_dion())


@register
def llama3_320m_dion2() -> JobConfig:
    return _320m(_dion2())


@register
def llama3_320m_adadion() -> JobConfig:
    return _320m(_adadion())


def _adadion_v2(adaptive: bool, rf: float = 0.25) -> Opt:
    return Opt(name="AdaDionV2", lr=0.02, mu=0.95, weight_decay=0.1, adaptive_rank=adaptive,
               rank_fraction_max=0.7 if adaptive else rf, init_rank_fraction=rf, rank_min=16, rank_quantize=8,
               rank_step_up=16, rank_step_down=8, erank_ema_beta=0.9, scalar_lr=3e-4, scalar_weight_decay=0.01)


def _320m_adadion_v2(adaptive: bool, init_rank_fraction: float = 0.5) -> JobConfig:
    """The reference's 320M AdaDionV2 trainer (ada_dion/optim/config_registry.py:102-191):
    Dion-matched hyper-parameters (lr 0.012, rank fraction 1/2), adaptive rank up to
    0.7, warm-up 610 then cosine to 0, selective AC every 2nd block, no LM-head lr
    scaling."""
    opt = Opt(name="AdaDionV2", lr=0.012, mu=0.95, rank_fraction=0.5, adaptive_rank=adaptive,
              init_rank_fraction=init_rank_fraction, rank_fraction_max=0.7, erank_ema_beta=0.5, rank_scale=1.5,
              rank_min=16, rank_quantize=8, weight_decay=0.1, scalar_lr=0.012, scalar_beta1=0.95,
              scalar_beta2=0.95, scalar_eps=1e-8, scalar_weight_decay=0.1, output_head_lr_scaling=False)
    cfg = _320m(opt)
    cfg.activation_checkpoint.mode = "selective"
    cfg.activation_checkpoint.selective_ac_option = "2"
    return cfg


@register
def llama3_320m_adadion_v2() -> JobConfig:
    return _320m_adadion_v2(True)


@register
def llama3_320m_adadion_v2_dion_lr() -> JobConfig:
    return _320m_adadion_v2(True)


@register
def llama3_320m_adadion_v2_dion_equivalent() -> JobConfig:
    """adaptive_rank off: exactly Dion at rank fraction 1/2 (must match llama3_320m_dion's val loss)."""
    return _320m_adadion_v2(False)


@register
def llama3_320m_adadion_v2_fixed() -> JobConfig:
    return _320m_adadion_v2(False)


# ---------------------------------------------------------------- debug (tiny, 10 steps, checkpoint every 10)
def _debug(opt: Opt) -> JobConfig:
    cfg = _base("debug", opt, steps=10, warmup=2, ckpt_interval=10, model_only=False)
    # the reference's debug schedule: 2 warm-up steps, linear decay to 0 over the last 80 %
    cfg.lr_scheduler = LRSchedulerConfig(warmup_steps=2, decay_ratio=0.8, decay_type="linear", min_lr_factor=0.0)
    cfg.metrics.enable_tensorboard = False
    cfg.metrics.enable_wandb = False
    return cfg


@register
def llama3_debug_adamw() -> JobConfig:
    return _debug(_adamw(3e-4))


@register
def llama3_debug_muon() -> JobConfig:
    return _debug(_muon())


@register
def llama3_debug_dion() -> JobConfig:
    return _debug(_dion())


@register
def llama3_debug_dion2() -> JobConfig:
    return _debug(_dion2())


@register
def llama3_debug_adadion() -> JobConfig:
    return _debug(_adadion())


@register
def llama3_debug_adadion_v2() -> JobConfig:
    return _debug(_adadion_v2(True))


@register
def llama3_debug_2gpu_adadion_v2() -> JobConfig:
    """The tiny model for 2 GPUs, 50 steps, 4 sequences per GPU
    (ada_dion/optim/config_registry.py:198-217)."""
    opt = Opt(name="AdaDionV2", lr=0.012, rank_fraction=0.5, adaptive_rank=True, init_rank_fraction=0.25,
              rank_fraction_max=0.7, erank_ema_beta=0.5, rank_scale=1.5, rank_min=8, rank_quantize=8,
              weight_decay=0.1, scalar_lr=0.012, scalar_weight_decay=0.1)
    cfg = _debug(opt)
    cfg.training.steps = 50
    cfg.training.local_batch_size = 4
    return cfg


# ---------------------------------------------------------------- B200 benchmark flavours
@register
def llama3_1b_muon() -> JobConfig:
    """1B decoder, seq 4096, 8 sequences per GPU, Muon + AdamW, FSDP2."""
    cfg = _base("1B", _muon(), steps=10000, lbs=8, seq=4096)
    cfg.optimizer.weight_decay = 0.01
    return cfg


def _8b(opt: Opt) -> JobConfig:
    # 32K tokens per GPU: keep GEMM / attention outputs, recompute the
    # elementwise work (~90 GB of activations fits next to the sharded state
    # in 180 GB of HBM, so full recomputation is not needed)
    cfg = _base("8B", opt, steps=10000, lbs=4, seq=8192)
    cfg.activation_checkpoint.mode = "selective"
    cfg.activation_checkpoint.selective_ac_option = "op"
    return cfg


@register
def llama3_8b_dion() -> JobConfig:
    """8B decoder, seq 8192, 4 sequences per GPU, Dion rank 1/4 + AdamW, FSDP2."""
    return _8b(_dion())


@register
def llama3_8b_adadion_v2() -> JobConfig:
    """8B decoder, AdaDionV2 adaptive rank (initial 1/4, max 1/4, min rank 1/16 of d)."""
    opt = _adadion_v2(True)
    opt.rank_fraction_max = 0.25
    opt.init_rank_fraction = 0.25
    opt.rank_min = 4096 // 16
    return _8b(opt)


@register
def llama3_8b_dion2_fsdp_tp() -> JobConfig:
    """8B decoder on a 2-D mesh: FSDP 4 x TP 2, Dion2 (fraction 1/4), seq 8192, 4 sequences per data-parallel rank."""
    opt = _dion2()
    cfg = _8b(opt)
    cfg.parallelism.data_parallel_shard_degree = 4
    cfg.parallelism.tensor_parallel_degree = 2
    return cfg
