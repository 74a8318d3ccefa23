"""Integration layer on CPU: param grouping, hybrid container, config
registry and CLI overrides, trainer steps, metrics JSONL and DCP checkpoint
round trip (reference tests: test_param_grouper.py, test_hybrid_optimizer.py,
test_adadion_e2e.py config/metrics sections)."""
import json
import math
import os

import pytest
import torch
import torch.nn as nn

from dion_b200.integration.config import apply_overrides
from dion_b200.integration.config_registry import REGISTRY, get_config
from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer, build_param_groups
from dion_b200.integration.param_grouper import count_params, group_params_for_hybrid
from dion_b200.models.llama3 import Transformer, llama3_config


class _MockLlama(nn.Module):
    def __init__(self, d=16, n_layers=2, vocab=64):
        super().__init__()
        self.tok_embeddings = nn.Embedding(vocab, d)
        self.layers = nn.ModuleDict()
        for i in range(n_layers):
            blk = nn.Module()
            blk.attention = nn.Module()
            for n in ("wq", "wk", "wv", "wo"):
                setattr(blk.attention, n, nn.Linear(d, d, bias=False))
            blk.feed_forward = nn.Module()
            for n in ("w1", "w2", "w3"):
                setattr(blk.feed_forward, n, nn.Linear(d, d, bias=False))
            blk.attention_norm = nn.LayerNorm(d)
            blk.ffn_norm = nn.LayerNorm(d)
            self.layers[str(i)] = blk
        self.norm = nn.LayerNorm(d)
        self.output = nn.Linear(d, vocab, bias=False)


def test_grouper_counts_and_disjoint():
    m = _MockLlama()
    g = group_params_for_hybrid(m)
    assert len(g.matrix_params) == 2 * 7
    assert len(g.embed_params) == 1 and len(g.output_params) == 1
    ids = [id(p) for grp in g for p in grp]
    assert len(ids) == len(set(ids)) == len(list(m.parameters()))
    c = count_params(g)
    assert c["total"] == sum(p.numel() for p in m.parameters())


def test_grouper_hf_and_gpt_names():
    class HF(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_tokens = nn.Embedding(10, 8)
            self.q_proj_holder = nn.Module()
            self.self_attn = nn.Module()
            self.self_attn.q_proj = nn.Linear(8, 8)
            self.mlp = nn.Module()
            self.mlp.c_fc = nn.Linear(8, 8)
            self.lm_head = nn.Linear(8, 10)

    g = group_params_for_hybrid(HF())
    assert len(g.embed_params) == 1 and len(g.output_params) == 2  # lm_head weight + bias
    assert len(g.matrix_params) == 2  # q_proj.weight, c_fc.weight
    assert len(g.norm_params) == 2  # biases


@pytest.mark.parametrize("name", ["Muon", "Dion", "Dion2", "AdaDion", "AdaDionV2", "AdamW"])
def test_container_steps_each_optimizer(name):
    torch.manual_seed(0)
    m = _MockLlama()
    cfg = HybridOptimizersContainer.Config(name=name, lr=0.01, rank_fraction=0.5, init_rank=4, rank_min=2,
                                           rank_max=8)
    c = HybridOptimizersContainer(cfg, model_parts=[m])
    assert len(c) == 1 and len(list(iter(c))) == 1
    before = [p.detach().clone() for p in m.parameters()]
    x = torch.randint(0, 64, (3,))
    out = m.output(m.layers["0"].attention.wq(m.tok_embeddings(x)))
    (out.sum() + sum(p.sum() for p in m.parameters())).backward()
    c.step()
    c.zero_grad()
    changed = sum(not torch.equal(a, b.detach()) for a, b in zip(before, m.parameters()))
    assert changed == len(before)
    groups = c.get_optimizers()[0].param_groups
    out_group = [g for g in groups if any(p is m.output.weight for p in g["params"])][0]
    if name != "AdamW":
        assert math.isclose(out_group["lr"], cfg.scalar_lr / math.sqrt(16))
    norm_group = [g for g in groups if any(p is m.norm.weight for p in g["params"])][0]
    assert norm_group["weight_decay"] == 0.0


def test_registry_names_and_fields():
    for n in ["llama3_160m_adamw", "llama3_160m_muon", "llama3_160m_dion", "llama3_160m_dion2",
              "llama3_160m_adadion", "llama3_320m_muon", "llama3_debug_muon", "llama3_debug_dion",
              "llama3_320m_adadion_v2", "llama3_1b_muon", "llama3_8b_dion"]:
        assert n in REGISTRY
    c = get_config("llama3_160m_dion")
    assert c.optimizer.name == "Dion" and c.optimizer.rank_fraction == 0.25
    assert c.training.seq_len == 2048 and c.training.local_batch_size == 8 and c.training.max_norm == 1.0
    assert c.lr_scheduler.warmup_steps == 200 and c.lr_scheduler.min_lr_factor == 0.1
    assert get_config("llama3_320m_muon").lr_scheduler.warmup_steps == 610
    assert get_config("llama3_320m_dion").lr_scheduler.min_lr_factor == 0.0
    a = get_config("llama3_320m_adamw").optimizer
    assert (a.lr, a.scalar_beta1, a.scalar_beta2) == (0.008, 0.95, 0.95)
    assert get_config("llama3_debug_dion").checkpoint.interval == 10
    ls = get_config("llama3_debug_muon").lr_scheduler
    assert (ls.warmup_steps, ls.decay_ratio, ls.decay_type, ls.min_lr_factor) == (2, 0.8, "linear", 0.0)


def test_cli_overrides():
    c = get_config("llama3_160m_muon")
    rest = apply_overrides(c, ["--optimizer.lr", "0.005", "--training.steps=50", "--parallelism.data_parallel_shard_degree",
                               "4", "--optimizer.no-nesterov", "--checkpoint.enable", "--other"])
    assert rest == ["--other"]
    assert c.optimizer.lr == 0.005 and c.training.steps == 50
    assert c.parallelism.data_parallel_shard_degree == 4
    assert c.optimizer.nesterov is False and c.checkpoint.enable is True
    with pytest.raises(ValueError):
        apply_overrides(c, ["--optimizer.not_a_field", "1"])


def test_train_entry_and_metrics(tmp_path):
    from dion_b200 import train

    out = tmp_path / "m"
    losses = train.main(["--config", "llama3_debug_muon", "--training.steps", "4", "--metrics.log_freq", "2",
                         "--training.seq_len", "32", "--training.local_batch_size", "2",
                         "--metrics.save_jsonl", str(out)])
    assert len(losses) == 2 and all(math.isfinite(v) for v in losses)
    with open(out / "optimizer_metrics.jsonl") as fh:
        recs = [json.loads(l) for l in fh]
    assert [r["step"] for r in recs] == [2, 4] and recs[0]["opt_0/type"] == "Muon"


def test_dcp_checkpoint_roundtrip(tmp_path):
    from dion_b200 import train

    ck = tmp_path / "ck"
    args = ["--config", "llama3_debug_dion", "--training.seq_len", "32", "--training.local_batch_size", "2",
            "--checkpoint.enable", "--checkpoint.folder", str(ck), "--checkpoint.interval", "2",
            "--checkpoint.no-last_save_model_only"]
    train.main(args + ["--training.steps", "2"])
    assert (ck / "step-2").exists()
    # resume: continues from step 2 to 4
    losses = train.main(args + ["--training.steps", "4", "--metrics.log_freq", "1"])
    assert len(losses) == 2
    assert (ck / "step-4").exists()


def test_resume_after_model_only_final_save(tmp_path):
    """Interval saves, then the final model-only export: a longer rerun
    resumes from the last full checkpoint (optimizer state and step), not
    from the model-only export; a final step on the interval still gets its
    full checkpoint."""
    from dion_b200 import train
    from dion_b200.checkpoint import CheckpointManager

    ck = tmp_path / "ck"
    args = ["--config", "llama3_debug_dion", "--training.seq_len", "32", "--training.local_batch_size", "2",
            "--checkpoint.enable", "--checkpoint.folder", str(ck), "--checkpoint.interval", "2",
            "--checkpoint.last_save_model_only"]
    train.main(args + ["--training.steps", "3"])
    assert (ck / "step-2").exists() and (ck / "step-3-model").exists() and not (ck / "step-3").exists()
    assert CheckpointManager(str(ck), None, None).latest() == str(ck / "step-2")
    losses = train.main(args + ["--training.steps", "4", "--metrics.log_freq", "1"])
    assert len(losses) == 2  # steps 3 and 4 only: resumed at step 2
    assert (ck / "step-4").exists() and (ck / "step-4-model").exists()


@pytest.mark.parametrize("mode,option", [("full", "1"), ("selective", "op"), ("selective", "2")])
def test_activation_checkpointing_matches(mode, option):
    """Checkpointed blocks give the same loss and gradients as plain ones."""
    from dion_b200.models.llama3 import Transformer, llama3_config

    torch.manual_seed(0)
    cfg = llama3_config("tiny", n_layers=3, vocab_size=256, max_seq_len=32)
    a = Transformer(cfg)
    a.init_weights("normal", generator=torch.Generator().manual_seed(1))
    b = Transformer(cfg)
    b.load_state_dict(a.state_dict())
    b.set_activation_checkpointing(mode, option)
    tok = torch.randint(0, 256, (2, 16))
    lab = torch.randint(0, 256, (2, 16))
    la = a(tok, labels=lab)
    la.backward()
    lb = b(tok, labels=lab)
    lb.backward()
    assert torch.allclose(la, lb, atol=1e-6)
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.allclose(pa.grad, pb.grad, atol=1e-5, rtol=1e-4), n
    assert [n for n, _ in a.named_parameters()] == [n for n, _ in b.named_parameters()]


def test_registry_8b_configs_use_selective_ac():
    from dion_b200.integration.config_registry import get_config

    for name in ("llama3_8b_dion", "llama3_8b_adadion_v2", "llama3_8b_dion2_fsdp_tp"):
        c = get_config(name)
        assert c.activation_checkpoint.mode == "selective" and c.training.seq_len == 8192
    c = get_config("llama3_8b_dion2_fsdp_tp")
    assert c.parallelism.tensor_parallel_degree == 2 and c.parallelism.data_parallel_shard_degree == 4


def test_launch_scripts_are_valid_bash():
    import glob
    import subprocess

    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "dion_b200", "launch")
    files = glob.glob(os.path.join(root, "*.sh")) + glob.glob(os.path.join(root, "slurm", "*"))
    assert len(files) >= 8
    for f in files:
        r = subprocess.run(["bash", "-n", f], capture_output=True, text=True)
        assert r.returncode == 0, (f, r.stderr)
        with open(f) as fh:
            text = fh.read()
        assert "torchtitan" not in text
    with open(os.path.join(root, "run_single_node.sh")) as fh:
        single = fh.read()
    assert "-m dion_b200.train" in single and "--parallelism.data_parallel_shard_degree" in single


def test_train_module_flag():
    from dion_b200.train import _load_config

    a = _load_config(None, "llama3_debug_dion")
    b = _load_config("ada_dion.integration.config_registry", "llama3_debug_dion")
    c = _load_config("dion_b200.integration.config_registry", "llama3_debug_dion")
    assert a.optimizer.name == b.optimizer.name == c.optimizer.name == "Dion"


def test_checkpoint_load_model_only_and_full(tmp_path):
    """A model-only checkpoint loads into a job with optimizers (step 0,
    optimizer untouched); a full one restores the optimizer and step; an
    optimizer state that does not fit the checkpoint raises instead of being
    skipped."""
    from dion_b200 import checkpoint as ckpt

    torch.manual_seed(0)
    m = _MockLlama()
    cfg = HybridOptimizersContainer.Config(name="Muon", lr=0.01)
    c = HybridOptimizersContainer(cfg, model_parts=[m])
    x = torch.randint(0, 64, (3,))
    out = m.output(m.layers["0"].attention.wq(m.tok_embeddings(x)))
    (out.sum() + sum(p.sum() for p in m.parameters())).backward()  # every parameter gets a gradient
    c.step()
    ckpt.save(str(tmp_path), m, c, step=3, model_only=True)
    ckpt.save(str(tmp_path), m, c, step=5)
    m2 = _MockLlama()
    c2 = HybridOptimizersContainer(cfg, model_parts=[m2])
    assert ckpt.load(str(tmp_path / "step-3-model"), m2, c2) == 0
    assert all(torch.equal(a, b) for a, b in zip(m.state_dict().values(), m2.state_dict().values()))
    assert ckpt.load(str(tmp_path / "step-5"), m2, c2) == 5
    mom = [v for k, v in c2.state_dict().items() if k.endswith("momentum_buffer") or k.endswith("momentum")]
    assert mom and any(float(t.abs().sum()) > 0 for t in mom)
    c3 = HybridOptimizersContainer(HybridOptimizersContainer.Config(name="AdamW", lr=0.01), model_parts=[_MockLlama()])
    from torch.distributed.checkpoint.api import CheckpointException  # a BaseException subclass

    with pytest.raises((CheckpointException, RuntimeError, KeyError)):
        ckpt.load(str(tmp_path / "step-5"), _MockLlama(), c3)


def _reshard_body(folder, phase, optimizer, rank, world, async_mode="disabled"):
    """phase "save": FSDP over `world` ranks, 2 steps, checkpoint, then 2 more
    steps; phase "load": resume the checkpoint and take the same 2 steps."""
    import torch.distributed as dist

    from dion_b200.checkpoint import CheckpointManager
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=4 // world, steps=4, warmup_steps=0, dp_shard=world,
                        optimizer=HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3), seed=5)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    ck = CheckpointManager(folder, tr.model, tr.optimizers, interval=2, model_only_last=False, async_mode=async_mode)
    if phase == "save":
        for s in (1, 2):
            tr.train_step(*tr.data.next())
            ck.maybe_save(tr, s)
    else:
        ck.maybe_load(tr)
        assert tr.step_idx == 2
    losses = []
    for _ in range(2):
        loss = tr.train_step(*tr.data.next()).detach().clone()
        if world > 1:  # mean over the data-parallel ranks = the global batch's loss
            dist.all_reduce(loss)
            loss /= world
        losses.append(float(loss))
    ck.wait()
    return losses


# Dion2 under FSDP selects rows per shard, so its update depends on the world
# size by definition: its checkpoint is resumed at the same size.
@pytest.mark.parametrize("optimizer,load_world", [("Dion", 1), ("Muon", 1), ("AdaDionV2", 1), ("Dion2", 2),
                                                  ("AdaDion", 2)])
def test_fsdp_checkpoint_reshards_across_world_sizes(tmp_path, optimizer, load_world):
    """A checkpoint (matrix optimizer + AdamW) written by 2 FSDP ranks (gloo)
    resumes on ``load_world`` ranks: the same global batches give the losses
    the uninterrupted 2-rank run reached (AdaDionV2 in adaptive-rank mode,
    whose local state is checkpointed as DTensors)."""
    import functools

    from test_distributed_cpu import spawn

    folder = str(tmp_path / "ck")
    saved = spawn(functools.partial(_reshard_body, folder, "save", optimizer), world=2)
    for r, (status, res) in saved.items():
        assert status == "ok", res
    loaded = spawn(functools.partial(_reshard_body, folder, "load", optimizer), world=load_world)
    assert loaded[0][0] == "ok", loaded[0][1]
    a, b = torch.tensor(saved[0][1]), torch.tensor(loaded[0][1])
    assert torch.allclose(a, b, rtol=1e-4, atol=1e-4), (a, b)


def test_train_entry_writes_profiler_traces(tmp_path):
    """--profiling.enable_profiling records one step every profile_freq steps
    as a Chrome trace per rank (torchtitan's folder layout), which the trace
    parser reads."""
    from dion_b200 import train
    from dion_b200.benchmarks.tiers import parse_profiler_trace

    folder = tmp_path / "traces"
    train.main(["--config", "llama3_debug_muon", "--training.steps", "4", "--training.seq_len", "32",
                "--training.local_batch_size", "2", "--profiling.enable_profiling", "--profiling.profile_freq", "2",
                "--profiling.save_traces_folder", str(folder)])
    got = sorted(p.name for p in folder.iterdir())
    assert got == ["iteration_2", "iteration_4"], got
    res = parse_profiler_trace(str(folder / "iteration_4" / "rank0_trace.json"))
    assert isinstance(res, dict) and res


def _accum_body(local, global_batch, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=local, global_batch_size=global_batch, steps=3, warmup_steps=0,
                        dp_shard=world, optimizer=HybridOptimizersContainer.Config(name="Muon", lr=0.02), seed=3)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    assert tr.grad_accum == global_batch // (local * world)
    out = []
    for _ in range(3):
        loss = tr.train_step(*tr.data.next()).detach().clone()
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(loss)
            loss /= world
        out.append(float(loss))
    return out


@pytest.mark.parametrize("world", [1, 2])
def test_gradient_accumulation_matches_full_batch(world):
    """global_batch_size = 2 x local x data-parallel degree accumulates two
    micro-batches per step and trains like one step on the whole batch."""
    import functools

    from test_distributed_cpu import spawn

    full = spawn(functools.partial(_accum_body, 4 // world, 4), world=world)
    acc = spawn(functools.partial(_accum_body, 2 // world, 4), world=world)
    for out in (full, acc):
        for r, (status, res) in out.items():
            assert status == "ok", res
    a, b = torch.tensor(full[0][1]), torch.tensor(acc[0][1])
    assert torch.allclose(a, b, rtol=1e-4, atol=1e-4), (a, b)


def test_global_batch_must_divide():
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    with pytest.raises(ValueError, match="multiple"):
        Trainer(TrainerConfig(model="tiny", seq_len=16, local_batch_size=3, global_batch_size=4, steps=1),
                device=torch.device("cpu"))


def test_debug_seed_and_global_batch_flags():
    """The reference's command lines use --debug.seed and
    --training.global-batch-size; both map onto the trainer."""
    from dion_b200.integration.config_registry import get_config
    from dion_b200.train import trainer_config_from_job

    job = get_config("llama3_debug_muon")
    assert apply_overrides(job, ["--debug.seed", "42", "--training.global-batch-size", "64"]) == []
    tc = trainer_config_from_job(job)
    assert tc.seed == 42 and tc.global_batch_size == 64


def test_train_entry_tensorboard(tmp_path):
    """--metrics.enable_tensorboard writes the step metrics as TensorBoard events."""
    pytest.importorskip("tensorboard")
    from dion_b200 import train

    tb = tmp_path / "tb"
    train.main(["--config", "llama3_debug_muon", "--training.steps", "2", "--training.seq_len", "32",
                "--training.local_batch_size", "2", "--metrics.log_freq", "1", "--metrics.enable_tensorboard",
                "--metrics.save_tb_folder", str(tb)])
    events = [p for p in tb.iterdir() if p.name.startswith("events.out.tfevents")]
    assert events and events[0].stat().st_size > 0
    from tensorboard.backend.event_processing.event_accumulator import EventAccumulator

    acc = EventAccumulator(str(tb))
    acc.Reload()
    assert "optimizer/loss" in acc.Tags()["scalars"]
    assert [e.step for e in acc.Scalars("optimizer/loss")] == [1, 2]


@pytest.mark.parametrize("experiment,count", [("perf", 5), ("convergence", 15), ("dion2", 3), ("adadion", 48),
                                              ("anchor", 6), ("sdion", 8)])
def test_experiment_launcher_runs_parse(experiment, count):
    """Every run the experiment launcher would start names a registered
    config and only overrides that the CLI accepts."""
    import shlex
    import subprocess

    script = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "dion_b200", "launch",
                          "run_experiments.sh")
    env = dict(os.environ, DRY_RUN="1", VAL_DATA="val.bin", TRAIN_DATA="train/")
    out = subprocess.run(["bash", script, experiment], capture_output=True, text=True, env=env, check=True).stdout
    runs = [l for l in out.splitlines() if l.startswith("DRY_RUN")]
    assert len(runs) == count
    for line in runs:
        head, _, args = line.partition(" args=")
        fields = dict(kv.split("=", 1) for kv in head.split()[1:])
        job = get_config(f"llama3_{fields['model']}_{fields['optimizer']}")
        assert apply_overrides(job, shlex.split(args)) == [], line


def _variant_body(name, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=2, steps=3, warmup_steps=0, dp_shard=world,
                        optimizer=HybridOptimizersContainer.Config(name=name, lr=0.02, init_rank=8, rank_min=4,
                                                                   rank_max=32, warmup_rank=16), seed=1)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    assert type(tr.optimizers.optimizers[0]).__name__ == {"AdaDionAnchor": "AdaDion"}.get(name, name)
    return [float(tr.train_step(*tr.data.next())) for _ in range(3)]


def _variants_body(rank, world):
    out = []
    for name in ["AdaDionAnchor", "SDion", "GSDion", "AGDion", "QCDion"]:
        out.extend(_variant_body(name, rank, world))
    return out


def test_container_trains_research_variants():
    """The research variants are selectable by name (--optimizer.name) and
    train under FSDP over 2 ranks (one pair of processes runs all five)."""
    from test_distributed_cpu import spawn

    out = spawn(_variants_body, world=2)
    for r, (status, res) in out.items():
        assert status == "ok", res
        assert len(res) == 15 and all(math.isfinite(v) for v in res)


def test_fp32_mixed_precision_flag():
    """--training.mixed_precision_param float32 trains with fp32 compute (the
    gathered parameters stay fp32) and gives a loss close to the bf16 run's."""
    from dion_b200 import train

    base = ["--config", "llama3_debug_muon", "--training.steps", "2", "--training.seq_len", "32",
            "--training.local_batch_size", "2", "--metrics.log_freq", "1"]
    bf16 = train.main(base)
    fp32 = train.main(base + ["--training.mixed_precision_param", "float32"])
    assert all(math.isfinite(v) for v in fp32) and abs(bf16[0] - fp32[0]) < 0.05, (bf16, fp32)


def test_reference_command_lines_parse():
    """The flags the reference's experiment scripts pass to torchtitan parse
    here as they are (hyphenated sections and fields, --compile.*,
    --hf-assets-path, the GSDion / Dion2 / SDion switches)."""
    from dion_b200.train import parse_job, trainer_config_from_job

    argv = ("--module ada_dion.integration.config_registry --config llama3_320m_adadion --training.steps 2000 "
            "--training.local-batch-size 32 --training.global-batch-size 256 --training.seq-len 2048 "
            "--hf-assets-path ./assets/hf/Meta-Llama-3.1-8B --optimizer.lr 0.02 --optimizer.init-rank 64 "
            "--optimizer.no-use-anchor --parallelism.data-parallel-shard-degree 8 "
            "--parallelism.data-parallel-replicate-degree 1 --parallelism.tensor_parallel_degree 1 --compile.enable "
            "--activation-checkpoint.mode selective --activation-checkpoint.selective-ac-option op "
            "--metrics.enable-wandb --metrics.enable-tensorboard --metrics.log-freq 10 --metrics.wandb_project p "
            "--metrics.wandb_run_name r --debug.seed 42 --validator.freq 200 --validator.steps 50 "
            "--profiling.enable_profiling --profiling.save_traces_folder t --optimizer.selection_method random "
            "--optimizer.no-use-adaptive-scalar --optimizer.no-rank-normalize --optimizer.use-rms-matching "
            "--optimizer.no-use-trust-region --optimizer.no-use-residual-rank --optimizer.sdion-mode skip "
            "--optimizer.no-adaptive-rank --optimizer.anchor-alpha 0.1 --optimizer.fraction 0.25 "
            "--optimizer.rank_fraction 0.25 --optimizer.mu 0.95").split()
    job = parse_job(argv)
    assert job.compile.enable and job.hf_assets_path.endswith("Meta-Llama-3.1-8B")
    assert job.activation_checkpoint.mode == "selective" and job.metrics.wandb_project == "p"
    o = job.optimizer
    assert (o.use_anchor, o.adaptive_rank, o.use_adaptive_scalar, o.rank_normalize, o.use_trust_region) == (
        False, False, False, False, False)
    assert o.use_rms_matching and o.selection_method == "random" and o.sdion_mode == "skip"
    tc = trainer_config_from_job(job)
    assert tc.seed == 42 and tc.global_batch_size == 256 and tc.local_batch_size == 32


def test_checkpoint_initial_load_and_load_step(tmp_path):
    """--checkpoint.initial_load_path starts a new run from another run's
    model-only export (weights only, step 0); --checkpoint.load_step resumes
    from a chosen full checkpoint rather than the newest."""
    from dion_b200 import train

    base = ["--config", "llama3_debug_muon", "--training.seq_len", "32", "--training.local_batch_size", "2",
            "--metrics.log_freq", "1", "--checkpoint.enable"]
    a = tmp_path / "a"
    train.main(base + ["--checkpoint.folder", str(a), "--checkpoint.interval", "2", "--training.steps", "4",
                       "--checkpoint.last_save_model_only"])
    assert (a / "step-2").exists() and (a / "step-4").exists() and (a / "step-4-model").exists()
    # a new run from the model-only export: starts at step 0 with run A's final weights
    b = tmp_path / "b"
    losses = train.main(base + ["--checkpoint.folder", str(b), "--checkpoint.interval", "100",
                                "--checkpoint.initial_load_path", str(a / "step-4-model"), "--training.steps", "2"])
    assert len(losses) == 2
    # resume run A from step 2 (not the newest, step 4): 2 more steps are logged
    losses = train.main(base + ["--checkpoint.folder", str(a), "--checkpoint.interval", "100",
                                "--checkpoint.load_step", "2", "--training.steps", "4"])
    assert len(losses) == 2
    with pytest.raises(FileNotFoundError):
        train.main(base + ["--checkpoint.folder", str(a), "--checkpoint.load_step", "3", "--training.steps", "4"])


def test_lr_schedule_shapes():
    """Warm-up, then cosine decay over the rest by default; with decay_ratio
    a stable phase first (warmup-stable-decay), and linear / sqrt shapes."""
    from dion_b200.integration.trainer import lr_lambda

    total, warm = 100, 10
    assert lr_lambda(0, warm, total, 0.1) == pytest.approx(1 / 11)
    assert lr_lambda(warm, warm, total, 0.1) == pytest.approx(1.0)
    assert lr_lambda(total, warm, total, 0.1) == pytest.approx(0.1)
    assert lr_lambda(55, warm, total, 0.1) == pytest.approx(0.1 + 0.9 * 0.5)  # cosine midpoint
    # WSD: flat until the last 20 steps, then linear / sqrt down to the floor
    assert lr_lambda(79, warm, total, 0.0, 0.2, "linear") == 1.0
    assert lr_lambda(90, warm, total, 0.0, 0.2, "linear") == pytest.approx(0.5)
    assert lr_lambda(90, warm, total, 0.0, 0.2, "sqrt") == pytest.approx(1 - 0.5 ** 0.5)
    with pytest.raises(ValueError):
        lr_lambda(90, warm, total, 0.0, 0.2, "step")
    from dion_b200.integration.config_registry import get_config
    from dion_b200.train import trainer_config_from_job

    job = get_config("llama3_debug_muon")
    apply_overrides(job, ["--lr_scheduler.decay_ratio", "0.2", "--lr_scheduler.decay_type", "linear"])
    tc = trainer_config_from_job(job)
    assert tc.decay_ratio == 0.2 and tc.decay_type == "linear"


def test_train_entry_wandb_offline_without_credentials(tmp_path, monkeypatch):
    """The registry's full-size configs enable W&B, as the reference's do;
    without credentials the run is recorded offline instead of waiting on the
    network."""
    pytest.importorskip("wandb")
    from dion_b200 import train

    monkeypatch.chdir(tmp_path)
    monkeypatch.delenv("WANDB_API_KEY", raising=False)
    monkeypatch.delenv("WANDB_MODE", raising=False)
    monkeypatch.setenv("WANDB_DIR", str(tmp_path))
    losses = train.main(["--config", "llama3_debug_muon", "--training.steps", "2", "--training.seq_len", "32",
                         "--training.local_batch_size", "2", "--metrics.log_freq", "1", "--metrics.enable_wandb",
                         "--metrics.wandb_project", "p", "--metrics.wandb_run_name", "r"])
    assert len(losses) == 2
    runs = list((tmp_path / "wandb").glob("offline-run-*"))
    assert runs, list(tmp_path.rglob("*"))[:20]


def test_reference_adadion_v2_configs():
    """The reference's AdaDionV2 trainer configs by name, with its
    hyper-parameters; the Dion-equivalent one sizes Q by rank_fraction, and
    output_head_lr_scaling=False keeps the LM head at scalar_lr."""
    for n in ["llama3_320m_adadion_v2", "llama3_320m_adadion_v2_dion_lr", "llama3_320m_adadion_v2_dion_equivalent",
              "llama3_debug_2gpu_adadion_v2"]:
        assert n in REGISTRY
    c = get_config("llama3_320m_adadion_v2")
    o = c.optimizer
    assert (o.lr, o.rank_fraction_max, o.init_rank_fraction, o.erank_ema_beta, o.rank_scale) == (0.012, 0.7, 0.5, 0.5,
                                                                                                  1.5)
    assert c.lr_scheduler.warmup_steps == 610 and c.lr_scheduler.min_lr_factor == 0.0
    assert c.activation_checkpoint.selective_ac_option == "2"
    d = get_config("llama3_debug_2gpu_adadion_v2")
    assert d.training.steps == 50 and d.training.local_batch_size == 4 and d.optimizer.rank_min == 8

    model = Transformer(llama3_config("debug"))
    eq = get_config("llama3_320m_adadion_v2_dion_equivalent").optimizer
    cont = HybridOptimizersContainer(eq, model_parts=[model])
    opt = cont.optimizers[0]
    assert type(opt).__name__ == "AdaDionV2" and not opt._adaptive_rank
    heads = [g for g in opt.param_groups if any(p is model.output.weight for p in g["params"])]
    assert heads and heads[0]["lr"] == eq.scalar_lr


def test_list_fields(capsys):
    from dion_b200 import train

    with pytest.raises(SystemExit):
        train.main(["--list-fields", "--config", "llama3_160m_dion"])
    out = capsys.readouterr().out
    assert "--optimizer.rank_fraction 0.25" in out and "--training.steps 10000" in out


def test_async_checkpoint_resume(tmp_path):
    """--checkpoint.async_mode async writes in the background; the resumed run
    continues exactly like one resumed from a synchronous checkpoint."""
    from dion_b200 import train

    base = ["--config", "llama3_debug_dion", "--training.seq_len", "32", "--training.local_batch_size", "2",
            "--metrics.log_freq", "1", "--checkpoint.enable", "--checkpoint.interval", "2",
            "--checkpoint.no-last_save_model_only"]
    out = {}
    for mode in ("disabled", "async"):
        ck = tmp_path / mode
        train.main(base + ["--checkpoint.folder", str(ck), "--checkpoint.async_mode", mode, "--training.steps", "2"])
        assert (ck / "step-2" / ".metadata").exists()
        out[mode] = train.main(base + ["--checkpoint.folder", str(ck), "--checkpoint.async_mode", mode,
                                       "--training.steps", "4"])
    assert out["disabled"] == out["async"] and len(out["async"]) == 2


def test_async_checkpoint_two_ranks(tmp_path):
    """Background checkpoint writes under FSDP over 2 ranks (on a group of
    their own) overlap the next steps and resume like synchronous ones."""
    import functools

    from test_distributed_cpu import spawn

    folder = str(tmp_path / "ck")
    saved = spawn(functools.partial(_reshard_body, folder, "save", "Dion", async_mode="async"), world=2)
    for r, (status, res) in saved.items():
        assert status == "ok", res
    loaded = spawn(functools.partial(_reshard_body, folder, "load", "Dion"), world=2)
    for r, (status, res) in loaded.items():
        assert status == "ok", res
    assert torch.allclose(torch.tensor(saved[0][1]), torch.tensor(loaded[0][1]), rtol=1e-4, atol=1e-4)


def test_model_only_export_dtype(tmp_path):
    """--checkpoint.export_dtype bfloat16 writes the final model-only export
    in bf16 (full checkpoints keep fp32), and it loads into an fp32 model."""
    import torch.distributed.checkpoint as dcp

    from dion_b200 import train

    ck = tmp_path / "ck"
    train.main(["--config", "llama3_debug_muon", "--training.steps", "2", "--training.seq_len", "32",
                "--training.local_batch_size", "2", "--metrics.log_freq", "1", "--checkpoint.enable",
                "--checkpoint.folder", str(ck), "--checkpoint.interval", "2", "--checkpoint.last_save_model_only",
                "--checkpoint.export_dtype", "bfloat16"])
    md = dcp.FileSystemReader(str(ck / "step-2-model")).read_metadata().state_dict_metadata
    full = dcp.FileSystemReader(str(ck / "step-2")).read_metadata().state_dict_metadata
    key = "model.output.weight"
    assert md[key].properties.dtype == torch.bfloat16 and full[key].properties.dtype == torch.float32
    from dion_b200.checkpoint import load

    m = Transformer(llama3_config("debug"))
    assert load(str(ck / "step-2-model"), m) == 0 and m.output.weight.dtype == torch.float32
