"""Sweep generator, tier A/C generators and the profiler-trace parser (CPU)."""
import json

from dion_b200.benchmarks import sweep, tiers


def test_sweep_grid_has_33_runs():
    cfgs = sweep.generate_sweep_configs(steps=100, num_gpus=8)
    assert len(cfgs) == 33
    assert len({c.name for c in cfgs}) == 33
    by_opt = {}
    for c in cfgs:
        by_opt[c.optimizer] = by_opt.get(c.optimizer, 0) + 1
    assert by_opt == {"adamw": 3, "muon": 3, "dion": 9, "dion2": 9, "adadion": 9}


def test_sweep_cli_parses_with_trainer_overrides():
    from dion_b200.integration import config as C
    from dion_b200.integration.config_registry import get_config

    c = [x for x in sweep.generate_sweep_configs(10, 8) if x.optimizer == "dion"][4]
    cli = sweep.sweep_config_to_cli(c)
    assert "-m dion_b200.train" in cli and "--config llama3_160m_dion" in cli
    job = get_config(c.config_fn)
    args = []
    for k, v in c.overrides.items():
        args += [f"--{k}", str(v)]
    C.apply_overrides(job, args)
    assert job.training.steps == 10
    assert abs(job.optimizer.lr - 0.02) < 1e-12 and abs(job.optimizer.rank_fraction - 0.25) < 1e-12


def test_sweep_script(tmp_path):
    s = sweep.generate_sweep_shell_script(10, 8)
    assert s.startswith("#!/usr/bin/env bash") and s.count("-m dion_b200.train") == 33


def test_tier_a_all_pass_cpu():
    res = tiers.run_tier_a("cpu")
    assert set(res) >= {"muon", "dion", "dion2", "adadion", "adadion_v2"}
    assert all(v["pass"] for v in res.values()), res


def test_tier_c_generators():
    c1 = tiers.generate_c1_fsdp_experiments()
    c2 = tiers.generate_c2_hsdp_experiments()
    assert len(c1) == 15 and len(c2) == 10
    cli = tiers.experiment_to_cli(c2[0])
    assert "--rdzv-backend=c10d" in cli and "--parallelism.data_parallel_replicate_degree 2" in cli
    cli1 = tiers.experiment_to_cli(c1[0])
    assert "--master-addr 127.0.0.1" in cli1


def test_trace_parser(tmp_path):
    ev = [{"name": "ncclDevKernel_AllGather_RING_LL", "dur": 100},
          {"name": "ncclDevKernel_ReduceScatter_Sum_bf16", "dur": 250},
          {"name": "ncclKernel_AllReduce", "dur": 50},
          {"name": "void bdion::gemm_kernel<...>", "dur": 400},
          {"name": "nvjet_tst_128x256", "dur": 300},
          {"name": "elementwise", "dur": 7}]
    p = tmp_path / "t.json"
    p.write_text(json.dumps({"traceEvents": ev}))
    r = tiers.parse_profiler_trace(str(p))
    assert r["nccl_allgather_count"] == 1 and abs(r["nccl_allgather_ms"] - 0.1) < 1e-9
    assert abs(r["nccl_reducescatter_ms"] - 0.25) < 1e-9 and abs(r["nccl_total_ms"] - 0.4) < 1e-9
    assert r["dion_b200_kernels_count"] == 1 and abs(r["library_kernels_ms"] - 0.3) < 1e-9
