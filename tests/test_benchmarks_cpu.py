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


def test_plots_write_svg(tmp_path):
    from dion_b200.benchmarks import plots

    runs = {"dion": {"tokens": [0, 1, 2], "val_loss": [3.0, 2.5, 2.2], "step": [1, 2, 3],
                     "tokens_per_sec": [10.0, 11.0, 12.0], "num_gpus": [1, 2, 4], "fwd_ms": 5.0, "bwd_ms": 9.0,
                     "opt_ms": 2.0, "nccl_ms": 1.0, "allreduce_bytes": 2**20, "allgather_bytes": 0,
                     "reducescatter_bytes": 2**21, "allreduce_ms": 0.1, "allgather_ms": 0.2,
                     "reducescatter_ms": 0.3, "comm_compute_ratio": [0.1, 0.2, 0.3]},
            "muon": {"tokens": [0, 1, 2], "val_loss": [3.0, 2.6, 2.4], "step": [1, 2, 3],
                     "tokens_per_sec": [9.0, 9.5, 9.0], "num_gpus": [1, 2, 4], "fwd_ms": 5.0, "bwd_ms": 9.0,
                     "opt_ms": 3.0, "nccl_ms": 2.0, "allreduce_bytes": 0, "allgather_bytes": 2**20,
                     "reducescatter_bytes": 2**20, "allreduce_ms": 0.0, "allgather_ms": 0.3,
                     "reducescatter_ms": 0.3, "comm_compute_ratio": [0.2, 0.3, 0.5]}}
    runs["dion"]["tokens_per_sec"] = [10.0, 19.0, 37.0]
    runs["muon"]["tokens_per_sec"] = [9.0, 17.0, 30.0]
    dd = {"step": [1, 2, 3], "rank_mean": [64, 64, 60], "residual_norm_mean": [1.0, 0.9, 0.8]}
    d2 = {"step": [1, 2], "alpha": [0.25], "sparsity": [0.75, 0.75], "selected_frac_mean": [0.25, 0.25]}
    ad = {"step": [1, 2], "rank_mean": [32, 40], "aerr_mean": [0.1, 0.08]}
    out = plots.save_all_plots(str(tmp_path), runs=runs, dion_data=dd, dion2_data=d2, adadion_data=ad)
    assert len(out) == 10
    for p in out:
        with open(p) as fh:
            s = fh.read()
        assert s.startswith("<svg") and s.rstrip().endswith("</svg>")


def test_logparse(tmp_path):
    from dion_b200.benchmarks import logparse

    log = tmp_path / "llama3_160m_dion.log"
    lines = ["Optimizer: Dion"]
    for s in (10, 20, 20, 30):
        lines.append(f"[titan] 2026-01-01 00:00:{s:02d},000 - INFO - step: {s:5d}  loss: {5 - s / 10:8.4f}  "
                     f"grad_norm:  1.2500  memory: 12.50GiB  tps: 1,234  tflops: 56.78  mfu: 12.34%")
    log.write_text("\n".join(lines))
    d = logparse.parse_log(str(log))
    assert d["optimizer"] == "dion" and d["step"] == [10, 20, 30]
    assert d["tps"] == [1234.0] * 3 and d["mfu"][0] == 12.34 and d["time_s"] == [0.0, 10.0, 20.0]
    ours = tmp_path / "muon_run.log"
    ours.write_text("step:    10  loss:   7.1234  grad_norm:  0.5000  memory:  3.00GiB  tps: 98,765  "
                    "tflops: 400.50  mfu: 20.00%\nvalidate step:    10  loss:   7.5000\n"
                    "validate step:    15  loss:   7.2500\n")
    mine = logparse.parse_log(str(ours))
    assert mine["step"] == [10] and mine["val_step"] == [10, 15] and mine["val_loss"] == [7.5, 7.25]
    out = logparse.generate_plots([str(log), str(ours)], str(tmp_path / "plots"), tokens_per_step=4096)
    assert any(p.endswith(".svg") for p in out)
    with open(out[-1]) as fh:
        assert "| muon_run | muon | 10 | 7.1234 | 98,765 |" in fh.read()


def test_optimizer_phases_show_in_profiler_trace(tmp_path):
    """Optimizer phases are record_function events when a profiler runs, and
    the trace parser reads the exported Chrome trace."""
    import torch
    from dion_b200.optim import Dion, Muon

    ps = [torch.nn.Parameter(torch.randn(16, 8)) for _ in range(2)]
    opts = [Muon(ps, lr=0.01), Dion([torch.nn.Parameter(torch.randn(16, 8))], lr=0.01)]
    for o in opts:
        for g in o.param_groups:
            for p in g["params"]:
                p.grad = torch.randn_like(p)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        for o in opts:
            o.step()
    names = {e.name for e in prof.events()}
    assert any(n.startswith("muon/local/") for n in names)
    assert any(n.startswith("dion/replicated/") for n in names)
    path = tmp_path / "trace.json"
    prof.export_chrome_trace(str(path))
    r = tiers.parse_profiler_trace(str(path))
    assert r["nccl_total_ms"] == 0.0


def test_cifar10_benchmark_runs(tmp_path):
    from dion_b200.benchmarks import cifar10

    logs = cifar10.main(["--epochs", "1", "--batch-size", "32", "--train-size", "256", "--optimizers",
                         "muon,dion_r03", "--log-freq", "2", "--outdir", str(tmp_path), "--data-dir",
                         str(tmp_path / "none")])
    assert set(logs) == {"muon", "dion_r03"}
    for l in logs.values():
        assert l["eval/val_acc"] and all(v == v for v in l["train_loss"])
    assert (tmp_path / "results.json").exists() and (tmp_path / "cifar10.svg").exists()


def test_optimizer_bench_cli_cases(capsys):
    """Every optimizer case parses; the reference arm of Dion2 reports that
    the reference environment has no Dion2 instead of failing."""
    import json

    from dion_b200.benchmarks import optimizer_bench as ob

    for name in ("muon", "dion", "dion2", "adadion_v2"):
        assert ob.parse(["--optimizer", name]).optimizer == name
    ob.main(["--optimizer", "dion2", "--impl", "reference"])
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def test_report_from_run_outputs(tmp_path):
    """The measured report is built from parity JSON, bench and optimizer-bench lines."""
    import json

    from dion_b200.benchmarks import report

    par = tmp_path / "p.json"
    par.write_text(json.dumps({"config": {"preset": "tiny", "optimizer": "dion"},
                               "ours": {"losses": [3.0, 2.5, 2.0], "seconds": 1.0},
                               "reference": {"losses": [3.0, 2.6, 2.1], "seconds": 2.0},
                               "comparison": {"final_ours": 2.0, "final_ref": 2.1, "mean_abs_diff": 0.07,
                                              "tail_rel_diff": 0.05}}))
    bench = tmp_path / "b.log"
    bench.write_text("noise\n" + json.dumps({"metric": "m", "value": 100.0, "n_gpus": 1, "impl": "ours",
                                             "config": {"model": "llama3-1B", "optimizer": "muon+adamw"},
                                             "e2e": {"value": 99.0}}) + "\n" +
                     json.dumps({"metric": "m", "value": 80.0, "n_gpus": 1, "impl": "reference",
                                 "config": {"model": "llama3-1B", "optimizer": "muon+adamw"}}) + "\n")
    ob = tmp_path / "o.log"
    ob.write_text(json.dumps({"metric": "optimizer_step_ms", "optimizer": "dion", "impl": "ours", "n_gpus": 2,
                              "ms": 50.0, "p2p": True, "matrices": "m"}) + "\n")
    data = report.collect([str(par)], [str(bench)], [str(ob)])
    assert len(data["parity"]) == 1 and len(data["bench"]) == 2 and len(data["optimizer"]) == 1
    out = report.render(data, str(tmp_path / "rep"))
    text = open(out).read()
    assert "tiny dion" in text and "| ours | 1 |" in text and "| dion | ours | 2 |" in text
    assert (tmp_path / "rep" / "loss_0.svg").exists() and (tmp_path / "rep" / "throughput.svg").exists()
    # regenerating from the saved data gives the same report
    report.main(["--data", str(tmp_path / "rep" / "data.json"), "--out", str(tmp_path / "rep2")])
    assert open(tmp_path / "rep2" / "report.md").read() == text


def test_step_trace_summary():
    """Device time by owner and idle gaps from a chrome trace."""
    from dion_b200.benchmarks.step_trace import summarize

    ev = [{"cat": "kernel", "name": "nvjet_tst_256x256", "ts": 0, "dur": 100},
          {"cat": "kernel", "name": "void bdion::gemm_tc2_kernel<...>", "ts": 150, "dur": 50},
          {"cat": "kernel", "name": "cudnn_generated_fort_native_sdpa", "ts": 180, "dur": 40},
          {"cat": "cpu_op", "name": "aten::mm", "ts": 0, "dur": 5}]
    s = summarize({"traceEvents": ev})
    assert s["kernels"] == 3
    assert abs(s["span_ms"] - 0.22) < 1e-9 and abs(s["idle_ms"] - 0.05) < 1e-9
    assert s["by_owner_ms"] == {"cuBLAS": 0.1, "dion_b200": 0.05, "cuDNN": 0.04}


def test_layout_check_reports_each_combination():
    """The layout checker trains an optimizer on a 2-rank layout (gloo) and
    reports combinations an optimizer declines as unsupported."""
    from dion_b200.benchmarks import layout_check

    rows = [layout_check.check("Muon", (1, 2, 1, 1), steps=2), layout_check.check("SDion", (1, 1, 2, 1), steps=2)]
    got = {(r["layout"], r["optimizer"]): r["status"] for r in rows}
    assert got == {("1x2x1x1", "Muon"): "ok", ("1x1x2x1", "SDion"): "unsupported"}, got
    assert all(len(r["losses"]) == 2 for r in rows if r["status"] == "ok")


def test_metrics_collector_records(tmp_path):
    """One JSONL record per collect(): step, optimizer type, its diagnostics
    (rank, effective rank, ...), and norms (the gradient norm only while
    gradients exist)."""
    import json

    import torch

    from dion_b200.benchmarks.metrics_collector import OptimizerMetricsCollector
    from dion_b200.optim import AdaDion

    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(32, 16))
    opt = AdaDion([p], lr=0.02, init_rank=4, rank_min=2, rank_max=8)
    col = OptimizerMetricsCollector(opt, output_dir=str(tmp_path))
    for step in (1, 2):
        p.grad = torch.randn_like(p)
        opt.step()
        rec = col.collect(step, loss=1.0)
    assert rec["opt_0/type"] == "AdaDion" and rec["loss"] == 1.0
    assert abs(rec["opt_0/grad_norm"] - float(p.grad.norm())) < 1e-4
    assert abs(rec["opt_0/param_norm"] - float(p.detach().norm())) < 1e-4
    assert any(k.startswith("opt_0/rank/") for k in rec)
    opt.zero_grad(set_to_none=True)
    rec = col.collect(3)
    assert "opt_0/grad_norm" not in rec and "opt_0/param_norm" in rec
    col.close()
    lines = [json.loads(l) for l in open(tmp_path / "optimizer_metrics.jsonl")]
    assert [r["step"] for r in lines] == [1, 2, 3]
    assert col.get_history()["loss"] == [1.0, 1.0]


def test_tier_b_times_each_optimizer_per_shape():
    from dion_b200.benchmarks import tiers

    res = tiers.run_tier_b("cpu", shapes=[(64, 32), (32, 96)], warmup=1, steps=2)
    assert set(res) == {"64x32", "32x96"}
    for row in res.values():
        assert set(row) == {"AdamW", "Muon", "Dion", "Dion2"}
        assert all(v["mean_ms"] > 0 and v["min_ms"] <= v["mean_ms"] for v in row.values())
