"""Research harnesses on tiny settings (CPU): QCDion protocol checks, GSDion
ladder, seed confirmation, snapshot collect + replay, and the local pipeline."""
import json

import pytest

from dion_b200.research import gsdion_ladder, pipeline_local, qcdion_protocol, replay, seed_confirmation


@pytest.mark.parametrize("name,fn", qcdion_protocol.CHECKS)
def test_qcdion_protocol(name, fn):
    fn()


def test_gsdion_ladder_tiny(tmp_path):
    res = gsdion_ladder.main(["--steps", "6", "--eval-freq", "3", "--hidden", "64", "--init-rank", "8",
                              "--configs", "1_dion_baseline,2_ranknorm_lrcomp,7_full_gsdion", "--outdir",
                              str(tmp_path), "--data-dir", str(tmp_path / "none")])
    assert set(res) == {"1_dion_baseline", "2_ranknorm_lrcomp", "7_full_gsdion"}
    assert res["2_ranknorm_lrcomp"]["lr"] == pytest.approx(0.02 * 8 ** 0.5)
    with open(tmp_path / "gsdion_ladder.json") as fh:
        assert json.load(fh)["data"] == "synthetic"


def test_seed_confirmation_tiny(tmp_path):
    rows, summary = seed_confirmation.main(["--steps", "4", "--seeds", "1,2", "--hidden", "64", "--init-rank", "8",
                                            "--outdir", str(tmp_path), "--data-dir", str(tmp_path / "none")])
    assert len(rows) == 2 and 0.0 < summary["cosine_mean"][0] <= 1.0


def test_replay_collect_and_replay(tmp_path):
    snaps = replay.collect(4, 2, str(tmp_path / "snaps"), data_dir=str(tmp_path / "none"))
    assert len(snaps) == 2
    rows = replay.replay(str(tmp_path / "snaps"), [8], str(tmp_path / "out"))
    assert rows and all(abs(r["dion/cos_to_dion"] - 1.0) < 1e-4 for r in rows)
    # rank normalisation with sqrt(r) lr compensation leaves the update unchanged
    assert all(abs(r["normdion/update_rms"] - r["dion/update_rms"]) < 1e-6 * max(1.0, r["dion/update_rms"])
               for r in rows)


def test_pipeline_local_tiny(tmp_path):
    out = pipeline_local.main(["--steps", "3", "--optimizers", "muon,dion", "--seq-len", "32", "--batch", "2",
                               "--outdir", str(tmp_path)])
    assert set(out["runs"]) == {"muon", "dion"} and out["sweep_runs"] == 33
    assert all(v["pass"] for v in out["tier_a"].values())
