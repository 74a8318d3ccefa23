"""Research harnesses for the Dion-family variants (the reference's
ada_dion/scripts/{part_a_replay,run_seed_confirmation,run_gsdion_comparison,
test_qcdion,run_full_pipeline_local}.py), re-built on this package's
optimizers and trainer:

  * ``replay``             snapshot collection during training + offline replay
                           of Dion / NormDion / NormDion+scalar / +RMS-matching
  * ``seed_confirmation``  Dion vs rank-normalised Dion over several seeds
  * ``gsdion_ladder``      GSDion ablation ladder (one mechanism at a time)
  * ``qcdion_protocol``    QCDion checks: equivalence with Dion when its controls
                           are off, quality signals, gate, extra power step,
                           rank boost, end-to-end training
  * ``pipeline_local``     every optimizer on a small Llama on this machine, with
                           metrics JSONL and the plot set (measured, not simulated)

Datasets: FashionMNIST from ``--data-dir`` when present, otherwise a
synthetic FashionMNIST-shaped set (there is no network here); every result
records which one it used.
"""
