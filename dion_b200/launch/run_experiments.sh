#!/usr/bin/env bash
# Experiment matrix of the reference's benchmark blueprint, on this package's trainer.
#
#   bash dion_b200/launch/run_experiments.sh <experiment> [extra --section.field overrides...]
#
# experiments:
#   perf        500 steps per optimizer on one node (FSDP over NGPU), profiler traces every 100 steps
#   convergence STEPS (default 10000) per optimizer x seeds 42 123 7, validation every 200 steps
#               (needs VAL_DATA=<held-out token files>; TRAIN_DATA=<token files>, else synthetic tokens)
#   dion2       Dion2 fraction ablation (0.25, 0.5, 1.0), 5000 steps
#   adadion     AdaDion sweep: lr {0.005,0.01,0.02,0.05} x init_rank {32,64,128} x adaptive {on,off}
#               x mu {0.9,0.95} = 48 runs (START_IDX / END_IDX select a slice)
#   anchor      3 candidates x seeds 42 123: Dion baseline, + anchor, + anchor with a faster refresh
#   sdion       SDion screening: modes baseline / skip / skip_consensus / skip_cons_anchor x seeds 42 123
#   all         perf, convergence, dion2
#
# Environment: NGPU (8), MODEL (320m for the AdaDion-family experiments, 160m otherwise),
# LOGDIR (logs/experiments), DRY_RUN=1 (print the runs only); the per-run log is
# $LOGDIR/<run>/train.log, and runs go on after a failure (the count of failed runs is printed
# at the end).
set -uo pipefail
EXP=${1:-all}
shift || true
NGPU=${NGPU:-8}
LOGDIR=${LOGDIR:-logs/experiments}
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
FAILED=0
RUNS=0
DATA_ARGS=()
[ -n "${TRAIN_DATA:-}" ] && DATA_ARGS+=(--dataloader.dataset "$TRAIN_DATA")

run() {  # run <name> <optimizer> <steps> [overrides...]
    local name=$1 opt=$2 steps=$3
    shift 3
    RUNS=$((RUNS + 1))
    if [ -n "${DRY_RUN:-}" ]; then  # print the run instead of starting it
        echo "DRY_RUN name=$name model=${MODEL:-160m} optimizer=$opt steps=$steps args=${DATA_ARGS[*]} $*"
        return
    fi
    mkdir -p "$LOGDIR/$name"
    echo "--- [$RUNS] $name ($opt, $steps steps, $NGPU GPUs) ---"
    if WANDB_RUN_NAME="$name" STEPS="$steps" NGPU="$NGPU" MODEL="${MODEL:-160m}" \
        bash "$HERE/run_single_node.sh" "$opt" "${DATA_ARGS[@]}" "$@" 2>&1 | tee "$LOGDIR/$name/train.log"; then
        echo "    done: $name"
    else
        echo "    FAILED: $name"
        FAILED=$((FAILED + 1))
    fi
}

perf() {
    for opt in adamw muon dion dion2 adadion; do
        run "perf_${opt}_${NGPU}gpu" "$opt" 500 --profiling.enable_profiling --profiling.profile_freq 100 \
            --profiling.save_traces_folder "$LOGDIR/perf_${opt}_${NGPU}gpu/traces" "$@"
    done
}

convergence() {
    local val=()
    [ -n "${VAL_DATA:-}" ] && val=(--validator.enable --validator.dataset "$VAL_DATA" --validator.freq 200
                                   --validator.steps 50)
    for seed in 42 123 7; do
        for opt in adamw muon dion dion2 adadion; do
            run "convergence_${opt}_seed${seed}" "$opt" "${STEPS:-10000}" --debug.seed "$seed" "${val[@]}" "$@"
        done
    done
}

dion2() {
    for frac in 0.25 0.5 1.0; do
        run "ablation_dion2_frac${frac}" dion2 5000 --optimizer.fraction "$frac" "$@"
    done
}

adadion() {
    local i=0 start=${START_IDX:-1} end=${END_IDX:-48}
    for lr in 0.005 0.01 0.02 0.05; do
        for rank in 32 64 128; do
            for adaptive in true false; do
                for mu in 0.9 0.95; do
                    i=$((i + 1))
                    [ "$i" -lt "$start" ] || [ "$i" -gt "$end" ] && continue
                    MODEL=${MODEL:-320m} run "adadion_lr${lr}_r${rank}_ad${adaptive}_mu${mu}" adadion "${STEPS:-2000}" \
                        --optimizer.lr "$lr" --optimizer.init_rank "$rank" --optimizer.adaptive_rank "$adaptive" \
                        --optimizer.mu "$mu" "$@"
                done
            done
        done
    done
}

anchor() {
    for seed in 42 123; do
        MODEL=${MODEL:-320m} run "anchor_baseline_s${seed}" adadion "${STEPS:-2000}" --debug.seed "$seed" \
            --optimizer.no-use_anchor "$@"
        MODEL=${MODEL:-320m} run "anchor_on_s${seed}" adadion "${STEPS:-2000}" --debug.seed "$seed" \
            --optimizer.use_anchor --optimizer.anchor_alpha 0.1 "$@"
        MODEL=${MODEL:-320m} run "anchor_fast_refresh_s${seed}" adadion "${STEPS:-2000}" --debug.seed "$seed" \
            --optimizer.use_anchor --optimizer.anchor_alpha 0.1 --optimizer.anchor_period 10 "$@"
    done
}

sdion() {
    for seed in 42 123; do
        for mode in baseline skip skip_consensus skip_cons_anchor; do
            MODEL=${MODEL:-320m} run "sdion_${mode}_s${seed}" adadion "${STEPS:-2000}" --debug.seed "$seed" \
                --optimizer.sdion_mode "$mode" "$@"
        done
    done
}

case "$EXP" in
    perf) perf "$@" ;;
    convergence) convergence "$@" ;;
    dion2) dion2 "$@" ;;
    adadion) adadion "$@" ;;
    anchor) anchor "$@" ;;
    sdion) sdion "$@" ;;
    all) perf "$@"; convergence "$@"; dion2 "$@" ;;
    *) echo "usage: $0 {perf|convergence|dion2|adadion|anchor|sdion|all} [overrides...]"; exit 2 ;;
esac
echo "=== $EXP: $RUNS runs, $FAILED failed ==="
[ "$FAILED" -eq 0 ]
