#!/usr/bin/env bash
# Run one experiment configuration and write its timing JSON (+ report).
#
# Usage: afd_demo_b200/scripts/run_single.sh <local|multinode> <batch> <seq> [options]
#
# Same positional arguments, options, file names and exit codes as the
# reference's scripts/run_single.sh:
#   --tokens N            generated tokens (default 5)
#   --no-dbo              serial baseline
#   --generate            autoregressive decode (default: prefill only)
#   --crosslayer          cross-layer decode pipeline
#   --warmup-p2p          untimed P2P warmup; --warmup-rounds N (default 3)
#   --comm-timing-mode M  enqueue (default) | completion
#   --visualize           pipeline Gantt PNG after the run
#   --verbose             verbose logging
#   --no-timing           no timing JSON / report
# Additions for B200:
#   --gpus N              1 (both roles on one GPU), 2 (1A+1F), 4 (2A+2F), 8 (4A+4F); default $GPUS or 2
#   --comm-impl I         auto (fused peer memory) | fused | nccl
#   --cuda-graph          capture decode steps in CUDA graphs
# Environment: MODEL_PATH (checkpoint dir or preset, default qwen3-30b-a3b with
# random weights), MASTER_PORT (default 29650), RESULTS_DIR (default results),
# NNODES / NODE_RANK / MASTER_ADDR for multinode (torchrun rendezvous).
#
# Output: $RESULTS_DIR/prefill_dbo/timing_{attention,ffn}_<suffix>.json, where
# suffix = [warmup_][serial_]<deployment>_b<B>_s<S>_t<T>[_crosslayer][_comm-<mode>].
# Exit codes: 0 ok, 1 failure, 2 out of memory.

HERE="$(cd "$(dirname "$0")" && pwd)"
ROOT="$(cd "$HERE/../.." && pwd)"
cd "$ROOT" || exit 1
RUN_START_TS=$(date +%s)

usage() { sed -n '2,28p' "$0" | sed 's/^# \{0,1\}//'; }
if [ "${1:-}" = "-h" ] || [ "${1:-}" = "--help" ]; then usage; exit 0; fi

DEPLOYMENT="${1:-}"; BATCH="${2:-}"; SEQ="${3:-}"
shift 3 2>/dev/null || true
if [ -z "$DEPLOYMENT" ] || [ -z "$BATCH" ] || [ -z "$SEQ" ]; then usage; exit 1; fi

TOKENS=5; NO_DBO=false; VISUALIZE=false; VERBOSE=false; GENERATE=false
WARMUP_P2P=false; WARMUP_ROUNDS=3; CROSSLAYER=false; COMM_TIMING_MODE=enqueue
TIMING=true; GPUS="${GPUS:-2}"; COMM_IMPL=auto; CUDA_GRAPH=false
while [ $# -gt 0 ]; do
    case "$1" in
        --tokens) TOKENS="$2"; shift 2;;
        --no-dbo) NO_DBO=true; shift;;
        --visualize) VISUALIZE=true; shift;;
        --verbose) VERBOSE=true; shift;;
        --generate) GENERATE=true; shift;;
        --warmup-p2p) WARMUP_P2P=true; shift;;
        --warmup-rounds) WARMUP_ROUNDS="$2"; shift 2;;
        --crosslayer) CROSSLAYER=true; shift;;
        --comm-timing-mode) COMM_TIMING_MODE="$2"; shift 2;;
        --no-timing) TIMING=false; shift;;
        --gpus) GPUS="$2"; shift 2;;
        --comm-impl) COMM_IMPL="$2"; shift 2;;
        --cuda-graph) CUDA_GRAPH=true; shift;;
        *) echo "ERROR: Unknown option: $1"; exit 1;;
    esac
done
case "$COMM_TIMING_MODE" in enqueue|completion) ;; *)
    echo "ERROR: --comm-timing-mode must be enqueue or completion"; exit 1;; esac

MODEL_PATH="${MODEL_PATH:-qwen3-30b-a3b}"
MASTER_PORT="${MASTER_PORT:-29650}"
RESULTS_DIR="${RESULTS_DIR:-results}"
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
export NCCL_BUFFSIZE="${NCCL_BUFFSIZE:-33554432}"
export NCCL_NCHANNELS_PER_NET_PEER="${NCCL_NCHANNELS_PER_NET_PEER:-1}"

# -- suffix (same rules as the reference) --------------------------------------
if [ "$NO_DBO" = true ]; then SUFFIX="serial_${DEPLOYMENT}_b${BATCH}_s${SEQ}_t${TOKENS}"
else SUFFIX="${DEPLOYMENT}_b${BATCH}_s${SEQ}_t${TOKENS}"; fi
FLAGS=(--model-name "$MODEL_PATH" --batch-size "$BATCH" --prefill-seq-len "$SEQ"
       --max-new-tokens "$TOKENS" --greedy --comm-impl "$COMM_IMPL"
       --comm-timing-mode "$COMM_TIMING_MODE" --results-dir "$RESULTS_DIR")
[ "$GENERATE" = true ] || FLAGS+=(--no-generate)
[ "$NO_DBO" = true ] && FLAGS+=(--no-dbo)
if [ "$WARMUP_P2P" = true ]; then
    FLAGS+=(--warmup-p2p --warmup-rounds "$WARMUP_ROUNDS"); SUFFIX="warmup_${SUFFIX}"
fi
if [ "$CROSSLAYER" = true ]; then FLAGS+=(--crosslayer); SUFFIX="${SUFFIX}_crosslayer"; fi
[ "$COMM_TIMING_MODE" != "enqueue" ] && SUFFIX="${SUFFIX}_comm-${COMM_TIMING_MODE}"
[ "$TIMING" = true ] && FLAGS+=(--timing --timing-suffix "$SUFFIX")
[ "$VERBOSE" = true ] && FLAGS+=(--verbose)
[ "$CUDA_GRAPH" = true ] && FLAGS+=(--cuda-graph)

echo "========================================"
echo "  Experiment: $SUFFIX  (gpus=$GPUS, comm=$COMM_IMPL)"
echo "  DBO: $([ "$NO_DBO" = true ] && echo disabled || echo enabled)  generate: $GENERATE"
echo "========================================"
LOGDIR="$RESULTS_DIR/prefill_dbo/logs"
mkdir -p "$LOGDIR"
LOG="$LOGDIR/run_${SUFFIX}.log"

run_local() {
    if [ "$GPUS" = 1 ]; then
        python -u -m afd_demo_b200.main --world-size 1 --rank 0 --local-rank 0 "${FLAGS[@]}" \
            > "$LOG" 2>&1
    else
        python -u -m torch.distributed.run --nnodes=1 --nproc-per-node "$GPUS" \
            --master-addr 127.0.0.1 --master-port "$MASTER_PORT" \
            -m afd_demo_b200.main --local-test "${FLAGS[@]}" > "$LOG" 2>&1
    fi
}

run_multinode() {
    # one torchrun per node; attention ranks come first (node 0)
    : "${NNODES:?set NNODES}" "${NODE_RANK:?set NODE_RANK}" "${MASTER_ADDR:?set MASTER_ADDR}"
    python -u -m torch.distributed.run --nnodes "$NNODES" --node-rank "$NODE_RANK" \
        --nproc-per-node "$GPUS" --master-addr "$MASTER_ADDR" --master-port "$MASTER_PORT" \
        -m afd_demo_b200.main --local-test "${FLAGS[@]}" 2>&1 | tee "$LOG"
    return "${PIPESTATUS[0]}"
}

case "$DEPLOYMENT" in
    local) run_local; RC=$?;;
    multinode) run_multinode; RC=$?;;
    *) echo "ERROR: Unknown deployment: $DEPLOYMENT (use 'local' or 'multinode')"; exit 1;;
esac
tail -5 "$LOG" | sed 's/^/[LOG] /'

if grep -q "OutOfMemoryError\|CUDA out of memory\|OOM" "$LOG" 2>/dev/null; then
    echo "OOM DETECTED for $SUFFIX"; exit 2
fi
if [ "$RC" -ne 0 ]; then echo "FAILED (rc=$RC) for $SUFFIX"; exit 1; fi

ATTN_TIMING="$RESULTS_DIR/prefill_dbo/timing_attention_${SUFFIX}.json"
FFN_TIMING="$RESULTS_DIR/prefill_dbo/timing_ffn_${SUFFIX}.json"
if [ "$TIMING" = true ] && { [ ! -f "$ATTN_TIMING" ] || [ ! -f "$FFN_TIMING" ]; }; then
    echo "Missing timing files for $SUFFIX"
    [ "$NO_DBO" = false ] && exit 1
fi

if [ "$VISUALIZE" = true ] && [ "$NO_DBO" = false ] && [ "$TIMING" = true ]; then
    python -m afd_demo_b200.scripts.visualize_dbo_pipeline --attn-timing "$ATTN_TIMING" \
        --ffn-timing "$FFN_TIMING" --output "$RESULTS_DIR/prefill_dbo/dbo_pipeline_${SUFFIX}.png" \
        --start-layer 1 --num-layers 4
fi

if [ "$TIMING" = true ] && [ -f "$ATTN_TIMING" ] && [ -f "$FFN_TIMING" ]; then
    if [ "$NO_DBO" = true ]; then MODE_TAG=serial
    elif [ "$GENERATE" = false ]; then MODE_TAG=prefill-dbo
    elif [ "$CROSSLAYER" = true ]; then MODE_TAG=decode-dbo-crosslayer
    else MODE_TAG=decode-dbo; fi
    CACHE="$RESULTS_DIR/serial/cache/b${BATCH}_s${SEQ}_t${TOKENS}.json"
    CMP=()
    [ -f "$CACHE" ] && [ "$NO_DBO" = false ] && CMP=(--serial-baseline "$CACHE")
    python -m afd_demo_b200.scripts.gen_experiment_report --attn-timing "$ATTN_TIMING" \
        --ffn-timing "$FFN_TIMING" --output "$RESULTS_DIR/prefill_dbo/report_${SUFFIX}.md" \
        --mode "$MODE_TAG" --batch "$BATCH" --seq "$SEQ" --tokens "$TOKENS" \
        --comm-timing-mode "$COMM_TIMING_MODE" "${CMP[@]}" || echo "[WARN] report generation failed"
fi
echo "Experiment completed: $SUFFIX ($(( $(date +%s) - RUN_START_TS ))s wall)"
exit 0
