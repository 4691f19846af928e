#!/usr/bin/env bash
# Sweep modes x seqs x batches through run_single.sh and write a summary CSV.
#
# Usage: afd_demo_b200/scripts/run_experiment_matrix.sh [options]
#   --modes M1,M2    serial,prefill-dbo,decode-dbo,decode-dbo-crosslayer (default: all)
#   --batches B,..   default 2,4,8,16,32,64
#   --seqs S,..      default 128,256,512
#   --tokens N       default 20
#   --deployment D   local (default) | multinode
#   --comm-timing-mode M   enqueue (default) | completion
#   --gpus N         GPUs per run (default $GPUS or 2)
#   --comm-impl I    auto | fused | nccl
#   --no-cache       re-run serial even when results/serial/cache has the cell
#   --dry-run        print the commands only
#
# Reference: scripts/run_experiment_matrix.sh. Same per-mode flags
# (serial: --no-dbo --generate; prefill-dbo: prefill only; decode-dbo:
# --generate; decode-dbo-crosslayer: --generate --crosslayer; all with
# --warmup-p2p --warmup-rounds 5), the same result layout
# results/<mode>/timing_{role}_<mode>_b<B>_s<S>_t<T>.json, the serial cache
# results/serial/cache/b<B>_s<S>_t<T>.json, and the summary CSV
# mode,batch,seq,tokens,status,report with status ok/cached/OOM/FAIL. The first
# OOM of a (mode, seq) stops escalating its batch.
set -u
HERE="$(cd "$(dirname "$0")" && pwd)"
cd "$HERE/../.." || exit 1

MODES="serial,prefill-dbo,decode-dbo,decode-dbo-crosslayer"
BATCHES="2,4,8,16,32,64"; SEQS="128,256,512"; TOKENS=20; DEPLOYMENT=local
COMM_TIMING_MODE=enqueue; NO_CACHE=false; DRY_RUN=false; GPUS="${GPUS:-2}"; COMM_IMPL=auto
RESULTS_DIR="${RESULTS_DIR:-results}"
while [ $# -gt 0 ]; do
    case "$1" in
        --modes) MODES="$2"; shift 2;;
        --batches) BATCHES="$2"; shift 2;;
        --seqs) SEQS="$2"; shift 2;;
        --tokens) TOKENS="$2"; shift 2;;
        --deployment) DEPLOYMENT="$2"; shift 2;;
        --comm-timing-mode) COMM_TIMING_MODE="$2"; shift 2;;
        --gpus) GPUS="$2"; shift 2;;
        --comm-impl) COMM_IMPL="$2"; shift 2;;
        --no-cache) NO_CACHE=true; shift;;
        --dry-run) DRY_RUN=true; shift;;
        -h|--help) sed -n '2,24p' "$0" | sed 's/^# \{0,1\}//'; exit 0;;
        *) echo "Unknown option: $1"; exit 1;;
    esac
done
IFS=',' read -ra MODE_ARR <<< "$MODES"
IFS=',' read -ra BATCH_ARR <<< "$BATCHES"
IFS=',' read -ra SEQ_ARR <<< "$SEQS"
mkdir -p "$RESULTS_DIR/serial/cache" "$RESULTS_DIR/prefill-dbo" "$RESULTS_DIR/decode-dbo" \
    "$RESULTS_DIR/decode-dbo-crosslayer"

run_one() {
    local mode="$1" batch="$2" seq="$3" tokens="$4" outdir="$5"
    local tag="${mode}_b${batch}_s${seq}_t${tokens}"
    local flags=(--tokens "$tokens" --gpus "$GPUS" --comm-impl "$COMM_IMPL")
    case "$mode" in
        serial) flags+=(--no-dbo --generate);;
        prefill-dbo) ;;
        decode-dbo) flags+=(--generate);;
        decode-dbo-crosslayer) flags+=(--generate --crosslayer);;
    esac
    flags+=(--warmup-p2p --warmup-rounds 5 --comm-timing-mode "$COMM_TIMING_MODE")
    [ "$COMM_TIMING_MODE" != "enqueue" ] && tag="${tag}_comm-${COMM_TIMING_MODE}"
    echo ""
    echo "=== Running: $tag ==="
    if [ "$DRY_RUN" = true ]; then
        echo "[dry-run] bash afd_demo_b200/scripts/run_single.sh $DEPLOYMENT $batch $seq ${flags[*]}"
        return 0
    fi
    MASTER_PORT=$((29500 + RANDOM % 2000)) RESULTS_DIR="$RESULTS_DIR" \
        bash afd_demo_b200/scripts/run_single.sh "$DEPLOYMENT" "$batch" "$seq" "${flags[@]}"
    local rc=$?
    [ $rc -eq 2 ] && { echo "[OOM] $tag"; return 2; }
    [ $rc -ne 0 ] && { echo "[FAIL rc=$rc] $tag"; return $rc; }
    local raw="warmup_${DEPLOYMENT}_b${batch}_s${seq}_t${tokens}"
    [ "$mode" = serial ] && raw="warmup_serial_${DEPLOYMENT}_b${batch}_s${seq}_t${tokens}"
    [ "$mode" = decode-dbo-crosslayer ] && raw="${raw}_crosslayer"
    [ "$COMM_TIMING_MODE" != "enqueue" ] && raw="${raw}_comm-${COMM_TIMING_MODE}"
    mkdir -p "$outdir"
    for role in attention ffn; do
        local src="$RESULTS_DIR/prefill_dbo/timing_${role}_${raw}.json"
        [ -f "$src" ] && mv -f "$src" "$outdir/timing_${role}_${tag}.json"
    done
    local attn="$outdir/timing_attention_${tag}.json"
    [ "$mode" = serial ] && [ -f "$attn" ] && \
        cp -f "$attn" "$RESULTS_DIR/serial/cache/b${batch}_s${seq}_t${tokens}.json"
    local cache="$RESULTS_DIR/serial/cache/b${batch}_s${seq}_t${tokens}.json" cmp=()
    [ -f "$cache" ] && [ "$mode" != serial ] && cmp=(--serial-baseline "$cache")
    python -m afd_demo_b200.scripts.gen_experiment_report --attn-timing "$attn" \
        --ffn-timing "$outdir/timing_ffn_${tag}.json" --output "$outdir/report_${tag}.md" \
        --mode "$mode" --batch "$batch" --seq "$seq" --tokens "$tokens" \
        --comm-timing-mode "$COMM_TIMING_MODE" "${cmp[@]}" || true
    return 0
}

SUMMARY="$RESULTS_DIR/experiment_matrix_summary.csv"
echo "mode,batch,seq,tokens,status,report" > "$SUMMARY"
for MODE in "${MODE_ARR[@]}"; do
    case "$MODE" in
        serial) OUTDIR="$RESULTS_DIR/serial";;
        prefill-dbo) OUTDIR="$RESULTS_DIR/prefill-dbo";;
        decode-dbo) OUTDIR="$RESULTS_DIR/decode-dbo";;
        decode-dbo-crosslayer) OUTDIR="$RESULTS_DIR/decode-dbo-crosslayer";;
        *) echo "Unknown mode: $MODE"; exit 1;;
    esac
    for SEQ in "${SEQ_ARR[@]}"; do
        for BATCH in "${BATCH_ARR[@]}"; do
            CACHE="$RESULTS_DIR/serial/cache/b${BATCH}_s${SEQ}_t${TOKENS}.json"
            if [ "$MODE" = serial ] && [ "$NO_CACHE" = false ] && [ -f "$CACHE" ]; then
                echo "[cache-hit] serial b${BATCH}_s${SEQ}_t${TOKENS}"
                echo "serial,$BATCH,$SEQ,$TOKENS,cached,$CACHE" >> "$SUMMARY"
                continue
            fi
            run_one "$MODE" "$BATCH" "$SEQ" "$TOKENS" "$OUTDIR"
            rc=$?
            if [ $rc -eq 2 ]; then
                echo "$MODE,$BATCH,$SEQ,$TOKENS,OOM," >> "$SUMMARY"
                echo "OOM for $MODE seq=$SEQ; skipping larger batches."
                break
            elif [ $rc -ne 0 ]; then
                echo "$MODE,$BATCH,$SEQ,$TOKENS,FAIL," >> "$SUMMARY"
            else
                echo "$MODE,$BATCH,$SEQ,$TOKENS,ok,$OUTDIR/report_${MODE}_b${BATCH}_s${SEQ}_t${TOKENS}.md" \
                    >> "$SUMMARY"
            fi
        done
    done
done
echo ""
echo "Matrix complete. Summary: $SUMMARY"
cat "$SUMMARY"
