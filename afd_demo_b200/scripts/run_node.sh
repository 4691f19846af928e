#!/usr/bin/env bash
# Start one rank by hand (one process per GPU), e.g. on each node of a
# multi-node run (reference: scripts/run_node.sh). Two forms:
#
#   run_node.sh <attention|ffn> [master_addr] [master_port] [options]
#       the reference's form: the role picks the rank (ATTN_RANK, default 0,
#       or FFN_RANK, default 1) and is passed on as --role
#   run_node.sh [options]
#       rank and rendezvous from the environment (RANK, MASTER_ADDR, ...)
#
# Environment:
#   MODEL_PATH     checkpoint dir or preset (default qwen3-30b-a3b, random weights)
#   CUDA_DEVICES   GPU(s) visible to this rank (default 0)
#   WORLD_SIZE     total ranks (default 2)
#   RANK           this rank (default 0); ranks [0, ATTN_GPUS) are attention ranks
#   LOCAL_RANK     device index inside CUDA_DEVICES (default 0)
#   ATTN_RANK / FFN_RANK   2-rank layout (default 0 / 1)
#   ATTN_GPUS / FFN_GPUS   topology for WORLD_SIZE > 2 (default half / half)
#   BATCH_SIZE     default 4; MAX_SEQ_LEN default 128; TOKENS default 20
#   MASTER_ADDR / MASTER_PORT   rendezvous (default 127.0.0.1:29500)
#   RUN_NODE_DRY_RUN=1   print the command instead of running it
# Options are passed to afd_demo_b200.main.
HERE="$(cd "$(dirname "$0")" && pwd)"
cd "$HERE/../.." || exit 1
export CUDA_VISIBLE_DEVICES="${CUDA_DEVICES:-0}"
WORLD_SIZE="${WORLD_SIZE:-2}"
EXTRA=()
case "${1:-}" in
    attention|ffn)
        ROLE="$1"
        shift
        if [ "$ROLE" = attention ]; then RANK="${ATTN_RANK:-0}"; else RANK="${FFN_RANK:-1}"; fi
        if [ $# -gt 0 ] && [ "${1#-}" = "$1" ]; then MASTER_ADDR="$1"; shift; fi
        if [ $# -gt 0 ] && [ "${1#-}" = "$1" ]; then MASTER_PORT="$1"; shift; fi
        EXTRA+=(--role "$ROLE")
        ;;
    -*|"") ;;
    *)
        echo "run_node.sh: role must be 'attention' or 'ffn', got '$1'" >&2
        exit 1
        ;;
esac
[ -n "${ATTN_GPUS:-}" ] && EXTRA+=(--attn-gpus "$ATTN_GPUS")
[ -n "${FFN_GPUS:-}" ] && EXTRA+=(--ffn-gpus "$FFN_GPUS")
CMD=(python -u -m afd_demo_b200.main
    --model-name "${MODEL_PATH:-qwen3-30b-a3b}"
    --world-size "$WORLD_SIZE" --rank "${RANK:-0}" --local-rank "${LOCAL_RANK:-0}"
    --attn-node-rank "${ATTN_RANK:-0}" --ffn-node-rank "${FFN_RANK:-1}"
    --master-addr "${MASTER_ADDR:-127.0.0.1}" --master-port "${MASTER_PORT:-29500}"
    --batch-size "${BATCH_SIZE:-4}" --max-seq-len "${MAX_SEQ_LEN:-128}"
    --max-new-tokens "${TOKENS:-20}" "${EXTRA[@]}" "$@")
if [ "${RUN_NODE_DRY_RUN:-0}" = 1 ]; then
    echo "${CMD[@]}"
    exit 0
fi
exec "${CMD[@]}"
