#!/usr/bin/env bash
# Start one rank by hand (one process per GPU), e.g. on each node of a
# multi-node run. Environment (reference: scripts/run_node.sh):
#   MODEL_PATH     checkpoint dir or preset (default qwen3-30b-a3b, random weights)
#   CUDA_DEVICES   GPU(s) visible to this rank (default 0)
#   WORLD_SIZE     total ranks (default 2)
#   RANK           this rank (default 0); ranks [0, ATTN_GPUS) are attention ranks
#   LOCAL_RANK     device index inside CUDA_DEVICES (default 0)
#   ATTN_RANK / FFN_RANK   2-rank layout (default 0 / 1)
#   ATTN_GPUS / FFN_GPUS   topology for WORLD_SIZE > 2 (default half / half)
#   BATCH_SIZE     default 4; MAX_SEQ_LEN default 128; TOKENS default 20
#   MASTER_ADDR / MASTER_PORT   rendezvous (default 127.0.0.1:29500)
# Extra arguments are passed to afd_demo_b200.main.
HERE="$(cd "$(dirname "$0")" && pwd)"
cd "$HERE/../.." || exit 1
export CUDA_VISIBLE_DEVICES="${CUDA_DEVICES:-0}"
WORLD_SIZE="${WORLD_SIZE:-2}"
EXTRA=()
[ -n "${ATTN_GPUS:-}" ] && EXTRA+=(--attn-gpus "$ATTN_GPUS")
[ -n "${FFN_GPUS:-}" ] && EXTRA+=(--ffn-gpus "$FFN_GPUS")
exec python -u -m afd_demo_b200.main \
    --model-name "${MODEL_PATH:-qwen3-30b-a3b}" \
    --world-size "$WORLD_SIZE" --rank "${RANK:-0}" --local-rank "${LOCAL_RANK:-0}" \
    --attn-node-rank "${ATTN_RANK:-0}" --ffn-node-rank "${FFN_RANK:-1}" \
    --master-addr "${MASTER_ADDR:-127.0.0.1}" --master-port "${MASTER_PORT:-29500}" \
    --batch-size "${BATCH_SIZE:-4}" --max-seq-len "${MAX_SEQ_LEN:-128}" \
    --max-new-tokens "${TOKENS:-20}" "${EXTRA[@]}" "$@"
