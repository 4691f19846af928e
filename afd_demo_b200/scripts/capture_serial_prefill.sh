#!/usr/bin/env bash
# Re-run serial prefill-only for every serial cache entry and merge its
# prefill_ms (reference: scripts/capture_serial_prefill.sh). Thin wrapper over
# capture_serial_split.py. Usage: capture_serial_prefill.sh [--skip-existing]
# Environment: SKIP_BATCHES (comma list), RESULTS_DIR (default results).
HERE="$(cd "$(dirname "$0")" && pwd)"
cd "$HERE/../.." || exit 1
ARGS=(--root "${RESULTS_DIR:-results}")
[ "${1:-}" = "--skip-existing" ] && ARGS+=(--skip-existing)
[ -n "${SKIP_BATCHES:-}" ] && ARGS+=(--skip-batches "$SKIP_BATCHES")
exec python -m afd_demo_b200.scripts.capture_serial_split "${ARGS[@]}"
