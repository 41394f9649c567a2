#!/usr/bin/env bash
# GSM8K launcher with fixed defaults for the four standard runs:
#   run_gsm8k.sh ar-1b | ar-8b | atlas | atlas-serial  [extra eval.gsm8k flags...]
# ar-1b / ar-8b: greedy AR of the drafter / target model alone; atlas: asynchronous ATLAS
# against a running target server (TARGET_URL); atlas-serial: tree -> verify -> commit with
# an in-process target.  Defaults come from the environment (DRAFTER_MODEL, TARGET_MODEL,
# TARGET_URL, GSM8K_FILE, OUTPUT_DIR, K, D, MAX_NEW_TOKENS, CONTEXT_LENGTH, WARMUP_RUNS,
# GPU_ID); flags after the run name are appended and win over them.
# Counterparts: the reference's scripts/run_gsm8k_{1b_ar,8b_ar,atlas,atlas_serial}.sh.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
cd "$here/../.."
run="${1:?usage: run_gsm8k.sh ar-1b|ar-8b|atlas|atlas-serial [flags...]}"
shift
drafter="${DRAFTER_MODEL:-llama-1b}"
target="${TARGET_MODEL:-llama-8b}"
common=(--data-file "${GSM8K_FILE:-gsm8k/test.jsonl}" --gpu-id "${GPU_ID:-0}"
        --k "${K:-3}" --d "${D:-4}" --max-new-tokens "${MAX_NEW_TOKENS:-512}"
        --context-length "${CONTEXT_LENGTH:-4096}" --warmup-runs "${WARMUP_RUNS:-1}")
case "$run" in
  ar-1b) args=(--backend ar --model "$drafter" --output-dir "${OUTPUT_DIR:-outputs/gsm8k_ar_1b}") ;;
  ar-8b) args=(--backend ar --model "$target" --output-dir "${OUTPUT_DIR:-outputs/gsm8k_ar_8b}") ;;
  atlas) args=(--backend atlas --model "$drafter" --target-url "${TARGET_URL:-http://127.0.0.1:18090}"
               --output-dir "${OUTPUT_DIR:-outputs/gsm8k_atlas}") ;;
  atlas-serial) args=(--backend atlas_serial --model "$drafter" --target-model "$target"
                      --output-dir "${OUTPUT_DIR:-outputs/gsm8k_atlas_serial}") ;;
  *) echo "unknown run '$run' (ar-1b, ar-8b, atlas, atlas-serial)" >&2; exit 2 ;;
esac
exec python -m 0709_b200.eval.gsm8k "${args[@]}" "${common[@]}" "$@"
