#!/usr/bin/env bash
# Full LayerAdam host-kernel sweep (the reference's benchmark/run_full_benchmark.sh
# capability): every model preset x thread counts x master layout, one JSON
# per preset in $OUT, then the summary.  COMPARE_REFERENCE=1 also times the
# reference's own cpu_adam (JIT-built from baseline/_ref) on each preset.
#   OUT=results/full THREADS=1,4,8,16 bash benchmark/run_full_benchmark.sh
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="${OUT:-results/full}"
PY="${PYTHON_BIN:-python}"
MODELS="${MODELS:-3B 8B 14B 32B 72B}"
mkdir -p "$OUT"
extra=()
if [[ -n "${THREADS:-}" ]]; then extra+=(--threads "$THREADS"); fi
if [[ "${COMPARE_REFERENCE:-0}" == "1" ]]; then extra+=(--compare-reference); fi
for m in $MODELS; do
  echo "== $m"
  "$PY" "$HERE/cpu_adam_benchmark.py" --model "$m" --steps "${STEPS:-3}" "${extra[@]}" --json "$OUT/adam_$m.json"
done
"$PY" "$HERE/analyze_results.py" "$OUT"/adam_*.json
