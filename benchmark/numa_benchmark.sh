#!/usr/bin/env bash
# LayerAdam host-kernel bandwidth under NUMA bindings (the reference's
# benchmark/numa_benchmark.sh capability): for every node N, threads on N
# with memory on N ("same"), memory on the next node ("cross"), and memory
# interleaved over all nodes ("interleave").  On a single-node host only the
# "default" run is made.  Results: $OUT/<binding>.json, summarised by
# analyze_results.py.
#   MODEL=8B THREADS=1,4,8,16 OUT=results/numa bash benchmark/numa_benchmark.sh
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
MODEL="${MODEL:-8B}"
OUT="${OUT:-results/numa}"
PY="${PYTHON_BIN:-python}"
mkdir -p "$OUT"
nodes=$(ls -d /sys/devices/system/node/node[0-9]* 2>/dev/null | wc -l)
targs=()
if [[ -n "${THREADS:-}" ]]; then targs=(--threads "$THREADS"); fi
if [[ "$nodes" -le 1 ]] || ! command -v numactl >/dev/null 2>&1; then
  echo "single NUMA node (or no numactl): default binding only"
  "$PY" "$HERE/cpu_adam_benchmark.py" --model "$MODEL" "${targs[@]}" --json "$OUT/default.json"
else
  for ((n = 0; n < nodes; n++)); do
    other=$(( (n + 1) % nodes ))
    numactl --cpunodebind="$n" --membind="$n" "$PY" "$HERE/cpu_adam_benchmark.py" --model "$MODEL" "${targs[@]}" --json "$OUT/same_node$n.json"
    numactl --cpunodebind="$n" --membind="$other" "$PY" "$HERE/cpu_adam_benchmark.py" --model "$MODEL" "${targs[@]}" --json "$OUT/cross_node$n.json"
    numactl --cpunodebind="$n" --interleave=all "$PY" "$HERE/cpu_adam_benchmark.py" --model "$MODEL" "${targs[@]}" --json "$OUT/interleave_node$n.json"
  done
fi
"$PY" "$HERE/analyze_results.py" "$OUT"/*.json
