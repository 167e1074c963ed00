#!/usr/bin/env bash
# NUMA-aware per-rank launcher (torchrun --no_python ./numa_launch.sh -- train.py ...).
# Pins each local rank to a block of cores on its GPU's NUMA node: CONTROLLER_CORES
# cores (default 1) for the launching thread, the rest for the host worker pool
# (LayerAdam, CPU reduce), exported as NUMA_CPU_ADAM_CORES / T1_HOST_THREADS.
set -euo pipefail
PYTHON_BIN=${PYTHON_BIN:-python}
if [[ "$#" -gt 0 && "$1" == "--" ]]; then shift; fi
if [[ "$#" -eq 0 ]]; then
  echo "usage: torchrun ... --no_python $0 -- <script.py> [args...]" >&2
  exit 1
fi
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
eval "$(PYTHONPATH="$HERE:${PYTHONPATH:-}" "$PYTHON_BIN" -m test1_b200.runtime.numa)"
if [[ "${NUMA_LAUNCH_DEBUG:-0}" == "1" ]]; then
  echo "[numa_launch] rank ${LOCAL_RANK:-0}: node $NUMA_NODE control $NUMA_CONTROL_CORES pool $NUMA_CPU_ADAM_CORES" >&2
fi
ALL_CPUS="$NUMA_CONTROL_CORES,$NUMA_CPU_ADAM_CORES"
if command -v numactl >/dev/null 2>&1; then
  exec numactl --physcpubind="$ALL_CPUS" --preferred="$NUMA_NODE" "$PYTHON_BIN" "$@"
elif command -v taskset >/dev/null 2>&1; then
  exec taskset -c "$ALL_CPUS" "$PYTHON_BIN" "$@"
else
  exec "$PYTHON_BIN" "$@"
fi
