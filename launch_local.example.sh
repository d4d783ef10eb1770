#!/bin/bash
# launch_local.example.sh - prepare a run directory, then sweep NP_LIST x
# RUN_TYPES on this node with the bundled launcher (no MPI needed).
set -euo pipefail
SCRIPT_DIR="$(cd "$(dirname "$0")" && pwd)"
cd "${SCRIPT_DIR}"
export CONFIG=${CONFIG:-benchmark.env}
export RUN_LABEL=${RUN_LABEL:-"$(hostname)_$(date +%Y%m%d_%H%M%S)"}
export LAUNCHER=${LAUNCHER:-local}
./run_suite.sh
RUN_DIR="${RESULTS_ROOT:-${SCRIPT_DIR}/results}/${RUN_LABEL}"
for np in ${NP_LIST:-1 2 4 8}; do
  for run_type in ${RUN_TYPES:-comm attention}; do
    case "${run_type}" in
      comm) NP="${np}" ./benchmark_comm.sh > "${RUN_DIR}/comm_np${np}.log" 2>&1 ;;
      attention) NP="${np}" ./benchmark_attention.sh > "${RUN_DIR}/attention_np${np}.log" 2>&1 ;;
    esac
  done
done
echo "logs in ${RUN_DIR}"
