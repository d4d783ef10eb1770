#!/bin/bash
# launch_mpirun.example.sh - the same sweep with an existing MPI installation
# (counterpart of the reference's launch_mpirun.example.sh:25-48)
# (mpirun only starts the ranks; they bootstrap through torch.distributed and
# communicate through the native runtime, not through MPI).
set -euo pipefail
SCRIPT_DIR="$(cd "$(dirname "$0")" && pwd)"
cd "${SCRIPT_DIR}"
export CONFIG=${CONFIG:-benchmark.env}
export RUN_LABEL=${RUN_LABEL:-"$(hostname)_$(date +%Y%m%d_%H%M%S)"}
export LAUNCHER=mpirun MASTER_ADDR=${MASTER_ADDR:-127.0.0.1} MASTER_PORT=${MASTER_PORT:-29517}
./run_suite.sh
RUN_DIR="${RESULTS_ROOT:-${SCRIPT_DIR}/results}/${RUN_LABEL}"
for np in ${NP_LIST:-2 4 8}; do
  NP="${np}" ./benchmark_comm.sh > "${RUN_DIR}/comm_np${np}.log" 2>&1
  NP="${np}" ./benchmark_attention.sh > "${RUN_DIR}/attention_np${np}.log" 2>&1
done
