#!/bin/bash
#SBATCH --job-name=ring-attn-b200
#SBATCH --nodes=1
#SBATCH --gres=gpu:8
#SBATCH --time=01:00:00
# batch_slurm.example.sh - one 8xB200 node (counterpart of the reference's
# batch_slurm.example.sh:5-9,54-78).  The batch step prepares the run and
# starts each sweep with the bundled launcher (one node, NVLink/NVSwitch).
set -euo pipefail
cd "${SLURM_SUBMIT_DIR:-$(dirname "$0")}"
unset SLURM_PROCID SLURM_NTASKS   # the wrappers refuse to run inside a rank
export CONFIG=${CONFIG:-benchmark.env} LAUNCHER=local
export RUN_LABEL=${RUN_LABEL:-"slurm_${SLURM_JOB_ID:-manual}"}
./run_suite.sh
RUN_DIR="${RESULTS_ROOT:-$(pwd)/results}/${RUN_LABEL}"
for np in ${NP_LIST:-1 2 4 8}; do
  NP="${np}" ./benchmark_comm.sh > "${RUN_DIR}/comm_np${np}.log" 2>&1
  NP="${np}" ./benchmark_attention.sh > "${RUN_DIR}/attention_np${np}.log" 2>&1
done
