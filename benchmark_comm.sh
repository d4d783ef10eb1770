#!/bin/bash
# benchmark_comm.sh - comm-only ring benchmark over backends and sizes
# (counterpart of the reference's benchmark_comm.sh, backend loop :107-129).
#
# Env / benchmark.env keys: NP WARMUP ITERS SIZES COMM_SIZES BACKENDS LAUNCHER
# (local | torchrun | mpirun | srun | none) MPIRUN HOSTFILE MPIRUN_EXTRA_ARGS SRUN
# SRUN_MPI_TYPE SRUN_EXTRA_ARGS.  SIZES overrides COMM_SIZES; SIZE_UNIT=elements reads
# the sizes as fp32 element counts (default bytes).  RESUME=1 with
# RAB_RESULTS_JSONL skips configurations that file already records.  INPROCESS=1 runs
# every (backend, size) in one launch of the ranks.  Stops at the first
# failing backend/size, like the reference wrapper.
set -euo pipefail

SCRIPT_DIR="$(cd "$(dirname "$0")" && pwd)"
cd "${SCRIPT_DIR}"
# shellcheck disable=SC1091
source "${SCRIPT_DIR}/ring_env.sh"

CONFIG=${CONFIG:-benchmark.env}
rab_load_config "${CONFIG}"
rab_setup_paths

if rab_inside_launched_rank; then
  echo "ERROR: benchmark_comm.sh should be run from a normal shell; it launches the ranks itself." >&2
  exit 1
fi

NP=${NP:-2}
WARMUP=${WARMUP:-10}
ITERS=${ITERS:-100}
COMM_SIZES=${COMM_SIZES:-"262144 524288 1048576 4194304 16777216"}
SIZES=${SIZES:-${COMM_SIZES}}
BACKENDS=${BACKENDS:-"staged staged_Isendrecv cuda_aware cuda_aware_Isendrecv nccl b200_fused"}
LAUNCHER=${LAUNCHER:-local}
export LAUNCHER MPIRUN HOSTFILE MPIRUN_EXTRA_ARGS SRUN SRUN_MPI_TYPE SRUN_EXTRA_ARGS

BIN_DIR="${SCRIPT_DIR}/bin"

echo "========== Communication (Loop) Benchmark =========="
echo "Date: $(date)"
echo "Hostname: $(hostname)"
echo "launcher=${LAUNCHER} np=${NP} warmup=${WARMUP} iters=${ITERS}"
echo "sizes=${SIZES} (${SIZE_UNIT:-bytes})"
echo "backends=${BACKENDS}"
echo ""

# INPROCESS=1: every (backend, size) in one launch of the ranks (one runtime
# set-up per job instead of one per run); the output lines are the same.
if [[ "${INPROCESS:-0}" == "1" ]]; then
  byte_list=""
  for size in ${SIZES}; do byte_list="${byte_list:+${byte_list},}$(size_to_bytes "${size}")"; done
  if ! launch_ranks "${NP}" -m ring_attention_benchmark_b200.cli sweep comm "${WARMUP}" "${ITERS}" \
      "${byte_list}" "$(echo ${BACKENDS} | tr ' ' ',')"; then
    echo "ERROR: in-process sweep failed"
    exit 1
  fi
  echo "========== Done =========="
  echo "Finished at: $(date)"
  exit 0
fi

for backend in ${BACKENDS}; do
  exe="${BIN_DIR}/ring_loop_${backend}"
  if [[ ! -f "${exe}" ]]; then
    echo "SKIP backend=${backend} (unknown backend)"
    echo ""
    continue
  fi
  echo "===== backend=${backend} ====="
  for size in ${SIZES}; do
    bytes=$(size_to_bytes "${size}")
    if [[ "${RESUME:-0}" == "1" && -n "${RAB_RESULTS_JSONL:-}" ]] &&
      "${RAB_PYTHON}" -m ring_attention_benchmark_b200.utils.results has --kind comm \
        --backend "${backend}" --bytes "${bytes}" --ranks "${NP}" --warmup "${WARMUP}" \
        --iters "${ITERS}"; then
      echo "SKIP backend=${backend} kv_size=${bytes} (already recorded in ${RAB_RESULTS_JSONL})"
      continue
    fi
    echo "--- kv_size=${bytes} bytes ---"
    if ! launch_ranks "${NP}" "${exe}" "${bytes}" "${WARMUP}" "${ITERS}"; then
      echo "ERROR: ${backend} failed with kv_size=${bytes}"
      exit 1
    fi
  done
  echo ""
done

echo "========== Done =========="
echo "Finished at: $(date)"
