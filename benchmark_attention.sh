#!/bin/bash
# benchmark_attention.sh - ring attention benchmark over backends and sizes
# (counterpart of the reference's benchmark_attention.sh, backend loop :109-131).
#
# Env / benchmark.env keys: NP WARMUP ITERS SIZES ATTENTION_SIZES ATTENTION_BACKENDS LAUNCHER
# (local | torchrun | mpirun | srun | none) MPIRUN HOSTFILE MPIRUN_EXTRA_ARGS SRUN
# SRUN_MPI_TYPE SRUN_EXTRA_ARGS, plus RAB_DATA (normal | ref_compat), RAB_PREC (fp32 |
# bf16), RAB_KERNEL (tcgen05 | simt), RAB_RING_MODE (direct | chain).  SIZES
# overrides ATTENTION_SIZES; SIZE_UNIT=elements reads the sizes as fp32 element counts
# (default bytes).  RESUME=1 with
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
  echo "ERROR: benchmark_attention.sh should be run from a normal shell; it launches the ranks itself." >&2
  exit 1
fi

NP=${NP:-2}
WARMUP=${WARMUP:-10}
ITERS=${ITERS:-100}
export RAB_DATA RAB_PREC RAB_KERNEL RAB_RING_MODE 2>/dev/null || true
ATTENTION_SIZES=${ATTENTION_SIZES:-"262144 524288 1048576"}
SIZES=${SIZES:-${ATTENTION_SIZES}}
ATTENTION_BACKENDS=${ATTENTION_BACKENDS:-"staged staged_Isendrecv staged_Isendrecv_overlap cuda_aware cuda_aware_Isendrecv cuda_aware_Isendrecv_overlap nccl b200_fused"}
LAUNCHER=${LAUNCHER:-local}
export LAUNCHER MPIRUN HOSTFILE MPIRUN_EXTRA_ARGS SRUN SRUN_MPI_TYPE SRUN_EXTRA_ARGS

BIN_DIR="${SCRIPT_DIR}/bin"

echo "========== Ring Attention Benchmark =========="
echo "Date: $(date)"
echo "Hostname: $(hostname)"
echo "launcher=${LAUNCHER} np=${NP} warmup=${WARMUP} iters=${ITERS}"
echo "sizes=${SIZES} (${SIZE_UNIT:-bytes})"
echo "attention_backends=${ATTENTION_BACKENDS}"
echo ""

# INPROCESS=1: every (backend, size) in one launch of the ranks (one runtime
# set-up per job instead of one per run); the output lines are the same.
if [[ "${INPROCESS:-0}" == "1" ]]; then
  byte_list=""
  for size in ${SIZES}; do byte_list="${byte_list:+${byte_list},}$(size_to_bytes "${size}")"; done
  if ! launch_ranks "${NP}" -m ring_attention_benchmark_b200.cli sweep attention "${WARMUP}" "${ITERS}" \
      "${byte_list}" "$(echo ${ATTENTION_BACKENDS} | tr ' ' ',')"; then
    echo "ERROR: in-process sweep failed"
    exit 1
  fi
  echo "========== Done =========="
  echo "Finished at: $(date)"
  exit 0
fi

for backend in ${ATTENTION_BACKENDS}; do
  exe="${BIN_DIR}/ring_attention_${backend}_gpu_bench"
  if [[ ! -f "${exe}" ]]; then
    echo "SKIP backend=${backend} (unknown backend)"
    echo ""
    continue
  fi
  echo "===== backend=${backend} ====="
  for size in ${SIZES}; do
    bytes=$(size_to_bytes "${size}")
    if [[ "${RESUME:-0}" == "1" && -n "${RAB_RESULTS_JSONL:-}" ]] &&
      "${RAB_PYTHON}" -m ring_attention_benchmark_b200.utils.results has --kind attention \
        --backend "${backend}" --bytes "${bytes}" --ranks "${NP}" --warmup "${WARMUP}" \
        --iters "${ITERS}" --prec "${RAB_PREC:-fp32}" --data "${RAB_DATA:-normal}"; then
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
