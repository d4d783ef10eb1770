#!/bin/bash
# run_suite.sh - preparation only: create results/<label>/, write the manifest,
# run context and launch examples, build the extension and collect the
# environment.  The benchmarks are then started with the example lines.
set -euo pipefail

SCRIPT_DIR="$(cd "$(dirname "$0")" && pwd)"
cd "${SCRIPT_DIR}"
# shellcheck disable=SC1091
source "${SCRIPT_DIR}/ring_env.sh"

CONFIG=${CONFIG:-benchmark.env}
rab_load_config "${CONFIG}"
rab_setup_paths

RUN_LABEL=${RUN_LABEL:-"$(hostname)_$(date +%Y%m%d_%H%M%S)"}
RESULTS_ROOT=${RESULTS_ROOT:-"${SCRIPT_DIR}/results"}
RUN_DIR="${RESULTS_ROOT}/${RUN_LABEL}"
NP_LIST=${NP_LIST:-"1 2 4 8"}
RUN_TYPES=${RUN_TYPES:-"comm attention"}
WARMUP=${WARMUP:-10}
ITERS=${ITERS:-100}
BACKENDS=${BACKENDS:-"staged staged_Isendrecv cuda_aware cuda_aware_Isendrecv nccl b200_fused"}
ATTENTION_BACKENDS=${ATTENTION_BACKENDS:-"staged staged_Isendrecv staged_Isendrecv_overlap cuda_aware cuda_aware_Isendrecv cuda_aware_Isendrecv_overlap nccl b200_fused"}
COMM_SIZES=${COMM_SIZES:-"262144 524288 1048576 4194304 16777216"}
ATTENTION_SIZES=${ATTENTION_SIZES:-"262144 524288 1048576"}
BUILD=${BUILD:-1}
COLLECT_ENV=${COLLECT_ENV:-1}
LAUNCHER=${LAUNCHER:-local}

if [[ "${CONFIG}" = /* ]]; then CONFIG_PATH="${CONFIG}"; else CONFIG_PATH="${SCRIPT_DIR}/${CONFIG}"; fi

write_manifest() {
  cat > "${RUN_DIR}/manifest.txt" <<MAN
run_label=${RUN_LABEL}
date=$(date)
hostname=$(hostname)
script_dir=${SCRIPT_DIR}
execution_model=external_launcher
config=${CONFIG}
results_root=${RESULTS_ROOT}
run_dir=${RUN_DIR}
np_list=${NP_LIST}
run_types=${RUN_TYPES}
warmup=${WARMUP}
iters=${ITERS}
backends=${BACKENDS}
attention_backends=${ATTENTION_BACKENDS}
comm_sizes=${COMM_SIZES}
attention_sizes=${ATTENTION_SIZES}
size_unit=${SIZE_UNIT:-bytes}
build=${BUILD}
collect_env=${COLLECT_ENV}
launcher=${LAUNCHER}
rab_data=${RAB_DATA:-normal}
rab_prec=${RAB_PREC:-fp32}
MAN
}

write_run_context() {
  cat > "${RUN_DIR}/run_context.env" <<CTX
RUN_LABEL="${RUN_LABEL}"
RESULTS_ROOT="${RESULTS_ROOT}"
RUN_DIR="${RUN_DIR}"
CONFIG="${CONFIG}"
NP_LIST="${NP_LIST}"
RUN_TYPES="${RUN_TYPES}"
BACKENDS="${BACKENDS}"
ATTENTION_BACKENDS="${ATTENTION_BACKENDS}"
COMM_SIZES="${COMM_SIZES}"
ATTENTION_SIZES="${ATTENTION_SIZES}"
SIZE_UNIT="${SIZE_UNIT:-bytes}"
CTX
}

write_launch_examples() {
  # results go to the run directory's JSONL file; RESUME=1 makes a rerun skip what it records
  local prefix="env CONFIG=\"${CONFIG_PATH}\" RUN_LABEL=\"${RUN_LABEL}\" RESULTS_ROOT=\"${RESULTS_ROOT}\" RAB_RESULTS_JSONL=\"${RUN_DIR}/results.jsonl\""
  {
    echo "# Ring attention benchmark launch examples"
    echo "# Preparation already created: ${RUN_DIR}"
    for launcher in local torchrun mpirun srun; do
      echo ""
      echo "# LAUNCHER=${launcher}"
      for np in ${NP_LIST}; do
        for run_type in ${RUN_TYPES}; do
          case "${run_type}" in
            comm) script=benchmark_comm.sh ;;
            attention) script=benchmark_attention.sh ;;
            *) continue ;;
          esac
          echo "${prefix} LAUNCHER=\"${launcher}\" NP=\"${np}\" \"${SCRIPT_DIR}/${script}\" > \"${RUN_DIR}/${run_type}_np${np}.log\" 2>&1"
        done
      done
    done
  } > "${RUN_DIR}/launch_examples.txt"
}

if rab_inside_launched_rank; then
  echo "ERROR: run_suite.sh is preparation-only; run it from a normal shell." >&2
  exit 1
fi

mkdir -p "${RUN_DIR}"
write_manifest
write_run_context
write_launch_examples
echo "Results directory: ${RUN_DIR}"
if [ "${BUILD}" = "1" ]; then
  echo "Building the native extension..."
  make -s build 2>&1 | tee "${RUN_DIR}/build.log"
else
  echo "Skipping build because BUILD=${BUILD}."
fi
if [ "${COLLECT_ENV}" = "1" ]; then
  echo "Collecting local environment..."
  ./collect_env.sh > "${RUN_DIR}/env_local.txt" 2>&1 || true
fi
echo "Preparation complete."
echo "Launch the benchmarks with the lines in ${RUN_DIR}/launch_examples.txt"
