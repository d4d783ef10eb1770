#!/bin/bash
# check_attention_correctness.sh - run attention backends with output dumps and
# compare them (counterpart of the reference's check_attention_correctness.sh:114-178,
# PASS rule at :166).
#
# Pairs compared with the reference's rule (PASS if max_abs_err <= ABS_TOL or
# max_rel_err <= REL_TOL): the reference's two pairs (staged_Isendrecv vs its
# overlap twin, cuda_aware_Isendrecv vs its overlap twin) plus nccl vs
# b200_fused.  With ORACLE=1 (default) every dumped backend is also checked
# against the float64 ring oracle, which the reference checker lacks.
# Keys: NP SIZE WARMUP ITERS BUILD ABS_TOL REL_TOL ORACLE LAUNCHER RUN_LABEL
# RESULTS_ROOT RAB_DATA RAB_PREC.
set -euo pipefail

SCRIPT_DIR="$(cd "$(dirname "$0")" && pwd)"
cd "${SCRIPT_DIR}"
# shellcheck disable=SC1091
source "${SCRIPT_DIR}/ring_env.sh"

CONFIG=${CONFIG:-benchmark.env}
rab_load_config "${CONFIG}"
rab_setup_paths

if rab_inside_launched_rank; then
  echo "ERROR: check_attention_correctness.sh should be run from a normal shell." >&2
  exit 1
fi

NP=${NP:-2}
SIZE=${SIZE:-262144}
WARMUP=${WARMUP:-1}
ITERS=${ITERS:-1}
BUILD=${BUILD:-1}
ABS_TOL=${ABS_TOL:-1e-3}
REL_TOL=${REL_TOL:-1e-5}
ORACLE=${ORACLE:-1}
LAUNCHER=${LAUNCHER:-local}
RAB_DATA=${RAB_DATA:-normal}
export LAUNCHER RAB_DATA RAB_PREC 2>/dev/null || true
RESULTS_ROOT=${RESULTS_ROOT:-"${SCRIPT_DIR}/results"}
RUN_LABEL=${RUN_LABEL:-"correctness_$(hostname)_$(date +%Y%m%d_%H%M%S)"}
RUN_DIR="${RESULTS_ROOT}/${RUN_LABEL}"
CHECK_DIR="${RUN_DIR}/attention_correctness_np${NP}_size${SIZE}"
mkdir -p "${CHECK_DIR}"

status=0

run_dump() {
  local backend="$1" dest="$2"
  rm -f ring_output_rank*.bin
  echo "--- ${backend} ---"
  ATTENTION_DUMP_OUTPUT=1 launch_ranks "${NP}" \
    "${SCRIPT_DIR}/bin/ring_attention_${backend}_gpu_bench" "${SIZE}" "${WARMUP}" "${ITERS}"
  mkdir -p "${dest}"
  local r
  for ((r = 0; r < NP; r++)); do
    mv "ring_output_rank${r}.bin" "${dest}/ring_output_rank${r}.bin"
  done
}

compare() {
  "${RAB_PYTHON}" -m ring_attention_benchmark_b200.utils.checker compare "$@" \
    "${NP}" "${ABS_TOL}" "${REL_TOL}" || status=1
}

oracle() {
  "${RAB_PYTHON}" -m ring_attention_benchmark_b200.utils.checker oracle "$1" "$2" "${NP}" \
    "${SIZE}" "${ABS_TOL}" "${REL_TOL}" --data "${RAB_DATA}" || status=1
}

run_pair() {
  local label="$1" base="$2" other="$3"
  echo ""
  echo "===== correctness pair=${label} ====="
  run_dump "${base}" "${CHECK_DIR}/${label}_baseline"
  run_dump "${other}" "${CHECK_DIR}/${label}_overlap"
  compare "${label}" "${CHECK_DIR}/${label}_baseline" "${CHECK_DIR}/${label}_overlap"
  if [ "${ORACLE}" = "1" ]; then
    oracle "${base}_vs_oracle" "${CHECK_DIR}/${label}_baseline"
    oracle "${other}_vs_oracle" "${CHECK_DIR}/${label}_overlap"
  fi
}

echo "========== Attention Correctness Check =========="
echo "Date: $(date)"
echo "Hostname: $(hostname)"
echo "launcher=${LAUNCHER} np=${NP} size=${SIZE} warmup=${WARMUP} iters=${ITERS} data=${RAB_DATA}"
echo "abs_tol=${ABS_TOL} rel_tol=${REL_TOL} oracle=${ORACLE}"
echo "results=${CHECK_DIR}"

if [ "${BUILD}" = "1" ]; then
  make -s build
fi

run_pair "staged_Isendrecv_vs_overlap" staged_Isendrecv staged_Isendrecv_overlap
run_pair "cuda_aware_Isendrecv_vs_overlap" cuda_aware_Isendrecv cuda_aware_Isendrecv_overlap
run_pair "nccl_vs_b200_fused" nccl b200_fused

rm -f ring_output_rank*.bin
echo ""
echo "========== Correctness Check Done =========="
exit "${status}"
