#!/bin/bash
# ring_env.sh - shell helpers shared by the benchmark scripts (sourced, not run).
#
#   configure_runtime_env            PATH / LD_LIBRARY_PATH from CUDA_HOME, NCCL_HOME, MPI_HOME
#   detect_world_rank / _size        rank variables set by mpirun, srun, PMI, torchrun
#   under_launcher                   true inside a launched rank (the scripts refuse to run there)
#   source_config_preserving_env F K...  source config F; variables K already set keep their value
#   launch_ranks NP CMD...           start NP ranks of CMD with the selected LAUNCHER
#
# Same precedence rule as the reference's scripts/mpi_env.sh: the environment
# overrides the config file.

RAB_ROOT="${RAB_ROOT:-$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)}"
RAB_PYTHON="${RAB_PYTHON:-$(command -v python3 || command -v python)}"

path_contains() {
  local needle="$1" value="$2" entry=""
  local -a entries=()
  [ -z "${value}" ] && return 1
  IFS=':' read -r -a entries <<< "${value}"
  for entry in "${entries[@]}"; do
    [ "${entry}" = "${needle}" ] && return 0
  done
  return 1
}

prepend_path_var() {
  local var_name="$1" dir="$2"
  local current="${!var_name:-}"
  if [ -z "${dir}" ] || [ ! -d "${dir}" ]; then return 0; fi
  if path_contains "${dir}" "${current}"; then return 0; fi
  if [ -n "${current}" ]; then
    printf -v "${var_name}" '%s:%s' "${dir}" "${current}"
  else
    printf -v "${var_name}" '%s' "${dir}"
  fi
  export "${var_name?}"
}

configure_runtime_env() {
  if [ -n "${CUDA_HOME:-}" ]; then
    prepend_path_var PATH "${CUDA_HOME}/bin"
    prepend_path_var LD_LIBRARY_PATH "${CUDA_HOME}/lib64"
  fi
  if [ -n "${NCCL_HOME:-}" ]; then
    prepend_path_var LD_LIBRARY_PATH "${NCCL_HOME}/lib"
  fi
  if [ -n "${MPI_HOME:-}" ]; then
    prepend_path_var PATH "${MPI_HOME}/bin"
    prepend_path_var LD_LIBRARY_PATH "${MPI_HOME}/lib"
    if [ -z "${MPIRUN:-}" ] && [ -x "${MPI_HOME}/bin/mpirun" ]; then
      MPIRUN="${MPI_HOME}/bin/mpirun"
      export MPIRUN
    fi
  fi
}

detect_world_rank() {
  local v
  for v in "${OMPI_COMM_WORLD_RANK:-}" "${PMIX_RANK:-}" "${PMI_RANK:-}" \
           "${MV2_COMM_WORLD_RANK:-}" "${SLURM_PROCID:-}" "${TORCHELASTIC_RUN_ID:+${RANK:-}}"; do
    if [ -n "${v}" ]; then printf '%s\n' "${v}"; return 0; fi
  done
  return 1
}

detect_world_size() {
  local v
  for v in "${OMPI_COMM_WORLD_SIZE:-}" "${PMIX_SIZE:-}" "${PMI_SIZE:-}" \
           "${MV2_COMM_WORLD_SIZE:-}" "${SLURM_NTASKS:-}"; do
    if [ -n "${v}" ]; then printf '%s\n' "${v}"; return 0; fi
  done
  return 1
}

under_launcher() {
  detect_world_rank >/dev/null 2>&1 || detect_world_size >/dev/null 2>&1
}

source_config_preserving_env() {
  local config_path="$1"
  shift
  [ -f "${config_path}" ] || return 0
  local -a restore=()
  local name quoted
  for name in "$@"; do
    if [ "${!name+x}" = "x" ]; then
      printf -v quoted '%q' "${!name}"
      restore+=("${name}=${quoted}" "export ${name}")
    fi
  done
  set -a
  # shellcheck disable=SC1090
  source "${config_path}"
  set +a
  for name in "${restore[@]}"; do
    eval "${name}"
  done
}

# size_to_bytes SIZE: the programs take a shard size in bytes, as the
# reference's do; with SIZE_UNIT=elements the configured sizes count fp32
# elements instead (the benchmark configs quote them that way), so each is
# multiplied by 4.
size_to_bytes() {
  case "${SIZE_UNIT:-bytes}" in
    bytes) echo "$1" ;;
    elements) echo $(( $1 * 4 )) ;;
    *) echo "ERROR: SIZE_UNIT must be bytes or elements (got ${SIZE_UNIT})" >&2; return 1 ;;
  esac
}

# launch_ranks NP exe args...  (LAUNCHER = local | torchrun | mpirun | srun | none)
launch_ranks() {
  local np="$1"
  shift
  case "${LAUNCHER:-local}" in
    local)
      "${RAB_PYTHON}" -m ring_attention_benchmark_b200.launch -np "${np}" \
        --timeout "${RANK_TIMEOUT:-1800}" "${RAB_PYTHON}" "$@"
      ;;
    torchrun)
      "${RAB_PYTHON}" -m torch.distributed.run --standalone --nnodes=1 \
        --nproc-per-node "${np}" "$@"
      ;;
    mpirun)
      local -a extra=()
      [ -n "${HOSTFILE:-}" ] && extra+=(--hostfile "${HOSTFILE}")
      [ -n "${MPIRUN_EXTRA_ARGS:-}" ] && read -r -a more <<< "${MPIRUN_EXTRA_ARGS}" && extra+=("${more[@]}")
      "${MPIRUN:-mpirun}" "${extra[@]}" -np "${np}" "$@"
      ;;
    srun)
      local -a extra=()
      [ -n "${SRUN_MPI_TYPE:-}" ] && extra+=(--mpi="${SRUN_MPI_TYPE}")
      [ -n "${SRUN_EXTRA_ARGS:-}" ] && read -r -a more <<< "${SRUN_EXTRA_ARGS}" && extra+=("${more[@]}")
      "${SRUN:-srun}" "${extra[@]}" -n "${np}" "$@"
      ;;
    none)
      if [ "${np}" != "1" ]; then
        echo "ERROR: LAUNCHER=none requires NP=1." >&2
        return 1
      fi
      "${RAB_PYTHON}" "$@"
      ;;
    *)
      echo "ERROR: unknown LAUNCHER=${LAUNCHER}. Use local, torchrun, mpirun, srun or none." >&2
      return 1
      ;;
  esac
}
