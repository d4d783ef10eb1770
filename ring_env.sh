#!/bin/bash
# ring_env.sh - shell helpers shared by the benchmark scripts (sourced, not run).
#
#   rab_load_config FILE             apply FILE's KEY=value settings; variables already
#                                    set in the shell or environment keep their value
#   rab_setup_paths                  PATH / LD_LIBRARY_PATH from CUDA_HOME, NCCL_HOME, MPI_HOME
#   rab_inside_launched_rank         true inside a rank started by mpirun, srun, PMI or
#                                    torchrun (the scripts refuse to run there: they
#                                    start the ranks themselves)
#   size_to_bytes SIZE               configured size -> the programs' byte argument
#   launch_ranks NP CMD...           start NP ranks of CMD with the selected LAUNCHER
#
# Precedence is the reference's (scripts/mpi_env.sh): the environment overrides
# the config file.  The file is parsed by utils/config.py, the parser the
# Python tools use, so scripts and tools agree on every value.

RAB_ROOT="${RAB_ROOT:-$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)}"
RAB_PYTHON="${RAB_PYTHON:-$(command -v python3 || command -v python)}"

rab_load_config() {
  local file="$1" key value listing
  [ -f "${file}" ] || return 0
  listing="$("${RAB_PYTHON}" "${RAB_ROOT}/ring_attention_benchmark_b200/utils/config.py" \
    --dump "${file}")" || return 1
  while IFS=$'\t' read -r key value; do
    [ -n "${key}" ] || continue
    # set already (even to an empty string): the shell's value wins
    [ -n "${!key+set}" ] && continue
    declare -gx "${key}=${value}"
  done <<< "${listing}"
}

# _rab_path_add VAR DIR: put DIR in front of the colon list VAR unless it is
# already listed or does not exist.
_rab_path_add() {
  local var="$1" dir="$2" list
  [ -n "${dir}" ] && [ -d "${dir}" ] || return 0
  list="${!var:-}"
  case ":${list}:" in
    *":${dir}:"*) return 0 ;;
  esac
  declare -gx "${var}=${dir}${list:+:${list}}"
}

rab_setup_paths() {
  local home
  for home in "${CUDA_HOME:-}" "${MPI_HOME:-}"; do
    [ -n "${home}" ] && _rab_path_add PATH "${home}/bin"
  done
  [ -n "${CUDA_HOME:-}" ] && _rab_path_add LD_LIBRARY_PATH "${CUDA_HOME}/lib64"
  for home in "${NCCL_HOME:-}" "${MPI_HOME:-}"; do
    [ -n "${home}" ] && _rab_path_add LD_LIBRARY_PATH "${home}/lib"
  done
  if [ -z "${MPIRUN:-}" ] && [ -n "${MPI_HOME:-}" ] && [ -x "${MPI_HOME}/bin/mpirun" ]; then
    declare -gx MPIRUN="${MPI_HOME}/bin/mpirun"
  fi
  return 0
}

# Rank variables exported by the launchers this suite knows (Open MPI, PMIx,
# MPICH/Hydra PMI, MVAPICH2, Slurm); torchrun is recognised by its run id.
_RAB_RANK_VARS=(OMPI_COMM_WORLD_RANK OMPI_COMM_WORLD_SIZE PMIX_RANK PMI_RANK PMI_SIZE
                MV2_COMM_WORLD_RANK SLURM_PROCID TORCHELASTIC_RUN_ID)

rab_inside_launched_rank() {
  local name
  for name in "${_RAB_RANK_VARS[@]}"; do
    [ -n "${!name:-}" ] && return 0
  done
  return 1
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
