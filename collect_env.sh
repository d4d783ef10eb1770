#!/bin/bash
# collect_env.sh - record the machine, driver, toolchain and library versions a
# result was measured with (counterpart of the reference's collect_env.sh:23-147).
# Read-only: nothing on the GPUs is changed.
set -uo pipefail

section() { echo ""; echo "===== $* ====="; }

section "host"
echo "hostname: $(hostname)"
echo "date: $(date)"
uname -a
[ -r /etc/os-release ] && grep -E '^(NAME|VERSION)=' /etc/os-release

section "cpu / memory"
lscpu 2>/dev/null | grep -E 'Model name|Socket|Core|Thread|NUMA' || true
free -g 2>/dev/null || true

section "gpus"
if command -v nvidia-smi >/dev/null 2>&1; then
  nvidia-smi --query-gpu=index,name,uuid,driver_version,memory.total,clocks.max.sm,power.limit --format=csv
  section "gpu topology"
  nvidia-smi topo -m 2>/dev/null || true
  section "nvlink"
  nvidia-smi nvlink -s 2>/dev/null | head -40 || true
else
  echo "nvidia-smi not found"
fi

section "toolchain"
command -v nvcc >/dev/null 2>&1 && nvcc --version | tail -2
gcc --version 2>/dev/null | head -1
PY="${RAB_PYTHON:-$(command -v python3 || command -v python)}"
"${PY}" - <<'PY'
import platform
print("python", platform.python_version())
try:
    import torch
    print("torch", torch.__version__, "cuda", torch.version.cuda)
    print("nccl (torch)", ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else "n/a")
    print("cuda available", torch.cuda.is_available(), "devices", torch.cuda.device_count())
except Exception as e:  # noqa: BLE001
    print("torch unavailable:", e)
try:
    import ring_attention_benchmark_b200 as r
    print("ring_attention_benchmark_b200", r.__version__, "extension built:", r.extension_available())
except Exception as e:  # noqa: BLE001
    print("package import failed:", e)
PY

section "mpi (optional)"
if command -v mpirun >/dev/null 2>&1; then
  mpirun --version 2>&1 | head -2
  command -v ompi_info >/dev/null 2>&1 && ompi_info --parsable --all 2>/dev/null | grep -i 'mpi_built_with_cuda_support' || true
else
  echo "mpirun not found (not needed: LAUNCHER=local/torchrun)"
fi

section "environment"
env | grep -E '^(CUDA|NCCL|RAB_|LAUNCHER|NP|WARMUP|ITERS|OMPI_|SLURM_|MASTER_)' | sort || true
