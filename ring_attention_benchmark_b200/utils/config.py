"""``benchmark.env`` handling for Python tools.

Precedence: a variable already set in the environment wins over the file,
the rule of the reference's ``scripts/mpi_env.sh`` (lines 126-153).  This
module is the one parser of the ``KEY=value`` syntax (optional quotes, ``#``
comments, ``export`` prefix; the file is parsed, never executed): Python tools
call `load_config`, and the shell scripts' ``rab_load_config`` (in
``ring_env.sh``) reads the file through ``config.py --dump`` and applies the
same rule, so both see the same values.

Size lists: the reference's wrappers read ``SIZES`` only, so ``COMM_SIZES`` /
``ATTENTION_SIZES`` from the config never reached them
(``benchmark_comm.sh`` lines 12 and 24).  Here ``SIZES`` overrides when given,
otherwise the per-family list is used.
"""
from __future__ import annotations

import os
import shlex
from typing import Dict, Iterable, List, Mapping, Optional

DEFAULTS: Dict[str, str] = {
    "NP_LIST": "2 4 8",
    "WARMUP": "10",
    "ITERS": "100",
    "BACKENDS": "staged staged_Isendrecv cuda_aware cuda_aware_Isendrecv nccl b200_fused",
    "ATTENTION_BACKENDS": ("staged staged_Isendrecv staged_Isendrecv_overlap cuda_aware "
                           "cuda_aware_Isendrecv cuda_aware_Isendrecv_overlap nccl b200_fused"),
    "RUN_TYPES": "comm attention",
    "COMM_SIZES": "262144 524288 1048576 4194304 16777216",
    "ATTENTION_SIZES": "262144 524288 1048576",
    "LAUNCHER": "local",
    "BUILD": "1",
    "COLLECT_ENV": "1",
}


def parse_env_file(path: str) -> Dict[str, str]:
    """Parse shell-style ``KEY=value`` lines (no command substitution)."""
    out: Dict[str, str] = {}
    if not os.path.isfile(path):
        return out
    with open(path) as f:
        for raw in f:
            line = raw.strip()
            if not line or line.startswith("#"):
                continue
            if line.startswith("export "):
                line = line[len("export "):].strip()
            if "=" not in line:
                continue
            key, _, val = line.partition("=")
            key = key.strip()
            if not key.replace("_", "").isalnum():
                continue
            try:
                parts = shlex.split(val, comments=True)
            except ValueError:
                parts = [val]
            out[key] = " ".join(parts)
    return out


def load_config(path: Optional[str] = None, env: Optional[Mapping[str, str]] = None,
                keys: Optional[Iterable[str]] = None) -> Dict[str, str]:
    """Defaults < config file < environment (for `keys`, default: all known)."""
    env = os.environ if env is None else env
    path = path or env.get("CONFIG", "benchmark.env")
    cfg = dict(DEFAULTS)
    cfg.update(parse_env_file(path))
    for k in (keys or set(cfg) | set(DEFAULTS) | {"SIZES", "NP", "CONFIG"}):
        if k in env:
            cfg[k] = env[k]
    return cfg


def sizes_for(run_type: str, cfg: Mapping[str, str]) -> List[int]:
    if cfg.get("SIZES"):
        return [int(s) for s in cfg["SIZES"].split()]
    key = "COMM_SIZES" if run_type == "comm" else "ATTENTION_SIZES"
    return [int(s) for s in cfg.get(key, DEFAULTS[key]).split()]


def _main(argv: List[str]) -> int:
    """``python config.py --dump FILE``: one ``KEY<TAB>value`` line per key of
    FILE, for ``rab_load_config`` in ``ring_env.sh`` (run as a plain script, so
    no package or torch import happens)."""
    import sys

    if len(argv) != 2 or argv[0] != "--dump":
        print("usage: config.py --dump FILE", file=sys.stderr)
        return 2
    for key, val in parse_env_file(argv[1]).items():
        if "\t" in val or "\n" in val:
            print(f"config.py: {key}: tabs and newlines are not supported in values",
                  file=sys.stderr)
            return 1
        print(f"{key}\t{val}")
    return 0


if __name__ == "__main__":
    import sys

    sys.exit(_main(sys.argv[1:]))
