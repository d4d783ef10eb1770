"""Interface compatibility with the reference benchmark, on CPU: output-line
grammar (label quirks included), config precedence (environment over file,
SIZES over the per-family lists), the correctness checker's PASS rule and its
oracle mode, and the shell scripts."""
import json
import os
import re
import subprocess
import sys

import numpy as np
import pytest

from ring_attention_benchmark_b200.utils import checker, config, results

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_comm_result_lines_match_reference_grammar():
    avg = {"d2h": 0.027, "mpi": 0.080, "h2d": 0.028, "total": 0.135, "kernel": 0.0}
    line = results.comm_result_line("staged", 262144, 2, 10, 100, avg)
    assert line == ("RESULT backend=staged bytes=262144 ranks=2 warmup=10 iters=100 "
                    "avg_d2h_ms=0.027 avg_mpi_ms=0.080 avg_h2d_ms=0.028 avg_total_ms=0.135 "
                    "total_GBps=1.942 mpi_GBps=3.277")
    assert results.comm_result_line("staged_Isendrecv", 4, 2, 1, 1, avg).startswith(
        "RESULT backend=isendrecv ")
    ca = results.comm_result_line("cuda_aware_Isendrecv", 4, 2, 1, 1, avg)
    assert ca.startswith("RESULT backend=cuda_aware ") and "avg_mpi_ms=" in ca
    nc = results.comm_result_line("nccl", 4, 2, 1, 1, avg)
    assert re.search(r"avg_nccl_ms=\S+ avg_total_ms=\S+ total_GBps=\S+ nccl_GBps=\S+$", nc)
    one = results.comm_result_line("nccl", 4, 1, 1, 1, avg)
    assert "total_GBps=n/a" in one  # one rank: nothing moves


def test_attention_lines():
    avg = {"total": 24.677, "D2H": 0.027, "MPI": 0.080, "H2D": 0.028, "attn": 24.218,
           "merge": 0.079, "final": 0.269}
    assert results.attn_header("staged", 10, 100) == "staged bench: warmup=10 iters=100"
    assert results.attn_result_line("staged", avg) == (
        "avg_total=24.677 ms avg_D2H=0.027 avg_MPI=0.080 avg_H2D=0.028 avg_attn=24.218 "
        "avg_merge=0.079 avg_final=0.269")
    assert results.attn_header("cuda_aware_Isendrecv_overlap", 1, 2) == \
        "CUDA-aware Isendrecv OVERLAP bench: warmup=1 iters=2"
    assert "avg_CUDA-aware=" in results.attn_result_line("cuda_aware_Isendrecv", avg)
    assert "avg_NCCL=" in results.attn_result_line("nccl", avg)


def test_config_precedence(tmp_path):
    f = tmp_path / "benchmark.env"
    f.write_text('# comment\nNP_LIST="2 4"\nexport WARMUP=3\nCOMM_SIZES="1024 2048"\n'
                 "ATTENTION_SIZES=256\n")
    cfg = config.load_config(str(f), env={"WARMUP": "7"})
    assert cfg["NP_LIST"] == "2 4" and cfg["WARMUP"] == "7"
    assert config.sizes_for("comm", cfg) == [1024, 2048]
    assert config.sizes_for("attention", cfg) == [256]
    cfg2 = config.load_config(str(f), env={"SIZES": "4096"})
    assert config.sizes_for("comm", cfg2) == [4096]


def test_checker_rule(tmp_path):
    a = np.linspace(1e4, 7e4, 64, dtype=np.float32)
    b = a * (1 + 5e-6)  # above ABS_TOL but within REL_TOL -> PASS (the reference's OR rule)
    r = checker.compare_arrays([a], [b.astype(np.float32)], 1e-3, 1e-5)
    assert r.passed and r.max_abs > 1e-3
    c = a.copy()
    c[3] += 1.0
    r2 = checker.compare_arrays([a], [c], 1e-3, 1e-5)
    assert not r2.passed
    assert r2.line("x").startswith("x: FAIL elements=64 max_abs_err=")


def test_checker_oracle_mode(tmp_path):
    outs = checker.oracle_outputs(2, 256 * 64 * 4 // 64 * 1)  # 64 tokens per rank
    for r, o in enumerate(outs):
        o.astype("<f4").tofile(tmp_path / f"ring_output_rank{r}.bin")
    assert checker.check_oracle(str(tmp_path), 2, 256 * 64 * 4 // 64).passed
    bad = outs[1].copy()
    bad[0] += 0.1
    bad.astype("<f4").tofile(tmp_path / "ring_output_rank1.bin")
    assert not checker.check_oracle(str(tmp_path), 2, 256 * 64 * 4 // 64).passed


@pytest.mark.parametrize("script", ["benchmark_comm.sh", "benchmark_attention.sh", "run_suite.sh",
                                    "check_attention_correctness.sh", "collect_env.sh",
                                    "ring_env.sh", "launch_local.example.sh",
                                    "launch_mpirun.example.sh", "batch_slurm.example.sh"])
def test_scripts_parse(script):
    r = subprocess.run(["bash", "-n", os.path.join(ROOT, script)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_env_overrides_config_in_shell(tmp_path):
    """rab_load_config: a variable set in the shell (exported or not) or in the
    environment keeps its value; the file fills in the rest, exported; quoted
    values, comments and `export` prefixes parse as in the Python tools."""
    f = tmp_path / "c.env"
    f.write_text('NP=4\nWARMUP=9\n# ITERS=1\nexport BACKENDS="nccl b200_fused"  # two\n'
                 'ITERS=50\nSIZES=\n')
    cmd = (f"source {ROOT}/ring_env.sh; NP=2; SIZES=7; "
           f"rab_load_config {f}; echo $NP $WARMUP $ITERS $SIZES; echo $BACKENDS; "
           "bash -c 'echo $WARMUP'")
    env = dict(os.environ, ITERS="3")
    env.pop("WARMUP", None)
    r = subprocess.run(["bash", "-c", cmd], capture_output=True, text=True, env=env)
    lines = r.stdout.splitlines()
    assert lines[0].split() == ["2", "9", "3", "7"], r.stderr
    assert lines[1] == "nccl b200_fused"
    assert lines[2] == "9"  # exported to child processes
    from ring_attention_benchmark_b200.utils.config import load_config
    cfg = load_config(str(f), env={"NP": "2", "ITERS": "3"})
    assert (cfg["NP"], cfg["WARMUP"], cfg["ITERS"], cfg["BACKENDS"]) == ("2", "9", "3",
                                                                         "nccl b200_fused")


def test_path_setup_prepends_once(tmp_path):
    home = tmp_path / "cuda"
    (home / "bin").mkdir(parents=True)
    (home / "lib64").mkdir()
    cmd = (f"source {ROOT}/ring_env.sh; export CUDA_HOME={home}; PATH=/usr/bin:/bin; "
           "LD_LIBRARY_PATH=; rab_setup_paths; rab_setup_paths; echo $PATH; echo $LD_LIBRARY_PATH")
    r = subprocess.run(["bash", "-c", cmd], capture_output=True, text=True)
    path, ld = r.stdout.splitlines()
    assert path == f"{home}/bin:/usr/bin:/bin"
    assert ld == f"{home}/lib64"


def test_size_unit_conversion():
    """SIZE_UNIT=elements turns configured fp32 element counts into the byte
    sizes the programs take; bytes (the default) passes them through."""
    def conv(unit, size):
        env = dict(os.environ)
        env.pop("SIZE_UNIT", None)
        if unit is not None:
            env["SIZE_UNIT"] = unit
        return subprocess.run(["bash", "-c", f"source ./ring_env.sh && size_to_bytes {size}"],
                              cwd=ROOT, env=env, capture_output=True, text=True)
    assert conv(None, 262144).stdout.strip() == "262144"
    assert conv("bytes", 1048576).stdout.strip() == "1048576"
    assert conv("elements", 262144).stdout.strip() == "1048576"
    bad = conv("words", 16)
    assert bad.returncode != 0 and "SIZE_UNIT" in bad.stderr


def test_wrappers_refuse_inside_a_launched_rank():
    env = dict(os.environ, OMPI_COMM_WORLD_RANK="0")
    r = subprocess.run([os.path.join(ROOT, "benchmark_comm.sh")], env=env, capture_output=True,
                       text=True, cwd=ROOT)
    assert r.returncode == 1 and "normal shell" in r.stderr


def test_run_suite_prepares_run_dir(tmp_path):
    env = dict(os.environ, BUILD="0", COLLECT_ENV="0", RESULTS_ROOT=str(tmp_path), RUN_LABEL="t",
               NP_LIST="1 2")
    r = subprocess.run([os.path.join(ROOT, "run_suite.sh")], env=env, capture_output=True,
                       text=True, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    for name in ("manifest.txt", "run_context.env", "launch_examples.txt"):
        assert (tmp_path / "t" / name).is_file()
    ex = (tmp_path / "t" / "launch_examples.txt").read_text()
    assert 'NP="2"' in ex and "benchmark_attention.sh" in ex and 'LAUNCHER="torchrun"' in ex


def test_bin_programs_exist_for_every_backend():
    for b in ("staged", "staged_Isendrecv", "cuda_aware", "cuda_aware_Isendrecv", "nccl",
              "b200_fused"):
        assert os.access(os.path.join(ROOT, "bin", f"ring_loop_{b}"), os.X_OK)
    for b in ("staged", "staged_Isendrecv", "staged_Isendrecv_overlap", "cuda_aware",
              "cuda_aware_Isendrecv", "cuda_aware_Isendrecv_overlap", "nccl", "b200_fused"):
        assert os.access(os.path.join(ROOT, "bin", f"ring_attention_{b}_gpu_bench"), os.X_OK)


def test_cli_argument_validation():
    from ring_attention_benchmark_b200 import cli

    assert cli.comm_main("nccl", []) == 1          # missing size (reference: usage, exit 1)
    assert cli.comm_main("nccl", ["6"]) == 1       # not a multiple of 4
    assert cli.attention_main("nccl", ["300"]) == 1  # not a multiple of 256
    assert cli.comm_main("nope", ["4"]) == 1


def test_resume_skips_recorded_configurations(tmp_path):
    """RESUME=1: a configuration already in RAB_RESULTS_JSONL is skipped without
    launching any rank; an unrecorded one is not."""
    from ring_attention_benchmark_b200.utils import results

    jl = tmp_path / "r.jsonl"
    rec = {"kind": "comm", "backend": "staged", "bytes": 4096, "ranks": 2, "warmup": 1,
           "iters": 2, "avg_ms": {}}
    jl.write_text(json.dumps(rec) + "\nnot json\n")
    assert results.has_record(str(jl), kind="comm", backend="staged", bytes=4096, ranks=2,
                              warmup=1, iters=2)
    assert not results.has_record(str(jl), kind="comm", backend="staged", bytes=8192, ranks=2,
                                  warmup=1, iters=2)
    env = dict(os.environ, RESUME="1", RAB_RESULTS_JSONL=str(jl), NP="2", WARMUP="1",
               ITERS="2", SIZES="4096", BACKENDS="staged", LAUNCHER="none",
               CONFIG=str(tmp_path / "none.env"))
    for k in ("OMPI_COMM_WORLD_RANK", "PMI_RANK", "SLURM_PROCID", "RANK", "SIZE_UNIT"):
        env.pop(k, None)
    r = subprocess.run([os.path.join(ROOT, "benchmark_comm.sh")], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "SKIP backend=staged kv_size=4096" in r.stdout and "--- kv_size" not in r.stdout


def test_sweep_table_from_jsonl():
    """`results table` turns a sweep's JSONL records into one markdown row per
    (ranks, backend) and one column per size."""
    from ring_attention_benchmark_b200.utils.results import sweep_table

    recs = [{"kind": "comm", "backend": "nccl", "bytes": 1 << 20, "ranks": 2,
             "avg_ms": {"total": 0.01}},
            {"kind": "comm", "backend": "b200_fused", "bytes": 1 << 20, "ranks": 2,
             "avg_ms": {"total": 0.005, "kernel": 0.004}},
            {"kind": "comm", "backend": "nccl", "bytes": 1 << 24, "ranks": 4,
             "avg_ms": {"total": 0.1}},
            {"kind": "attention", "backend": "nccl", "bytes": 262144, "ranks": 2,
             "avg_ms": {"total": 0.5}, "tflops": 1.2}]
    t = sweep_table(recs, "comm").splitlines()
    assert "| np | backend | 1048576 | 16777216 |" in t
    assert "| 2 | b200_fused | 209.7 (262.1) |  |" in t  # device-timed kernel GB/s in brackets
    assert "| 4 | nccl |  | 503.3 |" in t
    assert "| 2 | nccl | 0.500 ms / 1.20 |" in sweep_table(recs, "attention")


def test_sweep_program_rejects_bad_arguments():
    r = subprocess.run([sys.executable, "-m", "ring_attention_benchmark_b200.cli", "sweep",
                        "attention", "1", "1", "100", "nccl"], cwd=ROOT, capture_output=True,
                       text=True)
    assert r.returncode == 1 and "bad arguments" in r.stdout
