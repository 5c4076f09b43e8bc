"""CPU: bench.py's host-side pieces the benchmark contract rests on: the
workload table, the config block of the JSON line, the CPU baseline's host
memory cap, the switch record, and the reference arm's JSON line (run on a
tiny sample so it finishes in seconds)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_workloads_cover_the_configs():
    names = set(bench.WORKLOADS)
    assert {"mixtral", "qwen3", "dsv3", "dsv3-fp8", "qwen3-int8"} <= names
    H, I, E, k, quant, T, bias = bench.WORKLOADS["mixtral"]
    assert (H, I, E, k, quant, T) == (4096, 14336, 8, 2, "none", 4096)
    assert bench.WORKLOADS["dsv3-fp8"][4] == "fp8" and bench.WORKLOADS["qwen3"][6] > 0
    # the CPU-runnable configuration, fp32 activations
    assert bench.WORKLOADS["cfg0"][:6] == (512, 1024, 8, 2, "none", 64)
    assert bench.FP32_WORKLOADS == {"cfg0"} and bench.act_dtype_name("cfg0") == "f32"


def test_reference_arm_fp32_configuration():
    """--impl reference on the fp32 configuration times base.py's path in fp32."""
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--workload", "cfg0", "--steps", "1", "--warmup", "0"],
                         capture_output=True, text=True, timeout=600, cwd=str(ROOT),
                         env=dict(os.environ, OMP_NUM_THREADS="4"))
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["dtype"] == "f32" and "f32" in line["config"]["workload"]
    assert "torch-CPU f32" in line["cpu_baseline"]["sample"] and line["value"] > 0


def test_config_block():
    cfg = bench.workload_config("mixtral", 4096, 14336, 8, 2, "none", 4096, 1)
    assert cfg["parallelism"] == "single" and cfg["tokens_per_gpu"] == 4096
    assert "flushed" in cfg["l2"] and set(cfg["switches"]) >= {"pdl", "decode_path", "tail_halves",
                                                             "token_gather", "block_n"}
    ep = bench.workload_config("mixtral", 4096, 14336, 8, 2, "none", 4096, 8, "peer")
    assert ep["global_tokens"] == 8 * 4096 and "peer memory" in ep["parallelism"]
    dd = bench.workload_config("dsv3", 7168, 2048, 256, 8, "none", 8192, 4, "nccl-dedup")
    assert "one row per token and destination rank" in dd["parallelism"]
    assert "chunks" not in dd["parallelism"]
    ch = bench.workload_config("dsv3", 7168, 2048, 256, 8, "none", 8192, 4, "nccl-dedup", 3)
    assert "pipelined in 3 token chunks" in ch["parallelism"]


def test_cpu_baseline_memory_cap():
    # Mixtral's masters fit; DeepSeek-V3's 256 experts do not
    assert bench.cpu_experts(4096, 14336, 8, 2) == 8
    sub = bench.cpu_experts(7168, 2048, 256, 8)
    assert 8 <= sub < 256
    assert sub * 1.5 * 12 * 7168 * 2048 <= bench.CPU_WEIGHT_BUDGET
    assert bench.cpu_expert_note(4096, 14336, 8, 2) == ""
    assert "upper bound" in bench.cpu_expert_note(7168, 2048, 256, 8)


def test_switch_record(monkeypatch):
    for name in ("MOE_NO_PDL", "MOE_NO_DECODE_PATH", "MOE_NO_TAIL_HALVES",
                 "MOE_NO_TOKEN_GATHER", "MOE_BLOCK_N"):
        monkeypatch.delenv(name, raising=False)
    assert bench.active_switches() == {"pdl": True, "decode_path": True, "tail_halves": True,
                                       "token_gather": True, "block_n": "planner"}
    monkeypatch.setenv("MOE_NO_PDL", "1")
    monkeypatch.setenv("MOE_NO_DECODE_PATH", "0")
    monkeypatch.setenv("MOE_NO_TOKEN_GATHER", "1")
    monkeypatch.setenv("MOE_BLOCK_N", "128")
    sw = bench.active_switches()
    assert not sw["pdl"] and sw["decode_path"] and sw["block_n"] == "128"
    assert sw["tail_halves"] and not sw["token_gather"]


def test_reference_arm_json_line():
    """--impl reference prints one JSON line with the contract's keys (the
    reference's CPU path on the qwen3 layer, a small token count)."""
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--workload", "qwen3", "--tokens", "16", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600,
                         cwd=str(ROOT), env=dict(os.environ, OMP_NUM_THREADS="4"))
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"


def test_cpu_sample_is_fixed_per_workload():
    """Both CPU legs (cpu_baseline and --impl reference) time the same fixed
    batch of each workload, capped at the GPU batch."""
    assert set(bench.CPU_SAMPLE_TOKENS) == set(bench.WORKLOADS)
    for name, (_, _, _, _, _, T, _) in bench.WORKLOADS.items():
        n = bench.cpu_sample_tokens(name, T)
        assert 1 <= n <= T and n == bench.cpu_sample_tokens(name, T)
    assert bench.cpu_sample_tokens("mixtral", 64) == 64
    assert isinstance(bench.cpu_model(), str) and bench.cpu_model()
