"""CPU: the device-timed v0/v1 runner (kernelswift_b200.ab_runner) loads
modules the way auto_bench does, copies the state dict, compares outputs and
times both sides (host clock on the CPU)."""
from pathlib import Path

import pytest
import torch

from conftest import reference_file

from kernelswift_b200 import ab_runner

V0 = '''
import torch
import torch.nn as nn
SHAPE = (7, 5)
unused = torch.zeros(3)          # not a literal: dropped by the filter


class Model(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.w = nn.Parameter(torch.randn(n, n))

    def forward(self, x):
        return x @ self.w, torch.argmax(x, dim=-1)


def get_inputs():
    return [torch.randn(*SHAPE, device="cuda")]


def get_init_inputs():
    return [5]
'''

V1_SAME = V0.replace("class Model(", "class ModelNew(")
V1_OFF = V1_SAME.replace("return x @ self.w,", "return x @ self.w + 1.0,")


def test_runner_matches_and_times(tmp_path):
    (tmp_path / "v0.py").write_text(V0)
    (tmp_path / "v1.py").write_text(V1_SAME)
    r = ab_runner.run(tmp_path / "v0.py", tmp_path / "v1.py", device="cpu", warmup=1, repeat=3)
    assert r["match"] and r["differences"] == []
    assert r["v0_ms"] > 0 and r["v1_ms"] > 0 and r["speedup"] > 0


def test_runner_reports_differences(tmp_path):
    (tmp_path / "v0.py").write_text(V0)
    (tmp_path / "v1.py").write_text(V1_OFF)
    r = ab_runner.run(tmp_path / "v0.py", tmp_path / "v1.py", device="cpu", warmup=0, repeat=1)
    assert not r["match"] and "output[0]" in r["differences"][0]


def test_filter_drops_non_literal_globals(tmp_path):
    (tmp_path / "v0.py").write_text(V0)
    mod = ab_runner.load_module(tmp_path / "v0.py", "filtered")
    assert mod.SHAPE == (7, 5) and not hasattr(mod, "unused")


def test_compare_semantics():
    a = torch.tensor([1.0, 2.0])
    assert ab_runner.compare(a, a + 5e-3, 1e-2, 1e-2) == []
    assert ab_runner.compare(a, a + 1.0, 1e-2, 1e-2)
    assert ab_runner.compare(torch.tensor([1, 2]), torch.tensor([1, 3]), 1e-2, 1e-2)
    assert ab_runner.compare((a, [a]), (a, [a]), 0, 0) == []
    assert ab_runner.compare(a, a[:1], 1e-2, 1e-2)


def test_loads_the_reference_operator_module():
    """fused_moe/base.py under the filter, with the torch_mlu stub: its Model
    builds and runs on the CPU."""
    ref = reference_file("kernels/track1-triton/fused_moe/base.py")
    mod = ab_runner.load_module(ref, "ref_fused_moe")
    m = mod.Model(*mod.get_init_inputs())
    x = ab_runner._cpu_inputs(mod)
    with torch.no_grad():
        out = m(*x)
    assert out.shape == x[0].shape
