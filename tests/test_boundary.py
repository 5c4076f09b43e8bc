"""CPU tests of the drop-in boundary: the auto_bench v1 module survives the
harness's AST filter, and ModelNew keeps base.py's contract."""
import ast
import importlib.util
from pathlib import Path

import pytest

from conftest import reference_file

ROOT = Path(__file__).resolve().parent.parent
V1 = ROOT / "kernelswift_b200" / "ks_fused_moe.py"
V1_GTK = ROOT / "kernelswift_b200" / "ks_grouped_topk.py"


def kept_by_auto_bench_filter(node):
    """auto_bench.py:100-124 keeps imports, defs, classes and literal assigns."""
    return isinstance(node, (ast.Import, ast.ImportFrom, ast.ClassDef, ast.FunctionDef,
                             ast.AsyncFunctionDef))


@pytest.mark.parametrize("path", [V1, V1_GTK], ids=lambda p: p.name)
def test_v1_module_is_all_kept_by_the_filter(path):
    tree = ast.parse(path.read_text())
    dropped = [type(n).__name__ for n in tree.body
               if not kept_by_auto_bench_filter(n) and not (
                   isinstance(n, ast.Expr) and isinstance(getattr(n, "value", None), ast.Constant))]
    assert not dropped, dropped


def test_v1_module_defines_the_contract():
    spec = importlib.util.spec_from_file_location("ks_v1", V1)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert callable(mod.ModelNew) and mod.get_init_inputs() == [8, 2, 128, 64]
    m = mod.ModelNew(*mod.get_init_inputs())
    assert set(m.state_dict()) == {"w1", "w2"}


def test_v1_loads_through_the_real_harness_loader():
    """If the reference checkout is present, load the v1 file with
    auto_bench's own loader (its AST filter and exec)."""
    ab = reference_file("auto_bench.py")
    spec = importlib.util.spec_from_file_location("ks_auto_bench", ab)
    harness = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(harness)
    mod = harness.load_ks_module(V1)
    assert hasattr(mod, "ModelNew") and hasattr(mod, "get_inputs")


def test_grouped_topk_module_defines_the_contract():
    """ks_grouped_topk mirrors groupedtopk/base.py's constructor defaults."""
    spec = importlib.util.spec_from_file_location("ks_gtk", V1_GTK)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.get_init_inputs() == [8, True, 8, 4]
    m = mod.ModelNew(*mod.get_init_inputs())
    assert (m.topk, m.renormalize, m.num_expert_group, m.topk_group) == (8, True, 8, 4)
    assert m.scoring_func == "softmax" and m.routed_scaling_factor == 1.0
    assert not list(m.state_dict())


@pytest.mark.parametrize("path", [V1, V1_GTK], ids=lambda p: p.name)
def test_loads_through_the_real_harness_loader(path):
    ab = reference_file("auto_bench.py")
    spec = importlib.util.spec_from_file_location("ks_auto_bench2", ab)
    harness = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(harness)
    mod = harness.load_ks_module(path)
    assert hasattr(mod, "ModelNew") and hasattr(mod, "get_inputs")
