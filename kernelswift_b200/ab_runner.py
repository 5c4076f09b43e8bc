"""Device-timed v0/v1 comparison of two auto_bench-style operator modules.

    python -m kernelswift_b200.ab_runner \\
        --v0_file kernels/track1-triton/fused_moe/base.py \\
        --v1_file kernelswift_b200/ks_fused_moe.py [--warmup 20] [--repeat 100]

Each file is loaded the way the reference harness loads it (auto_bench.py):
only imports, function and class definitions and assignments of literals
survive (auto_bench.py:100-124); the v0 module's `Model` and the v1 module's
`ModelNew` are built on the CPU from `get_init_inputs()`, v0's state dict is
copied into v1 (auto_bench.py:637-650), both move to the device and run on
v0's `get_inputs()` (auto_bench.py:654). Outputs are compared like
auto_bench's compare_values (allclose for floating tensors, equality
otherwise, recursively through tuples and lists). Each forward is timed on
the device with CUDA events (`--device cpu`: host clock), median over the
repeats, without an L2 flush: this is the per-call latency auto_bench
reports, not bench.py's cold-cache step time.

A reference module that imports the Cambricon `torch_mlu` package (as
fused_moe/base.py:4-5 does) gets an empty stub of it, and tensors it creates
on "cuda" are moved to `--device`. Prints one JSON line.
"""
from __future__ import annotations

import argparse
import ast
import atexit
import importlib.util
import json
import shutil
import statistics
import sys
import tempfile
import time
from pathlib import Path

import torch


# ---------------------------------------------------------------------------
# module loading (auto_bench.py:85-124)
# ---------------------------------------------------------------------------

def _is_literal(node: ast.AST) -> bool:
    if isinstance(node, ast.Constant):
        return True
    if isinstance(node, (ast.Tuple, ast.List, ast.Set)):
        return all(_is_literal(e) for e in node.elts)
    if isinstance(node, ast.Dict):
        return all(k is None or _is_literal(k) for k in node.keys) and all(
            _is_literal(v) for v in node.values)
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.UAdd, ast.USub)):
        return _is_literal(node.operand)
    return False


def _filter(tree: ast.Module) -> ast.Module:
    keep = []
    for node in tree.body:
        if isinstance(node, (ast.Import, ast.ImportFrom, ast.ClassDef, ast.FunctionDef,
                             ast.AsyncFunctionDef)):
            keep.append(node)
        elif isinstance(node, ast.Assign) and _is_literal(node.value):
            keep.append(node)
        elif isinstance(node, ast.AnnAssign) and node.value is not None and _is_literal(
                node.value):
            keep.append(node)
    tree.body = keep
    ast.fix_missing_locations(tree)
    return tree


_STUB_DIR: Path | None = None


def _ensure_torch_mlu_stub() -> None:
    """An empty `torch_mlu` package (and torch_mlu.utils.gpu_migration)."""
    global _STUB_DIR
    try:
        import torch_mlu  # noqa: F401
        return
    except ImportError:
        pass
    if _STUB_DIR is None:
        _STUB_DIR = Path(tempfile.mkdtemp(prefix="torch_mlu_stub_"))
        atexit.register(shutil.rmtree, str(_STUB_DIR), True)  # removed when the process ends
        pkg = _STUB_DIR / "torch_mlu"
        (pkg / "utils").mkdir(parents=True)
        (pkg / "__init__.py").write_text("")
        (pkg / "utils" / "__init__.py").write_text("")
        (pkg / "utils" / "gpu_migration.py").write_text("")
        sys.path.insert(0, str(_STUB_DIR))


def load_module(path: str | Path, name: str):
    """Executes the filtered AST of `path` as a fresh module."""
    path = Path(path)
    src = path.read_text()
    if "torch_mlu" in src:
        _ensure_torch_mlu_stub()
    tree = _filter(ast.parse(src, filename=str(path)))
    spec = importlib.util.spec_from_loader(name, loader=None)
    mod = importlib.util.module_from_spec(spec)
    mod.__file__ = str(path)
    exec(compile(tree, str(path), "exec"), mod.__dict__)
    return mod


# ---------------------------------------------------------------------------
# comparison (auto_bench.py:296-381)
# ---------------------------------------------------------------------------

def compare(v0, v1, atol: float, rtol: float, path: str = "output") -> list[str]:
    """Differences between two outputs (empty when they match)."""
    if isinstance(v0, torch.Tensor) or isinstance(v1, torch.Tensor):
        if not (isinstance(v0, torch.Tensor) and isinstance(v1, torch.Tensor)):
            return [f"{path}: type {type(v0).__name__} vs {type(v1).__name__}"]
        if v0.shape != v1.shape:
            return [f"{path}: shape {tuple(v0.shape)} vs {tuple(v1.shape)}"]
        a, b = v0.detach(), v1.detach().to(v0.device)
        if a.dtype.is_floating_point or b.dtype.is_floating_point:
            if not torch.allclose(a, b.to(a.dtype), atol=atol, rtol=rtol, equal_nan=True):
                d = (a.float() - b.float()).abs()
                return [f"{path}: max_abs_diff={float(d.max()):.3e}"]
            return []
        if not torch.equal(a, b.to(a.dtype)):
            return [f"{path}: {int((a != b.to(a.dtype)).sum())} elements differ"]
        return []
    if isinstance(v0, (tuple, list)) and isinstance(v1, (tuple, list)):
        if len(v0) != len(v1):
            return [f"{path}: length {len(v0)} vs {len(v1)}"]
        out = []
        for i, (x, y) in enumerate(zip(v0, v1)):
            out += compare(x, y, atol, rtol, f"{path}[{i}]")
        return out
    return [] if v0 == v1 else [f"{path}: {v0!r} vs {v1!r}"]


# ---------------------------------------------------------------------------
# timing
# ---------------------------------------------------------------------------

def time_call(fn, device: torch.device, warmup: int, repeat: int) -> float:
    """Median milliseconds of fn() over `repeat` calls after `warmup` calls."""
    with torch.no_grad():
        for _ in range(warmup):
            fn()
        times = []
        if device.type == "cuda":
            torch.cuda.synchronize(device)
            for _ in range(repeat):
                s = torch.cuda.Event(enable_timing=True)
                e = torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                e.synchronize()
                times.append(s.elapsed_time(e))
        else:
            for _ in range(repeat):
                t0 = time.perf_counter()
                fn()
                times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times)


def _to(x, device):
    if isinstance(x, torch.Tensor):
        return x.to(device)
    if isinstance(x, (tuple, list)):
        return type(x)(_to(v, device) for v in x)
    return x


def run(v0_file, v1_file, device="cuda", warmup=20, repeat=100, atol=1e-2, rtol=1e-2,
        seed=42) -> dict:
    device = torch.device(device)
    m0 = load_module(v0_file, "ab_v0")
    m1 = load_module(v1_file, "ab_v1")
    torch.manual_seed(seed)
    model0 = m0.Model(*m0.get_init_inputs())
    model1 = m1.ModelNew(*m1.get_init_inputs())
    try:
        model1.load_state_dict(model0.state_dict())
    except RuntimeError as exc:  # auto_bench swallows this too (auto_bench.py:642-645)
        print(f"load_state_dict: {exc}", file=sys.stderr)
    model0 = model0.to(device).eval()
    model1 = model1.to(device).eval()
    if device.type == "cuda":
        inputs = m0.get_inputs()
    else:  # the reference modules create their inputs on "cuda"
        inputs = _cpu_inputs(m0)
    inputs = _to(inputs, device)
    with torch.no_grad():
        out0 = model0(*inputs)
        out1 = model1(*inputs)
    diffs = compare(out0, out1, atol, rtol)
    t0 = time_call(lambda: model0(*inputs), device, warmup, repeat)
    t1 = time_call(lambda: model1(*inputs), device, warmup, repeat)
    return {"v0_file": str(v0_file), "v1_file": str(v1_file), "device": str(device),
            "match": not diffs, "differences": diffs[:8], "v0_ms": t0, "v1_ms": t1,
            "speedup": t0 / t1 if t1 > 0 else None, "timing": (
                "CUDA events, median" if device.type == "cuda" else "host clock, median"),
            "warmup": warmup, "repeat": repeat}


def _cpu_inputs(mod):
    """get_inputs() with every device="cuda" request served on the CPU."""
    orig = {name: getattr(torch, name) for name in ("randn", "rand", "zeros", "ones", "empty",
                                                    "randint", "tensor", "full")}

    def wrap(fn):
        def inner(*a, **kw):
            if "device" in kw:
                kw["device"] = "cpu"
            return fn(*a, **kw)
        return inner

    try:
        for name, fn in orig.items():
            setattr(torch, name, wrap(fn))
        return mod.get_inputs()
    finally:
        for name, fn in orig.items():
            setattr(torch, name, fn)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--v0_file", required=True)
    ap.add_argument("--v1_file", required=True)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--repeat", type=int, default=100)
    ap.add_argument("--atol", type=float, default=1e-2)
    ap.add_argument("--rtol", type=float, default=1e-2)
    ap.add_argument("--seed", type=int, default=42)
    a = ap.parse_args()
    print(json.dumps(run(a.v0_file, a.v1_file, a.device, a.warmup, a.repeat, a.atol, a.rtol,
                         a.seed)))


if __name__ == "__main__":
    main()
