"""Generates tests/golden/*.npz from the reference operator itself.

Runs the unmodified kernels/track1-triton/fused_moe/base.py of the kernelswift
reference on CPU for every case of cases.py and stores, per case:
  out        the reference Model.forward output, as float32 [T, H]
  topk_ids   the routing ids, int32 [T, k] (the reference's own torch ops)
  expert_rows, expert_offsets
             for every expert e, the flat rows base.py:65-68 selects with
             `mask = flat_ids == e` (x_rep[mask] order), concatenated
  digest     SHA-256 of the regenerated inputs

base.py imports the Cambricon `torch_mlu` package (base.py:4-5), which is only
a leftover import; a stub package is written to a temporary directory and put
on sys.path so the module loads under stock torch.

Usage (needs the reference checkout; the outputs are committed):
    python tests/golden/make_golden.py <reference checkout>  (or set KS_REFERENCE_ROOT)
"""
from __future__ import annotations

import atexit
import importlib.util
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from cases import CASES, digest, make_inputs  # noqa: E402

BASE_REL = Path("kernels/track1-triton/fused_moe/base.py")


def reference_checkout() -> Path:
    """The reference checkout: the first argument, else KS_REFERENCE_ROOT."""
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KS_REFERENCE_ROOT")
    if not arg:
        raise SystemExit("usage: give the reference checkout as the first argument "
                         "or in KS_REFERENCE_ROOT")
    return Path(arg)


def _stub_torch_mlu(root: Path) -> None:
    pkg = root / "torch_mlu"
    (pkg / "utils").mkdir(parents=True)
    (pkg / "__init__.py").write_text("")
    (pkg / "utils" / "__init__.py").write_text("")
    (pkg / "utils" / "gpu_migration.py").write_text("")


def load_reference_base(ref_root: Path):
    tmp = Path(tempfile.mkdtemp(prefix="torch_mlu_stub_"))
    atexit.register(shutil.rmtree, str(tmp), True)  # removed when the process ends
    _stub_torch_mlu(tmp)
    sys.path.insert(0, str(tmp))
    spec = importlib.util.spec_from_file_location("ks_fused_moe_base", ref_root / BASE_REL)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ref_root = reference_checkout()
    base = load_reference_base(ref_root)
    torch.set_num_threads(8)
    for c in CASES:
        hidden, logits, w1, w2 = make_inputs(c)
        model = base.Model(c.E, c.k, c.H, c.I, c.renormalize)
        model.load_state_dict({"w1": w1, "w2": w2})
        model.eval()
        with torch.no_grad():
            out = model(hidden, logits)
        # routing ids with the reference's own ops (base.py:44-45)
        scores = torch.softmax(logits.float(), dim=-1)
        _, ids = torch.topk(scores, c.k, dim=-1)
        flat = ids.view(-1)
        rows, offs = [], [0]
        for e in range(c.E):
            sel = torch.nonzero(flat == e).view(-1)
            rows.append(sel)
            offs.append(offs[-1] + sel.numel())
        np.savez_compressed(
            HERE / f"{c.name}.npz",
            out=out.float().numpy(),
            topk_ids=ids.to(torch.int32).numpy(),
            expert_rows=torch.cat(rows).to(torch.int32).numpy(),
            expert_offsets=np.asarray(offs, dtype=np.int32),
            digest=np.asarray(digest(hidden, logits, w1, w2)),
        )
        print(f"{c.name}: out {tuple(out.shape)} {out.dtype}")


if __name__ == "__main__":
    main()
