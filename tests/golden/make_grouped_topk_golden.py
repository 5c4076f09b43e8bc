"""Generates tests/golden/gtk_*.npz from the reference grouped top-k operator.

Runs the unmodified kernels/track1-triton/groupedtopk/base.py of the
kernelswift reference (plain torch, CPU) on every case of
cases.GROUPED_CASES and stores, per case:
  topk_weights  fp32 [T, k]   the reference Model.forward outputs
  topk_ids      int32 [T, k]
  digest        SHA-256 of the regenerated inputs

Usage (needs the reference checkout; the outputs are committed):
    python tests/golden/make_grouped_topk_golden.py <reference checkout>  (or set KS_REFERENCE_ROOT)
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from cases import GROUPED_CASES, digest, make_grouped_inputs  # noqa: E402

BASE_REL = Path("kernels/track1-triton/groupedtopk/base.py")


def reference_checkout() -> Path:
    """The reference checkout: the first argument, else KS_REFERENCE_ROOT."""
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KS_REFERENCE_ROOT")
    if not arg:
        raise SystemExit("usage: give the reference checkout as the first argument "
                         "or in KS_REFERENCE_ROOT")
    return Path(arg)


def main() -> None:
    ref_root = reference_checkout()
    spec = importlib.util.spec_from_file_location("ks_grouped_topk_base", ref_root / BASE_REL)
    base = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(base)
    for c in GROUPED_CASES:
        hidden, logits = make_grouped_inputs(c)
        model = base.Model(c.topk, c.renormalize, c.num_expert_group, c.topk_group,
                           c.scoring_func, c.routed_scaling_factor).eval()
        with torch.no_grad():
            w, ids = model(hidden, logits)
        np.savez_compressed(HERE / f"{c.name}.npz", topk_weights=w.numpy(),
                            topk_ids=ids.numpy(), digest=np.asarray(digest(hidden, logits)))
        print(c.name, tuple(w.shape))


if __name__ == "__main__":
    main()
