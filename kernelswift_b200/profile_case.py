"""Runs the fused-MoE operator on one workload for a few steps, untimed.

Small, self-contained driver for profilers (ncu): it holds only the prepared
weights, the inputs and the workspace on the device (the Mixtral layer at
T=4096 needs about 3.5 GB), launches `--steps` forwards and exits.

    python -m kernelswift_b200.profile_case --workload mixtral --tokens 4096 --steps 3
"""
from __future__ import annotations

import argparse

import torch

from . import fused_moe as fm

WORKLOADS = {
    "mixtral": (4096, 14336, 8, 2, "none", 0.0),
    "qwen3": (2048, 768, 128, 8, "none", 0.5),
    "dsv3": (7168, 2048, 256, 8, "none", 0.0),
    "dsv3-fp8": (7168, 2048, 256, 8, "fp8", 0.0),
    "dsv3-fp8-ue8m0": (7168, 2048, 256, 8, "fp8-ue8m0", 0.0),
    "qwen3-int8": (2048, 768, 128, 8, "int8", 0.5),
}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mixtral")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--experts", type=int, default=0,
                    help="override the expert count (a smaller capture of the same kernel)")
    args = ap.parse_args()
    H, I, E, k, quant, bias = WORKLOADS[args.workload]
    E = args.experts or E
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    hidden = torch.randn(args.tokens, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(args.tokens, E, generator=g, device=dev)
    if bias:
        logits = logits + torch.randn(E, generator=g, device=dev) * bias
    w1 = torch.randn(E, 2 * I, H, generator=g, device=dev, dtype=torch.bfloat16) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g, device=dev, dtype=torch.bfloat16) / I ** 0.5
    prep = fm.prepare_weights(w1, w2, quant, torch.bfloat16)
    del w1, w2
    for _ in range(args.steps):
        tw, ti = fm.fused_topk(hidden, logits, k)
        out = fm.fused_experts(hidden, prep, None, tw.to(hidden.dtype), ti,
                               use_fp8_w8a8=quant.startswith("fp8"),
                               use_int8_w8a8=quant == "int8")
    torch.cuda.synchronize()
    print(f"profile_case {args.workload} T={args.tokens}: out {tuple(out.shape)} "
          f"finite={bool(torch.isfinite(out).all())}")


if __name__ == "__main__":
    main()
