"""Benchmark of the B200 fused-MoE operator (one JSON line on rank 0).

Default workload: the Mixtral-8x7B-shaped MoE layer (H=4096, I=14336, E=8,
top-2, bf16) on T=4096 tokens per GPU -- the configuration the headline
metric (fused-MoE layer tokens/s and TFLOP/s) is quoted on. A step is one
forward of the operator: routing (softmax/top-k/renormalise) + align +
gather + gate-up GEMM (SiLU fused) + down GEMM (top-k weight fused) + top-k
sum, over one batch of synthetic tokens (N(0,1) activations, N(0,1/fan_in)
weights, N(0,1) router logits).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg0|mixtral|qwen3|dsv3|dsv3-fp8|dsv3-fp8-ue8m0|qwen3-int8]
                    [--tokens T]

`value` is device time (CUDA events, inputs resident in HBM, L2 flushed
between steps outside the timed windows, max over ranks). On one GPU a step
is a replay of a CUDA graph that holds the whole forward (fused_moe.CapturedMoE;
`--no-graph` launches every kernel eagerly instead); expert parallelism
(N > 1) launches eagerly, exchanging rows through the NVLink peer-memory
dispatch/combine kernels (`--ep-exchange nccl`: NCCL all_to_all). `e2e` is
the same metric through the public API (fused_moe.HostPipeline) with pinned
host buffers: every step copies its hidden states and router logits in and
its output out, on copy streams that overlap the neighbouring steps'
compute.
`--impl reference` times the reference's CPU torch path (base.py:35-76,
restated in the oracle) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent

WORKLOADS = {
    # name: (H, I, E, k, quant, default T, logit bias std); activations bf16
    # except for the fp32 ones in FP32_WORKLOADS
    # the CPU-runnable fp32 configuration (tf32 tensor-core GEMMs on the GPU)
    "cfg0": (512, 1024, 8, 2, "none", 64, 0.0),
    "mixtral": (4096, 14336, 8, 2, "none", 4096, 0.0),
    "qwen3": (2048, 768, 128, 8, "none", 8192, 0.5),
    "dsv3": (7168, 2048, 256, 8, "none", 8192, 0.0),
    "dsv3-fp8": (7168, 2048, 256, 8, "fp8", 4096, 0.0),
    # the same layer with power-of-two block scales applied by the tensor core
    "dsv3-fp8-ue8m0": (7168, 2048, 256, 8, "fp8-ue8m0", 4096, 0.0),
    "qwen3-int8": (2048, 768, 128, 8, "int8", 8192, 0.5),
}
FP32_WORKLOADS = {"cfg0"}
METRIC = "fused-MoE layer tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20


class L2Flush:
    """Empties L2 between timed steps: writes a buffer twice the size of L2,
    then (unless MOE_BENCH_WRITE_FLUSH_ONLY=1) reads a second one, so the
    dirty lines of the write are written back before the timed window opens
    instead of inside it."""

    evict = os.environ.get("MOE_BENCH_WRITE_FLUSH_ONLY", "0") in ("", "0")

    def __init__(self, dev):
        import torch
        self.buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.rd = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev) if self.evict else None

    def __call__(self):
        self.buf.zero_()
        if self.rd is not None:
            self.rd.max()


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mixtral")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per GPU (0 = workload default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ep-exchange", choices=("auto", "nccl", "nccl-dedup", "peer"),
                    default="auto",
                    help="expert-parallel row exchange for --gpus > 1 (auto: NVLink peer "
                         "memory; nccl-dedup: all_to_all sending a token to a rank once)")
    ap.add_argument("--ep-chunks", type=int, default=1,
                    help="with --ep-exchange nccl/nccl-dedup: pipeline the exchange in this "
                         "many token chunks (deduplicated rows; each chunk's all_to_all "
                         "overlaps the previous chunk's experts)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every step eagerly instead of replaying a CUDA graph of the "
                         "whole forward (1 GPU runs use the graph by default)")
    ap.add_argument("--heat-seconds", type=float, default=1.0,
                    help="untimed busy period before timing, so clock samples see a loaded GPU")
    return ap.parse_args()


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def flops_per_token(H, I, k):
    # gate-up 2*H*2I + down 2*I*H multiply-adds per routed row
    return 6 * H * I * k


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        if not getattr(self, "lines", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        busy = [s for s, p in zip(sm, power) if p > 0.3 * max(power)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(smax),
                "power_w_max": max(power), "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# CPU side: the reference's torch path on the host cores
# ---------------------------------------------------------------------------

_CPU_WEIGHTS: dict = {}
CPU_WEIGHT_BUDGET = 24 << 30  # host bytes the CPU baseline may hold in weights


def cpu_experts(H, I, E, k):
    """Experts the CPU baseline can hold: base.py keeps fp32 masters
    (12*H*I bytes per expert) and makes bf16 copies on every call (half as
    much again). When all E do not fit in min(24 GB, 35% of host RAM), the
    baseline runs on the largest count that does (at least top_k), routing
    over those experts only; the per-call casts of the others are then not
    timed, so the baseline reads faster than the full layer."""
    try:
        import psutil
        budget = min(CPU_WEIGHT_BUDGET, int(0.35 * psutil.virtual_memory().total))
    except Exception:
        budget = CPU_WEIGHT_BUDGET
    per_expert = 1.5 * 12 * H * I
    return int(min(E, max(k, budget // per_expert)))


def cpu_reference_rate(H, I, E, k, quant, bias, sample_tokens, repeats, warmup=1,
                       min_seconds=0.0, act_dtype=None):
    """tokens/s of base.py's forward (oracle restatement) on the host CPU:
    median over `repeats` calls, more calls until `min_seconds` of timed work.
    Uses cpu_experts(...) of the E experts."""
    import torch
    from oracle import moe_oracle as orc

    E = cpu_experts(H, I, E, k)
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    hidden = torch.randn(sample_tokens, H, generator=g).to(act_dtype or torch.bfloat16)
    logits = torch.randn(sample_tokens, E, generator=g)
    if bias:
        logits = logits + torch.randn(E, generator=g) * bias
    # base.py keeps fp32 master weights and casts them on every call
    key = (E, I, H)
    if key not in _CPU_WEIGHTS:
        _CPU_WEIGHTS.clear()
        gw = torch.Generator().manual_seed(1)
        _CPU_WEIGHTS[key] = (torch.randn(E, 2 * I, H, generator=gw) / H ** 0.5,
                             torch.randn(E, H, I, generator=gw) / I ** 0.5)
    w1, w2 = _CPU_WEIGHTS[key]
    for _ in range(warmup):
        orc.model_forward_native(hidden, logits, w1, w2, k)
    times = []
    while len(times) < repeats or (sum(times) < min_seconds and len(times) < 50):
        t0 = time.perf_counter()
        orc.model_forward_native(hidden, logits, w1, w2, k)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return sample_tokens / med, med, torch.get_num_threads(), len(times)


# Tokens per CPU call of each workload: one fixed sample, the same for the
# cpu_baseline leg and the --impl reference arm, so both legs time the same
# batch (about 0.2-1 s per call on a 16-core host).
CPU_SAMPLE_TOKENS = {"cfg0": 64, "mixtral": 2048, "qwen3": 1024, "qwen3-int8": 1024, "dsv3": 512,
                     "dsv3-fp8": 512, "dsv3-fp8-ue8m0": 512}


def cpu_sample_tokens(workload: str, T: int) -> int:
    """Tokens per CPU call of the reference path (at most the GPU batch T)."""
    return max(1, min(T, CPU_SAMPLE_TOKENS[workload]))


def cpu_model() -> str:
    """The host CPU's model string (/proc/cpuinfo), for the baseline record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_expert_note(H, I, E, k) -> str:
    e_cpu = cpu_experts(H, I, E, k)
    if e_cpu == E:
        return ""
    return (f"; on {e_cpu} of the {E} experts (host RAM: their fp32 masters and per-call "
            f"bf16 casts would need {1.5 * 12 * H * I * E / 2**30:.0f} GiB), so the casts of "
            "the other experts are not timed and the rate is an upper bound")


def run_reference(args, H, I, E, k, quant, T, bias, rank):
    """--impl reference: the reference's CPU torch path, rank 0 only."""
    if rank != 0:
        return
    sample = cpu_sample_tokens(args.workload, T)
    import torch
    act = torch.float32 if args.workload in FP32_WORKLOADS else torch.bfloat16
    rate, med, cores, n = cpu_reference_rate(H, I, E, k, quant, bias, sample,
                                             repeats=max(1, args.steps), warmup=max(0, args.warmup),
                                             act_dtype=act)
    dname = act_dtype_name(args.workload)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": med * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dname, "data": "synthetic",
        "config": dict(workload_config(args.workload, H, I, E, k, quant, T, args.gpus),
                       l2="not applicable: host CPU run", parallelism="single host process"),
        "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{sample} tokens per step of the {args.workload} layer, "
                                   f"base.py forward restated in torch-CPU {dname} with the "
                                   f"per-call fp32->{dname} weight casts"
                                   + cpu_expert_note(H, I, E, k)},
        "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def act_dtype_name(name: str) -> str:
    return "f32" if name in FP32_WORKLOADS else "bf16"


def workload_config(name, H, I, E, k, quant, T, n, exchange=None, chunks=1):
    return {"workload": f"{name} MoE layer H={H} I={I} E={E} top-{k} "
                        f"{act_dtype_name(name) if quant == 'none' else quant + ' W8A8'}, "
                        f"{T} tokens/GPU",
            "hidden": H, "intermediate": I, "experts": E, "top_k": k, "quant": quant,
            "tokens_per_gpu": T, "global_tokens": T * n,
            "parallelism": (f"ep{n} (E/{n} experts per GPU, " + (
                "one row per token and destination rank, moved by dispatch/combine kernels "
                "over NVLink peer memory)"
                if exchange == "peer" else
                "NCCL all_to_all, one row per token and destination rank"
                + (f", pipelined in {chunks} token chunks)" if chunks > 1 else ")")
                if exchange == "nccl-dedup" else "NCCL all_to_all)")) if n > 1 else "single",
            "l2": f"flushed between steps outside the timed windows ({L2_FLUSH_BYTES >> 20} MB "
                  f"write{', then a read of another ' + str(L2_FLUSH_BYTES >> 20) + ' MB that evicts the dirty lines' if L2Flush.evict else ''}); "
                  "weights also exceed L2",
            "switches": active_switches()}


def active_switches() -> dict:
    """The library's environment switches as this run saw them."""
    def on(name, default):
        v = os.environ.get(name)
        return default if not v else v[0] != "0"  # the library's reading
    return {"pdl": not on("MOE_NO_PDL", False), "decode_path": not on("MOE_NO_DECODE_PATH", False),
            "tail_halves": not on("MOE_NO_TAIL_HALVES", False),
            "token_gather": not on("MOE_NO_TOKEN_GATHER", False),
            "block_n": os.environ.get("MOE_BLOCK_N") or "planner"}


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

def main():
    args = parse_args()
    H, I, E, k, quant, T0, bias = WORKLOADS[args.workload]
    T = args.tokens or T0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, H, I, E, k, quant, T, bias, rank)
        return

    import torch
    import torch.distributed as dist

    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        sys.exit(1)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from kernelswift_b200 import _lib
    from kernelswift_b200 import fused_moe as fm

    # ---- synthetic problem (weights N(0, 1/fan_in), tokens N(0, 1)) ----
    act_dtype = torch.float32 if args.workload in FP32_WORKLOADS else torch.bfloat16
    if world > 1 and act_dtype != torch.bfloat16:
        raise SystemExit(f"{args.workload}: the expert-parallel exchange moves 16-bit rows")
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    hidden = torch.randn(T, H, generator=g, device=dev).to(act_dtype)
    logits = torch.randn(T, E, generator=g, device=dev)
    if bias:
        logits = logits + torch.randn(E, generator=g, device=dev) * bias
    flush = L2Flush(dev)
    rows_per_launch = [T * k]  # routed rows the local gate-up GEMM saw (last step)
    experts_hit = [0]          # distinct local experts with rows (for the byte count)
    if world == 1:
        # the drop-in module: fp32 master weights as in base.py, prepared once
        # (created on the device: DeepSeek-V3's 45 GB of masters never touch
        # host memory)
        with torch.device(dev):
            model = fm.ModelNew(E, k, H, I)
        with torch.no_grad():
            model.w1.normal_(0.0, 1.0 / math.sqrt(H), generator=g)
            model.w2.normal_(0.0, 1.0 / math.sqrt(I), generator=g)
        prep = model.prepared(act_dtype, quant)

        def step(stage_arr=None):
            return fm.fused_moe(hidden, prep, None, logits, k,
                                use_fp8_w8a8=quant.startswith("fp8"),
                                use_int8_w8a8=quant == "int8", stage_events=stage_arr)
    else:
        # expert parallel: this rank holds E/world experts, routes its own T
        # tokens over all E; rows move through the peer-memory dispatch and
        # combine kernels (--ep-exchange nccl: NCCL all_to_all)
        from kernelswift_b200.ep import ExpertParallelMoE

        if E % world:
            raise SystemExit(f"{E} experts do not shard over {world} GPUs")
        el = E // world
        w1 = torch.randn(el, 2 * I, H, generator=g, device=dev, dtype=torch.bfloat16) / math.sqrt(H)
        w2 = torch.randn(el, H, I, generator=g, device=dev, dtype=torch.bfloat16) / math.sqrt(I)
        def make_ep(exchange):
            dedup = exchange == "nccl-dedup"
            chunks = args.ep_chunks if exchange in ("nccl", "nccl-dedup") else 1
            return ExpertParallelMoE(w1, w2, E, k, quant=quant,
                                     exchange="nccl" if dedup else exchange,
                                     max_tokens=T, dtype=hidden.dtype, dedup=dedup,
                                     chunks=chunks)

        try:
            ep = make_ep(args.ep_exchange)
        except RuntimeError as exc:  # raised on every rank alike
            if args.ep_exchange != "auto":
                raise
            print(f"peer exchange unavailable, using NCCL: {exc}", file=sys.stderr)
            ep = make_ep("nccl")

        def step(stage_arr=None, exchange_evs=None):
            tw, ti = fm.fused_topk(hidden, logits, k, weights_dtype=hidden.dtype)
            return ep(hidden, tw, ti, stage_events=stage_arr, exchange_events=exchange_evs)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        if ep.peer is not None and not ep.peer.all_ok() and args.ep_exchange == "auto":
            # a peer-exchange wait ran out on some rank: every rank switches
            print("peer exchange reported an error, using NCCL", file=sys.stderr)
            ep.close()
            ep = make_ep("nccl")
            for _ in range(max(3, args.warmup)):
                step()
            torch.cuda.synchronize()
        rows_per_launch[0] = ep.rows_received()  # the same routing every step
        if ep.peer is not None:
            ep.peer.check()
    _, ti0 = fm.fused_topk(hidden, logits, k)
    if world == 1:
        experts_hit[0] = int(torch.unique(ti0).numel())
    else:
        el = E // world
        got = torch.zeros(E, dtype=torch.int32, device=dev)
        got[torch.unique(ti0)] = 1
        dist.all_reduce(got)
        experts_hit[0] = int((got[rank * el:(rank + 1) * el] > 0).sum())

    K = args.steps
    clocks = ClockSampler(local_rank).__enter__()
    # keep the GPU busy for a second before timing so that the clock samples
    # cover a loaded GPU (these steps are untimed warm-up)
    # The number of heat steps is agreed across ranks (every rank must issue
    # the same collectives): time one step, take the max over ranks.
    t_one = time.perf_counter()
    step()
    torch.cuda.synchronize()
    t_one = torch.tensor([time.perf_counter() - t_one], device=dev)
    if world > 1:
        dist.all_reduce(t_one, op=dist.ReduceOp.MAX)
    n_heat = int(args.heat_seconds / max(float(t_one.item()), 1e-4))
    for _ in range(min(n_heat, 100000)):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    stage_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(_lib.STAGES) + 1)]
                 for _ in range(K)]
    for evs in stage_evs:
        for ev in evs:
            ev.record()  # create the events before the timed region
    stage_arrs = [fm.stage_event_array(evs) for evs in stage_evs]
    ex_evs = None
    if world > 1:
        from kernelswift_b200.ep import EXCHANGE_STAGES
        # boundaries of the exchange stages of every timed step
        ex_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(EXCHANGE_STAGES) + 1)]
                  for _ in range(K)]
        for evs in ex_evs:
            for ev in evs:
                ev.record()
    torch.cuda.synchronize()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    # the timed steps carry no events besides their start and end: an event
    # record between two kernels costs a few microseconds and breaks the
    # programmatic overlap of the launches around it
    for i in range(K):
        flush()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    use_graph = args.graph and world == 1
    stage_ms = {name: 0.0 for name in _lib.STAGES}
    exchange_ms = None
    if not use_graph:
        # per-stage breakdown from K more steps, instrumented (untimed as a whole)
        inst = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
        for i in range(K):
            flush()
            inst[i].record()
            if ex_evs is None:
                step(stage_arrs[i])
            else:
                step(stage_arrs[i], ex_evs[i])
        torch.cuda.synchronize()
        stage_ms = {name: sum(evs[j].elapsed_time(evs[j + 1]) for evs in stage_evs) / K
                    for j, name in enumerate(_lib.STAGES)}
        if ex_evs is not None:
            # per stage: the mean over the instrumented steps, then the max over
            # ranks ("route" = the routing kernel, from the step's start to the plan)
            names = ("route",) + EXCHANGE_STAGES
            per = [sum(inst[i].elapsed_time(ex_evs[i][0]) for i in range(K)) / K]
            per += [sum(ex_evs[i][j].elapsed_time(ex_evs[i][j + 1]) for i in range(K)) / K
                    for j in range(len(EXCHANGE_STAGES))]
            t = torch.tensor(per, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            exchange_ms = dict(zip(names, (float(x) for x in t.tolist())))
    graph = None
    if use_graph:
        # The whole forward (routing + all kernels) captured once and replayed:
        # no host launch gaps. A second capture carries stage events (event
        # record nodes) for the per-kernel breakdown.
        def graph_fn(hd, ld, stage_arr=None):
            return fm.fused_moe(hd, prep, None, ld, k, use_fp8_w8a8=quant.startswith("fp8"),
                                use_int8_w8a8=quant == "int8", stage_events=stage_arr)

        graph = fm.CapturedMoE(graph_fn, T, H, E, dtype=act_dtype, device=dev)
        graph.hidden.copy_(hidden)
        graph.logits.copy_(logits)
        gevs = stage_evs[0]
        gi = fm.CapturedMoE(lambda hd, ld: graph_fn(hd, ld, stage_arrs[0]), T, H, E,
                            dtype=act_dtype, device=dev)
        gi.hidden.copy_(hidden)
        gi.logits.copy_(logits)
        acc = [0.0] * len(_lib.STAGES)
        for i in range(K):
            flush()
            gi.replay()
            torch.cuda.synchronize()
            for j in range(len(_lib.STAGES)):
                acc[j] += gevs[j].elapsed_time(gevs[j + 1])
        stage_ms = {name: acc[j] / K for j, name in enumerate(_lib.STAGES)}
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        wall0 = time.perf_counter()
        for i in range(K):
            flush()
            starts[i].record()
            graph.replay()
            ends[i].record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        total_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    # the clock samples cover the heat steps and every timed step (the graph
    # replays included)
    clocks.__exit__(None, None, None)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / K
    tokens_per_s = T * world / (ms_per_step / 1e3)
    tflops = flops_per_token(H, I, k) * T * world / (ms_per_step / 1e3) / 1e12

    # ---- e2e through ModelNew.forward with host buffers ----
    e2e = None
    if not args.no_e2e:
        h_host = hidden.cpu().pin_memory()
        l_host = logits.cpu().pin_memory()
        out_host = torch.empty(T, H, dtype=act_dtype).pin_memory()
        if use_graph:
            def model_call(hd, ld):
                return graph(hd, ld)
        elif world == 1 and quant == "none":
            model_call = model
        else:
            def model_call(hd, ld):
                if world > 1:
                    tw, ti = fm.fused_topk(hd, ld, k, weights_dtype=hd.dtype)
                    return ep(hd, tw, ti)
                return fm.fused_moe(hd, prep, None, ld, k, use_fp8_w8a8=quant.startswith("fp8"),
                                    use_int8_w8a8=quant == "int8")

        # the public host-I/O pipeline: each step's H2D and D2H copies run on
        # their own streams, overlapping the neighbouring steps' compute
        pipe = fm.HostPipeline(model_call, T, H, E, dtype=act_dtype, device=dev)

        def e2e_step():
            pipe.submit(h_host, l_host, out_host)

        for _ in range(max(3, args.warmup)):
            e2e_step()
        pipe.flush()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K):
            e2e_step()
        pipe.flush()
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / K
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s",
               "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": hidden.numel() * hidden.element_size()
               + logits.numel() * logits.element_size(),
               "d2h_bytes_per_step": T * H * hidden.element_size(),
               "path": "HostPipeline over " + (
                   "CapturedMoE (CUDA graph of fused_moe: routing + experts)" if use_graph
                   else "ModelNew.forward (drop-in module)" if world == 1 and quant == "none"
                   else "fused_topk + " + ("ExpertParallelMoE.forward" if world > 1
                                           else "fused_experts"))
               + ", pinned host buffers; every step copies its inputs in and its output "
                 "out, on copy streams that overlap the neighbouring steps' compute"}

    # ---- roofline of the dominant kernel (gate-up GEMM) ----
    # Algorithmic work of one launch: 4*H*I*rows FLOPs; bytes = the w13 slices
    # of the experts hit + the gathered rows read + the activations written.
    # The binding resource is whichever of (FLOPs / tensor peak) and
    # (bytes / HBM peak) takes longer.
    peaks, peak_src = load_peaks()
    gu_ms = stage_ms["gate_up"]
    rows = rows_per_launch[0]
    gu_flops = 4 * H * I * rows
    a_bytes = torch.empty(0, dtype=act_dtype).element_size()
    w_bytes = a_bytes if quant == "none" else 1
    e_local = E if world == 1 else E // world
    hit = experts_hit[0] if experts_hit[0] else e_local
    gu_bytes = hit * 2 * I * H * w_bytes + rows * H * w_bytes + rows * I * a_bytes
    tensor_peak = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    tensor_note = f"bf16 dense, sustained, {peak_src}"
    if act_dtype == torch.float32 and quant == "none":
        tensor_peak /= 2
        tensor_note = f"bf16 dense sustained / 2 (tf32 operand rate), {peak_src}"
    if quant != "none":
        tensor_peak *= 2
        tensor_note = f"2x bf16 dense sustained ({quant} operand rate), {peak_src}"
    hbm_peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    t_tensor = gu_flops / (tensor_peak * 1e12)
    t_hbm = gu_bytes / (hbm_peak * 1e9)
    if t_tensor >= t_hbm:
        achieved = gu_flops / (gu_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": tensor_peak,
                "unit": "TFLOP/s", "frac": achieved / tensor_peak, "peak_source": tensor_note}
    else:
        achieved = gu_bytes / (gu_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_source": f"copy bandwidth, {peak_src}"}
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        try:
            entry = json.loads(tfile.read_text()).get(f"{args.workload}:{T}:gate_up")
            traffic = entry["bytes"] if entry and world == 1 else None
        except Exception:
            traffic = None
    roofline = {"kernel": "moe_grouped_gemm_kernel (gate-up, SiLU fused)", **roof,
                "traffic": traffic,
                "traffic_unit": "DRAM bytes per launch (ncu capture, profiles/)",
                "algorithmic": f"{gu_flops:.4g} FLOP (4*H*I*rows, rows={rows}) and "
                               f"{gu_bytes / 1e9:.4g} GB ({hit} experts' w13 + rows in + act out) "
                               "per launch",
                "launch_ms": gu_ms}
    if world == 1 and quant == "none" and fm.fused_experts_plan(T, H, I, E, k, quant,
                                                                 act_dtype)["decode_path"]:
        # decode sizes: the weight-streaming gate-up kernel (its stage) reads
        # the hit experts' w13 and the token rows, writes the act rows
        dec_bytes = hit * 2 * I * H * 2 + T * H * 2 + rows * I * 2
        achieved = dec_bytes / (gu_ms / 1e3) / 1e9
        roofline = {"kernel": "decode_gate_up_kernel (SiLU fused)", "bound": "hbm",
                    "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                    "frac": achieved / hbm_peak, "peak_source": f"copy bandwidth, {peak_src}",
                    "traffic": traffic,
                    "traffic_unit": "DRAM bytes per launch (ncu capture, profiles/)",
                    "algorithmic": f"{dec_bytes / 1e6:.4g} MB ({hit} experts' w13 + tokens in + "
                                   "act out) per launch",
                    "launch_ms": gu_ms}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = cpu_sample_tokens(args.workload, T)
        rate, med, cores, n = cpu_reference_rate(H, I, E, k, quant, bias, sample, repeats=3,
                                                 min_seconds=10.0, act_dtype=act_dtype)
        cpu = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
               "cpu_model": cpu_model(),
               "sample": f"{sample} tokens of the same layer per call, base.py forward "
                         f"restated in torch-CPU {act_dtype_name(args.workload)} with its "
                         "per-call weight casts "
                         f"(median of {n} calls, {med:.2f} s each)"
                         + cpu_expert_note(H, I, E, k)}

    # align is launch-bound: its time (graph stage, with one event record)
    # and the bytes it moves, ids in + sorted ids and block experts out
    if world == 1:
        n_ids = T * k
    elif ep.peer is not None:
        # align takes the received rows' k slots (the device-side count)
        n_ids = int(ep.peer.recv_count.item()) * k
    elif ep.dedup:
        n_ids = ep.last_rows_received * k  # k slots per received token row
    else:
        n_ids = int(rows_per_launch[0])
    e_al = E if world == 1 else E // world
    L_al = -(-(n_ids + e_al * 127) // 128) * 128
    al_bytes = n_ids * 4 + (L_al + L_al // 128) * 4
    al_ms = stage_ms.get("align", 0.0)
    align_report = {"us": al_ms * 1e3, "bytes": al_bytes,
                    "gbs": al_bytes / (al_ms * 1e-3) / 1e9 if al_ms > 0 else None}

    # our kernels per step: the routing kernel plus what the expert pass
    # launches for this shape (the plan's own count), plus the exchange
    if world == 1:
        launches_per_step = fm.fused_moe_launches(T, H, I, E, k, quant, act_dtype)
    elif ep.peer is not None:
        # routing, plan, dispatch, expert pass over the receive buffer
        # (top_k = k, bounded by the received count), signal, combine, step end
        launches_per_step = 1 + 2 + fm.fused_experts_launches(
            ep.peer.capacity, H, I, E // world, k, quant) + 3
    elif ep.dedup:
        # routing, plan, pack, expert pass over the received token rows
        # (top_k = k), combine
        launches_per_step = 1 + 2 + fm.fused_experts_launches(
            ep.last_rows_received, H, I, E // world, k, quant) + 1
    else:
        # routing, plan, pack, expert pass over the received rows (top_k = 1),
        # combine
        launches_per_step = 1 + 2 + fm.fused_experts_launches(
            rows_per_launch[0], H, I, E // world, 1, quant) + 1
    if rank == 0:
        line = {
            "metric": METRIC, "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": (act_dtype_name(args.workload) if quant == "none"
                      else ("int8" if quant == "int8" else "e4m3")),
            "data": "synthetic",
            "config": workload_config(args.workload, H, I, E, k, quant, T, world,
                                      None if world == 1 else
                                      (ep.exchange if ep.exchange == "peer" else
                                       "nccl-dedup" if ep.dedup else "nccl"),
                                      1 if world == 1 else ep.chunks),
            "tflops": tflops,
            "stage_ms": stage_ms,
            **({"exchange_ms": exchange_ms} if exchange_ms is not None else {}),
            "align": align_report,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * K,
            "cuda_graph": use_graph,
            "wall_s_timed": wall,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if ep.peer is not None:
            ep.peer.check()
        ep.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    main()
