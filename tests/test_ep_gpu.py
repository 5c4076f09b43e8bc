"""GPU: expert parallelism over NCCL, one process per GPU (never more ranks
than GPUs), checked against the fp32 oracle on each rank's tokens."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, cfg, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from kernelswift_b200.ep import ExpertParallelMoE
    from oracle import moe_oracle as orc

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        E, k, T, H, I, quant = cfg
        g = torch.Generator().manual_seed(0)
        w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
        w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
        el = E // world
        ep = ExpertParallelMoE(w1[rank * el:(rank + 1) * el].to(dev),
                               w2[rank * el:(rank + 1) * el].to(dev), E, k, quant=quant)
        gt = torch.Generator().manual_seed(10 + rank)
        hidden = torch.randn(T, H, generator=gt).to(torch.bfloat16)
        w, ids = orc.route(torch.randn(T, E, generator=gt), k)
        out = ep(hidden.to(dev), w.to(dev), ids.to(dev))
        torch.cuda.synchronize()
        if quant == "fp8":
            ref = orc.fused_experts_fp8(hidden, w1, w2, w, ids)
        else:
            ref = orc.fused_experts(hidden, w1, w2, w, ids)
        close = bool(torch.allclose(out.cpu().float(), ref, rtol=2e-2, atol=2e-2))
        q.put((rank, "ok", orc.rel_l2(out.cpu(), ref), close))
    except Exception as exc:
        q.put((rank, "error", repr(exc)[:300], False))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("quant", ["none", "fp8"])
def test_ep_matches_oracle(cuda_device, quant):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    cfg = (16, 4, 200, 256, 256, quant)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, status, rel, close in res:
        assert status == "ok", (rank, rel)
        if quant == "fp8":
            assert rel <= 5e-2, (rank, rel)  # relative L2 vs the dequantised oracle
        else:
            assert close, (rank, rel)  # rtol 2e-2 / atol 2e-2 vs the fp32 oracle
