"""GPU, 2 processes over NCCL: the expert-parallel layer against the CPU
oracle (the first tokens of each rank, through every expert they pick) and
against the single-GPU layer that holds all 256 experts, both within the
layer tolerance; partials travel in fp32, so the only bf16 rounding is the
final one.  Skipped on a box with fewer than two GPUs."""

from __future__ import annotations

import os
import datetime
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 2e-2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, q, capacity=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import __graft_entry__ as ge
        pkg = ge.load_package()
        ep = __import__("fib_b200.ep", fromlist=["ep"])
        E_l = 256 // world
        logits, bias, hs, hss = pkg.inputs.make_token_inputs(T, seed=200 + rank, device=dev)
        w13, s13, w2, s2 = pkg.inputs.make_expert_shard(0, 256, seed=5, device=dev)
        ref = torch.empty(T, 7168, dtype=torch.bfloat16, device=dev)
        pkg.kernel(logits, bias, hs, hss, w13, s13, w2, s2, 0, 2.5, ref)
        sl = slice(rank * E_l, (rank + 1) * E_l)
        layer = ep.from_library(capacity=capacity)
        out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=dev)
        layer(logits, bias, hs, hss, w13[sl], s13[sl], w2[sl], s2[sl], 2.5, out)
        out2 = torch.empty_like(out)
        layer(logits, bias, hs, hss, w13[sl], s13[sl], w2[sl], s2[sl], 2.5, out2)
        torch.cuda.synchronize()
        r, o = ref.float(), out.float()
        bad = int(((o - r).abs() > ATOL + RTOL * r.abs()).sum())
        # oracle for the first 4 tokens: their experts only, dequantised on the host
        from oracle import moe_ref
        n = 4
        lc, bc = logits[:n].cpu(), bias.cpu()
        ids, wts, _ = moe_ref.route(lc, bc, 2.5)
        used = sorted(set(ids.flatten().tolist()))
        acc = torch.zeros(n, 7168)
        for e in used:
            acc += moe_ref.experts_forward(ids, wts, hs[:n].cpu(), hss[:, :n].contiguous().cpu(),
                                           w13[e:e + 1].cpu(), s13[e:e + 1].cpu(), w2[e:e + 1].cpu(),
                                           s2[e:e + 1].cpu(), e)
        bad += int(((o[:n].cpu() - acc).abs() > ATOL + RTOL * acc.abs()).sum())
        q.put((rank, bad, bool(torch.isnan(o).any()), float((o - r).abs().max()),
               torch.equal(out.view(torch.int16), out2.view(torch.int16)), layer.last_stats))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("capacity", [None, 64])
def test_expert_parallel_two_gpus(cuda_dev, capacity):
    """Exact counts through the host, or fixed per-peer capacity (64 >= 48 tokens)."""
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 48, q, capacity)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    errs = [r for r in res if r[1] == "error"]
    assert not errs, errs[0][2]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, bad, nan, mx, det, stats in res:
        print(f"rank {rank}: max_abs {mx:.3e} stats {stats}")
        assert not nan and bad == 0, f"rank {rank}: {bad} elements outside tolerance (max {mx})"
        assert det
