"""GPU, one process: the expert-parallel plan/pack/unpack/combine kernels of
the library (moe_fp8_ds_ep_*) against their PyTorch statement in ep.py,
bit for bit, for 2, 4 and 8 ranks, including tokens whose experts all live on
one rank and an empty batch."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ep(pkg):
    return __import__("fib_b200.ep", fromlist=["ep"])


def _routing(T, seed, dev, hot_rank=None, world=2):
    g = torch.Generator().manual_seed(seed)
    rows = [torch.randperm(256, generator=g)[:8].sort().values for _ in range(T)]
    ids = (torch.stack(rows) if rows else torch.empty(0, 8, dtype=torch.long)).to(torch.int32)
    if hot_rank is not None and T:
        E_r = 256 // world
        ids[: T // 2] = torch.arange(hot_rank * E_r, hot_rank * E_r + 8, dtype=torch.int32)
    w = torch.rand(T, 8, generator=g)
    return ids.to(dev), w.to(dev)


@pytest.mark.parametrize("world,T,hot", [(2, 300, None), (4, 1000, 1), (8, 2500, None), (8, 64, 7), (2, 0, None)])
def test_plumbing_matches_torch(pkg, cuda_dev, world, T, hot):
    ep = _ep(pkg)
    E_r = 256 // world
    ids, w = _routing(T, 7 + world, cuda_dev, hot, world)
    hidden = torch.randint(0, 256, (T, 7168), dtype=torch.uint8, device=cuda_dev)
    hidden[hidden == 0x7F] = 0      # no NaN bytes (not needed for bit-exact copies, kept tidy)
    hidden = hidden.view(torch.float8_e4m3fn)
    scale = torch.rand(56, T, device=cuda_dev) + 0.5
    lib, ref = ep.LibPlumbing(), ep.TorchPlumbing()

    c1, s1, src1 = lib.plan(ids, world, E_r)
    c0, s0, src0 = ref.plan(ids, world, E_r)
    torch.cuda.synchronize()
    assert torch.equal(c1.cpu(), c0.cpu())
    assert torch.equal(s1.long().cpu(), s0.cpu())
    S = int(c0.sum())
    assert torch.equal(src1[:S].long().cpu(), src0.cpu())

    send1 = lib.pack(ids, w, hidden, scale, src1, S)
    send0 = ref.pack(ids, w, hidden, scale, src0, S)
    assert torch.equal(send1.cpu(), send0.cpu())

    for a, b in zip(lib.unpack(send1), ref.unpack(send0)):
        assert torch.equal(a.view(torch.uint8).cpu() if a.dtype == torch.float8_e4m3fn else a.cpu(),
                           b.view(torch.uint8).cpu() if b.dtype == torch.float8_e4m3fn else b.cpu())

    back = torch.randn(S, 7168, device=cuda_dev) * 4
    out1 = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    out0 = torch.empty(T, 7168, dtype=torch.bfloat16, device=cuda_dev)
    lib.combine(back, s1, T, out1)
    ref.combine(back, s0, T, out0)
    assert torch.equal(out1.view(torch.int16).cpu(), out0.view(torch.int16).cpu())


@pytest.mark.parametrize("world,T,cap,hot", [(2, 300, 300, None), (4, 1000, 1200, 1), (8, 64, 64, 7), (8, 0, 16, None)])
def test_fixed_capacity_plumbing_matches_torch(pkg, cuda_dev, world, T, cap, hot):
    """The fixed-capacity plan and pack (padding rows, rank blocks of `cap` rows)
    against their PyTorch statement, bit for bit; the combine reads the same slots."""
    ep = _ep(pkg)
    E_r = 256 // world
    ids, w = _routing(T, 11 + world, cuda_dev, hot, world)
    hidden = torch.randint(0, 256, (T, 7168), dtype=torch.uint8, device=cuda_dev)
    hidden[hidden == 0x7F] = 0
    hidden = hidden.view(torch.float8_e4m3fn)
    scale = torch.rand(56, T, device=cuda_dev) + 0.5
    lib, ref = ep.LibPlumbing(), ep.TorchPlumbing()

    c1, s1, src1 = lib.plan(ids, world, E_r, capacity=cap)
    c0, s0, src0 = ref.plan(ids, world, E_r, capacity=cap)
    torch.cuda.synchronize()
    assert torch.equal(c1.cpu(), c0.cpu())
    assert torch.equal(s1.long().cpu(), s0.cpu())
    assert torch.equal(src1.long().cpu(), src0.cpu())
    R = world * cap
    send1 = lib.pack(ids, w, hidden, scale, src1, R, world=world, E_l=E_r, capacity=cap)
    send0 = ref.pack(ids, w, hidden, scale, src0, R, world=world, E_l=E_r, capacity=cap)
    assert torch.equal(send1.cpu(), send0.cpu())
    # padding rows carry ids their receiver does not own
    r_ids = send1[:, 7168 + 224:7168 + 256].contiguous().view(torch.int32).view(R, 8).long().cpu()
    owner = torch.arange(R) // cap
    pad = src0.cpu() < 0
    assert ((r_ids[pad] // E_r) != owner[pad].unsqueeze(1)).all()

    back = torch.randn(R, 7168, device=cuda_dev) * 4
    out1 = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    out0 = torch.empty(T, 7168, dtype=torch.bfloat16, device=cuda_dev)
    lib.combine(back, s1, T, out1)
    ref.combine(back, s0, T, out0)
    assert torch.equal(out1.view(torch.int16).cpu(), out0.view(torch.int16).cpu())
