"""CPU: the PyTorch statement of the expert-parallel plumbing (the checker the
library's kernels are compared with bit for bit on the GPU) against a plain
per-token loop, for 2, 4 and 8 ranks, plus a pack -> unpack round trip."""

from __future__ import annotations

import pytest
import torch


def _ep():
    import __graft_entry__ as ge
    ge.load_package()
    return __import__("fib_b200.ep", fromlist=["ep"])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_plan_matches_loop(world):
    ep = _ep()
    g = torch.Generator().manual_seed(world)
    T = 37
    ids = torch.stack([torch.randperm(256, generator=g)[:8].sort().values for _ in range(T)]).to(torch.int32)
    E_r = 256 // world
    counts, slot, src = ep.plan_rows(ids, world, E_r)
    # plain loop: rank-major, tokens ascending, one row per (token, rank) pair
    rows = []
    for r in range(world):
        for t in range(T):
            if any(int(e) // E_r == r for e in ids[t]):
                rows.append((r, t))
    assert int(counts.sum()) == len(rows)
    for r in range(world):
        assert int(counts[r]) == sum(1 for rr, _ in rows if rr == r)
    assert src.tolist() == [t for _, t in rows]
    for i, (r, t) in enumerate(rows):
        assert int(slot[t, r]) == i
    assert int((slot >= 0).sum()) == len(rows)


def test_pack_unpack_round_trip():
    ep = _ep()
    g = torch.Generator().manual_seed(3)
    T, world = 19, 4
    ids = torch.stack([torch.randperm(256, generator=g)[:8].sort().values for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, 8, generator=g)
    hidden = torch.randint(0, 256, (T, 7168), generator=g, dtype=torch.uint8).view(torch.float8_e4m3fn)
    scale = torch.rand(56, T, generator=g)
    send, counts, src, slot = ep.pack_rows(ids, w, hidden, scale, world, 256 // world)
    assert send.shape == (int(counts.sum()), ep.ROW_BYTES)
    h2, s2, i2, w2 = ep.unpack_rows(send)
    assert torch.equal(h2.view(torch.uint8), hidden.view(torch.uint8)[src])
    assert torch.equal(s2, scale[:, src])
    assert torch.equal(i2, ids[src])
    assert torch.equal(w2, w[src])


@pytest.mark.parametrize("world,cap", [(2, 37), (4, 40), (8, 37)])
def test_fixed_capacity_plan_matches_compact(world, cap):
    """The fixed-capacity layout holds the compact layout's rows, rank r's block
    shifted to r * cap, padding (-1) after them; padding rows pack to zero rows
    whose expert ids the receiving rank does not own."""
    ep = _ep()
    g = torch.Generator().manual_seed(17 + world)
    T = 37
    ids = torch.stack([torch.randperm(256, generator=g)[:8].sort().values for _ in range(T)]).to(torch.int32)
    E_r = 256 // world
    c0, s0, src0 = ep.plan_rows(ids, world, E_r)
    c1, s1, src1 = ep.plan_rows(ids, world, E_r, capacity=cap)
    assert torch.equal(c0, c1)
    assert src1.shape == (world * cap,)
    base = torch.cumsum(c0, 0) - c0
    for r in range(world):
        n = int(c0[r])
        assert torch.equal(src1[r * cap:r * cap + n], src0[int(base[r]):int(base[r]) + n])
        assert (src1[r * cap + n:(r + 1) * cap] == -1).all()
    has = s0 >= 0
    shift = (torch.arange(world) * cap).unsqueeze(0) - base.unsqueeze(0)
    assert torch.equal(s1[has], (s0 + shift)[has])
    assert (s1[~has] == -1).all()
    w = torch.rand(T, 8, generator=g)
    hidden = torch.randint(0, 256, (T, 7168), generator=g, dtype=torch.uint8).view(torch.float8_e4m3fn)
    scale = torch.rand(56, T, generator=g)
    send = ep.gather_rows(ids, w, hidden, scale, src1, world, E_r, cap)
    h, sc, i2, w2 = ep.unpack_rows(send)
    pad = src1 < 0
    assert (h.view(torch.uint8)[pad] == 0).all() and (sc[:, pad] == 0).all() and (w2[pad] == 0).all()
    owner = torch.arange(world * cap) // cap
    assert ((i2[pad].long() // E_r) != owner[pad].unsqueeze(1)).all()
    real = ~pad
    assert torch.equal(i2[real], ids[src1[real]])
