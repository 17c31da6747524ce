"""CPU: routing when scores tie exactly.

The definition's top-k (``torch.topk``) leaves the order of equal scores open; the
reference's CUDA routing kernel (``solution/python/kernel.cu:84-160``) resolves it toward
the lower group and the lower expert id, and so does this library's ``route_token``.
``oracle.route_lowest_id_ties`` states that rule as a stable sort; here it is checked
against (a) a step-by-step restatement of the kernel's warp procedure on tied inputs and
(b) the reference definition's golden routing, where nothing ties.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden, tied_routing_inputs

ROUTE = ["route_T4096_s3", "route_T2048_skew_s4"]


def _kernel_procedure(sb_row: list[float]) -> list[int]:
    """The selection steps of ``kernel.cu:84-160`` for one token, in plain Python:
    a warp per group of 32 experts, lane = expert within the group."""
    inf = float("inf")
    # group score: the maximum, then the maximum with the lowest lane holding it removed
    gs = []
    for g in range(8):
        v = sb_row[g * 32:(g + 1) * 32]
        m1 = max(v)
        l1 = v.index(m1)
        m2 = max(x for i, x in enumerate(v) if i != l1)
        gs.append(m1 + m2)
    # four rounds of a strict ">" scan: the lower group keeps a tie
    tmp = list(gs)
    kept = set()
    for _ in range(4):
        best, bv = 0, tmp[0]
        for g in range(1, 8):
            if tmp[g] > bv:
                best, bv = g, tmp[g]
        kept.add(best)
        tmp[best] = -inf
    # eight candidates per group: each round the lowest lane holding the maximum
    cand_v, cand_i = [], []
    for g in range(8):
        cur = [x if g in kept else -inf for x in sb_row[g * 32:(g + 1) * 32]]
        for _ in range(8):
            m = max(cur)
            lane = cur.index(m)
            cand_v.append(m)
            cand_i.append(g * 32 + lane)
            cur[lane] = -inf
    # merge of the 64 candidates: lane l holds candidates 2l and 2l+1
    v0 = [cand_v[2 * l] for l in range(32)]
    v1 = [cand_v[2 * l + 1] for l in range(32)]
    picks = []
    for _ in range(8):
        pick0 = [v0[l] >= v1[l] for l in range(32)]
        v = [v0[l] if pick0[l] else v1[l] for l in range(32)]
        gmax = max(v)
        w = v.index(gmax)
        picks.append(cand_i[2 * w] if pick0[w] else cand_i[2 * w + 1])
        if pick0[w]:
            v0[w] = -inf
        else:
            v1[w] = -inf
    return sorted(picks)


@pytest.mark.parametrize("seed,bias_grid", [(0, False), (1, True), (2, False)])
def test_lowest_id_rule_matches_kernel_procedure(seed, bias_grid, oracle):
    logits, bias = tied_routing_inputs(96, seed, bias_grid)
    ids, w, _ = oracle.route_lowest_id_ties(logits, bias, 2.5)
    s = 1.0 / (1.0 + torch.exp(-logits))
    sb = (s + bias.float()).tolist()
    want = torch.tensor([_kernel_procedure(row) for row in sb])
    assert torch.equal(ids, want)
    # the inputs do tie: the definition's unordered top-k picks other sets
    ids_topk, _, _ = oracle.route(logits, bias, 2.5)
    assert not torch.equal(ids_topk, ids)
    # every pick carries its own weight; the weights add up to the scaling factor
    assert torch.allclose(w.sum(dim=1), torch.full((96,), 2.5), rtol=1e-6)


@pytest.mark.parametrize("name", ROUTE)
def test_lowest_id_rule_equals_definition_without_ties(name, pkg, oracle):
    g = load_golden(name)
    logits, bias = pkg.inputs.make_routing_inputs(g["T"], seed=g["seed"], skew=g["skew"])
    ids, w, _ = oracle.route_lowest_id_ties(logits, bias, 2.5)
    assert torch.equal(ids.to(torch.int32), g["topk_ids"])
    assert torch.equal(w, g["topk_w"])
