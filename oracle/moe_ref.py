"""CPU oracle for the fused FP8 block-scale DeepSeek-V3 MoE layer.

TEST INFRASTRUCTURE ONLY.  This module is the checker the CUDA path is
compared against; it is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product path never calls it and has no CPU
fallback.

It restates, in plain fp32 torch-on-CPU arithmetic, the reference layer
definition ``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``:

* ATen statement of the math: ``solution/cuda/moe.cu:137-240``
  (dequantise, route, per-expert fp32 GEMMs, SwiGLU, index_add, bf16 cast).
* Routing as the contest definition writes it:
  ``flashinfer/trace/templates/moe.py:109-185`` of flashinfer-python
  0.6.11.post2 (third-party, installed in the build image, not vendored in
  the reference): ``s = 1/(1+exp(-x))`` rather than ``at::sigmoid``, and
  unsorted top-k.  The in-reference Triton routing
  (``solution/triton/kernel.py:42-117``) and the CUDA routing
  (``solution/python/kernel.cu:56-200``) compute the same selection.

Pinning: ``tests/golden/make_golden.py`` runs the flashinfer reference
function on seeded inputs and commits its outputs as fixtures; the
``-m "not gpu"`` tests check this restatement against those fixtures.
"""

from __future__ import annotations

import torch

H = 7168            # hidden size            (moe.cu:150)
I = 2048            # intermediate size      (moe.cu:151)
BLOCK = 128         # quantisation block     (moe.cu:152)
E_GLOBAL = 256      # experts                (moe.cu:153)
TOP_K = 8           # experts per token      (moe.cu:154)
N_GROUP = 8         # routing groups         (moe.cu:155)
TOPK_GROUP = 4      # kept groups            (moe.cu:156)
FP8_MAX = 448.0     # largest finite e4m3fn value


# --------------------------------------------------------------------------
# FP8 e4m3fn decode (moe.cu:24-42): sign 1, exponent 4 (bias 7), mantissa 3,
# no infinities, 0x7f / 0xff are NaN, exponent 0 is subnormal (m * 2^-9).
# --------------------------------------------------------------------------
def _e4m3_table() -> torch.Tensor:
    vals = []
    for b in range(256):
        sign = -1.0 if b & 0x80 else 1.0
        exp = (b >> 3) & 0xF
        man = b & 0x7
        if exp == 0xF and man == 0x7:
            v = float("nan")
        elif exp == 0:
            v = sign * man * 2.0 ** -9
        else:
            v = sign * (8 + man) * 2.0 ** (exp - 10)
        vals.append(v)
    return torch.tensor(vals, dtype=torch.float32)


E4M3_TABLE = _e4m3_table()


def fp8_to_f32(x: torch.Tensor) -> torch.Tensor:
    """Decode an fp8 e4m3fn (or uint8 bit pattern) tensor to fp32 by table."""
    u8 = x.view(torch.uint8) if x.dtype != torch.uint8 else x
    return E4M3_TABLE[u8.long()]


# --------------------------------------------------------------------------
# Routing (flashinfer moe.py:140-170; moe.cu:178-206)
# --------------------------------------------------------------------------
def exp_correctly_rounded(x: torch.Tensor) -> torch.Tensor:
    """fp32 exp rounded once from a float64 evaluation (correct rounding except in
    cases closer to a rounding boundary than float64's own error, none of which
    occur in the tests' inputs)."""
    return torch.exp(x.to(torch.float64)).to(torch.float32)


def route(routing_logits: torch.Tensor, routing_bias: torch.Tensor,
          routed_scaling_factor: float, exp=torch.exp):
    """DeepSeek-V3 no-aux routing.

    Returns ``(topk_idx int64 [T,8], topk_w fp32 [T,8], dense_w fp32 [T,256])``.
    ``topk_idx`` is sorted ascending per token (the reference's top-k is
    unsorted, so only the set is defined); ``topk_w[t,k]`` is the weight of
    expert ``topk_idx[t,k]``.

    ``exp`` is the definition's ``torch.exp`` on CPU by default.  That function
    is not correctly rounded (on an MKL build of torch it is MKL's ``vsExp``,
    about 1% of results one ulp away from the correctly rounded value), so
    ``exp=exp_correctly_rounded`` gives the same definition with a correctly
    rounded exponential, which is what the CUDA routing computes.
    """
    T = routing_logits.shape[0]
    logits = routing_logits.to(torch.float32)
    bias = routing_bias.to(torch.float32).reshape(-1)
    s = 1.0 / (1.0 + exp(-logits))
    s_with_bias = s + bias
    gsz = E_GLOBAL // N_GROUP
    top2 = torch.topk(s_with_bias.view(T, N_GROUP, gsz), k=2, dim=2, sorted=False).values
    group_scores = top2.sum(dim=2)
    group_idx = torch.topk(group_scores, k=TOPK_GROUP, dim=1, sorted=False).indices
    group_mask = torch.zeros_like(group_scores)
    group_mask.scatter_(1, group_idx, 1.0)
    score_mask = group_mask.unsqueeze(2).expand(T, N_GROUP, gsz).reshape(T, E_GLOBAL)
    pruned = s_with_bias.masked_fill(score_mask == 0, torch.finfo(torch.float32).min)
    topk_idx = torch.topk(pruned, k=TOP_K, dim=1, sorted=False).indices
    return _route_weights(s, topk_idx, routed_scaling_factor)


def _route_weights(s: torch.Tensor, topk_idx: torch.Tensor, routed_scaling_factor: float):
    """Weights of the picked experts: s / (sum of the picked s + 1e-20) * scale,
    summed as a dense [T,256] row (flashinfer ``moe.py:109-185``)."""
    M = torch.zeros_like(s)
    M.scatter_(1, topk_idx, 1.0)
    raw = s * M
    dense_w = (raw / (raw.sum(dim=1, keepdim=True) + 1e-20)) * routed_scaling_factor
    topk_idx = topk_idx.sort(dim=1).values
    topk_w = dense_w.gather(1, topk_idx)
    return topk_idx, topk_w, dense_w


def route_lowest_id_ties(routing_logits: torch.Tensor, routing_bias: torch.Tensor,
                         routed_scaling_factor: float, exp=torch.exp):
    """``route`` with ties resolved as the reference's CUDA routing kernel does.

    ``torch.topk`` leaves the order of equal scores unspecified, so on inputs
    with exact ties the definition picks an implementation-defined set.  The
    reference's own kernel (``solution/python/kernel.cu:84-160``) keeps the
    lower group when group scores tie (strict ``>`` scan, ``:101-110``) and the
    lower expert id when scores tie (``__ffs`` of the ballot of equal lanes,
    ``:117-130`` inside a group, ``:147-160`` across groups), i.e. a stable
    descending sort.  Without ties this returns exactly what ``route`` does.
    """
    T = routing_logits.shape[0]
    logits = routing_logits.to(torch.float32)
    bias = routing_bias.to(torch.float32).reshape(-1)
    s = 1.0 / (1.0 + exp(-logits))
    s_with_bias = s + bias
    gsz = E_GLOBAL // N_GROUP
    top2 = torch.topk(s_with_bias.view(T, N_GROUP, gsz), k=2, dim=2, sorted=True).values
    group_scores = top2[..., 0] + top2[..., 1]
    group_idx = torch.sort(group_scores, dim=1, descending=True, stable=True).indices[:, :TOPK_GROUP]
    group_mask = torch.zeros_like(group_scores)
    group_mask.scatter_(1, group_idx, 1.0)
    score_mask = group_mask.unsqueeze(2).expand(T, N_GROUP, gsz).reshape(T, E_GLOBAL)
    pruned = s_with_bias.masked_fill(score_mask == 0, -float("inf"))
    topk_idx = torch.sort(pruned, dim=1, descending=True, stable=True).indices[:, :TOP_K]
    return _route_weights(s, topk_idx, routed_scaling_factor)


# --------------------------------------------------------------------------
# Dequantisation (moe.cu:52-91, 164-176)
# --------------------------------------------------------------------------
def dequant_hidden(hidden_states: torch.Tensor, hidden_states_scale: torch.Tensor) -> torch.Tensor:
    """fp8 [T,H] with scale [H/128, T] -> fp32 [T,H]."""
    T = hidden_states.shape[0]
    a = fp8_to_f32(hidden_states)
    sc = hidden_states_scale.to(torch.float32).t().contiguous()      # [T, H/128]
    return (a.view(T, H // BLOCK, BLOCK) * sc.unsqueeze(-1)).view(T, H)


def dequant_weight(w: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp8 [rows, cols] with scale [rows/128, cols/128] -> fp32 [rows, cols]."""
    rows, cols = w.shape
    f = fp8_to_f32(w).view(rows // BLOCK, BLOCK, cols // BLOCK, BLOCK)
    return (f * scale.to(torch.float32).view(rows // BLOCK, 1, cols // BLOCK, 1)).view(rows, cols)


def swiglu(g1: torch.Tensor) -> torch.Tensor:
    """silu(X2) * X1 with X1 = g1[:, :I], X2 = g1[:, I:]  (moe.cu:227-229)."""
    x1, x2 = g1[:, :I], g1[:, I:]
    return x2 / (1.0 + torch.exp(-x2)) * x1


# --------------------------------------------------------------------------
# Whole layer (moe.cu:137-240)
# --------------------------------------------------------------------------
@torch.no_grad()
def experts_forward(topk_idx, topk_w, hidden_states, hidden_states_scale,
                    gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                    local_expert_offset: int):
    """Contribution of the local experts for a given routing (moe.cu:208-236):
    fp32 [T, H] = sum over local picks, in ascending expert order, of w * expert(x)."""
    T = hidden_states.shape[0]
    E_l = gemm1_weights.shape[0]
    A = dequant_hidden(hidden_states, hidden_states_scale)
    acc = torch.zeros(T, H, dtype=torch.float32)
    for le in range(E_l):
        ge = local_expert_offset + le
        if ge < 0 or ge >= E_GLOBAL:
            continue
        hit = topk_idx == ge
        sel = hit.any(dim=1)
        if not bool(sel.any()):
            continue
        tok = sel.nonzero().squeeze(1)
        w_tok = (topk_w * hit.float()).sum(dim=1).index_select(0, tok)
        W13 = dequant_weight(gemm1_weights[le], gemm1_weights_scale[le])
        W2 = dequant_weight(gemm2_weights[le], gemm2_weights_scale[le])
        g1 = A.index_select(0, tok).matmul(W13.t())
        o = swiglu(g1).matmul(W2.t())
        acc.index_add_(0, tok, o * w_tok.unsqueeze(1))
    return acc


@torch.no_grad()
def moe_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                local_expert_offset: int, routed_scaling_factor: float,
                return_fp32: bool = False):
    """Reference forward on CPU (moe.cu:137-240).  Returns bf16 [T, H] (or the
    fp32 accumulator).  Only experts that receive a token are dequantised,
    which changes the cost, not the result, of the reference's full
    dequantisation."""
    topk_idx, topk_w, _ = route(routing_logits, routing_bias, routed_scaling_factor)
    acc = experts_forward(topk_idx, topk_w, hidden_states, hidden_states_scale, gemm1_weights,
                          gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset)
    return acc if return_fp32 else acc.to(torch.bfloat16)


# --------------------------------------------------------------------------
# Stage-level helpers used by the stage-parity tests
# --------------------------------------------------------------------------
def local_assignments(topk_idx: torch.Tensor, local_expert_offset: int, E_l: int):
    """Deterministic permutation the CUDA path builds: rows grouped by local
    expert, tokens ascending inside an expert.

    Returns ``(seg_offsets int64 [E_l+1], row_token int64 [R], row_k int64 [R],
    inv int64 [T,8])``, ``inv[t,k] = row`` or ``-1`` for a non-local pick.
    """
    T = topk_idx.shape[0]
    le = topk_idx - local_expert_offset
    local = (le >= 0) & (le < E_l)
    counts = torch.zeros(E_l, dtype=torch.int64)
    for e in range(E_l):
        counts[e] = int((le == e).sum())
    seg = torch.zeros(E_l + 1, dtype=torch.int64)
    seg[1:] = torch.cumsum(counts, 0)
    inv = torch.full((T, TOP_K), -1, dtype=torch.int64)
    row_token = torch.zeros(int(seg[-1]), dtype=torch.int64)
    row_k = torch.zeros(int(seg[-1]), dtype=torch.int64)
    fill = seg[:-1].clone()
    for t in range(T):
        for k in range(TOP_K):
            if bool(local[t, k]):
                e = int(le[t, k])
                r = int(fill[e])
                fill[e] += 1
                inv[t, k] = r
                row_token[r] = t
                row_k[r] = k
    return seg, row_token, row_k, inv


def quant_hilo(c: torch.Tensor):
    """Two-term 1x128 fp8 quantisation of the SwiGLU output used by the CUDA
    path between the two GEMMs: ``c ~= hi*s + lo*(s/16)`` with
    ``s = amax/448`` per 128-column block (1.0 for an all-zero block).

    Returns ``(hi fp8 [R, I], lo fp8 [R, I], s fp32 [R, I/128])``.
    The single-term fp8 requantisation of ``kernel.cu:1086-1145`` is ``hi``
    alone; the residual term ``lo`` keeps the layer inside the fp32-reference
    tolerance.
    """
    R = c.shape[0]
    cb = c.view(R, I // BLOCK, BLOCK)
    amax = cb.abs().amax(dim=2)
    s = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    hi = (cb * (1.0 / s).unsqueeze(-1)).to(torch.float8_e4m3fn)
    hi_f = fp8_to_f32(hi)
    resid = cb - hi_f * s.unsqueeze(-1)
    lo = (resid * (16.0 / s).unsqueeze(-1)).to(torch.float8_e4m3fn)
    return hi.view(R, I), lo.view(R, I), s
