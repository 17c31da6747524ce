"""Seeded synthetic inputs for the DeepSeek-V3 FP8 block-scale MoE layer.

The reference is measured on the contest's workload dataset, which is not
available here; these generators stand in for it with the shapes, dtypes and
value distributions of the layer definition
``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``
(``config.toml:3``; argument list ``solution/python/kernel.py:95-107``):

* ``routing_logits`` fp32 [T,256] ~ N(0,1); optional skew adds a constant to
  the columns of "hot" experts.
* ``routing_bias`` bf16 [256] = bf16(N(0,1) * 0.1).
* ``hidden_states`` fp32 ~ N(0,1) quantised to e4m3 per 1x128 block
  (scale = amax/448), ``hidden_states_scale`` [56,T].
* ``gemm1_weights`` [E_l,4096,7168] and ``gemm2_weights`` [E_l,7168,2048]
  ~ N(0,1) * K^-1/2, quantised per 128x128 block, scales [E_l,32,56] and
  [E_l,56,16].

Everything is drawn from one ``torch.Generator`` in a fixed order, so a seed
fixes the tensors bit for bit on a given device type.
"""

from __future__ import annotations

import torch

H, I, E_GLOBAL, BLOCK = 7168, 2048, 256, 128
FP8_MAX = 448.0
HOT_EXPERTS_DEFAULT = tuple(range(0, 8)) + tuple(range(32, 40))   # 16 experts in groups 0 and 1


def quant_rows_1x128(x: torch.Tensor):
    """fp32 [T, K] -> (e4m3 [T, K], scale fp32 [K/128, T]) with amax/448 per 1x128 block."""
    T, K = x.shape
    xb = x.view(T, K // BLOCK, BLOCK)
    amax = xb.abs().amax(dim=2)
    s = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (xb / s.unsqueeze(-1)).to(torch.float8_e4m3fn).view(T, K)
    return q, s.t().contiguous()


def quant_block_128x128(w: torch.Tensor):
    """fp32 [N, K] -> (e4m3 [N, K], scale fp32 [N/128, K/128])."""
    N, K = w.shape
    wb = w.view(N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    amax = wb.abs().amax(dim=(1, 3))
    s = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (wb / s.view(N // BLOCK, 1, K // BLOCK, 1)).to(torch.float8_e4m3fn).view(N, K)
    return q, s


@torch.no_grad()
def make_inputs(T: int, E_l: int = 32, local_expert_offset: int = 0, seed: int = 0,
                device: str | torch.device = "cpu", skew: float = 0.0,
                hot_experts=HOT_EXPERTS_DEFAULT, routed_scaling_factor: float = 2.5):
    """Build one call's arguments as a dict keyed by the reference's argument names.

    Tensors are generated on ``device`` with a generator of that device type
    (CPU generation is the portable, fixture-grade path; CUDA generation is
    used by the benchmark to build gigabytes of weights quickly).
    """
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    logits = torch.randn(T, E_GLOBAL, generator=g, device=dev, dtype=torch.float32)
    if skew:
        logits[:, list(hot_experts)] += skew
    bias = (torch.randn(E_GLOBAL, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    hidden = torch.randn(T, H, generator=g, device=dev)
    hs, hs_scale = quant_rows_1x128(hidden)
    del hidden
    w1 = torch.empty(E_l, 2 * I, H, dtype=torch.float8_e4m3fn, device=dev)
    s1 = torch.empty(E_l, 2 * I // BLOCK, H // BLOCK, dtype=torch.float32, device=dev)
    w2 = torch.empty(E_l, H, I, dtype=torch.float8_e4m3fn, device=dev)
    s2 = torch.empty(E_l, H // BLOCK, I // BLOCK, dtype=torch.float32, device=dev)
    for e in range(E_l):
        w = torch.randn(2 * I, H, generator=g, device=dev) * (H ** -0.5)
        w1[e], s1[e] = quant_block_128x128(w)
        w = torch.randn(H, I, generator=g, device=dev) * (I ** -0.5)
        w2[e], s2[e] = quant_block_128x128(w)
        del w
    return dict(
        routing_logits=logits,
        routing_bias=bias,
        hidden_states=hs,
        hidden_states_scale=hs_scale,
        gemm1_weights=w1,
        gemm1_weights_scale=s1,
        gemm2_weights=w2,
        gemm2_weights_scale=s2,
        local_expert_offset=int(local_expert_offset),
        routed_scaling_factor=float(routed_scaling_factor),
    )


@torch.no_grad()
def make_routing_inputs(T: int, seed: int = 0, device: str | torch.device = "cpu",
                        skew: float = 0.0, hot_experts=HOT_EXPERTS_DEFAULT):
    """Only (routing_logits, routing_bias), drawn exactly as the first two
    tensors of ``make_inputs`` with the same seed."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    logits = torch.randn(T, E_GLOBAL, generator=g, device=dev, dtype=torch.float32)
    if skew:
        logits[:, list(hot_experts)] += skew
    bias = (torch.randn(E_GLOBAL, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    return logits, bias


def input_digest(inp: dict) -> str:
    """sha256 over the raw bytes of every tensor argument (CPU tensors)."""
    import hashlib
    h = hashlib.sha256()
    for k in ARG_ORDER:
        v = inp[k]
        if isinstance(v, torch.Tensor):
            h.update(v.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes())
        else:
            h.update(repr(v).encode())
    return h.hexdigest()


@torch.no_grad()
def make_token_inputs(T: int, seed: int = 0, device: str | torch.device = "cpu", skew: float = 0.0,
                      hot_experts=HOT_EXPERTS_DEFAULT):
    """Token-side tensors only: (routing_logits, routing_bias, hidden_states, hidden_states_scale)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    logits = torch.randn(T, E_GLOBAL, generator=g, device=dev, dtype=torch.float32)
    if skew:
        logits[:, list(hot_experts)] += skew
    bias = (torch.randn(E_GLOBAL, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    hidden = torch.randn(T, H, generator=g, device=dev)
    hs, hs_scale = quant_rows_1x128(hidden)
    return logits, bias, hs, hs_scale


@torch.no_grad()
def make_expert_shard(first: int, count: int, seed: int = 0, device: str | torch.device = "cpu"):
    """Weights of global experts [first, first+count), each drawn from its own
    generator (seed, expert id), so any shard of the 256 experts is a slice of
    the same full set.  Returns (w13, s13, w2, s2)."""
    dev = torch.device(device)
    w1 = torch.empty(count, 2 * I, H, dtype=torch.float8_e4m3fn, device=dev)
    s1 = torch.empty(count, 2 * I // BLOCK, H // BLOCK, dtype=torch.float32, device=dev)
    w2 = torch.empty(count, H, I, dtype=torch.float8_e4m3fn, device=dev)
    s2 = torch.empty(count, H // BLOCK, I // BLOCK, dtype=torch.float32, device=dev)
    for i in range(count):
        g = torch.Generator(device=dev).manual_seed(seed * 1_000_003 + first + i)
        w = torch.randn(2 * I, H, generator=g, device=dev) * (H ** -0.5)
        w1[i], s1[i] = quant_block_128x128(w)
        w = torch.randn(H, I, generator=g, device=dev) * (I ** -0.5)
        w2[i], s2[i] = quant_block_128x128(w)
        del w
    return w1, s1, w2, s2


ARG_ORDER = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
             "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale",
             "local_expert_offset", "routed_scaling_factor")


def bench_batch(T_base: int, skew: float = 0.0, device: str | torch.device = "cuda"):
    """The benchmark's synthetic batch: ``T_base`` tokens and 32 local experts
    (offset 0) drawn from seed 0 on ``device``; ``skew`` > 0 gives the skewed
    stress batch (logits of experts 0-7 and 32-39 raised by ``skew``)."""
    return make_inputs(T_base, E_l=32, local_expert_offset=0, seed=0, device=device, skew=skew)


def token_slice(base: dict, T: int) -> dict:
    """The first ``T`` tokens of a batch (weights shared)."""
    d = dict(base)
    d["routing_logits"] = base["routing_logits"][:T].contiguous()
    d["hidden_states"] = base["hidden_states"][:T].contiguous()
    d["hidden_states_scale"] = base["hidden_states_scale"][:, :T].contiguous()
    return d


def as_args(inp: dict):
    """The positional argument tuple of ``kernel(...)`` (without ``output``)."""
    return tuple(inp[k] for k in ARG_ORDER)
