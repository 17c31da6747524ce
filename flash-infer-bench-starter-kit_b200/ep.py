"""Expert-parallel MoE layer: one process per GPU, experts sharded by rank.

The reference has no multi-GPU path (its only hook is ``local_expert_offset``,
``solution/python/kernel.py:104``).  Here the 256 experts are split evenly
over the ``world`` ranks of a process group (rank r owns global experts
``[r*E_l, (r+1)*E_l)``, ``E_l = 256/world``) and every rank brings its own
batch of tokens:

1. route the local tokens (fused routing kernel);
2. dispatch: each token row goes, once, to every rank that owns at least one
   of its 8 experts, packed with its 1x128 scales, ids and weights;
   per-destination row counts are exchanged first so the row all-to-all
   moves only real rows;
3. each rank runs the layer's expert part (``moe_fp8_ds_run_routed``) on the
   rows it received, for its own experts only;
4. combine: partial results go back to the token's home rank, which sums
   them in ascending rank order in fp32 and writes bf16.

Rows are ordered by (destination rank, token) and the combine sums in a fixed
rank order, so the result is deterministic.  The exchange uses
``torch.distributed`` collectives (NCCL over NVLink on GPUs, gloo on CPU for
the protocol tests); the per-rank compute is injected, so the same protocol
code runs with the CUDA library on GPUs and with the CPU oracle in tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

H, I, E_GLOBAL, TOP_K = 7168, 2048, 256, 8
SCALE_BYTES = (H // 128) * 4                    # 56 fp32 scales per row
ROW_BYTES = H + SCALE_BYTES + TOP_K * 4 + TOP_K * 4   # hidden | scales | ids | weights = 7456


def pack_rows(ids, w, hidden, hidden_scale, world, E_l):
    """Build the dispatch rows.

    Returns ``(send [S, ROW_BYTES] uint8, counts [world] int64, src_token [S] int64,
    slot [T, world] int64)``: rows grouped by destination rank, tokens ascending
    inside a group; ``slot[t, r]`` is the row of token t sent to rank r, or -1.
    """
    T = ids.shape[0]
    dev = ids.device
    owner = ids.long() // E_l                                   # [T, 8]
    dest = torch.zeros(T, world, dtype=torch.bool, device=dev)
    dest.scatter_(1, owner, True)
    counts = dest.sum(0)
    rt = dest.t().nonzero()                                     # (rank, token) sorted by rank, token
    src_token = rt[:, 1]
    slot = torch.full((T, world), -1, dtype=torch.long, device=dev)
    slot[rt[:, 1], rt[:, 0]] = torch.arange(rt.shape[0], device=dev)
    scale_rows = hidden_scale.t()                               # [T, 56] view
    send = torch.cat([
        hidden.view(torch.uint8).index_select(0, src_token),
        scale_rows.index_select(0, src_token).contiguous().view(torch.uint8),
        ids.to(torch.int32).index_select(0, src_token).contiguous().view(torch.uint8),
        w.to(torch.float32).index_select(0, src_token).contiguous().view(torch.uint8),
    ], dim=1)
    return send, counts, src_token, slot


def unpack_rows(recv):
    """Split received rows into the layer's argument layout."""
    R = recv.shape[0]
    hidden = recv[:, :H].contiguous().view(torch.float8_e4m3fn)
    scale = recv[:, H:H + SCALE_BYTES].contiguous().view(torch.float32).t().contiguous()   # [56, R]
    off = H + SCALE_BYTES
    ids = recv[:, off:off + TOP_K * 4].contiguous().view(torch.int32).view(R, TOP_K)
    w = recv[:, off + TOP_K * 4:].contiguous().view(torch.float32).view(R, TOP_K)
    return hidden, scale, ids, w


def combine_rows(back, slot, T):
    """out[t] = sum over ranks r ascending of back[slot[t, r]] (fp32)."""
    acc = torch.zeros(T, H, dtype=torch.float32, device=back.device)
    for r in range(slot.shape[1]):
        s = slot[:, r]
        has = s >= 0
        if bool(has.any()):
            rows = back.index_select(0, s.clamp_min(0)).float()
            acc += torch.where(has.unsqueeze(1), rows, torch.zeros((), device=back.device))
    return acc


def exchange(send, counts, group=None):
    """Count exchange then variable-size row all-to-all.  Returns (recv, in_splits, out_splits)."""
    world = dist.get_world_size(group)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    in_splits = counts.tolist()
    out_splits = recv_counts.tolist()
    recv = torch.empty(sum(out_splits), send.shape[1], dtype=send.dtype, device=send.device)
    dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)
    del world
    return recv, in_splits, out_splits


class ExpertParallelMoE:
    """One rank of the expert-parallel layer.

    ``route_fn(logits, bias, scale) -> (ids int32 [T,8] ascending, w fp32 [T,8])`` and
    ``expert_fn(ids, w, hidden, hidden_scale, w13, s13, w2, s2, offset) -> partial [R, H]``
    supply the per-rank compute; ``from_library`` wires the CUDA library.
    """

    def __init__(self, route_fn, expert_fn, group=None):
        self.route_fn = route_fn
        self.expert_fn = expert_fn
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E_GLOBAL % self.world:
            raise ValueError(f"{E_GLOBAL} experts do not split over {self.world} ranks")
        self.E_l = E_GLOBAL // self.world
        self.last_stats = {}

    @torch.no_grad()
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                routed_scaling_factor, output):
        if gemm1_weights.shape[0] != self.E_l:
            raise ValueError(f"rank holds {gemm1_weights.shape[0]} experts, expected {self.E_l}")
        T = hidden_states.shape[0]
        ids, w = self.route_fn(routing_logits, routing_bias, routed_scaling_factor)
        send, counts, src_token, slot = pack_rows(ids, w, hidden_states, hidden_states_scale,
                                                  self.world, self.E_l)
        recv, in_splits, out_splits = exchange(send, counts, self.group)
        r_hidden, r_scale, r_ids, r_w = unpack_rows(recv)
        part = self.expert_fn(r_ids, r_w, r_hidden, r_scale, gemm1_weights, gemm1_weights_scale,
                              gemm2_weights, gemm2_weights_scale, self.rank * self.E_l)
        back = torch.empty(send.shape[0], H, dtype=part.dtype, device=part.device)
        dist.all_to_all_single(back, part, in_splits, out_splits, group=self.group)
        acc = combine_rows(back, slot, T)
        output.copy_(acc.to(output.dtype))
        self.last_stats = {"sent_rows": int(send.shape[0]), "recv_rows": int(recv.shape[0])}
        return output

    __call__ = forward


def from_library(group=None, partial_dtype=torch.bfloat16):
    """ExpertParallelMoE whose routing and expert compute run in libmoe_fp8_ds.so."""
    import ctypes
    import importlib
    from . import _lib
    K = importlib.import_module(__package__ + ".kernel")   # the module, not the kernel() function

    def route_fn(logits, bias, scale):
        T = logits.shape[0]
        ids = torch.empty(T, TOP_K, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, TOP_K, dtype=torch.float32, device=logits.device)
        if T:
            _lib.check(_lib.load().moe_fp8_ds_route(
                ctypes.c_void_p(logits.data_ptr()), ctypes.c_void_p(bias.data_ptr()), T,
                ctypes.c_float(scale), ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "moe_fp8_ds_route")
        return ids, w

    def expert_fn(ids, w, hidden, scale, w13, s13, w2, s2, offset):
        R = hidden.shape[0]
        if partial_dtype == torch.float32:
            out = torch.empty(R, H, dtype=torch.float32, device=hidden.device)
            args = K.build_args(None, None, hidden, scale, w13, s13, w2, s2, offset, 1.0, None,
                                topk_ids=ids, topk_weights=w, output_f32=out)
        else:
            out = torch.empty(R, H, dtype=torch.bfloat16, device=hidden.device)
            args = K.build_args(None, None, hidden, scale, w13, s13, w2, s2, offset, 1.0, out,
                                topk_ids=ids, topk_weights=w)
        if R:
            ws = K.get_workspace(hidden.device, K.workspace_bytes(R, w13.shape[0]))
            K.run_with_workspace(args, ws, routed=True)
        return out

    return ExpertParallelMoE(route_fn, expert_fn, group)
