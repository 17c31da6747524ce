"""Expert-parallel MoE layer: one process per GPU, experts sharded by rank.

The reference has no multi-GPU path (its only hook is ``local_expert_offset``,
``solution/python/kernel.py:104``).  Here the 256 experts are split evenly
over the ``world`` ranks of a process group (rank r owns global experts
``[r*E_l, (r+1)*E_l)``, ``E_l = 256/world``) and every rank brings its own
batch of tokens:

1. route the local tokens (fused routing kernel);
2. dispatch: each token row goes, once, to every rank that owns at least one
   of its 8 experts, packed with its 1x128 scales, ids and weights.  With a
   fixed ``capacity`` (the most tokens any rank brings to a step) every peer
   gets ``capacity`` rows, real rows first and padding rows after (zero, with
   expert ids the receiver does not own), so both all-to-alls have fixed
   sizes and a step never waits for the device on the host.  Without one,
   per-destination row counts are exchanged first and read on the host, so
   the row all-to-all moves only real rows;
3. each rank runs the layer's expert part (``moe_fp8_ds_run_routed``) on the
   rows it received, for its own experts only;
4. combine: partial results go back to the token's home rank in fp32 (each
   rank's unrounded sum over its own experts), which sums them in ascending
   rank order in fp32 and rounds to bf16 once, as the single-GPU layer does.

Rows are ordered by (destination rank, token) and the combine sums in a fixed
rank order, so the result is deterministic.  The exchange uses
``torch.distributed`` collectives (NCCL over NVLink on GPUs, gloo on CPU for
the protocol tests).  The per-rank compute and the plan/pack/unpack/combine
steps are injected: ``from_library`` runs all of them as kernels of
libmoe_fp8_ds.so, the protocol tests run the PyTorch statement of the same
steps (``TorchPlumbing``) with the CPU oracle.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

H, I, E_GLOBAL, TOP_K = 7168, 2048, 256, 8
SCALE_BYTES = (H // 128) * 4                    # 56 fp32 scales per row
ROW_BYTES = H + SCALE_BYTES + TOP_K * 4 + TOP_K * 4   # hidden | scales | ids | weights = 7456


def plan_rows(ids, world, E_l, capacity=None):
    """Dispatch plan: ``(counts [world] int64, slot [T, world] int64, src_token int64)``.

    Rows are grouped by destination rank, tokens ascending inside a group;
    ``slot[t, r]`` is the send row of token t for rank r, or -1.  Compact
    layout: ``src_token`` has ``sum(counts)`` rows.  With ``capacity``: rank
    r's rows start at ``r * capacity`` and ``src_token`` has ``world *
    capacity`` rows, -1 for padding.
    """
    T = ids.shape[0]
    dev = ids.device
    owner = ids.long() // E_l                                   # [T, 8]
    dest = torch.zeros(T, world, dtype=torch.bool, device=dev)
    dest.scatter_(1, owner, True)
    counts = dest.sum(0)
    rt = dest.t().nonzero()                                     # (rank, token) sorted by rank, token
    row = torch.arange(rt.shape[0], device=dev)
    if capacity is None:
        src_token = rt[:, 1]
    else:
        row = rt[:, 0] * capacity + row - (torch.cumsum(counts, 0) - counts)[rt[:, 0]]
        src_token = torch.full((world * capacity,), -1, dtype=torch.long, device=dev)
        src_token[row] = rt[:, 1]
    slot = torch.full((T, world), -1, dtype=torch.long, device=dev)
    slot[rt[:, 1], rt[:, 0]] = row
    return counts, slot, src_token


def gather_rows(ids, w, hidden, hidden_scale, src_token, world=None, E_l=None, capacity=None):
    """Send rows ``[S, ROW_BYTES]`` uint8 for the tokens ``src_token``; a -1
    (fixed-capacity padding) gives a zero row whose 8 expert ids are the first
    expert of the next rank, which the receiving rank ``row // capacity``
    does not own."""
    scale_rows = hidden_scale.t()                               # [T, 56] view
    pad = src_token < 0
    S, dev = src_token.shape[0], src_token.device
    if hidden.shape[0] == 0:     # no tokens: every row is padding
        ids_rows = torch.zeros(S, TOP_K, dtype=torch.int32, device=dev)
        w_rows = torch.zeros(S, TOP_K, dtype=torch.float32, device=dev)
        hid = torch.zeros(S, H, dtype=torch.uint8, device=dev)
        sc = torch.zeros(S, H // 128, dtype=torch.float32, device=dev)
    else:
        src = src_token.clamp_min(0)
        ids_rows = ids.to(torch.int32).index_select(0, src)
        w_rows = w.to(torch.float32).index_select(0, src)
        hid = hidden.view(torch.uint8).index_select(0, src)
        sc = scale_rows.index_select(0, src).contiguous()
    if bool(pad.any()):
        r = torch.arange(src_token.shape[0], device=src_token.device) // capacity
        foreign = ((r + 1) % world * E_l).to(torch.int32)
        ids_rows = torch.where(pad.unsqueeze(1), foreign.unsqueeze(1).expand_as(ids_rows), ids_rows)
        w_rows = torch.where(pad.unsqueeze(1), torch.zeros((), dtype=w_rows.dtype, device=w_rows.device), w_rows)
        hid = torch.where(pad.unsqueeze(1), torch.zeros((), dtype=hid.dtype, device=hid.device), hid)
        sc = torch.where(pad.unsqueeze(1), torch.zeros((), dtype=sc.dtype, device=sc.device), sc)
    return torch.cat([hid, sc.view(torch.uint8), ids_rows.contiguous().view(torch.uint8),
                      w_rows.contiguous().view(torch.uint8)], dim=1)


def pack_rows(ids, w, hidden, hidden_scale, world, E_l):
    """``(send [S, ROW_BYTES] uint8, counts, src_token, slot)``, see ``plan_rows``."""
    counts, slot, src_token = plan_rows(ids, world, E_l)
    return gather_rows(ids, w, hidden, hidden_scale, src_token), counts, src_token, slot


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
    """out[t] = sum over ranks r ascending of back[slot[t, r]] (fp32, from +0)."""
    acc = torch.zeros(T, H, dtype=torch.float32, device=back.device)
    for r in range(slot.shape[1]):
        s = slot[:, r].long()
        has = s >= 0
        if bool(has.any()):
            rows = back.index_select(0, s.clamp_min(0)).float()
            acc += torch.where(has.unsqueeze(1), rows, torch.zeros((), device=back.device))
    return acc


class TorchPlumbing:
    """Plan/pack/unpack/combine in PyTorch: the protocol on CPU (gloo tests)
    and the checker the library's kernels are tested against."""

    def plan(self, ids, world, E_l, capacity=None):
        return plan_rows(ids, world, E_l, capacity)

    def pack(self, ids, w, hidden, hidden_scale, src_token, rows, world=None, E_l=None, capacity=None):
        return gather_rows(ids, w, hidden, hidden_scale, src_token[:rows].long(), world, E_l, capacity)

    def unpack(self, recv):
        return unpack_rows(recv)

    def combine(self, back, slot, T, output):
        output.copy_(combine_rows(back, slot, T).to(output.dtype))


class LibPlumbing:
    """The same steps as kernels of libmoe_fp8_ds.so (``moe_fp8_ds_ep_*``),
    one launch each, bit-identical to ``TorchPlumbing``."""

    def __init__(self):
        import ctypes
        from . import _lib
        self._c = ctypes
        self._L = _lib
        self._lib = _lib.load()

    def _p(self, t):
        return self._c.c_void_p(t.data_ptr() if t is not None and t.numel() else 0)

    def _s(self, dev):
        return self._c.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def plan(self, ids, world, E_l, capacity=None):
        T, dev = ids.shape[0], ids.device
        ids = ids.to(torch.int32).contiguous()
        counts = torch.empty(world, dtype=torch.int64, device=dev)
        slot = torch.empty(T, world, dtype=torch.int32, device=dev)
        if capacity is None:
            src = torch.empty(max(T * world, 1), dtype=torch.int32, device=dev)
            st = self._lib.moe_fp8_ds_ep_plan(self._p(ids), T, world, E_l, self._p(counts), self._p(slot),
                                              self._p(src), self._s(dev))
        else:
            src = torch.empty(world * capacity, dtype=torch.int32, device=dev)
            st = self._lib.moe_fp8_ds_ep_plan_capacity(self._p(ids), T, world, E_l, capacity, self._p(counts),
                                                       self._p(slot), self._p(src), self._s(dev))
        self._L.check(st, "moe_fp8_ds_ep_plan")
        return counts, slot, src

    def pack(self, ids, w, hidden, hidden_scale, src_token, rows, world=None, E_l=None, capacity=None):
        dev = hidden.device
        send = torch.empty(rows, ROW_BYTES, dtype=torch.uint8, device=dev)
        ids = ids.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        if capacity is None:
            st = self._lib.moe_fp8_ds_ep_pack(self._p(ids), self._p(w), self._p(hidden), self._p(hidden_scale),
                                              hidden.shape[0], self._p(src_token), rows, self._p(send),
                                              self._s(dev))
        else:
            if rows != world * capacity:
                raise ValueError("a fixed-capacity dispatch has world * capacity rows")
            st = self._lib.moe_fp8_ds_ep_pack_capacity(self._p(ids), self._p(w), self._p(hidden),
                                                       self._p(hidden_scale), hidden.shape[0], self._p(src_token),
                                                       world, E_l, capacity, self._p(send), self._s(dev))
        self._L.check(st, "moe_fp8_ds_ep_pack")
        return send

    def unpack(self, recv):
        R, dev = recv.shape[0], recv.device
        hidden = torch.empty(R, H, dtype=torch.float8_e4m3fn, device=dev)
        scale = torch.empty(H // 128, R, dtype=torch.float32, device=dev)
        ids = torch.empty(R, TOP_K, dtype=torch.int32, device=dev)
        w = torch.empty(R, TOP_K, dtype=torch.float32, device=dev)
        self._L.check(self._lib.moe_fp8_ds_ep_unpack(self._p(recv), R, self._p(hidden), self._p(scale),
                                                     self._p(ids), self._p(w), self._s(dev)), "moe_fp8_ds_ep_unpack")
        return hidden, scale, ids, w

    def combine(self, back, slot, T, output):
        if back.dtype != torch.float32 or output.dtype != torch.bfloat16 or not output.is_contiguous():
            raise TypeError("the library combine takes fp32 partials and a contiguous bf16 output")
        slot = slot.to(torch.int32).contiguous()
        self._L.check(self._lib.moe_fp8_ds_ep_combine(self._p(back), self._p(slot), T, slot.shape[1],
                                                      self._p(output), self._s(output.device)),
                      "moe_fp8_ds_ep_combine")


class ExpertParallelMoE:
    """One rank of the expert-parallel layer.

    ``route_fn(logits, bias, scale) -> (ids int32 [T,8] ascending, w fp32 [T,8])`` and
    ``expert_fn(ids, w, hidden, hidden_scale, w13, s13, w2, s2, offset) -> partial [R, H]``
    supply the per-rank compute, ``plumbing`` the plan/pack/unpack/combine
    steps; ``from_library`` wires the CUDA library for all of them.
    """

    def __init__(self, route_fn, expert_fn, group=None, plumbing=None, capacity=None):
        self.route_fn = route_fn
        self.expert_fn = expert_fn
        self.group = group
        self.plumbing = plumbing if plumbing is not None else TorchPlumbing()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E_GLOBAL % self.world:
            raise ValueError(f"{E_GLOBAL} experts do not split over {self.world} ranks")
        self.E_l = E_GLOBAL // self.world
        # Fixed capacity: the same on every rank (at least the most tokens any
        # rank brings to a step); None exchanges exact counts through the host.
        if capacity is not None and (self.world < 2 or capacity < 1):
            raise ValueError("a fixed capacity needs world >= 2 and capacity >= 1")
        self.capacity = capacity
        self.last_stats = {}
        self.profile = False
        self._events = None

    @torch.no_grad()
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                routed_scaling_factor, output):
        if gemm1_weights.shape[0] != self.E_l:
            raise ValueError(f"rank holds {gemm1_weights.shape[0]} experts, expected {self.E_l}")
        T = hidden_states.shape[0]
        pl = self.plumbing
        mark = self._marker(hidden_states.device)
        mark("start")
        ids, w = self.route_fn(routing_logits, routing_bias, routed_scaling_factor)
        mark("route")
        if self.capacity is not None:
            return self._forward_fixed(ids, w, hidden_states, hidden_states_scale, gemm1_weights,
                                       gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, output, mark)
        counts, slot, src_token = pl.plan(ids, self.world, self.E_l)
        mark("plan")
        # count exchange, then the row all-to-all moves only real rows (the
        # split sizes must be on the host: one device-to-host read per step)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        in_splits, out_splits = counts.tolist(), recv_counts.tolist()
        mark("count_a2a")
        send = pl.pack(ids, w, hidden_states, hidden_states_scale, src_token, sum(in_splits))
        mark("pack")
        recv = torch.empty(sum(out_splits), ROW_BYTES, dtype=torch.uint8, device=send.device)
        dist.all_to_all_single(recv, send, out_splits, in_splits, group=self.group)
        mark("row_a2a")
        r_hidden, r_scale, r_ids, r_w = pl.unpack(recv)
        part = self.expert_fn(r_ids, r_w, r_hidden, r_scale, gemm1_weights, gemm1_weights_scale,
                              gemm2_weights, gemm2_weights_scale, self.rank * self.E_l)
        mark("experts")
        back = torch.empty(send.shape[0], H, dtype=part.dtype, device=part.device)
        dist.all_to_all_single(back, part, in_splits, out_splits, group=self.group)
        mark("partial_a2a")
        pl.combine(back, slot, T, output)
        mark("combine")
        self.last_stats = {"sent_rows": int(send.shape[0]), "recv_rows": int(recv.shape[0])}
        return output

    def _forward_fixed(self, ids, w, hidden_states, hidden_states_scale, gemm1_weights, gemm1_weights_scale,
                       gemm2_weights, gemm2_weights_scale, output, mark):
        """One step with fixed per-peer capacity: no count leaves the device."""
        T, cap, world, pl = hidden_states.shape[0], self.capacity, self.world, self.plumbing
        if T > cap:
            raise ValueError(f"{T} tokens exceed the fixed capacity {cap}")
        counts, slot, src_token = pl.plan(ids, world, self.E_l, capacity=cap)
        mark("plan")
        send = pl.pack(ids, w, hidden_states, hidden_states_scale, src_token, world * cap,
                       world=world, E_l=self.E_l, capacity=cap)
        mark("pack")
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        mark("row_a2a")
        r_hidden, r_scale, r_ids, r_w = pl.unpack(recv)
        part = self.expert_fn(r_ids, r_w, r_hidden, r_scale, gemm1_weights, gemm1_weights_scale,
                              gemm2_weights, gemm2_weights_scale, self.rank * self.E_l)
        mark("experts")
        back = torch.empty_like(part)
        dist.all_to_all_single(back, part, group=self.group)
        mark("partial_a2a")
        pl.combine(back, slot, T, output)
        mark("combine")
        # real row counts only on request: reading them would synchronise
        self.last_stats = {"sent_rows": int(counts.sum())} if self.profile else {}
        return output

    def _marker(self, device):
        """Per-phase CUDA events when ``self.profile`` is set (read with ``phase_ms``)."""
        if not self.profile or device.type != "cuda":
            self._events = None
            return lambda name: None
        self._events = []

        def mark(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._events.append((name, ev))
        return mark

    def phase_ms(self):
        """{phase: ms} of the last profiled call (synchronises the device)."""
        if not self._events:
            return {}
        torch.cuda.synchronize()
        ev = self._events
        return {ev[i][0]: ev[i - 1][1].elapsed_time(ev[i][1]) for i in range(1, len(ev))}

    __call__ = forward


def from_library(group=None, capacity=None):
    """ExpertParallelMoE whose routing, plumbing and expert compute run in libmoe_fp8_ds.so
    (``capacity``: fixed per-peer rows, see ``ExpertParallelMoE``)."""
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
        out = torch.empty(R, H, dtype=torch.float32, device=hidden.device)
        args = K.build_args(None, None, hidden, scale, w13, s13, w2, s2, offset, 1.0, None,
                            topk_ids=ids, topk_weights=w, output_f32=out)
        if R:
            ws = K.get_workspace(hidden.device, K.workspace_bytes(R, w13.shape[0]))
            K.run_with_workspace(args, ws, routed=True)
        return out

    return ExpertParallelMoE(route_fn, expert_fn, group, plumbing=LibPlumbing(), capacity=capacity)
