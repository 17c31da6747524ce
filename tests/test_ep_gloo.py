"""CPU, multi-process: the expert-parallel dispatch/combine protocol over gloo.

Each rank routes its own tokens with the CPU oracle, exchanges rows with the
real ExpertParallelMoE code, and computes its experts' part with a cheap
deterministic stand-in (no weights needed), so the test checks the protocol:
every (token, rank) pair is sent once, rows come back to the right token, the
combine sums ranks in a fixed order, and the result equals the single-process
computation.  The CUDA expert compute is covered by the GPU tests.
"""

from __future__ import annotations

import os
import datetime
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H = 7168


def standin_experts(ids, w, hidden, scale, w13, s13, w2, s2, offset, E_l):
    """partial[t] = sum over local picks (ascending expert) of w * (dequant(x_t) * (e + 1) / 256)."""
    from oracle import moe_ref
    x = moe_ref.dequant_hidden(hidden, scale)
    out = torch.zeros(hidden.shape[0], H)
    for k in range(8):
        e = ids[:, k].long()
        loc = (e >= offset) & (e < offset + E_l)
        f = torch.where(loc, w[:, k] * (e.float() + 1) / 256, torch.zeros(()))
        out = out + x * f.unsqueeze(1)
    return out


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, q, capacity=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import __graft_entry__ as ge
        pkg = ge.load_package()
        from oracle import moe_ref
        ep_mod = __import__("fib_b200.ep", fromlist=["ep"])
        E_l = 256 // world

        def route_fn(logits, bias, scale):
            ids, w, _ = moe_ref.route(logits, bias, scale)
            return ids.to(torch.int32), w

        def expert_fn(ids, w, hidden, scale, w13, s13, w2, s2, offset):
            return standin_experts(ids, w, hidden, scale, w13, s13, w2, s2, offset, E_l)

        layer = ep_mod.ExpertParallelMoE(route_fn, expert_fn, capacity=capacity)
        layer.profile = True    # row statistics (CPU: no events)
        logits, bias, hs, hss = pkg.inputs.make_token_inputs(T, seed=100 + rank)
        dummy = torch.empty(E_l, 1)
        out = torch.empty(T, H, dtype=torch.bfloat16)
        layer(logits, bias, hs, hss, dummy, dummy, dummy, dummy, 2.5, out)
        out2 = torch.empty_like(out)
        layer(logits, bias, hs, hss, dummy, dummy, dummy, dummy, 2.5, out2)
        # single-process reference: all 256 experts local
        ids, w = route_fn(logits, bias, 2.5)
        ref = standin_experts(ids, w, hs, hss, None, None, None, None, 0, 256)
        q.put((rank, torch.equal(out.view(torch.int16), out2.view(torch.int16)),
               float((out.float() - ref).abs().max()), float(ref.abs().max()), layer.last_stats))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,capacity", [(2, None), (4, None), (8, None), (2, 32), (8, 24)])
def test_ep_protocol_matches_single_process(world, capacity):
    """Exact counts through the host (capacity None), or fixed per-peer capacity
    with padding rows (capacity >= the 24 tokens each rank brings)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 24, q, capacity)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    errs = [r for r in res if r[1] == "error"]
    assert not errs, errs[0][2]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, det, err, mx, stats in res:
        assert det, f"rank {rank}: two calls differ"
        assert err <= 1e-2 * max(mx, 1e-6) + 1e-5, f"rank {rank}: error {err} vs max {mx}"
        assert stats["sent_rows"] > 0


def _worker_dead_peer(rank, world, port, q):
    """Rank 1 fails before the exchange (an exception on the host) and leaves;
    rank 0 must get an error from its next collective, not hang."""
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    import __graft_entry__ as ge
    pkg = ge.load_package()
    from oracle import moe_ref
    ep_mod = __import__("fib_b200.ep", fromlist=["ep"])
    E_l = 256 // world

    def route_fn(logits, bias, scale):
        ids, w, _ = moe_ref.route(logits, bias, scale)
        return ids.to(torch.int32), w

    def expert_fn(ids, w, hidden, scale, w13, s13, w2, s2, offset):
        return standin_experts(ids, w, hidden, scale, w13, s13, w2, s2, offset, E_l)

    layer = ep_mod.ExpertParallelMoE(route_fn, expert_fn)
    logits, bias, hs, hss = pkg.inputs.make_token_inputs(8, seed=300 + rank)
    dummy = torch.empty(E_l, 1)
    out = torch.empty(8, H, dtype=torch.bfloat16)
    def report(msg):
        q.put(msg)
        q.close()
        q.join_thread()      # flush before the hard exit

    if rank == 1:
        report((rank, "left", 0.0))
        os._exit(0)          # the rank dies between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        layer(logits, bias, hs, hss, dummy, dummy, dummy, dummy, 2.5, out)
        report((rank, "no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001  (any collective error is the expected outcome)
        report((rank, "error:" + type(e).__name__, time.monotonic() - t0))
    os._exit(0)


def test_ep_dead_peer_raises_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=180) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert res[1][0] == "left"
    assert res[0][0].startswith("error:"), res[0]
    assert res[0][1] < 60.0, f"the surviving rank waited {res[0][1]:.1f} s"
