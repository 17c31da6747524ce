"""Solution entry point: ``kernel(...)`` for
``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``.

Drop-in for the reference's ``solution/python/kernel.py:95-120``: the same 11
positional arguments, destination-passing style (``output`` is allocated by
the caller and fully overwritten), work enqueued on the current torch CUDA
stream with no host synchronisation.  Instead of JIT-compiling a torch
extension on the first call (``kernel.py:57-92`` of the reference), it calls
the prebuilt sm_100a library ``libmoe_fp8_ds.so`` through its C ABI.  There
is no CPU or PyTorch fallback: without the library or a B200 the call raises.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

H, I, E_GLOBAL, TOP_K = 7168, 2048, 256, 8

# One workspace per (device, stream): calls on one stream run in order, so they
# can share a workspace; calls on different streams could overlap and get
# their own.  Each is allocated on its stream, so dropping a smaller one when
# it grows is ordered after that stream's earlier launches by torch's caching
# allocator (the reference allocates its buffers per call the same way,
# ``main.cpp:87-252``).  A workspace lives until ``release_workspaces`` drops
# it.  Next to it the entry keeps an event recorded after the last call that
# used it, so the device error word can be read without touching the stream
# itself (which the caller may have destroyed since).
_ws_lock = threading.Lock()


class _Workspace:
    __slots__ = ("buf", "event")

    def __init__(self, buf: torch.Tensor):
        self.buf = buf
        self.event = torch.cuda.Event()


_workspaces: dict[tuple[int, int], _Workspace] = {}   # (device index, stream handle) -> workspace


def workspace_bytes(num_tokens: int, num_local_experts: int) -> int:
    lib = _lib.load()
    n = ctypes.c_uint64(0)
    _lib.check(lib.moe_fp8_ds_workspace_size(int(num_tokens), int(num_local_experts), ctypes.byref(n)),
               "moe_fp8_ds_workspace_size")
    return int(n.value)


def workspace_layout(num_tokens: int, num_local_experts: int) -> _lib.MoeLayout:
    lib = _lib.load()
    lay = _lib.MoeLayout()
    _lib.check(lib.moe_fp8_ds_workspace_layout(int(num_tokens), int(num_local_experts), ctypes.byref(lay)),
               "moe_fp8_ds_workspace_layout")
    return lay


def _device_index(device: torch.device | None) -> int:
    if device is None or device.index is None:
        return torch.cuda.current_device()
    return device.index


def _entry(device: torch.device, nbytes: int, stream: torch.cuda.Stream | None = None) -> _Workspace:
    idx = _device_index(device)
    if stream is None:
        stream = torch.cuda.current_stream(idx)
    key = (idx, stream.cuda_stream)
    with _ws_lock:
        ent = _workspaces.get(key)
        if ent is None or ent.buf.numel() < nbytes:
            _workspaces.pop(key, None)
            with torch.cuda.device(idx), torch.cuda.stream(stream):
                ent = _Workspace(torch.zeros(max(nbytes, 256), dtype=torch.uint8,
                                             device=torch.device("cuda", idx)))
            _workspaces[key] = ent
        return ent


def get_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """The workspace of ``device``'s current stream, zero-filled on (re)allocation and at
    least ``nbytes`` long.  Launch the work that uses it on that same stream."""
    return _entry(device, nbytes).buf


def workspace_for(device: torch.device | None = None) -> torch.Tensor | None:
    """The workspace last used on ``device``'s current stream, or None."""
    idx = _device_index(device)
    ent = _workspaces.get((idx, torch.cuda.current_stream(idx).cuda_stream))
    return ent.buf if ent is not None else None


def release_workspaces(device: torch.device | None = None, stream: torch.cuda.Stream | None = None) -> int:
    """Drop cached workspaces and return how many were dropped: all of them, those of
    ``device``, or the one of ``stream``.  The memory goes back to torch's caching
    allocator, ordered after the work already enqueued on each workspace's stream; the
    next call on a released stream allocates (and zero-fills) a new workspace."""
    with _ws_lock:
        keys = [k for k in _workspaces
                if (device is None or k[0] == _device_index(device))
                and (stream is None or k[1] == stream.cuda_stream)]
        for k in keys:
            del _workspaces[k]
    return len(keys)


def _check_tensor(name, t, dtype, shape, device):
    # (cheap comparisons first: this runs for every argument of every call)
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.get_device() != device.index:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if t.dtype is not dtype:
        raise TypeError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if t.shape != shape:
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def build_args(routing_logits, routing_bias, hidden_states, hidden_states_scale,
               gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
               local_expert_offset, routed_scaling_factor, output, *,
               topk_ids=None, topk_weights=None, output_f32=None) -> _lib.MoeArgs:
    """Validate the call's tensors and fill ``struct moe_fp8_ds_args``."""
    dev = hidden_states.device
    if dev.type != "cuda":
        raise ValueError("kernel(...) needs CUDA tensors (no CPU path)")
    T = hidden_states.shape[0]
    E_l = gemm1_weights.shape[0]
    routed = topk_ids is not None
    if not routed:
        _check_tensor("routing_logits", routing_logits, torch.float32, (T, E_GLOBAL), dev)
        _check_tensor("routing_bias", routing_bias, torch.bfloat16, (E_GLOBAL,), dev)
    else:
        _check_tensor("topk_ids", topk_ids, torch.int32, (T, TOP_K), dev)
        _check_tensor("topk_weights", topk_weights, torch.float32, (T, TOP_K), dev)
    _check_tensor("hidden_states", hidden_states, torch.float8_e4m3fn, (T, H), dev)
    _check_tensor("hidden_states_scale", hidden_states_scale, torch.float32, (H // 128, T), dev)
    _check_tensor("gemm1_weights", gemm1_weights, torch.float8_e4m3fn, (E_l, 2 * I, H), dev)
    _check_tensor("gemm1_weights_scale", gemm1_weights_scale, torch.float32, (E_l, 2 * I // 128, H // 128), dev)
    _check_tensor("gemm2_weights", gemm2_weights, torch.float8_e4m3fn, (E_l, H, I), dev)
    _check_tensor("gemm2_weights_scale", gemm2_weights_scale, torch.float32, (E_l, H // 128, I // 128), dev)
    if output_f32 is not None:
        _check_tensor("output_f32", output_f32, torch.float32, (T, H), dev)
    else:
        _check_tensor("output", output, torch.bfloat16, (T, H), dev)
    a = _lib.MoeArgs()
    a.routing_logits = _ptr(routing_logits) if not routed else ctypes.c_void_p(0)
    a.routing_bias = _ptr(routing_bias) if not routed else ctypes.c_void_p(0)
    a.hidden_states = _ptr(hidden_states)
    a.hidden_states_scale = _ptr(hidden_states_scale)
    a.gemm1_weights = _ptr(gemm1_weights)
    a.gemm1_weights_scale = _ptr(gemm1_weights_scale)
    a.gemm2_weights = _ptr(gemm2_weights)
    a.gemm2_weights_scale = _ptr(gemm2_weights_scale)
    a.output = _ptr(output) if output_f32 is None else ctypes.c_void_p(0)
    a.num_tokens = int(T)
    a.num_local_experts = int(E_l)
    a.local_expert_offset = int(local_expert_offset)
    a.routed_scaling_factor = float(routed_scaling_factor)
    a.topk_ids = _ptr(topk_ids)
    a.topk_weights = _ptr(topk_weights)
    a.output_f32 = _ptr(output_f32)
    return a


def run_with_workspace(args: _lib.MoeArgs, ws: torch.Tensor, stream: int | None = None,
                       routed: bool = False) -> None:
    lib = _lib.load()
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    fn = lib.moe_fp8_ds_run_routed if routed else lib.moe_fp8_ds_run
    _lib.check(fn(ctypes.byref(args), ctypes.c_void_p(ws.data_ptr()), ctypes.c_uint64(ws.numel()),
                  ctypes.c_void_p(stream)), fn.__name__)


def kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale,
           gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
           local_expert_offset, routed_scaling_factor, output):
    """Fused FP8 block-scale MoE forward with DeepSeek-V3 routing (DPS: writes ``output``).

    The call may be captured in a CUDA graph (``torch.cuda.graph``): make one
    eager call on the capturing stream first, so its workspace exists before
    the capture; replays then rerun the same launches on the same buffers."""
    args = build_args(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                      local_expert_offset, routed_scaling_factor, output)
    dev = hidden_states.device
    if torch.cuda.current_device() != dev.index:
        with torch.cuda.device(dev):
            return kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                          gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                          local_expert_offset, routed_scaling_factor, output)
    stream = torch.cuda.current_stream(dev.index)
    ent = _entry(dev, workspace_bytes(args.num_tokens, args.num_local_experts), stream)
    run_with_workspace(args, ent.buf, stream.cuda_stream)
    # Under CUDA-graph capture the launches become graph nodes and the
    # last-use event is not recorded (an event recorded in a capture cannot
    # be waited on outside it); synchronise the replay stream before
    # read_device_error after replays.
    if not torch.cuda.is_current_stream_capturing():
        ent.event.record(stream)


def read_device_error(device: torch.device | None = None) -> int:
    """Wait for the last ``kernel(...)`` call on each of ``device``'s workspaces and return
    (and clear) their device error codes: the first non-zero one, or 0 when no device-side
    error happened since the last read.  The reads run on the current stream after it has
    waited on each workspace's last-use event, so streams the caller has destroyed since
    are never touched."""
    lib = _lib.load()
    idx = _device_index(device)
    with _ws_lock:
        mine = [ent for key, ent in _workspaces.items() if key[0] == idx]
    first = 0
    with torch.cuda.device(idx):
        cur = torch.cuda.current_stream(idx)
        for ent in mine:
            cur.wait_event(ent.event)
            code = ctypes.c_int32(0)
            st = lib.moe_fp8_ds_read_device_error(ctypes.c_void_p(ent.buf.data_ptr()),
                                                  ctypes.c_void_p(cur.cuda_stream), ctypes.byref(code))
            if st not in (_lib.MOE_OK, _lib.MOE_ERR_DEVICE_TIMEOUT, _lib.MOE_ERR_DEVICE_FAULT):
                _lib.check(st, "moe_fp8_ds_read_device_error")
            if first == 0:
                first = int(code.value)
    return first
