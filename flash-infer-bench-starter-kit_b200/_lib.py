"""ctypes binding of ``libmoe_fp8_ds.so`` (the C ABI declared in include/moe_fp8_ds.h).

This is the layer's only route to the GPU: there is no CPU or PyTorch
fallback.  If the library is missing, loading fails with an error naming
the build step.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libmoe_fp8_ds.so"

# Status codes (enum moe_status).
MOE_OK = 0
MOE_ERR_INVALID_ARGUMENT = 1
MOE_ERR_MISALIGNED = 2
MOE_ERR_WORKSPACE_TOO_SMALL = 3
MOE_ERR_CUDA = 4
MOE_ERR_NO_DEVICE = 5
MOE_ERR_DEVICE_TIMEOUT = 6
MOE_ERR_DEVICE_FAULT = 7
MOE_ERR_TOO_LARGE = 8


class MoeArgs(ctypes.Structure):
    """struct moe_fp8_ds_args."""
    _fields_ = [
        ("routing_logits", ctypes.c_void_p),
        ("routing_bias", ctypes.c_void_p),
        ("hidden_states", ctypes.c_void_p),
        ("hidden_states_scale", ctypes.c_void_p),
        ("gemm1_weights", ctypes.c_void_p),
        ("gemm1_weights_scale", ctypes.c_void_p),
        ("gemm2_weights", ctypes.c_void_p),
        ("gemm2_weights_scale", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("num_tokens", ctypes.c_int32),
        ("num_local_experts", ctypes.c_int32),
        ("local_expert_offset", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
        ("topk_ids", ctypes.c_void_p),
        ("topk_weights", ctypes.c_void_p),
        ("output_f32", ctypes.c_void_p),
    ]


class MoeLayout(ctypes.Structure):
    """struct moe_fp8_ds_layout."""
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "total_bytes", "error_word", "topk_ids", "topk_weights", "inv_row", "seg_offsets",
        "row_token", "block_masks", "block_bases", "inter", "inter_scale", "down", "act", "act_scale")] + [
        ("row_capacity", ctypes.c_int32), ("reserved", ctypes.c_int32)]


EXPORTS = (
    "moe_fp8_ds_workspace_size", "moe_fp8_ds_workspace_layout", "moe_fp8_ds_run",
    "moe_fp8_ds_run_routed", "moe_fp8_ds_route", "moe_fp8_ds_read_device_error",
    "moe_fp8_ds_status_string", "moe_fp8_ds_launches_per_call", "moe_fp8_ds_set_tile_override",
    "moe_fp8_ds_set_stage_events", "moe_fp8_ds_run_noalloc", "moe_fp8_ds_set_path_override",
    "moe_fp8_ds_ep_plan", "moe_fp8_ds_ep_pack", "moe_fp8_ds_ep_unpack", "moe_fp8_ds_ep_combine",
    "moe_fp8_ds_ep_plan_capacity", "moe_fp8_ds_ep_pack_capacity",
    "moe_fp8_ds_selftest_wait_timeout", "moe_fp8_ds_noalloc_read_device_error",
    "moe_fp8_ds_last_cuda_error_string",
)

_lib = None
_lock = threading.Lock()


class MoeError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (status {status})")


def load() -> ctypes.CDLL:
    """Load the shared library once (thread-safe) and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -c \"import __graft_entry__ as g; g.build()\"`")
        lib = ctypes.CDLL(str(LIB_PATH))
        P, I32, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint64
        lib.moe_fp8_ds_workspace_size.argtypes = [I32, I32, ctypes.POINTER(U64)]
        lib.moe_fp8_ds_workspace_layout.argtypes = [I32, I32, ctypes.POINTER(MoeLayout)]
        lib.moe_fp8_ds_run.argtypes = [ctypes.POINTER(MoeArgs), P, U64, P]
        lib.moe_fp8_ds_run_routed.argtypes = [ctypes.POINTER(MoeArgs), P, U64, P]
        lib.moe_fp8_ds_run_noalloc.argtypes = [ctypes.POINTER(MoeArgs), P]
        lib.moe_fp8_ds_set_path_override.argtypes = [I32]
        lib.moe_fp8_ds_route.argtypes = [P, P, I32, ctypes.c_float, P, P, P]
        lib.moe_fp8_ds_read_device_error.argtypes = [P, P, ctypes.POINTER(I32)]
        lib.moe_fp8_ds_status_string.argtypes = [ctypes.c_int]
        lib.moe_fp8_ds_status_string.restype = ctypes.c_char_p
        lib.moe_fp8_ds_last_cuda_error_string.argtypes = []
        lib.moe_fp8_ds_last_cuda_error_string.restype = ctypes.c_char_p
        lib.moe_fp8_ds_launches_per_call.argtypes = [I32]
        lib.moe_fp8_ds_set_tile_override.argtypes = [I32, I32]
        lib.moe_fp8_ds_set_stage_events.argtypes = [ctypes.POINTER(ctypes.c_void_p), I32]
        lib.moe_fp8_ds_ep_plan.argtypes = [P, I32, I32, I32, P, P, P, P]
        lib.moe_fp8_ds_ep_pack.argtypes = [P, P, P, P, I32, P, I32, P, P]
        lib.moe_fp8_ds_ep_unpack.argtypes = [P, I32, P, P, P, P, P]
        lib.moe_fp8_ds_ep_combine.argtypes = [P, P, I32, I32, P, P]
        lib.moe_fp8_ds_ep_plan_capacity.argtypes = [P, I32, I32, I32, I32, P, P, P, P]
        lib.moe_fp8_ds_ep_pack_capacity.argtypes = [P, P, P, P, I32, P, I32, I32, I32, P, P]
        lib.moe_fp8_ds_selftest_wait_timeout.argtypes = [P, P]
        for name in EXPORTS:
            if name not in ("moe_fp8_ds_status_string", "moe_fp8_ds_last_cuda_error_string"):
                getattr(lib, name).restype = ctypes.c_int
        _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().moe_fp8_ds_status_string(int(status)).decode()
    except ImportError:
        return f"status {status}"


def check(status: int, where: str) -> None:
    if status != MOE_OK:
        if status == MOE_ERR_CUDA:
            where = f"{where} ({load().moe_fp8_ds_last_cuda_error_string().decode()})"
        raise MoeError(status, where)
