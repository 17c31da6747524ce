"""CPU: the C-ABI library builds, loads and exports every symbol the header
declares; host-side argument checks answer without touching a GPU."""

from __future__ import annotations

import ctypes
import re
import sys

import pytest
import torch

from conftest import ROOT


def header_symbols():
    src = (ROOT / "include" / "moe_fp8_ds.h").read_text()
    return sorted(set(re.findall(r"MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = header_symbols()
    for name in ("moe_fp8_ds_run", "moe_fp8_ds_run_routed", "moe_fp8_ds_workspace_size",
                 "moe_fp8_ds_workspace_layout", "moe_fp8_ds_read_device_error", "moe_fp8_ds_route"):
        assert name in syms


def test_library_is_built_and_fresh(pkg):
    b = sys.modules["fib_b200_build"] if "fib_b200_build" in sys.modules else graft_build()
    assert b.LIB_PATH.exists()
    assert not b.is_stale(), "libmoe_fp8_ds.so is older than its sources; run __graft_entry__.build()"


def graft_build():
    import __graft_entry__ as g
    return g._load_build_module()


def test_library_exports_every_header_symbol(pkg):
    lib = ctypes.CDLL(str(sys.modules["fib_b200._lib"].LIB_PATH))
    for name in header_symbols():
        assert hasattr(lib, name), f"{name} declared in include/moe_fp8_ds.h but not exported"


def test_status_strings(pkg):
    L = sys.modules["fib_b200._lib"]
    lib = L.load()
    assert lib.moe_fp8_ds_status_string(0) == b"ok"
    for st in range(1, 9):
        assert lib.moe_fp8_ds_status_string(st) != b"unknown status"
    assert lib.moe_fp8_ds_launches_per_call(64) == 4
    assert lib.moe_fp8_ds_launches_per_call(4096) == 6


def test_argument_validation_without_gpu(pkg):
    L = sys.modules["fib_b200._lib"]
    lib = L.load()
    assert lib.moe_fp8_ds_run(None, None, 0, None) == L.MOE_ERR_INVALID_ARGUMENT
    a = L.MoeArgs()
    a.num_tokens = 0
    a.num_local_experts = 32
    assert lib.moe_fp8_ds_run(ctypes.byref(a), None, 0, None) == L.MOE_OK       # T = 0: nothing to do
    a.num_local_experts = 0
    assert lib.moe_fp8_ds_run(ctypes.byref(a), None, 0, None) == L.MOE_ERR_INVALID_ARGUMENT
    a.num_local_experts = 32
    a.num_tokens = 4
    assert lib.moe_fp8_ds_run(ctypes.byref(a), None, 0, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_set_tile_override(24, 0) == L.MOE_ERR_INVALID_ARGUMENT
    # expert-parallel plumbing: shapes are checked before any launch
    cnt = ctypes.c_void_p(16)
    assert lib.moe_fp8_ds_ep_plan(None, 0, 3, 85, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_plan(None, 0, 2, 64, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_plan(None, 0, 16, 16, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_plan(None, 4, 2, 128, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_pack(None, None, None, None, 4, None, 0, None, None) == L.MOE_OK
    assert lib.moe_fp8_ds_ep_pack(None, None, None, None, 4, None, 2, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    # fixed capacity: world >= 2, capacity >= tokens, src_token and counts required
    assert lib.moe_fp8_ds_ep_plan_capacity(None, 0, 1, 256, 4, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_plan_capacity(None, 8, 2, 128, 4, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_plan_capacity(None, 0, 2, 128, 4, cnt, None, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_pack_capacity(None, None, None, None, 8, None, 2, 128, 4, None, None) == \
        L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_ep_unpack(None, 0, None, None, None, None, None) == L.MOE_OK
    assert lib.moe_fp8_ds_ep_combine(None, None, 0, 2, None, None) == L.MOE_OK
    assert lib.moe_fp8_ds_ep_combine(None, None, 4, 9, None, None) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_set_tile_override(0, 0) == L.MOE_OK
    assert lib.moe_fp8_ds_set_path_override(3) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_set_path_override(-1) == L.MOE_ERR_INVALID_ARGUMENT
    assert lib.moe_fp8_ds_set_path_override(2) == L.MOE_OK
    assert lib.moe_fp8_ds_set_path_override(0) == L.MOE_OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU answer")
def test_workspace_query_reports_missing_device(pkg):
    L = sys.modules["fib_b200._lib"]
    n = ctypes.c_uint64(0)
    assert L.load().moe_fp8_ds_workspace_size(8, 32, ctypes.byref(n)) == L.MOE_ERR_NO_DEVICE


def test_python_entry_rejects_cpu_tensors(pkg):
    with pytest.raises(ValueError):
        pkg.kernel(*[torch.zeros(1)] * 2, torch.zeros(1, 7168).to(torch.float8_e4m3fn),
                   *[torch.zeros(1)] * 5, 0, 2.5, torch.zeros(1, 7168, dtype=torch.bfloat16))


def test_release_workspaces_drops_entries(pkg):
    """Workspaces live per (device, stream) until released; release by stream, by
    device and all at once (bookkeeping only, no GPU memory is touched)."""
    K = sys.modules["fib_b200.kernel"]
    saved = dict(K._workspaces)
    try:
        K._workspaces.clear()
        for key in ((0, 11), (0, 12), (1, 13)):
            K._workspaces[key] = K._Workspace(torch.zeros(256, dtype=torch.uint8))

        class FakeStream:
            cuda_stream = 12
        assert K.release_workspaces(torch.device("cuda", 0), FakeStream()) == 1
        assert set(K._workspaces) == {(0, 11), (1, 13)}
        assert K.release_workspaces(torch.device("cuda", 1)) == 1
        assert set(K._workspaces) == {(0, 11)}
        assert K.release_workspaces() == 1
        assert not K._workspaces
    finally:
        K._workspaces.clear()
        K._workspaces.update(saved)
