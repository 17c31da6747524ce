"""GPU: the allocation-free entry point moe_fp8_ds_run_noalloc.

It exists for callers that may not allocate device memory where they call
the layer (an external allocator owns all device memory, or cudaMalloc is
banned on the serving path).  Its workspace is an array built into the
library, so this test checks, through the C ABI, that two calls in a row give
the same result as the workspace-taking moe_fp8_ds_run -- bit for bit, since
both run the same deterministic kernels on the same plan -- with no device
error recorded, and that batches beyond the built-in limit are refused.  The file
is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes
import sys

import pytest
import torch

from conftest import cached_inputs

pytestmark = pytest.mark.gpu


def _run(pkg, inp, noalloc):
    K, L = sys.modules["fib_b200.kernel"], sys.modules["fib_b200._lib"]
    lib = L.load()
    T = inp["hidden_states"].shape[0]
    out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=inp["hidden_states"].device)
    args = K.build_args(*pkg.inputs.as_args(inp), out)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        L.check(lib.moe_fp8_ds_run_noalloc(ctypes.byref(args), stream), "moe_fp8_ds_run_noalloc")
    else:
        ws = torch.zeros(K.workspace_bytes(T, inp["gemm1_weights"].shape[0]), dtype=torch.uint8,
                         device=out.device)
        K.run_with_workspace(args, ws)
    torch.cuda.synchronize()
    return out


def test_noalloc_matches_workspace_entry_twice(pkg, cuda_dev):
    inp = {k: (v.to(cuda_dev) if isinstance(v, torch.Tensor) else v)
           for k, v in cached_inputs(16, 8, 0, 12).items()}
    L = sys.modules["fib_b200._lib"]
    ref = _run(pkg, inp, noalloc=False)
    for _ in range(2):
        got = _run(pkg, inp, noalloc=True)
        assert not torch.isnan(got.float()).any()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), "differs from moe_fp8_ds_run"
        code = ctypes.c_int32(-1)
        st = L.load().moe_fp8_ds_noalloc_read_device_error(
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(code))
        assert st == L.MOE_OK and code.value == 0


def test_noalloc_rejects_large_batch(pkg, cuda_dev):
    L = sys.modules["fib_b200._lib"]
    a = L.MoeArgs()
    a.num_tokens = 17
    a.num_local_experts = 8
    assert L.load().moe_fp8_ds_run_noalloc(ctypes.byref(a), None) == L.MOE_ERR_TOO_LARGE
