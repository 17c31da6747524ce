"""The grouped GEMMs' persistent work schedule, checked on the CPU.

``WorkSched`` (``csrc/kernels.cuh``) decides which CTA runs which (token tile, weight tile)
unit and which K iterations of it: full waves, then a stream-K tail whose split units are
finished by their last contributor from fixed partial slots.  ``tests/native/sched_check.cu``
includes the header unchanged, sweeps 6,144 shapes (token tiles 1..160, 1/7/16/56 weight
tiles, 1..112 iterations per unit, 1..296 workers) and checks exact coverage, contributor
ranges, slot reuse and the unit→tile map.  Replaces nothing in the reference, whose grouped
GEMM schedule lives inside CUTLASS (``moe_grouped_gemm_fp8.cu:821-948``).
"""

from __future__ import annotations

import shutil
import subprocess

import pytest

from conftest import ROOT

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def test_work_schedule_covers_every_iteration_once(tmp_path):
    if shutil.which(NVCC) is None:
        pytest.skip("nvcc not available")
    exe = tmp_path / "sched_check"
    subprocess.run([NVCC, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", str(ROOT / "flash-infer-bench-starter-kit_b200" / "csrc"),
                    "-o", str(exe), str(ROOT / "tests" / "native" / "sched_check.cu")],
                   check=True, capture_output=True, timeout=300)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.startswith("OK"), out.stdout
