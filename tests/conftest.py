"""Shared fixtures: the package under test, the CPU oracle and cached inputs."""

from __future__ import annotations

import functools
import pathlib
import sys

import pytest
import torch

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__ as graft  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


@pytest.fixture(scope="session")
def pkg():
    return graft.load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import moe_ref
    return moe_ref


@pytest.fixture(scope="session")
def cuda_dev():
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"needs an sm_100 device, found sm_{major}x")
    return torch.device("cuda", 0)


@functools.lru_cache(maxsize=8)
def cached_inputs(T, E_l, offset, seed, skew=0.0):
    """CPU inputs from the package generator (cached per session)."""
    pkg = graft.load_package()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    return pkg.inputs.make_inputs(T, E_l=E_l, local_expert_offset=offset, seed=seed, skew=skew)


def load_golden(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=True)


def tied_routing_inputs(T: int, seed: int, bias_grid: bool = False):
    """Routing inputs full of exact score ties: logits on a 0.5 grid in [-1, 1]
    and a zero bias (or a bias on a 0.25 grid), so many experts and groups of a
    token share one sigmoid-plus-bias value."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randint(-2, 3, (T, 256), generator=g).float() * 0.5
    if bias_grid:
        bias = (torch.randint(-1, 2, (256,), generator=g).float() * 0.25).to(torch.bfloat16)
    else:
        bias = torch.zeros(256, dtype=torch.bfloat16)
    return logits, bias
