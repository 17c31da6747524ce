"""Generate the golden fixtures of the CPU oracle from the reference definition.

The reference project has no tests or golden vectors of its own.  The layer
definition it implements is pinned by flashinfer-python 0.6.11.post2's
``flashinfer.trace.templates.moe._trtllm_fp8_block_scale_moe_ds_routing_reference``
(the contest's ground truth for ``moe_fp8_block_scale_ds_routing``), which is
importable in the build container.  This script runs it on seeded inputs from
``inputs.make_inputs`` and stores:

* ``full_*.pt``  : input digest, routing (ids ascending + weights) and the bf16 output;
* ``route_*.pt`` : routing only, for larger T and the skewed-logit stress case.

The routing is captured by wrapping the reference's expert runner, which the
routing function calls with ``(weights[T,8], topk_idx[T,8])``.

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import pathlib
import sys

import torch

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import __graft_entry__ as ge  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent

FULL_CASES = [
    # name, T, E_l, local_expert_offset, seed
    ("full_T8_E32_off0_s0", 8, 32, 0, 0),
    ("full_T16_E8_off64_s1", 16, 8, 64, 1),
    ("full_T1_E32_off224_s2", 1, 32, 224, 2),
]
ROUTE_CASES = [
    # name, T, seed, skew
    ("route_T4096_s3", 4096, 3, 0.0),
    ("route_T2048_skew_s4", 2048, 4, 3.0),
]


def _capture_reference():
    import flashinfer.trace.templates.moe as fm
    captured = {}
    orig = fm._fp8_moe_run_experts

    def wrapped(hs, hss, w1, s1, w2, s2, weights, topk_idx, local_expert_offset, E_global):
        captured["w"] = weights.clone()
        captured["idx"] = topk_idx.clone()
        if captured.get("skip_experts"):
            return torch.zeros(hs.shape[0], 7168, dtype=torch.bfloat16)
        return orig(hs, hss, w1, s1, w2, s2, weights, topk_idx, local_expert_offset, E_global)

    fm._fp8_moe_run_experts = wrapped
    return fm._trtllm_fp8_block_scale_moe_ds_routing_reference, captured


def _sorted_routing(idx, w):
    order = idx.argsort(dim=1)
    return idx.gather(1, order).to(torch.int32), w.gather(1, order).to(torch.float32)


def main():
    torch.set_num_threads(8)
    pkg = ge.load_package()
    ref, cap = _capture_reference()
    for name, T, E_l, off, seed in FULL_CASES:
        inp = pkg.inputs.make_inputs(T, E_l=E_l, local_expert_offset=off, seed=seed)
        a = pkg.inputs.as_args(inp)
        cap.clear()
        out = ref(*a[:8], 8, 8, 4, a[8], a[9])
        ids, w = _sorted_routing(cap["idx"], cap["w"])
        torch.save(dict(T=T, E_l=E_l, offset=off, seed=seed, digest=pkg.inputs.input_digest(inp),
                        topk_ids=ids, topk_w=w, output=out.to(torch.bfloat16)), OUT / f"{name}.pt")
        print(name, "done")
    for name, T, seed, skew in ROUTE_CASES:
        logits, bias = pkg.inputs.make_routing_inputs(T, seed=seed, skew=skew)
        cap.clear()
        cap["skip_experts"] = True
        dummy8 = torch.zeros(T, 7168, dtype=torch.float8_e4m3fn)
        ref(logits, bias, dummy8, torch.ones(56, T), None, None, None, None, 8, 8, 4, 0, 2.5)
        ids, w = _sorted_routing(cap["idx"], cap["w"])
        torch.save(dict(T=T, seed=seed, skew=skew, topk_ids=ids, topk_w=w), OUT / f"{name}.pt")
        print(name, "done")


if __name__ == "__main__":
    main()
