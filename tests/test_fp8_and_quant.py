"""CPU: e4m3 decoding known answers and the two-term intermediate quantisation."""

from __future__ import annotations

import math

import torch


def test_e4m3_known_answers(oracle):
    t = oracle.E4M3_TABLE
    assert t[0x00] == 0.0 and t[0x80] == 0.0
    assert t[0x7E] == 448.0 and t[0xFE] == -448.0            # largest finite
    assert t[0x08] == 2.0 ** -6                               # smallest normal
    assert t[0x01] == 2.0 ** -9                               # smallest subnormal
    assert t[0x38] == 1.0
    assert math.isnan(t[0x7F]) and math.isnan(t[0xFF])


def test_e4m3_table_matches_torch(oracle):
    codes = torch.arange(256, dtype=torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float()
    both_nan = torch.isnan(ref) & torch.isnan(oracle.E4M3_TABLE)
    assert torch.equal(ref[~both_nan], oracle.E4M3_TABLE[~both_nan])


def test_quant_hilo_error_bound(oracle):
    g = torch.Generator().manual_seed(0)
    c = torch.randn(64, 2048, generator=g) * torch.rand(64, 1, generator=g) * 3
    c[3, :128] = 0.0                                          # all-zero block -> scale 1
    hi, lo, s = oracle.quant_hilo(c)
    deq = (oracle.fp8_to_f32(hi).view(64, 16, 128) * s.unsqueeze(-1)
           + oracle.fp8_to_f32(lo).view(64, 16, 128) * (s / 16).unsqueeze(-1)).view(64, 2048)
    amax = c.view(64, 16, 128).abs().amax(2).repeat_interleave(128, 1)
    assert float(((deq - c).abs() / amax.clamp_min(1e-30)).max()) < 2e-3
    assert float(s[3, 0]) == 1.0 and torch.all(deq[3, :128] == 0)
    # single-term error is an order of magnitude larger
    single = (oracle.fp8_to_f32(hi).view(64, 16, 128) * s.unsqueeze(-1)).view(64, 2048)
    assert float((single - c).abs().max()) > 10 * float((deq - c).abs().max())
