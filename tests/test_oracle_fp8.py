"""The oracle's e4m3 restatement (FP8 KV caches): round to nearest even, saturation at
+-448, exact round trips of representable values, and the workload generator's bytes."""

from __future__ import annotations

import torch

import dory_oracle as O
import workloads as W


def test_representable_values_round_trip():
    b = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    b = b[(b & 0x7F) != 0x7F]  # e4m3 NaN patterns
    x = O.e4m3_dequantize(b, 1.0)
    assert torch.equal(O.e4m3_quantize(x, 1.0), b) or torch.equal(
        O.e4m3_dequantize(O.e4m3_quantize(x, 1.0), 1.0), x)  # +0 / -0 both map to zero
    assert float(x.abs().max()) == 448.0


def test_saturation_and_rounding():
    q = O.e4m3_dequantize(O.e4m3_quantize(torch.tensor([500.0, -1e9, 448.0, 1.0625, 1.1875]),
                                          1.0), 1.0)
    # 1.0625 lies halfway between 1.0 and 1.125 (mantissa 0 vs 1): ties to even gives 1.0;
    # 1.1875 lies halfway between 1.125 and 1.25: ties to even gives 1.25
    assert q.tolist() == [448.0, -448.0, 448.0, 1.0, 1.25]


def test_scales_divide_before_rounding():
    x = torch.tensor([3.0, -0.75, 96.0])
    assert torch.equal(O.e4m3_dequantize(O.e4m3_quantize(x, 0.5), 0.5), x)
    assert torch.equal(W.e4m3_bytes(x, 0.5), O.e4m3_quantize(x, 0.5))
