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


def _fp8_multi(case, ks, vs, key8, value8):
    width = case.tables.shape[1]
    return O.multi_from_raw_fp8(
        case.qk, case.v, case.sqk, case.sqk_factor, O.EPS,
        torch.zeros(case.tokens, dtype=torch.int64), key8.view(-1), value8.view(-1),
        tuple(key8.shape), key8.stride(), case.tables.reshape(-1),
        torch.tensor([r * width for r in case.table_rows]), case.seq_lens, case.window,
        case.scale, case.gate, case.num_heads, case.num_kv_heads, ks, vs,
        shared_cache=case.shared)


def test_shared_multi_token_equals_single_calls_in_position_order():
    """A shared-cache wavefront over an e4m3 cache equals the single-token calls in position
    order (each appending its row before the next attends), outputs and bytes."""
    case = W.wavefront(seed=1250, prompt=90, tokens=3, num_heads=8, num_kv_heads=2,
                       head_dim=128, pool_blocks=12)
    ks, vs = 0.5, 0.25
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    k_seq, v_seq = key8.clone(), value8.clone()
    want = torch.stack([
        O.from_raw_fp8(case.qk[t], case.v[t], case.sqk, case.sqk_factor, O.EPS, case.slot(t),
                       k_seq, v_seq, case.tables[0], case.seq_lens[t], case.window, case.scale,
                       case.gate[t], 8, 2, ks, vs) for t in range(case.tokens)])
    got = _fp8_multi(case, ks, vs, key8, value8)
    assert torch.equal(got, want)
    assert torch.equal(key8, k_seq) and torch.equal(value8, v_seq)


def test_unshared_single_token_matches_from_raw():
    case = W.single(seed=1251, context=70, pool_blocks=8, num_heads=8, num_kv_heads=2,
                    head_dim=128)
    ks, vs = 1.0, 2.0
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    k1, v1 = key8.clone(), value8.clone()
    want = O.from_raw_fp8(case.qk[0], case.v[0], case.sqk, case.sqk_factor, O.EPS,
                          case.slot(0), k1, v1, case.tables[0], case.seq_lens[0], case.window,
                          case.scale, case.gate[0], 8, 2, ks, vs)
    got = _fp8_multi(case, ks, vs, key8, value8)
    assert torch.equal(got[0], want)
    assert torch.equal(key8, k1) and torch.equal(value8, v1)
