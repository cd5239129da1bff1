"""The CPU oracle against the golden vectors the reference's own eager code produced.

Pins oracle/dory_oracle.py before any kernel is compared with it:
* inputs regenerated from the seeds hash to the digests stored by make_golden.py;
* with the reference's single q rounding the oracle reproduces `reference_attention` to
  FP32 accuracy; with the kernel's second rounding it stays inside the bf16 tolerance;
* the appended k / v rows match the reference's `normalize_rows` bit patterns on every
  element of every golden case, and the bf16 query on all but one element, where the
  reference's FP32 `torch.rsqrt` (1 / sqrt, rounded twice) is one FP32 ulp above the
  correctly rounded inverse square root and the oracle's value is the correctly rounded one.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import dory_oracle as O
import specs

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = specs.specs()


def load(name):
    return np.load(GOLDEN / f"{name}.npz")


def run_oracle(case, second_rounding):
    key = case.key.to(torch.bfloat16).clone()
    value = case.value.to(torch.bfloat16).clone()
    flat_k, flat_v = key.view(-1), value.view(-1)
    width = case.tables.shape[1]
    out = O.multi_from_raw(
        case.qk, case.v, case.sqk, case.sqk_factor, O.EPS,
        torch.zeros(case.tokens, dtype=torch.int64), flat_k, flat_v, tuple(key.shape),
        key.stride(), case.tables.reshape(-1),
        torch.tensor([r * width for r in case.table_rows]), case.seq_lens, case.window,
        case.scale, case.gate, case.num_heads, case.num_kv_heads, shared_cache=case.shared,
        second_rounding=second_rounding)
    return out, key, value


@pytest.mark.parametrize("name", sorted(CASES))
def test_inputs_regenerate(name):
    assert str(load(name)["digest"]) == specs.digest(CASES[name]())


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_attention(name):
    g = load(name)
    case = CASES[name]()
    out, _, _ = run_oracle(case, second_rounding=False)
    ref = torch.from_numpy(g["out"])
    assert out.shape == ref.shape
    torch.testing.assert_close(out, ref, atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_kernel_rounding_within_tolerance(name):
    g = load(name)
    out, _, _ = run_oracle(CASES[name](), second_rounding=True)
    torch.testing.assert_close(out, torch.from_numpy(g["out"]), atol=2e-2, rtol=1e-2)
    assert O.relative_error(out, torch.from_numpy(g["out"])) < 5e-3


def _ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """bf16 ulp distance of two int16 bit arrays (same-sign values)."""
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


# The one element of all golden cases where the oracle's bf16 query differs from the
# reference's normalize_rows result: (case, token, q head, dim, oracle bits, reference bits).
QUERY_DIFFERENCES = [("wavefront_window", 2, 17, 78, 15464, 15465)]


def test_normalisation_vs_reference_bits():
    """The canonical normalisation against the reference's normalize_rows bit patterns over
    every golden case: the appended k and v rows (the cache contents) match on every
    element; the bf16 query matches on every element but the one listed in
    QUERY_DIFFERENCES, one bf16 ulp away."""
    k_total = q_total = 0
    q_diffs = []
    for name, build in CASES.items():
        g = load(name)
        case = build()
        for t in range(case.tokens):
            q, k, v = O.raw_qkv(case.qk[t], case.v[t], case.sqk, case.sqk_factor, O.EPS,
                                case.num_heads, case.num_kv_heads, case.head_dim)
            km = k.view(torch.int16).numpy().reshape(g["k_new"][t].shape)
            assert np.array_equal(km, g["k_new"][t]), (name, t)
            assert np.array_equal(v.view(torch.int16).numpy(), g["v_new"][t]), (name, t)
            k_total += km.size
            ref = g["q_bf16"][t].reshape(q.shape)
            mine = q.view(torch.int16).numpy().reshape(ref.shape)
            q_total += mine.size
            for h, dim in np.argwhere(mine != ref):
                q_diffs.append((name, t, int(h), int(dim), int(mine[h, dim]), int(ref[h, dim])))
    assert q_diffs == QUERY_DIFFERENCES, q_diffs
    assert k_total == 22_272 and q_total == 91_136  # elements compared (113,408 in all)


def test_the_query_difference_is_the_reference_fp32_rsqrt():
    """The one query element the oracle rounds differently from the reference's eager code:
    the exact value (rational arithmetic on the same FP32 inputs) lies below the midpoint
    of its two bf16 neighbours, so round-to-nearest gives the oracle's bits.  The reference
    computes torch.rsqrt in FP32, which PyTorch evaluates as 1 / sqrt with two roundings:
    one FP32 ulp above the correctly rounded inverse square root, enough to push the product
    over the midpoint.  The same eager expression in FP64 gives the oracle's bits, so
    PyTorch eager itself gives two different bits for this element."""
    from fractions import Fraction
    name, t, h, dim, mine, ref_bits = QUERY_DIFFERENCES[0]
    case = CASES[name]()
    NH, HD = case.num_heads, case.head_dim
    x = case.qk[t][: NH * HD].view(NH, HD)[h]
    s2 = (case.sqk.float()[h * HD + dim] * case.sqk_factor).square()  # FP32, as the reference
    sum32 = x.square().sum() + O.EPS  # FP32 sum (equal to the FP64 sum rounded, here)
    assert float(sum32) == float(np.float32(np.float32((x.double() ** 2).sum().item()) +
                                            np.float32(O.EPS)))

    def bits(v: torch.Tensor) -> int:
        return int(v.to(torch.bfloat16).view(torch.int16))

    def bf16_value(b: int) -> Fraction:
        return Fraction(float(torch.tensor([b], dtype=torch.int16).view(torch.bfloat16)))

    # exact value of s2 * x[dim] / sqrt(sum32), compared with the bf16 midpoint by squaring
    # (all quantities positive): value < mid  <=>  (s2 * x)^2 < mid^2 * sum32
    mid = (bf16_value(mine) + bf16_value(ref_bits)) / 2
    num = (Fraction(float(s2)) * Fraction(float(x[dim]))) ** 2
    assert num < mid * mid * Fraction(float(sum32)), "the exact value is below the midpoint"
    assert bf16_value(mine) < mid < bf16_value(ref_bits)

    r32 = torch.rsqrt(sum32)  # the reference's FP32 inverse square root
    r64 = torch.rsqrt(sum32.double()).float()  # the correctly rounded FP32 value
    assert r32.item() == np.nextafter(np.float32(r64.item()), np.float32(1.0))  # one ulp above
    assert bits(s2 * (x[dim] * r32)) == ref_bits  # the reference's eager expression, FP32
    assert bits(s2 * (x[dim] * r64)) == mine      # the same in FP64 precision: the oracle
    q, _, _ = O.raw_qkv(case.qk[t], case.v[t], case.sqk, case.sqk_factor, O.EPS, NH,
                        case.num_kv_heads, HD)
    assert int(q.view(torch.int16).reshape(NH, HD)[h, dim]) == mine


def test_cache_after_append_is_reference_layout():
    """Only the appended slots change, and they hold the appended rows."""
    case = CASES["wavefront"]()
    out, key, value = run_oracle(case, second_rounding=True)
    before_k = case.key.to(torch.bfloat16)
    changed = (key != before_k).flatten(2).any(-1)  # [blocks, B]
    slots = {case.slot(t) for t in range(case.tokens)}
    B = case.block_size
    changed_slots = {int(b) * B + int(o) for b, o in changed.nonzero().tolist()}
    assert changed_slots <= slots


def test_split_layout_restatement():
    # dory_decode_attention.py:28-44 on hand-worked examples
    assert O.split_layout(641, 0, 16, 32, 1) == (641, 0, 0, 41, 2)
    assert O.split_layout(0, 0, 16, 32, 1) == (0, 0, 0, 0, 1)
    assert O.split_layout(3000, 1024, 16, 32, 1) == (3000, 1976, 123, 65, 3)
    assert O.split_layout(17, 0, 16, 32, 2) == (17, 0, 0, 1, 1)


def test_padding_token_zero_output_and_no_write():
    case = CASES["config1"]()
    key = case.key.to(torch.bfloat16).clone()
    value = case.value.to(torch.bfloat16).clone()
    before = key.clone()
    out = O.from_raw(case.qk[0], case.v[0], case.sqk, case.sqk_factor, O.EPS, -1, key, value,
                     case.tables[0], 0, 0, case.scale, case.gate[0], case.num_heads,
                     case.num_kv_heads)
    assert torch.count_nonzero(out) == 0
    assert torch.equal(key, before)


def test_nibble_major_layout():
    x = torch.arange(64, dtype=torch.float32)
    nm = O.nibble_major(x)
    assert nm.shape == (8, 8)
    for e in range(64):
        assert nm[e % 8, e // 8] == x[e]


@given(seq_len=st.integers(0, 20000), window=st.sampled_from([0, 1, 15, 16, 17, 1024, 4096]),
       block=st.sampled_from([16, 32, 64]), splits=st.integers(1, 148),
       bpt=st.integers(1, 8))
@settings(max_examples=400, deadline=None)
def test_split_layout_partitions_the_attended_blocks(seq_len, window, block, splits, bpt):
    """For any sequence length, window, block size, split count and tile size, the splits'
    tile ranges [s * tps, min((s + 1) * tps, tiles)) are contiguous, disjoint and cover every
    tile exactly once; the tiles cover the attended blocks; at most `splits` are active."""
    n, first, first_block, tiles, tps = O.split_layout(seq_len, window, block, splits, bpt)
    assert n == seq_len and tps >= 1
    assert first == (max(seq_len - window, 0) if window > 0 else 0)
    assert first_block == first // block
    num_blocks = -(-seq_len // block) - first_block
    assert tiles == -(-num_blocks // bpt)
    covered = []
    for s in range(splits):
        lo, hi = s * tps, min((s + 1) * tps, tiles)
        covered.extend(range(lo, hi))
    assert covered == list(range(tiles))
    active = -(-tiles // tps)
    assert active <= splits
    # blocks of the range: tiles * bpt reaches the last attended block, no tile is empty
    assert tiles * bpt >= num_blocks > (tiles - 1) * bpt or tiles == 0
