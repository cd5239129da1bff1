"""The CPU oracle against the golden vectors the reference's own eager code produced.

Pins oracle/dory_oracle.py before any kernel is compared with it:
* inputs regenerated from the seeds hash to the digests stored by make_golden.py;
* with the reference's single q rounding the oracle reproduces `reference_attention` to
  FP32 accuracy; with the kernel's second rounding it stays inside the bf16 tolerance;
* appended k / v / q match the reference's `normalize_rows` bit patterns (all but a
  fraction of rows to the bit, the rest within one bf16 ulp — FP32 summation order).
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


def test_normalisation_vs_reference_bits():
    """The canonical normalisation against the reference's normalize_rows bit patterns,
    over every golden case: exact on >= 99% of elements, never more than 1 ulp away."""
    total = exact = 0
    worst = 0
    for name, build in CASES.items():
        g = load(name)
        case = build()
        for t in range(case.tokens):
            q, k, v = O.raw_qkv(case.qk[t], case.v[t], case.sqk, case.sqk_factor, O.EPS,
                                case.num_heads, case.num_kv_heads, case.head_dim)
            for mine, ref in ((k, g["k_new"][t]), (q, g["q_bf16"][t].reshape(q.shape))):
                m = mine.view(torch.int16).numpy().reshape(ref.shape)
                d = _ulps(m, ref)
                total += d.size
                exact += int((d == 0).sum())
                worst = max(worst, int(d.max()))
            assert np.array_equal(v.view(torch.int16).numpy(), g["v_new"][t])
    assert worst <= 1
    assert exact / total >= 0.99, exact / total


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
