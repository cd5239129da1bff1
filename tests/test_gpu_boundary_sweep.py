"""Sequence lengths from 0 to 9000 around block and window boundaries (the reference's
edge-case sweep, EXPERIMENTS.md:325-327 and :535-536, whose script is not in the reference):
every length k * 16 - 1, k * 16, k * 16 + 1 for a stride of k up to 9000, the lengths around
window sizes and powers of two, and 0 (a padding request), as batched calls of independent
sequences (8q/2kv x 64 heads keep the CPU oracle fast) with full attention and windows that
start inside and on a block; the same lengths through FP8 caches; and four-token shared-cache
wavefronts that straddle a block boundary.  Outputs within the bf16 bar (2e-2 abs / 1e-2 rel)
of the oracle, the pool bit for bit after the appends.
"""

from __future__ import annotations

import pytest
import torch

import dory_oracle as O
import workloads as W
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run

pytestmark = pytest.mark.gpu

SHAPE = dict(num_heads=8, num_kv_heads=2, head_dim=64)


def boundary_lengths() -> list[int]:
    """seq_len values (the new token included) near block and window boundaries."""
    out = {1, 2, 3}
    for k in range(1, 563, 9):
        out.update({16 * k - 1, 16 * k, 16 * k + 1})
    for w in (1023, 1024, 1025, 2047, 2048, 2049, 4095, 4096, 4097, 8191, 8192, 8193, 9000):
        out.add(w)
    return sorted(n for n in out if 1 <= n <= 9000)


def batches(lens, size=48):
    return [lens[i:i + size] for i in range(0, len(lens), size)]


@pytest.mark.parametrize("window", [0, 1024, 1000, 17])
@pytest.mark.parametrize("part", range(4))
def test_batched_boundaries(window, part):
    lens = boundary_lengths()
    groups = batches(lens)
    for i, group in enumerate(groups):
        if i % 4 != part:
            continue
        ctx = [n - 1 for n in group] + [0]  # and a padding request
        case = W.batched(seed=1400 + i + window, lens=ctx, window=window, **SHAPE)
        case.seq_lens[-1] = 0
        out, d, before = run(case, "triton", splits=8, min_blocks_per_split=4)
        assert_close(out, oracle_out(case))
        exp = expected_raw(case, "triton", before, oracle_rows(case))
        assert torch.equal(d["raw"].cpu().view(torch.int16), exp.view(torch.int16))


@pytest.mark.parametrize("window", [0, 1000])
def test_fp8_boundaries(window):
    from test_gpu_fp8_cache import run_fp8
    lens = boundary_lengths()[::3]
    for i, group in enumerate(batches(lens, 40)):
        case = W.batched(seed=1500 + i + window, lens=[n - 1 for n in group], window=window,
                         num_heads=16, num_kv_heads=4, head_dim=128)
        out, want, (k, v), (k8, v8) = run_fp8(case, splits=8, scales=(0.5, 0.5))
        assert_close(out, want)
        assert torch.equal(k, k8) and torch.equal(v, v8)


@pytest.mark.parametrize("prompt", [14, 15, 16, 30, 1021, 1022, 2045, 8189])
@pytest.mark.parametrize("window", [0, 1024])
def test_wavefront_across_a_block_boundary(prompt, window):
    case = W.wavefront(seed=1600 + prompt, prompt=prompt, generated=0, tokens=4, window=window,
                       **SHAPE)
    out, d, before = run(case, "triton", splits=4)
    assert_close(out, oracle_out(case))
    exp = expected_raw(case, "triton", before, oracle_rows(case))
    assert torch.equal(d["raw"].cpu().view(torch.int16), exp.view(torch.int16))
