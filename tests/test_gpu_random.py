"""Seeded random sweep of the kernel's parameter space against the oracle.

Each case draws a head shape (head_dim 64/128/256, 1-16 query heads per KV head), a block
size (16/32/64), a window, a call form (single token through from_raw, a batch with padding
requests, a shared-cache wavefront of 1-16 tokens), a split setting (splits,
blocks_per_tile, min_blocks_per_split), the L2 prefetch distance, a cache layout and, half of the time, NaN in every
cache row no token attends.  Outputs must meet the bf16 bar (2e-2 abs / 1e-2 rel) against the oracle and the
whole pool must be bit for bit the oracle's after the append.
"""

from __future__ import annotations

import random

import pytest
import torch

import workloads as W
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run
from test_gpu_edge_rows import poison_outside

pytestmark = pytest.mark.gpu


def draw(seed: int):
    rng = random.Random(seed)
    hd = rng.choice([64, 128, 256])
    g = rng.choice([1, 2, 4, 8] + ([16] if hd <= 128 else []))
    nkv = rng.choice([1, 2, 4, 8])
    while g * nkv > 64:
        nkv //= 2
    nh = g * nkv
    block = rng.choice([16, 16, 32, 64])
    window = rng.choice([0, 0, rng.randint(1, 1500)])
    shape = dict(num_heads=nh, num_kv_heads=nkv, head_dim=hd, block_size=block)
    kind = rng.choice(["single", "batched", "wavefront"])
    if kind == "single":
        context = rng.randint(0, 3000)
        need = -(-(context + 1) // block)
        case = W.single(seed=seed, context=context, pool_blocks=need + rng.randint(0, 20),
                        window=window, **shape)
    elif kind == "batched":
        lens = [rng.randint(0, 2500) for _ in range(rng.randint(1, 12))]
        case = W.batched(seed=seed, lens=lens, window=window, **shape)
        for t in range(case.tokens):
            if rng.random() < 0.15:
                case.seq_lens[t] = 0  # padding request
    else:
        case = W.wavefront(seed=seed, prompt=rng.randint(1, 2000), generated=rng.randint(0, 50),
                           tokens=rng.randint(1, 16), window=window, **shape)
    launch = dict(splits=rng.choice([1, 2, 3, 8, 16, 32, 64]),
                  blocks_per_tile=rng.choice([1, 1, 2]),
                  min_blocks_per_split=rng.choice([1, 1, 4, 32]))
    layout = rng.choice(W.LAYOUTS)
    poison = rng.random() < 0.5
    # the L2 prefetch distance, from a second stream so the cases above stay those of
    # earlier sweeps
    rng2 = random.Random(seed * 7 + 1)
    launch["prefetch_chunks"] = rng2.choice([0, 0, -1, 1, 3, 1000])
    return case, launch, layout, poison


@pytest.mark.parametrize("seed", range(1000, 1160))
def test_random_case(seed):
    case, launch, layout, poison = draw(seed)
    if poison:
        case = poison_outside(case)
    out, d, before = run(case, layout, **launch)
    assert_close(out, oracle_out(case))
    exp = expected_raw(case, layout, before, oracle_rows(case))
    assert torch.equal(d["raw"].cpu().view(torch.int16), exp.view(torch.int16))
