"""The bench's workload definitions (CPU only): every named workload resolves, the reference
benchmark's shape (kernels/bench_decode_attention.py: 16q/4kv x 256, the two-loop decode
order, window 1024 on layers with layer % 4 != 3) is what the dory workloads run, and the
algorithmic byte count behind the roofline agrees with an independent count over the
oracle's attended ranges."""

from __future__ import annotations

import random
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
import dory_oracle as O  # noqa: E402
import workloads as W  # noqa: E402


def independent_bytes(seq_lens, shared, window, nh, nkv, hd, block=16):
    """Counts attended positions and table entries one by one."""
    ranges = [range(*O.attended(n, window)) for n in seq_lens]
    if shared:
        groups = [set().union(*map(set, ranges))]
    else:
        groups = [set(r) for r in ranges]
    unique = sum(len(g) for g in groups)
    entries = sum(len({p // block for p in g}) for g in groups)
    token_io = ((nh + nkv) * hd + nkv * hd + 2 * nh * hd) * 4
    return (unique * nkv * hd * 4 + len(seq_lens) * token_io + nh * hd * 2 + entries * 4
            + 4 * len(seq_lens))


@pytest.mark.parametrize("name", bench.WORKLOADS)
def test_every_workload_resolves(name):
    spec = bench.workload_spec(name)
    splits, mbs = bench.tuned_splits(name, 1)
    assert splits >= 1 and mbs >= 1
    assert spec.lens and spec.layers
    assert spec.nh % spec.nkv == 0 and spec.hd in (64, 128, 256)


def test_unknown_workload_is_an_error():
    with pytest.raises(SystemExit):
        bench.workload_spec("dory1000")


@pytest.mark.parametrize("context", [640, 2048, 8192])
def test_dory_shape(context):
    spec = bench.workload_spec(f"dory{context}")
    assert (spec.nh, spec.nkv, spec.hd) == (16, 4, 256)
    assert spec.lens == [context] and not spec.shared
    order = bench.DECODE_ORDER_2_LOOPS
    assert len(order) == 56 and order[:8] == list(range(8)) and order[-8:] == list(range(28, 36))
    # one cache per application, window by the decode-order layer it stands for
    assert spec.layers == list(range(56))
    for app, layer in enumerate(order):
        assert spec.window(app) == (1024 if layer % 4 != 3 else 0)
    assert sum(1 for a in spec.layers if spec.window(a) == 1024) == 42


def test_config5_bytes_pinned():
    """The per-launch byte count the committed config-5 roofline is quoted on."""
    lens = [n + 1 for n in W.config5_lens()]
    assert bench.algorithmic_bytes(lens, False, 0, 32, 8, 128) == 4_287_230_696


@pytest.mark.parametrize("window", [0, 1, 15, 16, 17, 1024])
@pytest.mark.parametrize("shared", [False, True])
def test_bytes_match_independent_count(window, shared):
    rng = random.Random(window * 2 + shared)
    if shared:
        p = rng.randint(1, 3000)
        lens = [p + t + 1 for t in range(4)]
    else:
        lens = [rng.randint(1, 3000) for _ in range(20)] + [1, 16, 17, 1024, 1025]
    for nh, nkv, hd in ((32, 8, 128), (16, 4, 256), (8, 8, 64)):
        assert bench.algorithmic_bytes(lens, shared, window, nh, nkv, hd) == \
            independent_bytes(lens, shared, window, nh, nkv, hd)


def test_cpu_sample_weights_windows():
    sample = bench.CpuSample("dory640")
    weights = {c.window: n for c, _, _, n in sample.cases}
    assert weights == {0: 14, 1024: 42}
    for c, _, _, _ in sample.cases:
        assert (c.num_heads, c.num_kv_heads, c.head_dim) == (16, 4, 256)
    measured, step = sample.once()
    assert 0 < measured < step  # two applications timed, the step's 56 estimated


def test_cpu_sample_covers_every_sequence():
    """The CPU pass runs one layer over ALL of a batched workload's sequences (config 3's
    64 here; config 5's 512 the same way), and a wavefront's four tokens for config 2."""
    sample = bench.CpuSample("config3")
    (case, key, value, n), = sample.cases
    assert n == 36 and case.tokens == 64 and sample.lens == W.config3_lens()
    assert key.dtype == torch.bfloat16 and key.shape[0] == case.num_blocks
    wave = bench.CpuSample("config2")
    assert wave.tokens == 4 and wave.cases[0][0].shared and wave.cases[0][3] == 20


def test_small_workloads_replay_several_steps_over_distinct_pools():
    """Config 1's 36 caches hold 97 MB, less than L2: a replay then covers enough steps,
    each over its own pools, to read more than 3 x 126 MB."""
    spec = bench.workload_spec("config1")
    pool = -(-(spec.lens[0] + 1) // 16) * 16 * 8 * 128 * 2 * 2
    reps = -(-int(bench.MIN_REPLAY_BYTES) // (pool * 36))
    assert reps == 4 and pool * 36 * reps > 3 * 126e6


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rank_sequences_cover_the_partition(world):
    """Each rank launches exactly its partition share; at 8+ GPUs config 5's shares run
    longest first, below that in request order."""
    lens = bench.workload_spec("config5").lens
    seen = []
    for rank in range(world):
        mine = bench.rank_sequences("config5", lens, world, rank)
        assert sorted(mine) == W.partition(lens, world)[rank]
        ctx = [lens[i] for i in mine]
        if world >= 8:
            assert ctx == sorted(ctx, reverse=True)
        else:
            assert mine == sorted(mine)
        seen += mine
    assert sorted(seen) == list(range(len(lens)))
    assert bench.tuned_splits("config5", world) == {1: (2, 64), 2: (4, 64), 4: (4, 64),
                                                     8: (3, 64)}[world]


def test_sublayer_bytes_add_the_residual_io():
    """--path sublayer adds, per token, the output GEMV's partials, the sublayer input, h in
    both layouts and the output statistic written and read; alpha once per launch."""
    H, lens = 2560, [100, 2000, 7]
    base = bench.algorithmic_bytes(lens, False, 1024, 16, 4, 256, bench.QKVG_SPLIT_K)
    sub = bench.algorithmic_bytes(lens, False, 1024, 16, 4, 256, bench.QKVG_SPLIT_K, H)
    per_token = bench.RESIDUAL_SPLIT_K * H * 4 + H * 2 + H * 2 + H * 4 + 8
    assert sub - base == len(lens) * per_token + H * 2
