"""Host logic of wavefront_binding (no GPU): the engine's per-loop cache offsets and loop
patterns (kernels/dory_wavefront_engine.py:257-332), on CPU tensors."""

from __future__ import annotations

import pytest
import torch

import wavefront_binding as WB

NKV, HD, B, BLOCKS = 2, 64, 16, 10


def carve(order, layout="pinned"):
    """Per-loop caches carved out of one buffer, loop i at slot order[i] (vLLM allocates a
    KV-cache group's layers as slices of one tensor)."""
    shape = (BLOCKS, NKV, B, 2 * HD) if layout == "pinned" else (BLOCKS, 2, B, NKV, HD)
    n = BLOCKS * NKV * B * 2 * HD
    buf = torch.zeros(len(order) * n, dtype=torch.bfloat16)
    return [buf[o * n:(o + 1) * n].view(shape) for o in order], n


def test_patterns_match_the_engine():
    assert WB.recurrent_pattern(3) == (2, 1, 0)
    assert WB.call_patterns(3) == [(0,), (1, 0), (2, 1, 0), (0,), (0, 0)]


@pytest.mark.parametrize("layout", ["pinned", "vllm"])
def test_offsets_are_whole_blocks_from_the_lowest_cache(layout):
    caches, n = carve([2, 0, 1], layout)  # loop 1's cache sits lowest in memory
    base, offsets = WB.loop_cache_offsets(caches)
    assert base == 1
    assert offsets == [2 * n, 0, n]
    layer = WB.WavefrontLayer(caches, [0, 1, 2], 7, NKV, HD)
    assert layer.key.data_ptr() == caches[1].data_ptr()
    per_block = layer.key.stride(0)
    assert all(o % per_block == 0 and o >= 0 for o in offsets)
    cache, table = layer.offsets((2, 1, 0))
    assert cache.tolist() == [offsets[2], offsets[1], offsets[0]]
    assert table.tolist() == [14, 7, 0]
    assert cache.dtype == table.dtype == torch.int64
    assert set(layer.token_cache_offsets) == {(0,), (1, 0), (2, 1, 0), (0, 0)}


def test_shared_cache_repeats_one_tensor():
    (cache,), _ = carve([0])
    layer = WB.WavefrontLayer([cache] * 3, [4] * 3, 5, NKV, HD)
    c, t = layer.offsets((2, 1, 0))
    assert c.tolist() == [0, 0, 0] and t.tolist() == [20, 20, 20]


def test_single_cache_layer_refuses_deeper_patterns():
    (cache,), _ = carve([0])
    layer = WB.WavefrontLayer([cache], [0], 5, NKV, HD)
    assert layer.offsets((0, 0))[0].tolist() == [0, 0]
    with pytest.raises(ValueError):
        layer.offsets((1, 0))


def test_layout_mismatch_is_refused():
    caches, _ = carve([0, 1])
    other = torch.zeros(BLOCKS + 1, NKV, B, 2 * HD, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        WB.loop_cache_offsets([caches[0], other])
    with pytest.raises(ValueError):
        WB.loop_cache_offsets([caches[0], caches[1].float()])
    with pytest.raises(ValueError):
        WB.WavefrontLayer(caches, [0], 5, NKV, HD)  # one table index per loop


def test_entry_slots():
    tables = torch.tensor([[5, 3, 9], [1, 2, 8]], dtype=torch.int32)
    slots = WB.entry_slots(tables, torch.tensor([17]), 16)
    assert slots.tolist() == [3 * 16 + 1, 2 * 16 + 1] and slots.dtype == torch.int64
    out = torch.empty(2, dtype=torch.int64)
    WB.entry_slots(tables, torch.tensor([40]), 16, out=out)
    assert out.tolist() == [9 * 16 + 8, 8 * 16 + 8]
