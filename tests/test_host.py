"""Host-side logic that needs no GPU: constructor contract, workloads, request partition."""

from __future__ import annotations

import math

import pytest
import torch

import workloads as W
from dory_decode_attention import DecodeAttention


def test_constructor_rejects_bad_group_like_reference():
    # dory_decode_attention.py:235-236
    with pytest.raises(ValueError, match="multiple of KV heads"):
        DecodeAttention(30, 8, 128, torch.device("cuda"))


def test_constructor_refuses_cpu():
    with pytest.raises(RuntimeError, match="CUDA"):
        DecodeAttention(32, 8, 128, torch.device("cpu"))


def test_config_lengths_match_the_stated_workloads():
    lens3 = W.config3_lens()
    assert len(lens3) == 64 and min(lens3) >= 128 and max(lens3) <= 1152
    assert sum(lens3) == 39362
    lens5 = W.config5_lens()
    assert len(lens5) == 512 and min(lens5) >= 128 and max(lens5) <= 8192
    assert sum(lens5) == 1_038_941


@pytest.mark.parametrize("parts", [1, 2, 4, 8])
def test_partition_is_complete_and_balanced(parts):
    lens = W.config5_lens()
    split = W.partition(lens, parts)
    flat = sorted(i for part in split for i in part)
    assert flat == list(range(len(lens)))
    loads = [sum(lens[i] + 1 for i in part) for part in split]
    # greedy LPT: every part within one longest request of the mean
    assert max(loads) - min(loads) <= max(lens) + 1
    assert max(loads) <= math.ceil(sum(loads) / parts) + max(lens)


def test_partition_deterministic():
    lens = W.config5_lens()
    assert W.partition(lens, 4) == W.partition(lens, 4)


@pytest.mark.parametrize("layout", W.LAYOUTS)
def test_cache_layouts_view_same_geometry(layout):
    raw, key, value = W.cache_views(3, 16, 8, 128, layout, "cpu")
    assert key.shape == value.shape == (3, 16, 8, 128)
    assert key.stride() == value.stride() and key.stride(-1) == 1
    key.zero_()
    value.fill_(1)
    assert torch.count_nonzero(key) == 0  # key and value do not overlap
    assert raw.float().sum() == 3 * 16 * 8 * 128


def test_case_slots_follow_block_table():
    case = W.single(seed=0)
    pos = 640
    assert case.slot(0) == int(case.tables[0, pos // 16]) * 16 + pos % 16
    wf = W.wavefront(seed=1, prompt=100, tokens=4)
    assert [wf.slot(t) % 16 for t in range(4)] == [(100 + t) % 16 for t in range(4)]
