"""vllm_binding on the host (no GPU): the cache views of both vLLM layouts and the refusal
of non-decode batches."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from vllm_binding import VllmDecodeBinding, kv_cache_views


def test_vllm_022_layout_views():
    kv = torch.arange(3 * 2 * 16 * 4 * 8, dtype=torch.float32).view(3, 2, 16, 4, 8)
    key, value = kv_cache_views(kv, 4, 8)
    assert key.shape == value.shape == (3, 16, 4, 8)
    assert torch.equal(key, kv[:, 0]) and torch.equal(value, kv[:, 1])
    assert key.stride() == value.stride() and key.stride(-1) == 1


def test_pinned_layout_views():
    kv = torch.arange(3 * 4 * 16 * 16, dtype=torch.float32).view(3, 4, 16, 16)
    key, value = kv_cache_views(kv, 4, 8)
    assert key.shape == value.shape == (3, 16, 4, 8)
    assert torch.equal(key[1, 5, 2], kv[1, 2, 5, :8]) and torch.equal(value[1, 5, 2], kv[1, 2, 5, 8:])
    assert key.stride() == value.stride() and key.stride(-1) == 1


def test_unrecognised_layout():
    with pytest.raises(ValueError):
        kv_cache_views(torch.zeros(3, 2, 16, 4, 16), 4, 8)


def test_prefill_batches_are_refused():
    attn = SimpleNamespace(max_tokens=4, device=torch.device("cpu"), num_kv_heads=4, head_dim=8)
    binding = VllmDecodeBinding(attn)
    meta = SimpleNamespace(max_query_len=5, seq_lens=torch.ones(2, dtype=torch.int32),
                           block_table=torch.zeros(2, 4, dtype=torch.int32))
    with pytest.raises(NotImplementedError):
        binding.decode(meta, torch.zeros(3, 2, 16, 4, 8), torch.zeros(2, 48), torch.zeros(2, 32),
                       None, 0.7, 1e-6, 0, 1.0, None, None)
