"""DecodeAttention fed from vLLM's own per-layer decode state.

The reference binds its fused decoder to vLLM through the model runner: for every attention
layer it takes vLLM's KV-cache tensor and attention metadata (`get_attention_context`,
kernels/dory_wavefront_engine.py:273), reads the BF16 Triton-backend cache through key /
value views (:292, kernels/dory_fused_model.py:137) and the layer's block table from the
metadata (each KV-cache group has its own table, :280-284).  This module
does that step for a decode batch:

* `kv_cache_views(kv_cache, num_kv_heads, head_dim)`: one layer's cache tensor ->
  [blocks, block_size, kv_heads, head_dim] key / value views.  vLLM 0.22's Triton backend
  allocates (blocks, 2, block_size, kv_heads, head_dim) and unbinds dim 1
  (TritonAttentionBackend.get_kv_cache_shape, TritonAttentionImpl.forward); the vLLM build
  the reference pins allocates (blocks, kv_heads, block_size, 2 * head_dim), read through
  transpose(1, 2).split(head_dim, -1).
* `VllmDecodeBinding(attention).decode(metadata, kv_cache, qk, v, ...)`: one decode step of
  one layer from the metadata's `seq_lens` (int32 [num_reqs], the new token included) and
  `block_table` (int32 [num_reqs, max_blocks], a row per request) as
  DecodeAttention.multi_from_raw, token t = request t.  The new token's k / v go to the
  slot the metadata's `slot_mapping` (int64 [num_tokens]) gives, as vLLM's backends write
  the cache (`reshape_and_cache`): a negative slot writes nothing; padded requests (seq_len
  0, slot -1 in vLLM's CUDA-graph padding) write nothing and output zero.

Only decode batches (max_query_len == 1) are taken: prefill stays on vLLM's attention, as in
the reference.  vLLM itself is not imported: the metadata is read by attribute.  Row
offsets are allocated once per block-table row stride and kept, so calls can be captured in
CUDA graphs after the first one.
"""

from __future__ import annotations

import torch

from dory_decode_attention import DecodeAttention


def kv_cache_views(kv_cache: torch.Tensor, num_kv_heads: int, head_dim: int):
    """(key, value) [blocks, block_size, kv_heads, head_dim] views of one layer's vLLM cache."""
    if (kv_cache.dim() == 5 and kv_cache.shape[1] == 2 and kv_cache.shape[3] == num_kv_heads
            and kv_cache.shape[4] == head_dim):
        key, value = kv_cache.unbind(1)
    elif (kv_cache.dim() == 4 and kv_cache.shape[1] == num_kv_heads
          and kv_cache.shape[3] == 2 * head_dim):
        key, value = kv_cache.transpose(1, 2).split(head_dim, dim=-1)
    else:
        raise ValueError(f"unrecognised vLLM KV-cache shape {tuple(kv_cache.shape)} for "
                         f"{num_kv_heads} kv heads of {head_dim} dims")
    return key, value


class VllmDecodeBinding:
    """One DecodeAttention instance (its scratch) serving vLLM decode steps layer by layer."""

    def __init__(self, attention: DecodeAttention):
        self.attention = attention
        n = attention.max_tokens
        self._cache_offsets = torch.zeros(n, dtype=torch.int64, device=attention.device)
        self._row_offsets: dict[int, torch.Tensor] = {}

    def _rows(self, stride: int) -> torch.Tensor:
        rows = self._row_offsets.get(stride)
        if rows is None:
            rows = torch.arange(self.attention.max_tokens, dtype=torch.int64,
                                device=self.attention.device) * stride
            self._row_offsets[stride] = rows
        return rows

    def decode(self, metadata, kv_cache: torch.Tensor, qk: torch.Tensor, v: torch.Tensor,
               sqk: torch.Tensor, sqk_factor: float, eps: float, window: int,
               softmax_scale: float, gate: torch.Tensor, out_nibble_major: torch.Tensor,
               out_sumsq: torch.Tensor | None = None, k_scale: float = 1.0,
               v_scale: float = 1.0) -> None:
        """qk FP32 [T, (heads + kv_heads) * head_dim] (rotated, not normalised), v FP32
        [T, kv_heads * head_dim], gate FP32 [T, heads * head_dim], out_nibble_major FP32
        [T, 8, heads * head_dim / 8], for the T = qk.shape[0] requests of the batch.  With
        an attention instance built for kv_cache_dtype="fp8", kv_cache is vLLM's fp8 cache
        (uint8 e4m3 bytes, the same shape) and k_scale / v_scale the layer's float scales."""
        if int(metadata.max_query_len) != 1:
            raise NotImplementedError("only decode batches (one query token per request); "
                                      "prefill stays on vLLM's attention")
        tokens = qk.shape[0]
        seq_lens, table = metadata.seq_lens, metadata.block_table
        if seq_lens.numel() < tokens or table.shape[0] < tokens:
            raise ValueError("metadata covers fewer requests than qk has rows")
        if table.dim() != 2 or table.stride(1) != 1:
            raise ValueError("block_table must be [num_reqs, max_blocks] with unit last stride")
        slots = metadata.slot_mapping
        if slots.dtype != torch.int64 or slots.numel() < tokens:
            raise ValueError("slot_mapping must be int64 with one entry per token")
        a = self.attention
        key, value = kv_cache_views(kv_cache, a.num_kv_heads, a.head_dim)
        a.multi_from_raw(qk, v, sqk, sqk_factor, eps, self._cache_offsets[:tokens], key, value,
                         table, self._rows(table.stride(0))[:tokens], seq_lens[:tokens], window,
                         softmax_scale, gate, out_nibble_major, out_sumsq=out_sumsq,
                         slot_mapping=slots[:tokens], k_scale=k_scale, v_scale=v_scale)
