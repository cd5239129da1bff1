"""The wavefront engine's KV-cache addressing for multi-token attention calls.

The reference's WavefrontEngine binds, once, every attention layer's vLLM caches and block
tables (`_bind_caches`, kernels/dory_wavefront_engine.py:257-332) and then runs each
recurrent-block call as one `multi_from_raw` over its in-flight rows
(`_multi_block`, :393-410): row t of a k-row call is at loop depth k - 1 - t (:314, :418),
and it reads the cache of that loop and the block table that loop's layer uses.  This
module is that binding on this build:

* `loop_cache_offsets(caches)`: the element offset of each loop's cache from a common base
  (a data-pointer delta, :295-300), after checking that the loops' caches share one layout.
  The base is the loop cache at the LOWEST address, so every offset is a non-negative whole
  number of cache blocks when the caches are slices of one allocation (as vLLM's are): the
  kernel then reaches every loop's blocks through the base view's tensor map; a negative or
  partial-block offset would send the call down the kernel's slower copy path.
* `WavefrontLayer`: one attention layer's key / value views (either vLLM layout, through
  `kv_cache_views`), its loops' cache offsets and block-table indices, and the int64
  per-token offset tensors of every loop pattern a call uses, built once (:312-323) so that
  calls can be captured in CUDA graphs: (k - 1, ..., 1, 0) for k = 1 .. loops, plus (0,)
  and (0, 0) for the readouts.
* `WavefrontAttention(attention).attention_call(layer, pattern, ...)`: the multi-token call of
  `_multi_block` for those rows; `shared_cache` for the recurrent layers of a "last_loop"
  cache (one cache that all loops overwrite, :330-331).
* `entry_slots(block_tables, position, block_size)`: the slot of a new token at `position`
  in each block table, as `_enter` computes it for its single-token `from_raw` calls
  (:372-374).
"""

from __future__ import annotations

import torch

from dory_decode_attention import DecodeAttention
from vllm_binding import kv_cache_views


def recurrent_pattern(rows: int) -> tuple[int, ...]:
    """Loop depth of each in-flight row of a `rows`-row recurrent call: row t at rows-1-t."""
    return tuple(rows - 1 - t for t in range(rows))


def call_patterns(loops: int) -> list[tuple[int, ...]]:
    """Every loop pattern the engine's calls use (:312-313)."""
    return [recurrent_pattern(k) for k in range(1, loops + 1)] + [(0,), (0, 0)]


def loop_cache_offsets(caches: list[torch.Tensor]) -> tuple[int, list[int]]:
    """(index of the base cache, element offset of each loop's cache from it).  ValueError
    when the loops' caches differ in shape, strides or dtype, or a delta is not a whole
    number of elements (the reference's check, :293-300)."""
    if not caches:
        raise ValueError("no caches")
    base = min(range(len(caches)), key=lambda i: caches[i].data_ptr())
    ref = caches[base]
    offsets = []
    for cache in caches:
        delta = cache.data_ptr() - ref.data_ptr()
        if (cache.stride() != ref.stride() or cache.shape != ref.shape
                or cache.dtype != ref.dtype or cache.device != ref.device
                or delta % cache.element_size()):
            raise ValueError("a layer's loop caches differ in layout")
        offsets.append(delta // cache.element_size())
    return base, offsets


class WavefrontLayer:
    """One attention layer bound for the wavefront's calls.

    kv_caches: the layer's vLLM KV-cache tensor of every loop, as the engine collects them
    (:270-276): a recurrent layer with per-loop caches lists one tensor per loop, a shared
    "last_loop" cache lists the same tensor for every loop, a non-recurrent layer lists
    one; table_indices: the block-table row each loop uses in the engine's [tables, width]
    block-table tensor; width: that tensor's row length."""

    def __init__(self, kv_caches: list[torch.Tensor], table_indices: list[int], width: int,
                 num_kv_heads: int, head_dim: int):
        if len(table_indices) != len(kv_caches):
            raise ValueError("one block-table index per loop cache")
        base, self.loop_offsets = loop_cache_offsets(kv_caches)
        self.key, self.value = kv_cache_views(kv_caches[base], num_kv_heads, head_dim)
        self.loops = len(kv_caches)
        self.table_indices = list(table_indices)
        self.width = width
        self.block_size = self.key.shape[1]
        dev = kv_caches[base].device
        self.token_cache_offsets: dict[tuple[int, ...], torch.Tensor] = {}
        self.token_table_offsets: dict[tuple[int, ...], torch.Tensor] = {}
        for pattern in call_patterns(self.loops):
            if max(pattern) >= self.loops:
                continue
            self.token_cache_offsets[pattern] = torch.tensor(
                [self.loop_offsets[loop] for loop in pattern], dtype=torch.int64, device=dev)
            self.token_table_offsets[pattern] = torch.tensor(
                [self.table_indices[loop] * width for loop in pattern], dtype=torch.int64,
                device=dev)

    def offsets(self, pattern: tuple[int, ...]) -> tuple[torch.Tensor, torch.Tensor]:
        """(cache offsets, block-table offsets) of a call's rows, int64 [rows] each."""
        try:
            return self.token_cache_offsets[pattern], self.token_table_offsets[pattern]
        except KeyError:
            raise ValueError(f"loop pattern {pattern} is not one this layer's calls use "
                             f"({self.loops} loop cache(s))") from None


class WavefrontAttention:
    """One DecodeAttention instance (its scratch) serving every layer's wavefront calls."""

    def __init__(self, attention: DecodeAttention):
        self.attention = attention

    def attention_call(self, layer: WavefrontLayer, pattern: tuple[int, ...],
                       qk: torch.Tensor, v: torch.Tensor, sqk: torch.Tensor, sqk_factor: float,
                       eps: float, block_tables: torch.Tensor, seq_lens: torch.Tensor,
                       window: int, softmax_scale: float, gate: torch.Tensor,
                       out_nibble_major: torch.Tensor, shared_cache: bool = False,
                       out_sumsq: torch.Tensor | None = None) -> None:
        """The rows' multi_from_raw (qk FP32 [rows, (heads + kv_heads) * head_dim], v, gate,
        out_nibble_major [rows, 8, heads * head_dim / 8], seq_lens int32 [rows]; row t at
        loop pattern[t]) against the layer's caches and the engine's block tables
        ([tables, width], contiguous)."""
        if block_tables.dim() != 2 or block_tables.shape[1] != layer.width:
            raise ValueError("block_tables must be [tables, width] with the layer's width")
        if len(pattern) != qk.shape[0]:
            raise ValueError("one loop depth per row")
        cache_offsets, table_offsets = layer.offsets(pattern)
        self.attention.multi_from_raw(qk, v, sqk, sqk_factor, eps, cache_offsets, layer.key,
                                      layer.value, block_tables, table_offsets, seq_lens,
                                      window, softmax_scale, gate, out_nibble_major,
                                      shared_cache=shared_cache, out_sumsq=out_sumsq)


def entry_slots(block_tables: torch.Tensor, position: torch.Tensor, block_size: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """int64 slot of a token at `position` (int64 [1], on the device) in every row of the
    block tables [tables, width]: table[position // block_size] * block_size + position %
    block_size (:372-374).  Device arithmetic only (no host read), so it can be captured."""
    physical = block_tables[:, torch.div(position, block_size, rounding_mode="floor")]
    slots = physical.reshape(-1).to(torch.int64) * block_size + position % block_size
    if out is not None:
        out.copy_(slots)
        return out
    return slots


__all__ = ["recurrent_pattern", "call_patterns", "loop_cache_offsets", "WavefrontLayer",
           "WavefrontAttention", "entry_slots"]
