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
* `WavefrontRecurrentBlock`: every non-GEMM step of the recurrent block's attention
  sublayers for a k-row call (`_recurrent` / `_multi_block`, :405-432), the GEMVs' split-K
  partials given, launched plainly or replayed as one CUDA graph per k (`_run`, :336-347).
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
                       out_sumsq: torch.Tensor | None = None, *, k_scale: float = 1.0,
                       v_scale: float = 1.0) -> None:
        """The rows' multi_from_raw (qk FP32 [rows, (heads + kv_heads) * head_dim], v, gate,
        out_nibble_major [rows, 8, heads * head_dim / 8], seq_lens int32 [rows]; row t at
        loop pattern[t]) against the layer's caches and the engine's block tables
        ([tables, width], contiguous).  k_scale / v_scale: the layer's FP8 cache scales
        (an instance built with kv_cache_dtype="fp8")."""
        if block_tables.dim() != 2 or block_tables.shape[1] != layer.width:
            raise ValueError("block_tables must be [tables, width] with the layer's width")
        if len(pattern) != qk.shape[0]:
            raise ValueError("one loop depth per row")
        cache_offsets, table_offsets = layer.offsets(pattern)
        self.attention.multi_from_raw(qk, v, sqk, sqk_factor, eps, cache_offsets, layer.key,
                                      layer.value, block_tables, table_offsets, seq_lens,
                                      window, softmax_scale, gate, out_nibble_major,
                                      shared_cache=shared_cache, out_sumsq=out_sumsq,
                                      k_scale=k_scale, v_scale=v_scale)


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


class AttentionSublayer:
    """One attention layer of the recurrent block: its bound caches (WavefrontLayer) and the
    per-layer inputs of the non-GEMM steps of `MultiTokenSublayers.attention`
    (kernels/dory_multi_token.py:183-210): sqk for the q normalisation, s_gate and the
    rotary cos/sin table for the q/k/v/gate epilogue, alpha for the residual update, the
    layer's window and softmax scale, and its FP8 cache scales (k_scale / v_scale, used when
    the block's DecodeAttention has kv_cache_dtype="fp8")."""

    def __init__(self, layer: WavefrontLayer, sqk: torch.Tensor, s_gate: torch.Tensor,
                 cos_sin: torch.Tensor, alpha: torch.Tensor, window: int, softmax_scale: float,
                 k_scale: float = 1.0, v_scale: float = 1.0):
        self.layer, self.sqk, self.s_gate, self.cos_sin = layer, sqk, s_gate, cos_sin
        self.alpha, self.window, self.softmax_scale = alpha, int(window), float(softmax_scale)
        self.k_scale, self.v_scale = float(k_scale), float(v_scale)


class WavefrontRecurrentBlock:
    """The attention sublayers of the wavefront engine's recurrent block for one k-row call
    (`_recurrent` / `_multi_block`, kernels/dory_wavefront_engine.py:405-432): for every
    attention layer in order, the q/k/v/gate epilogue on the layer's q/k/v/gate GEMV
    partials, the rows' multi_from_raw at loop pattern (k - 1, ..., 0) with the output's
    sum of squares, and the residual update on the layer's output-GEMV partials fed that
    statistic; each layer's h is the next layer's residual input (ping-pong buffers).

    The two GEMVs of each sublayer (NVFP4, outside this build) are the caller's, in one of
    two ways.  Given as hooks, `qkvg_gemv(i, h_nm, partials)` (layer i's input h, FP32
    nibble-major [k, 8, hidden / 8], into its q/k/v/gate partials) and `out_gemv(i,
    attention_out, partials)` (the gated attention output, FP32 nibble-major [k, 8, Q / 8],
    into its output-GEMV partials) are called at their places in the chain, so a graph
    replay includes them; without hooks, the caller writes the partials into
    `qkvg_partials(i, k)` / `out_partials(i, k)` (the engine's prefix views, [split_k, k,
    rows]) before a call, e.g. seeded stand-ins.  `run(k, ...)` launches the block;
    `replay(k, ...)` runs it as one CUDA graph per k, the first call for a k running it
    plainly and then capturing it (`_run`, :336-347).  shared_cache: the recurrent layers'
    "last_loop" caches (one per layer, written and read by every loop)."""

    def __init__(self, attention: DecodeAttention, layers: list[AttentionSublayer],
                 block_tables: torch.Tensor, hidden: int, sqk_factor: float,
                 s_gate_factor: float, alpha_scale: float, eps: float,
                 shared_cache: bool = True, qkvg_split_k: int = 2, out_split_k: int = 4,
                 qkvg_gemv=None, out_gemv=None):
        a = attention
        self.qkvg_gemv, self.out_gemv = qkvg_gemv, out_gemv
        self.wave = WavefrontAttention(a)
        self.layers, self.block_tables = layers, block_tables
        self.NH, self.NKV, self.HD = a.num_heads, a.num_kv_heads, a.head_dim
        self.hidden, self.sqk_factor, self.s_gate_factor = hidden, sqk_factor, s_gate_factor
        self.alpha_scale, self.eps, self.shared_cache = alpha_scale, eps, shared_cache
        self.qkvg_split_k, self.out_split_k = qkvg_split_k, out_split_k
        rows, dev = a.max_tokens, a.device
        Q, KV = self.NH * self.HD, self.NKV * self.HD
        self.qkvg_rows = 2 * (Q + KV)
        f32 = dict(dtype=torch.float32, device=dev)
        self._qkvg = [torch.zeros(qkvg_split_k * rows * self.qkvg_rows, **f32) for _ in layers]
        self._out = [torch.zeros(out_split_k * rows * hidden, **f32) for _ in layers]
        self.qk = torch.empty(rows, Q + KV, **f32)
        self.v = torch.empty(rows, KV, **f32)
        self.gate = torch.empty(rows, Q, **f32)
        self.attention_out = torch.empty(rows, 8, Q // 8, **f32)
        self.sumsq = torch.empty(rows, **f32)
        self.h = [torch.empty(rows, hidden, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.h_nm = [torch.empty(rows, 8, hidden // 8, **f32) for _ in range(2)]
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}

    def qkvg_partials(self, i: int, k: int) -> torch.Tensor:
        """Layer i's q/k/v/gate GEMV partials for a k-row call, FP32 [split_k, k, rows]."""
        n = self.qkvg_split_k * k * self.qkvg_rows
        return self._qkvg[i][:n].view(self.qkvg_split_k, k, self.qkvg_rows)

    def out_partials(self, i: int, k: int) -> torch.Tensor:
        """Layer i's output-GEMV partials for a k-row call, FP32 [split_k, k, hidden]."""
        n = self.out_split_k * k * self.hidden
        return self._out[i][:n].view(self.out_split_k, k, self.hidden)

    def run(self, k: int, positions: torch.Tensor, seq_lens: torch.Tensor,
            h_in: torch.Tensor, h_in_nm: torch.Tensor | None = None
            ) -> tuple[torch.Tensor, torch.Tensor]:
        """The block for rows 0 .. k-1 (row t at loop k - 1 - t; positions int64 [k],
        seq_lens int32 [k] = positions + 1) from the block input h_in (BF16 [k, hidden];
        h_in_nm, its FP32 nibble-major copy, for a qkvg_gemv hook); returns the last layer's
        h (BF16 [k, hidden]) and its nibble-major FP32 copy."""
        from dory_sublayer_steps import qkvg_epilogue, residual_tokens
        pattern = recurrent_pattern(k)
        overlap = self.wave.attention.overlap_launch
        x, x_nm = h_in, h_in_nm
        out = nm = None
        for i, sub in enumerate(self.layers):
            if self.qkvg_gemv is not None:
                self.qkvg_gemv(i, x_nm, self.qkvg_partials(i, k))
            qkvg_epilogue(self.qkvg_partials(i, k), positions[:k], sub.cos_sin, sub.s_gate,
                          self.s_gate_factor, self.qk[:k], self.v[:k], self.gate[:k], self.NH,
                          self.NKV, self.HD, overlap_launch=overlap)
            self.wave.attention_call(sub.layer, pattern, self.qk[:k], self.v[:k], sub.sqk,
                                     self.sqk_factor, self.eps, self.block_tables, seq_lens[:k],
                                     sub.window, sub.softmax_scale, self.gate[:k],
                                     self.attention_out[:k], shared_cache=self.shared_cache,
                                     out_sumsq=self.sumsq[:k], k_scale=sub.k_scale,
                                     v_scale=sub.v_scale)
            if self.out_gemv is not None:
                self.out_gemv(i, self.attention_out[:k], self.out_partials(i, k))
            out, nm = self.h[i % 2][:k], self.h_nm[i % 2][:k]
            residual_tokens(self.out_partials(i, k), None, x, sub.alpha, self.alpha_scale,
                            self.eps, out, nm, x_sumsq=self.sumsq[:k], overlap_launch=overlap)
            x, x_nm = out, nm
        return out, nm

    def replay(self, k: int, positions: torch.Tensor, seq_lens: torch.Tensor,
               h_in: torch.Tensor, h_in_nm: torch.Tensor | None = None
               ) -> tuple[torch.Tensor, torch.Tensor]:
        """`run` as one CUDA graph per k (fixed tensors: positions, seq_lens, h_in and h_in_nm
        must be the same tensors, updated in place, on every call with this k)."""
        graph = self.graphs.get(k)
        if graph is None:
            out = self.run(k, positions, seq_lens, h_in, h_in_nm)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self.run(k, positions, seq_lens, h_in, h_in_nm)
            self.graphs[k] = graph
            return out
        graph.replay()
        n = len(self.layers)
        return self.h[(n - 1) % 2][:k], self.h_nm[(n - 1) % 2][:k]


__all__ = ["recurrent_pattern", "call_patterns", "loop_cache_offsets", "WavefrontLayer",
           "WavefrontAttention", "entry_slots", "AttentionSublayer", "WavefrontRecurrentBlock"]
