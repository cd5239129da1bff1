"""Gated decode attention over vLLM's paged BF16 KV cache, on B200 (sm_100a).

Drop-in for the reference module `kernels/dory_decode_attention.py`: the class name,
constructor, the three call methods, their argument meaning, tensor contracts and
ValueError conditions are the same, so callers written against the reference
(`dory_fused_model.py:190-193`, `dory_wavefront_engine.py:393-396, 414-419`,
`dory_multi_token.py:202-205`) run unchanged with this directory on `sys.path`.

Each call is ONE launch of a hand-written CUDA kernel (libdory_decode.so, C ABI in
include/dory_decode.h) on the current CUDA stream: q/k normalisation, the K/V append at
vLLM's slot, split-KV flash decoding over the paged cache, the LSE merge of the splits,
the sigmoid gate product and the nibble-major FP32 store.  Nothing is allocated per call
and nothing waits on the device, so calls can be captured in CUDA graphs.  There is no
CPU or Triton path: CPU tensors, a missing library or an unsupported shape raise.

Cache views are stride-generic `[num_blocks, block_size, num_kv_heads, head_dim]` BF16
tensors with equal key/value strides and unit last stride — e.g. vLLM's Triton backend
cache `[blocks, kv_heads, block_size, 2 * head_dim]` seen through
`kv.transpose(1, 2).split(head_dim, -1)` (dory_fused_model.py:137), vLLM 0.22's
`(blocks, 2, block_size, kv_heads, head_dim).unbind(1)`, or the reference benchmark's
`[blocks, block_size, kv_heads, 2 * head_dim].split(head_dim, -1)`.
"""

from __future__ import annotations

import ctypes

import torch

import _native

EPS = 1e-6  # as the reference's dory_common.EPS (vLLM Dory justnorm)

_SQK_DTYPES = {torch.float32: _native.DTYPE_F32, torch.bfloat16: _native.DTYPE_BF16,
               torch.float16: _native.DTYPE_F16}


# kv_cache_dtype names (vLLM's) -> DoryDecodeParams.kv_dtype
_KV_DTYPES = {"auto": _native.DTYPE_BF16, "bf16": _native.DTYPE_BF16,
              "fp8": _native.DTYPE_FP8_E4M3, "fp8_e4m3": _native.DTYPE_FP8_E4M3}
_FP8_CACHE_DTYPES = (torch.float8_e4m3fn, torch.uint8)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class DecodeAttention:
    """Gated decode attention with scratch buffers for a fixed split count.

    One query token per call (__call__, from_raw), or up to max_tokens tokens at once
    (multi_from_raw), each with its own position, cache and block table.  Mirrors
    `DecodeAttention` of the reference (dory_decode_attention.py:225-331).

    num_warps, num_stages and dim_chunk are Triton launch knobs of the reference; they are
    accepted for signature compatibility and ignored (this kernel's pipeline depth and warp
    roles are fixed per head_dim).  blocks_per_tile keeps its meaning: the granularity, in
    cache blocks, of the split ranges.  min_blocks_per_split (B200 addition) keeps short
    sequences from being cut into splits of a block or two.  overlap_launch (B200 addition,
    off by default) launches each call as a programmatic dependent of the previous kernel on
    the stream, so its prologue and K/V loads overlap that kernel's tail; the kernel right
    before a call must then not write the call's seq_lens, block tables, offsets,
    slot_mapping or the cache rows it attends (q/k/v/gate inputs are still ordered).
    prefetch_chunks (B200 addition): how far ahead of its shared-memory ring each CTA starts
    the DRAM reads of its K/V chunks into L2; 0 picks automatically (a CTA's whole range
    for overlapped launches that fit in one wave of CTAs, else none), a negative value
    turns it off.  consumer (B200 addition): "mma" (default) computes the score and P.V dot
    products with mma.sync tensor-core tiles, "fma" with FP32 FMAs on the CUDA cores, the
    measured alternative (128-dim heads, at most 4 query heads per KV head, no shared cache).
    kv_cache_dtype (B200 addition, vLLM's name): "auto" / "bf16" for bf16 caches (the
    reference's), "fp8" / "fp8_e4m3" for caches of e4m3 bytes (torch.float8_e4m3fn or uint8
    views of the same shape), K = e4m3 * k_scale and V = e4m3 * v_scale, the scales passed
    to each call (vLLM's per-layer k_scale / v_scale, default 1.0); a raw call appends
    e4m3(bf16(k) / k_scale) and e4m3(bf16(v) / v_scale) (round to nearest even, saturated at
    +-448) and attends those values, shared caches included.  128/256-dim heads, at most 8
    query heads per KV head.
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, device: torch.device,
                 splits: int = 32, blocks_per_tile: int = 1, num_warps: int = 4,
                 num_stages: int = 2, dim_chunk: int = 64, max_tokens: int = 1,
                 min_blocks_per_split: int = 1, overlap_launch: bool = False,
                 prefetch_chunks: int = 0, consumer: str = "mma",
                 kv_cache_dtype: str = "auto"):
        if num_heads % num_kv_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.group = num_heads // num_kv_heads
        self.splits, self.blocks_per_tile, self.num_warps = splits, blocks_per_tile, num_warps
        self.num_stages, self.dim_chunk = num_stages, dim_chunk
        self.max_tokens = max_tokens
        self.min_blocks_per_split = min_blocks_per_split
        self.overlap_launch = bool(overlap_launch)
        self.prefetch_chunks = int(prefetch_chunks)
        if consumer not in ("mma", "fma"):
            raise ValueError("consumer must be 'mma' or 'fma'")
        self.consumer = consumer
        if kv_cache_dtype not in _KV_DTYPES:
            raise ValueError(f"kv_cache_dtype must be one of {sorted(_KV_DTYPES)}")
        self.kv_cache_dtype = kv_cache_dtype
        self._kv8 = _KV_DTYPES[kv_cache_dtype] == _native.DTYPE_FP8_E4M3
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("DecodeAttention runs on CUDA devices only (no CPU path)")
        self._lib = _native.load()
        self.no_offset = torch.zeros(1, dtype=torch.int64, device=self.device)
        nbytes = self._lib.dory_decode_scratch_bytes(max_tokens, splits, num_heads, num_kv_heads,
                                                     head_dim)
        if nbytes <= 0:
            raise ValueError("invalid scratch shape")
        # Partials [max_tokens, splits, heads, head_dim] + (max, sum) + merge counters + the
        # device error word, in one caller-owned buffer (the reference's partial_out /
        # partial_max / partial_sum, dory_decode_attention.py:242-246).
        self.scratch = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _native.check(self._lib.dory_decode_scratch_init(self.scratch.data_ptr(), nbytes,
                                                             stream))
        self._params = _native.DoryDecodeParams()
        self._params_ref = ctypes.byref(self._params)
        self._dev_index = self.scratch.get_device()
        # Fields fixed for this instance are set once; _launch sets the per-call ones.
        p = self._params
        p.scratch, p.scratch_bytes = self.scratch.data_ptr(), self.scratch.numel()
        p.num_heads, p.num_kv_heads, p.head_dim = num_heads, num_kv_heads, head_dim
        p.splits, p.blocks_per_tile = splits, blocks_per_tile
        p.min_blocks_per_split, p.max_tokens = min_blocks_per_split, max_tokens
        p.prefetch_chunks = self.prefetch_chunks
        self._base_flags = ((_native.FLAG_OVERLAP_LAUNCH if self.overlap_launch else 0) |
                            (_native.FLAG_FMA_CONSUMER if consumer == "fma" else 0))
        p.kv_dtype = _KV_DTYPES[kv_cache_dtype]
        p.k_scale = p.v_scale = 1.0

    # ---- the reference's three entry points ----

    def __call__(self, q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 block_table: torch.Tensor, seq_lens: torch.Tensor, window: int,
                 softmax_scale: float, gate: torch.Tensor, out_nibble_major: torch.Tensor,
                 out_sumsq: torch.Tensor | None = None, *, k_scale: float = 1.0,
                 v_scale: float = 1.0) -> None:
        """q: BF16 [heads * head_dim], already in the cache's k and v; block_table:
        [max_blocks] of this sequence; seq_lens: [1] tokens including this one;
        window: 0 for full attention; gate: FP32 [heads * head_dim];
        out_nibble_major: FP32 [8, heads * head_dim / 8]."""
        self._launch(q, key_cache, value_cache, block_table, seq_lens, window, softmax_scale,
                     gate, out_nibble_major, raw=None, tokens=1, cache_offsets=None,
                     out_sumsq=out_sumsq, k_scale=k_scale, v_scale=v_scale)

    def from_raw(self, qk: torch.Tensor, v: torch.Tensor, sqk: torch.Tensor, sqk_factor: float,
                 eps: float, slot_mapping: torch.Tensor, key_cache: torch.Tensor,
                 value_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                 window: int, softmax_scale: float, gate: torch.Tensor,
                 out_nibble_major: torch.Tensor, out_sumsq: torch.Tensor | None = None, *,
                 k_scale: float = 1.0, v_scale: float = 1.0) -> None:
        """Like __call__, from the rotated, unnormalized q and k heads (FP32
        [(heads + kv_heads) * head_dim]) and v (FP32 [kv_heads * head_dim]); also
        writes this token's k and v into the cache at slot_mapping[0]."""
        self._launch(qk, key_cache, value_cache, block_table, seq_lens, window, softmax_scale,
                     gate, out_nibble_major, raw=(v, sqk, sqk_factor, eps, slot_mapping),
                     tokens=1, cache_offsets=None, out_sumsq=out_sumsq, k_scale=k_scale,
                     v_scale=v_scale)

    def multi_from_raw(self, qk: torch.Tensor, v: torch.Tensor, sqk: torch.Tensor,
                       sqk_factor: float, eps: float, cache_offsets: torch.Tensor,
                       key_cache: torch.Tensor, value_cache: torch.Tensor,
                       block_tables: torch.Tensor, block_table_offsets: torch.Tensor,
                       seq_lens: torch.Tensor, window: int, softmax_scale: float,
                       gate: torch.Tensor, out_nibble_major: torch.Tensor,
                       shared_cache: bool = False, out_sumsq: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None, *, k_scale: float = 1.0,
                       v_scale: float = 1.0) -> None:
        """from_raw for T tokens: qk [T, (heads + kv_heads) * head_dim], v [T, kv_heads *
        head_dim], gate [T, heads * head_dim], out_nibble_major [T, 8, heads * head_dim / 8],
        seq_lens [T].  Token t is at position seq_lens[t] - 1 and uses the cache at
        key_cache / value_cache shifted by cache_offsets[t] elements and the block table at
        block_tables shifted by block_table_offsets[t] elements; it writes its key and value
        at the slot that block table gives for its position.  Offsets are int64.

        The tokens may be one sequence's wavefront (positions p..p+T-1) or T independent
        sequences (the batched decode: one table row each through block_table_offsets).

        shared_cache: tokens may read each other's slots (several loops sharing one cache,
        where an older token's slot holds its latest loop); every token then sees the
        others' new entries, as if all were cached before attention (the reference's
        write-all-first order), without a second launch.

        out_sumsq (optional, all three calls; no counterpart in the reference's signature):
        FP32 [T] receiving sum over e of out[t][e]^2, the gated output's squared norm that
        the consumer's output GEMV normalises by (dory_attention.py:114-117).

        slot_mapping (optional, no counterpart in the reference's signature): int64 [>= T];
        token t then writes its key and value at slot_mapping[t] instead of the slot its
        block table gives (a negative slot writes nothing), as vLLM's slot_mapping specifies
        it, padded rows included."""
        tokens = qk.shape[0]
        if (tokens > self.max_tokens or cache_offsets.dtype != torch.int64
                or block_table_offsets.dtype != torch.int64):
            raise ValueError("too many tokens for the scratch buffers, or non-int64 offsets")
        if slot_mapping is not None and (slot_mapping.numel() < tokens
                                         or not slot_mapping.is_contiguous()):
            raise ValueError("slot_mapping needs one contiguous int64 entry per token")
        self._launch(qk, key_cache, value_cache, block_tables, seq_lens, window, softmax_scale,
                     gate, out_nibble_major, raw=(v, sqk, sqk_factor, eps, slot_mapping),
                     tokens=tokens, cache_offsets=cache_offsets,
                     block_table_offsets=block_table_offsets, shared=shared_cache,
                     out_sumsq=out_sumsq, k_scale=k_scale, v_scale=v_scale)

    # ---- diagnostics ----

    def fetch_errors(self, clear: bool = True) -> int:
        """Device error bits (DORY_DEVERR_*) recorded since the last clear.  Synchronises the
        current stream; meant for tests and debugging, not for the decode loop."""
        flags = ctypes.c_uint32(0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.check(self._lib.dory_decode_fetch_errors(self.scratch.data_ptr(),
                                                         ctypes.byref(flags), int(clear), stream))
        return flags.value

    def check_errors(self) -> None:
        """Raises RuntimeError naming every device error bit recorded since the last check."""
        flags = self.fetch_errors(clear=True)
        if flags:
            names = [name for bit, name in _native.DEVERR_NAMES.items() if flags & bit]
            raise RuntimeError("decode attention device errors: " + ", ".join(names))

    # ---- launch ----

    def _launch(self, q, key_cache, value_cache, block_table, seq_lens, window, softmax_scale,
                gate, out_nibble_major, raw, tokens, cache_offsets,
                block_table_offsets=None, shared=False, out_sumsq=None, k_scale=1.0,
                v_scale=1.0) -> None:
        if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1:
            raise ValueError("key and value caches need equal strides and unit last stride")
        want = _FP8_CACHE_DTYPES if self._kv8 else (torch.bfloat16,)
        if key_cache.dtype not in want or value_cache.dtype not in want:
            raise ValueError("key and value caches must be bfloat16" if not self._kv8 else
                             "fp8 key and value caches must be float8_e4m3fn or uint8")
        if not key_cache.is_cuda:
            raise RuntimeError("DecodeAttention runs on CUDA tensors only (no CPU path)")
        dev = self._dev_index
        if key_cache.get_device() != dev:
            raise ValueError(f"caches on {key_cache.device}, this instance's scratch on "
                             f"{self.scratch.device}")
        _native.check_device_index(dev, q, value_cache, block_table, seq_lens, gate,
                                   out_nibble_major, out_sumsq, cache_offsets,
                                   block_table_offsets,
                                   *(raw[:2] + raw[4:] if raw is not None else ()))
        if key_cache.shape[-1] != self.head_dim or key_cache.shape[-2] != self.num_kv_heads:
            raise ValueError("cache view must be [blocks, block_size, kv_heads, head_dim]")
        if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
            raise ValueError("block tables and seq_lens must be int32")
        p = self._params
        flags = self._base_flags
        if raw is not None:
            v, sqk, sqk_factor, eps, slot_mapping = raw
            if q.dtype != torch.float32 or v.dtype != torch.float32:
                raise ValueError("raw q/k and v must be float32")
            sqk_dtype = _SQK_DTYPES.get(sqk.dtype)
            if sqk_dtype is None:
                raise ValueError(f"unsupported sqk dtype {sqk.dtype}")
            if slot_mapping is not None and slot_mapping.dtype != torch.int64:
                raise ValueError("slot_mapping must be int64")
            flags |= _native.FLAG_RAW_QKV
            p.v, p.sqk, p.slot_mapping = v.data_ptr(), sqk.data_ptr(), _ptr(slot_mapping)
            p.sqk_factor, p.eps, p.sqk_dtype = float(sqk_factor), float(eps), sqk_dtype
        else:
            if q.dtype != torch.bfloat16:
                raise ValueError("q must be bfloat16 (already normalised and scaled)")
            p.v = p.sqk = p.slot_mapping = None
            p.sqk_factor, p.eps, p.sqk_dtype = 0.0, 0.0, _native.DTYPE_F32
        if cache_offsets is not None:
            flags |= _native.FLAG_MULTI_TOKEN
            if shared:
                flags |= _native.FLAG_SHARED_CACHE
            p.cache_offsets, p.block_table_offsets = cache_offsets.data_ptr(), block_table_offsets.data_ptr()
        else:
            p.cache_offsets = p.block_table_offsets = None
        if gate.dtype != torch.float32 or out_nibble_major.dtype != torch.float32:
            raise ValueError("gate and out_nibble_major must be float32")
        for t in (q, gate, out_nibble_major, seq_lens):
            if not t.is_contiguous():
                raise ValueError("q/qk, v, gate, seq_lens and out_nibble_major must be contiguous")
        p.q, p.key_cache, p.value_cache = q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr()
        p.block_table, p.seq_lens = block_table.data_ptr(), seq_lens.data_ptr()
        p.gate, p.out_nibble_major = gate.data_ptr(), out_nibble_major.data_ptr()
        if out_sumsq is not None:
            if (out_sumsq.dtype != torch.float32 or not out_sumsq.is_contiguous()
                    or out_sumsq.numel() < tokens):
                raise ValueError("out_sumsq must be contiguous float32 with one entry per token")
            p.out_sumsq = out_sumsq.data_ptr()
        else:
            p.out_sumsq = None
        ks = key_cache.stride()
        p.stride_block, p.stride_offset, p.stride_head = ks[0], ks[1], ks[2]
        shape = key_cache.shape
        p.num_cache_blocks, p.block_size = shape[0], shape[1]
        p.softmax_scale = float(softmax_scale)
        if self._kv8:
            p.k_scale, p.v_scale = float(k_scale), float(v_scale)
        p.num_tokens, p.window, p.flags = tokens, int(window), flags
        # the current stream's handle (torch.cuda.current_stream(dev).cuda_stream, without
        # building the Stream object)
        stream = torch._C._cuda_getCurrentRawStream(dev)
        status = self._lib.dory_decode_attention(self._params_ref, stream)
        if status:
            _native.check(status)
