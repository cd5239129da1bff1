"""The separate q/k normalisation step of the reference's fused Dory attention sublayer
(kernels/dory_attention.py), on the B200 library.

The reference's FusedAttentionSublayer runs a q/k/v/gate GEMV, this step, the attention and
the output GEMV.  Only this step belongs to the decode-attention path: it produces the
normalised bf16 query that DecodeAttention.__call__ takes, and writes the token's k and v
into the paged cache (pre_attention, dory_attention.py:218-236) or returns them in bf16
(pre_attention_qkv, dory_attention.py:238-250).  The GEMVs are not part of this build.

* `qk_norm_cache(...)`: the step for one token or a batch of tokens.
* `_qk_norm_cache_kernel`: the reference kernel's launch form (dory_attention.py:69-96, as
  launched at dory_attention.py:231-236, 244-249 and bench_decode_attention.py:146-150),
  for code that launches it directly:
  `_qk_norm_cache_kernel[(NH + NKV,)](qk, v, sqk, q_out, key_cache, value_cache,
  slot_mapping, k_out, v_out, sqk_factor, eps, stride_block, stride_offset, stride_head,
  NUM_Q_HEADS=NH, HEAD_DIM=HD, CACHE_BLOCK=B, WRITE_CACHE=True, num_warps=2)`.

The arithmetic is the fused raw-mode kernel's: q_out = bf16((sqk * sqk_factor)^2 *
q * rsqrt(sum q^2 + eps)), k = bf16(k * rsqrt(sum k^2 + eps)), v = bf16(v), with the sum of
squares accumulated in FP64 and the inverse square root correctly rounded, so the separate
path and DecodeAttention.from_raw append the same bits.
"""

from __future__ import annotations

import ctypes

import torch

import _native
from dory_decode_attention import _SQK_DTYPES


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def qk_norm_cache(qk: torch.Tensor, v: torch.Tensor, sqk: torch.Tensor, sqk_factor: float,
                  eps: float, q_out: torch.Tensor, num_heads: int, head_dim: int, *,
                  key_cache: torch.Tensor | None = None, value_cache: torch.Tensor | None = None,
                  slot_mapping: torch.Tensor | None = None, k_out: torch.Tensor | None = None,
                  v_out: torch.Tensor | None = None,
                  error_word: torch.Tensor | None = None) -> None:
    """Normalises q and k of T tokens (qk FP32 [T, (NH + NKV) * HD] or [(NH + NKV) * HD],
    v FP32 [T, NKV * HD]) into q_out (bf16 [T, NH * HD]) and either writes k and v into the
    paged cache views key_cache / value_cache ([blocks, block_size, NKV, HD]) at
    slot_mapping[t] (int64; negative = padding, no write) or stores them in k_out / v_out
    (bf16 [T, NKV * HD]).  error_word: optional int32 device tensor that collects
    DORY_DEVERR_SLOT_OOB for slots outside the cache.  Enqueued on the current stream."""
    write_cache = key_cache is not None
    for name, t in (("qk", qk), ("v", v)):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous float32")
    if q_out.dtype != torch.bfloat16 or not q_out.is_contiguous():
        raise ValueError("q_out must be contiguous bfloat16")
    if not qk.is_cuda:
        raise RuntimeError("qk_norm_cache runs on CUDA tensors only (no CPU path)")
    num_tokens = qk.shape[0] if qk.dim() == 2 else 1
    num_kv_heads = v.shape[-1] // head_dim
    if qk.shape[-1] != (num_heads + num_kv_heads) * head_dim:
        raise ValueError("qk must hold num_heads q heads and num_kv_heads k heads")
    p = _native.DoryQkNormParams()
    p.qk, p.v, p.sqk, p.q_out = qk.data_ptr(), v.data_ptr(), sqk.data_ptr(), q_out.data_ptr()
    sqk_dtype = _SQK_DTYPES.get(sqk.dtype)
    if sqk_dtype is None:
        raise ValueError(f"unsupported sqk dtype {sqk.dtype}")
    if write_cache:
        if value_cache is None or slot_mapping is None:
            raise ValueError("the cache write needs value_cache and slot_mapping")
        if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1:
            raise ValueError("key and value caches need equal strides and unit last stride")
        if slot_mapping.dtype != torch.int64:
            raise ValueError("slot_mapping must be int64")
        p.key_cache, p.value_cache = key_cache.data_ptr(), value_cache.data_ptr()
        p.slot_mapping = slot_mapping.data_ptr()
        p.stride_block, p.stride_offset, p.stride_head = key_cache.stride()[:3]
        p.num_cache_blocks = key_cache.shape[0]
        p.block_size = key_cache.shape[1]
        p.flags = _native.QKNORM_WRITE_CACHE
    else:
        if k_out is None or v_out is None:
            raise ValueError("k_out and v_out are needed without a cache write")
        for name, t in (("k_out", k_out), ("v_out", v_out)):
            if t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous bfloat16")
        p.k_out, p.v_out = k_out.data_ptr(), v_out.data_ptr()
        p.flags = 0
    p.error_word = _ptr(error_word)
    p.sqk_factor, p.eps, p.sqk_dtype = float(sqk_factor), float(eps), sqk_dtype
    p.num_tokens, p.num_heads, p.num_kv_heads, p.head_dim = (num_tokens, num_heads,
                                                             num_kv_heads, head_dim)
    stream = torch.cuda.current_stream(qk.device).cuda_stream
    _native.check(_native.load().dory_qk_norm_cache(ctypes.byref(p), ctypes.c_void_p(stream)))


class _QkNormCacheLaunch:
    """`_qk_norm_cache_kernel[grid](...)`: the reference Triton kernel's launch form.  The
    grid is (NUM_Q_HEADS + kv_heads,); one token; WRITE_CACHE selects the cache write (the
    cache views' shapes give the block count) or k_out / v_out."""

    def __getitem__(self, grid):
        heads = grid[0] if isinstance(grid, (tuple, list)) else int(grid)

        def launch(qk, v, sqk, q_out, key_cache, value_cache, slot_mapping, k_out, v_out,
                   sqk_factor, eps, stride_block, stride_offset, stride_head, *,
                   NUM_Q_HEADS, HEAD_DIM, CACHE_BLOCK, WRITE_CACHE, num_warps=None,
                   num_stages=None):
            num_kv_heads = heads - NUM_Q_HEADS
            if v.numel() != num_kv_heads * HEAD_DIM:
                raise ValueError("grid must be (NUM_Q_HEADS + kv_heads,)")
            if WRITE_CACHE:
                if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1:
                    raise ValueError("key and value caches need equal strides and unit last "
                                     "stride")
                p_cache = dict(key_cache=key_cache, value_cache=value_cache,
                               slot_mapping=slot_mapping)
            else:
                p_cache = dict(k_out=k_out, v_out=v_out)
            if WRITE_CACHE and (tuple(key_cache.stride()[:3]) !=
                                (stride_block, stride_offset, stride_head)
                                or key_cache.shape[1] != CACHE_BLOCK):
                raise ValueError("strides / CACHE_BLOCK do not describe key_cache")
            qk_norm_cache(qk.view(-1), v.view(-1), sqk, sqk_factor, eps, q_out.view(-1),
                          NUM_Q_HEADS, HEAD_DIM, **p_cache)

        return launch


_qk_norm_cache_kernel = _QkNormCacheLaunch()

__all__ = ["qk_norm_cache", "_qk_norm_cache_kernel"]
