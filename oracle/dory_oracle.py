"""CPU oracle of the decode-attention + KV-append path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may
import this module, and only as the checker or the timed CPU baseline.  The product path
(dory-vllm-experiments_b200/) never calls it: it has no CPU fallback.

It restates, in PyTorch eager (FP32 on CPU) and NumPy, the semantics of the reference
chrisbennight/dory-vllm-experiments:

* justnorm / normalize_rows: x * rsqrt(sum(x^2) + eps), eps = 1e-6 inside the root
  (vllm-patched/vllm/model_executor/models/dory.py:43-47, kernels/dory_common.py:20,
  kernels/bench_decode_attention.py:100-101);
* the raw-mode q, k, v of the attention kernel (kernels/dory_decode_attention.py:110-114,
  :96): q = bf16((sqk * sqk_factor)^2 * norm(q)), k = bf16(norm(k)), v = bf16(v), and the
  query scaling q = bf16(float(q) * softmax_scale) (:123);
* the attended range [max(seq_len - window, 0), seq_len) or [0, seq_len) (:28-44, :131-133);
* softmax attention through the paged block table (kernels/bench_decode_attention.py:58-68,
  `reference_attention`), GQA by repeat_interleave;
* padding: seq_len 0 gives a zero output (:218-219), slot < 0 writes nothing (:118);
* gate product and the nibble-major store out[e % 8][e / 8] (:220-222,
  kernels/w4a16_gemv.py:91-93);
* the multi-token path's q/k/v/gate epilogue (kernels/dory_multi_token.py:53-80): split-K
  sum, rotary embedding on adjacent row pairs, the scaled sigmoid output gate;
* the residual update after the output GEMV (kernels/dory_multi_token.py:109-131,
  kernels/dory_common.py:55-81): the split-K sum over the input's norm (or over a given
  sum of squares), h = n(n(a) + |alpha * alpha_scale| * (n(b) - n(a)));
* multi-token calls (:270-305): token t uses cache_offsets[t] and block_table_offsets[t];
  shared_cache=True caches every token's k/v before any attention (:294-301), which the
  reference's own test checks against single-token calls in position order
  (kernels/bench_multi_token.py:160-197);
* FP8 (e4m3) caches, which the reference does not have (its docs/FUTURE_WORK.md lists them):
  the format of vLLM's fp8 kv_cache_dtype, restated in e4m3_quantize / e4m3_dequantize and
  the *_fp8 calls ("parity unpinned" for these: no reference output exists).

Normalisation arithmetic (bit-exact cache contract).  Sum x^2 is accumulated in FP64 and
rounded once to FP32, eps is added in FP32, and the inverse square root is the correctly
rounded FP32 value; the product x * r and the bf16 rounding are FP32 round-to-nearest-even.
This removes the dependence of the FP32 sum on reduction order, which differs between
PyTorch's CPU builds (AVX2 vs AVX-512) and GPU kernels; the CUDA kernel computes exactly
these quantities, so appended cache rows compare bit for bit.  Against PyTorch's own FP32
`normalize_rows` the result agrees to the bit on the large majority of rows and within one
bf16 ulp elsewhere (tests/test_oracle.py measures both).

Parity is pinned by tests/golden/*.npz, produced by tests/golden/make_golden.py from the
reference's own eager functions (`reference_attention`, `normalize_rows`, `to_nibble_major`).
"""

from __future__ import annotations

import math

import numpy as np
import torch

EPS = 1e-6


# ---------------------------------------------------------------------------------------
# normalisation (dory.py:43-47; dory_decode_attention.py:110-114)
# ---------------------------------------------------------------------------------------

def inv_norm(x: np.ndarray, eps: float = EPS) -> np.ndarray:
    """Canonical FP32 1/sqrt(sum(x^2) + eps) over the last axis of an FP32 array."""
    x = np.asarray(x, dtype=np.float32)
    s32 = np.sum(x.astype(np.float64) ** 2, axis=-1).astype(np.float32)
    t = (s32 + np.float32(eps)).astype(np.float32)
    return (1.0 / np.sqrt(t.astype(np.float64))).astype(np.float32)


def normalize(x: np.ndarray, eps: float = EPS) -> np.ndarray:
    """FP32 x * inv_norm(x) (the product rounded once to FP32)."""
    x = np.asarray(x, dtype=np.float32)
    return (x * inv_norm(x, eps)[..., None]).astype(np.float32)


def bf16(x) -> torch.Tensor:
    """Round-to-nearest-even FP32 -> bfloat16 (torch's conversion)."""
    return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(torch.bfloat16)


def raw_qkv(qk: torch.Tensor, v: torch.Tensor, sqk: torch.Tensor, sqk_factor: float,
            eps: float, num_heads: int, num_kv_heads: int, head_dim: int):
    """(q bf16 [NH, HD] before the softmax scale, k bf16 [NKV, HD], v bf16 [NKV, HD]) of one
    token, as the raw-mode kernel computes them (dory_decode_attention.py:93-96,110-114)."""
    NH, NKV, HD = num_heads, num_kv_heads, head_dim
    x = qk.detach().float().cpu().numpy().reshape(NH + NKV, HD)
    s = (sqk.detach().float().cpu().numpy().reshape(NH, HD).astype(np.float32)
         * np.float32(sqk_factor)).astype(np.float32)
    qn = normalize(x[:NH], eps)
    q = bf16((s * s).astype(np.float32) * qn)
    k = bf16(normalize(x[NH:], eps))
    vb = v.detach().float().cpu().reshape(NKV, HD).to(torch.bfloat16)
    return q, k, vb


def scaled_query(q_bf16: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    """The kernel's second rounding, q = bf16(float(q) * softmax_scale) (:123)."""
    return (q_bf16.float() * np.float32(softmax_scale)).to(torch.bfloat16)


# ---------------------------------------------------------------------------------------
# paged attention (bench_decode_attention.py:58-68; dory_decode_attention.py:28-44,130-161)
# ---------------------------------------------------------------------------------------

def attended(seq_len: int, window: int) -> tuple[int, int]:
    first = max(seq_len - window, 0) if window > 0 else 0
    return first, seq_len


def gather(cache: torch.Tensor, table: torch.Tensor, positions: torch.Tensor,
           block_size: int) -> torch.Tensor:
    """cache [blocks, B, NKV, HD] rows for logical positions -> FP32 [len, NKV, HD]."""
    blocks = table[positions // block_size].long()
    return cache[blocks, positions % block_size].float()


def attention(q: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
              table: torch.Tensor, seq_len: int, window: int, num_heads: int,
              block_size: int, softmax_scale: float, second_rounding: bool = True
              ) -> torch.Tensor:
    """FP32 softmax attention of one token from its bf16 query [NH, HD].

    second_rounding=True follows the attention kernel (q = bf16(float(q) * scale) before the
    dot products, dory_decode_attention.py:123); False follows the reference's FP32 test
    oracle `reference_attention` (bench_decode_attention.py:58-68), which scales the FP32
    scores instead.  Returns FP32 [NH * HD]; zero for seq_len 0 (:218-219)."""
    first, last = attended(seq_len, window)
    HD = key.shape[-1]
    if last <= first:
        return torch.zeros(num_heads * HD)
    positions = torch.arange(first, last)
    keys = gather(key, table, positions, block_size)
    values = gather(value, table, positions, block_size)
    group = num_heads // keys.shape[1]
    keys = keys.repeat_interleave(group, dim=1)
    values = values.repeat_interleave(group, dim=1)
    q = q.reshape(num_heads, -1).cpu()
    if second_rounding:
        scores = torch.einsum("hd,thd->ht", scaled_query(q, softmax_scale).float(), keys)
    else:
        scores = torch.einsum("hd,thd->ht", q.float(), keys) * softmax_scale
    return torch.einsum("ht,thd->hd", scores.softmax(dim=-1), values).reshape(-1)


def nibble_major(x: torch.Tensor) -> torch.Tensor:
    """FP32 [Q] -> [8, Q/8] with element [j, w] = x[8w + j] (w4a16_gemv.py:91-93)."""
    return x.float().reshape(-1, 8).t().contiguous()


# ---------------------------------------------------------------------------------------
# the three entry points (dory_decode_attention.py:248-305); caches are modified in place
# ---------------------------------------------------------------------------------------

def _write(key, value, slot: int, block_size: int, k_new, v_new):
    key[slot // block_size, slot % block_size] = k_new
    value[slot // block_size, slot % block_size] = v_new


def call(q: torch.Tensor, key, value, block_table, seq_len: int, window: int,
         softmax_scale: float, gate: torch.Tensor, num_heads: int,
         second_rounding: bool = True) -> torch.Tensor:
    """DecodeAttention.__call__: q bf16 [NH*HD] already normalised; returns [8, Q/8]."""
    B = key.shape[1]
    out = attention(q, key, value, block_table, seq_len, window, num_heads, B, softmax_scale,
                    second_rounding)
    return nibble_major(out * gate.float().cpu())


def from_raw(qk, v, sqk, sqk_factor, eps, slot: int, key, value, block_table, seq_len: int,
             window: int, softmax_scale: float, gate, num_heads: int, num_kv_heads: int,
             second_rounding: bool = True) -> torch.Tensor:
    """DecodeAttention.from_raw on CPU tensors: appends at `slot` (if >= 0 and the token is
    not padding) and returns the gated output [8, Q/8].  The attention sees the new k/v at
    position seq_len - 1 (the reference substitutes them from registers, :141-145)."""
    HD = key.shape[-1]
    B = key.shape[1]
    q, k_new, v_new = raw_qkv(qk, v, sqk, sqk_factor, eps, num_heads, num_kv_heads, HD)
    if seq_len > 0:
        pos = seq_len - 1
        phys = int(block_table[pos // B])
        saved_k = key[phys, pos % B].clone()
        saved_v = value[phys, pos % B].clone()
        key[phys, pos % B], value[phys, pos % B] = k_new, v_new
        out = attention(q, key, value, block_table, seq_len, window, num_heads, B,
                        softmax_scale, second_rounding)
        key[phys, pos % B], value[phys, pos % B] = saved_k, saved_v
        if slot >= 0:
            _write(key, value, slot, B, k_new, v_new)
    else:
        out = torch.zeros(num_heads * HD)
    return nibble_major(out * gate.float().cpu())


def multi_from_raw(qk, v, sqk, sqk_factor, eps, cache_offsets, key_flat, value_flat,
                   cache_shape, cache_strides, block_tables_flat, block_table_offsets,
                   seq_lens, window: int, softmax_scale: float, gate, num_heads: int,
                   num_kv_heads: int, shared_cache: bool = False,
                   second_rounding: bool = True) -> torch.Tensor:
    """DecodeAttention.multi_from_raw on CPU.  key_flat / value_flat are the flat storage
    the caches live in; token t's cache view is as_strided(cache_shape, cache_strides,
    offset = cache_offsets[t]), its table block_tables_flat[block_table_offsets[t]:].
    Returns the gated outputs [T, 8, Q/8]."""
    T = qk.shape[0]
    HD = cache_shape[-1]
    B = cache_shape[1]
    views = []
    news = []
    for t in range(T):
        off = int(cache_offsets[t])
        kv = key_flat.as_strided(cache_shape, cache_strides, off)
        vv = value_flat.as_strided(cache_shape, cache_strides, off)
        table = block_tables_flat[int(block_table_offsets[t]):]
        views.append((kv, vv, table))
        news.append(raw_qkv(qk[t], v[t], sqk, sqk_factor, eps, num_heads, num_kv_heads, HD))
    outs = []
    if shared_cache:
        # write-all-first (dory_decode_attention.py:294-301), in token order
        for t in range(T):
            n = int(seq_lens[t])
            if n > 0:
                kv, vv, table = views[t]
                pos = n - 1
                slot = int(table[pos // B]) * B + pos % B
                _write(kv, vv, slot, B, news[t][1], news[t][2])
        for t in range(T):
            kv, vv, table = views[t]
            out = attention(news[t][0], kv, vv, table, int(seq_lens[t]), window, num_heads,
                            B, softmax_scale, second_rounding)
            outs.append(nibble_major(out * gate[t].float().cpu()))
    else:
        for t in range(T):
            kv, vv, table = views[t]
            n = int(seq_lens[t])
            if n > 0:
                pos = n - 1
                slot = int(table[pos // B]) * B + pos % B
                saved_k, saved_v = kv[slot // B, slot % B].clone(), vv[slot // B, slot % B].clone()
                _write(kv, vv, slot, B, news[t][1], news[t][2])
                out = attention(news[t][0], kv, vv, table, n, window, num_heads, B,
                                softmax_scale, second_rounding)
                kv[slot // B, slot % B], vv[slot // B, slot % B] = saved_k, saved_v
            else:
                out = torch.zeros(num_heads * HD)
            outs.append(nibble_major(out * gate[t].float().cpu()))
        for t in range(T):  # the appends land after every token has attended
            kv, vv, table = views[t]
            n = int(seq_lens[t])
            if n > 0:
                pos = n - 1
                slot = int(table[pos // B]) * B + pos % B
                _write(kv, vv, slot, B, news[t][1], news[t][2])
    return torch.stack(outs)


def split_layout(seq_len: int, window: int, block_size: int, splits: int,
                 blocks_per_tile: int) -> tuple[int, int, int, int, int]:
    """The reference's _split_layout (dory_decode_attention.py:28-44): (seq_len, first,
    first_block, tiles, tiles_per_split)."""
    first = max(seq_len - window, 0) if window > 0 else 0
    first_block = first // block_size
    num_blocks = -(-seq_len // block_size) - first_block
    tiles = -(-num_blocks // blocks_per_tile)
    return seq_len, first, first_block, tiles, max(-(-tiles // splits), 1)


# ---------------------------------------------------------------------------------------
# the multi-token q/k/v/gate epilogue (kernels/dory_multi_token.py:53-80,
# _qkvg_epilogue_kernel): the producer of multi_from_raw's inputs in the wavefront path
# ---------------------------------------------------------------------------------------

def qkvg_epilogue(partials: torch.Tensor, positions, cos_sin: torch.Tensor,
                  s_gate: torch.Tensor, s_gate_factor: float, num_heads: int,
                  num_kv_heads: int, head_dim: int):
    """Split-K GEMV partials FP32 [split_k, T, 2 * (Q + KV)] (rows: q heads, k heads,
    v heads, output gate; Q = heads * head_dim, KV = kv_heads * head_dim) ->
    (qk FP32 [T, Q + KV], v FP32 [T, KV], gate FP32 [T, Q]).

    y = 0 + p_0 + p_1 + ... in split order (:63-65).  Rows 2i and 2i + 1 of a q or k head
    hold rotary dims i and i + head_dim / 2 (:66-76): out[i] = first * cos - second * sin,
    out[i + half] = second * cos + first * sin, cos = cos_sin[position, i], sin =
    cos_sin[position, half + i] as FP32; every product and sum rounded on its own (FP32,
    no fused multiply-add).  v = y (:77-78); gate = sigmoid(y * s * s) with s =
    float(s_gate) * s_gate_factor (:79-82)."""
    p = np.asarray(partials, dtype=np.float32)
    split_k, T, rows = p.shape
    Q, KV, HD = num_heads * head_dim, num_kv_heads * head_dim, head_dim
    if rows != 2 * (Q + KV):
        raise ValueError("partials rows must be 2 * (Q + KV)")
    y = np.zeros((T, rows), dtype=np.float32)
    for k in range(split_k):
        y = (y + p[k]).astype(np.float32)
    half = HD // 2
    cs = np.asarray(cos_sin.float() if isinstance(cos_sin, torch.Tensor) else cos_sin,
                    dtype=np.float32)
    pos = np.asarray(positions, dtype=np.int64).reshape(T)
    heads = num_heads + num_kv_heads
    pairs = y[:, :Q + KV].reshape(T, heads, half, 2)
    first, second = pairs[..., 0], pairs[..., 1]
    cos = cs[pos, :half][:, None, :]
    sin = cs[pos, half:HD][:, None, :]
    lo = ((first * cos).astype(np.float32) - (second * sin).astype(np.float32)).astype(np.float32)
    hi = ((second * cos).astype(np.float32) + (first * sin).astype(np.float32)).astype(np.float32)
    qk = np.concatenate([lo, hi], axis=-1).reshape(T, Q + KV)
    v = y[:, Q + KV:Q + 2 * KV]
    s = (np.asarray(s_gate.float() if isinstance(s_gate, torch.Tensor) else s_gate,
                    dtype=np.float32) * np.float32(s_gate_factor)).astype(np.float32)
    z = ((y[:, Q + 2 * KV:] * s).astype(np.float32) * s).astype(np.float32)
    gate = torch.sigmoid(torch.from_numpy(z)).numpy()
    return torch.from_numpy(qk.copy()), torch.from_numpy(v.copy()), torch.from_numpy(gate)


# ---------------------------------------------------------------------------------------
# the residual update after a sublayer's output GEMV (dory_multi_token.py:109-131,
# _residual_tokens_kernel; dory_common.py:55-81, residual_update): the consumer of the
# attention output and of its squared norm
# ---------------------------------------------------------------------------------------

def _inv_norm_of_sum(s32: np.ndarray, eps: float) -> np.ndarray:
    """Correctly rounded FP32 1/sqrt(s + eps) of FP32 sums s (eps added in FP32)."""
    t = (np.asarray(s32, dtype=np.float32) + np.float32(eps)).astype(np.float32)
    return (1.0 / np.sqrt(t.astype(np.float64))).astype(np.float32)


def residual_tokens(partials, x, x_sumsq, a, alpha, alpha_scale: float, eps: float = EPS):
    """Split-K partials FP32 [split_k, T, H] of the output GEMV W x (x unnormalised), the
    GEMV input x FP32 [T, K] or its sum of squares x_sumsq FP32 [T] (or neither: the
    partials are already b, as residual_update's b), the sublayer input a [T, H] and the
    per-dimension alpha [H] -> (h FP32 [T, H], h BF16 [T, H], h nibble-major FP32 [T, 8, H / 8]).

    b = (0 + p_0 + ... + p_{k-1}) * r_x in split order (:121-124), r_x = 1/sqrt(sum x^2 + eps)
    (:118-119); lr = |alpha * alpha_scale| (:126); h = n(n(a) + lr * (n(b) - n(a))) (:127-130)
    with n(y) = y * 1/sqrt(sum y^2 + eps).  Sums of squares in FP64, rounded once to FP32,
    inverse square roots correctly rounded, every product and sum rounded on its own (no
    fused multiply-add); h is stored as BF16 (round to nearest even) and as FP32 in the
    nibble-major order out[j][w] = h[8w + j] (dory_common.py:46-52)."""
    p = np.asarray(partials, dtype=np.float32)
    split_k, T, H = p.shape
    if H % 8:
        raise ValueError("hidden size must be a multiple of 8")
    if x is not None and x_sumsq is not None:
        raise ValueError("give x or x_sumsq, not both")
    y = np.zeros((T, H), dtype=np.float32)
    for k in range(split_k):
        y = (y + p[k]).astype(np.float32)
    if x is not None:
        xs = np.asarray(x, dtype=np.float32).reshape(T, -1)
        r_x = inv_norm(xs, eps)
    elif x_sumsq is not None:
        r_x = _inv_norm_of_sum(np.asarray(x_sumsq, dtype=np.float32).reshape(T), eps)
    else:
        r_x = np.ones(T, dtype=np.float32)
    b = (y * r_x[:, None]).astype(np.float32)
    av = np.asarray(a.float() if isinstance(a, torch.Tensor) else a, dtype=np.float32).reshape(T, H)
    al = np.asarray(alpha.float() if isinstance(alpha, torch.Tensor) else alpha,
                    dtype=np.float32).reshape(H)
    lr = np.abs((al * np.float32(alpha_scale)).astype(np.float32))
    ya, yb = normalize(av, eps), normalize(b, eps)
    z = (ya + (lr * (yb - ya).astype(np.float32)).astype(np.float32)).astype(np.float32)
    h = normalize(z, eps)
    h_t = torch.from_numpy(h.copy())
    return h_t, h_t.to(torch.bfloat16), h_t.reshape(T, H // 8, 8).transpose(1, 2).contiguous()


# ---------------------------------------------------------------------------------------
# FP8 (e4m3) KV cache (no counterpart in the reference, whose caches are bf16; the format
# of vLLM's "fp8" kv_cache_dtype: e4m3 bytes with per-layer scales).  Stored value
# e4m3(x / scale), round to nearest even, saturating at +-448; read back as e4m3 * scale.
# The appended k and v are the reference's bf16 rows (raw_qkv) quantised this way, and the
# attention reads every cache row, the new one included, dequantised.
# ---------------------------------------------------------------------------------------

E4M3_MAX = 448.0


def e4m3_quantize(x: torch.Tensor, scale: float) -> torch.Tensor:
    """FP32 (or bf16) values -> e4m3 bytes (uint8) of x / scale (FP32 division), rounded to
    nearest even with saturation at +-448."""
    return (x.float() / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(
        torch.uint8)


def e4m3_dequantize(b: torch.Tensor, scale: float) -> torch.Tensor:
    """e4m3 bytes (uint8) -> FP32 values times scale."""
    return b.view(torch.float8_e4m3fn).float() * scale


def call_fp8(q, key8, value8, block_table, seq_len: int, window: int, softmax_scale: float,
             gate, num_heads: int, k_scale: float, v_scale: float) -> torch.Tensor:
    """DecodeAttention.__call__ over e4m3 caches [blocks, B, NKV, HD] (uint8)."""
    return call(q, e4m3_dequantize(key8, k_scale), e4m3_dequantize(value8, v_scale),
                block_table, seq_len, window, softmax_scale, gate, num_heads)


def from_raw_fp8(qk, v, sqk, sqk_factor, eps, slot: int, key8, value8, block_table,
                 seq_len: int, window: int, softmax_scale: float, gate, num_heads: int,
                 num_kv_heads: int, k_scale: float, v_scale: float) -> torch.Tensor:
    """DecodeAttention.from_raw over e4m3 caches: the new bf16 k / v quantised with their
    scales, attended as such at position seq_len - 1 and appended at `slot` (if >= 0)."""
    HD = key8.shape[-1]
    B = key8.shape[1]
    q, k_new, v_new = raw_qkv(qk, v, sqk, sqk_factor, eps, num_heads, num_kv_heads, HD)
    k8, v8 = e4m3_quantize(k_new, k_scale), e4m3_quantize(v_new, v_scale)
    if seq_len <= 0:
        return nibble_major(torch.zeros(num_heads * HD) * gate.float().cpu())
    pos = seq_len - 1
    phys = int(block_table[pos // B])
    key = e4m3_dequantize(key8, k_scale)
    value = e4m3_dequantize(value8, v_scale)
    key[phys, pos % B] = e4m3_dequantize(k8, k_scale)
    value[phys, pos % B] = e4m3_dequantize(v8, v_scale)
    out = attention(q, key, value, block_table, seq_len, window, num_heads, B, softmax_scale)
    if slot >= 0:
        key8[slot // B, slot % B] = k8
        value8[slot // B, slot % B] = v8
    return nibble_major(out * gate.float().cpu())


def multi_from_raw_fp8(qk, v, sqk, sqk_factor, eps, cache_offsets, key8_flat, value8_flat,
                       cache_shape, cache_strides, block_tables_flat, block_table_offsets,
                       seq_lens, window: int, softmax_scale: float, gate, num_heads: int,
                       num_kv_heads: int, k_scale: float, v_scale: float,
                       shared_cache: bool = False) -> torch.Tensor:
    """DecodeAttention.multi_from_raw over e4m3 caches: multi_from_raw's semantics above
    (dory_decode_attention.py:270-305; shared caches write every token's row first,
    :294-301) with each token's new bf16 k / v quantised with the layer's scales, attended as
    those values and appended as those bytes.  key8_flat / value8_flat are the flat uint8
    storage; token t's view is as_strided(cache_shape, cache_strides, cache_offsets[t])."""
    T = qk.shape[0]
    HD = cache_shape[-1]
    B = cache_shape[1]
    keyf, valuef = e4m3_dequantize(key8_flat, k_scale), e4m3_dequantize(value8_flat, v_scale)
    views, news, slots = [], [], []
    for t in range(T):
        off = int(cache_offsets[t])
        table = block_tables_flat[int(block_table_offsets[t]):]
        views.append([x.as_strided(cache_shape, cache_strides, off)
                      for x in (keyf, valuef, key8_flat, value8_flat)] + [table])
        q, k_new, v_new = raw_qkv(qk[t], v[t], sqk, sqk_factor, eps, num_heads, num_kv_heads,
                                  HD)
        news.append((q, e4m3_quantize(k_new, k_scale), e4m3_quantize(v_new, v_scale)))
        n = int(seq_lens[t])
        slots.append(int(table[(n - 1) // B]) * B + (n - 1) % B if n > 0 else -1)

    def put(t, rows):
        kf, vf, k8, v8, _ = views[t]
        b, o = slots[t] // B, slots[t] % B
        saved = (kf[b, o].clone(), vf[b, o].clone())
        kf[b, o], vf[b, o] = rows
        return saved

    def deq(t):
        return (e4m3_dequantize(news[t][1], k_scale), e4m3_dequantize(news[t][2], v_scale))

    outs = []
    if shared_cache:
        for t in range(T):
            if slots[t] >= 0:
                put(t, deq(t))
    for t in range(T):
        kf, vf, _, _, table = views[t]
        n = int(seq_lens[t])
        if n <= 0:
            outs.append(nibble_major(torch.zeros(num_heads * HD) * gate[t].float().cpu()))
            continue
        saved = None if shared_cache else put(t, deq(t))
        out = attention(news[t][0], kf, vf, table, n, window, num_heads, B, softmax_scale)
        if saved is not None:
            put(t, saved)
        outs.append(nibble_major(out * gate[t].float().cpu()))
    for t in range(T):  # the appended bytes
        if slots[t] >= 0:
            _, _, k8, v8, _ = views[t]
            k8[slots[t] // B, slots[t] % B] = news[t][1]
            v8[slots[t] // B, slots[t] % B] = news[t][2]
    return torch.stack(outs)


def relative_error(x: torch.Tensor, reference: torch.Tensor) -> float:
    """Relative L2 error (kernels/bench_mlp.py:120-121)."""
    x, reference = x.float().flatten(), reference.float().flatten()
    denom = reference.norm().item()
    return (x - reference).norm().item() / (denom if denom > 0 else 1.0)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
