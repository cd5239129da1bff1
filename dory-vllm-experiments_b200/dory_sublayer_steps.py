"""The steps around DecodeAttention in the reference's attention sublayers, on the B200
library, under the reference kernels' own names and launch forms.

* The separate q/k normalisation step of the single-token sublayer
  (kernels/dory_attention.py, `_qk_norm_cache_kernel`): it produces the normalised bf16
  query that DecodeAttention.__call__ takes and writes the token's k and v into the paged
  cache (pre_attention, dory_attention.py:218-236) or returns them in bf16
  (pre_attention_qkv, :238-250).
  - `qk_norm_cache(...)`: the step for one token or a batch of tokens;
  - `_qk_norm_cache_kernel[(NH + NKV,)](qk, v, sqk, q_out, key_cache, value_cache,
    slot_mapping, k_out, v_out, sqk_factor, eps, stride_block, stride_offset, stride_head,
    NUM_Q_HEADS=NH, HEAD_DIM=HD, CACHE_BLOCK=B, WRITE_CACHE=True, num_warps=2)`: the
    reference kernel's launch form (dory_attention.py:69-96, launched at :231-236,
    :244-249 and bench_decode_attention.py:146-150).
  The arithmetic is the fused raw-mode kernel's: q_out = bf16((sqk * sqk_factor)^2 * q *
  rsqrt(sum q^2 + eps)), k = bf16(k * rsqrt(sum k^2 + eps)), v = bf16(v), the sum of
  squares accumulated in FP64 and the inverse square root correctly rounded, so the
  separate path and DecodeAttention.from_raw append the same bits.
* The q/k/v/gate epilogue of the multi-token sublayer (kernels/dory_multi_token.py:53-80,
  `_qkvg_epilogue_kernel`), run between its q/k/v/gate GEMV and multi_from_raw (:196-205):
  - `qkvg_epilogue(...)`: split-K sum, rotary embedding, sigmoid output gate;
  - `_qkvg_epilogue_kernel[(rows // HEAD_DIM, T)](partials, positions, cos_sin, s_gate,
    qk, v, gate, s_gate_factor, Q_ROWS=, KV_ROWS=, HEAD_DIM=, SPLIT_K=, T=, num_warps=4)`.
  Its outputs are the inputs of DecodeAttention.multi_from_raw.
* The residual update after a sublayer's output GEMV, the consumer of the attention output
  (kernels/dory_multi_token.py:109-131, `_residual_tokens_kernel`, launched by
  MultiTokenSublayers._residual after the attention output GEMV and the MLP down GEMV,
  :173-181; kernels/dory_common.py:55-81, `residual_update`, the single-token form):
  - `residual_tokens(...)`: b = (sum of the split-K partials) / |x|, h = n(n(a) +
    |alpha * alpha_scale| * (n(b) - n(a))), stored as BF16 and nibble-major FP32; |x| from
    x itself or from x_sumsq, the out_sumsq of the attention call, so the attention output
    is not read again;
  - `_residual_tokens_kernel[(T,)](partials, x, a, alpha, h_out, h_out_nm, alpha_scale, eps,
    H=, K_IN=, SPLIT_K=, T=, W_BLOCK=, X_BLOCK=, num_warps=8)`;
  - `residual_update(a, b, alpha, alpha_scale, h_out, h_out_nibble_major, num_warps=4)`.
* `route_reference_kernels()`: points the reference modules' own kernel names
  (dory_attention._qk_norm_cache_kernel, dory_multi_token._qkvg_epilogue_kernel,
  dory_multi_token._residual_tokens_kernel, and residual_update in dory_common,
  dory_attention and dory_mlp) at these steps, so the reference's sublayers (whose GEMVs
  are not part of this build) run them.

This module has its own name: putting this directory ahead of the reference's kernels/ on
sys.path replaces dory_decode_attention only, and the reference's dory_attention and
dory_multi_token stay importable.
"""

from __future__ import annotations

import ctypes

import torch

import _native
from dory_decode_attention import _SQK_DTYPES, EPS


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
    _native.check_devices(qk.device, v, sqk, q_out, key_cache, value_cache, slot_mapping,
                          k_out, v_out, error_word)
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


def qkvg_epilogue(partials: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                  s_gate: torch.Tensor, s_gate_factor: float, qk: torch.Tensor,
                  v: torch.Tensor, gate: torch.Tensor, num_heads: int, num_kv_heads: int,
                  head_dim: int, error_word: torch.Tensor | None = None,
                  overlap_launch: bool = False) -> None:
    """The multi-token path's q/k/v/gate epilogue: partials FP32 [split_k, T, 2 * (Q + KV)]
    (rows: q heads, k heads, v heads, output gate; rows 2i and 2i + 1 of a q or k head are
    rotary dims i and i + head_dim / 2) -> qk FP32 [T, Q + KV] (rotary embedding at
    positions[t] from cos_sin [max_position, head_dim]), v FP32 [T, KV] and gate FP32
    [T, Q] = sigmoid(y * s * s), s = s_gate * s_gate_factor.  error_word: optional int32
    device tensor that collects DORY_DEVERR_POSITION_OOB.  overlap_launch: launch as a
    programmatic dependent of the previous kernel (its partials are read after it
    completes); either way an attention call made with overlap_launch may start while this
    kernel runs, its reads of qk / v / gate waiting for it.  Enqueued on the current
    stream."""
    Q, KV = num_heads * head_dim, num_kv_heads * head_dim
    if (partials.dtype != torch.float32 or partials.dim() != 3 or partials.shape[2] != 2 * (Q + KV)
            or not partials.is_contiguous()):
        raise ValueError("partials must be contiguous float32 [split_k, T, 2 * (Q + KV)]")
    if not partials.is_cuda:
        raise RuntimeError("qkvg_epilogue runs on CUDA tensors only (no CPU path)")
    _native.check_devices(partials.device, positions, cos_sin, s_gate, qk, v, gate, error_word)
    tokens = partials.shape[1]
    if positions.dtype not in (torch.int64, torch.int32) or positions.numel() != tokens:
        raise ValueError("positions must be int64 or int32 with one entry per token")
    for name, t, n in (("qk", qk, tokens * (Q + KV)), ("v", v, tokens * KV),
                       ("gate", gate, tokens * Q)):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != n:
            raise ValueError(f"{name} must be contiguous float32 with {n} elements")
    if cos_sin.dim() != 2 or cos_sin.shape[1] != head_dim or cos_sin.dtype not in _SQK_DTYPES:
        raise ValueError("cos_sin must be [max_position, head_dim]")
    if s_gate.dtype not in _SQK_DTYPES or s_gate.numel() != Q:
        raise ValueError("s_gate must have num_heads * head_dim entries")
    p = _native.DoryQkvgParams()
    p.partials, p.positions = partials.data_ptr(), positions.data_ptr()
    p.cos_sin, p.s_gate = cos_sin.contiguous().data_ptr(), s_gate.contiguous().data_ptr()
    p.qk_out, p.v_out, p.gate_out = qk.data_ptr(), v.data_ptr(), gate.data_ptr()
    p.error_word = _ptr(error_word)
    p.s_gate_factor = float(s_gate_factor)
    p.num_tokens, p.num_heads, p.num_kv_heads, p.head_dim = tokens, num_heads, num_kv_heads, head_dim
    p.split_k, p.max_position = partials.shape[0], cos_sin.shape[0]
    p.positions_dtype = 0 if positions.dtype == torch.int64 else 1
    p.cos_sin_dtype, p.s_gate_dtype = _SQK_DTYPES[cos_sin.dtype], _SQK_DTYPES[s_gate.dtype]
    p.flags = _native.FLAG_OVERLAP_LAUNCH if overlap_launch else 0
    stream = torch.cuda.current_stream(partials.device).cuda_stream
    _native.check(_native.load().dory_qkvg_epilogue(ctypes.byref(p), ctypes.c_void_p(stream)))


class _QkvgEpilogueLaunch:
    """`_qkvg_epilogue_kernel[grid](...)`: the reference Triton kernel's launch form
    (kernels/dory_multi_token.py:53-58, launched at :199-202).  grid = (rows / HEAD_DIM, T);
    partials is viewed as [SPLIT_K, T, rows]."""

    def __getitem__(self, grid):
        def launch(partials_ptr, positions_ptr, cos_sin_ptr, s_gate_ptr, qk_ptr, v_ptr,
                   gate_ptr, s_gate_factor, *, Q_ROWS, KV_ROWS, HEAD_DIM, SPLIT_K, T,
                   num_warps=None, num_stages=None):
            rows = 2 * (Q_ROWS + KV_ROWS)
            blocks = grid[0] if isinstance(grid, (tuple, list)) else int(grid)
            if blocks * HEAD_DIM != rows:
                raise ValueError("grid must be (2 * (Q_ROWS + KV_ROWS) / HEAD_DIM, T)")
            qkvg_epilogue(partials_ptr.view(SPLIT_K, T, rows), positions_ptr[:T], cos_sin_ptr,
                          s_gate_ptr, s_gate_factor, qk_ptr, v_ptr, gate_ptr,
                          Q_ROWS // HEAD_DIM, KV_ROWS // HEAD_DIM, HEAD_DIM)

        return launch


_qkvg_epilogue_kernel = _QkvgEpilogueLaunch()


def residual_tokens(partials: torch.Tensor, x: torch.Tensor | None, a: torch.Tensor,
                    alpha: torch.Tensor, alpha_scale: float, eps: float, h_out: torch.Tensor,
                    h_out_nm: torch.Tensor, x_sumsq: torch.Tensor | None = None,
                    overlap_launch: bool = False) -> None:
    """The residual update of T tokens after an output GEMV.  partials FP32 [split_k, T, H]
    (the GEMV of the unnormalised input), x FP32 [T, K] (the GEMV input, any layout per
    token) or x_sumsq FP32 [T] (its sum of squares, e.g. DecodeAttention's out_sumsq) or
    neither (the partials are b already), a [T, H] the sublayer input (BF16 / FP16 / FP32),
    alpha [H] -> h_out BF16 [T, H] and h_out_nm FP32 [T, 8, H / 8] (nibble-major).
    h_out / h_out_nm must not alias a or the partials (ValueError).  overlap_launch: launch
    as a programmatic dependent of the previous kernel.  Enqueued on the current stream."""
    if partials.dtype != torch.float32 or partials.dim() != 3 or not partials.is_contiguous():
        raise ValueError("partials must be contiguous float32 [split_k, T, H]")
    if not partials.is_cuda:
        raise RuntimeError("residual_tokens runs on CUDA tensors only (no CPU path)")
    _native.check_devices(partials.device, x, a, alpha, h_out, h_out_nm, x_sumsq)
    split_k, tokens, hidden = partials.shape
    if x is not None and x_sumsq is not None:
        raise ValueError("give x or x_sumsq, not both")
    if x is not None and (x.dtype != torch.float32 or not x.is_contiguous()
                          or (tokens and (x.numel() % tokens or x.numel() == 0))):
        raise ValueError("x must be contiguous float32 with the same length for every token")
    if x_sumsq is not None and (x_sumsq.dtype != torch.float32 or not x_sumsq.is_contiguous()
                                or x_sumsq.numel() < tokens):
        raise ValueError("x_sumsq must be contiguous float32 with one entry per token")
    if a.dtype not in _SQK_DTYPES or not a.is_contiguous() or a.numel() != tokens * hidden:
        raise ValueError("a must be contiguous [T, H] float32, bfloat16 or float16")
    if alpha.dtype not in _SQK_DTYPES or not alpha.is_contiguous() or alpha.numel() != hidden:
        raise ValueError("alpha must be contiguous [H]")
    if (h_out.dtype != torch.bfloat16 or not h_out.is_contiguous()
            or h_out.numel() != tokens * hidden):
        raise ValueError("h_out must be contiguous bfloat16 [T, H]")
    if (h_out_nm.dtype != torch.float32 or not h_out_nm.is_contiguous()
            or h_out_nm.numel() != tokens * hidden):
        raise ValueError("h_out_nm must be contiguous float32 [T, 8, H / 8]")
    p = _native.DoryResidualParams()
    p.partials, p.x, p.x_sumsq = partials.data_ptr(), _ptr(x), _ptr(x_sumsq)
    p.a, p.alpha = a.data_ptr(), alpha.data_ptr()
    p.h_out, p.h_out_nibble_major = h_out.data_ptr(), h_out_nm.data_ptr()
    p.alpha_scale, p.eps = float(alpha_scale), float(eps)
    p.num_tokens, p.hidden, p.split_k = tokens, hidden, split_k
    p.x_dim = x.numel() // tokens if x is not None and tokens else 0
    p.a_dtype, p.alpha_dtype = _SQK_DTYPES[a.dtype], _SQK_DTYPES[alpha.dtype]
    p.flags = _native.FLAG_OVERLAP_LAUNCH if overlap_launch else 0
    stream = torch.cuda.current_stream(partials.device).cuda_stream
    _native.check(_native.load().dory_residual_update(ctypes.byref(p), ctypes.c_void_p(stream)))


class _ResidualTokensLaunch:
    """`_residual_tokens_kernel[grid](...)`: the reference Triton kernel's launch form
    (kernels/dory_multi_token.py:109-113, launched at :177-181).  grid = (T,); partials is
    viewed as [SPLIT_K, T, H] and x as [T, K_IN]."""

    def __getitem__(self, grid):
        def launch(partials_ptr, x_ptr, a_ptr, alpha_ptr, h_ptr, h_nibble_major_ptr,
                   alpha_scale, eps, *, H, K_IN, SPLIT_K, T, W_BLOCK=None, X_BLOCK=None,
                   num_warps=None, num_stages=None):
            tokens = grid[0] if isinstance(grid, (tuple, list)) else int(grid)
            if tokens != T:
                raise ValueError("grid must be (T,)")
            residual_tokens(partials_ptr.view(SPLIT_K, T, H), x_ptr.reshape(T, K_IN),
                            a_ptr.reshape(T, H), alpha_ptr, alpha_scale, eps,
                            h_ptr.reshape(T, H), h_nibble_major_ptr.reshape(T, 8, H // 8))

        return launch


_residual_tokens_kernel = _ResidualTokensLaunch()


def residual_update(a: torch.Tensor, b: torch.Tensor, alpha: torch.Tensor, alpha_scale: float,
                    h_out: torch.Tensor, h_out_nibble_major: torch.Tensor,
                    num_warps: int = 4) -> None:
    """a: BF16 [H] sublayer input; b: FP32 [H] sublayer output; alpha: [H] -> h_out BF16
    [H] and h_out_nibble_major FP32 [8, H / 8] (kernels/dory_common.py:71-81; num_warps is
    the Triton knob, accepted and unused).  ValueError if h_out aliases a, as there."""
    if h_out.data_ptr() == a.data_ptr():
        raise ValueError("output must not alias the sublayer input")
    hidden = a.numel()
    residual_tokens(b.reshape(1, 1, hidden), None, a.reshape(1, hidden), alpha, alpha_scale,
                    EPS, h_out.reshape(1, hidden), h_out_nibble_major.reshape(1, 8, hidden // 8))


def route_reference_kernels() -> list[str]:
    """Points the reference's module-level kernels at this build's steps: the reference's
    dory_attention._qk_norm_cache_kernel (launched by FusedAttentionSublayer.pre_attention
    and pre_attention_qkv), dory_multi_token._qkvg_epilogue_kernel and
    _residual_tokens_kernel (launched by MultiTokenSublayers.attention / _residual), and
    residual_update where dory_common defines it and dory_attention / dory_mlp import it
    (the unfused residual of FusedAttentionSublayer / FusedMlpSublayer).  The reference's kernels/ must be importable (after this
    directory on sys.path).  Returns the names it replaced."""
    import importlib
    routed = []
    for module, name, step in (("dory_attention", "_qk_norm_cache_kernel", _qk_norm_cache_kernel),
                               ("dory_multi_token", "_qkvg_epilogue_kernel", _qkvg_epilogue_kernel),
                               ("dory_multi_token", "_residual_tokens_kernel",
                                _residual_tokens_kernel),
                               ("dory_common", "residual_update", residual_update),
                               ("dory_attention", "residual_update", residual_update),
                               ("dory_mlp", "residual_update", residual_update)):
        mod = importlib.import_module(module)
        if not hasattr(mod, name):
            raise ImportError(f"{module} has no {name}: is it the reference's module?")
        setattr(mod, name, step)
        routed.append(f"{module}.{name}")
    return routed


__all__ = ["qk_norm_cache", "_qk_norm_cache_kernel", "qkvg_epilogue", "_qkvg_epilogue_kernel",
           "residual_tokens", "_residual_tokens_kernel", "residual_update",
           "route_reference_kernels"]
