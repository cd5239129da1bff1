/*
 * dory_decode.h — C ABI of the B200 (sm_100a) gated decode-attention + KV-append path.
 *
 * One entry point replaces the three Triton launches of the reference's
 * DecodeAttention (kernels/dory_decode_attention.py):
 *
 *   _decode_attention_kernel  (dory_decode_attention.py:47-161)   split-KV flash decoding,
 *                                                                  q/k normalisation, K/V append
 *   _write_new_kv_kernel      (dory_decode_attention.py:164-186)  shared-cache pre-write
 *   _combine_gate_kernel      (dory_decode_attention.py:189-222)  LSE merge, gate, nibble-major store
 *
 * as launched by DecodeAttention._launch (dory_decode_attention.py:307-331) for __call__
 * (:248-256), from_raw (:258-268) and multi_from_raw (:270-305).  Everything is enqueued
 * on the caller's stream with no host synchronisation, no allocation and no host read of
 * device data, so a call can be captured in a CUDA graph.
 *
 * All pointers are device pointers.  Strides and offsets are in ELEMENTS of the pointed-to
 * type, as in the reference (torch strides, int64 cache/table offsets).  No function
 * throws; every function returns a DoryStatus, and dory_decode_last_error() gives a
 * human-readable reason for the last non-OK status on the calling thread.
 */
#ifndef DORY_DECODE_H_
#define DORY_DECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DORY_DECODE_ABI_VERSION 8

/* Status codes returned by every entry point. */
typedef enum DoryStatus {
  DORY_OK = 0,
  DORY_ERR_INVALID_ARGUMENT = 1, /* shapes / counts the reference rejects with ValueError */
  DORY_ERR_UNSUPPORTED = 2,      /* a valid configuration this build has no kernel for  */
  DORY_ERR_ALIGNMENT = 3,        /* pointers / strides not 16-byte aligned               */
  DORY_ERR_CUDA = 4              /* a CUDA runtime call failed                           */
} DoryStatus;

/* Element type of the per-dimension query scale `sqk` (the checkpoint's dtype). */
typedef enum DoryDType {
  DORY_DTYPE_F32 = 0,
  DORY_DTYPE_BF16 = 1,
  DORY_DTYPE_F16 = 2,
  DORY_DTYPE_FP8_E4M3 = 3 /* DoryDecodeParams.kv_dtype only */
} DoryDType;

/* Call kinds (bit flags of DoryDecodeParams.flags). */
enum {
  /* q holds FP32 rotated, unnormalised q heads then k heads, v holds FP32 v, and the
   * kernel normalises q and k and appends k/v (reference RAW_QKV, from_raw). */
  DORY_FLAG_RAW_QKV = 1u,
  /* num_tokens query tokens, each with its own seq_len, cache_offsets[t] and
   * block_table_offsets[t]; the slot comes from the token's block table at
   * seq_len - 1 (reference MULTI_TOKEN, multi_from_raw). */
  DORY_FLAG_MULTI_TOKEN = 2u,
  /* Tokens of one call share one cache and read each other's new entries
   * (reference shared_cache=True: write-all-first semantics). */
  DORY_FLAG_SHARED_CACHE = 4u,
  /* Launch as a programmatic dependent of the previous kernel on the stream: the next
   * call's prologue and K/V loads overlap the end of this one.  Contract: the kernel
   * immediately before this call on the stream must not write this call's seq_lens, block
   * tables, offsets, slot_mapping or the cache rows it attends (q/k/v/gate and all outputs
   * are ordered as usual).  No counterpart in the reference (Triton launches). */
  DORY_FLAG_OVERLAP_LAUNCH = 8u,
  /* Score and P.V dot products on the CUDA cores (FP32 FMA) instead of mma.sync tensor-core
   * tiles; everything else (ring, normalisation, append, merge, outputs) is the same kernel.
   * The measured alternative that decides where the tensor-core tiles pay; head_dim 128, at
   * most 4 query heads per KV head, no SHARED_CACHE (DORY_ERR_UNSUPPORTED otherwise).  No
   * counterpart in the reference (its Triton kernel always uses tl.dot). */
  DORY_FLAG_FMA_CONSUMER = 16u
};

/* Device error bits, accumulated in the scratch header and read back with
 * dory_decode_fetch_errors(). The kernel skips the offending access instead of faulting. */
enum {
  DORY_DEVERR_BLOCK_OOB = 1u,     /* a block-table entry outside [0, num_cache_blocks)   */
  DORY_DEVERR_SLOT_OOB = 2u,      /* an append slot outside the cache                     */
  DORY_DEVERR_OFFSET_ALIGN = 4u,  /* a cache offset not a multiple of 8 elements          */
  DORY_DEVERR_WAIT_TIMEOUT = 8u,  /* a pipeline wait gave up after its iteration limit    */
  DORY_DEVERR_POSITION_OOB = 16u  /* dory_qkvg_epilogue: a rotary position outside
                                   * [0, max_position); that token's q and k are zero      */
};

/*
 * Parameters of one decode-attention call.  Shapes use NH = num_heads, NKV = num_kv_heads,
 * HD = head_dim, Q = NH * HD, T = num_tokens.
 */
typedef struct DoryDecodeParams {
  /* RAW_QKV: FP32 [T, (NH + NKV) * HD] (q heads, then k heads, RoPE applied).
   * otherwise: BF16 [T, NH * HD], already normalised and scaled by (sqk * sqk_factor)^2. */
  const void* q;
  const float* v;                 /* RAW_QKV: FP32 [T, NKV * HD]                          */
  const void* sqk;                /* RAW_QKV: [NH * HD] of sqk_dtype                        */
  const int64_t* slot_mapping;    /* RAW_QKV single-token: int64 [1]; < 0 = padding, no write.
                                   * RAW_QKV | MULTI_TOKEN: optional int64 [T] (NULL: each
                                   * token's slot is its block table's at seq_len - 1); token t
                                   * appends at slot_mapping[t], < 0 = no write (vLLM's
                                   * slot_mapping, padded rows -1).  No counterpart in the
                                   * reference's multi_from_raw.                              */
  void* key_cache;                /* BF16 view [num_cache_blocks, block_size, NKV, HD]      */
  void* value_cache;              /* same strides as key_cache, unit last stride            */
  const int32_t* block_table;     /* int32; the sequence's row (single) or the table base   */
  const int64_t* block_table_offsets; /* MULTI_TOKEN: int64 [T] element offsets, else NULL */
  const int64_t* cache_offsets;   /* MULTI_TOKEN: int64 [T] element offsets, else NULL      */
  const int32_t* seq_lens;        /* int32 [T]: tokens including this one (0 = padding)     */
  const float* gate;              /* FP32 [T, Q], post-sigmoid output gate                  */
  float* out_nibble_major;        /* FP32 [T, 8, Q / 8]: out[t][e % 8][e / 8] = gated attn[e] */
  float* out_sumsq;               /* optional FP32 [T] (NULL: not computed): sum over e of
                                   * out[t][e]^2, the statistic the consumer's output GEMV
                                   * normalises by (justnorm of the gated output,
                                   * dory_attention.py:114-117 reads all of x for it); summed
                                   * in a fixed order, so repeated calls agree to the bit   */
  void* scratch;                  /* dory_decode_scratch_bytes() bytes, zeroed once by
                                   * dory_decode_scratch_init(); partials, merge counters and
                                   * the device error word live here                         */
  int64_t scratch_bytes;
  int64_t stride_block;           /* key_cache.stride(0) */
  int64_t stride_offset;          /* key_cache.stride(1) */
  int64_t stride_head;            /* key_cache.stride(2) */
  int64_t num_cache_blocks;       /* key_cache.shape[0]; > 0 enables block / slot bounds checks */
  float softmax_scale;
  float sqk_factor;
  float eps;
  int32_t num_tokens;             /* T (1 for the single-token calls)                        */
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;               /* 64, 128 or 256                                         */
  int32_t block_size;             /* key_cache.shape[1]; a multiple of 16                   */
  int32_t window;                 /* 0: full attention; > 0: keys [seq_len - window, seq_len) */
  int32_t splits;                 /* split-KV partitions per (token, KV head)               */
  int32_t blocks_per_tile;        /* split granularity in cache blocks (reference knob)      */
  int32_t min_blocks_per_split;   /* lower bound on cache blocks per active split (>= 1)     */
  int32_t max_tokens;             /* scratch capacity in tokens                             */
  int32_t sqk_dtype;              /* DoryDType                                               */
  uint32_t flags;                 /* DORY_FLAG_*                                             */
  int32_t prefetch_chunks;        /* L2 prefetch distance, in 16-row chunks, ahead of the
                                   * shared-memory ring of each CTA: 0 = automatic (the whole
                                   * range for an OVERLAP_LAUNCH call whose grid runs in one
                                   * wave, else none), < 0 = none, > 0 = that many chunks    */
  int32_t kv_dtype;               /* cache element type: 0 or DORY_DTYPE_BF16 (bf16), or
                                   * DORY_DTYPE_FP8_E4M3: key_cache / value_cache hold e4m3
                                   * bytes (strides in bytes, multiples of 16), K = e4m3 *
                                   * k_scale and V = e4m3 * v_scale, and a raw call appends
                                   * e4m3(bf16(k) / k_scale) and e4m3(bf16(v) / v_scale),
                                   * rounded to nearest even and saturated at +-448, the
                                   * values it attends (SHARED_CACHE included).  128/256-dim
                                   * heads, at most 8 query heads per KV head,
                                   * num_cache_blocks > 0.
                                   * No counterpart in the reference (its caches are bf16;
                                   * vLLM's "fp8" kv_cache_dtype).                           */
  float k_scale;                  /* FP8 caches: positive, finite                           */
  float v_scale;
} DoryDecodeParams;

/* ABI version of the loaded library (DORY_DECODE_ABI_VERSION). */
int32_t dory_decode_abi_version(void);

/* sizeof(DoryDecodeParams) as compiled into the library, so a foreign-function binding
 * (ctypes, cgo, JNI) can check its own struct layout before the first call. */
int64_t dory_decode_params_bytes(void);

/* Bytes of scratch one DecodeAttention instance needs (partials, counters, error word).
 * Mirrors the buffers DecodeAttention.__init__ allocates (dory_decode_attention.py:242-246). */
int64_t dory_decode_scratch_bytes(int32_t max_tokens, int32_t splits, int32_t num_heads,
                                  int32_t num_kv_heads, int32_t head_dim);

/* Zeroes the scratch (merge counters and error word) on `stream` (a cudaStream_t). */
int32_t dory_decode_scratch_init(void* scratch, int64_t scratch_bytes, void* stream);

/*
 * Gated decode attention with optional q/k normalisation and K/V append, on `stream`.
 * Single token (flags without MULTI_TOKEN): DecodeAttention.__call__ / from_raw
 *   (dory_decode_attention.py:248-268).
 * MULTI_TOKEN (| SHARED_CACHE): DecodeAttention.multi_from_raw
 *   (dory_decode_attention.py:270-305), including the shared-cache write-all-first order
 *   of _write_new_kv_kernel (:164-186), done inside the same kernel.
 * Host-side argument errors return DORY_ERR_INVALID_ARGUMENT with the reference's
 * ValueError conditions (:235-236, :291-293, :310-311).
 */
int32_t dory_decode_attention(const DoryDecodeParams* params, void* stream);

/*
 * dory_decode_attention without caller-owned scratch, for callers that cannot allocate
 * device memory: serving engines that hand the whole device to their own KV-cache
 * allocator up front (nothing is left for a second allocator, and freeing would fragment
 * theirs), foreign-function hosts (C, Go, Java) that have no device allocator of their own,
 * and programs whose policy forbids device allocation after start-up.  No counterpart in
 * the reference.
 *
 * Takes the same parameters; `scratch` and `scratch_bytes` are ignored.  The split partials,
 * merge counters and error word live instead in one statically sized device array inside
 * this library (DORY_DECODE_STATIC_SCRATCH_BYTES = 4 MiB), which every GPU that loads the
 * library holds until the process exits.  A call whose layout needs more scratch than that
 * (max_tokens * splits * num_heads * head_dim * 4 bytes of partials, plus counters) fails
 * with DORY_ERR_INVALID_ARGUMENT, as does one whose layout arithmetic overflows.  Allocates
 * nothing: no cudaMalloc, no cudaFree.
 *
 * The array's device address is looked up (cudaGetSymbolAddress) by the first call in each
 * CUDA context: the device's primary context (the runtime's), or a context a driver-API
 * host made current itself.  Every call clears the merge counters on `stream` before its kernel; the device
 * error word is kept and gathers the DORY_DEVERR_* bits of every call until
 * dory_decode_static_scratch_fetch_errors reads it.  All calls share the one array and it
 * keeps the last call's contents, so calls that can overlap on the GPU (different streams,
 * without ordering between them) race.
 */
#define DORY_DECODE_STATIC_SCRATCH_BYTES (4ll << 20)
int32_t dory_decode_attention_static_scratch(const DoryDecodeParams* params, void* stream);

/* The device error word of dory_decode_attention_static_scratch (DORY_DEVERR_* bits of every
 * call in the current context since the last clear) into *flags_out, synchronising `stream`;
 * clears it when `clear` is non-zero.  No counterpart in the reference. */
int32_t dory_decode_static_scratch_fetch_errors(uint32_t* flags_out, int32_t clear, void* stream);

/*
 * The separate q/k normalisation step of the reference's attention sublayer:
 * _qk_norm_cache_kernel (kernels/dory_attention.py:69-96) as FusedAttentionSublayer launches
 * it in pre_attention (WRITE_CACHE, dory_attention.py:218-236) and pre_attention_qkv
 * (dory_attention.py:238-250), for num_tokens tokens (the reference launches one):
 *   q_out[t][h] = bf16((float(sqk[h]) * sqk_factor)^2 * q[t][h] * rsqrt(sum q[t][h]^2 + eps))
 *   k[t][g]     = bf16(k[t][g] * rsqrt(sum k[t][g]^2 + eps)),   v[t][g] = bf16(v[t][g])
 * with k and v written into the paged cache at slot_mapping[t] (DORY_QKNORM_WRITE_CACHE; a
 * negative slot is a padding token and writes nothing) or to k_out / v_out.  q_out is the
 * query dory_decode_attention takes without DORY_FLAG_RAW_QKV (DecodeAttention.__call__),
 * and the normalisation is the one the fused RAW_QKV kernel applies, so both paths append
 * the same bits.
 */
#define DORY_QKNORM_WRITE_CACHE 1u
typedef struct DoryQkNormParams {
  const float* qk;                /* FP32 [T, (NH + NKV) * HD]: q heads then k heads          */
  const float* v;                 /* FP32 [T, NKV * HD]                                       */
  const void* sqk;                /* [NH * HD] of sqk_dtype                                   */
  void* q_out;                    /* BF16 [T, NH * HD]                                        */
  void* key_cache;                /* WRITE_CACHE: BF16 view [num_cache_blocks, block_size,
                                   * NKV, HD]                                                 */
  void* value_cache;              /* WRITE_CACHE: same strides as key_cache, unit last stride */
  const int64_t* slot_mapping;    /* WRITE_CACHE: int64 [T]                                   */
  void* k_out;                    /* otherwise: BF16 [T, NKV * HD]                            */
  void* v_out;                    /* otherwise: BF16 [T, NKV * HD]                            */
  uint32_t* error_word;           /* optional (NULL: none): DORY_DEVERR_SLOT_OOB is or-ed in
                                   * for a slot outside the cache, which is then skipped       */
  int64_t stride_block;           /* key_cache.stride(0) */
  int64_t stride_offset;          /* key_cache.stride(1) */
  int64_t stride_head;            /* key_cache.stride(2) */
  int64_t num_cache_blocks;       /* key_cache.shape[0]; > 0 enables the slot bounds check    */
  float sqk_factor;
  float eps;
  int32_t num_tokens;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;               /* 64, 128 or 256 */
  int32_t block_size;             /* key_cache.shape[1] (reference CACHE_BLOCK)               */
  int32_t sqk_dtype;              /* DoryDType */
  uint32_t flags;                 /* DORY_QKNORM_WRITE_CACHE */
} DoryQkNormParams;

/* sizeof(DoryQkNormParams) as compiled into the library. */
int64_t dory_qk_norm_params_bytes(void);

/* One launch of the q/k normalisation (and cache write) on `stream`. */
int32_t dory_qk_norm_cache(const DoryQkNormParams* params, void* stream);

/*
 * The multi-token path's q/k/v/gate epilogue as its own launch: the reference's
 * _qkvg_epilogue_kernel (kernels/dory_multi_token.py:53-80), which MultiTokenSublayers.attention
 * runs between its q/k/v/gate GEMV and multi_from_raw (:196-205).  Reads the split-K
 * partials and writes qk FP32 [T, (NH + NKV) * HD] (rotary embedding applied), v FP32
 * [T, NKV * HD] and gate FP32 [T, NH * HD] (sigmoid applied): the inputs of a raw
 * multi-token call (dory_decode_attention with RAW_QKV | MULTI_TOKEN).
 */
typedef struct DoryQkvgParams {
  const float* partials;          /* FP32 [split_k, T, 2 * (Q + NKV * HD)], 16-byte aligned */
  const void* positions;          /* [T], int64 or int32 (positions_dtype)                   */
  const void* cos_sin;            /* [max_position, HD] of cos_sin_dtype                     */
  const void* s_gate;             /* [Q] of s_gate_dtype                                     */
  float* qk_out;                  /* FP32 [T, (NH + NKV) * HD]                               */
  float* v_out;                   /* FP32 [T, NKV * HD]                                      */
  float* gate_out;                /* FP32 [T, NH * HD]                                       */
  uint32_t* error_word;           /* optional: DORY_DEVERR_POSITION_OOB                      */
  float s_gate_factor;
  int32_t num_tokens;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;               /* 64, 128 or 256 */
  int32_t split_k;
  int32_t max_position;
  int32_t positions_dtype;        /* 0: int64, 1: int32 */
  int32_t cos_sin_dtype;          /* DoryDType */
  int32_t s_gate_dtype;           /* DoryDType */
  uint32_t flags;                 /* DORY_FLAG_OVERLAP_LAUNCH: launch as a programmatic
                                   * dependent of the previous kernel on the stream (the
                                   * partials are read after it completes); the kernel lets
                                   * its own dependent (an overlapped attention call) start
                                   * at once, whose reads of qk / v / gate wait for it */
} DoryQkvgParams;

/* sizeof(DoryQkvgParams) as compiled into the library. */
int64_t dory_qkvg_params_bytes(void);

/* One launch of the epilogue on `stream`. */
int32_t dory_qkvg_epilogue(const DoryQkvgParams* params, void* stream);

/*
 * The residual update after a sublayer's output GEMV, the consumer of the attention output:
 * the reference's _residual_tokens_kernel (kernels/dory_multi_token.py:109-131), which
 * MultiTokenSublayers._residual launches after the attention output GEMV and after the MLP
 * down GEMV (:173-181, :210, :225), and residual_update (kernels/dory_common.py:55-81), the
 * single-token form with b given.  For each of T tokens:
 *
 *   b = (0 + partials[0] + ... + partials[split_k - 1]) * r_x
 *   r_x = 1 / sqrt(sum x^2 + eps)   from x, from x_sumsq, or 1 when both are NULL
 *   h = n(n(a) + |alpha * alpha_scale| * (n(b) - n(a))),   n(y) = y / sqrt(sum y^2 + eps)
 *
 * and h is stored as BF16 in natural order and as FP32 nibble-major (h_nm[t][j][w] =
 * h[t][8w + j]), the next sublayer's GEMV input.  x_sumsq is the out_sumsq an attention
 * call (dory_decode_attention) produced, so the attention output is not read a second time.
 * The outputs must not overlap a or the partials.
 */
typedef struct DoryResidualParams {
  const float* partials;          /* FP32 [split_k, T, H], 16-byte aligned                   */
  const float* x;                 /* optional FP32 [T, x_dim]: the GEMV's input              */
  const float* x_sumsq;           /* optional FP32 [T]: sum of x^2 given directly            */
  const void* a;                  /* [T, H] of a_dtype: the sublayer input, 16-byte aligned  */
  const void* alpha;              /* [H] of alpha_dtype, 16-byte aligned                     */
  void* h_out;                    /* BF16 [T, H], 16-byte aligned                            */
  float* h_out_nibble_major;      /* FP32 [T, 8, H / 8], 16-byte aligned                     */
  float alpha_scale;
  float eps;
  int32_t num_tokens;
  int32_t hidden;                 /* H: a multiple of 8, at most 16384                       */
  int32_t x_dim;                  /* K: elements of x per token                              */
  int32_t split_k;
  int32_t a_dtype;                /* DoryDType */
  int32_t alpha_dtype;            /* DoryDType */
  uint32_t flags;                 /* DORY_FLAG_OVERLAP_LAUNCH: launch as a programmatic
                                   * dependent of the previous kernel on the stream (inputs
                                   * are read after it completes) */
} DoryResidualParams;

/* sizeof(DoryResidualParams) as compiled into the library. */
int64_t dory_residual_params_bytes(void);

/* One launch of the residual update on `stream` (one CTA per token). */
int32_t dory_residual_update(const DoryResidualParams* params, void* stream);

/* Copies the device error word (DORY_DEVERR_* bits) to *flags_out, synchronising `stream`;
 * clears it when `clear` is non-zero.  The only entry point that waits on the device. */
int32_t dory_decode_fetch_errors(void* scratch, uint32_t* flags_out, int32_t clear, void* stream);

/* Reason for the last non-OK status returned on this thread ("" if none). */
const char* dory_decode_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* DORY_DECODE_H_ */
