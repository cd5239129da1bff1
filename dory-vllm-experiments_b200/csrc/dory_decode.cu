// dory_decode.cu — B200 (sm_100a) gated decode attention with in-kernel q/k normalisation
// and K/V append over vLLM's paged BF16 cache.  Implements the C ABI of include/dory_decode.h.
//
// Reference behaviour (chrisbennight/dory-vllm-experiments, kernels/dory_decode_attention.py):
//   * _split_layout (:28-44)           -> split_layout() below, on the union range of a group
//   * _decode_attention_kernel (:47-161) -> decode_kernel(): one CTA per (split, KV head,
//     token group).  RAW mode normalises q (x * rsqrt(sum x^2 + eps), scaled by (sqk*f)^2,
//     rounded to bf16, then * softmax_scale rounded to bf16 again, :110-113,123), normalises
//     the new key (:114), writes k/v at the slot from the split that owns the token's block
//     (:115-122) and uses the new k/v instead of the cache row (:141-145).
//   * _write_new_kv_kernel (:164-186)  -> shared-cache mode: every CTA substitutes the new
//     k/v of ALL tokens of the call wherever its cache rows alias their slots, so a token
//     sees the others' new entries exactly as with write-all-first, without a second launch.
//   * _combine_gate_kernel (:189-222)  -> the last CTA to finish a (token group, KV head)
//     merges the splits' partials (max / sum / acc), applies the gate and stores nibble-major
//     out[e % 8][e / 8] (the layout w4a16_gemv.py:91-93 defines).
//
// B200 design:
//   * K/V chunks (16 cache rows of one KV head, K and V) are staged into an 8-stage ring in
//     shared memory by TMA: one 5-D tensor box (64 dims x 16 rows x 64-dim quarters x head
//     x block, 128-byte swizzle) per chunk, completing on an mbarrier.  The producer warp
//     stages the CTA's block ids and issues the first ring's worth; from then on each
//     consumer warp refills the stage it has just read (stages map to fixed warps), so no
//     cross-warp hand-off sits between a stage falling free and its next copy.  Offsets that
//     are not whole cache blocks take a cp.async copy path into the same swizzled layout.
//   * Four consumer warps run each chunk through mma.sync m16n8k16 (bf16 in, fp32
//     accumulate) with tokens on M and the GQA group's query rows (plus the other tokens of a
//     shared-cache group) on N: S^T = K Q^T, then O^T += V^T P^T; P^T moves from accumulator
//     to operand layout with movmatrix; the swizzle keeps every ldmatrix conflict-free.
//   * Softmax is online, in the log2 domain, with warp-shuffle row reductions.  Chunks at the
//     attended range's edges, with a bad block id or holding a new token's row take a slow
//     path (zeroing, substitution, the append itself).
//   * Split partials go to caller-owned scratch; the last CTA of a (token group, KV head) to
//     arrive (acquire-release counter, self-resetting) merges them in registers, applies the
//     gate and stores nibble-major, so one launch does what the reference does in two or
//     three.  Opt-in programmatic dependent launch overlaps a call's prologue and K/V copies
//     with the previous kernel's tail.
//   * Every wait is bounded: on timeout the kernel records DORY_DEVERR_WAIT_TIMEOUT and
//     drains its own copies before returning.  Out-of-range block ids / slots are recorded
//     and skipped, never dereferenced.
//   * A second small kernel is the reference's separate q/k normalisation + cache write
//     (_qk_norm_cache_kernel), the input side of the non-raw call; a third is the
//     multi-token path's q/k/v/gate epilogue (_qkvg_epilogue_kernel), the input side of the
//     raw multi-token call.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdarg.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "../../include/dory_decode.h"

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kChunk = 16;                           // cache rows per pipeline stage (MMA M)
constexpr int kMaxSub = 16;                          // new tokens a CTA can substitute
constexpr int kTab = 512;                            // block ids of a CTA's range kept in smem
constexpr long long kWaitLimitCycles = 500000000LL;  // ~0.25 s at 1.9 GHz, then give up
constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------------------------
// Kernel parameters (device-side copy of DoryDecodeParams plus derived values).
// ------------------------------------------------------------------------------------
// Field order matters: the kernel reads its parameters through the constant cache, and a
// CTA that is the first on its SM pays one L2 round trip per 64-byte line it touches.  The
// scalars and pointers of the prologue come first (lines 0-1), the rest next, the tensor
// maps (read by the copy engine) last; every CTA touches all lines at once on entry.
struct alignas(64) KParams {
  // line 0: scalars of the split layout and the prologue
  int T, NH, NKV, G, B, window, S, bpt;
  int tps_min, b_shift, cpb_shift, raw, multi, shared, nsub, q_stride;
  // line 1: the first dependent loads
  const int32_t* seq_lens;
  const int64_t* cache_offsets;
  const int64_t* table_offsets;
  const int32_t* table;
  int64_t sb, so, sh, ncache_blocks;
  // lines 2-3: inputs, outputs, scratch
  const void* q;
  const float* v;
  const void* sqk;
  const int64_t* slot_mapping;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  const float* gate;
  float* out;
  float* sumsq;          // optional [T]: sum over e of out[t][e]^2 (the output's justnorm statistic)
  uint32_t* err;
  int32_t* counters;
  int32_t* tok_counters;  // [max_tokens]: KV heads whose outputs are stored (sumsq)
  float* sumsq_part;      // [max_tokens][NKV]: each KV head's share of sumsq
  float2* pml;  // [max_tokens][S][NH] (max in log2 units, sum)
  float* po;    // [max_tokens][S][NH][HD]
  int64_t tm_blocks;  // extent of the block dimension of the tensor maps
  float scale, sqk_factor, eps;
  int min_bps, sqk_dtype, overlap;
  int pf;        // L2 prefetch distance in chunks beyond the ring (0: none)
  int tm_mode;   // 0: no tensor maps; 1: tmk covers K and V (V right after K); 2: tmk, tmv
  float k_scale, v_scale;  // FP8 cache: K = e4m3 * k_scale, V = e4m3 * v_scale
  CUtensorMap tmk;  // cache views as 5-D tensors (64 dims, rows, 64-dim quarters of a row,
  CUtensorMap tmv;  // KV head, block), one box = a chunk's K (and V) tile, 128-byte swizzle
};
static_assert(offsetof(KParams, seq_lens) == 64, "line 1 starts with the dependent pointers");
static_assert(offsetof(KParams, tmk) % 64 == 0, "tensor maps are 64-byte aligned");

// Scratch layout (bytes), shared by host and device.
struct ScratchLayout {
  int64_t counters, tok_counters, sumsq_part, pml, po, total;
};
__host__ __device__ inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }
__host__ __device__ inline ScratchLayout scratch_layout(int max_tokens, int S, int NH, int NKV,
                                                        int HD) {
  ScratchLayout L;
  L.counters = 256;  // [0, 256): header; word 0 = device error flags
  L.tok_counters = align256(L.counters + int64_t(max_tokens) * NKV * 4);
  L.sumsq_part = align256(L.tok_counters + int64_t(max_tokens) * 4);
  L.pml = align256(L.sumsq_part + int64_t(max_tokens) * NKV * 4);
  L.po = align256(L.pml + int64_t(max_tokens) * S * NH * 8);
  L.total = align256(L.po + int64_t(max_tokens) * S * NH * HD * 4);
  return L;
}
// Host side: the same layout with every product and sum checked for int64 overflow (the
// counts come from the caller); false if any step overflows or a count is not positive.
inline bool scratch_layout_checked(int max_tokens, int S, int NH, int NKV, int HD,
                                   ScratchLayout* out) {
  if (max_tokens < 1 || S < 1 || NH < 1 || NKV < 1 || HD < 1) return false;
  // The largest term is the partials, max_tokens * S * NH * HD * 4 bytes; the others are
  // smaller products of the same counts.  With every term at most 2^60 the layout's sum of
  // five terms and its alignment padding stays far below 2^63.
  const int64_t kLimit = int64_t(1) << 60;
  int64_t rows, po_bytes, ctr_bytes;
  if (__builtin_mul_overflow(int64_t(max_tokens), int64_t(S), &rows) ||
      __builtin_mul_overflow(rows, int64_t(NH), &rows) ||
      __builtin_mul_overflow(rows, int64_t(HD) * 4, &po_bytes) ||
      __builtin_mul_overflow(int64_t(max_tokens), int64_t(NKV) * 4, &ctr_bytes) ||
      po_bytes > kLimit || rows * 8 > kLimit || ctr_bytes > kLimit)
    return false;
  *out = scratch_layout(max_tokens, S, NH, NKV, HD);
  return true;
}

// Dynamic shared memory layout for one instantiation.  Each ring stage holds the K tile
// and then the V tile of one 16-row chunk, each as HD / 64 boxes of [16 rows][64 dims] bf16
// in the 128-byte swizzle of the tensor copies: the 16-byte piece j of row r sits at
// r * 128 + ((j ^ (r % 8)) * 16) within its box, so ldmatrix rows never share banks.
constexpr int kBoxBytes = kChunk * 128;
__host__ __device__ constexpr uint32_t tile_off(int r, int d) {  // d: a multiple of 8
  return uint32_t((d >> 6) * kBoxBytes + r * 128 + ((((d >> 3) & 7) ^ (r & 7)) << 4));
}
// FP8 (e4m3) caches: a 16-row tile is HD / 128 boxes of [16 rows][128 dims] bytes in the same
// 128-byte swizzle; piece j (dims 16j .. 16j + 15) of row r of a box sits at
// r * 128 + ((j ^ (r % 8)) * 16).  d: a multiple of 16.
__host__ __device__ constexpr uint32_t tile_off8(int r, int d) {
  return uint32_t((d >> 7) * kBoxBytes + r * 128 + ((((d >> 4) & 7) ^ (r & 7)) << 4));
}
template <int HD, int NS, bool KV8 = false>
struct Smem {
  static constexpr int kTile16 = (HD / 64) * kBoxBytes;       // a 16-bit K (or V) tile
  static constexpr int kTileBytes = KV8 ? (HD / 128) * kBoxBytes : kTile16;  // as copied
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = 0;                           // 1024-byte aligned at run time
  static constexpr int kRegion = NS * kStageBytes;            // reused after the loop
  static constexpr int kBars = kStages + NS * kStageBytes;    // full[NS], empty[NS]
  static constexpr int kMeta = kBars + 2 * NS * 8;            // int4 {phys, -, chunk, -}
  // bf16 [16][HD]; with one 8-row tile the upper half holds the CUDA-core consumer's P
  // buffers or the 128-dim FP8 kernel's query fragments
  static constexpr int kQ = kMeta + NS * 16;
  static constexpr int kSub = kQ + 16 * HD * 2;               // bf16 [nsub][2][HD]
  static int bytes(int nsub) { return kSub + (nsub > 0 ? nsub : 1) * 2 * HD * 2 + 1024; }
};

// ------------------------------------------------------------------------------------
// PTX helpers
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false after ~kWaitLimitCycles (the caller records the timeout).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitLimitCycles) return false;
  }
  return true;
}
// K/V rows are read once per launch: mark them first to leave L2 (evict_first), so the
// small, re-read data (block tables, seq lens, q/k/v/gate rows, split partials) stays.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}
// One box of a tensor map into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, int c4, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(bar), "l"(policy)
      : "memory");
}
// One box of a tensor map into L2 only (no shared memory, no completion to wait for): the
// DRAM read of a chunk the ring has no room for yet starts now, and its later copy into
// shared memory is served from L2.
__device__ __forceinline__ void tma_prefetch_5d(const CUtensorMap* map, int c0, int c1, int c2,
                                                int c3, int c4) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
// Programmatic dependent launch: wait for the previous grid on the stream to complete (and
// its writes to be visible); allow the next grid to launch.  No-ops without the attribute.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later tensor copies.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 16-byte global->shared copy; src_bytes 0 reads nothing and zero-fills the 16 bytes.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.cg.shared.global.L2::cache_hint.L2::256B [%0], [%1], 16, %2, %3;" ::"r"(dst),
      "l"(src), "r"(src_bytes), "l"(policy)
      : "memory");
}
// The mbarrier receives one arrival when all of this thread's earlier cp.async copies landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}
// Issues L2 prefetches for `bytes` bytes at `ptr`, one 128-byte line per lane.
__device__ __forceinline__ void prefetch_range(const void* ptr, int bytes, int lane) {
  const char* c = static_cast<const char*>(ptr);
  for (int off = lane * 128; off < bytes; off += 32 * 128) prefetch_l2(c + off);
}
__device__ __forceinline__ void named_barrier_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}
// Barrier 2: the producer warp announces that the pipeline's mbarriers are initialised
// (arrive, no wait); the consumer warps wait for it before their first stage.
__device__ __forceinline__ void pipeline_ready_arrive() {
  asm volatile("bar.arrive 2, %0;" ::"n"(kThreads) : "memory");
}
__device__ __forceinline__ void pipeline_ready_wait() {
  asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a0, uint32_t& a1, uint32_t& a2,
                                        uint32_t& a3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a0, uint32_t& a1, uint32_t& a2,
                                          uint32_t& a3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Two e4m3 values (the low byte is the lower element) to f16x2: every e4m3 value is an f16.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<uint16_t>(two_bytes)));
  return r;
}
// Two FP32 values to e4m3 (round to nearest even, saturating at +-448): lo in the low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// bf16x2 (lower element in the low half) to f16x2, exact for the normal f16 range.
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x) {
  const float lo = __uint_as_float(x << 16), hi = __uint_as_float(x & 0xffff0000u);
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// P for an f16 MMA: each value rounded to bf16 first (the P.V operand precision of the
// bf16 path), then packed as f16x2 (exact for the rounded values of the normal f16 range).
__device__ __forceinline__ uint32_t pack_p_f16x2(float lo, float hi) {
  const float l = __bfloat162float(__float2bfloat16_rn(lo));
  const float h = __bfloat162float(__float2bfloat16_rn(hi));
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(h), "f"(l));
  return r;
}
// x rounded to the nearest e4m3 value (ties to even, saturating at +-448), as FP32.
__device__ __forceinline__ float e4m3_round(float x) {
  const uint32_t h2 = e4m3x2_to_f16x2(f32x2_to_e4m3x2(x, 0.0f));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffffu)));
}
// A new token's k (normalised) or v value as the kernel keeps it: bf16, or for an FP8 cache
// the e4m3 value of bf16(x) / scale (as bf16, exact), the value appended and attended.
template <bool KV8>
__device__ __forceinline__ __nv_bfloat16 new_kv(float x, float scale) {
  if constexpr (KV8)
    return __float2bfloat16_rn(e4m3_round(__bfloat162float(__float2bfloat16_rn(x)) / scale));
  else
    return __float2bfloat16_rn(x);
}
template <bool F16>
__device__ __forceinline__ void mma16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                      uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (F16) mma_f16(d, a0, a1, a2, a3, b0, b1);
  else mma_bf16(d, a0, a1, a2, a3, b0, b1);
}
// O^T += V^T P^T over one 16-row stage (256-dim heads): [16 dims x 8 rows] per m-tile (k-step
// kk) and n-tile.  Lane l gives ldmatrix the address of V row (l & 7) + 8 * (l >> 4) of its
// matrix; MASK: a lane whose row is outside the attended range (row_ok false) gives the
// address of a zeroed 16-byte row instead, so that row enters the MMA as zeros.
template <int KT, int NT, bool MASK, bool F16 = false>
__device__ __forceinline__ void pv_accumulate(float (&o)[NT][KT][4], uint32_t vbase_s, int lane,
                                              const uint32_t (&pb)[NT][2], bool row_ok,
                                              uint32_t zero_row) {
  const int vr = (lane & 7) + ((lane >> 4) << 3), vd = ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int kk = 0; kk < KT; ++kk) {
    uint32_t a0, a1, a2, a3;
    const uint32_t addr = vbase_s + tile_off(vr, kk * 16 + vd);
    ldsm_x4_t((MASK && !row_ok) ? zero_row : addr, a0, a1, a2, a3);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mma16<F16>(o[nt][kk], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
  }
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void record_error(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

// ------------------------------------------------------------------------------------
// CUDA-core (FP32 FMA) form of a consumer warp's chunk step, 128-dim heads and at most 4
// query rows: the measured alternative to the mma.sync tiles (DORY_FLAG_FMA_CONSUMER).
// Lane l owns dims [4l, 4l + 4) of every row.  Per half chunk (8 tokens) it forms its 4-dim
// share of the 8 x 4 scores with FMAs; a transposing butterfly (each of 5 steps keeps half of
// the lane's values and adds the partner's share of them, received for the half it gives
// away) then leaves lane l the complete score of row l / 8 at token l % 8 of that half.
// Softmax as the tensor-core path: log2 domain, the running sum from unrounded P, P rounded
// to bf16 for P.V, which goes through a per-warp [16 tokens][4 rows] buffer and FMAs into
// this lane's 4 dims of each row's output.
// ------------------------------------------------------------------------------------
struct FmaRows {
  float o[4][4];  // [row][this lane's 4 dims]
  float m[4];     // running max of each row (log2 units), the same in every lane
  float l;        // this lane's share of the running sum of row lane / 8
};
__device__ __forceinline__ void unpack_bf16x4(uint2 w, float (&x)[4]) {
  x[0] = __uint_as_float(w.x << 16);
  x[1] = __uint_as_float(w.x & 0xffff0000u);
  x[2] = __uint_as_float(w.y << 16);
  x[3] = __uint_as_float(w.y & 0xffff0000u);
}
__device__ __forceinline__ void fma_chunk(FmaRows& st, const float (&q)[4][4], const uint8_t* kst,
                                          const uint8_t* vst, float* pbuf, int lane, int c,
                                          int rfirst, int rlen) {
  const int d8 = 8 * (lane >> 1);     // this lane's 16-byte piece of a row ...
  const int half8 = (lane & 1) * 8;   // ... and its 8-byte half
  float x[2];                         // x[h]: score (token 8h + lane % 8, row lane / 8)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float v[32];                      // v[r * 8 + t]: this lane's share of score (8h + t, r)
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      float k[4];
      unpack_bf16x4(*reinterpret_cast<const uint2*>(kst + tile_off(8 * h + t, d8) + half8), k);
#pragma unroll
      for (int r = 0; r < 4; ++r)
        v[r * 8 + t] =
            fmaf(q[r][3], k[3], fmaf(q[r][2], k[2], fmaf(q[r][1], k[1], q[r][0] * k[0])));
    }
#pragma unroll
    for (int lev = 0; lev < 5; ++lev) {
      const int half = 16 >> lev, mask = 16 >> lev;
      const bool up = lane & mask;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? v[i] : v[i + half];
        const float keep = up ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
      }
    }
    x[h] = v[0];
  }
  const int r = lane >> 3;
  const int tk = lane & 7;
  const int pos0 = c * kChunk + tk;
  const float x0 = (pos0 >= rfirst && pos0 < rlen) ? x[0] * kLog2e : -INFINITY;
  const float x1 = (pos0 + 8 >= rfirst && pos0 + 8 < rlen) ? x[1] * kLog2e : -INFINITY;
  float tmax = fmaxf(x0, x1);
  tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
  tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
  tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
  float alpha[4], a_own = 1.0f, m_own = 0.0f;
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const float mnew = fmaxf(st.m[rr], __shfl_sync(0xffffffffu, tmax, rr * 8));
    const float muse = (mnew == -INFINITY) ? 0.0f : mnew;
    alpha[rr] = fast_exp2(st.m[rr] - muse);
    st.m[rr] = mnew;
    if (rr == r) {
      a_own = alpha[rr];
      m_own = muse;
    }
  }
  const float p0 = fast_exp2(x0 - m_own), p1 = fast_exp2(x1 - m_own);
  st.l = st.l * a_own + p0 + p1;
  pbuf[tk * 4 + r] = __bfloat162float(__float2bfloat16_rn(p0));
  pbuf[(tk + 8) * 4 + r] = __bfloat162float(__float2bfloat16_rn(p1));
  __syncwarp();
#pragma unroll
  for (int rr = 0; rr < 4; ++rr)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[rr][j] *= alpha[rr];
#pragma unroll
  for (int t = 0; t < kChunk; ++t) {
    float vv[4];
    unpack_bf16x4(*reinterpret_cast<const uint2*>(vst + tile_off(t, d8) + half8), vv);
    const float4 pp = *reinterpret_cast<const float4*>(pbuf + t * 4);
    const float pr[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
    for (int rr = 0; rr < 4; ++rr)
#pragma unroll
      for (int j = 0; j < 4; ++j) st.o[rr][j] = fmaf(pr[rr], vv[j], st.o[rr][j]);
  }
  __syncwarp();  // the buffer is rewritten by this warp's next chunk
}

__device__ __forceinline__ float load_sqk(const void* sqk, int dtype, int64_t i) {
  if (dtype == DORY_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(sqk)[i]);
  if (dtype == DORY_DTYPE_F16) return __half2float(static_cast<const __half*>(sqk)[i]);
  return static_cast<const float*>(sqk)[i];
}

// Canonical normalisation factor of one row: Sum x^2 is accumulated in FP64 (every square
// is exact there and the sum carries 29 more bits than FP32, so its FP32 rounding depends on
// the summation order only when the sum lies within ~2^-53 of an FP32 rounding boundary),
// rounded to FP32, eps is added in FP32 (as the reference's `tl.sum(x * x) + eps`) and the
// inverse square root is the correctly rounded FP32 value.  The oracle computes the same
// quantities the same way.
__device__ __forceinline__ float inv_norm_from_sum(double acc, float eps) {
  const float sum32 = __double2float_rn(acc);
  const float t = __fadd_rn(sum32, eps);
  // 1 / sqrt(t), correctly rounded to FP32: the FP32 estimate refined by two Newton-Raphson
  // steps in FP64 for f(y) = 1 / y^2 - t, y <- y (3 - t y^2) / 2 (relative error well
  // below 1e-15 afterwards), then rounded once.
  const double td = double(t);
  double y = double(rsqrtf(t));
  y = y * (1.5 - 0.5 * td * y * y);
  y = y * (1.5 - 0.5 * td * y * y);
  return __double2float_rn(y);
}
// One row spread over the 32 lanes of a warp, PER_LANE elements each.
template <int PER_LANE>
__device__ __forceinline__ float row_inv_norm(const float (&x)[PER_LANE], float eps) {
  double acc = 0.0;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) acc += double(x[i]) * double(x[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return inv_norm_from_sum(acc, eps);
}

// x / d and x % d for x >= 0, by shifting when d is a power of two (shift >= 0).
__device__ __forceinline__ int div_p2(int x, int d, int shift) {
  return shift >= 0 ? (x >> shift) : x / d;
}
__device__ __forceinline__ int mod_p2(int x, int d, int shift) {
  return shift >= 0 ? (x & (d - 1)) : x % d;
}

// Split layout of the reference (_split_layout, dory_decode_attention.py:28-44) applied to
// the attended union [lo, hi) of a token group.
struct Split {
  int first_block, nblocks, tiles, tps, active;
};
__device__ __forceinline__ Split split_layout(int lo, int hi, int B, int b_shift, int S, int bpt,
                                              int tps_min) {
  Split s;
  if (hi <= 0) {
    s.first_block = 0;
    s.nblocks = 0;
    s.tiles = 0;
    s.tps = 1;
    s.active = 0;
    return s;
  }
  s.first_block = div_p2(lo, B, b_shift);
  s.nblocks = div_p2(hi + B - 1, B, b_shift) - s.first_block;
  s.tiles = bpt == 1 ? s.nblocks : (s.nblocks + bpt - 1) / bpt;
  int tps = (s.tiles + S - 1) / S;
  if (tps < tps_min) tps = tps_min;
  if (tps < 1) tps = 1;
  s.tps = tps;
  s.active = (s.tiles + tps - 1) / tps;
  return s;
}

// ------------------------------------------------------------------------------------
// Slow path of a ring stage (taken by few chunks):
//  * tensor path, heads up to 128 dims: zero the V rows outside [lo, hi) (all of them for a
//    bad block); 256-dim heads mask those rows in the MMA instead (pv_accumulate);
//  * put the new k/v of this call's tokens into the rows that hold their slots (by
//    position for tokens on this CTA's table, by physical block otherwise), as the
//    reference uses the new token from registers (dory_decode_attention.py:141-145) and
//    its shared-cache mode caches every token first (:294-301);
//  * append: the chunk holding a group token's position writes its k/v to the cache
//    in shared-cache calls (slot_mapping[t] when given, else the table's slot); other raw
//    calls leave the new row out of the chunk loop and append it in the prologue.
// Returns whether the stage was written (the caller then fences before tensor copies).
// ------------------------------------------------------------------------------------
// CTA constants the slow path needs, kept in shared memory so that the hot loop does not
// hold them in registers.
struct CtaInfo {
  long long coff, toff;
  int lo, hi, kvh, nsub, ibase, gcount, offset_ok, tok, reg_new;
};

template <int HD>
__device__ __forceinline__ bool fixup_stage(const KParams& p, uint8_t* kst, uint8_t* vst, int c,
                                         int phys, bool zero_rows, int lane,
                                         const CtaInfo& ci, const int* s_len, const int* s_phys,
                                         const long long* s_coff, const long long* s_toff,
                                         const __nv_bfloat16* subkv) {
  const long long coff = ci.coff, toff = ci.toff;
  const int lo = ci.lo, hi = ci.hi, kvh = ci.kvh, nsub = ci.nsub, ibase = ci.ibase;
  const int gcount = ci.gcount;
  const bool offset_ok = ci.offset_ok;
  constexpr int kVec = HD / 8;  // 16-byte pieces per row
  const int B = p.B;
  const int CPB = B / kChunk;
  bool touched = false;
  if (zero_rows) {
    const int r_lo = max(lo - c * kChunk, 0), r_hi = min(hi - c * kChunk, kChunk);
    for (int idx = lane; idx < kChunk * kVec; idx += 32) {
      const int r = idx / kVec, w = idx % kVec;
      if (phys < 0 || r < r_lo || r >= r_hi)
        *reinterpret_cast<uint4*>(vst + tile_off(r, w * 8)) = make_uint4(0, 0, 0, 0);
    }
    touched = true;
  }
  if (!p.raw || ci.reg_new) return touched;  // reg_new: the new row is masked, added apart
  for (int s = 0; s < nsub; ++s) {
    const int len = s_len[s];
    if (len <= 0) continue;
    const int pos = len - 1;
    const bool same = s_coff[s] == coff && s_toff[s] == toff;
    int r = -1;
    if (same) {
      if (pos / kChunk == c) r = pos % kChunk;
    } else if (phys >= 0 && s_phys[s] == phys && s_coff[s] == coff) {
      const int rr = mod_p2(pos, B, p.b_shift) - mod_p2(c, CPB, p.cpb_shift) * kChunk;
      if (rr >= 0 && rr < kChunk) r = rr;
    }
    if (r < 0) continue;
    for (int idx = lane; idx < 2 * kVec; idx += 32) {
      const bool is_v = idx >= kVec;
      const int w = is_v ? idx - kVec : idx;
      const uint4 val = reinterpret_cast<const uint4*>(subkv + (s * 2 + (is_v ? 1 : 0)) * HD)[w];
      *reinterpret_cast<uint4*>((is_v ? vst : kst) + tile_off(r, w * 8)) = val;
    }
    touched = true;
    if (!same || s < ibase || s >= ibase + gcount) continue;  // another CTA appends it
    long long slot;
    if (p.multi && p.slot_mapping) {
      // the caller's per-token slot (vLLM's slot_mapping); negative: not cached
      slot = p.slot_mapping[p.shared ? s : ci.tok];
      if (slot < 0) continue;
    } else if (p.multi) {
      if (phys < 0) continue;  // its block id was out of range (already recorded)
      slot = (long long)phys * B + mod_p2(pos, B, p.b_shift);
    } else {
      continue;  // single-token calls append outside the chunk loop (reg_new)
    }
    const long long blk = slot / B;
    if (blk < 0 || (p.ncache_blocks > 0 && blk >= p.ncache_blocks) || !offset_ok) {
      if (lane == 0) record_error(p.err, DORY_DEVERR_SLOT_OOB);
      continue;
    }
    const long long base = s_coff[s] + blk * p.sb + (slot % B) * p.so + (long long)kvh * p.sh;
    for (int idx = lane; idx < 2 * kVec; idx += 32) {
      const bool is_v = idx >= kVec;
      const int w = is_v ? idx - kVec : idx;
      const uint4 val = reinterpret_cast<const uint4*>(subkv + (s * 2 + (is_v ? 1 : 0)) * HD)[w];
      reinterpret_cast<uint4*>((is_v ? p.vc : p.kc) + base)[w] = val;
    }
  }
  return touched;
}

// The e4m3 bytes of 16 dims of a new row (exact e4m3 values held as bf16), dim 0 in byte 0.
__device__ __forceinline__ uint4 e4m3x16(const __nv_bfloat16* src) {
  uint32_t b[8];
#pragma unroll
  for (int e = 0; e < 8; ++e)
    b[e] = f32x2_to_e4m3x2(__bfloat162float(src[2 * e]), __bfloat162float(src[2 * e + 1]));
  return make_uint4(b[0] | (b[1] << 16), b[2] | (b[3] << 16), b[4] | (b[5] << 16),
                    b[6] | (b[7] << 16));
}

// FP8 shared caches: a stage that holds a sub token's new row gets the row's e4m3 bytes (the
// write-all-first order, as fixup_stage does for bf16 stages), and the rows of this CTA's
// own group tokens are appended to the cache here.  Rows outside the attended range and bad
// blocks need no zeroing: the consumer masks them.
template <int HD>
__device__ __forceinline__ void fixup_stage8(const KParams& p, uint8_t* kst, uint8_t* vst, int c,
                                             int phys, int lane, const CtaInfo& ci,
                                             const int* s_len, const int* s_phys,
                                             const long long* s_coff, const long long* s_toff,
                                             const __nv_bfloat16* subkv) {
  constexpr int kVec8 = HD / 16;  // 16-byte pieces per e4m3 row
  const int B = p.B;
  const int CPB = B / kChunk;
  for (int s = 0; s < ci.nsub; ++s) {
    const int len = s_len[s];
    if (len <= 0) continue;
    const int pos = len - 1;
    const bool same = s_coff[s] == ci.coff && s_toff[s] == ci.toff;
    int r = -1;
    if (same) {
      if (pos / kChunk == c) r = pos % kChunk;
    } else if (phys >= 0 && s_phys[s] == phys && s_coff[s] == ci.coff) {
      const int rr = mod_p2(pos, B, p.b_shift) - mod_p2(c, CPB, p.cpb_shift) * kChunk;
      if (rr >= 0 && rr < kChunk) r = rr;
    }
    if (r < 0) continue;
    long long base = -1;  // the cache row this CTA appends, if any
    if (same && s >= ci.ibase && s < ci.ibase + ci.gcount) {
      long long slot = -1;
      if (p.slot_mapping) slot = p.slot_mapping[s];  // negative: not cached
      else if (phys >= 0) slot = (long long)phys * B + mod_p2(pos, B, p.b_shift);
      if (slot >= 0) {
        const long long blk = slot / B;
        if ((p.ncache_blocks > 0 && blk >= p.ncache_blocks) || !ci.offset_ok) {
          if (lane == 0) record_error(p.err, DORY_DEVERR_SLOT_OOB);
        } else {
          base = s_coff[s] + blk * p.sb + (slot % B) * p.so + (long long)ci.kvh * p.sh;
        }
      }
    }
    for (int idx = lane; idx < 2 * kVec8; idx += 32) {
      const bool is_v = idx >= kVec8;
      const int w = is_v ? idx - kVec8 : idx;
      const uint4 val = e4m3x16(subkv + (s * 2 + (is_v ? 1 : 0)) * HD + w * 16);
      *reinterpret_cast<uint4*>((is_v ? vst : kst) + tile_off8(r, w * 16)) = val;
      if (base >= 0)
        reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(is_v ? p.vc : p.kc) + base)[w] = val;
    }
  }
}

// ------------------------------------------------------------------------------------
// Cross-split merge of one (token group, KV head) by its last CTA: thread tid owns output
// units tid + k * 128 (k < UPT), a unit being 4 consecutive dims of one query row.
// ------------------------------------------------------------------------------------
template <int HD, int UPT, int SB, bool SS>
__device__ __forceinline__ void merge_splits(const KParams& p, int tid, int nrows, int gstart,
                                             int kvh, int G, int active, float* sv) {
  constexpr int UPR = HD / 4;  // float4 units per row
  constexpr int NTHR = kConsumerWarps * 32;
  const int Q = p.NH * HD;
  const int64_t S = p.S;
  const int units = nrows * UPR;
  const int64_t ostride = int64_t(p.NH) * UPR;  // float4s between consecutive splits
  const float4* osrc[UPT];
  const float2* ssrc[UPT];
  float4 acc[UPT], gt[UPT];
  float Mx[UPT], Ls[UPT];
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const int u = tid + k * NTHR;
    const int r = u < units ? u / UPR : 0, d4 = u % UPR;
    const int t = gstart + r / G, head = kvh * G + r % G;
    osrc[k] = reinterpret_cast<const float4*>(p.po) + ((int64_t(t) * S) * p.NH + head) * UPR + d4;
    ssrc[k] = p.pml + (int64_t(t) * S) * p.NH + head;
    acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    Mx[k] = -INFINITY;
    Ls[k] = 0.0f;
    gt[k] = u < units ? *reinterpret_cast<const float4*>(p.gate + int64_t(t) * Q + head * HD + d4 * 4)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int s0 = 0; s0 < active; s0 += SB) {
    float4 v[UPT][SB];
    float2 st[UPT][SB];
#pragma unroll
    for (int k = 0; k < UPT; ++k)
#pragma unroll
      for (int j = 0; j < SB; ++j) {
        const bool ok = tid + k * NTHR < units && s0 + j < active;
        v[k][j] = ok ? __ldcg(osrc[k] + (s0 + j) * ostride) : make_float4(0.f, 0.f, 0.f, 0.f);
        st[k][j] = ok ? __ldcg(ssrc[k] + (s0 + j) * p.NH) : make_float2(-INFINITY, 0.f);
      }
#pragma unroll
    for (int k = 0; k < UPT; ++k) {
      float mb = Mx[k];
#pragma unroll
      for (int j = 0; j < SB; ++j) mb = fmaxf(mb, st[k][j].x);
      const float mu = (mb == -INFINITY) ? 0.0f : mb;
      const float wa = fast_exp2(Mx[k] - mu);
      float lsum = Ls[k] * wa;
      float4 a = make_float4(acc[k].x * wa, acc[k].y * wa, acc[k].z * wa, acc[k].w * wa);
#pragma unroll
      for (int j = 0; j < SB; ++j) {
        const float w = fast_exp2(st[k][j].x - mu);
        lsum += st[k][j].y * w;
        a.x += v[k][j].x * w; a.y += v[k][j].y * w; a.z += v[k][j].z * w; a.w += v[k][j].w * w;
      }
      acc[k] = a;
      Ls[k] = lsum;
      Mx[k] = mb;
    }
  }
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const int u = tid + k * NTHR;
    if (u >= units) continue;
    const int r = u / UPR, d4 = u % UPR;
    const int t = gstart + r / G, head = kvh * G + r % G;
    const float inv = 1.0f / (Ls[k] > 0.0f ? Ls[k] : 1.0f);
    const int e0 = head * HD + d4 * 4;  // 4 consecutive elements: same e / 8, e % 8 = j0..j0+3
    float* out = p.out + int64_t(t) * Q + (e0 % 8) * (Q / 8) + e0 / 8;
    const float o0 = acc[k].x * inv * gt[k].x, o1 = acc[k].y * inv * gt[k].y;
    const float o2 = acc[k].z * inv * gt[k].z, o3 = acc[k].w * inv * gt[k].w;
    out[0] = o0;
    out[Q / 8] = o1;
    out[2 * (Q / 8)] = o2;
    out[3 * (Q / 8)] = o3;
    if (SS) sv[u] = o0 * o0 + o1 * o1 + o2 * o2 + o3 * o3;  // unit u = r * UPR + d4
  }
}

// ------------------------------------------------------------------------------------
// The same merge with several units per thread (8-row tiles of 128-dim heads, 256-dim
// heads, 16-row tiles): thread tid owns the UPT
// adjacent output units tid * UPT .. tid * UPT + UPT - 1, a unit being 4 consecutive dims of
// one query row, all in one row (UPT divides the units per row), so one (max, sum) per split
// serves all of them.  Batches of SB splits whose statistics and partial outputs are in
// flight together (one L2 round trip per batch; the gate rides along the first), each
// folded in with one max, independent weights and one rescale.
// ------------------------------------------------------------------------------------
template <int HD, int UPT, int SB, bool SS>
__device__ __forceinline__ void merge_splits_rows(const KParams& p, int tid, int nrows, int gstart,
                                             int kvh, int G, int active, float* sv) {
  constexpr int UPR = HD / 4;  // float4 units per row
  static_assert(UPR % UPT == 0, "a thread's units share one row");
  const int Q = p.NH * HD;
  const int64_t S = p.S;
  const int units = nrows * UPR;
  const int u0 = tid * UPT;
  const bool mine = u0 < units;
  const int r = mine ? u0 / UPR : 0, d40 = u0 % UPR;
  const int t = gstart + r / G, head = kvh * G + r % G;
  const int64_t ostride = int64_t(p.NH) * UPR;  // float4s between consecutive splits
  const float4* osrc = reinterpret_cast<const float4*>(p.po) + ((int64_t(t) * S) * p.NH + head) * UPR + d40;
  const float2* ssrc = p.pml + (int64_t(t) * S) * p.NH + head;
  float4 acc[UPT], gt[UPT];
  float Mx = -INFINITY, Ls = 0.0f;
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    gt[k] = mine ? *reinterpret_cast<const float4*>(p.gate + int64_t(t) * Q + head * HD + (d40 + k) * 4)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int s0 = 0; s0 < active; s0 += SB) {
    float4 v[SB][UPT];
    float2 st[SB];
#pragma unroll
    for (int j = 0; j < SB; ++j) {
      const bool ok = mine && s0 + j < active;
      st[j] = ok ? __ldcg(ssrc + (s0 + j) * p.NH) : make_float2(-INFINITY, 0.f);
#pragma unroll
      for (int k = 0; k < UPT; ++k)
        v[j][k] = ok ? __ldcg(osrc + (s0 + j) * ostride + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mb = Mx;
#pragma unroll
    for (int j = 0; j < SB; ++j) mb = fmaxf(mb, st[j].x);
    const float mu = (mb == -INFINITY) ? 0.0f : mb;
    const float wa = fast_exp2(Mx - mu);
    float w[SB];
#pragma unroll
    for (int j = 0; j < SB; ++j) w[j] = fast_exp2(st[j].x - mu);
    float lsum = Ls * wa;
#pragma unroll
    for (int j = 0; j < SB; ++j) lsum += st[j].y * w[j];
#pragma unroll
    for (int k = 0; k < UPT; ++k) {
      float4 a = make_float4(acc[k].x * wa, acc[k].y * wa, acc[k].z * wa, acc[k].w * wa);
#pragma unroll
      for (int j = 0; j < SB; ++j) {
        a.x += v[j][k].x * w[j]; a.y += v[j][k].y * w[j];
        a.z += v[j][k].z * w[j]; a.w += v[j][k].w * w[j];
      }
      acc[k] = a;
    }
    Ls = lsum;
    Mx = mb;
  }
  if (!mine) return;
  const float inv = 1.0f / (Ls > 0.0f ? Ls : 1.0f);
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const int e0 = head * HD + (d40 + k) * 4;  // 4 consecutive elements: same e / 8, e % 8 = j0..j0+3
    float* out = p.out + int64_t(t) * Q + (e0 % 8) * (Q / 8) + e0 / 8;
    const float o0 = acc[k].x * inv * gt[k].x, o1 = acc[k].y * inv * gt[k].y;
    const float o2 = acc[k].z * inv * gt[k].z, o3 = acc[k].w * inv * gt[k].w;
    out[0] = o0;
    out[Q / 8] = o1;
    out[2 * (Q / 8)] = o2;
    out[3 * (Q / 8)] = o3;
    if (SS) sv[u0 + k] = o0 * o0 + o1 * o1 + o2 * o2 + o3 * o3;  // unit u = r * UPR + d4
  }
}

// ---- the output's justnorm statistic: sumsq[t] = sum over e of out[t][e]^2 ----
// Every output element is stored by one thread of the CTA that stores its (token group,
// KV head)'s outputs; `sv` holds the sum of squares of each (row, unit) of them, unit u of
// row r at [r * units + u].  The sums are taken in a fixed order (units of a row, rows of a
// token, KV heads of a token), so the statistic does not depend on which CTA finishes last.
// ALL: every thread of the CTA takes part (block barrier), else the consumer warps.
template <bool ALL>
__device__ __forceinline__ void sumsq_tail(const KParams& p, const float* sv, int units, int nrows,
                                           int gstart, int gcount, int G, int kvh, int tid,
                                           float* s_rowss) {
  constexpr int NTHR = ALL ? kThreads : kConsumerWarps * 32;
  auto sync = [] {
    if (ALL) __syncthreads();
    else named_barrier_consumers();
  };
  sync();
  for (int r = tid; r < nrows; r += NTHR) {
    float acc = 0.0f;
    for (int u = 0; u < units; ++u) acc += sv[r * units + u];
    s_rowss[r] = acc;
  }
  sync();
  if (tid < gcount) {
    const int t = gstart + tid;
    float part = 0.0f;
    for (int g = 0; g < G; ++g) part += s_rowss[tid * G + g];
    p.sumsq_part[int64_t(t) * p.NKV + kvh] = part;
    int prev;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(p.tok_counters + t)
                 : "memory");
    if (prev == p.NKV - 1) {  // the last KV head of this token: sum the heads in order
      float total = 0.0f;
      for (int h = 0; h < p.NKV; ++h) total += __ldcg(p.sumsq_part + int64_t(t) * p.NKV + h);
      p.sumsq[t] = total;
      p.tok_counters[t] = 0;  // self-reset for the next launch
    }
  }
}

// ------------------------------------------------------------------------------------
// The kernel.  grid = (splits, NKV, T); block = 160 threads (4 consumer warps + producer).
// ------------------------------------------------------------------------------------
// WIDE (128-dim FP8 instantiations for grids of several waves): compiled for 4 CTAs per SM
// (96 registers, a few spills) instead of 3, for more resident warps in the consumer-bound
// loop; slower on short grids, where the prologue and merge dominate.  SHK (FP8
// instantiations for shared caches): the only FP8 builds with the new-row slow path, whose
// code alone slowed the other FP8 builds by 2-3%.
template <int HD, int NT, int NS, bool SS, bool DM, bool FMA = false, bool KV8 = false,
          bool WIDE = false, bool SHK = false>
__global__ void __launch_bounds__(kThreads, NT == 1 && HD <= 128 ? (WIDE ? 4 : 3) : 1)
    decode_kernel(const __grid_constant__ KParams p) {
  static_assert(!FMA || (HD == 128 && NT == 1), "the CUDA-core consumer is 128-dim, one tile");
  static_assert(!KV8 || (NT == 1 && !FMA && HD >= 128), "FP8 caches: 128/256-dim, one tile");
  static_assert(!WIDE || (KV8 && HD == 128), "the 4-CTA build is the 128-dim FP8 kernel's");
  static_assert(!SHK || (KV8 && !WIDE), "shared-cache builds are FP8 3-CTA builds");
  using L = Smem<HD, NS, KV8>;
  constexpr int KT = HD / 16;          // MMA k-steps over head_dim / m-tiles of O^T
  constexpr int ROWS = NT * 8;         // query rows per CTA
  constexpr int PER_LANE = HD / 32;    // elements per lane in row-wise prologue math
  constexpr int TILE = L::kTileBytes;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Swizzled boxes need 1024-byte alignment; the allocation has the slack for it.
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  // Per-token info, indexed by token for shared-cache calls and by 0 otherwise.
  __shared__ int s_len[kMaxSub], s_phys[kMaxSub];
  __shared__ long long s_coff[kMaxSub], s_toff[kMaxSub];
  __shared__ int s_grouped, s_last, s_fail;
  // 256-dim heads: edge stages read a zero row in place of each V row outside the attended
  // range (pv_accumulate), and a single-token call's slot is read at entry.  Narrower heads
  // keep the zeroing slow path: that code measured faster for them.
  constexpr bool kRowMask = HD == 256;
  __shared__ uint4 s_zero_row;
  __shared__ int s_tab[kTab];  // block ids of the first kTab blocks of this CTA's range
  __shared__ CtaInfo s_ci;
  __shared__ float s_wm[kConsumerWarps][ROWS], s_wl[kConsumerWarps][ROWS];
  __shared__ float s_rowss[16];  // per-row sums of squared outputs (sumsq)
  __shared__ float s_newm[16];   // reg_new: the new token's score per row (log2 units)

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int tok = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = p.G;
  const int B = p.B;
  const int Q = p.NH * HD;

  // Pull every parameter line into the constant cache at once (see KParams).
  if (warp == 0 && lane * 64 < int(offsetof(KParams, tmk))) {
    const uint32_t word = reinterpret_cast<const uint32_t*>(&p)[lane * 16];
    asm volatile("" ::"r"(word));
  }
  // ---- token info: the group's tokens and the tokens whose new k/v this CTA may have to
  //      substitute (shared-cache: every token of the call; otherwise this token alone).
  const int ninfo = p.shared ? p.T : 1;
  if (warp == kConsumerWarps) {
    // This token's per-head inputs are needed once the sequence length is known; start
    // pulling them into L2 now, while that first load is in flight.
    const int hq = kvh * G;
    const int64_t qrow = int64_t(tok) * p.q_stride;
    if (p.raw) {
      const float* qf = static_cast<const float*>(p.q) + qrow;
      prefetch_range(qf + hq * HD, G * HD * 4, lane);
      prefetch_range(qf + (p.NH + kvh) * HD, HD * 4, lane);
      prefetch_range(p.v + int64_t(tok) * p.NKV * HD + kvh * HD, HD * 4, lane);
      prefetch_range(static_cast<const char*>(p.sqk) + (p.sqk_dtype == DORY_DTYPE_F32 ? 4 : 2) *
                         int64_t(hq) * HD,
                     G * HD * (p.sqk_dtype == DORY_DTYPE_F32 ? 4 : 2), lane);
    } else {
      prefetch_range(static_cast<const __nv_bfloat16*>(p.q) + qrow + hq * HD, G * HD * 2, lane);
    }
    prefetch_range(p.gate + int64_t(tok) * Q + hq * HD, G * HD * 4, lane);
    if (p.tm_mode && lane == 0) {
      prefetch_tensormap(&p.tmk);
      if (p.tm_mode == 2) prefetch_tensormap(&p.tmv);
    }
  }
  if (tid == 0) {
    s_grouped = 1;
    s_fail = 0;
  }
  if (tid < ninfo) {
    const int t = p.shared ? tid : tok;
    s_len[tid] = p.seq_lens[t];
    s_coff[tid] = p.multi ? p.cache_offsets[t] : 0;
    s_toff[tid] = p.multi ? p.table_offsets[t] : 0;
  }
  if (kRowMask) {
    if (tid == 64) s_zero_row = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  // ---- token group: shared-cache tokens that read one cache through one table share
  //      every K/V byte, so the CTAs of the group's first token serve all of them.
  int gstart = tok, gcount = 1;
  if (p.shared) {
    const int tpg = ROWS / G;
    gstart = (tok / tpg) * tpg;
    gcount = min(tpg, p.T - gstart);
    if (gcount > 1) {
      if (tid < gcount &&
          (s_coff[gstart + tid] != s_coff[gstart] || s_toff[gstart + tid] != s_toff[gstart]))
        s_grouped = 0;
      __syncthreads();
      if (!s_grouped) {
        gstart = tok;
        gcount = 1;
      } else if (tok != gstart) {
        return;  // the group's first token serves this one
      }
    }
  }
  const int ibase = p.shared ? gstart : 0;  // info index of group token 0
  int lo = 0x7fffffff, hi = 0;
  for (int j = 0; j < gcount; ++j) {
    const int len = s_len[ibase + j];
    if (len > 0) {
      const int first = p.window > 0 ? max(len - p.window, 0) : 0;
      lo = min(lo, first);
      hi = max(hi, len);
    }
  }
  if (hi == 0) lo = 0;
  const long long coff = s_coff[ibase];
  const long long toff = s_toff[ibase];
  const int nsub = p.nsub;
  const Split sp = split_layout(lo, hi, B, p.b_shift, p.S, p.bpt, p.tps_min);
  const int nrows = gcount * G;
  // Raw calls whose tokens each read their own cache (not shared): the new token's row
  // (position seq_len - 1) is left out of the chunk loop (attended cache rows [lo, hi_c))
  // and enters the merge from the k/v the kernel normalises, in the CTA that holds its
  // position, which also appends it in the prologue (off the chunk loop's critical path).
  const bool reg_new = p.raw && !p.shared;
  const int hi_c = reg_new ? hi - 1 : hi;

  if (sp.tiles == 0) {
    // Padding request(s): the reference's combine writes 0 * gate.
    if (split == 0) {
      grid_dependency_wait();
      float* sv0 = reinterpret_cast<float*>(smem + L::kStages);  // [nrows][HD] squares
      for (int i = tid; i < nrows * HD; i += kThreads) {
        const int r = i / HD, d = i % HD;
        const int t = gstart + r / G, head = kvh * G + r % G;
        const int e = head * HD + d;
        const float val = 0.0f * p.gate[int64_t(t) * Q + e];
        p.out[int64_t(t) * Q + (e % 8) * (Q / 8) + e / 8] = val;
        if (SS) sv0[i] = val * val;
      }
      if (SS) sumsq_tail<true>(p, sv0, HD, nrows, gstart, gcount, G, kvh, tid, s_rowss);
    }
    return;
  }
  const int tile_begin = split * sp.tps;
  if (tile_begin >= sp.tiles) return;
  const int tile_end = min(tile_begin + sp.tps, sp.tiles);
  const int bb = sp.first_block + tile_begin * p.bpt;
  const int be = min(sp.first_block + tile_end * p.bpt, sp.first_block + sp.nblocks);
  const int CPB = B / kChunk;
  const int cb = max(bb * CPB, lo / kChunk);
  const int ce = min(be * CPB, (hi_c + kChunk - 1) / kChunk);
  const int nchunks = max(ce - cb, 0);

  const uint32_t bars = smem_u32(smem + L::kBars);
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (NS + s); };
  int4* meta = reinterpret_cast<int4*>(smem + L::kMeta);
  __nv_bfloat16* q2 = reinterpret_cast<__nv_bfloat16*>(smem + L::kQ);
  __nv_bfloat16* subkv = reinterpret_cast<__nv_bfloat16*>(smem + L::kSub);

  const bool offset_ok = (coff & 7) == 0;
  const int b_first = div_p2(cb, CPB, p.cpb_shift);
  const int b_last = div_p2(ce - 1, CPB, p.cpb_shift);
  const int32_t* table = p.table + toff;
  // Tensor copies address the cache by block index, so an offset must be whole blocks.
  const long long coff_blocks = coff == 0 ? 0 : (coff % p.sb == 0 ? coff / p.sb : -1);
  const bool use_tma = p.tm_mode != 0 && offset_ok && coff_blocks >= 0 &&
                       coff_blocks + p.ncache_blocks <= p.tm_blocks;

  const uint64_t policy = l2_evict_first_policy();
  // Tensor path: arm the chunk's stage and copy its K (and V) tile; one thread.  Records the
  // stage's block id (-1 for an id outside the cache) and chunk index for the consumer.
  // L2 prefetch of chunk i (tensor path; chunks with a bad block id are skipped).
  auto prefetch_chunk = [&](int i) {
    const int c = cb + i;
    const int blk = div_p2(c, CPB, p.cpb_shift);
    const int phys = blk - b_first < kTab ? s_tab[blk - b_first] : table[blk];
    if (phys < 0 || (p.ncache_blocks > 0 && phys >= p.ncache_blocks)) return;
    const int row0 = mod_p2(c, CPB, p.cpb_shift) * kChunk;
    const int blkc = int(coff_blocks + phys);
    tma_prefetch_5d(&p.tmk, 0, row0, 0, kvh, blkc);
    if (p.tm_mode == 2) tma_prefetch_5d(&p.tmv, 0, row0, 0, kvh, blkc);
  };
  auto issue_chunk = [&](int i) {
    const int stage = i % NS;
    const int c = cb + i;
    const int blk = div_p2(c, CPB, p.cpb_shift);
    const int phys = blk - b_first < kTab ? s_tab[blk - b_first] : table[blk];
    const bool phys_ok = phys >= 0 && (p.ncache_blocks <= 0 || phys < p.ncache_blocks);
    // keep the L2 prefetch p.pf chunks ahead of the ring's copies
    if (i >= NS && p.pf > 0 && i + p.pf < nchunks) prefetch_chunk(i + p.pf);
    meta[stage] = make_int4(phys_ok ? phys : -1, 0, c, 0);
    if (phys_ok) {
      mbar_arrive_expect_tx(full_bar(stage), L::kStageBytes);
      const uint32_t kt = smem_u32(smem + L::kStages + stage * L::kStageBytes);
      const int row0 = mod_p2(c, CPB, p.cpb_shift) * kChunk;
      const int blkc = int(coff_blocks + phys);
      tma_load_5d(kt, &p.tmk, 0, row0, 0, kvh, blkc, full_bar(stage), policy);
      if (p.tm_mode == 2)
        tma_load_5d(kt + TILE, &p.tmv, 0, row0, 0, kvh, blkc, full_bar(stage), policy);
    } else {
      record_error(p.err, DORY_DEVERR_BLOCK_OOB);
      mbar_arrive(full_bar(stage));  // nothing to load; the consumer zeroes the tile
    }
  };

  if (warp == kConsumerWarps) {
    // =============================== producer warp ===============================
    // The pipeline's barriers are set up here, not by the whole CTA: the consumer warps go
    // straight on to their query rows (below) while this warp reads the block ids and
    // issues the first copies, and wait for the set-up only before their first stage.
    if (lane == 0) {
      for (int s = 0; s < NS; ++s) {
        // tensor path: the producer's arrive.expect_tx; copy path: 32 lanes' completions + 1
        mbar_init(full_bar(s), use_tma ? 1 : 33);
        mbar_init(empty_bar(s), 1);  // the consumer warp that read the stage
      }
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      if (!offset_ok) record_error(p.err, DORY_DEVERR_OFFSET_ALIGN);
    }
    __syncwarp();
    pipeline_ready_arrive();
    if (KV8 && !use_tma) {
      // FP8 caches are copied by tensor maps only (a cache offset that is not whole blocks,
      // or a cache beyond the map): recorded, and the consumers skip the chunks.
      if (lane == 0) record_error(p.err, DORY_DEVERR_OFFSET_ALIGN);
      return;
    }
    // Tensor path (the usual one): lane 0 publishes the stage's block id, arms full[stage]
    // with the stage's byte count and issues one box copy of the chunk's K and V tiles
    // (two, K then V, when V does not directly follow K in memory): 16 rows from row 0 of
    // the chunk, all 64-dim quarters of each row, at (KV head, block).  Rows of the box
    // outside the attended range are read too and zeroed by the consumer.
    if (use_tma) {
      // The block ids of this CTA's range go to shared memory; lane 0 then issues the first
      // ring's worth of chunks.  From there on each consumer warp refills the stage it has
      // just finished (stages map to fixed warps), so no producer hand-off sits between a
      // stage falling free and its next copy.
      for (int k = lane; k < kTab && b_first + k <= b_last; k += 32) s_tab[k] = table[b_first + k];
      __syncwarp();
      if (lane == 0)
        for (int i = 0; i < NS && i < nchunks; ++i) issue_chunk(i);
      // The chunks after the ring's first fill, up to p.pf of them, start their DRAM reads
      // now (into L2), one per lane; later ring refills keep the window p.pf chunks ahead.
      if (p.pf > 0) {
        const int pf_end = min(nchunks, NS + p.pf);
        for (int i = NS + lane; i < pf_end; i += 32) prefetch_chunk(i);
      }
      __syncwarp();
      grid_launch_dependents();
      return;
    }
    // Copy path: every lane copies 16-byte pieces with cp.async into the same swizzled
    // layout, zero-filling rows outside [lo, hi); completion reaches full[stage] through one
    // cp.async.mbarrier.arrive per lane, plus lane 0's arrive after publishing the block id.
    const __nv_bfloat16* kbase = p.kc + coff + int64_t(kvh) * p.sh;
    const __nv_bfloat16* vbase = p.vc + coff + int64_t(kvh) * p.sh;
    constexpr int VEC = HD / 8;                    // 16-byte pieces per row
    constexpr int PER_LANE = 2 * kChunk * VEC / 32;
    // Block-table window of 32 entries, prefetched one window ahead.
    int wbase = b_first;
    int win_cur = (b_first + lane <= b_last) ? table[b_first + lane] : -1;
    int win_nxt = (b_first + 32 + lane <= b_last) ? table[b_first + 32 + lane] : -1;
    int issued = 0;
    for (int i = 0; i < nchunks; ++i) {
      const int stage = i % NS;
      const uint32_t parity = ((i / NS) & 1) ^ 1;
      if (!mbar_wait(empty_bar(stage), parity)) {
        if (lane == 0) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
        break;
      }
      const int c = cb + i;
      const int blk = div_p2(c, CPB, p.cpb_shift);
      while (blk >= wbase + 32) {
        wbase += 32;
        win_cur = win_nxt;
        win_nxt = (wbase + 32 + lane <= b_last) ? table[wbase + 32 + lane] : -1;
      }
      const int phys = __shfl_sync(0xffffffffu, win_cur, blk - wbase);
      const bool phys_ok =
          phys >= 0 && (p.ncache_blocks <= 0 || phys < p.ncache_blocks) && offset_ok;
      if (!phys_ok && lane == 0 && offset_ok) record_error(p.err, DORY_DEVERR_BLOCK_OOB);
      const uint32_t kt = smem_u32(smem + L::kStages + stage * L::kStageBytes);
      const uint32_t vt = kt + TILE;
      const int64_t block_off = int64_t(phys_ok ? phys : 0) * p.sb +
                                int64_t(mod_p2(c, CPB, p.cpb_shift) * kChunk) * p.so;
#pragma unroll
      for (int k = 0; k < PER_LANE; ++k) {
        const int j = k * 32 + lane;
        const bool is_v = j >= kChunk * VEC;
        const int jj = is_v ? j - kChunk * VEC : j;
        const int r = jj / VEC, w = jj % VEC;
        const int pos = c * kChunk + r;
        const bool valid = phys_ok && pos >= lo && pos < hi_c;
        const __nv_bfloat16* src =
            valid ? (is_v ? vbase : kbase) + block_off + int64_t(r) * p.so + w * 8 : p.kc;
        cp_async_16((is_v ? vt : kt) + tile_off(r, w * 8), src, valid ? 16u : 0u, policy);
      }
      cp_async_arrive_noinc(full_bar(stage));
      if (lane == 0) {
        meta[stage] = make_int4(phys_ok ? phys : -1, 0, c, 0);
        mbar_arrive(full_bar(stage));
      }
      ++issued;
    }
    grid_launch_dependents();
    // Stay until this warp's copies have landed (bounded), then leave.
    for (int s = 0; s < NS && s < issued; ++s) {
      const int last = s + ((issued - 1 - s) / NS) * NS;
      mbar_wait(full_bar(s), (last / NS) & 1);
    }
    return;
  }

  // =============================== consumer warps ===============================
  // Everything below reads this step's inputs or writes outputs: after the previous grid.
  grid_dependency_wait();
  // (0) New tokens that read this CTA's cache through this CTA's table ("same") alias its
  //     rows by position.  Others (a shared-cache call whose tokens use different tables)
  //     alias by physical address, which needs the block id of their slot.
  if (warp == 0 && lane < nsub) {
    const int len = s_len[lane];
    const bool same = s_coff[lane] == coff && s_toff[lane] == toff;
    s_phys[lane] = (len > 0 && !same) ? p.table[s_toff[lane] + (len - 1) / B] : -1;
  }
  // The CTA holding the new token's position (the last active split) adds its row in the
  // merge and appends it; its slot is read now, in flight with the query rows' loads.
  const bool add_new = reg_new && split == sp.active - 1;
  long long slot_new = -1;
  if (add_new && p.raw && tid == 0) {
    const int pos = s_len[0] - 1;
    if (!p.multi) {
      slot_new = p.slot_mapping[0];
    } else if (p.slot_mapping) {
      slot_new = p.slot_mapping[tok];
    } else {
      const int ph = table[div_p2(pos, B, p.b_shift)];
      if (ph >= 0) slot_new = (long long)ph * B + mod_p2(pos, B, p.b_shift);
      else record_error(p.err, DORY_DEVERR_BLOCK_OOB);
    }
  }
  int sub_lo = 0x7fffffff, sub_hi = -1;  // chunks that may hold a same-table new row
  bool any_foreign = false;
  if (p.raw && !reg_new) {
    for (int s2 = 0; s2 < nsub; ++s2) {
      const int len = s_len[s2];
      if (len <= 0) continue;
      if (s_coff[s2] == coff && s_toff[s2] == toff) {
        sub_lo = min(sub_lo, (len - 1) / kChunk);
        sub_hi = max(sub_hi, (len - 1) / kChunk);
      } else {
        any_foreign = true;
      }
    }
  }
  const int c_full_lo = (lo + kChunk - 1) / kChunk;  // chunks in [c_full_lo, c_full_hi) have
  const int c_full_hi = hi_c / kChunk;               // every row inside [lo, hi_c)
  if (tid == 0) {
    s_ci.coff = coff;
    s_ci.toff = toff;
    s_ci.lo = lo;
    s_ci.hi = hi_c;
    s_ci.kvh = kvh;
    s_ci.nsub = nsub;
    s_ci.ibase = ibase;
    s_ci.gcount = gcount;
    s_ci.offset_ok = offset_ok;
    s_ci.reg_new = reg_new;
    s_ci.tok = tok;
  }
  // (1) query rows: normalise / scale / round, as the reference, into q2 [ROWS][HD] bf16;
  // (2) new keys / values of the sub tokens: k = bf16(k * inv_norm(k)), v = bf16(v).
  // Every load of this warp's rows (q, sqk) and of its first sub token (k, v) is issued
  // before any of the arithmetic: one L2 round trip, not one per dependent step.
  constexpr int RPW = ROWS / kConsumerWarps;  // query rows per consumer warp
  if constexpr (HD == 256) {
    const bool sub0 = p.raw && warp < nsub && (!reg_new || add_new);
    // 256-dim heads: 16-byte loads where the bases allow them (every row offset is a
    // multiple of 16 bytes), and in raw mode the FP64 sums of all of this warp's rows (its
    // query rows and its new token's k row) taken together, each in row_inv_norm's order
    // (same bits), so that their shuffle chains overlap.
    const bool vec = ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.v)) &
                      15) == 0;
    const bool vsqk = p.sqk_dtype == DORY_DTYPE_BF16 &&
                      (reinterpret_cast<uintptr_t>(p.sqk) & 15) == 0;
    auto load_f32 = [&](const float* src, float (&x)[PER_LANE]) {
      if (vec) {
#pragma unroll
        for (int i = 0; i < PER_LANE; i += 4) {
          const float4 a = *reinterpret_cast<const float4*>(src + lane * PER_LANE + i);
          x[i] = a.x; x[i + 1] = a.y; x[i + 2] = a.z; x[i + 3] = a.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) x[i] = src[lane * PER_LANE + i];
      }
    };
    auto load_bf16 = [&](const __nv_bfloat16* src, bool v16, float (&x)[PER_LANE]) {
      if (v16) {
#pragma unroll
        for (int i = 0; i < PER_LANE; i += 8) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + lane * PER_LANE + i);
          const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            x[i + 2 * k] = __uint_as_float(u[k] << 16);
            x[i + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) x[i] = __bfloat162float(src[lane * PER_LANE + i]);
      }
    };
    float qv[RPW][PER_LANE], sqv[RPW][PER_LANE], kv0[PER_LANE], vv0[PER_LANE];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int r = warp + j * kConsumerWarps;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) qv[j][i] = sqv[j][i] = 0.0f;
      if (r >= nrows) continue;
      const int t = gstart + r / G;
      const int head = kvh * G + r % G;
      if (p.raw) {
        load_f32(static_cast<const float*>(p.q) + int64_t(t) * p.q_stride + head * HD, qv[j]);
        if (vsqk) {
          load_bf16(static_cast<const __nv_bfloat16*>(p.sqk) + head * HD, true, sqv[j]);
        } else {
#pragma unroll
          for (int i = 0; i < PER_LANE; ++i)
            sqv[j][i] = load_sqk(p.sqk, p.sqk_dtype, head * HD + lane * PER_LANE + i);
        }
      } else {
        const __nv_bfloat16* src =
            static_cast<const __nv_bfloat16*>(p.q) + int64_t(t) * p.q_stride + head * HD;
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) qv[j][i] = __bfloat162float(src[lane * PER_LANE + i]);
      }
    }
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) kv0[i] = vv0[i] = 0.0f;
    if (sub0) {
      const int t = p.shared ? warp : tok;
      load_f32(static_cast<const float*>(p.q) + int64_t(t) * p.q_stride + (p.NH + kvh) * HD, kv0);
      load_f32(p.v + int64_t(t) * p.NKV * HD + kvh * HD, vv0);
    }
    if (p.raw) {
      double acc[RPW + 1];
#pragma unroll
      for (int j = 0; j <= RPW; ++j) {
        acc[j] = 0.0;
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
          const float x = j < RPW ? qv[j][i] : kv0[i];
          acc[j] += double(x) * double(x);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int j = 0; j <= RPW; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const int r = warp + j * kConsumerWarps;
        const float rn = inv_norm_from_sum(acc[j], p.eps);
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
          const float s = __fmul_rn(sqv[j][i], p.sqk_factor);
          const float qn = __fmul_rn(qv[j][i], rn);
          const float qb = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(s, s), qn)));
          q2[r * HD + lane * PER_LANE + i] =
              __float2bfloat16_rn(r < nrows ? __fmul_rn(qb, p.scale) : 0.0f);
        }
      }
      if (sub0) {
        const float rn = inv_norm_from_sum(acc[RPW], p.eps);
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
          const int d = lane * PER_LANE + i;
          subkv[(warp * 2 + 0) * HD + d] = new_kv<KV8>(__fmul_rn(kv0[i], rn), p.k_scale);
          subkv[(warp * 2 + 1) * HD + d] = new_kv<KV8>(vv0[i], p.v_scale);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const int r = warp + j * kConsumerWarps;
        if (r >= nrows) {
#pragma unroll
          for (int i = 0; i < PER_LANE; ++i) q2[r * HD + lane * PER_LANE + i] = __float2bfloat16_rn(0.0f);
          continue;
        }
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i)
          q2[r * HD + lane * PER_LANE + i] = __float2bfloat16_rn(__fmul_rn(qv[j][i], p.scale));
      }
    }
  } else {
    float qv[RPW][PER_LANE], sqv[RPW][PER_LANE], kv0[PER_LANE], vv0[PER_LANE];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int r = warp + j * kConsumerWarps;
      if (r >= nrows) continue;
      const int t = gstart + r / G;
      const int head = kvh * G + r % G;
      if (p.raw) {
        const float* src = static_cast<const float*>(p.q) + int64_t(t) * p.q_stride + head * HD;
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
          qv[j][i] = src[lane * PER_LANE + i];
          sqv[j][i] = load_sqk(p.sqk, p.sqk_dtype, head * HD + lane * PER_LANE + i);
        }
      } else {
        const __nv_bfloat16* src =
            static_cast<const __nv_bfloat16*>(p.q) + int64_t(t) * p.q_stride + head * HD;
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) qv[j][i] = __bfloat162float(src[lane * PER_LANE + i]);
      }
    }
    const bool sub0 = p.raw && warp < nsub && (!reg_new || add_new);
    if (sub0) {
      const int t = p.shared ? warp : tok;
      const float* ksrc =
          static_cast<const float*>(p.q) + int64_t(t) * p.q_stride + (p.NH + kvh) * HD;
      const float* vsrc = p.v + int64_t(t) * p.NKV * HD + kvh * HD;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        kv0[i] = ksrc[lane * PER_LANE + i];
        vv0[i] = vsrc[lane * PER_LANE + i];
      }
    }
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int r = warp + j * kConsumerWarps;
      if (r >= nrows) {
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) q2[r * HD + lane * PER_LANE + i] = __float2bfloat16_rn(0.0f);
        continue;
      }
      if (p.raw) {
        const float rn = row_inv_norm<PER_LANE>(qv[j], p.eps);
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
          const float s = __fmul_rn(sqv[j][i], p.sqk_factor);
          const float qn = __fmul_rn(qv[j][i], rn);
          const float qb = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(s, s), qn)));
          q2[r * HD + lane * PER_LANE + i] = __float2bfloat16_rn(__fmul_rn(qb, p.scale));
        }
      } else {
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i)
          q2[r * HD + lane * PER_LANE + i] = __float2bfloat16_rn(__fmul_rn(qv[j][i], p.scale));
      }
    }
    if (sub0) {
      const float rn = row_inv_norm<PER_LANE>(kv0, p.eps);
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int d = lane * PER_LANE + i;
        subkv[(warp * 2 + 0) * HD + d] = new_kv<KV8>(__fmul_rn(kv0[i], rn), p.k_scale);
        subkv[(warp * 2 + 1) * HD + d] = new_kv<KV8>(vv0[i], p.v_scale);
      }
    }
  }
  // Further sub tokens of a shared-cache call (more than four).
  if (p.raw) {
    for (int s = warp + kConsumerWarps; s < nsub; s += kConsumerWarps) {
      const int t = p.shared ? s : tok;
      const float* ksrc =
          static_cast<const float*>(p.q) + int64_t(t) * p.q_stride + (p.NH + kvh) * HD;
      const float* vsrc = p.v + int64_t(t) * p.NKV * HD + kvh * HD;
      float kv[PER_LANE];
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) kv[i] = ksrc[lane * PER_LANE + i];
      const float rn = row_inv_norm<PER_LANE>(kv, p.eps);
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int d = lane * PER_LANE + i;
        subkv[(s * 2 + 0) * HD + d] = new_kv<SHK>(__fmul_rn(kv[i], rn), p.k_scale);
        subkv[(s * 2 + 1) * HD + d] = new_kv<SHK>(vsrc[d], p.v_scale);
      }
    }
  }
  named_barrier_consumers();
  pipeline_ready_wait();  // the producer has initialised the stages' barriers
  if (add_new) {
    // The new token's score against each query row (bf16 operands, FP32 sum), for the merge.
    for (int r = warp; r < nrows; r += kConsumerWarps) {
      float dot = 0.0f;
      for (int d = 2 * lane; d < HD; d += 64) {
        const float2 qv2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q2 + r * HD + d));
        const float2 kv2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(subkv + d));
        dot = fmaf(qv2.x, kv2.x, dot);
        dot = fmaf(qv2.y, kv2.y, dot);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      if (lane == 0) s_newm[r] = dot * (KV8 ? kLog2e * p.k_scale : kLog2e);
    }
    // The append: the new k and v rows at the token's slot (a negative slot is a padding
    // token, which vLLM does not cache; a slot outside the cache is recorded and skipped).
    if (p.raw && warp == 0) {
      const long long slot = __shfl_sync(0xffffffffu, slot_new, 0);
      if (slot >= 0) {
        const long long blk = slot / B;
        if ((p.ncache_blocks > 0 && blk >= p.ncache_blocks) || !offset_ok) {
          if (lane == 0) record_error(p.err, DORY_DEVERR_SLOT_OOB);
        } else {
          const long long base = coff + blk * p.sb + (slot % B) * p.so + (long long)kvh * p.sh;
          if constexpr (KV8) {
            // e4m3 bytes (base in bytes): 16 per piece, from the exact e4m3 values in subkv
            constexpr int kVec8 = HD / 16;
            for (int idx = lane; idx < 2 * kVec8; idx += 32) {
              const bool is_v = idx >= kVec8;
              const int w = is_v ? idx - kVec8 : idx;
              const uint4 val = e4m3x16(subkv + (is_v ? HD : 0) + w * 16);
              uint8_t* dst = reinterpret_cast<uint8_t*>(is_v ? p.vc : p.kc) + base;
              reinterpret_cast<uint4*>(dst)[w] = val;
            }
          } else {
          constexpr int kVec = HD / 8;
          for (int idx = lane; idx < 2 * kVec; idx += 32) {
            const bool is_v = idx >= kVec;
            const int w = is_v ? idx - kVec : idx;
            const uint4 val = reinterpret_cast<const uint4*>(subkv + (is_v ? HD : 0))[w];
            reinterpret_cast<uint4*>((is_v ? p.vc : p.kc) + base)[w] = val;
          }
          }
        }
      }
    }
  }

  // (4) B fragments of Q^T (k = dims, n = query rows), resident for the whole loop.
  const int g = lane >> 2;
  const int t4 = lane & 3;
  uint32_t qb[NT][KT][2];
  // FP8, 128-dim heads: the fragments live in the upper half of the query area (free with
  // one 8-row tile), [KT / 2][32 lanes] x 16 bytes, reloaded per chunk rather than held in
  // 16 registers (256-dim heads keep them in registers: one CTA per SM leaves room).  Every
  // warp writes the same values and each lane reads back only what it wrote itself.
  constexpr bool kQFragSmem = KV8 && HD == 128;
  uint4* qfrag = reinterpret_cast<uint4*>(smem + L::kQ + 8 * HD * 2);
  if constexpr (KV8) {
    // k-step kk's slot pairs (2t4, 2t4+1), (2t4+8, 2t4+9) are the dims
    // HD/4 * t4 + 4kk + {0, 1}, {2, 3}, the order the K operands are read in
    static_assert(8 * HD * 2 >= (KT / 2) * 32 * 16, "the fragments fit in the free half");
    const uint32_t* row = reinterpret_cast<const uint32_t*>(q2 + g * HD);
#pragma unroll
    for (int j = 0; j < KT / 2; ++j) {
      const int pair = ((HD / 4) * t4 + 8 * j) / 2;
      const uint4 f = make_uint4(bf16x2_to_f16x2(row[pair]), bf16x2_to_f16x2(row[pair + 1]),
                                 bf16x2_to_f16x2(row[pair + 2]), bf16x2_to_f16x2(row[pair + 3]));
      if constexpr (kQFragSmem) {
        qfrag[j * 32 + lane] = f;
      } else {
        qb[0][2 * j][0] = f.x;
        qb[0][2 * j][1] = f.y;
        qb[0][2 * j + 1][0] = f.z;
        qb[0][2 * j + 1][1] = f.w;
      }
    }
  } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        const uint32_t* row =
            reinterpret_cast<const uint32_t*>(q2 + (nt * 8 + g) * HD + kk * 16);
        qb[nt][kk][0] = row[t4];
        qb[nt][kk][1] = row[t4 + 4];
      }
  }
  // Row bounds of the two query rows this lane accumulates per n-tile.
  int rfirst[NT][2], rlen[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = nt * 8 + 2 * t4 + i;
      int len = 0;
      if (r < nrows) len = s_len[ibase + r / G];
      rlen[nt][i] = (reg_new && len > 0) ? len - 1 : len;
      rfirst[nt][i] = (p.window > 0) ? max(len - p.window, 0) : 0;
    }

  float o[NT][KT][4];
  float m[NT][2], l[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int kk = 0; kk < KT; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nt][kk][e] = 0.0f;
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.0f;
  }
  // FP8 caches: scores carry k_scale (folded into the log2 factor), outputs v_scale (applied
  // to each warp's accumulator); the chunks run only with tensor-map copies.
  const float kscore = KV8 ? kLog2e * p.k_scale : kLog2e;
  const int nloop = (KV8 && !use_tma) ? 0 : nchunks;

  bool failed = false;
  // CUDA-core consumer state (FMA instantiations only): the query rows as FP32 (the same
  // bf16 values as the tensor-core B fragments), the attended range of this lane's row.
  FmaRows fst;
  float fq[4][4];
  int f_first = 0, f_len = 0;
  // Per-warp P buffer: the upper half of the query area (one 8-row tile uses the lower half).
  float* pbuf = reinterpret_cast<float*>(smem + L::kQ + 8 * HD * 2) + warp * 64;
  if constexpr (FMA) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint2 w = *reinterpret_cast<const uint2*>(q2 + r * HD + 4 * lane);
      unpack_bf16x4(w, fq[r]);
#pragma unroll
      for (int j = 0; j < 4; ++j) fst.o[r][j] = 0.0f;
      fst.m[r] = -INFINITY;
    }
    fst.l = 0.0f;
    const int r = lane >> 3;
    const int f_seq = r < nrows ? s_len[ibase + r / G] : 0;
    f_first = (p.window > 0) ? max(f_seq - p.window, 0) : 0;
    f_len = (reg_new && f_seq > 0) ? f_seq - 1 : f_seq;
    for (int i = warp; i < nchunks; i += kConsumerWarps) {
      const int stage = i % NS;
      if (!mbar_wait(full_bar(stage), (i / NS) & 1)) {
        if (lane == 0) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
        failed = true;
        break;
      }
      const int4 mt = meta[stage];
      const int phys = mt.x;
      const int c = mt.z;
      uint8_t* kst = smem + L::kStages + stage * L::kStageBytes;
      uint8_t* vst = kst + TILE;
      bool touched = false;
      const bool partial = use_tma && (c < c_full_lo || c >= c_full_hi || phys < 0);
      if (partial || (c >= sub_lo && c <= sub_hi) || any_foreign)
        touched = fixup_stage<HD>(p, kst, vst, c, phys, partial, lane, s_ci, s_len, s_phys,
                                  s_coff, s_toff, subkv);
      __syncwarp();
      fma_chunk(fst, fq, kst, vst, pbuf, lane, c, f_first, f_len);
      if (use_tma) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && i + NS < nchunks) issue_chunk(i + NS);
      } else {
        if (touched) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(stage));
      }
    }
    // Row sums: the 8 lanes of a row hold disjoint token pairs of it.
    fst.l += __shfl_xor_sync(0xffffffffu, fst.l, 1);
    fst.l += __shfl_xor_sync(0xffffffffu, fst.l, 2);
    fst.l += __shfl_xor_sync(0xffffffffu, fst.l, 4);
  } else {
  for (int i = warp; i < nloop; i += kConsumerWarps) {
    const int stage = i % NS;
    const uint32_t parity = (i / NS) & 1;
    if (!mbar_wait(full_bar(stage), parity)) {
      if (lane == 0) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
      failed = true;
      break;
    }
    const int4 mt = meta[stage];
    const int phys = mt.x;
    const int c = mt.z;
    uint8_t* kst = smem + L::kStages + stage * L::kStageBytes;
    uint8_t* vst = kst + TILE;
    // Boundary chunks, bad blocks and chunks holding a new token's row take the slow path
    // (zeroing, substitution, the append itself); the rest go straight to the math.
    bool touched = false;
    const bool partial = !KV8 && use_tma && (c < c_full_lo || c >= c_full_hi || phys < 0);
    if constexpr (SHK) {
      // FP8, shared caches: only stages holding a sub token's new row take a slow path (the
      // row's bytes, and its append); edges and bad blocks are masked by the consumer.
      if ((c >= sub_lo && c <= sub_hi) || any_foreign) {
        fixup_stage8<HD>(p, kst, vst, c, phys, lane, s_ci, s_len, s_phys, s_coff, s_toff,
                         subkv);
        __syncwarp();
      }
    } else if constexpr (KV8) {
      // FP8 without shared caches: no slow path (the new row enters the merge apart)
    } else {
      if ((partial && !kRowMask) || (c >= sub_lo && c <= sub_hi) || any_foreign)
        touched = fixup_stage<HD>(p, kst, vst, c, phys, partial && !kRowMask, lane, s_ci,
                                  s_len, s_phys, s_coff, s_toff, subkv);
      __syncwarp();
    }

    // S^T = K Q^T : [16 tokens x 8 rows] per n-tile, as two independent MMA chains (even
    // and odd k-steps) to halve the dependent latency.
    float sc[NT][4], sc2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] = sc2[nt][e] = 0.0f;
    if constexpr (KV8) {
      // e4m3 K straight into the f16 MMA operands: lane (g, t4) reads rows g and g + 8 at dims
      // [HD/4 * t4, HD/4 * (t4 + 1)); k-step kk takes its dims HD/4 * t4 + 4kk .. + 3 as the
      // slot pairs (2t4, 2t4+1) and (2t4+8, 2t4+9) (a dot product allows any order; the
      // query fragments follow it).
      constexpr int PK = HD / 64;  // 16-byte pieces per lane and row
      uint32_t kw[2][4 * PK];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int pi = 0; pi < PK; ++pi) {
          const uint4 w =
              *reinterpret_cast<const uint4*>(kst + tile_off8(g + 8 * h, (HD / 4) * t4 + 16 * pi));
          kw[h][4 * pi + 0] = w.x;
          kw[h][4 * pi + 1] = w.y;
          kw[h][4 * pi + 2] = w.z;
          kw[h][4 * pi + 3] = w.w;
        }
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        uint32_t b0 = qb[0][kk][0], b1 = qb[0][kk][1];
        if constexpr (kQFragSmem) {
          const uint4 qf = qfrag[(kk >> 1) * 32 + lane];
          b0 = (kk & 1) ? qf.z : qf.x;
          b1 = (kk & 1) ? qf.w : qf.y;
        }
        const uint32_t a0 = e4m3x2_to_f16x2(kw[0][kk] & 0xffffu);
        const uint32_t a2 = e4m3x2_to_f16x2(kw[0][kk] >> 16);
        const uint32_t a1 = e4m3x2_to_f16x2(kw[1][kk] & 0xffffu);
        const uint32_t a3 = e4m3x2_to_f16x2(kw[1][kk] >> 16);
        mma_f16((kk & 1) ? sc2[0] : sc[0], a0, a1, a2, a3, b0, b1);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[0][e] += sc2[0][e];
    } else {
      const uint32_t kbase_s = smem_u32(kst);
      const int kr = lane & 15, kd = (lane >> 4) * 8;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kbase_s + tile_off(kr, kk * 16 + kd), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          mma16<KV8>((kk & 1) ? sc2[nt] : sc[nt], a0, a1, a2, a3, qb[nt][kk][0], qb[nt][kk][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] += sc2[nt][e];
    }
    // Online softmax (log2 domain) and P^T operands.
    const int pos0 = c * kChunk + g;
    const int pos1 = pos0 + 8;
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float pv[4];
      float alpha[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const bool bad = KV8 && phys < 0;  // FP8: a bad block's stage was never loaded
        const bool v0 = !bad && pos0 >= rfirst[nt][i] && pos0 < rlen[nt][i];
        const bool v1 = !bad && pos1 >= rfirst[nt][i] && pos1 < rlen[nt][i];
        const float x0 = v0 ? sc[nt][i] * kscore : -INFINITY;
        const float x1 = v1 ? sc[nt][2 + i] * kscore : -INFINITY;
        float tmax = fmaxf(x0, x1);
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
        const float mnew = fmaxf(m[nt][i], tmax);
        const float muse = (mnew == -INFINITY) ? 0.0f : mnew;
        alpha[i] = fast_exp2(m[nt][i] - muse);
        pv[i] = fast_exp2(x0 - muse);
        pv[2 + i] = fast_exp2(x1 - muse);
        l[nt][i] = l[nt][i] * alpha[i] + pv[i] + pv[2 + i];
        m[nt][i] = mnew;
      }
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        o[nt][kk][0] *= alpha[0];
        o[nt][kk][1] *= alpha[1];
        o[nt][kk][2] *= alpha[0];
        o[nt][kk][3] *= alpha[1];
      }
      // accumulator [tok][row] -> operand P^T [k = tok][n = row] via 8x8 transposes
      pb[nt][0] = movmatrix_t(KV8 ? pack_p_f16x2(pv[0], pv[1]) : pack_bf16x2(pv[0], pv[1]));
      pb[nt][1] = movmatrix_t(KV8 ? pack_p_f16x2(pv[2], pv[3]) : pack_bf16x2(pv[2], pv[3]));
    }
    // O^T += V^T P^T : [16 dims x 8 rows] per m-tile and n-tile.
    if constexpr (KV8) {
      // e4m3 V^T operands: lane (g, t4) reads token rows 2t4, 2t4+1, 2t4+8, 2t4+9 at dims
      // [HD/8 * g, HD/8 * (g + 1)) (rows outside the attended range as zeros); m-tile mt takes
      // dims HD/8 * g + 2mt (m row g) and + 1 (m row g + 8), and byte permutes pair the two
      // tokens of each k slot.  The stage is then free for its next chunk.
      constexpr int PV = HD / 128;  // 16-byte pieces per lane and row
      uint32_t vw[4][4 * PV];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int r = 2 * t4 + (q4 & 1) + 8 * (q4 >> 1);
        const int pos = c * kChunk + r;
        const bool ok = phys >= 0 && pos >= s_ci.lo && pos < s_ci.hi;
#pragma unroll
        for (int pi = 0; pi < PV; ++pi) {
          uint4 w = *reinterpret_cast<const uint4*>(vst + tile_off8(r, (HD / 8) * g + 16 * pi));
          if (!ok) w = make_uint4(0u, 0u, 0u, 0u);
          vw[q4][4 * pi + 0] = w.x;
          vw[q4][4 * pi + 1] = w.y;
          vw[q4][4 * pi + 2] = w.z;
          vw[q4][4 * pi + 3] = w.w;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && i + NS < nchunks) issue_chunk(i + NS);
#pragma unroll
      for (int mt = 0; mt < KT; ++mt) {
        const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;
        const uint32_t plo = __byte_perm(vw[0][mt >> 1], vw[1][mt >> 1], sel);
        const uint32_t phi = __byte_perm(vw[2][mt >> 1], vw[3][mt >> 1], sel);
        const uint32_t a0 = e4m3x2_to_f16x2(plo & 0xffffu), a1 = e4m3x2_to_f16x2(plo >> 16);
        const uint32_t a2 = e4m3x2_to_f16x2(phi & 0xffffu), a3 = e4m3x2_to_f16x2(phi >> 16);
        mma_f16(o[0][mt], a0, a1, a2, a3, pb[0][0], pb[0][1]);
      }
    } else if constexpr (kRowMask) {
      // Rows outside [lo, hi) of an edge stage (every row of a bad block, whose stage was
      // not loaded) may hold anything, NaN included; P is zero there, but 0 * NaN is not.
      if (partial) {
        const int pos = c * kChunk + (lane & 7) + ((lane >> 4) << 3);  // this lane's V row
        const bool row_ok = phys >= 0 && pos >= s_ci.lo && pos < s_ci.hi;
        pv_accumulate<KT, NT, true>(o, smem_u32(vst), lane, pb, row_ok, smem_u32(&s_zero_row));
      } else {
        pv_accumulate<KT, NT, false, KV8>(o, smem_u32(vst), lane, pb, true, 0u);
      }
    } else {
      const uint32_t vbase_s = smem_u32(vst);
      const int vr = (lane & 7) + ((lane >> 4) << 3), vd = ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vbase_s + tile_off(vr, kk * 16 + vd), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16<KV8>(o[nt][kk], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
      }
    }
    if constexpr (KV8) {
      // the stage was refilled after its dequantisation
    } else if (use_tma) {
      // This warp's reads (and writes) of the stage, ordered before the copy that refills it.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && i + NS < nchunks) issue_chunk(i + NS);
    } else {
      if (touched) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(stage));
    }
  }

  // Row sums: lanes with equal t4 hold disjoint token subsets of the same rows.
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float v = l[nt][i];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      l[nt][i] = v;
    }
  }  // tensor-core consumer

  if (failed && lane == 0) s_fail = 1;
  grid_launch_dependents();  // streaming is done: the next grid may start its prologue
  named_barrier_consumers();
  // Every chunk this CTA copied has been waited for by its consumer warp unless a wait gave
  // up; only then can copies still be in flight, and they must land before the ring's
  // shared memory is reused or released (the drain's waits are bounded too).
  if (s_fail) {
    if (tid == 0) {
      bool drained = true;
      for (int s = 0; s < NS && s < nchunks; ++s) {
        const int last = s + ((nchunks - 1 - s) / NS) * NS;
        if (!mbar_wait(full_bar(s), (last / NS) & 1)) drained = false;
      }
      if (!drained) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
    }
    named_barrier_consumers();
  }

  // ---- merge the four consumer warps (shared memory, aliasing the drained ring) ----
  constexpr int OST = HD + 4;  // padded row stride of the per-warp O buffers (floats)
  float* wo = reinterpret_cast<float*>(smem + L::kStages);  // [warps][ROWS][OST]
  if constexpr (FMA) {
    // Rows 0-3 only: the CUDA-core consumer serves at most 4 rows (nrows <= 4).
    const int r = lane >> 3;
    if ((lane & 7) == 0) {
      float mr = fst.m[0];
#pragma unroll
      for (int rr = 1; rr < 4; ++rr)
        if (rr == r) mr = fst.m[rr];
      s_wm[warp][r] = mr;
      s_wl[warp][r] = fst.l;
    }
#pragma unroll
    for (int rr = 0; rr < 4; ++rr)
      *reinterpret_cast<float4*>(wo + (warp * ROWS + rr) * OST + 4 * lane) =
          make_float4(fst.o[rr][0], fst.o[rr][1], fst.o[rr][2], fst.o[rr][3]);
  } else {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = nt * 8 + 2 * t4 + i;
      if (g == 0) {
        s_wm[warp][r] = m[nt][i];
        s_wl[warp][r] = l[nt][i];
      }
      float* dst = wo + (warp * ROWS + r) * OST;
      const float vsc = KV8 ? p.v_scale : 1.0f;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        if constexpr (KV8) {  // m-tile kk holds dims HD/8 * g + 2kk (+ 1)
          dst[(HD / 8) * g + 2 * kk] = o[nt][kk][i] * vsc;
          dst[(HD / 8) * g + 2 * kk + 1] = o[nt][kk][2 + i] * vsc;
        } else {
          dst[kk * 16 + g] = o[nt][kk][i];
          dst[kk * 16 + g + 8] = o[nt][kk][2 + i];
        }
      }
    }
  }
  named_barrier_consumers();

  // Items: (row, 8 consecutive dims).  Each thread merges its items across warps.
  constexpr int IPR = HD / 8;
  const int items = nrows * IPR;
  const bool single = sp.active == 1;
  const int64_t S = p.S;
  // Squares of the stored outputs (sumsq), after the warps' buffers in the drained ring.
  constexpr int kSvOff = (kConsumerWarps * ROWS * OST * 4 + 15) & ~15;
  static_assert(kSvOff + ROWS * (HD / 4) * 4 <= L::kRegion, "sumsq buffer fits the ring");
  float* sv = reinterpret_cast<float*>(smem + L::kStages + kSvOff);
  for (int it = tid; it < items; it += kConsumerWarps * 32) {
    const int r = it / IPR, k8 = it % IPR;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s_wm[w][r]);
    if (add_new) M = fmaxf(M, s_newm[r]);
    const float Muse = (M == -INFINITY) ? 0.0f : M;
    float Lsum = 0.0f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float wt = fast_exp2(s_wm[w][r] - Muse);
      Lsum += wt * s_wl[w][r];
      const float4* src = reinterpret_cast<const float4*>(wo + (w * ROWS + r) * OST + k8 * 8);
      const float4 a = src[0], b = src[1];
      acc[0] += wt * a.x; acc[1] += wt * a.y; acc[2] += wt * a.z; acc[3] += wt * a.w;
      acc[4] += wt * b.x; acc[5] += wt * b.y; acc[6] += wt * b.z; acc[7] += wt * b.w;
    }
    if (add_new) {
      // the new token's row: P = exp2(score - M), V from the registers' bf16 copy
      const float wt = fast_exp2(s_newm[r] - Muse);
      Lsum += wt;
      const __nv_bfloat16* vn = subkv + HD + k8 * 8;
      const float vsn = KV8 ? wt * p.v_scale : wt;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += vsn * __bfloat162float(vn[e]);
    }
    const int t = gstart + r / G;
    const int head = kvh * G + r % G;
    if (single) {
      const float inv = 1.0f / (Lsum > 0.0f ? Lsum : 1.0f);
      const int e0 = head * HD + k8 * 8;
      const float* gt = p.gate + int64_t(t) * Q + e0;
      float* out = p.out + int64_t(t) * Q + e0 / 8;
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float val = acc[e] * inv * gt[e];
        out[e * (Q / 8)] = val;
        ss += val * val;
      }
      if (SS) sv[it] = ss;  // item it = r * IPR + k8
    } else {
      const int64_t pi = (int64_t(t) * S + split) * p.NH + head;
      if (k8 == 0) p.pml[pi] = make_float2(M, Lsum);
      float4* dst = reinterpret_cast<float4*>(p.po + pi * HD + k8 * 8);
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  if (single) {
    if (SS) sumsq_tail<false>(p, sv, IPR, nrows, gstart, gcount, G, kvh, tid, s_rowss);
    return;
  }
  // ---- cross-split merge of this (group, KV head) ----
  // The barrier orders every consumer thread's partial stores before thread 0's release
  // (release is cumulative).
  named_barrier_consumers();
  if constexpr (DM) {
    // Designated merger (see one_wave: the grid is resident at once, or its mergers cannot
    // hold every slot): the last active split, which holds the newest positions and
    // usually finishes last, merges.  The others publish
    // their partials with a release add that they do not wait for, and exit; the merger
    // waits (bounded) for all of them with acquire loads, then resets the counter for the
    // next launch.  Its poll typically finds them done: no round trip of its own atomic.
    int32_t* counter = p.counters + gstart * p.NKV + kvh;
    if (split != sp.active - 1) {
      if (tid == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(counter) : "memory");
      return;
    }
    if (tid == 0) {
      int seen = 0;
      long long start = 0;
      for (;;) {
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(counter) : "memory");
        if (seen >= sp.active - 1) break;
        if (start == 0) start = clock64();
        else if (clock64() - start > kWaitLimitCycles) {
          record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
          break;
        }
      }
      *counter = 0;  // for the next launch (stream order puts it after this grid)
    }
    named_barrier_consumers();
  } else {
    // Otherwise: the last CTA of this (group, KV head) to arrive merges; its acquire,
    // passed on by the second barrier, makes the other CTAs' partials visible to it.
    if (tid == 0) {
      int32_t* counter = p.counters + gstart * p.NKV + kvh;
      int prev;
      asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
      s_last = (prev == sp.active - 1);
      if (s_last) *counter = 0;  // self-reset for the next launch
    }
    named_barrier_consumers();
    if (!s_last) return;
  }
  // Merge over the splits in registers, per (row, 4 dims) unit: batches of SB splits whose
  // (max, sum) and partial outputs are all in flight together (one L2 round trip per
  // batch; the gate rides along the first), each batch folded in with one max, independent
  // weights and one rescale.
  // Instances only for the unit counts this tile can reach (no dead register demand).
  constexpr int NTHR = kConsumerWarps * 32;
  constexpr int kMaxUnits = ROWS * (HD / 4);
  if (nrows * (HD / 4) <= NTHR) {
    merge_splits<HD, 1, 16, SS>(p, tid, nrows, gstart, kvh, G, sp.active, sv);
  } else if constexpr (kMaxUnits <= 2 * NTHR) {
    merge_splits_rows<HD, 2, 8, SS>(p, tid, nrows, gstart, kvh, G, sp.active, sv);
  } else {
    if (nrows * (HD / 4) <= 2 * NTHR)
      merge_splits_rows<HD, 2, 8, SS>(p, tid, nrows, gstart, kvh, G, sp.active, sv);
    else
      merge_splits_rows<HD, 4, 8, SS>(p, tid, nrows, gstart, kvh, G, sp.active, sv);
  }
  if (SS) sumsq_tail<false>(p, sv, HD / 4, nrows, gstart, gcount, G, kvh, tid, s_rowss);
}

// ------------------------------------------------------------------------------------
// Separate q/k normalisation and cache write (reference _qk_norm_cache_kernel,
// kernels/dory_attention.py:69-96): one warp per (token, head) row; q heads give the scaled
// bf16 query, k heads the normalised key written with the bf16 value at the token's slot (or
// to k_out / v_out).  Every load of a row is issued before its arithmetic.
// ------------------------------------------------------------------------------------
struct QkNormArgs {
  const float* qk;
  const float* v;
  const void* sqk;
  __nv_bfloat16* q_out;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  const int64_t* slot_mapping;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  uint32_t* err;
  int64_t sb, so, sh, ncache_blocks;
  float sqk_factor, eps;
  int NH, NKV, B, sqk_dtype, write_cache;
};

template <int HD>
__global__ void __launch_bounds__(128) qk_norm_kernel(const __grid_constant__ QkNormArgs a) {
  constexpr int PL = HD / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);  // head index: q heads, then k heads
  const int t = blockIdx.y;
  const int heads = a.NH + a.NKV;
  if (row >= heads) return;
  const int d0 = lane * PL;
  float x[PL], y[PL];
  const float* src = a.qk + (int64_t(t) * heads + row) * HD + d0;
#pragma unroll
  for (int i = 0; i < PL; ++i) x[i] = src[i];
  if (row < a.NH) {
#pragma unroll
    for (int i = 0; i < PL; ++i) y[i] = load_sqk(a.sqk, a.sqk_dtype, int64_t(row) * HD + d0 + i);
    const float rn = row_inv_norm<PL>(x, a.eps);
    __nv_bfloat16* dst = a.q_out + (int64_t(t) * a.NH + row) * HD + d0;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const float sq = __fmul_rn(y[i], a.sqk_factor);
      dst[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(sq, sq), __fmul_rn(x[i], rn)));
    }
    return;
  }
  const int kvh = row - a.NH;
  const float* vsrc = a.v + (int64_t(t) * a.NKV + kvh) * HD + d0;
#pragma unroll
  for (int i = 0; i < PL; ++i) y[i] = vsrc[i];
  const float rn = row_inv_norm<PL>(x, a.eps);
  __nv_bfloat16* kd;
  __nv_bfloat16* vd;
  if (a.write_cache) {
    const long long slot = a.slot_mapping[t];
    if (slot < 0) return;  // a padding token, which vLLM does not cache
    const long long blk = slot / a.B;
    if (a.ncache_blocks > 0 && blk >= a.ncache_blocks) {
      if (lane == 0 && a.err) record_error(a.err, DORY_DEVERR_SLOT_OOB);
      return;
    }
    const long long base = blk * a.sb + (slot % a.B) * a.so + (long long)kvh * a.sh + d0;
    kd = a.kc + base;
    vd = a.vc + base;
  } else {
    kd = a.k_out + (int64_t(t) * a.NKV + kvh) * HD + d0;
    vd = a.v_out + (int64_t(t) * a.NKV + kvh) * HD + d0;
  }
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    kd[i] = __float2bfloat16_rn(__fmul_rn(x[i], rn));
    vd[i] = __float2bfloat16_rn(y[i]);
  }
}

// ------------------------------------------------------------------------------------
// The multi-token path's q/k/v/gate epilogue as its own launch (reference
// _qkvg_epilogue_kernel, kernels/dory_multi_token.py:53-80): grid (rows / HD, T), one thread
// per pair of rows.  The split-K sum in order from zero, the rotary products and sums
// rounded one by one (no fused multiply-add), the gate as sigmoid((y * s) * s).
// ------------------------------------------------------------------------------------
struct QkvgArgs {
  const float* partials;
  const void* positions;
  const void* cos_sin;
  const void* s_gate;
  float* qk;
  float* v;
  float* gate;
  uint32_t* err;
  float s_gate_factor;
  int T, NH, NKV, split_k, max_position, pos_dtype, cos_dtype, sgate_dtype;
};

template <int HD>
__global__ void __launch_bounds__(HD / 2) qkvg_epilogue_kernel(const __grid_constant__ QkvgArgs a) {
  constexpr int HALF = HD / 2;
  // Programmatic dependent launch (no-ops otherwise): the partials are read after the
  // previous grid; the next grid (an overlapped attention call, whose consumers wait for
  // this grid to complete before reading qk / v / gate) may start at once.
  grid_dependency_wait();
  grid_launch_dependents();
  const int b = blockIdx.x, t = blockIdx.y, i = threadIdx.x;
  const int64_t prow = 2 * int64_t(a.NH + a.NKV) * HD;
  const int64_t row = int64_t(b) * HD + 2 * i;
  float y0 = 0.0f, y1 = 0.0f;
  for (int k = 0; k < a.split_k; ++k) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(a.partials + (int64_t(k) * a.T + t) * prow + row));
    y0 = __fadd_rn(y0, v.x);
    y1 = __fadd_rn(y1, v.y);
  }
  if (b < a.NH + a.NKV) {  // q or k head b: rows 2i, 2i + 1 are rotary dims i, i + HALF
    const int64_t pos = a.pos_dtype == 0 ? static_cast<const int64_t*>(a.positions)[t]
                                         : int64_t(static_cast<const int32_t*>(a.positions)[t]);
    float lo = 0.0f, hi = 0.0f;
    if (pos >= 0 && pos < a.max_position) {
      const float c = load_sqk(a.cos_sin, a.cos_dtype, pos * HD + i);
      const float sn = load_sqk(a.cos_sin, a.cos_dtype, pos * HD + HALF + i);
      lo = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
      hi = __fadd_rn(__fmul_rn(y1, c), __fmul_rn(y0, sn));
    } else if (a.err && i == 0) {
      atomicOr(a.err, DORY_DEVERR_POSITION_OOB);
    }
    float* q = a.qk + int64_t(t) * (a.NH + a.NKV) * HD + int64_t(b) * HD;
    q[i] = lo;
    q[i + HALF] = hi;
  } else if (b < a.NH + 2 * a.NKV) {
    float* v = a.v + int64_t(t) * a.NKV * HD + int64_t(b - a.NH - a.NKV) * HD + 2 * i;
    v[0] = y0;
    v[1] = y1;
  } else {
    const int e = (b - a.NH - 2 * a.NKV) * HD + 2 * i;
    float g[2];
    const float y[2] = {y0, y1};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float s = __fmul_rn(load_sqk(a.s_gate, a.sgate_dtype, e + j), a.s_gate_factor);
      const float z = __fmul_rn(__fmul_rn(y[j], s), s);
      g[j] = 1.0f / (1.0f + expf(-z));
    }
    float* gp = a.gate + int64_t(t) * a.NH * HD + e;
    gp[0] = g[0];
    gp[1] = g[1];
  }
}

// ------------------------------------------------------------------------------------
// The residual update after a sublayer's output GEMV (reference _residual_tokens_kernel,
// kernels/dory_multi_token.py:109-131, and residual_update, kernels/dory_common.py:55-81):
// one CTA per token; thread w owns hidden elements 8w .. 8w + 7 (G = 4 groups of them, 512
// threads at most, when the hidden size exceeds 8192), which gives one 16-byte natural-order BF16 store and eight
// coalesced nibble-major stores per group.
//   b = (0 + p_0 + ... + p_{k-1}) * r_x, r_x = 1 / sqrt(sum x^2 + eps)  (1 without x)
//   h = n(n(a) + |alpha * alpha_scale| * (n(b) - n(a)))
// Every sum of squares is taken in FP64 and rounded once (inv_norm_from_sum); products and
// sums are rounded one by one.  All global loads are issued before the first barrier.
// ------------------------------------------------------------------------------------
struct ResidualArgs {
  const float* partials;
  const float* x;
  const float* x_sumsq;
  const void* a;
  const void* alpha;
  __nv_bfloat16* h;
  float* h_nm;
  float alpha_scale, eps;
  int T, H, K_IN, split_k, a_dtype, alpha_dtype;
};

// Eight consecutive elements [i, i + 8) of an FP32 / BF16 / FP16 array (16-byte aligned).
__device__ __forceinline__ void load8(const void* p, int dtype, int64_t i, float (&out)[8]) {
  if (dtype == DORY_DTYPE_F32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 u0 = __ldg(q), u1 = __ldg(q + 1);
    out[0] = u0.x; out[1] = u0.y; out[2] = u0.z; out[3] = u0.w;
    out[4] = u1.x; out[5] = u1.y; out[6] = u1.z; out[7] = u1.w;
    return;
  }
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (dtype == DORY_DTYPE_BF16) {
      out[2 * j] = __uint_as_float(w[j] << 16);
      out[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    } else {
      out[2 * j] = __half2float(__ushort_as_half(uint16_t(w[j] & 0xffffu)));
      out[2 * j + 1] = __half2float(__ushort_as_half(uint16_t(w[j] >> 16)));
    }
  }
}

// Sum over the CTA of N doubles; every thread gets the same totals (warps added in order).
template <int N>
__device__ __forceinline__ void block_sum(double (&v)[N], double* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int n = 0; n < N; ++n)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v[n] += __shfl_xor_sync(0xffffffffu, v[n], off);
  __syncthreads();  // the previous sum's readers are done with s_red
  if (lane == 0)
#pragma unroll
    for (int n = 0; n < N; ++n) s_red[warp * N + n] = v[n];
  __syncthreads();
#pragma unroll
  for (int n = 0; n < N; ++n) {
    double s = 0.0;
    for (int w = 0; w < nwarps; ++w) s += s_red[w * N + n];
    v[n] = s;
  }
}

template <int G>
__global__ void __launch_bounds__(G == 1 ? 1024 : 512) residual_kernel(const __grid_constant__ ResidualArgs a) {
  __shared__ double s_red[32 * 2];
  // Programmatic dependent launch (no-ops otherwise): inputs are read after the previous
  // grid; a dependent grid may start at once (it waits for this grid before reading h).
  grid_dependency_wait();
  grid_launch_dependents();
  const int t = blockIdx.x, tid = threadIdx.x, nthr = blockDim.x, W = a.H >> 3;
  float b[G][8], av[G][8];
  double sx = 0.0;
  // this thread's groups: split-K sum in order from zero, the sublayer input
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int w = tid + g * nthr;
#pragma unroll
    for (int j = 0; j < 8; ++j) b[g][j] = av[g][j] = 0.0f;
    if (w < W) {
      const int64_t e = int64_t(t) * a.H + 8 * w;
      for (int k = 0; k < a.split_k; ++k) {
        const float4* p = reinterpret_cast<const float4*>(a.partials + int64_t(k) * a.T * a.H + e);
        const float4 u0 = __ldg(p), u1 = __ldg(p + 1);
        const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) b[g][j] = __fadd_rn(b[g][j], u[j]);
      }
      load8(a.a, a.a_dtype, e, av[g]);
    }
  }
  // the GEMV input's sum of squares
  if (a.x) {
    const float* x = a.x + int64_t(t) * a.K_IN;
    if ((a.K_IN & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      for (int i = tid; i < (a.K_IN >> 2); i += nthr) {
        const float4 u = __ldg(x4 + i);
        sx += double(u.x) * u.x + double(u.y) * u.y + double(u.z) * u.z + double(u.w) * u.w;
      }
    } else {
      for (int i = tid; i < a.K_IN; i += nthr) {
        const float u = __ldg(x + i);
        sx += double(u) * u;
      }
    }
  }
  float r_x = 1.0f;
  if (a.x) {
    double v[1] = {sx};
    block_sum<1>(v, s_red);
    r_x = inv_norm_from_sum(v[0], a.eps);
  } else if (a.x_sumsq) {
    r_x = inv_norm_from_sum(double(__ldg(a.x_sumsq + t)), a.eps);
  }
  double s2[2] = {0.0, 0.0};
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      b[g][j] = __fmul_rn(b[g][j], r_x);
      s2[0] += double(av[g][j]) * av[g][j];
      s2[1] += double(b[g][j]) * b[g][j];
    }
  block_sum<2>(s2, s_red);
  const float ra = inv_norm_from_sum(s2[0], a.eps), rb = inv_norm_from_sum(s2[1], a.eps);
  double sz[1] = {0.0};
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int w = tid + g * nthr;
    float al[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) al[j] = 0.0f;
    if (w < W) load8(a.alpha, a.alpha_dtype, 8 * int64_t(w), al);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float lr = fabsf(__fmul_rn(al[j], a.alpha_scale));
      const float ya = __fmul_rn(av[g][j], ra), yb = __fmul_rn(b[g][j], rb);
      const float z = __fadd_rn(ya, __fmul_rn(lr, __fsub_rn(yb, ya)));
      b[g][j] = z;
      sz[0] += double(z) * z;
    }
  }
  block_sum<1>(sz, s_red);
  const float rz = inv_norm_from_sum(sz[0], a.eps);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int w = tid + g * nthr;
    if (w >= W) continue;
    float hv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) hv[j] = __fmul_rn(b[g][j], rz);
    const int64_t e = int64_t(t) * a.H + 8 * w;
    uint4 packed;
    packed.x = pack_bf16x2(hv[0], hv[1]);
    packed.y = pack_bf16x2(hv[2], hv[3]);
    packed.z = pack_bf16x2(hv[4], hv[5]);
    packed.w = pack_bf16x2(hv[6], hv[7]);
    *reinterpret_cast<uint4*>(a.h + e) = packed;
    float* nm = a.h_nm + int64_t(t) * a.H + w;
#pragma unroll
    for (int j = 0; j < 8; ++j) nm[int64_t(j) * W] = hv[j];
  }
}

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------
thread_local char g_last_error[512] = "";

int32_t fail(int32_t status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

template <int HD, int NT, int NS, bool SS, bool DM, bool FMA = false, bool KV8 = false,
          bool WIDE = false, bool SHK = false>
int32_t launch(const KParams& kp, dim3 grid, int smem_bytes, cudaStream_t stream) {
  auto fn = decode_kernel<HD, NT, NS, SS, DM, FMA, KV8, WIDE, SHK>;
  static int configured[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(DORY_ERR_CUDA, "cudaGetDevice failed");
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    // The largest dynamic size any call of this instantiation can ask for.
    const int max_bytes = Smem<HD, NS, KV8>::bytes(kMaxSub);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes);
    if (e != cudaSuccess)
      return fail(DORY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = size_t(smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = kp.overlap ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, kp);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return DORY_OK;
}

int sm_count();

// Whether the designated-merger scheme may run `grid` CTAs of `fn` with `smem` bytes of
// dynamic shared memory (occupancy per SM x SMs = the resident slots, cached per kernel and
// size).  Only the mergers wait, one per (token, KV head): the others always run to their
// end.  So the grid cannot stall when the whole grid is resident at once, or when the
// mergers alone (grid.y x grid.z at most) leave a slot free, through which every sibling a
// merger waits for is eventually dispatched (a programmatic dependent grid is launched only
// once every CTA of the previous one has started, so its CTAs never hold slots that one
// still needs).
template <typename F>
bool one_wave(F fn, dim3 grid, int smem, int max_smem) {
  struct Entry {
    const void* fn;
    int dev, smem, per_sm;
  };
  static Entry cache[64];
  static int used = 0;
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const long long ctas = (long long)grid.x * grid.y * grid.z;
  const long long mergers = (long long)grid.y * grid.z;
  auto fits = [&](int per_sm) {
    const long long slots = (long long)per_sm * sm_count();
    return ctas <= slots || mergers < slots;
  };
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == (const void*)fn && cache[i].dev == dev && cache[i].smem == smem)
      return fits(cache[i].per_sm);
  int per_sm = 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           max_smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem) != cudaSuccess)
    per_sm = 0;
  cudaGetLastError();
  if (used < 64) cache[used++] = Entry{(const void*)fn, dev, smem, per_sm};
  return fits(per_sm);
}

// Ring stages per instantiation: a multiple of the four consumer warps, so every stage keeps
// one consumer, which refills it; two stages per warp let each warp compute one chunk while
// its next one is in flight (64 KB of ring for 128-dim heads at 3 CTAs/SM; 128 KB for
// 256-dim heads, which run one CTA per SM).
template <int HD, int NT>
struct Depth {
  static constexpr int value = 8;
  // Required, not a tuning choice: with another count, the warp that refills stage s is not
  // the one that reads its next occupant, so a warp can wait on a stage two phases ahead of
  // the copy still landing there, which a parity wait cannot tell apart.
  static_assert(value % kConsumerWarps == 0, "ring stages must be a multiple of the consumer warps");
};

template <int HD, int NT>
int32_t dispatch(const KParams& kp, dim3 grid, cudaStream_t stream) {
  constexpr int NS = Depth<HD, NT>::value;
  static_assert(kConsumerWarps * NT * 8 * (HD + 4) * 4 <= NS * Smem<HD, NS>::kStageBytes,
                "the warps' merge buffer must fit in the ring");
  const int smem = Smem<HD, NS>::bytes(kp.nsub);
  // The designated merger waits for the other splits of its (group, KV head) to finish:
  // only when every CTA of the grid is resident at once, so that none of them can be
  // waiting for a slot the merger holds.
  const bool dm = one_wave(decode_kernel<HD, NT, NS, false, true>, grid, smem,
                           Smem<256, 8>::bytes(kMaxSub));
  // The sum-of-squares epilogue is a separate instantiation: compiled in, even unused, it
  // measured ~0.5 us slower on single-sequence calls.
  if (kp.sumsq)
    return dm ? launch<HD, NT, NS, true, true>(kp, grid, smem, stream)
              : launch<HD, NT, NS, true, false>(kp, grid, smem, stream);
  return dm ? launch<HD, NT, NS, false, true>(kp, grid, smem, stream)
            : launch<HD, NT, NS, false, false>(kp, grid, smem, stream);
}

// The CUDA-core consumer (DORY_FLAG_FMA_CONSUMER): 128-dim heads, one tile of at most 4
// rows; the same ring, prologue, merge and launch rules as the tensor-core kernel.
int32_t dispatch_fma(const KParams& kp, dim3 grid, cudaStream_t stream) {
  constexpr int NS = Depth<128, 1>::value;
  const int smem = Smem<128, NS>::bytes(kp.nsub);
  const bool dm = one_wave(decode_kernel<128, 1, NS, false, true, true>, grid, smem,
                           Smem<256, 8>::bytes(kMaxSub));
  if (kp.sumsq)
    return dm ? launch<128, 1, NS, true, true, true>(kp, grid, smem, stream)
              : launch<128, 1, NS, true, false, true>(kp, grid, smem, stream);
  return dm ? launch<128, 1, NS, false, true, true>(kp, grid, smem, stream)
            : launch<128, 1, NS, false, false, true>(kp, grid, smem, stream);
}

// FP8 (e4m3) caches: one 8-row tile and the FP8 ring.  A 16-row FP8 chunk carries half a
// bf16 chunk's bytes; 8 stages (32 KB for 128-dim heads) measured best (12 and 16 a little
// slower, 24 much slower: 2 CTAs per SM).
#ifndef DORY_KV8_STAGES
#define DORY_KV8_STAGES 8
#endif
constexpr int kStagesKV8 = DORY_KV8_STAGES;
#ifndef DORY_KV8_WIDE_WAVES
#define DORY_KV8_WIDE_WAVES 2
#endif
constexpr int kWideWaves = DORY_KV8_WIDE_WAVES;
template <int HD>
int32_t dispatch_kv8(const KParams& kp, dim3 grid, cudaStream_t stream) {
  constexpr int NS = kStagesKV8;
  static_assert(NS % kConsumerWarps == 0, "ring stages must be a multiple of the consumer warps");
  static_assert(kConsumerWarps * 8 * (HD + 4) * 4 <= Smem<HD, NS, true>::kRegion,
                "the warps' merge buffer must fit in the ring");
  const int smem = Smem<HD, NS, true>::bytes(kp.nsub);
  if (kp.shared) {
    const bool dm = one_wave(decode_kernel<HD, 1, NS, false, true, false, true, false, true>,
                             grid, smem, Smem<HD, NS, true>::bytes(kMaxSub));
    if (kp.sumsq)
      return dm ? launch<HD, 1, NS, true, true, false, true, false, true>(kp, grid, smem, stream)
                : launch<HD, 1, NS, true, false, false, true, false, true>(kp, grid, smem, stream);
    return dm ? launch<HD, 1, NS, false, true, false, true, false, true>(kp, grid, smem, stream)
              : launch<HD, 1, NS, false, false, false, true, false, true>(kp, grid, smem, stream);
  }
  const bool dm = one_wave(decode_kernel<HD, 1, NS, false, true, false, true>, grid, smem,
                           Smem<HD, NS, true>::bytes(kMaxSub));
  if constexpr (HD == 128) {
    // Grids of at least kWideWaves waves of 4 CTAs per SM (large batches) take the 4-CTA
    // build.
    const long long ctas = (long long)grid.x * grid.y * grid.z;
    if (!dm && ctas >= (long long)kWideWaves * 4 * sm_count())
      return kp.sumsq ? launch<HD, 1, NS, true, false, false, true, true>(kp, grid, smem, stream)
                      : launch<HD, 1, NS, false, false, false, true, true>(kp, grid, smem, stream);
  }
  if (kp.sumsq)
    return dm ? launch<HD, 1, NS, true, true, false, true>(kp, grid, smem, stream)
              : launch<HD, 1, NS, true, false, false, true>(kp, grid, smem, stream);
  return dm ? launch<HD, 1, NS, false, true, false, true>(kp, grid, smem, stream)
            : launch<HD, 1, NS, false, false, false, true>(kp, grid, smem, stream);
}

template <int HD>
int32_t dispatch_nt(const KParams& kp, int nt, dim3 grid, cudaStream_t stream) {
  if (nt == 1) return dispatch<HD, 1>(kp, grid, stream);
  if constexpr (HD <= 128) return dispatch<HD, 2>(kp, grid, stream);
  return fail(DORY_ERR_UNSUPPORTED, "head_dim %d supports at most 8 query rows per tile", HD);
}

// ---- tensor maps of the cache views ----
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapKey {
  const void* base;
  int64_t blocks, sb, so, sh;
  int B, NKV, quarters;
  int esize;  // bytes per element: 2 (bf16), 1 (e4m3)
  bool operator==(const MapKey& o) const {
    return base == o.base && blocks == o.blocks && sb == o.sb && so == o.so && sh == o.sh &&
           B == o.B && NKV == o.NKV && quarters == o.quarters && esize == o.esize;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool ok;
};

// 5-D map of a cache view: (64 dims, rows of a block, 64-dim quarters of a row [stride 128
// bytes], KV head, block); box 64 x 16 x quarters x 1 x 1 with 128-byte swizzle, so one
// copy lands a chunk's tile as `quarters` swizzled [16][64] boxes.  quarters = HD / 64 for
// a K or V tile, twice that for K and V together when V directly follows K.  Encoded maps
// are cached per thread (a call sequence revisits the same few caches).
bool cache_tensor_map(const MapKey& k, CUtensorMap* out) {
  constexpr int kSlots = 64;
  thread_local MapEntry cache[kSlots];
  thread_local int used = 0, next = 0;
  for (int i = 0; i < used; ++i)
    if (cache[i].key == k) {
      *out = cache[i].map;
      return cache[i].ok;
    }
  MapEntry e;
  e.key = k;
  e.ok = false;
  memset(&e.map, 0, sizeof(e.map));
  auto encode = tensor_map_encoder();
  if (encode && k.blocks > 0 && k.blocks <= 0x7fffffff && k.quarters <= 8) {
    // 128-byte rows of the box: 64 bf16 dims, or 128 e4m3 dims ("quarters" then counts
    // 128-dim pieces)
    const cuuint64_t inner = 128 / k.esize, es = cuuint64_t(k.esize);
    cuuint64_t dims[5] = {inner, cuuint64_t(k.B), cuuint64_t(k.quarters), cuuint64_t(k.NKV),
                          cuuint64_t(k.blocks)};
    cuuint64_t strides[4] = {cuuint64_t(k.so) * es, 128, cuuint64_t(k.sh) * es,
                             cuuint64_t(k.sb) * es};
    cuuint32_t box[5] = {cuuint32_t(inner), cuuint32_t(kChunk), cuuint32_t(k.quarters), 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = encode(&e.map, k.esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        5, const_cast<void*>(k.base),
                        dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    e.ok = r == CUDA_SUCCESS;
  }
  if (used < kSlots) {
    cache[used++] = e;
  } else {
    cache[next] = e;
    next = (next + 1) % kSlots;
  }
  *out = e.map;
  return e.ok;
}

// Streaming multiprocessors of the current device (cached per device ordinal).
int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

}  // namespace

extern "C" {

int32_t dory_decode_abi_version(void) { return DORY_DECODE_ABI_VERSION; }

int64_t dory_decode_params_bytes(void) { return int64_t(sizeof(DoryDecodeParams)); }

int64_t dory_decode_scratch_bytes(int32_t max_tokens, int32_t splits, int32_t num_heads,
                                  int32_t num_kv_heads, int32_t head_dim) {
  ScratchLayout SL;
  if (!scratch_layout_checked(max_tokens, splits, num_heads, num_kv_heads, head_dim, &SL)) return 0;
  return SL.total;
}

int32_t dory_decode_scratch_init(void* scratch, int64_t scratch_bytes, void* stream) {
  if (!scratch || scratch_bytes <= 0) return fail(DORY_ERR_INVALID_ARGUMENT, "null scratch");
  cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(scratch_bytes), (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return DORY_OK;
}

int32_t dory_decode_fetch_errors(void* scratch, uint32_t* flags_out, int32_t clear, void* stream) {
  if (!scratch || !flags_out) return fail(DORY_ERR_INVALID_ARGUMENT, "null argument");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(flags_out, scratch, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(scratch, 0, 4, s);
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "fetch errors: %s", cudaGetErrorString(e));
  return DORY_OK;
}

const char* dory_decode_last_error(void) { return g_last_error; }

int64_t dory_qk_norm_params_bytes(void) { return int64_t(sizeof(DoryQkNormParams)); }

int64_t dory_qkvg_params_bytes(void) { return int64_t(sizeof(DoryQkvgParams)); }

int32_t dory_qkvg_epilogue(const DoryQkvgParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  const DoryQkvgParams& a = *P;
  if (a.num_tokens < 0 || a.num_heads < 1 || a.num_kv_heads < 1 || a.split_k < 1 ||
      a.max_position < 1)
    return fail(DORY_ERR_INVALID_ARGUMENT, "counts must be positive");
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256)
    return fail(DORY_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128, 256)", a.head_dim);
  if (a.positions_dtype < 0 || a.positions_dtype > 1 || a.cos_sin_dtype < 0 ||
      a.cos_sin_dtype > 2 || a.s_gate_dtype < 0 || a.s_gate_dtype > 2)
    return fail(DORY_ERR_INVALID_ARGUMENT, "positions / cos_sin / s_gate dtype");
  if (!a.partials || !a.positions || !a.cos_sin || !a.s_gate || !a.qk_out || !a.v_out ||
      !a.gate_out)
    return fail(DORY_ERR_INVALID_ARGUMENT, "null tensor argument");
  if (reinterpret_cast<uintptr_t>(a.partials) & 15)
    return fail(DORY_ERR_ALIGNMENT, "partials need a 16-byte aligned base");
  if (a.num_tokens == 0) return DORY_OK;
  QkvgArgs k;
  memset(&k, 0, sizeof(k));
  k.partials = a.partials;
  k.positions = a.positions;
  k.cos_sin = a.cos_sin;
  k.s_gate = a.s_gate;
  k.qk = a.qk_out;
  k.v = a.v_out;
  k.gate = a.gate_out;
  k.err = a.error_word;
  k.s_gate_factor = a.s_gate_factor;
  k.T = a.num_tokens;
  k.NH = a.num_heads;
  k.NKV = a.num_kv_heads;
  k.split_k = a.split_k;
  k.max_position = a.max_position;
  k.pos_dtype = a.positions_dtype;
  k.cos_dtype = a.cos_sin_dtype;
  k.sgate_dtype = a.s_gate_dtype;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * (a.num_heads + a.num_kv_heads), a.num_tokens);
  cfg.blockDim = dim3(a.head_dim / 2);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (a.flags & DORY_FLAG_OVERLAP_LAUNCH) ? 1 : 0;
  cudaError_t e;
  if (a.head_dim == 64) e = cudaLaunchKernelEx(&cfg, qkvg_epilogue_kernel<64>, k);
  else if (a.head_dim == 128) e = cudaLaunchKernelEx(&cfg, qkvg_epilogue_kernel<128>, k);
  else e = cudaLaunchKernelEx(&cfg, qkvg_epilogue_kernel<256>, k);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return DORY_OK;
}

int64_t dory_residual_params_bytes(void) { return int64_t(sizeof(DoryResidualParams)); }

int32_t dory_residual_update(const DoryResidualParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  const DoryResidualParams& a = *P;
  if (a.num_tokens < 0 || a.split_k < 1)
    return fail(DORY_ERR_INVALID_ARGUMENT, "num_tokens must be >= 0 and split_k >= 1");
  if (a.hidden < 8 || a.hidden % 8)
    return fail(DORY_ERR_INVALID_ARGUMENT, "hidden %d is not a positive multiple of 8", a.hidden);
  if (a.hidden > 16384)
    return fail(DORY_ERR_UNSUPPORTED, "hidden %d (supported: up to 16384)", a.hidden);
  if (a.a_dtype < 0 || a.a_dtype > 2 || a.alpha_dtype < 0 || a.alpha_dtype > 2)
    return fail(DORY_ERR_INVALID_ARGUMENT, "a / alpha dtype");
  if (a.x && a.x_sumsq) return fail(DORY_ERR_INVALID_ARGUMENT, "give x or x_sumsq, not both");
  if (a.x && a.x_dim < 1) return fail(DORY_ERR_INVALID_ARGUMENT, "x_dim must be positive");
  if (a.num_tokens == 0) return DORY_OK;  // nothing is read: empty tensors may be NULL
  if (!a.partials || !a.a || !a.alpha || !a.h_out || !a.h_out_nibble_major)
    return fail(DORY_ERR_INVALID_ARGUMENT, "null tensor argument");
  const void* aligned[] = {a.partials, a.a, a.alpha, a.h_out, a.h_out_nibble_major};
  for (const void* q : aligned)
    if (reinterpret_cast<uintptr_t>(q) & 15)
      return fail(DORY_ERR_ALIGNMENT, "partials, a, alpha and the outputs need 16-byte aligned bases");
  // The outputs must not overlap the inputs the CTAs of other tokens still read (the
  // reference's residual_update refuses an h_out aliasing a, dory_common.py:74-75).
  const int64_t n = int64_t(a.num_tokens) * a.hidden;
  const int64_t a_bytes = n * (a.a_dtype == DORY_DTYPE_F32 ? 4 : 2);
  auto overlap = [](const void* p, int64_t pn, const void* q, int64_t qn) {
    const uintptr_t p0 = reinterpret_cast<uintptr_t>(p), q0 = reinterpret_cast<uintptr_t>(q);
    return pn > 0 && qn > 0 && p0 < q0 + uint64_t(qn) && q0 < p0 + uint64_t(pn);
  };
  if (overlap(a.h_out, n * 2, a.a, a_bytes) || overlap(a.h_out_nibble_major, n * 4, a.a, a_bytes) ||
      overlap(a.h_out, n * 2, a.partials, n * 4 * a.split_k) ||
      overlap(a.h_out_nibble_major, n * 4, a.partials, n * 4 * a.split_k))
    return fail(DORY_ERR_INVALID_ARGUMENT, "the outputs must not alias the sublayer input or the partials");
  ResidualArgs k;
  memset(&k, 0, sizeof(k));
  k.partials = a.partials;
  k.x = a.x;
  k.x_sumsq = a.x_sumsq;
  k.a = a.a;
  k.alpha = a.alpha;
  k.h = static_cast<__nv_bfloat16*>(a.h_out);
  k.h_nm = a.h_out_nibble_major;
  k.alpha_scale = a.alpha_scale;
  k.eps = a.eps;
  k.T = a.num_tokens;
  k.H = a.hidden;
  k.K_IN = a.x ? a.x_dim : 0;
  k.split_k = a.split_k;
  k.a_dtype = a.a_dtype;
  k.alpha_dtype = a.alpha_dtype;
  const int groups = a.hidden / 8;
  const int G = groups > 1024 ? 4 : 1;
  const int threads = ((groups + G - 1) / G + 31) / 32 * 32;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(a.num_tokens);
  cfg.blockDim = dim3(threads);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (a.flags & DORY_FLAG_OVERLAP_LAUNCH) ? 1 : 0;
  cudaError_t e = G == 1 ? cudaLaunchKernelEx(&cfg, residual_kernel<1>, k)
                         : cudaLaunchKernelEx(&cfg, residual_kernel<4>, k);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return DORY_OK;
}

int32_t dory_qk_norm_cache(const DoryQkNormParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  const DoryQkNormParams& a = *P;
  const bool write_cache = a.flags & DORY_QKNORM_WRITE_CACHE;
  if (a.num_tokens < 0 || a.num_heads < 1 || a.num_kv_heads < 1)
    return fail(DORY_ERR_INVALID_ARGUMENT, "token and head counts must be positive");
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256)
    return fail(DORY_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128, 256)", a.head_dim);
  if (a.sqk_dtype < 0 || a.sqk_dtype > 2) return fail(DORY_ERR_INVALID_ARGUMENT, "sqk dtype");
  if (!a.qk || !a.v || !a.sqk || !a.q_out)
    return fail(DORY_ERR_INVALID_ARGUMENT, "null tensor argument");
  if (write_cache && (!a.key_cache || !a.value_cache || !a.slot_mapping || a.block_size < 1))
    return fail(DORY_ERR_INVALID_ARGUMENT, "the cache write needs caches, a slot mapping and a block size");
  if (!write_cache && (!a.k_out || !a.v_out))
    return fail(DORY_ERR_INVALID_ARGUMENT, "k_out and v_out are needed without the cache write");
  if (a.num_tokens == 0) return DORY_OK;
  QkNormArgs k;
  memset(&k, 0, sizeof(k));
  k.qk = a.qk;
  k.v = a.v;
  k.sqk = a.sqk;
  k.q_out = static_cast<__nv_bfloat16*>(a.q_out);
  k.kc = static_cast<__nv_bfloat16*>(a.key_cache);
  k.vc = static_cast<__nv_bfloat16*>(a.value_cache);
  k.slot_mapping = a.slot_mapping;
  k.k_out = static_cast<__nv_bfloat16*>(a.k_out);
  k.v_out = static_cast<__nv_bfloat16*>(a.v_out);
  k.err = a.error_word;
  k.sb = a.stride_block;
  k.so = a.stride_offset;
  k.sh = a.stride_head;
  k.ncache_blocks = a.num_cache_blocks;
  k.sqk_factor = a.sqk_factor;
  k.eps = a.eps;
  k.NH = a.num_heads;
  k.NKV = a.num_kv_heads;
  k.B = a.block_size;
  k.sqk_dtype = a.sqk_dtype;
  k.write_cache = write_cache;
  const dim3 grid((a.num_heads + a.num_kv_heads + 3) / 4, a.num_tokens);
  cudaStream_t s = (cudaStream_t)stream;
  if (a.head_dim == 64) qk_norm_kernel<64><<<grid, 128, 0, s>>>(k);
  else if (a.head_dim == 128) qk_norm_kernel<128><<<grid, 128, 0, s>>>(k);
  else qk_norm_kernel<256><<<grid, 128, 0, s>>>(k);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return DORY_OK;
}

int32_t dory_decode_attention(const DoryDecodeParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  const DoryDecodeParams& a = *P;
  if (a.num_heads < 1 || a.num_kv_heads < 1 || a.num_heads % a.num_kv_heads)
    return fail(DORY_ERR_INVALID_ARGUMENT, "query heads must be a multiple of KV heads");
  const bool raw = a.flags & DORY_FLAG_RAW_QKV;
  const bool multi = a.flags & DORY_FLAG_MULTI_TOKEN;
  const bool shared = a.flags & DORY_FLAG_SHARED_CACHE;
  const bool overlap = a.flags & DORY_FLAG_OVERLAP_LAUNCH;
  const bool fma = a.flags & DORY_FLAG_FMA_CONSUMER;
  if (a.kv_dtype != 0 && a.kv_dtype != DORY_DTYPE_BF16 && a.kv_dtype != DORY_DTYPE_FP8_E4M3)
    return fail(DORY_ERR_INVALID_ARGUMENT, "kv_dtype %d (bf16 or fp8 e4m3)", a.kv_dtype);
  const bool kv8 = a.kv_dtype == DORY_DTYPE_FP8_E4M3;
  if (a.num_tokens < 0) return fail(DORY_ERR_INVALID_ARGUMENT, "negative token count");
  if (a.num_tokens > a.max_tokens)
    return fail(DORY_ERR_INVALID_ARGUMENT, "too many tokens for the scratch buffers");
  if (!multi && a.num_tokens != 1)
    return fail(DORY_ERR_INVALID_ARGUMENT, "single-token calls take exactly one token");
  if (shared && !(multi && raw))
    return fail(DORY_ERR_INVALID_ARGUMENT, "shared_cache needs a raw multi-token call");
  if (multi && (!a.cache_offsets || !a.block_table_offsets))
    return fail(DORY_ERR_INVALID_ARGUMENT, "multi-token calls need int64 cache/table offsets");
  if (raw && (!a.v || !a.sqk || (!multi && !a.slot_mapping)))
    return fail(DORY_ERR_INVALID_ARGUMENT, "raw calls need v, sqk and a slot mapping");
  if (!a.q || !a.key_cache || !a.value_cache || !a.block_table || !a.seq_lens || !a.gate ||
      !a.out_nibble_major || !a.scratch)
    return fail(DORY_ERR_INVALID_ARGUMENT, "null tensor argument");
  if (a.splits < 1 || a.blocks_per_tile < 1)
    return fail(DORY_ERR_INVALID_ARGUMENT, "splits and blocks_per_tile must be positive");
  if (a.window < 0) return fail(DORY_ERR_INVALID_ARGUMENT, "negative window");
  const int HD = a.head_dim;
  if (HD != 64 && HD != 128 && HD != 256)
    return fail(DORY_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128, 256)", HD);
  if (a.block_size < 16 || a.block_size % 16)
    return fail(DORY_ERR_UNSUPPORTED, "block_size %d is not a multiple of 16", a.block_size);
  const int G = a.num_heads / a.num_kv_heads;
  if (G > 16) return fail(DORY_ERR_UNSUPPORTED, "%d query heads per KV head (max 16)", G);
  if (kv8 && (HD < 128 || G > 8 || fma || a.num_cache_blocks <= 0))
    return fail(DORY_ERR_UNSUPPORTED,
                "FP8 caches take 128/256-dim heads, at most 8 query heads per KV head, a "
                "known block count and the tensor-core consumer");
  if (kv8 && !(a.k_scale > 0.0f && a.v_scale > 0.0f && a.k_scale < 3.4e38f && a.v_scale < 3.4e38f))
    return fail(DORY_ERR_INVALID_ARGUMENT, "FP8 caches need positive, finite k/v scales");
  if (fma && (HD != 128 || G > 4 || shared))
    return fail(DORY_ERR_UNSUPPORTED,
                "the CUDA-core consumer takes 128-dim heads, at most 4 query heads per KV head "
                "and no shared cache");
  if (shared && a.num_tokens > kMaxSub)
    return fail(DORY_ERR_UNSUPPORTED, "shared-cache calls take at most %d tokens", kMaxSub);
  if (a.sqk_dtype < 0 || a.sqk_dtype > 2) return fail(DORY_ERR_INVALID_ARGUMENT, "sqk dtype");
  if (reinterpret_cast<uintptr_t>(a.gate) & 15)
    return fail(DORY_ERR_ALIGNMENT, "gate needs a 16-byte aligned base");
  if ((reinterpret_cast<uintptr_t>(a.key_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(a.value_cache) & 15) || (a.stride_block & (kv8 ? 15 : 7)) ||
      (a.stride_offset & (kv8 ? 15 : 7)) || (a.stride_head & (kv8 ? 15 : 7)))
    return fail(DORY_ERR_ALIGNMENT,
                "key/value caches need 16-byte aligned bases and strides (multiples of 8)");
  ScratchLayout SL;
  if (!scratch_layout_checked(a.max_tokens, a.splits, a.num_heads, a.num_kv_heads, HD, &SL))
    return fail(DORY_ERR_INVALID_ARGUMENT, "max_tokens x splits x heads x head_dim overflows");
  if (a.scratch_bytes < SL.total)
    return fail(DORY_ERR_INVALID_ARGUMENT, "scratch too small (%lld < %lld bytes)",
                (long long)a.scratch_bytes, (long long)SL.total);
  if (a.num_tokens == 0) return DORY_OK;

  // One 8-row tile per CTA unless one KV head's group alone needs more rows: a shared-cache
  // wavefront then runs as groups of 8 / G tokens whose reads of the same blocks meet in L2,
  // which measured faster than 16-row tiles (twice the math and merge per CTA).
  int nt = G > 8 ? 2 : 1;
  if (HD == 256 && nt == 2) {
    if (G > 8) return fail(DORY_ERR_UNSUPPORTED, "head_dim 256 with more than 8 heads per KV head");
    nt = 1;
  }

  KParams kp;
  memset(&kp, 0, sizeof(kp));
  kp.q = a.q;
  kp.v = a.v;
  kp.sqk = a.sqk;
  kp.slot_mapping = a.slot_mapping;
  kp.kc = static_cast<__nv_bfloat16*>(a.key_cache);
  kp.vc = static_cast<__nv_bfloat16*>(a.value_cache);
  kp.table = a.block_table;
  kp.table_offsets = a.block_table_offsets;
  kp.cache_offsets = a.cache_offsets;
  kp.seq_lens = a.seq_lens;
  kp.gate = a.gate;
  kp.out = a.out_nibble_major;
  kp.sumsq = a.out_sumsq;
  uint8_t* base = static_cast<uint8_t*>(a.scratch);
  kp.err = reinterpret_cast<uint32_t*>(base);
  kp.counters = reinterpret_cast<int32_t*>(base + SL.counters);
  kp.tok_counters = reinterpret_cast<int32_t*>(base + SL.tok_counters);
  kp.sumsq_part = reinterpret_cast<float*>(base + SL.sumsq_part);
  kp.pml = reinterpret_cast<float2*>(base + SL.pml);
  kp.po = reinterpret_cast<float*>(base + SL.po);
  kp.sb = a.stride_block;
  kp.so = a.stride_offset;
  kp.sh = a.stride_head;
  kp.ncache_blocks = a.num_cache_blocks;
  kp.scale = a.softmax_scale;
  kp.k_scale = kv8 ? a.k_scale : 1.0f;
  kp.v_scale = kv8 ? a.v_scale : 1.0f;
  kp.sqk_factor = a.sqk_factor;
  kp.eps = a.eps;
  kp.T = a.num_tokens;
  kp.NH = a.num_heads;
  kp.NKV = a.num_kv_heads;
  kp.G = G;
  kp.B = a.block_size;
  kp.window = a.window;
  kp.S = a.splits;
  kp.bpt = a.blocks_per_tile;
  kp.min_bps = a.min_blocks_per_split < 1 ? 1 : a.min_blocks_per_split;
  kp.tps_min = (kp.min_bps + a.blocks_per_tile - 1) / a.blocks_per_tile;
  auto log2_exact = [](int v) {
    int k = 0;
    while ((1 << k) < v) ++k;
    return (1 << k) == v ? k : -1;
  };
  kp.b_shift = log2_exact(a.block_size);
  kp.cpb_shift = log2_exact(a.block_size / 16);
  kp.sqk_dtype = a.sqk_dtype;
  kp.raw = raw;
  kp.multi = multi;
  kp.shared = shared;
  kp.overlap = overlap;
  // L2 prefetch distance beyond the ring.  Automatic (0): an overlapped launch whose grid is
  // resident at once (one wave) prefetches every chunk of a CTA's range at the CTA's start,
  // so the reads it issues before waiting for the previous kernel cover its whole range and
  // its copies after the wait come from L2 (config 4: 14.5 -> 13.4 us per layer-step).
  // Plain launches keep to the ring: there the prefetches only queue ahead of the ring's
  // own copies (config 4: 14.6 -> 16.1 us), as do grids of several waves.
  {
    int pf = a.prefetch_chunks;
    if (pf == 0) {
      const int per_sm = (HD <= 128 && nt == 1) ? 3 : 1;
      const long long ctas = (long long)a.splits * a.num_kv_heads * a.num_tokens;
      pf = overlap && ctas <= (long long)sm_count() * per_sm ? (1 << 20) : -1;
    }
    kp.pf = pf > 0 ? pf : 0;
  }
  kp.q_stride = (raw ? a.num_heads + a.num_kv_heads : a.num_heads) * HD;
  kp.nsub = raw ? (shared ? a.num_tokens : 1) : 0;
  // Tensor maps of the K and V views.  Multi-token calls may shift the cache by whole
  // blocks (per-loop caches at cache_offsets[t]); the block extent then allows up to 64
  // caches' worth of blocks past the view.  Other offsets take the copy path.
  {
    const int64_t nb = a.num_cache_blocks > 0 ? a.num_cache_blocks : 0;
    const int64_t extent = multi ? (nb * 64 < 0x7fffffff ? nb * 64 : 0x7fffffff) : nb;
    const int esize = kv8 ? 1 : 2;
    const int q = kv8 ? HD / 128 : HD / 64;  // 128-byte pieces of a row's K (or V)
    kp.tm_mode = 0;
    kp.tm_blocks = extent;
    if (nb > 0) {
      const bool adjacent = static_cast<const char*>(a.value_cache) ==
                            static_cast<const char*>(a.key_cache) + HD * esize;
      MapKey both{a.key_cache, extent, a.stride_block, a.stride_offset, a.stride_head,
                  a.block_size, a.num_kv_heads, 2 * q, esize};
      if (adjacent && cache_tensor_map(both, &kp.tmk)) {
        kp.tm_mode = 1;
      } else {
        MapKey kk{a.key_cache, extent, a.stride_block, a.stride_offset, a.stride_head,
                  a.block_size, a.num_kv_heads, q, esize};
        MapKey vk = kk;
        vk.base = a.value_cache;
        if (cache_tensor_map(kk, &kp.tmk) && cache_tensor_map(vk, &kp.tmv)) kp.tm_mode = 2;
      }
    }
  }

  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid(a.splits, a.num_kv_heads, a.num_tokens);
  if (kv8) {
    if (kp.tm_mode == 0)
      return fail(DORY_ERR_UNSUPPORTED, "FP8 caches need a tensor map of the cache view");
    return HD == 128 ? dispatch_kv8<128>(kp, grid, s) : dispatch_kv8<256>(kp, grid, s);
  }
  if (HD == 64) return dispatch_nt<64>(kp, nt, grid, s);
  if (HD == 128) return fma ? dispatch_fma(kp, grid, s) : dispatch_nt<128>(kp, nt, grid, s);
  return dispatch_nt<256>(kp, nt, grid, s);
}

}  // extern "C"

// ------------------------------------------------------------------------------------
// Allocation-free entry point: the scratch is a file-scope device array of this library.
// ------------------------------------------------------------------------------------
namespace {

// Split partials, merge counters and error word for callers that cannot allocate device
// memory.  Device code could name it directly; host code only through the address
// cudaGetSymbolAddress returns (the host-side symbol is a stand-in, not a device pointer).
// Device globals start zeroed, so the error word and the counters start at zero.
__device__ __align__(256) uint8_t g_static_scratch[DORY_DECODE_STATIC_SCRATCH_BYTES];

// The array's device address belongs to a CUDA context (each context that loads this
// library has its own copy), so it is cached per context: the runtime's primary context
// of a device, or a context a driver-API host made current itself.
constexpr int kMaxContexts = 64;
std::mutex g_static_mutex;
struct StaticEntry {
  CUcontext ctx;
  void* ptr;
};
StaticEntry g_static_entries[kMaxContexts];
int g_static_used = 0;

PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
  });
  return fn;
}

CUcontext current_context() {
  CUcontext ctx = nullptr;
  auto get = ctx_get_current();
  if (!get || get(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of g_static_scratch in the calling thread's current context (the current
// device's primary context when none is bound), looked up once per context.
int32_t static_scratch_address(void** out) {
  CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (ctx)
    for (int i = 0; i < g_static_used; ++i)
      if (g_static_entries[i].ctx == ctx) {
        *out = g_static_entries[i].ptr;
        return DORY_OK;
      }
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
  if (e != cudaSuccess || ptr == nullptr)
    return fail(DORY_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
  if (!ctx) ctx = current_context();  // the runtime has now bound the primary context
  if (ctx) {
    if (g_static_used == kMaxContexts)
      return fail(DORY_ERR_UNSUPPORTED, "static scratch used from more than %d contexts",
                  kMaxContexts);
    g_static_entries[g_static_used++] = StaticEntry{ctx, ptr};
  }
  *out = ptr;
  return DORY_OK;
}

}  // namespace

extern "C" int32_t dory_decode_attention_static_scratch(const DoryDecodeParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  ScratchLayout SL;
  if (!scratch_layout_checked(P->max_tokens, P->splits, P->num_heads, P->num_kv_heads,
                              P->head_dim, &SL))
    return fail(DORY_ERR_INVALID_ARGUMENT, "invalid or overflowing scratch shape");
  if (SL.total > DORY_DECODE_STATIC_SCRATCH_BYTES)
    return fail(DORY_ERR_INVALID_ARGUMENT,
                "this call needs %lld bytes of scratch; the static scratch holds %lld "
                "(use fewer splits or tokens, or dory_decode_attention with caller scratch)",
                (long long)SL.total, (long long)DORY_DECODE_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int32_t st = static_scratch_address(&scratch);
  if (st != DORY_OK) return st;
  // The counters (merge and sum-of-squares) sit at different offsets for different call
  // shapes, so the previous call's must not leak into this one: clear them.  The error word
  // in front of them is kept; it gathers the device errors of every call until
  // dory_decode_static_scratch_fetch_errors reads (and optionally clears) it.
  cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + SL.counters, 0,
                                  size_t(SL.pml - SL.counters), (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  DoryDecodeParams a = *P;
  a.scratch = scratch;
  a.scratch_bytes = DORY_DECODE_STATIC_SCRATCH_BYTES;
  return dory_decode_attention(&a, stream);
}

extern "C" int32_t dory_decode_static_scratch_fetch_errors(uint32_t* flags_out, int32_t clear,
                                                           void* stream) {
  if (!flags_out) return fail(DORY_ERR_INVALID_ARGUMENT, "null argument");
  void* scratch = nullptr;
  const int32_t st = static_scratch_address(&scratch);
  if (st != DORY_OK) return st;
  return dory_decode_fetch_errors(scratch, flags_out, clear, stream);
}
