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
//   * K/V rows (head_dim * 2 bytes, contiguous for any of the three cache layouts) are
//     staged into a multi-stage shared-memory ring by the TMA engine (cp.async.bulk, one
//     row per lane of a producer warp, mbarrier complete_tx), rows padded by 16 bytes so
//     ldmatrix reads are bank-conflict free.  Only rows inside the attended range are read.
//   * Four consumer warps each own a ring slot in turn and run the 16-token chunk through
//     mma.sync m16n8k16 (bf16 in, fp32 accumulate) with tokens on M and the GQA group's query
//     rows (plus the other tokens of a shared-cache group) on N: S^T = K Q^T, then
//     O^T += V^T P^T; P^T moves from accumulator to operand layout with movmatrix.
//   * Softmax is online, in the log2 domain, with warp-shuffle row reductions.
//   * Split partials go to caller-owned scratch; the last-arriving CTA merges (atomic
//     counter, self-resetting), so one launch does what the reference does in two or three.
//   * Every wait is bounded: on timeout the kernel records DORY_DEVERR_WAIT_TIMEOUT and
//     drains its own copies before returning.  Out-of-range block ids / slots are recorded
//     and skipped, never dereferenced.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdarg.h>
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
constexpr long long kWaitLimitCycles = 500000000LL;  // ~0.25 s at 1.9 GHz, then give up
constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------------------------
// Kernel parameters (device-side copy of DoryDecodeParams plus derived values).
// ------------------------------------------------------------------------------------
struct KParams {
  const void* q;
  const float* v;
  const void* sqk;
  const int64_t* slot_mapping;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  const int32_t* table;
  const int64_t* table_offsets;
  const int64_t* cache_offsets;
  const int32_t* seq_lens;
  const float* gate;
  float* out;
  uint32_t* err;
  int32_t* counters;
  float2* pml;  // [max_tokens][S][NH] (max in log2 units, sum)
  float* po;    // [max_tokens][S][NH][HD]
  int64_t sb, so, sh, ncache_blocks;
  float scale, sqk_factor, eps;
  int T, NH, NKV, G, B, window, S, bpt, min_bps, sqk_dtype;
  int raw, multi, shared;
  int q_stride;  // elements of q per token
  int nsub;      // new tokens whose k/v this call substitutes (shared: T, raw: 1, else 0)
};

// Scratch layout (bytes), shared by host and device.
struct ScratchLayout {
  int64_t counters, pml, po, total;
};
__host__ __device__ inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }
__host__ __device__ inline ScratchLayout scratch_layout(int max_tokens, int S, int NH, int NKV,
                                                        int HD) {
  ScratchLayout L;
  L.counters = 256;  // [0, 256): header; word 0 = device error flags
  L.pml = align256(L.counters + int64_t(max_tokens) * NKV * 4);
  L.po = align256(L.pml + int64_t(max_tokens) * S * NH * 8);
  L.total = align256(L.po + int64_t(max_tokens) * S * NH * HD * 4);
  return L;
}

// Dynamic shared memory layout for one instantiation.
template <int HD, int NS>
struct Smem {
  static constexpr int kRowBytes = HD * 2 + 16;               // padded row
  static constexpr int kStageBytes = 2 * kChunk * kRowBytes;  // K rows then V rows
  static constexpr int kStages = 0;
  static constexpr int kBars = kStages + NS * kStageBytes;    // full[NS], empty[NS]
  static constexpr int kMeta = kBars + 2 * NS * 8;            // int4 {phys, mask, chunk, -}
  static constexpr int kQ = kMeta + NS * 16;                  // bf16 [16][HD]
  static constexpr int kSub = kQ + 16 * HD * 2;               // bf16 [nsub][2][HD]
  static int bytes(int nsub) { return kSub + (nsub > 0 ? nsub : 1) * 2 * HD * 2; }
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
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
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

__device__ __forceinline__ float load_sqk(const void* sqk, int dtype, int64_t i) {
  if (dtype == DORY_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(sqk)[i]);
  if (dtype == DORY_DTYPE_F16) return __half2float(static_cast<const __half*>(sqk)[i]);
  return static_cast<const float*>(sqk)[i];
}

// Canonical normalisation factor of one row: Sum x^2 is accumulated in FP64 (every square
// is exact there, so the FP32 rounding of the sum does not depend on summation order),
// rounded to FP32, eps is added in FP32 (as the reference's `tl.sum(x * x) + eps`) and the
// inverse square root is the correctly rounded FP32 value, from IEEE double sqrt and
// division.  The oracle computes the same quantities the same way.
template <int PER_LANE>
__device__ __forceinline__ float row_inv_norm(const float (&x)[PER_LANE], float eps) {
  double acc = 0.0;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) acc += double(x[i]) * double(x[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  const float sum32 = __double2float_rn(acc);
  const float t = __fadd_rn(sum32, eps);
  return __double2float_rn(1.0 / sqrt(double(t)));
}

// Split layout of the reference (_split_layout, dory_decode_attention.py:28-44) applied to
// the attended union [lo, hi) of a token group.
struct Split {
  int first_block, nblocks, tiles, tps, active;
};
__device__ __forceinline__ Split split_layout(int lo, int hi, int B, int S, int bpt, int min_bps) {
  Split s;
  if (hi <= 0) {
    s.first_block = 0;
    s.nblocks = 0;
    s.tiles = 0;
    s.tps = 1;
    s.active = 0;
    return s;
  }
  s.first_block = lo / B;
  s.nblocks = (hi + B - 1) / B - s.first_block;
  s.tiles = (s.nblocks + bpt - 1) / bpt;
  int tps = (s.tiles + S - 1) / S;
  const int tps_min = (min_bps + bpt - 1) / bpt;
  if (tps < tps_min) tps = tps_min;
  if (tps < 1) tps = 1;
  s.tps = tps;
  s.active = (s.tiles + tps - 1) / tps;
  return s;
}

// ------------------------------------------------------------------------------------
// The kernel.  grid = (splits, NKV, T); block = 160 threads (4 consumer warps + producer).
// ------------------------------------------------------------------------------------
template <int HD, int NT, int NS>
__global__ void __launch_bounds__(kThreads) decode_kernel(const __grid_constant__ KParams p) {
  using L = Smem<HD, NS>;
  constexpr int KT = HD / 16;          // MMA k-steps over head_dim / m-tiles of O^T
  constexpr int ROWS = NT * 8;         // query rows per CTA
  constexpr int PER_LANE = HD / 32;    // elements per lane in row-wise prologue math
  constexpr int ROWB = L::kRowBytes;

  extern __shared__ __align__(128) uint8_t smem[];
  // Per-token info, indexed by token for shared-cache calls and by 0 otherwise.
  __shared__ int s_len[kMaxSub], s_phys[kMaxSub];
  __shared__ long long s_coff[kMaxSub], s_toff[kMaxSub];
  __shared__ int s_grouped, s_last;
  __shared__ float s_wm[kConsumerWarps][ROWS], s_wl[kConsumerWarps][ROWS];

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int tok = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = p.G;
  const int B = p.B;
  const int Q = p.NH * HD;

  // ---- token info: the group's tokens and the tokens whose new k/v this CTA may have to
  //      substitute (shared-cache: every token of the call; otherwise this token alone).
  const int ninfo = p.shared ? p.T : 1;
  if (tid == 0) s_grouped = 1;
  if (tid < ninfo) {
    const int t = p.shared ? tid : tok;
    s_len[tid] = p.seq_lens[t];
    s_coff[tid] = p.multi ? p.cache_offsets[t] : 0;
    s_toff[tid] = p.multi ? p.table_offsets[t] : 0;
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
  const Split sp = split_layout(lo, hi, B, p.S, p.bpt, p.min_bps);
  const int nrows = gcount * G;

  if (sp.tiles == 0) {
    // Padding request(s): the reference's combine writes 0 * gate.
    if (split == 0) {
      for (int i = tid; i < nrows * HD; i += kThreads) {
        const int r = i / HD, d = i % HD;
        const int t = gstart + r / G, head = kvh * G + r % G;
        const int e = head * HD + d;
        p.out[int64_t(t) * Q + (e % 8) * (Q / 8) + e / 8] = 0.0f * p.gate[int64_t(t) * Q + e];
      }
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
  const int ce = min(be * CPB, (hi + kChunk - 1) / kChunk);
  const int nchunks = ce - cb;

  const uint32_t bars = smem_u32(smem + L::kBars);
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (NS + s); };
  int4* meta = reinterpret_cast<int4*>(smem + L::kMeta);
  __nv_bfloat16* q2 = reinterpret_cast<__nv_bfloat16*>(smem + L::kQ);
  __nv_bfloat16* subkv = reinterpret_cast<__nv_bfloat16*>(smem + L::kSub);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if ((coff & 7) != 0) record_error(p.err, DORY_DEVERR_OFFSET_ALIGN);
  }
  __syncthreads();
  const bool offset_ok = (coff & 7) == 0;

  if (warp == kConsumerWarps) {
    // =============================== producer warp ===============================
    const __nv_bfloat16* kbase = p.kc + coff + int64_t(kvh) * p.sh;
    const __nv_bfloat16* vbase = p.vc + coff + int64_t(kvh) * p.sh;
    const int32_t* table = p.table + toff;
    const int row = lane & 15;
    const bool is_v = lane >= 16;
    // Block-table window of 32 entries, prefetched one window ahead.
    const int b_first = cb / CPB;
    const int b_last = (ce - 1) / CPB;
    int wbase = b_first;
    int win_cur = (b_first + lane <= b_last) ? table[b_first + lane] : -1;
    int win_nxt = (b_first + 32 + lane <= b_last) ? table[b_first + 32 + lane] : -1;
    bool ok_all = true;
    for (int i = 0; i < nchunks; ++i) {
      const int stage = i % NS;
      const uint32_t parity = ((i / NS) & 1) ^ 1;
      if (!mbar_wait(empty_bar(stage), parity)) {
        if (lane == 0) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
        ok_all = false;
        break;
      }
      const int c = cb + i;
      const int blk = c / CPB;
      while (blk >= wbase + 32) {
        wbase += 32;
        win_cur = win_nxt;
        win_nxt = (wbase + 32 + lane <= b_last) ? table[wbase + 32 + lane] : -1;
      }
      const int phys = __shfl_sync(0xffffffffu, win_cur, blk - wbase);
      bool phys_ok = phys >= 0 && (p.ncache_blocks <= 0 || phys < p.ncache_blocks) && offset_ok;
      if (!phys_ok && lane == 0 && offset_ok) record_error(p.err, DORY_DEVERR_BLOCK_OOB);
      const int in_block = (c % CPB) * kChunk + row;
      const int pos = c * kChunk + row;
      const bool valid = phys_ok && pos >= lo && pos < hi;
      const uint32_t mask = __ballot_sync(0xffffffffu, valid) & 0xffffu;
      const uint32_t bytes = __popc(mask) * 2u * HD * 2u;
      if (lane == 0) {
        meta[stage] = make_int4(phys, int(mask), c, 0);
        mbar_arrive_expect_tx(full_bar(stage), bytes);
      }
      __syncwarp();
      if (valid) {
        const int64_t off = int64_t(phys) * p.sb + int64_t(in_block) * p.so;
        const uint32_t dst =
            smem_u32(smem + L::kStages + stage * L::kStageBytes + (is_v ? kChunk * ROWB : 0) +
                     row * ROWB);
        bulk_g2s(dst, (is_v ? vbase : kbase) + off, HD * 2, full_bar(stage));
      }
    }
    (void)ok_all;
    return;
  }

  // =============================== consumer warps ===============================
  // (0) physical block of each new token's slot (off the producer's dependent-load chain).
  if (warp == 0 && lane < nsub) {
    const int len = s_len[lane];
    s_phys[lane] = len > 0 ? p.table[s_toff[lane] + (len - 1) / B] : -1;
  }
  // (1) query rows: normalise / scale / round, as the reference, into q2 [16][HD] bf16.
  for (int r = warp; r < 16; r += kConsumerWarps) {
    if (r >= nrows) {
      for (int d = lane; d < HD; d += 32) q2[r * HD + d] = __float2bfloat16_rn(0.0f);
      continue;
    }
    const int t = gstart + r / G;
    const int head = kvh * G + r % G;
    float qv[PER_LANE];
    if (p.raw) {
      const float* src = static_cast<const float*>(p.q) + int64_t(t) * p.q_stride + head * HD;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) qv[i] = src[lane * PER_LANE + i];
      const float rn = row_inv_norm<PER_LANE>(qv, p.eps);
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int d = lane * PER_LANE + i;
        const float s = __fmul_rn(load_sqk(p.sqk, p.sqk_dtype, head * HD + d), p.sqk_factor);
        const float qn = __fmul_rn(qv[i], rn);
        const float qb = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(s, s), qn)));
        q2[r * HD + d] = __float2bfloat16_rn(__fmul_rn(qb, p.scale));
      }
    } else {
      const __nv_bfloat16* src =
          static_cast<const __nv_bfloat16*>(p.q) + int64_t(t) * p.q_stride + head * HD;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int d = lane * PER_LANE + i;
        q2[r * HD + d] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(src[d]), p.scale));
      }
    }
  }
  // (2) new keys / values of the sub tokens: k = bf16(k * inv_norm(k)), v = bf16(v).
  if (p.raw) {
    for (int s = warp; s < nsub; s += kConsumerWarps) {
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
        subkv[(s * 2 + 0) * HD + d] = __float2bfloat16_rn(__fmul_rn(kv[i], rn));
        subkv[(s * 2 + 1) * HD + d] = __float2bfloat16_rn(vsrc[d]);
      }
    }
  }
  named_barrier_consumers();

  // (3) append: the CTA whose chunk range holds a group token's position writes its k/v.
  if (p.raw && warp == 0) {
    for (int j = 0; j < gcount; ++j) {
      const int si = ibase + j;
      const int len = s_len[si];
      if (len <= 0) continue;
      const int pos = len - 1;
      const int c = pos / kChunk;
      if (c < cb || c >= ce) continue;
      long long slot;
      if (p.multi) {
        slot = (long long)s_phys[si] * B + pos % B;
      } else {
        slot = p.slot_mapping[0];
        if (slot < 0) continue;  // padding token: vLLM does not cache it
      }
      const long long blk = slot / B;
      if (blk < 0 || (p.ncache_blocks > 0 && blk >= p.ncache_blocks) || !offset_ok) {
        if (lane == 0) record_error(p.err, DORY_DEVERR_SLOT_OOB);
        continue;
      }
      const long long base = s_coff[si] + blk * p.sb + (slot % B) * p.so + (long long)kvh * p.sh;
      constexpr int kVec = HD / 8;  // 16-byte vectors per row
      for (int i = lane; i < 2 * kVec; i += 32) {
        const bool is_v = i >= kVec;
        const int w = is_v ? i - kVec : i;
        const uint4 val = reinterpret_cast<const uint4*>(subkv + (si * 2 + (is_v ? 1 : 0)) * HD)[w];
        reinterpret_cast<uint4*>((is_v ? p.vc : p.kc) + base)[w] = val;
      }
    }
  }

  // (4) B fragments of Q^T (k = dims, n = query rows), resident for the whole loop.
  const int g = lane >> 2;
  const int t4 = lane & 3;
  uint32_t qb[NT][KT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
      const uint32_t* row = reinterpret_cast<const uint32_t*>(q2 + (nt * 8 + g) * HD + kk * 16);
      qb[nt][kk][0] = row[t4];
      qb[nt][kk][1] = row[t4 + 4];
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
      rlen[nt][i] = len;
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

  bool failed = false;
  for (int i = warp; i < nchunks; i += kConsumerWarps) {
    const int stage = i % NS;
    const uint32_t parity = (i / NS) & 1;
    if (!mbar_wait(full_bar(stage), parity)) {
      if (lane == 0) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
      failed = true;
      break;
    }
    const int4 mt = meta[stage];
    const int phys = mt.x;
    const uint32_t mask = uint32_t(mt.y);
    const int c = mt.z;
    uint8_t* kst = smem + L::kStages + stage * L::kStageBytes;
    uint8_t* vst = kst + kChunk * ROWB;
    bool touched = false;
    // Rows not copied (outside [lo, hi) or a bad block) hold stale bytes: zero V there so
    // that p = 0 never multiplies a non-finite value.
    if (mask != 0xffffu) {
      constexpr int kVec = HD / 8;
      for (int idx = lane; idx < kChunk * kVec; idx += 32) {
        const int r = idx / kVec, w = idx % kVec;
        if (!((mask >> r) & 1u)) reinterpret_cast<uint4*>(vst + r * ROWB)[w] = make_uint4(0, 0, 0, 0);
      }
      touched = true;
    }
    // New entries of this call replace the rows that alias their slots.
    if (p.raw) {
      const int in_block0 = (c % CPB) * kChunk;
      for (int s = 0; s < nsub; ++s) {
        if (s_len[s] <= 0 || s_phys[s] != phys || s_coff[s] != coff) continue;
        const int r = ((s_len[s] - 1) % B) - in_block0;
        if (r < 0 || r >= kChunk) continue;
        constexpr int kVec = HD / 8;
        for (int idx = lane; idx < 2 * kVec; idx += 32) {
          const bool is_v = idx >= kVec;
          const int w = is_v ? idx - kVec : idx;
          const uint4 val = reinterpret_cast<const uint4*>(subkv + (s * 2 + (is_v ? 1 : 0)) * HD)[w];
          reinterpret_cast<uint4*>((is_v ? vst : kst) + r * ROWB)[w] = val;
        }
        touched = true;
      }
    }
    __syncwarp();

    // S^T = K Q^T : [16 tokens x 8 rows] per n-tile.
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
    {
      const uint32_t kaddr = smem_u32(kst) + (lane & 15) * ROWB + (lane >> 4) * 16;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kaddr + kk * 32, a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(sc[nt], a0, a1, a2, a3, qb[nt][kk][0], qb[nt][kk][1]);
      }
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
        const bool v0 = pos0 >= rfirst[nt][i] && pos0 < rlen[nt][i];
        const bool v1 = pos1 >= rfirst[nt][i] && pos1 < rlen[nt][i];
        const float x0 = v0 ? sc[nt][i] * kLog2e : -INFINITY;
        const float x1 = v1 ? sc[nt][2 + i] * kLog2e : -INFINITY;
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
      pb[nt][0] = movmatrix_t(pack_bf16x2(pv[0], pv[1]));
      pb[nt][1] = movmatrix_t(pack_bf16x2(pv[2], pv[3]));
    }
    // O^T += V^T P^T : [16 dims x 8 rows] per m-tile and n-tile.
    {
      const uint32_t vaddr =
          smem_u32(vst) + ((lane & 7) + ((lane >> 4) << 3)) * ROWB + ((lane >> 3) & 1) * 16;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vaddr + kk * 32, a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(o[nt][kk], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
      }
    }
    if (touched) fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(stage));
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

  // Drain: every copy this CTA issued must have landed before its shared memory is reused
  // or released (only matters after a timeout; otherwise these waits return at once).
  named_barrier_consumers();
  if (tid == 0) {
    bool drained = true;
    for (int s = 0; s < NS && s < nchunks; ++s) {
      const int last = s + ((nchunks - 1 - s) / NS) * NS;
      if (!mbar_wait(full_bar(s), (last / NS) & 1)) drained = false;
    }
    if (!drained) record_error(p.err, DORY_DEVERR_WAIT_TIMEOUT);
  }
  (void)failed;
  named_barrier_consumers();

  // ---- merge the four consumer warps (shared memory, aliasing the drained ring) ----
  constexpr int OST = HD + 4;  // padded row stride of the per-warp O buffers (floats)
  float* wo = reinterpret_cast<float*>(smem + L::kStages);  // [warps][ROWS][OST]
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
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        dst[kk * 16 + g] = o[nt][kk][i];
        dst[kk * 16 + g + 8] = o[nt][kk][2 + i];
      }
    }
  named_barrier_consumers();

  // Items: (row, 8 consecutive dims).  Each thread merges its items across warps.
  constexpr int IPR = HD / 8;
  const int items = nrows * IPR;
  const bool single = sp.active == 1;
  const int64_t S = p.S;
  for (int it = tid; it < items; it += kConsumerWarps * 32) {
    const int r = it / IPR, k8 = it % IPR;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s_wm[w][r]);
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
    const int t = gstart + r / G;
    const int head = kvh * G + r % G;
    if (single) {
      const float inv = 1.0f / (Lsum > 0.0f ? Lsum : 1.0f);
      const int e0 = head * HD + k8 * 8;
      const float* gt = p.gate + int64_t(t) * Q + e0;
      float* out = p.out + int64_t(t) * Q + e0 / 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e * (Q / 8)] = acc[e] * inv * gt[e];
    } else {
      const int64_t pi = (int64_t(t) * S + split) * p.NH + head;
      if (k8 == 0) p.pml[pi] = make_float2(M, Lsum);
      float4* dst = reinterpret_cast<float4*>(p.po + pi * HD + k8 * 8);
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  if (single) return;

  // ---- cross-split merge by the last CTA of this (group, KV head) to arrive ----
  __threadfence();
  named_barrier_consumers();
  if (tid == 0) {
    int32_t* counter = p.counters + gstart * p.NKV + kvh;
    const int prev = atomicAdd(counter, 1);
    s_last = (prev == sp.active - 1);
    if (s_last) *counter = 0;  // self-reset for the next launch
  }
  named_barrier_consumers();
  if (!s_last) return;
  __threadfence();
  for (int it = tid; it < items; it += kConsumerWarps * 32) {
    const int r = it / IPR, k8 = it % IPR;
    const int t = gstart + r / G;
    const int head = kvh * G + r % G;
    float M = -INFINITY, Lsum = 0.0f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    for (int s = 0; s < sp.active; ++s) {
      const int64_t pi = (int64_t(t) * S + s) * p.NH + head;
      const float2 ml = __ldcg(p.pml + pi);
      const float4* src = reinterpret_cast<const float4*>(p.po + pi * HD + k8 * 8);
      const float4 a = __ldcg(src), b = __ldcg(src + 1);
      const float Mn = fmaxf(M, ml.x);
      const float Mu = (Mn == -INFINITY) ? 0.0f : Mn;
      const float wa = fast_exp2(M - Mu), wb = fast_exp2(ml.x - Mu);
      Lsum = Lsum * wa + ml.y * wb;
      acc[0] = acc[0] * wa + a.x * wb; acc[1] = acc[1] * wa + a.y * wb;
      acc[2] = acc[2] * wa + a.z * wb; acc[3] = acc[3] * wa + a.w * wb;
      acc[4] = acc[4] * wa + b.x * wb; acc[5] = acc[5] * wa + b.y * wb;
      acc[6] = acc[6] * wa + b.z * wb; acc[7] = acc[7] * wa + b.w * wb;
      M = Mn;
    }
    const float inv = 1.0f / (Lsum > 0.0f ? Lsum : 1.0f);
    const int e0 = head * HD + k8 * 8;
    const float* gt = p.gate + int64_t(t) * Q + e0;
    float* out = p.out + int64_t(t) * Q + e0 / 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e * (Q / 8)] = acc[e] * inv * gt[e];
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

template <int HD, int NT, int NS>
int32_t launch(const KParams& kp, dim3 grid, int smem_bytes, cudaStream_t stream) {
  auto fn = decode_kernel<HD, NT, NS>;
  static int configured[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(DORY_ERR_CUDA, "cudaGetDevice failed");
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    // The largest dynamic size any call of this instantiation can ask for.
    const int max_bytes = Smem<HD, NS>::bytes(kMaxSub);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes);
    if (e != cudaSuccess)
      return fail(DORY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = 1;
  }
  fn<<<grid, kThreads, smem_bytes, stream>>>(kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return DORY_OK;
}

// Pipeline depth per head_dim: ~70 KB of ring per CTA.
template <int HD> struct Depth { static constexpr int value = HD >= 256 ? 4 : 8; };

template <int HD>
int32_t dispatch_nt(const KParams& kp, int nt, dim3 grid, cudaStream_t stream) {
  constexpr int NS = Depth<HD>::value;
  const int smem = Smem<HD, NS>::bytes(kp.nsub);
  if (nt == 1) return launch<HD, 1, NS>(kp, grid, smem, stream);
  if constexpr (HD <= 128) return launch<HD, 2, NS>(kp, grid, smem, stream);
  return fail(DORY_ERR_UNSUPPORTED, "head_dim %d supports at most 8 query rows per tile", HD);
}

}  // namespace

extern "C" {

int32_t dory_decode_abi_version(void) { return DORY_DECODE_ABI_VERSION; }

int64_t dory_decode_params_bytes(void) { return int64_t(sizeof(DoryDecodeParams)); }

int64_t dory_decode_scratch_bytes(int32_t max_tokens, int32_t splits, int32_t num_heads,
                                  int32_t num_kv_heads, int32_t head_dim) {
  if (max_tokens < 1 || splits < 1 || num_heads < 1 || num_kv_heads < 1 || head_dim < 1) return 0;
  return scratch_layout(max_tokens, splits, num_heads, num_kv_heads, head_dim).total;
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

int32_t dory_decode_attention(const DoryDecodeParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  const DoryDecodeParams& a = *P;
  if (a.num_heads < 1 || a.num_kv_heads < 1 || a.num_heads % a.num_kv_heads)
    return fail(DORY_ERR_INVALID_ARGUMENT, "query heads must be a multiple of KV heads");
  const bool raw = a.flags & DORY_FLAG_RAW_QKV;
  const bool multi = a.flags & DORY_FLAG_MULTI_TOKEN;
  const bool shared = a.flags & DORY_FLAG_SHARED_CACHE;
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
  if (shared && a.num_tokens > kMaxSub)
    return fail(DORY_ERR_UNSUPPORTED, "shared-cache calls take at most %d tokens", kMaxSub);
  if (a.sqk_dtype < 0 || a.sqk_dtype > 2) return fail(DORY_ERR_INVALID_ARGUMENT, "sqk dtype");
  if ((reinterpret_cast<uintptr_t>(a.key_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(a.value_cache) & 15) || (a.stride_block & 7) ||
      (a.stride_offset & 7) || (a.stride_head & 7))
    return fail(DORY_ERR_ALIGNMENT,
                "key/value caches need 16-byte aligned bases and strides (multiples of 8)");
  const ScratchLayout SL =
      scratch_layout(a.max_tokens, a.splits, a.num_heads, a.num_kv_heads, HD);
  if (a.scratch_bytes < SL.total)
    return fail(DORY_ERR_INVALID_ARGUMENT, "scratch too small (%lld < %lld bytes)",
                (long long)a.scratch_bytes, (long long)SL.total);
  if (a.num_tokens == 0) return DORY_OK;

  // Query rows per tile: one token's group, or up to 16 rows of shared-cache tokens.
  int rows = shared ? (a.num_tokens * G < 16 ? a.num_tokens * G : 16) : G;
  int nt = rows > 8 ? 2 : 1;
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
  uint8_t* base = static_cast<uint8_t*>(a.scratch);
  kp.err = reinterpret_cast<uint32_t*>(base);
  kp.counters = reinterpret_cast<int32_t*>(base + SL.counters);
  kp.pml = reinterpret_cast<float2*>(base + SL.pml);
  kp.po = reinterpret_cast<float*>(base + SL.po);
  kp.sb = a.stride_block;
  kp.so = a.stride_offset;
  kp.sh = a.stride_head;
  kp.ncache_blocks = a.num_cache_blocks;
  kp.scale = a.softmax_scale;
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
  kp.sqk_dtype = a.sqk_dtype;
  kp.raw = raw;
  kp.multi = multi;
  kp.shared = shared;
  kp.q_stride = (raw ? a.num_heads + a.num_kv_heads : a.num_heads) * HD;
  kp.nsub = raw ? (shared ? a.num_tokens : 1) : 0;

  dim3 grid(a.splits, a.num_kv_heads, a.num_tokens);
  cudaStream_t s = (cudaStream_t)stream;
  if (HD == 64) return dispatch_nt<64>(kp, nt, grid, s);
  if (HD == 128) return dispatch_nt<128>(kp, nt, grid, s);
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
__device__ __align__(256) uint8_t g_static_scratch[DORY_DECODE_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_static_mutex;
void* g_static_ptr[kMaxDevices] = {nullptr};

// Device address of g_static_scratch on the current device, looked up once per device.
int32_t static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(DORY_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (!g_static_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(DORY_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s",
                  cudaGetErrorString(e));
    g_static_ptr[dev] = ptr;
  }
  *out = g_static_ptr[dev];
  return DORY_OK;
}

}  // namespace

extern "C" int32_t dory_decode_attention_static_scratch(const DoryDecodeParams* P, void* stream) {
  if (!P) return fail(DORY_ERR_INVALID_ARGUMENT, "null params");
  if (P->max_tokens < 1 || P->splits < 1 || P->num_heads < 1 || P->num_kv_heads < 1 ||
      P->head_dim < 1)
    return fail(DORY_ERR_INVALID_ARGUMENT, "invalid scratch shape");
  const ScratchLayout SL =
      scratch_layout(P->max_tokens, P->splits, P->num_heads, P->num_kv_heads, P->head_dim);
  if (SL.total > DORY_DECODE_STATIC_SCRATCH_BYTES)
    return fail(DORY_ERR_INVALID_ARGUMENT,
                "this call needs %lld bytes of scratch; the static scratch holds %lld "
                "(use fewer splits or tokens, or dory_decode_attention with caller scratch)",
                (long long)SL.total, (long long)DORY_DECODE_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int32_t st = static_scratch_address(&scratch);
  if (st != DORY_OK) return st;
  // The previous call's counters and error word must not leak into this one.
  cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(SL.pml), (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(DORY_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  DoryDecodeParams a = *P;
  a.scratch = scratch;
  a.scratch_bytes = DORY_DECODE_STATIC_SCRATCH_BYTES;
  return dory_decode_attention(&a, stream);
}
