/*
 * The C ABI of libdory_decode.so from plain C (no Python, no torch): what a foreign-function
 * host (cgo, JNI, N-API, a C++ engine) sees through include/dory_decode.h.
 *
 *   - the library's ABI version and struct sizes equal this header's;
 *   - argument errors come back as status codes with a reason, nothing is launched;
 *   - a known answer: a non-raw call (DecodeAttention.__call__) over a paged BF16 cache whose
 *     value rows are all 1.0 returns the gate itself (the softmax weights sum to one), for any
 *     keys, block table and split count; a padding request (seq_len 0) returns 0;
 *   - a known answer of the residual update: a sublayer input and a GEMV output that are both
 *     constant vectors give h = 1 / sqrt(H) everywhere (2^-4 for H = 256, exact in BF16);
 *   - the device error word stays clear.
 *
 * Build and run (tests/test_c_abi.py does this):
 *   gcc -std=c99 -O2 tests/c_abi_check.c -I include -I <cuda>/include \
 *       -L dory-vllm-experiments_b200 -ldory_decode -L <cuda>/lib64 -lcudart \
 *       -Wl,-rpath,<package dir> -Wl,-rpath,<cuda>/lib64 -o c_abi_check
 *   ./c_abi_check        -> prints "c abi ok" and exits 0
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "dory_decode.h"

#define CHECK(cond, ...)                                                  \
  do {                                                                    \
    if (!(cond)) {                                                        \
      fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__);                \
      fprintf(stderr, __VA_ARGS__);                                       \
      fprintf(stderr, "\n");                                              \
      exit(1);                                                            \
    }                                                                     \
  } while (0)
#define CUDA(call) CHECK((call) == cudaSuccess, "%s", #call)

static uint32_t rng = 12345u;
static float uniform(void) {  /* [0, 1) */
  rng = rng * 1664525u + 1013904223u;
  return (float)(rng >> 8) / 16777216.0f;
}
static uint16_t bf16(float x) {  /* round to nearest even (finite inputs) */
  uint32_t u;
  memcpy(&u, &x, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

enum { NH = 32, NKV = 8, HD = 128, Q = NH * HD, B = 16, BLOCKS = 12, SPLITS = 4 };

static int run_call(const DoryDecodeParams* base, int32_t seq_len, float* out_host,
                    void* d_seq, void* d_out, cudaStream_t s) {
  DoryDecodeParams p = *base;
  CUDA(cudaMemcpy(d_seq, &seq_len, 4, cudaMemcpyHostToDevice));
  CUDA(cudaMemset(d_out, 0xff, Q * 4)); /* NaN */
  const int32_t st = dory_decode_attention(&p, (void*)s);
  CHECK(st == DORY_OK, "dory_decode_attention: %d (%s)", st, dory_decode_last_error());
  CUDA(cudaStreamSynchronize(s));
  CUDA(cudaMemcpy(out_host, d_out, Q * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int main(void) {
  /* ---- version and layout ---- */
  CHECK(dory_decode_abi_version() == DORY_DECODE_ABI_VERSION, "ABI version %d != %d",
        dory_decode_abi_version(), DORY_DECODE_ABI_VERSION);
  CHECK(dory_decode_params_bytes() == (int64_t)sizeof(DoryDecodeParams), "DoryDecodeParams size");
  CHECK(dory_qk_norm_params_bytes() == (int64_t)sizeof(DoryQkNormParams), "DoryQkNormParams size");
  CHECK(dory_qkvg_params_bytes() == (int64_t)sizeof(DoryQkvgParams), "DoryQkvgParams size");
  CHECK(dory_residual_params_bytes() == (int64_t)sizeof(DoryResidualParams),
        "DoryResidualParams size");

  /* ---- argument errors: statuses and reasons, nothing launched ---- */
  CHECK(dory_decode_attention(NULL, NULL) == DORY_ERR_INVALID_ARGUMENT, "null params");
  CHECK(strlen(dory_decode_last_error()) > 0, "a reason for the last error");
  DoryDecodeParams bad;
  memset(&bad, 0, sizeof(bad));
  bad.num_heads = 6;
  bad.num_kv_heads = 4; /* not a divisor: the reference's ValueError */
  CHECK(dory_decode_attention(&bad, NULL) == DORY_ERR_INVALID_ARGUMENT,
        "heads not a multiple of kv_heads");
  CHECK(dory_decode_scratch_bytes(1, SPLITS, NH, NKV, HD) > 0, "scratch size");
  DoryResidualParams rbad;
  memset(&rbad, 0, sizeof(rbad));
  rbad.num_tokens = 1;
  rbad.hidden = 12; /* not a multiple of 8 */
  rbad.split_k = 1;
  CHECK(dory_residual_update(&rbad, NULL) == DORY_ERR_INVALID_ARGUMENT, "hidden 12");

  cudaStream_t s;
  CUDA(cudaStreamCreate(&s));
  const int64_t scratch_bytes = dory_decode_scratch_bytes(1, SPLITS, NH, NKV, HD);
  void *d_scratch, *d_key, *d_value, *d_table, *d_seq, *d_q, *d_gate, *d_out;
  const size_t cache_elems = (size_t)BLOCKS * B * NKV * HD;
  CUDA(cudaMalloc(&d_scratch, (size_t)scratch_bytes));
  CUDA(cudaMalloc(&d_key, cache_elems * 2));
  CUDA(cudaMalloc(&d_value, cache_elems * 2));
  CUDA(cudaMalloc(&d_table, BLOCKS * 4));
  CUDA(cudaMalloc(&d_seq, 4));
  CUDA(cudaMalloc(&d_q, Q * 2));
  CUDA(cudaMalloc(&d_gate, Q * 4));
  CUDA(cudaMalloc(&d_out, Q * 4));
  CHECK(dory_decode_scratch_init(d_scratch, scratch_bytes, (void*)s) == DORY_OK, "scratch init");

  /* keys uniform in [-1, 1), values 1.0, a shuffled block table, q small, gate in (0, 1) */
  uint16_t* key = (uint16_t*)malloc(cache_elems * 2);
  uint16_t* value = (uint16_t*)malloc(cache_elems * 2);
  for (size_t i = 0; i < cache_elems; ++i) {
    key[i] = bf16(2.0f * uniform() - 1.0f);
    value[i] = bf16(1.0f);
  }
  int32_t table[BLOCKS];
  for (int i = 0; i < BLOCKS; ++i) table[i] = i;
  for (int i = BLOCKS - 1; i > 0; --i) {
    const int j = (int)(uniform() * (float)(i + 1));
    const int32_t t = table[i];
    table[i] = table[j];
    table[j] = t;
  }
  uint16_t q[Q];
  float gate[Q];
  for (int e = 0; e < Q; ++e) {
    q[e] = bf16(0.2f * (uniform() - 0.5f));
    gate[e] = 0.05f + 0.9f * uniform();
  }
  CUDA(cudaMemcpy(d_key, key, cache_elems * 2, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_value, value, cache_elems * 2, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_table, table, sizeof(table), cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_q, q, sizeof(q), cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_gate, gate, sizeof(gate), cudaMemcpyHostToDevice));

  /* cache views [BLOCKS, B, NKV, HD] (contiguous): strides in elements */
  DoryDecodeParams p;
  memset(&p, 0, sizeof(p));
  p.q = d_q;
  p.key_cache = d_key;
  p.value_cache = d_value;
  p.block_table = (const int32_t*)d_table;
  p.seq_lens = (const int32_t*)d_seq;
  p.gate = (const float*)d_gate;
  p.out_nibble_major = (float*)d_out;
  p.scratch = d_scratch;
  p.scratch_bytes = scratch_bytes;
  p.stride_block = (int64_t)B * NKV * HD;
  p.stride_offset = (int64_t)NKV * HD;
  p.stride_head = HD;
  p.num_cache_blocks = BLOCKS;
  p.softmax_scale = 1.0f / sqrtf((float)HD);
  p.num_tokens = 1;
  p.num_heads = NH;
  p.num_kv_heads = NKV;
  p.head_dim = HD;
  p.block_size = B;
  p.window = 0;
  p.splits = SPLITS;
  p.blocks_per_tile = 1;
  p.min_blocks_per_split = 1;
  p.max_tokens = 1;
  p.sqk_dtype = DORY_DTYPE_F32;
  p.flags = 0; /* non-raw single-token call */

  /* an unsupported head_dim is refused before any launch */
  DoryDecodeParams odd = p;
  odd.head_dim = 96;
  CHECK(dory_decode_attention(&odd, (void*)s) == DORY_ERR_UNSUPPORTED, "head_dim 96");

  float out[Q];
  const int32_t lens[] = {1, 15, 16, 17, 100, 191, BLOCKS * B};
  for (size_t k = 0; k < sizeof(lens) / sizeof(lens[0]); ++k) {
    run_call(&p, lens[k], out, d_seq, d_out, s);
    double worst = 0.0;
    int nan_seen = 0;
    for (int e = 0; e < Q; ++e) {
      const float got = out[(e % 8) * (Q / 8) + e / 8]; /* nibble-major */
      const double err = fabs((double)got - (double)gate[e]) / (double)gate[e];
      if (err != err) nan_seen = 1;
      else if (err > worst) worst = err;
    }
    CHECK(!nan_seen && worst < 1e-2,
          "seq_len %d: output differs from the gate by %.3g (relative), NaN %d", lens[k], worst,
          nan_seen);
  }
  /* padding request: seq_len 0 gives 0 * gate */
  run_call(&p, 0, out, d_seq, d_out, s);
  for (int e = 0; e < Q; ++e) CHECK(out[e] == 0.0f, "padding output %d is %g", e, out[e]);

  uint32_t flags = 1;
  CHECK(dory_decode_fetch_errors(d_scratch, &flags, 1, (void*)s) == DORY_OK, "fetch errors");
  CHECK(flags == 0, "device error word %u", flags);

  /* ---- residual update: constant a (2^-4 in BF16, unit norm at H = 256) and constant
   *      GEMV partials 1.5 + 0.5 over x = sixteen ones give h = 2^-4 ---- */
  enum { RH = 256, RT = 2, RK = 16 };
  float parts[2 * RT * RH], xs[RT * RK], alpha[RH], h_nm[RT * RH];
  uint16_t a_rows[RT * RH], h_rows[RT * RH];
  for (int i = 0; i < RT * RH; ++i) {
    parts[i] = 1.5f;
    parts[RT * RH + i] = 0.5f;
    a_rows[i] = bf16(0.0625f);
  }
  for (int i = 0; i < RT * RK; ++i) xs[i] = 1.0f;
  for (int i = 0; i < RH; ++i) alpha[i] = 0.01f * (float)(i % 7);
  void *d_parts, *d_x, *d_a, *d_alpha, *d_h, *d_hnm;
  CUDA(cudaMalloc(&d_parts, sizeof(parts)));
  CUDA(cudaMalloc(&d_x, sizeof(xs)));
  CUDA(cudaMalloc(&d_a, sizeof(a_rows)));
  CUDA(cudaMalloc(&d_alpha, sizeof(alpha)));
  CUDA(cudaMalloc(&d_h, sizeof(h_rows)));
  CUDA(cudaMalloc(&d_hnm, sizeof(h_nm)));
  CUDA(cudaMemcpy(d_parts, parts, sizeof(parts), cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_x, xs, sizeof(xs), cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_a, a_rows, sizeof(a_rows), cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(d_alpha, alpha, sizeof(alpha), cudaMemcpyHostToDevice));
  DoryResidualParams r;
  memset(&r, 0, sizeof(r));
  r.partials = (const float*)d_parts;
  r.x = (const float*)d_x;
  r.a = d_a;
  r.alpha = d_alpha;
  r.h_out = d_h;
  r.h_out_nibble_major = (float*)d_hnm;
  r.alpha_scale = 2.5f;
  r.eps = 1e-6f;
  r.num_tokens = RT;
  r.hidden = RH;
  r.x_dim = RK;
  r.split_k = 2;
  r.a_dtype = DORY_DTYPE_BF16;
  r.alpha_dtype = DORY_DTYPE_F32;
  const int32_t rs = dory_residual_update(&r, (void*)s);
  CHECK(rs == DORY_OK, "dory_residual_update: %d (%s)", rs, dory_decode_last_error());
  CUDA(cudaStreamSynchronize(s));
  CUDA(cudaMemcpy(h_rows, d_h, sizeof(h_rows), cudaMemcpyDeviceToHost));
  CUDA(cudaMemcpy(h_nm, d_hnm, sizeof(h_nm), cudaMemcpyDeviceToHost));
  for (int i = 0; i < RT * RH; ++i) {
    CHECK(h_rows[i] == bf16(0.0625f), "residual h[%d] bits %04x", i, (unsigned)h_rows[i]);
    CHECK(fabs((double)h_nm[i] - 0.0625) < 1e-7, "residual h_nm[%d] = %.9g", i, h_nm[i]);
  }
  cudaFree(d_parts);
  cudaFree(d_x);
  cudaFree(d_a);
  cudaFree(d_alpha);
  cudaFree(d_h);
  cudaFree(d_hnm);

  free(key);
  free(value);
  cudaFree(d_scratch);
  cudaFree(d_key);
  cudaFree(d_value);
  cudaFree(d_table);
  cudaFree(d_seq);
  cudaFree(d_q);
  cudaFree(d_gate);
  cudaFree(d_out);
  cudaStreamDestroy(s);
  printf("c abi ok\n");
  return 0;
}
