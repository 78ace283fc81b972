/*
 * CPU oracle for the Aegaeon per-token serving path — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load
 * this library, and only as the checker or the timed CPU baseline. The product path
 * (aegaeon_b200) never calls it.
 *
 * Each function restates the reference's algorithm for one operation of the path:
 *   orc_swap               aegaeon/ops/swap.cu:25-60 (per-block copy, block bytes from the
 *                          cache geometry, swap.cu:34)
 *   orc_copy_blocks        vLLM 0.5.1 copy_blocks on whole Aegaeon blocks (no reference call site;
 *                          migration stubs at aegaeon/aegaeon/block_manager.py:876-950)
 *   orc_reshape_and_cache  vLLM 0.5.1 reshape_and_cache_flash as reached from
 *                          aegaeon/aegaeon/worker.py:517-523 with slots from worker.py:628-633
 *   orc_paged_attention    the decode call of vLLM 0.5.1's FlashAttention backend
 *                          (flash_attn_with_kvcache with block_table, causal, one query token),
 *                          with block tables / seq_lens as built at worker.py:640-653
 * vLLM 0.5.1 and vllm-flash-attn are un-vendored pinned dependencies
 * (aegaeon/requirements.txt:9); their published semantics are restated here.
 *
 * Attention is computed in double precision (scores, softmax, weighted sum) from the fp16/bf16
 * storage values and rounded once to the storage type, so it is a tighter reference than the
 * fp32 kernels it checks. Copies move raw 16-bit patterns and are bit-exact.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORC_FP16 = 0, ORC_BF16 = 1 };

static double h2d(uint16_t h) {
  _Float16 f;
  memcpy(&f, &h, 2);
  return (double)f;
}
static double bf2d(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}
static uint16_t d2h(double x) {
  _Float16 f = (_Float16)x; /* correctly rounded, ties to even */
  uint16_t h;
  memcpy(&h, &f, 2);
  return h;
}
static uint16_t d2bf(double x) {
  float f = (float)x;
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb; /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

static double load(const uint16_t* p, int dtype) { return dtype == ORC_BF16 ? bf2d(*p) : h2d(*p); }

int orc_swap(uint8_t* dev_pool, uint8_t* host_pool, size_t block_bytes, const int64_t* src, const int64_t* dst,
             int64_t n, int is_swap_in) {
  for (int64_t i = 0; i < n; ++i) {
    if (is_swap_in)
      memcpy(dev_pool + (size_t)dst[i] * block_bytes, host_pool + (size_t)src[i] * block_bytes, block_bytes);
    else
      memcpy(host_pool + (size_t)dst[i] * block_bytes, dev_pool + (size_t)src[i] * block_bytes, block_bytes);
  }
  return 0;
}

int orc_copy_blocks(uint8_t* pool, size_t block_bytes, const int64_t* src, const int64_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    memmove(pool + (size_t)dst[i] * block_bytes, pool + (size_t)src[i] * block_bytes, block_bytes);
  return 0;
}

int orc_reshape_and_cache(const uint16_t* key, const uint16_t* value, int64_t key_stride, int64_t value_stride,
                          uint16_t* k_cache, uint16_t* v_cache, int64_t block_stride, int64_t num_blocks,
                          const int64_t* slots, int64_t T, int Hkv, int D) {
  const int64_t row = (int64_t)Hkv * D;
  int skipped_out_of_range = 0;
  for (int64_t t = 0; t < T; ++t) {
    const int64_t s = slots[t];
    if (s < 0) continue;
    if (s >= num_blocks * 16) {
      skipped_out_of_range = 1;
      continue;
    }
    const int64_t dst = (s / 16) * block_stride + (s % 16) * row;
    memcpy(k_cache + dst, key + t * key_stride, (size_t)row * 2);
    memcpy(v_cache + dst, value + t * value_stride, (size_t)row * 2);
  }
  return skipped_out_of_range;
}

/* out[b, h, :] for b < B, h < Hq; q/out token strides in elements, head stride D. */
int orc_paged_attention(uint16_t* out, int64_t out_stride, const uint16_t* q, int64_t q_stride,
                        const uint16_t* k_cache, const uint16_t* v_cache, int64_t block_stride,
                        const int32_t* tables, int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv,
                        int D, double scale, int dtype, int num_threads) {
  const int G = Hq / Hkv;
#ifdef _OPENMP
  if (num_threads > 0) omp_set_num_threads(num_threads);
#else
  (void)num_threads;
#endif
#pragma omp parallel
  {
    int cap = 0;
    double* sc = NULL;
    double* acc = (double*)malloc(sizeof(double) * (size_t)D);
    double* qd = (double*)malloc(sizeof(double) * (size_t)D);
#pragma omp for schedule(dynamic, 1) collapse(2)
    for (int b = 0; b < B; ++b) {
      for (int h = 0; h < Hq; ++h) {
        int n = seq_lens[b];
        if (n < 0) n = 0;
        if (n > table_stride * 16) n = table_stride * 16;
        if (n > cap) {
          cap = n;
          sc = (double*)realloc(sc, sizeof(double) * (size_t)cap);
        }
        const int kvh = h / G;
        for (int d = 0; d < D; ++d) qd[d] = load(q + (int64_t)b * q_stride + (int64_t)h * D + d, dtype);
        double mx = -INFINITY;
        for (int j = 0; j < n; ++j) {
          const int64_t blk = tables[(int64_t)b * table_stride + j / 16];
          const uint16_t* kr = k_cache + blk * block_stride + ((int64_t)(j % 16) * Hkv + kvh) * D;
          double s = 0.0;
          for (int d = 0; d < D; ++d) s += qd[d] * load(kr + d, dtype);
          s *= scale;
          sc[j] = s;
          if (s > mx) mx = s;
        }
        double l = 0.0;
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        for (int j = 0; j < n; ++j) {
          const double p = exp(sc[j] - mx);
          l += p;
          const int64_t blk = tables[(int64_t)b * table_stride + j / 16];
          const uint16_t* vr = v_cache + blk * block_stride + ((int64_t)(j % 16) * Hkv + kvh) * D;
          for (int d = 0; d < D; ++d) acc[d] += p * load(vr + d, dtype);
        }
        uint16_t* orow = out + (int64_t)b * out_stride + (int64_t)h * D;
        for (int d = 0; d < D; ++d) {
          const double v = n > 0 ? acc[d] / l : 0.0;
          orow[d] = dtype == ORC_BF16 ? d2bf(v) : d2h(v);
        }
      }
    }
    free(sc);
    free(acc);
    free(qd);
  }
  return 0;
}
