/*
 * kv_oracle.c — CPU restatement of sglang-mlx's paged-KV decode dataflow.
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU-baseline legs of bench.py as the checker; never part of libkvcache.
 *
 * It restates the reference serving path "gather the sequence's tokens out of
 * the pool, then scaled-dot-product attention" (memory_pool.py:139-159 and
 * bench_paged_vs_gather.py:83-103) over the paged cache layout of
 * paged_attention_kernels.metal, with that kernel's edge rules:
 *   - context_len == 0 or > max_seq_len -> zero output (:45-50)
 *   - kv_head = head / (num_heads / num_kv_heads)       (:57-58)
 *   - logit = scale * q.k + alibi * (t - C + 1)          (:88-97)
 *   - softmax denominator sum + 1e-6                     (:144)
 * Arithmetic is float64.  Parallel over (sequence, kv head) with OpenMP.
 *
 * Element codes: 0 = float32, 1 = float16, 2 = bfloat16 (raw bits in memory).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* IEEE 754 binary16 -> double, decoded field by field. */
static double half_to_double(uint16_t h) {
  const int sign = (h >> 15) & 1;
  const int exp = (h >> 10) & 0x1f;
  const int man = h & 0x3ff;
  double v;
  if (exp == 0) {
    v = ldexp((double)man, -24); /* subnormal: man * 2^-24 */
  } else if (exp == 31) {
    v = man ? NAN : INFINITY;
  } else {
    v = ldexp((double)(man | 0x400), exp - 25);
  }
  return sign ? -v : v;
}

/* bfloat16 is the upper half of a float32. */
static double bf16_to_double(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

static double load(const void* base, int64_t i, int code) {
  switch (code) {
    case 0: return (double)((const float*)base)[i];
    case 1: return half_to_double(((const uint16_t*)base)[i]);
    default: return bf16_to_double(((const uint16_t*)base)[i]);
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/*
 * out [B, Hq, D] float64.  key_cache [nb, Hkv, D/x, bs, x], value_cache
 * [nb, Hkv, D, bs] (dense), block_tables [B, max_blocks] (uint32 values),
 * context_lens [B].  seq_begin/seq_end restrict the work to a range of
 * sequences (the CPU baseline times a bounded sample).  threads <= 0: all.
 */
int oracle_paged_attention(double* out, const void* query, int q_code, const void* key_cache,
                           const void* value_cache, int cache_code, const uint32_t* block_tables,
                           const uint32_t* context_lens, int B, int Hq, int Hkv, int D, int bs, int max_blocks,
                           int max_seq_len, double scale, const float* alibi, int seq_begin, int seq_end,
                           int threads) {
  if (Hkv <= 0 || Hq % Hkv != 0 || D <= 0 || bs <= 0) return 1;
  const int G = Hq / Hkv;
  const int x = (cache_code == 0) ? 4 : 8;
  if (D % x != 0) return 1;
  if (seq_begin < 0) seq_begin = 0;
  if (seq_end > B || seq_end < 0) seq_end = B;
  const int64_t page = (int64_t)D * bs;
  const int64_t k_head_stride = page, k_block_stride = (int64_t)Hkv * page;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  int bad = 0;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = seq_begin; b < seq_end; ++b) {
    for (int kvh = 0; kvh < Hkv; ++kvh) {
      const uint32_t C = context_lens[b];
      double* o = out + ((int64_t)b * Hq + (int64_t)kvh * G) * D;
      if (C == 0 || C > (uint32_t)max_seq_len) {
        memset(o, 0, sizeof(double) * (size_t)G * D);
        continue;
      }
      /* gather: contiguous [C, D] K and V (memory_pool.py:149-152) */
      double* k = (double*)malloc(sizeof(double) * (size_t)C * D);
      double* v = (double*)malloc(sizeof(double) * (size_t)C * D);
      double* logits = (double*)malloc(sizeof(double) * (size_t)C);
      if (!k || !v || !logits) {
        free(k), free(v), free(logits);
#pragma omp atomic write
        bad = 1;
        continue;
      }
      for (uint32_t t = 0; t < C; ++t) {
        const int64_t blk = (int64_t)block_tables[(int64_t)b * max_blocks + t / bs];
        const int off = (int)(t % bs);
        const int64_t kb = blk * k_block_stride + kvh * k_head_stride;
        for (int d = 0; d < D; ++d) {
          k[(int64_t)t * D + d] = load(key_cache, kb + ((int64_t)(d / x) * bs + off) * x + d % x, cache_code);
          v[(int64_t)t * D + d] = load(value_cache, kb + (int64_t)d * bs + off, cache_code);
        }
      }
      /* SDPA per q head of the group */
      for (int g = 0; g < G; ++g) {
        const int h = kvh * G + g;
        const int64_t qo = ((int64_t)b * Hq + h) * D;
        double qv[512];
        for (int d = 0; d < D && d < 512; ++d) qv[d] = load(query, qo + d, q_code);
        const double slope = alibi ? (double)alibi[h] : 0.0;
        double m = -INFINITY;
        for (uint32_t t = 0; t < C; ++t) {
          double s = 0.0;
          const double* kr = k + (int64_t)t * D;
          for (int d = 0; d < D; ++d) s += qv[d] * kr[d];
          s *= scale;
          if (slope != 0.0) s += slope * ((double)t - (double)C + 1.0);
          logits[t] = s;
          if (s > m) m = s;
        }
        double sum = 0.0;
        for (uint32_t t = 0; t < C; ++t) {
          logits[t] = exp(logits[t] - m);
          sum += logits[t];
        }
        const double inv = 1.0 / (sum + 1e-6);
        double* orow = o + (int64_t)g * D;
        for (int d = 0; d < D; ++d) orow[d] = 0.0;
        for (uint32_t t = 0; t < C; ++t) {
          const double p = logits[t] * inv;
          const double* vr = v + (int64_t)t * D;
          for (int d = 0; d < D; ++d) orow[d] += p * vr[d];
        }
      }
      free(k);
      free(v);
      free(logits);
    }
  }
  return bad;
}

/*
 * reshape_and_cache (reshape_and_cache.metal:35-69) on raw element bits of
 * width `esize` (the caller converts dtypes first): key/value [T, H, D]
 * dense, caches in the vLLM layout, slots int64; slot < 0 skipped.
 */
int oracle_reshape_and_cache(const void* key, const void* value, void* key_cache, void* value_cache,
                             const int64_t* slots, int64_t T, int H, int D, int bs, int x, int esize,
                             int64_t num_blocks) {
  for (int64_t t = 0; t < T; ++t) {
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    const int64_t blk = slot / bs, off = slot % bs;
    if (blk >= num_blocks) return 1;
    for (int h = 0; h < H; ++h) {
      for (int d = 0; d < D; ++d) {
        const int64_t src = (t * H + h) * D + d;
        const int64_t kd = ((blk * H + h) * (D / x) + d / x) * (int64_t)bs * x + off * x + d % x;
        const int64_t vd = ((blk * H + h) * (int64_t)D + d) * bs + off;
        memcpy((char*)key_cache + kd * esize, (const char*)key + src * esize, (size_t)esize);
        memcpy((char*)value_cache + vd * esize, (const char*)value + src * esize, (size_t)esize);
      }
    }
  }
  return 0;
}
