// decode.cu — paged-attention decode for sm_100a: the single-pass form
// (paged_attention_v1), the split-K form with its log-sum-exp reduce, and the
// dispatch between the tensor-core kernel (decode_mma.cuh) and the generic
// CUDA-core kernel below.
//
// Semantics follow paged_attention_kernels.metal:
//   * context_len == 0 or context_len > max_seq_len -> zeros (:45-50)
//   * kv_head = head / (num_heads / num_kv_heads) (:57-58)
//   * logit = scale * q.k (+ alibi_slope * (token - context_len + 1)) (:88-97)
//   * out = sum_t exp(logit_t - max) v_t / (sum_t exp(logit_t - max) + 1e-6) (:122-168)
//   * block tables and context lengths are read as uint32 (:22-23)
// The reference keeps every logit of a sequence in threadgroup memory; here the
// softmax is online (running max / sum per warp, merged across warps), so
// max_seq_len has no shared-memory bound.
#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "kvc_common.cuh"

namespace kvc {

__device__ unsigned int g_decode_status = 0;

struct DecodeParams {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const uint32_t* block_tables;
  const uint32_t* context_lens;
  const float* alibi;
  float* part_max;
  float* part_sum;
  float* part_out;
  int num_seqs, num_heads, num_kv_heads, block_size;
  int max_seq_len, partition_size, num_partitions;
  int heads_per_cta;  // q heads of one KV group handled by one CTA
  int64_t num_blocks;
  int64_t q_seq_stride, q_head_stride, out_seq_stride, out_head_stride;
  int64_t k_block_stride, k_head_stride, v_block_stride, v_head_stride;
  int64_t k_tok_stride, v_tok_stride;  // token-major caches: elements between a block's tokens
  // shared-prefix decode: partitions [0, prefix_parts) are chunks of prefix_part_size tokens of the shared
  // prefix (the cascade kernel writes them); partition prefix_parts + i covers tokens
  // prefix_len + i * partition_size onwards.  part_offset is added to blockIdx.z by the partition kernels.
  int prefix_len, prefix_parts, prefix_part_size, part_offset;
  float k_scale, v_scale;  // one-byte caches: dequantisation scales (value = code * scale)
  int wait_prior_at_end;   // partition kernel: griddepcontrol.wait before exiting (shared-prefix launch order)
  int wait_prior_at_start; // partition kernel launched as a programmatic dependent of the kernel before it
                           // (an append): griddepcontrol.wait before its first global read
  int64_t table_stride;
  int64_t part_seq_stride, part_head_stride;
  int64_t part_out_seq_stride, part_out_head_stride, part_out_part_stride;
  float scale;
  // Planned split-K: CTA i of a 1-D grid runs work item i / num_kv_heads of the
  // plan (kvc_decode_plan) for KV head i % num_kv_heads; a sequence split in
  // several partitions has its partials merged by the CTA that finishes last
  // (plan_counters) when fused_merge is set, else by the reduce kernel.
  const uint32_t* plan_header;
  const uint32_t* plan_items;
  uint32_t* plan_counters;
  int fused_merge;
  // The step's append, folded into the decode (kvc_paged_attention_planned_append):
  // the CTA holding a sequence's last token writes that token's K row and V
  // column to slot slots[seq] before its first cache copy.
  const void* new_k;
  const void* new_v;
  const void* slots;
  int slots_i64;
  int64_t nk_tok_stride, nk_head_stride, nv_tok_stride, nv_head_stride;
};

// Programmatic dependent launch: the partition kernels let the split-K reduce be
// scheduled early; the reduce waits for their completion before reading.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Token range [begin, end) of this CTA's partition; returns false when the
// CTA has nothing to do.  `zero_out` is set when the sequence must produce
// zeros (reference edge rule) and this CTA owns writing them.
__device__ __forceinline__ bool partition_range(const DecodeParams& p, int seq, int part, uint32_t ctx, int* begin,
                                                int* end, bool* zero_out) {
  *zero_out = false;
  if (ctx == 0 || ctx > (uint32_t)p.max_seq_len) {
    // Single pass: this CTA writes the zeros.  Split: the reduce does.
    *zero_out = (p.num_partitions == 1);
    return false;
  }
  if (p.prefix_len > 0) {
    // shared-prefix decode: this kernel only runs the partitions after the prefix
    const int64_t b = (int64_t)p.prefix_len + (int64_t)(part - p.prefix_parts) * p.partition_size;
    if (part < p.prefix_parts || b >= (int64_t)ctx) return false;
    *begin = (int)b;
    const int64_t e = b + p.partition_size;
    *end = (int)((int64_t)ctx < e ? (int64_t)ctx : e);
    return true;
  }
  if (p.num_partitions == 1) {
    *begin = 0;
    *end = (int)ctx;
    return true;
  }
  const int64_t b = (int64_t)part * p.partition_size;
  if (b >= (int64_t)ctx) return false;  // the reduce never reads this partition
  *begin = (int)b;
  const int64_t e = b + p.partition_size;
  *end = (int)((int64_t)ctx < e ? (int64_t)ctx : e);
  return true;
}

template <typename T>
__device__ __forceinline__ void write_zero_heads(const DecodeParams& p, int seq, int h0, int nh, int D) {
  T* out = reinterpret_cast<T*>(p.out);
  for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    out[(int64_t)seq * p.out_seq_stride + (int64_t)(h0 + g) * p.out_head_stride + d] = from_float<T>(0.f);
  }
}

// ---------------------------------------------------------------------------
// Planned split-K (kvc_decode_plan + kvc_paged_attention_planned).
// ---------------------------------------------------------------------------

// The work item of this CTA: false when the CTA has none (past the plan's item
// count, or a plan written for other launch parameters, which is flagged).
__device__ __forceinline__ bool planned_item(const DecodeParams& p, int* kvh, int* seq, int* part) {
  const uint32_t* h = p.plan_header;
  if (h[0] != kPlanMagic || h[1] != (uint32_t)p.num_seqs || h[2] != (uint32_t)p.num_kv_heads ||
      h[3] != (uint32_t)p.max_seq_len || h[4] != (uint32_t)p.partition_size) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(&g_decode_status, KVC_STATUS_PLAN_MISMATCH);
    return false;
  }
  const uint32_t item_idx = blockIdx.x / (uint32_t)p.num_kv_heads;
  if (item_idx >= h[5]) return false;
  const uint32_t item = p.plan_items[item_idx];
  *kvh = (int)(blockIdx.x - item_idx * (uint32_t)p.num_kv_heads);
  *seq = (int)(item & 0xFFFFu);
  *part = (int)(item >> 16);
  return true;
}

// Partitions of a sequence of `ctx` tokens (valid ctx only).
__device__ __forceinline__ int planned_parts(const DecodeParams& p, uint32_t ctx) {
  return (int)((ctx + (uint32_t)p.partition_size - 1) / (uint32_t)p.partition_size);
}

// Merges the `nparts` (<= 32) partials of heads h0 .. h0 + G - 1 of `seq` into
// the output.  Every thread of the CTA calls it; the partials must be visible to
// the CTA, and `scratch` (at least G * 32 + G floats of shared memory) free.
template <typename T>
__device__ __forceinline__ void merge_head_partials(const DecodeParams& p, int seq, int h0, int G, int D, int nparts,
                                                    float* scratch) {
  // weights e^{m_k - M} of every partition, and 1 / (L + 1e-6), per head
  float* w = scratch;                 // [G][32]
  float* inv = scratch + G * 32;      // [G]
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    const int64_t o = (int64_t)seq * p.part_seq_stride + (int64_t)(h0 + g) * p.part_head_stride;
    float M = -INFINITY;
    for (int k = 0; k < nparts; ++k) M = fmaxf(M, __ldcg(p.part_max + o + k));
    float L = 0.f;
    for (int k = 0; k < nparts; ++k) {
      const float mk = __ldcg(p.part_max + o + k);
      const float wt = (M == -INFINITY || mk == -INFINITY) ? 0.f : expf(mk - M);
      w[g * 32 + k] = wt;
      L += wt * __ldcg(p.part_sum + o + k);
    }
    inv[g] = 1.f / (L + 1e-6f);  // paged_attention_kernels.metal:144
  }
  __syncthreads();
  T* out = reinterpret_cast<T*>(p.out);
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    const float* po = p.part_out + (int64_t)seq * p.part_out_seq_stride + (int64_t)(h0 + g) * p.part_out_head_stride + d;
    float a = 0.f;
    for (int k = 0; k < nparts; ++k) a += w[g * 32 + k] * __ldcg(po + (int64_t)k * p.part_out_part_stride);
    out[(int64_t)seq * p.out_seq_stride + (int64_t)(h0 + g) * p.out_head_stride + d] = from_float<T>(a * inv[g]);
  }
}

// Called by every thread of the CTA after it wrote its partition's partials:
// counts the arrival, and the CTA that completes the sequence's set merges
// the `nparts` (<= 32) partials into the output and resets the counter.
template <typename T>
__device__ __forceinline__ void planned_arrive_and_merge(const DecodeParams& p, int seq, int kvh, int h0, int G,
                                                         int D, int nparts, float* scratch) {
  __shared__ uint32_t s_last;
  __threadfence();  // this thread's partials are visible before the arrival below
  __syncthreads();
  uint32_t* counter = p.plan_counters + (int64_t)seq * p.num_kv_heads + kvh;
  if (threadIdx.x == 0) s_last = atomicAdd(counter, 1u) == (uint32_t)(nparts - 1) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  merge_head_partials<T>(p, seq, h0, G, D, nparts, scratch);
  if (threadIdx.x == 0) *counter = 0u;  // ready for the next call with this plan
}

// Writes one merged (max, sum, acc) triple: the final output in single-pass
// mode, the partition's partials in split mode.
template <typename T>
__device__ __forceinline__ void emit(const DecodeParams& p, int seq, int head, int part, int d, float m, float l,
                                     float acc, bool first_d, bool direct) {
  if (direct) {
    T* out = reinterpret_cast<T*>(p.out);
    // paged_attention_kernels.metal:144 — inv_sum = 1 / (sum + 1e-6)
    const float inv = 1.f / (l + 1e-6f);
    out[(int64_t)seq * p.out_seq_stride + (int64_t)head * p.out_head_stride + d] = from_float<T>(acc * inv);
  } else {
    p.part_out[(int64_t)seq * p.part_out_seq_stride + (int64_t)head * p.part_out_head_stride +
               (int64_t)part * p.part_out_part_stride + d] = acc;
    if (first_d) {
      const int64_t o = (int64_t)seq * p.part_seq_stride + (int64_t)head * p.part_head_stride + part;
      p.part_max[o] = m;
      p.part_sum[o] = l;
    }
  }
}

// ---------------------------------------------------------------------------
// Generic CUDA-core kernel: every (query, cache) dtype pair, every head size
// and block size of the validated set, any group size.  fp32 math throughout.
// CTA = (kv head x chunk of up to GC q heads, sequence, partition); each of
// the 4 warps walks every 4th page of the range with its own online softmax.
// ---------------------------------------------------------------------------
constexpr int kGenericWarps = 4;
constexpr int kGenericGC = 8;

template <typename Q_T, typename CACHE_T, int D>
__global__ void __launch_bounds__(kGenericWarps * 32) paged_decode_generic_kernel(DecodeParams p) {
  constexpr int X = 16 / sizeof(CACHE_T);
  constexpr int NCHUNK = D / X;
  constexpr int DPL = (D + 31) / 32;  // output dims per lane
  constexpr int GC = kGenericGC;
  __shared__ float qs[GC][D];
  __shared__ float ps[kGenericWarps][GC][32];
  __shared__ float red_m[kGenericWarps][GC];
  __shared__ float red_l[kGenericWarps][GC];
  __shared__ float red_o[kGenericWarps][GC][D];

  const int G = p.num_heads / p.num_kv_heads;
  const int chunks_per_kv = (G + GC - 1) / GC;
  const int kvh = blockIdx.x / chunks_per_kv;
  const int hc = blockIdx.x - kvh * chunks_per_kv;
  const int h0 = kvh * G + hc * GC;
  const int nh = min(GC, G - hc * GC);
  const int seq = blockIdx.y;
  const int part = blockIdx.z + p.part_offset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bs = p.block_size;
  grid_dependents_launch();  // lets the split-K reduce get scheduled during our tail

  const uint32_t ctx = p.context_lens[seq];
  int begin = 0, end = 0;
  bool zero_out = false;
  if (!partition_range(p, seq, part, ctx, &begin, &end, &zero_out)) {
    if (zero_out) write_zero_heads<Q_T>(p, seq, h0, nh, D);
    return;
  }

  const Q_T* q = reinterpret_cast<const Q_T*>(p.q);
  for (int i = threadIdx.x; i < GC * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    qs[g][d] = g < nh ? to_float(q[(int64_t)seq * p.q_seq_stride + (int64_t)(h0 + g) * p.q_head_stride + d]) : 0.f;
  }
  float slope[GC];
#pragma unroll
  for (int g = 0; g < GC; ++g) slope[g] = (p.alibi && g < nh) ? p.alibi[h0 + g] : 0.f;
  __syncthreads();

  float m[GC], l[GC], o[GC][DPL];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[g][i] = 0.f;
  }

  const CACHE_T* kcache = reinterpret_cast<const CACHE_T*>(p.k_cache);
  const CACHE_T* vcache = reinterpret_cast<const CACHE_T*>(p.v_cache);
  const uint32_t* table = p.block_tables + (int64_t)seq * p.table_stride;
  const int tpl = 32 / bs;  // lanes per token in the QK phase
  const int t = lane % bs, sub = lane / bs;
  const int first_page = begin / bs, last_page = (end - 1) / bs;

  for (int pg = first_page + warp; pg <= last_page; pg += kGenericWarps) {
    const int64_t blk = (int64_t)table[pg];
    const bool blk_ok = blk < p.num_blocks;
    if (!blk_ok) {
      if (lane == 0) set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
      continue;
    }
    // ---- QK: lanes (t, sub) take chunks sub, sub + tpl, ... of token t.
    const CACHE_T* kp = kcache + blk * p.k_block_stride + (int64_t)kvh * p.k_head_stride;
    float acc[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) acc[g] = 0.f;
    for (int c = sub; c < NCHUNK; c += tpl) {
      const uint4 raw = *reinterpret_cast<const uint4*>(kp + ((int64_t)c * bs + t) * X);
      const CACHE_T* kv = reinterpret_cast<const CACHE_T*>(&raw);
#pragma unroll
      for (int e = 0; e < X; ++e) {
        const float kf = to_float(kv[e]);
#pragma unroll
        for (int g = 0; g < GC; ++g) acc[g] += qs[g][c * X + e] * kf;
      }
    }
    for (int off = bs; off < 32; off <<= 1) {
#pragma unroll
      for (int g = 0; g < GC; ++g) acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], off);
    }
    const int token = pg * bs + t;
    const bool valid = token >= begin && token < end;
    float pexp[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      float s = acc[g] * p.scale;
      if (p.alibi) s += slope[g] * (float)(token - (int)ctx + 1);
      s = valid ? s : -INFINITY;
      float pm = s;
      for (int off = 1; off < bs; off <<= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, off));
      const float mn = fmaxf(m[g], pm);
      const float alpha = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
      const float e = valid ? expf(s - mn) : 0.f;
      float es = e;
      for (int off = 1; off < bs; off <<= 1) es += __shfl_xor_sync(0xffffffffu, es, off);
      l[g] = l[g] * alpha + es;
      m[g] = mn;
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[g][i] *= alpha;
      pexp[g] = e;
    }
    if (sub == 0) {
#pragma unroll
      for (int g = 0; g < GC; ++g) ps[warp][g][t] = pexp[g];
    }
    __syncwarp();
    // ---- PV: lane owns dims lane, lane + 32, ...  Tokens past the context
    // are skipped (paged_attention_kernels.metal:154): their slots may hold
    // anything, and 0 * NaN would poison the sum.
    const CACHE_T* vp = vcache + blk * p.v_block_stride + (int64_t)kvh * p.v_head_stride;
    const int nvalid = min(bs, end - pg * bs);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) {
        const CACHE_T* row = vp + (int64_t)d * bs;
        for (int t0 = 0; t0 < bs; t0 += X) {
          const uint4 raw = *reinterpret_cast<const uint4*>(row + t0);
          const CACHE_T* vv = reinterpret_cast<const CACHE_T*>(&raw);
#pragma unroll
          for (int e = 0; e < X; ++e) {
            const float vf = (t0 + e < nvalid) ? to_float(vv[e]) : 0.f;
#pragma unroll
            for (int g = 0; g < GC; ++g) o[g][i] += ps[warp][g][t0 + e] * vf;
          }
        }
      }
    }
    __syncwarp();
  }

  // ---- merge the warps' partial softmax states.
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      red_m[warp][g] = m[g];
      red_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i)
      if (lane + 32 * i < D) red_o[warp][g][lane + 32 * i] = o[g][i];
  __syncthreads();
  for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kGenericWarps; ++w) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kGenericWarps; ++w) {
        const float wt = red_m[w][g] == -INFINITY ? 0.f : expf(red_m[w][g] - M);
        L += wt * red_l[w][g];
        A += wt * red_o[w][g][d];
      }
    }
    emit<Q_T>(p, seq, h0 + g, part, d, M, L, A, d == 0, p.num_partitions == 1);
  }
}

// ---------------------------------------------------------------------------
// Split-K reduce: out = sum_p e^{m_p - M} o_p / (sum_p e^{m_p - M} l_p + 1e-6)
// over the partitions that hold tokens of the sequence, for many partitions
// (long contexts).  CTA = (head, seq, 32-dim slice): lane = dim, warp w
// accumulates partitions w, w + 8, ..., then the 8 partial rows are summed
// through shared memory.  Every CTA recomputes M and the weights from the
// (max, sum) pairs, which are small and L2-resident.  The reduce is a chain of
// dependent memory latencies after the partition kernel ends, so it issues
// its loads before using any: the warp's first kReducePre partial rows and the
// thread's (max, sum) pair go out together, the rest kReduceDepth at a time.
// Launched as a programmatic dependent of the partition kernel: it may start
// during that kernel's tail and waits (griddepcontrol.wait) before reading.
// ---------------------------------------------------------------------------
constexpr int kReduceWarps = 8;
constexpr int kReduceSlice = 32;
constexpr int kReducePre = 16, kReduceDepth = 8;

template <typename T>
__global__ void __launch_bounds__(kReduceWarps * 32) splitk_reduce_kernel(DecodeParams p, int head_size) {
  extern __shared__ float smem_f[];  // w[num_partitions] then acc[kReduceWarps][kReduceSlice]
  __shared__ float red[kReduceWarps];
  __shared__ float s_M, s_inv;
  grid_dependency_wait();
  const int head = blockIdx.x, seq = blockIdx.y;
  const int d = blockIdx.z * kReduceSlice + (threadIdx.x & 31);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ctx = p.context_lens[seq];
  T* out = reinterpret_cast<T*>(p.out) + (int64_t)seq * p.out_seq_stride + (int64_t)head * p.out_head_stride;
  if (ctx == 0 || ctx > (uint32_t)p.max_seq_len) {
    if (warp == 0 && d < head_size) out[d] = from_float<T>(0.f);
    return;
  }
  const int nparts = p.prefix_len > 0
                         ? p.prefix_parts + ((int)ctx > p.prefix_len
                                                 ? (int)((ctx - p.prefix_len + p.partition_size - 1) / p.partition_size)
                                                 : 0)
                         : (int)((ctx + p.partition_size - 1) / p.partition_size);
  const float* pm = p.part_max + (int64_t)seq * p.part_seq_stride + (int64_t)head * p.part_head_stride;
  const float* pl = p.part_sum + (int64_t)seq * p.part_seq_stride + (int64_t)head * p.part_head_stride;
  const float* po = p.part_out + (int64_t)seq * p.part_out_seq_stride + (int64_t)head * p.part_out_head_stride;
  float* w = smem_f;
  float* acc_s = smem_f + ((p.num_partitions + 3) & ~3);
  const bool dim_ok = d < head_size;

  // every load that needs nothing computed first
  float x[kReducePre];
#pragma unroll
  for (int u = 0; u < kReducePre; ++u) {
    const int i = warp + u * kReduceWarps;
    x[u] = (dim_ok && i < nparts) ? po[(int64_t)i * p.part_out_part_stride + d] : 0.f;
  }
  const int i0 = threadIdx.x;
  const float m0 = i0 < nparts ? pm[i0] : -INFINITY, l0 = i0 < nparts ? pl[i0] : 0.f;

  float M = m0;
  for (int i = i0 + blockDim.x; i < nparts; i += blockDim.x) M = fmaxf(M, pm[i]);
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    for (int i = 0; i < kReduceWarps; ++i) v = fmaxf(v, red[i]);
    s_M = v;
  }
  __syncthreads();
  M = s_M;
  float L = 0.f;
  if (i0 < nparts) {
    const float wt = (M == -INFINITY || m0 == -INFINITY) ? 0.f : expf(m0 - M);
    w[i0] = wt;
    L = wt * l0;
  }
  for (int i = i0 + blockDim.x; i < nparts; i += blockDim.x) {
    const float wt = (M == -INFINITY || pm[i] == -INFINITY) ? 0.f : expf(pm[i] - M);
    w[i] = wt;
    L += wt * pl[i];
  }
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  __syncthreads();  // red[] reuse, w[] complete
  if (lane == 0) red[warp] = L;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
    for (int i = 0; i < kReduceWarps; ++i) v += red[i];
    s_inv = 1.f / (v + 1e-6f);
  }
  float a = 0.f;
  if (dim_ok) {
#pragma unroll
    for (int u = 0; u < kReducePre; ++u) {
      const int i = warp + u * kReduceWarps;
      if (i < nparts) a += w[i] * x[u];
    }
    int i = warp + kReducePre * kReduceWarps;
    for (; i + (kReduceDepth - 1) * kReduceWarps < nparts; i += kReduceDepth * kReduceWarps) {
      float y[kReduceDepth];
#pragma unroll
      for (int u = 0; u < kReduceDepth; ++u) y[u] = po[(int64_t)(i + u * kReduceWarps) * p.part_out_part_stride + d];
#pragma unroll
      for (int u = 0; u < kReduceDepth; ++u) a += w[i + u * kReduceWarps] * y[u];
    }
    for (; i < nparts; i += kReduceWarps) a += w[i] * po[(int64_t)i * p.part_out_part_stride + d];
  }
  acc_s[warp * kReduceSlice + lane] = a;
  __syncthreads();
  if (warp == 0 && dim_ok) {
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kReduceWarps; ++k) sum += acc_s[k * kReduceSlice + lane];
    out[d] = from_float<T>(sum * s_inv);
  }
}

}  // namespace kvc

#include "decode_mma.cuh"
#include "cascade.cuh"
#include "prefill.cuh"
#include "prefill_umma.cuh"
#include "prefill_umma_pair.cuh"

namespace kvc {

template <typename Q_T, typename CACHE_T, int D>
static cudaError_t launch_generic(const DecodeParams& p, cudaStream_t stream) {
  const int G = p.num_heads / p.num_kv_heads;
  const int chunks = (G + kGenericGC - 1) / kGenericGC;
  dim3 grid((unsigned)(p.num_kv_heads * chunks), (unsigned)p.num_seqs, (unsigned)(p.num_partitions - p.part_offset));
  paged_decode_generic_kernel<Q_T, CACHE_T, D><<<grid, kGenericWarps * 32, 0, stream>>>(p);
  count_launch();
  return cudaGetLastError();
}

template <typename Q_T, typename CACHE_T>
static cudaError_t launch_generic_d(const DecodeParams& p, int D, cudaStream_t stream) {
  switch (D) {
    case 32: return launch_generic<Q_T, CACHE_T, 32>(p, stream);
    case 64: return launch_generic<Q_T, CACHE_T, 64>(p, stream);
    case 80: return launch_generic<Q_T, CACHE_T, 80>(p, stream);
    case 96: return launch_generic<Q_T, CACHE_T, 96>(p, stream);
    case 112: return launch_generic<Q_T, CACHE_T, 112>(p, stream);
    case 120: return launch_generic<Q_T, CACHE_T, 120>(p, stream);
    case 128: return launch_generic<Q_T, CACHE_T, 128>(p, stream);
    case 192: return launch_generic<Q_T, CACHE_T, 192>(p, stream);
    case 256: return launch_generic<Q_T, CACHE_T, 256>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

// Split-K reduce for few partitions (<= 32): one warp per (sequence, head),
// lanes over the head dimension, partitions walked in order.  Same result as
// splitk_reduce_kernel; a batch of sequences gives thousands of warps, so the
// whole reduce is a couple of memory latencies.
constexpr int kReduceHeadsPerCta = 4;

template <typename T, bool VEC>
__global__ void __launch_bounds__(kReduceHeadsPerCta * 32) splitk_reduce_few_kernel(DecodeParams p, int head_size) {
  grid_dependency_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.x * kReduceHeadsPerCta + warp, seq = blockIdx.y;
  if (head >= p.num_heads) return;
  // Every load is issued before any of them is used (one memory latency, not a
  // chain): the length, lane i's partial max and sum (i < num_partitions <= 32)
  // and this lane's columns of the first PRE partials.  Entries past the
  // sequence's own partitions may be stale; they are selected away below before
  // any arithmetic touches them.
  constexpr int PRE = 8;
  const int NP = p.num_partitions;
  const uint32_t ctx = p.context_lens[seq];
  const float* pm = p.part_max + (int64_t)seq * p.part_seq_stride + (int64_t)head * p.part_head_stride;
  const float* pl = p.part_sum + (int64_t)seq * p.part_seq_stride + (int64_t)head * p.part_head_stride;
  const float* po = p.part_out + (int64_t)seq * p.part_out_seq_stride + (int64_t)head * p.part_out_head_stride;
  const float m_raw = lane < NP ? pm[lane] : -INFINITY;
  const float l_raw = lane < NP ? pl[lane] : 0.f;
  const bool col = VEC && lane < head_size / 4;  // VEC: this lane's first 4 columns (4 * lane ..)
  float4 x[PRE];
#pragma unroll
  for (int i = 0; i < PRE; ++i)
    x[i] = (col && i < NP) ? reinterpret_cast<const float4*>(po + (int64_t)i * p.part_out_part_stride)[lane]
                           : make_float4(0.f, 0.f, 0.f, 0.f);
  T* out = reinterpret_cast<T*>(p.out) + (int64_t)seq * p.out_seq_stride + (int64_t)head * p.out_head_stride;
  if (ctx == 0 || ctx > (uint32_t)p.max_seq_len) {
    for (int d = lane; d < head_size; d += 32) out[d] = from_float<T>(0.f);
    return;
  }
  const int nparts = p.prefix_len > 0
                         ? p.prefix_parts + ((int)ctx > p.prefix_len
                                                 ? (int)((ctx - p.prefix_len + p.partition_size - 1) / p.partition_size)
                                                 : 0)
                         : (int)((ctx + p.partition_size - 1) / p.partition_size);
  const float mi = lane < nparts ? m_raw : -INFINITY;
  float M = mi;
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  // lane i's weight (0 for a partition without keys, or past the sequence)
  const float wi = (M == -INFINITY || mi == -INFINITY) ? 0.f : expf(mi - M);
  float L = lane < nparts ? wi * l_raw : 0.f;
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  const float inv = 1.f / (L + 1e-6f);
  if (VEC) {
    // lane's weight of partition i, broadcast (every lane takes part)
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    auto acc = [&](float4& s4, float w, const float4& y) {
      s4.x += w * y.x;
      s4.y += w * y.y;
      s4.z += w * y.z;
      s4.w += w * y.w;
    };
#pragma unroll
    for (int i = 0; i < PRE; ++i) {
      const float w = __shfl_sync(0xffffffffu, wi, i);
      if (i < nparts) acc(a, w, x[i]);
    }
    for (int i = PRE; i < nparts; ++i) {
      const float w = __shfl_sync(0xffffffffu, wi, i);
      if (col) acc(a, w, reinterpret_cast<const float4*>(po + (int64_t)i * p.part_out_part_stride)[lane]);
    }
    auto store4 = [&](int v4, const float4& s4) {
      out[4 * v4 + 0] = from_float<T>(s4.x * inv);
      out[4 * v4 + 1] = from_float<T>(s4.y * inv);
      out[4 * v4 + 2] = from_float<T>(s4.z * inv);
      out[4 * v4 + 3] = from_float<T>(s4.w * inv);
    };
    if (col) store4(lane, a);
    // head sizes above 128: the further columns, weights read back per partition
    for (int v4 = lane + 32; v4 < head_size / 4; v4 += 32) {
      float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int i = 0; i < nparts; ++i) {
        const float w = (M == -INFINITY || pm[i] == -INFINITY) ? 0.f : expf(pm[i] - M);
        acc(b, w, reinterpret_cast<const float4*>(po + (int64_t)i * p.part_out_part_stride)[v4]);
      }
      store4(v4, b);
    }
  } else {
    for (int d = lane; d < head_size; d += 32) {
      float a = 0.f;
      for (int i = 0; i < nparts; ++i) {
        const float w = (M == -INFINITY || pm[i] == -INFINITY) ? 0.f : expf(pm[i] - M);
        a += w * po[(int64_t)i * p.part_out_part_stride + d];
      }
      out[d] = from_float<T>(a * inv);
    }
  }
}

template <typename KERN>
static cudaError_t launch_pdl(KERN kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              const DecodeParams& p, int D) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, D);
  count_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename Q_T, bool VEC>
static cudaError_t launch_reduce_v(const DecodeParams& p, int D, cudaStream_t stream) {
  if (p.num_partitions <= 32) {
    dim3 grid((unsigned)((p.num_heads + kReduceHeadsPerCta - 1) / kReduceHeadsPerCta), (unsigned)p.num_seqs);
    return launch_pdl(splitk_reduce_few_kernel<Q_T, VEC>, grid, dim3(kReduceHeadsPerCta * 32), 0, stream, p, D);
  }
  auto kern = splitk_reduce_kernel<Q_T>;
  const size_t smem = (size_t)(((p.num_partitions + 3) & ~3) + kReduceWarps * kReduceSlice) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(kern, dim3((unsigned)p.num_heads, (unsigned)p.num_seqs, (unsigned)((D + kReduceSlice - 1) / kReduceSlice)),
                    dim3(kReduceWarps * 32), smem, stream, p, D);
}

template <typename Q_T>
static cudaError_t launch_reduce(const DecodeParams& p, int D, cudaStream_t stream) {
  const bool vec = (D % 4 == 0) && (reinterpret_cast<uintptr_t>(p.part_out) % 16 == 0) &&
                   (p.part_out_seq_stride % 4 == 0) && (p.part_out_head_stride % 4 == 0) &&
                   (p.part_out_part_stride % 4 == 0);
  return vec ? launch_reduce_v<Q_T, true>(p, D, stream) : launch_reduce_v<Q_T, false>(p, D, stream);
}

static DecodeParams to_params(const DecodeArgs& a) {
  DecodeParams p;
  p.out = a.out;
  p.q = a.q;
  p.k_cache = a.k_cache;
  p.v_cache = a.v_cache;
  p.block_tables = a.block_tables;
  p.context_lens = a.context_lens;
  p.alibi = a.alibi;
  p.part_max = a.part_max;
  p.part_sum = a.part_sum;
  p.part_out = a.part_out;
  p.num_seqs = a.num_seqs;
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.block_size = a.block_size;
  p.max_seq_len = a.max_seq_len;
  p.partition_size = a.partition_size;
  p.num_partitions = a.num_partitions;
  p.heads_per_cta = 0;
  p.num_blocks = a.num_blocks;
  p.q_seq_stride = a.q_seq_stride;
  p.q_head_stride = a.q_head_stride;
  p.out_seq_stride = a.out_seq_stride;
  p.out_head_stride = a.out_head_stride;
  p.k_block_stride = a.k_block_stride;
  p.k_head_stride = a.k_head_stride;
  p.v_block_stride = a.v_block_stride;
  p.v_head_stride = a.v_head_stride;
  p.k_tok_stride = a.k_tok_stride;
  p.v_tok_stride = a.v_tok_stride;
  p.prefix_len = a.prefix_len;
  p.prefix_parts = a.prefix_parts;
  p.prefix_part_size = a.prefix_part_size;
  p.part_offset = 0;
  p.wait_prior_at_end = 0;
  p.wait_prior_at_start = 0;
  p.new_k = a.new_k;
  p.new_v = a.new_v;
  p.slots = a.slots;
  p.slots_i64 = a.slot_type == ElemType::I64 ? 1 : 0;
  p.nk_tok_stride = a.nk_tok_stride;
  p.nk_head_stride = a.nk_head_stride;
  p.nv_tok_stride = a.nv_tok_stride;
  p.nv_head_stride = a.nv_head_stride;
  p.k_scale = a.cache_type == ElemType::U8 ? a.k_scale : 1.f;
  p.v_scale = a.cache_type == ElemType::U8 ? a.v_scale : 1.f;
  p.table_stride = a.table_stride;
  p.part_seq_stride = a.part_seq_stride;
  p.part_head_stride = a.part_head_stride;
  p.part_out_seq_stride = a.part_out_seq_stride;
  p.part_out_head_stride = a.part_out_head_stride;
  p.part_out_part_stride = a.part_out_part_stride;
  p.scale = a.scale;
  p.plan_header = a.plan;
  p.plan_items = a.plan ? a.plan + kPlanHeader : nullptr;
  p.plan_counters = a.plan ? a.plan + kPlanHeader + plan_max_items(a.num_seqs, a.max_seq_len, a.partition_size)
                           : nullptr;
  // the CTA that completes a sequence merges its partials when they are few
  p.fused_merge = a.plan && a.num_partitions <= 32 ? 1 : 0;
  return p;
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static bool pages_aligned(const DecodeArgs& a) {
  const int cs = elem_size(a.cache_type);
  return aligned16(a.k_cache) && aligned16(a.v_cache) && (a.k_block_stride * cs) % 16 == 0 &&
         (a.k_head_stride * cs) % 16 == 0 && (a.v_block_stride * cs) % 16 == 0 && (a.v_head_stride * cs) % 16 == 0;
}

cudaError_t launch_paged_decode(const DecodeArgs& a, cudaStream_t stream) {
  if (a.num_seqs > 65535) return cudaErrorInvalidValue;
  // the folded append runs in the tensor-core kernel's paged 16-bit forms, planned,
  // and reads the token's rows as pairs of elements (4-byte aligned rows)
  const bool pairs = a.new_k && (reinterpret_cast<uintptr_t>(a.new_k) & 3u) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.new_v) & 3u) == 0 && ((a.nk_tok_stride | a.nk_head_stride) & 1) == 0 &&
                     ((a.nv_tok_stride | a.nv_head_stride) & 1) == 0;
  if (a.new_k && (!pairs || !a.plan || a.flash || a.cache_type == ElemType::U8 || !mma_supported(a) ||
                  plan_max_items(a.num_seqs, a.max_seq_len, a.partition_size) * a.num_kv_heads > 0x7FFFFFFF))
    return cudaErrorNotSupported;
  DecodeParams p = to_params(a);
  if (a.plan && (!mma_supported(a) ||
                 plan_max_items(a.num_seqs, a.max_seq_len, a.partition_size) * a.num_kv_heads > 0x7FFFFFFF)) {
    // the plan only orders the work: without the tensor-core kernel it runs as plain split-K
    p.plan_header = p.plan_items = nullptr;
    p.plan_counters = nullptr;
    p.fused_merge = 0;
  }
  const int D = a.head_size;
  cudaError_t e = cudaErrorInvalidValue;
  // Loads are 16-byte vectors: page bases must be 16-byte aligned.
  const int cs = elem_size(a.cache_type);
  const bool pages_aligned = aligned16(a.k_cache) && aligned16(a.v_cache) && (a.k_block_stride * cs) % 16 == 0 &&
                             (a.k_head_stride * cs) % 16 == 0 && (a.v_block_stride * cs) % 16 == 0 &&
                             (a.v_head_stride * cs) % 16 == 0 &&
                             (!a.flash || ((a.k_tok_stride * cs) % 16 == 0 && (a.v_tok_stride * cs) % 16 == 0));
  if (!pages_aligned) return cudaErrorMisalignedAddress;
  if ((a.flash || a.cache_type == ElemType::U8) && !mma_supported(a))
    return cudaErrorNotSupported;  // no CUDA-core kernel for these caches
  if (mma_supported(a)) {
    e = launch_mma(p, a, stream);
  } else if (a.q_type == ElemType::F32) {
    if (a.cache_type == ElemType::F32) e = launch_generic_d<float, float>(p, D, stream);
    else if (a.cache_type == ElemType::F16) e = launch_generic_d<float, __half>(p, D, stream);
    else if (a.cache_type == ElemType::BF16) e = launch_generic_d<float, __nv_bfloat16>(p, D, stream);
  } else if (a.q_type == ElemType::F16 && a.cache_type == ElemType::F16) {
    e = launch_generic_d<__half, __half>(p, D, stream);
  } else if (a.q_type == ElemType::BF16 && a.cache_type == ElemType::BF16) {
    e = launch_generic_d<__nv_bfloat16, __nv_bfloat16>(p, D, stream);
  }
  if (e != cudaSuccess || a.num_partitions == 1 || p.fused_merge) return e;
  if (a.q_type == ElemType::F32) return launch_reduce<float>(p, D, stream);
  if (a.q_type == ElemType::F16) return launch_reduce<__half>(p, D, stream);
  return launch_reduce<__nv_bfloat16>(p, D, stream);
}

// ---------------------------------------------------------------------------
// Shared-prefix decode (cascade.cuh): the partitions after the prefix (the
// ordinary split-K partition kernel, offset past the prefix partitions), then
// the prefix kernel as a programmatic dependent that waits for them before it
// exits, then the reduce.  Stage ring: 16-token groups (32 for 32-token
// blocks), 6 stages (4 for 32-token blocks) of K and V pages.
// ---------------------------------------------------------------------------
template <typename T, int D, int BS>
static cudaError_t launch_cascade_prefix(const DecodeParams& p, cudaStream_t stream, bool pdl) {
  constexpr int GT = BS <= 16 ? 16 : 32;
  constexpr int STAGES = BS <= 16 ? 6 : 4;
  using CG = CascadeGeom<D, BS, STAGES, GT>;
  auto kern = cascade_prefix_kernel<T, D, BS, STAGES, GT>;
  static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CG::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int G = p.num_heads / p.num_kv_heads;
  const int64_t rows = (int64_t)p.num_seqs * G;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((rows + kCascadeRows - 1) / kCascadeRows), (unsigned)p.prefix_parts,
                     (unsigned)p.num_kv_heads);
  cfg.blockDim = dim3((kCascadeConsumers + 1) * 32);
  cfg.dynamicSmemBytes = CG::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  count_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename T>
static cudaError_t launch_cascade_prefix_t(const DecodeParams& p, int D, cudaStream_t stream, bool pdl) {
  if (D == 128) {
    if (p.block_size == 8) return launch_cascade_prefix<T, 128, 8>(p, stream, pdl);
    if (p.block_size == 16) return launch_cascade_prefix<T, 128, 16>(p, stream, pdl);
    return launch_cascade_prefix<T, 128, 32>(p, stream, pdl);
  }
  if (p.block_size == 8) return launch_cascade_prefix<T, 64, 8>(p, stream, pdl);
  if (p.block_size == 16) return launch_cascade_prefix<T, 64, 16>(p, stream, pdl);
  return launch_cascade_prefix<T, 64, 32>(p, stream, pdl);
}

cudaError_t launch_paged_decode_cascade(const DecodeArgs& a, cudaStream_t stream) {
  if (a.num_seqs > 65535 || a.prefix_len <= 0 || a.prefix_parts <= 0) return cudaErrorInvalidValue;
  if (!mma_supported(a) || a.alibi != nullptr || a.flash) return cudaErrorNotSupported;
  if (!pages_aligned(a)) return cudaErrorMisalignedAddress;
  DecodeParams p = to_params(a);
  const bool tail = p.num_partitions > p.prefix_parts;
  // the prefix: the tcgen05 kernel where the cache suits it, else the mma.sync one
  cudaError_t e = launch_cascade_prefix_umma(p, a, stream);
  if (e == cudaErrorNotSupported)
    e = a.q_type == ElemType::BF16 ? launch_cascade_prefix_t<__nv_bfloat16>(p, a.head_size, stream, false)
                                   : launch_cascade_prefix_t<__half>(p, a.head_size, stream, false);
  if (e != cudaSuccess) return e;
  if (tail) {
    p.part_offset = p.prefix_parts;
    p.wait_prior_at_end = 1;
    e = launch_mma(p, a, stream);
    if (e != cudaSuccess) return e;
    p.part_offset = 0;
    p.wait_prior_at_end = 0;
  }
  if (a.q_type == ElemType::BF16) return launch_reduce<__nv_bfloat16>(p, a.head_size, stream);
  return launch_reduce<__half>(p, a.head_size, stream);
}

// ---------------------------------------------------------------------------
// Decode plan (kvc_decode_plan): the work items of a split-K decode, longest
// first.  A sequence of C tokens (1 <= C <= max_seq_len) has n = ceil(C / P)
// partitions: n - 1 full ones of P tokens and a last one of C - (n - 1) P;
// a sequence whose length gives zeros (0, or past max_seq_len) gets one
// item of size 0 that writes them.  Items are ordered by size, descending (a
// counting sort over sizes 0..P), so the thread-block scheduler, which starts
// CTAs in index order as slots free up, hands out the long partitions first
// and fills the tail of the launch with the short ones (longest-processing-
// time-first list scheduling).  One CTA of 1024 threads; the size histogram
// (P + 1 counters) lives in shared memory.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

__device__ __forceinline__ void plan_classify(uint32_t C, int max_seq_len, int P, uint32_t* full, uint32_t* last) {
  if (C == 0 || C > (uint32_t)max_seq_len) {  // one item of size 0: writes the zeros
    *full = 0;
    *last = 0;
    return;
  }
  const uint32_t n = (C + (uint32_t)P - 1) / (uint32_t)P;
  *full = n - 1;
  *last = C - (n - 1) * (uint32_t)P;  // 1 .. P
}

__global__ void __launch_bounds__(kPlanThreads) decode_plan_kernel(const uint32_t* __restrict__ lens, int num_seqs,
                                                                   int num_kv_heads, int max_seq_len, int P,
                                                                   uint32_t* __restrict__ plan, int64_t max_items) {
  extern __shared__ uint32_t cursor[];  // [P + 1]: items of each size, then the next free position for that size
  __shared__ uint32_t warp_tot[kPlanThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i <= P; i += kPlanThreads) cursor[i] = 0u;
  __syncthreads();
  for (int b = tid; b < num_seqs; b += kPlanThreads) {
    uint32_t full, last;
    plan_classify(lens[b], max_seq_len, P, &full, &last);
    if (full) atomicAdd(&cursor[P], full);
    atomicAdd(&cursor[last], 1u);
  }
  __syncthreads();
  // exclusive scan in descending size order: thread t owns sizes P - t*K .. P - t*K - K + 1
  const int K = (P + 1 + kPlanThreads - 1) / kPlanThreads;
  uint32_t local = 0;
  for (int j = 0; j < K; ++j) {
    const int sz = P - (tid * K + j);
    if (sz >= 0) local += cursor[sz];
  }
  uint32_t incl = local;
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = warp_tot[lane];
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += u;
    }
    warp_tot[lane] = v;  // inclusive over warps
  }
  __syncthreads();
  uint32_t base = (warp ? warp_tot[warp - 1] : 0u) + incl - local;
  const uint32_t total = warp_tot[kPlanThreads / 32 - 1];
  for (int j = 0; j < K; ++j) {
    const int sz = P - (tid * K + j);
    if (sz >= 0) {
      const uint32_t c = cursor[sz];
      cursor[sz] = base;
      base += c;
    }
  }
  __syncthreads();
  uint32_t* items = plan + kPlanHeader;
  for (int b = tid; b < num_seqs; b += kPlanThreads) {
    uint32_t full, last;
    plan_classify(lens[b], max_seq_len, P, &full, &last);
    if (full) {
      const uint32_t o = atomicAdd(&cursor[P], full);
      for (uint32_t k = 0; k < full; ++k) items[o + k] = (k << 16) | (uint32_t)b;
    }
    items[atomicAdd(&cursor[last], 1u)] = (full << 16) | (uint32_t)b;
  }
  uint32_t* counters = items + max_items;
  const int64_t nc = (int64_t)num_seqs * num_kv_heads;
  for (int64_t i = tid; i < nc; i += kPlanThreads) counters[i] = 0u;
  if (tid == 0) {
    plan[0] = kPlanMagic;
    plan[1] = (uint32_t)num_seqs;
    plan[2] = (uint32_t)num_kv_heads;
    plan[3] = (uint32_t)max_seq_len;
    plan[4] = (uint32_t)P;
    plan[5] = total;
    plan[6] = 0u;
    plan[7] = 0u;
  }
}

cudaError_t launch_decode_plan(const uint32_t* context_lens, int num_seqs, int num_kv_heads, int max_seq_len,
                               int partition_size, uint32_t* plan, cudaStream_t stream) {
  if (num_seqs <= 0 || num_seqs > 65535 || partition_size <= 0 || partition_size > kPlanMaxPartition ||
      max_seq_len <= 0 || (max_seq_len + partition_size - 1) / partition_size > 65535)
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)(partition_size + 1) * sizeof(uint32_t);
  decode_plan_kernel<<<1, kPlanThreads, smem, stream>>>(context_lens, num_seqs, num_kv_heads, max_seq_len,
                                                        partition_size, plan,
                                                        plan_max_items(num_seqs, max_seq_len, partition_size));
  count_launch();
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Scratch of kvc_paged_attention_v2_noalloc: the split-K partials
// [tmp_out | max_logits | exp_sums] of one call, in a static array so callers
// that cannot allocate device memory still get the split-K decode.  Every GPU
// that loads this library holds the array until the process exits; all calls
// on a device share it (overlapping calls race; nothing needs zeroing, every
// partial the reduce reads is written first by the same call).
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_scratch[KVC_NOALLOC_SCRATCH_BYTES / sizeof(float)];

// The current CUDA context (driver entry point looked up through the runtime,
// so the library needs no link against libcuda); nullptr if unavailable.
static void* current_cuda_context() {
  typedef CUresult (*CtxGetCurrent)(CUcontext*);
  static CtxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrent>(f);
  });
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

// Host code must not use g_noalloc_scratch as an address (it names the host
// shadow).  The device address is looked up with cudaGetSymbolAddress, with
// the device current, and cached per device together with the CUDA context it
// belongs to: after cudaDeviceReset (a new context) it is looked up again.
// The lookup may load the module, which must not happen inside a stream
// capture: a first call that finds `stream` capturing gets
// cudaErrorStreamCaptureUnsupported back and nothing is launched.
static float* noalloc_scratch_address(cudaStream_t stream, cudaError_t* err) {
  struct Entry {
    void* ctx;
    float* addr;
  };
  static std::mutex mu;
  static Entry cache[64] = {};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  void* ctx = current_cuda_context();
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].addr != nullptr && cache[dev].ctx == ctx) return cache[dev].addr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone) {
    *err = cudaErrorStreamCaptureUnsupported;
    return nullptr;
  }
  void* p = nullptr;
  *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (*err != cudaSuccess) return nullptr;
  cache[dev].ctx = current_cuda_context();
  cache[dev].addr = static_cast<float*>(p);
  return cache[dev].addr;
}

cudaError_t launch_paged_decode_noalloc(DecodeArgs a, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.num_seqs * a.num_heads * a.num_partitions;
  const int64_t floats = rows * (a.head_size + 2);
  if (floats * (int64_t)sizeof(float) > (int64_t)KVC_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  cudaError_t err = cudaSuccess;
  float* base = noalloc_scratch_address(stream, &err);
  if (base == nullptr) return err;
  // tmp_out first (16-byte rows for the reduce's vector loads), then the two
  // [B, Hq, P] arrays.
  a.part_out = base;
  a.part_out_part_stride = a.head_size;
  a.part_out_head_stride = (int64_t)a.num_partitions * a.head_size;
  a.part_out_seq_stride = (int64_t)a.num_heads * a.part_out_head_stride;
  a.part_max = base + rows * a.head_size;
  a.part_sum = a.part_max + rows;
  a.part_head_stride = a.num_partitions;
  a.part_seq_stride = (int64_t)a.num_heads * a.num_partitions;
  return launch_paged_decode(a, stream);
}

}  // namespace kvc

unsigned int kvc_decode_status(int clear, cudaError_t* err) {
  unsigned int v = 0;
  *err = cudaMemcpyFromSymbol(&v, kvc::g_decode_status, sizeof(v));
  if (*err == cudaSuccess && clear) {
    const unsigned int zero = 0;
    *err = cudaMemcpyToSymbol(kvc::g_decode_status, &zero, sizeof(zero));
  }
  return v;
}
