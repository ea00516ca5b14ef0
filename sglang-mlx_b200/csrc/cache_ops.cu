// cache_ops.cu — KV append (reshape_and_cache, vLLM and flash layouts) and the
// pool slot gather of MHATokenPool.fetch, for sm_100a.
//
// All three are HBM-bound copies.  The kernels move data in 16-byte vectors
// where the layout allows and stage the vLLM-layout append through shared
// memory so that tokens landing in the same cache block are written as
// contiguous runs (the value cache is [block, head, dim, offset]: one token
// alone can only write 2-byte pieces at a stride of block_size elements).
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "kvc_common.cuh"

namespace kvc {

// Programmatic dependent launch: the appends let the decode that follows them
// on the stream get its CTAs resident while they run (the decode waits, with
// griddepcontrol.wait, for their completion before it reads anything).
__device__ __forceinline__ void let_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }


__device__ unsigned int g_cache_ops_status = 0;

// ---------------------------------------------------------------------------
// reshape_and_cache (vLLM layout)
//   key_cache   [nb, H, D/x, bs, x]     value_cache [nb, H, D, bs]
// Follows reshape_and_cache.metal:35-69: slot -> (block = slot / bs,
// offset = slot % bs); K element d goes to [block, h, d / x, offset, d % x],
// V element d to [block, h, d, offset]; slot < 0 skips the token.  Index
// arithmetic is 64-bit throughout (the Metal kernel's `int` source offsets
// overflow past 2^31 elements).
// ---------------------------------------------------------------------------
// Tokens per CTA: 32 for prefill-sized appends (long contiguous runs per
// block), 8 for decode-sized ones so that a 256-token append still spreads
// over hundreds of CTAs.
constexpr int kAppendThreads = 256;

struct ReshapeParams {
  const void* key;
  const void* value;
  void* key_cache;
  void* value_cache;
  const void* slots;
  int64_t num_tokens, num_blocks;
  int num_heads, head_size, block_size;
  int64_t key_tok_stride, key_head_stride, value_tok_stride, value_head_stride;
  int64_t kc_block_stride, kc_head_stride, vc_block_stride, vc_head_stride;
  int64_t kc_tok_stride, vc_tok_stride;
  bool slots_i64;
  bool k_vec_store;  // key_cache rows are 16-byte aligned
};

template <typename KV_T, typename CACHE_T, int kTokTile, bool VEC>
__global__ void __launch_bounds__(kAppendThreads) reshape_and_cache_kernel(ReshapeParams p) {
  constexpr int X = 16 / sizeof(CACHE_T);
  constexpr int VPAD = sizeof(CACHE_T) == 2 ? 2 : 1;  // odd word stride for the V tile
  extern __shared__ __align__(16) unsigned char smem_raw[];
  let_dependents_launch();
  __shared__ int64_t s_blk[kTokTile];
  __shared__ int s_off[kTokTile];

  const int D = p.head_size;
  const int kstride = D + X;  // one extra 16-byte chunk: conflict-free 16 B reads per lane
  const int vstride = D + VPAD;
  CACHE_T* ktile = reinterpret_cast<CACHE_T*>(smem_raw);
  CACHE_T* vtile = ktile + kTokTile * kstride;

  const int64_t t0 = (int64_t)blockIdx.x * kTokTile;
  const int h = blockIdx.y;
  const int ntok = (int)(p.num_tokens - t0 < kTokTile ? p.num_tokens - t0 : kTokTile);
  const int tid = threadIdx.x;

  if (tid < kTokTile) {
    int64_t blk = -1;
    int off = 0;
    if (tid < ntok) {
      const int64_t slot = p.slots_i64 ? reinterpret_cast<const int64_t*>(p.slots)[t0 + tid]
                                       : (int64_t)reinterpret_cast<const int32_t*>(p.slots)[t0 + tid];
      if (slot >= 0) {
        blk = slot / p.block_size;
        off = (int)(slot % p.block_size);
        if (blk >= p.num_blocks) {
          set_status(&g_cache_ops_status, KVC_STATUS_SLOT_OOB);
          blk = -1;
        }
      }
    }
    s_blk[tid] = blk;
    s_off[tid] = off;
  }

  // Stage the tile's K and V rows (converted to the cache type) in shared memory.
  const KV_T* key = reinterpret_cast<const KV_T*>(p.key);
  const KV_T* value = reinterpret_cast<const KV_T*>(p.value);
  if (VEC) {
    // 16-byte source loads (host checked alignment of rows and strides)
    constexpr int VIN = 16 / sizeof(KV_T);
    const int nvec = D / VIN;
    for (int i = tid; i < ntok * nvec; i += kAppendThreads) {
      const int t = i / nvec, d = (i - t * nvec) * VIN;
      const int64_t tok = t0 + t;
      const uint4 kr = *reinterpret_cast<const uint4*>(key + tok * p.key_tok_stride + h * p.key_head_stride + d);
      const uint4 vr =
          *reinterpret_cast<const uint4*>(value + tok * p.value_tok_stride + h * p.value_head_stride + d);
      const KV_T* ke = reinterpret_cast<const KV_T*>(&kr);
      const KV_T* ve = reinterpret_cast<const KV_T*>(&vr);
#pragma unroll
      for (int e = 0; e < VIN; ++e) {
        ktile[t * kstride + d + e] = Convert<KV_T, CACHE_T>::apply(ke[e]);
        vtile[t * vstride + d + e] = Convert<KV_T, CACHE_T>::apply(ve[e]);
      }
    }
  } else {
    for (int i = tid; i < ntok * D; i += kAppendThreads) {
      const int t = i / D, d = i - t * D;
      const int64_t tok = t0 + t;
      ktile[t * kstride + d] =
          Convert<KV_T, CACHE_T>::apply(key[tok * p.key_tok_stride + h * p.key_head_stride + d]);
      vtile[t * vstride + d] =
          Convert<KV_T, CACHE_T>::apply(value[tok * p.value_tok_stride + h * p.value_head_stride + d]);
    }
  }
  __syncthreads();

  // K: lane = token, one 16-byte chunk [d/x][offset][0:x] per store.  Tokens
  // at consecutive offsets of one block write one contiguous run.
  CACHE_T* kc = reinterpret_cast<CACHE_T*>(p.key_cache);
  const int nchunk = D / X;
  for (int i = tid; i < kTokTile * nchunk; i += kAppendThreads) {
    const int t = i & (kTokTile - 1), c = i / kTokTile;
    if (t >= ntok) continue;
    const int64_t blk = s_blk[t];
    if (blk < 0) continue;
    CACHE_T* dst = kc + blk * p.kc_block_stride + h * p.kc_head_stride + ((int64_t)c * p.block_size + s_off[t]) * X;
    const CACHE_T* src = ktile + t * kstride + c * X;
    if (p.k_vec_store) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    } else {
#pragma unroll
      for (int e = 0; e < X; ++e) dst[e] = src[e];
    }
  }

  // V: lane = token, element [d][offset].
  CACHE_T* vc = reinterpret_cast<CACHE_T*>(p.value_cache);
  for (int i = tid; i < kTokTile * D; i += kAppendThreads) {
    const int t = i & (kTokTile - 1), d = i / kTokTile;
    if (t >= ntok) continue;
    const int64_t blk = s_blk[t];
    if (blk < 0) continue;
    vc[blk * p.vc_block_stride + h * p.vc_head_stride + (int64_t)d * p.block_size + s_off[t]] = vtile[t * vstride + d];
  }
}

// ---------------------------------------------------------------------------
// Row copies: reshape_and_cache_flash (reshape_and_cache.metal:115-136) and
// the MHATokenPool slot gather (memory_pool.py:139-159).  One (token, head)
// row of D elements per work item; K and V rows in the same launch
// (blockIdx.y selects which).  `dir_store`: destination row is chosen by the
// slot (append); otherwise the source row is chosen by the index (gather).
// ---------------------------------------------------------------------------
struct RowCopyParams {
  const char* src[2];
  char* dst[2];
  const void* index;
  int64_t n_rows_tok;  // tokens (append) or indices (gather)
  int num_heads;
  int row_bytes;       // D * sizeof(T)
  int64_t num_index_targets;  // blocks (append) or slots (gather)
  int block_size;             // append only
  // byte strides
  int64_t src_tok[2], src_head[2];
  int64_t dst_blk[2], dst_tok[2], dst_head[2];
  bool index_i64;
  bool store;  // true = append into cache, false = gather out of pool
};

template <typename VEC>
__global__ void __launch_bounds__(256) row_copy_kernel(RowCopyParams p) {
  let_dependents_launch();
  const int which = blockIdx.y;
  const int vec_per_row = p.row_bytes / (int)sizeof(VEC);
  const int64_t rows = p.n_rows_tok * p.num_heads;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / vec_per_row;
    const int v = (int)(i - row * vec_per_row);
    const int64_t t = row / p.num_heads;
    const int h = (int)(row - t * p.num_heads);
    const int64_t idx = p.index_i64 ? reinterpret_cast<const int64_t*>(p.index)[t]
                                    : (int64_t)reinterpret_cast<const int32_t*>(p.index)[t];
    if (p.store) {
      if (idx < 0) continue;  // reshape_and_cache.metal:117-119
      const int64_t blk = idx / p.block_size, off = idx - blk * p.block_size;
      if (blk >= p.num_index_targets) {
        if (v == 0 && which == 0) set_status(&g_cache_ops_status, KVC_STATUS_SLOT_OOB);
        continue;
      }
      const VEC* s = reinterpret_cast<const VEC*>(p.src[which] + t * p.src_tok[which] + h * p.src_head[which]) + v;
      VEC* d = reinterpret_cast<VEC*>(p.dst[which] + blk * p.dst_blk[which] + off * p.dst_tok[which] +
                                      h * p.dst_head[which]) + v;
      *d = *s;
    } else {
      VEC* d = reinterpret_cast<VEC*>(p.dst[which] + t * p.dst_tok[which] + h * p.dst_head[which]) + v;
      if (idx < 0 || idx >= p.num_index_targets) {
        if (v == 0 && which == 0) set_status(&g_cache_ops_status, KVC_STATUS_INDEX_OOB);
        *d = VEC{};
        continue;
      }
      const VEC* s = reinterpret_cast<const VEC*>(p.src[which] + idx * p.src_tok[which] + h * p.src_head[which]) + v;
      *d = *s;
    }
  }
}

static int sm_count() {
  static std::atomic<int> count[64];  // per device, written once (any racing writer stores the same value)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    count[dev] = n;
  }
  return count[dev];
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static cudaError_t launch_row_copy(RowCopyParams& p, cudaStream_t stream) {
  bool vec16 = (p.row_bytes % 16) == 0;
  bool vec4 = (p.row_bytes % 4) == 0;
  for (int w = 0; w < 2; ++w) {
    const int64_t strides[5] = {p.src_tok[w], p.src_head[w], p.dst_blk[w], p.dst_tok[w], p.dst_head[w]};
    vec16 = vec16 && aligned16(p.src[w]) && aligned16(p.dst[w]);
    vec4 = vec4 && (reinterpret_cast<uintptr_t>(p.src[w]) % 4 == 0) && (reinterpret_cast<uintptr_t>(p.dst[w]) % 4 == 0);
    for (int64_t s : strides) {
      vec16 = vec16 && (s % 16 == 0);
      vec4 = vec4 && (s % 4 == 0);
    }
  }
  const int vbytes = vec16 ? 16 : (vec4 ? 4 : 2);
  const int64_t total = p.n_rows_tok * p.num_heads * (p.row_bytes / vbytes);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  dim3 grid((unsigned)blocks, 2);
  if (vec16)
    row_copy_kernel<uint4><<<grid, threads, 0, stream>>>(p);
  else if (vec4)
    row_copy_kernel<uint32_t><<<grid, threads, 0, stream>>>(p);
  else
    row_copy_kernel<uint16_t><<<grid, threads, 0, stream>>>(p);
  count_launch();
  return cudaGetLastError();
}

template <typename KV_T, typename CACHE_T, int TILE, bool VEC>
static cudaError_t launch_reshape_tile(const ReshapeParams& p, const ReshapeArgs& a, cudaStream_t stream) {
  constexpr int X = 16 / sizeof(CACHE_T);
  constexpr int VPAD = sizeof(CACHE_T) == 2 ? 2 : 1;
  auto kern = reshape_and_cache_kernel<KV_T, CACHE_T, TILE, VEC>;
  const size_t smem = (size_t)TILE * ((a.head_size + X) + (a.head_size + VPAD)) * sizeof(CACHE_T);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((unsigned)((a.num_tokens + TILE - 1) / TILE), (unsigned)a.num_heads);
  kern<<<grid, kAppendThreads, smem, stream>>>(p);
  count_launch();
  return cudaGetLastError();
}

template <typename KV_T, typename CACHE_T>
static cudaError_t launch_reshape_typed(const ReshapeArgs& a, cudaStream_t stream) {
  ReshapeParams p;
  p.key = a.key;
  p.value = a.value;
  p.key_cache = a.key_cache;
  p.value_cache = a.value_cache;
  p.slots = a.slots;
  p.num_tokens = a.num_tokens;
  p.num_blocks = a.num_blocks;
  p.num_heads = a.num_heads;
  p.head_size = a.head_size;
  p.block_size = a.block_size;
  p.key_tok_stride = a.key_tok_stride;
  p.key_head_stride = a.key_head_stride;
  p.value_tok_stride = a.value_tok_stride;
  p.value_head_stride = a.value_head_stride;
  p.kc_block_stride = a.kc_block_stride;
  p.kc_head_stride = a.kc_head_stride;
  p.vc_block_stride = a.vc_block_stride;
  p.vc_head_stride = a.vc_head_stride;
  p.kc_tok_stride = 0;
  p.vc_tok_stride = 0;
  p.slots_i64 = a.slot_type == ElemType::I64;
  constexpr int X = 16 / sizeof(CACHE_T);
  p.k_vec_store = aligned16(a.key_cache) && (a.kc_block_stride % X == 0) && (a.kc_head_stride % X == 0);
  constexpr int VIN = 16 / sizeof(KV_T);
  const bool vec_in = aligned16(a.key) && aligned16(a.value) && a.head_size % VIN == 0 &&
                      a.key_tok_stride % VIN == 0 && a.key_head_stride % VIN == 0 &&
                      a.value_tok_stride % VIN == 0 && a.value_head_stride % VIN == 0;
  if (a.num_tokens <= 4096) {
    return vec_in ? launch_reshape_tile<KV_T, CACHE_T, 8, true>(p, a, stream)
                  : launch_reshape_tile<KV_T, CACHE_T, 8, false>(p, a, stream);
  }
  return vec_in ? launch_reshape_tile<KV_T, CACHE_T, 32, true>(p, a, stream)
                : launch_reshape_tile<KV_T, CACHE_T, 32, false>(p, a, stream);
}

cudaError_t launch_reshape_and_cache(const ReshapeArgs& a, cudaStream_t stream) {
  if (a.num_tokens > (int64_t)INT32_MAX * 8) return cudaErrorInvalidValue;
  switch (a.kv_type) {
    case ElemType::F32:
      if (a.cache_type == ElemType::F32) return launch_reshape_typed<float, float>(a, stream);
      if (a.cache_type == ElemType::F16) return launch_reshape_typed<float, __half>(a, stream);
      if (a.cache_type == ElemType::BF16) return launch_reshape_typed<float, __nv_bfloat16>(a, stream);
      break;
    case ElemType::F16:
      if (a.cache_type == ElemType::F16) return launch_reshape_typed<__half, __half>(a, stream);
      break;
    case ElemType::BF16:
      if (a.cache_type == ElemType::BF16) return launch_reshape_typed<__nv_bfloat16, __nv_bfloat16>(a, stream);
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_reshape_and_cache_flash(const ReshapeArgs& a, cudaStream_t stream) {
  const int es = elem_size(a.kv_type);
  RowCopyParams p;
  p.src[0] = static_cast<const char*>(a.key);
  p.src[1] = static_cast<const char*>(a.value);
  p.dst[0] = static_cast<char*>(a.key_cache);
  p.dst[1] = static_cast<char*>(a.value_cache);
  p.index = a.slots;
  p.n_rows_tok = a.num_tokens;
  p.num_heads = a.num_heads;
  p.row_bytes = a.head_size * es;
  p.num_index_targets = a.num_blocks;
  p.block_size = a.block_size;
  p.src_tok[0] = a.key_tok_stride * es;
  p.src_tok[1] = a.value_tok_stride * es;
  p.src_head[0] = a.key_head_stride * es;
  p.src_head[1] = a.value_head_stride * es;
  p.dst_blk[0] = a.kc_block_stride * es;
  p.dst_blk[1] = a.vc_block_stride * es;
  p.dst_tok[0] = a.kc_tok_stride * es;
  p.dst_tok[1] = a.vc_tok_stride * es;
  p.dst_head[0] = a.kc_head_stride * es;
  p.dst_head[1] = a.vc_head_stride * es;
  p.index_i64 = a.slot_type == ElemType::I64;
  p.store = true;
  return launch_row_copy(p, stream);
}

cudaError_t launch_gather_kv(const GatherArgs& a, cudaStream_t stream) {
  const int es = elem_size(a.type);
  RowCopyParams p;
  p.src[0] = static_cast<const char*>(a.k_buf);
  p.src[1] = static_cast<const char*>(a.v_buf);
  p.dst[0] = static_cast<char*>(a.k_out);
  p.dst[1] = static_cast<char*>(a.v_out);
  p.index = a.indices;
  p.n_rows_tok = a.num_indices;
  p.num_heads = a.num_heads;
  p.row_bytes = a.head_size * es;
  p.num_index_targets = a.num_slots;
  p.block_size = 1;
  p.src_tok[0] = a.kb_slot_stride * es;
  p.src_tok[1] = a.vb_slot_stride * es;
  p.src_head[0] = a.kb_head_stride * es;
  p.src_head[1] = a.vb_head_stride * es;
  p.dst_blk[0] = 0;
  p.dst_blk[1] = 0;
  p.dst_tok[0] = a.ko_tok_stride * es;
  p.dst_tok[1] = a.vo_tok_stride * es;
  p.dst_head[0] = a.ko_head_stride * es;
  p.dst_head[1] = a.vo_head_stride * es;
  p.index_i64 = a.index_type == ElemType::I64;
  p.store = false;
  return launch_row_copy(p, stream);
}

// ---------------------------------------------------------------------------
// FP8 (one-byte) KV cache: quantising append and the elementwise codec.
// Values are quantised as code = encode(x / scale) and read back as
// decode(code) * scale (convert_fp8.metal:28-36).
//
// encode_fp8<.., SAT = false> gives the code float8.metal:69-118
// (detail::fp32_to_fp8) computes, step for step: NaN / Inf codes (:75-79);
// round to nearest even in the normal range with a carry past the last finite
// exponent going to +-Inf (:85-103); +-0 below the smallest subnormal
// (:106-107); otherwise the subnormal branch (:110-116): the mantissa with its
// implicit 1 shifted right by (1 - e) + (23 - MB), rounded half up, keeping
// only the MB mantissa bits.  That branch also takes the values past the last
// finite exponent (E4M3 256 <= |x| < 2^14) and drops a subnormal's carry into
// the smallest normal, as the reference's code does.  Where the reference's
// shift count turns negative (E4M3 |x| >= 2^14, E5M2 |x| >= 2^16; undefined
// behaviour there) the code is +-Inf.
// SAT = true (formats "e4m3-sat" / "e5m2-sat") follows the behaviour the
// reference's comment states instead (:65-68): +-Inf for every value past the
// last finite exponent, and a subnormal that rounds up carries into the
// smallest normal.
// ---------------------------------------------------------------------------
template <int EB, int MB, int BIAS, bool SAT>
__device__ __forceinline__ uint8_t encode_fp8(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint32_t s = (bits >> 31) << 7;
  const uint32_t a = bits & 0x7FFFFFFFu;
  const uint32_t top = ((1u << EB) - 1u) << MB;
  if (a >= 0x7F800000u) return (uint8_t)(s | top | (a != 0x7F800000u ? 1u : 0u));
  const int exp_max = (1 << EB) - 2;
  const int ef = (int)((a >> 23) & 0xFFu) - 127 + BIAS;
  const uint32_t m = a & 0x7FFFFFu;
  if (ef >= 1 && ef <= exp_max) {
    constexpr int SH = 23 - MB;
    uint32_t mant = m >> SH;
    const uint32_t rnd = (m >> (SH - 1)) & 1u;
    const uint32_t sticky = (m & ((1u << (SH - 1)) - 1u)) != 0u;
    mant += rnd & (sticky | (mant & 1u));
    int e = ef;
    if (mant >> MB) {
      mant = 0;
      if (++e > exp_max) return (uint8_t)(s | top);
    }
    return (uint8_t)(s | ((uint32_t)e << MB) | (mant & ((1u << MB) - 1u)));
  }
  if (ef < 1 - MB) return (uint8_t)s;
  const int rshift = (1 - ef) + (23 - MB);
  if (SAT ? ef > exp_max : rshift < 1) return (uint8_t)(s | top);
  const uint32_t rounded = ((0x800000u | m) + (1u << (rshift - 1))) >> rshift;
  return (uint8_t)(s | (SAT ? rounded : (rounded & ((1u << MB) - 1u))));  // SAT: rounded <= 1 << MB
}

template <int EB, int MB, int BIAS>
__device__ __forceinline__ float decode_fp8(uint32_t c) {
  const uint32_t e = (c >> MB) & ((1u << EB) - 1u), m = c & ((1u << MB) - 1u);
  float v;
  if (e == 0) v = ldexpf((float)m / (float)(1u << MB), 1 - BIAS);
  else if (e == (1u << EB) - 1u) v = m ? __int_as_float(0x7FC00000) : __int_as_float(0x7F800000);
  else v = ldexpf(1.f + (float)m / (float)(1u << MB), (int)e - BIAS);
  return (c & 0x80u) ? -v : v;
}

// FMT: 0 E4M3, 1 E5M2 (the reference's encoder), 2 E4M3-sat, 3 E5M2-sat.
template <int FMT>
__device__ __forceinline__ uint8_t fp8_encode(float f) {
  if constexpr (FMT == 0 || FMT == 2) return encode_fp8<4, 3, 7, FMT == 2>(f);
  else return encode_fp8<5, 2, 15, FMT == 3>(f);
}
template <int FMT>
__device__ __forceinline__ float fp8_decode(uint32_t c) {
  if constexpr (FMT == 0 || FMT == 2) return decode_fp8<4, 3, 7>(c);
  else return decode_fp8<5, 2, 15>(c);
}

// Append into one-byte caches in the vLLM layout (x = 16): K [nb, H, D/16, bs,
// 16], V [nb, H, D, bs].  Thread = (token, head, 16-dim chunk): it quantises
// the chunk of K (one 16-byte store) and of V (16 bytes at a stride of bs).
template <typename KV_T, int FMT>
__global__ void __launch_bounds__(256) reshape_and_cache_fp8_kernel(ReshapeArgs a) {
  let_dependents_launch();
  const int chunks = a.head_size / 16;
  const int64_t total = a.num_tokens * a.num_heads * chunks;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = (int)(i % chunks);
  const int h = (int)((i / chunks) % a.num_heads);
  const int64_t t = i / ((int64_t)chunks * a.num_heads);
  const int64_t slot = a.slot_type == ElemType::I64 ? static_cast<const int64_t*>(a.slots)[t]
                                                     : (int64_t) static_cast<const int32_t*>(a.slots)[t];
  if (slot < 0) return;  // reshape_and_cache.metal:36-39
  const int64_t blk = slot / a.block_size, off = slot % a.block_size;
  if (blk >= a.num_blocks) {
    set_status(&g_cache_ops_status, KVC_STATUS_SLOT_OOB);
    return;
  }
  const KV_T* k = static_cast<const KV_T*>(a.key) + t * a.key_tok_stride + h * a.key_head_stride + 16 * c;
  const KV_T* v = static_cast<const KV_T*>(a.value) + t * a.value_tok_stride + h * a.value_head_stride + 16 * c;
  uint32_t kw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int e = 0; e < 16; ++e)
    kw[e >> 2] |= (uint32_t)fp8_encode<FMT>(to_float(k[e]) / a.k_scale) << (8 * (e & 3));
  uint8_t* kc = static_cast<uint8_t*>(a.key_cache) + blk * a.kc_block_stride + h * a.kc_head_stride +
                (int64_t)c * a.block_size * 16 + off * 16;
  *reinterpret_cast<uint4*>(kc) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
  uint8_t* vc = static_cast<uint8_t*>(a.value_cache) + blk * a.vc_block_stride + h * a.vc_head_stride +
                (int64_t)(16 * c) * a.block_size + off;
#pragma unroll
  for (int e = 0; e < 16; ++e) vc[(int64_t)e * a.block_size] = fp8_encode<FMT>(to_float(v[e]) / a.v_scale);
}

template <typename KV_T>
static cudaError_t launch_fp8_append_t(const ReshapeArgs& a, cudaStream_t stream) {
  const int64_t total = a.num_tokens * a.num_heads * (a.head_size / 16);
  if (total == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((total + 255) / 256);
  switch (a.fp8_format) {
    case 1: reshape_and_cache_fp8_kernel<KV_T, 1><<<grid, 256, 0, stream>>>(a); break;
    case 2: reshape_and_cache_fp8_kernel<KV_T, 2><<<grid, 256, 0, stream>>>(a); break;
    case 3: reshape_and_cache_fp8_kernel<KV_T, 3><<<grid, 256, 0, stream>>>(a); break;
    default: reshape_and_cache_fp8_kernel<KV_T, 0><<<grid, 256, 0, stream>>>(a); break;
  }
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_reshape_and_cache_fp8(const ReshapeArgs& a, cudaStream_t stream) {
  if (a.kv_type == ElemType::F32) return launch_fp8_append_t<float>(a, stream);
  if (a.kv_type == ElemType::F16) return launch_fp8_append_t<__half>(a, stream);
  return launch_fp8_append_t<__nv_bfloat16>(a, stream);
}

// convert_fp8.metal:13-80: quantise (float types -> codes), dequantise (codes
// -> float types), rescale codes, or scale between float types; dense arrays.
template <typename SRC, typename DST, int FMT>
__global__ void __launch_bounds__(256) convert_fp8_kernel(const SRC* src, DST* dst, float scale, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (std::is_same<SRC, uint8_t>::value && std::is_same<DST, uint8_t>::value) {
      dst[i] = fp8_encode<FMT>(fp8_decode<FMT>(src[i]) * scale);
    } else if constexpr (std::is_same<SRC, uint8_t>::value) {
      dst[i] = from_float<DST>(fp8_decode<FMT>(src[i]) * scale);
    } else if constexpr (std::is_same<DST, uint8_t>::value) {
      dst[i] = fp8_encode<FMT>(to_float(src[i]) / scale);
    } else {
      dst[i] = from_float<DST>(to_float(src[i]) * scale);
    }
  }
}

template <typename SRC, typename DST>
static cudaError_t launch_convert_t(const void* src, void* dst, float scale, int64_t n, int fmt, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int64_t want = (n + 255) / 256;
  const unsigned grid = (unsigned)(want < 65535 * 8 ? want : 65535 * 8);
  const SRC* s = static_cast<const SRC*>(src);
  DST* d = static_cast<DST*>(dst);
  switch (fmt) {
    case 1: convert_fp8_kernel<SRC, DST, 1><<<grid, 256, 0, stream>>>(s, d, scale, n); break;
    case 2: convert_fp8_kernel<SRC, DST, 2><<<grid, 256, 0, stream>>>(s, d, scale, n); break;
    case 3: convert_fp8_kernel<SRC, DST, 3><<<grid, 256, 0, stream>>>(s, d, scale, n); break;
    default: convert_fp8_kernel<SRC, DST, 0><<<grid, 256, 0, stream>>>(s, d, scale, n); break;
  }
  count_launch();
  return cudaGetLastError();
}

template <typename SRC>
static cudaError_t launch_convert_src(ElemType dt, const void* src, void* dst, float scale, int64_t n, int fmt,
                                      cudaStream_t stream) {
  switch (dt) {
    case ElemType::U8: return launch_convert_t<SRC, uint8_t>(src, dst, scale, n, fmt, stream);
    case ElemType::F32: return launch_convert_t<SRC, float>(src, dst, scale, n, fmt, stream);
    case ElemType::F16: return launch_convert_t<SRC, __half>(src, dst, scale, n, fmt, stream);
    case ElemType::BF16: return launch_convert_t<SRC, __nv_bfloat16>(src, dst, scale, n, fmt, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_convert_fp8(ElemType src_type, ElemType dst_type, const void* src, void* dst, float scale,
                               int64_t n, int fmt, cudaStream_t stream) {
  switch (src_type) {
    case ElemType::U8: return launch_convert_src<uint8_t>(dst_type, src, dst, scale, n, fmt, stream);
    case ElemType::F32: return launch_convert_src<float>(dst_type, src, dst, scale, n, fmt, stream);
    case ElemType::F16: return launch_convert_src<__half>(dst_type, src, dst, scale, n, fmt, stream);
    case ElemType::BF16: return launch_convert_src<__nv_bfloat16>(dst_type, src, dst, scale, n, fmt, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace kvc

unsigned int kvc_cache_ops_status(int clear, cudaError_t* err) {
  unsigned int v = 0;
  *err = cudaMemcpyFromSymbol(&v, kvc::g_cache_ops_status, sizeof(v));
  if (*err == cudaSuccess && clear) {
    const unsigned int zero = 0;
    *err = cudaMemcpyToSymbol(kvc::g_cache_ops_status, &zero, sizeof(zero));
  }
  return v;
}
