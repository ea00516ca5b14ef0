// prefill.cuh — paged prefill / extend attention for sm_100a.
//
// Included by decode.cu after decode_mma.cuh: reuses MmaGeom, the copy
// helpers, GroupState and mma_group.
//
// A prefill (or chunked-prefill "extend") step appends q_len new tokens to a
// sequence whose cache then holds kv_len tokens (the prefix kv_len - q_len,
// then the new ones), and attends every new token to the cache under the
// causal rule of mlx-lm's create_attention_mask with an offset: new token t
// sees cache tokens [0, prefix + t] — and only the last `window` of them
// when a sliding window is set.  The reference builds that mask
// (memory_pool.py:240-270, PooledKVCache.make_mask) and runs the attention as
// mlx SDPA over the K/V that update_and_fetch gathers out of the pool
// (memory_pool.py:205-234); here the attention reads the pool in place.
//
//  * Rows are (new token, query head of the group) pairs of one KV head,
//    row R = t * G + g, so the G heads of a group share every K/V tile.
//  * CTA = (64-row tile, sequence, kv head).  Warp 4 (the producer) streams
//    the sequence's K/V over the tile's key range through a ring of STAGES
//    shared stages (whole pages of the paged layout, or single token rows of
//    the token-major layouts, by 1-D bulk copies; completion on `full[s]`),
//    keeping the block ids of the next kPrefillLookahead groups in registers;
//    warps 0-3 each own 16 rows and run the decode's tensor-core group math
//    on every stage with per-row causal ends (and window starts), releasing
//    the stage on `empty[s]`.
//  * Each warp holds all keys of its rows, so it normalises and stores its
//    rows itself: no split, no cross-warp merge.
//  * Tiles are issued last first (the longest causal ranges start first).
// Every wait is bounded; a timeout sets KVC_STATUS_WAIT_TIMEOUT and an abort
// flag that ends every loop of the CTA.  Inputs the host cannot check (device
// qo_indptr / kv_lens) that are out of range set KVC_STATUS_INDEX_OOB: rows
// past q or past max_q_len are not written, the others of such a sequence
// are zero.
#pragma once

namespace kvc {

using PrefillParams = PrefillArgs;  // (kvc_tensor.h) passed to the kernel as it is

constexpr int kPrefillConsumers = 4;
constexpr int kPrefillRows = 16 * kPrefillConsumers;  // query rows per CTA
constexpr int kPrefillLookahead = 8;                  // groups of block ids held ahead by the producer

template <int D, int BS, int STAGES, int MODE>
struct PrefillGeom {
  using Geo = MmaGeom<D, BS, 1, STAGES, 32, MODE>;  // stage: NBOX K boxes, then NBOX V boxes
  static constexpr int FULL_OFF = STAGES * Geo::STAGE;
  static constexpr int EMPTY_OFF = FULL_OFF + STAGES * 8;
  static constexpr int MASK_OFF = EMPTY_OFF + STAGES * 8;
  static constexpr int SMEM = MASK_OFF + STAGES * 4;
};

template <typename T>
__device__ __forceinline__ uint32_t pack_out(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack_out<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack_out<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// MODE: kBulk (paged layout, BS-token pages) or kFlashBulk (token-major rows;
// BS is then only a template placeholder and p.block_size is read at run time).
template <typename T, int D, int BS, int STAGES, int MODE>
__global__ void __launch_bounds__((kPrefillConsumers + 1) * 32) prefill_kernel(PrefillParams p) {
  using namespace mma_detail;
  using PG = PrefillGeom<D, BS, STAGES, MODE>;
  using Geo = typename PG::Geo;
  constexpr int GT = Geo::GT, NBOX = Geo::NBOX, BOX = Geo::BOX, VBS = Geo::VBS;
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  constexpr bool FLASH = Geo::FLASH;
  constexpr int NID = FLASH ? GT : NBOX;  // block ids per group
  constexpr int LA = kPrefillLookahead;
  static_assert(NID <= 32, "one lane per block id");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_abort;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PG::FULL_OFF);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + PG::EMPTY_OFF);
  uint32_t* masks = reinterpret_cast<uint32_t*>(smem + PG::MASK_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = blockIdx.y, kvh = blockIdx.z;
  const int G = p.num_heads / p.num_kv_heads;
  const int64_t q0 = p.qo_indptr[seq];
  const int64_t q1 = p.qo_indptr[seq + 1];
  const int64_t kvl = p.kv_lens[seq];
  const int64_t ql = q1 - q0;
  const int64_t rows = ql * G;
  const int64_t R0 = (int64_t)(gridDim.x - 1 - blockIdx.x) * kPrefillRows;  // last tiles first
  if (ql <= 0 || R0 >= rows) return;
  // Rows of this tile that the indices put outside q / the table are an input
  // error: flagged once, written as zeros.
  const bool bad = q1 > p.num_tokens || ql > p.max_q_len || kvl < ql ||
                   kvl > p.table_len * (int64_t)p.block_size || kvl > 0x7fffffffll - 64;
  if (bad && threadIdx.x == 0 && blockIdx.x == gridDim.x - 1 && kvh == 0)
    set_status(&g_decode_status, KVC_STATUS_INDEX_OOB);
  const int prefix = bad ? 0 : (int)(kvl - ql);
  const int64_t R_last = (R0 + kPrefillRows < rows ? R0 + kPrefillRows : rows) - 1;
  const int t_first = (int)(R0 / G), t_last = (int)(R_last / G);
  const int kv_end = bad ? 0 : prefix + t_last + 1;
  int kv_beg = p.window > 0 ? prefix + t_first + 1 - p.window : 0;
  kv_beg = kv_beg > 0 ? kv_beg / GT * GT : 0;  // groups start GT-aligned (whole pages)
  const int ngroups = kv_end > kv_beg ? (kv_end - kv_beg + GT - 1) / GT : 0;
  if (q1 > p.num_tokens) return;  // rows outside q / out: nothing may be written

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kPrefillConsumers);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kPrefillConsumers) {
    // ---- producer
    const T* kbase = reinterpret_cast<const T*>(p.k_cache) + (int64_t)kvh * p.k_head_stride;
    const T* vbase = reinterpret_cast<const T*>(p.v_cache) + (int64_t)kvh * p.v_head_stride;
    const uint32_t* table = p.block_tables + (int64_t)seq * p.table_stride;
    // lane i < NID: the block id of token i (token-major) or box i (paged) of group k
    auto load_id = [&](int k) -> uint32_t {
      uint32_t id = 0xffffffffu;
      if (lane < NID && k < ngroups) {
        const int tok = kv_beg + k * GT + lane * VBS;
        if (tok < kv_end) id = __ldg(table + (FLASH ? tok / p.block_size : tok / BS));
      }
      return id;
    };
    auto issue = [&](int k, int s, uint32_t id) {
      const int t0 = kv_beg + k * GT;
      uint8_t* st = smem + (size_t)s * Geo::STAGE;
      if constexpr (FLASH) {
        const int tok = t0 + lane;
        const bool in_range = lane < GT && tok < kv_end;
        const bool ok = in_range && (int64_t)id < p.num_blocks;
        if (in_range && !ok) set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
        const uint32_t mask = __ballot_sync(0xffffffffu, ok);
        if (lane == 0) {
          masks[s] = mask;
          if (mask) mbar_arrive_expect_tx(&full[s], (uint32_t)__popc(mask) * 2u * (uint32_t)Geo::ROWB);
          else mbar_arrive(&full[s]);
        }
        __syncwarp();
        if (ok) {
          const int64_t in_blk = tok % p.block_size;
          bulk_g2s(st + lane * BOX, kbase + (int64_t)id * p.k_block_stride + in_blk * p.k_tok_stride, Geo::ROWB,
                   &full[s]);
          bulk_g2s(st + (NBOX + lane) * BOX, vbase + (int64_t)id * p.v_block_stride + in_blk * p.v_tok_stride,
                   Geo::ROWB, &full[s]);
        }
      } else {
        uint32_t ids[NBOX];
#pragma unroll
        for (int i = 0; i < NBOX; ++i) ids[i] = __shfl_sync(0xffffffffu, id, i);
        if (lane == 0) {
          uint32_t mask = 0, bytes = 0;
#pragma unroll
          for (int i = 0; i < NBOX; ++i) {
            if (t0 + i * VBS < kv_end) {
              if ((int64_t)ids[i] < p.num_blocks) {
                mask |= 1u << i;
                bytes += 2 * BOX;
              } else {
                set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
              }
            }
          }
          masks[s] = mask;
          if (bytes) {
            mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
            for (int i = 0; i < NBOX; ++i) {
              if (mask & (1u << i)) {
                bulk_g2s(st + i * BOX, kbase + (int64_t)ids[i] * p.k_block_stride, BOX, &full[s]);
                bulk_g2s(st + (NBOX + i) * BOX, vbase + (int64_t)ids[i] * p.v_block_stride, BOX, &full[s]);
              }
            }
          } else {
            mbar_arrive(&full[s]);
          }
        }
      }
    };

    uint32_t idq[LA];
#pragma unroll
    for (int u = 0; u < LA; ++u) idq[u] = load_id(u);
    int issued = 0;
    bool stop = false;
    for (int k0 = 0; k0 < ngroups && !stop; k0 += LA) {
#pragma unroll
      for (int u = 0; u < LA; ++u) {
        const int k = k0 + u;
        if (k < ngroups && !stop) {
          const int s = k % STAGES;
          bool ok = true;
          if (k >= STAGES && lane == 0) ok = mbar_wait_bounded(&empty[s], (uint32_t)(((k / STAGES) - 1) & 1));
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            if (lane == 0) {
              s_abort = 1;
              set_status(&g_decode_status, KVC_STATUS_WAIT_TIMEOUT);
            }
            stop = true;
          } else if (__shfl_sync(0xffffffffu, *(volatile int*)&s_abort, 0)) {
            stop = true;
          } else {
            issue(k, s, idq[u]);
            ++issued;
            idq[u] = load_id(k + LA);
          }
        }
      }
    }
    // the CTA's shared memory must outlive every copy: bounded waits on the
    // last phase of each stage issued
    if (lane == 0)
      for (int k = issued - STAGES > 0 ? issued - STAGES : 0; k < issued; ++k)
        mbar_wait_bounded(&full[k % STAGES], (uint32_t)((k / STAGES) & 1));
    return;
  }

  // ---- consumers: 16 query rows per warp
  const int r = lane >> 2, q4 = lane & 3;
  const int64_t R_lo = R0 + warp * 16 + r, R_hi = R_lo + 8;
  const int t_lo = (int)(R_lo / G), g_lo = (int)(R_lo - (int64_t)t_lo * G);
  const int t_hi = (int)(R_hi / G), g_hi = (int)(R_hi - (int64_t)t_hi * G);
  const bool on_lo = R_lo < rows, on_hi = R_hi < rows;
  const int end_lo = on_lo && !bad ? prefix + t_lo + 1 : 0;
  const int end_hi = on_hi && !bad ? prefix + t_hi + 1 : 0;
  const int beg_lo = p.window > 0 ? end_lo - p.window : 0;
  const int beg_hi = p.window > 0 ? end_hi - p.window : 0;
  // key range any row of this warp sees: groups outside it are skipped
  int w_end = end_lo > end_hi ? end_lo : end_hi;
  int w_beg = beg_lo < beg_hi ? beg_lo : beg_hi;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    w_end = max(w_end, __shfl_xor_sync(0xffffffffu, w_end, o));
    w_beg = min(w_beg, __shfl_xor_sync(0xffffffffu, w_beg, o));
  }

  uint32_t qa[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const int d0 = ks * 16 + 2 * q4;
    uint32_t v[4] = {0u, 0u, 0u, 0u};
    if (on_lo) {
      const T* row = reinterpret_cast<const T*>(p.q) + (q0 + t_lo) * p.q_tok_stride +
                     (int64_t)(kvh * G + g_lo) * p.q_head_stride;
      v[0] = __ldg(reinterpret_cast<const unsigned int*>(row + d0));
      v[2] = __ldg(reinterpret_cast<const unsigned int*>(row + d0 + 8));
    }
    if (on_hi) {
      const T* row = reinterpret_cast<const T*>(p.q) + (q0 + t_hi) * p.q_tok_stride +
                     (int64_t)(kvh * G + g_hi) * p.q_head_stride;
      v[1] = __ldg(reinterpret_cast<const unsigned int*>(row + d0));
      v[3] = __ldg(reinterpret_cast<const unsigned int*>(row + d0 + 8));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) qa[ks][i] = v[i];
  }
  const float qk_scale = p.scale * kLog2e;
  GroupState<D> gs;
  gs.reset();
  for (int k = 0; k < ngroups; ++k) {
    const int s = k % STAGES;
    if (*(volatile int*)&s_abort) break;
    if (!mbar_wait_bounded(&full[s], (uint32_t)((k / STAGES) & 1))) {
      if (lane == 0) {
        s_abort = 1;
        set_status(&g_decode_status, KVC_STATUS_WAIT_TIMEOUT);
      }
      break;
    }
    const int tok0 = kv_beg + k * GT;
    if (tok0 < w_end && tok0 + GT > w_beg) {
      const uint8_t* st = smem + (size_t)s * Geo::STAGE;
      // bf16 P keeps the hi + lo split: one bf16 P misses 2e-3 abs / 1e-2 rel on short rows
      mma_group<T, Geo, D>(gs, qa, smem_u32(st), smem_u32(st + NBOX * BOX), tok0, kv_end, masks[s], 0, qk_scale,
                           false, 0.f, 0.f, lane, end_lo, end_hi, beg_lo, beg_hi);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- normalise and store this warp's rows (a row with no visible key is 0)
  const float l_lo = gs.quad_sum_lo(), l_hi = gs.quad_sum_hi();
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  auto store_row = [&](int t, int g, float inv, int half) {
    T* o = reinterpret_cast<T*>(p.out) + (q0 + t) * p.out_tok_stride + (int64_t)(kvh * G + g) * p.out_head_stride;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int d = 8 * nt + 2 * q4;
      *reinterpret_cast<uint32_t*>(o + d) = pack_out<T>(gs.o[nt][2 * half] * inv, gs.o[nt][2 * half + 1] * inv);
    }
  };
  if (on_lo) store_row(t_lo, g_lo, inv_lo, 0);
  if (on_hi) store_row(t_hi, g_hi, inv_hi, 1);
}

template <typename T, int D, int BS, int MODE>
static cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t stream) {
  constexpr int STAGES = 4;
  using PG = PrefillGeom<D, BS, STAGES, MODE>;
  auto kern = prefill_kernel<T, D, BS, STAGES, MODE>;
  static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PG::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int G = p.num_heads / p.num_kv_heads;
  const int64_t tiles = ((int64_t)p.max_q_len * G + kPrefillRows - 1) / kPrefillRows;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffll) return cudaErrorInvalidValue;
  kern<<<dim3((unsigned)tiles, (unsigned)p.num_seqs, (unsigned)p.num_kv_heads), (kPrefillConsumers + 1) * 32, PG::SMEM,
         stream>>>(p);
  count_launch();
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_prefill_layout(const PrefillParams& p, bool token_major, cudaStream_t stream) {
  if (token_major) return launch_prefill<T, D, 16, kFlashBulk>(p, stream);
  if (p.block_size == 8) return launch_prefill<T, D, 8, kBulk>(p, stream);
  if (p.block_size == 16) return launch_prefill<T, D, 16, kBulk>(p, stream);
  if (p.block_size == 32) return launch_prefill<T, D, 32, kBulk>(p, stream);
  return cudaErrorNotSupported;
}

// The mma.sync kernel: every layout, head size 64 / 128.
static cudaError_t launch_prefill_mma_any(const PrefillArgs& a, cudaStream_t stream) {
  if (a.head_size == 128)
    return a.q_type == ElemType::BF16 ? launch_prefill_layout<__nv_bfloat16, 128>(a, a.token_major, stream)
                                      : launch_prefill_layout<__half, 128>(a, a.token_major, stream);
  if (a.head_size == 64)
    return a.q_type == ElemType::BF16 ? launch_prefill_layout<__nv_bfloat16, 64>(a, a.token_major, stream)
                                      : launch_prefill_layout<__half, 64>(a, a.token_major, stream);
  return cudaErrorNotSupported;
}

}  // namespace kvc
