// cascade.cuh — shared-prefix ("cascade") decode for sm_100a.
//
// Included by decode.cu after decode_mma.cuh: reuses MmaGeom, the copy
// helpers and mma_group.
//
// When every sequence of a batch starts with the same blocks (a radix-cache
// hit: one system prompt, one document, many continuations), the plain decode
// streams that prefix once per sequence — 64 times for BASELINE config 4.  Here
// the prefix is attended once per KV head for all sequences together:
//
//  * The query rows of one KV head are (sequence, q head of the group) pairs,
//    row R = seq * G + g; B * G rows meet the same prefix K/V, so the tile
//    grows past the 16 rows of the per-sequence decode.
//  * CTA = (64-row tile, prefix chunk, kv head).  Warp 4 (the producer) moves
//    the chunk's pages once into a ring of STAGES shared stages (1-D bulk
//    copies, completion on `full[s]`); warps 0-3 each own 16 rows and run the
//    per-group tensor-core math of the decode on every stage, releasing it on
//    `empty[s]` (4 arrivals).  Page ids come from sequence 0's table row; the
//    producer's idle lanes check that the CTA's sequences carry the same ids
//    and flag KVC_STATUS_PREFIX_MISMATCH otherwise.
//  * Each warp writes split-K partials (natural-log max, sum, unnormalised
//    output) of its own rows for partition `chunk`; the tokens after the
//    prefix are partitions prefix_parts.. of the ordinary split-K kernel, and
//    the split-K reduce merges both.
//  * Launch order: this kernel (tensor-core bound), then the tail partitions
//    (HBM bound) as a programmatic dependent so the two run side by side —
//    every tail CTA waits for this grid (griddepcontrol.wait) before it exits
//    — then the reduce, which waits for the tail grid.
//  * P enters the P.V product as one bf16 value (no hi + lo split): over a
//    long shared prefix the rounding of the many terms averages out.
// Every wait is bounded; a timeout sets KVC_STATUS_WAIT_TIMEOUT and an abort
// flag that ends every loop of the CTA.
#pragma once

namespace kvc {

constexpr int kCascadeConsumers = 4;
constexpr int kCascadeRows = 16 * kCascadeConsumers;  // query rows per CTA

template <int D, int BS, int STAGES, int GT>
struct CascadeGeom {
  using Geo = MmaGeom<D, BS, 1, STAGES, GT, kBulk>;  // stage: NBOX K pages, then NBOX V pages
  static constexpr int FULL_OFF = STAGES * Geo::STAGE;
  static constexpr int EMPTY_OFF = FULL_OFF + STAGES * 8;
  static constexpr int MASK_OFF = EMPTY_OFF + STAGES * 8;
  static constexpr int SMEM = MASK_OFF + STAGES * 4;
};

template <typename T, int D, int BS, int STAGES, int GTOK>
__global__ void __launch_bounds__((kCascadeConsumers + 1) * 32)
    cascade_prefix_kernel(DecodeParams p) {
  using namespace mma_detail;
  using CG = CascadeGeom<D, BS, STAGES, GTOK>;
  using Geo = typename CG::Geo;
  constexpr int GT = Geo::GT, NBOX = Geo::NBOX, BOX = Geo::BOX;
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_abort;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + CG::FULL_OFF);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + CG::EMPTY_OFF);
  uint32_t* masks = reinterpret_cast<uint32_t*>(smem + CG::MASK_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, chunk = blockIdx.y, kvh = blockIdx.z;
  const int G = p.num_heads / p.num_kv_heads;
  const int M = p.num_seqs * G;
  const int c_begin = chunk * p.prefix_part_size;
  const int c_end = min(c_begin + p.prefix_part_size, p.prefix_len);
  const int ngroups = (c_end - c_begin + GT - 1) / GT;
  grid_dependents_launch();

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCascadeConsumers);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kCascadeConsumers) {
    // ---- producer: lane 0 streams the chunk's pages (sequence 0's block ids)
    if (lane == 0) {
      const T* kbase = reinterpret_cast<const T*>(p.k_cache) + (int64_t)kvh * p.k_head_stride;
      const T* vbase = reinterpret_cast<const T*>(p.v_cache) + (int64_t)kvh * p.v_head_stride;
      int issued = 0;
      for (int k = 0; k < ngroups; ++k) {
        const int s = k % STAGES;
        if (k >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((k / STAGES) - 1) & 1))) {
          s_abort = 1;
          set_status(&g_decode_status, KVC_STATUS_WAIT_TIMEOUT);
        }
        if (*(volatile int*)&s_abort) break;
        const int t0 = c_begin + k * GT;
        uint32_t mask = 0, bytes = 0;
        uint32_t ids[NBOX];
#pragma unroll
        for (int i = 0; i < NBOX; ++i) {
          ids[i] = 0;
          if (t0 + i * BS < c_end) {
            ids[i] = __ldg(p.block_tables + (t0 + i * BS) / BS);
            if ((int64_t)ids[i] < p.num_blocks) {
              mask |= 1u << i;
              bytes += 2 * BOX;
            } else {
              set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
            }
          }
        }
        masks[s] = mask;
        uint8_t* st = smem + (size_t)s * Geo::STAGE;
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
        ++issued;
      }
      // the CTA's shared memory must outlive every copy: bounded waits on the
      // last phase of each stage issued
      for (int k = issued - STAGES > 0 ? issued - STAGES : 0; k < issued; ++k)
        mbar_wait_bounded(&full[k % STAGES], (uint32_t)((k / STAGES) & 1));
    } else if (kvh == 0) {
      // lanes 1-31: every sequence of this tile must carry sequence 0's block
      // ids over the chunk (the caller's promise; checked once per tile/chunk)
      const int s0 = tile * kCascadeRows / G;
      const int s1 = min((tile + 1) * kCascadeRows, M) - 1;
      const int nseq = s1 / G - s0 + 1;
      const int b0 = c_begin / BS, nb = (c_end + BS - 1) / BS - b0;
      bool bad = false;
      for (int i = lane - 1; i < nseq * nb; i += 31) {
        const int sq = s0 + i / nb, b = b0 + i % nb;
        bad |= __ldg(p.block_tables + (int64_t)sq * p.table_stride + b) != __ldg(p.block_tables + b);
      }
      if (bad) set_status(&g_decode_status, KVC_STATUS_PREFIX_MISMATCH);
    }
    return;
  }

  // ---- consumers: 16 query rows per warp
  const int r = lane >> 2, q4 = lane & 3;
  const int R_lo = tile * kCascadeRows + warp * 16 + r, R_hi = R_lo + 8;
  const int seq_lo = R_lo / G, g_lo = R_lo - seq_lo * G;
  const int seq_hi = R_hi / G, g_hi = R_hi - seq_hi * G;
  auto row_end = [&](int R, int seq) -> int {
    if (R >= M) return 0;
    const uint32_t ctx = __ldg(p.context_lens + seq);
    if (ctx == 0 || ctx > (uint32_t)p.max_seq_len) return 0;
    return (int)ctx < c_end ? (int)ctx : c_end;
  };
  const int end_lo = row_end(R_lo, seq_lo), end_hi = row_end(R_hi, seq_hi);
  uint32_t qa[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const int d0 = ks * 16 + 2 * q4;
    uint32_t v[4] = {0u, 0u, 0u, 0u};
    if (R_lo < M) {
      const T* row = reinterpret_cast<const T*>(p.q) + (int64_t)seq_lo * p.q_seq_stride +
                     (int64_t)(kvh * G + g_lo) * p.q_head_stride;
      v[0] = __ldg(reinterpret_cast<const unsigned int*>(row + d0));
      v[2] = __ldg(reinterpret_cast<const unsigned int*>(row + d0 + 8));
    }
    if (R_hi < M) {
      const T* row = reinterpret_cast<const T*>(p.q) + (int64_t)seq_hi * p.q_seq_stride +
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
    const uint8_t* st = smem + (size_t)s * Geo::STAGE;
    mma_group<T, Geo, D, false>(gs, qa, smem_u32(st), smem_u32(st + NBOX * BOX), c_begin + k * GT, c_end, masks[s],
                                0, qk_scale, false, 0.f, 0.f, lane, end_lo, end_hi);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- partials of this warp's rows for partition `chunk`
  const float l_lo = gs.quad_sum_lo(), l_hi = gs.quad_sum_hi();
  auto write_row = [&](int R, int seq, int g, float m, float l, int half) {
    if (R >= M) return;
    const int head = kvh * G + g;
    float* po = p.part_out + (int64_t)seq * p.part_out_seq_stride + (int64_t)head * p.part_out_head_stride +
                (int64_t)chunk * p.part_out_part_stride;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int d = 8 * nt + 2 * q4;
      po[d] = gs.o[nt][2 * half];
      po[d + 1] = gs.o[nt][2 * half + 1];
    }
    if (q4 == 0) {
      const int64_t o = (int64_t)seq * p.part_seq_stride + (int64_t)head * p.part_head_stride + chunk;
      p.part_max[o] = m * kLn2;  // natural-log units, as the split-K kernels write
      p.part_sum[o] = l;
    }
  };
  write_row(R_lo, seq_lo, g_lo, gs.m_lo, l_lo, 0);
  write_row(R_hi, seq_hi, g_hi, gs.m_hi, l_hi, 1);
}

}  // namespace kvc
