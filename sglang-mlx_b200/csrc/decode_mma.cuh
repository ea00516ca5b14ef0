// decode_mma.cuh — tensor-core paged decode for sm_100a (f16/f16 and bf16/bf16).
//
// Included by decode.cu (shares DecodeParams, partition_range, the status word).
//
// CTA = (kv head, sequence, partition).  All G = num_heads / num_kv_heads query
// heads of the KV group are the M rows of one m16n8k16 tile (G <= 16), so each
// K/V page is fetched from HBM once for the whole group (the reference's grid
// is per query head and re-reads every page G times,
// paged_attention_kernels.metal:81-83).
//
// Data movement: each warp owns a ring of STAGES shared-memory stages.  A stage
// holds one 32-token group: 32/BS pages of K ([D/8][BS][8] elements, 16-byte
// rows per token) and of V ([D][BS]).  Pages are contiguous in HBM, so one lane
// moves each with a single CTA-local 1-D bulk copy (cp.async.bulk) that
// completes on the stage's mbarrier; STAGES-1 groups stay in flight while the
// warp computes on the current one.
//
// Math per group (natural token order):
//   S[head][tok] = sum_d Q[head][d] K[tok][d]   A = Q (registers, loaded once),
//       B = K^T via ldmatrix on the [D/8][BS][8] page: 8 tokens x 16 B rows.
//   online softmax in the log2 domain (row max across the quad of lanes that
//       share a head), masked tokens -> -inf.
//   O[head][d] += P[head][tok] V[tok][d]        A = P taken straight from the S
//       accumulators (two 8-token tiles form one 16-token k-step), B = V via
//       ldmatrix on the [D][BS] page: 8 dims x 16 B (8 tokens) rows.
// fp32 accumulation everywhere.  P enters the second product as f16, or for
// bf16 as a hi + lo pair of bf16 values (about 16 bits), close to the
// reference's fp32 P.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

namespace kvc {
namespace mma_detail {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase with `parity` to complete; gives up after ~1 s of wall
// time (returns false) so a lost transfer can never hang the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_timer_ns() - t0 > 1000000000ull) return false;
  }
}

// 16-byte global -> shared copy (L2 only); completion is reported to an
// mbarrier by cp_async_arrive.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// The same with `src_bytes` (0 or 16) read and the rest of the 16 bytes
// zero-filled: a masked copy without a branch (src must still be mapped).
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// One arrival on `bar` once every cp.async this thread issued before has
// completed (the barrier's expected count includes it).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Tiled tensor copies global -> shared (this CTA only), completion counted on
// `bar`.  Coordinates are innermost first.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Four rows (row0..row3 of a 2-D tensor map whose box is one row high) land
// one after another at `dst`.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int col, int row0, int row1, int row2,
                                            int row3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(col), "r"(row0), "r"(row1), "r"(row2), "r"(row3)
      : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transposing form: each lane's address is a row of 8 consecutive 16-bit
// elements; every 8x8 matrix is delivered transposed.
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  // (x0, x1) = hi + lo with hi = bf16(x) and lo = bf16(x - hi).
  static constexpr bool kSplitP = true;
  __device__ __forceinline__ static void pack_split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};
template <> struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static constexpr bool kSplitP = false;
  __device__ __forceinline__ static void pack_split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    hi = pack(x0, x1);
    lo = 0u;
  }
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two fp32 lanes per instruction (the f32x2 arithmetic of sm_100): the same
// round-to-nearest results as two scalar operations.
__device__ __forceinline__ float2 fma_x2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add_x2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nadd.rn.f32x2 rd, ra, rb;\n"
      "mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 sub_x2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nsub.rn.f32x2 rd, ra, rb;\n"
      "mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace mma_detail

// How a group's K and V reach shared memory, in "boxes" of VBS tokens:
//  kBulk      1-D bulk copies of whole pages (VBS = BS, so GT >= BS).
//  kTiles     tiled tensor copies of VBS = min(GT, BS) tokens: a 16-token box
//             of a 32-token page lands densely as [D/8][16][8] (K) and [D][16]
//             (V); the V box carries the 32/64-byte swizzle.
//  kSwizzledV K by 1-D bulk copy; V as a whole page through a tensor map that
//             views it as 128-byte rows, written with the 128-byte swizzle.
//  kFlash     token-major caches ([nb, bs, H, D], the MHATokenPool buffers
//             being bs = 1): every token's K row and V row (D * 2 bytes) is
//             copied by 16-byte cp.async spread over the warp, landing in a
//             shared row of D * 2 + 16 bytes (the 16-byte pad spreads the
//             ldmatrix rows of 8 tokens over all banks); V is read with
//             ldmatrix.trans.  A "box" is one token, so the stage mask has a
//             bit per token.
//  kFlashBulk the same rows, each its own 1-D bulk copy issued by the lane of
//             its token.
// A swizzled V box makes the ldmatrix reads of V rows (VBS * 2 bytes apart)
// hit distinct banks.
//  kFp8E4M3 / kFp8E5M2  one-byte caches in the paged layout (K pages
//             [D/16][bs][16], V pages [D][bs] bytes), 1-D bulk copies of whole
//             pages; mma_group_fp8 converts codes to f16 in registers.
//  kFlashTma  token-major caches whose blocks hold a multiple of 16 tokens in
//             consecutive rows ([nb, bs, H, D] with dense blocks, or a token pool
//             handing out whole pages): a group's GT rows of one head are one
//             tiled tensor copy per 64 dims, landing as GT rows of 128 bytes with
//             the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)),
//             K and V both read with ldmatrix (V transposed).  One copy per
//             (group, head, 64 dims) instead of a 16-byte cp.async per lane and row.
//  kFlashGather  token-major caches whose rows are dense ([slots, H, D] of the
//             token pool's slot lists, or [nb, bs, H, D] with any bs): the same
//             shared layout as kFlashTma, each token's row fetched where its own
//             slot is by 4-row tensor gathers (tile::gather4, 64 dims per
//             request): 16 requests per 16-token group and head at D = 128.
//             The stage mask has a bit per token; a token past the context or
//             with a bad slot gathers a valid token's row and is masked.
constexpr int kBulk = 0, kTiles = 1, kSwizzledV = 2, kFlash = 3, kFp8E4M3 = 4, kFp8E5M2 = 5, kFlashBulk = 6,
              kFlashTma = 7, kFlashGather = 8;

template <int D, int BS, int NW, int STAGES, int GT_ = 32, int MODE = kBulk>
struct MmaGeom {
  static constexpr int GT = GT_;                          // tokens per group (16, 32 or 64)
  static constexpr bool FLASH = MODE == kFlash || MODE == kFlashBulk;  // token-major K/V rows
  static constexpr bool CP_ASYNC = MODE == kFlash;        // stage completion: 32 cp.async arrivals
  static constexpr bool FP8 = MODE == kFp8E4M3 || MODE == kFp8E5M2;  // one-byte caches
  static constexpr bool GATHER = MODE == kFlashGather;   // token rows by 4-row tensor gathers
  static constexpr bool TROWS = MODE == kFlashTma || GATHER;  // token rows as swizzled 128-byte halves
  static constexpr bool TOKIDS = FLASH || GATHER;         // a block id per token (the id chunks)
  static constexpr int VBS = FLASH ? 1 : (TROWS ? GT : (MODE == kTiles ? (GT < BS ? GT : BS) : BS));  // tokens per box
  static constexpr int NBOX = GT / VBS;                   // boxes per group (K and V each)
  static constexpr int MBS = GATHER ? 1 : VBS;            // tokens per stage-mask bit
  static constexpr int NMB = GT / MBS;                    // mask bits per group
  static constexpr uint32_t FULL_MASK = NMB >= 32 ? 0xffffffffu : (1u << (NMB & 31)) - 1u;  // everything loaded
  static_assert(GT % 16 == 0 && GT % VBS == 0, "a group is whole boxes and whole 16-token k-steps");
  static_assert(!FLASH || GT == 16 || GT == 32, "token-major groups are 16 or 32 tokens (one mask bit per token)");
  static constexpr int ROWB = D * 2;                      // bytes of one token row (kFlash)
  static constexpr int BOX = FLASH ? ROWB + 16 : D * VBS * (FP8 ? 1 : 2);  // bytes (stride) of one K (or V) box
  static constexpr int VSWZ = MODE == kSwizzledV ? 128 : (MODE == kTiles && VBS * 2 >= 32 ? VBS * 2 : 0);
  static constexpr int STAGE = NBOX * 2 * BOX;            // K boxes then V boxes
  static constexpr int ALIGN = (MODE == kTiles || MODE == kSwizzledV || TROWS) ? 1024 : 0;  // ring alignment (swizzle atoms)
  static constexpr int RING = NW * STAGES * STAGE;
  static constexpr int BAR_OFF = ALIGN + RING;            // NW*STAGES mbarriers
  static constexpr int MASK_OFF = BAR_OFF + NW * STAGES * 8;
  static constexpr int COMBINE = NW * 16 * D * 4 + NW * 16 * 2 * 4;  // reuses the ring
  // kFlash: per warp, the block ids of two chunks of IDC groups (one id per
  // token), filled a chunk ahead of the copies that use them
  static constexpr int IDC = 8;
  static constexpr int IDS_OFF = (MASK_OFF + NW * STAGES * 4 + 15) / 16 * 16;
  static constexpr int SMEM = IDS_OFF + (TOKIDS ? NW * 2 * IDC * GT * 4 : 0);
  static_assert(!TOKIDS || (STAGES <= IDC && (IDC * GT) % 32 == 0), "id chunks cover the ring");
  static_assert(!GATHER || GT == 16, "a gathered group is 16 tokens (4 requests of 4 rows per 64 dims)");
  static_assert(COMBINE <= RING, "combine buffer must fit in the ring");
};

// Tensor maps of one launch (tensor-copy modes only).  kTiles: K as
// [nb][H][D/8][BS][8] and V as [nb][H][D][BS]; kSwizzledV: V as
// [nb][H][D*BS/64][64] (128-byte rows); innermost last in these brackets.
struct TmaMaps {
  CUtensorMap k;
  CUtensorMap v;
};

// Online-softmax state of one warp over the rows r (lo) and r + 8 (hi) of its
// 16-row tile: running max (log2 units), this lane's share of the row sums,
// and the unnormalised output accumulators (the P.V C fragments).
template <int D>
struct GroupState {
  float m_lo, m_hi, l_lo, l_hi;
  float o[D / 8][4];
  __device__ __forceinline__ void reset() {
    m_lo = m_hi = -INFINITY;
    l_lo = l_hi = 0.f;
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  }
  // Row sums completed across the quad of lanes that share a row.
  __device__ __forceinline__ float quad_sum_lo() const {
    float v = l_lo + __shfl_xor_sync(0xffffffffu, l_lo, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
  }
  __device__ __forceinline__ float quad_sum_hi() const {
    float v = l_hi + __shfl_xor_sync(0xffffffffu, l_hi, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
  }
};

// One GT-token group staged in shared memory (K boxes at `kst`, V boxes at
// `vst`): S = Q K^T on the tensor cores, the online-softmax update of `gs`,
// and O += P V.  Tokens at or past `end`, and boxes whose bit in `pmask` is
// clear (page not loaded), are masked.  `ctx` is the sequence's context
// length (ALiBi positions).  When the tile's rows belong to different
// sequences (the shared-prefix kernel), `end_lo` / `end_hi` further end the
// scores of this lane's rows r and r + 8; `end` still bounds the V data.
// `beg_lo` / `beg_hi` start them (sliding-window prefill); tokens before a
// row's start are masked like tokens past its end.
template <typename T, typename Geo, int D, bool SPLIT_P = true>
__device__ __forceinline__ void mma_group(GroupState<D>& gs, const uint32_t (&qa)[D / 16][4], uint32_t kst,
                                          uint32_t vst, int tok0, int end, uint32_t pmask, int ctx, float qk_scale,
                                          bool alibi, float slope_lo, float slope_hi, int lane,
                                          int end_lo = 2147483647, int end_hi = 2147483647, int beg_lo = 0,
                                          int beg_hi = 0) {
  using namespace mma_detail;
  constexpr int GT = Geo::GT, BOX = Geo::BOX, VBS = Geo::VBS;
  constexpr uint32_t VSW_MASK = Geo::VSWZ ? (uint32_t)(Geo::VSWZ / 16 - 1) : 0u;
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  constexpr int ST = GT / 8;
  constexpr int PK = GT / 16;
  const int q4 = lane & 3;
  const int row_end = end_lo < end_hi ? end_lo : end_hi;
  const bool tail = (tok0 + GT > end) || (tok0 + GT > row_end) || (pmask != Geo::FULL_MASK) ||
                    (tok0 < (beg_lo > beg_hi ? beg_lo : beg_hi));
  (void)KS;

  // ---- S = Q K^T : ST tiles of 8 tokens
  float sacc[ST][4];
#pragma unroll
  for (int j = 0; j < ST; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
  for (int j = 0; j < ST; ++j) {
    // lane -> matrix (lane >> 3): chunk 2*ks + (lane>>3); row (lane & 7): token 8j + (lane & 7)
    const int tok = 8 * j + (lane & 7);
    const int bx = tok / VBS, off = tok % VBS;
#pragma unroll
    for (int ks = 0; ks < KS; ks += 2) {
      const int chunk = 2 * ks + (lane >> 3);
      // kFlashTma: 64-dim halves of GT swizzled 128-byte rows
      const uint32_t addr = Geo::TROWS ? kst + (uint32_t)((chunk >> 3) * (GT * 128) + tok * 128 +
                                                         (((chunk & 7) ^ (tok & 7)) << 4))
                                       : kst + bx * BOX + (chunk * VBS + off) * 16;
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(addr, b0, b1, b2, b3);
      MmaOp<T>::run(sacc[j], qa[ks], b0, b1);
      MmaOp<T>::run(sacc[j], qa[ks + 1], b2, b3);
    }
  }

  // ---- online softmax (log2 domain).  Lane holds tokens 8j + 2*q4 + e.
  float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
  for (int j = 0; j < ST; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 8 * j + 2 * q4 + e;
      float x_lo = sacc[j][e] * qk_scale;
      float x_hi = sacc[j][2 + e] * qk_scale;
      if (alibi) {
        const float pos = (float)(tok0 + t - ctx + 1);
        x_lo += slope_lo * pos;
        x_hi += slope_hi * pos;
      }
      if (tail) {
        const bool ok = (tok0 + t < end) && ((pmask >> (t / Geo::MBS)) & 1u);
        x_lo = (ok && tok0 + t < end_lo && tok0 + t >= beg_lo) ? x_lo : -INFINITY;
        x_hi = (ok && tok0 + t < end_hi && tok0 + t >= beg_hi) ? x_hi : -INFINITY;
      }
      sacc[j][e] = x_lo;
      sacc[j][2 + e] = x_hi;
      mx_lo = fmaxf(mx_lo, x_lo);
      mx_hi = fmaxf(mx_hi, x_hi);
    }
  }
  mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
  mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
  mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
  mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
  const float mn_lo = fmaxf(gs.m_lo, mx_lo), mn_hi = fmaxf(gs.m_hi, mx_hi);
  // A row whose every token so far is masked keeps max -inf: use 0 as the
  // reference so exp2 sees -inf - 0 = -inf (never -inf - -inf = NaN).
  const float ref_lo = mn_lo == -INFINITY ? 0.f : mn_lo;
  const float ref_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
  const float a_lo = fast_exp2(gs.m_lo - ref_lo), a_hi = fast_exp2(gs.m_hi - ref_hi);
  gs.m_lo = mn_lo;
  gs.m_hi = mn_hi;
  float ps_lo = 0.f, ps_hi = 0.f;
#pragma unroll
  for (int j = 0; j < ST; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sacc[j][e] = fast_exp2(sacc[j][e] - ref_lo);
      sacc[j][2 + e] = fast_exp2(sacc[j][2 + e] - ref_hi);
      ps_lo += sacc[j][e];
      ps_hi += sacc[j][2 + e];
    }
  }
  gs.l_lo = gs.l_lo * a_lo + ps_lo;
  gs.l_hi = gs.l_hi * a_hi + ps_hi;
  // Once the row maxima settle most groups leave every factor at exactly 1:
  // the warp then skips the accumulator rescale.
  if (__any_sync(0xffffffffu, a_lo != 1.f || a_hi != 1.f)) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      gs.o[nt][0] *= a_lo;
      gs.o[nt][1] *= a_lo;
      gs.o[nt][2] *= a_hi;
      gs.o[nt][3] *= a_hi;
    }
  }

  // ---- O += P V : PK k-steps of 16 tokens x NT tiles of 8 dims
#pragma unroll
  for (int kk = 0; kk < PK; ++kk) {
    // A = P.  bf16 keeps 8 mantissa bits, so P is carried as hi + lo bf16
    // parts (two products into the same accumulators, ~16 bits of P); f16's
    // 11 bits are used as they are.  SPLIT_P = false (long shared prefixes,
    // where the rounding of many terms averages out) keeps only the hi part.
    uint32_t pa[4], pl[4];
    MmaOp<T>::pack_split(sacc[2 * kk][0], sacc[2 * kk][1], pa[0], pl[0]);
    MmaOp<T>::pack_split(sacc[2 * kk][2], sacc[2 * kk][3], pa[1], pl[1]);
    MmaOp<T>::pack_split(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1], pa[2], pl[2]);
    MmaOp<T>::pack_split(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3], pa[3], pl[3]);
    // lane -> matrix mi = lane >> 3: dims 8*(nt + mi/2) + (lane & 7), tokens 16kk + 8*(mi & 1) ..+7
    const int mi = lane >> 3;
    const int vtok = 16 * kk + 8 * (mi & 1);
    const int vbx = vtok / VBS, voff = vtok % VBS;
    // tokens this lane holds in the B fragments: 16kk + 2*q4 + e (b0/b2) and +8 (b1/b3)
    const int t_lo = tok0 + 16 * kk + 2 * q4;
    bool ok_lo0 = true, ok_lo1 = true, ok_hi0 = true, ok_hi1 = true;
    if (tail) {
      const int tl = 16 * kk + 2 * q4;
      ok_lo0 = (t_lo < end) && ((pmask >> (tl / Geo::MBS)) & 1u);
      ok_lo1 = (t_lo + 1 < end) && ((pmask >> ((tl + 1) / Geo::MBS)) & 1u);
      ok_hi0 = (t_lo + 8 < end) && ((pmask >> ((tl + 8) / Geo::MBS)) & 1u);
      ok_hi1 = (t_lo + 9 < end) && ((pmask >> ((tl + 9) / Geo::MBS)) & 1u);
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      const int dim = 8 * (nt + (mi >> 1)) + (lane & 7);
      // byte offset of (dim, voff) in the V box; with a swizzled box the
      // 16-byte chunk index (bits 4..) is XORed with address bits 7..
      uint32_t voffb = (uint32_t)(dim * VBS + voff) * 2;
      if (VSW_MASK) voffb ^= ((voffb >> 7) & VSW_MASK) << 4;
      uint32_t b0, b1, b2, b3;
      if constexpr (Geo::FLASH) {
        // token-major V rows: lane -> token 16kk + 8*(mi & 1) + (lane & 7),
        // 16-byte dim chunk nt + mi/2; transposed on load
        const uint32_t row = (uint32_t)(vtok + (lane & 7));
        ldmatrix_x4_trans(vst + row * BOX + (uint32_t)(nt + (mi >> 1)) * 16, b0, b1, b2, b3);
        (void)voffb;
      } else if constexpr (Geo::TROWS) {
        // the same rows as 64-dim halves of swizzled 128-byte rows
        const uint32_t row = (uint32_t)(vtok + (lane & 7));
        const uint32_t ch = (uint32_t)(nt + (mi >> 1));
        ldmatrix_x4_trans(vst + (ch >> 3) * (uint32_t)(GT * 128) + row * 128u + (((ch & 7u) ^ (row & 7u)) << 4), b0, b1,
                          b2, b3);
        (void)voffb;
      } else {
        ldmatrix_x4(vst + vbx * BOX + voffb, b0, b1, b2, b3);
      }
      if (tail) {
        // zero V of masked tokens: their slots may hold anything (NaN * 0 = NaN)
        const uint32_t m_lo_bits = (ok_lo0 ? 0x0000ffffu : 0u) | (ok_lo1 ? 0xffff0000u : 0u);
        const uint32_t m_hi_bits = (ok_hi0 ? 0x0000ffffu : 0u) | (ok_hi1 ? 0xffff0000u : 0u);
        b0 &= m_lo_bits;
        b2 &= m_lo_bits;
        b1 &= m_hi_bits;
        b3 &= m_hi_bits;
      }
      MmaOp<T>::run(gs.o[nt], pa, b0, b1);
      MmaOp<T>::run(gs.o[nt + 1], pa, b2, b3);
      if constexpr (MmaOp<T>::kSplitP && SPLIT_P) {
        MmaOp<T>::run(gs.o[nt], pl, b0, b1);
        MmaOp<T>::run(gs.o[nt + 1], pl, b2, b3);
      }
    }
  }
}

namespace mma_detail {

// Two codes (low byte first) -> f16x2; every E4M3 / E5M2 value is exact in f16.
template <int MODE>
__device__ __forceinline__ uint32_t fp8x2_to_f16x2(uint32_t two) {
  uint32_t d;
  const uint16_t v = (uint16_t)two;
  if constexpr (MODE == kFp8E4M3) {
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(v));
  } else {
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(d) : "h"(v));
  }
  return d;
}

// Four codes of `w` -> lo (bytes 0, 1) and hi (bytes 2, 3) as f16x2.  The
// hardware's E4M3 is the OCP E4M3FN variant (exponent 15 holds the finite
// values 256..448 and NaN); the KV cache's E4M3 keeps the all-ones exponent for
// Inf (mantissa 0) and NaN.  Such codes are written only for Inf, NaN or
// out-of-range inputs, so the group math converts every code the E4M3FN way,
// ORs e4m3_special_bits of its words into a flag, and when a warp vote finds
// one adds e4m3_specials' correction in one more product: (the FN value) + Inf
// = Inf and + NaN = NaN, the values the cache's format gives.
template <int MODE>
__device__ __forceinline__ void fp8x4_to_f16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = fp8x2_to_f16x2<MODE>(w);
  hi = fp8x2_to_f16x2<MODE>(w >> 16);
}

// Bit 7 of byte i is set iff code i of `w` has the all-ones exponent (the
// exponent field plus one carries into bit 7 only from 1111; no byte carries
// into the next).
__device__ __forceinline__ uint32_t e4m3_special_bits(uint32_t w) { return (w & 0x78787878u) + 0x08080808u; }

// f16 pairs holding, for each code of `w` with the all-ones exponent, its value
// in the cache's E4M3 (+-Inf for mantissa 0, NaN otherwise) and +0 elsewhere.
__device__ __forceinline__ void e4m3_specials(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = hi = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t c = (w >> (8 * i)) & 0xFFu;
    if ((c & 0x78u) == 0x78u) {
      const uint32_t h = ((c & 0x80u) << 8) | ((c & 0x07u) ? 0x7E00u : 0x7C00u);
      (i < 2 ? lo : hi) |= h << (16 * (i & 1));
    }
  }
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

}  // namespace mma_detail

// mma_group for one-byte caches: S = Q K^T and O += P V as f16 products.
// Permutations make plain 32-bit shared loads produce the fragments:
//  * K: column c of S tile j is token 16*(j/2) + 4*(c/2) + 2*(j%2) + c%2, and
//    the k index 2*q4 + e (+ 8) of a 16-dim step is dim 4*q4 + e (+ 2), so a
//    lane's 4 bytes (4 consecutive dims of one token) are its b0 / b1 and the
//    query fragments are loaded in the same dim order (the kernel does it);
//  * P: with that token order the S accumulators of tiles 2kk and 2kk + 1 are
//    exactly the A fragment of the 16-token step kk (tokens 4*q4 + 0..3), and
//    a lane's 4 bytes of a V row (dim, tokens 4*q4 .. 4*q4 + 3) are its b0 / b1.
// k_scale is folded into qk_scale by the caller and v_scale applied to O.
template <typename Geo, int D, int MODE>
__device__ __forceinline__ void mma_group_fp8(GroupState<D>& gs, const uint32_t (&qa)[D / 16][4], uint32_t kst,
                                              uint32_t vst, int tok0, int end, uint32_t pmask, int ctx,
                                              float qk_scale, bool alibi, float slope_lo, float slope_hi, int lane) {
  using namespace mma_detail;
  constexpr int GT = Geo::GT, BOX = Geo::BOX, VBS = Geo::VBS;
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  constexpr int ST = GT / 8;
  constexpr int PK = GT / 16;
  const int q4 = lane & 3, n = lane >> 2;
  const bool tail = (tok0 + GT > end) || (pmask != Geo::FULL_MASK);

  constexpr bool E4M3 = MODE == kFp8E4M3;
  auto k_row = [&](int j) -> uint32_t {  // this lane's K row of S tile j
    const int tok = 16 * (j >> 1) + 4 * (n >> 1) + 2 * (j & 1) + (n & 1);
    return kst + (uint32_t)((tok / VBS) * BOX + (tok % VBS) * 16 + 4 * q4);
  };

  // ---- S = Q K^T
  float sacc[ST][4];
  uint32_t special = 0u;  // E4M3: e4m3_special_bits of every word read
#pragma unroll
  for (int j = 0; j < ST; ++j) {
    sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
    const uint32_t krow = k_row(j);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t b0, b1;
      const uint32_t w = lds32(krow + (uint32_t)(ks * VBS * 16));
      if constexpr (E4M3) special |= e4m3_special_bits(w);
      fp8x4_to_f16<MODE>(w, b0, b1);
      MmaOp<__half>::run(sacc[j], qa[ks], b0, b1);
    }
  }
  if constexpr (E4M3) {
    if (__any_sync(0xffffffffu, (special & 0x80808080u) != 0u)) {  // rare: Inf / NaN codes in K
#pragma unroll
      for (int j = 0; j < ST; ++j) {
        const uint32_t krow = k_row(j);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t b0, b1;
          e4m3_specials(lds32(krow + (uint32_t)(ks * VBS * 16)), b0, b1);
          MmaOp<__half>::run(sacc[j], qa[ks], b0, b1);
        }
      }
    }
    special = 0u;
  }

  // ---- online softmax (log2 domain); element (j, e) of a lane is token
  // 16*(j/2) + 4*q4 + 2*(j%2) + e
  float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
  for (int j = 0; j < ST; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 16 * (j >> 1) + 4 * q4 + 2 * (j & 1) + e;
      float x_lo = sacc[j][e] * qk_scale;
      float x_hi = sacc[j][2 + e] * qk_scale;
      if (alibi) {
        const float pos = (float)(tok0 + t - ctx + 1);
        x_lo += slope_lo * pos;
        x_hi += slope_hi * pos;
      }
      if (tail) {
        const bool ok = (tok0 + t < end) && ((pmask >> (t / VBS)) & 1u);
        x_lo = ok ? x_lo : -INFINITY;
        x_hi = ok ? x_hi : -INFINITY;
      }
      sacc[j][e] = x_lo;
      sacc[j][2 + e] = x_hi;
      mx_lo = fmaxf(mx_lo, x_lo);
      mx_hi = fmaxf(mx_hi, x_hi);
    }
  }
  mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
  mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
  mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
  mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
  const float mn_lo = fmaxf(gs.m_lo, mx_lo), mn_hi = fmaxf(gs.m_hi, mx_hi);
  const float ref_lo = mn_lo == -INFINITY ? 0.f : mn_lo;
  const float ref_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
  const float a_lo = fast_exp2(gs.m_lo - ref_lo), a_hi = fast_exp2(gs.m_hi - ref_hi);
  gs.m_lo = mn_lo;
  gs.m_hi = mn_hi;
  float ps_lo = 0.f, ps_hi = 0.f;
#pragma unroll
  for (int j = 0; j < ST; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sacc[j][e] = fast_exp2(sacc[j][e] - ref_lo);
      sacc[j][2 + e] = fast_exp2(sacc[j][2 + e] - ref_hi);
      ps_lo += sacc[j][e];
      ps_hi += sacc[j][2 + e];
    }
  }
  gs.l_lo = gs.l_lo * a_lo + ps_lo;
  gs.l_hi = gs.l_hi * a_hi + ps_hi;
  // Once the row maxima settle most groups leave every factor at exactly 1:
  // the warp then skips the accumulator rescale.
  if (__any_sync(0xffffffffu, a_lo != 1.f || a_hi != 1.f)) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      gs.o[nt][0] *= a_lo;
      gs.o[nt][1] *= a_lo;
      gs.o[nt][2] *= a_hi;
      gs.o[nt][3] *= a_hi;
    }
  }

  // ---- O += P V
#pragma unroll
  for (int kk = 0; kk < PK; ++kk) {
    uint32_t pa[4];
    pa[0] = MmaOp<__half>::pack(sacc[2 * kk][0], sacc[2 * kk][1]);
    pa[1] = MmaOp<__half>::pack(sacc[2 * kk][2], sacc[2 * kk][3]);
    pa[2] = MmaOp<__half>::pack(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
    pa[3] = MmaOp<__half>::pack(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
    const int t4 = 16 * kk + 4 * q4;  // this lane's 4 tokens of the step
    const uint32_t vcol = vst + (uint32_t)((t4 / VBS) * BOX + t4 % VBS);
    uint32_t keep_lo = 0xFFFFFFFFu, keep_hi = 0xFFFFFFFFu;
    if (tail) {
      // zero V of masked tokens: their slots may hold anything (NaN * 0 = NaN)
      auto ok = [&](int t) { return (tok0 + t < end) && ((pmask >> (t / VBS)) & 1u); };
      keep_lo = (ok(t4) ? 0x0000FFFFu : 0u) | (ok(t4 + 1) ? 0xFFFF0000u : 0u);
      keep_hi = (ok(t4 + 2) ? 0x0000FFFFu : 0u) | (ok(t4 + 3) ? 0xFFFF0000u : 0u);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t b0, b1;
      const uint32_t w = lds32(vcol + (uint32_t)((8 * nt + n) * VBS));
      if constexpr (E4M3) special |= e4m3_special_bits(w);
      fp8x4_to_f16<MODE>(w, b0, b1);
      MmaOp<__half>::run(gs.o[nt], pa, b0 & keep_lo, b1 & keep_hi);
    }
    if constexpr (E4M3) {
      if (__any_sync(0xffffffffu, (special & 0x80808080u) != 0u)) {  // rare: Inf / NaN codes in V
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint32_t b0, b1;
          e4m3_specials(lds32(vcol + (uint32_t)((8 * nt + n) * VBS)), b0, b1);
          MmaOp<__half>::run(gs.o[nt], pa, b0 & keep_lo, b1 & keep_hi);
        }
      }
      special = 0u;
    }
  }
}

// The step's new token of sequence `seq` and KV head `kvh` (the append folded
// into the decode): its K row and V column written into the paged cache at slot
// slots[seq] (K page [D/8][BS][8], V page [D][BS]); a negative slot is a padding
// token (skipped), a slot past the cache sets SLOT_OOB and is skipped, as the
// append kernel does.  One warp; lane l takes elements l, l + 32, ...
template <typename T, int D, int BS>
__device__ __forceinline__ void append_token(const DecodeParams& p, int seq, int kvh, int lane) {
  const int64_t slot = p.slots_i64 ? reinterpret_cast<const int64_t*>(p.slots)[seq]
                                   : (int64_t)reinterpret_cast<const int32_t*>(p.slots)[seq];
  if (slot < 0) return;
  const int64_t blk = slot / BS;
  const int off = (int)(slot - blk * BS);
  if (blk >= p.num_blocks) {
    if (lane == 0) set_status(&g_decode_status, KVC_STATUS_SLOT_OOB);
    return;
  }
  const T* k = reinterpret_cast<const T*>(p.new_k) + (int64_t)seq * p.nk_tok_stride + (int64_t)kvh * p.nk_head_stride;
  const T* v = reinterpret_cast<const T*>(p.new_v) + (int64_t)seq * p.nv_tok_stride + (int64_t)kvh * p.nv_head_stride;
  T* kc = const_cast<T*>(reinterpret_cast<const T*>(p.k_cache)) + blk * p.k_block_stride + (int64_t)kvh * p.k_head_stride;
  T* vc = const_cast<T*>(reinterpret_cast<const T*>(p.v_cache)) + blk * p.v_block_stride + (int64_t)kvh * p.v_head_stride;
#pragma unroll
  for (int d = lane; d < D; d += 32) {
    kc[((d >> 3) * BS + off) * 8 + (d & 7)] = k[d];
    vc[d * BS + off] = v[d];
  }
}

template <typename T, int D, int BS, int NW, int STAGES, int GTOK, int MODE>
__global__ void __launch_bounds__(NW * 32)
    paged_decode_mma_kernel(DecodeParams p, const __grid_constant__ TmaMaps tm) {
  using namespace mma_detail;
  using Geo = MmaGeom<D, BS, NW, STAGES, GTOK, MODE>;
  constexpr int GT = Geo::GT, NBOX = Geo::NBOX, BOX = Geo::BOX, VBS = Geo::VBS;
  constexpr int KS = D / 16;    // k-steps of Q.K^T
  constexpr int NT = D / 8;     // n-tiles of P.V
  extern __shared__ __align__(128) uint8_t smem[];

  int kvh = blockIdx.x, seq = blockIdx.y, part = blockIdx.z + p.part_offset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, q4 = lane & 3;
  const int G = p.num_heads / p.num_kv_heads;

  grid_dependents_launch();
  if (p.plan_items && !planned_item(p, &kvh, &seq, &part)) return;  // planned: CTA -> work item of the plan
  const int h0 = kvh * G;
  const uint32_t ctx = p.context_lens[seq];
  int begin = 0, end = 0;
  bool zero_out = false;
  // the folded append runs in the paged 16-bit forms (the host refuses the others)
  constexpr bool APPEND = !Geo::FLASH && !Geo::FP8 && !Geo::TROWS;
  if (!partition_range(p, seq, part, ctx, &begin, &end, &zero_out)) {
    // planned: the item of a sequence with zero output (length 0 or past max_seq_len) writes it
    // (after the kernel before us, which may write the same output buffer, has finished);
    // with the folded append it also writes the sequence's new token
    if (p.wait_prior_at_start) grid_dependency_wait();
    if constexpr (APPEND) {
      if (p.new_k && p.plan_items && warp == 0) append_token<T, D, BS>(p, seq, kvh, lane);
    }
    if (zero_out || p.plan_items) write_zero_heads<T>(p, seq, h0, G, D);
    if (p.wait_prior_at_end) grid_dependency_wait();
    return;
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Geo::BAR_OFF) + warp * STAGES;
  uint32_t* masks = reinterpret_cast<uint32_t*>(smem + Geo::MASK_OFF) + warp * STAGES;
  constexpr int IDC = Geo::IDC, IDV = IDC * GT / 32;  // groups per id chunk, ids per lane per chunk
  uint32_t* ids = reinterpret_cast<uint32_t*>(smem + Geo::IDS_OFF) + warp * 2 * IDC * GT;
  // Tensor-copy modes: the ring starts on a 1024-byte boundary of the shared window, so the
  // swizzle pattern TMA applies (address bits 4.. ^= bits 7..) is the one the
  // ldmatrix addressing below undoes.
  uint8_t* ring_base = smem;
  if constexpr (Geo::ALIGN > 0) {
    constexpr uint32_t A = (uint32_t)Geo::ALIGN;
    ring_base += (A - (smem_u32(smem) & (A - 1u))) & (A - 1u);
  }
  uint8_t* ring = ring_base + (size_t)warp * STAGES * Geo::STAGE;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], Geo::CP_ASYNC ? 32 : 1);
    mbar_fence_init();
  }
  __syncwarp();

  // ---- Q as A fragments (natural dim order), rows = heads of the group.
  // One-byte caches: f16 fragments in mma_group_fp8's dim order (the k index
  // 2*q4 + e (+ 8) of a 16-dim step is dim 4*q4 + e (+ 2)).
  uint32_t qa[KS][4];
  if constexpr (Geo::FP8) {
    const T* qp = reinterpret_cast<const T*>(p.q) + (int64_t)seq * p.q_seq_stride;
    auto pair = [&](const T* row, int d) -> uint32_t {
      if constexpr (std::is_same<T, __half>::value) return *reinterpret_cast<const uint32_t*>(row + d);
      else return MmaOp<__half>::pack(to_float(row[d]), to_float(row[d + 1]));
    };
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int d0 = ks * 16 + 4 * q4;
      uint32_t v[4] = {0u, 0u, 0u, 0u};
      if (r < G) {
        const T* row = qp + (int64_t)(h0 + r) * p.q_head_stride;
        v[0] = pair(row, d0);
        v[2] = pair(row, d0 + 2);
      }
      if (r + 8 < G) {
        const T* row = qp + (int64_t)(h0 + r + 8) * p.q_head_stride;
        v[1] = pair(row, d0);
        v[3] = pair(row, d0 + 2);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[ks][i] = v[i];
    }
  } else {
    const T* qp = reinterpret_cast<const T*>(p.q) + (int64_t)seq * p.q_seq_stride;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int d0 = ks * 16 + 2 * q4;
      uint32_t v[4] = {0u, 0u, 0u, 0u};
      if (r < G) {
        const T* row = qp + (int64_t)(h0 + r) * p.q_head_stride;
        v[0] = *reinterpret_cast<const uint32_t*>(row + d0);
        v[2] = *reinterpret_cast<const uint32_t*>(row + d0 + 8);
      }
      if (r + 8 < G) {
        const T* row = qp + (int64_t)(h0 + r + 8) * p.q_head_stride;
        v[1] = *reinterpret_cast<const uint32_t*>(row + d0);
        v[3] = *reinterpret_cast<const uint32_t*>(row + d0 + 8);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[ks][i] = v[i];
    }
  }
  const float qk_scale = p.scale * kLog2e * (Geo::FP8 ? p.k_scale : 1.f);
  float slope_lo = 0.f, slope_hi = 0.f;  // ALiBi slopes of rows r and r + 8 (log2 units)
  if (p.alibi) {
    if (r < G) slope_lo = p.alibi[h0 + r] * kLog2e;
    if (r + 8 < G) slope_hi = p.alibi[h0 + r + 8] * kLog2e;
  }

  using CT = typename std::conditional<Geo::FP8, uint8_t, T>::type;  // cache element
  const CT* kbase = reinterpret_cast<const CT*>(p.k_cache) + (int64_t)kvh * p.k_head_stride;
  const CT* vbase = reinterpret_cast<const CT*>(p.v_cache) + (int64_t)kvh * p.v_head_stride;
  const uint32_t* table = p.block_tables + (int64_t)seq * p.table_stride;
  const int ngroups = (end - begin + GT - 1) / GT;
  const int n_mine = warp < ngroups ? (ngroups - warp + NW - 1) / NW : 0;
  const int rbs = Geo::TROWS ? p.block_size : BS;  // kFlashTma: the block size is read at run time
  const int page_end = (end + rbs - 1) / rbs;  // first page past the context

  // Lane i < NBOX fetches the block id of box i of group `k` of this warp.
  // Token-major caches: lane i < GT fetches the block id of token i of the
  // group (block size p.block_size, 1 for the token pool).
  // Token-major caches use the id chunks instead (load_ids / store_ids).
  auto load_block = [&](int k) -> uint32_t {
    uint32_t b = 0xffffffffu;
    if constexpr (!Geo::TOKIDS) {
      if (lane < NBOX && k < n_mine) {
        const int pg = (begin + (warp + k * NW) * GT + lane * VBS) / rbs;
        if (pg < page_end) b = __ldg(table + pg);
      }
    }
    return b;
  };
  // Token-major caches: the block ids of chunk c (groups c*IDC .. c*IDC +
  // IDC - 1 of this warp, one id per token; 0xffffffff past the context) are
  // loaded into registers one chunk before they are stored to the warp's id
  // buffer, so the table reads (one per token in the pool) overlap a whole
  // chunk of math instead of one group.
  // Token position -> (block, row in block) without a division per copy: the
  // token pool has one token per block; block sizes that are multiples of 16
  // hold a whole 16-token group (groups start 16-aligned when `begin` does).
  const int tbs = p.block_size;
  const bool tok_blocks = tbs == 1;
  const bool group_blocks = (tbs & 15) == 0 && (begin & 15) == 0;
  auto load_ids = [&](int c, uint32_t (&v)[IDV]) {
#pragma unroll
    for (int i = 0; i < IDV; ++i) {
      const int j = lane + 32 * i, kg = c * IDC + j / GT;
      const int tt = begin + (warp + kg * NW) * GT + j % GT;
      v[i] = kg < n_mine && tt < end ? __ldg(table + (tok_blocks ? tt : tt / tbs)) : 0xffffffffu;
    }
  };
  auto store_ids = [&](int c, const uint32_t (&v)[IDV]) {
#pragma unroll
    for (int i = 0; i < IDV; ++i) ids[(c & 1) * IDC * GT + lane + 32 * i] = v[i];
    __syncwarp();
  };
  // Lane 0 issues the copies of group `k` into stage `s`; `blk` holds lane
  // i's block id (from load_block).  Records which boxes were loaded.
  // Token-major caches: every lane with a token copies that token's K and V
  // rows (lane 0 first posts the byte count), the mask has a bit per token.
  auto issue = [&](int k, int s, uint32_t blk) {
    if constexpr (Geo::FLASH) {
      // kFlash: 16-byte cp.async copies spread over the warp: lane l takes
      // 16-byte column l % CPR of the RPL token rows (l / CPR) * RPL .. of both
      // K and V (rows outside the mask are zero-filled, no branch); every lane
      // then arrives on the stage's barrier when its copies have landed (the
      // barrier expects 32 arrivals in this mode).
      // kFlashBulk: lane l < GT copies token l's K and V rows as two bulk
      // copies after lane 0 has posted the stage's byte count.
      constexpr int CPR = Geo::ROWB / 16;   // 16-byte columns per row
      constexpr int RPP = 32 / CPR;         // rows per pass of the warp
      const uint32_t* cid = ids + ((k / IDC) & 1) * IDC * GT + (k % IDC) * GT;  // this group's ids
      const int t0 = begin + (warp + k * NW) * GT;
      const int tt = t0 + lane;
      const bool in_ctx = lane < GT && tt < end;
      const bool ok = in_ctx && (int64_t)cid[lane < GT ? lane : 0] < p.num_blocks;
      if (in_ctx && !ok) set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
      const uint32_t mask = __ballot_sync(0xffffffffu, ok);
      if (lane == 0) masks[s] = mask;
      uint8_t* st = ring + (size_t)s * Geo::STAGE;
      const int in0 = tok_blocks ? 0 : (group_blocks ? t0 % tbs : 0);  // row of token t0 in its block
      if constexpr (!Geo::CP_ASYNC) {
        if (lane == 0) {
          if (mask) mbar_arrive_expect_tx(&bars[s], (uint32_t)__popc(mask) * 2u * (uint32_t)Geo::ROWB);
          else mbar_arrive(&bars[s]);
        }
        __syncwarp();
        if (ok) {
          const uint32_t b = cid[lane];
          const int64_t in_blk = tok_blocks ? 0 : (group_blocks ? in0 + lane : tt % tbs);
          bulk_g2s(st + lane * BOX, kbase + (int64_t)b * p.k_block_stride + in_blk * p.k_tok_stride, Geo::ROWB,
                   &bars[s]);
          bulk_g2s(st + (NBOX + lane) * BOX, vbase + (int64_t)b * p.v_block_stride + in_blk * p.v_tok_stride,
                   Geo::ROWB, &bars[s]);
        }
        return;
      }
      if (mask) {  // (a set bit means num_blocks > 0: block 0 is mapped for the masked rows)
        constexpr int RPL = GT / RPP;  // rows per lane
        const int col = lane % CPR, r0 = (lane / CPR) * RPL;
        uint32_t rid[RPL];
#pragma unroll
        for (int i = 0; i < RPL; i += 4) {
          const uint4 v4 = *reinterpret_cast<const uint4*>(cid + r0 + i);
          rid[i] = v4.x;
          rid[i + 1] = v4.y;
          rid[i + 2] = v4.z;
          rid[i + 3] = v4.w;
        }
        const CT* kcol = kbase + col * (16 / (int)sizeof(CT));
        const CT* vcol = vbase + col * (16 / (int)sizeof(CT));
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int row = r0 + i;  // token of the group
          const bool on = (mask >> row) & 1u;
          const int64_t b = on ? rid[i] : 0;
          const int64_t in_blk = tok_blocks ? 0 : (group_blocks ? in0 + row : (t0 + row) % tbs);
          cp_async16_zfill(st + row * BOX + col * 16, kcol + b * p.k_block_stride + in_blk * p.k_tok_stride,
                           on ? 16u : 0u);
          cp_async16_zfill(st + (NBOX + row) * BOX + col * 16, vcol + b * p.v_block_stride + in_blk * p.v_tok_stride,
                           on ? 16u : 0u);
        }
      }
      cp_async_arrive(&bars[s]);
    } else if constexpr (Geo::GATHER) {
      // kFlashGather: token i's row is (block * bs + offset) * H + kvh of the
      // 2-D [rows][D] maps; lane 0 posts the bytes of the whole group (every
      // row is gathered: a token past the context or with a bad slot takes the
      // first valid token's row), then lane (kv, half, quad) < 2 * D / 64 * 4
      // gathers rows 4q .. 4q + 3 of K or V, 64 dims of them, to quad q of that
      // half (the 128-byte swizzle places them as the shared layout expects)
      const uint32_t* cid = ids + ((k / IDC) & 1) * IDC * GT + (k % IDC) * GT;
      const int t0 = begin + (warp + k * NW) * GT;
      const int tt = t0 + lane;
      const bool in_ctx = lane < GT && tt < end;
      const uint32_t b = cid[lane < GT ? lane : 0];
      const bool ok = in_ctx && (int64_t)b < p.num_blocks;
      if (in_ctx && !ok) set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
      const uint32_t mask = __ballot_sync(0xffffffffu, ok);
      int row = ok ? (int)(((tok_blocks ? (int64_t)b : (int64_t)b * tbs + tt % tbs) * p.num_kv_heads + kvh)) : 0;
      row = __shfl_sync(0xffffffffu, row, ok ? lane : (mask ? __ffs(mask) - 1 : 0));
      if (lane == 0) {
        masks[s] = mask;
        if (mask) mbar_arrive_expect_tx(&bars[s], 2u * (uint32_t)BOX);
        else mbar_arrive(&bars[s]);
      }
      __syncwarp();
      if (mask) {
        constexpr int Q = GT / 4, HALVES = D / 64;
        const int q = lane % Q, h = (lane / Q) % HALVES, kv = lane / (Q * HALVES);
        const int r0 = __shfl_sync(0xffffffffu, row, 4 * q), r1 = __shfl_sync(0xffffffffu, row, 4 * q + 1);
        const int r2 = __shfl_sync(0xffffffffu, row, 4 * q + 2), r3 = __shfl_sync(0xffffffffu, row, 4 * q + 3);
        if (lane < 2 * HALVES * Q)
          tma_gather4(ring + (size_t)s * Geo::STAGE + kv * BOX + h * (GT * 128) + q * 4 * 128, kv ? &tm.v : &tm.k,
                      64 * h, r0, r1, r2, r3, &bars[s]);
      }
    } else {
      uint32_t ids[NBOX];
#pragma unroll
      for (int i = 0; i < NBOX; ++i) ids[i] = __shfl_sync(0xffffffffu, blk, i);
      if (lane == 0) {
        const int t0 = begin + (warp + k * NW) * GT;
        uint32_t mask = 0, bytes = 0;
#pragma unroll
        for (int i = 0; i < NBOX; ++i) {
          if ((t0 + i * VBS) / rbs < page_end) {
            if ((int64_t)ids[i] < p.num_blocks) {
              mask |= 1u << i;
              bytes += 2 * BOX;
            } else {
              set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
            }
          }
        }
        masks[s] = mask;
        uint8_t* st = ring + (size_t)s * Geo::STAGE;
        if (bytes) {
          mbar_arrive_expect_tx(&bars[s], bytes);
#pragma unroll
          for (int i = 0; i < NBOX; ++i) {
            if (mask & (1u << i)) {
              if constexpr (Geo::TROWS) {
                // GT consecutive rows of block ids[i] (the group never crosses a block:
                // the block size is a multiple of 16 and groups start 16-aligned)
                const int row = (int)ids[i] * rbs + (t0 - (t0 / rbs) * rbs);
                constexpr int HALF = GT * 128;
#pragma unroll
                for (int h = 0; h < D / 64; ++h) {
                  tma_load_3d(st + i * BOX + h * HALF, &tm.k, 64 * h, kvh, row, &bars[s]);
                  tma_load_3d(st + (NBOX + i) * BOX + h * HALF, &tm.v, 64 * h, kvh, row, &bars[s]);
                }
              } else if constexpr (MODE == kTiles) {
                // token offset of the box inside its page: 0 or a multiple of 16
                // (16 tokens * 2 bytes = 32 B, so the innermost V coordinate is
                // 16-byte aligned as tiled copies require)
                const int toff = (t0 + i * VBS) % BS;
                tma_load_5d(st + i * BOX, &tm.k, 0, toff, 0, kvh, (int)ids[i], &bars[s]);
                tma_load_4d(st + (NBOX + i) * BOX, &tm.v, toff, 0, kvh, (int)ids[i], &bars[s]);
              } else if constexpr (MODE == kSwizzledV) {
                const int64_t b = (int64_t)ids[i];
                bulk_g2s(st + i * BOX, kbase + b * p.k_block_stride, BOX, &bars[s]);
                tma_load_4d(st + (NBOX + i) * BOX, &tm.v, 0, 0, kvh, (int)ids[i], &bars[s]);
              } else {
                const int64_t b = (int64_t)ids[i];
                bulk_g2s(st + i * BOX, kbase + b * p.k_block_stride, BOX, &bars[s]);
                bulk_g2s(st + (NBOX + i) * BOX, vbase + b * p.v_block_stride, BOX, &bars[s]);
              }
            }
          }
        } else {
          mbar_arrive(&bars[s]);
        }
      }
    }
  };

  // Launched as a programmatic dependent (wait_prior_at_start): what is read
  // above (the plan's header and items, lengths, block tables, queries) is
  // written by none of this library's kernels that let their dependents start
  // early (the appends write cache rows; the decode and prefill kernels write
  // outputs, partials and plan counters), so it was final before the kernel
  // before us started.  The cache, the partials and the counters are touched
  // only from here on, after that kernel has finished.
  if (p.wait_prior_at_start) grid_dependency_wait();

  // The folded append: in the CTA holding the sequence's last token
  // (partitions are whole blocks, so no other CTA reads that page), the warp
  // whose group holds it loads the token's K and V (pairs of dims, before its
  // first copies), stores it to the cache once those copies are issued without
  // waiting for the stores, and patches it into the shared copy of the page
  // once that copy has landed (the copy may have read the slot before or after
  // the store).  The patch applies when the caller's slot is the table's slot
  // of the last position, as the append kernel followed by the decode reads it.
  constexpr int AP = D / 64;  // dim pairs per lane
  uint32_t ap_k[AP], ap_v[AP];
  int append_pos = -1;
  int64_t ap_slot = -1;
  bool ap_mine = false;
  if constexpr (APPEND) {
    if (p.new_k && end == (int)ctx) {
      const int pos = (int)ctx - 1;
      ap_mine = ((pos - begin) / GT) % NW == warp;
      if (ap_mine) {
        ap_slot = p.slots_i64 ? reinterpret_cast<const int64_t*>(p.slots)[seq]
                              : (int64_t)reinterpret_cast<const int32_t*>(p.slots)[seq];
        const uint32_t* kn = reinterpret_cast<const uint32_t*>(
            reinterpret_cast<const T*>(p.new_k) + (int64_t)seq * p.nk_tok_stride + (int64_t)kvh * p.nk_head_stride);
        const uint32_t* vn = reinterpret_cast<const uint32_t*>(
            reinterpret_cast<const T*>(p.new_v) + (int64_t)seq * p.nv_tok_stride + (int64_t)kvh * p.nv_head_stride);
#pragma unroll
        for (int j = 0; j < AP; ++j) {
          ap_k[j] = __ldg(kn + 32 * j + lane);
          ap_v[j] = __ldg(vn + 32 * j + lane);
        }
        const uint32_t tb = __ldg(table + pos / BS);
        if (ap_slot >= 0 && (int64_t)tb < p.num_blocks && ap_slot == (int64_t)tb * BS + pos % BS) append_pos = pos;
      }
    }
  }

  // ---- prologue: fill the ring
  uint32_t ids_next[IDV];  // token-major caches: the chunk after the current one
  if constexpr (Geo::TOKIDS) {
    uint32_t first[IDV];
    load_ids(0, first);
    load_ids(1, ids_next);
    store_ids(0, first);
  }
#pragma unroll
  for (int s = 0; s < STAGES; ++s) {
    if (s < n_mine) issue(s, s, load_block(s));
  }
  if constexpr (APPEND) {
    // the folded append's stores (dims 64j + 2 lane, + 1 of K and V), not waited for
    if (ap_mine && ap_slot >= 0) {
      const int64_t blk = ap_slot / BS;
      const int off = (int)(ap_slot - blk * BS);
      if (blk >= p.num_blocks) {
        if (lane == 0) set_status(&g_decode_status, KVC_STATUS_SLOT_OOB);
      } else {
        T* kc = const_cast<T*>(reinterpret_cast<const T*>(p.k_cache)) + blk * p.k_block_stride +
                (int64_t)kvh * p.k_head_stride;
        T* vc = const_cast<T*>(reinterpret_cast<const T*>(p.v_cache)) + blk * p.v_block_stride +
                (int64_t)kvh * p.v_head_stride;
#pragma unroll
        for (int j = 0; j < AP; ++j) {
          const int d = 64 * j + 2 * lane;
          *reinterpret_cast<uint32_t*>(kc + ((d >> 3) * BS + off) * 8 + (d & 7)) = ap_k[j];
          reinterpret_cast<uint16_t*>(vc)[d * BS + off] = (uint16_t)(ap_v[j] & 0xFFFFu);
          reinterpret_cast<uint16_t*>(vc)[(d + 1) * BS + off] = (uint16_t)(ap_v[j] >> 16);
        }
      }
    }
  }

  GroupState<D> gs;
  gs.reset();
  int k_fail = -1;  // group whose wait gave up

  for (int k = 0; k < n_mine; ++k) {
    const int s = k % STAGES;
    if constexpr (Geo::TOKIDS) {
      // chunk c + 1 (loaded a chunk ago) replaces chunk c - 1, whose last
      // group was issued STAGES groups before this one; chunk c + 2 is loaded
      if (k % IDC == 0 && k + STAGES < n_mine) {
        store_ids(k / IDC + 1, ids_next);
        load_ids(k / IDC + 2, ids_next);
      }
    }
    const uint32_t next_blk = load_block(k + STAGES);  // latency hidden by this group's math
    if (!mbar_wait_bounded(&bars[s], (uint32_t)((k / STAGES) & 1))) {
      k_fail = k;
      break;
    }
    const uint8_t* st = ring + (size_t)s * Geo::STAGE;
    const uint32_t kst = smem_u32(st);
    const uint32_t vst = smem_u32(st + NBOX * BOX);
    const int tok0 = begin + (warp + k * NW) * GT;  // first token of the group
    const uint32_t pmask = masks[s];
    if constexpr (APPEND) {
      if (append_pos >= tok0 && append_pos < tok0 + GT) {  // this group holds the appended token
        const int t = append_pos - tok0, bx = t / VBS, off = t % VBS;
        if ((pmask >> (t / Geo::MBS)) & 1u) {
          constexpr uint32_t VSW = Geo::VSWZ ? (uint32_t)(Geo::VSWZ / 16 - 1) : 0u;
          uint8_t* kb = const_cast<uint8_t*>(st) + bx * BOX;
          uint8_t* vb = const_cast<uint8_t*>(st) + (NBOX + bx) * BOX;
#pragma unroll
          for (int j = 0; j < AP; ++j) {
            const int d = 64 * j + 2 * lane;
            *reinterpret_cast<uint32_t*>(kb + ((d >> 3) * VBS + off) * 16 + (d & 7) * 2) = ap_k[j];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              uint32_t vo = (uint32_t)((d + e) * VBS + off) * 2;  // (the V box's swizzle, as mma_group reads it)
              if (VSW) vo ^= ((vo >> 7) & VSW) << 4;
              *reinterpret_cast<uint16_t*>(vb + vo) = (uint16_t)(e ? ap_v[j] >> 16 : ap_v[j] & 0xFFFFu);
            }
          }
          __syncwarp();
        }
      }
    }
    if constexpr (Geo::FP8) {
      mma_group_fp8<Geo, D, MODE>(gs, qa, kst, vst, tok0, end, pmask, (int)ctx, qk_scale, p.alibi != nullptr,
                                  slope_lo, slope_hi, lane);
    } else {
      mma_group<T, Geo, D>(gs, qa, kst, vst, tok0, end, pmask, (int)ctx, qk_scale, p.alibi != nullptr, slope_lo,
                           slope_hi, lane);
    }

    // ---- recycle the stage
    __syncwarp();
    if (k + STAGES < n_mine) {
      fence_proxy_async();
      issue(k + STAGES, s, next_blk);
    }
  }

  if (k_fail >= 0) {
    // Groups k_fail .. k_fail + STAGES - 1 were issued and not consumed: give
    // each in-flight copy another bounded wait before the ring is reused.
    if (lane == 0) set_status(&g_decode_status, KVC_STATUS_WAIT_TIMEOUT);
    for (int kk = k_fail; kk < n_mine && kk < k_fail + STAGES; ++kk)
      mbar_wait_bounded(&bars[kk % STAGES], (uint32_t)((kk / STAGES) & 1));
  }

  if constexpr (Geo::FP8) {  // dequantisation scale of V, applied once to the accumulators
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      for (int i = 0; i < 4; ++i) gs.o[nt][i] *= p.v_scale;
  }

  // ---- merge: quad sums of l, then across warps through shared memory.
  const float l_lo = gs.quad_sum_lo(), l_hi = gs.quad_sum_hi();
  const float m_lo = gs.m_lo, m_hi = gs.m_hi;
  __syncthreads();  // every warp is done with its ring
  float* red_o = reinterpret_cast<float*>(smem);          // [NW][16][D]
  float* red_ml = red_o + NW * 16 * D;                     // [NW][16][2] (max, sum)
  {
    float* ow = red_o + (size_t)warp * 16 * D;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int d = 8 * nt + 2 * q4;
      ow[r * D + d] = gs.o[nt][0];
      ow[r * D + d + 1] = gs.o[nt][1];
      ow[(r + 8) * D + d] = gs.o[nt][2];
      ow[(r + 8) * D + d + 1] = gs.o[nt][3];
    }
    if (q4 == 0) {
      red_ml[(warp * 16 + r) * 2 + 0] = m_lo;
      red_ml[(warp * 16 + r) * 2 + 1] = l_lo;
      red_ml[(warp * 16 + r + 8) * 2 + 0] = m_hi;
      red_ml[(warp * 16 + r + 8) * 2 + 1] = l_hi;
    }
  }
  __syncthreads();
  // planned split-K with the merge fused: a sequence of one partition writes its
  // output directly, the others write partials and the last CTA merges them
  const int nparts = p.plan_items ? planned_parts(p, ctx) : p.num_partitions;
  const bool direct = p.num_partitions == 1 || (p.plan_items && p.fused_merge && nparts == 1);
  for (int i = threadIdx.x; i < G * D; i += NW * 32) {
    const int g = i / D, d = i - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, red_ml[(w * 16 + g) * 2]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float mw = red_ml[(w * 16 + g) * 2];
        const float wt = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
        L += wt * red_ml[(w * 16 + g) * 2 + 1];
        A += wt * red_o[((size_t)w * 16 + g) * D + d];
      }
    }
    // partial maxima are exchanged in natural-log units (as the generic kernel)
    emit<T>(p, seq, h0 + g, part, d, M * kLn2, L, A, d == 0, direct);
  }
  if (p.plan_items && p.fused_merge && !direct)
    planned_arrive_and_merge<T>(p, seq, kvh, h0, G, D, nparts, reinterpret_cast<float*>(smem));
  if (p.wait_prior_at_end) grid_dependency_wait();
}

// ---- dispatch -------------------------------------------------------------------
// (warps per CTA) x (ring stages per warp).  4x3 holds 192 KB of ring (one CTA
// per SM); 2x3 / 2x2 / 1x4 fit two or three CTAs per SM so one CTA's pipeline
// ramp overlaps another's streaming.  KVC_MMA_CONFIG="<warps>x<stages>"
// overrides the default for tuning runs.

static bool mma_disabled_by_env() {
  const char* v = getenv("KVC_DECODE_KERNEL");
  return v && (v[0] == 'g' || v[0] == 'G');  // "generic"
}

static bool mma_supported(const DecodeArgs& a) {
  if (a.cache_type == ElemType::U8) {  // one-byte caches have no other kernel
    const int G = a.num_heads / a.num_kv_heads;
    return (a.q_type == ElemType::F16 || a.q_type == ElemType::BF16) && (a.head_size == 64 || a.head_size == 128) &&
           (a.block_size == 8 || a.block_size == 16 || a.block_size == 32) && G >= 1 && G <= 16 && !a.flash &&
           (a.num_partitions == 1 || a.partition_size % 32 == 0) && (reinterpret_cast<uintptr_t>(a.q) & 3u) == 0 &&
           (a.q_seq_stride & 1) == 0 && (a.q_head_stride & 1) == 0;
  }
  if (mma_disabled_by_env()) return false;
  if (a.q_type != a.cache_type) return false;
  if (a.q_type != ElemType::F16 && a.q_type != ElemType::BF16) return false;
  if (!(a.head_size == 64 || a.head_size == 128)) return false;
  if (!a.flash && a.block_size != 8 && a.block_size != 16 && a.block_size != 32) return false;
  const int G = a.num_heads / a.num_kv_heads;
  if (G < 1 || G > 16) return false;
  if (a.num_partitions > 1 && a.partition_size % 32 != 0) return false;
  if (a.flash) return (reinterpret_cast<uintptr_t>(a.q) & 3u) == 0 && (a.q_seq_stride & 1) == 0 &&
                      (a.q_head_stride & 1) == 0;
  // q rows are read as 4-byte pairs
  if ((reinterpret_cast<uintptr_t>(a.q) & 3u) || (a.q_seq_stride & 1) || (a.q_head_stride & 1)) return false;
  return true;
}

// ---- tensor maps ---------------------------------------------------------------
// cuTensorMapEncodeTiled is a driver entry point; it is looked up through the
// runtime so the library needs no link against libcuda.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

struct MapKey {
  const void* k;
  const void* v;
  int64_t nb, hkv, ks[2], vs[2];
  int d, bs, vbs, swz, dt, dev, mode;
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(*this)) == 0; }
};

// Encodes (or finds in a small cache) the maps of one launch.  kTiles: K is
// [nb][H][D/8][BS][8] (box 8 x VBS x D/8: VBS tokens of every 16-byte chunk
// row) and V is [nb][H][D][BS] (box VBS x D, swizzled by `swz` bytes).
// kSwizzledV: only V, as [nb][H][D*BS/64][64] with one whole page per box and
// the 128-byte swizzle.
static bool make_tensor_maps(const DecodeParams& p, ElemType et, int D, int BS, int VBS, int swz, int mode,
                             TmaMaps* out) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  MapKey key;
  memset(&key, 0, sizeof(key));
  key.k = p.k_cache;
  key.v = p.v_cache;
  key.nb = p.num_blocks;
  key.hkv = p.num_kv_heads;
  key.ks[0] = p.k_head_stride;
  key.ks[1] = p.k_block_stride;
  key.vs[0] = p.v_head_stride;
  key.vs[1] = p.v_block_stride;
  if (mode == kFlashTma || mode == kFlashGather) {  // token rows: the row stride and the run-time block size
    key.ks[1] = p.k_tok_stride;
    key.vs[1] = p.v_tok_stride;
  }
  key.d = D;
  key.bs = (mode == kFlashTma || mode == kFlashGather) ? p.block_size : BS;
  key.vbs = VBS;
  key.swz = swz;
  key.dt = (int)et;
  key.mode = mode;
  cudaGetDevice(&key.dev);
  static std::mutex mu;
  static MapKey keys[32];
  static TmaMaps maps[32];
  static int used = 0, next = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i] == key) {
      *out = maps[i];
      return true;
    }
  const CUtensorMapDataType dt = et == ElemType::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t es = 2;
  TmaMaps m;
  memset(&m, 0, sizeof(m));
  cuuint32_t ones[5] = {1, 1, 1, 1, 1};
  if (mode == kFlashTma) {
    // [rows = num_blocks * bs][H][D] token rows (dense blocks), boxes of 64 dims x 1 head x VBS rows
    const cuuint64_t rows = (cuuint64_t)p.num_blocks * (cuuint64_t)p.block_size;
    cuuint64_t dim[3] = {(cuuint64_t)D, (cuuint64_t)p.num_kv_heads, rows};
    cuuint64_t kstr[2] = {(cuuint64_t)p.k_head_stride * es, (cuuint64_t)p.k_tok_stride * es};
    cuuint64_t vstr[2] = {(cuuint64_t)p.v_head_stride * es, (cuuint64_t)p.v_tok_stride * es};
    cuuint32_t box[3] = {64, 1, (cuuint32_t)VBS};
    if (enc(&m.k, dt, 3, const_cast<void*>(p.k_cache), dim, kstr, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS ||
        enc(&m.v, dt, 3, const_cast<void*>(p.v_cache), dim, vstr, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
      return false;
    keys[next] = key;
    maps[next] = m;
    next = (next + 1) % 32;
    if (used < 32) ++used;
    *out = m;
    return true;
  }
  if (mode == kFlashGather) {
    // [rows = num_blocks * bs * H][D]: dense token rows of every head, boxes of
    // 64 dims x 1 row (the 4-row gathers), landing with the 128-byte swizzle
    const cuuint64_t rows = (cuuint64_t)p.num_blocks * (cuuint64_t)p.block_size * (cuuint64_t)p.num_kv_heads;
    cuuint64_t dim[2] = {(cuuint64_t)D, rows};
    cuuint64_t str[1] = {(cuuint64_t)D * es};
    cuuint32_t box[2] = {64, 1};
    if (enc(&m.k, dt, 2, const_cast<void*>(p.k_cache), dim, str, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS ||
        enc(&m.v, dt, 2, const_cast<void*>(p.v_cache), dim, str, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
      return false;
    keys[next] = key;
    maps[next] = m;
    next = (next + 1) % 32;
    if (used < 32) ++used;
    *out = m;
    return true;
  }
  if (mode == kSwizzledV) {
    const cuuint64_t rows = (cuuint64_t)D * BS / 64;  // 128-byte rows per page
    cuuint64_t vdim[4] = {64, rows, (cuuint64_t)p.num_kv_heads, (cuuint64_t)p.num_blocks};
    cuuint64_t vstr[3] = {128, (cuuint64_t)p.v_head_stride * es, (cuuint64_t)p.v_block_stride * es};
    cuuint32_t vbox[4] = {64, (cuuint32_t)rows, 1, 1};
    if (rows > 256 ||
        enc(&m.v, dt, 4, const_cast<void*>(p.v_cache), vdim, vstr, vbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
      return false;
    keys[next] = key;
    maps[next] = m;
    next = (next + 1) % 32;
    if (used < 32) ++used;
    *out = m;
    return true;
  }
  cuuint64_t kdim[5] = {8, (cuuint64_t)BS, (cuuint64_t)(D / 8), (cuuint64_t)p.num_kv_heads, (cuuint64_t)p.num_blocks};
  cuuint64_t kstr[4] = {16, (cuuint64_t)BS * 16, (cuuint64_t)p.k_head_stride * es, (cuuint64_t)p.k_block_stride * es};
  cuuint32_t kbox[5] = {8, (cuuint32_t)VBS, (cuuint32_t)(D / 8), 1, 1};
  if (enc(&m.k, dt, 5, const_cast<void*>(p.k_cache), kdim, kstr, kbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return false;
  cuuint64_t vdim[4] = {(cuuint64_t)BS, (cuuint64_t)D, (cuuint64_t)p.num_kv_heads, (cuuint64_t)p.num_blocks};
  cuuint64_t vstr[3] = {(cuuint64_t)BS * es, (cuuint64_t)p.v_head_stride * es, (cuuint64_t)p.v_block_stride * es};
  cuuint32_t vbox[4] = {(cuuint32_t)VBS, (cuuint32_t)D, 1, 1};
  const CUtensorMapSwizzle sw = swz == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                          : (swz == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
  if (enc(&m.v, dt, 4, const_cast<void*>(p.v_cache), vdim, vstr, vbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  keys[next] = key;
  maps[next] = m;
  next = (next + 1) % 32;
  if (used < 32) ++used;
  *out = m;
  return true;
}

template <typename T, int D, int BS, int NW, int STAGES, int GT, int MODE = kBulk>
static cudaError_t launch_mma_nw(const DecodeParams& p, cudaStream_t stream) {
  using Geo = MmaGeom<D, BS, NW, STAGES, GT, MODE>;
  auto kern = paged_decode_mma_kernel<T, D, BS, NW, STAGES, GT, MODE>;
  TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (MODE == kTiles || MODE == kSwizzledV || MODE == kFlashTma || MODE == kFlashGather) {
    const ElemType et = std::is_same<T, __nv_bfloat16>::value ? ElemType::BF16 : ElemType::F16;
    if (!make_tensor_maps(p, et, D, BS, Geo::VBS, Geo::VSWZ, MODE, &maps)) return cudaErrorNotSupported;
  }
  static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid((unsigned)p.num_kv_heads, (unsigned)p.num_seqs, (unsigned)(p.num_partitions - p.part_offset));
  if (p.plan_items)  // planned: one CTA per (work item, KV head), items longest first
    grid = dim3((unsigned)(plan_max_items(p.num_seqs, p.max_seq_len, p.partition_size) * p.num_kv_heads));
  if (p.wait_prior_at_end) {
    // shared-prefix order: a programmatic dependent of the prefix kernel that
    // runs beside it and waits for it before exiting
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = Geo::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, maps);
    count_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  // a programmatic dependent of the kernel before it on the stream: its CTAs
  // become resident while that kernel (typically the append) finishes, and wait
  // for it before reading anything (wait_prior_at_start)
  DecodeParams pp = p;
  pp.wait_prior_at_start = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = Geo::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, pp, maps);
  count_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

// Variant id = warps * 1000 + stages * 100 + group tokens, + 100000 for tiled
// tensor copies ("<warps>x<stages>x<group>t"), + 200000 for bulk K with the
// swizzled whole-page V ("<warps>x<stages>x<group>s").
static int mma_variant() {
  const char* v = getenv("KVC_MMA_CONFIG");
  if (!v) return 0;
  int w = 0, s = 0, g = 32;
  char t = 0;
  const int n = sscanf(v, "%dx%dx%d%c", &w, &s, &g, &t);
  if (n < 2) return 0;
  return (t == 't' ? 100000 : (t == 's' ? 200000 : 0)) + w * 1000 + s * 100 + g;
}

// SMs of the current device (cached per device; any racing writer stores the same value).
static int decode_sm_count() {
  static std::atomic<int> sms[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  int n = dev >= 0 && dev < 64 ? sms[dev].load() : 0;
  if (n <= 0) {
    if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0 && dev < 64) sms[dev] = n;
  }
  return n;
}

template <typename T, int D, int BS>
static cudaError_t launch_mma_typed(const DecodeParams& p, cudaStream_t stream) {
  const int v = mma_variant();
  const int g = v % 100;
  const bool part_ok = p.num_partitions == 1 || (g > 0 && p.partition_size % g == 0);
  if (D == 128 && v && part_ok) {
    cudaError_t e = cudaErrorNotSupported;
    switch (v) {
      case 2332: e = launch_mma_nw<T, D, BS, 2, 3, 32>(p, stream); break;
      case 2232: e = launch_mma_nw<T, D, BS, 2, 2, 32>(p, stream); break;
      case 4316: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 4, 3, 16>(p, stream); break;
      case 1316: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 1, 3, 16>(p, stream); break;
      case 1416: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 1, 4, 16>(p, stream); break;
      case 2316: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 2, 3, 16>(p, stream); break;
      case 6216: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 6, 2, 16>(p, stream); break;
      case 8216: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 8, 2, 16>(p, stream); break;
      case 6316: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 6, 3, 16>(p, stream); break;
      case 8316: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 8, 3, 16>(p, stream); break;
      case 10216: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 10, 2, 16>(p, stream); break;
      case 12216: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 12, 2, 16>(p, stream); break;
      case 104316: e = launch_mma_nw<T, D, BS, 4, 3, 16, kTiles>(p, stream); break;
      case 102232: e = launch_mma_nw<T, D, BS, 2, 2, 32, kTiles>(p, stream); break;
      case 204316: if constexpr (BS <= 16) e = launch_mma_nw<T, D, BS, 4, 3, 16, kSwizzledV>(p, stream); break;
      case 202232: e = launch_mma_nw<T, D, BS, 2, 2, 32, kSwizzledV>(p, stream); break;
      case 203232: e = launch_mma_nw<T, D, BS, 3, 2, 32, kSwizzledV>(p, stream); break;
      case 202332: e = launch_mma_nw<T, D, BS, 2, 3, 32, kSwizzledV>(p, stream); break;
      default: break;
    }
    if (e != cudaErrorNotSupported) return e;
  }
  // The tail partitions of a shared-prefix decode (short, at most 256 tokens):
  // 2 warps x 3 stages, so each warp streams more of its partition before the
  // CTA's merge (config 4: 57.8 us against 62.2 us with 4 warps).
  if constexpr (BS <= 16) {
    if (p.part_offset > 0 && p.partition_size <= 256 && p.partition_size % 16 == 0)
      return launch_mma_nw<T, D, BS, 2, 3, 16>(p, stream);
  }
  // Defaults from sweeps on B200: 16-token groups, 4 warps x 3 stages (96 KB,
  // two CTAs and 8 warps per SM; 6 x 2 at D = 128, below) with whole-page 1-D bulk copies where the
  // block size allows (98% of copy bandwidth on config 2, against 81% for
  // 32-token groups).  32-token blocks: 32-token groups, 2 warps x 2 stages
  // (64 KB, three CTAs per SM), K by bulk copy and V through the 128-byte
  // swizzled tensor map (config 3: 77.7% against 73.9% with the 4-way bank
  // conflicts of unswizzled 64-byte V rows; config 5: 91% against 89%).
  // Tiled 16-token boxes of 32-token pages measured slower: such a box is
  // hundreds of 16-32 byte rows.  If no tensor map can be encoded for the
  // cache, plain bulk copies are used.
  if constexpr (BS <= 16) {
    // One rank's share of a head-sharded batch: a planned decode with at most
    // two (sequence, KV head) pairs per SM whose partitions hold whole
    // sequences runs on 10 warps x 2 stages (160 KB, one CTA per SM), so the
    // longest sequences, which end the launch, stream on more warps (256
    // sequences of U[512, 4096] tokens, one KV head: 1.71 ms per 32-layer step
    // against 1.89 with 4 warps and 2048-token partitions; 8 warps 1.74, 12
    // warps 1.71; with more pairs per SM the 4-warp CTAs are faster).
    if (D == 128 && p.plan_items && p.part_offset == 0 && p.partition_size >= 4096 && p.partition_size % 16 == 0 &&
        p.max_seq_len <= p.partition_size + 2 * BS &&
        (int64_t)p.num_seqs * p.num_kv_heads <= 2 * (int64_t)decode_sm_count())
      return launch_mma_nw<T, D, BS, 10, 2, 16>(p, stream);
    // Otherwise, at D = 128, 6 warps x 2 stages (96 KB, two CTAs and 12 warps
    // per SM).  Config 2 per 32-layer step against 4 warps x 3 stages: planned
    // at 2 / 4 / 8 KV heads per GPU 3.02 / 6.15 / 12.06 ms against 3.12 / 6.33 /
    // 12.62; single pass (v1) 12.22 against 13.11; split-K (v2) 15.29 against
    // 15.61.
    if (p.num_partitions == 1 || p.partition_size % 16 == 0) {
      if constexpr (D == 128) return launch_mma_nw<T, D, BS, 6, 2, 16>(p, stream);
      return launch_mma_nw<T, D, BS, 4, 3, 16>(p, stream);
    }
  } else {
    cudaError_t e = launch_mma_nw<T, D, BS, 2, 2, 32, kSwizzledV>(p, stream);
    if (e != cudaErrorNotSupported) return e;
  }
  return launch_mma_nw<T, D, BS, 2, 2, 32>(p, stream);
}

// One-byte caches: 16-token groups, 4 warps x 4 stages of 4 KB (three CTAs per
// SM) for blocks of up to 16 tokens; 32-token groups, 4 warps x 3 stages of
// 8 KB for 32-token blocks.
template <typename T, int D, int MODE>
static cudaError_t launch_mma_fp8(const DecodeParams& p, int block_size, cudaStream_t stream) {
  if (block_size == 8) return launch_mma_nw<T, D, 8, 4, 4, 16, MODE>(p, stream);
  if (block_size == 16) return launch_mma_nw<T, D, 16, 4, 4, 16, MODE>(p, stream);
  return launch_mma_nw<T, D, 32, 4, 3, 32, MODE>(p, stream);
}

template <typename T>
static cudaError_t launch_mma_t(const DecodeParams& p, const DecodeArgs& a, cudaStream_t stream) {
  if (a.cache_type == ElemType::U8) {
    const bool e5m2 = a.fp8_format == 1 || a.fp8_format == 3;  // the -sat formats decode alike
    if (a.head_size == 128)
      return e5m2 ? launch_mma_fp8<T, 128, kFp8E5M2>(p, a.block_size, stream)
                  : launch_mma_fp8<T, 128, kFp8E4M3>(p, a.block_size, stream);
    return e5m2 ? launch_mma_fp8<T, 64, kFp8E5M2>(p, a.block_size, stream)
                : launch_mma_fp8<T, 64, kFp8E4M3>(p, a.block_size, stream);
  }
  if (a.flash) {
    // token-major caches: 16-token groups, 6 warps x 2 stages for D = 128 and
    // 4 warps x 3 stages for D = 64 (two CTAs per SM); the block size is read
    // at run time.
    // KVC_FLASH_COPY=bulk selects per-row bulk copies (tuning runs).
    // KVC_FLASH_COPY=cpasync keeps the per-lane row copies where tensor copies apply (tuning runs).
    // KVC_FLASH_COPY=gather reads dense rows in any order by tensor gathers (below).
    const char* fc = getenv("KVC_FLASH_COPY");
    if (fc && fc[0] == 'b') {
      if (a.head_size == 128) return launch_mma_nw<T, 128, 16, 4, 3, 16, kFlashBulk>(p, stream);
      return launch_mma_nw<T, 64, 16, 4, 3, 16, kFlashBulk>(p, stream);
    }
    // blocks of 16k consecutive token rows: a tensor copy per (16-token group, head, 64 dims)
    const bool rows_ok = a.block_size % 16 == 0 && a.k_block_stride == (int64_t)a.block_size * a.k_tok_stride &&
                         a.v_block_stride == (int64_t)a.block_size * a.v_tok_stride &&
                         a.num_blocks * (int64_t)a.block_size < (int64_t)1 << 31 && !(fc && fc[0] == 'c');
    // D = 128: 6 warps x 2 stages (two CTAs and 12 warps per SM; config 2 on
    // the pool: page tables 12.67 against 13.54 ms per step with 4 x 3, slot
    // lists 15.67 against 16.66)
    const bool six = a.head_size == 128;
    if (rows_ok) {
      cudaError_t e = six ? launch_mma_nw<T, 128, 16, 6, 2, 16, kFlashTma>(p, stream)
                    : a.head_size == 128 ? launch_mma_nw<T, 128, 16, 4, 3, 16, kFlashTma>(p, stream)
                                         : launch_mma_nw<T, 64, 16, 4, 3, 16, kFlashTma>(p, stream);
      if (e != cudaErrorNotSupported) return e;
    }
    // KVC_FLASH_COPY=gather: dense token rows in any order (the pool's slot
    // lists) by 4-row tensor gathers.  Not the default: on config 2's slot-list
    // pool they measured 0.661 of the copy peak against 0.708 for the per-lane
    // row copies (16 gather requests per 16-token group and head, against 4
    // tensor copies for blocks of consecutive rows).
    // (block size 1, the pool's [slots, H, D]: a block is one row and carries no token stride)
    const int64_t D = a.head_size, H = a.num_kv_heads, rbs = a.block_size;
    const int64_t ktok = rbs == 1 ? H * D : a.k_tok_stride, vtok = rbs == 1 ? H * D : a.v_tok_stride;
    const bool dense = a.k_head_stride == D && ktok == H * D && a.k_block_stride == rbs * H * D &&
                       a.v_head_stride == D && vtok == H * D && a.v_block_stride == rbs * H * D &&
                       a.num_blocks * rbs * H < (int64_t)1 << 31 && fc && fc[0] == 'g';
    if (dense) {
      cudaError_t e = a.head_size == 128 ? launch_mma_nw<T, 128, 16, 4, 3, 16, kFlashGather>(p, stream)
                                         : launch_mma_nw<T, 64, 16, 4, 3, 16, kFlashGather>(p, stream);
      if (e != cudaErrorNotSupported) return e;
    }
    if (six) return launch_mma_nw<T, 128, 16, 6, 2, 16, kFlash>(p, stream);
    if (a.head_size == 128) return launch_mma_nw<T, 128, 16, 4, 3, 16, kFlash>(p, stream);
    return launch_mma_nw<T, 64, 16, 4, 3, 16, kFlash>(p, stream);
  }
  if (a.head_size == 128) {
    if (a.block_size == 8) return launch_mma_typed<T, 128, 8>(p, stream);
    if (a.block_size == 16) return launch_mma_typed<T, 128, 16>(p, stream);
    return launch_mma_typed<T, 128, 32>(p, stream);
  }
  if (a.block_size == 8) return launch_mma_typed<T, 64, 8>(p, stream);
  if (a.block_size == 16) return launch_mma_typed<T, 64, 16>(p, stream);
  return launch_mma_typed<T, 64, 32>(p, stream);
}

static cudaError_t launch_mma(const DecodeParams& p, const DecodeArgs& a, cudaStream_t stream) {
  if (a.q_type == ElemType::BF16) return launch_mma_t<__nv_bfloat16>(p, a, stream);
  return launch_mma_t<__half>(p, a, stream);
}

}  // namespace kvc
