// prefill_umma.cuh — tcgen05 (5th-generation tensor core) prefill / extend
// attention for sm_100a over the paged (vLLM) cache layout.
//
// Included by decode.cu after prefill.cuh: same PrefillArgs, same results as
// prefill_kernel (the offset-causal / window rule of PooledKVCache.make_mask,
// memory_pool.py:240-270), with the products on the tensor cores' own
// pipeline instead of mma.sync:
//
//  * Work item = 128 query rows (new token, query head of the group) of one
//    sequence and KV head (cascade form: 128 (sequence, head) rows and one
//    prefix chunk); row r of the item is TMEM lane r.  The grid is
//    persistent (one CTA per SM): CTA c takes item c, then claims further
//    items from a device counter until none is left.
//  * TMEM (512 columns): two S buffers of 128 fp32 columns (S = Q K^T of a
//    128-token tile), O (D fp32 columns) and two Q buffers (D/2 columns of
//    bf16/f16 pairs each: the next item's Q is staged while the current item
//    finishes).  P overwrites its own S buffer: hi parts in the first 64
//    columns, lo parts (bf16 only) in the next 64.
//  * Warp 8 (producer) claims the items, hands each to the other warps, and
//    streams its 128-token tiles into a ring of KST stages: K either as 4-row
//    gathers of the dense cache (one [D/8][128][8] no-swizzle K-major operand
//    per tile) or page by page as it is (its [D/8][bs][8] layout is that
//    operand layout for N = bs), each V page [D][bs] through a tensor map
//    that writes it with the bs*2-byte swizzle, the K-major operand layout of
//    P.V (tokens are its K).
//  * Warp 9 (one lane) issues S_j = Q K_j^T (A = Q from TMEM; N = 128 per
//    16-dim k-step for gathered K, else a chain per page with N = bs), then
//    O += P_{j-1} V_{j-1} (A = P from TMEM, N = D, 16 tokens per
//    instruction; bf16 P as hi + lo, two products), committing each to an
//    mbarrier.
//  * Warps 0-7 (warps w and w + 4 share TMEM lanes 32w .. 32w + 31, one
//    thread per row and half tile) read S_j, mask it (causal end, window
//    start, context end), keep the running max lazily (O is rescaled only
//    when a row's max rises by more than 2^8; until then P may exceed 1,
//    exactly as the final O / l needs), write P, and at the end normalise
//    O and store the row (cascade form: the split-K partials).
// Every wait is bounded (KVC_STATUS_WAIT_TIMEOUT and an abort flag end every
// loop); TMEM is freed only after a final commit shows every product done.
#pragma once

namespace kvc {
namespace umma {

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version of sm_100
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}
constexpr uint32_t kLayoutNone = 0, kLayoutSw64 = 4, kLayoutSw32 = 6;

// kind::f16 instruction descriptor: fp32 accumulate, A and B both `bf16`
// (else both f16), K-major A and B, M x N.
__host__ __device__ constexpr uint32_t instr_desc(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem descriptor]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mma_detail::smem_u32(bar))
               : "memory");
}
// Waits for the phase with `parity`, the thread suspended in the barrier
// (up to 200 us per try, woken when the phase completes) instead of spinning;
// gives up after ~1 s of wall time (returns false).  A phase already complete
// returns at the first test, without reading the clock.
__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
  if (mma_detail::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = mma_detail::global_timer_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(mma_detail::smem_u32(bar)), "r"(parity), "r"(200000u)
        : "memory");
    if (done) return true;
    if (mma_detail::global_timer_ns() - t0 > 1000000000ull) return false;
  }
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: this thread's lane, columns c .. c+31
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
  st16(taddr, r);
  st16(taddr + 16, r + 16);
}

// (the 4-row gather of the same chunk of four pages: mma_detail::tma_gather4)
using mma_detail::tma_gather4;

}  // namespace umma

constexpr int kUmmaRows = 128;   // query rows per CTA (TMEM lanes)
constexpr int kUmmaTile = 128;   // tokens per S tile
constexpr int kUmmaThreads = 320;  // 8 softmax warps, a producer warp, an MMA warp
constexpr int kProducerWarp = 8, kMmaWarp = 9;

template <int D, int BS>
struct UmmaGeom {
  static constexpr int PAGES = kUmmaTile / BS;
  static constexpr int PAGE = D * BS * 2;            // bytes of one K (or V) page of one head
  static constexpr int STAGE = 2 * PAGES * PAGE;     // K pages, then V pages
  static constexpr int KST = D == 128 ? 3 : 4;       // ring stages
  static constexpr int RING = KST * STAGE;
  static constexpr int BAR_OFF = 1024 + RING;        // (1024: alignment slack of the ring)
  static constexpr int NBARS = 2 * KST + 2 + 2 + 1 + 1 + 1 + 1;  // kv full/empty, s_full, p_full, pv_done, q_ready, done, xchg
  static constexpr int MASK_OFF = BAR_OFF + NBARS * 8;
  static constexpr int XBUF_OFF = (MASK_OFF + KST * 4 + 15) / 16 * 16;
  static constexpr int SMEM = XBUF_OFF + 2 * 2 * 128 * 4;
  // TMEM columns: S/P of two tiles, O, and Q of two items (the next item's Q is
  // staged while the current one finishes)
  static constexpr uint32_t SCOL = 0, OCOL = 256, QCOL = 256 + D;
  static_assert(QCOL + D <= 512, "TMEM columns");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Work item (the persistent grid walks them): a 128-row tile of one sequence
// (prefill) or of all sequences (cascade), one key range, one KV head.
// CTA c starts with item c; after that each CTA claims the next unclaimed item
// from a device counter, so a CTA that drew short items takes more of them.
// A launch uses one of kUmmaSchedSlots counter pairs and the last CTA of the
// launch to finish returns its pair to zero.  The host hands the pairs out in
// turn: launches recorded into a CUDA graph (replayed for as long as the graph
// lives) from the last kUmmaSchedCaptured pairs, the others from the rest, so
// two launches running at the same time share a pair only if one stream
// trails another by thousands of launches of this kernel.
struct UmmaSched {
  unsigned next, done;
};
constexpr int kUmmaSchedSlots = 4096, kUmmaSchedCaptured = 1024;
__device__ UmmaSched g_umma_sched[kUmmaSchedSlots];

struct UmmaItem {
  int64_t q0, rows, R0;
  int y, kvh, prefix, kv_beg, kv_end, ntiles;
  bool bad, skip, first_tile;
};

template <bool CASCADE>
__device__ __forceinline__ UmmaItem umma_item(const PrefillArgs& p, int idx, int tiles_x, int ny) {
  constexpr int KT = kUmmaTile;
  UmmaItem it;
  const int xi = idx % tiles_x;
  it.y = (idx / tiles_x) % ny;
  it.kvh = idx / (tiles_x * ny);
  it.R0 = (int64_t)(tiles_x - 1 - xi) * kUmmaRows;  // within a sequence, the last (longest) tiles first
  it.first_tile = xi == tiles_x - 1;
  it.q0 = 0;
  it.rows = 0;
  it.prefix = 0;
  it.kv_beg = 0;
  it.kv_end = 0;
  it.bad = false;
  it.skip = true;
  const int G = p.num_heads / p.num_kv_heads;
  if constexpr (CASCADE) {
    it.rows = (int64_t)p.num_seqs * G;
    if (it.R0 >= it.rows) return it;
    it.kv_beg = it.y * p.prefix_part_size;
    it.kv_end = it.kv_beg + p.prefix_part_size < p.prefix_len ? it.kv_beg + p.prefix_part_size : p.prefix_len;
  } else {
    it.q0 = p.qo_indptr[it.y];
    const int64_t q1 = p.qo_indptr[it.y + 1];
    const int64_t kvl = p.kv_lens[it.y];
    const int64_t ql = q1 - it.q0;
    it.rows = ql * G;
    if (ql <= 0 || it.R0 >= it.rows || q1 > p.num_tokens) {
      // (q1 past num_tokens: no row of it may be written; flagged below)
      it.bad = q1 > p.num_tokens && ql > 0;
      return it;
    }
    it.bad = ql > p.max_q_len || kvl < ql || kvl > p.table_len * (int64_t)p.block_size || kvl > 0x7fffffffll - 256;
    it.prefix = it.bad ? 0 : (int)(kvl - ql);
    const int64_t R_last = (it.R0 + kUmmaRows < it.rows ? it.R0 + kUmmaRows : it.rows) - 1;
    const int t_first = (int)(it.R0 / G), t_last = (int)(R_last / G);
    it.kv_end = it.bad ? 0 : it.prefix + t_last + 1;
    int kb = p.window > 0 ? it.prefix + t_first + 1 - p.window : 0;
    it.kv_beg = kb > 0 ? kb / KT * KT : 0;
  }
  it.ntiles = it.kv_end > it.kv_beg ? (it.kv_end - it.kv_beg + KT - 1) / KT : 0;
  it.skip = false;
  return it;
}

// GK: K reaches shared memory as [D/8 chunks][128 tokens][8] through 4-row
// gathers (a dense K cache; one gather per chunk and four pages), so S is one
// N = 128 product per k-step; else each K page is one bulk copy and S one
// N = BS chain per page.
// CASCADE: the shared-prefix decode form (rows = (sequence, head) pairs, keys =
// prefix chunk `y`, split-K partials out); else prefill / extend.  The grid is
// persistent: CTA c takes work item c, then claims further ones (of the
// tiles_x x ny x num_kv_heads items) until none is left, keeping TMEM, its
// barriers and its ring across them (every barrier phase below counts this
// CTA's tiles or items).
template <typename T, int D, int BS, bool GK, bool CASCADE = false>
__global__ void __launch_bounds__(kUmmaThreads, 1)
    prefill_umma_kernel(const PrefillArgs p, const __grid_constant__ TmaMaps maps, int tiles_x, int ny, int slot) {
  using namespace mma_detail;
  using UG = UmmaGeom<D, BS>;
  constexpr int PAGES = UG::PAGES, PAGE = UG::PAGE, KST = UG::KST, KT = kUmmaTile;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr bool SPLIT = BF16;  // bf16 P as hi + lo; f16 P as it is
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ int s_abort;
  __shared__ uint32_t s_tmem;
  // the items the producer hands the MMA and softmax warps, two deep
  __shared__ int s_item[2];
  __shared__ __align__(8) uint64_t item_bars[4];
  uint64_t* item_full = item_bars;       // the producer published slot i
  uint64_t* item_empty = item_bars + 2;  // the MMA lane and the 8 softmax warps read slot i
  uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + UG::BAR_OFF);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + KST;
  uint64_t* s_full = bars + 2 * KST;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_ready = pv_done + 1;
  uint64_t* all_done = q_ready + 1;
  uint64_t* xchg = all_done + 1;
  float* xbuf = reinterpret_cast<float*>(smem_raw + UG::XBUF_OFF);  // [2 phases][2 halves][128 rows]
  uint32_t* page_mask = reinterpret_cast<uint32_t*>(smem_raw + UG::MASK_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.num_heads / p.num_kv_heads;
  const int n_items = tiles_x * ny * p.num_kv_heads;
  const CUtensorMap* vmap = &maps.v;
  const CUtensorMap* kmap = &maps.k;
  static_assert(!GK || PAGES % 4 == 0, "the gathered K layout takes pages in fours");
  // The shared-prefix form is itself a programmatic dependent of the kernel
  // before it (the step's append, which lets its dependents start at once):
  // its set-up, query staging and block-id reads (nothing an append writes)
  // overlap that kernel, and its producer waits for it before the first cache
  // copy, then lets the tail partitions (a programmatic dependent that waits
  // for this grid before exiting) start beside it.
  if constexpr (!CASCADE) grid_dependents_launch();
  // (fewer items than CTAs: each CTA has its one item and nothing is claimed)
  const bool dynamic = n_items > (int)gridDim.x;
  // The producer decodes its first item and starts that item's first block-id
  // loads and the tensor-map descriptor fetches before the set-up below, so
  // their latency overlaps it.
  UmmaItem it0;
  uint32_t first_id = 0xffffffffu;
  if (warp == kProducerWarp) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.v)) : "memory");
      if (GK) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.k)) : "memory");
    }
    it0 = umma_item<CASCADE>(p, blockIdx.x, tiles_x, ny);
    const uint32_t* t0row = p.block_tables + (CASCADE ? (int64_t)0 : (int64_t)it0.y * p.table_stride);
    if (!it0.skip && lane < PAGES && it0.ntiles > 0 && it0.kv_beg + lane * BS < it0.kv_end)
      first_id = __ldg(t0row + (it0.kv_beg + lane * BS) / BS);
  }

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < KST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);
    }
    mbar_init(pv_done, 1);
    mbar_init(q_ready, 8);
    mbar_init(xchg, 8);
    mbar_init(all_done, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 9);
    }
    mbar_fence_init();
  }
  // Stale V of pages a tile does not load meets P = 0 (0 * NaN = NaN): the V
  // halves of the ring start from zeros.  (K of unloaded pages is only ever
  // masked, or replaced by a loaded page's rows in the gathered form.)
  constexpr int V16 = PAGES * PAGE / 16;  // 16-byte words of one stage's V pages
  for (int i = threadIdx.x; i < KST * V16; i += kUmmaThreads)
    reinterpret_cast<uint4*>(ring + (size_t)(i / V16) * UG::STAGE + PAGES * PAGE)[i % V16] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tmem = s_tmem;
  auto abort_now = [&]() -> bool { return *(volatile int*)&s_abort != 0; };
  auto give_up = [&]() {
    s_abort = 1;
    set_status(&g_decode_status, KVC_STATUS_WAIT_TIMEOUT);
  };

  if (warp == kProducerWarp) {
    if constexpr (CASCADE) {
      grid_dependency_wait();
      if (lane == 0) grid_dependents_launch();
    }
    // ---- producer: claims items, hands each one with rows to the other warps,
    // then loads its 128-token tiles of whole pages
    int gt = 0;    // tiles issued by this CTA so far
    int npub = 0;  // items handed over so far
    bool stop = false;
    // (lane 0) item idx into ring slot npub & 1, once both readers of the item
    // two back have taken it
    auto publish = [&](int idx) -> bool {
      const int sl = npub & 1;
      if (npub >= 2 && !umma::wait(&item_empty[sl], (uint32_t)(((npub >> 1) - 1) & 1))) return false;
      *(volatile int*)&s_item[sl] = idx;
      mbar_arrive(&item_full[sl]);  // (release: the index is seen by whoever waits on the slot)
      ++npub;
      return true;
    };
    UmmaSched* sched = &g_umma_sched[slot];
    for (int idx = blockIdx.x; idx < n_items && !stop;) {
      const bool first = idx == (int)blockIdx.x;  // (claimed items are all past the grid)
      const UmmaItem it = first ? it0 : umma_item<CASCADE>(p, idx, tiles_x, ny);
      if (!CASCADE && it.bad && it.first_tile && it.kvh == 0 && lane == 0)
        set_status(&g_decode_status, KVC_STATUS_INDEX_OOB);
      // the next item is claimed once this one's loads are issued
      auto claim = [&]() -> int {
        unsigned nx = (unsigned)n_items;
        if (dynamic && lane == 0) nx = gridDim.x + atomicAdd(&sched->next, 1u);
        nx = __shfl_sync(0xffffffffu, nx, 0);
        return nx < (unsigned)n_items ? (int)nx : n_items;
      };
      if (it.skip) {
        idx = claim();
        continue;
      }
      // the item's query rows toward L2: the softmax warps load them only after
      // finishing the item before this one
      if (!it.bad && it.ntiles > 0) {
        const int64_t nrows = it.rows - it.R0 < kUmmaRows ? it.rows - it.R0 : kUmmaRows;
        for (int r = lane; r < nrows; r += 32) {
          const int64_t R = it.R0 + r, t = R / G;
          const char* a = reinterpret_cast<const char*>(reinterpret_cast<const T*>(p.q) + (it.q0 + t) * p.q_tok_stride +
                                                        (int64_t)(it.kvh * G + (int)(R - t * G)) * p.q_head_stride);
#pragma unroll
          for (int b = 0; b < D * 2; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(a + b));
        }
      }
      bool handed = true;
      if (lane == 0) handed = publish(idx);
      if (!__shfl_sync(0xffffffffu, handed, 0)) {
        if (lane == 0) give_up();
        break;
      }
      if (__shfl_sync(0xffffffffu, abort_now() ? 1 : 0, 0)) break;
      const int kvh = it.kvh, kv_beg = it.kv_beg, kv_end = it.kv_end, ntiles = it.ntiles;
      const T* kbase = reinterpret_cast<const T*>(p.k_cache) + (int64_t)kvh * p.k_head_stride;
      const uint32_t* table = p.block_tables + (CASCADE ? (int64_t)0 : (int64_t)it.y * p.table_stride);
      auto load_id = [&](int j) -> uint32_t {
        uint32_t id = 0xffffffffu;
        const int tok = kv_beg + j * KT + lane * BS;
        if (lane < PAGES && j < ntiles && tok < kv_end) id = __ldg(table + tok / BS);
        return id;
      };
      uint32_t id = first ? first_id : load_id(0);
      for (int j = 0; j < ntiles; ++j) {
        const int g = gt + j, st = g % KST;
        bool ok = true;
        if (g >= KST && lane == 0) ok = umma::wait(&kv_empty[st], (uint32_t)(((g / KST) - 1) & 1));
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) give_up();
          stop = true;
          break;
        }
        if (__shfl_sync(0xffffffffu, abort_now() ? 1 : 0, 0)) {
          stop = true;
          break;
        }
        const int t0 = kv_beg + j * KT;
        const bool in_range = lane < PAGES && t0 + lane * BS < kv_end;
        const bool valid = in_range && (int64_t)id < p.num_blocks;
        if (in_range && !valid) set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
        const uint32_t mask = __ballot_sync(0xffffffffu, valid);
        uint32_t ids[PAGES];
#pragma unroll
        for (int i = 0; i < PAGES; ++i) ids[i] = __shfl_sync(0xffffffffu, id, i);
        id = load_id(j + 1);  // next tile's ids, in flight while this one is issued
        if (!p.single_issue) {
          // the tile's copies spread over the warp: lane 0 posts the byte count
          // first; then with GK lane c < D/8 issues the 4-row gathers of K chunk
          // c and lane 16 + i the V copy of page i, without GK lane i the K and V
          // copies of page i
          uint8_t* kst = ring + (size_t)st * UG::STAGE;
          uint8_t* vst = kst + PAGES * PAGE;
          if (lane == 0) {
            page_mask[st] = mask;
            if (mask)
              mbar_arrive_expect_tx(&kv_full[st], (uint32_t)((GK ? PAGES : 0) + (GK ? 1 : 2) * __popc(mask)) *
                                                      (uint32_t)PAGE);
            else
              mbar_arrive(&kv_full[st]);
          }
          __syncwarp();
          if (mask) {
            if constexpr (GK) {
              static_assert(D / 8 <= 16 && PAGES <= 16, "lanes of the spread issue");
              const uint32_t any = ids[__ffs(mask) - 1];  // pages without keys gather a loaded page's rows
              if (lane < D / 8) {
                int rb[PAGES];
#pragma unroll
                for (int i = 0; i < PAGES; ++i)
                  rb[i] = (int)(((int64_t)((mask >> i) & 1u ? ids[i] : any) * p.num_kv_heads + kvh) * (D / 8));
                const int c = lane;
#pragma unroll
                for (int q = 0; q < PAGES; q += 4)
                  umma::tma_gather4(kst + c * KT * 16 + q * BS * 16, kmap, 0, rb[q] + c, rb[q + 1] + c, rb[q + 2] + c,
                                    rb[q + 3] + c, &kv_full[st]);
              } else if (lane >= 16 && lane - 16 < PAGES && ((mask >> (lane - 16)) & 1u)) {
                const int i = lane - 16;
                tma_load_4d(vst + i * PAGE, vmap, 0, 0, kvh, (int)ids[i], &kv_full[st]);
              }
            } else {
              if (lane < PAGES && ((mask >> lane) & 1u)) {
                const int i = lane;
                bulk_g2s(kst + i * PAGE, kbase + (int64_t)ids[i] * p.k_block_stride, PAGE, &kv_full[st]);
                tma_load_4d(vst + i * PAGE, vmap, 0, 0, kvh, (int)ids[i], &kv_full[st]);
              }
            }
          }
        } else if (lane == 0) {
          page_mask[st] = mask;
          uint8_t* kst = ring + (size_t)st * UG::STAGE;
          uint8_t* vst = kst + PAGES * PAGE;
          // few and large requests (the copy engine serves them one by one):
          // per page one tensor copy of V and one bulk copy of K, or with GK one
          // 4-row gather per 8-dim chunk for the K of four pages
          if (mask) {
            if constexpr (GK) {
              mbar_arrive_expect_tx(&kv_full[st], (uint32_t)(PAGES + __popc(mask)) * (uint32_t)PAGE);
              const uint32_t any = ids[__ffs(mask) - 1];  // pages without keys gather a loaded page's rows
              int rb[PAGES];
#pragma unroll
              for (int i = 0; i < PAGES; ++i)
                rb[i] = (int)(((int64_t)((mask >> i) & 1u ? ids[i] : any) * p.num_kv_heads + kvh) * (D / 8));
#pragma unroll
              for (int c = 0; c < D / 8; ++c)
#pragma unroll
                for (int q = 0; q < PAGES; q += 4)  // pages q .. q + 3: tokens q*BS .. of the chunk row
                  umma::tma_gather4(kst + c * KT * 16 + q * BS * 16, kmap, 0, rb[q] + c, rb[q + 1] + c, rb[q + 2] + c,
                                    rb[q + 3] + c, &kv_full[st]);
            } else {
              mbar_arrive_expect_tx(&kv_full[st], (uint32_t)__popc(mask) * 2u * (uint32_t)PAGE);
            }
#pragma unroll
            for (int i = 0; i < PAGES; ++i) {
              if (mask & (1u << i)) {
                if constexpr (!GK)
                  bulk_g2s(kst + i * PAGE, kbase + (int64_t)ids[i] * p.k_block_stride, PAGE, &kv_full[st]);
                tma_load_4d(vst + i * PAGE, vmap, 0, 0, kvh, (int)ids[i], &kv_full[st]);
              }
            }
          } else {
            mbar_arrive(&kv_full[st]);
          }
        }
      }
      if (CASCADE && kvh == 0) {
        // every sequence of this tile must carry sequence 0's block ids over the
        // chunk (the caller's promise; checked once per tile and chunk, after
        // the item's copies are issued: it only sets a status bit)
        const int64_t R_last = (it.R0 + kUmmaRows < it.rows ? it.R0 + kUmmaRows : it.rows) - 1;
        const int s0 = (int)(it.R0 / G), nseq = (int)(R_last / G) - s0 + 1;
        const int b0 = kv_beg / BS, nb = (kv_end + BS - 1) / BS - b0;
        bool diff = false;
        for (int i = lane; i < nseq * nb; i += 32) {
          const int sq = s0 + i / nb, bb = b0 + i % nb;
          diff |= __ldg(p.block_tables + (int64_t)sq * p.table_stride + bb) != __ldg(p.block_tables + bb);
        }
        if (diff) set_status(&g_decode_status, KVC_STATUS_PREFIX_MISMATCH);
      }
      gt += ntiles;
      if (!stop) idx = claim();
    }
    // the end marker (n_items) for the other warps
    if (lane == 0 && !publish(n_items)) give_up();
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---- MMA issue (one lane), item after item
    if (lane == 0) {
      const uint32_t idS = umma::instr_desc(BF16, 128, GK ? KT : BS), idO = umma::instr_desc(BF16, 128, D);
      // Descriptors of stage 0, advanced by adding (byte offset >> 4) to the
      // start-address field (shared addresses stay below 256 KB: no carry).
      const uint32_t ring_addr = smem_u32(ring);
      const uint64_t k_desc0 = umma::smem_desc(ring_addr, (GK ? KT : BS) * 16, 128, umma::kLayoutNone);
      const uint64_t v_desc0 = BS == 32 ? umma::smem_desc(ring_addr + PAGES * PAGE, 16, 512, umma::kLayoutSw64)
                                        : umma::smem_desc(ring_addr + PAGES * PAGE, 16, 256, umma::kLayoutSw32);
      int gt = 0, nit = 0, nread = 0;  // tiles, items with keys, ring slots read of this CTA so far
      bool ok = true;
      for (;;) {
        const int sl = nread & 1;
        if (abort_now() || !umma::wait(&item_full[sl], (uint32_t)((nread >> 1) & 1))) {
          ok = false;
          break;
        }
        const int idx = *(volatile int*)&s_item[sl];
        mbar_arrive(&item_empty[sl]);
        ++nread;
        if (idx >= n_items) break;
        const UmmaItem it = umma_item<CASCADE>(p, idx, tiles_x, ny);
        if (it.skip || it.ntiles == 0) continue;  // (no Q is handed over for an item without keys)
        if (abort_now() || !umma::wait(q_ready, (uint32_t)(nit & 1))) {
          ok = false;
          break;
        }
        umma::fence_after();
        const uint32_t qcol = tmem + UG::QCOL + (uint32_t)(nit & 1) * (D / 2);  // this item's Q buffer
        ++nit;
        const int kv_beg = it.kv_beg, kv_end = it.kv_end, ntiles = it.ntiles;
        bool o_init = false;
        // O += P_j V_j of tile j (this CTA's tile g)
        auto issue_pv = [&](int j, int g) -> bool {
          const int b = g & 1, st = g % KST;
          if (!umma::wait(&p_full[b], (uint32_t)((g >> 1) & 1))) return false;
          umma::fence_after();
          const uint64_t vd = v_desc0 + (uint64_t)((st * UG::STAGE) >> 4);
          const int steps = (kv_end - (kv_beg + j * KT) + 15) / 16;  // 16-token k-steps with keys
          const uint32_t pcol = tmem + UG::SCOL + b * 128;
#pragma unroll
          for (int ks = 0; ks < KT / 16; ++ks) {
            if (ks < steps) {
              // k-step ks: tokens 16ks.. = page (16ks)/BS, byte (16ks % BS) * 2 of its rows
              const uint64_t d = vd + (uint64_t)((((16 * ks) / BS) * PAGE + ((16 * ks) % BS) * 2) >> 4);
              umma::mma_ts(tmem + UG::OCOL, pcol + 8 * ks, d, idO, (o_init || ks > 0) ? 1u : 0u);
              if (SPLIT) umma::mma_ts(tmem + UG::OCOL, pcol + 64 + 8 * ks, d, idO, 1u);
            }
          }
          o_init = true;
          umma::commit(pv_done);
          umma::commit(&kv_empty[st]);
          return true;
        };
        for (int j = 0; j < ntiles && ok; ++j) {
          const int g = gt + j, st = g % KST, b = g & 1;
          if (abort_now() || !umma::wait(&kv_full[st], (uint32_t)((g / KST) & 1))) {
            ok = false;
            break;
          }
          umma::fence_after();
          const int t0 = kv_beg + j * KT;
          const int live = (kv_end - t0 + BS - 1) / BS;  // pages with keys
          const uint64_t kd = k_desc0 + (uint64_t)((st * UG::STAGE) >> 4);
          if constexpr (GK) {
            // S = Q K^T as one N = 128 product per 16-dim k-step
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
              umma::mma_ts(tmem + UG::SCOL + b * 128, qcol + 8 * ks,
                           kd + (uint64_t)((ks * 2 * KT * 16) >> 4), idS, ks > 0 ? 1u : 0u);
            (void)live;
          } else {
            // S = Q K^T: per page a chain of D/16 products (N = BS); k-step
            // outer so consecutive products go to different pages' accumulators
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
              for (int pg = 0; pg < PAGES; ++pg) {
                if (pg < live)
                  umma::mma_ts(tmem + UG::SCOL + b * 128 + pg * BS, qcol + 8 * ks,
                               kd + (uint64_t)((pg * PAGE + ks * 2 * BS * 16) >> 4), idS, ks > 0 ? 1u : 0u);
              }
            }
          }
          umma::commit(&s_full[b]);
          if (j >= 1 && !issue_pv(j - 1, g - 1)) ok = false;
        }
        if (ok && ntiles > 0 && !abort_now()) ok = issue_pv(ntiles - 1, gt + ntiles - 1);
        gt += ntiles;
      }
      if (!ok) give_up();
      // every product issued so far is complete before TMEM can be freed
      umma::commit(all_done);
      umma::wait(all_done, 0);
    }
    __syncwarp();
  } else {
    // ---- softmax / epilogue: warps w and w + 4 share rows 32w .. 32w + 31
    // (TMEM lanes); `half` 0 takes tokens 0..63 of every tile and O columns
    // 0 .. D/2 - 1, half 1 the rest.  The halves exchange row maxima (and at
    // the end row sums) through shared memory on the `xchg` barrier.
    // The warps' TMEM loads and stores are warp-collective: every decision
    // ahead of one (a wait's outcome, the abort flag) is made for the whole warp.
    auto uwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, umma::wait(bar, parity));
    };
    auto uabort = [&]() -> bool { return __any_sync(0xffffffffu, abort_now()); };
    const int half = warp >> 2;
    const int r = threadIdx.x & 127;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    constexpr int HK = KT / 2;   // tokens of a tile per half
    constexpr int HD = D / 2;    // O columns per half
    constexpr int QC = D / 4;    // Q columns (element pairs) per half
    // O columns per rescale step (P's 64 registers are live there; the cascade
    // forms spill at 32)
    constexpr int RC = CASCADE ? 16 : 32;
    const float qk_scale = p.scale * kLog2e;
    bool ok = true;
    uint32_t xphase = 0;
    // both halves' values of this row: write mine, hand over, read the other's
    // (two buffers by phase parity: a warp a phase ahead cannot overwrite a
    // value the other half has yet to read, since that phase needs its arrival)
    auto exchange = [&](float mine) -> float {
      float* buf = xbuf + (xphase & 1u) * 256;
      buf[half * 128 + r] = mine;
      __syncwarp();
      if (lane == 0) mbar_arrive(xchg);
      const bool got = uwait(xchg, xphase & 1u);
      ++xphase;
      if (!got) {
        ok = false;
        return mine;
      }
      return buf[(half ^ 1) * 128 + r];
    };
    int gt = 0, nread = 0, nq = 0;  // tiles, ring slots read and items with keys of this CTA so far
    // An item as this thread's row sees it.
    struct RowItem {
      int64_t q0;
      int y, kvh, kv_beg, kv_end, ntiles;
      int t, g, end_r, beg_r;  // t: the new token (prefill) or the sequence (cascade) of the row
      bool in_tile;            // a row (else padding of the last tile)
    };
    // The next item with work: read from the producer's slots, and its Q rows
    // staged into TMEM buffer nq & 1 (columns QCOL + (nq & 1) D/2 .., element
    // pairs, QC per half) and handed over.  It is fetched while the previous
    // item's last P.V runs: that item used the other buffer, and every product
    // of the item before it (this buffer's last user) completed before its
    // epilogue.  False at the end marker or on a failed wait.
    auto next_item = [&](RowItem& ri) -> bool {
      for (;;) {
        const int sl = nread & 1;
        if (uabort() || !uwait(&item_full[sl], (uint32_t)((nread >> 1) & 1))) {
          ok = false;
          return false;
        }
        const int idx = *(volatile int*)&s_item[sl];
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[sl]);
        ++nread;
        if (idx >= n_items) return false;
        const UmmaItem it = umma_item<CASCADE>(p, idx, tiles_x, ny);
        if (it.skip) continue;
        ri.q0 = it.q0;
        ri.y = it.y;
        ri.kvh = it.kvh;
        ri.kv_beg = it.kv_beg;
        ri.kv_end = it.kv_end;
        ri.ntiles = it.ntiles;
        bool on;  // a row that sees keys
        const int64_t R = it.R0 + r;
        ri.in_tile = R < it.rows;
        ri.t = ri.in_tile ? (int)(R / G) : 0;
        ri.g = ri.in_tile ? (int)(R - (int64_t)ri.t * G) : 0;
        if constexpr (CASCADE) {
          // the row's sequence sees the chunk up to its own length; lengths the
          // reference zeroes (0 or past max_seq_len) see nothing
          const uint32_t ctx = ri.in_tile ? __ldg(p.context_lens + ri.t) : 0u;
          on = ri.in_tile && ctx != 0 && ctx <= (uint32_t)p.max_seq_len;
          ri.end_r = on ? ((int)ctx < it.kv_end ? (int)ctx : it.kv_end) : 0;
          ri.beg_r = 0;
        } else {
          on = ri.in_tile && !it.bad;
          ri.end_r = on ? it.prefix + ri.t + 1 : 0;
          ri.beg_r = p.window > 0 ? ri.end_r - p.window : 0;
        }
        // (an item without keys hands over no Q: the MMA warp could otherwise see
        // two phases of q_ready complete before it waits for the first)
        if (it.ntiles > 0) {
          const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
              reinterpret_cast<const T*>(p.q) + (it.q0 + ri.t) * p.q_tok_stride +
              (int64_t)(it.kvh * G + ri.g) * p.q_head_stride) + half * QC;
          uint32_t qv[32];
          if (on && (reinterpret_cast<uintptr_t>(qrow) & 15u) == 0) {  // 16-byte loads where the row allows
#pragma unroll
            for (int i = 0; i < QC; i += 4) {
              const uint4 v = __ldg(reinterpret_cast<const uint4*>(qrow + i));
              qv[i] = v.x;
              qv[i + 1] = v.y;
              qv[i + 2] = v.z;
              qv[i + 3] = v.w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < QC; ++i) qv[i] = on ? __ldg(qrow + i) : 0u;
          }
          const uint32_t qcol = lane_base + UG::QCOL + (uint32_t)(nq & 1) * (D / 2) + half * QC;
          if constexpr (QC == 32) umma::st32(qcol, qv);
          else umma::st16(qcol, qv);
          umma::wait_st();
          umma::fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(q_ready);
          ++nq;
        }
        return true;
      }
    };
    RowItem cur;
    bool have_cur = next_item(cur);
    while (ok && have_cur) {
      const int kvh = cur.kvh, kv_beg = cur.kv_beg, kv_end = cur.kv_end, ntiles = cur.ntiles;
      const int t = cur.t, g = cur.g, end_r = cur.end_r, beg_r = cur.beg_r;
      const bool in_tile = cur.in_tile;

      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < ntiles; ++j) {
        const int gg = gt + j, b = gg & 1, st = gg % KST;
        if (uabort() || !uwait(&s_full[b], (uint32_t)((gg >> 1) & 1))) {
          ok = false;
          break;
        }
        umma::fence_after();
        // (the stage's barrier orders the producer's page mask and the TMA-written
        // V before this thread reads or clears them; its phase cannot move on
        // before this tile's P is handed over)
        if (!uwait(&kv_full[st], (uint32_t)((gg / KST) & 1))) {
          ok = false;
          break;
        }
        const int t0 = kv_beg + j * KT + half * HK;  // first token of my half
        const uint32_t pm = page_mask[st];
        float x[HK];
#pragma unroll
        for (int c = 0; c < HK; c += 32) {
          uint32_t v[32];
          umma::ld32(lane_base + UG::SCOL + b * 128 + half * HK + c, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c + i] = __uint_as_float(v[i]);
        }
        umma::wait_ld();
        // A half tile every row of the warp sees whole (its pages loaded, inside
        // every row's [start, end)) needs no per-token mask.
        const uint32_t my_pages = HK >= BS ? ((1u << (HK / BS)) - 1u) << (half * HK / BS) : 0u;
        const bool whole =
            __all_sync(0xffffffffu, (pm & my_pages) == my_pages && t0 >= beg_r && t0 + HK <= end_r);
        float mx;  // row max of my scaled scores (log2 units)
        if (whole) {
          // the largest raw score, or the smallest for a negative scale
          float h0 = -INFINITY, h1 = -INFINITY;
          if (qk_scale >= 0.f) {
#pragma unroll
            for (int c = 0; c < HK; c += 2) {
              h0 = fmaxf(h0, x[c]);
              h1 = fmaxf(h1, x[c + 1]);
            }
            mx = fmaxf(h0, h1) * qk_scale;
          } else {
#pragma unroll
            for (int c = 0; c < HK; c += 2) {
              h0 = fmaxf(h0, -x[c]);
              h1 = fmaxf(h1, -x[c + 1]);
            }
            mx = -fmaxf(h0, h1) * qk_scale;
          }
        } else {
          mx = -INFINITY;
#pragma unroll
          for (int c = 0; c < HK; ++c) {
            const int tok = t0 + c;
            const bool vis = tok >= beg_r && tok < end_r && ((pm >> ((half * HK + c) / BS)) & 1u);
            x[c] = vis ? x[c] * qk_scale : -INFINITY;
            mx = fmaxf(mx, x[c]);
          }
        }
        mx = fmaxf(mx, exchange(mx));
        if (!ok) break;
        // lazy max (the same in both halves): rescale only when it rises by more than 2^8
        float alpha = 1.f;
        if (mx > m_ref + 8.f) {
          alpha = m_ref == -INFINITY ? 0.f : fast_exp2(m_ref - mx);
          m_ref = mx;
        }
        const float neg_ref = m_ref == -INFINITY ? 0.f : -m_ref;
        // P pairs packed as soon as they are exponentiated (the integer / FMA
        // work of the packing overlaps the special-function unit's exponentials):
        // hi = the upper 16 bits of each fp32 (a bf16, truncated), lo = the exact
        // remainder rounded to bf16, so hi + lo carries ~16 bits of P; f16 P is
        // one rounding.  Pairs of tokens 64h + 2i, + 1 go to hi column 32h + i.
        // The exponent, the row sum and the remainder run as f32x2 pairs.
        float2 ps = make_float2(0.f, 0.f);
        uint32_t hi[32], lo[32];
        auto pack_pair = [&](int i, float2 pp) {
          ps = add_x2(ps, pp);
          if constexpr (SPLIT) {
            const uint32_t u0 = __float_as_uint(pp.x), u1 = __float_as_uint(pp.y);
            hi[i] = __byte_perm(u0, u1, 0x7632);
            const float2 r = sub_x2(pp, make_float2(__uint_as_float(u0 & 0xFFFF0000u), __uint_as_float(u1 & 0xFFFF0000u)));
            lo[i] = MmaOp<T>::pack(r.x, r.y);
          } else {
            hi[i] = MmaOp<T>::pack(pp.x, pp.y);
            lo[i] = 0u;
          }
        };
        if (whole) {
          const float2 sc = make_float2(qk_scale, qk_scale), nr = make_float2(neg_ref, neg_ref);
#pragma unroll
          for (int i = 0; i < HK / 2; ++i) {
            const float2 e = fma_x2(make_float2(x[2 * i], x[2 * i + 1]), sc, nr);
            pack_pair(i, make_float2(fast_exp2(e.x), fast_exp2(e.y)));
          }
        } else {
          const float2 nr = make_float2(neg_ref, neg_ref);
#pragma unroll
          for (int i = 0; i < HK / 2; ++i) {
            const float2 e = add_x2(make_float2(x[2 * i], x[2 * i + 1]), nr);  // masked: exp2(-inf) = 0
            pack_pair(i, make_float2(fast_exp2(e.x), fast_exp2(e.y)));
          }
        }
        l = l * alpha + (ps.x + ps.y);  // this half's share of the row sum
        // O is rescaled once P.V of the previous tile is done.  P needs no wait:
        // it goes to this tile's S buffer, whose last reader (P.V two tiles
        // back) completed before this tile's S did.  pv_done cannot run two
        // phases ahead of this thread (P.V of this tile needs its P), so the
        // phases not waited for here keep the parity test exact.
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
          if (!uwait(pv_done, (uint32_t)((gg - 1) & 1))) {
            ok = false;
            break;
          }
          umma::fence_after();
#pragma unroll
          for (int c = 0; c < HD; c += RC) {
            uint32_t v[RC];
            if constexpr (RC == 16) umma::ld16(lane_base + UG::OCOL + half * HD + c, v);
            else umma::ld32(lane_base + UG::OCOL + half * HD + c, v);
            umma::wait_ld();
#pragma unroll
            for (int i = 0; i < RC; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            if constexpr (RC == 16) umma::st16(lane_base + UG::OCOL + half * HD + c, v);
            else umma::st32(lane_base + UG::OCOL + half * HD + c, v);
          }
        }
        // the last tile's partial page: V of tokens past the context end becomes 0
        // (its slots may hold anything and 0 * NaN = NaN); half 0, thread d clears row d
        const int tile0 = kv_beg + j * KT;
        if (half == 0 && tile0 + KT > kv_end && (kv_end - tile0) % BS != 0) {
          const int pg = (kv_end - tile0) / BS, from = (kv_end - tile0) % BS;
          if ((pm >> pg) & 1u) {
            uint8_t* vpage = ring + (size_t)st * UG::STAGE + PAGES * PAGE + pg * PAGE;
            const int d = r;
            if (d < D) {
              for (int tk = from; tk < BS; ++tk) {
                const int ch = tk / 8;
                const int phys = BS == 32 ? (ch ^ ((d >> 1) & 3)) : (ch ^ ((d >> 2) & 1));
                *reinterpret_cast<uint16_t*>(vpage + d * BS * 2 + phys * 16 + (tk % 8) * 2) = 0;
              }
            }
            fence_proxy_async();
          }
        }
        // P over the S buffer: hi pairs of tokens 64h .. 64h + 63 in columns
        // 32h .. 32h + 31, lo pairs 64 columns further
        umma::st32(lane_base + UG::SCOL + b * 128 + half * 32, hi);
        if constexpr (SPLIT) umma::st32(lane_base + UG::SCOL + b * 128 + 64 + half * 32, lo);
        umma::wait_st();
        umma::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
      }
      // the next item's Q goes in while this item's last P.V runs
      RowItem nxt;
      const bool have_nxt = ok && next_item(nxt);
      bool have = ok && ntiles > 0;
      if (have) {
        have = uwait(pv_done, (uint32_t)((gt + ntiles - 1) & 1));
        if (!have) ok = false;
        umma::fence_after();
      }
      // both halves must take the last exchange (or time out on it) alike
      const float l_all = l + exchange(l);
      have = have && ok;
      if constexpr (CASCADE) {
        // ---- partials of partition y (the chunk): natural-log max, sum,
        // unnormalised O (0 for a row without keys, whose max is -inf)
        const bool keep = have && l_all > 0.f;
        const int head = kvh * G + g;
        float* po = p.part_out + (int64_t)t * p.part_out_seq_stride + (int64_t)head * p.part_out_head_stride +
                    (int64_t)cur.y * p.part_out_part_stride + half * HD;
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t v[32];
          // (tcgen05.ld is warp-collective: every lane loads, only rows store)
          umma::ld32(lane_base + UG::OCOL + half * HD + c, v);
          umma::wait_ld();
          if (in_tile) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(po + c + i) =
                  keep ? make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                                     __uint_as_float(v[i + 3]))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        if (in_tile && half == 0) {
          const int64_t o = (int64_t)t * p.part_seq_stride + (int64_t)head * p.part_head_stride + cur.y;
          p.part_max[o] = keep ? m_ref * kLn2 : -INFINITY;
          p.part_sum[o] = keep ? l_all : 0.f;
        }
      } else {
        // ---- epilogue: O / l (a row with no visible key, or after an abort, is 0)
        const bool nonzero = have && l_all > 0.f;  // else explicit zeros (O may hold another item's values)
        const float inv = nonzero ? 1.f / l_all : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (cur.q0 + t) * p.out_tok_stride +
                  (int64_t)(kvh * G + g) * p.out_head_stride + half * HD;
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t v[32];
          umma::ld32(lane_base + UG::OCOL + half * HD + c, v);
          umma::wait_ld();
          if (in_tile) {
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              packed[i] =
                  nonzero ? pack_out<T>(__uint_as_float(v[2 * i]) * inv, __uint_as_float(v[2 * i + 1]) * inv) : 0u;
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<uint4*>(orow + c + 2 * i) =
                  make_uint4(packed[i], packed[i + 1], packed[i + 2], packed[i + 3]);
          }
        }
      }
      // (the next item's first P.V comes after these O loads)
      umma::fence_before();
      gt += ntiles;
      cur = nxt;
      have_cur = have_nxt;
    }
    if (!ok && lane == 0) give_up();
  }

  umma::fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    umma::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  // this CTA claims no more items: the last CTA out returns the counters to zero
  if (dynamic && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&g_umma_sched[slot].done, 1u) == gridDim.x - 1) {
      atomicExch(&g_umma_sched[slot].next, 0u);
      atomicExch(&g_umma_sched[slot].done, 0u);
    }
  }
}

// K viewed as rows of one 8-dim chunk of one page of one head: [nb * H * D/8][BS * 8]
// (needs the dense paged layout).
static bool make_k_gather_map(const PrefillArgs& a, int D, int BS, CUtensorMap* map) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)BS * 8, (cuuint64_t)a.num_blocks * a.num_kv_heads * (D / 8)};
  const cuuint64_t strides[1] = {(cuuint64_t)BS * 16};
  const cuuint32_t box[2] = {(cuuint32_t)BS * 8, 1};
  const cuuint32_t ones[2] = {1, 1};
  return enc(map, a.q_type == ElemType::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<void*>(a.k_cache), dims, strides, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// KVC_PREFILL_ISSUE=single: the producer's lane 0 issues every copy (tuning runs).
static int umma_single_issue() {
  const char* v = getenv("KVC_PREFILL_ISSUE");
  return v && v[0] == 's' ? 1 : 0;
}

// The persistent grid: one CTA per SM (the ring and TMEM allow one), fewer
// when there are fewer work items.
static int umma_persistent_ctas(int dev, int64_t items) {
  static std::atomic<int> sms[64];  // per device, written once (any racing writer stores the same value)
  int n = dev >= 0 && dev < 64 ? sms[dev].load() : 0;
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0 && dev < 64) sms[dev] = n;
  }
  return (int)(items < n ? items : n);
}

static int umma_sched_slot(cudaStream_t stream) {
  static std::atomic<unsigned> next{0}, next_captured{0};
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    (void)cudaGetLastError();  // (the launch on this stream reports any real fault)
    cs = cudaStreamCaptureStatusNone;
  }
  if (cs == cudaStreamCaptureStatusActive)
    return kUmmaSchedSlots - kUmmaSchedCaptured +
           (int)(next_captured.fetch_add(1u, std::memory_order_relaxed) % (unsigned)kUmmaSchedCaptured);
  return (int)(next.fetch_add(1u, std::memory_order_relaxed) % (unsigned)(kUmmaSchedSlots - kUmmaSchedCaptured));
}

// the two-tile form of the gathered-K kernel (prefill_umma_pair.cuh)
static bool pair_enabled();
template <typename T, int D, int BS, bool CASCADE>
static cudaError_t launch_pair(const PrefillArgs& a, const TmaMaps& maps, int64_t tiles, int ny, cudaStream_t stream);

template <typename T, int D, int BS, bool GK>
static cudaError_t launch_prefill_umma(const PrefillArgs& a, cudaStream_t stream) {
  using UG = UmmaGeom<D, BS>;
  DecodeParams dp;
  memset(&dp, 0, sizeof(dp));
  dp.k_cache = a.k_cache;
  dp.v_cache = a.v_cache;
  dp.num_blocks = a.num_blocks;
  dp.num_kv_heads = a.num_kv_heads;
  dp.k_head_stride = a.k_head_stride;
  dp.k_block_stride = a.k_block_stride;
  dp.v_head_stride = a.v_head_stride;
  dp.v_block_stride = a.v_block_stride;
  TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  // the kTiles maps: V as [nb][H][D][BS] pages, one whole page per box, bs*2-byte swizzle
  if (!make_tensor_maps(dp, std::is_same<T, __nv_bfloat16>::value ? ElemType::BF16 : ElemType::F16, D, BS, BS, BS * 2,
                        kTiles, &maps))
    return cudaErrorNotSupported;
  if (GK && !make_k_gather_map(a, D, BS, &maps.k)) return cudaErrorNotSupported;
  if constexpr (GK) {
    if (pair_enabled()) {
      const int G2 = a.num_heads / a.num_kv_heads;
      const int64_t tiles2 = ((int64_t)a.max_q_len * G2 + kUmmaRows - 1) / kUmmaRows;
      if (tiles2 <= 0 || a.num_seqs <= 0) return cudaSuccess;
      const cudaError_t e = launch_pair<T, D, BS, false>(a, maps, tiles2, (int)a.num_seqs, stream);
      if (e != cudaErrorNotSupported) return e;
    }
  }
  auto kern = prefill_umma_kernel<T, D, BS, GK>;
  static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, UG::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int G = a.num_heads / a.num_kv_heads;
  const int64_t tiles = ((int64_t)a.max_q_len * G + kUmmaRows - 1) / kUmmaRows;
  if (tiles <= 0 || a.num_seqs <= 0) return cudaSuccess;
  const int64_t items = tiles * a.num_seqs * a.num_kv_heads;
  if (items > 0x7fffffffll - 1024) return cudaErrorInvalidValue;
  const int ctas = umma_persistent_ctas(dev, items);
  const int slot = umma_sched_slot(stream);  // (runtime queries stay outside the launch statement)
  PrefillArgs aa = a;
  aa.single_issue = umma_single_issue();
  kern<<<ctas, kUmmaThreads, UG::SMEM, stream>>>(aa, maps, (int)tiles, (int)a.num_seqs, slot);
  count_launch();
  return cudaGetLastError();
}

// The tcgen05 kernel serves the paged layout with block size 16 or 32 (pages
// tile a 128-token S tile; V rows of 32 or 64 bytes match a swizzle mode).
static bool prefill_umma_supported(const PrefillArgs& a) {
  if (a.token_major || !(a.block_size == 16 || a.block_size == 32) || !(a.head_size == 64 || a.head_size == 128))
    return false;
  // rows are stored as 16-byte vectors
  if ((reinterpret_cast<uintptr_t>(a.out) & 15u) || (a.out_tok_stride & 7) || (a.out_head_stride & 7)) return false;
  const char* v = getenv("KVC_PREFILL_KERNEL");
  return !(v && (v[0] == 'm' || v[0] == 'M'));  // "mma": the mma.sync kernel
}

static cudaError_t launch_prefill_umma_any(const PrefillArgs& a, cudaStream_t stream) {
  const bool bf = a.q_type == ElemType::BF16;
  const int64_t D = a.head_size, BS = a.block_size;
  // the 4-row gathers need K rows uniformly strided: the dense paged layout
  const bool dense = a.k_head_stride == D * BS && a.k_block_stride == (int64_t)a.num_kv_heads * D * BS &&
                     a.num_blocks * a.num_kv_heads * (D / 8) < 0x7fffffffll;  // (row indices are 32-bit)
  if (a.head_size == 128) {
    if (a.block_size == 32) {
      if (dense)
        return bf ? launch_prefill_umma<__nv_bfloat16, 128, 32, true>(a, stream)
                  : launch_prefill_umma<__half, 128, 32, true>(a, stream);
      return bf ? launch_prefill_umma<__nv_bfloat16, 128, 32, false>(a, stream)
                : launch_prefill_umma<__half, 128, 32, false>(a, stream);
    }
    if (dense)
      return bf ? launch_prefill_umma<__nv_bfloat16, 128, 16, true>(a, stream)
                : launch_prefill_umma<__half, 128, 16, true>(a, stream);
    return bf ? launch_prefill_umma<__nv_bfloat16, 128, 16, false>(a, stream)
              : launch_prefill_umma<__half, 128, 16, false>(a, stream);
  }
  if (a.block_size == 32) {
    if (dense)
      return bf ? launch_prefill_umma<__nv_bfloat16, 64, 32, true>(a, stream)
                : launch_prefill_umma<__half, 64, 32, true>(a, stream);
    return bf ? launch_prefill_umma<__nv_bfloat16, 64, 32, false>(a, stream)
              : launch_prefill_umma<__half, 64, 32, false>(a, stream);
  }
  if (dense)
    return bf ? launch_prefill_umma<__nv_bfloat16, 64, 16, true>(a, stream)
              : launch_prefill_umma<__half, 64, 16, true>(a, stream);
  return bf ? launch_prefill_umma<__nv_bfloat16, 64, 16, false>(a, stream)
            : launch_prefill_umma<__half, 64, 16, false>(a, stream);
}

// ---- shared-prefix (cascade) decode through the tcgen05 kernel ----
template <typename T, int D, int BS, bool GK>
static cudaError_t launch_cascade_umma(const PrefillArgs& a, int prefix_parts, cudaStream_t stream) {
  using UG = UmmaGeom<D, BS>;
  DecodeParams dp;
  memset(&dp, 0, sizeof(dp));
  dp.k_cache = a.k_cache;
  dp.v_cache = a.v_cache;
  dp.num_blocks = a.num_blocks;
  dp.num_kv_heads = a.num_kv_heads;
  dp.k_head_stride = a.k_head_stride;
  dp.k_block_stride = a.k_block_stride;
  dp.v_head_stride = a.v_head_stride;
  dp.v_block_stride = a.v_block_stride;
  TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!make_tensor_maps(dp, std::is_same<T, __nv_bfloat16>::value ? ElemType::BF16 : ElemType::F16, D, BS, BS, BS * 2,
                        kTiles, &maps))
    return cudaErrorNotSupported;
  if (GK && !make_k_gather_map(a, D, BS, &maps.k)) return cudaErrorNotSupported;
  if constexpr (GK) {
    if (pair_enabled()) {
      const int G2 = a.num_heads / a.num_kv_heads;
      const cudaError_t e = launch_pair<T, D, BS, true>(
          a, maps, ((int64_t)a.num_seqs * G2 + kUmmaRows - 1) / kUmmaRows, prefix_parts, stream);
      if (e != cudaErrorNotSupported) return e;
    }
  }
  auto kern = prefill_umma_kernel<T, D, BS, GK, true>;
  static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, UG::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int G = a.num_heads / a.num_kv_heads;
  const int64_t tiles = ((int64_t)a.num_seqs * G + kUmmaRows - 1) / kUmmaRows;
  const int64_t items = tiles * prefix_parts * a.num_kv_heads;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffffll - 1024) return cudaErrorInvalidValue;
  const int ctas = umma_persistent_ctas(dev, items);
  const int slot = umma_sched_slot(stream);
  PrefillArgs aa = a;
  aa.single_issue = umma_single_issue();
  // a programmatic dependent of the kernel before it (see the kernel's start)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kUmmaThreads);
  cfg.dynamicSmemBytes = UG::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, aa, maps, (int)tiles, prefix_parts, slot);
  count_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

// The prefix of a shared-prefix decode on the tensor cores' own pipeline when
// the cache suits the gathered-K tcgen05 kernel (dense paged layout, block size
// 16 or 32, head size 64 / 128, prefix and chunks in whole blocks, partial
// buffers of 16-byte rows);
// cudaErrorNotSupported otherwise (the caller then runs the mma.sync prefix
// kernel).
static cudaError_t launch_cascade_prefix_umma(const DecodeParams& p, const DecodeArgs& da, cudaStream_t stream) {
  const int D = da.head_size, BS = da.block_size;
  // Only the gathered-K form (dense K): with per-page S chains (N = 16 for
  // block size 16, 64 products per tile) the single-lane product issue set the
  // pace and config 4 measured 69.0 us against 65.9 us for the mma.sync prefix
  // kernel.
  if (!(BS == 16 || BS == 32) || !(D == 64 || D == 128)) return cudaErrorNotSupported;
  if (!(p.k_head_stride == (int64_t)D * BS && p.k_block_stride == (int64_t)p.num_kv_heads * D * BS))
    return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(p.part_out) & 15u) || (p.part_out_seq_stride & 3) || (p.part_out_head_stride & 3) ||
      (p.part_out_part_stride & 3) || (p.prefix_len % BS) || (p.prefix_part_size % BS))
    return cudaErrorNotSupported;
  const char* v = getenv("KVC_PREFILL_KERNEL");
  if (v && (v[0] == 'm' || v[0] == 'M')) return cudaErrorNotSupported;
  PrefillArgs a;
  memset(&a, 0, sizeof(a));
  a.q = p.q;
  a.k_cache = p.k_cache;
  a.v_cache = p.v_cache;
  a.block_tables = p.block_tables;
  a.num_seqs = p.num_seqs;
  a.num_heads = p.num_heads;
  a.num_kv_heads = p.num_kv_heads;
  a.block_size = BS;
  a.num_blocks = p.num_blocks;
  a.table_stride = p.table_stride;
  a.q_tok_stride = p.q_seq_stride;
  a.q_head_stride = p.q_head_stride;
  a.k_block_stride = p.k_block_stride;
  a.k_head_stride = p.k_head_stride;
  a.v_block_stride = p.v_block_stride;
  a.v_head_stride = p.v_head_stride;
  a.scale = p.scale;
  a.q_type = da.q_type;
  a.head_size = D;
  a.context_lens = p.context_lens;
  a.max_seq_len = p.max_seq_len;
  a.prefix_len = p.prefix_len;
  a.prefix_part_size = p.prefix_part_size;
  a.part_max = p.part_max;
  a.part_sum = p.part_sum;
  a.part_out = p.part_out;
  a.part_seq_stride = p.part_seq_stride;
  a.part_head_stride = p.part_head_stride;
  a.part_out_seq_stride = p.part_out_seq_stride;
  a.part_out_head_stride = p.part_out_head_stride;
  a.part_out_part_stride = p.part_out_part_stride;
  const bool bf = a.q_type == ElemType::BF16;
  const bool dense = a.k_head_stride == (int64_t)D * BS && a.k_block_stride == (int64_t)a.num_kv_heads * D * BS &&
                     a.num_blocks * a.num_kv_heads * (D / 8) < 0x7fffffffll;
  const int parts = p.prefix_parts;
  if (!dense) return cudaErrorNotSupported;
  if (D == 128)
    return BS == 32 ? (bf ? launch_cascade_umma<__nv_bfloat16, 128, 32, true>(a, parts, stream)
                          : launch_cascade_umma<__half, 128, 32, true>(a, parts, stream))
                    : (bf ? launch_cascade_umma<__nv_bfloat16, 128, 16, true>(a, parts, stream)
                          : launch_cascade_umma<__half, 128, 16, true>(a, parts, stream));
  return BS == 32 ? (bf ? launch_cascade_umma<__nv_bfloat16, 64, 32, true>(a, parts, stream)
                        : launch_cascade_umma<__half, 64, 32, true>(a, parts, stream))
                  : (bf ? launch_cascade_umma<__nv_bfloat16, 64, 16, true>(a, parts, stream)
                        : launch_cascade_umma<__half, 64, 16, true>(a, parts, stream));
}

cudaError_t launch_paged_prefill(const PrefillArgs& a, cudaStream_t stream) {
  if (a.num_seqs <= 0 || a.max_q_len <= 0) return cudaSuccess;
  if (a.num_seqs > 65535 || a.num_kv_heads > 65535) return cudaErrorInvalidValue;
  if (prefill_umma_supported(a)) return launch_prefill_umma_any(a, stream);
  return launch_prefill_mma_any(a, stream);
}

}  // namespace kvc
