// prefill_umma_pair.cuh — the tcgen05 attention core with two 128-row query
// tiles per work item (sm_100a).  Included by decode.cu after
// prefill_umma.cuh; same arguments, items and results as prefill_umma_kernel
// in its gathered-K form (dense paged K cache, block size 16 or 32), prefill /
// extend and the shared-prefix (cascade) form.
//
// Why a second form: with one 128-row tile per CTA, one 128-token tile of keys
// takes ~1536 cycles of tensor work (S = Q K^T, then P.V as bf16 hi + lo) but
// ~3260 cycles of wall time, because the whole softmax chain of the tile (wait
// for S, row maxima, 16K exponentials on the SFU, P into TMEM) runs between
// its S and its P.V, and the two softmax halves of a row exchange maxima
// through shared memory.  Here a work item is 256 rows, tile A (rows 0..127)
// and tile B (rows 128..255) of the same sequence (or, in the cascade form,
// of the same batch) and KV head, both meeting the same key tiles:
//  * TMEM (512 columns): S/P of tile t at 128 t (P overwrites its S: for
//    tokens 32c .. 32c + 31, pair (2i, 2i + 1) in column 32c + i, bf16's lo
//    part 16 columns on), O of tile t at 256 + D t.  Q of both tiles lives in shared
//    memory as [D/8][128][8] K-major operands, so S = Q K^T reads A from a
//    shared-memory descriptor.
//  * Warps 0-3 are tile A's softmax, warps 4-7 tile B's: one thread per row,
//    every key column of the row, no exchange between threads.
//  * The MMA lane interleaves the tiles, P.V of A then S of A's next key tile,
//    then the same for B, so the tensor core runs one tile's products while
//    the other tile's softmax runs.
//  * K and V have rings of their own: a K tile is free once both tiles' S
//    have read it, a V tile only after both P.V, so K runs further ahead.
//    Warp 8 claims the items (the device counters of prefill_umma_kernel) and
//    gathers K (4-row gathers per 8-dim chunk of four pages); warp 10 copies
//    the V pages through the swizzled tensor map and records which pages of
//    the tile were loaded.
// The softmax reads each S tile twice from TMEM (row maxima, then the
// exponentials), 32 columns at a time.
// A key tile is streamed once for both tiles; tile A, whose rows end earlier
// (causal), stops after its own last key tile.  Every wait is bounded
// (KVC_STATUS_WAIT_TIMEOUT, then an abort flag ends every loop); TMEM is freed
// after a final commit shows every product done.
#pragma once

namespace kvc {

constexpr int kPairRows = 2 * kUmmaRows;  // query rows of one work item: tiles A and B
// 12 warps: softmax warpgroups 0 (tile A) and 1 (tile B), then warpgroup 2 =
// the K producer (warp 8), the MMA lane (warp 9), the V producer (warp 10) and
// an idle warp.  The softmax threads take most registers, so the
// register file is split after the launch (setmaxnreg): warpgroup 2 gives its
// registers down to kPairRegsOther, the softmax warpgroups take theirs up to
// kPairRegsSoftmax.  The launch provides kPairThreads x (the kernel's register
// count); the host launches the kernel only when that covers the split, since
// a setmaxnreg.inc the pool cannot serve would wait for good.
constexpr int kPairThreads = 384;
constexpr int kPairRegsSoftmax = 192, kPairRegsOther = 120;
constexpr int kPairRegsNeeded = 256 * kPairRegsSoftmax + 128 * kPairRegsOther;
constexpr int kPairVWarp = 10;

template <int D, int BS>
struct PairGeom {
  static constexpr int PAGES = kUmmaTile / BS;
  static constexpr int PAGE = D * BS * 2;            // bytes of one K (or V) page of one head
  static constexpr int TILE = PAGES * PAGE;          // one 128-token K (gathered) or V tile
  static constexpr int KS = D == 128 ? 3 : 4;        // K ring stages
  static constexpr int VS = D == 128 ? 2 : 4;        // V ring stages
  static constexpr int QTILE = kUmmaRows * D * 2;    // one Q tile, [D/8][128][8]
  static constexpr int V_OFF = KS * TILE, Q_OFF = V_OFF + VS * TILE;
  static constexpr int BAR_OFF = 1024 + Q_OFF + 2 * QTILE;  // (1024: alignment slack of the rings)
  // k full/empty, v full/empty, s_full, p_full, pv_done, q_ready (per tile), all_done
  static constexpr int NBARS = 2 * KS + 2 * VS + 2 + 2 + 2 + 2 + 1;
  static constexpr int MASK_OFF = BAR_OFF + NBARS * 8;  // loaded-page masks of the V stages
  static constexpr int SMEM = (MASK_OFF + VS * 4 + 15) / 16 * 16;
  static constexpr uint32_t SCOL = 0, OCOL = 256;    // TMEM columns: S/P of tile t at 128 t, O of tile t at 256 + D t
  static_assert(OCOL + 2 * D <= 512, "TMEM columns");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(TILE % 1024 == 0 && QTILE % 1024 == 0, "operand alignment");
};

// The two values of a packed T pair, widened to float.
template <typename T>
__device__ __forceinline__ float rounded_lo(uint32_t v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(v << 16);
  else return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu)));
}
template <typename T>
__device__ __forceinline__ float rounded_hi(uint32_t v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(v & 0xFFFF0000u);
  else return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
}

struct PairItem {
  UmmaItem u;  // the rows of both tiles (R0 .. R0 + 255), the union of their key ranges
  int nt[2];   // key tiles of tile A and of tile B (0: a tile without rows)
};

template <bool CASCADE>
__device__ __forceinline__ PairItem pair_item(const PrefillArgs& p, int idx, int pairs_x, int ny) {
  constexpr int KT = kUmmaTile;
  PairItem pi;
  UmmaItem& it = pi.u;
  const int xi = idx % pairs_x;
  it.y = (idx / pairs_x) % ny;
  it.kvh = idx / (pairs_x * ny);
  it.R0 = (int64_t)(pairs_x - 1 - xi) * kPairRows;  // within a sequence, the last (longest) rows first
  it.first_tile = xi == pairs_x - 1;
  it.q0 = 0;
  it.rows = 0;
  it.prefix = 0;
  it.kv_beg = 0;
  it.kv_end = 0;
  it.bad = false;
  it.skip = true;
  it.ntiles = 0;
  pi.nt[0] = pi.nt[1] = 0;
  const int G = p.num_heads / p.num_kv_heads;
  int end_a = 0;  // key range end of tile A's rows
  if constexpr (CASCADE) {
    it.rows = (int64_t)p.num_seqs * G;
    if (it.R0 >= it.rows) return pi;
    it.kv_beg = it.y * p.prefix_part_size;
    it.kv_end = it.kv_beg + p.prefix_part_size < p.prefix_len ? it.kv_beg + p.prefix_part_size : p.prefix_len;
    end_a = it.kv_end;
  } else {
    it.q0 = p.qo_indptr[it.y];
    const int64_t q1 = p.qo_indptr[it.y + 1];
    const int64_t kvl = p.kv_lens[it.y];
    const int64_t ql = q1 - it.q0;
    it.rows = ql * G;
    if (ql <= 0 || it.R0 >= it.rows || q1 > p.num_tokens) {
      it.bad = q1 > p.num_tokens && ql > 0;
      return pi;
    }
    it.bad = ql > p.max_q_len || kvl < ql || kvl > p.table_len * (int64_t)p.block_size || kvl > 0x7fffffffll - 256;
    it.prefix = it.bad ? 0 : (int)(kvl - ql);
    const int64_t R_last = (it.R0 + kPairRows < it.rows ? it.R0 + kPairRows : it.rows) - 1;
    const int64_t R_last_a = (it.R0 + kUmmaRows < it.rows ? it.R0 + kUmmaRows : it.rows) - 1;
    const int t_first = (int)(it.R0 / G), t_last = (int)(R_last / G), t_last_a = (int)(R_last_a / G);
    it.kv_end = it.bad ? 0 : it.prefix + t_last + 1;
    end_a = it.bad ? 0 : it.prefix + t_last_a + 1;
    int kb = p.window > 0 ? it.prefix + t_first + 1 - p.window : 0;
    it.kv_beg = kb > 0 ? kb / KT * KT : 0;
  }
  it.ntiles = it.kv_end > it.kv_beg ? (it.kv_end - it.kv_beg + KT - 1) / KT : 0;
  pi.nt[0] = end_a > it.kv_beg ? (end_a - it.kv_beg + KT - 1) / KT : 0;
  pi.nt[1] = it.R0 + kUmmaRows < it.rows ? it.ntiles : 0;
  it.skip = false;
  return pi;
}

namespace umma {
// 32 lanes x 32 consecutive 32-bit columns in one store
__device__ __forceinline__ void st32x(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// D[tmem] (+)= A[smem descriptor] * B[smem descriptor]
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
}  // namespace umma

template <typename T, int D, int BS, bool CASCADE = false>
__global__ void __launch_bounds__(kPairThreads, 1)
    prefill_pair_kernel(const PrefillArgs p, const __grid_constant__ TmaMaps maps, int pairs_x, int ny, int slot) {
  using namespace mma_detail;
  using PG = PairGeom<D, BS>;
  constexpr int PAGES = PG::PAGES, PAGE = PG::PAGE, KS = PG::KS, VS = PG::VS, KT = kUmmaTile;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr bool SPLIT = BF16;  // bf16 P as hi + lo; f16 P as it is
  static_assert(PAGES % 4 == 0, "the gathered K layout takes pages in fours");
  static_assert(D / 8 <= 32 && PAGES <= 32, "one lane per K chunk / V page");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ int s_abort;
  __shared__ uint32_t s_tmem;
  __shared__ int s_item[2];
  __shared__ __align__(8) uint64_t item_bars[4];
  uint64_t* item_full = item_bars;       // the K producer published slot i
  uint64_t* item_empty = item_bars + 2;  // its 10 readers (MMA lane, 8 softmax warps, V producer) took slot i
  uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* kring = ring;                 // K tiles [D/8][128][8]
  uint8_t* vring = ring + PG::V_OFF;     // V tiles: PAGES pages [D][BS] (swizzled)
  uint8_t* qsm = ring + PG::Q_OFF;       // Q of tiles A and B
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + PG::BAR_OFF);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + KS;
  uint64_t* v_full = bars + 2 * KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;       // [tile]
  uint64_t* p_full = s_full + 2;         // [tile]
  uint64_t* pv_done = p_full + 2;        // [tile]: the item's last P.V of the tile is done
  uint64_t* q_ready = pv_done + 2;       // [tile]: the tile's Q is in shared memory
  uint64_t* all_done = q_ready + 2;
  uint32_t* vmask = reinterpret_cast<uint32_t*>(smem_raw + PG::MASK_OFF);  // pages loaded, per V stage

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.num_heads / p.num_kv_heads;
  const int n_items = pairs_x * ny * p.num_kv_heads;
  const CUtensorMap* vmap = &maps.v;
  const CUtensorMap* kmap = &maps.k;
  grid_dependents_launch();  // (the shared-prefix form's tail partitions may start beside it)
  const bool dynamic = n_items > (int)gridDim.x;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);  // the tile's four softmax warps
      mbar_init(&pv_done[t], 1);
      mbar_init(&q_ready[t], 4);
    }
    mbar_init(all_done, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 10);
    }
    mbar_fence_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.k)) : "memory");
  } else if (warp == kPairVWarp && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.v)) : "memory");
  }
  // Stale V of pages a tile does not load meets P = 0 (0 * NaN = NaN): the V
  // ring starts from zeros.
  for (int i = threadIdx.x; i < VS * PG::TILE / 16; i += kPairThreads)
    reinterpret_cast<uint4*>(vring)[i] = make_uint4(0u, 0u, 0u, 0u);
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
  // (a producer warp) this lane's page of key tile j of an item: the block id,
  // or ~0 past the item's keys; `valid` = within the keys and a block of the cache
  auto page_id = [&](const uint32_t* table, int kv_beg, int kv_end, int j, bool& in_range) -> uint32_t {
    const int tok = kv_beg + j * KT + lane * BS;
    in_range = lane < PAGES && tok < kv_end;
    return in_range ? __ldg(table + tok / BS) : 0xffffffffu;
  };

  if (warp >= 8) {
    // warpgroup 2 gives registers up (one setmaxnreg for the whole warpgroup)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPairRegsOther));
    if (warp == kProducerWarp) {
      // ---- K producer: claims items, hands each one with rows to the other
      // warps, then gathers the K tiles of both tiles' union of keys
      int gk = 0;    // K tiles of this CTA so far
      int npub = 0;  // items handed over so far
      bool stop = false;
      auto publish = [&](int idx) -> bool {
        const int sl = npub & 1;
        if (npub >= 2 && !umma::wait(&item_empty[sl], (uint32_t)(((npub >> 1) - 1) & 1))) return false;
        *(volatile int*)&s_item[sl] = idx;
        mbar_arrive(&item_full[sl]);
        ++npub;
        return true;
      };
      UmmaSched* sched = &g_umma_sched[slot];
      for (int idx = blockIdx.x; idx < n_items && !stop;) {
        const PairItem pi = pair_item<CASCADE>(p, idx, pairs_x, ny);
        const UmmaItem& it = pi.u;
        if (!CASCADE && it.bad && it.first_tile && it.kvh == 0 && lane == 0)
          set_status(&g_decode_status, KVC_STATUS_INDEX_OOB);
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
        bool handed = true;
        if (lane == 0) handed = publish(idx);
        if (!__shfl_sync(0xffffffffu, handed, 0)) {
          if (lane == 0) give_up();
          break;
        }
        if (__shfl_sync(0xffffffffu, abort_now() ? 1 : 0, 0)) break;
        const int kvh = it.kvh, kv_beg = it.kv_beg, kv_end = it.kv_end, ntiles = it.ntiles;
        const uint32_t* table = p.block_tables + (CASCADE ? (int64_t)0 : (int64_t)it.y * p.table_stride);
        bool in_range;
        uint32_t id = page_id(table, kv_beg, kv_end, 0, in_range);
        for (int j = 0; j < ntiles; ++j) {
          const int g = gk + j, st = g % KS;
          bool ok = true;
          if (g >= KS && lane == 0) ok = umma::wait(&k_empty[st], (uint32_t)(((g / KS) - 1) & 1));
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
          const bool valid = in_range && (int64_t)id < p.num_blocks;
          if (in_range && !valid) set_status(&g_decode_status, KVC_STATUS_BLOCK_OOB);
          const uint32_t mask = __ballot_sync(0xffffffffu, valid);
          uint32_t ids[PAGES];
#pragma unroll
          for (int i = 0; i < PAGES; ++i) ids[i] = __shfl_sync(0xffffffffu, id, i);
          id = page_id(table, kv_beg, kv_end, j + 1, in_range);  // the next tile's ids, in flight meanwhile
          // lane 0 posts the byte count, then lane c < D/8 gathers chunk c of
          // the tile's pages (pages without keys gather a loaded page's rows)
          uint8_t* kst = kring + (size_t)st * PG::TILE;
          if (lane == 0) {
            if (mask) mbar_arrive_expect_tx(&k_full[st], (uint32_t)PG::TILE);
            else mbar_arrive(&k_full[st]);
          }
          __syncwarp();
          if (mask && lane < D / 8) {
            const uint32_t any = ids[__ffs(mask) - 1];
            int rb[PAGES];
#pragma unroll
            for (int i = 0; i < PAGES; ++i)
              rb[i] = (int)(((int64_t)((mask >> i) & 1u ? ids[i] : any) * p.num_kv_heads + kvh) * (D / 8));
            const int c = lane;
#pragma unroll
            for (int q = 0; q < PAGES; q += 4)
              umma::tma_gather4(kst + c * KT * 16 + q * BS * 16, kmap, 0, rb[q] + c, rb[q + 1] + c, rb[q + 2] + c,
                                rb[q + 3] + c, &k_full[st]);
          }
        }
        if (CASCADE && kvh == 0) {
          // every sequence of the item's rows must carry sequence 0's block ids
          // over the chunk (the caller's promise; checked once per item and chunk)
          const int64_t R_last = (it.R0 + kPairRows < it.rows ? it.R0 + kPairRows : it.rows) - 1;
          const int s0 = (int)(it.R0 / G), nseq = (int)(R_last / G) - s0 + 1;
          const int b0 = kv_beg / BS, nb = (kv_end + BS - 1) / BS - b0;
          bool diff = false;
          for (int i = lane; i < nseq * nb; i += 32) {
            const int sq = s0 + i / nb, bb = b0 + i % nb;
            diff |= __ldg(p.block_tables + (int64_t)sq * p.table_stride + bb) != __ldg(p.block_tables + bb);
          }
          if (diff) set_status(&g_decode_status, KVC_STATUS_PREFIX_MISMATCH);
        }
        gk += ntiles;
        if (!stop) idx = claim();
      }
      if (lane == 0 && !publish(n_items)) give_up();
      __syncwarp();
    } else if (warp == kPairVWarp) {
      // ---- V producer: the V pages of every key tile of the items handed over
      int gv = 0, nread = 0;  // V tiles and item slots of this CTA so far
      bool ok = true;
      while (ok) {
        const int sl = nread & 1;
        bool got = true;
        if (lane == 0) got = !abort_now() && umma::wait(&item_full[sl], (uint32_t)((nread >> 1) & 1));
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          break;
        }
        const int idx = *(volatile int*)&s_item[sl];
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[sl]);
        ++nread;
        if (idx >= n_items) break;
        const PairItem pi = pair_item<CASCADE>(p, idx, pairs_x, ny);
        const UmmaItem& it = pi.u;
        if (it.skip) continue;
        const int kvh = it.kvh, kv_beg = it.kv_beg, kv_end = it.kv_end, ntiles = it.ntiles;
        const uint32_t* table = p.block_tables + (CASCADE ? (int64_t)0 : (int64_t)it.y * p.table_stride);
        bool in_range;
        uint32_t id = page_id(table, kv_beg, kv_end, 0, in_range);
        for (int j = 0; j < ntiles && ok; ++j) {
          const int g = gv + j, st = g % VS;
          bool w = true;
          if (g >= VS && lane == 0) w = !abort_now() && umma::wait(&v_empty[st], (uint32_t)(((g / VS) - 1) & 1));
          if (!__shfl_sync(0xffffffffu, w, 0)) {
            ok = false;
            break;
          }
          const bool valid = in_range && (int64_t)id < p.num_blocks;
          const uint32_t mask = __ballot_sync(0xffffffffu, valid);
          const uint32_t my_id = id;
          id = page_id(table, kv_beg, kv_end, j + 1, in_range);
          if (lane == 0) {
            vmask[st] = mask;
            if (mask) mbar_arrive_expect_tx(&v_full[st], (uint32_t)__popc(mask) * (uint32_t)PAGE);
            else mbar_arrive(&v_full[st]);
          }
          __syncwarp();
          if (valid) tma_load_4d(vring + (size_t)st * PG::TILE + lane * PAGE, vmap, 0, 0, kvh, (int)my_id, &v_full[st]);
        }
        gv += ntiles;
      }
      if (!ok && lane == 0) give_up();
      __syncwarp();
    } else if (warp == kMmaWarp) {
      // ---- MMA issue (one lane): per key tile j, P.V of tile A then A's next
      // S, then the same for tile B
      if (lane == 0) {
        const uint32_t idS = umma::instr_desc(BF16, 128, KT), idO = umma::instr_desc(BF16, 128, D);
        // descriptors of stage 0 / Q tile 0, advanced by adding (byte offset >> 4)
        // to the start-address field (shared addresses stay below 256 KB: no carry)
        const uint64_t k_desc0 = umma::smem_desc(smem_u32(kring), KT * 16, 128, umma::kLayoutNone);
        const uint64_t v_desc0 = BS == 32 ? umma::smem_desc(smem_u32(vring), 16, 512, umma::kLayoutSw64)
                                          : umma::smem_desc(smem_u32(vring), 16, 256, umma::kLayoutSw32);
        const uint64_t q_desc0 = umma::smem_desc(smem_u32(qsm), kUmmaRows * 16, 128, umma::kLayoutNone);
        int gt = 0, nread = 0;  // key tiles and item slots of this CTA so far
        int np[2] = {0, 0};     // P hand-overs of each tile waited for so far
        int nq[2] = {0, 0};     // Q hand-overs of each tile waited for so far
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
          const PairItem pi = pair_item<CASCADE>(p, idx, pairs_x, ny);
          const UmmaItem& it = pi.u;
          if (it.skip || it.ntiles == 0) continue;
          const int kv_beg = it.kv_beg, kv_end = it.kv_end, n = it.ntiles;
          auto k_wait = [&](int j) -> bool {
            const int g = gt + j;
            if (abort_now() || !umma::wait(&k_full[g % KS], (uint32_t)((g / KS) & 1))) return false;
            umma::fence_after();
            return true;
          };
          auto issue_s = [&](int t, int j) {
            const uint64_t kd = k_desc0 + (uint64_t)((((gt + j) % KS) * PG::TILE) >> 4);
            const uint64_t qd = q_desc0 + (uint64_t)((t * PG::QTILE) >> 4);
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
              umma::mma_ss(tmem + PG::SCOL + t * 128, qd + (uint64_t)((ks * 2 * kUmmaRows * 16) >> 4),
                           kd + (uint64_t)((ks * 2 * KT * 16) >> 4), idS, ks > 0 ? 1u : 0u);
            umma::commit(&s_full[t]);
          };
          auto issue_pv = [&](int t, int j) -> bool {
            if (!umma::wait(&p_full[t], (uint32_t)(np[t] & 1))) return false;
            ++np[t];
            umma::fence_after();
            const uint64_t vd = v_desc0 + (uint64_t)((((gt + j) % VS) * PG::TILE) >> 4);
            const int steps = (kv_end - (kv_beg + j * KT) + 15) / 16;  // 16-token k-steps with keys
            const uint32_t pcol = tmem + PG::SCOL + t * 128;
            const uint32_t ocol = tmem + PG::OCOL + t * D;
#pragma unroll
            for (int ks = 0; ks < KT / 16; ++ks) {
              if (ks < steps) {
                const uint64_t d = vd + (uint64_t)((((16 * ks) / BS) * PAGE + ((16 * ks) % BS) * 2) >> 4);
                const uint32_t hi = pcol + 32 * (ks >> 1) + 8 * (ks & 1);  // P pairs of tokens 16ks .. 16ks + 15
                umma::mma_ts(ocol, hi, d, idO, (j > 0 || ks > 0) ? 1u : 0u);
                if (SPLIT) umma::mma_ts(ocol, hi + 16, d, idO, 1u);
              }
            }
            return true;
          };
          // a tile's Q is handed over (4 warps) only for an item where the
          // tile has keys; its first S goes out once that Q is in
          auto first_s = [&](int t) -> bool {
            if (abort_now() || !umma::wait(&q_ready[t], (uint32_t)(nq[t] & 1))) return false;
            ++nq[t];
            umma::fence_after();
            issue_s(t, 0);
            return true;
          };
          const int nA = pi.nt[0], nB = pi.nt[1];
          ok = k_wait(0);
          if (ok && nA > 0) ok = first_s(0);
          if (ok && nB > 0) ok = first_s(1);
          if (ok) umma::commit(&k_empty[gt % KS]);
          for (int j = 0; j < n && ok; ++j) {
            const int g = gt + j;
            if (abort_now() || !umma::wait(&v_full[g % VS], (uint32_t)((g / VS) & 1))) {
              ok = false;
              break;
            }
            umma::fence_after();
            if (j < nA) {
              if (!issue_pv(0, j)) {
                ok = false;
                break;
              }
              if (j + 1 == nA) umma::commit(&pv_done[0]);
            }
            if (j + 1 < n && !k_wait(j + 1)) {
              ok = false;
              break;
            }
            if (j + 1 < nA) issue_s(0, j + 1);
            if (j < nB) {
              if (!issue_pv(1, j)) {
                ok = false;
                break;
              }
              if (j + 1 == nB) umma::commit(&pv_done[1]);
            }
            if (j + 1 < nB) issue_s(1, j + 1);
            if (j + 1 < n) umma::commit(&k_empty[(g + 1) % KS]);
            umma::commit(&v_empty[g % VS]);
          }
          gt += n;
          if (!ok) break;
        }
        if (!ok) give_up();
        umma::commit(all_done);
        umma::wait(all_done, 0);
      }
      __syncwarp();
    }
  } else {
    // the softmax warpgroups take the registers warpgroup 2 gave up
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPairRegsSoftmax));
    // ---- softmax / epilogue: warps 0-3 tile A, warps 4-7 tile B; thread =
    // row (TMEM lane), every key column.  TMEM loads and stores are
    // warp-collective: every decision ahead of one is made for the whole warp.
    auto uwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, umma::wait(bar, parity));
    };
    auto uabort = [&]() -> bool { return __any_sync(0xffffffffu, abort_now()); };
    const int tl = warp >> 2;  // my tile
    const int r = threadIdx.x & 127;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t scol = lane_base + PG::SCOL + tl * 128, ocol = lane_base + PG::OCOL + tl * D;
    uint8_t* qtile = qsm + tl * PG::QTILE;
    const float qk_scale = p.scale * kLog2e;
    bool ok = true;
    int gt = 0, nread = 0, ns = 0, ndone = 0;  // key tiles, item slots, S tiles of my tile, items with my P.V
    while (ok) {
      const int sl = nread & 1;
      if (uabort() || !uwait(&item_full[sl], (uint32_t)((nread >> 1) & 1))) {
        ok = false;
        break;
      }
      const int idx = *(volatile int*)&s_item[sl];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[sl]);
      ++nread;
      if (idx >= n_items) break;
      const PairItem pi = pair_item<CASCADE>(p, idx, pairs_x, ny);
      const UmmaItem& it = pi.u;
      if (it.skip) continue;
      const int kvh = it.kvh, kv_beg = it.kv_beg, kv_end = it.kv_end, nu = it.ntiles, nt = pi.nt[tl];
      const int64_t R = it.R0 + tl * kUmmaRows + r;
      const bool in_tile = R < it.rows;
      const int t = in_tile ? (int)(R / G) : 0, g = in_tile ? (int)(R - (int64_t)t * G) : 0;
      bool on;
      int end_r, beg_r;
      if constexpr (CASCADE) {
        const uint32_t ctx = in_tile ? __ldg(p.context_lens + t) : 0u;
        on = in_tile && ctx != 0 && ctx <= (uint32_t)p.max_seq_len;
        end_r = on ? ((int)ctx < kv_end ? (int)ctx : kv_end) : 0;
        beg_r = 0;
      } else {
        on = in_tile && !it.bad;
        end_r = on ? it.prefix + t + 1 : 0;
        beg_r = p.window > 0 ? end_r - p.window : 0;
      }
      if (nt > 0) {
        // Q row -> my tile's [D/8][128][8] operand (zeros for a row without keys);
        // my tile's products of the previous item are done (its last P.V was
        // waited for before its epilogue).  A tile without keys hands over no Q:
        // its warps could otherwise run two hand-overs ahead of the MMA lane.
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
            reinterpret_cast<const T*>(p.q) + (it.q0 + t) * p.q_tok_stride + (int64_t)(kvh * G + g) * p.q_head_stride);
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (on) v = make_uint4(__ldg(qrow + 4 * c), __ldg(qrow + 4 * c + 1), __ldg(qrow + 4 * c + 2),
                                 __ldg(qrow + 4 * c + 3));
          *reinterpret_cast<uint4*>(qtile + (c * kUmmaRows + r) * 16) = v;
        }
        fence_proxy_async();  // the tensor core reads Q through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_ready[tl]);
      }
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < nt; ++j) {
        const int gg = gt + j, vst = gg % VS;
        if (uabort() || !uwait(&s_full[tl], (uint32_t)(ns & 1))) {
          ok = false;
          break;
        }
        ++ns;
        umma::fence_after();
        // (the V stage's barrier orders its page mask, and the V pages this
        // thread may clear; the stage moves on only after this tile's P.V)
        if (!uwait(&v_full[vst], (uint32_t)((gg / VS) & 1))) {
          ok = false;
          break;
        }
        const uint32_t pm = vmask[vst];
        const int tt = kv_beg + j * KT;
        // chunk c (32 tokens) is whole for this warp when its pages are loaded
        // and every row of the warp sees all of it
        auto whole_chunk = [&](int c) -> bool {
          const int t0 = tt + 32 * c;
          const uint32_t pages = BS == 32 ? (1u << c) : (3u << (2 * c));
          return __all_sync(0xffffffffu, (pm & pages) == pages && t0 >= beg_r && t0 + 32 <= end_r);
        };
        auto visible = [&](int c, int i) -> bool {
          const int tok = tt + 32 * c + i;
          return tok >= beg_r && tok < end_r && ((pm >> ((32 * c + i) / BS)) & 1u);
        };
        // (the chunk loops below are loops, their 32-key bodies unrolled: the
        // fully unrolled tile stalled on instruction fetch)
        uint32_t whole = 0u;  // bit c: chunk c whole
#pragma unroll
        for (int c = 0; c < 4; ++c) whole |= whole_chunk(c) ? 1u << c : 0u;
        // pass 1: the row maximum of the scaled scores (log2 units)
        float mx = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          umma::ld32(scol + 32 * c, v);
          umma::wait_ld();
          if ((whole >> c) & 1u) {
            float h[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            float m[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              h[i & 3] = fmaxf(h[i & 3], __uint_as_float(v[i]));
              m[i & 3] = fminf(m[i & 3], __uint_as_float(v[i]));
            }
            const float hi_raw = fmaxf(fmaxf(h[0], h[1]), fmaxf(h[2], h[3]));
            const float lo_raw = fminf(fminf(m[0], m[1]), fminf(m[2], m[3]));
            mx = fmaxf(mx, qk_scale >= 0.f ? hi_raw * qk_scale : lo_raw * qk_scale);
          } else {
            float h[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 32; ++i)
              h[i & 1] = fmaxf(h[i & 1], visible(c, i) ? __uint_as_float(v[i]) * qk_scale : -INFINITY);
            mx = fmaxf(mx, fmaxf(h[0], h[1]));
          }
        }
        // lazy max: O is rescaled only when the row max rises by more than 2^8
        float alpha = 1.f;
        if (mx > m_ref + 8.f) {
          alpha = m_ref == -INFINITY ? 0.f : fast_exp2(m_ref - mx);
          m_ref = mx;
        }
        const float neg_ref = m_ref == -INFINITY ? 0.f : -m_ref;
        // pass 2: P = 2^(s * scale - ref), chunk c (tokens 32c ..) read again
        // and its P stored over its own S columns: pair (2i, 2i + 1) in column
        // 32c + i; bf16 P is split into hi = the upper 16 bits of each fp32 (a
        // bf16, truncated) there and lo = the exact remainder rounded to bf16
        // in column 32c + 16 + i (~16 bits of P together: a row with few keys
        // has no rounding to average out); f16 P is one rounding.  Keys a row
        // does not see enter the exponential as -inf (a select, not a branch
        // around it).
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          umma::ld32(scol + 32 * c, v);
          umma::wait_ld();
          const bool w = (whole >> c) & 1u;
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float e0 = fmaf(__uint_as_float(v[2 * i]), qk_scale, neg_ref);
            float e1 = fmaf(__uint_as_float(v[2 * i + 1]), qk_scale, neg_ref);
            if (!w) {
              e0 = visible(c, 2 * i) ? e0 : -INFINITY;
              e1 = visible(c, 2 * i + 1) ? e1 : -INFINITY;
            }
            const float p0 = fast_exp2(e0), p1 = fast_exp2(e1);
            ps[i & 3] += p0 + p1;
            if constexpr (SPLIT) {
              const uint32_t u0 = __float_as_uint(p0), u1 = __float_as_uint(p1);
              hi[i] = __byte_perm(u0, u1, 0x7632);
              lo[i] = MmaOp<T>::pack(p0 - __uint_as_float(u0 & 0xFFFF0000u), p1 - __uint_as_float(u1 & 0xFFFF0000u));
            } else {
              hi[i] = MmaOp<T>::pack(p0, p1);
            }
          }
          umma::st16(scol + 32 * c, hi);
          if constexpr (SPLIT) umma::st16(scol + 32 * c + 16, lo);
        }
        l = l * alpha + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
        // O of my tile: its P.V of key tile j - 1 is done (s_full of tile j was
        // committed after it)
        if (__any_sync(0xffffffffu, alpha != 1.f) && j >= 1) {
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            uint32_t v[32];
            umma::ld32(ocol + c, v);
            umma::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            umma::st32(ocol + c, v);
          }
        }
        // the union's last tile: V of tokens past its key range becomes 0 (their
        // slots may hold anything and 0 * NaN = NaN); thread d clears row d.
        // Both tiles' warps may clear the same bytes (zeros over zeros).
        if (j == nu - 1 && tt + KT > kv_end && (kv_end - tt) % BS != 0) {
          const int pg = (kv_end - tt) / BS, from = (kv_end - tt) % BS;
          if ((pm >> pg) & 1u) {
            uint8_t* vpage = vring + (size_t)vst * PG::TILE + pg * PAGE;
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
        umma::wait_st();
        umma::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[tl]);
      }
      bool have = ok && nt > 0;
      if (have) {
        have = uwait(&pv_done[tl], (uint32_t)(ndone & 1));
        ++ndone;
        if (!have) ok = false;
        umma::fence_after();
      }
      if constexpr (CASCADE) {
        // ---- partials of partition y (the chunk): natural-log max, sum,
        // unnormalised O (0 for a row without keys, whose max is -inf)
        const bool keep = have && l > 0.f;
        const int head = kvh * G + g;
        float* po = p.part_out + (int64_t)t * p.part_out_seq_stride + (int64_t)head * p.part_out_head_stride +
                    (int64_t)it.y * p.part_out_part_stride;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          if (have) {
            umma::ld32(ocol + c, v);
            umma::wait_ld();
          }
          if (in_tile) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(po + c + i) =
                  keep ? make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                                     __uint_as_float(v[i + 3]))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        if (in_tile) {
          const int64_t o = (int64_t)t * p.part_seq_stride + (int64_t)head * p.part_head_stride + it.y;
          p.part_max[o] = keep ? m_ref * kLn2 : -INFINITY;
          p.part_sum[o] = keep ? l : 0.f;
        }
      } else {
        // ---- epilogue: O / l (a row with no visible key, or after an abort, is 0)
        const bool nonzero = have && l > 0.f;
        const float inv = nonzero ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (it.q0 + t) * p.out_tok_stride +
                  (int64_t)(kvh * G + g) * p.out_head_stride;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          if (have) {
            umma::ld32(ocol + c, v);
            umma::wait_ld();
          }
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
      umma::fence_before();
      gt += nu;
    }
    if (!ok && lane == 0) give_up();
  }

  umma::fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    umma::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  if (dynamic && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&g_umma_sched[slot].done, 1u) == gridDim.x - 1) {
      atomicExch(&g_umma_sched[slot].next, 0u);
      atomicExch(&g_umma_sched[slot].done, 0u);
    }
  }
}

// KVC_PREFILL_PAIR=1 runs the gathered-K launches on the two-tile kernel; by
// default (and with =0) they take the one-tile kernel, which measured faster
// (config-5 chunked prefill 0.441 ms against 0.59 - 0.67 ms for the two-tile
// builds: both are bound by the softmax chain, and a thread here takes twice
// the keys of a row).
static bool pair_enabled() {
  const char* v = getenv("KVC_PREFILL_PAIR");
  return v && v[0] == '1';
}

// Prefill / extend (CASCADE false) or the shared prefix (CASCADE true) on the
// two-tile kernel: `tiles` = 128-row tiles per sequence (prefill) or of the
// batch (cascade), `ny` = sequences (prefill) or prefix chunks (cascade).
// cudaErrorNotSupported (nothing launched) when the build's register count
// cannot serve the register split; the caller then runs the one-tile kernel.
template <typename T, int D, int BS, bool CASCADE>
static cudaError_t launch_pair(const PrefillArgs& a, const TmaMaps& maps, int64_t tiles, int ny,
                               cudaStream_t stream) {
  using PG = PairGeom<D, BS>;
  auto kern = prefill_pair_kernel<T, D, BS, CASCADE>;
  // per device: 0 not yet checked, 1 ready, 2 refused (the register split does
  // not fit the launch); checking twice is harmless
  static std::atomic<int> state[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const int s = dev >= 0 && dev < 64 ? state[dev].load() : 0;
  if (s == 2) return cudaErrorNotSupported;
  if (s == 0) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if ((int64_t)fa.numRegs * kPairThreads < kPairRegsNeeded) {
      if (dev >= 0 && dev < 64) state[dev] = 2;
      return cudaErrorNotSupported;
    }
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PG::SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) state[dev] = 1;
  }
  const int64_t pairs = (tiles + 1) / 2;
  const int64_t items = pairs * ny * a.num_kv_heads;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffffll - 1024) return cudaErrorInvalidValue;
  const int ctas = umma_persistent_ctas(dev, items);

  const int slot = umma_sched_slot(stream);
  kern<<<ctas, kPairThreads, PG::SMEM, stream>>>(a, maps, (int)pairs, ny, slot);
  count_launch();
  return cudaGetLastError();
}

}  // namespace kvc
