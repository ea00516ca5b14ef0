/*
 * kvcache.h — C ABI of libkvcache.so, the B200 (sm_100a) paged-KV hot path.
 *
 * This library replaces the MLX/nanobind extension `_ext` of sglang-mlx
 * (bindings.cpp, paged_attention/mlx_paged_attention.cpp,
 * paged_attention/mlx_cache.cpp, paged_attention/mlx_device.cpp).  Every
 * compute entry point takes tensors as DLPack `DLTensor` structs (restated
 * below from the public DLPack specification, layout-identical), plain scalars
 * and a CUDA stream handle.  Nothing here depends on PyTorch, MLX or Triton.
 *
 * Conventions
 *  - Return value: KVC_OK (0) or a KVC_E* code.  The message of the last
 *    failure on the calling thread is returned by kvc_last_error().  Messages of
 *    argument errors reuse the reference's `std::invalid_argument` texts so a
 *    Python shim can raise ValueError with the same wording.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  All launches
 *    are asynchronous; no entry point allocates device memory on the compute
 *    path (the caller owns `out` and any split-K workspace).
 *  - Tensors must live on a CUDA device (kDLCUDA or kDLCUDAManaged).  The
 *    launch runs on that device; the calling thread's current device is
 *    restored afterwards.
 *  - Kernels bounds-check slot ids and block ids against the cache extents and
 *    skip out-of-range entries instead of faulting; the skip is recorded in a
 *    sticky per-device status word read by kvc_get_status().
 */
#ifndef KVCACHE_H_
#define KVCACHE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- DLPack structs (DLPack v0.8+ ABI, public spec) ---------------------- */
typedef struct {
  int32_t device_type; /* 1 = CPU, 2 = CUDA, 3 = CUDA host, 13 = CUDA managed */
  int32_t device_id;
} kvc_dldevice;

typedef struct {
  uint8_t code;   /* 0 int, 1 uint, 2 float, 4 bfloat */
  uint8_t bits;
  uint16_t lanes; /* must be 1 */
} kvc_dldtype;

typedef struct {
  void* data;
  kvc_dldevice device;
  int32_t ndim;
  kvc_dldtype dtype;
  int64_t* shape;
  int64_t* strides; /* in elements; NULL = compact row-major */
  uint64_t byte_offset;
} kvc_dltensor;

/* ---- status codes --------------------------------------------------------- */
#define KVC_OK 0
#define KVC_EINVAL 1      /* bad shape / dtype / argument (reference: ValueError) */
#define KVC_ECUDA 2       /* CUDA runtime error */
#define KVC_ENOMEM 3      /* allocation failed (runtime helpers only) */
#define KVC_EUNSUPPORTED 4

/* Bits of the per-device status word (kvc_get_status). */
#define KVC_STATUS_SLOT_OOB 0x1u    /* a slot id beyond the cache was skipped */
#define KVC_STATUS_BLOCK_OOB 0x2u   /* a block-table entry beyond the cache was skipped */
#define KVC_STATUS_WAIT_TIMEOUT 0x4u /* a bounded pipeline wait gave up */
#define KVC_STATUS_INDEX_OOB 0x8u   /* a gather/copy index beyond its buffer was skipped */
#define KVC_STATUS_PREFIX_MISMATCH 0x10u /* a sequence's table did not start with the shared prefix blocks */
#define KVC_STATUS_PLAN_MISMATCH 0x20u /* a decode plan was made for other launch parameters (nothing written) */

/* ---- errors / info --------------------------------------------------------- */
/* Thread-local message of the last failing call ("" if none). */
const char* kvc_last_error(void);
/* Library version string. */
const char* kvc_version(void);
/* Reads (and optionally clears) the sticky status word of `device`.  This
 * synchronises the device. */
int kvc_get_status(int device, uint32_t* flags, int clear);

/* ---- paged attention (decode) --------------------------------------------
 * Replaces `_ext.paged_attention_v1` (bindings.cpp:44-65) and the C++ op
 * `paged_attention_v1` (paged_attention/mlx_paged_attention.cpp:150-213) with
 * its dispatch `PagedAttentionV1::eval_gpu` (mlx_paged_attention.cpp:93-144).
 *   out          [num_seqs, num_heads, head_size], dtype of query, written
 *   query        [num_seqs, num_heads, head_size]  f32 / f16 / bf16
 *   key_cache    [num_blocks, num_kv_heads, head_size/x, block_size, x], x = 16/sizeof(cache)
 *   value_cache  [num_blocks, num_kv_heads, head_size, block_size]
 *   block_tables [num_seqs, max_num_blocks_per_seq] int32 or uint32 (read as uint32)
 *   context_lens [num_seqs] int32 or uint32 (read as uint32)
 *   alibi_slopes [num_heads] f32, or NULL
 * Sequences with context_len == 0 or context_len > max_seq_len produce zeros
 * (paged_attention_kernels.metal:45-50).  Softmax denominator is
 * sum + 1e-6 (paged_attention_kernels.metal:144). */
int kvc_paged_attention_v1(kvc_dltensor* out, const kvc_dltensor* query,
                           const kvc_dltensor* key_cache, const kvc_dltensor* value_cache,
                           const kvc_dltensor* block_tables, const kvc_dltensor* context_lens,
                           int num_kv_heads, float scale, int block_size, int max_seq_len,
                           const kvc_dltensor* alibi_slopes, void* stream);

/* Split-K (partitioned) decode with a cross-partition log-sum-exp reduce.  No
 * reference counterpart: sglang-mlx defers it (README.md:11-20); the argument
 * list extends kvc_paged_attention_v1 with the caller-owned workspace
 *   max_logits [num_seqs, num_heads, max_num_partitions] f32
 *   exp_sums   [num_seqs, num_heads, max_num_partitions] f32
 *   tmp_out    [num_seqs, num_heads, max_num_partitions, head_size] f32
 * where max_num_partitions = ceil(max_seq_len / partition_size).  Results agree
 * with kvc_paged_attention_v1 within floating-point reassociation. */
int kvc_paged_attention_v2(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                           kvc_dltensor* tmp_out, const kvc_dltensor* query,
                           const kvc_dltensor* key_cache, const kvc_dltensor* value_cache,
                           const kvc_dltensor* block_tables, const kvc_dltensor* context_lens,
                           int num_kv_heads, float scale, int block_size, int max_seq_len,
                           const kvc_dltensor* alibi_slopes, int partition_size, void* stream);

/* Planned split-K decode: the same result as kvc_paged_attention_v2, for
 * batches too small to fill the GPU with one CTA per (sequence, KV head) (a
 * KV-head shard of a multi-GPU run, long contexts).  No reference counterpart
 * (split-K is deferred in sglang-mlx, README.md:11-20).
 *
 * kvc_decode_plan reads the context lengths on the device and writes a work
 * list into `plan`: every (sequence, partition) item, longest first, so the
 * GPU starts the long partitions first and ends the launch on short ones, plus
 * one arrival counter per (sequence, KV head).  Every layer of a decode step
 * has the same lengths, so one plan per step serves all of them.
 * kvc_paged_attention_planned then runs one CTA per (item, KV head); when a
 * sequence has up to 32 partitions the CTA that finishes its last partition
 * merges the partials into `out` (no separate reduce kernel) and resets the
 * counter; a sequence of one partition writes `out` directly.
 *   plan          int32/uint32 [>= kvc_decode_plan_size(...)] on the device,
 *                 written by kvc_decode_plan (nothing to initialise)
 *   workspace     exp_sums / max_logits / tmp_out of kvc_paged_attention_v2
 *   partition_size  a multiple of 32 and of block_size, at most 8192; the
 *                 same value (and num_seqs, num_kv_heads, max_seq_len) in both
 *                 calls: a decode given a plan made for other values writes
 *                 nothing and sets KVC_STATUS_PLAN_MISMATCH
 * Calls that share a plan or a workspace must not overlap on the GPU.  f32
 * queries and caches, head sizes other than 64/128 and groups above 16 query
 * heads run as kvc_paged_attention_v2 (the plan is then unused).
 * kvc_decode_plan_size returns the plan's element count, or -1 for arguments
 * a plan cannot cover (over 65535 sequences or partitions per sequence). */
int64_t kvc_decode_plan_size(int num_seqs, int num_kv_heads, int max_seq_len, int partition_size);
int kvc_decode_plan(kvc_dltensor* plan, const kvc_dltensor* context_lens, int num_kv_heads, int max_seq_len,
                    int partition_size, void* stream);
int kvc_paged_attention_planned(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                int max_seq_len, const kvc_dltensor* alibi_slopes, int partition_size,
                                kvc_dltensor* plan, void* stream);

/* A decode step's append and planned decode in one launch: the same results
 * (cache and `out`) as kvc_reshape_and_cache(key, value, key_cache,
 * value_cache, slot_mapping) followed by kvc_paged_attention_planned, for a
 * step that appends one token per sequence.  No reference counterpart (the
 * reference appends and decodes in two calls, metal_kernels.py:20-74); it
 * saves the append's launch, which a decode has to wait for.
 *   key, value    [num_seqs, num_kv_heads, head_size], the cache's dtype
 *                 (float16 / bfloat16), head_size dimension contiguous,
 *                 rows 4-byte aligned (even strides, aligned base)
 *   slot_mapping  int32/int64 [>= num_seqs]: sequence b's new token goes to
 *                 slot slot_mapping[b], which must be the slot of its last
 *                 position (context_lens[b] - 1) in block_tables[b]; a
 *                 negative slot skips the token (padding), a slot past the
 *                 cache is skipped and sets KVC_STATUS_SLOT_OOB
 * The CTA that holds a sequence's last token stores it to the cache and uses
 * the new values for that token in its own attention, without waiting for
 * the stores.  Paged float16/bfloat16 caches on the tensor-core decode only (query
 * of the cache's dtype, head size 64/128, block size 8/16/32, up to 16 query
 * heads per KV head): anything else returns KVC_EUNSUPPORTED and runs nothing. */
int kvc_paged_attention_planned_append(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                       kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key,
                                       const kvc_dltensor* value, kvc_dltensor* key_cache, kvc_dltensor* value_cache,
                                       const kvc_dltensor* slot_mapping, const kvc_dltensor* block_tables,
                                       const kvc_dltensor* context_lens, int num_kv_heads, float scale,
                                       int block_size, int max_seq_len, const kvc_dltensor* alibi_slopes,
                                       int partition_size, kvc_dltensor* plan, void* stream);

/* Paged decode over token-major caches: the reshape_and_cache_flash layout
 * [num_blocks, block_size, num_kv_heads, head_size], or the MHATokenPool
 * buffers [slots, num_kv_heads, head_size] (pool_size + 1 slots, slot 0 the
 * padding slot) with block_size 1, where a block table row is the sequence's
 * slot list.  This is the decode the reference leaves as a TODO over its pool
 * (memory_pool.py:110-112: attention straight on scattered pool slots instead
 * of the per-layer gather behind PooledKVCache.update_and_fetch,
 * memory_pool.py:206-234).  Same math and edge rules as
 * kvc_paged_attention_v1; partition_size 0 runs the single pass, otherwise
 * exp_sums / max_logits / tmp_out are the split-K workspace of
 * kvc_paged_attention_v2.  float16/bfloat16 query and caches of one dtype,
 * head_size 64 or 128, up to 16 query heads per KV head (else
 * KVC_EUNSUPPORTED); token rows must start on 16-byte boundaries. */
int kvc_paged_attention_flash(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                              kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                              const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                              const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                              int max_seq_len, const kvc_dltensor* alibi_slopes, int partition_size, void* stream);

/* Shared-prefix ("cascade") decode.  No counterpart in the reference; the
 * workload is BASELINE config 4 (a radix-cache hit shared by a whole batch,
 * radix_cache.py).  Precondition: the first shared_prefix_len / block_size
 * entries of every row of block_tables equal those of row 0 (checked on the
 * device: a sequence that breaks it sets KVC_STATUS_PREFIX_MISMATCH and its
 * output is not meaningful).  The prefix is attended once per KV head for all
 * sequences (chunks of prefix_partition_size tokens), the tokens after it by
 * split-K partitions of partition_size tokens, and a log-sum-exp reduce merges
 * them; sequences shorter than the prefix attend to their own length only.
 * Result = kvc_paged_attention_v1 on the same inputs, within floating-point
 * reassociation.  Workspace as kvc_paged_attention_v2 with
 * P = ceil(shared_prefix_len / prefix_partition_size)
 *   + ceil((max_seq_len - shared_prefix_len) / partition_size).
 * float16/bfloat16 query and cache of one dtype, head_size 64 or 128, up to 16
 * query heads per KV head, no ALiBi (else KVC_EUNSUPPORTED). */
int kvc_paged_attention_cascade(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                int max_seq_len, const kvc_dltensor* alibi_slopes, int shared_prefix_len,
                                int prefix_partition_size, int partition_size, void* stream);

/* Paged prefill / extend attention.  No kernel counterpart in the reference:
 * there a prefill stores the new K/V into the pool and gathers prefix + new
 * tokens back (PooledKVCache.update_and_fetch, memory_pool.py:205-234) for mlx
 * SDPA under the offset-causal mask of mlx-lm's create_attention_mask
 * (PooledKVCache.make_mask, memory_pool.py:240-270; model_runner.py:190-258).
 * This reads the cache in place.
 *   out, query      [num_tokens, num_heads, head_size]; the new tokens of all
 *                   sequences, sequence b's at rows qo_indptr[b] ..
 *                   qo_indptr[b + 1] - 1
 *   key_cache / value_cache  the paged layout ([nb, H, D/x, bs, x] /
 *                   [nb, H, D, bs]), the flash layout ([nb, bs, H, D]) or the
 *                   token pool ([slots, H, D], block_size 1)
 *   block_tables    [num_seqs, max_blocks] int32 (slot lists for the pool);
 *                   the new tokens' K/V are already stored
 *   qo_indptr       [num_seqs + 1] int32, non-decreasing
 *   kv_lens         [num_seqs] int32: cache tokens of sequence b including its
 *                   new ones, so its prefix is kv_lens[b] - (qo_indptr[b + 1] -
 *                   qo_indptr[b])
 *   max_q_len       at least every sequence's new-token count (sizes the grid)
 *   window_size     0: causal; w > 0: token t of the new ones sees only cache
 *                   tokens (prefix + t - w, prefix + t]
 * New token t of sequence b attends to cache tokens [0, prefix + t].  float16
 * / bfloat16 query and caches of one dtype, head_size 64 or 128, paged
 * block_size 8/16/32 (else KVC_EUNSUPPORTED).  Device-side index errors
 * (kv_lens below the new-token count or past the table, qo_indptr past
 * num_tokens or a count above max_q_len) set KVC_STATUS_INDEX_OOB. */
int kvc_paged_prefill(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                      const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                      const kvc_dltensor* qo_indptr, const kvc_dltensor* kv_lens, int num_kv_heads, float scale,
                      int block_size, int max_q_len, int window_size, void* stream);

/* Split-K decode for callers that cannot allocate device memory.  No
 * counterpart in the reference: sglang-mlx has no split-K decode at all.
 *
 * Same arguments and result as kvc_paged_attention_v2, minus the three
 * workspace tensors.  Some callers have no way to provide that workspace:
 * code that runs inside a host framework whose own pool owns all device
 * memory (a raw cudaMalloc beside it fragments or oversubscribes the pool),
 * serving loops that cannot afford cudaMalloc/cudaFree stalling the device,
 * and foreign-language bindings that carry no device allocator at all.  This
 * entry point allocates nothing: the partials live in a static device array of
 * KVC_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads the
 * library holds until the process exits.
 *   - Needs num_seqs * num_heads * ceil(max_seq_len / partition_size) *
 *     (head_size + 2) * 4 bytes <= KVC_NOALLOC_SCRATCH_BYTES; larger calls
 *     return KVC_EINVAL without launching anything.
 *   - The first call on a device looks up the array's device address (with that
 *     device current); make that first call before any stream capture (a first
 *     call made while `stream` is capturing returns KVC_EINVAL and launches
 *     nothing).  The address is remembered per device and CUDA context, so the
 *     first call after cudaDeviceReset looks it up again, with the same rule.
 *   - All calls on a device share the one array and it keeps the previous
 *     call's contents (nothing in it needs to start at zero).  Calls that overlap
 *     on the GPU — on different streams, or from different threads — race on it:
 *     serialise them (one stream, or events). */
#define KVC_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int kvc_paged_attention_v2_noalloc(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                   const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                   const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                   int max_seq_len, const kvc_dltensor* alibi_slopes, int partition_size,
                                   void* stream);

/* ---- cache ops -------------------------------------------------------------
 * Replaces `_ext.reshape_and_cache` (bindings.cpp:67-80), the C++ op
 * `reshape_and_cache` (paged_attention/mlx_cache.cpp:256-278) and
 * `ReshapeAndCache::eval_gpu` (mlx_cache.cpp:60-96).  key_cache/value_cache are
 * updated in place (the reference aliases them, mlx_cache.cpp:65-66).
 *   key, value   [num_tokens, num_kv_heads, head_size] f32 / f16 / bf16 (token stride free)
 *   slot_mapping [num_tokens] int32 or int64; slot < 0 skips the token. */
int kvc_reshape_and_cache(const kvc_dltensor* key, const kvc_dltensor* value,
                          kvc_dltensor* key_cache, kvc_dltensor* value_cache,
                          const kvc_dltensor* slot_mapping, void* stream);

/* Replaces `_ext.reshape_and_cache_flash` (bindings.cpp:82-95,
 * mlx_cache.cpp:280-300, eval mlx_cache.cpp:118-152).  Caches are
 * [num_blocks, block_size, num_kv_heads, head_size] (the MHATokenPool layout
 * (pool_size + 1, H, D) is the block_size = 1 case when passed as 3-D).  The
 * source may have any token and head strides, so MHATokenPool.store's
 * (1, H, S, D) -> (S, H, D) transpose (memory_pool.py:117-137) needs no copy. */
int kvc_reshape_and_cache_flash(const kvc_dltensor* key, const kvc_dltensor* value,
                                kvc_dltensor* key_cache, kvc_dltensor* value_cache,
                                const kvc_dltensor* slot_mapping, void* stream);

/* Slot gather behind MHATokenPool.fetch (memory_pool.py:139-159): for both K
 * and V, out[0, h, t, :] = buffer[indices[t], h, :].
 *   k_out, v_out         [1, H, T, D]  (any strides)
 *   k_buffer, v_buffer   [pool_size + 1, H, D] (or [nb, bs, H, D], slots flattened)
 *   indices              [T] int32 or int64 */
int kvc_gather_kv(kvc_dltensor* k_out, kvc_dltensor* v_out, const kvc_dltensor* k_buffer,
                  const kvc_dltensor* v_buffer, const kvc_dltensor* indices, void* stream);

/* Replaces `_ext.copy_blocks` (bindings.cpp:97-113, mlx_cache.cpp:302-346,
 * kernel copy_blocks.metal:9-44): for every layer i and every pair
 * (src, dst) of block_mapping, block dst of key_caches[i] and value_caches[i]
 * is overwritten with block src, in place.
 *   key_caches, value_caches  arrays of num_*_caches tensors, each dense with a
 *                             leading block dimension (any dtype; K and V of a
 *                             layer share dtype and elements per block)
 *   block_mapping             [num_pairs, 2] int32 / uint32 / int64, on the
 *                             caches' device or in host memory
 * Pairs run in parallel (a block both written and read by one call gives an
 * unspecified result, as on Metal).  Out-of-range block ids are skipped and
 * flagged with KVC_STATUS_INDEX_OOB. */
int kvc_copy_blocks(kvc_dltensor* key_caches, int num_key_caches, kvc_dltensor* value_caches,
                    int num_value_caches, const kvc_dltensor* block_mapping, void* stream);

/* Replaces `_ext.swap_blocks` (bindings.cpp:115-123, mlx_cache.cpp:348-370,
 * kernel copy_blocks.metal:60-75): block dst of `dst` is overwritten with block
 * src of `src` for every pair.  src and dst are dense with a leading block
 * dimension, equal dtype and elements per block; each may live on a CUDA device
 * or in host memory (kDLCPU, or pinned kDLCUDAHost for asynchronous copies).
 * Device-to-device on one GPU runs a kernel; otherwise one cudaMemcpyAsync per
 * run of consecutive pairs (out-of-range pairs are then rejected with
 * KVC_EINVAL before anything is copied). */
int kvc_swap_blocks(const kvc_dltensor* src, kvc_dltensor* dst, const kvc_dltensor* block_mapping, void* stream);

/* ---- FP8 (one-byte) KV cache ----------------------------------------------
 * The reference ships FP8 codecs (float8.metal:13-125) and an elementwise
 * converter (convert_fp8.metal:13-80) but no cache kernel stores one-byte
 * values (memory_pool.py:85, TODO(quant)).  Here the codes live in uint8
 * caches of the vLLM layout with x = 16: K [num_blocks, H, D/16, bs, 16],
 * V [num_blocks, H, D, bs]; a value is stored as encode(x / scale) and reads
 * back as decode(code) * scale, with one scale for K and one for V.
 * fp8_format 0 = E4M3 as float8.metal defines it (all-ones exponent kept for
 * Inf/NaN, largest finite 240), 1 = E5M2.  Encoding is bit-exact with the
 * reference's encoder code (float8.metal:69-118): round to nearest even in the
 * normal range (a carry past the last finite exponent gives +-Inf), gradual
 * underflow rounded half up, values past the last finite exponent sent down
 * the subnormal branch (E4M3: 256 <= |x| < 2^14 keep the low bits of that
 * shift; 300 encodes as 0) and a subnormal's carry into the smallest normal
 * dropped.  Where that code's shift count is negative (undefined in C++ and
 * MSL: E4M3 |x| >= 2^14, E5M2 |x| >= 2^16) the code is +-Inf.
 * fp8_format 2 = E4M3-sat and 3 = E5M2-sat encode with the behaviour the
 * reference's comment states instead (float8.metal:65-68): +-Inf past the
 * largest finite value and the carry kept; they decode like 0 and 1. */

/* reshape_and_cache into one-byte caches; key/value f32/f16/bf16, head_size a
 * multiple of 16, slot < 0 skips the token. */
int kvc_reshape_and_cache_fp8(const kvc_dltensor* key, const kvc_dltensor* value, kvc_dltensor* key_cache,
                              kvc_dltensor* value_cache, const kvc_dltensor* slot_mapping, float k_scale,
                              float v_scale, int fp8_format, void* stream);

/* Decode over one-byte caches: kvc_paged_attention_v1 semantics on the
 * dequantised cache (f16/bf16 query, head_size 64 or 128, block_size 8/16/32,
 * up to 16 query heads per KV head).  partition_size 0 runs the single pass,
 * otherwise exp_sums / max_logits / tmp_out are the split-K workspace of
 * kvc_paged_attention_v2.  The codes are converted to f16 in registers (exact)
 * and the products run as f16 with fp32 accumulation; k_scale scales the
 * logits and v_scale the output. */
int kvc_paged_attention_fp8(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                            kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                            const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                            const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                            int max_seq_len, const kvc_dltensor* alibi_slopes, float k_scale, float v_scale,
                            int fp8_format, int partition_size, void* stream);

/* kvc_paged_attention_fp8 as a planned split-K decode: the work list of
 * kvc_decode_plan (made for the same lengths, num_kv_heads, max_seq_len and
 * partition_size), longest items first, merge fused into the last partition of
 * each sequence; see kvc_paged_attention_planned.  No reference counterpart. */
int kvc_paged_attention_fp8_planned(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                    kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                    const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                    const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                    int max_seq_len, const kvc_dltensor* alibi_slopes, float k_scale, float v_scale,
                                    int fp8_format, int partition_size, kvc_dltensor* plan, void* stream);

/* convert_fp8_kernel (convert_fp8.metal:13-80) on dense arrays of one shape:
 * float -> uint8 quantises (encode(x / scale)), uint8 -> float dequantises
 * (decode(code) * scale), uint8 -> uint8 rescales, float -> float scales. */
int kvc_convert_fp8(kvc_dltensor* dst, const kvc_dltensor* src, float scale, int fp8_format, void* stream);

/* ---- device attributes (paged_attention/mlx_device.cpp) -------------------- */
/* mlx_device.cpp:16-20: max shared memory per block (opt-in) of `device`. */
int kvc_get_max_shared_memory_per_block_device_attribute(int device, int64_t* out);
/* mlx_device.cpp:12-14 throws on Metal; here it returns cudaDeviceGetAttribute. */
int kvc_get_device_attribute(int attribute, int device, int64_t* out);

/* ---- runtime helpers (the MLX allocator/stream roles, e.g.
 * mlx_paged_attention.cpp:99 `mx::allocator::malloc`; used by the Python
 * DeviceArray and the benches, never inside a compute entry point) ---------- */
int kvc_device_count(int* count);
int kvc_set_device(int device);
int kvc_get_device(int* device);
int kvc_malloc(void** ptr, size_t bytes);
int kvc_free(void* ptr);
int kvc_malloc_host(void** ptr, size_t bytes); /* pinned host memory */
int kvc_free_host(void* ptr);
/* kind: 0 host->host, 1 host->device, 2 device->host, 3 device->device, 4 default */
int kvc_memcpy_async(void* dst, const void* src, size_t bytes, int kind, void* stream);
int kvc_memset_async(void* dst, int value, size_t bytes, void* stream);
int kvc_stream_create(void** stream);
int kvc_stream_destroy(void* stream);
int kvc_stream_synchronize(void* stream);
int kvc_device_synchronize(void);
int kvc_event_create(void** event);
int kvc_event_destroy(void* event);
int kvc_event_record(void* event, void* stream);
/* Work queued on `stream` after this call waits for `event`'s recorded work
 * (overlapping host copies on one stream with compute on another). */
int kvc_stream_wait_event(void* stream, void* event);
int kvc_event_synchronize(void* event);
int kvc_event_elapsed_ms(void* start, void* end, float* ms);
/* Writes `bytes` of garbage over a device buffer to evict it from L2. */
int kvc_l2_flush(void* scratch, size_t bytes, void* stream);
/* CUDA graphs for launch-bound loops (a decode step is two launches per layer):
 * begin/end capture on a non-default stream, then replay the instantiated
 * graph.  Every entry point above is capturable once it has run once on the
 * device (first calls set kernel attributes).  The capture is thread-local
 * (cudaStreamCaptureModeThreadLocal). */
int kvc_stream_begin_capture(void* stream);
int kvc_stream_end_capture(void* stream, void** graph_exec);
int kvc_graph_launch(void* graph_exec, void* stream);
int kvc_graph_destroy(void* graph_exec);
/* Number of kernels this library has launched in this process. */
uint64_t kvc_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* KVCACHE_H_ */
