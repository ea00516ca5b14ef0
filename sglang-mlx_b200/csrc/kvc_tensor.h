// kvc_tensor.h — host-side view of a kvc_dltensor plus the parameter blocks the
// ABI layer hands to the kernel launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "kvcache.h"

namespace kvc {

enum class ElemType : int { F32 = 0, F16 = 1, BF16 = 2, I32 = 3, U32 = 4, I64 = 5, U8 = 6, INVALID = -1 };

inline int elem_size(ElemType t) {
  switch (t) {
    case ElemType::F32: case ElemType::I32: case ElemType::U32: return 4;
    case ElemType::F16: case ElemType::BF16: return 2;
    case ElemType::I64: return 8;
    case ElemType::U8: return 1;
    default: return 0;
  }
}

inline const char* elem_name(ElemType t) {
  switch (t) {
    case ElemType::F32: return "float32";
    case ElemType::F16: return "float16";
    case ElemType::BF16: return "bfloat16";
    case ElemType::I32: return "int32";
    case ElemType::U32: return "uint32";
    case ElemType::I64: return "int64";
    case ElemType::U8: return "uint8";
    default: return "invalid";
  }
}

struct View {
  char* data = nullptr;  // data + byte_offset
  ElemType dtype = ElemType::INVALID;
  int ndim = 0;
  int64_t shape[8] = {0};
  int64_t strides[8] = {0};  // elements
  int device = -1;
  bool on_cuda = false;  // kDLCUDA or kDLCUDAManaged
  bool on_host = false;  // kDLCPU or kDLCUDAHost (pinned)

  int64_t size(int i) const { return shape[i < 0 ? i + ndim : i]; }
  int64_t stride(int i) const { return strides[i < 0 ? i + ndim : i]; }
  int64_t numel() const {
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= shape[i];
    return n;
  }
  // True when dims [first, ndim) are dense row-major.
  bool dense_from(int first) const {
    int64_t expect = 1;
    for (int i = ndim - 1; i >= first; --i) {
      if (shape[i] != 1 && strides[i] != expect) return false;
      expect *= shape[i];
    }
    return true;
  }
};

// Parses `t` into `v`.  Returns false (and sets the error message) on a
// malformed descriptor.  `name` is used in messages.
bool parse(const kvc_dltensor* t, const char* name, View* v);

// Parameters of one decode launch (both the single-pass and split-K forms).
struct DecodeArgs {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const uint32_t* block_tables;
  const uint32_t* context_lens;
  const float* alibi;  // nullptr = off
  float* part_max;     // split-K workspace (nullptr = single pass)
  float* part_sum;
  float* part_out;
  ElemType q_type, cache_type;
  int num_seqs, num_heads, num_kv_heads, head_size, block_size;
  int max_blocks_per_seq, max_seq_len;
  int64_t num_blocks;
  int64_t q_seq_stride, q_head_stride;        // elements
  int64_t out_seq_stride, out_head_stride;    // elements
  int64_t k_block_stride, k_head_stride;      // elements
  int64_t v_block_stride, v_head_stride;      // elements
  int64_t k_tok_stride, v_tok_stride;         // token-major caches: elements between a block's tokens
  bool flash;                                 // token-major caches ([nb, bs, H, D] / [slots, H, D])
  int prefix_len, prefix_parts, prefix_part_size;  // shared-prefix decode (0 = off)
  float k_scale, v_scale;                     // one-byte (FP8) caches: value = code * scale
  int fp8_format;                             // 0 E4M3, 1 E5M2, 2 E4M3-sat, 3 E5M2-sat
  int64_t table_stride;                       // elements
  int partition_size;                         // tokens per partition (split-K)
  int num_partitions;                         // 1 = single pass
  int64_t part_seq_stride, part_head_stride;  // elements of part_max / part_sum
  int64_t part_out_seq_stride, part_out_head_stride, part_out_part_stride;
  float scale;
  // Planned split-K (kvc_paged_attention_planned): the work list of
  // kvc_decode_plan (header, items, arrival counters), or nullptr.
  uint32_t* plan;
  // kvc_paged_attention_planned_append: one new token per sequence (key/value
  // [num_seqs, H, D] of the cache's dtype) written to slot_mapping[seq] by the
  // CTA holding the sequence's last token; new_k == nullptr: no append.
  const void* new_k;
  const void* new_v;
  const void* slots;
  ElemType slot_type;
  int64_t nk_tok_stride, nk_head_stride, nv_tok_stride, nv_head_stride;  // elements
};

// Planned split-K decode: layout of the plan buffer (uint32 elements).
//   [0, kPlanHeader)                 header (kPlanMagic, num_seqs, num_kv_heads,
//                                    max_seq_len, partition_size, item count, 0, 0)
//   [kPlanHeader, + max_items)       work items, longest first: (partition << 16) | sequence
//   [.., + num_seqs * num_kv_heads)  per-(sequence, KV head) arrival counters, zero between calls
constexpr int kPlanHeader = 8;
constexpr uint32_t kPlanMagic = 0x4E4C5044u;  // "DPLN"
constexpr int kPlanMaxPartition = 8192;       // the planner's size histogram lives in shared memory
inline int64_t plan_max_items(int64_t num_seqs, int max_seq_len, int partition_size) {
  const int64_t parts = ((int64_t)max_seq_len + partition_size - 1) / partition_size;
  return num_seqs * (parts > 1 ? parts : 1);
}
inline int64_t plan_elems(int64_t num_seqs, int num_kv_heads, int max_seq_len, int partition_size) {
  return kPlanHeader + plan_max_items(num_seqs, max_seq_len, partition_size) + num_seqs * num_kv_heads;
}

// Paged prefill / extend attention (prefill.cuh).  Strides in elements.
struct PrefillArgs {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const uint32_t* block_tables;  // [num_seqs][table_stride]: block ids (slot ids for the token pool)
  const uint32_t* qo_indptr;     // [num_seqs + 1]: rows of sequence b are qo_indptr[b] .. qo_indptr[b + 1] - 1
  const uint32_t* kv_lens;       // [num_seqs]: cache tokens of sequence b, its new ones included
  int num_seqs, num_heads, num_kv_heads, block_size, window, max_q_len;
  int64_t num_tokens, num_blocks, table_len, table_stride;
  int64_t q_tok_stride, q_head_stride, out_tok_stride, out_head_stride;
  int64_t k_block_stride, k_head_stride, k_tok_stride;
  int64_t v_block_stride, v_head_stride, v_tok_stride;
  float scale;
  ElemType q_type;   // float16 / bfloat16 (the caches' type too)
  int head_size;     // 64 or 128
  bool token_major;  // [nb, bs, H, D] / [slots, H, D] caches; else the paged layout
  // Shared-prefix decode through the prefill kernel (the cascade form): rows
  // are (sequence, head) pairs of q [num_seqs][H][D], the keys are prefix chunk
  // blockIdx.y of sequence 0's table, and the results are split-K partials.
  const uint32_t* context_lens;
  int max_seq_len, prefix_len, prefix_part_size;
  float* part_max;
  float* part_sum;
  float* part_out;
  int64_t part_seq_stride, part_head_stride, part_out_seq_stride, part_out_head_stride, part_out_part_stride;
  int single_issue;  // tcgen05 kernel: the producer's lane 0 issues every copy of a tile (tuning; default: spread)
};

struct ReshapeArgs {
  const void* key;
  const void* value;
  void* key_cache;
  void* value_cache;
  const void* slots;
  ElemType kv_type, cache_type, slot_type;
  int64_t num_tokens;
  int num_heads, head_size, block_size;
  int64_t num_blocks;
  int64_t key_tok_stride, key_head_stride;      // elements
  int64_t value_tok_stride, value_head_stride;  // elements
  float k_scale, v_scale;                       // one-byte caches: code = encode(x / scale)
  int fp8_format;                               // 0 E4M3, 1 E5M2, 2 E4M3-sat, 3 E5M2-sat
  int64_t kc_block_stride, kc_head_stride;      // vLLM: [nb, H, D/x, bs, x]; flash: [nb, bs, H, D]
  int64_t vc_block_stride, vc_head_stride;
  int64_t kc_tok_stride, vc_tok_stride;         // flash layout only
};

struct GatherArgs {
  void* k_out;
  void* v_out;
  const void* k_buf;
  const void* v_buf;
  const void* indices;
  ElemType type, index_type;
  int64_t num_indices;
  int64_t num_slots;
  int num_heads, head_size;
  int64_t kb_slot_stride, kb_head_stride;
  int64_t vb_slot_stride, vb_head_stride;
  int64_t ko_tok_stride, ko_head_stride;
  int64_t vo_tok_stride, vo_head_stride;
};

cudaError_t launch_paged_decode(const DecodeArgs& a, cudaStream_t stream);
// Split-K decode with its partials in the library's static scratch array
// (kvc_paged_attention_v2_noalloc).  `a` carries no workspace pointers.
cudaError_t launch_paged_decode_noalloc(DecodeArgs a, cudaStream_t stream);
// Writes the work list of a planned split-K decode (one CTA).
cudaError_t launch_decode_plan(const uint32_t* context_lens, int num_seqs, int num_kv_heads, int max_seq_len,
                               int partition_size, uint32_t* plan, cudaStream_t stream);
// Shared-prefix decode: tail partitions, the cascade prefix kernel, the reduce.
cudaError_t launch_paged_decode_cascade(const DecodeArgs& a, cudaStream_t stream);
// Paged prefill / extend attention (prefill.cuh); enqueues one kernel.
cudaError_t launch_paged_prefill(const PrefillArgs& a, cudaStream_t stream);
// Whole-block copies (copy_blocks / swap_blocks).  A plane is one buffer
// pair; every plane of one launch has the same block size in bytes.
constexpr int kMaxBlockPlanes = 32;
struct BlockPlane {
  const void* src;
  void* dst;
  int64_t src_blocks, dst_blocks;
};
struct BlockCopyArgs {
  std::vector<BlockPlane> planes;
  int64_t block_bytes = 0;
  int64_t num_pairs = 0;
  const void* device_mapping = nullptr;  // [num_pairs, 2] on the launch device, or null
  bool mapping_i64 = false;
  std::vector<int64_t> host_mapping;     // the pairs, when device_mapping is null
};
cudaError_t launch_block_copies(const BlockCopyArgs& a, cudaStream_t stream);
cudaError_t launch_reshape_and_cache(const ReshapeArgs& a, cudaStream_t stream);
// Quantising append into one-byte caches (vLLM layout, x = 16).
cudaError_t launch_reshape_and_cache_fp8(const ReshapeArgs& a, cudaStream_t stream);
// Elementwise codec of convert_fp8.metal (U8 <-> F32/F16/BF16, U8 -> U8, float -> float).
cudaError_t launch_convert_fp8(ElemType src_type, ElemType dst_type, const void* src, void* dst, float scale,
                               int64_t n, int fmt, cudaStream_t stream);
cudaError_t launch_reshape_and_cache_flash(const ReshapeArgs& a, cudaStream_t stream);
cudaError_t launch_gather_kv(const GatherArgs& a, cudaStream_t stream);

}  // namespace kvc

// Host accessors of each translation unit's sticky status word.
unsigned int kvc_cache_ops_status(int clear, cudaError_t* err);
unsigned int kvc_decode_status(int clear, cudaError_t* err);
unsigned int kvc_block_ops_status(int clear, cudaError_t* err);
