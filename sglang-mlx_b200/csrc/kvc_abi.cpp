// kvc_abi.cpp — the extern "C" surface of libkvcache.so: argument validation
// (mirroring the reference's std::invalid_argument checks), device guards,
// dispatch to the kernel launchers, and the small runtime the Python shim uses
// in place of MLX's allocator and streams.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <cmath>
#include <string>
#include <vector>

#include "kvc_tensor.h"
#include "kvcache.h"

namespace kvc {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void set_error(const std::string& msg) { g_last_error = msg; }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

static int cuda_fail(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return fail(KVC_ECUDA, m);
}

static ElemType decode_dtype(const kvc_dldtype& d) {
  if (d.lanes != 1) return ElemType::INVALID;
  if (d.code == 2 && d.bits == 32) return ElemType::F32;
  if (d.code == 2 && d.bits == 16) return ElemType::F16;
  if (d.code == 4 && d.bits == 16) return ElemType::BF16;
  if (d.code == 0 && d.bits == 32) return ElemType::I32;
  if (d.code == 1 && d.bits == 32) return ElemType::U32;
  if (d.code == 0 && d.bits == 64) return ElemType::I64;
  if (d.code == 1 && d.bits == 8) return ElemType::U8;
  return ElemType::INVALID;
}

bool parse(const kvc_dltensor* t, const char* name, View* v) {
  if (t == nullptr) {
    set_error(std::string(name) + " is null");
    return false;
  }
  if (t->ndim < 0 || t->ndim > 8) {
    set_error(std::string(name) + ": unsupported rank " + std::to_string(t->ndim));
    return false;
  }
  v->dtype = decode_dtype(t->dtype);
  if (v->dtype == ElemType::INVALID) {
    set_error(std::string(name) + ": unsupported dtype (code " + std::to_string(t->dtype.code) +
              ", bits " + std::to_string(t->dtype.bits) + ", lanes " + std::to_string(t->dtype.lanes) + ")");
    return false;
  }
  v->ndim = t->ndim;
  int64_t expect = 1;
  for (int i = t->ndim - 1; i >= 0; --i) {
    v->shape[i] = t->shape[i];
    if (v->shape[i] < 0) {
      set_error(std::string(name) + ": negative extent");
      return false;
    }
    v->strides[i] = t->strides ? t->strides[i] : expect;
    expect *= v->shape[i];
  }
  v->data = static_cast<char*>(t->data) + t->byte_offset;
  v->on_cuda = (t->device.device_type == 2 || t->device.device_type == 13);
  v->on_host = (t->device.device_type == 1 || t->device.device_type == 3);
  v->device = t->device.device_id;
  return true;
}

// Sets the launch device from the tensors and restores the caller's device.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&prev_);
    if (device >= 0 && device != prev_) {
      ok_ = cudaSetDevice(device) == cudaSuccess;
      changed_ = true;
    }
  }
  ~DeviceGuard() {
    if (changed_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool changed_ = false;
  bool ok_ = true;
};

static bool is_valid_attention_config(int head_size, int block_size) {
  // mlx_paged_attention.cpp:52-59 (the Metal instantiation matrix).
  static const int hs[] = {32, 64, 80, 96, 112, 120, 128, 192, 256};
  static const int bs[] = {8, 16, 32};
  bool ok_hs = false, ok_bs = false;
  for (int v : hs) ok_hs |= (v == head_size);
  for (int v : bs) ok_bs |= (v == block_size);
  return ok_hs && ok_bs;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
static bool is_float(ElemType t) { return t == ElemType::F32 || t == ElemType::F16 || t == ElemType::BF16; }

// (query dtype, cache dtype) pairs of paged_attention_inst.metal:64-73 and
// (kv dtype, cache dtype) pairs of reshape_and_cache.metal:91-95.
static bool is_supported_pair(ElemType a, ElemType c) {
  if (a == c && is_float(a)) return true;
  return a == ElemType::F32 && (c == ElemType::F16 || c == ElemType::BF16);
}

static int check_all_cuda(std::initializer_list<const View*> views, int* device) {
  int dev = -1;
  for (const View* v : views) {
    if (v == nullptr) continue;
    if (!v->on_cuda) return fail(KVC_EINVAL, "all tensors must live on a CUDA device");
    if (dev < 0) dev = v->device;
    if (v->device != dev) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
  }
  *device = dev;
  return KVC_OK;
}

static int check_index_type(const View& v, const char* name, bool allow_i64) {
  if (v.dtype == ElemType::I32 || v.dtype == ElemType::U32) return KVC_OK;
  if (allow_i64 && v.dtype == ElemType::I64) return KVC_OK;
  return fail(KVC_EINVAL, std::string(name) + " must be int32 or uint32" + (allow_i64 ? " or int64" : ""));
}

// Shared validation + argument packing of the v1 and v2 decode entry points.
static int prepare_decode(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                          const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                          const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                          int max_seq_len, const kvc_dltensor* alibi_slopes, DecodeArgs* a, int* device,
                          bool fp8 = false) {
  View q, kc, vc, bt, cl, o, al;
  if (!parse(query, "query", &q) || !parse(key_cache, "key_cache", &kc) ||
      !parse(value_cache, "value_cache", &vc) || !parse(block_tables, "block_tables", &bt) ||
      !parse(context_lens, "context_lens", &cl) || !parse(out, "out", &o))
    return KVC_EINVAL;
  if (alibi_slopes && !parse(alibi_slopes, "alibi_slopes", &al)) return KVC_EINVAL;

  // mlx_paged_attention.cpp:156-188, same order and messages.
  if (q.ndim != 3) return fail(KVC_EINVAL, "query must have shape [num_seqs, num_heads, head_size]");
  if (kc.ndim != 5 || vc.ndim != 4)
    return fail(KVC_EINVAL, "key_cache/value_cache must use paged attention layouts");
  if (bt.ndim != 2 || cl.ndim != 1)
    return fail(KVC_EINVAL, "block_tables must be 2D and context_lens must be 1D");
  if (q.shape[0] != bt.shape[0] || q.shape[0] != cl.shape[0])
    return fail(KVC_EINVAL, "query, block_tables, and context_lens sequence counts differ");
  if (num_kv_heads <= 0 || q.shape[1] % num_kv_heads != 0)
    return fail(KVC_EINVAL, "num_heads must be divisible by num_kv_heads");
  if (kc.shape[1] != num_kv_heads || vc.shape[1] != num_kv_heads)
    return fail(KVC_EINVAL, "cache KV-head count does not match num_kv_heads");
  if (kc.shape[2] * kc.shape[4] != q.shape[2] || vc.shape[2] != q.shape[2])
    return fail(KVC_EINVAL, "cache head size does not match query head size");
  if (kc.shape[0] != vc.shape[0] || kc.shape[3] != block_size || vc.shape[3] != block_size)
    return fail(KVC_EINVAL, "cache block dimensions do not match block_size");
  if (alibi_slopes && (al.ndim != 1 || al.shape[0] != q.shape[1]))
    return fail(KVC_EINVAL, "alibi_slopes must have shape [num_heads]");
  if (max_seq_len <= 0) return fail(KVC_EINVAL, "max_seq_len must be positive");
  if ((int64_t)max_seq_len > bt.shape[1] * (int64_t)block_size)
    return fail(KVC_EINVAL, "max_seq_len exceeds block table capacity");
  const int head_size = (int)q.shape[2];
  if (!is_valid_attention_config(head_size, block_size))
    return fail(KVC_EINVAL, "Unsupported head_size/block_size for paged_attention");

  // Checks the Metal path leaves to kernel lookup or to luck.
  if (fp8) {
    if ((q.dtype != ElemType::F16 && q.dtype != ElemType::BF16) || kc.dtype != ElemType::U8 || vc.dtype != ElemType::U8)
      return fail(KVC_EINVAL, "paged_attention_fp8 needs a float16/bfloat16 query and uint8 caches");
  } else if (!is_float(q.dtype) || !is_float(kc.dtype) || kc.dtype != vc.dtype ||
             !is_supported_pair(q.dtype, kc.dtype))
    return fail(KVC_EINVAL, std::string("Unsupported dtype combination for paged_attention: query ") +
                                elem_name(q.dtype) + ", cache " + elem_name(kc.dtype) + "/" + elem_name(vc.dtype));
  const int x = 16 / elem_size(kc.dtype);
  if (kc.shape[4] != x)
    return fail(KVC_EINVAL, "key_cache last dimension must be x = 16 / sizeof(cache element) = " + std::to_string(x));
  if (int rc = check_index_type(bt, "block_tables", false)) return rc;
  if (int rc = check_index_type(cl, "context_lens", false)) return rc;
  if (alibi_slopes && al.dtype != ElemType::F32) return fail(KVC_EINVAL, "alibi_slopes must be float32");
  if (o.ndim != 3 || o.shape[0] != q.shape[0] || o.shape[1] != q.shape[1] || o.shape[2] != q.shape[2] ||
      o.dtype != q.dtype)
    return fail(KVC_EINVAL, "out must have the shape and dtype of query");
  if (q.stride(2) != 1 || o.stride(2) != 1) return fail(KVC_EINVAL, "query/out head_size dimension must be contiguous");
  if (!kc.dense_from(2) || !vc.dense_from(2))
    return fail(KVC_EINVAL, "key_cache/value_cache pages must be dense ([D/x, bs, x] and [D, bs])");
  if (bt.stride(1) != 1 || cl.stride(0) != 1 || (alibi_slopes && al.stride(0) != 1))
    return fail(KVC_EINVAL, "block_tables rows, context_lens and alibi_slopes must be contiguous");
  if (int rc = check_all_cuda({&q, &kc, &vc, &bt, &cl, &o, alibi_slopes ? &al : nullptr}, device)) return rc;

  memset(a, 0, sizeof(*a));
  a->out = o.data;
  a->q = q.data;
  a->k_cache = kc.data;
  a->v_cache = vc.data;
  a->block_tables = reinterpret_cast<const uint32_t*>(bt.data);
  a->context_lens = reinterpret_cast<const uint32_t*>(cl.data);
  a->alibi = alibi_slopes ? reinterpret_cast<const float*>(al.data) : nullptr;
  a->q_type = q.dtype;
  a->cache_type = kc.dtype;
  a->num_seqs = (int)q.shape[0];
  a->num_heads = (int)q.shape[1];
  a->num_kv_heads = num_kv_heads;
  a->head_size = head_size;
  a->block_size = block_size;
  a->max_blocks_per_seq = (int)bt.shape[1];
  a->max_seq_len = max_seq_len;
  a->num_blocks = kc.shape[0];
  a->q_seq_stride = q.stride(0);
  a->q_head_stride = q.stride(1);
  a->out_seq_stride = o.stride(0);
  a->out_head_stride = o.stride(1);
  a->k_block_stride = kc.stride(0);
  a->k_head_stride = kc.stride(1);
  a->v_block_stride = vc.stride(0);
  a->v_head_stride = vc.stride(1);
  a->table_stride = bt.stride(0);
  a->scale = scale;
  a->num_partitions = 1;
  a->partition_size = 0;
  a->k_scale = 1.f;
  a->v_scale = 1.f;
  return KVC_OK;
}

// block_mapping of copy_blocks / swap_blocks: [num_pairs, 2] of int32, uint32
// or int64 (mlx_cache.cpp:309-310,356-357 for the shape rule and message).
static int parse_block_mapping(const kvc_dltensor* t, View* m) {
  if (!parse(t, "block_mapping", m)) return KVC_EINVAL;
  if (m->ndim != 2 || m->shape[1] != 2) return fail(KVC_EINVAL, "block_mapping must have shape [num_pairs, 2]");
  if (m->dtype != ElemType::I32 && m->dtype != ElemType::U32 && m->dtype != ElemType::I64)
    return fail(KVC_EINVAL, "block_mapping must be int32, uint32 or int64");
  if (!m->dense_from(0)) return fail(KVC_EINVAL, "block_mapping must be contiguous");
  if (!m->on_cuda && !m->on_host) return fail(KVC_EINVAL, "block_mapping must live on a CUDA device or the host");
  return KVC_OK;
}

// The mapping's pairs as int64 on the host (a device mapping is copied back
// synchronously; only the host-memory paths need this).
static int read_block_mapping(const View& m, std::vector<int64_t>* out) {
  const int64_t n = 2 * m.shape[0];
  out->resize((size_t)n);
  std::vector<int32_t> tmp32;
  const void* src = m.data;
  if (m.on_cuda) {
    DeviceGuard g(m.device);
    if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
    const size_t bytes = (size_t)n * elem_size(m.dtype);
    if (m.dtype == ElemType::I64) {
      cudaError_t e = cudaMemcpy(out->data(), m.data, bytes, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) return cuda_fail(e, "block_mapping copy");
      return KVC_OK;
    }
    tmp32.resize((size_t)n);
    cudaError_t e = cudaMemcpy(tmp32.data(), m.data, bytes, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "block_mapping copy");
    src = tmp32.data();
  }
  for (int64_t i = 0; i < n; ++i) {
    if (m.dtype == ElemType::I64) (*out)[i] = static_cast<const int64_t*>(src)[i];
    else if (m.dtype == ElemType::U32) (*out)[i] = (int64_t) static_cast<const uint32_t*>(src)[i];
    else (*out)[i] = static_cast<const int32_t*>(src)[i];
  }
  return KVC_OK;
}

// Pairs for the kernel: a device mapping on the launch device is read by the
// kernel itself; anything else is handed over as host values.
static int attach_mapping(const View& m, int device, BlockCopyArgs* a) {
  a->num_pairs = m.shape[0];
  if (m.on_cuda && m.device == device && m.dtype != ElemType::U32) {
    a->device_mapping = m.data;
    a->mapping_i64 = m.dtype == ElemType::I64;
    return KVC_OK;
  }
  return read_block_mapping(m, &a->host_mapping);
}

// Split-K workspace of the v2-style entry points: exp_sums / max_logits
// [B, Hq, P] and tmp_out [B, Hq, P, D] (f32), P = ceil(max_seq_len / partition_size).
static int attach_splitk_workspace(kvc_dltensor* exp_sums, kvc_dltensor* max_logits, kvc_dltensor* tmp_out,
                                   int partition_size, int block_size, int max_seq_len, int device, DecodeArgs* a,
                                   int parts_override = 0) {
  if (partition_size <= 0 || partition_size % 32 != 0 || partition_size % block_size != 0)
    return fail(KVC_EINVAL, "partition_size must be a positive multiple of 32 and of block_size");
  View es, ml, to;
  if (!parse(exp_sums, "exp_sums", &es) || !parse(max_logits, "max_logits", &ml) || !parse(tmp_out, "tmp_out", &to))
    return KVC_EINVAL;
  const int parts = parts_override > 0 ? parts_override : (max_seq_len + partition_size - 1) / partition_size;
  if (es.dtype != ElemType::F32 || ml.dtype != ElemType::F32 || to.dtype != ElemType::F32)
    return fail(KVC_EINVAL, "exp_sums, max_logits and tmp_out must be float32");
  if (es.ndim != 3 || ml.ndim != 3 || to.ndim != 4 || es.shape[0] != a->num_seqs || es.shape[1] != a->num_heads ||
      es.shape[2] < parts || ml.shape[0] != a->num_seqs || ml.shape[1] != a->num_heads || ml.shape[2] < parts ||
      to.shape[0] != a->num_seqs || to.shape[1] != a->num_heads || to.shape[2] < parts || to.shape[3] != a->head_size)
    return fail(KVC_EINVAL,
                "split-K workspace must be exp_sums/max_logits [num_seqs, num_heads, P] and tmp_out "
                "[num_seqs, num_heads, P, head_size] with P >= " +
                    std::string(parts_override > 0 ? "the partition count " : "ceil(max_seq_len / partition_size) = ") +
                    std::to_string(parts));
  if (es.stride(2) != 1 || ml.stride(2) != 1 || to.stride(3) != 1 || es.stride(0) != ml.stride(0) ||
      es.stride(1) != ml.stride(1))
    return fail(KVC_EINVAL, "exp_sums and max_logits must share strides with a contiguous last dimension");
  int dev2 = -1;
  if (int rc = check_all_cuda({&es, &ml, &to}, &dev2)) return rc;
  if (dev2 != device) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
  a->part_sum = reinterpret_cast<float*>(es.data);
  a->part_max = reinterpret_cast<float*>(ml.data);
  a->part_out = reinterpret_cast<float*>(to.data);
  a->part_seq_stride = es.stride(0);
  a->part_head_stride = es.stride(1);
  a->part_out_seq_stride = to.stride(0);
  a->part_out_head_stride = to.stride(1);
  a->part_out_part_stride = to.stride(2);
  a->partition_size = partition_size;
  a->num_partitions = parts;
  return KVC_OK;
}

// Validation + packing of the token-major decode (kvc_paged_attention_flash).
// Caches are [num_blocks, block_size, num_kv_heads, head_size] (the
// reshape_and_cache_flash layout) or [slots, num_kv_heads, head_size] with
// block_size 1 (the MHATokenPool buffers); every token row is dense.
static int prepare_flash(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                         const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                         const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                         int max_seq_len, const kvc_dltensor* alibi_slopes, DecodeArgs* a, int* device) {
  View q, kc, vc, bt, cl, o, al;
  if (!parse(query, "query", &q) || !parse(key_cache, "key_cache", &kc) ||
      !parse(value_cache, "value_cache", &vc) || !parse(block_tables, "block_tables", &bt) ||
      !parse(context_lens, "context_lens", &cl) || !parse(out, "out", &o))
    return KVC_EINVAL;
  if (alibi_slopes && !parse(alibi_slopes, "alibi_slopes", &al)) return KVC_EINVAL;
  if (q.ndim != 3) return fail(KVC_EINVAL, "query must have shape [num_seqs, num_heads, head_size]");
  const bool pool = kc.ndim == 3;
  if (!((kc.ndim == 4 || kc.ndim == 3) && vc.ndim == kc.ndim))
    return fail(KVC_EINVAL, "key_cache/value_cache must be [num_blocks, block_size, num_kv_heads, head_size] "
                            "or [slots, num_kv_heads, head_size]");
  if (bt.ndim != 2 || cl.ndim != 1) return fail(KVC_EINVAL, "block_tables must be 2D and context_lens must be 1D");
  if (q.shape[0] != bt.shape[0] || q.shape[0] != cl.shape[0])
    return fail(KVC_EINVAL, "query, block_tables, and context_lens sequence counts differ");
  if (num_kv_heads <= 0 || q.shape[1] % num_kv_heads != 0)
    return fail(KVC_EINVAL, "num_heads must be divisible by num_kv_heads");
  const int hd = pool ? 1 : 2;  // head dimension of the cache
  if (kc.shape[hd] != num_kv_heads || vc.shape[hd] != num_kv_heads)
    return fail(KVC_EINVAL, "cache KV-head count does not match num_kv_heads");
  if (kc.shape[hd + 1] != q.shape[2] || vc.shape[hd + 1] != q.shape[2])
    return fail(KVC_EINVAL, "cache head size does not match query head size");
  const int64_t cache_bs = pool ? 1 : kc.shape[1];
  if (kc.shape[0] != vc.shape[0] || (!pool && vc.shape[1] != cache_bs) || block_size != cache_bs)
    return fail(KVC_EINVAL, "cache block dimensions do not match block_size");
  if (alibi_slopes && (al.ndim != 1 || al.shape[0] != q.shape[1]))
    return fail(KVC_EINVAL, "alibi_slopes must have shape [num_heads]");
  if (max_seq_len <= 0) return fail(KVC_EINVAL, "max_seq_len must be positive");
  if ((int64_t)max_seq_len > bt.shape[1] * (int64_t)block_size)
    return fail(KVC_EINVAL, "max_seq_len exceeds block table capacity");
  const int head_size = (int)q.shape[2];
  if (!(q.dtype == ElemType::F16 || q.dtype == ElemType::BF16) || kc.dtype != q.dtype || vc.dtype != q.dtype ||
      !(head_size == 64 || head_size == 128) || q.shape[1] / num_kv_heads > 16)
    return fail(KVC_EUNSUPPORTED,
                std::string("paged_attention_flash supports float16/bfloat16 query and caches of one dtype, "
                            "head_size 64 or 128 and up to 16 query heads per KV head (got query ") +
                    elem_name(q.dtype) + ", cache " + elem_name(kc.dtype) + ", head_size " +
                    std::to_string(head_size) + ")");
  if (int rc = check_index_type(bt, "block_tables", false)) return rc;
  if (int rc = check_index_type(cl, "context_lens", false)) return rc;
  if (alibi_slopes && al.dtype != ElemType::F32) return fail(KVC_EINVAL, "alibi_slopes must be float32");
  if (o.ndim != 3 || o.shape[0] != q.shape[0] || o.shape[1] != q.shape[1] || o.shape[2] != q.shape[2] ||
      o.dtype != q.dtype)
    return fail(KVC_EINVAL, "out must have the shape and dtype of query");
  if (q.stride(2) != 1 || o.stride(2) != 1) return fail(KVC_EINVAL, "query/out head_size dimension must be contiguous");
  if (kc.stride(-1) != 1 || vc.stride(-1) != 1)
    return fail(KVC_EINVAL, "key_cache/value_cache rows (head_size) must be contiguous");
  if (bt.stride(1) != 1 || cl.stride(0) != 1 || (alibi_slopes && al.stride(0) != 1))
    return fail(KVC_EINVAL, "block_tables rows, context_lens and alibi_slopes must be contiguous");
  if (int rc = check_all_cuda({&q, &kc, &vc, &bt, &cl, &o, alibi_slopes ? &al : nullptr}, device)) return rc;

  memset(a, 0, sizeof(*a));
  a->out = o.data;
  a->q = q.data;
  a->k_cache = kc.data;
  a->v_cache = vc.data;
  a->block_tables = reinterpret_cast<const uint32_t*>(bt.data);
  a->context_lens = reinterpret_cast<const uint32_t*>(cl.data);
  a->alibi = alibi_slopes ? reinterpret_cast<const float*>(al.data) : nullptr;
  a->q_type = q.dtype;
  a->cache_type = kc.dtype;
  a->num_seqs = (int)q.shape[0];
  a->num_heads = (int)q.shape[1];
  a->num_kv_heads = num_kv_heads;
  a->head_size = head_size;
  a->block_size = block_size;
  a->max_blocks_per_seq = (int)bt.shape[1];
  a->max_seq_len = max_seq_len;
  a->num_blocks = kc.shape[0];
  a->q_seq_stride = q.stride(0);
  a->q_head_stride = q.stride(1);
  a->out_seq_stride = o.stride(0);
  a->out_head_stride = o.stride(1);
  a->k_block_stride = kc.stride(0);
  a->v_block_stride = vc.stride(0);
  a->k_tok_stride = pool ? 0 : kc.stride(1);
  a->v_tok_stride = pool ? 0 : vc.stride(1);
  a->k_head_stride = kc.stride(hd);
  a->v_head_stride = vc.stride(hd);
  a->flash = true;
  a->table_stride = bt.stride(0);
  a->scale = scale;
  a->num_partitions = 1;
  a->partition_size = 0;
  a->k_scale = 1.f;
  a->v_scale = 1.f;
  return KVC_OK;
}

}  // namespace kvc

using namespace kvc;

extern "C" {

const char* kvc_last_error(void) { return g_last_error.c_str(); }

const char* kvc_version(void) { return "libkvcache 0.1.0 (sm_100a)"; }

uint64_t kvc_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int kvc_get_status(int device, uint32_t* flags, int clear) {
  if (!flags) return fail(KVC_EINVAL, "flags is null");
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e1 = cudaSuccess, e2 = cudaSuccess;
  cudaError_t e3 = cudaSuccess;
  unsigned int f =
      kvc_cache_ops_status(clear, &e1) | kvc_decode_status(clear, &e2) | kvc_block_ops_status(clear, &e3);
  if (e1 != cudaSuccess) return cuda_fail(e1, "kvc_get_status");
  if (e2 != cudaSuccess) return cuda_fail(e2, "kvc_get_status");
  if (e3 != cudaSuccess) return cuda_fail(e3, "kvc_get_status");
  *flags = f;
  return KVC_OK;
}

int kvc_paged_attention_v1(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                           const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                           const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                           int max_seq_len, const kvc_dltensor* alibi_slopes, void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_v1 launch");
  return KVC_OK;
}

int kvc_paged_attention_v2(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits, kvc_dltensor* tmp_out,
                           const kvc_dltensor* query, const kvc_dltensor* key_cache, const kvc_dltensor* value_cache,
                           const kvc_dltensor* block_tables, const kvc_dltensor* context_lens, int num_kv_heads,
                           float scale, int block_size, int max_seq_len, const kvc_dltensor* alibi_slopes,
                           int partition_size, void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                       device, &a))
    return rc;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_v2 launch");
  return KVC_OK;
}

// ---- planned split-K (work list longest first, merge fused into the last partition) ----

static int check_plan_args(int num_seqs, int num_kv_heads, int max_seq_len, int partition_size) {
  if (num_seqs < 0 || num_seqs > 65535) return fail(KVC_EINVAL, "a decode plan covers at most 65535 sequences");
  if (num_kv_heads <= 0) return fail(KVC_EINVAL, "num_kv_heads must be positive");
  if (max_seq_len <= 0) return fail(KVC_EINVAL, "max_seq_len must be positive");
  if (partition_size <= 0 || partition_size % 32 != 0 || partition_size > kPlanMaxPartition)
    return fail(KVC_EINVAL, "partition_size of a decode plan must be a positive multiple of 32, at most " +
                                std::to_string(kPlanMaxPartition));
  if ((max_seq_len + partition_size - 1) / partition_size > 65535)
    return fail(KVC_EINVAL, "a decode plan holds at most 65535 partitions per sequence");
  return KVC_OK;
}

// The plan tensor: 1-D int32/uint32, contiguous, on `device` (or any CUDA device
// when *device < 0), at least kvc_decode_plan_size elements.
static int parse_plan(kvc_dltensor* plan, int num_seqs, int num_kv_heads, int max_seq_len, int partition_size,
                      int* device, uint32_t** data) {
  View pl;
  if (!parse(plan, "plan", &pl)) return KVC_EINVAL;
  if (int rc = check_index_type(pl, "plan", false)) return rc;
  if (pl.ndim != 1 || pl.stride(0) != 1) return fail(KVC_EINVAL, "plan must be a contiguous 1-D array");
  const int64_t need = plan_elems(num_seqs, num_kv_heads, max_seq_len, partition_size);
  if (pl.shape[0] < need)
    return fail(KVC_EINVAL, "plan holds " + std::to_string(pl.shape[0]) + " elements; this decode needs " +
                                std::to_string(need) + " (kvc_decode_plan_size)");
  int dev = -1;
  if (int rc = check_all_cuda({&pl}, &dev)) return rc;
  if (*device >= 0 && dev != *device) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
  *device = dev;
  *data = reinterpret_cast<uint32_t*>(pl.data);
  return KVC_OK;
}

int64_t kvc_decode_plan_size(int num_seqs, int num_kv_heads, int max_seq_len, int partition_size) {
  if (check_plan_args(num_seqs, num_kv_heads, max_seq_len, partition_size) != KVC_OK) return -1;
  return plan_elems(num_seqs, num_kv_heads, max_seq_len, partition_size);
}

int kvc_decode_plan(kvc_dltensor* plan, const kvc_dltensor* context_lens, int num_kv_heads, int max_seq_len,
                    int partition_size, void* stream) {
  View cl;
  if (!parse(context_lens, "context_lens", &cl)) return KVC_EINVAL;
  if (cl.ndim != 1 || cl.stride(0) != 1) return fail(KVC_EINVAL, "context_lens must be a contiguous 1-D array");
  if (int rc = check_index_type(cl, "context_lens", false)) return rc;
  if (cl.shape[0] > 65535) return fail(KVC_EINVAL, "a decode plan covers at most 65535 sequences");
  const int num_seqs = (int)cl.shape[0];
  if (int rc = check_plan_args(num_seqs, num_kv_heads, max_seq_len, partition_size)) return rc;
  int device = -1;
  if (int rc = check_all_cuda({&cl}, &device)) return rc;
  uint32_t* data = nullptr;
  if (int rc = parse_plan(plan, num_seqs, num_kv_heads, max_seq_len, partition_size, &device, &data)) return rc;
  if (num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_decode_plan(reinterpret_cast<const uint32_t*>(cl.data), num_seqs, num_kv_heads, max_seq_len,
                                     partition_size, data, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode_plan launch");
  return KVC_OK;
}

int kvc_paged_attention_planned(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                int max_seq_len, const kvc_dltensor* alibi_slopes, int partition_size,
                                kvc_dltensor* plan, void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                       device, &a))
    return rc;
  if (int rc = check_plan_args(a.num_seqs, num_kv_heads, max_seq_len, partition_size)) return rc;
  if (int rc = parse_plan(plan, a.num_seqs, num_kv_heads, max_seq_len, partition_size, &device, &a.plan)) return rc;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_planned launch");
  return KVC_OK;
}

int kvc_paged_attention_flash(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                              kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                              const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                              const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                              int max_seq_len, const kvc_dltensor* alibi_slopes, int partition_size, void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_flash(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                             block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (partition_size != 0) {
    if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                         device, &a))
      return rc;
  }
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorMisalignedAddress)
    return fail(KVC_EINVAL, "key_cache/value_cache rows, blocks and heads must start on 16-byte boundaries");
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_flash launch");
  return KVC_OK;
}

int kvc_paged_attention_cascade(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                int max_seq_len, const kvc_dltensor* alibi_slopes, int shared_prefix_len,
                                int prefix_partition_size, int partition_size, void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (alibi_slopes) return fail(KVC_EUNSUPPORTED, "paged_attention_cascade does not take alibi_slopes");
  const int G = a.num_heads / a.num_kv_heads;
  if (a.q_type != a.cache_type || (a.q_type != ElemType::F16 && a.q_type != ElemType::BF16) ||
      !(a.head_size == 64 || a.head_size == 128) || G > 16)
    return fail(KVC_EUNSUPPORTED, "paged_attention_cascade supports float16/bfloat16 query and cache of one dtype, "
                                  "head_size 64 or 128 and up to 16 query heads per KV head");
  if (shared_prefix_len <= 0 || shared_prefix_len % block_size != 0 || shared_prefix_len > max_seq_len)
    return fail(KVC_EINVAL, "shared_prefix_len must be a positive multiple of block_size, at most max_seq_len");
  if (prefix_partition_size <= 0 || prefix_partition_size % 32 != 0 || prefix_partition_size % block_size != 0)
    return fail(KVC_EINVAL, "prefix_partition_size must be a positive multiple of 32 and of block_size");
  const int prefix_parts = (shared_prefix_len + prefix_partition_size - 1) / prefix_partition_size;
  const int tail_parts = partition_size > 0 && max_seq_len > shared_prefix_len
                             ? (max_seq_len - shared_prefix_len + partition_size - 1) / partition_size
                             : 0;
  if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                       device, &a, prefix_parts + tail_parts))
    return rc;
  a.prefix_len = shared_prefix_len;
  a.prefix_parts = prefix_parts;
  a.prefix_part_size = prefix_partition_size;
  a.num_partitions = prefix_parts + tail_parts;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode_cascade(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorMisalignedAddress)
    return fail(KVC_EINVAL, "key_cache/value_cache pages must start on 16-byte boundaries");
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_cascade launch");
  return KVC_OK;
}

// Paged prefill / extend attention: the new tokens of each sequence attend to
// its cache (prefix + themselves) under the offset-causal rule of mlx-lm's
// create_attention_mask (memory_pool.py:240-270), reading the cache in place
// instead of the update_and_fetch gather + SDPA of the reference
// (memory_pool.py:205-234, model_runner.py:190-258).
int kvc_paged_prefill(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                      const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                      const kvc_dltensor* qo_indptr, const kvc_dltensor* kv_lens, int num_kv_heads, float scale,
                      int block_size, int max_q_len, int window_size, void* stream) {
  View q, kc, vc, bt, qi, kl, o;
  if (!parse(query, "query", &q) || !parse(key_cache, "key_cache", &kc) ||
      !parse(value_cache, "value_cache", &vc) || !parse(block_tables, "block_tables", &bt) ||
      !parse(qo_indptr, "qo_indptr", &qi) || !parse(kv_lens, "kv_lens", &kl) || !parse(out, "out", &o))
    return KVC_EINVAL;
  if (q.ndim != 3) return fail(KVC_EINVAL, "query must have shape [num_tokens, num_heads, head_size]");
  const bool paged = kc.ndim == 5 && vc.ndim == 4;
  const bool flash = kc.ndim == 4 && vc.ndim == 4;
  const bool pool = kc.ndim == 3 && vc.ndim == 3;
  if (!paged && !flash && !pool)
    return fail(KVC_EINVAL, "key_cache/value_cache must be [num_blocks, num_kv_heads, head_size/x, block_size, x] / "
                            "[num_blocks, num_kv_heads, head_size, block_size], [num_blocks, block_size, "
                            "num_kv_heads, head_size] or [slots, num_kv_heads, head_size]");
  if (bt.ndim != 2 || qi.ndim != 1 || kl.ndim != 1)
    return fail(KVC_EINVAL, "block_tables must be 2D, qo_indptr and kv_lens 1D");
  if (qi.shape[0] != bt.shape[0] + 1 || kl.shape[0] != bt.shape[0])
    return fail(KVC_EINVAL, "qo_indptr must have num_seqs + 1 entries and kv_lens num_seqs");
  if (num_kv_heads <= 0 || q.shape[1] % num_kv_heads != 0)
    return fail(KVC_EINVAL, "num_heads must be divisible by num_kv_heads");
  const int hd = paged ? 1 : (flash ? 2 : 1);  // KV-head dimension of the caches
  if (kc.shape[hd] != num_kv_heads || vc.shape[hd] != num_kv_heads)
    return fail(KVC_EINVAL, "cache KV-head count does not match num_kv_heads");
  const int64_t D = q.shape[2];
  if ((paged && (kc.shape[2] * kc.shape[4] != D || vc.shape[2] != D)) ||
      (!paged && (kc.shape[hd + 1] != D || vc.shape[hd + 1] != D)))
    return fail(KVC_EINVAL, "cache head size does not match query head size");
  const int64_t cache_bs = paged ? kc.shape[3] : (flash ? kc.shape[1] : 1);
  if (kc.shape[0] != vc.shape[0] || block_size != cache_bs || (paged && vc.shape[3] != cache_bs) ||
      (flash && vc.shape[1] != cache_bs))
    return fail(KVC_EINVAL, "cache block dimensions do not match block_size");
  if (max_q_len < 0 || window_size < 0) return fail(KVC_EINVAL, "max_q_len and window_size must be non-negative");
  if (!(q.dtype == ElemType::F16 || q.dtype == ElemType::BF16) || kc.dtype != q.dtype || vc.dtype != q.dtype ||
      !(D == 64 || D == 128) || (paged && !(block_size == 8 || block_size == 16 || block_size == 32)))
    return fail(KVC_EUNSUPPORTED,
                std::string("paged_prefill supports float16/bfloat16 query and caches of one dtype, head_size 64 or "
                            "128 and (paged layout) block_size 8, 16 or 32 (got query ") +
                    elem_name(q.dtype) + ", cache " + elem_name(kc.dtype) + ", head_size " + std::to_string(D) +
                    ", block_size " + std::to_string(block_size) + ")");
  if (paged && kc.shape[4] != 16 / elem_size(kc.dtype))
    return fail(KVC_EINVAL, "key_cache last dimension must be x = 16 / sizeof(cache element)");
  if (int rc = check_index_type(bt, "block_tables", false)) return rc;
  if (int rc = check_index_type(qi, "qo_indptr", false)) return rc;
  if (int rc = check_index_type(kl, "kv_lens", false)) return rc;
  if (o.ndim != 3 || o.shape[0] != q.shape[0] || o.shape[1] != q.shape[1] || o.shape[2] != D || o.dtype != q.dtype)
    return fail(KVC_EINVAL, "out must have the shape and dtype of query");
  if (q.stride(2) != 1 || o.stride(2) != 1) return fail(KVC_EINVAL, "query/out head_size dimension must be contiguous");
  if ((q.stride(0) | q.stride(1) | o.stride(0) | o.stride(1)) & 1 || !aligned4(q.data) || !aligned4(o.data))
    return fail(KVC_EINVAL, "query/out rows must start on 4-byte boundaries");
  if (paged ? (!kc.dense_from(2) || !vc.dense_from(2)) : (kc.stride(-1) != 1 || vc.stride(-1) != 1))
    return fail(KVC_EINVAL, "key_cache/value_cache pages (paged layout) or rows must be contiguous");
  if (bt.stride(1) != 1 || qi.stride(0) != 1 || kl.stride(0) != 1)
    return fail(KVC_EINVAL, "block_tables rows, qo_indptr and kv_lens must be contiguous");
  const int64_t cs = elem_size(kc.dtype);
  const int64_t k_tok = paged || pool ? 0 : kc.stride(1), v_tok = paged || pool ? 0 : vc.stride(1);
  if (!aligned16(kc.data) || !aligned16(vc.data) || (kc.stride(0) * cs) % 16 || (vc.stride(0) * cs) % 16 ||
      (kc.stride(hd) * cs) % 16 || (vc.stride(hd) * cs) % 16 || (k_tok * cs) % 16 || (v_tok * cs) % 16)
    return fail(KVC_EINVAL, "key_cache/value_cache pages and rows must start on 16-byte boundaries");
  int device_of_call = -1;
  if (int rc = check_all_cuda({&q, &kc, &vc, &bt, &qi, &kl, &o}, &device_of_call)) return rc;
  PrefillArgs a;
  memset(&a, 0, sizeof(a));
  a.out = o.data;
  a.q = q.data;
  a.k_cache = kc.data;
  a.v_cache = vc.data;
  a.block_tables = reinterpret_cast<const uint32_t*>(bt.data);
  a.qo_indptr = reinterpret_cast<const uint32_t*>(qi.data);
  a.kv_lens = reinterpret_cast<const uint32_t*>(kl.data);
  a.num_seqs = (int)bt.shape[0];
  a.num_heads = (int)q.shape[1];
  a.num_kv_heads = num_kv_heads;
  a.block_size = block_size;
  a.window = window_size;
  a.max_q_len = max_q_len;
  a.num_tokens = q.shape[0];
  a.num_blocks = kc.shape[0];
  a.table_len = bt.shape[1];
  a.table_stride = bt.stride(0);
  a.q_tok_stride = q.stride(0);
  a.q_head_stride = q.stride(1);
  a.out_tok_stride = o.stride(0);
  a.out_head_stride = o.stride(1);
  a.k_block_stride = kc.stride(0);
  a.k_head_stride = kc.stride(hd);
  a.k_tok_stride = k_tok;
  a.v_block_stride = vc.stride(0);
  a.v_head_stride = vc.stride(hd);
  a.v_tok_stride = v_tok;
  a.scale = scale;
  a.q_type = q.dtype;
  a.head_size = (int)D;
  a.token_major = !paged;
  if (a.num_seqs == 0 || a.num_tokens == 0 || max_q_len == 0) return KVC_OK;
  if (a.num_seqs > 65535) return fail(KVC_EINVAL, "at most 65535 sequences per call");
  DeviceGuard g(device_of_call);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_prefill(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged_prefill launch");
  return KVC_OK;
}

// Split-K decode whose partials live in the library's static scratch array, for
// callers that cannot allocate device memory (see include/kvcache.h).
int kvc_paged_attention_v2_noalloc(kvc_dltensor* out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                   const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                   const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                   int max_seq_len, const kvc_dltensor* alibi_slopes, int partition_size,
                                   void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (partition_size <= 0 || partition_size % 32 != 0 || partition_size % block_size != 0)
    return fail(KVC_EINVAL, "partition_size must be a positive multiple of 32 and of block_size");
  const int parts = (max_seq_len + partition_size - 1) / partition_size;
  const int64_t need = (int64_t)a.num_seqs * a.num_heads * parts * (a.head_size + 2) * (int64_t)sizeof(float);
  if (need > (int64_t)KVC_NOALLOC_SCRATCH_BYTES)
    return fail(KVC_EINVAL, "paged_attention_v2_noalloc needs " + std::to_string(need) +
                                " bytes of split-K partials, more than its static scratch of " +
                                std::to_string((size_t)KVC_NOALLOC_SCRATCH_BYTES) +
                                " bytes; use kvc_paged_attention_v2 with caller-owned workspace");
  if (a.num_seqs == 0) return KVC_OK;
  a.partition_size = partition_size;
  a.num_partitions = parts;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode_noalloc(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorStreamCaptureUnsupported)
    return fail(KVC_EINVAL, "paged_attention_v2_noalloc: the first call on a device (and the first after "
                            "cudaDeviceReset) looks up the static scratch and must run outside stream capture; "
                            "call it once eagerly before capturing");
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_v2_noalloc launch");
  return KVC_OK;
}

// ---- copy_blocks / swap_blocks (copy_blocks.metal:9-88, mlx_cache.cpp:302-370) ----

int kvc_copy_blocks(kvc_dltensor* key_caches, int num_key_caches, kvc_dltensor* value_caches,
                    int num_value_caches, const kvc_dltensor* block_mapping, void* stream) {
  if (num_key_caches != num_value_caches) return fail(KVC_EINVAL, "key_caches and value_caches size mismatch");
  View m;
  if (int rc = parse_block_mapping(block_mapping, &m)) return rc;
  if (num_key_caches < 0) return fail(KVC_EINVAL, "key_caches and value_caches size mismatch");
  if (num_key_caches > 0 && (key_caches == nullptr || value_caches == nullptr))
    return fail(KVC_EINVAL, "key_caches/value_caches is null");
  // Layers with equal block sizes share launches.
  std::vector<BlockCopyArgs> groups;
  int device = -1;
  for (int i = 0; i < num_key_caches; ++i) {
    View kc, vc;
    const std::string kn = "key_caches[" + std::to_string(i) + "]", vn = "value_caches[" + std::to_string(i) + "]";
    if (!parse(&key_caches[i], kn.c_str(), &kc) || !parse(&value_caches[i], vn.c_str(), &vc)) return KVC_EINVAL;
    if (kc.ndim == 0 || vc.ndim == 0 || kc.shape[0] == 0 || vc.shape[0] == 0 || kc.shape[0] != vc.shape[0])
      return fail(KVC_EINVAL, "key/value caches must have matching block counts");
    if (kc.dtype != vc.dtype || kc.numel() / kc.shape[0] != vc.numel() / vc.shape[0])
      return fail(KVC_EINVAL, "key/value cache block layouts must match");
    if (!kc.dense_from(0) || !vc.dense_from(0)) return fail(KVC_EINVAL, "key/value caches must be contiguous");
    int layer_dev = -1;
    if (int rc = check_all_cuda({&kc, &vc}, &layer_dev)) return rc;
    if (device >= 0 && layer_dev != device) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
    device = layer_dev;
    const int64_t bb = kc.numel() / kc.shape[0] * elem_size(kc.dtype);
    BlockCopyArgs* g = nullptr;
    for (auto& x : groups)
      if (x.block_bytes == bb) g = &x;
    if (!g) {
      groups.emplace_back();
      g = &groups.back();
      g->block_bytes = bb;
    }
    g->planes.push_back({kc.data, kc.data, kc.shape[0], kc.shape[0]});
    g->planes.push_back({vc.data, vc.data, vc.shape[0], vc.shape[0]});
  }
  if (groups.empty() || m.shape[0] == 0) return KVC_OK;
  if (m.on_cuda && m.device != device) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
  for (auto& g : groups)
    if (int rc = attach_mapping(m, device, &g)) return rc;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  for (auto& g : groups) {
    cudaError_t e = launch_block_copies(g, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "copy_blocks launch");
  }
  return KVC_OK;
}

int kvc_swap_blocks(const kvc_dltensor* src, kvc_dltensor* dst, const kvc_dltensor* block_mapping, void* stream) {
  View s, d;
  if (!parse(src, "src", &s) || !parse(dst, "dst", &d)) return KVC_EINVAL;
  if (s.ndim == 0 || d.ndim == 0 || s.shape[0] == 0 || d.shape[0] == 0)
    return fail(KVC_EINVAL, "src and dst must have a leading block dimension");
  if (s.dtype != d.dtype || s.numel() / s.shape[0] != d.numel() / d.shape[0])
    return fail(KVC_EINVAL, "src and dst block layouts must match");
  View m;
  if (int rc = parse_block_mapping(block_mapping, &m)) return rc;
  if (!s.dense_from(0) || !d.dense_from(0)) return fail(KVC_EINVAL, "src and dst must be contiguous");
  if ((!s.on_cuda && !s.on_host) || (!d.on_cuda && !d.on_host))
    return fail(KVC_EINVAL, "src and dst must live on a CUDA device or in host memory");
  if (m.shape[0] == 0) return KVC_OK;
  const int64_t bb = s.numel() / s.shape[0] * elem_size(s.dtype);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (s.on_cuda && d.on_cuda && s.device == d.device) {
    BlockCopyArgs a;
    a.block_bytes = bb;
    a.planes.push_back({s.data, d.data, s.shape[0], d.shape[0]});
    if (m.on_cuda && m.device != s.device) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
    if (int rc = attach_mapping(m, s.device, &a)) return rc;
    DeviceGuard guard(s.device);
    if (!guard.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
    cudaError_t e = launch_block_copies(a, st);
    if (e != cudaSuccess) return cuda_fail(e, "swap_blocks launch");
    return KVC_OK;
  }
  // Host memory on either side (or two devices): one cudaMemcpyAsync per run
  // of consecutive pairs, on the stream's device.
  std::vector<int64_t> pairs;
  if (int rc = read_block_mapping(m, &pairs)) return rc;
  const int64_t n = m.shape[0];
  for (int64_t i = 0; i < n; ++i) {
    if (pairs[2 * i] < 0 || pairs[2 * i] >= s.shape[0] || pairs[2 * i + 1] < 0 || pairs[2 * i + 1] >= d.shape[0])
      return fail(KVC_EINVAL, "block_mapping entry " + std::to_string(i) + " is out of range");
  }
  DeviceGuard guard(s.on_cuda ? s.device : (d.on_cuda ? d.device : -1));
  if (!guard.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  for (int64_t i = 0; i < n;) {
    int64_t run = 1;
    while (i + run < n && pairs[2 * (i + run)] == pairs[2 * i] + run && pairs[2 * (i + run) + 1] == pairs[2 * i + 1] + run)
      ++run;
    cudaError_t e = cudaMemcpyAsync(d.data + pairs[2 * i + 1] * bb, s.data + pairs[2 * i] * bb, (size_t)(run * bb),
                                    cudaMemcpyDefault, st);
    if (e != cudaSuccess) return cuda_fail(e, "swap_blocks copy");
    i += run;
  }
  return KVC_OK;
}

// Shared validation of the two append layouts.
static int prepare_reshape(const kvc_dltensor* key, const kvc_dltensor* value, kvc_dltensor* key_cache,
                           kvc_dltensor* value_cache, const kvc_dltensor* slot_mapping, bool flash,
                           ReshapeArgs* a, int* device, bool fp8 = false) {
  View k, v, kc, vc, sm;
  if (!parse(key, "key", &k) || !parse(value, "value", &v) || !parse(key_cache, "key_cache", &kc) ||
      !parse(value_cache, "value_cache", &vc) || !parse(slot_mapping, "slot_mapping", &sm))
    return KVC_EINVAL;
  if (k.ndim != 3 || v.ndim != 3 || k.shape[0] != v.shape[0] || k.shape[1] != v.shape[1] || k.shape[2] != v.shape[2])
    return fail(KVC_EINVAL, "key and value must both have shape [num_tokens, num_heads, head_size]");
  // The Metal kernel reads slot_mapping[token] for token < key.shape(0), so a
  // longer mapping is accepted and its tail ignored (the reference test
  // fixture relies on this, test_paged_attention_kernel.py:171-177).
  if (sm.ndim != 1 || sm.shape[0] < k.shape[0])
    return fail(KVC_EINVAL, "slot_mapping must have shape [num_tokens]");
  if (int rc = check_index_type(sm, "slot_mapping", true)) return rc;
  if (fp8) {
    if (k.dtype != v.dtype || !is_float(k.dtype) || kc.dtype != ElemType::U8 || vc.dtype != ElemType::U8)
      return fail(KVC_EINVAL, "reshape_and_cache_fp8 needs float32/float16/bfloat16 key/value and uint8 caches");
  } else if (k.dtype != v.dtype || kc.dtype != vc.dtype || !is_supported_pair(k.dtype, kc.dtype))
    return fail(KVC_EINVAL, std::string("Unsupported dtype combination for reshape_and_cache: kv ") +
                                elem_name(k.dtype) + "/" + elem_name(v.dtype) + ", cache " + elem_name(kc.dtype) +
                                "/" + elem_name(vc.dtype));
  if (flash && kc.dtype != k.dtype)
    return fail(KVC_EINVAL, "reshape_and_cache_flash requires key and cache dtypes to match");
  const int64_t H = k.shape[1], D = k.shape[2];
  if (k.stride(2) != 1 || v.stride(2) != 1 || sm.stride(0) != 1)
    return fail(KVC_EINVAL, "key/value head_size dimension and slot_mapping must be contiguous");
  memset(a, 0, sizeof(*a));
  if (flash) {
    // [nb, bs, H, D] or the pool's [slots, H, D] (block_size 1).
    if (!((kc.ndim == 4 && vc.ndim == 4) || (kc.ndim == 3 && vc.ndim == 3)))
      return fail(KVC_EINVAL, "flash caches must have shape [num_blocks, block_size, num_heads, head_size]");
    for (int i = 0; i < kc.ndim; ++i)
      if (kc.shape[i] != vc.shape[i]) return fail(KVC_EINVAL, "key_cache and value_cache shapes differ");
    if (kc.size(-2) != H || kc.size(-1) != D)
      return fail(KVC_EINVAL, "cache num_heads/head_size do not match key");
    if (kc.stride(-1) != 1 || vc.stride(-1) != 1)
      return fail(KVC_EINVAL, "cache head_size dimension must be contiguous");
    a->block_size = kc.ndim == 4 ? (int)kc.shape[1] : 1;
    a->num_blocks = kc.shape[0];
    a->kc_block_stride = kc.stride(0);
    a->vc_block_stride = vc.stride(0);
    a->kc_tok_stride = kc.ndim == 4 ? kc.stride(1) : kc.stride(0);
    a->vc_tok_stride = vc.ndim == 4 ? vc.stride(1) : vc.stride(0);
    a->kc_head_stride = kc.stride(-2);
    a->vc_head_stride = vc.stride(-2);
  } else {
    const int x = 16 / elem_size(kc.dtype);
    if (kc.ndim != 5 || vc.ndim != 4)
      return fail(KVC_EINVAL, "key_cache/value_cache must use paged attention layouts");
    if (kc.shape[1] != H || vc.shape[1] != H)
      return fail(KVC_EINVAL, "cache KV-head count does not match key");
    if (kc.shape[2] * kc.shape[4] != D || vc.shape[2] != D)
      return fail(KVC_EINVAL, "cache head size does not match key head size");
    if (kc.shape[4] != x)
      return fail(KVC_EINVAL, "key_cache last dimension must be x = 16 / sizeof(cache element) = " + std::to_string(x));
    if (kc.shape[0] != vc.shape[0] || kc.shape[3] != vc.shape[3])
      return fail(KVC_EINVAL, "cache block dimensions of key_cache and value_cache differ");
    if (!kc.dense_from(2) || !vc.dense_from(2))
      return fail(KVC_EINVAL, "key_cache/value_cache pages must be dense ([D/x, bs, x] and [D, bs])");
    a->block_size = (int)kc.shape[3];
    a->num_blocks = kc.shape[0];
    a->kc_block_stride = kc.stride(0);
    a->kc_head_stride = kc.stride(1);
    a->vc_block_stride = vc.stride(0);
    a->vc_head_stride = vc.stride(1);
  }
  if (H <= 0 || D <= 0 || H * D > (int64_t)1 << 24) return fail(KVC_EINVAL, "unsupported num_heads * head_size");
  if (int rc = check_all_cuda({&k, &v, &kc, &vc, &sm}, device)) return rc;
  a->key = k.data;
  a->value = v.data;
  a->key_cache = kc.data;
  a->value_cache = vc.data;
  a->slots = sm.data;
  a->kv_type = k.dtype;
  a->cache_type = kc.dtype;
  a->slot_type = sm.dtype;
  a->num_tokens = k.shape[0];
  a->num_heads = (int)H;
  a->head_size = (int)D;
  a->key_tok_stride = k.stride(0);
  a->key_head_stride = k.stride(1);
  a->value_tok_stride = v.stride(0);
  a->value_head_stride = v.stride(1);
  return KVC_OK;
}

int kvc_reshape_and_cache(const kvc_dltensor* key, const kvc_dltensor* value, kvc_dltensor* key_cache,
                          kvc_dltensor* value_cache, const kvc_dltensor* slot_mapping, void* stream) {
  ReshapeArgs a;
  int device = -1;
  if (int rc = prepare_reshape(key, value, key_cache, value_cache, slot_mapping, false, &a, &device)) return rc;
  if (a.num_tokens == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_reshape_and_cache(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "reshape_and_cache launch");
  return KVC_OK;
}

int kvc_reshape_and_cache_flash(const kvc_dltensor* key, const kvc_dltensor* value, kvc_dltensor* key_cache,
                                kvc_dltensor* value_cache, const kvc_dltensor* slot_mapping, void* stream) {
  ReshapeArgs a;
  int device = -1;
  if (int rc = prepare_reshape(key, value, key_cache, value_cache, slot_mapping, true, &a, &device)) return rc;
  if (a.num_tokens == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_reshape_and_cache_flash(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "reshape_and_cache_flash launch");
  return KVC_OK;
}

int kvc_paged_attention_planned_append(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                       kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key,
                                       const kvc_dltensor* value, kvc_dltensor* key_cache, kvc_dltensor* value_cache,
                                       const kvc_dltensor* slot_mapping, const kvc_dltensor* block_tables,
                                       const kvc_dltensor* context_lens, int num_kv_heads, float scale,
                                       int block_size, int max_seq_len, const kvc_dltensor* alibi_slopes,
                                       int partition_size, kvc_dltensor* plan, void* stream) {
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device))
    return rc;
  if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                       device, &a))
    return rc;
  if (int rc = check_plan_args(a.num_seqs, num_kv_heads, max_seq_len, partition_size)) return rc;
  if (int rc = parse_plan(plan, a.num_seqs, num_kv_heads, max_seq_len, partition_size, &device, &a.plan)) return rc;
  ReshapeArgs r;
  int rdev = device;
  if (int rc = prepare_reshape(key, value, key_cache, value_cache, slot_mapping, false, &r, &rdev)) return rc;
  if (rdev != device) return fail(KVC_EINVAL, "all tensors must live on the same CUDA device");
  if (r.num_tokens != a.num_seqs)
    return fail(KVC_EINVAL, "key/value must hold one new token per sequence: [num_seqs, num_kv_heads, head_size]");
  if (r.kv_type != a.cache_type || a.cache_type == ElemType::U8)
    return fail(KVC_EUNSUPPORTED, "paged_attention_planned_append needs key/value of the cache's dtype "
                                  "(float16/bfloat16)");
  a.new_k = r.key;
  a.new_v = r.value;
  a.slots = r.slots;
  a.slot_type = r.slot_type;
  a.nk_tok_stride = r.key_tok_stride;
  a.nk_head_stride = r.key_head_stride;
  a.nv_tok_stride = r.value_tok_stride;
  a.nv_head_stride = r.value_head_stride;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)
    return fail(KVC_EUNSUPPORTED, "paged_attention_planned_append runs on the tensor-core decode only (float16/bfloat16 "
                                  "query and cache of one dtype, head size 64/128, block size 8/16/32, up to 16 query "
                                  "heads per KV head)");
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_planned_append launch");
  return KVC_OK;
}

int kvc_gather_kv(kvc_dltensor* k_out, kvc_dltensor* v_out, const kvc_dltensor* k_buffer,
                  const kvc_dltensor* v_buffer, const kvc_dltensor* indices, void* stream) {
  View ko, vo, kb, vb, ix;
  if (!parse(k_out, "k_out", &ko) || !parse(v_out, "v_out", &vo) || !parse(k_buffer, "k_buffer", &kb) ||
      !parse(v_buffer, "v_buffer", &vb) || !parse(indices, "indices", &ix))
    return KVC_EINVAL;
  if (ix.ndim != 1) return fail(KVC_EINVAL, "indices must be 1-D");
  if (int rc = check_index_type(ix, "indices", true)) return rc;
  if (!((kb.ndim == 3 && vb.ndim == 3) || (kb.ndim == 4 && vb.ndim == 4)))
    return fail(KVC_EINVAL, "k_buffer/v_buffer must have shape [slots, H, D] or [num_blocks, block_size, H, D]");
  for (int i = 0; i < kb.ndim; ++i)
    if (kb.shape[i] != vb.shape[i]) return fail(KVC_EINVAL, "k_buffer and v_buffer shapes differ");
  if (kb.dtype != vb.dtype || ko.dtype != kb.dtype || vo.dtype != kb.dtype || !is_float(kb.dtype))
    return fail(KVC_EINVAL, "gather buffers and outputs must share one float dtype");
  const int64_t H = kb.size(-2), D = kb.size(-1), T = ix.shape[0];
  if (ko.ndim != 4 || vo.ndim != 4 || ko.shape[0] != 1 || ko.shape[1] != H || ko.shape[2] != T || ko.shape[3] != D ||
      vo.shape[0] != 1 || vo.shape[1] != H || vo.shape[2] != T || vo.shape[3] != D)
    return fail(KVC_EINVAL, "k_out/v_out must have shape [1, H, T, D]");
  if (kb.stride(-1) != 1 || vb.stride(-1) != 1 || ko.stride(3) != 1 || vo.stride(3) != 1 || ix.stride(0) != 1)
    return fail(KVC_EINVAL, "head_size dimensions and indices must be contiguous");
  int64_t slots = kb.shape[0];
  int64_t kslot = kb.stride(0), vslot = vb.stride(0);
  if (kb.ndim == 4) {
    // [nb, bs, H, D] flattened to slots: requires the block dim to be a whole
    // multiple of the token stride.
    if (kb.stride(0) != kb.shape[1] * kb.stride(1) || vb.stride(0) != vb.shape[1] * vb.stride(1))
      return fail(KVC_EINVAL, "block-layout buffers must have dense [num_blocks, block_size] dims");
    slots = kb.shape[0] * kb.shape[1];
    kslot = kb.stride(1);
    vslot = vb.stride(1);
  }
  int device = -1;
  if (int rc = check_all_cuda({&ko, &vo, &kb, &vb, &ix}, &device)) return rc;
  if (T == 0 || H == 0 || D == 0) return KVC_OK;
  GatherArgs a;
  memset(&a, 0, sizeof(a));
  a.k_out = ko.data;
  a.v_out = vo.data;
  a.k_buf = kb.data;
  a.v_buf = vb.data;
  a.indices = ix.data;
  a.type = kb.dtype;
  a.index_type = ix.dtype;
  a.num_indices = T;
  a.num_slots = slots;
  a.num_heads = (int)H;
  a.head_size = (int)D;
  a.kb_slot_stride = kslot;
  a.kb_head_stride = kb.stride(-2);
  a.vb_slot_stride = vslot;
  a.vb_head_stride = vb.stride(-2);
  a.ko_tok_stride = ko.stride(2);
  a.ko_head_stride = ko.stride(1);
  a.vo_tok_stride = vo.stride(2);
  a.vo_head_stride = vo.stride(1);
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_gather_kv(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather_kv launch");
  return KVC_OK;
}

// ---- FP8 (one-byte) KV cache -------------------------------------------------

static int check_fp8_args(float k_scale, float v_scale, int fp8_format) {
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale))
    return fail(KVC_EINVAL, "k_scale and v_scale must be positive and finite");
  if (fp8_format < 0 || fp8_format > 3)
    return fail(KVC_EINVAL, "fp8_format must be 0 (e4m3), 1 (e5m2), 2 (e4m3-sat) or 3 (e5m2-sat)");
  return KVC_OK;
}

int kvc_reshape_and_cache_fp8(const kvc_dltensor* key, const kvc_dltensor* value, kvc_dltensor* key_cache,
                              kvc_dltensor* value_cache, const kvc_dltensor* slot_mapping, float k_scale,
                              float v_scale, int fp8_format, void* stream) {
  if (int rc = check_fp8_args(k_scale, v_scale, fp8_format)) return rc;
  ReshapeArgs a;
  int device = -1;
  if (int rc = prepare_reshape(key, value, key_cache, value_cache, slot_mapping, false, &a, &device, true)) return rc;
  if (a.head_size % 16 != 0) return fail(KVC_EINVAL, "head_size must be a multiple of 16 for one-byte caches");
  if ((reinterpret_cast<uintptr_t>(a.key_cache) & 15u) || (a.kc_block_stride & 15) || (a.kc_head_stride & 15))
    return fail(KVC_EINVAL, "key_cache pages must start on 16-byte boundaries");
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.fp8_format = fp8_format;
  if (a.num_tokens == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_reshape_and_cache_fp8(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "reshape_and_cache_fp8 launch");
  return KVC_OK;
}

int kvc_paged_attention_fp8(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                            kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                            const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                            const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                            int max_seq_len, const kvc_dltensor* alibi_slopes, float k_scale, float v_scale,
                            int fp8_format, int partition_size, void* stream) {
  if (int rc = check_fp8_args(k_scale, v_scale, fp8_format)) return rc;
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device, true))
    return rc;
  const int G = a.num_heads / a.num_kv_heads;
  if (!(a.head_size == 64 || a.head_size == 128) || G > 16)
    return fail(KVC_EUNSUPPORTED, "paged_attention_fp8 supports head_size 64 or 128 and up to 16 query heads per "
                                  "KV head");
  if (partition_size != 0) {
    if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                         device, &a))
      return rc;
  }
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.fp8_format = fp8_format;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_fp8 launch");
  return KVC_OK;
}

int kvc_paged_attention_fp8_planned(kvc_dltensor* out, kvc_dltensor* exp_sums, kvc_dltensor* max_logits,
                                    kvc_dltensor* tmp_out, const kvc_dltensor* query, const kvc_dltensor* key_cache,
                                    const kvc_dltensor* value_cache, const kvc_dltensor* block_tables,
                                    const kvc_dltensor* context_lens, int num_kv_heads, float scale, int block_size,
                                    int max_seq_len, const kvc_dltensor* alibi_slopes, float k_scale, float v_scale,
                                    int fp8_format, int partition_size, kvc_dltensor* plan, void* stream) {
  if (int rc = check_fp8_args(k_scale, v_scale, fp8_format)) return rc;
  DecodeArgs a;
  int device = -1;
  if (int rc = prepare_decode(out, query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, &a, &device, true))
    return rc;
  const int G = a.num_heads / a.num_kv_heads;
  if (!(a.head_size == 64 || a.head_size == 128) || G > 16)
    return fail(KVC_EUNSUPPORTED, "paged_attention_fp8 supports head_size 64 or 128 and up to 16 query heads per "
                                  "KV head");
  if (int rc = attach_splitk_workspace(exp_sums, max_logits, tmp_out, partition_size, block_size, max_seq_len,
                                       device, &a))
    return rc;
  if (int rc = check_plan_args(a.num_seqs, num_kv_heads, max_seq_len, partition_size)) return rc;
  if (int rc = parse_plan(plan, a.num_seqs, num_kv_heads, max_seq_len, partition_size, &device, &a.plan)) return rc;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.fp8_format = fp8_format;
  if (a.num_seqs == 0) return KVC_OK;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_paged_decode(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_fp8_planned launch");
  return KVC_OK;
}

int kvc_convert_fp8(kvc_dltensor* dst, const kvc_dltensor* src, float scale, int fp8_format, void* stream) {
  if (int rc = check_fp8_args(scale, 1.f, fp8_format)) return rc;
  View d, s;
  if (!parse(dst, "dst", &d) || !parse(src, "src", &s)) return KVC_EINVAL;
  if (d.ndim != s.ndim) return fail(KVC_EINVAL, "src and dst shapes differ");
  for (int i = 0; i < d.ndim; ++i)
    if (d.shape[i] != s.shape[i]) return fail(KVC_EINVAL, "src and dst shapes differ");
  auto ok_type = [](ElemType t) { return t == ElemType::U8 || is_float(t); };
  if (!ok_type(d.dtype) || !ok_type(s.dtype))
    return fail(KVC_EINVAL, "convert_fp8 converts between uint8 codes and float32/float16/bfloat16");
  if (!d.dense_from(0) || !s.dense_from(0)) return fail(KVC_EINVAL, "src and dst must be contiguous");
  int device = -1;
  if (int rc = check_all_cuda({&d, &s}, &device)) return rc;
  DeviceGuard g(device);
  if (!g.ok()) return fail(KVC_ECUDA, "cudaSetDevice failed");
  cudaError_t e = launch_convert_fp8(s.dtype, d.dtype, s.data, d.data, scale, s.numel(), fp8_format,
                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "convert_fp8 launch");
  return KVC_OK;
}

int kvc_get_max_shared_memory_per_block_device_attribute(int device, int64_t* out) {
  if (!out) return fail(KVC_EINVAL, "out is null");
  int v = 0;
  cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  *out = v;
  return KVC_OK;
}

int kvc_get_device_attribute(int attribute, int device, int64_t* out) {
  if (!out) return fail(KVC_EINVAL, "out is null");
  int v = 0;
  cudaError_t e = cudaDeviceGetAttribute(&v, static_cast<cudaDeviceAttr>(attribute), device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  *out = v;
  return KVC_OK;
}

// ---- runtime helpers ---------------------------------------------------------

int kvc_device_count(int* count) {
  if (!count) return fail(KVC_EINVAL, "count is null");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  *count = n;
  return KVC_OK;
}

int kvc_set_device(int device) {
  cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaSetDevice");
}

int kvc_get_device(int* device) {
  if (!device) return fail(KVC_EINVAL, "device is null");
  cudaError_t e = cudaGetDevice(device);
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaGetDevice");
}

int kvc_malloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(KVC_EINVAL, "ptr is null");
  *ptr = nullptr;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(KVC_ENOMEM, "cudaMalloc of " + std::to_string(bytes) + " bytes failed: out of device memory");
  }
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaMalloc");
}

int kvc_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaFree");
}

int kvc_malloc_host(void** ptr, size_t bytes) {
  if (!ptr) return fail(KVC_EINVAL, "ptr is null");
  *ptr = nullptr;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMallocHost(ptr, bytes);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(KVC_ENOMEM, "cudaMallocHost failed: out of pinned memory");
  }
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaMallocHost");
}

int kvc_free_host(void* ptr) {
  cudaError_t e = cudaFreeHost(ptr);
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaFreeHost");
}

int kvc_memcpy_async(void* dst, const void* src, size_t bytes, int kind, void* stream) {
  if (kind < 0 || kind > 4) return fail(KVC_EINVAL, "invalid memcpy kind");
  if (bytes == 0) return KVC_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, static_cast<cudaMemcpyKind>(kind), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaMemcpyAsync");
}

int kvc_memset_async(void* dst, int value, size_t bytes, void* stream) {
  if (bytes == 0) return KVC_OK;
  cudaError_t e = cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaMemsetAsync");
}

int kvc_stream_create(void** stream) {
  if (!stream) return fail(KVC_EINVAL, "stream is null");
  cudaStream_t s;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
  *stream = s;
  return KVC_OK;
}

int kvc_stream_destroy(void* stream) {
  cudaError_t e = cudaStreamDestroy(static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaStreamDestroy");
}

int kvc_stream_synchronize(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaStreamSynchronize");
}

int kvc_device_synchronize(void) {
  cudaError_t e = cudaDeviceSynchronize();
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaDeviceSynchronize");
}

int kvc_event_create(void** event) {
  if (!event) return fail(KVC_EINVAL, "event is null");
  cudaEvent_t ev;
  cudaError_t e = cudaEventCreate(&ev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
  *event = ev;
  return KVC_OK;
}

int kvc_event_destroy(void* event) {
  cudaError_t e = cudaEventDestroy(static_cast<cudaEvent_t>(event));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaEventDestroy");
}

int kvc_event_record(void* event, void* stream) {
  cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaEventRecord");
}

int kvc_stream_wait_event(void* stream, void* event) {
  cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0);
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaStreamWaitEvent");
}

int kvc_event_synchronize(void* event) {
  cudaError_t e = cudaEventSynchronize(static_cast<cudaEvent_t>(event));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaEventSynchronize");
}

int kvc_event_elapsed_ms(void* start, void* end, float* ms) {
  if (!ms) return fail(KVC_EINVAL, "ms is null");
  cudaError_t e = cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaEventElapsedTime");
}

int kvc_stream_begin_capture(void* stream) {
  if (!stream) return fail(KVC_EINVAL, "capture needs a non-default stream");
  cudaError_t e = cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeThreadLocal);
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaStreamBeginCapture");
}

int kvc_stream_end_capture(void* stream, void** graph_exec) {
  if (!graph_exec) return fail(KVC_EINVAL, "graph_exec is null");
  *graph_exec = nullptr;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &graph);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
  *graph_exec = exec;
  return KVC_OK;
}

int kvc_graph_launch(void* graph_exec, void* stream) {
  cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaGraphLaunch");
}

int kvc_graph_destroy(void* graph_exec) {
  cudaError_t e = cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "cudaGraphExecDestroy");
}

int kvc_l2_flush(void* scratch, size_t bytes, void* stream) {
  if (bytes == 0) return KVC_OK;
  cudaError_t e = cudaMemsetAsync(scratch, 0x5a, bytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_fail(e, "kvc_l2_flush");
}

}  // extern "C"
