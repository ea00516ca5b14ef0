// block_ops.cu — whole-block copies of paged caches for sm_100a: copy_blocks
// (copy-on-write of shared blocks inside every layer's K and V caches) and
// swap_blocks (blit between two caches, e.g. device <-> pinned host offload).
//
// Semantics follow copy_blocks.metal:9-88: for each pair (src, dst) of
// block_mapping, the numel_per_block elements of block src are written over
// block dst.  Pairs run in parallel: a block that is the destination of one
// pair and the source of another gives an unspecified result (as on Metal).
//
// One kernel serves both entry points.  A "plane" is one buffer pair (a
// layer's key cache, its value cache, or swap_blocks' src -> dst); the plane
// table travels as a kernel parameter, so nothing is allocated per call.  CTA
// (pair, plane) copies one block with the widest vector the base addresses and
// the block size allow.  HBM-bound: bytes moved = 2 * block bytes per (pair,
// plane).
#include <cuda_runtime.h>
#include <stdint.h>

#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "kvc_common.cuh"

namespace kvc {

__device__ unsigned int g_block_ops_status = 0;

constexpr int kBlockCopyThreads = 256;

// Pairs from a host-side mapping ride in the parameter block too, in chunks.
constexpr int kParamPairs = 128;

struct BlockCopyParams {
  const char* src[kMaxBlockPlanes];
  char* dst[kMaxBlockPlanes];
  int64_t src_blocks[kMaxBlockPlanes];
  int64_t dst_blocks[kMaxBlockPlanes];
  int64_t block_bytes;
  int num_planes;
  // mapping: device pointer (int32 or int64 pairs) or the inline pairs below
  const void* mapping;
  bool mapping_i64;
  int64_t num_pairs;
  int64_t inline_pairs[2 * kParamPairs];
};

template <typename V>
__global__ void __launch_bounds__(kBlockCopyThreads) block_copy_kernel(const __grid_constant__ BlockCopyParams p) {
  const int plane = blockIdx.y;
  for (int64_t pair = blockIdx.x; pair < p.num_pairs; pair += gridDim.x) {
    int64_t s, d;
    if (p.mapping == nullptr) {
      s = p.inline_pairs[2 * pair];
      d = p.inline_pairs[2 * pair + 1];
    } else if (p.mapping_i64) {
      s = static_cast<const int64_t*>(p.mapping)[2 * pair];
      d = static_cast<const int64_t*>(p.mapping)[2 * pair + 1];
    } else {
      s = static_cast<const int32_t*>(p.mapping)[2 * pair];
      d = static_cast<const int32_t*>(p.mapping)[2 * pair + 1];
    }
    if (s < 0 || d < 0 || s >= p.src_blocks[plane] || d >= p.dst_blocks[plane]) {
      if (threadIdx.x == 0) set_status(&g_block_ops_status, KVC_STATUS_INDEX_OOB);
      continue;
    }
    const V* src = reinterpret_cast<const V*>(p.src[plane] + s * p.block_bytes);
    V* dst = reinterpret_cast<V*>(p.dst[plane] + d * p.block_bytes);
    const int64_t n = p.block_bytes / (int64_t)sizeof(V);
    for (int64_t i = threadIdx.x; i < n; i += kBlockCopyThreads) dst[i] = src[i];
  }
}

template <typename V>
static cudaError_t launch_block_copy_v(const BlockCopyParams& p, cudaStream_t stream) {
  const int64_t gx = p.num_pairs < 65535 ? p.num_pairs : 65535;
  dim3 grid((unsigned)gx, (unsigned)p.num_planes);
  block_copy_kernel<V><<<grid, kBlockCopyThreads, 0, stream>>>(p);
  count_launch();
  return cudaGetLastError();
}

static cudaError_t launch_block_copy(BlockCopyParams& p, cudaStream_t stream) {
  if (p.num_pairs == 0 || p.num_planes == 0) return cudaSuccess;
  uintptr_t acc = (uintptr_t)p.block_bytes;
  for (int i = 0; i < p.num_planes; ++i) acc |= reinterpret_cast<uintptr_t>(p.src[i]) | reinterpret_cast<uintptr_t>(p.dst[i]);
  if ((acc & 15u) == 0) return launch_block_copy_v<uint4>(p, stream);
  if ((acc & 7u) == 0) return launch_block_copy_v<uint2>(p, stream);
  if ((acc & 3u) == 0) return launch_block_copy_v<uint32_t>(p, stream);
  if ((acc & 1u) == 0) return launch_block_copy_v<uint16_t>(p, stream);
  return launch_block_copy_v<uint8_t>(p, stream);
}

// Runs the planes of `a` in launches of at most kMaxBlockPlanes planes; a
// host-side mapping goes in parameter chunks of kParamPairs pairs.
cudaError_t launch_block_copies(const BlockCopyArgs& a, cudaStream_t stream) {
  if (a.num_pairs == 0 || a.planes.empty()) return cudaSuccess;
  BlockCopyParams p;
  memset(&p, 0, sizeof(p));
  p.block_bytes = a.block_bytes;
  for (size_t base = 0; base < a.planes.size(); base += kMaxBlockPlanes) {
    p.num_planes = (int)std::min<size_t>(kMaxBlockPlanes, a.planes.size() - base);
    for (int i = 0; i < p.num_planes; ++i) {
      const BlockPlane& pl = a.planes[base + i];
      p.src[i] = static_cast<const char*>(pl.src);
      p.dst[i] = static_cast<char*>(pl.dst);
      p.src_blocks[i] = pl.src_blocks;
      p.dst_blocks[i] = pl.dst_blocks;
    }
    if (a.device_mapping) {
      p.mapping = a.device_mapping;
      p.mapping_i64 = a.mapping_i64;
      p.num_pairs = a.num_pairs;
      cudaError_t e = launch_block_copy(p, stream);
      if (e != cudaSuccess) return e;
    } else {
      p.mapping = nullptr;
      for (int64_t c = 0; c < a.num_pairs; c += kParamPairs) {
        p.num_pairs = std::min<int64_t>(kParamPairs, a.num_pairs - c);
        for (int64_t i = 0; i < 2 * p.num_pairs; ++i) p.inline_pairs[i] = a.host_mapping[2 * c + i];
        cudaError_t e = launch_block_copy(p, stream);
        if (e != cudaSuccess) return e;
      }
    }
  }
  return cudaSuccess;
}

}  // namespace kvc

unsigned int kvc_block_ops_status(int clear, cudaError_t* err) {
  unsigned int v = 0;
  *err = cudaMemcpyFromSymbol(&v, kvc::g_block_ops_status, sizeof(v));
  if (*err == cudaSuccess && clear) {
    const unsigned int zero = 0;
    *err = cudaMemcpyToSymbol(kvc::g_block_ops_status, &zero, sizeof(zero));
  }
  return v;
}
