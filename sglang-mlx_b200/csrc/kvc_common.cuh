// kvc_common.cuh — shared device/host helpers of libkvcache (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "kvcache.h"
#include "kvc_tensor.h"

namespace kvc {

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

// Conversion into the cache element type.  Narrowing uses round-to-nearest-even,
// which is what Metal's static_cast<half/bfloat>(float) does
// (reshape_and_cache.metal:9-12).
template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename SRC, typename DST> struct Convert {
  __device__ __forceinline__ static DST apply(SRC v) { return from_float<DST>(to_float(v)); }
};
template <typename T> struct Convert<T, T> {
  __device__ __forceinline__ static T apply(T v) { return v; }
};

// ---- per-translation-unit sticky status word ---------------------------------
// Each .cu file that launches kernels defines its own status word and a host
// accessor; kvc_get_status ORs them.
__device__ __forceinline__ void set_status(unsigned int* word, unsigned int bit) {
  atomicOr(word, bit);
}

// ---- host-side launch bookkeeping ---------------------------------------------
void count_launch();
void set_error(const std::string& msg);

}  // namespace kvc
