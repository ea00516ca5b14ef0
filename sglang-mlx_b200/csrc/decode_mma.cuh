// decode_mma.cuh — tensor-core paged decode (placeholder: dispatch only).
#pragma once

namespace kvc {

static bool mma_supported(const DecodeArgs&) { return false; }

static cudaError_t launch_mma(const DecodeParams&, const DecodeArgs&, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace kvc
