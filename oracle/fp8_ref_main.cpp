/*
 * fp8_ref_main.cpp — runs the reference's own FP8 codec functions
 * (paged_attention/metal/float8.metal:14-125, compiled unmodified from the
 * reference checkout through oracle/msl_shim.h) to produce golden vectors.
 * Test infrastructure only; built into oracle/_ref/ by `make -C oracle ref`.
 *
 *   fp8_ref dec                 256 float32 values per format (E4M3 codes 0..255,
 *                               then E5M2), binary, to stdout
 *   fp8_ref enc                 float32 values on stdin -> one E4M3 and one E5M2
 *                               code per value (interleaved), binary, to stdout
 *   fp8_ref sweep e4m3|e5m2     the code of every float32 bit pattern 0 .. 2^32-1,
 *                               in order, binary, to stdout (4 GiB)
 *
 * Inputs on which the reference's encoder is undefined are not passed to it:
 * past the last finite exponent its subnormal branch shifts by
 * (1 - e) + (23 - MAN_BITS) with e the biased FP8 exponent, a negative shift
 * once |x| >= 2^14 (E4M3) or |x| >= 2^16 (E5M2), which is undefined behaviour in
 * C++ and in MSL.  For those inputs this program writes the saturated code
 * (sign | all-ones exponent | zero mantissa = +-Inf), the value the library
 * defines there; every other input gets the reference function's result.
 */
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "float8.metal"

namespace {

// True when float8.metal's encoder would shift by a count outside [0, 31] for
// this input (see the file comment).
template <int EXP_BITS, int MAN_BITS, int BIAS>
bool encoder_undefined(uint32_t bits) {
  const uint32_t a = bits & 0x7FFFFFFFu;
  if (a >= 0x7F800000u) return false;            // Inf / NaN branch
  const int e_fp8 = int((a >> 23) & 0xFF) - 127 + BIAS;
  const int exp_max = (1 << EXP_BITS) - 2;
  if (e_fp8 >= 1 && e_fp8 <= exp_max) return false;  // normal path
  if (e_fp8 < 1 - MAN_BITS) return false;            // flushed to zero
  const int rshift = (1 - e_fp8) + (23 - MAN_BITS);
  return rshift < 1 || rshift > 31;
}

template <int EXP_BITS, int MAN_BITS, int BIAS>
uint8_t encode(uint32_t bits) {
  if (encoder_undefined<EXP_BITS, MAN_BITS, BIAS>(bits))
    return uint8_t(((bits >> 31) << 7) | (((1u << EXP_BITS) - 1u) << MAN_BITS));
  float f;
  std::memcpy(&f, &bits, 4);
  return detail::fp32_to_fp8<EXP_BITS, MAN_BITS, BIAS>(f);
}

int write_all(const void* p, size_t n) { return fwrite(p, 1, n, stdout) == n ? 0 : 1; }

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    fprintf(stderr, "usage: fp8_ref dec | enc | sweep e4m3|e5m2\n");
    return 2;
  }
  if (!strcmp(argv[1], "dec")) {
    float out[512];
    for (int c = 0; c < 256; ++c) {
      out[c] = fp8_e4m3_to_float(uchar(c));
      out[256 + c] = fp8_e5m2_to_float(uchar(c));
    }
    return write_all(out, sizeof(out));
  }
  if (!strcmp(argv[1], "enc")) {
    uint32_t in[4096];
    uint8_t out[8192];
    size_t n;
    while ((n = fread(in, 4, 4096, stdin)) > 0) {
      for (size_t i = 0; i < n; ++i) {
        out[2 * i] = encode<4, 3, 7>(in[i]);
        out[2 * i + 1] = encode<5, 2, 15>(in[i]);
      }
      if (write_all(out, 2 * n)) return 1;
    }
    return 0;
  }
  if (!strcmp(argv[1], "sweep") && argc > 2) {
    const bool e4m3 = !strcmp(argv[2], "e4m3");
    std::vector<uint8_t> buf(1u << 24);
    for (uint64_t base = 0; base < (1ull << 32); base += buf.size()) {
      for (uint32_t i = 0; i < buf.size(); ++i) {
        const uint32_t bits = uint32_t(base + i);
        buf[i] = e4m3 ? encode<4, 3, 7>(bits) : encode<5, 2, 15>(bits);
      }
      if (write_all(buf.data(), buf.size())) return 1;
    }
    return 0;
  }
  fprintf(stderr, "unknown mode %s\n", argv[1]);
  return 2;
}
