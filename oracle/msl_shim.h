/*
 * msl_shim.h — just enough of the Metal Shading Language for the scalar FP8
 * codec functions of the reference (paged_attention/metal/float8.metal) to
 * compile as host C++.  Test infrastructure: only the recipe that builds
 * oracle/_ref/fp8_ref uses it (force-included with -include).
 *
 * What MSL provides and this header restates for the host:
 *   uint / uchar            32-bit and 8-bit unsigned integers
 *   as_type<T>(x)           bit reinterpretation between types of one size
 *   ldexp(float, int)       x * 2^e (exact for the codec's operands)
 *   NAN, INFINITY           float constants (<cmath>)
 * <metal_stdlib> resolves to an empty header in oracle/msl_include, and
 * `using namespace metal;` to the namespace below.
 */
#ifndef KVC_MSL_SHIM_H_
#define KVC_MSL_SHIM_H_

#include <cmath>
#include <cstdint>
#include <cstring>

typedef uint32_t uint;
typedef uint8_t uchar;

namespace metal {
template <typename T, typename F>
inline T as_type(F x) {
  static_assert(sizeof(T) == sizeof(F), "as_type needs types of one size");
  T out;
  std::memcpy(&out, &x, sizeof(T));
  return out;
}
inline float ldexp(float x, int e) { return std::ldexp(x, e); }
}  // namespace metal

#endif
