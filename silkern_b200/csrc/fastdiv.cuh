// Division by a run-time invariant divisor for non-negative int32 numerators.
//
// Method: Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication" (PLDI 1994), section 4, unsigned case with N = 32. For a
// divisor d in [1, 2^31], l = ceil(log2 d) and the (N+1)-bit multiplier
// m = 2^32 + m' with m' = floor(2^32 * (2^l - d) / d) + 1 give
//     floor(n / d) = floor(m * n / 2^(32 + l)) = (mulhi(m', n) + n) >> l
// for every 0 <= n < 2^32. Numerators here are token positions and
// intermediate quotients, all below 2^31, so mulhi(m', n) + n < 2^32 and the
// sum needs no 33rd bit. The host check silkern_fastdiv_selftest_v1 compares
// it against the hardware '/' over whole numerator ranges.
#pragma once

#include <cstdint>

namespace silkern {

struct FastDiv {
  uint32_t divisor;
  uint32_t magic;  // m'
  uint32_t shift;  // l
};

inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((uint64_t{1} << l) < d) ++l;
  const uint64_t m = ((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1;
  return FastDiv{d, static_cast<uint32_t>(m), l};
}

__host__ __device__ __forceinline__ uint32_t fastdiv(uint32_t n, const FastDiv& d) {
#ifdef __CUDA_ARCH__
  const uint32_t hi = __umulhi(n, d.magic);
#else
  const uint32_t hi = static_cast<uint32_t>((static_cast<uint64_t>(n) * d.magic) >> 32);
#endif
  return (hi + n) >> d.shift;
}

}  // namespace silkern
