// int8 activation codes from fp16 values: the arithmetic every quantizer of this library shares
// (the reference's pack shader, native/aexrt_d3d12_runtime.cpp:3333-3344: q = round_half_even(
// x * (127 / amax)), low byte kept, no clamp).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace aexrt {

// Adds 1.5*2^23 to both halves of a packed fl32 product: the low byte of each sum's bits is
// round_half_even(product) & 0xFF for |product| < 2^22.  Scalar __fadd_rn, which is never
// merged into a multiply-add, keeps the product rounded on its own (a fused x * mult + 1.5*2^23
// rounds once and differs from the two-step result near .5).
__device__ __forceinline__ void magic_round2(uint64_t vq, uint32_t& a, uint32_t& b) {
  float x, y;
  f2_unpack(vq, x, y);
  a = __float_as_uint(__fadd_rn(x, 12582912.0f));
  b = __float_as_uint(__fadd_rn(y, 12582912.0f));
}

// int8 codes of 8 fp16 values, q = low byte of round_half_even(fl32(x * mult)), four per word.
// kMagic: the rounding comes from adding 1.5*2^23 (exact for |x * mult| < 2^22); else float-to-int.
template <bool kMagic>
__device__ __forceinline__ void codes8(const uint4& v, float mult, uint32_t& q0, uint32_t& q1) {
  const __half2* h2 = reinterpret_cast<const __half2*>(&v);
  const uint64_t m2 = f2_pack(mult, mult);
  uint32_t b[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __half22float2(h2[e]);
    const uint64_t vq = f2_mul(f2_pack(f.x, f.y), m2);
    if (kMagic) {
      magic_round2(vq, b[2 * e], b[2 * e + 1]);
    } else {
      float a, c;
      f2_unpack(vq, a, c);
      b[2 * e] = static_cast<uint32_t>(__float2int_rn(a));
      b[2 * e + 1] = static_cast<uint32_t>(__float2int_rn(c));
    }
  }
  q0 = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
  q1 = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
}

}  // namespace aexrt
