// Packed INT8 quantiser arithmetic shared by the fused rmsnorm + quantiser
// and the standalone quantisers (quant_matmul/reference.py:16-24).
#pragma once

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace b200 {

// INT8 codes of eight 16-bit values y (one 16-byte vector of T's bits) for
// the row scale s, rs = RN(1/s):
//  - bf16: q = RN_bf16(y * rs) without Markstein's correction.  y and s
//    have 8-bit significands, so y / s is either exactly representable in
//    bf16 or a fraction p/q (q odd, q <= 255) at least 2^-17 (relative) away
//    from every bf16 rounding midpoint; y * rs is within 2^-23 of y / s, so
//    both round to the same bf16 value (and the fp32 rounding of the
//    quotient, which the reference performs first, cannot land on a
//    midpoint either).  fp16's 11-bit significands leave no such margin, so
//    fp16 keeps the corrected quotient;
//  - the clamp to [-127, 127] is one min.xorsign.abs on the packed pair
//    (rint commutes with clamping at an integer), before the integer
//    rounding: bf16 adds 1.5 * 2^23 to each widened half (the low byte of
//    the sum's bits is rint(v) as int8), fp16 adds 1.5 * 2^10 to the packed
//    pair.
template <typename T>
__device__ __forceinline__ uint2 quant_vec8(const uint4& yv, float s, float rs) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t* yw = reinterpret_cast<const uint32_t*>(&yv);
  uint32_t h[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float v0, v1;
    if constexpr (kBF16) {
      const float y0 = __uint_as_float(yw[k] << 16), y1 = __uint_as_float(yw[k] & 0xFFFF0000u);
      float q0, q1;
      sm100::fmul2_bcast(q0, q1, y0, y1, rs);
      uint32_t pk;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pk) : "f"(q1), "f"(q0));
      asm("min.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(pk) : "r"(pk), "r"(0x42FE42FEu));  // +-127
      asm("{ .reg .b16 l, h; mov.b32 {l, h}, %2; add.rn.f32.bf16 %0, l, %3; add.rn.f32.bf16 %1, h, %3; }"
          : "=f"(v0), "=f"(v1) : "r"(pk), "f"(12582912.0f));
    } else {
      const float2 yf = __half22float2(*reinterpret_cast<const __half2*>(&yw[k]));
      float q0, q1, e0, e1;
      sm100::fmul2_bcast(q0, q1, yf.x, yf.y, rs);
      sm100::ffma2(e0, e1, q0, q1, -s, -s, yf.x, yf.y);
      sm100::ffma2(v0, v1, e0, e1, rs, rs, q0, q1);
      uint32_t pk;
      asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(pk) : "f"(v1), "f"(v0));
      asm("min.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(pk) : "r"(pk), "r"(0x57F057F0u));  // +-127
      // + 1536 (1.5 * 2^10) in f16x2: the sums lie in [1409, 1663], where
      // the fp16 spacing is 1, so the add rounds v half to even and the low
      // byte of each half's bits (0x6600 + rint(v)) is rint(v) as int8
      asm("add.rn.f16x2 %0, %1, %2;" : "=r"(h[k]) : "r"(pk), "r"(0x66006600u));
      continue;
    }
    h[k] = __byte_perm(__float_as_uint(v0), __float_as_uint(v1), 0x0040);
  }
  if constexpr (kBF16)
    return make_uint2(__byte_perm(h[0], h[1], 0x5410), __byte_perm(h[2], h[3], 0x5410));
  else  // codes in bytes 0 and 2 of each word
    return make_uint2(__byte_perm(h[0], h[1], 0x6420), __byte_perm(h[2], h[3], 0x6420));
}

// Absolute maxima of two packed pairs of 16-bit values, as a packed pair: the
// magnitude of each half is max(|a|, |b|) (its sign is not meaningful).
template <typename T>
__device__ __forceinline__ uint32_t absmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// The larger magnitude of a packed pair, widened to fp32 (exact).
template <typename T>
__device__ __forceinline__ float absmax_of_pair(uint32_t w) {
  const uint32_t m = w & 0x7FFF7FFFu;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
  else
    return fmaxf(__half2float(__ushort_as_half((unsigned short)(m & 0xFFFFu))),
                 __half2float(__ushort_as_half((unsigned short)(m >> 16))));
}

}  // namespace b200
