// pl_fp16.cuh -- picolm's FP32 -> FP16 encoding and its RoPE arithmetic,
// restated for the device so that KV rows written on the B200 are
// bit-identical to the ones picolm writes on the CPU.
//
// picolm/quant.c:41-78 does NOT round to nearest even: in the normal range
// it adds half an FP16 ulp to the FP32 mantissa and truncates, i.e. ties go
// away from zero.  cvt.rn.f16.f32 / __float2half_rn round ties to even and
// would differ on every tie, so the conversion is done with integer ops.
#pragma once
#include <cstdint>

namespace pl {

__device__ __forceinline__ uint16_t picolm_f32_to_f16(float f) {
  const uint32_t b = __float_as_uint(f);
  const uint32_t s = (b >> 16) & 0x8000u;
  const uint32_t E = (b >> 23) & 0xFFu;
  const uint32_t m = b & 0x7FFFFFu;
  if (E == 0) return static_cast<uint16_t>(s);                       // zero, FP32 subnormal
  if (E == 0xFFu) return static_cast<uint16_t>(s | 0x7C00u | (m ? 0x0200u : 0u));  // Inf/NaN
  const int e = static_cast<int>(E) - 112;                           // FP16 biased exponent
  if (e >= 31) return static_cast<uint16_t>(s | 0x7C00u);            // overflow
  if (e <= 0) {                                                      // FP16 subnormal
    if (e < -10) return static_cast<uint16_t>(s);
    const uint32_t full = m | 0x800000u;
    const uint32_t sh = static_cast<uint32_t>(14 - e);
    return static_cast<uint16_t>(s | ((full + (1u << (sh - 1))) >> sh));
  }
  // exponent and mantissa adjacent so the rounding carry propagates
  const uint32_t r = (((static_cast<uint32_t>(e) << 23) | m) + 0x1000u) >> 13;
  return static_cast<uint16_t>(r >= 0x7C00u ? (s | 0x7C00u) : (s | r));
}

// One RoPE rotation as picolm/tensor.c:583-600 evaluates it on the CPU:
// two separately rounded products and one rounded sum, never fused.
__device__ __forceinline__ void rope_pair(float x0, float x1, float c, float s, float& y0,
                                          float& y1) {
  y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

}  // namespace pl
