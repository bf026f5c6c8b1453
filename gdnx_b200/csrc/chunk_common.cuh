// Device helpers shared by the chunked tensor-core scans.
#pragma once

#include "common.cuh"

namespace gdnx {
namespace chunk {

GDNX_DEV void load8_bf16(const void* base, int64_t off, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off);
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(p[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// Raw bits of one element (converted later, so a prefetch does not stall on its load).
GDNX_DEV uint32_t ld_raw(const void* base, int dtype, int64_t off) {
  if (dtype == GDNX_F32) return reinterpret_cast<const uint32_t*>(base)[off];
  return reinterpret_cast<const uint16_t*>(base)[off];
}
GDNX_DEV float raw_f32(uint32_t r, int dtype) {
  if (dtype == GDNX_F32) return __uint_as_float(r);
  if (dtype == GDNX_BF16) return __uint_as_float(r << 16);
  return __half2float(__ushort_as_half((unsigned short)r));
}

// sin and cos of an fp32 angle: Cody-Waite reduction by 2*pi (2*pi split into a
// float head and tail, so the reduced argument is exact to ~1e-10 for |x| up to
// ~1e5), then the hardware sine/cosine on [-pi, pi] (absolute error ~5e-7).
GDNX_DEV void sincos_reduced(float x, float* s, float* c) {
  constexpr float kInv2Pi = 0.15915494309189535f;
  constexpr float k2PiHi = 6.2831854820251465f;    // float(2*pi)
  constexpr float k2PiLo = -1.7484556000744e-07f;  // 2*pi - float(2*pi)
  const float k = rintf(x * kInv2Pi);
  float r = fmaf(-k, k2PiHi, x);
  r = fmaf(-k, k2PiLo, r);
  __sincosf(r, s, c);
}

// 2^x with the hardware base-2 exponential (ex2.approx.ftz: relative error about
// 2^-22, subnormal results flushed to zero); used where a decay factor feeds a
// bf16 operand or an fp32 accumulation with looser tolerance than that.
GDNX_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace chunk
}  // namespace gdnx
