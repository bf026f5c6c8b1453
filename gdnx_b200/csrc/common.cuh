// Shared device helpers for the GDNX sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "gdnx.h"

#define GDNX_DEV __device__ __forceinline__

namespace gdnx {

// Load element `off` (in elements) of a view as fp32.
GDNX_DEV float ld_as_f32(const void* base, int dtype, int64_t off) {
  if (dtype == GDNX_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[off]);
  if (dtype == GDNX_F16) return __half2float(reinterpret_cast<const __half*>(base)[off]);
  return reinterpret_cast<const float*>(base)[off];
}

GDNX_DEV void st_from_f32(void* base, int dtype, int64_t off, float x) {
  if (dtype == GDNX_BF16) reinterpret_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(x);
  else if (dtype == GDNX_F16) reinterpret_cast<__half*>(base)[off] = __float2half_rn(x);
  else reinterpret_cast<float*>(base)[off] = x;
}

// Offset of element [b, t, h, m, (slot,) 0] of a view.
GDNX_DEV int64_t view_off(const gdnx_view& v, int64_t b, int64_t t, int64_t h, int64_t m, int64_t s = 0) {
  return b * v.sb + t * v.st + h * v.sh + m * v.sm + s * v.ss;
}

// Exact delta-rule write coefficient alpha(c) = (1 - e^-c) / c, with the
// reference's Taylor branch for |c| < 1e-6 (gdn3/gdn3_upgrade.py:641-648).
// Uses CUDA's expm1f.
GDNX_DEV float stable_alpha(float c) {
  if (fabsf(c) < 1e-6f) return 1.0f - c * 0.5f + c * c * (1.0f / 6.0f);
  return -expm1f(-c) / c;
}

GDNX_DEV float softplus_f(float x) {
  // torch.nn.functional.softplus (beta=1, threshold=20)
  return x > 20.0f ? x : log1pf(expf(x));
}

// Decay factor of one chain-token from a dim-1 (or braided dim-4) decay view.
GDNX_DEV float decay_factor(const gdnx_view& d, int kind, int64_t off, bool clamp01,
                            const float* rates, float braid_clamp) {
  if (kind == GDNX_DECAY_BRAIDED) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float g = fminf(softplus_f(ld_as_f32(d.ptr, d.dtype, off + i)), 5.0f);
      acc += expf(-g * rates[i]);
    }
    return fminf(acc * 0.25f, braid_clamp);
  }
  float x = ld_as_f32(d.ptr, d.dtype, off);
  float g = (kind == GDNX_DECAY_LOG) ? expf(x) : x;
  if (clamp01) g = fminf(fmaxf(g, 0.0f), 1.0f);
  return g;
}

GDNX_DEV float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Apply the reference's lane RoPE in place on a K-vector held in shared
// memory by one warp:  x1' = x1 c - x2 s;  x2' = x1' s + x2 c.
GDNX_DEV void rope_row_warp(float* row, const gdnx_rope& rp, int lane_m, int64_t pos, int lane) {
  if (!rp.enable || lane_m >= 4) return;
  const int d = rp.pairs[lane_m];
  if (d <= 0) return;
  const float scale = rp.scale[lane_m];
  const float den = rp.den[lane_m];
  const float p = (float)pos * scale;
  for (int i = lane; i < d; i += 32) {
    const float inv_freq = 1.0f / powf(10000.0f, (float)i / den);
    const float ang = p * inv_freq;
    float s, c;
    sincosf(ang, &s, &c);
    const float x1 = row[i], x2 = row[i + d];
    const float n1 = x1 * c - x2 * s;
    row[i] = n1;
    row[i + d] = n1 * s + x2 * c;
  }
}

// Lane RoPE from a precomputed cos/sin row: x1' = x1 c - x2 s; x2' = x1' s + x2 c
// (the reference's in-place update), same fp32 values as rope_row_warp when the
// table holds sincosf(((float)pos * scale) * inv_freq_i).
GDNX_DEV void rope_row_table(float* row, int d, const float* cs, const float* sn, int lane) {
  for (int i = lane; i < d; i += 32) {
    const float c = cs[i], s = sn[i];
    const float x1 = row[i], x2 = row[i + d];
    const float n1 = x1 * c - x2 * s;
    row[i] = n1;
    row[i + d] = n1 * s + x2 * c;
  }
}

}  // namespace gdnx
