// Output epilogues of the recurrent layers, one warp per (batch, token, head) row:
//
//   GDN3 lane routing (gdn3/gdn3_upgrade.py:842-856):
//     w_m = softmax_m(router_logits[b,t,h,:]);  r = sum_m w_m y[b,t,h,m,:]
//     out = r / max(|r|_2, 1e-6) * sqrt(V) * norm
//   KMD-2 gated RMS norm (Qwen3_5RMSNormGated, gdn3/kmd2_native.py:66,176):
//     out = weight * y * rsqrt(mean(y^2) + eps) * silu(z)
//
// Both stream each input once and write each output once (HBM-bound); with the
// lane sum done here the per-lane outputs never leave the GPU and the multi-GPU
// all-gather moves [B,T,H,V] instead of [B,T,H,M,V].
#include "common.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int NT = 256;  // 8 rows per CTA

GDNX_DEV void ld4f(const void* p, int dtype, int64_t off, float* x) {
  if (dtype == GDNX_F32) {
    const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + off);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else if (dtype == GDNX_BF16) {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + off);
    x[0] = __uint_as_float(u.x << 16); x[1] = __uint_as_float(u.x & 0xffff0000u);
    x[2] = __uint_as_float(u.y << 16); x[3] = __uint_as_float(u.y & 0xffff0000u);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + off);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  }
}
GDNX_DEV void st4f(void* p, int dtype, int64_t off, const float* x) {
  if (dtype == GDNX_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + off) = make_float4(x[0], x[1], x[2], x[3]);
  } else if (dtype == GDNX_BF16) {
    __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + off) = u;
  } else {
    __half2 a = __floats2half2_rn(x[0], x[1]), b = __floats2half2_rn(x[2], x[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + off) = u;
  }
}

__global__ void __launch_bounds__(NT) epilogue_kernel(const gdnx_epilogue_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (row >= a.B * a.T * a.H) return;
  const int64_t h = row % a.H, t = (row / a.H) % a.T, b = row / (a.H * a.T);
  const int V = (int)a.V;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.kind == GDNX_EPILOGUE_LANE_ROUTE) {
    float lg[8];
    float mx = -INFINITY;
    for (int m = 0; m < a.M; ++m) {
      lg[m] = ld_as_f32(a.router.ptr, a.router.dtype, b * a.router.sb + t * a.router.st + h * a.router.sh + m * a.router.sm);
      mx = fmaxf(mx, lg[m]);
    }
    float den = 0.f;
    for (int m = 0; m < a.M; ++m) {
      lg[m] = expf(lg[m] - mx);
      den += lg[m];
    }
    for (int m = 0; m < a.M; ++m) {
      const float w = lg[m] / den;
      const int c = 4 * lane;  // V <= 128: four values per lane
      if (c < V) {
        float y[4];
        ld4f(a.y.ptr, a.y.dtype, b * a.y.sb + t * a.y.st + h * a.y.sh + m * a.y.sm + c, y);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = fmaf(w, y[e], acc[e]);
      }
    }
    const float ss = warp_sum(acc[0] * acc[0] + acc[1] * acc[1] + acc[2] * acc[2] + acc[3] * acc[3]);
    const float sc = sqrtf((float)V) / fmaxf(sqrtf(ss), 1e-6f);
    const int c = 4 * lane;
    if (c < V) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = acc[e] * sc * (a.weight ? a.weight[c + e] : 1.f);
      st4f(a.out, a.out_dtype, b * a.out_sb + t * a.out_st + h * a.out_sh + c, o);
    }
  } else {  // GDNX_EPILOGUE_RMS_GATED
    const int c = 4 * lane;
    float y[4] = {0.f, 0.f, 0.f, 0.f}, z[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < V) {
      ld4f(a.y.ptr, a.y.dtype, b * a.y.sb + t * a.y.st + h * a.y.sh + c, y);
      ld4f(a.gate.ptr, a.gate.dtype, b * a.gate.sb + t * a.gate.st + h * a.gate.sh + c, z);
    }
    const float ss = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
    const float r = rsqrtf(ss / (float)V + a.eps);
    if (c < V) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float sil = z[e] / (1.f + expf(-z[e]));
        o[e] = (a.weight ? a.weight[c + e] : 1.f) * (y[e] * r) * sil;
      }
      st4f(a.out, a.out_dtype, b * a.out_sb + t * a.out_st + h * a.out_sh + c, o);
    }
  }
}

}  // namespace

gdnx_status launch_epilogue(const gdnx_epilogue_args& a, cudaStream_t st) {
  const int64_t rows = a.B * a.T * a.H;
  const int64_t blocks = (rows + NT / 32 - 1) / (NT / 32);
  if (blocks > int64_t(0x7fffffff)) return GDNX_EUNSUPPORTED;
  epilogue_kernel<<<(unsigned)blocks, NT, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
