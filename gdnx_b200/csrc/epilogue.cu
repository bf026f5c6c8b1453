// Output epilogues of the recurrent layers, half a warp per (batch, token, head) row:
//
//   GDN3 lane routing (gdn3/gdn3_upgrade.py:842-856):
//     w_m = softmax_m(router_logits[b,t,h,:]);  r = sum_m w_m y[b,t,h,m,:]
//     out = r / max(|r|_2, 1e-6) * sqrt(V) * norm
//     [* silu(z[b,t,h,:]) with an output gate z: the layer's Qwen3.5 gate when
//      H V = D, i.e. no _agg_proj between the two (gdn3/gdn3_upgrade.py:861-871)]
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

// Destination buffers of the scattering routing (identical layouts, `a.out`'s strides).
struct PeerOuts {
  void* p[kMaxPeerOuts];
  int n;
};

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

// Eight consecutive elements as fp32 (16-byte aligned).
GDNX_DEV void ld8f(const void* p, int dtype, int64_t off, float* x) {
  if (dtype == GDNX_BF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + off);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
    return;
  }
  ld4f(p, dtype, off, x);
  ld4f(p, dtype, off + 4, x + 4);
}
GDNX_DEV void st8f(void* p, int dtype, int64_t off, const float* x) {
  if (dtype == GDNX_BF16) {  // one 16-byte store
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 t = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&t);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p) + off) = u;
    return;
  }
  st4f(p, dtype, off, x);
  st4f(p, dtype, off + 4, x + 4);
}
// Sum over the 16 lanes of a half warp.
GDNX_DEV float half_sum(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Lane routing: a half warp per row (8 channels per lane), two passes of two rows per
// warp with every load of both passes issued before the arithmetic.  bf16 scan outputs
// stay packed in registers until they are summed, so four CTAs fit on an SM (two with eight lanes).
// With SCAT the routed rows are stored to every buffer of `outs` (this GPU's and its peers'
// over NVLink: the routing fused with the all-gather of its output) instead of a.out, and
// each thread fences at system scope after its stores, so that once the kernel has
// completed its writes are visible to the peers.
template <int MT, bool BF16IN, bool GATE, bool SCAT>
__global__ void __launch_bounds__(NT, MT >= 8 ? 2 : 4) lane_route_kernel(const gdnx_epilogue_args a,
                                                                         const PeerOuts outs) {
  const int lane = threadIdx.x & 31, hw = lane >> 4, c = 8 * (lane & 15);
  const int64_t rows = a.B * a.T * a.H;
  const int64_t base = ((int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5)) * 4;
  const int V = (int)a.V;
  uint4 raw[2][MT];
  float lg[2][MT];
  int64_t rb[2], rt[2], rh[2];
  bool live[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t row = base + 2 * p + hw;
    live[p] = row < rows && c < V;
    {  // 32-bit index arithmetic (the launcher guarantees B*T*H < 2^31)
      const uint32_t r32 = (uint32_t)row, H32 = (uint32_t)a.H, T32 = (uint32_t)a.T;
      const uint32_t bt = r32 / H32;
      rh[p] = r32 - bt * H32;
      rb[p] = bt / T32;
      rt[p] = bt - (uint32_t)rb[p] * T32;
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      raw[p][m] = make_uint4(0u, 0u, 0u, 0u);
      lg[p][m] = m < a.M ? 0.f : -INFINITY;  // lanes past M get zero weight
      if (live[p] && m < a.M) {
        const int64_t off = rb[p] * a.y.sb + rt[p] * a.y.st + rh[p] * a.y.sh + m * a.y.sm + c;
        if (BF16IN) raw[p][m] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.y.ptr) + off);
        lg[p][m] = ld_as_f32(a.router.ptr, a.router.dtype,
                             rb[p] * a.router.sb + rt[p] * a.router.st + rh[p] * a.router.sh + m * a.router.sm);
      }
    }
  }
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float mx = lg[p][0];
#pragma unroll
    for (int m = 1; m < MT; ++m) mx = fmaxf(mx, lg[p][m]);
    float den = 0.f, w[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      w[m] = expf(lg[p][m] - mx);
      den += w[m];
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float wm = w[m] / den;
      float y[8];
      if (BF16IN) {
        const uint32_t u[4] = {raw[p][m].x, raw[p][m].y, raw[p][m].z, raw[p][m].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          y[2 * i] = __uint_as_float(u[i] << 16);
          y[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
        }
      } else if (live[p] && m < a.M) {
        ld8f(a.y.ptr, a.y.dtype, rb[p] * a.y.sb + rt[p] * a.y.st + rh[p] * a.y.sh + m * a.y.sm + c, y);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wm, y[e], acc[e]);
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(acc[e], acc[e], ss);
    ss = half_sum(ss);
    const float sc = sqrtf((float)V) / fmaxf(sqrtf(ss), 1e-6f);
    if (live[p]) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = acc[e] * sc * (a.weight ? a.weight[c + e] : 1.f);
      if (GATE) {
        float z[8];
        ld8f(a.gate.ptr, a.gate.dtype, rb[p] * a.gate.sb + rt[p] * a.gate.st + rh[p] * a.gate.sh + c, z);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= z[e] / (1.f + expf(-z[e]));
      }
      const int64_t oo = rb[p] * a.out_sb + rt[p] * a.out_st + rh[p] * a.out_sh + c;
      if (SCAT) {
#pragma unroll 1
        for (int d = 0; d < outs.n; ++d) st8f(outs.p[d], a.out_dtype, oo, o);
      } else {
        st8f(a.out, a.out_dtype, oo, o);
      }
    }
  }
  if (SCAT) __threadfence_system();
}

// Gated RMS norm: a half warp per row, four rows per warp, loads first.
__global__ void __launch_bounds__(NT, 4) rms_gated_kernel(const gdnx_epilogue_args a) {
  const int lane = threadIdx.x & 31, hw = lane >> 4, c = 8 * (lane & 15);
  const int64_t rows = a.B * a.T * a.H;
  const int64_t base = ((int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5)) * 4;
  const int V = (int)a.V;
  float y[2][8], z[2][8];
  int64_t rb[2], rt[2], rh[2];
  bool live[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t row = base + 2 * p + hw;
    live[p] = row < rows && c < V;
    {  // 32-bit index arithmetic (the launcher guarantees B*T*H < 2^31)
      const uint32_t r32 = (uint32_t)row, H32 = (uint32_t)a.H, T32 = (uint32_t)a.T;
      const uint32_t bt = r32 / H32;
      rh[p] = r32 - bt * H32;
      rb[p] = bt / T32;
      rt[p] = bt - (uint32_t)rb[p] * T32;
    }
    if (live[p]) {
      ld8f(a.y.ptr, a.y.dtype, rb[p] * a.y.sb + rt[p] * a.y.st + rh[p] * a.y.sh + c, y[p]);
      ld8f(a.gate.ptr, a.gate.dtype, rb[p] * a.gate.sb + rt[p] * a.gate.st + rh[p] * a.gate.sh + c, z[p]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) y[p][e] = z[p][e] = 0.f;
    }
  }
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(y[p][e], y[p][e], ss);
    ss = half_sum(ss);
    const float r = rsqrtf(ss / (float)V + a.eps);
    if (live[p]) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float sil = z[p][e] / (1.f + expf(-z[p][e]));
        o[e] = (a.weight ? a.weight[c + e] : 1.f) * (y[p][e] * r) * sil;
      }
      st8f(a.out, a.out_dtype, rb[p] * a.out_sb + rt[p] * a.out_st + rh[p] * a.out_sh + c, o);
    }
  }
}

template <bool GATE, bool SCAT>
void launch_route(const gdnx_epilogue_args& a, const PeerOuts& o, bool bf, int64_t blocks, cudaStream_t st) {
  if (a.M == 1) {
    if (bf) lane_route_kernel<1, true, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
    else lane_route_kernel<1, false, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
  } else if (a.M == 2) {
    if (bf) lane_route_kernel<2, true, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
    else lane_route_kernel<2, false, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
  } else if (a.M <= 4) {
    if (bf) lane_route_kernel<4, true, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
    else lane_route_kernel<4, false, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
  } else {
    if (bf) lane_route_kernel<8, true, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
    else lane_route_kernel<8, false, GATE, SCAT><<<(unsigned)blocks, NT, 0, st>>>(a, o);
  }
}

}  // namespace

gdnx_status launch_epilogue(const gdnx_epilogue_args& a, cudaStream_t st) {
  const int64_t rows = a.B * a.T * a.H;
  const int64_t per_block = 4 * (NT / 32);  // four rows per warp
  const int64_t blocks = (rows + per_block - 1) / per_block;
  if (rows >= int64_t(0x7fffffff)) return GDNX_EUNSUPPORTED;
  if (a.kind == GDNX_EPILOGUE_RMS_GATED) {
    rms_gated_kernel<<<(unsigned)blocks, NT, 0, st>>>(a);
  } else {
    const bool bf = a.y.dtype == GDNX_BF16;
    PeerOuts none{};
    if (a.gate.ptr) launch_route<true, false>(a, none, bf, blocks, st);
    else launch_route<false, false>(a, none, bf, blocks, st);
  }
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx

namespace gdnx {

gdnx_status launch_epilogue_scatter(const gdnx_epilogue_args& a, void* const* outs, int n, cudaStream_t st) {
  const int64_t rows = a.B * a.T * a.H;
  const int64_t blocks = (rows + 4 * (NT / 32) - 1) / (4 * (NT / 32));
  if (rows >= int64_t(0x7fffffff) || n < 1 || n > kMaxPeerOuts) return GDNX_EUNSUPPORTED;
  PeerOuts o{};
  for (int d = 0; d < n; ++d) o.p[d] = outs[d];
  o.n = n;
  const bool bf = a.y.dtype == GDNX_BF16;
  if (a.gate.ptr) launch_route<true, true>(a, o, bf, blocks, st);
  else launch_route<false, true>(a, o, bf, blocks, st);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
