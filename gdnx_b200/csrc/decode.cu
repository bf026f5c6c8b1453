// Memory-bound single-token decode step for K = V = 128 dense states.
//
// One CTA of 8 warps owns one chain's 128 x 128 fp32 state (64 KB).  Warp w
// streams rows [16w, 16w+16): each lane loads one float4 of every row
// (coalesced 512-byte rows, evict-first), so a warp has 16 independent
// 128-bit loads in flight.  The 16 rows x 2 dot products (S h and S q) are
// reduced across the warp with a transpose-reduction (31 shuffles for all 32
// sums, lane l ends up holding sum l) instead of 32 separate butterflies.
// Each state element is read once and written once; q, k, v and the gates of
// the chain are a few hundred bytes next to the 64 KB state.
#include "common.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int kRowsPerWarp = 16;
constexpr int kWarps = 8;

template <int HALF>
GDNX_DEV void tr_stage(float* vals, int lane) {
  const bool up = (lane & HALF) != 0;
#pragma unroll
  for (int i = 0; i < HALF; ++i) {
    const float send = up ? vals[i] : vals[i + HALF];
    const float keep = up ? vals[i + HALF] : vals[i];
    vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, HALF);
  }
}

// 32 per-lane partial values -> lane l holds the warp total of value l.
GDNX_DEV float transpose_reduce32(float* vals, int lane) {
  tr_stage<16>(vals, lane);
  tr_stage<8>(vals, lane);
  tr_stage<4>(vals, lane);
  tr_stage<2>(vals, lane);
  tr_stage<1>(vals, lane);
  return vals[0];
}

struct DecParams {
  gdnx_decode_args a;
  int vec_e, vec_w, chan_decay, kmd2;
};

__global__ void __launch_bounds__(256) decode128_kernel(const DecParams P) {
  constexpr int K = 128, V = 128;
  __shared__ float stage[kWarps][2][K];
  const gdnx_decode_args& a = P.a;
  const int64_t n = blockIdx.x;
  const int64_t m = n % a.M;
  const int64_t h = (n / a.M) % a.H;
  const int64_t b = n / (a.M * a.H);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // ---- chain vectors: k, effective q (slots mixed), lane RoPE ----
  float* sk = stage[warp][0];
  float* sq = stage[warp][1];
  const int64_t ko = view_off(a.k, b, 0, h, m);
  for (int i = lane; i < K; i += 32) sk[i] = ld_as_f32(a.k.ptr, a.k.dtype, ko + i);
  for (int i = lane; i < K; i += 32) {
    float acc;
    if (a.r_out <= 1) {
      acc = ld_as_f32(a.q.ptr, a.q.dtype, view_off(a.q, b, 0, h, m) + i);
    } else {
      acc = 0.f;
      for (int r = 0; r < a.r_out; ++r)
        acc += a.out_mix[h * a.r_out + r] * ld_as_f32(a.q.ptr, a.q.dtype, view_off(a.q, b, 0, h, m, r) + i);
    }
    sq[i] = acc;
  }
  __syncwarp();
  rope_row_warp(sk, a.rope, (int)m, a.rope.pos0, lane);
  rope_row_warp(sq, a.rope, (int)m, a.rope.pos0, lane);
  __syncwarp();
  const int k0 = 4 * lane;
  float4 k4 = *reinterpret_cast<const float4*>(sk + k0);
  float4 q4 = *reinterpret_cast<const float4*>(sq + k0);
  float4 h4 = k4;
  const int64_t eo = a.gate_e.ptr ? view_off(a.gate_e, b, 0, h, m) : 0;
  const int64_t wo = a.gate_w.ptr ? view_off(a.gate_w, b, 0, h, m) : 0;
  if (P.vec_e) {
    h4.x *= ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo + k0 + 0);
    h4.y *= ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo + k0 + 1);
    h4.z *= ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo + k0 + 2);
    h4.w *= ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo + k0 + 3);
  }
  const float kh = warp_sum(k4.x * h4.x + k4.y * h4.y + k4.z * h4.z + k4.w * h4.w);
  const float kq = warp_sum(k4.x * q4.x + k4.y * q4.y + k4.z * q4.z + k4.w * q4.w);
  float ce, cw;
  if (P.kmd2) {
    ce = ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo);
    cw = ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo);
  } else {
    const float be = P.vec_e ? 1.f : ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo);
    const float bw = P.vec_w ? 1.f : ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo);
    const float al = stable_alpha(P.vec_e ? kh : be * kh);
    ce = al * be;
    cw = al * bw;
  }
  const int64_t dof = view_off(a.decay, b, 0, h, m);
  float gam = 1.f;
  float4 g4 = make_float4(1.f, 1.f, 1.f, 1.f);
  if (P.chan_decay) {
    float gg[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float g = ld_as_f32(a.decay.ptr, a.decay.dtype, dof + k0 + e);
      if (a.decay_kind == GDNX_DECAY_LOG) g = expf(g);
      if (!P.kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
      gg[e] = g;
    }
    g4 = make_float4(gg[0], gg[1], gg[2], gg[3]);
  } else {
    gam = decay_factor(a.decay, a.decay_kind, dof, !P.kmd2, a.braid_rates, a.braid_clamp);
  }

  // ---- stream the warp's 16 rows ----
  const int row0 = warp * kRowsPerWarp;
  float* Sbase = a.S + (n * V + row0) * K + k0;
  float4 S[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) S[r] = __ldcs(reinterpret_cast<const float4*>(Sbase + r * K));
  // write value for the row this lane will finalise (lanes 0..15)
  float u = 0.f;
  {
    const int rr = lane & 15;
    const int64_t vo = view_off(a.v, b, 0, h, m);
    u = ld_as_f32(a.v.ptr, a.v.dtype, vo + row0 + rr);
    if (P.vec_w) u *= ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo + row0 + rr);
  }
  float vals[32];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    float4 s = S[r];
    if (P.chan_decay) {
      s.x *= g4.x; s.y *= g4.y; s.z *= g4.z; s.w *= g4.w;
      S[r] = s;
    }
    vals[r] = s.x * h4.x + s.y * h4.y + s.z * h4.z + s.w * h4.w;
    vals[r + 16] = s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w;
  }
  const float tot = transpose_reduce32(vals, lane);
  // lane l < 16: tot = (S h)_row(l); lane l >= 16: tot = (S q)_row(l-16)
  const float d_own = cw * u - ce * (gam * tot);
  const float d_row = __shfl_sync(0xffffffffu, d_own, lane & 15);
  if (lane >= 16) {
    const float y = fmaf(d_row, kq, gam * tot);
    const int64_t yo = b * a.y_sb + h * a.y_sh + m * a.y_sm + row0 + (lane - 16);
    st_from_f32(a.y, a.y_dtype, yo, y);
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float d = __shfl_sync(0xffffffffu, d_own, r);
    float4 s = S[r];
    s.x = fmaf(gam, s.x, d * k4.x);
    s.y = fmaf(gam, s.y, d * k4.y);
    s.z = fmaf(gam, s.z, d * k4.z);
    s.w = fmaf(gam, s.w, d * k4.w);
    __stcs(reinterpret_cast<float4*>(Sbase + r * K), s);
  }
}

}  // namespace

gdnx_status launch_decode_128(const gdnx_decode_args& a, cudaStream_t st) {
  DecParams P;
  P.a = a;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.vec_e = !P.kmd2 && a.gate_e.dim > 1;
  P.vec_w = !P.kmd2 && a.gate_w.dim > 1;
  P.chan_decay = a.decay.dim == a.K && a.decay_kind != GDNX_DECAY_BRAIDED;
  const int64_t N = a.B * a.H * a.M;
  if (N == 0) return GDNX_OK;
  decode128_kernel<<<(unsigned)N, 256, 0, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
