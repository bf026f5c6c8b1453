// KMD-2 prologue: from the outputs of KMD2NativeAttn.forward's input GEMMs to the
// inputs of its scan (gdn3/kmd2_native.py:140-172), in two passes:
//
//   theta_cumsum_kernel  Theta[b,t,h,i] = sum_{s<=t} softplus(theta[b,s,h,i]) for the
//                        dk/2 rotation pairs of every head (one thread per (b, pair),
//                        left to right like torch.cumsum on the CPU; the loads of a run
//                        of tokens are issued before their sums)
//   kmd2_row_kernel      one warp per (b, t, h) row: depthwise causal conv + SiLU of the
//                        q|k|v channels, L2 normalisation (eps 1e-6) and the 1/sqrt(dk)
//                        query scale, beta_e / beta_w, the per-channel decay, the query
//                        slot scales, and the plane rotation of k and every slot by Theta
//
// Lane l owns channels l, l+32, l+64, l+96 of a 128-wide head, so both halves of its two
// rotation pairs (l, l+64) and (l+32, l+96) are in its own registers.  HBM-bound: every
// input is read once (the conv's previous tokens hit in L1/L2), every output written once.
#include "common.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int kDK = 128;
constexpr int kRun = 16;   // tokens whose loads are issued together in the cumulative sum
constexpr int NT = 128;    // four rows per CTA, a warp per row

GDNX_DEV float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void __launch_bounds__(128) theta_cumsum_kernel(const gdnx_kmd2_prologue_args a) {
  const int64_t pairs = a.H * (a.dk / 2);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= a.B * pairs) return;
  const int64_t b = idx / pairs, ch = idx % pairs;  // ch = h * dk/2 + i
  float acc = 0.f;
  for (int64_t t0 = 0; t0 < a.T; t0 += kRun) {
    float x[kRun];
#pragma unroll
    for (int j = 0; j < kRun; ++j)
      x[j] = (t0 + j < a.T) ? ld_as_f32(a.theta.ptr, a.theta.dtype, b * a.theta.sb + (t0 + j) * a.theta.st + ch) : 0.f;
#pragma unroll
    for (int j = 0; j < kRun; ++j) {
      if (t0 + j < a.T) {
        acc += softplus_f(x[j]);
        a.theta_ws[(b * a.T + t0 + j) * pairs + ch] = acc;
      }
    }
  }
}

__global__ void __launch_bounds__(NT) kmd2_row_kernel(const gdnx_kmd2_prologue_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (row >= a.B * a.T * a.H) return;
  const int64_t h = row % a.H, t = (row / a.H) % a.T, b = row / (a.H * a.T);
  const int64_t kd = a.H * kDK;  // key_dim
  const int K = a.conv_k;
  // every global load first: conv taps of the q, k, v channels, the gates, the angles
  float xq[4][8], xk[4][8], xv[4][8];  // [channel j][tap] (conv_k <= 8)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t cq = h * kDK + lane + 32 * j, ck = kd + cq, cv = 2 * kd + cq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xq[j][i] = xk[j][i] = xv[j][i] = 0.f;
      const int64_t ts = t - (K - 1) + i;
      if (i < K && ts >= 0) {
        const int64_t o = b * a.mixed.sb + ts * a.mixed.st;
        xq[j][i] = ld_as_f32(a.mixed.ptr, a.mixed.dtype, o + cq);
        xk[j][i] = ld_as_f32(a.mixed.ptr, a.mixed.dtype, o + ck);
        xv[j][i] = ld_as_f32(a.mixed.ptr, a.mixed.dtype, o + cv);
      }
    }
  }
  const float braw = ld_as_f32(a.b.ptr, a.b.dtype, b * a.b.sb + t * a.b.st + h);
  const float araw = ld_as_f32(a.a.ptr, a.a.dtype, b * a.a.sb + t * a.a.st + h);
  const float* th = a.theta_ws + ((b * a.T + t) * a.H + h) * (kDK / 2);
  const float th0 = th[lane], th1 = th[lane + 32];
  // conv + SiLU
  float q[4], k[4], v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t cq = h * kDK + lane + 32 * j, ck = kd + cq, cv = 2 * kd + cq;
    float sq = 0.f, sk = 0.f, sv = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < K) {
        sq = fmaf(a.conv_w[cq * K + i], xq[j][i], sq);
        sk = fmaf(a.conv_w[ck * K + i], xk[j][i], sk);
        sv = fmaf(a.conv_w[cv * K + i], xv[j][i], sv);
      }
    }
    q[j] = sq * sigmoidf_(sq);
    k[j] = sk * sigmoidf_(sk);
    v[j] = sv * sigmoidf_(sv);
  }
  // normalisation (F.normalize: x / max(|x|, eps)) and the query scale
  float nq = 0.f, nk = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    nq = fmaf(q[j], q[j], nq);
    nk = fmaf(k[j], k[j], nk);
  }
  nq = warp_sum(nq);
  nk = warp_sum(nk);
  const float dq = fmaxf(sqrtf(nq), 1e-6f), dkn = fmaxf(sqrtf(nk), 1e-6f);
  constexpr float kQScale = 0.08838834764831845f;  // dk^-0.5 for dk = 128, rounded to fp32 as torch does
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    q[j] = (q[j] / dq) * kQScale;
    k[j] = k[j] / dkn;
  }
  // rotation of the pairs (lane, lane+64) and (lane+32, lane+96)
  float s0, c0, s1, c1;
  sincosf(th0, &s0, &c0);
  sincosf(th1, &s1, &c1);
  const int64_t ro = (b * a.T + t) * a.H + h;
  {
    float* ko = a.k_out + ro * kDK;
    ko[lane] = k[0] * c0 - k[2] * s0;
    ko[lane + 64] = k[0] * s0 + k[2] * c0;
    ko[lane + 32] = k[1] * c1 - k[3] * s1;
    ko[lane + 96] = k[1] * s1 + k[3] * c1;
  }
  for (int r = 0; r < a.r_out; ++r) {
    float qs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      qs[j] = a.q_slot_scale ? q[j] * (1.f + a.q_slot_scale[(h * a.r_out + r) * kDK + lane + 32 * j]) : q[j];
    float* qo = a.q_out + (ro * a.r_out + r) * kDK;
    qo[lane] = qs[0] * c0 - qs[2] * s0;
    qo[lane + 64] = qs[0] * s0 + qs[2] * c0;
    qo[lane + 32] = qs[1] * c1 - qs[3] * s1;
    qo[lane + 96] = qs[1] * s1 + qs[3] * c1;
  }
  // values, decays, betas
  const float gh = -expf(a.A_log[h]) * softplus_f(araw + a.dt_bias[h]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane + 32 * j;
    a.v_out[ro * a.dv + c] = v[j];
    a.g_out[ro * kDK + c] = fminf(expf(gh + a.decay_chan[h * kDK + c]), 1.f);
  }
  if (lane == 0) {
    a.beta_e_out[ro] = sigmoidf_(braw);
    a.beta_w_out[ro] = sigmoidf_(braw + a.bw_off[h]);
  }
}

}  // namespace

gdnx_status launch_kmd2_prologue(const gdnx_kmd2_prologue_args& a, cudaStream_t st) {
  const int64_t cs = a.B * a.H * (a.dk / 2);
  const int64_t rows = a.B * a.T * a.H;
  if ((cs + 127) / 128 > int64_t(0x7fffffff) || (rows + NT / 32 - 1) / (NT / 32) > int64_t(0x7fffffff))
    return GDNX_EUNSUPPORTED;
  theta_cumsum_kernel<<<(unsigned)((cs + 127) / 128), 128, 0, st>>>(a);
  kmd2_row_kernel<<<(unsigned)((rows + NT / 32 - 1) / (NT / 32)), NT, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
