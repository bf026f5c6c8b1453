// Exact token-recurrent dense scan (CUDA cores, fp32 state and math).
//
// One CTA owns one chain.  Thread (v, j) keeps row v of the V x K state in
// registers (TPR threads per row, interleaved float4 key chunks so the two
// threads of a row hit different shared-memory banks).  Inputs are staged TB
// tokens at a time into shared memory by the warps (gates, lane RoPE, alpha,
// decay and the k.q products are computed there, once per token), after which
// every thread runs the TB token updates on its own row with no further
// synchronisation:
//     dh = g (S h), dq = g (S q)          (row dot products)
//     d  = cw u_v - ce dh                 (delta-rule update coefficient)
//     y  = dq + d (k.q)                   (read of the post-update state)
//     S  = g S + d k^T
// GDN3:  ce = alpha * b, cw = alpha * w  (scalar gates) -- the loop body of
//        gdn3/_reference_recurrence.py:61-84 with the Kronecker part zero.
// KMD-2: ce = beta_e, cw = beta_w, per-channel decay applied to the state
//        columns first -- research/kernel_ab/ref_scan.py:40-47.
// With r_out > 1 query slots, y = sum_r mix_r (q_r . S) = (sum_r mix_r q_r) . S,
// so the slots are mixed into one effective query during staging.
#include "common.cuh"
#include "kernels.h"

namespace gdnx {

namespace {

constexpr int kTB = 16;  // tokens staged per block

struct RecParams {
  gdnx_scan_args a;
  int vec_e, vec_w, chan_decay, want_scores, kmd2;
};

template <int K, int V>
struct RecSmem {
  // floats per staged token
  static constexpr int kK = 0;             // k
  static constexpr int kH = K;             // h = b (.) k (vector erase gate only)
  static constexpr int kQ = 2 * K;         // effective query
  static constexpr int kD = 3 * K;         // per-channel decay
  static constexpr int kU = 4 * K;         // u = w (.) v  (or v)
  static constexpr int kS = 4 * K + V;     // scalars: gam, ce, cw, kq, |k|
  static constexpr int kPer = 4 * K + V + 8;
  static constexpr int kTok = kTB * kPer;  // staged block
  static constexpr int kOut = 2 * kTB * V; // y and d buffers
  static constexpr int kFloats = kTok + kOut;
};

// Two CTAs per SM at K = 128 (the row state alone is 64 registers a thread).
template <int K, int V, int TPR>
__global__ void __launch_bounds__(V * TPR, K >= 128 ? 2 : 1)
recurrent_scan_kernel(const RecParams P) {
  using SM = RecSmem<K, V>;
  constexpr int NT = V * TPR;
  constexpr int NW = NT / 32;
  constexpr int KC = K / 4 / TPR;  // float4 chunks per thread
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  float* ybuf = sm + SM::kTok;
  float* dbuf = ybuf + kTB * V;

  const gdnx_scan_args& a = P.a;
  const int64_t n = blockIdx.x;
  const int64_t m = n % a.M;
  const int64_t h = (n / a.M) % a.H;
  const int64_t b = n / (a.M * a.H);
  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int v = tid / TPR, j = tid % TPR;

  float4 S[KC];
  if (a.state_in) {
    const float* s0 = a.state_in + (n * V + v) * K;
#pragma unroll
    for (int c = 0; c < KC; ++c) S[c] = *reinterpret_cast<const float4*>(s0 + 4 * (c * TPR + j));
  } else {
#pragma unroll
    for (int c = 0; c < KC; ++c) S[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  for (int64_t t0 = 0; t0 < a.T; t0 += kTB) {
    const int nt = (int)((a.T - t0) < kTB ? (a.T - t0) : kTB);
    // ---------------- stage nt tokens (one warp per token) ----------------
    // Every global load of a token is issued before any of them is used, so a staged token
    // costs about one memory round trip instead of one per loop iteration.
    for (int tt = warp; tt < nt; tt += NW) {
      const int64_t t = t0 + tt;
      float* tok = sm + tt * SM::kPer;
      float* sk = tok + SM::kK;
      float* sq = tok + SM::kQ;
      constexpr int KL = (K + 31) / 32, VL = (V + 31) / 32;
      const int64_t ko = view_off(a.k, b, t, h, m);
      const int64_t qo = view_off(a.q, b, t, h, m);
      const int64_t eo = a.gate_e.ptr ? view_off(a.gate_e, b, t, h, m) : 0;
      const int64_t vo = view_off(a.v, b, t, h, m);
      const int64_t wo = a.gate_w.ptr ? view_off(a.gate_w, b, t, h, m) : 0;
      const int64_t dof = view_off(a.decay, b, t, h, m);
      float rk[KL], rq[KL], re[KL], rd[KL], rv[VL], rw[VL];
#pragma unroll
      for (int c = 0; c < KL; ++c) {
        const int i = lane + 32 * c;
        rk[c] = rq[c] = re[c] = rd[c] = 0.f;
        if (i < K) {
          rk[c] = ld_as_f32(a.k.ptr, a.k.dtype, ko + i);
          if (a.r_out <= 1) rq[c] = ld_as_f32(a.q.ptr, a.q.dtype, qo + i);
          if (P.vec_e) re[c] = ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo + i);
          if (P.chan_decay) rd[c] = ld_as_f32(a.decay.ptr, a.decay.dtype, dof + i);
        }
      }
#pragma unroll
      for (int c = 0; c < VL; ++c) {
        const int i = lane + 32 * c;
        rv[c] = 0.f;
        rw[c] = 1.f;
        if (i < V) {
          rv[c] = ld_as_f32(a.v.ptr, a.v.dtype, vo + i);
          if (P.vec_w) rw[c] = ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo + i);
        }
      }
      // scalar gates (every lane loads them: uniform, and in flight with the rows above)
      const bool sc_e = P.kmd2 || !P.vec_e, sc_w = P.kmd2 || !P.vec_w;
      const float ge = sc_e ? ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo) : 1.f;
      const float gw = sc_w ? ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo) : 1.f;
      const float gam = P.chan_decay ? 1.0f
                                     : decay_factor(a.decay, a.decay_kind, dof, !P.kmd2, a.braid_rates, a.braid_clamp);
#pragma unroll
      for (int c = 0; c < KL; ++c) {
        const int i = lane + 32 * c;
        if (i < K) {
          sk[i] = rk[c];
          if (a.r_out <= 1) sq[i] = rq[c];
        }
      }
      if (a.r_out > 1) {
        for (int i = lane; i < K; i += 32) {
          float acc = 0.f;
          for (int r = 0; r < a.r_out; ++r)
            acc += a.out_mix[h * a.r_out + r] *
                   ld_as_f32(a.q.ptr, a.q.dtype, view_off(a.q, b, t, h, m, r) + i);
          sq[i] = acc;
        }
      }
      __syncwarp();
      rope_row_warp(sk, a.rope, (int)m, a.rope.pos0 + t, lane);
      rope_row_warp(sq, a.rope, (int)m, a.rope.pos0 + t, lane);
      __syncwarp();
      // erase key, dots
      float kh = 0.f, kq = 0.f, kk = 0.f;
#pragma unroll
      for (int c = 0; c < KL; ++c) {
        const int i = lane + 32 * c;
        if (i < K) {
          const float kv = sk[i];
          float hv = kv;
          if (P.vec_e) {
            hv = re[c] * kv;
            tok[SM::kH + i] = hv;
          }
          kh += kv * hv;
          kq += kv * sq[i];
          kk += kv * kv;
        }
      }
      kh = warp_sum(kh);
      kq = warp_sum(kq);
      kk = warp_sum(kk);
      // write value
#pragma unroll
      for (int c = 0; c < VL; ++c) {
        const int i = lane + 32 * c;
        if (i < V) tok[SM::kU + i] = P.vec_w ? rv[c] * rw[c] : rv[c];
      }
      // per-channel decay
      if (P.chan_decay) {
#pragma unroll
        for (int c = 0; c < KL; ++c) {
          const int i = lane + 32 * c;
          if (i < K) {
            float g = rd[c];
            if (a.decay_kind == GDNX_DECAY_LOG) g = expf(g);
            if (!P.kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
            tok[SM::kD + i] = g;
          }
        }
      }
      if (lane == 0) {
        float ce, cw;
        if (P.kmd2) {
          ce = ge;
          cw = gw;
        } else {
          const float be = P.vec_e ? 1.f : ge;
          const float bw = P.vec_w ? 1.f : gw;
          const float c = P.vec_e ? kh : be * kh;   // k . h
          const float al = stable_alpha(c);
          ce = al * be;
          cw = al * bw;
        }
        float* sc = tok + SM::kS;
        sc[0] = gam; sc[1] = ce; sc[2] = cw; sc[3] = kq; sc[4] = sqrtf(kk);
      }
    }
    __syncthreads();
    // ---------------- nt sequential token updates ----------------
    for (int tt = 0; tt < nt; ++tt) {
      const float* tok = sm + tt * SM::kPer;
      const float* kr = tok + SM::kK;
      const float* hr = P.vec_e ? tok + SM::kH : kr;
      const float* qr = tok + SM::kQ;
      const float* sc = tok + SM::kS;
      if (P.chan_decay) {
        const float* dr = tok + SM::kD;
#pragma unroll
        for (int c = 0; c < KC; ++c) {
          const float4 g4 = *reinterpret_cast<const float4*>(dr + 4 * (c * TPR + j));
          S[c].x *= g4.x; S[c].y *= g4.y; S[c].z *= g4.z; S[c].w *= g4.w;
        }
      }
      float dh = 0.f, dq = 0.f;
#pragma unroll
      for (int c = 0; c < KC; ++c) {
        const int kk = 4 * (c * TPR + j);
        const float4 h4 = *reinterpret_cast<const float4*>(hr + kk);
        const float4 q4 = *reinterpret_cast<const float4*>(qr + kk);
        dh = fmaf(S[c].x, h4.x, dh); dh = fmaf(S[c].y, h4.y, dh);
        dh = fmaf(S[c].z, h4.z, dh); dh = fmaf(S[c].w, h4.w, dh);
        dq = fmaf(S[c].x, q4.x, dq); dq = fmaf(S[c].y, q4.y, dq);
        dq = fmaf(S[c].z, q4.z, dq); dq = fmaf(S[c].w, q4.w, dq);
      }
      if (TPR == 2) {
        dh += __shfl_xor_sync(0xffffffffu, dh, 1);
        dq += __shfl_xor_sync(0xffffffffu, dq, 1);
      }
      const float gam = sc[0];
      dh *= gam;
      dq *= gam;
      const float d = sc[2] * tok[SM::kU + v] - sc[1] * dh;
      const float y = fmaf(d, sc[3], dq);
#pragma unroll
      for (int c = 0; c < KC; ++c) {
        const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * (c * TPR + j));
        S[c].x = fmaf(gam, S[c].x, d * k4.x);
        S[c].y = fmaf(gam, S[c].y, d * k4.y);
        S[c].z = fmaf(gam, S[c].z, d * k4.z);
        S[c].w = fmaf(gam, S[c].w, d * k4.w);
      }
      if (j == 0) {
        ybuf[tt * V + v] = y;
        dbuf[tt * V + v] = d;
      }
    }
    __syncthreads();
    // ---------------- flush outputs ----------------
    {
      char* yb = reinterpret_cast<char*>(a.y);
      const int esz = a.y_dtype == GDNX_F32 ? 4 : 2;
      for (int idx = tid; idx < nt * V; idx += NT) {
        const int tt = idx / V, vv = idx % V;
        const int64_t off = b * a.y_sb + (t0 + tt) * a.y_st + h * a.y_sh + m * a.y_sm + vv;
        st_from_f32(yb, a.y_dtype, off, ybuf[idx]);
        (void)esz;
      }
      if (P.want_scores) {
        for (int tt = warp; tt < nt; tt += NW) {
          float s2 = 0.f;
          for (int i = lane; i < V; i += 32) s2 += dbuf[tt * V + i] * dbuf[tt * V + i];
          s2 = warp_sum(s2);
          if (lane == 0) {
            const float kn = sm[tt * SM::kPer + SM::kS + 4];
            a.scores[((b * a.T + t0 + tt) * a.H + h) * a.M + m] = kn * sqrtf(s2);
          }
        }
      }
    }
  }
  if (a.state_out) {
    float* s1 = a.state_out + (n * V + v) * K;
#pragma unroll
    for (int c = 0; c < KC; ++c) *reinterpret_cast<float4*>(s1 + 4 * (c * TPR + j)) = S[c];
  }
}

template <int K, int V, int TPR>
gdnx_status launch(const RecParams& P, cudaStream_t st) {
  constexpr int NT = V * TPR;
  const size_t smem = RecSmem<K, V>::kFloats * sizeof(float);
  auto kfn = recurrent_scan_kernel<K, V, TPR>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return GDNX_ELAUNCH;
  const int64_t N = P.a.B * P.a.H * P.a.M;
  kfn<<<(unsigned)N, NT, smem, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace

gdnx_status launch_recurrent_scan(const gdnx_scan_args& a, cudaStream_t st) {
  RecParams P;
  P.a = a;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.vec_e = !P.kmd2 && a.gate_e.dim > 1;
  P.vec_w = !P.kmd2 && a.gate_w.dim > 1;
  P.chan_decay = a.decay.dim == a.K && a.decay_kind != GDNX_DECAY_BRAIDED && a.K > 1;
  P.want_scores = a.scores != nullptr;
  if (a.K != a.V) return GDNX_EUNSUPPORTED;
  switch (a.K) {
    case 32: return launch<32, 32, 1>(P, st);
    case 64: return launch<64, 64, 1>(P, st);
    case 128: return launch<128, 128, 2>(P, st);
    default: return GDNX_EUNSUPPORTED;
  }
}

}  // namespace gdnx
