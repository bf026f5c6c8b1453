// Backward of the dense gated delta-rule scan (GDN3 with compaction off, KMD-2):
// exact fp32 reverse-mode through the token recurrence, one CTA of 512 threads per
// chain, the 128 x 128 state and its gradient held in registers (row v over four
// threads, 32 columns each).
//
// Forward step, per token (gdn3/_reference_recurrence.py:61-84 with A = 0;
// research/kernel_ab/ref_scan.py:40-47):
//   P = S_{t-1} diag(G_t)          (G_t = gamma_t 1 for GDN3, the channel decays g_t for KMD-2)
//   m = P h_t;  d = cw_t u_t - ce_t m;  S_t = P + d k_t^T;  y_t = S_t q_t
// Reverse step, with dS the gradient of S_t (dy folded in first):
//   dS += dy q^T;  dq = S_t^T dy;  dd = dS k;  dk += dS^T d;  du = cw dd;
//   dcw = dd.u;  dce = -dd.m;  dh = -ce P^T dd;  dP = dS - ce dd h^T;
//   dG = colsum(dP (.) S_{t-1});  dS_{t-1} = dP diag(G)
// and the chain rule through the gates: GDN3 h = b (.) k, u = w (.) v,
// ce = cw = alpha(k.h) (gdn3/gdn3_upgrade.py:641-648); KMD-2 h = k, ce = beta_e,
// cw = beta_w, q = sum_r out_mix_r q_r (gdn3/kmd2_fast_scan.py:143-160 is the
// reference's backward of the same map, through its chunked TRSM).
//
// States are recomputed, not stored per token: a first sweep writes the state at
// every 64-token block start; the reverse sweep, per block, recomputes the eight
// 8-token sub-block starts, then per sub-block the eight token states (an L2-resident
// ring of nine 64 KB states per chain), and runs the reverse steps over them.
#include "common.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int NT = 512;
constexpr int KD = 128, VD = 128;
constexpr int BLK = 64, SUB = 8;
constexpr int NW = NT / 32;
constexpr size_t STATE = (size_t)VD * KD;  // floats

struct BwdParams {
  gdnx_scan_bwd_args a;
  int kmd2, vec_e, vec_w, chan_decay;
  int prefetch;  // rows 4-element aligned: the next staging's rows go by cp.async (see stage())
  int64_t nblk;
  float* ckpt;   // [N][nblk][V][K]
  float* sub;    // [N][8][V][K]
  float* ring;   // [N][9][V][K]
};

// Per-token vectors staged in shared memory for one 8-token sub-block.
constexpr int MAXR = 4;  // query slots staged for the out_mix gradient (more are read from global)
struct Tok {
  float q[KD], k[KD], h[KD], u[VD], G[KD], dy[VD], b[KD], w[VD], v[VD];
  float qs[MAXR][KD];
  float ce, cw, kh, pad;
};

GDNX_DEV float rowsum4(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

// d alpha / d c for alpha(c) = (1 - e^-c) / c (the reference's Taylor branch below 1e-6).
GDNX_DEV float alpha_grad(float c) {
  if (fabsf(c) < 1e-6f) return -0.5f + c * (1.0f / 3.0f);
  const float e = expf(-c);
  return (e * (c + 1.f) - 1.f) / (c * c);
}

// Decay factor and d factor / d raw for one decay element.
GDNX_DEV void decay_factor_grad(float raw, int kind, bool kmd2, float* f, float* df) {
  if (kind == GDNX_DECAY_LOG) {
    const float g = kmd2 ? raw : fminf(raw, 0.f);
    *f = expf(g);
    *df = (kmd2 || raw <= 0.f) ? *f : 0.f;
  } else {
    *f = kmd2 ? raw : fminf(fmaxf(raw, 0.f), 1.f);
    *df = (kmd2 || (raw >= 0.f && raw <= 1.f)) ? 1.f : 0.f;
  }
}

// Raw rows of one staged token, fetched ahead with cp.async: query slots 0-3, k, v, vector erase
// gate, vector write gate, per-channel decay, dy (128 elements of up to 4 bytes each).
constexpr int RAWROW = 512, RAW_Q = 0, RAW_K = 4, RAW_V = 5, RAW_B = 6, RAW_W = 7, RAW_D = 8, RAW_DY = 9,
              RAWROWS = 10, RAWTOK = RAWROWS * RAWROW;

// The stagings of one chain, in the order the kernel runs them (index k): the forward sweep's
// full sub-blocks, then per block from the last one down the sub-block start states (no dy)
// and the sub-blocks in reverse (with dy).
struct StageCall {
  int64_t t0;
  int nt, dy;
};
GDNX_DEV int64_t stage_calls(const BwdParams& P) {
  const int64_t T = P.a.fwd.T, nb_last = T - (P.nblk - 1) * BLK, ns_last = (nb_last + SUB - 1) / SUB;
  return (P.nblk - 1) * (BLK / SUB) + (2 * ns_last - 1) + (P.nblk - 1) * (2 * (BLK / SUB) - 1);
}
GDNX_DEV StageCall stage_call(const BwdParams& P, int64_t k) {
  const int64_t T = P.a.fwd.T, F = (P.nblk - 1) * (BLK / SUB);
  if (k < F) return {k * SUB, SUB, 0};
  k -= F;
  const int64_t nb_last = T - (P.nblk - 1) * BLK, ns_last = (nb_last + SUB - 1) / SUB, c0 = 2 * ns_last - 1;
  int64_t blk, j, nsub;
  if (k < c0) {
    blk = P.nblk - 1;
    j = k;
    nsub = ns_last;
  } else {
    k -= c0;
    blk = P.nblk - 2 - k / (2 * (BLK / SUB) - 1);
    j = k % (2 * (BLK / SUB) - 1);
    nsub = BLK / SUB;
  }
  const int64_t tb = blk * BLK;
  if (j < nsub - 1) return {tb + SUB * j, SUB, 0};
  const int64_t sb = nsub - 1 - (j - (nsub - 1)), t0 = tb + SUB * sb;
  return {t0, (int)((T - t0) < SUB ? (T - t0) : SUB), 1};
}
GDNX_DEV float raw_elem(const uint8_t* row, int dt, int i) {
  if (dt == GDNX_F32) return reinterpret_cast<const float*>(row)[i];
  if (dt == GDNX_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[i]);
  return __half2float(reinterpret_cast<const __half*>(row)[i]);
}
// Scalars of the staged token (fetched with the rows, into registers).
struct RawScal {
  float be, bw, sg;
};
// Warp `warp` fetches its token of staging k into raw buffer k & 1 (nothing past the last staging).
GDNX_DEV void prefetch(const BwdParams& P, uint8_t* raw, int64_t k, int64_t b, int64_t h, int64_t m, int warp,
                       int lane, RawScal& sc) {
  const gdnx_scan_args& a = P.a.fwd;
  if (k >= stage_calls(P)) return;
  const StageCall c = stage_call(P, k);
  if (warp >= c.nt) return;
  const int64_t t = c.t0 + warp;
  uint8_t* rt = raw + ((k & 1) * SUB + warp) * RAWTOK;
  auto cp_row = [&](int r, const gdnx_view& vw, int64_t off) {  // this lane's 4 elements
    const int es = vw.dtype == GDNX_F32 ? 4 : 2;
    const char* src = reinterpret_cast<const char*>(vw.ptr) + (off + 4 * lane) * es;
    const uint32_t dst = (uint32_t)__cvta_generic_to_shared(rt + r * RAWROW + 4 * es * lane);
    if (es == 4)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    else
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
  };
  const int rs = a.r_out <= 1 ? 1 : (a.r_out < MAXR ? a.r_out : MAXR);
  for (int r = 0; r < rs; ++r) cp_row(RAW_Q + r, a.q, view_off(a.q, b, t, h, m, r));
  cp_row(RAW_K, a.k, view_off(a.k, b, t, h, m));
  cp_row(RAW_V, a.v, view_off(a.v, b, t, h, m));
  if (P.vec_e) cp_row(RAW_B, a.gate_e, view_off(a.gate_e, b, t, h, m));
  if (P.vec_w) cp_row(RAW_W, a.gate_w, view_off(a.gate_w, b, t, h, m));
  if (P.chan_decay) cp_row(RAW_D, a.decay, view_off(a.decay, b, t, h, m));
  if (c.dy) cp_row(RAW_DY, P.a.dy, view_off(P.a.dy, b, t, h, m));
  asm volatile("cp.async.commit_group;" ::: "memory");
  sc.be = P.vec_e ? 0.f : ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m));
  sc.bw = P.vec_w ? 0.f : ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m));
  sc.sg = P.chan_decay ? 0.f : ld_as_f32(a.decay.ptr, a.decay.dtype, view_off(a.decay, b, t, h, m));
}

// Stage tokens t0 .. t0 + nt - 1 (nt <= SUB) of chain (b, h, m): warp j < nt takes token j,
// lane l channels l, l + 32, l + 64, l + 96.  With P.prefetch this is staging k: its rows are
// already in raw buffer k & 1 (fetched by the same warp during staging k - 1), and staging
// k + 1's rows are fetched into the other buffer before this one is converted.
GDNX_DEV void stage(const BwdParams& P, Tok* tk, float* graw, int64_t b, int64_t h, int64_t m, int64_t t0, int nt,
                    int warp, int lane, bool with_dy, uint8_t* raw, int64_t k, RawScal& sc) {
  const gdnx_scan_args& a = P.a.fwd;
  RawScal cur = sc;
  const uint8_t* rt = raw + ((k & 1) * SUB + warp) * RAWTOK;
  if (P.prefetch) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
    prefetch(P, raw, k + 1, b, h, m, warp, lane, sc);
  }
  if (warp >= nt) return;
  const int64_t t = t0 + warp;
  Tok& T = tk[warp];
  float kh = 0.f;
  const float be = P.vec_e ? 0.f : (P.prefetch ? cur.be : ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m)));
  const float bw = P.vec_w ? 0.f : (P.prefetch ? cur.bw : ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m)));
  const float sg = P.chan_decay ? 0.f : (P.prefetch ? cur.sg : ld_as_f32(a.decay.ptr, a.decay.dtype, view_off(a.decay, b, t, h, m)));
  // every global load first (four channels per lane), then the shared-memory writes: the
  // stores go through a generic reference, so loads issued after them would be serialised
  float qv[4] = {0.f, 0.f, 0.f, 0.f}, qsv[MAXR][4], kv[4], vv[4], bvv[4], wvv[4], rv[4], dyv[4];
  const int rs = a.r_out <= 1 ? 1 : (a.r_out < MAXR ? a.r_out : MAXR);
  if (P.prefetch) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane + 32 * i;
#pragma unroll
      for (int r = 0; r < MAXR; ++r) qsv[r][i] = r < rs ? raw_elem(rt + (RAW_Q + r) * RAWROW, a.q.dtype, c) : 0.f;
      kv[i] = raw_elem(rt + RAW_K * RAWROW, a.k.dtype, c);
      vv[i] = raw_elem(rt + RAW_V * RAWROW, a.v.dtype, c);
      bvv[i] = P.vec_e ? raw_elem(rt + RAW_B * RAWROW, a.gate_e.dtype, c) : be;
      wvv[i] = P.vec_w ? raw_elem(rt + RAW_W * RAWROW, a.gate_w.dtype, c) : bw;
      rv[i] = P.chan_decay ? raw_elem(rt + RAW_D * RAWROW, a.decay.dtype, c) : sg;
      dyv[i] = with_dy ? raw_elem(rt + RAW_DY * RAWROW, P.a.dy.dtype, c) : 0.f;
    }
  } else
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
#pragma unroll
    for (int r = 0; r < MAXR; ++r)
      qsv[r][i] = r < rs ? ld_as_f32(a.q.ptr, a.q.dtype, view_off(a.q, b, t, h, m, r) + c) : 0.f;
    kv[i] = ld_as_f32(a.k.ptr, a.k.dtype, view_off(a.k, b, t, h, m) + c);
    vv[i] = ld_as_f32(a.v.ptr, a.v.dtype, view_off(a.v, b, t, h, m) + c);
    bvv[i] = P.vec_e ? ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m) + c) : be;
    wvv[i] = P.vec_w ? ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m) + c) : bw;
    rv[i] = P.chan_decay ? ld_as_f32(a.decay.ptr, a.decay.dtype, view_off(a.decay, b, t, h, m) + c) : sg;
    dyv[i] = with_dy ? ld_as_f32(P.a.dy.ptr, P.a.dy.dtype, view_off(P.a.dy, b, t, h, m) + c) : 0.f;
  }
  if (a.r_out <= 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] = qsv[0][i];
  } else {
    for (int r = 0; r < a.r_out; ++r) {
      const float mix = a.out_mix[h * a.r_out + r];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qr = r < MAXR ? qsv[r < MAXR ? r : 0][i]
                                  : ld_as_f32(a.q.ptr, a.q.dtype, view_off(a.q, b, t, h, m, r) + lane + 32 * i);
        qv[i] = fmaf(mix, qr, qv[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    float f, df;
    decay_factor_grad(rv[i], a.decay_kind, P.kmd2 != 0, &f, &df);
    const float hv = P.kmd2 ? kv[i] : bvv[i] * kv[i];
    T.q[c] = qv[i];
#pragma unroll
    for (int r = 0; r < MAXR; ++r) T.qs[r][c] = qsv[r][i];
    T.k[c] = kv[i];
    T.h[c] = hv;
    T.b[c] = bvv[i];
    T.w[c] = wvv[i];
    T.v[c] = vv[i];
    T.u[c] = P.kmd2 ? vv[i] : wvv[i] * vv[i];
    T.G[c] = f;
    graw[warp * KD + c] = df;
    T.dy[c] = dyv[i];
    kh = fmaf(kv[i], hv, kh);
  }
  kh = warp_sum(kh);
  if (lane == 0) {
    T.kh = kh;
    if (P.kmd2) {
      T.ce = be;
      T.cw = bw;
    } else {
      T.ce = T.cw = stable_alpha(kh);
    }
  }
}

// A thread owns row v and the 32 columns 16 i + 4 qd + e (i < 8, e < 4) -- interleaved
// 4-column groups, so the four threads of a row read shared vectors conflict-free.
GDNX_DEV int colof(int qd, int i) { return 16 * i + 4 * qd; }

GDNX_DEV void fwd_step(float* S, const Tok& T, int v, int qd) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = colof(qd, i);
    const float4 g = *reinterpret_cast<const float4*>(T.G + c);
    const float4 hh = *reinterpret_cast<const float4*>(T.h + c);
    S[4 * i] *= g.x; S[4 * i + 1] *= g.y; S[4 * i + 2] *= g.z; S[4 * i + 3] *= g.w;
    m = fmaf(S[4 * i], hh.x, m);
    m = fmaf(S[4 * i + 1], hh.y, m);
    m = fmaf(S[4 * i + 2], hh.z, m);
    m = fmaf(S[4 * i + 3], hh.w, m);
  }
  m = rowsum4(m);
  const float d = T.cw * T.u[v] - T.ce * m;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 kk = *reinterpret_cast<const float4*>(T.k + colof(qd, i));
    S[4 * i] = fmaf(d, kk.x, S[4 * i]);
    S[4 * i + 1] = fmaf(d, kk.y, S[4 * i + 1]);
    S[4 * i + 2] = fmaf(d, kk.z, S[4 * i + 2]);
    S[4 * i + 3] = fmaf(d, kk.w, S[4 * i + 3]);
  }
}

GDNX_DEV void ld_state(const float* base, int v, int qd, float* S) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = *reinterpret_cast<const float4*>(base + (size_t)v * KD + colof(qd, i));
    S[4 * i] = f.x; S[4 * i + 1] = f.y; S[4 * i + 2] = f.z; S[4 * i + 3] = f.w;
  }
}
GDNX_DEV void st_state(float* base, int v, int qd, const float* S) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<float4*>(base + (size_t)v * KD + colof(qd, i)) =
        make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
}

// Reduce a 32-value column partial over the eight rows of a warp (lane bits 2-4) by
// halving exchanges (28 shuffles); the lane ends with four consecutive columns, which
// it stores to red[col .. col + 3].
template <int O>
GDNX_DEV void halve(float* a, int lane) {
  const bool up = (lane & O) != 0;
#pragma unroll
  for (int e = 0; e < O; ++e) {
    const float send = up ? a[e] : a[e + O];
    const float keep = up ? a[e + O] : a[e];
    a[e] = keep + __shfl_xor_sync(0xffffffffu, send, O);
  }
}
GDNX_DEV void colreduce_store(float* a, float* red, int lane, int qd) {
  halve<16>(a, lane);
  halve<8>(a, lane);
  halve<4>(a, lane);
  const int i = 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
  *reinterpret_cast<float4*>(red + colof(qd, i)) = make_float4(a[0], a[1], a[2], a[3]);
}

// Gradients of one token's inputs from the reduced vectors: warps 0-3 write the
// per-channel outputs (channel = tid), warps 4-7 the per-token scalars.
GDNX_DEV void write_token_grads(const BwdParams& P, const Tok& T, const float (*gv)[KD], const float* dd,
                                const float* graw, float dcw, float dce, int64_t ct, int64_t b, int64_t t,
                                int64_t h, int64_t m, int tid, int warp, int lane) {
  const gdnx_scan_bwd_args& A = P.a;
  const gdnx_scan_args& a = A.fwd;
  const bool kmd2 = P.kmd2 != 0;
  const int de = a.gate_e.dim, dw = a.gate_w.dim, ddim = a.decay.dim;
  // GDN3: ce = cw = alpha(k.h), so d alpha = dce + dcw and dc = d alpha alpha'(k.h)
  const float dc = kmd2 ? 0.f : (dce + dcw) * alpha_grad(T.kh);
  if (warp < 4) {
    const int c = tid;
    const float gq = gv[0][c], gk1 = gv[1][c], gh = gv[2][c], gG = gv[3][c];
    const float k = T.k[c];
    const float dht = gh + dc * k;  // d/dh including alpha's dependence on k.h
    const float dk = kmd2 ? gk1 + gh : gk1 + dc * T.h[c] + T.b[c] * dht;
    const float du = T.cw * dd[c];
    const float dv = kmd2 ? du : T.w[c] * du;
    A.dk[ct * KD + c] = dk;
    A.dv[ct * VD + c] = dv;
    if (a.r_out <= 1) {
      A.dq[ct * KD + c] = gq;
    } else {
      for (int r = 0; r < a.r_out; ++r) A.dq[(ct * a.r_out + r) * KD + c] = a.out_mix[h * a.r_out + r] * gq;
    }
    if (!kmd2 && de != 1) A.dgate_e[ct * de + c] = dht * k;
    if (!kmd2 && dw != 1) A.dgate_w[ct * dw + c] = T.v[c] * du;
    if (ddim != 1) A.ddecay[ct * ddim + c] = gG * graw[c];
  } else if (warp == 4) {  // scalar erase gate
    if (kmd2) {
      if (lane == 0) A.dgate_e[ct] = dce;
    } else if (de == 1) {
      float acc = 0.f;
      for (int c = lane; c < KD; c += 32) acc += (gv[2][c] + dc * T.k[c]) * T.k[c];
      acc = warp_sum(acc);
      if (lane == 0) A.dgate_e[ct] = acc;
    }
  } else if (warp == 5) {  // scalar write gate
    if (kmd2) {
      if (lane == 0) A.dgate_w[ct] = dcw;
    } else if (dw == 1) {
      float acc = 0.f;
      for (int c = lane; c < VD; c += 32) acc += T.v[c] * T.cw * dd[c];
      acc = warp_sum(acc);
      if (lane == 0) A.dgate_w[ct] = acc;
    }
  } else if (warp == 6) {  // scalar decay
    if (ddim == 1) {
      float acc = 0.f;
      for (int c = lane; c < KD; c += 32) acc += gv[3][c];
      acc = warp_sum(acc);
      if (lane == 0) A.ddecay[ct] = acc * graw[0];
    }
  } else if (warp == 7 && a.r_out > 1 && A.dout_mix) {  // query-slot mix weights
    for (int r = 0; r < a.r_out; ++r) {
      float acc = 0.f;
      for (int c = lane; c < KD; c += 32)
        acc += (r < MAXR ? T.qs[r][c] : ld_as_f32(a.q.ptr, a.q.dtype, view_off(a.q, b, t, h, m, r) + c)) * gv[0][c];
      acc = warp_sum(acc);
      if (lane == 0) atomicAdd(A.dout_mix + h * a.r_out + r, acc);
    }
  }
}

#ifdef GDNX_PHASE_PROBE
__device__ unsigned long long g_bwd_probe[8];
#define BWD_MARK(slot)                                            \
  do {                                                            \
    if (threadIdx.x == 0) {                                       \
      const long long n_ = clock64();                             \
      pacc[slot] += (unsigned long long)(n_ - pmark);             \
      pmark = n_;                                                 \
    }                                                             \
  } while (0)
#else
#define BWD_MARK(slot) \
  do {                 \
  } while (0)
#endif

// shared memory
struct BwdSmem {
  Tok tk[SUB];
  uint8_t raw[2 * SUB * RAWTOK];  // rows fetched ahead (two stagings)
  float graw[SUB][KD];       // d factor / d raw decay per channel
  float red[4][NW][KD];      // column partials per warp: dq, dk (S part), dh, dG
  float gvec[4][KD];         // their sums
  float dd[2][VD];           // dS k per row (by token parity: the next token's writes
                             // may run while a slow thread still reads these)
  float scal[2][NW][2];      // per-warp partials of dcw, dce (same double buffering)
};

__global__ void __launch_bounds__(NT, 1) scan_bwd_kernel(const BwdParams P) {
  // the dynamic shared block is 16-byte aligned; deriving the struct from it without an
  // integer round trip keeps the accesses in the shared address space
  extern __shared__ __align__(16) uint8_t smraw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>(smraw);
  const gdnx_scan_bwd_args& A = P.a;
  const gdnx_scan_args& a = A.fwd;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int v = tid >> 2, qd = tid & 3;
  const int64_t n = blockIdx.x;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int64_t T = a.T;
  float* ckpt = P.ckpt + (size_t)n * P.nblk * STATE;
  float* subs = P.sub + (size_t)n * SUB * STATE;
  float* ring = P.ring + (size_t)n * (SUB + 1) * STATE;
  float S[32];
#ifdef GDNX_PHASE_PROBE
  long long pmark = clock64();
  unsigned long long pacc[8] = {};
#endif

  int64_t kcall = 0;  // index of the next staging (the prefetch schedule follows it)
  RawScal rsc{0.f, 0.f, 0.f};
  if (P.prefetch) prefetch(P, sm.raw, 0, b, h, m, warp, lane, rsc);
  // ---- forward sweep: state at every block start ----
  if (a.state_in) ld_state(a.state_in + (size_t)n * STATE, v, qd, S);
  else
#pragma unroll
    for (int e = 0; e < 32; ++e) S[e] = 0.f;
  for (int64_t blk = 0; blk < P.nblk; ++blk) {
    st_state(ckpt + blk * STATE, v, qd, S);
    if (blk == P.nblk - 1) break;  // the last block's end state is not needed
    for (int64_t t0 = blk * BLK; t0 < (blk + 1) * BLK; t0 += SUB) {
      BWD_MARK(0);
      stage(P, sm.tk, &sm.graw[0][0], b, h, m, t0, SUB, warp, lane, false, sm.raw, kcall++, rsc);
      __syncthreads();
      BWD_MARK(7);
#pragma unroll 1
      for (int j = 0; j < SUB; ++j) fwd_step(S, sm.tk[j], v, qd);
      __syncthreads();
    }
  }

  BWD_MARK(0);
  // ---- reverse sweep ----
  float dS[32];
  if (A.dstate_out) ld_state(A.dstate_out + (size_t)n * STATE, v, qd, dS);
  else
#pragma unroll
    for (int e = 0; e < 32; ++e) dS[e] = 0.f;
  const int64_t ct_stride = a.H * a.M;  // chain-token index = (b T + t) H M + h M + m
  for (int64_t blk = P.nblk - 1; blk >= 0; --blk) {
    const int64_t tb = blk * BLK;
    const int nb = (int)((T - tb) < BLK ? (T - tb) : BLK);
    const int nsub = (nb + SUB - 1) / SUB;
    ld_state(ckpt + blk * STATE, v, qd, S);
    for (int sb = 0; sb < nsub; ++sb) {  // sub-block start states
      st_state(subs + sb * STATE, v, qd, S);
      if (sb == nsub - 1) break;
      stage(P, sm.tk, &sm.graw[0][0], b, h, m, tb + SUB * sb, SUB, warp, lane, false, sm.raw, kcall++, rsc);
      __syncthreads();
#pragma unroll 1
      for (int j = 0; j < SUB; ++j) fwd_step(S, sm.tk[j], v, qd);
      __syncthreads();
    }
    BWD_MARK(1);
    for (int sb = nsub - 1; sb >= 0; --sb) {
      const int64_t t0 = tb + SUB * sb;
      const int nt = (int)((T - t0) < SUB ? (T - t0) : SUB);
      stage(P, sm.tk, &sm.graw[0][0], b, h, m, t0, nt, warp, lane, true, sm.raw, kcall++, rsc);
      ld_state(subs + sb * STATE, v, qd, S);
      st_state(ring, v, qd, S);
      __syncthreads();
#pragma unroll 1
      for (int j = 0; j < nt; ++j) {  // token states S_t0 .. S_{t0+nt-1} into ring[1 .. nt]
        fwd_step(S, sm.tk[j], v, qd);
        st_state(ring + (j + 1) * STATE, v, qd, S);
      }
      float Sc[32];
      ld_state(ring + nt * STATE, v, qd, Sc);  // S_t of the first reverse step
      BWD_MARK(2);
#pragma unroll 1
      for (int j = nt - 1; j >= 0; --j) {
        const Tok& Tk = sm.tk[j];
        float Sp[32];
        ld_state(ring + j * STATE, v, qd, Sp);  // S_{t-1}
        const float dyv = Tk.dy[v];
        float part[32];
        // dq partials (S_t^T dy) and dS += dy q^T
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 qq = *reinterpret_cast<const float4*>(Tk.q + colof(qd, i));
          const float q4[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            part[4 * i + e] = Sc[4 * i + e] * dyv;
            dS[4 * i + e] = fmaf(dyv, q4[e], dS[4 * i + e]);
          }
        }
        colreduce_store(part, &sm.red[0][warp][0], lane, qd);
        // m = P h, dd = dS k
        float mrow = 0.f, ddr = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = colof(qd, i);
          const float4 g = *reinterpret_cast<const float4*>(Tk.G + c);
          const float4 hh = *reinterpret_cast<const float4*>(Tk.h + c);
          const float4 kk = *reinterpret_cast<const float4*>(Tk.k + c);
          const float g4[4] = {g.x, g.y, g.z, g.w}, h4[4] = {hh.x, hh.y, hh.z, hh.w}, k4[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            mrow = fmaf(Sp[4 * i + e] * g4[e], h4[e], mrow);
            ddr = fmaf(dS[4 * i + e], k4[e], ddr);
          }
        }
        mrow = rowsum4(mrow);
        ddr = rowsum4(ddr);
        const float d = Tk.cw * Tk.u[v] - Tk.ce * mrow;
        const float ced = Tk.ce * ddr;
        // dk (S part) = dS^T d
#pragma unroll
        for (int e = 0; e < 32; ++e) part[e] = dS[e] * d;
        colreduce_store(part, &sm.red[1][warp][0], lane, qd);
        // dh = -ce P^T dd
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 g = *reinterpret_cast<const float4*>(Tk.G + colof(qd, i));
          const float g4[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) part[4 * i + e] = -Sp[4 * i + e] * g4[e] * ced;
        }
        colreduce_store(part, &sm.red[2][warp][0], lane, qd);
        // dP = dS - ce dd h^T;  dG = colsum(dP (.) S_{t-1});  dS <- dP G
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = colof(qd, i);
          const float4 g = *reinterpret_cast<const float4*>(Tk.G + c);
          const float4 hh = *reinterpret_cast<const float4*>(Tk.h + c);
          const float g4[4] = {g.x, g.y, g.z, g.w}, h4[4] = {hh.x, hh.y, hh.z, hh.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int x = 4 * i + e;
            const float dP = fmaf(-ced, h4[e], dS[x]);
            part[x] = dP * Sp[x];
            dS[x] = dP * g4[e];
          }
        }
        colreduce_store(part, &sm.red[3][warp][0], lane, qd);
        // dcw = dd.u, dce = -dd.m (one thread per row contributes)
        {
          float s0 = qd == 0 ? ddr * Tk.u[v] : 0.f, s1 = qd == 0 ? -ddr * mrow : 0.f;
          s0 = warp_sum(s0);
          s1 = warp_sum(s1);
          if (lane == 0) {
            sm.scal[j & 1][warp][0] = s0;
            sm.scal[j & 1][warp][1] = s1;
          }
          if (qd == 0) sm.dd[j & 1][v] = ddr;
        }
        BWD_MARK(3);
        __syncthreads();
        BWD_MARK(4);
        {
          const int vec = tid >> 7, c = tid & 127;
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < NW; ++w) acc += sm.red[vec][w][c];
          sm.gvec[vec][c] = acc;
        }
        __syncthreads();
        BWD_MARK(5);
        // per-token gradients
        float dcw = 0.f, dce = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          dcw += sm.scal[j & 1][w][0];
          dce += sm.scal[j & 1][w][1];
        }
        const int64_t t = t0 + j;
        const int64_t ct = (b * T + t) * ct_stride + h * a.M + m;
        write_token_grads(P, Tk, sm.gvec, sm.dd[j & 1], &sm.graw[j][0], dcw, dce, ct, b, t, h, m, tid, warp, lane);
#pragma unroll
        for (int e = 0; e < 32; ++e) Sc[e] = Sp[e];
        BWD_MARK(6);
      }
      __syncthreads();
    }
  }
  if (A.dstate_in) st_state(A.dstate_in + (size_t)n * STATE, v, qd, dS);
#ifdef GDNX_PHASE_PROBE
  if (threadIdx.x == 0)
    for (int i = 0; i < 8; ++i) atomicAdd(&g_bwd_probe[i], pacc[i]);
#endif
}

}  // namespace

#ifdef GDNX_PHASE_PROBE
extern "C" GDNX_API int gdnx_debug_bwd_probe(unsigned long long* out8) {
  if (cudaMemcpyFromSymbol(out8, g_bwd_probe, 8 * sizeof(unsigned long long)) != cudaSuccess) return 1;
  unsigned long long z[8] = {};
  return cudaMemcpyToSymbol(g_bwd_probe, z, sizeof(z)) == cudaSuccess ? 0 : 1;
}
#endif

bool scan_bwd_supported(const gdnx_scan_bwd_args& A) {
  const gdnx_scan_args& a = A.fwd;
  if (a.K != KD || a.V != VD || a.rope.enable || a.decay_kind == GDNX_DECAY_BRAIDED) return false;
  if (a.decay.dim != 1 && a.decay.dim != KD) return false;
  if (a.state_in && (reinterpret_cast<uintptr_t>(a.state_in) & 15)) return false;
  if (A.dstate_out && (reinterpret_cast<uintptr_t>(A.dstate_out) & 15)) return false;
  if (A.dstate_in && (reinterpret_cast<uintptr_t>(A.dstate_in) & 15)) return false;
  return true;
}

size_t scan_bwd_workspace_bytes(const gdnx_scan_bwd_args& A) {
  const gdnx_scan_args& a = A.fwd;
  const int64_t N = a.B * a.H * a.M, nblk = (a.T + BLK - 1) / BLK;
  return (size_t)N * (nblk + SUB + SUB + 1) * STATE * sizeof(float);
}

gdnx_status launch_scan_bwd(const gdnx_scan_bwd_args& A, cudaStream_t st) {
  const gdnx_scan_args& a = A.fwd;
  BwdParams P;
  P.a = A;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.vec_e = a.gate_e.dim != 1;
  P.vec_w = a.gate_w.dim != 1;
  P.chan_decay = a.decay.dim == KD;
  // rows are fetched ahead as 8/16-byte pieces of 4 elements: every row start must keep that alignment
  auto row_ok = [](const gdnx_view& vw) {
    const int es = vw.dtype == GDNX_F32 ? 4 : 2;
    return (reinterpret_cast<uintptr_t>(vw.ptr) % (4 * es)) == 0 && vw.sb % 4 == 0 && vw.st % 4 == 0 &&
           vw.sh % 4 == 0 && vw.sm % 4 == 0 && vw.ss % 4 == 0;
  };
  P.prefetch = row_ok(a.q) && row_ok(a.k) && row_ok(a.v) && (!P.vec_e || row_ok(a.gate_e)) &&
               (!P.vec_w || row_ok(a.gate_w)) && (!P.chan_decay || row_ok(a.decay)) && row_ok(A.dy);
  const int64_t N = a.B * a.H * a.M;
  P.nblk = (a.T + BLK - 1) / BLK;
  float* ws = reinterpret_cast<float*>(A.workspace);
  P.ckpt = ws;
  P.sub = ws + (size_t)N * P.nblk * STATE;
  P.ring = P.sub + (size_t)N * SUB * STATE;
  const int smem = (int)sizeof(BwdSmem) + 16;
  if (cudaFuncSetAttribute(scan_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return GDNX_ELAUNCH;
  scan_bwd_kernel<<<(unsigned)N, NT, smem, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
