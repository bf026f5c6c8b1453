// Rearrangement-SVD compaction of one chain, executed by one CTA on shared
// memory (gdn3/gdn3_upgrade.py:650-719 semantics):
//
//   R_mat (m x n) = sum_r vec(A_r) vec(B_r)^T + rearrange(U Vb^T)   [built by the caller]
//   Y = R G ; twice  Y = R (R^T Y)          (randomized range finder, G given)
//   Q = orth(Y)                             (modified Gram-Schmidt, two passes)
//   Bm = Q^T R  (q x n) ;  Bm = Ub S Vh     (one-sided Jacobi SVD, Hestenes)
//   A_svd_r = (Q Ub)[:, r] S_r ,  B_svd_r = Vh[r]        (r < R, descending S)
//   A <- d A + (1-d) A_svd ;  B <- d B + (1-d) B_svd   ;  U, Vb untouched
//   err = |R|_F^2 - sum_{r<R} S_r^2
//
// The joint sign of each (A_svd_r, B_svd_r) pair is fixed so that the
// largest-|.| entry of B_svd_r is positive; the span-level results (and Q's
// own column signs) do not depend on the QR convention.
#pragma once

#include "common.cuh"

namespace gdnx {

constexpr int kCompMaxQ = 8;    // sketch width  q = min(R+4, m, n) <= 8
constexpr int kCompMaxN = 64;   // n = b_v * b_k <= 64
constexpr int kCompMaxM = 256;  // m = a_v * a_k <= 256
constexpr int kCompThreads = 256;
constexpr int kCompPT = 16;     // slots per staged tile of U / Vb

// Compile-time Kronecker shape: A_r is a_v x a_k, B_r is b_v x b_k, rank R.
// Constant dimensions turn every index split in the hot loops into shifts.
template <int AV, int AK, int BV, int BK, int RR>
struct KDims {
  static constexpr int R = RR, a_v = AV, a_k = AK, b_v = BV, b_k = BK;
  static constexpr int m = AV * AK, n = BV * BK;
  static constexpr int q = (RR + 4) < (m < n ? m : n) ? (RR + 4) : (m < n ? m : n);
  float delta;
};
using Dims16x8 = KDims<16, 16, 8, 8, 4>;  // K = V = 128 (the reference's defaults)
using Dims8x8 = KDims<8, 8, 8, 8, 4>;     // K = V = 64

// Shared-memory floats the core needs beyond R_mat (which is m x (n+1), padded).
__host__ __device__ constexpr int compact_work_floats() {
  return 2 * kCompMaxM * kCompMaxQ      // Y, Q
         + kCompMaxN * kCompMaxQ        // Z
         + kCompMaxQ * kCompMaxN        // Bm
         + kCompMaxN * kCompMaxQ        // G
         + kCompMaxQ * kCompMaxQ        // J
         + 64;                          // scalars / reductions
}
__host__ __device__ constexpr int compact_ld(int n) { return n + 1; }

GDNX_DEV float block_sum(float x, float* red) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  x = warp_sum(x);
  __syncthreads();
  if (lane == 0) red[warp] = x;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x / 32;
  for (int i = 0; i < nw; ++i) t += red[i];
  __syncthreads();
  return t;
}

// Returns err (discarded energy, not clamped) to every thread.  Rm (m x ld)
// is read only.  A_s [R][m], B_s [R][n] hold the current (true) factors and
// are overwritten with the blended ones.  G is [n][q] in global memory.
//
// sketch = 1 selects the reference's compact_mode "sketch" / "sketch_noqr"
// (gdn3/gdn3_upgrade.py:579-596; the two modes run the same code there):
//   Y = R G (G is [n][R]) ; Q = Y with unit columns (norms clamped at 1e-12)
//   Bm = Q^T R (R x n) ; b_r = |Bm_r| (clamped at 1e-12)
//   A_svd_r = Q_r b_r ,  B_svd_r = Bm_r / b_r ;  same blend ;  err = 0
template <class CD>
GDNX_DEV float compact_core(const float* Rm, float* A_s, float* B_s, const float* G,
                            float* work, const CD d, int sketch = 0) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid % 32, warp = tid / 32;
  const int m = d.m, n = d.n, q = d.q, R = d.R;
  const int ld = compact_ld(n);
  float* Y = work;
  float* Qm = Y + kCompMaxM * kCompMaxQ;
  float* Z = Qm + kCompMaxM * kCompMaxQ;
  float* Bm = Z + kCompMaxN * kCompMaxQ;
  float* Gs = Bm + kCompMaxQ * kCompMaxN;
  float* J = Gs + kCompMaxN * kCompMaxQ;
  float* red = J + kCompMaxQ * kCompMaxQ;  // 64 floats

  // energy (the sketch mode reports none)
  float total = 0.f;
  if (!sketch) {
    float e = 0.f;
    for (int idx = tid; idx < m * n; idx += nt) {
      const float x = Rm[(idx / n) * ld + idx % n];
      e += x * x;
    }
    total = block_sum(e, red);
    for (int idx = tid; idx < n * q; idx += nt) Gs[idx] = G[idx];
  } else {  // G is [n][R]: the product below runs on q columns, the ones past R zero
    for (int idx = tid; idx < n * q; idx += nt) {
      const int j = idx / q, c = idx % q;
      Gs[idx] = c < R ? G[j * R + c] : 0.f;
    }
  }
  __syncthreads();
  static_assert(CD::q == kCompMaxQ, "register-blocked products assume q = 8");
  // Y = R X (m x 8) for X = G or Z (n x 8): one thread per row i, X rows broadcast
  auto row_times = [&](const float* X) {
    for (int i = tid; i < m; i += nt) {
      float acc[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = 0.f;
      for (int jj = 0; jj < n; ++jj) {
        const float r = Rm[i * ld + jj];
        const float4 x0 = *reinterpret_cast<const float4*>(X + jj * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(X + jj * 8 + 4);
        acc[0] = fmaf(r, x0.x, acc[0]); acc[1] = fmaf(r, x0.y, acc[1]);
        acc[2] = fmaf(r, x0.z, acc[2]); acc[3] = fmaf(r, x0.w, acc[3]);
        acc[4] = fmaf(r, x1.x, acc[4]); acc[5] = fmaf(r, x1.y, acc[5]);
        acc[6] = fmaf(r, x1.z, acc[6]); acc[7] = fmaf(r, x1.w, acc[7]);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) Y[i * 8 + c] = acc[c];
    }
  };
  // Out[j][c] = sum_i R[i][j] X[i][c] (n x 8, X = Y or Q): lane group g = lane / 8 of warp w
  // takes column j = 8 w + lane % 8 over the rows i with (i / 8) % 4 == g (R reads hit 32
  // distinct banks), eight independent sums; the four groups' sums meet by shuffles
  auto col_times = [&](const float* X, float* Out, int out_stride_j, int out_stride_c) {
    const int g = lane >> 3, jj = warp * 8 + (lane & 7);
    const bool has = jj < n && warp * 8 < n;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
    if (has) {
      for (int i0 = 8 * g; i0 < m; i0 += 32) {
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const int i = i0 + b;
          if (i >= m) break;
          const float r = Rm[i * ld + jj];
          const float4 x0 = *reinterpret_cast<const float4*>(X + i * 8);
          const float4 x1 = *reinterpret_cast<const float4*>(X + i * 8 + 4);
          acc[0] = fmaf(r, x0.x, acc[0]); acc[1] = fmaf(r, x0.y, acc[1]);
          acc[2] = fmaf(r, x0.z, acc[2]); acc[3] = fmaf(r, x0.w, acc[3]);
          acc[4] = fmaf(r, x1.x, acc[4]); acc[5] = fmaf(r, x1.y, acc[5]);
          acc[6] = fmaf(r, x1.z, acc[6]); acc[7] = fmaf(r, x1.w, acc[7]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 8);
      acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 16);
    }
    if (has) {  // group g writes outputs 2 g, 2 g + 1
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if ((c >> 1) == g) Out[jj * out_stride_j + c * out_stride_c] = acc[c];
    }
  };
  row_times(Gs);
  __syncthreads();
  if (sketch) {
    // column norms of Y (warp c < R), then Q = Y / |Y_c| in place (columns past R stay 0)
    if (warp < R) {
      float s2 = 0.f;
      for (int i = lane; i < m; i += 32) s2 = fmaf(Y[i * q + warp], Y[i * q + warp], s2);
      s2 = warp_sum(s2);
      if (lane == 0) red[warp] = fmaxf(sqrtf(s2), 1e-12f);
    }
    __syncthreads();
    for (int idx = tid; idx < m * q; idx += nt) {
      const int c = idx % q;
      Qm[idx] = c < R ? Y[idx] / red[c] : 0.f;
    }
    __syncthreads();
    col_times(Qm, Bm, 1, n);  // Bm = Q^T R, rows past R zero
    __syncthreads();
    if (warp < R) {
      float s2 = 0.f;
      for (int j = lane; j < n; j += 32) s2 = fmaf(Bm[warp * n + j], Bm[warp * n + j], s2);
      s2 = warp_sum(s2);
      if (lane == 0) red[8 + warp] = fmaxf(sqrtf(s2), 1e-12f);
    }
    __syncthreads();
    const float dd = d.delta, od = 1.f - d.delta;
    for (int idx = tid; idx < R * m; idx += nt) {
      const int r = idx / m, i = idx % m;
      A_s[idx] = dd * A_s[idx] + od * (Qm[i * q + r] * red[8 + r]);
    }
    for (int idx = tid; idx < R * n; idx += nt) {
      const int r = idx / n, j = idx % n;
      B_s[idx] = dd * B_s[idx] + od * (Bm[r * n + j] / red[8 + r]);
    }
    __syncthreads();
    return 0.f;
  }
  for (int it = 0; it < 2; ++it) {
    col_times(Y, Z, 8, 1);  // Z = R^T Y
    __syncthreads();
    row_times(Z);           // Y = R Z
    __syncthreads();
  }
  // Q = orth(Y): classical Gram-Schmidt applied twice per column ("twice is enough") on
  // one warp, lane l holding rows l + 32 r, so every projection is a warp reduction of
  // <= 8 dot products (no block barriers); the other warps wait at the barrier below.
  static_assert(kCompMaxM <= 32 * 8, "one warp holds every row of Y");
  if (warp == 0) {
    float qv[kCompMaxQ][8];  // qv[p][r] = Q[lane + 32 r][p]
#pragma unroll
    for (int c = 0; c < kCompMaxQ; ++c) {
      if (c >= q) break;
      float y[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int i = lane + 32 * r;
        y[r] = i < m ? Y[i * q + c] : 0.f;
      }
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        if (c == 0) break;
        float dp[kCompMaxQ];
#pragma unroll
        for (int p = 0; p < kCompMaxQ; ++p) {
          float acc = 0.f;
          if (p < c)
#pragma unroll
            for (int r = 0; r < 8; ++r) acc = fmaf(qv[p][r], y[r], acc);
          dp[p] = acc;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int p = 0; p < kCompMaxQ; ++p)
            if (p < c) dp[p] += __shfl_xor_sync(0xffffffffu, dp[p], o);
#pragma unroll
        for (int p = 0; p < kCompMaxQ; ++p)
          if (p < c)
#pragma unroll
            for (int r = 0; r < 8; ++r) y[r] = fmaf(-dp[p], qv[p][r], y[r]);
      }
      float nn = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) nn = fmaf(y[r], y[r], nn);
      nn = warp_sum(nn);
      const float inv = nn > 1e-30f ? rsqrtf(nn) : 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) qv[c][r] = y[r] * inv;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int i = lane + 32 * r;
      if (i < m)
#pragma unroll
        for (int c = 0; c < kCompMaxQ; ++c)
          if (c < q) Qm[i * q + c] = qv[c][r];
    }
  }
  __syncthreads();
  // Bm = Q^T R   (q x n), Bm[c][j]
  col_times(Qm, Bm, 1, n);
  __syncthreads();
  // One-sided Jacobi on W = Bm^T (n x q), columns c of W = rows of Bm in shared memory.
  // Each round s = 1..7 rotates the four disjoint pairs (i, i ^ s); warps 0-3 take one pair
  // each (lane: rows lane and lane + 32), the accumulated rotation J (q x q, row-major in
  // shared memory) alongside, and meet at a 128-thread barrier between rounds.
  float* Js = Gs;  // the sketch's space is free once Bm is formed: J [8][8], then the sweep flags
  volatile float* flags = Js + kCompMaxQ * kCompMaxQ;  // [4] per-warp max off, [4] Frobenius parts
  if (warp < 4) {
    const bool r0 = lane < n, r1 = lane + 32 < n;
    // Frobenius scale of W: rotations below fp32 resolution of the whole matrix are skipped,
    // so near-zero (noise) columns cannot keep a sweep alive
    float fp = 0.f;
    for (int c = 2 * warp; c < 2 * warp + 2; ++c)
      if (c < q) {
        const float a0 = r0 ? Bm[c * n + lane] : 0.f, a1 = r1 ? Bm[c * n + lane + 32] : 0.f;
        fp += a0 * a0 + a1 * a1;
      }
    fp = warp_sum(fp);
    if (lane == 0) flags[4 + warp] = fp;
    for (int c = lane; c < kCompMaxQ * kCompMaxQ; c += 32) Js[c] = (c / kCompMaxQ == c % kCompMaxQ) ? 1.f : 0.f;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const float fro = flags[4] + flags[5] + flags[6] + flags[7];
    for (int sweep = 0; sweep < 30; ++sweep) {
      float off = 0.f;
      for (int sr = 1; sr < kCompMaxQ; ++sr) {
        // this warp's pair: the warp-th i with i < (i ^ sr)
        int i = 0, found = -1;
#pragma unroll
        for (int ii = 0; ii < kCompMaxQ; ++ii)
          if (ii < (ii ^ sr)) {
            if (++found == warp) i = ii;
          }
        const int j = i ^ sr;
        float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
        if (j < q) {
          a0 = r0 ? Bm[i * n + lane] : 0.f;
          a1 = r1 ? Bm[i * n + lane + 32] : 0.f;
          b0 = r0 ? Bm[j * n + lane] : 0.f;
          b1 = r1 ? Bm[j * n + lane + 32] : 0.f;
        }
        float al = a0 * a0 + a1 * a1, be = b0 * b0 + b1 * b1, ga = a0 * b0 + a1 * b1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          al += __shfl_xor_sync(0xffffffffu, al, o);
          be += __shfl_xor_sync(0xffffffffu, be, o);
          ga += __shfl_xor_sync(0xffffffffu, ga, o);
        }
        // thresholds on squares (no square roots): ga^2 against 1e-12 al be
        const float p2 = al * be, g2 = ga * ga;
        const bool rot = j < q && p2 > 1e-37f && g2 > 1e-12f * p2 && fabsf(ga) > 1e-9f * fro;
        if (rot) {
          off = fmaxf(off, __fdividef(g2, p2));
          // the sweep corrects rotation-parameter rounding; |2 ga| > 1e-6 sqrt(al be) keeps zeta in range
          const float zeta = __fdividef(be - al, 2.f * ga);
          const float w1z = fmaf(zeta, zeta, 1.f);
          const float t = copysignf(__fdividef(1.f, fabsf(zeta) + w1z * rsqrtf(w1z)), zeta);
          const float cs = rsqrtf(fmaf(t, t, 1.f)), sn = cs * t;
          if (r0) {
            Bm[i * n + lane] = cs * a0 - sn * b0;
            Bm[j * n + lane] = sn * a0 + cs * b0;
          }
          if (r1) {
            Bm[i * n + lane + 32] = cs * a1 - sn * b1;
            Bm[j * n + lane + 32] = sn * a1 + cs * b1;
          }
          if (lane < q) {
            const float ja = Js[lane * kCompMaxQ + i], jb = Js[lane * kCompMaxQ + j];
            Js[lane * kCompMaxQ + i] = cs * ja - sn * jb;
            Js[lane * kCompMaxQ + j] = sn * ja + cs * jb;
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      if (lane == 0) flags[warp] = off;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const float offall = fmaxf(fmaxf(flags[0], flags[1]), fmaxf(flags[2], flags[3]));
      asm volatile("bar.sync 1, 128;" ::: "memory");  // every warp has read the flags
      if (offall < 4e-12f) break;  // (ga^2 / al be) < (2e-6)^2: columns orthogonal to fp32 working accuracy
    }
  }
  __syncthreads();
  if (warp == 0) {
    const bool r0 = lane < n, r1 = lane + 32 < n;
    float w0[kCompMaxQ], w1[kCompMaxQ], jr[kCompMaxQ];
#pragma unroll
    for (int c = 0; c < kCompMaxQ; ++c) {
      w0[c] = (c < q && r0) ? Bm[c * n + lane] : 0.f;
      w1[c] = (c < q && r1) ? Bm[c * n + lane + 32] : 0.f;
      jr[c] = lane < kCompMaxQ ? Js[lane * kCompMaxQ + c] : 0.f;
    }
    // singular values, descending order (selection; q <= 8)
    float sv[kCompMaxQ];
#pragma unroll
    for (int c = 0; c < kCompMaxQ; ++c) sv[c] = c < q ? sqrtf(warp_sum(w0[c] * w0[c] + w1[c] * w1[c])) : -1.f;
    int order[kCompMaxQ];
#pragma unroll
    for (int c = 0; c < kCompMaxQ; ++c) order[c] = c;
    for (int a = 0; a < q; ++a)
      for (int b = a + 1; b < q; ++b)
        if (sv[order[b]] > sv[order[a]]) { int tmp = order[a]; order[a] = order[b]; order[b] = tmp; }
    // Z <- right singular vectors of Bm (= normalised columns of W), columns r < R
    // J <- Ub (left), sorted; red[0..R) <- singular values
    for (int r = 0; r < R; ++r) {
      int c = order[0];
#pragma unroll
      for (int cc = 0; cc < kCompMaxQ; ++cc) if (cc < q && order[r] == cc) c = cc;
      float wc0 = 0.f, wc1 = 0.f, jc = 0.f;
#pragma unroll
      for (int cc = 0; cc < kCompMaxQ; ++cc) if (cc == c) { wc0 = w0[cc]; wc1 = w1[cc]; jc = jr[cc]; }
      const float s = sv[c];
      const float inv = s > 1e-30f ? 1.f / s : 0.f;
      float v0 = wc0 * inv, v1 = wc1 * inv;
      // sign: largest-|.| entry of the right vector positive (first index on ties)
      float best = r0 ? fabsf(v0) : -1.f;
      int bidx = lane;
      float bval = v0;
      if (r1 && fabsf(v1) > best) { best = fabsf(v1); bidx = lane + 32; bval = v1; }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        const float ov = __shfl_xor_sync(0xffffffffu, bval, o);
        if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; bval = ov; }
      }
      const float sg = bval < 0.f ? -1.f : 1.f;
      if (r0) Z[lane * kCompMaxQ + r] = sg * v0;
      if (r1) Z[(lane + 32) * kCompMaxQ + r] = sg * v1;
      if (lane < q) J[lane * kCompMaxQ + r] = sg * jc;
      if (lane == 0) red[32 + r] = s;
    }
  }
  __syncthreads();
  // blend: A_r += (1-d)(Q Ub_r S_r - A_r) ; B_r likewise with Vs_r
  const float dd = d.delta, od = 1.f - d.delta;
  for (int idx = tid; idx < R * m; idx += nt) {
    const int r = idx / m, i = idx % m;
    float acc = 0.f;
    for (int c = 0; c < q; ++c) acc = fmaf(Qm[i * q + c], J[c * kCompMaxQ + r], acc);
    A_s[idx] = dd * A_s[idx] + od * (acc * red[32 + r]);
  }
  for (int idx = tid; idx < R * n; idx += nt) {
    const int r = idx / n, j = idx % n;
    B_s[idx] = dd * B_s[idx] + od * Z[j * kCompMaxQ + r];
  }
  float kept = 0.f;
  for (int r = 0; r < R; ++r) kept += red[32 + r] * red[32 + r];
  __syncthreads();
  return total - kept;
}

// Adds sum_r vec(A_r) vec(B_r)^T to Rm (m x ld), A_s [R][m], B_s [R][n].
template <class CD>
GDNX_DEV void add_kron_rmat(float* Rm, const float* A_s, const float* B_s, const CD d) {
  const int ld = compact_ld(d.n);
  for (int idx = threadIdx.x; idx < d.m * d.n; idx += blockDim.x) {
    const int i = idx / d.n, j = idx % d.n;
    float acc = 0.f;
    for (int r = 0; r < d.R; ++r) acc = fmaf(A_s[r * d.m + i], B_s[r * d.n + j], acc);
    Rm[i * ld + j] += acc;
  }
}

// Rearranged position of dense residual element (v, k):
// R[(av, ak)][(bv, bk)] = S[av*b_v + bv][ak*b_k + bk].
template <class CD>
GDNX_DEV int rmat_index(int v, int k, const CD d) {
  const int av = v / d.b_v, bv = v % d.b_v, ak = k / d.b_k, bk = k % d.b_k;
  return (av * d.a_k + ak) * compact_ld(d.n) + bv * d.b_k + bk;
}

// Rm += rearrange(U diag(dsl) Vb^T) for V*K <= 64*256, built in registers tile by
// tile (dsl = per-slot scale, nullptr = 1).  Needs blockDim.x == kCompThreads.
// tileU / tileV hold two tiles each ((V + K) x kCompPT x 2 floats): when P is a
// multiple of 4 the next tile is fetched with cp.async while the current one is used.
template <class CD>
GDNX_DEV void add_residual_rmat(float* Rm, const float* U, const float* Vb, const float* dsl, int V, int K, int P,
                                float* tileU, float* tileV, const CD d) {
  const int tid = threadIdx.x;
  const int per = (V * K + kCompThreads - 1) / kCompThreads;  // <= 64
  constexpr int KK = CD::a_k * CD::b_k;
  static_assert(kCompThreads % KK == 0, "thread -> key mapping");
  const int kk = tid % KK, v0 = tid / KK;
  const bool async = (P & 3) == 0 && ((reinterpret_cast<uintptr_t>(U) | reinterpret_cast<uintptr_t>(Vb)) & 15) == 0;
  // tile t of slots p0 = t * kCompPT into buffer t & 1 (zero past P)
  auto fetch = [&](int p0, int buf) {
    float* tu = tileU + buf * V * kCompPT;
    float* tvb = tileV + buf * K * kCompPT;
    const int np = min(kCompPT, P - p0);
    if (async) {
      for (int idx = tid; idx < (V + K) * (kCompPT / 4); idx += kCompThreads) {
        const int r = idx / (kCompPT / 4), c4 = idx % (kCompPT / 4);
        const bool isu = r < V;
        const int rr = isu ? r : r - V;
        const float* src = (isu ? U : Vb) + (int64_t)rr * P + p0 + 4 * c4;
        float* dst = (isu ? tu + rr * kCompPT : tvb + rr * kCompPT) + 4 * c4;
        const uint32_t sd = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
        const int bytes = 4 * c4 < np ? 16 : 0;  // np is a multiple of 4 here
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sd), "l"(bytes ? src : U), "r"(bytes)
                     : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
      for (int idx = tid; idx < V * kCompPT; idx += kCompThreads) {
        const int vv = idx / kCompPT, pp = idx % kCompPT;
        tu[idx] = pp < np ? U[(int64_t)vv * P + p0 + pp] : 0.f;
      }
      for (int idx = tid; idx < K * kCompPT; idx += kCompThreads) {
        const int kv = idx / kCompPT, pp = idx % kCompPT;
        tvb[idx] = pp < np ? Vb[(int64_t)kv * P + p0 + pp] : 0.f;
      }
    }
  };
  float acc[64];
#pragma unroll
  for (int e = 0; e < 64; ++e) acc[e] = 0.f;
  __syncthreads();
  fetch(0, 0);
  for (int p0 = 0, t = 0; p0 < P; p0 += kCompPT, ++t) {
    if (async) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();  // tile t is in place; every thread is done with tile t - 1
    if (p0 + kCompPT < P) fetch(p0 + kCompPT, (t + 1) & 1);
    const float* tu = tileU + (t & 1) * V * kCompPT;
    const float* tvb = tileV + (t & 1) * K * kCompPT;
    // element e of this thread is (v = tid / K + (threads / K) e, k = tid % K): its key
    // row of the tile (times the slot scales) is the same for every e, so it is held in registers
    float tv[kCompPT];
#pragma unroll
    for (int pp = 0; pp < kCompPT; pp += 4) {
      const float4 t4 = *reinterpret_cast<const float4*>(tvb + kk * kCompPT + pp);
      tv[pp] = t4.x; tv[pp + 1] = t4.y; tv[pp + 2] = t4.z; tv[pp + 3] = t4.w;
    }
#pragma unroll
    for (int pp = 0; pp < kCompPT; ++pp)
      if (dsl) tv[pp] *= (p0 + pp < P) ? dsl[p0 + pp] : 0.f;
#pragma unroll
    for (int e = 0; e < 64; ++e) {
      if (e >= per) break;
      const int vv = v0 + (kCompThreads / KK) * e;
      float s = acc[e];
#pragma unroll
      for (int pp = 0; pp < kCompPT; pp += 4) {
        const float4 u4 = *reinterpret_cast<const float4*>(tu + vv * kCompPT + pp);
        s = fmaf(u4.x, tv[pp], s);
        s = fmaf(u4.y, tv[pp + 1], s);
        s = fmaf(u4.z, tv[pp + 2], s);
        s = fmaf(u4.w, tv[pp + 3], s);
      }
      acc[e] = s;
    }
  }
#pragma unroll
  for (int e = 0; e < 64; ++e) {
    if (e >= per) break;
    const int idx = tid + kCompThreads * e;
    if (idx >= V * K) break;
    Rm[rmat_index(idx / K, idx % K, d)] += acc[e];
  }
  __syncthreads();
}

}  // namespace gdnx
