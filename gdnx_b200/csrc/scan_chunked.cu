// Chunked WY/UT gated delta-rule scan on the 5th-generation tensor cores.
//
// One CTA (8 warps) owns one chain and walks its 64-token chunks in order;
// the fp32 state S (V x K = 128 x 128) stays resident in TMEM for the whole
// sequence.  With L_i the cumulative log-decay inside the chunk, S0 the state
// at the chunk start and per-token coefficients ce (erase) / cw (write)
// [GDN3 scalar gates: ce = a b, cw = a w, a = alpha(b |k|^2); KMD-2: beta_e, beta_w]:
//
//   (I + A) W = RHS,  A_jl = ce_j e^{L_j - L_l} (k_j . k_l)   (l < j)
//                     RHS_j = cw_j v_j - ce_j e^{L_j} S0 k_j
//   y_i  = e^{L_i} S0 q_i + sum_{j <= i} e^{L_i - L_j} (q_i . k_j) W_j
//   S_C  = e^{L_C} S0 + sum_j e^{L_C - L_j} W_j k_j^T
//
// Only differences L_i - L_j (i >= j) and L_i are exponentiated, so no factor
// exceeds 1 (no decay ratios, no overflow for strong decays).  Per chunk the
// tensor-core work is six bf16 UMMAs with fp32 accumulation in TMEM (the
// transposed products put V = 128 on the M axis):
//   G1  [K;Q] K^T    -> k.k Gram (rows 0-63) and q.k Gram (rows 64-127)
//   G2  S0 K^T       -> S0 k_j            G3  S0 Qd^T -> e^{L_i} S0 q_i
//   G4  RHS^T T^T    -> W^T               G5  W^T Mq^T (accumulated on G3) -> y
//   G6  W'^T K       -> accumulated on e^{L_C} S0 in TMEM (K read MN-major)
// and T = (I + A)^{-1} (64 x 64 unit lower triangular) is formed on the CUDA
// cores by blocked forward substitution (16 x 16 diagonal blocks, then three
// levels of block products).  The prologue (lane RoPE, decay, alpha, gates) is
// fused into the chunk load.  Every mbarrier wait is bounded; on a timeout the
// kernel records GDNX_ETIMEOUT in the workspace error word, frees its TMEM
// and exits.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace gdnx {
namespace {

constexpr int C = 64;         // chunk length
constexpr int KD = 128;       // key dim
constexpr int VD = 128;       // value dim
constexpr int NT = 256;       // threads
constexpr int TMEM_COLS = 256;

// shared-memory map (bytes from a 1024-aligned base)
constexpr int OFF_KQ = 0;                   // [2 kb][128 rows][64] bf16: rows 0-63 K, 64-127 Q (then Qd)
constexpr int OFF_S0 = OFF_KQ + 32768;      // [2 kb][128 rows v][64] bf16
constexpr int OFF_RHS = OFF_S0 + 32768;     // [128 rows v][64 j] bf16 (RHS^T, later W'^T)
constexpr int OFF_W = OFF_RHS + 16384;      // [128 rows v][64 j] bf16 (W^T)
constexpr int OFF_T = OFF_W + 16384;        // [64 rows j][64 l] bf16
constexpr int OFF_MQ = OFF_T + 8192;        // [64 rows i][64 j] bf16
constexpr int OFF_LM = OFF_MQ + 8192;       // fp32 [64][65]  A (strictly lower)
constexpr int OFF_TM = OFF_LM + 64 * 65 * 4;  // fp32 [64][65]  T (+ upper-block scratch)
constexpr int OFF_SC = OFF_TM + 64 * 65 * 4;  // fp32 scalars: L, eL, eLC, ce, cw, kn2, inv_freq (7 x 64)
constexpr int OFF_BAR = OFF_SC + 7 * 64 * 4;
constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;  // + alignment slack

struct ChunkParams {
  gdnx_scan_args a;
  int kmd2;
  int* err;
};

__device__ __forceinline__ void load8_bf16(const void* base, int64_t off, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off);
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(p[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__global__ void __launch_bounds__(NT, 1) chunked_scan_kernel(const ChunkParams P) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  char* cKQ = reinterpret_cast<char*>(sm + OFF_KQ);
  char* cS0 = reinterpret_cast<char*>(sm + OFF_S0);
  char* cRHS = reinterpret_cast<char*>(sm + OFF_RHS);
  char* cW = reinterpret_cast<char*>(sm + OFF_W);
  char* cT = reinterpret_cast<char*>(sm + OFF_T);
  char* cMQ = reinterpret_cast<char*>(sm + OFF_MQ);
  float* Lm = reinterpret_cast<float*>(sm + OFF_LM);
  float* Tm = reinterpret_cast<float*>(sm + OFF_TM);
  float* sL = reinterpret_cast<float*>(sm + OFF_SC);
  float* sE = sL + 64;
  float* sEC = sL + 128;
  float* sCE = sL + 192;
  float* sCW = sL + 256;
  float* sKN = sL + 320;
  float* sInv = sL + 384;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  float* s_misc = reinterpret_cast<float*>(sm + OFF_BAR + 16);

  const gdnx_scan_args& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hf = warp >> 2;
  const int row = quad * 32 + lane;  // TMEM lane owned by this thread
  const int64_t n = blockIdx.x;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int lm = (int)m;
  const int dpairs = (a.rope.enable && lm < 4) ? a.rope.pairs[lm] : 0;
  const int dch = dpairs / 8;

  if (warp == 0) tc::tmem_alloc(s_tmem, TMEM_COLS);
  if (tid == 0) tc::mbar_init(mbar, 1);
  if (dpairs > 0 && tid < 64) sInv[tid] = 1.0f / powf(10000.0f, (float)tid / a.rope.den[lm]);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t lbase = (uint32_t)(quad * 32) << 16;
  const uint32_t tS = tmem, tD1 = tmem + 128, tD2 = tmem + 192;
  const uint32_t sKQ = tc::smem_u32(cKQ), sS0 = tc::smem_u32(cS0), sRHS = tc::smem_u32(cRHS);
  const uint32_t sW = tc::smem_u32(cW), sT = tc::smem_u32(cT), sMQ = tc::smem_u32(cMQ);
  constexpr uint32_t ID_N64 = tc::idesc_bf16(128, 64, false, false);
  constexpr uint32_t ID_N128_BMN = tc::idesc_bf16(128, 128, false, true);

  // ---- initial state into TMEM ----
  {
    float vals[32];
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      const int col = 64 * hf + 32 * c2;
      if (a.state_in) {
        const float* src = a.state_in + (n * VD + row) * KD + col;
#pragma unroll
        for (int e = 0; e < 32; ++e) vals[e] = src[e];
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) vals[e] = 0.f;
      }
      tc::tmem_st32(tS + lbase + col, vals);
    }
  }
  tc::fence_before();
  __syncthreads();

  uint32_t phase = 0;
  bool aborted = false;
  const int64_t nchunks = (a.T + C - 1) / C;
  for (int64_t ch = 0; ch < nchunks && !aborted; ++ch) {
    const int64_t t0 = ch * C;
    const int nt = (int)((a.T - t0) < C ? (a.T - t0) : C);

    // ================= Phase A: fused prologue =================
    for (int it = tid; it < C * 16; it += NT) {
      const int j = it >> 4, cc = it & 15;
      const bool partner_only = dch > 0 && cc >= dch && cc < 2 * dch;
      float kx[8], qx[8], k2[8], q2[8];
      float nrm = 0.f;
      if (!partner_only) {
        const bool valid = j < nt;
        const int64_t tt = t0 + j;
        if (valid) {
          load8_bf16(a.k.ptr, view_off(a.k, b, tt, h, m) + 8 * cc, kx);
          load8_bf16(a.q.ptr, view_off(a.q, b, tt, h, m) + 8 * cc, qx);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) kx[e] = qx[e] = 0.f;
        }
        if (cc < dch) {
          const int c2 = cc + dch;
          if (valid) {
            load8_bf16(a.k.ptr, view_off(a.k, b, tt, h, m) + 8 * c2, k2);
            load8_bf16(a.q.ptr, view_off(a.q, b, tt, h, m) + 8 * c2, q2);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) k2[e] = q2[e] = 0.f;
          }
          const float pos = (float)(a.rope.pos0 + tt) * a.rope.scale[lm];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float s, c;
            sincosf(pos * sInv[8 * cc + e], &s, &c);
            const float k1n = kx[e] * c - k2[e] * s;
            k2[e] = k1n * s + k2[e] * c;
            kx[e] = k1n;
            const float q1n = qx[e] * c - q2[e] * s;
            q2[e] = q1n * s + q2[e] * c;
            qx[e] = q1n;
          }
          tc::st_chunk_bf16(cKQ, tc::sw128(j, c2, 128), k2);
          tc::st_chunk_bf16(cKQ, tc::sw128(64 + j, c2, 128), q2);
#pragma unroll
          for (int e = 0; e < 8; ++e) nrm += k2[e] * k2[e];
        }
        tc::st_chunk_bf16(cKQ, tc::sw128(j, cc, 128), kx);
        tc::st_chunk_bf16(cKQ, tc::sw128(64 + j, cc, 128), qx);
#pragma unroll
        for (int e = 0; e < 8; ++e) nrm += kx[e] * kx[e];
      }
      // the 16 items of token j sit in 16 consecutive lanes
      nrm += __shfl_xor_sync(0xffffffffu, nrm, 8);
      nrm += __shfl_xor_sync(0xffffffffu, nrm, 4);
      nrm += __shfl_xor_sync(0xffffffffu, nrm, 2);
      nrm += __shfl_xor_sync(0xffffffffu, nrm, 1);
      if (cc == 0) sKN[j] = nrm;
    }
    __syncthreads();
    if (warp == 0) {
      float lg[2], ce[2], cw[2];
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int j = lane + 32 * s;
        lg[s] = 0.f; ce[s] = 0.f; cw[s] = 0.f;
        if (j < nt) {
          const int64_t tt = t0 + j;
          const int64_t dof = view_off(a.decay, b, tt, h, m);
          float l;
          if (a.decay_kind == GDNX_DECAY_LOG) {
            l = ld_as_f32(a.decay.ptr, a.decay.dtype, dof);
            if (!P.kmd2) l = fminf(l, 0.f);
          } else {
            const float g = decay_factor(a.decay, a.decay_kind, dof, !P.kmd2, a.braid_rates, a.braid_clamp);
            l = logf(fmaxf(g, 1e-30f));
          }
          lg[s] = fmaxf(l, -80.f);
          const float be = ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, tt, h, m));
          const float bw = ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, tt, h, m));
          if (P.kmd2) {
            ce[s] = be; cw[s] = bw;
          } else {
            const float al = stable_alpha(be * sKN[j]);
            ce[s] = al * be; cw[s] = al * bw;
          }
        }
      }
      // inclusive scan of the log-decays over the 64 tokens
      float s0 = lg[0], s1 = lg[1];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u0 = __shfl_up_sync(0xffffffffu, s0, o);
        const float u1 = __shfl_up_sync(0xffffffffu, s1, o);
        if (lane >= o) { s0 += u0; s1 += u1; }
      }
      s1 += __shfl_sync(0xffffffffu, s0, 31);
      const float Lc = __shfl_sync(0xffffffffu, s1, 31);
      sL[lane] = s0; sL[lane + 32] = s1;
      sE[lane] = expf(s0); sE[lane + 32] = expf(s1);
      sEC[lane] = expf(Lc - s0); sEC[lane + 32] = expf(Lc - s1);
      sCE[lane] = ce[0]; sCE[lane + 32] = ce[1];
      sCW[lane] = cw[0]; sCW[lane + 32] = cw[1];
      if (lane == 0) s_misc[0] = expf(Lc);
    }
    __syncthreads();
    // S (fp32, TMEM) -> bf16 operand tile S0; TMEM S <- e^{L_C} S
    {
      const float eLC = s_misc[0];
      float vals[32];
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        const int col = 64 * hf + 32 * c2;
        tc::tmem_ld32(tS + lbase + col, vals);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) tc::st_chunk_bf16(cS0, tc::sw128(row, col / 8 + q4, 128), vals + 8 * q4);
#pragma unroll
        for (int e = 0; e < 32; ++e) vals[e] *= eLC;
        tc::tmem_st32(tS + lbase + col, vals);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();

    // ================= Phase B: G1, G2 =================
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t ko = (s >> 2) * 16384 + (s & 3) * 32;
        const uint64_t dk = tc::smem_desc(sKQ + ko, 16, 1024);
        tc::mma_bf16(tD1, tc::smem_desc(sKQ + ko, 16, 1024), dk, ID_N64, s > 0);
        tc::mma_bf16(tD2, tc::smem_desc(sS0 + ko, 16, 1024), dk, ID_N64, s > 0);
      }
      tc::commit(mbar);
    }
    // prefetch the values this thread needs for RHS while the MMAs run
    float vv[32];
    {
      const int64_t vo = view_off(a.v, b, 0, h, m) + row;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int j = 32 * hf + e;
        vv[e] = j < nt ? ld_as_f32(a.v.ptr, a.v.dtype, vo + (t0 + j) * a.v.st) : 0.f;
      }
    }
    {
      const bool ok = tc::mbar_wait(mbar, phase & 1);
      ++phase;
      if (__syncthreads_or(!ok)) { aborted = true; break; }
    }
    tc::fence_after();

    // ================= Phase C: masks, RHS, Qd, T = (I+A)^{-1} =================
    {
      float d[32];
      tc::tmem_ld32(tD1 + lbase + 32 * hf, d);
      if (row < 64) {
        const int j = row;
        const float Lj = sL[j], cej = sCE[j];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int l = 32 * hf + e;
          Lm[j * 65 + l] = (l < j) ? cej * expf(Lj - sL[l]) * d[e] : 0.f;
        }
      } else {
        const int i = row - 64;
        const float Li = sL[i];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int jj = 32 * hf + e;
          d[e] = (jj <= i) ? expf(Li - sL[jj]) * d[e] : 0.f;
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) tc::st_chunk_bf16(cMQ, tc::sw128(i, 4 * hf + q4, 64), d + 8 * q4);
      }
      tc::tmem_ld32(tD2 + lbase + 32 * hf, d);
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int j = 32 * hf + e;
        d[e] = sCW[j] * vv[e] - sCE[j] * sE[j] * d[e];
      }
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tc::st_chunk_bf16(cRHS, tc::sw128(row, 4 * hf + q4, 128), d + 8 * q4);
      // Qd = e^{L_i} q_i in place (rows 64..127 of KQ; G1 has consumed them)
      for (int it = tid; it < C * 16; it += NT) {
        const int i = it >> 4, cc = it & 15;
        const uint32_t off = tc::sw128(64 + i, cc, 128);
        uint4 u = *reinterpret_cast<uint4*>(cKQ + off);
        __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
        const float e = sE[i];
        float x[8];
#pragma unroll
        for (int z = 0; z < 4; ++z) {
          const float2 f = __bfloat1622float2(p[z]);
          x[2 * z] = f.x * e;
          x[2 * z + 1] = f.y * e;
        }
        tc::st_chunk_bf16(cKQ, off, x);
      }
    }
    __syncthreads();
    // diagonal 16x16 blocks: warp w < 4 inverts block w, lane c < 16 builds column c
    if (warp < 4 && lane < 16) {
      const int o = 16 * warp, c = lane;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float s = (i == c) ? 1.f : 0.f;
#pragma unroll
        for (int l = 0; l < i; ++l) s -= Lm[(o + i) * 65 + o + l] * x[l];
        x[i] = s;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) Tm[(o + i) * 65 + o + c] = x[i];
    }
    __syncthreads();
    // off-diagonal blocks by distance d:  T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj.
    // The partial sum X_ij is parked in the (unused) upper block (j, i) of Tm.
    for (int dd = 1; dd < 4; ++dd) {
      const int nblk = 4 - dd;
      for (int o = tid; o < nblk * 256; o += NT) {
        const int bj = o >> 8, bi = bj + dd, rr = (o >> 4) & 15, cc = o & 15;
        float s = 0.f;
        for (int bk = bj; bk < bi; ++bk) {
#pragma unroll
          for (int t = 0; t < 16; ++t) s += Lm[(16 * bi + rr) * 65 + 16 * bk + t] * Tm[(16 * bk + t) * 65 + 16 * bj + cc];
        }
        Tm[(16 * bj + rr) * 65 + 16 * bi + cc] = s;
      }
      __syncthreads();
      for (int o = tid; o < nblk * 256; o += NT) {
        const int bj = o >> 8, bi = bj + dd, rr = (o >> 4) & 15, cc = o & 15;
        float s = 0.f;
#pragma unroll
        for (int t = 0; t < 16; ++t) s += Tm[(16 * bi + rr) * 65 + 16 * bi + t] * Tm[(16 * bj + t) * 65 + 16 * bi + cc];
        Tm[(16 * bi + rr) * 65 + 16 * bj + cc] = -s;
      }
      __syncthreads();
    }
    // T -> bf16 operand tile (rows j, K = l), zero above the block diagonal
    for (int it = tid; it < C * 8; it += NT) {
      const int j = it >> 3, cc = it & 7;
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int l = 8 * cc + e;
        x[e] = ((l >> 4) <= (j >> 4)) ? Tm[j * 65 + l] : 0.f;
      }
      tc::st_chunk_bf16(cT, tc::sw128(j, cc, 64), x);
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();

    // ================= Phase D: G4 (W), G3 (S0 Qd) =================
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma_bf16(tD2, tc::smem_desc(sRHS + s * 32, 16, 1024), tc::smem_desc(sT + s * 32, 16, 1024), ID_N64, s > 0);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t ko = (s >> 2) * 16384 + (s & 3) * 32;
        tc::mma_bf16(tD1, tc::smem_desc(sS0 + ko, 16, 1024), tc::smem_desc(sKQ + ko + 64 * 128, 16, 1024), ID_N64,
                     s > 0);
      }
      tc::commit(mbar);
    }
    {
      const bool ok = tc::mbar_wait(mbar, phase & 1);
      ++phase;
      if (__syncthreads_or(!ok)) { aborted = true; break; }
    }
    tc::fence_after();

    // ================= Phase E: W^T -> bf16 tiles W and W' = W e^{L_C - L_j} =================
    {
      float w[32], w2[32];
      tc::tmem_ld32(tD2 + lbase + 32 * hf, w);
#pragma unroll
      for (int e = 0; e < 32; ++e) w2[e] = w[e] * sEC[32 * hf + e];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        tc::st_chunk_bf16(cW, tc::sw128(row, 4 * hf + q4, 128), w + 8 * q4);
        tc::st_chunk_bf16(cRHS, tc::sw128(row, 4 * hf + q4, 128), w2 + 8 * q4);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();

    // ================= Phase F: G5 (y += W Mq), G6 (S += W' K) =================
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma_bf16(tD1, tc::smem_desc(sW + s * 32, 16, 1024), tc::smem_desc(sMQ + s * 32, 16, 1024), ID_N64, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma_bf16(tS, tc::smem_desc(sRHS + s * 32, 16, 1024), tc::smem_desc(sKQ + s * 2048, 16384, 1024),
                     ID_N128_BMN, 1);
      tc::commit(mbar);
    }
    {
      const bool ok = tc::mbar_wait(mbar, phase & 1);
      ++phase;
      if (__syncthreads_or(!ok)) { aborted = true; break; }
    }
    tc::fence_after();

    // ================= Phase G: outputs =================
    {
      float yv[32];
      tc::tmem_ld32(tD1 + lbase + 32 * hf, yv);
      const int64_t yo = b * a.y_sb + h * a.y_sh + m * a.y_sm + row;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int i = 32 * hf + e;
        if (i < nt) st_from_f32(a.y, a.y_dtype, yo + (t0 + i) * a.y_st, yv[e]);
      }
    }
    tc::fence_before();
    __syncthreads();
  }

  if (!aborted && a.state_out) {
    tc::fence_after();
    float vals[32];
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      const int col = 64 * hf + 32 * c2;
      tc::tmem_ld32(tS + lbase + col, vals);
      float* dst = a.state_out + (n * VD + row) * KD + col;
#pragma unroll
      for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(vals[e], vals[e + 1], vals[e + 2], vals[e + 3]);
    }
  }
  if (aborted && tid == 0 && P.err) atomicExch(P.err, (int)GDNX_ETIMEOUT);
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool chunked_eligible(const gdnx_scan_args& a) {
  if (a.algo == GDNX_ALGO_RECURRENT) return false;
  if (a.K != KD || a.V != VD || (a.chunk != 0 && a.chunk != C)) return false;
  if (a.r_out != 1) return false;
  if (a.scores) return false;  // update-norm scores are produced by the recurrent kernel only
  if (a.gate_e.dim != 1 || a.gate_w.dim != 1) return false;
  if (a.decay.dim != 1 && a.decay_kind != GDNX_DECAY_BRAIDED) return false;
  if (a.q.dtype != GDNX_BF16 || a.k.dtype != GDNX_BF16) return false;
  if (!aligned16(a.q.ptr) || !aligned16(a.k.ptr)) return false;
  const int64_t st[8] = {a.q.sb, a.q.st, a.q.sh, a.q.sm, a.k.sb, a.k.st, a.k.sh, a.k.sm};
  for (int i = 0; i < 8; ++i)
    if (st[i] % 8) return false;
  if (a.rope.enable)
    for (int i = 0; i < 4; ++i)
      if (a.rope.pairs[i] % 8) return false;
  if (a.state_in && !aligned16(a.state_in)) return false;
  if (a.state_out && !aligned16(a.state_out)) return false;
  return true;
}

size_t chunked_workspace_bytes(const gdnx_scan_args&) { return 256; }  // device error word

gdnx_status launch_chunked_scan(const gdnx_scan_args& a, cudaStream_t st) {
  ChunkParams P;
  P.a = a;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.err = reinterpret_cast<int*>(a.workspace);
  if (cudaFuncSetAttribute(chunked_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
      cudaSuccess)
    return GDNX_ELAUNCH;
  const int64_t N = a.B * a.H * a.M;
  chunked_scan_kernel<<<(unsigned)N, NT, SMEM_BYTES, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the scratch (the kernel's device error word) sits in
// a file-scope device array instead of a caller-provided workspace.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = 256;  // maximum scratch this variant offers
static __device__ __align__(256) unsigned char g_chunked_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};  // device address of g_chunked_scratch, per device

// Looks up the array's device address once per device, with that device current.
gdnx_status static_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDNX_ELAUNCH;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_chunked_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return GDNX_ELAUNCH;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return GDNX_OK;
}

}  // namespace

gdnx_status launch_chunked_scan_static_scratch(const gdnx_scan_args& a, cudaStream_t st) {
  if (!chunked_eligible(a)) return GDNX_EUNSUPPORTED;
  if (chunked_workspace_bytes(a) > kStaticScratchBytes) return GDNX_EWORKSPACE;
  void* scratch = nullptr;
  const gdnx_status s = static_scratch(&scratch);
  if (s != GDNX_OK) return s;
  // the error word must start at zero on every call
  if (cudaMemsetAsync(scratch, 0, kStaticScratchBytes, st) != cudaSuccess) return GDNX_ELAUNCH;
  ChunkParams P;
  P.a = a;
  P.a.workspace = scratch;
  P.a.workspace_bytes = kStaticScratchBytes;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.err = reinterpret_cast<int*>(scratch);
  if (cudaFuncSetAttribute(chunked_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
      cudaSuccess)
    return GDNX_ELAUNCH;
  const int64_t N = a.B * a.H * a.M;
  chunked_scan_kernel<<<(unsigned)N, NT, SMEM_BYTES, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
