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

#include "chunk_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace gdnx {
namespace {

using namespace chunk;

constexpr int C = 64;         // chunk length
constexpr int KD = 128;       // key dim
constexpr int VD = 128;       // value dim
constexpr int NT = 512;       // threads: 16 warps, four per TMEM lane quadrant
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
constexpr int OFF_STQ = OFF_SC + 7 * 64 * 4;  // bf16 [64 tokens][128] raw q of the next chunk (cp.async)
constexpr int OFF_STK = OFF_STQ + 16384;       // raw k
constexpr int OFF_STV = OFF_STK + 16384;       // raw v
constexpr int OFF_BAR = OFF_STV + 16384;
constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;  // + alignment slack

struct ChunkParams {
  gdnx_scan_args a;
  int kmd2;
  int* err;
};


__device__ __forceinline__ void bulk_row(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(mbar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(mbar), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(NT, 1) chunked_scan_kernel(const ChunkParams P) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = tc::align_smem(smraw, 1024);
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
  const char* cSTQ = reinterpret_cast<const char*>(sm + OFF_STQ);
  const char* cSTK = reinterpret_cast<const char*>(sm + OFF_STK);
  const __nv_bfloat16* hSTV = reinterpret_cast<const __nv_bfloat16*>(sm + OFF_STV);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  float* s_misc = reinterpret_cast<float*>(sm + OFF_BAR + 16);
  uint64_t* stage_bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 32);

  const gdnx_scan_args& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, qg = warp >> 2;  // lane quadrant, column group (0..3)
  const int row = quad * 32 + lane;  // TMEM lane owned by this thread
  const int64_t n = blockIdx.x;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int lm = (int)m;
  const int dpairs = (a.rope.enable && lm < 4) ? a.rope.pairs[lm] : 0;
  const int dch = dpairs / 8;

  if (warp == 0) tc::tmem_alloc(s_tmem, TMEM_COLS);
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    tc::mbar_init(stage_bar, 1);
  }
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
    for (int c2 = 0; c2 < 1; ++c2) {
      const int col = 32 * qg;
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
  const bool braided = a.decay_kind == GDNX_DECAY_BRAIDED;
  const bool y_tile = a.y_dtype == GDNX_BF16 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 &&
                      a.y_sb % 8 == 0 && a.y_st % 8 == 0 && a.y_sh % 8 == 0 && a.y_sm % 8 == 0;
  // next-chunk prefetch: q/k/v rows into the staging tiles with cp.async, and the
  // per-token scalars (raw bits) into warp 0's registers
  uint32_t pr_be[2], pr_bw[2], pr_dec[2][4];
  // Next-chunk staging of the raw q/k/v rows: one 256-byte bulk copy per token row
  // (3 x 64 per chunk, issued by warps 0-5), counted on stage_bar; rows past T are
  // zero-filled with plain stores instead.
  const __nv_bfloat16* pf_src = nullptr;
  int64_t pf_st = 0;
  if (warp < 6) {
    const gdnx_view& vw = warp < 2 ? a.q : (warp < 4 ? a.k : a.v);
    pf_src = reinterpret_cast<const __nv_bfloat16*>(vw.ptr) + view_off(vw, b, 0, h, m);
    pf_st = vw.st;
  }
  const uint32_t sbar = tc::smem_u32(stage_bar);
  const uint32_t pf_dst = tc::smem_u32(sm + OFF_STQ) + (warp >> 1) * 16384 + ((warp & 1) * 32 + lane) * 256;
  uint32_t stage_phase = 0;
  auto prefetch_rows = [&](int64_t chn, int, int) {
    const int64_t tb = chn * C;
    const int nv = (int)((a.T - tb) < C ? (a.T - tb) : C);
    if (tid == 0) mbar_expect_tx(sbar, 3u * nv * 256u);
    __syncwarp();
    if (warp < 6) {
      const int j = (warp & 1) * 32 + lane;
      if (j < nv) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bulk_row(pf_dst, pf_src + (tb + j) * pf_st, 256, sbar);
      } else {
        uint4* z = reinterpret_cast<uint4*>(sm + OFF_STQ + (warp >> 1) * 16384 + j * 256);
#pragma unroll
        for (int c = 0; c < 16; ++c) z[c] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  const int64_t sc_e0 = view_off(a.gate_e, b, 0, h, m), sc_w0 = view_off(a.gate_w, b, 0, h, m);
  const int64_t sc_d0 = view_off(a.decay, b, 0, h, m);
  auto prefetch_scalars = [&](int64_t chn) {
    if (warp != 0) return;
    const int64_t tb = chn * C;
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2) {
      const int64_t tt = tb + lane + 32 * s2;
      pr_be[s2] = pr_bw[s2] = 0u;
#pragma unroll
      for (int z = 0; z < 4; ++z) pr_dec[s2][z] = 0u;
      if (tt < a.T) {
        pr_be[s2] = ld_raw(a.gate_e.ptr, a.gate_e.dtype, sc_e0 + tt * a.gate_e.st);
        pr_bw[s2] = ld_raw(a.gate_w.ptr, a.gate_w.dtype, sc_w0 + tt * a.gate_w.st);
#pragma unroll
        for (int z = 0; z < 4; ++z)
          if (z == 0 || braided) pr_dec[s2][z] = ld_raw(a.decay.ptr, a.decay.dtype, sc_d0 + tt * a.decay.st + z);
      }
    }
  };
  prefetch_rows(0, 0, 3);
  prefetch_scalars(0);
  for (int64_t ch = 0; ch < nchunks && !aborted; ++ch) {
    const int64_t t0 = ch * C;
    const int nt = (int)((a.T - t0) < C ? (a.T - t0) : C);

    // ================= Phase A: fused prologue =================
    {
      // staged rows of this chunk: bulk copies (mbarrier) and zero-filled tails (barrier)
      const bool ok = tc::mbar_wait(stage_bar, stage_phase & 1);
      ++stage_phase;
      if (__syncthreads_or(!ok)) { aborted = true; break; }
    }
    // RoPE angle table for the chunk (spread evenly over all threads), parked in Tm
    float* tabC = Tm;
    float* tabS = Tm + C * 32;
    if (dpairs > 0) {
      const float sc = a.rope.scale[lm];
      for (int idx = tid; idx < C * dpairs; idx += NT) {
        const int j = idx / dpairs, i = idx - j * dpairs;
        float sn, cs;
        sincos_reduced((float)(a.rope.pos0 + t0 + j) * sc * sInv[i], &sn, &cs);
        tabC[j * 32 + i] = cs;
        tabS[j * 32 + i] = sn;
      }
      __syncthreads();
    }
    for (int it = tid; it < C * 16; it += NT) {
      const int j = it >> 4, cc = it & 15;
      const bool partner_only = dch > 0 && cc >= dch && cc < 2 * dch;
      float kx[8], qx[8], k2[8], q2[8];
      float nrm = 0.f;
      if (!partner_only) {
        load8_bf16(cSTK, j * 128 + 8 * cc, kx);
        load8_bf16(cSTQ, j * 128 + 8 * cc, qx);
        if (cc < dch) {
          const int c2 = cc + dch;
          load8_bf16(cSTK, j * 128 + 8 * c2, k2);
          load8_bf16(cSTQ, j * 128 + 8 * c2, q2);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float s = tabS[j * 32 + 8 * cc + e], c = tabC[j * 32 + 8 * cc + e];
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
          float l;
          if (a.decay_kind == GDNX_DECAY_LOG) {
            l = raw_f32(pr_dec[s][0], a.decay.dtype);
            if (!P.kmd2) l = fminf(l, 0.f);
          } else if (braided) {
            float acc = 0.f;
#pragma unroll
            for (int z = 0; z < 4; ++z)
              acc += expf(-fminf(softplus_f(raw_f32(pr_dec[s][z], a.decay.dtype)), 5.0f) * a.braid_rates[z]);
            l = logf(fmaxf(fminf(acc * 0.25f, a.braid_clamp), 1e-30f));
          } else {
            float g = raw_f32(pr_dec[s][0], a.decay.dtype);
            if (!P.kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
            l = logf(fmaxf(g, 1e-30f));
          }
          lg[s] = fmaxf(l, -80.f) * 1.4426950408889634f;  // log2 units from here on
          const float be = raw_f32(pr_be[s], a.gate_e.dtype);
          const float bw = raw_f32(pr_bw[s], a.gate_w.dtype);
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
      sE[lane] = exp2f(s0); sE[lane + 32] = exp2f(s1);
      sEC[lane] = exp2f(Lc - s0); sEC[lane + 32] = exp2f(Lc - s1);
      sCE[lane] = ce[0]; sCE[lane + 32] = ce[1];
      sCW[lane] = cw[0]; sCW[lane + 32] = cw[1];
      if (lane == 0) s_misc[0] = exp2f(Lc);
    }
    __syncthreads();
    // S (fp32, TMEM) -> bf16 operand tile S0; TMEM S <- e^{L_C} S
    {
      const float eLC = s_misc[0];
      float vals[32];
#pragma unroll
      for (int c2 = 0; c2 < 1; ++c2) {
        const int col = 32 * qg;
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
    {
      const bool ok = tc::mbar_wait(mbar, phase & 1);
      ++phase;
      if (__syncthreads_or(!ok)) { aborted = true; break; }
    }
    tc::fence_after();

    // ================= Phase C: masks, RHS, Qd, T = (I+A)^{-1} =================
    {
      float d[16];
      tc::tmem_ld16(tD1 + lbase + 16 * qg, d);
      if (row < 64) {
        const int j = row;
        const float Lj = sL[j], cej = sCE[j];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int l = 16 * qg + e;
          Lm[j * 65 + l] = (l < j) ? cej * exp2f(Lj - sL[l]) * d[e] : 0.f;
        }
      } else {
        const int i = row - 64;
        const float Li = sL[i];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int jj = 16 * qg + e;
          d[e] = (jj <= i) ? exp2f(Li - sL[jj]) * d[e] : 0.f;
        }
#pragma unroll
        for (int q4 = 0; q4 < 2; ++q4) tc::st_chunk_bf16(cMQ, tc::sw128(i, 2 * qg + q4, 64), d + 8 * q4);
      }
      tc::tmem_ld16(tD2 + lbase + 16 * qg, d);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = 16 * qg + e;
        d[e] = sCW[j] * __bfloat162float(hSTV[j * VD + row]) - sCE[j] * sE[j] * d[e];
      }
#pragma unroll
      for (int q4 = 0; q4 < 2; ++q4) tc::st_chunk_bf16(cRHS, tc::sw128(row, 2 * qg + q4, 128), d + 8 * q4);
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
    if (ch + 1 < nchunks) {  // this chunk's staged rows and scalars are consumed: fetch the next
      prefetch_rows(ch + 1, 0, 3);
      prefetch_scalars(ch + 1);
    }
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
    // Off-diagonal blocks.  With P_ij = T_ii A_ij (i > j, all six formed in one step and
    // parked in the unused upper block (j, i)):  T_ij = -sum_{k=j}^{i-1} P_ik T_kj,
    // evaluated by block distance 1, 2, 3.
    for (int o = tid; o < 6 * 256; o += NT) {
      const int pb = o >> 8, rr = (o >> 4) & 15, cc = o & 15;
      const int bi = pb < 3 ? pb + 1 : (pb < 5 ? pb - 1 : 3);   // (1,0) (2,1) (3,2) (2,0) (3,1) (3,0)
      const int bj = pb < 3 ? pb : (pb < 5 ? pb - 3 : 0);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int t = 0; t < 16; t += 2) {
        s0 = fmaf(Tm[(16 * bi + rr) * 65 + 16 * bi + t], Lm[(16 * bi + t) * 65 + 16 * bj + cc], s0);
        s1 = fmaf(Tm[(16 * bi + rr) * 65 + 16 * bi + t + 1], Lm[(16 * bi + t + 1) * 65 + 16 * bj + cc], s1);
      }
      Tm[(16 * bj + rr) * 65 + 16 * bi + cc] = s0 + s1;
    }
    __syncthreads();
    for (int dd = 1; dd < 4; ++dd) {
      for (int o = tid; o < (4 - dd) * 256; o += NT) {
        const int bj = o >> 8, bi = bj + dd, rr = (o >> 4) & 15, cc = o & 15;
        float s0 = 0.f, s1 = 0.f;
        for (int bk = bj; bk < bi; ++bk) {
          const float* pr = Tm + (16 * bk + rr) * 65 + 16 * bi;   // P_{i,k}[rr][:]
          const float* tc_ = Tm + (16 * bk) * 65 + 16 * bj + cc;  // T_{k,j}[:][cc]
#pragma unroll
          for (int t = 0; t < 16; t += 2) {
            s0 = fmaf(pr[t], tc_[t * 65], s0);
            s1 = fmaf(pr[t + 1], tc_[(t + 1) * 65], s1);
          }
        }
        Tm[(16 * bi + rr) * 65 + 16 * bj + cc] = -(s0 + s1);
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
      float w[16], w2[16];
      tc::tmem_ld16(tD2 + lbase + 16 * qg, w);
#pragma unroll
      for (int e = 0; e < 16; ++e) w2[e] = w[e] * sEC[16 * qg + e];
#pragma unroll
      for (int q4 = 0; q4 < 2; ++q4) {
        tc::st_chunk_bf16(cW, tc::sw128(row, 2 * qg + q4, 128), w + 8 * q4);
        tc::st_chunk_bf16(cRHS, tc::sw128(row, 2 * qg + q4, 128), w2 + 8 * q4);
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
      float yv[16];
      tc::tmem_ld16(tD1 + lbase + 16 * qg, yv);
      if (y_tile) {
        // stage the chunk's outputs as bf16 [token][v] (in the A-matrix scratch), then
        // write each token's 256-byte row with 16-byte stores
        __nv_bfloat16* ys = reinterpret_cast<__nv_bfloat16*>(Lm);
#pragma unroll
        for (int e = 0; e < 16; ++e) ys[(16 * qg + e) * VD + row] = __float2bfloat16_rn(yv[e]);
        __syncthreads();
        const int64_t ybase = b * a.y_sb + h * a.y_sh + m * a.y_sm;
        for (int it = tid; it < C * 16; it += NT) {
          const int i = it >> 4, cc = it & 15;
          if (i < nt)
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y) + ybase + (t0 + i) * a.y_st + 8 * cc) =
                *reinterpret_cast<const uint4*>(ys + i * VD + 8 * cc);
        }
      } else {
        const int64_t yo = b * a.y_sb + h * a.y_sh + m * a.y_sm + row;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int i = 16 * qg + e;
          if (i < nt) st_from_f32(a.y, a.y_dtype, yo + (t0 + i) * a.y_st, yv[e]);
        }
      }
    }
    tc::fence_before();
    __syncthreads();
  }

  if (!aborted && a.state_out) {
    tc::fence_after();
    float vals[32];
#pragma unroll
    for (int c2 = 0; c2 < 1; ++c2) {
      const int col = 32 * qg;
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
  if (a.v.dtype != GDNX_BF16) return false;
  if (!aligned16(a.q.ptr) || !aligned16(a.k.ptr) || !aligned16(a.v.ptr)) return false;
  const int64_t st[12] = {a.q.sb, a.q.st, a.q.sh, a.q.sm, a.k.sb, a.k.st, a.k.sh, a.k.sm,
                          a.v.sb, a.v.st, a.v.sh, a.v.sm};
  for (int i = 0; i < 12; ++i)
    if (st[i] % 8) return false;
  if (a.rope.enable)
    for (int i = 0; i < 4; ++i)
      if (a.rope.pairs[i] % 8) return false;
  if (a.state_in && !aligned16(a.state_in)) return false;
  if (a.state_out && !aligned16(a.state_out)) return false;
  return true;
}

size_t chunked_workspace_bytes(const gdnx_scan_args& a) { return wy_workspace_bytes(a); }

// Single-pass kernel: needs only the device error word (the first 256 bytes).
gdnx_status launch_fused_chunked_scan(const gdnx_scan_args& a, cudaStream_t st) {
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

gdnx_status launch_chunked_scan(const gdnx_scan_args& a, cudaStream_t st) {
  const gdnx_status s = launch_wy_scan(a, st);
  return s == GDNX_EUNSUPPORTED ? launch_fused_chunked_scan(a, st) : s;
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the scratch (the kernel's device error word) sits in
// a file-scope device array instead of a caller-provided workspace.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = 256;  // maximum scratch this variant offers
static __device__ __align__(256) unsigned char g_chunked_scratch[kStaticScratchBytes];
// The single-pass kernel's whole scratch need is its int32 error word; a kernel change
// that needs more must grow the array (or this entry point must reject the request).
static_assert(sizeof(int) <= kStaticScratchBytes, "the chunked kernel's scratch fits the static array");

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

gdnx_status static_scratch_status(int* out, cudaStream_t st) {
  void* scratch = nullptr;
  const gdnx_status s = static_scratch(&scratch);
  if (s != GDNX_OK) return s;
  int word = 0;
  if (cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return GDNX_ELAUNCH;
  *out = word;
  return GDNX_OK;
}

gdnx_status launch_chunked_scan_static_scratch(const gdnx_scan_args& a, cudaStream_t st) {
  if (!chunked_eligible(a)) return GDNX_EUNSUPPORTED;
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
