// Two-pass chunked gated-delta scan on sm_100a (dense GDN3 / KMD-2 with
// per-chain scalar gates and decay, d_k = d_v = 128, C = 64).
//
// The delta rule over one chunk of one chain (tokens j = 0..63, log2 decay
// prefix L_j, erase/write coefficients ce_j, cw_j; gdn3/_reference_recurrence.py:61-84,
// research/kernel_ab/ref_scan.py:40-47 for the single-token step) is, in the
// WY/UT form,
//   A   = strictly-lower( ce_j 2^{L_j - L_l} k_j.k_l )          (64 x 64)
//   T   = (I + A)^{-1}
//   W   = T diag(cw) V - T diag(ce 2^L) K S0^T                 (64 x 128)
//   y_i = 2^{L_i} S0 q_i + sum_{j<=i} 2^{L_i - L_j} (q_i.k_j) W_j
//   S   = 2^{L_C} S0 + sum_j 2^{L_C - L_j} W_j k_j^T
// Everything before the first use of S0 is independent of the state, so it is
// split off:
//   pass 1 (wy_prep_kernel, one CTA per pair of chunks, all chunks in parallel):
//     lane RoPE on k, gates (alpha, ce, cw), decay prefix L, the Gram matrix
//     k k^T on the tensor cores, the masks, T by forward substitution in fp32,
//     and T_e = T diag(ce 2^L), T_w = T diag(cw) written as bf16 tiles already
//     in the 128-byte-swizzled UMMA layout, plus L.
//   pass 2 (wy_scan_kernel, one CTA per chain, chunks in sequence):
//     TMA loads of q/k/v (two stages ahead), bulk loads of T_e, T_w, L,
//     lane RoPE of q/k in shared memory, then three tcgen05 groups per chunk:
//       G1  [K;Q] K^T -> masks, K^T T_e^T -> Wk^T, V^T T_w^T -> W^T (init),
//           S0 Q^T -> y_S                                    (S0 = bf16 state)
//       G2  W^T -= S0 Wk^T
//       G3  y_W = W^T Mq^T,  S += W'^T K                    (K read MN-major)
//     with the fp32 state in TMEM for the whole sequence.
// The state is kept as S = 2^{ls} S_tmem with a running log2 scale ls, so the
// per-chunk decay 2^{L_C} is folded into scalars of the read-outs instead of a
// TMEM read-modify-write; the scale is applied to TMEM and reset when ls < -40
// and on chunks that take the exact path (see FOLD_MIN_LC).  Every mbarrier wait is bounded (GDNX_ETIMEOUT in the
// workspace error word, TMEM freed, kernel returns).
#include <cuda.h>
#include <cstdlib>
#include <mutex>

#include "chunk_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace gdnx {
namespace {

using namespace chunk;

constexpr int C = 64;
constexpr int KD = 128;
constexpr int VD = 128;
constexpr int LDA = 68;                    // fp32 row stride of the A matrices (16-byte rows)
constexpr int64_t TT_ELEMS = 3 * C * C;    // bf16 elements of T_e, T_w, Mq^T per chain-chunk
constexpr size_t ERR_BYTES = 256;
// Chunks whose total log2 decay L_C is at least this take the folded path: the chunk's
// decays go into scalars of the read-outs instead of passes over q and k.  With the
// state held as 2^{ls} S_tmem (ls in [-40, 0] at the chunk start), pass 1 stores the
// undecayed mask Mq_il = q_i.k_l (l <= i), pass 2 writes -Wk 2^{ls} as the G2 operand,
// reads W out as W diag(f), f_l = 2^{-L_l - ls} (<= 2^100), updates S_tmem += (W diag f)^T K
// and scales y_i by 2^{L_i + ls}.  Below it (the exact path), the state is normalised
// to ls = 0 and scaled by 2^{L_C} in TMEM, pass 1 stores Mq_il = 2^{L_i - L_l} q_i.k_l and
// pass 2 forms Qd = 2^{L} q and K' = 2^{L_C - L} k in shared memory.
constexpr float FOLD_MIN_LC = -60.f;

struct WyScanMaps {
  CUtensorMap q, k, v, y;
  int use_m[4];  // per map: 1 if the lane coordinate is a real dimension
  int y_tma;     // y written with TMA stores (bf16, 16-byte strides)
};

GDNX_DEV void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                          uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(mbar)
      : "memory");
}
GDNX_DEV void tma_store_5d(const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4, uint32_t src) {
  asm volatile(
      "cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4, %5}], [%6];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(src)
      : "memory");
}
GDNX_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
GDNX_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
GDNX_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
GDNX_DEV void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
}
GDNX_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(mbar)
               : "memory");
}
GDNX_DEV void expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes) : "memory");
}

// ------------------------------- pass 1 ------------------------------------
constexpr int P_NT = 256;
constexpr int P_STORE_TID = 128;  // issues (and waits for) the Mq^T bulk stores; thread 0 issues the MMAs
// [2 kb][256 rows][128 B] bf16, rows: Qa | Ka | Qb | Kb (a, b: the pair's chunks), so that
// Ka / Kb (rows 64-127 / 192-255) are the A operands and [Qa;Ka] / [Qb;Kb] (rows 0-127 /
// 128-255) the B operands of the two Gram products
constexpr int P_OFF_KQ = 0;
constexpr int P_OFF_A = 0;                          // fp32 [2][64][LDA] over the tiles after the MMAs
constexpr int P_OFF_MQS = 36864;                    // Mq^T staging [2][64 l][64 i] bf16 over the tiles
constexpr int P_OFF_L1 = 53248;                     // level-1 block-product operands (see the kernel)
constexpr int P_OFF_L1A2 = P_OFF_L1 + 8192;
constexpr int P_OFF_L1B2 = P_OFF_L1A2 + 2048;
constexpr int P_OFF_L2 = P_OFF_MQS;                 // level-2 operands, once the Mq^T staging is stored
constexpr int P_OFF_L2B = P_OFF_L2 + 8192;
constexpr int P_OFF_L2B2 = P_OFF_L2B + 4096;
constexpr int P_OFF_SC = P_OFF_KQ + 65536;          // L, ce, cw, kn, 2^-L [2][64] each; inv_freq [64]
constexpr int P_OFF_BAR = P_OFF_SC + (10 * 64 + 64) * 4;
constexpr int P_SMEM = P_OFF_BAR + 64 + 1024;
static_assert(2 * C * LDA * 4 <= P_OFF_MQS && P_OFF_MQS + 16384 <= 65536, "A and Mq^T over the k/q tiles");

struct WyParams {
  gdnx_scan_args a;
  int kmd2;
  int64_t nchunks;
  __nv_bfloat16* tt;  // [N][nchunks][3][64*64] bf16 (T_e, T_w, Mq^T; swizzled tiles)
  float* lsum;        // [N][nchunks][64] log2 decay prefix
  int* err;
  int64_t n0;         // first chain of this launch (a launch covers chains n0 .. n0 + grid chains - 1)
};

// Forward substitution for column c of one 16 x 16 diagonal block of T = (I + A)^{-1}
// (block rows / columns B0 .. B0 + 15); x[i] = T[B0 + i][B0 + c].  The block's values
// are written back over A's block (its strictly-lower part is consumed).
GDNX_DEV void subst_block16(float* A, int B0, int c, float* x) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float s0 = (i == c) ? 1.f : 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int l = 0; l < i; l += 4) {
      const float4 a4 = *reinterpret_cast<const float4*>(A + (B0 + i) * LDA + B0 + l);
      s0 = fmaf(-a4.x, x[l], s0);
      if (l + 1 < i) s1 = fmaf(-a4.y, x[l + 1], s1);
      if (l + 2 < i) s2 = fmaf(-a4.z, x[l + 2], s2);
      if (l + 3 < i) s3 = fmaf(-a4.w, x[l + 3], s3);
    }
    x[i] = (s0 + s1) + (s2 + s3);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 16; ++i) A[(B0 + i) * LDA + B0 + c] = x[i];
}


__global__ void __launch_bounds__(P_NT, 3) wy_prep_kernel(const WyParams P, const __grid_constant__ WyScanMaps maps) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = tc::align_smem(smraw, 1024);
  char* cKQ = reinterpret_cast<char*>(sm + P_OFF_KQ);
  float* sA = reinterpret_cast<float*>(sm + P_OFF_A);
  float* sL = reinterpret_cast<float*>(sm + P_OFF_SC);  // [2][64] log2 decay prefix
  float* sCE = sL + 128;                                // T_e column factor ce_l 2^{L_l}
  float* sCW = sL + 256;
  float* sKN = sL + 384;  // |k|^2
  float* sInv = sL + 512;
  float* sNE = sL + 576;  // [2][64] 2^{-L_l}
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);
  uint64_t* tbar = mbar + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + P_OFF_BAR + 16);

  const gdnx_scan_args& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t npairs = (P.nchunks + 1) / 2;
  const int64_t n = P.n0 + blockIdx.x / npairs, pair = blockIdx.x % npairs;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int lm = (int)m;
  const int dpairs = (a.rope.enable && lm < 4) ? a.rope.pairs[lm] : 0;
  const int dch = dpairs / 8;
  const int64_t tbase = pair * 2 * C;  // first token of the pair
  const uint32_t sKQ = tc::smem_u32(cKQ);
  const bool braided = a.decay_kind == GDNX_DECAY_BRAIDED;

  // Set-up work away from warps 0-1 (the decay prefix) and thread 0 (the MMA issuer):
  // warp 7 issues the tile loads, warp 6 allocates TMEM, warps 2-3 the RoPE frequencies.
  if (tid == 224) {
    tc::mbar_init(mbar, 1);
    tc::mbar_init(tbar, 1);
    // rows Qa | Ka | Qb | Kb of each K block (TMA zero-fills tokens past T)
    const uint32_t bar = tc::smem_u32(tbar);
    expect_tx(bar, 8 * 8192);
    const int ck_m = maps.use_m[1] ? lm : 0, cq_m = maps.use_m[0] ? lm : 0;
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      const uint32_t blk = sKQ + kb * 32768;
      tma_load_5d(blk, &maps.q, 64 * kb, cq_m, (int)h, (int)tbase, (int)b, bar);
      tma_load_5d(blk + 8192, &maps.k, 64 * kb, ck_m, (int)h, (int)tbase, (int)b, bar);
      tma_load_5d(blk + 16384, &maps.q, 64 * kb, cq_m, (int)h, (int)(tbase + C), (int)b, bar);
      tma_load_5d(blk + 24576, &maps.k, 64 * kb, ck_m, (int)h, (int)(tbase + C), (int)b, bar);
    }
  }
  // this thread: token j of chunk ci, the TMEM lane of row j of that chunk's M = 64 Gram
  // accumulator (lane 32 q + 16 ci + j % 16 of quadrant q = j / 16); warps 0-3 / 4-7 take
  // the 32-column halves h of its masks row (k_j.k_l) and Mq^T row (k_j.q_i)
  const int quad = warp & 3, half = warp >> 2;
  const int ci = lane >> 4, j = 16 * quad + (lane & 15);
  const int64_t tj = tbase + ci * C + j;
  // gate and decay loads first, as raw bits (converted where used, so nothing waits on them
  // here): their latency overlaps the set-up and the tile loads
  uint32_t rbe = 0, rbw = 0, rdec[2] = {0, 0};
  if (tj < a.T) {
    rbe = ld_raw(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, tj, h, m));
    rbw = ld_raw(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, tj, h, m));
  }
  if (warp < 2 && !braided) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int64_t t = tbase + warp * C + lane + 32 * s;
      if (t < a.T) rdec[s] = ld_raw(a.decay.ptr, a.decay.dtype, view_off(a.decay, b, t, h, m));
    }
  }
  if (warp == 6) tc::tmem_alloc(s_tmem, 128);
  if (dpairs > 0 && tid >= 64 && tid < 128) sInv[tid - 64] = 1.0f / powf(10000.0f, (float)(tid - 64) / a.rope.den[lm]);
  // warps 0, 1: log2 decay prefix of chunk `warp` (independent of k)
  if (warp < 2) {
    float lg[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int64_t t = tbase + warp * C + lane + 32 * s;
      lg[s] = 0.f;
      if (t < a.T) {
        const int64_t od = view_off(a.decay, b, t, h, m);
        float l;
        if (a.decay_kind == GDNX_DECAY_LOG) {
          l = raw_f32(rdec[s], a.decay.dtype);
          if (!P.kmd2) l = fminf(l, 0.f);
        } else if (braided) {
          float acc = 0.f;
#pragma unroll
          for (int z = 0; z < 4; ++z)
            acc += expf(-fminf(softplus_f(ld_as_f32(a.decay.ptr, a.decay.dtype, od + z)), 5.0f) * a.braid_rates[z]);
          l = logf(fmaxf(fminf(acc * 0.25f, a.braid_clamp), 1e-30f));
        } else {
          float g = raw_f32(rdec[s], a.decay.dtype);
          if (!P.kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
          l = logf(fmaxf(g, 1e-30f));
        }
        lg[s] = fmaxf(l, -80.f) * 1.4426950408889634f;  // log2 units
      }
    }
    float s0 = lg[0], s1 = lg[1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u0 = __shfl_up_sync(0xffffffffu, s0, o);
      const float u1 = __shfl_up_sync(0xffffffffu, s1, o);
      if (lane >= o) { s0 += u0; s1 += u1; }
    }
    s1 += __shfl_sync(0xffffffffu, s0, 31);
    sL[warp * C + lane] = s0;
    sL[warp * C + lane + 32] = s1;
    sNE[warp * C + lane] = fast_exp2(-s0);
    sNE[warp * C + lane + 32] = fast_exp2(-s1);
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  bool ok = tc::mbar_wait(tbar, 0);
  ok = !__syncthreads_or(!ok);

  // lane RoPE of token t's k and q in place (rotated chunk pairs only; one set of angles)
  if (ok) {
    const float sc = dpairs > 0 ? a.rope.scale[lm] : 0.f;
    for (int it = tid; it < 2 * C * dch; it += P_NT) {
      const int rr = it / dch, cc = it - rr * dch;  // rr: token of the pair
      const int jj = rr & 63;
      const int qr = (rr < C ? 0 : 2 * C) + jj;      // Qa rows 0-63, Qb rows 128-191
      const int kr = qr + C;                         // Ka rows 64-127, Kb rows 192-255
      float x1[8], x2[8], y1[8], y2[8];
      const uint32_t o1 = tc::sw128(kr, cc, 256), o2 = tc::sw128(kr, cc + dch, 256);
      const uint32_t p1 = tc::sw128(qr, cc, 256), p2 = tc::sw128(qr, cc + dch, 256);
      load8_bf16(cKQ + o1, 0, x1);
      load8_bf16(cKQ + o2, 0, x2);
      load8_bf16(cKQ + p1, 0, y1);
      load8_bf16(cKQ + p2, 0, y2);
      const float pos = (float)(a.rope.pos0 + tbase + rr);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float sn, cs;
        sincos_reduced(pos * sc * sInv[8 * cc + e], &sn, &cs);
        const float a1 = x1[e] * cs - x2[e] * sn;
        x2[e] = a1 * sn + x2[e] * cs;
        x1[e] = a1;
        const float b1 = y1[e] * cs - y2[e] * sn;
        y2[e] = b1 * sn + y2[e] * cs;
        y1[e] = b1;
      }
      tc::st_chunk_bf16(cKQ, o1, x1);
      tc::st_chunk_bf16(cKQ, o2, x2);
      tc::st_chunk_bf16(cKQ, p1, y1);
      tc::st_chunk_bf16(cKQ, p2, y2);
    }
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  // on the tensor cores, two M = 64 Gram products in 128 TMEM columns: chunk a's
  // Ka [Qa;Ka]^T in lanes 0-15 of each quadrant, chunk b's Kb [Qb;Kb]^T in lanes 16-31
  // (lane offset 16); columns 0-63 hold k_j.q_i, 64-127 k_j.k_l
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t ID = tc::idesc_bf16(64, 128, false, false);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const uint32_t ko = sKQ + (s >> 2) * 32768 + (s & 3) * 32;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        const uint32_t kc = ko + c2 * 128 * 128;  // chunk c2: [Q;K] rows, K at +64 rows
        tc::mma_bf16(tmem + ((uint32_t)(16 * c2) << 16), tc::smem_desc(kc + 64 * 128, 16, 1024),
                     tc::smem_desc(kc, 16, 1024), ID, s > 0);
      }
    }
    tc::commit(mbar);
  }
  if (ok) ok = tc::mbar_wait(mbar, 0);
  ok = !__syncthreads_or(!ok);
  tc::fence_after();
  const uint32_t lrow = (uint32_t)(quad * 32) << 16;
  const float* L = sL + ci * C;
  const float* NE = sNE + ci * C;
  const bool fold = L[C - 1] >= FOLD_MIN_LC;
  const float Lj = L[j];
  // masks, all warps: this thread's half (32 columns) of row j of k k^T
  if (ok) {
    float d[32];
    tc::tmem_ld32(tmem + lrow + 64 + 32 * half, d);
    if ((j >> 5) == half) {  // |k_j|^2 is the diagonal (selected without a dynamic register index)
      const int id = j & 31;  // d[id] by halving selects (static register indices only)
      float t[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) t[e] = (id & 16) ? d[e + 16] : d[e];
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int e = 0; e < w; ++e) t[e] = (id & w) ? t[e + w] : t[e];
      sKN[ci * C + j] = t[0];
    }
  }
  __syncthreads();
  if (ok) {
    // A[j][l] = ce_j 2^{L_j - L_l} (k_j.k_l) for l < j
    float cej = 0.f, cwj = 0.f;
    if (tj < a.T) {
      const float be = raw_f32(rbe, a.gate_e.dtype), bw = raw_f32(rbw, a.gate_w.dtype);
      if (P.kmd2) {
        cej = be;
        cwj = bw;
      } else {
        const float al = stable_alpha(be * sKN[ci * C + j]);
        cej = al * be;
        cwj = al * bw;
      }
    }
    const float ej = fast_exp2(Lj);
    if (half == 0) {
      sCE[ci * C + j] = cej * ej;
      sCW[ci * C + j] = cwj;
    }
    const float rj = cej * ej;  // 2^{L_j - L_l} as 2^{L_j} 2^{-L_l} on folded chunks
    float* Arow = sA + (ci * C + j) * LDA + 32 * half;
    float d[32];
    tc::tmem_ld32(tmem + lrow + 64 + 32 * half, d);  // again (not held across the barrier)
    if (32 * half >= 16 * quad + 16) {  // l >= j for the whole half row (warp-uniform)
#pragma unroll
      for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(Arow + e) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (fold) {  // (lanes of one warp can be on different chunks: a per-lane branch, rarely divergent)
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 ne = *reinterpret_cast<const float4*>(NE + 32 * half + e);
        const float n4[4] = {ne.x, ne.y, ne.z, ne.w};
        float g[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) g[u] = (32 * half + e + u < j) ? rj * n4[u] * d[e + u] : 0.f;
        *reinterpret_cast<float4*>(Arow + e) = make_float4(g[0], g[1], g[2], g[3]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        float g[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int l = 32 * half + e + u;
          g[u] = (l < j) ? cej * fast_exp2(Lj - L[l]) * d[e + u] : 0.f;
        }
        *reinterpret_cast<float4*>(Arow + e) = make_float4(g[0], g[1], g[2], g[3]);
      }
    }
    // Mq^T row l = j, columns i of this half: Mq[i][l] = 2^{L_i - L_l} (q_i.k_l) for i >= l
    // (q_i.k_l undecayed on folded chunks); rows l, 64 i: the MN-major B operand of
    // y += W^T Mq^T, staged over the consumed tiles
    float dq[32];
    tc::tmem_ld32(tmem + lrow + 32 * half, dq);
    char* mqt = reinterpret_cast<char*>(sm + P_OFF_MQS + ci * 8192);
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      float v[8];
      if (32 * half + 32 <= 16 * quad) {  // i < j for the whole half row (warp-uniform)
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      } else if (fold) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = (32 * half + 8 * c8 + e >= j) ? dq[8 * c8 + e] : 0.f;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = 32 * half + 8 * c8 + e;
          v[e] = (i >= j) ? fast_exp2(L[i] - Lj) * dq[8 * c8 + e] : 0.f;
        }
      }
      tc::st_chunk_bf16(mqt, tc::sw128(j, 4 * half + c8, C), v);
    }
    tc::fence_async_smem();
  }
  __syncthreads();
  // T = (I + A)^{-1}: the eight 16 x 16 diagonal blocks by substitution (warps 0-3, two
  // blocks per warp) while warps 4-7 stack the level-1 A21 blocks; then the off-diagonal blocks
  // by two levels of block products on the tensor cores (bf16 operands, fp32 accumulate):
  //   level 1 (16-blocks, problems p = 2 ci + beta): R = A21 T11, T21 = -T22 R
  //   level 2 (32-blocks, problems p = ci):         R = A21 T11, T21 = -T22 R
  // Each level stacks its problems as M = 64 rows and N = 64 columns of one MMA; the
  // diagonal N blocks are the products (the rest is unused).  Operand tiles: level 1 in
  // the free tail of the tile region, level 2 over the Mq^T staging once it is stored.
  char* cL1 = reinterpret_cast<char*>(sm + P_OFF_L1);    // K-major 64 rows: K chunk 0 A21 stack, chunk 1 T11 columns
  char* cL1A2 = reinterpret_cast<char*>(sm + P_OFF_L1A2);  // MN-major [16 k][64 m]: T22 stack
  char* cL1B2 = reinterpret_cast<char*>(sm + P_OFF_L1B2);  // MN-major [16 k][64 n]: R stack
  char* cL2 = reinterpret_cast<char*>(sm + P_OFF_L2);    // K-major 64 rows: chunks 0-1 A21, 2-3 T22
  char* cL2B = reinterpret_cast<char*>(sm + P_OFF_L2B);  // MN-major [32 k][64 n]: T11 rows
  char* cL2B2 = reinterpret_cast<char*>(sm + P_OFF_L2B2);  // MN-major [32 k][64 n]: R rows
  if (ok) {
    if (warp < 4) {
      const int cs_ = warp >> 1, blk = 2 * (warp & 1) + (lane >> 4), c = lane & 15;
      float* A = sA + cs_ * C * LDA;
      float x[16];
      subst_block16(A, 16 * blk, c, x);
      const int pp = 2 * cs_ + (blk >> 1);  // level-1 problem
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (blk & 1)  // T22 of the problem, column c as MN-major row k = c, M offset 16 pp
          tc::st_chunk_bf16(cL1A2, tc::sw128(c, 2 * pp + hh, 16), x + 8 * hh);
        else  // T11 column c as K-major row n = 16 pp + c, K chunk 1
          tc::st_chunk_bf16(cL1, tc::sw128(16 * pp + c, 2 + hh, 64), x + 8 * hh);
      }
    } else {
      // level-1 A21 stack: row m = 16 pp + r holds A[32 beta + 16 + r][32 beta .. + 15]
      {
        const int t = tid - 128, m = t >> 1, hh = t & 1;  // 64 rows x 2 halves
        const int pp = m >> 4, r = m & 15, cs_ = pp >> 1, beta = pp & 1;
        const float* src = sA + (cs_ * C + 32 * beta + 16 + r) * LDA + 32 * beta + 8 * hh;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = src[e];
        tc::st_chunk_bf16(cL1, tc::sw128(m, hh, 64), v);
      }
      tc::fence_async_smem();
    }
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  if (ok && tid == P_STORE_TID) {  // staged Mq^T tiles -> global with bulk copies
    for (int c2 = 0; c2 < 2; ++c2) {
      const int64_t chn = pair * 2 + c2;
      if (chn < P.nchunks)
        bulk_store(P.tt + (n * P.nchunks + chn) * TT_ELEMS + 2 * C * C, tc::smem_u32(sm + P_OFF_MQS + c2 * 8192), 8192);
    }
    bulk_commit();
  }
  uint32_t mph = 1;  // the Gram MMAs completed phase 0
  constexpr uint32_t ID_KK = tc::idesc_bf16(64, 64, false, false);
  constexpr uint32_t ID_MNMN = tc::idesc_bf16(64, 64, true, true);
  constexpr uint32_t ID_KMN = tc::idesc_bf16(64, 64, false, true);
  const uint32_t sL1 = tc::smem_u32(cL1), sL1A2 = tc::smem_u32(cL1A2), sL1B2 = tc::smem_u32(cL1B2);
  const uint32_t sL2 = tc::smem_u32(cL2), sL2B = tc::smem_u32(cL2B), sL2B2 = tc::smem_u32(cL2B2);
  // an M = 64 accumulator row m sits in TMEM lane (m / 16) * 32 + m % 16: warps 0-3, lanes < 16
  const bool drow = warp < 4 && lane < 16;
  const int dm = 16 * quad + lane;  // accumulator row held by this thread (when drow)
  const uint32_t dl = (uint32_t)(32 * quad) << 16;
  auto mma_round = [&](auto issue) -> bool {  // one MMA group, all threads wait for it
    if (ok && tid == 0) {
      tc::fence_after();
      issue();
      tc::commit(mbar);
    }
    bool w = ok ? tc::mbar_wait(mbar, mph & 1) : false;
    ++mph;
    w = !__syncthreads_or(!w);
    tc::fence_after();
    return w;
  };
  // level 1: R = A21 T11
  ok = mma_round([&] { tc::mma_bf16(tmem, tc::smem_desc(sL1, 16, 1024), tc::smem_desc(sL1 + 32, 16, 1024), ID_KK, 0); });
  if (ok && warp < 4) {  // tcgen05.ld is warp-collective: all 32 lanes load, rows < 16 are used
    float d16[16];
    tc::tmem_ld16(tmem + dl + 16 * quad, d16);  // problem pp = quad: R[r = lane][0..15]
    if (drow) tc::st_chunk_bf16(cL1B2, tc::sw128(lane, 2 * quad, 16), d16);
    if (drow) tc::st_chunk_bf16(cL1B2, tc::sw128(lane, 2 * quad + 1, 16), d16 + 8);
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  // level 1: T21 = -T22 R
  ok = mma_round([&] {
    tc::mma_bf16(tmem + 64, tc::smem_desc(sL1A2, 8192, 1024), tc::smem_desc(sL1B2, 8192, 1024), ID_MNMN, 0);
  });
  if (ok && warp < 4) {
    float d16[16];
    tc::tmem_ld16(tmem + 64 + dl + 16 * quad, d16);
    const int cs_ = quad >> 1, beta = quad & 1;
    float* dst = sA + (cs_ * C + 32 * beta + 16 + (lane & 15)) * LDA + 32 * beta;
    if (drow)
#pragma unroll
      for (int e = 0; e < 16; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(-d16[e], -d16[e + 1], -d16[e + 2], -d16[e + 3]);
  }
  tc::fence_before();
  if (tid == P_STORE_TID) bulk_wait_read();  // the Mq^T staging is free for the level-2 tiles
  __syncthreads();
  // level-2 operands: rows m = 32 ci + r of A21 (chunks 0-1) and T22 (chunks 2-3); T11 rows
  for (int it = tid; it < 2 * 32 * 8; it += P_NT) {
    const int m = it >> 3, c8 = it & 7, cs_ = m >> 5, r = m & 31;
    const float* src = sA + (cs_ * C + 32 + r) * LDA + 8 * c8;  // cols 0-31: A21, 32-63: T22
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = src[e];
    tc::st_chunk_bf16(cL2, tc::sw128(m, c8, 64), v);
  }
  for (int it = tid; it < 2 * 32 * 4; it += P_NT) {
    const int cs_ = it >> 7, k = (it >> 2) & 31, c8 = it & 3;
    const float* src = sA + (cs_ * C + k) * LDA + 8 * c8;  // T11 row k, columns 0-31
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = src[e];
    tc::st_chunk_bf16(cL2B, tc::sw128(k, 4 * cs_ + c8, 32), v);
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  // level 2: R = A21 T11 (K = 32)
  ok = mma_round([&] {
    tc::mma_bf16(tmem, tc::smem_desc(sL2, 16, 1024), tc::smem_desc(sL2B, 8192, 1024), ID_KMN, 0);
    tc::mma_bf16(tmem, tc::smem_desc(sL2 + 32, 16, 1024), tc::smem_desc(sL2B + 2048, 8192, 1024), ID_KMN, 1);
  });
  if (ok && warp < 4) {
    float d32[32];
    const int cs_ = quad >> 1, r = dm & 31;
    tc::tmem_ld32(tmem + dl + 32 * cs_, d32);  // R[r][0..31] of chunk cs_
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4)
      if (drow) tc::st_chunk_bf16(cL2B2, tc::sw128(r, 4 * cs_ + q4, 32), d32 + 8 * q4);
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  // level 2: T21 = -T22 R (T22 in K chunks 2-3 of the level-2 tile)
  ok = mma_round([&] {
    tc::mma_bf16(tmem + 64, tc::smem_desc(sL2 + 64, 16, 1024), tc::smem_desc(sL2B2, 8192, 1024), ID_KMN, 0);
    tc::mma_bf16(tmem + 64, tc::smem_desc(sL2 + 96, 16, 1024), tc::smem_desc(sL2B2 + 2048, 8192, 1024), ID_KMN, 1);
  });
  if (ok && warp < 4) {
    float d32[32];
    const int cs_ = quad >> 1, r = dm & 31;
    tc::tmem_ld32(tmem + 64 + dl + 32 * cs_, d32);
    float* dst = sA + (cs_ * C + 32 + r) * LDA;
#pragma unroll
    for (int e = 0; e < 32; e += 4)
      if (drow) *reinterpret_cast<float4*>(dst + e) = make_float4(-d32[e], -d32[e + 1], -d32[e + 2], -d32[e + 3]);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 6) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 128);
  }
  if (!ok) {
    if (tid == 0 && P.err) atomicExch(P.err, (int)GDNX_ETIMEOUT);
    if (tid == P_STORE_TID) bulk_wait_all();
    return;
  }
  // T_e = T diag(ce 2^L), T_w = T diag(cw) as bf16 tiles in the swizzled UMMA layout,
  // straight to global (T's upper block T12 is zero); then L
  for (int it = tid; it < 2 * C * 8; it += P_NT) {
    const int cj = it >> 9, jj = (it >> 3) & 63, c8 = it & 7;
    const int64_t chn = pair * 2 + cj;
    if (chn >= P.nchunks) continue;
    float te[8], tw[8];
    if (c8 >= 4 && jj < 32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) te[e] = tw[e] = 0.f;
    } else {
      const float* src = sA + (cj * C + jj) * LDA + 8 * c8;
      const float4 u0 = *reinterpret_cast<const float4*>(src), u1 = *reinterpret_cast<const float4*>(src + 4);
      const float4* ce4 = reinterpret_cast<const float4*>(sCE + cj * C + 8 * c8);
      const float4* cw4 = reinterpret_cast<const float4*>(sCW + cj * C + 8 * c8);
      const float4 e0 = ce4[0], e1 = ce4[1], w0 = cw4[0], w1 = cw4[1];
      const float t8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      const float ce8[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
      const float cw8[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        te[e] = t8[e] * ce8[e];
        tw[e] = t8[e] * cw8[e];
      }
    }
    char* dst = reinterpret_cast<char*>(P.tt + (n * P.nchunks + chn) * TT_ELEMS);
    const uint32_t off = tc::sw128(jj, c8, C);
    tc::st_chunk_bf16(dst, off, te);
    tc::st_chunk_bf16(dst + 8192, off, tw);
  }
  if (tid < 2 * C) {
    const int64_t chn = pair * 2 + (tid >> 6);
    if (chn < P.nchunks) P.lsum[(n * P.nchunks + chn) * C + (tid & 63)] = sL[tid];
  }
  if (tid == P_STORE_TID) bulk_wait_read();  // the Mq^T stores have read shared memory
}

// Timing probe (off by default): with GDNX_PHASE_PROBE defined, one thread per warp group adds
// the cycles it spends in each wait of pass 2 to g_wy_probe, read by gdnx_debug_wy_probe:
// [0] state group waiting for `ready`, [1] state group waiting for G2, [2] for G3,
// [3] prologue waiting for its stage, [4] for G1, [5] for the previous chunk's G3 (y out),
// [6] pass-2 CTA lifetime.
#ifdef GDNX_PHASE_PROBE
__device__ unsigned long long g_wy_probe[16];
#define WY_TIMED(slot, cond, expr)                                  \
  [&]() {                                                           \
    if (!(cond)) return (expr);                                     \
    const long long t0_ = clock64();                                \
    auto r_ = (expr);                                               \
    probe_acc[slot] += (unsigned long long)(clock64() - t0_);       \
    return r_;                                                      \
  }()
#define WY_MARK(slot)                                                                 \
  do {                                                                                \
    if (tid == 0) {                                                                   \
      const long long n_ = clock64();                                                 \
      probe_acc[slot] += (unsigned long long)(n_ - pmark);                            \
      pmark = n_;                                                                     \
    }                                                                                 \
  } while (0)
#define WY_ISSUE_BEGIN() const long long iss0_ = clock64()
#define WY_ISSUE_END(slot) probe_acc[slot] += (unsigned long long)(clock64() - iss0_)
#else
#define WY_ISSUE_BEGIN() \
  do {                   \
  } while (0)
#define WY_ISSUE_END(slot) \
  do {                     \
  } while (0)
#define WY_TIMED(slot, cond, expr) (expr)
#define WY_MARK(slot) \
  do {                \
  } while (0)
#endif

// ------------------------------- pass 2 ------------------------------------
constexpr int S_NT = 512;  // warps 0-7: state group, warps 8-15: prologue / output group
constexpr int G_NT = 256;  // threads per group
// Shared memory.  Each stage's q/k tile has 192 rows per 64-wide K block:
//   stage 0: rows 0-63 k, 64-127 -Wk (G2 B rows [Wk; Q]), 128-191 q
//   stage 1: rows 0-63 k, 64-127 q,  128-191 -Wk      (G2 B rows [Q; Wk])
// and Mq^T sits one block-stride before (stage 0) or two after (stage 1) the
// k rows, so that G3's MN-major B operand [Mq^T | K'] / [K' | Mq^T] is one
// descriptor with LBO = the block stride.
constexpr int KB = 24576;                        // K-block stride of a q/k tile
constexpr int S_OFF_MQ0 = 0;                     // Mq^T stage 0 [64 j][64 i]
// (bytes 8192 .. KB - 1 are free: W^T is an A operand in TMEM)
constexpr int S_OFF_KQ0 = S_OFF_MQ0 + KB;        // stage 0 tile (2 blocks)
constexpr int S_OFF_KQ1 = S_OFF_KQ0 + 2 * KB;    // stage 1 tile
constexpr int S_OFF_MQ1 = S_OFF_KQ1 + 2 * KB;    // Mq^T stage 1
constexpr int S_OFF_V = S_OFF_MQ1 + 8192;        // 2 stages x [2 vb][64 tokens][128 B]
constexpr int S_OFF_TT = S_OFF_V + 2 * 16384;    // 2 stages x (T_e 8 KB | T_w 8 KB)
constexpr int S_OFF_SB = S_OFF_TT + 2 * 16384;   // (unused: the bf16 state is in TMEM)
constexpr int S_OFF_L = S_OFF_SB + 32768;        // 2 stages x L[64]
constexpr int S_OFF_PSC = S_OFF_L + 512;         // 2 x 2^L, 2 x K' factor: 4 x 64 fp32
constexpr int S_OFF_SF = S_OFF_PSC + 1024;       // 2 x {2^ls, rescale factor, rescale flag, -}
constexpr int S_OFF_INV = S_OFF_SF + 32;         // inv_freq[64]
constexpr int S_OFF_BAR = S_OFF_INV + 256;       // 8 mbarriers, TMEM base, abort flag, final ls
constexpr int S_SMEM = S_OFF_BAR + 128 + 1024;
static_assert(S_OFF_MQ1 == S_OFF_KQ1 + 2 * KB, "stage-1 Mq^T position");
static_assert(S_OFF_KQ0 - KB == S_OFF_MQ0, "stage-0 Mq^T position");
static_assert(S_SMEM <= 232448, "shared memory");
constexpr uint32_t STAGE_TX = 6 * 8192 + 3 * 8192 + 256;

// TMEM columns: W^T0 | y0 | state (128) | y1 | W^T1 | Wk (64) | S bf16 (64), so that G2
// writes [W^T0 | y0] / [y1 | W^T1] and G3 writes [y0 | S] / [S | y1] with one MMA each.  Wk
// [64 j][128 k] is two M = 64 accumulators: k block kb in lanes 32 q + 16 kb + (j % 16)
// of quadrant q = j / 16 (the M = 64 layout, the second block at lane offset 16).
// The A operands of G2 (S0) and G3 (W^T) are read from TMEM: S0 packed as bf16 pairs in
// the last 64 columns, W^T packed in place over its fp32 accumulator (tokens 32 h .. 32 h
// + 31 in columns 32 h .. 32 h + 15 of the buffer), so neither goes through shared memory.
constexpr uint32_t T_W0 = 0, T_Y0 = 64, T_S = 128, T_Y1 = 256, T_W1 = 320, T_WK = 384, T_SB = 448;

// 16 TMEM lanes x 32 consecutive 32-bit columns in the 16x256b fragment layout:
// for each 8-column group p, registers 4p..4p+3 hold (lane g, column 2(t%4)),
// (lane g, column 2(t%4)+1), (lane g+8, column 2(t%4)), (lane g+8, column 2(t%4)+1),
// with g = t/4 (t = thread of the warp): the layout of an m16n8 accumulator, which
// stmatrix stores 8x8 at a time.  The completion wait is in the same asm statement.
GDNX_DEV void tmem_ld_16x256b_x4(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Four 8x8 bf16 matrices (fragment: thread t holds row t/4, columns 2(t%4), +1 of
// each) stored transposed: thread t gives the address of stored row t%8 of matrix t/8.
GDNX_DEV void stmatrix_x4_trans(uint32_t saddr, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(a0),
               "r"(a1), "r"(a2), "r"(a3)
               : "memory");
}

GDNX_DEV bool try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait that also gives up when the other group has raised the abort flag.
GDNX_DEV bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = tc::smem_u32(bar);
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    if (try_wait(a, parity)) return true;
    if (*abort_flag) return false;
  }
  *abort_flag = 1;
  return false;
}
GDNX_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}
GDNX_DEV void group_sync(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(G_NT) : "memory"); }
// Group barrier that returns the OR of `v` over the group (the same value in every thread).
GDNX_DEV bool group_any(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(G_NT)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(S_NT, 1)
    wy_scan_kernel(const WyParams P, const __grid_constant__ WyScanMaps maps) {
#ifdef GDNX_PHASE_PROBE
  const long long t_life = clock64();
  unsigned long long probe_acc[16] = {};
#endif
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = tc::align_smem(smraw, 1024);
  float* sEL = reinterpret_cast<float*>(sm + S_OFF_PSC);  // [2][64] y factors / Qd factors
  float* sFK = sEL + 128;                                  // [2][64] W factors / K' factors
  float4* sSF = reinterpret_cast<float4*>(sm + S_OFF_SF);
  float* sInv = reinterpret_cast<float*>(sm + S_OFF_INV);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S_OFF_BAR);
  uint64_t* full = bars;       // [2] stage loaded (TMA + bulk, tx-counted)
  uint64_t* g1 = bars + 2;     // G1 complete (prologue group's MMAs)
  uint64_t* g2 = bars + 3;     // G2 complete
  uint64_t* g3 = bars + 4;     // [2] G3 complete (per stage / y buffer)
  uint64_t* ready = bars + 6;  // [2] prologue of the chunk done (operands in place)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + S_OFF_BAR + 68);
  float* s_lsfin = reinterpret_cast<float*>(sm + S_OFF_BAR + 72);

  const gdnx_scan_args& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3;
  const int row = quad * 32 + lane;
  const uint32_t lbase = (uint32_t)(quad * 32) << 16;
  const int64_t n = P.n0 + blockIdx.x;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int lm = (int)m;
  const int dpairs = (a.rope.enable && lm < 4) ? a.rope.pairs[lm] : 0;
  const int dch = dpairs / 8;
  const float rsc = dpairs > 0 ? a.rope.scale[lm] : 0.f;
  const int64_t nchunks = P.nchunks;
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t sV = sbase + S_OFF_V, sTT = sbase + S_OFF_TT, sLst = sbase + S_OFF_L;
  const __nv_bfloat16* ttg = P.tt + n * nchunks * TT_ELEMS;
  const float* lsg = P.lsum + n * nchunks * C;
  // per-stage geometry (rows within a 192-row K block)
  auto kq_off = [](int s) { return s ? S_OFF_KQ1 : S_OFF_KQ0; };
  auto q_row = [](int s) { return s ? 64 : 128; };
  auto wk_row = [](int s) { return s ? 128 : 64; };
  auto mq_off = [](int s) { return s ? S_OFF_MQ1 : S_OFF_MQ0; };

  if (warp == 0) tc::tmem_alloc(s_tmem, 512);
  if (tid == 0) {
    for (int i = 0; i < 8; ++i) tc::mbar_init(bars + i, 1);
    *s_abort = 0;
    *s_lsfin = 0.f;
  }
  if (dpairs > 0 && tid < 64) sInv[tid] = 1.0f / powf(10000.0f, (float)tid / a.rope.den[lm]);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;

  // TMA coordinates: {x (dim), lane, head, token, batch}
  const int cq_m = maps.use_m[0] ? lm : 0, ck_m = maps.use_m[1] ? lm : 0, cv_m = maps.use_m[2] ? lm : 0;
  auto issue_stage = [&](int64_t chn) {  // one thread
    const int s = (int)(chn & 1);
    const uint32_t bar = tc::smem_u32(full + s);
    const int t0 = (int)(chn * C);
    tc::fence_async_smem();
    expect_tx(bar, STAGE_TX);
    const uint32_t kq = sbase + kq_off(s);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      tma_load_5d(kq + kb * KB, &maps.k, 64 * kb, ck_m, (int)h, t0, (int)b, bar);
      tma_load_5d(kq + kb * KB + q_row(s) * 128, &maps.q, 64 * kb, cq_m, (int)h, t0, (int)b, bar);
      tma_load_5d(sV + s * 16384 + kb * 8192, &maps.v, 64 * kb, cv_m, (int)h, t0, (int)b, bar);
    }
    bulk_load(sTT + s * 16384, ttg + chn * TT_ELEMS, 16384, bar);
    bulk_load(sbase + mq_off(s), ttg + chn * TT_ELEMS + 2 * C * C, 8192, bar);
    bulk_load(sLst + s * 256, lsg + chn * C, 256, bar);
  };
  if (tid == 0) {
    const CUtensorMap* mps[4] = {&maps.q, &maps.k, &maps.v, &maps.y};
    for (int i = 0; i < (maps.y_tma ? 4 : 3); ++i)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(mps[i])) : "memory");
    issue_stage(0);
    if (nchunks > 1) issue_stage(1);
  }

  // initial state into TMEM (all 16 warps, 32 columns each)
  {
    float vals[32];
    const int col = 32 * (warp >> 2);
    if (a.state_in) {
      const float* src = a.state_in + (n * VD + row) * KD + col;
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 f = *reinterpret_cast<const float4*>(src + e);
        vals[e] = f.x; vals[e + 1] = f.y; vals[e + 2] = f.z; vals[e + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) vals[e] = 0.f;
    }
    tc::tmem_st32(tmem + T_S + lbase + col, vals);
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  constexpr uint32_t ID_MN_K = tc::idesc_bf16(128, 64, true, false);
  constexpr uint32_t ID_WK = tc::idesc_bf16(64, 64, false, true);
  constexpr uint32_t ID_G2 = tc::idesc_bf16(128, 128, false, false);
  constexpr uint32_t ID_G3 = tc::idesc_bf16(128, 192, false, true);

  if (warp < 8) {
    // ======================= state group: S0 -> G2 -> W -> G3 =======================
    const int half = warp >> 2;
#ifdef GDNX_PHASE_PROBE
    long long pmark = clock64();
#endif
    for (int64_t ch = 0; ch < nchunks; ++ch) {
      const int s = (int)(ch & 1);
      bool ok = WY_TIMED(0, tid == 0, wait_or_abort(ready + s, (uint32_t)((ch >> 1) & 1), s_abort));
      if (group_any(2, !ok)) break;
      WY_MARK(7);  // tail of the previous chunk + the ready wait
      // S_tmem -> bf16 operand (times 2^ls when the chunk normalises the state), and the
      // TMEM write-back of a normalisation (exact path: also the chunk decay 2^{L_C})
      {
        const float4 sf = sSF[s];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int col = 64 * half + 32 * hh;
          float vals[32];
          uint32_t pk[16];
          tc::tmem_ld32(tmem + T_S + lbase + col, vals);
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = tc::pack_bf16(vals[2 * e] * sf.x, vals[2 * e + 1] * sf.x);
          tc::tmem_st16u(tmem + T_SB + lbase + col / 2, pk);
          if (sf.z != 0.f) {
#pragma unroll
            for (int e = 0; e < 32; ++e) vals[e] *= sf.y;
            tc::tmem_st32(tmem + T_S + lbase + col, vals);
          }
        }
      }
      tc::fence_before();
      if (group_any(2, *s_abort != 0)) break;
      WY_MARK(8);  // conversion
      // G2: [W^T | y] += S0 [-Wk; Qd]^T  (W^T holds V^T T_w^T from G1, y was zeroed)
      const uint32_t kq = sbase + kq_off(s);
      if (tid == 0) {
        tc::fence_after();
        const uint32_t d = tmem + (s ? T_Y1 : T_W0);
        WY_ISSUE_BEGIN();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ko = (k >> 2) * KB + (k & 3) * 32;
          tc::mma_bf16_ts(d, tmem + T_SB + 8 * k, tc::smem_desc(kq + ko + 64 * 128, 16, 1024), ID_G2, 1);
        }
        tc::commit(g2);
        WY_ISSUE_END(13);
      }
      ok = WY_TIMED(1, tid == 0, wait_or_abort(g2, (uint32_t)(ch & 1), s_abort));
      tc::fence_after();
      if (group_any(2, !ok)) break;
      WY_MARK(9);  // G2 issue + wait
      // W^T -> bf16 A operand
      {
        float w[32];
        tc::tmem_ld32(tmem + (s ? T_W1 : T_W0) + lbase + 32 * half, w);
        if (sSF[s].w != 0.f) {  // folded chunk: W diag(f)
          const float4* f4 = reinterpret_cast<const float4*>(sFK + 64 * s + 32 * half);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 f = f4[e];
            w[4 * e] *= f.x;
            w[4 * e + 1] *= f.y;
            w[4 * e + 2] *= f.z;
            w[4 * e + 3] *= f.w;
          }
        }
        // packed in place: tokens 32 half + 2e, +1 in column 32 half + e of the W^T buffer
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = tc::pack_bf16(w[2 * e], w[2 * e + 1]);
        tc::tmem_st16u(tmem + (s ? T_W1 : T_W0) + lbase + 32 * half, pk);
      }
      tc::fence_before();
      if (group_any(2, *s_abort != 0)) break;
      WY_MARK(10);  // W read-out
      // G3: [y | S] or [S | y] += W^T [Mq^T | K] / [K | Mq^T]   (B MN-major; W^T carries the
      // decay factors on folded chunks, K carries them on the exact path)
      if (tid == 0) {
        tc::fence_after();
        const uint32_t d = tmem + (s ? T_S : T_Y0);
        WY_ISSUE_BEGIN();
        const uint32_t bb = s ? kq : sbase + S_OFF_MQ0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16_ts(d, tmem + (s ? T_W1 : T_W0) + 32 * (k >> 1) + 8 * (k & 1),
                          tc::smem_desc(bb + k * 2048, KB, 1024), ID_G3, 1);
        tc::commit(g3 + s);
        WY_ISSUE_END(14);
      }
      ok = WY_TIMED(2, tid == 0, wait_or_abort(g3 + s, (uint32_t)((ch >> 1) & 1), s_abort));
      tc::fence_after();
      if (group_any(2, !ok)) break;
      WY_MARK(11);  // G3 issue + wait
      // stage s is consumed: fetch chunk ch + 2 into it (a thread outside warp 0, which
      // issues the next MMAs; the others go on to the next chunk's wait)
      if (tid == 32 && ch + 2 < nchunks) WY_TIMED(12, true, (issue_stage(ch + 2), 0));
    }
  } else {
    // ========== prologue / output group: RoPE, G1, -Wk, Qd, y zero, y out ==========
    const int ptid = tid - G_NT, half = (warp - 8) >> 2;
    const int64_t ybase = b * a.y_sb + h * a.y_sh + m * a.y_sm;
    float ls = 0.f;  // state = 2^ls * S_tmem at the start of the chunk being prepared
    const int cy_m = maps.use_m[3] ? lm : 0;
    // y of chunk `c` (its G3 complete) -> global.  With TMA: staged as two
    // swizzled [64 tokens][64 v] boxes in the -Wk rows of the chunk's stage (G2 has
    // consumed them; the next writer waits for the stores' reads).
    auto y_out = [&](int64_t c) -> bool {
      const int sp = (int)(c & 1);
      const bool ok = WY_TIMED(5, ptid == 0, wait_or_abort(g3 + sp, (uint32_t)((c >> 1) & 1), s_abort));
      tc::fence_after();
      if (group_any(1, !ok)) return false;
      const bool folded = sSF[sp].w != 0.f;  // y_i = 2^{L_i + ls} y_tmem on folded chunks
      const uint32_t ty = tmem + (sp ? T_Y1 : T_Y0);
      if (maps.y_tma) {
        // rows v (TMEM lanes) x tokens i -> [token][v] swizzled tiles: 16x256b loads give
        // 8x8 fragments, stored transposed by stmatrix
        float ya[16], yb[16];
        tmem_ld_16x256b_x4(ty + lbase + 32 * half, ya);                       // lanes 32q + 0..15
        tmem_ld_16x256b_x4(ty + lbase + (16u << 16) + 32 * half, yb);         // lanes 32q + 16..31
        const int t4 = lane & 3, mi = lane >> 3, jr = lane & 7;
        const uint32_t stg = sbase + kq_off(sp) + wk_row(sp) * 128;
        const int v0 = 32 * quad + 8 * mi;  // this thread's address: matrix mi, stored row jr
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          float f0 = 1.f, f1 = 1.f;
          if (folded) {
            f0 = sEL[64 * sp + 32 * half + 8 * p + 2 * t4];
            f1 = sEL[64 * sp + 32 * half + 8 * p + 2 * t4 + 1];
          }
          const uint32_t m0 = tc::pack_bf16(ya[4 * p] * f0, ya[4 * p + 1] * f1);
          const uint32_t m1 = tc::pack_bf16(ya[4 * p + 2] * f0, ya[4 * p + 3] * f1);
          const uint32_t m2 = tc::pack_bf16(yb[4 * p] * f0, yb[4 * p + 1] * f1);
          const uint32_t m3 = tc::pack_bf16(yb[4 * p + 2] * f0, yb[4 * p + 3] * f1);
          const int i = 32 * half + 8 * p + jr;
          const uint32_t addr = stg + (uint32_t)((v0 >> 6) * KB + i * 128 + ((((v0 & 63) >> 3) ^ (i & 7)) << 4));
          stmatrix_x4_trans(addr, m0, m1, m2, m3);
        }
        tc::fence_async_smem();
        group_sync(1);
        if (ptid == 0) {
          const uint32_t src = sbase + kq_off(sp) + wk_row(sp) * 128;
          tma_store_5d(&maps.y, 0, cy_m, (int)h, (int)(c * C), (int)b, src);
          tma_store_5d(&maps.y, 64, cy_m, (int)h, (int)(c * C), (int)b, src + KB);
          bulk_commit();
        }
      } else {
        float yv[32];
        tc::tmem_ld32(ty + lbase + 32 * half, yv);
        const int nt = (int)((a.T - c * C) < C ? (a.T - c * C) : C);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int i = 32 * half + e;
          const float f = folded ? sEL[64 * sp + i] : 1.f;
          if (i < nt) st_from_f32(a.y, a.y_dtype, ybase + row + (c * C + i) * a.y_st, yv[e] * f);
        }
      }
      return true;
    };
    bool alive = true;
    for (int64_t ch = 0; ch < nchunks; ++ch) {
      const int s = (int)(ch & 1);
      const int64_t t0 = ch * C;
      char* kq = reinterpret_cast<char*>(sm + kq_off(s));
      const int qr = q_row(s), wr = wk_row(s);
      bool ok = WY_TIMED(3, ptid == 0, wait_or_abort(full + s, (uint32_t)((ch >> 1) & 1), s_abort));
      if (group_any(1, !ok)) { alive = false; break; }
      const float* Lst = reinterpret_cast<const float*>(sm + S_OFF_L + s * 256);
      const float Lc = Lst[C - 1];
      const bool fold = Lc >= FOLD_MIN_LC;
      // normalise the state (S_tmem *= 2^ls, ls = 0) when ls < -40, and always on the exact path
      const bool norm = !fold || ls < -40.f;
      const float lsc = norm ? 0.f : ls;  // ls during this chunk
      const float wk_mult = fold ? exp2f(lsc) : 1.f;
      if (ptid < 64) {
        const float Lj = Lst[ptid];
        sEL[64 * s + ptid] = fold ? exp2f(Lj + lsc) : exp2f(Lj);    // y factor / Qd factor
        sFK[64 * s + ptid] = fold ? exp2f(-Lj - lsc) : exp2f(Lc - Lj);  // W factor / K' factor
      }
      // S read-out: bf16 operand factor, TMEM write-back factor, write-back flag, folded flag
      if (ptid == 64)
        sSF[s] = make_float4(norm ? exp2f(ls) : 1.f, fold ? exp2f(ls) : exp2f(ls + Lc), norm ? 1.f : 0.f,
                             fold ? 1.f : 0.f);
      ls = fold ? lsc + Lc : 0.f;
      // G1, first part (needs no rotated k): W^T = V^T T_w^T; and this stage's y buffer to
      // zero (its chunk two back is written out) while the tensor core runs it
      const uint32_t skq = sbase + kq_off(s), stt = sTT + s * 16384, sv = sV + s * 16384;
      if (ptid == 0) {
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16(tmem + (s ? T_W1 : T_W0), tc::smem_desc(sv + k * 2048, 8192, 1024),
                       tc::smem_desc(stt + 8192 + k * 32, 16, 1024), ID_MN_K, k > 0);
      }
      {
        float z[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) z[e] = 0.f;
        tc::tmem_st32(tmem + (s ? T_Y1 : T_Y0) + lbase + 32 * half, z);
      }
      // lane RoPE of token j's k (row j) and q (row qr + j) in place, one set of angles
      for (int it = ptid; it < C * dch; it += G_NT) {
        const int j = it / dch, cc = it - j * dch;
        float k1[8], k2[8], q1[8], q2[8];
        const uint32_t o1 = tc::sw128(j, cc, 192), o2 = tc::sw128(j, cc + dch, 192);
        const uint32_t p1 = tc::sw128(qr + j, cc, 192), p2 = tc::sw128(qr + j, cc + dch, 192);
        load8_bf16(kq + o1, 0, k1);
        load8_bf16(kq + o2, 0, k2);
        load8_bf16(kq + p1, 0, q1);
        load8_bf16(kq + p2, 0, q2);
        const float pos = (float)(a.rope.pos0 + t0 + j);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float sn, cs;
          sincos_reduced(pos * rsc * sInv[8 * cc + e], &sn, &cs);
          const float a1 = k1[e] * cs - k2[e] * sn;
          k2[e] = a1 * sn + k2[e] * cs;
          k1[e] = a1;
          const float b1 = q1[e] * cs - q2[e] * sn;
          q2[e] = b1 * sn + q2[e] * cs;
          q1[e] = b1;
        }
        tc::st_chunk_bf16(kq, o1, k1);
        tc::st_chunk_bf16(kq, o2, k2);
        tc::st_chunk_bf16(kq, p1, q1);
        tc::st_chunk_bf16(kq, p2, q2);
      }
      tc::fence_async_smem();
      tc::fence_before();
      group_sync(1);
      // G1, second part: Wk = T_e K (per 64-feature block of k); one commit covers both parts
      if (ptid == 0) {
        tc::fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_bf16(tmem + T_WK + ((uint32_t)(16 * kb) << 16), tc::smem_desc(stt + k * 32, 16, 1024),
                         tc::smem_desc(skq + kb * KB + k * 2048, KB, 1024), ID_WK, k > 0);
        tc::commit(g1);
      }
      ok = WY_TIMED(4, ptid == 0, wait_or_abort(g1, (uint32_t)(ch & 1), s_abort));
      tc::fence_after();
      if (ptid == 0) bulk_wait_read();  // y stores of chunk ch - 2 have read the -Wk rows
      if (group_any(1, !ok)) { alive = false; break; }
      if (!fold) {  // exact path: Qd = 2^{L_i} q_i and K' = 2^{L_C - L_j} k_j in place (G1 has read K)
        for (int it = ptid; it < 2 * C * 16; it += G_NT) {
          const int r = it >> 4, cc = it & 15;
          const bool isq = r >= C;
          const int rr = r & 63;
          const uint32_t off = tc::sw128(isq ? qr + rr : rr, cc, 192);
          float x[8];
          load8_bf16(kq + off, 0, x);
          const float f = isq ? sEL[64 * s + rr] : sFK[64 * s + rr];
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] *= f;
          tc::st_chunk_bf16(kq, off, x);
        }
      }
      // -Wk as rows of the G2 B operand (K-major [j][k]), all 8 warps: lane l of quadrant q
      // holds row j = 16 q + l % 16 of k block l / 16; half h takes 32 of its 64 columns
      {
        float d[32];
        const int j = 16 * quad + (lane & 15);
        char* base = kq + (lane >> 4) * KB;
        tc::tmem_ld32(tmem + T_WK + lbase + 32 * half, d);
#pragma unroll
        for (int e = 0; e < 32; ++e) d[e] = -d[e] * wk_mult;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) tc::st_chunk_bf16(base, tc::sw128(wr + j, 4 * half + q4, 192), d + 8 * q4);
      }
      tc::fence_async_smem();
      tc::fence_before();
      group_sync(1);
      if (ptid == 0) mbar_arrive(ready + s);
      // outputs of the previous chunk (its G3 overlaps this chunk's prologue)
      if (ch > 0 && !y_out(ch - 1)) { alive = false; break; }
    }
    if (alive && nchunks > 0) y_out(nchunks - 1);
    if (ptid == 0) {
      *s_lsfin = ls;
      bulk_wait_all();
    }
  }

  __syncthreads();
  tc::fence_after();
  const bool aborted = *s_abort != 0;
  if (!aborted && a.state_out) {
    float vals[32];
    const int col = 32 * (warp >> 2);
    tc::tmem_ld32(tmem + T_S + lbase + col, vals);
    const float f = exp2f(*s_lsfin);
    float* dst = a.state_out + (n * VD + row) * KD + col;
#pragma unroll
    for (int e = 0; e < 32; e += 4)
      *reinterpret_cast<float4*>(dst + e) = make_float4(vals[e] * f, vals[e + 1] * f, vals[e + 2] * f, vals[e + 3] * f);
  }
  if (aborted && tid == 0) {
    if (P.err) atomicExch(P.err, (int)GDNX_ETIMEOUT);
    // let loads still in flight land before the CTA's shared memory is released
    for (int s = 0; s < 2; ++s) {
      tc::mbar_wait(full + s, 0, 1u << 16);
      tc::mbar_wait(full + s, 1, 1u << 16);
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
#ifdef GDNX_PHASE_PROBE
  if (tid == 0) probe_acc[6] = (unsigned long long)(clock64() - t_life);
  if (tid == 0 || tid == 32 || tid == G_NT)
    for (int i = 0; i < 16; ++i)
      if (probe_acc[i]) atomicAdd(&g_wy_probe[i], probe_acc[i]);
#endif
}

// ------------------------------- host side ----------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_encode_mu;
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
  std::lock_guard<std::mutex> lk(g_encode_mu);
  if (!g_encode) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(f);
    else
      cudaGetLastError();
  }
  return g_encode;
}

// 5-D map {dim, lane, head, token, batch} over a [B,T,H,M,128] bf16 view, box
// {64, 1, 1, 64, 1}, 128-byte swizzle.  A lane stride of 0 (shared q/k/v) or a
// single lane drops the lane coordinate (size 1).
bool make_map(const gdnx_view& v, const gdnx_scan_args& a, CUtensorMap* map, int* use_m) {
  if (v.dtype != GDNX_BF16 || (reinterpret_cast<uintptr_t>(v.ptr) & 15)) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  *use_m = (v.sm != 0 && a.M > 1) ? 1 : 0;
  const cuuint64_t kb = 2;  // bytes per element
  cuuint64_t dims[5] = {(cuuint64_t)KD, (cuuint64_t)(*use_m ? a.M : 1), (cuuint64_t)a.H, (cuuint64_t)a.T,
                        (cuuint64_t)a.B};
  cuuint64_t strides[4] = {(cuuint64_t)(*use_m ? v.sm : KD) * kb, (cuuint64_t)v.sh * kb, (cuuint64_t)v.st * kb,
                           (cuuint64_t)v.sb * kb};
  // size-1 dimensions may carry any stride; give them a valid one
  if (a.H == 1) strides[1] = strides[0];
  if (a.T == 1) strides[2] = strides[1];
  if (a.B == 1) strides[3] = strides[2];
  for (int i = 0; i < 4; ++i)
    if (strides[i] == 0 || strides[i] % 16 || strides[i] >= (1ull << 40)) return false;
  cuuint32_t box[5] = {64, 1, 1, (cuuint32_t)C, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(v.ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

#ifdef GDNX_PHASE_PROBE
extern "C" GDNX_API int gdnx_debug_wy_probe(unsigned long long* out8) {
  if (cudaMemcpyFromSymbol(out8, g_wy_probe, 16 * sizeof(unsigned long long)) != cudaSuccess) return 1;
  unsigned long long z[16] = {};
  return cudaMemcpyToSymbol(g_wy_probe, z, sizeof(z)) == cudaSuccess ? 0 : 1;
}
#endif

size_t wy_workspace_bytes(const gdnx_scan_args& a) {
  const int64_t N = a.B * a.H * a.M, nch = (a.T + C - 1) / C;
  return ERR_BYTES + (size_t)N * nch * (TT_ELEMS * 2 + C * 4);
}

constexpr int kMaxPieces = 8, kMaxSideStreams = 64;
// A side stream (plus its events) belongs to one (device, caller stream) pair, so that
// unrelated callers' pass-1 launches are never tied together and a capture of one
// caller's stream pulls in only that caller's side stream.  Created on first use outside
// stream capture, kept until exit.
struct SideStream {
  int dev = -1;
  cudaStream_t caller = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev[kMaxPieces + 1] = {};
  std::mutex mu;  // held while a call enqueues on this side stream
};
std::mutex g_side_mu;
SideStream g_side[kMaxSideStreams];
int g_side_count = 0;

// The side stream of (dev, caller), created if `may_create`; nullptr when none is available
// (table full, creation failed, or not created during a capture).
SideStream* side_stream_for(int dev, cudaStream_t caller, bool may_create) {
  std::lock_guard<std::mutex> lk(g_side_mu);
  for (int i = 0; i < g_side_count; ++i)
    if (g_side[i].dev == dev && g_side[i].caller == caller) return &g_side[i];
  if (!may_create || g_side_count == kMaxSideStreams) return nullptr;
  SideStream& ss = g_side[g_side_count];
  if (cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  int made = 0;
  for (; made < kMaxPieces + 1; ++made)
    if (cudaEventCreateWithFlags(&ss.ev[made], cudaEventDisableTiming) != cudaSuccess) break;
  if (made < kMaxPieces + 1) {  // undo the partial set-up
    cudaGetLastError();
    for (int i = 0; i < made; ++i) cudaEventDestroy(ss.ev[i]);
    cudaStreamDestroy(ss.stream);
    ss.stream = nullptr;
    return nullptr;
  }
  ss.dev = dev;
  ss.caller = caller;
  ++g_side_count;
  return &ss;
}

// Pieces for the pass-1 / pass-2 overlap: enough that each piece's pass 2 (one CTA per
// chain and per SM) is a single wave; none when that would take more than kMaxPieces
// (multi-wave pieces measured slower than one launch).  The environment variable
// GDNX_WY_PIECES overrides the count (1 = no overlap); never more pieces than chains.
int wy_pieces(int64_t n_chains, int sms) {
  static const int forced = [] {
    const char* e = getenv("GDNX_WY_PIECES");
    return e ? atoi(e) : 0;
  }();
  int64_t p;
  if (forced > 0) {
    p = forced > kMaxPieces ? kMaxPieces : forced;
  } else {
    p = (n_chains + sms - 1) / sms;
    if (p > kMaxPieces) p = 1;
  }
  if (p > n_chains) p = n_chains;
  return p < 1 ? 1 : (int)p;
}

gdnx_status launch_wy_scan(const gdnx_scan_args& a, cudaStream_t st) {
  // TMA coordinates are 32-bit and pass 1 runs one CTA per (chain, chunk pair)
  const int64_t n_chains = a.B * a.H * a.M, n_pairs = ((a.T + C - 1) / C + 1) / 2;
  if (a.T > (int64_t(1) << 30) || a.B > (int64_t(1) << 30) || a.H > (int64_t(1) << 30) ||
      n_chains * n_pairs > int64_t(0x7fffffff))
    return GDNX_EUNSUPPORTED;
  WyScanMaps maps;
  if (!make_map(a.q, a, &maps.q, &maps.use_m[0]) || !make_map(a.k, a, &maps.k, &maps.use_m[1]) ||
      !make_map(a.v, a, &maps.v, &maps.use_m[2]))
    return GDNX_EUNSUPPORTED;
  gdnx_view yv;
  yv.ptr = a.y;
  yv.dtype = a.y_dtype;
  yv.dim = VD;
  yv.sb = a.y_sb;
  yv.st = a.y_st;
  yv.sh = a.y_sh;
  yv.sm = a.y_sm;
  yv.ss = 0;
  maps.y_tma = make_map(yv, a, &maps.y, &maps.use_m[3]) ? 1 : 0;
  const int64_t N = a.B * a.H * a.M, nch = (a.T + C - 1) / C;
  WyParams P;
  P.a = a;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.nchunks = nch;
  char* ws = reinterpret_cast<char*>(a.workspace);
  P.err = reinterpret_cast<int*>(ws);
  P.tt = reinterpret_cast<__nv_bfloat16*>(ws + ERR_BYTES);
  P.lsum = reinterpret_cast<float*>(ws + ERR_BYTES + (size_t)N * nch * TT_ELEMS * 2);
  if (cudaMemsetAsync(ws, 0, ERR_BYTES, st) != cudaSuccess) return GDNX_ELAUNCH;
  if (cudaFuncSetAttribute(wy_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(wy_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess ||
      cudaFuncSetAttribute(wy_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S_SMEM) != cudaSuccess)
    return GDNX_ELAUNCH;
  const int64_t npairs = (nch + 1) / 2;
  // The chains go in pieces: pass 1 of every piece on a side stream, pass 2 of piece i on
  // the caller's stream once pass 1 of piece i is done, so pass 1 of later pieces fills
  // the SMs that pass 2 (one CTA per SM) leaves idle in its last wave.
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    return GDNX_ELAUNCH;
  int pieces = wy_pieces(N, sms);
  SideStream* ss = nullptr;
  if (pieces > 1) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return GDNX_ELAUNCH;
    ss = side_stream_for(dev, st, cap == cudaStreamCaptureStatusNone);
    if (!ss) pieces = 1;
  }
  if (pieces == 1) {
    P.n0 = 0;
    wy_prep_kernel<<<(unsigned)(N * npairs), P_NT, P_SMEM, st>>>(P, maps);
    wy_scan_kernel<<<(unsigned)N, S_NT, S_SMEM, st>>>(P, maps);
  } else {
    std::lock_guard<std::mutex> lk(ss->mu);
    // fork: the side stream starts after the caller's earlier work (and the error-word clear)
    if (cudaEventRecord(ss->ev[kMaxPieces], st) != cudaSuccess ||
        cudaStreamWaitEvent(ss->stream, ss->ev[kMaxPieces], 0) != cudaSuccess)
      return GDNX_ELAUNCH;
    gdnx_status status = GDNX_OK;
    for (int i = 0; i < pieces && status == GDNX_OK; ++i) {
      const int64_t c0 = N * i / pieces, c1 = N * (i + 1) / pieces;
      WyParams Pi = P;
      Pi.n0 = c0;
      wy_prep_kernel<<<(unsigned)((c1 - c0) * npairs), P_NT, P_SMEM, ss->stream>>>(Pi, maps);
      if (cudaEventRecord(ss->ev[i], ss->stream) != cudaSuccess || cudaStreamWaitEvent(st, ss->ev[i], 0) != cudaSuccess) {
        status = GDNX_ELAUNCH;
        break;
      }
      wy_scan_kernel<<<(unsigned)(c1 - c0), S_NT, S_SMEM, st>>>(Pi, maps);
    }
    // join: every side-stream launch is ordered before the caller's later work (on an error
    // too, so nothing enqueued here outlives the call unjoined)
    if (status != GDNX_OK) {
      cudaGetLastError();
      if (cudaEventRecord(ss->ev[kMaxPieces], ss->stream) == cudaSuccess)
        cudaStreamWaitEvent(st, ss->ev[kMaxPieces], 0);
      return status;
    }
  }
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
