// General two-pass chunked gated-delta scan on sm_100a: the input forms the
// reference modules pass to their scans, on the tensor cores.
//
//   * separate read key h and write key k: GDN3 vector erase gates h = b (.) k
//     and write gates u = w (.) v (gdn3/gdn3_upgrade.py:472-473,497), or scalar
//     gates; KMD-2's beta_e / beta_w (gdn3/kmd2_fast_scan.py:221-229);
//   * per-key-channel decay (KMD-2, gdn3/kmd2_fast_scan.py:202-205) or one decay
//     per chain-token (GDN3; gamma, log or braided logits);
//   * KMD-2 query slots mixed by out_mix (gdn3/kmd2_fast_scan.py:245) and the
//     update-norm scores |k| |d| (gdn3/kmd2_fast_scan.py:234-235);
//   * q/k/v/gates in fp32, bf16 or fp16 (bf16 tensor-core operands, fp32
//     accumulation and fp32 state), lane RoPE, strided and lane-shared views.
//
// Per chunk of C = 64 tokens of one chain, with G_j the diagonal of cumulative
// decays (per key channel) through token j, read keys h_j, write keys k_j and
// coefficients ce_j (erase), cw_j (write), the delta rule in WY form is
//   A_jl = ce_j (G_j h_j).(k_l / G_l)   (l < j),   T = (I + A)^{-1}
//   W    = T diag(cw) U - T diag(ce) (G H) S0^T     (rows W_j: the token updates)
//   y_i  = S0 (G_i q_i) + sum_{l<=i} ((G_i q_i).(k_l / G_l)) W_l
//   S_C  = S0 G_C + sum_l W_l (k_l G_C / G_l)^T
// (GDN3: ce = cw = alpha(k.h); KMD-2: ce = beta_e, cw = beta_w, h = k.)
//
// Pass 1 (wyg_prep_kernel, one CTA per chain-chunk, all chunks in parallel)
// does every per-token and per-channel step and writes one record per
// chain-chunk: Qd = G q, K' = k G_C / G, -Wk = -T diag(ce) G H, W0^T =
// (T diag(cw) U)^T, Mq^T (the masked query-key Gram) as bf16 tiles in the
// 128-byte-swizzled UMMA layouts, plus G_C and |k|.  The ratios G_j / G_l are
// never formed: the two Gram products run per 16-token row block J of the
// query side, with block anchor b_J = log2 G at token 16J - 1, as
//   (k_l 2^{b_J - L_l}) . (h_j 2^{L_j - b_J})
// (every factor within 2^{+-126} while one block's decay is), on the tensor
// cores (M = 64 keys, N = 32 = 16 read keys + 16 queries of block J).  T is
// formed on the CUDA cores in fp32 (16 x 16 diagonal blocks by substitution,
// then block products).  The per-token log2 decay is clamped to [-7.875,
// 7.875] so one 16-token block spans at most 2^126 -- the same domain as the
// reference's chunk-16 fast scan, whose kDn = k / cumprod(g) assumes a 16-token
// cumulative decay >= 1e-38 (gdn3/kmd2_fast_scan.py:203-205).
//
// Pass 2 (wyg_chain_kernel, one CTA per chain, chunks in sequence) is the state
// chain alone, with the fp32 state in TMEM:
//   G1  W^T  = W0^T I                         (initialises the W accumulator)
//   G2  W^T += S0 (-Wk)^T,  y = S0 Qd^T        (S0 = bf16 copy of the state)
//   G3  y   += W^T Mq^T,    S = S0 G_C + W^T K'
// Warps 0-7 run the chain; warps 8-15 read y (and the update norms for the
// scores) out of TMEM while the next chunk runs.  Every wait is bounded
// (GDNX_ETIMEOUT in the workspace error word, TMEM freed, kernel returns).
#include <cstdlib>

#include "chunk_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "pipe.cuh"
#include "tc.cuh"

namespace gdnx {
namespace {

using namespace chunk;

constexpr int C = 64;
constexpr int KD = 128;
constexpr int VD = 128;
constexpr float kLog2DecayLimit = 7.875f;  // 16 tokens x 7.875 = 126
constexpr size_t ERR_BYTES = 256;

// one record per chain-chunk (bytes): bf16 tiles [2 k blocks][64 rows][128 B] unless noted
constexpr int R_KP = 0;          // K' = k G_C / G
constexpr int R_WK = 16384;      // -Wk
constexpr int R_QD = 32768;      // Qd = G q
constexpr int R_MQ = 49152;      // Mq^T [64 l][64 i] (one block)
constexpr int R_W0 = 57344;      // W0^T [128 v][64 j] (one block)
constexpr int R_GC = 73728;      // fp32 G_C [128], then |k| [64] at +512
constexpr int REC = 74752;

struct GenParams {
  gdnx_scan_args a;
  int kmd2, vec_e, vec_w, chan_decay, scores;
  int64_t nchunks;
  char* rec;  // [N][nchunks][REC]
  int* err;
  int64_t t_off, T_total;  // first token of this slab and the full sequence length (scores layout)
};

// Four consecutive elements (offset a multiple of 4, view 8/16-byte aligned) as fp32.
GDNX_DEV float4 ld4(const void* base, int dtype, int64_t off) {
  if (dtype == GDNX_F32) return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
  const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(base) + off);
  float4 r;
  if (dtype == GDNX_BF16) {
    r.x = __uint_as_float(u.x << 16);
    r.y = __uint_as_float(u.x & 0xffff0000u);
    r.z = __uint_as_float(u.y << 16);
    r.w = __uint_as_float(u.y & 0xffff0000u);
  } else {
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x), b = *reinterpret_cast<const __half2*>(&u.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    r = make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  return r;
}
GDNX_DEV void to4(const float4 v, float* x) { x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w; }

// Byte offset of channels 4 l .. 4 l + 3 of `row` in a K-major SW128 tile of
// 128 channels ([2 blocks][rows][128 B]).
GDNX_DEV uint32_t sw_off4(int row, int l, int rows) {
  const int kb = l >> 4, c16 = (l & 15) >> 1;
  return (uint32_t)(kb * rows * 128 + row * 128 + ((c16 ^ (row & 7)) << 4) + 8 * (l & 1));
}
GDNX_DEV void st4_bf16(char* base, uint32_t off, float a, float b, float c, float d) {
  uint2 u;
  u.x = tc::pack_bf16(a, b);
  u.y = tc::pack_bf16(c, d);
  *reinterpret_cast<uint2*>(base + off) = u;
}

// log2 of one chain-token's decay factor from a dim-1 / braided view.
GDNX_DEV float scalar_log2_decay(const gdnx_scan_args& a, bool kmd2, int64_t off) {
  float l;
  if (a.decay_kind == GDNX_DECAY_BRAIDED) {
    float acc = 0.f;
#pragma unroll
    for (int z = 0; z < 4; ++z)
      acc += expf(-fminf(softplus_f(ld_as_f32(a.decay.ptr, a.decay.dtype, off + z)), 5.0f) * a.braid_rates[z]);
    l = log2f(fminf(acc * 0.25f, a.braid_clamp));
  } else if (a.decay_kind == GDNX_DECAY_LOG) {
    float g = ld_as_f32(a.decay.ptr, a.decay.dtype, off);
    if (!kmd2) g = fminf(g, 0.f);
    l = g * 1.4426950408889634f;
  } else {
    float g = ld_as_f32(a.decay.ptr, a.decay.dtype, off);
    if (!kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
    l = log2f(g);
  }
  return fminf(fmaxf(l, -kLog2DecayLimit), kLog2DecayLimit);  // also maps -inf (a zero factor)
}
GDNX_DEV float chan_log2_decay(float g, int kind, bool kmd2) {
  float l;
  if (kind == GDNX_DECAY_LOG) {
    if (!kmd2) g = fminf(g, 0.f);
    l = g * 1.4426950408889634f;
  } else {
    if (!kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
    l = log2f(g);
  }
  return fminf(fmaxf(l, -kLog2DecayLimit), kLog2DecayLimit);
}

// ------------------------------- pass 1 ------------------------------------
constexpr int P_NT = 256;
constexpr int LDT = 64;  // fp32 row stride of the A / R matrices
// shared memory (bytes from a 1024-aligned base)
constexpr int P_OFF_HQ = 0;        // [2 kb][128 rows][128 B]: block J rows 32J.. h^, 32J+16.. q^;
                                   // later T_e | T_w bf16 [64][128 B] each
constexpr int P_OFF_KB = 32768;    // 2 x [2 kb][64 rows][128 B] K^(J) buffers; later A (fp32 [64][64]) | R
constexpr int P_OFF_H0 = 65536;    // G h  [2 kb][64][128 B]
constexpr int P_OFF_U = 81920;     // u    [2 kb][64][128 B]
constexpr int P_OFF_SC = 98304;    // fp32: anchors [4][128], warp totals [8][128], L_C [128],
                                   // ce, cw, |k| [64] each, inv_freq [64]
constexpr int P_OFF_ANC = P_OFF_SC;
constexpr int P_OFF_WT = P_OFF_ANC + 4 * 128 * 4;
constexpr int P_OFF_LC = P_OFF_WT + 8 * 128 * 4;
constexpr int P_OFF_CE = P_OFF_LC + 128 * 4;
constexpr int P_OFF_CW = P_OFF_CE + 256;
constexpr int P_OFF_KN = P_OFF_CW + 256;
constexpr int P_OFF_INV = P_OFF_KN + 256;
constexpr int P_OFF_BAR = P_OFF_INV + 256;
constexpr int P_SMEM = P_OFF_BAR + 64 + 1024;
static_assert(2 * 64 * LDT * 4 <= 32768, "A and R over the K^(J) buffers");

// Column c of one 16 x 16 diagonal block of T = (I + A)^{-1} by forward substitution,
// written over that block of A (block rows/columns B0 .. B0 + 15).
GDNX_DEV void subst16(float* A, int B0, int c) {
  float x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float s0 = (i == c) ? 1.f : 0.f, s1 = 0.f;
#pragma unroll
    for (int l = 0; l < i; l += 2) {
      s0 = fmaf(-A[(B0 + i) * LDT + B0 + l], x[l], s0);
      if (l + 1 < i) s1 = fmaf(-A[(B0 + i) * LDT + B0 + l + 1], x[l + 1], s1);
    }
    x[i] = (i < c) ? 0.f : s0 + s1;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 16; ++i) A[(B0 + i) * LDT + B0 + c] = x[i];
}

__global__ void __launch_bounds__(P_NT, 2) wyg_prep_kernel(const GenParams P) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = tc::align_smem(smraw, 1024);
  char* cHQ = reinterpret_cast<char*>(sm + P_OFF_HQ);
  char* cH0 = reinterpret_cast<char*>(sm + P_OFF_H0);
  char* cU = reinterpret_cast<char*>(sm + P_OFF_U);
  float* sAnc = reinterpret_cast<float*>(sm + P_OFF_ANC);
  float* sWT = reinterpret_cast<float*>(sm + P_OFF_WT);
  float* sLC = reinterpret_cast<float*>(sm + P_OFF_LC);
  float* sCE = reinterpret_cast<float*>(sm + P_OFF_CE);
  float* sCW = reinterpret_cast<float*>(sm + P_OFF_CW);
  float* sKN = reinterpret_cast<float*>(sm + P_OFF_KN);
  float* sInv = reinterpret_cast<float*>(sm + P_OFF_INV);
  uint64_t* gbar = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);  // [2] MMA completion
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + P_OFF_BAR + 16);

  const gdnx_scan_args& a = P.a;
  const bool kmd2 = P.kmd2 != 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n = blockIdx.x / P.nchunks, ch = blockIdx.x % P.nchunks;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int lm = (int)m;
  const int64_t t0 = ch * C;
  const int dpairs = (a.rope.enable && lm < 4) ? a.rope.pairs[lm] : 0;
  const int dp4 = dpairs / 4;
  const float rsc = dpairs > 0 ? a.rope.scale[lm] : 0.f;
  char* rec = P.rec + (size_t)(n * P.nchunks + ch) * REC;

  if (warp == 7) tc::tmem_alloc(s_tmem, 256);
  if (tid == 0) {
    tc::mbar_init(gbar, 1);
    tc::mbar_init(gbar + 1, 1);
  }
  if (dpairs > 0 && tid >= 64 && tid < 128) sInv[tid - 64] = 1.0f / powf(10000.0f, (float)(tid - 64) / a.rope.den[lm]);

  // ---- 1. log2 decay prefix: warp w holds tokens 8w .. 8w+7, lane l channels 4l .. 4l+3 ----
  float Lr[8][4];
  {
    float run[4] = {0.f, 0.f, 0.f, 0.f};
    float sl = 0.f;  // scalar decays: lane jj < 8 holds token 8w + jj
    if (!P.chan_decay && lane < 8) {
      const int64_t t = t0 + 8 * warp + lane;
      if (t < a.T) sl = scalar_log2_decay(a, kmd2, view_off(a.decay, b, t, h, m));
    }
    float4 graw[8];  // per-channel decays of the warp's 8 tokens, all loads issued first
    if (P.chan_decay) {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int64_t t = t0 + 8 * warp + jj;
        graw[jj] = t < a.T ? ld4(a.decay.ptr, a.decay.dtype, view_off(a.decay, b, t, h, m) + 4 * lane)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int64_t t = t0 + 8 * warp + jj;
      float l4[4];
      if (P.chan_decay) {
        if (t < a.T) {
          to4(graw[jj], l4);
#pragma unroll
          for (int e = 0; e < 4; ++e) l4[e] = chan_log2_decay(l4[e], a.decay_kind, kmd2);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) l4[e] = 0.f;
        }
      } else {
        const float s = __shfl_sync(0xffffffffu, sl, jj);
#pragma unroll
        for (int e = 0; e < 4; ++e) l4[e] = s;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        run[e] += l4[e];
        Lr[jj][e] = run[e];
      }
    }
    *reinterpret_cast<float4*>(sWT + warp * 128 + 4 * lane) = make_float4(run[0], run[1], run[2], run[3]);
  }
  __syncthreads();
  {
    float off[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < warp; ++w) {
      const float4 t = *reinterpret_cast<const float4*>(sWT + w * 128 + 4 * lane);
      off[0] += t.x; off[1] += t.y; off[2] += t.z; off[3] += t.w;
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
#pragma unroll
      for (int e = 0; e < 4; ++e) Lr[jj][e] += off[e];
    // row-block anchors b_J = L at token 16J - 1 (b_0 = 0), and L_C = L at token 63
    if (warp == 0) *reinterpret_cast<float4*>(sAnc + 4 * lane) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (warp & 1) {
      float* dst = (warp == 7) ? sLC : sAnc + ((warp + 1) / 2) * 128;
      *reinterpret_cast<float4*>(dst + 4 * lane) = make_float4(Lr[7][0], Lr[7][1], Lr[7][2], Lr[7][3]);
    }
  }
  __syncthreads();

  // ---- 2. token rows: loads, lane RoPE, gates, operands ----
  // A warp's next token is fetched with cp.async into its staging slot (over the K^(J)
  // buffers, free until section 3) while the current one is processed: rows of q (each
  // query slot), k, v and the vector gates, this lane's 4 elements of each.
  constexpr int kStgRows = 6, kStgBytes = kStgRows * 128 * 4;
  const bool stage = a.r_out <= 4 && a.r_out + 2 + P.vec_e + P.vec_w <= kStgRows;
  char* stg = reinterpret_cast<char*>(sm + P_OFF_KB) + warp * kStgBytes;
  const int nq = a.r_out > 1 ? a.r_out : 1;
  auto es_of = [](int dt) { return dt == GDNX_F32 ? 4 : 2; };
  auto cp_row = [&](int row, const gdnx_view& v, int64_t off) {  // this lane's 4 elements
    const int es = es_of(v.dtype);
    const char* src = reinterpret_cast<const char*>(v.ptr) + (off + 4 * lane) * es;
    const uint32_t dst = tc::smem_u32(stg + row * 512 + 16 * lane);
    if (es == 4)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    else
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
  };
  auto rd_row = [&](int row, int dt, float* x) {  // this lane's 4 staged elements as fp32
    const char* p = stg + row * 512 + 16 * lane;
    if (dt == GDNX_F32) {
      to4(*reinterpret_cast<const float4*>(p), x);
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(p);
      if (dt == GDNX_BF16) {
        x[0] = __uint_as_float(u.x << 16); x[1] = __uint_as_float(u.x & 0xffff0000u);
        x[2] = __uint_as_float(u.y << 16); x[3] = __uint_as_float(u.y & 0xffff0000u);
      } else {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        x[0] = lo.x; x[1] = lo.y; x[2] = hi.x; x[3] = hi.y;
      }
    }
  };
  float nbe = 0.f, nbw = 0.f;  // scalar gates of the staged token
  auto issue = [&](int jj) {
    const int64_t t = t0 + 8 * warp + jj;
    if (t >= a.T) return;
    for (int r = 0; r < nq; ++r)
      cp_row(r, a.q, a.r_out <= 1 ? view_off(a.q, b, t, h, m) : view_off(a.q, b, t, h, m, r));
    cp_row(nq, a.k, view_off(a.k, b, t, h, m));
    cp_row(nq + 1, a.v, view_off(a.v, b, t, h, m));
    if (P.vec_e) cp_row(nq + 2, a.gate_e, view_off(a.gate_e, b, t, h, m));
    else nbe = ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m));
    if (P.vec_w) cp_row(nq + 2 + P.vec_e, a.gate_w, view_off(a.gate_w, b, t, h, m));
    else nbw = ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m));
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (stage) issue(0);
  float kreg[8][4];
  {
    const bool role1 = lane < dp4, role2 = lane >= dp4 && lane < 2 * dp4;
    const int partner = role1 ? lane + dp4 : (role2 ? lane - dp4 : lane);
    const float4 lc4 = *reinterpret_cast<const float4*>(sLC + 4 * lane);
    const float lc[4] = {lc4.x, lc4.y, lc4.z, lc4.w};
#pragma unroll 1
    for (int jj = 0; jj < 8; ++jj) {
      const int j = 8 * warp + jj;
      const int64_t t = t0 + j;
      const bool valid = t < a.T;
      float q[4] = {0.f, 0.f, 0.f, 0.f}, k[4] = {0.f, 0.f, 0.f, 0.f}, hv[4], u[4] = {0.f, 0.f, 0.f, 0.f};
      float ce = 0.f, cw = 0.f;
      float sge[4] = {0.f, 0.f, 0.f, 0.f}, sgw[4] = {0.f, 0.f, 0.f, 0.f}, sbe = 0.f, sbw = 0.f;
      if (stage) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (valid) {
          if (a.r_out <= 1) {
            rd_row(0, a.q.dtype, q);
          } else {
            for (int r = 0; r < a.r_out; ++r) {
              float qr[4];
              rd_row(r, a.q.dtype, qr);
              const float mix = a.out_mix[h * a.r_out + r];
#pragma unroll
              for (int e = 0; e < 4; ++e) q[e] = fmaf(mix, qr[e], q[e]);
            }
          }
          rd_row(nq, a.k.dtype, k);
          rd_row(nq + 1, a.v.dtype, u);
          if (P.vec_e) rd_row(nq + 2, a.gate_e.dtype, sge);
          if (P.vec_w) rd_row(nq + 2 + P.vec_e, a.gate_w.dtype, sgw);
          sbe = nbe;
          sbw = nbw;
        }
        __syncwarp();
        if (jj + 1 < 8) issue(jj + 1);
      } else if (valid) {
        if (a.r_out <= 1) {
          to4(ld4(a.q.ptr, a.q.dtype, view_off(a.q, b, t, h, m) + 4 * lane), q);
        } else {
          for (int r = 0; r < a.r_out; ++r) {
            float qr[4];
            to4(ld4(a.q.ptr, a.q.dtype, view_off(a.q, b, t, h, m, r) + 4 * lane), qr);
            const float mix = a.out_mix[h * a.r_out + r];
#pragma unroll
            for (int e = 0; e < 4; ++e) q[e] = fmaf(mix, qr[e], q[e]);
          }
        }
        to4(ld4(a.k.ptr, a.k.dtype, view_off(a.k, b, t, h, m) + 4 * lane), k);
        to4(ld4(a.v.ptr, a.v.dtype, view_off(a.v, b, t, h, m) + 4 * lane), u);
      }
      // lane RoPE: pair i = (x[i], x[i + dpairs]); x1' = x1 c - x2 s, x2' = x1' s + x2 c
      if (dpairs > 0) {
        float pk[4], pq[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          pk[e] = __shfl_sync(0xffffffffu, k[e], partner);
          pq[e] = __shfl_sync(0xffffffffu, q[e], partner);
        }
        if (role1 || role2) {
          const float pos = (float)(a.rope.pos0 + t);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = role1 ? 4 * lane + e : 4 * lane + e - dpairs;
            float sn, cs;
            sincos_reduced(pos * rsc * sInv[i], &sn, &cs);
            const float k1 = role1 ? k[e] : pk[e], k2 = role1 ? pk[e] : k[e];
            const float q1 = role1 ? q[e] : pq[e], q2 = role1 ? pq[e] : q[e];
            const float nk = k1 * cs - k2 * sn, nq = q1 * cs - q2 * sn;
            k[e] = role1 ? nk : nk * sn + k2 * cs;
            q[e] = role1 ? nq : nq * sn + q2 * cs;
          }
        }
      }
      // gates: read key h, write value u, coefficients ce / cw
      float be = 0.f, bw = 0.f;
      if (valid) {
        if (P.vec_e) {
          float g4[4];
          if (stage) {
#pragma unroll
            for (int e = 0; e < 4; ++e) g4[e] = sge[e];
          } else {
            to4(ld4(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m) + 4 * lane), g4);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) hv[e] = g4[e] * k[e];
        } else {
          be = stage ? sbe : ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m));
#pragma unroll
          for (int e = 0; e < 4; ++e) hv[e] = kmd2 ? k[e] : be * k[e];
        }
        if (P.vec_w) {
          float w4[4];
          if (stage) {
#pragma unroll
            for (int e = 0; e < 4; ++e) w4[e] = sgw[e];
          } else {
            to4(ld4(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m) + 4 * lane), w4);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) u[e] *= w4[e];
        } else {
          bw = stage ? sbw : ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m));
          if (!kmd2)
#pragma unroll
            for (int e = 0; e < 4; ++e) u[e] *= bw;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) hv[e] = 0.f;
      }
      const float kh = warp_sum(k[0] * hv[0] + k[1] * hv[1] + k[2] * hv[2] + k[3] * hv[3]);
      const float kk = warp_sum(k[0] * k[0] + k[1] * k[1] + k[2] * k[2] + k[3] * k[3]);
      if (valid) {
        if (kmd2) {
          ce = be;
          cw = bw;
        } else {
          ce = cw = stable_alpha(kh);
        }
      }
      if (lane == 0) {
        sCE[j] = ce;
        sCW[j] = cw;
        sKN[j] = sqrtf(kk);
      }
      // operands (bf16, swizzled rows)
      const int J = j >> 4;
      const float4 an4 = *reinterpret_cast<const float4*>(sAnc + J * 128 + 4 * lane);
      const float an[4] = {an4.x, an4.y, an4.z, an4.w};
      float fb[4], f0[4], fc[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        fb[e] = exp2f(Lr[jj][e] - an[e]);  // <= 1 within the block
        f0[e] = exp2f(Lr[jj][e]);
        fc[e] = exp2f(lc[e] - Lr[jj][e]);
      }
      const int rh = 32 * J + (j & 15);
      st4_bf16(cHQ, sw_off4(rh, lane, 128), hv[0] * fb[0], hv[1] * fb[1], hv[2] * fb[2], hv[3] * fb[3]);
      st4_bf16(cHQ, sw_off4(rh + 16, lane, 128), q[0] * fb[0], q[1] * fb[1], q[2] * fb[2], q[3] * fb[3]);
      st4_bf16(cH0, sw_off4(j, lane, 64), hv[0] * f0[0], hv[1] * f0[1], hv[2] * f0[2], hv[3] * f0[3]);
      st4_bf16(cU, sw_off4(j, lane, 64), u[0], u[1], u[2], u[3]);
      st4_bf16(rec + R_QD, sw_off4(j, lane, 64), q[0] * f0[0], q[1] * f0[1], q[2] * f0[2], q[3] * f0[3]);
      st4_bf16(rec + R_KP, sw_off4(j, lane, 64), k[0] * fc[0], k[1] * fc[1], k[2] * fc[2], k[3] * fc[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) kreg[jj][e] = k[e];
    }
  }

  // ---- 3. Gram products per query row block J on the tensor cores ----
  // D[l][32J + c]: c < 16: (k_l.h_j) 2^{L_j - L_l}, j = 16J + c;  c >= 16: (k_l.q_i) 2^{L_i - L_l}
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t sHQ = tc::smem_u32(cHQ);
  bool ok = true;
  uint32_t gph[2] = {0, 0};
  constexpr uint32_t ID_G = tc::idesc_bf16(64, 32, false, false);
#pragma unroll 1
  for (int J = 0; J < 4; ++J) {
    char* kb = reinterpret_cast<char*>(sm + P_OFF_KB + 16384 * (J & 1));
    if (J >= 2) {  // the buffer's previous products are done
      ok = ok && tc::mbar_wait(gbar + (J & 1), gph[J & 1]);
      gph[J & 1] ^= 1;
    }
    const float4 an4 = *reinterpret_cast<const float4*>(sAnc + J * 128 + 4 * lane);
    const float an[4] = {an4.x, an4.y, an4.z, an4.w};
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int l = 8 * warp + jj;
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = (J >= (l >> 4)) ? kreg[jj][e] * exp2f(an[e] - Lr[jj][e]) : 0.f;
      st4_bf16(kb, sw_off4(l, lane, 64), x[0], x[1], x[2], x[3]);
    }
    tc::fence_async_smem();
    tc::fence_before();
    ok = !__syncthreads_or(!ok);
    if (ok && tid == 0) {
      tc::fence_after();
      const uint32_t skb = tc::smem_u32(kb);
#pragma unroll
      for (int s = 0; s < 8; ++s)
        tc::mma_bf16(tmem + 32 * J, tc::smem_desc(skb + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024),
                     tc::smem_desc(sHQ + (s >> 2) * 16384 + 32 * J * 128 + (s & 3) * 32, 16, 1024), ID_G, s > 0);
      tc::commit(gbar + (J & 1));
    }
  }
  ok = ok && tc::mbar_wait(gbar + 0, gph[0]);
  gph[0] ^= 1;
  ok = ok && tc::mbar_wait(gbar + 1, gph[1]);
  gph[1] ^= 1;
  ok = !__syncthreads_or(!ok);
  tc::fence_after();

  // ---- 4. masks: A (fp32, rows j) and Mq^T (bf16 record tile, rows l) ----
  float* sA = reinterpret_cast<float*>(sm + P_OFF_KB);
  float* sR = sA + 64 * LDT;
  const int quad = warp & 3;
  const int lrow = 16 * quad + (lane & 15);  // M = 64 accumulator row of this thread (lanes < 16)
  const uint32_t tl = (uint32_t)(32 * quad) << 16;
  if (ok) {
    if (warp < 4) {
#pragma unroll
      for (int J = 0; J < 4; ++J) {
        float d[16];
        tc::tmem_ld16(tmem + tl + 32 * J, d);
        if (lane < 16)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int j = 16 * J + e;
            if (lrow < j) sA[j * LDT + lrow] = sCE[j] * d[e];
          }
      }
    } else {
      char* mq = rec + R_MQ;
#pragma unroll
      for (int J = 0; J < 4; ++J) {
        float d[16];
        tc::tmem_ld16(tmem + tl + 32 * J + 16, d);
        if (lane < 16)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float v8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v8[e] = (16 * J + 8 * hh + e >= lrow) ? d[8 * hh + e] : 0.f;
            tc::st_chunk_bf16(mq, tc::sw128(lrow, 2 * J + hh, 64), v8);
          }
      }
    }
  }
  __syncthreads();

  // ---- 5. T = (I + A)^{-1}: diagonal blocks, R_IK = T_II A_IK, then T_IJ by block products ----
  if (ok && tid < 64) subst16(sA, 16 * (tid >> 4), tid & 15);
  __syncthreads();
  if (ok) {
    // R_IK for the six blocks I > K: 1536 elements
    for (int it = tid; it < 6 * 256; it += P_NT) {
      const int blk = it >> 8, e = it & 255, r = e >> 4, c = e & 15;
      // blocks (I, K): (1,0) (2,0) (3,0) (2,1) (3,1) (3,2)
      const int Ii = (blk == 0) ? 1 : (blk == 1) ? 2 : (blk == 2) ? 3 : (blk == 3) ? 2 : 3;
      const int Kk = (blk < 3) ? 0 : (blk < 5) ? 1 : 2;
      float s = 0.f;
#pragma unroll
      for (int x = 0; x < 16; ++x) s = fmaf(sA[(16 * Ii + r) * LDT + 16 * Ii + x], sA[(16 * Ii + x) * LDT + 16 * Kk + c], s);
      sR[(16 * Ii + r) * LDT + 16 * Kk + c] = s;
    }
  }
  __syncthreads();
  // T_IJ = -sum_{K=J}^{I-1} R_IK T_KJ, by distance I - J (T_JJ on the diagonal of A; the
  // off-diagonal T blocks replace A's, which R has consumed)
#pragma unroll 1
  for (int dist = 1; dist < 4; ++dist) {
    if (ok) {
      const int nblk = 4 - dist;
      for (int it = tid; it < nblk * 256; it += P_NT) {
        const int J = it >> 8, e = it & 255, r = e >> 4, c = e & 15, I = J + dist;
        float s = 0.f;
        for (int K = J; K < I; ++K)
#pragma unroll
          for (int x = 0; x < 16; ++x) s = fmaf(sR[(16 * I + r) * LDT + 16 * K + x], sA[(16 * K + x) * LDT + 16 * J + c], s);
        sA[(16 * I + r) * LDT + 16 * J + c] = -s;
      }
    }
    __syncthreads();
  }

  // ---- 6. T_e = T diag(ce), T_w = T diag(cw) as bf16 K-major tiles over HQ ----
  char* cTe = cHQ;
  char* cTw = cHQ + 8192;
  if (ok) {
    for (int it = tid; it < 64 * 8; it += P_NT) {
      const int j = it >> 3, c8 = it & 7;
      float te[8], tw[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int l = 8 * c8 + e;
        const float tv = ((l >> 4) <= (j >> 4)) ? sA[j * LDT + l] : 0.f;
        te[e] = tv * sCE[l];
        tw[e] = tv * sCW[l];
      }
      tc::st_chunk_bf16(cTe, tc::sw128(j, c8, 64), te);
      tc::st_chunk_bf16(cTw, tc::sw128(j, c8, 64), tw);
    }
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  // ---- 7. Wk = T_e (G H) -> TMEM cols 0..127 (M = 64);  W0^T = U^T T_w^T -> cols 128..191 ----
  if (ok && tid == 0) {
    tc::fence_after();
    const uint32_t sTe = tc::smem_u32(cTe), sTw = tc::smem_u32(cTw);
    const uint32_t sH0 = tc::smem_u32(cH0), sU = tc::smem_u32(cU);
    constexpr uint32_t ID_WK = tc::idesc_bf16(64, 128, false, true);
    constexpr uint32_t ID_W0 = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma_bf16(tmem, tc::smem_desc(sTe + k * 32, 16, 1024), tc::smem_desc(sH0 + k * 2048, 8192, 1024), ID_WK, k > 0);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma_bf16(tmem + 128, tc::smem_desc(sU + k * 2048, 8192, 1024), tc::smem_desc(sTw + k * 32, 16, 1024), ID_W0,
                   k > 0);
    tc::commit(gbar);
  }
  ok = ok && tc::mbar_wait(gbar, gph[0]);
  ok = !__syncthreads_or(!ok);
  tc::fence_after();
  // ---- 8. read-outs to the record ----
  if (ok) {
    const int half = warp >> 2;
    {  // -Wk rows j = lrow (lanes < 16), k block `half`
      float d[32];
      char* wk = rec + R_WK;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        tc::tmem_ld32(tmem + tl + 64 * half + 32 * hh, d);
        if (lane < 16)
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            float v8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v8[e] = -d[8 * q4 + e];
            tc::st_chunk_bf16(wk, half * 8192 + tc::sw128(lrow, 4 * hh + q4, 64), v8);
          }
      }
    }
    {  // W0^T rows v = 32 quad + lane, columns j of half `half`
      float d[32];
      tc::tmem_ld32(tmem + 128 + tl + 32 * half, d);
      const int v = 32 * quad + lane;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tc::st_chunk_bf16(rec + R_W0, tc::sw128(v, 4 * half + q4, 128), d + 8 * q4);
    }
    float* gc = reinterpret_cast<float*>(rec + R_GC);
    if (tid < 128) gc[tid] = exp2f(sLC[tid]);
    else if (tid < 192) gc[128 + (tid - 128)] = sKN[tid - 128];
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 7) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
  if (!ok && tid == 0 && P.err) atomicExch(P.err, (int)GDNX_ETIMEOUT);
}

// ------------------------------- pass 2 ------------------------------------
constexpr int S_NT = 512;  // warps 0-7: state chain; warps 8-15: output
constexpr int G_NT = 256;
constexpr int KB = 24576;  // k-block stride of a stage's [K' ; -Wk ; Qd] tile (192 rows)
constexpr int ST_KQ = 0, ST_MQ = 49152, ST_W0 = 57344, ST_GC = 73728, ST_BYTES = REC;
constexpr int S_OFF_I = 2 * ST_BYTES;          // identity [64][64] (S0 and W^T operands live in TMEM)
constexpr int S_OFF_KN = S_OFF_I + 8192;       // [2][64] |k| copies, [2][64] score sums
constexpr int S_OFF_BAR = S_OFF_KN + 1024;
constexpr int S_SMEM = S_OFF_BAR + 128 + 1024;
static_assert(S_SMEM <= 232448, "shared memory");
static_assert(ST_GC + 1024 == ST_BYTES, "stage layout");
// TMEM columns: S | W^T(0) | y(0) | W^T(1) | y(1) | S bf16 (64) | W^T bf16 (32).  The A operands of
// G2 (S0) and G3 (W^T) are read from TMEM as packed bf16 pairs; the fp32 W^T stays for the scores.
constexpr uint32_t T_S = 0, T_SB = 384, T_WB = 448;
GDNX_DEV uint32_t t_w(int s) { return 128u + 128u * (uint32_t)s; }
GDNX_DEV uint32_t t_y(int s) { return 192u + 128u * (uint32_t)s; }

__global__ void __launch_bounds__(S_NT, 1) wyg_chain_kernel(const GenParams P) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = tc::align_smem(smraw, 1024);
  float* sKNc = reinterpret_cast<float*>(sm + S_OFF_KN);  // [2][64]
  float* sSum = sKNc + 128;                               // [2][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S_OFF_BAR);
  uint64_t* full = bars;       // [2] stage loaded
  uint64_t* g2 = bars + 2;     // G1 + G2 complete
  uint64_t* g3 = bars + 3;     // [2] G3 complete
  uint64_t* drained = bars + 5;  // [2] output group done with a stage's TMEM
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + S_OFF_BAR + 72);

  const gdnx_scan_args& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, row = 32 * quad + lane;
  const uint32_t lbase = (uint32_t)(32 * quad) << 16;
  const int64_t n = blockIdx.x;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int64_t nchunks = P.nchunks;
  const uint32_t sbase = tc::smem_u32(sm);
  const char* recs = P.rec + (size_t)n * nchunks * REC;

  if (warp == 0) tc::tmem_alloc(s_tmem, 512);
  if (tid == 0) {
    for (int i = 0; i < 7; ++i) tc::mbar_init(bars + i, 1);
    *s_abort = 0;
  }
  // identity tile (bf16, K-major [64][64])
  for (int it = tid; it < 64 * 8; it += S_NT) {
    const int r = it >> 3, c8 = it & 7;
    float v8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v8[e] = (8 * c8 + e == r) ? 1.f : 0.f;
    tc::st_chunk_bf16(reinterpret_cast<char*>(sm + S_OFF_I), tc::sw128(r, c8, 64), v8);
  }
  if (tid < 128) sSum[tid] = 0.f;
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;

  auto issue_stage = [&](int64_t c) {  // one thread
    const int s = (int)(c & 1);
    const uint32_t bar = tc::smem_u32(full + s);
    const uint32_t st = sbase + s * ST_BYTES;
    const char* r = recs + (size_t)c * REC;
    pipe::expect_tx(bar, ST_BYTES);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      pipe::bulk_load(st + ST_KQ + kb * KB, r + R_KP + kb * 8192, 8192, bar);
      pipe::bulk_load(st + ST_KQ + kb * KB + 64 * 128, r + R_WK + kb * 8192, 8192, bar);
      pipe::bulk_load(st + ST_KQ + kb * KB + 128 * 128, r + R_QD + kb * 8192, 8192, bar);
    }
    pipe::bulk_load(st + ST_MQ, r + R_MQ, 8192, bar);
    pipe::bulk_load(st + ST_W0, r + R_W0, 16384, bar);
    pipe::bulk_load(st + ST_GC, r + R_GC, 1024, bar);
  };
  if (tid == 0) {
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

  constexpr uint32_t ID_N64 = tc::idesc_bf16(128, 64, false, false);
  constexpr uint32_t ID_Y3 = tc::idesc_bf16(128, 64, false, true);
  constexpr uint32_t ID_S3 = tc::idesc_bf16(128, 128, false, true);
  const uint32_t sI = sbase + S_OFF_I;

  if (warp < 8) {
    // ============================ state chain ============================
    const int half = warp >> 2;
    for (int64_t c = 0; c < nchunks; ++c) {
      const int s = (int)(c & 1);
      const uint32_t st = sbase + s * ST_BYTES;
      bool ok = pipe::wait_or_abort(full + s, (uint32_t)((c >> 1) & 1), s_abort);
      if (ok && c >= 2) ok = pipe::wait_or_abort(drained + s, (uint32_t)(((c - 2) >> 1) & 1), s_abort);
      if (pipe::group_any(2, G_NT, !ok)) break;
      tc::fence_after();
      // G1: W^T = W0^T I (independent of the state; overlaps the conversion below)
      if (tid == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16(tmem + t_w(s), tc::smem_desc(st + ST_W0 + k * 32, 16, 1024),
                       tc::smem_desc(sI + k * 32, 16, 1024), ID_N64, k > 0);
      }
      // S -> bf16 operand; S <- S G_C in TMEM (per key column)
      {
        const float* gc = reinterpret_cast<const float*>(sm + s * ST_BYTES + ST_GC);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int col = 64 * half + 32 * hh;
          float vals[32];
          tc::tmem_ld32(tmem + T_S + lbase + col, vals);
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = tc::pack_bf16(vals[2 * e], vals[2 * e + 1]);
          tc::tmem_st16u(tmem + T_SB + lbase + col / 2, pk);
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 g = *reinterpret_cast<const float4*>(gc + col + e);
            vals[e] *= g.x; vals[e + 1] *= g.y; vals[e + 2] *= g.z; vals[e + 3] *= g.w;
          }
          tc::tmem_st32(tmem + T_S + lbase + col, vals);
        }
      }
      tc::fence_before();
      pipe::group_sync(2, G_NT);
      // G2: W^T += S0 (-Wk)^T;  y = S0 Qd^T
      if (tid == 0) {
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t a_t = tmem + T_SB + 8 * k;
          const uint32_t kq = st + ST_KQ + (k >> 2) * KB + (k & 3) * 32;
          tc::mma_bf16_ts(tmem + t_w(s), a_t, tc::smem_desc(kq + 64 * 128, 16, 1024), ID_N64, 1);
          tc::mma_bf16_ts(tmem + t_y(s), a_t, tc::smem_desc(kq + 128 * 128, 16, 1024), ID_N64, k > 0);
        }
        tc::commit(g2);
      }
      ok = pipe::wait_or_abort(g2, (uint32_t)(c & 1), s_abort);
      tc::fence_after();
      if (pipe::group_any(2, G_NT, !ok)) break;
      {  // W^T -> bf16 A operand
        float w[32];
        tc::tmem_ld32(tmem + t_w(s) + lbase + 32 * half, w);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = tc::pack_bf16(w[2 * e], w[2 * e + 1]);
        tc::tmem_st16u(tmem + T_WB + lbase + 16 * half, pk);
      }
      tc::fence_before();
      pipe::group_sync(2, G_NT);
      // G3: y += W^T Mq^T;  S += W^T K'
      if (tid == 0) {
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t a_t = tmem + T_WB + 8 * k;
          tc::mma_bf16_ts(tmem + t_y(s), a_t, tc::smem_desc(st + ST_MQ + k * 2048, 8192, 1024), ID_Y3, 1);
          tc::mma_bf16_ts(tmem + T_S, a_t, tc::smem_desc(st + ST_KQ + k * 2048, KB, 1024), ID_S3, 1);
        }
        tc::commit(g3 + s);
      }
      ok = pipe::wait_or_abort(g3 + s, (uint32_t)((c >> 1) & 1), s_abort);
      tc::fence_after();
      if (pipe::group_any(2, G_NT, !ok)) break;
      // stage s is consumed: keep its |k| for the scores, then fetch chunk c + 2 into it
      if (warp == 1) {
        const float* kn = reinterpret_cast<const float*>(sm + s * ST_BYTES + ST_GC) + 128;
        sKNc[64 * s + lane] = kn[lane];
        sKNc[64 * s + 32 + lane] = kn[32 + lane];
        __syncwarp();
        if (lane == 0 && c + 2 < nchunks) issue_stage(c + 2);
      }
    }
  } else {
    // ============================== output ==============================
    const int ptid = tid - G_NT, half = (warp - 8) >> 2;
    const int64_t ybase = b * a.y_sb + h * a.y_sh + m * a.y_sm;
    for (int64_t c = 0; c < nchunks; ++c) {
      const int s = (int)(c & 1);
      const bool ok = pipe::wait_or_abort(g3 + s, (uint32_t)((c >> 1) & 1), s_abort);
      tc::fence_after();
      if (pipe::group_any(1, G_NT, !ok)) break;
      const int nt = (int)((a.T - c * C) < C ? (a.T - c * C) : C);
      {
        float yv[32];
        tc::tmem_ld32(tmem + t_y(s) + lbase + 32 * half, yv);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int i = 32 * half + e;
          if (i < nt) st_from_f32(a.y, a.y_dtype, ybase + row + (c * C + i) * a.y_st, yv[e]);
        }
      }
      if (P.scores) {
        // |W_j|^2 = sum_v W^T[v][j]^2: a transposing warp reduction leaves column `lane`
        // of this warp's 32 in lane `lane`; the four row quadrants meet in shared memory
        float w[32];
        tc::tmem_ld32(tmem + t_w(s) + lbase + 32 * half, w);
#pragma unroll
        for (int e = 0; e < 32; ++e) w[e] *= w[e];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
#pragma unroll
          for (int e = 0; e < o; ++e) {
            const bool up = (lane & o) != 0;
            const float send = up ? w[e] : w[e + o];
            const float keep = up ? w[e + o] : w[e];
            w[e] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        atomicAdd(sSum + 64 * s + 32 * half + lane, w[0]);
        pipe::group_sync(1, G_NT);
        if (ptid < 64) {
          const int i = ptid;
          if (i < nt)
            a.scores[((b * P.T_total + P.t_off + c * C + i) * a.H + h) * a.M + m] =
                sKNc[64 * s + i] * sqrtf(sSum[64 * s + i]);
          sSum[64 * s + i] = 0.f;
        }
      }
      tc::fence_before();
      pipe::group_sync(1, G_NT);
      if (ptid == 0) pipe::mbar_arrive(drained + s);
    }
  }

  __syncthreads();
  tc::fence_after();
  const bool aborted = *s_abort != 0;
  if (!aborted && a.state_out) {
    float vals[32];
    const int col = 32 * (warp >> 2);
    tc::tmem_ld32(tmem + T_S + lbase + col, vals);
    float* dst = a.state_out + (n * VD + row) * KD + col;
#pragma unroll
    for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(vals[e], vals[e + 1], vals[e + 2], vals[e + 3]);
  }
  if (aborted && tid == 0) {
    if (P.err) atomicExch(P.err, (int)GDNX_ETIMEOUT);
    for (int s = 0; s < 2; ++s) {  // let loads in flight land before shared memory is released
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
}

bool vec_view_ok(const gdnx_view& v, int64_t M) {
  const int al = v.dtype == GDNX_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(v.ptr) % al) return false;
  const int64_t st[5] = {v.sb, v.st, v.sh, M > 1 ? v.sm : 0, v.ss};
  for (int i = 0; i < 5; ++i)
    if (st[i] % 4) return false;
  return true;
}

}  // namespace

bool wy_general_eligible(const gdnx_scan_args& a) {
  if (a.algo == GDNX_ALGO_RECURRENT) return false;
  if (a.K != KD || a.V != VD || (a.chunk != 0 && a.chunk != C)) return false;
  if (a.r_out < 1 || (a.r_out > 1 && !a.out_mix)) return false;
  if (!vec_view_ok(a.q, a.M) || !vec_view_ok(a.k, a.M) || !vec_view_ok(a.v, a.M)) return false;
  if (a.gate_e.dim != 1 && !vec_view_ok(a.gate_e, a.M)) return false;
  if (a.gate_w.dim != 1 && !vec_view_ok(a.gate_w, a.M)) return false;
  if (a.decay.dim == KD && (a.decay_kind == GDNX_DECAY_BRAIDED || !vec_view_ok(a.decay, a.M))) return false;
  if (a.rope.enable)
    for (int i = 0; i < 4; ++i)
      if (a.rope.pairs[i] % 4) return false;
  if (a.state_in && (reinterpret_cast<uintptr_t>(a.state_in) & 15)) return false;
  if (a.state_out && (reinterpret_cast<uintptr_t>(a.state_out) & 15)) return false;
  const int64_t N = a.B * a.H * a.M, nch = (a.T + C - 1) / C;
  if (N * nch > int64_t(0x7fffffff) || N > int64_t(0x7fffffff)) return false;
  return true;
}

// Records are bounded: a long call runs as slabs of whole chunks, the state carried
// between slabs in the workspace, so the workspace stays under about 1 GiB per call.
constexpr size_t kMaxRecordBytes = size_t(1) << 30;

int64_t slab_chunks(const gdnx_scan_args& a) {
  const int64_t N = a.B * a.H * a.M, nch = (a.T + C - 1) / C;
  int64_t per = (int64_t)(kMaxRecordBytes / ((size_t)N * REC));
  if (per < 1) per = 1;
  return per < nch ? per : nch;
}

size_t wy_general_workspace_bytes(const gdnx_scan_args& a) {
  const int64_t N = a.B * a.H * a.M, nch = (a.T + C - 1) / C, sc = slab_chunks(a);
  size_t bytes = ERR_BYTES + (size_t)N * sc * REC;
  if (sc < nch) bytes += (size_t)N * VD * KD * sizeof(float);  // state between slabs
  return bytes;
}

namespace {
int esize(int dtype) { return dtype == GDNX_F32 ? 4 : 2; }
void shift_view(gdnx_view& v, int64_t t) {
  if (v.ptr) v.ptr = reinterpret_cast<const char*>(v.ptr) + t * v.st * esize(v.dtype);
}
}  // namespace

gdnx_status launch_wy_general(const gdnx_scan_args& a, cudaStream_t st) {
  GenParams P;
  P.a = a;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.vec_e = a.gate_e.dim != 1;
  P.vec_w = a.gate_w.dim != 1;
  P.chan_decay = a.decay.dim == KD && a.decay_kind != GDNX_DECAY_BRAIDED;
  P.scores = a.scores != nullptr;
  P.T_total = a.T;
  char* ws = reinterpret_cast<char*>(a.workspace);
  P.err = reinterpret_cast<int*>(ws);
  P.rec = ws + ERR_BYTES;
  const int64_t N = a.B * a.H * a.M, nch = (a.T + C - 1) / C, sc = slab_chunks(a);
  float* carry = sc < nch ? reinterpret_cast<float*>(ws + ERR_BYTES + (size_t)N * sc * REC) : nullptr;
  if (cudaMemsetAsync(ws, 0, ERR_BYTES, st) != cudaSuccess) return GDNX_ELAUNCH;
  if (cudaFuncSetAttribute(wyg_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(wyg_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess ||
      cudaFuncSetAttribute(wyg_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S_SMEM) != cudaSuccess)
    return GDNX_ELAUNCH;
  for (int64_t c0 = 0; c0 < nch; c0 += sc) {
    const int64_t t_off = c0 * C, len = (a.T - t_off) < sc * C ? (a.T - t_off) : sc * C;
    GenParams Q = P;
    Q.t_off = t_off;
    Q.nchunks = (len + C - 1) / C;
    gdnx_scan_args& b = Q.a;
    b.T = len;
    shift_view(b.q, t_off);
    shift_view(b.k, t_off);
    shift_view(b.v, t_off);
    shift_view(b.gate_e, t_off);
    shift_view(b.gate_w, t_off);
    shift_view(b.decay, t_off);
    b.y = reinterpret_cast<char*>(a.y) + t_off * a.y_st * esize(a.y_dtype);
    b.rope.pos0 = a.rope.pos0 + t_off;
    b.state_in = c0 == 0 ? a.state_in : carry;
    b.state_out = c0 + sc >= nch ? a.state_out : carry;
    wyg_prep_kernel<<<(unsigned)(N * Q.nchunks), P_NT, P_SMEM, st>>>(Q);
    wyg_chain_kernel<<<(unsigned)N, S_NT, S_SMEM, st>>>(Q);
    if (cudaGetLastError() != cudaSuccess) return GDNX_ELAUNCH;
  }
  return GDNX_OK;
}

}  // namespace gdnx
