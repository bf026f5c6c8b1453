// Memory-bound single-token decode step for K = V = 128 dense states.
//
// Persistent CTAs (one per SM, 8 update warps + 1 copy warp) stream their
// chains' 64 KB fp32 states through three shared-memory stages with bulk
// asynchronous copies (cp.async.bulk, completion counted on an mbarrier): the
// state of chain j+2 is in flight while chain j is updated in place in shared
// memory, and chain j's updated state drains back to HBM with a bulk store.
// The copy warp issues every load and store and waits for a stage's store to
// have read it before refilling it; the update warps signal "stage updated" on
// a second mbarrier and never wait for a store themselves.  The per-chain
// vectors (q, k, v, gates, decay) of chain j+1 are loaded as raw bits into
// registers before chain j's math and converted after it, so no dependent
// global-memory latency sits on the per-chain path.  The lane-RoPE cos/sin
// depend only on (lane, pair) within one launch (every chain is at the same
// position) and are tabulated once per CTA.  Each state byte is read once
// and written once.
//
// Math per chain (warp w owns rows 16w..16w+15, lane l the float4 at key 4l):
// the 16 rows x 2 dot products (S h and S q) are reduced with a transpose
// reduction (31 shuffles for all 32 sums, lane l holds sum l), then
//   d_v = cw u_v - ce g (S h)_v ;  y_v = g (S q)_v + d_v (k.q) ;  S_v <- g S_v + d_v k
// (GDN3: ce = a b, cw = a w with a = alpha(k.h); KMD-2: beta_e, beta_w and a
// per-channel decay applied to S first) -- the loop body of
// gdn3/_reference_recurrence.py:61-84 (Kronecker part zero) and
// research/kernel_ab/ref_scan.py:40-47.  Query slots (r_out > 1) take the
// exact recurrent kernel instead (gdnx_api.cu).
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace gdnx {
namespace {

constexpr int K = 128, V = 128;
constexpr int kRowsPerWarp = 16;
constexpr int kWarps = 8;
constexpr int kStages = 3;
constexpr int kStateBytes = K * V * 4;
constexpr int kPiece = 16384;  // bytes per bulk copy
constexpr uint32_t kWaitLimit = 1u << 24;

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

GDNX_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(mbar) : "memory");
}
GDNX_DEV void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" :: "l"(dst), "r"(src), "r"(bytes)
               : "memory");
}
GDNX_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
GDNX_DEV void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
GDNX_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
GDNX_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}
GDNX_DEV void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(mbar), "r"(bytes) : "memory");
}

// Raw bits of one element (converted later, so the load does not stall here).
GDNX_DEV uint32_t ld_raw(const void* base, int dtype, int64_t off) {
  if (dtype == GDNX_F32) return reinterpret_cast<const uint32_t*>(base)[off];
  return reinterpret_cast<const uint16_t*>(base)[off];
}
GDNX_DEV float raw_f32(uint32_t r, int dtype) {
  if (dtype == GDNX_F32) return __uint_as_float(r);
  if (dtype == GDNX_BF16) return __uint_as_float(r << 16);
  return __half2float(__ushort_as_half((unsigned short)r));
}

struct DecParams {
  gdnx_decode_args a;
  int vec_e, vec_w, chan_decay, kmd2;
  int64_t N;
};

// Raw per-lane inputs of one chain.
struct ChainRaw {
  uint32_t k[4], q[4], e[4], d[4], v, w;
};

// Per-lane values of one chain ready for the state update.
struct ChainVals {
  float4 k4, q4, h4, g4;
  float kq, ce, cw, gam, u;
};

GDNX_DEV void chain_index(const gdnx_decode_args& a, int64_t n, int64_t& b, int64_t& h, int64_t& m) {
  m = n % a.M;
  h = (n / a.M) % a.H;
  b = n / (a.M * a.H);
}

GDNX_DEV void load_raw(const DecParams& P, int64_t n, int warp, int lane, ChainRaw& r) {
  const gdnx_decode_args& a = P.a;
  int64_t b, h, m;
  chain_index(a, n, b, h, m);
  const int k0 = 4 * lane;
  const int64_t ko = view_off(a.k, b, 0, h, m) + k0, qo = view_off(a.q, b, 0, h, m) + k0;
  const int64_t eo = view_off(a.gate_e, b, 0, h, m), wo = view_off(a.gate_w, b, 0, h, m);
  const int64_t dof = view_off(a.decay, b, 0, h, m);
  const int row = warp * kRowsPerWarp + (lane & 15);
  const bool dvec = P.chan_decay || a.decay_kind == GDNX_DECAY_BRAIDED;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r.k[i] = ld_raw(a.k.ptr, a.k.dtype, ko + i);
    r.q[i] = ld_raw(a.q.ptr, a.q.dtype, qo + i);
    r.e[i] = (P.vec_e || i == 0) ? ld_raw(a.gate_e.ptr, a.gate_e.dtype, eo + (P.vec_e ? k0 + i : 0)) : 0u;
    r.d[i] = (dvec || i == 0) ? ld_raw(a.decay.ptr, a.decay.dtype, dof + (P.chan_decay ? k0 + i : i)) : 0u;
  }
  r.v = ld_raw(a.v.ptr, a.v.dtype, view_off(a.v, b, 0, h, m) + row);
  r.w = ld_raw(a.gate_w.ptr, a.gate_w.dtype, wo + (P.vec_w ? row : 0));
}

GDNX_DEV void finish_chain(const DecParams& P, int64_t n, int lane, const ChainRaw& r, float* sk, float* sq,
                           const float* ropeC, const float* ropeS, ChainVals& c) {
  const gdnx_decode_args& a = P.a;
  int64_t b, h, m;
  chain_index(a, n, b, h, m);
  const int k0 = 4 * lane;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sk[k0 + i] = raw_f32(r.k[i], a.k.dtype);
    sq[k0 + i] = raw_f32(r.q[i], a.q.dtype);
  }
  __syncwarp();
  if (a.rope.enable && m < 4 && a.rope.pairs[m] > 0) {
    rope_row_table(sk, a.rope.pairs[m], ropeC + 64 * m, ropeS + 64 * m, lane);
    rope_row_table(sq, a.rope.pairs[m], ropeC + 64 * m, ropeS + 64 * m, lane);
  }
  __syncwarp();
  c.k4 = *reinterpret_cast<const float4*>(sk + k0);
  c.q4 = *reinterpret_cast<const float4*>(sq + k0);
  __syncwarp();  // sk/sq are rewritten for the next chain
  c.h4 = c.k4;
  if (P.vec_e) {
    c.h4.x *= raw_f32(r.e[0], a.gate_e.dtype);
    c.h4.y *= raw_f32(r.e[1], a.gate_e.dtype);
    c.h4.z *= raw_f32(r.e[2], a.gate_e.dtype);
    c.h4.w *= raw_f32(r.e[3], a.gate_e.dtype);
  }
  const float4 k4 = c.k4, q4 = c.q4, h4 = c.h4;
  const float kh = warp_sum(k4.x * h4.x + k4.y * h4.y + k4.z * h4.z + k4.w * h4.w);
  c.kq = warp_sum(k4.x * q4.x + k4.y * q4.y + k4.z * q4.z + k4.w * q4.w);
  const float ge = raw_f32(r.e[0], a.gate_e.dtype), gw = raw_f32(r.w, a.gate_w.dtype);
  if (P.kmd2) {
    c.ce = ge;
    c.cw = gw;
  } else {
    const float be = P.vec_e ? 1.f : ge;
    const float bw = P.vec_w ? 1.f : gw;
    const float al = stable_alpha(P.vec_e ? kh : be * kh);
    c.ce = al * be;
    c.cw = al * bw;
  }
  c.u = raw_f32(r.v, a.v.dtype) * (P.vec_w ? gw : 1.f);
  c.gam = 1.f;
  c.g4 = make_float4(1.f, 1.f, 1.f, 1.f);
  if (P.chan_decay) {
    float gg[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float g = raw_f32(r.d[e], a.decay.dtype);
      if (a.decay_kind == GDNX_DECAY_LOG) g = expf(g);
      if (!P.kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
      gg[e] = g;
    }
    c.g4 = make_float4(gg[0], gg[1], gg[2], gg[3]);
  } else if (a.decay_kind == GDNX_DECAY_BRAIDED) {
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      acc += expf(-fminf(softplus_f(raw_f32(r.d[e], a.decay.dtype)), 5.0f) * a.braid_rates[e]);
    c.gam = fminf(acc * 0.25f, a.braid_clamp);
  } else {
    float g = raw_f32(r.d[0], a.decay.dtype);
    if (a.decay_kind == GDNX_DECAY_LOG) g = expf(g);
    if (!P.kmd2) g = fminf(fmaxf(g, 0.f), 1.f);
    c.gam = g;
  }
}

constexpr int kThreads = (kWarps + 1) * 32;  // eight update warps and one copy warp

__global__ void __launch_bounds__(kThreads, 1) decode128_kernel(const DecParams P) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = tc::align_smem(smraw, 128);
  float* stage_f = reinterpret_cast<float*>(sm);                       // kStages x 128 x 128
  float* vecs = reinterpret_cast<float*>(sm + kStages * kStateBytes);  // kWarps x 2 x 128
  float* ropeC = vecs + kWarps * 2 * K;                                // [4 lanes][64 pairs]
  float* ropeS = ropeC + 4 * 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(ropeS + 4 * 64);  // [kStages] state loaded
  uint64_t* done = full + kStages;                                 // [kStages] state updated in place
  volatile int* s_abort = reinterpret_cast<volatile int*>(done + kStages);

  const gdnx_decode_args& a = P.a;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t nmine = P.N > blockIdx.x ? (P.N - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  auto chain_of = [&](int64_t j) { return (int64_t)blockIdx.x + j * (int64_t)gridDim.x; };
  float* sk = vecs + warp * 2 * K;
  float* sq = sk + K;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&done[s], kWarps);
    }
    *s_abort = 0;
  }
  if (a.rope.enable) {
    for (int idx = threadIdx.x; idx < 4 * 64; idx += blockDim.x) {
      const int lm = idx >> 6, i = idx & 63;
      if (lm < a.M && i < a.rope.pairs[lm]) {
        const float inv_freq = 1.0f / powf(10000.0f, (float)i / a.rope.den[lm]);
        sincosf(((float)a.rope.pos0 * a.rope.scale[lm]) * inv_freq, &ropeS[idx], &ropeC[idx]);
      }
    }
  }
  __syncthreads();
  auto issue_load = [&](int64_t j) {
    const int s = (int)(j % kStages);
    const uint32_t mb = tc::smem_u32(&full[s]);
    const char* src = reinterpret_cast<const char*>(a.S + chain_of(j) * (int64_t)V * K);
    mbar_expect_tx(mb, kStateBytes);
    const uint32_t dst = tc::smem_u32(stage_f + (size_t)s * V * K);
#pragma unroll
    for (int p = 0; p < kStateBytes / kPiece; ++p) bulk_load(dst + p * kPiece, src + p * kPiece, kPiece, mb);
  };
  if (warp == kWarps) {
    // ---- copy warp: loads two states ahead, stores each updated state, refills its stage ----
    if (lane == 0) {
      for (int64_t j = 0; j < nmine && j < kStages - 1; ++j) issue_load(j);
      int64_t j = 0;
      for (; j < nmine; ++j) {
        const int s = (int)(j % kStages);
        if (!tc::mbar_wait(&done[s], (uint32_t)((j / kStages) & 1), kWaitLimit) || *s_abort) {
          *s_abort = 1;
          break;
        }
        bulk_store(a.S + chain_of(j) * (int64_t)V * K, tc::smem_u32(stage_f + (size_t)s * V * K), kStateBytes);
        bulk_commit();
        // the stage of chain j-1 is free once its store has read shared memory
        if (j + kStages - 1 < nmine) {
          bulk_wait_read_le1();
          issue_load(j + kStages - 1);
        }
      }
      bulk_wait_all();
      if (j < nmine) {
        // gave up: drain the loads still in flight (bounded) before exiting
        const int64_t issued = nmine < j + kStages - 1 ? nmine : j + kStages - 1;
        for (int64_t jj = j; jj < issued; ++jj)
          tc::mbar_wait(&full[jj % kStages], (uint32_t)((jj / kStages) & 1), kWaitLimit);
      }
    }
  } else {
    // ---- update warps: each owns 16 rows of every state ----
    ChainRaw raw;
    ChainVals cur;
    if (nmine > 0) {
      load_raw(P, chain_of(0), warp, lane, raw);
      finish_chain(P, chain_of(0), lane, raw, sk, sq, ropeC, ropeS, cur);
    }
    const int row0 = warp * kRowsPerWarp;
    for (int64_t j = 0; j < nmine; ++j) {
      const int64_t n = chain_of(j);
      int64_t b, h, m;
      chain_index(a, n, b, h, m);
      const int s = (int)(j % kStages);
      if (!tc::mbar_wait(&full[s], (uint32_t)((j / kStages) & 1), kWaitLimit)) *s_abort = 1;
      if (*s_abort) break;
      // next chain's vectors: raw loads now, consumed after this chain's math
      if (j + 1 < nmine) load_raw(P, chain_of(j + 1), warp, lane, raw);

      float* Sst = stage_f + (size_t)s * V * K + row0 * K + 4 * lane;
      float4 S[kRowsPerWarp];
      float vals[32];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        float4 x = *reinterpret_cast<const float4*>(Sst + r * K);
        if (P.chan_decay) {
          x.x *= cur.g4.x; x.y *= cur.g4.y; x.z *= cur.g4.z; x.w *= cur.g4.w;
        }
        S[r] = x;
        vals[r] = x.x * cur.h4.x + x.y * cur.h4.y + x.z * cur.h4.z + x.w * cur.h4.w;
        vals[r + 16] = x.x * cur.q4.x + x.y * cur.q4.y + x.z * cur.q4.z + x.w * cur.q4.w;
      }
      const float tot = transpose_reduce32(vals, lane);
      // lane l < 16: tot = (S h)_row(l); lane l >= 16: tot = (S q)_row(l-16)
      const float d_own = cur.cw * cur.u - cur.ce * (cur.gam * tot);
      const float d_row = __shfl_sync(0xffffffffu, d_own, lane & 15);
      if (lane >= 16) {
        const float y = fmaf(d_row, cur.kq, cur.gam * tot);
        st_from_f32(a.y, a.y_dtype, b * a.y_sb + h * a.y_sh + m * a.y_sm + row0 + (lane - 16), y);
      }
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const float d = __shfl_sync(0xffffffffu, d_own, r);
        float4 x = S[r];
        x.x = fmaf(cur.gam, x.x, d * cur.k4.x);
        x.y = fmaf(cur.gam, x.y, d * cur.k4.y);
        x.z = fmaf(cur.gam, x.z, d * cur.k4.z);
        x.w = fmaf(cur.gam, x.w, d * cur.k4.w);
        *reinterpret_cast<float4*>(Sst + r * K) = x;
      }
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[s]);  // this warp's rows are written back (the copy warp stores them)
      if (j + 1 < nmine) finish_chain(P, chain_of(j + 1), lane, raw, sk, sq, ropeC, ropeS, cur);
    }
  }
  __syncthreads();
}

}  // namespace

gdnx_status launch_decode_128(const gdnx_decode_args& a, cudaStream_t st) {
  DecParams P;
  P.a = a;
  P.kmd2 = a.mode == GDNX_MODE_KMD2;
  P.vec_e = !P.kmd2 && a.gate_e.dim > 1;
  P.vec_w = !P.kmd2 && a.gate_w.dim > 1;
  P.chan_decay = a.decay.dim == a.K && a.decay_kind != GDNX_DECAY_BRAIDED;
  P.N = a.B * a.H * a.M;
  if (P.N == 0) return GDNX_OK;
  if (a.r_out != 1 || (reinterpret_cast<uintptr_t>(a.S) & 15) != 0) return GDNX_EUNSUPPORTED;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return GDNX_ELAUNCH;
  const size_t smem = (size_t)kStages * kStateBytes + kWarps * 2 * K * 4 + 2 * 4 * 64 * 4 + 2 * kStages * 8 + 16 + 128;
  if (cudaFuncSetAttribute(decode128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return GDNX_ELAUNCH;
  const int64_t grid = P.N < sms ? P.N : sms;
  decode128_kernel<<<(unsigned)grid, kThreads, smem, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
