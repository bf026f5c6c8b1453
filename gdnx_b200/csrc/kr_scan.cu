// GDN3 Kronecker-residual scan with periodic compaction (gdnx_kr_scan_fwd).
//
// Semantics: the frozen token loop gdn3/_reference_recurrence.py:60-90, per
// chain and token
//     A *= g; Bk *= g; Vb *= g                       (Kronecker part decays g^2)
//     h = b(.)k ; u = w(.)v ; r = u - S h ; a = alpha(k.h)
//     y = S q + a (k.q) r ;  U[:,p] = a r ; Vb[:,p] = k ; p += 1
//     p == P  ->  compaction (A, Bk blended, U/Vb kept) ; p = 0
// with S x = vec(sum_r A_r X B_r^T) + U (Vb^T x).
//
// Design (one CTA of 256 threads per chain):
//  * the residual operator U Vb^T (V x K) is kept DENSE in registers, row v
//    split over TPR threads; each token applies the rank-2 update
//    "decay, evict the overwritten slot, add the new write".  Compactions read
//    it from the registers; it is rebuilt exactly from the slots at call start
//    and every kExactEvery-th compaction, so rounding cannot drift over a long
//    sequence;
//  * the slot ring lives in the caller's U / Vb buffers (global, L2
//    resident).  New writes store the raw key and a per-slot decay factor
//    d_p (smem) carries Vb = d_p k_p, exactly the product of per-token
//    decays the reference applies;
//  * A, Bk live in shared memory with one pending scalar decay fac
//    (true A = fac A_s), folded in before each compaction;
//  * the Kronecker operator sum_r A_r (x) B_r is materialised densely in
//    registers next to the residual whenever A, Bk change, so its read shares
//    the residual's loads (its per-token decay is the scalar fac^2);
//  * compaction runs in-kernel on shared memory (compact.cuh);
//  * bf16 q/k/v rows of the next block of tokens are fetched with cp.async into
//    a staging area while the current block's sequential updates run.
#include "compact.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int kNT = kCompThreads;  // 256
constexpr int kTB = 32;            // tokens staged per block (<= P handled by the block split)
constexpr int kMaxP = 1024;
constexpr int kExactEvery = 16;  // compactions between exact rebuilds of the residual

struct KrParams {
  gdnx_kr_scan_args a;
  float delta;
  int vec_e, vec_w;
};

template <int K, int V>
struct KrSmem {
  static constexpr int kTokK = 0, kTokH = K, kTokQ = 2 * K, kTokKold = 3 * K;
  static constexpr int kTokU = 4 * K, kTokUold = 4 * K + V, kTokSc = 4 * K + 2 * V;
  static constexpr int kTokPer = 4 * K + 2 * V + 8;
};

// Floats of the region shared by the compaction (Rm, work) and the token vectors.
template <class CD, int K, int V>
__host__ __device__ constexpr int kr_union_floats() {
  return (CD::a_v * CD::a_k) * compact_ld(CD::b_v * CD::b_k) + compact_work_floats() > kTB * KrSmem<K, V>::kTokPer
             ? (CD::a_v * CD::a_k) * compact_ld(CD::b_v * CD::b_k) + compact_work_floats()
             : kTB * KrSmem<K, V>::kTokPer;
}

// Cluster barrier (release / acquire at cluster scope: orders the CTAs' global-memory
// slot writes and reads).
GDNX_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
GDNX_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// CL = 1: one CTA per chain.  CL = 2: a cluster of two CTAs per chain, CTA r owning state
// rows r V/2 .. (r+1) V/2 - 1 (the rows evolve independently given the token's vectors);
// both CTAs form the token vectors and run each compaction on the whole state (the same
// inputs give the same factors), and cluster barriers order the slot ring's global
// reads and writes between them.
template <class CD, int CL>
__global__ void __launch_bounds__(kNT, 1) kr_scan_kernel(const KrParams P) {
  constexpr int K = CD::a_k * CD::b_k, V = CD::a_v * CD::b_v;
  constexpr int VL = V / CL;       // state rows of this CTA
  constexpr int TPR = kNT / VL;    // threads per state row
  constexpr int KC = K / 4 / TPR;  // float4 key chunks per thread
  using SMT = KrSmem<K, V>;
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const gdnx_kr_scan_args& A = P.a;
  const gdnx_scan_args& a = A.base;
  CD d;
  d.delta = P.delta;
  const int R = d.R, Pn = A.P;
  const int ld = compact_ld(d.n);

  // ---- shared memory carve-up ----
  // The compaction's Rm and work space and a block's token vectors share one region: the token
  // vectors are dead while a compaction (or a rebuild) runs, and vice versa.
  float* Rm = sm;                                  // m x ld (compaction / rebuild)
  float* work = Rm + d.m * ld;                     // compaction work
  float* tok = sm;                                 // kTB x kTokPer (token phases)
  float* A_s = sm + kr_union_floats<CD, K, V>();   // R x m
  float* B_s = A_s + R * d.m;                      // R x n
  float* dsl = B_s + R * d.n;                      // per-slot decay [P]
  float* ybuf = dsl + kMaxP;                       // kTB x V
  float* nbuf = ybuf + kTB * V;                    // kTB x V (new U columns)
  float* tileU = nbuf + kTB * V;                   // 2 x V x kCompPT
  float* tileV = tileU + 2 * V * kCompPT;          // 2 x K x kCompPT
  float* misc = tileV + 2 * K * kCompPT;           // 32 floats
  float* ropeC = misc + 32;                        // kTB x 64 (cos of this block's angles)
  float* ropeS = ropeC + kTB * 64;                 // kTB x 64
  float* sInv = ropeS + kTB * 64;                  // 64 inverse frequencies
  // kTB tokens x (k, q, v) raw bf16 rows of the next block (16-byte aligned)
  __nv_bfloat16* rawst =
      reinterpret_cast<__nv_bfloat16*>((reinterpret_cast<uintptr_t>(sInv + 64) + 15) & ~uintptr_t(15));

  const int cr = CL == 1 ? 0 : (int)cluster_rank();
  const int64_t n = blockIdx.x / CL;
  const int64_t m = n % a.M, h = (n / a.M) % a.H, b = n / (a.M * a.H);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int v = cr * VL + tid / TPR, j = tid % TPR;
  const int av = v / d.b_v, bv = v % d.b_v;

  float* Ug = A.U + n * (int64_t)V * Pn;
  float* Vg = A.Vb + n * (int64_t)K * Pn;
  float* Ag = A.A + n * (int64_t)R * d.m;
  float* Bg = A.Bk + n * (int64_t)R * d.n;
  const int sketch_mode = A.compact_mode == GDNX_COMPACT_SKETCH;
  const float* Gg = A.sketch + n * (int64_t)d.n * (sketch_mode ? d.R : d.q);

  for (int i = tid; i < R * d.m; i += kNT) A_s[i] = Ag[i];
  for (int i = tid; i < R * d.n; i += kNT) B_s[i] = Bg[i];
  for (int i = tid; i < Pn; i += kNT) dsl[i] = 1.f;
  int p = A.slot[n];
  const int dpairs = (a.rope.enable && m < 4) ? a.rope.pairs[m] : 0;
  if (tid < 64 && dpairs > 0) sInv[tid] = 1.0f / powf(10000.0f, (float)tid / a.rope.den[m]);
  float fac = 1.f, err_acc = 0.f;

  float4 Rs[KC];
  // rebuild the dense residual from the slots (exact) into registers
  auto rebuild = [&]() {
    for (int i = tid; i < d.m * ld; i += kNT) Rm[i] = 0.f;
    __syncthreads();
    add_residual_rmat(Rm, Ug, Vg, dsl, V, K, Pn, tileU, tileV, d);
#pragma unroll
    for (int c = 0; c < KC; ++c) {
      const int k0 = 4 * (c * TPR + j);
      Rs[c].x = Rm[rmat_index(v, k0 + 0, d)];
      Rs[c].y = Rm[rmat_index(v, k0 + 1, d)];
      Rs[c].z = Rm[rmat_index(v, k0 + 2, d)];
      Rs[c].w = Rm[rmat_index(v, k0 + 3, d)];
    }
    __syncthreads();
  };
  // Rm = rearrange(residual) from the registers (both CTAs' rows: the other CTA's half arrives
  // through distributed shared memory).  The register residual carries the per-token rounding
  // of its updates, so every kExactEvery-th compaction rebuilds it exactly from the slots instead.
  auto rm_from_regs = [&]() {
    uint32_t rbase = 0;
    if (CL > 1) {
      const uint32_t lbase = static_cast<uint32_t>(__cvta_generic_to_shared(Rm));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbase) : "r"(lbase), "r"(1u - (uint32_t)cr));
    }
#pragma unroll
    for (int c = 0; c < KC; ++c) {
      const int k0 = 4 * (c * TPR + j);
      const float x4[4] = {Rs[c].x, Rs[c].y, Rs[c].z, Rs[c].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = rmat_index(v, k0 + e, d);
        Rm[ri] = x4[e];
        if (CL > 1)
          asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(rbase + 4u * (uint32_t)ri), "f"(x4[e]) : "memory");
      }
    }
    if (CL > 1) cluster_sync_all();
    __syncthreads();
  };
  int comp_count = 0;
  // dense Kronecker operator sum_r A_r (x) B_r (row v, this thread's keys), materialised
  // whenever A_s / B_s change (start, compaction); its decay is the scalar fac^2
  float4 Ks[KC];
  auto build_kron = [&]() {
#pragma unroll
    for (int c = 0; c < KC; ++c) {
      float kv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kk = 4 * (c * TPR + j) + e;
        const int ak = kk / CD::b_k, bk = kk % CD::b_k;
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < CD::R; ++r) acc = fmaf(A_s[r * d.m + av * d.a_k + ak], B_s[r * d.n + bv * d.b_k + bk], acc);
        kv[e] = acc;
      }
      Ks[c] = make_float4(kv[0], kv[1], kv[2], kv[3]);
    }
  };
  rebuild();
  build_kron();

  // asynchronous staging of bf16 q/k/v rows (16-byte aligned views only)
  const bool raw_ok = a.k.dtype == GDNX_BF16 && a.q.dtype == GDNX_BF16 && a.v.dtype == GDNX_BF16 &&
                      ((reinterpret_cast<uintptr_t>(a.k.ptr) | reinterpret_cast<uintptr_t>(a.q.ptr) |
                        reinterpret_cast<uintptr_t>(a.v.ptr)) & 15) == 0 &&
                      ((a.k.sb | a.k.st | a.k.sh | a.k.sm | a.q.sb | a.q.st | a.q.sh | a.q.sm | a.v.sb | a.v.st |
                        a.v.sh | a.v.sm) & 7) == 0;
  constexpr int kRowK = K / 8, kRowV = V / 8;  // 16-byte chunks per row
  constexpr int kRawPer = 2 * K + V;           // bf16 elements per staged token
  // the scalar gates and decay of the next block are loaded into registers with its rows: lane
  // 3 i + c of warp w holds component c (erase gate, write gate, raw decay) of token w + 8 i, and
  // stage A (warp w takes tokens w, w + 8, ...) shuffles them out
  static_assert(kTB <= 8 * 10, "three scalars of every token of a warp fit in its lanes");
  const bool sc_ok = raw_ok && a.decay_kind != GDNX_DECAY_BRAIDED;
  float pf_sc = 0.f;
  auto prefetch_raw = [&](int64_t ts) {
    const int nb = kTB < Pn ? kTB : Pn;  // a block never holds more than P tokens
    if (sc_ok && lane < 3 * ((nb + 7) / 8)) {
      const int tt = warp + 8 * (lane / 3), c = lane % 3;
      const int64_t t = ts + tt;
      if (tt < nb && t < a.T && (c != 0 || !P.vec_e) && (c != 1 || !P.vec_w))
        pf_sc = c == 0   ? ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, view_off(a.gate_e, b, t, h, m))
                : c == 1 ? ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, view_off(a.gate_w, b, t, h, m))
                         : ld_as_f32(a.decay.ptr, a.decay.dtype, view_off(a.decay, b, t, h, m));
    }
    for (int idx = tid; idx < nb * (2 * kRowK + kRowV); idx += kNT) {
      const int tt = idx / (2 * kRowK + kRowV), c = idx - tt * (2 * kRowK + kRowV);
      const int64_t t = ts + tt;
      if (t >= a.T) continue;
      const __nv_bfloat16* src;
      if (c < kRowK) src = reinterpret_cast<const __nv_bfloat16*>(a.k.ptr) + view_off(a.k, b, t, h, m) + 8 * c;
      else if (c < 2 * kRowK)
        src = reinterpret_cast<const __nv_bfloat16*>(a.q.ptr) + view_off(a.q, b, t, h, m) + 8 * (c - kRowK);
      else src = reinterpret_cast<const __nv_bfloat16*>(a.v.ptr) + view_off(a.v, b, t, h, m) + 8 * (c - 2 * kRowK);
      const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(rawst + tt * kRawPer + 8 * c));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (raw_ok) prefetch_raw(0);

  int64_t t0 = 0;
  while (t0 < a.T) {
    int64_t nt64 = a.T - t0;
    if (nt64 > kTB) nt64 = kTB;
    if (nt64 > Pn - p) nt64 = Pn - p;
    const int nt = (int)nt64;
    // ---------- stage A: RoPE angles of the block, then per-token vectors (one warp per token) ----------
    if (raw_ok) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
    }
    if (dpairs > 0) {
      for (int idx = tid; idx < nt * dpairs; idx += kNT) {
        const int tt = idx / dpairs, i = idx - tt * dpairs;
        sincosf(((float)(a.rope.pos0 + t0 + tt) * a.rope.scale[m]) * sInv[i], &ropeS[tt * 64 + i], &ropeC[tt * 64 + i]);
      }
      __syncthreads();
    }
    for (int tt = warp; tt < nt; tt += kNT / 32) {
      const int64_t t = t0 + tt;
      float* tk = tok + tt * SMT::kTokPer;
      float* sk = tk + SMT::kTokK;
      float* sh = tk + SMT::kTokH;
      float* sq = tk + SMT::kTokQ;
      const int64_t ko = view_off(a.k, b, t, h, m), qo = view_off(a.q, b, t, h, m), vo = view_off(a.v, b, t, h, m);
      const int64_t eo = view_off(a.gate_e, b, t, h, m), wo = view_off(a.gate_w, b, t, h, m);
      const __nv_bfloat16* raw = rawst + tt * kRawPer;
      // every global load of the token first (one memory round trip), uses after
      constexpr int KW = (K + 31) / 32, VW = (V + 31) / 32;
      float rk[KW], rq[KW], re[KW], rv[VW], rw[VW];
#pragma unroll
      for (int c = 0; c < KW; ++c) {
        const int i = lane + 32 * c;
        rk[c] = rq[c] = re[c] = 0.f;
        if (i < K) {
          rk[c] = raw_ok ? __bfloat162float(raw[i]) : ld_as_f32(a.k.ptr, a.k.dtype, ko + i);
          rq[c] = raw_ok ? __bfloat162float(raw[K + i]) : ld_as_f32(a.q.ptr, a.q.dtype, qo + i);
          if (P.vec_e) re[c] = ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo + i);
        }
      }
#pragma unroll
      for (int c = 0; c < VW; ++c) {
        const int i = lane + 32 * c;
        rv[c] = rw[c] = 0.f;
        if (i < V) {
          rv[c] = raw_ok ? __bfloat162float(raw[2 * K + i]) : ld_as_f32(a.v.ptr, a.v.dtype, vo + i);
          if (P.vec_w) rw[c] = ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo + i);
        }
      }
      float be, bw, gdec;
      if (sc_ok) {
        const int li = 3 * (tt / 8);
        const float se = __shfl_sync(0xffffffffu, pf_sc, li), sw = __shfl_sync(0xffffffffu, pf_sc, li + 1);
        const float x = __shfl_sync(0xffffffffu, pf_sc, li + 2);
        be = P.vec_e ? 1.f : se;
        bw = P.vec_w ? 1.f : sw;
        gdec = fminf(fmaxf(a.decay_kind == GDNX_DECAY_LOG ? expf(x) : x, 0.f), 1.f);
      } else {
        be = P.vec_e ? 1.f : ld_as_f32(a.gate_e.ptr, a.gate_e.dtype, eo);
        bw = P.vec_w ? 1.f : ld_as_f32(a.gate_w.ptr, a.gate_w.dtype, wo);
        gdec = decay_factor(a.decay, a.decay_kind, view_off(a.decay, b, t, h, m), true, a.braid_rates, a.braid_clamp);
      }
#pragma unroll
      for (int c = 0; c < KW; ++c) {
        const int i = lane + 32 * c;
        if (i < K) {
          sk[i] = rk[c];
          sq[i] = rq[c];
        }
      }
      __syncwarp();
      if (dpairs > 0) {
        rope_row_table(sk, dpairs, ropeC + tt * 64, ropeS + tt * 64, lane);
        rope_row_table(sq, dpairs, ropeC + tt * 64, ropeS + tt * 64, lane);
      }
      __syncwarp();
      float kh = 0.f, kq = 0.f;
#pragma unroll
      for (int c = 0; c < KW; ++c) {
        const int i = lane + 32 * c;
        if (i < K) {
          const float hv = (P.vec_e ? re[c] : be) * sk[i];
          sh[i] = hv;
          kh += sk[i] * hv;
          kq += sk[i] * sq[i];
        }
      }
      kh = warp_sum(kh);
      kq = warp_sum(kq);
#pragma unroll
      for (int c = 0; c < VW; ++c) {
        const int i = lane + 32 * c;
        if (i < V) tk[SMT::kTokU + i] = (P.vec_w ? rw[c] : bw) * rv[c];
      }
      if (lane == 0) {
        float* sc = tk + SMT::kTokSc;
        sc[0] = gdec;
        sc[1] = stable_alpha(kh);
        sc[2] = kq;
      }
    }
    // the slots this block overwrites (p .. p+nt-1): rows of U and Vb, nt contiguous floats each
    for (int idx = tid; idx < K * nt; idx += kNT) {
      const int kk = idx / nt, tt = idx - kk * nt;
      tok[tt * SMT::kTokPer + SMT::kTokKold + kk] = Vg[(int64_t)kk * Pn + p + tt];
    }
    for (int idx = tid; idx < VL * nt; idx += kNT) {  // this CTA's rows
      const int vv = cr * VL + idx / nt, tt = idx % nt;
      tok[tt * SMT::kTokPer + SMT::kTokUold + vv] = Ug[(int64_t)vv * Pn + p + tt];
    }
    __syncthreads();
    if (CL > 1) cluster_sync_all();  // both CTAs have read the evicted slots before either flushes
    if (raw_ok && t0 + nt < a.T) prefetch_raw(t0 + nt);  // the staging has been read
    // ---------- stage B: running decays (thread 0) ----------
    if (tid == 0) {
      float f = fac, pre = 1.f;
      for (int tt = 0; tt < nt; ++tt) {
        float* sc = tok + tt * SMT::kTokPer + SMT::kTokSc;
        f *= sc[0];
        pre *= sc[0];
        sc[3] = f * f;                  // Kronecker scale
        sc[4] = dsl[p + tt] * pre;      // decay of the evicted slot through t
      }
      misc[0] = f;
      misc[1] = pre;
    }
    __syncthreads();
    // ---------- sequential token updates ----------
    for (int tt = 0; tt < nt; ++tt) {
      const float* tk = tok + tt * SMT::kTokPer;
      const float* sc = tk + SMT::kTokSc;
      const float gam = sc[0], al = sc[1], kq = sc[2], ks = sc[3], ev = sc[4];
      float krh = 0.f, krq = 0.f, dh = 0.f, dq = 0.f;
#pragma unroll
      for (int c = 0; c < KC; ++c) {
        const int k0 = 4 * (c * TPR + j);
        const float4 h4 = *reinterpret_cast<const float4*>(tk + SMT::kTokH + k0);
        const float4 q4 = *reinterpret_cast<const float4*>(tk + SMT::kTokQ + k0);
        dh = fmaf(Rs[c].x, h4.x, dh); dh = fmaf(Rs[c].y, h4.y, dh);
        dh = fmaf(Rs[c].z, h4.z, dh); dh = fmaf(Rs[c].w, h4.w, dh);
        dq = fmaf(Rs[c].x, q4.x, dq); dq = fmaf(Rs[c].y, q4.y, dq);
        dq = fmaf(Rs[c].z, q4.z, dq); dq = fmaf(Rs[c].w, q4.w, dq);
        krh = fmaf(Ks[c].x, h4.x, krh); krh = fmaf(Ks[c].y, h4.y, krh);
        krh = fmaf(Ks[c].z, h4.z, krh); krh = fmaf(Ks[c].w, h4.w, krh);
        krq = fmaf(Ks[c].x, q4.x, krq); krq = fmaf(Ks[c].y, q4.y, krq);
        krq = fmaf(Ks[c].z, q4.z, krq); krq = fmaf(Ks[c].w, q4.w, krq);
      }
#pragma unroll
      for (int o = 1; o < TPR; o <<= 1) {
        krh += __shfl_xor_sync(0xffffffffu, krh, o);
        krq += __shfl_xor_sync(0xffffffffu, krq, o);
        dh += __shfl_xor_sync(0xffffffffu, dh, o);
        dq += __shfl_xor_sync(0xffffffffu, dq, o);
      }
      const float s_h = ks * krh + gam * dh;
      const float r = tk[SMT::kTokU + v] - s_h;
      const float wnew = al * r;
      const float y = ks * krq + gam * dq + al * kq * r;
      const float cold = tk[SMT::kTokUold + v] * ev;
#pragma unroll
      for (int c = 0; c < KC; ++c) {
        const int k0 = 4 * (c * TPR + j);
        const float4 ko4 = *reinterpret_cast<const float4*>(tk + SMT::kTokKold + k0);
        const float4 k4 = *reinterpret_cast<const float4*>(tk + SMT::kTokK + k0);
        Rs[c].x = fmaf(gam, Rs[c].x, fmaf(wnew, k4.x, -cold * ko4.x));
        Rs[c].y = fmaf(gam, Rs[c].y, fmaf(wnew, k4.y, -cold * ko4.y));
        Rs[c].z = fmaf(gam, Rs[c].z, fmaf(wnew, k4.z, -cold * ko4.z));
        Rs[c].w = fmaf(gam, Rs[c].w, fmaf(wnew, k4.w, -cold * ko4.w));
      }
      if (j == 0) {
        ybuf[tt * V + v] = y;
        nbuf[tt * V + v] = wnew;
      }
    }
    __syncthreads();
    // ---------- flush: outputs, new slots, slot decays ----------
    for (int idx = tid; idx < nt * VL; idx += kNT) {
      const int tt = idx / VL, vv = cr * VL + idx % VL;
      st_from_f32(a.y, a.y_dtype, b * a.y_sb + (t0 + tt) * a.y_st + h * a.y_sh + m * a.y_sm + vv, ybuf[tt * V + vv]);
    }
    for (int idx = tid; idx < VL * nt; idx += kNT) {
      const int vv = cr * VL + idx / nt, tt = idx % nt;
      Ug[(int64_t)vv * Pn + p + tt] = nbuf[tt * V + vv];
    }
    if (cr == 0)
      for (int idx = tid; idx < K * nt; idx += kNT) {
        const int kk = idx / nt, tt = idx % nt;
        Vg[(int64_t)kk * Pn + p + tt] = tok[tt * SMT::kTokPer + SMT::kTokK + kk];
      }
    {
      const float pre = misc[1];
      for (int s = tid; s < Pn; s += kNT) {
        if (s >= p && s < p + nt) {
          float f = 1.f;  // decays after the write, through the block end
          for (int u = s - p + 1; u < nt; ++u) f *= tok[u * SMT::kTokPer + SMT::kTokSc];
          dsl[s] = f;
        } else {
          dsl[s] *= pre;
        }
      }
    }
    fac = misc[0];
    p += nt;
    t0 += nt;
    __syncthreads();
    if (p == Pn) {
      // ---------- compaction at the window end ----------
      for (int i = tid; i < R * d.m; i += kNT) A_s[i] *= fac;
      for (int i = tid; i < R * d.n; i += kNT) B_s[i] *= fac;
      fac = 1.f;
      if (CL > 1) cluster_sync_all();  // the other CTA's slot writes are visible
      if (++comp_count % kExactEvery == 0) rebuild();  // Rm = rearrange(U Vb^T), Rs exact again
      else rm_from_regs();
      add_kron_rmat(Rm, A_s, B_s, d);
      __syncthreads();
      err_acc += compact_core(Rm, A_s, B_s, Gg, work, d, sketch_mode);
      p = 0;
      __syncthreads();
      build_kron();
    }
  }
  // ---------- materialise the state ----------
  if (CL > 1) {
    cluster_sync_all();  // the other CTA is done reading the slots
    if (cr != 0) return;
  }
  for (int i = tid; i < R * d.m; i += kNT) Ag[i] = A_s[i] * fac;
  for (int i = tid; i < R * d.n; i += kNT) Bg[i] = B_s[i] * fac;
  for (int idx = tid; idx < K * Pn; idx += kNT) Vg[idx] *= dsl[idx % Pn];
  if (tid == 0) {
    A.slot[n] = p;
    if (A.comp_err) A.comp_err[n] += err_acc;
  }
}

template <class CD>
gdnx_status launch_kr(const KrParams& P, cudaStream_t st) {
  constexpr int K = CD::a_k * CD::b_k, V = CD::a_v * CD::b_v;
  const CD d{};
  const size_t floats = (size_t)kr_union_floats<CD, K, V>() + d.R * (d.m + d.n) + kMaxP + 2 * kTB * V +
                        2 * (V + K) * kCompPT + 32 + 2 * kTB * 64 + 64;
  const size_t smem = floats * sizeof(float) + (size_t)kTB * (2 * K + V) * 2 + 16;  // + bf16 staging
  const int64_t N = P.a.base.B * P.a.base.H * P.a.base.M;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return GDNX_ELAUNCH;
  if (2 * N <= sms) {  // idle SMs: two CTAs (a cluster) per chain
    auto fn = kr_scan_kernel<CD, 2>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return GDNX_ELAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * N));
    cfg.blockDim = dim3(kNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, fn, P) != cudaSuccess) return GDNX_ELAUNCH;
    return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
  }
  auto fn = kr_scan_kernel<CD, 1>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return GDNX_ELAUNCH;
  fn<<<(unsigned)N, kNT, smem, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace

gdnx_status launch_kr_scan(const gdnx_kr_scan_args& a, cudaStream_t st) {
  KrParams P;
  P.a = a;
  P.vec_e = a.base.gate_e.dim > 1;
  P.vec_w = a.base.gate_w.dim > 1;
  P.delta = a.slow_decay;
  if (a.P > kMaxP) return GDNX_EUNSUPPORTED;
  const int64_t K = a.base.K, V = a.base.V;
  const bool r4 = a.R == 4;
  if (r4 && K == 128 && V == 128 && a.a_v == 16 && a.a_k == 16 && a.b_v == 8 && a.b_k == 8)
    return launch_kr<Dims16x8>(P, st);
  if (r4 && K == 64 && V == 64 && a.a_v == 8 && a.a_k == 8 && a.b_v == 8 && a.b_k == 8)
    return launch_kr<Dims8x8>(P, st);
  return GDNX_EUNSUPPORTED;
}

}  // namespace gdnx
