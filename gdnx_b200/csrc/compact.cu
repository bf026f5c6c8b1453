// Batched compaction entry (gdnx_compact): one CTA per chain.
#include "compact.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int kThreads = kCompThreads;
constexpr int kPT = kCompPT;

struct CompParams {
  gdnx_compact_args a;
  float delta;
};

template <class CD>
__global__ void __launch_bounds__(kThreads) compact_kernel(const CompParams P) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  CD d;
  d.delta = P.delta;
  const gdnx_compact_args& a = P.a;
  const int64_t n = blockIdx.x;
  const int ld = compact_ld(d.n);
  float* Rm = sm;
  float* work = Rm + d.m * ld;
  float* A_s = work + compact_work_floats();
  float* B_s = A_s + d.R * d.m;
  float* tileU = B_s + d.R * d.n;
  float* tileV = tileU + 2 * a.V * kPT;

  float* Ag = a.A + n * d.R * d.m;
  float* Bg = a.Bk + n * d.R * d.n;
  for (int i = threadIdx.x; i < d.R * d.m; i += kThreads) A_s[i] = Ag[i];
  for (int i = threadIdx.x; i < d.R * d.n; i += kThreads) B_s[i] = Bg[i];
  for (int i = threadIdx.x; i < d.m * ld; i += kThreads) Rm[i] = 0.f;
  __syncthreads();
  add_residual_rmat(Rm, a.U + n * a.V * a.P, a.Vb + n * a.K * a.P, nullptr, a.V, a.K, a.P, tileU, tileV, d);
  add_kron_rmat(Rm, A_s, B_s, d);
  __syncthreads();
  const int sk = a.compact_mode == GDNX_COMPACT_SKETCH;
  const float err = compact_core(Rm, A_s, B_s, a.sketch + n * d.n * (sk ? d.R : d.q), work, d, sk);
  for (int i = threadIdx.x; i < d.R * d.m; i += kThreads) Ag[i] = A_s[i];
  for (int i = threadIdx.x; i < d.R * d.n; i += kThreads) Bg[i] = B_s[i];
  if (a.err && threadIdx.x == 0) a.err[n] = err;
}

template <class CD>
gdnx_status launch_compact_t(const gdnx_compact_args& a, cudaStream_t st) {
  CompParams P;
  P.a = a;
  P.delta = a.slow_decay;
  const CD d{};
  if (a.V > 128 || a.K > 128 || a.V * a.K > 64 * kThreads) return GDNX_EUNSUPPORTED;
  const size_t smem = sizeof(float) * (size_t)(d.m * compact_ld(d.n) + compact_work_floats() + d.R * (d.m + d.n) +
                                               2 * (a.V + a.K) * kPT);
  if (cudaFuncSetAttribute(compact_kernel<CD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return GDNX_ELAUNCH;
  compact_kernel<CD><<<(unsigned)a.N, kThreads, smem, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace

gdnx_status launch_compact(const gdnx_compact_args& a, cudaStream_t st) {
  if (a.R == 4 && a.a_v == 16 && a.a_k == 16 && a.b_v == 8 && a.b_k == 8) return launch_compact_t<Dims16x8>(a, st);
  if (a.R == 4 && a.a_v == 8 && a.a_k == 8 && a.b_v == 8 && a.b_k == 8) return launch_compact_t<Dims8x8>(a, st);
  return GDNX_EUNSUPPORTED;
}

}  // namespace gdnx
