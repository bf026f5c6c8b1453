// GDN3 projection prologue: everything between the layer's input GEMMs and the
// scan, in one pass per (batch, token, head) row (gdn3/gdn3_upgrade.py:747-807
// with the coproduct blend of :201-250):
//
//   conv   depthwise causal conv1d over the q|k|v channels of the qkv projection
//          (kernel conv_k, left-padded, no bias; :752-755)
//   blend  q = (1 - s(mix_qk)) q_conv + s(mix_qk) str_qk coprod(q_a, q_b), the same
//          for k, and for v with mix_v / str_v; coprod(a, b)[i*b_dim + j] =
//          sum_c a[c,i] b[c,j] / sqrt(C)   (s = sigmoid; :201-250)
//   gates  b = sigmoid(b_proj + 0.1 proj_a),  w = sigmoid(w_proj + 0.1 proj_b)
//          per lane (:797-807)
//
// The lane expansion and the lane RoPE are not materialised: q/k/v are written
// once per head and the scan kernels read them through stride-0 lane views and
// rotate them in their own prologues; the braided decay is likewise computed
// inside the scan.  HBM-bound: every input is read once (the conv's three
// previous tokens hit in L1/L2) and every output written once.
#include "common.cuh"
#include "kernels.h"

namespace gdnx {
namespace {

constexpr int NT = 128;  // four rows per CTA, a warp per row

GDNX_DEV float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void __launch_bounds__(NT) proj_prologue_kernel(const gdnx_prologue_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (row >= a.B * a.T * a.H) return;
  const int64_t h = row % a.H, t = (row / a.H) % a.T, b = row / (a.H * a.T);
  const int K = (int)a.K, V = (int)a.V;
  const float rsC = a.C > 0 ? rsqrtf((float)a.C) : 0.f;
  const float aqk = a.mix_qk ? sigmoidf_(a.mix_qk[h]) : 0.f;
  const float av = a.mix_v ? sigmoidf_(a.mix_v[h]) : 0.f;
  const float sqk = a.str_qk ? a.str_qk[h] : 1.f;
  const float sv = a.str_v ? a.str_v[h] : 1.f;
  // parts 0, 1, 2 = q, k, v (channel c of part p of head h is qkv channel (3h + p) K + c)
  for (int p = 0; p < 3; ++p) {
    const int D = p < 2 ? K : V;
    const gdnx_view& fa = p == 0 ? a.q_a : (p == 1 ? a.k_a : a.v_a);
    const gdnx_view& fb = p == 0 ? a.q_b : (p == 1 ? a.k_b : a.v_b);
    const int bdim = p < 2 ? a.b_k : a.b_v;
    const float al = p < 2 ? aqk : av, st = p < 2 ? sqk : sv;
    void* out = p == 0 ? a.q_out : (p == 1 ? a.k_out : a.v_out);
    const int64_t oo = b * a.out_sb + t * a.out_st + h * a.out_sh;
    for (int c = lane; c < D; c += 32) {
      const int64_t ch = (3 * h + p) * K + c;  // v uses its first V channels of the K-wide slot
      float x = 0.f;
      for (int i = 0; i < a.conv_k; ++i) {
        const int64_t ts = t - (a.conv_k - 1) + i;
        if (ts >= 0) x = fmaf(a.conv_w[ch * a.conv_k + i], ld_as_f32(a.qkv.ptr, a.qkv.dtype, b * a.qkv.sb + ts * a.qkv.st + ch), x);
      }
      float y = x;
      if (fa.ptr && a.C > 0) {
        const int i = c / bdim, j = c - i * bdim;
        float cp = 0.f;
        for (int cc = 0; cc < a.C; ++cc) {
          const float va = ld_as_f32(fa.ptr, fa.dtype, b * fa.sb + t * fa.st + h * fa.sh + cc * fa.ss + i);
          const float vb = ld_as_f32(fb.ptr, fb.dtype, b * fb.sb + t * fb.st + h * fb.sh + cc * fb.ss + j);
          cp = fmaf(va, vb, cp);
        }
        y = (1.f - al) * x + al * st * (cp * rsC);
      }
      st_from_f32(out, a.out_dtype, oo + c, y);
    }
  }
  // gates, per lane
  const float pa = a.proj_a.ptr ? ld_as_f32(a.proj_a.ptr, a.proj_a.dtype, b * a.proj_a.sb + t * a.proj_a.st + h * a.proj_a.sh) : 0.f;
  const float pb = a.proj_b.ptr ? ld_as_f32(a.proj_b.ptr, a.proj_b.dtype, b * a.proj_b.sb + t * a.proj_b.st + h * a.proj_b.sh) : 0.f;
  for (int m = 0; m < a.M; ++m) {
    if (a.b_proj.ptr) {
      const int64_t io = b * a.b_proj.sb + t * a.b_proj.st + h * a.b_proj.sh + m * a.b_proj.sm;
      const int64_t oo = b * a.gate_sb + t * a.gate_st + h * a.gate_sh + m * a.gate_sm;
      for (int c = lane; c < K; c += 32)
        st_from_f32(a.b_out, a.gate_dtype, oo + c, sigmoidf_(ld_as_f32(a.b_proj.ptr, a.b_proj.dtype, io + c) + 0.1f * pa));
    }
    if (a.w_proj.ptr) {
      const int64_t io = b * a.w_proj.sb + t * a.w_proj.st + h * a.w_proj.sh + m * a.w_proj.sm;
      const int64_t oo = b * a.wgate_sb + t * a.wgate_st + h * a.wgate_sh + m * a.wgate_sm;
      for (int c = lane; c < V; c += 32)
        st_from_f32(a.w_out, a.gate_dtype, oo + c, sigmoidf_(ld_as_f32(a.w_proj.ptr, a.w_proj.dtype, io + c) + 0.1f * pb));
    }
  }
}

}  // namespace

gdnx_status launch_proj_prologue(const gdnx_prologue_args& a, cudaStream_t st) {
  const int64_t rows = a.B * a.T * a.H;
  const int64_t blocks = (rows + NT / 32 - 1) / (NT / 32);
  if (blocks > int64_t(0x7fffffff)) return GDNX_EUNSUPPORTED;
  proj_prologue_kernel<<<(unsigned)blocks, NT, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? GDNX_OK : GDNX_ELAUNCH;
}

}  // namespace gdnx
