// C-ABI entry points: host-side validation and kernel dispatch.
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>

#include "gdnx.h"
#include "kernels.h"

namespace {

bool is_device_ptr(const void* p) {
  if (p == nullptr) return false;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

bool dtype_ok(int dt) { return dt == GDNX_F32 || dt == GDNX_BF16 || dt == GDNX_F16; }

// A required view: device pointer, known dtype, the expected last-dim size.
bool view_ok(const gdnx_view& v, int dim_a, int dim_b = -1) {
  if (!is_device_ptr(v.ptr) || !dtype_ok(v.dtype)) return false;
  if (v.dim != dim_a && v.dim != dim_b) return false;
  if (v.sb < 0 || v.st < 0 || v.sh < 0 || v.sm < 0 || v.ss < 0) return false;
  return true;
}

bool rope_ok(const gdnx_rope& r, int64_t K) {
  if (!r.enable) return true;
  for (int i = 0; i < 4; ++i) {
    if (r.pairs[i] < 0 || 2 * (int64_t)r.pairs[i] > K) return false;
    if (r.pairs[i] > 0 && !(r.den[i] > 0.f)) return false;
  }
  return r.pos0 >= 0;
}

gdnx_status check_common(int64_t B, int64_t H, int64_t M, int64_t K, int64_t V, int mode, int r_out,
                         const gdnx_view& q, const gdnx_view& k, const gdnx_view& v,
                         const gdnx_view& ge, const gdnx_view& gw, const gdnx_view& dec,
                         int decay_kind, const gdnx_rope& rope, const float* out_mix) {
  if (B < 0 || H <= 0 || M <= 0 || K <= 0 || V <= 0) return GDNX_EINVAL;
  if (mode != GDNX_MODE_GDN3 && mode != GDNX_MODE_KMD2) return GDNX_EINVAL;
  if (r_out < 1 || r_out > 16) return GDNX_EINVAL;
  if (mode == GDNX_MODE_GDN3 && r_out != 1) return GDNX_EINVAL;
  if (r_out > 1 && !is_device_ptr(out_mix)) return GDNX_EINVAL;
  if (!view_ok(q, (int)K) || !view_ok(k, (int)K) || !view_ok(v, (int)V)) return GDNX_EINVAL;
  if (mode == GDNX_MODE_GDN3) {
    if (!view_ok(ge, (int)K, 1) || !view_ok(gw, (int)V, 1)) return GDNX_EINVAL;
  } else {
    if (!view_ok(ge, 1) || !view_ok(gw, 1)) return GDNX_EINVAL;
  }
  if (decay_kind == GDNX_DECAY_BRAIDED) {
    if (!view_ok(dec, 4)) return GDNX_EINVAL;
  } else if (decay_kind == GDNX_DECAY_GAMMA || decay_kind == GDNX_DECAY_LOG) {
    if (!view_ok(dec, 1, (int)K)) return GDNX_EINVAL;
  } else {
    return GDNX_EINVAL;
  }
  if (!rope_ok(rope, K)) return GDNX_EINVAL;
  if (rope.enable && M > 4) return GDNX_EINVAL;
  return GDNX_OK;
}

// Which kernel family gdnx_scan_fwd runs for a request.
enum class Path { kRecurrent, kWy, kGeneral };

Path select_path(const gdnx_scan_args& a) {
  if (a.algo == GDNX_ALGO_RECURRENT) return Path::kRecurrent;
  if (gdnx::chunked_eligible(a)) return Path::kWy;
  if (!gdnx::wy_general_eligible(a)) return Path::kRecurrent;
  if (a.algo == GDNX_ALGO_CHUNKED) return Path::kGeneral;
  // automatic choice: GDN3 with fp32 q/k/v keeps the exact fp32 recurrence (its contract is
  // fp32 accuracy); every other form takes the tensor cores
  const bool f32 = a.q.dtype == GDNX_F32 || a.k.dtype == GDNX_F32 || a.v.dtype == GDNX_F32;
  if (a.mode == GDNX_MODE_GDN3 && f32) return Path::kRecurrent;
  return Path::kGeneral;
}

}  // namespace

extern "C" {

const char* gdnx_status_string(gdnx_status s) {
  switch (s) {
    case GDNX_OK: return "GDNX_OK";
    case GDNX_EINVAL: return "GDNX_EINVAL: invalid argument (shape, stride, dtype, alignment or non-device pointer)";
    case GDNX_ELAUNCH: return "GDNX_ELAUNCH: CUDA launch failed";
    case GDNX_ETIMEOUT: return "GDNX_ETIMEOUT: a bounded device-side wait ran out";
    case GDNX_EUNSUPPORTED: return "GDNX_EUNSUPPORTED: no kernel for this configuration in this build";
    case GDNX_EWORKSPACE: return "GDNX_EWORKSPACE: workspace missing or too small";
  }
  return "GDNX_UNKNOWN";
}

const char* gdnx_version(void) { return "gdnx-b200 0.1 sm_100a"; }

size_t gdnx_scan_workspace_bytes(const gdnx_scan_args* a) {
  if (!a) return 0;
  switch (select_path(*a)) {
    case Path::kWy: return gdnx::chunked_workspace_bytes(*a);
    case Path::kGeneral: return gdnx::wy_general_workspace_bytes(*a);
    default: return 0;
  }
}

gdnx_status gdnx_scan_fwd(const gdnx_scan_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->M <= 0 || a->K <= 0 || a->V <= 0) return GDNX_EINVAL;
  if (a->B == 0 || a->T == 0) {
    // nothing to scan (zero-size inputs carry no pointers): the final state
    // equals the initial one
    if (a->state_out && a->state_out != a->state_in && a->B > 0) {
      if (!is_device_ptr(a->state_out) || (a->state_in && !is_device_ptr(a->state_in))) return GDNX_EINVAL;
      const size_t bytes = (size_t)(a->B * a->H * a->M * a->V * a->K) * sizeof(float);
      cudaError_t e = a->state_in
          ? cudaMemcpyAsync(a->state_out, a->state_in, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
          : cudaMemsetAsync(a->state_out, 0, bytes, (cudaStream_t)stream);
      if (e != cudaSuccess) return GDNX_ELAUNCH;
    }
    return GDNX_OK;
  }
  gdnx_status s = check_common(a->B, a->H, a->M, a->K, a->V, a->mode, a->r_out, a->q, a->k, a->v,
                               a->gate_e, a->gate_w, a->decay, a->decay_kind, a->rope, a->out_mix);
  if (s != GDNX_OK) return s;
  if (a->T < 0) return GDNX_EINVAL;
  if (!is_device_ptr(a->y) || !dtype_ok(a->y_dtype)) return GDNX_EINVAL;
  if (a->scores && !is_device_ptr(a->scores)) return GDNX_EINVAL;
  if (a->state_in && !is_device_ptr(a->state_in)) return GDNX_EINVAL;
  if (a->state_out && !is_device_ptr(a->state_out)) return GDNX_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  const Path path = select_path(*a);
  if (a->algo == GDNX_ALGO_CHUNKED && path == Path::kRecurrent) return GDNX_EUNSUPPORTED;
  if (path != Path::kRecurrent) {
    const size_t need = gdnx_scan_workspace_bytes(a);
    if (a->workspace_bytes < need) return GDNX_EWORKSPACE;
    if (need && !is_device_ptr(a->workspace)) return GDNX_EWORKSPACE;
    return path == Path::kWy ? gdnx::launch_chunked_scan(*a, st) : gdnx::launch_wy_general(*a, st);
  }
  return gdnx::launch_recurrent_scan(*a, st);
}

gdnx_status gdnx_scan_fwd_noalloc(const gdnx_scan_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->M <= 0 || a->K <= 0 || a->V <= 0) return GDNX_EINVAL;
  if (a->B == 0 || a->T == 0) return GDNX_EUNSUPPORTED;  // nothing for the kernel to do; use gdnx_scan_fwd
  gdnx_status s = check_common(a->B, a->H, a->M, a->K, a->V, a->mode, a->r_out, a->q, a->k, a->v,
                               a->gate_e, a->gate_w, a->decay, a->decay_kind, a->rope, a->out_mix);
  if (s != GDNX_OK) return s;
  if (!is_device_ptr(a->y) || !dtype_ok(a->y_dtype)) return GDNX_EINVAL;
  if (a->scores) return GDNX_EUNSUPPORTED;
  if (a->state_in && !is_device_ptr(a->state_in)) return GDNX_EINVAL;
  if (a->state_out && !is_device_ptr(a->state_out)) return GDNX_EINVAL;
  if (a->algo == GDNX_ALGO_RECURRENT) return GDNX_EUNSUPPORTED;
  return gdnx::launch_chunked_scan_static_scratch(*a, (cudaStream_t)stream);
}

gdnx_status gdnx_scan_noalloc_status(int32_t* device_error, void* stream) {
  if (!device_error) return GDNX_EINVAL;
  int word = 0;
  const gdnx_status s = gdnx::static_scratch_status(&word, (cudaStream_t)stream);
  if (s == GDNX_OK) *device_error = word;
  return s;
}

gdnx_status gdnx_decode_step(const gdnx_decode_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->B == 0) return GDNX_OK;
  gdnx_status s = check_common(a->B, a->H, a->M, a->K, a->V, a->mode, a->r_out, a->q, a->k, a->v,
                               a->gate_e, a->gate_w, a->decay, a->decay_kind, a->rope, a->out_mix);
  if (s != GDNX_OK) return s;
  if (!is_device_ptr(a->S) || !is_device_ptr(a->y) || !dtype_ok(a->y_dtype)) return GDNX_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  if (a->K == 128 && a->V == 128 && a->r_out == 1 && (reinterpret_cast<uintptr_t>(a->S) & 15) == 0)
    return gdnx::launch_decode_128(*a, st);
  // other head sizes: one step of the exact recurrent kernel, state in place
  gdnx_scan_args sa = {};
  sa.B = a->B; sa.T = 1; sa.H = a->H; sa.M = a->M; sa.K = a->K; sa.V = a->V;
  sa.mode = a->mode; sa.algo = GDNX_ALGO_RECURRENT; sa.r_out = a->r_out; sa.chunk = 64;
  sa.q = a->q; sa.k = a->k; sa.v = a->v; sa.gate_e = a->gate_e; sa.gate_w = a->gate_w;
  sa.decay = a->decay; sa.decay_kind = a->decay_kind;
  for (int i = 0; i < 4; ++i) sa.braid_rates[i] = a->braid_rates[i];
  sa.braid_clamp = a->braid_clamp;
  sa.rope = a->rope;
  sa.out_mix = a->out_mix;
  sa.y = a->y; sa.y_dtype = a->y_dtype;
  sa.y_sb = a->y_sb; sa.y_st = 0; sa.y_sh = a->y_sh; sa.y_sm = a->y_sm;
  sa.state_in = a->S; sa.state_out = a->S;
  return gdnx::launch_recurrent_scan(sa, st);
}

gdnx_status gdnx_compact(const gdnx_compact_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->N < 0 || a->R < 1 || a->P < 1) return GDNX_EINVAL;
  if (a->a_v * a->b_v != a->V || a->a_k * a->b_k != a->K) return GDNX_EINVAL;
  if (a->N == 0) return GDNX_OK;
  if (!is_device_ptr(a->sketch) || !is_device_ptr(a->A) || !is_device_ptr(a->Bk) ||
      !is_device_ptr(a->U) || !is_device_ptr(a->Vb))
    return GDNX_EINVAL;
  if (a->err && !is_device_ptr(a->err)) return GDNX_EINVAL;
  if (a->compact_mode != GDNX_COMPACT_SVD && a->compact_mode != GDNX_COMPACT_SKETCH) return GDNX_EINVAL;
  return gdnx::launch_compact(*a, (cudaStream_t)stream);
}

gdnx_status gdnx_epilogue(const gdnx_epilogue_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->V <= 0 || a->V > 128 || a->V % 8) return GDNX_EINVAL;
  if (a->kind != GDNX_EPILOGUE_LANE_ROUTE && a->kind != GDNX_EPILOGUE_RMS_GATED) return GDNX_EINVAL;
  if (a->B == 0 || a->T == 0) return GDNX_OK;
  auto vec_ok = [](const gdnx_view& v, int64_t dim) {
    if (!is_device_ptr(v.ptr) || !dtype_ok(v.dtype) || v.dim != dim) return false;
    if (reinterpret_cast<uintptr_t>(v.ptr) % 16) return false;
    return v.sb % 8 == 0 && v.st % 8 == 0 && v.sh % 8 == 0 && v.sm % 8 == 0 && v.sb >= 0 && v.st >= 0 &&
           v.sh >= 0 && v.sm >= 0;
  };
  if (!vec_ok(a->y, a->V)) return GDNX_EINVAL;
  if (a->kind == GDNX_EPILOGUE_LANE_ROUTE) {
    if (a->M < 1 || a->M > 8) return GDNX_EINVAL;
    if (!is_device_ptr(a->router.ptr) || !dtype_ok(a->router.dtype) || a->router.dim != 1) return GDNX_EINVAL;
    if (a->gate.ptr && !vec_ok(a->gate, a->V)) return GDNX_EINVAL;  // optional output gate
  } else {
    if (!vec_ok(a->gate, a->V) || !(a->eps >= 0.f)) return GDNX_EINVAL;
  }
  if (a->weight && !is_device_ptr(a->weight)) return GDNX_EINVAL;
  if (!is_device_ptr(a->out) || !dtype_ok(a->out_dtype)) return GDNX_EINVAL;
  const int al = 16;  // 8-element rows are stored as 16-byte (bf16) or 2 x 16-byte (fp32) chunks
  if (reinterpret_cast<uintptr_t>(a->out) % al || a->out_sb % 8 || a->out_st % 8 || a->out_sh % 8) return GDNX_EINVAL;
  return gdnx::launch_epilogue(*a, (cudaStream_t)stream);
}

gdnx_status gdnx_epilogue_scatter(const gdnx_epilogue_args* a, void* const* outs, int32_t n_outs, void* stream) {
  if (!a || !outs || n_outs < 1 || n_outs > gdnx::kMaxPeerOuts) return GDNX_EINVAL;
  if (a->kind != GDNX_EPILOGUE_LANE_ROUTE) return GDNX_EINVAL;
  const int al = 16;  // 8-element rows are stored as 16-byte (bf16) or 2 x 16-byte (fp32) chunks
  for (int d = 0; d < n_outs; ++d)
    if (!is_device_ptr(outs[d]) || reinterpret_cast<uintptr_t>(outs[d]) % al) return GDNX_EINVAL;
  // the single-destination checks, on a copy whose `out` is the first destination
  gdnx_epilogue_args one = *a;
  one.out = outs[0];
  if (one.B == 0 || one.T == 0) return GDNX_OK;
  if (one.B < 0 || one.T < 0 || one.H <= 0 || one.V <= 0 || one.V > 128 || one.V % 8 || one.M < 1 || one.M > 8)
    return GDNX_EINVAL;
  if (!is_device_ptr(one.y.ptr) || !dtype_ok(one.y.dtype) || one.y.dim != one.V ||
      reinterpret_cast<uintptr_t>(one.y.ptr) % 16 || one.y.sb % 8 || one.y.st % 8 || one.y.sh % 8 || one.y.sm % 8 ||
      one.y.sb < 0 || one.y.st < 0 || one.y.sh < 0 || one.y.sm < 0)
    return GDNX_EINVAL;
  if (!is_device_ptr(one.router.ptr) || !dtype_ok(one.router.dtype) || one.router.dim != 1) return GDNX_EINVAL;
  if (one.gate.ptr && (!is_device_ptr(one.gate.ptr) || !dtype_ok(one.gate.dtype) || one.gate.dim != one.V ||
                       reinterpret_cast<uintptr_t>(one.gate.ptr) % 16 || one.gate.sb % 8 || one.gate.st % 8 ||
                       one.gate.sh % 8))
    return GDNX_EINVAL;
  if (one.weight && !is_device_ptr(one.weight)) return GDNX_EINVAL;
  if (!dtype_ok(one.out_dtype) || one.out_sb % 8 || one.out_st % 8 || one.out_sh % 8) return GDNX_EINVAL;
  return gdnx::launch_epilogue_scatter(one, outs, n_outs, (cudaStream_t)stream);
}

gdnx_status gdnx_device_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return GDNX_EINVAL;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    *ptr = nullptr;
    return GDNX_ELAUNCH;
  }
  return GDNX_OK;
}

gdnx_status gdnx_device_free(void* ptr) {
  if (!ptr) return GDNX_OK;
  return cudaFree(ptr) == cudaSuccess ? GDNX_OK : GDNX_EINVAL;
}

gdnx_status gdnx_ipc_handle(const void* base, void* handle) {
  if (!base || !handle) return GDNX_EINVAL;
  static_assert(sizeof(cudaIpcMemHandle_t) == GDNX_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return GDNX_EINVAL;
  }
  memcpy(handle, &h, sizeof(h));
  return GDNX_OK;
}

gdnx_status gdnx_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return GDNX_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    *ptr = nullptr;
    return GDNX_EINVAL;
  }
  return GDNX_OK;
}

gdnx_status gdnx_ipc_close(void* ptr) {
  if (!ptr) return GDNX_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? GDNX_OK : GDNX_EINVAL;
}

gdnx_status gdnx_kmd2_prologue(const gdnx_kmd2_prologue_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->dk != 128 || a->dv != 128 || a->r_out < 1 || a->r_out > 64 ||
      a->conv_k < 1 || a->conv_k > 8)
    return GDNX_EINVAL;
  if (a->B == 0 || a->T == 0) return GDNX_OK;
  const int64_t C = 2 * a->H * a->dk + a->H * a->dv;
  auto view_ok = [](const gdnx_view& v, int64_t dim) {
    return is_device_ptr(v.ptr) && dtype_ok(v.dtype) && v.dim == dim && v.sb >= 0 && v.st >= 0;
  };
  if (!view_ok(a->mixed, C) || !view_ok(a->b, a->H) || !view_ok(a->a, a->H) || !view_ok(a->theta, a->H * a->dk / 2))
    return GDNX_EINVAL;
  if (!is_device_ptr(a->conv_w) || !is_device_ptr(a->dt_bias) || !is_device_ptr(a->A_log) ||
      !is_device_ptr(a->decay_chan) || !is_device_ptr(a->bw_off))
    return GDNX_EINVAL;
  if ((a->r_out > 1) != (a->q_slot_scale != nullptr) || (a->q_slot_scale && !is_device_ptr(a->q_slot_scale)))
    return GDNX_EINVAL;
  if (!is_device_ptr(a->q_out) || !is_device_ptr(a->k_out) || !is_device_ptr(a->v_out) || !is_device_ptr(a->g_out) ||
      !is_device_ptr(a->beta_e_out) || !is_device_ptr(a->beta_w_out) || !is_device_ptr(a->theta_ws))
    return GDNX_EINVAL;
  return gdnx::launch_kmd2_prologue(*a, (cudaStream_t)stream);
}

gdnx_status gdnx_gdn3_prologue(const gdnx_prologue_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->M <= 0 || a->K <= 0 || a->V <= 0 || a->V > a->K) return GDNX_EINVAL;
  if (a->conv_k < 1 || a->C < 0) return GDNX_EINVAL;
  if (a->B == 0 || a->T == 0) return GDNX_OK;
  if (!is_device_ptr(a->qkv.ptr) || !dtype_ok(a->qkv.dtype) || a->qkv.dim != 3 * a->H * a->K) return GDNX_EINVAL;
  if (!is_device_ptr(a->conv_w)) return GDNX_EINVAL;
  const bool coprod = a->q_a.ptr != nullptr;
  if (coprod) {
    if (a->C < 1 || a->a_k * a->b_k != a->K || a->a_v * a->b_v != a->V) return GDNX_EINVAL;
    const gdnx_view* f[6] = {&a->q_a, &a->q_b, &a->k_a, &a->k_b, &a->v_a, &a->v_b};
    const int64_t d[6] = {a->a_k, a->b_k, a->a_k, a->b_k, a->a_v, a->b_v};
    for (int i = 0; i < 6; ++i)
      if (!is_device_ptr(f[i]->ptr) || !dtype_ok(f[i]->dtype) || f[i]->dim != d[i]) return GDNX_EINVAL;
    if (!is_device_ptr(a->mix_qk) || !is_device_ptr(a->mix_v) || !is_device_ptr(a->str_qk) || !is_device_ptr(a->str_v))
      return GDNX_EINVAL;
  }
  if (a->b_proj.ptr && (!view_ok(a->b_proj, (int)a->K) || !view_ok(a->proj_a, 1) || !is_device_ptr(a->b_out)))
    return GDNX_EINVAL;
  if (a->w_proj.ptr && (!view_ok(a->w_proj, (int)a->V) || !view_ok(a->proj_b, 1) || !is_device_ptr(a->w_out)))
    return GDNX_EINVAL;
  if (!is_device_ptr(a->q_out) || !is_device_ptr(a->k_out) || !is_device_ptr(a->v_out) || !dtype_ok(a->out_dtype) ||
      !dtype_ok(a->gate_dtype))
    return GDNX_EINVAL;
  return gdnx::launch_proj_prologue(*a, (cudaStream_t)stream);
}

size_t gdnx_scan_bwd_workspace_bytes(const gdnx_scan_bwd_args* a) {
  if (!a || a->fwd.B <= 0 || a->fwd.T <= 0) return 0;
  return gdnx::scan_bwd_workspace_bytes(*a);
}

gdnx_status gdnx_scan_bwd(const gdnx_scan_bwd_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  const gdnx_scan_args& f = a->fwd;
  if (f.B < 0 || f.T < 0 || f.H <= 0 || f.M <= 0) return GDNX_EINVAL;
  if (f.B == 0 || f.T == 0) return GDNX_EUNSUPPORTED;  // nothing to differentiate through
  gdnx_status s = check_common(f.B, f.H, f.M, f.K, f.V, f.mode, f.r_out, f.q, f.k, f.v, f.gate_e, f.gate_w,
                               f.decay, f.decay_kind, f.rope, f.out_mix);
  if (s != GDNX_OK) return s;
  if (!gdnx::scan_bwd_supported(*a)) return GDNX_EUNSUPPORTED;
  if (!view_ok(a->dy, (int)f.V)) return GDNX_EINVAL;
  if (!is_device_ptr(a->dq) || !is_device_ptr(a->dk) || !is_device_ptr(a->dv) || !is_device_ptr(a->dgate_e) ||
      !is_device_ptr(a->dgate_w) || !is_device_ptr(a->ddecay))
    return GDNX_EINVAL;
  if (f.state_in && !is_device_ptr(f.state_in)) return GDNX_EINVAL;
  if (a->dstate_out && !is_device_ptr(a->dstate_out)) return GDNX_EINVAL;
  if (a->dstate_in && !is_device_ptr(a->dstate_in)) return GDNX_EINVAL;
  if (f.r_out > 1 && a->dout_mix && !is_device_ptr(a->dout_mix)) return GDNX_EINVAL;
  const size_t need = gdnx::scan_bwd_workspace_bytes(*a);
  if (a->workspace_bytes < need || !is_device_ptr(a->workspace)) return GDNX_EWORKSPACE;
  return gdnx::launch_scan_bwd(*a, (cudaStream_t)stream);
}

gdnx_status gdnx_kr_scan_fwd(const gdnx_kr_scan_args* a, void* stream) {
  if (!a) return GDNX_EINVAL;
  const gdnx_scan_args& b = a->base;
  if (b.mode != GDNX_MODE_GDN3) return GDNX_EINVAL;
  if (b.B == 0 || b.T == 0) return GDNX_OK;
  gdnx_status s = check_common(b.B, b.H, b.M, b.K, b.V, b.mode, b.r_out, b.q, b.k, b.v,
                               b.gate_e, b.gate_w, b.decay, b.decay_kind, b.rope, b.out_mix);
  if (s != GDNX_OK) return s;
  if (b.decay.dim != 1 && b.decay_kind != GDNX_DECAY_BRAIDED) return GDNX_EINVAL;  // scalar decay per chain
  if (b.T < 0 || !is_device_ptr(b.y) || !dtype_ok(b.y_dtype)) return GDNX_EINVAL;
  if (a->R < 1 || a->P < 1 || a->a_v * a->b_v != b.V || a->a_k * a->b_k != b.K) return GDNX_EINVAL;
  if (!is_device_ptr(a->sketch) || !is_device_ptr(a->A) || !is_device_ptr(a->Bk) ||
      !is_device_ptr(a->U) || !is_device_ptr(a->Vb) || !is_device_ptr(a->slot))
    return GDNX_EINVAL;
  if (a->comp_err && !is_device_ptr(a->comp_err)) return GDNX_EINVAL;
  if (a->compact_mode != GDNX_COMPACT_SVD && a->compact_mode != GDNX_COMPACT_SKETCH) return GDNX_EINVAL;
  return gdnx::launch_kr_scan(*a, (cudaStream_t)stream);
}

}  // extern "C"
