// Internal launcher declarations (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include "gdnx.h"

namespace gdnx {

gdnx_status launch_recurrent_scan(const gdnx_scan_args& a, cudaStream_t st);
gdnx_status launch_decode_128(const gdnx_decode_args& a, cudaStream_t st);
gdnx_status launch_compact(const gdnx_compact_args& a, cudaStream_t st);
gdnx_status launch_kr_scan(const gdnx_kr_scan_args& a, cudaStream_t st);
gdnx_status launch_epilogue(const gdnx_epilogue_args& a, cudaStream_t st);
constexpr int kMaxPeerOuts = 8;  // destinations of the scattering lane routing
gdnx_status launch_epilogue_scatter(const gdnx_epilogue_args& a, void* const* outs, int n, cudaStream_t st);
gdnx_status launch_proj_prologue(const gdnx_prologue_args& a, cudaStream_t st);
gdnx_status launch_kmd2_prologue(const gdnx_kmd2_prologue_args& a, cudaStream_t st);
// Backward of the dense scan (scan_backward.cu).
bool scan_bwd_supported(const gdnx_scan_bwd_args& a);
size_t scan_bwd_workspace_bytes(const gdnx_scan_bwd_args& a);
gdnx_status launch_scan_bwd(const gdnx_scan_bwd_args& a, cudaStream_t st);

// Chunked tensor-core scan (dense GDN3 / KMD-2 with per-chain scalar decay).
bool chunked_eligible(const gdnx_scan_args& a);
size_t chunked_workspace_bytes(const gdnx_scan_args& a);
gdnx_status launch_chunked_scan(const gdnx_scan_args& a, cudaStream_t st);
// Two-pass WY scan (scan_wy.cu): workspace = error word + per-chunk T tiles and
// decay prefixes.  Returns GDNX_EUNSUPPORTED when q/k/v cannot be described by
// TMA tensor maps (the single-pass kernel then runs instead).
size_t wy_workspace_bytes(const gdnx_scan_args& a);
gdnx_status launch_wy_scan(const gdnx_scan_args& a, cudaStream_t st);
// General two-pass WY scan (scan_wy_general.cu): vector gates, per-channel decay,
// query slots, scores, fp32/bf16/fp16 inputs.  Workspace = error word + one
// record per chain and 64-token chunk.
bool wy_general_eligible(const gdnx_scan_args& a);
size_t wy_general_workspace_bytes(const gdnx_scan_args& a);
gdnx_status launch_wy_general(const gdnx_scan_args& a, cudaStream_t st);
// Single-pass kernel with its scratch in a library-owned static device array (no allocation).
gdnx_status launch_chunked_scan_static_scratch(const gdnx_scan_args& a, cudaStream_t st);
// Error word of that static array, read after the stream's work (synchronises the stream).
gdnx_status static_scratch_status(int* out, cudaStream_t st);

}  // namespace gdnx
