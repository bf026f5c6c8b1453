/*
 * gdnx.h -- C ABI of the B200 (sm_100a) GDN3 / KMD-2 recurrent-scan library.
 *
 * Every entry point takes a POD argument struct of device pointers, int64
 * strides (in ELEMENTS) and scalars, enqueues work on the caller's stream and
 * returns a gdnx_status.  The library never allocates or frees device memory
 * on these paths: inputs, outputs, state and any workspace are caller-owned.
 * There is no host synchronisation and no CPU fallback; host pointers are
 * rejected with GDNX_EINVAL.
 *
 * Chains.  A chain is one independent recurrent state.  Chains are numbered
 * n = (b*H + h)*M + m  (batch, head, lane -- lane fastest), exactly as the
 * reference flattens them (gdn3/_reference_recurrence.py:47-50 and
 * gdn3/gdn3_upgrade.py:427-431).  KMD-2 uses M = 1.
 *
 * State layouts (fp32, row-major, caller-owned):
 *   dense  S  [N, V, K]            operator S with y = S q   (row v, key k)
 *   GDN3-KR A [N, R, a_v, a_k], Bk [N, R, b_v, b_k], U [N, V, P], Vb [N, K, P]
 *           -- the reference's own layouts (gdn3/_reference_recurrence.py:52-55).
 *   The KMD-2 reference keeps S as [N, dk, dv] (research/kernel_ab/ref_scan.py:36);
 *   this library's dense state is its transpose.
 */
#ifndef GDNX_H_
#define GDNX_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDNX_API __attribute__((visibility("default")))
#else
#define GDNX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GDNX_OK = 0,
  GDNX_EINVAL = 1,       /* bad shape / stride / dtype / alignment / host pointer */
  GDNX_ELAUNCH = 2,      /* CUDA launch or attribute error                         */
  GDNX_ETIMEOUT = 3,     /* a bounded device-side wait ran out (error word set)   */
  GDNX_EUNSUPPORTED = 4, /* valid request this build has no kernel for            */
  GDNX_EWORKSPACE = 5    /* workspace missing or too small                        */
} gdnx_status;

typedef enum { GDNX_F32 = 0, GDNX_BF16 = 1, GDNX_F16 = 2 } gdnx_dtype;

/* Recurrence family. */
typedef enum {
  /* GDN3: h = b (.) k, u = w (.) v, a = (1 - e^-(k.h)) / (k.h);
   * S <- g S;  r = u - S h;  y = S q + a (k.q) r;  S <- S + a r k^T
   * (gdn3/_reference_recurrence.py:60-84). */
  GDNX_MODE_GDN3 = 0,
  /* KMD-2: S <- diag-decay S; m = S k; d = beta_w v - beta_e m;  S <- S + d k^T;
   * y = sum_slots mix * (q_slot . S)  (research/kernel_ab/ref_scan.py:40-47). */
  GDNX_MODE_KMD2 = 1
} gdnx_mode;

/* How the decay view is interpreted. */
typedef enum {
  GDNX_DECAY_GAMMA = 0,   /* multiplicative factor, clamped to [0,1] as the reference does */
  GDNX_DECAY_LOG = 1,     /* log of the factor (g <= 0); factor = exp(g)                   */
  GDNX_DECAY_BRAIDED = 2  /* 4 logits x per chain-token:
                             factor = min(mean_i exp(-min(softplus(x_i),5)*rate_i), clamp)
                             (gdn3/gdn3_upgrade.py:812-822)                              */
} gdnx_decay_kind;

/* Kernel choice for gdnx_scan_fwd. */
typedef enum {
  GDNX_ALGO_AUTO = 0,      /* chunked tensor-core kernel when eligible, else recurrent */
  GDNX_ALGO_RECURRENT = 1, /* exact token-recurrent CUDA-core kernel (fp32 math)       */
  GDNX_ALGO_CHUNKED = 2    /* chunked WY/UT tcgen05 kernel (bf16 operands, fp32 acc)   */
} gdnx_algo;

/*
 * A strided view of a logical [B, T, H, M, (S,) D] tensor whose last dim is
 * contiguous.  Any of sb/st/sh/sm/ss may be 0 to broadcast (e.g. q/k/v shared
 * by the M lanes of a head).  dim = size of the last dim (K, V, 1 for a
 * scalar gate, 4 for braided logits).  ss is the stride of the query-slot
 * dim (KMD-2 r_out slots), ignored elsewhere.  ptr == NULL means "absent".
 */
typedef struct {
  const void* ptr;
  int32_t dtype; /* gdnx_dtype */
  int32_t dim;
  int64_t sb, st, sh, sm, ss;
} gdnx_view;

/* Lane-specific partial RoPE on q and k (gdn3/gdn3_upgrade.py:342-401).
 * For lane m (m < 4): pairs i < pairs[m] are (x[i], x[i+pairs[m]]); the angle is
 * ((pos0 + t) * scale[m]) * inv_freq_i with inv_freq_i = 1 / 10000^(i / den[m]);
 * x1' = x1 cos - x2 sin;  x2' = x1' sin + x2 cos  (the reference's in-place
 * update, reproduced exactly).  pairs[m] = 0 disables lane m. */
typedef struct {
  int32_t enable;
  int32_t pairs[4];
  float scale[4];
  float den[4];
  int64_t pos0;
} gdnx_rope;

typedef struct {
  int64_t B, T, H, M, K, V;
  int32_t mode;     /* gdnx_mode            */
  int32_t algo;     /* gdnx_algo            */
  int32_t r_out;    /* query slots (KMD-2); 1 otherwise */
  int32_t chunk;    /* chunk length for GDNX_ALGO_CHUNKED (64)  */

  gdnx_view q;      /* [B,T,H,M,(r_out,)K]                                         */
  gdnx_view k;      /* [B,T,H,M,K]                                                 */
  gdnx_view v;      /* [B,T,H,M,V]                                                 */
  gdnx_view gate_e; /* GDN3: erase gate b, dim K or 1.   KMD-2: beta_e, dim 1      */
  gdnx_view gate_w; /* GDN3: write gate w, dim V or 1.   KMD-2: beta_w, dim 1      */
  gdnx_view decay;  /* dim 1 (per chain-token), K (per key channel), or 4 (braided) */
  int32_t decay_kind;         /* gdnx_decay_kind */
  float braid_rates[4];       /* GDNX_DECAY_BRAIDED */
  float braid_clamp;
  gdnx_rope rope;

  const float* out_mix;       /* [H, r_out] fp32 device, KMD-2 r_out > 1 */

  void* y;                    /* output [B,T,H,M,V] with strides below   */
  int32_t y_dtype;
  int64_t y_sb, y_st, y_sh, y_sm;
  float* scores;              /* optional [B,T,H,M] fp32 contiguous: |k| |update| */

  const float* state_in;      /* optional dense S0 [N,V,K]; NULL = zero state      */
  float* state_out;           /* optional final dense S [N,V,K] (may equal state_in) */

  void* workspace;            /* see gdnx_scan_workspace_bytes */
  size_t workspace_bytes;
} gdnx_scan_args;

/* Dense GDN3 / KMD-2 prefill scan.
 * Replaces GDN3LinearAttn._gdn3_recurrent_state (gdn3/gdn3_upgrade.py:403-531)
 * when compaction is off, kmd2_fast_scan.scan / scan_with_update_norm
 * (gdn3/kmd2_fast_scan.py:163-282) and KMD2NativeAttn._scan
 * (gdn3/kmd2_native.py:97-132). */
GDNX_API gdnx_status gdnx_scan_fwd(const gdnx_scan_args* args, void* stream);

/* Workspace the chosen kernel of gdnx_scan_fwd needs (0 if none).  For the
 * chunked tensor-core path it holds a 256-byte error word followed by the
 * per-chunk tiles of the parallel pass (24.25 KB per chain and 64-token chunk).
 * The first int32 of the workspace is cleared on the stream by every call and
 * is GDNX_ETIMEOUT after the call if a kernel gave up waiting (its outputs are
 * then invalid); reading it is optional and costs a synchronisation. */
GDNX_API size_t gdnx_scan_workspace_bytes(const gdnx_scan_args* args);

/* Allocation-free chunked scan.  No counterpart in the reference.
 * For callers that cannot allocate device memory at call time -- for example
 * a host runtime that owns a fixed memory pool, or code running where a
 * cudaMalloc would synchronise the device or fail.  Same arguments and
 * results as gdnx_scan_fwd with algo = GDNX_ALGO_CHUNKED, but `workspace` /
 * `workspace_bytes` are ignored: the kernel's scratch (its device error word)
 * lives in a 256-byte array that the library keeps in every GPU that loads it
 * until the process exits.  The single-pass kernel this entry point runs needs
 * only that word (a compile-time check keeps it within the array).  Requests
 * the chunked kernel cannot take return GDNX_EUNSUPPORTED.  The first call on
 * a device looks the array's device address up (once per device); make that
 * first call before any stream capture.  Every call shares the array and
 * clears it on the stream before the kernel, so calls that overlap on the GPU
 * (other streams, other host threads) race on it.  Nothing is allocated or
 * freed.  gdnx_scan_noalloc_status reads the word back. */
GDNX_API gdnx_status gdnx_scan_fwd_noalloc(const gdnx_scan_args* args, void* stream);

/* Device error word of gdnx_scan_fwd_noalloc's static array after the work on
 * `stream` has finished (the call synchronises `stream`): 0, or GDNX_ETIMEOUT
 * when a kernel gave up a bounded wait and its outputs are invalid.  The next
 * gdnx_scan_fwd_noalloc call clears it.  No counterpart in the reference. */
GDNX_API gdnx_status gdnx_scan_noalloc_status(int32_t* device_error, void* stream);

/* Compaction methods: the rearrangement SVD (randomised range finder, power
 * iterations, QR, SVD of the projection; gdn3/gdn3_upgrade.py:598-629 and
 * :650-719) and the reference's GDN3_COMPACT_MODE "sketch" / "sketch_noqr"
 * (one sketch product, column / row normalisation, no SVD;
 * gdn3/gdn3_upgrade.py:579-596). */
#define GDNX_COMPACT_SVD 0
#define GDNX_COMPACT_SKETCH 1

/* Kronecker-residual (GDN3-KR) scan with periodic compaction. */
typedef struct {
  gdnx_scan_args base;        /* mode must be GDN3; state_in/state_out unused      */
  int32_t R, P, a_v, a_k, b_v, b_k;
  float slow_decay;           /* delta of the two-timescale blend (0.97)            */
  const float* sketch;        /* G [N, b_v*b_k, q], q = min(R+4, a_v*a_k, b_v*b_k);
                                 the reference draws it with torch's CPU generator,
                                 seed 1234 (gdn3/gdn3_upgrade.py:679-682)           */
  /* state, updated in place (zero it for a fresh sequence): */
  float* A;                   /* [N,R,a_v,a_k] */
  float* Bk;                  /* [N,R,b_v,b_k] */
  float* U;                   /* [N,V,P]       */
  float* Vb;                  /* [N,K,P]       */
  int32_t* slot;              /* [N] slot pointer p (int32)                          */
  float* comp_err;            /* optional [N] accumulated discarded energy           */
  int32_t compact_mode;       /* GDNX_COMPACT_SVD (0) or GDNX_COMPACT_SKETCH; with the
                                 sketch mode `sketch` is G [N, b_v*b_k, R]           */
} gdnx_kr_scan_args;

/* Replaces GDN3LinearAttn._gdn3_recurrent_state with compaction
 * (gdn3/gdn3_upgrade.py:403-531; semantics of gdn3/_reference_recurrence.py:33-94,
 * including per-token decay of the Kronecker factors). */
GDNX_API gdnx_status gdnx_kr_scan_fwd(const gdnx_kr_scan_args* args, void* stream);

/* One rearrangement-SVD compaction per chain, in place on A and Bk.
 * Replaces GDN3LinearAttn._compact_vec / _compact_fast (gdn3/gdn3_upgrade.py:565-719).
 * Singular-vector signs are fixed so the largest-|.| entry of each B factor
 * is positive (the reference inherits LAPACK's arbitrary sign). */
typedef struct {
  int64_t N;
  int32_t R, P, V, K, a_v, a_k, b_v, b_k;
  float slow_decay;
  const float* sketch;        /* [N, b_v*b_k, q] */
  float* A;                   /* [N,R,a_v,a_k] in/out */
  float* Bk;                  /* [N,R,b_v,b_k] in/out */
  const float* U;             /* [N,V,P] */
  const float* Vb;            /* [N,K,P] */
  float* err;                 /* optional [N]: discarded energy of this call (written;
                                 0 in the sketch mode, like the reference)           */
  int32_t compact_mode;       /* GDNX_COMPACT_SVD (0) or GDNX_COMPACT_SKETCH; with the
                                 sketch mode `sketch` is G [N, b_v*b_k, R]           */
} gdnx_compact_args;

GDNX_API gdnx_status gdnx_compact(const gdnx_compact_args* args, void* stream);

/* Single-token decode step from a supplied dense state, S updated in place.
 * One iteration of the loop body of gdn3/_reference_recurrence.py:61-84
 * (GDN3, A = 0) or research/kernel_ab/ref_scan.py:40-47 (KMD-2).  Views use
 * T = 1 (st ignored); rope.pos0 is the token's absolute position. */
typedef struct {
  int64_t B, H, M, K, V;
  int32_t mode;
  int32_t r_out;
  gdnx_view q, k, v, gate_e, gate_w, decay;
  int32_t decay_kind;
  float braid_rates[4];
  float braid_clamp;
  gdnx_rope rope;
  const float* out_mix;
  float* S;                   /* [N,V,K] fp32, in place */
  void* y;                    /* [B,H,M,V] */
  int32_t y_dtype;
  int64_t y_sb, y_sh, y_sm;
} gdnx_decode_args;

GDNX_API gdnx_status gdnx_decode_step(const gdnx_decode_args* args, void* stream);

/* Backward of the dense scan (exact fp32 reverse mode, states recomputed from
 * checkpoints).  `fwd` holds the forward call's arguments (q, k, v, gates, decay,
 * r_out, out_mix, state_in); its y, scores, state_out and workspace are ignored.
 * Lane RoPE and braided decays are not supported (GDNX_EUNSUPPORTED); K = V = 128.
 * Gradients are written per chain-token (the lane dim always present, fp32,
 * contiguous); inputs shared across lanes or broadcast take the sum over those dims. */
typedef struct {
  gdnx_scan_args fwd;
  gdnx_view dy;               /* [B,T,H,M,V] gradient of y                              */
  const float* dstate_out;    /* optional [N,V,K] gradient of the final state           */
  float* dq;                  /* [B,T,H,M,r_out,K]                                       */
  float* dk;                  /* [B,T,H,M,K]                                             */
  float* dv;                  /* [B,T,H,M,V]                                             */
  float* dgate_e;             /* [B,T,H,M,gate_e.dim]                                    */
  float* dgate_w;             /* [B,T,H,M,gate_w.dim]                                    */
  float* ddecay;              /* [B,T,H,M,decay.dim]                                     */
  float* dstate_in;           /* optional [N,V,K] gradient of the initial state         */
  float* dout_mix;            /* [H, r_out] when r_out > 1, accumulated (zero it first) */
  void* workspace;            /* see gdnx_scan_bwd_workspace_bytes                       */
  size_t workspace_bytes;
} gdnx_scan_bwd_args;

/* Replaces the backward of kmd2_fast_scan.scan (its _TrsmFn, gdn3/kmd2_fast_scan.py:103-160)
 * and autograd through GDN3LinearAttn._gdn3_recurrent_state without compaction. */
GDNX_API size_t gdnx_scan_bwd_workspace_bytes(const gdnx_scan_bwd_args* args);
GDNX_API gdnx_status gdnx_scan_bwd(const gdnx_scan_bwd_args* args, void* stream);

/* Output epilogues of the recurrent layers (one pass over the scan output). */
typedef enum {
  /* GDN3 lane routing + head norm (gdn3/gdn3_upgrade.py:842-856):
   *   w = softmax_m(router[b,t,h,:]); r = sum_m w_m y[b,t,h,m,:];
   *   out = r / max(|r|, 1e-6) * sqrt(V) * weight  [* silu(gate) when `gate` is
   *   set: the layer's output gate where H V = D (no _agg_proj), :861-871]     */
  GDNX_EPILOGUE_LANE_ROUTE = 0,
  /* KMD-2 gated RMS norm (Qwen3_5RMSNormGated; gdn3/kmd2_native.py:66,176):
   *   out = weight * y * rsqrt(mean(y^2) + eps) * silu(gate)                   */
  GDNX_EPILOGUE_RMS_GATED = 1
} gdnx_epilogue_kind;

typedef struct {
  int64_t B, T, H, M, V;      /* M <= 8 lanes (LANE_ROUTE); V <= 128, a multiple of 8;
                                 y/gate/out strides multiples of 8 elements, their
                                 base addresses 16-byte aligned */
  int32_t kind;               /* gdnx_epilogue_kind */
  float eps;                  /* RMS_GATED */
  gdnx_view y;                /* [B,T,H,M,V] (LANE_ROUTE) or [B,T,H,V] (RMS_GATED)      */
  gdnx_view router;           /* [B,T,H,M] router logits, dim 1 (LANE_ROUTE)           */
  gdnx_view gate;             /* [B,T,H,V] gate z (RMS_GATED; optional in LANE_ROUTE)   */
  const float* weight;        /* [V] fp32 device: the layer's norm weight; NULL = ones  */
  void* out;                  /* [B,T,H,V] */
  int32_t out_dtype;
  int64_t out_sb, out_st, out_sh;
} gdnx_epilogue_args;

/* Replaces the lane routing and per-head norm that follow
 * GDN3LinearAttn._gdn3_recurrent_state (gdn3/gdn3_upgrade.py:842-856) and the
 * Qwen3_5RMSNormGated call after KMD2NativeAttn._scan (gdn3/kmd2_native.py:176). */
GDNX_API gdnx_status gdnx_epilogue(const gdnx_epilogue_args* args, void* stream);

/* The GDN3 lane routing (kind GDNX_EPILOGUE_LANE_ROUTE) fused with the all-gather
 * of its output across the GPUs of a node: every routed row is stored to each of
 * the n_outs (1..8) buffers `outs` -- this GPU's own and its peers', opened with
 * gdnx_ipc_open -- at the offset `args->out_*` strides give it (args->out itself is
 * not used), and each thread fences at system scope after its stores.  The peers
 * may read the rows once this kernel has completed (order that by a collective
 * or another cross-GPU signal issued after it).  Replaces lane routing followed by
 * an all-gather of the routed [B,T,H,V] output; the reference has no multi-GPU path. */
GDNX_API gdnx_status gdnx_epilogue_scatter(const gdnx_epilogue_args* args, void* const* outs, int32_t n_outs,
                                           void* stream);

/* Device buffers that other processes of the node can map (cudaMalloc'd, so their
 * base address is what the IPC handle refers to), and the CUDA IPC handle calls on
 * them: gdnx_ipc_handle writes GDNX_IPC_HANDLE_BYTES bytes; gdnx_ipc_open maps a
 * peer's buffer into this process (peer access enabled on first use);
 * gdnx_ipc_close unmaps it.  Plumbing for gdnx_epilogue_scatter. */
#define GDNX_IPC_HANDLE_BYTES 64
GDNX_API gdnx_status gdnx_device_alloc(size_t bytes, void** ptr);
GDNX_API gdnx_status gdnx_device_free(void* ptr);
GDNX_API gdnx_status gdnx_ipc_handle(const void* base, void* handle);
GDNX_API gdnx_status gdnx_ipc_open(const void* handle, void** ptr);
GDNX_API gdnx_status gdnx_ipc_close(void* ptr);

/* GDN3 projection prologue: the per-element work between the layer's input GEMMs
 * and the scan.  Views as elsewhere ([B,T,H,(M|C,)D], last dim contiguous);
 * `qkv` is the [B,T,3*H*K] qkv projection (sb, st used; channel (3h + p) K + c
 * holds part p = q, k, v of head h).  A NULL coproduct factor skips the blend
 * (dense features only); NULL b_proj / w_proj skips that gate. */
typedef struct {
  int64_t B, T, H, M, K, V;
  int32_t C;                   /* coproduct rank (4 in the reference)            */
  int32_t a_k, b_k, a_v, b_v;  /* a_k * b_k = K, a_v * b_v = V                   */
  int32_t conv_k;              /* causal conv kernel size                        */
  gdnx_view qkv;
  const float* conv_w;         /* [3*H*K, conv_k] fp32 (depthwise Conv1d weight) */
  gdnx_view q_a, q_b, k_a, k_b, v_a, v_b; /* [B,T,H,C,dim]; ss = stride of C      */
  const float* mix_qk;         /* [H] raw blend logits (sigmoid applied here)    */
  const float* mix_v;
  const float* str_qk;         /* [H] strengths                                  */
  const float* str_v;
  gdnx_view b_proj, w_proj;    /* [B,T,H,M,K] / [B,T,H,M,V] gate pre-activations */
  gdnx_view proj_a, proj_b;    /* [B,T,H] (dim 1)                                */
  void* q_out;                 /* [B,T,H,K] (q, k), [B,T,H,V] (v), strides below */
  void* k_out;
  void* v_out;
  int32_t out_dtype;
  int64_t out_sb, out_st, out_sh;
  void* b_out;                 /* [B,T,H,M,K] erase gates */
  void* w_out;                 /* [B,T,H,M,V] write gates */
  int32_t gate_dtype;
  int64_t gate_sb, gate_st, gate_sh, gate_sm;
  int64_t wgate_sb, wgate_st, wgate_sh, wgate_sm;
} gdnx_prologue_args;

/* Replaces the causal conv, coproduct blend and gate activations of
 * GDN3LinearAttn.forward (gdn3/gdn3_upgrade.py:752-807, blend :201-250). */
GDNX_API gdnx_status gdnx_gdn3_prologue(const gdnx_prologue_args* args, void* stream);

/* KMD-2 prologue: everything between KMD2NativeAttn.forward's input GEMMs and its
 * scan (gdn3/kmd2_native.py:140-172), from the GEMM outputs to the scan inputs:
 *   depthwise causal conv (conv_k taps) + SiLU over the q|k|v channels of `mixed`;
 *   q = normalize(q, eps 1e-6) / sqrt(dk), k = normalize(k, eps 1e-6), v as is;
 *   beta_e = sigmoid(b), beta_w = sigmoid(b + bw_off[h]);
 *   g[i] = min(exp(-exp(A_log[h]) softplus(a + dt_bias[h]) + decay_chan[h][i]), 1);
 *   Theta = cumsum over t of softplus(theta) (per pair i < dk/2), and k and every
 *   query slot q (1 + q_slot_scale[h][r]) rotated pairwise: (x_i, x_{i+dk/2}) ->
 *   (x_i cos - x_{i+dk/2} sin, x_i sin + x_{i+dk/2} cos).
 * Inputs are the GEMM outputs as views ([B,T,C]: sb, st used, channels contiguous);
 * outputs fp32 contiguous.  dk = dv = 128, K-heads = V-heads = H. */
typedef struct {
  int64_t B, T, H, dk, dv;
  int32_t r_out, conv_k;
  gdnx_view mixed;             /* [B,T,2*H*dk + H*dv] in_proj_qkv output (dim = channel count) */
  const float* conv_w;         /* [2*H*dk + H*dv, conv_k] fp32 (depthwise Conv1d weight) */
  gdnx_view b, a;              /* [B,T,H] in_proj_b / in_proj_a outputs (dim = H)          */
  gdnx_view theta;             /* [B,T,H*dk/2] rot_proj output, bias included (dim = H*dk/2) */
  const float* dt_bias;        /* [H] */
  const float* A_log;          /* [H] */
  const float* decay_chan;     /* [H, dk] */
  const float* bw_off;         /* [H] */
  const float* q_slot_scale;   /* [H, r_out, dk], NULL when r_out == 1 */
  float* q_out;                /* [B,T,H,r_out,dk] */
  float* k_out;                /* [B,T,H,dk] */
  float* v_out;                /* [B,T,H,dv] */
  float* g_out;                /* [B,T,H,dk] */
  float* beta_e_out;           /* [B,T,H] */
  float* beta_w_out;           /* [B,T,H] */
  float* theta_ws;             /* [B,T,H,dk/2] workspace: the cumulative angles */
} gdnx_kmd2_prologue_args;

GDNX_API gdnx_status gdnx_kmd2_prologue(const gdnx_kmd2_prologue_args* args, void* stream);

GDNX_API const char* gdnx_status_string(gdnx_status s);

/* Library build identification (for load checks). */
GDNX_API const char* gdnx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDNX_H_ */
