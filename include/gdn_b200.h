/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) gated-DeltaNet token-mixing library.
 *
 * The library implements the gated delta rule used by archbench's `gdn` and `nsgdn`
 * mixers.  Per (batch b, head h), with a DV x DK fp32 state S:
 *
 *     S_t = alpha_t * S_{t-1}                       (alpha_t = exp(la_t))
 *     r_t = v_t - S_t k_t
 *     S_t = S_t + r_t u_t^T                         (u_t = beta_t k_t unless u is given)
 *     y_t = S_t q_t
 *
 * which is the per-token loop of archbench/layers/nsgdn.py:408-417 (nsgdn_ref) with the
 * write vector u of nsgdn.py:61-75 (write_direction).  q is used as given: the caller
 * pre-scales it by DK^-1/2 exactly as archbench/layers/nsgdn.py:527 does.
 *
 * Conventions
 *   - Tensors are dense with a unit-stride last dimension.  Token tensors (q, k, u, v, y)
 *     are indexed [b][t][h][d] through explicit element strides (stride_b, stride_t,
 *     stride_h); gate tensors (la, beta) are contiguous (B, T, H) fp32.
 *   - The state is (B, H, DV, DK) fp32 row-major: row i of S (a DV index) holds DK
 *     contiguous values, the layout of nsgdn_ref's S (nsgdn.py:410).
 *   - Every pointer is a device pointer; `stream` is a cudaStream_t (NULL = legacy stream).
 *   - All calls are asynchronous on `stream`, allocate nothing, keep no state between
 *     calls and are re-entrant.  Errors are returned as negative gdn_status codes before
 *     anything is launched; no C++ exception crosses this boundary.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_B200_ABI_VERSION 2

typedef enum {
  GDN_OK = 0,
  GDN_ERR_NULL = -1,         /* a required pointer is NULL */
  GDN_ERR_SHAPE = -2,        /* a size is out of range or inconsistent */
  GDN_ERR_DTYPE = -3,        /* unsupported dtype combination */
  GDN_ERR_ALIGN = -4,        /* pointer or stride not aligned as the kernel needs */
  GDN_ERR_UNSUPPORTED = -5,  /* valid request that no kernel of this build implements */
  GDN_ERR_DEVICE = -6,       /* current device is not an sm_100 GPU */
  GDN_ERR_LAUNCH = -7,       /* the CUDA launch itself failed */
  GDN_ERR_TIMEOUT = -8,      /* a bounded device-side wait gave up (kernel reported it) */
  GDN_ERR_WORKSPACE = -9     /* the problem needs more scratch than GDN_STATIC_WORKSPACE_BYTES */
} gdn_status;

typedef enum { GDN_DTYPE_F32 = 0, GDN_DTYPE_BF16 = 1 } gdn_dtype;

typedef enum {
  GDN_IMPL_AUTO = 0,       /* the fastest kernel that applies (see gdn_prefill_select_impl) */
  GDN_IMPL_CHUNK = 1,      /* chunkwise tcgen05/TMEM kernel (bf16 I/O, DK = 128, DV a multiple of 128) */
  GDN_IMPL_RECURRENT = 2,  /* token-serial fp32 kernel (any supported dtype and head size) */
  GDN_IMPL_SEGMENTED = 3,  /* chunk kernel split into sequence segments for few long sequences;
                              needs the workspace gdn_prefill_workspace_bytes reports */
  GDN_IMPL_CHUNK_CLUSTER = 4, /* chunk kernel on a two-CTA cluster per sequence (DV = 128, u = NULL) */
  GDN_IMPL_CHUNK_SINGLE = 5,  /* chunk kernel on one CTA per sequence and 128-row state tile */
  GDN_IMPL_CHUNK_SPLIT = 6    /* every chunk's state-independent products in one parallel pass, then
                                 one state-only CTA per sequence and 128-row state tile reading them
                                 (any DV multiple of 128, u given or not); needs the workspace
                                 gdn_prefill_workspace_bytes reports (24 KB per (b, h, chunk)) */
} gdn_impl;

/* Strides of one token tensor, in elements.  The last (feature) dimension has stride 1. */
typedef struct {
  int64_t b, t, h;
} gdn_strides;

/*
 * Prefill: the whole (B, T) block in one call.
 *
 * Replaces the scan ops archbench dispatches to from NStepGDN.forward
 * (archbench/layers/nsgdn.py:537-538): nsgdn_scan_chunk (nsgdn.py:400-405, which runs the
 * custom op archbench::nsgdn_chunk_fwd, nsgdn.py:352-363), nsgdn_scan (nsgdn.py:219-221)
 * and nsgdn_ref (nsgdn.py:408-417); and fla's chunk_gated_delta_rule as called by the
 * `gdn` mixer (fla/layers/gated_deltanet.py:266-279, via archbench/layers/fla.py:36-38).
 * Unlike those it also takes an initial state and returns the final state.
 */
typedef struct {
  const void* q;      /* [B][T][H][DK], dtype `in_dtype` */
  const void* k;      /* [B][T][H][DK], read vector */
  const void* u;      /* [B][T][H][DK] write vector, or NULL: u_t = beta_t * k_t */
  const void* v;      /* [B][T][H][DV] */
  const float* beta;  /* (B, T, H) fp32; required when u == NULL, ignored otherwise */
  const float* la;    /* (B, T, H) fp32 natural-log retention, la <= 0 */
  const float* s0;    /* (B, H, DV, DK) fp32 initial state, or NULL for S_0 = 0 */
  void* y;            /* [B][T][H][DV], dtype `out_dtype` */
  float* s_out;       /* (B, H, DV, DK) fp32 final state, or NULL; may equal s0 */
  gdn_strides sq, sk, su, sv, sy;
  int64_t B, T, H, DK, DV;
  int32_t in_dtype;   /* gdn_dtype of q, k, u, v */
  int32_t out_dtype;  /* gdn_dtype of y */
  int32_t impl;       /* gdn_impl */
  int32_t reserved;
  void* workspace;    /* device scratch for GDN_IMPL_SEGMENTED / GDN_IMPL_CHUNK_SPLIT (16-byte
                         aligned), or NULL */
  uint64_t workspace_bytes;
} gdn_prefill_args;

int gdn_prefill_fwd(const gdn_prefill_args* args, void* stream);

/*
 * Decode: one new token per sequence, state updated in place.
 *
 * Replaces fla's fused_recurrent_gated_delta_rule as the `gdn` layer calls it for
 * q_len <= 64 at inference (fla/layers/gated_deltanet.py:219,281-294), with the state in
 * the nsgdn (B, H, DV, DK) layout instead of fla's [N, H, K, V].  archbench itself has no
 * single-step path (archbench/model.py:122, archbench/core_eval.py:136-142 re-run the
 * prefix); this is the step its recurrence (nsgdn.py:413-416) takes for one token.
 */
typedef struct {
  const void* q;      /* [B][H][DK] (token tensors with T = 1; stride_t unused) */
  const void* k;      /* [B][H][DK] */
  const void* u;      /* [B][H][DK] or NULL: u = beta * k */
  const void* v;      /* [B][H][DV] */
  const float* beta;  /* (B, H) fp32 when u == NULL */
  const float* la;    /* (B, H) fp32 */
  float* state;       /* (B, H, DV, DK) fp32, read and written in place */
  void* y;            /* [B][H][DV], dtype `out_dtype` */
  gdn_strides sq, sk, su, sv, sy;
  int64_t B, H, DK, DV;
  int32_t in_dtype;
  int32_t out_dtype;
} gdn_decode_args;

int gdn_decode_step(const gdn_decode_args* args, void* stream);

/*
 * Bytes of device workspace the call needs for these arguments (0 when none).  The segmented path
 * is chosen for few (b, h) sequences with long T: phase A writes a (DV + 128) x 128 fp32 pair of
 * segment states per (b, h, segment), phase B combines them, phase C reads them back; where the
 * split chunk kernels serve it, every chunk's products (24 KB per (b, h, chunk)) follow the segment
 * states.  The split path (GDN_IMPL_CHUNK_SPLIT; under GDN_IMPL_AUTO for DV > 128 or explicit write
 * vectors) needs the products alone.  Under GDN_IMPL_AUTO a call without enough workspace runs a
 * single-pass chunk kernel instead; GDN_IMPL_SEGMENTED or GDN_IMPL_CHUNK_SPLIT without it fails with
 * GDN_ERR_SHAPE.
 */
int gdn_prefill_workspace_bytes(const gdn_prefill_args* args, size_t* bytes);

/*
 * Segmented prefill that allocates nothing.  It has no counterpart in the reference.
 *
 * For callers that cannot allocate device memory when they call: a plugin whose host framework
 * owns all device memory and passes only input and output pointers, or a serving loop that
 * forbids cudaMalloc after start-up (it synchronises the device and breaks a pre-planned pool).
 * Same computation as gdn_prefill_fwd's segmented path (few, long sequences), with the segment
 * workspace taken from an array of GDN_STATIC_WORKSPACE_BYTES that the library reserves on every
 * GPU that loads it and holds until the process exits; args->impl, args->workspace and
 * args->workspace_bytes are ignored (any impl value is accepted).  Explicit write vectors
 * (args->u, nsgdn's n_steps > 1) are served as in gdn_prefill_fwd.  When the usual segmentation
 * would need more, fewer and longer segments are used; if none fits, the call fails with
 * GDN_ERR_WORKSPACE (on a 148-SM B200 every shape the segmented path takes fits: its largest
 * segment-state slot is under 5 MB).  Arguments the segmented path does not serve (many
 * sequences, short T, T = 0) fail with GDN_ERR_UNSUPPORTED.
 * Calls no cudaMalloc, cudaFree or allocating routine.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before any stream capture.
 * Every call shares the one array and leaves its contents behind: calls that overlap on the GPU
 * (other streams, other threads) race on it and must be serialised by the caller.
 */
#define GDN_STATIC_WORKSPACE_BYTES (16u << 20)
int gdn_prefill_fwd_static_workspace(const gdn_prefill_args* args, void* stream);

/*
 * Layer prologue: the token-mixing inputs of one gated-DeltaNet layer, from its projections, in one
 * bandwidth-bound kernel.  Per (b, t, h): q, k, v = SiLU(depthwise causal conv of conv_size taps)
 * of their projections (computed in the projection dtype, as F.conv1d and F.silu do); then
 * q = q / max(|q|, l2_eps) * q_scale, k = k / max(|k|, l2_eps); la = -softplus(a + dt_bias) *
 * exp(A_log), clamped below at la_min when flags has GDN_PROLOGUE_CLAMP_LA; beta =
 * sigmoid(b + b_bias) * beta_scale.  The last conv_size - 1 projection rows of every channel
 * (with the incoming state before t = 0) are written as the next call's conv state.
 *
 * Replaces the torch ops between the projections and the scan in archbench's NStepGDN.forward
 * (archbench/layers/nsgdn.py:520-536: ShortConv nsgdn.py:457-470, F.normalize, the gate and
 * beta; the n-step write vector of nsgdn.py:61-75) and in fla's GatedDeltaNet.forward (fla/layers/gated_deltanet.py:240-279:
 * q/k/v_conv1d, the kernel-side l2norm with eps 1e-6, the gate and beta).
 */
#define GDN_PROLOGUE_CLAMP_LA 1
typedef struct {
  const void* xq;     /* q projection [B][T][H*DK] before the conv, dtype in_dtype */
  const void* xk;     /* k projection [B][T][H*DK] */
  const void* xv;     /* v projection [B][T][H*DV] */
  int64_t sxq_b, sxq_t, sxk_b, sxk_t, sxv_b, sxv_t;  /* element strides of b and t (16-byte multiples) */
  const void* xa;     /* gate pre-activation a [B][T][H], dtype in_dtype */
  const void* xb;     /* beta pre-activation b [B][T][H] */
  int64_t sxa_b, sxa_t, sxb_b, sxb_t;
  const float* wq;    /* conv weights (conv_size, H*DK) fp32, tap-major (the transpose of the
                         layer's (channels, 1, conv_size) parameter), 16-byte aligned, or NULL:
                         no conv, SiLU only */
  const float* wk;
  const float* wv;    /* (conv_size, H*DV) */
  const void* cq_in;  /* conv states (B, channels, conv_size - 1), dtype in_dtype, or NULL: zero history */
  const void* ck_in;
  const void* cv_in;
  void* cq_out;       /* next conv states, same layout, or NULL; must not overlap the _in states */
  void* ck_out;
  void* cv_out;
  int64_t scq_b, sck_b, scv_b;  /* batch strides of the conv states, in elements */
  const float* A_log; /* (H) fp32 */
  const float* dt_bias; /* (H) fp32 */
  const float* b_bias;  /* (H) fp32, or NULL */
  void* q;            /* [B][T][H][DK] contiguous, dtype out_dtype */
  void* k;
  void* v;            /* [B][T][H][DV] contiguous */
  float* la;          /* (B, T, H) fp32 */
  float* beta;        /* (B, T, H) fp32 */
  int64_t B, T, H, DK, DV;  /* DK in {64, 128, 256}, DK <= DV <= 2 DK, DV a power of two */
  int32_t conv_size;  /* 1 .. 4 taps */
  int32_t flags;      /* GDN_PROLOGUE_CLAMP_LA */
  int32_t in_dtype;   /* gdn_dtype of the projections and conv states */
  int32_t out_dtype;  /* gdn_dtype of q, k, v */
  float q_scale, l2_eps, la_min, beta_scale;
  /* n-step write vectors (archbench/layers/nsgdn.py:61-75, NStepGDN n_steps > 1): with n_steps > 1 the
   * kernel also writes u = beta k, then n_steps - 1 times u -= lam beta (p . u) (p - (p . k) k) with
   * p the previous token's normalised k (k_prev_in before t = 0, zero when NULL). */
  void* u;            /* [B][T][H][DK] contiguous, dtype out_dtype; required when n_steps > 1 */
  const float* lam;   /* (H) fp32 step sizes (the layer's softplus(lam)); required when n_steps > 1 */
  const float* k_prev_in;  /* (B, H, DK) fp32, or NULL */
  float* k_prev_out;  /* (B, H, DK) fp32 normalised k of token T - 1, or NULL */
  int32_t n_steps;    /* 0 or 1: no write vectors; 2 .. 8 */
  int32_t reserved;
} gdn_prologue_args;

int gdn_layer_prologue(const gdn_prologue_args* args, void* stream);

/*
 * Layer epilogue: o = y / sqrt(mean(y^2) + eps) * weight * SiLU(g) over each head's DV values, in
 * fp32 and rounded once to o_dtype (g == NULL: no gate).  Replaces the RMSNorm and gate of
 * archbench's NStepGDN.forward (archbench/layers/nsgdn.py:539-541) and fla's FusedRMSNormGated
 * in GatedDeltaNet.forward (fla/layers/gated_deltanet.py:307-313).
 */
typedef struct {
  const void* y;      /* [B][T][H][DV] token-mixing output, 16-byte aligned */
  gdn_strides sy;
  const void* g;      /* gate [B][T][H*DV], or NULL */
  int64_t sg_b, sg_t;
  const float* weight;  /* (DV) fp32 */
  void* o;            /* [B][T][H*DV] */
  int64_t so_b, so_t;
  int64_t B, T, H, DV;  /* DV in {64, 128, 256, 512}; B * T * H < 2^26 */
  int32_t y_dtype, g_dtype, o_dtype;
  float eps;
} gdn_epilogue_args;

int gdn_layer_epilogue(const gdn_epilogue_args* args, void* stream);

/*
 * Prefill backward: gradients of gdn_prefill_fwd's outputs (y and, optionally, the final state)
 * with respect to q, k, u (or beta), v, la and the initial state, for DK = 128 and DV a multiple of
 * 128 up to 1024 (a state of more than 128 rows runs as 128-row slices, one after another).
 *
 * Replaces the backward of the custom ops archbench's scan runs under autograd:
 * archbench::nsgdn_chunk_bwd (archbench/layers/nsgdn.py:369-384, registered as the autograd
 * formula of nsgdn_chunk_fwd at nsgdn.py:386-397) and archbench::nsgdn_bwd (nsgdn.py:185-216,
 * the recurrent scan's backward); and, for the `gdn` mixer, fla's chunk_gated_delta_rule
 * backward.  Inputs are the forward's inputs (the forward saves nothing: every chunk product is
 * recomputed) plus dy and, when the final state was an output, ds_T.
 *
 * Outputs are fp32 and contiguous: dq, dk (and du) (B, T, H, DK); dv (B, T, H, DV); dla and dbeta
 * (B, T, H); ds0 (B, H, DV, DK) or NULL.  With u == NULL (u = beta k) dk includes the write
 * vector's path and dbeta is written; with u given, du is written and beta/dbeta are ignored.
 * Token tensors need 16-byte aligned rows.  The workspace (gdn_prefill_bwd_workspace_bytes,
 * 256-byte aligned) holds per chunk T, A, W, T V, the fp16 operands of the two state chains, the
 * state entering the chunk and the state gradient leaving it: about 208 KB per (b, h, 64-token
 * chunk).  One memset and four launches on `stream`.
 */
typedef struct {
  const void* q;       /* [B][T][H][DK], dtype in_dtype */
  const void* k;
  const void* u;       /* write vector or NULL (u = beta k) */
  const void* v;       /* [B][T][H][DV] */
  const float* beta;   /* (B, T, H) when u == NULL */
  const float* la;     /* (B, T, H) */
  const float* s0;     /* (B, H, DV, DK) initial state or NULL (zero) */
  const void* dy;      /* [B][T][H][DV] gradient of y, dtype dy_dtype */
  const float* ds_T;   /* (B, H, DV, DK) gradient of the final state, or NULL (zero) */
  float* dq;
  float* dk;
  float* du;           /* when u is given */
  float* dv;
  float* dbeta;        /* when u == NULL */
  float* dla;
  float* ds0;          /* or NULL */
  gdn_strides sq, sk, su, sv, sdy;
  int64_t B, T, H, DK, DV;
  int32_t in_dtype;    /* gdn_dtype of q, k, u, v */
  int32_t dy_dtype;    /* gdn_dtype of dy */
  void* workspace;
  uint64_t workspace_bytes;
} gdn_backward_args;

int gdn_prefill_bwd_workspace_bytes(const gdn_backward_args* args, size_t* bytes);
int gdn_prefill_bwd(const gdn_backward_args* args, void* stream);

/*
 * Backward of the layer prologue for training (no incoming conv state): gradients of the q, k, v
 * projections, the gate pre-activations, the conv weights and A_log / dt_bias / b_bias, given the
 * gradients of q, k, v (dtype grad_dtype, contiguous [B][T][H][D]) and of la, beta.  Replaces the
 * autograd of the torch ops it fuses (archbench/layers/nsgdn.py:457-470, 520-536; the ShortConv backward
 * at nsgdn.py:426-454).  Parameter gradients are fp32, zeroed and then accumulated with atomic adds
 * (their summation order is not fixed).  DK = 64 or 128, DV in {DK, 2 DK}.
 */
typedef struct {
  const void* xq;     /* forward inputs, as in gdn_prologue_args */
  const void* xk;
  const void* xv;
  int64_t sxq_b, sxq_t, sxk_b, sxk_t, sxv_b, sxv_t;
  const void* xa;
  const void* xb;
  int64_t sxa_b, sxa_t, sxb_b, sxb_t;
  const float* wq;    /* (conv_size, H*DK) fp32 tap-major, or NULL */
  const float* wk;
  const float* wv;
  const float* A_log;
  const float* dt_bias;
  const float* b_bias;
  const void* dq;     /* [B][T][H][DK] contiguous, dtype grad_dtype */
  const void* dk;
  const void* dv;     /* [B][T][H][DV] */
  const float* dla;   /* (B, T, H) */
  const float* dbeta;
  void* dxq;          /* projection gradients, dtype in_dtype, element strides of b and t below */
  void* dxk;
  void* dxv;
  int64_t sdxq_b, sdxq_t, sdxk_b, sdxk_t, sdxv_b, sdxv_t;
  void* dxa;
  void* dxb;
  int64_t sdxa_b, sdxa_t, sdxb_b, sdxb_t;
  float* dwq;         /* (conv_size, H*DK) fp32; NULL exactly when wq is NULL */
  float* dwk;
  float* dwv;
  float* dA_log;      /* (H) fp32 */
  float* ddt_bias;
  float* db_bias;     /* or NULL */
  int64_t B, T, H, DK, DV;
  int32_t conv_size, flags, in_dtype, grad_dtype;
  float q_scale, l2_eps, la_min, beta_scale;
} gdn_prologue_bwd_args;

int gdn_layer_prologue_bwd(const gdn_prologue_bwd_args* args, void* stream);

/*
 * Backward of the layer epilogue: dy ([B][T][H][DV] contiguous, dtype y_dtype), dg ([B][T][H*DV]
 * with the strides given, dtype g_dtype; when g is given) and dweight ((DV) fp32, zeroed then accumulated with
 * atomic adds) for the gradient `dout` of o.  Replaces the autograd of RMSNorm x SiLU(g)
 * (archbench/layers/nsgdn.py:539-541; fla's FusedRMSNormGated).
 */
typedef struct {
  const void* y;
  gdn_strides sy;
  const void* g;      /* or NULL */
  int64_t sg_b, sg_t;
  const float* weight;
  const void* dout;   /* [B][T][H*DV], element strides of b and t below, dtype do_dtype */
  int64_t sdo_b, sdo_t;
  void* dy;
  void* dg;
  int64_t sdg_b, sdg_t;  /* element strides of b and t of dg (unit channel stride) */
  float* dweight;
  int64_t B, T, H, DV;  /* B * T * H < 2^26 */
  int32_t y_dtype, g_dtype, do_dtype;
  float eps;
} gdn_epilogue_bwd_args;

int gdn_layer_epilogue_bwd(const gdn_epilogue_bwd_args* args, void* stream);

/*
 * Backward of nsgdn's n-step write vectors (replaces autograd through `write_direction`,
 * archbench/layers/nsgdn.py:61-75, as NStepGDN.forward calls it at nsgdn.py:529-533): u is built
 * from the normalised k of token t, p = k of token t - 1 (zero at t = 0, no cache in training),
 * beta and the head's step size lam.  Given du, adds the write vectors' share to dk (both the
 * token's own and its successor's, through p) and writes dbeta and dlam.  All tensors contiguous;
 * k, du and dk 16-byte aligned.  dlam is summed with fp32 atomics (order not fixed).
 */
typedef struct gdn_write_vectors_bwd_args {
  const void* k;       /* (B, T, H, DK), k_dtype: the normalised keys */
  const float* beta;   /* (B, T, H) */
  const float* lam;    /* (H): softplus of the layer's lam */
  const float* du;     /* (B, T, H, DK): gradient of the write vectors */
  float* dk;           /* (B, T, H, DK), in/out: the write vectors' share is added */
  float* dbeta;        /* (B, T, H), out */
  float* dlam;         /* (H), out */
  int64_t B, T, H, DK; /* DK 64 or 128; B * T * H < 2^30 */
  int32_t k_dtype;     /* GDN_DTYPE_BF16 or GDN_DTYPE_F32 */
  int32_t n_steps;     /* 2 .. 8 */
} gdn_write_vectors_bwd_args;

int gdn_write_vectors_bwd(const gdn_write_vectors_bwd_args* args, void* stream);

/* Which kernel a prefill with these arguments runs (GDN_IMPL_CHUNK_CLUSTER, _CHUNK_SINGLE,
 * _CHUNK_SPLIT, _SEGMENTED or _RECURRENT; GDN_IMPL_CHUNK resolves to one of the two single-launch
 * chunk variants), or a negative gdn_status if the arguments are invalid.  Launches nothing. */
int gdn_prefill_select_impl(const gdn_prefill_args* args);

/*
 * Read (and, if `reset` is non-zero, clear) the library's sticky device-side status word.
 * A kernel whose bounded wait on an mbarrier gave up stores GDN_ERR_TIMEOUT there, skips the
 * rest of its work, releases its tensor memory and returns, so the context stays usable.
 * Synchronises the current device (cudaMemcpyFromSymbol).  `*status` is GDN_OK when no kernel
 * reported a problem.
 */
int gdn_device_status(int* status, int reset);

/*
 * Failure-detection self test: launches one CTA that waits on an mbarrier nothing arrives on,
 * gives up after `max_cycles` SM clocks (0 < max_cycles <= 4e9), stores GDN_ERR_TIMEOUT in the
 * device status word and exits normally -- the same bounded-wait path every kernel uses.  Read
 * the outcome with gdn_device_status.  The context stays usable.
 */
int gdn_selftest_bounded_wait(long long max_cycles, void* stream);

/* Static description of a status code. */
const char* gdn_status_string(int status);

/* GDN_B200_ABI_VERSION of the loaded library. */
int gdn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
