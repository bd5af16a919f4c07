// Layer prologue and epilogue of the gated-DeltaNet mixers, each one bandwidth-bound kernel.
//
// Prologue: from the layer's projections to the token-mixing inputs.  Per (b, t, h):
//   q, k, v  <- SiLU(depthwise causal conv over conv_size taps of the projection), computed in the
//               projection's dtype as archbench/layers/nsgdn.py:457-470 does (F.conv1d then F.silu);
//   q        <- q / max(|q|, eps) * q_scale,  k <- k / max(|k|, eps)          (nsgdn.py:526-527)
//   la       <- -softplus(a + dt_bias) * exp(A_log), optionally clamped below  (nsgdn.py:530-532)
//   beta     <- sigmoid(b + b_bias) * beta_scale                                (nsgdn.py:533)
// and the last conv_size - 1 projection rows of every channel as the next call's conv state.
// fla's gdn mixer (fla/layers/gated_deltanet.py:240-279) is the same computation with three
// separately projected inputs, eps = 1e-6 and no b_bias.
//
// Epilogue: o = y / sqrt(mean(y^2) + eps) * weight * SiLU(g) over each head's DV values
// (nsgdn.py:539-541; fla's FusedRMSNormGated), in fp32, rounded once to the output dtype.
//
// Prologue: one warp per (b, h) and run of up to 16 consecutive tokens, a lane owning DK/32 channels
// of q and k and DV/32 of v; the run's projection rows are staged in shared memory with asynchronous
// copies, so each projection row is read once and a warp's loads are all in flight together.
// Epilogue: one warp per (b, t, h).
#include <math.h>
#include <string.h>

#include "gdn_common.cuh"

namespace gdn {
namespace layer_io {

constexpr int MAX_TAPS = 4;   // largest conv_size served (the reference uses 4)
constexpr int TOKS = 4;       // warps per prologue block

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}
// SiLU with the fast exponential and division (a few ulps of fp32, far below the bf16 rounding of
// the projections; for fp32 projections within 1e-6 relative of torch's): the prologue is
// otherwise bound by the instruction cost of the precise forms.
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }  // torch's threshold

// N consecutive outputs with vector stores of up to 16 bytes (the address is aligned to them).
template <typename TO, int N>
__device__ __forceinline__ void store_vec(TO* p, const float (&v)[N]) {
  if constexpr (sizeof(TO) == 2) {
    static_assert(N % 2 == 0, "pairs of bf16");
    uint32_t w[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
#pragma unroll
    for (int i = 0; i < N / 2; i += 4) {
      if (N / 2 - i >= 4) *reinterpret_cast<uint4*>(p + 2 * i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
      else if (N / 2 - i >= 2) *reinterpret_cast<uint2*>(p + 2 * i) = make_uint2(w[i], w[i + 1]);
      else *reinterpret_cast<uint32_t*>(p + 2 * i) = w[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      if (N - i >= 4) *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      else if (N - i >= 2) *reinterpret_cast<float2*>(p + i) = make_float2(v[i], v[i + 1]);
      else p[i] = v[i];
    }
  }
}

// N consecutive fp32 values with 16-byte loads (the address is 16-byte aligned).
template <int N>
__device__ __forceinline__ void load_f32(const float* p, float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(p + i));
      v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = __ldg(p + i);
  }
}

struct Comp {            // one of q, k, v
  const void* x;         // projection [B][T][channels] with strides
  int64_t sb, st;
  const float* w;        // (taps, channels) fp32, tap-major, or NULL: no convolution (SiLU only)
  int64_t wch;           // channels (the row length of w)
  const void* cin;       // conv state in (B, channels, taps - 1) with batch stride, or NULL
  void* cout;            // conv state out, or NULL
  int64_t csb;
  void* out;             // [B][T][H][D] contiguous
};

struct PrologueParams {
  Comp q, k, v;
  const void* xa;
  const void* xb;
  int64_t sa_b, sa_t, sb_b, sb_t;
  const float* A_log;
  const float* dt_bias;
  const float* b_bias;
  float* la;
  float* beta;
  int B, T, H, DK, DV, taps, clamp;
  int run;  // tokens per warp (set at launch)
  float q_scale, eps, la_min, beta_scale;
  int n_steps;            // write-vector steps (nsgdn.py:61-75); > 1: u below
  void* u;                // [B][T][H][DK] contiguous, out dtype
  const float* lam;       // (H) step sizes (the layer's softplus(lam))
  const float* kprev_in;  // (B, H, DK) fp32 normalised k before t = 0, or NULL (zero)
  float* kprev_out;       // (B, H, DK) fp32 normalised k of token T - 1, or NULL
};

// Row `t` (t < 0: the incoming conv state, or zeros) of channels [c0, c0 + NPL) of a component.
template <typename TX, int NPL>
__device__ __forceinline__ void load_row(const Comp& cp, int b, int t, int taps, int c0, float (&r)[NPL]) {
  if (t >= 0) {
    load_vec<NPL>(reinterpret_cast<const TX*>(cp.x) + (int64_t)b * cp.sb + (int64_t)t * cp.st + c0, r);
  } else {
#pragma unroll
    for (int n = 0; n < NPL; ++n) r[n] = 0.f;
    if (cp.cin) {
      const TX* pc = reinterpret_cast<const TX*>(cp.cin) + (int64_t)b * cp.csb;
#pragma unroll
      for (int n = 0; n < NPL; ++n) r[n] = to_f32(pc[(int64_t)(c0 + n) * (taps - 1) + (taps - 1) + t]);
    }
  }
}

// One block per (b, h) and TOKS runs of p.run consecutive tokens, one run per warp.  The block stages the
// head's conv weights (rounded to the projection dtype) in shared memory; each warp copies the projection
// rows of its run (and the TAPS - 1 rows before it) into shared memory with asynchronous copies, all in
// flight at once, then computes its tokens from there: every projection row is read from HBM once.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

// SiLU(conv) of one component at one token from staged rows (row j of the window at rows + j * ld),
// taps accumulated in order 0 .. TAPS - 1, in the projection dtype as F.conv1d(x, weight.to(x.dtype)).
template <typename TX, int TAPS, int NPL>
__device__ __forceinline__ void conv_tok(const TX* rows, int ld, const float* w, int wld, bool has_w, float (&out)[NPL]) {
  if (has_w) {
    float acc[NPL];
#pragma unroll
    for (int n = 0; n < NPL; ++n) acc[n] = 0.f;
#pragma unroll
    for (int j = 0; j < TAPS; ++j) {
      float wj[NPL], xj[NPL];
      load_vec<NPL>(w + j * wld, wj);
      load_vec<NPL>(rows + j * ld, xj);
#pragma unroll
      for (int n = 0; n < NPL; ++n) acc[n] = fmaf(wj[n], xj[n], acc[n]);
    }
#pragma unroll
    for (int n = 0; n < NPL; ++n) out[n] = round_to<TX>(silu(round_to<TX>(acc[n])));
  } else {
    float x[NPL];
    load_vec<NPL>(rows + (TAPS - 1) * ld, x);
#pragma unroll
    for (int n = 0; n < NPL; ++n) out[n] = round_to<TX>(silu(x[n]));
  }
}

template <typename TX, typename TO, int NK, int NV, int TAPS>
__global__ void __launch_bounds__(32 * TOKS) prologue_kernel(const PrologueParams p) {
  extern __shared__ __align__(16) float sw[];  // weights [q | k | v] x TAPS x (DK or DV), then the warps' rows
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int RUN = p.run;  // tokens per warp
  constexpr int W = 2 * 32 * NK + 32 * NV;  // elements per staged row
  const int runs = (p.T + RUN - 1) / RUN, rgroups = (runs + TOKS - 1) / TOKS;
  const int bh = blockIdx.x / rgroups, rg = blockIdx.x - bh * rgroups;
  const int b = bh / p.H, h = bh - b * p.H;
  constexpr int DK = 32 * NK, DV = 32 * NV;  // == p.DK, p.DV
  const Comp* cs[3] = {&p.q, &p.k, &p.v};
  constexpr int off[3] = {0, DK, 2 * DK}, len[3] = {DK, DK, DV};
  float* swc[3] = {sw, sw + TAPS * DK, sw + 2 * TAPS * DK};
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    if (!cs[c]->w) continue;
    for (int i = threadIdx.x; i < TAPS * len[c]; i += blockDim.x) {
      const int j = i / len[c], ch = i - j * len[c];
      swc[c][i] = round_to<TX>(cs[c]->w[(int64_t)j * cs[c]->wch + (int64_t)h * len[c] + ch]);
    }
  }
  TX* stage = reinterpret_cast<TX*>(sw + TAPS * W) + (size_t)wid * (RUN + TAPS) * W;
  const bool nstep = p.n_steps > 1;
  const int lead = nstep ? 1 : 0;  // n-step write vectors need k of the token before the run
  __syncthreads();
  const int run = rg * TOKS + wid;
  if (run >= runs) return;
  const int t0 = run * RUN, t1 = min(p.T, t0 + RUN), nrows = t1 - t0 + TAPS - 1 + lead;
  // staged row r holds token t0 - (TAPS - 1) - lead + r; tokens before 0 come from the incoming conv state
  constexpr int EPC = 16 / sizeof(TX);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const Comp& cp = *cs[c];
    constexpr int chunks_[3] = {len[0] / EPC, len[1] / EPC, len[2] / EPC};
    const int chunks = chunks_[c], hc = h * len[c];
    for (int i = lane; i < nrows * chunks; i += 32) {
      const int r = i / chunks, q = i - r * chunks, t = t0 - (TAPS - 1) - lead + r;
      TX* dst = stage + (size_t)r * W + off[c] + q * EPC;
      if (t >= 0) {
        cp16(dst, reinterpret_cast<const TX*>(cp.x) + (int64_t)b * cp.sb + (int64_t)t * cp.st + hc + q * EPC);
      } else if (t < -(TAPS - 1)) {  // before the conv state: only reached for k of token -1, which is unused
#pragma unroll
        for (int e = 0; e < EPC; ++e) store_as(dst + e, 0.f);
      } else {
        const TX* pc = cp.cin ? reinterpret_cast<const TX*>(cp.cin) + (int64_t)b * cp.csb : nullptr;
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
          const int ch = hc + q * EPC + e;
          store_as(dst + e, pc ? to_f32(pc[(int64_t)ch * (TAPS - 1) + (TAPS - 1) + t]) : 0.f);
        }
      }
    }
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncwarp();
  const bool wq = p.q.w != nullptr, wk = p.k.w != nullptr, wv = p.v.w != nullptr;
  const float dtb = p.dt_bias[h], Ae = expf(p.A_log[h]), bb_h = p.b_bias ? p.b_bias[h] : 0.f;
  // n-step write vectors: p = k of the previous token (normalised), from the run's lead row, the
  // incoming k_prev at t = 0, or zero
  float kp[NK];
#pragma unroll
  for (int n = 0; n < NK; ++n) kp[n] = 0.f;
  const float lam_h = nstep ? p.lam[h] : 0.f;
  // beta of token t0 + lane (a run has at most 16 tokens), loaded and formed before the token loop, which
  // takes it by shuffle: a load per token there would put its latency on the loop's critical path
  float bt_lane = 0.f;
  if (nstep && t0 + lane < t1) {
    const float xbt = to_f32(reinterpret_cast<const TX*>(p.xb)[(int64_t)b * p.sb_b + (int64_t)(t0 + lane) * p.sb_t + h]);
    bt_lane = p.beta_scale / (1.f + expf(-(xbt + bb_h)));
  }
  if (nstep) {
    if (t0 > 0) {
      conv_tok<TX, TAPS, NK>(stage + DK + lane * NK, W, swc[1] + lane * NK, DK, wk, kp);
      float s2 = 0.f;
#pragma unroll
      for (int n = 0; n < NK; ++n) s2 = fmaf(kp[n], kp[n], s2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      const float ik = 1.f / fmaxf(sqrtf(s2), p.eps);
#pragma unroll
      for (int n = 0; n < NK; ++n) kp[n] *= ik;
    } else if (p.kprev_in) {
      load_f32<NK>(p.kprev_in + ((int64_t)b * p.H + h) * DK + lane * NK, kp);
    }
  }
#pragma unroll 1
  for (int t = t0; t < t1; ++t) {
    const TX* rows = stage + (size_t)(t - t0 + lead) * W;
    float q[NK], k[NK], v[NV];
    conv_tok<TX, TAPS, NK>(rows + lane * NK, W, swc[0] + lane * NK, DK, wq, q);
    conv_tok<TX, TAPS, NK>(rows + DK + lane * NK, W, swc[1] + lane * NK, DK, wk, k);
    conv_tok<TX, TAPS, NV>(rows + 2 * DK + lane * NV, W, swc[2] + lane * NV, DV, wv, v);
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int n = 0; n < NK; ++n) {
      sq = fmaf(q[n], q[n], sq);
      sk = fmaf(k[n], k[n], sk);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    const float iq = p.q_scale / fmaxf(sqrtf(sq), p.eps), ik = 1.f / fmaxf(sqrtf(sk), p.eps);
    const int64_t tok = ((int64_t)b * p.T + t) * p.H + h;
#pragma unroll
    for (int n = 0; n < NK; ++n) {
      q[n] *= iq;
      k[n] *= ik;
    }
    store_vec<TO, NK>(reinterpret_cast<TO*>(p.q.out) + tok * DK + lane * NK, q);
    store_vec<TO, NK>(reinterpret_cast<TO*>(p.k.out) + tok * DK + lane * NK, k);
    store_vec<TO, NV>(reinterpret_cast<TO*>(p.v.out) + tok * DV + lane * NV, v);
    if (nstep) {  // u = beta k, then n - 1 steps u -= lam beta (p . u) (p - (p . k) k)   (nsgdn.py:61-75)
      const float bt = __shfl_sync(0xffffffffu, bt_lane, t - t0);
      float pk = 0.f;
#pragma unroll
      for (int n = 0; n < NK; ++n) pk = fmaf(kp[n], k[n], pk);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pk += __shfl_xor_sync(0xffffffffu, pk, o);
      float u[NK], pp[NK];
#pragma unroll
      for (int n = 0; n < NK; ++n) {
        pp[n] = kp[n] - pk * k[n];
        u[n] = bt * k[n];
      }
      const float lb = lam_h * bt;
#pragma unroll 1
      for (int st = 1; st < p.n_steps; ++st) {
        float pu = 0.f;
#pragma unroll
        for (int n = 0; n < NK; ++n) pu = fmaf(kp[n], u[n], pu);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pu += __shfl_xor_sync(0xffffffffu, pu, o);
#pragma unroll
        for (int n = 0; n < NK; ++n) u[n] -= lb * pu * pp[n];
      }
      store_vec<TO, NK>(reinterpret_cast<TO*>(p.u) + tok * DK + lane * NK, u);
#pragma unroll
      for (int n = 0; n < NK; ++n) kp[n] = k[n];
    }
  }
  if (nstep && t1 == p.T && p.kprev_out) {
#pragma unroll
    for (int n = 0; n < NK; ++n) p.kprev_out[((int64_t)b * p.H + h) * DK + lane * NK + n] = kp[n];
  }
  // the gates, one token per lane
  for (int t = t0 + lane; t < t1; t += 32) {
    const int64_t tok = ((int64_t)b * p.T + t) * p.H + h;
    const float a = to_f32(reinterpret_cast<const TX*>(p.xa)[(int64_t)b * p.sa_b + (int64_t)t * p.sa_t + h]);
    const float bb = to_f32(reinterpret_cast<const TX*>(p.xb)[(int64_t)b * p.sb_b + (int64_t)t * p.sb_t + h]);
    float la = -softplus(a + dtb) * Ae;
    if (p.clamp) la = fmaxf(la, p.la_min);
    p.la[tok] = la;
    p.beta[tok] = p.beta_scale / (1.f + expf(-(bb + bb_h)));
  }
  // the next call's conv state: tokens T - (TAPS - 1) .. T - 1, staged rows t1 - t0 .. t1 - t0 + TAPS - 2
  if (t1 == p.T && TAPS > 1) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const Comp& cp = *cs[c];
      if (!cp.cout) continue;
      TX* pc = reinterpret_cast<TX*>(cp.cout) + (int64_t)b * cp.csb;
      for (int i = lane; i < (TAPS - 1) * len[c]; i += 32) {
        const int j = i / len[c], ch = i - j * len[c];
        pc[(int64_t)(h * len[c] + ch) * (TAPS - 1) + j] = stage[(size_t)(t1 - t0 + lead + j) * W + off[c] + ch];
      }
    }
  }
}

// One-token calls (decode steps): one warp per (b, h) and nothing staged.  The same arithmetic as
// prologue_kernel at T = 1, in the same order: the window is the incoming conv state and the token's
// projection row, the conv weights are rounded to the projection dtype as read from the fp32 copy.
// The new conv state of a channel is written by the lane that read the old one, after reading it,
// so it may overwrite the incoming state in place.
template <typename TX, int TAPS, int NPL>
__device__ __forceinline__ void conv_window(const Comp& cp, int b, int c0, float (&r)[TAPS][NPL], float (&out)[NPL]) {
#pragma unroll
  for (int j = 0; j < TAPS; ++j) load_row<TX, NPL>(cp, b, j - (TAPS - 1), TAPS, c0, r[j]);
  if (cp.w) {
    float acc[NPL];
#pragma unroll
    for (int n = 0; n < NPL; ++n) acc[n] = 0.f;
#pragma unroll
    for (int j = 0; j < TAPS; ++j) {
      float wj[NPL];
      load_f32<NPL>(cp.w + (int64_t)j * cp.wch + c0, wj);
#pragma unroll
      for (int n = 0; n < NPL; ++n) acc[n] = fmaf(round_to<TX>(wj[n]), r[j][n], acc[n]);
    }
#pragma unroll
    for (int n = 0; n < NPL; ++n) out[n] = round_to<TX>(silu(round_to<TX>(acc[n])));
  } else {
#pragma unroll
    for (int n = 0; n < NPL; ++n) out[n] = round_to<TX>(silu(r[TAPS - 1][n]));
  }
}

template <typename TX, int TAPS, int NPL>
__device__ __forceinline__ void conv_state_out(const Comp& cp, int b, int c0, const float (&r)[TAPS][NPL]) {
  if (TAPS < 2 || !cp.cout) return;
  TX* pc = reinterpret_cast<TX*>(cp.cout) + (int64_t)b * cp.csb;
#pragma unroll
  for (int n = 0; n < NPL; ++n)
#pragma unroll
    for (int j = 0; j + 1 < TAPS; ++j) store_as(pc + (int64_t)(c0 + n) * (TAPS - 1) + j, r[j + 1][n]);
}

template <typename TX, typename TO, int NK, int NV, int TAPS>
__global__ void __launch_bounds__(128) prologue_decode_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (bh >= p.B * p.H) return;
  const int b = bh / p.H, h = bh - b * p.H;
  constexpr int DK = 32 * NK, DV = 32 * NV;
  float rq[TAPS][NK], rk[TAPS][NK], rv[TAPS][NV];
  float q[NK], k[NK], v[NV];
  conv_window<TX, TAPS, NK>(p.q, b, h * DK + lane * NK, rq, q);
  conv_window<TX, TAPS, NK>(p.k, b, h * DK + lane * NK, rk, k);
  conv_window<TX, TAPS, NV>(p.v, b, h * DV + lane * NV, rv, v);
  const bool nstep = p.n_steps > 1;
  float kp[NK];
#pragma unroll
  for (int n = 0; n < NK; ++n) kp[n] = 0.f;
  if (nstep && p.kprev_in) load_f32<NK>(p.kprev_in + ((int64_t)b * p.H + h) * DK + lane * NK, kp);
  conv_state_out<TX, TAPS, NK>(p.q, b, h * DK + lane * NK, rq);
  conv_state_out<TX, TAPS, NK>(p.k, b, h * DK + lane * NK, rk);
  conv_state_out<TX, TAPS, NV>(p.v, b, h * DV + lane * NV, rv);
  float sq = 0.f, sk = 0.f;
#pragma unroll
  for (int n = 0; n < NK; ++n) {
    sq = fmaf(q[n], q[n], sq);
    sk = fmaf(k[n], k[n], sk);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    sk += __shfl_xor_sync(0xffffffffu, sk, o);
  }
  const float iq = p.q_scale / fmaxf(sqrtf(sq), p.eps), ik = 1.f / fmaxf(sqrtf(sk), p.eps);
  const int64_t tok = (int64_t)b * p.H + h;  // T = 1
#pragma unroll
  for (int n = 0; n < NK; ++n) {
    q[n] *= iq;
    k[n] *= ik;
  }
  store_vec<TO, NK>(reinterpret_cast<TO*>(p.q.out) + tok * DK + lane * NK, q);
  store_vec<TO, NK>(reinterpret_cast<TO*>(p.k.out) + tok * DK + lane * NK, k);
  store_vec<TO, NV>(reinterpret_cast<TO*>(p.v.out) + tok * DV + lane * NV, v);
  const float dtb = p.dt_bias[h], Ae = expf(p.A_log[h]), bb_h = p.b_bias ? p.b_bias[h] : 0.f;
  const float xbt = to_f32(reinterpret_cast<const TX*>(p.xb)[(int64_t)b * p.sb_b + h]);
  if (nstep) {  // u = beta k, then n - 1 steps u -= lam beta (p . u) (p - (p . k) k)   (nsgdn.py:61-75)
    const float bt = p.beta_scale / (1.f + expf(-(xbt + bb_h)));
    const float lam_h = p.lam[h];
    float pk = 0.f;
#pragma unroll
    for (int n = 0; n < NK; ++n) pk = fmaf(kp[n], k[n], pk);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) pk += __shfl_xor_sync(0xffffffffu, pk, o);
    float u[NK], pp[NK];
#pragma unroll
    for (int n = 0; n < NK; ++n) {
      pp[n] = kp[n] - pk * k[n];
      u[n] = bt * k[n];
    }
    const float lb = lam_h * bt;
#pragma unroll 1
    for (int st = 1; st < p.n_steps; ++st) {
      float pu = 0.f;
#pragma unroll
      for (int n = 0; n < NK; ++n) pu = fmaf(kp[n], u[n], pu);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pu += __shfl_xor_sync(0xffffffffu, pu, o);
#pragma unroll
      for (int n = 0; n < NK; ++n) u[n] -= lb * pu * pp[n];
    }
    store_vec<TO, NK>(reinterpret_cast<TO*>(p.u) + tok * DK + lane * NK, u);
    if (p.kprev_out) {
#pragma unroll
      for (int n = 0; n < NK; ++n) p.kprev_out[((int64_t)b * p.H + h) * DK + lane * NK + n] = k[n];
    }
  }
  if (lane == 0) {  // the gates of the token
    const float a = to_f32(reinterpret_cast<const TX*>(p.xa)[(int64_t)b * p.sa_b + h]);
    float la = -softplus(a + dtb) * Ae;
    if (p.clamp) la = fmaxf(la, p.la_min);
    p.la[tok] = la;
    p.beta[tok] = p.beta_scale / (1.f + expf(-(xbt + bb_h)));
  }
}

template <typename TX, typename TO, int NK, int NV>
int launch_prologue_decode(const PrologueParams& p, cudaStream_t s) {
  const unsigned blocks = (unsigned)(((int64_t)p.B * p.H + 3) / 4);
  switch (p.taps) {
    case 1: prologue_decode_kernel<TX, TO, NK, NV, 1><<<blocks, 128, 0, s>>>(p); break;
    case 2: prologue_decode_kernel<TX, TO, NK, NV, 2><<<blocks, 128, 0, s>>>(p); break;
    case 3: prologue_decode_kernel<TX, TO, NK, NV, 3><<<blocks, 128, 0, s>>>(p); break;
    case 4: prologue_decode_kernel<TX, TO, NK, NV, 4><<<blocks, 128, 0, s>>>(p); break;
    default: return GDN_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

struct EpilogueParams {
  const void* y;
  gdn_strides sy;
  const void* g;
  int64_t sg_b, sg_t;
  const float* weight;
  void* o;
  int64_t so_b, so_t;
  int B, T, H, DV;
  float eps;
};

template <typename TY, typename TG, typename TO, int NPL>
__global__ void __launch_bounds__(128) epilogue_kernel(const EpilogueParams p) {
  // 32-bit index arithmetic (B * T * H * 32 < 2^31 is checked on the host): 64-bit divisions would
  // dominate this kernel's instruction count.
  const unsigned row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= (unsigned)p.B * (unsigned)p.T * (unsigned)p.H) return;
  const unsigned bt = row / (unsigned)p.H;
  const int h = (int)(row - bt * (unsigned)p.H);
  const int b = (int)(bt / (unsigned)p.T), t = (int)(bt - (unsigned)b * (unsigned)p.T);
  const int c0 = lane * NPL;
  float y[NPL];
  load_vec<NPL>(reinterpret_cast<const TY*>(p.y) + b * p.sy.b + t * p.sy.t + h * p.sy.h + c0, y);
  float ss = 0.f;
#pragma unroll
  for (int n = 0; n < NPL; ++n) ss = fmaf(y[n], y[n], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)p.DV + p.eps);
  float g[NPL];
  if (p.g) load_vec<NPL>(reinterpret_cast<const TG*>(p.g) + b * p.sg_b + t * p.sg_t + (int64_t)h * p.DV + c0, g);
  TO* po = reinterpret_cast<TO*>(p.o) + b * p.so_b + t * p.so_t + (int64_t)h * p.DV + c0;
  float wv[NPL];
  load_vec<NPL>(p.weight + c0, wv);
#pragma unroll
  for (int n = 0; n < NPL; ++n) {
    y[n] *= r * wv[n];
    if (p.g) y[n] *= silu(g[n]);
  }
  store_vec<TO, NPL>(po, y);
}

bool device_ok() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int PROLOGUE_SMEM_MAX = 96 * 1024;

// Shared memory of one prologue block: the weights and TOKS warps' staged rows.
size_t prologue_smem(const PrologueParams& p, int run, int es) {
  const size_t W = 2 * (size_t)p.DK + p.DV;
  return (size_t)p.taps * W * 4 + (size_t)TOKS * (run + p.taps) * W * es;
}

template <typename TX, typename TO, int NK, int NV, int TAPS>
int launch_prologue_one(const PrologueParams& p, unsigned blocks, size_t sm, cudaStream_t s) {
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)prologue_kernel<TX, TO, NK, NV, TAPS>, (int)PROLOGUE_SMEM_MAX}}))
    return GDN_ERR_LAUNCH;
  prologue_kernel<TX, TO, NK, NV, TAPS><<<blocks, 32 * TOKS, sm, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

template <typename TX, typename TO, int NK, int NV>
int launch_prologue_taps(const PrologueParams& p, unsigned blocks, size_t sm, cudaStream_t s) {
  switch (p.taps) {
    case 1: return launch_prologue_one<TX, TO, NK, NV, 1>(p, blocks, sm, s);
    case 2: return launch_prologue_one<TX, TO, NK, NV, 2>(p, blocks, sm, s);
    case 3: return launch_prologue_one<TX, TO, NK, NV, 3>(p, blocks, sm, s);
    case 4: return launch_prologue_one<TX, TO, NK, NV, 4>(p, blocks, sm, s);
    default: return GDN_ERR_SHAPE;
  }
}

template <typename TX, typename TO>
int launch_prologue(PrologueParams p, cudaStream_t s) {
  if (p.T == 1) {  // decode steps: one warp per (b, h), no staging
    p.run = 1;
    const int nk = p.DK / 32, nv = p.DV / 32;
#define GDN_PRO1(NK, NV) \
    if (nk == NK && nv == NV) return launch_prologue_decode<TX, TO, NK, NV>(p, s);
    GDN_PRO1(2, 2) GDN_PRO1(2, 4) GDN_PRO1(4, 4) GDN_PRO1(4, 8) GDN_PRO1(8, 8) GDN_PRO1(8, 16)
#undef GDN_PRO1
    return GDN_ERR_UNSUPPORTED;
  }
  // the longest run (16, 8, .. 1 tokens per warp) whose staging leaves room for 5 blocks per SM (44 KB),
  // else the longest that fits the budget
  int run = 16;
  while (run > 1 && prologue_smem(p, run, sizeof(TX)) > 44 * 1024) run /= 2;
  if (prologue_smem(p, run, sizeof(TX)) > 44 * 1024) {
    run = 16;
    while (run > 1 && prologue_smem(p, run, sizeof(TX)) > PROLOGUE_SMEM_MAX) run /= 2;
  }
  const size_t sm = prologue_smem(p, run, sizeof(TX));
  if (sm > PROLOGUE_SMEM_MAX) return GDN_ERR_UNSUPPORTED;
  p.run = run;
  const int64_t runs = (p.T + run - 1) / run;
  const int64_t blocks = (int64_t)p.B * p.H * ((runs + TOKS - 1) / TOKS);
  if (blocks > 0x7fffffff) return GDN_ERR_SHAPE;
  const int nk = p.DK / 32, nv = p.DV / 32;
#define GDN_PRO(NK, NV) \
  if (nk == NK && nv == NV) return launch_prologue_taps<TX, TO, NK, NV>(p, (unsigned)blocks, sm, s);
  GDN_PRO(2, 2) GDN_PRO(2, 4) GDN_PRO(4, 4) GDN_PRO(4, 8) GDN_PRO(8, 8) GDN_PRO(8, 16)
#undef GDN_PRO
  return GDN_ERR_UNSUPPORTED;
}

template <typename TY, typename TG, typename TO>
int launch_epilogue(const EpilogueParams& p, cudaStream_t s) {
  const int64_t rows = (int64_t)p.B * p.T * p.H;
  const int blocks = (int)((rows * 32 + 127) / 128);
  switch (p.DV / 32) {
    case 2: epilogue_kernel<TY, TG, TO, 2><<<blocks, 128, 0, s>>>(p); break;
    case 4: epilogue_kernel<TY, TG, TO, 4><<<blocks, 128, 0, s>>>(p); break;
    case 8: epilogue_kernel<TY, TG, TO, 8><<<blocks, 128, 0, s>>>(p); break;
    case 16: epilogue_kernel<TY, TG, TO, 16><<<blocks, 128, 0, s>>>(p); break;
    default: return GDN_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace layer_io
}  // namespace gdn

using namespace gdn::layer_io;

extern "C" {

int gdn_layer_prologue(const gdn_prologue_args* a, void* stream) {
  if (!a) return GDN_ERR_NULL;
  if (!a->xq || !a->xk || !a->xv || !a->xa || !a->xb || !a->A_log || !a->dt_bias || !a->q || !a->k || !a->v ||
      !a->la || !a->beta)
    return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->H < 1 || a->B * a->T * a->H > (int64_t)1 << 31) return GDN_ERR_SHAPE;
  const bool dk_ok = a->DK == 64 || a->DK == 128 || a->DK == 256, dv_ok = a->DV == 64 || a->DV == 128 || a->DV == 256 || a->DV == 512;
  if (!dk_ok || !dv_ok || a->DV < a->DK || a->DV > 2 * a->DK) return GDN_ERR_SHAPE;
  if (a->conv_size < 1 || a->conv_size > MAX_TAPS) return GDN_ERR_SHAPE;
  if (a->in_dtype != GDN_DTYPE_BF16 && a->in_dtype != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  if (a->out_dtype != GDN_DTYPE_BF16 && a->out_dtype != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  // Lanes load DK/32 or DV/32 consecutive channels with one vector load: 16-byte aligned rows.
  const int64_t es = a->in_dtype == GDN_DTYPE_BF16 ? 2 : 4;
  const int64_t sts[] = {a->sxq_b, a->sxq_t, a->sxk_b, a->sxk_t, a->sxv_b, a->sxv_t};
  for (int64_t st : sts)
    if ((st * es) % 16) return GDN_ERR_ALIGN;
  if (!a16(a->xq) || !a16(a->xk) || !a16(a->xv)) return GDN_ERR_ALIGN;
  const int64_t out_es = a->out_dtype == GDN_DTYPE_BF16 ? 2 : 4;
  if (!a16(a->q) || !a16(a->k) || !a16(a->v) || (a->DK / 32 * out_es) % 4) return GDN_ERR_ALIGN;
  if (!device_ok()) return GDN_ERR_DEVICE;
  PrologueParams p;
  memset(&p, 0, sizeof(p));
  p.q = {a->xq, a->sxq_b, a->sxq_t, a->wq, a->H * a->DK, a->cq_in, a->cq_out, a->scq_b, a->q};
  p.k = {a->xk, a->sxk_b, a->sxk_t, a->wk, a->H * a->DK, a->ck_in, a->ck_out, a->sck_b, a->k};
  p.v = {a->xv, a->sxv_b, a->sxv_t, a->wv, a->H * a->DV, a->cv_in, a->cv_out, a->scv_b, a->v};
  if ((a->wq && !a16(a->wq)) || (a->wk && !a16(a->wk)) || (a->wv && !a16(a->wv))) return GDN_ERR_ALIGN;
  p.xa = a->xa; p.xb = a->xb;
  p.sa_b = a->sxa_b; p.sa_t = a->sxa_t; p.sb_b = a->sxb_b; p.sb_t = a->sxb_t;
  p.A_log = a->A_log; p.dt_bias = a->dt_bias; p.b_bias = a->b_bias;
  p.la = a->la; p.beta = a->beta;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DK = (int)a->DK; p.DV = (int)a->DV;
  p.taps = a->conv_size; p.clamp = (a->flags & GDN_PROLOGUE_CLAMP_LA) != 0;
  p.q_scale = a->q_scale; p.eps = a->l2_eps; p.la_min = a->la_min; p.beta_scale = a->beta_scale;
  p.n_steps = a->n_steps < 1 ? 1 : a->n_steps;
  if (p.n_steps > 8) return GDN_ERR_SHAPE;
  if (p.n_steps > 1) {
    if (!a->u || !a->lam) return GDN_ERR_NULL;
    if (!a16(a->u) || (a->k_prev_in && !a16(a->k_prev_in))) return GDN_ERR_ALIGN;
  }
  p.u = a->u; p.lam = a->lam; p.kprev_in = a->k_prev_in; p.kprev_out = a->k_prev_out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->in_dtype == GDN_DTYPE_BF16)
    return a->out_dtype == GDN_DTYPE_BF16 ? launch_prologue<__nv_bfloat16, __nv_bfloat16>(p, s)
                                          : launch_prologue<__nv_bfloat16, float>(p, s);
  return a->out_dtype == GDN_DTYPE_BF16 ? launch_prologue<float, __nv_bfloat16>(p, s) : launch_prologue<float, float>(p, s);
}

int gdn_layer_epilogue(const gdn_epilogue_args* a, void* stream) {
  if (!a) return GDN_ERR_NULL;
  if (!a->y || !a->weight || !a->o) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->H < 1 || (a->DV != 64 && a->DV != 128 && a->DV != 256 && a->DV != 512)) return GDN_ERR_SHAPE;
  if (a->B * a->T * a->H * 32 > 0x7fffffffLL) return GDN_ERR_SHAPE;
  for (int32_t dt : {a->y_dtype, a->g_dtype, a->o_dtype})
    if (dt != GDN_DTYPE_BF16 && dt != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  if (!a16(a->y) || (a->g && !a16(a->g)) || !a16(a->o)) return GDN_ERR_ALIGN;
  if (!device_ok()) return GDN_ERR_DEVICE;
  EpilogueParams p;
  p.y = a->y; p.sy = a->sy; p.g = a->g; p.sg_b = a->sg_b; p.sg_t = a->sg_t; p.weight = a->weight;
  p.o = a->o; p.so_b = a->so_b; p.so_t = a->so_t;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DV = (int)a->DV; p.eps = a->eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using bf = __nv_bfloat16;
  const int key = a->y_dtype * 4 + a->g_dtype * 2 + a->o_dtype;  // F32 = 0, BF16 = 1
  switch (key) {
    case 7: return launch_epilogue<bf, bf, bf>(p, s);
    case 6: return launch_epilogue<bf, bf, float>(p, s);
    case 3: return launch_epilogue<float, bf, bf>(p, s);
    case 2: return launch_epilogue<float, bf, float>(p, s);
    case 5: return launch_epilogue<bf, float, bf>(p, s);
    case 4: return launch_epilogue<bf, float, float>(p, s);
    case 1: return launch_epilogue<float, float, bf>(p, s);
    default: return launch_epilogue<float, float, float>(p, s);
  }
}

}  // extern "C"
