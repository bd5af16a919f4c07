// Token-serial gated delta rule on CUDA cores, fp32 state in registers (sm_100a).
//
// This is the recurrent form of archbench/layers/nsgdn.py:408-417 (nsgdn_ref) and of the
// Triton token scan archbench/layers/nsgdn.py:80-106 (one program per (b, h, 16 rows of S)).
// It serves three callers:
//   * the decode step (T = 1, state read and written once: an HBM-bound stream),
//   * prefill in fp32 I/O, where the 1e-5 tolerance rules out fp16 tensor-core operands,
//   * prefill for head sizes the chunked tensor-core kernel does not cover.
//
// Work split: one warp owns ROWS consecutive rows (DV indices) of one (b, h) state; lane l
// holds columns [l*CPL, (l+1)*CPL) of each row, CPL = DK / 32.  Rows of S evolve
// independently given (k, u, q, v_i, alpha), so warps never communicate.  Per token:
//     alpha = exp(la);  uq = u.q                         (one warp reduction)
//     d1 = S_i.k, d2 = S_i.q                             (two reductions per row, from old S)
//     r_i = v_i - alpha d1
//     y_i = alpha d2 + r_i uq                            (= (alpha S_i + r_i u) . q)
//     S_i = alpha S_i + r_i u
// which is nsgdn_ref's update with y computed from the pre-update dot products.
#include "gdn_common.cuh"

namespace gdn {
namespace {

struct RecParams {
  const void* q;
  const void* k;
  const void* u;
  const void* v;
  const float* beta;
  const float* la;
  const float* s_in;
  float* s_out;
  void* y;
  gdn_strides sq, sk, su, sv, sy;
  int B, T, H, DV;
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int N>
__device__ __forceinline__ void load_f32_vec(const float* __restrict__ p, float (&out)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      float4 t = *reinterpret_cast<const float4*>(p + i);
      out[i] = t.x; out[i + 1] = t.y; out[i + 2] = t.z; out[i + 3] = t.w;
    }
  } else if constexpr (N == 2) {
    float2 t = *reinterpret_cast<const float2*>(p);
    out[0] = t.x; out[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = p[i];
  }
}

template <int N>
__device__ __forceinline__ void store_f32_vec(float* __restrict__ p, const float (&in)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      *reinterpret_cast<float4*>(p + i) = make_float4(in[i], in[i + 1], in[i + 2], in[i + 3]);
  } else if constexpr (N == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(in[0], in[1]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = in[i];
  }
}

template <int DK, int ROWS, int NWARPS, typename TIn, typename TOut, bool HAS_U>
__global__ void __launch_bounds__(NWARPS * 32) recurrent_kernel(const RecParams p) {
  constexpr int CPL = DK / 32;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps_per_head = (p.DV + ROWS - 1) / ROWS;
  const int64_t gw = (int64_t)blockIdx.x * NWARPS + warp;
  if (gw >= (int64_t)p.B * p.H * warps_per_head) return;
  const int bh = (int)(gw / warps_per_head);
  const int row0 = (int)(gw % warps_per_head) * ROWS;
  const int b = bh / p.H, h = bh % p.H;
  const int nrows = min(ROWS, p.DV - row0);

  const TIn* qb = static_cast<const TIn*>(p.q) + b * p.sq.b + h * p.sq.h + lane * CPL;
  const TIn* kb = static_cast<const TIn*>(p.k) + b * p.sk.b + h * p.sk.h + lane * CPL;
  const TIn* ub = HAS_U ? static_cast<const TIn*>(p.u) + b * p.su.b + h * p.su.h + lane * CPL : nullptr;
  const TIn* vb = static_cast<const TIn*>(p.v) + b * p.sv.b + h * p.sv.h + row0;
  TOut* yb = static_cast<TOut*>(p.y) + b * p.sy.b + h * p.sy.h + row0;
  const int64_t gate0 = (int64_t)b * p.T * p.H + h;

  float S[ROWS][CPL];
  const int64_t s_off = ((int64_t)bh * p.DV + row0) * DK + lane * CPL;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    if (p.s_in != nullptr && r < nrows) {
      load_f32_vec<CPL>(p.s_in + s_off + (int64_t)r * DK, S[r]);
    } else {
#pragma unroll
      for (int c = 0; c < CPL; ++c) S[r][c] = 0.f;
    }
  }

  // Register double buffer: the loads of token t+1 are issued before the maths of token t.
  float qn[CPL], kn[CPL], un[CPL];
  float vn = 0.f, lan = 0.f, bn = 0.f;
  auto fetch = [&](int t) {
    load_vec<CPL>(qb + t * p.sq.t, qn);
    load_vec<CPL>(kb + t * p.sk.t, kn);
    if constexpr (HAS_U) load_vec<CPL>(ub + t * p.su.t, un);
    vn = lane < nrows ? to_f32(vb[t * p.sv.t + lane]) : 0.f;
    lan = p.la[gate0 + (int64_t)t * p.H];
    if constexpr (!HAS_U) bn = p.beta[gate0 + (int64_t)t * p.H];
  };
  if (p.T > 0) fetch(0);

  for (int t = 0; t < p.T; ++t) {
    float qv[CPL], kv[CPL], uv[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      qv[c] = qn[c];
      kv[c] = kn[c];
      uv[c] = HAS_U ? un[c] : 0.f;
    }
    const float v_lane = vn;
    const float alpha = expf(lan);
    const float bt = bn;
    if (t + 1 < p.T) fetch(t + 1);
    if constexpr (!HAS_U) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) uv[c] = bt * kv[c];
    }
    float uq = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) uq = fmaf(uv[c], qv[c], uq);
    uq = warp_sum(uq);

    float d1[ROWS], d2[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      float a = 0.f, c2 = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        a = fmaf(S[r][c], kv[c], a);
        c2 = fmaf(S[r][c], qv[c], c2);
      }
      d1[r] = a;
      d2[r] = c2;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        d1[r] += __shfl_xor_sync(0xffffffffu, d1[r], o);
        d2[r] += __shfl_xor_sync(0xffffffffu, d2[r], o);
      }
    }
    float y_mine = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float vr = __shfl_sync(0xffffffffu, v_lane, r);
      const float rr = vr - alpha * d1[r];
      const float yr = fmaf(alpha, d2[r], rr * uq);
      if (lane == r) y_mine = yr;
#pragma unroll
      for (int c = 0; c < CPL; ++c) S[r][c] = fmaf(alpha, S[r][c], rr * uv[c]);
    }
    if (lane < nrows) store_as(yb + t * p.sy.t + lane, y_mine);
  }

  if (p.s_out != nullptr) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
      if (r < nrows) store_f32_vec<CPL>(p.s_out + s_off + (int64_t)r * DK, S[r]);
  }
}

template <int DK, int ROWS, typename TIn, typename TOut, bool HAS_U>
int launch_t(const RecParams& p, cudaStream_t stream) {
  constexpr int NWARPS = 4;
  const int64_t warps = (int64_t)p.B * p.H * ((p.DV + ROWS - 1) / ROWS);
  const int64_t blocks = (warps + NWARPS - 1) / NWARPS;
  if (blocks > 0x7fffffff) return GDN_ERR_SHAPE;
  recurrent_kernel<DK, ROWS, NWARPS, TIn, TOut, HAS_U><<<(unsigned)blocks, NWARPS * 32, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

template <int DK, int ROWS, typename TIn, typename TOut>
int launch_u(const RecParams& p, cudaStream_t s) {
  return p.u ? launch_t<DK, ROWS, TIn, TOut, true>(p, s) : launch_t<DK, ROWS, TIn, TOut, false>(p, s);
}

template <int DK, int ROWS>
int launch_dk(const RecParams& p, int in_dtype, int out_dtype, cudaStream_t s) {
  using bf = __nv_bfloat16;
  if (in_dtype == GDN_DTYPE_BF16)
    return out_dtype == GDN_DTYPE_BF16 ? launch_u<DK, ROWS, bf, bf>(p, s) : launch_u<DK, ROWS, bf, float>(p, s);
  return out_dtype == GDN_DTYPE_BF16 ? launch_u<DK, ROWS, float, bf>(p, s) : launch_u<DK, ROWS, float, float>(p, s);
}

}  // namespace
}  // namespace gdn

int gdn_launch_recurrent(const gdn_prefill_args* a, const float* s_in, float* s_out, cudaStream_t stream) {
  gdn::RecParams p;
  p.q = a->q; p.k = a->k; p.u = a->u; p.v = a->v;
  p.beta = a->beta; p.la = a->la; p.s_in = s_in; p.s_out = s_out; p.y = a->y;
  p.sq = a->sq; p.sk = a->sk; p.su = a->su; p.sv = a->sv; p.sy = a->sy;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DV = (int)a->DV;
  switch (a->DK) {
    case 32: return gdn::launch_dk<32, 16>(p, a->in_dtype, a->out_dtype, stream);
    case 64: return gdn::launch_dk<64, 16>(p, a->in_dtype, a->out_dtype, stream);
    case 128: return gdn::launch_dk<128, 16>(p, a->in_dtype, a->out_dtype, stream);
    case 256: return gdn::launch_dk<256, 8>(p, a->in_dtype, a->out_dtype, stream);
    default: return GDN_ERR_UNSUPPORTED;
  }
}
