// Backward of the layer prologue and epilogue (gdn_layer_io.cu), so that training runs the fused
// kernels too.  Everything the forward computed is recomputed from its inputs.
//
// Prologue, per (b, t, h) and component (conv weights w, taps TAPS):
//   c_t = sum_j w_j x_{t-(TAPS-1)+j},  s_t = SiLU(c_t);  q = q_scale s / max(|s|, eps), k likewise, v = s.
//   ds = scale / m (dq - [|s| > eps] s^ (s^ . dq)) with m = max(|s|, eps), s^ = s / m (v: ds = dv);
//   dc = ds SiLU'(c);  dx_t = sum_j w_j dc_{t+(TAPS-1)-j};  dw_j = sum_t dc_t x_{t-(TAPS-1)+j};
//   la = -softplus(a + dt_bias) exp(A_log) (zero gradient where clamped at la_min):
//     da = dla (-sigmoid(a + dt_bias) exp(A_log)), ddt_bias = sum da, dA_log = sum dla la;
//   beta = beta_scale sigmoid(b + b_bias): db = dbeta beta_scale sigmoid (1 - sigmoid), db_bias = sum db.
// One block per component (q, k or v), (b, h) and 4 runs of RUN tokens, one warp per run; the run's rows
// of the component (and the conv halo on both sides) are staged in shared memory by cp.async, the next
// token's incoming gradient is loaded while the current one is used; dc of the last TAPS tokens is kept
// in registers, so dx of a token is finished as soon as dc of the TAPS - 1 tokens after it is known.
// Parameter gradients are reduced over the block's warps in shared memory and added to the outputs
// with one atomic add per element and block (fp32; the summation order across blocks is not fixed).
//
// Epilogue, per (b, t, h) over DV: o = y r w SiLU(g), r = (mean(y^2) + eps)^-1/2:
//   z = w SiLU(g) do;  dy = r z - y r^3 mean(y z);  dg = do y r w SiLU'(g);  dw = sum do y r SiLU(g).
#include <math.h>
#include <string.h>

#include "gdn_common.cuh"

namespace gdn {
namespace layer_io_bwd {

constexpr int MAX_TAPS = 4;
constexpr int WARPS = 4;  // warps per prologue block
constexpr int RUN = 16;   // tokens per warp

// Logistic sigmoid with the fast exponential and division, as the forward kernels' SiLU (a few ulps of
// fp32; 0 once 1 + exp(-x) exceeds 2^126, where the exact value is below fp32's normal range): the backward passes
// are bound by their per-element instruction count.
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float dsilu(float c) {
  const float s = sigm(c);
  return s * (1.f + c * (1.f - s));
}

template <typename TO, int N>
__device__ __forceinline__ void stv(TO* p, const float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) store_as(p + i, v[i]);
}

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

struct CompB {             // one of q, k, v
  const void* x;           // projection [B][T][channels] with strides
  int64_t sb, st;
  const float* w;          // (taps, channels) fp32 or NULL
  int64_t wch;
  const void* g;           // incoming gradient [B][T][H][D] contiguous (grad dtype)
  void* dx;                // projection gradient, strides dsb, dst (projection dtype)
  int64_t dsb, dst;
  float* dw;               // (taps, channels) fp32 accumulated, or NULL
};

struct ProBwdParams {
  CompB q, k, v;
  const void* xa;
  const void* xb;
  int64_t sa_b, sa_t, sb_b, sb_t;
  void* dxa;
  void* dxb;
  int64_t dsa_b, dsa_t, dsb_b, dsb_t;
  const float* dla;
  const float* dbeta;
  const float* A_log;
  const float* dt_bias;
  const float* b_bias;
  float* dA_log;
  float* ddt_bias;
  float* db_bias;
  int B, T, H, DK, DV, clamp;
  float q_scale, eps, la_min, beta_scale;
};

// One component of one lane: dc window (last TAPS tokens), conv-weight gradient accumulators.
template <int TAPS, int NPL>
struct Lane {
  float win[TAPS][NPL];  // win[j] = dc of token t - (TAPS - 1) + j after the latest push
  float dw[TAPS][NPL];
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int j = 0; j < TAPS; ++j)
#pragma unroll
      for (int n = 0; n < NPL; ++n) win[j][n] = dw[j][n] = 0.f;
  }
  __device__ __forceinline__ void push(const float (&dc)[NPL]) {
#pragma unroll
    for (int j = 0; j + 1 < TAPS; ++j)
#pragma unroll
      for (int n = 0; n < NPL; ++n) win[j][n] = win[j + 1][n];
#pragma unroll
    for (int n = 0; n < NPL; ++n) win[TAPS - 1][n] = dc[n];
  }
};

// dx of the token TAPS - 1 before the latest push: sum_j w_j dc_{tau + (TAPS-1) - j} = sum_j w_j win[TAPS-1-j].
template <int TAPS, int NPL>
__device__ __forceinline__ void dx_of(const Lane<TAPS, NPL>& L, const float* w, int wld, bool has_w, float (&o)[NPL]) {
  if (has_w) {
#pragma unroll
    for (int n = 0; n < NPL; ++n) o[n] = 0.f;
#pragma unroll
    for (int j = 0; j < TAPS; ++j) {
      float wj[NPL];
      load_vec<NPL>(w + j * wld, wj);
#pragma unroll
      for (int n = 0; n < NPL; ++n) o[n] = fmaf(wj[n], L.win[TAPS - 1 - j][n], o[n]);
    }
  } else {
#pragma unroll
    for (int n = 0; n < NPL; ++n) o[n] = L.win[0][n];
  }
}

// One component (q, k or v: blockIdx.y) of one (b, h) and WARPS runs of RUN tokens per block, one run per
// warp; the v blocks also do the gates.
template <typename TX, typename TG, int NPL, bool NORM, int TAPS>
__device__ __forceinline__ void prologue_bwd_comp(const ProBwdParams& p, const CompB& cp, float scale, bool gates,
                                                  float* sw) {
  constexpr int D = 32 * NPL;
  constexpr int NROWS = RUN + 2 * (TAPS - 1);  // staged tokens t0 - (TAPS - 1) .. t1 + TAPS - 2
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int runs = (p.T + RUN - 1) / RUN, rgroups = (runs + WARPS - 1) / WARPS;
  const int bh = blockIdx.x / rgroups, rg = blockIdx.x - bh * rgroups;
  const int b = bh / p.H, h = bh - b * p.H;
  const bool has_w = cp.w != nullptr;
  if (has_w)
    for (int i = threadIdx.x; i < TAPS * D; i += blockDim.x) {
      const int j = i / D, ch = i - j * D;
      sw[i] = cp.w[(int64_t)j * cp.wch + (int64_t)h * D + ch];
    }
  TX* stage = reinterpret_cast<TX*>(sw + TAPS * D) + (size_t)wid * NROWS * D;
  __syncthreads();
  const int run = rg * WARPS + wid;
  const bool active = run < runs;
  const int t0 = run * RUN, t1 = active ? min(p.T, t0 + RUN) : t0;
  const int tend = min(p.T, t1 + TAPS - 1);  // dc is needed for tokens t0 .. tend - 1
  constexpr int EPC = 16 / sizeof(TX), CHUNKS = D / EPC;
  if (active) {
    const int nrows = tend - t0 + TAPS - 1, hc = h * D;
    for (int i = lane; i < nrows * CHUNKS; i += 32) {
      const int r = i / CHUNKS, q = i - r * CHUNKS, t = t0 - (TAPS - 1) + r;
      TX* dst = stage + (size_t)r * D + q * EPC;
      if (t >= 0) {
        cp16(dst, reinterpret_cast<const TX*>(cp.x) + (int64_t)b * cp.sb + (int64_t)t * cp.st + hc + q * EPC);
      } else {
#pragma unroll
        for (int e = 0; e < EPC; ++e) store_as(dst + e, 0.f);  // training calls start from zero history
      }
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  Lane<TAPS, NPL> L;
  L.clear();
  const int64_t tokb = ((int64_t)b * p.T) * p.H + h;  // token (b, 0, h)
  const float* wl = sw + lane * NPL;
  if (active) {
    // the next token's incoming gradient is loaded while this token's is used
    float gnext[NPL];
    load_vec<NPL>(reinterpret_cast<const TG*>(cp.g) + (tokb + (int64_t)t0 * p.H) * D + lane * NPL, gnext);
#pragma unroll 1
    for (int t = t0; t <= t1 + TAPS - 2; ++t) {
      float dc[NPL];
      if (t < tend) {
        float g[NPL];
#pragma unroll
        for (int n = 0; n < NPL; ++n) g[n] = gnext[n];
        if (t + 1 < tend)
          load_vec<NPL>(reinterpret_cast<const TG*>(cp.g) + (tokb + (int64_t)(t + 1) * p.H) * D + lane * NPL, gnext);
        const TX* rows = stage + (size_t)(t - t0) * D + lane * NPL;
        float c[NPL], xs[TAPS][NPL];
#pragma unroll
        for (int j = 0; j < TAPS; ++j) load_vec<NPL>(rows + j * D, xs[j]);
        if (has_w) {
#pragma unroll
          for (int n = 0; n < NPL; ++n) c[n] = 0.f;
#pragma unroll
          for (int j = 0; j < TAPS; ++j) {
            float wj[NPL];
            load_vec<NPL>(wl + j * D, wj);
#pragma unroll
            for (int n = 0; n < NPL; ++n) c[n] = fmaf(wj[n], xs[j][n], c[n]);
          }
        } else {
#pragma unroll
          for (int n = 0; n < NPL; ++n) c[n] = xs[TAPS - 1][n];
        }
        float sg_[NPL], s[NPL];
#pragma unroll
        for (int n = 0; n < NPL; ++n) {
          sg_[n] = sigm(c[n]);
          s[n] = c[n] * sg_[n];
        }
        if (NORM) {
          float ss = 0.f, sgd = 0.f;
#pragma unroll
          for (int n = 0; n < NPL; ++n) {
            ss = fmaf(s[n], s[n], ss);
            sgd = fmaf(s[n], g[n], sgd);
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
            sgd += __shfl_xor_sync(0xffffffffu, sgd, o);
          }
          const float nrm = sqrtf(ss), m = fmaxf(nrm, p.eps), inv = 1.f / m;
          const float proj = nrm > p.eps ? sgd * inv * inv : 0.f;
#pragma unroll
          for (int n = 0; n < NPL; ++n) g[n] = scale * inv * (g[n] - s[n] * proj);
        }
#pragma unroll
        for (int n = 0; n < NPL; ++n) dc[n] = g[n] * (sg_[n] * (1.f + c[n] * (1.f - sg_[n])));
        if (t < t1) {  // conv-weight gradient of this run's tokens
#pragma unroll
          for (int j = 0; j < TAPS; ++j)
#pragma unroll
            for (int n = 0; n < NPL; ++n) L.dw[j][n] = fmaf(dc[n], xs[j][n], L.dw[j][n]);
        }
      } else {
#pragma unroll
        for (int n = 0; n < NPL; ++n) dc[n] = 0.f;
      }
      L.push(dc);
      const int tau = t - (TAPS - 1);
      if (tau >= t0) {
        float o[NPL];
        dx_of<TAPS, NPL>(L, wl, D, has_w, o);
        stv<TX, NPL>(reinterpret_cast<TX*>(cp.dx) + (int64_t)b * cp.dsb + (int64_t)tau * cp.dst + h * D + lane * NPL, o);
      }
    }
  }
  if (gates) {  // one token per lane; parameter gradients summed over the warp
    float s_dt = 0.f, s_al = 0.f, s_bb = 0.f;
    if (active) {
      const float dtb = p.dt_bias[h], Ae = expf(p.A_log[h]), bb_h = p.b_bias ? p.b_bias[h] : 0.f;
      for (int t = t0 + lane; t < t1; t += 32) {
        const int64_t tok = tokb + (int64_t)t * p.H;
        const float a = to_f32(reinterpret_cast<const TX*>(p.xa)[(int64_t)b * p.sa_b + (int64_t)t * p.sa_t + h]);
        const float bb = to_f32(reinterpret_cast<const TX*>(p.xb)[(int64_t)b * p.sb_b + (int64_t)t * p.sb_t + h]);
        const float z = a + dtb, la = -softplus(z) * Ae, gl = p.dla[tok];
        const bool live = !(p.clamp && la < p.la_min);
        const float dz = live ? gl * (-sigm(z) * Ae) : 0.f;
        s_dt += dz;
        s_al += live ? gl * la : 0.f;
        const float sb = sigm(bb + bb_h), dzb = p.dbeta[tok] * p.beta_scale * sb * (1.f - sb);
        s_bb += dzb;
        store_as(reinterpret_cast<TX*>(p.dxa) + (int64_t)b * p.dsa_b + (int64_t)t * p.dsa_t + h, dz);
        store_as(reinterpret_cast<TX*>(p.dxb) + (int64_t)b * p.dsb_b + (int64_t)t * p.dsb_t + h, dzb);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s_dt += __shfl_xor_sync(0xffffffffu, s_dt, o);
      s_al += __shfl_xor_sync(0xffffffffu, s_al, o);
      s_bb += __shfl_xor_sync(0xffffffffu, s_bb, o);
    }
    if (lane == 0 && active) {
      atomicAdd(p.ddt_bias + h, s_dt);
      atomicAdd(p.dA_log + h, s_al);
      if (p.db_bias) atomicAdd(p.db_bias + h, s_bb);
    }
  }
  // conv-weight gradient: the block's warps summed in shared memory, one atomic per element
  if (!has_w) return;
  __syncthreads();  // every warp is done with its staged rows
  float* red = sw + TAPS * D;  // WARPS x TAPS x D floats fit in the staging area
#pragma unroll
  for (int j = 0; j < TAPS; ++j)
#pragma unroll
    for (int n = 0; n < NPL; ++n) red[((size_t)wid * TAPS + j) * D + lane * NPL + n] = L.dw[j][n];
  __syncthreads();
  for (int i = threadIdx.x; i < TAPS * D; i += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) v += red[(size_t)w * TAPS * D + i];
    const int j = i / D, ch = i - j * D;
    atomicAdd(cp.dw + (int64_t)j * cp.wch + (int64_t)h * D + ch, v);
  }
}

template <typename TX, typename TG, int NK, int NV, int TAPS>
__global__ void __launch_bounds__(32 * WARPS) prologue_bwd_kernel(const ProBwdParams p) {
  extern __shared__ __align__(16) float sw[];  // this component's weights (TAPS x D), then staged rows per warp
  switch (blockIdx.y) {
    case 0: prologue_bwd_comp<TX, TG, NK, true, TAPS>(p, p.q, p.q_scale, false, sw); break;
    case 1: prologue_bwd_comp<TX, TG, NK, true, TAPS>(p, p.k, 1.f, false, sw); break;
    default: prologue_bwd_comp<TX, TG, NV, false, TAPS>(p, p.v, 1.f, true, sw); break;
  }
}

// ---- epilogue backward ------------------------------------------------------------------------------
struct EpiBwdParams {
  const void* y;
  gdn_strides sy;
  const void* g;
  int64_t sg_b, sg_t;
  const float* weight;
  const void* dout;
  int64_t sdo_b, sdo_t;
  void* dy;   // [B][T][H][DV] contiguous
  void* dg;   // [B][T][H*DV], strides sdg_b, sdg_t
  int64_t sdg_b, sdg_t;
  float* dweight;
  int B, T, H, DV;
  float eps;
};

template <typename TY, typename TG, typename TD, int NPL>
__global__ void __launch_bounds__(128) epilogue_bwd_kernel(const EpiBwdParams p) {
  const int lane = threadIdx.x & 31;
  const unsigned rows = (unsigned)p.B * (unsigned)p.T * (unsigned)p.H;
  const int c0 = lane * NPL;
  float w[NPL], dw[NPL];
  load_vec<NPL>(p.weight + c0, w);
#pragma unroll
  for (int n = 0; n < NPL; ++n) dw[n] = 0.f;
  const unsigned warps = gridDim.x * (blockDim.x >> 5);
  for (unsigned row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const unsigned bt = row / (unsigned)p.H;
    const int h = (int)(row - bt * (unsigned)p.H);
    const int b = (int)(bt / (unsigned)p.T), t = (int)(bt - (unsigned)b * (unsigned)p.T);
    float y[NPL], d[NPL], g[NPL], s[NPL];
    load_vec<NPL>(reinterpret_cast<const TY*>(p.y) + b * p.sy.b + t * p.sy.t + h * p.sy.h + c0, y);
    load_vec<NPL>(reinterpret_cast<const TD*>(p.dout) + b * p.sdo_b + t * p.sdo_t + (int64_t)h * p.DV + c0, d);
    if (p.g) {
      load_vec<NPL>(reinterpret_cast<const TG*>(p.g) + b * p.sg_b + t * p.sg_t + (int64_t)h * p.DV + c0, g);
#pragma unroll
      for (int n = 0; n < NPL; ++n) s[n] = g[n] * sigm(g[n]);
    } else {
#pragma unroll
      for (int n = 0; n < NPL; ++n) s[n] = 1.f;
    }
    float ss = 0.f, yz = 0.f, z[NPL];
#pragma unroll
    for (int n = 0; n < NPL; ++n) {
      z[n] = w[n] * s[n] * d[n];
      ss = fmaf(y[n], y[n], ss);
      yz = fmaf(y[n], z[n], yz);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      yz += __shfl_xor_sync(0xffffffffu, yz, o);
    }
    const float r = rsqrtf(ss / (float)p.DV + p.eps), k3 = r * r * r * yz / (float)p.DV;
    float oy[NPL], og[NPL];
#pragma unroll
    for (int n = 0; n < NPL; ++n) {
      oy[n] = r * z[n] - y[n] * k3;
      dw[n] = fmaf(d[n] * y[n] * r, s[n], dw[n]);
      og[n] = p.g ? d[n] * y[n] * r * w[n] * dsilu(g[n]) : 0.f;
    }
    const int64_t tok = ((int64_t)b * p.T + t) * p.H + h;
    stv<TY, NPL>(reinterpret_cast<TY*>(p.dy) + tok * p.DV + c0, oy);
    if (p.g) stv<TG, NPL>(reinterpret_cast<TG*>(p.dg) + b * p.sdg_b + t * p.sdg_t + (int64_t)h * p.DV + c0, og);
  }
  __shared__ float red[4][512];
  const int wid = threadIdx.x >> 5;
#pragma unroll
  for (int n = 0; n < NPL; ++n) red[wid][c0 + n] = dw[n];
  __syncthreads();
  for (int i = threadIdx.x; i < p.DV; i += blockDim.x)
    atomicAdd(p.dweight + i, (red[0][i] + red[1][i]) + (red[2][i] + red[3][i]));
}

bool a16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

bool device_ok() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

template <typename TX, typename TG, int NK, int NV, int TAPS>
int launch_pro(const ProBwdParams& p, cudaStream_t s) {
  constexpr int D = 32 * (NK > NV ? NK : NV);
  const size_t stage = (size_t)WARPS * (RUN + 2 * (TAPS - 1)) * D * sizeof(TX);
  const size_t red = (size_t)WARPS * TAPS * D * sizeof(float);
  const size_t sm = (size_t)TAPS * D * 4 + (stage > red ? stage : red);
  if (sm > 100 * 1024) return GDN_ERR_UNSUPPORTED;
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)prologue_bwd_kernel<TX, TG, NK, NV, TAPS>, 100 * 1024}}))
    return GDN_ERR_LAUNCH;
  const int64_t runs = (p.T + RUN - 1) / RUN;
  const int64_t blocks = (int64_t)p.B * p.H * ((runs + WARPS - 1) / WARPS);
  if (blocks > 0x7fffffff) return GDN_ERR_SHAPE;
  prologue_bwd_kernel<TX, TG, NK, NV, TAPS><<<dim3((unsigned)blocks, 3), 32 * WARPS, sm, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

template <typename TX, typename TG, int NK, int NV>
int launch_pro_taps(const ProBwdParams& p, int taps, cudaStream_t s) {
  switch (taps) {
    case 1: return launch_pro<TX, TG, NK, NV, 1>(p, s);
    case 2: return launch_pro<TX, TG, NK, NV, 2>(p, s);
    case 3: return launch_pro<TX, TG, NK, NV, 3>(p, s);
    case 4: return launch_pro<TX, TG, NK, NV, 4>(p, s);
    default: return GDN_ERR_SHAPE;
  }
}

template <typename TX, typename TG>
int launch_pro_dims(const ProBwdParams& p, int taps, cudaStream_t s) {
  const int nk = p.DK / 32, nv = p.DV / 32;
  if (nk == 4 && nv == 4) return launch_pro_taps<TX, TG, 4, 4>(p, taps, s);
  if (nk == 4 && nv == 8) return launch_pro_taps<TX, TG, 4, 8>(p, taps, s);
  if (nk == 2 && nv == 2) return launch_pro_taps<TX, TG, 2, 2>(p, taps, s);
  if (nk == 2 && nv == 4) return launch_pro_taps<TX, TG, 2, 4>(p, taps, s);
  return GDN_ERR_UNSUPPORTED;
}

template <typename TY, typename TG, typename TD>
int launch_epi(const EpiBwdParams& p, cudaStream_t s) {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t rows = (int64_t)p.B * p.T * p.H;
  int64_t blocks = (rows + 3) / 4;
  if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
  switch (p.DV / 32) {
    case 2: epilogue_bwd_kernel<TY, TG, TD, 2><<<(unsigned)blocks, 128, 0, s>>>(p); break;
    case 4: epilogue_bwd_kernel<TY, TG, TD, 4><<<(unsigned)blocks, 128, 0, s>>>(p); break;
    case 8: epilogue_bwd_kernel<TY, TG, TD, 8><<<(unsigned)blocks, 128, 0, s>>>(p); break;
    case 16: epilogue_bwd_kernel<TY, TG, TD, 16><<<(unsigned)blocks, 128, 0, s>>>(p); break;
    default: return GDN_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------
// Backward of nsgdn's n-step write vectors (archbench/layers/nsgdn.py:61-75), per (b, t, h) with
// p = k_{t-1} (zero at t = 0):
//   c = p.k,  pp = p - c k,  u_0 = beta k,  s_i = p.u_{i-1},  u_i = u_{i-1} - lam beta s_i pp  (0 < i < n).
// From g = du_{n-1}, for i = n-1 .. 1 with e = pp.g:
//   dpp -= lam beta s_i g;  dp -= lam beta e u_{i-1};  dlam -= beta s_i e;  dbeta -= lam s_i e;
//   g <- g - lam beta e p   (= du_{i-1});
// then dbeta += k.g, dc = -k.dpp, dk_t += beta g - c dpp + dc p and dp += dpp + dc k, which is token
// t-1's share of dk.  One warp per (b, h) and run of WV_RUN tokens, walking the run backwards so that
// each token's dp is in registers when the token before it is finished; the token after the run is
// recomputed for its dp.  Each lane holds DK/32 consecutive channels; the forward is recomputed in
// registers (n <= 8).  dlam: one fp32 atomic per run (summation order across runs not fixed).
constexpr int WV_RUN = 16;
constexpr int WV_MAXN = 8;

struct WvParams {
  const void* k;
  const float* beta;
  const float* lam;
  const float* du;
  float* dk;
  float* dbeta;
  float* dlam;
  int B, T, H, n_steps;
};

__device__ __forceinline__ float wv_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename TK, int NK>
__device__ __forceinline__ void wv_token(const WvParams& p, int b, int t, int h, int lane, float lam, float (&dks)[NK],
                                         float (&dp)[NK], float& dbeta, float& dlam) {
  const int64_t row = ((int64_t)b * p.T + t) * p.H + h;
  const TK* kb = static_cast<const TK*>(p.k);
  float k[NK], pv[NK], g[NK], pp[NK], dpp[NK];
  load_vec<NK>(kb + row * (NK * 32) + lane * NK, k);
  if (t > 0) {
    load_vec<NK>(kb + (row - p.H) * (NK * 32) + lane * NK, pv);
  } else {
#pragma unroll
    for (int i = 0; i < NK; ++i) pv[i] = 0.f;
  }
  load_vec<NK>(p.du + row * (NK * 32) + lane * NK, g);
  const float beta = p.beta[row], lb = lam * beta;
  float c = 0.f;
#pragma unroll
  for (int i = 0; i < NK; ++i) c = fmaf(pv[i], k[i], c);
  c = wv_sum(c);
  float u[WV_MAXN][NK], s[WV_MAXN];
#pragma unroll
  for (int i = 0; i < NK; ++i) {
    pp[i] = pv[i] - c * k[i];
    u[0][i] = beta * k[i];
    dpp[i] = 0.f;
    dp[i] = 0.f;
  }
  s[0] = 0.f;
#pragma unroll
  for (int j = 1; j < WV_MAXN; ++j) {
    s[j] = 0.f;
    if (j < p.n_steps) {
      float sj = 0.f;
#pragma unroll
      for (int i = 0; i < NK; ++i) sj = fmaf(pv[i], u[j - 1][i], sj);
      sj = wv_sum(sj);
      s[j] = sj;
#pragma unroll
      for (int i = 0; i < NK; ++i) u[j][i] = u[j - 1][i] - lb * sj * pp[i];
    }
  }
  dbeta = 0.f;
  dlam = 0.f;
#pragma unroll
  for (int j = WV_MAXN - 1; j >= 1; --j) {
    if (j < p.n_steps) {
      float e = 0.f;
#pragma unroll
      for (int i = 0; i < NK; ++i) e = fmaf(pp[i], g[i], e);
      e = wv_sum(e);
      const float sj = s[j];
#pragma unroll
      for (int i = 0; i < NK; ++i) {
        dpp[i] -= lb * sj * g[i];
        dp[i] -= lb * e * u[j - 1][i];
        g[i] -= lb * e * pv[i];
      }
      dlam -= beta * sj * e;
      dbeta -= lam * sj * e;
    }
  }
  float kg = 0.f, kd = 0.f;
#pragma unroll
  for (int i = 0; i < NK; ++i) {
    kg = fmaf(k[i], g[i], kg);
    kd = fmaf(k[i], dpp[i], kd);
  }
  kg = wv_sum(kg);
  const float dc = -wv_sum(kd);
  dbeta += kg;
#pragma unroll
  for (int i = 0; i < NK; ++i) {
    dks[i] = beta * g[i] - c * dpp[i] + dc * pv[i];
    dp[i] += dpp[i] + dc * k[i];
  }
}

template <typename TK, int NK>
__global__ void __launch_bounds__(128) write_vectors_bwd_kernel(const WvParams p) {
  const int lane = threadIdx.x & 31;
  const int nrun = (p.T + WV_RUN - 1) / WV_RUN;
  const int64_t w = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (w >= (int64_t)p.B * p.H * nrun) return;  // whole warps leave together
  const int r = (int)(w % nrun);
  const int64_t bh = w / nrun;
  const int h = (int)(bh % p.H), b = (int)(bh / p.H);
  const float lam = p.lam[h];
  const int t0 = r * WV_RUN, t1 = min(p.T, t0 + WV_RUN);
  float dks[NK], dp[NK], dp_next[NK], db, dl, dl_run = 0.f;
#pragma unroll
  for (int i = 0; i < NK; ++i) dp_next[i] = 0.f;
  if (t1 < p.T) wv_token<TK, NK>(p, b, t1, h, lane, lam, dks, dp_next, db, dl);  // only its dp is used
#pragma unroll 1
  for (int t = t1 - 1; t >= t0; --t) {
    wv_token<TK, NK>(p, b, t, h, lane, lam, dks, dp, db, dl);
    const int64_t row = ((int64_t)b * p.T + t) * p.H + h;
    float* dkr = p.dk + row * (NK * 32) + lane * NK;
    float cur[NK];
    load_vec<NK>(dkr, cur);
#pragma unroll
    for (int i = 0; i < NK; ++i) {
      dkr[i] = cur[i] + dks[i] + dp_next[i];
      dp_next[i] = dp[i];
    }
    if (lane == 0) p.dbeta[row] = db;
    dl_run += dl;
  }
  if (lane == 0) atomicAdd(p.dlam + h, dl_run);
}

}  // namespace layer_io_bwd
}  // namespace gdn

using namespace gdn::layer_io_bwd;

extern "C" {

int gdn_layer_prologue_bwd(const gdn_prologue_bwd_args* a, void* stream) {
  if (!a) return GDN_ERR_NULL;
  if (!a->xq || !a->xk || !a->xv || !a->xa || !a->xb || !a->A_log || !a->dt_bias || !a->dq || !a->dk || !a->dv ||
      !a->dla || !a->dbeta || !a->dxq || !a->dxk || !a->dxv || !a->dxa || !a->dxb || !a->dA_log || !a->ddt_bias)
    return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->H < 1 || a->B * a->T * a->H > (int64_t)1 << 31) return GDN_ERR_SHAPE;
  if (a->conv_size < 1 || a->conv_size > MAX_TAPS) return GDN_ERR_SHAPE;
  if ((a->wq != nullptr) != (a->dwq != nullptr) || (a->wk != nullptr) != (a->dwk != nullptr) ||
      (a->wv != nullptr) != (a->dwv != nullptr))
    return GDN_ERR_NULL;
  if (a->in_dtype != GDN_DTYPE_BF16 && a->in_dtype != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  if (a->grad_dtype != GDN_DTYPE_BF16 && a->grad_dtype != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  const int64_t es = a->in_dtype == GDN_DTYPE_BF16 ? 2 : 4;
  const int64_t sts[] = {a->sxq_b, a->sxq_t, a->sxk_b, a->sxk_t, a->sxv_b, a->sxv_t};
  for (int64_t st : sts)
    if ((st * es) % 16) return GDN_ERR_ALIGN;
  if (!a16(a->xq) || !a16(a->xk) || !a16(a->xv) || !a16(a->dq) || !a16(a->dk) || !a16(a->dv)) return GDN_ERR_ALIGN;
  if (!device_ok()) return GDN_ERR_DEVICE;
  ProBwdParams p;
  memset(&p, 0, sizeof(p));
  p.q = {a->xq, a->sxq_b, a->sxq_t, a->wq, a->H * a->DK, a->dq, a->dxq, a->sdxq_b, a->sdxq_t, a->dwq};
  p.k = {a->xk, a->sxk_b, a->sxk_t, a->wk, a->H * a->DK, a->dk, a->dxk, a->sdxk_b, a->sdxk_t, a->dwk};
  p.v = {a->xv, a->sxv_b, a->sxv_t, a->wv, a->H * a->DV, a->dv, a->dxv, a->sdxv_b, a->sdxv_t, a->dwv};
  p.xa = a->xa; p.xb = a->xb;
  p.sa_b = a->sxa_b; p.sa_t = a->sxa_t; p.sb_b = a->sxb_b; p.sb_t = a->sxb_t;
  p.dxa = a->dxa; p.dxb = a->dxb;
  p.dsa_b = a->sdxa_b; p.dsa_t = a->sdxa_t; p.dsb_b = a->sdxb_b; p.dsb_t = a->sdxb_t;
  p.dla = a->dla; p.dbeta = a->dbeta;
  p.A_log = a->A_log; p.dt_bias = a->dt_bias; p.b_bias = a->b_bias;
  p.dA_log = a->dA_log; p.ddt_bias = a->ddt_bias; p.db_bias = a->db_bias;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DK = (int)a->DK; p.DV = (int)a->DV;
  p.clamp = (a->flags & GDN_PROLOGUE_CLAMP_LA) != 0;
  p.q_scale = a->q_scale; p.eps = a->l2_eps; p.la_min = a->la_min; p.beta_scale = a->beta_scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // parameter gradients accumulate atomically: start from zero
  const size_t tb = (size_t)a->conv_size * 4;
  if ((a->dwq && cudaMemsetAsync(a->dwq, 0, tb * a->H * a->DK, s) != cudaSuccess) ||
      (a->dwk && cudaMemsetAsync(a->dwk, 0, tb * a->H * a->DK, s) != cudaSuccess) ||
      (a->dwv && cudaMemsetAsync(a->dwv, 0, tb * a->H * a->DV, s) != cudaSuccess) ||
      cudaMemsetAsync(a->dA_log, 0, a->H * 4, s) != cudaSuccess || cudaMemsetAsync(a->ddt_bias, 0, a->H * 4, s) != cudaSuccess ||
      (a->db_bias && cudaMemsetAsync(a->db_bias, 0, a->H * 4, s) != cudaSuccess))
    return GDN_ERR_LAUNCH;
  using bf = __nv_bfloat16;
  const bool xb = a->in_dtype == GDN_DTYPE_BF16, gb = a->grad_dtype == GDN_DTYPE_BF16;
  if (xb && gb) return launch_pro_dims<bf, bf>(p, a->conv_size, s);
  if (xb) return launch_pro_dims<bf, float>(p, a->conv_size, s);
  if (gb) return launch_pro_dims<float, bf>(p, a->conv_size, s);
  return launch_pro_dims<float, float>(p, a->conv_size, s);
}

int gdn_layer_epilogue_bwd(const gdn_epilogue_bwd_args* a, void* stream) {
  if (!a) return GDN_ERR_NULL;
  if (!a->y || !a->weight || !a->dout || !a->dy || !a->dweight || (a->g && !a->dg)) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->H < 1 || (a->DV != 64 && a->DV != 128 && a->DV != 256 && a->DV != 512)) return GDN_ERR_SHAPE;
  if (a->B * a->T * a->H * 32 > 0x7fffffffLL) return GDN_ERR_SHAPE;
  for (int32_t dt : {a->y_dtype, a->g_dtype, a->do_dtype})
    if (dt != GDN_DTYPE_BF16 && dt != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  if (!a16(a->y) || (a->g && !a16(a->g)) || !a16(a->dout)) return GDN_ERR_ALIGN;
  if (!device_ok()) return GDN_ERR_DEVICE;
  EpiBwdParams p;
  p.y = a->y; p.sy = a->sy; p.g = a->g; p.sg_b = a->sg_b; p.sg_t = a->sg_t; p.weight = a->weight;
  p.dout = a->dout; p.sdo_b = a->sdo_b; p.sdo_t = a->sdo_t; p.dy = a->dy; p.dg = a->dg; p.dweight = a->dweight;
  p.sdg_b = a->sdg_b; p.sdg_t = a->sdg_t;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DV = (int)a->DV; p.eps = a->eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(a->dweight, 0, a->DV * 4, s) != cudaSuccess) return GDN_ERR_LAUNCH;
  using bf = __nv_bfloat16;
  const int key = a->y_dtype * 4 + a->g_dtype * 2 + a->do_dtype;  // F32 = 0, BF16 = 1
  switch (key) {
    case 7: return launch_epi<bf, bf, bf>(p, s);
    case 6: return launch_epi<bf, bf, float>(p, s);
    case 3: return launch_epi<float, bf, bf>(p, s);
    case 2: return launch_epi<float, bf, float>(p, s);
    case 5: return launch_epi<bf, float, bf>(p, s);
    case 4: return launch_epi<bf, float, float>(p, s);
    case 1: return launch_epi<float, float, bf>(p, s);
    default: return launch_epi<float, float, float>(p, s);
  }
}

int gdn_write_vectors_bwd(const gdn_write_vectors_bwd_args* a, void* stream) {
  if (!a) return GDN_ERR_NULL;
  if (!a->k || !a->beta || !a->lam || !a->du || !a->dk || !a->dbeta || !a->dlam) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->H < 1 || (a->DK != 64 && a->DK != 128) || a->n_steps < 2 || a->n_steps > WV_MAXN)
    return GDN_ERR_SHAPE;
  if (a->B * a->T * a->H > 0x3fffffffLL) return GDN_ERR_SHAPE;
  if (a->k_dtype != GDN_DTYPE_BF16 && a->k_dtype != GDN_DTYPE_F32) return GDN_ERR_DTYPE;
  if (!a16(a->k) || !a16(a->du) || !a16(a->dk)) return GDN_ERR_ALIGN;
  if (!device_ok()) return GDN_ERR_DEVICE;
  WvParams p;
  p.k = a->k; p.beta = a->beta; p.lam = a->lam; p.du = a->du; p.dk = a->dk; p.dbeta = a->dbeta; p.dlam = a->dlam;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.n_steps = a->n_steps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(a->dlam, 0, a->H * 4, s) != cudaSuccess) return GDN_ERR_LAUNCH;
  const int64_t warps = a->B * a->H * ((a->T + WV_RUN - 1) / WV_RUN);
  const unsigned blocks = (unsigned)((warps + 3) / 4);
  using bf = __nv_bfloat16;
  const bool kb = a->k_dtype == GDN_DTYPE_BF16;
  if (a->DK == 128) {
    if (kb) write_vectors_bwd_kernel<bf, 4><<<blocks, 128, 0, s>>>(p);
    else write_vectors_bwd_kernel<float, 4><<<blocks, 128, 0, s>>>(p);
  } else {
    if (kb) write_vectors_bwd_kernel<bf, 2><<<blocks, 128, 0, s>>>(p);
    else write_vectors_bwd_kernel<float, 2><<<blocks, 128, 0, s>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // extern "C"
