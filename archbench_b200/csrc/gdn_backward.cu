// Chunked backward of the gated delta rule (the training path), sm_100a.
//
// Forward, per (b, h) and 64-token chunk, state S (DV x DK) entering the chunk as S0 (the WY form of
// archbench/layers/nsgdn.py:240-249, with g the chunk-local cumsum of la, gamma = exp(g),
// d_j = exp(g_C - g_j), E_tj = exp(g_t - g_j)):
//
//   L = strict_tril(K U^T o E),  T = (I + L)^-1,  W = T Gamma K,  Uw = T V,  A = tril(Q U^T o E)
//   R = Uw - W S0^T,  Y = Gamma Q S0^T + A R,  S1 = gamma_C S0 + R^T diag(d) U
//
// Backward for incoming dY and dS1 (the gradient of the state leaving the chunk):
//
//   dR  = A^T dY + diag(d) U dS1^T                  dS0 = gamma_C dS1 + dY^T Gamma Q - dR^T W
//   dA  = tril(dY R^T)                              dQ  = Gamma dY S0 + (dA o E) U
//   dW  = -dR S0,  dT = dW (Gamma K)^T + dR V^T     dL  = strict_tril(-T^T dT T^T)
//   dK  = Gamma T^T dW + (dL o E) U                 dU  = diag(d) R dS1 + (dA o E)^T Q + (dL o E)^T K
//   dV  = T^T dR                                    dg  from every exp(.) factor, dla = reverse cumsum of dg
//
// The state and its gradient cross chunks, so the work splits in four launches:
//   amax_kernel   (one block per chunk): the largest |dY| (and |dS_T|) of every (b, h).
//   prep_kernel   (one block per chunk, all chunks in parallel): g, T, W, Uw, A into the workspace, the
//                 fp16 operands the chains stream (U, d U) and the backward chain's dS-independent terms
//                 A^T dY and dY^T Gamma Q (dY times the gradient scale).
//   chain_kernel  (two blocks per (b, h)): one walks the chunks forwards and records S0 of every chunk,
//                 the other walks them backwards and records dS1 of every chunk; each warp owns 16
//                 state rows as mma accumulators (rows of S are independent in both chains).
//   local_kernel  (one block per chunk, in parallel): every gradient of the chunk from S0, dS1 and the
//                 prep products.
// The reference computes the same quantities with fla's chunk kernels (nsgdn.py:369-397) and its own
// WY backward (nsgdn.py:274-330); the decomposition above and its kernels are this library's own.
//
// Products run on the warp-level tensor-core path (mma.sync m16n8k16, fp16 operands staged in shared
// memory, fp32 accumulation).  The backward is linear in (dY, dS_T), so both are multiplied by a power
// of two per (b, h) that brings max|dY|, max|dS_T| into [0.5, 1) before they meet fp16, and every
// gradient is divided by it at the end: small training gradients keep full fp16 precision.
#include <math.h>

#include "gdn_common.cuh"
#include "gdn_tiles.cuh"
#include "sm100_ptx.cuh"

namespace gdn {
namespace bwd {

constexpr int C = 64;          // tokens per chunk
constexpr int D = 128;         // DK = DV
constexpr int LDT = D + 8;     // halves per row of C x 128 and 128 x 128 tiles (272-byte rows)
constexpr int LDC = C + 8;     // halves per row of C x C tiles (144-byte rows)
constexpr int NTHR = 256;
constexpr int TILE_CD = C * LDT;
constexpr int TILE_DD = D * LDT;
constexpr int TILE_CC = C * LDC;

struct Params {
  const void *q, *k, *u, *v, *dy;
  const float *beta, *la, *s0, *dsT;
  float *dq, *dk, *du, *dv, *dbeta, *dla, *ds0;
  int64_t sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, su_b, su_t, su_h, sv_b, sv_t, sv_h, sd_b, sd_t, sd_h;
  int T, H, NC, BH;
  int DVt, vofs, accum;  // total DV; first state row of this 128-row slice; add dq/dk/du/dla/dbeta to the outputs
  int pf;                 // prep: chunks between a block and the one whose tiles it prefetches into L2 (0: none)
  __half *wT, *wA, *wW, *wUw, *wS, *wdS;  // per chunk: T, A (C x C), W, Uw (C x D), S0, dS1 (D x D)
  __half *wU, *wDU, *wdY, *wdR0;         // per chunk: U, d U, scaled dY, A^T dY (C x D)
  __half* wPc;                            // per chunk: dY^T Gamma Q (D x D)
  float* wg;                              // per chunk: g (C)
  unsigned* amax;                         // per (b, h): max |dY| as float bits
  float* scale;                           // per (b, h): power-of-two gradient scale
};

// ---- small helpers ------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t h2u(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 u2f(uint32_t v) { return __half22float2(*reinterpret_cast<__half2*>(&v)); }
__device__ __forceinline__ uint32_t sm(const void* p) { return ptx::smem_u32(p); }

template <typename TI>
__device__ __forceinline__ void ld8(const TI* p, float (&f)[8]) {
  if constexpr (sizeof(TI) == 2) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
}

// A C x 128 token tile held in registers as loaded (8-element segments, C * 16 / NTH per thread of an
// NTH-thread block), so that several tiles' loads are in flight together before any is converted.
template <typename TI, int NTH = NTHR>
struct RawTile {
  static constexpr int PER = C * 16 / NTH;
  uint4 v[PER][sizeof(TI) / 2];
};
template <typename TI, int NTH>
__device__ __forceinline__ void raw_load(RawTile<TI, NTH>& t, const TI* base, int64_t st, int nvalid) {
#pragma unroll
  for (int it = 0; it < RawTile<TI, NTH>::PER; ++it) {
    const int i = threadIdx.x + it * NTH, r = i >> 4, seg = i & 15;
#pragma unroll
    for (int w = 0; w < (int)(sizeof(TI) / 2); ++w)
      t.v[it][w] = r < nvalid ? __ldg(reinterpret_cast<const uint4*>(base + r * st + seg * 8) + w) : make_uint4(0, 0, 0, 0);
  }
}
// Raw tile -> fp16 shared tile (LDT pitch), row r times mul * rs[r] (rs may be null).
template <typename TI, int NTH>
__device__ __forceinline__ void raw_store(__half* dst, const RawTile<TI, NTH>& t, const float* rs, float mul) {
#pragma unroll
  for (int it = 0; it < RawTile<TI, NTH>::PER; ++it) {
    const int i = threadIdx.x + it * NTH, r = i >> 4, seg = i & 15;
    float f[8];
    if constexpr (sizeof(TI) == 2) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&t.v[it][0]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 x = __bfloat1622float2(h[q]);
        f[2 * q] = x.x;
        f[2 * q + 1] = x.y;
      }
    } else {
      const float* x = reinterpret_cast<const float*>(&t.v[it][0]);
#pragma unroll
      for (int q = 0; q < 8; ++q) f[q] = x[q];
    }
    const float m = rs ? mul * rs[r] : mul;
    *reinterpret_cast<uint4*>(dst + r * LDT + seg * 8) =
        make_uint4(h2u(m * f[0], m * f[1]), h2u(m * f[2], m * f[3]), h2u(m * f[4], m * f[5]), h2u(m * f[6], m * f[7]));
  }
}

// Asynchronous copies global -> shared of 16 bytes (cp.async, L2 only), in commit groups.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Dense fp16 rows x cols (global, row-major) -> shared tile with `ld` halves per row, asynchronously.
template <int NTH = NTHR>
__device__ __forceinline__ void tile_async(__half* dst, int ld, const __half* src, int rows, int cols) {
  const int segs = cols >> 3;
  for (int i = threadIdx.x; i < rows * segs; i += NTH) {
    const int r = i / segs, sg = i - r * segs;
    cp16(dst + r * ld + sg * 8, src + (int64_t)r * cols + sg * 8);
  }
}

// fp16 C x 128 tile in shared memory (LDT pitch) -> dense rows in the workspace.
__device__ __forceinline__ void tile_store(__half* dst, const __half* src) {
  for (int i = threadIdx.x; i < C * 16; i += NTHR) {
    const int r = i >> 4, sg = i & 15;
    *reinterpret_cast<uint4*>(dst + r * D + sg * 8) = *reinterpret_cast<const uint4*>(src + r * LDT + sg * 8);
  }
}

// acc[MT][NT][4] += opA (16 MT x K) * opB (K x 8 NT), fp16 shared-memory operands, fp32 accumulators.
//   A_T = false: A(m, k) at a[m * lda + k];  A_T = true: A(m, k) at a[k * lda + m]
//   B_T = false: B(k, n) at b[n * ldb + k];  B_T = true: B(k, n) at b[k * ldb + n]
// Accumulator element e of tile (mt, nt): row m0 + 16 mt + lane/4 + 8 (e >> 1), column
// n0 + 8 nt + 2 (lane % 4) + (e & 1).
template <int MT, int NT, bool A_T, bool B_T, int K, bool FULL = false>
__device__ __forceinline__ void mma_acc(float (&acc)[MT][NT][4], const __half* a, int lda, int m0, const __half* b,
                                        int ldb, int n0, int lane) {
  static_assert(NT % 2 == 0, "B fragments are loaded for pairs of n tiles");
  static_assert(K % 32 == 0, "K is a multiple of 32");
  const int j = lane >> 3, r = lane & 7;
  const uint32_t abase = sm(a), bbase = sm(b);
  auto step = [&](int k0) {
    uint32_t af[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      if constexpr (!A_T) {
        const int row = m0 + 16 * mt + (lane & 15), col = k0 + ((lane >> 4) << 3);
        ptx::ldsm_x4(abase + (uint32_t)(row * lda + col) * 2u, af[mt]);
      } else {
        const int krow = k0 + ((j >> 1) << 3) + r, mcol = m0 + 16 * mt + ((j & 1) << 3);
        ptx::ldsm_x4_t(abase + (uint32_t)(krow * lda + mcol) * 2u, af[mt]);
      }
    }
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      uint32_t bf[4];
      if constexpr (!B_T) {
        const int nrow = n0 + 16 * np + ((j >> 1) << 3) + r, kcol = k0 + ((j & 1) << 3);
        ptx::ldsm_x4(bbase + (uint32_t)(nrow * ldb + kcol) * 2u, bf);
      } else {
        const int krow = k0 + ((j & 1) << 3) + r, ncol = n0 + 16 * np + ((j >> 1) << 3);
        ptx::ldsm_x4_t(bbase + (uint32_t)(krow * ldb + ncol) * 2u, bf);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        ptx::hmma16816(acc[mt][2 * np], af[mt], bf[0], bf[1]);
        ptx::hmma16816(acc[mt][2 * np + 1], af[mt], bf[2], bf[3]);
      }
    }
  };
  // Unrolled (fully, or by two): the next step's fragments load while this step's products run.
  if constexpr (FULL) {
#pragma unroll
    for (int k0 = 0; k0 < K; k0 += 16) step(k0);
  } else {
#pragma unroll 2
    for (int k0 = 0; k0 < K; k0 += 16) step(k0);
  }
}

template <int MT, int NT>
__device__ __forceinline__ void zero(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
}

// One 16-row accumulator strip (MT = 1) -> fp16 shared tile, times `mul`.
template <int NT>
__device__ __forceinline__ void strip_to_smem(__half* dst, int ld, int m0, int n0, const float (&acc)[1][NT][4], int lane,
                                              float mul) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int col = n0 + 8 * nt + 2 * t4;
    *reinterpret_cast<uint32_t*>(dst + (m0 + g) * ld + col) = h2u(mul * acc[0][nt][0], mul * acc[0][nt][1]);
    *reinterpret_cast<uint32_t*>(dst + (m0 + g + 8) * ld + col) = h2u(mul * acc[0][nt][2], mul * acc[0][nt][3]);
  }
}

// Sum over the 4 lanes of a quad (the lanes holding one accumulator row).
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

// Block-wide reductions (all NTH threads call; `red` holds NTH / 32 floats).
template <int NTH = NTHR>
__device__ __forceinline__ float block_sum(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NTH / 32; ++i) s += red[i];
  return s;
}
__device__ __forceinline__ float block_max(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NTHR / 32; ++i) s = fmaxf(s, red[i]);
  return s;
}

// Row and column sums of one warp's 16 x 32 strip of a C x C product into the partial arrays: rs[hf] holds
// this lane's part of row m0 + lane/4 + 8 hf, cs[nt][x] its part of column c0 + 8 nt + 2 (lane % 4) + x.
// Lane (lane % 4 == 0) writes the rows, lanes 0..3 the columns: one writer per element.
__device__ __forceinline__ void add_row_col(float* rows, float* cols, float (&rs)[2], float (&cs)[4][2], int m0, int c0,
                                            int lane) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) rs[hf] = quad_sum(rs[hf]);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) cs[nt][x] += __shfl_xor_sync(0xffffffffu, cs[nt][x], o);
  if (t4 == 0) {
    rows[m0 + g] += rs[0];
    rows[m0 + g + 8] += rs[1];
  }
  if (g == 0) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      cols[c0 + 8 * nt + 2 * t4] += cs[nt][0];
      cols[c0 + 8 * nt + 2 * t4 + 1] += cs[nt][1];
    }
  }
}

template <typename TI>
__device__ __forceinline__ const TI* tok(const void* base, int64_t sb, int64_t st, int64_t sh, int b, int t, int h) {
  return reinterpret_cast<const TI*>(base) + (int64_t)b * sb + (int64_t)t * st + (int64_t)h * sh;
}

// Every 128-byte line of [ptr, ptr + bytes) into L2, spread over the block's threads.
__device__ __forceinline__ void prefetch_span(const void* ptr, int64_t bytes) {
  const char* c = reinterpret_cast<const char*>(ptr);
  for (int64_t o = (int64_t)threadIdx.x * 128; o < bytes; o += (int64_t)NTHR * 128) ptx::prefetch_l2(c + o);
}

// The q and v rows of chunk `task` (and k's, dY's and u's when asked) into L2, one row per thread.
template <typename TI, typename TD>
__device__ __forceinline__ void prefetch_rows(const Params& p, int task, bool with_k, bool with_dy, bool with_u) {
  const int bh = task / p.NC, c = task - bh * p.NC;
  const int b = bh / p.H, h = bh - b * p.H, t0 = c * C, nv = min(C, p.T - t0);
  for (int e = threadIdx.x; e < 5 * C; e += NTHR) {
    const int which = e / C, r = e - which * C;
    if (r >= nv || (which == 0 && !with_k) || (which == 3 && !with_dy) || (which == 4 && !with_u)) continue;
    const char* row;
    int bytes = D * (int)sizeof(TI);
    switch (which) {
      case 0: row = reinterpret_cast<const char*>(tok<TI>(p.k, p.sk_b, p.sk_t, p.sk_h, b, t0 + r, h)); break;
      case 1: row = reinterpret_cast<const char*>(tok<TI>(p.q, p.sq_b, p.sq_t, p.sq_h, b, t0 + r, h)); break;
      case 2: row = reinterpret_cast<const char*>(tok<TI>(p.v, p.sv_b, p.sv_t, p.sv_h, b, t0 + r, h)); break;
      case 3:
        row = reinterpret_cast<const char*>(tok<TD>(p.dy, p.sd_b, p.sd_t, p.sd_h, b, t0 + r, h));
        bytes = D * (int)sizeof(TD);
        break;
      default: row = reinterpret_cast<const char*>(tok<TI>(p.u, p.su_b, p.su_t, p.su_h, b, t0 + r, h)); break;
    }
    for (int o = 0; o < bytes; o += 128) ptx::prefetch_l2(row + o);
  }
}

// Power of two that brings max |dY|, max |dS_T| of one (b, h) into [0.5, 1) (1 when they are 0).
__device__ __forceinline__ float grad_scale(unsigned bits) {
  const float a = __uint_as_float(bits);
  if (!(a > 0.f) || !isfinite(a)) return 1.f;
  int e;
  frexpf(a, &e);
  return ldexpf(1.f, -e);
}

// ---- max |dY| (and |dS_T|) per (b, h) -------------------------------------------------------------------
template <typename TD>
__global__ void __launch_bounds__(NTHR) amax_kernel(Params p) {
  __shared__ float red[NTHR / 32];
  const int task = blockIdx.x, bh = task / p.NC, c = task - bh * p.NC;
  const int b = bh / p.H, h = bh - b * p.H, t0 = c * C, nvalid = min(C, p.T - t0);
  const TD* dyp = tok<TD>(p.dy, p.sd_b, p.sd_t, p.sd_h, b, t0, h);
  constexpr int PER = C * 16 / NTHR;
  float f[PER][8];
#pragma unroll
  for (int it = 0; it < PER; ++it) {
    const int i = threadIdx.x + it * NTHR, r = i >> 4, seg = i & 15;
    if (r < nvalid) {
      ld8(dyp + r * p.sd_t + seg * 8, f[it]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[it][j] = 0.f;
    }
  }
  float m = 0.f;
#pragma unroll
  for (int it = 0; it < PER; ++it)
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(f[it][j]));
  if (c == 0 && p.dsT) {
    const float4* s = reinterpret_cast<const float4*>(p.dsT + ((int64_t)bh * p.DVt + p.vofs) * D);
    for (int i = threadIdx.x; i < D * D / 4; i += NTHR) {
      const float4 x = __ldg(s + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
    }
  }
  m = block_max(m, red);
  if (threadIdx.x == 0 && m > 0.f) atomicMax(p.amax + bh, __float_as_uint(m));
}

// ---- prep: per chunk g, T, A, W, Uw and the chains' fp16 operands U, d U, Gamma Q, scaled dY ---------------
// REUSE (the state slices after the first of DV > 128): g, T, A, W, U and d U do not depend on the slice
// and are in the workspace from the first slice's prep; only T V, the scaled dY, A^T dY and dY^T Gamma Q
// are formed, from T and A read back.
constexpr int PREP_SMEM = 5 * TILE_CD * 2 + TILE_CC * 2 + C * (C + 1) * 4 + 5 * C * 4 + 64;

template <typename TI, typename TD, bool REUSE>
__global__ void __launch_bounds__(NTHR) prep_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __half* sK = reinterpret_cast<__half*>(smem);  // later T in fp32 (C x (C + 1))
  __half* sU = sK + TILE_CD;
  __half* sQ = sU + TILE_CD;
  __half* sV = sQ + TILE_CD;
  __half* sGK = sV + TILE_CD;
  __half* sT = sGK + TILE_CD;
  float* sL = reinterpret_cast<float*>(sT + TILE_CC);  // C x (C + 1) floats: L in fp16 and its diagonal blocks in fp32
  float* sg = sL + C * (C + 1);
  float* sgam = sg + C;
  float* sd = sgam + C;
  float* sbeta = sd + C;
  __half* sL16 = reinterpret_cast<__half*>(sL);                                           // C rows of LD16 bytes
  float* sLd = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sL) + C * tiles::LD16);  // 4 x 16 x LDG
  static_assert(C * tiles::LD16 + 4 * 16 * tiles::LDG * 4 <= C * (C + 1) * 4, "L16 and its diagonal blocks fit");
  static_assert(LDC * 2 == tiles::LD16, "T rows as the block merges address them");

  const int task = blockIdx.x, bh = task / p.NC, c = task - bh * p.NC;
  const int b = bh / p.H, h = bh - b * p.H;
  const int t0 = c * C, nvalid = min(C, p.T - t0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // This chunk's q, k, (u,) v and dY tiles in flight first, under the gate scan below.
  RawTile<TI> rk, rq, rv, ru;
  RawTile<TD> rd;
  if constexpr (!REUSE) raw_load(rk, tok<TI>(p.k, p.sk_b, p.sk_t, p.sk_h, b, t0, h), p.sk_t, nvalid);
  raw_load(rq, tok<TI>(p.q, p.sq_b, p.sq_t, p.sq_h, b, t0, h), p.sq_t, nvalid);
  raw_load(rv, tok<TI>(p.v, p.sv_b, p.sv_t, p.sv_h, b, t0, h), p.sv_t, nvalid);
  raw_load(rd, tok<TD>(p.dy, p.sd_b, p.sd_t, p.sd_h, b, t0, h), p.sd_t, nvalid);
  if (!REUSE && p.u) raw_load(ru, tok<TI>(p.u, p.su_b, p.su_t, p.su_h, b, t0, h), p.su_t, nvalid);
  // The tiles of the chunk p.pf blocks on (one resident wave: its block starts about when this one
  // ends) into L2, so that its loads do not wait on HBM.
  if (p.pf > 0 && (int64_t)task + p.pf < (int64_t)p.NC * p.BH)
    prefetch_rows<TI, TD>(p, task + p.pf, !REUSE, true, !REUSE && p.u != nullptr);
  const float scale = grad_scale(p.amax[bh]);
  if (c == 0 && tid == 0) p.scale[bh] = scale;

  if (tid < C) {
    const int64_t gi = ((int64_t)b * p.T + t0 + tid) * p.H + h;
    float la = tid < nvalid ? p.la[gi] : 0.f;
    sbeta[tid] = (p.beta != nullptr && tid < nvalid) ? p.beta[gi] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float x = __shfl_up_sync(0xffffffffu, la, o);
      if (lane >= o) la += x;
    }
    sg[tid] = la;
  }
  __syncthreads();
  if (tid >= 32 && tid < C) sg[tid] += sg[31];
  __syncthreads();
  if (tid < C) {
    sgam[tid] = expf(sg[tid]);
    sd[tid] = expf(sg[C - 1] - sg[tid]);
    if (!REUSE) p.wg[(int64_t)task * C + tid] = sg[tid];
  }
  __syncthreads();

  {
    if constexpr (REUSE) {
      tile_async(sT, LDC, p.wT + (int64_t)task * C * C, C, C);
      cp_commit();
    } else {
      // k feeds three tiles (K, beta K = U, Gamma K)
      raw_store(sK, rk, nullptr, 1.f);
      raw_store(sGK, rk, sgam, 1.f);
      if (p.u) {
        raw_store(sU, ru, nullptr, 1.f);
      } else {
        raw_store(sU, rk, sbeta, 1.f);
      }
    }
    raw_store(sQ, rq, nullptr, 1.f);
    raw_store(sV, rv, nullptr, 1.f);
    // dY times the gradient scale -> the workspace (dense rows), straight from registers
    __half* wd = p.wdY + (int64_t)task * C * D;
#pragma unroll
    for (int it = 0; it < RawTile<TD>::PER; ++it) {
      const int i = tid + it * NTHR, r = i >> 4, seg = i & 15;
      float f[8];
      if constexpr (sizeof(TD) == 2) {
        const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&rd.v[it][0]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 x = __bfloat1622float2(hh[q]);
          f[2 * q] = x.x;
          f[2 * q + 1] = x.y;
        }
      } else {
        const float* x = reinterpret_cast<const float*>(&rd.v[it][0]);
#pragma unroll
        for (int q = 0; q < 8; ++q) f[q] = x[q];
      }
      *reinterpret_cast<uint4*>(wd + r * D + seg * 8) =
          make_uint4(h2u(scale * f[0], scale * f[1]), h2u(scale * f[2], scale * f[3]), h2u(scale * f[4], scale * f[5]),
                     h2u(scale * f[6], scale * f[7]));
    }
  }
  __syncthreads();

  if constexpr (REUSE) {
    cp_wait<0>();
    __syncthreads();
  } else {
    // M = K U^T -> L (strictly lower, fp16; its diagonal blocks also fp32); P = Q U^T -> A (fp16, lower incl.
    // diagonal, to the workspace)
    {
      const int m0 = 16 * (warp & 3), n0 = 32 * (warp >> 2), g = lane >> 2, t4 = lane & 3;
      float accM[1][4][4], accP[1][4][4];
      zero(accM);
      zero(accP);
      mma_acc<1, 4, false, false, D>(accM, sK, LDT, m0, sU, LDT, n0, lane);
      mma_acc<1, 4, false, false, D>(accP, sQ, LDT, m0, sU, LDT, n0, lane);
      __half* Aout = p.wA + (int64_t)task * C * C;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int row = m0 + g + 8 * hf, col = n0 + 8 * nt + 2 * t4;
          float e[2], a[2], l[2];
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const int cc = col + x;
            e[x] = cc <= row ? __expf(sg[row] - sg[cc]) : 0.f;
            l[x] = cc < row ? accM[0][nt][2 * hf + x] * e[x] : 0.f;
            a[x] = accP[0][nt][2 * hf + x] * e[x];
          }
          *reinterpret_cast<uint32_t*>(sL16 + row * (tiles::LD16 / 2) + col) = h2u(l[0], l[1]);
          if ((row >> 4) == (col >> 4))  // the diagonal blocks also in fp32, for the substitution
            *reinterpret_cast<float2*>(sLd + row * tiles::LDG + (col & 15)) = make_float2(l[0], l[1]);
          *reinterpret_cast<uint32_t*>(Aout + row * C + col) = h2u(a[0], a[1]);
        }
    }
    __syncthreads();  // L complete

    // T = (I + L)^-1: the diagonal blocks D_b = (I + L_bb)^-1 by fp32 forward substitution (one column
    // per thread) into L16's diagonal blocks, then block column J of T on warp J by mma.sync merges of
    // the fp16 blocks, T_iJ = -D_i sum_{k=J}^{i-1} L_ik T_kJ (tiles::merge_column_core).
    if (tid < C) {
      const int bb = tid >> 4, j = tid & 15;
      const float* Lb = sLd + bb * 16 * tiles::LDG;
      float x[16], acc[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        x[m] = (m == j) ? 1.f : (m > j ? -acc[m] : 0.f);
#pragma unroll
        for (int r = m + 1; r < 16; ++r) acc[r] = fmaf(Lb[r * tiles::LDG + m], x[m], acc[r]);
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) sL16[(bb * 16 + r) * (tiles::LD16 / 2) + bb * 16 + j] = __float2half_rn(x[r]);
    }
    __syncthreads();
    if (warp < 4) {
      const uint32_t tT = ptx::smem_u32(sT);
      auto emit = [&](int i, const float (&f)[8]) {
        const uint32_t v[4] = {h2u(f[0], f[1]), h2u(f[2], f[3]), h2u(f[4], f[5]), h2u(f[6], f[7])};
        ptx::stsm_x4_t(tiles::frag_addr_plain(tT, LDC * 2, 16 * i, 16 * warp, lane), v);
      };
      auto zero = [&](int i) {
        const uint32_t z[4] = {0u, 0u, 0u, 0u};
        ptx::stsm_x4_t(tiles::frag_addr_plain(tT, LDC * 2, 16 * i, 16 * warp, lane), z);
      };
      tiles::merge_column_core(warp, ptx::smem_u32(sL16), lane, emit, zero);
    }
    __syncthreads();
    {
      __half* Tout = p.wT + (int64_t)task * C * C;
      for (int i = tid; i < C * C / 8; i += NTHR) {
        const int row = i >> 3, seg = i & 7;
        *reinterpret_cast<uint4*>(Tout + row * C + seg * 8) = *reinterpret_cast<const uint4*>(sT + row * LDC + seg * 8);
      }
    }
  }

  // W = T (Gamma K), Uw = T V -> workspace (fp16)
  {
    const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2), g = lane >> 2, t4 = lane & 3;
    float acc[1][8][4];
#pragma unroll 1
    for (int which = REUSE ? 1 : 0; which < 2; ++which) {
      zero(acc);
      mma_acc<1, 8, false, true, C>(acc, sT, LDC, m0, which ? sV : sGK, LDT, n0, lane);
      __half* out = (which ? p.wUw : p.wW) + (int64_t)task * C * D;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = n0 + 8 * nt + 2 * t4;
        *reinterpret_cast<uint32_t*>(out + (m0 + g) * D + col) = h2u(acc[0][nt][0], acc[0][nt][1]);
        *reinterpret_cast<uint32_t*>(out + (m0 + g + 8) * D + col) = h2u(acc[0][nt][2], acc[0][nt][3]);
      }
    }
  }
  __syncthreads();  // Gamma K, T and L are no longer read

  // The backward chain's dS-independent terms, once per chunk here instead of on the chain:
  // dR0 = A^T dY (C x DV) and Pc = dY^T Gamma Q (DV x DK).  Gamma Q is built in K's space, dY (scaled, as
  // written above) and A come back from the workspace into the spaces of Gamma K and L.
  __half* sGQ = sK;
  __half* sdY = sGK;
  __half* sA = reinterpret_cast<__half*>(sL);
  tile_async(sdY, LDT, p.wdY + (int64_t)task * C * D, C, D);
  tile_async(sA, LDC, p.wA + (int64_t)task * C * C, C, C);
  cp_commit();
  {
    const int64_t o = (int64_t)task * C * D;
    for (int i = tid; i < C * 16; i += NTHR) {
      const int r = i >> 4, sg8 = (i & 15) * 8;
      const uint4 q = *reinterpret_cast<const uint4*>(sQ + r * LDT + sg8);
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
      uint32_t gq[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 bq = u2f(qw[j]);
        gq[j] = h2u(sgam[r] * bq.x, sgam[r] * bq.y);
      }
      *reinterpret_cast<uint4*>(sGQ + r * LDT + sg8) = make_uint4(gq[0], gq[1], gq[2], gq[3]);
      if constexpr (!REUSE) {
        const uint4 u = *reinterpret_cast<const uint4*>(sU + r * LDT + sg8);
        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
        uint32_t du[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = u2f(uw[j]);
          du[j] = h2u(sd[r] * a.x, sd[r] * a.y);
        }
        *reinterpret_cast<uint4*>(p.wU + o + r * D + sg8) = u;
        *reinterpret_cast<uint4*>(p.wDU + o + r * D + sg8) = make_uint4(du[0], du[1], du[2], du[3]);
      }
    }
  }
  cp_wait<0>();
  __syncthreads();
  {
    const int g = lane >> 2, t4 = lane & 3;
    float acc[1][8][4];
    // dR0: warp -> rows 16 (warp & 3).., columns 64 (warp >> 2)..
    const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
    zero(acc);
    mma_acc<1, 8, true, true, C>(acc, sA, LDC, m0, sdY, LDT, n0, lane);
    __half* out = p.wdR0 + (int64_t)task * C * D;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = n0 + 8 * nt + 2 * t4;
      *reinterpret_cast<uint32_t*>(out + (m0 + g) * D + col) = h2u(acc[0][nt][0], acc[0][nt][1]);
      *reinterpret_cast<uint32_t*>(out + (m0 + g + 8) * D + col) = h2u(acc[0][nt][2], acc[0][nt][3]);
    }
    // Pc: warp -> rows 16 warp.., all 128 columns in two halves
    __half* pc = p.wPc + (int64_t)task * D * D;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      zero(acc);
      mma_acc<1, 8, true, true, C>(acc, sdY, LDT, 16 * warp, sGQ, LDT, 64 * half, lane);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = 64 * half + 8 * nt + 2 * t4;
        *reinterpret_cast<uint32_t*>(pc + (16 * warp + g) * D + col) = h2u(acc[0][nt][0], acc[0][nt][1]);
        *reinterpret_cast<uint32_t*>(pc + (16 * warp + g + 8) * D + col) = h2u(acc[0][nt][2], acc[0][nt][3]);
      }
    }
  }
}

// ---- chains: S0 of every chunk (forwards), dS1 of every chunk (backwards) ----------------------------
// Per chunk the block streams its operands from the workspace with cp.async into one of two buffers,
// the next chunk's while it works on this one.  Buffer: forward [W | Uw | U], backward [A^T dY | d U | W |
// dY^T Gamma Q]; the chunk's g beside each.
constexpr int CHAIN_BUF = 3 * TILE_CD + TILE_DD;
constexpr int CHAIN_SMEM = (TILE_DD + TILE_CD + 2 * CHAIN_BUF) * 2 + 2 * C * 4 + 64;

__global__ void __launch_bounds__(NTHR, 1) chain_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int bh = blockIdx.x >> 1;
  const bool forward = (blockIdx.x & 1) == 0;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const int row0 = 16 * w + g, row1 = row0 + 8;  // this lane's state rows

  __half* sX = reinterpret_cast<__half*>(smem);  // fp16 copy of S (forward) or dS (backward); warp w owns rows 16w..
  __half* sP = sX + TILE_DD;                      // d R (forward) or -dR (backward); warp w owns columns 16w..
  __half* buf = sP + TILE_CD;                     // 2 x CHAIN_BUF
  float* sgb = reinterpret_cast<float*>(buf + 2 * CHAIN_BUF);  // 2 x C: g of the buffered chunk

  auto issue = [&](int c, int bi) {
    const int64_t task = (int64_t)bh * p.NC + c;
    __half* bb = buf + bi * CHAIN_BUF;
    if (forward) {
      tile_async(bb, LDT, p.wW + task * C * D, C, D);
      tile_async(bb + TILE_CD, LDT, p.wUw + task * C * D, C, D);
      tile_async(bb + 2 * TILE_CD, LDT, p.wU + task * C * D, C, D);
    } else {
      tile_async(bb, LDT, p.wdR0 + task * C * D, C, D);
      tile_async(bb + TILE_CD, LDT, p.wDU + task * C * D, C, D);
      tile_async(bb + 2 * TILE_CD, LDT, p.wW + task * C * D, C, D);
      tile_async(bb + 3 * TILE_CD, LDT, p.wPc + task * D * D, D, D);
    }
    if (tid < C / 4) cp16(sgb + bi * C + 4 * tid, p.wg + task * C + 4 * tid);
    cp_commit();
  };

  float acc[1][16][4];
  const float* init = forward ? p.s0 : p.dsT;
  const float scale = forward ? 1.f : p.scale[bh];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int col = 8 * nt + 2 * t4;
    float2 a = make_float2(0.f, 0.f), c2 = make_float2(0.f, 0.f);
    if (init) {
      a = *reinterpret_cast<const float2*>(init + ((int64_t)bh * p.DVt + p.vofs + row0) * D + col);
      c2 = *reinterpret_cast<const float2*>(init + ((int64_t)bh * p.DVt + p.vofs + row1) * D + col);
    }
    acc[0][nt][0] = scale * a.x; acc[0][nt][1] = scale * a.y; acc[0][nt][2] = scale * c2.x; acc[0][nt][3] = scale * c2.y;
  }

  issue(forward ? 0 : p.NC - 1, 0);
#pragma unroll 1
  for (int it = 0; it < p.NC; ++it) {
    const int c = forward ? it : p.NC - 1 - it, bi = it & 1;
    if (it + 1 < p.NC) issue(forward ? c + 1 : c - 1, bi ^ 1);
    else cp_commit();  // an empty group keeps the wait count below uniform
    // this warp's rows -> fp16 (its own rows of sX) and the workspace
    __half* wout = (forward ? p.wS : p.wdS) + ((int64_t)bh * p.NC + c) * D * D;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int col = 8 * nt + 2 * t4;
      const uint32_t x0 = h2u(acc[0][nt][0], acc[0][nt][1]), x1 = h2u(acc[0][nt][2], acc[0][nt][3]);
      *reinterpret_cast<uint32_t*>(sX + row0 * LDT + col) = x0;
      *reinterpret_cast<uint32_t*>(sX + row1 * LDT + col) = x1;
      *reinterpret_cast<uint32_t*>(wout + row0 * D + col) = x0;
      *reinterpret_cast<uint32_t*>(wout + row1 * D + col) = x1;
    }
    cp_wait<1>();     // this thread's copies of chunk c have landed
    __syncthreads();  // ... and everyone's
    const __half* bb = buf + bi * CHAIN_BUF;
    const float* sg = sgb + bi * C;
    const float gl = sg[C - 1], gC = __expf(gl);
    float r[4][2][4];
    zero(r);
    if (forward) {
      const __half *W = bb, *Uw = bb + TILE_CD, *U = bb + 2 * TILE_CD;
      // R = Uw - W S^T for this warp's 16 columns (= its state rows); d R -> sP
      mma_acc<4, 2, false, false, D, true>(r, W, LDT, 0, sX, LDT, 16 * w, lane);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int tr = 16 * mt + g + 8 * hf;
          const float dd = __expf(gl - sg[tr]);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int dc = 16 * w + 8 * nt + 2 * t4;
            const float2 uw = u2f(*reinterpret_cast<const uint32_t*>(Uw + tr * LDT + dc));
            *reinterpret_cast<uint32_t*>(sP + tr * LDT + dc) =
                h2u(dd * (uw.x - r[mt][nt][2 * hf]), dd * (uw.y - r[mt][nt][2 * hf + 1]));
          }
        }
      __syncwarp();
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[0][nt][e] *= gC;
      // S = gamma_C S + (d R)^T U
      mma_acc<1, 16, true, true, C, true>(acc, sP, LDT, 16 * w, U, LDT, 0, lane);
    } else {
      const __half *dR0 = bb, *DU = bb + TILE_CD, *W = DU + TILE_CD, *Pc = W + TILE_CD;
      // dR = A^T dY + (d U) dS^T for this warp's 16 columns; -dR -> sP
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int tr = 16 * mt + g + 8 * hf, dc = 16 * w + 8 * nt + 2 * t4;
            const float2 x = u2f(*reinterpret_cast<const uint32_t*>(dR0 + tr * LDT + dc));
            r[mt][nt][2 * hf] = x.x;
            r[mt][nt][2 * hf + 1] = x.y;
          }
      mma_acc<4, 2, false, false, D, true>(r, DU, LDT, 0, sX, LDT, 16 * w, lane);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int tr = 16 * mt + g + 8 * hf, dc = 16 * w + 8 * nt + 2 * t4;
            *reinterpret_cast<uint32_t*>(sP + tr * LDT + dc) = h2u(-r[mt][nt][2 * hf], -r[mt][nt][2 * hf + 1]);
          }
      __syncwarp();
      // dS = gamma_C dS + dY^T (Gamma Q) - dR^T W
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int col = 8 * nt + 2 * t4;
        const float2 x0 = u2f(*reinterpret_cast<const uint32_t*>(Pc + row0 * LDT + col));
        const float2 x1 = u2f(*reinterpret_cast<const uint32_t*>(Pc + row1 * LDT + col));
        acc[0][nt][0] = gC * acc[0][nt][0] + x0.x;
        acc[0][nt][1] = gC * acc[0][nt][1] + x0.y;
        acc[0][nt][2] = gC * acc[0][nt][2] + x1.x;
        acc[0][nt][3] = gC * acc[0][nt][3] + x1.y;
      }
      mma_acc<1, 16, true, true, C, true>(acc, sP, LDT, 16 * w, W, LDT, 0, lane);
    }
    __syncthreads();  // every warp is done with buffer bi before the next iteration refills it
  }
  cp_wait<0>();
  if (!forward && p.ds0) {
    const float inv = 1.f / scale;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int col = 8 * nt + 2 * t4;
      *reinterpret_cast<float2*>(p.ds0 + ((int64_t)bh * p.DVt + p.vofs + row0) * D + col) =
          make_float2(inv * acc[0][nt][0], inv * acc[0][nt][1]);
      *reinterpret_cast<float2*>(p.ds0 + ((int64_t)bh * p.DVt + p.vofs + row1) * D + col) =
          make_float2(inv * acc[0][nt][2], inv * acc[0][nt][3]);
    }
  }
}

// ---- local: every gradient of one chunk ------------------------------------------------------------
constexpr int LOCAL_SMEM = (8 * TILE_CD + 2 * TILE_CC + 2 * TILE_DD) * 2 + 15 * C * 4;

template <typename TI, typename TD>
__global__ void __launch_bounds__(NTHR, 1) local_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __half* sQ = reinterpret_cast<__half*>(smem);
  __half* sK = sQ + TILE_CD;
  __half* sU = sK + TILE_CD;
  __half* sV = sU + TILE_CD;
  __half* sdY = sV + TILE_CD;
  __half* sNW = sdY + TILE_CD;  // W, later dW
  __half* sR = sNW + TILE_CD;
  __half* sdR = sR + TILE_CD;
  __half* sT = sdR + TILE_CD;
  __half* sA = sT + TILE_CC;
  __half* sB0 = sA + TILE_CC;  // S0, later dP and dT
  __half* sB1 = sB0 + TILE_DD; // dS1, later Y1 and dM
  float* sg = reinterpret_cast<float*>(sB1 + TILE_DD);
  float* sgam = sg + C;
  float* sd = sgam + C;
  float* sbeta = sd + C;
  // Gate-gradient partials, each element written by one lane only (in program order), then summed in a
  // fixed order: bitwise reproducible.  Rows by column half (warp >> 2), columns by row tile (warp & 3).
  float* sdgr = sbeta + C;     // [2][C] row contributions to dg
  float* scol = sdgr + 2 * C;  // [4][C] column contributions to dg (subtracted)
  float* sdd = scol + 4 * C;   // [2][C] dd_t = (R dS1)_t . u_t
  float* sdb = sdd + 2 * C;    // [2][C] dbeta partials
  float* red = sdb + 2 * C;
  __half* sdP = sB0;
  __half* sdT = sB0 + TILE_CC;
  __half* sY1 = sB1;
  __half* sdM = sB1 + TILE_CC;

  const int task = blockIdx.x, bh = task / p.NC, c = task - bh * p.NC;
  const int b = bh / p.H, h = bh - b * p.H;
  const int t0 = c * C, nvalid = min(C, p.T - t0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const float scale = p.scale[bh], inv = 1.f / scale;

  if (tid < C) {
    const float* gg = p.wg + (int64_t)task * C;
    const float gt = gg[tid];
    const int64_t gi = ((int64_t)b * p.T + t0 + tid) * p.H + h;
    sg[tid] = gt;
    sgam[tid] = __expf(gt);
    sd[tid] = __expf(gg[C - 1] - gt);
    sbeta[tid] = (p.beta != nullptr && tid < nvalid) ? p.beta[gi] : 0.f;
  }
  for (int i = tid; i < 10 * C; i += NTHR) sdgr[i] = 0.f;  // sdgr, scol, sdd, sdb are contiguous
  __syncthreads();
  {
    const int64_t oc = (int64_t)task * C * D;
    tile_async(sU, LDT, p.wU + oc, C, D);
    tile_async(sdY, LDT, p.wdY + oc, C, D);
    tile_async(sNW, LDT, p.wW + oc, C, D);
    tile_async(sT, LDC, p.wT + (int64_t)task * C * C, C, C);
    tile_async(sA, LDC, p.wA + (int64_t)task * C * C, C, C);
    tile_async(sB0, LDT, p.wS + (int64_t)task * D * D, D, D);
    tile_async(sB1, LDT, p.wdS + (int64_t)task * D * D, D, D);
    cp_commit();
  }
  {
    RawTile<TI> rq, rk, rv;
    raw_load(rq, tok<TI>(p.q, p.sq_b, p.sq_t, p.sq_h, b, t0, h), p.sq_t, nvalid);
    raw_load(rk, tok<TI>(p.k, p.sk_b, p.sk_t, p.sk_h, b, t0, h), p.sk_t, nvalid);
    raw_load(rv, tok<TI>(p.v, p.sv_b, p.sv_t, p.sv_h, b, t0, h), p.sv_t, nvalid);
    // One block per SM loads its chunk and then computes with the SM's loads idle: the chunk one
    // resident wave on (its block starts about when this one ends) goes into L2 meanwhile.
    if (p.pf > 0 && (int64_t)task + p.pf < (int64_t)p.NC * p.BH) {
      const int64_t nt = task + p.pf, oc = nt * C * D;
      prefetch_span(p.wU + oc, C * D * 2);
      prefetch_span(p.wdY + oc, C * D * 2);
      prefetch_span(p.wW + oc, C * D * 2);
      prefetch_span(p.wT + nt * C * C, C * C * 2);
      prefetch_span(p.wA + nt * C * C, C * C * 2);
      prefetch_span(p.wS + nt * D * D, D * D * 2);
      prefetch_span(p.wdS + nt * D * D, D * D * 2);
      prefetch_rows<TI, TD>(p, (int)nt, true, false, false);
    }
    raw_store(sQ, rq, nullptr, 1.f);
    raw_store(sK, rk, nullptr, 1.f);
    raw_store(sV, rv, nullptr, 1.f);
  }
  cp_wait<0>();
  __syncthreads();

  // 64 x 128 outputs: warp -> rows m0..m0+15, columns n0..n0+63
  const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2), hw = warp >> 2;
  const int ra = m0 + g, rb = ra + 8;
  float acc[1][8][4];

  // R = T V - W S0^T
  zero(acc);
  mma_acc<1, 8, false, false, D>(acc, sNW, LDT, m0, sB0, LDT, n0, lane);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[0][nt][e] = -acc[0][nt][e];
  mma_acc<1, 8, false, true, C>(acc, sT, LDC, m0, sV, LDT, n0, lane);
  strip_to_smem(sR, LDT, m0, n0, acc, lane, 1.f);
  // dR = d (U dS1^T) + A^T dY
  zero(acc);
  mma_acc<1, 8, false, false, D>(acc, sU, LDT, m0, sB1, LDT, n0, lane);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    acc[0][nt][0] *= sd[ra]; acc[0][nt][1] *= sd[ra];
    acc[0][nt][2] *= sd[rb]; acc[0][nt][3] *= sd[rb];
  }
  mma_acc<1, 8, true, true, C>(acc, sA, LDC, m0, sdY, LDT, n0, lane);
  strip_to_smem(sdR, LDT, m0, n0, acc, lane, 1.f);
  __syncthreads();

  // X = dY S0: dg_t += gamma_t q_t . X_t;  dQ = Gamma X (+ dP U below)
  float aQ[1][8][4];
  zero(aQ);
  mma_acc<1, 8, false, true, D>(aQ, sdY, LDT, m0, sB0, LDT, n0, lane);
  {
    float pa = 0.f, pb = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = n0 + 8 * nt + 2 * t4;
      const float2 qa = u2f(*reinterpret_cast<const uint32_t*>(sQ + ra * LDT + col));
      const float2 qb = u2f(*reinterpret_cast<const uint32_t*>(sQ + rb * LDT + col));
      pa += qa.x * aQ[0][nt][0] + qa.y * aQ[0][nt][1];
      pb += qb.x * aQ[0][nt][2] + qb.y * aQ[0][nt][3];
    }
    pa = quad_sum(pa);
    pb = quad_sum(pb);
    if (t4 == 0) {
      sdgr[hw * C + ra] += sgam[ra] * pa;
      sdgr[hw * C + rb] += sgam[rb] * pb;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      aQ[0][nt][0] *= sgam[ra]; aQ[0][nt][1] *= sgam[ra];
      aQ[0][nt][2] *= sgam[rb]; aQ[0][nt][3] *= sgam[rb];
    }
  }
  // Z = R dS1: dd_t = Z_t . u_t;  dU = d Z (+ dP^T Q + dM^T K below)
  float aU[1][8][4];
  zero(aU);
  mma_acc<1, 8, false, true, D>(aU, sR, LDT, m0, sB1, LDT, n0, lane);
  {
    float pa = 0.f, pb = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = n0 + 8 * nt + 2 * t4;
      const float2 ua = u2f(*reinterpret_cast<const uint32_t*>(sU + ra * LDT + col));
      const float2 ub = u2f(*reinterpret_cast<const uint32_t*>(sU + rb * LDT + col));
      pa += ua.x * aU[0][nt][0] + ua.y * aU[0][nt][1];
      pb += ub.x * aU[0][nt][2] + ub.y * aU[0][nt][3];
    }
    pa = quad_sum(pa);
    pb = quad_sum(pb);
    if (t4 == 0) {
      sdd[hw * C + ra] += pa;
      sdd[hw * C + rb] += pb;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      aU[0][nt][0] *= sd[ra]; aU[0][nt][1] *= sd[ra];
      aU[0][nt][2] *= sd[rb]; aU[0][nt][3] *= sd[rb];
    }
  }
  // dW = -dR S0 -> sNW (every warp has finished reading W)
  zero(acc);
  mma_acc<1, 8, false, true, D>(acc, sdR, LDT, m0, sB0, LDT, n0, lane);
  strip_to_smem(sNW, LDT, m0, n0, acc, lane, -1.f);
  // <dS1, S0>
  float dot = 0.f;
  for (int i = tid; i < D * D / 2; i += NTHR) {
    const int row = i >> 6, col = 2 * (i & 63);
    const float2 a = u2f(*reinterpret_cast<const uint32_t*>(sB0 + row * LDT + col));
    const float2 bb = u2f(*reinterpret_cast<const uint32_t*>(sB1 + row * LDT + col));
    dot += a.x * bb.x + a.y * bb.y;
  }
  dot = block_sum(dot, red);  // (its barriers also end every read of S0 and dS1)

  // C x C products: warp -> rows m0..m0+15, columns c0..c0+31
  const int c0 = 32 * (warp >> 2);
  float sq[1][4][4];
  // dA = tril(dY R^T): dg += rowsum(dA o A) - colsum(dA o A);  dP = dA o E
  zero(sq);
  mma_acc<1, 4, false, false, D>(sq, sdY, LDT, m0, sR, LDT, c0, lane);
  {
    float rs[2] = {0.f, 0.f}, cs[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      cs[nt][0] = cs[nt][1] = 0.f;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = m0 + g + 8 * hf, col = c0 + 8 * nt + 2 * t4;
        float o[2];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int cc = col + x;
          const float da = cc <= row ? sq[0][nt][2 * hf + x] : 0.f;
          const float pr = da * __half2float(sA[row * LDC + cc]);
          rs[hf] += pr;
          cs[nt][x] += pr;
          o[x] = cc <= row ? da * __expf(sg[row] - sg[cc]) : 0.f;
        }
        *reinterpret_cast<uint32_t*>(sdP + row * LDC + col) = h2u(o[0], o[1]);
      }
    }
    add_row_col(sdgr + hw * C, scol + (warp & 3) * C, rs, cs, m0, c0, lane);
  }
  // dT = (dW K^T) diag(gamma) + dR V^T
  zero(sq);
  mma_acc<1, 4, false, false, D>(sq, sNW, LDT, m0, sK, LDT, c0, lane);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int col = c0 + 8 * nt + 2 * t4;
    sq[0][nt][0] *= sgam[col]; sq[0][nt][1] *= sgam[col + 1];
    sq[0][nt][2] *= sgam[col]; sq[0][nt][3] *= sgam[col + 1];
  }
  mma_acc<1, 4, false, false, D>(sq, sdR, LDT, m0, sV, LDT, c0, lane);
  strip_to_smem(sdT, LDC, m0, c0, sq, lane, 1.f);
  __syncthreads();
  // Y1 = dT T^T
  zero(sq);
  mma_acc<1, 4, false, false, C>(sq, sdT, LDC, m0, sT, LDC, c0, lane);
  strip_to_smem(sY1, LDC, m0, c0, sq, lane, 1.f);
  __syncthreads();
  // dL = strict_tril(-T^T Y1);  M = K U^T, L = M o E;  dg += rowsum(dL o L) - colsum(dL o L);  dM = dL o E
  {
    float mm[1][4][4];
    zero(sq);
    zero(mm);
    mma_acc<1, 4, true, true, C>(sq, sT, LDC, m0, sY1, LDC, c0, lane);
    mma_acc<1, 4, false, false, D>(mm, sK, LDT, m0, sU, LDT, c0, lane);
    float rs[2] = {0.f, 0.f}, cs[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      cs[nt][0] = cs[nt][1] = 0.f;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = m0 + g + 8 * hf, col = c0 + 8 * nt + 2 * t4;
        float o[2];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int cc = col + x;
          const float e = cc < row ? __expf(sg[row] - sg[cc]) : 0.f;
          const float dl = -sq[0][nt][2 * hf + x];
          const float pr = dl * mm[0][nt][2 * hf + x] * e;
          rs[hf] += pr;
          cs[nt][x] += pr;
          o[x] = dl * e;
        }
        *reinterpret_cast<uint32_t*>(sdM + row * LDC + col) = h2u(o[0], o[1]);
      }
    }
    add_row_col(sdgr + hw * C, scol + (warp & 3) * C, rs, cs, m0, c0, lane);
  }
  __syncthreads();

  // dK = Gamma T^T dW + dM U;  dg_t += gamma_t (T^T dW)_t . k_t
  float aK[1][8][4];
  zero(aK);
  mma_acc<1, 8, true, true, C>(aK, sT, LDC, m0, sNW, LDT, n0, lane);
  {
    float pa = 0.f, pb = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = n0 + 8 * nt + 2 * t4;
      const float2 ka = u2f(*reinterpret_cast<const uint32_t*>(sK + ra * LDT + col));
      const float2 kb = u2f(*reinterpret_cast<const uint32_t*>(sK + rb * LDT + col));
      pa += ka.x * aK[0][nt][0] + ka.y * aK[0][nt][1];
      pb += kb.x * aK[0][nt][2] + kb.y * aK[0][nt][3];
    }
    pa = quad_sum(pa);
    pb = quad_sum(pb);
    if (t4 == 0) {
      sdgr[hw * C + ra] += sgam[ra] * pa;
      sdgr[hw * C + rb] += sgam[rb] * pb;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      aK[0][nt][0] *= sgam[ra]; aK[0][nt][1] *= sgam[ra];
      aK[0][nt][2] *= sgam[rb]; aK[0][nt][3] *= sgam[rb];
    }
  }
  mma_acc<1, 8, false, true, C>(aK, sdM, LDC, m0, sU, LDT, n0, lane);
  // dQ += dP U;  dU += dP^T Q + dM^T K
  mma_acc<1, 8, false, true, C>(aQ, sdP, LDC, m0, sU, LDT, n0, lane);
  mma_acc<1, 8, true, true, C>(aU, sdP, LDC, m0, sQ, LDT, n0, lane);
  mma_acc<1, 8, true, true, C>(aU, sdM, LDC, m0, sK, LDT, n0, lane);
  // dV = T^T dR
  zero(acc);
  mma_acc<1, 8, true, true, C>(acc, sT, LDC, m0, sdR, LDT, n0, lane);

  // outputs (fp32, contiguous (B, T, H, DK) and (B, T, H, DV)), divided by the gradient scale; dq, dk, du
  // are added to the previous slice's when the state has more than 128 rows
  const bool has_u = p.u != nullptr;
  float pa = 0.f, pb = 0.f;  // dbeta partials: dU . k
  // A later slice adds its part with reduction stores (no load to wait on: a load of one output may
  // not pass a store to another that could alias it, so read-add-write serialised on every load);
  // one add per element per launch, after the first slice's store in stream order, so the sums are
  // the same bits in the same order as a read-add-write.
  auto put = [&](float* dst, float x, float y) {
    float2* q2 = reinterpret_cast<float2*>(dst);
    if (p.accum) atomicAdd(q2, make_float2(x, y));
    else *q2 = make_float2(x, y);
  };
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int row = hf ? rb : ra;
    if (row >= nvalid) continue;
    const int64_t tokrow = ((int64_t)b * p.T + t0 + row) * p.H + h;
    const int64_t o = tokrow * D, ov = tokrow * p.DVt + p.vofs;
    const float bt = sbeta[row];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = n0 + 8 * nt + 2 * t4;
      const int e0 = 2 * hf;
      put(p.dq + o + col, inv * aQ[0][nt][e0], inv * aQ[0][nt][e0 + 1]);
      *reinterpret_cast<float2*>(p.dv + ov + col) = make_float2(inv * acc[0][nt][e0], inv * acc[0][nt][e0 + 1]);
      if (has_u) {
        put(p.dk + o + col, inv * aK[0][nt][e0], inv * aK[0][nt][e0 + 1]);
        put(p.du + o + col, inv * aU[0][nt][e0], inv * aU[0][nt][e0 + 1]);
      } else {
        // u = beta k: dk += beta dU, dbeta = dU . k
        const float2 kk = u2f(*reinterpret_cast<const uint32_t*>(sK + row * LDT + col));
        put(p.dk + o + col, inv * (aK[0][nt][e0] + bt * aU[0][nt][e0]), inv * (aK[0][nt][e0 + 1] + bt * aU[0][nt][e0 + 1]));
        const float s = aU[0][nt][e0] * kk.x + aU[0][nt][e0 + 1] * kk.y;
        if (hf) pb += s; else pa += s;
      }
    }
  }
  if (!has_u) {
    pa = quad_sum(pa);
    pb = quad_sum(pb);
    if (t4 == 0) {
      sdb[hw * C + ra] += pa;
      sdb[hw * C + rb] += pb;
    }
  }
  __syncthreads();
  // gate gradients: the d_j = exp(g_C - g_j) and gamma_C factors, then dla = reverse cumsum of dg
  if (warp == 0) {
    float dd0 = sdd[lane] + sdd[C + lane], dd1 = sdd[lane + 32] + sdd[C + lane + 32];
    auto colsum = [&](int j) { return (scol[j] + scol[C + j]) + (scol[2 * C + j] + scol[3 * C + j]); };
    float dg0 = (sdgr[lane] + sdgr[C + lane]) - colsum(lane) - dd0 * sd[lane];
    float dg1 = (sdgr[lane + 32] + sdgr[C + lane + 32]) - colsum(lane + 32) - dd1 * sd[lane + 32];
    float tot = dd0 * sd[lane] + dd1 * sd[lane + 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (lane == 31) dg1 += tot + sgam[C - 1] * dot;
    // reverse inclusive scan over 64 values: lanes hold j = lane (dg0) and j = lane + 32 (dg1)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float x0 = __shfl_down_sync(0xffffffffu, dg0, o), x1 = __shfl_down_sync(0xffffffffu, dg1, o);
      if (lane + o < 32) {
        dg0 += x0;
        dg1 += x1;
      }
    }
    dg0 += __shfl_sync(0xffffffffu, dg1, 0);
    const int64_t gi = ((int64_t)b * p.T + t0) * p.H + h;
    auto put1 = [&](float* dst, float x) {
      if (p.accum) atomicAdd(dst, x);
      else *dst = x;
    };
    if (lane < nvalid) put1(p.dla + gi + (int64_t)lane * p.H, inv * dg0);
    if (lane + 32 < nvalid) put1(p.dla + gi + (int64_t)(lane + 32) * p.H, inv * dg1);
    if (!has_u) {
      if (lane < nvalid) put1(p.dbeta + gi + (int64_t)lane * p.H, inv * (sdb[lane] + sdb[C + lane]));
      if (lane + 32 < nvalid) put1(p.dbeta + gi + (int64_t)(lane + 32) * p.H, inv * (sdb[lane + 32] + sdb[C + lane + 32]));
    }
  }
}

// ---- host side ----------------------------------------------------------------------------------------
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Layout {
  size_t T, A, W, Uw, U, DU, dY, dR0, Pc, S, dS, g, amax, scale, total;
};

Layout layout(int64_t nch, int64_t bh) {
  Layout l;
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
  l.T = take((size_t)nch * C * C * 2);
  l.A = take((size_t)nch * C * C * 2);
  l.W = take((size_t)nch * C * D * 2);
  l.Uw = take((size_t)nch * C * D * 2);
  l.U = take((size_t)nch * C * D * 2);
  l.DU = take((size_t)nch * C * D * 2);
  l.dY = take((size_t)nch * C * D * 2);
  l.dR0 = take((size_t)nch * C * D * 2);
  l.Pc = take((size_t)nch * D * D * 2);
  l.S = take((size_t)nch * D * D * 2);
  l.dS = take((size_t)nch * D * D * 2);
  l.g = take((size_t)nch * C * 4);
  l.amax = take((size_t)bh * 4);
  l.scale = take((size_t)bh * 4);
  l.total = o;
  return l;
}

template <typename TI, typename TD>
int launch(const Params& p, cudaStream_t s) {
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)prep_kernel<TI, TD, false>, (int)PREP_SMEM},
                           {(const void*)prep_kernel<TI, TD, true>, (int)PREP_SMEM},
                           {(const void*)chain_kernel, (int)CHAIN_SMEM},
                           {(const void*)local_kernel<TI, TD>, (int)LOCAL_SMEM}}))
    return GDN_ERR_LAUNCH;
  const int64_t nch = (int64_t)p.NC * p.BH;
  // The prep and local blocks prefetch the chunk one resident wave ahead (0: no prefetch).
  Params pp = p, pl = p;
  int dev = 0, sms = 0, per_sm = 0;
  const bool have_sms =
      cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess;
  pp.pf = have_sms && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, prep_kernel<TI, TD, false>, NTHR, PREP_SMEM) == cudaSuccess
              ? sms * per_sm : 0;
  pl.pf = have_sms && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, local_kernel<TI, TD>, NTHR, LOCAL_SMEM) == cudaSuccess
              ? sms * per_sm : 0;
  if (cudaMemsetAsync(p.amax, 0, (size_t)p.BH * 4, s) != cudaSuccess) return GDN_ERR_LAUNCH;
  amax_kernel<TD><<<(unsigned)nch, NTHR, 0, s>>>(p);
  if (p.accum)  // a later state slice of the same call: the first slice's slice-independent products are in the workspace
    prep_kernel<TI, TD, true><<<(unsigned)nch, NTHR, PREP_SMEM, s>>>(pp);
  else
    prep_kernel<TI, TD, false><<<(unsigned)nch, NTHR, PREP_SMEM, s>>>(pp);
  chain_kernel<<<(unsigned)(2 * p.BH), NTHR, CHAIN_SMEM, s>>>(p);
  local_kernel<TI, TD><<<(unsigned)nch, NTHR, LOCAL_SMEM, s>>>(pl);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int esize(int dt) { return dt == GDN_DTYPE_BF16 ? 2 : (dt == GDN_DTYPE_F32 ? 4 : 0); }

int validate(const gdn_backward_args* a) {
  if (!a) return GDN_ERR_NULL;
  if (a->B <= 0 || a->H <= 0 || a->T < 0) return GDN_ERR_SHAPE;
  if (a->DK != D || a->DV < D || a->DV % D != 0 || a->DV > 8 * D) return GDN_ERR_UNSUPPORTED;
  if (a->B * a->H > (1LL << 24) || a->T > (1LL << 30)) return GDN_ERR_SHAPE;
  const int es = esize(a->in_dtype), ed = esize(a->dy_dtype);
  if (!es || !ed) return GDN_ERR_DTYPE;
  if (a->T > 0) {
    if (!a->q || !a->k || !a->v || !a->la || !a->dy || !a->dq || !a->dk || !a->dv || !a->dla) return GDN_ERR_NULL;
    if (a->u ? !a->du : (!a->beta || !a->dbeta)) return GDN_ERR_NULL;
  }
  auto al = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  auto st = [](const gdn_strides& s, int e) {
    return s.b >= 0 && s.t >= 0 && s.h >= 0 && (s.b * e) % 16 == 0 && (s.t * e) % 16 == 0 && (s.h * e) % 16 == 0;
  };
  if (!al(a->q) || !al(a->k) || !al(a->v) || !al(a->dy) || (a->u && !al(a->u))) return GDN_ERR_ALIGN;
  if (!st(a->sq, es) || !st(a->sk, es) || !st(a->sv, es) || !st(a->sdy, ed) || (a->u && !st(a->su, es)))
    return GDN_ERR_ALIGN;
  if (!al(a->dq) || !al(a->dk) || !al(a->dv) || (a->du && !al(a->du)) || (a->s0 && !al(a->s0)) ||
      (a->ds_T && !al(a->ds_T)) || (a->ds0 && !al(a->ds0)))
    return GDN_ERR_ALIGN;
  return GDN_OK;
}

}  // namespace bwd
}  // namespace gdn

using namespace gdn::bwd;

extern "C" {

int gdn_prefill_bwd_workspace_bytes(const gdn_backward_args* a, size_t* bytes) {
  if (!bytes) return GDN_ERR_NULL;
  const int st = validate(a);
  if (st != GDN_OK) return st;
  const int64_t nc = (a->T + C - 1) / C;
  *bytes = a->T > 0 ? layout(nc * a->B * a->H, a->B * a->H).total : 0;
  return GDN_OK;
}

int gdn_prefill_bwd(const gdn_backward_args* a, void* stream) {
  int st = validate(a);
  if (st != GDN_OK) return st;
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess || major != 10 || minor != 0)
    return GDN_ERR_DEVICE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t BH = a->B * a->H;
  if (a->T == 0) {  // no tokens: the initial-state gradient is the final-state gradient
    if (!a->ds0) return GDN_OK;
    const size_t n = (size_t)BH * a->DV * D * 4;
    const cudaError_t e = a->ds_T ? cudaMemcpyAsync(a->ds0, a->ds_T, n, cudaMemcpyDeviceToDevice, s) : cudaMemsetAsync(a->ds0, 0, n, s);
    return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
  }
  const int64_t NC = (a->T + C - 1) / C;
  const Layout l = layout(NC * BH, BH);
  if (!a->workspace || a->workspace_bytes < l.total) return GDN_ERR_WORKSPACE;
  if (((uintptr_t)a->workspace & 255u) != 0) return GDN_ERR_ALIGN;
  if (NC * BH > 0x7fffffffLL) return GDN_ERR_SHAPE;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  Params p{};
  p.q = a->q; p.k = a->k; p.u = a->u; p.v = a->v; p.dy = a->dy;
  p.beta = a->u ? nullptr : a->beta; p.la = a->la; p.s0 = a->s0; p.dsT = a->ds_T;
  p.dq = a->dq; p.dk = a->dk; p.du = a->du; p.dv = a->dv; p.dbeta = a->dbeta; p.dla = a->dla; p.ds0 = a->ds0;
  p.sq_b = a->sq.b; p.sq_t = a->sq.t; p.sq_h = a->sq.h;
  p.sk_b = a->sk.b; p.sk_t = a->sk.t; p.sk_h = a->sk.h;
  p.su_b = a->su.b; p.su_t = a->su.t; p.su_h = a->su.h;
  p.sv_b = a->sv.b; p.sv_t = a->sv.t; p.sv_h = a->sv.h;
  p.sd_b = a->sdy.b; p.sd_t = a->sdy.t; p.sd_h = a->sdy.h;
  p.T = (int)a->T; p.H = (int)a->H; p.NC = (int)NC; p.BH = (int)BH;
  p.wT = reinterpret_cast<__half*>(ws + l.T);
  p.wA = reinterpret_cast<__half*>(ws + l.A);
  p.wW = reinterpret_cast<__half*>(ws + l.W);
  p.wUw = reinterpret_cast<__half*>(ws + l.Uw);
  p.wS = reinterpret_cast<__half*>(ws + l.S);
  p.wdS = reinterpret_cast<__half*>(ws + l.dS);
  p.wU = reinterpret_cast<__half*>(ws + l.U);
  p.wDU = reinterpret_cast<__half*>(ws + l.DU);
  p.wdY = reinterpret_cast<__half*>(ws + l.dY);
  p.wdR0 = reinterpret_cast<__half*>(ws + l.dR0);
  p.wPc = reinterpret_cast<__half*>(ws + l.Pc);
  p.wg = reinterpret_cast<float*>(ws + l.g);
  p.amax = reinterpret_cast<unsigned*>(ws + l.amax);
  p.scale = reinterpret_cast<float*>(ws + l.scale);
  const bool in_bf = a->in_dtype == GDN_DTYPE_BF16, dy_bf = a->dy_dtype == GDN_DTYPE_BF16;
  // The rows of the state are independent: a DV > 128 state is 128-row slices, each a full backward of
  // its own v / dy columns (sharing q, k, u, la), whose dq, dk, du, dla, dbeta add up.
  p.DVt = (int)a->DV;
  const int es_in = in_bf ? 2 : 4, es_dy = dy_bf ? 2 : 4;
  for (int sl = 0; sl < (int)(a->DV / D); ++sl) {
    p.vofs = sl * D;
    p.accum = sl > 0;
    p.v = static_cast<const uint8_t*>(a->v) + (size_t)sl * D * es_in;
    p.dy = static_cast<const uint8_t*>(a->dy) + (size_t)sl * D * es_dy;
    int r;
    if (in_bf && dy_bf) r = launch<__nv_bfloat16, __nv_bfloat16>(p, s);
    else if (in_bf) r = launch<__nv_bfloat16, float>(p, s);
    else if (dy_bf) r = launch<float, __nv_bfloat16>(p, s);
    else r = launch<float, float>(p, s);
    if (r != GDN_OK) return r;
  }
  return GDN_OK;
}

}  // extern "C"
