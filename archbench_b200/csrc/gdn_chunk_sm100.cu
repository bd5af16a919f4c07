// Chunkwise-parallel gated delta rule on the 5th-generation tensor cores (sm_100a).
//
// Replaces archbench's chunked scan (archbench/layers/nsgdn.py:240-405: _wy_L_kernel, fla's
// solve_tril, recompute_w_u_fwd, chunk_gated_delta_rule_fwd_h and chunk_fwd_o -- five
// launches that round-trip L, A, w, u, h and v_new through HBM) with ONE kernel per call that
// keeps the fp32 state in TMEM across chunks and reads q, k, v, beta, la once and writes y once.
//
// Maths per (b, h) and 64-token chunk, state S (DV x DK) at chunk start, g = cumsum(la) inside
// the chunk, gamma_t = exp(g_t), u_t = beta_t k_t (or the given write vector):
//   L[t][j] = (k_t . u_j) exp(g_t - g_j)  (j <  t)      T = (I + L)^-1
//   A[t][j] = (q_t . u_j) exp(g_t - g_j)  (j <= t)
//   W = T diag(gamma) K,   U = T V,   R = U - W S^T           (rows r_t = v_t - alpha_t S_{t-1} k_t)
//   y_t = gamma_t S q_t + sum_j A[t][j] r_j
//   S  <- gamma_C S + sum_t exp(g_C - g_t) r_t u_t^T
// the WY form of the per-token loop of nsgdn.py:408-417 (derivation as in nsgdn.py:240-249).
//
// Tensor-core mapping.  Every product runs "transposed" so that its M dimension is a feature
// dimension of 128 (the TMEM lane count): state rows i (DV) or key columns d (DK) live on TMEM
// lanes, tokens on TMEM columns.  All MMA operands are fp16 in 128-byte-swizzled shared memory
// (bf16 inputs convert to fp16 exactly; computed operands are rounded once to fp16, whose 11-bit
// significand keeps the result within the 1e-3 relative tolerance where bf16 operands would
// not), accumulation is fp32 in TMEM:
//   G   = [K;Q] K^T (or [K;Q] U^T)   M=128 N=64  K=128   lanes 0-63 -> L rows, 64-127 -> A rows
//   W^T = K^T (T diag gamma)^T        M=128 N=64  K=64    A = K tile read MN-major
//   U^T = V^T T^T                     M=128 N=64  K=64    A = V tile read MN-major
//   R^T = U^T - S W^T                 M=128 N=64  K=128   A-negate, accumulates onto U^T
//   Z   = S Q^T                       M=128 N=64  K=128
//   Yi  = R^T A^T                     M=128 N=64  K=64
//   S  += (R diag w)^T K              M=128 N=128 K=64    B = K tile read MN-major
// One CTA of 128 threads owns one (b, h) sequence and walks its chunks in order; thread i owns
// TMEM lane i.  q/k/v tiles arrive by TMA (64 tokens x 64 features per box, no multicast) into a
// two-stage ring so the next chunk's loads overlap the current chunk's maths.
#include <cudaTypedefs.h>

#include "gdn_common.cuh"
#include "sm100_ptx.cuh"

namespace gdn {
namespace chunk {

constexpr int C = 64;     // tokens per chunk
constexpr int D = 128;    // DK = DV
constexpr int NT = 128;   // threads per CTA
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_G = 128, COL_W = 192, COL_R = 256, COL_Z = 320, COL_Y = 384;
constexpr int LSTRIDE = 65;  // padded row stride of the fp32 64x64 work matrices
constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;  // ~2 s at 1.9 GHz

constexpr uint32_t TILE = 8192;  // one 64 x 64 fp16/bf16 box
constexpr uint32_t union_bytes() {
  return ((2 * C * LSTRIDE * 4 + 3 * 256 * 4) + 1023) / 1024 * 1024;  // L, T, block scratch
}

template <bool HAS_U, int STAGES>
struct Layout {
  static constexpr uint32_t STAGE = HAS_U ? 8 * TILE : 6 * TILE;  // [K0][Q0][K1][Q1][V0][V1]([U0][U1])
  static constexpr uint32_t KQ = 0, V = 4 * TILE, U = 6 * TILE;   // offsets inside a stage
  static constexpr uint32_t S16 = STAGES * STAGE;                 // 128 x 128 fp16, 2 k-blocks
  static constexpr uint32_t W16 = S16 + 4 * TILE;                 // 128 (d) x 64 (t) fp16
  static constexpr uint32_t A16 = W16 + 2 * TILE;                 // 64 x 64
  static constexpr uint32_t T16 = A16 + TILE;
  static constexpr uint32_t TG16 = T16 + TILE;
  static constexpr uint32_t UNION = TG16 + TILE;                  // {L32, T32, M} | {R16, RP16}
  static constexpr uint32_t R16 = UNION, RP16 = UNION + 2 * TILE;
  static constexpr uint32_t SMALL = UNION + union_bytes();        // per-chunk vectors
  static constexpr uint32_t BARS = SMALL + 6 * C * 4;
  static constexpr uint32_t TOTAL = BARS + 64;
  static constexpr uint32_t DYN = TOTAL + 1024;                   // slack for 1024-B alignment
};

struct Params {
  const float* beta;
  const float* la;
  const float* s0;
  float* s_out;
  void* y;
  gdn_strides sy;
  int B, T, H;
  int srows;  // state rows per (b, h) of the full state (DV)
  int nsl;    // 128-row state slices per (b, h): CTA (bh, sl) serves rows [128 sl, 128 sl + 128)
};

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128-byte-row, 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Write 64 floats as one fp16 row of a swizzled tile.
__device__ __forceinline__ void store_row_f16(uint8_t* tile, uint32_t row, const float* v) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 q;
    q.x = pack_h2(v[c * 8 + 0], v[c * 8 + 1]);
    q.y = pack_h2(v[c * 8 + 2], v[c * 8 + 3]);
    q.z = pack_h2(v[c * 8 + 4], v[c * 8 + 5]);
    q.w = pack_h2(v[c * 8 + 6], v[c * 8 + 7]);
    *reinterpret_cast<uint4*>(tile + sw128(row, c)) = q;
  }
}

// (I + L)^-1 for a 64 x 64 strictly-lower L: 16 x 16 diagonal blocks by forward substitution,
// then the block rows below the diagonal level by level, T_ij = -D_i sum_{k=j}^{i-1} L_ik T_kj.
__device__ void invert_unit_lower(const float* __restrict__ L, float* __restrict__ T, float* __restrict__ M, int tid) {
  for (int i = tid; i < C * LSTRIDE; i += NT) T[i] = 0.f;
  __syncthreads();
  if (tid < 64) {
    const int o = (tid >> 4) * 16, j = tid & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s = 0.f;
#pragma unroll
      for (int m = 0; m < r; ++m) s = fmaf(L[(o + r) * LSTRIDE + o + m], x[m], s);
      x[r] = (r == j) ? 1.f : (r > j ? -s : 0.f);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) T[(o + r) * LSTRIDE + o + j] = x[r];
  }
  __syncthreads();
  for (int lvl = 1; lvl <= 3; ++lvl) {
    const int nblk = 4 - lvl;
    for (int e = tid; e < nblk * 256; e += NT) {
      const int blk = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      const int jb = blk, ib = blk + lvl;
      float s = 0.f;
      for (int kb = jb; kb < ib; ++kb) {
#pragma unroll
        for (int m = 0; m < 16; ++m)
          s = fmaf(L[(ib * 16 + r) * LSTRIDE + kb * 16 + m], T[(kb * 16 + m) * LSTRIDE + jb * 16 + cc], s);
      }
      M[blk * 256 + r * 16 + cc] = s;
    }
    __syncthreads();
    for (int e = tid; e < nblk * 256; e += NT) {
      const int blk = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      const int jb = blk, ib = blk + lvl;
      float s = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) s = fmaf(T[(ib * 16 + r) * LSTRIDE + ib * 16 + m], M[blk * 256 + m * 16 + cc], s);
      T[(ib * 16 + r) * LSTRIDE + jb * 16 + cc] = -s;
    }
    __syncthreads();
  }
}

__device__ int g_status = 0;  // sticky device-side status (GDN_ERR_TIMEOUT when a wait gave up)

template <bool HAS_U, int STAGES, typename TOut>
__global__ void __launch_bounds__(NT, 1)
    chunk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_u, const Params p) {
  using LY = Layout<HAS_U, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x / p.nsl, sl = blockIdx.x % p.nsl, b = bh / p.H, h = bh % p.H;
  const int dv0 = sl * D;  // first state row (v / y column) of this CTA's slice
  const int nchunks = (p.T + C - 1) / C;

  float* la_s = reinterpret_cast<float*>(sm + LY::SMALL);
  float* beta_s = la_s + C;
  float* g_s = beta_s + C;
  float* gam_s = g_s + C;
  float* w_s = gam_s + C;
  float* misc_s = w_s + C;  // [0] = gamma_C
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + LY::BARS);
  uint64_t* mma_bar = tma_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  float* L32 = reinterpret_cast<float*>(sm + LY::UNION);
  float* T32 = L32 + C * LSTRIDE;
  float* M32 = T32 + C * LSTRIDE;

  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < STAGES; ++s) ptx::mbar_init(&tma_bar[s], 1);
    ptx::mbar_init(mma_bar, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tensormap(&tm_q);
    ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_v);
    if (HAS_U) ptx::prefetch_tensormap(&tm_u);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t my = tmem + lane_base;

  // Initial state -> TMEM (thread i owns state row i).
  {
    const float* src = p.s0 ? p.s0 + ((int64_t)bh * p.srows + dv0 + tid) * D : nullptr;
#pragma unroll 1
    for (int c4 = 0; c4 < 4; ++c4) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 t4 = src ? *reinterpret_cast<const float4*>(src + c4 * 32 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = t4.x; v[i + 1] = t4.y; v[i + 2] = t4.z; v[i + 3] = t4.w;
      }
      ptx::tmem_st32(my + COL_S + c4 * 32, v);
    }
    ptx::tc_wait_st();
  }

  auto issue_tma = [&](int c, int s) {
    uint8_t* st = sm + s * LY::STAGE;
    uint64_t* bar = &tma_bar[s];
    ptx::mbar_arrive_expect_tx(bar, LY::STAGE);
    const int t0 = c * C;
    ptx::tma_load_4d(st + LY::KQ + 0 * TILE, &tm_k, bar, 0, h, t0, b);
    ptx::tma_load_4d(st + LY::KQ + 1 * TILE, &tm_q, bar, 0, h, t0, b);
    ptx::tma_load_4d(st + LY::KQ + 2 * TILE, &tm_k, bar, 64, h, t0, b);
    ptx::tma_load_4d(st + LY::KQ + 3 * TILE, &tm_q, bar, 64, h, t0, b);
    ptx::tma_load_4d(st + LY::V + 0 * TILE, &tm_v, bar, dv0, h, t0, b);
    ptx::tma_load_4d(st + LY::V + 1 * TILE, &tm_v, bar, dv0 + 64, h, t0, b);
    if (HAS_U) {
      ptx::tma_load_4d(st + LY::U + 0 * TILE, &tm_u, bar, 0, h, t0, b);
      ptx::tma_load_4d(st + LY::U + 1 * TILE, &tm_u, bar, 64, h, t0, b);
    }
  };

  const uint32_t sbase = ptx::smem_u32(sm);
  constexpr uint32_t ID_N64 = ptx::idesc_f16_f32(128, 64, false, false, false);
  constexpr uint32_t ID_N64_AMN = ptx::idesc_f16_f32(128, 64, true, false, false);
  constexpr uint32_t ID_N64_BMN_NEG = ptx::idesc_f16_f32(128, 64, false, true, true);
  constexpr uint32_t ID_N128_BMN = ptx::idesc_f16_f32(128, 128, false, true, false);

  uint32_t mma_phase = 0;
  bool abort = false;
  auto wait_mma = [&]() -> bool {
    const bool ok = ptx::mbar_wait_bounded(mma_bar, mma_phase, WAIT_LIMIT_CYCLES);
    if (ok) mma_phase ^= 1u;
    ptx::tc_fence_after();
    return ok;
  };

  if (tid == 0) issue_tma(0, 0);

  // Per chunk: TMA wait -> fp16 conversion + gates -> G -> L, A -> T -> W^T, U^T (overlapped
  // with S -> fp16) -> R^T, Z -> R, R diag(w) -> Yi, S update -> y.  Each MMA group is issued by
  // thread 0 and completes on mma_bar; every wait is bounded and a timeout aborts the CTA.
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int s = STAGES == 2 ? (c & 1) : 0;
    const int t0 = c * C;
    uint8_t* st = sm + s * LY::STAGE;
    const uint32_t st_a = sbase + s * LY::STAGE;
    if (tid == 0) {
      if (STAGES == 2 && c + 1 < nchunks) issue_tma(c + 1, s ^ 1);  // prefetch into the idle stage
      if (STAGES == 1 && c > 0) issue_tma(c, 0);                     // single stage: refill now
    }

    if (tid < C) {
      const int tok = t0 + tid;
      const bool valid = tok < p.T;
      const int64_t gi = ((int64_t)b * p.T + tok) * p.H + h;
      la_s[tid] = valid ? p.la[gi] : 0.f;
      beta_s[tid] = (!HAS_U && valid) ? p.beta[gi] : 0.f;
    }
    const uint32_t parity = STAGES == 2 ? ((c >> 1) & 1) : (c & 1);
    const bool tma_ok = ptx::mbar_wait_bounded(&tma_bar[s], parity, WAIT_LIMIT_CYCLES);
    if (__syncthreads_or(!tma_ok)) { abort = true; break; }

    // bf16 -> fp16 in place (elementwise, so the swizzled layout is preserved).
    {
      uint4* q4 = reinterpret_cast<uint4*>(st);
      const int n16 = LY::STAGE / 16;
      for (int i = tid; i < n16; i += NT) {
        uint4 r = q4[i];
        __nv_bfloat162* b2 = reinterpret_cast<__nv_bfloat162*>(&r);
        uint4 o;
        uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(b2[k]);
          o32[k] = pack_h2(f.x, f.y);
        }
        q4[i] = o;
      }
    }
    if (warp == 0) {  // chunk-local cumulative log-decay and the per-token weights
      float a0 = la_s[lane], a1 = la_s[lane + 32];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n0 = __shfl_up_sync(0xffffffffu, a0, o);
        const float n1 = __shfl_up_sync(0xffffffffu, a1, o);
        if (lane >= o) { a0 += n0; a1 += n1; }
      }
      a1 += __shfl_sync(0xffffffffu, a0, 31);
      const float gC = __shfl_sync(0xffffffffu, a1, 31);
      g_s[lane] = a0;
      g_s[lane + 32] = a1;
      gam_s[lane] = expf(a0);
      gam_s[lane + 32] = expf(a1);
      const float b0 = HAS_U ? 1.f : beta_s[lane], b1 = HAS_U ? 1.f : beta_s[lane + 32];
      w_s[lane] = b0 * expf(gC - a0);
      w_s[lane + 32] = b1 * expf(gC - a1);
      if (lane == 0) misc_s[0] = expf(gC);
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();

    // ---- G = [K;Q] K^T (or U^T) ----
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t kb = k >> 2, kk = k & 3;
        const uint64_t a = ptx::sdesc_sw128(st_a + LY::KQ + kb * 2 * TILE + kk * 32, 16, 1024);
        const uint64_t bdesc = HAS_U ? ptx::sdesc_sw128(st_a + LY::U + kb * TILE + kk * 32, 16, 1024)
                                     : ptx::sdesc_sw128(st_a + LY::KQ + kb * 2 * TILE + kk * 32, 16, 1024);
        ptx::mma_f16_ss(tmem + COL_G, a, bdesc, ID_N64, k > 0);
      }
      ptx::mma_commit(mma_bar);
    }
    if (__syncthreads_or(!wait_mma())) { abort = true; break; }

    // ---- L (threads 0-63) and A (threads 64-127) rows from G ----
    {
      float gv[64];
      ptx::tmem_ld32(my + COL_G, *reinterpret_cast<float(*)[32]>(gv));
      ptx::tmem_ld32(my + COL_G + 32, *reinterpret_cast<float(*)[32]>(gv + 32));
      ptx::tc_wait_ld();
      const int t = tid & 63;
      const float gt = g_s[t];
      if (tid < 64) {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float coef = (HAS_U ? 1.f : beta_s[j]) * expf(gt - g_s[j]);
          L32[t * LSTRIDE + j] = (j < t) ? gv[j] * coef : 0.f;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float coef = (HAS_U ? 1.f : beta_s[j]) * expf(gt - g_s[j]);
          gv[j] = (j <= t) ? gv[j] * coef : 0.f;
        }
        store_row_f16(sm + LY::A16, t, gv);
      }
    }
    ptx::tc_fence_before();
    __syncthreads();
    invert_unit_lower(L32, T32, M32, tid);
    {
      const int t = tid & 63;
      float row[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) row[j] = T32[t * LSTRIDE + j] * (tid < 64 ? 1.f : gam_s[j]);
      store_row_f16(sm + (tid < 64 ? LY::T16 : LY::TG16), t, row);
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();

    // ---- W^T = K^T (T diag gamma)^T ; U^T = V^T T^T (into the R accumulator) ----
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ak = ptx::sdesc_sw128(st_a + LY::KQ + k * 2048, 2 * TILE, 1024);
        const uint64_t bt = ptx::sdesc_sw128(sbase + LY::TG16 + k * 32, 16, 1024);
        ptx::mma_f16_ss(tmem + COL_W, ak, bt, ID_N64_AMN, k > 0);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t av = ptx::sdesc_sw128(st_a + LY::V + k * 2048, TILE, 1024);
        const uint64_t bt = ptx::sdesc_sw128(sbase + LY::T16 + k * 32, 16, 1024);
        ptx::mma_f16_ss(tmem + COL_R, av, bt, ID_N64_AMN, k > 0);
      }
      ptx::mma_commit(mma_bar);
    }
    // Meanwhile: S16 <- fp16(S), and S <- gamma_C S in TMEM (the update MMA accumulates onto it).
    {
      const float gC = misc_s[0];
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        float v[32];
        ptx::tmem_ld32(my + COL_S + c4 * 32, v);
        ptx::tc_wait_ld();
        uint8_t* half = sm + LY::S16 + (c4 >> 1) * 2 * TILE;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 pk;
          pk.x = pack_h2(v[q * 8 + 0], v[q * 8 + 1]);
          pk.y = pack_h2(v[q * 8 + 2], v[q * 8 + 3]);
          pk.z = pack_h2(v[q * 8 + 4], v[q * 8 + 5]);
          pk.w = pack_h2(v[q * 8 + 6], v[q * 8 + 7]);
          *reinterpret_cast<uint4*>(half + sw128(tid, (c4 & 1) * 4 + q)) = pk;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= gC;
        ptx::tmem_st32(my + COL_S + c4 * 32, v);
      }
      ptx::tc_wait_st();
    }
    if (__syncthreads_or(!wait_mma())) { abort = true; break; }
    {
      float wv[64];
      ptx::tmem_ld32(my + COL_W, *reinterpret_cast<float(*)[32]>(wv));
      ptx::tmem_ld32(my + COL_W + 32, *reinterpret_cast<float(*)[32]>(wv + 32));
      ptx::tc_wait_ld();
      store_row_f16(sm + LY::W16, tid, wv);
    }
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();

    // ---- R^T = U^T - S W^T ; Z = S Q^T ----
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t kb = k >> 2, kk = k & 3;
        const uint64_t as = ptx::sdesc_sw128(sbase + LY::S16 + kb * 2 * TILE + kk * 32, 16, 1024);
        const uint64_t bw = ptx::sdesc_sw128(sbase + LY::W16 + k * 2048, 16, 1024);
        ptx::mma_f16_ss(tmem + COL_R, as, bw, ID_N64_BMN_NEG, 1);
        const uint64_t bq = ptx::sdesc_sw128(st_a + LY::KQ + TILE + kb * 2 * TILE + kk * 32, 16, 1024);
        ptx::mma_f16_ss(tmem + COL_Z, as, bq, ID_N64, k > 0);
      }
      ptx::mma_commit(mma_bar);
    }
    if (__syncthreads_or(!wait_mma())) { abort = true; break; }
    {
      float rv[64];
      ptx::tmem_ld32(my + COL_R, *reinterpret_cast<float(*)[32]>(rv));
      ptx::tmem_ld32(my + COL_R + 32, *reinterpret_cast<float(*)[32]>(rv + 32));
      ptx::tc_wait_ld();
      store_row_f16(sm + LY::R16, tid, rv);
#pragma unroll
      for (int t = 0; t < 64; ++t) rv[t] *= w_s[t];
      store_row_f16(sm + LY::RP16, tid, rv);
    }
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();

    // ---- Yi = R^T A^T ; S += (R diag w)^T K (or U) ----
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ar = ptx::sdesc_sw128(sbase + LY::R16 + k * 32, 16, 1024);
        const uint64_t ba = ptx::sdesc_sw128(sbase + LY::A16 + k * 32, 16, 1024);
        ptx::mma_f16_ss(tmem + COL_Y, ar, ba, ID_N64, k > 0);
        const uint64_t ap = ptx::sdesc_sw128(sbase + LY::RP16 + k * 32, 16, 1024);
        const uint64_t bk = HAS_U ? ptx::sdesc_sw128(st_a + LY::U + k * 2048, TILE, 1024)
                                  : ptx::sdesc_sw128(st_a + LY::KQ + k * 2048, 2 * TILE, 1024);
        ptx::mma_f16_ss(tmem + COL_S, ap, bk, ID_N128_BMN, 1);
      }
      ptx::mma_commit(mma_bar);
    }
    if (__syncthreads_or(!wait_mma())) { abort = true; break; }

    // ---- y_t = gamma_t Z + Yi (thread i writes feature i of every token) ----
    {
      TOut* yb = static_cast<TOut*>(p.y) + (int64_t)b * p.sy.b + (int64_t)h * p.sy.h + dv0 + tid;
      const int nvalid = min(C, p.T - t0);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float z[32], yi[32];
        ptx::tmem_ld32(my + COL_Z + half * 32, z);
        ptx::tmem_ld32(my + COL_Y + half * 32, yi);
        ptx::tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int t = half * 32 + j;
          if (t < nvalid) store_as(yb + (int64_t)(t0 + t) * p.sy.t, fmaf(gam_s[t], z[j], yi[j]));
        }
      }
    }
    ptx::tc_fence_before();
    __syncthreads();
  }

  if (!abort && p.s_out != nullptr) {
    float* dst = p.s_out + ((int64_t)bh * p.srows + dv0 + tid) * D;
#pragma unroll 1
    for (int c4 = 0; c4 < 4; ++c4) {
      float v[32];
      ptx::tmem_ld32(my + COL_S + c4 * 32, v);
      ptx::tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + c4 * 32 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  }
  if (abort && tid == 0) atomicExch(&g_status, GDN_ERR_TIMEOUT);
  // On abort an MMA or TMA may still be in flight; give it a bounded chance to land before
  // the TMEM it writes is released.
  if (abort && tid == 0) {
    ptx::mbar_wait_bounded(mma_bar, mma_phase, WAIT_LIMIT_CYCLES);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 0) ptx::tmem_dealloc(tmem, TMEM_COLS);
}

// ---- host side -------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [B][T][H][D] bf16 view -> 4-D tensor map (d, h, t, b), box 64 x 1 x 64 x 1, 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, const gdn_prefill_args* a, const gdn_strides& s, int64_t width = D) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)width, (cuuint64_t)a->H, (cuuint64_t)a->T, (cuuint64_t)a->B};
  cuuint64_t strides[3] = {(cuuint64_t)s.h * 2, (cuuint64_t)s.t * 2, (cuuint64_t)s.b * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)C, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool HAS_U, int STAGES, typename TOut>
int launch(const gdn_prefill_args* a, cudaStream_t stream) {
  using LY = Layout<HAS_U, STAGES>;
  CUtensorMap mq, mk, mv, mu;
  if (!make_map(&mq, a->q, a, a->sq) || !make_map(&mk, a->k, a, a->sk) || !make_map(&mv, a->v, a, a->sv, a->DV))
    return GDN_ERR_LAUNCH;
  if (HAS_U) {
    if (!make_map(&mu, a->u, a, a->su)) return GDN_ERR_LAUNCH;
  } else {
    mu = mk;
  }
  auto kern = chunk_kernel<HAS_U, STAGES, TOut>;
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)kern, (int)(LY::DYN)}})) return GDN_ERR_LAUNCH;
  Params p;
  p.beta = a->beta; p.la = a->la; p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.sy = a->sy;
  p.srows = (int)a->DV;
  // The state's rows are independent: a DV = 128 n state runs as n CTAs per (b, h), each over 128 rows
  // with its own v columns, y columns and state rows (q, k, u and the gates shared, read through L2 by
  // the n neighbouring CTAs), all in one launch.
  p.nsl = (int)(a->DV / D);
  p.s0 = a->s0;
  p.s_out = a->s_out;
  p.y = a->y;
  kern<<<(unsigned)(a->B * a->H * p.nsl), NT, LY::DYN, stream>>>(mq, mk, mv, mu, p);
  if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  return GDN_OK;
}

bool tma_ok(const void* ptr, const gdn_strides& s) {
  auto a16 = [](int64_t x) { return x > 0 && (x * 2) % 16 == 0 && x * 2 < (1LL << 40); };
  return ptr && ((uintptr_t)ptr % 16 == 0) && a16(s.h) && a16(s.t) && a16(s.b);
}

}  // namespace chunk
}  // namespace gdn

// The chunked path: the warp-specialised kernel (gdn_chunk_ws_sm100.cu) for DV any multiple of
// 128, with u = beta k or an explicit write vector u (nsgdn n_steps > 1), where y's rows are 16-byte
// aligned (it stores y by TMA); this single-warp-group kernel for an explicit u with any y strides
// (one CTA per 128 state rows, all in one launch).  Both need 16-byte-aligned q/k/u/v rows for TMA.
bool gdn_chunk_supported(const gdn_prefill_args* a) {
  using namespace gdn::chunk;
  if (a->in_dtype != GDN_DTYPE_BF16 || a->DK != D || a->T < 1) return false;
  if (!tma_ok(a->q, a->sq) || !tma_ok(a->k, a->sk) || !tma_ok(a->v, a->sv)) return false;
  if (a->u && !tma_ok(a->u, a->su)) return false;
  if ((a->s0 && (uintptr_t)a->s0 % 16) || (a->s_out && (uintptr_t)a->s_out % 16)) return false;
  if (a->u) return a->DV % D == 0 && a->DV <= 8 * D;
  return gdn_chunk_ws_supported(a);
}

int gdn_launch_chunk_sm100(const gdn_prefill_args* a, cudaStream_t stream) {
  using namespace gdn::chunk;
  if (gdn_chunk_ws_supported(a)) return gdn_launch_chunk_ws(a, stream);
  return a->out_dtype == GDN_DTYPE_BF16 ? launch<true, 1, __nv_bfloat16>(a, stream) : launch<true, 1, float>(a, stream);
}

int gdn_chunk_read_status(int* out, int reset) {
  int ws = 0;
  int st = gdn_chunk_ws_read_status(&ws, reset);
  if (st != GDN_OK) return st;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::chunk::g_status, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (reset) {
    int z = 0;
    if (cudaMemcpyToSymbol(gdn::chunk::g_status, &z, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  }
  *out = v != 0 ? v : ws;
  return GDN_OK;
}
