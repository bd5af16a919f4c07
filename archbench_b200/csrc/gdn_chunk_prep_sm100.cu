// Chunk products of the gated delta rule for every chunk at once (sm_100a): the state-independent
// half of the chunkwise prefill, written to a workspace for the state-only chunk kernel.
//
// Per (b, h, 64-token chunk), with g the chunk-local cumsum of la and gamma = exp(g) (the WY form of
// archbench/layers/nsgdn.py:240-249):
//
//   G = [K;Q] U^T  (U = beta K unless the write vectors are given)
//   L = strict_tril(K U^T o E),  A = tril(Q U^T o E),  E_tj = exp(g_t - g_j)
//   T = (I + L)^-1,  T Gamma
//
// A, T and T Gamma leave as three fp16 64 x 64 tiles in the 128-byte-swizzled layout the state
// CTA's MMAs read (24 KB per chunk, [A16][T16][TG16]), so that the state-only kernel takes them
// with one bulk copy.  The arithmetic is the prep pipeline of the two-CTA cluster kernel
// (gdn_chunk_pair_sm100.cu), operation for operation: the products are bitwise the same.
//
// CTAs of 128 threads, as many as fit on the GPU at once, each looping over chunks (no chunk depends
// on another) with the next chunk's tiles prefetched into L2.  Tile loads by TMA (no multicast); the G MMA on tcgen05
// (bf16 operands as loaded, fp32 accumulator in 64 TMEM columns); T by fp32 forward substitution on
// 16 x 16 diagonal blocks and fp16 mma.sync block-column merges (gdn_tiles.cuh).
#include <algorithm>

#include "gdn_tiles.cuh"

namespace gdn {
namespace prep {

using namespace gdn::tiles;

constexpr int NT = 128;
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clocks
constexpr uint32_t PS_BYTES = 3 * TILE;         // [A16][T16][TG16]

// Shared-memory map (bytes from a 1024-aligned base).  The staged products reuse the tile
// buffer once the G MMA, its only reader, has completed.  With u tiles (OVERLAY) the buffer is
// 48 KB: the fp16 L matrix, the diagonal blocks and the decay tables then take its last 24 KB too
// (the tables computed after the MMA), which keeps a CTA at ~50 KB and four of them on an SM.
template <bool HAS_U>
struct Map {
  static constexpr bool OVERLAY = HAS_U;
  static constexpr uint32_t KQ = 0;                                  // [K0][Q0][K1][Q1] (+ [U0][U1])
  static constexpr uint32_t KQ_BYTES = (HAS_U ? 6 : 4) * TILE;
  static constexpr uint32_t ST = 0;                                  // staged [A16][T16][TG16]
  static constexpr uint32_t L16 = OVERLAY ? ST + PS_BYTES : KQ + KQ_BYTES;  // 64 rows x LD16 bytes
  static constexpr uint32_t LDIAG = L16 + 64 * LD16;                 // 4 x 16 x LDG floats
  static constexpr uint32_t EXPT = LDIAG + 4 * 16 * LDG * 4;         // 64 + 4x64 + 4x16x20 floats
  static constexpr uint32_t EXPT_END = EXPT + (64 + 4 * 64 + 4 * 16 * 20) * 4;
  static constexpr uint32_t GS = OVERLAY ? KQ + KQ_BYTES : EXPT_END;  // beta[64], g[64], gamma[64]
  static constexpr uint32_t BARS = GS + 3 * C * 4;                   // 2 mbarriers, TMEM slot, abort flag
  static constexpr uint32_t TOTAL = BARS + 32;
  static constexpr uint32_t DYN = TOTAL + 1024;
  static_assert(KQ_BYTES >= PS_BYTES, "staging fits in the tile buffer");
  static_assert(!OVERLAY || EXPT_END <= KQ + KQ_BYTES, "the overlaid tables fit in the tile buffer");
  static_assert(L16 % 16 == 0 && BARS % 8 == 0, "alignment");
};

struct Params {
  const float* beta;  // NULL when the write vectors are given
  const float* la;
  uint8_t* prod;      // [B * H][NCt] x PS_BYTES
  int B, T, H, NCt;
};

__device__ int g_status = 0;

template <bool HAS_U>
__global__ void __launch_bounds__(NT)
    prep_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_u, const Params p) {
  using M = Map<HAS_U>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntask = p.B * p.H * p.NCt;

  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + M::BARS);  // 0: tiles, 1: G
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + M::BARS + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + M::BARS + 20);
  float* eT = reinterpret_cast<float*>(sm + M::EXPT);  // [64]      exp(g_t - g_{16 floor(t/16)})
  float* eJ = eT + C;                                   // [4][64]   beta_j exp(g_{16b} - g_j), j < 16b
  float* Ed = eJ + 4 * C;                               // [4][16][20] beta_{16b+c} exp(g_{16b+r} - g_{16b+c}), c <= r
  float* beta_s = reinterpret_cast<float*>(sm + M::GS);
  float* g_s = beta_s + C;
  float* gam_s = g_s + C;
  uint8_t* st = sm + M::ST;

  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, 64);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    ptx::mbar_init(&bars[0], 1);
    ptx::mbar_init(&bars[1], 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tensormap(&tm_q);
    ptx::prefetch_tensormap(&tm_k);
    if (HAS_U) ptx::prefetch_tensormap(&tm_u);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t my = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM lane quarter
  const uint64_t D_K = ptx::sdesc_sw128(sb, 16, 1024);
  constexpr uint32_t ID_G = ptx::idesc_bf16_f32(128, 64);

  // Tile coordinates (b, h, t0) of a task.
  auto coords = [&](int task, int& b, int& h, int& t0) {
    const int bh = task / p.NCt, c = task - bh * p.NCt;
    b = bh / p.H;
    h = bh - b * p.H;
    t0 = c * C;
  };

  // A persistent loop over the chunks: while one chunk is worked on, the next one's tiles are pulled
  // into L2, so that its TMA load (issued once the staged products have left the tile buffer they
  // share) waits on L2 rather than on HBM.
  uint32_t it = 0;
#pragma unroll 1
  for (int task = blockIdx.x; task < ntask; task += gridDim.x, ++it) {
    const uint32_t ph = it & 1u;
    int b, h, t0;
    coords(task, b, h, t0);
    if (tid == 0) {
      ptx::mbar_arrive_expect_tx(&bars[0], M::KQ_BYTES);
      ptx::tma_load_4d(sm + M::KQ + 0 * TILE, &tm_k, &bars[0], 0, h, t0, b);
      ptx::tma_load_4d(sm + M::KQ + 1 * TILE, &tm_q, &bars[0], 0, h, t0, b);
      ptx::tma_load_4d(sm + M::KQ + 2 * TILE, &tm_k, &bars[0], 64, h, t0, b);
      ptx::tma_load_4d(sm + M::KQ + 3 * TILE, &tm_q, &bars[0], 64, h, t0, b);
      if (HAS_U) {
        ptx::tma_load_4d(sm + M::KQ + 4 * TILE, &tm_u, &bars[0], 0, h, t0, b);
        ptx::tma_load_4d(sm + M::KQ + 5 * TILE, &tm_u, &bars[0], 64, h, t0, b);
      }
      if (task + (int)gridDim.x < ntask) {
        int nb, nh, nt0;
        coords(task + (int)gridDim.x, nb, nh, nt0);
        ptx::tma_prefetch_4d(&tm_k, 0, nh, nt0, nb);
        ptx::tma_prefetch_4d(&tm_k, 64, nh, nt0, nb);
        ptx::tma_prefetch_4d(&tm_q, 0, nh, nt0, nb);
        ptx::tma_prefetch_4d(&tm_q, 64, nh, nt0, nb);
        if (HAS_U) {
          ptx::tma_prefetch_4d(&tm_u, 0, nh, nt0, nb);
          ptx::tma_prefetch_4d(&tm_u, 64, nh, nt0, nb);
        }
      }
    }
    if (warp == 1) {  // chunk-local cumulative log-decay; beta = 1 with explicit write vectors
      float la0 = 0.f, la1 = 0.f, be0 = 0.f, be1 = 0.f;
      const int64_t gi = ((int64_t)b * p.T + t0) * p.H + h;
      if (t0 + lane < p.T) {
        la0 = p.la[gi + (int64_t)lane * p.H];
        be0 = HAS_U ? 1.f : p.beta[gi + (int64_t)lane * p.H];
      }
      if (t0 + lane + 32 < p.T) {
        la1 = p.la[gi + (int64_t)(lane + 32) * p.H];
        be1 = HAS_U ? 1.f : p.beta[gi + (int64_t)(lane + 32) * p.H];
      }
      float a0 = la0, a1 = la1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n0 = __shfl_up_sync(0xffffffffu, a0, o);
        const float n1 = __shfl_up_sync(0xffffffffu, a1, o);
        if (lane >= o) {
          a0 += n0;
          a1 += n1;
        }
      }
      a1 += __shfl_sync(0xffffffffu, a0, 31);
      beta_s[lane] = be0;
      beta_s[lane + 32] = be1;
      g_s[lane] = a0;
      g_s[lane + 32] = a1;
      gam_s[lane] = expf(a0);
      gam_s[lane + 32] = expf(a1);
    }
    bool fail = false;
    if (warp == 0) {  // G = [K;Q] K^T (or [K;Q] U^T) from the bf16 tiles as loaded
      if (lane == 0) fail = !ptx::mbar_wait_abortable(&bars[0], ph, WAIT_LIMIT, abort_flag);
      fail = __shfl_sync(0xffffffffu, fail, 0);
      if (!fail) {
        ptx::tc_fence_after();
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = D_K + (uint64_t)((M::KQ + (kk >> 2) * 2 * TILE + (kk & 3) * 32) >> 4);
          const uint64_t bu = HAS_U ? D_K + (uint64_t)((M::KQ + (4 + (kk >> 2)) * TILE + (kk & 3) * 32) >> 4) : a;
          ptx::mma_f16_ss_elect(tmem, a, bu, ID_G, kk > 0);
        }
        ptx::mma_commit_elect(&bars[1]);
      }
    }
    if (ptx::named_bar_or(1, NT, fail)) {  // the tiles did not arrive in time: no MMA was issued on them
      if (tid == 0) {
        ptx::mbar_wait_bounded(&bars[0], ph, WAIT_LIMIT);  // the loads may still land in this CTA's memory
        atomicExch(&g_status, GDN_ERR_TIMEOUT);
      }
      break;
    }
    // Decay tables: 1,344 exponentials per chunk instead of one per (t, j) pair; every factor is exp
    // of a non-positive number, so none overflows whatever the decay.  Computed while the G MMA
    // runs, or after it where they overlay the tile buffer it reads.
    auto tables = [&]() {
#pragma unroll 1
      for (int e = tid; e < 5 * C; e += NT) {
        if (e < C) {
          eT[e] = __expf(g_s[e] - g_s[e & ~15]);
        } else {
          const int bb = (e - C) >> 6, j = (e - C) & 63;
          eJ[bb * C + j] = (bb > 0 && j < 16 * bb) ? beta_s[j] * __expf(g_s[16 * bb] - g_s[j]) : 0.f;
        }
      }
#pragma unroll 1
      for (int n = 0; n < 8; ++n) {
        const int e = tid + NT * n;  // 1024 diagonal-block entries
        const int bb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
        Ed[(bb * 16 + r) * 20 + cc] = cc <= r ? beta_s[16 * bb + cc] * __expf(g_s[16 * bb + r] - g_s[16 * bb + cc]) : 0.f;
      }
    };
    if (!M::OVERLAY) tables();
    if (tid == 0) fail = !ptx::mbar_wait_abortable(&bars[1], ph, WAIT_LIMIT, abort_flag);
    if (ptx::named_bar_or(1, NT, fail)) {  // the MMA did not complete: drain it before TMEM is freed
      if (tid == 0) {
        ptx::mbar_wait_bounded(&bars[1], ph, WAIT_LIMIT);
        atomicExch(&g_status, GDN_ERR_TIMEOUT);
      }
      break;
    }
    if (M::OVERLAY) {
      tables();
      __syncthreads();
    }
    ptx::tc_fence_after();
    // Row tid of G: rows 0-63 give L (strictly lower), rows 64-127 give A (lower with diagonal), one
    // 16-column block at a time.
    {
      const int t = tid & 63, tb = t >> 4;
      const bool is_l = tid < 64;
      const float et = eT[t];
#pragma unroll 1
      for (int jb = 0; jb < 4; ++jb) {
        float gv[16], e[16];
        ptx::tmem_ld16(my + 16 * jb, gv);
        const float4* src4 = jb < tb ? reinterpret_cast<const float4*>(eJ + tb * C + 16 * jb)
                                     : reinterpret_cast<const float4*>(Ed + (tb * 16 + (t & 15)) * 20);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 f = src4[v];
          e[4 * v] = f.x; e[4 * v + 1] = f.y; e[4 * v + 2] = f.z; e[4 * v + 3] = f.w;
        }
        const float sc = jb < tb ? et : (jb == tb ? 1.f : 0.f);
        ptx::tc_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          float ej = e[jj] * sc;
          if (is_l && 16 * jb + jj == t) ej = 0.f;
          gv[jj] *= ej;
        }
        uint4 h0, h1;
        h0.x = pack_h2(gv[0], gv[1]);   h0.y = pack_h2(gv[2], gv[3]);
        h0.z = pack_h2(gv[4], gv[5]);   h0.w = pack_h2(gv[6], gv[7]);
        h1.x = pack_h2(gv[8], gv[9]);   h1.y = pack_h2(gv[10], gv[11]);
        h1.z = pack_h2(gv[12], gv[13]); h1.w = pack_h2(gv[14], gv[15]);
        if (is_l) {
          uint8_t* lrow = sm + M::L16 + t * LD16 + jb * 32;
          *reinterpret_cast<uint4*>(lrow) = h0;
          *reinterpret_cast<uint4*>(lrow + 16) = h1;
          if (jb == tb) {  // the diagonal block also in fp32, for the substitution
            float* drow = reinterpret_cast<float*>(sm + M::LDIAG) + (tb * 16 + (t & 15)) * LDG;
#pragma unroll
            for (int q = 0; q < 16; q += 4)
              *reinterpret_cast<float4*>(drow + q) = make_float4(gv[q], gv[q + 1], gv[q + 2], gv[q + 3]);
          }
        } else {  // A16 row t, columns 16 jb .. 16 jb + 15
          *reinterpret_cast<uint4*>(st + sw128((uint32_t)t, 2 * jb)) = h0;
          *reinterpret_cast<uint4*>(st + sw128((uint32_t)t, 2 * jb + 1)) = h1;
        }
      }
    }
    ptx::tc_fence_before();  // G is read out: the next chunk's MMA may overwrite it after the barrier
    __syncthreads();
    if (tid < 64) {
      // D_b = (I + L_bb)^-1, one column per thread; right-looking fp32 forward substitution.
      const int bb = tid >> 4, j = tid & 15;
      const float* Lb = reinterpret_cast<const float*>(sm + M::LDIAG) + bb * 16 * LDG;
      float x[16], acc[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        x[m] = (m == j) ? 1.f : (m > j ? -acc[m] : 0.f);
#pragma unroll
        for (int r = m + 1; r < 16; ++r) acc[r] = fmaf(Lb[r * LDG + m], x[m], acc[r]);
      }
      __half* l16 = reinterpret_cast<__half*>(sm + M::L16);
#pragma unroll
      for (int r = 0; r < 16; ++r) l16[(bb * 16 + r) * (LD16 / 2) + bb * 16 + j] = __float2half_rn(x[r]);
    }
    __syncthreads();
    merge_column_any<false>(warp, sb + M::L16, sb + M::ST + TILE, 0u, sb + M::ST + 2 * TILE, gam_s, lane);
    ptx::fence_proxy_async_smem();  // the staged products, for the bulk store
    __syncthreads();
    if (tid == 0) {
      // The staging shares the tile buffer: the next chunk's tile load waits until this store has
      // read it (the store's completion is awaited before the CTA exits).
      ptx::bulk_store(p.prod + (int64_t)task * PS_BYTES, st, PS_BYTES);
      ptx::bulk_commit();
      ptx::bulk_wait_read0();
    }
    ptx::tc_fence_after();
  }
  if (tid == 0) ptx::bulk_wait0();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 0) ptx::tmem_dealloc(tmem, 64);
}

template <bool HAS_U>
int launch(const gdn_prefill_args* a, uint8_t* prod, cudaStream_t stream) {
  CUtensorMap mq, mk, mu;
  if (!make_map(&mq, a->q, a->DK, a, a->sq) || !make_map(&mk, a->k, a->DK, a, a->sk)) return GDN_ERR_LAUNCH;
  if (HAS_U) {
    if (!make_map(&mu, a->u, a->DK, a, a->su)) return GDN_ERR_LAUNCH;
  } else {
    mu = mk;
  }
  auto kern = prep_kernel<HAS_U>;
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)kern, (int)Map<HAS_U>::DYN}})) return GDN_ERR_LAUNCH;
  Params p;
  p.beta = a->beta;
  p.la = a->la;
  p.prod = prod;
  p.B = (int)a->B;
  p.T = (int)a->T;
  p.H = (int)a->H;
  p.NCt = (int)((a->T + C - 1) / C);
  const int64_t ntask = a->B * a->H * (int64_t)p.NCt;
  if (ntask <= 0 || ntask > 0x7fffffff) return GDN_ERR_SHAPE;
  // A persistent grid: as many CTAs as fit at once (shared memory bounds them), each looping over
  // chunks with a stride of the grid.
  int dev = 0, sms = 0, smem_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  // CTAs per SM by shared memory (1 KB of it reserved per CTA); 4 x 64 TMEM columns at most.
  const int per_sm = std::min(4, std::max(1, smem_sm / (int)(Map<HAS_U>::DYN + 1024)));
  const int64_t grid = std::min<int64_t>(ntask, (int64_t)std::max(1, sms) * per_sm);
  kern<<<(unsigned)grid, NT, Map<HAS_U>::DYN, stream>>>(mq, mk, mu, p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace prep
}  // namespace gdn

size_t gdn_chunk_prep_bytes(const gdn_prefill_args* a) {
  return (size_t)(a->B * a->H) * (size_t)((a->T + 63) / 64) * gdn::prep::PS_BYTES;
}

int gdn_launch_chunk_prep(const gdn_prefill_args* a, void* prod, cudaStream_t stream) {
  if (prod == nullptr || (uintptr_t)prod % 16) return GDN_ERR_ALIGN;
  uint8_t* pb = static_cast<uint8_t*>(prod);
  return a->u != nullptr ? gdn::prep::launch<true>(a, pb, stream) : gdn::prep::launch<false>(a, pb, stream);
}

int gdn_chunk_prep_read_status(int* out, int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::prep::g_status, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (reset) {
    int z = 0;
    if (cudaMemcpyToSymbol(gdn::prep::g_status, &z, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  }
  *out = v;
  return GDN_OK;
}
