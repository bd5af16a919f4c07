// Warp-specialised chunkwise gated delta rule (u = beta k) on tcgen05 / TMEM, sm_100a.
//
// Same mathematics as gdn_chunk_sm100.cu (the WY form of archbench/layers/nsgdn.py:408-417,
// derivation as in nsgdn.py:240-249); this version overlaps the state-independent work of
// chunk c+1 with the state recurrence of chunk c.  One CTA of 384 threads per (b, h, 128-row
// slice of the state), three warp groups, each thread bound to the TMEM lane of its warp's
// quarter:
//
//   prep  (warps 0-3)  chunk c+1: G = [K;Q] K^T (bf16 operands, exact), gates and cumulative
//                      log-decay, bf16 -> fp16 conversion of K, V and gamma-scaled Q, the rows
//                      of L and A, T = (I + L)^-1 (fp32 16x16 diagonal blocks, fp16 mma.sync
//                      block columns), W^T = K^T (T Gamma)^T and U^T = V^T T^T on tcgen05.
//   chain (warps 4-7)  chunk c: S -> fp16, S <- gamma_C S, R^T = U^T - S W^T and
//                      Y = S (Gamma Q)^T, R and R diag(w) -> fp16, S += (R diag w)^T K and
//                      Y += R^T A^T.
//   epilogue (8-11)    chunk c-1: Y from TMEM to y in HBM.
//
// Buffers between the groups: q/k tiles in a 3-deep TMA ring (the chain reads K and Gamma Q
// of its chunk while prep converts the next one and the one after that is in flight), v tiles in
// a 2-deep ring, U^T and Y double-buffered in TMEM (S 128 + G 64 + W 64 + U 2x64 + Y 2x64 = 512
// columns), A double-buffered in shared memory.  S16 shares its 32 KB with R16/R'16 and W16 its
// 16 KB with T16/(T Gamma)16, ordered by the MMA completion barriers.  Every mbarrier wait is
// bounded and abortable: a timeout raises a shared flag that makes every other wait return,
// the issuing threads drain their MMAs (bounded) and the CTA releases TMEM and exits.
#include <cudaTypedefs.h>

#include "gdn_common.cuh"
#include "sm100_ptx.cuh"

namespace gdn {
namespace ws {

constexpr int C = 64;
constexpr int D = 128;
constexpr int NT = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_G = 128, COL_W = 192, COL_U = 256, COL_Y = 384;  // U, Y: +64 per buffer
constexpr uint32_t TILE = 8192;
constexpr uint32_t LD16 = 144;  // bytes per row of the fp16 L matrix (72 halves, conflict-free ldmatrix)
constexpr uint32_t LDG = 20;    // floats per row of the fp32 diagonal blocks
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clocks

// Shared-memory map (bytes from a 1024-aligned base).
constexpr uint32_t KQ = 0;                        // 3 x [K0][Q0][K1][Q1]
constexpr uint32_t KQ_BYTES = 4 * TILE;
constexpr uint32_t VB = KQ + 3 * KQ_BYTES;        // 2 x [V0][V1]
constexpr uint32_t V_BYTES = 2 * TILE;
constexpr uint32_t SR = VB + 2 * V_BYTES;         // S16 (2 x 16 KB) | R16 (16 KB) + R'16 (16 KB)
constexpr uint32_t TW = SR + 4 * TILE;            // T16 (8 KB) + TG16 (8 KB) | W16 (16 KB)
constexpr uint32_t AB = TW + 2 * TILE;            // 2 x A16 (8 KB)
constexpr uint32_t L16 = AB + 2 * TILE;           // 64 rows x 144 B (diagonal blocks hold D_b)
constexpr uint32_t LDIAG = L16 + 64 * LD16;       // 4 x 16 x LDG floats
constexpr uint32_t SMALL = LDIAG + 4 * 16 * LDG * 4;
constexpr uint32_t SLOT = 6 * C;                  // floats per gate slot: la, beta, g, gam, w, misc
constexpr uint32_t BARS = SMALL + 3 * SLOT * 4;
constexpr uint32_t NBARS = 16;
constexpr uint32_t TOTAL = BARS + NBARS * 8 + 16;
constexpr uint32_t DYN = TOTAL + 1024;
static_assert(DYN <= 232448, "shared memory budget");
static_assert(SR % 1024 == 0 && TW % 1024 == 0 && AB % 1024 == 0, "swizzled tiles need 1 KB alignment");

enum Bar { B_KQ = 0, B_V = 3, B_G = 5, B_WU = 6, B_PREP = 7, B_R = 8, B_S = 9, B_YF = 10, B_YE = 12, B_DRAIN = 14 };

struct Params {
  const float* beta;
  const float* la;
  const float* s0;
  float* s_out;
  void* y;
  gdn_strides sy;
  int B, T, H, DV;
};

__device__ int g_status = 0;

__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

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

// Address of the 16-byte row `lane` supplies to ldmatrix/stmatrix x4 for the 16x16 block at
// (row0, col0) of a plain row-major fp16 matrix with `ld` bytes per row.
__device__ __forceinline__ uint32_t frag_addr_plain(uint32_t base, uint32_t ld, int row0, int col0, int lane) {
  const int m = lane >> 3, r = lane & 7;
  return base + (uint32_t)(row0 + r + ((m >> 1) << 3)) * ld + (uint32_t)(col0 + ((m & 1) << 3)) * 2u;
}
// Same for a 128B-swizzled fp16 tile (64 columns per 128-byte row).
__device__ __forceinline__ uint32_t frag_addr_sw(uint32_t base, int row0, int col0, int lane) {
  const int m = lane >> 3, r = lane & 7;
  const uint32_t row = (uint32_t)(row0 + r + ((m >> 1) << 3));
  const uint32_t chunk = (uint32_t)((col0 >> 3) + (m & 1));
  return base + sw128(row, chunk);
}

// Block column J of T = (I + L)^-1, computed transposed so that C fragments chain into A
// fragments: T^T_{J,i} = -(sum_{k=J}^{i-1} T^T_{J,k} L^T_{k,i}) D_i^T, with D_i = (I + L_ii)^-1 in
// the diagonal blocks of L16.  Writes T (to T16) and T diag(gamma) (to TG16), block column J,
// including the zero blocks above the diagonal.
template <int J>
__device__ __forceinline__ void merge_column(uint32_t l16, uint32_t t16, uint32_t tg16, const float* gam, int lane) {
  const int g = lane >> 2;
  const float g0 = gam[16 * J + g], g8 = gam[16 * J + g + 8];
  uint32_t X[4][4];
  ptx::ldsm_x4_t(frag_addr_plain(l16, LD16, 16 * J, 16 * J, lane), X[J]);
  auto emit = [&](int i, const uint32_t (&a)[4]) {
    ptx::stsm_x4_t(frag_addr_sw(t16, 16 * i, 16 * J, lane), a);
    uint32_t s[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float2 f = unpack_h2(a[r]);
      const float sc = (r & 1) ? g8 : g0;
      s[r] = pack_h2(f.x * sc, f.y * sc);
    }
    ptx::stsm_x4_t(frag_addr_sw(tg16, 16 * i, 16 * J, lane), s);
  };
  emit(J, X[J]);
  const uint32_t z[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < J; ++i) {
    ptx::stsm_x4_t(frag_addr_sw(t16, 16 * i, 16 * J, lane), z);
    ptx::stsm_x4_t(frag_addr_sw(tg16, 16 * i, 16 * J, lane), z);
  }
#pragma unroll
  for (int i = J + 1; i < 4; ++i) {
    float P[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = J; k < i; ++k) {
      uint32_t Bf[4];
      ptx::ldsm_x4(frag_addr_plain(l16, LD16, 16 * i, 16 * k, lane), Bf);
      ptx::hmma16816(*reinterpret_cast<float(*)[4]>(&P[0]), X[k], Bf[0], Bf[1]);
      ptx::hmma16816(*reinterpret_cast<float(*)[4]>(&P[4]), X[k], Bf[2], Bf[3]);
    }
    const uint32_t Pa[4] = {pack_h2(-P[0], -P[1]), pack_h2(-P[2], -P[3]), pack_h2(-P[4], -P[5]), pack_h2(-P[6], -P[7])};
    uint32_t Db[4];
    ptx::ldsm_x4(frag_addr_plain(l16, LD16, 16 * i, 16 * i, lane), Db);
    float Tt[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    ptx::hmma16816(*reinterpret_cast<float(*)[4]>(&Tt[0]), Pa, Db[0], Db[1]);
    ptx::hmma16816(*reinterpret_cast<float(*)[4]>(&Tt[4]), Pa, Db[2], Db[3]);
    X[i][0] = pack_h2(Tt[0], Tt[1]);
    X[i][1] = pack_h2(Tt[2], Tt[3]);
    X[i][2] = pack_h2(Tt[4], Tt[5]);
    X[i][3] = pack_h2(Tt[6], Tt[7]);
    ptx::stsm_x4_t(frag_addr_sw(t16, 16 * i, 16 * J, lane), X[i]);
    const uint32_t s[4] = {pack_h2(Tt[0] * g0, Tt[1] * g0), pack_h2(Tt[2] * g8, Tt[3] * g8),
                           pack_h2(Tt[4] * g0, Tt[5] * g0), pack_h2(Tt[6] * g8, Tt[7] * g8)};
    ptx::stsm_x4_t(frag_addr_sw(tg16, 16 * i, 16 * J, lane), s);
  }
}

template <typename TOut>
__global__ void __launch_bounds__(NT, 1)
    ws_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dv_tiles = p.DV / D;
  const int bh = blockIdx.x / dv_tiles, dv0 = (blockIdx.x % dv_tiles) * D;
  const int b = bh / p.H, h = bh % p.H;
  const int nch = (p.T + C - 1) / C;

  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* small = reinterpret_cast<float*>(sm + SMALL);

  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < 3; ++i) ptx::mbar_init(&bars[B_KQ + i], 1);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_V + i], 1);
    ptx::mbar_init(&bars[B_G], 1);
    ptx::mbar_init(&bars[B_WU], 1);
    ptx::mbar_init(&bars[B_PREP], 1);
    ptx::mbar_init(&bars[B_R], 1);
    ptx::mbar_init(&bars[B_S], 1);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_YF + i], 1);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_YE + i], 128);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_DRAIN + i], 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tensormap(&tm_q);
    ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_v);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t my = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lane quarter
  const int row = tid & 127;                                         // = TMEM lane of this thread

  // One elected thread of a 128-thread group waits on the mbarrier; a reducing named barrier
  // hands the outcome to the whole group, so all of its threads take the same branch.
  auto gwait = [&](int bar, uint32_t parity, bool leader, int group) -> bool {
    bool fail = false;
    if (leader) fail = !ptx::mbar_wait_abortable(&bars[bar], parity, WAIT_LIMIT, abort_flag);
    return !ptx::named_bar_or(group, 128, fail);
  };
  auto issue_kq = [&](int c) {
    uint8_t* dst = sm + KQ + (c % 3) * KQ_BYTES;
    uint64_t* bar = &bars[B_KQ + c % 3];
    ptx::mbar_arrive_expect_tx(bar, KQ_BYTES);
    const int t0 = c * C;
    ptx::tma_load_4d(dst + 0 * TILE, &tm_k, bar, 0, h, t0, b);
    ptx::tma_load_4d(dst + 1 * TILE, &tm_q, bar, 0, h, t0, b);
    ptx::tma_load_4d(dst + 2 * TILE, &tm_k, bar, 64, h, t0, b);
    ptx::tma_load_4d(dst + 3 * TILE, &tm_q, bar, 64, h, t0, b);
  };
  auto issue_v = [&](int c) {
    uint8_t* dst = sm + VB + (c & 1) * V_BYTES;
    uint64_t* bar = &bars[B_V + (c & 1)];
    ptx::mbar_arrive_expect_tx(bar, V_BYTES);
    ptx::tma_load_4d(dst + 0 * TILE, &tm_v, bar, dv0, h, c * C, b);
    ptx::tma_load_4d(dst + 1 * TILE, &tm_v, bar, dv0 + 64, h, c * C, b);
  };

  constexpr uint32_t ID_G = ptx::idesc_bf16_f32(128, 64);
  constexpr uint32_t ID_N64 = ptx::idesc_f16_f32(128, 64, false, false, false);
  constexpr uint32_t ID_N64_AMN = ptx::idesc_f16_f32(128, 64, true, false, false);
  constexpr uint32_t ID_N64_BMN_NEG = ptx::idesc_f16_f32(128, 64, false, true, true);
  constexpr uint32_t ID_N128_BMN = ptx::idesc_f16_f32(128, 128, false, true, false);

  if (warp < 4) {
    // =============================== prep ===============================
    const int pt = tid;
    bool issued = false;  // MMAs issued by this thread since the last completed wait
    int v_issued = 0;     // V loads issued (chunks [0, v_issued))
    if (pt == 0) {
      issue_v(0);
      v_issued = 1;
      if (nch > 1) { issue_v(1); v_issued = 2; }
    }
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int pb = c & 1;
      const uint32_t kq_a = sb + KQ + (c % 3) * KQ_BYTES;
      uint8_t* kq = sm + KQ + (c % 3) * KQ_BYTES;
      uint8_t* vv = sm + VB + pb * V_BYTES;
      const uint32_t v_a = sb + VB + pb * V_BYTES;
      float* la_s = small + (c % 3) * SLOT;
      float* beta_s = la_s + C;
      float* g_s = beta_s + C;
      float* gam_s = g_s + C;
      float* w_s = gam_s + C;
      float* misc_s = w_s + C;
      const int t0 = c * C;

      if (!gwait(B_KQ + c % 3, (uint32_t)(c / 3) & 1u, pt == 0, 1)) break;
      if (pt == 0) {  // G = [K;Q] K^T from the bf16 tiles as loaded
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t kb = k >> 2, kk = k & 3;
          const uint64_t a = ptx::sdesc_sw128(kq_a + kb * 2 * TILE + kk * 32, 16, 1024);
          ptx::mma_f16_ss(tmem + COL_G, a, a, ID_G, k > 0);
        }
        ptx::mma_commit(&bars[B_G]);
        issued = true;
      }
      if (warp == 0) {  // gates and chunk-local cumulative log-decay (log-space, fp32)
        float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
        const int64_t gi = ((int64_t)b * p.T + t0) * p.H + h;
        if (t0 + lane < p.T) { a0 = p.la[gi + (int64_t)lane * p.H]; b0 = p.beta[gi + (int64_t)lane * p.H]; }
        if (t0 + lane + 32 < p.T) { a1 = p.la[gi + (int64_t)(lane + 32) * p.H]; b1 = p.beta[gi + (int64_t)(lane + 32) * p.H]; }
        beta_s[lane] = b0;
        beta_s[lane + 32] = b1;
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
        w_s[lane] = b0 * expf(gC - a0);
        w_s[lane + 32] = b1 * expf(gC - a1);
        if (lane == 0) misc_s[0] = expf(gC);
      }
      // V(c) must have landed too (issued two chunks ahead by this group's leader).
      if (!gwait(B_V + pb, (uint32_t)(c >> 1) & 1u, pt == 0, 1)) break;
      if (!gwait(B_G, (uint32_t)c & 1u, pt == 0, 1)) break;
      if (pt == 0) issued = false;
      ptx::tc_fence_after();

      // bf16 -> fp16 in place: K (tiles 0, 2), gamma-scaled Q (tiles 1, 3), V (2 tiles).
#pragma unroll 4
      for (int i = pt; i < 6 * 512; i += 128) {
        const int tile = i >> 9;
        uint8_t* base = tile < 4 ? kq + tile * TILE : vv + (tile - 4) * TILE;
        const int off = (i & 511) * 16;
        const float sc = (tile == 1 || tile == 3) ? gam_s[off >> 7] : 1.f;
        uint4 r = *reinterpret_cast<uint4*>(base + off);
        __nv_bfloat162* b2 = reinterpret_cast<__nv_bfloat162*>(&r);
        uint4 o;
        uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(b2[k]);
          o32[k] = pack_h2(f.x * sc, f.y * sc);
        }
        *reinterpret_cast<uint4*>(base + off) = o;
      }
      // Rows of L (threads 0-63, TMEM lanes 0-63) and A (threads 64-127) from G.
      float gv[64];
      ptx::tmem_ld32(my + COL_G, *reinterpret_cast<float(*)[32]>(gv));
      ptx::tmem_ld32(my + COL_G + 32, *reinterpret_cast<float(*)[32]>(gv + 32));
      ptx::tc_wait_ld();
      const int t = pt & 63;
      const float gt = g_s[t];
      const int jmax_blk = (warp & 1) ? 4 : 2;  // 16-column blocks that can hold j <= t in this warp
#pragma unroll
      for (int jb = 0; jb < 4; ++jb) {
        if (jb < jmax_blk) {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = jb * 16 + jj;
            const bool keep = (pt < 64) ? (j < t) : (j <= t);
            gv[j] = keep ? gv[j] * beta_s[j] * expf(gt - g_s[j]) : 0.f;
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) gv[jb * 16 + jj] = 0.f;
        }
      }
      if (pt < 64) {
        uint8_t* lrow = sm + L16 + t * LD16;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 v4;
          v4.x = pack_h2(gv[q * 8 + 0], gv[q * 8 + 1]);
          v4.y = pack_h2(gv[q * 8 + 2], gv[q * 8 + 3]);
          v4.z = pack_h2(gv[q * 8 + 4], gv[q * 8 + 5]);
          v4.w = pack_h2(gv[q * 8 + 6], gv[q * 8 + 7]);
          *reinterpret_cast<uint4*>(lrow + q * 16) = v4;
        }
        float* drow = reinterpret_cast<float*>(sm + LDIAG) + ((t >> 4) * 16 + (t & 15)) * LDG;
        const int bt = t >> 4;
        float dv[16];  // gv[16 bt + q] with static register indices
#pragma unroll
        for (int q = 0; q < 16; ++q) dv[q] = bt == 0 ? gv[q] : bt == 1 ? gv[16 + q] : bt == 2 ? gv[32 + q] : gv[48 + q];
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4*>(drow + q) = make_float4(dv[q], dv[q + 1], dv[q + 2], dv[q + 3]);
      }
      ptx::named_bar(1, 128);
      // W16(c-1), which shares T16/TG16's space, must have been consumed by R(c-1), and A16[p]
      // by Yi(c-2).
      if (c > 0 && !gwait(B_R, (uint32_t)(c - 1) & 1u, pt == 0, 1)) break;
      if (c >= 2 && !gwait(B_YF + pb, (uint32_t)((c - 2) >> 1) & 1u, pt == 0, 1)) break;
      if (pt >= 64) {
        store_row_f16(sm + AB + pb * TILE, t, gv);
      } else {
        // D_b = (I + L_bb)^-1, one column per thread, fp32 forward substitution.
        const int bb = pt >> 4, j = pt & 15;
        const float* Lb = reinterpret_cast<const float*>(sm + LDIAG) + bb * 16 * LDG;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float s = 0.f;
#pragma unroll
          for (int m = 0; m < r; ++m) s = fmaf(Lb[r * LDG + m], x[m], s);
          x[r] = (r == j) ? 1.f : (r > j ? -s : 0.f);
        }
        __half* l16 = reinterpret_cast<__half*>(sm + L16);
#pragma unroll
        for (int r = 0; r < 16; ++r) l16[(bb * 16 + r) * (LD16 / 2) + bb * 16 + j] = __float2half_rn(x[r]);
      }
      ptx::named_bar(1, 128);
      {
        const uint32_t l16a = sb + L16, t16a = sb + TW, tg16a = sb + TW + TILE;
        switch (warp) {
          case 0: merge_column<0>(l16a, t16a, tg16a, gam_s, lane); break;
          case 1: merge_column<1>(l16a, t16a, tg16a, gam_s, lane); break;
          case 2: merge_column<2>(l16a, t16a, tg16a, gam_s, lane); break;
          default: merge_column<3>(l16a, t16a, tg16a, gam_s, lane); break;
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::named_bar(1, 128);
      if (pt == 0) {  // W^T = K^T (T Gamma)^T, U^T = V^T T^T
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ak = ptx::sdesc_sw128(kq_a + k * 2048, 2 * TILE, 1024);
          const uint64_t bt = ptx::sdesc_sw128(sb + TW + TILE + k * 32, 16, 1024);
          ptx::mma_f16_ss(tmem + COL_W, ak, bt, ID_N64_AMN, k > 0);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t av = ptx::sdesc_sw128(v_a + k * 2048, TILE, 1024);
          const uint64_t bt = ptx::sdesc_sw128(sb + TW + k * 32, 16, 1024);
          ptx::mma_f16_ss(tmem + COL_U + 64 * pb, av, bt, ID_N64_AMN, k > 0);
        }
        ptx::mma_commit(&bars[B_WU]);
        issued = true;
      }
      if (!gwait(B_WU, (uint32_t)c & 1u, pt == 0, 1)) break;
      if (pt == 0) {
        issued = false;
        if (c + 2 < nch) { issue_v(c + 2); v_issued = c + 3; }  // V(c) consumed by U^T(c)
      }
      ptx::tc_fence_after();
      {
        float wv[64];
        ptx::tmem_ld32(my + COL_W, *reinterpret_cast<float(*)[32]>(wv));
        ptx::tmem_ld32(my + COL_W + 32, *reinterpret_cast<float(*)[32]>(wv + 32));
        ptx::tc_wait_ld();
        store_row_f16(sm + TW, pt, wv);  // W16: row d = TMEM lane, 64 tokens
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      ptx::named_bar(1, 128);
      if (pt == 0) ptx::mbar_arrive(&bars[B_PREP]);
    }
    if (*abort_flag && pt == 0) {  // drain this thread's MMAs and V loads before the CTA exits
      if (issued) {
        ptx::mma_commit(&bars[B_DRAIN]);
        ptx::mbar_wait_bounded(&bars[B_DRAIN], 0, WAIT_LIMIT);
      }
      for (int c = v_issued - 2 < 0 ? 0 : v_issued - 2; c < v_issued; ++c)
        ptx::mbar_wait_bounded(&bars[B_V + (c & 1)], (uint32_t)(c >> 1) & 1u, WAIT_LIMIT);
    }
  } else if (warp < 8) {
    // =============================== chain ===============================
    const int ct = tid - 128;
    bool issued = false;
    {
      const float* src = p.s0 ? p.s0 + ((int64_t)bh * p.DV + dv0 + ct) * D : nullptr;
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 t4 = src ? *reinterpret_cast<const float4*>(src + c4 * 32 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[i] = t4.x; v[i + 1] = t4.y; v[i + 2] = t4.z; v[i + 3] = t4.w;
        }
        ptx::tmem_st32(my + COL_S + c4 * 32, v);
      }
      ptx::tc_wait_st();
    }
    int kq_issued = 0;  // q/k loads issued (chunks [0, kq_issued))
    if (ct == 0) {
      issue_kq(0);
      kq_issued = 1;
      if (nch > 1) { issue_kq(1); kq_issued = 2; }
    }
    int c = 0;
#pragma unroll 1
    for (; c < nch; ++c) {
      const int pb = c & 1;
      const uint32_t kq_a = sb + KQ + (c % 3) * KQ_BYTES;
      const float* slot = small + (c % 3) * SLOT;
      const float* w_s = slot + 4 * C;
      if (!gwait(B_PREP, (uint32_t)c & 1u, ct == 0, 2)) break;
      const float gC = slot[5 * C];  // written by prep(c): read only after its ready barrier
      if (c > 0) {
        if (!gwait(B_S, (uint32_t)(c - 1) & 1u, ct == 0, 2)) break;
        if (ct == 0) issued = false;
      }
      ptx::tc_fence_after();
      if (ct == 0 && c + 2 < nch) { issue_kq(c + 2); kq_issued = c + 3; }  // buffer of chunk c-1, freed by S(c-1)
      // S16 <- fp16(S); S <- gamma_C S
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        float v[32];
        ptx::tmem_ld32(my + COL_S + c4 * 32, v);
        ptx::tc_wait_ld();
        uint8_t* half = sm + SR + (c4 >> 1) * 2 * TILE;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 pk;
          pk.x = pack_h2(v[q * 8 + 0], v[q * 8 + 1]);
          pk.y = pack_h2(v[q * 8 + 2], v[q * 8 + 3]);
          pk.z = pack_h2(v[q * 8 + 4], v[q * 8 + 5]);
          pk.w = pack_h2(v[q * 8 + 6], v[q * 8 + 7]);
          *reinterpret_cast<uint4*>(half + sw128(ct, (c4 & 1) * 4 + q)) = pk;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= gC;
        ptx::tmem_st32(my + COL_S + c4 * 32, v);
      }
      ptx::tc_wait_st();
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      ptx::named_bar(2, 128);
      bool r_ok = true;
      if (ct == 0) {  // R^T = U^T - S W^T ; Y = S (Gamma Q)^T
        ptx::tc_fence_after();
        if (c >= 2)  // Y[p] drained by the epilogue
          r_ok = ptx::mbar_wait_abortable(&bars[B_YE + pb], (uint32_t)((c - 2) >> 1) & 1u, WAIT_LIMIT, abort_flag);
        if (r_ok) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t kb = k >> 2, kk = k & 3;
            const uint64_t as = ptx::sdesc_sw128(sb + SR + kb * 2 * TILE + kk * 32, 16, 1024);
            const uint64_t bw = ptx::sdesc_sw128(sb + TW + k * 2048, 16, 1024);
            ptx::mma_f16_ss(tmem + COL_U + 64 * pb, as, bw, ID_N64_BMN_NEG, 1);
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t kb = k >> 2, kk = k & 3;
            const uint64_t as = ptx::sdesc_sw128(sb + SR + kb * 2 * TILE + kk * 32, 16, 1024);
            const uint64_t bq = ptx::sdesc_sw128(kq_a + TILE + kb * 2 * TILE + kk * 32, 16, 1024);
            ptx::mma_f16_ss(tmem + COL_Y + 64 * pb, as, bq, ID_N64, k > 0);
          }
          ptx::mma_commit(&bars[B_R]);
          issued = true;
        }
      }
      {
        bool fail = false;
        if (ct == 0) fail = !r_ok || !ptx::mbar_wait_abortable(&bars[B_R], (uint32_t)c & 1u, WAIT_LIMIT, abort_flag);
        if (ptx::named_bar_or(2, 128, fail)) break;
      }
      if (ct == 0) issued = false;
      ptx::tc_fence_after();
      {
        float rv[64];
        ptx::tmem_ld32(my + COL_U + 64 * pb, *reinterpret_cast<float(*)[32]>(rv));
        ptx::tmem_ld32(my + COL_U + 64 * pb + 32, *reinterpret_cast<float(*)[32]>(rv + 32));
        ptx::tc_wait_ld();
        store_row_f16(sm + SR, ct, rv);  // R16 (S16 is free: R and Y read it and completed)
#pragma unroll
        for (int t = 0; t < 64; ++t) rv[t] *= w_s[t];
        store_row_f16(sm + SR + 2 * TILE, ct, rv);  // R'16 = R diag(w)
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      ptx::named_bar(2, 128);
      if (ct == 0) {  // S += (R diag w)^T K ; Y += R^T A^T
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ap = ptx::sdesc_sw128(sb + SR + 2 * TILE + k * 32, 16, 1024);
          const uint64_t bk = ptx::sdesc_sw128(kq_a + k * 2048, 2 * TILE, 1024);
          ptx::mma_f16_ss(tmem + COL_S, ap, bk, ID_N128_BMN, 1);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ar = ptx::sdesc_sw128(sb + SR + k * 32, 16, 1024);
          const uint64_t ba = ptx::sdesc_sw128(sb + AB + pb * TILE + k * 32, 16, 1024);
          ptx::mma_f16_ss(tmem + COL_Y + 64 * pb, ar, ba, ID_N64, 1);
        }
        ptx::mma_commit(&bars[B_S]);
        ptx::mma_commit(&bars[B_YF + pb]);
        issued = true;
      }
    }
    if (!*abort_flag && nch > 0 && gwait(B_S, (uint32_t)(nch - 1) & 1u, ct == 0, 2)) {
      if (ct == 0) issued = false;
      ptx::tc_fence_after();
      if (p.s_out != nullptr) {
        float* dst = p.s_out + ((int64_t)bh * p.DV + dv0 + ct) * D;
#pragma unroll 1
        for (int c4 = 0; c4 < 4; ++c4) {
          float v[32];
          ptx::tmem_ld32(my + COL_S + c4 * 32, v);
          ptx::tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + c4 * 32 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
    }
    if (*abort_flag && ct == 0) {  // drain this thread's MMAs and q/k loads before the CTA exits
      if (issued) {
        ptx::mma_commit(&bars[B_DRAIN + 1]);
        ptx::mbar_wait_bounded(&bars[B_DRAIN + 1], 0, WAIT_LIMIT);
      }
      for (int c = kq_issued - 3 < 0 ? 0 : kq_issued - 3; c < kq_issued; ++c)
        ptx::mbar_wait_bounded(&bars[B_KQ + c % 3], (uint32_t)(c / 3) & 1u, WAIT_LIMIT);
    }
  } else {
    // =============================== epilogue ===============================
    const int et = tid - 256;
    TOut* yb = static_cast<TOut*>(p.y) + (int64_t)b * p.sy.b + (int64_t)h * p.sy.h + dv0 + et;
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int pp = c & 1;
      if (!gwait(B_YF + pp, (uint32_t)(c >> 1) & 1u, et == 0, 3)) break;
      ptx::tc_fence_after();
      float y0[32], y1[32];
      ptx::tmem_ld32(my + COL_Y + 64 * pp, y0);
      ptx::tmem_ld32(my + COL_Y + 64 * pp + 32, y1);
      ptx::tc_wait_ld();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&bars[B_YE + pp]);
      const int t0 = c * C, nvalid = min(C, p.T - t0);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) store_as(yb + (int64_t)(t0 + j) * p.sy.t, y0[j]);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (32 + j < nvalid) store_as(yb + (int64_t)(t0 + 32 + j) * p.sy.t, y1[j]);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (tid == 0 && *abort_flag) atomicExch(&g_status, GDN_ERR_TIMEOUT);
  if (warp == 0) ptx::tmem_dealloc(tmem, TMEM_COLS);
}

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

// [B][T][H][F] bf16 view -> 4-D tensor map (f, h, t, b), box 64 x 1 x 64 x 1, 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, int64_t F, const gdn_prefill_args* a, const gdn_strides& s) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)F, (cuuint64_t)a->H, (cuuint64_t)a->T, (cuuint64_t)a->B};
  cuuint64_t strides[3] = {(cuuint64_t)s.h * 2, (cuuint64_t)s.t * 2, (cuuint64_t)s.b * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)C, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename TOut>
int launch(const gdn_prefill_args* a, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, a->q, a->DK, a, a->sq) || !make_map(&mk, a->k, a->DK, a, a->sk) ||
      !make_map(&mv, a->v, a->DV, a, a->sv))
    return GDN_ERR_LAUNCH;
  auto kern = ws_kernel<TOut>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN) != cudaSuccess)
      return GDN_ERR_LAUNCH;
    attr_set = true;
  }
  Params p;
  p.beta = a->beta; p.la = a->la; p.s0 = a->s0; p.s_out = a->s_out; p.y = a->y; p.sy = a->sy;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DV = (int)a->DV;
  const int64_t grid = a->B * a->H * (a->DV / D);
  kern<<<(unsigned)grid, NT, DYN, stream>>>(mq, mk, mv, p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace ws
}  // namespace gdn

// DK = 128, DV a multiple of 128, u = beta k (no explicit write vector).
bool gdn_chunk_ws_supported(const gdn_prefill_args* a) {
  return a->u == nullptr && a->DK == 128 && a->DV % 128 == 0 && a->DV >= 128;
}

int gdn_launch_chunk_ws(const gdn_prefill_args* a, cudaStream_t stream) {
  return a->out_dtype == GDN_DTYPE_BF16 ? gdn::ws::launch<__nv_bfloat16>(a, stream) : gdn::ws::launch<float>(a, stream);
}

namespace gdn {
namespace ws {
// Exercises the bounded-wait path of the kernels on purpose: waits on an mbarrier that nothing
// ever arrives on, gives up after `max_cycles`, records GDN_ERR_TIMEOUT and returns normally.
__global__ void selftest_wait_kernel(long long max_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !ptx::mbar_wait_bounded(&bar, 0, max_cycles)) atomicExch(&g_status, GDN_ERR_TIMEOUT);
}
}  // namespace ws
}  // namespace gdn

int gdn_launch_selftest_wait(long long max_cycles, cudaStream_t stream) {
  if (max_cycles <= 0 || max_cycles > 4000000000LL) return GDN_ERR_SHAPE;
  gdn::ws::selftest_wait_kernel<<<1, 32, 0, stream>>>(max_cycles);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_chunk_ws_read_status(int* out, int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::ws::g_status, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (reset) {
    int z = 0;
    if (cudaMemcpyToSymbol(gdn::ws::g_status, &z, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  }
  *out = v;
  return GDN_OK;
}
