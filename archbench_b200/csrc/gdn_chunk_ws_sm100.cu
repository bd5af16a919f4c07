// Warp-specialised chunkwise gated delta rule (u = beta k) on tcgen05 / TMEM, sm_100a.
//
// The WY form of archbench/layers/nsgdn.py:408-417 (derivation as in nsgdn.py:240-249), with the
// state-independent work of chunk c+1 overlapped with the state recurrence of chunk c.  y goes out
// by TMA tile stores, or, where y's rows are not 16-byte aligned, by each thread's own stores.  One CTA of 384 threads per (b, h, 128-row
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
#include <string.h>

#include "gdn_tiles.cuh"

namespace gdn {
namespace ws {

using namespace gdn::tiles;

constexpr int NT = 384;     // warps 0-3: state chain; warps 4-11: workers (prep + output)
constexpr int NWORK = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_G = 128, COL_W = 192, COL_U = 256, COL_Y = 384;  // U, Y: +64 per buffer
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clocks

// Shared-memory map (bytes from a 1024-aligned base).
constexpr uint32_t KQ = 0;                        // 3 x [K0][Q0][K1][Q1]
constexpr uint32_t KQ_BYTES = 4 * TILE;
constexpr uint32_t VB = KQ + 3 * KQ_BYTES;        // 2 x [V0][V1]
constexpr uint32_t V_BYTES = 2 * TILE;
constexpr uint32_t SR = VB + 2 * V_BYTES;         // S16 (2 x 16 KB) | R16 (16 KB) + R'16 (16 KB)
constexpr uint32_t TW = SR + 4 * TILE;            // T_hi (bf16, 8 KB) + TG16 (8 KB) | W16 (16 KB)
constexpr uint32_t AB = TW + 2 * TILE;            // 2 x A16 (8 KB)
constexpr uint32_t TLO = AB + 2 * TILE;           // T_lo (bf16, 8 KB): T = T_hi + T_lo to ~2^-16
constexpr uint32_t L16 = TLO + TILE;              // 64 rows x 144 B (diagonal blocks hold D_b)
constexpr uint32_t LDIAG = L16 + 64 * LD16;       // 4 x 16 x LDG floats
constexpr uint32_t EXPT = LDIAG + 4 * 16 * LDG * 4;  // decay tables: 64 + 4x64 + 4x16x17 floats
constexpr uint32_t SMALL = EXPT + (64 + 4 * 64 + 4 * 16 * 20) * 4;
constexpr uint32_t SLOT = 6 * C;                  // floats per gate slot: la, beta, g, gam, w, misc
constexpr uint32_t BARS = SMALL + 3 * SLOT * 4;
constexpr uint32_t NBARS = 18;
constexpr uint32_t TOTAL = BARS + NBARS * 8 + 16;
constexpr uint32_t DYN = TOTAL + 1024;
static_assert(DYN <= 232448, "shared memory budget");
static_assert(SR % 1024 == 0 && TW % 1024 == 0 && AB % 1024 == 0 && TLO % 1024 == 0, "swizzled tiles need 1 KB alignment");

enum Bar { B_KQ = 0, B_V = 3, B_G = 5, B_WU = 6, B_PREP = 7, B_R = 8, B_S = 9, B_YF = 10, B_YE = 12, B_DRAIN = 14, B_UU = 16 };

struct Params {
  const float* beta;
  const float* la;
  const float* s0;
  float* s_out;
  void* y;
  gdn_strides sy;
  int B, T, H, DV;
  // Segments: CTA (b, h, seg, tile) runs chunks [seg * seg_len, (seg + 1) * seg_len).
  int nseg, seg_len;
  int nv;      // real 128-row state tiles (DV / 128)
  int ntiles;  // tiles per (b, h, seg): nv, or nv + 1 in state mode (the transition block)
  int mode;    // 0: outputs y (and S_T of the last segment); 1: segment states only, no y
  const float* seg_s0;  // mode 0: initial state of segment s >= 1 at slot (bh, s - 1)
  float* seg_out;       // mode 1: [N_s; M_s] of each segment at slot (bh, s)
  int ws_stride;        // slots per (b, h) in the segment workspace
  int y_direct;         // y rows not 16-byte aligned (no TMA store): each thread writes its feature directly
};

__device__ int g_status = 0;

// HAS_U: an explicit write vector u (nsgdn n_steps > 1) replaces beta k where the state is written
// (G = [K;Q] U^T for L and A, S += (R diag w)^T U with w free of beta); its tiles ride in the q/k
// ring, which is then two entries of [K0][Q0][K1][Q1][U0][U1] instead of three of [K0][Q0][K1][Q1].
template <bool HAS_U, typename TOut>
__global__ void __launch_bounds__(NT, 1)
    ws_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_y,
              const __grid_constant__ CUtensorMap tm_u, const Params p) {
  constexpr int NR = HAS_U ? 2 : 3;                       // ring entries
  constexpr uint32_t KQB = HAS_U ? 6 * TILE : KQ_BYTES;   // bytes per ring entry
  constexpr int NCONV = HAS_U ? 6 : 4;                    // tiles converted to fp16 in place
  static_assert(NR * KQB == 3 * KQ_BYTES, "the ring keeps its footprint");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % p.ntiles, rest = blockIdx.x / p.ntiles;
  const int seg = rest % p.nseg, bh = rest / p.nseg;
  const int dv0 = tile * D;
  const int b = bh / p.H, h = bh % p.H;
  const bool virt = tile >= p.nv;   // state mode: the transition block (v = 0, S_0 = I)
  const bool want_y = p.mode == 0;
  const int cb = seg * p.seg_len;    // first chunk of this CTA's segment
  const int nch = max(0, min((p.T + C - 1) / C - cb, p.seg_len));

  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* small = reinterpret_cast<float*>(sm + SMALL);
  float* eT = reinterpret_cast<float*>(sm + EXPT);      // [64]      exp(g_t - g_{16 floor(t/16)})
  float* eJ = eT + C;                                    // [4][64]   beta_j exp(g_{16b} - g_j), j < 16b
  float* Ed = eJ + 4 * C;                                // [4][16][20] beta_{16b+c} exp(g_{16b+r} - g_{16b+c}), c <= r

  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < 3; ++i) ptx::mbar_init(&bars[B_KQ + i], 1);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_V + i], 1);
    ptx::mbar_init(&bars[B_G], 1);
    ptx::mbar_init(&bars[B_WU], 1);
    ptx::mbar_init(&bars[B_UU], 1);
    ptx::mbar_init(&bars[B_PREP], 1);
    ptx::mbar_init(&bars[B_R], 1);
    ptx::mbar_init(&bars[B_S], 1);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_YF + i], 1);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_YE + i], 4);  // one arrival per output warp
    for (int i = 0; i < 2; ++i) ptx::mbar_init(&bars[B_DRAIN + i], 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tensormap(&tm_q);
    ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_v);
    if (!p.y_direct) ptx::prefetch_tensormap(&tm_y);
    if (HAS_U) ptx::prefetch_tensormap(&tm_u);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t my = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lane quarter
  const int row = tid & 127;                                         // TMEM lane of this thread

  // One elected thread of a group waits on the mbarrier; a reducing named barrier hands the
  // outcome to the whole group, so all of its threads take the same branch.
  auto gwait = [&](int bar, uint32_t parity, bool leader, int group, int n) -> bool {
    bool fail = false;
    if (leader) fail = !ptx::mbar_wait_abortable(&bars[bar], parity, WAIT_LIMIT, abort_flag);
    return !ptx::named_bar_or(group, n, fail);
  };
  auto issue_kq = [&](int c) {
    uint8_t* dst = sm + KQ + (c % NR) * KQB;
    uint64_t* bar = &bars[B_KQ + c % NR];
    ptx::mbar_arrive_expect_tx(bar, KQB);
    const int t0 = (cb + c) * C;
    ptx::tma_load_4d(dst + 0 * TILE, &tm_k, bar, 0, h, t0, b);
    ptx::tma_load_4d(dst + 1 * TILE, &tm_q, bar, 0, h, t0, b);
    ptx::tma_load_4d(dst + 2 * TILE, &tm_k, bar, 64, h, t0, b);
    ptx::tma_load_4d(dst + 3 * TILE, &tm_q, bar, 64, h, t0, b);
    if (HAS_U) {
      ptx::tma_load_4d(dst + 4 * TILE, &tm_u, bar, 0, h, t0, b);
      ptx::tma_load_4d(dst + 5 * TILE, &tm_u, bar, 64, h, t0, b);
    }
  };
  auto issue_v = [&](int c) {
    uint8_t* dst = sm + VB + (c & 1) * V_BYTES;
    uint64_t* bar = &bars[B_V + (c & 1)];
    ptx::mbar_arrive_expect_tx(bar, V_BYTES);
    ptx::tma_load_4d(dst + 0 * TILE, &tm_v, bar, dv0, h, (cb + c) * C, b);
    ptx::tma_load_4d(dst + 1 * TILE, &tm_v, bar, dv0 + 64, h, (cb + c) * C, b);
  };

  constexpr uint32_t ID_G = ptx::idesc_bf16_f32(128, 64);
  constexpr uint32_t ID_U_BF16 = ptx::idesc_bf16_f32(128, 64, true, false);  // V^T (bf16, MN-major) x T^T
  constexpr uint32_t ID_N64 = ptx::idesc_f16_f32(128, 64, false, false, false);
  constexpr uint32_t ID_N64_AMN = ptx::idesc_f16_f32(128, 64, true, false, false);
  constexpr uint32_t ID_N64_BMN_NEG = ptx::idesc_f16_f32(128, 64, false, true, true);
  constexpr uint32_t ID_N128_BMN = ptx::idesc_f16_f32(128, 128, false, true, false);
  // Descriptor templates: an operand at byte offset `o` from the shared base is tmpl + (o >> 4).
  const uint64_t D_K = ptx::sdesc_sw128(sb, 16, 1024);           // K-major operands
  const uint64_t D_MN16K = ptx::sdesc_sw128(sb, 2 * TILE, 1024); // MN-major, 64-blocks 16 KB apart
  const uint64_t D_MN8K = ptx::sdesc_sw128(sb, TILE, 1024);      // MN-major, 64-blocks 8 KB apart
  auto at = [](uint64_t tmpl, uint32_t off) { return tmpl + (uint64_t)(off >> 4); };

  if (warp >= 4) {
    // ============================ workers: prep of chunk c, y of chunk c-1 ============================
    const int wt = tid - 128;            // 0..255
    const int ww = wt >> 5;              // worker warp 0..7
    const int hf = ww >> 2;              // column half (0: 0-31, 1: 32-63) of every 64-column tile
    const bool leader = wt == 0;
    bool issued = false;
    int v_issued = 0;
    float ga0 = 0.f, ga1 = 0.f, gb0 = 0.f, gb1 = 0.f;  // prefetched gates of the next chunk (worker warp 1)
    auto load_gates = [&](int c) {
      ga0 = ga1 = gb0 = gb1 = 0.f;
      const int t0 = (cb + c) * C;
      const int64_t gi = ((int64_t)b * p.T + t0) * p.H + h;
      if (t0 + lane < p.T) { ga0 = p.la[gi + (int64_t)lane * p.H]; gb0 = HAS_U ? 1.f : p.beta[gi + (int64_t)lane * p.H]; }
      if (t0 + lane + 32 < p.T) {
        ga1 = p.la[gi + (int64_t)(lane + 32) * p.H];
        gb1 = HAS_U ? 1.f : p.beta[gi + (int64_t)(lane + 32) * p.H];
      }
    };
    if (ww == 1) load_gates(0);
    if (leader && !virt && nch > 0) {
      issue_v(0);
      v_issued = 1;
      if (nch > 1) { issue_v(1); v_issued = 2; }
    }
    // y of chunk c: TMEM -> shared staging -> HBM by TMA tile stores, done by the output warps
    // (worker warps 4-7 = warps 8-11).  The staging buffer is A16 of chunk c, whose reader Yi(c)
    // has completed once Y(c) is ready; the next writer of that buffer is prep(c+2), after this
    // group's final wait for its stores to be read.  Y[c & 1] is released with one mbarrier
    // arrival per warp.
    auto epilogue = [&](int c) -> bool {
      const int pp = c & 1;
      if (!gwait(B_YF + pp, (uint32_t)(c >> 1) & 1u, wt == 128, 3, 128)) return false;
      ptx::tc_fence_after();
      float yv[64];
      ptx::tmem_ld32(my + COL_Y + 64 * pp, *reinterpret_cast<float(*)[32]>(yv));
      ptx::tmem_ld32(my + COL_Y + 64 * pp + 32, *reinterpret_cast<float(*)[32]>(yv + 32));
      ptx::tc_wait_ld();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[B_YE + pp]);
      if (p.y_direct) {
        // y rows not 16-byte aligned: every thread stores its feature of the chunk's tokens itself
        // (a warp writes 32 consecutive features of one token per store), tokens past T skipped.
        const int t0 = (cb + c) * C;
        TOut* yrow = static_cast<TOut*>(p.y) + (int64_t)b * p.sy.b + (int64_t)h * p.sy.h + dv0 + row;
#pragma unroll 8
        for (int j = 0; j < C; ++j)
          if (t0 + j < p.T) store_as(yrow + (int64_t)(t0 + j) * p.sy.t, yv[j]);
        return true;
      }
      constexpr int ROWS = (int)(TILE / (D * sizeof(TOut)));  // tokens per 8 KB staging piece
      TOut* stage = reinterpret_cast<TOut*>(sm + AB + pp * TILE);
#pragma unroll
      for (int piece = 0; piece < C / ROWS; ++piece) {
        if (piece > 0) {  // the previous piece's bytes must have been read out first
          if (wt == 128) ptx::bulk_wait_read0();
          ptx::named_bar(3, 128);
        }
#pragma unroll
        for (int j = 0; j < ROWS; ++j) store_as(stage + j * D + row, yv[piece * ROWS + j]);
        ptx::fence_proxy_async_smem();
        ptx::named_bar(3, 128);
        if (wt == 128) {
          ptx::tma_store_4d(&tm_y, stage, dv0, h, (cb + c) * C + piece * ROWS, b);
          ptx::bulk_commit();
        }
      }
      if (wt == 128) ptx::bulk_wait_read0();
      return true;
    };
    int c = 0;
#pragma unroll 1
    for (; c < nch; ++c) {
      const int pb = c & 1;
      const uint32_t kq_o = KQ + (c % NR) * KQB;
      uint8_t* kq = sm + kq_o;
      const uint32_t v_o = VB + pb * V_BYTES;
      float* la_s = small + (c % 3) * SLOT;
      float* beta_s = la_s + C;
      float* g_s = beta_s + C;
      float* gam_s = g_s + C;
      float* w_s = gam_s + C;
      float* misc_s = w_s + C;

      if (!gwait(B_KQ + c % NR, (uint32_t)(c / NR) & 1u, leader, 1, NWORK)) break;
      if (leader) {  // G = [K;Q] K^T (or [K;Q] U^T) from the bf16 tiles as loaded
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a = at(D_K, kq_o + (k >> 2) * 2 * TILE + (k & 3) * 32);
          const uint64_t bu = HAS_U ? at(D_K, kq_o + (4 + (k >> 2)) * TILE + (k & 3) * 32) : a;
          ptx::mma_f16_ss(tmem + COL_G, a, bu, ID_G, k > 0);
        }
        ptx::mma_commit(&bars[B_G]);
        issued = true;
      }
      if (ww == 1) {  // chunk-local cumulative log-decay (not on the MMA-issuing warp)
        float a0 = ga0, a1 = ga1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float n0 = __shfl_up_sync(0xffffffffu, a0, o);
          const float n1 = __shfl_up_sync(0xffffffffu, a1, o);
          if (lane >= o) { a0 += n0; a1 += n1; }
        }
        a1 += __shfl_sync(0xffffffffu, a0, 31);
        const float gC = __shfl_sync(0xffffffffu, a1, 31);
        beta_s[lane] = gb0;
        beta_s[lane + 32] = gb1;
        g_s[lane] = a0;
        g_s[lane + 32] = a1;
        gam_s[lane] = expf(a0);
        gam_s[lane + 32] = expf(a1);
        w_s[lane] = gb0 * expf(gC - a0);
        w_s[lane + 32] = gb1 * expf(gC - a1);
        if (lane == 0) misc_s[0] = expf(gC);
      }
      ptx::named_bar(1, NWORK);
      // Decay tables: 1,280 exponentials per chunk instead of one per (t, j) pair.  Every factor
      // is exp of a non-positive number, so none overflows whatever the decay.
#pragma unroll
      for (int n = 0; n < 2; ++n) {  // 64 + 256 entries
        const int e = wt + NWORK * n;
        if (e < C) {
          eT[e] = __expf(g_s[e] - g_s[e & ~15]);
        } else if (e < 5 * C) {
          const int bb = (e - C) >> 6, j = (e - C) & 63;
          eJ[bb * C + j] = (bb > 0 && j < 16 * bb) ? beta_s[j] * __expf(g_s[16 * bb] - g_s[j]) : 0.f;
        }
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int e = wt + NWORK * n;  // 1024 diagonal-block entries
        const int bb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
        Ed[(bb * 16 + r) * 20 + cc] = cc <= r ? beta_s[16 * bb + cc] * __expf(g_s[16 * bb + r] - g_s[16 * bb + cc]) : 0.f;
      }
      if (!virt && !gwait(B_V + pb, (uint32_t)(c >> 1) & 1u, leader, 1, NWORK)) break;
      if (!gwait(B_G, (uint32_t)c & 1u, leader, 1, NWORK)) break;
      if (leader) issued = false;
      ptx::tc_fence_after();

      // bf16 -> fp16 in place: K (tiles 0, 2), gamma-scaled Q (tiles 1, 3) and U (tiles 4, 5).  V
      // stays bf16.
#pragma unroll 4
      for (int i = wt; i < NCONV * 512; i += NWORK) {
        const int tile = i >> 9;
        uint8_t* base = kq + tile * TILE;
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
      // Half-rows of L (TMEM lanes 0-63) and A (lanes 64-127) from G: columns 32 hf .. 32 hf + 31.
      float gv[32];
      ptx::tmem_ld32(my + COL_G + 32 * hf, gv);
      ptx::tc_wait_ld();
      const int t = row & 63, tb = t >> 4;
      const bool is_l = row < 64;
      const float et = eT[t];
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        const int jb = 2 * hf + q2;
        // This thread's decay factors for the 16 columns of block jb (vector loads; the block's
        // case -- below, on or above the diagonal block -- is fixed per thread).
        float e[16];
        const float4* src4 = jb < tb ? reinterpret_cast<const float4*>(eJ + tb * C + 16 * jb)
                                     : reinterpret_cast<const float4*>(Ed + (tb * 16 + (t & 15)) * 20);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 f = src4[v];
          e[4 * v] = f.x; e[4 * v + 1] = f.y; e[4 * v + 2] = f.z; e[4 * v + 3] = f.w;
        }
        const float sc = jb < tb ? et : (jb == tb ? 1.f : 0.f);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          float ej = e[jj] * sc;
          if (is_l && 16 * jb + jj == t) ej = 0.f;
          gv[16 * q2 + jj] *= ej;
        }
      }
      if (is_l) {
        uint8_t* lrow = sm + L16 + t * LD16 + hf * 64;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v4;
          v4.x = pack_h2(gv[q * 8 + 0], gv[q * 8 + 1]);
          v4.y = pack_h2(gv[q * 8 + 2], gv[q * 8 + 3]);
          v4.z = pack_h2(gv[q * 8 + 4], gv[q * 8 + 5]);
          v4.w = pack_h2(gv[q * 8 + 6], gv[q * 8 + 7]);
          *reinterpret_cast<uint4*>(lrow + q * 16) = v4;
        }
        if ((tb >> 1) == hf) {  // this half holds the row's diagonal block: keep it in fp32
          float* drow = reinterpret_cast<float*>(sm + LDIAG) + (tb * 16 + (t & 15)) * LDG;
          const bool second = (tb & 1) != 0;
#pragma unroll
          for (int q = 0; q < 16; q += 4)
            *reinterpret_cast<float4*>(drow + q) =
                second ? make_float4(gv[16 + q], gv[17 + q], gv[18 + q], gv[19 + q]) : make_float4(gv[q], gv[q + 1], gv[q + 2], gv[q + 3]);
        }
      }
      ptx::named_bar(1, NWORK);
      // W16(c-1) shares T16/TG16's space (needs R(c-1) done); A16[pb] was read by Yi(c-2).
      if (c > 0 && !gwait(B_R, (uint32_t)(c - 1) & 1u, leader, 1, NWORK)) break;
      if (want_y && c >= 2 && !gwait(B_YF + pb, (uint32_t)((c - 2) >> 1) & 1u, leader, 1, NWORK)) break;
      if (!is_l) {
        uint8_t* arow = sm + AB + pb * TILE;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v4;
          v4.x = pack_h2(gv[q * 8 + 0], gv[q * 8 + 1]);
          v4.y = pack_h2(gv[q * 8 + 2], gv[q * 8 + 3]);
          v4.z = pack_h2(gv[q * 8 + 4], gv[q * 8 + 5]);
          v4.w = pack_h2(gv[q * 8 + 6], gv[q * 8 + 7]);
          *reinterpret_cast<uint4*>(arow + sw128(t, 4 * hf + q)) = v4;
        }
      } else if (wt < 64) {
        // D_b = (I + L_bb)^-1, one column per thread; right-looking fp32 forward substitution
        // (after x_m is known, every later row's sum takes its term at once: 15 independent FMAs).
        const int bb = wt >> 4, j = wt & 15;
        const float* Lb = reinterpret_cast<const float*>(sm + LDIAG) + bb * 16 * LDG;
        float x[16], acc[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          x[m] = (m == j) ? 1.f : (m > j ? -acc[m] : 0.f);
#pragma unroll
          for (int r = m + 1; r < 16; ++r) acc[r] = fmaf(Lb[r * LDG + m], x[m], acc[r]);
        }
        __half* l16 = reinterpret_cast<__half*>(sm + L16);
#pragma unroll
        for (int r = 0; r < 16; ++r) l16[(bb * 16 + r) * (LD16 / 2) + bb * 16 + j] = __float2half_rn(x[r]);
      }
      bool epi_ok = true;
      if (ww >= 4) {
        if (want_y && c >= 1) epi_ok = epilogue(c - 1);  // overlaps the diagonal blocks and the merges
      } else {
        ptx::named_bar(4, 128);  // D_b in L16 before the merges read it (warps 4-7 only)
        const uint32_t l16a = sb + L16, thi = sb + TW, tlo = sb + TLO, tg16a = sb + TW + TILE;
        merge_column_of<true>(ww, l16a, thi, tlo, tg16a, gam_s, lane);
      }
      ptx::fence_proxy_async_smem();
      if (ptx::named_bar_or(1, NWORK, !epi_ok)) break;
      if (leader) {  // W^T = K^T (T Gamma)^T (waited for below), then U^T = V^T T^T (checked at ready)
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::mma_f16_ss(tmem + COL_W, at(D_MN16K, kq_o + k * 2048), at(D_K, TW + TILE + k * 32), ID_N64_AMN, k > 0);
        ptx::mma_commit(&bars[B_WU]);
        if (!virt) {  // the transition block has v = 0, hence U = 0
#pragma unroll
          for (int k = 0; k < 4; ++k)
            ptx::mma_f16_ss(tmem + COL_U + 64 * pb, at(D_MN8K, v_o + k * 2048), at(D_K, TW + k * 32), ID_U_BF16, k > 0);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            ptx::mma_f16_ss(tmem + COL_U + 64 * pb, at(D_MN8K, v_o + k * 2048), at(D_K, TLO + k * 32), ID_U_BF16, 1);
        }
        ptx::mma_commit(&bars[B_UU]);
        issued = true;
      }
      if (ww == 1 && c + 1 < nch) load_gates(c + 1);  // latency hidden behind the MMAs below
      if (!gwait(B_WU, (uint32_t)c & 1u, leader, 1, NWORK)) break;
      ptx::tc_fence_after();
      {
        float wv[32];
        ptx::tmem_ld32(my + COL_W + 32 * hf, wv);
        ptx::tc_wait_ld();
        uint8_t* wrow = sm + TW;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v4;
          v4.x = pack_h2(wv[q * 8 + 0], wv[q * 8 + 1]);
          v4.y = pack_h2(wv[q * 8 + 2], wv[q * 8 + 3]);
          v4.z = pack_h2(wv[q * 8 + 4], wv[q * 8 + 5]);
          v4.w = pack_h2(wv[q * 8 + 6], wv[q * 8 + 7]);
          *reinterpret_cast<uint4*>(wrow + sw128(row, 4 * hf + q)) = v4;  // W16: row d, 64 tokens
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      {
        bool fail = false;
        if (leader) fail = !ptx::mbar_wait_abortable(&bars[B_UU], (uint32_t)c & 1u, WAIT_LIMIT, abort_flag);
        if (ptx::named_bar_or(1, NWORK, fail)) break;
      }
      if (leader) {
        issued = false;
        ptx::mbar_arrive(&bars[B_PREP]);
        if (!virt && c + 2 < nch) { issue_v(c + 2); v_issued = c + 3; }  // V(c) consumed by U^T(c)
      }
    }
    if (want_y && c == nch && nch > 0 && ww >= 4) epilogue(nch - 1);
    if (wt == 128) ptx::bulk_wait0();
    if (*abort_flag && leader) {  // drain this thread's MMAs and V loads before the CTA exits
      if (issued) {
        ptx::mma_commit(&bars[B_DRAIN]);
        ptx::mbar_wait_bounded(&bars[B_DRAIN], 0, WAIT_LIMIT);
      }
      for (int cc = v_issued - 2 < 0 ? 0 : v_issued - 2; cc < v_issued; ++cc)
        ptx::mbar_wait_bounded(&bars[B_V + (cc & 1)], (uint32_t)(cc >> 1) & 1u, WAIT_LIMIT);
    }
  } else {
    // ==================================== state chain ====================================
    const int ct = tid;
    const bool leader = ct == 0;
    bool issued = false;
    {
      // Initial state: the caller's S_0 (first segment), the combined state of the previous
      // segments (later segments), or in state mode 0 (v block) / the identity (transition block).
      const float* src = nullptr;
      if (want_y) {
        if (seg == 0) {
          if (p.s0) src = p.s0 + ((int64_t)bh * p.DV + dv0 + ct) * D;
        } else {
          src = p.seg_s0 + ((int64_t)(bh * p.ws_stride + seg - 1) * (p.DV + D) + dv0 + ct) * D;
        }
      }
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 t4 = src ? *reinterpret_cast<const float4*>(src + c4 * 32 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[i] = t4.x; v[i + 1] = t4.y; v[i + 2] = t4.z; v[i + 3] = t4.w;
        }
        if (virt) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = (c4 * 32 + i == ct) ? 1.f : 0.f;
        }
        ptx::tmem_st32(my + COL_S + c4 * 32, v);
      }
      ptx::tc_wait_st();
    }
    int kq_issued = 0;
    if (leader) {
      issue_kq(0);
      kq_issued = 1;
      if (nch > 1) { issue_kq(1); kq_issued = 2; }
    }
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int pb = c & 1;
      const uint32_t kq_o = KQ + (c % NR) * KQB;
      const float* slot = small + (c % 3) * SLOT;
      const float* w_s = slot + 4 * C;
      // The next tile load goes into the ring entry of chunk c-1, freed by S(c-1).  With two entries
      // (HAS_U) it is chunk c+1's, which prep(c+1) waits for, so it is issued before waiting for prep(c).
      if (HAS_U) {
        if (c > 0) {
          if (!gwait(B_S, (uint32_t)(c - 1) & 1u, leader, 2, 128)) break;
          if (leader) issued = false;
        }
        ptx::tc_fence_after();
        const int nxt = c + NR - 1;
        if (leader && nxt < nch && nxt >= kq_issued) { issue_kq(nxt); kq_issued = nxt + 1; }
      }
      if (!gwait(B_PREP, (uint32_t)c & 1u, leader, 2, 128)) break;
      const float gC = slot[5 * C];  // written by prep(c): read only after its ready barrier
      if (!HAS_U) {
        if (c > 0) {
          if (!gwait(B_S, (uint32_t)(c - 1) & 1u, leader, 2, 128)) break;
          if (leader) issued = false;
        }
        ptx::tc_fence_after();
        const int nxt = c + NR - 1;
        if (leader && nxt < nch && nxt >= kq_issued) { issue_kq(nxt); kq_issued = nxt + 1; }
      }
      ptx::tc_fence_after();
      // S16 <- fp16(S): four loads, one wait.
      float sv[128];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) ptx::tmem_ld32(my + COL_S + c4 * 32, *reinterpret_cast<float(*)[32]>(sv + 32 * c4));
      ptx::tc_wait_ld();
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        uint4 pk;
        pk.x = pack_h2(sv[q * 8 + 0], sv[q * 8 + 1]);
        pk.y = pack_h2(sv[q * 8 + 2], sv[q * 8 + 3]);
        pk.z = pack_h2(sv[q * 8 + 4], sv[q * 8 + 5]);
        pk.w = pack_h2(sv[q * 8 + 6], sv[q * 8 + 7]);
        *reinterpret_cast<uint4*>(sm + SR + (q >> 3) * 2 * TILE + sw128(ct, q & 7)) = pk;
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      ptx::named_bar(2, 128);
      bool r_ok = true;
      if (leader) {  // R^T = U^T - S W^T ; Y = S (Gamma Q)^T
        ptx::tc_fence_after();
        if (want_y && c >= 2)  // Y[pb] drained by the workers
          r_ok = ptx::mbar_wait_abortable(&bars[B_YE + pb], (uint32_t)((c - 2) >> 1) & 1u, WAIT_LIMIT, abort_flag);
        if (r_ok) {
#pragma unroll
          for (int k = 0; k < 8; ++k)  // onto U^T; the transition block starts from U = 0
            ptx::mma_f16_ss(tmem + COL_U + 64 * pb, at(D_K, SR + (k >> 2) * 2 * TILE + (k & 3) * 32),
                            at(D_K, TW + k * 2048), ID_N64_BMN_NEG, virt ? (k > 0) : 1);
          if (want_y) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
              ptx::mma_f16_ss(tmem + COL_Y + 64 * pb, at(D_K, SR + (k >> 2) * 2 * TILE + (k & 3) * 32),
                              at(D_K, kq_o + TILE + (k >> 2) * 2 * TILE + (k & 3) * 32), ID_N64, k > 0);
          }
          ptx::mma_commit(&bars[B_R]);
          issued = true;
        }
      }
      // S <- gamma_C S while the MMAs run (they do not touch the S columns).
#pragma unroll
      for (int i = 0; i < 128; ++i) sv[i] *= gC;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) ptx::tmem_st32(my + COL_S + c4 * 32, *reinterpret_cast<float(*)[32]>(sv + 32 * c4));
      ptx::tc_wait_st();
      {
        bool fail = false;
        if (leader) fail = !r_ok || !ptx::mbar_wait_abortable(&bars[B_R], (uint32_t)c & 1u, WAIT_LIMIT, abort_flag);
        if (ptx::named_bar_or(2, 128, fail)) break;
      }
      if (leader) issued = false;
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
      if (leader) {  // S += (R diag w)^T K ; Y += R^T A^T
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::mma_f16_ss(tmem + COL_S, at(D_K, SR + 2 * TILE + k * 32),
                          HAS_U ? at(D_MN8K, kq_o + 4 * TILE + k * 2048) : at(D_MN16K, kq_o + k * 2048), ID_N128_BMN, 1);
        if (want_y) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            ptx::mma_f16_ss(tmem + COL_Y + 64 * pb, at(D_K, SR + k * 32), at(D_K, AB + pb * TILE + k * 32), ID_N64, 1);
        }
        ptx::mma_commit(&bars[B_S]);
        if (want_y) ptx::mma_commit(&bars[B_YF + pb]);
        issued = true;
      }
    }
    if (!*abort_flag && nch > 0 && gwait(B_S, (uint32_t)(nch - 1) & 1u, leader, 2, 128)) {
      if (leader) issued = false;
      ptx::tc_fence_after();
      float* dst = nullptr;
      if (want_y && seg == p.nseg - 1 && p.s_out != nullptr) dst = p.s_out + ((int64_t)bh * p.DV + dv0 + ct) * D;
      if (!want_y) dst = p.seg_out + ((int64_t)(bh * p.ws_stride + seg) * (p.DV + D) + dv0 + ct) * D;
      if (dst != nullptr) {
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
    if (*abort_flag && leader) {  // drain this thread's MMAs and q/k loads before the CTA exits
      if (issued) {
        ptx::mma_commit(&bars[B_DRAIN + 1]);
        ptx::mbar_wait_bounded(&bars[B_DRAIN + 1], 0, WAIT_LIMIT);
      }
      for (int c = kq_issued - NR < 0 ? 0 : kq_issued - NR; c < kq_issued; ++c)
        ptx::mbar_wait_bounded(&bars[B_KQ + c % NR], (uint32_t)(c / NR) & 1u, WAIT_LIMIT);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (tid == 0 && *abort_flag) atomicExch(&g_status, GDN_ERR_TIMEOUT);
  if (warp == 0) ptx::tmem_dealloc(tmem, TMEM_COLS);
}

struct Segmentation {
  int mode = 0, nseg = 1, seg_len = 0, ws_stride = 0;
  const float* seg_s0 = nullptr;
  float* seg_out = nullptr;
};

template <bool HAS_U, typename TOut>
int launch(const gdn_prefill_args* a, const Segmentation& sg, cudaStream_t stream) {
  CUtensorMap mq, mk, mv, my, mu;
  const bool y_tma = gdn_y_tma_ok(a);  // else y is written by direct stores (no tensor map)
  memset(&my, 0, sizeof(my));
  if (!make_map(&mq, a->q, a->DK, a, a->sq) || !make_map(&mk, a->k, a->DK, a, a->sk) ||
      !make_map(&mv, a->v, a->DV, a, a->sv) || (y_tma && !make_store_map<TOut>(&my, a->y, a->DV, a, a->sy)))
    return GDN_ERR_LAUNCH;
  if (HAS_U != (a->u != nullptr)) return GDN_ERR_UNSUPPORTED;
  if (HAS_U) {
    if (!make_map(&mu, a->u, a->DK, a, a->su)) return GDN_ERR_LAUNCH;
  } else {
    mu = mk;
  }
  auto kern = ws_kernel<HAS_U, TOut>;
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)kern, (int)(DYN)}})) return GDN_ERR_LAUNCH;
  const int nch = (int)((a->T + C - 1) / C);
  Params p;
  p.beta = a->beta; p.la = a->la; p.s0 = a->s0; p.s_out = a->s_out; p.y = a->y; p.sy = a->sy;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DV = (int)a->DV;
  p.nv = (int)(a->DV / D);
  p.mode = sg.mode;
  p.ntiles = p.nv + (sg.mode == 1 ? 1 : 0);
  p.nseg = sg.nseg;
  p.seg_len = sg.seg_len > 0 ? sg.seg_len : nch;
  p.seg_s0 = sg.seg_s0;
  p.seg_out = sg.seg_out;
  p.ws_stride = sg.ws_stride;
  p.y_direct = y_tma ? 0 : 1;
  const int64_t grid = a->B * a->H * (int64_t)p.nseg * p.ntiles;
  if (grid <= 0 || grid > 0x7fffffff) return GDN_ERR_SHAPE;
  kern<<<(unsigned)grid, NT, DYN, stream>>>(mq, mk, mv, my, mu, p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

template <typename TOut>
int launch(const gdn_prefill_args* a, cudaStream_t stream) {
  return a->u ? launch<true, TOut>(a, Segmentation(), stream) : launch<false, TOut>(a, Segmentation(), stream);
}

}  // namespace ws
}  // namespace gdn

// DK = 128, DV a multiple of 128; u = beta k or an explicit write vector u.
// y can be stored by TMA: 16-byte-aligned base and row strides.
bool gdn_y_tma_ok(const gdn_prefill_args* a) {
  const int64_t es = a->out_dtype == GDN_DTYPE_BF16 ? 2 : 4;
  auto ok = [&](int64_t x) { return x > 0 && (x * es) % 16 == 0; };
  return a->y && (uintptr_t)a->y % 16 == 0 && ok(a->sy.h) && ok(a->sy.t) && ok(a->sy.b);
}

// DK = 128 and DV a multiple of 128; y of any strides (TMA stores where y allows them, direct
// stores otherwise).
bool gdn_chunk_ws_supported(const gdn_prefill_args* a) {
  return a->DK == 128 && a->DV % 128 == 0 && a->DV >= 128 && a->DV <= 8 * 128;
}

namespace {
// A row of a [B][T][H][D] bf16 tensor can be TMA-loaded: 16-byte-aligned base and strides.
bool tma_ok(const void* ptr, const gdn_strides& s) {
  auto a16 = [](int64_t x) { return x > 0 && (x * 2) % 16 == 0 && x * 2 < (1LL << 40); };
  return ptr && ((uintptr_t)ptr % 16 == 0) && a16(s.h) && a16(s.t) && a16(s.b);
}
}  // namespace

// The chunked path (the single-CTA kernel, or the cluster kernel where it applies): bf16 inputs,
// DK = 128, DV a multiple of 128 up to 1024, u = beta k or an explicit write vector u (nsgdn
// n_steps > 1), 16-byte-aligned q/k/u/v rows for the TMA loads and states for the vector accesses.
bool gdn_chunk_supported(const gdn_prefill_args* a) {
  if (a->in_dtype != GDN_DTYPE_BF16 || a->DK != 128 || a->T < 1) return false;
  if (!tma_ok(a->q, a->sq) || !tma_ok(a->k, a->sk) || !tma_ok(a->v, a->sv)) return false;
  if (a->u && !tma_ok(a->u, a->su)) return false;
  if ((a->s0 && (uintptr_t)a->s0 % 16) || (a->s_out && (uintptr_t)a->s_out % 16)) return false;
  return gdn_chunk_ws_supported(a);
}

int gdn_launch_chunk_sm100(const gdn_prefill_args* a, cudaStream_t stream) { return gdn_launch_chunk_ws(a, stream); }

int gdn_chunk_read_status(int* out, int reset) { return gdn_chunk_ws_read_status(out, reset); }

int gdn_launch_chunk_ws(const gdn_prefill_args* a, cudaStream_t stream) {
  return a->out_dtype == GDN_DTYPE_BF16 ? gdn::ws::launch<__nv_bfloat16>(a, stream) : gdn::ws::launch<float>(a, stream);
}

// One pass of the segmented prefill.  mode 1: segments [0, nseg) write [N_s; M_s] to `ws`
// (slots of `ws_stride` per (b, h)); mode 0: segment s >= 1 starts from the state stored at slot
// s - 1 of `ws`, the last segment writes S_T.
int gdn_launch_chunk_ws_segments(const gdn_prefill_args* a, int mode, int nseg, int seg_len, float* ws, int ws_stride,
                                 cudaStream_t stream) {
  gdn::ws::Segmentation sg;
  sg.mode = mode;
  sg.nseg = nseg;
  sg.seg_len = seg_len;
  sg.ws_stride = ws_stride;
  sg.seg_s0 = ws;
  sg.seg_out = ws;
  if (a->u != nullptr)
    return a->out_dtype == GDN_DTYPE_BF16 ? gdn::ws::launch<true, __nv_bfloat16>(a, sg, stream)
                                          : gdn::ws::launch<true, float>(a, sg, stream);
  return a->out_dtype == GDN_DTYPE_BF16 ? gdn::ws::launch<false, __nv_bfloat16>(a, sg, stream)
                                        : gdn::ws::launch<false, float>(a, sg, stream);
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
