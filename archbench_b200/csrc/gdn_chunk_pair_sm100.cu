// Cluster-pair chunkwise gated delta rule (u = beta k) on tcgen05 / TMEM, sm_100a.
//
// Same mathematics as gdn_chunk_ws_sm100.cu (the WY form of archbench/layers/nsgdn.py:408-417,
// derivation as in nsgdn.py:240-249).  One cluster of two CTAs per (b, h) sequence, on two SMs,
// so that a batch of few sequences still covers most of the GPU and the state recurrence does
// not share its SM with the state-independent work:
//
//   prep CTA (rank 1)   two chunks in flight (warps 0-3: even chunks, warps 4-7: odd chunks):
//                       G = [K;Q] K^T (bf16 operands as loaded), gates and decay tables, the rows
//                       of L and A, T = (I + L)^-1 (fp32 16x16 diagonal blocks, fp16 mma.sync
//                       block columns) and T Gamma.  A, T and T Gamma (fp16, 24 KB per chunk) go
//                       straight into a product slot in the state CTA's shared memory.
//   state CTA (rank 0)  chain (warps 0-3): U^T = V^T T^T, S -> fp16, then one N = 128 MMA for
//                       [R^T | Y] = [U^T | 0] - S [W | -Gamma Q]^T, S <- gamma_C S + (R diag w)^T K,
//                       Y += R^T A^T.  The fp16 copies of S, R and R diag(w) stay in tensor memory
//                       as the A operands of their MMAs; R and S are each committed alone.
//                       convert (warps 4-7): gates, W^T = K^T (T Gamma)^T -> W16; issues the v tile
//                       loads.
//                       output (warps 8-11): Y -> y through a staging tile and TMA stores (and Y
//                       zeroed for the next chunk), QT16 = (-Gamma Q)^T of the next chunk; issues
//                       the k/q tile loads.  W16 and QT16, both with DK rows, sit side by side as
//                       the B operand of the fused MMA.
//                       The convert warps turn each chunk's k tiles, the output warps its v tiles, to
//                       fp16 in place.
//
// Handoff: prep pipeline p stages its chunk's products locally (two staging buffers per pipeline)
// and sends them into slot p of the state CTA with one asynchronous bulk copy that completes on
// the slot's full barrier there; the output warps hand the slot back by arriving on the
// pipeline's empty barrier once the chunk's last MMA (the one that reads A) has completed.  A
// staging buffer is rewritten two pipeline chunks later, after the pipeline has seen the slot of
// the chunk in between given back, so its copy has long completed.  The prep CTA loads each chunk's k and q
// tiles with TMA and pulls its v tile into L2, so the state CTA's own tile loads (issued as soon
// as the chunk two back has released their buffers) are L2 hits.
//
// Every mbarrier wait is bounded and abortable.  An abort raised in either CTA is copied into the
// other; both drain their own MMAs and tile loads, and the two CTAs leave through one cluster
// barrier, so neither exits while the other may still write into its shared memory.
//
// State-only mode (SPLIT): the state CTA alone, one per (b, h, segment, 128-row state tile), no
// cluster.  The products of every chunk were written beforehand by the prep kernel
// (gdn_chunk_prep_sm100.cu, the same arithmetic as the prep CTA here), and the output warps bulk-load
// chunk c + 2's into the product slot chunk c has released.  This serves what one prep CTA per
// state tile cannot: state rows beyond 128 (DV = 256: two state CTAs share one chunk's products
// instead of each preparing them), explicit write vectors (HAS_U: the u tiles ride in a two-entry
// k/q ring and replace k where the state is written, S += (R diag w)^T U, w free of beta) and the
// passes of the segmented prefill (mode 1: no y; the transition block, S_0 = I and v = 0, as an extra
// tile; the segment's end state written to the segment workspace).
#include "gdn_tiles.cuh"

namespace gdn {
namespace pair {

using namespace gdn::tiles;

constexpr int NT = 384;
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clocks

constexpr uint32_t KQ_BYTES = 4 * TILE;  // [K0][Q0][K1][Q1]: features 0-63 and 64-127 of k and q
constexpr uint32_t V_BYTES = 2 * TILE;   // [V0][V1]
constexpr uint32_t PS_BYTES = 3 * TILE;  // product slot: [A16][T16][TG16]
constexpr int NB = 3;                    // k/q tile buffers of the state CTA: chunk c uses buffer c % NB
constexpr int NBV = 2;                   // v tile buffers: chunk c uses buffer c % NBV
constexpr uint32_t RING_BYTES = NB * KQ_BYTES;  // the k/q ring: three [K0][Q0][K1][Q1] entries, or
                                                // two [K0][Q0][K1][Q1][U0][U1] with write vectors

// State CTA shared-memory map (bytes from a 1024-aligned base).
constexpr uint32_t S_KQ = 0;                       // NB x KQ: bf16 as loaded -> fp16 K (and U) in place (q stays bf16)
constexpr uint32_t S_V = S_KQ + RING_BYTES;        // NBV x V: bf16 -> fp16 in place
constexpr uint32_t S_WQ = S_V + NBV * V_BYTES;     // [W16 | QT16]: DK rows x 64 tokens each, 16 KB apart
constexpr uint32_t S_PS = S_WQ + 4 * TILE;         // 2 product slots, written by the prep CTA
constexpr uint32_t S_YS = S_PS + 2 * PS_BYTES;     // y staging: one bf16 chunk (or half an fp32 one)
constexpr uint32_t YS_BYTES = 2 * TILE;
constexpr uint32_t S_GS = S_YS + YS_BYTES;         // NB gate slots: gamma[64], w[64], gamma_C
constexpr uint32_t GSLOT = 2 * C + 4;              // floats per gate slot
constexpr uint32_t S_BARS = S_GS + NB * GSLOT * 4;
constexpr uint32_t S_NBARS = 18;

// Prep CTA shared-memory map: pipeline p at p * P_STRIDE.
constexpr uint32_t P_KQ = 0;                                  // KQ tile set, bf16 as loaded
constexpr uint32_t P_ST = P_KQ + KQ_BYTES;                    // 2 staging buffers [A16][T16][TG16]
constexpr uint32_t P_L16 = P_ST + 2 * PS_BYTES;               // 64 rows x LD16 bytes (diagonal blocks hold D_b)
constexpr uint32_t P_LDIAG = P_L16 + 64 * LD16;               // 4 x 16 x LDG floats
constexpr uint32_t P_EXPT = P_LDIAG + 4 * 16 * LDG * 4;       // decay tables: 64 + 4x64 + 4x16x20 floats
constexpr uint32_t P_GS = P_EXPT + (64 + 4 * 64 + 4 * 16 * 20) * 4;  // beta[64], g[64], gamma[64]
constexpr uint32_t P_STRIDE = ((P_GS + 3 * C * 4) + 1023) / 1024 * 1024;
constexpr uint32_t P_BARS = 2 * P_STRIDE;
constexpr uint32_t P_NBARS = 8;

constexpr uint32_t cmax(uint32_t a, uint32_t b) { return a > b ? a : b; }
// Control words: TMEM base, abort flag, k/q and v tile loads issued (state), product slots seen by
// the chain (state, per slot), product copies issued (written into the state CTA by the prep, per
// slot).
constexpr uint32_t CTRL = (cmax(S_BARS + S_NBARS * 8, P_BARS + P_NBARS * 8) + 15) / 16 * 16;
constexpr uint32_t TOTAL = CTRL + 32;
constexpr uint32_t DYN = TOTAL + 1024;
static_assert(DYN <= 232448, "shared memory budget");
static_assert(S_V % 1024 == 0 && S_WQ % 1024 == 0 && S_PS % 1024 == 0, "swizzled tiles need 1 KB alignment");
static_assert(P_STRIDE % 1024 == 0 && P_ST % 1024 == 0, "swizzled tiles need 1 KB alignment");

// TMEM columns of the state CTA (all 512) and of the prep CTA (128: G of each pipeline).  S16, R16
// and RW16 hold two fp16 values per column; Y follows U (the fused MMA's 128 output columns).
constexpr uint32_t COL_S = 0, COL_S16 = 128, COL_U = 192, COL_Y = 256, COL_R16 = 320, COL_RW16 = 352, COL_W = 384;

enum SBar {
  SB_PF = 0,                                                       // per product slot (2)
  SB_KQR = 2, SB_KQF = 5,                                          // per k/q tile buffer (NB)
  SB_VF = 8,                                                       // per v tile buffer (NBV)
  SB_WM = 10, SB_W16R = 11, SB_R = 12, SB_S = 13, SB_YF = 14, SB_YE = 15, SB_DRAIN = 16  // DRAIN: 2
};
enum PBar { PB_KQF = 0, PB_G = 2, PB_PE = 4, PB_DRAIN = 6 };

struct Params {
  const float* beta;  // NULL with explicit write vectors
  const float* la;
  const float* s0;
  float* s_out;
  int B, T, H, DV;
  // Segments: cluster (b, h, seg) runs chunks [seg * seg_len, (seg + 1) * seg_len); segment s >= 1
  // starts from the state at slot (bh, s - 1) of seg_s0 ((DV + 128) x 128 floats per slot).
  int nseg, seg_len;
  const float* seg_s0;
  int ws_stride;
  // State-only mode: chunk products [B * H][NCt] x PS_BYTES from the prep kernel; state tiles per
  // (b, h, seg) (nv real ones of 128 rows, plus the transition block in mode 1); mode 1 writes
  // [N_s; M_s] of segment s to slot (bh, s) of seg_out instead of y.
  const uint8_t* prod;
  int NCt, nv, ntiles, mode;
  float* seg_out;
};

__device__ int g_status = 0;

__device__ __forceinline__ void cumsum_gates(float la0, float la1, float& g0, float& g1, float& gC) {
  const int lane = threadIdx.x & 31;
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
  gC = __shfl_sync(0xffffffffu, a1, 31);
  g0 = a0;
  g1 = a1;
}

// This thread's share (`ht` = 0..127 of a warp group) of the bf16 -> fp16 conversion in place of
// two 64x64 tiles: the k tiles of a chunk (convert warps) or its v tiles (output warps).  All eight
// loads are in flight before the first store; the writes are then fenced for the tensor core.  Not
// inlined: one copy serves both groups (the kernel's instruction working set, not latency, is what
// limits it when many clusters share a GPC).
__device__ __noinline__ void convert_pair(uint8_t* t0, uint8_t* t1, int ht) {
  uint4 r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = ht + 128 * j;
    r[j] = *reinterpret_cast<const uint4*>(((i >> 9) ? t1 : t0) + (i & 511) * 16);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = ht + 128 * j;
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&r[j]);
    uint4 o;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(b2[k]);
      o32[k] = pack_h2(f.x, f.y);
    }
    *reinterpret_cast<uint4*>(((i >> 9) ? t1 : t0) + (i & 511) * 16) = o;
  }
  ptx::fence_proxy_async_smem();
}

template <bool SPLIT, bool HAS_U, typename TOut>
__global__ void __launch_bounds__(NT, 1)
    pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_y,
                const __grid_constant__ CUtensorMap tm_u, const Params p) {
  static_assert(SPLIT || !HAS_U, "explicit write vectors take the state-only mode");
  constexpr int NBK = HAS_U ? 2 : NB;                           // k/q ring entries
  constexpr uint32_t KQB = HAS_U ? 6 * TILE : KQ_BYTES;         // bytes per ring entry
  static_assert(NBK * KQB == RING_BYTES, "the ring keeps its footprint");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = SPLIT ? 0u : ptx::cluster_ctarank();
  const int tile = SPLIT ? (int)(blockIdx.x % (unsigned)p.ntiles) : 0;
  const int rest = SPLIT ? (int)(blockIdx.x / (unsigned)p.ntiles) : (int)(blockIdx.x >> 1);
  const int seg = rest % p.nseg, bh = rest / p.nseg;
  const int b = bh / p.H, h = bh % p.H;
  const int cb = seg * p.seg_len;  // first chunk of this cluster's segment
  const int nch = max(0, min((p.T + C - 1) / C - cb, p.seg_len));
  const bool virt = SPLIT && tile >= p.nv;   // mode 1's transition block: S_0 = I, v = 0
  const bool want_y = !SPLIT || p.mode == 0;
  const int dv0 = virt ? 0 : D * tile;       // first state row (and v / y feature) of this tile

  uint64_t* sbar = reinterpret_cast<uint64_t*>(sm + S_BARS);
  uint64_t* pbar = reinterpret_cast<uint64_t*>(sm + P_BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + CTRL);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + CTRL + 4);
  volatile int* loads_issued = reinterpret_cast<volatile int*>(sm + CTRL + 8);
  volatile int* v_loads_issued = reinterpret_cast<volatile int*>(sm + CTRL + 12);
  const uint32_t peer_abort = SPLIT ? 0u : ptx::mapa_shared(sb + CTRL + 4, rank ^ 1u);
  // Abort here and in the other CTA of the cluster (idempotent).
  auto raise_abort = [&]() {
    *abort_flag = 1;
    if (!SPLIT) ptx::st_cluster_u32(peer_abort, 1u);
  };

  const uint32_t tmem_cols = rank == 0 ? 512u : 128u;
  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, tmem_cols);
    ptx::tmem_relinquish();
  }
  if (tid == 32) {
    if (rank == 0) {
      for (int i = 0; i < (int)S_NBARS; ++i)
        ptx::mbar_init(&sbar[i], i == SB_YE ? 4 : (i == SB_W16R || (i >= SB_KQR && i < SB_KQR + NB)) ? 2 : 1);
      ptx::prefetch_tensormap(&tm_y);
    } else {
      for (int i = 0; i < (int)P_NBARS; ++i) ptx::mbar_init(&pbar[i], 1);
    }
    ptx::prefetch_tensormap(&tm_q);
    ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_v);
    if (HAS_U) ptx::prefetch_tensormap(&tm_u);
    *abort_flag = 0;
    *loads_issued = 0;
    *v_loads_issued = 0;
    for (int i = 4; i < 8; ++i) reinterpret_cast<volatile int*>(sm + CTRL)[i] = 0;
    ptx::fence_mbar_init();
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (!SPLIT) ptx::cluster_sync();  // both CTAs' barriers exist before any remote arrive
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t my = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lane quarter
  const int row = tid & 127;                                         // TMEM lane of this thread

  const uint64_t D_K = ptx::sdesc_sw128(sb, 16, 1024);            // K-major operands
  const uint64_t D_MN16K = ptx::sdesc_sw128(sb, 2 * TILE, 1024);  // MN-major, 64-blocks 16 KB apart
  const uint64_t D_MN8K = ptx::sdesc_sw128(sb, TILE, 1024);       // MN-major, 64-blocks 8 KB apart
  auto at = [](uint64_t tmpl, uint32_t off) { return tmpl + (uint64_t)(off >> 4); };
  constexpr uint32_t ID_G = ptx::idesc_bf16_f32(128, 64);
  constexpr uint32_t ID_N64 = ptx::idesc_f16_f32(128, 64, false, false, false);
  constexpr uint32_t ID_N64_AMN = ptx::idesc_f16_f32(128, 64, true, false, false);
  constexpr uint32_t ID_N128_BMN_NEG = ptx::idesc_f16_f32(128, 128, false, true, true);
  constexpr uint32_t ID_N64_BMN_NEG = ptx::idesc_f16_f32(128, 64, false, true, true);
  constexpr uint32_t ID_N128_BMN = ptx::idesc_f16_f32(128, 128, false, true, false);

  // la and beta of 64 tokens, two per lane (zero past the end of the sequence; beta = 1 with
  // explicit write vectors, which carry it).
  auto load_gates = [&](int c, float& la0, float& la1, float& be0, float& be1) {
    la0 = la1 = be0 = be1 = 0.f;
    const int t0 = (cb + c) * C;
    const int64_t gi = ((int64_t)b * p.T + t0) * p.H + h;
    if (t0 + lane < p.T) {
      la0 = p.la[gi + (int64_t)lane * p.H];
      be0 = HAS_U ? 1.f : p.beta[gi + (int64_t)lane * p.H];
    }
    if (t0 + lane + 32 < p.T) {
      la1 = p.la[gi + (int64_t)(lane + 32) * p.H];
      be1 = HAS_U ? 1.f : p.beta[gi + (int64_t)(lane + 32) * p.H];
    }
  };
  auto issue_kq = [&](uint8_t* dst, uint64_t* bar, int c) {  // the caller has set the barrier's byte count
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

  if (rank == 0) {
    // ======================================= state CTA =======================================
    // One elected thread of a group waits; a reducing named barrier hands the outcome to the group.
    auto gwait = [&](int bar, uint32_t parity, bool leader, int group, bool cluster_scope) -> bool {
      bool fail = false;
      if (leader) {
        fail = cluster_scope ? !ptx::mbar_wait_abortable_cluster(&sbar[bar], parity, WAIT_LIMIT, abort_flag)
                             : !ptx::mbar_wait_abortable(&sbar[bar], parity, WAIT_LIMIT, abort_flag);
        if (fail) raise_abort();
      }
      return !ptx::named_bar_or(group, 128, fail);
    };
    // Several waits of one elected thread handed to its group with one reducing barrier: `fail`
    // accumulates the waits (each a no-op once one has failed); agree() raises the abort and
    // returns whether the whole group goes on.
    auto lwait = [&](bool& fail, int bar, uint32_t parity) {
      if (!fail) fail = !ptx::mbar_wait_abortable(&sbar[bar], parity, WAIT_LIMIT, abort_flag);
    };
    auto agree = [&](bool fail, bool leader, int group) -> bool {
      if (leader && fail) raise_abort();
      return !ptx::named_bar_or(group, 128, leader && fail);
    };
    // k and q (and u) tiles of chunk c into buffer c % NBK (one thread of the output warps; every
    // MMA of the buffer's previous chunk, c - NBK, has completed).  The state-only kernel has no prep
    // CTA pulling its tiles into L2 a chunk ahead: it prefetches the next chunk's tiles itself.
    auto issue_loads = [&](int c) {
      uint64_t* bar = &sbar[SB_KQF + c % NBK];
      ptx::mbar_arrive_expect_tx(bar, KQB);
      issue_kq(sm + S_KQ + (c % NBK) * KQB, bar, c);
      *loads_issued = c + 1;
      if (SPLIT && c + 1 < nch) {
        const int t1 = (cb + c + 1) * C;
        ptx::tma_prefetch_4d(&tm_k, 0, h, t1, b);
        ptx::tma_prefetch_4d(&tm_k, 64, h, t1, b);
        ptx::tma_prefetch_4d(&tm_q, 0, h, t1, b);
        ptx::tma_prefetch_4d(&tm_q, 64, h, t1, b);
        if (HAS_U) {
          ptx::tma_prefetch_4d(&tm_u, 0, h, t1, b);
          ptx::tma_prefetch_4d(&tm_u, 64, h, t1, b);
        }
        if (!virt) {
          ptx::tma_prefetch_4d(&tm_v, dv0, h, t1, b);
          ptx::tma_prefetch_4d(&tm_v, dv0 + 64, h, t1, b);
        }
      }
    };
    // v tiles of chunk c into buffer c % NBV (convert warps; the buffer's previous chunk's U MMA,
    // covered by that chunk's R commit, has completed).  The transition block has none (v = 0).
    auto issue_v_loads = [&](int c) {
      uint64_t* bar = &sbar[SB_VF + c % NBV];
      uint8_t* dst = sm + S_V + (c % NBV) * V_BYTES;
      ptx::mbar_arrive_expect_tx(bar, V_BYTES);
      ptx::tma_load_4d(dst, &tm_v, bar, dv0, h, (cb + c) * C, b);
      ptx::tma_load_4d(dst + TILE, &tm_v, bar, dv0 + 64, h, (cb + c) * C, b);
      *v_loads_issued = c + 1;
    };
    // State-only mode: the products of chunk c into slot c & 1 (the slot's previous chunk, c - 2,
    // has completed every MMA), counted per slot for the abort drain.
    auto issue_products = [&](int c) {
      const int s = c & 1;
      ptx::mbar_arrive_expect_tx(&sbar[SB_PF + s], PS_BYTES);
      ptx::bulk_load(sm + S_PS + s * PS_BYTES, p.prod + ((int64_t)bh * p.NCt + cb + c) * PS_BYTES, PS_BYTES,
                     &sbar[SB_PF + s]);
      reinterpret_cast<volatile int*>(sm + CTRL + 24)[s] = (c >> 1) + 1;
    };
    float* gslots = reinterpret_cast<float*>(sm + S_GS);

    if (warp < 4) {
      // ----------------------------------- state chain -----------------------------------
      const bool leader = tid == 0;
      bool issued = false;
      {
        // Initial state: the caller's S_0 (first segment) or the combined state of the segments
        // before; in mode 1, zero (a real tile) or the identity (the transition block).
        const float* src = nullptr;
        if (want_y) {
          if (seg == 0) {
            if (p.s0) src = p.s0 + ((int64_t)bh * p.DV + dv0 + row) * D;
          } else {
            src = p.seg_s0 + ((int64_t)(bh * p.ws_stride + seg - 1) * (p.DV + D) + dv0 + row) * D;
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
            for (int i = 0; i < 32; ++i) v[i] = (c4 * 32 + i == row) ? 1.f : 0.f;
          }
          ptx::tmem_st32(my + COL_S + c4 * 32, v);
        }
        float z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0.f;
        ptx::tmem_st32(my + COL_Y, z);  // the fused MMA accumulates Y onto zeros
        ptx::tmem_st32(my + COL_Y + 32, z);
        ptx::tc_wait_st();
      }
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int s = c & 1, tb = c % NBK;  // product slot; k/q tile buffer
        const uint32_t ph = (uint32_t)(c >> 1) & 1u, tph = (uint32_t)(c / NBK) & 1u;
        const uint32_t kq_o = S_KQ + tb * KQB, v_o = S_V + (c % NBV) * V_BYTES, ps_o = S_PS + s * PS_BYTES;
        const float* gs = gslots + tb * GSLOT;
        {
          // S(c-1) done; fp16 K and V and the gates of chunk c; A, T, T Gamma of chunk c from the
          // prep CTA.
          bool fail = false;
          if (leader) {
            if (c > 0) lwait(fail, SB_S, (uint32_t)(c - 1) & 1u);
            lwait(fail, SB_KQR + tb, tph);
            if (!fail) fail = !ptx::mbar_wait_abortable_cluster(&sbar[SB_PF + s], ph, WAIT_LIMIT, abort_flag);
          }
          if (!agree(fail, leader, 1)) break;
        }
        if (leader) *reinterpret_cast<volatile int*>(sm + CTRL + 16 + 4 * s) = (c >> 1) + 1;
        const float gC = gs[2 * C];
        ptx::tc_fence_after();
        if (warp == 0 && !virt) {  // U^T = V^T T^T while the state is converted (issued from the converged warp)
#pragma unroll 1
          for (int k = 0; k < 4; ++k)
            ptx::mma_f16_ss_elect(tmem + COL_U, at(D_MN8K, v_o + k * 2048), at(D_K, ps_o + TILE + k * 32), ID_N64_AMN,
                                  k > 0);
          issued = true;
        }
        // S -> S16 (fp16, tensor memory: the A operand of the fused MMA) and S <- gamma_C S, in
        // quarters of 32 columns (a short loop body: instruction fetch, not latency, limits this
        // kernel when many clusters share a GPC).  No MMA in flight touches these columns.
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {
          float sv[32];
          ptx::tmem_ld32(my + COL_S + 32 * q4, sv);
          ptx::tc_wait_ld();
          uint32_t hv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) hv[i] = pack_h2(sv[2 * i], sv[2 * i + 1]);
          ptx::tmem_st16(my + COL_S16 + 16 * q4, hv);
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] *= gC;
          ptx::tmem_st32(my + COL_S + 32 * q4, sv);
        }
        ptx::tc_wait_st();
        ptx::tc_fence_before();
        ptx::named_bar(1, 128);  // every chain warp's S16 stores are complete
        {
          // [R^T | Y] = [U^T | 0] - S [W | -Gamma Q]^T, committed as R, once W16 and QT16 of chunk c
          // are written and Y has been read out (and zeroed) by the output warps for chunk c-1.
          bool fail = false;
          if (warp == 0) {
            if (leader) {
              lwait(fail, SB_W16R, (uint32_t)c & 1u);
              if (c >= 1) lwait(fail, SB_YE, (uint32_t)(c - 1) & 1u);
            }
            fail = __shfl_sync(0xffffffffu, fail, 0);
            ptx::tc_fence_after();
            if (!fail) {
              // Without y (mode 1) only the R half, N = 64; the transition block has U = 0, so its
              // first K step overwrites the accumulator.
              const uint32_t idf = want_y ? ID_N128_BMN_NEG : ID_N64_BMN_NEG;
#pragma unroll 1
              for (int k = 0; k < 8; ++k)
                ptx::mma_f16_ts_elect(tmem + COL_U, tmem + COL_S16 + 8 * k, at(D_MN16K, S_WQ + k * 2048), idf,
                                      (k > 0 || !virt) ? 1u : 0u);
              issued = true;
              ptx::mma_commit_elect(&sbar[SB_R]);
              if (leader) lwait(fail, SB_R, (uint32_t)c & 1u);
            }
          }
          if (!agree(fail, leader, 1)) break;
        }
        if (warp == 0) issued = false;
        ptx::tc_fence_after();
        {
          // R -> R16 and R diag(w) -> RW16 (fp16, tensor memory), in halves of 32 tokens.
#pragma unroll 1
          for (int h2 = 0; h2 < 2; ++h2) {
            const float* w_s = gs + C + 32 * h2;
            float rv[32];
            ptx::tmem_ld32(my + COL_U + 32 * h2, rv);
            ptx::tc_wait_ld();
            uint32_t hv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) hv[i] = pack_h2(rv[2 * i], rv[2 * i + 1]);
            ptx::tmem_st16(my + COL_R16 + 16 * h2, hv);
#pragma unroll
            for (int i = 0; i < 16; ++i) hv[i] = pack_h2(rv[2 * i] * w_s[2 * i], rv[2 * i + 1] * w_s[2 * i + 1]);
            ptx::tmem_st16(my + COL_RW16 + 16 * h2, hv);
          }
          ptx::tc_wait_st();
        }
        ptx::tc_fence_before();
        ptx::named_bar(1, 128);
        if (warp == 0) {  // S += (R diag w)^T K (or U; committed alone), then Y += R^T A^T
          ptx::tc_fence_after();
          // The write side of the state: K tiles 16 KB apart, or the U tiles 8 KB apart.
          const uint64_t bw = HAS_U ? at(D_MN8K, kq_o + 4 * TILE) : at(D_MN16K, kq_o);
#pragma unroll 1
          for (int k = 0; k < 4; ++k)
            ptx::mma_f16_ts_elect(tmem + COL_S, tmem + COL_RW16 + 8 * k, bw + (uint64_t)(k * 2048 >> 4), ID_N128_BMN, 1);
          ptx::mma_commit_elect(&sbar[SB_S]);
          if (want_y) {
#pragma unroll 1
            for (int k = 0; k < 4; ++k)
              ptx::mma_f16_ts_elect(tmem + COL_Y, tmem + COL_R16 + 8 * k, at(D_K, ps_o + k * 32), ID_N64, 1);
          }
          ptx::mma_commit_elect(&sbar[SB_YF]);
          issued = true;
        }
      }
      // The last Y MMA may still run after this wait: `issued` stays set for the abort drain.
      if (!*abort_flag && nch > 0 && gwait(SB_S, (uint32_t)(nch - 1) & 1u, leader, 1, false)) {
        ptx::tc_fence_after();
        float* dst = nullptr;
        if (!want_y)  // mode 1: N_s (a real tile) or M_s (the transition block) of this segment
          dst = p.seg_out + ((int64_t)(bh * p.ws_stride + seg) * (p.DV + D) + (virt ? p.DV : dv0) + row) * D;
        else if (seg == p.nseg - 1 && p.s_out != nullptr)
          dst = p.s_out + ((int64_t)bh * p.DV + dv0 + row) * D;
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
      if (*abort_flag && warp == 0 && issued) {  // drain this warp's MMAs
        ptx::mma_commit_elect(&sbar[SB_DRAIN]);
        if (leader) ptx::mbar_wait_bounded(&sbar[SB_DRAIN], 0, WAIT_LIMIT);
        __syncwarp();
      }
    } else if (warp < 8) {
      // ------------------------- convert: gates, fp16 tiles, W ----------------------------
      const int wt = tid - 128, ww = wt >> 5;
      const bool leader = wt == 0;
      bool issued = false;
      float la0 = 0.f, la1 = 0.f, be0 = 0.f, be1 = 0.f;
      if (ww == 1 && nch > 0) load_gates(0, la0, la1, be0, be1);
      if (leader && !virt)
        for (int c = 0; c < NBV && c < nch; ++c) issue_v_loads(c);
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int s = c & 1, tb = c % NBK;  // product slot; k/q tile buffer
        const uint32_t ph = (uint32_t)(c >> 1) & 1u, tph = (uint32_t)(c / NBK) & 1u;
        const uint32_t kq_o = S_KQ + tb * KQB, ps_o = S_PS + s * PS_BYTES;
        float* gs = gslots + tb * GSLOT;
        float g0 = 0.f, g1 = 0.f, gC = 0.f;
        if (ww == 1) cumsum_gates(la0, la1, g0, g1, gC);
        {
          bool fail = false;  // k, q and v tiles of chunk c
          if (leader) lwait(fail, SB_KQF + tb, tph);
          if (!agree(fail, leader, 2)) break;
        }
        if (ww == 1) {
          gs[lane] = __expf(g0);  // arguments are sums of log decays (<= 0)
          gs[lane + 32] = __expf(g1);
          gs[C + lane] = be0 * __expf(gC - g0);
          gs[C + lane + 32] = be1 * __expf(gC - g1);
          if (lane == 0) gs[2 * C] = __expf(gC);
          if (c + 1 < nch) load_gates(c + 1, la0, la1, be0, be1);
        }
        convert_pair(sm + kq_o, sm + kq_o + 2 * TILE, wt);  // K -> fp16 (the output warps take V)
        if (HAS_U) convert_pair(sm + kq_o + 4 * TILE, sm + kq_o + 5 * TILE, wt);  // and U
        ptx::named_bar(2, 128);                              // gate slot and fp16 K written
        if (leader) ptx::mbar_arrive(&sbar[SB_KQR + tb]);
        // W^T = K^T (T Gamma)^T once T Gamma has arrived (the W columns were read out by this group
        // for chunk c-1); W16 is rewritten only after the fused MMA of chunk c-1 has read it, which
        // also frees the v buffer of chunk c-1 (its U MMA came first) for chunk c+1.
        if (!gwait(SB_PF + s, ph, leader, 2, true)) break;
        if (ww == 0) {  // issued from the converged warp
          ptx::tc_fence_after();
#pragma unroll 1
          for (int k = 0; k < 4; ++k)
            ptx::mma_f16_ss_elect(tmem + COL_W, at(D_MN16K, kq_o + k * 2048), at(D_K, ps_o + 2 * TILE + k * 32),
                                  ID_N64_AMN, k > 0);
          ptx::mma_commit_elect(&sbar[SB_WM]);
          issued = true;
        }
        {
          bool fail = false;  // the fused MMA of chunk c-1 (reader of W16 and of v buffer c+1) and W
          if (leader) {
            if (c > 0) {
              lwait(fail, SB_R, (uint32_t)(c - 1) & 1u);
              if (!fail && c + 1 < nch && !virt) issue_v_loads(c + 1);
            }
            lwait(fail, SB_WM, (uint32_t)c & 1u);
          }
          if (!agree(fail, leader, 2)) break;
          if (ww == 0) issued = false;
        }
        ptx::tc_fence_after();
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {  // W16: row d, 64 tokens, in halves of 32
          float wv[32];
          ptx::tmem_ld32(my + COL_W + 32 * h2, wv);
          ptx::tc_wait_ld();
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            *reinterpret_cast<uint4*>(sm + S_WQ + sw128((uint32_t)row, (uint32_t)(4 * h2 + c4))) =
                make_uint4(pack_h2(wv[8 * c4], wv[8 * c4 + 1]), pack_h2(wv[8 * c4 + 2], wv[8 * c4 + 3]),
                           pack_h2(wv[8 * c4 + 4], wv[8 * c4 + 5]), pack_h2(wv[8 * c4 + 6], wv[8 * c4 + 7]));
        }
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        ptx::named_bar(2, 128);
        if (leader) ptx::mbar_arrive(&sbar[SB_W16R]);
      }
      if (*abort_flag && ww == 0 && issued) {
        ptx::mma_commit_elect(&sbar[SB_DRAIN + 1]);
        if (leader) ptx::mbar_wait_bounded(&sbar[SB_DRAIN + 1], 0, WAIT_LIMIT);
        __syncwarp();
      }
    } else {
      // ------------------------------ output: Y -> y ---------------------------------------
      // Iteration c: the k/q tile loads of chunk c + 2; V of chunk c + 1 to fp16; the QT16 half of
      // chunk c + 1's fused MMA; chunk c's y stored from tensor memory, then its Y zeroed for that
      // MMA.  Iteration -1 only prepares chunk 0.
      const bool leader = tid == 256;
      const int ow = (tid - 256) >> 5;
      const uint32_t peer_pe0 = SPLIT ? 0u : ptx::mapa_shared(ptx::smem_u32(&pbar[PB_PE]), 1u);
      constexpr int ROWS = (int)(YS_BYTES / (D * sizeof(TOut)));  // tokens per staging piece
      TOut* stage = reinterpret_cast<TOut*>(sm + S_YS);
      if (SPLIT && leader)
        for (int c = 0; c < 2 && c < nch; ++c) issue_products(c);
#pragma unroll 1
      for (int c = -1; c < nch; ++c) {
        const int cn = c + 1;
        if (leader && !SPLIT) {
          // Every MMA of chunk c-1 has completed (its Y was read out last iteration): its tile
          // buffer takes the loads of chunk c + NBK - 1.  Iteration -1 issues those of chunks
          // 0 .. NBK - 2.  One call site.
          for (int l = c < 0 ? 0 : c + NBK - 1; l <= c + NBK - 1 && l < nch; ++l) issue_loads(l);
        }
        if (leader && SPLIT && c < 0) {  // state-only: every buffer at once, then one per chunk done
          for (int l = 0; l < NBK && l < nch; ++l) issue_loads(l);
        }
        if (cn < nch && !virt) {  // V of chunk c + 1 -> fp16 (the convert warps take K and the gates)
          if (!gwait(SB_VF + cn % NBV, (uint32_t)(cn / NBV) & 1u, leader, 3, false)) break;
          const uint32_t v_o = S_V + (cn % NBV) * V_BYTES;
          convert_pair(sm + v_o, sm + v_o + TILE, tid - 256);
          ptx::named_bar(3, 128);
          if (leader) ptx::mbar_arrive(&sbar[SB_KQR + cn % NBK]);
        } else if (cn < nch && leader) {  // the transition block has no v tile
          ptx::mbar_arrive(&sbar[SB_KQR + cn % NBK]);
        }
        if (cn < nch) {
          // QT16 = (-Gamma Q)^T of chunk c + 1, DK rows x 64 tokens (the Y half of the fused MMA's B
          // operand; its A-negation restores the sign), from the bf16 q tiles as loaded: each 8x8
          // block is read by ldmatrix (a token per row), scaled, and written transposed by
          // stmatrix.  Warp ow covers features 32 ow .. 32 ow + 31.  Built as soon as the fused MMA
          // of chunk c, the last reader of QT16, has completed, before chunk c's Y is read out.
          bool fail = false;  // the fused MMA of chunk c; q tiles and gates of chunk c + 1
          if (leader) {
            if (c >= 0) lwait(fail, SB_R, (uint32_t)c & 1u);
            lwait(fail, SB_KQR + cn % NBK, (uint32_t)(cn / NBK) & 1u);
          }
          if (!agree(fail, leader, 3)) break;
          const float* gs = gslots + (cn % NBK) * GSLOT;
          float ng[8];  // -gamma of the 8 tokens this lane scales: 8 j + lane / 4
#pragma unroll
          for (int j = 0; j < 8; ++j) ng[j] = -gs[8 * j + (lane >> 2)];
          const uint32_t qs = sb + S_KQ + (cn % NBK) * KQB + TILE, qd = sb + S_WQ + 2 * TILE;
          const int m = lane >> 3, r8 = lane & 7;
#pragma unroll 1
          for (int fq = 0; fq < (want_y ? 4 : 0); ++fq) {  // mode 1 has no y: the fused MMA leaves out QT16
            const int fb = 4 * ow + fq;  // feature block
            const uint32_t src = qs + (uint32_t)(fb >> 3) * 2 * TILE;
            uint32_t x[2][4];
#pragma unroll
            for (int hb = 0; hb < 2; ++hb)  // token blocks 4 hb .. 4 hb + 3
              ptx::ldsm_x4(src + sw128((uint32_t)(8 * (4 * hb + m) + r8), (uint32_t)(fb & 7)), x[hb]);
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x[hb][i]));
                x[hb][i] = pack_h2(f.x * ng[4 * hb + i], f.y * ng[4 * hb + i]);
              }
              ptx::stsm_x4_t(qd + sw128((uint32_t)(8 * fb + r8), (uint32_t)(4 * hb + m)), x[hb]);
            }
          }
          ptx::fence_proxy_async_smem();
          ptx::named_bar(3, 128);
          if (leader) ptx::mbar_arrive(&sbar[SB_W16R]);
        }
        if (c >= 0) {
          if (!gwait(SB_YF, (uint32_t)c & 1u, leader, 3, false)) break;  // every MMA of chunk c
          // Chunk c's product slot goes back to the prep CTA at once (its copy of chunk c + 2 waits),
          // or, state-only, takes chunk c + 2's products from the workspace.
          if (leader) {
            if (SPLIT) {
              // Without a prep CTA to pull the tiles into L2 ahead, the loads go out as early as
              // possible: chunk c's buffer is free now, before its y is read out.
              if (c + NBK < nch) issue_loads(c + NBK);
              if (c + 2 < nch) issue_products(c + 2);
            } else {
              ptx::mbar_arrive_remote_relaxed(peer_pe0 + 8u * (uint32_t)(c & 1));
            }
          }
          ptx::tc_fence_after();
          // y of chunk c straight from tensor memory, 16 tokens at a time (a short loop body), through
          // the staging tile: one TMA store per piece.
#pragma unroll 1
          for (int piece = 0; piece < (want_y ? C / ROWS : 0); ++piece) {
            // The staging tile's previous store (the last chunk's, or the previous piece) must have
            // been read out first.
            if (leader) ptx::bulk_wait_read0();
            ptx::named_bar(3, 128);
#pragma unroll 1
            for (int g = 0; g < ROWS / 16; ++g) {
              float yv[16];
              ptx::tmem_ld16(my + COL_Y + piece * ROWS + 16 * g, yv);
              ptx::tc_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) store_as(stage + (16 * g + j) * D + row, yv[j]);
            }
            ptx::fence_proxy_async_smem();
            ptx::named_bar(3, 128);
            if (leader) {
              ptx::tma_store_4d(&tm_y, stage, dv0, h, (cb + c) * C + piece * ROWS, b);
              ptx::bulk_commit();
            }
          }
          // Y is accumulated afresh by the fused MMA of chunk c + 1: zero it, then hand it back.
          if (want_y) {
            float z[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) z[j] = 0.f;
            ptx::tmem_st32(my + COL_Y, z);
            ptx::tmem_st32(my + COL_Y + 32, z);
            ptx::tc_wait_st();
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&sbar[SB_YE]);
        }
      }
      if (leader) ptx::bulk_wait0();
    }
  } else {
    // ======================================== prep CTA ========================================
    if (warp < 8) {
      const int pp = warp >> 2;  // pipeline: chunks pp, pp + 2, ...
      const int pt = tid & 127, pw = pt >> 5;
      const bool leader = pt == 0;
      const uint32_t base = pp * P_STRIDE;
      uint8_t* kq = sm + base + P_KQ;
      float* eT = reinterpret_cast<float*>(sm + base + P_EXPT);  // [64]      exp(g_t - g_{16 floor(t/16)})
      float* eJ = eT + C;                                         // [4][64]   beta_j exp(g_{16b} - g_j), j < 16b
      float* Ed = eJ + 4 * C;                                     // [4][16][20] beta_{16b+c} exp(g_{16b+r} - g_{16b+c}), c <= r
      float* beta_s = reinterpret_cast<float*>(sm + base + P_GS);
      float* g_s = beta_s + C;
      float* gam_s = g_s + C;
      const uint32_t remote_slot = ptx::mapa_shared(sb + S_PS + pp * PS_BYTES, 0u);
      const uint32_t remote_copies = ptx::mapa_shared(sb + CTRL + 24 + 4 * pp, 0u);
      int copies = 0;
      const uint32_t remote_pf = ptx::mapa_shared(ptx::smem_u32(&sbar[SB_PF + pp]), 0u);
      auto gwait = [&](int bar, uint32_t parity, bool cluster_scope) -> bool {
        bool fail = false;
        if (leader) {
          fail = cluster_scope ? !ptx::mbar_wait_abortable_cluster(&pbar[bar], parity, WAIT_LIMIT, abort_flag)
                               : !ptx::mbar_wait_abortable(&pbar[bar], parity, WAIT_LIMIT, abort_flag);
          if (fail) raise_abort();
        }
        return !ptx::named_bar_or(1 + pp, 128, fail);
      };
      auto issue = [&](int c) {
        ptx::mbar_arrive_expect_tx(&pbar[PB_KQF + pp], KQ_BYTES);
        issue_kq(kq, &pbar[PB_KQF + pp], c);
        ptx::tma_prefetch_4d(&tm_v, 0, h, (cb + c) * C, b);  // the state CTA's v tile, into L2
        ptx::tma_prefetch_4d(&tm_v, 64, h, (cb + c) * C, b);
      };
      bool issued = false;
      int last_load = -1;  // index k of the last tile set requested
      float la0 = 0.f, la1 = 0.f, be0 = 0.f, be1 = 0.f;
      if (leader && pp < nch) { issue(pp); last_load = 0; }
      if (pw == 1 && pp < nch) load_gates(pp, la0, la1, be0, be1);
      int k = 0;
#pragma unroll 1
      for (int c = pp; c < nch; c += 2, ++k) {
        const uint32_t ph = (uint32_t)k & 1u;
        const uint32_t st_o = base + P_ST + (uint32_t)(k & 1) * PS_BYTES;
        uint8_t* st = sm + st_o;
        if (!gwait(PB_KQF + pp, ph, false)) break;
        if (pw == 0) {  // G = [K;Q] K^T from the bf16 tiles as loaded (issued from the converged warp)
          ptx::tc_fence_after();
#pragma unroll 1
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = at(D_K, base + P_KQ + (kk >> 2) * 2 * TILE + (kk & 3) * 32);
            ptx::mma_f16_ss_elect(tmem + 64 * pp, a, a, ID_G, kk > 0);
          }
          ptx::mma_commit_elect(&pbar[PB_G + pp]);
          issued = true;
        }
        if (pw == 1) {  // chunk-local cumulative log-decay
          float g0, g1, gC;
          cumsum_gates(la0, la1, g0, g1, gC);
          beta_s[lane] = be0;
          beta_s[lane + 32] = be1;
          g_s[lane] = g0;
          g_s[lane + 32] = g1;
          gam_s[lane] = expf(g0);
          gam_s[lane + 32] = expf(g1);
        }
        ptx::named_bar(1 + pp, 128);
        // Decay tables: 1,344 exponentials per chunk instead of one per (t, j) pair; every factor is
        // exp of a non-positive number, so none overflows whatever the decay.
#pragma unroll 1
        for (int e = pt; e < 5 * C; e += 128) {
          if (e < C) {
            eT[e] = __expf(g_s[e] - g_s[e & ~15]);
          } else {
            const int bb = (e - C) >> 6, j = (e - C) & 63;
            eJ[bb * C + j] = (bb > 0 && j < 16 * bb) ? beta_s[j] * __expf(g_s[16 * bb] - g_s[j]) : 0.f;
          }
        }
#pragma unroll 1
        for (int n = 0; n < 8; ++n) {
          const int e = pt + 128 * n;  // 1024 diagonal-block entries
          const int bb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
          Ed[(bb * 16 + r) * 20 + cc] = cc <= r ? beta_s[16 * bb + cc] * __expf(g_s[16 * bb + r] - g_s[16 * bb + cc]) : 0.f;
        }
        if (!gwait(PB_G + pp, ph, false)) break;  // also orders the tables
        if (pw == 0) issued = false;
        if (leader && c + 2 < nch) {  // the tile set is free once G has been formed: fetch chunk c + 2
          issue(c + 2);
          last_load = k + 1;
        }
        if (pw == 1 && c + 2 < nch) load_gates(c + 2, la0, la1, be0, be1);
        ptx::tc_fence_after();
        // Row pt of G: rows 0-63 give L (strictly lower), rows 64-127 give A (lower with diagonal),
        // one 16-column block at a time (a rolled loop: the prep's instruction working set matters
        // more than the three extra tensor-memory round trips).
        {
          const int t = pt & 63, tb = t >> 4;
          const bool is_l = pt < 64;
          const float et = eT[t];
#pragma unroll 1
          for (int jb = 0; jb < 4; ++jb) {
            float gv[16], e[16];
            ptx::tmem_ld16(my + 64 * pp + 16 * jb, gv);
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
              uint8_t* lrow = sm + base + P_L16 + t * LD16 + jb * 32;
              *reinterpret_cast<uint4*>(lrow) = h0;
              *reinterpret_cast<uint4*>(lrow + 16) = h1;
              if (jb == tb) {  // the diagonal block also in fp32, for the substitution
                float* drow = reinterpret_cast<float*>(sm + base + P_LDIAG) + (tb * 16 + (t & 15)) * LDG;
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
        ptx::named_bar(1 + pp, 128);
        if (pt < 64) {
          // D_b = (I + L_bb)^-1, one column per thread; right-looking fp32 forward substitution.
          const int bb = pt >> 4, j = pt & 15;
          const float* Lb = reinterpret_cast<const float*>(sm + base + P_LDIAG) + bb * 16 * LDG;
          float x[16], acc[16];
#pragma unroll
          for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll
          for (int m = 0; m < 16; ++m) {
            x[m] = (m == j) ? 1.f : (m > j ? -acc[m] : 0.f);
#pragma unroll
            for (int r = m + 1; r < 16; ++r) acc[r] = fmaf(Lb[r * LDG + m], x[m], acc[r]);
          }
          __half* l16 = reinterpret_cast<__half*>(sm + base + P_L16);
#pragma unroll
          for (int r = 0; r < 16; ++r) l16[(bb * 16 + r) * (LD16 / 2) + bb * 16 + j] = __float2half_rn(x[r]);
        }
        ptx::named_bar(1 + pp, 128);
        merge_column_any<false>(pw, sb + base + P_L16, sb + st_o + TILE, 0u, sb + st_o + 2 * TILE, gam_s, lane);
        ptx::fence_proxy_async_smem();  // the staged products, for the bulk copy
        // The slot this pipeline used two chunks ago must have been given back; the group wait
        // (or the barrier) also orders every thread's staging stores before the copy.
        if (k > 0) {
          if (!gwait(PB_PE + pp, (uint32_t)(k - 1) & 1u, true)) break;
        } else {
          ptx::named_bar(1 + pp, 128);
        }
        if (leader) {
          ptx::mbar_arrive_expect_tx_remote(remote_pf, PS_BYTES);
          ptx::bulk_copy_to_cluster(remote_slot, st, PS_BYTES, remote_pf);
          ptx::st_cluster_u32(remote_copies, (uint32_t)++copies);
        }
      }
      if (*abort_flag && pw == 0) {  // drain this pipeline's MMA and tile loads
        if (issued) {
          ptx::mma_commit_elect(&pbar[PB_DRAIN + pp]);
          if (leader) ptx::mbar_wait_bounded(&pbar[PB_DRAIN + pp], 0, WAIT_LIMIT);
        }
        if (leader && last_load >= 0) ptx::mbar_wait_bounded(&pbar[PB_KQF + pp], (uint32_t)last_load & 1u, WAIT_LIMIT);
        __syncwarp();
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (rank == 0 && tid == 0 && *abort_flag) {  // tile loads still in flight: the last one per buffer
    const int n = *loads_issued, nv = *v_loads_issued;
    for (int c = n - NBK < 0 ? 0 : n - NBK; c < n; ++c)
      ptx::mbar_wait_bounded(&sbar[SB_KQF + c % NBK], (uint32_t)(c / NBK) & 1u, WAIT_LIMIT);
    for (int c = nv - NBV < 0 ? 0 : nv - NBV; c < nv; ++c)
      ptx::mbar_wait_bounded(&sbar[SB_VF + c % NBV], (uint32_t)(c / NBV) & 1u, WAIT_LIMIT);
  }
  __syncwarp();
  if (SPLIT)
    __syncthreads();
  else
    ptx::cluster_sync();  // every remote store, arrive and copy of both CTAs has been issued
  if (rank == 0 && tid == 0 && *abort_flag) {  // product copies still in flight into this CTA
    for (int sl = 0; sl < 2; ++sl) {
      const int issued_n = *reinterpret_cast<volatile int*>(sm + CTRL + 24 + 4 * sl);
      for (int k = *reinterpret_cast<volatile int*>(sm + CTRL + 16 + 4 * sl); k < issued_n; ++k)
        ptx::mbar_wait_bounded(&sbar[SB_PF + sl], (uint32_t)k & 1u, WAIT_LIMIT);
    }
  }
  __syncwarp();
  if (SPLIT)
    __syncthreads();
  else
    ptx::cluster_sync();  // neither CTA leaves while the other may still read from or write into it
  ptx::tc_fence_after();
  if (tid == 0 && *abort_flag) atomicExch(&g_status, GDN_ERR_TIMEOUT);
  if (warp == 0) ptx::tmem_dealloc(tmem, tmem_cols);
}

// Parameters shared by both modes; the caller fills the segment and state-only fields.
inline Params base_params(const gdn_prefill_args* a) {
  Params p = {};
  p.beta = a->beta; p.la = a->la; p.s0 = a->s0; p.s_out = a->s_out;
  p.B = (int)a->B; p.T = (int)a->T; p.H = (int)a->H; p.DV = (int)a->DV;
  p.NCt = (int)((a->T + C - 1) / C);
  p.nseg = 1;
  p.seg_len = p.NCt;
  p.nv = (int)(a->DV / D);
  p.ntiles = p.nv;
  return p;
}

// SPLIT: one CTA per (b, h, segment, state tile), no cluster; otherwise two-CTA clusters.
template <bool SPLIT, bool HAS_U, typename TOut>
int launch(const gdn_prefill_args* a, const Params& p, cudaStream_t stream) {
  CUtensorMap mq, mk, mv, my, mu;
  if (!make_map(&mq, a->q, a->DK, a, a->sq) || !make_map(&mk, a->k, a->DK, a, a->sk) ||
      !make_map(&mv, a->v, a->DV, a, a->sv) || !make_store_map<TOut>(&my, a->y, a->DV, a, a->sy, YS_BYTES))
    return GDN_ERR_LAUNCH;
  if (HAS_U) {
    if (!make_map(&mu, a->u, a->DK, a, a->su)) return GDN_ERR_LAUNCH;
  } else {
    mu = mk;
  }
  auto kern = pair_kernel<SPLIT, HAS_U, TOut>;
  static std::atomic<unsigned long long> opted{0};  // per device (see opt_in_smem)
  if (!opt_in_smem(opted, {{(const void*)kern, (int)(DYN)}})) return GDN_ERR_LAUNCH;
  const int64_t grid = (SPLIT ? (int64_t)p.ntiles : 2) * a->B * a->H * (int64_t)p.nseg;
  if (grid <= 0 || grid > 0x7fffffff) return GDN_ERR_SHAPE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = DYN;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = SPLIT ? 0 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, my, mu, p) != cudaSuccess) return GDN_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

template <bool SPLIT, bool HAS_U>
int launch_dt(const gdn_prefill_args* a, const Params& p, cudaStream_t stream) {
  return a->out_dtype == GDN_DTYPE_BF16 ? launch<SPLIT, HAS_U, __nv_bfloat16>(a, p, stream)
                                        : launch<SPLIT, HAS_U, float>(a, p, stream);
}

// Clusters of this kernel that fit on the device at once (0 if the query fails).
int max_active_clusters() {
  static std::atomic<int> cached[64] = {};  // per device; any host thread may call
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int known = cached[dev].load(std::memory_order_relaxed);
  if (known > 0) return known;
  auto kern = pair_kernel<false, false, __nv_bfloat16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = DYN;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace pair
}  // namespace gdn

// DK = DV = 128, u = beta k; the rest as the single-CTA kernel, and y stored by TMA.
bool gdn_chunk_pair_supported(const gdn_prefill_args* a) {
  return a->DV == 128 && a->in_dtype == GDN_DTYPE_BF16 && gdn_chunk_ws_supported(a) && gdn_y_tma_ok(a);
}

int gdn_chunk_pair_max_clusters() { return gdn::pair::max_active_clusters(); }

int gdn_launch_chunk_pair(const gdn_prefill_args* a, int nseg, int seg_len, const float* seg_s0, int ws_stride,
                          cudaStream_t stream) {
  gdn::pair::Params p = gdn::pair::base_params(a);
  p.nseg = nseg;
  if (seg_len > 0) p.seg_len = seg_len;
  p.seg_s0 = seg_s0;
  p.ws_stride = ws_stride;
  return gdn::pair::launch_dt<false, false>(a, p, stream);
}

// The state-only chunk kernel: any DV multiple of 128, u = beta k or explicit write vectors, y
// stored by TMA.
bool gdn_chunk_split_supported(const gdn_prefill_args* a) { return gdn_chunk_supported(a) && gdn_y_tma_ok(a); }

int gdn_launch_chunk_split(const gdn_prefill_args* a, const void* prod, int mode, int nseg, int seg_len, float* ws,
                           int ws_stride, cudaStream_t stream) {
  if (prod == nullptr || (uintptr_t)prod % 16) return GDN_ERR_ALIGN;
  gdn::pair::Params p = gdn::pair::base_params(a);
  p.prod = static_cast<const uint8_t*>(prod);
  p.mode = mode;
  p.nseg = nseg;
  if (seg_len > 0) p.seg_len = seg_len;
  p.ws_stride = ws_stride;
  if (mode == 1) {
    p.seg_out = ws;
    p.ntiles = p.nv + 1;
  } else {
    p.seg_s0 = ws;
  }
  return a->u != nullptr ? gdn::pair::launch_dt<true, true>(a, p, stream)
                         : gdn::pair::launch_dt<true, false>(a, p, stream);
}

int gdn_chunk_pair_read_status(int* out, int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::pair::g_status, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (reset) {
    int z = 0;
    if (cudaMemcpyToSymbol(gdn::pair::g_status, &z, sizeof(int)) != cudaSuccess) return GDN_ERR_LAUNCH;
  }
  *out = v;
  return GDN_OK;
}
