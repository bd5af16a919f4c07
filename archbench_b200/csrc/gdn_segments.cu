// Segment-parallel prefill for few, long sequences (sm_100a).
//
// A sequence with too few (b, h) units to fill the GPU is cut into P segments of L chunks; the
// per-chunk transition S -> gamma_C S + (U - W S^T)^T diag(w) K is affine in S, so a segment
// maps its entry state to S_out = S_in M_s + N_s.  Three passes, all on the stream:
//   A. a chunk kernel in state mode over segments 0..P-2: N_s from S = 0 with the real v, M_s from
//      S = I with v = 0 (one extra 128-row tile per (b, h, segment)); no y.
//   B. combine_kernel: S_{s+1} = S_s M_s + N_s, s = 0..P-2, fp32 on CUDA cores, the state rows
//      split over CTAs (rows evolve independently), the contraction over four threads per column,
//      M_s double-buffered in shared memory, result written over N_s.
//   C. the chunk kernel in output mode over all P segments, segment s starting from S_s.
// The chunk kernel is the state-only one of gdn_chunk_pair_sm100.cu after one prep pass over every
// chunk (gdn_chunk_prep_sm100.cu), whose products both passes read; where y cannot be stored by TMA,
// and for the entry point without allocation, the single-CTA kernel of gdn_chunk_ws_sm100.cu, which
// prepares the products in every tile itself.
// Workspace (caller-allocated): B*H*(P-1) slots of (DV + 128) x 128 fp32, then (split kernels) the
// chunk products, 24 KB per (b, h, chunk).
// The reference computes the same recurrence sequentially (archbench/layers/nsgdn.py:408-417,
// fla's chunk_gated_delta_rule_fwd_h walks chunks in order); this split is this build's own.
#include <mutex>

#include "gdn_common.cuh"

namespace gdn {
namespace seg {

constexpr int D = 128;
constexpr int RB = 4;                                 // state rows per combine CTA
constexpr int KS = 4;                                 // threads per state column (contraction quarters)
constexpr int NMB = 2;                                // transition matrices in flight per combine CTA
constexpr uint32_t COMB_SMEM = NMB * D * D * 4u;     // NMB transition matrices M_s (64 KB each)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// S_{s+1} = S_s M_s + N_s for s = 0..nslots-1, RB state rows per CTA (rows evolve independently).
// Thread (j, ks) of the KS x D threads takes state column j and the ks-th quarter of the
// contraction; the quarters meet in shared memory in a fixed order.  M_s is staged in shared memory
// by cp.async, the copies of the next NMB - 1 steps in flight while the current step computes: the
// chain of steps is bound by the step's own latency instead of by L2 latency.
__global__ void __launch_bounds__(KS * D) combine_kernel(float* __restrict__ ws, const float* __restrict__ s0, int DV,
                                                         int nslots, int rblocks) {
  extern __shared__ __align__(16) float msm[];  // [NMB][D][D]
  __shared__ float srow[RB][D];
  __shared__ float part[KS][RB][D];
  const int bh = blockIdx.x / rblocks, r0 = (blockIdx.x % rblocks) * RB;
  const int j = threadIdx.x % D, ks = threadIdx.x / D;
  constexpr int KQ = D / KS;  // contraction indices per thread
  float s[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) s[r] = (ks == 0 && s0) ? s0[((int64_t)bh * DV + r0 + r) * D + j] : 0.f;
  auto slot = [&](int t) { return ws + (int64_t)(bh * nslots + t) * (DV + D) * D; };
  auto prefetch = [&](int t) {
    const float* M = slot(t) + (int64_t)DV * D;
    float* dst = msm + (t % NMB) * D * D;
#pragma unroll 2
    for (int i = threadIdx.x; i < D * D / 4; i += KS * D) cp_async16(dst + 4 * i, M + 4 * i);
    cp_async_commit();
  };
  for (int t = 0; t < NMB - 1 && t < nslots; ++t) prefetch(t);
  // N_t's rows (written over by S_{t+1} at the end of step t) are loaded a step ahead, into registers.
  float accn[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) accn[r] = (ks == 0 && nslots > 0) ? slot(0)[(int64_t)(r0 + r) * D + j] : 0.f;
#pragma unroll 1
  for (int t = 0; t < nslots; ++t) {
    float* mat = slot(t);
    float acc[RB];
    if (ks == 0) {
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        srow[r][j] = s[r];
        acc[r] = accn[r];
      }
      if (t + 1 < nslots) {
        const float* nxt = slot(t + 1);
#pragma unroll
        for (int r = 0; r < RB; ++r) accn[r] = nxt[(int64_t)(r0 + r) * D + j];
      }
    }
    // The copy of step t + NMB - 1 goes into the buffer step t - 1 read (barriers below); then every
    // copy but the newest NMB - 2 has landed, step t's among them.
    if (t + NMB - 1 < nslots) {
      prefetch(t + NMB - 1);
      cp_async_wait<NMB - 1>();
    } else if (t + 1 < nslots) {
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // srow written; M_t copied by every thread
    const float* M = msm + (t % NMB) * D * D + ks * KQ * D;
    float pr[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) pr[r] = 0.f;
#pragma unroll 8
    for (int k = 0; k < KQ; ++k) {
      const float m = M[k * D + j];
#pragma unroll
      for (int r = 0; r < RB; ++r) pr[r] = fmaf(srow[r][ks * KQ + k], m, pr[r]);
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) part[ks][r][j] = pr[r];
    __syncthreads();  // every quarter written; M_t and srow read
    if (ks == 0) {
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        float v = acc[r];
#pragma unroll
        for (int q = 0; q < KS; ++q) v += part[q][r][j];
        s[r] = v;
        mat[(int64_t)(r0 + r) * D + j] = v;
      }
    }
  }
}

int sm_count() {
  static std::atomic<int> cached[64] = {};  // per device; any host thread may call
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) {
    const int known = cached[dev].load(std::memory_order_relaxed);
    if (known > 0) return known;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace seg
}  // namespace gdn

// Segment plan for these arguments; false when the single-pass kernel is the better choice.
// `max_bytes` (0 = no limit) caps the workspace by using fewer, longer segments.
static bool plan(const gdn_prefill_args* a, int sms, size_t max_bytes, int* nseg, int* seg_len, size_t* bytes) {
  if (!gdn_chunk_supported(a)) return false;
  const int64_t nch = (a->T + 63) / 64;
  const int64_t units = a->B * a->H * (a->DV / 128);
  if (sms <= 0 || units * 4 > sms || nch < 8) return false;
  int64_t P = sms / units;
  if (P > nch / 2) P = nch / 2;
  const size_t slot = (size_t)(a->B * a->H) * (size_t)(a->DV + 128) * 128 * sizeof(float);
  if (max_bytes > 0 && P > 1 && (size_t)(P - 1) * slot > max_bytes) P = (int64_t)(max_bytes / slot) + 1;
  if (P < 2) return false;
  const int64_t L = (nch + P - 1) / P;
  P = (nch + L - 1) / L;
  if (P < 2) return false;
  *nseg = (int)P;
  *seg_len = (int)L;
  *bytes = (size_t)(P - 1) * slot;
  return true;
}

// The split chunk kernels (prep pass, then the state-only kernel for both passes) where they apply:
// the workspace then holds the segment slots, then every chunk's products.
static size_t slots_rounded(size_t slot_bytes) { return (slot_bytes + 255) / 256 * 256; }

bool gdn_segmented_plan(const gdn_prefill_args* a, int sms, int* nseg, int* seg_len, size_t* bytes) {
  if (!plan(a, sms, 0, nseg, seg_len, bytes)) return false;
  if (gdn_chunk_split_supported(a)) *bytes = slots_rounded(*bytes) + gdn_chunk_prep_bytes(a);
  return true;
}

int gdn_segmented_sms() { return gdn::seg::sm_count(); }

static int launch_combine(const gdn_prefill_args* a, float* ws, int P, cudaStream_t stream) {
  const int rblocks = (int)(a->DV / gdn::seg::RB);
  const int64_t grid = a->B * a->H * rblocks;
  static std::atomic<unsigned long long> opted{0};  // per device (see gdn::opt_in_smem)
  if (!gdn::opt_in_smem(opted, {{(const void*)gdn::seg::combine_kernel, (int)gdn::seg::COMB_SMEM}}))
    return GDN_ERR_LAUNCH;
  gdn::seg::combine_kernel<<<(unsigned)grid, gdn::seg::KS * gdn::seg::D, gdn::seg::COMB_SMEM, stream>>>(ws, a->s0, (int)a->DV, P - 1,
                                                                                          rblocks);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

// The three passes on the single-CTA kernel (each state tile prepares its own chunk products).
static int launch_plan(const gdn_prefill_args* a, float* ws, size_t ws_bytes, int P, int L, size_t need,
                       cudaStream_t stream) {
  if (ws == nullptr || ws_bytes < need) return GDN_ERR_SHAPE;
  if ((uintptr_t)ws % 16) return GDN_ERR_ALIGN;
  int st = gdn_launch_chunk_ws_segments(a, 1, P - 1, L, ws, P - 1, stream);
  if (st != GDN_OK) return st;
  st = launch_combine(a, ws, P, stream);
  if (st != GDN_OK) return st;
  return gdn_launch_chunk_ws_segments(a, 0, P, L, ws, P - 1, stream);
}

// The same passes on the split kernels: every chunk's products once, then the state-only kernel
// in state mode (segments 0..P-2), the combine, and the state-only kernel in output mode.
static int launch_plan_split(const gdn_prefill_args* a, float* ws, size_t ws_bytes, int P, int L, size_t slot_bytes,
                             cudaStream_t stream) {
  const size_t off = slots_rounded(slot_bytes);
  if (ws == nullptr || ws_bytes < off + gdn_chunk_prep_bytes(a)) return GDN_ERR_SHAPE;
  if ((uintptr_t)ws % 16) return GDN_ERR_ALIGN;
  void* prod = reinterpret_cast<uint8_t*>(ws) + off;
  int st = gdn_launch_chunk_prep(a, prod, stream);
  if (st != GDN_OK) return st;
  st = gdn_launch_chunk_split(a, prod, 1, P - 1, L, ws, P - 1, stream);
  if (st != GDN_OK) return st;
  st = launch_combine(a, ws, P, stream);
  if (st != GDN_OK) return st;
  return gdn_launch_chunk_split(a, prod, 0, P, L, ws, P - 1, stream);
}

int gdn_launch_segmented(const gdn_prefill_args* a, float* ws, size_t ws_bytes, int sms, cudaStream_t stream) {
  int P = 0, L = 0;
  size_t need = 0;
  if (!plan(a, sms, 0, &P, &L, &need)) return GDN_ERR_UNSUPPORTED;
  if (gdn_chunk_split_supported(a)) return launch_plan_split(a, ws, ws_bytes, P, L, need, stream);
  return launch_plan(a, ws, ws_bytes, P, L, need, stream);
}

// ---- the same prefill without any allocation --------------------------------------------------
// Callers that cannot allocate device memory when they call us -- a plugin whose host framework
// owns all device memory and hands over only input and output pointers, or a serving loop that
// forbids cudaMalloc after start-up because it synchronises the device and breaks a pre-planned
// memory pool -- get the segment workspace from this fixed array instead.  It is reserved on every
// GPU that loads the library and held until the process exits.  In host code `g_static_ws` only
// names the symbol; its device address comes from cudaGetSymbolAddress, looked up once per device
// with that device current, on the first call there.
static __device__ __align__(256) float g_static_ws[GDN_STATIC_WORKSPACE_BYTES / sizeof(float)];

namespace {
std::mutex g_static_ws_mu;
float* g_static_ws_ptr[64] = {};
}  // namespace

static float* static_ws_address(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = GDN_ERR_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_static_ws_mu);
  if (g_static_ws_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_ws);
    if (e != cudaSuccess || ptr == nullptr) {
      *status = GDN_ERR_LAUNCH;
      return nullptr;
    }
    g_static_ws_ptr[dev] = static_cast<float*>(ptr);
  }
  return g_static_ws_ptr[dev];
}

// Segmented prefill with the workspace in g_static_ws: the plan uses fewer, longer segments when
// the usual one would need more than GDN_STATIC_WORKSPACE_BYTES.  Nothing in the workspace has
// to start at zero (phase A writes every slot before phase B reads it).
int gdn_launch_segmented_static(const gdn_prefill_args* a, int sms, cudaStream_t stream) {
  int P = 0, L = 0;
  size_t need = 0;
  if (!plan(a, sms, 0, &P, &L, &need)) return GDN_ERR_UNSUPPORTED;
  if (need > GDN_STATIC_WORKSPACE_BYTES &&
      (!plan(a, sms, GDN_STATIC_WORKSPACE_BYTES, &P, &L, &need) || need > GDN_STATIC_WORKSPACE_BYTES))
    return GDN_ERR_WORKSPACE;
  int st = GDN_OK;
  float* ws = static_ws_address(&st);
  if (ws == nullptr) return st;
  return launch_plan(a, ws, GDN_STATIC_WORKSPACE_BYTES, P, L, need, stream);
}
