// Segment-parallel prefill for few, long sequences (sm_100a).
//
// A sequence with too few (b, h) units to fill the GPU is cut into P segments of L chunks; the
// per-chunk transition S -> gamma_C S + (U - W S^T)^T diag(w) K is affine in S, so a segment
// maps its entry state to S_out = S_in M_s + N_s.  Three passes, all on the stream:
//   A. gdn_chunk_ws_sm100.cu in state mode over segments 0..P-2: N_s from S = 0 with the real
//      v, M_s from S = I with v = 0 (one extra 128-row tile per (b, h, segment)); no y.
//   B. combine_kernel: S_{s+1} = S_s M_s + N_s, s = 0..P-2, fp32 on CUDA cores, the 128 state
//      rows split over CTAs (rows evolve independently), result written over N_s.
//   C. the chunk kernel in output mode over all P segments, segment s starting from S_s.
// Workspace (caller-allocated): B*H*(P-1) slots of (DV + 128) x 128 fp32.
// The reference computes the same recurrence sequentially (archbench/layers/nsgdn.py:408-417,
// fla's chunk_gated_delta_rule_fwd_h walks chunks in order); this split is this build's own.
#include "gdn_common.cuh"

namespace gdn {
namespace seg {

constexpr int D = 128;
constexpr int RB = 4;  // state rows per combine CTA

__global__ void __launch_bounds__(D) combine_kernel(float* __restrict__ ws, const float* __restrict__ s0, int DV,
                                                    int nslots, int rblocks) {
  const int bh = blockIdx.x / rblocks, r0 = (blockIdx.x % rblocks) * RB;
  const int j = threadIdx.x;
  __shared__ float srow[RB][D];
  float s[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) s[r] = s0 ? s0[((int64_t)bh * DV + r0 + r) * D + j] : 0.f;
#pragma unroll 1
  for (int t = 0; t < nslots; ++t) {
    float* mat = ws + (int64_t)(bh * nslots + t) * (DV + D) * D;
#pragma unroll
    for (int r = 0; r < RB; ++r) srow[r][j] = s[r];
    __syncthreads();
    float acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = mat[(int64_t)(r0 + r) * D + j];
    const float* M = mat + (int64_t)DV * D;
#pragma unroll 8
    for (int k = 0; k < D; ++k) {
      const float m = M[(int64_t)k * D + j];
#pragma unroll
      for (int r = 0; r < RB; ++r) acc[r] = fmaf(srow[r][k], m, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      s[r] = acc[r];
      mat[(int64_t)(r0 + r) * D + j] = acc[r];
    }
    __syncthreads();
  }
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

}  // namespace seg
}  // namespace gdn

// Segment plan for these arguments; false when the single-pass kernel is the better choice.
bool gdn_segmented_plan(const gdn_prefill_args* a, int sms, int* nseg, int* seg_len, size_t* bytes) {
  if (!gdn_chunk_supported(a) || a->u != nullptr) return false;
  const int64_t nch = (a->T + 63) / 64;
  const int64_t units = a->B * a->H * (a->DV / 128);
  if (sms <= 0 || units * 4 > sms || nch < 8) return false;
  int64_t P = sms / units;
  if (P > nch / 2) P = nch / 2;
  if (P < 2) return false;
  const int64_t L = (nch + P - 1) / P;
  P = (nch + L - 1) / L;
  if (P < 2) return false;
  *nseg = (int)P;
  *seg_len = (int)L;
  *bytes = (size_t)(a->B * a->H * (P - 1)) * (size_t)(a->DV + 128) * 128 * sizeof(float);
  return true;
}

int gdn_segmented_sms() { return gdn::seg::sm_count(); }

int gdn_launch_segmented(const gdn_prefill_args* a, float* ws, size_t ws_bytes, int sms, cudaStream_t stream) {
  int P = 0, L = 0;
  size_t need = 0;
  if (!gdn_segmented_plan(a, sms, &P, &L, &need)) return GDN_ERR_UNSUPPORTED;
  if (ws == nullptr || ws_bytes < need) return GDN_ERR_SHAPE;
  if ((uintptr_t)ws % 16) return GDN_ERR_ALIGN;
  int st = gdn_launch_chunk_ws_segments(a, 1, P - 1, L, ws, P - 1, stream);
  if (st != GDN_OK) return st;
  const int rblocks = (int)(a->DV / gdn::seg::RB);
  const int64_t grid = a->B * a->H * rblocks;
  gdn::seg::combine_kernel<<<(unsigned)grid, gdn::seg::D, 0, stream>>>(ws, a->s0, (int)a->DV, P - 1, rblocks);
  if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  return gdn_launch_chunk_ws_segments(a, 0, P, L, ws, P - 1, stream);
}
