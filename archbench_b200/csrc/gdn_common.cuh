// Shared helpers of the gated-DeltaNet kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <initializer_list>

#include "gdn_b200.h"

namespace gdn {

// Element loads/stores for the two I/O dtypes.
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ void store_as(float* p, float x) { *p = x; }
__device__ __forceinline__ void store_as(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }

// Load N consecutive elements (N * sizeof(T) bytes, naturally aligned) as floats.
template <int N, typename T>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  if constexpr (sizeof(T) * N == 16) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f32(e[i]);
  } else if constexpr (sizeof(T) * N == 8) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f32(e[i]);
  } else if constexpr (sizeof(T) * N == 4) {
    uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f32(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f32(p[i]);
  }
}

template <typename T>
struct DtypeOf;
template <>
struct DtypeOf<float> {
  static constexpr int value = GDN_DTYPE_F32;
};
template <>
struct DtypeOf<__nv_bfloat16> {
  static constexpr int value = GDN_DTYPE_BF16;
};

// Opt kernels into more than 48 KB of dynamic shared memory on the current device.  A function
// attribute belongs to the function as loaded in one device's context, so it is set once per
// device: bit `dev` of `done` records that the current device's context has it.  Setting it twice
// from two host threads is harmless (the call is idempotent); `done` is atomic, so any thread may
// call.  Devices past 63 set the attribute on every call.
struct SmemOptIn {
  const void* kernel;
  int bytes;
};

inline bool opt_in_smem(std::atomic<unsigned long long>& done, std::initializer_list<SmemOptIn> kernels) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const unsigned long long bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return true;
  for (const SmemOptIn& k : kernels)
    if (cudaFuncSetAttribute(k.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, k.bytes) != cudaSuccess) return false;
  if (bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

}  // namespace gdn

// Host-side entry points of the individual kernels (defined in their .cu files).  They
// assume validated arguments and return a gdn_status.
int gdn_launch_recurrent(const gdn_prefill_args* a, const float* s_in, float* s_out,
                         cudaStream_t stream);
int gdn_launch_chunk_sm100(const gdn_prefill_args* a, cudaStream_t stream);
bool gdn_chunk_supported(const gdn_prefill_args* a);
int gdn_chunk_read_status(int* out, int reset);
bool gdn_chunk_ws_supported(const gdn_prefill_args* a);
bool gdn_y_tma_ok(const gdn_prefill_args* a);
int gdn_launch_chunk_ws(const gdn_prefill_args* a, cudaStream_t stream);
int gdn_chunk_ws_read_status(int* out, int reset);
int gdn_launch_selftest_wait(long long max_cycles, cudaStream_t stream);
int gdn_launch_chunk_ws_segments(const gdn_prefill_args* a, int mode, int nseg, int seg_len, float* ws, int ws_stride,
                                 cudaStream_t stream);
bool gdn_segmented_plan(const gdn_prefill_args* a, int sms, int* nseg, int* seg_len, size_t* bytes);
int gdn_segmented_sms();
int gdn_launch_segmented(const gdn_prefill_args* a, float* ws, size_t ws_bytes, int sms, cudaStream_t stream);
int gdn_launch_segmented_static(const gdn_prefill_args* a, int sms, cudaStream_t stream);
bool gdn_chunk_pair_supported(const gdn_prefill_args* a);
int gdn_chunk_pair_max_clusters();
int gdn_launch_chunk_pair(const gdn_prefill_args* a, int nseg, int seg_len, const float* seg_s0, int ws_stride,
                          cudaStream_t stream);
int gdn_chunk_pair_read_status(int* out, int reset);
// Split chunk path: the prep kernel writes every chunk's products (A, T, T Gamma; 24 KB per chunk) to
// `prod`, then the state-only chunk kernel streams them back.  mode 0 writes y (segment s >= 1 starts
// from slot s - 1 of `ws`); mode 1 writes [N_s; M_s] of each segment to slot s of `ws`.
size_t gdn_chunk_prep_bytes(const gdn_prefill_args* a);
int gdn_launch_chunk_prep(const gdn_prefill_args* a, void* prod, cudaStream_t stream);
int gdn_chunk_prep_read_status(int* out, int reset);
bool gdn_chunk_split_supported(const gdn_prefill_args* a);
int gdn_launch_chunk_split(const gdn_prefill_args* a, const void* prod, int mode, int nseg, int seg_len, float* ws,
                           int ws_stride, cudaStream_t stream);
