// Tile helpers shared by the tcgen05 chunk kernels (sm_100a): 128-byte-swizzled fp16/bf16
// tiles, fragment addressing for ldmatrix/stmatrix, the block-column merge of the 64x64
// triangular inverse T = (I + L)^-1, and the TMA tensor maps over [B][T][H][F] tensors.
#pragma once

#include <cudaTypedefs.h>

#include "gdn_common.cuh"
#include "sm100_ptx.cuh"

namespace gdn {
namespace tiles {

constexpr int C = 64;            // tokens per chunk
constexpr int D = 128;           // key dimension and state rows per tile
constexpr uint32_t TILE = 8192;  // one 64 x 64 16-bit tile (64 rows of 128 bytes)
constexpr uint32_t LD16 = 144;   // bytes per row of the fp16 L matrix (72 halves, conflict-free ldmatrix)
constexpr uint32_t LDG = 20;     // floats per row of the fp32 diagonal blocks

__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 64 fp32 values -> one 128-byte row of a swizzled fp16 tile.
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
// the diagonal blocks of the fp16 L matrix at `l16` (LD16 bytes per row).  Writes block column J
// (including the zero blocks above the diagonal) of T and of T Gamma (fp16, for
// W^T = K^T (T Gamma)^T) into swizzled 64x64 tiles.  SPLIT: T as a bf16 pair T_hi + T_lo (to
// ~2^-16, the B operand of U^T = V^T T^T against the bf16 V tile as loaded); otherwise T in
// fp16 at `thi` (against an fp16 V tile) and `tlo` unused.
template <int J, bool SPLIT>
__device__ __forceinline__ void merge_column(uint32_t l16, uint32_t thi, uint32_t tlo, uint32_t tg16, const float* gam,
                                             int lane) {
  const int g = lane >> 2;
  const float g0 = gam[16 * J + g], g8 = gam[16 * J + g + 8];
  uint32_t X[4][4];
  ptx::ldsm_x4_t(frag_addr_plain(l16, LD16, 16 * J, 16 * J, lane), X[J]);
  // fp32 fragment (8 values in A-fragment order) -> T (and T_lo), T Gamma tiles, block (i, J).
  auto emit = [&](int i, const float (&f)[8]) {
    uint32_t hi[4], lo[4], gs[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float a = f[2 * r], b = f[2 * r + 1];
      if constexpr (SPLIT) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        const float2 hf = __bfloat1622float2(h);
        hi[r] = *reinterpret_cast<const uint32_t*>(&h);
        lo[r] = pack_bf2(a - hf.x, b - hf.y);
      } else {
        hi[r] = pack_h2(a, b);
      }
      const float sc = (r & 1) ? g8 : g0;
      gs[r] = pack_h2(a * sc, b * sc);
    }
    ptx::stsm_x4_t(frag_addr_sw(thi, 16 * i, 16 * J, lane), hi);
    if constexpr (SPLIT) ptx::stsm_x4_t(frag_addr_sw(tlo, 16 * i, 16 * J, lane), lo);
    ptx::stsm_x4_t(frag_addr_sw(tg16, 16 * i, 16 * J, lane), gs);
  };
  {
    float f[8];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float2 v = unpack_h2(X[J][r]);
      f[2 * r] = v.x;
      f[2 * r + 1] = v.y;
    }
    emit(J, f);
  }
  const uint32_t z[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < J; ++i) {
    ptx::stsm_x4_t(frag_addr_sw(thi, 16 * i, 16 * J, lane), z);
    if constexpr (SPLIT) ptx::stsm_x4_t(frag_addr_sw(tlo, 16 * i, 16 * J, lane), z);
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
    emit(i, Tt);
  }
}

template <bool SPLIT>
__device__ __forceinline__ void merge_column_of(int J, uint32_t l16, uint32_t thi, uint32_t tlo, uint32_t tg16,
                                                const float* gam, int lane) {
  switch (J) {
    case 0: merge_column<0, SPLIT>(l16, thi, tlo, tg16, gam, lane); break;
    case 1: merge_column<1, SPLIT>(l16, thi, tlo, tg16, gam, lane); break;
    case 2: merge_column<2, SPLIT>(l16, thi, tlo, tg16, gam, lane); break;
    default: merge_column<3, SPLIT>(l16, thi, tlo, tg16, gam, lane); break;
  }
}

// Block column J of T = (I + L)^-1 for a J known only at run time (warp-uniform): one code path for
// all four columns, so that the warps merging different columns share their instructions (a smaller
// instruction working set than four specialised copies).  Same arithmetic as merge_column<J>; the
// output is left to the caller: emit(i, f) receives block (i, J) of T as an fp32 fragment of T^T in
// A-fragment order (for stmatrix .trans), zero(i) is called for the blocks i < J above the diagonal.
template <typename Emit, typename Zero>
__device__ __forceinline__ void merge_column_core(int J, uint32_t l16, int lane, Emit&& emit, Zero&& zero) {
  uint32_t X[4][4];
  // Diagonal block D_J (held transposed in the fragments).
  uint32_t xd[4];
  ptx::ldsm_x4_t(frag_addr_plain(l16, LD16, 16 * J, 16 * J, lane), xd);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
#pragma unroll
    for (int r = 0; r < 4; ++r) X[kk][r] = kk == J ? xd[r] : 0u;  // static register indices throughout
  {
    float f[8];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float2 v = unpack_h2(xd[r]);
      f[2 * r] = v.x;
      f[2 * r + 1] = v.y;
    }
    emit(J, f);
  }
#pragma unroll 1
  for (int i = 0; i < J; ++i) zero(i);  // blocks above the diagonal
#pragma unroll
  for (int i = 1; i < 4; ++i) {
    if (i <= J) continue;
    float P[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      if (k < J || k >= i) continue;
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
    emit(i, Tt);
  }
}

// merge_column<J, SPLIT> for a run-time J, through merge_column_core: block column J of T (and T_lo)
// and of T Gamma into swizzled 64x64 tiles.
template <bool SPLIT>
__device__ __forceinline__ void merge_column_any(int J, uint32_t l16, uint32_t thi, uint32_t tlo, uint32_t tg16,
                                                 const float* gam, int lane) {
  const int g = lane >> 2;
  const float g0 = gam[16 * J + g], g8 = gam[16 * J + g + 8];
  auto emit = [&](int i, const float (&f)[8]) {
    uint32_t hi[4], lo[4], gs[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float a = f[2 * r], b = f[2 * r + 1];
      if constexpr (SPLIT) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        const float2 hf = __bfloat1622float2(h);
        hi[r] = *reinterpret_cast<const uint32_t*>(&h);
        lo[r] = pack_bf2(a - hf.x, b - hf.y);
      } else {
        hi[r] = pack_h2(a, b);
      }
      const float sc = (r & 1) ? g8 : g0;
      gs[r] = pack_h2(a * sc, b * sc);
    }
    ptx::stsm_x4_t(frag_addr_sw(thi, 16 * i, 16 * J, lane), hi);
    if constexpr (SPLIT) ptx::stsm_x4_t(frag_addr_sw(tlo, 16 * i, 16 * J, lane), lo);
    ptx::stsm_x4_t(frag_addr_sw(tg16, 16 * i, 16 * J, lane), gs);
  };
  auto zero = [&](int i) {
    const uint32_t z[4] = {0u, 0u, 0u, 0u};
    ptx::stsm_x4_t(frag_addr_sw(thi, 16 * i, 16 * J, lane), z);
    if constexpr (SPLIT) ptx::stsm_x4_t(frag_addr_sw(tlo, 16 * i, 16 * J, lane), z);
    ptx::stsm_x4_t(frag_addr_sw(tg16, 16 * i, 16 * J, lane), z);
  };
  merge_column_core(J, l16, lane, emit, zero);
}

// ---- host: tensor maps ---------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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
inline bool make_map(CUtensorMap* m, const void* base, int64_t F, const gdn_prefill_args* a, const gdn_strides& s) {
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

// y [B][T][H][DV] -> 4-D store map (f, h, t, b), box 128 features x 1 x (box_bytes / row bytes)
// tokens, no swizzle.
template <typename TOut>
bool make_store_map(CUtensorMap* m, void* base, int64_t F, const gdn_prefill_args* a, const gdn_strides& s,
                    uint32_t box_bytes = TILE) {
  auto fn = encode_fn();
  if (!fn) return false;
  constexpr int es = (int)sizeof(TOut);
  cuuint64_t dims[4] = {(cuuint64_t)F, (cuuint64_t)a->H, (cuuint64_t)a->T, (cuuint64_t)a->B};
  cuuint64_t strides[3] = {(cuuint64_t)s.h * es, (cuuint64_t)s.t * es, (cuuint64_t)s.b * es};
  cuuint32_t box[4] = {(cuuint32_t)D, 1, (cuuint32_t)(box_bytes / (D * es)), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tiles
}  // namespace gdn
