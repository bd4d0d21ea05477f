// int4 -> 16-bit dequantization and bulk-copy helpers shared by the W4A16 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cb_ptx.cuh"

namespace cb {

template <typename T>
struct Dq;
template <>
struct Dq<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  // 0x4300 = 128.0; nibble (offset by 8) lands in the low mantissa bits.
  static constexpr uint32_t kOrXor = 0x43084308u;
  static __device__ __forceinline__ T2 bias() { return __floats2bfloat162_rn(136.0f, 136.0f); }
  static __device__ __forceinline__ T2 from_f(float f) { return __float2bfloat162_rn(f); }
};
template <>
struct Dq<__half> {
  using T2 = __half2;
  // 0x6400 = 1024.0 in f16; ulp 1 in [1024, 2048).
  static constexpr uint32_t kOrXor = 0x64086408u;
  static __device__ __forceinline__ T2 bias() { return __floats2half2_rn(1032.0f, 1032.0f); }
  static __device__ __forceinline__ T2 from_f(float f) { return __float2half2_rn(f); }
};

template <typename T>
__device__ __forceinline__ uint32_t dq_pair(uint32_t word, int shift, typename Dq<T>::T2 bias,
                                            typename Dq<T>::T2 sc, bool apply_scale) {
  using T2 = typename Dq<T>::T2;
  uint32_t bits = ((word >> shift) & 0x000F000Fu) ^ Dq<T>::kOrXor;
  T2 v = *reinterpret_cast<T2*>(&bits);
  v = __hsub2(v, bias);
  if (apply_scale) v = __hmul2(v, sc);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}


// Stores one dequantized weight row (128 k values as 64 packed pairs r[0..63],
// pair i holding k = 2i, 2i+1) into a K-major tile of 128 rows x 128 k stored
// as two 128-byte-swizzled sub-tiles of 128 rows x 64 k: 16-byte chunk q of the
// row (k = 8q..8q+7) lands in sub-tile q / 8 at chunk position (q % 8) ^ (row % 8).
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int row, const uint32_t (&r)[64]) {
  uint8_t* base = tile + row * 128;
  const int rx = row & 7;
#pragma unroll
  for (int q = 0; q < 16; ++q)
    *reinterpret_cast<uint4*>(base + (q >> 3) * (128 * 128) + (((q & 7) ^ rx) << 4)) =
        make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
}

// Dequantizes row `row` of a native 8 KiB int4 tile (rows of 64 bytes, 16-byte
// chunk j stored at j ^ ((row >> 1) & 3)) into 64 packed 16-bit pairs, scaled
// by `sc` when apply_scale.
template <typename T>
__device__ __forceinline__ void dequant_native_row(const uint8_t* tile, int row, typename Dq<T>::T2 sc,
                                                   bool apply_scale, uint32_t (&r)[64]) {
  const uint4* wrow = reinterpret_cast<const uint4*>(tile + row * 64);
  const int swz = (row >> 1) & 3;
  const typename Dq<T>::T2 bias = Dq<T>::bias();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 v = wrow[c ^ swz];
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
      for (int pi = 0; pi < 4; ++pi) r[c * 16 + wi * 4 + pi] = dq_pair<T>(words[wi], 4 * pi, bias, sc, apply_scale);
  }
}

}  // namespace cb
