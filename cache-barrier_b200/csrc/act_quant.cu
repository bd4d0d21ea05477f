// Dynamic per-(batch, token) symmetric INT8 activation quantization.
//
// Restates the arithmetic of _quant_act_kernel (profiling/w8a8/w8a8_bmm.py:30-41):
//   amax  = max_k |a|                          (fp32)
//   scale = max(amax / 127, 1e-8)              (fp32, IEEE-rounded division)
//   q     = int8(trunc(a / scale + 0.5*sign))  (sign(0) = +1; half away from zero)
// One CTA per row; the row is read twice (amax pass, quantize pass), the second
// time from L1/L2. The kernel releases its dependents (the W8A8 GEMM launched
// with programmatic serialization) as soon as it starts, so the GEMM's weight
// stream overlaps this kernel; the GEMM reads q and scale only after its
// griddepcontrol.wait.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cb_internal.h"
#include "cb_ptx.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ int8_t quant1(float x, float scale) {
  const float y = __fadd_rn(__fdiv_rn(x, scale), x >= 0.0f ? 0.5f : -0.5f);
  return static_cast<int8_t>(__float2int_rz(y));
}

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (kThreads / 32) ? red[lane] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

template <typename T>
__global__ void __launch_bounds__(kThreads) act_quant_kernel(const T* __restrict__ a, long long a_sb,
                                                              long long a_sm, int8_t* __restrict__ q,
                                                              long long q_sb, long long q_sm,
                                                              float* __restrict__ scale, long long s_sb, int M,
                                                              int K, int vec_ok) {
  // Release the dependent GEMM at once (it prefetches weights only), then wait
  // for the preceding kernel before reading a or overwriting q and scale.
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ float red[kThreads / 32];
  const int row = blockIdx.x;
  const int b = row / M, m = row % M;
  const T* ar = a + b * a_sb + m * a_sm;
  int8_t* qr = q + b * q_sb + m * q_sm;

  float amax = 0.0f;
  if (vec_ok) {
    const int nvec = K / 8;
    const uint4* av = reinterpret_cast<const uint4*>(ar);
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      uint4 u = av[i];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(to_f32(e[j])));
    }
  } else {
    for (int i = threadIdx.x; i < K; i += kThreads) amax = fmaxf(amax, fabsf(to_f32(ar[i])));
  }
  amax = block_max(amax, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);

  if (vec_ok) {
    const int nvec = K / 8;
    const uint4* av = reinterpret_cast<const uint4*>(ar);
    uint2* qv = reinterpret_cast<uint2*>(qr);
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      uint4 u = av[i];
      const T* e = reinterpret_cast<const T*>(&u);
      uint2 o;
      int8_t* ob = reinterpret_cast<int8_t*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) ob[j] = quant1(to_f32(e[j]), s);
      qv[i] = o;
    }
  } else {
    for (int i = threadIdx.x; i < K; i += kThreads) qr[i] = quant1(to_f32(ar[i]), s);
  }
  if (threadIdx.x == 0) scale[b * s_sb + m] = s;
}

}  // namespace

int launch_act_quant(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_sb, int64_t a_sm,
                     int8_t* q, int64_t q_sb, int64_t q_sm, float* scale, int64_t s_sb, cudaStream_t stream) {
  const long long rows = batch * M;
  if (rows == 0 || K == 0) return CB_OK;
  if (rows > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  const size_t esz = 2;
  const int vec_ok = (K % 8 == 0) && aligned16(a) && ((a_sb * esz) % 16 == 0) && ((a_sm * esz) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(q) % 8 == 0) && (q_sb % 8 == 0) && (q_sm % 8 == 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int Mi = static_cast<int>(M), Ki = static_cast<int>(K);
  cudaError_t e;
  if (a_dtype == CB_DTYPE_BF16) {
    e = cudaLaunchKernelEx(&cfg, act_quant_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(a),
                           static_cast<long long>(a_sb), static_cast<long long>(a_sm), q, static_cast<long long>(q_sb),
                           static_cast<long long>(q_sm), scale, static_cast<long long>(s_sb), Mi, Ki, vec_ok);
  } else if (a_dtype == CB_DTYPE_F16) {
    e = cudaLaunchKernelEx(&cfg, act_quant_kernel<__half>, static_cast<const __half*>(a), static_cast<long long>(a_sb),
                           static_cast<long long>(a_sm), q, static_cast<long long>(q_sb), static_cast<long long>(q_sm),
                           scale, static_cast<long long>(s_sb), Mi, Ki, vec_ok);
  } else {
    return CB_ERR_DTYPE;
  }
  return cuda_status(e);
}

}  // namespace cb
