// Fused RMSNorm -> dynamic per-token INT8 quantization (one launch).
//
// The reference measures the act-quant tax of W8A8 decode and its removal by
// fusing the quantization into the preceding norm (+2.2 us fused vs 8.4 us
// separate on H100, profiling/mechanisms/RESULTS.md:17,
// profiling/dense_qwen/results_fused_normquant_h100.json). This kernel computes,
// per row of x [rows, H]:
//   r   = 1 / sqrt(sum_k x_k^2 / H + eps)           (fp32 sum, IEEE sqrt and divide)
//   y_k = cvt(x_k * r * w_k)                          (rounded to x's 16-bit dtype, as an
//                                                      RMSNorm layer would output it)
//   scale = max(amax_k |y_k| / 127, 1e-8),  q_k = trunc(y_k / scale + 0.5*sign(y_k))
// i.e. the RMSNorm output quantized by the rules of _quant_act_kernel
// (profiling/w8a8/w8a8_bmm.py:35-39), and optionally writes y. One CTA per row;
// the row is read from global memory three times (the second and third reads
// hit L1/L2). Launched with programmatic dependent launch like act_quant.cu, so
// a following W8A8 GEMM streams its weights while this runs.
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
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (kThreads / 32) ? red[lane] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, u) : v + u;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ int8_t quant1(float y, float scale) {
  return static_cast<int8_t>(__float2int_rz(__fadd_rn(__fdiv_rn(y, scale), y >= 0.0f ? 0.5f : -0.5f)));
}

// y_k for element k of the row (identical arithmetic in every pass)
template <typename T, typename W>
__device__ __forceinline__ T norm1(T x, W w, float r) {
  return from_f32<T>(__fmul_rn(__fmul_rn(to_f32(x), r), to_f32(w)));
}

template <typename T, typename W>
__global__ void __launch_bounds__(kThreads) rmsnorm_quant_kernel(const T* __restrict__ x, long long x_sm,
                                                                 const W* __restrict__ w, float eps, int H,
                                                                 int8_t* __restrict__ q, long long q_sm,
                                                                 float* __restrict__ scale, T* __restrict__ y,
                                                                 long long y_sm) {
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ float red[kThreads / 32];
  const long long row = blockIdx.x;
  const T* xr = x + row * x_sm;

  float ss = 0.0f;
  for (int k = threadIdx.x; k < H; k += kThreads) {
    const float v = to_f32(xr[k]);
    ss = __fmaf_rn(v, v, ss);
  }
  ss = block_reduce(ss, red, false);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps)));

  float amax = 0.0f;
  for (int k = threadIdx.x; k < H; k += kThreads) amax = fmaxf(amax, fabsf(to_f32(norm1(xr[k], w[k], r))));
  amax = block_reduce(amax, red, true);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);

  int8_t* qr = q + row * q_sm;
  T* yr = y ? y + row * y_sm : nullptr;
  for (int k = threadIdx.x; k < H; k += kThreads) {
    const T yk = norm1(xr[k], w[k], r);
    qr[k] = quant1(to_f32(yk), s);
    if (yr) yr[k] = yk;
  }
  if (threadIdx.x == 0) scale[row] = s;
}

template <typename T, typename W>
int launch_typed(const void* x, long long x_sm, const void* w, float eps, long long rows, int H, int8_t* q,
                 long long q_sm, float* scale, void* y, long long y_sm, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel<T, W>, static_cast<const T*>(x), x_sm,
                                        static_cast<const W*>(w), eps, H, q, q_sm, scale, static_cast<T*>(y), y_sm));
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" CB_API int cb_rmsnorm_quant_i8(const void* x, int x_dtype, const void* weight, int w_dtype, float eps,
                                          int64_t rows, int64_t H, int64_t x_sm, int8_t* q, int64_t q_sm,
                                          float* scale, void* y_out, int64_t y_sm, cb_stream_t stream) {
  if (rows < 0 || H < 0) return CB_ERR_INVALID_ARG;
  if (rows == 0 || H == 0) return CB_OK;
  if (!x || !weight || !q || !scale) return CB_ERR_INVALID_ARG;
  if (x_dtype != CB_DTYPE_BF16 && x_dtype != CB_DTYPE_F16) return CB_ERR_DTYPE;
  if (w_dtype != CB_DTYPE_BF16 && w_dtype != CB_DTYPE_F16 && w_dtype != CB_DTYPE_F32) return CB_ERR_DTYPE;
  if (rows > 0x7fffffffLL || H > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  if (x_sm < H || q_sm < H || (y_out && y_sm < H)) return CB_ERR_STRIDE;
  if (!(eps >= 0.0f)) return CB_ERR_INVALID_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int h = static_cast<int>(H);
  if (x_dtype == CB_DTYPE_BF16) {
    if (w_dtype == CB_DTYPE_BF16)
      return launch_typed<__nv_bfloat16, __nv_bfloat16>(x, x_sm, weight, eps, rows, h, q, q_sm, scale, y_out, y_sm, s);
    if (w_dtype == CB_DTYPE_F16)
      return launch_typed<__nv_bfloat16, __half>(x, x_sm, weight, eps, rows, h, q, q_sm, scale, y_out, y_sm, s);
    return launch_typed<__nv_bfloat16, float>(x, x_sm, weight, eps, rows, h, q, q_sm, scale, y_out, y_sm, s);
  }
  if (w_dtype == CB_DTYPE_BF16)
    return launch_typed<__half, __nv_bfloat16>(x, x_sm, weight, eps, rows, h, q, q_sm, scale, y_out, y_sm, s);
  if (w_dtype == CB_DTYPE_F16)
    return launch_typed<__half, __half>(x, x_sm, weight, eps, rows, h, q, q_sm, scale, y_out, y_sm, s);
  return launch_typed<__half, float>(x, x_sm, weight, eps, rows, h, q, q_sm, scale, y_out, y_sm, s);
}
