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
#include <cuda_fp8.h>

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

// Long rows held in registers: one CTA of kRegThreads threads per row loads the
// whole row at once (NV 16-byte vectors per thread, all in flight together),
// reduces the amax and quantizes from the same registers, so a row costs one
// memory round trip instead of a loop of dependent loads and a second pass
// over the row. Same arithmetic as act_quant_kernel (the maximum does not
// depend on the order of the elements).
constexpr int kRegThreads = 512;

template <typename T, int NV>
__global__ void __launch_bounds__(kRegThreads) act_quant_reg_kernel(const T* __restrict__ a, long long a_sb,
                                                                     long long a_sm, int8_t* __restrict__ q,
                                                                     long long q_sb, long long q_sm,
                                                                     float* __restrict__ scale, long long s_sb, int M,
                                                                     int K) {
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ float red[kRegThreads / 32];
  const int row = blockIdx.x;
  const int b = row / M, m = row % M;
  const uint4* av = reinterpret_cast<const uint4*>(a + b * a_sb + m * a_sm);
  uint2* qv = reinterpret_cast<uint2*>(q + b * q_sb + m * q_sm);
  const int nvec = K / 8;
  uint4 u[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int idx = threadIdx.x + i * kRegThreads;
    if (idx < nvec) u[i] = av[idx];
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (threadIdx.x + i * kRegThreads < nvec) {
      const T* e = reinterpret_cast<const T*>(&u[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(to_f32(e[j])));
    }
  }
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  if (warp == 0) {
    float v = lane < kRegThreads / 32 ? red[lane] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float s = fmaxf(__fdiv_rn(red[0], 127.0f), 1e-8f);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int idx = threadIdx.x + i * kRegThreads;
    if (idx < nvec) {
      const T* e = reinterpret_cast<const T*>(&u[i]);
      uint2 o;
      int8_t* ob = reinterpret_cast<int8_t*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) ob[j] = quant1(to_f32(e[j]), s);
      qv[idx] = o;
    }
  }
  if (threadIdx.x == 0) scale[b * s_sb + m] = s;
}

// Short rows (K <= kWarpRowMaxK), many of them (a batch of heads x tokens): one
// warp per row, kThreads / 32 rows per CTA, the same arithmetic as
// act_quant_kernel. A CTA per row would spend its time launching.
constexpr int kWarpRowMaxK = 2048;

template <typename T>
__global__ void __launch_bounds__(kThreads) act_quant_rows_kernel(const T* __restrict__ a, long long a_sb,
                                                                   long long a_sm, int8_t* __restrict__ q,
                                                                   long long q_sb, long long q_sm,
                                                                   float* __restrict__ scale, long long s_sb, int M,
                                                                   int K, long long rows) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const long long b = row / M, m = row % M;
  const T* ar = a + b * a_sb + m * a_sm;
  int8_t* qr = q + b * q_sb + m * q_sm;
  float amax = 0.0f;
  for (int i = lane; i < K; i += 32) amax = fmaxf(amax, fabsf(to_f32(ar[i])));
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
  for (int i = lane; i < K; i += 32) qr[i] = quant1(to_f32(ar[i]), s);
  if (lane == 0) scale[b * s_sb + m] = s;
}

// ---------------------------------------------------------------------------
// e4m3 fp8 activations (the operands of the fp8 W8A8 GEMM), in the three modes
// of vLLM's scaled_fp8_quant, the call the reference's dense harnesses make
// (profiling/dense_qwen/bench_l2_boundary.py:54-57):
//   scale = max(amax / 448, 1 / (448 * 512))   (dynamic; IEEE-rounded division)
//   q     = e4m3(clamp(a / scale, -448, 448))   (round to nearest even)
// One CTA per row. For one scale per batch entry (per-tensor dynamic) a single
// CTA per batch entry first reduces the entry's amax.
// ---------------------------------------------------------------------------
constexpr float kFp8Max = 448.0f;

__device__ __forceinline__ float fp8_scale_of(float amax) {
  return fmaxf(__fdiv_rn(amax, kFp8Max), 1.0f / (kFp8Max * 512.0f));
}

__device__ __forceinline__ uint8_t fp8_of(float x, float scale) {
  const float y = fminf(fmaxf(__fdiv_rn(x, scale), -kFp8Max), kFp8Max);
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3));
}

template <typename T>
__device__ __forceinline__ float row_amax(const T* ar, int K, int vec_ok) {
  float amax = 0.0f;
  if (vec_ok) {
    const uint4* av = reinterpret_cast<const uint4*>(ar);
    for (int i = threadIdx.x; i < K / 8; i += kThreads) {
      uint4 u = av[i];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(to_f32(e[j])));
    }
  } else {
    for (int i = threadIdx.x; i < K; i += kThreads) amax = fmaxf(amax, fabsf(to_f32(ar[i])));
  }
  return amax;
}

// mode 0: per-row scale; 1: scale given per batch entry (per-tensor, computed by
// fp8_amax_kernel or passed in).
template <typename T>
__global__ void __launch_bounds__(kThreads) act_quant_fp8_kernel(const T* __restrict__ a, long long a_sb,
                                                                  long long a_sm, uint8_t* __restrict__ q,
                                                                  long long q_sb, long long q_sm,
                                                                  float* __restrict__ scale, long long s_sb, int M,
                                                                  int K, int vec_ok, int given_scale) {
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ float red[kThreads / 32];
  const int row = blockIdx.x;
  const int b = row / M, m = row % M;
  const T* ar = a + b * a_sb + m * a_sm;
  uint8_t* qr = q + b * q_sb + m * q_sm;
  float s;
  if (given_scale) {
    s = scale[b * s_sb];
  } else {
    s = fp8_scale_of(block_max(row_amax(ar, K, vec_ok), red));
  }
  if (vec_ok) {
    const uint4* av = reinterpret_cast<const uint4*>(ar);
    uint2* qv = reinterpret_cast<uint2*>(qr);
    for (int i = threadIdx.x; i < K / 8; i += kThreads) {
      uint4 u = av[i];
      const T* e = reinterpret_cast<const T*>(&u);
      uint2 o;
      uint8_t* ob = reinterpret_cast<uint8_t*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) ob[j] = fp8_of(to_f32(e[j]), s);
      qv[i] = o;
    }
  } else {
    for (int i = threadIdx.x; i < K; i += kThreads) qr[i] = fp8_of(to_f32(ar[i]), s);
  }
  if (!given_scale && threadIdx.x == 0) scale[b * s_sb + m] = s;
}

// One CTA per batch entry: the entry's amax over all M rows -> scale[b * s_sb].
template <typename T>
__global__ void __launch_bounds__(kThreads) fp8_amax_kernel(const T* __restrict__ a, long long a_sb, long long a_sm,
                                                             float* __restrict__ scale, long long s_sb, int M, int K,
                                                             int vec_ok) {
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ float red[kThreads / 32];
  const int b = blockIdx.x;
  float amax = 0.0f;
  for (int m = 0; m < M; ++m) amax = fmaxf(amax, row_amax(a + b * a_sb + m * a_sm, K, vec_ok));
  amax = block_max(amax, red);
  if (threadIdx.x == 0) scale[b * s_sb] = fp8_scale_of(amax);
}

}  // namespace

int launch_act_quant_fp8(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_sb, int64_t a_sm,
                         uint8_t* q, int64_t q_sb, int64_t q_sm, float* scale, int64_t s_sb, int mode,
                         cudaStream_t stream) {
  const long long rows = batch * M;
  if (rows == 0 || K == 0) return CB_OK;
  if (rows > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  if (mode != CB_FP8_PER_TOKEN && mode != CB_FP8_PER_TENSOR_DYNAMIC && mode != CB_FP8_STATIC) return CB_ERR_INVALID_ARG;
  const int vec_ok = (K % 8 == 0) && aligned16(a) && ((a_sb * 2) % 16 == 0) && ((a_sm * 2) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(q) % 8 == 0) && (q_sb % 8 == 0) && (q_sm % 8 == 0);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int Mi = static_cast<int>(M), Ki = static_cast<int>(K);
  const long long asb = a_sb, asm_ = a_sm, qsb = q_sb, qsm = q_sm, ssb = s_sb;
  cudaError_t e = cudaSuccess;
  if (a_dtype != CB_DTYPE_BF16 && a_dtype != CB_DTYPE_F16) return CB_ERR_DTYPE;
  if (mode == CB_FP8_PER_TENSOR_DYNAMIC) {
    cfg.gridDim = dim3(static_cast<unsigned>(batch));
    if (a_dtype == CB_DTYPE_BF16)
      e = cudaLaunchKernelEx(&cfg, fp8_amax_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(a), asb, asm_,
                             scale, ssb, Mi, Ki, vec_ok);
    else
      e = cudaLaunchKernelEx(&cfg, fp8_amax_kernel<__half>, static_cast<const __half*>(a), asb, asm_, scale, ssb, Mi,
                             Ki, vec_ok);
    if (e != cudaSuccess) return CB_ERR_CUDA;
  }
  const int given = mode == CB_FP8_PER_TOKEN ? 0 : 1;
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  if (a_dtype == CB_DTYPE_BF16)
    e = cudaLaunchKernelEx(&cfg, act_quant_fp8_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(a), asb, asm_,
                           q, qsb, qsm, scale, ssb, Mi, Ki, vec_ok, given);
  else
    e = cudaLaunchKernelEx(&cfg, act_quant_fp8_kernel<__half>, static_cast<const __half*>(a), asb, asm_, q, qsb, qsm,
                           scale, ssb, Mi, Ki, vec_ok, given);
  return cuda_status(e);
}

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
  if (K <= kWarpRowMaxK && rows >= 64) {
    cfg.gridDim = dim3(static_cast<unsigned>((rows + kThreads / 32 - 1) / (kThreads / 32)));
    if (a_dtype == CB_DTYPE_BF16)
      e = cudaLaunchKernelEx(&cfg, act_quant_rows_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(a),
                             static_cast<long long>(a_sb), static_cast<long long>(a_sm), q,
                             static_cast<long long>(q_sb), static_cast<long long>(q_sm), scale,
                             static_cast<long long>(s_sb), Mi, Ki, rows);
    else if (a_dtype == CB_DTYPE_F16)
      e = cudaLaunchKernelEx(&cfg, act_quant_rows_kernel<__half>, static_cast<const __half*>(a),
                             static_cast<long long>(a_sb), static_cast<long long>(a_sm), q,
                             static_cast<long long>(q_sb), static_cast<long long>(q_sm), scale,
                             static_cast<long long>(s_sb), Mi, Ki, rows);
    else
      return CB_ERR_DTYPE;
    return cuda_status(e);
  }
  if (vec_ok && K / 8 <= 8 * kRegThreads) {
    // whole row in registers: NV vectors per thread, the smallest of 2, 4, 8 that holds it
    cfg.blockDim = dim3(kRegThreads);
    const int nvec = static_cast<int>(K / 8);
    const bool bf = a_dtype == CB_DTYPE_BF16;
    if (!bf && a_dtype != CB_DTYPE_F16) return CB_ERR_DTYPE;
#define CB_ACTQ_REG(NV)                                                                                            \
  (bf ? cudaLaunchKernelEx(&cfg, act_quant_reg_kernel<__nv_bfloat16, NV>, static_cast<const __nv_bfloat16*>(a),    \
                           static_cast<long long>(a_sb), static_cast<long long>(a_sm), q, static_cast<long long>(q_sb), \
                           static_cast<long long>(q_sm), scale, static_cast<long long>(s_sb), Mi, Ki)                  \
      : cudaLaunchKernelEx(&cfg, act_quant_reg_kernel<__half, NV>, static_cast<const __half*>(a),                  \
                           static_cast<long long>(a_sb), static_cast<long long>(a_sm), q, static_cast<long long>(q_sb), \
                           static_cast<long long>(q_sm), scale, static_cast<long long>(s_sb), Mi, Ki))
    if (nvec <= 2 * kRegThreads)
      e = CB_ACTQ_REG(2);
    else if (nvec <= 4 * kRegThreads)
      e = CB_ACTQ_REG(4);
    else
      e = CB_ACTQ_REG(8);
#undef CB_ACTQ_REG
    return cuda_status(e);
  }
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
