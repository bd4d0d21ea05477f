// extern "C" entry points declared in include/cb200.h: argument validation,
// tensor-map construction, workspace accounting and kernel dispatch.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "cb200.h"
#include "cb_internal.h"

namespace cb {

namespace {
std::atomic<unsigned long long> g_debug_wait_ns{0};
std::atomic<bool> g_force_last_arriver{false};
}  // namespace

unsigned long long debug_wait_ns() { return g_debug_wait_ns.load(std::memory_order_relaxed); }
bool debug_force_last_arriver() { return g_force_last_arriver.load(std::memory_order_relaxed); }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (dev < 0 || dev >= 64) return 0;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}
}  // namespace

int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_elems, uint64_t stride2_elems, uint32_t box0, uint32_t box1,
                   CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return CB_ERR_CUDA;
  uint64_t esz = 1;
  if (dtype == CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 || dtype == CU_TENSOR_MAP_DATA_TYPE_FLOAT16) esz = 2;
  if (dtype == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 || dtype == CU_TENSOR_MAP_DATA_TYPE_INT32) esz = 4;
  uint64_t s1 = stride1_elems * esz;
  uint64_t s2 = stride2_elems * esz;
  if (d2 <= 1) s2 = s1 * (d1 > 0 ? d1 : 1);  // unused dimension: any legal stride
  if (s1 % 16 != 0 || s2 % 16 != 0 || !aligned16(base)) return CB_ERR_ALIGNMENT;
  cuuint64_t dims[3] = {d0, d1, d2 > 0 ? d2 : 1};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CB_OK : CB_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Weight repack / unpack kernels (offline preparation and the W4A4 operands)
// ---------------------------------------------------------------------------
namespace {

// Signed nibble q[b, k, n] of a reference-layout source.
__device__ __forceinline__ int ref_nibble(const uint8_t* src, int layout, long long b, long long k, long long n,
                                          long long K, long long N) {
  if (layout == CB_W4_REF_U8_KN) {
    const uint8_t byte = src[(b * (K / 2) + k / 2) * N + n];
    int v = (k & 1) ? (byte >> 4) : (byte & 0xF);
    return v;
  } else {
    const uint32_t w = reinterpret_cast<const uint32_t*>(src)[(b * (K / 8) + k / 8) * N + n];
    return static_cast<int>((w >> (4 * (k & 7))) & 0xF);
  }
}

// Nibble position of k (0..7) inside a native 32-bit word: order k0,k2,k4,k6,k1,k3,k5,k7.
__host__ __device__ __forceinline__ int native_nibble_pos(int k8) { return (k8 & 1) ? 4 + (k8 >> 1) : (k8 >> 1); }

// One thread per native 32-bit word: (b, nt, kt, r, word w in 0..15).
__global__ void repack_w4_kernel(const uint8_t* __restrict__ src, int layout, uint32_t* __restrict__ dst,
                                 long long batch, long long K, long long N, long long n_tiles, long long k_tiles) {
  const long long total = batch * n_tiles * k_tiles * 128 * 16;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int wpos = static_cast<int>(i & 15);  // stored word position within the 64-byte row
    const int r = static_cast<int>((i >> 4) & 127);
    long long t = i >> 11;
    const long long kt = t % k_tiles;
    t /= k_tiles;
    const long long nt = t % n_tiles;
    const long long b = t / n_tiles;
    // stored chunk position c' holds logical chunk c = c' ^ ((r >> 1) & 3)
    const int chunk = (wpos >> 2) ^ ((r >> 1) & 3);
    const int word_in_chunk = wpos & 3;
    const long long n = nt * 128 + r;
    const long long k0 = kt * 128 + chunk * 32 + word_in_chunk * 8;
    uint32_t out = 0;
    if (n < N) {
      for (int j = 0; j < 8; ++j) {
        const long long k = k0 + j;
        if (k < K) {
          const uint32_t v = static_cast<uint32_t>(ref_nibble(src, layout, b, k, n, K, N)) & 0xFu;
          out |= v << (4 * native_nibble_pos(j));
        }
      }
    }
    dst[i] = out;
  }
}

__global__ void transpose_i8_kernel(const int8_t* __restrict__ src, int8_t* __restrict__ dst, long long K,
                                    long long N) {
  __shared__ int8_t tile[32][33];
  const long long b = blockIdx.z;
  const long long k0 = static_cast<long long>(blockIdx.y) * 32, n0 = static_cast<long long>(blockIdx.x) * 32;
  const int8_t* s = src + b * K * N;
  int8_t* d = dst + b * K * N;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const long long k = k0 + i, n = n0 + threadIdx.x;
    if (k < K && n < N) tile[i][threadIdx.x] = s[k * N + n];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const long long n = n0 + i, k = k0 + threadIdx.x;
    if (k < K && n < N) d[n * K + k] = tile[threadIdx.x][i];
  }
}

// Value of a nibble: sign-extended (mode 0) or, in the reference-wrap mode, the
// result of `v - 16` on a uint8 lane for v >= 8 (240..255), stored as uint8.
__device__ __forceinline__ uint8_t nibble_value(int v, int wrap) {
  return static_cast<uint8_t>(v >= 8 ? (wrap ? v + 240 : v - 16) : v);
}

// Unpack packed int4 rows (byte i holds k = 2i low nibble, 2i+1 high) to 8-bit [rows, K].
__global__ void unpack_rows_i4_kernel(const uint8_t* __restrict__ src, long long ld, uint8_t* __restrict__ dst,
                                      long long rows, long long K, int wrap) {
  const long long half = K / 2;
  const long long total = rows * half;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / half, c = i % half;
    const uint8_t byte = src[r * ld + c];
    dst[r * K + 2 * c] = nibble_value(byte & 0xF, wrap);
    dst[r * K + 2 * c + 1] = nibble_value(byte >> 4, wrap);
  }
}

// Unpack B [K/2, N] (k-packed along rows) to 8-bit K-major [N, K] through
// shared memory, one CTA per 64 (packed k-pairs) x 64 (n) tile (1-D grid, n
// tiles fastest): source rows are read as 64 contiguous bytes per row and each
// destination row is written as 128 contiguous bytes, 32 per thread in two
// 16-byte stores, so both sides are coalesced. Requires K % 32 == 0 (checked by
// the caller) and a 16-byte aligned dst.
constexpr int kUnpackTile = 64;
__global__ void __launch_bounds__(256) unpack_cols_i4_tiled_kernel(const uint8_t* __restrict__ src, long long ld,
                                                                   uint8_t* __restrict__ dst, long long K, long long N,
                                                                   int wrap) {
  __shared__ __align__(16) uint8_t tile[kUnpackTile][kUnpackTile + 16];  // [k-pair][n], rows 16-byte aligned
  const long long half = K / 2;
  const long long n_tiles = (N + kUnpackTile - 1) / kUnpackTile;
  const long long c0 = (blockIdx.x / n_tiles) * kUnpackTile;
  const long long n0 = (blockIdx.x % n_tiles) * kUnpackTile;
  {
    const int r = threadIdx.x >> 2, q = threadIdx.x & 3;  // row r, bytes 16q..16q+15 of the tile row
    const long long c = c0 + r;
    const long long nb = n0 + q * 16;
    const uint8_t* sp = src + c * ld + nb;
    if (c < half && nb + 16 <= N && (reinterpret_cast<uintptr_t>(sp) & 15u) == 0) {
      *reinterpret_cast<uint4*>(&tile[r][q * 16]) = *reinterpret_cast<const uint4*>(sp);
    } else {
#pragma unroll
      for (int b = 0; b < 16; ++b) tile[r][q * 16 + b] = (c < half && nb + b < N) ? sp[b] : 0;
    }
  }
  __syncthreads();
  const int nn = threadIdx.x >> 2, q = threadIdx.x & 3;  // destination row n0 + nn, k-pairs 16q..16q+15
  const long long n = n0 + nn;
  const long long cq = c0 + q * 16;
  if (n < N && cq < half) {  // half % 16 == 0: the thread's 16 k-pairs are all in range
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint8_t b0 = tile[q * 16 + 2 * i][nn], b1 = tile[q * 16 + 2 * i + 1][nn];
      w[i] = static_cast<uint32_t>(nibble_value(b0 & 0xF, wrap)) | (static_cast<uint32_t>(nibble_value(b0 >> 4, wrap)) << 8) |
             (static_cast<uint32_t>(nibble_value(b1 & 0xF, wrap)) << 16) |
             (static_cast<uint32_t>(nibble_value(b1 >> 4, wrap)) << 24);
    }
    uint4* d = reinterpret_cast<uint4*>(dst + n * K + 2 * cq);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

int grid_for(long long total, int threads) {
  long long g = (total + threads - 1) / threads;
  int sms = sm_count();
  long long cap = sms > 0 ? static_cast<long long>(sms) * 16 : 2048;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

bool valid_out_dtype(int d) { return d == CB_DTYPE_F16 || d == CB_DTYPE_BF16 || d == CB_DTYPE_F32; }

}  // namespace

int validate_w8a8(const int8_t* aq, const int8_t* w, void* out, int out_dtype, int64_t batch, int64_t M,
                  int64_t N, int64_t K, const int64_t* st) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (!st) return CB_ERR_INVALID_ARG;
  if (batch * M * N == 0) return CB_OK;
  if (!aq || !w || !out) return CB_ERR_INVALID_ARG;
  if (!valid_out_dtype(out_dtype)) return CB_ERR_DTYPE;
  if (K == 0 || K % 16 != 0) return CB_ERR_SHAPE;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL || batch > 0xffffLL) return CB_ERR_TOO_LARGE;
  if (!aligned16(aq) || !aligned16(w)) return CB_ERR_ALIGNMENT;
  if (st[1] % 16 != 0 || st[3] % 16 != 0 || (batch > 1 && (st[0] % 16 != 0 || st[2] % 16 != 0)))
    return CB_ERR_ALIGNMENT;
  if (st[1] < K || st[3] < K) return CB_ERR_STRIDE;
  return CB_OK;
}

int read_and_clear_status(void* scratch, int* device_status, cudaStream_t s) {
  int host = 0;
  if (cudaMemcpyAsync(&host, scratch, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return CB_ERR_CUDA;
  if (device_status) *device_status = host;
  if (host != 0) {
    // A kernel that gave up a wait may have left arrival counters behind: clear
    // them with the status word so the next call starts from zero.
    if (cudaMemsetAsync(scratch, 0, kWsHeader + kWsCounters, s) != cudaSuccess) return CB_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return CB_ERR_CUDA;
    return CB_ERR_DEVICE_TIMEOUT;
  }
  return CB_OK;
}

}  // namespace cb

using namespace cb;

extern "C" {

const char* cb_status_str(int status) {
  switch (status) {
    case CB_OK:
      return "ok";
    case CB_ERR_INVALID_ARG:
      return "invalid argument";
    case CB_ERR_SHAPE:
      return "unsupported shape";
    case CB_ERR_DTYPE:
      return "unsupported dtype";
    case CB_ERR_ALIGNMENT:
      return "pointer or stride not 16-byte aligned";
    case CB_ERR_STRIDE:
      return "innermost dimension not contiguous";
    case CB_ERR_WORKSPACE:
      return "workspace missing or too small";
    case CB_ERR_CUDA:
      return "CUDA runtime error";
    case CB_ERR_DEVICE_TIMEOUT:
      return "device-side wait timed out";
    case CB_ERR_UNSUPPORTED:
      return "unsupported device or layout";
    case CB_ERR_TOO_LARGE:
      return "size beyond the supported maximum";
    default:
      return "unknown status";
  }
}

int cb_version(void) { return 100; }

int cb_device_sm_count(void) { return sm_count(); }

size_t cb_workspace_bytes(int op, int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return 0;
  switch (op) {
    case CB_OP_W8A8:
      return w8a8_workspace_bytes(batch, M, N, K);
    case CB_OP_W4A16:
      return w4a16_workspace_bytes(batch, M, N, K);
    case CB_OP_NVFP4:
      return nvfp4_workspace_bytes(M);
    case CB_OP_W4A4: {
      // the int8 GEMM scratch, then unpacked A [M, K] and B [N, K] (8-bit).
      const size_t a = align_up(static_cast<size_t>(M) * K, 256);
      const size_t b = align_up(static_cast<size_t>(N) * K, 256);
      return align_up(w8a8_workspace_bytes(1, M, N, K), 256) + a + b;
    }
    default:
      return 0;
  }
}

int cb_workspace_status(void* workspace, int* device_status, cb_stream_t stream) {
  if (!workspace) return CB_ERR_INVALID_ARG;
  return read_and_clear_status(workspace, device_status, reinterpret_cast<cudaStream_t>(stream));
}

void cb_debug_force_wait_timeout(uint64_t limit_ns) {
  g_debug_wait_ns.store(static_cast<unsigned long long>(limit_ns), std::memory_order_relaxed);
}

void cb_debug_force_last_arriver(int on) { g_force_last_arriver.store(on != 0, std::memory_order_relaxed); }

int cb_quant_act_i8(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_stride_b,
                    int64_t a_stride_m, int8_t* q, int64_t q_stride_b, int64_t q_stride_m, float* scale,
                    int64_t scale_stride_b, cb_stream_t stream) {
  if (batch < 0 || M < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (batch * M * K == 0) return CB_OK;
  if (!a || !q || !scale) return CB_ERR_INVALID_ARG;
  if (a_dtype != CB_DTYPE_F16 && a_dtype != CB_DTYPE_BF16) return CB_ERR_DTYPE;
  if (K > 0x7fffffffLL || M > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  return launch_act_quant(a, a_dtype, batch, M, K, a_stride_b, a_stride_m, q, q_stride_b, q_stride_m, scale,
                          scale_stride_b, reinterpret_cast<cudaStream_t>(stream));
}

int cb_w8a8_gemm(const int8_t* aq, const float* a_scale, const int8_t* w, const float* w_scale, void* out,
                 int out_dtype, int32_t* acc_out, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const int64_t* strides, void* workspace, size_t workspace_bytes, cb_stream_t stream) {
  return cb_w8a8_gemm_bias(aq, a_scale, w, w_scale, nullptr, CB_DTYPE_F32, 0, out, out_dtype, acc_out, batch, M, N,
                           K, strides, workspace, workspace_bytes, stream);
}

int cb_w8a8_gemm_bias(const int8_t* aq, const float* a_scale, const int8_t* w, const float* w_scale,
                      const void* bias, int bias_dtype, int64_t bias_stride_b, void* out, int out_dtype,
                      int32_t* acc_out, int64_t batch, int64_t M, int64_t N, int64_t K, const int64_t* strides,
                      void* workspace, size_t workspace_bytes, cb_stream_t stream) {
  int v = validate_w8a8(aq, w, out, out_dtype, batch, M, N, K, strides);
  if (v != CB_OK || batch * M * N == 0) return v;
  if (!a_scale || !w_scale) return CB_ERR_INVALID_ARG;
  if (bias && !valid_out_dtype(bias_dtype)) return CB_ERR_DTYPE;
  if (bias && batch > 1 && bias_stride_b < N) return CB_ERR_STRIDE;
  W8A8Launch L = {};
  L.aq = aq;
  L.a_scale = a_scale;
  L.w = w;
  L.w_scale = w_scale;
  L.out = out;
  L.out_dtype = out_dtype;
  L.acc_out = acc_out;
  L.batch = batch;
  L.M = M;
  L.N = N;
  L.K = K;
  L.aq_sb = strides[0];
  L.aq_sm = strides[1];
  L.w_sb = strides[2];
  L.w_sn = strides[3];
  L.out_sb = strides[4];
  L.out_sm = strides[5];
  L.as_sb = strides[6];
  L.ws_sb = strides[7];
  L.raw_f32 = 0;
  L.bias = bias;
  L.bias_dtype = bias_dtype;
  L.bias_sb = bias_stride_b;
  L.workspace = workspace;
  L.workspace_bytes = workspace_bytes;
  return launch_w8a8(L, reinterpret_cast<cudaStream_t>(stream));
}

int cb_w8a8_gemm_dynamic(const void* a, int a_dtype, int8_t* q_buf, float* s_buf, const int8_t* w,
                         const float* w_scale, void* out, int out_dtype, int64_t batch, int64_t M, int64_t N,
                         int64_t K, const int64_t* strides, void* workspace, size_t workspace_bytes,
                         cb_stream_t stream) {
  if (!strides) return CB_ERR_INVALID_ARG;
  const int64_t st8[8] = {M * K, K, strides[2], strides[3], strides[4], strides[5], M, strides[6]};
  int v = validate_w8a8(q_buf, w, out, out_dtype, batch, M, N, K, st8);
  if (v != CB_OK || batch * M * N == 0) return v;
  if (!a || !s_buf || !w_scale) return CB_ERR_INVALID_ARG;
  if (a_dtype != CB_DTYPE_F16 && a_dtype != CB_DTYPE_BF16) return CB_ERR_DTYPE;
  const size_t need = w8a8_workspace_bytes(batch, M, N, K);
  if (!workspace || workspace_bytes < need) return CB_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  W8A8Launch L = {};
  L.aq = q_buf;
  L.a_scale = s_buf;
  L.w = w;
  L.w_scale = w_scale;
  L.out = out;
  L.out_dtype = out_dtype;
  L.acc_out = nullptr;
  L.batch = batch;
  L.M = M;
  L.N = N;
  L.K = K;
  L.aq_sb = M * K;
  L.aq_sm = K;
  L.w_sb = strides[2];
  L.w_sn = strides[3];
  L.out_sb = strides[4];
  L.out_sm = strides[5];
  L.as_sb = M;
  L.ws_sb = strides[6];
  L.workspace = workspace;
  L.workspace_bytes = workspace_bytes;
  // One token of a single GEMM with a short row: the GEMV quantizes the row
  // itself (same arithmetic, q and scale still stored to q_buf / s_buf), one
  // launch.
  if (w8a8_gemv_dynamic_eligible(L, a, a_dtype, strides[1])) return launch_w8a8_gemv_dynamic(L, a, a_dtype, strides[1], s);
  int r = launch_act_quant(a, a_dtype, batch, M, K, strides[0], strides[1], q_buf, M * K, K, s_buf, M, s);
  if (r != CB_OK) return r;
  return launch_w8a8(L, s);
}

int cb_quant_act_fp8(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_stride_b,
                     int64_t a_stride_m, uint8_t* q, int64_t q_stride_b, int64_t q_stride_m, float* scale,
                     int64_t scale_stride_b, int mode, cb_stream_t stream) {
  if (batch < 0 || M < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (batch * M * K == 0) return CB_OK;
  if (!a || !q || !scale) return CB_ERR_INVALID_ARG;
  if (a_dtype != CB_DTYPE_F16 && a_dtype != CB_DTYPE_BF16) return CB_ERR_DTYPE;
  if (K > 0x7fffffffLL || M > 0x7fffffffLL || batch > 0xffffLL) return CB_ERR_TOO_LARGE;
  return launch_act_quant_fp8(a, a_dtype, batch, M, K, a_stride_b, a_stride_m, q, q_stride_b, q_stride_m, scale,
                              scale_stride_b, mode, reinterpret_cast<cudaStream_t>(stream));
}

int cb_fp8_gemm(const uint8_t* aq, const float* a_scale, int a_scale_per_tensor, const uint8_t* w,
                const float* w_scale, int w_scale_per_tensor, const void* bias, int bias_dtype, void* out,
                int out_dtype, int64_t batch, int64_t M, int64_t N, int64_t K, const int64_t* strides,
                void* workspace, size_t workspace_bytes, cb_stream_t stream) {
  int v = validate_w8a8(reinterpret_cast<const int8_t*>(aq), reinterpret_cast<const int8_t*>(w), out, out_dtype,
                        batch, M, N, K, strides);
  if (v != CB_OK || batch * M * N == 0) return v;
  if (!a_scale || !w_scale) return CB_ERR_INVALID_ARG;
  if (bias && !valid_out_dtype(bias_dtype)) return CB_ERR_DTYPE;
  W8A8Launch L = {};
  L.aq = reinterpret_cast<const int8_t*>(aq);
  L.a_scale = a_scale;
  L.w = reinterpret_cast<const int8_t*>(w);
  L.w_scale = w_scale;
  L.out = out;
  L.out_dtype = out_dtype;
  L.batch = batch;
  L.M = M;
  L.N = N;
  L.K = K;
  L.aq_sb = strides[0];
  L.aq_sm = strides[1];
  L.w_sb = strides[2];
  L.w_sn = strides[3];
  L.out_sb = strides[4];
  L.out_sm = strides[5];
  L.as_sb = strides[6];
  L.ws_sb = strides[7];
  L.fp8 = 1;
  L.scale_per_tensor_a = a_scale_per_tensor ? 1 : 0;
  L.scale_per_tensor_w = w_scale_per_tensor ? 1 : 0;
  L.bias = bias;
  L.bias_dtype = bias_dtype;
  L.bias_sb = 0;
  L.workspace = workspace;
  L.workspace_bytes = workspace_bytes;
  return launch_w8a8(L, reinterpret_cast<cudaStream_t>(stream));
}

int cb_w4a16_gemm(const void* a, int a_dtype, const uint8_t* w_native, const void* scales, int scale_dtype,
                  int64_t group_size, void* out, int out_dtype, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const int64_t* strides, void* workspace, size_t workspace_bytes, cb_stream_t stream) {
  if (batch < 0 || M < 0 || N < 0 || K < 0 || !strides) return CB_ERR_INVALID_ARG;
  if (batch * M * N == 0) return CB_OK;
  if (!a || !w_native || !scales || !out) return CB_ERR_INVALID_ARG;
  if (a_dtype != CB_DTYPE_F16 && a_dtype != CB_DTYPE_BF16) return CB_ERR_DTYPE;
  if (!valid_out_dtype(scale_dtype) || !valid_out_dtype(out_dtype)) return CB_ERR_DTYPE;
  if (K == 0 || K % 8 != 0) return CB_ERR_SHAPE;
  if (group_size <= 0 || (group_size < K && group_size % 128 != 0)) return CB_ERR_SHAPE;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL || batch > 0xffffLL) return CB_ERR_TOO_LARGE;
  if (!aligned16(a) || !aligned16(w_native)) return CB_ERR_ALIGNMENT;
  if ((strides[1] * 2) % 16 != 0 || (batch > 1 && (strides[0] * 2) % 16 != 0)) return CB_ERR_ALIGNMENT;
  if (strides[1] < K) return CB_ERR_STRIDE;
  W4A16Launch L = {};
  L.a = a;
  L.a_dtype = a_dtype;
  L.w = w_native;
  L.scales = scales;
  L.scale_dtype = scale_dtype;
  L.group_size = group_size >= K ? K : group_size;
  L.out = out;
  L.out_dtype = out_dtype;
  L.batch = batch;
  L.M = M;
  L.N = N;
  L.K = K;
  L.a_sb = strides[0];
  L.a_sm = strides[1];
  L.s_sb = strides[2];
  L.s_sg = strides[3];
  L.out_sb = strides[4];
  L.out_sm = strides[5];
  L.workspace = workspace;
  L.workspace_bytes = workspace_bytes;
  return launch_w4a16(L, reinterpret_cast<cudaStream_t>(stream));
}

int cb_nvfp4_quantize(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t x_stride, const float* global_scale,
                      uint8_t* q, int64_t q_stride, uint8_t* sf, cb_stream_t stream) {
  if (rows < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (rows == 0 || K == 0) return CB_OK;
  if (!x || !global_scale || !q || !sf) return CB_ERR_INVALID_ARG;
  if (x_dtype != CB_DTYPE_BF16 && x_dtype != CB_DTYPE_F16) return CB_ERR_DTYPE;
  if (K % 64 != 0) return CB_ERR_SHAPE;
  if (rows > 0x7fffffffLL || K > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  if (x_stride < K || q_stride < K / 2) return CB_ERR_STRIDE;
  if (!aligned16(x) || x_stride % 8 != 0 || reinterpret_cast<uintptr_t>(q) % 8 != 0 || q_stride % 8 != 0)
    return CB_ERR_ALIGNMENT;
  return launch_nvfp4_quant(x, x_dtype, rows, K, x_stride, global_scale, q, q_stride, sf,
                            reinterpret_cast<cudaStream_t>(stream));
}

int cb_nvfp4_gemm(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, const float* alpha,
                  void* out, int out_dtype, int64_t M, int64_t N, int64_t K, int64_t a_stride, int64_t b_stride,
                  int64_t out_stride, void* workspace, size_t workspace_bytes, cb_stream_t stream) {
  if (M < 0 || N < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (M * N == 0) return CB_OK;
  if (!a || !a_sf || !b || !b_sf || !alpha || !out) return CB_ERR_INVALID_ARG;
  if (!valid_out_dtype(out_dtype)) return CB_ERR_DTYPE;
  if (K == 0 || K % 64 != 0) return CB_ERR_SHAPE;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  if (a_stride < K / 2 || b_stride < K / 2 || out_stride < N) return CB_ERR_STRIDE;
  if (!aligned16(a) || !aligned16(b) || !aligned16(a_sf) || !aligned16(b_sf) || a_stride % 16 != 0 ||
      b_stride % 16 != 0)
    return CB_ERR_ALIGNMENT;
  Nvfp4Launch L = {};
  L.a = a;
  L.a_sf = a_sf;
  L.b = b;
  L.b_sf = b_sf;
  L.alpha = alpha;
  L.out = out;
  L.out_dtype = out_dtype;
  L.M = M;
  L.N = N;
  L.K = K;
  L.a_sm = a_stride;
  L.b_sn = b_stride;
  L.out_sm = out_stride;
  L.workspace = workspace;
  L.workspace_bytes = workspace_bytes;
  return launch_nvfp4_gemm(L, reinterpret_cast<cudaStream_t>(stream));
}

int cb_w4a4_gemm(const uint8_t* a_packed, const uint8_t* b_packed, float* c, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc, int nibble_mode, void* workspace, size_t workspace_bytes,
                 cb_stream_t stream) {
  if (nibble_mode != CB_W4A4_SIGNED && nibble_mode != CB_W4A4_REF_UINT8_WRAP) return CB_ERR_INVALID_ARG;
  const int wrap = nibble_mode == CB_W4A4_REF_UINT8_WRAP ? 1 : 0;
  if (M < 0 || N < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (M * N == 0) return CB_OK;
  if (!a_packed || !b_packed || !c) return CB_ERR_INVALID_ARG;
  if (K == 0 || K % 32 != 0) return CB_ERR_SHAPE;
  if (lda < K / 2 || ldb < N || ldc < N) return CB_ERR_STRIDE;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  const size_t need = cb_workspace_bytes(CB_OP_W4A4, 1, M, N, K);
  if (!workspace || workspace_bytes < need) return CB_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The GEMM's split-K scratch sits at the start of the workspace, where every
  // op keeps its (always re-zeroed) arrival counters; the unpacked operands follow.
  const size_t gemm_bytes = align_up(w8a8_workspace_bytes(1, M, N, K), 256);
  void* gemm_ws = workspace;
  uint8_t* a8 = static_cast<uint8_t*>(workspace) + gemm_bytes;
  uint8_t* b8 = a8 + align_up(static_cast<size_t>(M) * K, 256);
  unpack_rows_i4_kernel<<<grid_for(M * K / 2, 256), 256, 0, s>>>(a_packed, lda, a8, M, K, wrap);
  {
    const long long tiles = ((N + kUnpackTile - 1) / kUnpackTile) * ((K / 2 + kUnpackTile - 1) / kUnpackTile);
    if (tiles > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
    unpack_cols_i4_tiled_kernel<<<static_cast<unsigned>(tiles), 256, 0, s>>>(b_packed, ldb, b8, K, N, wrap);
  }
  if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
  W8A8Launch L = {};
  L.aq = reinterpret_cast<const int8_t*>(a8);
  L.w = reinterpret_cast<const int8_t*>(b8);
  L.unsigned_operands = wrap;
  L.out = c;
  L.out_dtype = CB_DTYPE_F32;
  L.batch = 1;
  L.M = M;
  L.N = N;
  L.K = K;
  L.aq_sb = M * K;
  L.aq_sm = K;
  L.w_sb = N * K;
  L.w_sn = K;
  L.out_sb = M * ldc;
  L.out_sm = ldc;
  L.raw_f32 = 1;
  L.workspace = gemm_ws;
  L.workspace_bytes = gemm_bytes;
  return launch_w8a8(L, s);
}

size_t cb_w4_native_bytes(int64_t batch, int64_t K, int64_t N) {
  if (batch < 0 || K < 0 || N < 0) return 0;
  const size_t nt = static_cast<size_t>((N + 127) / 128), kt = static_cast<size_t>((K + 127) / 128);
  return static_cast<size_t>(batch) * nt * kt * 128 * 64;
}

int cb_repack_w4(const void* src, int src_layout, uint8_t* dst_native, int64_t batch, int64_t K, int64_t N,
                 cb_stream_t stream) {
  if (batch < 0 || K < 0 || N < 0) return CB_ERR_INVALID_ARG;
  if (batch * K * N == 0) return CB_OK;
  if (!src || !dst_native) return CB_ERR_INVALID_ARG;
  if (src_layout != CB_W4_REF_U8_KN && src_layout != CB_W4_I32_K8N) return CB_ERR_UNSUPPORTED;
  if (src_layout == CB_W4_REF_U8_KN && K % 2 != 0) return CB_ERR_SHAPE;
  if (src_layout == CB_W4_I32_K8N && K % 8 != 0) return CB_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(dst_native) & 3u) != 0) return CB_ERR_ALIGNMENT;
  const long long nt = (N + 127) / 128, kt = (K + 127) / 128;
  const long long words = batch * nt * kt * 128 * 16;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  repack_w4_kernel<<<grid_for(words, 256), 256, 0, s>>>(static_cast<const uint8_t*>(src), src_layout,
                                                         reinterpret_cast<uint32_t*>(dst_native), batch, K, N, nt,
                                                         kt);
  return cuda_status(cudaGetLastError());
}

int cb_repack_w8_kmajor(const int8_t* src_kn, int8_t* dst_nk, int64_t batch, int64_t K, int64_t N,
                        cb_stream_t stream) {
  if (batch < 0 || K < 0 || N < 0) return CB_ERR_INVALID_ARG;
  if (batch * K * N == 0) return CB_OK;
  if (!src_kn || !dst_nk) return CB_ERR_INVALID_ARG;
  if (batch > 65535 || (K + 31) / 32 > 65535) return CB_ERR_TOO_LARGE;
  dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((K + 31) / 32), static_cast<unsigned>(batch));
  transpose_i8_kernel<<<grid, dim3(32, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(src_kn, dst_nk, K, N);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
