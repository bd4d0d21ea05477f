// Allocation-free entry point for the W8A8 GEMM.
//
// Some callers cannot allocate device memory: a host program whose device
// memory is entirely owned by another component's pool allocator, or a
// foreign-language binding that holds raw device pointers but no allocator to
// call. cb_w8a8_gemm_noalloc lets them run the split-K W8A8 GEMM by passing only
// inputs and outputs: its scratch (status word, arrival counters, partial
// accumulators) lives in the file-scope device array below, which every GPU that
// loads this library holds until the process exits.
//
// Rules of use:
//   - the array is 8 MiB; a problem whose scratch need (cb_workspace_bytes for
//     CB_OP_W8A8) exceeds it is rejected with CB_ERR_TOO_LARGE. On a 148-SM B200
//     that admits up to 32 tokens (M <= 32) per call;
//   - the first call on a device looks the array's device address up
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture;
//   - the cached address belongs to the device's CUDA context at the time of
//     the first call: after a device reset (cudaDeviceReset, or a reset of the
//     primary context) the library must be reloaded before calling it again;
//   - every call on a device shares the one array and leaves its last contents
//     there: the call clears the arrival counters on its stream before
//     launching, and two calls whose kernels overlap on the GPU (different
//     streams, no ordering) race on the array;
//   - the status word at the start of the array is not cleared by a call: a
//     bounded device-side wait that expired in any call stays recorded until
//     cb_w8a8_noalloc_status reads (and clears) it;
//   - nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda_runtime.h>

#include <mutex>

#include "cb200.h"
#include "cb_internal.h"

namespace cb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

// Host code must not use this name as a device address: in host code it is a
// host-side stand-in. The device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of the scratch array on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return CB_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return CB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return CB_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return CB_OK;
}

}  // namespace
}  // namespace cb

extern "C" int cb_w8a8_gemm_noalloc(const int8_t* aq, const float* a_scale, const int8_t* w, const float* w_scale,
                                    void* out, int out_dtype, int32_t* acc_out, int64_t batch, int64_t M, int64_t N,
                                    int64_t K, const int64_t* strides, cb_stream_t stream) {
  using namespace cb;
  int v = validate_w8a8(aq, w, out, out_dtype, batch, M, N, K, strides);
  if (v != CB_OK || batch * M * N == 0) return v;
  if (!a_scale || !w_scale) return CB_ERR_INVALID_ARG;
  if (w8a8_workspace_bytes(batch, M, N, K) > kNoAllocScratchBytes) return CB_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != CB_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The arrival counters must start at zero (a call that gave up a wait can
  // leave some behind); the partial slots are fully written before they are
  // read. The status word is left alone, so a timeout recorded by an earlier
  // call survives until cb_w8a8_noalloc_status reads it.
  if (cudaMemsetAsync(static_cast<char*>(scratch) + kWsHeader, 0, kWsCounters, s) != cudaSuccess) return CB_ERR_CUDA;
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
  L.workspace = scratch;
  L.workspace_bytes = kNoAllocScratchBytes;
  return launch_w8a8(L, s);
}

extern "C" int cb_w8a8_noalloc_status(int* device_status, cb_stream_t stream) {
  using namespace cb;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != CB_OK) return st;
  return read_and_clear_status(scratch, device_status, reinterpret_cast<cudaStream_t>(stream));
}
