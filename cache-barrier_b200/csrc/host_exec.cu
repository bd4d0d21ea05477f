// Host-buffer executor: the W8A8 dynamic-quantization GEMM called with
// activations and outputs in host memory (no counterpart in the reference,
// whose w8a8_bmm_full takes device tensors; profiling/w8a8/w8a8_bmm.py:143-149).
//
// One call = copy the activations in, quantize + GEMM (the PDL-chained pair of
// cb_w8a8_gemm_dynamic), copy the result out. The three steps run on three
// streams of the executor, linked by events, with kSlots device buffers in a
// ring, so call j's input copy and call j-1's output copy overlap call j-1's and
// call j's kernels: a sequence of calls costs about max(kernels, copies) per
// call instead of their sum. The calling thread only enqueues (two copies, two
// launches, a few event records and waits).
//
// Ordering per slot s (calls j and j + kSlots share s):
//   in-copy(j)  waits compute(j - kSlots)  (the quantizer read a[s])
//   compute(j)  waits in-copy(j), out-copy(j - kSlots)  (out[s] was read back)
//   out-copy(j) waits compute(j)
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <new>

#include "cb200.h"
#include "cb_internal.h"

namespace cb {
namespace {

constexpr int kSlots = 2;

struct Slot {
  void* a = nullptr;
  int8_t* q = nullptr;
  float* s = nullptr;
  void* out = nullptr;
  bool used = false;
  cudaEvent_t in_done = nullptr, compute_done = nullptr, out_done = nullptr;
};

size_t dtype_bytes(int d) { return d == CB_DTYPE_F32 ? 4 : 2; }

}  // namespace
}  // namespace cb

struct cb_exec {
  int device = 0;
  cudaStream_t in_stream = nullptr, compute = nullptr, out_stream = nullptr;
  cudaEvent_t join = nullptr;
  cb::Slot slot[cb::kSlots];
  size_t a_cap = 0, q_cap = 0, s_cap = 0, out_cap = 0;  // bytes per slot
  void* workspace = nullptr;
  size_t ws_cap = 0;
  long long calls = 0;
};

using namespace cb;

namespace {

void free_buffers(cb_exec* e) {
  for (Slot& sl : e->slot) {
    cudaFree(sl.a);
    cudaFree(sl.q);
    cudaFree(sl.s);
    cudaFree(sl.out);
    sl.a = sl.q = nullptr;
    sl.s = nullptr;
    sl.out = nullptr;
    sl.used = false;
  }
  cudaFree(e->workspace);
  e->workspace = nullptr;
  e->a_cap = e->q_cap = e->s_cap = e->out_cap = e->ws_cap = 0;
}

int drain(cb_exec* e) {
  if (cudaStreamSynchronize(e->in_stream) != cudaSuccess || cudaStreamSynchronize(e->compute) != cudaSuccess ||
      cudaStreamSynchronize(e->out_stream) != cudaSuccess)
    return CB_ERR_CUDA;
  return CB_OK;
}

// Grows the slot buffers and the split-K workspace to fit one call. Growing
// waits for the executor's work in flight first (the old buffers may be in use).
int reserve(cb_exec* e, size_t a_bytes, size_t q_bytes, size_t s_bytes, size_t out_bytes, size_t ws_bytes) {
  if (a_bytes <= e->a_cap && q_bytes <= e->q_cap && s_bytes <= e->s_cap && out_bytes <= e->out_cap &&
      ws_bytes <= e->ws_cap)
    return CB_OK;
  int r = drain(e);
  if (r != CB_OK) return r;
  const size_t a = a_bytes > e->a_cap ? a_bytes : e->a_cap;
  const size_t q = q_bytes > e->q_cap ? q_bytes : e->q_cap;
  const size_t s = s_bytes > e->s_cap ? s_bytes : e->s_cap;
  const size_t o = out_bytes > e->out_cap ? out_bytes : e->out_cap;
  const size_t w = ws_bytes > e->ws_cap ? ws_bytes : e->ws_cap;
  free_buffers(e);
  for (Slot& sl : e->slot) {
    if (cudaMalloc(&sl.a, align_up(a, 256)) != cudaSuccess || cudaMalloc(&sl.q, align_up(q, 256)) != cudaSuccess ||
        cudaMalloc(&sl.s, align_up(s, 256)) != cudaSuccess || cudaMalloc(&sl.out, align_up(o, 256)) != cudaSuccess) {
      free_buffers(e);
      return CB_ERR_CUDA;
    }
  }
  // The split-K scratch starts zeroed; the kernels leave it zeroed.
  if (cudaMalloc(&e->workspace, w) != cudaSuccess || cudaMemset(e->workspace, 0, w) != cudaSuccess) {
    free_buffers(e);
    return CB_ERR_CUDA;
  }
  e->a_cap = a;
  e->q_cap = q;
  e->s_cap = s;
  e->out_cap = o;
  e->ws_cap = w;
  return CB_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

int cb_exec_create(int device, cb_exec** exec) {
  if (!exec) return CB_ERR_INVALID_ARG;
  *exec = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return CB_ERR_INVALID_ARG;
  DeviceGuard g(device);
  cb_exec* e = new (std::nothrow) cb_exec();
  if (!e) return CB_ERR_CUDA;
  e->device = device;
  bool ok = cudaStreamCreateWithFlags(&e->in_stream, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&e->compute, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&e->out_stream, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&e->join, cudaEventDisableTiming) == cudaSuccess;
  for (Slot& sl : e->slot)
    ok = ok && cudaEventCreateWithFlags(&sl.in_done, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&sl.compute_done, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&sl.out_done, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cb_exec_destroy(e);
    return CB_ERR_CUDA;
  }
  *exec = e;
  return CB_OK;
}

void cb_exec_destroy(cb_exec* e) {
  if (!e) return;
  DeviceGuard g(e->device);
  if (e->in_stream && e->compute && e->out_stream) drain(e);
  free_buffers(e);
  for (Slot& sl : e->slot) {
    if (sl.in_done) cudaEventDestroy(sl.in_done);
    if (sl.compute_done) cudaEventDestroy(sl.compute_done);
    if (sl.out_done) cudaEventDestroy(sl.out_done);
  }
  if (e->join) cudaEventDestroy(e->join);
  if (e->in_stream) cudaStreamDestroy(e->in_stream);
  if (e->compute) cudaStreamDestroy(e->compute);
  if (e->out_stream) cudaStreamDestroy(e->out_stream);
  delete e;
}

int cb_exec_after(cb_exec* e, cb_stream_t stream) {
  if (!e) return CB_ERR_INVALID_ARG;
  DeviceGuard g(e->device);
  if (cudaEventRecord(e->join, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaStreamWaitEvent(e->in_stream, e->join, 0) != cudaSuccess ||
      cudaStreamWaitEvent(e->compute, e->join, 0) != cudaSuccess ||
      cudaStreamWaitEvent(e->out_stream, e->join, 0) != cudaSuccess)
    return CB_ERR_CUDA;
  return CB_OK;
}

int cb_exec_before(cb_exec* e, cb_stream_t stream) {
  if (!e) return CB_ERR_INVALID_ARG;
  DeviceGuard g(e->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Every call ends on the out stream, whose work waited for that call's
  // compute, which waited for its in-copy: joining the out stream and the
  // in stream (copies of calls not yet computed cannot exist) covers all.
  cudaStream_t from[2] = {e->in_stream, e->out_stream};
  for (cudaStream_t f : from) {
    if (cudaEventRecord(e->join, f) != cudaSuccess || cudaStreamWaitEvent(s, e->join, 0) != cudaSuccess)
      return CB_ERR_CUDA;
  }
  return CB_OK;
}

int cb_exec_synchronize(cb_exec* e, int* device_status) {
  if (!e) return CB_ERR_INVALID_ARG;
  DeviceGuard g(e->device);
  int r = drain(e);
  if (r != CB_OK) return r;
  if (device_status) *device_status = 0;
  if (!e->workspace) return CB_OK;
  return read_and_clear_status(e->workspace, device_status, e->compute);
}

int cb_exec_w8a8_dynamic_host(cb_exec* e, const void* a_host, int a_dtype, const int8_t* w, const float* w_scale,
                              int64_t w_stride_b, int64_t w_stride_n, int64_t w_scale_stride_b, void* out_host,
                              int out_dtype, int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (!e) return CB_ERR_INVALID_ARG;
  if (batch < 0 || M < 0 || N < 0 || K < 0) return CB_ERR_INVALID_ARG;
  if (batch * M * N == 0) return CB_OK;
  if (!a_host || !out_host || !w || !w_scale) return CB_ERR_INVALID_ARG;
  if (a_dtype != CB_DTYPE_F16 && a_dtype != CB_DTYPE_BF16) return CB_ERR_DTYPE;
  if (out_dtype != CB_DTYPE_F16 && out_dtype != CB_DTYPE_BF16 && out_dtype != CB_DTYPE_F32) return CB_ERR_DTYPE;
  DeviceGuard g(e->device);
  const size_t a_bytes = static_cast<size_t>(batch * M * K) * 2;
  const size_t out_bytes = static_cast<size_t>(batch * M * N) * dtype_bytes(out_dtype);
  const size_t ws = w8a8_workspace_bytes(batch, M, N, K);
  int r = reserve(e, a_bytes, static_cast<size_t>(batch * M * K), static_cast<size_t>(batch * M) * 4, out_bytes, ws);
  if (r != CB_OK) return r;
  Slot& sl = e->slot[e->calls % kSlots];
  if (sl.used && cudaStreamWaitEvent(e->in_stream, sl.compute_done, 0) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaMemcpyAsync(sl.a, a_host, a_bytes, cudaMemcpyHostToDevice, e->in_stream) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaEventRecord(sl.in_done, e->in_stream) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaStreamWaitEvent(e->compute, sl.in_done, 0) != cudaSuccess) return CB_ERR_CUDA;
  if (sl.used && cudaStreamWaitEvent(e->compute, sl.out_done, 0) != cudaSuccess) return CB_ERR_CUDA;
  const int64_t strides[7] = {M * K, K, w_stride_b, w_stride_n, M * N, N, w_scale_stride_b};
  r = cb_w8a8_gemm_dynamic(sl.a, a_dtype, sl.q, sl.s, w, w_scale, sl.out, out_dtype, batch, M, N, K, strides,
                           e->workspace, e->ws_cap, reinterpret_cast<cb_stream_t>(e->compute));
  if (r != CB_OK) return r;
  if (cudaEventRecord(sl.compute_done, e->compute) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaStreamWaitEvent(e->out_stream, sl.compute_done, 0) != cudaSuccess) return CB_ERR_CUDA;
  if (cudaMemcpyAsync(out_host, sl.out, out_bytes, cudaMemcpyDeviceToHost, e->out_stream) != cudaSuccess)
    return CB_ERR_CUDA;
  if (cudaEventRecord(sl.out_done, e->out_stream) != cudaSuccess) return CB_ERR_CUDA;
  sl.used = true;
  ++e->calls;
  return CB_OK;
}

}  // extern "C"
