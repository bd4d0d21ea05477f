// One-shot all-reduce over NVLink peer memory for the small partial outputs of
// row-parallel projections (a [T, hidden] bf16/f16 tensor per rank, tens to
// hundreds of KiB), where a library ring all-reduce is latency-bound.
//
// Each rank owns a symmetric area (allocated once by cb_symm_alloc, mapped into
// every peer's address space through CUDA IPC handles exchanged by the host):
//   data  [2 parities][world][slot_elems]   16-bit partials written by the ranks
//   flags [2 parities][world][kMaxCtas]     epoch stamps, one per (rank, CTA)
//   epoch [kMaxCtas]                        this rank's per-CTA call counters
// A call runs the same grid on every rank. CTA b of rank r takes chunk b of the
// tensor: it stores the chunk into slot r of every rank's data area (plain
// stores, local or peer), fences at system scope, then stamps flags[p][r][b] =
// epoch on every rank with a release store. It waits (bounded) until all world
// stamps for chunk b in its own flags read the epoch, sums the world slots in
// rank order in fp32 and writes the rounded result, so every rank produces the
// same values. The two parities double-buffer consecutive calls: a rank writes
// parity p of call e+1 only after it saw every peer's stamp of call e, and a
// peer stamps call e only after it finished reading call e-1 (same parity as
// e+1) in the same CTA. The per-CTA counters advance on the device, so the
// call sequence works inside CUDA graphs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "cb_internal.h"
#include "cb_ptx.cuh"

namespace cb {
namespace {

constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 64;
constexpr int kThreads = 256;

struct PeerArgs {
  const uint16_t* in;
  uint16_t* out;
  long long n;
  long long slot_elems;
  int dtype;
  int rank, world;
  uint16_t* data[kMaxWorld];  // every rank's data area, as mapped in this process
  int* flags[kMaxWorld];      // every rank's flag area
  int* epoch;                 // this rank's per-CTA counters
  int* status;                // this rank's status word (bit CB_DEVERR_TIMEOUT on a wait that ran out)
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float to_f(uint16_t v, int dtype) {
  if (dtype == CB_DTYPE_BF16) return __bfloat162float(__ushort_as_bfloat16(v));
  return __half2float(__ushort_as_half(v));
}
__device__ __forceinline__ uint16_t from_f(float v, int dtype) {
  if (dtype == CB_DTYPE_BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}

__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(const PeerArgs a) {
  pdl_launch_dependents();
  pdl_wait_primary();  // the partial comes from the preceding kernel
  __shared__ int sh_epoch;
  __shared__ int sh_ok;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    sh_epoch = ++a.epoch[b];
    sh_ok = 1;
  }
  __syncthreads();
  const int e = sh_epoch;
  const int par = e & 1;
  const long long c0 = static_cast<long long>(b) * a.n / gridDim.x;
  const long long c1 = static_cast<long long>(b + 1) * a.n / gridDim.x;
  const long long slot = static_cast<long long>(par) * a.world * a.slot_elems + static_cast<long long>(a.rank) * a.slot_elems;

  // 1. push this rank's chunk into slot `rank` of every rank: 16-byte stores
  //    (one NVLink write carries 8 values; 2-byte stores would each be a packet)
  const long long v0 = (c0 + 7) / 8, v1 = c1 / 8;  // whole 8-element vectors inside the chunk
  for (long long j = v0 + threadIdx.x; j < v1; j += blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(a.in)[j];
    for (int r = 0; r < a.world; ++r) reinterpret_cast<uint4*>(a.data[r] + slot)[j] = v;
  }
  for (long long i = c0 + threadIdx.x; i < c1; i += blockDim.x) {  // ragged ends
    if (i >= v0 * 8 && i < v1 * 8) continue;
    const uint16_t v = a.in[i];
    for (int r = 0; r < a.world; ++r) a.data[r][slot + i] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < a.world; ++r)
      st_release_sys(a.flags[r] + (par * kMaxWorld + a.rank) * kMaxCtas + b, e);
  }
  // 2. wait for every rank's stamp of this chunk (bounded)
  if (threadIdx.x < a.world) {
    const int* f = a.flags[a.rank] + (par * kMaxWorld + threadIdx.x) * kMaxCtas + b;
    const unsigned long long t0 = global_timer_ns();
    while (ld_acquire_sys(f) != e) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        sh_ok = 0;
        atomicOr(a.status, CB_DEVERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
  if (!sh_ok) return;
  // 3. sum the world slots in rank order
  const uint16_t* mine = a.data[a.rank] + static_cast<long long>(par) * a.world * a.slot_elems;
  for (long long j = v0 + threadIdx.x; j < v1; j += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < a.world; ++r) {
      const uint4 v = reinterpret_cast<const uint4*>(mine + static_cast<long long>(r) * a.slot_elems)[j];
      const uint16_t* h = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += to_f(h[q], a.dtype);
    }
    uint4 o;
    uint16_t* oh = reinterpret_cast<uint16_t*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oh[q] = from_f(acc[q], a.dtype);
    reinterpret_cast<uint4*>(a.out)[j] = o;
  }
  for (long long i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    if (i >= v0 * 8 && i < v1 * 8) continue;
    float acc = 0.0f;
    for (int r = 0; r < a.world; ++r) acc += to_f(mine[static_cast<long long>(r) * a.slot_elems + i], a.dtype);
    a.out[i] = from_f(acc, a.dtype);
  }
}

}  // namespace

size_t symm_bytes(int world, int64_t slot_elems) {
  const size_t data = 2ull * world * static_cast<size_t>(slot_elems) * 2;
  const size_t flags = 2ull * kMaxWorld * kMaxCtas * sizeof(int);
  return align_up(data, 256) + flags + kMaxCtas * sizeof(int) + 256;
}

}  // namespace cb

using namespace cb;

extern "C" {

CB_API size_t cb_symm_bytes(int world, int64_t slot_elems) {
  if (world < 1 || world > kMaxWorld || slot_elems < 0) return 0;
  return symm_bytes(world, slot_elems);
}

CB_API int cb_symm_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return CB_ERR_INVALID_ARG;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return CB_ERR_CUDA;
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return CB_ERR_CUDA;
  }
  *ptr = p;
  return CB_OK;
}

CB_API int cb_symm_free(void* ptr) { return ptr ? cuda_status(cudaFree(ptr)) : CB_OK; }

CB_API int cb_ipc_get_handle(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return CB_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return CB_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  return CB_OK;
}

CB_API int cb_ipc_open_handle(const void* handle_in, void** peer_ptr) {
  if (!handle_in || !peer_ptr) return CB_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle_in, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return CB_ERR_CUDA;
  *peer_ptr = p;
  return CB_OK;
}

CB_API int cb_ipc_close_handle(void* peer_ptr) { return peer_ptr ? cuda_status(cudaIpcCloseMemHandle(peer_ptr)) : CB_OK; }

CB_API int cb_peer_allreduce(const void* in, void* out, int64_t elems, int dtype, void* const* symm_areas, int rank,
                             int world, int64_t slot_elems, int* status, cb_stream_t stream) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || elems < 0 || slot_elems < 0)
    return CB_ERR_INVALID_ARG;
  if (dtype != CB_DTYPE_BF16 && dtype != CB_DTYPE_F16) return CB_ERR_DTYPE;
  if (elems > slot_elems) return CB_ERR_TOO_LARGE;
  if (elems == 0) return CB_OK;
  if (!in || !out || !symm_areas || !status) return CB_ERR_INVALID_ARG;
  // 16-byte vector paths: in, out and every slot start on a 16-byte boundary
  if (!aligned16(in) || !aligned16(out) || slot_elems % 8 != 0) return CB_ERR_ALIGNMENT;
  PeerArgs a = {};
  a.in = static_cast<const uint16_t*>(in);
  a.out = static_cast<uint16_t*>(out);
  a.n = elems;
  a.slot_elems = slot_elems;
  a.dtype = dtype;
  a.rank = rank;
  a.world = world;
  const size_t data_bytes = align_up(2ull * world * static_cast<size_t>(slot_elems) * 2, 256);
  for (int r = 0; r < world; ++r) {
    if (!symm_areas[r]) return CB_ERR_INVALID_ARG;
    char* base = static_cast<char*>(symm_areas[r]);
    a.data[r] = reinterpret_cast<uint16_t*>(base);
    a.flags[r] = reinterpret_cast<int*>(base + data_bytes);
  }
  a.epoch = reinterpret_cast<int*>(static_cast<char*>(symm_areas[rank]) + data_bytes + 2ull * kMaxWorld * kMaxCtas * sizeof(int));
  a.status = status;
  // one CTA per ~4K elements, at most kMaxCtas; the grid depends only on elems,
  // so every rank runs the same grid for the same call
  long long ctas = (elems + 4095) / 4096;
  if (ctas > kMaxCtas) ctas = kMaxCtas;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, a));
}

}  // extern "C"
