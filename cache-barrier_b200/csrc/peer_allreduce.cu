// One-shot all-reduce over NVLink peer memory for the small partial outputs of
// row-parallel projections (a [T, hidden] bf16/f16 tensor per rank, tens to
// hundreds of KiB), where a library ring all-reduce is latency-bound.
//
// Low-latency protocol: every 8-byte word a rank sends carries two 16-bit
// values and the 32-bit number of the call, written with one 64-bit store
// (single-copy atomic), so a reader that sees the call number in a word has
// its data too: no fences and no separate flags. Each rank owns a symmetric
// area (allocated once by cb_symm_alloc, mapped into every peer's address space
// through CUDA IPC handles exchanged by the host):
//   recv  [2 parities][world][slot_pairs] 64-bit words (data | call << 32)
//   ctl   [call number of the last completed call, CTA finish counter]
// A call runs the same grid on every rank; CTA b takes pairs [p0, p1) of the
// tensor. It stores its pairs into slot `rank` of every rank's recv area (plain
// 64-bit stores, local or peer), then polls its own recv area (bounded) until
// every rank's word for each of its pairs carries this call's number, sums the
// world values in rank order in fp32 and writes the rounded result, so every
// rank produces the same values. The call number is read from ctl after
// griddepcontrol.wait and advanced by the last CTA to finish, so calls work
// inside CUDA graphs. The two parities keep a fast rank's next-but-one call
// from overwriting words a slow rank still reads: a rank starts call e + 2 only
// after finishing call e + 1, which needed every peer's call-(e + 1) words,
// which each peer sent only after finishing call e.
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
constexpr int kMaxCtas = 128;
constexpr int kThreads = 256;
constexpr long long kPairsPerCta = 512;

struct PeerArgs {
  const uint16_t* in;
  uint16_t* out;
  long long n;           // elements
  long long slot_pairs;  // words per (parity, rank) slot
  int dtype;
  int rank, world;
  unsigned long long* recv[kMaxWorld];  // every rank's recv area, as mapped in this process
  unsigned int* ctl;                    // this rank's [last call, finish counter]
  int* status;                          // this rank's status word (bit CB_DEVERR_TIMEOUT on a wait that ran out)
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float to_f(uint32_t v, int dtype) {
  const uint16_t h = static_cast<uint16_t>(v);
  if (dtype == CB_DTYPE_BF16) return __bfloat162float(__ushort_as_bfloat16(h));
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t from_f(float v, int dtype) {
  if (dtype == CB_DTYPE_BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}

__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(const PeerArgs a) {
  pdl_launch_dependents();
  pdl_wait_primary();  // the partial comes from the preceding kernel
  __shared__ unsigned int sh_call;
  __shared__ int sh_abort;
  if (threadIdx.x == 0) {
    sh_call = *reinterpret_cast<volatile unsigned int*>(a.ctl) + 1u;
    sh_abort = 0;
  }
  __syncthreads();
  const unsigned int call = sh_call;
  const unsigned long long tag = static_cast<unsigned long long>(call) << 32;
  const int par = static_cast<int>(call & 1u);
  const long long pairs = (a.n + 1) / 2;
  const long long p0 = static_cast<long long>(blockIdx.x) * pairs / gridDim.x;
  const long long p1 = static_cast<long long>(blockIdx.x + 1) * pairs / gridDim.x;
  const long long my_slot = (static_cast<long long>(par) * a.world + a.rank) * a.slot_pairs;

  // 1. push: this rank's pairs into slot `rank` of every rank (8-byte words)
  for (long long i = p0 + threadIdx.x; i < p1; i += blockDim.x) {
    const uint32_t lo = a.in[2 * i];
    const uint32_t hi = (2 * i + 1 < a.n) ? a.in[2 * i + 1] : 0u;
    const unsigned long long w = tag | (hi << 16) | lo;
    for (int r = 0; r < a.world; ++r) st_relaxed_sys_u64(a.recv[r] + my_slot + i, w);
  }
  // 2. pull: wait (bounded) for every rank's word of each pair, sum in rank order
  const unsigned long long* mine = a.recv[a.rank] + static_cast<long long>(par) * a.world * a.slot_pairs;
  const unsigned long long t0 = global_timer_ns();
  for (long long i = p0 + threadIdx.x; i < p1; i += blockDim.x) {
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int r = 0; r < a.world; ++r) {
      const unsigned long long* src = mine + static_cast<long long>(r) * a.slot_pairs + i;
      unsigned long long w = ld_relaxed_sys_u64(src);
      int spins = 0;
      while ((w >> 32) != call) {
        if ((++spins & 63) == 0) {
          if (*reinterpret_cast<volatile int*>(&sh_abort)) break;
          if (global_timer_ns() - t0 > kWaitLimitNs) {
            sh_abort = 1;
            atomicOr(a.status, CB_DEVERR_TIMEOUT);
            break;
          }
        }
        w = ld_relaxed_sys_u64(src);
      }
      acc0 += to_f(static_cast<uint32_t>(w), a.dtype);
      acc1 += to_f(static_cast<uint32_t>(w >> 16), a.dtype);
    }
    a.out[2 * i] = from_f(acc0, a.dtype);
    if (2 * i + 1 < a.n) a.out[2 * i + 1] = from_f(acc1, a.dtype);
  }
  // 3. the last CTA to finish records this call as completed
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.ctl[1], 1u) == gridDim.x - 1) {
      a.ctl[1] = 0;
      a.ctl[0] = call;
      __threadfence();
    }
  }
}

}  // namespace

size_t symm_bytes(int world, int64_t slot_elems) {
  const size_t recv = 2ull * world * static_cast<size_t>((slot_elems + 1) / 2) * 8;
  return align_up(recv, 256) + 256;  // + ctl
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
  // 16-bit elements
  if ((reinterpret_cast<uintptr_t>(in) & 1u) || (reinterpret_cast<uintptr_t>(out) & 1u)) return CB_ERR_ALIGNMENT;
  PeerArgs a = {};
  a.in = static_cast<const uint16_t*>(in);
  a.out = static_cast<uint16_t*>(out);
  a.n = elems;
  a.slot_pairs = (slot_elems + 1) / 2;
  a.dtype = dtype;
  a.rank = rank;
  a.world = world;
  const size_t recv_bytes = align_up(2ull * world * static_cast<size_t>(a.slot_pairs) * 8, 256);
  for (int r = 0; r < world; ++r) {
    if (!symm_areas[r]) return CB_ERR_INVALID_ARG;
    a.recv[r] = static_cast<unsigned long long*>(symm_areas[r]);
  }
  a.ctl = reinterpret_cast<unsigned int*>(static_cast<char*>(symm_areas[rank]) + recv_bytes);
  a.status = status;
  // one CTA per kPairsPerCta pairs, at most kMaxCtas; the grid depends only on
  // elems, so every rank runs the same grid for the same call
  long long ctas = ((elems + 1) / 2 + kPairsPerCta - 1) / kPairsPerCta;
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
