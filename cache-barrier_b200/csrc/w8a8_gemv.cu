// W8A8 for one or two tokens per batch entry (decode with T <= 2): int8 x int8
// on the integer dot-product units (dp4a) instead of the tensor cores.
//
// Math (_w8a8_bmm_kernel, profiling/w8a8/w8a8_bmm.py:44-81):
//   acc[n] = sum_k aq[k] * w[n, k]                  (int32, exact in any order)
//   out[n] = cvt(((float)acc * a_scale) * w_scale[n] (+ bias[n]))
// with the same fp32 operations, in the same order, as the tensor-core kernel's
// epilogue, so the two paths give identical bits.
//
// Layout: the weights are K-major ([batch, N, K]), rows contiguous. A warp
// works through "items": a block of RB = R * (32 / LPR) consecutive rows
// times one k-step of KCH * 16 * LPR bytes. In an item, LPR lanes share a row
// and each lane loads KCH 16-byte chunks of each of its R rows (R * KCH
// chunks, 4 KiB per warp for every launched shape: one 4 KiB slice of a long
// row, or 8 rows of 512 B ... 32 rows of 128 B), so a warp instruction reads
// 512 contiguous bytes. A warp's items are its row blocks b = gw, gw + W,
// gw + 2W, ... (W warps in a persistent grid) in k-step order; the chunks of
// the next D items are in flight while the current one is summed (a ring of
// D + 1 register buffers, indexed statically by unrolling over the ring), so
// the stream of weight requests does not drain between rows. The first D items
// are requested before griddepcontrol.wait (the weights are not written by the
// preceding kernel, the quantized token is). Activations are read per chunk
// after the wait (16 bytes per lane, L1 hits once a warp of the SM has read
// them). Row bookkeeping is 32-bit with one division per block: with 64-bit
// divisions per row the short-row shapes were issue-bound (H = 128, K = 128:
// 1.7 TB/s). The int32 partial sums of a row are added over its LPR lanes with
// shuffles; lane r of the row's group runs the epilogue of the block's r-th
// row. No split-K and no scratch: only the status word of the caller's
// workspace is touched, by the failure-detection test hook.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "cb_gemm_common.cuh"
#include "cb_internal.h"
#include "cb_ptx.cuh"

namespace cb {
namespace {

constexpr int kWgThreads = 128;
// Items in flight ahead of the one being summed: three for long rows (one row
// slice per item; 168 registers, three CTAs per SM), one for short rows (eight
// rows per lane and item: with three, 226 registers and two CTAs per SM).
// Measured at K = N = 8192: 13.9 / 15.9 / 13.1 us with one / two / three;
// H = 128, K = 128, N = 4096: 16.2 / 18.6 / 21.8 us.
constexpr int kDepthLong = 3;
constexpr int kDepthShort = 1;
// Above this many weight bytes the tensor-core kernel's stream-K split reads
// HBM faster (K = N = 16384: 45.5 vs 47.9 us; H = 128, K = 128, N = 10240:
// 43.7 vs 44.5 us); below it the GEMV's lower fixed cost wins.
constexpr long long kGemvMaxWeightBytes = 128ll << 20;
// Two tokens double the activation reads per weight chunk (L1 / load-unit
// traffic), which costs more than the tensor-core kernel's fixed cost once the
// weights are large: at 16 MiB (K = N = 4096) 6.4 vs 8.2 us, at 30 MiB
// (K = 5120, N = 6144) 12.7 vs 10.8 us, at 64 MiB 19.6 vs 14.7 us.
constexpr long long kGemv2MaxWeightBytes = 16ll << 20;
constexpr int kW8GemvMaxTokens = 2;

struct WgParams {
  const int8_t* aq;
  long long aq_sb, aq_sm;
  const float* a_scale;
  long long as_sb, as_sm;
  const int8_t* w;
  long long w_sb, w_sn;
  const float* w_scale;
  long long ws_sb, ws_sn;
  void* out;
  int out_dtype;
  long long out_sb, out_sm;
  int32_t* acc_out;
  int raw_f32;
  const void* bias;
  int bias_dtype;
  long long bias_sb;
  int N, K;
  int rows;                        // batch * N
  int* status;                     // the workspace's status word
  unsigned long long dbg_wait_ns;  // test hook: nonzero = wait this long on a flag nothing sets
};

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 16-byte weight load that does not allocate in L1: the streamed weights would
// otherwise evict the activation row that every warp of the SM re-reads. Used
// for long rows (K = N = 8192: 13.1 -> 12.4 us); with short rows the plain
// load is faster (H = 128, K = 128, N = 4096: 16.2 vs 16.7 us).
__device__ __forceinline__ uint4 ld_stream16(const void* ptr) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(ptr));
  return v;
}

// TM tokens (1 or 2) share each weight chunk.
template <int LPR, int KCH, int R, int D, int TM>
__global__ void __launch_bounds__(kWgThreads) w8a8_gemv_kernel(const WgParams p) {
  constexpr int kCh = R * KCH;            // chunks per lane per item
  constexpr int kRowsPerStep = 32 / LPR;  // rows covered by one chunk column of the warp
  constexpr int kRb = R * kRowsPerStep;   // rows per item
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, li = lane % LPR;  // row within a chunk column, lane within the row
  const int warps = static_cast<int>(gridDim.x) * (kWgThreads / 32);
  const int gw = static_cast<int>(blockIdx.x) * (kWgThreads / 32) + (threadIdx.x >> 5);
  const int kstep = KCH * 16 * LPR;
  const int nks = (p.K + kstep - 1) / kstep;
  const int blocks = (p.rows + kRb - 1) / kRb;
  const int my_blocks = gw < blocks ? (blocks - gw + warps - 1) / warps : 0;
  const int n_items = my_blocks * nks;
  // (batch entry, column) of this lane's R rows in block b (h = -1 past the
  // end): one 32-bit division per block, the rows of a block are consecutive
  auto locate = [&](int b, int(&hh)[R], int(&nn)[R]) {
    const int row0 = b * kRb;
    const int h0 = row0 / p.N;
    const int n0 = row0 - h0 * p.N;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = r * kRowsPerStep + sub;
      int n = n0 + o, h = h0;
      while (n >= p.N) {  // at most kRb / N + 1 steps
        n -= p.N;
        ++h;
      }
      hh[r] = row0 + o < p.rows ? h : -1;
      nn[r] = n;
    }
  };
  auto load_item = [&](uint4(&buf)[kCh], int b, int ks) {
    int hh[R], nn[R];
    locate(b, hh, nn);
    const int k0 = ks * kstep;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int8_t* wr = p.w + (hh[r] < 0 ? 0 : hh[r]) * p.w_sb + static_cast<long long>(nn[r]) * p.w_sn;
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        const int k = k0 + c * 16 * LPR + li * 16;
        buf[r * KCH + c] =
            (hh[r] < 0 || k >= p.K) ? make_uint4(0u, 0u, 0u, 0u)
            : R == 1                ? ld_stream16(wr + k)
                                    : __ldg(reinterpret_cast<const uint4*>(wr + k));
      }
    }
  };
  pdl_launch_dependents();
  uint4 ring[D + 1][kCh];
  // item i of this warp is (block gw + j * warps, k-step ks), i = j * nks + ks;
  // (pj, pk) runs D items ahead of (cj, ck)
  int pj = 0, pk = 0;
#pragma unroll
  for (int s = 0; s < D; ++s) {
    if (s < n_items) load_item(ring[s], gw + pj * warps, pk);
    if (++pk == nks) pk = 0, ++pj;
  }
  pdl_wait_primary();
  // Failure-detection test hook (cb_debug_force_wait_timeout): one thread per
  // CTA waits, with a short limit, on a workspace word that nothing sets; the
  // expired wait is recorded in the status word and the CTA skips its rows.
  if (p.dbg_wait_ns != 0) {
    __shared__ int sh_abort;
    if (threadIdx.x == 0) {
      sh_abort = 0;
      wait_counter(p.status + 1, 1, &sh_abort, p.status, p.dbg_wait_ns);
    }
    __syncthreads();
    if (sh_abort) return;
  }
  int acc[R][TM];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < TM; ++m) acc[r][m] = 0;
  int cj = 0, ck = 0;
  for (int base = 0; base < n_items; base += D + 1) {
#pragma unroll
    for (int s = 0; s <= D; ++s) {
      const int i = base + s;
      if (i >= n_items) break;
      if (i + D < n_items) load_item(ring[(s + D) % (D + 1)], gw + pj * warps, pk);
      if (++pk == nks) pk = 0, ++pj;
      const int b = gw + cj * warps;
      const int ks = ck;
      if (++ck == nks) ck = 0, ++cj;
      int hh[R], nn[R];
      locate(b, hh, nn);
      const int k0 = ks * kstep;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int8_t* ar = p.aq + (hh[r] < 0 ? 0 : hh[r]) * p.aq_sb;
#pragma unroll
        for (int c = 0; c < KCH; ++c) {
          const int k = k0 + c * 16 * LPR + li * 16;
          const uint4 w = ring[s][r * KCH + c];
#pragma unroll
          for (int m = 0; m < TM; ++m) {
            const uint4 a = (hh[r] >= 0 && k < p.K) ? __ldg(reinterpret_cast<const uint4*>(ar + m * p.aq_sm + k))
                                                    : make_uint4(0u, 0u, 0u, 0u);
            acc[r][m] = dp4a_ss(w.x, a.x, acc[r][m]);
            acc[r][m] = dp4a_ss(w.y, a.y, acc[r][m]);
            acc[r][m] = dp4a_ss(w.z, a.z, acc[r][m]);
            acc[r][m] = dp4a_ss(w.w, a.w, acc[r][m]);
          }
        }
      }
      if (ks != nks - 1) continue;
      // block done: sum each row over its LPR lanes (aligned groups of
      // consecutive lanes); lane li of the group finishes row r = li
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int m = 0; m < TM; ++m) {
#pragma unroll
          for (int o = LPR / 2; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
        }
      }
      int v[TM], h = hh[0], n = nn[0];
#pragma unroll
      for (int m = 0; m < TM; ++m) v[m] = acc[0][m];
#pragma unroll
      for (int r = 1; r < R; ++r) {
#pragma unroll
        for (int m = 0; m < TM; ++m) v[m] = li == r ? acc[r][m] : v[m];
        h = li == r ? hh[r] : h;
        n = li == r ? nn[r] : n;
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < TM; ++m) acc[r][m] = 0;
      if (li >= R || h < 0) continue;
      const float ws = p.raw_f32 ? 1.0f : p.w_scale[h * p.ws_sb + static_cast<long long>(n) * p.ws_sn];
      const float bv = p.bias ? load_elem(p.bias, p.bias_dtype, h * p.bias_sb + n) : 0.0f;
#pragma unroll
      for (int m = 0; m < TM; ++m) {
        const long long oi = h * p.out_sb + m * p.out_sm + n;
        if (p.acc_out) p.acc_out[oi] = v[m];
        float f = __int2float_rn(v[m]);
        if (!p.raw_f32) {
          const float as = p.a_scale[h * p.as_sb + m * p.as_sm];
          f = __fmul_rn(__fmul_rn(f, as), ws);
          if (p.bias) f = __fadd_rn(f, bv);
        }
        store_elem(p.out, p.out_dtype, oi, f);
      }
    }
  }
}

template <int LPR, int KCH, int R, int D, int TM>
int launch_cfg(const WgParams& g, cudaStream_t stream) {
  constexpr int kRb = R * (32 / LPR);
  auto kern = w8a8_gemv_kernel<LPR, KCH, R, D, TM>;
  static int per_sm = 0;  // resident CTAs per SM (register-limited), looked up once
  if (per_sm == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, kWgThreads, 0) != cudaSuccess || v <= 0) v = 1;
    per_sm = v;
  }
  const int sms = sm_count();
  if (sms <= 0) return CB_ERR_CUDA;
  const long long blocks = (static_cast<long long>(g.rows) + kRb - 1) / kRb;
  const long long need = (blocks + kWgThreads / 32 - 1) / (kWgThreads / 32);
  const long long full = static_cast<long long>(sms) * per_sm;
  const long long grid = need < full ? need : full;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kWgThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, g));
}

template <int TM>
int launch_tm(const W8A8Launch& L, const WgParams& g, cudaStream_t stream) {
  if (L.K > 2048) return launch_cfg<32, 8, 1, kDepthLong, TM>(g, stream);
  if (L.K > 1024) return launch_cfg<32, 4, 2, kDepthShort, TM>(g, stream);
  if (L.K > 512) return launch_cfg<32, 2, 4, kDepthShort, TM>(g, stream);
  if (L.K > 256) return launch_cfg<32, 1, 8, kDepthShort, TM>(g, stream);
  if (L.K > 128) return launch_cfg<16, 1, 8, kDepthShort, TM>(g, stream);
  return launch_cfg<8, 1, 8, kDepthShort, TM>(g, stream);
}

}  // namespace

bool w8a8_gemv_eligible(const W8A8Launch& L) {
  // one or two tokens per batch entry, signed int8 operands, 16-byte aligned
  // rows, at most kGemvMaxWeightBytes (two tokens: kGemv2MaxWeightBytes) of
  // weights, which also keeps rows and items far below 2^31 for the 32-bit
  // bookkeeping
  return L.M >= 1 && L.M <= kW8GemvMaxTokens && !L.fp8 && !L.unsigned_operands && L.K % 16 == 0 &&
         L.batch * L.N * L.K <= (L.M == 1 ? kGemvMaxWeightBytes : kGemv2MaxWeightBytes) && aligned16(L.aq) &&
         aligned16(L.w) && L.w_sn % 16 == 0 &&
         (L.M == 1 || L.aq_sm % 16 == 0) && (L.batch == 1 || (L.w_sb % 16 == 0 && L.aq_sb % 16 == 0));
}

int launch_w8a8_gemv(const W8A8Launch& L, cudaStream_t stream) {
  // no split-K scratch: only the status word of the caller's workspace is used
  if (L.workspace == nullptr || L.workspace_bytes < kWsHeader) return CB_ERR_WORKSPACE;
  WgParams g = {};
  g.aq = L.aq;
  g.aq_sb = L.aq_sb;
  g.aq_sm = L.aq_sm;
  g.a_scale = L.a_scale;
  g.as_sb = L.as_sb;
  g.as_sm = L.scale_per_tensor_a ? 0 : 1;
  g.w = L.w;
  g.w_sb = L.w_sb;
  g.w_sn = L.w_sn;
  g.w_scale = L.w_scale;
  g.ws_sb = L.ws_sb;
  g.ws_sn = L.scale_per_tensor_w ? 0 : 1;
  g.out = L.out;
  g.out_dtype = L.out_dtype;
  g.out_sb = L.out_sb;
  g.out_sm = L.out_sm;
  g.acc_out = L.acc_out;
  g.raw_f32 = L.raw_f32;
  g.bias = L.raw_f32 ? nullptr : L.bias;
  g.bias_dtype = L.bias_dtype;
  g.bias_sb = L.bias_sb;
  g.N = static_cast<int>(L.N);
  g.K = static_cast<int>(L.K);
  g.rows = static_cast<int>(L.batch * L.N);
  g.status = static_cast<int*>(L.workspace);
  g.dbg_wait_ns = debug_wait_ns();
  // 4 KiB of weights per warp and item: one row slice of 4 KiB for long rows,
  // 8 rows x 512 B ... 32 rows x 128 B for short ones
  if (L.M == 1) return launch_tm<1>(L, g, stream);
  return launch_tm<2>(L, g, stream);
}

}  // namespace cb
