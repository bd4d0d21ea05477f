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
// Longest row quantized inside the GEMV (FUSE, one token). Every CTA
// quantizes the whole row while its first weight items are in flight; for long
// rows that work (two passes over the row, one IEEE division per element)
// delays the weight stream more than a separate quantizer launch costs, whose
// dependent GEMM starts streaming while it runs: K = 256 2.7 vs 3.9 us, K =
// 1024 3.2 vs 3.7 us, K = 4096 7.2 vs 7.3 us, K = 8192 17.6 vs 15.4 us.
constexpr int kFuseMaxRowBytes = 1024;

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
  // FUSE: the 16-bit activation rows (batch of one) quantized by every CTA
  const void* a;
  int a_dtype;
  long long a_sm;
  int8_t* q_out;  // the quantized rows and their scales, written by CTA 0
  float* s_out;
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

__device__ __forceinline__ float act16_f32(uint32_t half_bits, int dtype) {
  return dtype == CB_DTYPE_BF16 ? __uint_as_float(half_bits << 16)
                                : __half2float(__ushort_as_half(static_cast<unsigned short>(half_bits)));
}

// Per-token int8 quantization with _quant_act_kernel's arithmetic
// (profiling/w8a8/w8a8_bmm.py:30-41), the same operations as act_quant.cu:
// scale = max(amax / 127, 1e-8), q = trunc(a / scale + 0.5 sign(a)).
__device__ __forceinline__ uint32_t quant4(float x0, float x1, float x2, float x3, float sc) {
  auto q1 = [sc](float x) {
    const float y = __fadd_rn(__fdiv_rn(x, sc), x >= 0.0f ? 0.5f : -0.5f);
    return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(__float2int_rz(y))));
  };
  return q1(x0) | (q1(x1) << 8) | (q1(x2) << 16) | (q1(x3) << 24);
}

// TM tokens (1 or 2) share each weight chunk. FUSE (one token of a single
// GEMM, short rows): every CTA quantizes the 16-bit token row itself into
// shared memory after the dependency wait, while its first weight items are in
// flight, instead of a separate quantizer launch; CTA 0 also stores q and the
// scale.
template <int LPR, int KCH, int R, int D, int TM, bool FUSE>
__global__ void __launch_bounds__(kWgThreads) w8a8_gemv_kernel(const WgParams p) {
  extern __shared__ __align__(16) int8_t gv_q[];  // FUSE: [TM][K] quantized rows
  __shared__ float gv_red[kWgThreads / 32][TM];
  __shared__ float gv_scale[TM];
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
  if constexpr (FUSE) {
    // amax of each row (16-byte vectors, K % 8 == 0), then quantize from L1
    const int nv = p.K / 8;
    const int lane0 = threadIdx.x & 31, wq = threadIdx.x >> 5;
#pragma unroll
    for (int m = 0; m < TM; ++m) {
      const uint4* av = reinterpret_cast<const uint4*>(static_cast<const char*>(p.a) + m * p.a_sm * 2);
      float amax = 0.0f;
#pragma unroll 8
      for (int v = threadIdx.x; v < nv; v += kWgThreads) {
        const uint4 u = __ldg(av + v);
        const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          amax = fmaxf(amax, fmaxf(fabsf(act16_f32(wd[j] & 0xFFFFu, p.a_dtype)), fabsf(act16_f32(wd[j] >> 16, p.a_dtype))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane0 == 0) gv_red[wq][m] = amax;
    }
    __syncthreads();
    if (threadIdx.x < TM) {
      float amax = gv_red[0][threadIdx.x];
#pragma unroll
      for (int w = 1; w < kWgThreads / 32; ++w) amax = fmaxf(amax, gv_red[w][threadIdx.x]);
      const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
      gv_scale[threadIdx.x] = sc;
      if (blockIdx.x == 0) p.s_out[threadIdx.x] = sc;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < TM; ++m) {
      const uint4* av = reinterpret_cast<const uint4*>(static_cast<const char*>(p.a) + m * p.a_sm * 2);
      const float sc = gv_scale[m];
#pragma unroll 8
      for (int v = threadIdx.x; v < nv; v += kWgThreads) {
        const uint4 u = __ldg(av + v);
        uint2 qv;
        qv.x = quant4(act16_f32(u.x & 0xFFFFu, p.a_dtype), act16_f32(u.x >> 16, p.a_dtype),
                      act16_f32(u.y & 0xFFFFu, p.a_dtype), act16_f32(u.y >> 16, p.a_dtype), sc);
        qv.y = quant4(act16_f32(u.z & 0xFFFFu, p.a_dtype), act16_f32(u.z >> 16, p.a_dtype),
                      act16_f32(u.w & 0xFFFFu, p.a_dtype), act16_f32(u.w >> 16, p.a_dtype), sc);
        *reinterpret_cast<uint2*>(gv_q + m * p.K + v * 8) = qv;
        if (blockIdx.x == 0) *reinterpret_cast<uint2*>(p.q_out + m * p.aq_sm + v * 8) = qv;
      }
    }
    __syncthreads();
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
            uint4 a = make_uint4(0u, 0u, 0u, 0u);
            if (hh[r] >= 0 && k < p.K)
              a = FUSE ? *reinterpret_cast<const uint4*>(gv_q + m * p.K + k)
                       : __ldg(reinterpret_cast<const uint4*>(ar + m * p.aq_sm + k));
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
          const float as = FUSE ? gv_scale[m] : p.a_scale[h * p.as_sb + m * p.as_sm];
          f = __fmul_rn(__fmul_rn(f, as), ws);
          if (p.bias) f = __fadd_rn(f, bv);
        }
        store_elem(p.out, p.out_dtype, oi, f);
      }
    }
  }
}

template <int LPR, int KCH, int R, int D, int TM, bool FUSE>
int launch_cfg(const WgParams& g, cudaStream_t stream) {
  constexpr int kRb = R * (32 / LPR);
  auto kern = w8a8_gemv_kernel<LPR, KCH, R, D, TM, FUSE>;
  const size_t smem = FUSE ? static_cast<size_t>(TM) * g.K : 0;
  static int per_sm = 0;  // resident CTAs per SM, looked up once (at the largest fused row)
  if (per_sm == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, kWgThreads, FUSE ? kFuseMaxRowBytes : 0) !=
            cudaSuccess ||
        v <= 0)
      v = 1;
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
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, g));
}

template <int TM, bool FUSE>
int launch_tm(const W8A8Launch& L, const WgParams& g, cudaStream_t stream) {
  if (L.K > 2048) return launch_cfg<32, 8, 1, kDepthLong, TM, FUSE>(g, stream);
  if (L.K > 1024) return launch_cfg<32, 4, 2, kDepthShort, TM, FUSE>(g, stream);
  if (L.K > 512) return launch_cfg<32, 2, 4, kDepthShort, TM, FUSE>(g, stream);
  if (L.K > 256) return launch_cfg<32, 1, 8, kDepthShort, TM, FUSE>(g, stream);
  if (L.K > 128) return launch_cfg<16, 1, 8, kDepthShort, TM, FUSE>(g, stream);
  return launch_cfg<8, 1, 8, kDepthShort, TM, FUSE>(g, stream);
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

namespace {
WgParams gemv_params(const W8A8Launch& L) {
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
  return g;
}
}  // namespace

int launch_w8a8_gemv(const W8A8Launch& L, cudaStream_t stream) {
  // no split-K scratch: only the status word of the caller's workspace is used
  if (L.workspace == nullptr || L.workspace_bytes < kWsHeader) return CB_ERR_WORKSPACE;
  const WgParams g = gemv_params(L);
  // 4 KiB of weights per warp and item: one row slice of 4 KiB for long rows,
  // 8 rows x 512 B ... 32 rows x 128 B for short ones
  if (L.M == 1) return launch_tm<1, false>(L, g, stream);
  return launch_tm<2, false>(L, g, stream);
}

bool w8a8_gemv_dynamic_eligible(const W8A8Launch& L, const void* a, int a_dtype, int64_t a_sm) {
  // one token of a single GEMM, a 16-bit row read as 16-byte vectors and at
  // most kFuseMaxRowBytes long; L.aq / L.a_scale are the q and scale outputs
  (void)a_sm;
  return L.batch == 1 && L.M == 1 && w8a8_gemv_eligible(L) &&
         (a_dtype == CB_DTYPE_BF16 || a_dtype == CB_DTYPE_F16) && L.K % 8 == 0 && aligned16(a) &&
         L.K <= kFuseMaxRowBytes && !L.scale_per_tensor_a && !L.raw_f32;
}

int launch_w8a8_gemv_dynamic(const W8A8Launch& L, const void* a, int a_dtype, int64_t a_sm, cudaStream_t stream) {
  if (L.workspace == nullptr || L.workspace_bytes < kWsHeader) return CB_ERR_WORKSPACE;
  WgParams g = gemv_params(L);
  g.a = a;
  g.a_dtype = a_dtype;
  g.a_sm = a_sm;
  g.q_out = const_cast<int8_t*>(L.aq);
  g.s_out = const_cast<float*>(L.a_scale);
  return launch_tm<1, true>(L, g, stream);
}

}  // namespace cb
