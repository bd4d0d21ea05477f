// Weight-stationary W4A16 GEMM for many token rows and small K (K <= 512) on sm_100a.
//
// Same math as w4a16_gemm.cu (kernel_batched_w4a16_simple,
// profiling/bench_l2_barrier.py:36-85, with g128 or per-channel scales):
//   out[b, m, n] = sum_k a[b, m, k] * q[b, k, n] * s[b, k / G, n]
// for problems where the token dimension is long and K is short, e.g. the MLA
// latent reconstruction (latents [16, b*L, 512] x per-head W_UK / W_UV
// [16, 512, 128], profiling/int4_batched_gemm.py:272-275). There the decode
// kernel would dequantize the same weight k-blocks once per 16..128-token tile.
//
// Work: the (panel, m-tile) pairs, a panel being the weights of one batch
// entry and 128 output columns (its K / 128 native 8 KiB tiles), split into
// contiguous ranges over the SMs. For each run of m-tiles of one panel a CTA
//   1. dequantizes the panel once into tensor memory as the MMA's A operand
//      (M = 128 output columns in the lanes, K along the columns as bf16/f16
//      pairs; g128 scales folded in): warps 2-5 read the packed tiles from
//      global memory and write them with tcgen05.st (warp w owns lanes
//      32 (w % 4) .. +31);
//   2. streams the activation m-tiles through a TMA ring of 128-token x 64-k
//      boxes that has all of shared memory (warp 0); warp 6 waits for each box
//      and hands it to warp 1 over a named barrier; warp 1 issues tcgen05.mma
//      kind::f16 with A = the panel in tensor memory, B = the token box
//      (N = 128 tokens), fp32 accumulators [128 columns x 128 tokens] in TMEM,
//      double-buffered across m-tiles;
//   3. warps 2-5 convert each finished accumulator (per-channel scale applied
//      in fp32 here when G >= K). The thread of lane n holds output column n
//      for the tile's 128 tokens; for 16-bit outputs (N % 8 == 0, 16-byte
//      aligned rows) each warp stages 16 tokens x its 32 columns in shared
//      memory and writes them back as 16-byte vectors of 8 columns, one eighth
//      of the store instructions of column-per-thread 2-byte stores (those
//      made the epilogue, at ~8K cycles per m-tile, the kernel's limit);
//      otherwise each thread stores its column element by element.
// Runs that start a new panel wait until the previous panel's MMAs are done
// (its last accumulator was drained) before overwriting it.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "cb_dequant.cuh"
#include "cb_gemm_common.cuh"
#include "cb_internal.h"
#include "cb_ptx.cuh"

namespace cb {
namespace {

constexpr int kBM = 128;               // tokens per m-tile (MMA N)
constexpr int kBN = 128;               // output columns per panel (MMA M)
constexpr int kBK = 128;               // k per weight tile
constexpr int kMaxKB = 4;              // resident panels up to K = 512
constexpr int kThreads = 7 * 32;       // producer, MMA, 4 dequant/epilogue warps, stage waiter
constexpr int kWaiterWarp = 6;
constexpr int kPanelBar = 2;           // named barrier: epilogue warps (arrive) -> MMA warp (sync)
constexpr int kPanelCount = 5 * 32;
constexpr int kStageBar = 3;           // named barrier: stage waiter <-> MMA warp
constexpr uint32_t kBoxBytes = kBM * 128;         // 128 tokens x 64 16-bit k
constexpr uint32_t kPackedTileBytes = kBN * kBK / 2;
constexpr uint32_t kPanelCol = 2 * kBM;           // after two accumulators of 128 fp32 columns
constexpr uint32_t kTmemCols = 512;               // + the panel: 64 columns per 128 k, K <= 512
constexpr int kMaxRingStages = 16;
constexpr uint32_t kStageTileBytes = 16 * 32 * 2;  // per epilogue warp: 16 tokens x 32 columns, 16-bit
constexpr uint32_t kEpiStageBytes = 4 * kStageTileBytes;

struct RParams {
  int M, N, K, H;
  int n_tiles, m_tiles, kb;  // kb = K / 128 (<= 4)
  int stages;
  long long items;            // panels * m_tiles
  const uint8_t* w;           // native tiles
  const void* scales;
  int scale_dtype;
  long long s_sb, s_sg;
  int kb_per_group;
  int per_channel;            // scale applied in the epilogue (group >= K)
  void* out;
  int out_dtype;
  long long out_sb, out_sm;
  int vec_out;                // 16-bit output, N % 8 == 0, 16-byte aligned rows: vector stores
  int* status;
};

__device__ __forceinline__ long long range_start(const RParams& p, int c) {
  return static_cast<long long>(c) * p.items / gridDim.x;
}

template <typename T, int OUT>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_resident_kernel(const __grid_constant__ CUtensorMap tmap_a, const RParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxRingStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxRingStages];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ int sh_issued, sh_consumed;
  volatile int* abort_ptr = &abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;  // stages x 16 KiB activation boxes
  uint16_t* epi_stage = reinterpret_cast<uint16_t*>(smem + p.stages * kBoxBytes);  // 4 x 1 KiB

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.stages;
  const long long i0 = range_start(p, blockIdx.x);
  const long long i1 = range_start(p, blockIdx.x + 1);
  const int boxes_per_tile = 2 * p.kb;

  if (threadIdx.x == 0) {
    pdl_launch_dependents();
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&drain_bar, 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    abort_flag = 0;
    sh_issued = sh_consumed = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
  }
  __syncwarp();
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      // activations stream once, or twice at about the same time when the CTAs of two
      // column panels of one batch entry walk the same m-tiles: keep them normal
      const uint64_t pol_a = policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      pdl_wait_primary();  // activations come from the preceding kernel
      for (long long i = i0; i < i1 && ok;) {
        const long long pan = i / p.m_tiles;
        const long long run_end = (pan + 1) * p.m_tiles < i1 ? (pan + 1) * p.m_tiles : i1;
        const int h = static_cast<int>(pan / p.n_tiles);
        for (; i < run_end && ok; ++i) {
          const int mt = static_cast<int>(i % p.m_tiles);
          for (int bx = 0; bx < boxes_per_tile; ++bx) {
            if (issued >= S && !mbar_wait(&empty_bar[stage], phase ^ 1u, abort_ptr, p.status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full_bar[stage], kBoxBytes);
            tma_load_3d(ring + stage * kBoxBytes, &tmap_a, &full_bar[stage], bx * 64, mt * kBM, h, pol_a);
            ++issued;
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      sh_issued = issued;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_f16_f32(kBN, kBM, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
    int stage = 0, consumed = 0, tiles = 0;
    bool bad = false, stop = false;
    for (long long i = i0; i < i1 && !stop;) {
      const long long pan = i / p.m_tiles;
      const long long run_end = (pan + 1) * p.m_tiles < i1 ? (pan + 1) * p.m_tiles : i1;
      named_bar_sync(kPanelBar, kPanelCount);  // the panel for this run is in tensor memory
      for (; i < run_end && !stop; ++i) {
        const int acc = tiles & 1;
        if (lane == 0 && !bad && tiles >= 2)
          bad = !mbar_wait(&acc_empty[acc], static_cast<uint32_t>(((tiles >> 1) - 1) & 1), abort_ptr, p.status);
        const uint32_t d = tmem_base + acc * kBM;
        for (int bx = 0; bx < boxes_per_tile; ++bx) {
          if (named_bar_or(kStageBar, 64, bad)) {
            stop = true;
            break;
          }
          if (lane == 0) {
            tc_fence_after();
            // box bx = k 64 bx .. 64 bx + 63: panel columns 32 bx .. (two k per column)
            const uint32_t b0 = smem_u32(ring + stage * kBoxBytes);
            const uint32_t a0 = tmem_base + kPanelCol + 32 * bx;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ts(d, a0 + kk * 8, smem_desc_sw128(b0 + kk * 32), idesc, (bx == 0 && kk == 0) ? 0u : 1u);
            mma_commit(&empty_bar[stage]);
          }
          __syncwarp();
          ++consumed;
          if (++stage == S) stage = 0;
        }
        if (stop) break;
        if (lane == 0) mma_commit(&acc_full[acc]);
        __syncwarp();
        ++tiles;
      }
    }
    if (lane == 0) {
      sh_consumed = consumed;
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, p.status);
    }
    // every commit arrival lane 0 issued must land before the CTA exits; one
    // lane per barrier so the waits overlap
    consumed = __shfl_sync(0xffffffffu, consumed, 0);
    tiles = __shfl_sync(0xffffffffu, tiles, 0);
    {
      const int j = consumed - 1 - lane;
      if (lane < S && j >= 0) mbar_wait(&empty_bar[j % S], static_cast<uint32_t>((j / S) & 1), nullptr, p.status);
      const int t = tiles - 1 - (lane - 30);
      if (lane >= 30 && t >= 0) mbar_wait(&acc_full[t & 1], static_cast<uint32_t>((t >> 1) & 1), nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == kWaiterWarp) {
    // ---------------- stage waiter ----------------
    int stage = 0;
    uint32_t phase = 0;
    const long long total = (i1 - i0) * boxes_per_tile;
    for (long long j = 0; j < total; ++j) {
      bool bad = false;
      if (lane == 0) bad = !mbar_wait(&full_bar[stage], phase, abort_ptr, p.status);
      bad = __shfl_sync(0xffffffffu, bad, 0);
      if (named_bar_or(kStageBar, 64, bad)) break;
      if (++stage == S) {
        stage = 0;
        phase ^= 1u;
      }
    }
    __syncwarp();
  } else {
    // ---------------- dequant + epilogue (warps 2-5) ----------------
    // Control flow is uniform: after a failed wait the work is skipped but every
    // arrival still happens.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane = panel row = output column within the panel
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    int tiles = 0;
    for (long long i = i0; i < i1;) {
      const long long pan = i / p.m_tiles;
      const long long run_end = (pan + 1) * p.m_tiles < i1 ? (pan + 1) * p.m_tiles : i1;
      const int h = static_cast<int>(pan / p.n_tiles);
      const int nt = static_cast<int>(pan % p.n_tiles);
      const int n = nt * kBN + row;
      // 1. dequantize the panel into tensor memory (the previous run's MMAs
      //    are done: its last accumulator was drained below before this point)
      // All of the row's packed bytes (K <= 512: at most 4 x 64 bytes) and group
      // scales are loaded before the first tensor-memory store: the stores'
      // ordering would otherwise keep each k-tile's loads behind the previous
      // k-tile's, one global round trip per k-tile before the first MMA.
      float col_scale = 1.0f;
      if (p.per_channel && n < p.N) col_scale = load_elem(p.scales, p.scale_dtype, h * p.s_sb + n);
      uint4 raw[kMaxKB][4];
      float svs[kMaxKB];
      const int swz = (row >> 1) & 3;
#pragma unroll
      for (int kb = 0; kb < kMaxKB; ++kb) {
        svs[kb] = 1.0f;
        if (kb < p.kb) {
          if (!p.per_channel && n < p.N)
            svs[kb] = load_elem(p.scales, p.scale_dtype, h * p.s_sb + (kb / p.kb_per_group) * p.s_sg + n);
          const uint4* wrow = reinterpret_cast<const uint4*>(p.w + (pan * p.kb + kb) * kPackedTileBytes + row * 64);
#pragma unroll
          for (int c = 0; c < 4; ++c) raw[kb][c] = __ldg(wrow + (c ^ swz));
        }
      }
      const typename Dq<T>::T2 bias = Dq<T>::bias();
#pragma unroll
      for (int kb = 0; kb < kMaxKB; ++kb) {
        if (kb < p.kb) {
          const typename Dq<T>::T2 sc = Dq<T>::from_f(svs[kb]);
          uint32_t lo[32], hi[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t words[4] = {raw[kb][c].x, raw[kb][c].y, raw[kb][c].z, raw[kb][c].w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
#pragma unroll
              for (int pi = 0; pi < 4; ++pi) {
                const uint32_t v = dq_pair<T>(words[wi], 4 * pi, bias, sc, !p.per_channel);
                const int idx = c * 16 + wi * 4 + pi;  // pair index: k = 2 idx, 2 idx + 1
                if (idx < 32)
                  lo[idx] = v;
                else
                  hi[idx - 32] = v;
              }
          }
          tmem_st32(tmem_base + lane_off + kPanelCol + 64 * kb, lo);
          tmem_st32(tmem_base + lane_off + kPanelCol + 64 * kb + 32, hi);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      named_bar_arrive(kPanelBar, kPanelCount);
      // 2. drain the accumulators of this run's m-tiles. The panel above is
      //    weights only, so it was built while the preceding kernel finished;
      //    the output may still be read by that kernel until this wait.
      pdl_wait_primary();
      for (; i < run_end; ++i, ++tiles) {
        const int acc = tiles & 1;
        const int mt = static_cast<int>(i % p.m_tiles);
        const bool ready = mbar_wait(&acc_full[acc], static_cast<uint32_t>((tiles >> 1) & 1), abort_ptr, p.status);
        const bool live = __all_sync(0xffffffffu, ready);
        tc_fence_after();
        if (live && OUT != CB_DTYPE_F32 && p.vec_out) {  // warp-uniform (tcgen05.ld is warp-wide)
          uint16_t* stg = epi_stage + (warp - 2) * (kStageTileBytes / 2);
          const int q8 = lane & 3;  // 8-column chunk of this warp's 32 columns
          const int n8 = nt * kBN + quarter * 32 + q8 * 8;
          uint16_t* out16 = static_cast<uint16_t*>(p.out) + h * p.out_sb + n8;
#pragma unroll 1
          for (int c = 0; c < kBM / 16; ++c) {
            uint32_t rr[16];
            __syncwarp();
            tmem_ld16(tmem_base + lane_off + acc * kBM + c * 16, rr);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v = __uint_as_float(rr[j]);
              if (p.per_channel) v = __fmul_rn(v, col_scale);
              const uint16_t b = OUT == CB_DTYPE_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                      : __half_as_ushort(__float2half_rn(v));
              stg[j * 32 + lane] = b;  // token j, column lane
            }
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const int jt = (lane >> 2) + 8 * r;
              const int m = mt * kBM + c * 16 + jt;
              const uint4 v = *reinterpret_cast<const uint4*>(stg + jt * 32 + q8 * 8);
              if (m < p.M && n8 < p.N) *reinterpret_cast<uint4*>(out16 + static_cast<long long>(m) * p.out_sm) = v;
            }
          }
          __syncwarp();
        } else if (live) {  // warp-uniform: every lane takes part in the warp-wide tcgen05.ld
          const long long base = h * p.out_sb + n;
#pragma unroll 1
          for (int c = 0; c < kBM / 16; ++c) {
            uint32_t rr[16];
            __syncwarp();
            tmem_ld16(tmem_base + lane_off + acc * kBM + c * 16, rr);
            tmem_ld_wait();
            if (n < p.N) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = mt * kBM + c * 16 + j;
                if (m < p.M) {
                  float v = __uint_as_float(rr[j]);
                  if (p.per_channel) v = __fmul_rn(v, col_scale);
                  store_elem(p.out, OUT, base + static_cast<long long>(m) * p.out_sm, v);
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
      }
    }
  }

  __syncthreads();
  if (warp == 0) {
    if (lane == 0 && abort_flag) {
      // copies issued but never consumed must land before the CTA exits
      for (int j = sh_consumed; j < sh_issued; ++j) mbar_wait(&full_bar[j % S], (j / S) & 1, nullptr, p.status);
    }
    __syncwarp();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <typename T, int OUT>
int launch_typed(const W4A16Launch& L, cudaStream_t stream, const RParams& prm, int grid) {
  CUtensorMap ta;
  const CUtensorMapDataType dt =
      (L.a_dtype == CB_DTYPE_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int st = encode_tmap_3d(&ta, dt, L.a, static_cast<uint64_t>(L.K), static_cast<uint64_t>(L.M),
                          static_cast<uint64_t>(L.batch), L.a_sm, L.a_sb, 64, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CB_OK) return st;
  const size_t smem = static_cast<size_t>(prm.stages) * kBoxBytes + kEpiStageBytes + 1024;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < smem) {
    cudaError_t e = cudaFuncSetAttribute(w4a16_resident_kernel<T, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return CB_ERR_CUDA;
    configured_dev = dev;
    configured_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, w4a16_resident_kernel<T, OUT>, ta, prm));
}

template <typename T>
int launch_out(const W4A16Launch& L, cudaStream_t stream, const RParams& prm, int grid) {
  switch (L.out_dtype) {
    case CB_DTYPE_BF16:
      return launch_typed<T, CB_DTYPE_BF16>(L, stream, prm, grid);
    case CB_DTYPE_F16:
      return launch_typed<T, CB_DTYPE_F16>(L, stream, prm, grid);
    default:
      return launch_typed<T, CB_DTYPE_F32>(L, stream, prm, grid);
  }
}

}  // namespace

bool w4a16_resident_eligible(const W4A16Launch& L) {
  return L.K % kBK == 0 && L.K / kBK <= kMaxKB && L.M > kBM;
}

int launch_w4a16_resident(const W4A16Launch& L, cudaStream_t stream) {
  RParams p = {};
  p.M = static_cast<int>(L.M);
  p.N = static_cast<int>(L.N);
  p.K = static_cast<int>(L.K);
  p.H = static_cast<int>(L.batch);
  p.kb = static_cast<int>(L.K / kBK);
  p.n_tiles = static_cast<int>((L.N + kBN - 1) / kBN);
  p.m_tiles = static_cast<int>((L.M + kBM - 1) / kBM);
  p.items = static_cast<long long>(p.H) * p.n_tiles * p.m_tiles;
  const int sms = sm_count();
  if (sms <= 0) return CB_ERR_CUDA;
  const int grid = static_cast<int>(p.items < sms ? p.items : sms);
  // ring: ~220 KiB of shared memory (the panel lives in tensor memory)
  int stages = static_cast<int>((220u * 1024u - kEpiStageBytes) / kBoxBytes);
  if (stages > kMaxRingStages) stages = kMaxRingStages;
  if (stages < 2) return CB_ERR_UNSUPPORTED;
  p.stages = stages;
  p.w = L.w;
  p.scales = L.scales;
  p.scale_dtype = L.scale_dtype;
  p.s_sb = L.s_sb;
  p.s_sg = L.s_sg;
  p.per_channel = L.group_size >= L.K ? 1 : 0;
  p.kb_per_group = static_cast<int>(L.group_size / kBK) > 0 ? static_cast<int>(L.group_size / kBK) : 1;
  p.out = L.out;
  p.out_dtype = L.out_dtype;
  p.out_sb = L.out_sb;
  p.out_sm = L.out_sm;
  p.vec_out = (L.out_dtype != CB_DTYPE_F32 && L.N % 8 == 0 && aligned16(L.out) && L.out_sm % 8 == 0 &&
               (L.batch == 1 || L.out_sb % 8 == 0))
                  ? 1
                  : 0;
  if (L.workspace == nullptr || L.workspace_bytes < kWsHeader) return CB_ERR_WORKSPACE;
  p.status = carve_workspace(L.workspace, grid).status;
  if (L.a_dtype == CB_DTYPE_BF16) return launch_out<__nv_bfloat16>(L, stream, p, grid);
  return launch_out<__half>(L, stream, p, grid);
}

}  // namespace cb
