// NVFP4 (W4A4, e2m1 values with ue4m3 scales per 16 elements) for sm_100a:
// the matched-precision path the reference measures through vLLM on B200
// (profiling/cuda_validation/bench_moe_nvfp4_native.py:97-108, 140-160:
// `scaled_fp4_quant` + `run_cutlass_moe_fp4`), as a dense GEMM on the tensor
// cores' native FP4 path (tcgen05.mma kind::mxf4nvf4, block scales in TMEM).
//
// Formats are vLLM's (vllm 0.22.0, vllm/model_executor/layers/quantization/
// utils/nvfp4_emulation_utils.py:328-453, nvfp4_utils.py:13-60), so tensors
// quantized by either library work with the other's GEMM:
//   values  uint8 [rows, K/2], element 2i in the low nibble, 2i+1 in the high;
//           nibble = sign << 3 | index into {0, 0.5, 1, 1.5, 2, 3, 4, 6}
//   scales  e4m3 bytes in 512-byte atoms of 128 rows x 4 scale columns:
//           offset(r, c) = ((r / 128) * ceil(C / 4) + c / 4) * 512
//                          + (r % 32) * 16 + ((r % 128) / 32) * 4 + c % 4
//           (C = K / 16 scale columns; rows padded to 128, columns to 4)
//   value   x ~= e2m1 * e4m3 / global_scale
//
// cb_nvfp4_quantize restates ref_nvfp4_quant (nvfp4_emulation_utils.py:439-453):
//   s   = e4m3(clamp(gs * (amax_block * f32(1/6)), +-448))        (round to nearest even)
//   o   = 1 / (f32(s) * (1 / gs))                                  (IEEE fp32 divisions; 1e-8 for s = 0)
//   q_i = e2m1(clamp(x_i * o, +-6))                                (round to nearest even)
// cb_nvfp4_gemm computes out[m, n] = alpha * sum_k A[m, k] * B[n, k] with A the
// activations [M, K] and B the weights [N, K], as vLLM's cutlass_scaled_fp4_mm
// (a, b, a_sf, b_sf, alpha, out_dtype). Swap-AB as in the int8 kernel: the
// weight tile is the MMA's M = 128 operand, the token tile its N operand.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "cb_dequant.cuh"
#include "cb_gemm_common.cuh"
#include "cb_internal.h"
#include "cb_ptx.cuh"

namespace cb {
namespace {

// ------------------------------------------------------------------------
// Quantizer
// ------------------------------------------------------------------------
constexpr int kQThreads = 256;

// Element j (0..7) of 8 packed 16-bit activations as fp32.
template <bool kBf16>
__device__ __forceinline__ float act_elem(const uint4& u, int j) {
  const uint32_t w = j < 2 ? u.x : j < 4 ? u.y : j < 6 ? u.z : u.w;
  const uint32_t h = (j & 1) ? (w >> 16) : (w & 0xffffu);
  if constexpr (kBf16) return __uint_as_float(h << 16);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

__host__ __device__ __forceinline__ long long sf_offset(long long r, long long c, long long c_tiles) {
  return ((r >> 7) * c_tiles + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

// e2m1 nibble of v (round to nearest even on {0, 0.5, 1, 1.5, 2, 3, 4, 6},
// saturating at 6; the sign bit follows v's sign, so -0 rounds to 0x8).
__device__ __forceinline__ uint32_t e2m1_nibble(float v) {
  const uint32_t sign = (__float_as_uint(v) >> 31) << 3;
  const float a = fabsf(v);
  uint32_t m;
  if (a <= 0.25f) m = 0;
  else if (a < 0.75f) m = 1;
  else if (a <= 1.25f) m = 2;
  else if (a < 1.75f) m = 3;
  else if (a <= 2.5f) m = 4;
  else if (a < 3.5f) m = 5;
  else if (a <= 5.0f) m = 6;
  else m = 7;
  return sign | m;
}

template <bool kBf16>
__global__ void __launch_bounds__(kQThreads) nvfp4_quant_kernel(const uint16_t* __restrict__ x, long long x_sm,
                                                                  int rows, int K, const float* __restrict__ gs_ptr,
                                                                  uint8_t* __restrict__ q, long long q_sm,
                                                                  uint8_t* __restrict__ sf, int rows_pad,
                                                                  int c_pad) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int C = K / 16;
  const long long c_tiles = c_pad / 4;
  const long long total = static_cast<long long>(rows_pad) * c_pad;  // every scale byte, padding included
  const float gs = *gs_ptr;
  const float rgs = __fdiv_rn(1.0f, gs + (gs == 0.0f ? 1e8f : 0.0f));
  const float r6 = 1.0f / 6.0f;  // the fp32 value of 1/6 (rounded at compile time)
  for (long long i = blockIdx.x * static_cast<long long>(kQThreads) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * kQThreads) {
    const int r = static_cast<int>(i / c_pad);
    const int c = static_cast<int>(i - static_cast<long long>(r) * c_pad);
    if (r >= rows || c >= C) {
      sf[sf_offset(r, c, c_tiles)] = 0;
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(r) * x_sm + c * 16);
    const uint4 u0 = src[0], u1 = src[1];
    float v[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = act_elem<kBf16>(u0, j);
      v[8 + j] = act_elem<kBf16>(u1, j);
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
    float s = __fmul_rn(gs, __fmul_rn(amax, r6));
    s = fminf(fmaxf(s, -448.0f), 448.0f);
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(s, __NV_SATFINITE, __NV_E4M3);
    const float sq = __half2float(__half(__nv_cvt_fp8_to_halfraw(s8, __NV_E4M3)));
    const float t = __fmul_rn(sq, rgs);
    const float o = __fdiv_rn(1.0f, t + (t == 0.0f ? 1e8f : 0.0f));
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float y = fminf(fmaxf(__fmul_rn(v[j], o), -6.0f), 6.0f);
      w[j >> 3] |= e2m1_nibble(y) << ((j & 7) * 4);
    }
    *reinterpret_cast<uint2*>(q + static_cast<long long>(r) * q_sm + c * 8) = make_uint2(w[0], w[1]);
    sf[sf_offset(r, c, c_tiles)] = static_cast<uint8_t>(s8);
  }
}

// ------------------------------------------------------------------------
// GEMM
// ------------------------------------------------------------------------
constexpr int kBlockN = 128;       // weight rows per tile (MMA M)
constexpr int kStageK = 256;       // k per stage: 128 packed bytes per row (one 128-byte swizzle row)
constexpr int kStageRowBytes = 128;
constexpr int kThreads = 352;
constexpr int kWaiterWarp = 6;
constexpr int kSfWarp0 = 7;  // warps 7..10 write the block scales into tensor memory
constexpr int kHandoffBar = 2;
constexpr uint32_t kWTileBytes = kBlockN * kStageRowBytes;  // 16 KiB
constexpr uint32_t kSfAtom = 512;
constexpr uint32_t kSfStage = 4 * kSfAtom;  // 4 atoms = 256 k of 128 rows

struct Params {
  int M, N, K;
  int n_tiles, m_tiles, kb_per_tile;
  int stages;
  StreamK sk;
  const uint8_t* sfw;  // weight scales (swizzled), rows N
  const uint8_t* sfx;  // activation scales (swizzled), rows M
  int k_atoms;         // K / 64: scale atoms along K
  const float* alpha;
  void* out;
  int out_dtype;
  long long out_sm;
  int vec_out;  // 16-bit output, N % 8 == 0, 16-byte aligned rows: vector stores
  float* partials;  // [grid][2][TN][128]
  int* counters;
  int* status;
};

__device__ __forceinline__ void decode_tile(const Params& p, long long tile, int& nt, int& mt) {
  int h;
  split_tile(tile, p.m_tiles, p.n_tiles, h, nt, mt);  // one batch entry: h = 0
}

template <int TN>
__device__ __forceinline__ void sum_published(const Params& p, int c_lo, int c_hi, int c, int row, float (&v)[16]) {
  for (int cc = c_lo; cc <= c_hi; ++cc) {
    const float* src = p.partials + static_cast<long long>(cc * 2) * TN * kBlockN + (c * 16) * kBlockN + row;
    float part[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) part[j] = __ldcg(src + j * kBlockN);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], part[j]);
  }
}

// emit_row for 16-bit outputs through shared memory: the warp stages its 32
// columns x 16 tokens (thread = column) and stores them back as 16-byte vectors
// of 8 columns, one eighth of the store instructions. Same arithmetic and
// rounding as emit_row.
template <int OUT_BF16>
__device__ __forceinline__ void emit_chunk_vec(const Params& p, int n_warp0, int lane, int m0, int t0,
                                               const float (&v)[16], float alpha, uint16_t* stg) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float f = __fmul_rn(v[j], alpha);
    stg[j * 32 + lane] =
        OUT_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(f)) : __half_as_ushort(__float2half_rn(f));
  }
  __syncwarp();
  const int q8 = lane & 3;
  const int n8 = n_warp0 + q8 * 8;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int jt = (lane >> 2) + 8 * r;
    const int m = m0 + t0 + jt;
    const uint4 val = *reinterpret_cast<const uint4*>(stg + jt * 32 + q8 * 8);
    if (m < p.M && n8 < p.N)
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + static_cast<long long>(m) * p.out_sm + n8) = val;
  }
  __syncwarp();
}

__device__ __forceinline__ void emit_row(const Params& p, int n, int m0, int t0, const float (&v)[16], float alpha) {
  if (n >= p.N) return;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + t0 + j;
    if (m < p.M) store_elem(p.out, p.out_dtype, static_cast<long long>(m) * p.out_sm + n, __fmul_rn(v[j], alpha));
  }
}

template <int TN>
__global__ void __launch_bounds__(kThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                      const Params p) {
  constexpr uint32_t kXTileBytes = TN * kStageRowBytes;
  constexpr uint32_t kAccCols = TN < 32 ? 32 : TN;
  // one scale buffer of 32 columns per ring stage (16 weight + 16 activation:
  // 4 MMAs x 4), after the accumulator; the launcher keeps kAccCols + 32 S <= 512
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kSfCol0 = kAccCols;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];   // weight + activation tiles landed
  __shared__ __align__(8) uint64_t sfdat_bar[kMaxStages];  // the stage's scale atoms landed
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t tfull_bar, tempty_bar, drain_bar;
  __shared__ __align__(8) uint64_t sf_full[kMaxStages];  // the stage's scales are in tensor memory
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ long long sh_pend_tile;
  __shared__ int sh_issued, sh_consumed, sh_is_last;
  volatile int* abort_ptr = &abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint8_t* smem_w = smem;
  uint8_t* smem_x = smem + S * kWTileBytes;
  uint8_t* smem_sfw = smem_x + S * kXTileBytes;
  uint8_t* smem_sfx = smem_sfw + S * kSfStage;
  // per epilogue warp: 16 tokens x 32 columns of 16-bit output (vector-store staging)
  uint16_t* epi_stage = reinterpret_cast<uint16_t*>(smem_sfx + S * kSfStage);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = p.kb_per_tile;
  const long long g0 = p.sk.start(blockIdx.x);
  const long long g1 = p.sk.start(blockIdx.x + 1);

  if (threadIdx.x == 0) {
    pdl_launch_dependents();
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&sfdat_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar, 1);
    mbar_init(&tempty_bar, 4);
    mbar_init(&drain_bar, 1);
    for (int b = 0; b < S; ++b) mbar_init(&sf_full[b], 4);
    abort_flag = 0;
    sh_issued = 0;
    sh_consumed = 0;
    sh_is_last = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  __syncwarp();
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base_sh;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // Weights and their scales are static; activations and their scales come
    // from the preceding kernel. The first ring pass of weights goes out
    // before griddepcontrol.wait.
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const long long nmine = g1 - g0;
    const int pro = static_cast<int>(nmine < S ? nmine : S);
    // Scale atoms go out ahead of their stage's tiles (their own barrier), so
    // the scale writers can place them in tensor memory before the tiles land.
    if (lane < pro) {
      KCursor c;
      c.seek(p, g0 + lane);
      const int atoms = min(4, p.k_atoms - 4 * c.kb);
      mbar_arrive_expect_tx(&sfdat_bar[lane], 2u * atoms * kSfAtom);
      bulk_copy_g2s(smem_sfw + lane * kSfStage,
                    p.sfw + (static_cast<long long>(c.nt) * p.k_atoms + 4 * c.kb) * kSfAtom, atoms * kSfAtom,
                    &sfdat_bar[lane], pol_w);
      mbar_arrive_expect_tx(&full_bar[lane], kWTileBytes + kXTileBytes);
      tma_load_3d(smem_w + lane * kWTileBytes, &tmap_w, &full_bar[lane], c.kb * kStageRowBytes, c.nt * kBlockN, 0,
                  pol_w);
    }
    __syncwarp();
    pdl_wait_primary();
    if (lane < pro) {
      KCursor c;
      c.seek(p, g0 + lane);
      const int atoms = min(4, p.k_atoms - 4 * c.kb);
      bulk_copy_g2s(smem_sfx + lane * kSfStage,
                    p.sfx + (static_cast<long long>((c.mt * TN) >> 7) * p.k_atoms + 4 * c.kb) * kSfAtom,
                    atoms * kSfAtom, &sfdat_bar[lane], pol_x);
      tma_load_3d(smem_x + lane * kXTileBytes, &tmap_x, &full_bar[lane], c.kb * kStageRowBytes, c.mt * TN, 0, pol_x);
    }
    __syncwarp();
    if (lane == 0) {
      KCursor cur;
      cur.seek(p, g0 + pro);
      int issued = pro;
      int stage = pro % S;
      uint32_t phase = (pro == S) ? 1u : 0u;
      for (long long g = g0 + pro; g < g1; ++g) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_ptr, p.status)) break;
        const int atoms = min(4, p.k_atoms - 4 * cur.kb);
        mbar_arrive_expect_tx(&sfdat_bar[stage], 2u * atoms * kSfAtom);
        bulk_copy_g2s(smem_sfw + stage * kSfStage,
                      p.sfw + (static_cast<long long>(cur.nt) * p.k_atoms + 4 * cur.kb) * kSfAtom, atoms * kSfAtom,
                      &sfdat_bar[stage], pol_w);
        bulk_copy_g2s(smem_sfx + stage * kSfStage,
                      p.sfx + (static_cast<long long>((cur.mt * TN) >> 7) * p.k_atoms + 4 * cur.kb) * kSfAtom,
                      atoms * kSfAtom, &sfdat_bar[stage], pol_x);
        mbar_arrive_expect_tx(&full_bar[stage], kWTileBytes + kXTileBytes);
        tma_load_3d(smem_w + stage * kWTileBytes, &tmap_w, &full_bar[stage], cur.kb * kStageRowBytes,
                    cur.nt * kBlockN, 0, pol_w);
        tma_load_3d(smem_x + stage * kXTileBytes, &tmap_x, &full_bar[stage], cur.kb * kStageRowBytes, cur.mt * TN, 0,
                    pol_x);
        cur.next(p);
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      sh_issued = issued;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // One K = 64 MMA per scale atom of the stage; the scales are already in
    // tensor memory (the stage's buffer, written by warps 7..10).
    const uint32_t idesc = idesc_nvf4(kBlockN, TN);
    int stage = 0;
    uint32_t acc_phase = 0;
    int consumed = 0;
    int n_tfull = 0;
    bool bad = false;
    long long g = g0;
    int kb_first = static_cast<int>(g0 % KB);
    KCursor cur;
    cur.seek(p, g0);
    while (g < g1) {
      const long long seg_len = (KB - kb_first) < (g1 - g) ? (KB - kb_first) : (g1 - g);
      const long long seg_end = g + seg_len;
      kb_first = 0;
      if (lane == 0) bad = !mbar_wait(&tempty_bar, acc_phase ^ 1u, abort_ptr, p.status);
      bad = __shfl_sync(0xffffffffu, bad, 0);
      acc_phase ^= 1u;
      bool stop = false;
      for (bool first = true; g < seg_end; ++g, first = false) {
        if (named_bar_or(kHandoffBar, 64, bad)) {
          stop = true;
          break;
        }
        if (lane == 0) {
          tc_fence_after();
          const int atoms = min(4, p.k_atoms - 4 * cur.kb);
          const uint32_t wa = smem_u32(smem_w + stage * kWTileBytes);
          const uint32_t xa = smem_u32(smem_x + stage * kXTileBytes);
          const uint32_t sfa = tmem_d + kSfCol0 + 32 * stage;
          for (int i = 0; i < atoms; ++i) {
            mma_nvf4_ss(tmem_d, smem_desc_sw128(wa + i * 32), smem_desc_sw128(xa + i * 32), idesc, sfa + 4 * i,
                        sfa + 16 + 4 * i, (first && i == 0) ? 0u : 1u);
          }
          mma_commit(&empty_bar[stage]);
        }
        __syncwarp();
        cur.next(p);
        ++consumed;
        if (++stage == S) stage = 0;
      }
      if (stop) break;
      if (lane == 0) mma_commit(&tfull_bar);
      __syncwarp();
      ++n_tfull;
    }
    if (lane == 0) {
      sh_consumed = consumed;
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, p.status);
    }
    consumed = __shfl_sync(0xffffffffu, consumed, 0);
    n_tfull = __shfl_sync(0xffffffffu, n_tfull, 0);
    {
      const int j = consumed - 1 - lane;
      if (lane < S && j >= 0) mbar_wait(&empty_bar[j % S], static_cast<uint32_t>((j / S) & 1), nullptr, p.status);
      if (lane == 31 && n_tfull > 0)
        mbar_wait(&tfull_bar, static_cast<uint32_t>((n_tfull - 1) & 1), nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == kWaiterWarp) {
    // ---------------- stage waiter ----------------
    // Hands a k-block to the MMA warp once its operands and its scales (the
    // stage's buffer, same phase) are in.
    int stage = 0;
    uint32_t phase = 0;
    for (long long g = g0; g < g1; ++g) {
      bool bad = false;
      if (lane == 0) {
        bad = !mbar_wait(&full_bar[stage], phase, abort_ptr, p.status);
        if (!bad) bad = !mbar_wait(&sf_full[stage], phase, abort_ptr, p.status);
      }
      bad = __shfl_sync(0xffffffffu, bad, 0);
      if (named_bar_or(kHandoffBar, 64, bad)) break;
      if (++stage == S) {
        stage = 0;
        phase ^= 1u;
      }
    }
    __syncwarp();
  } else if (warp >= kSfWarp0) {
    // ---------------- scale writers (warps 7..10) ----------------
    // The scales go to tensor memory in the layout of a 32x128b.warpx4 copy of
    // each 512-byte atom: warp w (lane quarter w % 4) writes, in every one of
    // its 32 lanes r, the atom's row r (16 bytes = rows r, r+32, r+64, r+96 of
    // the tile, four scales each) into 4 columns: buffer + 4 a for the weights'
    // atom a, buffer + 16 + 4 a for the activations'. Each ring stage has its
    // own buffer: the stage's scale atoms land only after the producer refilled
    // the stage, i.e. after the MMAs that read the buffer's previous contents
    // completed, so the writers wait for nothing but the atoms.
    const int q = warp & 3;
    const uint32_t rowoff = static_cast<uint32_t>(16 * lane);
    int stage = 0;
    uint32_t phase = 0;
    KCursor cur;
    cur.seek(p, g0);
    for (long long g = g0; g < g1; ++g) {
      bool bad = false;
      if (lane == 0) bad = !mbar_wait(&sfdat_bar[stage], phase, abort_ptr, p.status);
      if (__shfl_sync(0xffffffffu, bad, 0)) break;
      const int atoms = min(4, p.k_atoms - 4 * cur.kb);
      const uint8_t* sw = smem_sfw + stage * kSfStage + rowoff;
      const uint8_t* sx = smem_sfx + stage * kSfStage + rowoff;
      const uint32_t col = tmem_d + (static_cast<uint32_t>(q * 32) << 16) + kSfCol0 + 32 * static_cast<uint32_t>(stage);
      tc_fence_after();
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        if (a < atoms) {
          tmem_st4(col + 4 * a, *reinterpret_cast<const uint4*>(sw + a * kSfAtom));
          tmem_st4(col + 16 + 4 * a, *reinterpret_cast<const uint4*>(sx + a * kSfAtom));
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sf_full[stage]);
      cur.next(p);
      if (++stage == S) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait_primary();
    const float alpha = __ldg(p.alpha);
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_d + (static_cast<uint32_t>(quarter * 32) << 16);
    uint32_t acc_phase = 0;
    long long g = g0;
    long long tile = g0 / KB;
    int kb0 = static_cast<int>(g0 - tile * KB);
    int pend_old = -1;         // thread 64: counter value its deferred bump returned
    long long pend_tile = -1;  // thread 64: tile of that bump (-1: none)
    for (; g < g1; ++tile, kb0 = 0) {
      const long long seg_len = (KB - kb0) < (g1 - g) ? (KB - kb0) : (g1 - g);
      const int kb1 = kb0 + static_cast<int>(seg_len);
      g += seg_len;
      const bool whole = (kb0 == 0 && kb1 == KB);
      int c_first = 0, c_last = 0;
      if (!whole) {
        const long long cc = cut_contributors(p.sk.total, p.sk.grid, KB, tile);
        c_first = static_cast<int>(cc & 0xffffffffLL);
        c_last = static_cast<int>(cc >> 32);
      }
      const int n_contrib = c_last - c_first + 1;
      const bool is_first = static_cast<int>(blockIdx.x) == c_first;
      int nt, mt;
      decode_tile(p, tile, nt, mt);
      const int n = nt * kBlockN + row;
      const int m0 = mt * TN;
      // Cut tile: the first contributor polls for the others' parts for at most
      // p.sk.first_poll_ns and then reduces without publishing, pulling the
      // parts in while its own last MMAs run. The others publish and bump the
      // tile's counter without waiting for the result, which they check once
      // their other segments are done: the last to arrive (when the first
      // contributor's poll expired and it published too) reduces then. Either
      // way the sum is the first contributor's part + the left fold of the
      // others in CTA order.
      constexpr bool kPrefetch = TN <= 32;
      float other[kPrefetch ? TN : 1];
      bool last = false;
      if (!whole && is_first) {
        if (threadIdx.x == 64)
          sh_is_last =
              (p.sk.first_poll_ns && poll_counter(&p.counters[c_first], n_contrib - 1, abort_ptr, p.sk.first_poll_ns))
                  ? 1
                  : 0;
        named_bar_sync(1, 128);
        last = sh_is_last != 0;
        if constexpr (kPrefetch) {
          if (last) {
#pragma unroll
            for (int c = 0; c < TN / 16; ++c) {
              float t[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) t[j] = 0.0f;
              sum_published<TN>(p, c_first + 1, c_last, c, row, t);
#pragma unroll
              for (int j = 0; j < 16; ++j) other[c * 16 + j] = t[j];
            }
            // Complete the loads now, not at their use after the accumulator wait.
#pragma unroll
            for (int j = 0; j < TN; ++j) asm volatile("" ::"f"(other[j]));
          }
        }
      }
      const bool got = mbar_wait(&tfull_bar, acc_phase, abort_ptr, p.status);
      acc_phase ^= 1u;
      const bool live = __all_sync(0xffffffffu, got);
      tc_fence_after();
      auto emit = [&](int c, const float (&v)[16]) {
        if (p.vec_out) {
          uint16_t* stg = epi_stage + (warp - 2) * 512;
          if (p.out_dtype == CB_DTYPE_BF16)
            emit_chunk_vec<1>(p, n - lane, lane, m0, c * 16, v, alpha, stg);
          else
            emit_chunk_vec<0>(p, n - lane, lane, m0, c * 16, v, alpha, stg);
        } else {
          emit_row(p, n, m0, c * 16, v, alpha);
        }
      };
      if (whole) {
        if (live) {
#pragma unroll
          for (int c = 0; c < TN / 16; ++c) {
            uint32_t r[16];
            __syncwarp();
            tmem_ld16(lane_addr + c * 16, r);
            tmem_ld_wait();
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
            emit(c, v);
          }
        }
      } else {
        const bool prefetched = kPrefetch && last;
        if (!last) {
          // Publish this CTA's part and count it.
          const int slot = static_cast<int>(blockIdx.x) * 2 + p.sk.kind(blockIdx.x, tile);
          float* dst = p.partials + static_cast<long long>(slot) * TN * kBlockN;
          if (live) {
#pragma unroll 1
            for (int c = 0; c < TN / 16; ++c) {
              uint32_t r[16];
              __syncwarp();
              tmem_ld16(lane_addr + c * 16, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) dst[(c * 16 + j) * kBlockN + row] = __uint_as_float(r[j]);
            }
          }
          __threadfence();
          named_bar_sync(1, 128);
          if (is_first) {
            // the poll expired: last-arriver fallback, checked at once
            if (threadIdx.x == 64)
              sh_is_last = (!*abort_ptr && atomicAdd(&p.counters[c_first], 1) == n_contrib - 1) ? 1 : 0;
            named_bar_sync(1, 128);
            last = sh_is_last != 0;
            if (last) __threadfence();
          } else if (threadIdx.x == 64 && !*abort_ptr) {
            // only a CTA's first segment can start inside a tile: one per CTA
            pend_old = atomicAdd(&p.counters[c_first], 1);
            pend_tile = tile;
          }
        }
        if (last && live) {
          // part of contributor cc, chunk c of this thread's row
          auto part = [&](int cc, int c, float (&v)[16]) {
            const int slot = cc * 2 + p.sk.kind(cc, tile);
            const float* src = p.partials + static_cast<long long>(slot) * TN * kBlockN + (c * 16) * kBlockN + row;
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __ldcg(src + j * kBlockN);
          };
#pragma unroll(kPrefetch ? 2 : 1)
          for (int c = 0; c < TN / 16; ++c) {
            uint32_t r[16];
            __syncwarp();
            tmem_ld16(lane_addr + c * 16, r);
            tmem_ld_wait();
            float own[16], v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) own[j] = __uint_as_float(r[j]);
            if (prefetched) {
              if constexpr (kPrefetch) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = other[c * 16 + j];
              }
            } else {
              for (int cc = c_first + 1; cc <= c_last; ++cc) {
                float w[16];
                if (cc == static_cast<int>(blockIdx.x)) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) w[j] = own[j];
                } else {
                  part(cc, c, w);
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = cc == c_first + 1 ? w[j] : __fadd_rn(v[j], w[j]);
              }
            }
            float pf[16];
            if (is_first) {
#pragma unroll
              for (int j = 0; j < 16; ++j) pf[j] = own[j];
            } else {
              part(c_first, c, pf);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(pf[j], v[j]);
            emit(c, v);
          }
          if (threadIdx.x == 64) p.counters[c_first] = 0;  // next launch starts from zero
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar);
    }
    // Deferred check of the part this CTA published without waiting: if its
    // bump was the tile's last arrival, the tile is reduced here from the
    // partial slots (this CTA's part included).
    if (threadIdx.x == 64) {
      const int cf = pend_tile >= 0 ? p.sk.owner(pend_tile * KB) : 0;
      const int cl = pend_tile >= 0 ? p.sk.owner((pend_tile + 1) * KB - 1) : 0;
      sh_is_last = (pend_tile >= 0 && !*abort_ptr && pend_old == cl - cf) ? 1 : 0;
      sh_pend_tile = pend_tile;
    }
    named_bar_sync(1, 128);
    if (sh_is_last) {
      __threadfence();
      const long long t = sh_pend_tile;
      const int cf = p.sk.owner(t * KB);
      const int cl = p.sk.owner((t + 1) * KB - 1);
      int nt, mt;
      decode_tile(p, t, nt, mt);
      const int n = nt * kBlockN + row;
      const int m0 = mt * TN;
      auto part = [&](int cc, int c, float (&v)[16]) {
        const int slot = cc * 2 + p.sk.kind(cc, t);
        const float* src = p.partials + static_cast<long long>(slot) * TN * kBlockN + (c * 16) * kBlockN + row;
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __ldcg(src + j * kBlockN);
      };
#pragma unroll 1
      for (int c = 0; c < TN / 16; ++c) {
        float v[16], w[16];
        for (int cc = cf + 1; cc <= cl; ++cc) {
          part(cc, c, w);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = cc == cf + 1 ? w[j] : __fadd_rn(v[j], w[j]);
        }
        part(cf, c, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(w[j], v[j]);
        if (p.vec_out) {
          uint16_t* stg = epi_stage + (warp - 2) * 512;
          if (p.out_dtype == CB_DTYPE_BF16)
            emit_chunk_vec<1>(p, n - lane, lane, m0, c * 16, v, alpha, stg);
          else
            emit_chunk_vec<0>(p, n - lane, lane, m0, c * 16, v, alpha, stg);
        } else {
          emit_row(p, n, m0, c * 16, v, alpha);
        }
      }
      if (threadIdx.x == 64) p.counters[cf] = 0;  // next launch starts from zero
    }
  }

  __syncthreads();
  if (warp == 0) {
    if (lane == 0 && abort_flag) {
      for (int j = sh_consumed; j < sh_issued; ++j) {
        mbar_wait(&full_bar[j % S], (j / S) & 1, nullptr, p.status);
        mbar_wait(&sfdat_bar[j % S], (j / S) & 1, nullptr, p.status);
      }
    }
    __syncwarp();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_d, kTmemCols);
  }
}

template <int TN>
int launch_tn(const Nvfp4Launch& L, cudaStream_t stream, int grid, const Params& prm) {
  CUtensorMap tw, tx;
  // packed bytes: [N, K/2] weights, [M, K/2] activations, 128-byte boxes (256 k)
  int st = encode_tmap_3d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.b, static_cast<uint64_t>(L.K / 2),
                          static_cast<uint64_t>(L.N), 1, static_cast<uint64_t>(L.b_sn), 0, kStageRowBytes, kBlockN,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CB_OK) return st;
  st = encode_tmap_3d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.a, static_cast<uint64_t>(L.K / 2),
                      static_cast<uint64_t>(L.M), 1, static_cast<uint64_t>(L.a_sm), 0, kStageRowBytes, TN,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CB_OK) return st;
  const size_t stage_bytes = kWTileBytes + static_cast<size_t>(TN) * kStageRowBytes + 2 * kSfStage;
  const size_t smem = static_cast<size_t>(prm.stages) * stage_bytes + 4 * 1024 + 1024;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < smem) {
    if (cudaFuncSetAttribute(nvfp4_gemm_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return CB_ERR_CUDA;
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
  return cuda_status(cudaLaunchKernelEx(&cfg, nvfp4_gemm_kernel<TN>, tw, tx, prm));
}

// Token tile: one tile up to 128 tokens; 128-token tiles beyond (each then
// starts on a 128-row scale atom).
int nvfp4_token_tile(int64_t M) { return M <= 128 ? token_tile(M, 128) : 128; }

}  // namespace

size_t nvfp4_workspace_bytes(int64_t M) {
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  return workspace_need(sms, static_cast<size_t>(nvfp4_token_tile(M)) * kBlockN * sizeof(float));
}

int launch_nvfp4_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t x_sm, const float* global_scale,
                       uint8_t* q, int64_t q_sm, uint8_t* sf, cudaStream_t stream) {
  const int rows_pad = static_cast<int>((rows + 127) / 128 * 128);
  const int c_pad = static_cast<int>((K / 16 + 3) / 4 * 4);
  const long long total = static_cast<long long>(rows_pad) * c_pad;
  int sms = sm_count();
  if (sms <= 0) return CB_ERR_CUDA;
  long long blocks = (total + kQThreads - 1) / kQThreads;
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kQThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  const int r = static_cast<int>(rows), k = static_cast<int>(K);
  if (x_dtype == CB_DTYPE_BF16)
    return cuda_status(cudaLaunchKernelEx(&cfg, nvfp4_quant_kernel<true>, xs, static_cast<long long>(x_sm), r, k,
                                          global_scale, q, static_cast<long long>(q_sm), sf, rows_pad, c_pad));
  return cuda_status(cudaLaunchKernelEx(&cfg, nvfp4_quant_kernel<false>, xs, static_cast<long long>(x_sm), r, k,
                                        global_scale, q, static_cast<long long>(q_sm), sf, rows_pad, c_pad));
}

int launch_nvfp4_gemm(const Nvfp4Launch& L, cudaStream_t stream) {
  if (L.M == 0 || L.N == 0) return CB_OK;
  const int TN = nvfp4_token_tile(L.M);
  Params p = {};
  p.M = static_cast<int>(L.M);
  p.N = static_cast<int>(L.N);
  p.K = static_cast<int>(L.K);
  p.n_tiles = static_cast<int>((L.N + kBlockN - 1) / kBlockN);
  p.m_tiles = static_cast<int>((L.M + TN - 1) / TN);
  p.kb_per_tile = static_cast<int>((L.K + kStageK - 1) / kStageK);
  p.k_atoms = static_cast<int>(L.K / 64);
  const long long tiles = static_cast<long long>(p.n_tiles) * p.m_tiles;
  const long long total = tiles * p.kb_per_tile;
  int sms = sm_count();
  if (sms <= 0) return CB_ERR_CUDA;
  const int grid = stream_k_grid(total, sms, TN, p.kb_per_tile);
  const size_t need = workspace_need(grid, static_cast<size_t>(TN) * kBlockN * sizeof(float));
  if (L.workspace == nullptr || L.workspace_bytes < need) return CB_ERR_WORKSPACE;
  const size_t stage_bytes = kWTileBytes + static_cast<size_t>(TN) * kStageRowBytes + 2 * kSfStage;
  int stages = static_cast<int>((200u * 1024u) / stage_bytes);
  if (stages > kMaxStages) stages = kMaxStages;
  // one 32-column scale buffer per stage after the accumulator, in 512 columns
  const int acc_cols = TN < 32 ? 32 : TN;
  if (stages > (512 - acc_cols) / 32) stages = (512 - acc_cols) / 32;
  if (stages < 2) stages = 2;
  p.stages = stages;
  p.sk.total = total;
  p.sk.grid = grid;
  p.sk.kb_per_tile = p.kb_per_tile;
  p.sk.first_poll_ns = debug_force_last_arriver() ? 0 : kFirstPollNs;
  p.sfw = L.b_sf;
  p.sfx = L.a_sf;
  p.alpha = L.alpha;
  p.out = L.out;
  p.out_dtype = L.out_dtype;
  p.out_sm = L.out_sm;
  p.vec_out = ((L.out_dtype == CB_DTYPE_BF16 || L.out_dtype == CB_DTYPE_F16) && L.N % 8 == 0 && aligned16(L.out) &&
               L.out_sm % 8 == 0)
                  ? 1
                  : 0;
  Workspace ws = carve_workspace(L.workspace, grid);
  p.partials = static_cast<float*>(ws.partials);
  p.counters = ws.counters;
  p.status = ws.status;
  switch (TN) {
    case 16:
      return launch_tn<16>(L, stream, grid, p);
    case 32:
      return launch_tn<32>(L, stream, grid, p);
    case 64:
      return launch_tn<64>(L, stream, grid, p);
    default:
      return launch_tn<128>(L, stream, grid, p);
  }
}

}  // namespace cb
