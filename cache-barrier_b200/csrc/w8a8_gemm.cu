// W8A8 INT8 GEMM for sm_100a: TMA -> shared memory ring -> tcgen05.mma kind::i8
// (int32 accumulators in TMEM) -> fused per-token x per-channel epilogue.
//
// Math follows _w8a8_bmm_kernel (profiling/w8a8/w8a8_bmm.py:44-81):
//   acc[m, n] = sum_k aq[m, k] * w[k, n]            (int32, exact)
//   out[m, n] = cvt(((float)acc * a_scale[m]) * w_scale[n])
//
// Orientation ("swap-AB"): the weight tile is the MMA's M = 128 operand (rows =
// output channels n, K-major) and the token tile is the MMA's N = TN operand, so
// decode batches of 1..32 tokens still fill 128-row MMAs. Work is split over
// all SMs with the stream-K partition of cb_gemm_common.cuh.
//
// Warp roles (352 threads):
//   warp 0     TMA producer (one lane): weight tile 128 x 128 B + token tile TN x 128 B
//              per k-block, 128-byte swizzle. Weight loads of the first ring pass
//              are issued before griddepcontrol.wait; token loads after it.
//   warp 1     TMEM allocation + MMA issuer (one lane), 4 MMAs (K = 32) per k-block.
//   warps 2-5, 7-10  two epilogue groups taking alternate tiles: tcgen05.ld of
//              the accumulator, scaling, bf16/f16/f32 stores (16-bit outputs
//              staged per warp in shared memory and written as 16-byte
//              vectors), split-K slot writes and the deterministic reduction.
//   warp 6     stage waiter: waits for each stage's TMA bytes (and, at a tile's
//              first k-block, for a free accumulator of the TMEM ring) and hands
//              the k-block to warp 1 through a named barrier, so the MMA issuer
//              never waits on shared memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cb_gemm_common.cuh"
#include "cb_internal.h"
#include "cb_ptx.cuh"

#include <type_traits>

namespace cb {
namespace {

constexpr int kBlockN = 128;   // weight rows per tile (MMA M)
constexpr int kBlockK = 128;   // int8 K per k-block (one 128-byte swizzle row)
// Threads of the kernel with EG epilogue groups: producer, MMA, EG x 4
// epilogue warps and the stage waiter.
constexpr int threads_for(int eg) { return eg == 2 ? 352 : 224; }
// Largest k-blocks per tile for which the two-group epilogue is launched: with
// short K every tile is a segment of one or a few k-blocks and the epilogue's
// per-tile latency sets the rate; with long K one group keeps up, and the
// smaller CTA leaves registers for a kernel overlapping it (the activation
// quantizer under programmatic dependent launch).
constexpr int kMaxKbTwoGroups = 8;
constexpr int kWaiterWarp = 6;
constexpr int kHandoffBar = 2;  // named barrier: MMA warp + stage waiter
// Named barriers of the two epilogue warpgroups (128 threads each).
constexpr int kEpiBar0 = 1, kEpiBar1 = 3;
constexpr uint32_t kWTileBytes = kBlockN * kBlockK;
// Fewest k-blocks a CTA takes when the problem has fewer k-blocks than that
// many per SM: small GEMMs then run on fewer CTAs instead of cutting each tile
// into many one-k-block partials that one CTA must sum.
constexpr int kMinKbPerCta = 8;
// Segments (tiles) whose scales the epilogue has in flight: they are copied
// into shared memory (cp.async) kScaleRing - 1 segments ahead, so a short
// segment (one k-block) does not wait a memory round trip for its scales.
constexpr int kScaleRing = 4;

__device__ __forceinline__ void cp_async_f32(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Operand kinds: signed int8 (W8A8), unsigned 8-bit (the W4A4 reference-wrap
// mode), both with int32 accumulators; e4m3 fp8 with fp32 accumulators. All are
// 8-bit operands, so the tiles, ring and MMA K (32) are the same.
constexpr int kKindS8 = 0, kKindU8 = 1, kKindE4M3 = 2;
template <int KIND>
struct AccOf {
  using T = int32_t;
};
template <>
struct AccOf<kKindE4M3> {
  using T = float;
};
__device__ __forceinline__ float acc_f(int32_t v) { return __int2float_rn(v); }
__device__ __forceinline__ float acc_f(float v) { return v; }
template <typename Acc>
__device__ __forceinline__ Acc acc_from_bits(uint32_t b);
template <>
__device__ __forceinline__ int32_t acc_from_bits<int32_t>(uint32_t b) {
  return static_cast<int32_t>(b);
}
template <>
__device__ __forceinline__ float acc_from_bits<float>(uint32_t b) {
  return __uint_as_float(b);
}
// Keeps a value live at this point (the compiler may not sink its load past it).
__device__ __forceinline__ void keep(int32_t v) { asm volatile("" ::"r"(v)); }
__device__ __forceinline__ void keep(float v) { asm volatile("" ::"f"(v)); }

struct Params {
  int M, N, K, H;
  int n_tiles, m_tiles, kb_per_tile;
  int stages;
  StreamK sk;
  const float* a_scale;
  long long as_sb, as_sm;  // a_scale[h * as_sb + m * as_sm] (as_sm = 0: one scale per batch entry)
  const float* w_scale;
  long long ws_sb, ws_sn;  // w_scale[h * ws_sb + n * ws_sn]
  void* out;
  int out_dtype;
  long long out_sb, out_sm;
  int32_t* acc_out;
  int raw_f32;
  const void* bias;  // optional per-output-channel bias, added in fp32 before the rounding
  int bias_dtype;
  long long bias_sb;
  unsigned long long dbg_wait_ns;  // test hook: nonzero = wait this long on a flag nothing sets
  int vec_out;  // 16-bit output, N % 8 == 0, 16-byte aligned rows, no acc_out: vector stores
  void* partials;  // [grid][2][TN][128] accumulators (int32 or fp32)
  int* counters;      // [grid]
  int* status;
};

__device__ __forceinline__ void decode_tile(const Params& p, long long tile, int& h, int& nt, int& mt) {
  split_tile(tile, p.m_tiles, p.n_tiles, h, nt, mt);
}

template <int TN, typename Acc>
__device__ __forceinline__ void emit_row(const Params& p, int h, int n, int m0, int t0, const Acc (&v)[16]) {
  if (n >= p.N) return;
  // All scale loads are issued before any store: a load placed after a store
  // that may alias it would otherwise wait for the previous iteration.
  const float ws = p.raw_f32 ? 1.0f : __ldg(p.w_scale + h * p.ws_sb + n * p.ws_sn);
  const float bv = p.bias ? load_elem(p.bias, p.bias_dtype, h * p.bias_sb + n) : 0.0f;
  float as[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + t0 + j;
    as[j] = (!p.raw_f32 && m < p.M) ? __ldg(p.a_scale + h * p.as_sb + m * p.as_sm) : 1.0f;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + t0 + j;
    if (m < p.M) {
      const long long idx = h * p.out_sb + static_cast<long long>(m) * p.out_sm + n;
      float f = acc_f(v[j]);
      if (!p.raw_f32) f = __fmul_rn(__fmul_rn(f, as[j]), ws);
      if (p.bias) f = __fadd_rn(f, bv);
      store_elem(p.out, p.out_dtype, idx, f);
      if constexpr (std::is_same<Acc, int32_t>::value) {
        if (p.acc_out) p.acc_out[idx] = v[j];
      }
    }
  }
}

// emit_row with the scales (and bias) already in registers (loaded when the segment began).
template <typename Acc>
__device__ __forceinline__ void emit_row_pre(const Params& p, int h, int n, int m0, int t0, const Acc (&v)[16],
                                             float ws, float bv, const float (&as)[16]) {
  if (n >= p.N) return;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + t0 + j;
    if (m < p.M) {
      const long long idx = h * p.out_sb + static_cast<long long>(m) * p.out_sm + n;
      float f = acc_f(v[j]);
      if (!p.raw_f32) f = __fmul_rn(__fmul_rn(f, as[j]), ws);
      if (p.bias) f = __fadd_rn(f, bv);
      store_elem(p.out, p.out_dtype, idx, f);
      if constexpr (std::is_same<Acc, int32_t>::value) {
        if (p.acc_out) p.acc_out[idx] = v[j];
      }
    }
  }
}

// emit_row_pre for 16-bit outputs through shared memory: the warp stages its
// 32 columns x 16 tokens (thread = column) and stores them back as 16-byte
// vectors of 8 columns, one eighth of the store instructions of the
// column-per-thread form. Those stores set the kernel's tail: the reducing CTA's
// sum-and-store after its last MMA took ~1 / 1.8 / 3.3 us at T = 1 / 16 / 32.
// Same arithmetic and rounding as emit_row_pre.
template <int OUT_BF16, typename Acc>
__device__ __forceinline__ void emit_chunk_vec(const Params& p, int h, int n_warp0, int lane, int m0, int t0,
                                               const Acc (&v)[16], float ws, float bv, const float (&as)[16],
                                               uint16_t* stg) {
  const bool has_bias = p.bias != nullptr;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float f = __fmul_rn(__fmul_rn(acc_f(v[j]), as[j]), ws);
    if (has_bias) f = __fadd_rn(f, bv);
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
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + h * p.out_sb + static_cast<long long>(m) * p.out_sm +
                                n8) = val;
  }
  __syncwarp();
}

// Warp-collective store of one 16-token chunk with its scales at hand (from
// registers or the shared-memory scale ring): the vector path for 16-bit
// outputs, else element stores. Same arithmetic and rounding as emit_row.
template <typename Acc>
__device__ __forceinline__ void emit_pre(const Params& p, int h, int n, int lane, int m0, int t0, const Acc (&v)[16],
                                         float ws, float bv, const float (&as)[16], uint16_t* stg) {
  if (p.vec_out) {
    if (p.out_dtype == CB_DTYPE_BF16)
      emit_chunk_vec<1, Acc>(p, h, n - lane, lane, m0, t0, v, ws, bv, as, stg);
    else
      emit_chunk_vec<0, Acc>(p, h, n - lane, lane, m0, t0, v, ws, bv, as, stg);
  } else {
    emit_row_pre<Acc>(p, h, n, m0, t0, v, ws, bv, as);
  }
}

// Warp-collective store of one 16-token chunk for the paths without preloaded
// scales (token tiles above 32): loads the scales as emit_row does, then takes
// the vector path for 16-bit outputs.
template <int TN, typename Acc>
__device__ __forceinline__ void emit_row_any(const Params& p, int h, int n, int lane, int m0, int t0,
                                             const Acc (&v)[16], uint16_t* stg) {
  if (!p.vec_out) {
    emit_row<TN, Acc>(p, h, n, m0, t0, v);
    return;
  }
  const float ws = n < p.N ? __ldg(p.w_scale + h * p.ws_sb + n * p.ws_sn) : 1.0f;
  const float bv = (p.bias && n < p.N) ? load_elem(p.bias, p.bias_dtype, h * p.bias_sb + n) : 0.0f;
  float as[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + t0 + j;
    as[j] = m < p.M ? __ldg(p.a_scale + h * p.as_sb + m * p.as_sm) : 1.0f;
  }
  if (p.out_dtype == CB_DTYPE_BF16)
    emit_chunk_vec<1, Acc>(p, h, n - lane, lane, m0, t0, v, ws, bv, as, stg);
  else
    emit_chunk_vec<0, Acc>(p, h, n - lane, lane, m0, t0, v, ws, bv, as, stg);
}

// Adds the published parts of contributors [c_lo, c_hi] (each its first
// segment, slot kind 0) for chunk c of this thread's row; loads of four
// contributors are in flight together.
template <int TN, typename Acc>
__device__ __forceinline__ void sum_published(const Params& p, int c_lo, int c_hi, int c, int row, Acc (&v)[16]) {
  for (int cc = c_lo; cc <= c_hi; cc += 4) {
    Acc part[4][16];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c2 = cc + u;
      const Acc* src =
          static_cast<const Acc*>(p.partials) + static_cast<long long>(c2 * 2) * TN * kBlockN + (c * 16) * kBlockN + row;
#pragma unroll
      for (int j = 0; j < 16; ++j) part[u][j] = c2 <= c_hi ? __ldcg(src + j * kBlockN) : Acc(0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += part[u][j];
  }
}

template <int TN, int KIND, int EG>
__global__ void __launch_bounds__(threads_for(EG), 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                     const Params p) {
  using Acc = typename AccOf<KIND>::T;
  constexpr uint32_t kATileBytes = TN * kBlockK;
  constexpr uint32_t kStageBytes = kWTileBytes + kATileBytes;
  constexpr uint32_t kAccCols = TN < 32 ? 32 : TN;
  // Accumulator ring in TMEM: segment s uses accumulator s % kNumAcc, so the
  // MMAs run up to kNumAcc - 1 segments ahead of the epilogue (short-K problems
  // have one k-block per tile, and the epilogue's per-tile latency would
  // otherwise gate every tile's MMAs).
  constexpr int kNumAcc = static_cast<int>(512 / kAccCols) < 8 ? static_cast<int>(512 / kAccCols) : 8;
  constexpr uint32_t kTmemCols = kNumAcc * kAccCols;
  static_assert((kNumAcc & (kNumAcc - 1)) == 0 && kTmemCols <= 512, "accumulator ring must fit TMEM");

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t tfull_bar[kNumAcc], tempty_bar[kNumAcc], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ long long sh_pend_tile[2];
  __shared__ int sh_issued, sh_consumed;
  __shared__ int sh_is_last[2];  // per epilogue group: whether this CTA reduces the cut tile at hand
  // scales of the next kScaleRing segments (epilogue, token tiles up to 32)
  __shared__ __align__(16) float ws_ring[EG][kScaleRing][kBlockN];
  __shared__ __align__(16) float as_ring[EG][kScaleRing][TN];
  volatile int* abort_ptr = &abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_w = smem;
  uint8_t* smem_a = smem + p.stages * kWTileBytes;
  // per epilogue warp (8): 16 tokens x 32 columns of 16-bit output (vector-store staging)
  uint16_t* epi_stage = reinterpret_cast<uint16_t*>(smem_a + p.stages * (TN * kBlockK));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.stages;
  const int KB = p.kb_per_tile;
  const long long g0 = p.sk.start(blockIdx.x);
  const long long g1 = p.sk.start(blockIdx.x + 1);

  if (threadIdx.x == 0) {
    // The next kernel in the stream may launch now: it only prefetches weights
    // before its griddepcontrol.wait, which waits for this grid to complete.
    pdl_launch_dependents();
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < kNumAcc; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    sh_issued = 0;
    sh_consumed = 0;
    sh_is_last[0] = 0;
    sh_is_last[1] = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_a);
  }
  // Lanes of a warp reach every CTA-wide barrier together (aligned barriers
  // count a warp as arrived when any of its lanes arrives).
  __syncwarp();
  // First ring pass of weight loads: lane j of warp 0 issues stage j, as soon as
  // the barriers exist and before the CTA-wide setup (TMEM allocation), so the
  // weight stream starts within a few hundred cycles of the CTA's launch.
  const long long nmine = g1 - g0;
  const int pro = static_cast<int>(nmine < S ? nmine : S);
  const uint64_t pol_w = policy_evict_first();
  if (warp == 0 && lane < pro) {
    KCursor c;
    c.seek(p, g0 + lane);
    mbar_arrive_expect_tx(&full_bar[lane], kStageBytes);
    tma_load_3d(smem_w + lane * kWTileBytes, &tmap_w, &full_bar[lane], c.kb * kBlockK, c.nt * kBlockN, c.h, pol_w);
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
  const uint32_t tmem_d = tmem_base_sh;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t pol_a = policy_evict_last();
    // Activations and scales are produced by the preceding kernel.
    pdl_wait_primary();
    if (lane < pro) {
      KCursor c;
      c.seek(p, g0 + lane);
      tma_load_3d(smem_a + lane * kATileBytes, &tmap_a, &full_bar[lane], c.kb * kBlockK, c.mt * TN, c.h, pol_a);
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
        mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
        tma_load_3d(smem_w + stage * kWTileBytes, &tmap_w, &full_bar[stage], cur.kb * kBlockK, cur.nt * kBlockN,
                    cur.h, pol_w);
        tma_load_3d(smem_a + stage * kATileBytes, &tmap_a, &full_bar[stage], cur.kb * kBlockK, cur.mt * TN, cur.h,
                    pol_a);
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
    // Lane 0 issues. The tensor core's instruction queue is shallow, so any
    // stall of the issuing thread idles the tensor core; a shared-memory access
    // (an mbarrier wait, a flag read) stalls it behind the tensor core's own
    // operand reads. The stage-full waits are therefore done by warp 6, which
    // hands each k-block over through a named barrier (no shared memory); the
    // barrier's OR also carries a failed wait of either side, so both warps
    // leave their loops at the same k-block.
    const uint32_t idesc = KIND == kKindU8     ? idesc_u8_s32(kBlockN, TN)
                           : KIND == kKindE4M3 ? idesc_e4m3_f32(kBlockN, TN)
                                               : idesc_i8_s32(kBlockN, TN);
    int stage = 0;
    int consumed = 0;
    int n_tfull = 0;
    long long g = g0;
    int kb_first = static_cast<int>(g0 % KB);
    for (int seg = 0; g < g1; ++seg) {
      const long long seg_len = (KB - kb_first) < (g1 - g) ? (KB - kb_first) : (g1 - g);
      const long long seg_end = g + seg_len;
      kb_first = 0;
      // Segment seg accumulates into accumulator seg % kNumAcc; the stage waiter
      // hands the segment's first k-block over only once the epilogue has
      // drained that accumulator's previous segment.
      const int acc = seg & (kNumAcc - 1);
      const uint32_t tmem_acc = tmem_d + acc * kAccCols;
      bool stop = false;
      for (bool first = true; g < seg_end; ++g, first = false) {
        if (named_bar_or(kHandoffBar, 64, false)) {
          stop = true;
          break;
        }
        if (lane == 0) {
          tc_fence_after();
          const uint32_t wa = smem_u32(smem_w + stage * kWTileBytes);
          const uint32_t aa = smem_u32(smem_a + stage * kATileBytes);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 32; ++kk) {
            if constexpr (KIND == kKindE4M3)
              mma_f8_ss(tmem_acc, smem_desc_sw128(wa + kk * 32), smem_desc_sw128(aa + kk * 32), idesc,
                        (first && kk == 0) ? 0u : 1u);
            else
              mma_i8_ss(tmem_acc, smem_desc_sw128(wa + kk * 32), smem_desc_sw128(aa + kk * 32), idesc,
                        (first && kk == 0) ? 0u : 1u);
          }
          mma_commit(&empty_bar[stage]);
        }
        __syncwarp();
        ++consumed;
        if (++stage == S) stage = 0;
      }
      if (stop) break;
      if (lane == 0) mma_commit(&tfull_bar[acc]);
      __syncwarp();
      ++n_tfull;
    }
    if (lane == 0) {
      sh_consumed = consumed;
      // All issued MMAs must finish before TMEM is released.
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, p.status);
    }
    // Every commit arrival lane 0 issued must land before the CTA exits (an
    // arrive on released shared memory faults): the releases of the last S
    // stages (lanes 0..S-1, S <= 16) and the last kNumAcc accumulator hand-offs
    // (lanes 16..16+kNumAcc-1). One lane per barrier, so the waits overlap
    // instead of adding up.
    consumed = __shfl_sync(0xffffffffu, consumed, 0);
    n_tfull = __shfl_sync(0xffffffffu, n_tfull, 0);
    {
      const int j = consumed - 1 - lane;  // lane l waits the (l+1)-th most recent stage release
      if (lane < S && j >= 0) mbar_wait(&empty_bar[j % S], static_cast<uint32_t>((j / S) & 1), nullptr, p.status);
      const int t = n_tfull - 1 - (lane - 16);  // lanes 16.. : the last kNumAcc accumulator hand-offs
      if (lane >= 16 && lane < 16 + kNumAcc && t >= 0)
        mbar_wait(&tfull_bar[t & (kNumAcc - 1)], static_cast<uint32_t>((t / kNumAcc) & 1), nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == kWaiterWarp) {
    // ---------------- stage waiter ----------------
    // Waits for each stage's TMA bytes (and, before a segment's first k-block,
    // for the epilogue to free the segment's accumulator) and hands the k-block
    // to the MMA warp: one named-barrier round per k-block, the same count as
    // the MMA warp's.
    int stage = 0;
    uint32_t phase = 0;
    int kb = static_cast<int>(g0 % KB);  // k-block within its tile
    int seg = -1;
    for (long long g = g0; g < g1; ++g) {
      bool bad = false;
      if (g == g0 || kb == 0) ++seg;
      if (lane == 0) {
        if (g == g0 || kb == 0)
          bad = !mbar_wait(&tempty_bar[seg & (kNumAcc - 1)], static_cast<uint32_t>(((seg / kNumAcc) & 1) ^ 1),
                           abort_ptr, p.status);
        if (!bad) bad = !mbar_wait(&full_bar[stage], phase, abort_ptr, p.status);
      }
      bad = __shfl_sync(0xffffffffu, bad, 0);
      if (named_bar_or(kHandoffBar, 64, bad)) break;
      if (++stage == S) {
        stage = 0;
        phase ^= 1u;
      }
      if (++kb == KB) kb = 0;
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (group 0: warps 2..5, group 1: warps 7..10) ----------------
    // The two groups take alternate segments (group s % 2 drains segment s),
    // so one group's scale loads, TMEM reads and stores overlap the other's;
    // with one k-block per tile (short K) a single group's per-tile latency
    // would set the kernel's rate. Each accumulator of the ring belongs to one
    // group (the ring size is even). Control flow is uniform across a group's
    // 128 threads even after an aborted wait: work is skipped, but every named
    // barrier is still reached by all of them, so no thread can be left
    // waiting on a barrier.
    const int grp = (EG == 2 && warp > kWaiterWarp) ? 1 : 0;
    const int leader = grp == 0 ? 64 : (kWaiterWarp + 1) * 32;  // runs the group's counter operations
    const int ebar = grp == 0 ? kEpiBar0 : kEpiBar1;
    uint16_t* const stg = epi_stage + (grp == 0 ? warp - 2 : warp - 3) * 512;  // this warp's staging
    pdl_wait_primary();
    // Failure-detection test hook (cb_debug_force_wait_timeout): one thread
    // waits, with a short limit, on a workspace word that nothing ever sets, so
    // the wait expires and every role of the CTA takes its abort path.
    if (p.dbg_wait_ns != 0 && threadIdx.x == 64)
      wait_counter(p.status + 1, 1, abort_ptr, p.status, p.dbg_wait_ns);
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr0 = tmem_d + (static_cast<uint32_t>(quarter * 32) << 16);
    int seg = 0;
    long long g = g0;
    long long tile = g0 / KB;
    int kb0 = static_cast<int>(g0 - tile * KB);
    int pend_old = -1;         // leader: counter value its deferred bump returned
    long long pend_tile = -1;  // leader: tile of that bump (-1: none)
    constexpr bool kPrefetch = TN <= 32;  // token scales in registers
    // the first contributor of a cut tile sums the others' parts into registers
    // while its own last MMAs run
    constexpr bool kPrefetchParts = TN <= 64;
    const long long last_tile = (g1 - 1) / KB;
    // Copies (cp.async, one commit group per own segment) of the scales of the
    // group's k-th own segment into its ring slot k % kScaleRing: each thread
    // its row's w_scale, threads 0..TN-1 one a_scale each.
    // Tile coordinates of the current segment (cur) and of the own segment
    // whose scales are copied next (pre, kScaleRing - 1 own segments ahead:
    // each own segment is two tiles on).
    TileCursor cur, pre;
    cur.seek(tile, p.m_tiles, p.n_tiles);
    pre = cur;
    if (grp) pre.next(p.m_tiles, p.n_tiles);
    auto issue_scales = [&](long long t, int slot) {
      if (t <= last_tile && !p.raw_f32) {
        const int nn = pre.nt * kBlockN + row;
        if (nn < p.N) cp_async_f32(&ws_ring[grp][slot][row], p.w_scale + pre.h * p.ws_sb + nn * p.ws_sn);
#pragma unroll
        for (int r = row; r < TN; r += kBlockN) {
          const int mm = pre.mt * TN + r;
          if (mm < p.M) cp_async_f32(&as_ring[grp][slot][r], p.a_scale + pre.h * p.as_sb + mm * p.as_sm);
        }
      }
      cp_async_commit();
#pragma unroll
      for (int e = 0; e < EG; ++e) pre.next(p.m_tiles, p.n_tiles);
    };
#pragma unroll
    for (int d = 0; d < kScaleRing - 1; ++d) issue_scales(tile + grp + EG * d, d);
    for (; g < g1; ++tile, kb0 = 0, cur.next(p.m_tiles, p.n_tiles), ++seg) {
      const long long seg_len = (KB - kb0) < (g1 - g) ? (KB - kb0) : (g1 - g);
      const int kb1 = kb0 + static_cast<int>(seg_len);
      g += seg_len;
      if (EG == 2 && (seg & 1) != grp) continue;  // the other group's segment
      const int own = EG == 2 ? seg >> 1 : seg;   // index among this group's segments
      const bool whole = (kb0 == 0 && kb1 == KB);
      int c_first = 0, c_last = 0;
      if (!whole) {
        const long long cc = cut_contributors(p.sk.total, p.sk.grid, KB, tile);
        c_first = static_cast<int>(cc & 0xffffffffLL);
        c_last = static_cast<int>(cc >> 32);
      }
      const int h = cur.h, nt = cur.nt, mt = cur.mt;
      const int n = nt * kBlockN + row;
      const int m0 = mt * TN;
      // Scales of the rows this segment stores: copied into the ring
      // kScaleRing - 1 segments ago; wait for this segment's group, make every
      // thread's copies visible, then reuse the slot the previous segment read.
      // Token tiles up to 32 keep their token scales in registers; wider ones
      // read them from the ring slot per 16-token chunk (scales16).
      float ws_pre = 1.0f;
      float bias_pre = 0.0f;
      float as_pre[kPrefetch ? TN : 1];
      const int slot = own % kScaleRing;
      cp_async_wait<kScaleRing - 2>();
      named_bar_sync(ebar, 128);
      issue_scales(tile + EG * (kScaleRing - 1), (own + kScaleRing - 1) % kScaleRing);
      if (!p.raw_f32 && n < p.N) ws_pre = ws_ring[grp][slot][row];
      if (p.bias && n < p.N) bias_pre = load_elem(p.bias, p.bias_dtype, h * p.bias_sb + n);
      auto scales16 = [&](int c, float (&as16)[16]) {
#pragma unroll
        for (int j = 0; j < 16; ++j) as16[j] = (!p.raw_f32 && m0 + c * 16 + j < p.M) ? as_ring[grp][slot][c * 16 + j] : 1.0f;
      };
      if constexpr (kPrefetch) {
        if (!p.raw_f32) {
#pragma unroll
          for (int j4 = 0; j4 < TN / 4; ++j4) {
            const float4 a4 = reinterpret_cast<const float4*>(as_ring[grp][slot])[j4];
            as_pre[4 * j4 + 0] = m0 + 4 * j4 + 0 < p.M ? a4.x : 1.0f;
            as_pre[4 * j4 + 1] = m0 + 4 * j4 + 1 < p.M ? a4.y : 1.0f;
            as_pre[4 * j4 + 2] = m0 + 4 * j4 + 2 < p.M ? a4.z : 1.0f;
            as_pre[4 * j4 + 3] = m0 + 4 * j4 + 3 < p.M ? a4.w : 1.0f;
          }
        } else {
#pragma unroll
          for (int j = 0; j < TN; ++j) as_pre[j] = 1.0f;
        }
      }
      // Cut tile. Its first contributor (whose range ends in this tile; the
      // others covered it at the start of theirs, so they are done first when
      // all CTAs run together) polls for the others' parts for at most
      // p.sk.first_poll_ns and then reduces without publishing its own, pulling
      // the parts in while its last MMAs run. Every other contributor publishes
      // its part and bumps the tile's counter without waiting for the atomic's
      // result; it looks at that result once its other segments are done, and
      // if it arrived last (the first contributor gave up its poll and
      // published too) it reduces the tile then. Both reductions sum in one
      // order (the first contributor's part + the left fold of the others in
      // CTA order), so results do not depend on who reduces, and no CTA waits
      // on another beyond the bounded poll.
      const int n_contrib = c_last - c_first + 1;
      const bool is_first = static_cast<int>(blockIdx.x) == c_first;
      bool last = false;
      Acc other[kPrefetchParts ? TN : 1];
      if (!whole && is_first) {
        if (threadIdx.x == leader)
          sh_is_last[grp] =
              (p.sk.first_poll_ns && poll_counter(&p.counters[c_first], n_contrib - 1, abort_ptr, p.sk.first_poll_ns))
                  ? 1
                  : 0;
        named_bar_sync(ebar, 128);
        last = sh_is_last[grp] != 0;
        if constexpr (kPrefetchParts) {
          if (last) {
#pragma unroll
            for (int c = 0; c < TN / 16; ++c) {
              Acc v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = Acc(0);
              sum_published<TN, Acc>(p, c_first + 1, c_last, c, row, v);
#pragma unroll
              for (int j = 0; j < 16; ++j) other[c * 16 + j] = v[j];
            }
            // complete the loads now, while this CTA's last MMAs run
#pragma unroll
            for (int j = 0; j < TN; ++j) keep(other[j]);
          }
        }
      }
      const int acc = seg & (kNumAcc - 1);
      const uint32_t lane_addr = lane_addr0 + acc * kAccCols;
      const bool got = mbar_wait(&tfull_bar[acc], static_cast<uint32_t>((seg / kNumAcc) & 1), abort_ptr, p.status);
      const bool live = __all_sync(0xffffffffu, got);
      tc_fence_after();
      if (whole) {
        // Whole tile in this CTA: epilogue straight from TMEM.
        if (live) {
          if constexpr (kPrefetch) {
#pragma unroll
            for (int c = 0; c < TN / 16; ++c) {
              uint32_t r[16];
              __syncwarp();
              tmem_ld16(lane_addr + c * 16, r);
              tmem_ld_wait();
              Acc v[16];
              float as16[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                v[j] = acc_from_bits<Acc>(r[j]);
                as16[j] = as_pre[c * 16 + j];
              }
              if (p.vec_out) {
                if (p.out_dtype == CB_DTYPE_BF16)
                  emit_chunk_vec<1, Acc>(p, h, n - lane, lane, m0, c * 16, v, ws_pre, bias_pre, as16, stg);
                else
                  emit_chunk_vec<0, Acc>(p, h, n - lane, lane, m0, c * 16, v, ws_pre, bias_pre, as16, stg);
              } else {
                emit_row_pre<Acc>(p, h, n, m0, c * 16, v, ws_pre, bias_pre, as16);
              }
            }
          } else {
#pragma unroll 1
            for (int c = 0; c < TN / 16; ++c) {
              uint32_t r[16];
              __syncwarp();
              tmem_ld16(lane_addr + c * 16, r);
              tmem_ld_wait();
              Acc v[16];
              float as16[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = acc_from_bits<Acc>(r[j]);
              scales16(c, as16);
              emit_pre<Acc>(p, h, n, lane, m0, c * 16, v, ws_pre, bias_pre, as16, stg);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      } else {
        const bool prefetched = kPrefetchParts && last && is_first;
        if (!last) {
          // publish this CTA's part (raw accumulator bits) and count it
          const int slot = static_cast<int>(blockIdx.x) * 2 + p.sk.kind(blockIdx.x, tile);
          uint32_t* dst = static_cast<uint32_t*>(p.partials) + static_cast<long long>(slot) * TN * kBlockN;
          if (live) {
#pragma unroll 1
            for (int c = 0; c < TN / 16; ++c) {
              uint32_t r[16];
              __syncwarp();
              tmem_ld16(lane_addr + c * 16, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) dst[(c * 16 + j) * kBlockN + row] = r[j];
            }
          }
          __threadfence();
          named_bar_sync(ebar, 128);
          if (is_first) {
            // the poll expired: last-arriver fallback, checked at once
            if (threadIdx.x == leader)
              sh_is_last[grp] = (!*abort_ptr && atomicAdd(&p.counters[c_first], 1) == n_contrib - 1) ? 1 : 0;
            named_bar_sync(ebar, 128);
            last = sh_is_last[grp] != 0;
            if (last) __threadfence();
          } else if (threadIdx.x == leader && !*abort_ptr) {
            // only a CTA's first segment can start inside a tile, so there is
            // at most one of these per CTA
            pend_old = atomicAdd(&p.counters[c_first], 1);
            pend_tile = tile;
          }
        }
        if (last && live) {
          // part of contributor cc, chunk c of this thread's row
          auto part = [&](int cc, int c, Acc (&v)[16]) {
            const int slot = cc * 2 + p.sk.kind(cc, tile);
            const Acc* src = static_cast<const Acc*>(p.partials) + static_cast<long long>(slot) * TN * kBlockN +
                             (c * 16) * kBlockN + row;
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __ldcg(src + j * kBlockN);
          };
#pragma unroll(kPrefetchParts ? TN / 16 : 1)
          for (int c = 0; c < TN / 16; ++c) {
            uint32_t r[16];
            __syncwarp();
            tmem_ld16(lane_addr + c * 16, r);
            tmem_ld_wait();
            Acc own[16], v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) own[j] = acc_from_bits<Acc>(r[j]);
            // S = left fold of the parts of c_first + 1 .. c_last
            if (prefetched) {
              if constexpr (kPrefetchParts) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = other[c * 16 + j];
              }
            } else {
              for (int cc = c_first + 1; cc <= c_last; ++cc) {
                Acc w[16];
                if (cc == static_cast<int>(blockIdx.x)) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) w[j] = own[j];
                } else {
                  part(cc, c, w);
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = cc == c_first + 1 ? w[j] : v[j] + w[j];
              }
            }
            // + the first contributor's part
            Acc pf[16];
            if (is_first) {
#pragma unroll
              for (int j = 0; j < 16; ++j) pf[j] = own[j];
            } else {
              part(c_first, c, pf);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = pf[j] + v[j];
            if constexpr (kPrefetch) {
              float as16[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) as16[j] = as_pre[c * 16 + j];
              if (p.vec_out) {
                if (p.out_dtype == CB_DTYPE_BF16)
                  emit_chunk_vec<1, Acc>(p, h, n - lane, lane, m0, c * 16, v, ws_pre, bias_pre, as16, stg);
                else
                  emit_chunk_vec<0, Acc>(p, h, n - lane, lane, m0, c * 16, v, ws_pre, bias_pre, as16, stg);
              } else {
                emit_row_pre<Acc>(p, h, n, m0, c * 16, v, ws_pre, bias_pre, as16);
              }
            } else {
              float as16[16];
              scales16(c, as16);
              emit_pre<Acc>(p, h, n, lane, m0, c * 16, v, ws_pre, bias_pre, as16, stg);
            }
          }
          if (threadIdx.x == leader) p.counters[c_first] = 0;  // next launch starts from zero
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      }
    }
    // Deferred check of the part this CTA published without waiting: if its
    // bump was the tile's last arrival, the tile is reduced here, every part
    // (this CTA's included) read back from the partial slots.
    if (threadIdx.x == leader) {
      const int cf = pend_tile >= 0 ? p.sk.owner(pend_tile * KB) : 0;
      const int cl = pend_tile >= 0 ? p.sk.owner((pend_tile + 1) * KB - 1) : 0;
      sh_is_last[grp] = (pend_tile >= 0 && !*abort_ptr && pend_old == cl - cf) ? 1 : 0;
      sh_pend_tile[grp] = pend_tile;
    }
    named_bar_sync(ebar, 128);
    if (sh_is_last[grp]) {
      __threadfence();
      const long long t = sh_pend_tile[grp];
      const int cf = p.sk.owner(t * KB);
      const int cl = p.sk.owner((t + 1) * KB - 1);
      int h, nt, mt;
      decode_tile(p, t, h, nt, mt);
      auto part = [&](int cc, int c, Acc (&v)[16]) {
        const int slot = cc * 2 + p.sk.kind(cc, t);
        const Acc* src =
            static_cast<const Acc*>(p.partials) + static_cast<long long>(slot) * TN * kBlockN + (c * 16) * kBlockN + row;
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __ldcg(src + j * kBlockN);
      };
#pragma unroll 1
      for (int c = 0; c < TN / 16; ++c) {
        Acc v[16], w[16];
        for (int cc = cf + 1; cc <= cl; ++cc) {
          part(cc, c, w);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = cc == cf + 1 ? w[j] : v[j] + w[j];
        }
        part(cf, c, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = w[j] + v[j];
        emit_row_any<TN, Acc>(p, h, nt * kBlockN + row, lane, mt * TN, c * 16, v, stg);
      }
      if (threadIdx.x == leader) p.counters[cf] = 0;  // next launch starts from zero
    }
  }

  cp_async_wait<0>();  // no scale copy outlives the CTA (the epilogue consumed all of them)
  __syncthreads();
  if (warp == 0) {
    if (lane == 0 && abort_flag) {
      // Loads issued but never consumed must land before the CTA exits.
      for (int j = sh_consumed; j < sh_issued; ++j) mbar_wait(&full_bar[j % S], (j / S) & 1, nullptr, p.status);
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

template <int TN, int KIND, int EG>
int launch_tn(const W8A8Launch& L, cudaStream_t stream, int grid, int stages, const Params& prm) {
  CUtensorMap tw, ta;
  int st = encode_tmap_3d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.w, static_cast<uint64_t>(L.K),
                          static_cast<uint64_t>(L.N), static_cast<uint64_t>(L.batch), L.w_sn, L.w_sb, kBlockK,
                          kBlockN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CB_OK) return st;
  st = encode_tmap_3d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.aq, static_cast<uint64_t>(L.K),
                      static_cast<uint64_t>(L.M), static_cast<uint64_t>(L.batch), L.aq_sm, L.aq_sb, kBlockK, TN,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CB_OK) return st;
  const size_t smem = static_cast<size_t>(stages) * (kWTileBytes + TN * kBlockK) + EG * 4 * 1024 + 1024;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < smem) {
    cudaError_t e = cudaFuncSetAttribute(w8a8_gemm_kernel<TN, KIND, EG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return CB_ERR_CUDA;
    configured_dev = dev;
    configured_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads_for(EG));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, w8a8_gemm_kernel<TN, KIND, EG>, tw, ta, prm));
}

template <int KIND>
int dispatch_tn(const W8A8Launch& L, cudaStream_t stream, int TN, int grid, int stages, const Params& p) {
  const bool two_groups = p.kb_per_tile <= kMaxKbTwoGroups;
  switch (TN) {
    case 16:
      return two_groups ? launch_tn<16, KIND, 2>(L, stream, grid, stages, p)
                        : launch_tn<16, KIND, 1>(L, stream, grid, stages, p);
    case 32:
      return two_groups ? launch_tn<32, KIND, 2>(L, stream, grid, stages, p)
                        : launch_tn<32, KIND, 1>(L, stream, grid, stages, p);
    case 64:
      return launch_tn<64, KIND, 1>(L, stream, grid, stages, p);
    case 128:
      return launch_tn<128, KIND, 1>(L, stream, grid, stages, p);
    default:
      return launch_tn<256, KIND, 1>(L, stream, grid, stages, p);
  }
}

}  // namespace

size_t w8a8_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K) {
  (void)batch;
  (void)N;
  (void)K;
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const int TN = token_tile(M);
  return workspace_need(sms, static_cast<size_t>(TN) * kBlockN * sizeof(int32_t));
}

int launch_w8a8(const W8A8Launch& L, cudaStream_t stream) {
  if (L.batch == 0 || L.M == 0 || L.N == 0) return CB_OK;
  if (w8a8_gemv_eligible(L)) return launch_w8a8_gemv(L, stream);
  const int TN = token_tile(L.M);
  Params p = {};
  p.M = static_cast<int>(L.M);
  p.N = static_cast<int>(L.N);
  p.K = static_cast<int>(L.K);
  p.H = static_cast<int>(L.batch);
  p.n_tiles = static_cast<int>((L.N + kBlockN - 1) / kBlockN);
  p.m_tiles = static_cast<int>((L.M + TN - 1) / TN);
  p.kb_per_tile = static_cast<int>((L.K + kBlockK - 1) / kBlockK);
  const long long tiles = static_cast<long long>(p.H) * p.n_tiles * p.m_tiles;
  const long long total = tiles * p.kb_per_tile;
  int sms = sm_count();
  if (sms <= 0) return CB_ERR_CUDA;
  const int grid = stream_k_grid(total, sms, TN, p.kb_per_tile, kMinKbPerCta);
  const size_t need = workspace_need(grid, static_cast<size_t>(TN) * kBlockN * sizeof(int32_t));
  if (L.workspace == nullptr || L.workspace_bytes < need) return CB_ERR_WORKSPACE;
  // Ring depth: as many stages as ~200 KiB of shared memory holds.
  const size_t stage_bytes = kWTileBytes + static_cast<size_t>(TN) * kBlockK;
  int stages = static_cast<int>((200u * 1024u) / stage_bytes);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) stages = 2;
  p.stages = stages;
  p.sk.total = total;
  p.sk.grid = grid;
  p.sk.kb_per_tile = p.kb_per_tile;
  p.sk.first_poll_ns = debug_force_last_arriver() ? 0 : kFirstPollNs;
  p.a_scale = L.a_scale;
  p.as_sb = L.as_sb;
  p.as_sm = L.scale_per_tensor_a ? 0 : 1;
  p.w_scale = L.w_scale;
  p.ws_sb = L.ws_sb;
  p.ws_sn = L.scale_per_tensor_w ? 0 : 1;
  p.out = L.out;
  p.out_dtype = L.out_dtype;
  p.out_sb = L.out_sb;
  p.out_sm = L.out_sm;
  p.acc_out = L.acc_out;
  p.raw_f32 = L.raw_f32;
  p.bias = L.raw_f32 ? nullptr : L.bias;
  p.bias_dtype = L.bias_dtype;
  p.bias_sb = L.bias_sb;
  p.dbg_wait_ns = debug_wait_ns();
  p.vec_out = (!L.raw_f32 && L.acc_out == nullptr &&
               (L.out_dtype == CB_DTYPE_BF16 || L.out_dtype == CB_DTYPE_F16) && L.N % 8 == 0 && aligned16(L.out) &&
               L.out_sm % 8 == 0 && (L.batch == 1 || L.out_sb % 8 == 0))
                  ? 1
                  : 0;
  Workspace ws = carve_workspace(L.workspace, grid);
  p.partials = ws.partials;
  p.counters = ws.counters;
  p.status = ws.status;
  if (L.fp8) return dispatch_tn<kKindE4M3>(L, stream, TN, grid, stages, p);
  if (L.unsigned_operands) return dispatch_tn<kKindU8>(L, stream, TN, grid, stages, p);
  return dispatch_tn<kKindS8>(L, stream, TN, grid, stages, p);
}

}  // namespace cb
