// W4A16 int4 group-dequant GEMM (and batched INT4 BMM) for sm_100a.
//
// Math: out[h, m, n] = sum_k a[h, m, k] * q[h, k, n] * s[h, k / G, n]
// following kernel_batched_w4a16_simple (profiling/bench_l2_barrier.py:36-85),
// whose per-output-channel scale is the single-group case G = K; the reference
// applies that scale once to the fp32 accumulator (:80-82), and so does this
// kernel when G >= K. For G = 128 (one group per k-block) the scale is folded
// into the dequantized weight before the MMA.
//
// Data path per k-block (128 rows of N x 128 of K):
//   1. warp 0 copies the 8 KiB native weight tile with one cp.async.bulk and the
//      token tile (TN x 128 activations, two 128-byte-swizzled TMA boxes);
//   2. a dequant warpgroup (4 warps, one weight row per thread) reads its row's
//      64 bytes from shared memory, turns nibbles into bf16/f16 pairs with one
//      LOP3 (mask + exponent-bias OR + sign flip) and one packed subtract, applies
//      the group scale, and stores the row into its A buffer in shared memory in
//      the 128-byte-swizzled K-major layout the MMA reads;
//   3. the warpgroup hands the buffer to warp 1 through a named barrier, and
//      warp 1 issues 8 tcgen05.mma kind::f16 (K = 16 each, both operands from
//      shared memory), accumulating fp32 in TMEM.
// Three dequant warpgroups take every third k-block, each with its own A
// buffer; the first group also runs the epilogue. Split-K and the
// deterministic reduction are the stream-K scheme of cb_gemm_common.cuh.
//
// Throughput limit: moving the dequantized operand (32 KiB of 16-bit values per
// k-block) through the SM costs about as much whether it is written to TMEM
// (tcgen05.st, A read from TMEM) or to shared memory (A read by the MMA from
// shared memory); both measured about 1.2K cycles per k-block per SM at T = 16.
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

constexpr int kBlockN = 128;
constexpr int kBlockK = 128;
constexpr int kDqGroups = 2;  // dequant warpgroups; group g takes the k-blocks j with j % 2 == g
constexpr int kEpiWarp0 = 2 + 4 * kDqGroups;        // first of the 4 epilogue warps
constexpr int kEpiThread0 = kEpiWarp0 * 32;
constexpr int kThreads = (kEpiWarp0 + 4) * 32;      // producer, MMA, 2 x 4 dequant warps, 4 epilogue warps
constexpr uint32_t kWTileBytes = kBlockN * kBlockK / 2;  // 8 KiB
constexpr int kNumABuf = kDqGroups;  // shared-memory A buffer b belongs to dequant group b
// One dequantized A tile: 128 rows x 128 k of 16-bit values, stored as two
// 128-byte-swizzled K-major sub-tiles of 128 rows x 64 k (16 KiB each).
constexpr uint32_t kASubBytes = kBlockN * 128;
constexpr uint32_t kABufBytes = 2 * kASubBytes;
// Named barriers 2..(1 + kNumABuf) hand A buffer b from dequant warpgroup b (4 warps,
// bar.arrive) to the MMA warp (bar.sync); barrier 1 is the epilogue's.
constexpr int kAFullBar0 = 2;
constexpr int kAFullCount = 5 * 32;
// Largest token tile used: 128 (M > 128 is covered by several 128-token tiles).
constexpr int kMaxTokenTile = 128;

struct Params {
  int M, N, K, H;
  int n_tiles, m_tiles, kb_per_tile;
  int stages;
  StreamK sk;
  const uint8_t* w;  // native tiles
  const void* scales;
  int scale_dtype;
  long long s_sb, s_sg;
  int group_size;
  int kb_per_group;  // k-blocks of 128 per scale group (group_size / 128)
  int scale_in_epilogue;
  void* out;
  int out_dtype;
  long long out_sb, out_sm;
  int vec_out;  // 16-bit output, N % 8 == 0, 16-byte aligned rows: vector stores
  float* partials;  // [grid][2][TN][128]
  int* counters;
  int* status;
};

__device__ __forceinline__ void decode_tile(const Params& p, long long tile, int& h, int& nt, int& mt) {
  split_tile(tile, p.m_tiles, p.n_tiles, h, nt, mt);
}

__device__ __forceinline__ void emit_row(const Params& p, int h, int n, int m0, int t0, const float (&v)[16]) {
  if (n >= p.N) return;
  const float sc = p.scale_in_epilogue ? load_elem(p.scales, p.scale_dtype, h * p.s_sb + n) : 1.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + t0 + j;
    if (m < p.M) {
      const long long idx = h * p.out_sb + static_cast<long long>(m) * p.out_sm + n;
      const float f = p.scale_in_epilogue ? __fmul_rn(v[j], sc) : v[j];
      store_elem(p.out, p.out_dtype, idx, f);
    }
  }
}

// emit_row for 16-bit outputs through shared memory: the warp stages its 32
// columns x 16 tokens (thread = column) and stores them back as 16-byte vectors
// of 8 columns, one eighth of the store instructions. Same arithmetic and
// rounding as emit_row.
template <int OUT_BF16>
__device__ __forceinline__ void emit_chunk_vec(const Params& p, int h, int n, int lane, int m0, int t0,
                                               const float (&v)[16], uint16_t* stg) {
  const float sc = (p.scale_in_epilogue && n < p.N) ? load_elem(p.scales, p.scale_dtype, h * p.s_sb + n) : 1.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float f = p.scale_in_epilogue ? __fmul_rn(v[j], sc) : v[j];
    stg[j * 32 + lane] =
        OUT_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(f)) : __half_as_ushort(__float2half_rn(f));
  }
  __syncwarp();
  const int q8 = lane & 3;
  const int n8 = n - lane + q8 * 8;
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

// Warp-collective store of one 16-token chunk (every lane of the warp calls it).
__device__ __forceinline__ void emit_chunk(const Params& p, int h, int n, int lane, int m0, int t0,
                                           const float (&v)[16], uint16_t* stg) {
  if (p.vec_out) {
    if (p.out_dtype == CB_DTYPE_BF16)
      emit_chunk_vec<1>(p, h, n, lane, m0, t0, v, stg);
    else
      emit_chunk_vec<0>(p, h, n, lane, m0, t0, v, stg);
  } else {
    emit_row(p, h, n, m0, t0, v);
  }
}

// Adds (in contributor order) the published parts of contributors [c_lo, c_hi]
// (each its first segment, slot kind 0) for chunk c of this thread's row.
template <int TN>
__device__ __forceinline__ void sum_published(const Params& p, int c_lo, int c_hi, int c, int row, float (&v)[16]) {
  for (int cc = c_lo; cc <= c_hi; cc += 2) {
    float part[2][16];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c2 = cc + u;
      const float* src = p.partials + static_cast<long long>(c2 * 2) * TN * kBlockN + (c * 16) * kBlockN + row;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) part[u][jj] = c2 <= c_hi ? __ldcg(src + jj * kBlockN) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        if (cc + u <= c_hi) v[jj] = __fadd_rn(v[jj], part[u][jj]);
  }
}

template <typename T, int TN>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const Params p) {
  constexpr uint32_t kATileBytes = TN * kBlockK * 2;  // two 128-byte-swizzled boxes of TN x 64
  constexpr uint32_t kBoxBytes = TN * 128;
  constexpr uint32_t kStageBytes = kWTileBytes + kATileBytes;
  constexpr uint32_t kAccCols = TN < 32 ? 32 : TN;
  // Accumulator ring in TMEM (the A operand lives in shared memory): segment s
  // uses accumulator s % kNumAcc, so with short K (one k-block per tile) the
  // MMAs run up to kNumAcc - 1 tiles ahead of the epilogue.
  constexpr int kNumAcc = static_cast<int>(512 / kAccCols) < 8 ? static_cast<int>(512 / kAccCols) : 8;
  constexpr uint32_t kTmemCols = kNumAcc * kAccCols;
  static_assert((kNumAcc & (kNumAcc - 1)) == 0 && kTmemCols <= 512, "accumulator ring must fit TMEM");

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t aempty_bar[kNumABuf];
  __shared__ __align__(8) uint64_t tfull_bar[kNumAcc], tempty_bar[kNumAcc], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ long long sh_pend_tile;
  __shared__ int sh_issued, sh_consumed, sh_is_last;
  volatile int* abort_ptr = &abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_abuf = smem;                                  // dequantized A tiles (1024-aligned)
  uint8_t* smem_a = smem + kNumABuf * kABufBytes;             // token tiles (1024-aligned)
  uint8_t* smem_w = smem_a + p.stages * kATileBytes;          // packed weight tiles
  // per epilogue warp: 16 tokens x 32 columns of 16-bit output (vector-store staging)
  uint16_t* epi_stage = reinterpret_cast<uint16_t*>(smem_w + p.stages * kWTileBytes);

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
      mbar_init(&empty_bar[s], 5);  // 4 dequant warps + 1 MMA commit
    }
    for (int b = 0; b < kNumABuf; ++b) mbar_init(&aempty_bar[b], 1);
    for (int a = 0; a < kNumAcc; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    sh_issued = 0;
    sh_consumed = 0;
    sh_is_last = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
  }
  // Lanes of a warp reach every CTA-wide barrier together (aligned barriers
  // count a warp as arrived when any of its lanes arrives).
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
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      const long long nmine = g1 - g0;
      const int pro = static_cast<int>(nmine < S ? nmine : S);
      KCursor start_cur;
      start_cur.seek(p, g0);
      KCursor cur = start_cur;
      auto wsrc = [&](const KCursor& c) {
        return p.w + ((static_cast<long long>(c.h) * p.n_tiles + c.nt) * KB + c.kb) * kWTileBytes;
      };
      for (int j = 0; j < pro; ++j) {
        mbar_arrive_expect_tx(&full_bar[j], kStageBytes);
        bulk_copy_g2s(smem_w + j * kWTileBytes, wsrc(cur), kWTileBytes, &full_bar[j], pol_w);
        cur.next(p);
      }
      pdl_wait_primary();
      cur = start_cur;
      for (int j = 0; j < pro; ++j) {
        uint8_t* dst = smem_a + j * kATileBytes;
        tma_load_3d(dst, &tmap_a, &full_bar[j], cur.kb * kBlockK, cur.mt * TN, cur.h, pol_a);
        tma_load_3d(dst + kBoxBytes, &tmap_a, &full_bar[j], cur.kb * kBlockK + 64, cur.mt * TN, cur.h, pol_a);
        cur.next(p);
      }
      int issued = pro;
      int stage = pro % S;
      uint32_t phase = (pro == S) ? 1u : 0u;
      for (long long g = g0 + pro; g < g1; ++g) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_ptr, p.status)) break;
        mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
        bulk_copy_g2s(smem_w + stage * kWTileBytes, wsrc(cur), kWTileBytes, &full_bar[stage], pol_w);
        uint8_t* dst = smem_a + stage * kATileBytes;
        tma_load_3d(dst, &tmap_a, &full_bar[stage], cur.kb * kBlockK, cur.mt * TN, cur.h, pol_a);
        tma_load_3d(dst + kBoxBytes, &tmap_a, &full_bar[stage], cur.kb * kBlockK + 64, cur.mt * TN, cur.h, pol_a);
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
    // A dequant warpgroup hands each filled TMEM A buffer over through a named
    // barrier (it waited for the stage's TMA bytes first, so the token tile is
    // in place too). The issuing thread then touches no shared memory per
    // k-block: an access there stalls it behind the tensor core's operand
    // reads, and the tensor core idles while its issuer is stalled. Every
    // k-block's barrier is reached even after a failed wait, so the dequant
    // warps never wait on a barrier this warp abandoned.
    const uint32_t idesc = idesc_f16_f32(kBlockN, TN, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
    int consumed = 0;
    int n_tfull = 0;
    bool bad = false;
    long long g = g0;
    int kb_first = static_cast<int>(g0 % KB);
    int s = 0;
    for (int seg = 0; g < g1; ++seg) {
      const long long seg_len = (KB - kb_first) < (g1 - g) ? (KB - kb_first) : (g1 - g);
      const long long seg_end = g + seg_len;
      kb_first = 0;
      // segment `seg` accumulates into accumulator seg % kNumAcc, free once the
      // epilogue drained the segment kNumAcc back
      const int acc = seg & (kNumAcc - 1);
      const uint32_t tmem_d = tmem_base + acc * kAccCols;
      if (lane == 0 && !bad)
        bad = !mbar_wait(&tempty_bar[acc], static_cast<uint32_t>(((seg / kNumAcc) & 1) ^ 1), abort_ptr, p.status);
      for (bool first = true; g < seg_end; ++g, first = false) {
        const int j = static_cast<int>(g - g0);
        const int b = j % kNumABuf;
        named_bar_sync(kAFullBar0 + b, kAFullCount);
        if (lane == 0 && !bad) {
          tc_fence_after();
          const uint32_t b_base = smem_u32(smem_a + s * kATileBytes);
          const uint32_t w_base = smem_u32(smem_abuf + b * kABufBytes);
#pragma unroll
          for (int i = 0; i < kBlockK / 16; ++i) {
            const uint32_t waddr = w_base + (i >> 2) * kASubBytes + (i & 3) * 32;
            const uint32_t baddr = b_base + (i >> 2) * kBoxBytes + (i & 3) * 32;
            mma_f16_ss(tmem_d, smem_desc_sw128(waddr), smem_desc_sw128(baddr), idesc, (first && i == 0) ? 0u : 1u);
          }
          mma_commit(&aempty_bar[b]);
          mma_commit(&empty_bar[s]);
          ++consumed;
        }
        __syncwarp();
        if (++s == S) s = 0;
      }
      if (lane == 0 && !bad) {
        mma_commit(&tfull_bar[acc]);
        ++n_tfull;
      }
      __syncwarp();
    }
    if (lane == 0) {
      sh_consumed = consumed;
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, p.status);
    }
    // Every commit arrival lane 0 issued must land before the CTA exits (an
    // arrive on released shared memory faults): the releases of the last S
    // stages, of the last use of each A buffer, and the last accumulator
    // hand-offs. One lane per barrier, so the waits overlap.
    consumed = __shfl_sync(0xffffffffu, consumed, 0);
    n_tfull = __shfl_sync(0xffffffffu, n_tfull, 0);
    {
      const int j = consumed - 1 - lane;
      if (lane < S && j >= 0) mbar_wait(&empty_bar[j % S], static_cast<uint32_t>((j / S) & 1), nullptr, p.status);
      const int ja = consumed - 1 - (lane - 24);  // lanes 24.. : A-buffer releases
      if (lane >= 24 && lane < 24 + kNumABuf && ja >= 0)
        mbar_wait(&aempty_bar[ja % kNumABuf], static_cast<uint32_t>((ja / kNumABuf) & 1), nullptr, p.status);
      const int t = n_tfull - 1 - (lane - 16);  // lanes 16.. : the last kNumAcc accumulator hand-offs
      if (lane >= 16 && lane < 16 + kNumAcc && t >= 0)
        mbar_wait(&tfull_bar[t & (kNumAcc - 1)], static_cast<uint32_t>((t / kNumAcc) & 1), nullptr, p.status);
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---------------- dequant warpgroups (warps 2-5: group 0, 6-9: group 1) ----------------
    // Control flow stays uniform after an aborted wait (work is skipped, every
    // barrier arrival and named barrier still happens), so no warp is left
    // waiting on a collective that another warp abandoned.
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const typename Dq<T>::T2 bias = Dq<T>::bias();
    const bool fold_scale = !p.scale_in_epilogue;
    pdl_wait_primary();
    long long g = g0;
    long long tile = g0 / KB;
    int kb0 = static_cast<int>(g0 - tile * KB);
    int s_next = 0;  // ring stage and phase of k-block j, advanced per k-block
    uint32_t ph_next = 0;
    TileCursor cur;  // (batch, n-tile, m-tile) of the segment's tile, advanced without division
    cur.seek(tile, p.m_tiles, p.n_tiles);
    for (; g < g1; ++tile, kb0 = 0, cur.next(p.m_tiles, p.n_tiles)) {
      const long long seg_len = (KB - kb0) < (g1 - g) ? (KB - kb0) : (g1 - g);
      const int kb1 = kb0 + static_cast<int>(seg_len);
      const int h = cur.h, nt = cur.nt;
      const int n = nt * kBlockN + row;
      // Group scales are prefetched one k-block of this group ahead (a group
      // takes every fourth k-block), so their global-load latency is off the
      // dequant's critical path.
      auto group_scale = [&](int kbx) {
        return n < p.N ? load_elem(p.scales, p.scale_dtype, h * p.s_sb + (kbx / p.kb_per_group) * p.s_sg + n) : 0.0f;
      };
      const int kb_mine = kb0 + (grp - static_cast<int>((g - g0) % kDqGroups) + kDqGroups) % kDqGroups;  // this group's first
      float sv_next = (fold_scale && kb_mine < kb1) ? group_scale(kb_mine) : 0.0f;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int j = static_cast<int>(g - g0) + (kb - kb0);
        const int s = s_next;
        const uint32_t ph = ph_next;
        if (++s_next == S) {
          s_next = 0;
          ph_next ^= 1u;
        }
        if (j % kDqGroups != grp) continue;
        const float sv = sv_next;
        if (fold_scale && kb + kDqGroups < kb1) sv_next = group_scale(kb + kDqGroups);
        const int b = grp;
        const uint32_t aph = static_cast<uint32_t>((j / kNumABuf) & 1);
        // Load the row's 64 bytes and dequantize the first half before waiting
        // for the MMA to release this group's A buffer; only the TMEM stores
        // depend on that release.
        bool got = mbar_wait(&full_bar[s], ph, abort_ptr, p.status);
        const bool have = __all_sync(0xffffffffu, got);
        const typename Dq<T>::T2 sc = Dq<T>::from_f(fold_scale ? sv : 1.0f);
        uint4 v[4];
        uint32_t r[32];
        if (have) {
          const uint4* wrow = reinterpret_cast<const uint4*>(smem_w + s * kWTileBytes + row * 64);
          const int swz = (row >> 1) & 3;
#pragma unroll
          for (int c = 0; c < 4; ++c) v[c] = wrow[c ^ swz];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t words[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
#pragma unroll
              for (int pi = 0; pi < 4; ++pi) r[c * 16 + wi * 4 + pi] = dq_pair<T>(words[wi], 4 * pi, bias, sc, fold_scale);
          }
        }
        got = mbar_wait(&aempty_bar[b], aph ^ 1u, abort_ptr, p.status) && got;
        const bool live = __all_sync(0xffffffffu, got);
        if (live) {
          // Row `row` of the A tile: 16-byte chunk q (k = 8q..8q+7) goes to
          // sub-tile q / 8, chunk position (q % 8) ^ (row % 8) of the row's 128 bytes.
          uint8_t* arow = smem_abuf + b * kABufBytes + row * 128;
          const int rx = row & 7;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(arow + (((q & 7) ^ rx) << 4)) =
                make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
#pragma unroll
          for (int c = 2; c < 4; ++c) {
            const uint32_t words[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
            uint32_t r2[16];
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
#pragma unroll
              for (int pi = 0; pi < 4; ++pi) r2[wi * 4 + pi] = dq_pair<T>(words[wi], 4 * pi, bias, sc, fold_scale);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const int q = (c - 2) * 4 + q4;  // chunk within sub-tile 1
              *reinterpret_cast<uint4*>(arow + kASubBytes + ((q ^ rx) << 4)) =
                  make_uint4(r2[4 * q4], r2[4 * q4 + 1], r2[4 * q4 + 2], r2[4 * q4 + 3]);
            }
          }
          // Generic-proxy stores become visible to the tensor core's reads.
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        named_bar_arrive(kAFullBar0 + b, kAFullCount);
      }
      g += seg_len;
    }
  } else {
    // ---------------- epilogue (warps kEpiWarp0 .. kEpiWarp0 + 3) ----------------
    // Drains accumulator seg % 2 of each segment while the MMA fills the other.
    // Control flow is uniform across the 128 epilogue threads even after an
    // aborted wait, so every named barrier is reached by all of them.
    pdl_wait_primary();
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    long long g = g0;
    long long tile = g0 / KB;
    int kb0 = static_cast<int>(g0 - tile * KB);
    int pend_old = -1;         // kEpiThread0: counter value its deferred bump returned
    long long pend_tile = -1;  // kEpiThread0: tile of that bump (-1: none)
    TileCursor cur;  // (batch, n-tile, m-tile) of the segment's tile, advanced without division
    cur.seek(tile, p.m_tiles, p.n_tiles);
    for (int seg = 0; g < g1; ++tile, kb0 = 0, ++seg, cur.next(p.m_tiles, p.n_tiles)) {
      const long long seg_len = (KB - kb0) < (g1 - g) ? (KB - kb0) : (g1 - g);
      const int kb1 = kb0 + static_cast<int>(seg_len);
      g += seg_len;
      const int h = cur.h, nt = cur.nt, mt = cur.mt;
      const int n = nt * kBlockN + row;
      const int acc = seg & (kNumAcc - 1);
      const bool whole = (kb0 == 0 && kb1 == KB);
      int c_first = 0, c_last = 0;
      if (!whole) {
        const long long cc = cut_contributors(p.sk.total, p.sk.grid, KB, tile);
        c_first = static_cast<int>(cc & 0xffffffffLL);
        c_last = static_cast<int>(cc >> 32);
      }
      const int n_contrib = c_last - c_first + 1;
      const bool is_first = static_cast<int>(blockIdx.x) == c_first;
      constexpr bool kPrefetch = TN <= 32;
      float other[kPrefetch ? TN : 1];
      bool last = false;
      if (!whole && is_first) {
        // Cut tile. Its first contributor (whose range ends in this tile; the
        // others covered it at the start of theirs, so they are done first when
        // all CTAs run together) polls for the others' parts for at most
        // p.sk.first_poll_ns and then reduces without publishing its own,
        // pulling the parts in while its last MMAs run. Every other contributor
        // publishes its part and bumps the tile's counter without waiting for
        // the atomic's result; it looks at that result once its other segments
        // are done and, if it arrived last (the first contributor gave up its
        // poll and published too), reduces the tile then. Both reductions sum
        // in one order (the first contributor's part + the left fold of the
        // others in CTA order), so results do not depend on who reduces.
        if (threadIdx.x == kEpiThread0)
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
              float v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = 0.0f;
              sum_published<TN>(p, c_first + 1, c_last, c, row, v);
#pragma unroll
              for (int j = 0; j < 16; ++j) other[c * 16 + j] = v[j];
            }
            // Complete the partial sums now, while this CTA's last MMAs run; the
            // compiler would otherwise sink the loads to their use after the wait.
#pragma unroll
            for (int j = 0; j < TN; ++j) asm volatile("" ::"f"(other[j]));
          }
        }
      }
      const bool got = mbar_wait(&tfull_bar[acc], static_cast<uint32_t>((seg / kNumAcc) & 1), abort_ptr, p.status);
      const bool live = __all_sync(0xffffffffu, got);
      tc_fence_after();
      const int m0 = mt * TN;
      const uint32_t d_addr = tmem_base + acc * kAccCols + lane_off;
      if (whole) {
        if (live) {
#pragma unroll 1
          for (int c = 0; c < TN / 16; ++c) {
            uint32_t r[16];
            __syncwarp();
            tmem_ld16(d_addr + c * 16, r);
            tmem_ld_wait();
            float v[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v[jj] = __uint_as_float(r[jj]);
            emit_chunk(p, h, n, lane, m0, c * 16, v, epi_stage + (warp - kEpiWarp0) * 512);
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
              tmem_ld16(d_addr + c * 16, r);
              tmem_ld_wait();
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) dst[(c * 16 + jj) * kBlockN + row] = __uint_as_float(r[jj]);
            }
          }
          __threadfence();
          named_bar_sync(1, 128);
          if (is_first) {
            // the poll expired: last-arriver fallback, checked at once
            if (threadIdx.x == kEpiThread0)
              sh_is_last = (!*abort_ptr && atomicAdd(&p.counters[c_first], 1) == n_contrib - 1) ? 1 : 0;
            named_bar_sync(1, 128);
            last = sh_is_last != 0;
            if (last) __threadfence();
          } else if (threadIdx.x == kEpiThread0 && !*abort_ptr) {
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
            for (int jj = 0; jj < 16; ++jj) v[jj] = __ldcg(src + jj * kBlockN);
          };
          if (prefetched) {
            if constexpr (kPrefetch) {
#pragma unroll
              for (int c = 0; c < TN / 16; ++c) {
                uint32_t r[16];
                __syncwarp();
                tmem_ld16(d_addr + c * 16, r);
                tmem_ld_wait();
                float v[16];
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) v[jj] = __fadd_rn(__uint_as_float(r[jj]), other[c * 16 + jj]);
                emit_chunk(p, h, n, lane, m0, c * 16, v, epi_stage + (warp - kEpiWarp0) * 512);
              }
            }
          } else {
#pragma unroll 1
            for (int c = 0; c < TN / 16; ++c) {
              uint32_t r[16];
              __syncwarp();
              tmem_ld16(d_addr + c * 16, r);
              tmem_ld_wait();
              float own[16], v[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) own[jj] = __uint_as_float(r[jj]);
              // left fold of the parts of c_first + 1 .. c_last
              for (int cc = c_first + 1; cc <= c_last; ++cc) {
                float w[16];
                if (cc == static_cast<int>(blockIdx.x)) {
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj) w[jj] = own[jj];
                } else {
                  part(cc, c, w);
                }
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) v[jj] = cc == c_first + 1 ? w[jj] : __fadd_rn(v[jj], w[jj]);
              }
              // + the first contributor's part
              float pf[16];
              if (is_first) {
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) pf[jj] = own[jj];
              } else {
                part(c_first, c, pf);
              }
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) v[jj] = __fadd_rn(pf[jj], v[jj]);
              emit_chunk(p, h, n, lane, m0, c * 16, v, epi_stage + (warp - kEpiWarp0) * 512);
            }
          }
          if (threadIdx.x == kEpiThread0) p.counters[c_first] = 0;  // next launch starts from zero
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
    // Deferred check of the part this CTA published without waiting: if its
    // bump was the tile's last arrival, the tile is reduced here from the
    // partial slots (this CTA's part included).
    if (threadIdx.x == kEpiThread0) {
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
      int h, nt, mt;
      decode_tile(p, t, h, nt, mt);
      auto part = [&](int cc, int c, float (&v)[16]) {
        const int slot = cc * 2 + p.sk.kind(cc, t);
        const float* src = p.partials + static_cast<long long>(slot) * TN * kBlockN + (c * 16) * kBlockN + row;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) v[jj] = __ldcg(src + jj * kBlockN);
      };
#pragma unroll 1
      for (int c = 0; c < TN / 16; ++c) {
        float v[16], w[16];
        for (int cc = cf + 1; cc <= cl; ++cc) {
          part(cc, c, w);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) v[jj] = cc == cf + 1 ? w[jj] : __fadd_rn(v[jj], w[jj]);
        }
        part(cf, c, w);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) v[jj] = __fadd_rn(w[jj], v[jj]);
        emit_chunk(p, h, nt * kBlockN + row, lane, mt * TN, c * 16, v, epi_stage + (warp - kEpiWarp0) * 512);
      }
      if (threadIdx.x == kEpiThread0) p.counters[cf] = 0;  // next launch starts from zero
    }
  }

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
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <typename T, int TN>
int launch_typed(const W4A16Launch& L, cudaStream_t stream, int grid, int stages, const Params& prm) {
  CUtensorMap ta;
  const CUtensorMapDataType dt =
      (L.a_dtype == CB_DTYPE_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int st = encode_tmap_3d(&ta, dt, L.a, static_cast<uint64_t>(L.K), static_cast<uint64_t>(L.M),
                          static_cast<uint64_t>(L.batch), L.a_sm, L.a_sb, 64, TN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CB_OK) return st;
  const size_t smem =
      kNumABuf * kABufBytes + static_cast<size_t>(stages) * (kWTileBytes + TN * kBlockK * 2) + 4 * 1024 + 1024;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < smem) {
    cudaError_t e = cudaFuncSetAttribute(w4a16_gemm_kernel<T, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  return cuda_status(cudaLaunchKernelEx(&cfg, w4a16_gemm_kernel<T, TN>, ta, prm));
}

template <typename T>
int launch_dtype(const W4A16Launch& L, cudaStream_t stream, int TN, int grid, int stages, const Params& p) {
  switch (TN) {
    case 16:
      return launch_typed<T, 16>(L, stream, grid, stages, p);
    case 32:
      return launch_typed<T, 32>(L, stream, grid, stages, p);
    case 64:
      return launch_typed<T, 64>(L, stream, grid, stages, p);
    default:
      return launch_typed<T, 128>(L, stream, grid, stages, p);
  }
}

}  // namespace

size_t w4a16_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K) {
  (void)batch;
  (void)N;
  (void)K;
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const size_t tc = workspace_need(sms, static_cast<size_t>(token_tile(M, kMaxTokenTile)) * kBlockN * sizeof(float));
  // the dp4a path for up to kGemvMaxTokens tokens: at most kGemvCtasPerSm CTAs per SM
  const size_t gv = workspace_need(kGemvCtasPerSm * sms, static_cast<size_t>(kGemvMaxTokens) * kBlockN * sizeof(float));
  return tc > gv ? tc : gv;
}

int launch_w4a16(const W4A16Launch& L, cudaStream_t stream) {
  if (L.batch == 0 || L.M == 0 || L.N == 0) return CB_OK;
  if (w4a16_resident_eligible(L)) {
    const int st = launch_w4a16_resident(L, stream);
    if (st != CB_ERR_UNSUPPORTED) return st;
  }
  if (w4a16_gemv_eligible(L)) {
    const int st = launch_w4a16_gemv(L, stream);
    if (st != CB_ERR_UNSUPPORTED) return st;
  }
  const int TN = token_tile(L.M, kMaxTokenTile);
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
  const int sms = sm_count();
  if (sms <= 0) return CB_ERR_CUDA;
  const int grid = stream_k_grid(total, sms, TN, p.kb_per_tile);
  const size_t need = workspace_need(grid, static_cast<size_t>(TN) * kBlockN * sizeof(float));
  if (L.workspace == nullptr || L.workspace_bytes < need) return CB_ERR_WORKSPACE;
  const size_t stage_bytes = kWTileBytes + static_cast<size_t>(TN) * kBlockK * 2;
  int stages = static_cast<int>((220u * 1024u - kNumABuf * kABufBytes) / stage_bytes);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) stages = 2;
  p.stages = stages;
  p.sk.total = total;
  p.sk.grid = grid;
  p.sk.kb_per_tile = p.kb_per_tile;
  p.sk.first_poll_ns = debug_force_last_arriver() ? 0 : kFirstPollNs;
  p.w = L.w;
  p.scales = L.scales;
  p.scale_dtype = L.scale_dtype;
  p.s_sb = L.s_sb;
  p.s_sg = L.s_sg;
  p.group_size = static_cast<int>(L.group_size);
  p.scale_in_epilogue = L.group_size >= L.K ? 1 : 0;
  p.kb_per_group = static_cast<int>(L.group_size / kBlockK) > 0 ? static_cast<int>(L.group_size / kBlockK) : 1;
  p.out = L.out;
  p.out_dtype = L.out_dtype;
  p.out_sb = L.out_sb;
  p.out_sm = L.out_sm;
  p.vec_out = ((L.out_dtype == CB_DTYPE_BF16 || L.out_dtype == CB_DTYPE_F16) && L.N % 8 == 0 && aligned16(L.out) &&
               L.out_sm % 8 == 0 && (L.batch == 1 || L.out_sb % 8 == 0))
                  ? 1
                  : 0;
  Workspace ws = carve_workspace(L.workspace, grid);
  p.partials = static_cast<float*>(ws.partials);
  p.counters = ws.counters;
  p.status = ws.status;
  if (L.a_dtype == CB_DTYPE_BF16) return launch_dtype<__nv_bfloat16>(L, stream, TN, grid, stages, p);
  return launch_dtype<__half>(L, stream, TN, grid, stages, p);
}

}  // namespace cb
