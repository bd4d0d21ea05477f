// W4A16 for one or two tokens: int4 x 16-bit activations on the integer dot
// product units (dp4a) instead of the tensor cores.
//
// Math (kernel_batched_w4a16_simple, profiling/bench_l2_barrier.py:36-85, with
// group scales; the per-output-channel scale is the single-group case):
//   out[h, m, n] = sum_k a[h, m, k] * q[h, k, n] * s[h, k / G, n]
// computed as
//   out = 2^-e_m * sum_{k-blocks j} s[j, n] * S_j,   S_j = sum_{k in j} q[k, n] * X[m, k]
// where X = rint(a * 2^e_m) is a 15-bit fixed-point image of the token's row
// (e_m from the amax of the row's part that the CTA sums, so that 2^13 <=
// amax * 2^e_m < 2^14: each element's rounding error is half a step, at most
// 2^-14 of that amax, which is at most the row's amax), split exactly into two
// int8 halves X = 256 hi + lo. Each S_j is an exact int32 sum of dp4a products;
// the weights enter dp4a as the unsigned bytes q + 8 of the native nibbles
// (XOR 8), and 8 * sum X over the k-block is subtracted back. The group scale
// is applied per k-block in fp32 (per-channel scales once at the end, as the
// reference applies its scale to the fp32 accumulator, :80-82). Compared with
// the tensor-core kernel, which rounds q * s to the activation dtype before
// its MMAs, this path keeps the weights exact.
//
// Why: a decode step with one or two tokens has 2 FLOP per weight byte pair;
// on the tensor cores the MMA costs the same for N = 1 as for N = 128, while
// here every instruction does useful work: per 8 KiB k-block tile a thread
// (one weight row) issues 4 16-byte loads and ~100 integer instructions, well
// within the SM's issue rate at the HBM byte rate.
//
// Layout: a CTA of 128 threads owns one (batch entry, 128-row n-tile) and a
// contiguous range of k-blocks (split-K over the CTAs of a tile when there
// are few tiles), or, when there are more tiles than CTA slots, several
// n-tiles of one batch entry with all their k-blocks (the reference's gate
// shapes, H = 128, K = 128, W = 128 MB: 14.8 -> 11.8 us at T = 1). Every CTA
// first reduces each token's amax over its own k-range (the whole row unless
// K is split: a split CTA reads 1/ksplit of the row instead of all of it, and
// the second read of its part hits L1), then writes the fixed-point halves of
// its own k-range into shared memory, permuted to the nibble order of the
// native words (k0,k4,k1,k5 | k2,k6,k3,k7 per 8 k). The main loop streams the
// weight rows with 16-byte global loads, up to four k-blocks in flight. A split tile
// is summed deterministically: each CTA writes its fp32 partial to its own
// workspace slot and bumps the tile's counter; the CTA that completes the
// count sums the slots in split order and stores (nobody waits).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "cb_gemm_common.cuh"
#include "cb_internal.h"
#include "cb_ptx.cuh"

namespace cb {
namespace {

constexpr int kGvThreads = 128;
constexpr int kGvRows = 128;       // weight rows (n) per tile
constexpr int kGvKb = 128;         // k per k-block (one native tile)
constexpr int kGvTileBytes = kGvRows * kGvKb / 2;
constexpr long long kGvNoL1Bytes = 64ll << 20;  // packed weights from which loads bypass L1

struct GvParams {
  const void* a;
  int a_dtype;
  long long a_sb, a_sm;
  const uint8_t* w;
  const void* scales;
  int scale_dtype;
  long long s_sb, s_sg;
  int kb_per_group;
  int scale_at_end;  // group size >= K: one scale per channel, applied to the sum
  void* out;
  int out_dtype;
  long long out_sb, out_sm;
  int M, N, K, KB, n_tiles, ksplit;
  int tpc, ctas_per_h;  // n-tiles per CTA (1 when K is split), CTAs per batch entry
  int a_vec;  // rows 16-byte aligned and K % 8 == 0: activations read as 16-byte vectors
  int w_no_l1;      // large weights: stream them past L1 (ld.global.nc.L1::no_allocate)
  float* partials;  // [grid][M][128] (split-K only)
  int* counters;    // [tiles] (split-K only)
};

__device__ __forceinline__ float act_f32(const void* a, int dtype, long long i) {
  return dtype == CB_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a)[i])
                                : __half2float(reinterpret_cast<const __half*>(a)[i]);
}

__device__ __forceinline__ int dp4a_us(uint32_t w_u8, uint32_t x_s8, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_u8), "r"(x_s8), "r"(c));
  return d;
}

// 16-byte load that does not allocate in L1. For large weight sets it is
// faster (22528^2: 70.6 -> 65.7 us; 16384^2: 37.2 -> 35.4 us; the gate shape at
// W = 320 MB: 26.1 -> 24.6 us); below ~64 MiB of packed weights the cached
// load is (8192^2: 12.8 vs 13.1 us; W = 128 MB: 11.7 vs 13.1 us): the two
// 16-byte chunks of a row that share a 32-byte sector are read by different
// load instructions, and the second hits L1 only if the first allocated it.
__device__ __forceinline__ uint4 ld_na16(const void* ptr) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(ptr));
  return v;
}

__device__ __forceinline__ uint32_t pack4(int b0, int b1, int b2, int b3) {
  return (static_cast<uint32_t>(b0) & 0xFFu) | ((static_cast<uint32_t>(b1) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(b2) & 0xFFu) << 16) | ((static_cast<uint32_t>(b3) & 0xFFu) << 24);
}

// TM: tokens (1 or 2); DEPTH: items of weights in flight per thread (4 for
// long ranges, 1 when a CTA has one or two items and occupancy matters more);
// MULTI: the CTA may own several n-tiles (no K split). The one-tile variant
// keeps the per-item bookkeeping out of the loop (1-10 % faster on split-K
// shapes than the general one).
template <int TM, int DEPTH, bool MULTI>
__global__ void __launch_bounds__(kGvThreads) w4a16_gemv_kernel(const GvParams p) {
  extern __shared__ __align__(16) uint8_t gv_smem[];
  __shared__ float red[kGvThreads / 32][TM];
  __shared__ int sh_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ks = static_cast<int>(blockIdx.x % p.ksplit);
  const long long q = blockIdx.x / p.ksplit;  // (batch entry, tile group); the tile itself when K is split
  const int h = static_cast<int>(q / p.ctas_per_h);
  const int nt0 = static_cast<int>(q % p.ctas_per_h) * p.tpc;
  const int ntl = MULTI ? min(p.tpc, p.n_tiles - nt0) : 1;  // n-tiles of this CTA
  const int kb0 = static_cast<int>(static_cast<long long>(ks) * p.KB / p.ksplit);
  const int kb1 = static_cast<int>(static_cast<long long>(ks + 1) * p.KB / p.ksplit);
  const int nkb = kb1 - kb0;
  // shared memory: per (k-block, group of 8 k, token) one uint4 {hiA, hiB, loA, loB},
  // then per (k-block, token) the int sum of X
  uint4* xw = reinterpret_cast<uint4*>(gv_smem);
  int* xsum = reinterpret_cast<int*>(gv_smem + static_cast<size_t>(nkb) * 16 * TM * sizeof(uint4));

  pdl_launch_dependents();
  // The weights and scales are not written by the preceding kernel: the
  // first DEPTH k-blocks of this thread's row are requested before the
  // dependency wait, so they stream in while the activations are prepared.
  const int r = tid;
  const int swz = (r >> 1) & 3;
  // this thread's row of the CTA's first n-tile: 64 bytes per k-block tile
  const uint8_t* wrow0 = p.w + ((static_cast<long long>(h) * p.n_tiles + nt0) * p.KB) * kGvTileBytes + r * 64;
  auto load_scale = [&](int kb, int n) -> float {
    if (p.scale_at_end || n >= p.N) return 1.0f;
    const long long idx = h * p.s_sb + static_cast<long long>(kb / p.kb_per_group) * p.s_sg + n;
    return load_elem(p.scales, p.scale_dtype, idx);
  };
  // the CTA's work is nit = ntl * nkb items (n-tile t, k-block kbl) in
  // t-major order, one weight pipeline across its n-tiles
  const int nit = ntl * nkb;
  float acc[TM];
#pragma unroll
  for (int m = 0; m < TM; ++m) acc[m] = 0.0f;
  // DEPTH items of the row in flight: buffer d holds item it + d of the
  // current round and is refilled with item it + d + DEPTH as soon as it has
  // been consumed. (it_t, it_k) is the (n-tile, k-block) of the next item to
  // request.
  uint4 buf[DEPTH][4];
  float sbuf[DEPTH];
  int it_t = 0, it_k = 0;
  auto issue = [&](uint4 (&dst)[4], float& sdst) {
    if (MULTI ? it_t < ntl : it_k < nkb) {
      const int tt = MULTI ? it_t : 0;
      const uint4* src =
          reinterpret_cast<const uint4*>(wrow0 + (static_cast<long long>(tt) * p.KB + kb0 + it_k) * kGvTileBytes);
#pragma unroll
      for (int c = 0; c < 4; ++c)  // logical chunk c sits at position c ^ swz
        dst[c] = p.w_no_l1 ? ld_na16(src + (c ^ swz)) : __ldg(src + (c ^ swz));
      sdst = load_scale(kb0 + it_k, (nt0 + tt) * kGvRows + r);
      if (!MULTI)
        ++it_k;
      else if (++it_k == nkb)
        it_k = 0, ++it_t;
    }
  };
#pragma unroll
  for (int d = 0; d < DEPTH; ++d) issue(buf[d], sbuf[d]);
  pdl_wait_primary();

  // 1. per-token amax over this CTA's k-range -> fixed-point exponent (the
  // whole row unless K is split; the parts of a split tile are scaled by
  // their own 2^-e, exactly, before they are summed)
  const int k_lo = kb0 * kGvKb, k_hi = min(kb1 * kGvKb, p.K);
  const char* abase = static_cast<const char*>(p.a);
  float amax[TM];
#pragma unroll
  for (int m = 0; m < TM; ++m) {
    amax[m] = 0.0f;
    if (m < p.M) {
      const long long off = h * p.a_sb + static_cast<long long>(m) * p.a_sm;
      if (p.a_vec) {
        // eight 16-bit values per load, several loads in flight per thread
        const uint4* av = reinterpret_cast<const uint4*>(abase + off * 2);
        const int nvec = k_hi / 8;
#pragma unroll(DEPTH == 1 ? 1 : 8)
        for (int i = k_lo / 8 + tid; i < nvec; i += kGvThreads) {
          const uint4 u = __ldg(av + i);
          const uint32_t wds[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float lo = p.a_dtype == CB_DTYPE_BF16 ? __uint_as_float(wds[j] << 16)
                                                         : __half2float(__ushort_as_half(static_cast<unsigned short>(wds[j] & 0xFFFFu)));
            const float hi = p.a_dtype == CB_DTYPE_BF16 ? __uint_as_float(wds[j] & 0xFFFF0000u)
                                                         : __half2float(__ushort_as_half(static_cast<unsigned short>(wds[j] >> 16)));
            amax[m] = fmaxf(amax[m], fmaxf(fabsf(lo), fabsf(hi)));
          }
        }
      } else {
        for (int k = k_lo + tid; k < k_hi; k += kGvThreads)
          amax[m] = fmaxf(amax[m], fabsf(act_f32(abase, p.a_dtype, off + k)));
      }
    }
    for (int o = 16; o > 0; o >>= 1) amax[m] = fmaxf(amax[m], __shfl_xor_sync(0xffffffffu, amax[m], o));
    if (lane == 0) red[warp][m] = amax[m];
  }
  __syncthreads();
  int ex[TM];
#pragma unroll
  for (int m = 0; m < TM; ++m) {
    float v = red[0][m];
#pragma unroll
    for (int w = 1; w < kGvThreads / 32; ++w) v = fmaxf(v, red[w][m]);
    int E = 0;
    if (v > 0.0f) frexpf(v, &E);  // v = f * 2^E, f in [0.5, 1)
    ex[m] = v > 0.0f ? 14 - E : 0;  // v * 2^ex in [2^13, 2^14)
  }

  // 2. fixed-point halves of this CTA's k-range, in the native word order.
  // Rounds of kGvRounds x 128 groups: every 16-byte activation load of a batch
  // of rounds is issued before any is used. Every lane runs every round (the
  // k-block sums are 16-lane shuffles); lanes past the range form whole 16-lane
  // groups and write nothing.
  // loads in flight per thread: more for long ranges with few tokens; one where
  // occupancy (registers) matters more (one or two k-blocks per CTA)
  constexpr int kGvRounds = DEPTH == 1 ? 1 : TM == 1 ? 4 : 2;
  const int ngroups = nkb * 16;
  for (int base0 = 0; base0 < ngroups; base0 += kGvRounds * kGvThreads) {
    uint4 raw[kGvRounds][TM];
#pragma unroll
    for (int u = 0; u < kGvRounds; ++u) {
      const int gi = base0 + u * kGvThreads + tid;
      const int kbase = (kb0 + (gi >> 4)) * kGvKb + (gi & 15) * 8;
#pragma unroll
      for (int m = 0; m < TM; ++m) {
        raw[u][m] = make_uint4(0u, 0u, 0u, 0u);
        if (gi < ngroups && m < p.M && p.a_vec && kbase + 8 <= p.K)
          raw[u][m] = __ldg(reinterpret_cast<const uint4*>(
              abase + (h * p.a_sb + static_cast<long long>(m) * p.a_sm + kbase) * 2));
      }
    }
#pragma unroll
    for (int u = 0; u < kGvRounds; ++u) {
      const int gi = base0 + u * kGvThreads + tid;
      const bool valid = gi < ngroups;
      const int kbl = gi >> 4, g8 = gi & 15;
      const int kbase = (kb0 + kbl) * kGvKb + g8 * 8;
#pragma unroll
      for (int m = 0; m < TM; ++m) {
        int hi[8], lo[8];
        int xs = 0;
        const long long off = h * p.a_sb + static_cast<long long>(m) * p.a_sm;
        float vals[8];
        if (p.a_vec) {
          const uint32_t wds[4] = {raw[u][m].x, raw[u][m].y, raw[u][m].z, raw[u][m].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            vals[2 * j] = p.a_dtype == CB_DTYPE_BF16
                              ? __uint_as_float(wds[j] << 16)
                              : __half2float(__ushort_as_half(static_cast<unsigned short>(wds[j] & 0xFFFFu)));
            vals[2 * j + 1] = p.a_dtype == CB_DTYPE_BF16
                                  ? __uint_as_float(wds[j] & 0xFFFF0000u)
                                  : __half2float(__ushort_as_half(static_cast<unsigned short>(wds[j] >> 16)));
          }
          if (kbase + 8 > p.K) {  // a ragged last group (K % 8 != 0 cannot occur here: a_vec needs K % 8 == 0)
#pragma unroll
            for (int j = 0; j < 8; ++j) vals[j] = 0.0f;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            vals[j] = (valid && m < p.M && kbase + j < p.K) ? act_f32(abase, p.a_dtype, off + kbase + j) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int X = __float2int_rn(ldexpf(vals[j], ex[m]));
          const int hj = (X + 128) >> 8;  // round(X / 256), ties up
          hi[j] = hj;
          lo[j] = X - 256 * hj;           // in [-128, 127]
          xs += X;
        }
        // word A holds k0, k4, k1, k5; word B holds k2, k6, k3, k7
        if (valid)
          xw[(kbl * 16 + g8) * TM + m] = make_uint4(pack4(hi[0], hi[4], hi[1], hi[5]), pack4(hi[2], hi[6], hi[3], hi[7]),
                                                    pack4(lo[0], lo[4], lo[1], lo[5]), pack4(lo[2], lo[6], lo[3], lo[7]));
        // sum of X over the k-block: the 16 groups of a k-block are 16 consecutive lanes
        for (int o = 8; o > 0; o >>= 1) xs += __shfl_xor_sync(0xffffffffu, xs, o);
        if (valid && (lane & 15) == 0) xsum[kbl * TM + m] = xs;
      }
    }
  }
  __syncthreads();

  // 4. epilogue of n-tile t: out = v * s_channel * 2^-e
  auto finish = [&](const float (&v)[TM], int t, bool apply_ex) {
    const int n = (nt0 + t) * kGvRows + r;
    if (n >= p.N) return;
    const float sc = p.scale_at_end ? load_elem(p.scales, p.scale_dtype, h * p.s_sb + n) : 1.0f;
#pragma unroll
    for (int m = 0; m < TM; ++m) {
      if (m < p.M) {
        float f = p.scale_at_end ? __fmul_rn(v[m], sc) : v[m];
        if (apply_ex) f = ldexpf(f, -ex[m]);
        store_elem(p.out, p.out_dtype, h * p.out_sb + static_cast<long long>(m) * p.out_sm + n, f);
      }
    }
  };

  // 3. the weight stream (its first DEPTH items were issued before the
  // dependency wait); (ct, kbl) is the item being summed
  int ct = 0, kbl = 0;
  for (int it0 = 0; it0 < nit; it0 += DEPTH) {
#pragma unroll
    for (int d = 0; d < DEPTH; ++d) {
      if (it0 + d < nit) {
        int dh[TM], dl[TM];
#pragma unroll
        for (int m = 0; m < TM; ++m) dh[m] = dl[m] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // logical chunk c: k = 32c .. 32c + 31
          const uint4 v = buf[d][c];
          const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t wu = words[wi] ^ 0x88888888u;  // nibble q & 15 -> q + 8
            const uint32_t wa = wu & 0x0F0F0F0Fu, wb = (wu >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int m = 0; m < TM; ++m) {
              const uint4 x = xw[(kbl * 16 + c * 4 + wi) * TM + m];
              dh[m] = dp4a_us(wa, x.x, dh[m]);
              dh[m] = dp4a_us(wb, x.y, dh[m]);
              dl[m] = dp4a_us(wa, x.z, dl[m]);
              dl[m] = dp4a_us(wb, x.w, dl[m]);
            }
          }
        }
        const float sc = sbuf[d];
#pragma unroll
        for (int m = 0; m < TM; ++m) {
          const int S = 256 * dh[m] + dl[m] - 8 * xsum[kbl * TM + m];  // exact: |S| < 2^24
          acc[m] = __fmaf_rn(sc, static_cast<float>(S), acc[m]);
        }
        issue(buf[d], sbuf[d]);
        if (MULTI && ++kbl == nkb) {  // n-tile ct complete
          finish(acc, ct, true);
#pragma unroll
          for (int m = 0; m < TM; ++m) acc[m] = 0.0f;
          kbl = 0;
          ++ct;
        } else if (!MULTI) {
          ++kbl;
        }
      }
    }
  }
  if (MULTI) return;
  if (p.ksplit == 1) {
    finish(acc, 0, true);
    return;
  }
  // split tile (one n-tile per CTA): deterministic sum of the parts
  const long long tile = q;
  float* slot = p.partials + static_cast<long long>(blockIdx.x) * TM * kGvRows;
#pragma unroll
  for (int m = 0; m < TM; ++m) slot[m * kGvRows + r] = ldexpf(acc[m], -ex[m]);
  __threadfence();
  __syncthreads();
  if (tid == 0) sh_last = atomicAdd(&p.counters[tile], 1) == p.ksplit - 1 ? 1 : 0;
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  float sum[TM];
#pragma unroll
  for (int m = 0; m < TM; ++m) sum[m] = 0.0f;
  for (int k2 = 0; k2 < p.ksplit; ++k2) {
    const float* src = p.partials + (tile * p.ksplit + k2) * TM * kGvRows;
#pragma unroll
    for (int m = 0; m < TM; ++m) sum[m] = __fadd_rn(sum[m], __ldcg(src + m * kGvRows + r));
  }
  finish(sum, 0, false);
  if (tid == 0) p.counters[tile] = 0;  // next launch starts from zero
}

template <int TM, int DEPTH, bool MULTI>
int launch_tm(const GvParams& g, int grid, size_t smem, cudaStream_t stream) {
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && (configured_dev != dev || configured_smem < smem)) {
    if (cudaFuncSetAttribute(w4a16_gemv_kernel<TM, DEPTH, MULTI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return CB_ERR_CUDA;
    configured_dev = dev;
    configured_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, w4a16_gemv_kernel<TM, DEPTH, MULTI>, g));
}

}  // namespace

bool w4a16_gemv_eligible(const W4A16Launch& L) { return L.M >= 1 && L.M <= kGemvMaxTokens; }

int launch_w4a16_gemv(const W4A16Launch& L, cudaStream_t stream) {
  GvParams g = {};
  g.a = L.a;
  g.a_dtype = L.a_dtype;
  g.a_sb = L.a_sb;
  g.a_sm = L.a_sm;
  g.w = L.w;
  g.scales = L.scales;
  g.scale_dtype = L.scale_dtype;
  g.s_sb = L.s_sb;
  g.s_sg = L.s_sg;
  g.scale_at_end = L.group_size >= L.K ? 1 : 0;
  g.kb_per_group = static_cast<int>(L.group_size / kGvKb) > 0 ? static_cast<int>(L.group_size / kGvKb) : 1;
  g.out = L.out;
  g.out_dtype = L.out_dtype;
  g.out_sb = L.out_sb;
  g.out_sm = L.out_sm;
  g.M = static_cast<int>(L.M);
  g.N = static_cast<int>(L.N);
  g.K = static_cast<int>(L.K);
  g.KB = static_cast<int>((L.K + kGvKb - 1) / kGvKb);
  g.n_tiles = static_cast<int>((L.N + kGvRows - 1) / kGvRows);
  g.w_no_l1 = L.batch * L.N * L.K / 2 >= kGvNoL1Bytes ? 1 : 0;
  g.a_vec = (L.K % 8 == 0 && aligned16(L.a) && (L.a_sb * 2) % 16 == 0 && (L.a_sm * 2) % 16 == 0) ? 1 : 0;
  const long long tiles = L.batch * g.n_tiles;
  if (tiles > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  // Split K only when the tiles alone would leave SMs idle, and only as far as
  // the workspace's slots and counters allow. With more tiles than CTA slots,
  // a CTA takes several n-tiles of one batch entry (its activation prologue
  // then serves all of them, and its weight stream runs across them), as many
  // CTAs per batch entry as fill kGemvCtasPerSm CTAs per SM.
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const long long slots = static_cast<long long>(kGemvCtasPerSm) * sms;
  long long ksplit = 1;
  if (tiles < slots) {
    ksplit = slots / tiles;  // grid <= slots
    if (ksplit > g.KB) ksplit = g.KB;
    if (ksplit < 1) ksplit = 1;
  }
  g.ksplit = static_cast<int>(ksplit);
  long long cph = g.n_tiles;
  if (tiles > slots) {
    cph = slots / L.batch;
    if (cph < 1) cph = 1;
    if (cph > g.n_tiles) cph = g.n_tiles;
  }
  g.tpc = static_cast<int>((g.n_tiles + cph - 1) / cph);
  g.ctas_per_h = static_cast<int>((g.n_tiles + g.tpc - 1) / g.tpc);
  const long long grid = L.batch * g.ctas_per_h * ksplit;
  if (grid > 0x7fffffffLL) return CB_ERR_TOO_LARGE;
  if (ksplit > 1) {
    const size_t need = workspace_need(static_cast<int>(grid), static_cast<size_t>(kGemvMaxTokens) * kGvRows * sizeof(float));
    if (L.workspace == nullptr || L.workspace_bytes < need) return CB_ERR_WORKSPACE;
    Workspace ws = carve_workspace(L.workspace, static_cast<int>(grid));
    g.partials = static_cast<float*>(ws.partials);
    g.counters = ws.counters;
  }
  const int kb_max = static_cast<int>((g.KB + ksplit - 1) / ksplit);
  const int TM = g.M <= 1 ? 1 : 2;
  const size_t smem = static_cast<size_t>(kb_max) * 16 * TM * 16 + static_cast<size_t>(kb_max) * TM * 4;
  if (smem > 200 * 1024) return CB_ERR_UNSUPPORTED;
  const bool deep = static_cast<long long>(kb_max) * g.tpc > 2;
  const int gi = static_cast<int>(grid);
  if (g.tpc > 1) {  // several n-tiles per CTA (ksplit == 1)
    if (TM == 1) return deep ? launch_tm<1, 4, true>(g, gi, smem, stream) : launch_tm<1, 1, true>(g, gi, smem, stream);
    return deep ? launch_tm<2, 4, true>(g, gi, smem, stream) : launch_tm<2, 1, true>(g, gi, smem, stream);
  }
  if (TM == 1) return deep ? launch_tm<1, 4, false>(g, gi, smem, stream) : launch_tm<1, 1, false>(g, gi, smem, stream);
  return deep ? launch_tm<2, 4, false>(g, gi, smem, stream) : launch_tm<2, 1, false>(g, gi, smem, stream);
}

}  // namespace cb
