// Shared pieces of the split-K ("stream-K") GEMM kernels.
//
// Work decomposition: an output tile is (batch h, 128 rows of N, TN tokens of M).
// Each tile needs KB k-blocks. All tiles' k-blocks are laid end to end
// (tile-major) and cut into G equal contiguous ranges, one per CTA, so every SM
// streams the same number of weight bytes whatever the shape. A tile whose
// k-blocks fall in one CTA's range is finished by that CTA; a tile cut by a
// range boundary is reduced deterministically. The tile's first contributor
// (lowest CTA index; its range ends in the tile) keeps its part in tensor
// memory; every other contributor writes its part to its own slot and bumps
// the tile's arrival counter, keeping the value its atomic returned. The first
// contributor polls that counter for a short bounded time and, when every
// part is in, sums the slots in CTA order and runs the epilogue. If the poll
// expires it publishes its part and bumps the counter too, and whichever
// contributor's bump completes the count (the first at once, or another one
// when it checks its returned value at the end of its range) reduces the tile
// from the slots in the same order. No CTA ever waits for one that may not be
// running, and the bits do not depend on who reduces.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cb200.h"

namespace cb {

// How long the first contributor of a cut tile polls for the other
// contributors' parts before it publishes its own part instead. Contributors
// that are resident together finish well inside it; when some are not (another
// kernel holds SMs), the last one to arrive reduces the tile, so no CTA ever
// waits on one that may not be running.
constexpr unsigned long long kFirstPollNs = 10000;

struct StreamK {
  long long total;  // tiles * kb_per_tile
  int grid;         // number of CTAs
  int kb_per_tile;
  // first contributor's poll limit: kFirstPollNs, or 0 (no poll at all) under
  // the test hook that forces the last-arriver path (cb_debug_force_last_arriver)
  unsigned long long first_poll_ns;

  __host__ __device__ long long start(int c) const { return static_cast<long long>(c) * total / grid; }
  // CTA whose range holds global k-block g.
  __host__ __device__ int owner(long long g) const {
    return static_cast<int>(((g + 1) * grid - 1) / total);
  }
  // Slot kind of CTA c's contribution to tile t: 0 if the contribution is the
  // first segment of c's range, 1 if it is the last one.
  __host__ __device__ int kind(int c, long long tile) const {
    return start(c) >= tile * kb_per_tile ? 0 : 1;
  }
};

// (batch h, n-tile, m-tile) of a tile index (tiles ordered batch-major, m-tile
// fastest). 32-bit divisions when the index fits: the epilogues decode tiles
// per segment, and with one k-block per tile (short K) 64-bit divisions would
// dominate their time.
__device__ __forceinline__ void split_tile(long long tile, int m_tiles, int n_tiles, int& h, int& nt, int& mt) {
  if (tile < 0x7fffffffLL) {
    const unsigned t = static_cast<unsigned>(tile), ml = static_cast<unsigned>(m_tiles);
    const unsigned nl = static_cast<unsigned>(n_tiles);
    const unsigned r = t / ml;
    mt = static_cast<int>(t - r * ml);
    const unsigned hh = r / nl;
    nt = static_cast<int>(r - hh * nl);
    h = static_cast<int>(hh);
    return;
  }
  mt = static_cast<int>(tile % m_tiles);
  const long long r = tile / m_tiles;
  nt = static_cast<int>(r % n_tiles);
  h = static_cast<int>(r / n_tiles);
}

// (batch, n-tile, m-tile) of consecutive tiles, advanced without division (an
// epilogue walks its range one tile per segment).
struct TileCursor {
  int h, nt, mt;
  __device__ __forceinline__ void seek(long long tile, int m_tiles, int n_tiles) {
    split_tile(tile, m_tiles, n_tiles, h, nt, mt);
  }
  __device__ __forceinline__ void next(int m_tiles, int n_tiles) {
    if (++mt == m_tiles) {
      mt = 0;
      if (++nt == n_tiles) {
        nt = 0;
        ++h;
      }
    }
  }
};

// First and last contributor of a cut tile, packed as c_first | c_last << 32.
// Out of line so that its two 64-bit divisions run only for cut tiles (at most
// the first and the last segment of a CTA's range), never speculatively.
static __device__ __noinline__ long long cut_contributors(long long total, int grid, int kb_per_tile, long long tile) {
  const long long first_kb = tile * kb_per_tile;
  const long long last_kb = first_kb + kb_per_tile - 1;
  const long long cf = ((first_kb + 1) * grid - 1) / total;
  const long long cl = ((last_kb + 1) * grid - 1) / total;
  return cf | (cl << 32);
}

// Coordinates of a k-block, advanced without division (the producer walks its
// range one k-block at a time; 64-bit divisions per step would dominate it).
struct KCursor {
  int kb, h, nt, mt;
  template <class P>
  __device__ __forceinline__ void seek(const P& p, long long g) {
    if (g < 0x7fffffffLL) {  // 32-bit divisions are several times cheaper
      const unsigned gg = static_cast<unsigned>(g), kbt = static_cast<unsigned>(p.kb_per_tile);
      const unsigned tile = gg / kbt, mtl = static_cast<unsigned>(p.m_tiles), ntl = static_cast<unsigned>(p.n_tiles);
      kb = static_cast<int>(gg - tile * kbt);
      mt = static_cast<int>(tile % mtl);
      const unsigned r = tile / mtl;
      nt = static_cast<int>(r % ntl);
      h = static_cast<int>(r / ntl);
      return;
    }
    const long long tile = g / p.kb_per_tile;
    kb = static_cast<int>(g - tile * p.kb_per_tile);
    mt = static_cast<int>(tile % p.m_tiles);
    const long long r = tile / p.m_tiles;
    nt = static_cast<int>(r % p.n_tiles);
    h = static_cast<int>(r / p.n_tiles);
  }
  template <class P>
  __device__ __forceinline__ void next(const P& p) {
    if (++kb == p.kb_per_tile) {
      kb = 0;
      if (++mt == p.m_tiles) {
        mt = 0;
        if (++nt == p.n_tiles) {
          nt = 0;
          ++h;
        }
      }
    }
  }
};

// Output element store for the runtime-selected dtype.
__device__ __forceinline__ void store_elem(void* out, int dtype, long long idx, float v) {
  if (dtype == CB_DTYPE_BF16) {
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  } else if (dtype == CB_DTYPE_F16) {
    reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
  } else {
    reinterpret_cast<float*>(out)[idx] = v;
  }
}

__device__ __forceinline__ float load_elem(const void* p, int dtype, long long idx) {
  if (dtype == CB_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
  if (dtype == CB_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(p)[idx]);
  return reinterpret_cast<const float*>(p)[idx];
}

}  // namespace cb
