// Warp-cooperative selection over ordered 64-bit candidate keys (see make_key
// in cvs_device.cuh: larger key = higher score, ties broken by the smaller row).
//
// warp_kth_key finds the k-th largest of m unique keys with an MSB-first radix
// select (8-bit digits, one 256-bin shared-memory histogram per warp). It stops
// as soon as the bucket holding the k-th key is fully selected, so on real
// score distributions it takes 2-4 passes over the keys instead of 8.
//
// This replaces the reference's per-lane replace-the-minimum list
// (cuda_vector_search/csrc/kernels.cu:187-275) for every list longer than a
// warp: per-chunk candidate lists, per-query candidate buffers and the final
// cross-chunk merge.
#pragma once

#include <cstdint>

namespace cvs {

constexpr unsigned kFullMask = 0xffffffffu;

__device__ __forceinline__ uint64_t shfl_u64(uint64_t v, int src) {
  const uint32_t lo = __shfl_sync(kFullMask, static_cast<uint32_t>(v), src);
  const uint32_t hi = __shfl_sync(kFullMask, static_cast<uint32_t>(v >> 32), src);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const uint64_t o = shfl_u64(v, (threadIdx.x & 31) ^ off);
    v = o < v ? o : v;
  }
  return v;
}

// Key accessor over a contiguous array (shared or global memory).
struct ContigKeys {
  const uint64_t* p;
  __device__ __forceinline__ uint64_t operator()(int i) const { return p[i]; }
};

// Returns the k-th largest of the m keys produced by acc(0..m-1). Requires
// 1 <= k <= m and unique keys. `hist` is this warp's 256-entry shared scratch.
// Must be called by all 32 lanes of the warp with identical arguments.
template <class Acc>
__device__ uint64_t warp_kth_key(const Acc& acc, int m, int k, uint32_t* hist, int lane) {
  uint64_t prefix = 0;
  uint64_t pmask = 0;
  int want = k;  // rank of the target among keys that match `prefix`
#pragma unroll 1
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = lane; i < 256; i += 32) hist[i] = 0u;
    __syncwarp();
    for (int i0 = 0; i0 < m; i0 += 128) {  // four loads in flight per lane
      uint64_t key[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u + lane;
        key[u] = i < m ? acc(i) : 0ull;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + 32 * u + lane < m && (key[u] & pmask) == prefix)
          atomicAdd(&hist[(key[u] >> shift) & 255u], 1u);
      }
    }
    __syncwarp();
    // Lane l owns bins 255-8l .. 248-8l, visited from the highest digit down.
    uint32_t c[8];
    uint32_t tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = hist[255 - 8 * lane - j];
      tot += c[j];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t v = __shfl_up_sync(kFullMask, incl, off);
      if (lane >= off) incl += v;
    }
    const uint32_t excl = incl - tot;
    const bool mine = excl < static_cast<uint32_t>(want) && static_cast<uint32_t>(want) <= incl;
    const unsigned owner = __ballot_sync(kFullMask, mine);
    int digit = 0;
    uint32_t above = 0, in_bin = 0;
    if (mine) {
      uint32_t run = excl;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (in_bin == 0 && run + c[j] >= static_cast<uint32_t>(want)) {
          digit = 255 - 8 * lane - j;
          above = run;
          in_bin = c[j];
        }
        run += c[j];
      }
    }
    const int src = __ffs(owner) - 1;
    digit = __shfl_sync(kFullMask, digit, src);
    above = __shfl_sync(kFullMask, above, src);
    in_bin = __shfl_sync(kFullMask, in_bin, src);
    want -= static_cast<int>(above);
    prefix |= static_cast<uint64_t>(digit) << shift;
    pmask |= static_cast<uint64_t>(255u) << shift;
    if (in_bin == static_cast<uint32_t>(want)) {
      // Every key in this bucket is selected: the k-th key is its smallest.
      uint64_t mn = ~0ull;
      for (int i = lane; i < m; i += 32) {
        const uint64_t key = acc(i);
        if ((key & pmask) == prefix && key < mn) mn = key;
      }
      __syncwarp();
      return warp_min_u64(mn);
    }
  }
  __syncwarp();
  return prefix;  // all 64 bits fixed: this is the k-th key itself
}

// Keeps, in place and in their original order, the keys of list[0..m) that are
// >= kth. Returns how many were kept. Whole warp.
__device__ __forceinline__ int warp_compact_ge(uint64_t* list, int m, uint64_t kth, int lane) {
  int base = 0;
  for (int i0 = 0; i0 < m; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t key = i < m ? list[i] : 0ull;
    const bool keep = i < m && key >= kth;
    const unsigned bal = __ballot_sync(kFullMask, keep);
    if (keep) list[base + __popc(bal & ((1u << lane) - 1u))] = key;
    base += __popc(bal);
  }
  __syncwarp();
  return base;
}

// A lower bound on the query's k-th best from n published per-list values
// row[0..n) (ordered score bits, 0 = none), computed by the whole warp. If k
// lists hold a score >= v, at least k rows score >= v, so any v with at least k
// published values >= v bounds the query's k-th best from below; the best such
// v is the k-th largest published value. Each lane loads up to PER_LANE values
// in one round trip; a bisection on the ordered bits between the smallest and
// the largest published value (the smallest qualifies: k or more values are at
// or above it) then finds that value to within 2^-16 of the range -- stopping
// early only returns a slightly lower, still valid, bound. Returns 0 when fewer
// than k lists have published. Requires n <= 32 * PER_LANE.
template <int PER_LANE>
__device__ __forceinline__ void load_tops(const uint32_t* row, int n, int lane, uint32_t (&v)[PER_LANE]) {
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int i = lane + 32 * j;
    v[j] = 0;
    if (i < n) asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v[j]) : "l"(row + i));
  }
}

template <int PER_LANE>
__device__ __forceinline__ uint32_t kth_of_tops(const uint32_t (&v)[PER_LANE], int k) {
  uint32_t cnt = 0, mx = 0, mn = 0xFFFFFFFFu;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    cnt += v[j] != 0 ? 1u : 0u;
    mx = max(mx, v[j]);
    mn = min(mn, v[j] != 0 ? v[j] : 0xFFFFFFFFu);
  }
  if (__reduce_add_sync(kFullMask, cnt) < static_cast<uint32_t>(k)) return 0;
  uint32_t lo = __reduce_min_sync(kFullMask, mn);  // count(>= lo) >= k
  uint32_t hi = __reduce_max_sync(kFullMask, mx);  // the answer is <= hi
#pragma unroll 1
  for (int step = 0; step < 16 && lo < hi; ++step) {
    const uint32_t mid = lo + (hi - lo + 1) / 2;
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j) c += v[j] >= mid ? 1u : 0u;
    if (__reduce_add_sync(kFullMask, c) >= static_cast<uint32_t>(k)) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int PER_LANE>
__device__ __forceinline__ uint32_t warp_kth_top(const uint32_t* row, int n, int k, int lane) {
  uint32_t v[PER_LANE];
  load_tops<PER_LANE>(row, n, lane, v);
  return kth_of_tops<PER_LANE>(v, k);
}

}  // namespace cvs
