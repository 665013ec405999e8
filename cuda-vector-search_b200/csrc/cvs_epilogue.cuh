// Epilogues of the tcgen05 score kernels (one-CTA and CTA-pair variants).
// Each sees, per call, 32 consecutive corpus scores of the thread's own query
// (TMEM lane = query, columns = corpus rows), loaded with one tcgen05.ld.
#pragma once

#include <type_traits>

#include "cvs_device.cuh"
#include "cvs_kernels.h"
#include "cvs_select.cuh"

namespace cvs {

// ---------------------------------------------------------------------------
// Epilogues. consume() sees 32 consecutive corpus scores of this thread's
// query (rows row0 .. row0+31, of which the first `nvalid` exist).
// ---------------------------------------------------------------------------

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Largest of the 32 scores: 17 three-input maxima in a depth-4 tree, so the
// per-chunk fast reject costs about half an instruction per score.
__device__ __forceinline__ float max32(const uint32_t (&r)[32]) {
  float m[11];
#pragma unroll
  for (int i = 0; i < 10; ++i)
    m[i] = fmax3(__uint_as_float(r[3 * i]), __uint_as_float(r[3 * i + 1]), __uint_as_float(r[3 * i + 2]));
  m[10] = fmaxf(__uint_as_float(r[30]), __uint_as_float(r[31]));
  const float a = fmax3(m[0], m[1], m[2]);
  const float b = fmax3(m[3], m[4], m[5]);
  const float c = fmax3(m[6], m[7], m[8]);
  return fmaxf(fmax3(a, b, c), fmaxf(m[9], m[10]));
}

// Rounds at which a query's bound is recomputed from the lists' published
// values: after tiles 0..7, then after every 16th tile. In each round one list
// per query (a rotating choice, spreading the work over the CTAs) does it,
// kDryRefreshers lists in dry rounds. Later refreshes tighten an already close
// bound little, and each one delays its warp's next drain -- with 16 drain
// warps per CTA pair behind one accumulator barrier, a slow warp stalls the
// MMA: every 16th tile instead of every 4th measured -5% at 4M x 768, b=1024,
// k=100 and -4% at C4 k=100, neutral elsewhere.
__device__ __forceinline__ bool tops_round(int t) { return t < 8 || (t & 15) == 15; }

// The r lists h, h+1, ..., h+r-1 (mod lists) refresh query q in round t, with
// h = r * q + a per-round offset: consecutive queries get consecutive windows,
// so the 32 queries of a drain warp put at most ceil(32 r / lists) + 1 refreshes
// on any one list (a multiplicative hash put up to 4-5 on some warps, and the
// slowest warp holds the accumulator for the next MMA): C4 k=100 -0.8%, C2
// -0.3%.
__device__ __forceinline__ bool tops_refresher(int q, int t, int list, int lists, int r) {
  const unsigned h = (static_cast<unsigned>(q) * static_cast<unsigned>(r) + static_cast<unsigned>(t) * 40503u) %
                     static_cast<unsigned>(lists);
  return (static_cast<unsigned>(list) + static_cast<unsigned>(lists) - h) % static_cast<unsigned>(lists) <
         static_cast<unsigned>(r);
}

// Refreshers per query in dry rounds: the epilogue idles there (a dry tile
// costs a few hundred cycles against several thousand of MMA per tile), and the
// first real tile needs every query's bound in place, so a refresher that runs
// late on one CTA must not leave its query without one.
constexpr int kDryRefreshers = 6;

// Shared per-query lower bound: the largest k-th-best score any list of this
// query has reached (ordered bits, 0 = none yet). Every list of the query --
// other column stripes of this CTA and other corpus segments -- holds k
// candidates at or above it, so the query's final k-th best is at least this
// high and a score strictly below it can be dropped by every list.
__device__ __forceinline__ float load_bound(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v ? score_of_bits(v) : -INFINITY;
}

__device__ __forceinline__ void publish_bound(uint32_t* p, float kth, uint32_t& published) {
  if (kth == -INFINITY) return;
  const uint32_t o = ordered_bits(kth);
  if (o > published) {
    atomicMax(p, o);
    published = o;
  }
}

// Plans with a single dry tile (at most two tiles per CTA: small corpora) have
// their first real tile ready right after the dry one, and a query that drains
// it before the other CTAs' refreshers have set its bound sends every column of
// its first chunks through the insertion path. With register lists such queries
// first poll the bound for up to kBoundPollCycles (~4 us); a timeout is not an
// error, the drain then runs without one. Measured: 20000 x 384, b = 32
// 0.041 -> 0.022 ms; 75000 x 384, b = 64, k = 32 0.069 -> 0.033 ms; 20000 x 768,
// b = 256 (CTA pairs) 0.053 -> 0.035 ms. Not in buffer-list kernels: the code
// alone (never run there, their large plans have two dry tiles) cost C4 1.6%.
// Called by the whole warp; p is this lane's query bound, want its query valid.
constexpr long long kBoundPollCycles = 8000;

static __device__ __noinline__ float poll_bound(const uint32_t* p, bool want, float fresh) {
  const long long p0 = clock64();
  while (__any_sync(kFullMask, want && fresh == -INFINITY) && clock64() - p0 < kBoundPollCycles) {
    __nanosleep(256);
    if (want && fresh == -INFINITY) fresh = load_bound(p);
  }
  return fresh;
}

// Bit j set when score j is at least lim = max(list threshold, shared bound)
// (only the first nvalid scores count). Scores equal to the list threshold are
// kept: a list revisits its first tiles last, so an equal score may belong to a
// smaller row id and rank higher. Four independent OR chains.
__device__ __forceinline__ uint32_t above_mask(const uint32_t (&r)[32], float lim, int nvalid) {
  uint32_t m[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float s = __uint_as_float(r[j]);
    m[j & 3] |= (s >= lim ? 1u : 0u) << j;
  }
  const uint32_t all = (m[0] | m[1]) | (m[2] | m[3]);
  return nvalid >= 32 ? all : (all & ((1u << nvalid) - 1u));
}

// r[j] for a run-time j without indexing the register array (which would move
// it to local memory): a 5-level select tree on the bits of j.
__device__ __forceinline__ float pick(const uint32_t (&r)[32], int j) {
  uint32_t l[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) l[i] = (j & 1) ? r[2 * i + 1] : r[2 * i];
#pragma unroll
  for (int w = 8, bit = 2; w >= 1; w >>= 1, bit <<= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) l[i] = (j & bit) ? l[2 * i + 1] : l[2 * i];
  return __uint_as_float(l[0]);
}

constexpr int kTopsPerLane = 10;  // lists per query <= 320 for the in-kernel refresh

// Raises the shared bound of every query in `need` (the lanes of this warp whose
// query this list refreshes in this round) to the m-th largest value its lists
// published (warp_kth_top). The whole warp serves one query at a time, and the
// next query's published values are loaded while the current one is bisected,
// so consecutive refreshes do not each wait a global-memory round trip.
__device__ __forceinline__ void refresh_bounds(unsigned need, const uint32_t* tops, uint32_t* gthr, int q,
                                               int lists, int m, float& bound, int lane) {
  if (!need) return;
  uint32_t cur[kTopsPerLane], nxt[kTopsPerLane];
  int src = __ffs(need) - 1;
  need &= need - 1;
  int qs = __shfl_sync(kFullMask, q, src);
  load_tops<kTopsPerLane>(tops + static_cast<size_t>(qs) * lists, lists, lane, cur);
  while (true) {
    int nsrc = -1, nqs = 0;
    if (need) {
      nsrc = __ffs(need) - 1;
      need &= need - 1;
      nqs = __shfl_sync(kFullMask, q, nsrc);
      load_tops<kTopsPerLane>(tops + static_cast<size_t>(nqs) * lists, lists, lane, nxt);
    }
    const uint32_t kth = kth_of_tops<kTopsPerLane>(cur, m);
    if (lane == src && kth != 0) {
      atomicMax(gthr + qs, kth);
      bound = fmaxf(bound, score_of_bits(kth));
    }
    if (nsrc < 0) break;
    src = nsrc;
    qs = nqs;
#pragma unroll
    for (int j = 0; j < kTopsPerLane; ++j) cur[j] = nxt[j];
  }
}

// Dry tiles. A list starts empty, so without a shared bound its first tile
// would send dozens of scores per query through the slow insertion path while
// the tensor cores wait (two accumulators let the MMA run only one tile ahead).
// Instead the first kDryTiles tiles a CTA works on are read "dry" -- they only
// raise the value each list publishes for the query's bound -- and are computed
// again, for real, after the CTA's last tile, when the bound from every list's
// first tiles is in place. The host sets the count (TcArgs::dry, at most
// kDryTiles from cvs_kernels.h): two when a CTA can expect three or more tiles,
// one for two; the extra MMA work is the dry count / tiles per CTA.

// Largest of the first nvalid scores.
__device__ __forceinline__ float max_valid(const uint32_t (&r)[32], int nvalid) {
  if (nvalid >= 32) return max32(r);
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nvalid) m = fmaxf(m, __uint_as_float(r[j]));
  return m;
}



// Sorted (score desc, row asc) list of KP slots in registers holding the best
// k <= KP candidates in its LAST k slots; the first KP-k slots are parked at
// +inf so no finite score displaces them. The k-th best is then always the
// last slot (a run-time slot index would push the list to local memory).
template <int KP>
struct EpiTopkReg {
  // Two column stripes per TMEM quadrant (8 epilogue warps, 320 threads).
  static constexpr int kSubs = 2;
  static constexpr bool kTops = true;
  static constexpr int kScratchKeys = 0;
  float tv[KP];
  uint32_t ti[KP];
  float thr;         // this list's k-th best (its last slot)
  float bound;       // shared lower bound of the query (refreshed per tile)
  float best;        // this list's best score so far
  uint32_t published;
  uint32_t top_published;
  int k;

  __device__ __forceinline__ void init(const TcArgs& a) {
    k = a.k;
    bound = -INFINITY;
    best = -INFINITY;
    published = 0;
    top_published = 0;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      tv[j] = (j < KP - k) ? INFINITY : -INFINITY;
      ti[j] = 0xFFFFFFFFu;
    }
    thr = -INFINITY;
  }

  // The list is sorted, so "candidate ranks before slot j" is false for the
  // leading slots and true from the insertion point on. All KP tests are
  // independent and the shift is one select per slot: no serial chain.
  __device__ __forceinline__ void insert(float s, uint32_t row) {
    bool gt[KP];
#pragma unroll
    for (int j = 0; j < KP; ++j) gt[j] = (s > tv[j]) || (s == tv[j] && row < ti[j]);
#pragma unroll
    for (int j = KP - 1; j > 0; --j) {
      tv[j] = gt[j] ? (gt[j - 1] ? tv[j - 1] : s) : tv[j];
      ti[j] = gt[j] ? (gt[j - 1] ? ti[j - 1] : row) : ti[j];
    }
    tv[0] = gt[0] ? s : tv[0];
    ti[0] = gt[0] ? row : ti[0];
    thr = tv[KP - 1];
    best = fmaxf(best, s);
  }

  // Every list of a query publishes its best score in its own slot of
  // a.tops[q][list]. If k different lists hold a score >= v, at least k rows
  // score >= v, so the query's k-th best is >= v: the k-th largest published
  // maximum is a bound close to the k-th best of ALL rows seen so far (the
  // per-list k-th bests alone only give a much weaker one).
  __device__ __forceinline__ void publish_top(const TcArgs& a, int q, int list, int lists) {
    if (best == -INFINITY) return;
    const uint32_t o = ordered_bits(best);
    if (o > top_published) {
      asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(a.tops + static_cast<size_t>(q) * lists + list),
                   "r"(o)
                   : "memory");
      top_published = o;
    }
  }

  __device__ __forceinline__ void consume(const uint32_t (&r)[32], int row0, int nvalid,
                                          bool qvalid, uint32_t*) {
    if (!qvalid) return;
    const float mx = max32(r);
    const float lim = fmaxf(thr, bound);
    if (!(mx >= lim)) return;
    uint32_t m = above_mask(r, lim, nvalid);
    while (m) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      const float s = pick(r, j);
      if (s >= thr) insert(s, static_cast<uint32_t>(row0 + j));  // no-op unless it ranks in
    }
  }

  static __device__ __forceinline__ bool dry_ok(const TcArgs&) { return true; }
  // Dry tile: only the published best moves.
  __device__ __forceinline__ void dry(const uint32_t (&r)[32], int nvalid, bool qvalid) {
    if (qvalid) best = fmaxf(best, max_valid(r, nvalid));
  }

  static __device__ __forceinline__ int jrank(int, int) { return 1; }  // publishes its best

  __device__ __forceinline__ void finish(const TcArgs& a, int q, int list, bool qvalid, uint32_t*, uint64_t*,
                                         int) {
    if (!qvalid) return;
    uint64_t* out = a.part + (static_cast<size_t>(q) * a.segs * kSubs + list) * a.cap;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      if (j >= KP - k) out[j - (KP - k)] = (tv[j] == -INFINITY) ? 0ull : make_key(tv[j], ti[j]);
    }
  }
};

// Per-query candidate buffer of `cap` keys in global memory (L2 resident) for
// k > 32. A key is appended when its score beats the list's k-th best (as of
// its last compaction) and the query's shared bound; when a list could
// overflow on the next chunk, the warp loads it into shared memory in one round
// trip, radix-selects its top k and J-th best there, writes the top k back and
// publishes the J-th best for the query's bound.
template <int RJ>
struct EpiTopkBuf {
  // Two column stripes per TMEM quadrant, as the register lists.
  static constexpr int kSubs = 2;
  static constexpr bool kTops = true;
  static constexpr int kScratchKeys = 256;  // shared-memory compaction up to 256 keys (cap 256: k <= 112)
  static constexpr int kRegJ = RJ;  // J-th best tracked in registers for J <= kRegJ
  static __device__ __forceinline__ int jrank(int k, int lists) { return tops_j(k, lists, RJ); }
  uint64_t* list;
  int cnt;
  int jr;           // J: rank of the value this list publishes
  float thr;        // k-th best at the last compaction
  float bound;      // shared lower bound of the query (refreshed per tile)
  float best;       // value this list publishes: a lower bound on its J-th best
  float tj[kRegJ];  // best kRegJ scores appended so far, descending
  bool redo;        // second pass over dry tiles: their scores are already in tj
  uint32_t published;
  uint32_t top_published;

  __device__ __forceinline__ void init(const TcArgs& a) {
    list = nullptr;
    cnt = 0;
    jr = tops_j(a.k, a.segs * kSubs, RJ);
    thr = -INFINITY;
    bound = -INFINITY;
    best = -INFINITY;
#pragma unroll
    for (int i = 0; i < kRegJ; ++i) tj[i] = -INFINITY;
    redo = false;
    published = 0;
    top_published = 0;
  }

  // Keeps tj the kRegJ largest appended scores (compare-exchange chain).
  __device__ __forceinline__ void track(float s) {
#pragma unroll
    for (int i = 0; i < kRegJ; ++i) {
      const float hi = fmaxf(tj[i], s);
      s = fminf(tj[i], s);
      tj[i] = hi;
    }
  }

  // tj[jr - 1] without a run-time register index.
  __device__ __forceinline__ float reg_jth() const {
    float v = tj[0];
#pragma unroll
    for (int i = 1; i < kRegJ; ++i) v = jr > i ? tj[i] : v;
    return v;
  }

  // Keeps the top min(k, m) keys of lane src's list and records its k-th best
  // and J-th best; scratch = this warp's shared buffer (kScratchKeys keys).
  __device__ __forceinline__ void compact_one(int src, const TcArgs& a, int jrank, uint32_t* hist,
                                              uint64_t* scratch, int lane) {
    uint64_t* L = reinterpret_cast<uint64_t*>(shfl_u64(reinterpret_cast<uint64_t>(list), src));
    const int m = __shfl_sync(kFullMask, cnt, src);
    uint64_t kth = 0, jth = 0;
    if (m <= kScratchKeys) {
      constexpr int kPerLane = kScratchKeys / 32;
      uint64_t v[kPerLane];
#pragma unroll
      for (int u = 0; u < kPerLane; ++u) {
        const int i = lane + 32 * u;
        v[u] = i < m ? L[i] : 0ull;
      }
#pragma unroll
      for (int u = 0; u < kPerLane; ++u) scratch[lane + 32 * u] = v[u];
      __syncwarp();
      if (m > a.k) {
        kth = warp_kth_key(ContigKeys{scratch}, m, a.k, hist, lane);
        int base = 0;
        for (int i0 = 0; i0 < m; i0 += 32) {
          const int i = i0 + lane;
          const uint64_t key = i < m ? scratch[i] : 0ull;
          const bool keep = i < m && key >= kth;
          const unsigned bal = __ballot_sync(kFullMask, keep);
          if (keep) L[base + __popc(bal & ((1u << lane) - 1u))] = key;
          base += __popc(bal);
        }
      }
      if (jrank > kRegJ && m >= jrank) jth = warp_kth_key(ContigKeys{scratch}, m, jrank, hist, lane);
      __syncwarp();
    } else {
      kth = warp_kth_key(ContigKeys{L}, m, a.k, hist, lane);
      warp_compact_ge(L, m, kth, lane);
      if (jrank > kRegJ) jth = warp_kth_key(ContigKeys{L}, a.k, jrank, hist, lane);
    }
    if (lane == src) {
      if (m > a.k) {
        cnt = a.k;
        thr = key_score(kth);
      }
      if (jth != 0ull) best = fmaxf(best, key_score(jth));
    }
  }

  __device__ __forceinline__ void compact_lanes(unsigned need, const TcArgs& a, int jrank, uint32_t* hist,
                                                uint64_t* scratch, int lane) {
    while (need) {
      const int src = __ffs(need) - 1;
      need &= need - 1;
      compact_one(src, a, jrank, hist, scratch, lane);
    }
  }

  __device__ __forceinline__ void consume(const uint32_t (&r)[32], int row0, int nvalid,
                                          bool qvalid, uint32_t*) {
    const float mx = max32(r);
    const float lim = fmaxf(thr, bound);
    if (qvalid && mx >= lim) {
      uint32_t m = above_mask(r, lim, nvalid);
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        const float s = pick(r, j);
        list[cnt++] = make_key(s, static_cast<uint32_t>(row0 + j));
        if (!redo) track(s);
      }
    }
  }

  // Dry tiles need the J-th best in registers.
  static __device__ __forceinline__ bool dry_ok(const TcArgs& a) { return tops_j(a.k, a.segs * kSubs, RJ) <= kRegJ; }
  __device__ __forceinline__ void dry(const uint32_t (&r)[32], int nvalid, bool qvalid) {
    if (!qvalid) return;
    // Only scores that beat the kRegJ-th tracked one can change tj; when one
    // does, all 32 go through the compare-exchange chain with static register
    // indices (2 kRegJ min/max each; a score at or below tj's last entry leaves
    // it unchanged). Selecting the candidates one by one cost ~60 instructions
    // each, and a fresh list's first chunk has 32 of them.
    const float lo = tj[kRegJ - 1];
    if (!(max_valid(r, nvalid) > lo)) return;
#pragma unroll
    for (int j = 0; j < 32; ++j) track(j < nvalid ? __uint_as_float(r[j]) : -INFINITY);
  }

  // The list's segment holds at least J rows scoring >= best (the value is the
  // J-th best of the rows seen so far); m = ceil(k / J) lists reaching a value v
  // therefore prove k rows >= v.
  __device__ __forceinline__ void publish_top(const TcArgs& a, int q, int list_idx, int lists) {
    if (jr <= kRegJ) best = fmaxf(best, reg_jth());
    if (best == -INFINITY) return;
    const uint32_t o = ordered_bits(best);
    if (o > top_published) {
      asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(a.tops + static_cast<size_t>(q) * lists + list_idx),
                   "r"(o)
                   : "memory");
      top_published = o;
    }
  }

  // The list stays as it is (at most cap keys, unsorted); the merge reads
  // counts[q][list] keys of it. Lists whose J is beyond the register range
  // compact once more so that their J-th best can be published.
  __device__ __forceinline__ void finish(const TcArgs& a, int q, int list_idx, bool qvalid, uint32_t* hist,
                                         uint64_t* scratch, int lists) {
    const int lane = threadIdx.x & 31;
    if (jr > kRegJ)
      compact_lanes(__ballot_sync(kFullMask, qvalid && cnt >= jr), a, jr, hist, scratch, lane);
    if (qvalid) {
      a.counts[static_cast<size_t>(q) * lists + list_idx] = cnt;
      publish_top(a, q, list_idx, lists);
    }
  }
};

// Writes the score tile to [b][n] (fp32 or fp16).
template <bool F32>
struct EpiStore {
  static constexpr int kSubs = 2;
  static constexpr bool kTops = false;
  static constexpr int kScratchKeys = 0;
  __device__ __forceinline__ void init(const TcArgs&) {}
  __device__ __forceinline__ void consume_store(const uint32_t (&r)[32], int row0, int nvalid,
                                                bool qvalid, const TcArgs& a, int q) {
    if (!qvalid) return;
    const size_t o = static_cast<size_t>(q) * a.n + row0;
    if (F32) {
      float* dst = reinterpret_cast<float*>(a.scores_out) + o;
      if (nvalid == 32 && (o & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid) dst[j] = __uint_as_float(r[j]);
      }
    } else {
      __half* dst = reinterpret_cast<__half*>(a.scores_out) + o;
      if (nvalid == 32 && (o & 7) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint32_t w[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const __half2 h = __floats2half2_rn(__uint_as_float(r[j + 2 * t]),
                                                __uint_as_float(r[j + 2 * t + 1]));
            w[t] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(dst + j) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid) dst[j] = __float2half_rn(__uint_as_float(r[j]));
      }
    }
  }
};

template <class E>
struct is_buf : std::false_type {};
template <int RJ>
struct is_buf<EpiTopkBuf<RJ>> : std::true_type {};

template <class E>
struct is_store : std::false_type {};
template <bool F>
struct is_store<EpiStore<F>> : std::true_type {};


}  // namespace cvs
