// CTA-pair (tcgen05 cta_group::2) variant of the fused score + top-k kernel,
// used for batches of more than 128 queries.
//
// A cluster of two CTAs on neighbouring SMs computes 256 queries x 256 corpus
// rows per tile with one M=256, N=256 MMA stream issued by the even CTA:
//   * each CTA holds its own 128-query tile (the MMA's A rows) and HALF of the
//     corpus tile (128 rows, the MMA's B columns); the tensor cores of the pair
//     read the other CTA's half directly, so every corpus row is fetched from
//     L2/HBM exactly once per pair and the per-SM query traffic is half that
//     of the one-CTA kernel;
//   * each CTA's TMEM receives the 128 x 256 fp32 scores of its own queries and
//     its epilogue warps run the same per-query top-k as the one-CTA kernel.
//
// Synchronisation (every wait bounded, see cvs_device.cuh):
//   full[s]   (even CTA) its producer arms it for BOTH CTAs' bytes; the odd
//             CTA's TMA loads land in the odd CTA's shared memory but complete
//             on the even CTA's barrier (cta_group::2 form of the TMA load).
//   empty[s]  the even CTA's MMA thread commits to empty[s] in both CTAs.
//   tfull[a]  likewise: accumulator a is ready in both CTAs.
//   tempty[a] (even CTA) both CTAs' epilogue warps arrive when they drained a.
// Both CTAs meet at a cluster barrier before TMEM is released.
//
// Replaces, for large batches, the reference's fused kernel
// (cuda_vector_search/csrc/kernels.cu:313-371), whose WMMA tiles re-read the
// corpus once per 16/32/64-query block.
#include <type_traits>

#include "cvs_device.cuh"
#include "cvs_epilogue.cuh"
#include "cvs_kernels.h"
#include "cvs_sched.cuh"
#include "cvs_select.cuh"

namespace cvs {

namespace {

constexpr int kRows = kTcN / 2;                  // corpus rows per CTA per tile
constexpr int kQSlice = kTcM * kTcK * 2;         // 16 KB: 128 queries x 64 halves
constexpr int kXHalf = kRows * kTcK * 2;         // 16 KB: 128 corpus rows x 64 halves
constexpr int kStages = kTcMaxStages;  // barrier arrays are sized for this many stages
constexpr uint32_t kTmemCols = 512;

__host__ __device__ constexpr int pair_epi_warps(int subs) { return 4 * subs; }
__host__ __device__ constexpr int pair_threads(int subs) { return 64 + 32 * pair_epi_warps(subs); }

// Shared-memory carve-up, as for the one-CTA kernel: the ring takes what the
// resident queries, barriers, log and (buffer epilogues) histograms and
// compaction buffers leave, at most kStages stages -- at d_pad = 384 with
// resident queries 8 stages of 16 KB (register lists) or 6 (buffer lists),
// with streamed queries 7 of 32 KB (register lists) or 6.
struct PairLayout {
  int stages;       // offset of the stage ring (after resident queries)
  int nstages;      // ring depth
  int stage_bytes;
  int bars;
  int log;
  int hist;
  int scratch;
  int total;
};

__host__ __device__ constexpr PairLayout pair_layout(bool qres, int ksl, int subs, int scratch_keys) {
  PairLayout l{};
  l.stage_bytes = qres ? kXHalf : (kXHalf + kQSlice);
  l.stages = qres ? ksl * kQSlice : 0;
  // full[], empty[], tfull[2], tempty[2], qfull, done; tmem holder, abort; log; histograms; buffers
  const int bar_bytes = 8 * (2 * kStages + 6) + 16;
  const int hist_bytes = scratch_keys > 0 ? pair_epi_warps(subs) * 256 * 4 : 0;
  const int tail = bar_bytes + 8 * kLogSlots + hist_bytes + pair_epi_warps(subs) * scratch_keys * 8;
  const int n = (kSmemBudget - l.stages - tail) / l.stage_bytes;
  l.nstages = n < kStages ? n : kStages;
  l.bars = l.stages + l.nstages * l.stage_bytes;
  l.log = l.bars + bar_bytes;
  l.hist = l.log + 8 * kLogSlots;
  l.scratch = l.hist + hist_bytes;
  l.total = l.scratch + pair_epi_warps(subs) * scratch_keys * 8;
  return l;
}

struct PairShared {
  uint8_t* base;
  PairLayout l;
  __device__ uint8_t* qres(int ks) const { return base + ks * kQSlice; }
  __device__ uint8_t* stage_x(int s) const { return base + l.stages + s * l.stage_bytes; }
  __device__ uint8_t* stage_q(int s) const { return base + l.stages + s * l.stage_bytes + kXHalf; }
  __device__ uint64_t* bar(int i) const { return reinterpret_cast<uint64_t*>(base + l.bars) + i; }
  __device__ uint64_t* full(int s) const { return bar(s); }
  __device__ uint64_t* empty(int s) const { return bar(kStages + s); }
  __device__ uint64_t* tfull(int a) const { return bar(2 * kStages + a); }
  __device__ uint64_t* tempty(int a) const { return bar(2 * kStages + 2 + a); }
  __device__ uint64_t* qfull() const { return bar(2 * kStages + 4); }
  __device__ uint64_t* done() const { return bar(2 * kStages + 5); }
  __device__ uint32_t* tmem_holder() const {
    return reinterpret_cast<uint32_t*>(base + l.bars + 8 * (2 * kStages + 6));
  }
  __device__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(base + l.bars + 8 * (2 * kStages + 6) + 4);
  }
  __device__ uint64_t* log() const { return reinterpret_cast<uint64_t*>(base + l.log); }
  __device__ uint32_t* hist(int w) const { return reinterpret_cast<uint32_t*>(base + l.hist) + 256 * w; }
  __device__ uint64_t* scratch(int w, int keys) const {
    return reinterpret_cast<uint64_t*>(base + l.scratch) + static_cast<size_t>(keys) * w;
  }
};

template <bool QRES, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads(Epi::kSubs), 1)
    tc_pair_kernel(const __grid_constant__ CUtensorMap qmap,
                   const __grid_constant__ CUtensorMap xmap, const TcArgs a) {
  constexpr int kEpiWarps = pair_epi_warps(Epi::kSubs);
  extern __shared__ uint8_t smem_raw[];
  PairShared sh;
  sh.base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
  sh.l = pair_layout(QRES, a.ksl, Epi::kSubs, Epi::kScratchKeys);
  const int kS = sh.l.nstages;  // ring depth

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs; 1: its partner
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int qp = pair % a.qtiles;           // query-pair tile (256 queries)
  const int seg = pair / a.qtiles;
  const int qrow0 = qp * (2 * kTcM) + static_cast<int>(rank) * kTcM;  // this CTA's queries
  const int t_begin = seg * a.tiles_per_seg;
  const int t_end = min(a.ntiles, t_begin + a.tiles_per_seg);
  int nd = 0;  // dry tiles (see kDryTiles): the first nd claimed tiles, revisited at the end
  if constexpr (Epi::kTops) nd = Epi::dry_ok(a) ? a.dry : 0;
  volatile int* abort = sh.abort_flag();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(sh.full(s), 1);
      mbar_init(sh.empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(sh.tfull(t), 1);
      mbar_init(sh.tempty(t), leader ? 2 * kEpiWarps : 1);
    }
    mbar_init(sh.qfull(), 1);
    mbar_init(sh.done(), 1);
    log_init(sh.log());
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&xmap);
  }
  if (warp == 1) {
    tmem_alloc_pair(sh.tmem_holder(), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the partner's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *sh.tmem_holder();
  // Launched programmatically after the workspace clear (or the caller's previous
  // kernel): the set-up above overlapped it; everything below reads its results.
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) ----------------
    if (elect_one_lane()) {
      const uint64_t pol_x = l2_policy_evict_first();
      // Dry tiles are read again at the end: keep them in L2 until then.
      const uint64_t pol_keep = l2_policy_evict_last();
      const uint64_t pol_q = l2_policy_evict_last();
      // Completion of both CTAs' copies is counted on the even CTA's barriers.
      auto even_bar = [&](uint64_t* bar) { return map_to_rank(smem_u32(bar), 0); };
      auto load = [&](void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, uint64_t pol) {
        if (leader) tma_load_2d(dst, map, bar, x, y, pol);
        else tma_load_2d_to_pair_bar(dst, map, even_bar(bar), x, y, pol);
      };
      if (QRES) {
        if (leader) mbar_arrive_expect_tx(sh.qfull(), static_cast<uint32_t>(2 * a.ksl * kQSlice));
        for (int ks = 0; ks < a.ksl; ++ks) load(sh.qres(ks), &qmap, sh.qfull(), ks * kTcK, qrow0, pol_q);
      }
      const uint32_t tx = QRES ? kXHalf : (kXHalf + kQSlice);
      // The even CTA claims the pair's tiles and logs them in both CTAs.
      TileSource src;
      src.init(a.tile_counter ? a.tile_counter + qp : nullptr, a.ntiles, t_begin, t_end, nd);
      const uint32_t peer_log = map_to_rank(smem_u32(sh.log()), 1);
      int it = 0;
      bool ok = true;
      for (int t = 0; ok; ++t) {
        uint32_t v;
        if (leader) {
          v = src.next();
          log_put(sh.log(), t, v);
          log_put_remote(peer_log, t, v);
        } else if (!log_get(sh.log(), t, &v, abort, a.err, 15)) {
          ok = false;
          break;
        }
        if (v == kLogEnd) break;
        const uint64_t pol_t = (v & kLogDry) ? pol_keep : pol_x;
        const int row0 = static_cast<int>(v & kLogTileMask) * kTcN + static_cast<int>(rank) * kRows;
        for (int ks = 0; ks < a.ksl; ++ks, ++it) {
          const int s = it % kS;
          const uint32_t ph = (it / kS) & 1;
          if (!mbar_wait(sh.empty(s), ph ^ 1, abort, a.err, 11)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(sh.full(s), 2 * tx);
          load(sh.stage_x(s), &xmap, sh.full(s), ks * kTcK, row0, pol_t);
          if (!QRES) load(sh.stage_q(s), &qmap, sh.full(s), ks * kTcK, qrow0, pol_q);
        }
      }
      if (!ok && leader) {
        // Leaving early: the even CTA's barriers count both CTAs' copies, so
        // waiting (bounded) on the phases it armed lets the pair's copies land;
        // the odd CTA stays resident until the final cluster barrier.
        for (int j = max(0, it - kS); j < it; ++j)
          mbar_wait_drain(sh.full(j % kS), (j / kS) & 1);
        if (QRES) mbar_wait_drain(sh.qfull(), 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (elect_one_lane()) {
      if (leader) {
        // ---------------------------- MMA issuer (even CTA) -----------------
        const uint32_t idesc = idesc_f16_f32(2 * kTcM, kTcN);
        bool ok = true;
        if (QRES) ok = mbar_wait(sh.qfull(), 0, abort, a.err, 12);
        int it = 0;
        for (int t = 0; ok; ++t) {
          uint32_t v;
          if (!log_get(sh.log(), t, &v, abort, a.err, 16)) {
            ok = false;
            break;
          }
          if (v == kLogEnd) break;
          const int acc = t & 1;
          const uint32_t use = static_cast<uint32_t>(t >> 1);
          if (!mbar_wait(sh.tempty(acc), (use & 1) ^ 1, abort, a.err, 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcN);
          for (int ks = 0; ks < a.ksl; ++ks, ++it) {
            const int s = it % kS;
            const uint32_t ph = (it / kS) & 1;
            if (!mbar_wait(sh.full(s), ph, abort, a.err, 14)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t qa = smem_u32(QRES ? sh.qres(ks) : sh.stage_q(s));
            const uint32_t xa = smem_u32(sh.stage_x(s));
#pragma unroll
            for (int kk = 0; kk < kTcK / 16; ++kk) {
              tc_mma_f16_pair(d_tmem, smem_desc_sw128(qa + kk * 32), smem_desc_sw128(xa + kk * 32),
                              idesc, (ks | kk) != 0 ? 1u : 0u);
            }
            tc_commit_pair(sh.empty(s), 0x3);
          }
          if (!ok) break;
          tc_commit_pair(sh.tfull(acc), 0x3);
        }
        tc_commit_pair(sh.done(), 0x3);  // both CTAs learn when every MMA has retired
        mbar_wait_drain(sh.done(), 0);
      } else {
        // Odd CTA: no MMA to issue; wait (bounded) until every pair MMA, which
        // reads this CTA's shared memory and writes its TMEM, has retired.
        mbar_wait_drain(sh.done(), 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue (both CTAs) --------------------
    constexpr int kChunks = kTcN / 32 / Epi::kSubs;
    const int ew = warp - 2;
    const int sub = ew >> 2;
    const int quad = warp & 3;
    const int q = qrow0 + quad * 32 + lane;
    const bool qvalid = q < a.b;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    Epi epi;
    epi.init(a);
    if constexpr (is_buf<Epi>::value) {
      if (qvalid)
        epi.list = a.part + (static_cast<size_t>(q) * a.segs * Epi::kSubs + seg * Epi::kSubs + sub) * a.cap;
    }
    bool ok = true;
    for (int t = 0;; ++t) {
      uint32_t v = 0;
      int got = 1;
      if (lane == 0) got = log_get(sh.log(), t, &v, abort, a.err, 18) ? 1 : 0;
      got = __shfl_sync(kFullMask, got, 0);
      v = __shfl_sync(kFullMask, v, 0);
      if (!got) {
        ok = false;
        break;
      }
      if (v == kLogEnd) break;
      const bool dry = (v & kLogDry) != 0;
      const int acc = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      float fresh = -INFINITY;
      if constexpr (!is_store<Epi>::value) {
        // Overlaps the wait below, except on the first real tile after dry
        // tiles: that tile reads the bound after its wait, by which time the
        // other lists' refresh after the last dry tile has landed.
        if (qvalid && (t != nd || nd == 0)) fresh = load_bound(a.gthr + q);
      }
      if (!mbar_wait(sh.tfull(acc), use & 1, abort, a.err, 17)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if constexpr (!is_store<Epi>::value) {
        if (qvalid && t == nd && nd > 0) fresh = load_bound(a.gthr + q);
        if constexpr (Epi::kTops && !is_buf<Epi>::value) {
          // Single-dry-tile plans (small corpora): see poll_bound.
          const int lists = a.segs * Epi::kSubs;
          if (t == nd && nd == 1 && lists <= 32 * kTopsPerLane && lists >= a.k)
            fresh = poll_bound(a.gthr + q, qvalid, fresh);
        }
        epi.bound = fmaxf(epi.bound, fresh);
      }
      const int row0 = static_cast<int>(v & kLogTileMask) * kTcN;
      const int valid = min(kTcN, a.n - row0);
      if constexpr (is_buf<Epi>::value) epi.redo = (v & kLogRedo) != 0;
      for (int c = sub * kChunks; c < (sub + 1) * kChunks; ++c) {
        if (c * 32 >= valid) break;
        // A query still without a shared bound (one tile per CTA, or a first
        // real tile drained before the dry tiles' bound landed) drains every
        // column of its chunks through the insertion path: it looks for a
        // bound before each chunk and shares its own k-th best after each.
        bool unbounded = false;
        float fb = -INFINITY;
        if constexpr (!is_store<Epi>::value) {
          unbounded = !dry && qvalid && epi.bound == -INFINITY;
          if (unbounded) fb = load_bound(a.gthr + q);
        }
        uint32_t r[32];
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(acc * kTcN + c * 32), r);
        tmem_wait_ld();
        const int nv = min(32, valid - c * 32);
        if constexpr (is_store<Epi>::value) {
          epi.consume_store(r, row0 + c * 32, nv, qvalid, a, q);
        } else if (dry) {
          epi.dry(r, nv, qvalid);
        } else {
          epi.bound = fmaxf(epi.bound, fb);
          epi.consume(r, row0 + c * 32, nv, qvalid, sh.hist(ew));
          if constexpr (is_buf<Epi>::value) {
            epi.compact_lanes(__ballot_sync(kFullMask, qvalid && epi.cnt > a.cap - 32), a,
                              Epi::jrank(a.k, a.segs * Epi::kSubs), sh.hist(ew),
                              sh.scratch(ew, Epi::kScratchKeys), lane);
          }
          if (unbounded) publish_bound(a.gthr + q, epi.thr, epi.published);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(sh.tempty(acc));
        else mbar_arrive_cluster(map_to_rank(smem_u32(sh.tempty(acc)), 0));
      }
      if constexpr (!is_store<Epi>::value) {
        if (qvalid) publish_bound(a.gthr + q, epi.thr, epi.published);
      }
      if constexpr (Epi::kTops) {
        const int lists = a.segs * Epi::kSubs;
        const int list = seg * Epi::kSubs + sub;
        if (qvalid) epi.publish_top(a, q, list, lists);
        if (tops_round(t) && lists <= 32 * kTopsPerLane) {
          // This round's refresher of each query raises the query's shared bound
          // to the k-th largest published maximum; the whole warp serves each.
          const unsigned need =
              __ballot_sync(kFullMask, qvalid && tops_refresher(q, t, list, lists, dry ? kDryRefreshers : 1));
          const int mneed = (a.k + Epi::jrank(a.k, lists) - 1) / Epi::jrank(a.k, lists);
          refresh_bounds(need, a.tops, a.gthr, q, lists, mneed, epi.bound, lane);
        }
      }
    }
    if constexpr (!is_store<Epi>::value) {
      if (ok) epi.finish(a, q, seg * Epi::kSubs + sub, qvalid, sh.hist(ew), sh.scratch(ew, Epi::kScratchKeys),
                          a.segs * Epi::kSubs);
    }
  }

  // This CTA's results are written (or it is leaving on an error): the merge,
  // launched programmatically, may be scheduled as CTAs finish; it still waits
  // for the whole grid before reading.
  grid_launch_dependents();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA releases TMEM or leaves while the other still works
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <bool QRES, class Epi>
const void* pair_kernel_ptr() {
  return reinterpret_cast<const void*>(tc_pair_kernel<QRES, Epi>);
}

template <bool QRES, class Epi>
cudaError_t pair_launch_one(const CUtensorMap* qmap, const CUtensorMap* xmap, const TcArgs& a,
                            cudaStream_t stream) {
  const PairLayout l = pair_layout(QRES, a.ksl, Epi::kSubs, Epi::kScratchKeys);
  const size_t smem = static_cast<size_t>(l.total) + 1024;
  auto kern = tc_pair_kernel<QRES, Epi>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = 2u * static_cast<unsigned>(a.qtiles) * static_cast<unsigned>(a.segs);
  return launch_programmatic(kern, dim3(grid), dim3(pair_threads(Epi::kSubs)), smem, stream, *qmap, *xmap, a);
}

template <bool QRES, class Epi>
int pair_clusters_one(int ksl) {
  const PairLayout l = pair_layout(QRES, ksl, Epi::kSubs, Epi::kScratchKeys);
  const size_t smem = static_cast<size_t>(l.total) + 1024;
  auto kern = tc_pair_kernel<QRES, Epi>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(pair_threads(Epi::kSubs), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) return 0;
  return n;
}

template <bool QRES>
cudaError_t pair_launch_epi(int epi, const CUtensorMap* qmap, const CUtensorMap* xmap, const TcArgs& a,
                            cudaStream_t stream) {
  switch (epi) {
    case kEpiTopkReg16: return pair_launch_one<QRES, EpiTopkReg<16>>(qmap, xmap, a, stream);
    case kEpiTopkReg32: return pair_launch_one<QRES, EpiTopkReg<32>>(qmap, xmap, a, stream);
    case kEpiTopkBuf: return pair_launch_one<QRES, EpiTopkBuf<4>>(qmap, xmap, a, stream);
    case kEpiTopkBuf8: return pair_launch_one<QRES, EpiTopkBuf<8>>(qmap, xmap, a, stream);
    case kEpiStoreF32: return pair_launch_one<QRES, EpiStore<true>>(qmap, xmap, a, stream);
    case kEpiStoreF16: return pair_launch_one<QRES, EpiStore<false>>(qmap, xmap, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <bool QRES>
int pair_clusters_epi(int epi, int ksl) {
  switch (epi) {
    case kEpiTopkReg16: return pair_clusters_one<QRES, EpiTopkReg<16>>(ksl);
    case kEpiTopkReg32: return pair_clusters_one<QRES, EpiTopkReg<32>>(ksl);
    case kEpiTopkBuf: return pair_clusters_one<QRES, EpiTopkBuf<4>>(ksl);
    case kEpiTopkBuf8: return pair_clusters_one<QRES, EpiTopkBuf<8>>(ksl);
    case kEpiStoreF32: return pair_clusters_one<QRES, EpiStore<true>>(ksl);
    case kEpiStoreF16: return pair_clusters_one<QRES, EpiStore<false>>(ksl);
    default: return 0;
  }
}

}  // namespace

bool tc_pair_resident_queries(int epi, int ksl) {
  const int subs = is_buf_epi(epi) ? EpiTopkBuf<4>::kSubs : 2;
  const int scratch = is_buf_epi(epi) ? EpiTopkBuf<4>::kScratchKeys : 0;
  return pair_layout(true, ksl, subs, scratch).nstages >= 6;
}

int tc_pair_max_clusters(int epi, bool resident_queries, int ksl) {
  return resident_queries ? pair_clusters_epi<true>(epi, ksl) : pair_clusters_epi<false>(epi, ksl);
}

cudaError_t tc_pair_launch(int epi, bool resident_queries, const CUtensorMap* qmap,
                           const CUtensorMap* xmap, const TcArgs& a, cudaStream_t stream) {
  if (resident_queries && !tc_pair_resident_queries(epi, a.ksl)) return cudaErrorInvalidValue;
  return resident_queries ? pair_launch_epi<true>(epi, qmap, xmap, a, stream)
                          : pair_launch_epi<false>(epi, qmap, xmap, a, stream);
}

}  // namespace cvs
