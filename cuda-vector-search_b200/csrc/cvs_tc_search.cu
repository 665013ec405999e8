// tcgen05 score kernel with fused per-query top-k (or score-store) epilogue.
//
// Replaces the reference's WMMA tile + fused top-k kernel
// (cuda_vector_search/csrc/kernels.cu:123-177 score_tile, :313-371
// fused_topk_kernel) and its full-matrix score kernel (:285-311).
//
// Operand orientation: A = a 128-query tile (MMA M, TMEM lanes), B = a 256-row
// corpus tile (MMA N, TMEM columns), both K-major fp16 with the 128-byte
// swizzle, fp32 accumulation in TMEM. Thread i of epilogue warp w therefore
// reads, with one tcgen05.ld, 32 consecutive corpus scores of ONE query and can
// run that query's top-k on its own, with no cross-lane traffic.
//
// Grid: one CTA per (query tile, corpus segment); the CTAs of one segment are
// adjacent in launch order so they stream the same corpus tiles at the same
// time and the second read of a tile hits L2. Each CTA: warp 0 issues TMA,
// warp 1 issues tcgen05.mma (one elected thread each), warps 2-5 drain two
// double-buffered 128x256 fp32 accumulators (all 512 TMEM columns).
// Corpus slices stream through a ring of stages; the query tile either stays
// resident in shared memory for the whole kernel (d_pad <= 448, 3 stages) or
// streams beside each corpus slice (it is L2 resident; 4 stages).
#include <type_traits>

#include "cvs_device.cuh"
#include "cvs_epilogue.cuh"
#include "cvs_kernels.h"
#include "cvs_sched.cuh"
#include "cvs_select.cuh"

namespace cvs {

namespace {

constexpr int kQSliceBytes = kTcM * kTcK * 2;  // 16 KB
constexpr int kXSliceBytes = kTcN * kTcK * 2;  // 32 KB
constexpr uint32_t kTmemCols = 512;
// Epilogue warps: kSubs per TMEM lane quadrant (each epilogue type chooses
// kSubs). Warp 2+e drains quadrant (2+e)%4, column stripe e/4 of every tile.
__host__ __device__ constexpr int epi_warps(int subs) { return 4 * subs; }
__host__ __device__ constexpr int tc_threads(int subs) { return 64 + 32 * epi_warps(subs); }

// Shared-memory carve-up (offsets from a 1024-byte aligned base): resident
// query slices (if any), the ring of stages, barriers, iteration log, and for
// buffer epilogues the per-warp radix histograms and compaction buffers. The
// ring takes what is left (at most kTcMaxStages stages): resident queries at
// d_pad = 384 leave 4 stages of 32 KB, streamed queries 4 of 48 KB.
struct Layout {
  int q_res;      // resident query slices
  int stages;     // ring of stages
  int nstages;    // ring depth
  int stage_bytes;
  int bars;       // mbarriers
  int log;        // iteration log (cvs_sched.cuh)
  int hist;       // per epilogue warp radix histograms (buffer epilogue)
  int scratch;    // per epilogue warp compaction buffers (buffer epilogue)
  int total;
};

__host__ __device__ constexpr Layout make_layout(bool qres, int ksl, int subs, int scratch_keys) {
  Layout l{};
  l.q_res = 0;
  l.stage_bytes = qres ? kXSliceBytes : (kXSliceBytes + kQSliceBytes);
  l.stages = qres ? ksl * kQSliceBytes : 0;
  // full[], empty[], tfull[2], tempty[2], qfull, done, tmem holder, abort; log; histograms; buffers
  const int bar_bytes = 8 * (2 * kTcMaxStages + 6) + 16;
  const int hist_bytes = scratch_keys > 0 ? epi_warps(subs) * 256 * 4 : 0;
  const int tail = bar_bytes + 8 * kLogSlots + hist_bytes + epi_warps(subs) * scratch_keys * 8;
  const int n = (kSmemBudget - l.stages - tail) / l.stage_bytes;
  l.nstages = n < kTcMaxStages ? n : kTcMaxStages;
  l.bars = l.stages + l.nstages * l.stage_bytes;
  l.log = l.bars + bar_bytes;
  l.hist = l.log + 8 * kLogSlots;
  l.scratch = l.hist + hist_bytes;
  l.total = l.scratch + epi_warps(subs) * scratch_keys * 8;
  return l;
}

struct Shared {
  uint8_t* base;
  Layout l;
  __device__ uint8_t* qres(int ks) const { return base + l.q_res + ks * kQSliceBytes; }
  __device__ uint8_t* stage_x(int s) const { return base + l.stages + s * l.stage_bytes; }
  __device__ uint8_t* stage_q(int s) const {
    return base + l.stages + s * l.stage_bytes + kXSliceBytes;
  }
  __device__ uint64_t* bar(int i) const { return reinterpret_cast<uint64_t*>(base + l.bars) + i; }
  __device__ uint64_t* full(int s) const { return bar(s); }
  __device__ uint64_t* empty(int s) const { return bar(kTcMaxStages + s); }
  __device__ uint64_t* tfull(int a) const { return bar(2 * kTcMaxStages + a); }
  __device__ uint64_t* tempty(int a) const { return bar(2 * kTcMaxStages + 2 + a); }
  __device__ uint64_t* qfull() const { return bar(2 * kTcMaxStages + 4); }
  __device__ uint64_t* done() const { return bar(2 * kTcMaxStages + 5); }
  __device__ uint32_t* tmem_holder() const {
    return reinterpret_cast<uint32_t*>(base + l.bars + 8 * (2 * kTcMaxStages + 6));
  }
  __device__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(base + l.bars + 8 * (2 * kTcMaxStages + 6) + 4);
  }
  __device__ uint64_t* log() const { return reinterpret_cast<uint64_t*>(base + l.log); }
  __device__ uint32_t* hist(int w) const {
    return reinterpret_cast<uint32_t*>(base + l.hist) + 256 * w;
  }
  __device__ uint64_t* scratch(int w, int keys) const {
    return reinterpret_cast<uint64_t*>(base + l.scratch) + static_cast<size_t>(keys) * w;
  }
};

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <bool QRES, class Epi>
__global__ void __launch_bounds__(tc_threads(Epi::kSubs), 1)
    tc_search_kernel(const __grid_constant__ CUtensorMap qmap,
                     const __grid_constant__ CUtensorMap xmap, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Shared sh;
  sh.base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
  sh.l = make_layout(QRES, a.ksl, Epi::kSubs, Epi::kScratchKeys);
  const int kS = sh.l.nstages;  // ring depth

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x % a.qtiles;
  const int seg = blockIdx.x / a.qtiles;
  const int t_begin = seg * a.tiles_per_seg;
  const int t_end = min(a.ntiles, t_begin + a.tiles_per_seg);
  int nd = 0;  // dry tiles (see kDryTiles): the first nd claimed tiles, revisited at the end
  if constexpr (Epi::kTops) nd = Epi::dry_ok(a) ? a.dry : 0;
  volatile int* abort = sh.abort_flag();
  const long long wlim = a.wait_cycles > 0 ? a.wait_cycles : kWaitCycles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(sh.full(s), 1);
      mbar_init(sh.empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(sh.tfull(t), 1);
      mbar_init(sh.tempty(t), epi_warps(Epi::kSubs));
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
    tmem_alloc(sh.tmem_holder(), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *sh.tmem_holder();
  // Launched programmatically after the workspace clear (or the caller's previous
  // kernel): the set-up above overlapped it; everything below reads its results.
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    // (a.stall: a test of the failure path -- nothing is claimed, logged or
    // loaded, so the other roles' waits run out.)
    if (elect_one_lane() && !a.stall) {
      const uint64_t pol_x = l2_policy_evict_first();
      // Dry tiles are read again at the end: keep them in L2 until then.
      const uint64_t pol_keep = l2_policy_evict_last();
      const uint64_t pol_q = l2_policy_evict_last();
      const int qrow0 = qt * kTcM;
      if (QRES) {
        mbar_arrive_expect_tx(sh.qfull(), static_cast<uint32_t>(a.ksl * kQSliceBytes));
        for (int ks = 0; ks < a.ksl; ++ks)
          tma_load_2d(sh.qres(ks), &qmap, sh.qfull(), ks * kTcK, qrow0, pol_q);
      }
      const uint32_t tx = QRES ? kXSliceBytes : (kXSliceBytes + kQSliceBytes);
      TileSource src;
      src.init(a.tile_counter ? a.tile_counter + qt : nullptr, a.ntiles, t_begin, t_end, nd);
      int it = 0;
      bool ok = true;
      for (int t = 0; ok; ++t) {
        const uint32_t v = src.next();
        log_put(sh.log(), t, v);
        if (v == kLogEnd) break;
        const uint64_t pol_t = (v & kLogDry) ? pol_keep : pol_x;
        const int row0 = static_cast<int>(v & kLogTileMask) * kTcN;
        for (int ks = 0; ks < a.ksl; ++ks, ++it) {
          const int s = it % kS;
          const uint32_t ph = (it / kS) & 1;
          if (!mbar_wait(sh.empty(s), ph ^ 1, abort, a.err, 1, wlim)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(sh.full(s), tx);
          tma_load_2d(sh.stage_x(s), &xmap, sh.full(s), ks * kTcK, row0, pol_t);
          if (!QRES) tma_load_2d(sh.stage_q(s), &qmap, sh.full(s), ks * kTcK, qrow0, pol_q);
        }
      }
      if (!ok) {
        // Leaving early: let every copy already issued land before the CTA exits.
        for (int j = max(0, it - kS); j < it; ++j)
          mbar_wait_drain(sh.full(j % kS), (j / kS) & 1);
        if (QRES) mbar_wait_drain(sh.qfull(), 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (elect_one_lane()) {
      const uint32_t idesc = idesc_f16_f32(kTcM, kTcN);
      bool ok = true;
      if (QRES) ok = mbar_wait(sh.qfull(), 0, abort, a.err, 2, wlim);
      int it = 0;
      for (int t = 0; ok; ++t) {
        uint32_t v;
        if (!log_get(sh.log(), t, &v, abort, a.err, 6, wlim)) {
          ok = false;
          break;
        }
        if (v == kLogEnd) break;
        const int acc = t & 1;
        const uint32_t use = static_cast<uint32_t>(t >> 1);
        if (!mbar_wait(sh.tempty(acc), (use & 1) ^ 1, abort, a.err, 3, wlim)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTcN);
        for (int ks = 0; ks < a.ksl; ++ks, ++it) {
          const int s = it % kS;
          const uint32_t ph = (it / kS) & 1;
          if (!mbar_wait(sh.full(s), ph, abort, a.err, 4, wlim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qa = smem_u32(QRES ? sh.qres(ks) : sh.stage_q(s));
          const uint32_t xa = smem_u32(sh.stage_x(s));
#pragma unroll
          for (int kk = 0; kk < kTcK / 16; ++kk) {
            tc_mma_f16(d_tmem, smem_desc_sw128(qa + kk * 32), smem_desc_sw128(xa + kk * 32), idesc,
                       (ks | kk) != 0 ? 1u : 0u);
          }
          tc_commit(sh.empty(s));
        }
        if (!ok) break;
        tc_commit(sh.tfull(acc));
      }
      // Every MMA must retire before the accumulators are released.
      tc_commit(sh.done());
      mbar_wait_drain(sh.done(), 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ----------------------------------
    constexpr int kChunks = kTcN / 32 / Epi::kSubs;  // 32-column chunks per warp per tile
    const int ew = warp - 2;             // 0 .. 4*kSubs-1
    const int sub = ew >> 2;             // column stripe
    const int quad = warp & 3;           // TMEM lane quadrant this warp may access
    const int q = qt * kTcM + quad * 32 + lane;
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
      if (lane == 0) got = log_get(sh.log(), t, &v, abort, a.err, 7, wlim) ? 1 : 0;
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
      if (!mbar_wait(sh.tfull(acc), use & 1, abort, a.err, 5, wlim)) {
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
      if (lane == 0) mbar_arrive(sh.tempty(acc));
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <bool QRES, class Epi>
cudaError_t launch_one(const CUtensorMap* qmap, const CUtensorMap* xmap, const TcArgs& a,
                       cudaStream_t stream) {
  const Layout l = make_layout(QRES, a.ksl, Epi::kSubs, Epi::kScratchKeys);
  const size_t smem = static_cast<size_t>(l.total) + 1024;
  auto kern = tc_search_kernel<QRES, Epi>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(a.qtiles) * static_cast<unsigned>(a.segs);
  return launch_programmatic(kern, dim3(grid), dim3(tc_threads(Epi::kSubs)), smem, stream, *qmap, *xmap, a);
}

template <bool QRES>
cudaError_t launch_epi(int epi, const CUtensorMap* qmap, const CUtensorMap* xmap, const TcArgs& a,
                       cudaStream_t stream) {
  switch (epi) {
    case kEpiTopkReg16: return launch_one<QRES, EpiTopkReg<16>>(qmap, xmap, a, stream);
    case kEpiTopkReg32: return launch_one<QRES, EpiTopkReg<32>>(qmap, xmap, a, stream);
    case kEpiTopkBuf: return launch_one<QRES, EpiTopkBuf<4>>(qmap, xmap, a, stream);
    case kEpiTopkBuf8: return launch_one<QRES, EpiTopkBuf<8>>(qmap, xmap, a, stream);
    case kEpiStoreF32: return launch_one<QRES, EpiStore<true>>(qmap, xmap, a, stream);
    case kEpiStoreF16: return launch_one<QRES, EpiStore<false>>(qmap, xmap, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool tc_resident_queries(int epi, int ksl) {
  if (ksl > kTcMaxResidentSlices) return false;
  const int subs = is_buf_epi(epi) ? EpiTopkBuf<4>::kSubs : 2;
  const int scratch = is_buf_epi(epi) ? EpiTopkBuf<4>::kScratchKeys : 0;
  return make_layout(true, ksl, subs, scratch).nstages >= 3;
}

int tc_lists_per_segment(int epi) {
  switch (epi) {
    case kEpiTopkReg16: return EpiTopkReg<16>::kSubs;
    case kEpiTopkReg32: return EpiTopkReg<32>::kSubs;
    case kEpiTopkBuf:
    case kEpiTopkBuf8: return EpiTopkBuf<4>::kSubs;
    default: return 1;
  }
}

cudaError_t tc_launch(int epi, bool resident_queries, const CUtensorMap* qmap,
                      const CUtensorMap* xmap, const TcArgs& a, cudaStream_t stream) {
  if (resident_queries && !tc_resident_queries(epi, a.ksl)) return cudaErrorInvalidValue;
  return resident_queries ? launch_epi<true>(epi, qmap, xmap, a, stream)
                          : launch_epi<false>(epi, qmap, xmap, a, stream);
}

}  // namespace cvs
