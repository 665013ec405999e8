// Dynamic corpus-tile scheduling for the tcgen05 search kernels.
//
// The SMs of a B200 do not stream corpus tiles at the same rate: with a fixed
// split of the corpus into equal segments, some CTAs of the same launch finish
// a third later than others, the same SMs run after run. So the search kernels
// hand out tiles at run time instead: one thread per CTA (per CTA pair) claims
// the next 256-row tile of its query tile from a global counter and records
// "iteration i works on tile t" in a small log in shared memory, from which the
// CTA's other roles (and the odd CTA of a pair, whose log the claiming thread
// writes remotely) take their tile numbers.
//
// The log has kLogSlots entries, reused round-robin. An entry holds its
// iteration number next to the tile, so a reader waits until the slot carries
// the iteration it wants. No reader can fall kLogSlots iterations behind the
// writer: the writer reaches iteration i only after the stage ring and the two
// TMEM accumulators let it, that is after every role of both CTAs has started
// iteration i - 9 or later (six stages, two accumulators).
//
// Dry tiles (cvs_epilogue.cuh; at most kDryTiles, cvs_kernels.h) fit in as follows: the first
// `dry` tiles a CTA claims are logged as dry, and once the counter runs out
// they are logged again, as redo iterations, before the end marker.
#pragma once

#include <cstdint>

#include "cvs_device.cuh"

namespace cvs {

constexpr int kLogSlots = 16;
constexpr uint32_t kLogEnd = 0xFFFFFFFFu;     // no more iterations
constexpr uint32_t kLogDry = 1u << 30;        // iteration reads its tile dry
constexpr uint32_t kLogRedo = 1u << 29;       // iteration revisits a dry tile
constexpr uint32_t kLogTileMask = kLogRedo - 1u;

__device__ __forceinline__ uint64_t log_entry(int iter, uint32_t v) {
  return (static_cast<uint64_t>(static_cast<uint32_t>(iter)) << 32) | v;
}

// Marks every slot as holding iteration -1 (run by one thread before the CTA's
// (cluster's) start-up barrier).
__device__ __forceinline__ void log_init(uint64_t* log) {
  for (int s = 0; s < kLogSlots; ++s) log[s] = log_entry(-1, kLogEnd);
}

__device__ __forceinline__ void log_put(uint64_t* log, int iter, uint32_t v) {
  asm volatile("st.volatile.shared.u64 [%0], %1;" ::"r"(smem_u32(log + (iter % kLogSlots))),
               "l"(log_entry(iter, v))
               : "memory");
}

// Writes the entry into the log of another CTA of the cluster (log_cluster: the
// shared::cluster address of that CTA's log).
__device__ __forceinline__ void log_put_remote(uint32_t log_cluster, int iter, uint32_t v) {
  asm volatile("st.relaxed.cluster.shared::cluster.u64 [%0], %1;" ::"r"(log_cluster +
                                                                        8u * static_cast<uint32_t>(iter % kLogSlots)),
               "l"(log_entry(iter, v))
               : "memory");
}

// Waits (bounded, like mbar_wait) until the slot of iteration `iter` carries
// that iteration, and returns its value in *v.
__device__ __forceinline__ bool log_get(const uint64_t* log, int iter, uint32_t* v, volatile int* abort,
                                        int* err, int site, long long limit = kWaitCycles) {
  const uint32_t addr = smem_u32(log + (iter % kLogSlots));
  long long t0 = 0;
  for (int spin = 0;; ++spin) {
    uint64_t e;
    asm volatile("ld.relaxed.cluster.shared.u64 %0, [%1];" : "=l"(e) : "r"(addr) : "memory");
    if (static_cast<uint32_t>(e >> 32) == static_cast<uint32_t>(iter)) {
      *v = static_cast<uint32_t>(e);
      return true;
    }
    if (spin == 0) t0 = clock64();
    if (*abort) return false;
    if (clock64() - t0 > limit) {
      *abort = 1;
      report_error(err, kErrTimeout | site);
      return false;
    }
    // Back off so a waiting reader does not take issue slots from the producer
    // and MMA warps sharing its scheduler.
    __nanosleep(64);
  }
}

// The claiming side: the sequence of tiles one CTA (pair) works on.
// counter == nullptr: a fixed segment [t_begin, t_end) instead of claims.
struct TileSource {
  int* counter;
  int ntiles;
  int t_next;   // fixed segment: next tile
  int t_end;
  int dry;      // leading tiles read dry and revisited at the end
  int claimed;  // tiles handed out so far (excluding redo)
  int redo;     // dry tiles revisited so far
  int first0;   // the dry tiles, revisited at the end (kDryTiles <= 2);
  int first1;   // scalars rather than an array so they stay in registers

  __device__ __forceinline__ void init(int* c, int n, int begin, int end, int d) {
    counter = c;
    ntiles = n;
    t_next = begin;
    t_end = end;
    dry = d;
    claimed = 0;
    redo = 0;
    first0 = first1 = 0;
  }

  // Value for the next log entry.
  __device__ __forceinline__ uint32_t next() {
    if (redo == 0) {
      int t;
      if (counter != nullptr) {
        t = atomicAdd(counter, 1);
        if (t >= ntiles) t = -1;
      } else {
        t = t_next < t_end ? t_next++ : -1;
      }
      if (t >= 0) {
        uint32_t v = static_cast<uint32_t>(t);
        if (claimed < dry) {
          if (claimed == 0) first0 = t;
          else first1 = t;
          v |= kLogDry;
        }
        ++claimed;
        return v;
      }
    }
    const int nd = claimed < dry ? claimed : dry;
    if (redo < nd) {
      const int t = redo == 0 ? first0 : first1;
      ++redo;
      return static_cast<uint32_t>(t) | kLogRedo;
    }
    redo = nd + 1;  // stays exhausted
    return kLogEnd;
  }
};

}  // namespace cvs
