// Final merge: per query, the top-k of all per-segment candidate lists, emitted
// best first (score descending, then smaller row id).
//
// Replaces the reference's merge kernel (cuda_vector_search/csrc/kernels.cu:
// 373-445: warp replace-the-minimum list plus k serial argmax rounds) and the
// chunk merge of the fp32 ground truth (cuda_vector_search/reference.py:22-33).
// Here one warp per query runs the radix select on the ordered 64-bit keys,
// gathers the k winners into shared memory and writes each one straight to its
// output rank (rank = number of winners with a larger key), so there is no
// serial sort phase.
//
// merge_lists_kernel is the same merge over [lists][b][len] (score, int64 id)
// arrays, used after the multi-GPU gather of per-shard results.
#include <algorithm>

#include "cvs_device.cuh"
#include "cvs_kernels.h"
#include "cvs_select.cuh"

namespace cvs {

namespace {

constexpr int kMergeWarps = 2;       // queries per CTA of the list merge
constexpr int kMergeMaxK = 1024;
constexpr int kKeysThreads = 256;     // one CTA (8 warps) per query in the key merge
constexpr int kKeysWarps = kKeysThreads / 32;
constexpr int kKeysBatch = 8;         // keys in flight per lane
constexpr int kMergeTopsPerLane = 32;  // up to 1024 lists per query

// Keys of one query staged in shared memory by the list merge (one 64-bit key
// per (score, id) pair), so that the radix passes re-read shared memory instead
// of global memory: up to 2048 keys, e.g. 8 ranks x k = 256.
constexpr int kMergeStageKeys = 2048;

// Shared memory per warp of the list merge: radix histogram, k selected keys,
// staged keys.
__host__ __device__ constexpr size_t merge_warp_bytes(int k) {
  return 256 * 4 + static_cast<size_t>(k) * 8 + static_cast<size_t>(kMergeStageKeys) * 8;
}

// Survivors of the bound filter kept in shared memory (4k, at least 512).
__host__ __device__ constexpr int survivor_cap(int k) { return 4 * k > 512 ? 4 * k : 512; }
constexpr int kScanLists = 1024;      // counted lists merged through the offset scan
// Key-merge CTA: histogram, k selected keys, survivors, two counters and the
// bound, per-warp scan totals, list offsets.
__host__ __device__ constexpr size_t keys_smem(int k) {
  return 256 * 4 + static_cast<size_t>(k) * 8 + static_cast<size_t>(survivor_cap(k)) * 8 + 16 +
         kKeysWarps * 4 + kScanLists * 4;
}

// Keys of one query: `lists` lists of `stride` slots, of which the first
// min(count, stride) hold keys (count = counts[list], or per_list for all).
struct PartKeys {
  const uint64_t* p;  // this query's [lists][stride] block
  const int* counts;  // this query's [lists] counts or null
  int stride;
  int per_list;
  __device__ __forceinline__ uint64_t operator()(int i) const {
    const int l = i / stride;
    const int j = i - l * stride;
    const int used = counts ? min(counts[l], stride) : per_list;
    return j < used ? p[i] : 0ull;
  }
};

struct ListKeys {
  const float* v;
  const long long* ids;
  long long v_stride;
  long long i_stride;
  int len;
  int q;
  __device__ __forceinline__ uint64_t operator()(int i) const {
    const long long l = i / len;
    const long long o = static_cast<long long>(q) * len + (i % len);
    const long long id = ids[l * i_stride + o];
    if (id < 0) return 0ull;  // empty slot
    return make_key(v[l * v_stride + o], static_cast<uint32_t>(id));
  }
};

__device__ __forceinline__ void emit_key(uint64_t key, int rank, long long id_offset, float* out_v,
                                         long long* out_i) {
  if (key == 0ull) {
    out_v[rank] = -INFINITY;
    out_i[rank] = -1;
  } else {
    out_v[rank] = key_score(key);
    out_i[rank] = static_cast<long long>(key_row(key)) + id_offset;
  }
}

// One warp: selects the k best keys of acc(0..m) and writes them in rank order.
// Empty keys (0) fill the tail when fewer than k real candidates exist.
template <class Acc>
__device__ void select_and_emit(const Acc& acc, int m, int k, long long id_offset, uint32_t* hist,
                                uint64_t* sel, float* out_v, long long* out_i, int lane) {
  const uint64_t kth = (m > k) ? warp_kth_key(acc, m, k, hist, lane) : 0ull;
  int cnt = 0;
  for (int i0 = 0; i0 < m; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t key = i < m ? acc(i) : 0ull;
    const bool take = i < m && key != 0ull && key >= kth;
    const unsigned bal = __ballot_sync(kFullMask, take);
    if (take) {
      const int pos = cnt + __popc(bal & ((1u << lane) - 1u));
      if (pos < k) sel[pos] = key;
    }
    cnt += __popc(bal);
  }
  cnt = min(cnt, k);
  for (int j = cnt + lane; j < k; j += 32) sel[j] = 0ull;
  __syncwarp();
  for (int j = lane; j < k; j += 32) {
    const uint64_t key = sel[j];
    int rank = 0;
    for (int t = 0; t < k; ++t) {
      const uint64_t o = sel[t];
      rank += (o > key) || (o == key && t < j);
    }
    emit_key(key, rank, id_offset, out_v, out_i);
  }
  __syncwarp();
}

// One CTA per query. Warp 0 forms the query's bound: the kernel's running
// bound (a.bounds) raised to the tops_m-th largest per-list published score.
// All eight warps then walk the query's lists, one list per lane up to its key
// count (eight loads in flight), and append the keys at or above the bound -- typically one
// to three times k of them -- to a shared survivor buffer; warp 0 radix-selects
// the k-th best survivor, the k winners are gathered, and every thread writes
// some of them straight to their output rank (the number of larger winners).
// If more survivors than the buffer holds appear (no bound, or a weak one),
// warp 0 selects over all keys instead.
__global__ void __launch_bounds__(kKeysThreads) merge_keys_kernel(const MergeKeysArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = blockIdx.x;
  const int scap = survivor_cap(a.k);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem);
  uint64_t* sel = reinterpret_cast<uint64_t*>(smem + 256 * 4);
  uint64_t* surv = sel + a.k;
  int* s_cnt = reinterpret_cast<int*>(surv + scap);  // [0] survivors, [1] winners
  uint32_t* s_bound = reinterpret_cast<uint32_t*>(s_cnt + 2);
  int* s_warp = reinterpret_cast<int*>(s_bound + 2);  // [kKeysWarps]
  int* s_off = s_warp + kKeysWarps;                   // [kScanLists]
  // Launched as a programmatic dependent of the search kernel: everything the
  // search kernel wrote is visible once this returns. (It does not release the
  // next kernel early: measured, letting the next call's ingest and workspace
  // clear become resident during the merge gained nothing.)
  grid_dependency_wait();
  const uint64_t* base = a.part + static_cast<size_t>(q) * a.lists * a.stride;
  const int* counts = a.counts ? a.counts + static_cast<size_t>(q) * a.lists : nullptr;
  float* out_v = a.out_v + static_cast<size_t>(q) * a.k;
  long long* out_i = a.out_i + static_cast<size_t>(q) * a.k;

  if (warp == 0) {
    uint32_t bound = 0;
    if (a.bounds != nullptr) {
      asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(bound) : "l"(a.bounds + q));
      // Per-lane register arrays sized to the list count: the bisection
      // visits every slot of the array at each of its steps.
      const uint32_t* tq = a.tops + static_cast<size_t>(q) * a.tops_n;
      if (a.tops != nullptr) {
        if (a.tops_n <= 32 * 5) bound = max(bound, warp_kth_top<5>(tq, a.tops_n, a.tops_m, lane));
        else if (a.tops_n <= 32 * 10) bound = max(bound, warp_kth_top<10>(tq, a.tops_n, a.tops_m, lane));
        else if (a.tops_n <= 32 * kMergeTopsPerLane)
          bound = max(bound, warp_kth_top<kMergeTopsPerLane>(tq, a.tops_n, a.tops_m, lane));
      }
    }
    if (lane == 0) {
      *s_bound = bound;
      s_cnt[0] = 0;
      s_cnt[1] = 0;
    }
  }
  __syncthreads();
  const uint32_t bound = *s_bound;
  const PartKeys all{base, counts, a.stride, a.per_list};
  const int m = a.lists * a.stride;
  if (bound == 0) {  // nothing to filter with
    if (warp == 0) select_and_emit(all, m, a.k, a.id_offset, hist, sel, out_v, out_i, lane);
    return;
  }

  const int S = a.stride;
  // Appends the keys of one batch that are at or above the bound (whole warp).
  auto keep_batch = [&](const uint64_t (&keys)[kKeysBatch]) {
#pragma unroll
    for (int u = 0; u < kKeysBatch; ++u) {
      const bool keep = keys[u] != 0ull && static_cast<uint32_t>(keys[u] >> 32) >= bound;
      const unsigned bal = __ballot_sync(kFullMask, keep);
      if (bal) {
        int pos = 0;
        if (lane == __ffs(bal) - 1) pos = atomicAdd(s_cnt, __popc(bal));
        pos = __shfl_sync(kFullMask, pos, __ffs(bal) - 1) + __popc(bal & ((1u << lane) - 1u));
        if (keep && pos < scap) surv[pos] = keys[u];
      }
    }
  };
  if (counts == nullptr || a.lists <= kScanLists) {
    // The used keys as one flat run: packed lists directly, counted lists
    // through a block-wide exclusive scan of their counts (s_off) and a binary
    // search per key. Every thread keeps eight loads in flight.
    int total;
    if (counts == nullptr) {
      total = a.lists * a.per_list;
    } else {
      const int per = (a.lists + kKeysThreads - 1) / kKeysThreads;  // <= kScanLists / 256
      int mine[kScanLists / kKeysThreads];
      int sum = 0;
#pragma unroll
      for (int u = 0; u < kScanLists / kKeysThreads; ++u) {
        const int l = threadIdx.x * per + u;
        mine[u] = (u < per && l < a.lists) ? min(max(counts[l], 0), S) : 0;
        sum += mine[u];
      }
      int incl = sum;  // warp inclusive scan, then across warps
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) s_warp[warp] = incl;
      __syncthreads();
      int before = 0;
      total = 0;
#pragma unroll
      for (int w = 0; w < kKeysWarps; ++w) {
        const int t = s_warp[w];
        before += w < warp ? t : 0;
        total += t;
      }
      int excl = before + incl - sum;
#pragma unroll
      for (int u = 0; u < kScanLists / kKeysThreads; ++u) {
        const int l = threadIdx.x * per + u;
        if (u < per && l < a.lists) s_off[l] = excl;
        excl += mine[u];
      }
      __syncthreads();
    }
    for (int i0 = 0; i0 < total; i0 += kKeysThreads * kKeysBatch) {
      uint64_t keys[kKeysBatch];
#pragma unroll
      for (int u = 0; u < kKeysBatch; ++u) {
        const int i = i0 + u * kKeysThreads + static_cast<int>(threadIdx.x);
        keys[u] = 0ull;
        if (i < total) {
          if (counts == nullptr) {
            keys[u] = base[i];
          } else {
            int lo = 0, hi = a.lists - 1;  // last list whose offset is <= i
            while (lo < hi) {
              const int mid = (lo + hi + 1) >> 1;
              if (s_off[mid] <= i) lo = mid;
              else hi = mid - 1;
            }
            keys[u] = base[static_cast<size_t>(lo) * S + (i - s_off[lo])];
          }
        }
      }
      keep_batch(keys);
    }
  } else {
    // Many counted lists: lane l of warp w walks list 32 * (8g + w) + l up to
    // its count, eight keys in flight per lane.
    for (int l0 = warp * 32; l0 < a.lists; l0 += kKeysWarps * 32) {
      const int l = l0 + lane;
      const int used = l < a.lists ? min(max(counts[l], 0), S) : 0;
      const int most = __reduce_max_sync(kFullMask, used);
      const uint64_t* lp = base + static_cast<size_t>(l) * S;
      for (int j0 = 0; j0 < most; j0 += kKeysBatch) {
        uint64_t keys[kKeysBatch];
#pragma unroll
        for (int u = 0; u < kKeysBatch; ++u) keys[u] = (j0 + u < used) ? lp[j0 + u] : 0ull;
        keep_batch(keys);
      }
    }
  }
  __syncthreads();
  const int cnt = s_cnt[0];
  if (cnt > scap) {
    if (warp == 0) select_and_emit(all, m, a.k, a.id_offset, hist, sel, out_v, out_i, lane);
    return;
  }
  if (cnt <= 32 && a.k <= 32) {
    // Typical for small k (the bound leaves a few dozen keys at most): warp 0
    // ranks the survivors against each other directly.
    if (warp == 0) {
      const uint64_t key = lane < cnt ? surv[lane] : 0ull;
      int rank = 0;
#pragma unroll
      for (int t = 0; t < 32; ++t) rank += shfl_u64(key, t) > key ? 1 : 0;
      if (lane < cnt && rank < a.k) emit_key(key, rank, a.id_offset, out_v, out_i);
      for (int j = cnt + lane; j < a.k; j += 32) emit_key(0ull, j, a.id_offset, out_v, out_i);
    }
    return;
  }
  if (cnt <= kKeysThreads) {
    // At most one survivor per thread: each ranks its own against all the
    // others (shared-memory broadcast reads) and, if it ranks within k, writes
    // it to its output slot -- one pass of the whole CTA instead of a
    // single-warp radix select, a gather and a second ranking pass (C4 k=100:
    // 6.0 -> 3.6 us). Keys are unique, so the ranks are too. (Four survivors
    // per thread, to cover k = 256, measured slower everywhere: the extra
    // registers cost the whole kernel.)
    const int i = threadIdx.x;
    if (i < cnt) {
      const uint64_t key = surv[i];
      int rank = 0;
#pragma unroll 4
      for (int t = 0; t < cnt; ++t) rank += surv[t] > key ? 1 : 0;
      if (rank < a.k) emit_key(key, rank, a.id_offset, out_v, out_i);
    }
    for (int j = cnt + i; j < a.k; j += kKeysThreads) emit_key(0ull, j, a.id_offset, out_v, out_i);
    return;
  }
  // k-th best survivor (warp 0), then the winners (keys are unique, so exactly
  // min(k, cnt) survivors are >= it).
  if (warp == 0) {
    const uint64_t kth = cnt > a.k ? warp_kth_key(ContigKeys{surv}, cnt, a.k, hist, lane) : 0ull;
    if (lane == 0) *reinterpret_cast<uint64_t*>(hist) = kth;
  }
  __syncthreads();
  const uint64_t kth = *reinterpret_cast<const uint64_t*>(hist);
  for (int i0 = warp * 32; i0 < cnt; i0 += kKeysThreads) {
    const int i = i0 + lane;
    const uint64_t key = i < cnt ? surv[i] : 0ull;
    const bool take = i < cnt && key >= kth;
    const unsigned bal = __ballot_sync(kFullMask, take);
    if (bal) {
      int pos = 0;
      if (lane == __ffs(bal) - 1) pos = atomicAdd(s_cnt + 1, __popc(bal));
      pos = __shfl_sync(kFullMask, pos, __ffs(bal) - 1) + __popc(bal & ((1u << lane) - 1u));
      if (take && pos < a.k) sel[pos] = key;
    }
  }
  __syncthreads();
  const int won = min(s_cnt[1], a.k);
  for (int j = won + threadIdx.x; j < a.k; j += kKeysThreads) sel[j] = 0ull;
  __syncthreads();
  for (int j = threadIdx.x; j < a.k; j += kKeysThreads) {
    const uint64_t key = sel[j];
    int rank = 0;
    for (int t = 0; t < a.k; ++t) {
      const uint64_t o = sel[t];
      rank += (o > key) || (o == key && t < j);
    }
    emit_key(key, rank, a.id_offset, out_v, out_i);
  }
}

__global__ void __launch_bounds__(kMergeWarps * 32) merge_lists_kernel(const MergeListsArgs a) {
  extern __shared__ uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = blockIdx.x * kMergeWarps + warp;
  uint8_t* mine = smem + static_cast<size_t>(warp) * merge_warp_bytes(a.k);
  uint32_t* hist = reinterpret_cast<uint32_t*>(mine);
  uint64_t* sel = reinterpret_cast<uint64_t*>(mine + 256 * 4);
  if (q >= a.b) return;
  const ListKeys acc{a.v, a.ids, a.v_stride, a.i_stride, a.len, q};
  const int m = a.lists * a.len;
  float* out_v = a.out_v + static_cast<size_t>(q) * a.k;
  long long* out_i = a.out_i + static_cast<size_t>(q) * a.k;
  if (m <= kMergeStageKeys) {
    // Each (score, id) pair is read from global memory once, four pairs in
    // flight per lane, and becomes a key in shared memory for the selection.
    uint64_t* stage = sel + a.k;
    for (int i0 = 0; i0 < m; i0 += 128) {
      uint64_t key[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u + lane;
        key[u] = i < m ? acc(i) : 0ull;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u + lane;
        if (i < m) stage[i] = key[u];
      }
    }
    __syncwarp();
    select_and_emit(ContigKeys{stage}, m, a.k, 0, hist, sel, out_v, out_i, lane);
    return;
  }
  select_and_emit(acc, m, a.k, 0, hist, sel, out_v, out_i, lane);
}

size_t merge_smem(int k) { return kMergeWarps * merge_warp_bytes(k); }

// Workspace preparation before a search: zeroes the cleared words and, for
// padded query tiles, copies the queries (16-byte chunks) into the padded buffer
// with zero rows after them.
__global__ void __launch_bounds__(256) prepare_kernel(uint32_t* p, size_t words, const uint4* q_src, uint4* q_dst,
                                                      size_t q_chunks, size_t pad_chunks) {
  grid_launch_dependents();
  // Launched programmatically: the previous kernel (the query ingest, or the
  // previous call's merge, which reads the workspace) finishes first.
  grid_dependency_wait();
  const size_t stride = static_cast<size_t>(gridDim.x) * 256;
  for (size_t i = blockIdx.x * 256ull + threadIdx.x; i < words; i += stride) p[i] = 0u;
  for (size_t i = blockIdx.x * 256ull + threadIdx.x; i < pad_chunks; i += stride)
    q_dst[i] = i < q_chunks ? q_src[i] : make_uint4(0u, 0u, 0u, 0u);
}

}  // namespace

cudaError_t merge_keys_launch(const MergeKeysArgs& a, cudaStream_t stream) {
  if (a.k < 1 || a.k > kMergeMaxK || a.b < 1 || a.stride < 1) return cudaErrorInvalidValue;
  // Lists without counts must be packed (the filter walks them as one run).
  if (!a.counts && a.per_list != a.stride) return cudaErrorInvalidValue;
  const size_t smem = keys_smem(a.k);
  cudaError_t e = cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // Programmatic dependent launch: the merge grid may be scheduled while the
  // search kernel's last CTAs finish (it waits for their results on the device).
  return launch_programmatic(merge_keys_kernel, dim3(static_cast<unsigned>(a.b)), dim3(kKeysThreads), smem,
                             stream, a);
}

cudaError_t prepare_launch(void* p, size_t bytes, const void* q_src, void* q_dst, int b, int d_pad,
                           int rows_pad, cudaStream_t stream) {
  const size_t words = bytes / 4;
  const size_t row_chunks = static_cast<size_t>(d_pad) / 8;  // 16-byte chunks per fp16 row
  const size_t q_chunks = q_dst ? static_cast<size_t>(b) * row_chunks : 0;
  const size_t pad_chunks = q_dst ? static_cast<size_t>(rows_pad) * row_chunks : 0;
  const size_t work = std::max(words, pad_chunks);
  if (work == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>(std::min<size_t>((work + 255) / 256, 1024));
  return launch_programmatic(prepare_kernel, dim3(grid), dim3(256), 0, stream, static_cast<uint32_t*>(p), words,
                             static_cast<const uint4*>(q_src), static_cast<uint4*>(q_dst), q_chunks, pad_chunks);
}

cudaError_t merge_lists_launch(const MergeListsArgs& a, cudaStream_t stream) {
  if (a.k < 1 || a.k > kMergeMaxK || a.b < 1) return cudaErrorInvalidValue;
  const size_t smem = merge_smem(a.k);
  cudaError_t e = cudaFuncSetAttribute(merge_lists_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>((a.b + kMergeWarps - 1) / kMergeWarps);
  merge_lists_kernel<<<grid, kMergeWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace cvs
