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
#include "cvs_device.cuh"
#include "cvs_kernels.h"
#include "cvs_select.cuh"

namespace cvs {

namespace {

constexpr int kMergeWarps = 2;
constexpr int kMergeMaxK = 1024;
constexpr int kSurvivorCap = 512;
constexpr int kMergeTopsPerLane = 16;  // up to 512 lists per query

// Shared memory per warp: radix histogram, k selected keys, survivor buffer.
__host__ __device__ constexpr size_t merge_warp_bytes(int k) {
  return 256 * 4 + static_cast<size_t>(k) * 8 + static_cast<size_t>(kSurvivorCap) * 8;
}

struct PartKeys {
  const uint64_t* p;  // this query's [lists][stride] block
  int stride;
  int per_list;
  __device__ __forceinline__ uint64_t operator()(int i) const {
    if (stride == per_list) return p[i];
    return p[static_cast<size_t>(i / per_list) * stride + (i % per_list)];
  }
};

struct ListKeys {
  const float* v;
  const long long* ids;
  int b;
  int len;
  int q;
  __device__ __forceinline__ uint64_t operator()(int i) const {
    const size_t o = (static_cast<size_t>(i / len) * b + q) * len + (i % len);
    const long long id = ids[o];
    if (id < 0) return 0ull;  // empty slot
    return make_key(v[o], static_cast<uint32_t>(id));
  }
};

// Selects the k best keys of acc(0..m) and writes them in rank order. Empty
// keys (0) fill the tail when fewer than k real candidates exist.
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
    if (key == 0ull) {
      out_v[rank] = -INFINITY;
      out_i[rank] = -1;
    } else {
      out_v[rank] = key_score(key);
      out_i[rank] = static_cast<long long>(key_row(key)) + id_offset;
    }
  }
  __syncwarp();
}

// Per query: when the search kernel left a lower bound on the query's k-th best
// score (a.bounds), one coalesced pass keeps only the keys at or above it --
// typically a few times k of the lists*k keys -- in shared memory, and the
// selection runs there. Without a bound, or if more than kSurvivorCap keys
// survive, the selection runs over all keys.
__global__ void __launch_bounds__(kMergeWarps * 32) merge_keys_kernel(const MergeKeysArgs a) {
  extern __shared__ uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = blockIdx.x * kMergeWarps + warp;
  uint8_t* mine = smem + static_cast<size_t>(warp) * merge_warp_bytes(a.k);
  uint32_t* hist = reinterpret_cast<uint32_t*>(mine);
  uint64_t* sel = reinterpret_cast<uint64_t*>(mine + 256 * 4);
  uint64_t* surv = sel + a.k;
  if (q >= a.b) return;  // whole warp
  const PartKeys acc{a.part + static_cast<size_t>(q) * a.lists * a.stride, a.stride, a.per_list};
  const int m = a.lists * a.per_list;
  float* out_v = a.out_v + static_cast<size_t>(q) * a.k;
  long long* out_i = a.out_i + static_cast<size_t>(q) * a.k;
  if (a.bounds != nullptr) {
    uint32_t bound;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(bound) : "l"(a.bounds + q));
    // The k-th largest of the lists' final best scores is usually a much
    // tighter bound than the kernel's running one.
    if (a.tops != nullptr && a.tops_n <= 32 * kMergeTopsPerLane)
      bound = max(bound, warp_kth_top<kMergeTopsPerLane>(a.tops + static_cast<size_t>(q) * a.tops_n,
                                                         a.tops_n, a.tops_m, lane));
    int cnt = 0;
    constexpr int kBatch = 8;  // loads in flight per lane before any is used
    for (int i0 = 0; i0 < m; i0 += 32 * kBatch) {
      uint64_t keys[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + 32 * u + lane;
        keys[u] = i < m ? acc(i) : 0ull;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const bool keep = keys[u] != 0ull && static_cast<uint32_t>(keys[u] >> 32) >= bound;
        const unsigned bal = __ballot_sync(kFullMask, keep);
        if (keep) {
          const int pos = cnt + __popc(bal & ((1u << lane) - 1u));
          if (pos < kSurvivorCap) surv[pos] = keys[u];
        }
        cnt += __popc(bal);
      }
    }
    __syncwarp();
    if (cnt <= kSurvivorCap) {
      select_and_emit(ContigKeys{surv}, cnt, a.k, a.id_offset, hist, sel, out_v, out_i, lane);
      return;
    }
  }
  select_and_emit(acc, m, a.k, a.id_offset, hist, sel, out_v, out_i, lane);
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
  const ListKeys acc{a.v, a.ids, a.b, a.len, q};
  select_and_emit(acc, a.lists * a.len, a.k, 0, hist, sel, a.out_v + static_cast<size_t>(q) * a.k,
                  a.out_i + static_cast<size_t>(q) * a.k, lane);
}

size_t merge_smem(int k) { return kMergeWarps * merge_warp_bytes(k); }

}  // namespace

cudaError_t merge_keys_launch(const MergeKeysArgs& a, cudaStream_t stream) {
  if (a.k < 1 || a.k > kMergeMaxK || a.b < 1) return cudaErrorInvalidValue;
  const size_t smem = merge_smem(a.k);
  cudaError_t e = cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>((a.b + kMergeWarps - 1) / kMergeWarps);
  merge_keys_kernel<<<grid, kMergeWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
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
