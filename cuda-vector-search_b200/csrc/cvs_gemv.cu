// CUDA-core GEMV + top-k for one to eight queries (k <= 32). One query: the
// HBM-bound case, at every corpus size. Two to eight: only on small corpora
// (at most two tiles per CTA for the tcgen05 kernel, and little work: the
// planner's gemv_preferred), where that kernel's dry tile and bound wait, not
// the stream, set its time; on larger corpora the tcgen05 kernel streams at
// least as fast from two queries on, and from three on this kernel's per-row
// arithmetic exceeds the stream. Replaces the
// reference's fused kernel at bq=16 for tiny batches
// (cuda_vector_search/csrc/kernels.cu:313-371 run with nq = 1..8, where the
// other query rows of its 16 are padding).
//
// Each warp owns whole corpus rows: lane l reads 16-byte chunks l, l+32, ... of
// a row (a warp load is 512 contiguous bytes), R rows are loaded before any math
// so R * ceil(d_pad/256) 16-byte loads per lane are in flight. Products use the
// sm_100 mixed-precision FMA (fp16 x fp16 + fp32 -> fp32, no conversions); the
// row sum is a butterfly shuffle reduction, so every lane ends with the same
// score and the top-k test is warp-uniform.
//
// Per (warp, query) top-k: a sorted list spread over the 32 lanes (lane j holds
// the j-th best). A new candidate finds its slot with one ballot and the lanes
// below it shift down by one with one shuffle. At the end the CTA merges its
// warps' lists with the warp radix select and writes k keys per query.
#include <map>
#include <mutex>
#include <utility>

#include "cvs_device.cuh"
#include "cvs_kernels.h"
#include "cvs_select.cuh"

namespace cvs {

namespace {

constexpr int kWarps = kGemvThreads / 32;

// acc += x.lo * q.lo, acc2 += x.hi * q.hi (fp16 products, fp32 sums).
__device__ __forceinline__ void fma_h2(uint32_t x2, uint32_t q2, float& acc, float& acc2) {
  asm("{ .reg .f16 xl, xh, ql, qh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "mov.b32 {ql, qh}, %3;\n\t"
      "fma.rn.f32.f16 %0, xl, ql, %0;\n\t"
      "fma.rn.f32.f16 %1, xh, qh, %1; }"
      : "+f"(acc), "+f"(acc2)
      : "r"(x2), "r"(q2));
}

__device__ __forceinline__ float warp_allreduce_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
  return v;
}

// Sorted-list insert of a warp-uniform candidate (s, row) that ranks before the
// current k-th entry. Lane j holds entry j.
__device__ __forceinline__ void warp_list_insert(float& v, uint32_t& id, float s, uint32_t row,
                                                 int lane) {
  const bool after = (s > v) || (s == v && row < id);  // candidate ranks before my entry
  const unsigned m = __ballot_sync(kFullMask, after);   // a suffix of the lanes
  const int p = __ffs(m) - 1;
  const float vu = __shfl_up_sync(kFullMask, v, 1);
  const uint32_t iu = __shfl_up_sync(kFullMask, id, 1);
  if (lane > p) {
    v = vu;
    id = iu;
  } else if (lane == p) {
    v = s;
    id = row;
  }
}

template <int NQ, int CPL, int R>
__global__ void __launch_bounds__(kGemvThreads) gemv_topk_kernel(const GemvArgs a) {
  __shared__ uint64_t cand[NQ][kWarps][kGemvMaxK];
  __shared__ uint32_t hist[kWarps][256];

  // Launched programmatically after the workspace clear: wait for it (and for
  // the kernels before it) before reading anything.
  grid_dependency_wait();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int chunks = a.d_pad >> 3;  // 16-byte chunks per row
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);

  uint4 qv[NQ][CPL];
#pragma unroll
  for (int qi = 0; qi < NQ; ++qi)
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane + 32 * j;
      qv[qi][j] = (qi < a.b && c < chunks)
                      ? __ldg(reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(qi) * a.d_pad) + c)
                      : zero;
    }

  float lv[NQ];
  uint32_t li[NQ];
  float thr[NQ];
#pragma unroll
  for (int qi = 0; qi < NQ; ++qi) {
    lv[qi] = -INFINITY;
    li[qi] = 0xFFFFFFFFu;
    thr[qi] = -INFINITY;
  }

  const long long r0 = static_cast<long long>(blockIdx.x) * a.rows_per_seg;
  const long long r1 = min(static_cast<long long>(a.n), r0 + a.rows_per_seg);
  const int kk = a.k;

  for (long long base = r0 + static_cast<long long>(warp) * R; base < r1;
       base += static_cast<long long>(kWarps) * R) {
    uint4 xv[R][CPL];
#pragma unroll
    for (int rr = 0; rr < R; ++rr)
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int c = lane + 32 * j;
        const long long row = base + rr;
        xv[rr][j] = (row < r1 && c < chunks)
                        ? __ldcs(reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(row) * a.d_pad) + c)
                        : zero;
      }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      float s[NQ];
#pragma unroll
      for (int qi = 0; qi < NQ; ++qi) {
        float acc = 0.f, acc2 = 0.f;
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          fma_h2(xv[rr][j].x, qv[qi][j].x, acc, acc2);
          fma_h2(xv[rr][j].y, qv[qi][j].y, acc, acc2);
          fma_h2(xv[rr][j].z, qv[qi][j].z, acc, acc2);
          fma_h2(xv[rr][j].w, qv[qi][j].w, acc, acc2);
        }
        s[qi] = warp_allreduce_sum(acc + acc2);
      }
      const long long row = base + rr;
      if (row < r1) {
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) {
          if (s[qi] > thr[qi]) {  // warp-uniform
            warp_list_insert(lv[qi], li[qi], s[qi], static_cast<uint32_t>(row), lane);
            thr[qi] = __shfl_sync(kFullMask, lv[qi], kk - 1);
          }
        }
      }
    }
  }

  // Merge the warps' lists: k keys per (query, CTA).
#pragma unroll
  for (int qi = 0; qi < NQ; ++qi) {
    cand[qi][warp][lane] = (lane < kk && lv[qi] != -INFINITY) ? make_key(lv[qi], li[qi]) : 0ull;
  }
  __syncthreads();
  for (int qi = warp; qi < NQ && qi < a.b; qi += kWarps) {
    // Lists are stored at stride kGemvMaxK; only their first k slots count.
    const uint64_t* base = &cand[qi][0][0];
    const int m = kWarps * kk;
    struct Acc {
      const uint64_t* p;
      int k;
      __device__ uint64_t operator()(int i) const { return p[(i / k) * kGemvMaxK + (i % k)]; }
    } acc{base, kk};
    const uint64_t kth = warp_kth_key(acc, m, kk, hist[warp], lane);
    // This CTA's k-th best bounds the query's k-th best from below; the merge
    // uses the largest such bound to skip most candidates.
    if (lane == 0 && kth != 0ull) atomicMax(a.bounds + qi, static_cast<uint32_t>(kth >> 32));
    // ... and its best score is published for the merge's k-th-largest-maximum bound.
    uint64_t best = 0ull;
    for (int i = lane; i < m; i += 32) best = max(best, acc(i));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) best = max(best, shfl_u64(best, lane ^ off));
    if (lane == 0) a.tops[static_cast<size_t>(qi) * a.segs + blockIdx.x] = static_cast<uint32_t>(best >> 32);
    uint64_t* out = a.part + (static_cast<size_t>(qi) * a.segs + blockIdx.x) * kk;
    // Emit keys >= kth (exactly k when kth != 0); pad with empty keys otherwise.
    int pos = 0;
    for (int i0 = 0; i0 < m; i0 += 32) {
      const int i = i0 + lane;
      const uint64_t key = i < m ? acc(i) : 0ull;
      const bool take = i < m && key != 0ull && key >= kth;
      const unsigned bal = __ballot_sync(kFullMask, take);
      if (take) out[pos + __popc(bal & ((1u << lane) - 1u))] = key;
      pos += __popc(bal);
    }
    for (int j = pos + lane; j < kk; j += 32) out[j] = 0ull;
  }
}

using GemvKernel = void (*)(const GemvArgs);

template <int NQ, int CPL>
GemvKernel kernel_cpl() {
  return gemv_topk_kernel<NQ, CPL, 4>;
}

template <int NQ>
GemvKernel kernel_nq(int d_pad) {
  switch ((d_pad / 8 + 31) / 32) {
    case 1: return kernel_cpl<NQ, 1>();
    case 2: return kernel_cpl<NQ, 2>();
    case 3: return kernel_cpl<NQ, 3>();
    case 4: return kernel_cpl<NQ, 4>();
    default: return nullptr;
  }
}

// The instantiation for b queries (NQ = 1, 2, 4 or 8: a batch runs in the
// smallest that holds it, its missing queries zero) of width d_pad; CPL =
// 16-byte chunks per lane per row.
GemvKernel select_kernel(int b, int d_pad) {
  if (b <= 1) return kernel_nq<1>(d_pad);
  if (b == 2) return kernel_nq<2>(d_pad);
  if (b <= 4) return kernel_nq<4>(d_pad);
  return kernel_nq<8>(d_pad);
}

}  // namespace

bool gemv_supported(int b, int k, int d_pad) {
  return b >= 1 && b <= kGemvMaxBatch && k >= 1 && k <= kGemvMaxK && d_pad >= 64 && d_pad <= 1024;
}

// Resident blocks per SM of the instantiation that gemv_launch will use, so the
// grid is exactly one full wave.
int gemv_blocks_per_sm(int b, int d_pad) {
  GemvKernel k = select_kernel(b, d_pad);
  if (!k) return 1;
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> cache;  // (device, kernel) -> blocks
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(k));
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, kGemvThreads, 0) != cudaSuccess) blocks = 1;
  blocks = blocks > 0 ? blocks : 1;
  cache.emplace(key, blocks);
  return blocks;
}

cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t stream) {
  if (!gemv_supported(a.b, a.k, a.d_pad)) return cudaErrorInvalidValue;
  GemvKernel k = select_kernel(a.b, a.d_pad);
  if (!k) return cudaErrorInvalidValue;
  return launch_programmatic(k, dim3(a.segs), dim3(kGemvThreads), 0, stream, a);
}

}  // namespace cvs
