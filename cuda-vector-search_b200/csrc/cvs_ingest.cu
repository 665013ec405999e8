// Corpus / query ingest in one pass: source dtype -> fp16, optional L2
// normalisation, zero padding of the width to d_pad.
//
// Replaces the reference's storage path (cuda_vector_search/index.py:69-77):
// `x.to(device, float16)`, `_normalize_` (index.py:35-41: per row, fp32
// x / max(||x||, 1e-12) on the fp16-rounded values, rounded back to fp16) and
// `_pad_width` (index.py:27-32). The order of roundings is the reference's:
// the source is first rounded to fp16, the norm is taken in fp32 over those
// fp16 values, and the quotient is rounded to fp16 again.
//
// One warp per row; each lane keeps its slice of the row in registers between
// the norm and the write, so the kernel may run in place (src == dst, fp16,
// d == d_pad, src_stride == d_pad). Rows whose width is a multiple of 8 with
// 16-byte aligned source rows take a vectorised path (16-byte loads/stores).
#include <cuda_bf16.h>

#include "cvs_device.cuh"
#include "cvs_kernels.h"

namespace cvs {

namespace {

constexpr int kIngestThreads = 256;
constexpr int kIngestMaxPerLane = 64;  // d <= 2048 handled from registers

// The ingest kernels are launched programmatically (launch_programmatic): they
// may be scheduled while the previous kernel on the stream finishes, and wait
// for it (its writes to the source, its reads of memory the destination may
// reuse) before touching memory. The next kernel may likewise be scheduled
// early; it waits for this grid in the same way.
__device__ __forceinline__ void ingest_prologue() {
  grid_launch_dependents();
  grid_dependency_wait();
}

template <int T>
__device__ __forceinline__ __half load_as_half(const void* src, size_t i) {
  if constexpr (T == kSrcF32) return __float2half_rn(static_cast<const float*>(src)[i]);
  if constexpr (T == kSrcF16) return static_cast<const __half*>(src)[i];
  if constexpr (T == kSrcBF16) return __float2half_rn(__bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]));
  if constexpr (T == kSrcF64) return __double2half(static_cast<const double*>(src)[i]);
  return __half();
}

// Work a search launch adds to its query ingest (cvs_search): zero `words`
// 32-bit words at `p` (the workspace's bounds and counters) and write rows
// n .. rows_pad-1 of the destination as zeros (the padding rows of the last
// query tile), so that no separate preparation kernel is needed.
struct IngestExtra {
  uint32_t* p;
  size_t words;
  long long rows_pad;
};

__device__ __forceinline__ void ingest_extra(const IngestExtra& x, long long n, int d_pad, __half* dst) {
  const size_t tid = static_cast<size_t>(blockIdx.x) * kIngestThreads + threadIdx.x;
  const size_t nthreads = static_cast<size_t>(gridDim.x) * kIngestThreads;
  for (size_t i = tid; i < x.words; i += nthreads) x.p[i] = 0u;
  const size_t pad_chunks = static_cast<size_t>(x.rows_pad - n) * (d_pad / 8);  // 16-byte chunks
  uint4* zdst = reinterpret_cast<uint4*>(dst + static_cast<size_t>(n) * d_pad);
  for (size_t i = tid; i < pad_chunks; i += nthreads) zdst[i] = make_uint4(0u, 0u, 0u, 0u);
}

template <int T>
__global__ void __launch_bounds__(kIngestThreads) ingest_kernel(const void* src, long long n, int d,
                                                                long long src_stride, int d_pad,
                                                                int cosine, __half* dst, IngestExtra extra) {
  ingest_prologue();
  ingest_extra(extra, n, d_pad, dst);
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (kIngestThreads / 32);
  for (long long row = static_cast<long long>(blockIdx.x) * (kIngestThreads / 32) + (threadIdx.x >> 5);
       row < n; row += warps) {
    const size_t sbase = static_cast<size_t>(row) * src_stride;
    __half h[kIngestMaxPerLane];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kIngestMaxPerLane; ++j) {
      const int c = lane + 32 * j;
      h[j] = (c < d) ? load_as_half<T>(src, sbase + c) : __float2half_rn(0.f);
      const float f = __half2float(h[j]);
      ss = fmaf(f, f, ss);
    }
    float den = 1.f;
    if (cosine) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      den = fmaxf(sqrtf(ss), 1e-12f);
    }
    __syncwarp();
    const size_t dbase = static_cast<size_t>(row) * d_pad;
#pragma unroll
    for (int j = 0; j < kIngestMaxPerLane; ++j) {
      const int c = lane + 32 * j;
      if (c < d) {
        dst[dbase + c] = cosine ? __float2half_rn(__fdiv_rn(__half2float(h[j]), den)) : h[j];
      } else if (c < d_pad) {
        dst[dbase + c] = __float2half_rn(0.f);
      }
    }
  }
}

// Vectorised variant for d % 8 == 0 with 16-byte aligned source rows: lane l
// handles 8-element chunks l, l+32, ... (CPL of them), read with 16/32/64-byte
// loads and written as one 16-byte store each.
template <int T>
struct Chunk8 {
  static __device__ __forceinline__ void load(const void* src, size_t e, __half (&h)[8]) {
    if constexpr (T == kSrcF16 || T == kSrcBF16) {
      const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(src) + e);
      const uint16_t* w = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if constexpr (T == kSrcF16) h[j] = __ushort_as_half(w[j]);
        else h[j] = __float2half_rn(__bfloat162float(__ushort_as_bfloat16(w[j])));
      }
    } else if constexpr (T == kSrcF32) {
      const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(src) + e);
      const float4 a = f[0], b = f[1];
      h[0] = __float2half_rn(a.x); h[1] = __float2half_rn(a.y); h[2] = __float2half_rn(a.z); h[3] = __float2half_rn(a.w);
      h[4] = __float2half_rn(b.x); h[5] = __float2half_rn(b.y); h[6] = __float2half_rn(b.z); h[7] = __float2half_rn(b.w);
    } else {
      const double2* f = reinterpret_cast<const double2*>(static_cast<const double*>(src) + e);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const double2 v = f[j];
        h[2 * j] = __double2half(v.x);
        h[2 * j + 1] = __double2half(v.y);
      }
    }
  }
};

template <int T, int CPL>
__global__ void __launch_bounds__(kIngestThreads) ingest_vec_kernel(const void* src, long long n, int d,
                                                                    long long src_stride, int d_pad,
                                                                    int cosine, __half* dst, IngestExtra extra) {
  ingest_prologue();
  ingest_extra(extra, n, d_pad, dst);
  const int lane = threadIdx.x & 31;
  const int dchunks = d >> 3, pchunks = d_pad >> 3;
  const long long warps = static_cast<long long>(gridDim.x) * (kIngestThreads / 32);
  for (long long row = static_cast<long long>(blockIdx.x) * (kIngestThreads / 32) + (threadIdx.x >> 5);
       row < n; row += warps) {
    __half h[CPL][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane + 32 * j;
      if (c < dchunks) {
        Chunk8<T>::load(src, static_cast<size_t>(row) * src_stride + static_cast<size_t>(c) * 8, h[j]);
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) h[j][t] = __float2half_rn(0.f);
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float f = __half2float(h[j][t]);
        ss = fmaf(f, f, ss);
      }
    }
    float den = 1.f;
    if (cosine) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      den = fmaxf(sqrtf(ss), 1e-12f);
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane + 32 * j;
      if (c < pchunks) {
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int t = 0; t < 8; ++t)
          oh[t] = cosine ? __float2half_rn(__fdiv_rn(__half2float(h[j][t]), den)) : h[j][t];
        *reinterpret_cast<uint4*>(dst + static_cast<size_t>(row) * d_pad + static_cast<size_t>(c) * 8) = o;
      }
    }
  }
}

template <int T>
cudaError_t launch_vec(const void* src, long long n, int d, long long src_stride, int d_pad, int cosine,
                       __half* dst, unsigned grid, const IngestExtra& extra, cudaStream_t stream) {
  const int cpl = (d_pad / 8 + 31) / 32;
#define CVS_INGEST_VEC(C)                                                                          \
  if (cpl <= C) {                                                                                 \
    return launch_programmatic(ingest_vec_kernel<T, C>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, \
                               src_stride, d_pad, cosine, dst, extra);                             \
  }
  CVS_INGEST_VEC(1) CVS_INGEST_VEC(2) CVS_INGEST_VEC(3) CVS_INGEST_VEC(4) CVS_INGEST_VEC(6) CVS_INGEST_VEC(8)
#undef CVS_INGEST_VEC
  return cudaErrorInvalidValue;
}

size_t elem_size(int t) { return t == kSrcF32 ? 4 : t == kSrcF64 ? 8 : 2; }

}  // namespace

cudaError_t ingest_launch(const void* src, int src_dtype, long long n, int d, long long src_stride,
                          int d_pad, int cosine, __half* dst, int num_sms, cudaStream_t stream,
                          uint32_t* clear, size_t clear_words, long long rows_pad) {
  if (n < 0 || d < 1 || d > 32 * kIngestMaxPerLane || d_pad < d) return cudaErrorInvalidValue;
  if (rows_pad < n) rows_pad = n;
  if (n == 0 && rows_pad == 0 && clear_words == 0) return cudaSuccess;
  const IngestExtra extra{clear, clear ? clear_words : 0, rows_pad};
  // One warp per row; enough threads for the clear and the padding rows too.
  const long long extra_work = static_cast<long long>(std::max<size_t>(extra.words, static_cast<size_t>(rows_pad - n) * (d_pad / 8)));
  const long long want = std::max<long long>((n + (kIngestThreads / 32) - 1) / (kIngestThreads / 32),
                                             (extra_work + kIngestThreads - 1) / kIngestThreads);
  const unsigned grid = static_cast<unsigned>(std::max<long long>(1, std::min<long long>(want, static_cast<long long>(num_sms) * 8)));
  const size_t es = elem_size(src_dtype);
  const bool vec = d % 8 == 0 && d_pad <= 2048 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
                   (static_cast<size_t>(src_stride) * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  if (vec) {
    switch (src_dtype) {
      case kSrcF32: return launch_vec<kSrcF32>(src, n, d, src_stride, d_pad, cosine, dst, grid, extra, stream);
      case kSrcF16: return launch_vec<kSrcF16>(src, n, d, src_stride, d_pad, cosine, dst, grid, extra, stream);
      case kSrcBF16: return launch_vec<kSrcBF16>(src, n, d, src_stride, d_pad, cosine, dst, grid, extra, stream);
      case kSrcF64: return launch_vec<kSrcF64>(src, n, d, src_stride, d_pad, cosine, dst, grid, extra, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  cudaError_t e;
  switch (src_dtype) {
    case kSrcF32:
      e = launch_programmatic(ingest_kernel<kSrcF32>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst, extra);
      break;
    case kSrcF16:
      e = launch_programmatic(ingest_kernel<kSrcF16>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst, extra);
      break;
    case kSrcBF16:
      e = launch_programmatic(ingest_kernel<kSrcBF16>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst, extra);
      break;
    case kSrcF64:
      e = launch_programmatic(ingest_kernel<kSrcF64>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst, extra);
      break;
    default: return cudaErrorInvalidValue;
  }
  return e;
}

}  // namespace cvs
