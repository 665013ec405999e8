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

template <int T>
__global__ void __launch_bounds__(kIngestThreads) ingest_kernel(const void* src, long long n, int d,
                                                                long long src_stride, int d_pad,
                                                                int cosine, __half* dst) {
  ingest_prologue();
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
                                                                    int cosine, __half* dst) {
  ingest_prologue();
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
                       __half* dst, unsigned grid, cudaStream_t stream) {
  const int cpl = (d_pad / 8 + 31) / 32;
#define CVS_INGEST_VEC(C)                                                                          \
  if (cpl <= C) {                                                                                 \
    return launch_programmatic(ingest_vec_kernel<T, C>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, \
                               src_stride, d_pad, cosine, dst);                                    \
  }
  CVS_INGEST_VEC(1) CVS_INGEST_VEC(2) CVS_INGEST_VEC(3) CVS_INGEST_VEC(4) CVS_INGEST_VEC(6) CVS_INGEST_VEC(8)
#undef CVS_INGEST_VEC
  return cudaErrorInvalidValue;
}

size_t elem_size(int t) { return t == kSrcF32 ? 4 : t == kSrcF64 ? 8 : 2; }

}  // namespace

cudaError_t ingest_launch(const void* src, int src_dtype, long long n, int d, long long src_stride,
                          int d_pad, int cosine, __half* dst, int num_sms, cudaStream_t stream) {
  if (n < 0 || d < 1 || d > 32 * kIngestMaxPerLane || d_pad < d) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const long long want = (n + (kIngestThreads / 32) - 1) / (kIngestThreads / 32);
  const unsigned grid = static_cast<unsigned>(std::min<long long>(want, static_cast<long long>(num_sms) * 8));
  const size_t es = elem_size(src_dtype);
  const bool vec = d % 8 == 0 && d_pad <= 2048 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
                   (static_cast<size_t>(src_stride) * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  if (vec) {
    switch (src_dtype) {
      case kSrcF32: return launch_vec<kSrcF32>(src, n, d, src_stride, d_pad, cosine, dst, grid, stream);
      case kSrcF16: return launch_vec<kSrcF16>(src, n, d, src_stride, d_pad, cosine, dst, grid, stream);
      case kSrcBF16: return launch_vec<kSrcBF16>(src, n, d, src_stride, d_pad, cosine, dst, grid, stream);
      case kSrcF64: return launch_vec<kSrcF64>(src, n, d, src_stride, d_pad, cosine, dst, grid, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  cudaError_t e;
  switch (src_dtype) {
    case kSrcF32:
      e = launch_programmatic(ingest_kernel<kSrcF32>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst);
      break;
    case kSrcF16:
      e = launch_programmatic(ingest_kernel<kSrcF16>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst);
      break;
    case kSrcBF16:
      e = launch_programmatic(ingest_kernel<kSrcBF16>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst);
      break;
    case kSrcF64:
      e = launch_programmatic(ingest_kernel<kSrcF64>, dim3(grid), dim3(kIngestThreads), 0, stream, src, n, d, src_stride,
                              d_pad, cosine, dst);
      break;
    default: return cudaErrorInvalidValue;
  }
  return e;
}

}  // namespace cvs
