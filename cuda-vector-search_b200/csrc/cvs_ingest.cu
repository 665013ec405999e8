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
// d == d_pad, src_stride == d_pad).
#include <cuda_bf16.h>

#include "cvs_device.cuh"
#include "cvs_kernels.h"

namespace cvs {

namespace {

constexpr int kIngestThreads = 256;
constexpr int kIngestMaxPerLane = 64;  // d <= 2048 handled from registers

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

}  // namespace

cudaError_t ingest_launch(const void* src, int src_dtype, long long n, int d, long long src_stride,
                          int d_pad, int cosine, __half* dst, int num_sms, cudaStream_t stream) {
  if (n < 0 || d < 1 || d > 32 * kIngestMaxPerLane || d_pad < d) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const long long want = (n + (kIngestThreads / 32) - 1) / (kIngestThreads / 32);
  const unsigned grid = static_cast<unsigned>(std::min<long long>(want, static_cast<long long>(num_sms) * 8));
  switch (src_dtype) {
    case kSrcF32: ingest_kernel<kSrcF32><<<grid, kIngestThreads, 0, stream>>>(src, n, d, src_stride, d_pad, cosine, dst); break;
    case kSrcF16: ingest_kernel<kSrcF16><<<grid, kIngestThreads, 0, stream>>>(src, n, d, src_stride, d_pad, cosine, dst); break;
    case kSrcBF16: ingest_kernel<kSrcBF16><<<grid, kIngestThreads, 0, stream>>>(src, n, d, src_stride, d_pad, cosine, dst); break;
    case kSrcF64: ingest_kernel<kSrcF64><<<grid, kIngestThreads, 0, stream>>>(src, n, d, src_stride, d_pad, cosine, dst); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace cvs
