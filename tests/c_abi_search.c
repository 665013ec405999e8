/*
 * A plain C program that uses the search library through include/cvs.h only:
 * no Python, no torch. It is what a non-Python host (a C/C++ service, or a
 * cgo / JNI / FFI binding) does -- allocate device memory with the CUDA
 * runtime, ingest a corpus, search raw fp32 queries, read the results back.
 *
 *   c_abi_search <dir> <n> <d> <b> <k> <cosine>
 *
 * The corpus and queries come from a fixed linear congruential generator
 * (uniform in [-1, 1)); the program writes them (fp32, row-major) and the
 * results to <dir>/corpus.f32, queries.f32, scores.f32, ids.i64 so that a test
 * can check them against a CPU oracle. Exit status 0 on success.
 * Test infrastructure for tests/test_c_abi_program_gpu.py.
 */
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "cvs.h"

static uint64_t g_state = 0x9E3779B97F4A7C15ull;

static float next_uniform(void) {
  g_state = g_state * 6364136223846793005ull + 1442695040888963407ull;
  return (float)((double)(g_state >> 40) / (double)(1ull << 24) * 2.0 - 1.0);
}

static int write_file(const char* dir, const char* name, const void* p, size_t bytes) {
  char path[4096];
  snprintf(path, sizeof(path), "%s/%s", dir, name);
  FILE* f = fopen(path, "wb");
  if (!f) return 1;
  size_t w = fwrite(p, 1, bytes, f);
  fclose(f);
  return w == bytes ? 0 : 1;
}

#define CHECK_CUDA(call)                                                        \
  do {                                                                          \
    cudaError_t e_ = (call);                                                    \
    if (e_ != cudaSuccess) {                                                    \
      fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));               \
      return 2;                                                                 \
    }                                                                           \
  } while (0)

#define CHECK_CVS(call)                                                         \
  do {                                                                          \
    cvs_status s_ = (call);                                                     \
    if (s_ != CVS_OK) {                                                         \
      fprintf(stderr, "%s: status %d: %s\n", #call, (int)s_, cvs_last_error()); \
      return 3;                                                                 \
    }                                                                           \
  } while (0)

int main(int argc, char** argv) {
  if (argc != 7) {
    fprintf(stderr, "usage: %s dir n d b k cosine\n", argv[0]);
    return 1;
  }
  const char* dir = argv[1];
  const int64_t n = atoll(argv[2]);
  const int d = atoi(argv[3]);
  const int64_t b = atoll(argv[4]);
  const int k = atoi(argv[5]);
  const int cosine = atoi(argv[6]);
  const int d_pad = cvs_pad_width(d);
  if (cvs_abi_version() != CVS_ABI_VERSION) return 4;

  float* x = (float*)malloc((size_t)n * d * sizeof(float));
  float* q = (float*)malloc((size_t)b * d * sizeof(float));
  float* scores = (float*)malloc((size_t)b * k * sizeof(float));
  int64_t* ids = (int64_t*)malloc((size_t)b * k * sizeof(int64_t));
  if (!x || !q || !scores || !ids) return 5;
  for (size_t i = 0; i < (size_t)n * d; ++i) x[i] = next_uniform();
  for (size_t i = 0; i < (size_t)b * d; ++i) q[i] = next_uniform();

  void *x_src, *x_dev, *q_dev, *ws, *out_v, *out_i;
  size_t ws_bytes = 0;
  CHECK_CVS(cvs_search_workspace_size(b, n, d_pad, k, &ws_bytes));
  CHECK_CUDA(cudaMalloc(&x_src, (size_t)n * d * sizeof(float)));
  CHECK_CUDA(cudaMalloc(&x_dev, (size_t)n * d_pad * 2));
  CHECK_CUDA(cudaMalloc(&q_dev, (size_t)b * d * sizeof(float)));
  CHECK_CUDA(cudaMalloc(&ws, ws_bytes > 256 ? ws_bytes : 256));
  CHECK_CUDA(cudaMalloc(&out_v, (size_t)b * k * sizeof(float)));
  CHECK_CUDA(cudaMalloc(&out_i, (size_t)b * k * sizeof(int64_t)));
  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreate(&stream));
  CHECK_CUDA(cudaMemcpyAsync(x_src, x, (size_t)n * d * sizeof(float), cudaMemcpyHostToDevice, stream));
  CHECK_CUDA(cudaMemcpyAsync(q_dev, q, (size_t)b * d * sizeof(float), cudaMemcpyHostToDevice, stream));

  /* Corpus: fp32 -> fp16, normalised for cosine, zero-padded to d_pad. */
  CHECK_CVS(cvs_ingest(x_src, CVS_F32, n, d, d, d_pad, cosine, x_dev, (void*)stream));
  /* Two searches from the raw fp32 queries (the second reuses the workspace). */
  for (int rep = 0; rep < 2; ++rep)
    CHECK_CVS(cvs_search(q_dev, CVS_F32, b, d, d, cosine, x_dev, n, d_pad, k, 0, (float*)out_v,
                         (int64_t*)out_i, ws, ws_bytes > 256 ? ws_bytes : 256, (void*)stream));
  CHECK_CUDA(cudaMemcpyAsync(scores, out_v, (size_t)b * k * sizeof(float), cudaMemcpyDeviceToHost, stream));
  CHECK_CUDA(cudaMemcpyAsync(ids, out_i, (size_t)b * k * sizeof(int64_t), cudaMemcpyDeviceToHost, stream));
  CHECK_CUDA(cudaStreamSynchronize(stream));
  int code = 0;
  CHECK_CVS(cvs_poll_device_error(0, &code));

  if (write_file(dir, "corpus.f32", x, (size_t)n * d * sizeof(float)) ||
      write_file(dir, "queries.f32", q, (size_t)b * d * sizeof(float)) ||
      write_file(dir, "scores.f32", scores, (size_t)b * k * sizeof(float)) ||
      write_file(dir, "ids.i64", ids, (size_t)b * k * sizeof(int64_t)))
    return 6;
  cudaFree(x_src);
  cudaFree(x_dev);
  cudaFree(q_dev);
  cudaFree(ws);
  cudaFree(out_v);
  cudaFree(out_i);
  cudaStreamDestroy(stream);
  free(x);
  free(q);
  free(scores);
  free(ids);
  printf("c_abi_search ok\n");
  return 0;
}
