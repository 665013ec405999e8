// Launch-side declarations shared by the kernel translation units and the
// C-ABI host code (cvs_capi.cu). Nothing here is part of the public ABI; the
// public entry points are declared in include/cvs.h.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

namespace cvs {

// ---- tcgen05 fused score + top-k / score-store kernel ----------------------
constexpr int kTcM = 128;          // queries per tile (MMA M; TMEM lanes)
constexpr int kTcN = 256;          // corpus rows per tile (MMA N; TMEM columns)
constexpr int kTcK = 64;           // halves per K slice (one 128-byte swizzled row)
// Ring stages of the tcgen05 kernels: as many as the shared memory left after
// the resident queries, barriers, iteration log and (buffer epilogues) radix
// histograms and compaction buffers holds, at most this many (the barrier
// arrays are sized for it).
constexpr int kTcMaxStages = 8;
constexpr int kSmemBudget = 232448 - 1024;  // dynamic shared memory per CTA, less the alignment slack
constexpr int kTcMaxResidentSlices = 7;  // queries stay in smem when d_pad <= 448
// Dry tiles of the top-k epilogues (see cvs_epilogue.cuh): at most this many
// (TileSource in cvs_sched.cuh keeps two).
constexpr int kDryTiles = 2;

enum TcEpilogue : int {
  kEpiTopkReg16 = 0,   // k <= 16: per-query sorted list in registers
  kEpiTopkReg32 = 1,   // k <= 32
  kEpiTopkBuf = 2,     // k  > 32: per-query candidate buffer in global memory
  kEpiStoreF32 = 3,    // write the score matrix as fp32
  kEpiStoreF16 = 4,    // write the score matrix as fp16
  kEpiTopkBuf8 = 5,    // k > 32 with fewer lists: candidate buffers, 8 ranks tracked in registers
};

// Rank J of the per-list value a buffer list (k > 32) publishes (its J-th best)
// and how many lists m must reach a value for it to bound the query's k-th best
// (m lists x J rows >= k rows). Aim: J = ceil(2k / lists), so m is about half
// the lists; but J is held to regj (the ranks the epilogue tracks in registers,
// which is what lets it publish from the first tile on) whenever m = ceil(k / J)
// still fits in the lists. The merge uses the same pair.
__host__ __device__ inline int tops_j(int k, int lists, int regj) {
  lists = lists < 1 ? 1 : lists;
  int j = (2 * k + lists - 1) / lists;
  const int jmin = (k + lists - 1) / lists;  // smallest J with m <= lists
  if (j > regj) j = jmin > regj ? jmin : regj;
  return j < 1 ? 1 : (j > k ? k : j);
}
__host__ __device__ inline int tops_m(int k, int lists, int regj) {
  const int j = tops_j(k, lists, regj);
  return (k + j - 1) / j;
}

// Ranks a buffer epilogue tracks in registers (kEpiTopkBuf: 4, kEpiTopkBuf8: 8;
// more ranks cost registers in the drain loop, so 8 only where 4 cannot serve).
__host__ __device__ inline int buf_reg_ranks(int epi) { return epi == kEpiTopkBuf8 ? 8 : 4; }
__host__ __device__ inline bool is_buf_epi(int epi) { return epi == kEpiTopkBuf || epi == kEpiTopkBuf8; }


struct TcArgs {
  int b;              // queries
  int n;              // corpus rows
  int d_pad;          // row width in halves (multiple of 64)
  int ksl;            // d_pad / 64
  int qtiles;         // ceil(b / 128)
  int segs;           // corpus segments (each a contiguous run of 256-row tiles)
  int tiles_per_seg;
  int ntiles;         // ceil(n / 256)
  int k;              // candidates kept per (query, segment)
  int cap;            // slots per candidate list; cap >= k
  uint64_t* part;     // [b][segs * lists per segment][cap] ordered keys
  uint32_t* gthr;     // [b] shared per-query lower bounds (ordered bits), zeroed per call
  uint32_t* tops;     // [b][segs * lists per segment] each list's published score (ordered bits), zeroed per call
  int* counts;        // [b][segs * lists per segment] keys each buffer list ends with (buffer epilogue)
  int* tile_counter;  // [qtiles] next unclaimed corpus tile per query tile, zeroed per call;
                      // null: CTA s works on the fixed tiles [s*tiles_per_seg, (s+1)*tiles_per_seg)
  int dry;            // tiles each CTA reads dry first (0 or kDryTiles)
  void* scores_out;   // [b][n] fp32/fp16 for the store epilogues
  int* err;           // device error word
  // Failure-path test hook (one-CTA kernel only; cvs_debug_stall_next_search):
  // stall != 0 makes the producer claim and load nothing, and wait_cycles > 0
  // replaces the ~1 s limit of the kernel's waits, so every wait runs out.
  long long wait_cycles;
  int stall;
};

// Candidate lists each (query, segment) produces with this epilogue (one per
// epilogue column stripe); the workspace holds b * segs * lists * cap keys.
int tc_lists_per_segment(int epi);
// Whether the query tile can stay resident in shared memory next to the stage
// ring and this epilogue's scratch (one-CTA kernel).
bool tc_resident_queries(int epi, int ksl);
cudaError_t tc_launch(int epi, bool resident_queries, const CUtensorMap* qmap,
                      const CUtensorMap* xmap, const TcArgs& a, cudaStream_t stream);

// CTA-pair variant (batches > 128): a.qtiles counts 256-query pair tiles, the
// corpus tensor map uses 128-row boxes, the grid is 2 * qtiles * segs CTAs.
bool tc_pair_resident_queries(int epi, int ksl);
int tc_pair_max_clusters(int epi, bool resident_queries, int ksl);
cudaError_t tc_pair_launch(int epi, bool resident_queries, const CUtensorMap* qmap,
                           const CUtensorMap* xmap, const TcArgs& a, cudaStream_t stream);

// ---- CUDA-core GEMV + top-k for one to eight queries -----------------------
constexpr int kGemvThreads = 256;
constexpr int kGemvMaxK = 32;
constexpr int kGemvMaxBatch = 8;  // queries per GEMV launch (small corpora only from 2 on)

struct GemvArgs {
  const __half* x;    // [n][d_pad]
  const __half* q;    // [b][d_pad]
  int b;
  int n;
  int d_pad;
  int k;
  int segs;           // grid size; segment s covers rows [s*rows_per_seg, ...)
  int rows_per_seg;
  uint64_t* part;     // [b][segs][k]
  uint32_t* bounds;   // [b] per-query lower bounds on the k-th best (ordered bits), zeroed per call
  uint32_t* tops;     // [b][segs] each CTA's best score (ordered bits)
  int* err;
};

bool gemv_supported(int b, int k, int d_pad);
cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t stream);
int gemv_blocks_per_sm(int b, int d_pad);

// ---- merge of per-segment candidate lists into the final sorted top-k ------
struct MergeKeysArgs {
  const uint64_t* part;  // [b][lists][stride], first per_list entries of each used
  const int* counts;     // [b][lists] entries used per list (then per_list is ignored) or null
  int b;
  int lists;
  int stride;
  int per_list;
  int k;
  long long id_offset;   // added to every returned row id
  const uint32_t* bounds;  // [b] lower bounds on each query's k-th best (ordered bits) or null
  const uint32_t* tops;    // [b][tops_n] per-list published scores (ordered bits, 0 = none) or null
  int tops_n;
  int tops_m;              // the tops_m-th largest published score bounds the k-th best
  float* out_v;          // [b][k]
  long long* out_i;      // [b][k]
  int* err;
};
cudaError_t merge_keys_launch(const MergeKeysArgs& a, cudaStream_t stream);

// Zeroes `bytes` bytes at p (4-byte aligned); if q_dst is given, also copies the
// b x d_pad fp16 queries q_src into q_dst and zeroes its rows b..rows_pad-1. Lets
// the next kernel, launched programmatically, start its prologue meanwhile.
cudaError_t prepare_launch(void* p, size_t bytes, const void* q_src, void* q_dst, int b, int d_pad,
                           int rows_pad, cudaStream_t stream);

// Launches `kernel` with programmatic stream serialisation: it may start while
// the previous kernel on the stream finishes and must call
// grid_dependency_wait() before touching that kernel's results.
template <class... Params, class... Args>
cudaError_t launch_programmatic(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

struct MergeListsArgs {
  const float* v;        // [lists] x [b][len] scores, lists v_stride floats apart
  const long long* ids;  // [lists] x [b][len] ids (must lie in [0, 2^31)), lists i_stride apart
  long long v_stride;
  long long i_stride;
  int b;
  int lists;
  int len;
  int k;
  float* out_v;          // [b][k]
  long long* out_i;      // [b][k]
  int* err;
};
cudaError_t merge_lists_launch(const MergeListsArgs& a, cudaStream_t stream);

// ---- ingest: dtype conversion, optional L2 normalisation, width padding ----
enum SrcDtype : int { kSrcF32 = 0, kSrcF16 = 1, kSrcBF16 = 2, kSrcF64 = 3 };
// With `clear` given, the same launch also zeroes clear_words 32-bit words there,
// and rows n .. rows_pad-1 of dst are written as zeros (a search's workspace
// preparation folded into its query ingest).
cudaError_t ingest_launch(const void* src, int src_dtype, long long n, int d, long long src_stride,
                          int d_pad, int cosine, __half* dst, int num_sms, cudaStream_t stream,
                          uint32_t* clear = nullptr, size_t clear_words = 0, long long rows_pad = 0);

}  // namespace cvs
