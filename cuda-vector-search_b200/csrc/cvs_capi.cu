// Host side of the C ABI declared in include/cvs.h: argument contracts,
// launch planning, TMA descriptors, kernel launches and status reporting.
//
// The contracts mirror the reference's check_matrix / check_pair
// (cuda_vector_search/csrc/kernels.cu:451-470) and fused_topk's k checks
// (:509-510); the planner replaces its bq / chunk heuristics (:512-536), which
// were tuned for a 40-SM T4, with one keyed on the B200's SM count: one CTA per
// SM, query tiles of 128, corpus segments of whole 256-row tiles.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <climits>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "cvs.h"
#include "cvs_kernels.h"

namespace cvs {
namespace {

__device__ int g_device_error;  // one word per device; written by kernels on a failed wait

thread_local std::string g_last_error;
thread_local int64_t g_stall_cycles = 0;  // armed failure-path test (cvs_debug_stall_next_search)

cvs_status fail(cvs_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
cvs_status fail(cvs_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

cvs_status cuda_fail(cudaError_t e, const char* what) {
  return fail(CVS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
  int* err = nullptr;  // device address of g_device_error
};

std::mutex g_mu;
std::unordered_map<int, DeviceInfo> g_devices;
cudaEvent_t g_prof_start = nullptr;
cudaEvent_t g_prof_stop = nullptr;

cvs_status device_info(DeviceInfo* out, int* dev_out = nullptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev_out) *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_devices.find(dev);
  if (it == g_devices.end()) {
    DeviceInfo d;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    if (d.major != 10 || d.minor != 0)
      return fail(CVS_ERR_UNSUPPORTED,
                  "device %d has compute capability %d.%d; this library is built for sm_100a (B200)",
                  dev, d.major, d.minor);
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_device_error)) != cudaSuccess)
      return cuda_fail(e, "cudaGetSymbolAddress(device error word)");
    d.err = static_cast<int*>(p);
    it = g_devices.emplace(dev, d).first;
  }
  *out = it->second;
  return CVS_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D fp16 tensor [rows][cols], boxes of 64 columns x box_rows rows, 128-byte swizzle.
cvs_status make_map(CUtensorMap* m, const void* base, int64_t rows, int cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(CVS_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CVS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return CVS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cvs_status check_pair(const void* q, int64_t b, const void* x, int64_t n, int d_pad) {
  if (b < 0 || b >= INT_MAX) return fail(CVS_ERR_INVALID_ARGUMENT, "query count %lld out of range", (long long)b);
  if (n < 1 || n >= INT_MAX)
    return fail(CVS_ERR_INVALID_ARGUMENT, "corpus must have 1 .. 2^31-1 rows (got %lld)", (long long)n);
  if (d_pad < CVS_PAD || d_pad % CVS_PAD != 0)
    return fail(CVS_ERR_INVALID_ARGUMENT, "width must be a positive multiple of 64 (zero-pad it); got %d", d_pad);
  if (!x || !aligned16(x)) return fail(CVS_ERR_INVALID_ARGUMENT, "corpus must be a non-null 16-byte aligned pointer");
  if (b > 0 && (!q || !aligned16(q)))
    return fail(CVS_ERR_INVALID_ARGUMENT, "queries must be a non-null 16-byte aligned pointer");
  return CVS_OK;
}

struct Plan {
  bool gemv = false;
  bool pair = false;  // CTA-pair tcgen05 kernel (batches > 128)
  int epi = 0;
  bool qres = false;
  int qtiles = 0, segs = 0, tiles_per_seg = 0, ntiles = 0;
  int cap = 0;
  int lists = 0;  // candidate lists per query (segments x lists per segment)
  size_t bound_bytes = 0;  // per-query bounds, per-list tops and counts at the start of the workspace
  size_t clear_bytes = 0;  // the part of it cleared per call
  int rows_per_seg = 0;
  int qpad_rows = 0;      // > 0: queries copied into a zero-padded workspace buffer of this many rows
  size_t qpad_offset = 0; // its offset in the workspace
  size_t ws_bytes = 0;
};

constexpr size_t kWsAlign = 256;

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Clusters of the pair kernel that can be resident at once (cached: it is a
// property of the kernel, its shared memory and the device).
int pair_clusters(int epi, bool qres, int ksl, int sms) {
  static std::mutex mu;
  static std::unordered_map<long long, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  // dev | epilogue | resident flag | K slices, each in its own field (ksl is
  // d_pad / 64, unbounded by the C ABI, so it gets the low 31 bits).
  const long long key = (static_cast<long long>(dev) << 40) | (static_cast<long long>(epi) << 32) |
                        (qres ? 1LL << 31 : 0LL) | static_cast<long long>(ksl);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = tc_pair_max_clusters(epi, qres, ksl);
  if (n <= 0) n = sms / 2;
  cache.emplace(key, n);
  return n;
}

// Corpus segmentation for the tcgen05 kernels: one CTA (or CTA pair) per SM
// (pair) in total. Batches of more than 128 queries use the pair kernel, whose
// query tiles hold 256 queries.
void plan_tc_grid(Plan* p, int64_t b, int64_t n, int sms, int chunks, int epi, int d_pad, int bq = 0) {
  const int ksl = d_pad / kTcK;
  // bq hint: 16..128 keeps 128-query tiles on one CTA, 256 asks for CTA pairs.
  // Automatic: CTA pairs for more than 128 queries unless their 256-query tiles
  // would pad more rows than 128-query tiles (b = 300: 512 against 384 rows;
  // measured 20-30% slower), since every padded row costs MMA work.
  const int64_t pair_rows = (b + 2 * kTcM - 1) / (2 * kTcM) * (2 * kTcM);
  const int64_t cta_rows = (b + kTcM - 1) / kTcM * kTcM;
  p->pair = bq > 0 ? (bq > kTcM && b > kTcM) : (b > kTcM && pair_rows == cta_rows);
  p->ntiles = static_cast<int>((n + kTcN - 1) / kTcN);
  int slots;
  if (p->pair) {
    p->qtiles = static_cast<int>((b + 2 * kTcM - 1) / (2 * kTcM));
    p->qres = tc_pair_resident_queries(epi, ksl);
    slots = pair_clusters(epi, p->qres, ksl, sms);
  } else {
    p->qtiles = static_cast<int>((b + kTcM - 1) / kTcM);
    p->qres = tc_resident_queries(epi, ksl);
    slots = sms;
  }
  int segs = chunks > 0 ? chunks : std::max(1, slots / std::max(1, p->qtiles));
  segs = std::max(1, std::min(segs, p->ntiles));
  p->tiles_per_seg = (p->ntiles + segs - 1) / segs;
  p->segs = (p->ntiles + p->tiles_per_seg - 1) / p->tiles_per_seg;
}

// The GEMV's arithmetic per corpus row grows with the batch, the tcgen05
// kernel's does not, so from two queries on the tcgen05 kernel streams a large
// corpus faster. On a small one (at most two tiles per CTA, one dry tile) the
// tcgen05 kernel costs what its dry tile and the wait for a shared bound cost:
// 17-25 us at k <= 16 with d_pad <= 640, while at k <= 32 a query whose bound
// comes late drains 32-slot register lists without one (24-135 us measured,
// varying from run to run). The GEMV costs ~13 us plus ~0.15 ns per (row x
// max(d_pad, 256) x query of its instantiation) -- narrow rows do not get
// cheaper than 256 columns, the shuffle reduction per row and query stays. So
// for 2..8 queries it is taken on such corpora when d_pad <= 640 and that
// product stays below 3e7 (k <= 16) or 1.2e8 (k <= 32). Measured, GEMV against
// tcgen05: 20000 x 384, b = 2: 0.014 / 0.019 ms; b = 8: 0.033 / 0.021 ms
// (tcgen05 taken); 20000 x 128, b = 8: 0.027 / 0.017 ms (tcgen05 taken); 75000 x
// 384, b = 4, k = 32: 0.041 / 0.135 ms. The choice follows the automatic grid
// (one CTA per SM) even when a segment count is given, so that for a given
// batch the workspace grows with the segment count along one path.
bool gemv_preferred(int64_t b, int64_t n, int d_pad, int k, int sms) {
  if (b <= 1) return true;
  const int64_t ntiles = (n + kTcN - 1) / kTcN;
  if (ntiles > static_cast<int64_t>(kDryTiles) * sms || d_pad > 640) return false;
  const int64_t nq = b <= 2 ? b : (b <= 4 ? 4 : 8);  // queries the instantiation computes
  const double work = static_cast<double>(n) * std::max(d_pad, 256) * nq;
  return work <= (k <= 16 ? 3.0e7 : 1.2e8);
}

// own_queries: the search ingests its queries itself (cvs_search), into a
// buffer of whole query tiles at the end of the workspace.
cvs_status plan_fused(int64_t b, int64_t n, int d_pad, int k, int chunks, const DeviceInfo& dev,
                      Plan* p, int bq = 0, bool own_queries = false) {
  if (k < 1 || k > CVS_MAX_FUSED_K)
    return fail(CVS_ERR_INVALID_ARGUMENT, "fused top-k supports 1 <= k <= %d (got %d)", CVS_MAX_FUSED_K, k);
  if (k > n) return fail(CVS_ERR_INVALID_ARGUMENT, "k (%d) must not exceed the corpus size (%lld)", k, (long long)n);
  if (chunks < 0) return fail(CVS_ERR_INVALID_ARGUMENT, "chunks must be >= 0");
  // bq = 0 (automatic): the CUDA-core GEMV for one query, and for up to
  // kGemvMaxBatch queries on corpora too small for the tcgen05 kernel's dry
  // tiles (gemv_preferred); an explicit bq asks for the tcgen05 tiles whatever
  // the batch.
  if (bq == 0 && gemv_supported(static_cast<int>(b), k, d_pad) && gemv_preferred(b, n, d_pad, k, dev.sms)) {
    p->gemv = true;
    int segs = chunks > 0 ? chunks : dev.sms * gemv_blocks_per_sm(static_cast<int>(b), d_pad);
    segs = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(segs, n)));
    p->rows_per_seg = static_cast<int>((n + segs - 1) / segs);
    p->segs = static_cast<int>((n + p->rows_per_seg - 1) / p->rows_per_seg);
    p->cap = k;
    p->lists = p->segs;
    p->clear_bytes = static_cast<size_t>(b) * 4 * (1 + p->lists);
    p->bound_bytes = round_up(p->clear_bytes, kWsAlign);
    p->ws_bytes = p->bound_bytes + round_up(static_cast<size_t>(b) * p->lists * p->cap * 8, kWsAlign);
    if (own_queries) {
      p->qpad_rows = static_cast<int>(b);
      p->qpad_offset = p->ws_bytes;
      p->ws_bytes += round_up(static_cast<size_t>(b) * d_pad * 2, kWsAlign);
    }
    return CVS_OK;
  }
  p->gemv = false;
  if (k <= 16) {
    p->epi = kEpiTopkReg16;
    p->cap = k;
  } else if (k <= 32) {
    p->epi = kEpiTopkReg32;
    p->cap = k;
  } else {
    p->epi = kEpiTopkBuf;
    // Room for 2k keys and at least 256 (the shared-memory compaction buffer),
    // and always a chunk (32 keys) above k. Lists start appending with a bound
    // in place (dry tiles), so they rarely compact: none at all in the C4 and
    // b = 1024, k = 100 shapes.
    p->cap = static_cast<int>(round_up(static_cast<size_t>(std::max({2 * k, k + 32, 256})), 32));
  }
  plan_tc_grid(p, b, n, dev.sms, chunks, p->epi, d_pad, bq);
  p->lists = p->segs * tc_lists_per_segment(p->epi);
  // Buffer lists track their published rank in registers: 4 ranks when that
  // rank is enough for the lists at hand, 8 when there are too few lists
  // (large batches share the SMs among more query tiles).
  if (p->epi == kEpiTopkBuf && tops_j(k, p->lists, 8) > 4 && tops_j(k, p->lists, 8) <= 8) p->epi = kEpiTopkBuf8;
  // Per-query shared bound, per-list published scores, (buffer lists) per-list
  // key counts and the per-query-tile tile counters, all cleared per call.
  const bool counted = is_buf_epi(p->epi);
  p->clear_bytes = static_cast<size_t>(b) * 4 * (1 + p->lists * (counted ? 2 : 1)) + 4 * static_cast<size_t>(p->qtiles);
  p->bound_bytes = round_up(p->clear_bytes, kWsAlign);
  p->ws_bytes = p->bound_bytes + round_up(static_cast<size_t>(b) * p->lists * p->cap * 8, kWsAlign);
  // Streamed queries are re-loaded for every corpus tile; rows of a partial query
  // tile that lie outside the query matrix would be zero-filled by the TMA unit
  // on every load, which costs up to a fifth of the kernel time at small
  // batches. Such batches are copied into a zero-padded buffer of whole tiles.
  const int tile_rows = p->pair ? 2 * kTcM : kTcM;
  if (own_queries || (!p->qres && b % tile_rows != 0)) {
    p->qpad_rows = p->qtiles * tile_rows;
    p->qpad_offset = p->ws_bytes;
    p->ws_bytes += round_up(static_cast<size_t>(p->qpad_rows) * d_pad * 2, kWsAlign);
  }
  return CVS_OK;
}

cvs_status check_outputs(const Plan& p, float* out_scores, int64_t* out_ids, void* workspace,
                         size_t workspace_bytes) {
  if (!out_scores || !out_ids) return fail(CVS_ERR_INVALID_ARGUMENT, "null output pointer");
  if (!workspace || workspace_bytes < p.ws_bytes || (reinterpret_cast<uintptr_t>(workspace) % kWsAlign) != 0)
    return fail(CVS_ERR_WORKSPACE, "workspace of %zu bytes (256-byte aligned) required, got %zu at %p",
                p.ws_bytes, workspace_bytes, workspace);
  return CVS_OK;
}

// Launches the search kernel and the merge for a planned call whose queries are
// readable at q_tiles (padded as the plan says) and whose workspace is cleared
// (by a kernel already enqueued on the stream).
cvs_status launch_search(const Plan& p, const DeviceInfo& dev, const void* q_tiles, int64_t b, const void* x_f16,
                         int64_t n, int d_pad, int k, int64_t id_offset, float* out_scores, int64_t* out_ids,
                         void* workspace, cudaStream_t s) {
  const int64_t stall_cycles = g_stall_cycles;
  g_stall_cycles = 0;  // one call only
  if (stall_cycles > 0 && (p.gemv || p.pair))
    return fail(CVS_ERR_INVALID_ARGUMENT, "the stall test hook needs a one-CTA tcgen05 plan (up to 128 queries, not a GEMV plan)");
  uint32_t* bounds = static_cast<uint32_t*>(workspace);
  uint64_t* part = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + p.bound_bytes);
  const bool prof = g_prof_start && g_prof_stop;
  cvs_status st;
  cudaError_t e;
  if (prof && (e = cudaEventRecord(g_prof_start, s)) != cudaSuccess) return cuda_fail(e, "profile event");
  if (p.gemv) {
    GemvArgs a{};
    a.x = static_cast<const __half*>(x_f16);
    a.q = static_cast<const __half*>(q_tiles);
    a.b = static_cast<int>(b);
    a.n = static_cast<int>(n);
    a.d_pad = d_pad;
    a.k = k;
    a.segs = p.segs;
    a.rows_per_seg = p.rows_per_seg;
    a.part = part;
    a.bounds = bounds;
    a.tops = bounds + b;
    a.err = dev.err;
    if ((e = gemv_launch(a, s)) != cudaSuccess) return cuda_fail(e, "gemv top-k launch");
  } else {
    CUtensorMap qmap, xmap;
    if ((st = make_map(&qmap, q_tiles, p.qpad_rows > 0 ? p.qpad_rows : b, d_pad, kTcM)) != CVS_OK) return st;
    if ((st = make_map(&xmap, x_f16, n, d_pad, p.pair ? kTcN / 2 : kTcN)) != CVS_OK) return st;
    TcArgs a{};
    a.b = static_cast<int>(b);
    a.n = static_cast<int>(n);
    a.d_pad = d_pad;
    a.ksl = d_pad / kTcK;
    a.qtiles = p.qtiles;
    a.segs = p.segs;
    a.tiles_per_seg = p.tiles_per_seg;
    a.ntiles = p.ntiles;
    a.k = k;
    a.cap = p.cap;
    a.part = part;
    a.gthr = bounds;
    a.tops = bounds + b;
    const size_t list_words = static_cast<size_t>(b) * p.lists * (is_buf_epi(p.epi) ? 2 : 1);
    a.counts = is_buf_epi(p.epi) ? reinterpret_cast<int*>(bounds + b + static_cast<size_t>(b) * p.lists) : nullptr;
    // Tiles are claimed at run time; a.segs CTAs (pairs) per query tile share them.
    a.tile_counter = reinterpret_cast<int*>(bounds + b + list_words);
    // Two dry tiles whenever a CTA can expect three or more tiles, one below:
    // the empty-list cost of a first real tile without a bound outweighs whole
    // extra tiles (measured with L2 flushed before each call: 100k x 384, b=32
    // takes 0.054 ms with two, 0.080 with one, 0.088 with none), and the second
    // dry tile gives the other CTAs' bound refresh a tile's time to land. Even
    // a CTA with a single tile reads it dry first: the bound that the other
    // CTAs' dry reads produce reaches its real pass within a chunk or two
    // (20000 x 384, b = 16, k = 32: 0.160 -> 0.061 ms; b = 32, k = 10: 0.058 ->
    // 0.041 ms; the tile is re-read from L2).
    a.dry = p.tiles_per_seg >= 3 ? kDryTiles : 1;
    a.err = dev.err;
    if (stall_cycles > 0) {
      a.stall = 1;
      a.wait_cycles = stall_cycles;
    }
    e = p.pair ? tc_pair_launch(p.epi, p.qres, &qmap, &xmap, a, s) : tc_launch(p.epi, p.qres, &qmap, &xmap, a, s);
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 search launch");
  }
  if (prof && (e = cudaEventRecord(g_prof_stop, s)) != cudaSuccess) return cuda_fail(e, "profile event");
  MergeKeysArgs m{};
  m.part = part;
  m.b = static_cast<int>(b);
  m.lists = p.lists;
  m.stride = p.cap;
  m.per_list = k;
  // Buffer lists end with up to cap keys each; their counts follow the tops.
  m.counts = (!p.gemv && is_buf_epi(p.epi))
                 ? reinterpret_cast<const int*>(bounds + b + static_cast<size_t>(b) * p.lists)
                 : nullptr;
  m.k = k;
  m.id_offset = id_offset;
  m.bounds = bounds;
  m.tops = bounds + b;
  m.tops_n = p.lists;
  // Register lists and GEMV CTAs publish their best score (m = k lists needed);
  // buffer lists publish their J-th best (m = tops_m lists needed).
  m.tops_m = (!p.gemv && is_buf_epi(p.epi)) ? tops_m(k, p.lists, buf_reg_ranks(p.epi)) : k;
  m.out_v = out_scores;
  m.out_i = reinterpret_cast<long long*>(out_ids);
  m.err = dev.err;
  if ((e = merge_keys_launch(m, s)) != cudaSuccess) return cuda_fail(e, "merge launch");
  return CVS_OK;
}


}  // namespace
}  // namespace cvs

using namespace cvs;

extern "C" {

const char* cvs_last_error(void) { return g_last_error.c_str(); }

int cvs_abi_version(void) { return CVS_ABI_VERSION; }

int cvs_pad_width(int d) { return d <= 0 ? 0 : (d + CVS_PAD - 1) / CVS_PAD * CVS_PAD; }

cvs_status cvs_ingest(const void* src, int src_dtype, int64_t n, int d, int64_t src_row_stride,
                      int d_pad, int cosine, void* dst_f16, void* stream) {
  if (n < 0) return fail(CVS_ERR_INVALID_ARGUMENT, "row count must be >= 0");
  if (n == 0) return CVS_OK;
  if (!src || !dst_f16) return fail(CVS_ERR_INVALID_ARGUMENT, "null source or destination");
  if (d < 1 || d > 2048) return fail(CVS_ERR_INVALID_ARGUMENT, "width must be in 1 .. 2048 (got %d)", d);
  if (d_pad < d || d_pad % CVS_PAD != 0)
    return fail(CVS_ERR_INVALID_ARGUMENT, "d_pad (%d) must be a multiple of 64 and >= d (%d)", d_pad, d);
  if (src_row_stride < d) return fail(CVS_ERR_INVALID_ARGUMENT, "source row stride smaller than the width");
  if (src_dtype < CVS_F32 || src_dtype > CVS_F64) return fail(CVS_ERR_INVALID_ARGUMENT, "unknown source dtype %d", src_dtype);
  if (src == dst_f16 && !(src_dtype == CVS_F16 && d == d_pad && src_row_stride == d_pad))
    return fail(CVS_ERR_INVALID_ARGUMENT, "in-place ingest needs fp16 input with d == d_pad == stride");
  DeviceInfo dev;
  cvs_status st = device_info(&dev);
  if (st != CVS_OK) return st;
  cudaError_t e = ingest_launch(src, src_dtype, n, d, src_row_stride, d_pad, cosine,
                                static_cast<__half*>(dst_f16), dev.sms, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "ingest launch");
  return CVS_OK;
}

cvs_status cvs_fused_topk_workspace_size(int64_t b, int64_t n, int d_pad, int k, int plan_bq,
                                         int plan_chunks, size_t* bytes) {
  (void)plan_bq;
  if (!bytes) return fail(CVS_ERR_INVALID_ARGUMENT, "bytes must not be null");
  *bytes = 0;
  if (b < 0 || b >= INT_MAX) return fail(CVS_ERR_INVALID_ARGUMENT, "query count out of range");
  if (n < 1 || n >= INT_MAX) return fail(CVS_ERR_INVALID_ARGUMENT, "corpus must have 1 .. 2^31-1 rows");
  if (d_pad < CVS_PAD || d_pad % CVS_PAD != 0) return fail(CVS_ERR_INVALID_ARGUMENT, "width must be a multiple of 64");
  if (b == 0) return CVS_OK;
  DeviceInfo dev;
  cvs_status st = device_info(&dev);
  if (st != CVS_OK) return st;
  Plan p;
  st = plan_fused(b, n, d_pad, k, plan_chunks, dev, &p, plan_bq);
  if (st != CVS_OK) return st;
  *bytes = p.ws_bytes;
  return CVS_OK;
}

cvs_status cvs_fused_topk(const void* q_f16, int64_t b, const void* x_f16, int64_t n, int d_pad,
                          int k, int64_t id_offset, float* out_scores, int64_t* out_ids,
                          void* workspace, size_t workspace_bytes, int plan_bq, int plan_chunks,
                          int64_t* plan_out, void* stream) {
  cvs_status st = check_pair(q_f16, b, x_f16, n, d_pad);
  if (st != CVS_OK) return st;
  DeviceInfo dev;
  if ((st = device_info(&dev)) != CVS_OK) return st;
  Plan p;
  if ((st = plan_fused(b, n, d_pad, k, plan_chunks, dev, &p, plan_bq)) != CVS_OK) return st;
  if (plan_out) {
    plan_out[0] = plan_bq > 0 ? plan_bq : (p.gemv ? static_cast<int64_t>(b) : static_cast<int64_t>(p.pair ? 2 * kTcM : kTcM));
    plan_out[1] = p.segs;
  }
  if (b == 0) return CVS_OK;
  if ((st = check_outputs(p, out_scores, out_ids, workspace, workspace_bytes)) != CVS_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* bounds = static_cast<uint32_t*>(workspace);
  cudaError_t e;
  // The shared per-query bounds must start at "none" (0) on every call.
  const void* q_tiles = q_f16;  // what the tensor map reads
  if (p.qpad_rows > 0) {
    void* qpad = static_cast<char*>(workspace) + p.qpad_offset;
    if ((e = prepare_launch(bounds, round_up(p.clear_bytes, 4), q_f16, qpad, static_cast<int>(b), d_pad,
                            p.qpad_rows, s)) != cudaSuccess)
      return cuda_fail(e, "clearing the workspace and padding the queries");
    q_tiles = qpad;
  } else if (p.clear_bytes && (e = prepare_launch(bounds, round_up(p.clear_bytes, 4), nullptr, nullptr, 0,
                                                   d_pad, 0, s)) != cudaSuccess)
    return cuda_fail(e, "clearing the per-query bounds");
  return launch_search(p, dev, q_tiles, b, x_f16, n, d_pad, k, id_offset, out_scores, out_ids, workspace, s);
}

cvs_status cvs_search_workspace_size(int64_t b, int64_t n, int d_pad, int k, size_t* bytes) {
  if (!bytes) return fail(CVS_ERR_INVALID_ARGUMENT, "bytes must not be null");
  *bytes = 0;
  if (b < 0 || b >= INT_MAX) return fail(CVS_ERR_INVALID_ARGUMENT, "query count out of range");
  if (n < 1 || n >= INT_MAX) return fail(CVS_ERR_INVALID_ARGUMENT, "corpus must have 1 .. 2^31-1 rows");
  if (d_pad < CVS_PAD || d_pad % CVS_PAD != 0) return fail(CVS_ERR_INVALID_ARGUMENT, "width must be a multiple of 64");
  if (b == 0) return CVS_OK;
  DeviceInfo dev;
  cvs_status st = device_info(&dev);
  if (st != CVS_OK) return st;
  Plan p;
  if ((st = plan_fused(b, n, d_pad, k, 0, dev, &p, 0, true)) != CVS_OK) return st;
  *bytes = p.ws_bytes;
  return CVS_OK;
}

cvs_status cvs_search(const void* q_src, int src_dtype, int64_t b, int d, int64_t src_row_stride, int cosine,
                      const void* x_f16, int64_t n, int d_pad, int k, int64_t id_offset, float* out_scores,
                      int64_t* out_ids, void* workspace, size_t workspace_bytes, void* stream) {
  if (b < 0 || b >= INT_MAX) return fail(CVS_ERR_INVALID_ARGUMENT, "query count %lld out of range", (long long)b);
  if (b == 0) return CVS_OK;
  if (!q_src) return fail(CVS_ERR_INVALID_ARGUMENT, "queries must not be null");
  if (d < 1 || d > 2048) return fail(CVS_ERR_INVALID_ARGUMENT, "query width must be in 1 .. 2048 (got %d)", d);
  if (d > d_pad) return fail(CVS_ERR_INVALID_ARGUMENT, "query width %d exceeds the corpus width %d", d, d_pad);
  if (src_row_stride < d) return fail(CVS_ERR_INVALID_ARGUMENT, "query row stride smaller than the width");
  if (src_dtype < CVS_F32 || src_dtype > CVS_F64) return fail(CVS_ERR_INVALID_ARGUMENT, "unknown query dtype %d", src_dtype);
  // Queries are read by the ingest, not by TMA: only the corpus needs the
  // alignment check (a stand-in 16-byte aligned query pointer passes it).
  cvs_status st = check_pair(x_f16, b, x_f16, n, d_pad);
  if (st != CVS_OK) return st;
  DeviceInfo dev;
  if ((st = device_info(&dev)) != CVS_OK) return st;
  Plan p;
  if ((st = plan_fused(b, n, d_pad, k, 0, dev, &p, 0, true)) != CVS_OK) return st;
  if ((st = check_outputs(p, out_scores, out_ids, workspace, workspace_bytes)) != CVS_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // One launch converts, normalises and pads the queries into whole query
  // tiles in the workspace and clears the bounds; the search kernel follows.
  __half* qbuf = reinterpret_cast<__half*>(static_cast<char*>(workspace) + p.qpad_offset);
  cudaError_t e = ingest_launch(q_src, src_dtype, b, d, src_row_stride, d_pad, cosine, qbuf, dev.sms, s,
                                static_cast<uint32_t*>(workspace), round_up(p.clear_bytes, 4) / 4, p.qpad_rows);
  if (e != cudaSuccess) return cuda_fail(e, "query ingest and workspace clear");
  return launch_search(p, dev, qbuf, b, x_f16, n, d_pad, k, id_offset, out_scores, out_ids, workspace, s);
}

cvs_status cvs_scores(const void* q_f16, int64_t b, const void* x_f16, int64_t n, int d_pad,
                      void* out, int out_fp32, void* stream) {
  cvs_status st = check_pair(q_f16, b, x_f16, n, d_pad);
  if (st != CVS_OK) return st;
  if (b == 0) return CVS_OK;
  if (!out) return fail(CVS_ERR_INVALID_ARGUMENT, "null output pointer");
  DeviceInfo dev;
  if ((st = device_info(&dev)) != CVS_OK) return st;
  Plan p;
  const int epi = out_fp32 ? kEpiStoreF32 : kEpiStoreF16;
  plan_tc_grid(&p, b, n, dev.sms, 0, epi, d_pad);
  CUtensorMap qmap, xmap;
  if ((st = make_map(&qmap, q_f16, b, d_pad, kTcM)) != CVS_OK) return st;
  if ((st = make_map(&xmap, x_f16, n, d_pad, p.pair ? kTcN / 2 : kTcN)) != CVS_OK) return st;
  TcArgs a{};
  a.b = static_cast<int>(b);
  a.n = static_cast<int>(n);
  a.d_pad = d_pad;
  a.ksl = d_pad / kTcK;
  a.qtiles = p.qtiles;
  a.segs = p.segs;
  a.tiles_per_seg = p.tiles_per_seg;
  a.ntiles = p.ntiles;
  a.k = 1;
  a.cap = 1;
  a.scores_out = out;
  a.err = dev.err;
  cudaError_t e = p.pair ? tc_pair_launch(epi, p.qres, &qmap, &xmap, a, static_cast<cudaStream_t>(stream))
                         : tc_launch(epi, p.qres, &qmap, &xmap, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 score launch");
  return CVS_OK;
}

cvs_status cvs_merge_lists_strided(const float* scores, int64_t scores_list_stride, const int64_t* ids,
                                   int64_t ids_list_stride, int64_t lists, int64_t b, int64_t len, int k,
                                   float* out_scores, int64_t* out_ids, void* stream) {
  if (lists < 1 || b < 0 || len < 1 || lists * len >= INT_MAX)
    return fail(CVS_ERR_INVALID_ARGUMENT, "bad list shape [%lld][%lld][%lld]", (long long)lists,
                (long long)b, (long long)len);
  if (scores_list_stride < b * len || ids_list_stride < b * len)
    return fail(CVS_ERR_INVALID_ARGUMENT, "list strides (%lld, %lld) below b * len (%lld)",
                (long long)scores_list_stride, (long long)ids_list_stride, (long long)(b * len));
  if (k < 1 || k > CVS_MAX_FUSED_K) return fail(CVS_ERR_INVALID_ARGUMENT, "k out of range (%d)", k);
  if (b == 0) return CVS_OK;
  if (!scores || !ids || !out_scores || !out_ids) return fail(CVS_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo dev;
  cvs_status st = device_info(&dev);
  if (st != CVS_OK) return st;
  MergeListsArgs a{};
  a.v = scores;
  a.ids = reinterpret_cast<const long long*>(ids);
  a.v_stride = scores_list_stride;
  a.i_stride = ids_list_stride;
  a.b = static_cast<int>(b);
  a.lists = static_cast<int>(lists);
  a.len = static_cast<int>(len);
  a.k = k;
  a.out_v = out_scores;
  a.out_i = reinterpret_cast<long long*>(out_ids);
  a.err = dev.err;
  cudaError_t e = merge_lists_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return CVS_OK;
}

cvs_status cvs_merge_lists(const float* scores, const int64_t* ids, int64_t lists, int64_t b,
                           int64_t len, int k, float* out_scores, int64_t* out_ids, void* stream) {
  return cvs_merge_lists_strided(scores, b * len, ids, b * len, lists, b, len, k, out_scores, out_ids, stream);
}

cvs_status cvs_poll_device_error(int device, int* code) {
  if (!code) return fail(CVS_ERR_INVALID_ARGUMENT, "code must not be null");
  *code = 0;
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  DeviceInfo dev;
  cvs_status st = device_info(&dev);
  if (st == CVS_OK) {
    int zero = 0;
    if ((e = cudaMemcpy(code, dev.err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(dev.err, &zero, sizeof(int), cudaMemcpyHostToDevice)) != cudaSuccess)
      st = cuda_fail(e, "reading the device error word");
  }
  cudaSetDevice(prev);
  if (st != CVS_OK) return st;
  if (*code != 0)
    return fail(CVS_ERR_DEVICE_TIMEOUT, "a kernel gave up waiting on its pipeline (code 0x%x)", *code);
  return CVS_OK;
}

cvs_status cvs_debug_stall_next_search(int64_t wait_cycles) {
  if (wait_cycles < 1000 || wait_cycles > (int64_t{1} << 40))
    return fail(CVS_ERR_INVALID_ARGUMENT, "wait_cycles must be in 1000 .. 2^40 (got %lld)", (long long)wait_cycles);
  g_stall_cycles = wait_cycles;
  return CVS_OK;
}

cvs_status cvs_set_profile_events(void* start_event, void* stop_event) {
  g_prof_start = static_cast<cudaEvent_t>(start_event);
  g_prof_stop = static_cast<cudaEvent_t>(stop_event);
  return CVS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free search entry point.
//
// Some callers cannot hand this library a device workspace: a host program that
// owns the whole device-memory budget through its own pool and does not let
// plugins call cudaMalloc, a latency-critical serving loop where cudaMalloc's
// implicit synchronisation is not acceptable, or a foreign-language binding
// (Go, Java, ...) with no device allocator of its own. cvs_fused_topk_noalloc
// serves them: it runs the same search kernels as cvs_fused_topk, but their
// per-segment candidate lists live in the fixed array below instead of a
// caller-provided workspace.
//
// The array is a static __device__ object, so every GPU that loads this library
// keeps kNoAllocScratchBytes reserved for it until the process exits. Host code
// cannot use the array's name as a device address; the address is looked up once
// per device with cudaGetSymbolAddress, on the first call made on that device.
// That first call therefore does a little set-up work and should be made before
// any stream capture begins.
//
// All calls on a device share the one array. The only part that has to start at
// zero, the per-query bound words at its front, is cleared by every call before
// its kernels run; every candidate slot the merge reads is written first. Two
// calls whose kernels overlap on the GPU -- different streams, or different
// host threads -- race on the array; serialise them on one stream.
// ---------------------------------------------------------------------------
namespace cvs {
namespace {

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(16) << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
std::unordered_map<int, void*> g_noalloc_addr;

// Device address of g_noalloc_scratch on the current device (looked up once).
cvs_status noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  auto it = g_noalloc_addr.find(dev);
  if (it == g_noalloc_addr.end()) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    it = g_noalloc_addr.emplace(dev, p).first;
  }
  *out = it->second;
  return CVS_OK;
}

}  // namespace
}  // namespace cvs

extern "C" cvs_status cvs_fused_topk_noalloc(const void* q_f16, int64_t b, const void* x_f16,
                                             int64_t n, int d_pad, int k, int64_t id_offset,
                                             float* out_scores, int64_t* out_ids, int plan_chunks,
                                             void* stream) {
  cvs_status st = check_pair(q_f16, b, x_f16, n, d_pad);
  if (st != CVS_OK) return st;
  if (b == 0) return CVS_OK;
  DeviceInfo dev;
  if ((st = device_info(&dev)) != CVS_OK) return st;
  Plan p;
  if ((st = plan_fused(b, n, d_pad, k, plan_chunks, dev, &p)) != CVS_OK) return st;
  if (p.ws_bytes > kNoAllocScratchBytes && plan_chunks == 0) {
    // Automatic plan too large: the most corpus segments whose candidate lists
    // fit. The binary search assumes the workspace size never shrinks as the
    // segment count grows: it is b * lists * cap * 8 bytes plus fixed parts,
    // lists = segments x a per-epilogue constant, and cap depends on k alone.
    // A planner change that let the epilogue (its list count or cap) depend on
    // the segment count would break that; the check after the search catches
    // it and falls back to scanning down one segment count at a time.
    int lo = 1, hi = p.segs - 1, best = 0;
    while (lo <= hi) {
      const int mid = (lo + hi) / 2;
      Plan t;
      if ((st = plan_fused(b, n, d_pad, k, mid, dev, &t)) != CVS_OK) return st;
      if (t.ws_bytes <= kNoAllocScratchBytes) {
        best = mid;
        lo = mid + 1;
      } else {
        hi = mid - 1;
      }
    }
    if (best > 0 && best + 1 < p.segs) {
      Plan t;
      if ((st = plan_fused(b, n, d_pad, k, best + 1, dev, &t)) != CVS_OK) return st;
      if (t.ws_bytes <= kNoAllocScratchBytes) {  // not monotonic after all: scan down instead
        for (best = p.segs - 1; best > 0; --best) {
          if ((st = plan_fused(b, n, d_pad, k, best, dev, &t)) != CVS_OK) return st;
          if (t.ws_bytes <= kNoAllocScratchBytes) break;
        }
      }
    }
    if (best > 0) {
      plan_chunks = best;
      if ((st = plan_fused(b, n, d_pad, k, plan_chunks, dev, &p)) != CVS_OK) return st;
    }
  }
  if (p.ws_bytes > kNoAllocScratchBytes)
    return fail(CVS_ERR_WORKSPACE,
                "this search needs %zu bytes of scratch but the built-in scratch holds %zu "
                "(b * segments * list slots * 8 bytes); use fewer queries per call, a smaller k "
                "or fewer chunks, or call cvs_fused_topk with a workspace",
                p.ws_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch)) != CVS_OK) return st;
  return cvs_fused_topk(q_f16, b, x_f16, n, d_pad, k, id_offset, out_scores, out_ids, scratch,
                        kNoAllocScratchBytes, 0, plan_chunks, nullptr, stream);
}
