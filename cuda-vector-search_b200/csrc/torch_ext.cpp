// Thin PyTorch binding over the C ABI (include/cvs.h). It re-exports the
// reference's extension module functions with the same names and arguments:
//   scores(q, x, out_fp32=True)                 cuda_vector_search/csrc/kernels.cu:472-497,588
//   fused_topk(q, x, k, bq=0, chunks=0)         cuda_vector_search/csrc/kernels.cu:501-582,590
// plus the ingest / merge / diagnostics entry points this build adds. Contract
// violations raise RuntimeError through TORCH_CHECK, as the reference's
// check_matrix / check_pair do (kernels.cu:451-470). Everything runs on the
// current CUDA stream of the input's device, with no host synchronisation.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdint>
#include <vector>

#include "cvs.h"

namespace {

void check(cvs_status s, const char* what) {
  TORCH_CHECK(s == CVS_OK, what, ": ", cvs_last_error());
}

void check_matrix(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kHalf, name, " must be float16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.size(1) % CVS_PAD == 0, name, " width must be a multiple of 64 (zero-pad it)");
  TORCH_CHECK(reinterpret_cast<std::uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
}

void check_pair(const torch::Tensor& q, const torch::Tensor& x) {
  check_matrix(q, "queries");
  check_matrix(x, "corpus");
  TORCH_CHECK(q.device() == x.device(), "queries and corpus must be on the same device");
  TORCH_CHECK(q.size(1) == x.size(1), "queries and corpus must have the same width");
  TORCH_CHECK(x.size(0) < INT32_MAX, "corpus must have fewer than 2^31 rows");
  TORCH_CHECK(q.size(0) < INT32_MAX, "too many queries");
}

void* stream_of(const torch::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

torch::Tensor scores(torch::Tensor q, torch::Tensor x, bool out_fp32) {
  check_pair(q, x);
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty({q.size(0), x.size(0)},
                          q.options().dtype(out_fp32 ? torch::kFloat : torch::kHalf));
  if (q.size(0) == 0) return out;
  check(cvs_scores(q.data_ptr(), q.size(0), x.data_ptr(), x.size(0), static_cast<int>(x.size(1)),
                   out.data_ptr(), out_fp32 ? 1 : 0, stream_of(q)),
        "scores");
  return out;
}

// Returns [scores f32 [b,k], ids i64 [b,k], plan i64 [2] = {bq, chunks}] (CPU plan
// tensor as in the reference). Ids are int64 here (the reference returns int32 and
// Index.search widens them).
std::vector<torch::Tensor> fused_topk(torch::Tensor q, torch::Tensor x, int64_t k, int64_t bq,
                                      int64_t chunks) {
  check_pair(q, x);
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(k >= 1 && k <= CVS_MAX_FUSED_K, "fused_topk supports 1 <= k <= ", CVS_MAX_FUSED_K);
  TORCH_CHECK(k <= x.size(0), "k must not exceed the corpus size");
  TORCH_CHECK(bq == 0 || bq == 16 || bq == 32 || bq == 64 || bq == 128 || bq == 256,
              "bq must be 0 (auto), 16, 32, 64, 128 or 256");
  TORCH_CHECK(chunks >= 0 && chunks <= INT32_MAX, "chunks must be >= 0");
  const int64_t b = q.size(0), n = x.size(0);
  const int d_pad = static_cast<int>(x.size(1));
  auto out_v = torch::empty({b, k}, q.options().dtype(torch::kFloat));
  auto out_i = torch::empty({b, k}, q.options().dtype(torch::kLong));
  size_t ws_bytes = 0;
  check(cvs_fused_topk_workspace_size(b, n, d_pad, static_cast<int>(k), static_cast<int>(bq),
                                      static_cast<int>(chunks), &ws_bytes),
        "fused_topk");
  auto ws = torch::empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 256))},
                         q.options().dtype(torch::kUInt8));
  int64_t plan[2] = {0, 0};
  check(cvs_fused_topk(q.data_ptr(), b, x.data_ptr(), n, d_pad, static_cast<int>(k), 0,
                       out_v.data_ptr<float>(), out_i.data_ptr<int64_t>(), ws.data_ptr(),
                       static_cast<size_t>(ws.numel()), static_cast<int>(bq),
                       static_cast<int>(chunks), plan, stream_of(q)),
        "fused_topk");
  auto plan_t = torch::tensor({plan[0], plan[1]}, torch::kLong);
  return {out_v, out_i, plan_t};
}

// Fused top-k with caller-provided outputs/workspace and a global id offset
// (row-sharded corpora). Returns the plan.
std::vector<int64_t> fused_topk_into(torch::Tensor q, torch::Tensor x, int64_t k,
                                     int64_t id_offset, torch::Tensor out_v, torch::Tensor out_i,
                                     torch::Tensor ws, int64_t chunks) {
  check_pair(q, x);
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(out_v.is_cuda() && out_v.scalar_type() == torch::kFloat && out_v.is_contiguous() &&
                  out_v.numel() == q.size(0) * k,
              "out_v must be a contiguous float32 CUDA tensor of b*k elements");
  TORCH_CHECK(out_i.is_cuda() && out_i.scalar_type() == torch::kLong && out_i.is_contiguous() &&
                  out_i.numel() == q.size(0) * k,
              "out_i must be a contiguous int64 CUDA tensor of b*k elements");
  TORCH_CHECK(ws.is_cuda() && ws.is_contiguous(), "workspace must be a contiguous CUDA tensor");
  int64_t plan[2] = {0, 0};
  check(cvs_fused_topk(q.data_ptr(), q.size(0), x.data_ptr(), x.size(0),
                       static_cast<int>(x.size(1)), static_cast<int>(k), id_offset,
                       out_v.data_ptr<float>(), out_i.data_ptr<int64_t>(), ws.data_ptr(),
                       static_cast<size_t>(ws.numel() * ws.element_size()), 0,
                       static_cast<int>(chunks), plan, stream_of(q)),
        "fused_topk");
  return {plan[0], plan[1]};
}

void check_raw_queries(const torch::Tensor& q, const torch::Tensor& x) {
  TORCH_CHECK(q.is_cuda(), "queries must be a CUDA tensor");
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1, "queries must be 2-D with contiguous rows");
  TORCH_CHECK(q.device() == x.device(), "queries and corpus must be on the same device");
  TORCH_CHECK(q.size(1) <= x.size(1), "queries are wider than the corpus");
}

int src_code(const torch::Tensor& t);

// Search from raw queries (any supported float dtype, not yet normalised or
// padded): [scores f32 [b,k], ids i64 [b,k]].
std::vector<torch::Tensor> search(torch::Tensor q, torch::Tensor x, int64_t k, bool cosine) {
  check_matrix(x, "corpus");
  check_raw_queries(q, x);
  TORCH_CHECK(k >= 1 && k <= CVS_MAX_FUSED_K, "search supports 1 <= k <= ", CVS_MAX_FUSED_K);
  TORCH_CHECK(k <= x.size(0), "k must not exceed the corpus size");
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t b = q.size(0), n = x.size(0);
  const int d_pad = static_cast<int>(x.size(1));
  auto out_v = torch::empty({b, k}, x.options().dtype(torch::kFloat));
  auto out_i = torch::empty({b, k}, x.options().dtype(torch::kLong));
  if (b == 0) return {out_v, out_i};
  size_t ws_bytes = 0;
  check(cvs_search_workspace_size(b, n, d_pad, static_cast<int>(k), &ws_bytes), "search");
  auto ws = torch::empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 256))}, x.options().dtype(torch::kUInt8));
  check(cvs_search(q.data_ptr(), src_code(q), b, static_cast<int>(q.size(1)), q.stride(0), cosine ? 1 : 0,
                   x.data_ptr(), n, d_pad, static_cast<int>(k), 0, out_v.data_ptr<float>(), out_i.data_ptr<int64_t>(),
                   ws.data_ptr(), static_cast<size_t>(ws.numel()), stream_of(x)),
        "search");
  return {out_v, out_i};
}

// The same into caller-provided outputs and workspace, with a global id offset
// (row-sharded corpora).
void search_into(torch::Tensor q, torch::Tensor x, int64_t k, bool cosine, int64_t id_offset, torch::Tensor out_v,
                 torch::Tensor out_i, torch::Tensor ws) {
  check_matrix(x, "corpus");
  check_raw_queries(q, x);
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(out_v.is_cuda() && out_v.scalar_type() == torch::kFloat && out_v.is_contiguous() &&
                  out_v.numel() == q.size(0) * k,
              "out_v must be a contiguous float32 CUDA tensor of b*k elements");
  TORCH_CHECK(out_i.is_cuda() && out_i.scalar_type() == torch::kLong && out_i.is_contiguous() &&
                  out_i.numel() == q.size(0) * k,
              "out_i must be a contiguous int64 CUDA tensor of b*k elements");
  TORCH_CHECK(ws.is_cuda() && ws.is_contiguous(), "workspace must be a contiguous CUDA tensor");
  check(cvs_search(q.data_ptr(), src_code(q), q.size(0), static_cast<int>(q.size(1)), q.stride(0), cosine ? 1 : 0,
                   x.data_ptr(), x.size(0), static_cast<int>(x.size(1)), static_cast<int>(k), id_offset,
                   out_v.data_ptr<float>(), out_i.data_ptr<int64_t>(), ws.data_ptr(),
                   static_cast<size_t>(ws.numel() * ws.element_size()), stream_of(x)),
        "search");
}

int64_t search_workspace_size(int64_t b, int64_t n, int64_t d_pad, int64_t k) {
  size_t bytes = 0;
  check(cvs_search_workspace_size(b, n, static_cast<int>(d_pad), static_cast<int>(k), &bytes), "search_workspace_size");
  return static_cast<int64_t>(bytes);
}

int64_t workspace_size(int64_t b, int64_t n, int64_t d_pad, int64_t k, int64_t chunks) {
  size_t bytes = 0;
  check(cvs_fused_topk_workspace_size(b, n, static_cast<int>(d_pad), static_cast<int>(k), 0,
                                      static_cast<int>(chunks), &bytes),
        "workspace_size");
  return static_cast<int64_t>(bytes);
}

int src_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat: return CVS_F32;
    case torch::kHalf: return CVS_F16;
    case torch::kBFloat16: return CVS_BF16;
    case torch::kDouble: return CVS_F64;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type(), " (float32/16, bfloat16, float64)");
  }
  return -1;
}

// dst[:, :] = pad(normalise?(fp16(src))). src: 2-D CUDA tensor (any supported
// float dtype, rows contiguous); dst: [n, d_pad] fp16 CUDA tensor (may alias src).
void ingest_into(torch::Tensor src, torch::Tensor dst, bool cosine) {
  TORCH_CHECK(src.is_cuda() && dst.is_cuda(), "ingest expects CUDA tensors");
  TORCH_CHECK(src.device() == dst.device(), "source and destination must be on the same device");
  TORCH_CHECK(src.dim() == 2 && dst.dim() == 2, "ingest expects 2-D tensors");
  TORCH_CHECK(src.stride(1) == 1, "source rows must be contiguous");
  TORCH_CHECK(dst.scalar_type() == torch::kHalf && dst.is_contiguous(), "destination must be contiguous fp16");
  TORCH_CHECK(dst.size(0) == src.size(0), "row count mismatch");
  const c10::cuda::CUDAGuard guard(src.device());
  check(cvs_ingest(src.data_ptr(), src_code(src), src.size(0), static_cast<int>(src.size(1)),
                   src.stride(0), static_cast<int>(dst.size(1)), cosine ? 1 : 0, dst.data_ptr(),
                   stream_of(src)),
        "ingest");
}

std::vector<torch::Tensor> merge_lists(torch::Tensor v, torch::Tensor i, int64_t k) {
  TORCH_CHECK(v.is_cuda() && i.is_cuda(), "merge_lists expects CUDA tensors");
  TORCH_CHECK(v.dim() == 3 && i.sizes() == v.sizes(), "expects [lists, b, len] scores and ids");
  TORCH_CHECK(v.scalar_type() == torch::kFloat && i.scalar_type() == torch::kLong,
              "scores must be float32 and ids int64");
  // Each [b, len] list must be dense; the lists themselves may be any stride
  // apart (e.g. views into one gathered buffer per rank).
  TORCH_CHECK(v.stride(2) == 1 && v.stride(1) == v.size(2) && i.stride(2) == 1 && i.stride(1) == i.size(2),
              "each [b, len] list must be contiguous");
  const c10::cuda::CUDAGuard guard(v.device());
  const int64_t b = v.size(1);
  auto out_v = torch::empty({b, k}, v.options());
  auto out_i = torch::empty({b, k}, i.options());
  check(cvs_merge_lists_strided(v.data_ptr<float>(), v.size(0) > 1 ? v.stride(0) : b * v.size(2),
                                i.data_ptr<int64_t>(), i.size(0) > 1 ? i.stride(0) : b * i.size(2), v.size(0),
                                b, v.size(2), static_cast<int>(k), out_v.data_ptr<float>(),
                                out_i.data_ptr<int64_t>(), stream_of(v)),
        "merge_lists");
  return {out_v, out_i};
}

int64_t poll_device_error(int64_t device) {
  int code = 0;
  const cvs_status s = cvs_poll_device_error(static_cast<int>(device), &code);
  TORCH_CHECK(s == CVS_OK || s == CVS_ERR_DEVICE_TIMEOUT, "poll_device_error: ", cvs_last_error());
  return code;
}

void set_profile_events(int64_t start, int64_t stop) {
  check(cvs_set_profile_events(reinterpret_cast<void*>(start), reinterpret_cast<void*>(stop)),
        "set_profile_events");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 exact top-k search: tcgen05 fused score + top-k, GEMV, merge, ingest";
  m.def("scores", &scores, "Full score matrix q @ x^T", py::arg("q"), py::arg("x"),
        py::arg("out_fp32") = true);
  m.def("fused_topk", &fused_topk, "Fused score + top-k", py::arg("q"), py::arg("x"), py::arg("k"),
        py::arg("bq") = 0, py::arg("chunks") = 0);
  m.def("fused_topk_into", &fused_topk_into, "Fused top-k into given outputs with an id offset",
        py::arg("q"), py::arg("x"), py::arg("k"), py::arg("id_offset"), py::arg("out_v"),
        py::arg("out_i"), py::arg("workspace"), py::arg("chunks") = 0);
  m.def("search", &search, "Search from raw queries (prepared in the search's first launch)", py::arg("q"),
        py::arg("x"), py::arg("k"), py::arg("cosine"));
  m.def("search_into", &search_into, "search() into given outputs and workspace, with an id offset", py::arg("q"),
        py::arg("x"), py::arg("k"), py::arg("cosine"), py::arg("id_offset"), py::arg("out_v"), py::arg("out_i"),
        py::arg("ws"));
  m.def("search_workspace_size", &search_workspace_size, "Workspace bytes for search_into", py::arg("b"),
        py::arg("n"), py::arg("d_pad"), py::arg("k"));
  m.def("workspace_size", &workspace_size, "Workspace bytes for fused_topk_into", py::arg("b"),
        py::arg("n"), py::arg("d_pad"), py::arg("k"), py::arg("chunks") = 0);
  m.def("ingest_into", &ingest_into, "Convert / normalise / pad rows into an fp16 matrix",
        py::arg("src"), py::arg("dst"), py::arg("cosine"));
  m.def("merge_lists", &merge_lists, "Merge [lists, b, len] result lists into the best k",
        py::arg("v"), py::arg("i"), py::arg("k"));
  m.def("poll_device_error", &poll_device_error, "Read and clear the device error word",
        py::arg("device"));
  m.def("set_profile_events", &set_profile_events, "Record events around the search kernel",
        py::arg("start"), py::arg("stop"));
}
