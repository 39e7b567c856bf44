// Python bindings of the inference kernels: paged KV write / gather, paged
// split-KV decode attention and the fused sampler.
#include <cstdlib>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_runtime.h>

namespace astrai_host {
int num_sms(int device);
void paged_kv_write(const void* k, const void* v, long long ld_src, const int* slot, int T, int Hkv, int page_size,
                    int n_pages, void* kc, void* vc, int D, cudaStream_t s);
void paged_kv_gather(const void* kc, const void* vc, const int* table, int max_pages, const int* lens, int B, int S_out,
                     int Hkv, int page_size, int n_pages, void* ko, void* vo, int D, cudaStream_t s);
void paged_decode_launch(const void* q, long long ldq, const void* kc, const void* vc, const int* table, int max_pages,
                         int n_pages, const int* lens, int B, int Hq, int Hkv, int page_size, int splits, float scale_log2,
                         float* part_acc, float* part_ml, void* out, long long ldo, int D, cudaStream_t s);
int decode_splits(int B, int Hkv, int max_len, int sms);
bool paged_decode_tc_supported(int D, int G, int page_size);
void decode_combine(const float* part_acc, const float* part_ml, int B, int Hq, int Hkv, int splits, void* out,
                    long long ldo, int D, cudaStream_t s);
void paged_decode_tc(const void* q, long long ldq, const void* kc, const void* vc, const int* table, int max_pages,
                     int n_pages, const int* lens, int B, int Hq, int Hkv, int page_size, int splits,
                     float scale_log2, float* part_acc, float* part_ml, void* out, long long ldo, int D,
                     cudaStream_t s);
void sample_tokens(const void* logits, int f32, long long ld, int rows, int V, const float* temperature,
                   const int* top_k, const float* top_p, const float* penalty, const long long* hist, int hist_len,
                   long long ld_hist, const unsigned long long* rng, long long* out_tok, float* out_lp,
                   cudaStream_t s);
}  // namespace astrai_host

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }
// ASTRAI_DECODE_TC=0 keeps decode on the CUDA-core kernel (for comparisons)
bool decode_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_DECODE_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

// [n_pages, Hkv, page_size, D] bf16 contiguous, D = 64 or 128; returns D
int check_cache(const at::Tensor& c, const char* name) {
  TORCH_CHECK(c.is_cuda() && c.scalar_type() == at::kBFloat16, name, " must be a CUDA bfloat16 tensor");
  TORCH_CHECK(c.dim() == 4 && (c.size(3) == 128 || c.size(3) == 64) && c.is_contiguous(), name,
              " must be contiguous [n_pages, n_kv_heads, page_size, head_dim] with head_dim 64 or 128");
  return static_cast<int>(c.size(3));
}

void check_i32(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), name,
              " must be a contiguous CUDA int32 tensor");
}

void check_rows16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a CUDA bfloat16 tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with a contiguous inner dimension");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " rows must be 16-byte aligned");
}

// k / v: [T, >= Hkv*D] row views (e.g. column slices of a fused qkv buffer)
void paged_kv_write(const at::Tensor& k, const at::Tensor& v, const at::Tensor& slot, at::Tensor& kc, at::Tensor& vc) {
  check_rows16(k, "k");
  check_rows16(v, "v");
  TORCH_CHECK(k.stride(0) == v.stride(0), "k and v must share a row stride");
  check_i32(slot, "slot");
  const int D = check_cache(kc, "k_cache");
  TORCH_CHECK(check_cache(vc, "v_cache") == D && vc.sizes() == kc.sizes(), "k_cache / v_cache shapes differ");
  const int T = static_cast<int>(k.size(0));
  TORCH_CHECK(slot.numel() == T && v.size(0) == T, "slot / v row count mismatch");
  const int Hkv = static_cast<int>(kc.size(1));
  TORCH_CHECK(k.size(1) >= Hkv * D && v.size(1) >= Hkv * D, "k/v narrower than n_kv_heads * head_dim");
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(k.device());
  astrai_host::paged_kv_write(k.data_ptr(), v.data_ptr(), k.stride(0), slot.data_ptr<int>(), T, Hkv,
                              static_cast<int>(kc.size(2)), static_cast<int>(kc.size(0)), kc.data_ptr(), vc.data_ptr(),
                              D, cur_stream());
}

// -> (k, v) [B, S_out, Hkv, D]; rows past lens[b] are zero
std::vector<at::Tensor> paged_kv_gather(const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& table,
                                        const at::Tensor& lens, int64_t S_out) {
  const int D = check_cache(kc, "k_cache");
  TORCH_CHECK(check_cache(vc, "v_cache") == D && vc.sizes() == kc.sizes(), "k_cache / v_cache shapes differ");
  check_i32(table, "page_table");
  check_i32(lens, "lens");
  TORCH_CHECK(table.dim() == 2 && lens.numel() == table.size(0), "page_table [B, max_pages] / lens [B] mismatch");
  const int B = static_cast<int>(table.size(0));
  const int Hkv = static_cast<int>(kc.size(1));
  auto ko = at::empty({B, S_out, Hkv, D}, kc.options());
  auto vo = at::empty({B, S_out, Hkv, D}, kc.options());
  if (B == 0 || S_out == 0) return {ko, vo};
  const c10::cuda::CUDAGuard g(kc.device());
  astrai_host::paged_kv_gather(kc.data_ptr(), vc.data_ptr(), table.data_ptr<int>(), static_cast<int>(table.size(1)),
                               lens.data_ptr<int>(), B, static_cast<int>(S_out), Hkv, static_cast<int>(kc.size(2)),
                               static_cast<int>(kc.size(0)), ko.data_ptr(), vo.data_ptr(), D, cur_stream());
  return {ko, vo};
}

int64_t decode_splits(int64_t B, int64_t Hkv, int64_t max_len, int64_t device) {
  return astrai_host::decode_splits(static_cast<int>(B), static_cast<int>(Hkv), static_cast<int>(max_len),
                                    astrai_host::num_sms(static_cast<int>(device)));
}

// q: [B, >= Hq*D] rows; out: [B, Hq*D] rows; workspace fp32 with
// >= B*Hq*splits*(D + 2) elements when splits > 1
void paged_decode(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& table,
                  const at::Tensor& lens, at::Tensor& out, int64_t Hq, double scale, int64_t splits,
                  const c10::optional<at::Tensor>& workspace) {
  check_rows16(q, "q");
  check_rows16(out, "out");
  const int D = check_cache(kc, "k_cache");
  TORCH_CHECK(check_cache(vc, "v_cache") == D && vc.sizes() == kc.sizes(), "k_cache / v_cache shapes differ");
  check_i32(table, "page_table");
  check_i32(lens, "lens");
  const int B = static_cast<int>(q.size(0));
  const int Hkv = static_cast<int>(kc.size(1));
  TORCH_CHECK(Hq % Hkv == 0, "n_heads must be a multiple of n_kv_heads");
  const int G = static_cast<int>(Hq / Hkv);
  const int page_size = static_cast<int>(kc.size(2));
  const bool tc = decode_tc_enabled() && astrai_host::paged_decode_tc_supported(D, G, page_size);
  TORCH_CHECK(tc || G == 1 || G == 2 || G == 4 || G == 8,
              "paged_decode: n_heads / n_kv_heads must be 1 - 8, 12 or 16 with head_dim 64 / 128 and page_size a "
              "multiple or divisor of 128 (otherwise 1, 2, 4 or 8)");
  TORCH_CHECK(table.dim() == 2 && table.size(0) == B && lens.numel() == B, "page_table / lens batch mismatch");
  TORCH_CHECK(q.size(1) >= Hq * D && out.size(0) == B && out.size(1) >= Hq * D, "q/out shape mismatch");
  TORCH_CHECK(splits >= 1 && splits <= 64, "splits must be in [1, 64]");
  if (B == 0) return;
  float* part_acc = nullptr;
  float* part_ml = nullptr;
  if (splits > 1) {
    TORCH_CHECK(workspace.has_value(), "paged_decode: splits > 1 needs a workspace");
    const auto& w = *workspace;
    TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kFloat && w.is_contiguous(), "workspace must be fp32 CUDA");
    const long long need = (long long)B * Hq * splits * (D + 2);
    TORCH_CHECK(w.numel() >= need, "workspace too small: need ", need, " fp32 elements");
    part_acc = w.data_ptr<float>();
    part_ml = part_acc + (long long)B * Hq * splits * D;
  }
  const c10::cuda::CUDAGuard g(q.device());
  if (tc) {
    astrai_host::paged_decode_tc(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), table.data_ptr<int>(),
                                 static_cast<int>(table.size(1)), static_cast<int>(kc.size(0)), lens.data_ptr<int>(), B,
                                 static_cast<int>(Hq), Hkv, page_size, static_cast<int>(splits),
                                 static_cast<float>(scale * 1.4426950408889634), part_acc, part_ml, out.data_ptr(),
                                 out.stride(0), D, cur_stream());
    if (splits > 1)
      astrai_host::decode_combine(part_acc, part_ml, B, static_cast<int>(Hq), Hkv, static_cast<int>(splits),
                                  out.data_ptr(), out.stride(0), D, cur_stream());
    return;
  }
  astrai_host::paged_decode_launch(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), table.data_ptr<int>(),
                                   static_cast<int>(table.size(1)), static_cast<int>(kc.size(0)), lens.data_ptr<int>(),
                                   B, static_cast<int>(Hq), Hkv,
                                   static_cast<int>(kc.size(2)), static_cast<int>(splits),
                                   static_cast<float>(scale * 1.4426950408889634), part_acc, part_ml, out.data_ptr(),
                                   out.stride(0), D, cur_stream());
}

// logits [rows, V] (bf16 or fp32, unit inner stride); per-row parameters are
// device tensors (None -> defaults: temperature 1, top_k 0, top_p 1, penalty 0);
// hist [rows, H] int64 with -1 padding; rng int64 [2] = (seed, counter)
void sample(const at::Tensor& logits, const c10::optional<at::Tensor>& temperature,
            const c10::optional<at::Tensor>& top_k, const c10::optional<at::Tensor>& top_p,
            const c10::optional<at::Tensor>& penalty, const c10::optional<at::Tensor>& hist, const at::Tensor& rng,
            at::Tensor& out_tok, const c10::optional<at::Tensor>& out_lp) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D CUDA rows");
  const bool f32 = logits.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || logits.scalar_type() == at::kBFloat16, "logits must be fp32 or bf16");
  const int rows = static_cast<int>(logits.size(0));
  auto f32p = [&](const c10::optional<at::Tensor>& t, const char* n) -> const float* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == rows, n,
                " must be a contiguous CUDA fp32 tensor with one entry per row");
    return t->data_ptr<float>();
  };
  const int* tk = nullptr;
  if (top_k.has_value()) {
    check_i32(*top_k, "top_k");
    TORCH_CHECK(top_k->numel() == rows, "top_k needs one entry per row");
    tk = top_k->data_ptr<int>();
  }
  const long long* hp = nullptr;
  int hl = 0;
  long long ldh = 0;
  if (hist.has_value() && hist->numel() > 0) {
    TORCH_CHECK(hist->is_cuda() && hist->scalar_type() == at::kLong && hist->dim() == 2 && hist->size(0) == rows &&
                    hist->stride(1) == 1,
                "hist must be a CUDA int64 [rows, H] tensor");
    hp = reinterpret_cast<const long long*>(hist->data_ptr<int64_t>());
    hl = static_cast<int>(hist->size(1));
    ldh = hist->stride(0);
  }
  TORCH_CHECK(rng.is_cuda() && rng.scalar_type() == at::kLong && rng.numel() >= 2, "rng must be CUDA int64 [2]");
  TORCH_CHECK(out_tok.is_cuda() && out_tok.scalar_type() == at::kLong && out_tok.numel() == rows &&
                  out_tok.is_contiguous(),
              "out_tok must be CUDA int64 [rows]");
  float* lp = nullptr;
  if (out_lp.has_value()) {
    TORCH_CHECK(out_lp->is_cuda() && out_lp->scalar_type() == at::kFloat && out_lp->numel() == rows &&
                    out_lp->is_contiguous(),
                "out_logprob must be CUDA fp32 [rows]");
    lp = out_lp->data_ptr<float>();
  }
  if (rows == 0) return;
  const c10::cuda::CUDAGuard g(logits.device());
  astrai_host::sample_tokens(logits.data_ptr(), f32 ? 1 : 0, logits.stride(0), rows, static_cast<int>(logits.size(1)),
                             f32p(temperature, "temperature"), tk, f32p(top_p, "top_p"), f32p(penalty, "penalty"), hp,
                             hl, ldh, reinterpret_cast<const unsigned long long*>(rng.data_ptr<int64_t>()),
                             reinterpret_cast<long long*>(out_tok.data_ptr<int64_t>()), lp, cur_stream());
}

}  // namespace

void register_inference(pybind11::module& m) {
  namespace py = pybind11;
  m.def("paged_kv_write", &paged_kv_write, py::arg("k"), py::arg("v"), py::arg("slot"), py::arg("k_cache"),
        py::arg("v_cache"));
  m.def("paged_kv_gather", &paged_kv_gather, py::arg("k_cache"), py::arg("v_cache"), py::arg("page_table"),
        py::arg("lens"), py::arg("s_out"));
  m.def("decode_splits", &decode_splits);
  m.def("paged_decode", &paged_decode, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("page_table"),
        py::arg("lens"), py::arg("out"), py::arg("n_heads"), py::arg("scale"), py::arg("splits"),
        py::arg("workspace") = py::none());
  m.def("sample", &sample, py::arg("logits"), py::arg("temperature"), py::arg("top_k"), py::arg("top_p"),
        py::arg("penalty"), py::arg("hist"), py::arg("rng"), py::arg("out_tok"), py::arg("out_logprob"));
}
