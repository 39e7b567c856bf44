// Python bindings of the MoE router and expert-parallel dispatch / return / combine kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_runtime.h>

#include "ep_arena.h"

namespace astrai_host {
int* error_word(int device);
int num_sms(int device);
void moe_router(const void* logits, int f32, long long ld, int T, int E, int k, float* probs, int* idx, float* w,
                int* counts, int* pos, cudaStream_t s);
astrai::EPArena make_arena(const long long* peer_base, int rank, int world, const long long* offs, long long rows_cap,
                           long long slots_cap, int d, unsigned* done, unsigned* expect, int* err,
                           unsigned long long wait_ns);
void ep_dispatch(const astrai::EPArena& a, const void* x, long long ldx, const int* idx, const int* pos,
                 const int* base_row, int n_slots, int k, int e_local, int* slot_row, int ctas, cudaStream_t s);
void ep_wait(const astrai::EPArena& a, int phase, cudaStream_t s);
void ep_layout(const astrai::EPArena& a, const int* counts, int E, int e_local, int* base_row, int* n_rows, int* starts,
               int* k_count, int* group_tile, int max_tiles, int* total, cudaStream_t s);
void ep_dispatch_fp8(const astrai::EPArena& a, const void* x, long long ldx, const int* idx, const int* pos,
                     const int* base_row, int n_slots, int k, int e_local, int* slot_row, int ctas,
                     cudaStream_t s);
void ep_dequant(const astrai::EPArena& a, long long rows, int ctas, cudaStream_t s);
void ep_return(const astrai::EPArena& a, const void* rows, long long total_rows, const int* group_tile,
               const int* starts, const int* n_rows, int to_ret2, int ctas, cudaStream_t s);
void ep_combine(const void* slots, const float* w, const void* add, void* out, int T, int k, int d, cudaStream_t s);
void ep_combine_bwd(const astrai::EPArena& a, const void* dout, const void* slots, const float* w, const int* idx,
                    const int* slot_row, int n_slots, int k, int e_local, float* dw, int ctas, cudaStream_t s);
void ep_zero_pad(const astrai::EPArena& a, int which_dyin, long long total_rows, const int* group_tile,
                 const int* starts, const int* n_rows, cudaStream_t s);
void gemm_grouped_bf16(int mode, const void* A, const void* B, void* D, const void* C, int M, int N, int K,
                       int groups, int b_mn, long long lda, long long ldb, long long strideB, long long ldd,
                       long long strideD, const int* group_tile, const int* k_start, const int* k_count,
                       float alpha, float beta, cudaStream_t stream);
}  // namespace astrai_host

namespace {

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream().stream(); }

void chk(const at::Tensor& t, at::ScalarType st, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == st && t.is_contiguous(), n, ": wrong dtype / device / layout");
}

// Arena description passed from Python: peer_base int64 [W], offs [9] (flags, srcmap, xin, dyin, ret, ret2,
// xin8, xsc, counts; xin8 / xsc are 0 without fp8 dispatch), the local grid-completion counter and the
// local per-phase round counters (int32 [5]).
astrai::EPArena arena_of(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                         const at::Tensor& expect, int64_t rank, int64_t world, int64_t rows_cap, int64_t slots_cap,
                         int64_t d, double wait_s) {
  chk(peer_base, at::kLong, "peer_base");
  chk(done, at::kInt, "done");
  chk(expect, at::kInt, "expect");
  TORCH_CHECK(offs.size() == 9 && peer_base.numel() == world && d % 8 == 0 && expect.numel() == astrai::kEPPhases,
              "bad arena description");
  static thread_local long long o[9];
  for (int i = 0; i < 9; ++i) o[i] = offs[i];
  return astrai_host::make_arena(reinterpret_cast<const long long*>(peer_base.data_ptr<int64_t>()),
                                 static_cast<int>(rank), static_cast<int>(world), o, rows_cap, slots_cap,
                                 static_cast<int>(d), reinterpret_cast<unsigned*>(done.data_ptr<int>()),
                                 reinterpret_cast<unsigned*>(expect.data_ptr<int>()),
                                 astrai_host::error_word(peer_base.device().index()),
                                 static_cast<unsigned long long>(wait_s * 1e9));
}

void moe_router(const at::Tensor& logits, int64_t k, at::Tensor& probs, at::Tensor& idx, at::Tensor& w,
                at::Tensor& counts, at::Tensor& pos) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D CUDA rows");
  const bool f32 = logits.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || logits.scalar_type() == at::kBFloat16, "logits must be fp32 or bf16");
  const int T = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1));
  chk(probs, at::kFloat, "probs");
  chk(idx, at::kInt, "idx");
  chk(w, at::kFloat, "w");
  chk(counts, at::kInt, "counts");
  chk(pos, at::kInt, "pos");
  TORCH_CHECK(probs.numel() == (int64_t)T * E && idx.numel() == T * k && w.numel() == T * k && pos.numel() == T * k &&
                  counts.numel() == E,
              "moe_router: output sizes");
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(logits.device());
  astrai_host::moe_router(logits.data_ptr(), f32, logits.stride(0), T, E, static_cast<int>(k), probs.data_ptr<float>(),
                          idx.data_ptr<int>(), w.data_ptr<float>(), counts.data_ptr<int>(), pos.data_ptr<int>(), cur());
}

int ctas_for(const at::Tensor& t) { return astrai_host::num_sms(t.device().index()); }

void ep_dispatch_any(bool fp8, const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                     const at::Tensor& expect, int64_t rank, int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s,
                     const at::Tensor& x, const at::Tensor& idx, const at::Tensor& pos, const at::Tensor& base_row,
                     int64_t e_local, at::Tensor& slot_row) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && x.size(1) == d &&
                  (x.stride(0) * 2) % 16 == 0,
              "x must be bf16 [T, d] rows");
  chk(idx, at::kInt, "idx");
  chk(pos, at::kInt, "pos");
  chk(base_row, at::kInt, "base_row");
  chk(slot_row, at::kInt, "slot_row");
  const int64_t n_slots = idx.numel();
  TORCH_CHECK(n_slots <= slots_cap && pos.numel() == n_slots && slot_row.numel() == n_slots, "slot counts");
  const int k = static_cast<int>(n_slots / x.size(0));
  const c10::cuda::CUDAGuard g(x.device());
  (fp8 ? astrai_host::ep_dispatch_fp8 : astrai_host::ep_dispatch)(a, x.data_ptr(), x.stride(0), idx.data_ptr<int>(), pos.data_ptr<int>(),
                           base_row.data_ptr<int>(), static_cast<int>(n_slots), k, static_cast<int>(e_local),
                           slot_row.data_ptr<int>(), ctas_for(x), cur());
}

void ep_dispatch(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                 const at::Tensor& expect, int64_t rank,
                 int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s, const at::Tensor& x,
                 const at::Tensor& idx, const at::Tensor& pos, const at::Tensor& base_row, int64_t e_local,
                 at::Tensor& slot_row) {
  ep_dispatch_any(false, peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s, x, idx, pos, base_row,
                  e_local, slot_row);
}

// Token rows as fp8 e4m3 with one fp32 scale per 128 columns (the arena's fp8 block).
void ep_dispatch_fp8(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                     const at::Tensor& expect, int64_t rank, int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s,
                     const at::Tensor& x, const at::Tensor& idx, const at::Tensor& pos, const at::Tensor& base_row,
                     int64_t e_local, at::Tensor& slot_row) {
  ep_dispatch_any(true, peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s, x, idx, pos, base_row,
                  e_local, slot_row);
}

// bf16 expert-input rows [0, rows) of this rank's arena from its fp8 block.
void ep_dequant(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                 const at::Tensor& expect, int64_t rank,
                int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s, int64_t rows) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  const c10::cuda::CUDAGuard g(peer_base.device());
  astrai_host::ep_dequant(a, rows, ctas_for(peer_base), cur());
}

void ep_wait(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                 const at::Tensor& expect, int64_t rank,
             int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s, int64_t phase) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  const c10::cuda::CUDAGuard g(peer_base.device());
  astrai_host::ep_wait(a, static_cast<int>(phase), cur());
}

// Counts exchange + dispatch layout on the device; outputs int32: base_row [E], n_rows / starts / k_count
// [e_local], group_tile [max_tiles], total [1].
void ep_layout(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
               const at::Tensor& expect, int64_t rank, int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d,
               double wait_s, const at::Tensor& counts, int64_t e_local, at::Tensor& base_row, at::Tensor& n_rows,
               at::Tensor& starts, at::Tensor& k_count, at::Tensor& group_tile, at::Tensor& total) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&counts, &base_row, &n_rows, &starts, &k_count,
                                                                      &group_tile, &total})
    chk(*t, at::kInt, "ep_layout tables");
  const int64_t E = counts.numel();
  TORCH_CHECK(base_row.numel() == E && n_rows.numel() == e_local && starts.numel() == e_local &&
                  k_count.numel() == e_local && total.numel() == 1 && group_tile.numel() * 128 <= rows_cap,
              "ep_layout: table sizes");
  const c10::cuda::CUDAGuard g(counts.device());
  astrai_host::ep_layout(a, counts.data_ptr<int>(), static_cast<int>(E), static_cast<int>(e_local),
                         base_row.data_ptr<int>(), n_rows.data_ptr<int>(), starts.data_ptr<int>(),
                         k_count.data_ptr<int>(), group_tile.data_ptr<int>(), static_cast<int>(group_tile.numel()),
                         total.data_ptr<int>(), cur());
}

void ep_return(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                 const at::Tensor& expect, int64_t rank,
               int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s, const at::Tensor& rows,
               const at::Tensor& group_tile, const at::Tensor& starts, const at::Tensor& n_rows, int64_t to_ret2) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  chk(rows, at::kBFloat16, "rows");
  chk(group_tile, at::kInt, "group_tile");
  chk(starts, at::kInt, "starts");
  chk(n_rows, at::kInt, "n_rows");
  const int64_t total = rows.numel() / d;
  TORCH_CHECK(total % 128 == 0 && group_tile.numel() == total / 128 && total <= rows_cap, "rows must be [M_total, d]");
  const c10::cuda::CUDAGuard g(rows.device());
  astrai_host::ep_return(a, rows.data_ptr(), total, group_tile.data_ptr<int>(), starts.data_ptr<int>(),
                         n_rows.data_ptr<int>(), static_cast<int>(to_ret2), ctas_for(rows), cur());
}

void ep_combine(const at::Tensor& slots, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& add,
                at::Tensor& out, int64_t k) {
  chk(slots, at::kBFloat16, "slots");
  chk(out, at::kBFloat16, "out");
  const int64_t T = out.size(0), d = out.size(1);
  TORCH_CHECK(out.dim() == 2 && d % 8 == 0 && slots.numel() >= T * k * d, "combine shapes");
  const float* wp = nullptr;
  if (w.has_value()) {
    chk(*w, at::kFloat, "w");
    TORCH_CHECK(w->numel() == T * k, "w must be [T, k]");
    wp = w->data_ptr<float>();
  }
  const void* ap = nullptr;
  if (add.has_value()) {
    chk(*add, at::kBFloat16, "add");
    TORCH_CHECK(add->numel() == T * d, "add must be [T, d]");
    ap = add->data_ptr();
  }
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(out.device());
  astrai_host::ep_combine(slots.data_ptr(), wp, ap, out.data_ptr(), static_cast<int>(T), static_cast<int>(k),
                          static_cast<int>(d), cur());
}

void ep_combine_bwd(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                    const at::Tensor& expect, int64_t rank, int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s,
                    const at::Tensor& dout, const at::Tensor& slots, const at::Tensor& w, const at::Tensor& idx,
                    const at::Tensor& slot_row, int64_t e_local, at::Tensor& dw) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  chk(dout, at::kBFloat16, "dout");
  chk(slots, at::kBFloat16, "slots");
  chk(w, at::kFloat, "w");
  chk(idx, at::kInt, "idx");
  chk(slot_row, at::kInt, "slot_row");
  chk(dw, at::kFloat, "dw");
  const int64_t n_slots = idx.numel();
  TORCH_CHECK(dout.size(1) == d && w.numel() == n_slots && dw.numel() == n_slots && slot_row.numel() == n_slots,
              "combine_bwd shapes");
  const int k = static_cast<int>(n_slots / dout.size(0));
  const c10::cuda::CUDAGuard g(dout.device());
  astrai_host::ep_combine_bwd(a, dout.data_ptr(), slots.data_ptr(), w.data_ptr<float>(), idx.data_ptr<int>(),
                              slot_row.data_ptr<int>(), static_cast<int>(n_slots), k, static_cast<int>(e_local),
                              dw.data_ptr<float>(), ctas_for(dout), cur());
}

void ep_zero_pad(const at::Tensor& peer_base, const std::vector<int64_t>& offs, const at::Tensor& done,
                 const at::Tensor& expect, int64_t rank,
                 int64_t world, int64_t rows_cap, int64_t slots_cap, int64_t d, double wait_s, int64_t which_dyin,
                 int64_t total_rows, const at::Tensor& group_tile, const at::Tensor& starts,
                 const at::Tensor& n_rows) {
  auto a = arena_of(peer_base, offs, done, expect, rank, world, rows_cap, slots_cap, d, wait_s);
  chk(group_tile, at::kInt, "group_tile");
  chk(starts, at::kInt, "starts");
  chk(n_rows, at::kInt, "n_rows");
  TORCH_CHECK(total_rows <= rows_cap && total_rows % 128 == 0 && group_tile.numel() == total_rows / 128,
              "zero_pad beyond capacity");
  const c10::cuda::CUDAGuard g(peer_base.device());
  astrai_host::ep_zero_pad(a, static_cast<int>(which_dyin), total_rows, group_tile.data_ptr<int>(),
                           starts.data_ptr<int>(), n_rows.data_ptr<int>(), cur());
}

// mode 0 (grouped-M): a [M_total, K], b [G, N, K] (b_mn 0) / [G, K, N] (b_mn 1), d [M_total, N],
//        groups = b.size(0), tables: group_tile [M_total / 128].
// mode 1 (grouped-K): a [K_total, M], b [K_total, N], d [G, M, N], tables: k_start / k_count [G].
void gemm_grouped(int64_t mode, const at::Tensor& a, const at::Tensor& b, at::Tensor& d,
                  const c10::optional<at::Tensor>& c, const c10::optional<at::Tensor>& group_tile,
                  const c10::optional<at::Tensor>& k_start, const c10::optional<at::Tensor>& k_count, int64_t b_mn,
                  double alpha, double beta) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&a, &b, &d}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous(),
                "gemm_grouped: operands must be contiguous CUDA bf16");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "gemm_grouped: 16-byte aligned operands");
  }
  const void* cp = nullptr;
  if (c.has_value()) {
    TORCH_CHECK(c->is_cuda() && c->scalar_type() == at::kBFloat16 && c->sizes() == d.sizes() && c->is_contiguous(),
                "gemm_grouped: c must match d");
    cp = c->data_ptr();
  }
  int M, N, K, G;
  long long strideB = 0, strideD = 0;
  const int *gt = nullptr, *ks = nullptr, *kc = nullptr;
  if (mode == 0) {
    TORCH_CHECK(a.dim() == 2 && b.dim() == 3 && d.dim() == 2, "grouped-M: a [M, K], b [G, ., .], d [M, N]");
    M = a.size(0);
    K = a.size(1);
    G = b.size(0);
    N = b_mn ? b.size(2) : b.size(1);
    TORCH_CHECK((b_mn ? b.size(1) : b.size(2)) == K && d.size(0) == M && d.size(1) == N && M % 128 == 0,
                "grouped-M shapes (M_total must be a multiple of 128)");
    TORCH_CHECK(group_tile.has_value() && group_tile->scalar_type() == at::kInt && group_tile->is_cuda() &&
                    group_tile->numel() == M / 128,
                "grouped-M needs group_tile int32 [M / 128]");
    strideB = b.stride(0);
    gt = group_tile->data_ptr<int>();
  } else {
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && d.dim() == 3, "grouped-K: a [K, M], b [K, N], d [G, M, N]");
    K = a.size(0);
    M = a.size(1);
    N = b.size(1);
    G = d.size(0);
    TORCH_CHECK(b.size(0) == K && d.size(1) == M && d.size(2) == N, "grouped-K shapes");
    TORCH_CHECK(k_start.has_value() && k_count.has_value() && k_start->numel() == G && k_count->numel() == G &&
                    k_start->scalar_type() == at::kInt && k_count->scalar_type() == at::kInt,
                "grouped-K needs k_start / k_count int32 [G]");
    strideD = d.stride(0);
    ks = k_start->data_ptr<int>();
    kc = k_count->data_ptr<int>();
    b_mn = 1;
  }
  const c10::cuda::CUDAGuard g(a.device());
  astrai_host::gemm_grouped_bf16(static_cast<int>(mode), a.data_ptr(), b.data_ptr(), d.data_ptr(), cp, M, N, K, G,
                                 static_cast<int>(b_mn), a.stride(0), b_mn ? (mode == 0 ? b.stride(1) : b.stride(0))
                                                                            : b.stride(1),
                                 strideB, d.stride(mode == 0 ? 0 : 1), strideD, gt, ks, kc, static_cast<float>(alpha),
                                 static_cast<float>(beta), cur());
}

at::Tensor symm_view(int64_t ptr, int64_t nbytes, int64_t device) {
  return at::from_blob(reinterpret_cast<void*>(ptr), {nbytes},
                       at::TensorOptions().dtype(at::kByte).device(at::kCUDA, static_cast<int>(device)));
}

}  // namespace

void register_moe(pybind11::module& m) {
  m.def("moe_router", &moe_router);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_dispatch_fp8", &ep_dispatch_fp8);
  m.def("ep_dequant", &ep_dequant);
  m.def("ep_layout", &ep_layout);
  m.def("ep_wait", &ep_wait);
  m.def("ep_return", &ep_return);
  m.def("ep_combine", &ep_combine, pybind11::arg("slots"), pybind11::arg("w"), pybind11::arg("add"),
        pybind11::arg("out"), pybind11::arg("k"));
  m.def("ep_combine_bwd", &ep_combine_bwd);
  m.def("ep_zero_pad", &ep_zero_pad);
  m.def("gemm_grouped", &gemm_grouped, pybind11::arg("mode"), pybind11::arg("a"), pybind11::arg("b"),
        pybind11::arg("d"), pybind11::arg("c") = pybind11::none(), pybind11::arg("group_tile") = pybind11::none(),
        pybind11::arg("k_start") = pybind11::none(), pybind11::arg("k_count") = pybind11::none(),
        pybind11::arg("b_mn") = 0, pybind11::arg("alpha") = 1.0, pybind11::arg("beta") = 0.0);
  m.def("symm_view", &symm_view, "uint8 tensor over device memory owned elsewhere (no deleter)");
}
