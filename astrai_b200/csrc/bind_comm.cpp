// Python bindings of the NVLink peer-memory collectives.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_runtime.h>

namespace astrai_host {
int* error_word(int device);
void* symm_alloc(long long bytes, void* handle_out);
void* symm_open(const void* handle);
void symm_close(void* p);
void symm_free(void* p);
void fused_allreduce(const long long* seg_ptr, const long long* seg_off, int n_seg, long long N, int rank, int world,
                     long long R, const long long* peer_base, long long off_flag_a, long long off_flag_b,
                     long long off_sumsq, long long off_recv, long long off_gather, unsigned epoch0, int ctas,
                     float* sumsq_out, float* clip_coef, float max_norm, unsigned* done, int* err,
                     unsigned long long wait_ns, cudaStream_t s);
void muon_apply_peers(const long long* pptr, const long long* poff, const long long* peer_base, const void* X,
                      int batch, int R, int C, int transpose, float decay, float adj_lr, int rank, int world,
                      long long flag_off, int slot, unsigned epoch, unsigned* done, cudaStream_t s);
void peer_flags_wait(const unsigned* flags, int rank, int world, int rows, unsigned epoch, double wait_s,
                     cudaStream_t s);
void row_reduce_bcast(const void* part, const void* recv, void* out, long long ld, int M, int N, int rank, int world,
                      int rpo, const long long* rank_delta, unsigned* flag, unsigned epoch, unsigned* done,
                      int sms, cudaStream_t s);
int num_sms(int device);
void fsdp_reduce(const long long* peer_grad, const long long* seg_off, const long long* seg_vec, int n_seg,
                 long long total_vec, int rank, int world, float scale, float* sumsq, cudaStream_t s);
void fsdp_raise(const long long* peer_base, long long flag_off, int row, int rank, int world, unsigned epoch,
                cudaStream_t s);
}  // namespace astrai_host

namespace {

pybind11::tuple symm_alloc(int64_t bytes) {
  char h[64];
  void* p = astrai_host::symm_alloc(bytes, h);
  return pybind11::make_tuple(reinterpret_cast<int64_t>(p), pybind11::bytes(h, 64));
}

int64_t symm_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == 64, "symm_open: an IPC handle has 64 bytes");
  return reinterpret_cast<int64_t>(astrai_host::symm_open(handle.data()));
}

void i64_check(const at::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.is_contiguous(), n, " must be a CUDA int64 tensor");
}

void fused_allreduce(const at::Tensor& seg_ptr, const at::Tensor& seg_off, int64_t N, int64_t rank, int64_t world,
                     int64_t R, const at::Tensor& peer_base, int64_t off_flag_a, int64_t off_flag_b, int64_t off_sumsq,
                     int64_t off_recv, int64_t off_gather, int64_t epoch0, int64_t ctas, at::Tensor& sumsq_out,
                     const c10::optional<at::Tensor>& clip_coef, double max_norm, at::Tensor& done, double wait_s) {
  i64_check(seg_ptr, "seg_ptr");
  i64_check(seg_off, "seg_off");
  i64_check(peer_base, "peer_base");
  TORCH_CHECK(seg_off.numel() == seg_ptr.numel() + 1, "seg_off needs n_seg + 1 entries");
  TORCH_CHECK(peer_base.numel() == world && rank >= 0 && rank < world, "peer_base / rank mismatch");
  TORCH_CHECK(N % 8 == 0 && R % (8 * world) == 0, "sizes must be multiples of 8 elements per rank");
  TORCH_CHECK(sumsq_out.is_cuda() && sumsq_out.scalar_type() == at::kFloat, "sumsq_out must be CUDA fp32");
  TORCH_CHECK(done.is_cuda() && done.scalar_type() == at::kInt, "done must be CUDA int32");
  float* cc = nullptr;
  if (clip_coef.has_value()) {
    TORCH_CHECK(clip_coef->is_cuda() && clip_coef->scalar_type() == at::kFloat, "clip_coef must be CUDA fp32");
    cc = clip_coef->data_ptr<float>();
  }
  if (N == 0) return;
  const c10::cuda::CUDAGuard g(sumsq_out.device());
  astrai_host::fused_allreduce(reinterpret_cast<const long long*>(seg_ptr.data_ptr<int64_t>()),
                               reinterpret_cast<const long long*>(seg_off.data_ptr<int64_t>()),
                               static_cast<int>(seg_ptr.numel()), N, static_cast<int>(rank), static_cast<int>(world), R,
                               reinterpret_cast<const long long*>(peer_base.data_ptr<int64_t>()), off_flag_a,
                               off_flag_b, off_sumsq, off_recv, off_gather, static_cast<unsigned>(epoch0),
                               static_cast<int>(ctas), sumsq_out.data_ptr<float>(), cc, static_cast<float>(max_norm),
                               reinterpret_cast<unsigned*>(done.data_ptr<int>()),
                               astrai_host::error_word(sumsq_out.device().index()),
                               static_cast<unsigned long long>(wait_s * 1e9), at::cuda::getCurrentCUDAStream().stream());
}

// Owner-sharded Muon: apply the orthogonalised update X (bf16 [batch][R][C], or [batch][C][R] when
// transpose) to the parameters at pptr and store the result into every rank's copy (peer_base[q] + poff).
void muon_apply_peers(const c10::optional<at::Tensor>& pptr, const c10::optional<at::Tensor>& poff,
                      const at::Tensor& peer_base,
                      const c10::optional<at::Tensor>& X, int64_t batch, int64_t R, int64_t C, bool transpose,
                      double decay, double adj_lr, int64_t rank, int64_t world, int64_t flag_off, int64_t slot,
                      int64_t epoch, at::Tensor& done) {
  i64_check(peer_base, "peer_base");
  TORCH_CHECK(peer_base.numel() == world && rank >= 0 && rank < world, "peer_base / rank mismatch");
  TORCH_CHECK(done.is_cuda() && done.scalar_type() == at::kInt && done.numel() >= 1, "done must be CUDA int32");
  TORCH_CHECK(flag_off % 4 == 0 && slot >= -1, "bad flag offset / slot (-1: raise no flag)");
  const void* xp = nullptr;
  const long long* pp = nullptr;
  const long long* po = nullptr;
  if (batch > 0) {
    TORCH_CHECK(pptr.has_value() && poff.has_value(), "pptr / poff are required when batch > 0");
    i64_check(*pptr, "pptr");
    i64_check(*poff, "poff");
    TORCH_CHECK(pptr->numel() == batch && poff->numel() == batch, "pptr / poff need one entry per matrix");
    TORCH_CHECK(X.has_value() && X->is_cuda() && X->scalar_type() == at::kBFloat16 && X->is_contiguous() &&
                    X->numel() == batch * R * C,
                "X must be a contiguous CUDA bf16 [batch, R, C] (or [batch, C, R]) tensor");
    xp = X->data_ptr();
    pp = reinterpret_cast<const long long*>(pptr->data_ptr<int64_t>());
    po = reinterpret_cast<const long long*>(poff->data_ptr<int64_t>());
  }
  const c10::cuda::CUDAGuard g(done.device());
  astrai_host::muon_apply_peers(pp, po, reinterpret_cast<const long long*>(peer_base.data_ptr<int64_t>()), xp,
                                static_cast<int>(batch), static_cast<int>(R), static_cast<int>(C), transpose ? 1 : 0,
                                static_cast<float>(decay), static_cast<float>(adj_lr), static_cast<int>(rank),
                                static_cast<int>(world), flag_off, static_cast<int>(slot),
                                static_cast<unsigned>(epoch), reinterpret_cast<unsigned*>(done.data_ptr<int>()),
                                at::cuda::getCurrentCUDAStream().stream());
}

// Wait (bounded) until every peer raised flag rows [0, rows) of `flags` (u32 [rows][world], this rank's copy).
void peer_flags_wait(int64_t flags_addr, int64_t device, int64_t rank, int64_t world, int64_t rows, int64_t epoch,
                     double wait_s) {
  TORCH_CHECK(flags_addr % 4 == 0 && rank >= 0 && rank < world && rows >= 0, "bad peer_flags_wait arguments");
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  astrai_host::peer_flags_wait(reinterpret_cast<const unsigned*>(flags_addr), static_cast<int>(rank),
                               static_cast<int>(world), static_cast<int>(rows), static_cast<unsigned>(epoch), wait_s,
                               at::cuda::getCurrentCUDAStream().stream());
}

// Owner-side gradient reduction of the fused FSDP: peer_grad int64 [world] pool bases, seg_off int64
// [n] byte offsets of this rank's owned gradients, seg_vec int64 [n + 1] prefix sums of their 16-byte
// vectors; sumsq fp32 [1] (accumulated).
void fsdp_reduce(const at::Tensor& peer_grad, const at::Tensor& seg_off, const at::Tensor& seg_vec, int64_t total_vec,
                 int64_t rank, int64_t world, double scale, at::Tensor& sumsq) {
  for (const at::Tensor* t : {&peer_grad, &seg_off, &seg_vec})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kLong && t->is_contiguous(), "fsdp_reduce: int64 CUDA tables");
  TORCH_CHECK(peer_grad.numel() == world && seg_vec.numel() == seg_off.numel() + 1, "fsdp_reduce: table sizes");
  TORCH_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == at::kFloat && sumsq.numel() == 1, "fsdp_reduce: sumsq");
  const c10::cuda::CUDAGuard g(peer_grad.device());
  astrai_host::fsdp_reduce(reinterpret_cast<const long long*>(peer_grad.data_ptr<int64_t>()),
                           reinterpret_cast<const long long*>(seg_off.data_ptr<int64_t>()),
                           reinterpret_cast<const long long*>(seg_vec.data_ptr<int64_t>()),
                           static_cast<int>(seg_off.numel()), total_vec, static_cast<int>(rank),
                           static_cast<int>(world), static_cast<float>(scale), sumsq.data_ptr<float>(),
                           at::cuda::getCurrentCUDAStream().stream());
}

// One device-to-device copy on the current stream, by the copy engines (addresses may be peer mappings).
void peer_copy(int64_t dst, int64_t src, int64_t nbytes) {
  TORCH_CHECK(nbytes >= 0 && (nbytes == 0 || (dst != 0 && src != 0)), "peer_copy: bad arguments");
  if (nbytes == 0) return;
  const cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src),
                                        static_cast<size_t>(nbytes), cudaMemcpyDeviceToDevice,
                                        at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(e == cudaSuccess, "peer_copy: ", cudaGetErrorString(e));
}

void fsdp_raise(const at::Tensor& peer_base, int64_t flag_off, int64_t row, int64_t rank, int64_t world,
                int64_t epoch) {
  TORCH_CHECK(peer_base.is_cuda() && peer_base.scalar_type() == at::kLong && peer_base.numel() == world,
              "fsdp_raise: peer_base int64 [world]");
  TORCH_CHECK(flag_off % 4 == 0 && row >= 0 && rank >= 0 && rank < world, "fsdp_raise: bad arguments");
  const c10::cuda::CUDAGuard g(peer_base.device());
  astrai_host::fsdp_raise(reinterpret_cast<const long long*>(peer_base.data_ptr<int64_t>()), flag_off,
                          static_cast<int>(row), static_cast<int>(rank), static_cast<int>(world),
                          static_cast<unsigned>(epoch), at::cuda::getCurrentCUDAStream().stream());
}

}  // namespace

// Row-parallel all-reduce, second half: sum this rank's rows of the partial products (own partial
// at part_addr, peers' in the receive slots at recv_addr) and store the result into every rank's
// output (out_addr + rank_deltas[q]); the last CTA raises flag_addr on every peer.
static void row_reduce_bcast(int64_t part_addr, int64_t recv_addr, int64_t out_addr, int64_t ld, int64_t M, int64_t N,
                      int64_t rank, int64_t world, int64_t rpo, const std::vector<int64_t>& rank_deltas,
                      int64_t flag_addr, int64_t epoch, int64_t done_addr, int64_t device) {
  TORCH_CHECK((int64_t)rank_deltas.size() == world && world >= 1 && world <= 8, "row_reduce_bcast: one delta per rank");
  TORCH_CHECK(part_addr % 16 == 0 && recv_addr % 16 == 0 && out_addr % 16 == 0 && N % 8 == 0 && ld % 8 == 0,
              "row_reduce_bcast: 16-byte aligned rows");
  std::vector<long long> d(rank_deltas.begin(), rank_deltas.end());
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  astrai_host::row_reduce_bcast(reinterpret_cast<const void*>(part_addr), reinterpret_cast<const void*>(recv_addr),
                                reinterpret_cast<void*>(out_addr), ld, (int)M, (int)N, (int)rank, (int)world, (int)rpo,
                                d.data(), reinterpret_cast<unsigned*>(flag_addr), (unsigned)epoch,
                                reinterpret_cast<unsigned*>(done_addr), astrai_host::num_sms((int)device),
                                at::cuda::getCurrentCUDAStream().stream());
}

void register_comm(pybind11::module& m) {
  m.def("row_reduce_bcast", &row_reduce_bcast);
  m.def("muon_apply_peers", &muon_apply_peers);
  m.def("peer_flags_wait", &peer_flags_wait);
  m.def("fsdp_reduce", &fsdp_reduce);
  m.def("fsdp_raise", &fsdp_raise);
  m.def("peer_copy", &peer_copy);
  m.def("symm_alloc", &symm_alloc, "cudaMalloc + IPC handle -> (address, 64-byte handle)");
  m.def("symm_open", &symm_open, "map a peer's IPC handle -> address");
  m.def("symm_close", [](int64_t p) { astrai_host::symm_close(reinterpret_cast<void*>(p)); });
  m.def("symm_free", [](int64_t p) { astrai_host::symm_free(reinterpret_cast<void*>(p)); });
  m.def("fused_allreduce", &fused_allreduce, pybind11::arg("seg_ptr"), pybind11::arg("seg_off"), pybind11::arg("N"),
        pybind11::arg("rank"), pybind11::arg("world"), pybind11::arg("R"), pybind11::arg("peer_base"),
        pybind11::arg("off_flag_a"), pybind11::arg("off_flag_b"), pybind11::arg("off_sumsq"),
        pybind11::arg("off_recv"), pybind11::arg("off_gather"), pybind11::arg("epoch0"), pybind11::arg("ctas"),
        pybind11::arg("sumsq_out"), pybind11::arg("clip_coef"), pybind11::arg("max_norm"), pybind11::arg("done"),
        pybind11::arg("wait_s") = 20.0);
}
