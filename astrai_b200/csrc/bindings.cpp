// Python bindings of the astrai_b200 CUDA kernels.
//
// The .cu files are torch-free (raw pointers + cudaStream_t); this file owns
// every tensor check (device, dtype, contiguity of the innermost dimension,
// 16-byte alignment required by TMA and vector loads) and passes the current
// PyTorch stream, so all kernels order correctly with the rest of autograd.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_runtime.h>

namespace astrai_host {
long long launch_count();
void add_launches(long long n);
void skinny_gemm(const void* X, long long ldx, const void* W, long long ldw, const void* residual, long long ldr,
                 void* Y, long long ldy, int M, int N, int K, int sms, cudaStream_t s);
int num_sms(int device);
int read_and_clear_error();
struct GatherArgs {
  int npeers;
  long long peer_delta[7];
  unsigned* flag;
  unsigned* done;
  unsigned epoch;
  int scatter_rpo, scatter_rank;
  long long scatter_recv_off;
  long long rank_delta[8];
};
void gemm_bf16(const void* A, const void* B, void* D, const void* C, int M, int N, int K, int batch, int a_mn,
               long long lda, long long strideA, int b_mn, long long ldb, long long strideB, long long ldd,
               long long strideD, int out_f32, long long ldc, long long strideC, float alpha, float beta,
               int force_bn, cudaStream_t stream, const GatherArgs* gather = nullptr, int sym = 0);
void gemm_profile_set(unsigned long long* counters);
void gemm_plan(int M, int N, int K, int batch, int* out);
void gemm_rope_bf16(const void* A, long long lda, const void* B, long long ldb, void* D, long long ldd, int M, int N,
                    int K, const void* cs, const int* pos, int seq, int rope_cols, int head_dim, int max_pos,
                    cudaStream_t stream);
void gemm_swiglu_bf16(int mode, const void* A, long long lda, const void* B, long long ldb, int b_mn, void* D,
                      long long ldd, void* aux, long long ldaux, const void* h, long long ldh, int M, int F, int K,
                      cudaStream_t stream);
void rmsnorm_fwd(const void* x, long long ldx, const void* w, void* y, long long ldy, float* rstd, int rows, int D,
                 float eps, cudaStream_t s);
long long rmsnorm_bwd_scratch(int rows, int D, int* nblocks_out);
void rmsnorm_bwd(const void* dy, long long lddy, const void* x, long long ldx, const void* w, const float* rstd,
                 void* dx, long long lddx, void* dw_bf16, float* dw_f32, float* scratch, int rows, int D,
                 cudaStream_t s, const void* dres = nullptr, long long ldres = 0);
void rope_apply(void* x, long long ld, int rows, int col0, int n_heads, int head_dim, const int* pos, int seq_len,
                const void* cs, int inverse, int rot_dim, int rot_off, int max_pos, cudaStream_t s);
void swiglu_fwd(const void* h, long long ldh, void* out, long long ldo, int rows, int F, const int* live_rows,
                cudaStream_t s);
void swiglu_bwd(const void* dy, long long lddy, const void* h, long long ldh, void* dh, long long lddh, int rows, int F,
                const int* live_rows, cudaStream_t s);
void embedding_fwd(const long long* ids, const void* w, void* out, int n_tok, int d, int vocab, cudaStream_t s);
void embedding_bwd(const long long* ids, const void* g, float* gw, int n_tok, int d, int vocab, cudaStream_t s);
void f32_to_bf16(const float* in, void* out, long long n, int accumulate, cudaStream_t s);
void transpose_bf16(const void* in, void* out, int batch, int R, int C, cudaStream_t s);
void ce_fwd(const void* logits, long long ld, const long long* target, int rows, int V, float smoothing,
            long long ignore_index, int mode, float* lse, float* out, cudaStream_t s);
void ce_bwd(const void* logits, long long ld, const long long* target, int rows, int V, float smoothing,
            long long ignore_index, int mode, const float* lse, const float* gscale, const float* grow,
            void* dlogits, long long ldd, cudaStream_t s);
void grad_sumsq(const void* chunks, int n_chunks, const long long* gptr, const int* group, float* acc, cudaStream_t s);
void clip_coef(const float* acc, int n, float max_norm, float* coef, float* norm_out, cudaStream_t s);
void adamw_step(const void* chunks, int n_chunks, const long long* pptr, const long long* gptr, const long long* mptr,
                const long long* vptr, const float* wd, int fp32_params, float lr, float b1, float b2, float eps,
                float bc1, float bc2, const float* coef, cudaStream_t s);
void muon_momentum(const long long* gptr, const long long* bufptr, int buf_fp32, void* U, int batch, long long numel,
                   float mu, int nesterov, const float* coef, float* sumsq, cudaStream_t s);
void muon_normalize(const void* U, void* X, int batch, int R, int C, int transpose, const float* sumsq, float eps,
                    cudaStream_t s);
void muon_apply(const long long* pptr, int fp32_params, const void* X, int batch, int R, int C, int transpose,
                float decay, float adj_lr, cudaStream_t s);
}  // namespace astrai_host

namespace {

#define I64(t) reinterpret_cast<const long long*>((t).data_ptr<int64_t>())

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}
void check_rows(const at::Tensor& t, const char* name) {
  // 2-D view with unit inner stride and 16-byte aligned row stride / base
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have a contiguous inner dimension");
  TORCH_CHECK((t.stride(0) * t.element_size()) % 16 == 0, name, ": row stride must be a multiple of 16 bytes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

// ----------------------------------------------------------------- skinny GEMM (decode)
// y [M, N] = x [M, K] @ w [N, K]^T (+ residual), 1 <= M <= 16.
void skinny_gemm(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& residual) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(y, "y");
  check_rows(x, "x");
  check_rows(w, "w");
  TORCH_CHECK(y.dim() == 2 && y.stride(1) == 1, "y must be 2-D rows");  // scalar stores: any row stride
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)w.size(0);
  TORCH_CHECK(w.size(1) == K && y.size(0) == M && y.size(1) == N, "skinny_gemm: shape mismatch");
  const void* r = nullptr;
  long long ldr = 0;
  if (residual.has_value() && residual->defined()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->dim() == 2 && residual->size(0) == M && residual->size(1) == N &&
                    residual->stride(1) == 1, "residual must be [M, N] rows");
    r = residual->data_ptr();
    ldr = residual->stride(0);
  }
  c10::cuda::CUDAGuard g(x.device());
  astrai_host::skinny_gemm(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), r, ldr, y.data_ptr(), y.stride(0), M, N,
                           K, astrai_host::num_sms(x.device().index()), stream());
}

// ----------------------------------------------------------------- GEMM
// D = alpha * op(A) op(B)^T + beta * C over 2-D or batched 3-D operands.
// SwiGLU GEMMs (2-D, bf16):
//   mode 1: x [M, K] @ w_ug [2F, K]^T -> h [M, 2F] and a = silu(g) * u [M, F] (out);  h_saved unused
//   mode 2: dy [M, K] @ W_down^T (w: [K, F] = W_down's storage [out=K][in=F], read MN-major) with the
//           saved h [M, 2F] -> dh [M, 2F] (out); the product da is never stored
void gemm_swiglu(int64_t mode, const at::Tensor& a, const at::Tensor& w, const c10::optional<at::Tensor>& h_out,
                 at::Tensor& out, const c10::optional<at::Tensor>& h_saved) {
  check_bf16(a, "a");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(a.dim() == 2 && w.dim() == 2 && out.dim() == 2, "gemm_swiglu: 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_swiglu: contiguous rows");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "gemm_swiglu: 16-byte row strides");
  const int M = (int)a.size(0), K = (int)a.size(1);
  c10::cuda::CUDAGuard g(a.device());
  if (mode == 1) {
    // h_out None: only a = silu(g) * u is stored (inference; the backward needs h)
    const bool has_h = h_out.has_value() && h_out->defined();
    if (has_h) check_bf16(*h_out, "h_out");
    const int F = (int)w.size(0) / 2;
    TORCH_CHECK(w.size(0) == 2 * F && w.size(1) == K && out.size(0) == M && out.size(1) == F &&
                    (!has_h || (h_out->size(0) == M && h_out->size(1) == 2 * F && h_out->stride(1) == 1)),
                "gemm_swiglu mode 1: shapes x [M, K], w [2F, K], h [M, 2F] (or None), a [M, F]");
    astrai_host::gemm_swiglu_bf16(1, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), 0,
                                  has_h ? h_out->data_ptr() : nullptr, has_h ? h_out->stride(0) : 0, out.data_ptr(),
                                  out.stride(0), nullptr, 0, M, F, K, stream());
  } else {
    TORCH_CHECK(mode == 2 && h_saved.has_value() && h_saved->defined(), "gemm_swiglu mode 2 needs h_saved");
    check_bf16(*h_saved, "h_saved");
    const int F = (int)w.size(1);
    TORCH_CHECK(w.size(0) == K && h_saved->size(0) == M && h_saved->size(1) == 2 * F && out.size(0) == M &&
                    out.size(1) == 2 * F && h_saved->stride(1) == 1,
                "gemm_swiglu mode 2: shapes dy [M, K], w [K, F], h [M, 2F], dh [M, 2F]");
    astrai_host::gemm_swiglu_bf16(2, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), 1, nullptr, 0,
                                  out.data_ptr(), out.stride(0), h_saved->data_ptr(), h_saved->stride(0), M, F, K,
                                  stream());
  }
}

// out [M, N] = x [M, K] @ w [N, K]^T with RoPE on columns [0, rope_cols) (heads of head_dim columns):
// the row's position is positions[row] (int32) or row % seq_len; table is fp32 [max_pos, head_dim/2, 2].
void gemm_rope(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const at::Tensor& table,
               const c10::optional<at::Tensor>& positions, int64_t seq_len, int64_t rope_cols, int64_t head_dim) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 &&
                  out.stride(1) == 1, "gemm_rope: 2-D operands with contiguous rows");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "gemm_rope: 16-byte row strides");
  TORCH_CHECK(w.size(1) == x.size(1) && out.size(0) == x.size(0) && out.size(1) == w.size(0), "gemm_rope: shapes");
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kFloat && table.is_contiguous(), "rope table");
  const int* pos = nullptr;
  if (positions.has_value() && positions->defined()) {
    TORCH_CHECK(positions->scalar_type() == at::kInt && positions->is_contiguous() &&
                    positions->numel() == x.size(0), "positions: int32, one per row");
    pos = positions->data_ptr<int>();
  }
  const int64_t max_pos = table.numel() / head_dim;
  c10::cuda::CUDAGuard g(x.device());
  astrai_host::gemm_rope_bf16(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
                              (int)x.size(0), (int)w.size(0), (int)x.size(1), table.data_ptr(), pos, (int)seq_len,
                              (int)rope_cols, (int)head_dim, (int)max_pos, stream());
}

//   a: [.., M, K] when a_mn == 0, [.., K, M] when a_mn == 1
//   b: [.., N, K] when b_mn == 0, [.., K, N] when b_mn == 1
void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& d, const c10::optional<at::Tensor>& c, int64_t a_mn,
          int64_t b_mn, double alpha, double beta, int64_t force_bn, bool sym) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_cuda(d, "d");
  TORCH_CHECK(d.scalar_type() == at::kBFloat16 || d.scalar_type() == at::kFloat, "d must be bf16 or fp32");
  TORCH_CHECK(a.dim() == b.dim() && a.dim() == d.dim() && (a.dim() == 2 || a.dim() == 3), "rank mismatch");
  const bool batched = a.dim() == 3;
  const int batch = batched ? (int)a.size(0) : 1;
  const int ar = batched ? 1 : 0;
  const long long M = a_mn ? a.size(ar + 1) : a.size(ar);
  const long long K = a_mn ? a.size(ar) : a.size(ar + 1);
  const long long N = b_mn ? b.size(ar + 1) : b.size(ar);
  const long long Kb = b_mn ? b.size(ar) : b.size(ar + 1);
  TORCH_CHECK(K == Kb, "gemm: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(d.size(ar) == M && d.size(ar + 1) == N, "gemm: output shape mismatch");
  TORCH_CHECK(a.stride(ar + 1) == 1 && b.stride(ar + 1) == 1 && d.stride(ar + 1) == 1,
              "gemm: operands need a contiguous inner dimension");
  TORCH_CHECK((a.stride(ar) * 2) % 16 == 0 && (b.stride(ar) * 2) % 16 == 0, "gemm: row strides must be 16B multiples");
  if (batched) TORCH_CHECK(b.size(0) == batch && d.size(0) == batch, "gemm: batch mismatch");
  const void* cptr = nullptr;
  long long ldc = 0, sc = 0;
  if (c.has_value() && c->defined()) {
    TORCH_CHECK(c->scalar_type() == d.scalar_type(), "gemm: c must match d dtype");
    TORCH_CHECK(c->sizes() == d.sizes() && c->stride(ar + 1) == 1, "gemm: c shape mismatch");
    cptr = c->data_ptr();
    ldc = c->stride(ar);
    sc = batched ? c->stride(0) : 0;
  }
  c10::cuda::CUDAGuard g(a.device());
  astrai_host::gemm_bf16(a.data_ptr(), b.data_ptr(), d.data_ptr(), cptr, (int)M, (int)N, (int)K, batch, (int)a_mn,
                         a.stride(ar), batched ? a.stride(0) : 0, (int)b_mn, b.stride(ar), batched ? b.stride(0) : 0,
                         d.stride(ar), batched ? d.stride(0) : 0, d.scalar_type() == at::kFloat ? 1 : 0, ldc, sc,
                         (float)alpha, (float)beta, (int)force_bn, stream(), nullptr, sym ? 1 : 0);
}

// GEMM fused with an all-gather over NVLink peer memory: d is this rank's column block of the
// gathered output inside a symmetric buffer; the epilogue also stores every output vector into each
// peer's copy (d + peer_deltas[q] bytes) and the last CTA raises this rank's flag on every peer
// (flag_addr + peer_deltas[q] <- epoch). The caller waits for the peers' flags.
void gemm_gather(const at::Tensor& a, const at::Tensor& b, at::Tensor& d, const std::vector<int64_t>& peer_deltas,
                 int64_t flag_addr, int64_t done_addr, int64_t epoch, int64_t a_mn, int64_t b_mn,
                 int64_t scatter_rpo, int64_t scatter_rank, int64_t scatter_recv_off,
                 const std::vector<int64_t>& rank_deltas) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(d, "d");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && d.dim() == 2, "gemm_gather: 2-D operands");
  TORCH_CHECK(peer_deltas.size() <= 7, "gemm_gather: at most 7 peers");
  TORCH_CHECK(flag_addr % 4 == 0 && done_addr % 4 == 0 && flag_addr != 0 && done_addr != 0, "gemm_gather: flags");
  const long long M = a_mn ? a.size(1) : a.size(0);
  const long long K = a_mn ? a.size(0) : a.size(1);
  const long long N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm_gather: K mismatch");
  TORCH_CHECK(d.size(0) == M && d.size(1) == N && d.stride(1) == 1, "gemm_gather: output shape");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && (a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0,
              "gemm_gather: operands need contiguous rows with 16-byte strides");
  astrai_host::GatherArgs g{};
  g.npeers = (int)peer_deltas.size();
  for (size_t q = 0; q < peer_deltas.size(); ++q) g.peer_delta[q] = peer_deltas[q];
  g.flag = reinterpret_cast<unsigned*>(flag_addr);
  g.done = reinterpret_cast<unsigned*>(done_addr);
  g.epoch = (unsigned)epoch;
  g.scatter_rpo = (int)scatter_rpo;
  g.scatter_rank = (int)scatter_rank;
  g.scatter_recv_off = scatter_recv_off;
  if (scatter_rpo > 0) {
    TORCH_CHECK(rank_deltas.size() == peer_deltas.size() + 1 && scatter_rank >= 0 &&
                    scatter_rank < (int64_t)rank_deltas.size() && d.is_contiguous(),
                "gemm_gather: reduce-scatter push needs one delta per rank and a contiguous partial");
    for (size_t q = 0; q < rank_deltas.size(); ++q) g.rank_delta[q] = rank_deltas[q];
  }
  c10::cuda::CUDAGuard guard(a.device());
  astrai_host::gemm_bf16(a.data_ptr(), b.data_ptr(), d.data_ptr(), nullptr, (int)M, (int)N, (int)K, 1, (int)a_mn,
                         a.stride(0), 0, (int)b_mn, b.stride(0), 0, d.stride(0), 0, 0, 0, 0, 1.f, 0.f, 0, stream(),
                         &g);
}

// ----------------------------------------------------------------- RMSNorm
void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, c10::optional<at::Tensor> rstd, double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(y, "y");
  check_rows(x, "x");
  check_rows(y, "y");
  const int D = (int)x.size(1);
  TORCH_CHECK(w.numel() == D && w.is_contiguous(), "w shape");
  TORCH_CHECK(D % 8 == 0 && D <= 8192 && (D <= 256 ? D % 32 == 0 : true), "rmsnorm: unsupported width ", D);
  float* r = nullptr;
  if (rstd.has_value() && rstd->defined()) {
    TORCH_CHECK(rstd->scalar_type() == at::kFloat && rstd->numel() == x.size(0), "rstd");
    r = rstd->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(x.device());
  astrai_host::rmsnorm_fwd(x.data_ptr(), x.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), r, (int)x.size(0), D,
                           (float)eps, stream());
}

int64_t rmsnorm_bwd_scratch(int64_t rows, int64_t D) { return astrai_host::rmsnorm_bwd_scratch((int)rows, (int)D, nullptr); }

// dres (optional): gradient of a second use of x (the residual branch), added into dx by the kernel.
void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd, at::Tensor& dx,
                 at::Tensor& dw, at::Tensor& scratch, const c10::optional<at::Tensor>& dres) {
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  check_bf16(dx, "dx");
  check_rows(dy, "dy");
  check_rows(x, "x");
  check_rows(dx, "dx");
  const int D = (int)x.size(1);
  TORCH_CHECK(D % 8 == 0 && D <= 4096, "rmsnorm_bwd: D must be a multiple of 8 and at most 4096");
  TORCH_CHECK(scratch.scalar_type() == at::kFloat && scratch.numel() >= rmsnorm_bwd_scratch(x.size(0), D), "scratch");
  const void* dr = nullptr;
  long long ldr = 0;
  if (dres.has_value() && dres->defined()) {
    check_bf16(*dres, "dres");
    check_rows(*dres, "dres");
    TORCH_CHECK(dres->sizes() == x.sizes(), "rmsnorm_bwd: dres must have the shape of x");
    dr = dres->data_ptr();
    ldr = dres->stride(0);
  }
  c10::cuda::CUDAGuard g(x.device());
  astrai_host::rmsnorm_bwd(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), w.data_ptr(),
                           rstd.data_ptr<float>(), dx.data_ptr(), dx.stride(0),
                           dw.scalar_type() == at::kBFloat16 ? dw.data_ptr() : nullptr,
                           dw.scalar_type() == at::kFloat ? dw.data_ptr<float>() : nullptr, scratch.data_ptr<float>(),
                           (int)x.size(0), D, stream(), dr, ldr);
}

// ----------------------------------------------------------------- RoPE / SwiGLU / embedding
void rope_(at::Tensor& x, int64_t col0, int64_t n_heads, int64_t head_dim, const c10::optional<at::Tensor>& pos,
           int64_t seq_len, const at::Tensor& cs, bool inverse, int64_t rot_dim, int64_t rot_off) {
  check_bf16(x, "x");
  check_rows(x, "x");
  TORCH_CHECK(cs.scalar_type() == at::kFloat && cs.is_contiguous() && cs.is_cuda() &&
                  reinterpret_cast<uintptr_t>(cs.data_ptr()) % 16 == 0,
              "cos/sin table: contiguous CUDA fp32, 16-byte aligned (the kernel reads it as float4)");
  TORCH_CHECK(rot_dim % 8 == 0 && (col0 + rot_off) % 8 == 0 && head_dim % 8 == 0, "rope: alignment");
  const int* p = nullptr;
  if (pos.has_value() && pos->defined()) {
    TORCH_CHECK(pos->scalar_type() == at::kInt && pos->is_contiguous() && pos->numel() == x.size(0), "positions");
    p = pos->data_ptr<int>();
  }
  const int64_t max_pos = cs.numel() / rot_dim;  // [max_pos][rot_dim / 2] (cos, sin) pairs
  TORCH_CHECK(p != nullptr || seq_len <= max_pos, "rope: sequence longer than the position table");
  c10::cuda::CUDAGuard g(x.device());
  astrai_host::rope_apply(x.data_ptr(), x.stride(0), (int)x.size(0), (int)col0, (int)n_heads, (int)head_dim, p,
                          (int)seq_len, cs.data_ptr(), inverse ? 1 : 0, (int)rot_dim, (int)rot_off, (int)max_pos,
                          stream());
}

const int* live_ptr(const c10::optional<at::Tensor>& live) {
  if (!live.has_value()) return nullptr;
  TORCH_CHECK(live->is_cuda() && live->scalar_type() == at::kInt && live->numel() == 1, "live_rows: CUDA int32 [1]");
  return live->data_ptr<int>();
}

// live_rows (optional CUDA int32 [1]): only that many leading rows are processed
void swiglu_fwd(const at::Tensor& h, at::Tensor& out, const c10::optional<at::Tensor>& live_rows) {
  check_bf16(h, "h");
  check_bf16(out, "out");
  check_rows(h, "h");
  check_rows(out, "out");
  const int F = (int)out.size(1);
  TORCH_CHECK(h.size(1) == 2 * F && F % 8 == 0, "swiglu: h must be [rows, 2F] with F % 8 == 0");
  c10::cuda::CUDAGuard g(h.device());
  astrai_host::swiglu_fwd(h.data_ptr(), h.stride(0), out.data_ptr(), out.stride(0), (int)h.size(0), F,
                          live_ptr(live_rows), stream());
}

void swiglu_bwd(const at::Tensor& dy, const at::Tensor& h, at::Tensor& dh,
                const c10::optional<at::Tensor>& live_rows) {
  check_bf16(dy, "dy");
  check_bf16(h, "h");
  check_bf16(dh, "dh");
  check_rows(dy, "dy");
  check_rows(h, "h");
  check_rows(dh, "dh");
  const int F = (int)dy.size(1);
  c10::cuda::CUDAGuard g(h.device());
  astrai_host::swiglu_bwd(dy.data_ptr(), dy.stride(0), h.data_ptr(), h.stride(0), dh.data_ptr(), dh.stride(0),
                          (int)h.size(0), F, live_ptr(live_rows), stream());
}

void embedding_fwd(const at::Tensor& ids, const at::Tensor& w, at::Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.is_cuda(), "ids");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(w.is_contiguous() && out.is_contiguous() && w.size(1) % 8 == 0, "embedding layout");
  c10::cuda::CUDAGuard g(w.device());
  astrai_host::embedding_fwd(I64(ids), w.data_ptr(), out.data_ptr(), (int)ids.numel(), (int)w.size(1),
                             (int)w.size(0), stream());
}

void embedding_bwd(const at::Tensor& ids, const at::Tensor& grad, at::Tensor& gw_f32) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids");
  check_bf16(grad, "grad");
  TORCH_CHECK(gw_f32.scalar_type() == at::kFloat && gw_f32.is_contiguous() && grad.is_contiguous(), "layout");
  c10::cuda::CUDAGuard g(grad.device());
  astrai_host::embedding_bwd(I64(ids), grad.data_ptr(), gw_f32.data_ptr<float>(), (int)ids.numel(),
                             (int)gw_f32.size(1), (int)gw_f32.size(0), stream());
}

void f32_to_bf16(const at::Tensor& in, at::Tensor& out, bool accumulate) {
  TORCH_CHECK(in.scalar_type() == at::kFloat && in.is_contiguous() && out.is_contiguous(), "layout");
  check_bf16(out, "out");
  TORCH_CHECK(in.numel() == out.numel(), "numel");
  c10::cuda::CUDAGuard g(in.device());
  astrai_host::f32_to_bf16(in.data_ptr<float>(), out.data_ptr(), in.numel(), accumulate ? 1 : 0, stream());
}

void transpose_bf16(const at::Tensor& in, at::Tensor& out) {
  check_bf16(in, "in");
  check_bf16(out, "out");
  TORCH_CHECK(in.is_contiguous() && out.is_contiguous() && in.dim() == 3, "transpose: contiguous [B,R,C]");
  c10::cuda::CUDAGuard g(in.device());
  astrai_host::transpose_bf16(in.data_ptr(), out.data_ptr(), (int)in.size(0), (int)in.size(1), (int)in.size(2),
                              stream());
}

// ----------------------------------------------------------------- cross entropy
void ce_fwd(const at::Tensor& logits, const at::Tensor& target, double smoothing, int64_t ignore_index, int64_t mode,
            at::Tensor& lse, at::Tensor& out) {
  check_bf16(logits, "logits");
  check_rows(logits, "logits");
  TORCH_CHECK(target.scalar_type() == at::kLong && target.is_contiguous() && target.numel() == logits.size(0), "target");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat, "lse/out must be fp32");
  c10::cuda::CUDAGuard g(logits.device());
  astrai_host::ce_fwd(logits.data_ptr(), logits.stride(0), I64(target), (int)logits.size(0),
                      (int)logits.size(1), (float)smoothing, ignore_index, (int)mode, lse.data_ptr<float>(),
                      out.data_ptr<float>(), stream());
}

void ce_bwd(const at::Tensor& logits, const at::Tensor& target, double smoothing, int64_t ignore_index, int64_t mode,
            const at::Tensor& lse, const c10::optional<at::Tensor>& gscale, const c10::optional<at::Tensor>& grow,
            at::Tensor& dlogits) {
  check_bf16(logits, "logits");
  check_bf16(dlogits, "dlogits");
  check_rows(logits, "logits");
  check_rows(dlogits, "dlogits");
  const float* gs = (gscale.has_value() && gscale->defined()) ? gscale->data_ptr<float>() : nullptr;
  const float* gr = (grow.has_value() && grow->defined()) ? grow->data_ptr<float>() : nullptr;
  TORCH_CHECK(mode == 0 ? gs != nullptr : gr != nullptr, "ce_bwd: missing gradient input");
  c10::cuda::CUDAGuard g(logits.device());
  astrai_host::ce_bwd(logits.data_ptr(), logits.stride(0), I64(target), (int)logits.size(0),
                      (int)logits.size(1), (float)smoothing, ignore_index, (int)mode, lse.data_ptr<float>(), gs, gr,
                      dlogits.data_ptr(), dlogits.stride(0), stream());
}

// ----------------------------------------------------------------- optimizer
void grad_sumsq(const at::Tensor& chunks, const at::Tensor& gptr, const c10::optional<at::Tensor>& group,
                at::Tensor& acc) {
  const int n = (int)(chunks.numel() * chunks.element_size() / 16);
  c10::cuda::CUDAGuard g(acc.device());
  astrai_host::grad_sumsq(chunks.data_ptr(), n, I64(gptr),
                          (group.has_value() && group->defined()) ? group->data_ptr<int>() : nullptr,
                          acc.data_ptr<float>(), stream());
}

void clip_coef(const at::Tensor& acc, double max_norm, at::Tensor& coef, at::Tensor& norm_out) {
  c10::cuda::CUDAGuard g(acc.device());
  astrai_host::clip_coef(acc.data_ptr<float>(), (int)acc.numel(), (float)max_norm, coef.data_ptr<float>(),
                         norm_out.data_ptr<float>(), stream());
}

void adamw_step(const at::Tensor& chunks, const at::Tensor& pptr, const at::Tensor& gptr, const at::Tensor& mptr,
                const at::Tensor& vptr, const at::Tensor& wd, bool fp32_params, double lr, double b1, double b2,
                double eps, double bc1, double bc2, const c10::optional<at::Tensor>& coef) {
  const int n = (int)(chunks.numel() * chunks.element_size() / 16);
  c10::cuda::CUDAGuard g(pptr.device());
  astrai_host::adamw_step(chunks.data_ptr(), n, I64(pptr), I64(gptr),
                          I64(mptr), I64(vptr), wd.data_ptr<float>(), fp32_params ? 1 : 0,
                          (float)lr, (float)b1, (float)b2, (float)eps, (float)bc1, (float)bc2,
                          (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr, stream());
}

void muon_momentum(const at::Tensor& gptr, const at::Tensor& bufptr, bool buf_fp32, at::Tensor& U, double mu,
                   bool nesterov, const c10::optional<at::Tensor>& coef, at::Tensor& sumsq) {
  check_bf16(U, "U");
  TORCH_CHECK(U.dim() == 3 && U.is_contiguous(), "U must be contiguous [B, R, C]");
  c10::cuda::CUDAGuard g(U.device());
  astrai_host::muon_momentum(I64(gptr), I64(bufptr), buf_fp32 ? 1 : 0, U.data_ptr(),
                             (int)U.size(0), U.size(1) * U.size(2), (float)mu, nesterov ? 1 : 0,
                             (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr,
                             sumsq.data_ptr<float>(), stream());
}

void muon_normalize(const at::Tensor& U, at::Tensor& X, bool transpose, const at::Tensor& sumsq, double eps) {
  c10::cuda::CUDAGuard g(U.device());
  astrai_host::muon_normalize(U.data_ptr(), X.data_ptr(), (int)U.size(0), (int)U.size(1), (int)U.size(2),
                              transpose ? 1 : 0, sumsq.data_ptr<float>(), (float)eps, stream());
}

void muon_apply(const at::Tensor& pptr, bool fp32_params, const at::Tensor& X, int64_t R, int64_t C, bool transpose,
                double decay, double adj_lr) {
  c10::cuda::CUDAGuard g(X.device());
  astrai_host::muon_apply(I64(pptr), fp32_params ? 1 : 0, X.data_ptr(), (int)X.size(0), (int)R, (int)C,
                          transpose ? 1 : 0, (float)decay, (float)adj_lr, stream());
}

int64_t num_sms(int64_t device) { return astrai_host::num_sms((int)device); }
int64_t read_error() { return astrai_host::read_and_clear_error(); }

}  // namespace

void register_attention(pybind11::module& m);
void register_inference(pybind11::module& m);
void register_moe(pybind11::module& m);
void register_comm(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "astrai_b200 sm_100a kernels";
  m.def("launch_count", []() { return static_cast<int64_t>(astrai_host::launch_count()); },
        "kernel launches issued by this library so far (host counter)");
  m.def("add_launches", [](int64_t n) { astrai_host::add_launches(n); },
        "count kernels that ran from a CUDA-graph replay (captured launches x replays)");
  m.def("skinny_gemm", &skinny_gemm, py::arg("x"), py::arg("w"), py::arg("y"), py::arg("residual") = py::none());
  m.def("gemm", &gemm, "bf16 tcgen05 GEMM", py::arg("a"), py::arg("b"), py::arg("d"), py::arg("c") = py::none(),
        py::arg("a_mn") = 0, py::arg("b_mn") = 0, py::arg("alpha") = 1.0, py::arg("beta") = 0.0,
        py::arg("force_bn") = 0, py::arg("sym") = false);
  m.def("gemm_gather", &gemm_gather, "bf16 GEMM whose epilogue also stores into every peer's copy (fused all-gather)",
        py::arg("a"), py::arg("b"), py::arg("d"), py::arg("peer_deltas"), py::arg("flag_addr"), py::arg("done_addr"),
        py::arg("epoch"), py::arg("a_mn") = 0, py::arg("b_mn") = 0, py::arg("scatter_rpo") = 0,
        py::arg("scatter_rank") = 0, py::arg("scatter_recv_off") = 0,
        py::arg("rank_deltas") = std::vector<int64_t>{});
  m.def("gemm_plan", [](int64_t M, int64_t N, int64_t K, int64_t batch) {
    int o[7] = {0, 0, 0, 0, 0, 0, 0};
    astrai_host::gemm_plan((int)M, (int)N, (int)K, (int)batch, o);
    return py::make_tuple(o[0], o[1], (bool)o[2], o[3], o[4], (bool)o[5], (bool)o[6]);
  }, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("batch") = 1);
  m.def("gemm_profile_set", [](const c10::optional<at::Tensor>& counters) {
    // int64 [4] CUDA tensor that later GEMM launches add their wait cycles to, or None (off)
    if (counters.has_value() && counters->defined()) {
      TORCH_CHECK(counters->is_cuda() && counters->scalar_type() == at::kLong && counters->numel() >= 4,
                  "counters: CUDA int64 [4]");
      astrai_host::gemm_profile_set(reinterpret_cast<unsigned long long*>(counters->data_ptr<int64_t>()));
    } else {
      astrai_host::gemm_profile_set(nullptr);
    }
  });
  m.def("gemm_rope", &gemm_rope, "GEMM with RoPE applied in the epilogue", py::arg("x"), py::arg("w"),
        py::arg("out"), py::arg("table"), py::arg("positions"), py::arg("seq_len"), py::arg("rope_cols"),
        py::arg("head_dim"));
  m.def("gemm_swiglu", &gemm_swiglu, "GEMM with a fused SwiGLU epilogue (mode 1 forward, mode 2 backward)",
        py::arg("mode"), py::arg("a"), py::arg("w"), py::arg("h_out"), py::arg("out"), py::arg("h_saved"));
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd_scratch", &rmsnorm_bwd_scratch);
  m.def("rmsnorm_bwd", &rmsnorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dx"),
        py::arg("dw"), py::arg("scratch"), py::arg("dres") = py::none());
  m.def("rope_", &rope_);
  m.def("swiglu_fwd", &swiglu_fwd, pybind11::arg("h"), pybind11::arg("out"), pybind11::arg("live_rows") = pybind11::none());
  m.def("swiglu_bwd", &swiglu_bwd, pybind11::arg("dy"), pybind11::arg("h"), pybind11::arg("dh"),
        pybind11::arg("live_rows") = pybind11::none());
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("f32_to_bf16", &f32_to_bf16);
  m.def("transpose_bf16", &transpose_bf16);
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd", &ce_bwd);
  m.def("grad_sumsq", &grad_sumsq);
  m.def("clip_coef", &clip_coef);
  m.def("adamw_step", &adamw_step);
  m.def("muon_momentum", &muon_momentum);
  m.def("muon_normalize", &muon_normalize);
  m.def("muon_apply", &muon_apply);
  m.def("num_sms", &num_sms);
  m.def("read_error", &read_error);
  register_attention(m);
  register_inference(m);
  register_moe(m);
  register_comm(m);
}
