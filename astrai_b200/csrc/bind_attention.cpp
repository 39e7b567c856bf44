// Python bindings for the tcgen05 flash-attention kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

namespace astrai_host {
void flash_fwd(const void* q, long long ldq, int q_col0, const void* k, long long ldk, int k_col0, const void* v,
               long long ldv, int v_col0, void* o, long long ldo, float* lse, int B, int Sq, int Sk, int Hq, int Hkv,
               float scale, int causal, const int* seg, cudaStream_t s);
void flash_fwd_pair(const void* q, long long ldq, int q_col0, const void* k, long long ldk, int k_col0, const void* v,
                    long long ldv, int v_col0, void* o, long long ldo, float* lse, int B, int Sq, int Sk, int Hq,
                    int Hkv, int D, float scale, int causal, const int* seg, cudaStream_t s);
void flash_bwd(const void* q, long long ldq, int q_col0, const void* k, long long ldk, int k_col0, const void* v,
               long long ldv, int v_col0, const void* o, long long ldo, const void* dO, long long ld_do, int do_col0,
               const float* lse, float* delta, float* dq_acc, void* dq, long long ld_dq, int dq_col0, void* dk,
               void* dv, long long ld_dkv, int dk_col0, int dv_col0, int B, int Sq, int Sk, int Hq, int Hkv,
               float scale, int causal, const int* seg, cudaStream_t s);
}  // namespace astrai_host

namespace {

void check_buf(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a bf16 CUDA tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D [tokens, cols] with contiguous columns");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " needs 16-byte aligned rows");
}

const int* seg_ptr(const c10::optional<at::Tensor>& seg, int64_t B, int64_t Sk) {
  if (!seg.has_value() || !seg->defined()) return nullptr;
  TORCH_CHECK(seg->scalar_type() == at::kInt && seg->is_contiguous() && seg->numel() == B * Sk, "seg must be int32 [B, Sk]");
  return seg->data_ptr<int>();
}

// q/k/v: [B*S, ld] buffers; head h of q lives at columns q_col0 + h*128 (same for k/v with kv heads).
void flash_fwd(const at::Tensor& q, int64_t q_col0, const at::Tensor& k, int64_t k_col0, const at::Tensor& v,
               int64_t v_col0, at::Tensor& o, at::Tensor& lse, int64_t B, int64_t Sq, int64_t Sk, int64_t Hq,
               int64_t Hkv, double scale, bool causal, const c10::optional<at::Tensor>& seg) {
  check_buf(q, "q");
  check_buf(k, "k");
  check_buf(v, "v");
  check_buf(o, "o");
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(q.size(0) == B * Sq && k.size(0) == B * Sk && v.size(0) == B * Sk && o.size(0) == B * Sq, "rows");
  TORCH_CHECK(o.size(1) >= Hq * 128, "o too narrow");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * Hq * Sq, "lse must be fp32 [B, Hq, Sq]");
  TORCH_CHECK(q_col0 % 8 == 0 && k_col0 % 8 == 0 && v_col0 % 8 == 0, "column offsets must be 16-byte aligned");
  c10::cuda::CUDAGuard g(q.device());
  astrai_host::flash_fwd(q.data_ptr(), q.stride(0), (int)q_col0, k.data_ptr(), k.stride(0), (int)k_col0, v.data_ptr(),
                         v.stride(0), (int)v_col0, o.data_ptr(), o.stride(0), lse.data_ptr<float>(), (int)B, (int)Sq,
                         (int)Sk, (int)Hq, (int)Hkv, (float)scale, causal ? 1 : 0, seg_ptr(seg, B, Sk),
                         at::cuda::getCurrentCUDAStream().stream());
}

// Two query tiles per CTA, P in tensor memory; head_dim 64 or 128.
void flash_fwd2(const at::Tensor& q, int64_t q_col0, const at::Tensor& k, int64_t k_col0, const at::Tensor& v,
                int64_t v_col0, at::Tensor& o, at::Tensor& lse, int64_t B, int64_t Sq, int64_t Sk, int64_t Hq,
                int64_t Hkv, int64_t D, double scale, bool causal, const c10::optional<at::Tensor>& seg) {
  check_buf(q, "q");
  check_buf(k, "k");
  check_buf(v, "v");
  check_buf(o, "o");
  TORCH_CHECK(D == 64 || D == 128, "flash_fwd2: head_dim must be 64 or 128");
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(q.size(0) == B * Sq && k.size(0) == B * Sk && v.size(0) == B * Sk && o.size(0) == B * Sq, "rows");
  TORCH_CHECK(q.size(1) >= q_col0 + Hq * D && k.size(1) >= k_col0 + Hkv * D && v.size(1) >= v_col0 + Hkv * D,
              "q/k/v too narrow for the heads");
  TORCH_CHECK(o.size(1) >= Hq * D, "o too narrow");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == B * Hq * Sq,
              "lse must be fp32 [B, Hq, Sq]");
  TORCH_CHECK(q_col0 % 8 == 0 && k_col0 % 8 == 0 && v_col0 % 8 == 0, "column offsets must be 16-byte aligned");
  c10::cuda::CUDAGuard g(q.device());
  astrai_host::flash_fwd_pair(q.data_ptr(), q.stride(0), (int)q_col0, k.data_ptr(), k.stride(0), (int)k_col0,
                              v.data_ptr(), v.stride(0), (int)v_col0, o.data_ptr(), o.stride(0), lse.data_ptr<float>(),
                              (int)B, (int)Sq, (int)Sk, (int)Hq, (int)Hkv, (int)D, (float)scale, causal ? 1 : 0,
                              seg_ptr(seg, B, Sk), at::cuda::getCurrentCUDAStream().stream());
}

void flash_bwd(const at::Tensor& q, int64_t q_col0, const at::Tensor& k, int64_t k_col0, const at::Tensor& v,
               int64_t v_col0, const at::Tensor& o, const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta,
               at::Tensor& dq_acc, at::Tensor& dq, int64_t dq_col0, at::Tensor& dk, int64_t dk_col0, at::Tensor& dv,
               int64_t dv_col0, int64_t B, int64_t Sq, int64_t Sk, int64_t Hq, int64_t Hkv, double scale, bool causal,
               const c10::optional<at::Tensor>& seg) {
  check_buf(q, "q");
  check_buf(k, "k");
  check_buf(v, "v");
  check_buf(o, "o");
  check_buf(dout, "dout");
  check_buf(dq, "dq");
  check_buf(dk, "dk");
  check_buf(dv, "dv");
  TORCH_CHECK(dk.stride(0) == dv.stride(0), "dk and dv must share a row stride");
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() && dq_acc.numel() == B * Sq * Hq * 128,
              "dq_acc must be fp32 [B*Sq, Hq*128] contiguous");
  const int64_t Sq_pad = (Sq + 63) / 64 * 64;
  TORCH_CHECK(delta.scalar_type() == at::kFloat && delta.is_contiguous() && delta.numel() >= 2 * B * Hq * Sq_pad,
              "delta workspace must be fp32 with >= 2*B*Hq*ceil(Sq/64)*64 elements");
  c10::cuda::CUDAGuard g(q.device());
  astrai_host::flash_bwd(q.data_ptr(), q.stride(0), (int)q_col0, k.data_ptr(), k.stride(0), (int)k_col0, v.data_ptr(),
                         v.stride(0), (int)v_col0, o.data_ptr(), o.stride(0), dout.data_ptr(), dout.stride(0), 0,
                         lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(), dq.data_ptr(),
                         dq.stride(0), (int)dq_col0, dk.data_ptr(), dv.data_ptr(), dk.stride(0), (int)dk_col0,
                         (int)dv_col0, (int)B, (int)Sq, (int)Sk, (int)Hq, (int)Hkv, (float)scale, causal ? 1 : 0,
                         seg_ptr(seg, B, Sk), at::cuda::getCurrentCUDAStream().stream());
}

}  // namespace

void register_attention(pybind11::module& m) {
  m.def("flash_fwd", &flash_fwd);
  m.def("flash_fwd2", &flash_fwd2);
  m.def("flash_bwd", &flash_bwd);
}
