// Fused softmax cross-entropy (with label smoothing and ignore_index) and
// fused token log-probabilities, straight from bf16 logits (sm_100a).
//
// The reference materialises fp32 logits and calls F.cross_entropy
// (astrai/trainer/strategy.py:215-226, :246-269) or log_softmax + gather for
// DPO/GRPO (strategy.py:31-76). Here one CTA streams one row of bf16 logits
// once for the statistics (online max / sum-exp, sum of logits, target logit)
// and once more in backward to write d(logits) in bf16; no fp32 copy of the
// [tokens, vocab] matrix exists at any point.
//
//   loss_r   = lse_r - (1 - eps) * x[r, t_r] - eps / V * sum_j x[r, j]
//   dlogit   = g_r * (softmax_j - (1 - eps) * [j == t_r] - eps / V)      (CE)
//   logp_r   = x[r, t_r] - lse_r,  dlogit = g_r * ([j == t_r] - softmax_j)  (logprob)
#include <cfloat>

#include "common.cuh"

namespace astrai {

constexpr int CE_THREADS = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

// Row statistics: lse and (optionally) per-row CE loss / logprob.
// mode 0: CE with smoothing -> out[r] = loss (0 for ignored rows)
// mode 1: logprob          -> out[r] = x_t - lse
__global__ void __launch_bounds__(CE_THREADS) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                            const long long* __restrict__ target, int V,
                                                            float smoothing, long long ignore_index, int mode,
                                                            float* __restrict__ lse_out, float* __restrict__ out) {
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (long long)row * ld;
  float m = -INFINITY, s = 0.f, sx = 0.f;
  const int nvec = V / 8;
  for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + i * 8);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(w[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
    float lm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ls += __expf(v[j] - lm);
      sx += v[j];
    }
    online_merge(m, s, lm, ls);
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += CE_THREADS) {
    const float v = __bfloat162float(x[i]);
    online_merge(m, s, v, 1.f);
    sx += v;
  }
  // warp then block reduction of (m, s) and sx
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffff, m, o);
    const float s2 = __shfl_xor_sync(0xffffffff, s, o);
    online_merge(m, s, m2, s2);
    sx += __shfl_xor_sync(0xffffffff, sx, o);
  }
  __shared__ float sm_m[CE_THREADS / 32], sm_s[CE_THREADS / 32], sm_x[CE_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
    sm_x[warp] = sx;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < CE_THREADS / 32 ? sm_m[lane] : -INFINITY;
    s = lane < CE_THREADS / 32 ? sm_s[lane] : 0.f;
    sx = lane < CE_THREADS / 32 ? sm_x[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffff, m, o);
      const float s2 = __shfl_xor_sync(0xffffffff, s, o);
      online_merge(m, s, m2, s2);
      sx += __shfl_xor_sync(0xffffffff, sx, o);
    }
    if (lane == 0) {
      const float lse = m + __logf(s);
      lse_out[row] = lse;
      const long long t = target[row];
      if (mode == 0) {
        if (t == ignore_index || t < 0 || t >= V) {
          out[row] = 0.f;
        } else {
          const float xt = __bfloat162float(x[t]);
          out[row] = lse - (1.f - smoothing) * xt - smoothing / (float)V * sx;
        }
      } else {
        const long long tt = (t < 0 || t >= V) ? 0 : t;
        out[row] = __bfloat162float(x[tt]) - lse;
      }
    }
  }
}

// grad: mode 0 -> g_r = gscale[0] (shared by all non-ignored rows)
//       mode 1 -> g_r = grow[r]
__global__ void __launch_bounds__(CE_THREADS) ce_bwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                            const long long* __restrict__ target, int V,
                                                            float smoothing, long long ignore_index, int mode,
                                                            const float* __restrict__ lse_in,
                                                            const float* __restrict__ gscale,
                                                            const float* __restrict__ grow,
                                                            __nv_bfloat16* __restrict__ dlogits, long long ldd) {
  const int row = blockIdx.x;
  const long long t = target[row];
  float g;
  float on_t, off;  // coefficient for the target column and constant for all columns
  if (mode == 0) {
    const bool ign = (t == ignore_index) || t < 0 || t >= V;
    g = ign ? 0.f : gscale[0];
    on_t = -(1.f - smoothing);
    off = -smoothing / (float)V;
  } else {
    g = -grow[row];  // d(x_t - lse) = [j==t] - p_j  ->  -(p_j - [j==t])
    on_t = -1.f;
    off = 0.f;
  }
  const float lse = lse_in[row];
  const __nv_bfloat16* x = logits + (long long)row * ld;
  __nv_bfloat16* d = dlogits + (long long)row * ldd;
  const int nvec = V / 8;
  for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + i * 8);
    uint32_t w[4] = {u.x, u.y, u.z, u.w}, o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(w[j]);
      const int c0 = i * 8 + 2 * j;
      float a = __expf(f.x - lse) + off + (c0 == t ? on_t : 0.f);
      float b = __expf(f.y - lse) + off + (c0 + 1 == t ? on_t : 0.f);
      o[j] = pack_bf16(a * g, b * g);
    }
    *reinterpret_cast<uint4*>(d + i * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += CE_THREADS) {
    const float f = __bfloat162float(x[i]);
    d[i] = __float2bfloat16_rn(g * (__expf(f - lse) + off + (i == t ? on_t : 0.f)));
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

void ce_fwd(const void* logits, long long ld, const long long* target, int rows, int V, float smoothing,
            long long ignore_index, int mode, float* lse, float* out, cudaStream_t s) {
  (astrai::note_launch(), ce_fwd_kernel<<<rows, CE_THREADS, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), ld, target, V, smoothing,
                                            ignore_index, mode, lse, out));
}

void ce_bwd(const void* logits, long long ld, const long long* target, int rows, int V, float smoothing,
            long long ignore_index, int mode, const float* lse, const float* gscale, const float* grow,
            void* dlogits, long long ldd, cudaStream_t s) {
  (astrai::note_launch(), ce_bwd_kernel<<<rows, CE_THREADS, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), ld, target, V, smoothing,
                                            ignore_index, mode, lse, gscale, grow,
                                            static_cast<__nv_bfloat16*>(dlogits), ldd));
}

}  // namespace astrai_host
