// Optimizer kernels (sm_100a): global gradient norm + clip coefficient,
// multi-tensor AdamW, and the elementwise stages of batched Muon.
//
// Parity targets: torch.optim.AdamW(fused=True) and torch.optim.Muon as
// configured by the reference's MuonMix (scripts/tools/train.py:18-94), and
// clip_grad_norm_ (astrai/parallel/executor.py:162-166). Everything stays on
// the device: the clip coefficient is computed into device memory and read
// by the update kernels, so an optimizer step needs no host synchronisation.
//
// Tensors are addressed through device-side pointer tables built once per
// parameter set: one launch updates every parameter.
#include "common.cuh"

namespace astrai {

// Work item table: block b handles elements [start, start+len) of tensor idx.
struct Chunk {
  int tensor;
  int len;
  long long start;
};

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float sh[32];
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? sh[l] : 0.f;
  if (w == 0) v = warp_sum(v);
  __syncthreads();
  return v;
}

// acc[group[tensor]] += sum(g^2) over the chunk (g bf16)
__global__ void sumsq_kernel(const Chunk* __restrict__ chunks, const long long* __restrict__ gptr,
                             const int* __restrict__ group, float* __restrict__ acc) {
  const Chunk c = chunks[blockIdx.x];
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(gptr[c.tensor]) + c.start;
  float s = 0.f;
  if ((reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    // 16-byte loads, two in flight per thread; the tail (len % 8) element-wise
    const int nv = c.len / 8;
    const uint4* gv = reinterpret_cast<const uint4*>(g);
    for (int j = threadIdx.x; j < nv; j += 2 * blockDim.x) {
      const uint4 a = gv[j];
      const uint4 b = j + (int)blockDim.x < nv ? gv[j + blockDim.x] : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float2 f = unpack_bf16(w[e]);
        s = fmaf(f.x, f.x, s);
        s = fmaf(f.y, f.y, s);
      }
    }
    for (int i = nv * 8 + threadIdx.x; i < c.len; i += blockDim.x) {
      const float v = __bfloat162float(g[i]);
      s += v * v;
    }
  } else {
    for (int i = threadIdx.x; i < c.len; i += blockDim.x) {
      const float v = __bfloat162float(g[i]);
      s += v * v;
    }
  }
  s = block_sum(s);
  if (threadIdx.x == 0) atomicAdd(&acc[group ? group[c.tensor] : 0], s);
}

// coef = min(1, max_norm / (sqrt(sum acc) + 1e-6)); norm_out = sqrt(sum acc)
__global__ void clip_coef_kernel(const float* __restrict__ acc, int n, float max_norm, float* __restrict__ coef,
                                 float* __restrict__ norm_out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s += acc[i];
    const float nrm = sqrtf(s);
    norm_out[0] = nrm;
    coef[0] = max_norm > 0.f ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
  }
}

// AdamW, decoupled weight decay (torch semantics):
//   p *= 1 - lr*wd;  m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   p -= lr * (m / bc1) / (sqrt(v / bc2) + eps)
// g = grad * coef (clip). Moments fp32, params/grads bf16 or fp32.
// 8 consecutive elements <-> fp32 registers (16-byte aligned addresses)
__device__ __forceinline__ void load8(const __nv_bfloat16* a, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(a);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void load8(const float* a, float (&f)[8]) {
  *reinterpret_cast<float4*>(&f[0]) = reinterpret_cast<const float4*>(a)[0];
  *reinterpret_cast<float4*>(&f[4]) = reinterpret_cast<const float4*>(a)[1];
}
__device__ __forceinline__ void store8(__nv_bfloat16* a, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(a) =
      make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}
__device__ __forceinline__ void store8(float* a, const float (&f)[8]) {
  reinterpret_cast<float4*>(a)[0] = *reinterpret_cast<const float4*>(&f[0]);
  reinterpret_cast<float4*>(a)[1] = *reinterpret_cast<const float4*>(&f[4]);
}

template <typename P>
__global__ void adamw_kernel(const Chunk* __restrict__ chunks, const long long* __restrict__ pptr,
                             const long long* __restrict__ gptr, const long long* __restrict__ mptr,
                             const long long* __restrict__ vptr, const float* __restrict__ wd_per_tensor, float lr,
                             float b1, float b2, float eps, float bc1, float bc2, const float* __restrict__ coef) {
  const Chunk c = chunks[blockIdx.x];
  P* p = reinterpret_cast<P*>(pptr[c.tensor]) + c.start;
  const P* g = reinterpret_cast<const P*>(gptr[c.tensor]) + c.start;
  float* m = reinterpret_cast<float*>(mptr[c.tensor]) + c.start;
  float* v = reinterpret_cast<float*>(vptr[c.tensor]) + c.start;
  const float k = coef ? coef[0] : 1.f;
  const float decay = 1.f - lr * wd_per_tensor[c.tensor];
  const float step = lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  // 8 elements per thread per step with 16-byte accesses when the chunk allows it (every chunk of a
  // contiguous tensor does): a scalar loop keeps too few bytes in flight to reach HBM bandwidth
  int i0 = 0;
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
                     reinterpret_cast<uintptr_t>(v)) & 15) == 0;
  if (vec) {
    const int nv = c.len / 8;
    for (int j = threadIdx.x; j < nv; j += blockDim.x) {
      float pf[8], gf[8], mf[8], vf[8];
      load8(p + 8 * j, pf);
      load8(g + 8 * j, gf);
      *reinterpret_cast<float4*>(&mf[0]) = reinterpret_cast<const float4*>(m + 8 * j)[0];
      *reinterpret_cast<float4*>(&mf[4]) = reinterpret_cast<const float4*>(m + 8 * j)[1];
      *reinterpret_cast<float4*>(&vf[0]) = reinterpret_cast<const float4*>(v + 8 * j)[0];
      *reinterpret_cast<float4*>(&vf[4]) = reinterpret_cast<const float4*>(v + 8 * j)[1];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float gi = gf[e] * k;
        mf[e] = b1 * mf[e] + (1.f - b1) * gi;
        vf[e] = b2 * vf[e] + (1.f - b2) * gi * gi;
        pf[e] = pf[e] * decay - step * mf[e] / (sqrtf(vf[e]) * rbc2 + eps);
      }
      reinterpret_cast<float4*>(m + 8 * j)[0] = *reinterpret_cast<const float4*>(&mf[0]);
      reinterpret_cast<float4*>(m + 8 * j)[1] = *reinterpret_cast<const float4*>(&mf[4]);
      reinterpret_cast<float4*>(v + 8 * j)[0] = *reinterpret_cast<const float4*>(&vf[0]);
      reinterpret_cast<float4*>(v + 8 * j)[1] = *reinterpret_cast<const float4*>(&vf[4]);
      store8(p + 8 * j, pf);
    }
    i0 = nv * 8;
  }
  for (int i = i0 + threadIdx.x; i < c.len; i += blockDim.x) {
    const float gi = to_f(g[i]) * k;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = to_f(p[i]) * decay;
    pi -= step * mi / (sqrtf(vi) * rbc2 + eps);
    p[i] = from_f<P>(pi);
  }
}

// Muon stage 1: buf = mu*buf + (1-mu)*g ; u = nesterov ? g + mu*(buf-g) : buf
// u is written into the batched buffer U[b] (same row-major layout as the
// parameter) and sum(u^2) is accumulated per matrix.
template <typename B>
__global__ void muon_momentum_kernel(const long long* __restrict__ gptr, const long long* __restrict__ bufptr,
                                     __nv_bfloat16* __restrict__ U, long long numel, float mu, int nesterov,
                                     const float* __restrict__ coef, float* __restrict__ sumsq) {
  const int b = blockIdx.y;
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(gptr[b]);
  B* buf = reinterpret_cast<B*>(bufptr[b]);
  __nv_bfloat16* u = U + (long long)b * numel;
  const float k = coef ? coef[0] : 1.f;
  float s = 0.f;
  // 8 elements per thread per step with 16-byte accesses (parameters are contiguous matrices)
  long long i0 = 0;
  const bool vec = (numel % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(buf) | reinterpret_cast<uintptr_t>(u)) &
                    15) == 0;
  if (vec) {
    const long long nv = numel / 8;
    for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < nv; j += (long long)gridDim.x * blockDim.x) {
      float gf[8], bf[8], uf[8];
      load8(g + 8 * j, gf);
      load8(buf + 8 * j, bf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float gi = gf[e] * k;
        bf[e] = mu * bf[e] + (1.f - mu) * gi;
        uf[e] = nesterov ? gi + mu * (bf[e] - gi) : bf[e];
      }
      store8(buf + 8 * j, bf);
      store8(u + 8 * j, uf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float r = __bfloat162float(__float2bfloat16_rn(uf[e]));  // the norm of the stored bf16 values
        s += r * r;
      }
    }
    i0 = numel;
  }
  for (long long i = i0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < numel; i += (long long)gridDim.x * blockDim.x) {
    const float gi = __bfloat162float(g[i]) * k;
    const float bi = mu * to_f(buf[i]) + (1.f - mu) * gi;
    buf[i] = from_f<B>(bi);
    const float ui = nesterov ? gi + mu * (bi - gi) : bi;
    const __nv_bfloat16 ub = __float2bfloat16_rn(ui);
    u[i] = ub;
    const float uf = __bfloat162float(ub);
    s += uf * uf;
  }
  s = block_sum(s);
  if (threadIdx.x == 0) atomicAdd(&sumsq[b], s);
}

// Muon stage 2: X[b] = (transpose ? U[b]^T : U[b]) / max(||U[b]||_F, eps)
__global__ void muon_normalize_kernel(const __nv_bfloat16* __restrict__ U, __nv_bfloat16* __restrict__ X, int R, int C,
                                      int transpose, const float* __restrict__ sumsq, float eps) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int b = blockIdx.z;
  const float scale = 1.f / fmaxf(sqrtf(sumsq[b]), eps);
  const __nv_bfloat16* src = U + (long long)b * R * C;
  __nv_bfloat16* dst = X + (long long)b * R * C;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  if (!transpose) {
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int r = r0 + i, c = c0 + threadIdx.x;
      if (r < R && c < C) dst[(long long)r * C + c] = __float2bfloat16_rn(__bfloat162float(src[(long long)r * C + c]) * scale);
    }
    return;
  }
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = src[(long long)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) dst[(long long)c * R + r] = __float2bfloat16_rn(__bfloat162float(tile[threadIdx.x][i]) * scale);
  }
}

// Vector form of muon_normalize_kernel (U and X are whole, 16-byte aligned work buffers): 8 elements
// per 16-byte access; transposed, 64 x 64 tiles go through shared memory (R and C multiples of 64).
__global__ void __launch_bounds__(256) muon_normalize_vec_kernel(const __nv_bfloat16* __restrict__ U,
                                                                 __nv_bfloat16* __restrict__ X, int R, int C,
                                                                 int transpose, const float* __restrict__ sumsq,
                                                                 float eps) {
  const int b = blockIdx.z;
  const float scale = 1.f / fmaxf(sqrtf(sumsq[b]), eps);
  const __nv_bfloat16* src = U + (long long)b * R * C;
  __nv_bfloat16* dst = X + (long long)b * R * C;
  if (!transpose) {
    const long long nv = (long long)R * C / 8;
    for (long long j = (long long)blockIdx.x * 256 + threadIdx.x; j < nv; j += (long long)gridDim.x * 256) {
      float f[8];
      load8(src + 8 * j, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= scale;
      store8(dst + 8 * j, f);
    }
    return;
  }
  __shared__ float tile[64][65];  // [r][c] of U
  const int c0 = blockIdx.x * 64, r0 = blockIdx.y * 64;
  for (int v = threadIdx.x; v < 512; v += 256) {
    const int ri = v >> 3, cv = (v & 7) * 8;
    float f[8];
    load8(src + (long long)(r0 + ri) * C + c0 + cv, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) tile[ri][cv + e] = f[e];
  }
  __syncthreads();
  // X = U^T: 64 rows (c) x 8 vectors (r)
  for (int v = threadIdx.x; v < 512; v += 256) {
    const int ci = v >> 3, rv = (v & 7) * 8;
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = tile[rv + e][ci] * scale;
    store8(dst + (long long)(c0 + ci) * R + r0 + rv, f);
  }
}

// Muon stage 3: p[b] = p[b] * (1 - lr*wd) - adj_lr * (transpose ? X[b]^T : X[b])
template <typename P>
__global__ void muon_apply_kernel(const long long* __restrict__ pptr, const __nv_bfloat16* __restrict__ X, int R, int C,
                                  int transpose, float decay, float adj_lr) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  P* p = reinterpret_cast<P*>(pptr[b]);
  const __nv_bfloat16* x = X + (long long)b * R * C;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  if (!transpose) {
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int r = r0 + i, c = c0 + threadIdx.x;
      if (r < R && c < C) {
        const long long o = (long long)r * C + c;
        p[o] = from_f<P>(to_f(p[o]) * decay - adj_lr * __bfloat162float(x[o]));
      }
    }
    return;
  }
  // X[b] is stored [C][R]; read it tiled and transpose through smem
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = __bfloat162float(x[(long long)c * R + r]);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) {
      const long long o = (long long)r * C + c;
      p[o] = from_f<P>(to_f(p[o]) * decay - adj_lr * tile[threadIdx.x][i]);
    }
  }
}

// Muon stage 3 with 16-byte accesses. Not transposed: 8 consecutive elements per thread. Transposed
// (X[b] stored [C][R]): 64 x 64 tiles, read along R and written along C in 8-element vectors,
// transposed through shared memory.
template <typename P>
__global__ void __launch_bounds__(256) muon_apply_vec_kernel(const long long* __restrict__ pptr,
                                                             const __nv_bfloat16* __restrict__ X, int R, int C,
                                                             int transpose, float decay, float adj_lr) {
  const int b = blockIdx.z;
  P* p = reinterpret_cast<P*>(pptr[b]);
  const __nv_bfloat16* x = X + (long long)b * R * C;
  const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15) == 0;  // X is a fresh, aligned buffer
  if (!transpose && !aligned) {
    for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < (long long)R * C; i += (long long)gridDim.x * 256)
      p[i] = from_f<P>(to_f(p[i]) * decay - adj_lr * __bfloat162float(x[i]));
    return;
  }
  if (!transpose) {
    const long long nv = (long long)R * C / 8;
    for (long long j = (long long)blockIdx.x * 256 + threadIdx.x; j < nv; j += (long long)gridDim.x * 256) {
      float pf[8], xf[8];
      load8(p + 8 * j, pf);
      load8(x + 8 * j, xf);
#pragma unroll
      for (int e = 0; e < 8; ++e) pf[e] = pf[e] * decay - adj_lr * xf[e];
      store8(p + 8 * j, pf);
    }
    return;
  }
  __shared__ float tile[64][65];  // [c][r]
  const int c0 = blockIdx.x * 64, r0 = blockIdx.y * 64;
  // 64 rows (c) x 8 vectors (r) of X
  for (int v = threadIdx.x; v < 512; v += 256) {
    const int ci = v >> 3, rv = (v & 7) * 8;
    float f[8];
    load8(x + (long long)(c0 + ci) * R + r0 + rv, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) tile[ci][rv + e] = f[e];
  }
  __syncthreads();
  // 64 rows (r) x 8 vectors (c) of p
  for (int v = threadIdx.x; v < 512; v += 256) {
    const int ri = v >> 3, cv = (v & 7) * 8;
    P* dst = p + (long long)(r0 + ri) * C + c0 + cv;
    if (!aligned) {
#pragma unroll
      for (int e = 0; e < 8; ++e) dst[e] = from_f<P>(to_f(dst[e]) * decay - adj_lr * tile[cv + e][ri]);
      continue;
    }
    float pf[8];
    load8(dst, pf);
#pragma unroll
    for (int e = 0; e < 8; ++e) pf[e] = pf[e] * decay - adj_lr * tile[cv + e][ri];
    store8(dst, pf);
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

void grad_sumsq(const void* chunks, int n_chunks, const long long* gptr, const int* group, float* acc, cudaStream_t s) {
  if (n_chunks <= 0) return;
  (astrai::note_launch(), sumsq_kernel<<<n_chunks, 256, 0, s>>>(static_cast<const Chunk*>(chunks), gptr, group, acc));
}

void clip_coef(const float* acc, int n, float max_norm, float* coef, float* norm_out, cudaStream_t s) {
  (astrai::note_launch(), clip_coef_kernel<<<1, 32, 0, s>>>(acc, n, max_norm, coef, norm_out));
}

void adamw_step(const void* chunks, int n_chunks, const long long* pptr, const long long* gptr, const long long* mptr,
                const long long* vptr, const float* wd, int fp32_params, float lr, float b1, float b2, float eps,
                float bc1, float bc2, const float* coef, cudaStream_t s) {
  if (n_chunks <= 0) return;
  if (fp32_params)
    (astrai::note_launch(), adamw_kernel<float><<<n_chunks, 256, 0, s>>>(static_cast<const Chunk*>(chunks), pptr, gptr, mptr, vptr, wd, lr, b1,
                                                  b2, eps, bc1, bc2, coef));
  else
    (astrai::note_launch(), adamw_kernel<__nv_bfloat16><<<n_chunks, 256, 0, s>>>(static_cast<const Chunk*>(chunks), pptr, gptr, mptr, vptr, wd,
                                                          lr, b1, b2, eps, bc1, bc2, coef));
}

void muon_momentum(const long long* gptr, const long long* bufptr, int buf_fp32, void* U, int batch, long long numel,
                   float mu, int nesterov, const float* coef, float* sumsq, cudaStream_t s) {
  int gx = (int)((numel + 256 * 8 - 1) / (256 * 8));
  if (gx > 1024) gx = 1024;
  dim3 grid(gx, batch);
  if (buf_fp32)
    (astrai::note_launch(), muon_momentum_kernel<float><<<grid, 256, 0, s>>>(gptr, bufptr, static_cast<__nv_bfloat16*>(U), numel, mu, nesterov,
                                                     coef, sumsq));
  else
    (astrai::note_launch(), muon_momentum_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(gptr, bufptr, static_cast<__nv_bfloat16*>(U), numel, mu,
                                                             nesterov, coef, sumsq));
}

void muon_normalize(const void* U, void* X, int batch, int R, int C, int transpose, const float* sumsq, float eps,
                    cudaStream_t s) {
  const bool al = (reinterpret_cast<uintptr_t>(U) % 16) == 0 && (reinterpret_cast<uintptr_t>(X) % 16) == 0;
  if (al && (transpose ? (R % 64 == 0 && C % 64 == 0) : ((long long)R * C % 8 == 0))) {
    const dim3 grid = transpose ? dim3(C / 64, R / 64, batch)
                                : dim3((unsigned)std::min<long long>(((long long)R * C / 8 + 255) / 256, 1024), 1, batch);
    (astrai::note_launch(), muon_normalize_vec_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(U),
                                                                          static_cast<__nv_bfloat16*>(X), R, C, transpose,
                                                                          sumsq, eps));
    return;
  }
  dim3 grid((C + 31) / 32, (R + 31) / 32, batch);
  (astrai::note_launch(), muon_normalize_kernel<<<grid, dim3(32, 8), 0, s>>>(static_cast<const __nv_bfloat16*>(U),
                                                     static_cast<__nv_bfloat16*>(X), R, C, transpose, sumsq, eps));
}

void muon_apply(const long long* pptr, int fp32_params, const void* X, int batch, int R, int C, int transpose,
                float decay, float adj_lr, cudaStream_t s) {
  // the vector kernel needs whole 8-element vectors (rows of 64 x 64 tiles when transposed); the
  // parameters' own alignment is checked by the caller's contiguous, 16-byte aligned storage
  const bool vec = transpose ? (R % 64 == 0 && C % 64 == 0) : (((long long)R * C) % 8 == 0);
  if (vec) {
    const dim3 grid = transpose ? dim3(C / 64, R / 64, batch)
                                : dim3((unsigned)std::min<long long>(((long long)R * C / 8 + 255) / 256, 1024), 1, batch);
    if (fp32_params)
      (astrai::note_launch(), muon_apply_vec_kernel<float><<<grid, 256, 0, s>>>(
                                  pptr, static_cast<const __nv_bfloat16*>(X), R, C, transpose, decay, adj_lr));
    else
      (astrai::note_launch(), muon_apply_vec_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
                                  pptr, static_cast<const __nv_bfloat16*>(X), R, C, transpose, decay, adj_lr));
    return;
  }
  dim3 grid((C + 31) / 32, (R + 31) / 32, batch);
  if (fp32_params)
    (astrai::note_launch(), muon_apply_kernel<float><<<grid, dim3(32, 8), 0, s>>>(pptr, static_cast<const __nv_bfloat16*>(X), R, C, transpose,
                                                          decay, adj_lr));
  else
    (astrai::note_launch(), muon_apply_kernel<__nv_bfloat16><<<grid, dim3(32, 8), 0, s>>>(pptr, static_cast<const __nv_bfloat16*>(X), R, C,
                                                                  transpose, decay, adj_lr));
}

}  // namespace astrai_host
