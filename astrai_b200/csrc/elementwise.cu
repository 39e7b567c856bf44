// Bandwidth-bound elementwise kernels (sm_100a): interleaved RoPE, SwiGLU,
// embedding gather / scatter-add, batched bf16 transpose.
//
// RoPE parity: astrai/model/components/rope.py:26-33 rotates interleaved
// pairs (x[2i], x[2i+1]) by angle pos * theta_i with theta_i = base^(-2i/d),
// in fp32. Here the angle table is precomputed on the host as fp32
// (cos, sin) pairs [max_pos, d/2] and applied in place on the q / k columns
// of the fused QKV projection output (any row stride), so no copy of q or k
// is ever made. Backward is the same kernel with the rotation negated.
// SwiGLU parity: astrai/model/components/mlp.py:22-25 (up * silu(gate)).
#include <algorithm>

#include "common.cuh"

namespace astrai {

// x: [rows, ld] bf16; heads occupy columns [col0, col0 + n_heads*head_dim).
// pos: per-row position (nullable -> row % seq_len). cs: float2 [max_pos][head_dim/2].
// A position outside [0, max_pos) records kErrBadArg and leaves the chunk unrotated (no table read).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, long long ld, int rows, int col0, int n_heads, int head_dim,
                            const int* __restrict__ pos, int seq_len, const float2* __restrict__ cs, float sign,
                            int rot_dim, int rot_off, int max_pos, int* err) {
  // a kernel launched after this one with programmatic dependent launch may start now (it waits for
  // this grid to finish before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Row-walking: block b takes rows b, b + gridDim.x, ... two at a time (both rows' loads issued
  // before the math); thread k owns the 8-element chunks k, k + blockDim.x, ... of a row's
  // n_heads * rot_dim / 8, whose head and offsets are computed once; a row's position is read once.
  const int per_head = rot_dim / 8, nchunk = n_heads * per_head, T = blockDim.x;
  for (int k = threadIdx.x; k < nchunk; k += T) {
    const int h = k / per_head, chunk = k - h * per_head;
    const int coff = col0 + h * head_dim + rot_off + chunk * 8;
    for (int row = blockIdx.x; row < rows; row += 2 * gridDim.x) {
      const int rr[2] = {row, row + (int)gridDim.x};
      int p[2];
      uint4 u[2];
      float4 c[2][2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        p[q] = -1;
        if (rr[q] >= rows) continue;
        p[q] = pos ? pos[rr[q]] : rr[q] % seq_len;
        if (p[q] < 0 || p[q] >= max_pos) {
          set_error(err, kErrBadArg);
          p[q] = -1;
          continue;
        }
        u[q] = *reinterpret_cast<const uint4*>(x + (long long)rr[q] * ld + coff);
        const float4* cp = reinterpret_cast<const float4*>(cs + (long long)p[q] * (rot_dim / 2) + chunk * 4);
        c[q][0] = cp[0];
        c[q][1] = cp[1];
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (p[q] < 0) continue;
        uint32_t w[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
        const float2 r4[4] = {make_float2(c[q][0].x, c[q][0].y), make_float2(c[q][0].z, c[q][0].w),
                              make_float2(c[q][1].x, c[q][1].y), make_float2(c[q][1].z, c[q][1].w)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 v = unpack_bf16(w[j]);
          const float sn = sign * r4[j].y;
          w[j] = pack_bf16(v.x * r4[j].x - v.y * sn, v.x * sn + v.y * r4[j].x);
        }
        *reinterpret_cast<uint4*>(x + (long long)rr[q] * ld + coff) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// silu / sigmoid with the fast division (__fdividef: at most 2 ulp from the quotient for
// denominators below 2^126; above, i.e. g < -87, it returns 0, where the quotient is below 1e-37):
// invisible after the bf16 rounding of every output, and a tenth of the IEEE division's instructions
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.f + __expf(-g)); }
__device__ __forceinline__ float sigm_f(float g) { return __fdividef(1.f, 1.f + __expf(-g)); }

// Row-walking layout of the SwiGLU kernels: block b takes rows b, b + gridDim.x, ...; its threads
// cover the row's F / 8 16-byte chunks, two per thread per pass (both loads issued before the math),
// so no index division is needed and two chunks' loads are in flight per thread.
// h: [rows, ldh] with up = h[:, 0:F], gate = h[:, F:2F];  out: [rows, ldo]
// live_rows (optional device count): only the first *live_rows of the `rows` rows hold data (an expert
// block sized for its capacity); the rest are left untouched.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ h, long long ldh, __nv_bfloat16* __restrict__ out,
                                  long long ldo, int rows, int F, const int* __restrict__ live_rows) {
  // a kernel launched after this one with programmatic dependent launch may start now (it waits for
  // this grid to finish before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int per_row = F / 8, T = blockDim.x;
  const int nrows = live_rows ? min(rows, max(0, *live_rows)) : rows;
  for (int row = blockIdx.x; row < nrows; row += gridDim.x) {
    const __nv_bfloat16* hr = h + (long long)row * ldh;
    __nv_bfloat16* orow = out + (long long)row * ldo;
    for (int c0 = threadIdx.x; c0 < per_row; c0 += 2 * T) {
      uint4 uu[2], gg[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = (c0 + k * T) * 8;
        const bool ok = c0 + k * T < per_row;
        uu[k] = ok ? *reinterpret_cast<const uint4*>(hr + c) : make_uint4(0u, 0u, 0u, 0u);
        gg[k] = ok ? *reinterpret_cast<const uint4*>(hr + F + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (c0 + k * T >= per_row) break;
        const uint32_t u[4] = {uu[k].x, uu[k].y, uu[k].z, uu[k].w}, g[4] = {gg[k].x, gg[k].y, gg[k].z, gg[k].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = unpack_bf16(u[j]), b = unpack_bf16(g[j]);
          o[j] = pack_bf16(a.x * silu_f(b.x), a.y * silu_f(b.y));
        }
        *reinterpret_cast<uint4*>(orow + (c0 + k * T) * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// dh[:, :F] = dy * silu(g);  dh[:, F:] = dy * up * silu'(g)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long long lddy,
                                  const __nv_bfloat16* __restrict__ h, long long ldh, __nv_bfloat16* __restrict__ dh,
                                  long long lddh, int rows, int F, const int* __restrict__ live_rows) {
  const int per_row = F / 8, T = blockDim.x;
  const int nrows = live_rows ? min(rows, max(0, *live_rows)) : rows;
  for (int row = blockIdx.x; row < nrows; row += gridDim.x) {
    const __nv_bfloat16* hr = h + (long long)row * ldh;
    const __nv_bfloat16* dr = dy + (long long)row * lddy;
    __nv_bfloat16* dhr = dh + (long long)row * lddh;
    for (int c0 = threadIdx.x; c0 < per_row; c0 += 2 * T) {
      uint4 uu[2], gg[2], dd[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = (c0 + k * T) * 8;
        const bool ok = c0 + k * T < per_row;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        uu[k] = ok ? *reinterpret_cast<const uint4*>(hr + c) : z;
        gg[k] = ok ? *reinterpret_cast<const uint4*>(hr + F + c) : z;
        dd[k] = ok ? *reinterpret_cast<const uint4*>(dr + c) : z;
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (c0 + k * T >= per_row) break;
        const uint32_t u[4] = {uu[k].x, uu[k].y, uu[k].z, uu[k].w}, g[4] = {gg[k].x, gg[k].y, gg[k].z, gg[k].w},
                       d[4] = {dd[k].x, dd[k].y, dd[k].z, dd[k].w};
        uint32_t du[4], dg[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = unpack_bf16(u[j]), b = unpack_bf16(g[j]), e = unpack_bf16(d[j]);
          const float s0 = sigm_f(b.x), s1 = sigm_f(b.y);
          du[j] = pack_bf16(e.x * b.x * s0, e.y * b.y * s1);
          dg[j] = pack_bf16(e.x * a.x * s0 * (1.f + b.x * (1.f - s0)), e.y * a.y * s1 * (1.f + b.y * (1.f - s1)));
        }
        const int c = (c0 + k * T) * 8;
        *reinterpret_cast<uint4*>(dhr + c) = make_uint4(du[0], du[1], du[2], du[3]);
        *reinterpret_cast<uint4*>(dhr + F + c) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
      }
    }
  }
}

// out[t, :] = w[ids[t], :]   (d multiple of 8)
__global__ void embedding_fwd_kernel(const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ w,
                                     __nv_bfloat16* __restrict__ out, int n_tok, int d, int vocab, int* err) {
  // a kernel launched after this one with programmatic dependent launch may start now (it waits for
  // this grid to finish before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int per = d / 8;
  const long long total = (long long)n_tok * per;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int t = idx / per, c = (idx % per) * 8;
    long long id = ids[t];
    if (id < 0 || id >= vocab) {
      set_error(err, kErrBadArg);
      id = 0;
    }
    *reinterpret_cast<uint4*>(out + (long long)t * d + c) = *reinterpret_cast<const uint4*>(w + id * d + c);
  }
}

// gw_f32[ids[t], :] += g[t, :]
__global__ void embedding_bwd_kernel(const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ g,
                                     float* __restrict__ gw, int n_tok, int d, int vocab) {
  const int per = d / 8;
  const long long total = (long long)n_tok * per;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int t = idx / per, c = (idx % per) * 8;
    const long long id = ids[t];
    if (id < 0 || id >= vocab) continue;
    const uint4 u = *reinterpret_cast<const uint4*>(g + (long long)t * d + c);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float* dst = gw + id * d + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(w[j]);
      atomicAdd(dst + 2 * j, f.x);
      atomicAdd(dst + 2 * j + 1, f.y);
    }
  }
}

// out (bf16 or accumulate into bf16) from fp32 buffer
__global__ void f32_to_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, long long n,
                                   int accumulate) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float v = in[i];
    if (accumulate) v += __bfloat162float(out[i]);
    out[i] = __float2bfloat16_rn(v);
  }
}

// Batched transpose of bf16 matrices: out[b][c][r] = in[b][r][c]; 32x32 tiles via smem.
__global__ void transpose_bf16_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int R,
                                      int C, long long in_bstride, long long out_bstride) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int b = blockIdx.z;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const __nv_bfloat16* src = in + b * in_bstride;
  __nv_bfloat16* dst = out + b * out_bstride;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = src[(long long)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) dst[(long long)c * R + r] = tile[threadIdx.x][i];
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

static inline int ew_grid(long long work) {
  long long g = (work + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}

void rope_apply(void* x, long long ld, int rows, int col0, int n_heads, int head_dim, const int* pos, int seq_len,
                const void* cs, int inverse, int rot_dim, int rot_off, int max_pos, cudaStream_t s) {
  if (rows <= 0 || n_heads <= 0) return;
  // threads = the row's 16-byte chunks (rounded to a warp, at most 1024); blocks walk rows in pairs
  const int nchunk = n_heads * (rot_dim / 8);
  const int T = std::min(1024, std::max(32, (nchunk + 31) / 32 * 32));
  int dev = 0;
  cudaGetDevice(&dev);
  const long long cap = (long long)num_sms(dev) * (2048 / T);
  const int grid = (int)std::max(1LL, std::min<long long>((rows + 1) / 2, cap));
  (astrai::note_launch(), rope_kernel<<<grid, T, 0, s>>>(static_cast<__nv_bfloat16*>(x), ld, rows, col0, n_heads, head_dim, pos,
                                            seq_len, static_cast<const float2*>(cs), inverse ? -1.f : 1.f, rot_dim,
                                            rot_off, max_pos, error_word(dev)));
}

// Row-walking launch of the SwiGLU kernels: threads = half the row's 16-byte chunks (rounded to a
// warp, at most 1024), blocks = rows, capped at what fills every SM with 2048 threads.
static inline void row_launch_dims(int rows, int F, int* grid, int* threads) {
  const int chunks = std::max(1, F / 8);
  int T = ((chunks + 1) / 2 + 31) / 32 * 32;
  T = std::min(1024, std::max(32, T));
  int dev = 0;
  cudaGetDevice(&dev);
  const long long cap = (long long)num_sms(dev) * (2048 / T);
  *threads = T;
  *grid = (int)std::max(1LL, std::min<long long>(rows, cap));
}

void swiglu_fwd(const void* h, long long ldh, void* out, long long ldo, int rows, int F, const int* live_rows,
                cudaStream_t s) {
  if (rows <= 0) return;
  int grid = 1, T = 32;
  row_launch_dims(rows, F, &grid, &T);
  (astrai::note_launch(), swiglu_fwd_kernel<<<grid, T, 0, s>>>(static_cast<const __nv_bfloat16*>(h), ldh,
                                                                static_cast<__nv_bfloat16*>(out), ldo, rows, F,
                                                                live_rows));
}

void swiglu_bwd(const void* dy, long long lddy, const void* h, long long ldh, void* dh, long long lddh, int rows, int F,
                const int* live_rows, cudaStream_t s) {
  if (rows <= 0) return;
  int grid = 1, T = 32;
  row_launch_dims(rows, F, &grid, &T);
  (astrai::note_launch(), swiglu_bwd_kernel<<<grid, T, 0, s>>>(
      static_cast<const __nv_bfloat16*>(dy), lddy, static_cast<const __nv_bfloat16*>(h), ldh,
      static_cast<__nv_bfloat16*>(dh), lddh, rows, F, live_rows));
}

void embedding_fwd(const long long* ids, const void* w, void* out, int n_tok, int d, int vocab, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  (astrai::note_launch(), embedding_fwd_kernel<<<ew_grid((long long)n_tok * d / 8), 256, 0, s>>>(
      ids, static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(out), n_tok, d, vocab, error_word(dev)));
}

void embedding_bwd(const long long* ids, const void* g, float* gw, int n_tok, int d, int vocab, cudaStream_t s) {
  (astrai::note_launch(), embedding_bwd_kernel<<<ew_grid((long long)n_tok * d / 8), 256, 0, s>>>(ids, static_cast<const __nv_bfloat16*>(g),
                                                                          gw, n_tok, d, vocab));
}

void f32_to_bf16(const float* in, void* out, long long n, int accumulate, cudaStream_t s) {
  (astrai::note_launch(), f32_to_bf16_kernel<<<ew_grid(n), 256, 0, s>>>(in, static_cast<__nv_bfloat16*>(out), n, accumulate));
}

void transpose_bf16(const void* in, void* out, int batch, int R, int C, cudaStream_t s) {
  dim3 grid((C + 31) / 32, (R + 31) / 32, batch);
  (astrai::note_launch(), transpose_bf16_kernel<<<grid, dim3(32, 8), 0, s>>>(static_cast<const __nv_bfloat16*>(in),
                                                     static_cast<__nv_bfloat16*>(out), R, C, (long long)R * C,
                                                     (long long)R * C));
}

}  // namespace astrai_host
