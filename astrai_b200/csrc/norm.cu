// RMSNorm forward / backward (sm_100a, bandwidth-bound).
//
//   y = x * rsqrt(mean(x^2) + eps) * w          (astrai/model/components/norm.py:14-15)
//
// One warp per row; each lane owns a fixed set of 16-byte column chunks, so
// the weight-gradient partial sums of a block stay in registers. Rows are
// processed in fp32. Backward writes dx and per-block fp32 partials of dw,
// which a second kernel reduces (dw is a sum over all rows).
#include "common.cuh"

namespace astrai {

template <int CHUNKS>  // 16-byte chunks (8 bf16) per lane; D = CHUNKS * 256
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, long long ldy,
                                                          float* __restrict__ rstd_out, int rows, int D, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (long long)row * ldx;
  float v[CHUNKS][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < D) {
      uint4 u = *reinterpret_cast<const uint4*>(xr + col);
      uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = unpack_bf16(uu[j]);
        v[c][2 * j] = f.x;
        v[c][2 * j + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[c][j] = 0.f;
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = r;
  __nv_bfloat16* yr = y + (long long)row * ldy;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < D) {
      uint4 wu = *reinterpret_cast<const uint4*>(w + col);
      uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 wf = unpack_bf16(ww[j]);
        o[j] = pack_bf16(v[c][2 * j] * r * wf.x, v[c][2 * j + 1] * r * wf.y);
      }
      *reinterpret_cast<uint4*>(yr + col) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Small-D variant (D <= 256, e.g. per-head QK-norm): 8 rows per warp-quarter.
__global__ void __launch_bounds__(256) rmsnorm_fwd_small_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                const __nv_bfloat16* __restrict__ w,
                                                                __nv_bfloat16* __restrict__ y, long long ldy,
                                                                float* __restrict__ rstd_out, int rows, int D,
                                                                float eps) {
  // one warp per row, each lane handles D/32 elements (D multiple of 32)
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (long long)row * ldx;
  float v[8];
  float ss = 0.f;
  const int per = D / 32;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = (j < per) ? __bfloat162float(xr[lane * per + j]) : 0.f;
    ss += v[j] * v[j];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = r;
  __nv_bfloat16* yr = y + (long long)row * ldy;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j < per) yr[lane * per + j] = __float2bfloat16_rn(v[j] * r * __bfloat162float(w[lane * per + j]));
}

// dx = r*w*dy - x * r^3 * mean(dy*w*x);   dw_partial[block] = sum_rows dy*x*r
template <int CHUNKS>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long long lddy,
                                                          const __nv_bfloat16* __restrict__ x, long long ldx,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const float* __restrict__ rstd,
                                                          __nv_bfloat16* __restrict__ dx, long long lddx,
                                                          const __nv_bfloat16* __restrict__ dres, long long ldres,
                                                          float* __restrict__ dw_part, int rows, int D,
                                                          int rows_per_block) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float wv[CHUNKS][8];
  float acc[CHUNKS][8];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = (c * 32 + lane) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[c][j] = 0.f;
    if (col < D) {
      uint4 wu = *reinterpret_cast<const uint4*>(w + col);
      uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = unpack_bf16(ww[j]);
        wv[c][2 * j] = f.x;
        wv[c][2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[c][j] = 0.f;
    }
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += 8) {
    const float r = rstd[row];
    float xv[CHUNKS][8], gv[CHUNKS][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < D) {
        uint4 xu = *reinterpret_cast<const uint4*>(x + (long long)row * ldx + col);
        uint4 gu = *reinterpret_cast<const uint4*>(dy + (long long)row * lddy + col);
        uint32_t xx[4] = {xu.x, xu.y, xu.z, xu.w}, gg[4] = {gu.x, gu.y, gu.z, gu.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 xf = unpack_bf16(xx[j]), gf = unpack_bf16(gg[j]);
          xv[c][2 * j] = xf.x;
          xv[c][2 * j + 1] = xf.y;
          gv[c][2 * j] = gf.x;
          gv[c][2 * j + 1] = gf.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[c][j] = gv[c][j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        dot += gv[c][j] * wv[c][j] * xv[c][j];
        acc[c][j] += gv[c][j] * xv[c][j] * r;
      }
    }
    dot = warp_sum(dot);
    const float k = dot * r * r * r / (float)D;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < D) {
        float add[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (dres) {  // gradient of the residual branch that also reads x
          const uint4 ru = *reinterpret_cast<const uint4*>(dres + (long long)row * ldres + col);
          const uint32_t rr[4] = {ru.x, ru.y, ru.z, ru.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_bf16(rr[j]);
            add[2 * j] = f.x;
            add[2 * j + 1] = f.y;
          }
        }
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = pack_bf16(r * wv[c][2 * j] * gv[c][2 * j] - xv[c][2 * j] * k + add[2 * j],
                           r * wv[c][2 * j + 1] * gv[c][2 * j + 1] - xv[c][2 * j + 1] * k + add[2 * j + 1]);
        *reinterpret_cast<uint4*>(dx + (long long)row * lddx + col) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  // reduce the 8 warps' partial dw through shared memory, one row per block
  extern __shared__ float red[];  // [8][D]
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < D) {
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp * D + col + j] = acc[c][j];
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k * D + col];
    dw_part[(long long)blockIdx.x * D + col] = s;
  }
}

// Small-D backward (D <= 256): one warp per row, dw partial per block.
__global__ void __launch_bounds__(256) rmsnorm_bwd_small_kernel(const __nv_bfloat16* __restrict__ dy, long long lddy,
                                                                const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                const __nv_bfloat16* __restrict__ w,
                                                                const float* __restrict__ rstd,
                                                                __nv_bfloat16* __restrict__ dx, long long lddx,
                                                                const __nv_bfloat16* __restrict__ dres,
                                                                long long ldres, float* __restrict__ dw_part, int rows,
                                                                int D, int rows_per_block) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = D / 32;
  float wv[8], acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    wv[j] = j < per ? __bfloat162float(w[lane * per + j]) : 0.f;
    acc[j] = 0.f;
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += 8) {
    const float r = rstd[row];
    float xv[8], gv[8], dot = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xv[j] = j < per ? __bfloat162float(x[(long long)row * ldx + lane * per + j]) : 0.f;
      gv[j] = j < per ? __bfloat162float(dy[(long long)row * lddy + lane * per + j]) : 0.f;
      dot += gv[j] * wv[j] * xv[j];
      acc[j] += gv[j] * xv[j] * r;
    }
    dot = warp_sum(dot);
    const float k = dot * r * r * r / (float)D;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < per)
        dx[(long long)row * lddx + lane * per + j] = __float2bfloat16_rn(
            r * wv[j] * gv[j] - xv[j] * k +
            (dres ? __bfloat162float(dres[(long long)row * ldres + lane * per + j]) : 0.f));
  }
  __shared__ float red[8][256];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j < per) red[warp][lane * per + j] = acc[j];
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][col];
    dw_part[(long long)blockIdx.x * D + col] = s;
  }
}

// dw[col] = sum_b part[b, col]
__global__ void reduce_cols_kernel(const float* __restrict__ part, int nblocks, int D, __nv_bfloat16* __restrict__ out_bf16,
                                   float* __restrict__ out_f32) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= D) return;
  float s = 0.f;
  for (int b = 0; b < nblocks; ++b) s += part[(long long)b * D + col];
  if (out_f32) out_f32[col] = s;
  if (out_bf16) out_bf16[col] = __float2bfloat16_rn(s);
}

}  // namespace astrai

namespace astrai_host {

void rmsnorm_fwd(const void* x, long long ldx, const void* w, void* y, long long ldy, float* rstd, int rows, int D,
                 float eps, cudaStream_t s) {
  using namespace astrai;
  const int grid = (rows + 7) / 8;
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto Y = static_cast<__nv_bfloat16*>(y);
  if (D <= 256 && D % 32 == 0) {
    (astrai::note_launch(), rmsnorm_fwd_small_kernel<<<grid, 256, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps));
  } else if (D <= 1024) {
    (astrai::note_launch(), rmsnorm_fwd_kernel<4><<<grid, 256, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps));
  } else if (D <= 2048) {
    (astrai::note_launch(), rmsnorm_fwd_kernel<8><<<grid, 256, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps));
  } else if (D <= 4096) {
    (astrai::note_launch(), rmsnorm_fwd_kernel<16><<<grid, 256, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps));
  } else {
    (astrai::note_launch(), rmsnorm_fwd_kernel<32><<<grid, 256, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps));
  }
}

// Number of fp32 scratch elements rmsnorm_bwd needs for dw partials.
long long rmsnorm_bwd_scratch(int rows, int D, int* nblocks_out) {
  const int rpb = 64;
  const int nb = (rows + rpb - 1) / rpb;
  if (nblocks_out) *nblocks_out = nb;
  return (long long)nb * D;
}

void rmsnorm_bwd(const void* dy, long long lddy, const void* x, long long ldx, const void* w, const float* rstd,
                 void* dx, long long lddx, void* dw_bf16, float* dw_f32, float* scratch, int rows, int D,
                 cudaStream_t s, const void* dres, long long ldres) {
  using namespace astrai;
  int nb = 0;
  rmsnorm_bwd_scratch(rows, D, &nb);
  const int rpb = 64;
  auto DY = static_cast<const __nv_bfloat16*>(dy);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto DX = static_cast<__nv_bfloat16*>(dx);
  auto DR = static_cast<const __nv_bfloat16*>(dres);
  const size_t sm = (size_t)8 * D * sizeof(float);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaFuncSetAttribute(rmsnorm_bwd_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 1024 * 4);
    cudaFuncSetAttribute(rmsnorm_bwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 2048 * 4);
    cudaFuncSetAttribute(rmsnorm_bwd_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 4096 * 4);
    attr_done[dev & 63] = true;
  }
  if (D <= 256 && D % 32 == 0) {
    (astrai::note_launch(), rmsnorm_bwd_small_kernel<<<nb, 256, 0, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
  } else if (D <= 1024) {
    (astrai::note_launch(), rmsnorm_bwd_kernel<4><<<nb, 256, sm, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
  } else if (D <= 2048) {
    (astrai::note_launch(), rmsnorm_bwd_kernel<8><<<nb, 256, sm, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
  } else {
    (astrai::note_launch(), rmsnorm_bwd_kernel<16><<<nb, 256, sm, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
  }
  (astrai::note_launch(), reduce_cols_kernel<<<(D + 255) / 256, 256, 0, s>>>(scratch, nb, D, static_cast<__nv_bfloat16*>(dw_bf16), dw_f32));
}

}  // namespace astrai_host

// ---------------------------------------------------------------------------
// Allocation-free RMSNorm backward (declared and documented in astrai_c_api.h;
// no counterpart in the reference project). Same kernels as rmsnorm_bwd above,
// with the dw partials in a fixed device array instead of caller scratch.
#include <cstdio>
#include <mutex>

#include "astrai_c_api.h"

namespace {

static __device__ __align__(256) float g_rmsnorm_bwd_scratch[ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};
cudaError_t g_setup_err[kMaxDevices] = {};
std::once_flag g_setup_once[kMaxDevices];

// Once per device, with that device current: the array's address and the
// kernels' dynamic shared-memory limits. Allocates nothing.
void static_scratch_setup(int dev) {
  float* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_rmsnorm_bwd_scratch);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(astrai::rmsnorm_bwd_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 1024 * 4);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(astrai::rmsnorm_bwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 2048 * 4);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(astrai::rmsnorm_bwd_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 4096 * 4);
  g_setup_err[dev] = e;
  g_scratch_ptr[dev] = e == cudaSuccess ? p : nullptr;
}

}  // namespace

extern "C" int astrai_rmsnorm_bwd_static_scratch(const void* dy, long long lddy, const void* x, long long ldx,
                                                 const void* w, const float* rstd, void* dx, long long lddx,
                                                 void* dw_bf16, float* dw_f32, int rows, int D, void* stream) {
  using namespace astrai;
  if (rows <= 0 || D <= 0 || D % 8 != 0 || D > 4096) {
    std::fprintf(stderr, "astrai_rmsnorm_bwd_static_scratch: unsupported shape rows=%d D=%d "
                         "(need rows > 0, D a multiple of 8, D <= 4096)\n", rows, D);
    return -1;
  }
  const int rpb = 64;
  const long long nb = (static_cast<long long>(rows) + rpb - 1) / rpb;
  const long long need = nb * D;
  if (need > ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS) {
    std::fprintf(stderr, "astrai_rmsnorm_bwd_static_scratch: rows=%d D=%d needs %lld floats of scratch, "
                         "more than the %lld in the static array\n", rows, D, need,
                 static_cast<long long>(ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS));
    return -1;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) {
    std::fprintf(stderr, "astrai_rmsnorm_bwd_static_scratch: device %d is beyond the supported %d\n", dev,
                 kMaxDevices);
    return -1;
  }
  std::call_once(g_setup_once[dev], static_scratch_setup, dev);
  if (g_setup_err[dev] != cudaSuccess) return static_cast<int>(g_setup_err[dev]);
  float* scratch = g_scratch_ptr[dev];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto DY = static_cast<const __nv_bfloat16*>(dy);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto DX = static_cast<__nv_bfloat16*>(dx);
  const int blocks = static_cast<int>(nb);
  const size_t sm = static_cast<size_t>(8) * D * sizeof(float);
  if (D <= 256 && D % 32 == 0) {
    (astrai::note_launch(), rmsnorm_bwd_small_kernel<<<blocks, 256, 0, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, nullptr, 0, scratch, rows, D, rpb));
  } else if (D <= 1024) {
    (astrai::note_launch(), rmsnorm_bwd_kernel<4><<<blocks, 256, sm, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, nullptr, 0, scratch, rows, D, rpb));
  } else if (D <= 2048) {
    (astrai::note_launch(), rmsnorm_bwd_kernel<8><<<blocks, 256, sm, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, nullptr, 0, scratch, rows, D, rpb));
  } else {
    (astrai::note_launch(), rmsnorm_bwd_kernel<16><<<blocks, 256, sm, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, nullptr, 0, scratch, rows, D, rpb));
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  (astrai::note_launch(), reduce_cols_kernel<<<(D + 255) / 256, 256, 0, s>>>(scratch, blocks, D, static_cast<__nv_bfloat16*>(dw_bf16),
                                                     dw_f32));
  return static_cast<int>(cudaGetLastError());
}
