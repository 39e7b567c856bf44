// RMSNorm forward / backward (sm_100a, bandwidth-bound).
//
//   y = x * rsqrt(mean(x^2) + eps) * w          (astrai/model/components/norm.py:14-15)
//
// Block per row: the 256 threads of a block share one row, each owning V fixed groups of 8
// columns (16-byte loads and stores), and a block walks a contiguous range of rows. The loads of
// row i + 1 are issued before row i's block-wide reduction, so each thread keeps one row's worth
// of DRAM reads in flight while it waits on the reduction barrier; with every block resident
// (about 4 per SM) that is enough memory parallelism to approach copy bandwidth. Rows are
// processed in fp32. Backward writes dx (plus the residual-branch gradient when given) and one
// fp32 dw partial per block, which stays in registers over the block's rows; a second kernel sums
// the partials (dw is a sum over all rows). Small D (<= 256, per-head norms) uses one warp per row.
#include <algorithm>

#include "common.cuh"

namespace astrai {

constexpr int kNormThreads = 256;
constexpr int kNormBlocksTarget = 592;     // forward: 4 resident 256-thread blocks on each of 148 SMs
constexpr int kNormBwdBlocksTarget = 444;  // backward (<= 85 registers): 3 per SM, one wave

// Sum of v over the block (nw warps), through red[buf] (double-buffered by the caller so that one
// barrier per row suffices: a buffer is rewritten only after the next row's barrier).
__device__ __forceinline__ float block_sum(float v, float* red, int nw) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int k = 0; k < nw; ++k) t += red[k];
  return t;
}

template <int V>  // 8-column groups per thread; D <= V * 8 * blockDim.x
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   __nv_bfloat16* __restrict__ y, long long ldy,
                                                                   float* __restrict__ rstd_out, int rows, int D,
                                                                   float eps, int rows_per_block) {
  // a kernel launched after this one with programmatic dependent launch may start now (it waits for
  // this grid to finish before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float red[2][32];
  const int T = blockDim.x, nw = T >> 5;
  int col[V];
  uint4 wp[V], cur[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    col[v] = (v * T + threadIdx.x) * 8;
    wp[v] = col[v] < D ? *reinterpret_cast<const uint4*>(w + col[v]) : make_uint4(0u, 0u, 0u, 0u);
  }
  const int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
#pragma unroll
  for (int v = 0; v < V; ++v)
    cur[v] = (r0 < r1 && col[v] < D) ? *reinterpret_cast<const uint4*>(x + (long long)r0 * ldx + col[v])
                                     : make_uint4(0u, 0u, 0u, 0u);
  for (int row = r0; row < r1; ++row) {
    uint4 nxt[V];
#pragma unroll
    for (int v = 0; v < V; ++v)
      nxt[v] = (row + 1 < r1 && col[v] < D) ? *reinterpret_cast<const uint4*>(x + (long long)(row + 1) * ldx + col[v])
                                            : make_uint4(0u, 0u, 0u, 0u);
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const uint32_t u[4] = {cur[v].x, cur[v].y, cur[v].z, cur[v].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16(u[j]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    ss = block_sum(ss, red[row & 1], nw);
    const float r = rsqrtf(ss / (float)D + eps);
    if (threadIdx.x == 0 && rstd_out) rstd_out[row] = r;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (col[v] < D) {
        const uint32_t u[4] = {cur[v].x, cur[v].y, cur[v].z, cur[v].w};
        const uint32_t ww[4] = {wp[v].x, wp[v].y, wp[v].z, wp[v].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16(u[j]), wf = unpack_bf16(ww[j]);
          o[j] = pack_bf16(f.x * r * wf.x, f.y * r * wf.y);
        }
        *reinterpret_cast<uint4*>(y + (long long)row * ldy + col[v]) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      cur[v] = nxt[v];
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

// dx = r*w*dy - x * r^3 * mean(dy*w*x) (+ dres);   dw_partial[block] = sum over the block's rows of dy*x*r
// Issue-bound at this size once the loads overlap, so the inner loop is kept short: w is
// converted to fp32 once per block, each row's x and dy once (g*w is reused by the dot product and
// by dx), and dx / dw are single FMAs per element.
template <int V>
__global__ void __launch_bounds__(kNormThreads, V == 1 ? 3 : 2) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long long lddy,
                                                                   const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   const float* __restrict__ rstd,
                                                                   __nv_bfloat16* __restrict__ dx, long long lddx,
                                                                   const __nv_bfloat16* __restrict__ dres,
                                                                   long long ldres, float* __restrict__ dw_part,
                                                                   int rows, int D, int rows_per_block) {
  __shared__ float red[2][32];
  const int T = blockDim.x, nw = T >> 5;
  int col[V];
  float wf[V][8], acc[V][8];
  uint4 cx[V], cg[V], cr[V];
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int v = 0; v < V; ++v) {
    col[v] = (v * T + threadIdx.x) * 8;
    const uint4 wu = col[v] < D ? *reinterpret_cast<const uint4*>(w + col[v]) : z;
    const uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16(ww[j]);
      wf[v][2 * j] = f.x;
      wf[v][2 * j + 1] = f.y;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[v][j] = 0.f;
  }
  const int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
  const __nv_bfloat16* xp = x + (long long)r0 * ldx;
  const __nv_bfloat16* gp = dy + (long long)r0 * lddy;
  const __nv_bfloat16* rp = dres ? dres + (long long)r0 * ldres : nullptr;
  __nv_bfloat16* op = dx + (long long)r0 * lddx;
  float crs = r0 < r1 ? rstd[r0] : 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const bool ok = r0 < r1 && col[v] < D;
    cx[v] = ok ? *reinterpret_cast<const uint4*>(xp + col[v]) : z;
    cg[v] = ok ? *reinterpret_cast<const uint4*>(gp + col[v]) : z;
    cr[v] = (ok && rp) ? *reinterpret_cast<const uint4*>(rp + col[v]) : z;
  }
  for (int row = r0; row < r1; ++row) {
    // next row's loads first: they overlap this row's reduction
    const bool more = row + 1 < r1;
    const float nrs = more ? rstd[row + 1] : 0.f;
    uint4 nx[V], ng[V], nr[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const bool ok = more && col[v] < D;
      nx[v] = ok ? *reinterpret_cast<const uint4*>(xp + ldx + col[v]) : z;
      ng[v] = ok ? *reinterpret_cast<const uint4*>(gp + lddy + col[v]) : z;
      nr[v] = (ok && rp) ? *reinterpret_cast<const uint4*>(rp + ldres + col[v]) : z;
    }
    float xf[V][8], gw[V][8], gf[V][8];
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const uint32_t xx[4] = {cx[v].x, cx[v].y, cx[v].z, cx[v].w}, gg[4] = {cg[v].x, cg[v].y, cg[v].z, cg[v].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack_bf16(xx[j]), b = unpack_bf16(gg[j]);
        xf[v][2 * j] = a.x;
        xf[v][2 * j + 1] = a.y;
        gf[v][2 * j] = b.x;
        gf[v][2 * j + 1] = b.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        gw[v][j] = gf[v][j] * wf[v][j];
        dot = fmaf(gw[v][j], xf[v][j], dot);
      }
    }
    dot = block_sum(dot, red[row & 1], nw);
    const float r = crs, nk = -dot * r * r * r / (float)D;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (col[v] < D) {
        const uint32_t rr[4] = {cr[v].x, cr[v].y, cr[v].z, cr[v].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 af = unpack_bf16(rr[j]);
          o[j] = pack_bf16(fmaf(r, gw[v][2 * j], fmaf(xf[v][2 * j], nk, af.x)),
                           fmaf(r, gw[v][2 * j + 1], fmaf(xf[v][2 * j + 1], nk, af.y)));
        }
        *reinterpret_cast<uint4*>(op + col[v]) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[v][j] = fmaf(gf[v][j] * r, xf[v][j], acc[v][j]);
      }
      cx[v] = nx[v];
      cg[v] = ng[v];
      cr[v] = nr[v];
    }
    crs = nrs;
    xp += ldx;
    gp += lddy;
    if (rp) rp += ldres;
    op += lddx;
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    if (col[v] < D) {
      float4* o = reinterpret_cast<float4*>(dw_part + (long long)blockIdx.x * D + col[v]);
      o[0] = make_float4(acc[v][0], acc[v][1], acc[v][2], acc[v][3]);
      o[1] = make_float4(acc[v][4], acc[v][5], acc[v][6], acc[v][7]);
    }
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

// dw[col] = sum_b part[b, col]: 8 columns (one 32-byte sector per partial row) per block of 1024
// threads, the partial rows split over 128 thread rows with 2 accumulators each, then a tree sum
// through smem. D / 8 blocks spread the reads over the SMs.
__global__ void __launch_bounds__(1024) reduce_cols_kernel(const float* __restrict__ part, int nblocks, int D,
                                                           __nv_bfloat16* __restrict__ out_bf16,
                                                           float* __restrict__ out_f32) {
  __shared__ float s[128][9];
  const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
  const int col = blockIdx.x * 8 + tx;
  float a0 = 0.f, a1 = 0.f;
  if (col < D) {
    int b = ty;
    for (; b + 128 < nblocks; b += 256) {
      a0 += part[(long long)b * D + col];
      a1 += part[(long long)(b + 128) * D + col];
    }
    if (b < nblocks) a0 += part[(long long)b * D + col];
  }
  s[ty][tx] = a0 + a1;
  __syncthreads();
#pragma unroll
  for (int h = 64; h > 0; h >>= 1) {
    if (ty < h) s[ty][tx] += s[ty + h][tx];
    __syncthreads();
  }
  if (ty == 0 && col < D) {
    const float t = s[0][tx];
    if (out_f32) out_f32[col] = t;
    if (out_bf16) out_bf16[col] = __float2bfloat16_rn(t);
  }
}

}  // namespace astrai

namespace astrai_host {

// Rows per block for the block-per-row kernels: about `target` blocks (at most `cap`), each a
// contiguous range of rows.
static int norm_rows_per_block(int rows, long long cap, int target = astrai::kNormBwdBlocksTarget) {
  long long nb = std::min<long long>(std::min<long long>(rows, target), std::max(1LL, cap));
  return (int)((rows + nb - 1) / nb);
}
static bool norm_small(int D) { return D <= 256 && D % 32 == 0; }
constexpr int kSmallRowsPerBlock = 64;

void rmsnorm_fwd(const void* x, long long ldx, const void* w, void* y, long long ldy, float* rstd, int rows, int D,
                 float eps, cudaStream_t s) {
  using namespace astrai;
  if (rows <= 0) return;
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto Y = static_cast<__nv_bfloat16*>(y);
  if (norm_small(D)) {
    (astrai::note_launch(), rmsnorm_fwd_small_kernel<<<(rows + 7) / 8, 256, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps));
    return;
  }
  const int rpb = norm_rows_per_block(rows, 1LL << 30, kNormBlocksTarget);
  const int nb = (rows + rpb - 1) / rpb;
  const int T = std::min(kNormThreads, ((D / 8 + 31) / 32) * 32);
  if (D <= 8 * kNormThreads)
    (astrai::note_launch(), rmsnorm_fwd_kernel<1><<<nb, T, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps, rpb));
  else if (D <= 16 * kNormThreads)
    (astrai::note_launch(), rmsnorm_fwd_kernel<2><<<nb, kNormThreads, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps, rpb));
  else
    (astrai::note_launch(), rmsnorm_fwd_kernel<4><<<nb, kNormThreads, 0, s>>>(X, ldx, W, Y, ldy, rstd, rows, D, eps, rpb));
}

// Launch the backward kernels for nb blocks of rpb rows; dw partials go to scratch [nb][D].
static void rmsnorm_bwd_launch(const void* dy, long long lddy, const void* x, long long ldx, const void* w,
                               const float* rstd, void* dx, long long lddx, const void* dres, long long ldres,
                               void* dw_bf16, float* dw_f32, float* scratch, int rows, int D, int nb, int rpb,
                               cudaStream_t s) {
  using namespace astrai;
  auto DY = static_cast<const __nv_bfloat16*>(dy);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto DX = static_cast<__nv_bfloat16*>(dx);
  auto DR = static_cast<const __nv_bfloat16*>(dres);
  if (norm_small(D)) {
    (astrai::note_launch(), rmsnorm_bwd_small_kernel<<<nb, 256, 0, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
  } else {
    const int T = std::min(kNormThreads, ((D / 8 + 31) / 32) * 32);
    if (D <= 8 * kNormThreads)
      (astrai::note_launch(), rmsnorm_bwd_kernel<1><<<nb, T, 0, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
    else
      (astrai::note_launch(), rmsnorm_bwd_kernel<2><<<nb, kNormThreads, 0, s>>>(DY, lddy, X, ldx, W, rstd, DX, lddx, DR, ldres, scratch, rows, D, rpb));
  }
  (astrai::note_launch(), reduce_cols_kernel<<<(D + 7) / 8, 1024, 0, s>>>(scratch, nb, D, static_cast<__nv_bfloat16*>(dw_bf16), dw_f32));
}

// Number of fp32 scratch elements rmsnorm_bwd needs for dw partials.
long long rmsnorm_bwd_scratch(int rows, int D, int* nblocks_out) {
  const int rpb = norm_small(D) ? kSmallRowsPerBlock : norm_rows_per_block(rows, 1LL << 30);
  const int nb = (rows + rpb - 1) / rpb;
  if (nblocks_out) *nblocks_out = nb;
  return (long long)nb * D;
}

void rmsnorm_bwd(const void* dy, long long lddy, const void* x, long long ldx, const void* w, const float* rstd,
                 void* dx, long long lddx, void* dw_bf16, float* dw_f32, float* scratch, int rows, int D,
                 cudaStream_t s, const void* dres, long long ldres) {
  if (rows <= 0) return;
  int nb = 0;
  rmsnorm_bwd_scratch(rows, D, &nb);
  const int rpb = (rows + nb - 1) / nb;
  rmsnorm_bwd_launch(dy, lddy, x, ldx, w, rstd, dx, lddx, dres, ldres, dw_bf16, dw_f32, scratch, rows, D, nb, rpb, s);
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
std::mutex g_setup_mutex;

// The array's device address on the current device `dev`. Looked up once per device with that device
// current and kept for the life of the process; a failed lookup is not kept, so a later call retries.
// Allocates nothing.
cudaError_t static_scratch_address(int dev, float** out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    float* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_rmsnorm_bwd_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int astrai_rmsnorm_bwd_static_scratch(const void* dy, long long lddy, const void* x, long long ldx,
                                                 const void* w, const float* rstd, void* dx, long long lddx,
                                                 void* dw_bf16, float* dw_f32, int rows, int D, void* stream) {
  if (rows <= 0 || D <= 0 || D % 8 != 0 || D > 4096) {
    std::fprintf(stderr, "astrai_rmsnorm_bwd_static_scratch: unsupported shape rows=%d D=%d "
                         "(need rows > 0, D a multiple of 8, D <= 4096)\n", rows, D);
    return -1;
  }
  // Size rule (documented in astrai_c_api.h, independent of the launch's block count): the problem
  // is accepted when ceil(rows / 64) * D floats fit the static array.
  const long long need = (static_cast<long long>(rows) + 63) / 64 * D;
  if (need > ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS) {
    std::fprintf(stderr, "astrai_rmsnorm_bwd_static_scratch: rows=%d D=%d needs %lld floats of scratch, "
                         "more than the %lld in the static array\n", rows, D, need,
                 static_cast<long long>(ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS));
    return -1;
  }
  // the launch itself uses at most ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS / D blocks
  const long long cap = ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS / D;
  const int rpb = astrai_host::norm_small(D) ? astrai_host::kSmallRowsPerBlock
                                             : astrai_host::norm_rows_per_block(rows, cap);
  const long long nb = (static_cast<long long>(rows) + rpb - 1) / rpb;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) {
    std::fprintf(stderr, "astrai_rmsnorm_bwd_static_scratch: device %d is beyond the supported %d\n", dev,
                 kMaxDevices);
    return -1;
  }
  float* scratch = nullptr;
  e = static_scratch_address(dev, &scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  astrai_host::rmsnorm_bwd_launch(dy, lddy, x, ldx, w, rstd, dx, lddx, nullptr, 0, dw_bf16, dw_f32, scratch, rows,
                                  D, static_cast<int>(nb), rpb, static_cast<cudaStream_t>(stream));
  // the runtime's per-thread last error: this call's launches, or an error that earlier runtime calls
  // of the calling thread left pending (reported and cleared here, as the header states)
  return static_cast<int>(cudaGetLastError());
}
