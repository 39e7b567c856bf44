// Skinny GEMM for decode: Y[M, N] = X[M, K] @ W[N, K]^T (+ residual), M <= 16.
//
// Decode steps multiply a handful of token rows by every weight matrix once,
// so the cost is reading W from HBM (N * K * 2 bytes); the 128-row tensor-core
// tiles of the training GEMM would launch only N / 256 CTAs. Here every warp
// streams two weight rows with 16-byte loads (UNROLL chunks = 2 * UNROLL loads
// in flight per lane before any math) and multiplies them with the token rows
// (read through L1: they are tiny and shared by all warps). K is split over
// the KS CTAs of a thread-block cluster; the cluster reduces its partial dot
// products through distributed shared memory and its first CTA adds the
// residual and writes bf16 Y. One launch per product: no workspace, no
// atomics, no second kernel.
#include <cooperative_groups.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace astrai {

constexpr int SK_WARPS = 8;   // warps per CTA
constexpr int SK_COLS = 2;    // output columns per warp
constexpr int SK_UNROLL = 4;  // 256-element K chunks loaded before the math

template <int MT>
__global__ void __launch_bounds__(SK_WARPS * 32) skinny_gemm_kernel(const __nv_bfloat16* __restrict__ X, long long ldx,
                                                                    const __nv_bfloat16* __restrict__ W, long long ldw,
                                                                    const __nv_bfloat16* __restrict__ R, long long ldr,
                                                                    __nv_bfloat16* __restrict__ Y, long long ldy, int M,
                                                                    int N, int K, int kchunk) {
  __shared__ float part[SK_WARPS][MT][SK_COLS];
  cg::cluster_group cl = cg::this_cluster();
  const int ks = (int)cl.num_blocks();
  const int kr = ks > 1 ? (int)cl.block_rank() : 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n0 = (blockIdx.x * SK_WARPS + warp) * SK_COLS;
  const bool live = n0 < N;
  const bool has1 = n0 + 1 < N;
  const int kb = kr * kchunk;
  const int ke = min(K, kb + kchunk);
  float s[MT][SK_COLS];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < SK_COLS; ++c) s[m][c] = 0.f;
  // Programmatic dependent launch: this grid may start while the kernel before it (which writes X
  // or R) is still running. The weights do not depend on it, so their lines are prefetched into L2
  // first; X and R are read only after griddepcontrol.wait (the previous grid complete and its
  // memory visible). Nothing is written before the wait. The next kernel may launch as soon as every
  // CTA of this one has started.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (live) {
    const char* r0p = reinterpret_cast<const char*>(W + (long long)n0 * ldw + kb);
    const char* r1p = reinterpret_cast<const char*>(W + (long long)(has1 ? n0 + 1 : n0) * ldw + kb);
    const int lines = ((ke - kb) * 2 + 127) / 128;
    for (int l = lane; l < lines; l += 32) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(r0p + l * 128));
      if (has1) asm volatile("prefetch.global.L2 [%0];" ::"l"(r1p + l * 128));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (live) {
    const __nv_bfloat16* w0 = W + (long long)n0 * ldw;
    const __nv_bfloat16* w1 = W + (long long)(has1 ? n0 + 1 : n0) * ldw;
    for (int k0 = kb + lane * 8; k0 < ke; k0 += 256 * SK_UNROLL) {
      uint4 a[SK_UNROLL], b[SK_UNROLL];
#pragma unroll
      for (int u = 0; u < SK_UNROLL; ++u) {
        const int k = k0 + u * 256;
        if (k < ke) {
          a[u] = __ldg(reinterpret_cast<const uint4*>(w0 + k));
          b[u] = __ldg(reinterpret_cast<const uint4*>(w1 + k));
        } else {
          a[u] = b[u] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < SK_UNROLL; ++u) {
        const int k = k0 + u * 256;
        if (k >= ke) continue;
        float wa[8], wb[8];
        const uint32_t ua[4] = {a[u].x, a[u].y, a[u].z, a[u].w}, ub[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fa = unpack_bf16(ua[j]), fb = unpack_bf16(ub[j]);
          wa[2 * j] = fa.x;
          wa[2 * j + 1] = fa.y;
          wb[2 * j] = fb.x;
          wb[2 * j + 1] = fb.y;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < M) {
            const uint4 xv = __ldg(reinterpret_cast<const uint4*>(X + (long long)m * ldx + k));
            const uint32_t ux[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 fx = unpack_bf16(ux[j]);
              s[m][0] += fx.x * wa[2 * j] + fx.y * wa[2 * j + 1];
              s[m][1] += fx.x * wb[2 * j] + fx.y * wb[2 * j + 1];
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < SK_COLS; ++c) s[m][c] = warp_sum(s[m][c]);
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < SK_COLS; ++c) part[warp][m][c] = s[m][c];
  }
  if (ks > 1) cl.sync(); else __syncthreads();
  if (kr == 0) {
    // thread t of the first CTA finishes output (m, n0 + c) of warp w
    for (int t = threadIdx.x; t < SK_WARPS * MT * SK_COLS; t += blockDim.x) {
      const int w = t / (MT * SK_COLS), m = (t / SK_COLS) % MT, c = t % SK_COLS;
      const int n = (blockIdx.x * SK_WARPS + w) * SK_COLS + c;
      if (m >= M || n >= N) continue;
      float v = 0.f;
      for (int r = 0; r < ks; ++r) v += ks > 1 ? *cl.map_shared_rank(&part[w][m][c], r) : part[w][m][c];
      if (R) v += __bfloat162float(R[(long long)m * ldr + n]);
      Y[(long long)m * ldy + n] = __float2bfloat16_rn(v);
    }
  }
  if (ks > 1) cl.sync();  // peers keep their shared memory until the first CTA has read it
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

// ASTRAI_SKINNY_PDL=0 launches the skinny GEMM only after the previous kernel ends
static bool skinny_pdl() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_SKINNY_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int MT>
static void launch_skinny(dim3 grid, int ks, cudaStream_t s, const __nv_bfloat16* X, long long ldx,
                          const __nv_bfloat16* W, long long ldw, const __nv_bfloat16* R, long long ldr,
                          __nv_bfloat16* Y, long long ldy, int M, int N, int K, int kchunk) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(SK_WARPS * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ks;
  attr[0].val.clusterDim.z = 1;
  // may start before the previous kernel on the stream ends (the kernel waits before reading X)
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = skinny_pdl() ? 2 : 1;
  note_launch();
  const cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_gemm_kernel<MT>, X, ldx, W, ldw, R, ldr, Y, ldy, M, N, K,
                                           kchunk);
  if (e != cudaSuccess) throw std::runtime_error(std::string("skinny_gemm: launch failed: ") + cudaGetErrorString(e));
}

void skinny_gemm(const void* X, long long ldx, const void* W, long long ldw, const void* residual, long long ldr,
                 void* Y, long long ldy, int M, int N, int K, int sms, cudaStream_t s) {
  if (M < 1 || M > 16) throw std::runtime_error("skinny_gemm: 1 <= M <= 16");
  if (K % 8) throw std::runtime_error("skinny_gemm: K must be a multiple of 8");
  const int cols_per_cta = SK_WARPS * SK_COLS;
  const int gx = (N + cols_per_cta - 1) / cols_per_cta;
  // K split into whole 256-element chunks over a cluster of up to 8 CTAs, aiming
  // at >= 2 CTAs per SM while every warp keeps at least 4 chunks of work
  const int chunks = (K + 255) / 256;
  int ks = std::max(1, std::min(8, (2 * sms + gx - 1) / gx));
  ks = std::min(ks, std::max(1, chunks / 4));
  const int kchunk = ((chunks + ks - 1) / ks) * 256;
  ks = (K + kchunk - 1) / kchunk;
  dim3 grid(gx, ks);
  auto Xp = static_cast<const __nv_bfloat16*>(X);
  auto Wp = static_cast<const __nv_bfloat16*>(W);
  auto Rp = static_cast<const __nv_bfloat16*>(residual);
  auto Yp = static_cast<__nv_bfloat16*>(Y);
  if (M <= 1) launch_skinny<1>(grid, ks, s, Xp, ldx, Wp, ldw, Rp, ldr, Yp, ldy, M, N, K, kchunk);
  else if (M <= 2) launch_skinny<2>(grid, ks, s, Xp, ldx, Wp, ldw, Rp, ldr, Yp, ldy, M, N, K, kchunk);
  else if (M <= 4) launch_skinny<4>(grid, ks, s, Xp, ldx, Wp, ldw, Rp, ldr, Yp, ldy, M, N, K, kchunk);
  else if (M <= 8) launch_skinny<8>(grid, ks, s, Xp, ldx, Wp, ldw, Rp, ldr, Yp, ldy, M, N, K, kchunk);
  else launch_skinny<16>(grid, ks, s, Xp, ldx, Wp, ldw, Rp, ldr, Yp, ldy, M, N, K, kchunk);
}

}  // namespace astrai_host
