// Fully sharded data parallelism over NVLink peer memory (sm_100a): the
// gradient reduction to parameter owners and the epoch flags around it.
//
// Every parameter has one owner rank (astrai_b200/parallel/fsdp.py). All ranks
// accumulate full-size bf16 gradients into a symmetric (CUDA IPC) pool with
// the same layout everywhere, so rank q's gradient of a parameter is
// grad_base[q] + offset. After the last micro-batch each owner runs
//
//   fsdp_reduce_kernel: g = (1 / world) * sum_q grad_q   (fp32 sum, bf16 out)
//
// over its own parameters only: it pulls the W - 1 peer copies over NVLink
// with 16-byte loads (four vectors per thread in flight per peer), writes the
// mean into its local gradient (in place) and adds the squared L2 norm of the
// means into a device scalar for clipping. That is the reduce-scatter of the
// reference's FSDP2 (astrai/parallel/executor.py:339-376, one NCCL
// reduce-scatter per wrapped module and micro-batch when gradients sync),
// fused with the cast, the 1/world scale and the norm, once per optimizer step.
//
// Flags: a block of u32 words [rows][world] in the symmetric pool;
// fsdp_raise_kernel stores `epoch` into row `row`, column `rank`, of every
// peer (release, system scope); peer_flags_wait (dist_optim.cu) waits,
// bounded, until every peer's word of a row reached the epoch.
#include <stdexcept>

#include "common.cuh"

namespace astrai {

namespace {

__device__ __forceinline__ void st_release_u32_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

}  // namespace

constexpr int FR_THREADS = 256;
constexpr int FR_UNROLL = 4;
constexpr int FR_MAX_WORLD = 16;

struct FsdpReduceParams {
  const long long* peer_grad;  // [world] gradient pool base of every rank, mapped here
  const long long* seg_off;    // [n_seg] byte offsets of the owned gradients in the pool
  const long long* seg_vec;    // [n_seg + 1] prefix sums of 16-byte vectors per segment
  int n_seg, rank, world;
  float scale;
  float* sumsq;                // += squared norm of the reduced gradients
};

__device__ __forceinline__ void acc8(float (&a)[8], const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16(w[i]);
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}

__global__ void __launch_bounds__(FR_THREADS) fsdp_reduce_kernel(FsdpReduceParams p) {
  const long long total = p.seg_vec[p.n_seg];
  const long long stride = (long long)gridDim.x * FR_THREADS;
  float sq = 0.f;
  int seg = 0;
  for (long long v0 = (long long)blockIdx.x * FR_THREADS + threadIdx.x; v0 < total; v0 += stride * FR_UNROLL) {
    long long vi[FR_UNROLL];
    long long off[FR_UNROLL];
#pragma unroll
    for (int u = 0; u < FR_UNROLL; ++u) {
      vi[u] = v0 + u * stride;
      off[u] = -1;
      if (vi[u] < total) {
        // segments are visited in increasing order by every thread: advance, never search back
        while (p.seg_vec[seg + 1] <= vi[u]) ++seg;
        off[u] = p.seg_off[seg] + (vi[u] - p.seg_vec[seg]) * 16;
      }
    }
    float a[FR_UNROLL][8];
#pragma unroll
    for (int u = 0; u < FR_UNROLL; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) a[u][i] = 0.f;
    for (int q = 0; q < p.world; ++q) {
      const char* base = reinterpret_cast<const char*>(p.peer_grad[q]);
      uint4 v[FR_UNROLL];
#pragma unroll
      for (int u = 0; u < FR_UNROLL; ++u)
        if (off[u] >= 0) v[u] = *reinterpret_cast<const uint4*>(base + off[u]);
#pragma unroll
      for (int u = 0; u < FR_UNROLL; ++u)
        if (off[u] >= 0) acc8(a[u], v[u]);
    }
    char* mine = reinterpret_cast<char*>(p.peer_grad[p.rank]);
#pragma unroll
    for (int u = 0; u < FR_UNROLL; ++u) {
      if (off[u] < 0) continue;
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat16 x = __float2bfloat16_rn(a[u][2 * i] * p.scale);
        const __nv_bfloat16 y = __float2bfloat16_rn(a[u][2 * i + 1] * p.scale);
        const float fx = __bfloat162float(x), fy = __bfloat162float(y);
        sq += fx * fx + fy * fy;
        w[i] = (uint32_t)__bfloat16_as_ushort(x) | ((uint32_t)__bfloat16_as_ushort(y) << 16);
      }
      *reinterpret_cast<uint4*>(mine + off[u]) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  sq = warp_sum(sq);
  __shared__ float part[FR_THREADS / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < FR_THREADS / 32 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0 && v != 0.f) atomicAdd(p.sumsq, v);
  }
}

// One thread per peer: flags[row][rank] <- epoch on every rank (this rank's own word included).
__global__ void fsdp_raise_kernel(const long long* peer_base, long long flag_off, int row, int rank, int world,
                                  unsigned epoch) {
  const int q = threadIdx.x;
  if (q >= world) return;
  __threadfence_system();
  unsigned* f = reinterpret_cast<unsigned*>(peer_base[q] + flag_off) + row * world + rank;
  st_release_u32_sys(f, epoch);
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

int num_sms(int device);

void fsdp_reduce(const long long* peer_grad, const long long* seg_off, const long long* seg_vec, int n_seg,
                 long long total_vec, int rank, int world, float scale, float* sumsq, cudaStream_t s) {
  if (world < 1 || world > FR_MAX_WORLD) throw std::runtime_error("fsdp_reduce: world must be in [1, 16]");
  if (n_seg == 0 || total_vec == 0) return;
  int dev = 0;
  cudaGetDevice(&dev);
  const long long per = (long long)FR_THREADS * FR_UNROLL;
  const int blocks = (int)std::max<long long>(1, std::min<long long>((total_vec + per - 1) / per, 4LL * num_sms(dev)));
  FsdpReduceParams p{peer_grad, seg_off, seg_vec, n_seg, rank, world, scale, sumsq};
  (astrai::note_launch(), fsdp_reduce_kernel<<<blocks, FR_THREADS, 0, s>>>(p));
}

void fsdp_raise(const long long* peer_base, long long flag_off, int row, int rank, int world, unsigned epoch,
                cudaStream_t s) {
  if (world < 1 || world > 1024) throw std::runtime_error("fsdp_raise: bad world size");
  (astrai::note_launch(), fsdp_raise_kernel<<<1, 32 * ((world + 31) / 32), 0, s>>>(peer_base, flag_off, row, rank,
                                                                                     world, epoch));
}

}  // namespace astrai_host
