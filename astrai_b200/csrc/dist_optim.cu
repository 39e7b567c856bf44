// Sharded Muon: the weight update of the matrices this rank owns, written into
// every rank's replica of the parameter over NVLink peer memory (sm_100a).
//
// Data-parallel Muon is redundant: after the gradient all-reduce every rank
// holds the same gradients and would run the same Newton-Schulz iterations on
// every hidden matrix. Here matrix i of a shape group is owned by rank
// i % world; the owner runs momentum + Newton-Schulz on its matrices only and
// this kernel applies
//     p = p * (1 - lr * wd) - adj_lr * O        (O: the orthogonalised update)
// and stores the new bf16 values into its own parameter and into the same
// parameter on every peer. The parameters live at the same offset of a
// symmetric buffer on every rank, so peer q's copy is peer_base[q] + offset.
// Stores are 16-byte vectors (8 bf16) per thread, the update tile staged
// through shared memory so the transposed case (tall matrices orthogonalised
// as their transpose) reads the update coalesced.
//
// Completion: every CTA fences its stores at system scope and counts itself
// done; the last CTA raises this launch's flag (one flag row per shape group)
// on every peer with a release store. peer_flags_wait then waits, bounded,
// until every peer has raised every row of the current epoch: after it the
// whole model is updated on this rank.
#include <stdexcept>
#include <string>

#include "common.cuh"

namespace astrai {

struct PeerApplyParams {
  const long long* pptr;       // [batch] local parameter addresses (bf16 [R][C], inside the symmetric buffer)
  const long long* poff;       // [batch] byte offsets of the same parameters inside the symmetric buffer
  const long long* peer_base;  // [world] symmetric buffer base of every rank, mapped here
  const __nv_bfloat16* X;      // [batch][R][C], or [batch][C][R] when transpose
  int batch, R, C, transpose;
  float decay, adj_lr;
  int rank, world;
  long long flag_off;  // byte offset of the flag block [rows][world] (u32) in the symmetric buffer
  int slot;            // flag row raised by this launch (< 0: none, a later launch of the group raises it)
  unsigned epoch;
  unsigned* done;      // local grid-completion counter, zero between launches
};

constexpr int PA_TILE = 64;
constexpr int PA_THREADS = 256;

__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys_flag(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(PA_THREADS) muon_apply_peers_kernel(PeerApplyParams p) {
  __shared__ float tile[PA_TILE][PA_TILE + 1];
  const int b = blockIdx.z;
  if (b < p.batch) {
    const int c0 = blockIdx.x * PA_TILE, r0 = blockIdx.y * PA_TILE;
    const __nv_bfloat16* x = p.X + (long long)b * p.R * p.C;
    for (int i = threadIdx.x; i < PA_TILE * PA_TILE; i += PA_THREADS) {
      const int a = i / PA_TILE, e = i % PA_TILE;  // e runs along the contiguous dimension of X
      if (!p.transpose) {
        const int r = r0 + a, c = c0 + e;
        tile[a][e] = (r < p.R && c < p.C) ? __bfloat162float(x[(long long)r * p.C + c]) : 0.f;
      } else {
        const int c = c0 + a, r = r0 + e;
        tile[e][a] = (r < p.R && c < p.C) ? __bfloat162float(x[(long long)c * p.R + r]) : 0.f;
      }
    }
    __syncthreads();
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.pptr[b]);
    const bool vec = (p.C % 8) == 0;
    for (int v = threadIdx.x; v < PA_TILE * (PA_TILE / 8); v += PA_THREADS) {
      const int a = v / (PA_TILE / 8), g = v % (PA_TILE / 8);
      const int r = r0 + a, c = c0 + g * 8;
      if (r >= p.R || c >= p.C) continue;
      const long long o = (long long)r * p.C + c;
      if (vec) {
        const uint4 old = *reinterpret_cast<const uint4*>(dst + o);
        const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
        uint32_t nw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16(ow[j]);
          nw[j] = pack_bf16(f.x * p.decay - p.adj_lr * tile[a][g * 8 + 2 * j],
                            f.y * p.decay - p.adj_lr * tile[a][g * 8 + 2 * j + 1]);
        }
        const uint4 nv = make_uint4(nw[0], nw[1], nw[2], nw[3]);
        *reinterpret_cast<uint4*>(dst + o) = nv;
        for (int q = 0; q < p.world; ++q) {
          if (q == p.rank) continue;
          __nv_bfloat16* pd = reinterpret_cast<__nv_bfloat16*>(p.peer_base[q] + p.poff[b]) + o;
          *reinterpret_cast<uint4*>(pd) = nv;
        }
      } else {
        for (int j = 0; j < 8 && c + j < p.C; ++j) {
          const __nv_bfloat16 nv =
              __float2bfloat16_rn(__bfloat162float(dst[o + j]) * p.decay - p.adj_lr * tile[a][g * 8 + j]);
          dst[o + j] = nv;
          for (int q = 0; q < p.world; ++q)
            if (q != p.rank) reinterpret_cast<__nv_bfloat16*>(p.peer_base[q] + p.poff[b])[o + j] = nv;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(p.done, 1u) == total - 1) {
      __threadfence_system();
      for (int q = 0; q < p.world && p.slot >= 0; ++q) {
        if (q == p.rank) continue;
        unsigned* f = reinterpret_cast<unsigned*>(p.peer_base[q] + p.flag_off) + p.slot * p.world + p.rank;
        st_release_sys_u32(f, p.epoch);
      }
      *p.done = 0u;
    }
  }
}

// One thread per (flag row, peer): wait, bounded, until the peer raised the row for `epoch`.
__global__ void peer_flags_wait_kernel(const unsigned* flags, int rank, int world, int rows, unsigned epoch,
                                       unsigned long long wait_ns, int* err) {
  for (int t = threadIdx.x; t < rows * world; t += blockDim.x) {
    if (t % world == rank) continue;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys_flag(flags + t) < epoch) {
      if (globaltimer() - t0 > wait_ns) {
        set_error(err, kErrWaitPeer);
        break;
      }
      __nanosleep(256);
    }
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

void muon_apply_peers(const long long* pptr, const long long* poff, const long long* peer_base, const void* X,
                      int batch, int R, int C, int transpose, float decay, float adj_lr, int rank, int world,
                      long long flag_off, int slot, unsigned epoch, unsigned* done, cudaStream_t s) {
  PeerApplyParams p;
  p.pptr = pptr;
  p.poff = poff;
  p.peer_base = peer_base;
  p.X = static_cast<const __nv_bfloat16*>(X);
  p.batch = batch;
  p.R = R;
  p.C = C;
  p.transpose = transpose;
  p.decay = decay;
  p.adj_lr = adj_lr;
  p.rank = rank;
  p.world = world;
  p.flag_off = flag_off;
  p.slot = slot;
  p.epoch = epoch;
  p.done = done;
  const dim3 grid(batch > 0 ? (C + PA_TILE - 1) / PA_TILE : 1, batch > 0 ? (R + PA_TILE - 1) / PA_TILE : 1,
                  batch > 0 ? batch : 1);
  if (grid.y > 65535 || grid.z > 65535) throw std::runtime_error("muon_apply_peers: matrix too large");
  (astrai::note_launch(), muon_apply_peers_kernel<<<grid, PA_THREADS, 0, s>>>(p));
}

void peer_flags_wait(const unsigned* flags, int rank, int world, int rows, unsigned epoch, double wait_s,
                     cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long ns = (unsigned long long)(wait_s * 1e9);
  (astrai::note_launch(), peer_flags_wait_kernel<<<1, 256, 0, s>>>(flags, rank, world, rows, epoch, ns,
                                                                      error_word(dev)));
}

}  // namespace astrai_host
