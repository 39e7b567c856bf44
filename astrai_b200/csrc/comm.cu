// NVLink peer-memory collectives (sm_100a): symmetric buffers over CUDA IPC
// and the fused data-parallel gradient all-reduce.
//
// Symmetric buffer: every rank cudaMallocs the same number of bytes, exports
// a CUDA IPC handle, and maps every peer's buffer (the handles are exchanged
// by the host over the process group). All ranks use the same layout inside
// the buffer, so a kernel addresses any rank's region as peer_base[q] + off.
//
// Fused all-reduce (mean) + global grad-norm^2 + clip coefficient, one kernel:
// the gradients are a list of bf16 tensors seen as one flat array, cut into
// rounds of R elements; each round into W slices (slice s is owned by rank s);
// each slice into chunks handled by the CTAs in a fixed interleave (CTA b
// takes chunks b, b+G, ...). For every round:
//   A  scatter: rank r stores its part of slice s straight into rank s's
//      receive region (P2P stores over NVLink), then raises flagA on rank s;
//   B  reduce:  rank s waits for flagA from every peer, sums its own slice
//      with the W-1 received copies in fp32, scales by 1/W, rounds to bf16,
//      writes the result to its own gradients, pushes it into every peer's
//      gather region, accumulates the squared norm of the rounded values,
//      and raises flagB on every peer (with its running per-CTA sum);
//   C  gather:  rank r waits for flagB from every peer and copies the other
//      slices from its gather region into its gradients.
// CTA b only ever waits for CTA b of the other ranks (the partition is the
// same on every rank), so no grid-wide barrier is needed. Receive and gather
// regions are double-buffered by round parity: a region is rewritten two
// rounds later, after its reader has provably passed the flags of the round
// in between. Flags hold monotonically increasing epochs (no reset).
// The last CTA to finish sums the per-(rank, CTA) squared norms in a fixed
// order, so every rank gets bitwise the same total and clip coefficient.
//
// Every wait is bounded (wait_ns, default 20 s: ranks may arrive skewed by a
// whole backward pass); on expiry the CTA records kErrWaitPeer in the error
// word and skips the rest of its work.
#include <stdexcept>
#include <string>

#include "common.cuh"


namespace astrai {

struct ARParams {
  const long long* seg_ptr;  // [n_seg] bf16 gradient base addresses
  const long long* seg_off;  // [n_seg + 1] prefix offsets in elements
  int n_seg;
  long long N;               // total elements (multiple of 8)
  int rank, world;
  long long R;               // elements per round (multiple of 8 * world)
  const long long* peer_base;  // [world] symmetric buffer base of every rank, mapped here
  long long off_flag_a, off_flag_b, off_sumsq, off_recv, off_gather;
  unsigned epoch0;
  float scale;
  float* sumsq_out;
  float* clip_coef;
  float max_norm;
  unsigned* done;
  int* err;
  unsigned long long wait_ns;
};

constexpr int AR_THREADS = 512;
constexpr int AR_UNROLL = 4;
constexpr long long AR_CHUNK = (long long)AR_THREADS * AR_UNROLL * 8;  // elements per chunk

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Resolve a flat element index to its address (segment cached per thread).
struct SegCursor {
  int seg = 0;
  long long lo = 0, hi = -1;
  __device__ __forceinline__ __nv_bfloat16* at(const ARParams& p, long long i) {
    if (i < lo || i >= hi) {
      int a = 0, b = p.n_seg - 1;
      while (a < b) {
        const int m = (a + b + 1) >> 1;
        if (p.seg_off[m] <= i) a = m; else b = m - 1;
      }
      seg = a;
      lo = p.seg_off[a];
      hi = p.seg_off[a + 1];
    }
    return reinterpret_cast<__nv_bfloat16*>(p.seg_ptr[seg]) + (i - lo);
  }
};

__device__ __forceinline__ char* region(const ARParams& p, int q, long long off) {
  return reinterpret_cast<char*>(p.peer_base[q]) + off;
}

// Bounded wait (thread 0) until flags[q * G + b] >= epoch for every q != rank.
__device__ bool wait_flags(const ARParams& p, long long off, int b, unsigned epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const unsigned* flags = reinterpret_cast<const unsigned*>(region(p, p.rank, off));
    const uint64_t t0 = globaltimer();
    for (int q = 0; q < p.world && ok; ++q) {
      if (q == p.rank) continue;
      while (ld_acquire_sys(flags + q * gridDim.x + b) < epoch) {
        if (globaltimer() - t0 > p.wait_ns) {
          set_error(p.err, kErrWaitPeer);
          ok = 0;
          break;
        }
        __nanosleep(256);
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

// Publish: fence this CTA's prior stores system-wide, then raise flag [rank][b] on every peer.
__device__ void raise_flags(const ARParams& p, long long off, int b, unsigned epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.world; ++q) {
      if (q == p.rank) continue;
      unsigned* f = reinterpret_cast<unsigned*>(region(p, q, off)) + p.rank * gridDim.x + b;
      st_release_sys(f, epoch);
    }
  }
}

__device__ __forceinline__ void add8(float* a, uint4 u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = unpack_bf16(w[j]);
    a[2 * j] += f.x;
    a[2 * j + 1] += f.y;
  }
}

template <int W>
__global__ void __launch_bounds__(AR_THREADS) fused_allreduce_kernel(ARParams p) {
  // phase B keeps UB chunks x W vectors in flight per thread (8 loads)
  constexpr int UB = W >= 8 ? 1 : 8 / W;
  const int b = blockIdx.x, G = gridDim.x, r = p.rank;
  const long long S = p.R / W;  // slice elements
  const int n_rounds = (int)((p.N + p.R - 1) / p.R);
  SegCursor cur;
  float cta_sumsq = 0.f;  // running over rounds (thread 0 holds the block total)
  bool alive = true;
  for (int rd = 0; rd < n_rounds && alive; ++rd) {
    const unsigned epoch = p.epoch0 + rd;
    const int par = rd & 1;
    const long long base = (long long)rd * p.R;
    // ---------------- A: scatter slices s != r to their owners
#pragma unroll 1
    for (int s = 0; s < W; ++s) {
      if (s == r) continue;
      const long long s0 = base + s * S;
      const long long s1 = min(s0 + S, p.N);
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(region(p, s, p.off_recv)) + ((long long)par * W + r) * S;
      for (long long c0 = s0 + (long long)b * AR_CHUNK; c0 < s1; c0 += (long long)G * AR_CHUNK) {
        uint4 v[AR_UNROLL];
#pragma unroll
        for (int u = 0; u < AR_UNROLL; ++u) {
          const long long i = c0 + ((long long)u * AR_THREADS + threadIdx.x) * 8;
          if (i < s1) v[u] = *reinterpret_cast<const uint4*>(cur.at(p, i));
        }
#pragma unroll
        for (int u = 0; u < AR_UNROLL; ++u) {
          const long long i = c0 + ((long long)u * AR_THREADS + threadIdx.x) * 8;
          if (i < s1) *reinterpret_cast<uint4*>(dst + (i - s0)) = v[u];
        }
      }
    }
    raise_flags(p, p.off_flag_a, b, epoch);
    // ---------------- B: reduce own slice, push to every peer's gather region
    float local_sq = 0.f;
    if (!wait_flags(p, p.off_flag_a, b, epoch)) { alive = false; break; }
    {
      const long long s0 = base + r * S;
      const long long s1 = min(s0 + S, p.N);
      const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(region(p, r, p.off_recv)) + (long long)par * W * S;
      for (long long c0 = s0 + (long long)b * AR_CHUNK; c0 < s1; c0 += (long long)G * AR_CHUNK) {
#pragma unroll 1
        for (int u0 = 0; u0 < AR_UNROLL; u0 += UB) {
          uint4 in[UB][W];
          __nv_bfloat16* gp[UB];
#pragma unroll
          for (int u = 0; u < UB; ++u) {
            const long long i = c0 + ((long long)(u0 + u) * AR_THREADS + threadIdx.x) * 8;
            gp[u] = nullptr;
            if (i < s1) {
              gp[u] = cur.at(p, i);
#pragma unroll
              for (int q = 0; q < W; ++q)
                in[u][q] = q == r ? *reinterpret_cast<const uint4*>(gp[u])
                                  : *reinterpret_cast<const uint4*>(recv + (long long)q * S + (i - s0));
            }
          }
#pragma unroll
          for (int u = 0; u < UB; ++u) {
            if (gp[u] == nullptr) continue;
            const long long i = c0 + ((long long)(u0 + u) * AR_THREADS + threadIdx.x) * 8;
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = 0; q < W; ++q) add8(acc, in[u][q]);
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              o[j] = pack_bf16(acc[2 * j] * p.scale, acc[2 * j + 1] * p.scale);
              const float2 f = unpack_bf16(o[j]);
              local_sq += f.x * f.x + f.y * f.y;
            }
            const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(gp[u]) = ov;
#pragma unroll
            for (int q = 0; q < W; ++q) {
              if (q == r) continue;
              __nv_bfloat16* gq = reinterpret_cast<__nv_bfloat16*>(region(p, q, p.off_gather)) + ((long long)par * W + r) * S;
              *reinterpret_cast<uint4*>(gq + (i - s0)) = ov;
            }
          }
        }
      }
    }
    // block-reduce the squared norm; thread 0 publishes the running total with flagB
    local_sq = warp_sum(local_sq);
    __shared__ float red[AR_THREADS / 32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = local_sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < AR_THREADS / 32; ++w) t += red[w];
      cta_sumsq += t;
      for (int q = 0; q < W; ++q)
        reinterpret_cast<float*>(region(p, q, p.off_sumsq))[r * G + b] = cta_sumsq;
    }
    raise_flags(p, p.off_flag_b, b, epoch);
    // ---------------- C: collect the other slices
    if (!wait_flags(p, p.off_flag_b, b, epoch)) { alive = false; break; }
    for (int s = 0; s < W; ++s) {
      if (s == r) continue;
      const long long s0 = base + s * S;
      const long long s1 = min(s0 + S, p.N);
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(region(p, r, p.off_gather)) + ((long long)par * W + s) * S;
      for (long long c0 = s0 + (long long)b * AR_CHUNK; c0 < s1; c0 += (long long)G * AR_CHUNK) {
        uint4 v[AR_UNROLL];
#pragma unroll
        for (int u = 0; u < AR_UNROLL; ++u) {
          const long long i = c0 + ((long long)u * AR_THREADS + threadIdx.x) * 8;
          if (i < s1) v[u] = *reinterpret_cast<const uint4*>(src + (i - s0));
        }
#pragma unroll
        for (int u = 0; u < AR_UNROLL; ++u) {
          const long long i = c0 + ((long long)u * AR_THREADS + threadIdx.x) * 8;
          if (i < s1) *reinterpret_cast<uint4*>(cur.at(p, i)) = v[u];
        }
      }
    }
    __syncthreads();  // all reads of this round's gather region precede the next round's flags
  }
  // ---------------- finalise: the last CTA sums the (rank, CTA) norms in a fixed order
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.done, 1u);
    if (prev == (unsigned)G - 1) {
      __threadfence();
      const float* slots = reinterpret_cast<const float*>(region(p, r, p.off_sumsq));
      float total = 0.f;
      for (int q = 0; q < W; ++q) {
        float t = 0.f;
        for (int c = 0; c < G; ++c) t += *(volatile const float*)(slots + q * G + c);
        total += t;
      }
      if (p.sumsq_out) *p.sumsq_out = total;
      if (p.clip_coef) {
        const float norm = sqrtf(total);
        *p.clip_coef = p.max_norm > 0.f ? fminf(1.f, p.max_norm / (norm + 1e-6f)) : 1.f;
      }
      *p.done = 0u;
    }
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

// ------------------------------------------------------------------ symmetric buffers (CUDA IPC)
void* symm_alloc(long long bytes, void* handle_out /* 64 bytes */) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) throw std::runtime_error(std::string("symm_alloc: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    throw std::runtime_error(std::string("symm_alloc: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  return p;
}

void* symm_open(const void* handle) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) throw std::runtime_error(std::string("symm_open: ") + cudaGetErrorString(e));
  return p;
}

void symm_close(void* p) { cudaIpcCloseMemHandle(p); }
void symm_free(void* p) { cudaFree(p); }

void fused_allreduce(const long long* seg_ptr, const long long* seg_off, int n_seg, long long N, int rank, int world,
                     long long R, const long long* peer_base, long long off_flag_a, long long off_flag_b,
                     long long off_sumsq, long long off_recv, long long off_gather, unsigned epoch0, int ctas,
                     float* sumsq_out, float* clip_coef, float max_norm, unsigned* done, int* err,
                     unsigned long long wait_ns, cudaStream_t s) {
  ARParams p;
  p.seg_ptr = seg_ptr;
  p.seg_off = seg_off;
  p.n_seg = n_seg;
  p.N = N;
  p.rank = rank;
  p.world = world;
  p.R = R;
  p.peer_base = peer_base;
  p.off_flag_a = off_flag_a;
  p.off_flag_b = off_flag_b;
  p.off_sumsq = off_sumsq;
  p.off_recv = off_recv;
  p.off_gather = off_gather;
  p.epoch0 = epoch0;
  p.scale = 1.f / static_cast<float>(world);
  p.sumsq_out = sumsq_out;
  p.clip_coef = clip_coef;
  p.max_norm = max_norm;
  p.done = done;
  p.err = err;
  p.wait_ns = wait_ns;
  switch (world) {
    case 2: (astrai::note_launch(), fused_allreduce_kernel<2><<<ctas, AR_THREADS, 0, s>>>(p)); break;
    case 4: (astrai::note_launch(), fused_allreduce_kernel<4><<<ctas, AR_THREADS, 0, s>>>(p)); break;
    case 8: (astrai::note_launch(), fused_allreduce_kernel<8><<<ctas, AR_THREADS, 0, s>>>(p)); break;
    default: throw std::runtime_error("fused_allreduce: world size must be 2, 4 or 8");
  }
}

}  // namespace astrai_host
