// Inference kernels (sm_100a): paged KV-cache write / gather, paged split-KV
// decode attention, split combine, and the fused token sampler.
//
// Paged KV layout (per layer):  cache[page][kv_head][slot][D]  (bf16, D = 64 or 128)
// so the keys of one head inside a page are contiguous and a decode warp
// streams them with fully coalesced 256-byte rows.
//
// Decode (replaces gather + repeat_kv + SDPA over the gathered cache of the
// reference, astrai/inference/core/cache.py:256-276 + attention.py:89-101):
// grid (split, kv_head, batch); a CTA reads each K/V row of its key range
// ONCE and applies it to all Hq/Hkv query heads of the group; lanes split
// the head dimension, warps split the keys, online softmax in fp32. Split
// partials (m, l, acc) are merged by a second kernel (flash-decoding).
// Decode is bound by HBM bandwidth (one pass over the live KV), so CUDA-core
// math is enough; the kernel reads the page table itself - nothing is
// gathered.
//
// Sampling (replaces astrai/inference/sample.py:18-375): one CTA per row
// applies temperature, top-k (k-th largest logit found by a binary search on
// the float bit pattern), top-p (nucleus threshold by a binary search on
// probability: keep token i iff the mass of strictly more likely tokens is
// <= top_p), the frequency penalty (count of each token in the row's history
// window) and draws from the final distribution with a block-wide prefix
// scan; it also returns log p(token) under that distribution. Greedy rows
// (temperature 0) take the argmax of the raw logits. No host
// synchronisation, no sort.
#include <cfloat>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace astrai {

constexpr int DEC_MAXG = 16;

// ------------------------------------------------------------------ KV write / gather
// src k/v: [T, Hkv, D] rows with row stride ld (elements); slot[t] = page * page_size + offset
__global__ void paged_kv_write_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                      long long ld_src, const int* __restrict__ slot, int T, int Hkv, int page_size,
                                      int n_pages, __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                      int D) {
  const int per = D / 8;  // 16-byte chunks per head row
  const long long total = (long long)T * Hkv * per;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = i % per;
    const long long th = i / per;
    const int h = th % Hkv;
    const int t = th / Hkv;
    const int s = slot[t];
    if (s < 0 || s >= n_pages * page_size) continue;  // -1 = skip; never write outside the cache
    const int page = s / page_size, off = s % page_size;
    const long long dst = (((long long)page * Hkv + h) * page_size + off) * D + c * 8;
    const long long src = (long long)t * ld_src + h * D + c * 8;
    *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + src);
    *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + src);
  }
}

// out k/v: [B, S_out, Hkv, D] contiguous; positions >= len[b] are zero-filled
__global__ void paged_kv_gather_kernel(const __nv_bfloat16* __restrict__ kc, const __nv_bfloat16* __restrict__ vc,
                                       const int* __restrict__ table, int max_pages, const int* __restrict__ lens,
                                       int B, int S_out, int Hkv, int page_size, int n_pages, __nv_bfloat16* __restrict__ ko,
                                       __nv_bfloat16* __restrict__ vo, int D) {
  const int per = D / 8;
  const long long total = (long long)B * S_out * Hkv * per;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = i % per;
    long long r = i / per;
    const int h = r % Hkv;
    r /= Hkv;
    const int pos = r % S_out;
    const int b = r / S_out;
    uint4 kk = make_uint4(0, 0, 0, 0), vv = kk;
    if (pos < lens[b] && pos / page_size < max_pages) {
      const int page = table[(long long)b * max_pages + pos / page_size];
      if (page >= 0 && page < n_pages) {
        const long long src = (((long long)page * Hkv + h) * page_size + pos % page_size) * D + c * 8;
        kk = *reinterpret_cast<const uint4*>(kc + src);
        vv = *reinterpret_cast<const uint4*>(vc + src);
      }
    }
    const long long dst = (((long long)b * S_out + pos) * Hkv + h) * D + c * 8;
    *reinterpret_cast<uint4*>(ko + dst) = kk;
    *reinterpret_cast<uint4*>(vo + dst) = vv;
  }
}

// ------------------------------------------------------------------ decode attention
struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, D] (row stride ldq per batch row, head stride D)
  long long ldq;
  const __nv_bfloat16* kc;
  const __nv_bfloat16* vc;
  const int* table;  // [B, max_pages]
  int max_pages;
  int n_pages;       // pages in the cache: table entries outside [0, n_pages) are skipped
  const int* lens;   // [B] number of cached keys (including the current token)
  int B, Hq, Hkv, page_size, splits;
  float scale_log2;
  float* part_acc;   // [B, Hkv, splits, G, D]
  float* part_ml;    // [B, Hkv, splits, G, 2]
  __nv_bfloat16* out;  // [B, Hq, D] (row stride ldo)
  long long ldo;
};

__device__ __forceinline__ float ex2f_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// head-dim elements of a K/V row held by one lane: D / 32 (4 for D = 128, 2 for D = 64), loaded as one
// 8- or 4-byte vector
template <int DPL>
struct LaneVec;
template <>
struct LaneVec<4> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&f)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
    f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
  }
};
template <>
struct LaneVec<2> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&f)[2]) {
    const float2 a = unpack_bf16(*reinterpret_cast<const uint32_t*>(p));
    f[0] = a.x, f[1] = a.y;
  }
};

template <int G, int D>
__global__ void __launch_bounds__(128) paged_decode_kernel(DecodeParams p) {
  constexpr int DPL = D / 32;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = p.lens[b];
  // this row's keys are divided evenly over the splits (multiples of 16 keys)
  const int kps = ((len + p.splits - 1) / p.splits + 15) & ~15;
  const int k0 = split * kps;
  const int k1 = min(len, k0 + kps);
  // q for the G heads of this group: lane owns dims [DPL*lane, DPL*lane + DPL)
  float q[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    LaneVec<DPL>::load(p.q + (long long)b * p.ldq + (hk * G + g) * D + lane * DPL, q[g]);
#pragma unroll
    for (int i = 0; i < DPL; ++i) q[g][i] *= p.scale_log2;
  }
  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
  }
  const int* trow = p.table + (long long)b * p.max_pages;
  // each warp takes 4 consecutive keys per iteration: 8 independent 8-byte
  // loads per lane in flight before any math
  constexpr int KU = 4;
  for (int kb = k0 + warp * KU; kb < k1; kb += 4 * KU) {
    float kf[KU][DPL], vf[KU][DPL];
    bool ok[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int k = kb + u;
      const int pidx = k / p.page_size;
      const int page = (k < k1 && pidx < p.max_pages) ? trow[pidx] : -1;
      ok[u] = page >= 0 && page < p.n_pages;
      if (ok[u]) {
        const long long row = (((long long)page * p.Hkv + hk) * p.page_size + k % p.page_size) * D + lane * DPL;
        LaneVec<DPL>::load(p.kc + row, kf[u]);
        LaneVec<DPL>::load(p.vc + row, vf[u]);
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) kf[u][i] = vf[u][i] = 0.f;
      }
    }
    float s[KU][G];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) d = fmaf(q[g][i], kf[u][i], d);
        s[u][g] = d;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int u = 0; u < KU; ++u)
#pragma unroll
        for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffff, s[u][g], o);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < KU; ++u)
        if (ok[u]) mx = fmaxf(mx, s[u][g]);
      if (mx == -INFINITY) continue;
      const float corr = ex2f_fast(m[g] - mx);
      m[g] = mx;
      l[g] *= corr;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[g][i] *= corr;
#pragma unroll
      for (int u = 0; u < KU; ++u) {
        if (!ok[u]) continue;
        const float e = ex2f_fast(s[u][g] - mx);
        l[g] += e;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(e, vf[u][i], acc[g][i]);
      }
    }
  }
  // merge the 4 warps through shared memory
  __shared__ float sm_ml[4][G][2];
  __shared__ float sm_acc[4][G][D];
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_ml[warp][g][0] = m[g];
      sm_ml[warp][g][1] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i) sm_acc[warp][g][lane * DPL + i] = acc[g][i];
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += 128) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[w][g][0]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float c = ex2f_fast(sm_ml[w][g][0] - M);
        L += sm_ml[w][g][1] * c;
        A += sm_acc[w][g][d] * c;
      }
    }
    if (p.splits == 1) {
      p.out[(long long)b * p.ldo + (hk * G + g) * D + d] = __float2bfloat16_rn(L > 0.f ? A / L : 0.f);
    } else {
      const long long base = (((long long)b * p.Hkv + hk) * p.splits + split) * G + g;
      p.part_acc[base * D + d] = A;
      if (d == 0) {
        p.part_ml[base * 2] = M;
        p.part_ml[base * 2 + 1] = L;
      }
    }
  }
}

// merge split partials: one block per (b, q head), D threads
__global__ void decode_combine_kernel(const float* __restrict__ part_acc, const float* __restrict__ part_ml, int B,
                                      int Hq, int Hkv, int splits, __nv_bfloat16* __restrict__ out, long long ldo,
                                      int D) {
  // a kernel launched after this one with programmatic dependent launch may start now (it waits for
  // this grid to finish before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int bh = blockIdx.x;
  const int b = bh / Hq, h = bh % Hq;
  const int G = Hq / Hkv, hk = h / G, g = h % G;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s)
    M = fmaxf(M, part_ml[((((long long)b * Hkv + hk) * splits + s) * G + g) * 2]);
  float L = 0.f, A = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const long long base = (((long long)b * Hkv + hk) * splits + s) * G + g;
      const float c = ex2f_fast(part_ml[base * 2] - M);
      L += part_ml[base * 2 + 1] * c;
      A += part_acc[base * D + d] * c;
    }
  }
  out[(long long)b * ldo + h * D + d] = __float2bfloat16_rn(L > 0.f ? A / L : 0.f);
}

// ------------------------------------------------------------------ sampling
// One thread-block cluster per row: CTA r of the cluster holds vocabulary
// chunk [r * 16384, (r + 1) * 16384) in registers (1024 threads x 16 values),
// so a row is read from HBM exactly once. Row-wide sums / maxima are block
// reductions merged across the cluster through distributed shared memory.
constexpr int SMP_THREADS = 1024;
constexpr int SMP_PER = 16;
constexpr int SMP_CHUNK = SMP_THREADS * SMP_PER;  // 16384 tokens per CTA
constexpr int SMP_MAX_CLUSTER = 16;               // non-portable cluster size -> V <= 262144

// SplitMix64 finaliser (public-domain construction): uniform in [0, 1)
__device__ __forceinline__ float uniform_from(unsigned long long seed, unsigned long long a, unsigned long long b) {
  unsigned long long z = seed + 0x9E3779B97F4A7C15ull * (a * 0x100000001B3ull + b + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

// order-preserving map of floats to uint32 (greater float -> greater key)
__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

enum RedOp { RED_SUM = 0, RED_MAX = 1 };

__device__ __forceinline__ float red2(float a, float b, int op) { return op == RED_MAX ? fmaxf(a, b) : a + b; }

// Row-wide reduction: block reduction, then (cluster > 1) a merge of the
// per-CTA results read from every CTA's shared memory.
__device__ __forceinline__ float row_reduce(float v, int op, float* sh, int csize) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = red2(v, __shfl_xor_sync(0xffffffff, v, o), op);
  if (lane == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = sh[lane];  // SMP_THREADS / 32 == 32 partials
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = red2(v, __shfl_xor_sync(0xffffffff, v, o), op);
    if (lane == 0) sh[32] = v;
  }
  if (csize == 1) {
    __syncthreads();
    v = sh[32];
    __syncthreads();  // sh reusable by the next reduction
    return v;
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  float r = op == RED_MAX ? -INFINITY : 0.f;
  for (int c = 0; c < csize; ++c) r = red2(r, *cl.map_shared_rank(sh + 32, c), op);
  cl.sync();
  return r;
}

// Exclusive prefix of a per-CTA value over cluster ranks (rank order)
__device__ __forceinline__ float cluster_exclusive(float v, float* slot, int csize, int rank) {
  if (csize == 1) return 0.f;
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) *slot = v;
  cl.sync();
  float r = 0.f;
  for (int c = 0; c < rank; ++c) r += *cl.map_shared_rank(slot, c);
  cl.sync();
  return r;
}

constexpr int SMP_CAND = 1024;  // survivors of top-k handled in shared memory

// Sum / min over this CTA only (all CTAs of a row hold the same candidate list).
__device__ __forceinline__ float block_sum_local(float v, float* scratch) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[w] = v;
  __syncthreads();
  if (w == 0) {
    v = warp_sum(scratch[lane]);
    if (lane == 0) scratch[32] = v;
  }
  __syncthreads();
  return scratch[32];
}

__device__ __forceinline__ float block_min_local(float v, float* scratch) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffff, v, o));
  __syncthreads();
  if (lane == 0) scratch[w] = v;
  __syncthreads();
  if (w == 0) {
    v = scratch[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffff, v, o));
    if (lane == 0) scratch[32] = v;
  }
  __syncthreads();
  return scratch[32];
}

// Row-wide sums of NV values at once (block, then cluster through DSMEM):
// one synchronisation round for all of them.
template <int NV>
__device__ __forceinline__ void row_reduce_vec(float (&v)[NV], float* scratch /* [32 * NV + NV] */, int csize) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffff, v[i], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) scratch[w * NV + i] = v[i];
  }
  __syncthreads();
  float* tot = scratch + 32 * NV;
  if (threadIdx.x < NV) {
    float acc = 0.f;
    for (int ww = 0; ww < SMP_THREADS / 32; ++ww) acc += scratch[ww * NV + threadIdx.x];
    tot[threadIdx.x] = acc;
  }
  if (csize == 1) {
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = tot[i];
    __syncthreads();
    return;
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float acc = 0.f;
    for (int c = 0; c < csize; ++c) acc += *cl.map_shared_rank(tot + i, c);
    v[i] = acc;
  }
  cl.sync();
}

__global__ void __launch_bounds__(SMP_THREADS, 1) sample_kernel(
    const void* __restrict__ logits, int logits_f32, long long ld, int V, const float* __restrict__ temperature,
    const int* __restrict__ top_k, const float* __restrict__ top_p, const float* __restrict__ penalty,
    const long long* __restrict__ hist, int hist_len, long long ld_hist,
    const unsigned long long* __restrict__ rng, long long* __restrict__ out_tok, float* __restrict__ out_lp) {
  __shared__ float sh[33];
  __shared__ float sh_scan[SMP_THREADS / 32];
  __shared__ float sh_slot;
  const int cs = (int)cg::this_cluster().num_blocks();
  const int rank = cs > 1 ? (int)cg::this_cluster().block_rank() : 0;
  const int row = blockIdx.x / cs;
  const int t = threadIdx.x;
  const int base = rank * SMP_CHUNK;
  float x[SMP_PER];
  float raw_max = -INFINITY;
#pragma unroll
  for (int j = 0; j < SMP_PER; ++j) {
    const int i = base + t + j * SMP_THREADS;
    float v = -INFINITY;
    if (i < V) {
      v = logits_f32 ? reinterpret_cast<const float*>(logits)[(long long)row * ld + i]
                     : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[(long long)row * ld + i]);
      if (v != v) v = -INFINITY;  // NaN never wins
    }
    x[j] = v;
    raw_max = fmaxf(raw_max, v);
  }
  const float temp = temperature ? temperature[row] : 1.f;
  const float gmax = row_reduce(raw_max, RED_MAX, sh, cs);
  if (temp == 0.f) {
    // greedy: first index of the maximum; logprob under softmax(raw logits)
    float sum = 0.f;
    int best = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j) {
      sum += (x[j] == -INFINITY) ? 0.f : __expf(x[j] - gmax);
      if (x[j] == gmax && best == 0x7fffffff && base + t + j * SMP_THREADS < V) best = base + t + j * SMP_THREADS;
    }
    const float Z = row_reduce(sum, RED_SUM, sh, cs);
    const float bi = row_reduce(best == 0x7fffffff ? -3.0e38f : -(float)best, RED_MAX, sh, cs);
    if (t == 0 && rank == 0) {
      out_tok[row] = bi < -1.0e38f ? 0 : (long long)(-bi);
      if (out_lp) out_lp[row] = gmax == -INFINITY ? -INFINITY : -__logf(Z);
    }
    return;
  }
  const float inv_t = 1.f / fmaxf(temp, 1e-8f);
#pragma unroll
  for (int j = 0; j < SMP_PER; ++j) x[j] *= inv_t;
  const float mx = gmax * inv_t;  // scaling by a positive factor keeps the argmax
  // ---- top-k: the largest key L with count(key >= L) >= k; keep key >= L.
  // 8-ary search over the 32-bit key space: 7 thresholds per round, one
  // fused row reduction each, about 11 rounds.
  constexpr int NT = 7;
  __shared__ float red_scratch[33 * NT];
  const int k = top_k ? top_k[row] : 0;
  if (k > 0 && k < V) {
    unsigned long long lo = 0, hi = fkey(mx);  // invariant: count(>= lo) >= k, answer <= hi
    while (lo < hi) {
      uint32_t th[NT];
      float c[NT];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        th[i] = (uint32_t)(lo + ((hi - lo) * (unsigned long long)(i + 1) + NT) / (NT + 1));
        c[i] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < SMP_PER; ++j) {
        if (x[j] == -INFINITY) continue;
        const uint32_t key = fkey(x[j]);
#pragma unroll
        for (int i = 0; i < NT; ++i) c[i] += key >= th[i] ? 1.f : 0.f;
      }
      row_reduce_vec<NT>(c, red_scratch, cs);
      int best = -1;
#pragma unroll
      for (int i = 0; i < NT; ++i)
        if (c[i] >= (float)k) best = i;  // counts fall as thresholds rise
      if (best >= 0 && c[best] == (float)k) {  // exactly the k largest
        lo = hi = th[best];
        break;
      }
      const unsigned long long nlo = best >= 0 ? (unsigned long long)th[best] : lo;
      const unsigned long long nhi = best + 1 < NT ? (unsigned long long)th[best + 1] - 1 : hi;
      if (nlo == lo && nhi == hi) break;  // range too small to split further: lo is exact
      lo = nlo;
      hi = nhi < nlo ? nlo : nhi;
    }
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j)
      if (x[j] != -INFINITY && fkey(x[j]) < (uint32_t)lo) x[j] = -INFINITY;
  }
  // ---- top-p: keep token i iff the mass of strictly larger tokens <= top_p.
  const float pp = top_p ? top_p[row] : 1.f;
  bool topp_done = false;
  if (pp < 1.f && k > 0 && k <= SMP_CAND) {
    // after top-k at most k values (plus ties) survive: gather them (cluster-wide,
    // rank order, so every CTA holds the same list) and decide on the list
    __shared__ float cand_local[SMP_CAND], cand[SMP_CAND];
    __shared__ int sh_cnt[SMP_THREADS / 32 + 1];
    __shared__ int sh_n;
    __shared__ float sh_thr;
    int mine = 0;
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j) mine += x[j] != -INFINITY;
    const int lane = t & 31, w = t >> 5;
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffff, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) sh_cnt[w] = incl;
    __syncthreads();
    if (w == 0) {
      int v = sh_cnt[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffff, v, o);
        if (lane >= o) v += y;
      }
      sh_cnt[lane] = v;  // inclusive warp totals
    }
    __syncthreads();
    const int cta_n = sh_cnt[SMP_THREADS / 32 - 1];
    int off = incl - mine + (w > 0 ? sh_cnt[w - 1] : 0);
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j)
      if (x[j] != -INFINITY && off < SMP_CAND) cand_local[off++] = x[j];
    if (t == 0) sh_n = cta_n;
    int n = 0;
    if (cs > 1) {
      cg::cluster_group cl = cg::this_cluster();
      cl.sync();
      for (int c = 0; c < cs; ++c) {
        const int nc = *cl.map_shared_rank(&sh_n, c);
        const float* src = cl.map_shared_rank(cand_local, c);
        for (int i = t; i < nc && n + i < SMP_CAND; i += SMP_THREADS) cand[n + i] = src[i];
        n += nc;
      }
      cl.sync();
    } else {
      __syncthreads();
      n = cta_n;
      for (int i = t; i < n && i < SMP_CAND; i += SMP_THREADS) cand[i] = cand_local[i];
    }
    if (n <= SMP_CAND) {  // (more survivors than fit only with massive ties: use the search below)
      __syncthreads();
      float e1[1] = {0.f};
      if (t < n) e1[0] = __expf(cand[t] - mx);
      const float ct = t < n ? cand[t] : 0.f;
      float zsum = e1[0];
      zsum = block_sum_local(zsum, red_scratch);
      float greater = 0.f;
      if (t < n)
        for (int j = 0; j < n; ++j)
          if (cand[j] > ct) greater += __expf(cand[j] - mx);
      const bool keep = t < n && greater <= pp * zsum;
      float kept_min = keep ? ct : INFINITY;
      kept_min = block_min_local(kept_min, red_scratch);
      if (t == 0) sh_thr = kept_min;
      __syncthreads();
      const float thr = sh_thr;
#pragma unroll
      for (int j = 0; j < SMP_PER; ++j)
        if (x[j] < thr) x[j] = -INFINITY;
      topp_done = true;
    }
  }
  if (pp < 1.f && !topp_done) {
    // the smallest key L with mass(key > L) <= top_p * Z (8-ary search as above)
    float s1[1] = {0.f};
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j) s1[0] += (x[j] == -INFINITY) ? 0.f : __expf(x[j] - mx);
    row_reduce_vec<1>(s1, red_scratch, cs);
    const float target = pp * s1[0];
    unsigned long long lo = 0, hi = fkey(mx);  // invariant: mass(> hi) <= target; answer >= lo
    while (lo < hi) {
      uint32_t th[NT];
      float m[NT];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        th[i] = (uint32_t)(lo + ((hi - lo) * (unsigned long long)(i + 1)) / (NT + 1));
        m[i] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < SMP_PER; ++j) {
        if (x[j] == -INFINITY) continue;
        const uint32_t key = fkey(x[j]);
        const float e = __expf(x[j] - mx);
#pragma unroll
        for (int i = 0; i < NT; ++i) m[i] += key > th[i] ? e : 0.f;
      }
      row_reduce_vec<NT>(m, red_scratch, cs);
      int first = NT;
#pragma unroll
      for (int i = NT - 1; i >= 0; --i)
        if (m[i] <= target) first = i;  // masses fall as thresholds rise
      const unsigned long long nhi = first < NT ? (unsigned long long)th[first] : hi;
      const unsigned long long nlo = first > 0 ? (unsigned long long)th[first - 1] + 1 : lo;
      if (nlo == lo && nhi == hi) {  // thresholds collapsed onto the range: finish bisecting
        const unsigned long long mid = lo + (hi - lo) / 2;
        float mm[1] = {0.f};
#pragma unroll
        for (int j = 0; j < SMP_PER; ++j)
          if (x[j] != -INFINITY && (unsigned long long)fkey(x[j]) > mid) mm[0] += __expf(x[j] - mx);
        row_reduce_vec<1>(mm, red_scratch, cs);
        if (mm[0] <= target) hi = mid; else lo = mid + 1;
        continue;
      }
      lo = nlo;
      hi = nhi < nlo ? nlo : nhi;
    }
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j)
      if (x[j] != -INFINITY && fkey(x[j]) < (uint32_t)lo) x[j] = -INFINITY;
  }
  // ---- frequency penalty: subtract penalty * count(token in the history window)
  const float pen = penalty ? penalty[row] : 0.f;
  if (pen != 0.f && hist) {
    for (int h = 0; h < hist_len; ++h) {
      const long long id = hist[(long long)row * ld_hist + h];
      if (id < base || id >= base + SMP_CHUNK || id >= V) continue;
      const int local = (int)(id - base);
      if ((local % SMP_THREADS) != t) continue;
      const int j = local / SMP_THREADS;
#pragma unroll
      for (int jj = 0; jj < SMP_PER; ++jj)
        if (jj == j && x[jj] != -INFINITY) x[jj] -= pen;
    }
  }
  // ---- draw from softmax(x) by inverse CDF over a fixed token order
  float m2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < SMP_PER; ++j) m2 = fmaxf(m2, x[j]);
  m2 = row_reduce(m2, RED_MAX, sh, cs);
  float tsum = 0.f;
#pragma unroll
  for (int j = 0; j < SMP_PER; ++j) tsum += (x[j] == -INFINITY) ? 0.f : __expf(x[j] - m2);
  const int lane = t & 31, w = t >> 5;
  float incl = tsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffff, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sh_scan[w] = incl;
  __syncthreads();
  if (w == 0) {
    float v = sh_scan[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffff, v, o);
      if (lane >= o) v += y;
    }
    sh_scan[lane] = v;  // inclusive warp totals
  }
  __syncthreads();
  const float cta_total = sh_scan[SMP_THREADS / 32 - 1];
  const float cta_before = cluster_exclusive(cta_total, &sh_slot, cs, rank);
  const float Z = row_reduce(t == 0 ? cta_total : 0.f, RED_SUM, sh, cs);
  // the last thread (in token order) holding any mass takes rounding leftovers
  const float last_owner = row_reduce(tsum > 0.f ? (float)(rank * SMP_THREADS + t) : -1.f, RED_MAX, sh, cs);
  const float before = cta_before + (incl - tsum) + (w > 0 ? sh_scan[w - 1] : 0.f);
  const float u = uniform_from(rng[0], rng[1], (unsigned long long)row) * Z;
  const bool is_last = (float)(rank * SMP_THREADS + t) == last_owner;
  if (tsum > 0.f && u >= before && (u < before + tsum || is_last)) {
    float c = before;
    int pick = -1, last_nz = -1;
#pragma unroll
    for (int j = 0; j < SMP_PER; ++j) {
      const float e = (x[j] == -INFINITY) ? 0.f : __expf(x[j] - m2);
      if (e > 0.f) last_nz = j;
      if (pick < 0 && e > 0.f && u < c + e) pick = j;
      c += e;
    }
    if (pick < 0) pick = last_nz;
    float xv = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < SMP_PER; ++jj)
      if (jj == pick) xv = x[jj];
    out_tok[row] = base + t + pick * SMP_THREADS;
    if (out_lp) out_lp[row] = (xv - m2) - __logf(Z);
  } else if (last_owner < 0.f && t == 0 && rank == 0) {
    out_tok[row] = 0;  // every logit was -inf / NaN
    if (out_lp) out_lp[row] = -INFINITY;
  }
}

// ------------------------------------------------------------------ sampling, histogram thresholds
// Vocabularies up to 32768: the row lives in the registers of the CS CTAs of a thread-block cluster
// (32 values per thread): one 1024-thread CTA (CS = 1), or four 256-thread CTAs on four SMs (CS = 4,
// for small batches: a quarter of the per-SM instructions, a cluster barrier per row-wide step). The
// top-k and top-p thresholds come from a 4096-bin histogram of the order-preserving key (its top 12
// bits: sign, exponent and 3 mantissa bits) instead of a threshold search: one pass counts (top-k)
// or sums the probability mass (top-p) per bin, a suffix scan over the cluster's summed bins finds
// the bin holding the threshold, and only that bin's values are gathered (from every CTA, through
// distributed shared memory) and resolved exactly: rank, or mass of strictly larger values. A bin
// of more than SMH_CAND values (massive ties) falls back to bisecting the key inside the bin. Same
// results as sample_kernel: keep key >= the k-th largest key (ties kept), then keep a value iff the
// mass of strictly larger values <= top_p * Z, then the frequency penalty, then an inverse-CDF draw
// in a fixed order.
constexpr int SMH_PER = 32;
constexpr int SMH_MAXV = 32768;
constexpr int SMH_BINS = 4096;
constexpr int SMH_CAND = 2048;

template <int THREADS, int CS>
struct SmhRow {
  static constexpr int NW = THREADS / 32;
  float* red;   // [NW + 1] block scratch
  float* xch;   // [2] this CTA's value exchanged with the cluster
  int rank;

  // row-wide max / sum of v (every thread of every CTA of the row gets it)
  __device__ __forceinline__ float reduce(float v, bool is_max) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, y) : v + y;
    }
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
      float t = lane < NW ? red[lane] : (is_max ? -INFINITY : 0.f);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float y = __shfl_xor_sync(0xffffffffu, t, o);
        t = is_max ? fmaxf(t, y) : t + y;
      }
      if (lane == 0) red[NW] = t;
    }
    __syncthreads();
    float r = red[NW];
    if constexpr (CS > 1) {
      cg::cluster_group cl = cg::this_cluster();
      if (threadIdx.x == 0) xch[0] = r;
      cl.sync();
      r = is_max ? -INFINITY : 0.f;
#pragma unroll
      for (int q = 0; q < CS; ++q) {
        const float y = *cl.map_shared_rank(xch, q);
        r = is_max ? fmaxf(r, y) : r + y;
      }
      cl.sync();
    }
    return r;
  }
  __device__ __forceinline__ float max(float v) { return reduce(v, true); }
  __device__ __forceinline__ float sum(float v) { return reduce(v, false); }
  __device__ __forceinline__ float min(float v) { return -reduce(-v, true); }

  // exclusive prefix of v over (CTA rank, thread) order; the row total in `total`
  __device__ __forceinline__ float exclusive(float v, float& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    float incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) red[w] = incl;
    __syncthreads();
    if (w == 0) {
      float t = lane < NW ? red[lane] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      if (lane < NW) red[lane] = t;  // inclusive warp totals
    }
    __syncthreads();
    const float block_total = red[NW - 1];
    float before = incl - v + (w > 0 ? red[w - 1] : 0.f);
    total = block_total;
    if constexpr (CS > 1) {
      cg::cluster_group cl = cg::this_cluster();
      if (threadIdx.x == 0) xch[1] = block_total;
      cl.sync();
      float lower = 0.f, all = 0.f;
#pragma unroll
      for (int q = 0; q < CS; ++q) {
        const float y = *cl.map_shared_rank(xch + 1, q);
        all += y;
        if (q < rank) lower += y;
      }
      cl.sync();
      before += lower;
      total = all;
    }
    return before;
  }
};

// Bin b* (scanning from the top) where the running total of the cluster's summed bins first exceeds
// `target` (strictly), or reaches it when `reach`; the total of the bins above b* in `above`. -1 when
// the total never gets there. Every CTA computes the same answer from the same sums.
template <int THREADS, int CS>
__device__ __forceinline__ int smh_find_bin(float* bins, float target, bool reach, SmhRow<THREADS, CS>& row,
                                            int* s_bin, float* s_above, float& above) {
  constexpr int BPT = SMH_BINS / THREADS;
  const int t = threadIdx.x;
  float h[BPT];
  if constexpr (CS > 1) {
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();  // every CTA's histogram is complete
#pragma unroll
    for (int i = 0; i < BPT; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q < CS; ++q) acc += *cl.map_shared_rank(bins + BPT * t + i, q);
      h[i] = acc;
    }
    cl.sync();  // peers may reuse their bins from here on
  } else {
#pragma unroll
    for (int i = 0; i < BPT; ++i) h[i] = bins[BPT * t + i];
  }
  float own = 0.f;
#pragma unroll
  for (int i = 0; i < BPT; ++i) own += h[i];
  // bins above this thread's range: the total minus the inclusive prefix up to this thread (block order
  // = bin order; the cluster part of the prefix is not wanted here: every CTA holds all bins)
  const int lane = t & 31, w = t >> 5;
  float incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) row.red[w] = incl;
  __syncthreads();
  if (w == 0) {
    float v = lane < THREADS / 32 ? row.red[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane < THREADS / 32) row.red[lane] = v;
  }
  __syncthreads();
  const float total = row.red[THREADS / 32 - 1];
  const float prefix = incl + (w > 0 ? row.red[w - 1] : 0.f);
  float cum = total - prefix;
  if (t == 0) *s_bin = -1;
  __syncthreads();
#pragma unroll
  for (int i = BPT - 1; i >= 0; --i) {
    const bool hit = reach ? (cum < target && cum + h[i] >= target) : (cum <= target && cum + h[i] > target);
    if (hit && h[i] > 0.f) {
      *s_bin = BPT * t + i;
      *s_above = cum;
    }
    cum += h[i];
  }
  __syncthreads();
  above = *s_above;
  return *s_bin;
}

// Values of x in bin `bin` (bin < 0: every finite value) from every CTA of the row, into `all`
// (same order on every CTA); returns their count, or a count > SMH_CAND when they do not fit.
template <int THREADS, int CS>
__device__ __forceinline__ int smh_gather(const float (&x)[SMH_PER], int bin, float* mine, float* all, int* s_cnt,
                                          int* s_tot) {
  __syncthreads();
  if (threadIdx.x == 0) *s_cnt = 0;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < SMH_PER; ++j)
    if (x[j] != -INFINITY && (bin < 0 || (int)(fkey(x[j]) >> 20) == bin)) {
      const int slot = atomicAdd(s_cnt, 1);
      if (slot < SMH_CAND) mine[slot] = x[j];
    }
  if constexpr (CS == 1) {
    __syncthreads();
    const int n = *s_cnt;
    for (int i = threadIdx.x; i < n && i < SMH_CAND; i += THREADS) all[i] = mine[i];
    __syncthreads();
    return n;
  } else {
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    int n = 0;
#pragma unroll
    for (int q = 0; q < CS; ++q) {
      const int nq = *cl.map_shared_rank(s_cnt, q);
      const float* src = cl.map_shared_rank(mine, q);
      for (int i = threadIdx.x; i < nq && n + i < SMH_CAND; i += THREADS) all[n + i] = src[i];
      n += nq;
    }
    if (threadIdx.x == 0) *s_tot = n;
    cl.sync();
    return n;
  }
}

template <int THREADS, int CS>
__global__ void __launch_bounds__(THREADS, 1) sample_hist_kernel(
    const void* __restrict__ logits, int logits_f32, long long ld, int V, const float* __restrict__ temperature,
    const int* __restrict__ top_k, const float* __restrict__ top_p, const float* __restrict__ penalty,
    const long long* __restrict__ hist, int hist_len, long long ld_hist,
    const unsigned long long* __restrict__ rng, long long* __restrict__ out_tok, float* __restrict__ out_lp) {
  constexpr int CHUNK = THREADS * SMH_PER;
  __shared__ float bins[SMH_BINS];
  __shared__ float cand_mine[SMH_CAND], cand[SMH_CAND];
  __shared__ float red[THREADS / 32 + 1], xch[2];
  __shared__ int s_cnt, s_tot, s_bin;
  __shared__ float s_above;
  const int rank = CS > 1 ? (int)cg::this_cluster().block_rank() : 0;
  const int row = blockIdx.x / CS, t = threadIdx.x;
  SmhRow<THREADS, CS> rw{red, xch, rank};
  const int base = rank * CHUNK;
  float x[SMH_PER];
  float raw_max = -INFINITY;
#pragma unroll
  for (int j = 0; j < SMH_PER; ++j) {
    const int i = base + t + j * THREADS;
    float v = -INFINITY;
    if (i < V) {
      v = logits_f32 ? reinterpret_cast<const float*>(logits)[(long long)row * ld + i]
                     : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[(long long)row * ld + i]);
      if (v != v) v = -INFINITY;  // NaN never wins
    }
    x[j] = v;
    raw_max = fmaxf(raw_max, v);
  }
  const float temp = temperature ? temperature[row] : 1.f;
  const float gmax = rw.max(raw_max);
  if (temp == 0.f) {
    float sum = 0.f, best = 3.0e38f;
#pragma unroll
    for (int j = 0; j < SMH_PER; ++j) {
      sum += (x[j] == -INFINITY) ? 0.f : __expf(x[j] - gmax);
      if (x[j] == gmax) best = fminf(best, (float)(base + t + j * THREADS));
    }
    const float Z = rw.sum(sum);
    const float bi = rw.min(best);
    if (t == 0 && rank == 0) {
      out_tok[row] = bi > 1.0e38f ? 0 : (long long)bi;
      if (out_lp) out_lp[row] = gmax == -INFINITY ? -INFINITY : -__logf(Z);
    }
    return;
  }
  const float inv_t = 1.f / fmaxf(temp, 1e-8f);
#pragma unroll
  for (int j = 0; j < SMH_PER; ++j) x[j] *= inv_t;
  const float mx = gmax * inv_t;
  // ---- top-k
  const int k = top_k ? top_k[row] : 0;
  uint32_t thr = 0;  // keep fkey >= thr
  if (k > 0 && k < V) {
    for (int b = t; b < SMH_BINS; b += THREADS) bins[b] = 0.f;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < SMH_PER; ++j)
      if (x[j] != -INFINITY) atomicAdd(&bins[fkey(x[j]) >> 20], 1.f);
    __syncthreads();
    float above;
    const int bstar = smh_find_bin<THREADS, CS>(bins, (float)k, true, rw, &s_bin, &s_above, above);
    if (bstar >= 0) {
      const int need = k - (int)above;  // values of bin b* to keep (its `need` largest, ties kept)
      const int nb = smh_gather<THREADS, CS>(x, bstar, cand_mine, cand, &s_cnt, &s_tot);
      if (nb <= SMH_CAND) {
        // the smallest value with fewer than `need` strictly larger values in the bin
        float kth = INFINITY;
        for (int i = t; i < nb; i += THREADS) {
          const float c = cand[i];
          int greater = 0;
          for (int j = 0; j < nb; ++j) greater += cand[j] > c;
          if (greater < need) kth = fminf(kth, c);
        }
        thr = fkey(rw.min(kth));
      } else {
        // massive ties: bisect the key inside the bin (count of keys >= mid must stay >= k)
        uint32_t lo = (uint32_t)bstar << 20, hi = lo | 0xFFFFFu;
        while (lo < hi) {
          const uint32_t mid = lo + (hi - lo + 1) / 2;
          float c = 0.f;
#pragma unroll
          for (int j = 0; j < SMH_PER; ++j) c += (x[j] != -INFINITY && fkey(x[j]) >= mid) ? 1.f : 0.f;
          if (rw.sum(c) >= (float)k) lo = mid; else hi = mid - 1;
        }
        thr = lo;
      }
#pragma unroll
      for (int j = 0; j < SMH_PER; ++j)
        if (x[j] != -INFINITY && fkey(x[j]) < thr) x[j] = -INFINITY;
    }
  }
  // ---- top-p: keep a value iff the mass of strictly larger values <= top_p * Z
  const float pp = top_p ? top_p[row] : 1.f;
  bool topp_done = false;
  if (pp < 1.f && thr != 0u) {
    // after top-k only the k largest (plus ties) survive: decide on all of them at once
    const int n = smh_gather<THREADS, CS>(x, -1, cand_mine, cand, &s_cnt, &s_tot);
    if (n <= SMH_CAND) {
      float e = 0.f;
      for (int i = t; i < n; i += THREADS) e += __expf(cand[i] - mx);
      // every CTA holds all n survivors: a block sum is the row sum
      const float target = pp * SmhRow<THREADS, 1>{red, xch, 0}.sum(e);
      float kept_min = INFINITY;
      for (int i = t; i < n; i += THREADS) {
        const float c = cand[i];
        float greater = 0.f;
        for (int j = 0; j < n; ++j)
          if (cand[j] > c) greater += __expf(cand[j] - mx);
        if (greater <= target) kept_min = fminf(kept_min, c);
      }
      kept_min = SmhRow<THREADS, 1>{red, xch, 0}.min(kept_min);
#pragma unroll
      for (int j = 0; j < SMH_PER; ++j)
        if (x[j] < kept_min) x[j] = -INFINITY;
      topp_done = true;
    }
  }
  if (pp < 1.f && !topp_done) {
    __syncthreads();
    for (int b = t; b < SMH_BINS; b += THREADS) bins[b] = 0.f;
    __syncthreads();
    float zs = 0.f;
#pragma unroll
    for (int j = 0; j < SMH_PER; ++j) {
      if (x[j] == -INFINITY) continue;
      const float e = __expf(x[j] - mx);
      zs += e;
      atomicAdd(&bins[fkey(x[j]) >> 20], e);
    }
    const float Z = rw.sum(zs);
    const float target = pp * Z;
    float above;
    const int bstar = smh_find_bin<THREADS, CS>(bins, target, false, rw, &s_bin, &s_above, above);
    if (bstar >= 0) {
      const int nb = smh_gather<THREADS, CS>(x, bstar, cand_mine, cand, &s_cnt, &s_tot);
      float kept_min = INFINITY;
      if (nb <= SMH_CAND) {
        // keep a value of bin b* when the mass above the bin plus the larger values in it fits
        for (int i = t; i < nb; i += THREADS) {
          const float c = cand[i];
          float greater = above;
          for (int j = 0; j < nb; ++j)
            if (cand[j] > c) greater += __expf(cand[j] - mx);
          if (greater <= target) kept_min = fminf(kept_min, c);
        }
        kept_min = SmhRow<THREADS, 1>{red, xch, 0}.min(kept_min);
        const uint32_t cut = kept_min == INFINITY ? ((uint32_t)(bstar + 1) << 20) : fkey(kept_min);
#pragma unroll
        for (int j = 0; j < SMH_PER; ++j)
          if (x[j] != -INFINITY && fkey(x[j]) < cut) x[j] = -INFINITY;
      } else {
        // bisect the key inside the bin: the smallest key whose strictly larger mass fits
        uint32_t lo = (uint32_t)bstar << 20, hi = lo | 0xFFFFFu;
        while (lo < hi) {
          const uint32_t mid = lo + (hi - lo) / 2;
          float m = 0.f;
#pragma unroll
          for (int j = 0; j < SMH_PER; ++j)
            if (x[j] != -INFINITY && fkey(x[j]) > mid) m += __expf(x[j] - mx);
          if (rw.sum(m) <= target) hi = mid; else lo = mid + 1;
        }
#pragma unroll
        for (int j = 0; j < SMH_PER; ++j)
          if (x[j] != -INFINITY && fkey(x[j]) < lo) x[j] = -INFINITY;
      }
    }
  }
  // ---- frequency penalty: subtract penalty * count(token in the history window)
  const float pen = penalty ? penalty[row] : 0.f;
  if (pen != 0.f && hist) {
    for (int h = 0; h < hist_len; ++h) {
      const long long id = hist[(long long)row * ld_hist + h];
      if (id < base || id >= base + CHUNK || id >= V) continue;
      const int local = (int)(id - base);
      if (local % THREADS != t) continue;
      const int jj = local / THREADS;
#pragma unroll
      for (int j = 0; j < SMH_PER; ++j)
        if (j == jj && x[j] != -INFINITY) x[j] -= pen;
    }
  }
  // ---- draw from softmax(x) by inverse CDF in (CTA, thread, slot) order
  float m2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < SMH_PER; ++j) m2 = fmaxf(m2, x[j]);
  m2 = rw.max(m2);
  float tsum = 0.f;
#pragma unroll
  for (int j = 0; j < SMH_PER; ++j) tsum += (x[j] == -INFINITY) ? 0.f : __expf(x[j] - m2);
  float Z;
  const float before = rw.exclusive(tsum, Z);
  const int me = rank * THREADS + t;
  const float last_owner = rw.max(tsum > 0.f ? (float)me : -1.f);
  const float u = uniform_from(rng[0], rng[1], (unsigned long long)row) * Z;
  const bool is_last = (float)me == last_owner;
  if (tsum > 0.f && u >= before && (u < before + tsum || is_last)) {
    float c = before;
    int pick = -1, last_nz = -1;
    float xv = -INFINITY, xlast = -INFINITY;
#pragma unroll
    for (int j = 0; j < SMH_PER; ++j) {
      const float e = (x[j] == -INFINITY) ? 0.f : __expf(x[j] - m2);
      if (e > 0.f) {
        last_nz = j;
        xlast = x[j];
      }
      if (pick < 0 && e > 0.f && u < c + e) {
        pick = j;
        xv = x[j];
      }
      c += e;
    }
    if (pick < 0) {
      pick = last_nz;
      xv = xlast;
    }
    out_tok[row] = base + t + pick * THREADS;
    if (out_lp) out_lp[row] = (xv - m2) - __logf(Z);
  } else if (last_owner < 0.f && t == 0 && rank == 0) {
    out_tok[row] = 0;  // every logit was -inf / NaN
    if (out_lp) out_lp[row] = -INFINITY;
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

void paged_kv_write(const void* k, const void* v, long long ld_src, const int* slot, int T, int Hkv, int page_size,
                    int n_pages, void* kc, void* vc, int D, cudaStream_t s) {
  const long long work = (long long)T * Hkv * (D / 8);
  int blocks = (int)std::min<long long>((work + 255) / 256, 148 * 8);
  if (blocks < 1) blocks = 1;
  (astrai::note_launch(), paged_kv_write_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(k),
                                               static_cast<const __nv_bfloat16*>(v), ld_src, slot, T, Hkv, page_size, n_pages,
                                               static_cast<__nv_bfloat16*>(kc), static_cast<__nv_bfloat16*>(vc), D));
}

void paged_kv_gather(const void* kc, const void* vc, const int* table, int max_pages, const int* lens, int B, int S_out,
                     int Hkv, int page_size, int n_pages, void* ko, void* vo, int D, cudaStream_t s) {
  const long long work = (long long)B * S_out * Hkv * (D / 8);
  int blocks = (int)std::min<long long>((work + 255) / 256, 148 * 16);
  if (blocks < 1) blocks = 1;
  (astrai::note_launch(), paged_kv_gather_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(kc),
                                                static_cast<const __nv_bfloat16*>(vc), table, max_pages, lens, B, S_out,
                                                Hkv, page_size, n_pages, static_cast<__nv_bfloat16*>(ko),
                                                static_cast<__nv_bfloat16*>(vo), D));
}

template <int D>
static void decode_dispatch(const DecodeParams& p, dim3 grid, int G, cudaStream_t s) {
  switch (G) {
    case 1: (astrai::note_launch(), paged_decode_kernel<1, D><<<grid, 128, 0, s>>>(p)); break;
    case 2: (astrai::note_launch(), paged_decode_kernel<2, D><<<grid, 128, 0, s>>>(p)); break;
    case 4: (astrai::note_launch(), paged_decode_kernel<4, D><<<grid, 128, 0, s>>>(p)); break;
    case 8: (astrai::note_launch(), paged_decode_kernel<8, D><<<grid, 128, 0, s>>>(p)); break;
    default: throw std::runtime_error("paged_decode: n_heads / n_kv_heads must be 1, 2, 4 or 8");
  }
}

// splits > 1 writes partials to part_acc [B*Hq*splits*D] / part_ml [B*Hq*splits*2]; D = 64 or 128
void paged_decode_launch(const void* q, long long ldq, const void* kc, const void* vc, const int* table, int max_pages,
                         int n_pages, const int* lens, int B, int Hq, int Hkv, int page_size, int splits, float scale_log2,
                         float* part_acc, float* part_ml, void* out, long long ldo, int D, cudaStream_t s) {
  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.kc = static_cast<const __nv_bfloat16*>(kc);
  p.vc = static_cast<const __nv_bfloat16*>(vc);
  p.table = table;
  p.max_pages = max_pages;
  p.n_pages = n_pages;
  p.lens = lens;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.page_size = page_size;
  p.splits = splits;
  p.scale_log2 = scale_log2;
  p.part_acc = part_acc;
  p.part_ml = part_ml;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  dim3 grid(splits, Hkv, B);
  if (D == 128)
    decode_dispatch<128>(p, grid, Hq / Hkv, s);
  else if (D == 64)
    decode_dispatch<64>(p, grid, Hq / Hkv, s);
  else
    throw std::runtime_error("paged_decode: head_dim must be 64 or 128");
  if (splits > 1)
    (astrai::note_launch(), decode_combine_kernel<<<B * Hq, D, 0, s>>>(part_acc, part_ml, B, Hq, Hkv, splits,
                                                                      static_cast<__nv_bfloat16*>(out), ldo, D));
}

void decode_combine(const float* part_acc, const float* part_ml, int B, int Hq, int Hkv, int splits, void* out,
                    long long ldo, int D, cudaStream_t s) {
  (astrai::note_launch(), decode_combine_kernel<<<B * Hq, D, 0, s>>>(part_acc, part_ml, B, Hq, Hkv, splits,
                                                                    static_cast<__nv_bfloat16*>(out), ldo, D));
}

// Splits per (batch row, kv head). The tensor-core kernel runs one persistent CTA per SM over
// (row, kv head, split) items of 128-key tiles, and every item boundary drains its pipeline: split
// only as far as needed to give each SM an item (B32 x 4096 keys, Hkv 4: 1 split 63 us, 2 74 us,
// 10 80 us on B200), keeping at least 2 tiles (256 keys of capacity) per split; at most 32.
int decode_splits(int B, int Hkv, int max_len, int sms) {
  const int pairs = std::max(1, B * Hkv);
  const int want = std::max(1, sms / pairs);
  const int max_splits = std::max(1, (max_len + 255) / 256);
  return std::max(1, std::min(want, std::min(max_splits, 32)));
}

// ASTRAI_SAMPLE_CTA=0 keeps every vocabulary on the cluster kernel (for comparisons)
static bool sample_cta_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_SAMPLE_CTA");
    return !(e && e[0] == '0');
  }();
  return on;
}

void sample_tokens(const void* logits, int f32, long long ld, int rows, int V, const float* temperature,
                   const int* top_k, const float* top_p, const float* penalty, const long long* hist, int hist_len,
                   long long ld_hist, const unsigned long long* rng, long long* out_tok, float* out_lp,
                   cudaStream_t s) {
  if (V <= SMH_MAXV && sample_cta_enabled()) {
    // a cluster of four 256-thread CTAs per row while the rows leave SMs idle, one 1024-thread CTA after
    if ((long long)rows * 4 <= 2LL * 148) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(rows * 4);
      cfg.blockDim = dim3(256);
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 4;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      note_launch();
      const cudaError_t e = cudaLaunchKernelEx(&cfg, sample_hist_kernel<256, 4>, logits, f32, ld, V, temperature, top_k,
                                               top_p, penalty, hist, hist_len, ld_hist, rng, out_tok, out_lp);
      if (e != cudaSuccess) throw std::runtime_error(std::string("sample: launch failed: ") + cudaGetErrorString(e));
    } else {
      (astrai::note_launch(), sample_hist_kernel<1024, 1><<<rows, 1024, 0, s>>>(logits, f32, ld, V, temperature, top_k,
                                                                                top_p, penalty, hist, hist_len, ld_hist,
                                                                                rng, out_tok, out_lp));
    }
    return;
  }
  const int cs = (V + SMP_CHUNK - 1) / SMP_CHUNK;
  if (cs > SMP_MAX_CLUSTER) throw std::runtime_error("sample: vocabulary larger than 262144 is not supported");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows * cs);
  cfg.blockDim = dim3(SMP_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cs > 8) {
    static bool nonportable_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!nonportable_set[dev & 63]) {
      cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      nonportable_set[dev & 63] = true;
    }
  }
  note_launch();
  const cudaError_t e = cudaLaunchKernelEx(&cfg, sample_kernel, logits, f32, ld, V, temperature, top_k, top_p, penalty,
                                           hist, hist_len, ld_hist, rng, out_tok, out_lp);
  if (e != cudaSuccess) throw std::runtime_error(std::string("sample: launch failed: ") + cudaGetErrorString(e));
}

}  // namespace astrai_host
