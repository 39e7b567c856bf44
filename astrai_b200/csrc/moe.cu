// Mixture-of-experts kernels (sm_100a): router, expert-parallel dispatch /
// return over NVLink peer memory, weighted combine.
//
// Router (astrai/model/components/mlp.py:83-87 semantics): one warp per
// token, fp32 softmax over E experts, top-k by repeated warp argmax (ties to
// the lower index), weights renormalised to sum 1; it also counts slots per
// expert and gives every (token, k) slot its position among the slots of its
// expert (atomic ticket), which fixes where the slot's row lands in the
// expert's input block.
//
// Expert parallelism: experts are split over W ranks (E_local = E / W each).
// Every rank has a symmetric arena (same layout on all ranks, mapped into
// every peer). Rank r's expert e_l owns rows [start_el, start_el + n_el) of
// r's input block (each expert padded to whole 128-row tiles, so the grouped
// expert GEMMs see no tile spanning two experts), source ranks in rank
// order. Kernels:
//   dispatch   token rows -> owning rank's input block (P2P stores) + a
//              return address per row (source rank, slot);
//   return     expert output rows -> the source rank's slot block (P2P);
//   combine    out[t] = add[t] + sum_j w[t, j] * slot[t, j] (fp32);
//   combine_bwd dw[t, j] = <dout[t], slot[t, j]>, and w[t, j] * dout[t] ->
//              the expert input-gradient block on the owning rank (P2P);
//   zero_pad   clears the padding rows of an expert block.
//   layout     counts exchange + the dispatch layout, computed on the device
//              (no host round trip, so a MoE step can be captured in a CUDA graph).
// A scatter kernel ends with a grid-completion count; the last CTA fences
// system-wide and adds 1 to its column of the phase's arrival counters on every
// rank. The consumer's ep_wait (bounded by wait_ns; kErrWaitPeer on expiry)
// waits until every column reached the number of rounds this rank has consumed
// plus one, a count kept in device memory; no host-side epoch is involved, so
// replaying a captured graph continues the sequence. Row indices are
// bounds-checked against the arena capacity (kErrBadArg, row skipped) so a bad
// layout cannot fault.
#include <stdexcept>
#include <string>

#include <cuda_fp8.h>

#include "common.cuh"
#include "ep_arena.h"

namespace astrai {

// ------------------------------------------------------------------ router
__device__ __forceinline__ unsigned long long topk_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order-preserving
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(idx));
}

template <int EPL>  // experts per lane
__global__ void __launch_bounds__(256) moe_router_kernel(const void* __restrict__ logits, int logits_f32, long long ld,
                                                         int T, int E, int k, float* __restrict__ probs,
                                                         int* __restrict__ idx_out, float* __restrict__ w_out,
                                                         int* __restrict__ counts, int* __restrict__ pos) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    float v[EPL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      float x = -INFINITY;
      if (e < E) {
        x = logits_f32 ? reinterpret_cast<const float*>(logits)[(long long)t * ld + e]
                       : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[(long long)t * ld + e]);
      }
      v[i] = x;
      mx = fmaxf(mx, x);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      v[i] = (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
      sum += v[i];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      v[i] *= inv;
      if (lane + 32 * i < E) probs[(long long)t * E + lane + 32 * i] = v[i];
    }
    // top-k: k warp-wide argmax rounds
    float sel_p[8];
    int sel_e[8];
    float sel_sum = 0.f;
    float cand[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) cand[i] = (lane + 32 * i < E) ? v[i] : -INFINITY;
    for (int j = 0; j < k; ++j) {
      unsigned long long best = 0ull;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const unsigned long long key = topk_key(cand[i], lane + 32 * i);
        best = key > best ? key : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffff, best, o);
        best = other > best ? other : best;
      }
      const int e = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
      const int owner = e & 31, slot = e >> 5;
      float pe = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (i == slot && lane == owner) {
          pe = cand[i];
          cand[i] = -INFINITY;
        }
      pe = __shfl_sync(0xffffffff, pe, owner);
      if (j < 8) {
        sel_p[j] = pe;
        sel_e[j] = e;
      }
      sel_sum += pe;
    }
    if (lane == 0) {
      const float rs = 1.f / sel_sum;
      for (int j = 0; j < k && j < 8; ++j) {
        idx_out[(long long)t * k + j] = sel_e[j];
        w_out[(long long)t * k + j] = sel_p[j] * rs;
        pos[(long long)t * k + j] = atomicAdd(counts + sel_e[j], 1);
      }
    }
  }
}

// ------------------------------------------------------------------ EP arena plumbing


__device__ __forceinline__ char* arena(const EPArena& a, int q, long long off) {
  return reinterpret_cast<char*>(a.peer_base[q]) + off;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_sys_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// This rank's arrival at `phase` on every rank (itself included): counter [phase][rank] += 1.
__device__ __forceinline__ void arrive_all(const EPArena& a, int phase) {
  __threadfence_system();
  for (int q = 0; q < a.world; ++q)
    red_release_sys_add_u32(reinterpret_cast<unsigned*>(arena(a, q, a.off_flags)) + phase * a.world + a.rank, 1u);
}

// Last CTA to finish announces this rank's arrival at `phase`.
__device__ void grid_done_signal(const EPArena& a, int phase) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {
      arrive_all(a, phase);
      *a.done = 0u;
    }
  }
}

// Bounded wait of one thread until counter [phase][q] of this rank's block reaches `want`
// (wrap-around safe); false after flagging kErrWaitPeer.
__device__ bool wait_arrival(const EPArena& a, int phase, int q, unsigned want) {
  const unsigned* f = reinterpret_cast<const unsigned*>(arena(a, a.rank, a.off_flags)) + phase * a.world + q;
  const uint64_t t0 = globaltimer();
  while (static_cast<int>(ld_acquire_sys_u32(f) - want) < 0) {
    if (globaltimer() - t0 > a.wait_ns) {
      set_error(a.err, kErrWaitPeer);
      return false;
    }
    __nanosleep(128);
  }
  return true;
}

__device__ __forceinline__ void copy_row(char* dst, const char* src, int d, int lane) {
  const int nv = d / 8;  // 16-byte vectors
  for (int v = lane; v < nv; v += 32)
    reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(src)[v];
}

__global__ void __launch_bounds__(512) ep_dispatch_kernel(EPArena a, const __nv_bfloat16* __restrict__ x,
                                                          long long ldx, const int* __restrict__ idx,
                                                          const int* __restrict__ pos, const int* __restrict__ base_row,
                                                          int n_slots, int k, int e_local, int* __restrict__ slot_row) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int s = gw; s < n_slots; s += nw) {
    const int e = idx[s];
    const int r = e / e_local;
    const long long row = (long long)base_row[e] + pos[s];
    if (r < 0 || r >= a.world || row < 0 || row >= a.rows_cap) {
      if (lane == 0) set_error(a.err, kErrBadArg);
      continue;
    }
    if (lane == 0) {
      slot_row[s] = static_cast<int>(row);
      reinterpret_cast<long long*>(arena(a, r, a.off_srcmap))[row] =
          (static_cast<long long>(a.rank) << 32) | static_cast<unsigned>(s);
    }
    copy_row(arena(a, r, a.off_xin) + row * a.d * 2, reinterpret_cast<const char*>(x + (long long)(s / k) * ldx), a.d,
             lane);
  }
  grid_done_signal(a, kPhDispatch);
}

// fp8 dispatch (opt-in; the reference only moves bf16): the token row is quantised to e4m3 with one
// fp32 scale per 128 columns (scale = amax / 448, the largest finite e4m3) and stored into the
// owner's fp8 block (d bytes) and scale block (d / 128 floats) instead of the bf16 block (2 d
// bytes): half the NVLink bytes. The owner rebuilds the bf16 block with ep_dequant_kernel.
// A warp covers 256 columns per step: 16 lanes x 8 columns form one 128-column scale block.
__global__ void __launch_bounds__(512) ep_dispatch_fp8_kernel(EPArena a, const __nv_bfloat16* __restrict__ x,
                                                              long long ldx, const int* __restrict__ idx,
                                                              const int* __restrict__ pos,
                                                              const int* __restrict__ base_row, int n_slots, int k,
                                                              int e_local, int* __restrict__ slot_row) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int s = gw; s < n_slots; s += nw) {
    const int e = idx[s];
    const int r = e / e_local;
    const long long row = (long long)base_row[e] + pos[s];
    if (r < 0 || r >= a.world || row < 0 || row >= a.rows_cap) {
      if (lane == 0) set_error(a.err, kErrBadArg);
      continue;
    }
    if (lane == 0) {
      slot_row[s] = static_cast<int>(row);
      reinterpret_cast<long long*>(arena(a, r, a.off_srcmap))[row] =
          (static_cast<long long>(a.rank) << 32) | static_cast<unsigned>(s);
    }
    const __nv_bfloat16* src = x + (long long)(s / k) * ldx;
    unsigned char* q8 = reinterpret_cast<unsigned char*>(arena(a, r, a.off_xin8)) + row * a.d;
    float* sc = reinterpret_cast<float*>(arena(a, r, a.off_xsc)) + row * (a.d / 128);
    for (int c0 = 0; c0 < a.d; c0 += 256) {
      const int col = c0 + lane * 8;
      float v[8];
      float amax = 0.f;
      if (col < a.d) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + col);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16(w[j]);
          v[2 * j] = f.x;
          v[2 * j + 1] = f.y;
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, o));  // 16-lane block
      const float scale = amax > 0.f ? amax / 448.f : 1.f;
      const float inv = 1.f / scale;
      if (col < a.d) {
        uint32_t pk[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * j] * inv, v[4 * j + 1] * inv),
                                                                   __NV_SATFINITE, __NV_E4M3);
          const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
              make_float2(v[4 * j + 2] * inv, v[4 * j + 3] * inv), __NV_SATFINITE, __NV_E4M3);
          pk[j] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        *reinterpret_cast<uint2*>(q8 + col) = make_uint2(pk[0], pk[1]);
        if ((lane & 15) == 0) sc[col / 128] = scale;
      }
    }
  }
  grid_done_signal(a, kPhDispatch);
}

// bf16 expert-input rows [0, rows) <- fp8 rows x their 128-column scales (own arena).
__global__ void __launch_bounds__(256) ep_dequant_kernel(EPArena a, long long rows) {
  const int vpr = a.d / 8;
  const long long n = rows * vpr;
  const unsigned char* q8 = reinterpret_cast<const unsigned char*>(arena(a, a.rank, a.off_xin8));
  const float* sc = reinterpret_cast<const float*>(arena(a, a.rank, a.off_xsc));
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(arena(a, a.rank, a.off_xin));
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < n; v += (long long)gridDim.x * blockDim.x) {
    const long long row = v / vpr;
    const int col = (int)(v % vpr) * 8;
    const uint2 u = *reinterpret_cast<const uint2*>(q8 + row * a.d + col);
    const float s = sc[row * (a.d / 128) + col / 128];
    const uint32_t w[2] = {u.x, u.y};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 lo = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[j] & 0xffffu), __NV_E4M3)));
      const float2 hi = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[j] >> 16), __NV_E4M3)));
      o[2 * j] = pack_bf16(lo.x * s, lo.y * s);
      o[2 * j + 1] = pack_bf16(hi.x * s, hi.y * s);
    }
    *reinterpret_cast<uint4*>(out + row * a.d + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Bounded wait for every rank's next arrival at `phase`; then this rank's round count advances.
__global__ void ep_wait_kernel(EPArena a, int phase) {
  __shared__ unsigned want;
  if (threadIdx.x == 0) want = a.expect[phase] + 1u;
  __syncthreads();
  const int q = threadIdx.x;
  if (q < a.world) wait_arrival(a, phase, q, want);
  __syncthreads();
  if (threadIdx.x == 0) a.expect[phase] = want;
}

// Valid rows of the local expert blocks -> the slot block of their source rank.
// Block layout: expert el owns rows [starts[el], starts[el] + n_rows[el]) of `rows`
// (padded to 128-row tiles; group_tile[row / 128] = el).
__global__ void __launch_bounds__(512) ep_return_kernel(EPArena a, const __nv_bfloat16* __restrict__ rows,
                                                        long long total_rows, const int* __restrict__ group_tile,
                                                        const int* __restrict__ starts, const int* __restrict__ n_rows,
                                                        long long ret_off, int phase) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  const long long* srcmap = reinterpret_cast<const long long*>(arena(a, a.rank, a.off_srcmap));
  for (long long row = gw; row < total_rows; row += nw) {
    const int el = group_tile[row >> 7];
    if (el < 0 || row - starts[el] >= n_rows[el]) continue;  // unused tile / padding row
    const long long key = srcmap[row];
    const int q = static_cast<int>(key >> 32);
    const long long s = static_cast<long long>(key & 0xFFFFFFFFll);
    if (q < 0 || q >= a.world || s >= a.slots_cap) {
      if (lane == 0) set_error(a.err, kErrBadArg);
      continue;
    }
    copy_row(arena(a, q, ret_off) + s * a.d * 2, reinterpret_cast<const char*>(rows + row * a.d), a.d, lane);
  }
  grid_done_signal(a, phase);
}

// out[t] = add[t] + sum_j w[t, j] * slots[t * k + j]   (w == nullptr: weights 1)
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* __restrict__ slots,
                                                         const float* __restrict__ w, const __nv_bfloat16* __restrict__ add,
                                                         __nv_bfloat16* __restrict__ out, int T, int k, int d) {
  const int lane = threadIdx.x & 31;
  const int nv = d / 8;
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += gridDim.x * (blockDim.x >> 5)) {
    for (int v = lane; v < nv; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (add) {
        const uint4 u = reinterpret_cast<const uint4*>(add + (long long)t * d)[v];
        const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16(ww[j]);
          acc[2 * j] = f.x;
          acc[2 * j + 1] = f.y;
        }
      }
      for (int j = 0; j < k; ++j) {
        const float g = w ? w[(long long)t * k + j] : 1.f;
        const uint4 u = reinterpret_cast<const uint4*>(slots + ((long long)t * k + j) * d)[v];
        const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16(ww[q]);
          acc[2 * q] += g * f.x;
          acc[2 * q + 1] += g * f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16(acc[0], acc[1]);
      o.y = pack_bf16(acc[2], acc[3]);
      o.z = pack_bf16(acc[4], acc[5]);
      o.w = pack_bf16(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + (long long)t * d)[v] = o;
    }
  }
}

// dw[s] = <dout[t], slots[s]>;  w[s] * dout[t] -> dyin row of slot s on its expert's rank
__global__ void __launch_bounds__(512) ep_combine_bwd_kernel(EPArena a, const __nv_bfloat16* __restrict__ dout,
                                                             const __nv_bfloat16* __restrict__ slots,
                                                             const float* __restrict__ w, const int* __restrict__ idx,
                                                             const int* __restrict__ slot_row, int n_slots, int k,
                                                             int e_local, float* __restrict__ dw) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int nv = a.d / 8;
  for (int s = gw; s < n_slots; s += nw) {
    const int t = s / k;
    const int r = idx[s] / e_local;
    const long long row = slot_row[s];
    const bool ok = r >= 0 && r < a.world && row >= 0 && row < a.rows_cap;
    if (!ok && lane == 0) set_error(a.err, kErrBadArg);
    const float g = w[s];
    float dot = 0.f;
    uint4* dst = ok ? reinterpret_cast<uint4*>(arena(a, r, a.off_dyin) + row * a.d * 2) : nullptr;
    for (int v = lane; v < nv; v += 32) {
      const uint4 du = reinterpret_cast<const uint4*>(dout + (long long)t * a.d)[v];
      const uint4 su = reinterpret_cast<const uint4*>(slots + (long long)s * a.d)[v];
      const uint32_t dd[4] = {du.x, du.y, du.z, du.w}, ss[4] = {su.x, su.y, su.z, su.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fd = unpack_bf16(dd[j]), fs = unpack_bf16(ss[j]);
        dot += fd.x * fs.x + fd.y * fs.y;
        o[j] = pack_bf16(g * fd.x, g * fd.y);
      }
      if (ok) dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[s] = dot;
  }
  grid_done_signal(a, kPhScatterBwd);
}

// Zero the padding rows (row - starts[el] >= n_rows[el]) of a block at `off` (own arena).
__global__ void ep_zero_pad_kernel(EPArena a, long long off, long long total_rows, const int* __restrict__ group_tile,
                                   const int* __restrict__ starts, const int* __restrict__ n_rows) {
  const int nv = a.d / 8;
  const long long total = total_rows * nv;
  uint4* base = reinterpret_cast<uint4*>(arena(a, a.rank, off));
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / nv;
    const int el = group_tile[row >> 7];
    if (el >= 0 && row - starts[el] >= n_rows[el]) base[i] = make_uint4(0, 0, 0, 0);
  }
}

// Counts exchange and dispatch layout on the device (one CTA). Every rank publishes its routed-slot
// counts per expert into every rank's counts block and announces it (phase kPhCounts); once all W
// rows are in, thread 0 derives what the host used to compute after an all-gather:
//   loads[e]  = sum over source ranks of counts[q][e]   (rows expert e receives)
//   padded[e] = loads[e] rounded up to 128-row tiles; experts of rank r' back to back from row 0
//   base_row[e] (this rank's first row in expert e's block on its owner) = start of e on the owner
//               + rows that lower source ranks send to e
// and for this rank's own experts the row count, start and padded size of each block, the block's
// total rows, and group_tile[t] = the expert of 128-row tile t (-1 past the total: the grouped GEMMs
// and the row kernels skip those tiles). If a rank would need more rows than the arena holds, the
// kernel flags kErrBadArg and publishes an empty layout (base rows out of range: the dispatch skips
// every row) instead of writing past the blocks.
constexpr int kEPMaxExperts = 256;
__global__ void __launch_bounds__(256) ep_layout_kernel(EPArena a, const int* __restrict__ counts, int E, int e_local,
                                                       int* __restrict__ base_row, int* __restrict__ n_rows,
                                                       int* __restrict__ starts, int* __restrict__ k_count,
                                                       int* __restrict__ group_tile, int max_tiles,
                                                       int* __restrict__ total_out) {
  __shared__ int s_load[kEPMaxExperts], s_start[kEPMaxExperts], s_before[kEPMaxExperts], s_total, s_over;
  __shared__ unsigned want;
  const int W = a.world;
  // 1. publish this rank's counts row on every rank, then announce it
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) {
    const int q = i / E, e = i % E;
    reinterpret_cast<int*>(arena(a, q, a.off_counts))[a.rank * E + e] = counts[e];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    arrive_all(a, kPhCounts);
    want = a.expect[kPhCounts] + 1u;
  }
  __syncthreads();
  // 2. wait for every rank's row (one thread per source rank)
  if (threadIdx.x < W) wait_arrival(a, kPhCounts, threadIdx.x, want);
  __syncthreads();
  // 3. the layout, one thread per expert: its load over all source ranks, the rows sent by lower ranks,
  //    and its first row inside its owner's block (padded loads of the owner's earlier experts)
  const volatile int* c = reinterpret_cast<const volatile int*>(arena(a, a.rank, a.off_counts));
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int load = 0, before = 0;
    for (int q = 0; q < W; ++q) {
      const int v = c[q * E + e];
      load += v;
      if (q < a.rank) before += v;
    }
    s_load[e] = load;
    s_before[e] = before;
  }
  if (threadIdx.x == 0) a.expect[kPhCounts] = want;
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int row = 0;
    for (int f = (e / e_local) * e_local; f < e; ++f) row += (s_load[f] + 127) / 128 * 128;
    s_start[e] = row;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bool over = false;
    int mine = 0;
    for (int r = 0; r < W; ++r) {
      const int last = (r + 1) * e_local - 1;
      const int rows = s_start[last] + (s_load[last] + 127) / 128 * 128;
      if (rows > a.rows_cap) over = true;
      if (r == a.rank) mine = rows;
    }
    if (over) {
      set_error(a.err, kErrBadArg);
      mine = 0;
    }
    s_over = over ? 1 : 0;
    s_total = mine;
    *total_out = mine;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) base_row[e] = s_over ? 0x40000000 : s_start[e] + s_before[e];
  const int first = a.rank * e_local;
  for (int el = threadIdx.x; el < e_local; el += blockDim.x) {
    const int load = s_total ? s_load[first + el] : 0;
    n_rows[el] = load;
    starts[el] = s_total ? s_start[first + el] : 0;
    k_count[el] = (load + 127) / 128 * 128;
  }
  for (int t = threadIdx.x; t < max_tiles; t += blockDim.x) {
    int g = -1;
    const int row = t * 128;
    if (row < s_total) {
      for (int el = 0; el < e_local; ++el) {
        const int st = s_start[first + el], len = (s_load[first + el] + 127) / 128 * 128;
        if (row >= st && row < st + len) g = el;
      }
    }
    group_tile[t] = g;
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

void moe_router(const void* logits, int f32, long long ld, int T, int E, int k, float* probs, int* idx, float* w,
                int* counts, int* pos, cudaStream_t s) {
  if (k < 1 || k > 8 || k > E) throw std::runtime_error("moe_router: need 1 <= top_k <= min(8, n_experts)");
  const int blocks = std::max(1, std::min((T + 7) / 8, 148 * 8));
  if (E <= 32) (astrai::note_launch(), moe_router_kernel<1><<<blocks, 256, 0, s>>>(logits, f32, ld, T, E, k, probs, idx, w, counts, pos));
  else if (E <= 64) (astrai::note_launch(), moe_router_kernel<2><<<blocks, 256, 0, s>>>(logits, f32, ld, T, E, k, probs, idx, w, counts, pos));
  else if (E <= 128) (astrai::note_launch(), moe_router_kernel<4><<<blocks, 256, 0, s>>>(logits, f32, ld, T, E, k, probs, idx, w, counts, pos));
  else if (E <= 256) (astrai::note_launch(), moe_router_kernel<8><<<blocks, 256, 0, s>>>(logits, f32, ld, T, E, k, probs, idx, w, counts, pos));
  else throw std::runtime_error("moe_router: at most 256 experts");
}

EPArena make_arena(const long long* peer_base, int rank, int world, const long long* offs, long long rows_cap,
                   long long slots_cap, int d, unsigned* done, unsigned* expect, int* err,
                   unsigned long long wait_ns) {
  EPArena a;
  a.peer_base = peer_base;
  a.rank = rank;
  a.world = world;
  a.off_flags = offs[0];
  a.off_srcmap = offs[1];
  a.off_xin = offs[2];
  a.off_dyin = offs[3];
  a.off_ret = offs[4];
  a.off_ret2 = offs[5];
  a.off_xin8 = offs[6];
  a.off_xsc = offs[7];
  a.off_counts = offs[8];
  a.expect = expect;
  a.rows_cap = rows_cap;
  a.slots_cap = slots_cap;
  a.d = d;
  a.done = done;
  a.err = err;
  a.wait_ns = wait_ns;
  return a;
}

void ep_dispatch(const EPArena& a, const void* x, long long ldx, const int* idx, const int* pos, const int* base_row,
                 int n_slots, int k, int e_local, int* slot_row, int ctas, cudaStream_t s) {
  (astrai::note_launch(), ep_dispatch_kernel<<<ctas, 512, 0, s>>>(a, static_cast<const __nv_bfloat16*>(x), ldx, idx, pos, base_row, n_slots, k,
                                          e_local, slot_row));
}

void ep_dispatch_fp8(const EPArena& a, const void* x, long long ldx, const int* idx, const int* pos,
                     const int* base_row, int n_slots, int k, int e_local, int* slot_row, int ctas,
                     cudaStream_t s) {
  if (a.off_xin8 == 0 || a.off_xsc == 0 || a.d % 128 != 0)
    throw std::runtime_error("ep_dispatch_fp8: the arena has no fp8 block, or d is not a multiple of 128");
  (astrai::note_launch(), ep_dispatch_fp8_kernel<<<ctas, 512, 0, s>>>(a, static_cast<const __nv_bfloat16*>(x), ldx, idx,
                                                                        pos, base_row, n_slots, k, e_local, slot_row));
}

void ep_dequant(const EPArena& a, long long rows, int ctas, cudaStream_t s) {
  if (rows <= 0) return;
  if (a.off_xin8 == 0 || rows > a.rows_cap) throw std::runtime_error("ep_dequant: no fp8 block or too many rows");
  (astrai::note_launch(), ep_dequant_kernel<<<ctas * 4, 256, 0, s>>>(a, rows));
}

void ep_wait(const EPArena& a, int phase, cudaStream_t s) {
  if (a.world > 32) throw std::runtime_error("ep_wait: at most 32 ranks");
  (astrai::note_launch(), ep_wait_kernel<<<1, 32, 0, s>>>(a, phase));
}

void ep_layout(const EPArena& a, const int* counts, int E, int e_local, int* base_row, int* n_rows, int* starts,
               int* k_count, int* group_tile, int max_tiles, int* total, cudaStream_t s) {
  if (E > kEPMaxExperts || E != e_local * a.world || a.world > 256)
    throw std::runtime_error("ep_layout: need n_experts = e_local * world <= 256");
  (astrai::note_launch(), ep_layout_kernel<<<1, 256, 0, s>>>(a, counts, E, e_local, base_row, n_rows, starts, k_count,
                                                            group_tile, max_tiles, total));
}

void ep_return(const EPArena& a, const void* rows, long long total_rows, const int* group_tile, const int* starts,
               const int* n_rows, int to_ret2, int ctas, cudaStream_t s) {
  (astrai::note_launch(), ep_return_kernel<<<ctas, 512, 0, s>>>(a, static_cast<const __nv_bfloat16*>(rows), total_rows,
                                                               group_tile, starts, n_rows,
                                                               to_ret2 ? a.off_ret2 : a.off_ret,
                                                               to_ret2 ? kPhReturnBwd : kPhReturn));
}

void ep_combine(const void* slots, const float* w, const void* add, void* out, int T, int k, int d, cudaStream_t s) {
  const int blocks = std::max(1, std::min((T + 7) / 8, 148 * 16));
  (astrai::note_launch(), ep_combine_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(slots), w,
                                           static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out), T,
                                           k, d));
}

void ep_combine_bwd(const EPArena& a, const void* dout, const void* slots, const float* w, const int* idx,
                    const int* slot_row, int n_slots, int k, int e_local, float* dw, int ctas, cudaStream_t s) {
  (astrai::note_launch(), ep_combine_bwd_kernel<<<ctas, 512, 0, s>>>(a, static_cast<const __nv_bfloat16*>(dout),
                                             static_cast<const __nv_bfloat16*>(slots), w, idx, slot_row, n_slots, k,
                                             e_local, dw));
}

void ep_zero_pad(const EPArena& a, int which_dyin, long long total_rows, const int* group_tile, const int* starts,
                 const int* n_rows, cudaStream_t s) {
  (astrai::note_launch(), ep_zero_pad_kernel<<<148 * 4, 256, 0, s>>>(a, which_dyin ? a.off_dyin : a.off_xin,
                                                                    total_rows, group_tile, starts, n_rows));
}

}  // namespace astrai_host
