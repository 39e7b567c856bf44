// Paged split-KV decode attention on the tensor cores (sm_100a).
//
// One query token per sequence attends over its paged K/V cache
// (cache[page][kv_head][slot][D], bf16, D = 64 or 128). The G = Hq / Hkv
// query heads of one KV head share every K/V row, so the kernel computes
//
//   S^T = K_tile Q^T    M = 128 keys, N = 64 (the G heads, padded), K = D
//   O^T += V_tile^T P^T M = 128 (D rows, padded for D = 64), N = 64, K = 128 keys
//
// with tcgen05.mma: each K/V tile is read from HBM once by TMA and used for
// all G heads, the scores land in TMEM one key per lane, and the online
// softmax runs one key per thread. This replaces the gather + repeat_kv +
// SDPA decode of the reference (astrai/inference/core/cache.py:256-276,
// astrai/model/components/attention.py:89-101) and plays the role of its
// mma.sync split-KV kernels (csrc/kernels/attn_paged_decode_split_kv_mma.cuh).
//
// Persistent CTAs walk work items (batch row, kv head, split) round-robin:
//   warp 0      TMA producer: the page table is read by one thread; each
//               128-key tile is 1 (page_size % 128 == 0) or 128 / page_size
//               boxes per 64-column chunk, into a 2-stage K / V ring
//   warp 1      TMEM owner + MMA issuer
//   warps 2..5  Q staging, softmax (thread = key = TMEM lane), P^T to smem,
//               lazy O rescaling (only when a head's running max grows by
//               more than 2^8), and the epilogue (thread = head-dim row of O^T)
// Split partials (m, l, acc) go to the workspace merged by
// decode_combine_kernel (inference.cu), in the same layout as the CUDA-core
// kernel, which stays the path for other page sizes and head counts.
// All waits are time-bounded (common.cuh).
#include <cstdint>
#include <stdexcept>

#include "common.cuh"

namespace astrai {

namespace {

constexpr int DT_THREADS = 192;
constexpr int DT_N = 64;                // MMA N: query heads of one KV head, padded
constexpr int DT_KCHUNK = 128 * 128;    // one [128 keys][64 d] bf16 chunk, 128B-swizzled (16 KB)
constexpr int DT_QCHUNK = DT_N * 128;   // one [64 heads][64 d] chunk (8 KB)
constexpr int DT_PSLOT = 128 * 128;     // P^T [128 keys][64 heads] (16 KB)
// Ring depths: a K stage frees as soon as its S MMA is done, a V stage (with the P^T slot) only
// after its P V MMA, so K runs ahead by a stage. Shared memory at D = 128: 3 x 32 KB K + 2 x 32 KB V
// + 2 x 16 KB Q (double-buffered over items) + 2 x 16 KB P^T = 224 KB.
template <int D>
struct DtStages;
template <>
struct DtStages<128> {
  static constexpr int K = 3, V = 2;
};
template <>
struct DtStages<64> {
  static constexpr int K = 4, V = 4;
};

__device__ __forceinline__ uint32_t swz128(uint32_t base, int r, int g) {
  return base + r * 128 + ((g ^ (r & 7)) << 4);
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void fence_proxy_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 32 lanes x 8 columns of TMEM -> 8 registers per thread
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

}  // namespace

struct DecodeTcParams {
  const __nv_bfloat16* q;  // [B, Hq * D] rows (stride ldq)
  long long ldq;
  const int* table;        // [B, max_pages]
  int max_pages, n_pages;  // table entries outside [0, n_pages) are skipped
  const int* lens;         // [B] cached keys, the current token included
  int B, Hq, Hkv, page_size, splits, box_rows;
  float scale_log2;
  float* part_acc;         // [B, Hkv, splits, G, D]
  float* part_ml;          // [B, Hkv, splits, G, 2]
  __nv_bfloat16* out;      // [B, Hq * D] rows (stride ldo), when splits == 1
  long long ldo;
  int* err;
};

template <int D, int G>
__global__ void __launch_bounds__(DT_THREADS, 1)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           DecodeTcParams p) {
  // a kernel launched after this one with programmatic dependent launch may start now (it waits for
  // this grid to finish before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(G >= 1 && G <= 16, "1 to 16 query heads per KV head");
  constexpr int NCH = D / 64;                       // 64-column chunks per row
  constexpr int KV_BYTES = NCH * DT_KCHUNK;         // one K (or V) tile
  constexpr int GC = G <= 8 ? 8 : 16;               // TMEM columns read per thread (x8 / x16 loads)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KST = DtStages<D>::K, VST = DtStages<D>::V;
  // K ring | V ring | Q (2 item buffers x 2 chunks) | P^T (2 slots) | reductions | barriers. For D = 64
  // the unused half of the V^T operand's M reads the 16 KB after a V stage (the next stage or Q).
  uint8_t* sK = smem;
  uint8_t* sV = sK + KST * KV_BYTES;
  uint8_t* sQ = sV + VST * KV_BYTES;
  uint8_t* sP = sQ + 2 * 2 * DT_QCHUNK;
  float* sRed = reinterpret_cast<float*>(sP + 2 * DT_PSLOT);  // [2][4 warps][G] maxima, then [4][G] sums
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRed + 2 * 4 * 16 + 4 * 16);
  uint64_t* kfull = bars;           // [KST] K tile landed
  uint64_t* kfree = kfull + KST;    // [KST] S MMA of the K tile done
  uint64_t* vfull = kfree + KST;    // [VST] V tile landed
  uint64_t* vfree = vfull + VST;    // [VST] P V of the tile done: V stage and P^T slot free, O^T updated
  uint64_t* sfull = vfree + VST;    // [2] S^T of the buffer in TMEM
  uint64_t* sfree = sfull + 2;      // [2] S^T read by the softmax (4 warps)
  uint64_t* pfull = sfree + 2;      // [2] P^T written (4 warps)
  uint64_t* qfull = pfull + 2;      // [2] Q of an item staged in buffer n & 1 (4 warps)
  uint64_t* qfree = qfull + 2;      // [2] last S MMA of the item in buffer n & 1 done
  uint64_t* ofree = qfree + 2;      // [2] O^T buffer n & 1 read out (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ofree + 2);

  const int warp = warp_id(), lane = lane_id();
  const int items = p.B * p.Hkv * p.splits;
  if (threadIdx.x == 0) {
    for (int i = 0; i < KST; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kfree[i], 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(&vfull[i], 1);
      mbar_init(&vfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], 4);
      mbar_init(&pfull[i], 4);
      mbar_init(&qfull[i], 4);
      mbar_init(&qfree[i], 1);
      mbar_init(&ofree[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S^T buffers at tmem + 0 / + 64, O^T of item n at tmem + 128 + 64 (n & 1)
  auto tO = [&](int n) { return tmem + 128u + 64u * (uint32_t)(n & 1); };

  // tile range of an item: tiles are the 128-key blocks of the row, split evenly
  auto item_range = [&](int item, int& b, int& hk, int& split, int& t0, int& t1, int& len) {
    split = item % p.splits;
    hk = (item / p.splits) % p.Hkv;
    b = item / (p.splits * p.Hkv);
    len = p.lens[b];
    const int tiles = (max(len, 0) + 127) / 128;
    const int tps = (tiles + p.splits - 1) / p.splits;
    t0 = min(tiles, split * tps);
    t1 = min(tiles, t0 + tps);
  };

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producers: lane 0 K, lane 1 V
    if (lane < 2) {
      const bool isk = lane == 0;
      const CUtensorMap* map = isk ? &tmK : &tmV;
      prefetch_tmap(map);
      const int ST = isk ? KST : VST;
      uint64_t* full = isk ? kfull : vfull;
      uint64_t* freeb = isk ? kfree : vfree;
      uint8_t* ring = isk ? sK : sV;
      const int nsub = 128 / p.box_rows;
      const uint32_t sub_bytes = (uint32_t)p.box_rows * 128u;
      long long g = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        int b, hk, split, t0, t1, len;
        item_range(item, b, hk, split, t0, t1, len);
        const int* trow = p.table + (long long)b * p.max_pages;
        for (int t = t0; t < t1; ++t, ++g) {
          const int s = (int)(g % ST);
          if (g >= ST && !(ok = mbar_wait(&freeb[s], (uint32_t)(((g / ST) - 1) & 1), p.err, kErrWaitEmpty))) break;
          int rows[8];  // TMA row coordinate of each sub-block, -1 when skipped (nsub <= 8 needs box_rows >= 16)
          uint32_t bytes = 0;
          for (int i = 0; i < nsub; ++i) {
            const int key = t * 128 + i * p.box_rows;
            const int pidx = key / p.page_size;
            const int page = (key < len && pidx < p.max_pages) ? trow[pidx] : -1;
            rows[i] = (page >= 0 && page < p.n_pages)
                          ? (int)(((long long)page * p.Hkv + hk) * p.page_size + key % p.page_size)
                          : -1;
            if (rows[i] >= 0) bytes += sub_bytes * NCH;
          }
          uint8_t* dst = ring + s * KV_BYTES;
          mbar_expect_tx(&full[s], bytes);
          for (int i = 0; i < nsub; ++i)
            if (rows[i] >= 0)
#pragma unroll
              for (int c = 0; c < NCH; ++c) tma_load_2d(dst + c * DT_KCHUNK + i * sub_bytes, map, &full[s], c * 64, rows[i]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, DT_N, 0, 0);  // S^T: K (K-major) x Q (K-major)
      constexpr uint32_t idO = idesc_bf16(128, DT_N, 1, 1);  // O^T: V^T (MN-major) x P^T (MN-major)
      long long g = 0;
      bool ok = true;
      int n_it = 0;
      auto issue_pv = [&](long long gg, bool first, int n) -> bool {
        const int vs = (int)(gg % VST), ps = (int)(gg & 1);
        if (!mbar_wait(&pfull[ps], (uint32_t)((gg >> 1) & 1), p.err, kErrWaitAccFull) ||
            !mbar_wait(&vfull[vs], (uint32_t)((gg / VST) & 1), p.err, kErrWaitFull))
          return false;
        tc_fence_after();
        // V^T as A: M = head-dim rows in 64-row chunks DT_KCHUNK apart
        const uint64_t dV = sdesc_sw128(smem_u32(sV + vs * KV_BYTES), DT_KCHUNK, 1024);
        const uint64_t dP = sdesc_sw128(smem_u32(sP + ps * DT_PSLOT), DT_PSLOT, 1024);
#pragma unroll
        for (int k = 0; k < 8; ++k)  // 16 keys per step: +2048 bytes in both MN-major operands
          umma_bf16(tO(n), dV + (uint64_t)(k * 128), dP + (uint64_t)(k * 128), idO, !(first && k == 0));
        umma_commit(&vfree[vs]);
        return true;
      };
      // n_it counts the items with keys (the softmax warps stage Q / read O^T for those only)
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        int b, hk, split, t0, t1, len;
        item_range(item, b, hk, split, t0, t1, len);
        if (t1 <= t0) continue;
        const int qb = n_it & 1;
        if (!(ok = mbar_wait(&qfull[qb], (uint32_t)((n_it >> 1) & 1), p.err, kErrWaitFull))) break;
        // the first P V of this item overwrites O^T buffer qb: the epilogue of item n_it - 2 must have read it
        if (n_it >= 2 && !(ok = mbar_wait(&ofree[qb], (uint32_t)(((n_it - 2) >> 1) & 1), p.err, kErrWaitAccEmpty)))
          break;
        const uint64_t dQ = sdesc_sw128(smem_u32(sQ + qb * 2 * DT_QCHUNK), 16, 1024);
        for (int t = t0; t < t1 && ok; ++t, ++g) {
          const int ks = (int)(g % KST), sb = (int)(g & 1);
          if (!(ok = mbar_wait(&kfull[ks], (uint32_t)((g / KST) & 1), p.err, kErrWaitFull))) break;
          if (g >= 2 && !(ok = mbar_wait(&sfree[sb], (uint32_t)(((g - 2) >> 1) & 1), p.err, kErrWaitAccEmpty))) break;
          tc_fence_after();
          const uint64_t dK = sdesc_sw128(smem_u32(sK + ks * KV_BYTES), 16, 1024);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t ok_ = (uint64_t)(((k >> 2) * DT_KCHUNK + (k & 3) * 32) >> 4);
            const uint64_t oq = (uint64_t)(((k >> 2) * DT_QCHUNK + (k & 3) * 32) >> 4);
            umma_bf16(tmem + sb * 64, dK + ok_, dQ + oq, idS, k > 0);
          }
          umma_commit(&sfull[sb]);
          umma_commit(&kfree[ks]);
          if (t == t1 - 1) umma_commit(&qfree[qb]);
          // P V of the previous tile overlaps this tile's softmax
          if (t > t0) ok = issue_pv(g - 1, t - 1 == t0, n_it);
        }
        if (ok) ok = issue_pv(g - 1, t1 - 1 == t0, n_it);
        ++n_it;
      }
    }
  } else {
    // ---------------------------------------------------------- softmax + epilogue (128 threads)
    const int w4 = warp - 2;  // TMEM lane quarter of this warp (warps 2..5 -> lanes 64..127, 0..63: warp % 4)
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // key row of the tile == TMEM lane == head-dim row of O^T
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int tid = w4 * 32 + lane;
    long long g = 0;
    int n_it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      int b, hk, split, t0, t1, len;
      item_range(item, b, hk, split, t0, t1, len);
      const long long pbase = (((long long)b * p.Hkv + hk) * p.splits + split) * G;
      if (t1 <= t0) {  // no keys for this split: empty partial
        if (p.splits > 1) {
          for (int i = tid; i < G * D; i += 128) p.part_acc[pbase * D + i] = 0.f;
          if (tid < G) {
            p.part_ml[(pbase + tid) * 2] = -INFINITY;
            p.part_ml[(pbase + tid) * 2 + 1] = 0.f;
          }
        } else {
          for (int i = tid; i < G * D; i += 128)
            p.out[(long long)b * p.ldo + (hk * G + i / D) * D + i % D] = __float2bfloat16_rn(0.f);
        }
        continue;  // the MMA warp skips this item too
      }
      // stage Q into buffer n & 1: rows = the G heads, K-major 128B-swizzled chunks; the last S MMA of
      // item n - 2 (the buffer's previous user) is done
      const int qb = n_it & 1;
      if (n_it >= 2 && !(ok = mbar_wait(&qfree[qb], (uint32_t)(((n_it - 2) >> 1) & 1), p.err, kErrWaitAccFull))) break;
      {
        const __nv_bfloat16* qrow = p.q + (long long)b * p.ldq + (long long)hk * G * D;
        uint8_t* qbuf = sQ + qb * 2 * DT_QCHUNK;
        for (int i = tid; i < G * (D / 8); i += 128) {
          const int h = i / (D / 8), gr = i % (D / 8);
          const uint4 v = *reinterpret_cast<const uint4*>(qrow + h * D + gr * 8);
          sts128(swz128(smem_u32(qbuf + (gr >> 3) * DT_QCHUNK), h, gr & 7), v.x, v.y, v.z, v.w);
        }
      }
      fence_proxy_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&qfull[qb]);
      // validity of this thread's key per tile: inside the row and on a valid page
      const int* trow = p.table + (long long)b * p.max_pages;
      float m_run[G], l_t[G];
#pragma unroll
      for (int h = 0; h < G; ++h) m_run[h] = -INFINITY, l_t[h] = 0.f;
      for (int t = t0; t < t1; ++t, ++g) {
        const int s = (int)(g & 1);
        const uint32_t ph = (uint32_t)((g >> 1) & 1);
        const int key = t * 128 + r;
        const int pidx = key / p.page_size;
        const int page = (key < len && pidx < p.max_pages) ? trow[pidx] : -1;
        const bool valid = page >= 0 && page < p.n_pages;
        if (!(ok = mbar_wait(&sfull[s], ph, p.err, kErrWaitAccFull))) break;
        tc_fence_after();
        uint32_t raw[GC];
        if constexpr (GC == 8) {
          tmem_ld8(tmem + s * 64 + lane_off, *reinterpret_cast<uint32_t(*)[8]>(raw));
        } else {
          tmem_ld16(tmem + s * 64 + lane_off, *reinterpret_cast<uint32_t(*)[16]>(raw));
        }
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[s]);
        float sc[G];
#pragma unroll
        for (int h = 0; h < G; ++h) sc[h] = valid ? __uint_as_float(raw[h]) * p.scale_log2 : -INFINITY;
        // tile maximum of every head over the 128 keys
        float* red = sRed + (g & 1) * 4 * 16;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float v = sc[h];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == 0) red[w4 * 16 + h] = v;
        }
        named_bar_sync(1, 128);
        bool grow = false;
        float m_new[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float mt = fmaxf(fmaxf(red[h], red[16 + h]), fmaxf(red[32 + h], red[48 + h]));
          m_new[h] = fmaxf(m_run[h], mt);
          // lazy rescaling: keep the old maximum while the new one is at most 2^8 above it
          grow |= m_new[h] > m_run[h] + 8.f;
        }
        if (grow) {
          float alpha[G];
#pragma unroll
          for (int h = 0; h < G; ++h) {
            alpha[h] = m_run[h] == -INFINITY ? 0.f : ex2_approx(m_run[h] - m_new[h]);
            l_t[h] *= alpha[h];
            m_run[h] = m_new[h];
          }
          if (t > t0) {
            // O^T holds the PV of tile t-1 once its commit arrived; rescale this thread's row in place
            if (!(ok = mbar_wait(&vfree[(int)((g - 1) % VST)], (uint32_t)(((g - 1) / VST) & 1), p.err,
                                 kErrWaitAccFull)))
              break;
            tc_fence_after();
            uint32_t o[GC];
            if constexpr (GC == 8) {
              tmem_ld8(tO(n_it) + lane_off, *reinterpret_cast<uint32_t(*)[8]>(o));
            } else {
              tmem_ld16(tO(n_it) + lane_off, *reinterpret_cast<uint32_t(*)[16]>(o));
            }
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < G; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
            if constexpr (GC == 8) {
              tmem_st8(tO(n_it) + lane_off, *reinterpret_cast<uint32_t(*)[8]>(o));
            } else {
              tmem_st16(tO(n_it) + lane_off, *reinterpret_cast<uint32_t(*)[16]>(o));
            }
            tmem_wait_st();
          }
        }
        uint32_t pk[GC / 2];
#pragma unroll
        for (int h = 0; h < GC / 2; ++h) pk[h] = 0u;
#pragma unroll
        for (int h = 0; h < G; h += 2) {
          const float b0 = m_run[h] == -INFINITY ? 0.f : m_run[h];
          const float p0 = ex2_approx(sc[h] - b0);
          float p1 = 0.f;
          if (h + 1 < G) {
            const float b1 = m_run[h + 1] == -INFINITY ? 0.f : m_run[h + 1];
            p1 = ex2_approx(sc[h + 1] - b1);
            l_t[h + 1] += p1;
          }
          l_t[h] += p0;
          pk[h / 2] = pack_bf16(p0, p1);
        }
        // a key outside the row (or on a skipped page) has p = 0, but its V row holds whatever the page
        // or an earlier tile left there, possibly NaN: zero it once the V tile has landed
        if (!valid) {
          const int vs = (int)(g % VST);
          if (!(ok = mbar_wait(&vfull[vs], (uint32_t)((g / VST) & 1), p.err, kErrWaitFull))) break;
          const uint32_t vb = smem_u32(sV + vs * KV_BYTES);
#pragma unroll
          for (int c = 0; c < NCH; ++c)
#pragma unroll
            for (int q = 0; q < 8; ++q) sts128(swz128(vb + c * DT_KCHUNK, r, q), 0u, 0u, 0u, 0u);
        }
        // the P^T slot was last read by the PV of tile g-2
        if (g >= 2 && !(ok = mbar_wait(&vfree[(int)((g - 2) % VST)], (uint32_t)(((g - 2) / VST) & 1), p.err,
                                       kErrWaitAccFull)))
          break;
        const uint32_t pb = smem_u32(sP + s * DT_PSLOT);
#pragma unroll
        for (int q = 0; q < GC / 8; ++q) sts128(swz128(pb, r, q), pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        fence_proxy_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[s]);
      }
      if (!ok) break;
      // epilogue: O^T row r (head-dim index), after the last PV of the item
      const long long gl = g - 1;
      if (!(ok = mbar_wait(&vfree[(int)(gl % VST)], (uint32_t)((gl / VST) & 1), p.err, kErrWaitAccFull))) break;
      tc_fence_after();
      uint32_t o[GC];
      if constexpr (GC == 8) {
        tmem_ld8(tO(n_it) + lane_off, *reinterpret_cast<uint32_t(*)[8]>(o));
      } else {
        tmem_ld16(tO(n_it) + lane_off, *reinterpret_cast<uint32_t(*)[16]>(o));
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ofree[qb]);
      float* sums = sRed + 2 * 4 * 16;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float v = warp_sum(l_t[h]);
        if (lane == 0) sums[w4 * 16 + h] = v;
      }
      named_bar_sync(1, 128);
      if (r < D) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float L = sums[h] + sums[16 + h] + sums[32 + h] + sums[48 + h];
          const float A = __uint_as_float(o[h]);
          if (p.splits == 1) {
            p.out[(long long)b * p.ldo + (hk * G + h) * D + r] = __float2bfloat16_rn(L > 0.f ? A / L : 0.f);
          } else {
            p.part_acc[(pbase + h) * D + r] = A;
            if (r == 0) {
              p.part_ml[(pbase + h) * 2] = m_run[h];
              p.part_ml[(pbase + h) * 2 + 1] = L;
            }
          }
        }
      }
      // the sums are rewritten by the next item only after its first tile's barrier
      ++n_it;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

void make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);
int num_sms(int device);
int* error_word(int device);

template <int D, int G>
static void launch_dt(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeTcParams& p, int grid, size_t smem,
                      cudaStream_t s) {
  auto k = paged_decode_tc_kernel<D, G>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  (astrai::note_launch(), k<<<grid, DT_THREADS, smem, s>>>(tk, tv, p));
}

// True when the tensor-core kernel takes this shape: head_dim 64 / 128, 1 - 8, 12 or 16 query heads
// per KV head, page_size a multiple of 128 or a divisor of 128 of at least 16.
bool paged_decode_tc_supported(int D, int G, int page_size) {
  if (D != 64 && D != 128) return false;
  if (!(G >= 1 && (G <= 8 || G == 12 || G == 16))) return false;
  return page_size % 128 == 0 || (page_size >= 16 && 128 % page_size == 0);
}

void paged_decode_tc(const void* q, long long ldq, const void* kc, const void* vc, const int* table, int max_pages,
                     int n_pages, const int* lens, int B, int Hq, int Hkv, int page_size, int splits,
                     float scale_log2, float* part_acc, float* part_ml, void* out, long long ldo, int D,
                     cudaStream_t s) {
  const int G = Hq / Hkv;
  if (!paged_decode_tc_supported(D, G, page_size)) throw std::runtime_error("paged_decode_tc: unsupported shape");
  DecodeTcParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.table = table;
  p.max_pages = max_pages;
  p.n_pages = n_pages;
  p.lens = lens;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.page_size = page_size;
  p.splits = splits;
  p.box_rows = page_size % 128 == 0 ? 128 : page_size;
  p.scale_log2 = scale_log2;
  p.part_acc = part_acc;
  p.part_ml = part_ml;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = error_word(dev);
  // the cache as rows of D columns: row (page * Hkv + head) * page_size + slot
  CUtensorMap tk, tv;
  const uint64_t rows = (uint64_t)n_pages * Hkv * page_size;
  uint64_t dims[2] = {(uint64_t)D, rows};
  uint64_t strides[1] = {(uint64_t)D * 2};
  uint32_t box[2] = {64, (uint32_t)p.box_rows};
  make_tmap_bf16(&tk, kc, 2, dims, strides, box, true);
  make_tmap_bf16(&tv, vc, 2, dims, strides, box, true);
  const int dev_sms = num_sms(dev);
  const int items = B * Hkv * splits;
  const int grid = std::max(1, std::min(items, dev_sms));
  const int stages = D == 128 ? DtStages<128>::K + DtStages<128>::V : DtStages<64>::K + DtStages<64>::V;
  const size_t smem = 1024 + (size_t)stages * (D / 64) * DT_KCHUNK + 2 * 2 * DT_QCHUNK + 2 * DT_PSLOT +
                      (2 * 4 * 16 + 4 * 16) * sizeof(float) + 32 * sizeof(uint64_t);
#define ASTRAI_DT_CASE(DD, GG) \
  if (D == DD && G == GG) return launch_dt<DD, GG>(tk, tv, p, grid, smem, s);
  ASTRAI_DT_CASE(128, 1) ASTRAI_DT_CASE(128, 2) ASTRAI_DT_CASE(128, 3) ASTRAI_DT_CASE(128, 4) ASTRAI_DT_CASE(128, 5)
  ASTRAI_DT_CASE(128, 6) ASTRAI_DT_CASE(128, 7) ASTRAI_DT_CASE(128, 8) ASTRAI_DT_CASE(128, 12) ASTRAI_DT_CASE(128, 16)
  ASTRAI_DT_CASE(64, 1) ASTRAI_DT_CASE(64, 2) ASTRAI_DT_CASE(64, 3) ASTRAI_DT_CASE(64, 4) ASTRAI_DT_CASE(64, 5)
  ASTRAI_DT_CASE(64, 6) ASTRAI_DT_CASE(64, 7) ASTRAI_DT_CASE(64, 8) ASTRAI_DT_CASE(64, 12) ASTRAI_DT_CASE(64, 16)
#undef ASTRAI_DT_CASE
}

}  // namespace astrai_host
