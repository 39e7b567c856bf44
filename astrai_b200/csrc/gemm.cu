// Persistent bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   D[b, m, n] = alpha * sum_k A[b, m, k] * B[b, n, k] + beta * C[b, m, n]
//
// A and B may each be stored K-major (row = m or n, contiguous k) or MN-major
// (row = k, contiguous m or n); the four combinations cover forward
// (x W^T), data-grad (dY W) and weight-grad (dY^T X) of a linear layer and the
// Newton-Schulz products of Muon without any transpose copies.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128B-swizzled tiles into a STAGES-deep smem ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (128 x BN x 16)
//   warps 2..5  epilogue: tcgen05.ld the fp32 accumulator, apply alpha/beta,
//               convert and store; overlaps the next tile's MMAs because the
//               accumulator is double-buffered in TMEM (2 x BN columns).
// Synchronisation is mbarrier-only (full/empty per stage, acc_full/acc_empty
// per accumulator); every wait is time-bounded (common.cuh).
//
// Replaces the cuBLAS calls behind F.linear in the reference
// (astrai/model/components/linear.py:23-24) and the ATen matmuls of
// torch.optim.Muon used by scripts/tools/train.py:58-72.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>
#include <stdexcept>

#include "common.cuh"

namespace astrai {

constexpr int kMaxGatherPeers = 7;  // 8 ranks per node

struct GemmParams {
  int M, N, K, batch;
  int tiles_m, tiles_n, k_blocks;
  void* D;
  long long ldd, strideD;
  const void* C;
  long long ldc, strideC;
  float alpha, beta;
  int vec_ok;  // 16-byte vector stores/loads legal for D and C
  int* err;
  // Grouped modes (mixture-of-experts); all null for a plain / batched GEMM.
  //   group_tile: grouped-M. A and D are one [M_total, .] matrix whose 128-row
  //               tiles belong to group group_tile[m_tile]; B is batched by group.
  //   k_start / k_count: grouped-K. Batch b reduces over rows
  //               [k_start[b], k_start[b] + k_count[b]) of single A / B matrices
  //               (MN-major); D is batched by b. k_count 0 writes beta * C.
  const int* group_tile;
  const int* k_start;
  const int* k_count;
  // Fused SwiGLU epilogues (epi 0: plain GEMM).
  //   epi 1 (forward, B K-major = the packed [up; gate] weight [2F, K]): tile n covers output
  //         columns j in [n * BN/2, (n+1) * BN/2) of F; its B tile is up rows j.. and gate rows
  //         F + j.., so the accumulator holds u and g of the same columns. Writes h = (u, g) to D
  //         ([M, 2F], ldd) and a = silu(g) * u to aux ([M, F], ldaux).
  //   epi 2 (backward, D = dY W_down would be da [M, F]): da stays in TMEM; with the saved
  //         h ([M, 2F], ldh) the epilogue writes dh = (da * silu(g), da * u * silu'(g)) to aux.
  // optional wait-cycle counters (nullptr: off): [0] producer on empty, [1] MMA on full,
  // [2] MMA on acc_empty, [3] epilogue on acc_full (summed over the waiting threads' CTAs)
  unsigned long long* prof;
  int epi;
  int F;
  __nv_bfloat16* aux;
  long long ldaux;
  const __nv_bfloat16* h;
  long long ldh;
  // epi 3 (RoPE): rotate interleaved pairs of output columns [0, rope_cols) (heads of rope_hd
  // columns) by the angles of the row's position (rope_pos[row], or row % rope_seq) from the
  // fp32 (cos, sin) table [rope_max][rope_hd / 2], before rounding to bf16.
  const float2* rope_cs;
  const int* rope_pos;
  int rope_seq, rope_cols, rope_hd, rope_max;
  // Stream-K (sk_units > 0; plain GEMMs only): tiles [0, dp_tiles) are computed whole (CTA c takes
  // c, c + G, ...); the k-blocks of the remaining tiles (sk_units = their count x k_blocks) are
  // split evenly over the G CTAs, CTA c taking units [c U / G, (c + 1) U / G). Each CTA walks its
  // unit range from the end, so its first stream-K item is the only one that can lack the tile's
  // last k-block. Such a part (non-owner) stores its fp32 partial into its own slot sk_ws[c] and
  // raises sk_flags[c]; the tile's owner (the CTA holding its last k-block, always the highest of
  // the tile's CTAs) processes that tile last, waits for the flags of the lower CTAs that hold the
  // tile's other parts, adds their slots into its accumulator, runs the normal epilogue and clears
  // the flags for the next launch. Every wait is on a part that a lower CTA computed first.
  int dp_tiles;
  long long sk_units;
  float* sk_ws;
  int* sk_flags;
  // Fused all-gather (npeers > 0; plain bf16 GEMMs without C): D is this rank's column block of a
  // row-major output that every rank holds at the same offset of a symmetric buffer. Every vector
  // the epilogue stores at D + o is also stored at D + o + peer_delta[q] bytes (rank q's copy, over
  // NVLink) for q < npeers. When the grid's last tile is stored, the last CTA to finish raises
  // this rank's flag on every peer (gather_flag + peer_delta[q] <- gather_epoch, release).
  int npeers;
  long long peer_delta[kMaxGatherPeers];
  unsigned* gather_flag;
  unsigned* gather_done;  // grid-completion counter, zero between launches
  unsigned gather_epoch;
  // Fused reduce-scatter push (scatter_rpo > 0, with npeers / peer_delta / gather_* set for the
  // completion flag): D holds this rank's partial product; rows are owned in blocks of scatter_rpo
  // (rank o owns [o rpo, (o + 1) rpo)). After a tile is stored, its rows owned by another rank o go
  // into o's receive slot for this rank, D + scatter_recv_off + (rank rpo + row - o rpo) ldd (+ col)
  // elements, at rank o's copy (rank_delta[o] bytes away).
  int scatter_rpo, scatter_rank;
  long long scatter_recv_off;  // bytes from D to the receive slots
  long long rank_delta[kMaxGatherPeers + 1];
  // Symmetric output (sym != 0; M == N, D known to equal D^T, e.g. X X^T or A A with A symmetric):
  // tiles lying entirely below the diagonal (every column < every row; tiles of sym_bm x sym_bn) are
  // not computed, and sym_mirror_kernel copies the transpose of the upper triangle into them
  // afterwards. sym 2 (square tiles): the tile index space holds only the upper tiles (gemm_tile);
  // sym 1: the walk skips the lower ones.
  int sym, sym_bm, sym_bn;
};

// Fused all-gather: after the epilogue warps stored tile (b, mb, nb) into the local D, copy it from
// L2 to every peer's copy, one 16-byte vector per thread and consecutive threads along a row, so a
// warp writes 512 contiguous bytes per instruction over NVLink (the row-per-thread layout of the
// epilogue stores would send 16-byte fragments of 32 different rows).
template <int BM, int BN>
__device__ __forceinline__ void gather_copy_tile(const GemmParams& p, int b, int mb, int nb, int et, int nthreads) {
  constexpr int VPR = BN / 8;  // 16-byte vectors per tile row
  const __nv_bfloat16* D = reinterpret_cast<const __nv_bfloat16*>(p.D) + (long long)b * p.strideD;
  for (int i = et; i < BM * VPR; i += nthreads) {
    const int row = mb * BM + i / VPR, col = nb * BN + (i % VPR) * 8;
    if (row >= p.M || col >= p.N) continue;
    const __nv_bfloat16* src = D + (long long)row * p.ldd + col;
    char* dst0 = reinterpret_cast<char*>(const_cast<__nv_bfloat16*>(src));
    if (col + 8 <= p.N && p.vec_ok) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src));
#pragma unroll
      for (int q = 0; q < kMaxGatherPeers; ++q)
        if (q < p.npeers) *reinterpret_cast<uint4*>(dst0 + p.peer_delta[q]) = v;
    } else {
      for (int e = 0; e < 8 && col + e < p.N; ++e) {
        const __nv_bfloat16 v = src[e];
#pragma unroll
        for (int q = 0; q < kMaxGatherPeers; ++q)
          if (q < p.npeers) *reinterpret_cast<__nv_bfloat16*>(dst0 + 2 * e + p.peer_delta[q]) = v;
      }
    }
  }
}

// Fused reduce-scatter push of tile (b, mb, nb): rows owned by other ranks go to their receive slots
// (row-contiguous 16-byte stores, as in gather_copy_tile).
template <int BM, int BN>
__device__ __forceinline__ void scatter_copy_tile(const GemmParams& p, int mb, int nb, int et, int nthreads) {
  constexpr int VPR = BN / 8;
  const __nv_bfloat16* D = reinterpret_cast<const __nv_bfloat16*>(p.D);
  for (int i = et; i < BM * VPR; i += nthreads) {
    const int row = mb * BM + i / VPR, col = nb * BN + (i % VPR) * 8;
    if (row >= p.M || col >= p.N) continue;
    const int o = row / p.scatter_rpo;
    if (o == p.scatter_rank) continue;
    long long dl = 0;
#pragma unroll
    for (int q = 0; q <= kMaxGatherPeers; ++q)
      if (q == o) dl = p.rank_delta[q];
    const __nv_bfloat16* src = D + (long long)row * p.ldd + col;
    char* dst = reinterpret_cast<char*>(const_cast<__nv_bfloat16*>(D)) + p.scatter_recv_off + dl +
                ((long long)(p.scatter_rank * p.scatter_rpo + row - o * p.scatter_rpo) * p.ldd + col) * 2;
    if (col + 8 <= p.N && p.vec_ok) {
      *reinterpret_cast<uint4*>(dst) = __ldcg(reinterpret_cast<const uint4*>(src));
    } else {
      for (int e = 0; e < 8 && col + e < p.N; ++e) reinterpret_cast<__nv_bfloat16*>(dst)[e] = src[e];
    }
  }
}

// Programmatic dependent launch (the launch attribute set by the host launchers below): `trigger`
// lets the next kernel on the stream be scheduled, `wait` blocks until the previous grid has
// completed and its memory operations are visible. Both are no-ops in a launch without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// One unit of a CTA's work: tile `tile`, k-blocks [kb0, kb1).
struct WorkItem {
  int tile, kb0, kb1;
  int sk;       // stream-K tile index (tile - dp_tiles), -1 for a whole tile
  int ord;      // number of lower CTAs holding parts of the tile
  bool owner;   // holds the tile's last k-block
  bool partial; // the tile is split over several CTAs
};

// Grouped-M tiles whose group is negative are unused (an expert block sized for its capacity, of which
// only a device-side count of tiles is live): every role of the kernel skips them through WorkIter.
__device__ __forceinline__ bool tile_skipped(const GemmParams& p, int tile);

// Work walk of one worker (a CTA, or a CTA pair in gemm_pair_kernel): `idx` of `cnt` workers.
struct WorkIter {
  int t, idx, cnt;
  long long u, u_end;
  __device__ __forceinline__ void init(const GemmParams& p) { init(p, blockIdx.x, gridDim.x); }
  __device__ __forceinline__ void init(const GemmParams& p, int worker, int workers) {
    idx = worker;
    cnt = workers;
    t = worker;
    if (p.sk_units > 0) {
      u = (long long)worker * p.sk_units / workers;
      u_end = (long long)(worker + 1) * p.sk_units / workers;
    } else {
      u = u_end = 0;
    }
  }
  // worker whose unit range contains unit v (every range is non-empty: sk_units >= workers)
  __device__ __forceinline__ int worker_of_unit(const GemmParams& p, long long v) const {
    return (int)(((v + 1) * cnt - 1) / p.sk_units);
  }
  __device__ __forceinline__ bool next(const GemmParams& p, int num_tiles, int kblk_full, WorkItem& w) {
    const int limit = p.sk_units > 0 ? p.dp_tiles : num_tiles;
    if (p.group_tile || p.sym == 1)
      while (t < limit && tile_skipped(p, t)) t += cnt;
    if (t < limit) {
      w = {t, 0, kblk_full, -1, 0, true, false};
      t += cnt;
      return true;
    }
    if (u >= u_end) return false;
    // the last tile of the remaining range [u, u_end)
    const int KB = p.k_blocks;
    const long long tr = (u_end - 1) / KB;
    const long long tbeg = tr * KB;
    const long long lo = u > tbeg ? u : tbeg;
    w.tile = p.dp_tiles + (int)tr;
    w.kb0 = (int)(lo - tbeg);
    w.kb1 = (int)(u_end - tbeg);
    w.sk = (int)tr;
    w.ord = idx - worker_of_unit(p, tbeg);  // lower workers holding parts of this tile
    w.owner = w.kb1 == KB;
    w.partial = !(w.kb0 == 0 && w.kb1 == KB);
    u_end = lo;
    return true;
  }
};

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu_s32(int* f, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
// Bounded wait until *f == want (other CTAs of this launch, all resident, advance it).
__device__ __forceinline__ bool wait_flag_eq(const int* f, int want, int* err) {
  const uint64_t t0 = globaltimer();
  while (ld_acquire_gpu_s32(f) != want) {
    if (globaltimer() - t0 > ASTRAI_WAIT_NS) {
      set_error(err, kErrWaitFull);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// fast division (__fdividef: at most 2 ulp off for denominators below 2^126, 0 above, i.e. for
// g < -87 where the quotient is below 1e-37), as in the separate SwiGLU kernels
__device__ __forceinline__ float sigmoid_f(float g) { return __fdividef(1.f, 1.f + __expf(-g)); }

// accumulator columns one epilogue thread drains in the fused modes (BN / CSPLIT); the paired
// SwiGLU forward reads them as half as many (u, g) pairs
template <int BN, int CSPLIT>
__host__ __device__ constexpr int p_epi_per() { return BN / CSPLIT; }

// Operand batch coordinates and K range of one output tile.
struct TileK {
  int bA, bB, kbase, kblk;
};

__device__ __forceinline__ TileK tile_k(const GemmParams& p, int b, int mb, int bk) {
  TileK t{b, b, 0, p.k_blocks};
  if (p.group_tile) {
    t.bA = 0;
    t.bB = p.group_tile[mb];
  }
  if (p.k_count) {
    t.bA = t.bB = 0;
    t.kbase = p.k_start[b];
    t.kblk = (p.k_count[b] + bk - 1) / bk;
  }
  return t;
}

// Tile shapes: BM x BN per CTA, BK = 64 (one 128-byte swizzle atom of bf16).
//   BM = 128: one 128 x BN UMMA per k-step, accumulator double-buffered in
//             TMEM so the epilogue of tile t overlaps the MMAs of tile t+1.
//   BM = 256: two 128 x 256 UMMAs per k-step share the B tile (half the
//             L2->SM bytes per FLOP of BM = 128); both accumulators fill TMEM,
//             8 epilogue warps drain them.
template <int BM_, int BN_>
struct GemmCfg {
  static constexpr int BM = BM_;
  static constexpr int BN = BN_;
  static constexpr int BK = 64;
  static constexpr int MH = BM / 128;                 // 128-row MMA halves
  static constexpr int NACC = (BM == 128) ? 2 : 1;    // accumulator buffers
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES_FIT = (225 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr int TMEM_COLS = NACC * MH * BN;
  // BM = 256: 16 epilogue warps, each pair of warps on one TMEM lane quadrant
  // splits the columns, so a thread holds half a row (fits the early release)
  static constexpr int CSPLIT = MH;
  static constexpr int EPI_WARPS = 4 * MH * CSPLIT;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(TMEM_COLS <= 512, "accumulators exceed tensor memory");
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& b, int& mb, int& nb) {
  const int per = tiles_m * tiles_n;
  b = tile / per;
  int t = tile - b * per;
  constexpr int G = 8;  // group 8 row-tiles so B tiles stay hot in L2
  const int span = G * tiles_n;
  const int group = t / span;
  const int first = group * G;
  const int gsize = min(tiles_m - first, G);
  const int r = t - group * span;
  mb = first + r % gsize;
  nb = r / gsize;
}

// Symmetric output on square tiles (sym == 2): only the tiles on or above the diagonal exist in the
// tile index space, column by column (column nb holds rows 0 .. nb), so every worker's share of the
// walk is live work; 1-tile-wide columns keep each B tile hot in L2 across its column.
__device__ __forceinline__ int sym_tiles(int T) { return T * (T + 1) / 2; }
__device__ __forceinline__ void gemm_tile(const GemmParams& p, int tile, int& b, int& mb, int& nb) {
  if (p.sym == 2) {
    const int per = sym_tiles(p.tiles_m);
    b = tile / per;
    const int r = tile - b * per;
    int c = (int)((sqrtf(8.f * (float)r + 1.f) - 1.f) * 0.5f);
    while ((c + 1) * (c + 2) / 2 <= r) ++c;
    while (c * (c + 1) / 2 > r) --c;
    nb = c;
    mb = r - c * (c + 1) / 2;
    return;
  }
  tile_coords(tile, p.tiles_m, p.tiles_n, b, mb, nb);
}
__device__ __forceinline__ int gemm_num_tiles(const GemmParams& p) {
  return p.batch * (p.sym == 2 ? sym_tiles(p.tiles_m) : p.tiles_m * p.tiles_n);
}

__device__ __forceinline__ bool tile_skipped(const GemmParams& p, int tile) {
  int b, mb, nb;
  tile_coords(tile, p.tiles_m, p.tiles_n, b, mb, nb);
  if (p.sym) return (long long)(nb + 1) * p.sym_bn <= (long long)mb * p.sym_bm;
  return p.group_tile[mb] < 0;
}

// Lower triangle of a symmetric output from its upper triangle: one 32 x 32 block pair per CTA
// (block (bi, bj), bi >= bj, is written from the transpose of block (bj, bi)).
template <typename T>
__global__ void sym_mirror_kernel(T* __restrict__ D, int M, long long ldd, long long strideD) {
  __shared__ T tile[32][33];
  const int bi = blockIdx.x, bj = blockIdx.y;
  if (bj > bi) return;
  T* d = D + (long long)blockIdx.z * strideD;
  const int tx = threadIdx.x, ty = threadIdx.y;
  // read block (bj, bi) (rows bj*32.., cols bi*32..): upper side
  for (int r = ty; r < 32; r += blockDim.y) {
    const int row = bj * 32 + r, col = bi * 32 + tx;
    if (row < M && col < M) tile[r][tx] = d[(long long)row * ldd + col];
  }
  __syncthreads();
  // write block (bi, bj) = transpose; on the diagonal only below it
  for (int r = ty; r < 32; r += blockDim.y) {
    const int row = bi * 32 + r, col = bj * 32 + tx;
    if (row < M && col < M && row > col) d[(long long)row * ldd + col] = tile[tx][r];
  }
}

// bf16 version on 64 x 64 blocks, one CTA per block (bi, bj) with bi >= bj (blockIdx.x enumerates
// them row by row; blockIdx.y is the batch): the source block (bj, bi) is read with 16-byte row loads
// into shared memory (33-word row pitch: conflict-free stores) and written transposed with 16-byte
// stores, eight threads per 128-byte output row, so a warp stores four whole rows. Diagonal blocks
// and blocks cut by M take an element-wise path that writes only below the diagonal.
__global__ void __launch_bounds__(256) sym_mirror64_kernel(__nv_bfloat16* __restrict__ D, int M, long long ldd,
                                                          long long strideD) {
  __shared__ uint32_t tile[64 * 33];
  const int r = blockIdx.x;
  int bi = (int)((sqrtf(8.f * (float)r + 1.f) - 1.f) * 0.5f);  // r = bi (bi + 1) / 2 + bj, 0 <= bj <= bi
  while (bi * (bi + 1) / 2 > r) --bi;
  while ((bi + 1) * (bi + 2) / 2 <= r) ++bi;
  const int bj = r - bi * (bi + 1) / 2;
  const int i0 = bi * 64, j0 = bj * 64;
  __nv_bfloat16* d = D + (long long)blockIdx.y * strideD;
  const int tid = threadIdx.x;
  if (bi != bj && i0 + 64 <= M) {
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int q = tid + 256 * it, rr = q >> 3, k = q & 7;
      const uint4 v = *reinterpret_cast<const uint4*>(d + (long long)(j0 + rr) * ldd + i0 + 8 * k);
      uint32_t* t = tile + rr * 33 + 4 * k;
      t[0] = v.x;
      t[1] = v.y;
      t[2] = v.z;
      t[3] = v.w;
    }
    __syncthreads();
    const unsigned short* th = reinterpret_cast<const unsigned short*>(tile);
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int q = tid + 256 * it, c = q >> 3, k = q & 7;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t lo = th[(8 * k + 2 * e) * 66 + c], hi = th[(8 * k + 2 * e + 1) * 66 + c];
        w[e] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4*>(d + (long long)(i0 + c) * ldd + j0 + 8 * k) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return;
  }
  __nv_bfloat16* th = reinterpret_cast<__nv_bfloat16*>(tile);
  for (int idx = tid; idx < 64 * 64; idx += 256) {
    const int rr = idx >> 6, cc = idx & 63;
    if (j0 + rr < M && i0 + cc < M) th[rr * 66 + cc] = d[(long long)(j0 + rr) * ldd + i0 + cc];
  }
  __syncthreads();
  for (int idx = tid; idx < 64 * 64; idx += 256) {
    const int c = idx >> 6, rc = idx & 63;
    const int row = i0 + c, col = j0 + rc;
    if (row < M && col < M && row > col) d[(long long)row * ldd + col] = th[rc * 66 + c];
  }
}

template <int BM, int BN, int A_MN, int B_MN, int OUT_F32>
__global__ void __launch_bounds__(GemmCfg<BM, BN>::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = GemmCfg<BM, BN>;
  constexpr int BK = Cfg::BK, STAGES = Cfg::STAGES, MH = Cfg::MH, NACC = Cfg::NACC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = warp_id();
  const int lane = lane_id();
  // programmatic dependent launch: the next kernel on the stream may be scheduled now (it waits for
  // this grid before reading anything), and this one reads global memory only after the wait below
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], Cfg::EPI_WARPS);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS < 32 ? 32 : Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous grid has completed and its writes are visible

  const int num_tiles = gemm_num_tiles(p);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      WorkIter wi;
      wi.init(p);
      WorkItem w;
      while (ok && wi.next(p, num_tiles, p.k_blocks, w)) {
        const int tile = w.tile;
        int b, mb, nb;
        gemm_tile(p, tile, b, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        const TileK tk = tile_k(p, b, mb, BK);
        const int kbeg = w.sk >= 0 ? w.kb0 : 0, kend = w.sk >= 0 ? w.kb1 : tk.kblk;
        for (int kb = kbeg; kb < kend; ++kb) {
          const long long tw0 = p.prof ? clock64() : 0;
          const bool got = mbar_wait(&empty[stage], phase ^ 1, p.err, kErrWaitEmpty);
          if (p.prof) atomicAdd(p.prof + 0, (unsigned long long)(clock64() - tw0));
          if (!got) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          const int k0 = tk.kbase + kb * BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_3d(a_dst + c * 8192, &tmA, &full[stage], m0 + c * 64, k0, tk.bA);
          } else {
#pragma unroll
            for (int h = 0; h < MH; ++h) tma_load_3d(a_dst + h * 16384, &tmA, &full[stage], k0, m0 + h * 128, tk.bA);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(b_dst + c * 8192, &tmB, &full[stage], n0 + c * 64, k0, tk.bB);
          } else if (p.epi == 1) {
            // up rows then gate rows of the same BN/2 output columns (box = BN/2 rows)
            tma_load_3d(b_dst, &tmB, &full[stage], k0, nb * (BN / 2), tk.bB);
            tma_load_3d(b_dst + (BN / 2) * 128, &tmB, &full[stage], k0, p.F + nb * (BN / 2), tk.bB);
          } else {
            tma_load_3d(b_dst, &tmB, &full[stage], k0, n0, tk.bB);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_bf16(128, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      WorkIter wi;
      wi.init(p);
      WorkItem w;
      while (ok && wi.next(p, num_tiles, p.k_blocks, w)) {
        const int tile = w.tile;
        int b, mb, nb;
        gemm_tile(p, tile, b, mb, nb);
        const int kblk = tile_k(p, b, mb, BK).kblk;
        const int kbeg = w.sk >= 0 ? w.kb0 : 0, kend = w.sk >= 0 ? w.kb1 : kblk;
        const long long ta0 = p.prof ? clock64() : 0;
        const bool got_acc = mbar_wait(&acc_empty[acc], acc_phase ^ 1, p.err, kErrWaitAccEmpty);
        if (p.prof) atomicAdd(p.prof + 2, (unsigned long long)(clock64() - ta0));
        if (!got_acc) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * MH * BN;
        for (int kb = kbeg; kb < kend; ++kb) {
          const long long tf0 = p.prof ? clock64() : 0;
          const bool got = mbar_wait(&full[stage], phase, p.err, kErrWaitFull);
          if (p.prof) atomicAdd(p.prof + 1, (unsigned long long)(clock64() - tf0));
          if (!got) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t bd = B_MN ? sdesc_sw128(b_base + k * 2048, 8192, 1024) : sdesc_sw128(b_base + k * 32, 16, 1024);
#pragma unroll
            for (int h = 0; h < MH; ++h) {
              const uint64_t ad = A_MN ? sdesc_sw128(a_base + h * 16384 + k * 2048, 8192, 1024)
                                       : sdesc_sw128(a_base + h * 16384 + k * 32, 16, 1024);
              umma_bf16(d_tmem + h * BN, ad, bd, idesc, (kb != kbeg) || k != 0);
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&acc_full[acc]);
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                     // TMEM lane quadrant this warp may access
    const int half = ((warp - 2) >> 2) % MH;    // which 128-row MMA half (BM = 256)
    const int cpart = (warp - 2) >> (2 + (MH - 1));  // which column part (BM = 256)
    constexpr int BNP = BN / Cfg::CSPLIT;       // columns drained by one thread
    int acc = 0;
    uint32_t acc_phase = 0;
    WorkIter wi;
    wi.init(p);
    WorkItem w;
    constexpr int EPI_THREADS = Cfg::EPI_WARPS * 32;
    const int et = threadIdx.x - 64;  // epilogue thread index
    while (wi.next(p, num_tiles, p.k_blocks, w)) {
      const int tile = w.tile;
      int b, mb, nb;
      gemm_tile(p, tile, b, mb, nb);
      const long long te0 = (p.prof && lane == 0) ? clock64() : 0;
      const bool got_full = mbar_wait(&acc_full[acc], acc_phase, p.err, kErrWaitAccFull);
      if (p.prof && lane == 0 && warp == 2) atomicAdd(p.prof + 3, (unsigned long long)(clock64() - te0));
      if (!got_full) break;
      tc_fence_after();
      if (w.partial) {
        // stream-K part: a non-owner parks its fp32 partial in its own slot; the owner adds the
        // lower CTAs' slots into its accumulator, then the regular epilogue below reads the sum.
        // Slot layout is thread-major (float4 v of epilogue thread et at [v][et]), so every warp
        // access is 512 contiguous bytes; owner and non-owner threads drain the same TMEM cells.
        const uint32_t t_part = tmem_base + ((uint32_t)(q * 32) << 16) + (acc * MH + half) * BN + cpart * BNP;
        if (!w.owner) {
          float4* slot = reinterpret_cast<float4*>(p.sk_ws + (long long)blockIdx.x * BM * BN) + et;
#pragma unroll 1
          for (int c = 0; c < BNP; c += 32) {
            uint32_t r[32];
            tmem_ld32(t_part + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4)
              slot[(c / 4 + v4) * EPI_THREADS] =
                  make_float4(__uint_as_float(r[4 * v4]), __uint_as_float(r[4 * v4 + 1]),
                              __uint_as_float(r[4 * v4 + 2]), __uint_as_float(r[4 * v4 + 3]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
          __threadfence();
          named_bar_sync(1, EPI_THREADS);
          if (et == 0) st_release_gpu_s32(p.sk_flags + blockIdx.x, 1);
          if (++acc == NACC) {
            acc = 0;
            acc_phase ^= 1;
          }
          continue;
        }
        const int c_first = (int)blockIdx.x - w.ord;
        if (et == 0)
          for (int j = c_first; j < (int)blockIdx.x; ++j)
            if (!wait_flag_eq(p.sk_flags + j, 1, p.err)) break;
        named_bar_sync(1, EPI_THREADS);
#pragma unroll 1
        for (int c = 0; c < BNP; c += 32) {
          float4 y[8];
          {
            const float4* src = reinterpret_cast<const float4*>(p.sk_ws + (long long)c_first * BM * BN) + et;
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4) y[v4] = __ldcg(src + (c / 4 + v4) * EPI_THREADS);
          }
#pragma unroll 1
          for (int j = c_first + 1; j < (int)blockIdx.x; ++j) {
            const float4* src = reinterpret_cast<const float4*>(p.sk_ws + (long long)j * BM * BN) + et;
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4) {
              const float4 z = __ldcg(src + (c / 4 + v4) * EPI_THREADS);
              y[v4].x += z.x;
              y[v4].y += z.y;
              y[v4].z += z.z;
              y[v4].w += z.w;
            }
          }
          uint32_t r[32];
          tmem_ld32(t_part + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) {
            r[4 * v4] = __float_as_uint(__uint_as_float(r[4 * v4]) + y[v4].x);
            r[4 * v4 + 1] = __float_as_uint(__uint_as_float(r[4 * v4 + 1]) + y[v4].y);
            r[4 * v4 + 2] = __float_as_uint(__uint_as_float(r[4 * v4 + 2]) + y[v4].z);
            r[4 * v4 + 3] = __float_as_uint(__uint_as_float(r[4 * v4 + 3]) + y[v4].w);
          }
          tmem_st32(t_part + c, r);
        }
        tmem_wait_st();
        named_bar_sync(1, EPI_THREADS);  // every thread has read the slots
        if (et == 0)
          for (int j = c_first; j < (int)blockIdx.x; ++j) p.sk_flags[j] = 0;  // ready for the next launch
      }
      const bool no_k = tile_k(p, b, mb, 64).kblk == 0;  // nothing accumulated: the product is 0
      const int row = mb * BM + half * 128 + q * 32 + lane;
      const int n0 = nb * BN + cpart * BNP;
      const bool row_ok = row < p.M;
      using OutT = typename std::conditional<OUT_F32, float, __nv_bfloat16>::type;
      OutT* drow = reinterpret_cast<OutT*>(p.D) + (long long)b * p.strideD + (long long)row * p.ldd;
      const OutT* crow = p.C ? reinterpret_cast<const OutT*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc
                             : nullptr;
      const uint32_t t_acc = tmem_base + ((uint32_t)(q * 32) << 16) + (acc * MH + half) * BN + cpart * BNP;
      if (MH == 1 && !OUT_F32 && p.epi != 0) {
        // Fused epilogues (BM = 128 tiles only: their accumulator is double-buffered, so this work
        // overlaps the next tile's MMAs): chunks of the thread's accumulator row are drained into
        // packed bf16 registers, TMEM is released after the last chunk's reads, and the chunk's
        // outputs are computed and stored. Rounding to bf16 first matches what the separate
        // SwiGLU / RoPE kernels would read.
        constexpr int HALF = BN / 2;
        constexpr int PER = p_epi_per<BN, Cfg::CSPLIT>();  // output columns per thread (epi 2, 3)
        constexpr int PER1 = PER / 2;                      // (u, g) pairs per thread (epi 1)
        constexpr int CH = 128;                             // columns per chunk
        constexpr int CH1 = CH / 2;                        // pairs per chunk
        const int pos = (p.epi == 3) ? (p.rope_pos ? p.rope_pos[min(row, p.M - 1)] : row % p.rope_seq) : 0;
        const bool pos_ok = pos >= 0 && pos < p.rope_max;
        if (p.epi == 3 && row_ok && !pos_ok && lane == 0) set_error(p.err, kErrBadArg);
        const int n_chunks = (p.epi == 1 ? PER1 : PER) / (p.epi == 1 ? CH1 : CH);
#pragma unroll 1
        for (int ck = 0; ck < n_chunks; ++ck) {
          // packed bf16 values; epi 1 keeps u in pa[0, CH1 / 2) and g in pa[CH1 / 2, CH1)
          uint32_t pa[CH / 2];
          uint32_t* pb = pa + CH1 / 2;
          if (p.epi == 1) {
            const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (acc * MH + half) * BN + cpart * PER1 + ck * CH1;
#pragma unroll
            for (int part = 0; part < 2; ++part) {  // u columns, then g columns: one 32-column load live
#pragma unroll
              for (int c = 0; c < CH1; c += 32) {
                uint32_t r[32];
                tmem_ld32(tb + part * HALF + c, r);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e)
                  pa[part * (CH1 / 2) + c / 2 + e] =
                      pack_bf16(__uint_as_float(r[2 * e]) * p.alpha, __uint_as_float(r[2 * e + 1]) * p.alpha);
              }
            }
          } else {
#pragma unroll
            for (int c = 0; c < CH; c += 32) {
              uint32_t r[32];
              tmem_ld32(t_acc + ck * CH + c, r);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e)
                pa[c / 2 + e] = no_k ? 0u : pack_bf16(__uint_as_float(r[2 * e]) * p.alpha,
                                                      __uint_as_float(r[2 * e + 1]) * p.alpha);
            }
          }
          if (ck + 1 == n_chunks) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
          }
          if (!row_ok) continue;
          if (p.epi == 1) {
            // h = (u, g) and a = silu(g) * u for output columns j0 .. j0 + CH1
            const int j0 = nb * HALF + cpart * PER1 + ck * CH1;
            const bool store_h = p.D != nullptr;  // h = (u, g) is kept for the backward only
            __nv_bfloat16* hrow = reinterpret_cast<__nv_bfloat16*>(p.D) + (long long)row * p.ldd;
            __nv_bfloat16* arow = p.aux + (long long)row * p.ldaux;
#pragma unroll
            for (int g8 = 0; g8 < CH1; g8 += 8) {
              const int j = j0 + g8;
              uint32_t ha[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 ub = unpack_bf16(pa[g8 / 2 + e]), gb = unpack_bf16(pb[g8 / 2 + e]);
                ha[e] = pack_bf16(ub.x * gb.x * sigmoid_f(gb.x), ub.y * gb.y * sigmoid_f(gb.y));
              }
              if (j + 8 <= p.F && p.vec_ok) {
                if (store_h) {
                  *reinterpret_cast<uint4*>(hrow + j) =
                      make_uint4(pa[g8 / 2], pa[g8 / 2 + 1], pa[g8 / 2 + 2], pa[g8 / 2 + 3]);
                  *reinterpret_cast<uint4*>(hrow + p.F + j) =
                      make_uint4(pb[g8 / 2], pb[g8 / 2 + 1], pb[g8 / 2 + 2], pb[g8 / 2 + 3]);
                }
                *reinterpret_cast<uint4*>(arow + j) = make_uint4(ha[0], ha[1], ha[2], ha[3]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  if (j + e >= p.F) continue;
                  const int sh = (e & 1) * 16;
                  if (store_h) {
                    hrow[j + e] = __ushort_as_bfloat16((unsigned short)(pa[g8 / 2 + e / 2] >> sh));
                    hrow[p.F + j + e] = __ushort_as_bfloat16((unsigned short)(pb[g8 / 2 + e / 2] >> sh));
                  }
                  arow[j + e] = __ushort_as_bfloat16((unsigned short)(ha[e >> 1] >> sh));
                }
              }
            }
          } else if (p.epi == 2) {
            // dh = (da * silu(g), da * u * silu'(g)) with the saved h
            const __nv_bfloat16* hr = p.h + (long long)row * p.ldh;
            __nv_bfloat16* dh = p.aux + (long long)row * p.ldaux;
#pragma unroll
            for (int g8 = 0; g8 < CH; g8 += 8) {
              const int j = n0 + ck * CH + g8;
              if (j >= p.N) break;
              float u[8], gt[8];
              if (j + 8 <= p.N && p.vec_ok) {
                const uint4 uu = *reinterpret_cast<const uint4*>(hr + j);
                const uint4 gg = *reinterpret_cast<const uint4*>(hr + p.F + j);
                const uint32_t uw[4] = {uu.x, uu.y, uu.z, uu.w}, gw[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 a2 = unpack_bf16(uw[e]), b2 = unpack_bf16(gw[e]);
                  u[2 * e] = a2.x;
                  u[2 * e + 1] = a2.y;
                  gt[2 * e] = b2.x;
                  gt[2 * e + 1] = b2.y;
                }
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  u[e] = j + e < p.N ? __bfloat162float(hr[j + e]) : 0.f;
                  gt[e] = j + e < p.N ? __bfloat162float(hr[p.F + j + e]) : 0.f;
                }
              }
              uint32_t du[4], dg[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 d2 = unpack_bf16(pa[g8 / 2 + e]);
                const float s0 = sigmoid_f(gt[2 * e]), s1 = sigmoid_f(gt[2 * e + 1]);
                du[e] = pack_bf16(d2.x * gt[2 * e] * s0, d2.y * gt[2 * e + 1] * s1);
                dg[e] = pack_bf16(d2.x * u[2 * e] * s0 * (1.f + gt[2 * e] * (1.f - s0)),
                                  d2.y * u[2 * e + 1] * s1 * (1.f + gt[2 * e + 1] * (1.f - s1)));
              }
              if (j + 8 <= p.N && p.vec_ok) {
                *reinterpret_cast<uint4*>(dh + j) = make_uint4(du[0], du[1], du[2], du[3]);
                *reinterpret_cast<uint4*>(dh + p.F + j) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  if (j + e >= p.N) continue;
                  const int sh = (e & 1) * 16;
                  dh[j + e] = __ushort_as_bfloat16((unsigned short)(du[e >> 1] >> sh));
                  dh[p.F + j + e] = __ushort_as_bfloat16((unsigned short)(dg[e >> 1] >> sh));
                }
              }
            }
          } else {
            // epi 3: RoPE on the bf16-rounded values (as the separate in-place kernel does)
            __nv_bfloat16* dr = reinterpret_cast<__nv_bfloat16*>(p.D) + (long long)row * p.ldd;
            const int jb = n0 + ck * CH;
#pragma unroll
            for (int e = 0; e < CH / 2; ++e) {
              const int j = jb + 2 * e;
              if (pos_ok && j < p.rope_cols) {
                const float2 x = unpack_bf16(pa[e]);
                const float2 cs = p.rope_cs[(long long)pos * (p.rope_hd / 2) + (j % p.rope_hd) / 2];
                pa[e] = pack_bf16(x.x * cs.x - x.y * cs.y, x.x * cs.y + x.y * cs.x);
              }
            }
#pragma unroll
            for (int g8 = 0; g8 < CH; g8 += 8) {
              const int j = jb + g8;
              if (j + 8 <= p.N && p.vec_ok) {
                *reinterpret_cast<uint4*>(dr + j) =
                    make_uint4(pa[g8 / 2], pa[g8 / 2 + 1], pa[g8 / 2 + 2], pa[g8 / 2 + 3]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (j + e < p.N)
                    dr[j + e] = __ushort_as_bfloat16((unsigned short)(pa[g8 / 2 + e / 2] >> ((e & 1) * 16)));
              }
            }
          }
        }
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if (MH == 2 && !OUT_F32 && (crow == nullptr || p.beta == 0.f)) {
        // BM = 256 (one accumulator buffer) without a C operand: drain the whole
        // accumulator row slice into packed bf16 registers, release TMEM, then
        // store, so the next tile's MMAs wait only for the TMEM reads.
        uint32_t pk[MH == 2 ? BNP / 2 : 1];
#pragma unroll
        for (int c = 0; c < BNP; c += 32) {
          uint32_t r[32];
          tmem_ld32(t_acc + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[c / 2 + i] = no_k ? 0u
                                 : pack_bf16(__uint_as_float(r[2 * i]) * p.alpha,
                                             __uint_as_float(r[2 * i + 1]) * p.alpha);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        if (row_ok) {
          __nv_bfloat16* dr = reinterpret_cast<__nv_bfloat16*>(drow);
#pragma unroll
          for (int c = 0; c < BNP; c += 8) {
            const int col = n0 + c;
            if (col + 8 <= p.N && p.vec_ok) {
              *reinterpret_cast<uint4*>(dr + col) =
                  make_uint4(pk[c / 2], pk[c / 2 + 1], pk[c / 2 + 2], pk[c / 2 + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                if (col + i < p.N) {
                  const uint32_t w = pk[(c + i) / 2];
                  const unsigned short h = (i & 1) ? (unsigned short)(w >> 16) : (unsigned short)(w & 0xffffu);
                  dr[col + i] = __ushort_as_bfloat16(h);
                }
              }
            }
          }
        }
        if (p.npeers > 0) {
          named_bar_sync(1, EPI_THREADS);  // the whole tile is in the local D
          if (p.scatter_rpo > 0)
            scatter_copy_tile<BM, BN>(p, mb, nb, et, EPI_THREADS);
          else
            gather_copy_tile<BM, BN>(p, b, mb, nb, et, EPI_THREADS);
        }
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      // chunks of SUBS x 32 columns (one sub-chunk when the register budget is
      // that of the 576-thread BM = 256 kernel)
      constexpr int SUBS = MH == 2 ? 1 : 2;
#pragma unroll 1
      for (int c = 0; c < BNP; c += 32 * SUBS) {
        uint32_t r2[32 * SUBS];
#pragma unroll
        for (int sub = 0; sub < SUBS; ++sub)
          tmem_ld32(t_acc + c + sub * 32, *reinterpret_cast<uint32_t(*)[32]>(&r2[sub * 32]));
        tmem_wait_ld();
        if (c + 32 * SUBS >= BNP) {
          // last chunk read: release the accumulator before the global stores
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
#pragma unroll
        for (int sub = 0; sub < SUBS; ++sub) {
          const uint32_t* r = &r2[sub * 32];
          const int col = n0 + c + sub * 32;
          if (!row_ok || col >= p.N) continue;
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = no_k ? 0.f : __uint_as_float(r[i]) * p.alpha;
          const bool full_chunk = (col + 32 <= p.N) && p.vec_ok;
          if (full_chunk) {
            if (crow && p.beta != 0.f) {
              if (OUT_F32) {
                const float4* src = reinterpret_cast<const float4*>(crow + col);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  float4 t = src[i];
                  v[4 * i] += p.beta * t.x;
                  v[4 * i + 1] += p.beta * t.y;
                  v[4 * i + 2] += p.beta * t.z;
                  v[4 * i + 3] += p.beta * t.w;
                }
              } else {
                const uint4* src = reinterpret_cast<const uint4*>(crow + col);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  uint4 t = src[i];
                  uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    float2 f = unpack_bf16(w[j]);
                    v[8 * i + 2 * j] += p.beta * f.x;
                    v[8 * i + 2 * j + 1] += p.beta * f.y;
                  }
                }
              }
            }
            if (OUT_F32) {
              float4* dst = reinterpret_cast<float4*>(drow + col);
#pragma unroll
              for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(drow + col);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_uint4(pack_bf16(v[8 * i], v[8 * i + 1]), pack_bf16(v[8 * i + 2], v[8 * i + 3]),
                                    pack_bf16(v[8 * i + 4], v[8 * i + 5]), pack_bf16(v[8 * i + 6], v[8 * i + 7]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (col + i < p.N) {
                float x = v[i];
                if (crow && p.beta != 0.f) x += p.beta * to_f(crow[col + i]);
                if (OUT_F32)
                  reinterpret_cast<float*>(drow)[col + i] = x;
                else
                  reinterpret_cast<__nv_bfloat16*>(drow)[col + i] = __float2bfloat16_rn(x);
              }
            }
          }
        }
      }
      if (!OUT_F32 && p.npeers > 0) {
        named_bar_sync(1, EPI_THREADS);  // the whole tile is in the local D
        if (p.scatter_rpo > 0)
          scatter_copy_tile<BM, BN>(p, mb, nb, et, EPI_THREADS);
        else
          gather_copy_tile<BM, BN>(p, b, mb, nb, et, EPI_THREADS);
      }
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  if (p.npeers > 0) __threadfence_system();  // this thread's peer stores, before the grid count
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS < 32 ? 32 : Cfg::TMEM_COLS);
  }
  if (p.npeers > 0 && threadIdx.x == 0 && atomicAdd(p.gather_done, 1u) == gridDim.x - 1) {
    // last CTA: every CTA's stores are fenced; tell every peer that this rank's block has landed
    __threadfence_system();
#pragma unroll
    for (int q = 0; q < kMaxGatherPeers; ++q)
      if (q < p.npeers) {
        unsigned* f = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(p.gather_flag) + p.peer_delta[q]);
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(p.gather_epoch) : "memory");
      }
    *p.gather_done = 0u;
  }
}


// ---------------------------------------------------------------------------------------------
// CTA-pair GEMM (plain and batched modes): a cluster of two CTAs on two SMs computes one 256 x 256
// output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16 per instruction), issued by
// one thread of the even CTA. Each CTA stages its own 128 rows of A and 128 of the tile's 256 B
// rows (N), so the smem bytes per FLOP of each SM equal those of the single-CTA 256 x 256 tile,
// but each CTA's accumulator (its 128 rows x 256 columns) takes only 256 TMEM columns: two fit,
// and the epilogue of tile t overlaps the MMAs of tile t+1 (the single-CTA 256 x 256 tile fills
// TMEM, so its MMAs stall while the epilogue drains). Each CTA's stage is 32 KB: a 6-deep ring.
// (A 256 x 128 pair tile moves 1.5x the operand bytes per FLOP and measured 0.5 - 0.75x the speed of
// 256 x 256 on every training shape, so it is not instantiated. 256 x 192 tiles, 1.17x the bytes
// per FLOP, are instantiated for a K-major B and picked by pair_tile_n where their waves finish
// sooner: wave quantisation of 256-wide tiles costs more on those shapes.)
//
//   warp 0     TMA producer (both CTAs): loads into its own smem, completion counted on the
//              even CTA's `full` barrier (cta_group::2 form of the tiled load, no multicast)
//   warp 1     TMEM allocation for the pair (both CTAs); MMA issuer (even CTA only): commits
//              release the stage in both CTAs and publish an accumulator to both epilogues
//              (tcgen05.commit ... multicast::cluster, mask 0b11)
//   warps 2-9  epilogue: two warps per TMEM lane quadrant, BN / 2 columns each; they drain this
//              CTA's accumulator and arrive on the even CTA's acc_empty barrier
// All waits are time-bounded (common.cuh); both CTAs meet at a cluster barrier before the TMEM
// is freed, so neither leaves while the other can still signal its barriers.
template <int BN_>
struct PairCfg {
  static constexpr int BN = BN_;                 // output columns of a pair tile (256, 192 or 128)
  static constexpr int BK = 64;
  static constexpr int A_BYTES = 128 * BK * 2;   // this CTA's 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's BN / 2 of the tile's B rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;  // 6 for BN 256
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int TMEM_COLS = 2 * BN;       // two accumulators
  // tcgen05.alloc takes a power of two of at least 32 columns
  static constexpr int TMEM_ALLOC = TMEM_COLS <= 32 ? 32 : TMEM_COLS <= 64 ? 64 : TMEM_COLS <= 128 ? 128
                                    : TMEM_COLS <= 256 ? 256 : 512;
  static_assert(BN == 256 || BN == 192 || BN == 128, "pair tiles are 256 x 256, 256 x 192 or 256 x 128");
  static_assert(TMEM_COLS <= 512, "accumulators exceed tensor memory");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// shared::cluster address of the same smem offset in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// tiled 3-D load into this CTA's smem whose completion is counted on `bar_cluster`, a barrier of
// either CTA of the pair
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (same smem offset) in both CTAs once this thread's MMAs are done
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

template <int BN, int A_MN, int B_MN, int OUT_F32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<BN>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = PairCfg<BN>;
  constexpr int BK = Cfg::BK, A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES, STAGE_BYTES = Cfg::STAGE_BYTES;
  constexpr int STAGES = Cfg::STAGES, EPI_WARPS = Cfg::EPI_WARPS, TMEM_ALLOC = Cfg::TMEM_ALLOC;
  // 256 x 192 tiles: K-major B only (an MN-major B stage is loaded in whole 64-column boxes)
  static_assert(BN != 192 || !B_MN, "256 x 192 pair tiles take a K-major B");
  constexpr int BNH = BN / 2;  // B rows per CTA; output columns per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();  // 0: MMA issuer of the pair
  const int pair_id = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  pdl_trigger();  // as in gemm_kernel: global memory is read only after pdl_wait below

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * EPI_WARPS);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_ALLOC)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  const int num_tiles = gemm_num_tiles(p);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      WorkIter wi;
      wi.init(p, pair_id, npairs);
      WorkItem w;
      while (ok && wi.next(p, num_tiles, p.k_blocks, w)) {
        int b, mb, nb;
        gemm_tile(p, w.tile, b, mb, nb);
        const int m0 = mb * 256 + (int)rank * 128;
        // epi 1 (SwiGLU forward): the even CTA stages up rows, the odd one the gate rows of the same
        // BNH output columns, so each accumulator holds u in columns [0, BNH) and g in [BNH, BN)
        const int n0 = p.epi == 1 ? nb * BNH + (int)rank * p.F : nb * BN + (int)rank * BNH;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * STAGE_BYTES);
          const uint32_t bar = mapa_shared(&full[stage], 0);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if (A_MN) {
            tma_load_3d_pair(a_dst, &tmA, bar, m0, k0, b);
            tma_load_3d_pair(a_dst + 8192, &tmA, bar, m0 + 64, k0, b);
          } else {
            tma_load_3d_pair(a_dst, &tmA, bar, k0, m0, b);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BNH / 64; ++c) tma_load_3d_pair(b_dst + c * 8192, &tmB, bar, n0 + c * 64, k0, b);
          } else {
            tma_load_3d_pair(b_dst, &tmB, bar, k0, n0, b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------- MMA issuer (even CTA)
      constexpr uint32_t idesc = idesc_bf16(256, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      WorkIter wi;
      wi.init(p, pair_id, npairs);
      WorkItem w;
      while (ok && wi.next(p, num_tiles, p.k_blocks, w)) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, p.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_base + k * 2048, 8192, 1024) : sdesc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_base + k * 2048, 8192, 1024) : sdesc_sw128(b_base + k * 32, 16, 1024);
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb != w.kb0) || k != 0);
          }
          umma_commit_pair(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;              // TMEM lane quadrant this warp may access
    const int cpart = (warp - 2) >> 2;   // column half: [cpart * BNH, (cpart + 1) * BNH)
    const uint32_t empty_bar0 = mapa_shared(&acc_empty[0], 0);
    const uint32_t empty_bar1 = mapa_shared(&acc_empty[1], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    using OutT = typename std::conditional<OUT_F32, float, __nv_bfloat16>::type;
    const bool use_c = p.C != nullptr && p.beta != 0.f;
    constexpr int EPI_THREADS = EPI_WARPS * 32;
    const int et = threadIdx.x - 64;  // epilogue thread index
    WorkIter wi;
    wi.init(p, pair_id, npairs);
    WorkItem w;
    while (wi.next(p, num_tiles, p.k_blocks, w)) {
      int b, mb, nb;
      gemm_tile(p, w.tile, b, mb, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, p.err, kErrWaitAccFull)) break;
      tc_fence_after();
      if (w.partial) {
        // Stream-K part (see GemmParams): per CTA, as in the single-CTA kernel. A non-owner parks this
        // CTA's 128 x BN fp32 partial in its own slot (thread-major float4s) and raises its flag; the
        // owner waits for the same-rank CTAs of the lower pairs holding the tile's other parts and
        // adds their slots into its accumulator before the regular epilogue below.
        const uint32_t t_part = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cpart * BNH;
        if (!w.owner) {
          float4* slot = reinterpret_cast<float4*>(p.sk_ws + (long long)blockIdx.x * 128 * BN) + et;
#pragma unroll 1
          for (int c = 0; c < BNH; c += 32) {
            uint32_t r[32];
            tmem_ld32(t_part + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4)
              slot[(c / 4 + v4) * EPI_THREADS] =
                  make_float4(__uint_as_float(r[4 * v4]), __uint_as_float(r[4 * v4 + 1]),
                              __uint_as_float(r[4 * v4 + 2]), __uint_as_float(r[4 * v4 + 3]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc ? empty_bar1 : empty_bar0);
          __threadfence();
          named_bar_sync(1, EPI_THREADS);
          if (et == 0) st_release_gpu_s32(p.sk_flags + blockIdx.x, 1);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
          continue;
        }
        const int first = pair_id - w.ord;  // lowest pair holding a part of this tile
        if (et == 0)
          for (int j = first; j < pair_id; ++j)
            if (!wait_flag_eq(p.sk_flags + 2 * j + (int)rank, 1, p.err)) break;
        named_bar_sync(1, EPI_THREADS);
#pragma unroll 1
        for (int c = 0; c < BNH; c += 32) {
          float4 y[8];
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) y[v4] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
          for (int j = first; j < pair_id; ++j) {
            const float4* src =
                reinterpret_cast<const float4*>(p.sk_ws + (long long)(2 * j + (int)rank) * 128 * BN) + et;
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4) {
              const float4 z = __ldcg(src + (c / 4 + v4) * EPI_THREADS);
              y[v4].x += z.x;
              y[v4].y += z.y;
              y[v4].z += z.z;
              y[v4].w += z.w;
            }
          }
          uint32_t r[32];
          tmem_ld32(t_part + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) {
            r[4 * v4] = __float_as_uint(__uint_as_float(r[4 * v4]) + y[v4].x);
            r[4 * v4 + 1] = __float_as_uint(__uint_as_float(r[4 * v4 + 1]) + y[v4].y);
            r[4 * v4 + 2] = __float_as_uint(__uint_as_float(r[4 * v4 + 2]) + y[v4].z);
            r[4 * v4 + 3] = __float_as_uint(__uint_as_float(r[4 * v4 + 3]) + y[v4].w);
          }
          tmem_st32(t_part + c, r);
        }
        tmem_wait_st();
        named_bar_sync(1, EPI_THREADS);  // every thread has read the slots
        if (et == 0)
          for (int j = first; j < pair_id; ++j) p.sk_flags[2 * j + (int)rank] = 0;  // ready for the next launch
      }
      const int row = mb * 256 + (int)rank * 128 + q * 32 + lane;
      const int n0 = nb * BN + cpart * BNH;
      const bool row_ok = row < p.M;
      // epi 3 (RoPE in the QKV projection): this row's position, read once per tile
      int rope_p = 0;
      bool rope_ok = false;
      if (p.epi == 3) {
        rope_p = p.rope_pos ? p.rope_pos[min(row, p.M - 1)] : row % p.rope_seq;
        rope_ok = rope_p >= 0 && rope_p < p.rope_max;
        if (row_ok && !rope_ok) set_error(p.err, kErrBadArg);
      }
      OutT* drow = reinterpret_cast<OutT*>(p.D) + (long long)b * p.strideD + (long long)row * p.ldd;
      const OutT* crow =
          use_c ? reinterpret_cast<const OutT*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc : nullptr;
      if (p.epi == 1) {
        // SwiGLU forward: h = (u, g) and a = silu(g) * u for output columns j0 .. j0 + BNH / 2, 32
        // columns at a time straight from TMEM (only one chunk's u and g live in registers; the
        // accumulator is handed back after the last chunk's loads, as in the plain epilogue)
        constexpr int PER = BNH / 2;
        const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
        const int j0 = nb * BNH + cpart * PER;
        const bool store_h = p.D != nullptr;  // h = (u, g) is kept for the backward only
        __nv_bfloat16* hrow = reinterpret_cast<__nv_bfloat16*>(p.D) + (long long)row * p.ldd;
        __nv_bfloat16* arow = p.aux + (long long)row * p.ldaux;
#pragma unroll 1
        for (int c = 0; c < PER; c += 32) {
          uint32_t ru[32], rg[32];
          tmem_ld32(t_row + cpart * PER + c, ru);
          tmem_ld32(t_row + BNH + cpart * PER + c, rg);
          tmem_wait_ld();
          if (c + 32 >= PER) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? empty_bar1 : empty_bar0);
          }
          if (!row_ok) continue;
#pragma unroll
          for (int g8 = 0; g8 < 32; g8 += 8) {
            const int j = j0 + c + g8;
            uint32_t pu[4], pg[4], ha[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // rounded to bf16 first: the values the separate SwiGLU kernel would read from h
              pu[e] = pack_bf16(__uint_as_float(ru[g8 + 2 * e]), __uint_as_float(ru[g8 + 2 * e + 1]));
              pg[e] = pack_bf16(__uint_as_float(rg[g8 + 2 * e]), __uint_as_float(rg[g8 + 2 * e + 1]));
              const float2 ub = unpack_bf16(pu[e]), gb = unpack_bf16(pg[e]);
              ha[e] = pack_bf16(ub.x * gb.x * sigmoid_f(gb.x), ub.y * gb.y * sigmoid_f(gb.y));
            }
            if (j + 8 <= p.F && p.vec_ok) {
              if (store_h) {
                *reinterpret_cast<uint4*>(hrow + j) = make_uint4(pu[0], pu[1], pu[2], pu[3]);
                *reinterpret_cast<uint4*>(hrow + p.F + j) = make_uint4(pg[0], pg[1], pg[2], pg[3]);
              }
              *reinterpret_cast<uint4*>(arow + j) = make_uint4(ha[0], ha[1], ha[2], ha[3]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (j + e >= p.F) continue;
                const int sh = (e & 1) * 16;
                if (store_h) {
                  hrow[j + e] = __ushort_as_bfloat16((unsigned short)(pu[e >> 1] >> sh));
                  hrow[p.F + j + e] = __ushort_as_bfloat16((unsigned short)(pg[e >> 1] >> sh));
                }
                arow[j + e] = __ushort_as_bfloat16((unsigned short)(ha[e >> 1] >> sh));
              }
            }
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      const uint32_t t_acc = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cpart * BNH;
#pragma unroll 1
      for (int c = 0; c < BNH; c += 32) {
        uint32_t r[32];
        tmem_ld32(t_acc + c, r);
        tmem_wait_ld();
        if (c + 32 >= BNH) {
          // last chunk read: hand the accumulator back before the global stores
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc ? empty_bar1 : empty_bar0);
        }
        const int col = n0 + c;
        if (!row_ok || col >= p.N) continue;
        if (p.epi == 2) {
          // SwiGLU backward: da (rounded to bf16, as stored by the unfused path) never leaves TMEM;
          // dh = (da * silu(g), da * u * silu'(g)) with the saved h = (u, g)
          const __nv_bfloat16* hr = p.h + (long long)row * p.ldh;
          __nv_bfloat16* dh = p.aux + (long long)row * p.ldaux;
#pragma unroll
          for (int g8 = 0; g8 < 32; g8 += 8) {
            const int j = col + g8;
            if (j >= p.N) break;
            float u[8], gt[8];
            if (j + 8 <= p.N && p.vec_ok) {
              const uint4 uu = *reinterpret_cast<const uint4*>(hr + j);
              const uint4 gg = *reinterpret_cast<const uint4*>(hr + p.F + j);
              const uint32_t uw[4] = {uu.x, uu.y, uu.z, uu.w}, gw[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 a2 = unpack_bf16(uw[e]), b2 = unpack_bf16(gw[e]);
                u[2 * e] = a2.x;
                u[2 * e + 1] = a2.y;
                gt[2 * e] = b2.x;
                gt[2 * e + 1] = b2.y;
              }
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                u[e] = j + e < p.N ? __bfloat162float(hr[j + e]) : 0.f;
                gt[e] = j + e < p.N ? __bfloat162float(hr[p.F + j + e]) : 0.f;
              }
            }
            uint32_t du[4], dg[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 d2 = unpack_bf16(pack_bf16(__uint_as_float(r[g8 + 2 * e]), __uint_as_float(r[g8 + 2 * e + 1])));
              const float s0 = sigmoid_f(gt[2 * e]), s1 = sigmoid_f(gt[2 * e + 1]);
              du[e] = pack_bf16(d2.x * gt[2 * e] * s0, d2.y * gt[2 * e + 1] * s1);
              dg[e] = pack_bf16(d2.x * u[2 * e] * s0 * (1.f + gt[2 * e] * (1.f - s0)),
                                d2.y * u[2 * e + 1] * s1 * (1.f + gt[2 * e + 1] * (1.f - s1)));
            }
            if (j + 8 <= p.N && p.vec_ok) {
              *reinterpret_cast<uint4*>(dh + j) = make_uint4(du[0], du[1], du[2], du[3]);
              *reinterpret_cast<uint4*>(dh + p.F + j) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (j + e >= p.N) continue;
                const int sh = (e & 1) * 16;
                dh[j + e] = __ushort_as_bfloat16((unsigned short)(du[e >> 1] >> sh));
                dh[p.F + j + e] = __ushort_as_bfloat16((unsigned short)(dg[e >> 1] >> sh));
              }
            }
          }
          continue;
        }
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
        if (p.epi == 3 && rope_ok && col < p.rope_cols) {
          // RoPE of interleaved pairs on the bf16-rounded values (what the separate in-place kernel
          // reads); the 32 columns lie in one head (head_dim and rope_cols are multiples of 32), so
          // their 16 (cos, sin) pairs are contiguous in the table: eight 16-byte loads
          const float4* tcs = reinterpret_cast<const float4*>(p.rope_cs + (long long)rope_p * (p.rope_hd / 2) +
                                                              (col % p.rope_hd) / 2);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 c2 = tcs[q4];
            const float x0 = __bfloat162float(__float2bfloat16_rn(v[4 * q4])),
                        y0 = __bfloat162float(__float2bfloat16_rn(v[4 * q4 + 1])),
                        x1 = __bfloat162float(__float2bfloat16_rn(v[4 * q4 + 2])),
                        y1 = __bfloat162float(__float2bfloat16_rn(v[4 * q4 + 3]));
            v[4 * q4] = x0 * c2.x - y0 * c2.y;
            v[4 * q4 + 1] = x0 * c2.y + y0 * c2.x;
            v[4 * q4 + 2] = x1 * c2.z - y1 * c2.w;
            v[4 * q4 + 3] = x1 * c2.w + y1 * c2.z;
          }
        }
        if (col + 32 <= p.N && p.vec_ok) {
          if (crow) {
            if (OUT_F32) {
              const float4* src = reinterpret_cast<const float4*>(crow + col);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 t = src[i];
                v[4 * i] += p.beta * t.x;
                v[4 * i + 1] += p.beta * t.y;
                v[4 * i + 2] += p.beta * t.z;
                v[4 * i + 3] += p.beta * t.w;
              }
            } else {
              const uint4* src = reinterpret_cast<const uint4*>(crow + col);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 t = src[i];
                const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 f = unpack_bf16(w[j]);
                  v[8 * i + 2 * j] += p.beta * f.x;
                  v[8 * i + 2 * j + 1] += p.beta * f.y;
                }
              }
            }
          }
          if (OUT_F32) {
            float4* dst = reinterpret_cast<float4*>(drow + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(drow + col);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(pack_bf16(v[8 * i], v[8 * i + 1]), pack_bf16(v[8 * i + 2], v[8 * i + 3]),
                                  pack_bf16(v[8 * i + 4], v[8 * i + 5]), pack_bf16(v[8 * i + 6], v[8 * i + 7]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (col + i < p.N) {
              float x = v[i];
              if (crow) x += p.beta * to_f(crow[col + i]);
              if (OUT_F32)
                reinterpret_cast<float*>(drow)[col + i] = x;
              else
                reinterpret_cast<__nv_bfloat16*>(drow)[col + i] = __float2bfloat16_rn(x);
            }
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair is done with each other's barriers and tensor memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_ALLOC)
                 : "memory");
  }
}

}  // namespace astrai

namespace astrai_host {

using astrai::GemmCfg;
using astrai::GemmParams;

// When set (gemm_profile_set), every GEMM launch adds its wait cycles to these 4 counters.
static unsigned long long* g_gemm_prof = nullptr;
void gemm_profile_set(unsigned long long* counters) { g_gemm_prof = counters; }

// Programmatic dependent launch of the GEMM kernels (they wait for the previous grid after their
// prologue: barrier init, TMEM allocation, tensor-map prefetch). Not used for the fused all-gather /
// reduce-scatter launches, whose peer traffic then starts strictly after the previous kernel.
// ASTRAI_GEMM_PDL=0 turns it off.
static bool gemm_pdl() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_GEMM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}
template <typename Kern>
static void launch_gemm_ex(Kern kern, int grid, int threads, int smem, cudaStream_t stream, bool pdl,
                           const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  astrai::note_launch();
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("astrai gemm: launch failed: ") + cudaGetErrorString(e));
}

template <int BM, int BN, int A_MN, int B_MN, int OUT_F32>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
                        cudaStream_t stream) {
  auto kern = astrai::gemm_kernel<BM, BN, A_MN, B_MN, OUT_F32>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BM, BN>::SMEM);
    attr_set[dev & 63] = true;
  }
  const bool pdl = gemm_pdl() && p.npeers == 0 && p.scatter_rpo == 0;
  launch_gemm_ex(kern, grid, GemmCfg<BM, BN>::THREADS, GemmCfg<BM, BN>::SMEM, stream, pdl, ta, tb, p);
}

template <int BM, int BN>
static void dispatch_majors(int a_mn, int b_mn, int out_f32, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmParams& p, int grid, cudaStream_t s) {
#define ASTRAI_GEMM_CASE(AM, BMJ, OF) \
  if (a_mn == AM && b_mn == BMJ && out_f32 == OF) return launch_gemm<BM, BN, AM, BMJ, OF>(ta, tb, p, grid, s);
  ASTRAI_GEMM_CASE(0, 0, 0)
  ASTRAI_GEMM_CASE(0, 1, 0)
  ASTRAI_GEMM_CASE(1, 0, 0)
  ASTRAI_GEMM_CASE(1, 1, 0)
  ASTRAI_GEMM_CASE(0, 0, 1)
  ASTRAI_GEMM_CASE(0, 1, 1)
  ASTRAI_GEMM_CASE(1, 0, 1)
  ASTRAI_GEMM_CASE(1, 1, 1)
#undef ASTRAI_GEMM_CASE
}

// Clusters of two that can be resident at once on this device (queried once per device; every
// instantiation of the pair kernel has the same footprint: one CTA per SM by its shared memory).
static int pair_clusters(int dev) {
  static int max_clusters[64] = {0};
  if (max_clusters[dev & 63] == 0) {
    using pr = astrai::PairCfg<256>;
    auto kern = astrai::gemm_pair_kernel<256, 0, 0, 0>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pr::SMEM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms(dev) & ~1);
    cfg.blockDim = dim3(pr::THREADS);
    cfg.dynamicSmemBytes = pr::SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = num_sms(dev) / 2;
    }
    max_clusters[dev & 63] = n;
  }
  return max_clusters[dev & 63];
}

// CTA-pair kernel launch on `pairs` clusters of two (persistent; at most pair_clusters(dev)).
template <int BN, int A_MN, int B_MN, int OUT_F32>
static void launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int pairs,
                             cudaStream_t stream) {
  using pr = astrai::PairCfg<BN>;
  auto kern = astrai::gemm_pair_kernel<BN, A_MN, B_MN, OUT_F32>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pr::SMEM);
    attr_set[dev & 63] = true;
  }
  launch_gemm_ex(kern, 2 * pairs, pr::THREADS, pr::SMEM, stream, gemm_pdl(), ta, tb, p);
}

template <int BN>
static void dispatch_pair(int a_mn, int b_mn, int out_f32, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmParams& p, int pairs, cudaStream_t s) {
#define ASTRAI_PAIR_CASE(AM, BMJ, OF) \
  if (a_mn == AM && b_mn == BMJ && out_f32 == OF) return launch_gemm_pair<BN, AM, BMJ, OF>(ta, tb, p, pairs, s);
  ASTRAI_PAIR_CASE(0, 0, 0)
  ASTRAI_PAIR_CASE(0, 1, 0)
  ASTRAI_PAIR_CASE(1, 0, 0)
  ASTRAI_PAIR_CASE(1, 1, 0)
  ASTRAI_PAIR_CASE(0, 0, 1)
  ASTRAI_PAIR_CASE(0, 1, 1)
  ASTRAI_PAIR_CASE(1, 0, 1)
  ASTRAI_PAIR_CASE(1, 1, 1)
#undef ASTRAI_PAIR_CASE
}

// 256 x 192 pair tiles (K-major B only): A K- or MN-major, bf16 or fp32 output.
static void dispatch_pair192(int a_mn, int out_f32, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                             int pairs, cudaStream_t s) {
  if (a_mn == 0 && out_f32 == 0) return launch_gemm_pair<192, 0, 0, 0>(ta, tb, p, pairs, s);
  if (a_mn == 1 && out_f32 == 0) return launch_gemm_pair<192, 1, 0, 0>(ta, tb, p, pairs, s);
  if (a_mn == 0 && out_f32 == 1) return launch_gemm_pair<192, 0, 0, 1>(ta, tb, p, pairs, s);
  return launch_gemm_pair<192, 1, 0, 1>(ta, tb, p, pairs, s);
}

// Pair tile width for a GEMM with a K-major B: 192 where its waves of 256 x 192 tiles finish sooner
// than the waves of 256 x 256 tiles by at least 3 %, else 256. A 192-wide wave does 0.75 of the
// work but measured 0.88 of the time at 32 k-blocks (8192 x 3072 x 2048: 7 waves 80.7 us against 6
// waves 77.8 us) and 0.76 at 88 (8192 x 2048 x 5632: 154.1 against 161.4 us; L2 flushed), so the
// wave cost is 0.88 below 64 k-blocks and 0.76 from there. One-wave grids (a 2048-token prefill's
// 2048 x 1536 projections) always take the smaller tile: 21.0 / 45.2 against 22.7 / 49.2 us.
static int pair_tile_n(int M, int N, int K, int batch, int pairs) {
  if (N <= 192 || pairs <= 0) return 256;
  const long long tm = (long long)((M + 255) / 256) * batch;
  const long long t256 = tm * ((N + 255) / 256), t192 = tm * ((N + 191) / 192);
  const double w192 = (K + 63) / 64 >= 64 ? 0.76 : 0.88;
  const double c256 = (double)((t256 + pairs - 1) / pairs), c192 = w192 * (double)((t192 + pairs - 1) / pairs);
  return c192 < 0.97 * c256 ? 192 : 256;
}

// CTA-pair policy: plain and batched GEMMs with M > 128 and N > 128 run on the pair kernel.
// Measured on B200 over the 1.1B step's GEMMs (kernel_bench gemm, CUDA events), the pair kernel
// was faster than the single-CTA kernel on every shape: 8192x3072x2048 1345 vs 1158 TFLOP/s,
// 8192x32000x2048 1508 vs 1319, 8192x5632x2048 (MN-major B) 1135 vs 910, 2048x2048x8192 (both
// MN-major; single-CTA 128x256) 1366 vs 1063, 11264x2048x8192 1449 vs 1430 (single-CTA with
// Stream-K), 8192^3 equal. ASTRAI_GEMM_PAIR=0 keeps the single-CTA kernel.
static bool pair_on() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Stream-K decision: whole waves of tiles plus the last partial wave split into k-block units over
// all CTAs (see GemmParams). Measured on B200 over the 1.1B step's GEMMs, the split paid off on
// every shape with long K (>= 128 k-blocks: weight gradients over 8192 tokens, K = 32000) and at
// least half a wave of tiles (0.26 vs 0.33 ms for 11264x2048x8192, 0.69 vs 0.73 ms for
// 8192x2048x32000), and lost 5 - 20 us on shorter K (2048 - 5632) and on grids of fewer than half
// the SMs, where the unsplit tiles run faster per CTA for want of contention. So it is used only
// there, and only when every CTA gets at least 4 k-blocks and the split saves at least 16 k-blocks
// of time. ASTRAI_STREAMK=0 disables it.
static bool streamk_on() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_STREAMK");
    return !(e && e[0] == '0');
  }();
  return on;
}
static bool use_streamk(long long tiles, int kb, int sms) {
  if (!streamk_on() || tiles <= 0 || sms <= 0) return false;
  const long long rem = tiles % sms;
  if (kb < 128 || 2 * tiles < sms) return false;
  if (rem == 0 || rem * kb < 4LL * sms) return false;
  const double dp = (double)(tiles / sms + 1), sk = (double)tiles / sms + 0.08;
  return (dp - sk) * kb >= 16.0;
}
// Stream-K for the pair kernel over `pairs` workers: the last partial wave of 256 x 256 tiles can
// be split when every pair gets at least 4 k-blocks of it and the split would save at least 8
// k-blocks of time per pair. Measured on B200 it LOST on every step shape it applies to (8192 x
// 3072 x 2048: 0.0847 vs 0.0768 ms unsplit; 8192 x 2048 x 2048: 0.0585 vs 0.0513; 11264 x 2048 x
// 8192: 0.2848 vs 0.2663): the fix-up tail (partials out, flags, partials in, then the epilogue)
// is exposed at the end of the launch. So it is opt-in (ASTRAI_PAIR_STREAMK=1, or force_bn 1026).
static bool pair_streamk_on() {
  static const bool on = [] {
    const char* e = std::getenv("ASTRAI_PAIR_STREAMK");
    return e && e[0] == '1';
  }();
  return on;
}
static bool use_streamk_pair(long long tiles, int kb, int pairs) {
  if (tiles <= 0 || pairs <= 0) return false;
  const long long rem = tiles % pairs;
  if (rem == 0 || tiles < pairs || rem * kb < 4LL * pairs) return false;
  const double whole = (double)(tiles / pairs + 1), split = (double)tiles / pairs + 0.05;
  return (whole - split) * kb >= 8.0;
}
// Automatic k-block split of the pair kernel (0 none, 1 the last partial wave, 2 every k-block of
// every tile over all pairs). Measured on B200 (L2 flushed, `kernel_bench gemm_shapes`), the fix-up
// (partials out, flags, partials in) costs 10 - 20 us, so a split pays only where it saves many
// k-blocks per pair:
//   3072 x 2048 x 8192 weight gradient (96 tiles, 1.3 waves, 128 k-blocks): 151.6 us unsplit, 119.9
//     last wave, 111.6 every k-block;  2048 x 5632 x 8192 (176 tiles, last wave 38 % full): 149.6,
//     137.0, 146.9;  11264 x 2048 x 8192 (last wave 76 % full): 236.9, 234.6, 277.0;
//   2048 x 1536 x 6912 (48 tiles < 74 pairs, 108 k-blocks): 49.1 unsplit, 48.1 every k-block;
//     2048 x 2048 x 8192 (64 tiles): 81.3 unsplit, 85.1 every k-block;
//   short K (32 k-blocks: 8192 x 3072 x 2048, 8192 x 2048 x 2048, lm_head) lost 10 - 15 % split.
// So: at least 64 k-blocks; fewer tiles than pairs: every k-block if that saves >= 32 k-blocks per
// pair; otherwise the last wave must save >= 64 k-blocks per pair, split over every k-block when the
// grid is under two waves, else the last wave only.
static int pair_split_mode(long long tiles, int kb, int pairs) {
  if (tiles <= 0 || pairs <= 0 || kb < 64 || tiles * kb < 4LL * pairs) return 0;
  if (tiles < pairs) return kb - (double)tiles * kb / pairs >= 32.0 ? 2 : 0;
  const long long rem = tiles % pairs;
  if (rem == 0) return 0;
  if (kb * (1.0 - (double)rem / pairs) < 64.0) return 0;
  return tiles < 2LL * pairs ? 2 : 1;
}
static double effective_waves(long long tiles, int kb, int sms) {
  return use_streamk(tiles, kb, sms) ? (double)tiles / sms + 0.08 : (double)((tiles + sms - 1) / sms);
}

// Stream-K fix-up buffers, one set per (device, stream), made once outside graph capture:
// fp32 [sms][256 x 256] partial-tile slots (one per CTA) and [sms] slot flags (zero between launches).
struct SkBuf {
  cudaStream_t s;
  float* ws;
  int* flags;
};
static std::mutex g_sk_mu;
static std::vector<SkBuf> g_sk_bufs[64];
static bool sk_buffers(int dev, cudaStream_t s, int sms, float** ws, int** flags) {
  std::lock_guard<std::mutex> lock(g_sk_mu);
  for (const SkBuf& b : g_sk_bufs[dev & 63]) {
    if (b.s == s) {
      *ws = b.ws;
      *flags = b.flags;
      return true;
    }
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
  SkBuf b{s, nullptr, nullptr};
  if (cudaMalloc(&b.ws, (size_t)sms * 256 * 256 * sizeof(float)) != cudaSuccess) return false;
  if (cudaMalloc(&b.flags, (size_t)sms * sizeof(int)) != cudaSuccess) {
    cudaFree(b.ws);
    return false;
  }
  cudaMemsetAsync(b.flags, 0, (size_t)sms * sizeof(int), s);
  g_sk_bufs[dev & 63].push_back(b);
  *ws = b.ws;
  *flags = b.flags;
  return true;
}

// Pick the tile shape minimising (waves x per-tile cost); per-tile costs are
// relative throughputs of the three variants (256x256 moves the fewest bytes
// per FLOP, 128x128 the most). Waves are fractional where Stream-K applies.
static void pick_tile(int M, int N, int batch, int sms, int& bm, int& bn, int kb = 0) {
  // Measured on B200 (relative per-tile throughput at large K): 256x256 1.0,
  // 128x256 0.93; 128x128 is slower on every training shape and only used
  // when N <= 128.
  struct Opt { int bm, bn; double rel_speed; };
  const Opt opts[2] = {{256, 256, 1.0}, {128, 256, 0.93}};
  double best = 1e30;
  bm = 128;
  bn = N <= 128 ? 128 : 256;
  if (N <= 128) return;
  for (const Opt& o : opts) {
    if (o.bm == 256 && M <= 128) continue;
    const long long tiles = (long long)((M + o.bm - 1) / o.bm) * ((N + o.bn - 1) / o.bn) * batch;
    const double waves = kb > 0 ? effective_waves(tiles, kb, sms) : (double)((tiles + sms - 1) / sms);
    const double t = waves * o.bm * o.bn / o.rel_speed;
    if (t < best * 0.999) {
      best = t;
      bm = o.bm;
      bn = o.bn;
    }
  }
}

// Row strides (lda, ldb, ldd, ldc) and batch strides are in elements.
// a_mn == 0: A stored [batch][M][lda] (K contiguous); a_mn == 1: [batch][K][lda] (M contiguous).
// b_mn == 0: B stored [batch][N][ldb];                b_mn == 1: [batch][K][ldb].
// force_bn: 0 = automatic; 128 / 256 = BM 128 with that BN; 512 = 256 x 256 tiles; 1024 = 256 x 256
// tiles on a CTA pair; 1026 = the same with a Stream-K last wave where it applies;
// 2 = automatic among the single-CTA shapes (with Stream-K where it applies).
// Fused all-gather arguments of gemm_bf16 (see GemmParams::npeers).
struct GatherArgs {
  int npeers;
  long long peer_delta[astrai::kMaxGatherPeers];
  unsigned* flag;
  unsigned* done;
  unsigned epoch;
  int scatter_rpo, scatter_rank;  // > 0: reduce-scatter push instead of the all-gather copy
  long long scatter_recv_off;
  long long rank_delta[astrai::kMaxGatherPeers + 1];
};

// The plan gemm_bf16 would use for a plain GEMM on the current device: tile shape and whether the
// last partial wave is split Stream-K style (out: bm, bn, streamk, tiles, sms, pair, pair_streamk).
void gemm_plan(int M, int N, int K, int batch, int* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  int BM = 128, BN = 256;
  pick_tile(M, N, batch, sms, BM, BN, (K + 63) / 64);
  const long long tiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN) * batch;
  out[0] = BM;
  out[1] = BN;
  out[2] = use_streamk(tiles, (K + 63) / 64, sms) ? 1 : 0;
  out[3] = (int)tiles;
  out[4] = sms;
  // out[5]: the automatic choice runs this GEMM on 256 x 256 CTA-pair tiles instead (out[0..3]
  // describe the single-CTA plan, which force_bn 2 selects)
  out[5] = (M > 128 && N > 128 && pair_on()) ? 1 : 0;
  // out[6]: the pair plan with Stream-K allowed (force_bn 1026) splits its last wave
  const long long ptiles = (long long)((M + 255) / 256) * ((N + 255) / 256) * batch;
  out[6] = use_streamk_pair(ptiles, (K + 63) / 64, pair_clusters(dev)) ? 1 : 0;
}

static void sym_mirror(void* D, int out_f32, int M, long long ldd, long long strideD, int batch, cudaStream_t s) {
  if (out_f32) {
    const int nb = (M + 31) / 32;
    const dim3 grid(nb, nb, batch), block(32, 8);
    (astrai::note_launch(), astrai::sym_mirror_kernel<float><<<grid, block, 0, s>>>(static_cast<float*>(D), M, ldd, strideD));
    return;
  }
  // 64 x 64 blocks on or below the diagonal; 16-byte vectors need 16-byte rows (the GEMM checks ldd)
  const int t64 = (M + 63) / 64;
  if ((ldd * 2) % 16 || (reinterpret_cast<uintptr_t>(D) % 16) || (batch > 1 && (strideD * 2) % 16) || batch > 65535)
    throw std::runtime_error("astrai gemm: symmetric output needs 16-byte aligned rows and batch <= 65535");
  const dim3 grid(t64 * (t64 + 1) / 2, batch);
  (astrai::note_launch(), astrai::sym_mirror64_kernel<<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(D), M, ldd, strideD));
}

void gemm_bf16(const void* A, const void* B, void* D, const void* C, int M, int N, int K, int batch, int a_mn,
               long long lda, long long strideA, int b_mn, long long ldb, long long strideB, long long ldd,
               long long strideD, int out_f32, long long ldc, long long strideC, float alpha, float beta,
               int force_bn, cudaStream_t stream, const GatherArgs* gather, int sym) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) throw std::runtime_error("astrai gemm: empty problem");
  if (sym && (M != N || gather != nullptr)) throw std::runtime_error("astrai gemm: a symmetric output needs M == N");
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  int BM = 128, BN = 256;
  if (force_bn == 128 || force_bn == 256) {
    BN = force_bn;
  } else if (force_bn == 512 || force_bn == 1024) {
    BM = 256;
  } else {
    pick_tile(M, N, batch, sms, BM, BN, (K + 63) / 64);
  }
  // 256 x 256 tiles on a CTA pair (force_bn 1024, or the automatic pick under the pair policy);
  // 256 x 192 for a K-major B where pair_tile_n picks it (force_bn 192 forces it)
  const bool pair = gather == nullptr && (force_bn == 192 || force_bn == 1024 || force_bn == 1026 ||
                                          force_bn == 1027 || (force_bn == 0 && M > 128 && N > 128 && pair_on()));
  if (pair) {
    if (force_bn == 192 && (b_mn || sym)) throw std::runtime_error("astrai gemm: 256 x 192 tiles take a K-major B");
    BM = 256;
    BN = force_bn == 192 ? 192
                         : (force_bn == 0 && !b_mn && !sym ? pair_tile_n(M, N, K, batch, pair_clusters(dev)) : 256);
  }

  CUtensorMap ta, tb;
  {
    const uint64_t rows = a_mn ? (uint64_t)K : (uint64_t)M;
    const uint64_t inner = a_mn ? (uint64_t)M : (uint64_t)K;
    const uint64_t bstride = batch > 1 ? (uint64_t)strideA * 2 : (uint64_t)rows * lda * 2;
    uint64_t dims[3] = {inner, rows, (uint64_t)batch};
    uint64_t strides[2] = {(uint64_t)lda * 2, bstride ? bstride : 16};
    uint32_t box[3] = {64, a_mn ? 64u : 128u, 1};
    make_tmap_bf16(&ta, A, 3, dims, strides, box, true);
  }
  {
    const uint64_t rows = b_mn ? (uint64_t)K : (uint64_t)N;
    const uint64_t inner = b_mn ? (uint64_t)N : (uint64_t)K;
    const uint64_t bstride = batch > 1 ? (uint64_t)strideB * 2 : (uint64_t)rows * ldb * 2;
    uint64_t dims[3] = {inner, rows, (uint64_t)batch};
    uint64_t strides[2] = {(uint64_t)ldb * 2, bstride ? bstride : 16};
    uint32_t box[3] = {64, b_mn ? 64u : (uint32_t)(pair ? BN / 2 : BN), 1};
    make_tmap_bf16(&tb, B, 3, dims, strides, box, true);
  }
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.tiles_m = (M + BM - 1) / BM;
  p.tiles_n = (N + BN - 1) / BN;
  p.k_blocks = (K + 63) / 64;
  p.D = D;
  p.ldd = ldd;
  p.strideD = strideD;
  p.C = C;
  p.ldc = ldc;
  p.strideC = strideC;
  p.alpha = alpha;
  p.beta = beta;
  const int esz = out_f32 ? 4 : 2;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(D) % 16) == 0) && ((ldd * esz) % 16 == 0) &&
             (batch == 1 || (strideD * esz) % 16 == 0) &&
             (C == nullptr || (((reinterpret_cast<uintptr_t>(C) % 16) == 0) && ((ldc * esz) % 16 == 0) &&
                               (batch == 1 || (strideC * esz) % 16 == 0)));
  p.err = error_word(dev);
  p.group_tile = nullptr;
  p.k_start = nullptr;
  p.k_count = nullptr;
  p.prof = g_gemm_prof;
  p.epi = 0;
  p.F = 0;
  p.aux = nullptr;
  p.ldaux = 0;
  p.h = nullptr;
  p.ldh = 0;
  p.rope_cs = nullptr;
  p.rope_pos = nullptr;
  p.rope_seq = 1;
  p.rope_cols = 0;
  p.rope_hd = 2;
  p.rope_max = 0;
  p.dp_tiles = 0;
  p.sk_units = 0;
  p.sk_ws = nullptr;
  p.sk_flags = nullptr;
  p.npeers = 0;
  p.gather_flag = nullptr;
  p.gather_done = nullptr;
  p.gather_epoch = 0;
  p.scatter_rpo = 0;
  p.scatter_rank = 0;
  p.scatter_recv_off = 0;
  p.sym = 0;
  p.sym_bm = 1;
  p.sym_bn = 1;
  int tiles = batch * p.tiles_m * p.tiles_n;
  if (sym) {
    // square tiles: the tile walk enumerates the upper triangle only (gemm_tile); otherwise the
    // walk skips the tiles below the diagonal
    p.sym = BM == BN ? 2 : 1;
    p.sym_bm = BM;
    p.sym_bn = BN;
    if (p.sym == 2) tiles = batch * (p.tiles_m * (p.tiles_m + 1) / 2);
  }
  if (pair) {
    const int pmax = pair_clusters(dev);
    int pairs = std::min(tiles, pmax);
    // force_bn 1026: the last wave split wherever use_streamk_pair allows it (also ASTRAI_PAIR_STREAMK=1);
    // force_bn 1027: every k-block split over all pairs whatever the shape (needs tiles * kb >= pairs);
    // force_bn 0: pair_split_mode
    const int automatic = (force_bn == 0 && BN == 256 && streamk_on()) ? pair_split_mode(tiles, p.k_blocks, pmax) : 0;
    const bool split = !sym && BN == 256 && (force_bn == 1026 || automatic == 1 ||
                                             (force_bn != 1024 && force_bn != 1027 && pair_streamk_on() &&
                                              streamk_on()));
    const bool all_units = !sym && BN == 256 &&
                           (force_bn == 1027 ? (long long)tiles * p.k_blocks >= pmax : automatic == 2);
    if (all_units && sk_buffers(dev, stream, sms, &p.sk_ws, &p.sk_flags)) {
      p.dp_tiles = 0;
      p.sk_units = (long long)tiles * p.k_blocks;
      pairs = pmax;
    } else if (split && use_streamk_pair(tiles, p.k_blocks, pmax) &&
               sk_buffers(dev, stream, sms, &p.sk_ws, &p.sk_flags)) {
      p.dp_tiles = tiles / pmax * pmax;
      p.sk_units = (long long)(tiles - p.dp_tiles) * p.k_blocks;
      pairs = pmax;
    }
    if (BN == 192)
      dispatch_pair192(a_mn, out_f32, ta, tb, p, pairs, stream);
    else
      dispatch_pair<256>(a_mn, b_mn, out_f32, ta, tb, p, pairs, stream);
    if (sym) sym_mirror(D, out_f32, M, ldd, strideD, batch, stream);
    return;
  }
  int grid = std::min(tiles, sms);
  if (gather != nullptr) {
    if (C != nullptr || out_f32 || batch != 1 || gather->npeers < 0 || gather->npeers > astrai::kMaxGatherPeers)
      throw std::runtime_error("astrai gemm: the fused all-gather takes a plain bf16 GEMM and at most 7 peers");
    p.npeers = gather->npeers;
    for (int q = 0; q < gather->npeers; ++q) p.peer_delta[q] = gather->peer_delta[q];
    p.gather_flag = gather->flag;
    p.gather_done = gather->done;
    p.gather_epoch = gather->epoch;
    p.scatter_rpo = gather->scatter_rpo;
    p.scatter_rank = gather->scatter_rank;
    p.scatter_recv_off = gather->scatter_recv_off;
    for (int q = 0; q <= astrai::kMaxGatherPeers; ++q) p.rank_delta[q] = gather->rank_delta[q];
  } else if (!sym && use_streamk(tiles, p.k_blocks, sms) && sk_buffers(dev, stream, sms, &p.sk_ws, &p.sk_flags)) {
    p.dp_tiles = tiles / sms * sms;
    p.sk_units = (long long)(tiles - p.dp_tiles) * p.k_blocks;
    grid = sms;
  }
  if (BM == 256)
    dispatch_majors<256, 256>(a_mn, b_mn, out_f32, ta, tb, p, grid, stream);
  else if (BN == 256)
    dispatch_majors<128, 256>(a_mn, b_mn, out_f32, ta, tb, p, grid, stream);
  else
    dispatch_majors<128, 128>(a_mn, b_mn, out_f32, ta, tb, p, grid, stream);
  if (sym) sym_mirror(D, out_f32, M, ldd, strideD, batch, stream);
}


// Grouped GEMMs for mixture-of-experts blocks (BM = 128 tiles).
//  mode 0 (grouped-M): A [M_total, K] K-major (lda), D [M_total, N] (ldd), B batched by group
//         [groups][N][K] (b_mn 0) or [groups][K][N] (b_mn 1); group_tile[M_total / 128].
//  mode 1 (grouped-K): A [K_total, M] and B [K_total, N] MN-major, D [groups][M][N];
//         group g reduces rows [k_start[g], k_start[g] + k_count[g]) (multiples of 64).
void gemm_grouped_bf16(int mode, const void* A, const void* B, void* D, const void* C, int M, int N, int K,
                       int groups, int b_mn, long long lda, long long ldb, long long strideB, long long ldd,
                       long long strideD, const int* group_tile, const int* k_start, const int* k_count,
                       float alpha, float beta, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || groups <= 0) throw std::runtime_error("astrai grouped gemm: empty problem");
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  constexpr int BM = 128;
  const int BN = N <= 128 ? 128 : 256;
  CUtensorMap ta, tb;
  const int a_mn = mode == 1 ? 1 : 0;
  if (mode == 1) b_mn = 1;
  {
    const uint64_t rows = a_mn ? (uint64_t)K : (uint64_t)M;
    const uint64_t inner = a_mn ? (uint64_t)M : (uint64_t)K;
    uint64_t dims[3] = {inner, rows, 1};
    uint64_t strides[2] = {(uint64_t)lda * 2, (uint64_t)rows * lda * 2};
    uint32_t box[3] = {64, a_mn ? 64u : 128u, 1};
    make_tmap_bf16(&ta, A, 3, dims, strides, box, true);
  }
  {
    const uint64_t rows = b_mn ? (uint64_t)K : (uint64_t)N;
    const uint64_t inner = b_mn ? (uint64_t)N : (uint64_t)K;
    const uint64_t nb = mode == 0 ? (uint64_t)groups : 1;
    const uint64_t bstride = mode == 0 ? (uint64_t)strideB * 2 : (uint64_t)rows * ldb * 2;
    uint64_t dims[3] = {inner, rows, nb};
    uint64_t strides[2] = {(uint64_t)ldb * 2, bstride};
    uint32_t box[3] = {64, b_mn ? 64u : (uint32_t)BN, 1};
    make_tmap_bf16(&tb, B, 3, dims, strides, box, true);
  }
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = mode == 0 ? 1 : groups;
  p.tiles_m = (M + BM - 1) / BM;
  p.tiles_n = (N + BN - 1) / BN;
  p.k_blocks = (K + 63) / 64;
  p.D = D;
  p.ldd = ldd;
  p.strideD = mode == 0 ? 0 : strideD;
  p.C = C;
  p.ldc = ldd;
  p.strideC = p.strideD;
  p.alpha = alpha;
  p.beta = beta;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(D) % 16) == 0) && ((ldd * 2) % 16 == 0) && ((p.strideD * 2) % 16 == 0) &&
             (C == nullptr || (reinterpret_cast<uintptr_t>(C) % 16) == 0);
  p.err = error_word(dev);
  p.group_tile = mode == 0 ? group_tile : nullptr;
  p.k_start = mode == 1 ? k_start : nullptr;
  p.k_count = mode == 1 ? k_count : nullptr;
  p.prof = g_gemm_prof;
  p.epi = 0;
  p.F = 0;
  p.aux = nullptr;
  p.ldaux = 0;
  p.h = nullptr;
  p.ldh = 0;
  p.rope_cs = nullptr;
  p.rope_pos = nullptr;
  p.rope_seq = 1;
  p.rope_cols = 0;
  p.rope_hd = 2;
  p.rope_max = 0;
  p.dp_tiles = 0;
  p.sk_units = 0;
  p.sk_ws = nullptr;
  p.sk_flags = nullptr;
  p.npeers = 0;
  p.gather_flag = nullptr;
  p.gather_done = nullptr;
  p.gather_epoch = 0;
  p.scatter_rpo = 0;
  p.scatter_rank = 0;
  p.scatter_recv_off = 0;
  p.sym = 0;
  p.sym_bm = 1;
  p.sym_bn = 1;
  const int tiles = p.batch * p.tiles_m * p.tiles_n;
  const int grid = std::min(tiles, sms);
  if (BN == 256)
    dispatch_majors<128, 256>(a_mn, b_mn, 0, ta, tb, p, grid, stream);
  else
    dispatch_majors<128, 128>(a_mn, b_mn, 0, ta, tb, p, grid, stream);
}


// GEMMs with a fused SwiGLU epilogue (see GemmParams::epi). A is K-major [M, K] (lda).
//  mode 1: B = packed [up; gate] weight [2F, K] K-major (ldb); writes h [M, 2F] (ldd; skipped when D
//          is null) and a = silu(g) * u [M, F] (ldaux). Needs F % 128 == 0 (tiles pair 128 up and 128
//          gate rows).
//  mode 2: B = W_down stored [K][F] (b_mn 1) or [F][K] (b_mn 0); with the saved h [M, 2F] (ldh)
//          writes dh [M, 2F] (ldaux); da = A @ B^T itself is never stored.
void gemm_swiglu_bf16(int mode, const void* A, long long lda, const void* B, long long ldb, int b_mn, void* D,
                      long long ldd, void* aux, long long ldaux, const void* h, long long ldh, int M, int F, int K,
                      cudaStream_t stream) {
  if (M <= 0 || F <= 0 || K <= 0) throw std::runtime_error("astrai gemm_swiglu: empty problem");
  if (mode == 1 && (F % 128 || b_mn)) throw std::runtime_error("gemm_swiglu mode 1: F % 128 == 0, K-major B");
  if (mode != 1 && mode != 2) throw std::runtime_error("gemm_swiglu: mode 1 or 2");
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  const int BN = 256;
  // 256-row tiles on a CTA pair (double-buffered accumulators, see gemm_pair_kernel) where the pair
  // policy applies, else 128-row single-CTA tiles (double-buffered accumulator)
  const bool pair = M > 128 && pair_on();
  const int BM = pair ? 256 : 128;
  if (mode == 2 && F <= 128) throw std::runtime_error("gemm_swiglu mode 2: F > 128");
  CUtensorMap ta, tb;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, 1};
    uint64_t strides[2] = {(uint64_t)lda * 2, (uint64_t)M * lda * 2};
    uint32_t box[3] = {64, 128u, 1};
    make_tmap_bf16(&ta, A, 3, dims, strides, box, true);
  }
  {
    const uint64_t rows = mode == 1 ? (uint64_t)2 * F : (b_mn ? (uint64_t)K : (uint64_t)F);
    const uint64_t inner = mode == 1 ? (uint64_t)K : (b_mn ? (uint64_t)F : (uint64_t)K);
    uint64_t dims[3] = {inner, rows, 1};
    uint64_t strides[2] = {(uint64_t)ldb * 2, rows * ldb * 2};
    const uint32_t box_rows = mode == 1 ? (uint32_t)(BN / 2) : (b_mn ? 64u : (uint32_t)(pair ? BN / 2 : BN));
    uint32_t box[3] = {64, box_rows, 1};
    make_tmap_bf16(&tb, B, 3, dims, strides, box, true);
  }
  GemmParams p;
  p.M = M;
  p.N = mode == 1 ? 2 * F : F;
  p.K = K;
  p.batch = 1;
  p.tiles_m = (M + BM - 1) / BM;
  p.tiles_n = mode == 1 ? F / (BN / 2) : (F + BN - 1) / BN;
  p.k_blocks = (K + 63) / 64;
  p.D = mode == 1 ? D : aux;
  p.ldd = mode == 1 ? ldd : ldaux;
  p.strideD = 0;
  p.C = nullptr;
  p.ldc = 0;
  p.strideC = 0;
  p.alpha = 1.f;
  p.beta = 0.f;
  const auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 16) == 0; };
  p.vec_ok = al16(aux) && (ldaux * 2) % 16 == 0 && (mode == 1 ? (al16(D) && (ldd * 2) % 16 == 0)
                                                              : (al16(h) && (ldh * 2) % 16 == 0)) && F % 8 == 0;
  p.err = error_word(dev);
  p.group_tile = nullptr;
  p.k_start = nullptr;
  p.k_count = nullptr;
  p.prof = g_gemm_prof;
  p.epi = mode;
  p.F = F;
  p.aux = static_cast<__nv_bfloat16*>(aux);
  p.ldaux = ldaux;
  p.h = static_cast<const __nv_bfloat16*>(h);
  p.ldh = ldh;
  p.rope_cs = nullptr;
  p.rope_pos = nullptr;
  p.rope_seq = 1;
  p.rope_cols = 0;
  p.rope_hd = 2;
  p.rope_max = 0;
  p.dp_tiles = 0;
  p.sk_units = 0;
  p.sk_ws = nullptr;
  p.sk_flags = nullptr;
  p.npeers = 0;
  p.gather_flag = nullptr;
  p.gather_done = nullptr;
  p.gather_epoch = 0;
  p.scatter_rpo = 0;
  p.scatter_rank = 0;
  p.scatter_recv_off = 0;
  p.sym = 0;
  p.sym_bm = 1;
  p.sym_bn = 1;
  const int tiles = p.tiles_m * p.tiles_n;
  if (pair)
    return dispatch_pair<256>(0, mode == 1 ? 0 : b_mn, 0, ta, tb, p, std::min(tiles, pair_clusters(dev)), stream);
  const int grid = std::min(tiles, sms);
  dispatch_majors<128, 256>(0, mode == 1 ? 0 : b_mn, 0, ta, tb, p, grid, stream);
}


// x [M, K] @ w [N, K]^T with RoPE applied in the epilogue to columns [0, rope_cols) (see GemmParams).
void gemm_rope_bf16(const void* A, long long lda, const void* B, long long ldb, void* D, long long ldd, int M, int N,
                    int K, const void* cs, const int* pos, int seq, int rope_cols, int head_dim, int max_pos,
                    cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) throw std::runtime_error("astrai gemm_rope: empty problem");
  if (head_dim % 32 || rope_cols % head_dim || rope_cols > N || seq <= 0)
    throw std::runtime_error("gemm_rope: head_dim multiple of 32, whole heads, seq > 0");
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  // 256 x 256 tiles on a CTA pair where the pair policy applies (as in gemm_bf16), else 128-row
  // single-CTA tiles; both double-buffer the accumulator, so the rotation overlaps the next MMAs
  const bool pair = M > 128 && N > 128 && pair_on();
  const int BM = pair ? 256 : 128;
  const int BN = pair ? pair_tile_n(M, N, K, 1, pair_clusters(dev)) : (N <= 128 ? 128 : 256);
  if (reinterpret_cast<uintptr_t>(cs) % 16) throw std::runtime_error("gemm_rope: cos/sin table must be 16-byte aligned");
  CUtensorMap ta, tb;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, 1};
    uint64_t strides[2] = {(uint64_t)lda * 2, (uint64_t)M * lda * 2};
    uint32_t box[3] = {64, 128u, 1};
    make_tmap_bf16(&ta, A, 3, dims, strides, box, true);
  }
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, 1};
    uint64_t strides[2] = {(uint64_t)ldb * 2, (uint64_t)N * ldb * 2};
    uint32_t box[3] = {64, (uint32_t)(pair ? BN / 2 : BN), 1};
    make_tmap_bf16(&tb, B, 3, dims, strides, box, true);
  }
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = 1;
  p.tiles_m = (M + BM - 1) / BM;
  p.tiles_n = (N + BN - 1) / BN;
  p.k_blocks = (K + 63) / 64;
  p.D = D;
  p.ldd = ldd;
  p.strideD = 0;
  p.C = nullptr;
  p.ldc = 0;
  p.strideC = 0;
  p.alpha = 1.f;
  p.beta = 0.f;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(D) % 16) == 0) && ((ldd * 2) % 16 == 0);
  p.err = error_word(dev);
  p.group_tile = nullptr;
  p.k_start = nullptr;
  p.k_count = nullptr;
  p.prof = g_gemm_prof;
  p.epi = 3;
  p.F = 0;
  p.aux = nullptr;
  p.ldaux = 0;
  p.h = nullptr;
  p.ldh = 0;
  p.rope_cs = static_cast<const float2*>(cs);
  p.rope_pos = pos;
  p.rope_seq = seq;
  p.rope_cols = rope_cols;
  p.rope_hd = head_dim;
  p.rope_max = max_pos;
  p.dp_tiles = 0;
  p.sk_units = 0;
  p.sk_ws = nullptr;
  p.sk_flags = nullptr;
  p.npeers = 0;
  p.gather_flag = nullptr;
  p.gather_done = nullptr;
  p.gather_epoch = 0;
  p.scatter_rpo = 0;
  p.scatter_rank = 0;
  p.scatter_recv_off = 0;
  p.sym = 0;
  p.sym_bm = 1;
  p.sym_bn = 1;
  const int tiles = p.tiles_m * p.tiles_n;
  if (pair && BN == 192) return dispatch_pair192(0, 0, ta, tb, p, std::min(tiles, pair_clusters(dev)), stream);
  if (pair) return dispatch_pair<256>(0, 0, 0, ta, tb, p, std::min(tiles, pair_clusters(dev)), stream);
  const int grid = std::min(tiles, sms);
  if (BN == 256)
    dispatch_majors<128, 256>(0, 0, 0, ta, tb, p, grid, stream);
  else
    dispatch_majors<128, 128>(0, 0, 0, ta, tb, p, grid, stream);
}

}  // namespace astrai_host
