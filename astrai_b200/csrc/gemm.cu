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
#include <stdexcept>

#include "common.cuh"

namespace astrai {

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
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
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

template <int BN, int A_MN, int B_MN, int OUT_F32>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.batch * p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int b, mb, nb;
        tile_coords(tile, p.tiles_m, p.tiles_n, b, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) tma_load_3d(a_dst + c * 8192, &tmA, &full[stage], m0 + c * 64, k0, b);
          } else {
            tma_load_3d(a_dst, &tmA, &full[stage], k0, m0, b);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_3d(b_dst + c * 8192, &tmB, &full[stage], n0 + c * 64, k0, b);
          } else {
            tma_load_3d(b_dst, &tmB, &full[stage], k0, n0, b);
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
      constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, p.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_base + k * 2048, 8192, 1024) : sdesc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_base + k * 2048, 8192, 1024) : sdesc_sw128(b_base + k * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int b, mb, nb;
      tile_coords(tile, p.tiles_m, p.tiles_n, b, mb, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, p.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const int n0 = nb * BN;
      const bool row_ok = row < p.M;
      using OutT = typename std::conditional<OUT_F32, float, __nv_bfloat16>::type;
      OutT* drow = reinterpret_cast<OutT*>(p.D) + (long long)b * p.strideD + (long long)row * p.ldd;
      const OutT* crow = p.C ? reinterpret_cast<const OutT*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc
                             : nullptr;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + c, r);
        tmem_wait_ld();
        const int col = n0 + c;
        if (!row_ok || col >= p.N) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
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
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace astrai

namespace astrai_host {

using astrai::GemmCfg;
using astrai::GemmParams;

template <int BN, int A_MN, int B_MN, int OUT_F32>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
                        cudaStream_t stream) {
  auto kern = astrai::gemm_kernel<BN, A_MN, B_MN, OUT_F32>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM);
    attr_set[dev & 63] = true;
  }
  kern<<<grid, 192, GemmCfg<BN>::SMEM, stream>>>(ta, tb, p);
}

template <int BN>
static void dispatch_majors(int a_mn, int b_mn, int out_f32, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmParams& p, int grid, cudaStream_t s) {
#define ASTRAI_GEMM_CASE(AM, BMJ, OF) \
  if (a_mn == AM && b_mn == BMJ && out_f32 == OF) return launch_gemm<BN, AM, BMJ, OF>(ta, tb, p, grid, s);
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

static int pick_bn(int M, int N, int batch, int sms) {
  if (N <= 128) return 128;
  auto eff = [&](int bn) {
    long long tiles = (long long)((M + 127) / 128) * ((N + bn - 1) / bn) * batch;
    long long waves = (tiles + sms - 1) / sms;
    return (double)tiles / (double)(waves * sms);
  };
  // 256-wide tiles halve A re-reads; only drop to 128 when it fixes a bad tail.
  return eff(128) > eff(256) + 0.12 ? 128 : 256;
}

// Row strides (lda, ldb, ldd, ldc) and batch strides are in elements.
// a_mn == 0: A stored [batch][M][lda] (K contiguous); a_mn == 1: [batch][K][lda] (M contiguous).
// b_mn == 0: B stored [batch][N][ldb];                b_mn == 1: [batch][K][ldb].
void gemm_bf16(const void* A, const void* B, void* D, const void* C, int M, int N, int K, int batch, int a_mn,
               long long lda, long long strideA, int b_mn, long long ldb, long long strideB, long long ldd,
               long long strideD, int out_f32, long long ldc, long long strideC, float alpha, float beta,
               int force_bn, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) throw std::runtime_error("astrai gemm: empty problem");
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  const int BN = force_bn ? force_bn : pick_bn(M, N, batch, sms);

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
    uint32_t box[3] = {64, b_mn ? 64u : (uint32_t)BN, 1};
    make_tmap_bf16(&tb, B, 3, dims, strides, box, true);
  }
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.tiles_m = (M + 127) / 128;
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
  const int tiles = batch * p.tiles_m * p.tiles_n;
  const int grid = std::min(tiles, sms);
  if (BN == 256)
    dispatch_majors<256>(a_mn, b_mn, out_f32, ta, tb, p, grid, stream);
  else
    dispatch_majors<128>(a_mn, b_mn, out_f32, ta, tb, p, grid, stream);
}

}  // namespace astrai_host
