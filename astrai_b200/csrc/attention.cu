// Causal GQA flash attention on tcgen05 (sm_100a), forward and backward.
//
// Replaces F.scaled_dot_product_attention + repeat_kv of the reference
// (astrai/model/components/attention.py:15-23, :96-101). K/V heads are shared
// by Hq/Hkv query heads without materialising repeated K/V; q, k and v are
// read by TMA directly out of the fused QKV projection output (any row
// stride), and the output is written in the [tokens, Hq*D] layout the
// o-projection GEMM consumes.
//
// Forward, one CTA per (128-query block, query head, batch):
//   warp 0      TMA: Q once, then K_j / V_j into a 2-stage ring
//   warp 1      TMEM owner + MMA issuer:
//                 S_j = Q K_j^T      (128x128x128, both K-major) -> TMEM (2 buffers)
//                 O  += P_j V_j      (P K-major from smem, V MN-major)
//   warps 2..5  softmax, one query row per thread: row max from TMEM, lazy
//               rescaling of O (only when the running max grows by > 2^8),
//               P_j = exp2(S*scale*log2e - m) written bf16 into a 128B-swizzled
//               smem tile for the PV MMA; final O / l and log-sum-exp.
// Backward, one CTA per (128-key block, kv head, batch), looping over the
// query heads of the group and the causal query blocks:
//   S^T = K Q^T, dP^T = V dO^T (TMEM), P^T back to TMEM and dS^T (scaled) to smem,
//   dV += P^T dO (P^T from TMEM), dK += dS^T Q (TMEM accumulators for the whole CTA),
//   dQ_part = dS K -> fp32 atomics into a dQ accumulator.
// All waits are time-bounded (common.cuh).
#include <cfloat>
#include <stdexcept>

#include "common.cuh"

namespace astrai {

struct FlashFwdParams {
  int B, Sq, Sk, Hq, Hkv;
  int q_col0, k_col0, v_col0;  // column of head 0 inside each tensor map's buffer
  __nv_bfloat16* O;
  long long ldo;  // row stride of O (elements); head h at column h*128
  float* lse;     // [B, Hq, Sq] natural-log LSE
  float scale_log2;
  int causal;
  const int* seg;  // optional [B, Sk] segment ids: q attends k only if seg equal
  int* err;
};

constexpr int FA_D = 128;
constexpr int FA_BM = 128;
constexpr int FA_BN = 128;
constexpr int FA_TILE = 128 * 64 * 2;  // one 128-row x 64-col swizzled chunk (16 KB)
constexpr int FA_FWD_SMEM = (2 + 4 + 4 + 4) * FA_TILE + 1024 + 256;

// Swizzled address of the 16-byte granule `g` (0..7) of row `r` inside a
// 128-row x 64-col (bf16) chunk: matches TMA SWIZZLE_128B and the UMMA layout.
__device__ __forceinline__ uint32_t swz(uint32_t chunk_base, int r, int g) {
  return chunk_base + r * 128 + ((g ^ (r & 7)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void ld_shared_v4f(uint32_t addr, float& a, float& b, float& c, float& d) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(a), "=f"(b), "=f"(c), "=f"(d) : "r"(addr));
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// bits [lo, hi) set in a 64-bit mask held as two words (lo/hi clamped to [0, 64])
__device__ __forceinline__ void row_mask64(int lo, int hi, uint32_t (&m)[2]) {
  lo = max(0, min(64, lo));
  hi = max(0, min(64, hi));
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const int a = max(0, min(32, lo - 32 * w)), b = max(0, min(32, hi - 32 * w));
    const uint32_t upto_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
    const uint32_t upto_a = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
    m[w] = b > a ? (upto_b & ~upto_a) : 0u;
  }
}
// bits [0, hi) set in a 128-bit mask held as four words
__device__ __forceinline__ void row_mask128(int hi, uint32_t (&m)[4]) {
  hi = max(0, min(128, hi));
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int b = max(0, min(32, hi - 32 * w));
    m[w] = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA pipe instead of the MUFU unit, so both pipes share
// the softmax's exponentials. Split x = n + f with n = floor(x) (a round-down
// add of 1.5 * 2^23 leaves n in the low mantissa bits), approximate 2^f on
// [0, 1) by 1 + c1 f + c2 f^2 + c3 f^3 (coefficients from a relative-error
// least-squares fit with Lawson reweighting, max relative error 8.6e-5, well
// under bf16 resolution), and put n into the exponent field (exponent-field
// construction as in Schraudolph, 1999). x < -127 gives 0.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -127.f);
  const float t = __fadd_rd(xc, 12582912.f);
  const float n = t - 12582912.f;
  const float f = xc - n;
  const float p = fmaf(fmaf(fmaf(0.07706134f, f, 0.22765121f), f, 0.69511539f), f, 1.f);
  const int ni = __float_as_int(t) - 0x4B400000;
  const float y = __int_as_float(__float_as_int(p) + (ni << 23));
  return x < -127.f ? 0.f : y;
}
// of every 16 exponential pairs in the forward softmax, this many go to exp2_fma
// (7 of 16 measured no faster than MUFU only at B4 S2048 H16/4: the softmax is not MUFU-bound)
constexpr int FA_EMU_PAIRS = 0;

__global__ void __launch_bounds__(192, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FlashFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // 2 chunks
  uint8_t* sK = sQ + 2 * FA_TILE;        // 2 stages x 2 chunks
  uint8_t* sV = sK + 4 * FA_TILE;        // 2 stages x 2 chunks
  uint8_t* sP = sV + 4 * FA_TILE;        // 2 slots x 2 chunks
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 4 * FA_TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]  released when S_j is computed
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]  released when PV_j is computed
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* p_ready = bars + 11;
  uint64_t* pv_done = bars + 12;  // [2] per P slot: PV of the block that used the slot is done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = warp_id(), lane = lane_id();
  const int n_mblocks = (p.Sq + FA_BM - 1) / FA_BM;
  // 1-D grid in longest-first order: CTAs start in index order, so every causal
  // query block of the last position (the most key blocks) of all heads and
  // batches is issued before any lighter one and the light blocks fill the tail
  const int hb = p.Hq * p.B;
  const int mb = n_mblocks - 1 - (int)(blockIdx.x / hb);
  const int h = (int)(blockIdx.x % hb) % p.Hq, b = (int)(blockIdx.x % hb) / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int m0 = mb * FA_BM;
  const int off = p.Sk - p.Sq;  // causal offset (queries are the last Sq positions)
  int n_blocks = (p.Sk + FA_BN - 1) / FA_BN;
  if (p.causal) n_blocks = min(n_blocks, max(0, (m0 + FA_BM - 1 + off) / FA_BN + 1));

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    mbar_init(p_ready, 4);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0 && n_blocks > 0) {
      mbar_expect_tx(q_full, 2 * FA_TILE);
      tma_load_3d(sQ, &tmQ, q_full, p.q_col0 + h * FA_D, m0, b);
      tma_load_3d(sQ + FA_TILE, &tmQ, q_full, p.q_col0 + h * FA_D + 64, m0, b);
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[st], par, p.err, kErrWaitEmpty)) break;
        mbar_expect_tx(&k_full[st], 2 * FA_TILE);
        uint8_t* k = sK + st * 2 * FA_TILE;
        tma_load_3d(k, &tmK, &k_full[st], p.k_col0 + hk * FA_D, j * FA_BN, b);
        tma_load_3d(k + FA_TILE, &tmK, &k_full[st], p.k_col0 + hk * FA_D + 64, j * FA_BN, b);
        if (!mbar_wait(&v_empty[st], par, p.err, kErrWaitEmpty)) break;
        mbar_expect_tx(&v_full[st], 2 * FA_TILE);
        uint8_t* v = sV + st * 2 * FA_TILE;
        tma_load_3d(v, &tmV, &v_full[st], p.v_col0 + hk * FA_D, j * FA_BN, b);
        tma_load_3d(v + FA_TILE, &tmV, &v_full[st], p.v_col0 + hk * FA_D + 64, j * FA_BN, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_blocks > 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idO = idesc_bf16(128, 128, 0, 1);
      bool ok = mbar_wait(q_full, 0, p.err, kErrWaitFull);
      const uint32_t q_base = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + st * 2 * FA_TILE);
#pragma unroll
        for (int k = 0; k < FA_D / 16; ++k) {
          const uint32_t o = (k >> 2) * FA_TILE + (k & 3) * 32;
          umma_bf16(tS + st * 128, sdesc_sw128(q_base + o, 16, 1024), sdesc_sw128(k_base + o, 16, 1024), idS, k > 0);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      const uint32_t p_base = smem_u32(sP);
      for (int j = 0; j < n_blocks && ok; ++j) {
        const int st = j & 1;
        // S_{j+1} overlaps the softmax of S_j (its buffer was released by p_ready_{j-1})
        if (j + 1 < n_blocks && !issue_s(j + 1)) break;
        if (!mbar_wait(p_ready, j & 1, p.err, kErrWaitAccFull)) break;
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t v_base = smem_u32(sV + st * 2 * FA_TILE);
#pragma unroll
        for (int k = 0; k < FA_BN / 16; ++k) {
          const uint64_t ad = sdesc_sw128(p_base + st * 2 * FA_TILE + (k >> 2) * FA_TILE + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_base + k * 2048, FA_TILE, 1024);
          umma_bf16(tO, ad, bd, idO, (j | k) != 0);
        }
        umma_commit(&pv_done[st]);
        umma_commit(&v_empty[st]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row inside the block == TMEM lane
    const int qi = m0 + r;         // query position
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t p_base = smem_u32(sP);
    const int seg_q = (p.seg && qi < p.Sq) ? p.seg[(long long)b * p.Sk + qi + off] : 0;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;  // m_used in scaled log2 units
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1, p.err, kErrWaitAccFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * FA_BN;
      const bool need_mask = (p.causal && (k0 + FA_BN - 1 > m0 + off)) || (k0 + FA_BN > p.Sk) || p.seg;
      uint32_t vis[4];
      if (need_mask) {
        const int hi = min(p.Sk - k0, p.causal ? qi + off - k0 + 1 : FA_BN);  // one past last visible key
        row_mask128(hi, vis);
        if (p.seg) {
#pragma unroll 1
          for (int c = 0; c < FA_BN; ++c) {
            const int ki = k0 + c;
            if (ki < p.Sk && p.seg[(long long)b * p.Sk + ki] != seg_q) vis[c >> 5] &= ~(1u << (c & 31));
          }
        }
      }
      // the whole 128-column row of S in registers: 4 loads, one wait
      uint32_t v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t(&vc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]);
        tmem_ld32(tS + st * 128 + lane_off + c * 32, vc);
      }
      tmem_wait_ld();
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          v[i] = ((vis[i >> 5] >> (i & 31)) & 1u) ? v[i] : __float_as_uint(-INFINITY);
      }
      // raw row max (scale > 0, so scaling commutes with max)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        mx0 = fmaxf(mx0, __uint_as_float(v[i]));
        mx1 = fmaxf(mx1, __uint_as_float(v[i + 1]));
      }
      const float m_new = fmaxf(m_used, fmaxf(mx0, mx1) * sl2);
      const bool need = (m_used == -INFINITY && m_new != -INFINITY) || (m_new - m_used > 8.f);
      // P slot st was last read by PV_{j-2}
      if (j >= 2) {
        if (!mbar_wait(&pv_done[st], ((j - 2) >> 1) & 1, p.err, kErrWaitAccFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const bool rescale = __any_sync(0xffffffff, need);
      if (rescale && j >= 1) {
        // O must be stable: PV_{j-1} done
        if (!mbar_wait(&pv_done[st ^ 1], ((j - 1) >> 1) & 1, p.err, kErrWaitAccFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (rescale) {
        const float factor = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
        if (j > 0) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t o[64];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t(&oc)[16] = *reinterpret_cast<uint32_t(*)[16]>(&o[c * 16]);
              tmem_ld16(tO + lane_off + hf * 64 + c * 16, oc);
            }
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 64; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t(&oc)[16] = *reinterpret_cast<const uint32_t(*)[16]>(&o[c * 16]);
              tmem_st16(tO + lane_off + hf * 64 + c * 16, oc);
            }
          }
          tmem_wait_st();
        }
        l *= factor;
        m_used = m_new;
      }
      const float msafe = (m_used == -INFINITY) ? 0.f : m_used;
      // p = 2^(s*scale*log2e - m), bf16 into the swizzled P tile
      float l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = fmaf(__uint_as_float(v[c * 32 + 2 * i]), sl2, -msafe);
          const float x1 = fmaf(__uint_as_float(v[c * 32 + 2 * i + 1]), sl2, -msafe);
          const bool emu = i < FA_EMU_PAIRS;  // compile-time after unrolling
          const float e0 = emu ? exp2_fma(x0) : ex2(x0);
          const float e1 = emu ? exp2_fma(x1) : ex2(x1);
          l0 += e0;
          l1 += e1;
          pk[i] = pack_bf16(e0, e1);
        }
        const uint32_t cb = p_base + st * 2 * FA_TILE + (c >> 1) * FA_TILE;
#pragma unroll
        for (int g = 0; g < 4; ++g)
          st_shared_v4(swz(cb, r, (c & 1) * 4 + g), pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
      }
      l += l0 + l1;
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
    }
    if (ok && n_blocks > 0 &&
        mbar_wait(&pv_done[(n_blocks - 1) & 1], ((n_blocks - 1) >> 1) & 1, p.err, kErrWaitAccFull)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = qi < p.Sq;
      __nv_bfloat16* orow = p.O + ((long long)b * p.Sq + qi) * p.ldo + h * FA_D;
      uint32_t ov[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t(&oc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&ov[c * 32]);
        tmem_ld32(tO + lane_off + c * 32, oc);
      }
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t* v = &ov[c * 32];
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int g = 0; g < 4; ++g)
            dst[g] = make_uint4(pack_bf16(__uint_as_float(v[8 * g]) * inv, __uint_as_float(v[8 * g + 1]) * inv),
                                pack_bf16(__uint_as_float(v[8 * g + 2]) * inv, __uint_as_float(v[8 * g + 3]) * inv),
                                pack_bf16(__uint_as_float(v[8 * g + 4]) * inv, __uint_as_float(v[8 * g + 5]) * inv),
                                pack_bf16(__uint_as_float(v[8 * g + 6]) * inv, __uint_as_float(v[8 * g + 7]) * inv));
        }
      }
      if (row_ok)
        p.lse[((long long)b * p.Hq + h) * p.Sq + qi] =
            (l > 0.f) ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
    } else if (n_blocks == 0 && qi < p.Sq) {
      __nv_bfloat16* orow = p.O + ((long long)b * p.Sq + qi) * p.ldo + h * FA_D;
      for (int c = 0; c < FA_D; ++c) orow[c] = __float2bfloat16_rn(0.f);
      p.lse[((long long)b * p.Hq + h) * p.Sq + qi] = -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================== backward
struct FlashBwdParams {
  int B, Sq, Sk, Hq, Hkv;
  int q_col0, k_col0, v_col0, do_col0;
  const float* lse2;   // [B, Hq, Sq_pad] LSE in log2 units (+inf past Sq)
  const float* delta;  // [B, Hq, Sq_pad] rowsum(dO * O) (0 past Sq)
  int Sq_pad;          // Sq rounded up to the 64-query tile
  float* dq_acc;       // [B*Sq, Hq*128] fp32, zeroed by flash_bwd_pre_kernel
  __nv_bfloat16* dk;   // [B*Sk, ldk_out]  head hk at column dk_col0 + hk*128
  __nv_bfloat16* dv;
  long long ld_dkv;
  int dk_col0, dv_col0;
  float scale, scale_log2;
  int causal;
  const int* seg;
  int* err;
};

// Query tile of the backward pass (keys per CTA stay 128).
constexpr int FB_BM = 64;
constexpr int FB_QT = 64 * 64 * 2;  // one 64-row x 64-col swizzled chunk (8 KB)
// smem: K(2 chunks) V(2) | Q ring FB_QD x 2 chunks(8K) | dO ring FB_QD x 2 | dS^T [2 slots][128x64]
// | lse / delta ring | dQ staging. The Q/dO ring is 3 deep so the loads of a query tile are issued one
// tile earlier than a 2-deep ring allows (a slot frees only when the gradient MMAs of its tile finish,
// which follow that tile's softmax). P^T stays in TMEM (the dP^T columns of its buffer) as the A
// operand of the dV MMA; dS^T, needed as an operand in shared memory by the dK and dQ MMAs, has two
// slots, so the softmax of tile t only waits for the MMAs of tile t-2 (keeping P^T out of shared
// memory removes its 16 KB write and the dV MMA's 16 KB of A reads per tile; the 128 x 64 x 16 MMAs
// are limited by their instruction rate, ~69 cycles each, more than by operand bandwidth). 227 KB.
constexpr int FB_QD = 3;
constexpr int FB_DQ_BYTES = 64 * 128 * 4;  // fp32 dQ staging tile [64 q][128 d]
constexpr int FA_BWD_SMEM =
    4 * FA_TILE + 2 * FB_QD * 2 * FB_QT + 2 * FA_TILE + 2 * FB_QD * 64 * 4 + FB_DQ_BYTES + 1024 + 512;
static_assert(FA_BWD_SMEM <= 227 * 1024, "flash backward exceeds the shared memory of one CTA");
constexpr int FB_THREADS = 320;

__global__ void __launch_bounds__(FB_THREADS, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                     const __grid_constant__ CUtensorMap tmdQ, FlashBwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;                   // 2 chunks [128 keys][64 d]
  uint8_t* sV = sK + 2 * FA_TILE;       // 2 chunks
  uint8_t* sQ = sV + 2 * FA_TILE;              // [FB_QD slots][2 chunks][64 q][64 d]
  uint8_t* sdO = sQ + FB_QD * 2 * FB_QT;       // same
  uint8_t* sdS = sdO + FB_QD * 2 * FB_QT;      // [2 slots][128 keys][64 q] dS^T (P^T lives in TMEM)
  float* sLse = reinterpret_cast<float*>(sdS + 2 * FA_TILE);  // [FB_QD][64] log2 units
  float* sDelta = sLse + FB_QD * 64;                       // [FB_QD][64]
  float* sdQ = sDelta + FB_QD * 64;                        // [64][128] fp32 staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sdQ) + FB_DQ_BYTES);
  // TMEM: two score buffers of 128 columns (S^T in the first 64, dP^T in the
  // next 64), dV at 256, dK at 384. Iteration `it` uses buffer it & 1; its dQ^T
  // (64 columns) is written over its own S^T once the softmax has read it, and
  // the buffer is free again when the dQ warps have drained dQ^T. So the S/dP
  // MMAs of the next query tile run while this tile's softmax works.
  uint64_t* kv_full = bars;                   // K, V loaded
  uint64_t* qd_full = bars + 1;               // [FB_QD] Q/dO slot loaded (+ stats written)
  uint64_t* qd_empty = qd_full + FB_QD;       // [FB_QD] dV/dK MMAs done with the slot
  uint64_t* sd_full = qd_empty + FB_QD;       // [2] S^T and dP^T of buffer i in TMEM
  uint64_t* ps_ready = sd_full + 2;           // [2] P^T/dS^T of tile t in smem, buffer t & 1 read (4 warps)
  uint64_t* dq_full = ps_ready + 2;           // [2] dQ^T in buffer i; all MMAs of the tile done
  uint64_t* dq_free = dq_full + 2;            // [2] dQ^T of buffer i read out (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_free + 2);

  const int warp = warp_id(), lane = lane_id();
  // 1-D grid in longest-first order: with a causal mask key block 0 sees every
  // query tile, the last one the fewest, so block nb = rank of the work size
  const int hb = p.Hkv * p.B;
  const int nb = (int)(blockIdx.x / hb);
  const int hk = (int)(blockIdx.x % hb) % p.Hkv, b = (int)(blockIdx.x % hb) / p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int n0 = nb * FA_BN;
  const int off = p.Sk - p.Sq;
  const int n_mblocks = (p.Sq + FB_BM - 1) / FB_BM;
  int mb_first = 0;
  if (p.causal) mb_first = max(0, (n0 - off) / FB_BM);
  const int per_head = max(0, n_mblocks - mb_first);
  const int iters = G * per_head;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < FB_QD; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dq_full[i], 1);
      mbar_init(&sd_full[i], 1);
      mbar_init(&ps_ready[i], 4);
      mbar_init(&dq_free[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tdV = tmem + 256, tdK = tmem + 384;
  // buffer i: S^T at tmem + 128 i (also dQ^T), dP^T at tmem + 128 i + 64

  if (warp == 0) {
    // ---------------------------------------------------------- loads
    if (lane == 0 && iters > 0) {
      mbar_expect_tx(kv_full, 4 * FA_TILE);
      tma_load_3d(sK, &tmK, kv_full, p.k_col0 + hk * FA_D, n0, b);
      tma_load_3d(sK + FA_TILE, &tmK, kv_full, p.k_col0 + hk * FA_D + 64, n0, b);
      tma_load_3d(sV, &tmV, kv_full, p.v_col0 + hk * FA_D, n0, b);
      tma_load_3d(sV + FA_TILE, &tmV, kv_full, p.v_col0 + hk * FA_D + 64, n0, b);
    }
    for (int it = 0; it < iters; ++it) {
      const int slot = it % FB_QD;
      const int h = hk * G + it / per_head;
      const int m0 = (mb_first + it % per_head) * FB_BM;
      // slot reuse: qd_empty(it - FB_QD) follows the dV/dK MMAs of that tile, which were
      // issued after its softmax (the stats reader) arrived on ps_ready
      if (lane == 0 && it >= FB_QD &&
          !mbar_wait(&qd_empty[slot], ((it / FB_QD) - 1) & 1, p.err, kErrWaitEmpty))
        break;
      if (lane == 0) {
        mbar_expect_tx(&qd_full[slot], 4 * FB_QT + 2 * 64 * 4);
        const long long so = ((long long)b * p.Hq + h) * p.Sq_pad + m0;
        bulk_load(sLse + slot * 64, p.lse2 + so, 256, &qd_full[slot]);
        bulk_load(sDelta + slot * 64, p.delta + so, 256, &qd_full[slot]);
        uint8_t* q = sQ + slot * 2 * FB_QT;
        uint8_t* d = sdO + slot * 2 * FB_QT;
        tma_load_3d(q, &tmQ, &qd_full[slot], p.q_col0 + h * FA_D, m0, b);
        tma_load_3d(q + FB_QT, &tmQ, &qd_full[slot], p.q_col0 + h * FA_D + 64, m0, b);
        tma_load_3d(d, &tmdO, &qd_full[slot], p.do_col0 + h * FA_D, m0, b);
        tma_load_3d(d + FB_QT, &tmdO, &qd_full[slot], p.do_col0 + h * FA_D + 64, m0, b);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && iters > 0) {
      constexpr uint32_t idSP = idesc_bf16(128, 64, 0, 0);   // S^T, dP^T : K/V x Q/dO (both K-major)
      constexpr uint32_t idGR = idesc_bf16(128, 128, 0, 1);  // dV, dK    : P^T/dS^T K-major, dO/Q MN-major
      constexpr uint32_t idDQ = idesc_bf16(128, 64, 1, 1);   // dQ^T      : K^T MN-major, dS^T MN-major
      bool ok = mbar_wait(kv_full, 0, p.err, kErrWaitFull);
      // Descriptors are built once; a K step only advances the start-address field (16-byte units,
      // no carry: shared addresses stay below 2^18 bytes). The 128x64x16 MMAs of this kernel last
      // ~32 tensor-core cycles each and the issuing warp shares its SM sub-partition with a softmax
      // and a dQ warp, so building two descriptors per MMA left the tensor core waiting on issue.
      const uint64_t dK_k = sdesc_sw128(smem_u32(sK), 16, 1024);         // K as A, K-major
      const uint64_t dV_k = sdesc_sw128(smem_u32(sV), 16, 1024);         // V as A, K-major
      const uint64_t dK_mn = sdesc_sw128(smem_u32(sK), FA_TILE, 1024);   // K^T as A, MN-major
      uint64_t dS_k[2], dS_mn[2];  // dS^T slot i as A (K-major) / as B (MN-major)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        dS_k[i] = sdesc_sw128(smem_u32(sdS + i * FA_TILE), 16, 1024);
        dS_mn[i] = sdesc_sw128(smem_u32(sdS + i * FA_TILE), 2 * FA_TILE, 1024);
      }
      uint64_t dQ_k[FB_QD], dO_k[FB_QD], dQ_mn[FB_QD], dO_mn[FB_QD];
#pragma unroll
      for (int i = 0; i < FB_QD; ++i) {
        const uint32_t qb = smem_u32(sQ + i * 2 * FB_QT), ob = smem_u32(sdO + i * 2 * FB_QT);
        dQ_k[i] = sdesc_sw128(qb, 16, 1024);
        dO_k[i] = sdesc_sw128(ob, 16, 1024);
        dQ_mn[i] = sdesc_sw128(qb, FB_QT, 1024);
        dO_mn[i] = sdesc_sw128(ob, FB_QT, 1024);
      }
      // slot-indexed descriptors by selects, so the arrays stay in registers
      auto pick = [](const uint64_t (&a)[FB_QD], int i) { return i == 0 ? a[0] : (i == 1 ? a[1] : a[2]); };
      static_assert(FB_QD == 3, "pick() covers three slots");
      auto issue_grads = [&](int it) -> bool {
        // dV += P^T dO ; dK += dS^T Q   (M = keys, N = d, K = 64 queries)
        const int slot = it & 1, qs = it % FB_QD;
        const uint64_t bo = pick(dO_mn, qs), bq = pick(dQ_mn, qs);
        // P^T of this iteration sits in TMEM (the dP^T columns of its buffer, bf16 pairs): the dV MMA
        // takes it as the A operand, so only dO is read from shared memory
        const uint32_t tP = tmem + slot * 128 + 64;
#pragma unroll
        for (int k = 0; k < FB_BM / 16; ++k) {
          umma_bf16_ts(tdV, tP + (uint32_t)(k * 8), bo + (uint64_t)(k * 128), idGR, (it | k) != 0);
          umma_bf16(tdK, (slot ? dS_k[1] : dS_k[0]) + (uint64_t)(k * 2), bq + (uint64_t)(k * 128), idGR, (it | k) != 0);
        }
        umma_commit(&qd_empty[qs]);
        // dQ^T = K^T dS^T  (M = d, N = 64 queries, K = 128 keys) over this iteration's S^T,
        // which the softmax has read (ps_ready waited by the caller)
#pragma unroll
        for (int k = 0; k < FA_BN / 16; ++k)
          umma_bf16(tmem + slot * 128, dK_mn + (uint64_t)(k * 128), (slot ? dS_mn[1] : dS_mn[0]) + (uint64_t)(k * 128), idDQ, k > 0);
        umma_commit(&dq_full[slot]);
        return true;
      };
      for (int it = 0; it < iters && ok; ++it) {
        const int slot = it & 1, qs = it % FB_QD;
        ok = mbar_wait(&qd_full[qs], (it / FB_QD) & 1, p.err, kErrWaitFull);
        // buffer `slot` is free once the dQ^T of it-2 (written over its S^T) was drained
        if (ok && it >= 2) ok = mbar_wait(&dq_free[slot], ((it - 2) >> 1) & 1, p.err, kErrWaitAccEmpty);
        if (!ok) break;
        tc_fence_after();
        const uint64_t bq = pick(dQ_k, qs), bo = pick(dO_k, qs);
        const uint32_t tS = tmem + slot * 128, tdP = tS + 64;
        // S^T = K Q^T ; dP^T = V dO^T   (M = 128 keys, N = 64 queries, K = d)
#pragma unroll
        for (int k = 0; k < FA_D / 16; ++k) {
          const uint64_t o = (uint64_t)(((k >> 2) * FA_TILE + (k & 3) * 32) >> 4);
          const uint64_t oq = (uint64_t)(((k >> 2) * FB_QT + (k & 3) * 32) >> 4);
          umma_bf16(tS, dK_k + o, bq + oq, idSP, k > 0);
          umma_bf16(tdP, dV_k + o, bo + oq, idSP, k > 0);
        }
        umma_commit(&sd_full[slot]);
        // gradients of it-1 once its softmax is done; they overlap the softmax of it
        if (it >= 1) {
          ok = mbar_wait(&ps_ready[slot ^ 1], ((it - 1) >> 1) & 1, p.err, kErrWaitAccEmpty);
          if (ok) {
            tc_fence_after();
            ok = issue_grads(it - 1);
          }
        }
      }
      if (ok && mbar_wait(&ps_ready[(iters - 1) & 1], ((iters - 1) >> 1) & 1, p.err, kErrWaitAccEmpty)) {
        tc_fence_after();
        issue_grads(iters - 1);
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------- softmax warps: P^T, dS^T
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // key row in block == TMEM lane
    const int ki = n0 + r;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int seg_k = (p.seg && ki < p.Sk) ? p.seg[(long long)b * p.Sk + ki] : 0;
    bool ok = true;
    for (int it = 0; it < iters; ++it) {
      const int slot = it & 1, qs = it % FB_QD;
      const int m0 = (mb_first + it % per_head) * FB_BM;
      ok = mbar_wait(&sd_full[slot], (it >> 1) & 1, p.err, kErrWaitAccFull) &&
           mbar_wait(&qd_full[qs], (it / FB_QD) & 1, p.err, kErrWaitAccFull);
      if (!ok) break;
      tc_fence_after();
      // visible query columns of this key row, as a 64-bit mask
      uint32_t vis[2];
      {
        const int lo = p.causal ? ki - off - m0 : 0;  // first visible column
        const int hi = min(FB_BM, p.Sq - m0);         // one past the last
        row_mask64(ki < p.Sk ? lo : FB_BM, hi, vis);
        if (p.seg) {
#pragma unroll 1
          for (int c = 0; c < FB_BM; ++c) {
            const int qi = m0 + c;
            if (qi < p.Sq && p.seg[(long long)b * p.Sk + qi + off] != seg_k) vis[c >> 5] &= ~(1u << (c & 31));
          }
        }
      }
      const uint32_t lse_a = smem_u32(sLse + qs * 64), dlt_a = smem_u32(sDelta + qs * 64);
      const uint32_t dc = smem_u32(sdS + slot * FA_TILE);
      uint32_t sv[64], dpv[64];
      const uint32_t tS = tmem + slot * 128, tdP = tS + 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(tS + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
        tmem_ld32(tdP + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&dpv[c * 32]));
      }
      tmem_wait_ld();
      uint32_t pk[2][16], dk[2][16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t* s = &sv[c * 32];
        const uint32_t* dp = &dpv[c * 32];
        float lse2[32], dlt[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ld_shared_v4f(lse_a + (c * 32 + 4 * j) * 4, lse2[4 * j], lse2[4 * j + 1], lse2[4 * j + 2], lse2[4 * j + 3]);
          ld_shared_v4f(dlt_a + (c * 32 + 4 * j) * 4, dlt[4 * j], dlt[4 * j + 1], dlt[4 * j + 2], dlt[4 * j + 3]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float pv[2], dsv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int qc = c * 32 + 2 * i + e;
            float pr = ex2(fmaf(__uint_as_float(s[2 * i + e]), p.scale_log2, -lse2[2 * i + e]));
            pr = ((vis[qc >> 5] >> (qc & 31)) & 1u) ? pr : 0.f;
            pv[e] = pr;
            dsv[e] = pr * (__uint_as_float(dp[2 * i + e]) - dlt[2 * i + e]) * p.scale;
          }
          pk[c][i] = pack_bf16(pv[0], pv[1]);
          dk[c][i] = pack_bf16(dsv[0], dsv[1]);
        }
      }
      // P^T into the dP^T columns of this buffer (already read into registers): bf16 pairs, the A operand
      // of the dV MMA
      tmem_st16(tdP + lane_off, pk[0]);
      tmem_st16(tdP + 16 + lane_off, pk[1]);
      // dS^T slot it & 1 was last read by the gradient MMAs of it-2: wait only now, so this tile's math
      // overlapped them
      if (it >= 2 && !mbar_wait(&dq_full[slot], ((it - 2) >> 1) & 1, p.err, kErrWaitAccFull)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int g = 0; g < 4; ++g)
          st_shared_v4(swz(dc, r, c * 4 + g), dk[c][4 * g], dk[c][4 * g + 1], dk[c][4 * g + 2], dk[c][4 * g + 3]);
      }
      tmem_wait_st();
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ps_ready[slot]);
    }
    // final dK / dV: TMEM rows -> bf16 global (after the last iteration's MMAs)
    if (ok && iters > 0 && mbar_wait(&dq_full[(iters - 1) & 1], ((iters - 1) >> 1) & 1, p.err, kErrWaitAccFull)) {
      tc_fence_after();
      const bool row_ok = ki < p.Sk;
      __nv_bfloat16* dkrow = p.dk + ((long long)b * p.Sk + ki) * p.ld_dkv + p.dk_col0 + hk * FA_D;
      __nv_bfloat16* dvrow = p.dv + ((long long)b * p.Sk + ki) * p.ld_dkv + p.dv_col0 + hk * FA_D;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t a[32], bb[32];
        tmem_ld32(tdK + lane_off + c * 32, a);
        tmem_ld32(tdV + lane_off + c * 32, bb);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            reinterpret_cast<uint4*>(dkrow + c * 32)[g] =
                make_uint4(pack_bf16(__uint_as_float(a[8 * g]), __uint_as_float(a[8 * g + 1])),
                           pack_bf16(__uint_as_float(a[8 * g + 2]), __uint_as_float(a[8 * g + 3])),
                           pack_bf16(__uint_as_float(a[8 * g + 4]), __uint_as_float(a[8 * g + 5])),
                           pack_bf16(__uint_as_float(a[8 * g + 6]), __uint_as_float(a[8 * g + 7])));
            reinterpret_cast<uint4*>(dvrow + c * 32)[g] =
                make_uint4(pack_bf16(__uint_as_float(bb[8 * g]), __uint_as_float(bb[8 * g + 1])),
                           pack_bf16(__uint_as_float(bb[8 * g + 2]), __uint_as_float(bb[8 * g + 3])),
                           pack_bf16(__uint_as_float(bb[8 * g + 4]), __uint_as_float(bb[8 * g + 5])),
                           pack_bf16(__uint_as_float(bb[8 * g + 6]), __uint_as_float(bb[8 * g + 7])));
          }
        }
      }
    } else if (iters == 0 && ki < p.Sk) {
      __nv_bfloat16* dkrow = p.dk + ((long long)b * p.Sk + ki) * p.ld_dkv + p.dk_col0 + hk * FA_D;
      __nv_bfloat16* dvrow = p.dv + ((long long)b * p.Sk + ki) * p.ld_dkv + p.dv_col0 + hk * FA_D;
      for (int c = 0; c < FA_D; ++c) {
        dkrow[c] = __float2bfloat16_rn(0.f);
        dvrow[c] = __float2bfloat16_rn(0.f);
      }
    }
  } else {
    // ---------------------------------------------------------- dQ epilogue warps
    // TMEM lane = head-dim index d, column = query in tile. The tile is staged
    // in smem as [64 q][128 d] fp32 and added into the fp32 dQ accumulator by
    // one TMA bulk reduce-add (the TMA unit does the atomic accumulation).
    const int q4 = warp & 3;
    const int d = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t sdq_a = smem_u32(sdQ);
    for (int it = 0; it < iters; ++it) {
      const int h = hk * G + it / per_head;
      const int m0 = (mb_first + it % per_head) * FB_BM;
      if (!mbar_wait(&dq_full[it & 1], (it >> 1) & 1, p.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const uint32_t tdQ = tmem + (it & 1) * 128;
      uint32_t v[64];
      tmem_ld32(tdQ + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tdQ + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      // dQ^T is drained from TMEM: the buffer can take the next S^T / dP^T
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[it & 1]);
      // staging buffer must be free: the previous bulk reduce finished reading it
      if (it > 0) {
        if (warp == 6 && lane == 0) bulk_wait_read0();
        named_bar_sync(1, 128);
      }
#pragma unroll
      for (int i = 0; i < 64; ++i) st_shared_f32(sdq_a + (i * 128 + d) * 4, __uint_as_float(v[i]));
      fence_async_smem();
      named_bar_sync(1, 128);
      if (warp == 6 && lane == 0) {
        tma_reduce_add_3d(&tmdQ, sdQ, h * FA_D, m0, b);
        bulk_commit();
      }
    }
    if (warp == 6 && lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Backward preprocessing, one warp per query row (all heads of the row):
//   delta[b, h, s] = sum_d dO[b*S+s, h*D+d] * O[b*S+s, h*D+d]
//   lse2[b, h, s]  = lse * log2(e)  (+inf for empty rows)
// Both arrays are padded to Sq_pad (lse2 = +inf, delta = 0 in the padding) so
// the main kernel fetches whole 64-query tiles with bulk copies. Each lane
// loads 16-byte vectors; 16 lanes cover one 128-wide head, so a warp reduces
// two heads per step with 4 shuffles.
__global__ void flash_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dO, long long ld_do, int do_col0,
                                     const __nv_bfloat16* __restrict__ O, long long ldo,
                                     const float* __restrict__ lse, float* __restrict__ lse2,
                                     float* __restrict__ delta, int B, int S, int S_pad, int H,
                                     float* __restrict__ dq_acc, int dq_width) {
  // One warp per (batch, query row padded to 64-query tiles): delta = rowsum(dO * O) per head and
  // lse2 = lse * log2(e) (padding rows get 0 and +inf), and the row's fp32 dQ accumulator is zeroed
  // (the main kernel reduce-adds into it). The loads of four heads (two per half-warp) are issued
  // before their reductions.
  const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)B * S_pad) return;
  const int b = (int)(w / S_pad), si = (int)(w % S_pad);
  const int half = lane >> 4, sub = lane & 15;
  if (si < S && dq_acc != nullptr) {
    float4* z = reinterpret_cast<float4*>(dq_acc + ((long long)b * S + si) * dq_width);
    for (int c = lane; c < dq_width / 4; c += 32) z[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const long long row = (long long)b * S + si;
  for (int h0 = 0; h0 < H; h0 += 4) {
    uint4 ua[2], uo[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int h = h0 + 2 * k + half;
      if (si < S && h < H) {
        ua[k] = *reinterpret_cast<const uint4*>(dO + row * ld_do + do_col0 + h * FA_D + sub * 8);
        uo[k] = *reinterpret_cast<const uint4*>(O + row * ldo + h * FA_D + sub * 8);
      } else {
        ua[k] = uo[k] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int h = h0 + 2 * k + half;
      const uint32_t a4[4] = {ua[k].x, ua[k].y, ua[k].z, ua[k].w}, o4[4] = {uo[k].x, uo[k].y, uo[k].z, uo[k].w};
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack_bf16(a4[j]), o = unpack_bf16(o4[j]);
        sum = fmaf(a.x, o.x, fmaf(a.y, o.y, sum));
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, off);
      if (sub == 0 && h < H) {
        const long long out = ((long long)b * H + h) * S_pad + si;
        if (si >= S) {
          delta[out] = 0.f;
          lse2[out] = INFINITY;
        } else {
          delta[out] = sum;
          const float ls = lse[((long long)b * H + h) * S + si];
          lse2[out] = (ls == -INFINITY) ? INFINITY : ls * 1.4426950408889634f;
        }
      }
    }
  }
}

// dq_out[row, col0 + c] = bf16(dq_acc[row, c]): blocks walk rows, each thread converts two float4s
// of a row per pass (both loads issued first), no index division
__global__ void flash_dq_convert_kernel(const float* __restrict__ acc, int width, long long rows,
                                        __nv_bfloat16* __restrict__ out, long long ld_out, int col0) {
  const int nv = width / 4, T = blockDim.x;
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    const float4* src = reinterpret_cast<const float4*>(acc + row * width);
    __nv_bfloat16* dst = out + row * ld_out + col0;
    for (int c0 = threadIdx.x; c0 < nv; c0 += 2 * T) {
      float4 v[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) v[k] = c0 + k * T < nv ? src[c0 + k * T] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = c0 + k * T;
        if (c < nv)
          *reinterpret_cast<uint2*>(dst + 4 * c) = make_uint2(pack_bf16(v[k].x, v[k].y), pack_bf16(v[k].z, v[k].w));
      }
    }
  }
}

}  // namespace astrai

namespace astrai_host {
using namespace astrai;

// 3-D map over a [B][S][cols] bf16 buffer with row stride `ld` (elements):
// box = 64 columns x 128 rows x 1 batch, 128-byte swizzle.
static void make_rows_map(CUtensorMap* m, const void* base, int B, int S, long long ld, uint32_t rows = 128) {
  uint64_t dims[3] = {(uint64_t)ld, (uint64_t)S, (uint64_t)B};
  uint64_t strides[2] = {(uint64_t)ld * 2, (uint64_t)S * ld * 2};
  uint32_t box[3] = {64, rows, 1};
  make_tmap_bf16(m, base, 3, dims, strides, box, true);
}

void flash_fwd(const void* q, long long ldq, int q_col0, const void* k, long long ldk, int k_col0, const void* v,
               long long ldv, int v_col0, void* o, long long ldo, float* lse, int B, int Sq, int Sk, int Hq, int Hkv,
               float scale, int causal, const int* seg, cudaStream_t s) {
  CUtensorMap tq, tk, tv;
  make_rows_map(&tq, q, B, Sq, ldq);
  make_rows_map(&tk, k, B, Sk, ldk);
  make_rows_map(&tv, v, B, Sk, ldv);
  FlashFwdParams p;
  p.B = B;
  p.Sq = Sq;
  p.Sk = Sk;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.q_col0 = q_col0;
  p.k_col0 = k_col0;
  p.v_col0 = v_col0;
  p.O = static_cast<__nv_bfloat16*>(o);
  p.ldo = ldo;
  p.lse = lse;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.seg = seg;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = error_word(dev);
  static bool attr[64] = {false};
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_FWD_SMEM);
    attr[dev & 63] = true;
  }
  const unsigned grid = (unsigned)((Sq + FA_BM - 1) / FA_BM) * Hq * B;
  (astrai::note_launch(), flash_fwd_kernel<<<grid, 192, FA_FWD_SMEM, s>>>(tq, tk, tv, p));
}

void flash_bwd(const void* q, long long ldq, int q_col0, const void* k, long long ldk, int k_col0, const void* v,
               long long ldv, int v_col0, const void* o, long long ldo, const void* dO, long long ld_do, int do_col0,
               const float* lse, float* delta, float* dq_acc, void* dq, long long ld_dq, int dq_col0, void* dk,
               void* dv, long long ld_dkv, int dk_col0, int dv_col0, int B, int Sq, int Sk, int Hq, int Hkv,
               float scale, int causal, const int* seg, cudaStream_t s) {
  // 1) delta = rowsum(dO * O), lse2 = lse * log2(e); both padded to 64-query tiles
  if (ld_do % 8 || do_col0 % 8 || ldo % 8 || reinterpret_cast<uintptr_t>(dO) % 16 ||
      reinterpret_cast<uintptr_t>(o) % 16)
    throw std::runtime_error("flash_bwd: dO / O need 16-byte aligned rows");
  const int Sq_pad = (Sq + FB_BM - 1) / FB_BM * FB_BM;
  float* lse2 = delta + (long long)B * Hq * Sq_pad;
  {
    const long long warps = (long long)B * Sq_pad;  // one warp per query row
    const int blocks = (int)((warps * 32 + 255) / 256);
    (astrai::note_launch(), flash_bwd_pre_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(dO), ld_do, do_col0,
                                                static_cast<const __nv_bfloat16*>(o), ldo, lse, lse2, delta, B, Sq,
                                                Sq_pad, Hq, dq_acc, Hq * FA_D));
  }
  // 2) main kernel
  CUtensorMap tq, tk, tv, tdo;
  make_rows_map(&tq, q, B, Sq, ldq, FB_BM);
  make_rows_map(&tk, k, B, Sk, ldk);
  make_rows_map(&tv, v, B, Sk, ldv);
  make_rows_map(&tdo, dO, B, Sq, ld_do, FB_BM);
  FlashBwdParams p;
  p.B = B;
  p.Sq = Sq;
  p.Sk = Sk;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.q_col0 = q_col0;
  p.k_col0 = k_col0;
  p.v_col0 = v_col0;
  p.do_col0 = do_col0;
  p.lse2 = lse2;
  p.delta = delta;
  p.Sq_pad = Sq_pad;
  p.dq_acc = dq_acc;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.ld_dkv = ld_dkv;
  p.dk_col0 = dk_col0;
  p.dv_col0 = dv_col0;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.seg = seg;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = error_word(dev);
  static bool attr[64] = {false};
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_BWD_SMEM);
    attr[dev & 63] = true;
  }
  const unsigned grid = (unsigned)((Sk + FA_BN - 1) / FA_BN) * Hkv * B;
  CUtensorMap tdq;
  {
    uint64_t dims[3] = {(uint64_t)Hq * FA_D, (uint64_t)Sq, (uint64_t)B};
    uint64_t strides[2] = {(uint64_t)Hq * FA_D * 4, (uint64_t)Sq * Hq * FA_D * 4};
    uint32_t box[3] = {FA_D, FB_BM, 1};
    make_tmap_f32(&tdq, dq_acc, 3, dims, strides, box);
  }
  (astrai::note_launch(), flash_bwd_kernel<<<grid, FB_THREADS, FA_BWD_SMEM, s>>>(tq, tk, tv, tdo, tdq, p));
  // 3) dQ fp32 -> bf16 into its destination columns
  {
    const long long rows = (long long)B * Sq;
    const int width = Hq * FA_D;
    const int blocks = (int)std::max(1LL, std::min<long long>(rows, (long long)num_sms(dev) * 8));
    (astrai::note_launch(), flash_dq_convert_kernel<<<blocks, 256, 0, s>>>(dq_acc, width, rows, static_cast<__nv_bfloat16*>(dq), ld_dq,
                                                   dq_col0));
  }
}

}  // namespace astrai_host
