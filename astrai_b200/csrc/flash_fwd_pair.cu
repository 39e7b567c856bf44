// Flash-attention forward with two query tiles per CTA and P kept in tensor memory (sm_100a).
//
// Same contract as flash_fwd_kernel (attention.cu: q/k/v read by TMA out of the fused QKV
// projection, O written in the [tokens, Hq*D] layout of the o-projection, fp32 LSE, optional
// segment ids, causal offset Sk - Sq), for head_dim D = 64 or 128. It replaces SDPA + repeat_kv of
// the reference's attention (astrai/model/components/attention.py:15-23, :96-101).
//
// One CTA owns two 128-query tiles that read the same K/V blocks: two query heads of one GQA
// group at the same rows (Hq/Hkv even), otherwise two consecutive row blocks of one head. K/V are
// loaded once per block for both tiles. Roles:
//   warp 0      TMA: Q0, Q1 once; K_j and V_j into a ring of STAGES slots
//   warp 1      TMEM owner + MMA issuer (one elected thread), per key block j:
//                 PV0_{j-1}, S0_j, PV1_{j-1}, S1_j  with  S_i = Q_i K_j^T  (smem x smem -> TMEM)
//                 and O_i += P_i V_j  with P_i read from TMEM as the A operand (tcgen05.mma [a-tmem])
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1; one query row per thread: row max
//               from TMEM, lazy rescale of O_i (only when the running max grows by more than 2^8),
//               P = exp2(S*scale*log2e - m) packed to bf16 and stored back into TMEM over the upper
//               half of S_i's columns, then the final O / l and the log-sum-exp.
// While one softmax group works on its tile, the tensor cores run the other tile's PV and S MMAs,
// so the exponentials and the MMAs overlap; P never goes through shared memory.
//
// Ordering facts the pipeline relies on: tcgen05.mma operations issued by one thread execute in
// issue order, and tcgen05.commit tracks every earlier tcgen05 operation of that thread. So when
// the softmax of tile i sees S_i(j) complete, PV_i(j-1) (issued before S_i(j)) is complete too: O_i
// may be rescaled and P_i's columns may be overwritten without another barrier.
//
// TMEM (512 columns): S0 [0,128), S1 [128,256) (P_i over columns 64..127 of S_i), O0 at 256, O1 at
// 256 + D. Every wait is time-bounded (common.cuh).
#include <cfloat>
#include <cstdlib>
#include <stdexcept>

#include "common.cuh"

namespace astrai {
namespace {

struct PairFwdParams {
  int B, Sq, Sk, Hq, Hkv;
  int q_col0, k_col0, v_col0;  // column of head 0 inside each tensor map's buffer
  __nv_bfloat16* O;
  long long ldo;
  float* lse;  // [B, Hq, Sq] natural-log LSE
  float scale_log2;
  int causal;
  const int* seg;   // optional [B, Sk] segment ids
  int pair_heads;   // 1: tiles are heads (h, h+1) at rows m0; 0: rows (m0, m0+128) of head h
  int* err;
};

template <int D>
struct PairCfg {
  static constexpr int CHUNK = 128 * 64 * 2;  // one 128-row x 64-column swizzled chunk (16 KB)
  static constexpr int CH = D / 64;           // chunks per 128-row tile
  static constexpr int TILE = CH * CHUNK;
  static constexpr int STAGES = D == 64 ? 4 : 2;
  static constexpr int SMEM = (2 + 2 * STAGES) * TILE + 1024 + 256;
  static_assert(SMEM <= 227 * 1024, "flash_fwd_pair exceeds the shared memory of one CTA");
};

constexpr int kPairThreads = 320;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for x <= 0, so that part of the softmax's exponentials leave the MUFU unit
// (16 exponentials per clock per SM on sm_100, which a two-tile CTA saturates). x = n + f with
// n = floor(x): adding 1.5 * 2^23 with round-down leaves n in the low mantissa bits; 2^f on [0, 1) is
// 1 + c1 f + c2 f^2 + c3 f^3 (relative-error least-squares fit with Lawson reweighting, max relative
// error 8.6e-5, below bf16 resolution); n goes into the exponent field (exponent-field construction as
// in Schraudolph, 1999). x < -127 (masked scores) gives 0.
__device__ __forceinline__ float exp2_poly(float x) {
  const float xc = fmaxf(x, -127.f);
  const float t = __fadd_rd(xc, 12582912.f);
  const float n = t - 12582912.f;
  const float f = xc - n;
  const float p = fmaf(fmaf(fmaf(0.07706134f, f, 0.22765121f), f, 0.69511539f), f, 1.f);
  const int ni = __float_as_int(t) - 0x4B400000;
  const float y = __int_as_float(__float_as_int(p) + (ni << 23));
  return x < -127.f ? 0.f : y;
}

// Packed fp32 pairs (sm_100 f32x2 instructions): two lanes of work per issued instruction.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// three-input maximum (sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// bits [0, hi) of a 128-bit row mask held as four words
__device__ __forceinline__ void mask_upto(int hi, uint32_t (&m)[4]) {
  hi = max(0, min(128, hi));
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int b = max(0, min(32, hi - 32 * w));
    m[w] = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
  }
}

// EMU: of every 16 exponential pairs of a 32-column chunk, this many are computed by exp2_poly
template <int D, int EMU>
__global__ void __launch_bounds__(kPairThreads, 1)
    flash_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, PairFwdParams p) {
  using Cfg = PairCfg<D>;
  constexpr int ST = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // [2 tiles]
  uint8_t* sK = sQ + 2 * Cfg::TILE;        // [ST]
  uint8_t* sV = sK + ST * Cfg::TILE;       // [ST]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * Cfg::TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;            // [ST]
  uint64_t* k_empty = k_full + ST;        // [ST] both S MMAs of the block done
  uint64_t* v_full = k_empty + ST;        // [ST]
  uint64_t* v_empty = v_full + ST;        // [ST] both PV MMAs of the block done
  uint64_t* s_full = v_empty + ST;        // [2] S_i(j) in TMEM
  uint64_t* p_ready = s_full + 2;         // [2] P_i(j) in TMEM (4 warps arrive)
  uint64_t* pv_done = p_ready + 2;        // [2] PV_i(j) done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);

  const int warp = warp_id(), lane = lane_id();
  const int G = p.Hq / p.Hkv;
  const int n_mblocks = (p.Sq + 127) / 128;
  // 1-D grid, heaviest units first (the causal row blocks of the last positions see the most keys)
  int h0, h1, m00, m01, b;
  if (p.pair_heads) {
    const int per = p.B * (p.Hq / 2);
    const int mb = n_mblocks - 1 - (int)(blockIdx.x / per);
    const int rest = (int)(blockIdx.x % per);
    h0 = 2 * (rest % (p.Hq / 2));
    h1 = h0 + 1;
    b = rest / (p.Hq / 2);
    m00 = m01 = mb * 128;
  } else {
    const int per = p.B * p.Hq;
    const int n_pairs = (n_mblocks + 1) / 2;
    const int mp = n_pairs - 1 - (int)(blockIdx.x / per);
    const int rest = (int)(blockIdx.x % per);
    h0 = h1 = rest % p.Hq;
    b = rest / p.Hq;
    m00 = mp * 256;
    m01 = m00 + 128;
  }
  const int hk = h0 / G;
  const int off = p.Sk - p.Sq;  // queries are the last Sq positions
  const int last_row = min(max(m00, m01) + 127, p.Sq - 1);
  int n_blocks = (p.Sk + 127) / 128;
  if (p.causal) n_blocks = min(n_blocks, max(0, (last_row + off) / 128 + 1));

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && n_blocks > 0) {
      mbar_expect_tx(q_full, 2 * Cfg::TILE);
#pragma unroll
      for (int c = 0; c < Cfg::CH; ++c) {
        tma_load_3d(sQ + c * Cfg::CHUNK, &tmQ, q_full, p.q_col0 + h0 * D + c * 64, m00, b);
        tma_load_3d(sQ + Cfg::TILE + c * Cfg::CHUNK, &tmQ, q_full, p.q_col0 + h1 * D + c * 64, m01, b);
      }
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j % ST;
        const uint32_t par = ((j / ST) & 1) ^ 1;
        if (!mbar_wait(&k_empty[st], par, p.err, kErrWaitEmpty)) break;
        mbar_expect_tx(&k_full[st], Cfg::TILE);
        uint8_t* k = sK + st * Cfg::TILE;
#pragma unroll
        for (int c = 0; c < Cfg::CH; ++c)
          tma_load_3d(k + c * Cfg::CHUNK, &tmK, &k_full[st], p.k_col0 + hk * D + c * 64, j * 128, b);
        if (!mbar_wait(&v_empty[st], par, p.err, kErrWaitEmpty)) break;
        mbar_expect_tx(&v_full[st], Cfg::TILE);
        uint8_t* v = sV + st * Cfg::TILE;
#pragma unroll
        for (int c = 0; c < Cfg::CH; ++c)
          tma_load_3d(v + c * Cfg::CHUNK, &tmV, &v_full[st], p.v_col0 + hk * D + c * 64, j * 128, b);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && n_blocks > 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);  // S = Q K^T, both K-major
      constexpr uint32_t idO = idesc_bf16(128, D, 0, 1);    // O += P V, V MN-major
      // Descriptors are built once; a K step only advances the 14-bit start-address field (in 16-byte
      // units, no carry: shared addresses stay below 2^18 bytes), so each MMA costs a few instructions.
      // The issuing warp shares its SM sub-partition with two softmax warps, and a 128x128x16 MMA
      // lasts only ~64 tensor-core cycles, so issue cost decides whether the tensor core waits.
      uint64_t dq[2], dk[ST], dv[ST];
#pragma unroll
      for (int i = 0; i < 2; ++i) dq[i] = sdesc_sw128(smem_u32(sQ + i * Cfg::TILE), 16, 1024);
#pragma unroll
      for (int st = 0; st < ST; ++st) {
        dk[st] = sdesc_sw128(smem_u32(sK + st * Cfg::TILE), 16, 1024);
        dv[st] = sdesc_sw128(smem_u32(sV + st * Cfg::TILE), Cfg::CHUNK, 1024);
      }
      auto issue_s = [&](int i, int j) {
        const uint64_t a = dq[i], b = dk[j % ST];
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t o = (uint64_t)(((k >> 2) * Cfg::CHUNK + (k & 3) * 32) >> 4);
          umma_bf16(tmem + 128 * i, a + o, b + o, idS, k > 0);
        }
        umma_commit(&s_full[i]);
      };
      auto issue_pv = [&](int i, int j) {
        const uint64_t b = dv[j % ST];
        const uint32_t tP = tmem + 128 * i + 64, tO = tmem + 256 + D * i;
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k)
          umma_bf16_ts(tO, tP + k * 8, b + (uint64_t)(k * (2048 >> 4)), idO, (j | k) != 0);
        umma_commit(&pv_done[i]);
      };
      bool ok = mbar_wait(q_full, 0, p.err, kErrWaitFull) && mbar_wait(&k_full[0], 0, p.err, kErrWaitFull);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_blocks && ok; ++j) {
        const int st = j % ST, st1 = (j + 1) % ST;
        const bool more = j + 1 < n_blocks;
        ok = mbar_wait(&v_full[st], (j / ST) & 1, p.err, kErrWaitFull) &&
             mbar_wait(&p_ready[0], j & 1, p.err, kErrWaitAccFull);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          if (!mbar_wait(&k_full[st1], ((j + 1) / ST) & 1, p.err, kErrWaitFull)) break;
          tc_fence_after();
          issue_s(0, j + 1);
        }
        if (!mbar_wait(&p_ready[1], j & 1, p.err, kErrWaitAccFull)) break;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&v_empty[st]);
        if (more) {
          issue_s(1, j + 1);
          umma_commit(&k_empty[st1]);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax warps
    const int tile = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row inside the tile == TMEM lane
    const int h = tile ? h1 : h0;
    const int m0 = tile ? m01 : m00;
    const int qi = m0 + r;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tmem + 128 * tile, tP = tS + 64, tO = tmem + 256 + D * tile;
    const int seg_q = (p.seg && qi < p.Sq) ? p.seg[(long long)b * p.Sk + qi + off] : 0;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;  // running max in scaled log2 units, row sum
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      if (!mbar_wait(&s_full[tile], j & 1, p.err, kErrWaitAccFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * 128;
      const bool need_mask = (p.causal && (k0 + 127 > m0 + off)) || (k0 + 128 > p.Sk) || p.seg;
      uint32_t vis[4];
      if (need_mask) {
        mask_upto(min(p.Sk - k0, p.causal ? qi + off - k0 + 1 : 128), vis);
        if (p.seg) {
#pragma unroll 1
          for (int c = 0; c < 128; ++c) {
            const int ki = k0 + c;
            if (ki < p.Sk && p.seg[(long long)b * p.Sk + ki] != seg_q) vis[c >> 5] &= ~(1u << (c & 31));
          }
        }
      }
      uint32_t v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tmem_wait_ld();
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < 128; ++i) v[i] = ((vis[i >> 5] >> (i & 31)) & 1u) ? v[i] : __float_as_uint(-INFINITY);
      }
      // row max: three-input maxima over four independent chains
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 128; i += 8) {
#pragma unroll
        for (int c = 0; c < 4; ++c) mx[c] = max3f(mx[c], __uint_as_float(v[i + 2 * c]), __uint_as_float(v[i + 2 * c + 1]));
      }
      const float m_new = fmaxf(m_used, max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * sl2);
      const bool need = (m_used == -INFINITY && m_new != -INFINITY) || (m_new - m_used > 8.f);
      if (__any_sync(0xffffffff, need)) {
        const float factor = (m_used == -INFINITY) ? 0.f : ex2f(m_used - m_new);
        if (j > 0) {  // O_i is stable: PV_i(j-1) finished before S_i(j)
          // 16 columns at a time: the 128 S values of this row stay live in registers meanwhile
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t o[16];
            tmem_ld16(tO + lane_off + c * 16, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st16(tO + lane_off + c * 16, o);
          }
        }
        l *= factor;
        m_used = m_new;
      }
      const float msafe = (m_used == -INFINITY) ? 0.f : m_used;
      // x = s * scale * log2(e) - m two lanes per instruction; row sums in two packed accumulators
      const uint64_t scale2 = f2_pack(sl2, sl2), negm2 = f2_pack(-msafe, -msafe);
      uint64_t sum2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(v[c * 32 + 2 * i]), __uint_as_float(v[c * 32 + 2 * i + 1])),
                                     scale2, negm2);
          float x0, x1;
          f2_unpack(x2, x0, x1);
          const bool emu = i < EMU;  // resolved at compile time after unrolling
          const float e0 = emu ? exp2_poly(x0) : ex2f(x0);
          const float e1 = emu ? exp2_poly(x1) : ex2f(x1);
          sum2[i & 1] = f2_add(sum2[i & 1], f2_pack(e0, e1));
          pk[i] = pack_bf16(e0, e1);
        }
        tmem_st16(tP + lane_off + c * 16, pk);
      }
      float a0, a1, b0, b1;
      f2_unpack(sum2[0], a0, a1);
      f2_unpack(sum2[1], b0, b1);
      l += (a0 + a1) + (b0 + b1);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[tile]);
    }
    const bool row_ok = qi < p.Sq;
    if (ok && n_blocks > 0 &&
        mbar_wait(&pv_done[tile], (n_blocks - 1) & 1, p.err, kErrWaitAccFull)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.O + ((long long)b * p.Sq + qi) * p.ldo + h * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + lane_off + c * 32, o);
        tmem_wait_ld();
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int g = 0; g < 4; ++g)
            dst[g] = make_uint4(pack_bf16(__uint_as_float(o[8 * g]) * inv, __uint_as_float(o[8 * g + 1]) * inv),
                                pack_bf16(__uint_as_float(o[8 * g + 2]) * inv, __uint_as_float(o[8 * g + 3]) * inv),
                                pack_bf16(__uint_as_float(o[8 * g + 4]) * inv, __uint_as_float(o[8 * g + 5]) * inv),
                                pack_bf16(__uint_as_float(o[8 * g + 6]) * inv, __uint_as_float(o[8 * g + 7]) * inv));
        }
      }
      if (row_ok)
        p.lse[((long long)b * p.Hq + h) * p.Sq + qi] =
            (l > 0.f) ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
    } else if (n_blocks == 0 && row_ok) {
      __nv_bfloat16* orow = p.O + ((long long)b * p.Sq + qi) * p.ldo + h * D;
      for (int c = 0; c < D; ++c) orow[c] = __float2bfloat16_rn(0.f);
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

// 3-D map over a [B][S][ld] bf16 buffer: box = 64 columns x 128 rows x 1 batch, 128-byte swizzle.
void rows_map(CUtensorMap* m, const void* base, int B, int S, long long ld) {
  uint64_t dims[3] = {(uint64_t)ld, (uint64_t)S, (uint64_t)B};
  uint64_t strides[2] = {(uint64_t)ld * 2, (uint64_t)S * ld * 2};
  uint32_t box[3] = {64, 128, 1};
  astrai_host::make_tmap_bf16(m, base, 3, dims, strides, box, true);
}

template <int D, int EMU>
void launch_pair(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const PairFwdParams& p,
                 cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {false};
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(flash_fwd_pair_kernel<D, EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         PairCfg<D>::SMEM);
    attr[dev & 63] = true;
  }
  const int n_mblocks = (p.Sq + 127) / 128;
  const unsigned grid = p.pair_heads ? (unsigned)n_mblocks * p.B * (p.Hq / 2)
                                     : (unsigned)((n_mblocks + 1) / 2) * p.B * p.Hq;
  (astrai::note_launch(),
   flash_fwd_pair_kernel<D, EMU><<<grid, kPairThreads, PairCfg<D>::SMEM, s>>>(tq, tk, tv, p));
}

template <int D>
void launch_pair_emu(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const PairFwdParams& p,
                     int emu, cudaStream_t s) {
  switch (emu) {
    case 0: launch_pair<D, 0>(tq, tk, tv, p, s); break;
    case 2: launch_pair<D, 2>(tq, tk, tv, p, s); break;
    case 4: launch_pair<D, 4>(tq, tk, tv, p, s); break;
    default: launch_pair<D, 3>(tq, tk, tv, p, s); break;
  }
}

// exponential pairs per 16 computed on the FMA pipe (0, 2, 3 or 4; ASTRAI_FA_EMU overrides the default 0:
// at B4 S2048 H16/4 the kernel measured fastest with every exponential on MUFU)
int emu_pairs() {
  static int v = [] {
    const char* e = std::getenv("ASTRAI_FA_EMU");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

}  // namespace
}  // namespace astrai

namespace astrai_host {

// head_dim 64 or 128; q/k/v/o rows 16-byte aligned, column offsets multiples of 8 elements
void flash_fwd_pair(const void* q, long long ldq, int q_col0, const void* k, long long ldk, int k_col0, const void* v,
                    long long ldv, int v_col0, void* o, long long ldo, float* lse, int B, int Sq, int Sk, int Hq,
                    int Hkv, int D, float scale, int causal, const int* seg, cudaStream_t s) {
  using namespace astrai;
  if (D != 64 && D != 128) throw std::runtime_error("flash_fwd_pair: head_dim must be 64 or 128");
  if (Hq % Hkv) throw std::runtime_error("flash_fwd_pair: Hq must be a multiple of Hkv");
  CUtensorMap tq, tk, tv;
  rows_map(&tq, q, B, Sq, ldq);
  rows_map(&tk, k, B, Sk, ldk);
  rows_map(&tv, v, B, Sk, ldv);
  PairFwdParams p;
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
  p.pair_heads = (Hq / Hkv) % 2 == 0 ? 1 : 0;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = error_word(dev);
  if (D == 128)
    launch_pair_emu<128>(tq, tk, tv, p, emu_pairs(), s);
  else
    launch_pair_emu<64>(tq, tk, tv, p, emu_pairs(), s);
}

}  // namespace astrai_host
