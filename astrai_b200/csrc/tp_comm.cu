// Second half of the row-parallel linear's fused all-reduce (sm_100a, NVLink peer memory).
//
// RowParallelLinear (reference: astrai/parallel/module.py:18-63, all_reduce SUM of x_r @ w_r^T)
// runs as: (1) the GEMM of every rank, whose epilogue pushes the rows of its partial product that
// other ranks own into their receive slots as each tile finishes (gemm.cu, scatter_copy_tile);
// (2) this kernel on every rank, after the partials of its own rows have landed: it sums its
// rows over all ranks in fp32 and stores the bf16 result into every rank's output over NVLink
// (row-contiguous 16-byte stores), then the last CTA raises this rank's flag on every peer.
// Bytes over NVLink per rank: 2 (W - 1) / W of the output, as a ring all-reduce.
#include <stdexcept>

#include "common.cuh"

namespace astrai {

constexpr int kTpMaxRanks = 8;

struct RowReduceParams {
  const __nv_bfloat16* part;  // [M][ld] this rank's partial product
  const __nv_bfloat16* recv;  // [W][rpo][ld] receive slots (slot q: rank q's partial of my rows)
  __nv_bfloat16* out;         // [M][ld] the all-reduced output (this rank's copy)
  long long ld;
  int M, N, rank, world, rpo;
  long long rank_delta[kTpMaxRanks];  // bytes from a local address to the same place on rank q
  unsigned* flag;                     // local address of this rank's flag in the flag row
  unsigned epoch;
  unsigned* done;                     // grid-completion counter, zero between launches
};

__global__ void __launch_bounds__(256) row_reduce_bcast_kernel(const RowReduceParams p) {
  const int r0 = p.rank * p.rpo;
  const int rows = min(p.M, r0 + p.rpo) - r0;
  const int vpr = p.N / 8;  // N % 8 == 0 (checked by the host)
  const long long nvec = rows > 0 ? (long long)rows * vpr : 0;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
       v += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(v / vpr), c = (int)(v % vpr) * 8;
    const long long off = (long long)(r0 + i) * p.ld + c;
    float acc[8];
    {
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p.part + off));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16(w[j]);
        acc[2 * j] = f.x;
        acc[2 * j + 1] = f.y;
      }
    }
#pragma unroll
    for (int q = 0; q < kTpMaxRanks; ++q) {
      if (q >= p.world || q == p.rank) continue;
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p.recv + ((long long)(q * p.rpo + i)) * p.ld + c));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16(w[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    const uint4 o = make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                               pack_bf16(acc[6], acc[7]));
    char* dst = reinterpret_cast<char*>(p.out + off);
#pragma unroll
    for (int q = 0; q < kTpMaxRanks; ++q)
      if (q < p.world) *reinterpret_cast<uint4*>(dst + p.rank_delta[q]) = o;  // rank_delta[rank] == 0
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(p.done, 1u) == gridDim.x - 1) {
    __threadfence_system();
#pragma unroll
    for (int q = 0; q < kTpMaxRanks; ++q)
      if (q < p.world && q != p.rank) {
        unsigned* f = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(p.flag) + p.rank_delta[q]);
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(p.epoch) : "memory");
      }
    *p.done = 0u;
  }
}

}  // namespace astrai

namespace astrai_host {

void row_reduce_bcast(const void* part, const void* recv, void* out, long long ld, int M, int N, int rank, int world,
                      int rpo, const long long* rank_delta, unsigned* flag, unsigned epoch, unsigned* done,
                      int sms, cudaStream_t s) {
  using namespace astrai;
  if (world < 1 || world > kTpMaxRanks || N % 8 != 0 || ld % 8 != 0 || rpo <= 0)
    throw std::runtime_error("row_reduce_bcast: unsupported shape or world size");
  RowReduceParams p;
  p.part = static_cast<const __nv_bfloat16*>(part);
  p.recv = static_cast<const __nv_bfloat16*>(recv);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld = ld;
  p.M = M;
  p.N = N;
  p.rank = rank;
  p.world = world;
  p.rpo = rpo;
  for (int q = 0; q < kTpMaxRanks; ++q) p.rank_delta[q] = q < world ? rank_delta[q] : 0;
  p.flag = flag;
  p.epoch = epoch;
  p.done = done;
  (astrai::note_launch(), row_reduce_bcast_kernel<<<sms * 4, 256, 0, s>>>(p));
}

}  // namespace astrai_host
