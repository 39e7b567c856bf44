"""Per-role timeline of the flash-attention backward kernel (B4 S2048 H16/4 D128 causal).

``python -m astrai_b200.utils.fa_bwd_timeline`` makes a copy of ``csrc/attention.cu`` in a
temporary directory with ``clock64()`` stamps written by CTA 0 (the longest key block) at every
wait and issue point of each role (TMA, MMA, softmax, dQ), compiles it with ``nvcc`` for sm_100a
together with ``csrc/runtime.cu`` and a small ``main()``, runs it (8 launches, the last 5 timed with
CUDA events) and prints the stamps of a few iterations and the cycles per 64-query iteration.
The committed kernel is not changed; the copy only adds the stamps.
"""

import os
import subprocess
import sys
import tempfile

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")
_SRC = {"text": ""}


def _rep(a: str, b: str, cnt: int = 1) -> None:
    assert a in _SRC["text"], "attention.cu changed: stamp anchor not found: " + a[:80]
    _SRC["text"] = _SRC["text"].replace(a, b, cnt)


def make_source() -> str:
    with open(os.path.join(CSRC, "attention.cu")) as fh:
        _SRC["text"] = fh.read()
    _stamps()
    return _SRC["text"] + _MAIN


def _stamps() -> None:
    exec(compile(_STAMPS, "fa_bwd_timeline_stamps", "exec"), {"_rep": _rep})


_STAMPS = r"""
_rep('constexpr int FB_THREADS = 320;','''constexpr int FB_THREADS = 320;
__device__ unsigned long long g_ts[4][128][6];
#define TS(r, j, k) do { if (blockIdx.x == 0 && (j) >= 0 && (j) < 128) g_ts[r][j][k] = clock64(); } while (0)''')
# loader
_rep('''      if (lane == 0 && it >= FB_QD &&
          !mbar_wait(&qd_empty[slot], ((it / FB_QD) - 1) & 1, p.err, kErrWaitEmpty))
        break;''','''      if (lane == 0) TS(3, it, 0);
      if (lane == 0 && it >= FB_QD &&
          !mbar_wait(&qd_empty[slot], ((it / FB_QD) - 1) & 1, p.err, kErrWaitEmpty))
        break;
      if (lane == 0) TS(3, it, 1);''')
# MMA
_rep('''        if (!ok) break;
        tc_fence_after();
        const uint64_t bq = pick(dQ_k, qs), bo = pick(dO_k, qs);''','''        if (!ok) break;
        TS(0, it, 0);
        tc_fence_after();
        const uint64_t bq = pick(dQ_k, qs), bo = pick(dO_k, qs);''')
_rep('''        umma_commit(&sd_full[slot]);
        // gradients of it-1 once its softmax is done; they overlap the softmax of it
        if (it >= 1) {
          ok = mbar_wait(&ps_ready[slot ^ 1], ((it - 1) >> 1) & 1, p.err, kErrWaitAccEmpty);
          if (ok) {
            tc_fence_after();
            ok = issue_grads(it - 1);
          }
        }''','''        umma_commit(&sd_full[slot]);
        TS(0, it, 1);
        // gradients of it-1 once its softmax is done; they overlap the softmax of it
        if (it >= 1) {
          ok = mbar_wait(&ps_ready[slot ^ 1], ((it - 1) >> 1) & 1, p.err, kErrWaitAccEmpty);
          TS(0, it, 2);
          if (ok) {
            tc_fence_after();
            ok = issue_grads(it - 1);
          }
          TS(0, it, 3);
        }''')
# softmax
_rep('''      const int m0 = (mb_first + it % per_head) * FB_BM;
      ok = mbar_wait(&sd_full[slot], (it >> 1) & 1, p.err, kErrWaitAccFull) &&''','''      const int m0 = (mb_first + it % per_head) * FB_BM;
      if (warp == 2 && lane == 0) TS(1, it, 0);
      ok = mbar_wait(&sd_full[slot], (it >> 1) & 1, p.err, kErrWaitAccFull) &&''')
_rep('''      if (!ok) break;
      tc_fence_after();
      // visible query columns of this key row, as a 64-bit mask''','''      if (!ok) break;
      if (warp == 2 && lane == 0) TS(1, it, 1);
      tc_fence_after();
      // visible query columns of this key row, as a 64-bit mask''')
_rep('''      tmem_wait_ld();
      uint32_t pk[2][16], dk[2][16];''','''      tmem_wait_ld();
      if (warp == 2 && lane == 0) TS(1, it, 2);
      uint32_t pk[2][16], dk[2][16];''')
_rep('''      // dS^T slot it & 1 was last read by the gradient MMAs of it-2: wait only now, so this tile's math''','''      if (warp == 2 && lane == 0) TS(1, it, 3);
      // dS^T slot it & 1 was last read by the gradient MMAs of it-2: wait only now, so this tile's math''')
_rep('''#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int g = 0; g < 4; ++g)
          st_shared_v4(swz(dc, r, c * 4 + g)''','''      if (warp == 2 && lane == 0) TS(1, it, 4);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int g = 0; g < 4; ++g)
          st_shared_v4(swz(dc, r, c * 4 + g)''')
_rep('''      if (lane == 0) mbar_arrive(&ps_ready[slot]);
    }''','''      if (lane == 0) mbar_arrive(&ps_ready[slot]);
      if (warp == 2 && lane == 0) TS(1, it, 5);
    }''')
# dQ warps
_rep('''      if (!mbar_wait(&dq_full[it & 1], (it >> 1) & 1, p.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const uint32_t tdQ = tmem + (it & 1) * 128;''','''      if (warp == 6 && lane == 0) TS(2, it, 0);
      if (!mbar_wait(&dq_full[it & 1], (it >> 1) & 1, p.err, kErrWaitAccFull)) break;
      if (warp == 6 && lane == 0) TS(2, it, 1);
      tc_fence_after();
      const uint32_t tdQ = tmem + (it & 1) * 128;''')
_rep('''      if (warp == 6 && lane == 0) {
        tma_reduce_add_3d(&tmdQ, sdQ, h * FA_D, m0, b);
        bulk_commit();
      }''','''      if (warp == 6 && lane == 0) TS(2, it, 2);
      if (warp == 6 && lane == 0) {
        tma_reduce_add_3d(&tmdQ, sdQ, h * FA_D, m0, b);
        bulk_commit();
      }
      if (warp == 6 && lane == 0) TS(2, it, 3);''')
"""

_MAIN = r"""
#include <cstdio>
#include <vector>
namespace astrai_host {
void make_tmap_bf16(CUtensorMap*, const void*, int, const uint64_t*, const uint64_t*, const uint32_t*, bool);
}
int main() {
  int B = 4, S = 2048, Hq = 16, Hkv = 4, D = 128;
  long long ld = (Hq + 2 * Hkv) * D;
  size_t n = (size_t)B * S * ld;
  std::vector<__nv_bfloat16> h(n);
  unsigned x = 1;
  for (auto& e : h) { x = x * 1664525u + 1013904223u; e = __float2bfloat16(((x >> 9) & 0xffff) / 65536.f - 0.5f); }
  void *qkv, *o, *dO, *dqkv; float *lse, *delta, *dq_acc;
  cudaMalloc(&qkv, n * 2); cudaMalloc(&dqkv, n * 2);
  cudaMalloc(&o, (size_t)B * S * Hq * D * 2); cudaMalloc(&dO, (size_t)B * S * Hq * D * 2);
  cudaMalloc(&lse, (size_t)B * Hq * S * 4); cudaMemset(lse, 0, (size_t)B * Hq * S * 4);
  cudaMalloc(&delta, (size_t)2 * B * Hq * S * 4); cudaMalloc(&dq_acc, (size_t)B * S * Hq * D * 4);
  cudaMemcpy(qkv, h.data(), n * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(o, h.data(), (size_t)B * S * Hq * D * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dO, h.data() + 7, (size_t)B * S * Hq * D * 2, cudaMemcpyHostToDevice);
  cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
  float tot = 0.f;
  for (int it = 0; it < 8; ++it) {
    cudaMemset(dq_acc, 0, (size_t)B * S * Hq * D * 4);
    cudaEventRecord(a);
    astrai_host::flash_bwd(qkv, ld, 0, qkv, ld, Hq * D, qkv, ld, (Hq + Hkv) * D, o, Hq * D, dO, Hq * D, 0, lse, delta,
                           dq_acc, dqkv, ld, 0, dqkv, dqkv, ld, Hq * D, (Hq + Hkv) * D, B, S, S, Hq, Hkv, 0.0883883f, 1,
                           nullptr, 0);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    if (it >= 3) tot += ms;
  }
  unsigned long long ts[4][128][6];
  cudaMemcpyFromSymbol(ts, astrai::g_ts, sizeof(ts));
  printf("bwd ms %.4f err %s\n", tot / 5, cudaGetErrorString(cudaGetLastError()));
  unsigned long long t0 = ts[0][0][0];
  auto d = [&](int r, int j, int k) { return (long long)(ts[r][j][k] - t0); };
  for (int j = 1; j < 128; j += (j < 8 ? 1 : 15)) {
    printf("it=%3d MMA go %7lld sdp %7lld psw %7lld gr %7lld | SM w %7lld in %7lld ld %7lld math %7lld dqw %7lld arr %7lld"
           " | DQ w %7lld in %7lld tma %7lld | LD w %7lld in %7lld\n", j,
           d(0, j, 0), d(0, j, 1), d(0, j, 2), d(0, j, 3), d(1, j, 0), d(1, j, 1), d(1, j, 2), d(1, j, 3), d(1, j, 4),
           d(1, j, 5), d(2, j, 0), d(2, j, 1), d(2, j, 3), d(3, j, 0), d(3, j, 1));
  }
  printf("per-iteration (it 8..120): %.0f clk\n", (double)(ts[0][120][0] - ts[0][8][0]) / 112.0);
  return 0;
}
"""


def main() -> None:
    work = tempfile.mkdtemp(prefix="fa_bwd_timeline_")
    cu = os.path.join(work, "fa_bwd_timeline.cu")
    with open(cu, "w") as fh:
        fh.write(make_source())
    exe = os.path.join(work, "fa_bwd_timeline")
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-I", CSRC, cu,
                    os.path.join(CSRC, "runtime.cu"), "-o", exe], check=True)
    sys.exit(subprocess.run([exe]).returncode)


if __name__ == "__main__":
    main()
