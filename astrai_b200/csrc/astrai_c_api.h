// C entry points of the astrai_b200 kernel library (exported from _C.so).
//
// astrai_rmsnorm_bwd_static_scratch has no counterpart in the reference
// project. It is the RMSNorm backward of the library (dx and dw of
// y = x * rsqrt(mean(x^2) + eps) * w) for callers that cannot allocate device
// memory at call time: a C/C++ runtime that has handed all device memory to
// its own pool up front and keeps a fixed footprint, or code running inside
// an allocator callback / out-of-memory handler, where asking an allocator
// for memory again would recurse or fail. The regular entry point takes a
// caller-allocated scratch buffer for the per-block dw partial sums; this one
// uses a fixed array compiled into the library instead and allocates nothing
// (no cudaMalloc / cudaFree, no PyTorch or other allocating library call).
//
// Scratch: one file-scope device array of ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS
// floats (4 MiB) per device. A call needs ceil(rows / 64) * D floats of it;
// larger problems are rejected (return value -1, message on stderr) before
// anything is launched, e.g. D = 2048 allows up to 32768 rows.
//
// Sharing: every call on a device uses the same array, and the array keeps
// whatever the last call left in it. Nothing in it has to start at zero: each
// call writes every partial it later reads. Calls that overlap in time on one
// device (two streams, two host threads) race on the array and give wrong
// dw; order them on one stream or serialise them.
//
// Setup: the first call on each device looks up the array's device address
// (cudaGetSymbolAddress) with that device current, and keeps it for the life
// of the process (a failed lookup is not kept; the next call tries again).
// Make that first call before any stream capture begins. A device reset
// (cudaDeviceReset, or a reset of the primary context) after the first call is
// not supported: the kept address would be stale.
//
// Arguments: bf16 row-major dy / x / dx with row strides in elements (16-byte
// aligned rows), bf16 weight w [D], fp32 rstd [rows] from the forward pass;
// dw is written as bf16 (dw_bf16) and/or fp32 (dw_f32), either may be NULL;
// stream is a cudaStream_t (NULL = legacy default stream). D must be a
// multiple of 8 and at most 4096.
//
// Returns 0 on success, -1 for rejected sizes, otherwise a cudaError_t: of
// the failing setup call, or the calling thread's pending runtime error after
// the launches (cudaGetLastError). That pending error can also be one that an
// earlier, unrelated runtime call of the same thread left behind; this call
// reports and clears it. Check your own calls' errors before calling this.
#ifndef ASTRAI_C_API_H_
#define ASTRAI_C_API_H_

#ifdef __cplusplus
extern "C" {
#endif

#define ASTRAI_RMSNORM_BWD_SCRATCH_FLOATS (1LL << 20)

int astrai_rmsnorm_bwd_static_scratch(const void* dy, long long lddy, const void* x, long long ldx, const void* w,
                                      const float* rstd, void* dx, long long lddx, void* dw_bf16, float* dw_f32,
                                      int rows, int D, void* stream);

#ifdef __cplusplus
}
#endif

#endif  // ASTRAI_C_API_H_
