// Host runtime shared by every kernel launcher: device error word, SM count
// cache and TMA descriptor encoding through the driver entry point (so the
// extension does not link libcuda directly).
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

#include <atomic>

#include "common.cuh"

namespace astrai_host {

int num_sms(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (cache[device] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    cache[device] = n > 0 ? n : 148;
  }
  return cache[device];
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) throw std::runtime_error("astrai: cuTensorMapEncodeTiled unavailable from the CUDA driver");
  return fn;
}

void make_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("astrai: TMA base address must be 16-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    gstride[i] = strides_bytes[i];
    if (gstride[i] % 16 != 0) throw std::runtime_error("astrai: TMA strides must be multiples of 16 bytes");
  }
  CUresult r = get_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), gdim, gstride,
                               bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("astrai: cuTensorMapEncodeTiled (f32) failed");
}

void make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("astrai: TMA base address must be 16-byte aligned");
  // Encoding needs a current context; autograd's backward worker threads may
  // not have made the primary context current yet.
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    gstride[i] = strides_bytes[i];
    if (gstride[i] % 16 != 0) throw std::runtime_error("astrai: TMA strides must be multiples of 16 bytes");
  }
  CUresult r = get_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), gdim, gstride,
                               bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[256];
    snprintf(msg, sizeof(msg), "astrai: cuTensorMapEncodeTiled failed (%d) rank=%d dims=%llu,%llu box=%u,%u",
             (int)r, rank, (unsigned long long)dims[0], (unsigned long long)(rank > 1 ? dims[1] : 0), box[0],
             rank > 1 ? box[1] : 0);
    throw std::runtime_error(msg);
  }
}

int* error_word(int device) {
  static int* words[64] = {nullptr};
  static std::mutex mu;
  if (device < 0 || device >= 64) device = 0;
  std::lock_guard<std::mutex> g(mu);
  if (!words[device]) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) throw std::runtime_error("astrai: cannot allocate error word");
    cudaMemset(p, 0, sizeof(int));
    cudaSetDevice(prev);
    words[device] = p;
  }
  return words[device];
}

int read_and_clear_error() {
  int dev = 0;
  cudaGetDevice(&dev);
  int* w = error_word(dev);
  int h = 0;
  cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost);
  cudaMemset(w, 0, sizeof(int));
  return h;
}

}  // namespace astrai_host

namespace astrai {
static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace astrai

namespace astrai_host {
long long launch_count() { return astrai::g_launches.load(std::memory_order_relaxed); }
// Launches that ran without passing a host launch site: CUDA-graph replays of captured kernels.
void add_launches(long long n) { astrai::g_launches.fetch_add(n, std::memory_order_relaxed); }
}  // namespace astrai_host
