// Global scale of a bf16 tensor with no caller-provided device workspace.
//
// nvfp4b200_global_scale needs a small device workspace from its caller.
// Some callers cannot provide one: code that runs inside a memory pool or
// arena that owns all device memory and forbids new allocations, plugin
// hosts that hand the library only the tensors of the call, and paths that
// must not call cudaMalloc/cudaFree because those calls can synchronise the
// device.  This entry point keeps its scratch in a fixed array in the
// library's own device memory instead, so it allocates nothing.
//
// Scratch: NOALLOC_MAX_PARTIALS per-CTA partial maxima plus a completion
// counter (about 16 KB).  Every GPU that loads the library holds this array
// until the process exits.  Each CTA reduces NOALLOC_CHUNK elements, so one
// call handles at most NOALLOC_MAX_PARTIALS * NOALLOC_CHUNK = 2^30 elements;
// larger inputs are rejected.  All calls share the array: calls whose work
// overlaps on the GPU (for example on two streams) race and must be avoided.
#include "common.cuh"

#include <mutex>

namespace nvfp4b200 {
namespace noalloc {

constexpr int MAX_PARTIALS = 4096;           // one partial maximum per CTA
constexpr int64_t CHUNK = int64_t(1) << 18;  // elements reduced by one CTA
constexpr int64_t MAX_ELEMS = MAX_PARTIALS * CHUNK;
constexpr int COUNTER = MAX_PARTIALS;        // index of the completion counter
constexpr int THREADS = 256;

// [0, MAX_PARTIALS): partial maxima (float bits); [MAX_PARTIALS]: counter.
static __device__ __align__(256) uint32_t g_scratch[MAX_PARTIALS + 64];

// |x| max of 8 bf16 values as float bits, NaN ignored.
__device__ __forceinline__ uint32_t absmax8(const uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t a = w[i] & 0x7FFF7FFFu;
    a &= ~__vcmpgtu2(a, 0x7F807F80u);
    m = __vmaxu2(m, a);
  }
  return max(m & 0xFFFFu, m >> 16) << 16;
}

__device__ __forceinline__ uint32_t block_max(uint32_t v, uint32_t* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = __reduce_max_sync(0xffffffffu, v);
  if (lane == 0) red[wid] = v;
  __syncthreads();
  uint32_t m = 0;
  if (threadIdx.x < 32) {
    m = (threadIdx.x < THREADS / 32) ? red[threadIdx.x] : 0u;
    m = __reduce_max_sync(0xffffffffu, m);
  }
  __syncthreads();
  return m;  // valid in thread 0
}

__global__ void __launch_bounds__(THREADS) amax_partials_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                uint32_t* scratch, float* g_out, float* amax_out) {
  __shared__ uint32_t red[THREADS / 32];
  __shared__ int is_last;
  const int64_t begin = (int64_t)blockIdx.x * CHUNK;
  const int64_t end = imin64(n, begin + CHUNK);
  const int64_t vend = begin + ((end - begin) / 8) * 8;  // begin is a multiple of 8
  uint32_t m = 0;
  for (int64_t i = begin + 8 * (int64_t)threadIdx.x; i < vend; i += 8 * THREADS)
    m = max(m, absmax8(__ldg(reinterpret_cast<const uint4*>(x + i))));
  for (int64_t i = vend + threadIdx.x; i < end; i += THREADS) {
    const uint32_t a = x[i] & 0x7FFFu;
    if (a <= 0x7F80u) m = max(m, a << 16);
  }
  const uint32_t bm = block_max(m, red);
  if (threadIdx.x == 0) {
    scratch[blockIdx.x] = bm;
    __threadfence();
    const uint32_t done = atomicAdd(&scratch[COUNTER], 1u);
    is_last = done == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  uint32_t t = 0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += THREADS) t = max(t, *(volatile uint32_t*)&scratch[i]);
  const uint32_t tm = block_max(t, red);
  if (threadIdx.x == 0) {
    const float amax = __uint_as_float(tm);
    const float g = (amax > 0.0f && amax <= 3.402823466e38f) ? __fdiv_rn(amax, 2688.0f) : 1.0f;
    *g_out = g;
    if (amax_out) *amax_out = amax;
    scratch[COUNTER] = 0u;
  }
}

// Device address of g_scratch for the current device, looked up once per
// device (host code may not use the symbol itself as a device pointer).
static int scratch_address(uint32_t** out) {
  static std::mutex mu;
  static uint32_t* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  if (dev < 0 || dev >= 64) return NVFP4B200_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return NVFP4B200_ERR_CUDA;
    cache[dev] = static_cast<uint32_t*>(p);
  }
  *out = cache[dev];
  return NVFP4B200_OK;
}

}  // namespace noalloc
}  // namespace nvfp4b200

using namespace nvfp4b200;

extern "C" int nvfp4b200_global_scale_noalloc(const void* x, int64_t n, float* global_scale_out, float* amax_out,
                                              void* stream) {
  if (!x || !global_scale_out) return NVFP4B200_ERR_INVALID_ARG;
  if (n <= 0 || n > noalloc::MAX_ELEMS) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  uint32_t* scratch = nullptr;
  if ((rc = noalloc::scratch_address(&scratch))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // the completion counter must start at zero (partials are written before they are read)
  if (cudaMemsetAsync(scratch + noalloc::COUNTER, 0, sizeof(uint32_t), st) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  const unsigned grid = (unsigned)ceil_div(n, noalloc::CHUNK);
  noalloc::amax_partials_kernel<<<grid, noalloc::THREADS, 0, st>>>(static_cast<const uint16_t*>(x), n, scratch,
                                                                   global_scale_out, amax_out);
  return launch_status();
}
