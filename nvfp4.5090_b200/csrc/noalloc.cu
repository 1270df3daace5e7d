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
// Scratch: MAX_PARTIALS per-CTA partial maxima plus a completion counter
// (about 16 KB).  Every GPU that loads the library holds this array until the
// process exits.  The grid is at most MAX_PARTIALS CTAs, each striding over
// the input, and one call handles at most MAX_ELEMS = 2^30 elements; larger
// inputs are rejected.  All calls share the array: calls whose work overlaps
// on the GPU (for example on two streams) race and must be avoided.
#include "common.cuh"

#include <algorithm>

namespace nvfp4b200 {
namespace noalloc {

constexpr int MAX_PARTIALS = 4096;               // one partial maximum per CTA: the grid limit
constexpr int64_t MAX_ELEMS = int64_t(1) << 30;  // elements per call
constexpr int COUNTER = MAX_PARTIALS;            // index of the completion counter
constexpr int THREADS = 256;
constexpr int UNROLL = 4;                        // 16-byte loads in flight per thread

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

// Grid-stride over the input's 16-byte vectors, four loads in flight per
// thread; block 0 also takes the scalar tail.  Each CTA writes its maximum to
// scratch[blockIdx.x]; the last CTA to finish (completion counter) reduces
// the partials, writes the global scale and resets the counter to zero.
__global__ void __launch_bounds__(THREADS) amax_partials_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                uint32_t* scratch, float* g_out, float* amax_out) {
  __shared__ uint32_t red[THREADS / 32];
  __shared__ int is_last;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  const int64_t n_vec = n / 8;
  const int64_t stride = (int64_t)gridDim.x * THREADS;
  int64_t i = (int64_t)blockIdx.x * THREADS + threadIdx.x;
  uint32_t m = 0;
  for (; i + (UNROLL - 1) * stride < n_vec; i += UNROLL * stride) {
    uint4 v[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) v[u] = __ldg(xv + i + u * stride);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) m = max(m, absmax8(v[u]));
  }
  for (; i < n_vec; i += stride) m = max(m, absmax8(__ldg(xv + i)));
  if (blockIdx.x == 0 && n_vec * 8 + (int64_t)threadIdx.x < n) {   // the last n % 8 elements
    const uint32_t a = x[n_vec * 8 + threadIdx.x] & 0x7FFFu;
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
  for (int j = threadIdx.x; j < (int)gridDim.x; j += THREADS) t = max(t, *(volatile uint32_t*)&scratch[j]);
  const uint32_t tm = block_max(t, red);
  if (threadIdx.x == 0) {
    const float amax = __uint_as_float(tm);
    const float g = (amax > 0.0f && amax <= 3.402823466e38f) ? __fdiv_rn(amax, 2688.0f) : 1.0f;
    *g_out = g;
    if (amax_out) *amax_out = amax;
    scratch[COUNTER] = 0u;
  }
}

// CTAs for n elements: enough for four 16-byte loads per thread, at most 8
// per SM and at most MAX_PARTIALS (the partials array).
static unsigned grid_for(int64_t n) {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int sm = 148;
  if (dev >= 0 && dev < 64) {
    if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sms[dev] > 0) sm = sms[dev];
  }
  const int64_t want = ceil_div(n, (int64_t)8 * THREADS * UNROLL);
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>({want, (int64_t)8 * sm, (int64_t)MAX_PARTIALS}));
}

// Device address of g_scratch in the current context.  Host code may not use
// the symbol itself as a device pointer.  The address is looked up on every
// call, not cached: the runtime resolves it from its own per-context module
// table (after the first call on a device, which loads the module, this is a
// host-side lookup), so a cudaDeviceReset between calls, after which the
// module is loaded again and the array can move, is handled.
static int scratch_address(uint32_t** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return NVFP4B200_ERR_CUDA;
  *out = static_cast<uint32_t*>(p);
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
  noalloc::amax_partials_kernel<<<noalloc::grid_for(n), noalloc::THREADS, 0, st>>>(
      static_cast<const uint16_t*>(x), n, scratch, global_scale_out, amax_out);
  return launch_status();
}
