// Shared device/host helpers for the NVFP4 B200 library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/nvfp4_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "this library is written for sm_100a only"
#endif

namespace nvfp4b200 {

// ---------------------------------------------------------------------------
// host-side checks shared by every entry point
// ---------------------------------------------------------------------------

// Returns NVFP4B200_OK when the current device is a compute-capability-10.0
// part (B200 family).  Cached per device; safe to call from many threads.
int check_device();

// Returns and clears the quantizer kernels' device error word (0 if none).
int take_quant_device_error();

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NVFP4B200_OK : NVFP4B200_ERR_LAUNCH;
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// ---------------------------------------------------------------------------
// numeric helpers (device)
// ---------------------------------------------------------------------------

// bf16 pair (one 32-bit word) -> two floats, exactly (shift into the high half).
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// float -> E4M3 with round-to-nearest-even and saturation to +-448, the same
// conversion instruction the reference quantizer uses (float4utils.py:64-68).
__device__ __forceinline__ uint32_t e4m3_rn_satfinite(float v) {
  uint16_t packed;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(packed) : "f"(v), "f"(v));
  return packed & 0xFFu;
}

// E4M3 code (non-negative, finite) -> float, exactly.  Integer decode:
// exponent field 0 is subnormal (m * 2^-9), otherwise (8 + m) * 2^(e - 10).
__device__ __forceinline__ float e4m3_decode(uint32_t c) {
  const uint32_t e = (c >> 3) & 0xF, m = c & 7;
  return e == 0 ? __uint_as_float(0) + (float)m * 0.001953125f
                : __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// Pack 8 floats into 8 E2M1 nibbles (low nibble = even element,
// float4utils.py:141), each nibble equal to the reference's comparison ladder
// (float4utils.py:127-139): magnitude code = #{t in {0.25,0.75,1.25,1.75,
// 2.5,3.5,5} : !(|f * inv_scale| < t)} after clamping to 6 (ties round away
// from zero, NaN gives 7), sign bit = (f < 0).
//
// The conversion instruction cvt.rn.satfinite.e2m1x2.f32 rounds to nearest
// with ties to even and saturates to +-6.  Three adjustments of its input
// make it equal to the ladder for every f32 input:
//   * p = fma(f, inv_scale, +0): the product rounded once, except that
//     f = -0.0 gives +0 (the reference's sign test f < 0 is false there),
//     while a negative product that underflows keeps its sign;
//   * bits | 1: every tie point of the E2M1 grid has a zero lowest mantissa
//     bit, so setting it moves an exact tie just above the tie (rounding away
//     from zero) and cannot move any other value across a tie;
//   * min(bits, 0xFF7FFFFF): -inf (whose "| 1" would be a NaN) becomes
//     -FLT_MAX, which saturates to -6 like the ladder; arithmetic NaN results
//     are the positive canonical NaN, which the instruction turns into +6.
// An exhaustive GPU sweep over every f32 bit pattern checks this identity.
__device__ __forceinline__ float fma_plus_zero(float a, float b) {
  float r;
  asm("fma.rn.f32 %0, %1, %2, 0f00000000;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// CLAMP = false skips the -inf adjustment; valid whenever the block amax is
// finite (then no product is -inf).
template <bool CLAMP = true>
__device__ __forceinline__ float e2m1_input(float f, float inv_scale) {
  const uint32_t b = __float_as_uint(fma_plus_zero(f, inv_scale));
  return __uint_as_float((CLAMP ? min(b, 0xFF7FFFFFu) : b) | 1u);
}
template <bool CLAMP = true>
__device__ __forceinline__ uint32_t encode8(const float* f, float inv_scale) {
  float q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = e2m1_input<CLAMP>(f[i], inv_scale);
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  return out;
}

// Block scale from a block amax (float4utils.py:109-116 with the global scale
// g folded in; g == 1 is bit-identical to the reference):
//   code      = e4m3_satfinite((amax * (1/6)) * inv_g)        (0 when amax == 0)
//   inv_scale = code decodes to s > 0 ? 1 / (s * g) : 1
__device__ __forceinline__ uint32_t block_scale(float amax, float g, float inv_g, float& inv_scale) {
  uint32_t code = 0;
  inv_scale = 1.0f;
  if (amax > 0.0f) {
    const float scale_f = (amax * (1.0f / 6.0f)) * inv_g;
    code = e4m3_rn_satfinite(scale_f);
    const float s = e4m3_decode(code);
    inv_scale = (s > 0.0f) ? __frcp_rn(s * g) : 1.0f;
  }
  return code;
}

// 16 floats (one block) -> 8 bytes of nibbles, the -inf adjustment only when
// the block amax is infinite.
__device__ __forceinline__ uint2 encode16(const float (&f)[16], float inv_scale, float amax) {
  if (amax <= 3.402823466e38f) return make_uint2(encode8<false>(f, inv_scale), encode8<false>(f + 8, inv_scale));
  return make_uint2(encode8<true>(f, inv_scale), encode8<true>(f + 8, inv_scale));
}

// E4M3 block-scale code of a block amax (float4utils.py:109-116 with the
// global scale folded in): e4m3_satfinite((amax * (1/6)) * inv_g), 0 when
// amax == 0.  The matching 1/(scale * g) comes from inv_scale_table.
__device__ __forceinline__ uint32_t block_code(float amax, float inv_g) {
  return amax > 0.0f ? e4m3_rn_satfinite((amax * (1.0f / 6.0f)) * inv_g) : 0u;
}

// Table of inv_scale for every block-scale code under global scale g:
// 1 / (decode(c) * g) rounded once (the value block_scale computes), 1 for a
// zero scale.  Filled by the CTA's threads before first use.
__device__ __forceinline__ void fill_inv_scale_table(float* tab, float g) {
  for (int c = threadIdx.x; c < 256; c += blockDim.x) {
    const float sv = e4m3_decode((uint32_t)c & 0x7Fu);
    tab[c] = sv > 0.0f ? __frcp_rn(sv * g) : 1.0f;
  }
}

// Block amax of 16 bf16 values held as 8 words: integer max of |x| bit
// patterns.  Returns the 16-bit pattern (above 0x7F80 means a NaN is present).
__device__ __forceinline__ uint32_t absmax16_bits(const uint32_t (&w)[8]) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = __vmaxu2(m, w[i] & 0x7FFF7FFFu);
  return max(m & 0xFFFFu, m >> 16);
}

// fmaxf-semantics amax over 16 floats (NaN dropped).
__device__ __forceinline__ float fmax_abs16(const float (&f)[16]) {
  float a = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) a = fmaxf(a, fabsf(f[i]));
  return a;
}

// Block amax of 8 bf16 values held as 4 words: integer max of |x| bit
// patterns (positive bf16 order like integers).  Returns the 16-bit pattern.
__device__ __forceinline__ uint32_t absmax8_bits(const uint32_t (&w)[4]) {
  uint32_t m = __vmaxu2(__vmaxu2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                        __vmaxu2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu));
  return max(m & 0xFFFFu, m >> 16);
}

// fmaxf-semantics amax (NaN dropped) over floats, used on the rare blocks
// whose integer max is a NaN pattern.
__device__ __forceinline__ float fmax_abs8(const float (&f)[8]) {
  float a = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(f[i]));
  return a;
}

// Swizzled scale byte offset (float4utils.py:118-122): atom (r/128, c/4) of
// 512 bytes; line r%32 holds the four 32-row groups x four block columns.
__device__ __forceinline__ int64_t swz_offset(int64_t r, int64_t c, int64_t pad_cols) {
  const int64_t tile = (r >> 7) * (pad_cols >> 2) + (c >> 2);
  const int64_t rin = r & 127;
  return (tile << 9) + ((rin & 31) << 4) + ((rin >> 5) << 2) + (c & 3);
}

// Offset of (r%128, c%4) inside one 512-byte atom.
__device__ __forceinline__ int atom_offset(int rin, int cin) {
  return ((rin & 31) << 4) + ((rin >> 5) << 2) + cin;
}

__device__ __forceinline__ float load_global_scale(const float* g) { return g ? *g : 1.0f; }

// ---------------------------------------------------------------------------
// global amax: block reduce + last-block finalize (all threads must call)
// ---------------------------------------------------------------------------

// ws[0]: running max of |x| as float bits (non-negative floats order like
// uint32); ws[1]: number of blocks done.  The last block turns the max into
// g = amax / (6*448) and resets both words to zero for the next call.
__device__ __forceinline__ void amax_commit(uint32_t thread_max_bits, uint32_t* ws, float* g_out, float* amax_out) {
  __shared__ uint32_t warp_max[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint32_t m = __reduce_max_sync(0xffffffffu, thread_max_bits);
  if (lane == 0) warp_max[wid] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    uint32_t bm = 0;
    for (int i = 0; i < nw; ++i) bm = max(bm, warp_max[i]);
    atomicMax(&ws[0], bm);
    __threadfence();
    const uint32_t nblocks = gridDim.x * gridDim.y * gridDim.z;
    const uint32_t done = atomicAdd(&ws[1], 1u);
    if (done == nblocks - 1) {
      __threadfence();
      const uint32_t bits = atomicExch(&ws[0], 0u);
      const float amax = __uint_as_float(bits);
      const float g = (amax > 0.0f && amax <= 3.402823466e38f) ? __fdiv_rn(amax, 2688.0f) : 1.0f;
      if (g_out) *g_out = g;
      if (amax_out) *amax_out = amax;
      __threadfence();
      atomicExch(&ws[1], 0u);
    }
  }
}


}  // namespace nvfp4b200
