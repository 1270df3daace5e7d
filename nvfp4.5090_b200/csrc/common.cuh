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

// SwiGLU backward of one element: gate g, up u, upstream gradient d (all
// bf16 values), sg = sigmoid(g).  du = d * (g * sg) and
// dg = (d * u) * (sg * (1 + g * (1 - sg))), every step rounded as written and
// 1 + g * (1 - sg) one fused multiply-add, so the element-wise kernel and the
// GEMM epilogue that both use this give identical bits.
__device__ __forceinline__ void swiglu_grad(float g, float u, float d, float sg, float& dg, float& du) {
  du = __fmul_rn(d, __fmul_rn(g, sg));
  dg = __fmul_rn(__fmul_rn(d, u), __fmul_rn(sg, __fmaf_rn(g, __fsub_rn(1.0f, sg), 1.0f)));
}

// ---------------------------------------------------------------------------
// packed f32 pairs: one 64-bit register holds two floats and each f32x2
// instruction performs two independent IEEE single-precision operations,
// with the same results as two scalar ones (round to nearest, no flush).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// a * b + (+0, +0), one rounding per lane
__device__ __forceinline__ uint64_t f2mul_plus_zero(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(0ull));
  return r;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// bf16 pair word -> {lo, hi} as a packed f32 pair, exactly
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t w) { return f2pack(bf16lo(w), bf16hi(w)); }
// swiglu_grad on two elements at once (per lane the same roundings; 1 - sg
// as fma(sg, -1, 1), one rounding of the exact difference like the subtraction)
__device__ __forceinline__ void swiglu_grad2(uint64_t g, uint64_t u, uint64_t d, uint64_t sg, uint64_t& dg,
                                             uint64_t& du) {
  const uint64_t one = f2pack(1.0f, 1.0f), neg1 = f2pack(-1.0f, -1.0f);
  du = f2mul(d, f2mul(g, sg));
  dg = f2mul(f2mul(d, u), f2mul(sg, f2fma(g, f2fma(sg, neg1, one), one)));
}

// encode8_pairs: 8 values (4 packed pairs) -> 8 E2M1 nibbles (low nibble = even element,
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
template <bool CLAMP = true>
__device__ __forceinline__ uint32_t encode8_pairs(const uint64_t* p, float inv_scale) {
  const uint64_t is2 = f2pack(inv_scale, inv_scale);
  float q[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t r = f2mul_plus_zero(p[j], is2);
    const uint32_t lo = __float_as_uint(f2lo(r)), hi = __float_as_uint(f2hi(r));
    q[2 * j] = __uint_as_float((CLAMP ? min(lo, 0xFF7FFFFFu) : lo) | 1u);
    q[2 * j + 1] = __uint_as_float((CLAMP ? min(hi, 0xFF7FFFFFu) : hi) | 1u);
  }
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
// 8 packed pairs (one block) -> 8 bytes of nibbles; -inf adjustment only for an infinite amax.
__device__ __forceinline__ uint2 encode16_pairs(const uint64_t (&p)[8], float inv_scale, float amax) {
  if (amax <= 3.402823466e38f) return make_uint2(encode8_pairs<false>(p, inv_scale), encode8_pairs<false>(p + 4, inv_scale));
  return make_uint2(encode8_pairs<true>(p, inv_scale), encode8_pairs<true>(p + 4, inv_scale));
}
// Two output rows at once: p[t] = {row a value t, row b value t} for t < 16
// (a block of each row).  Returns the nibbles of row a (x) and row b (y)
// with per-row inverse scales; the -inf adjustment only when a block amax is
// infinite.
__device__ __forceinline__ void encode16_two_rows(const uint64_t (&p)[16], float inv_a, float inv_b, float amax_a,
                                                  float amax_b, uint2& out_a, uint2& out_b) {
  const uint64_t is2 = f2pack(inv_a, inv_b);
  const bool clamp = !(amax_a <= 3.402823466e38f) || !(amax_b <= 3.402823466e38f);
  float qa[16], qb[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const uint64_t r = f2mul_plus_zero(p[t], is2);
    uint32_t lo = (uint32_t)r, hi = (uint32_t)(r >> 32);
    if (clamp) {
      lo = min(lo, 0xFF7FFFFFu);
      hi = min(hi, 0xFF7FFFFFu);
    }
    qa[t] = __uint_as_float(lo | 1u);
    qb[t] = __uint_as_float(hi | 1u);
  }
  uint32_t w[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float* q = h < 2 ? qa + 8 * h : qb + 8 * (h - 2);
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
        "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
        : "=r"(w[h])
        : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  }
  out_a = make_uint2(w[0], w[1]);
  out_b = make_uint2(w[2], w[3]);
}

// fmaxf-semantics amax over 8 packed pairs (NaN dropped).
__device__ __forceinline__ float fmax_abs16_pairs(const uint64_t (&p)[8]) {
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) a = fmaxf(a, fmaxf(fabsf(f2lo(p[j])), fabsf(f2hi(p[j]))));
  return a;
}

// E4M3 block-scale code of a block amax (float4utils.py:109-116 with the
// global scale folded in): e4m3_satfinite((amax * (1/6)) * inv_g), 0 when
// amax == 0.  The matching 1/(scale * g) comes from inv_scale_table.
__device__ __forceinline__ uint32_t block_code(float amax, float inv_g) {
  return amax > 0.0f ? e4m3_rn_satfinite((amax * (1.0f / 6.0f)) * inv_g) : 0u;
}

// Table of inv_scale for every block-scale code under global scale g:
// 1 / (decode(c) * g) rounded once (float4utils.py:114-116 with g folded in), 1
// for a zero scale.  Filled by the CTA's threads before first use.
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
