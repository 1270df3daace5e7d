// NVFP4 quantizers for B200 (sm_100a): plain / scaled, fused RMSNorm,
// transposed, and the global-amax reduction.
//
// All kernels are HBM-bound.  The per-element arithmetic follows the
// reference quantizer (float4utils.py:79-148): block amax with fmaxf
// semantics, E4M3 block scale by cvt.rn.satfinite, reciprocal-then-multiply,
// the away-from-zero E2M1 ladder, low-nibble-first packing and the 128x4
// swizzled scale layout -- see common.cuh for each helper.  What differs is
// the data movement: warps read 512 contiguous bytes per instruction and
// write 256 contiguous bytes of nibbles (the transposed quantizer stages a
// tile's nibbles in shared memory and writes whole 32-byte sectors), and
// scale atoms are staged in shared memory and written as whole 512-byte
// atoms, so no separate zero-fill of the scale tensor is needed.
#include "common.cuh"

#include <cuda.h>

#include <algorithm>
#include <mutex>

namespace nvfp4b200 {

// ---------------------------------------------------------------------------
// device check (shared by every entry point)
// ---------------------------------------------------------------------------

int check_device() {
  static std::mutex mu;
  static int cached[64];
  static bool init[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  if (dev < 0 || dev >= 64) return NVFP4B200_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lk(mu);
  if (!init[dev]) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return NVFP4B200_ERR_CUDA;
    cached[dev] = (major == 10 && minor == 0) ? NVFP4B200_OK : NVFP4B200_ERR_UNSUPPORTED_DEVICE;
    init[dev] = true;
  }
  return cached[dev];
}

// ---------------------------------------------------------------------------
// global amax: block reduce + last-block finalize
// ---------------------------------------------------------------------------

// |x| max of 8 bf16 (4 words) as float bits, NaN ignored.
__device__ __forceinline__ uint32_t absmax8_nonan_f32bits(const uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t a = w[i] & 0x7FFF7FFFu;
    const uint32_t nan = __vcmpgtu2(a, 0x7F807F80u);  // 0xFFFF per NaN half
    a &= ~nan;
    m = __vmaxu2(m, a);
  }
  return max(m & 0xFFFFu, m >> 16) << 16;
}

__global__ void __launch_bounds__(256) global_amax_kernel(const uint4* __restrict__ x, int64_t n_vec,
                                                          const uint16_t* __restrict__ tail, int n_tail,
                                                          uint32_t* ws, float* g_out, float* amax_out) {
  uint32_t m = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n_vec; i += 4 * stride) {
    const uint4 a = __ldg(x + i), b = __ldg(x + i + stride), c = __ldg(x + i + 2 * stride),
                d = __ldg(x + i + 3 * stride);
    m = max(m, max(max(absmax8_nonan_f32bits(a), absmax8_nonan_f32bits(b)),
                   max(absmax8_nonan_f32bits(c), absmax8_nonan_f32bits(d))));
  }
  for (; i < n_vec; i += stride) m = max(m, absmax8_nonan_f32bits(__ldg(x + i)));
  if (blockIdx.x == 0 && (int)threadIdx.x < n_tail) {
    uint32_t a = tail[threadIdx.x] & 0x7FFFu;
    if (a <= 0x7F80u) m = max(m, a << 16);
  }
  amax_commit(m, ws, g_out, amax_out);
}

// ---------------------------------------------------------------------------
// tile quantizer: 128 rows x 512 columns per CTA
// ---------------------------------------------------------------------------
// Each lane owns one 16-element block column of the tile (32 B of every row);
// a warp covers 16 rows, read 2 rows per pass with the next pass's loads in
// flight while the current one is encoded.  Per row a warp reads 1 KB and
// writes 256 B of nibbles; the tile's 8 scale atoms (4 KB, contiguous in the
// swizzled layout) are staged in shared memory and written whole.

constexpr int QT_ROWS = 128;
constexpr int QT_COLS = 512;       // 32 blocks = 8 scale atoms
constexpr int QT_THREADS = 256;    // 8 warps x 16 rows


// The scaled variants (row scale and / or gamma) keep 2 rows per pass: at
// 80 registers and 3 CTAs per SM that was +34% over 4 rows per pass at 131
// registers (2 CTAs per SM), where each CTA's cold first load was exposed.
// Both kinds are capped at 64 registers for 4 CTAs per SM: the plain variant
// without spills (+3% at 32768 x 4096 and 16384 x 8192 over 68 registers and
// 3 CTAs), the scaled ones with 84 bytes of spills (+3% over 80 registers and
// 3 CTAs at those shapes; small inputs of a few hundred rows lose ~5%).
template <bool HAS_ROW, bool HAS_GAMMA>
__global__ void __launch_bounds__(QT_THREADS, 4) quant_tile_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ row_scale,
    const uint16_t* __restrict__ gamma, uint8_t* __restrict__ q, uint8_t* __restrict__ s,
    int64_t rows, int64_t k, int64_t pad_cols, const float* __restrict__ gptr, int q8) {
  constexpr int QT_PASS = 2;  // rows per pipelined pass
  __shared__ __align__(16) uint8_t s_tile[8 * 512];
  __shared__ float inv_tab[256];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t tile_r0 = (int64_t)blockIdx.y * QT_ROWS;
  const int64_t col = (int64_t)blockIdx.x * QT_COLS + 16 * lane;  // this lane's block
  const bool col_ok = col < k;                                    // k % 16 == 0: all or nothing
  const float g = load_global_scale(gptr);
  const float inv_g = __frcp_rn(g);
  fill_inv_scale_table(inv_tab, g);

  uint64_t gam[8];   // gamma as packed pairs
  if (HAS_GAMMA) {
    uint4 ga = make_uint4(0, 0, 0, 0), gb = ga;
    if (col_ok) {
      ga = __ldg(reinterpret_cast<const uint4*>(gamma + col));
      gb = __ldg(reinterpret_cast<const uint4*>(gamma + col) + 1);
    }
    const uint32_t gw[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) gam[j] = bf16x2_to_f2(gw[j]);
  }
  __syncthreads();  // inv_tab

  auto load_pass = [&](int pass, uint4 (&buf)[QT_PASS][2]) {
#pragma unroll
    for (int i = 0; i < QT_PASS; ++i) {
      const int64_t r = tile_r0 + wid * 16 + pass * QT_PASS + i;
      buf[i][0] = make_uint4(0, 0, 0, 0);
      buf[i][1] = buf[i][0];
      if (col_ok && r < rows) {
        const uint4* p = reinterpret_cast<const uint4*>(x + r * k + col);
        buf[i][0] = __ldg(p);
        buf[i][1] = __ldg(p + 1);
      }
    }
  };
  uint4 cur[QT_PASS][2], nxt[QT_PASS][2];
  load_pass(0, cur);
#pragma unroll
  for (int pass = 0; pass < 16 / QT_PASS; ++pass) {
    if (pass + 1 < 16 / QT_PASS) load_pass(pass + 1, nxt);
#pragma unroll
    for (int i = 0; i < QT_PASS; ++i) {
      const int rl = wid * 16 + pass * QT_PASS + i;  // row inside the tile
      const int64_t r = tile_r0 + rl;
      const bool ok = col_ok && r < rows;
      const uint32_t w[8] = {cur[i][0].x, cur[i][0].y, cur[i][0].z, cur[i][0].w,
                             cur[i][1].x, cur[i][1].y, cur[i][1].z, cur[i][1].w};
      uint64_t f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = bf16x2_to_f2(w[j]);
      float amax;
      if (HAS_ROW || HAS_GAMMA) {
        const float rs = HAS_ROW ? (r < rows ? __ldg(row_scale + r) : 0.0f) : 1.0f;
        const uint64_t rs2 = f2pack(rs, rs);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (HAS_ROW) f[j] = f2mul(f[j], rs2);
          if (HAS_GAMMA) f[j] = f2mul(f[j], gam[j]);
        }
        amax = fmax_abs16_pairs(f);
      } else {
        const uint32_t mb = absmax16_bits(w);
        amax = (mb > 0x7F80u) ? fmax_abs16_pairs(f) : __uint_as_float(mb << 16);
      }
      const uint32_t code = ok ? block_code(amax, inv_g) : 0u;
      const uint2 packed = encode16_pairs(f, inv_tab[code], amax);
      if (ok) {
        uint8_t* dst = q + r * (k >> 1) + (col >> 1);
        if (q8) {
          *reinterpret_cast<uint2*>(dst) = packed;
        } else {
          reinterpret_cast<uint32_t*>(dst)[0] = packed.x;
          reinterpret_cast<uint32_t*>(dst)[1] = packed.y;
        }
      }
      s_tile[(lane >> 2) * 512 + atom_offset(rl, lane & 3)] = (uint8_t)code;
    }
    if (pass + 1 < 16 / QT_PASS) {
#pragma unroll
      for (int i = 0; i < QT_PASS; ++i) { cur[i][0] = nxt[i][0]; cur[i][1] = nxt[i][1]; }
    }
  }
  __syncthreads();
  // the (up to) 8 atoms of this tile: contiguous 4 KB of the swizzled tensor
  const int64_t atom0 = (int64_t)blockIdx.x * 8;
  const int64_t n_atoms = imin64(8, (pad_cols >> 2) - atom0);
  const int64_t dst = ((int64_t)blockIdx.y * (pad_cols >> 2) + atom0) * 512;
  if ((int64_t)threadIdx.x * 16 < n_atoms * 512)
    *reinterpret_cast<uint4*>(s + dst + threadIdx.x * 16) = reinterpret_cast<const uint4*>(s_tile)[threadIdx.x];
}

// ---------------------------------------------------------------------------
// fused RMSNorm -> quantize: reduction helpers
// ---------------------------------------------------------------------------
// One warp handles a row; lane L of the warp owns the 16-element blocks c = 32 j + L (chunk j of 512
// columns).  The sum of squares reproduces the reference's fp32 order exactly
// (float4utils.py:183-222, 256 threads per row): thread t accumulates
// ``sum_sq += a0 * a0 + a1 * a1`` over its blocks t, t + 256, ... word by
// word; each warp of 32 threads reduces with shfl_down 16, 8, 4, 2, 1; the 8
// warp sums are reduced the same way by warp 0.  Here virtual thread
// t = 32 m + L is lane L's partial sum m = j mod 8, the 8 warp trees are run
// on the 8 partials, and the last tree over 8 values (the other 24 lanes hold
// 0) is written out in registers.

constexpr int RMS_WARPS = 4;

// Sum of squares of one 16-element block, accumulated into `acc` in the
// reference's order.
__device__ __forceinline__ float sumsq_block(float acc, const uint4 v0, const uint4 v1) {
  const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a0 = bf16lo(w[i]), a1 = bf16hi(w[i]);
    acc += a0 * a0 + a1 * a1;
  }
  return acc;
}

// The reference's two-level shfl_down reduction of the 256 per-thread sums,
// given lane L's partial sums for threads L, 32 + L, ..., 224 + L.  Result
// valid in every lane.
__device__ __forceinline__ float reduce_like_reference(float (&ps)[8]) {
#pragma unroll
  for (int m = 0; m < 8; ++m) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps[m] += __shfl_down_sync(0xffffffffu, ps[m], off);
  }
  // warp 0's tree over (s0..s7, 0, ..., 0): offsets 16 and 8 add zeros
  const float t0 = (ps[0] + 0.0f) + ps[4], t1 = (ps[1] + 0.0f) + ps[5];
  const float t2 = (ps[2] + 0.0f) + ps[6], t3 = (ps[3] + 0.0f) + ps[7];
  const float total = (t0 + t2) + (t1 + t3);
  return __shfl_sync(0xffffffffu, total, 0);
}

// 1/RMS for rows wider than the row kernel covers (k > 16384): one warp per row,
// the same per-thread order and reduction tree.
__global__ void __launch_bounds__(RMS_WARPS * 32) rms_inv_stream_kernel(
    const uint16_t* __restrict__ x, float* __restrict__ inv_rms, int64_t rows, int64_t k, float eps) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * RMS_WARPS + wid;
  if (r >= rows) return;
  const int64_t nblk = k >> 4;
  float ps[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) ps[m] = 0.0f;
  for (int64_t j0 = 0; 32 * j0 < nblk; j0 += 8) {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int64_t c = 32 * (j0 + m) + lane;
      if (c < nblk) {
        const uint4* p = reinterpret_cast<const uint4*>(x + r * k + 16 * c);
        ps[m] = sumsq_block(ps[m], __ldg(p), __ldg(p + 1));
      }
    }
  }
  const float inv = rsqrtf((reduce_like_reference(ps) / (float)k) + eps);
  if (lane == 0) inv_rms[r] = inv;
}

// ---------------------------------------------------------------------------
// RMSNorm rows: one CTA per row, the reference's thread layout
// ---------------------------------------------------------------------------
// Thread t of a CTA owns the blocks c = t, t + 256, ... of the row, exactly
// as the reference kernel (float4utils.py:169-295, 256 threads per row), so
// the sum of squares, the per-warp shfl_down tree and the cross-warp tree are
// the reference's own and 1/RMS is bit-identical.  CTAs are persistent and
// keep the next row's loads in flight in registers while the current row is
// reduced and quantized.  A CTA has min(256, padded blocks) threads; threads
// the reference has beyond that hold no blocks and add zeros to the trees.
// Every thread keeps its blocks' floats between the reduction and the
// quantization.  Block codes of threads 4i..4i+3 form one 32-bit word of the
// swizzled scale layout.

__device__ int g_quant_error = 0;

template <int BPT, bool HAS_GAMMA>
__global__ void __launch_bounds__(256) rmsnorm_cta_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma, uint8_t* __restrict__ q,
    uint8_t* __restrict__ s, float* __restrict__ inv_rms_out, int64_t rows, int64_t pad_rows, int64_t k,
    int64_t pad_cols, float eps, const float* __restrict__ gptr, int q8) {
  __shared__ float warp_sum[8];
  __shared__ float row_inv;
  __shared__ float inv_tab[256];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int nwarps = blockDim.x >> 5;
  const int64_t nblk = k >> 4;
  const int64_t cover = pad_rows;
  const float g = load_global_scale(gptr);
  const float inv_g = __frcp_rn(g);
  fill_inv_scale_table(inv_tab, g);
  uint64_t gam[BPT][8];   // gamma as packed pairs
  if (HAS_GAMMA) {
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      const int64_t c = t + 256 * b;
      uint4 g0 = make_uint4(0, 0, 0, 0), g1 = g0;
      if (c < nblk) {
        const uint4* gp = reinterpret_cast<const uint4*>(gamma + 16 * c);
        g0 = __ldg(gp);
        g1 = __ldg(gp + 1);
      }
      const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) gam[b][j] = bf16x2_to_f2(gw[j]);
    }
  }
  auto load_row = [&](int64_t r, uint4 (&buf)[BPT][2]) {
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      const int64_t c = t + 256 * b;
      buf[b][0] = make_uint4(0, 0, 0, 0);
      buf[b][1] = buf[b][0];
      if (r < rows && c < nblk) {
        const uint4* p = reinterpret_cast<const uint4*>(x + r * k + 16 * c);
        buf[b][0] = __ldg(p);
        buf[b][1] = __ldg(p + 1);
      }
    }
  };
  uint4 cur[BPT][2], nxt[BPT][2];
  int64_t r = blockIdx.x;
  load_row(r, cur);
  __syncthreads();  // inv_tab
  for (; r < cover; r += gridDim.x) {
    load_row(r + gridDim.x, nxt);
    if (r >= rows) {  // padding row of the scale tensor: zero codes
      for (int64_t c = 4 * t; c < pad_cols; c += 4 * blockDim.x)
        *reinterpret_cast<uint32_t*>(s + swz_offset(r, c, pad_cols)) = 0u;
      continue;
    }
    uint64_t f[BPT][8];
    float ss = 0.0f;
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      const uint32_t w[8] = {cur[b][0].x, cur[b][0].y, cur[b][0].z, cur[b][0].w,
                             cur[b][1].x, cur[b][1].y, cur[b][1].z, cur[b][1].w};
#pragma unroll
      for (int j = 0; j < 8; ++j) f[b][j] = bf16x2_to_f2(w[j]);
      if (t + 256 * b < nblk) {
        // ``ss += a0 * a0 + a1 * a1`` (the squares of bf16 values are exact in fp32, so
        // the packed product gives the reference's terms bit for bit)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t sq = f2mul(f[b][j], f[b][j]);
          ss += f2lo(sq) + f2hi(sq);
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_down_sync(0xffffffffu, ss, off);
    if (lane == 0) warp_sum[wid] = ss;
    __syncthreads();
    if (wid == 0) {   // the reference's final tree over the warp sums
      float v = (lane < nwarps) ? warp_sum[lane] : 0.0f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
      if (lane == 0) {
        const float iv = rsqrtf((v / (float)k) + eps);
        row_inv = iv;
        if (inv_rms_out) inv_rms_out[r] = iv;
      }
    }
    __syncthreads();
    const float inv = row_inv;
    const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      const int64_t c = t + 256 * b;
      const bool in = c < nblk;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        f[b][j] = f2mul(f[b][j], inv2);
        if (HAS_GAMMA) f[b][j] = f2mul(f[b][j], gam[b][j]);
      }
      const float amax = in ? fmax_abs16_pairs(f[b]) : 0.0f;
      const uint32_t code = in ? block_code(amax, inv_g) : 0u;
      const uint2 packed = encode16_pairs(f[b], inv_tab[code], amax);
      if (in) {
        uint8_t* dst = q + r * (k >> 1) + 8 * c;
        if (q8) {
          *reinterpret_cast<uint2*>(dst) = packed;
        } else {
          reinterpret_cast<uint32_t*>(dst)[0] = packed.x;
          reinterpret_cast<uint32_t*>(dst)[1] = packed.y;
        }
      }
      const uint32_t c1 = __shfl_down_sync(0xffffffffu, code, 1);
      const uint32_t c2 = __shfl_down_sync(0xffffffffu, code, 2);
      const uint32_t c3 = __shfl_down_sync(0xffffffffu, code, 3);
      if ((lane & 3) == 0 && c < pad_cols)
        *reinterpret_cast<uint32_t*>(s + swz_offset(r, c, pad_cols)) = code | (c1 << 8) | (c2 << 16) | (c3 << 24);
    }
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      cur[b][0] = nxt[b][0];
      cur[b][1] = nxt[b][1];
    }
  }
}

// ---------------------------------------------------------------------------
// row statistics of the global-scale RMSNorm path (no reference counterpart)
// ---------------------------------------------------------------------------
// inv_rms[r] and the amax of (x * inv_rms) * gamma over the whole tensor.  The
// path has no reference counterpart, so the sum of squares is free of the
// reference's reduction order: each thread accumulates its 16-element blocks
// (t, t + 256, ...) in a packed pair of fp32 sums with fma.f32x2, warps reduce
// with butterflies, and every thread adds the 8 warp sums in the same fixed
// order, so all threads hold the same 1/RMS after one CTA barrier per row
// (partials double-buffered across rows).  1/RMS agrees with the
// reference-order kernel to ~1 ulp.  Persistent CTAs (as many as fit) keep
// DEPTH rows in flight ahead of the one being reduced and re-read gamma from
// L1 where that frees registers: with one 32-byte slice per thread (k <= 4096)
// two rows ahead at 4 CTAs per SM measured 66 us vs 90 us for one row ahead at
// 32768 x 4096; wider rows already keep 64+ bytes per thread in flight and stay
// at one row ahead (16384 x 8192: 67.6 us either way).
template <int BPT, bool HAS_GAMMA, int DEPTH, bool GAMMA_L1>
__global__ void __launch_bounds__(256, BPT == 1 ? 4 : 1) rms_stats_kernel(const uint16_t* __restrict__ x,
                                                                        const uint16_t* __restrict__ gamma,
                                                                        float* __restrict__ inv_rms_out, int64_t rows,
                                                                        int64_t k, float eps, uint32_t* ws,
                                                                        float* g_out) {
  __shared__ float red[2][8];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int64_t nblk = k >> 4;
  uint64_t gam[GAMMA_L1 ? 1 : BPT][8];
  auto load_gamma = [&](int b, uint32_t (&gw)[8]) {
    const int64_t c = t + 256 * b;
    uint4 g0 = make_uint4(0, 0, 0, 0), g1 = g0;
    if (c < nblk) {
      const uint4* gp = reinterpret_cast<const uint4*>(gamma + 16 * c);
      g0 = __ldg(gp);
      g1 = __ldg(gp + 1);
    }
    gw[0] = g0.x; gw[1] = g0.y; gw[2] = g0.z; gw[3] = g0.w;
    gw[4] = g1.x; gw[5] = g1.y; gw[6] = g1.z; gw[7] = g1.w;
  };
  if (HAS_GAMMA && !GAMMA_L1) {
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      uint32_t gw[8];
      load_gamma(b, gw);
#pragma unroll
      for (int j = 0; j < 8; ++j) gam[b][j] = bf16x2_to_f2(gw[j]);
    }
  }
  auto load_row = [&](int64_t r, uint4 (&buf)[BPT][2]) {
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      const int64_t c = t + 256 * b;
      buf[b][0] = make_uint4(0, 0, 0, 0);
      buf[b][1] = buf[b][0];
      if (r < rows && c < nblk) {
        const uint4* p = reinterpret_cast<const uint4*>(x + r * k + 16 * c);
        buf[b][0] = __ldg(p);
        buf[b][1] = __ldg(p + 1);
      }
    }
  };
  const float inv_k = 1.0f / (float)k;
  const int64_t G = gridDim.x;
  float am = 0.0f;
  uint4 buf[DEPTH + 1][BPT][2];   // buf[0]: the row being reduced; buf[1..DEPTH]: rows in flight
  int64_t r = blockIdx.x;
#pragma unroll
  for (int d = 0; d < DEPTH; ++d) load_row(r + d * G, buf[d]);
  for (int it = 0; r < rows; r += G, ++it) {
    load_row(r + DEPTH * G, buf[DEPTH]);
    uint64_t acc = 0;   // packed (0.0f, 0.0f)
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      const uint32_t w[8] = {buf[0][b][0].x, buf[0][b][0].y, buf[0][b][0].z, buf[0][b][0].w,
                             buf[0][b][1].x, buf[0][b][1].y, buf[0][b][1].z, buf[0][b][1].w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint64_t f = bf16x2_to_f2(w[j]);
        acc = f2fma(f, f, acc);   // out-of-range blocks were loaded as zeros
      }
    }
    float ss = f2lo(acc) + f2hi(acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[it & 1][wid] = ss;
    __syncthreads();
    const float* rw = red[it & 1];
    const float tot = ((rw[0] + rw[1]) + (rw[2] + rw[3])) + ((rw[4] + rw[5]) + (rw[6] + rw[7]));
    const float inv = rsqrtf(tot * inv_k + eps);
    if (t == 0) inv_rms_out[r] = inv;
    const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
    for (int b = 0; b < BPT; ++b) {
      if (t + 256 * b >= nblk) continue;
      const uint32_t w[8] = {buf[0][b][0].x, buf[0][b][0].y, buf[0][b][0].z, buf[0][b][0].w,
                             buf[0][b][1].x, buf[0][b][1].y, buf[0][b][1].z, buf[0][b][1].w};
      uint32_t gw[8];
      if (HAS_GAMMA && GAMMA_L1) load_gamma(b, gw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint64_t y = f2mul(bf16x2_to_f2(w[j]), inv2);
        if (HAS_GAMMA) y = f2mul(y, GAMMA_L1 ? bf16x2_to_f2(gw[j]) : gam[b][j]);
        am = fmaxf(am, fmaxf(fabsf(f2lo(y)), fabsf(f2hi(y))));
      }
    }
#pragma unroll
    for (int d = 0; d < DEPTH; ++d) {
#pragma unroll
      for (int b = 0; b < BPT; ++b) {
        buf[d][b][0] = buf[d + 1][b][0];
        buf[d][b][1] = buf[d + 1][b][1];
      }
    }
  }
  amax_commit(__float_as_uint(am), ws, g_out, nullptr);
}

// ---------------------------------------------------------------------------
// transposed quantizer: x [rows, cols] -> quantize x^T along rows
// ---------------------------------------------------------------------------
// Persistent CTAs walk 128 x 128 input tiles (input rows t0.., input columns
// d0..).  Thread 0 keeps the next tile's TMA load (and its 128 row scales)
// in flight into the other half of a double buffer while all 256 threads
// encode the current one: thread (qtr, p) owns output rows d0 + 2p, 2p + 1
// (input columns) and the blocks 2 qtr, 2 qtr + 1 of the tile (input rows
// t0 + 32 qtr .. + 32), reads its column pair down the tile (a warp reads 128
// contiguous bytes of a tile row) and produces 16 bytes of nibbles per output
// row.  The nibbles (staged in the tile's input buffer once it is read) and
// the tile's 2 scale atoms (1 KB) go out whole from shared memory, the
// buffer's next load after that.  Waits are bounded; a timeout sets
// g_quant_error.

constexpr int TQ_T = 128;                  // input rows per tile = output k extent (8 blocks)
constexpr int TQ_D = 128;                  // input columns per tile = output rows
constexpr int TQ_TILE_BYTES = TQ_T * TQ_D * 2;
constexpr long long TQ_WAIT_LIMIT = 4000000000LL;

struct TqSmem {
  uint16_t tile[2][TQ_T * TQ_D];
  float rs[2][TQ_T];
  uint8_t atoms[2][2 * 512];
  float inv_tab[256];
  uint64_t full[2];
};

__device__ __forceinline__ uint32_t tq_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool tq_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

template <bool HAS_ROW, bool HAS_GAMMA>
__global__ void __launch_bounds__(256, 3) quant_t_kernel(
    const __grid_constant__ CUtensorMap xmap, const float* __restrict__ row_scale,
    const uint16_t* __restrict__ gamma, uint8_t* __restrict__ q, uint8_t* __restrict__ s, int64_t rows,
    int64_t cols, int64_t pad_cols_out, int n_tiles_t, int n_tiles, const float* __restrict__ gptr, int q16) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  TqSmem& sm = *reinterpret_cast<TqSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int p = tid & 63;      // column pair
  const int qtr = tid >> 6;    // blocks 2 qtr, 2 qtr + 1
  const int dl0 = 2 * p;
  const float g = load_global_scale(gptr);
  const float inv_g = __frcp_rn(g);
  fill_inv_scale_table(sm.inv_tab, g);

  auto issue = [&](int tile, int buf) {  // thread 0
    const int64_t t0 = (int64_t)(tile % n_tiles_t) * TQ_T;
    const int64_t d0 = (int64_t)(tile / n_tiles_t) * TQ_D;
    const uint32_t bar = tq_smem(&sm.full[buf]);
    uint32_t bytes = TQ_TILE_BYTES;
    int64_t nrs = 0;
    if (HAS_ROW) {
      nrs = imin64(TQ_T, rows - t0);
      if (nrs > 0) bytes += (uint32_t)(nrs * 4);
    }
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            tq_smem(sm.tile[buf])),
        "l"(&xmap), "r"((int)d0), "r"((int)t0), "r"(bar)
        : "memory");
    if (HAS_ROW && nrs > 0)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       tq_smem(sm.rs[buf])),
                   "l"(row_scale + t0), "r"((uint32_t)(nrs * 4)), "r"(bar)
                   : "memory");
  };
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tq_smem(&sm.full[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tq_smem(&sm.full[1])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
    if ((int)blockIdx.x < n_tiles) issue(blockIdx.x, 0);
    if ((int)blockIdx.x + (int)gridDim.x < n_tiles) issue(blockIdx.x + gridDim.x, 1);
  }
  __syncthreads();  // barriers initialised, inv_tab filled

  bool ok = true;
  int it = 0;
  for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
    const int buf = it & 1;
    const int64_t t0 = (int64_t)(tile % n_tiles_t) * TQ_T;
    const int64_t d0 = (int64_t)(tile / n_tiles_t) * TQ_D;
    {
      const uint32_t bar = tq_smem(&sm.full[buf]);
      const uint32_t par = (uint32_t)((it >> 1) & 1);
      bool done = tq_try_wait(bar, par);
      const long long w0 = clock64();
      while (!done && clock64() - w0 < TQ_WAIT_LIMIT) done = tq_try_wait(bar, par);
      ok = __syncthreads_and(done);
      if (!ok) break;
    }
    const uint16_t* tl = sm.tile[buf];
    float gam0 = 1.0f, gam1 = 1.0f;
    if (HAS_GAMMA) {
      if (d0 + dl0 < cols) gam0 = __uint_as_float((uint32_t)gamma[d0 + dl0] << 16);
      if (d0 + dl0 + 1 < cols) gam1 = __uint_as_float((uint32_t)gamma[d0 + dl0 + 1] << 16);
    }
    const uint64_t gam2 = f2pack(gam0, gam1);
    uint32_t qwa[4], qwb[4];
    uint32_t codes_a = 0, codes_b = 0;
#pragma unroll
    for (int bi = 0; bi < 2; ++bi) {
      const int b = 2 * qtr + bi;
      uint64_t pr[16];   // {output row dl0, output row dl0 + 1} at input row t
      float ama = 0.0f, amb = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = b * 16 + j;
        pr[j] = bf16x2_to_f2(*reinterpret_cast<const uint32_t*>(tl + t * TQ_D + dl0));
        if (HAS_ROW) {
          const float rsv = sm.rs[buf][t];
          pr[j] = f2mul(pr[j], f2pack(rsv, rsv));
        }
        if (HAS_GAMMA) pr[j] = f2mul(pr[j], gam2);
        ama = fmaxf(ama, fabsf(f2lo(pr[j])));
        amb = fmaxf(amb, fabsf(f2hi(pr[j])));
      }
      const bool blk_ok = t0 + b * 16 < rows;   // rows % 16 == 0: a block is all in or all out
      const uint32_t ca = blk_ok ? block_code(ama, inv_g) : 0u;
      const uint32_t cb = blk_ok ? block_code(amb, inv_g) : 0u;
      uint2 pa, pb;
      encode16_two_rows(pr, sm.inv_tab[ca], sm.inv_tab[cb], ama, amb, pa, pb);
      qwa[2 * bi] = pa.x;
      qwa[2 * bi + 1] = pa.y;
      qwb[2 * bi] = pb.x;
      qwb[2 * bi + 1] = pb.y;
      codes_a |= ca << (8 * bi);
      codes_b |= cb << (8 * bi);
    }
    __syncthreads();  // every thread is done reading this buffer
    // The tile's nibbles (128 output rows x 64 bytes: 16 per thread and row, at
    // byte column 16 qtr) are staged in the input buffer just read, 16-byte
    // column c of row r at c ^ ((r >> 1) & 3) (at most 2-way bank conflicts on
    // the way in, none on the way out), and leave below as whole 32-byte
    // sectors, two threads per output row: +3% (row scale + gamma) and +6%
    // (plain) at 32768 x 4096 over each thread writing its 16-byte pieces of
    // 128 output rows directly.  The buffer's next load goes out once the
    // staged bytes are read.
    {
      uint8_t* nib = reinterpret_cast<uint8_t*>(sm.tile[buf]);
      const uint32_t* qw[2] = {qwa, qwb};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = dl0 + h;
        const int c = qtr ^ ((r >> 1) & 3);
        *reinterpret_cast<uint4*>(nib + r * 64 + c * 16) = make_uint4(qw[h][0], qw[h][1], qw[h][2], qw[h][3]);
      }
    }
    // scale codes: output row dl, blocks 2 qtr, 2 qtr + 1 = atom qtr / 2, columns (2 qtr) % 4 + 0, 1
    uint8_t* at = sm.atoms[buf] + (qtr >> 1) * 512;
    const int c0 = (2 * qtr) & 3;
    *reinterpret_cast<uint16_t*>(at + atom_offset(dl0, c0)) = (uint16_t)((d0 + dl0 < cols) ? codes_a : 0u);
    *reinterpret_cast<uint16_t*>(at + atom_offset(dl0 + 1, c0)) = (uint16_t)((d0 + dl0 + 1 < cols) ? codes_b : 0u);
    __syncthreads();
    const int64_t atom0 = (int64_t)(tile % n_tiles_t) * 2;
    const int64_t n_atoms = imin64(2, (pad_cols_out >> 2) - atom0);
    const int64_t dst = ((int64_t)(tile / n_tiles_t) * (pad_cols_out >> 2) + atom0) * 512;
    if ((int64_t)tid * 4 < n_atoms * 512)
      *reinterpret_cast<uint32_t*>(s + dst + tid * 4) = reinterpret_cast<const uint32_t*>(sm.atoms[buf])[tid];
    {
      // thread tid writes output row d0 + tid / 2, bytes [32 (tid & 1), +32) of the tile's 64
      const int r = tid >> 1, hb = tid & 1;
      const uint8_t* nib = reinterpret_cast<const uint8_t*>(sm.tile[buf]);
      const int64_t orow = d0 + r;
      const int64_t bcol = (t0 >> 1) + 32 * hb;            // byte column in the output row
      const int64_t avail = (rows >> 1) - bcol;             // bytes of this half inside the row (a multiple of 8)
      if (orow < cols && avail > 0) {
        uint8_t* dstp = q + orow * (rows >> 1) + bcol;
        const int ca = (2 * hb) ^ ((r >> 1) & 3), cb = (2 * hb + 1) ^ ((r >> 1) & 3);
        const uint4 va = *reinterpret_cast<const uint4*>(nib + r * 64 + ca * 16);
        const uint4 vb = *reinterpret_cast<const uint4*>(nib + r * 64 + cb * 16);
        if (avail >= 32 && q16) {
          reinterpret_cast<uint4*>(dstp)[0] = va;
          reinterpret_cast<uint4*>(dstp)[1] = vb;
        } else {   // 8-byte granules: output rows only 8-byte aligned, or the row ends inside this half
          const uint2 w[4] = {make_uint2(va.x, va.y), make_uint2(va.z, va.w), make_uint2(vb.x, vb.y),
                              make_uint2(vb.z, vb.w)};
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (avail >= 8 * (i + 1)) reinterpret_cast<uint2*>(dstp)[i] = w[i];
        }
      }
    }
    __syncthreads();   // the staged nibbles are read before the buffer is loaded again
    if (tid == 0 && tile + 2 * (int)gridDim.x < n_tiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(tile + 2 * gridDim.x, buf);
    }
  }
  if (!ok && tid == 0) {
    atomicExch(&g_quant_error, NVFP4B200_ERR_TIMEOUT);
    const long long w0 = clock64();  // let loads still in flight land before the CTA exits
    for (int b = 0; b < 2; ++b)
      for (uint32_t par = 0; par < 2; ++par)
        while (!tq_try_wait(tq_smem(&sm.full[b]), par) && clock64() - w0 < TQ_WAIT_LIMIT) {
        }
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFnQ)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D bf16 tensor [rows, cols] (row stride cols) with box {box_cols, box_rows},
// no swizzle; loads outside the tensor read zeros.
static bool make_bf16_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  static EncodeTiledFnQ fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnQ>(ptr);
  });
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


static int launch_quant_tile(const void* x, const float* row_scale, const void* gamma, void* q,
                             void* s, int64_t rows, int64_t k, const float* g, cudaStream_t st) {
  const int64_t pad_rows = round_up(rows, 128), pad_cols = round_up(k / 16, 4);
  dim3 grid((unsigned)ceil_div(pad_cols * 16, QT_COLS), (unsigned)(pad_rows / 128));
  auto xs = static_cast<const uint16_t*>(x);
  auto gm = static_cast<const uint16_t*>(gamma);
  auto qq = static_cast<uint8_t*>(q);
  auto ss = static_cast<uint8_t*>(s);
  const int q8 = aligned(q, 8) ? 1 : 0;
  if (row_scale && gamma)
    quant_tile_kernel<true, true><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g, q8);
  else if (row_scale)
    quant_tile_kernel<true, false><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g, q8);
  else if (gamma)
    quant_tile_kernel<false, true><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g, q8);
  else
    quant_tile_kernel<false, false><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g, q8);
  return launch_status();
}

static int check_quant_args(const void* x, const void* q, const void* s, int64_t rows, int64_t k) {
  if (!x || !q || !s) return NVFP4B200_ERR_INVALID_ARG;
  if (rows < 0 || k <= 0 || k % 16) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(q, 4) || !aligned(s, 16)) return NVFP4B200_ERR_MISALIGNED;
  return NVFP4B200_OK;
}

static int launch_rms_cta(const void* x, const void* gamma, void* q, void* s, float* inv_rms, int64_t rows, int64_t k,
                          float eps, const float* g, cudaStream_t st) {
  const int64_t pad_rows = round_up(rows, 128), pad_cols = round_up(k / 16, 4);
  const int64_t cover = pad_rows;
  const int64_t span = pad_cols;  // blocks a CTA must cover
  const int bpt = (int)ceil_div(span, 256);
  const int threads = (int)std::min<int64_t>(256, round_up(span, 32));
  const int q8 = (q == nullptr || aligned(q, 8)) ? 1 : 0;
  auto run = [&](auto kern) -> int {
    int per_sm = 0, dev = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) != cudaSuccess || per_sm < 1)
      return NVFP4B200_ERR_CUDA;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(cover, (int64_t)sms * per_sm));
    kern<<<(unsigned)grid, threads, 0, st>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(gamma),
                                             static_cast<uint8_t*>(q), static_cast<uint8_t*>(s), inv_rms, rows,
                                             pad_rows, k, pad_cols, eps, g, q8);
    return launch_status();
  };
#define NVFP4_RMS_CASE(B)                                                         \
  if (bpt <= B)                                                                   \
    return gamma ? run(rmsnorm_cta_kernel<B, true>) : run(rmsnorm_cta_kernel<B, false>);
  NVFP4_RMS_CASE(1)
  NVFP4_RMS_CASE(2)
  NVFP4_RMS_CASE(4)
#undef NVFP4_RMS_CASE
  return NVFP4B200_ERR_BAD_SHAPE;
}

static bool rms_cta_fits(int64_t k) { return round_up(k / 16, 4) <= 4 * 256; }

int take_quant_device_error() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_quant_error, sizeof(int)) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  if (v && cudaMemcpyToSymbol(g_quant_error, &zero, sizeof(int)) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  return v;
}

}  // namespace nvfp4b200

using namespace nvfp4b200;

extern "C" {

int nvfp4b200_api_version(void) { return NVFP4B200_API_VERSION; }

const char* nvfp4b200_status_string(int status) {
  switch (status) {
    case NVFP4B200_OK: return "ok";
    case NVFP4B200_ERR_INVALID_ARG: return "invalid argument";
    case NVFP4B200_ERR_BAD_SHAPE: return "unsupported shape";
    case NVFP4B200_ERR_MISALIGNED: return "misaligned pointer";
    case NVFP4B200_ERR_UNSUPPORTED_DEVICE: return "device is not sm_100 (B200)";
    case NVFP4B200_ERR_LAUNCH: return "kernel launch failed";
    case NVFP4B200_ERR_TIMEOUT: return "bounded device wait timed out";
    case NVFP4B200_ERR_CUDA: return "CUDA call failed";
    default: return "unknown status";
  }
}

int nvfp4b200_device_check(void) { return check_device(); }

int nvfp4b200_quant_nvfp4(const void* x, void* q, void* s, int64_t rows, int64_t k,
                          const float* global_scale, void* stream) {
  int rc = check_quant_args(x, q, s, rows, k);
  if (rc) return rc;
  if ((rc = check_device())) return rc;
  if (rows == 0) return NVFP4B200_OK;
  return launch_quant_tile(x, nullptr, nullptr, q, s, rows, k, global_scale, (cudaStream_t)stream);
}

int nvfp4b200_scaled_quant_nvfp4(const void* x, const float* row_scale, const void* gamma, void* q,
                                 void* s, int64_t rows, int64_t k, const float* global_scale,
                                 void* stream) {
  int rc = check_quant_args(x, q, s, rows, k);
  if (rc) return rc;
  if (gamma && !aligned(gamma, 16)) return NVFP4B200_ERR_MISALIGNED;
  if ((rc = check_device())) return rc;
  if (rows == 0) return NVFP4B200_OK;
  return launch_quant_tile(x, row_scale, gamma, q, s, rows, k, global_scale, (cudaStream_t)stream);
}

int nvfp4b200_rmsnorm_quant_nvfp4(const void* x, const void* gamma, void* q, void* s, float* inv_rms,
                                  int64_t rows, int64_t k, float eps, const float* global_scale,
                                  void* stream) {
  int rc = check_quant_args(x, q, s, rows, k);
  if (rc) return rc;
  if (!inv_rms && rows > 0) return NVFP4B200_ERR_INVALID_ARG;
  if (gamma && !aligned(gamma, 16)) return NVFP4B200_ERR_MISALIGNED;
  if ((rc = check_device())) return rc;
  if (rows == 0) return NVFP4B200_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (rms_cta_fits(k))
    return launch_rms_cta(x, gamma, q, s, inv_rms, rows, k, eps, global_scale, st);
  // wide rows: 1/RMS pass, then the scaled tile quantizer reads x again
  rms_inv_stream_kernel<<<(unsigned)ceil_div(rows, RMS_WARPS), RMS_WARPS * 32, 0, st>>>(
      static_cast<const uint16_t*>(x), inv_rms, rows, k, eps);
  rc = launch_status();
  if (rc) return rc;
  return launch_quant_tile(x, inv_rms, gamma, q, s, rows, k, global_scale, st);
}

int nvfp4b200_rmsnorm_stats(const void* x, const void* gamma, float* inv_rms, int64_t rows, int64_t k,
                            float eps, uint32_t* ws, float* global_scale_out, void* stream) {
  if (!x || !inv_rms || !ws || !global_scale_out) return NVFP4B200_ERR_INVALID_ARG;
  if (rows <= 0 || k <= 0 || k % 16 || !rms_cta_fits(k)) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || (gamma && !aligned(gamma, 16)) || !aligned(ws, 4)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  auto X = static_cast<const uint16_t*>(x);
  auto G = static_cast<const uint16_t*>(gamma);
  auto run = [&](auto kern) -> int {
    int per_sm = 0, dev = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0) != cudaSuccess || per_sm < 1)
      return NVFP4B200_ERR_CUDA;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned grid = (unsigned)std::min<int64_t>(rows, (int64_t)sms * per_sm);
    kern<<<grid, 256, 0, st>>>(X, G, inv_rms, rows, k, eps, ws, global_scale_out);
    return launch_status();
  };
  const int bpt = (int)ceil_div(k / 16, (int64_t)256);
  if (bpt == 1) return gamma ? run(rms_stats_kernel<1, true, 2, true>) : run(rms_stats_kernel<1, false, 2, true>);
  if (bpt == 2) return gamma ? run(rms_stats_kernel<2, true, 1, true>) : run(rms_stats_kernel<2, false, 1, true>);
  // k <= 16384 (rms_cta_fits)
  return gamma ? run(rms_stats_kernel<4, true, 1, true>) : run(rms_stats_kernel<4, false, 1, true>);
}

int nvfp4b200_quant_nvfp4_t(const void* x, const float* row_scale, const void* gamma, void* q, void* s,
                            int64_t rows, int64_t cols, const float* global_scale, void* stream) {
  if (!x || !q || !s) return NVFP4B200_ERR_INVALID_ARG;
  if (rows <= 0 || cols <= 0 || rows % 16 || cols % 8) return NVFP4B200_ERR_BAD_SHAPE;
  if (rows > (1ll << 31) - TQ_T || cols > (1ll << 31) - TQ_D) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(q, 16) || !aligned(s, 16)) return NVFP4B200_ERR_MISALIGNED;
  if (gamma && !aligned(gamma, 2)) return NVFP4B200_ERR_MISALIGNED;
  if (row_scale && !aligned(row_scale, 16)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  const int64_t pad_rows_out = round_up(cols, 128), pad_cols_out = round_up(rows / 16, 4);
  const int64_t n_tiles_t = ceil_div(pad_cols_out * 16, TQ_T), n_tiles_d = pad_rows_out / TQ_D;
  if (n_tiles_t * n_tiles_d > (1ll << 31) - 1) return NVFP4B200_ERR_BAD_SHAPE;
  CUtensorMap xmap;
  if (!make_bf16_map(&xmap, x, rows, cols, TQ_D, TQ_T)) return NVFP4B200_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  const int q16 = ((rows >> 1) % 16 == 0) ? 1 : 0;
  const int n_tiles = (int)(n_tiles_t * n_tiles_d);
  auto run = [&](auto kern) -> int {
    const int smem = (int)sizeof(TqSmem);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return NVFP4B200_ERR_CUDA;
    int per_sm = 0, dev = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem) != cudaSuccess || per_sm < 1)
      return NVFP4B200_ERR_CUDA;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = (int)std::min<int64_t>(n_tiles, (int64_t)sms * per_sm);
    kern<<<grid, 256, smem, st>>>(xmap, row_scale, static_cast<const uint16_t*>(gamma), static_cast<uint8_t*>(q),
                                  static_cast<uint8_t*>(s), rows, cols, pad_cols_out, (int)n_tiles_t, n_tiles,
                                  global_scale, q16);
    return launch_status();
  };
  if (row_scale && gamma) return run(quant_t_kernel<true, true>);
  if (row_scale) return run(quant_t_kernel<true, false>);
  if (gamma) return run(quant_t_kernel<false, true>);
  return run(quant_t_kernel<false, false>);
}

int nvfp4b200_global_scale(const void* x, int64_t n, uint32_t* ws, float* global_scale_out,
                           float* amax_out, void* stream) {
  if (!x || !ws || !global_scale_out) return NVFP4B200_ERR_INVALID_ARG;
  if (n <= 0) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(ws, 4)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  static int num_sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && num_sms[dev] == 0)
    cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int sms = (dev >= 0 && dev < 64 && num_sms[dev] > 0) ? num_sms[dev] : 148;
  const int64_t n_vec = n / 8;
  const int n_tail = (int)(n % 8);
  const int64_t want = ceil_div(std::max<int64_t>(n_vec, 1), 256 * 4);
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
  global_amax_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      static_cast<const uint4*>(x), n_vec, static_cast<const uint16_t*>(x) + n_vec * 8, n_tail, ws,
      global_scale_out, amax_out);
  return launch_status();
}

}  // extern "C"
