// NVFP4 quantizers for B200 (sm_100a): plain / scaled, fused RMSNorm,
// transposed, and the global-amax reduction.
//
// All kernels are HBM-bound.  The per-element arithmetic follows the
// reference quantizer (float4utils.py:79-148): block amax with fmaxf
// semantics, E4M3 block scale by cvt.rn.satfinite, reciprocal-then-multiply,
// the away-from-zero E2M1 ladder, low-nibble-first packing and the 128x4
// swizzled scale layout -- see common.cuh for each helper.  What differs is
// the data movement: warps read 512 contiguous bytes per instruction, write
// 128 contiguous bytes of nibbles, and scale atoms are staged in shared
// memory and written as whole 512-byte atoms, so no separate zero-fill of
// the scale tensor is needed.
#include "common.cuh"

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
// tile quantizer: 128 rows x 256 columns per CTA
// ---------------------------------------------------------------------------

constexpr int QT_ROWS = 128;
constexpr int QT_COLS = 256;       // 16 blocks = 4 scale atoms
constexpr int QT_THREADS = 256;    // 8 warps x 16 rows

template <bool HAS_ROW, bool HAS_GAMMA>
__global__ void __launch_bounds__(QT_THREADS) quant_tile_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ row_scale,
    const uint16_t* __restrict__ gamma, uint8_t* __restrict__ q, uint8_t* __restrict__ s,
    int64_t rows, int64_t k, int64_t pad_cols, const float* __restrict__ gptr) {
  __shared__ __align__(16) uint8_t s_tile[4 * 512];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t r0 = (int64_t)blockIdx.y * QT_ROWS;
  const int64_t c0 = (int64_t)blockIdx.x * QT_COLS;  // element column
  const int64_t col = c0 + 8 * lane;
  const bool col_ok = col < k;
  const float g = load_global_scale(gptr);
  const float inv_g = __frcp_rn(g);

  float gam[8];
  if (HAS_GAMMA) {
    uint4 gv = make_uint4(0, 0, 0, 0);
    if (col_ok) gv = __ldg(reinterpret_cast<const uint4*>(gamma + col));
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) { gam[2 * i] = bf16lo(gw[i]); gam[2 * i + 1] = bf16hi(gw[i]); }
  }

  // issue all 16 row loads of this warp first (memory-level parallelism)
  uint4 v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int64_t r = r0 + wid * 16 + i;
    v[i] = make_uint4(0, 0, 0, 0);
    if (col_ok && r < rows) v[i] = __ldg(reinterpret_cast<const uint4*>(x + r * k + col));
  }

  const int blk = lane >> 1;             // block index inside the 256-col tile (0..15)
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int rl = wid * 16 + i;         // row inside the tile
    const int64_t r = r0 + rl;
    const bool ok = col_ok && r < rows;
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) { f[2 * j] = bf16lo(w[j]); f[2 * j + 1] = bf16hi(w[j]); }
    float amax;
    if (HAS_ROW || HAS_GAMMA) {
      const float rs = HAS_ROW ? (ok ? __ldg(row_scale + r) : 0.0f) : 1.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (HAS_ROW) f[j] = f[j] * rs;
        if (HAS_GAMMA) f[j] = f[j] * gam[j];
      }
      amax = fmax_abs8(f);
    } else {
      uint32_t mb = absmax8_bits(w);
      amax = (mb > 0x7F80u) ? fmax_abs8(f) : __uint_as_float(mb << 16);
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    float inv_scale;
    const uint32_t code = ok ? block_scale(amax, g, inv_g, inv_scale) : 0u;
    if (!ok) inv_scale = 1.0f;
    const uint32_t packed = encode8(f, inv_scale);
    if (ok) *reinterpret_cast<uint32_t*>(q + r * (k >> 1) + (col >> 1)) = packed;
    if ((lane & 1) == 0) s_tile[(blk >> 2) * 512 + atom_offset(rl, blk & 3)] = (uint8_t)code;
  }
  __syncthreads();
  // write the (up to) 4 atoms of this tile: contiguous 2 KB in the swizzled tensor
  const int64_t atom0 = (int64_t)blockIdx.x * 4;
  const int64_t n_atoms = imin64(4, (pad_cols >> 2) - atom0);
  const int64_t dst = ((int64_t)blockIdx.y * (pad_cols >> 2) + atom0) * 512;
  if ((int64_t)threadIdx.x * 8 < n_atoms * 512)
    *reinterpret_cast<uint2*>(s + dst + threadIdx.x * 8) = reinterpret_cast<const uint2*>(s_tile)[threadIdx.x];
}

// ---------------------------------------------------------------------------
// fused RMSNorm -> quantize: one warp per row, the row held in registers
// ---------------------------------------------------------------------------

constexpr int RMS_WARPS = 4;

// MODE 0: quantize (computes inv_rms, writes it).  MODE 1: statistics only
// (inv_rms + global amax of the normalised row).
template <int NV, bool HAS_GAMMA, int MODE>
__global__ void __launch_bounds__(RMS_WARPS * 32) rmsnorm_row_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma, uint8_t* __restrict__ q,
    uint8_t* __restrict__ s, float* __restrict__ inv_rms_out, int64_t rows, int64_t pad_rows,
    int64_t k, int64_t pad_cols, float eps, const float* __restrict__ gptr, uint32_t* ws,
    float* g_out) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * RMS_WARPS + wid;
  const bool row_ok = r < rows;
  uint4 v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int64_t col = (int64_t)j * 256 + 8 * lane;
    v[j] = make_uint4(0, 0, 0, 0);
    if (row_ok && col < k) v[j] = __ldg(reinterpret_cast<const uint4*>(x + r * k + col));
  }
  // sum of squares in fp32 (thread-sequential, then a butterfly)
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a0 = bf16lo(w[i]), a1 = bf16hi(w[i]);
      ss += a0 * a0 + a1 * a1;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / (float)k + eps);
  if (row_ok && lane == 0 && inv_rms_out) inv_rms_out[r] = inv;

  if (MODE == 1) {
    float am = 0.0f;
    if (row_ok) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int64_t col = (int64_t)j * 256 + 8 * lane;
        if (col >= k) continue;
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        float gam[8];
        if (HAS_GAMMA) {
          const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma + col));
          const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) { gam[2 * i] = bf16lo(gw[i]); gam[2 * i + 1] = bf16hi(gw[i]); }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float a0 = bf16lo(w[i]) * inv, a1 = bf16hi(w[i]) * inv;
          if (HAS_GAMMA) { a0 = a0 * gam[2 * i]; a1 = a1 * gam[2 * i + 1]; }
          am = fmaxf(am, fmaxf(fabsf(a0), fabsf(a1)));
        }
      }
    }
    amax_commit(__float_as_uint(am), ws, g_out, nullptr);
    return;
  }

  const float g = load_global_scale(gptr);
  const float inv_g = __frcp_rn(g);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int64_t col = (int64_t)j * 256 + 8 * lane;
    if ((int64_t)j * 256 >= pad_cols * 16) break;  // whole chunk beyond the padded scale columns
    const bool ok = row_ok && col < k;
    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[2 * i] = bf16lo(w[i]) * inv; f[2 * i + 1] = bf16hi(w[i]) * inv; }
    if (HAS_GAMMA && ok) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma + col));
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) { f[2 * i] = f[2 * i] * bf16lo(gw[i]); f[2 * i + 1] = f[2 * i + 1] * bf16hi(gw[i]); }
    }
    float amax = fmax_abs8(f);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    float inv_scale = 1.0f;
    uint32_t code = ok ? block_scale(amax, g, inv_g, inv_scale) : 0u;
    const uint32_t packed = encode8(f, inv_scale);
    if (ok) *reinterpret_cast<uint32_t*>(q + r * (k >> 1) + (col >> 1)) = packed;
    // gather the 4 block scales of each 4-block group into one word
    const uint32_t c1 = __shfl_down_sync(0xffffffffu, code, 2);
    const uint32_t c2 = __shfl_down_sync(0xffffffffu, code, 4);
    const uint32_t c3 = __shfl_down_sync(0xffffffffu, code, 6);
    const int64_t bcol = (int64_t)j * 16 + (lane >> 1);  // block column of this lane
    if ((lane & 7) == 0 && bcol < pad_cols && r < pad_rows) {
      const uint32_t word = code | (c1 << 8) | (c2 << 16) | (c3 << 24);
      *reinterpret_cast<uint32_t*>(s + swz_offset(r, bcol, pad_cols)) = word;
    }
  }
}

// Streaming 1/RMS for rows too wide to hold in registers (k > 8192): one
// warp per row, same fp32 thread-sequential + butterfly order as above.
__global__ void __launch_bounds__(RMS_WARPS * 32) rms_inv_stream_kernel(
    const uint16_t* __restrict__ x, float* __restrict__ inv_rms, int64_t rows, int64_t k, float eps) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * RMS_WARPS + wid;
  if (r >= rows) return;
  float ss = 0.0f;
  for (int64_t col = 8 * lane; col < k; col += 256) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + r * k + col));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a0 = bf16lo(w[i]), a1 = bf16hi(w[i]);
      ss += a0 * a0 + a1 * a1;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) inv_rms[r] = rsqrtf(ss / (float)k + eps);
}

// ---------------------------------------------------------------------------
// transposed quantizer: x [rows, cols] -> quantize x^T along rows
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

constexpr int TQ_T = 256;          // input rows per CTA = output k extent (16 blocks)
constexpr int TQ_D = 128;          // input cols per CTA = output rows (one atom group)
constexpr int TQ_STRIDE = TQ_D + 8;  // smem row stride in bf16 (272 bytes)

template <bool HAS_ROW, bool HAS_GAMMA>
__global__ void __launch_bounds__(256) quant_t_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ row_scale,
    const uint16_t* __restrict__ gamma, uint8_t* __restrict__ q, uint8_t* __restrict__ s,
    int64_t rows, int64_t cols, int64_t pad_cols_out, const float* __restrict__ gptr) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t* tile = reinterpret_cast<uint16_t*>(smem_raw);                       // [TQ_T][TQ_STRIDE]
  uint8_t* s_tile = smem_raw + TQ_T * TQ_STRIDE * 2;                            // 2048 bytes
  float* rs_tile = reinterpret_cast<float*>(s_tile + 2048);                     // [TQ_T]
  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * TQ_T;
  const int64_t d0 = (int64_t)blockIdx.y * TQ_D;

  // load 256 x 128 bf16 (16 uint4 per row, 16 rows per pass of 256 threads)
#pragma unroll 4
  for (int it = 0; it < 16; ++it) {
    const int t = it * 16 + (tid >> 4);
    const int dv = (tid & 15) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (t0 + t < rows && d0 + dv < cols)
      val = __ldg(reinterpret_cast<const uint4*>(x + (t0 + t) * cols + d0 + dv));
    *reinterpret_cast<uint4*>(tile + t * TQ_STRIDE + dv) = val;
  }
  if (HAS_ROW) rs_tile[tid] = (t0 + tid < rows) ? __ldg(row_scale + t0 + tid) : 0.0f;
  __syncthreads();

  const float g = load_global_scale(gptr);
  const float inv_g = __frcp_rn(g);
  const int p = tid & 63;          // d pair
  const int qtr = tid >> 6;        // blocks 4*qtr .. 4*qtr+3
  const int dl0 = 2 * p;
  float gam0 = 1.0f, gam1 = 1.0f;
  if (HAS_GAMMA) {
    if (d0 + dl0 < cols) gam0 = __uint_as_float((uint32_t)gamma[d0 + dl0] << 16);
    if (d0 + dl0 + 1 < cols) gam1 = __uint_as_float((uint32_t)gamma[d0 + dl0 + 1] << 16);
  }
  uint32_t codes_a = 0, codes_b = 0;
  uint32_t qwa[8], qwb[8];   // packed nibbles: 4 blocks x 8 bytes for each of the two output rows
#pragma unroll
  for (int bi = 0; bi < 4; ++bi) {
    const int b = qtr * 4 + bi;
    float fa[16], fb[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = b * 16 + j;
      const uint32_t w = *reinterpret_cast<const uint32_t*>(tile + t * TQ_STRIDE + dl0);
      float a = bf16lo(w), c = bf16hi(w);
      if (HAS_ROW) { const float rsv = rs_tile[t]; a = a * rsv; c = c * rsv; }
      if (HAS_GAMMA) { a = a * gam0; c = c * gam1; }
      fa[j] = a;
      fb[j] = c;
    }
    const bool blk_ok = t0 + b * 16 < rows;
    float ama = 0.0f, amb = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) { ama = fmaxf(ama, fabsf(fa[j])); amb = fmaxf(amb, fabsf(fb[j])); }
    float isa = 1.0f, isb = 1.0f;
    const uint32_t ca = blk_ok ? block_scale(ama, g, inv_g, isa) : 0u;
    const uint32_t cb = blk_ok ? block_scale(amb, g, inv_g, isb) : 0u;
    float la[8], ha[8], lb[8], hb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { la[j] = fa[j]; ha[j] = fa[8 + j]; lb[j] = fb[j]; hb[j] = fb[8 + j]; }
    qwa[2 * bi] = encode8(la, isa);
    qwa[2 * bi + 1] = encode8(ha, isa);
    qwb[2 * bi] = encode8(lb, isb);
    qwb[2 * bi + 1] = encode8(hb, isb);
    codes_a |= ca << (8 * bi);
    codes_b |= cb << (8 * bi);
  }
  // output rows d0+dl0 and d0+dl0+1; 32 bytes each at column (t0 + 64*qtr)/2
  const int64_t kout = rows;
  const int64_t tcol = t0 + 64 * qtr;
  if (tcol < rows) {
    // rows/2 is a multiple of 8, so an output row start is 8-byte aligned;
    // 16-byte stores only when the whole 32 bytes are in range and aligned.
    const int64_t nbytes = imin64(32, (rows - tcol) >> 1);
    const uint32_t* qw[2] = {qwa, qwb};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (d0 + dl0 + h >= cols) continue;
      uint8_t* dst = q + (d0 + dl0 + h) * (kout >> 1) + (tcol >> 1);
      if (nbytes == 32 && aligned16(dst)) {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(qw[h][0], qw[h][1], qw[h][2], qw[h][3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(qw[h][4], qw[h][5], qw[h][6], qw[h][7]);
      } else {
        for (int i = 0; i < nbytes / 8; ++i)
          reinterpret_cast<uint2*>(dst)[i] = make_uint2(qw[h][2 * i], qw[h][2 * i + 1]);
      }
    }
  }
  // scale codes: output row dl, blocks 4*qtr..4*qtr+3 = atom qtr, columns 0..3
  *reinterpret_cast<uint32_t*>(s_tile + qtr * 512 + atom_offset(dl0, 0)) = (d0 + dl0 < cols) ? codes_a : 0u;
  *reinterpret_cast<uint32_t*>(s_tile + qtr * 512 + atom_offset(dl0 + 1, 0)) = (d0 + dl0 + 1 < cols) ? codes_b : 0u;
  __syncthreads();
  const int64_t atom0 = (int64_t)blockIdx.x * 4;
  const int64_t n_atoms = imin64(4, (pad_cols_out >> 2) - atom0);
  const int64_t dst = ((int64_t)blockIdx.y * (pad_cols_out >> 2) + atom0) * 512;
  if ((int64_t)tid * 8 < n_atoms * 512)
    *reinterpret_cast<uint2*>(s + dst + tid * 8) = reinterpret_cast<const uint2*>(s_tile)[tid];
}

constexpr size_t TQ_SMEM = (size_t)TQ_T * TQ_STRIDE * 2 + 2048 + TQ_T * 4;

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------

static int launch_quant_tile(const void* x, const float* row_scale, const void* gamma, void* q,
                             void* s, int64_t rows, int64_t k, const float* g, cudaStream_t st) {
  const int64_t pad_rows = round_up(rows, 128), pad_cols = round_up(k / 16, 4);
  dim3 grid((unsigned)ceil_div(pad_cols * 16, QT_COLS), (unsigned)(pad_rows / 128));
  auto xs = static_cast<const uint16_t*>(x);
  auto gm = static_cast<const uint16_t*>(gamma);
  auto qq = static_cast<uint8_t*>(q);
  auto ss = static_cast<uint8_t*>(s);
  if (row_scale && gamma)
    quant_tile_kernel<true, true><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g);
  else if (row_scale)
    quant_tile_kernel<true, false><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g);
  else if (gamma)
    quant_tile_kernel<false, true><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g);
  else
    quant_tile_kernel<false, false><<<grid, QT_THREADS, 0, st>>>(xs, row_scale, gm, qq, ss, rows, k, pad_cols, g);
  return launch_status();
}

static int check_quant_args(const void* x, const void* q, const void* s, int64_t rows, int64_t k) {
  if (!x || !q || !s) return NVFP4B200_ERR_INVALID_ARG;
  if (rows < 0 || k <= 0 || k % 16) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(q, 4) || !aligned(s, 16)) return NVFP4B200_ERR_MISALIGNED;
  return NVFP4B200_OK;
}

template <int MODE>
static int launch_rms_rows(const void* x, const void* gamma, void* q, void* s, float* inv_rms,
                           int64_t rows, int64_t k, float eps, const float* g, uint32_t* ws,
                           float* g_out, cudaStream_t st) {
  const int64_t pad_rows = round_up(rows, 128), pad_cols = round_up(k / 16, 4);
  const int64_t cover = MODE == 0 ? pad_rows : rows;
  dim3 grid((unsigned)std::max<int64_t>(1, ceil_div(cover, RMS_WARPS)));
  auto xs = static_cast<const uint16_t*>(x);
  auto gm = static_cast<const uint16_t*>(gamma);
  auto qq = static_cast<uint8_t*>(q);
  auto ss = static_cast<uint8_t*>(s);
  const int nv = (int)ceil_div(k, 256);
#define NVFP4_RMS_CASE(NVV)                                                                       \
  if (nv <= NVV) {                                                                                \
    if (gamma)                                                                                    \
      rmsnorm_row_kernel<NVV, true, MODE><<<grid, RMS_WARPS * 32, 0, st>>>(                      \
          xs, gm, qq, ss, inv_rms, rows, pad_rows, k, pad_cols, eps, g, ws, g_out);               \
    else                                                                                          \
      rmsnorm_row_kernel<NVV, false, MODE><<<grid, RMS_WARPS * 32, 0, st>>>(                     \
          xs, gm, qq, ss, inv_rms, rows, pad_rows, k, pad_cols, eps, g, ws, g_out);               \
    return launch_status();                                                                       \
  }
  NVFP4_RMS_CASE(1)
  NVFP4_RMS_CASE(2)
  NVFP4_RMS_CASE(4)
  NVFP4_RMS_CASE(8)
  NVFP4_RMS_CASE(16)
  NVFP4_RMS_CASE(32)
#undef NVFP4_RMS_CASE
  return NVFP4B200_ERR_BAD_SHAPE;
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
  if (k <= 32 * 256)
    return launch_rms_rows<0>(x, gamma, q, s, inv_rms, rows, k, eps, global_scale, nullptr, nullptr, st);
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
  if (rows <= 0 || k <= 0 || k % 16 || k > 32 * 256) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || (gamma && !aligned(gamma, 16)) || !aligned(ws, 4)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  return launch_rms_rows<1>(x, gamma, nullptr, nullptr, inv_rms, rows, k, eps, nullptr, ws,
                            global_scale_out, (cudaStream_t)stream);
}

int nvfp4b200_quant_nvfp4_t(const void* x, const float* row_scale, const void* gamma, void* q, void* s,
                            int64_t rows, int64_t cols, const float* global_scale, void* stream) {
  if (!x || !q || !s) return NVFP4B200_ERR_INVALID_ARG;
  if (rows <= 0 || cols <= 0 || rows % 16 || cols % 8) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(q, 16) || !aligned(s, 16)) return NVFP4B200_ERR_MISALIGNED;
  if (gamma && !aligned(gamma, 2)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  const int64_t pad_rows_out = round_up(cols, 128), pad_cols_out = round_up(rows / 16, 4);
  dim3 grid((unsigned)ceil_div(pad_cols_out * 16, TQ_T), (unsigned)(pad_rows_out / TQ_D));
  cudaStream_t st = (cudaStream_t)stream;
  auto xs = static_cast<const uint16_t*>(x);
  auto gm = static_cast<const uint16_t*>(gamma);
  auto qq = static_cast<uint8_t*>(q);
  auto ss = static_cast<uint8_t*>(s);
#define NVFP4_TQ(HR, HG)                                                                        \
  {                                                                                             \
    if (cudaFuncSetAttribute(quant_t_kernel<HR, HG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             (int)TQ_SMEM) != cudaSuccess)                                      \
      return NVFP4B200_ERR_CUDA;                                                                \
    quant_t_kernel<HR, HG><<<grid, 256, TQ_SMEM, st>>>(xs, row_scale, gm, qq, ss, rows, cols,  \
                                                       pad_cols_out, global_scale);             \
  }
  if (row_scale && gamma) NVFP4_TQ(true, true)
  else if (row_scale) NVFP4_TQ(true, false)
  else if (gamma) NVFP4_TQ(false, true)
  else NVFP4_TQ(false, false)
#undef NVFP4_TQ
  return launch_status();
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
