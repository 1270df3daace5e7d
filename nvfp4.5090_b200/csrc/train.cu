// Element-wise and row-reduction kernels of the NVFP4 SwiGLU MLP training
// step (B200, sm_100a).  The reference trains with a bf16 backward
// (float4utils.py:653-683) and ships no MLP; these kernels carry the
// activations, gradients and optimizer state between the NVFP4 GEMMs.
// All are HBM-bound: 16-byte vector accesses, grid sized to the SM count.
#include "common.cuh"

#include <algorithm>

namespace nvfp4b200 {

static int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev] > 0 ? cache[dev] : 148;
}

static unsigned grid_for(int64_t work_items, int threads, int per_sm = 8) {
  const int64_t want = ceil_div(std::max<int64_t>(work_items, 1), threads);
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count() * per_sm));
}

// sigmoid with the fast exponential and division intrinsics; 0 for x -> -inf
// (the division returns 0 when the denominator is infinite), 1 for x -> +inf.
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// |bf16 pair| max as float bits (NaN ignored)
__device__ __forceinline__ uint32_t absmax_word_bits(uint32_t w) {
  uint32_t a = w & 0x7FFF7FFFu;
  a &= ~__vcmpgtu2(a, 0x7F807F80u);
  return max(a & 0xFFFFu, a >> 16) << 16;
}

// Column of gate value c in a gu row, and the distance to its up value:
// [gate | up] halves (il = 0) or blocks of 128 alternating (il = 128).
__device__ __forceinline__ int64_t gate_col(int64_t c, int il) { return il ? ((c >> 7) << 8) + (c & 127) : c; }

// h = silu(gate) * up with gu = [gate | up] per row (or interleaved blocks);
// optional global amax of h.  CTAs stride over rows, threads over 8-column
// vectors of a row (a vector never straddles a 128-column block).
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const uint16_t* __restrict__ gu, uint16_t* __restrict__ h,
                                                         int64_t tokens, int64_t ff, int il, uint32_t* ws,
                                                         float* g_out) {
  const int64_t up_off = il ? 128 : ff;
  uint32_t m = 0;
  for (int64_t t = blockIdx.x; t < tokens; t += gridDim.x) {
    const uint16_t* grow = gu + t * 2 * ff;
    uint16_t* hrow = h + t * ff;
    for (int64_t c = 8 * (int64_t)threadIdx.x; c < ff; c += 8 * (int64_t)blockDim.x) {
      const int64_t gc = gate_col(c, il);
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(grow + gc));
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(grow + gc + up_off));
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g0 = bf16lo(gw[j]), g1 = bf16hi(gw[j]);
        const float h0 = g0 * sigmoidf_(g0) * bf16lo(uw[j]);
        const float h1 = g1 * sigmoidf_(g1) * bf16hi(uw[j]);
        o[j] = pack2(h0, h1);
        m = max(m, absmax_word_bits(o[j]));
      }
      *reinterpret_cast<uint4*>(hrow + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (ws) amax_commit(m, ws, g_out, nullptr);
}

// dgate = dh * up * silu'(gate), dup = dh * silu(gate);
// silu'(g) = s * (1 + g * (1 - s)), s = sigmoid(g).
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const uint16_t* __restrict__ gu,
                                                         const uint16_t* __restrict__ dh, uint16_t* __restrict__ dgu,
                                                         int64_t tokens, int64_t ff, int il, uint32_t* ws,
                                                         float* g_out) {
  const int64_t up_off = il ? 128 : ff;
  uint32_t m = 0;
  for (int64_t t = blockIdx.x; t < tokens; t += gridDim.x) {
    const uint16_t* grow = gu + t * 2 * ff;
    const uint16_t* drow = dh + t * ff;
    uint16_t* orow = dgu + t * 2 * ff;
    for (int64_t c = 8 * (int64_t)threadIdx.x; c < ff; c += 8 * (int64_t)blockDim.x) {
      const int64_t gc = gate_col(c, il);
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(grow + gc));
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(grow + gc + up_off));
      const uint4 dv = __ldg(reinterpret_cast<const uint4*>(drow + c));
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w},
                     dw[4] = {dv.x, dv.y, dv.z, dv.w};
      uint32_t og[4], ou[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float dg[2], du[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float g = e ? bf16hi(gw[j]) : bf16lo(gw[j]);
          const float u = e ? bf16hi(uw[j]) : bf16lo(uw[j]);
          const float d = e ? bf16hi(dw[j]) : bf16lo(dw[j]);
          swiglu_grad(g, u, d, sigmoidf_(g), dg[e], du[e]);
        }
        og[j] = pack2(dg[0], dg[1]);
        ou[j] = pack2(du[0], du[1]);
        m = max(m, max(absmax_word_bits(og[j]), absmax_word_bits(ou[j])));
      }
      *reinterpret_cast<uint4*>(orow + gc) = make_uint4(og[0], og[1], og[2], og[3]);
      *reinterpret_cast<uint4*>(orow + gc + up_off) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    }
  }
  if (ws) amax_commit(m, ws, g_out, nullptr);
}

// RMSNorm backward.  Persistent CTAs of 512 threads walk a band of rows;
// thread t owns columns {4096 v + 8 t + i}.  The next row's x and dy are
// loaded while the current row is reduced.  Per row: s = sum(dy*gamma*xn)
// (block reduction), dx = inv*(dy*gamma - xn*s/k) + dres; dgamma partial
// sums stay in registers for the band and are added to global once.
constexpr int RB_THREADS = 512;
template <int NV>
__global__ void __launch_bounds__(RB_THREADS) rmsnorm_bwd_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma, const float* __restrict__ inv_rms,
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ dres, uint16_t* __restrict__ dx,
    float* __restrict__ dgamma, int64_t rows, int64_t k, int64_t rows_per_cta) {
  __shared__ float red[2][RB_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float gam[NV][8], dgam[NV][8];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int64_t col = (int64_t)v * 4096 + 8 * tid;
    uint4 gv = make_uint4(0, 0, 0, 0);
    if (col < k) gv = gamma ? __ldg(reinterpret_cast<const uint4*>(gamma + col))
                            : make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    const uint32_t w[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      gam[v][2 * j] = bf16lo(w[j]);
      gam[v][2 * j + 1] = bf16hi(w[j]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) dgam[v][j] = 0.0f;
  }
  const int64_t r_begin = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r_end = imin64(rows, r_begin + rows_per_cta);
  auto load = [&](int64_t r, uint4 (&xv)[NV], uint4 (&dv)[NV]) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int64_t col = (int64_t)v * 4096 + 8 * tid;
      xv[v] = make_uint4(0, 0, 0, 0);
      dv[v] = xv[v];
      if (r < r_end && col < k) {
        xv[v] = __ldg(reinterpret_cast<const uint4*>(x + r * k + col));
        dv[v] = __ldg(reinterpret_cast<const uint4*>(dy + r * k + col));
      }
    }
  };
  uint4 cx[NV], cd[NV], nx[NV], nd[NV];
  load(r_begin, cx, cd);
  int buf = 0;
  for (int64_t r = r_begin; r < r_end; ++r) {
    load(r + 1, nx, nd);
    // the residual gradient is read at the top of the row, so its latency
    // hides behind the reduction (read after the barrier it was exposed once
    // per row: 262 vs 213 us at 16384 x 8192, 123 vs 115 us at 16384 x 4096)
    uint4 cr[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int64_t col = (int64_t)v * 4096 + 8 * tid;
      cr[v] = make_uint4(0, 0, 0, 0);
      if (dres && col < k) cr[v] = __ldg(reinterpret_cast<const uint4*>(dres + r * k + col));
    }
    const float inv = __ldg(inv_rms + r);
    float part = 0.0f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const uint32_t xw[4] = {cx[v].x, cx[v].y, cx[v].z, cx[v].w}, dw[4] = {cd[v].x, cd[v].y, cd[v].z, cd[v].w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xn = (j & 1 ? bf16hi(xw[j >> 1]) : bf16lo(xw[j >> 1])) * inv;
        const float d = j & 1 ? bf16hi(dw[j >> 1]) : bf16lo(dw[j >> 1]);
        dgam[v][j] += d * xn;
        part += (d * gam[v][j]) * xn;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) red[buf][wid] = part;
    __syncthreads();
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < RB_THREADS / 32; ++i) sum += red[buf][i];
    buf ^= 1;
    const float mean = sum / (float)k;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int64_t col = (int64_t)v * 4096 + 8 * tid;
      if (col >= k) continue;
      const uint32_t xw[4] = {cx[v].x, cx[v].y, cx[v].z, cx[v].w}, dw[4] = {cd[v].x, cd[v].y, cd[v].z, cd[v].w};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xn = (j & 1 ? bf16hi(xw[j >> 1]) : bf16lo(xw[j >> 1])) * inv;
        const float d = j & 1 ? bf16hi(dw[j >> 1]) : bf16lo(dw[j >> 1]);
        o[j] = inv * (d * gam[v][j] - xn * mean);
      }
      if (dres) {
        const uint4 rv = cr[v];
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[2 * j] += bf16lo(rw[j]);
          o[2 * j + 1] += bf16hi(rw[j]);
        }
      }
      *reinterpret_cast<uint4*>(dx + r * k + col) =
          make_uint4(pack2(o[0], o[1]), pack2(o[2], o[3]), pack2(o[4], o[5]), pack2(o[6], o[7]));
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      cx[v] = nx[v];
      cd[v] = nd[v];
    }
  }
  if (dgamma) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int64_t col = (int64_t)v * 4096 + 8 * tid;
      if (col >= k) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(dgamma + col + j, dgam[v][j]);
    }
  }
}

__global__ void __launch_bounds__(256) add_bf16_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                                                       uint16_t* __restrict__ y, int64_t n) {
  const int64_t nv = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 av = __ldg(reinterpret_cast<const uint4*>(a) + i), bv = __ldg(reinterpret_cast<const uint4*>(b) + i);
    const uint32_t aw[4] = {av.x, av.y, av.z, av.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack2(bf16lo(aw[j]) + bf16lo(bw[j]), bf16hi(aw[j]) + bf16hi(bw[j]));
    reinterpret_cast<uint4*>(y)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int64_t i = nv * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float s = __uint_as_float((uint32_t)a[i] << 16) + __uint_as_float((uint32_t)b[i] << 16);
    const __nv_bfloat16 hb = __float2bfloat16_rn(s);
    y[i] = *reinterpret_cast<const uint16_t*>(&hb);
  }
}

struct AdamArgs {
  float lr, b1, b2, eps, wd, bc1, bc2, gscale;
};

// One AdamW element update on a bf16 parameter, every operation rounded
// once (explicit _rn intrinsics: no contraction into FMAs), so that a float32
// restatement in the same order reproduces m, v and the unrounded parameter
// bit for bit:
//   g = grad * grad_scale; m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*(g*g);
//   p = p - lr*((m/bc1)/(sqrt(v/bc2)+eps) + wd*p).
__device__ __forceinline__ float adam_one(float p, float g, float& m, float& v, const AdamArgs& a) {
  g = __fmul_rn(g, a.gscale);
  m = __fadd_rn(__fmul_rn(a.b1, m), __fmul_rn(__fsub_rn(1.0f, a.b1), g));
  v = __fadd_rn(__fmul_rn(a.b2, v), __fmul_rn(__fsub_rn(1.0f, a.b2), __fmul_rn(g, g)));
  const float mh = __fdiv_rn(m, a.bc1), vh = __fdiv_rn(v, a.bc2);
  const float upd = __fadd_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps)), __fmul_rn(a.wd, p));
  return __fsub_rn(p, __fmul_rn(a.lr, upd));
}

// AdamW on an fp32 master weight in the operation order of
// torch.optim.AdamW (decoupled decay first, lerp for m, addcmul for v,
// sqrt(v)/sqrt(bc2) + eps, addcdiv with step size lr/bc1), each operation
// rounded once:
//   w = w*(1 - lr*wd); m = m + (1-b1)*(g - m); v = b2*v + (1-b2)*(g*g);
//   w = w - (lr/bc1) * (m / (sqrt(v)/sqrt(bc2) + eps)).
// The scalars lr*wd, lr/bc1 and sqrt(bc2) arrive precomputed (MasterArgs).
struct MasterArgs {
  float one_minus_lr_wd, one_minus_b1, b2, one_minus_b2, eps, step_size, bc2_sqrt, gscale;
};

__device__ __forceinline__ float adam_master_one(float w, float g, float& m, float& v, const MasterArgs& a) {
  g = __fmul_rn(g, a.gscale);
  w = __fmul_rn(w, a.one_minus_lr_wd);
  m = __fadd_rn(m, __fmul_rn(a.one_minus_b1, __fsub_rn(g, m)));
  v = __fadd_rn(__fmul_rn(v, a.b2), __fmul_rn(a.one_minus_b2, __fmul_rn(g, g)));
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.bc2_sqrt), a.eps);
  return __fsub_rn(w, __fmul_rn(a.step_size, __fdiv_rn(m, denom)));
}

__device__ __forceinline__ void load_grad8(const void* grad, int64_t i, bool f32, float (&g)[8]) {
  if (f32) {
    const float4 g0 = reinterpret_cast<const float4*>(grad)[2 * i], g1 = reinterpret_cast<const float4*>(grad)[2 * i + 1];
    g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
  } else {
    const uint4 gv = reinterpret_cast<const uint4*>(grad)[i];
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { g[2 * j] = bf16lo(gw[j]); g[2 * j + 1] = bf16hi(gw[j]); }
  }
}

__device__ __forceinline__ void load_f32x8(const float* p, int64_t i, float (&x)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[2 * i], b = reinterpret_cast<const float4*>(p)[2 * i + 1];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ void store_f32x8(float* p, int64_t i, const float (&x)[8]) {
  reinterpret_cast<float4*>(p)[2 * i] = make_float4(x[0], x[1], x[2], x[3]);
  reinterpret_cast<float4*>(p)[2 * i + 1] = make_float4(x[4], x[5], x[6], x[7]);
}

__device__ __forceinline__ float grad_at(const void* grad, int64_t i, bool f32) {
  return f32 ? static_cast<const float*>(grad)[i]
             : __uint_as_float((uint32_t)static_cast<const uint16_t*>(grad)[i] << 16);
}

__device__ __forceinline__ uint16_t bf16_bits_rn(float x) {
  const __nv_bfloat16 hb = __float2bfloat16_rn(x);
  return *reinterpret_cast<const uint16_t*>(&hb);
}

template <bool GRAD_F32>
__global__ void __launch_bounds__(256) adamw_kernel(uint16_t* __restrict__ p, const void* __restrict__ grad,
                                                    float* __restrict__ m, float* __restrict__ v, int64_t n,
                                                    AdamArgs a) {
  const int64_t nv = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 pv = reinterpret_cast<const uint4*>(p)[i];
    float g[8], mm[8], vv[8];
    load_grad8(grad, i, GRAD_F32, g);
    load_f32x8(m, i, mm);
    load_f32x8(v, i, vv);
    const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
    float pf[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) { pf[2 * j] = bf16lo(pw[j]); pf[2 * j + 1] = bf16hi(pw[j]); }
#pragma unroll
    for (int j = 0; j < 8; ++j) pf[j] = adam_one(pf[j], g[j], mm[j], vv[j], a);
    reinterpret_cast<uint4*>(p)[i] = make_uint4(pack2(pf[0], pf[1]), pack2(pf[2], pf[3]), pack2(pf[4], pf[5]), pack2(pf[6], pf[7]));
    store_f32x8(m, i, mm);
    store_f32x8(v, i, vv);
  }
  for (int64_t i = nv * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float mm = m[i], vv = v[i];
    const float r = adam_one(__uint_as_float((uint32_t)p[i] << 16), grad_at(grad, i, GRAD_F32), mm, vv, a);
    m[i] = mm;
    v[i] = vv;
    p[i] = bf16_bits_rn(r);
  }
}

// fp32 master weights: w, m, v are updated in fp32 and the bf16 parameter is
// written as round-to-nearest-even of the new w.  Updates smaller than half a
// bf16 ulp of the parameter accumulate in w instead of being rounded away.
// |bf16| of a packed pair as float bits (the larger one), NaN ignored
__device__ __forceinline__ uint32_t absmax_pair_bits(uint32_t w) { return absmax_word_bits(w); }

// amax_bits (optional): max |bf16 parameter| written by this launch, as float
// bits, combined into *amax_bits with atomicMax (the caller zeroes it first);
// NaN is ignored, as in the global-scale kernels.
template <bool GRAD_F32>
__global__ void __launch_bounds__(256) adamw_master_kernel(uint16_t* __restrict__ p, float* __restrict__ w,
                                                           const void* __restrict__ grad, float* __restrict__ m,
                                                           float* __restrict__ v, int64_t n, MasterArgs a,
                                                           uint32_t* __restrict__ amax_bits) {
  const int64_t nv = n / 8;
  uint32_t am = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float g[8], mm[8], vv[8], ww[8];
    load_grad8(grad, i, GRAD_F32, g);
    load_f32x8(m, i, mm);
    load_f32x8(v, i, vv);
    load_f32x8(w, i, ww);
#pragma unroll
    for (int j = 0; j < 8; ++j) ww[j] = adam_master_one(ww[j], g[j], mm[j], vv[j], a);
    const uint4 pv = make_uint4(pack2(ww[0], ww[1]), pack2(ww[2], ww[3]), pack2(ww[4], ww[5]), pack2(ww[6], ww[7]));
    reinterpret_cast<uint4*>(p)[i] = pv;
    am = max(am, max(max(absmax_pair_bits(pv.x), absmax_pair_bits(pv.y)),
                     max(absmax_pair_bits(pv.z), absmax_pair_bits(pv.w))));
    store_f32x8(w, i, ww);
    store_f32x8(m, i, mm);
    store_f32x8(v, i, vv);
  }
  for (int64_t i = nv * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float mm = m[i], vv = v[i];
    const float r = adam_master_one(w[i], grad_at(grad, i, GRAD_F32), mm, vv, a);
    m[i] = mm;
    v[i] = vv;
    w[i] = r;
    const uint16_t b = bf16_bits_rn(r);
    p[i] = b;
    am = max(am, absmax_pair_bits((uint32_t)b));
  }
  if (amax_bits) {
    am = __reduce_max_sync(0xffffffffu, am);
    if ((threadIdx.x & 31) == 0 && am) atomicMax(amax_bits, am);
  }
}

// g_i = amax_i / (6 * 448) from float bits (1 when the amax is 0 or not finite)
__global__ void global_scale_from_amax_kernel(const uint32_t* __restrict__ amax_bits, float* __restrict__ g, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float amax = __uint_as_float(amax_bits[i]);
  g[i] = (amax > 0.0f && amax <= 3.402823466e38f) ? __fdiv_rn(amax, 2688.0f) : 1.0f;
}

}  // namespace nvfp4b200

using namespace nvfp4b200;

extern "C" {

int nvfp4b200_swiglu_fwd(const void* gu, void* h, int64_t tokens, int64_t ff, int interleave, uint32_t* ws,
                         float* global_scale_out, void* stream) {
  if (!gu || !h) return NVFP4B200_ERR_INVALID_ARG;
  if ((ws == nullptr) != (global_scale_out == nullptr)) return NVFP4B200_ERR_INVALID_ARG;
  if (interleave != 0 && interleave != 128) return NVFP4B200_ERR_INVALID_ARG;
  if (tokens < 0 || ff <= 0 || ff % 8 || (interleave && ff % 128)) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(gu, 16) || !aligned(h, 16)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (tokens == 0) return NVFP4B200_OK;
  swiglu_fwd_kernel<<<(unsigned)std::min<int64_t>(tokens, (int64_t)sm_count() * 8), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const uint16_t*>(gu), static_cast<uint16_t*>(h), tokens, ff, interleave, ws, global_scale_out);
  return launch_status();
}

int nvfp4b200_swiglu_bwd(const void* gu, const void* dh, void* dgu, int64_t tokens, int64_t ff, int interleave,
                         uint32_t* ws, float* global_scale_out, void* stream) {
  if (!gu || !dh || !dgu) return NVFP4B200_ERR_INVALID_ARG;
  if ((ws == nullptr) != (global_scale_out == nullptr)) return NVFP4B200_ERR_INVALID_ARG;
  if (interleave != 0 && interleave != 128) return NVFP4B200_ERR_INVALID_ARG;
  if (tokens < 0 || ff <= 0 || ff % 8 || (interleave && ff % 128)) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(gu, 16) || !aligned(dh, 16) || !aligned(dgu, 16)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (tokens == 0) return NVFP4B200_OK;
  swiglu_bwd_kernel<<<(unsigned)std::min<int64_t>(tokens, (int64_t)sm_count() * 8), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const uint16_t*>(gu), static_cast<const uint16_t*>(dh), static_cast<uint16_t*>(dgu), tokens, ff,
      interleave, ws, global_scale_out);
  return launch_status();
}

int nvfp4b200_rmsnorm_bwd(const void* x, const void* gamma, const float* inv_rms, const void* dy, const void* dres,
                          void* dx, float* dgamma_acc, int64_t rows, int64_t k, void* stream) {
  if (!x || !inv_rms || !dy || !dx) return NVFP4B200_ERR_INVALID_ARG;
  if (rows < 0 || k <= 0 || k % 8 || k > 2 * 4096) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(dy, 16) || !aligned(dx, 16) || (gamma && !aligned(gamma, 16)) ||
      (dres && !aligned(dres, 16)) || !aligned(inv_rms, 4))
    return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (rows == 0) return NVFP4B200_OK;
  // one resident CTA per SM at k > 4096 (128 registers x 512 threads), two below
  const int64_t ctas = std::min<int64_t>(rows, (int64_t)sm_count() * (k > 4096 ? 1 : 2));
  const int64_t rpc = ceil_div(rows, ctas);
  const unsigned grid = (unsigned)ceil_div(rows, rpc);
  cudaStream_t st = (cudaStream_t)stream;
  auto X = static_cast<const uint16_t*>(x);
  auto G = static_cast<const uint16_t*>(gamma);
  auto DY = static_cast<const uint16_t*>(dy);
  auto DR = static_cast<const uint16_t*>(dres);
  auto DX = static_cast<uint16_t*>(dx);
  if (k <= 4096)
    rmsnorm_bwd_kernel<1><<<grid, RB_THREADS, 0, st>>>(X, G, inv_rms, DY, DR, DX, dgamma_acc, rows, k, rpc);
  else
    rmsnorm_bwd_kernel<2><<<grid, RB_THREADS, 0, st>>>(X, G, inv_rms, DY, DR, DX, dgamma_acc, rows, k, rpc);
  return launch_status();
}

int nvfp4b200_add_bf16(const void* a, const void* b, void* y, int64_t n, void* stream) {
  if (!a || !b || !y) return NVFP4B200_ERR_INVALID_ARG;
  if (n < 0) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(y, 16)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (n == 0) return NVFP4B200_OK;
  add_bf16_kernel<<<grid_for(n / 8 + 1, 256), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const uint16_t*>(a), static_cast<const uint16_t*>(b), static_cast<uint16_t*>(y), n);
  return launch_status();
}

int nvfp4b200_adamw_step(void* param, const void* grad, int grad_dtype, float* m, float* v, int64_t n, float lr,
                         float beta1, float beta2, float eps, float weight_decay, float bias_corr1, float bias_corr2,
                         float grad_scale, void* stream) {
  if (!param || !grad || !m || !v) return NVFP4B200_ERR_INVALID_ARG;
  if (grad_dtype != NVFP4B200_BF16 && grad_dtype != NVFP4B200_F32) return NVFP4B200_ERR_INVALID_ARG;
  if (n < 0) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(param, 16) || !aligned(grad, 16) || !aligned(m, 16) || !aligned(v, 16)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (n == 0) return NVFP4B200_OK;
  AdamArgs a{lr, beta1, beta2, eps, weight_decay, bias_corr1, bias_corr2, grad_scale};
  const unsigned grid = grid_for(n / 8 + 1, 256);
  if (grad_dtype == NVFP4B200_F32)
    adamw_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(static_cast<uint16_t*>(param), grad, m, v, n, a);
  else
    adamw_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(static_cast<uint16_t*>(param), grad, m, v, n, a);
  return launch_status();
}

int nvfp4b200_adamw_master_step(void* param, float* master, const void* grad, int grad_dtype, float* m, float* v,
                                int64_t n, float one_minus_lr_wd, float one_minus_beta1, float beta2,
                                float one_minus_beta2, float eps, float step_size, float bias_corr2_sqrt,
                                float grad_scale, uint32_t* amax_bits, void* stream) {
  if (!param || !master || !grad || !m || !v) return NVFP4B200_ERR_INVALID_ARG;
  if (amax_bits && !aligned(amax_bits, 4)) return NVFP4B200_ERR_MISALIGNED;
  if (grad_dtype != NVFP4B200_BF16 && grad_dtype != NVFP4B200_F32) return NVFP4B200_ERR_INVALID_ARG;
  if (n < 0) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(param, 16) || !aligned(master, 16) || !aligned(grad, 16) || !aligned(m, 16) || !aligned(v, 16))
    return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (n == 0) return NVFP4B200_OK;
  MasterArgs a{one_minus_lr_wd, one_minus_beta1, beta2, one_minus_beta2, eps, step_size, bias_corr2_sqrt, grad_scale};
  const unsigned grid = grid_for(n / 8 + 1, 256);
  auto P = static_cast<uint16_t*>(param);
  if (grad_dtype == NVFP4B200_F32)
    adamw_master_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(P, master, grad, m, v, n, a, amax_bits);
  else
    adamw_master_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(P, master, grad, m, v, n, a, amax_bits);
  return launch_status();
}

int nvfp4b200_global_scale_from_amax(const uint32_t* amax_bits, float* global_scale_out, int64_t n, void* stream) {
  if (!amax_bits || !global_scale_out) return NVFP4B200_ERR_INVALID_ARG;
  if (n < 0 || n > (1 << 20)) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(amax_bits, 4) || !aligned(global_scale_out, 4)) return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (n == 0) return NVFP4B200_OK;
  global_scale_from_amax_kernel<<<(unsigned)ceil_div(n, (int64_t)256), 256, 0, (cudaStream_t)stream>>>(
      amax_bits, global_scale_out, (int)n);
  return launch_status();
}

}  // extern "C"
