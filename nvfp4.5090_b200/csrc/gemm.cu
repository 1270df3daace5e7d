// NVFP4 block-scaled GEMM for B200: tcgen05.mma kind::mxf4nvf4 (scale_vec::4X,
// E4M3 scales per 1x16 block), TMA-fed, TMEM accumulators, warp-specialised
// persistent kernel.
//
//   D[m, n] = epilogue(alpha * sum_k A[m,k] * B[n,k] + bias[n])
//
// Contract of the reference op gn_kernels::cutlass_sm120a_nvfp4_mm
// (cutlass_mm_fp4.cu:167-272): A packed E2M1 [m, k/2] row-major, B packed
// [n, k/2] (the reference's column-major B), scales in the 128x4-atom
// swizzled layout, scalar output scale, optional bf16 bias, bf16 output.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile 128x256 (SW128), B tile 256x256 (SW128)
//               and the scale atoms (plain bulk copies: the swizzled global
//               layout already is the tcgen05 scale-atom layout, so a
//               128-row x 256-k scale slab is 2 KB contiguous).
//   warp 1      TMEM allocator + MMA issuer: per stage, tcgen05.cp moves the
//               scale atoms into TMEM (32x128b.warpx4: each 512-byte atom
//               fills 4 columns across all 128 lanes), then 4 MMAs
//               128x256x64 accumulate into TMEM columns [0, 256).
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, scale, bias,
//               activation, convert and store; the accumulator is released
//               as soon as the last column block is in registers.
// Every mbarrier wait is bounded: on timeout the CTA records
// NVFP4B200_ERR_TIMEOUT in a device error word, drains what it issued and
// returns, so a broken pipeline cannot hang the GPU.
#include "common.cuh"

#include <cuda.h>
#include <algorithm>
#include <mutex>

namespace nvfp4b200 {

__device__ int g_device_error = 0;

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 256;   // BK counts fp4 elements
constexpr int BK_BYTES = BK / 2;              // 128 bytes: one SW128 row
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK_BYTES;        // 16 KB
constexpr int B_BYTES = BN * BK_BYTES;        // 32 KB
constexpr int SFA_BYTES = BM * (BK / 16);     // 2 KB = 4 atoms
constexpr int SFB_BYTES = BN * (BK / 16);     // 4 KB = 2 row groups x 4 atoms
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0;
constexpr int SFA_COL = 256;                  // 4 MMAs x 4 columns
constexpr int SFB_COL = 272;                  // 4 MMAs x 8 columns
constexpr int NUM_BARS = 2 * STAGES + 3;
constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES) + 1024 + 256;
constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;  // about 2 s at 2 GHz
constexpr int GROUP_M = 16;                   // tile raster: 16 m-tiles per group

// Instruction descriptor (kind::mxf4nvf4): A/B E2M1 (=1), K-major, E4M3
// scales, N>>3 at bit 17, M>>4 at bit 24, dense K=64.
constexpr uint32_t IDESC = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

struct Params {
  const uint8_t* sfa;
  const uint8_t* sfb;
  const float* scale_a;
  const float* scale_b;
  const uint16_t* bias;
  const uint16_t* residual;   // bf16 [m, n] with row stride ldd, added after bias
  void* d;
  int64_t m, n, k, ldd;
  int64_t sf_atoms;       // scale atoms per 128-row group = ceil(k/64)
  int64_t sfb_groups;     // 128-row groups of B's scale tensor
  int num_m_tiles, num_n_tiles, num_k_tiles;
  int d_f32, accumulate, epilogue;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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
// Bounded wait for the phase with the given parity to complete.  Returns
// false when the CTA-wide abort flag is raised or the limit expires.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort_flag) return false;
      if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    }
  }
}
__device__ __forceinline__ void raise_abort(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicExch(&g_device_error, NVFP4B200_ERR_TIMEOUT);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_cp_scales(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t sfa, uint32_t sfb,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major with 128-byte swizzle: 8-row
// core groups 1024 bytes apart (SBO), version 1, layout type 2.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Descriptor of one 512-byte scale atom for tcgen05.cp 32x128b: 32 rows of
// 16 bytes, no swizzle, 8-row core groups 128 bytes apart.
__device__ __forceinline__ uint64_t desc_scales(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (8ull << 32) | (1ull << 46);
}

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& mb, int& nb) {
  const int group_size = GROUP_M * p.num_n_tiles;
  const int group = tile / group_size;
  const int first_m = group * GROUP_M;
  const int gsz = min(p.num_m_tiles - first_m, GROUP_M);
  const int in_group = tile - group * group_size;
  mb = first_m + in_group % gsz;
  nb = in_group / gsz;
}

__device__ __forceinline__ int kblocks_in_tile(const Params& p, int kt) {
  const int64_t rem = p.k - (int64_t)kt * BK;
  return (int)imin64(4, (rem + 63) / 64);
}

__device__ __forceinline__ float apply_epi(float v, int epi) {
  if (epi == NVFP4B200_EPI_RELU) return fmaxf(v, 0.0f);
  if (epi == NVFP4B200_EPI_RELU2) {
    const float r = fmaxf(v, 0.0f);
    return r * r;
  }
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(NUM_THREADS, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + STAGES * SFB_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  const uint32_t tmem_full_bar = smem_u32(bars + 2 * STAGES);
  const uint32_t tmem_empty_bar = smem_u32(bars + 2 * STAGES + 1);
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tmem_full_bar, 1);
    mbar_init(tmem_empty_bar, 4);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.num_m_tiles * p.num_n_tiles;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int armed_phase[STAGES];
      for (int s = 0; s < STAGES; ++s) armed_phase[s] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int ngroups_b = (2 * nb + 1 < p.sfb_groups) ? 2 : 1;
        for (int kt = 0; kt < p.num_k_tiles; ++kt) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const int nkb = kblocks_in_tile(p, kt);
          const uint32_t sf_bytes = (uint32_t)nkb * 512u;
          mbar_expect_tx(full_bar(stage), A_BYTES + B_BYTES + sf_bytes * (1 + ngroups_b));
          armed_phase[stage] = (int)phase;
          tma_load_2d(smem_u32(sA + stage * A_BYTES), &tmap_a, full_bar(stage), kt * BK_BYTES, mb * BM);
          tma_load_2d(smem_u32(sB + stage * B_BYTES), &tmap_b, full_bar(stage), kt * BK_BYTES, nb * BN);
          bulk_load(smem_u32(sSFA + stage * SFA_BYTES), p.sfa + ((int64_t)mb * p.sf_atoms + (int64_t)kt * 4) * 512,
                    sf_bytes, full_bar(stage));
          for (int g = 0; g < ngroups_b; ++g)
            bulk_load(smem_u32(sSFB + stage * SFB_BYTES + g * 2048),
                      p.sfb + ((int64_t)(2 * nb + g) * p.sf_atoms + (int64_t)kt * 4) * 512, sf_bytes, full_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        raise_abort(abort_flag);
        // wait (bounded) for the copies this thread issued before returning
        const long long t0 = clock64();
        for (int s = 0; s < STAGES; ++s) {
          if (armed_phase[s] < 0) continue;
          while (!mbar_try_wait(full_bar(s), (uint32_t)armed_phase[s]) && clock64() - t0 < WAIT_LIMIT_CYCLES) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true, issued = false;
      const uint32_t acc = tmem_base + ACC_COL;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        if (!mbar_wait(tmem_empty_bar, acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        acc_phase ^= 1;
        tc_fence_after();
        for (int kt = 0; kt < p.num_k_tiles; ++kt) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = kblocks_in_tile(p, kt);
          const uint32_t a_s = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_s = smem_u32(sB + stage * B_BYTES);
          const uint32_t sfa_s = smem_u32(sSFA + stage * SFA_BYTES);
          const uint32_t sfb_s = smem_u32(sSFB + stage * SFB_BYTES);
          for (int j = 0; j < nkb; ++j) {
            tc_cp_scales(tmem_base + SFA_COL + 4 * j, desc_scales(sfa_s + 512 * j));
            tc_cp_scales(tmem_base + SFB_COL + 8 * j, desc_scales(sfb_s + 512 * j));
            tc_cp_scales(tmem_base + SFB_COL + 8 * j + 4, desc_scales(sfb_s + 2048 + 512 * j));
          }
          const uint64_t adesc = desc_sw128(a_s), bdesc = desc_sw128(b_s);
          for (int j = 0; j < nkb; ++j) {
            // advance 32 bytes (64 fp4) along K inside the swizzled 128-byte row
            tc_mma(acc, adesc + 2 * j, bdesc + 2 * j, tmem_base + SFA_COL + 4 * j, tmem_base + SFB_COL + 8 * j,
                   (kt | j) != 0);
          }
          issued = true;
          tc_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(tmem_full_bar);
      }
      if (!ok) {
        raise_abort(abort_flag);
        if (issued) {
          tc_commit(drain_bar);
          const long long t0 = clock64();
          while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {
          }
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lanes this warp may access: [32*quad, 32*quad+32)
    const float alpha = (p.scale_a ? *p.scale_a : 1.0f) * (p.scale_b ? *p.scale_b : 1.0f);
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      bool ok = mbar_wait(tmem_full_bar, acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) raise_abort(abort_flag);
        break;
      }
      acc_phase ^= 1;
      tc_fence_after();
      const int64_t row = (int64_t)mb * BM + quad * 32 + lane;
      const bool row_ok = row < p.m;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        __syncwarp();  // tcgen05.ld is .sync.aligned: reconverge after the guarded stores
        tmem_ld32(tmem_base + ACC_COL + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 32), r);
        tmem_ld_wait();
        if (c == BN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tmem_empty_bar);
        }
        const int64_t col0 = (int64_t)nb * BN + c * 32;
        if (!row_ok || col0 >= p.n) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * alpha;
        if (p.bias) {
#pragma unroll
          for (int i8 = 0; i8 < 4; ++i8) {
            if (col0 + 8 * i8 >= p.n) break;
            const uint4 bv = __ldg(reinterpret_cast<const uint4*>(p.bias + col0 + 8 * i8));
            const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[8 * i8 + 2 * j] += bf16lo(bw[j]);
              v[8 * i8 + 2 * j + 1] += bf16hi(bw[j]);
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = apply_epi(v[i], p.epilogue);
        if (p.residual) {
          const uint16_t* res = p.residual + row * p.ldd + col0;
#pragma unroll
          for (int i8 = 0; i8 < 4; ++i8) {
            if (col0 + 8 * i8 >= p.n) break;
            const uint4 rv = *reinterpret_cast<const uint4*>(res + 8 * i8);
            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[8 * i8 + 2 * j] += bf16lo(rw[j]);
              v[8 * i8 + 2 * j + 1] += bf16hi(rw[j]);
            }
          }
        }
        if (!p.d_f32) {
          uint16_t* dst = static_cast<uint16_t*>(p.d) + row * p.ldd + col0;
#pragma unroll
          for (int i8 = 0; i8 < 4; ++i8) {
            if (col0 + 8 * i8 >= p.n) break;
            uint4 o;
            o.x = pack_bf16x2(v[8 * i8 + 0], v[8 * i8 + 1]);
            o.y = pack_bf16x2(v[8 * i8 + 2], v[8 * i8 + 3]);
            o.z = pack_bf16x2(v[8 * i8 + 4], v[8 * i8 + 5]);
            o.w = pack_bf16x2(v[8 * i8 + 6], v[8 * i8 + 7]);
            reinterpret_cast<uint4*>(dst)[i8] = o;
          }
        } else {
          float* dst = static_cast<float*>(p.d) + row * p.ldd + col0;
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            if (col0 + 4 * i4 >= p.n) break;
            float4 o = make_float4(v[4 * i4], v[4 * i4 + 1], v[4 * i4 + 2], v[4 * i4 + 3]);
            if (p.accumulate) {
              const float4 old = reinterpret_cast<const float4*>(dst)[i4];
              o.x += old.x;
              o.y += old.y;
              o.z += old.z;
              o.w += old.w;
            }
            reinterpret_cast<float4*>(dst)[i4] = o;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D byte tensor [rows, row_bytes], box 128 bytes x box_rows, 128B swizzle.
static bool make_operand_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)BK_BYTES, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev] > 0 ? cache[dev] : 148;
}

static int run(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
               const float* scale_b, const void* bias, const void* residual, void* d, int d_dtype, int accumulate, int epilogue, int64_t m,
               int64_t n, int64_t k, int64_t ldd, cudaStream_t stream) {
  if (!a || !b || !sfa || !sfb || !d) return NVFP4B200_ERR_INVALID_ARG;
  if (d_dtype != NVFP4B200_BF16 && d_dtype != NVFP4B200_F32) return NVFP4B200_ERR_INVALID_ARG;
  if (epilogue < 0 || epilogue > 2) return NVFP4B200_ERR_INVALID_ARG;
  if (accumulate && d_dtype != NVFP4B200_F32) return NVFP4B200_ERR_INVALID_ARG;
  if (m < 0 || n < 0 || k <= 0 || k % 32 || n % 8 || ldd < n || ldd % 8) return NVFP4B200_ERR_BAD_SHAPE;
  if (m > (1ll << 30) || n > (1ll << 30) || k > (1ll << 30)) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(sfa, 16) || !aligned(sfb, 16) || !aligned(d, 16) ||
      (bias && !aligned(bias, 16)) || (residual && !aligned(residual, 16)))
    return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (m == 0 || n == 0) return NVFP4B200_OK;

  CUtensorMap ma, mb;
  if (!make_operand_map(&ma, a, m, k / 2, BM) || !make_operand_map(&mb, b, n, k / 2, BN)) return NVFP4B200_ERR_CUDA;
  Params p;
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.bias = static_cast<const uint16_t*>(bias);
  p.residual = static_cast<const uint16_t*>(residual);
  p.d = d;
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldd = ldd;
  p.sf_atoms = ceil_div(k, 64);
  p.sfb_groups = ceil_div(n, 128);
  p.num_m_tiles = (int)ceil_div(m, BM);
  p.num_n_tiles = (int)ceil_div(n, BN);
  p.num_k_tiles = (int)ceil_div(k, BK);
  p.d_f32 = d_dtype == NVFP4B200_F32;
  p.accumulate = accumulate;
  p.epilogue = epilogue;
  const int64_t tiles = (int64_t)p.num_m_tiles * p.num_n_tiles;
  const int grid = (int)std::min<int64_t>(tiles, num_sms());
  if (cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
      cudaSuccess)
    return NVFP4B200_ERR_CUDA;
  nvfp4_gemm_kernel<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
  return launch_status();
}

}  // namespace gemm
}  // namespace nvfp4b200

using namespace nvfp4b200;

extern "C" {

int nvfp4b200_get_device_error(int* out) {
  if (!out) return NVFP4B200_ERR_INVALID_ARG;
  int rc = check_device();
  if (rc) return rc;
  int zero = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return NVFP4B200_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out, g_device_error, sizeof(int)) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  return NVFP4B200_OK;
}

int nvfp4b200_gemm(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
                   const float* scale_b, const void* bias, const void* residual, void* d, int d_dtype,
                   int accumulate, int epilogue, int64_t m, int64_t n, int64_t k, int64_t ldd, void* stream) {
  return gemm::run(a, b, sfa, sfb, scale_a, scale_b, bias, residual, d, d_dtype, accumulate, epilogue, m, n, k, ldd,
                   (cudaStream_t)stream);
}

int nvfp4b200_nvfp4_mm(const void* a, const void* b, const void* sfa, const void* sfb, const float* output_scale,
                       const void* bias, void* d, int64_t m, int64_t n, int64_t k, void* stream) {
  return gemm::run(a, b, sfa, sfb, output_scale, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_NONE, m, n, k,
                   n, (cudaStream_t)stream);
}

int nvfp4b200_nvfp4_mm_relu(const void* a, const void* b, const void* sfa, const void* sfb, const float* output_scale,
                            const void* bias, void* d, int64_t m, int64_t n, int64_t k, void* stream) {
  return gemm::run(a, b, sfa, sfb, output_scale, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_RELU, m, n, k,
                   n, (cudaStream_t)stream);
}

int nvfp4b200_nvfp4_mm_relu_2(const void* a, const void* b, const void* sfa, const void* sfb,
                              const float* output_scale, const void* bias, void* d, int64_t m, int64_t n, int64_t k,
                              void* stream) {
  return gemm::run(a, b, sfa, sfb, output_scale, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_RELU2, m, n, k,
                   n, (cudaStream_t)stream);
}

}  // extern "C"
