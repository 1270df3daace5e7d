// NVFP4 block-scaled GEMM for B200: tcgen05.mma.cta_group::2 kind::mxf4nvf4
// (scale_vec::4X, E4M3 scale per 1x16 block), TMA-fed, TMEM accumulators,
// warp-specialised persistent kernel on CTA pairs.
//
//   D[m, n] = epilogue(alpha * sum_k A[m,k] * B[n,k] + bias[n]) + residual[m, n]
//
// Contract of the reference op gn_kernels::cutlass_sm120a_nvfp4_mm
// (cutlass_mm_fp4.cu:167-272): A packed E2M1 [m, k/2] row-major, B packed
// [n, k/2] (the reference's column-major B), scales in the 128x4-atom
// swizzled layout, scalar output scale, optional bf16 bias, bf16 output.
//
// Structure: clusters of 2 CTAs (one per SM) own 256x256 output tiles.
//   CTA r of the pair holds A rows [128r, 128r+128) and B rows
//   [128r, 128r+128) of the tile in shared memory, its own 128 rows of A's
//   scales and all 256 rows of B's scales; each CTA's TMEM accumulates its
//   128 x 256 half of the tile.
//   warp 0      TMA producer (both CTAs): A, B (128B swizzle) and the scale
//               slabs (the swizzled global scale layout already is the
//               tcgen05 scale-atom layout: a 128-row x 256-k slab is 2 KB
//               contiguous, loaded as a 2-D box over 256-byte rows).  All
//               loads signal the leader CTA's stage barrier.
//   warp 1      TMEM allocator (both CTAs) and, in the leader CTA, the MMA
//               issuer: per 256-k stage, 12 tcgen05.cp.cta_group::2 scale
//               copies (32x128b.warpx4: one 512-byte atom -> 4 columns x 128
//               lanes in both CTAs) and 4 MMAs 256x256x64.  One thread's
//               tcgen05 operations execute in issue order, so one scale slot
//               is reused by every stage.  tcgen05.commit multicasts stage
//               release / accumulator-ready to both CTAs.
//   warps 2-9   epilogue (both CTAs): two warps per TMEM lane quadrant, each
//               drains 128 columns in two 64-column chunks and stores them.
// TMEM holds two 256-column accumulators that share 64 columns (buffer 0:
// [0,256), buffer 1: [192,448)) plus the scale slot [448,496).  Tiles
// alternate buffers; the epilogue drains the shared 64 columns first and
// releases them, so the next tile's MMAs start while the epilogue is still
// draining and storing the rest.
// The producer, MMA and epilogue loops run on converged warps; TMA, copy and
// MMA instructions are issued by one elect.sync-chosen lane from warp-uniform
// operands.
// Modes (launch parameters of the same kernel):
//   NVFP4 (kind::mxf4nvf4, E4M3 scale per 1x16 block) or MXFP4 (kind::mxf4,
//   UE8M0 scale per 1x32 block, cutlass_mm_fp4.cu:71-165);
//   epilogues: bf16 store (+bias, ReLU / ReLU^2, residual), f32 store or
//   reduce-add, SwiGLU (gate/up tile -> h, gate/up, max |h|) and SwiGLU
//   backward (dh tile + TMA-loaded gate/up -> dgu, max |dgu|; 4 stages, the
//   fifth stage's shared memory holds the gate/up slots).
// Every mbarrier wait is bounded: on timeout the CTA records
// NVFP4B200_ERR_TIMEOUT in a device error word, drains what it issued and
// returns, so a broken pipeline cannot hang the GPU.  No TMA load uses
// cluster multicast.
#include "common.cuh"

#include <cuda.h>
#include <algorithm>
#include <cstring>
#include <atomic>
#include <mutex>

namespace nvfp4b200 {

__device__ int g_device_error = 0;

namespace gemm {

constexpr int TILE_M = 256, TILE_N = 256, BK = 256;   // pair tile; BK counts fp4 elements per stage
constexpr int KBLOCKS = BK / 64;                      // MMAs (K = 64) per stage
constexpr int CTA_M = 128, CTA_N = 128;               // rows of A / B held by one CTA
constexpr int BK_BYTES = BK / 2;                      // one 128-byte swizzle row per operand row
constexpr int STAGES = 5;
constexpr int A_BYTES = CTA_M * BK_BYTES;
constexpr int B_BYTES = CTA_N * BK_BYTES;
constexpr int SFA_BYTES = 512 * KBLOCKS;              // 128 rows x 16 scales = 4 atoms
constexpr int SFB_BYTES = 1024 * KBLOCKS;             // 2 row groups x 4 atoms
constexpr int SFB_G1 = 512 * KBLOCKS;                 // offset of B's second row group
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr uint32_t STAGE_TX = 2u * STAGE_BYTES;       // bytes landing per stage across the pair
// MXFP4 (1x32 blocks, UE8M0 scales): a stage's 256 k hold 8 scales per row,
// i.e. 2 atoms per 128-row group; the scale buffers are half used.
constexpr int SFA_BYTES_MX = 256 * KBLOCKS;
constexpr int SFB_BYTES_MX = 512 * KBLOCKS;
constexpr int SFB_G1_MX = 256 * KBLOCKS;
constexpr uint32_t STAGE_TX_MX = 2u * (A_BYTES + B_BYTES + SFA_BYTES_MX + SFB_BYTES_MX);
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = 32 * (2 + EPI_WARPS);
constexpr int TMEM_COLS = 512;
constexpr int ACC_COLS = 256;                         // one accumulator buffer
constexpr int ACC1_COL = 192;                         // buffer 1 starts inside buffer 0's last 64 columns
constexpr int SF_COL = 448;                           // scale slot: A 4 x 4 columns, then B 4 x 8 columns
constexpr int SF_COLS = 12 * KBLOCKS;
static_assert(ACC1_COL + ACC_COLS <= SF_COL && SF_COL + SF_COLS <= TMEM_COLS, "TMEM columns");
// Tile schedule: a cluster's first tile is its cluster id; every further
// tile is claimed from a per-launch counter in global memory (dynamic
// scheduling: clusters that start late, for example behind a collective
// kernel holding some SMs, simply claim fewer tiles).  The leader CTA's
// producer warp claims tile ids and publishes them, through a ring of
// TILE_RING slots in both CTAs' shared memory, to every warp of the pair that
// walks tiles; -1 ends the walk.
constexpr int TILE_RING = 4;
// readers of every ring slot: leader MMA warp + 8 epilogue warps, peer producer + 8 epilogue warps
constexpr int RING_READERS = 2 * (1 + EPI_WARPS);
constexpr int SCHED_SLOTS = 256;                      // per-launch tile counters, used round robin
constexpr int NUM_BARS = 2 * STAGES + 3 + EPI_WARPS + 2 * TILE_RING;  // + ring full / empty
constexpr int BAR_BYTES = 512;                        // mbarriers + TMEM address slot + abort flag + tile ring
static_assert(NUM_BARS * 8 + 8 + 4 * TILE_RING <= BAR_BYTES, "barrier area");
constexpr int OUT_CHUNK_BYTES = 32 * 128;             // one epilogue warp's 32 rows x 64 bf16 output chunk
constexpr int OUT_BYTES = EPI_WARPS * OUT_CHUNK_BYTES;  // bf16 output staging for the TMA stores
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_BYTES + 1024 + BAR_BYTES;  // + worst-case 1 KB alignment
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
// SwiGLU-backward epilogue: one stage fewer, two 4 KB slots per epilogue warp
// (the gate and up inputs arrive there by TMA; the gradients leave from there).
constexpr int DSW_STAGES = STAGES - 1;
constexpr int DSW_SLOT_BYTES = 32 * 128;               // 32 rows x 64 bf16, 128-byte swizzle
constexpr int DSW_OUT_BYTES = EPI_WARPS * 2 * DSW_SLOT_BYTES;
constexpr int DSW_SMEM_BYTES = DSW_STAGES * STAGE_BYTES + DSW_OUT_BYTES + 1024 + BAR_BYTES;
static_assert(DSW_SMEM_BYTES <= SMEM_BYTES, "the launch attribute covers both layouts");
constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;  // about 2 s at 2 GHz
// raster: groups of 32 pair-rows (8192 rows); inside a group the m-tiles are
// walked first, so a group's A rows stay in L2 while B streams through once
// per group (8192^3: 88 MB of DRAM reads instead of 136 MB with groups of 8)
constexpr int GROUP_M = 32;

// Instruction descriptor (kind::mxf4nvf4): A/B E2M1 (=1), K-major, E4M3
// scales, N>>3 at bit 17, M>>4 at bit 24 (M = 256 across the CTA pair), K=64.
constexpr uint32_t IDESC =
    (1u << 7) | (1u << 10) | ((uint32_t)(TILE_N >> 3) << 17) | ((uint32_t)(TILE_M >> 4) << 24);

// kind::mxf4 (MXFP4): same fields, UE8M0 scales (bit 23); the scale-factor IDs
// (bits 4-5 for B, 29-30 for A) are set per MMA.
constexpr uint32_t IDESC_MX =
    (1u << 7) | (1u << 10) | ((uint32_t)(TILE_N >> 3) << 17) | (1u << 23) | ((uint32_t)(TILE_M >> 4) << 24);

struct Params {
  const float* scale_a;
  const float* scale_b;
  const uint16_t* bias;
  const uint16_t* residual;  // bf16 [m, n], row stride ldd, added after the activation
  void* d;
  int64_t m, n, k, ldd;
  int64_t sf_atoms;          // scale atoms per 128-row group = ceil(k/64), or ceil(k/128) for MXFP4
  int num_m_tiles, num_n_tiles, num_k_tiles;
  int d_f32, accumulate, epilogue;
  int swiglu;                // B rows interleaved [gate 128 | up 128] per tile: d = silu(gate)*up
  int store_gu;              // swiglu: also store the bf16 gate/up tile (tmap_d)
  uint32_t* h_amax;          // swiglu / dswiglu: atomic max of |h| or |dgu| (float bits), or null
  int dswiglu;               // D = dh -> dgu = SwiGLU backward against gate/up (tmap_h loads, tmap_d stores)
  int stages;                // pipeline stages in use (STAGES, or DSW_STAGES with dswiglu)
  int out_bytes;             // epilogue staging bytes (OUT_BYTES or DSW_OUT_BYTES)
  int mx;                    // MXFP4 operands: 1x32 blocks, UE8M0 scales (kind::mxf4)
  int sched_slot;            // this launch's tile counter: g_tile_sched[sched_slot]
};

// Per-launch tile counters: [0] tiles claimed beyond the first wave, [1]
// clusters that have finished claiming.  The last cluster to finish resets
// both to zero, so a slot is clean for the launch that reuses it (launches
// take slots round robin).  Every wait in the kernel is bounded, so even a
// launch that gives up reaches the reset.
__device__ uint32_t g_tile_sched[SCHED_SLOTS][2];

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Arrive on a barrier of either CTA of the pair (address from mapa).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Arrive with release semantics at cluster scope (orders this thread's prior
// shared-memory accesses, local or remote, before the arrival).
__device__ __forceinline__ void mbar_arrive_release_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void st_cluster_s32(uint32_t cluster_addr, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
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
// Same, with cluster-scope acquire: for barriers that the peer CTA signals.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  Returns
// false when the CTA-wide abort flag is raised or the limit expires.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          long long limit_cycles = WAIT_LIMIT_CYCLES) {
  auto try_once = [&]() { return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
  if (try_once()) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (try_once()) return true;
    if ((it & 63) == 0) {
      if (*abort_flag) return false;
      if (clock64() - t0 > limit_cycles) return false;
    }
  }
}
// Warp-wide bounded wait: every lane polls, the result is uniform across the warp.
template <bool CLUSTER = false>
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = mbar_wait<CLUSTER>(bar, parity, abort_flag);
  return __all_sync(0xffffffffu, ok);
}
// One lane of a converged warp (the lowest), chosen by elect.sync.  Async
// tcgen05 / TMA instructions are issued under this predicate from warp-
// uniform operands, so they issue from uniform registers.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}
__device__ __forceinline__ void raise_abort(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicExch(&g_device_error, NVFP4B200_ERR_TIMEOUT);
}

// 2-D tiled TMA load into this CTA's shared memory; completion bytes are
// counted on `bar`, which may be the pair leader's barrier (.cta_group::2).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
// 3-D tiled TMA load, otherwise as tma_load_2d_pair.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// 2-D tiled TMA store of a shared-memory box (bulk async-group of the issuing
// thread).  The output is marked evict-first in L2: it is not read again by
// this kernel, and keeping the operand tiles resident instead measured 0.3-2%
// faster (8192^3 to 16384^3).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile(
      "{\n\t.reg .b64 pol;\n\t"
      "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], pol;\n\t}" ::"l"(map),
      "r"(src), "r"(x), "r"(y)
      : "memory");
}
// 2-D tiled TMA reduce-add of a shared-memory box into global memory (the
// element type, f32 here, comes from the tensor map; L2 performs the add).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
// 2-D tiled TMA load into this CTA's shared memory, completion on this CTA's barrier.
__device__ __forceinline__ void tma_load_2d_local(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// L2 prefetch of a 2-D tensor box (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y) : "memory");
}
// tma_load_2d_local for data read once: its L2 lines are marked evict-first.
__device__ __forceinline__ void tma_load_2d_local_once(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                                       int y) {
  asm volatile(
      "{\n\t.reg .b64 pol;\n\t"
      "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], pol;\n\t}" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrive once on `bar` (same shared-memory offset) in both CTAs of the pair
// when all prior tcgen05 operations of this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tc_cp_scales_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t sfa, uint32_t sfb,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}
// MXFP4 MMA (kind::mxf4, 1x32 blocks).  A 4-byte TMEM scale cell holds the
// scales of 128 k, two MMAs' worth: the byte the MMA starts at (0 or 2) is
// given both in the scale addresses' two top bits and in the descriptor's
// scale-factor ID fields.
__device__ __forceinline__ void tc_mma_pair_mx(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t sfa, uint32_t sfb,
                                               uint32_t sf_byte, uint32_t accumulate) {
  const uint32_t idesc = IDESC_MX | (sf_byte << 29) | (sf_byte << 4);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa | (sf_byte << 30)), "r"(sfb | (sf_byte << 30))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
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
  return (int)imin64(KBLOCKS, (rem + 63) / 64);
}

__device__ __forceinline__ float apply_epi(float v, int epi) {
  if (epi == NVFP4B200_EPI_RELU) return fmaxf(v, 0.0f);
  if (epi == NVFP4B200_EPI_RELU2) {
    const float r = fmaxf(v, 0.0f);
    return r * r;
  }
  return v;
}

// sigmoid for SwiGLU, the same expression as the element-wise SwiGLU kernels
__device__ __forceinline__ float silu_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 64 accumulator columns [c0, c0+64) of this thread's row -> final values,
// in place (float bits in `v`): scale, bias, activation, residual.
__device__ __forceinline__ void finish64(uint32_t* v, const Params& p, float alpha, int64_t row, int64_t col0,
                                         bool row_ok) {
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
  if (p.bias) {
#pragma unroll
    for (int i8 = 0; i8 < 8; ++i8) {
      if (col0 + 8 * i8 < p.n) {
        const uint4 bv = __ldg(reinterpret_cast<const uint4*>(p.bias + col0 + 8 * i8));
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[8 * i8 + 2 * j] = __float_as_uint(__uint_as_float(v[8 * i8 + 2 * j]) + bf16lo(bw[j]));
          v[8 * i8 + 2 * j + 1] = __float_as_uint(__uint_as_float(v[8 * i8 + 2 * j + 1]) + bf16hi(bw[j]));
        }
      }
    }
  }
  if (p.epilogue != NVFP4B200_EPI_NONE) {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __float_as_uint(apply_epi(__uint_as_float(v[i]), p.epilogue));
  }
  if (p.residual && row_ok) {
    const uint16_t* res = p.residual + row * p.ldd + col0;
#pragma unroll
    for (int i8 = 0; i8 < 8; ++i8) {
      if (col0 + 8 * i8 < p.n) {
        const uint4 rv = *reinterpret_cast<const uint4*>(res + 8 * i8);
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[8 * i8 + 2 * j] = __float_as_uint(__uint_as_float(v[8 * i8 + 2 * j]) + bf16lo(rw[j]));
          v[8 * i8 + 2 * j + 1] = __float_as_uint(__uint_as_float(v[8 * i8 + 2 * j + 1]) + bf16hi(rw[j]));
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                      const __grid_constant__ CUtensorMap tmap_d, const __grid_constant__ CUtensorMap tmap_h,
                      const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nst = p.stages;
  uint8_t* sA = smem;
  uint8_t* sB = sA + nst * A_BYTES;
  uint8_t* sSFA = sB + nst * B_BYTES;
  uint8_t* sSFB = sSFA + nst * SFA_BYTES;
  uint8_t* sOut = sSFB + nst * SFB_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + p.out_bytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* tile_ring = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();          // 0 = leader (issues the MMAs)
  const bool leader = rank == 0;
  auto full_bar = [&](int s) { return smem_u32(bars + s); };             // leader: all bytes of the stage landed
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };    // both: MMAs done with the stage
  const uint32_t tmem_full_bar = smem_u32(bars + 2 * STAGES);            // both: a tile's accumulator is final
  const uint32_t overlap_free_bar = smem_u32(bars + 2 * STAGES + 1);     // leader: shared columns drained
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 2);            // leader: error-path drain
  auto load_bar = [&](int w) { return smem_u32(bars + 2 * STAGES + 3 + w); };  // epilogue warp w's TMA loads
  // tile ring: full (each CTA, one arrival from the leader's producer), empty (leader, RING_READERS arrivals)
  auto ring_full = [&](int i) { return smem_u32(bars + 2 * STAGES + 3 + EPI_WARPS + i); };
  auto ring_empty = [&](int i) { return smem_u32(bars + 2 * STAGES + 3 + EPI_WARPS + TILE_RING + i); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tmem_full_bar, 1);
    mbar_init(overlap_free_bar, 2 * EPI_WARPS);
    mbar_init(drain_bar, 1);
    for (int w = 0; w < EPI_WARPS; ++w) mbar_init(load_bar(w), 1);
    for (int i = 0; i < TILE_RING; ++i) {
      mbar_init(ring_full(i), 1);
      mbar_init(ring_empty(i), RING_READERS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_sfa);
    prefetch_tmap(&tmap_sfb);
    prefetch_tmap(&tmap_d);
    if (p.swiglu || p.dswiglu) prefetch_tmap(&tmap_h);
  }
  if (warp == 1) {
    tmem_alloc2(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.num_m_tiles * p.num_n_tiles;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  // The i-th tile id of this cluster, read from the ring by a whole warp (the
  // slot is then released to the leader's producer).  -1: no more tiles.
  // Returns false when the bounded wait gave up.
  auto ring_read = [&](int i, int& tile) -> bool {
    const int slot = i % TILE_RING;
    if (!warp_wait<true>(ring_full(slot), (uint32_t)(i / TILE_RING) & 1u, abort_flag)) return false;
    tile = tile_ring[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive_release_cluster(map_to_rank(ring_empty(slot), 0));
    return true;
  };

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs, whole warp; one lane issues) ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, armed_parity = 0;  // leader: stages whose barrier expects bytes, and the phase armed
    bool ok = true;
    uint32_t* sched = g_tile_sched[p.sched_slot];
    int tile = cluster_id, next = -1;
    for (int i = 0; ok; ++i) {
      if (leader) {
        // publish tile i in both CTAs' rings
        const int slot = i % TILE_RING;
        if (!warp_wait<true>(ring_empty(slot), ((uint32_t)(i / TILE_RING) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          tile_ring[slot] = tile;
          st_cluster_s32(map_to_rank(smem_u32((const void*)(tile_ring + slot)), 1), tile);
          mbar_arrive_release_cluster(map_to_rank(ring_full(slot), 0));
          mbar_arrive_release_cluster(map_to_rank(ring_full(slot), 1));
        }
        __syncwarp();
        if (tile < 0) break;
        // claim the tile after this one now: the atomic's latency hides behind this tile's loads
        if (lane == 0) {
          const uint32_t c = atomicAdd(&sched[0], 1u);
          next = c < (uint32_t)(total_tiles - num_clusters) ? num_clusters + (int)c : -1;
        }
        next = __shfl_sync(0xffffffffu, next, 0);
      } else {
        if (!ring_read(i, tile)) {
          ok = false;
          break;
        }
        if (tile < 0) break;
      }
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int a_row = mb * TILE_M + (int)rank * CTA_M;
      const int b_row = nb * TILE_N + (int)rank * CTA_N;
      // scale slabs are rows of 256 bytes; slab (group, kt) starts at row (group * atoms + 4 * kt) * 2
      const int64_t sfa_row0 = ((int64_t)(2 * mb + (int)rank) * p.sf_atoms) * 2;
      for (int kt = 0; kt < p.num_k_tiles; ++kt) {
        if (!warp_wait(empty_bar(stage), phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t lbar = map_to_rank(full_bar(stage), 0);
        const int sf_dy = (p.mx ? KBLOCKS : 2 * KBLOCKS) * kt;   // scale rows of 256 bytes per stage
        if (elect_one()) {
          if (leader) mbar_expect_tx(full_bar(stage), p.mx ? STAGE_TX_MX : STAGE_TX);
          tma_load_2d_pair(smem_u32(sA + stage * A_BYTES), &tmap_a, lbar, kt * BK_BYTES, a_row);
          tma_load_2d_pair(smem_u32(sB + stage * B_BYTES), &tmap_b, lbar, kt * BK_BYTES, b_row);
          tma_load_2d_pair(smem_u32(sSFA + stage * SFA_BYTES), &tmap_sfa, lbar, 0, (int)(sfa_row0 + sf_dy));
          // both 128-row scale groups of the B tile in one load (3-D map: bytes, slab rows, group)
          tma_load_3d_pair(smem_u32(sSFB + stage * SFB_BYTES), &tmap_sfb, lbar, 0, sf_dy, 2 * nb);
        }
        __syncwarp();
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == nst) {
          stage = 0;
          phase ^= 1;
        }
      }
      tile = next;
    }
    if (leader && lane == 0) {
      // this cluster claims no more tiles; the last cluster to get here resets the counters
      if (atomicAdd(&sched[1], 1u) == (uint32_t)num_clusters - 1u) {
        atomicExch(&sched[0], 0u);
        atomicExch(&sched[1], 0u);
      }
    }
    if (!ok && lane == 0) {
      raise_abort(abort_flag);
      if (leader) {  // the leader's stage barriers count both CTAs' copies: let them land
        const long long t0 = clock64();
        for (int st = 0; st < nst; ++st) {
          if (!((armed >> st) & 1u)) continue;
          while (!mbar_try_wait(full_bar(st), (armed_parity >> st) & 1u) && clock64() - t0 < WAIT_LIMIT_CYCLES) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA, whole warp; one lane issues) ----------------
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      const uint32_t sfa_t = tmem_base + SF_COL;
      const uint32_t sfb_t = sfa_t + 4 * KBLOCKS;
      for (int it = 0; ok; ++it) {   // it: tiles of this cluster so far; buffer = it & 1
        int tile;
        if (!ring_read(it, tile)) {
          ok = false;
          break;
        }
        if (tile < 0) break;
        // The previous tile's epilogue has drained the 64 columns its buffer
        // shares with this tile's buffer.  Every epilogue warp finished the tile
        // before it first, so this buffer's own previous use is drained too.
        if (!warp_wait<true>(overlap_free_bar, (it & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + ((it & 1) ? ACC1_COL : 0);
        for (int kt = 0; kt < p.num_k_tiles; ++kt) {
          // operands and scale atoms of both CTAs landed
          if (!warp_wait<true>(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = kblocks_in_tile(p, kt);
          const uint64_t adesc = desc_sw128(smem_u32(sA + stage * A_BYTES));
          const uint64_t bdesc = desc_sw128(smem_u32(sB + stage * B_BYTES));
          const uint64_t sfa_d = desc_scales(smem_u32(sSFA + stage * SFA_BYTES));
          const uint64_t sfb_d = desc_scales(smem_u32(sSFB + stage * SFB_BYTES));
          if (elect_one()) {
            // per MMA: its three scale atoms (A, B rows 0-127, B rows 128-255), then
            // the MMA, which advances 32 bytes (64 fp4) along K inside the swizzled
            // row; a full stage is unrolled (measured 5-6% faster than the loop)
            auto kblock = [&](int j) {
              tc_cp_scales_pair(sfa_t + 4 * j, sfa_d + 32 * j);  // +512 bytes per atom
              tc_cp_scales_pair(sfb_t + 8 * j, sfb_d + 32 * j);
              tc_cp_scales_pair(sfb_t + 8 * j + 4, sfb_d + (SFB_G1 >> 4) + 32 * j);
              tc_mma_pair(acc, adesc + 2 * j, bdesc + 2 * j, sfa_t + 4 * j, sfb_t + 8 * j, (kt | j) != 0);
            };
            if (!p.mx && nkb == KBLOCKS) {
#pragma unroll
              for (int j = 0; j < KBLOCKS; ++j) kblock(j);
            } else if (!p.mx) {
              for (int j = 0; j < nkb; ++j) kblock(j);
            } else {
              for (int j = 0; j < nkb; ++j) {
                const int a = j >> 1;   // an atom's 4 scales per row cover the 128 k of MMAs 2a, 2a + 1
                if ((j & 1) == 0) {
                  tc_cp_scales_pair(sfa_t + 4 * a, sfa_d + 32 * a);
                  tc_cp_scales_pair(sfb_t + 8 * a, sfb_d + 32 * a);
                  tc_cp_scales_pair(sfb_t + 8 * a + 4, sfb_d + (SFB_G1_MX >> 4) + 32 * a);
                }
                tc_mma_pair_mx(acc, adesc + 2 * j, bdesc + 2 * j, sfa_t + 4 * a, sfb_t + 8 * a, 2u * (j & 1),
                               (kt | j) != 0);
              }
            }
            tc_commit_pair(empty_bar(stage));
          }
          __syncwarp();
          issued = true;
          if (++stage == nst) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (elect_one()) tc_commit_pair(tmem_full_bar);
        __syncwarp();
      }
      if (!ok && elect_one()) {  // the lane that issued the MMAs commits the drain
        raise_abort(abort_flag);
        if (issued) {
          tc_commit_pair(drain_bar);
          const long long t0 = clock64();
          while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {
          }
        }
      }
    }
  } else if (p.dswiglu) {
    // ---------------- SwiGLU-backward epilogue (warps 2..9, both CTAs) ----------------
    // The accumulator is dh (rounded to bf16 exactly as a stored dh would be);
    // the gate/up tensor gu [m, 2n] holds [gate 128 | up 128] per 256 columns,
    // and dgu (same layout) = (dgate, dup) of swiglu_grad.  Warp (quad, half)
    // owns rows [32 quad, +32) of its CTA's half tile and dh columns
    // [128 half, +128), i.e. interleave block t = 2 nb + half (gu columns
    // [256 t, 256 t + 256)).  Per 64-column chunk the warp's two slots receive
    // the gate and the up values by TMA, are overwritten with the two
    // gradients and stored.  The next chunk's (or next tile's first chunk's)
    // loads are issued as soon as the stores have read the slots, so the first
    // chunk of a tile is in flight while the warp waits for the accumulator.
    // At the start of a chunk the next chunk's gate/up boxes are prefetched
    // into L2, so its loads, issued one chunk's arithmetic later, find them
    // there; gu is read once, so its loads mark the lines evict-first (both
    // together: -3% at K = 4096, -4% at K = 8192; the epilogue's gu/dgu
    // traffic, not its arithmetic, is what lengthens this GEMM).
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int ew = warp - 2;
    const uint32_t leader_overlap_free = map_to_rank(overlap_free_bar, 0);
    const float alpha = (p.scale_a ? *p.scale_a : 1.0f) * (p.scale_b ? *p.scale_b : 1.0f);
    const uint64_t alpha2 = f2pack(alpha, alpha);
    const uint32_t slot_g = smem_u32(sOut + ew * 2 * DSW_SLOT_BYTES);
    const uint32_t slot_u = slot_g + DSW_SLOT_BYTES;
    const uint32_t lbar = load_bar(ew);
    uint32_t ld_par = 0;
    bool ld_pending = false;
    // max |dgu| over this warp's rows, taken on the fp32 values before rounding
    // (round-to-nearest is monotonic, so bf16(max |x|) = max |bf16(x)|; fmaxf
    // skips NaN like the element-wise kernels' amax)
    float amax = 0.0f;
    auto issue_loads = [&](int mb_, int nb_, int c) {
      const int y = mb_ * TILE_M + (int)rank * CTA_M + quad * 32;
      const int gcol = 256 * (2 * nb_ + half) + 64 * c;   // gate column of the chunk (elements)
      if (elect_one()) {
        mbar_expect_tx(lbar, 2 * DSW_SLOT_BYTES);
        tma_load_2d_local_once(slot_g, &tmap_h, lbar, 2 * gcol, y);          // x in bytes
        tma_load_2d_local_once(slot_u, &tmap_h, lbar, 2 * (gcol + 128), y);
      }
      __syncwarp();
      ld_pending = true;
    };
    auto prefetch_gu = [&](int mb_, int nb_, int c) {
      const int y = mb_ * TILE_M + (int)rank * CTA_M + quad * 32;
      const int gcol = 256 * (2 * nb_ + half) + 64 * c;
      if (elect_one()) {
        tma_prefetch_l2_2d(&tmap_h, 2 * gcol, y);
        tma_prefetch_l2_2d(&tmap_h, 2 * (gcol + 128), y);
      }
      __syncwarp();
    };
    int it = 0;
    int tile = -1, next_tile = -1;
    bool ok = ring_read(0, tile);
    if (ok && tile >= 0) {
      int mb0, nb0;
      tile_coords(tile, p, mb0, nb0);
      issue_loads(mb0, nb0, half == 1 ? 1 : 0);   // tile 0 uses buffer 0: half 1 drains chunk 1 first
    }
    for (; ok && tile >= 0; tile = next_tile, ++it) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      ok = __all_sync(0xffffffffu, mbar_wait(tmem_full_bar, (uint32_t)(it & 1), abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int buf = it & 1;
      const int first = (buf == 0 && half == 1) ? 1 : 0;   // the chunk in the columns both buffers share
      const int y0 = mb * TILE_M + (int)rank * CTA_M + quad * 32;
      const bool row_ok = y0 + lane < p.m;
      const uint32_t tbase =
          tmem_base + (buf ? ACC1_COL : 0) + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * 128);
      const uint32_t orow_g = slot_g + lane * 128, orow_u = slot_u + lane * 128;
      for (int r = 0; r < 2; ++r) {
        const int c = r ^ first;
        if (r == 0) {
          prefetch_gu(mb, nb, c ^ 1);
        } else {   // the next tile's first chunk
          if (!ring_read(it + 1, next_tile)) {
            ok = false;
            break;
          }
          if (next_tile >= 0) {
            int mb2, nb2;
            tile_coords(next_tile, p, mb2, nb2);
            prefetch_gu(mb2, nb2, (((it + 1) & 1) == 0 && half == 1) ? 1 : 0);
          }
        }
        uint32_t acc[64];
        __syncwarp();
        tmem_ld32(tbase + c * 64, acc);
        tmem_ld32(tbase + c * 64 + 32, acc + 32);
        tmem_ld_wait();
        if (r == 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_overlap_free);
        }
        ok = warp_wait(lbar, ld_par, abort_flag);
        if (!ok) break;   // the load stays pending: waited for (bounded) before exit
        ld_par ^= 1u;
        ld_pending = false;
        // two 32-column halves: all shared loads of a half first, then its 16
        // independent element pairs, then its stores (a load after a store
        // cannot move up, so interleaving them would serialise the pairs)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t gw[16], uw[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t off = (uint32_t)(((4 * hh + q) ^ (lane & 7)) << 4);
            const uint4 gv = ld_shared_v4(orow_g + off);
            const uint4 uv = ld_shared_v4(orow_u + off);
            gw[4 * q] = gv.x; gw[4 * q + 1] = gv.y; gw[4 * q + 2] = gv.z; gw[4 * q + 3] = gv.w;
            uw[4 * q] = uv.x; uw[4 * q + 1] = uv.y; uw[4 * q + 2] = uv.z; uw[4 * q + 3] = uv.w;
          }
          uint32_t og[16], ou[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int i = 32 * hh + 2 * e;
            const uint64_t dh2 = f2mul(f2pack(__uint_as_float(acc[i]), __uint_as_float(acc[i + 1])), alpha2);
            const uint32_t dw = pack_bf16x2(f2lo(dh2), f2hi(dh2));   // dh as a stored bf16 dh
            const uint64_t g2 = bf16x2_to_f2(gw[e]);
            const uint64_t sg2 = f2pack(silu_sigmoid(f2lo(g2)), silu_sigmoid(f2hi(g2)));
            uint64_t dg2, du2;
            swiglu_grad2(g2, bf16x2_to_f2(uw[e]), bf16x2_to_f2(dw), sg2, dg2, du2);
            og[e] = pack_bf16x2(f2lo(dg2), f2hi(dg2));
            ou[e] = pack_bf16x2(f2lo(du2), f2hi(du2));
            if (row_ok)
              amax = fmaxf(fmaxf(amax, fmaxf(fabsf(f2lo(dg2)), fabsf(f2hi(dg2)))),
                           fmaxf(fabsf(f2lo(du2)), fabsf(f2hi(du2))));
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t off = (uint32_t)(((4 * hh + q) ^ (lane & 7)) << 4);
            st_shared_v4(orow_g + off, og[4 * q], og[4 * q + 1], og[4 * q + 2], og[4 * q + 3]);
            st_shared_v4(orow_u + off, ou[4 * q], ou[4 * q + 1], ou[4 * q + 2], ou[4 * q + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        const int gcol = 256 * (2 * nb + half) + 64 * c;
        if (lane == 0 && y0 < p.m) {
          tma_store_2d(&tmap_d, slot_g, 2 * gcol, y0);
          tma_store_2d(&tmap_d, slot_u, 2 * (gcol + 128), y0);
          bulk_commit();
        }
        if (lane == 0) bulk_wait_read();   // the slots are free again
        __syncwarp();
        if (r == 0) {
          issue_loads(mb, nb, c ^ 1);
        } else {   // the next tile's first chunk goes out while this warp waits for its accumulator
          if (next_tile >= 0) {
            int mb2, nb2;
            tile_coords(next_tile, p, mb2, nb2);
            issue_loads(mb2, nb2, (((it + 1) & 1) == 0 && half == 1) ? 1 : 0);
          }
        }
      }
      if (!ok) break;
    }
    if (!ok && lane == 0) raise_abort(abort_flag);
    if (ld_pending) {   // a load still in flight lands before the CTA exits
      if (lane == 0) {
        const long long t0 = clock64();
        while (!mbar_try_wait(lbar, ld_par) && clock64() - t0 < WAIT_LIMIT_CYCLES) {
        }
      }
      __syncwarp();
    }
    if (p.h_amax) {
      const uint32_t a16 = __reduce_max_sync(0xffffffffu, pack_bf16x2(amax, 0.0f) & 0xFFFFu);
      if (lane == 0 && a16) atomicMax(p.h_amax, a16 << 16);
    }
    if (lane == 0) bulk_wait_all();
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int quad = warp & 3;               // TMEM lanes [32*quad, 32*quad+32)
    const int half = (warp - 2) >> 2;        // accumulator columns [128*half, 128*half+128)
    const uint32_t leader_overlap_free = map_to_rank(overlap_free_bar, 0);
    const float alpha = (p.scale_a ? *p.scale_a : 1.0f) * (p.scale_b ? *p.scale_b : 1.0f);
    for (int it = 0;; ++it) {
      int tile;
      if (!ring_read(it, tile)) {
        if (lane == 0) raise_abort(abort_flag);
        break;
      }
      if (tile < 0) break;
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      bool ok = mbar_wait(tmem_full_bar, (uint32_t)(it & 1), abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) raise_abort(abort_flag);
        break;
      }
      tc_fence_after();
      const int buf = it & 1;
      // This warp's 64-column chunk inside the columns the two buffers share is
      // drained first: buffer 0's tile columns [192,256) (half 1, chunk 1) and
      // buffer 1's tile columns [0,64) (half 0, chunk 0).
      const int first = (buf == 0 && half == 1) ? 1 : 0;
      const int64_t row = (int64_t)mb * TILE_M + (int64_t)rank * CTA_M + quad * 32 + lane;
      const bool row_ok = row < p.m;
      const int64_t colbase = (int64_t)nb * TILE_N + half * 128;
      const uint32_t tbase =
          tmem_base + (buf ? ACC1_COL : 0) + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * 128);
      if (p.swiglu) {
        // SwiGLU: this warp owns gate columns [64 half, +64) and the matching up
        // columns [128 + 64 half, +64) of the tile.  The operand holding the
        // columns shared with the other accumulator buffer is drained first
        // (buffer 0: the up chunk of half 1; buffer 1: the gate chunk of half
        // 0), then released.  gate/up are rounded to bf16 (and stored when
        // asked), h = silu(gate) * up is computed from the rounded values and
        // stored as bf16; |h| feeds the global amax.
        const uint32_t obuf = smem_u32(sOut + (warp - 2) * OUT_CHUNK_BYTES);
        const uint32_t orow = obuf + lane * 128;
        const int y0 = mb * TILE_M + (int)rank * CTA_M + quad * 32;
        const uint32_t lane_base = tmem_base + (buf ? ACC1_COL : 0) + ((uint32_t)(quad * 32) << 16);
        const int up_first = (buf == 0 && half == 1) ? 1 : 0;
        const int col_first = up_first ? 128 + 64 * half : 64 * half;   // tile columns
        const int col_second = up_first ? 64 * half : 128 + 64 * half;
        uint32_t fr[64];   // first operand, bf16-rounded values as float bits
        __syncwarp();
        tmem_ld32(lane_base + col_first, fr);
        tmem_ld32(lane_base + col_first + 32, fr + 32);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(leader_overlap_free);
        const bool y_ok = y0 < p.m;
        // bf16-round the first operand; stage and store it as part of gate/up
        if (lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            w[e] = pack_bf16x2(__uint_as_float(fr[8 * j + 2 * e]) * alpha, __uint_as_float(fr[8 * j + 2 * e + 1]) * alpha);
            fr[8 * j + 2 * e] = __float_as_uint(bf16lo(w[e]));
            fr[8 * j + 2 * e + 1] = __float_as_uint(bf16hi(w[e]));
          }
          if (p.store_gu) st_shared_v4(orow + ((j ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
        if (p.store_gu) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && y_ok) {
            tma_store_2d(&tmap_d, obuf, (int)(2 * ((int64_t)nb * TILE_N + col_first)), y0);
            bulk_commit();
          }
        }
        uint32_t hw[32];   // h as packed bf16 pairs (64 values)
        float hmax = 0.0f;  // max |h| before rounding: bf16(max |h|) = max |bf16(h)| (NaN skipped)
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          uint32_t sr[32];
          tmem_ld32(lane_base + col_second + 32 * pp, sr);
          tmem_ld_wait();
          if (pp == 0 && p.store_gu) {
            if (lane == 0) bulk_wait_read();
            __syncwarp();
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 8 * j + 2 * e;   // value index inside this 32-column pass
              w[e] = pack_bf16x2(__uint_as_float(sr[i]) * alpha, __uint_as_float(sr[i + 1]) * alpha);
              const float s0 = bf16lo(w[e]), s1 = bf16hi(w[e]);
              const float f0 = __uint_as_float(fr[32 * pp + i]), f1 = __uint_as_float(fr[32 * pp + i + 1]);
              const float g0 = up_first ? s0 : f0, g1 = up_first ? s1 : f1;
              const float u0 = up_first ? f0 : s0, u1 = up_first ? f1 : s1;
              const float h0 = g0 * silu_sigmoid(g0) * u0, h1 = g1 * silu_sigmoid(g1) * u1;
              hw[16 * pp + 4 * j + e] = pack_bf16x2(h0, h1);
              hmax = fmaxf(hmax, fmaxf(fabsf(h0), fabsf(h1)));
            }
            if (p.store_gu) st_shared_v4(orow + (((4 * pp + j) ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
          }
        }
        if (p.store_gu) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && y_ok) {
            tma_store_2d(&tmap_d, obuf, (int)(2 * ((int64_t)nb * TILE_N + col_second)), y0);
            bulk_commit();
          }
        }
        // h: 64 columns at h column 128 nb + 64 half
        if (lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(orow + ((j ^ (lane & 7)) << 4), hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && y_ok) {
          tma_store_2d(&tmap_h, obuf, (int)(2 * ((int64_t)nb * (TILE_N / 2) + 64 * half)), y0);
          bulk_commit();
        }
        if (p.h_amax) {
          const uint32_t h16 = __reduce_max_sync(0xffffffffu, row_ok ? (pack_bf16x2(hmax, 0.0f) & 0xFFFFu) : 0u);
          if (lane == 0 && h16) atomicMax(p.h_amax, h16 << 16);
        }
      } else if (!p.d_f32) {
        // bf16: each 32-row x 64-column chunk goes through this warp's shared
        // staging buffer (128-byte swizzle: 16-byte piece j of row i at
        // (j ^ (i % 8)) * 16) and out with one TMA store, which drops rows and
        // columns outside the matrix.
        const uint32_t obuf = smem_u32(sOut + (warp - 2) * OUT_CHUNK_BYTES);
        const uint32_t orow = obuf + lane * 128;
        const int y0 = mb * TILE_M + (int)rank * CTA_M + quad * 32;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int c = r ^ first;
          uint32_t acc[64];
          __syncwarp();
          tmem_ld32(tbase + c * 64, acc);
          tmem_ld32(tbase + c * 64 + 32, acc + 32);
          tmem_ld_wait();
          if (r == 0) {  // the shared columns are in registers: the next tile's MMAs may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_overlap_free);
          }
          finish64(acc, p, alpha, row, colbase + c * 64, row_ok);
          if (lane == 0) bulk_wait_read();  // the previous store has read the staging buffer
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_v4(orow + ((j ^ (lane & 7)) << 4),
                         pack_bf16x2(__uint_as_float(acc[8 * j + 0]), __uint_as_float(acc[8 * j + 1])),
                         pack_bf16x2(__uint_as_float(acc[8 * j + 2]), __uint_as_float(acc[8 * j + 3])),
                         pack_bf16x2(__uint_as_float(acc[8 * j + 4]), __uint_as_float(acc[8 * j + 5])),
                         pack_bf16x2(__uint_as_float(acc[8 * j + 6]), __uint_as_float(acc[8 * j + 7])));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && y0 < p.m && colbase + c * 64 < p.n) {  // x in bytes (the map views d as bytes)
            tma_store_2d(&tmap_d, obuf, (int)(2 * (colbase + c * 64)), y0);
            bulk_commit();
          }
        }
      } else {
        // f32: each 32-row x 32-column piece (4 KB) goes through the staging
        // buffer and out with one TMA store, or with a TMA reduce-add when
        // accumulating (D += result, the add done in L2; no read of D here).
        const uint32_t obuf = smem_u32(sOut + (warp - 2) * OUT_CHUNK_BYTES);
        const uint32_t orow = obuf + lane * 128;
        const int y0 = mb * TILE_M + (int)rank * CTA_M + quad * 32;
#pragma unroll 1
        for (int r = 0; r < 2; ++r) {
          const int c = r ^ first;
          uint32_t acc[64];
          __syncwarp();
          tmem_ld32(tbase + c * 64, acc);
          tmem_ld32(tbase + c * 64 + 32, acc + 32);
          tmem_ld_wait();
          if (r == 0) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_overlap_free);
          }
          finish64(acc, p, alpha, row, colbase + c * 64, row_ok);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (lane == 0) bulk_wait_read();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              st_shared_v4(orow + ((j ^ (lane & 7)) << 4), acc[32 * hh + 4 * j], acc[32 * hh + 4 * j + 1],
                           acc[32 * hh + 4 * j + 2], acc[32 * hh + 4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            const int64_t x0 = colbase + c * 64 + 32 * hh;  // element column (the f32 map counts elements)
            if (lane == 0 && y0 < p.m && x0 < p.n) {
              if (p.accumulate)
                tma_reduce_add_2d(&tmap_d, obuf, (int)x0, y0);
              else
                tma_store_2d(&tmap_d, obuf, (int)x0, y0);
              bulk_commit();
            }
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // output stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc2(tmem_base, TMEM_COLS);
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

// 2-D f32 tensor [rows, cols] (row stride ld elements) with box {32, 32} and
// 128-byte swizzle: the output map of f32 results (store and reduce-add).
static bool make_map_f32(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D byte tensor [rows, row_bytes] with box {box_x bytes, box_rows}.
static bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box_x, int box_rows,
                     CUtensorMapSwizzle swz, int64_t stride_bytes = 0) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(stride_bytes ? stride_bytes : row_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Scale tensor as [groups][rows_per_group][256 bytes] (a 128-row group's
// atoms are rows_per_group rows of 256 bytes); one box = one k-slab
// (box_rows rows) of two consecutive groups.  Groups past the end read zeros.
static bool make_map_sf_groups(CUtensorMap* map, const void* base, int64_t groups, int64_t rows_per_group,
                               int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {256, (cuuint64_t)rows_per_group, (cuuint64_t)groups};
  cuuint64_t strides[2] = {256, (cuuint64_t)(rows_per_group * 256)};
  cuuint32_t box[3] = {256, (cuuint32_t)box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DeviceInfo {
  int sms = 0;
  int max_clusters = 0;
};

// Process-wide cap on the SMs a GEMM launch occupies (0 = no cap).
static std::atomic<int> g_gemm_max_sms{0};

static DeviceInfo device_info() {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return DeviceInfo{148, 74};
  std::lock_guard<std::mutex> lk(mu);
  DeviceInfo& d = cache[dev];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * std::max(1, d.sms / 2), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) ==
            cudaSuccess &&
        cudaOccupancyMaxActiveClusters(&n, nvfp4_gemm_kernel, &cfg) == cudaSuccess && n > 0)
      d.max_clusters = n;
    else
      d.max_clusters = std::max(1, d.sms / 2);
    cudaGetLastError();
  }
  return d;
}

// SwiGLU outputs of the gate/up GEMM (nvfp4b200_gemm_swiglu): d is h [m, n/2].
struct SwigluOut {
  void* gu;          // bf16 [m, n] gate/up (interleaved like B's rows), or null
  uint32_t* ws;      // 2-word amax workspace (zero on entry and on return), or null
  float* g_out;      // global scale of h = amax(h) / (6 * 448), or null
};

// g = amax / 2688 from the amax bits in ws[0] (1 when 0 or not finite); resets ws[0].
// Failure-path self-test: one warp waits, through the pipeline's bounded wait,
// for a barrier phase that nothing completes; the wait gives up after
// limit_cycles, records NVFP4B200_ERR_TIMEOUT and the kernel returns.
__global__ void wait_selftest_kernel(long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bar), 0, &abort_flag, limit_cycles));
  if (!ok && threadIdx.x == 0) raise_abort(&abort_flag);
}

__global__ void h_scale_finalize_kernel(uint32_t* ws, float* g_out) {
  const float amax = __uint_as_float(ws[0]);
  *g_out = (amax > 0.0f && amax <= 3.402823466e38f) ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  ws[0] = 0u;
}

// SwiGLU backward in the epilogue: gate/up input [m, 2n] (interleaved blocks of
// 128), d is the dgu output [m, 2n]; optional global scale of dgu.
struct DswigluIn {
  const void* gu;
  uint32_t* ws;
  float* g_out;
};

static int run(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
               const float* scale_b, const void* bias, const void* residual, void* d, int d_dtype, int accumulate,
               int epilogue, int64_t m, int64_t n, int64_t k, int64_t ldd, cudaStream_t stream,
               const SwigluOut* sw = nullptr, const DswigluIn* dsw = nullptr, int mx = 0) {
  if (!a || !b || !sfa || !sfb || !d) return NVFP4B200_ERR_INVALID_ARG;
  if (d_dtype != NVFP4B200_BF16 && d_dtype != NVFP4B200_F32) return NVFP4B200_ERR_INVALID_ARG;
  if (epilogue < 0 || epilogue > 2) return NVFP4B200_ERR_INVALID_ARG;
  if (accumulate && d_dtype != NVFP4B200_F32) return NVFP4B200_ERR_INVALID_ARG;
  if (residual && d_dtype != NVFP4B200_BF16) return NVFP4B200_ERR_INVALID_ARG;
  if (m < 0 || n < 0 || k <= 0 || k % 32 || n % 8 || ldd < n || ldd % 8) return NVFP4B200_ERR_BAD_SHAPE;
  if (m > (1ll << 30) || n > (1ll << 30) || k > (1ll << 30)) return NVFP4B200_ERR_BAD_SHAPE;
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(sfa, 16) || !aligned(sfb, 16) || !aligned(d, 16) ||
      (bias && !aligned(bias, 16)) || (residual && !aligned(residual, 16)))
    return NVFP4B200_ERR_MISALIGNED;
  int rc = check_device();
  if (rc) return rc;
  if (m == 0 || n == 0) return NVFP4B200_OK;

  // scale atoms (512 bytes: 128 rows x 4 scales) per 128-row group: 64 k each
  // (NVFP4, 1x16 blocks) or 128 k each (MXFP4, 1x32 blocks)
  const int64_t sf_atoms = ceil_div(k, mx ? 128 : 64);
  const int sf_box_rows = mx ? KBLOCKS : 2 * KBLOCKS;
  const int64_t pad_m = round_up(m, 128), pad_n = round_up(n, 128);
  CUtensorMap ma, mb, msa, msb, md;
  memset(&md, 0, sizeof(md));
  // scale tensors viewed as rows of 256 bytes (pad_rows * pad_cols is a multiple of 512)
  const CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_map(&ma, a, m, k / 2, BK_BYTES, CTA_M, swz) ||
      !make_map(&mb, b, n, k / 2, BK_BYTES, CTA_N, swz) ||
      !make_map(&msa, sfa, pad_m * sf_atoms * 4 / 256, 256, 256, sf_box_rows, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_sf_groups(&msb, sfb, pad_n / 128, sf_atoms * 2, sf_box_rows))
    return NVFP4B200_ERR_CUDA;
  // bf16 output viewed as bytes: [m rows, 2n bytes], row stride 2*ldd, boxes of 32 rows x 128 bytes
  CUtensorMap mh;
  memset(&mh, 0, sizeof(mh));
  if (dsw) {
    // gate/up input and dgu output, both bf16 [m, 2n] viewed as bytes
    if (!make_map(&mh, dsw->gu, m, 4 * n, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B, 4 * n) ||
        !make_map(&md, d, m, 4 * n, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B, 4 * n))
      return NVFP4B200_ERR_CUDA;
  } else if (sw) {
    // h [m, n/2] and the optional gate/up [m, n], both bf16 viewed as bytes
    if (!make_map(&mh, d, m, n, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B, n)) return NVFP4B200_ERR_CUDA;
    if (sw->gu && !make_map(&md, sw->gu, m, 2 * n, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B, 2 * n))
      return NVFP4B200_ERR_CUDA;
  } else {
    if (d_dtype == NVFP4B200_BF16 && !make_map(&md, d, m, 2 * n, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B, 2 * ldd))
      return NVFP4B200_ERR_CUDA;
    if (d_dtype == NVFP4B200_F32 && !make_map_f32(&md, d, m, n, ldd)) return NVFP4B200_ERR_CUDA;
  }
  Params p;
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.bias = static_cast<const uint16_t*>(bias);
  p.residual = static_cast<const uint16_t*>(residual);
  p.d = d;
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldd = ldd;
  p.sf_atoms = sf_atoms;
  p.num_m_tiles = (int)ceil_div(m, TILE_M);
  p.num_n_tiles = (int)ceil_div(n, TILE_N);
  p.num_k_tiles = (int)ceil_div(k, BK);
  p.d_f32 = d_dtype == NVFP4B200_F32;
  p.accumulate = accumulate;
  p.epilogue = epilogue;
  p.swiglu = sw ? 1 : 0;
  p.store_gu = (sw && sw->gu) ? 1 : 0;
  p.h_amax = sw ? sw->ws : (dsw ? dsw->ws : nullptr);
  p.dswiglu = dsw ? 1 : 0;
  p.mx = mx;
  p.stages = dsw ? DSW_STAGES : STAGES;
  p.out_bytes = dsw ? DSW_OUT_BYTES : OUT_BYTES;
  const int smem_bytes = dsw ? DSW_SMEM_BYTES : SMEM_BYTES;
  const int64_t tiles = (int64_t)p.num_m_tiles * p.num_n_tiles;
  const DeviceInfo info = device_info();
  int cap = info.max_clusters;
  const int max_sms = g_gemm_max_sms.load(std::memory_order_relaxed);
  if (max_sms > 0) cap = std::max(1, std::min(cap, max_sms / 2));
  const int clusters = (int)std::min<int64_t>(tiles, cap);
  {
    static std::atomic<uint32_t> seq[64];
    int dev = 0;
    cudaGetDevice(&dev);
    p.sched_slot = (int)(seq[dev & 63].fetch_add(1u, std::memory_order_relaxed) % SCHED_SLOTS);
  }
  if (cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
      cudaSuccess)
    return NVFP4B200_ERR_CUDA;
  nvfp4_gemm_kernel<<<2 * clusters, NUM_THREADS, smem_bytes, stream>>>(ma, mb, msa, msb, md, mh, p);
  uint32_t* ws = sw ? sw->ws : (dsw ? dsw->ws : nullptr);
  if (ws) {
    const int lrc = launch_status();
    if (lrc) return lrc;
    h_scale_finalize_kernel<<<1, 1, 0, stream>>>(ws, sw ? sw->g_out : dsw->g_out);
  }
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
  const int qe = take_quant_device_error();
  if (qe == NVFP4B200_ERR_CUDA) return qe;
  if (*out == 0) *out = qe;
  if (*out != 0) {   // a launch gave up: make sure no tile counter is left dirty (the device is idle here)
    static const uint32_t zeros[gemm::SCHED_SLOTS][2] = {};
    if (cudaMemcpyToSymbol(gemm::g_tile_sched, zeros, sizeof(zeros)) != cudaSuccess) return NVFP4B200_ERR_CUDA;
  }
  return NVFP4B200_OK;
}

int nvfp4b200_wait_selftest(int64_t limit_cycles, void* stream) {
  if (limit_cycles < 1 || limit_cycles > (1ll << 32)) return NVFP4B200_ERR_INVALID_ARG;
  int rc = check_device();
  if (rc) return rc;
  gemm::wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((long long)limit_cycles);
  return launch_status();
}

int nvfp4b200_set_gemm_max_sms(int max_sms) {
  if (max_sms < 0) return NVFP4B200_ERR_INVALID_ARG;
  gemm::g_gemm_max_sms.store(max_sms, std::memory_order_relaxed);
  return NVFP4B200_OK;
}

int nvfp4b200_gemm(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
                   const float* scale_b, const void* bias, const void* residual, void* d, int d_dtype,
                   int accumulate, int epilogue, int64_t m, int64_t n, int64_t k, int64_t ldd, void* stream) {
  return gemm::run(a, b, sfa, sfb, scale_a, scale_b, bias, residual, d, d_dtype, accumulate, epilogue, m, n, k, ldd,
                   (cudaStream_t)stream);
}

int nvfp4b200_gemm_swiglu(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
                          const float* scale_b, void* h, void* gu, uint32_t* ws, float* h_global_scale_out, int64_t m,
                          int64_t n, int64_t k, void* stream) {
  if (!h || (ws == nullptr) != (h_global_scale_out == nullptr)) return NVFP4B200_ERR_INVALID_ARG;
  if (n <= 0 || n % gemm::TILE_N) return NVFP4B200_ERR_BAD_SHAPE;   // whole gate|up tiles
  if ((gu && !aligned(gu, 16)) || (ws && !aligned(ws, 4))) return NVFP4B200_ERR_MISALIGNED;
  gemm::SwigluOut sw{gu, ws, h_global_scale_out};
  return gemm::run(a, b, sfa, sfb, scale_a, scale_b, nullptr, nullptr, h, NVFP4B200_BF16, 0, NVFP4B200_EPI_NONE, m, n,
                   k, n, (cudaStream_t)stream, &sw);
}

int nvfp4b200_gemm_dswiglu(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
                           const float* scale_b, const void* gu, void* dgu, uint32_t* ws, float* dgu_global_scale_out,
                           int64_t m, int64_t n, int64_t k, void* stream) {
  if (!gu || !dgu || (ws == nullptr) != (dgu_global_scale_out == nullptr)) return NVFP4B200_ERR_INVALID_ARG;
  if (n <= 0 || n % gemm::TILE_N) return NVFP4B200_ERR_BAD_SHAPE;   // whole 256-column dh tiles
  if (!aligned(gu, 16) || (ws && !aligned(ws, 4))) return NVFP4B200_ERR_MISALIGNED;
  gemm::DswigluIn dsw{gu, ws, dgu_global_scale_out};
  return gemm::run(a, b, sfa, sfb, scale_a, scale_b, nullptr, nullptr, dgu, NVFP4B200_BF16, 0, NVFP4B200_EPI_NONE, m,
                   n, k, n, (cudaStream_t)stream, nullptr, &dsw);
}

int nvfp4b200_nvfp4_mm(const void* a, const void* b, const void* sfa, const void* sfb, const float* output_scale,
                       const void* bias, void* d, int64_t m, int64_t n, int64_t k, void* stream) {
  return gemm::run(a, b, sfa, sfb, output_scale, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_NONE, m,
                   n, k, n, (cudaStream_t)stream);
}

int nvfp4b200_mxfp4_mm(const void* a, const void* b, const void* sfa, const void* sfb, const void* bias, void* d,
                       int64_t m, int64_t n, int64_t k, void* stream) {
  return gemm::run(a, b, sfa, sfb, nullptr, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_NONE, m, n, k,
                   n, (cudaStream_t)stream, nullptr, nullptr, /*mx=*/1);
}

int nvfp4b200_nvfp4_mm_relu(const void* a, const void* b, const void* sfa, const void* sfb, const float* output_scale,
                            const void* bias, void* d, int64_t m, int64_t n, int64_t k, void* stream) {
  return gemm::run(a, b, sfa, sfb, output_scale, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_RELU, m,
                   n, k, n, (cudaStream_t)stream);
}

int nvfp4b200_nvfp4_mm_relu_2(const void* a, const void* b, const void* sfa, const void* sfb,
                              const float* output_scale, const void* bias, void* d, int64_t m, int64_t n, int64_t k,
                              void* stream) {
  return gemm::run(a, b, sfa, sfb, output_scale, nullptr, bias, nullptr, d, NVFP4B200_BF16, 0, NVFP4B200_EPI_RELU2,
                   m, n, k, n, (cudaStream_t)stream);
}

}  // extern "C"
