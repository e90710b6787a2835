// Shared device helpers for the sm_100a kernels of libh3b200: status word, bounded mbarrier waits, TMA / bulk copies,
// tcgen05 (TMEM alloc, MMA, commit, ld/st, smem->TMEM copy), UMMA descriptors and the numeric conversions the NVFP4 /
// FP8 paths use.  Everything here is written against the PTX ISA (8.7+) for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace h3 {

// ------------------------------------------------------------------------------------------------ status
// Sticky device status word (0 = ok).  A bounded wait that gives up records where it gave up here; the host reads it
// with h3_device_status().  Codes: 1xx GEMM, 2xx attention; the low digits name the wait.  The library is one
// translation unit (h3b200.cu includes every kernel file), so this is its only definition.
__device__ int g_status;

__device__ __forceinline__ void set_status(int code) { atomicCAS(&g_status, 0, code); }
__device__ __forceinline__ bool status_bad() { return *(volatile int*)&g_status != 0; }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------------ smem / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Issue helpers marked "warp-wide" below are called by all 32 lanes of a converged warp with the same arguments;
// elect.sync inside the instruction sequence picks the one lane that issues.  The operands then stay in warp-uniform
// registers: issuing the same instructions from a lane-0 branch instead costs tens of cycles each (a tcgen05.mma
// from a lane-0 branch takes ~60 cycles to issue, from the whole warp ~7), which starves the tensor pipe.
#define H3_ELECT "elect.sync rx|e, 0xffffffff;\n\t"
// warp-wide: one arrival that also expects `bytes` of transaction data
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
               "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but a thread whose phase is not complete is suspended until it completes or `ns` nanoseconds
// pass.  A suspended warp issues nothing: polling warps would otherwise fill the SM sub-partition's memory-I/O queue,
// which the working warps' TMEM, MUFU and tcgen05.mma instructions also go through.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Wait until the barrier's phase with the given parity completes.  Gives up after ~2 s of wall time (or at once when
// another wait of the grid already gave up), records `code` and returns false: every caller then leaves its loop, so
// a lost arrival ends the kernel with an error status instead of a hang.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kSuspendNs = 1000000u;   // longest single suspension; the limit is checked after each
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
    if (status_bad() || globaltimer() - t0 > kWaitLimitNs) {
      set_status(code);
      return false;
    }
  }
}

// ------------------------------------------------------------------------------------------------ TMA / bulk copies
// warp-wide: one 2-D tile of a tensor map into shared memory, completing on `bar`
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
      "@e cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n\t}" ::"r"(smem_u32(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// warp-wide: contiguous global -> shared copy; both addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
               "@e cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n\t}"
               ::"r"(smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
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

// warp-wide: MMA completion -> one arrival on an mbarrier (tracks every tcgen05 op the issuing thread issued before
// it; the elected lane is the same lane each time, as every lane of the warp is active)
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
               "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
               ::"r"(smem_u32(bar))
               : "memory");
}

// warp-wide: D[tmem] (+)= A[smem] x B[smem]^T with NVFP4 operands and UE4M3 scales per 16 elements read from TMEM
__device__ __forceinline__ void mma_nvfp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t" H3_ELECT
      "@e tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// warp-wide: D[tmem] (+)= A[smem] x B[smem]^T, e4m3 x e4m3 -> fp32
__device__ __forceinline__ void mma_fp8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t" H3_ELECT
      "@e tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// warp-wide: D[tmem] (+)= A[tmem] x B[smem]^T, e4m3 x e4m3 -> fp32 (A read from TMEM, K-major: lane = row)
__device__ __forceinline__ void mma_fp8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t" H3_ELECT
      "@e tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// warp-wide: 32 lanes x 128 bits from shared memory, replicated to the four 32-lane quadrants of TMEM (scale factors)
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
               "@e tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------ CTA pairs (cta_group::2)
// A cluster of two CTAs on two SMs sharing one MMA: rank 0 (the leader) issues every tcgen05.mma / tcgen05.cp of the
// pair; each CTA holds its half of the A rows and of the B rows in its own shared memory and its half of the
// accumulator rows in its own TMEM (the same columns in both).  No load here multicasts: each CTA loads its own data.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of both CTAs: orders prior shared-memory writes (barrier inits) before the peer's accesses
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of this CTA's shared variable at `p` as seen in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// one arrival on an mbarrier of another CTA of the cluster (cluster address from cluster_addr)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// warp-wide: a 2-D tile into this CTA's shared memory whose completed bytes count on the leader's barrier
// (bar_cluster: the leader's mbarrier as a cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
      "@e cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];\n\t}" ::"r"(smem_u32(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// TMEM allocation of the pair (one warp in each CTA executes it; the same columns in both CTAs)
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// warp-wide (leader): completion of the pair's MMAs -> one arrival on the barrier at this shared offset in each CTA of
// `mask` (bit r: CTA rank r)
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
               "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               "\n\t}" ::"r"(smem_u32(bar)), "h"(mask)
               : "memory");
}
// warp-wide (leader): D (+)= A x B^T over the pair: M = 256 (rows 0-127 from the leader's A tile, 128-255 from the
// peer's at the same offset), N split the same way over the two B tiles; NVFP4 with UE4M3 scales from TMEM
__device__ __forceinline__ void mma_nvfp4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t" H3_ELECT
      "@e tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// warp-wide (leader): tcgen05.cp 32x128b.warpx4 in both CTAs of the pair, each from its own shared memory
__device__ __forceinline__ void tmem_cp_pair_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t" H3_ELECT
               "@e tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// ------------------------------------------------------------------------------------------------ UMMA descriptors
// Shared-memory matrix descriptor (sm_100 format): start address >> 4 in bits 0-13, leading byte offset >> 4 in
// 16-29, stride byte offset >> 4 in 32-45, version 1 in 46-47, base offset 0, layout type in 61-63.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 7) << 61;
  return d;
}
// K-major operand tile, 128-byte rows, 128-byte swizzle (as TMA writes with CU_TENSOR_MAP_SWIZZLE_128B): 8-row groups
// 1024 bytes apart.  The tile base must be 1024-byte aligned; a K step inside the 128-byte row adds its byte offset
// to the start address.
constexpr uint32_t kLayoutSW128 = 2;
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t saddr) { return make_sdesc(saddr, 16, 1024, kLayoutSW128); }
// Scale-factor atom for tcgen05.cp 32x128b: 32 rows of 16 bytes, contiguous (8-row core matrices 128 bytes apart).
__device__ __forceinline__ uint64_t sdesc_sf_atom(uint32_t saddr) { return make_sdesc(saddr, 0, 128, 0); }

// Instruction descriptors.  Block-scaled NVFP4 (kind::mxf4nvf4): A/B format E2M1 = 1 in bits 7-9 / 10-12, scale
// format UE4M3 = 0 in bit 23, N >> 3 in bits 17-22, M >> 4 in bits 24-28, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_nvfp4(int M, int N) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// kind::f8f6f4 with e4m3 x e4m3 and an fp32 accumulator (C format F32 = 1 in bits 4-5).
__host__ __device__ constexpr uint32_t idesc_fp8(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------------------ numerics
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);   // .x = lo (low 16 bits), .y = hi
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// fp32 pair -> two e4m3 bytes (round to nearest even, saturating): `lo` in bits 0-7, `hi` in bits 8-15.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t e4m3(float x) { return e4m3x2(x, 0.f) & 0xFF; }
// e4m3 byte -> fp32 (exact; NaN byte 0x7F is never produced by the saturating conversions here).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t e = (b >> 3) & 15, m = b & 7;
  float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20)) : (float)m * 0.001953125f;
  return (b & 0x80) ? -v : v;
}
// Eight fp32 values -> eight e2m1 codes in one word (round to nearest even, saturating at 6), element i in bits
// 4i..4i+3 (two a byte, even element in the low nibble).  Adding +0.0 first maps -0.0 to +0.0, so each code equals
// the threshold form sign(v < 0) | |v|-bucket of the reference quantiser.
__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
  float a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = __fadd_rn(v[i], 0.0f);
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(a[0]), "f"(a[1]), "f"(a[2]), "f"(a[3]), "f"(a[4]), "f"(a[5]), "f"(a[6]), "f"(a[7]));
  return r;
}

// Quantise 16 consecutive values (already bf16-rounded, fp32) of one NVFP4 group under the global reciprocal
// inv_g: returns the group's e4m3 scale byte and writes 8 code bytes (2 a byte, even element low) into `codes`.
// 1 / max(e4m3(b), 1e-30) for a scale byte b in [0, 126], without a division.  A normal e4m3 value is
// 2^(e - 7) (1 + m / 8), so its reciprocal is 2^(7 - e) * 8 / (8 + m): the correctly rounded fp32 of 8 / (8 + m),
// scaled by an exact power of two.  A subnormal one is m / 512, reciprocal 512 / m, and byte 0 gives 1 / 1e-30.  The
// sixteen constants are the correctly rounded quotients, so the result equals the IEEE division bit for bit
// (checked on the GPU against __fdiv_rn for every byte).
__device__ __forceinline__ float sel8(uint32_t m, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t c4,
                                      uint32_t c5, uint32_t c6, uint32_t c7) {
  const uint32_t a = (m & 1) ? c1 : c0, b = (m & 1) ? c3 : c2, d = (m & 1) ? c5 : c4, f = (m & 1) ? c7 : c6;
  const uint32_t lo = (m & 2) ? b : a, hi = (m & 2) ? f : d;
  return __uint_as_float((m & 4) ? hi : lo);
}
__device__ __forceinline__ float e4m3_rcp(uint32_t b) {
  const uint32_t e = b >> 3, m = b & 7;
  const float nrm = __fmul_rn(sel8(m, 0x3f800000u, 0x3f638e39u, 0x3f4ccccdu, 0x3f3a2e8cu, 0x3f2aaaabu, 0x3f1d89d9u,
                                   0x3f124925u, 0x3f088889u),
                              __uint_as_float((134u - e) << 23));
  const float sub = sel8(m, 0x7149f2cau, 0x44000000u, 0x43800000u, 0x432aaaabu, 0x43000000u, 0x42cccccdu, 0x42aaaaabu,
                         0x42924925u);
  return e ? nrm : sub;
}
// x / 6 rounded to nearest even for x >= 0, without a division: q0 = x * RN(1/6), the exact remainder
// r = x - 6 q0 by one fma, then q0 + r * RN(1/6) (Markstein's correction step for division by a known constant,
// P. Markstein, "IA-64 and Elementary Functions", 2000).  Checked on the GPU against __fdiv_rn(x, 6) over every
// non-negative finite fp32.
__device__ __forceinline__ float div6_rn(float x) {
  constexpr float c6 = 0.16666667163372039794921875f;   // RN(1/6) = 0x3e2aaaab
  const float q0 = __fmul_rn(x, c6);
  return __fmaf_rn(__fmaf_rn(-6.0f, q0, x), c6, q0);
}

__device__ __forceinline__ uint32_t quant_group16(const float (&v)[16], float inv_g, uint32_t (&codes)[2]) {
  float xs[16];
  float gmax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    xs[i] = __fmul_rn(v[i], inv_g);
    gmax = fmaxf(gmax, fabsf(xs[i]));
  }
  uint32_t sf = e4m3(div6_rn(gmax));
  float inv = e4m3_rcp(sf);
#pragma unroll
  for (int i = 0; i < 16; ++i) xs[i] = __fmul_rn(xs[i], inv);
  codes[0] = e2m1x8(xs);
  codes[1] = e2m1x8(xs + 8);
  return sf;
}


// Byte offset of scale (row r, group k16) in the tiled scale layout the GEMM reads (128-row x 4-group atoms of 512
// bytes, [row block][group block] order; inside an atom (r % 32) * 16 + (r / 32 % 4) * 4 + k16 % 4).
__host__ __device__ __forceinline__ size_t sf_tiled_offset(size_t r, size_t k16, size_t kgroups) {
  return ((r >> 7) * (kgroups >> 2) + (k16 >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (k16 & 3);
}

// atomicMax on a non-negative float stored in a 32-bit word (int ordering equals float ordering for >= 0).  The
// word only grows, so a value that does not exceed what is already there is dropped after a plain read: tens of
// thousands of warps updating one scale slot would otherwise serialise on that address.
__device__ __forceinline__ void atomic_max_pos(float* addr, float v) {
  if (v > *reinterpret_cast<volatile float*>(addr)) atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace h3
