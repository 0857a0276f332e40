// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits,
// TMA / bulk copies, tcgen05 (TMEM alloc, MMA, commit, ld) and small bit tricks.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "../../include/rolaq_b200.h"

namespace rolaq {

// Upper bound on polls of one mbarrier phase.  mbarrier.try_wait itself suspends
// for a hardware-defined time slice per poll, so this bounds a wait to well under
// a few seconds while never firing on a healthy pipeline.
constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ void report(int32_t* err, int32_t bits) {
  if (err != nullptr) atomicOr(err, bits);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wall-clock bound of one wait: far above any healthy pipeline stall.
constexpr uint64_t kWaitNs = 2000000000ull;

// Bounded wait.  Returns false (and reports ROLAQ_DEV_TIMEOUT) when the phase did
// not complete within kWaitNs of wall-clock time or kWaitPolls polls, whichever
// comes first; callers then skip their remaining work and leave the kernel.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < kWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && global_ns() - t0 > kWaitNs) break;
  }
  report(err, ROLAQ_DEV_TIMEOUT);
  return false;
}

// ---- TMA and bulk copies (global -> shared, completion on an mbarrier) -----------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 ---------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (BF16 inputs, FP32 accumulator).
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 8 columns -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// 32 registers per thread -> 32 lanes x 32 columns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f8f6f4 (A must be K-major in TMEM).
__device__ __forceinline__ void umma_f8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f8f6f4.
__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor: kind::f8f6f4 with E4M3 A and B, FP32 accumulator.
// a_mn / b_mn select the MN-major (transposed) smem layout for A / B.
__host__ __device__ constexpr uint32_t idesc_e4m3(uint32_t m, uint32_t n, uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Shared-memory descriptor of an MN-major operand in the canonical swizzled layout:
// rows are K (one row = `row_bytes` of MN elements), 8 rows per swizzle atom.
//   SW128: 128-byte rows, 1024-byte atoms (layout type 2)
//   SW32 :  32-byte rows,  256-byte atoms (layout type 6)
__device__ __forceinline__ uint64_t mn_major_desc(uint32_t smem_addr, uint32_t row_bytes) {
  const uint32_t atom = row_bytes * 8;
  const uint64_t layout = row_bytes == 128 ? 2u : 6u;
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                 // leading byte offset (one MN atom: unused)
  d |= static_cast<uint64_t>((atom >> 4) & 0x3FFFu) << 32;  // stride byte offset: next 8 K-rows
  d |= static_cast<uint64_t>(1u) << 46;
  d |= layout << 61;
  return d;
}

// 8 registers per thread -> 32 lanes x 8 columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// 16 registers per thread -> 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 lanes x 16 columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 2 columns -> 2 registers per thread.
__device__ __forceinline__ void tmem_ld2(uint32_t taddr, uint32_t (&r)[2]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
}

// 4 registers per thread -> 32 lanes x 4 columns.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// Shared-memory descriptor for a K-major operand in the canonical 64-byte swizzled layout
// (CU_TENSOR_MAP_SWIZZLE_64B): rows of 32 BF16 (64 B), 8-row atoms of 512 B, start address
// advanced by 32 B per K = 16 step inside the row.  Tile base 512-byte aligned.
__device__ __forceinline__ uint64_t sw64_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                     // leading byte offset (unused here)
  d |= static_cast<uint64_t>(512u >> 4) << 32;              // stride byte offset: 8-row atom
  d |= static_cast<uint64_t>(1u) << 46;                     // descriptor version (sm_100)
  d |= static_cast<uint64_t>(4u) << 61;                     // SWIZZLE_64B
  return d;
}

// 32 lanes x 4 columns -> 4 registers per thread.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// N consecutive TMEM columns (32 lanes) -> r[0..N), as x16 / x8 / x4 / x2 / x1 loads of at most
// ALIGN columns each (ALIGN: a power of two dividing the start column), so that every load
// starts at a multiple of its own width.
template <int N, int ALIGN, int OFF = 0>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
  constexpr int REM = N - OFF;
  if constexpr (REM >= 16 && ALIGN >= 16) {
    uint32_t t[16];
    tmem_ld16(taddr + OFF, t);
#pragma unroll
    for (int i = 0; i < 16; ++i) r[OFF + i] = t[i];
    tmem_ld_cols<N, ALIGN, OFF + 16>(taddr, r);
  } else if constexpr (REM >= 8 && ALIGN >= 8) {
    uint32_t t[8];
    tmem_ld8(taddr + OFF, t);
#pragma unroll
    for (int i = 0; i < 8; ++i) r[OFF + i] = t[i];
    tmem_ld_cols<N, ALIGN, OFF + 8>(taddr, r);
  } else if constexpr (REM >= 4 && ALIGN >= 4) {
    uint32_t t[4];
    tmem_ld4(taddr + OFF, t);
#pragma unroll
    for (int i = 0; i < 4; ++i) r[OFF + i] = t[i];
    tmem_ld_cols<N, ALIGN, OFF + 4>(taddr, r);
  } else if constexpr (REM >= 2 && ALIGN >= 2) {
    uint32_t t[2];
    tmem_ld2(taddr + OFF, t);
    r[OFF] = t[0];
    r[OFF + 1] = t[1];
    tmem_ld_cols<N, ALIGN, OFF + 2>(taddr, r);
  } else if constexpr (REM >= 1) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[OFF]) : "r"(taddr + OFF));
    tmem_ld_cols<N, ALIGN, OFF + 1>(taddr, r);
  }
}

// r[0..N) -> N consecutive TMEM columns (32 lanes), as x16 / x8 / x4 stores of at most ALIGN
// columns each (N and ALIGN multiples of 4).
template <int N, int ALIGN, int OFF = 0>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t* r) {
  constexpr int REM = N - OFF;
  static_assert(N % 4 == 0 && ALIGN % 4 == 0, "whole x4 groups");
  if constexpr (REM >= 16 && ALIGN >= 16) {
    uint32_t t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = r[OFF + i];
    tmem_st16(taddr + OFF, t);
    tmem_st_cols<N, ALIGN, OFF + 16>(taddr, r);
  } else if constexpr (REM >= 8 && ALIGN >= 8) {
    uint32_t t[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) t[i] = r[OFF + i];
    tmem_st8(taddr + OFF, t);
    tmem_st_cols<N, ALIGN, OFF + 8>(taddr, r);
  } else if constexpr (REM >= 4) {
    uint32_t t[4] = {r[OFF], r[OFF + 1], r[OFF + 2], r[OFF + 3]};
    tmem_st4(taddr + OFF, t);
    tmem_st_cols<N, ALIGN, OFF + 4>(taddr, r);
  }
}

// The largest power of two (<= 16) dividing n: the column alignment of starts n * k.
__host__ __device__ constexpr int pow2_align(int n) {
  return (n % 16 == 0) ? 16 : (n % 8 == 0) ? 8 : (n % 4 == 0) ? 4 : (n % 2 == 0) ? 2 : 1;
}

// Ties registers written by tcgen05.ld to the preceding tcgen05.wait::ld, so that no
// consumer is scheduled above the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Bulk prefetch of [p, p + bytes) into L2 (p and bytes 16-byte aligned).
// Pull the line holding `p` into L2 (no registers, nothing waits on it).
__device__ __forceinline__ void prefetch_line_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 2^x for x <= 0 (MUFU; -inf -> 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// FP16x2 -> two E4M3 bytes (round to nearest, saturating): .x -> low byte.
__device__ __forceinline__ uint32_t half2_to_e4m3x2(__half2 h) {
  return static_cast<uint32_t>(
      __nv_cvt_halfraw2_to_fp8x2(static_cast<__half2_raw>(h), __NV_SATFINITE, __NV_E4M3));
}

// Programmatic dependent launch: a kernel launched with the programmatic stream
// serialization attribute may start once every CTA of the kernel before it in the stream
// has executed launch_dependents (or exited); griddepcontrol.wait then blocks until that
// grid has completed and its memory operations are visible.  Without such a launch the
// wait returns at once.
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Maximum of v over the 32 lanes of a full warp (one instruction on sm_100a).
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Two floats -> two E4M3 bytes (round to nearest, saturating): .x -> low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}
// Two E4M3 bytes -> FP16x2 (exact): low byte -> low half.
__device__ __forceinline__ __half2 e4m3x2_to_half2(uint32_t v) {
  const __half2_raw r = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v & 0xFFFFu), __NV_E4M3);
  return *reinterpret_cast<const __half2*>(&r);
}

// Shared-memory matrix descriptor for a K-major operand in the canonical 128-byte
// swizzled layout written by TMA with CU_TENSOR_MAP_SWIZZLE_128B: rows of 64 BF16
// (128 B), 8-row atoms of 1024 B.  The tile base must be 1024-byte aligned; the
// start address may then be advanced by 32 B per K = 16 step inside the atom.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                     // leading byte offset (unused here)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;             // stride byte offset: 8-row atom
  d |= static_cast<uint64_t>(1u) << 46;                     // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                     // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, BF16 A and B (both K-major), FP32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t m, uint32_t n) {
  return (1u << 4)            // D format: F32
         | (1u << 7)          // A format: BF16
         | (1u << 10)         // B format: BF16
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// ---- warp-level tensor-core MMA (m16n8k16, BF16 in, FP32 accumulate) ------------

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  return (a & mask) | orv;  // one LOP3
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

__device__ __forceinline__ int64_t load_index(const void* p, int is64, int64_t i) {
  return is64 ? static_cast<const int64_t*>(p)[i] : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// The codec's FP32 group reductions, in the one order the test oracle restates:
// eight running sums acc[c % 8] over columns in increasing order, then the tree
// ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)).  Every add is a separate round-to-nearest.
struct GroupSum {
  float a[8];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = 0.f;
  }
  __device__ __forceinline__ void add(int k, float v) { a[k] = __fadd_rn(a[k], v); }
  __device__ __forceinline__ float total() const {
    return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                     __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
  }
};

// Lloyd code of one normalised value: [n >= -t] + [n >= 0] + [n >= t] with
// n = diff / std rounded to nearest (IEEE division, as the reference computes it).
__device__ __forceinline__ uint32_t lloyd_code(float diff, float std_, float t) {
  const float n = __fdiv_rn(diff, std_);
  return static_cast<uint32_t>(n >= -t) + static_cast<uint32_t>(n >= 0.f) + static_cast<uint32_t>(n >= t);
}

// OSCAR's uniform min/max INT2 step of one group (mla_quant/oscar.py:91-101): the FP32
// range divided by 3, or 1 for a (near-)constant group (torch compares |max - min| with
// the scalar 1e-8 rounded to FP32).
__device__ __forceinline__ float uniform_scale(float mn, float mx) {
  const float r = __fsub_rn(mx, mn);
  return fabsf(r) > 1e-8f ? __fdiv_rn(r, 3.0f) : 1.0f;
}
// code = clamp(round((x - min) / scale), 0, 3) with torch.round's ties-to-even (rintf).
__device__ __forceinline__ uint32_t uniform_code(float x, float mn, float scale) {
  const float q = rintf(__fdiv_rn(__fsub_rn(x, mn), scale));
  return static_cast<uint32_t>(fminf(fmaxf(q, 0.f), 3.f));
}
// The stored zero point of the uniform codec, so that (code - zero) * scale ~ code * scale + min.
__device__ __forceinline__ float uniform_zero(float mn, float scale) { return __fdiv_rn(-mn, scale); }

// Neighbouring FP32 values (towards -inf / +inf), zeros included.
__device__ __forceinline__ float f32_prev(float d) {
  const int b = __float_as_int(d);
  if ((b & 0x7FFFFFFF) == 0) return __int_as_float(0x80000001);
  return __int_as_float(d > 0.f ? b - 1 : b + 1);
}
__device__ __forceinline__ float f32_next(float d) {
  const int b = __float_as_int(d);
  if ((b & 0x7FFFFFFF) == 0) return __int_as_float(0x00000001);
  return __int_as_float(d > 0.f ? b + 1 : b - 1);
}

// The smallest FP32 d with RN(d / std_) >= c (IEEE quotient, round to nearest even), for
// a normal c and 0 < std_ < 2^24.  RN(d / std_) does not decrease as d grows, so
// [RN(diff / std_) >= c] == [diff >= bound] for every diff: the Lloyd code
// [n >= -t] + [n >= 0] + [n >= t] becomes compares with the reference's IEEE-quotient
// semantics.  RN(q) >= c exactly when q is above the midpoint m between c and the float
// below it, or equal to it when c's last mantissa bit is even (the tie rounds to c).  m has
// 25 significant bits, so m * std_ (<= 49 bits) is exact in FP64, and the bound is the
// first float at or above it (one past it at an odd-c tie).
__device__ __forceinline__ float quotient_bound(float c, float std_) {
  const double m = (static_cast<double>(f32_prev(c)) + static_cast<double>(c)) * 0.5;
  const double t = m * static_cast<double>(std_);
  float b = __double2float_ru(t);
  if (static_cast<double>(b) == t && (__float_as_uint(c) & 1u)) b = f32_next(b);
  return b;
}

// The smallest FP32 d with RN(d / std_) >= 0, for 0 < std_ < 2^24: d / std_ rounds to -0
// exactly when |d| = k * 2^-149 with k <= std_ / 2 (ties to even give 0), so the bound is
// -floor(std_ / 2) * 2^-149, a denormal (or -0 when std_ < 2).
__device__ __forceinline__ float quotient_bound_zero(float std_) {
  const uint32_t k = static_cast<uint32_t>(floorf(__fmul_rn(std_, 0.5f)));
  return __int_as_float(static_cast<int>(0x80000000u | k));
}

}  // namespace rolaq
