// Inline-PTX helpers for the 5th-generation tensor cores of sm_100a (tcgen05):
// tensor-memory (TMEM) allocation, shared-memory matrix descriptors, the
// instruction descriptor of kind::f16 MMAs, the MMA itself, its commit to an
// mbarrier, and TMEM <-> register moves.
//
// Conventions used by the kernels here (cta_group::1, one CTA per MMA):
// - A is M x K, B is N x K (K-major: K contiguous) or K x N (MN-major: N
//   contiguous), both in shared memory with the 128-byte swizzle: a row of
//   64 FP16 values is 128 B, its 16-byte chunk c stored at chunk c ^ (row % 8),
//   8 rows forming a 1024-byte atom.  Tiles start on 1024-byte boundaries.
// - D (FP32) lives in TMEM: row i of a 128-row tile in lane i, column j in
//   TMEM column base + j.  A warp reads the 32 lanes 32 * (warp % 4) .. +31.
// - One thread issues the MMAs; tcgen05.commit makes an mbarrier track their
//   completion (it arrives once all previously issued MMAs of the thread are
//   done).
#pragma once

#include <stdint.h>

namespace pkv::tc {

// --- TMEM allocation (warp-wide) -------------------------------------------
// Allocate `ncols` TMEM columns (a power of two >= 32); the base address is
// written to shared memory at `dst_smem`.
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

// --- ordering of tcgen05 operations across thread synchronisation ----------
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// --- descriptors -------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (all in 16-byte units), version 1, layout type.
constexpr uint64_t kSwizzle128B = 2;

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (static_cast<uint64_t>((addr >> 4) & 0x3fffu)) |
           (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3fffu) << 16) |
           (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3fffu) << 32) |
           (1ull << 46) |                 // version 1
           (kSwizzle128B << 61);
}

// K-major operand with the 128-byte swizzle: rows of 64 FP16 (128 B), 8-row
// atoms 1024 B apart.  The k-th 16-element slice of the row starts 32 * k
// bytes further (the swizzle is applied to the final address).
__device__ __forceinline__ uint64_t desc_k_major_sw128(uint32_t addr) { return smem_desc(addr, 16, 1024); }

// MN-major operand with the 128-byte swizzle, at most 64 FP16 wide in MN: K
// rows of 128 B, 8-row atoms 1024 B apart (the stride between MN atoms is
// not used at this width).
__device__ __forceinline__ uint64_t desc_mn_major_sw128(uint32_t addr) { return smem_desc(addr, 8192, 1024); }

// Instruction descriptor of tcgen05.mma kind::f16 with FP16 A and B and an
// FP32 accumulator: M (64/128/256) and N (multiple of 8 or 16, <= 256), each
// operand K-major (false) or MN-major (true).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) |                                   // D format: F32
           (0u << 7) | (0u << 10) |                      // A, B format: F16
           (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// --- MMA and commit (one thread) -----------------------------------------
// D[tmem] (+)= A[smem] . B[smem]^T; `accumulate` false overwrites D.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
    const uint32_t acc = accumulate ? 1u : 0u;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
        : "memory");
}

// The same with A in TMEM (M lanes x K 16-bit values packed two to a 32-bit
// column, K-major) and B in shared memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
    const uint32_t acc = accumulate ? 1u : 0u;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc)
        : "memory");
}

// The mbarrier at `bar` (this CTA's shared memory) receives one arrival once
// every MMA this thread issued before has completed.
__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// --- TMEM <-> registers (warp-wide, 32 lanes x 32 consecutive columns) ----
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column) relative to an allocation's base.
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t column) {
    return base + (lane << 16) + column;
}

}  // namespace pkv::tc
