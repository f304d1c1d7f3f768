// tcgen05.cuh — device helpers shared by the tensor-core kernels (gemm_tc.cu, gemm_tc_grouped.cu): TMA tile loads,
// UMMA shared-memory and instruction descriptors for kind::i8, MMA issue/commit, tensor-memory loads; and the host's
// cached 2-D tensor-map encoder. No load here uses cluster multicast.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace b200 {

__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * map, int c0, int c1, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor of one K = 32 slice of a K-major tile whose rows are 128 bytes (four K blocks),
// written by TMA with 128-byte swizzle into a 1024-byte-aligned tile: start address (tile + 32 * block) >> 4, leading
// byte offset 16 B (unused by swizzled K-major layouts), stride byte offset 1024 B (eight 128-byte rows), descriptor
// version 1, layout SWIZZLE_128B (2). The swizzle is a function of the address bits, so stepping the start address
// by 32 bytes inside the atom selects the next K block.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void * tile, int block) {
    const uint64_t a = (uint64_t) ((smem_addr(tile) + 32 * block) & 0x3FFFF) >> 4;
    return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::i8: D s32, A s8, B s8, both K-major, M = 128, N = n (a multiple of 16
// in [16, 256]; a run-time value is allowed, the descriptor is a register operand).
__device__ __forceinline__ uint32_t idesc_i8_n(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (n >> 3) << 17) | ((uint32_t) (128 >> 4) << 24);
}
template <int NT>
__device__ __forceinline__ uint32_t idesc_i8() { return idesc_i8_n(NT); }

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}

// The same MMA adding into the accumulator when `accumulate` is non-zero (D = A B + D), else overwriting it.
__device__ __forceinline__ void mma_i8_acc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit values from tensor memory (this warp's lane quarter), one column per register.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int * r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,"
        "%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
          "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
          "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int * r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
          "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Fetches a tensor map's descriptor ahead of its first use (a __grid_constant__ kernel parameter).
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap * m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// Asks L2 to fetch a 2-D tile ahead of its TMA load (no shared-memory destination, no multicast).
__device__ __forceinline__ void prefetch_l2_2d(const CUtensorMap * map, int c0, int c1) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(c0), "r"(c1) : "memory");
}

// Host: a 2-D tensor map (inner extent, outer extent, row pitch in bytes, box), cached by its arguments. False when
// the driver entry point is missing or refuses the map (base not 16-byte aligned, pitch not a multiple of 16, ...).
bool make_map_2d(CUtensorMap * m, CUtensorMapDataType dt, const void * base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);
bool tensor_maps_available();

}  // namespace b200
