// common.cuh — shared device code of the B200 quantized-product backend (sm_100a only).
//
// Weight layout in HBM ("repacked", set once at upload). A GGUF tensor of `type` with ne0 = K values per row and
// R = ne1 * ne2 rows is stored as a structure of arrays, one array per block field, each row-contiguous and each
// array starting on a 256-byte boundary:
//   Q8_0 : qs  int8  [R][K]          | d    fp16 [R][K/32]
//   Q4_K : qs  u8    [R][K/2]        | meta u8   [R][K/256][16]   (d, dmin, 12 scale bytes: the block's first 16 B)
//   Q5_K : qs  u8    [R][K/2]        | meta u8   [R][K/256][16]  | qh u8 [R][K/8]
//   Q6_K : ql  u8    [R][K/2]        | qh   u8   [R][K/4]        | sc int8 [R][K/256][16] | d fp16 [R][K/256]
//   BF16 : w   bf16  [R][K]
// The map from a GGUF byte offset to its place is a bijection (layout.cu), so set_tensor / get_tensor of any byte
// range work as they do on a plain buffer, and the bytes read per weight equal the GGUF bytes (34 B / 32 for Q8_0,
// 144 B / 256 for Q4_K, 210 B / 256 for Q6_K, 2 B for BF16). Every row's quant bytes start 16-byte aligned, so the
// kernels stream them with 128-bit loads.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define B200_TYPE_F32 0
#define B200_TYPE_F16 1
#define B200_TYPE_Q8_0 8
#define B200_TYPE_Q4_K 12
#define B200_TYPE_Q5_K 13
#define B200_TYPE_Q6_K 14
#define B200_TYPE_Q8_K 15
#define B200_TYPE_BF16 30

namespace b200 {

constexpr int kWarp = 32;

// ------------------------------------------------------------------------------------------------------------------
// Field arrays of a repacked weight (pointers into one device allocation).
// ------------------------------------------------------------------------------------------------------------------
struct WeightView {
    int type;
    int64_t K;      // values per row
    int64_t rows;   // rows of all matrices (ne1 * ne2)
    const uint8_t * f0;  // Q8_0 qs | Q4_K qs | Q6_K ql | BF16 w
    const uint8_t * f1;  // Q8_0 d  | Q4_K meta | Q6_K qh
    const uint8_t * f2;  // Q6_K sc   | Q5_K qh
    const uint8_t * f3;  // Q6_K d
};

// Byte sizes of the fields of `rows` rows of K values, in order; returns the number of fields.
__host__ __device__ inline int field_sizes(int type, int64_t K, int64_t rows, int64_t * sz) {
    switch (type) {
    case B200_TYPE_Q8_0: sz[0] = rows * K; sz[1] = rows * (K / 32) * 2; return 2;
    case B200_TYPE_Q4_K: sz[0] = rows * (K / 2); sz[1] = rows * (K / 256) * 16; return 2;
    case B200_TYPE_Q5_K: sz[0] = rows * (K / 2); sz[1] = rows * (K / 256) * 16; sz[2] = rows * (K / 8); return 3;
    case B200_TYPE_Q6_K:
        sz[0] = rows * (K / 2); sz[1] = rows * (K / 4); sz[2] = rows * (K / 256) * 16; sz[3] = rows * (K / 256) * 2;
        return 4;
    case B200_TYPE_BF16: sz[0] = rows * K * 2; return 1;
    case B200_TYPE_F32: sz[0] = rows * K * 4; return 1;
    default: return 0;
    }
}

__host__ __device__ inline int64_t align256(int64_t v) { return (v + 255) & ~(int64_t) 255; }

// ------------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch (PDL). In a kernel launched with the programmatic-serialization attribute,
// `pdl_wait` blocks until the previous kernel in the stream has completed and its writes are visible, and
// `pdl_launch_dependents` lets the next kernel start its CTAs early (its prologue streams weights, which depend on
// nothing). Both are no-ops in an ordinary launch.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ------------------------------------------------------------------------------------------------------------------
// mbarriers and bulk (TMA) copies, global -> shared, no multicast. Waits are bounded: after kSpinLimit polls a wait
// gives up and reports false, so no kernel can hang on a copy that never lands.
// ------------------------------------------------------------------------------------------------------------------
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// `count` arrivals at once (a thread arriving for itself and for threads that skip the phase).
__device__ __forceinline__ void mbar_arrive_n(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Waits for the phase with the given parity to complete; false if it did not within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    for (uint32_t i = 0; i < kSpinLimit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// The same wait with a suspend-time hint: a thread whose phase is not complete sleeps (up to ~0.5 us per poll, woken
// early when the phase completes) instead of re-polling, which leaves issue slots to the warps doing work. Bounded by
// kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t * bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    for (uint32_t i = 0; i < kSpinLimit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(500u)
            : "memory");
        if (done) return true;
    }
    return false;
}

// One bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) from global to this CTA's shared memory,
// completing `bytes` of the barrier's transaction count.
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// 128-bit streaming load of weight bytes: read once, do not keep in L1.
__device__ __forceinline__ int4 ld_stream(const void * p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------------------------------------------------------------
// Activation quantizers, bit-identical to the CPU oracle (oracle/oracle.c) and so to ggml's reference row
// quantizers: IEEE division / reciprocal (no fast-math), round-half-away for q8_0, round-half-even for q8_K.
// ------------------------------------------------------------------------------------------------------------------

// One q8_0 block held one value per lane: returns this lane's int8 and (via *d_out) the fp16-rounded scale as float,
// and (via *d_half) the fp16 bits.
__device__ __forceinline__ int8_t quantize_q8_0_lane(float v, float * d_out, uint16_t * d_half) {
    const float amax = warp_max(fabsf(v));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const __half dh = __float2half_rn(d);
    *d_out = __half2float(dh);
    *d_half = __half_as_ushort(dh);
    return (int8_t) (int) roundf(__fmul_rn(v, id));
}

// q8_0 of one 32-value block held 4 per lane by 8 consecutive lanes (lanes 8k .. 8k + 7, lane 8k + i holding values
// 4i .. 4i + 3): the arithmetic of quantize_q8_0_lane. Returns the 4 int8 packed little-endian; *d_out = the fp16 scale
// as float. All 32 lanes must call it.
__device__ __forceinline__ uint32_t quantize_q8_0_quad(float4 v, float * d_out) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    *d_out = __half2float(__float2half_rn(d));
    const uint32_t q0 = (uint32_t) (int) roundf(__fmul_rn(v.x, id)) & 0xFFu;
    const uint32_t q1 = (uint32_t) (int) roundf(__fmul_rn(v.y, id)) & 0xFFu;
    const uint32_t q2 = (uint32_t) (int) roundf(__fmul_rn(v.z, id)) & 0xFFu;
    const uint32_t q3 = (uint32_t) (int) roundf(__fmul_rn(v.w, id)) & 0xFFu;
    return q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
}

// One q8_K block of 256 values held 8 per lane (lane l holds values 8l .. 8l+7): the largest magnitude (first index on
// ties) sets iscale = -127 / max; q = min(127, round-half-even(iscale * v)); d = 1 / iscale (0 for an all-zero
// block). Returns this lane's 8 int8, the sum of the 16 values of the pair (lane & ~1, lane | 1) (valid in both
// lanes), and d.
__device__ __forceinline__ void quantize_q8_K_warp(const float v[8], int8_t q[8], int16_t * bsum, float * d) {
    const int lane = threadIdx.x & 31;
    float amax = 0.0f, vmax = 0.0f;
    int imax = 1 << 30;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float av = fabsf(v[j]);
        if (av > amax) { amax = av; vmax = v[j]; imax = lane * 8 + j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, o);
        const int oi = __shfl_xor_sync(0xffffffffu, imax, o);
        if (oa > amax || (oa == amax && oi < imax)) { amax = oa; vmax = ov; imax = oi; }
    }
    int s = 0;
    if (amax == 0.0f) {
#pragma unroll
        for (int j = 0; j < 8; j++) q[j] = 0;
        *d = 0.0f;
    } else {
        const float iscale = __fdiv_rn(-127.0f, vmax);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int t = __float2int_rn(__fmul_rn(iscale, v[j]));
            t = t < 127 ? t : 127;
            q[j] = (int8_t) t;
            s += t;
        }
        *d = __fdiv_rn(1.0f, iscale);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    *bsum = (int16_t) s;
}

// SiLU as ggml's CPU defines it, x / (1 + exp(-x)), with the hardware exponential and division (relative error
// ~1e-6). Used where the result is judged within a tolerance (the tensor-core expert path).
__device__ __forceinline__ float silu(float x) { return __fdividef(x, __fadd_rn(1.0f, __expf(-x))); }

// SiLU evaluated in double and rounded once to float32: the order-free definition the CPU oracle uses. Any accurate
// evaluation rounds to the same float32 except in rare near-ties, so the decode step's chain of products, whose
// activation quantization would turn a last-bit difference into a different int8, stays identical to the oracle's.
__device__ __forceinline__ float silu_exact(float x) {
    const double xd = (double) x;
    return __double2float_rn(xd / (1.0 + exp(-xd)));
}

// The float32 step of a product: the exact sum of its (super-)block terms (float32 scale product times the exact int32
// sum, each exact in double), accumulated in double and rounded once at the end; the CPU oracle defines it the same
// way, so the result does not depend on how lanes split the blocks.
__device__ __forceinline__ double acc_term(double acc, float scale, int sumi) { return fma((double) scale, (double) sumi, acc); }

// The mean of K squares summed in double, rounded once to float32: sum / K, where a power-of-two K scales exactly by
// 2^-log2(K) (a multiplication gives the same double as the division, without its latency on the decode step's chain).
__device__ __forceinline__ float mean_rounded(double sum, int64_t K) {
    if ((K & (K - 1)) == 0) {
        const int lg = 63 - __clzll((unsigned long long) K);
        return __double2float_rn(sum * __longlong_as_double((long long) (1023 - lg) << 52));
    }
    return __double2float_rn(sum / (double) K);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Asynchronous 4-byte global -> shared copy (completes at cp_async_wait_all; the issuing thread does not stall).
__device__ __forceinline__ void cp_async4(void * smem_dst, const void * gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

}  // namespace b200
