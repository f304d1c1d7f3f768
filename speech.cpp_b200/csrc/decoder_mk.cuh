// decoder_mk.cuh — the decode step as ONE persistent kernel (one CTA per SM for the whole step).
//
// A decode step is a chain of dependent products (4 per layer + head, 113 for the 28-layer talker), each needing the
// complete output of the one before it. Launching them one by one pays a kernel boundary per product. Here every
// CTA runs the whole chain:
//   - its producer warp streams the CTA's row slice of EVERY product's weights, in order, through one ring of
//     shared-memory slots with bulk async copies (cp.async.bulk, no multicast; mbarrier transaction counts). Weights
//     depend on nothing, so the ring runs ahead of the computation by up to its capacity;
//   - its consumer warps, for product s, load the input vector from L2 into registers, apply the fused prologue
//     (RMSNorm * weight, SwiGLU, grouped-query value broadcast), quantize it to the vec_dot type bit-identically to
//     the CPU oracle, reduce their rows from the ring and write the outputs (+ residual).
// Vectors passed between products are tagged: element k is one 8-byte word {value, tag}, written by a single store,
// with tag = epoch * nstages + s + 1 for the product s that wrote it. A consumer's load of its input both fetches the
// values and proves they are ready (each word carries its own tag), so no completion counter and no second round trip
// to L2 sits between two products. Every product reads its whole input vector, so a CTA can run at most one product
// ahead of the slowest; the buffers are laid out so that no vector is rewritten while a CTA may still read it (the
// host's product list). The epoch is a device word, advanced at the end of every launch, so tags never repeat
// between steps (also under graph replay).
// All CTAs must be co-resident: the kernel is launched cooperatively with one CTA per SM. Every wait is bounded; a
// wait that gives up records B200_DEVERR_TIMEOUT and the CTA leaves the chain, so the others give up in turn.
#pragma once

#include "gemv_tma.cuh"

namespace b200 {

struct MkStage {
    WeightView w;
    int64_t N;
    int pro;
    int pro_k;
    int pro_rep;
    float eps;
    const float * x;       // input vector (written earlier in the chain: read through L2); tagged: {value, tag} words
    const float * norm_w;  // RMSNorm weights
    const float * res;     // residual (same rows as y, written by this CTA) or null; tagged: {value, tag} words
    float * y;             // output; tagged: {value, tag} words
    int x_tagged;
    int res_tagged;
    int y_tagged;
    int glu;          // 1: a gate|up product: its rows are F gate rows then F up rows (N = 2F), a CTA's slice is a range of
                      // F features, and it writes silu(gate) * up for them (F values)
    // precomputed by the host (no divisions on the device's critical path)
    int row_bytes;    // GGUF bytes of one weight row
    int rps;          // rows per ring slot
    int slice_base;   // N / G
    int slice_extra;  // N % G
    int gqa_shift;    // log2(pro_k * pro_rep) for PRO_GQA (-1: not a power of two)
    int hd_shift;     // log2(pro_k) for PRO_GQA (-1: not a power of two)
};


struct MkParams {
    const MkStage * stages;
    int nstages;
    unsigned * epoch;      // steps completed (tags of this launch: epoch * nstages + s + 1)
    unsigned * finished;   // CTAs that finished this launch (zero between launches)
    unsigned * err;
};

constexpr int kMkConsumerWarps = 8;
constexpr int kMkThreads = 32 * (kMkConsumerWarps + 1);
// Ring: four 48 KB slots (a CTA's slice of most products fits one slot, so it is one bulk-copy chunk); measured on
// B200 against 6 x 32 KB: config 2 step 492 -> 484 us, config 3 step 835 -> 790 us (8 x 24 KB, 12 x 16 KB and
// 3 x 64 KB slower).
constexpr int kMkSlotBytes = 48 * 1024;
constexpr int kMkSlots = 4;
constexpr int kMkMaxK = 6144;
constexpr size_t kMkActBytes = 2 * kMkMaxK + (kMkMaxK / 32) * 4 + (kMkMaxK / 16) * 2 + 256;  // bf16 needs 2K bytes
constexpr size_t kMkSmemBytes = (size_t) kMkSlots * kMkSlotBytes + kMkActBytes + 2 * kMkSlots * 8 + 64;

// Conditions under which a product can run in the persistent step (host and device agree).
template <class T>
__host__ __device__ inline bool mk_type_fits(int64_t K) {
    int64_t rb = 0;
    for (int i = 0; i < T::kFields; i++) {
        if (T::field_row_bytes(K, i) % 16 != 0) return false;
        rb += T::field_row_bytes(K, i);
    }
    return rb <= kMkSlotBytes;
}

__host__ __device__ inline int64_t mk_row_bytes(int type, int64_t K) {
    switch (type) {
    case B200_TYPE_Q8_0: return K + K / 16;
    case B200_TYPE_Q4_K: return K / 2 + K / 16;
    case B200_TYPE_Q6_K: return K / 2 + K / 4 + K / 16 + K / 128;
    case B200_TYPE_BF16: return 2 * K;
    default: return 0;
    }
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void mk_sync() { asm volatile("bar.sync 1, %0;" ::"r"(32 * kMkConsumerWarps) : "memory"); }

// The same barrier, returning whether v was non-zero in any consumer thread.
__device__ __forceinline__ int mk_sync_or(int v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 q, %1, 0;\n\tbar.red.or.pred p, 1, %2, q;\n\tselp.s32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(v), "r"(32 * kMkConsumerWarps)
        : "memory");
    return r;
}

// Rows [r0, r1) of a product that CTA `cta` computes (contiguous, balanced; base = N / G, extra = N % G).
__device__ __forceinline__ void mk_slice(const MkStage & S, int cta, int64_t & r0, int64_t & r1) {
    const int base = S.slice_base, extra = S.slice_extra;
    r0 = (int64_t) cta * base + (cta < extra ? cta : extra);
    r1 = r0 + base + (cta < extra ? 1 : 0);
}

// Four tagged values starting at element k (16-byte aligned pairs of {value, tag} words). mk_ll4_try reads them once
// and reports whether every tag is `tag` (the asm is not volatile, so the compiler may issue a thread's first reads of
// all its chunks back to back: one L2 round trip, not one per chunk); mk_ll4 re-reads until they all are, bounded:
// after kSpinLimit reads it records a timeout in *fail and returns what it has.
__device__ __forceinline__ float4 mk_ll4_try(const float * base, int k, unsigned tag, int & ok) {
    const uint32_t * p = reinterpret_cast<const uint32_t *>(base) + 2 * (int64_t) k;
    uint32_t a0, t0, a1, t1, a2, t2, a3, t3;
    asm("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a0), "=r"(t0), "=r"(a1), "=r"(t1) : "l"(p));
    asm("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a2), "=r"(t2), "=r"(a3), "=r"(t3) : "l"(p + 4));
    ok = ((t0 ^ tag) | (t1 ^ tag) | (t2 ^ tag) | (t3 ^ tag)) == 0;
    return make_float4(__uint_as_float(a0), __uint_as_float(a1), __uint_as_float(a2), __uint_as_float(a3));
}

__device__ __forceinline__ float4 mk_ll4(const float * base, int k, unsigned tag, int * fail) {
    const uint32_t * p = reinterpret_cast<const uint32_t *>(base) + 2 * (int64_t) k;
    uint32_t a0, t0, a1, t1, a2, t2, a3, t3;
    for (uint32_t i = 0;; i++) {
        asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a0), "=r"(t0), "=r"(a1), "=r"(t1) : "l"(p) : "memory");
        asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a2), "=r"(t2), "=r"(a3), "=r"(t3) : "l"(p + 4) : "memory");
        if (((t0 ^ tag) | (t1 ^ tag) | (t2 ^ tag) | (t3 ^ tag)) == 0) break;
        if (i >= kSpinLimit) {
            *fail = 1;
            break;
        }
    }
    return make_float4(__uint_as_float(a0), __uint_as_float(a1), __uint_as_float(a2), __uint_as_float(a3));
}

// Four raw input values at element k of the input vector: one read (ok: they are the ones this product waits for;
// untagged inputs are always ready), or re-read until ready (wait == true).
__device__ __forceinline__ float4 mk_raw4(const MkStage & S, int k, unsigned tag, bool wait, int & ok, int * fail) {
    if (!S.x_tagged) {
        ok = 1;
        return __ldcg(reinterpret_cast<const float4 *>(S.x + k));
    }
    if (wait) {
        ok = 1;
        return mk_ll4(S.x, k, tag, fail);
    }
    return mk_ll4_try(S.x, k, tag, ok);
}

// Input values k .. k + 3 of product S after its prologue's element-wise part (SwiGLU, the grouped-query broadcast).
__device__ __forceinline__ float4 mk_load4(const MkStage & S, int k, unsigned tag, bool wait, int & ok, int * fail) {
    switch (S.pro) {
    case PRO_SWIGLU: {
        int ok2;
        const float4 g = mk_raw4(S, k, tag, wait, ok, fail);
        const float4 u = mk_raw4(S, S.pro_k + k, tag, wait, ok2, fail);
        ok &= ok2;
        return make_float4(__fmul_rn(silu_exact(g.x), u.x), __fmul_rn(silu_exact(g.y), u.y), __fmul_rn(silu_exact(g.z), u.z),
                           __fmul_rn(silu_exact(g.w), u.w));
    }
    case PRO_GQA: {
        if (S.gqa_shift >= 0 && S.hd_shift >= 0)
            return mk_raw4(S, ((k >> S.gqa_shift) << S.hd_shift) + (k & (S.pro_k - 1)), tag, wait, ok, fail);
        const int span = S.pro_k * S.pro_rep;
        return mk_raw4(S, (k / span) * S.pro_k + k % S.pro_k, tag, wait, ok, fail);
    }
    default:
        return mk_raw4(S, k, tag, wait, ok, fail);
    }
}

// Stages product S's quantized input in the act arrays (consumer threads only; ends with a barrier, whose result is
// whether any thread's tagged loads timed out).
// q8_0 (K % 1024 == 0): thread t holds values 4t + 1024 i; eight consecutive threads form one 32-block.
// q8_K (K % 2048 == 0): thread t holds values 8t + 2048 i; one warp forms one 256-block.
__device__ __forceinline__ int mk_stage_input(const MkStage & S, const Act & a, double * part, unsigned tag, int * fail) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = (int) S.w.K;
    const int kind = act_kind(S.w.type);
    const bool rmsnorm = S.pro == PRO_RMSNORM;
    if (kind == B200_TYPE_Q8_K) {
        constexpr int kMax = kMkMaxK / 2048;
        float v[kMax][8];
        double sq = 0.0;
        // every chunk read once (all reads in flight together), then re-read until ready if any was early
        int ready = 1;
#pragma unroll
        for (int pass = 0; pass < 2; pass++) {
            if (pass == 1 && ready) break;
#pragma unroll
            for (int i = 0; i < kMax; i++) {
                if (i < K / 2048) {
                    const int k = 8 * tid + 2048 * i;
                    int ok0, ok1;
                    const float4 lo = mk_load4(S, k, tag, pass == 1, ok0, fail), hi = mk_load4(S, k + 4, tag, pass == 1, ok1, fail);
                    ready &= ok0 & ok1;
                    v[i][0] = lo.x; v[i][1] = lo.y; v[i][2] = lo.z; v[i][3] = lo.w;
                    v[i][4] = hi.x; v[i][5] = hi.y; v[i][6] = hi.z; v[i][7] = hi.w;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kMax; i++)
            if (i < K / 2048)
#pragma unroll
                for (int j = 0; j < 8; j++) sq = fma((double) v[i][j], (double) v[i][j], sq);
        float rms = 0.0f;
        if (rmsnorm) {  // squares summed in double, the mean rounded once to float32 (the oracle's definition)
            sq = warp_sum_d(sq);
            if (lane == 0) part[warp] = sq;
            mk_sync();
            static_assert(kMkConsumerWarps == 8, "the warps' partial sums are added as a tree of eight");
            const double t = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
            rms = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean_rounded(t, K), S.eps)));
        }
#pragma unroll
        for (int i = 0; i < kMax; i++) {
            if (i < K / 2048) {
                const int k = 8 * tid + 2048 * i;
                if (rmsnorm) {  // norm weights: read-only, cached after the first step
                    const float4 w0 = __ldg(reinterpret_cast<const float4 *>(S.norm_w + k));
                    const float4 w1 = __ldg(reinterpret_cast<const float4 *>(S.norm_w + k + 4));
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int j = 0; j < 8; j++) v[i][j] = __fmul_rn(__fmul_rn(v[i][j], rms), wv[j]);
                }
                int8_t q[8];
                int16_t bsum;
                float d;
                quantize_q8_K_warp(v[i], q, &bsum, &d);
                int2 packed;
                packed.x = (int) (uint8_t) q[0] | ((int) (uint8_t) q[1] << 8) | ((int) (uint8_t) q[2] << 16) | ((int) (uint8_t) q[3] << 24);
                packed.y = (int) (uint8_t) q[4] | ((int) (uint8_t) q[5] << 8) | ((int) (uint8_t) q[6] << 16) | ((int) (uint8_t) q[7] << 24);
                *reinterpret_cast<int2 *>(a.q + k) = packed;
                const int b = k / 256;
                if ((lane & 1) == 0) a.bs[b * 16 + lane / 2] = bsum;
                if (lane == 0) a.d[b] = d;
            }
        }
    } else {
        constexpr int kMax = kMkMaxK / 1024;
        float4 v[kMax];
        double sq = 0.0;
        // every chunk read once (all reads in flight together), then re-read until ready if any was early
        int ready = 1;
#pragma unroll
        for (int pass = 0; pass < 2; pass++) {
            if (pass == 1 && ready) break;
#pragma unroll
            for (int i = 0; i < kMax; i++) {
                if (i < K / 1024) {
                    int ok;
                    v[i] = mk_load4(S, 4 * tid + 1024 * i, tag, pass == 1, ok, fail);
                    ready &= ok;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kMax; i++) {
            if (i < K / 1024) {
                sq = fma((double) v[i].x, (double) v[i].x, sq);
                sq = fma((double) v[i].y, (double) v[i].y, sq);
                sq = fma((double) v[i].z, (double) v[i].z, sq);
                sq = fma((double) v[i].w, (double) v[i].w, sq);
            }
        }
        float rms = 0.0f;
        if (rmsnorm) {  // squares summed in double, the mean rounded once to float32 (the oracle's definition)
            sq = warp_sum_d(sq);
            if (lane == 0) part[warp] = sq;
            mk_sync();
            static_assert(kMkConsumerWarps == 8, "the warps' partial sums are added as a tree of eight");
            const double t = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
            rms = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean_rounded(t, K), S.eps)));
        }
#pragma unroll
        for (int i = 0; i < kMax; i++) {
            if (i < K / 1024) {
                const int k = 4 * tid + 1024 * i;
                float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
                if (rmsnorm) {  // norm weights: read-only, cached after the first step
                    const float4 w = __ldg(reinterpret_cast<const float4 *>(S.norm_w + k));
                    e[0] = __fmul_rn(__fmul_rn(e[0], rms), w.x);
                    e[1] = __fmul_rn(__fmul_rn(e[1], rms), w.y);
                    e[2] = __fmul_rn(__fmul_rn(e[2], rms), w.z);
                    e[3] = __fmul_rn(__fmul_rn(e[3], rms), w.w);
                }
                if (kind == B200_TYPE_BF16) {
#pragma unroll
                    for (int j = 0; j < 4; j++) a.b[k + j] = __float2bfloat16_rn(e[j]);
                    continue;
                }
                float amax = fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3])));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                int w = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) w |= ((int) (uint8_t) (int8_t) (int) roundf(__fmul_rn(e[j], id))) << (8 * j);
                *reinterpret_cast<int *>(a.q + k) = w;
                if ((tid & 7) == 0) a.d[k / 32] = __half2float(__float2half_rn(d));
            }
        }
    }
    cp_async_wait_all();  // this thread's residual copies (issued before staging) have landed
    return mk_sync_or(*fail);
}

constexpr int kMkResRows = 64;  // residual values of a CTA's slice kept in shared memory (more: read from L2)

// Output row r of product S: value v (+ the residual), one {value, tag} word when tagged.
__device__ __forceinline__ void mk_store(const MkStage & S, int64_t r, int64_t r0, const float * res_s, float v, unsigned tag) {
    float out = v;
    if (S.res) out = __fadd_rn(r - r0 < kMkResRows ? res_s[r - r0] : __ldcg(S.res + (S.res_tagged ? 2 * r : r)), v);
    if (S.y_tagged)
        asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(S.y + 2 * r), "r"(__float_as_uint(out)), "r"(tag) : "memory");
    else
        S.y[r] = out;
}

// Rows of one landed chunk, two per warp at a time. res_s holds the residuals of the CTA's rows [r0, r0 + 64).
template <class T, bool kForms>
__device__ __forceinline__ void mk_rows(const MkStage & S, const Act & a, const uint8_t * slot, int64_t rps, int64_t rows,
                                        int64_t first, int64_t r0, const float * res_s, unsigned tag) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t K = S.w.K;
    const uint8_t * f[4];
    const uint8_t * b = slot;
    for (int i = 0; i < 4; i++) {
        f[i] = b;
        if (i < T::kFields) b += rps * T::field_row_bytes(K, i);
    }
    auto store = [&](int j, float v) { mk_store(S, first + j, r0, res_s, v, tag); };
    if constexpr (kForms) smem_rows<T, false>(f, K, (int) rows, a, S.w, warp, kMkConsumerWarps, store);
    else if (T::units_per_row(K) <= 64) smem_rows_lpr<T, 8>(f, K, (int) rows, a, S.w, warp, kMkConsumerWarps, store);
    else smem_rows_lpr<T, 32>(f, K, (int) rows, a, S.w, warp, kMkConsumerWarps, store);
}

// A gate|up product's chunk (features [first, first + rows)): the gate sums into gu_s[0], the up sums into gu_s[1],
// indexed by the feature's place in the CTA's slice. A slot holds per field the chunk's gate rows, then (from row rps)
// its up rows; one reduction walks rows [0, rps + rows) (so the row code is compiled once), and rows [rows, rps) of a
// short last chunk, which hold stale bytes, are reduced but not stored.
template <class T, bool kForms>
__device__ __forceinline__ void mk_rows_glu(const MkStage & S, const Act & a, const uint8_t * slot, int64_t rps, int64_t rows,
                                            int64_t first, int64_t r0, float (*gu_s)[kMkResRows]) {
    const int warp = threadIdx.x >> 5;
    const int64_t K = S.w.K;
    const uint8_t * f[4];
    const uint8_t * b = slot;
    for (int i = 0; i < 4; i++) {
        f[i] = b;
        if (i < T::kFields) b += 2 * rps * T::field_row_bytes(K, i);
    }
    const int64_t base = first - r0;
    auto store = [&](int j, float v) {
        if (j < rows) gu_s[0][base + j] = v;
        else if (j >= rps) gu_s[1][base + (j - rps)] = v;
    };
    const int n = (int) (rps + rows);
    if constexpr (kForms) smem_rows<T, false>(f, K, n, a, S.w, warp, kMkConsumerWarps, store);
    else if (T::units_per_row(K) <= 64) smem_rows_lpr<T, 8>(f, K, n, a, S.w, warp, kMkConsumerWarps, store);
    else smem_rows_lpr<T, 32>(f, K, n, a, S.w, warp, kMkConsumerWarps, store);
}

template <class T>
__device__ __forceinline__ void mk_issue(const MkStage & S, uint8_t * slot, int64_t rps, int64_t first, int64_t rows, uint64_t * bar) {
    const uint8_t * fb[4] = {S.w.f0, S.w.f1, S.w.f2, S.w.f3};
    uint8_t * dst = slot;
    for (int i = 0; i < T::kFields; i++) {
        const int64_t rb = T::field_row_bytes(S.w.K, i);
        bulk_g2s(dst, fb[i] + first * rb, (uint32_t) (rows * rb), bar);
        if (S.glu) bulk_g2s(dst + rps * rb, fb[i] + (S.N / 2 + first) * rb, (uint32_t) (rows * rb), bar);  // the up rows
        dst += (S.glu ? 2 : 1) * rps * rb;
    }
}

// kForms: the K-quant rows use their own lane layouts (smem_rows) rather than the generic unit reduction. The two
// instantiations differ only there, but register allocation is per kernel: a step whose products are all Q8_0 runs
// the generic one (measured on B200, config 2 step: 495 us against 552 us with the K-quant forms compiled in), a step
// with K-quant products the other (config 3 step: 845 us against 890 us).
template <bool kForms>
// One CTA per SM of kMkThreads threads: nine warps put three on one SM sub-partition, whose 16K registers then allow
// 168 a thread.
__global__ void __launch_bounds__(kMkThreads, 1) decoder_mk_kernel(MkParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double part[kMkConsumerWarps];
    __shared__ int give_up;
    __shared__ float res_s[kMkResRows];
    __shared__ float gu_s[2][kMkResRows];  // a gate|up product's sums of the CTA's features: gate, up
    __shared__ __align__(16) MkStage desc[3];  // this product's, the next one's, and the one after (being copied)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    uint8_t * ring = smem;
    uint8_t * act = smem + (size_t) kMkSlots * kMkSlotBytes;
    uint64_t * full = reinterpret_cast<uint64_t *>(act + kMkActBytes);
    uint64_t * empty = full + kMkSlots;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMkSlots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMkConsumerWarps);
        }
        fence_mbar_init();
        give_up = 0;
    }
    __syncthreads();

    if (warp == kMkConsumerWarps) {
        // ---- producer: every product's slice of weights, in chain order ----
        if (lane == 0) {
            uint32_t ctr = 0;
            for (int s = 0; s < P.nstages; s++) {
                const MkStage & S = P.stages[s];
                const int64_t rb = S.row_bytes;
                const int64_t rps = S.rps;
                int64_t r0, r1;
                mk_slice(S, cta, r0, r1);
                for (int64_t first = r0; first < r1; first += rps, ctr++) {
                    const int slot = (int) (ctr % kMkSlots);
                    const uint32_t it = ctr / kMkSlots;
                    if (it > 0 && !mbar_wait(&empty[slot], (it - 1) & 1)) {
                        atomicOr(P.err, 4u);
                        return;
                    }
                    const int64_t rows = r1 - first < rps ? r1 - first : rps;
                    mbar_arrive_expect_tx(&full[slot], (uint32_t) ((S.glu ? 2 : 1) * rows * rb));
                    uint8_t * dst = ring + (size_t) slot * kMkSlotBytes;
                    switch (S.w.type) {
                    case B200_TYPE_Q8_0: mk_issue<TQ8_0>(S, dst, rps, first, rows, &full[slot]); break;
                    case B200_TYPE_Q4_K: mk_issue<TQ4_K>(S, dst, rps, first, rows, &full[slot]); break;
                    case B200_TYPE_Q6_K: mk_issue<TQ6_K>(S, dst, rps, first, rows, &full[slot]); break;
                    default: mk_issue<TBF16>(S, dst, rps, first, rows, &full[slot]); break;
                    }
                }
            }
        }
        return;
    }

    // ---- consumers ----
    constexpr int kDescWords = sizeof(MkStage) / 4;
    static_assert(sizeof(MkStage) % 4 == 0, "descriptor copy by words");
    if (threadIdx.x < kDescWords) {
        reinterpret_cast<uint32_t *>(&desc[0])[threadIdx.x] = reinterpret_cast<const uint32_t *>(&P.stages[0])[threadIdx.x];
        if (P.nstages > 1)
            reinterpret_cast<uint32_t *>(&desc[1])[threadIdx.x] = reinterpret_cast<const uint32_t *>(&P.stages[1])[threadIdx.x];
    }
    const unsigned epoch = *reinterpret_cast<volatile unsigned *>(P.epoch);
    mk_sync();
    uint32_t ctr = 0;
    for (int s = 0; s < P.nstages; s++) {
        const MkStage & S = desc[s % 3];
        const unsigned in_tag = epoch * (unsigned) P.nstages + (unsigned) s;  // written by product s - 1
        const unsigned out_tag = in_tag + 1u;
        int64_t r0, r1;
        mk_slice(S, cta, r0, r1);
        // residuals of this CTA's rows (its own earlier outputs): asynchronous copies, complete before the staging
        // barrier below
        if (S.res && (int64_t) threadIdx.x < r1 - r0 && threadIdx.x < kMkResRows)
            cp_async4(&res_s[threadIdx.x], S.res + (S.res_tagged ? 2 * (r0 + threadIdx.x) : r0 + threadIdx.x));
        Act a;
        a.K = S.w.K;
        a.q = reinterpret_cast<int8_t *>(act);
        a.d = reinterpret_cast<float *>(act + 2 * kMkMaxK);
        a.bs = reinterpret_cast<int16_t *>(act + 2 * kMkMaxK + (kMkMaxK / 32) * 4);
        a.b = reinterpret_cast<__nv_bfloat16 *>(act);
        int fail = 0;
        if (mk_stage_input(S, a, part, in_tag, &fail)) {  // ends with a barrier: res_s is complete
            if (threadIdx.x == 0) atomicOr(P.err, 4u);
            break;
        }
        // the descriptor after next goes to the third buffer (this one, s % 3, stays readable during product s)
        if (s + 2 < P.nstages && threadIdx.x < kDescWords)
            cp_async4(reinterpret_cast<uint32_t *>(&desc[(s + 2) % 3]) + threadIdx.x, reinterpret_cast<const uint32_t *>(&P.stages[s + 2]) + threadIdx.x);

        const int64_t rps = S.rps;
        for (int64_t first = r0; first < r1; first += rps, ctr++) {
            const int slot = (int) (ctr % kMkSlots);
            if (!mbar_wait(&full[slot], (ctr / kMkSlots) & 1)) {
                if (lane == 0) atomicOr(P.err, 4u);
                give_up = 1;
                break;
            }
            const int64_t rows = r1 - first < rps ? r1 - first : rps;
            const uint8_t * sp = ring + (size_t) slot * kMkSlotBytes;
            if (S.glu) {
                switch (S.w.type) {
                case B200_TYPE_Q8_0: mk_rows_glu<TQ8_0, kForms>(S, a, sp, rps, rows, first, r0, gu_s); break;
                case B200_TYPE_Q4_K: mk_rows_glu<TQ4_K, kForms>(S, a, sp, rps, rows, first, r0, gu_s); break;
                case B200_TYPE_Q6_K: mk_rows_glu<TQ6_K, kForms>(S, a, sp, rps, rows, first, r0, gu_s); break;
                default: mk_rows_glu<TBF16, kForms>(S, a, sp, rps, rows, first, r0, gu_s); break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                continue;
            }
            switch (S.w.type) {
            case B200_TYPE_Q8_0: mk_rows<TQ8_0, kForms>(S, a, sp, rps, rows, first, r0, res_s, out_tag); break;
            case B200_TYPE_Q4_K: mk_rows<TQ4_K, kForms>(S, a, sp, rps, rows, first, r0, res_s, out_tag); break;
            case B200_TYPE_Q6_K: mk_rows<TQ6_K, kForms>(S, a, sp, rps, rows, first, r0, res_s, out_tag); break;
            default: mk_rows<TBF16, kForms>(S, a, sp, rps, rows, first, r0, res_s, out_tag); break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        cp_async_wait_all();  // the next descriptor has landed
        mk_sync();  // all outputs of this CTA for product s are written; the act arrays may be reused
        if (give_up) break;
        if (S.glu && (int64_t) threadIdx.x < r1 - r0) {
            // silu(gate) * up of the CTA's features, once each (SiLU evaluated exactly, as the oracle defines it)
            const float v = __fmul_rn(silu_exact(gu_s[0][threadIdx.x]), gu_s[1][threadIdx.x]);
            const int64_t r = r0 + threadIdx.x;
            asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(S.y + 2 * r), "r"(__float_as_uint(v)), "r"(out_tag) : "memory");
        }
    }
    // ---- end of the launch: once every CTA is here (all have read the epoch), CTA 0 advances it ----
    if (threadIdx.x == 0) {
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(P.finished), "r"(1u) : "memory");
        if (cta == 0) {
            uint32_t i = 0;
            while (ld_acquire(P.finished) < (unsigned) G)
                if (++i >= kSpinLimit) {
                    atomicOr(P.err, 4u);
                    break;
                }
            *reinterpret_cast<volatile unsigned *>(P.finished) = 0u;
            __threadfence();
            atomicAdd(P.epoch, 1u);
        }
    }
}

}  // namespace b200
