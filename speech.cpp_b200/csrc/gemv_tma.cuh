// gemv_tma.cuh — the TMA-streamed mat-vec: the HBM-bound form of gemv_kernel for rows whose fields are whole
// 16-byte lines (Q8_0 / Q4_K with K % 256 == 0, Q6_K with K % 2048 == 0, BF16 with K % 8 == 0).
//
// Each CTA owns a contiguous slice of rows. One producer warp streams that slice through a ring of shared-memory
// stages with bulk asynchronous copies (cp.async.bulk, one per field per stage, no multicast), each stage tracked by
// an mbarrier's transaction count; eight consumer warps stage the activations, then reduce each landed row from
// shared memory and hand the stage back. The producer issues its first stages before griddepcontrol.wait: weights
// depend on nothing, so in a chain of products (a decode step) a product's whole weight slice is in flight while
// the previous product finishes, and the memory system sees every byte of the slice requested at once.
// Every wait is bounded (mbar_wait): one that gives up sets B200_DEVERR_TIMEOUT and the CTA stops consuming.
#pragma once

#include "gemv.cuh"

namespace b200 {

constexpr int kTmaConsumerWarps = 8;
constexpr int kTmaThreads = 32 * (kTmaConsumerWarps + 1);
constexpr unsigned kDevErrTimeout = 4u;  // B200_DEVERR_TIMEOUT

template <class T>
__host__ __device__ inline int64_t tma_row_bytes(int64_t K) {
    int64_t b = 0;
    for (int i = 0; i < T::kFields; i++) b += T::field_row_bytes(K, i);
    return b;
}

template <class T>
__host__ __device__ inline bool tma_fits(int64_t K) {
    for (int i = 0; i < T::kFields; i++)
        if (T::field_row_bytes(K, i) % 16 != 0 || T::field_row_bytes(K, i) == 0) return false;
    return true;
}

// Shared memory: [ring: stages x stage bytes][activation staging][2 x stages mbarriers]
template <class T, int NC>
__host__ __device__ inline size_t tma_smem_bytes(int wtype, int64_t K, int rows_per_stage, int stages) {
    const size_t ring = (size_t) stages * rows_per_stage * tma_row_bytes<T>(K);
    return ring + ((act_smem_bytes(wtype, K, NC) + 15) & ~(size_t) 15) + 16 * (size_t) stages + 16;
}

// Two warp sums at once (their shuffles interleave, halving the reduction's latency per row).
__device__ __forceinline__ void warp_sum2(float & a, float & b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ta = __shfl_xor_sync(0xffffffffu, a, o);
        const float tb = __shfl_xor_sync(0xffffffffu, b, o);
        a += ta;
        b += tb;
    }
}

// Single-column products of `rows` landed rows (field pointers f, row j at local index j). A warp works on 32 / LPR
// rows at once, LPR lanes per row, each lane taking every LPR-th unit of its row (independent units: their loads and
// dp4a chains overlap), then an LPR-lane reduction. LPR = 8 for rows of up to 64 units, else 32. store(j, value).
template <class T, int LPR, class Store>
__device__ __forceinline__ void smem_rows_lpr(const uint8_t * const * f, int64_t K, int rows, const Act & a, const WeightView & w,
                                              int warp, int nwarps, Store store) {
    const int lane = threadIdx.x & 31;
    const int upr = (int) T::units_per_row(K);
    constexpr int kRowsPerPass = 32 / LPR;
    const int sub = lane / LPR, li = lane % LPR;
    for (int j0 = warp * kRowsPerPass; j0 < rows; j0 += nwarps * kRowsPerPass) {
        const int j = j0 + sub;
        const bool row_ok = j < rows;
        float acc[1] = {0.0f};
        constexpr int kU = T::kSmemUnroll;
        for (int u0 = 0; u0 < upr; u0 += LPR * kU) {
            typename T::Unit U[kU];
#pragma unroll
            for (int t = 0; t < kU; t++) {
                const int u = u0 + t * LPR + li;
                if (row_ok && u < upr) U[t] = T::load_s(f, K, j, u);
                else U[t] = T::load(w, 0, 0, false);
            }
#pragma unroll
            for (int t = 0; t < kU; t++) {
                const int u = u0 + t * LPR + li;
                T::template dot<1>(U[t], u, row_ok && u < upr, a, acc, nullptr);
            }
        }
        float v = acc[0];
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (row_ok && li == 0) store(j, v);
    }
}

// Lanes per row: 8 for rows of up to 64 units (a warp reduces 4 rows at once), 32 for longer rows. A function of K
// alone, so a row's summation order does not depend on how rows are chunked (launch geometry never changes results).
template <class T, class Store>
__device__ __forceinline__ void smem_rows(const uint8_t * const * f, int64_t K, int rows, const Act & a, const WeightView & w,
                                          int warp, int nwarps, Store store) {
    if (T::units_per_row(K) <= 64) smem_rows_lpr<T, 8>(f, K, rows, a, w, warp, nwarps, store);
    else smem_rows_lpr<T, 32>(f, K, rows, a, w, warp, nwarps, store);
}

template <class T, int NC>
__global__ void __launch_bounds__(kTmaThreads, 2) gemv_tma_kernel(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t K = p.w.K;
    const int rps = p.rows_per_stage, stages = p.stages;
    const int64_t row_bytes = tma_row_bytes<T>(K);
    const int64_t stage_bytes = (int64_t) rps * row_bytes;
    uint8_t * ring = smem;
    uint8_t * act_base = smem + stages * stage_bytes;
    uint64_t * full = reinterpret_cast<uint64_t *>(act_base + ((act_smem_bytes(p.w.type, K, NC) + 15) & ~(size_t) 15));
    uint64_t * empty = full + stages;

    const int64_t r_begin = (int64_t) blockIdx.x * p.rows_per_cta;
    const int64_t r_end = r_begin + p.rows_per_cta < p.N ? r_begin + p.rows_per_cta : p.N;
    const int64_t nrows = r_end > r_begin ? r_end - r_begin : 0;
    const int64_t nchunks = (nrows + rps - 1) / rps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // released by the one warp that consumed it
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kTmaConsumerWarps) {
        // ---- producer ----
        if (lane == 0) {
            const uint8_t * fb[4] = {p.w.f0, p.w.f1, p.w.f2, p.w.f3};
            for (int64_t c = 0; c < nchunks; c++) {
                const int s = (int) (c % stages);
                const int64_t it = c / stages;
                if (it > 0 && !mbar_wait(&empty[s], (uint32_t) ((it - 1) & 1))) {
                    atomicOr(p.err, kDevErrTimeout);
                    break;
                }
                const int64_t first = r_begin + c * rps;
                const int64_t rows = nrows - c * rps < rps ? nrows - c * rps : rps;
                mbar_arrive_expect_tx(&full[s], (uint32_t) (rows * row_bytes));
                uint8_t * dst = ring + s * stage_bytes;
                for (int i = 0; i < T::kFields; i++) {
                    const int64_t rb = T::field_row_bytes(K, i);
                    bulk_g2s(dst, fb[i] + (p.row0 + first) * rb, (uint32_t) (rows * rb), &full[s]);
                    dst += (int64_t) rps * rb;
                }
                if (c == 0) pdl_launch_dependents();
            }
            if (nchunks == 0) pdl_launch_dependents();
        }
        return;
    }

    // ---- consumers (threads 0 .. 255) ----
    const int nthr = 32 * kTmaConsumerWarps;
    pdl_launch_dependents();
    pdl_wait();
    Act a;
    const int kind = act_kind(p.w.type);
    {
        uint8_t * s = act_base;
        a.K = K;
        a.q = nullptr; a.d = nullptr; a.bs = nullptr; a.b = nullptr;
        if (kind == B200_TYPE_BF16) {
            a.b = reinterpret_cast<__nv_bfloat16 *>(s);
        } else {
            a.q = reinterpret_cast<int8_t *>(s);
            s += ((size_t) NC * K + 15) & ~(size_t) 15;
            a.d = reinterpret_cast<float *>(s);
            if (kind == B200_TYPE_Q8_K) {
                s += (size_t) NC * (K / 256) * 4;
                a.bs = reinterpret_cast<int16_t *>(s);
            }
        }
    }
    const int nc = p.ncols < NC ? p.ncols : NC;
    float * xs = reinterpret_cast<float *>(act_base + act_base_bytes(p.w.type, K, NC));
    if (NC == 1 && !p.aq && single_fast(K)) stage_one(p, a, kind, nc > 0 ? column_src(p, 0) : p.x, xs, xs + 2 * K, nthr);
    else stage_activations<NC>(p, a, kind, 0, nc, nthr);

    const int64_t upr = T::units_per_row(K);
    const int nsums = T::sums_per_row(K);
    // chunk c belongs to consumer warp c % W (W = min(8, stages); the host makes stages a multiple of W), so every
    // ring slot is consumed by one warp, which waits for the slot's phases strictly in order (a parity wait cannot
    // tell phase n from phase n + 2: a slot shared between warps could be taken a phase early)
    const int W = stages < kTmaConsumerWarps ? stages : kTmaConsumerWarps;
    for (int64_t c = warp; warp < W && c < nchunks; c += W) {
        const int s = (int) (c % stages);
        if (!mbar_wait(&full[s], (uint32_t) ((c / stages) & 1))) {
            if (lane == 0) atomicOr(p.err, kDevErrTimeout);
            break;
        }
        const int64_t rows = nrows - c * rps < rps ? nrows - c * rps : rps;
        const uint8_t * f[4];
        {
            const uint8_t * b = ring + s * stage_bytes;
            for (int i = 0; i < 4; i++) {
                f[i] = b;
                if (i < T::kFields) b += (int64_t) rps * T::field_row_bytes(K, i);
            }
        }
        const int64_t base = r_begin + c * rps;
        if (NC == 1 && !p.sums) {
            smem_rows<T>(f, K, (int) rows, a, p.w, 0, 1, [&](int j, float v) {
                if (nc > 0) {
                    const int64_t r = base + j;
                    p.y[r] = p.res ? __fadd_rn(p.res[r], v) : v;
                }
            });
        } else {
            for (int64_t j = 0; j < rows; j++) {
                const int64_t r = base + j;  // output row
                int32_t * sums = p.sums ? p.sums + r * nsums : nullptr;
                float acc[NC];
#pragma unroll
                for (int q = 0; q < NC; q++) acc[q] = 0.0f;
                for (int64_t u0 = 0; u0 < upr; u0 += 32) {
                    const int64_t u = u0 + lane;
                    const bool valid = u < upr;
                    typename T::Unit U;
                    if (valid) U = T::load_s(f, K, j, u);
                    else U = T::load(p.w, 0, 0, false);
                    T::template dot<NC>(U, u, valid, a, acc, sums);
                }
#pragma unroll
                for (int q = 0; q < NC; q++) {
                    const float v = warp_sum(acc[q]);
                    if (lane == 0 && q < nc && !p.sums) {
                        float out = v;
                        if (p.res) out = __fadd_rn(p.res[(int64_t) q * p.ldres + r], v);
                        p.y[(int64_t) q * p.ldy + r] = out;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

}  // namespace b200
