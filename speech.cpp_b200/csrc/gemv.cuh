// gemv.cuh — batch-1..8 dequant-fused matrix-vector products (ggml MUL_MAT with few src1 columns).
//
// Replaces the decode-step products of speech.cpp (src/common/qwen3-decoder.cpp:362-364, 403, 406-407, 410, 426, and
// the kept step graph :462-490) that ggml runs as mul_mat nodes (src/common/graph.h:15-19).
//
// Per launch: every CTA first stages the NC activation columns in shared memory, already quantized to the weight
// type's vec_dot type exactly as the CPU oracle does (q8_0 for Q8_0, q8_K for Q4_K/Q6_K, bf16 for BF16), optionally
// after a fused prologue (RMSNorm x weight, SwiGLU, or the grouped-query broadcast of a one-position attention).
// Warps then stream weight rows with 128-bit non-allocating loads (double-buffered, so the next unit's bytes are in
// flight while the current one is reduced), form the exact int32 (sub-)block sums with dp4a, scale them in float32,
// and warp-reduce each output. No tensor cores: one weight byte meets NC <= 8 activations, far below the ridge.
//
// With PDL, each CTA issues its first weight loads before griddepcontrol.wait, so a chain of products (a decode
// step) overlaps the next product's weight stream with the tail of the previous one.
#pragma once

#include "common.cuh"

namespace b200 {

enum Prologue : int {
    PRO_COPY = 0,     // x as given
    PRO_RMSNORM = 1,  // (x * 1/sqrt(mean(x^2) + eps)) * norm_w      (ggml_rms_norm then ggml_mul)
    PRO_SWIGLU = 2,   // silu(x[k]) * x[pro_k + k]                     (ggml_swiglu_split of gate | up)
    PRO_GQA = 3,      // x[(k / (pro_k * pro_rep)) * pro_k + k % pro_k] (attention over one position: o = v per head)
};

struct GemvParams {
    WeightView w;
    int64_t N;       // output rows of this launch
    int64_t row0;    // first weight row (expert offset / column shard)
    const float * x;
    int64_t ldx;     // floats between activation columns
    int pro;
    const float * norm_w;
    float eps;
    int64_t pro_k;
    int pro_rep;
    float * y;
    int64_t ldy;     // floats between output columns
    const float * res;
    int64_t ldres;
    int32_t * sums;  // when set: int32 (sub-)block sums of column 0, [N][sums_per_row], instead of y
    unsigned * err;  // device error word (bounded waits that give up set B200 timeout bits here)
    int rows_per_cta;     // TMA path: contiguous rows of one CTA
    int rows_per_stage;   // TMA path: rows per ring stage
    int stages;           // TMA path: ring stages
    int ncols;                // activation columns (without groups)
    const int32_t * col_src;  // optional: column c reads x row col_src[c]
    const int32_t * col_dst;  // optional: column c writes y (and reads res) row col_dst[c]
    const int32_t * grp_off;  // optional: CTA row blockIdx.y computes group g's columns [grp_off[g], grp_off[g+1])
    int64_t grp_rows;         //   with weight rows row0 + g * grp_rows (one expert's matrix)
    // optional: activations already quantized (b200 internal layout, rows of x): aq int8 [R][K], ad float
    // [R][K/32 or K/256], abs int16 [R][K/16]. Column c uses row col_src[c] (or c). Prologues do not apply.
    const int8_t * aq;
    const float * ad;
    const int16_t * abs;
};

// Shared-memory staging of NC quantized activation columns.
struct Act {
    int8_t * q;           // [NC][K]
    float * d;            // [NC][K/32] (q8_0) or [NC][K/256] (q8_K)
    int16_t * bs;         // [NC][K/16] (q8_K)
    __nv_bfloat16 * b;    // [NC][K] (bf16)
    int64_t K;
};

inline __host__ __device__ int act_kind(int wtype) {
    return wtype == B200_TYPE_Q8_0 ? B200_TYPE_Q8_0 : wtype == B200_TYPE_BF16 ? B200_TYPE_BF16 : B200_TYPE_Q8_K;
}

// The single-column path (a decode step's products) first copies its raw input rows into shared memory with
// coalesced 128-bit loads (up to 2K floats of input and K floats of norm weights), so that the prologue and the
// quantization read shared memory instead of waiting on global loads one after another.
inline __host__ __device__ bool single_fast(int64_t K) { return K % 32 == 0 && K * 13 + 4096 <= 180 * 1024; }

inline __host__ __device__ size_t act_base_bytes(int wtype, int64_t K, int nc) {
    const int kind = act_kind(wtype);
    if (kind == B200_TYPE_BF16) return (((size_t) nc * K * 2) + 15) & ~(size_t) 15;
    size_t s = (size_t) nc * K;                                   // q
    s = (s + 15) & ~(size_t) 15;
    if (kind == B200_TYPE_Q8_0) s += (size_t) nc * (K / 32) * 4;  // d
    else s += (size_t) nc * (K / 256) * 4 + (size_t) nc * (K / 16) * 2;
    return (s + 15) & ~(size_t) 15;
}

inline __host__ __device__ size_t act_smem_bytes(int wtype, int64_t K, int nc) {
    size_t s = act_base_bytes(wtype, K, nc);
    if (nc == 1 && single_fast(K)) s += (size_t) 12 * K;  // xs [2K] + ws [K]
    return s + 64;
}

// ---------------------------------------------------------------------------------------------------------------
// Prologue value of column c at index k.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float pro_value(const GemvParams & p, const float * xc, int c, int64_t k, const float * rms) {
    if (!xc) return 0.0f;
    switch (p.pro) {
    case PRO_RMSNORM: return __fmul_rn(__fmul_rn(xc[k], rms[c]), p.norm_w[k]);
    case PRO_SWIGLU: return __fmul_rn(silu_exact(xc[k]), xc[p.pro_k + k]);
    case PRO_GQA: {
        const int64_t span = p.pro_k * p.pro_rep;
        return xc[(k / span) * p.pro_k + k % p.pro_k];
    }
    default: return xc[k];
    }
}

// Stages NC columns (block-wide; ends with __syncthreads).
__device__ __forceinline__ const float * column_src(const GemvParams & p, int64_t c) {
    return p.x + (p.col_src ? (int64_t) p.col_src[c] : c) * p.ldx;
}

// Single-column staging (nc == 1, no prequantized rows, single_fast(K)). Block-wide; ends with __syncthreads.
// Arithmetic is that of the general path below (and of the CPU oracle), value by value.
// Barrier over the first nthr threads of the CTA (all of them: __syncthreads; fewer: named barrier 1).
__device__ __forceinline__ void sync_threads(int nthr) {
    if (nthr == (int) blockDim.x) __syncthreads();
    else asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
}

__device__ __forceinline__ void stage_one(const GemvParams & p, const Act & a, int kind, const float * xc, float * xs, float * ws,
                                          int nthr) {
    __shared__ double part[32];
    __shared__ float rms;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
    const int K = (int) a.K;
    const int hd = (int) p.pro_k, rep = p.pro_rep;
    // raw input -> xs; norm weights -> ws
    const int lin = p.pro == PRO_GQA ? K / rep : K;
    auto copy = [&](float * dst, const float * src, int n) {
        if ((((uintptr_t) src) & 15) == 0 && (n & 3) == 0) {
            const float4 * s4 = reinterpret_cast<const float4 *>(src);
            float4 * d4 = reinterpret_cast<float4 *>(dst);
            for (int i = tid; i < n / 4; i += nthr) d4[i] = s4[i];
        } else {
            for (int i = tid; i < n; i += nthr) dst[i] = src[i];
        }
    };
    copy(xs, xc, lin);
    if (p.pro == PRO_SWIGLU) copy(xs + K, xc + p.pro_k, K);
    if (p.pro == PRO_RMSNORM) copy(ws, p.norm_w, K);
    sync_threads(nthr);
    if (p.pro == PRO_RMSNORM) {
        // squares summed in double (exact products; the order changes nothing that survives the rounding to float32)
        double sq = 0.0;
        for (int k = tid; k < K; k += nthr) sq = fma((double) xs[k], (double) xs[k], sq);
        sq = warp_sum_d(sq);
        if (lane == 0) part[warp] = sq;
        sync_threads(nthr);
        if (warp == 0) {
            double t = lane < nwarps ? part[lane] : 0.0;
            t = warp_sum_d(t);
            if (lane == 0) rms = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean_rounded(t, K), p.eps)));
        }
        sync_threads(nthr);
    }
    auto value = [&](int k) -> float {
        switch (p.pro) {
        case PRO_RMSNORM: return __fmul_rn(__fmul_rn(xs[k], rms), ws[k]);
        case PRO_SWIGLU: return __fmul_rn(silu_exact(xs[k]), xs[K + k]);
        case PRO_GQA: return xs[(k / (hd * rep)) * hd + k % hd];
        default: return xs[k];
        }
    };
    if (kind == B200_TYPE_Q8_0) {
        // 8 threads per 32-block, 4 values each; the loop bound is uniform per warp so shuffles see all lanes
        const int nb = K / 32;
        for (int base = warp * 4; base < nb; base += nwarps * 4) {
            const int b = base + (lane >> 3), j = lane & 7;
            const bool on = b < nb;
            float v[4];
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                v[i] = on ? value(b * 32 + 4 * j + i) : 0.0f;
                amax = fmaxf(amax, fabsf(v[i]));
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
            if (on) {
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                int w = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) w |= ((int) (uint8_t) (int8_t) (int) roundf(__fmul_rn(v[i], id))) << (8 * i);
                reinterpret_cast<int *>(a.q)[b * 8 + j] = w;
                if (j == 0) a.d[b] = __half2float(__float2half_rn(d));
            }
        }
    } else if (kind == B200_TYPE_Q8_K) {
        const int nb = K / 256;
        for (int b = warp; b < nb; b += nwarps) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = value(b * 256 + lane * 8 + i);
            int8_t q[8];
            int16_t bsum;
            float d;
            quantize_q8_K_warp(v, q, &bsum, &d);
            int2 packed;
            packed.x = (int) (uint8_t) q[0] | ((int) (uint8_t) q[1] << 8) | ((int) (uint8_t) q[2] << 16) | ((int) (uint8_t) q[3] << 24);
            packed.y = (int) (uint8_t) q[4] | ((int) (uint8_t) q[5] << 8) | ((int) (uint8_t) q[6] << 16) | ((int) (uint8_t) q[7] << 24);
            *reinterpret_cast<int2 *>(a.q + b * 256 + lane * 8) = packed;
            if ((lane & 1) == 0) a.bs[b * 16 + lane / 2] = bsum;
            if (lane == 0) a.d[b] = d;
        }
    } else {
        for (int k = tid; k < K; k += nthr) a.b[k] = __float2bfloat16_rn(value(k));
    }
    sync_threads(nthr);
}

// Stages columns c0 .. c0+nc-1 (nc <= NC; the rest are zeros). Block-wide; ends with __syncthreads.
template <int NC>
__device__ void stage_activations(const GemvParams & p, const Act & a, int kind, int64_t c0, int nc, int nthr) {
    __shared__ float rms[NC];
    __shared__ const float * xcol[NC];
    if (threadIdx.x < NC) xcol[threadIdx.x] = (int) threadIdx.x < nc ? column_src(p, c0 + threadIdx.x) : nullptr;
    sync_threads(nthr);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = nthr >> 5;
    const int64_t K = a.K;
    if (p.pro == PRO_RMSNORM) {
        __shared__ double part[NC][32];
        for (int c = 0; c < NC; c++) {
            const float * xc = xcol[c];
            double s = 0.0;
            if (xc)
                for (int64_t k = threadIdx.x; k < K; k += nthr) s = fma((double) xc[k], (double) xc[k], s);
            s = warp_sum_d(s);
            if (lane == 0) part[c][warp] = s;
        }
        sync_threads(nthr);
        if (warp == 0) {
            for (int c = 0; c < NC; c++) {
                double s = lane < nwarps ? part[c][lane] : 0.0;
                s = warp_sum_d(s);
                if (lane == 0) rms[c] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean_rounded(s, K), p.eps)));
            }
        }
        sync_threads(nthr);
    }
    if (p.aq) {
        // prequantized rows: copy into shared memory
        for (int c = 0; c < NC; c++) {
            const int64_t row = c < nc ? (p.col_src ? (int64_t) p.col_src[c0 + c] : c0 + c) : -1;
            const int4 * src = row >= 0 ? reinterpret_cast<const int4 *>(p.aq + row * K) : nullptr;
            int4 * dst = reinterpret_cast<int4 *>(a.q + (int64_t) c * K);
            for (int64_t i = threadIdx.x; i < K / 16; i += nthr) dst[i] = src ? src[i] : make_int4(0, 0, 0, 0);
            const int64_t nd = kind == B200_TYPE_Q8_0 ? K / 32 : K / 256;
            for (int64_t i = threadIdx.x; i < nd; i += nthr) a.d[(int64_t) c * nd + i] = src ? p.ad[row * nd + i] : 0.0f;
            if (kind == B200_TYPE_Q8_K)
                for (int64_t i = threadIdx.x; i < K / 16; i += nthr)
                    a.bs[(int64_t) c * (K / 16) + i] = src ? p.abs[row * (K / 16) + i] : (int16_t) 0;
        }
    } else if (kind == B200_TYPE_Q8_0) {
        // one thread per 32-block: the shortest critical path when a step's products wait on one another
        const int64_t nb = K / 32;
        for (int64_t i = threadIdx.x; i < NC * nb; i += nthr) {
            const int c = (int) (i / nb);
            const int64_t b = i % nb;
            const float * xc = xcol[c];
            float v[32];
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                v[j] = pro_value(p, xc, c, b * 32 + j, rms);
                amax = fmaxf(amax, fabsf(v[j]));
            }
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            int packed[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                int w = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) w |= ((int) (uint8_t) (int8_t) (int) roundf(__fmul_rn(v[4 * j + t], id))) << (8 * t);
                packed[j] = w;
            }
            int4 * dst = reinterpret_cast<int4 *>(a.q + (int64_t) c * K + b * 32);
            dst[0] = make_int4(packed[0], packed[1], packed[2], packed[3]);
            dst[1] = make_int4(packed[4], packed[5], packed[6], packed[7]);
            a.d[(int64_t) c * nb + b] = __half2float(__float2half_rn(d));
        }
    } else if (kind == B200_TYPE_Q8_K) {
        const int64_t nb = K / 256;
        for (int64_t i = warp; i < NC * nb; i += nwarps) {
            const int c = (int) (i / nb);
            const int64_t b = i % nb;
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = pro_value(p, xcol[c], c, b * 256 + lane * 8 + j, rms);
            int8_t q[8];
            int16_t bsum;
            float d;
            quantize_q8_K_warp(v, q, &bsum, &d);
            int2 packed;
            packed.x = (int) (uint8_t) q[0] | ((int) (uint8_t) q[1] << 8) | ((int) (uint8_t) q[2] << 16) | ((int) (uint8_t) q[3] << 24);
            packed.y = (int) (uint8_t) q[4] | ((int) (uint8_t) q[5] << 8) | ((int) (uint8_t) q[6] << 16) | ((int) (uint8_t) q[7] << 24);
            *reinterpret_cast<int2 *>(a.q + (int64_t) c * K + b * 256 + lane * 8) = packed;
            if ((lane & 1) == 0) a.bs[(int64_t) c * (K / 16) + b * 16 + lane / 2] = bsum;
            if (lane == 0) a.d[(int64_t) c * nb + b] = d;
        }
    } else {
        for (int64_t i = threadIdx.x; i < NC * K; i += nthr) {
            const int c = (int) (i / K);
            a.b[i] = __float2bfloat16_rn(pro_value(p, xcol[c], c, i % K, rms));
        }
    }
    sync_threads(nthr);
}

// ---------------------------------------------------------------------------------------------------------------
// Per-type streaming units. A "unit" is what one lane loads per step; lanes of one (sub-)block cooperate through
// shuffles, so every lane calls dot() for every step (invalid units contribute zero).
// ---------------------------------------------------------------------------------------------------------------

// Byte i (0..15) of a 16-byte register value, without spilling it to local memory.
__device__ __forceinline__ int byte_of(const int4 & v, int i) {
    const int w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    return (w >> (8 * (i & 3))) & 0xFF;
}

struct TQ8_0 {
    // unit = one whole 32-block: 32 bytes of qs and its fp16 scale (one lane per block, no shuffles). Lanes 4..7 of
    // every 8 read the block's second 16 bytes first: each 8-lane phase of a 128-bit shared load then covers all 32
    // banks once (blocks are 32 bytes apart), for the weights and the activations alike.
    struct Unit { int4 q0; int4 q1; uint16_t d; };
    static constexpr int kUnroll = 2;
    static constexpr int kSmemUnroll = 2;  // units in flight per lane when reducing rows from shared memory
    __device__ static int64_t units_per_row(int64_t K) { return K / 32; }
    __device__ static int sums_per_row(int64_t K) { return (int) (K / 32); }
    __device__ static Unit load(const WeightView & w, int64_t row, int64_t u, bool valid) {
        Unit r;
        if (valid) {
            const uint8_t * p = w.f0 + row * w.K + u * 32;
            const int h = (threadIdx.x >> 2) & 1;
            r.q0 = ld_stream(p + 16 * h);
            r.q1 = ld_stream(p + 16 * (1 - h));
            r.d = __ldg(reinterpret_cast<const unsigned short *>(w.f1) + row * (w.K / 32) + u);
        } else {
            r.q0 = r.q1 = make_int4(0, 0, 0, 0);
            r.d = 0;
        }
        return r;
    }
    // shared-memory staging of rows (TMA path): field 0 = qs [rows][K], field 1 = d [rows][K/32]
    static constexpr int kFields = 2;
    __host__ __device__ static int64_t field_row_bytes(int64_t K, int i) { return i == 0 ? K : i == 1 ? K / 16 : 0; }
    __device__ static Unit load_s(const uint8_t * const * f, int64_t K, int64_t row, int64_t u) {
        Unit r;
        const int off = (int) row * (int) K + (int) u * 32;
        const int h = (threadIdx.x >> 2) & 1;
        r.q0 = *reinterpret_cast<const int4 *>(f[0] + off + 16 * h);
        r.q1 = *reinterpret_cast<const int4 *>(f[0] + off + 16 * (1 - h));
        r.d = reinterpret_cast<const uint16_t *>(f[1])[(int) row * (int) (K / 32) + (int) u];
        return r;
    }
    template <int NC>
    __device__ static void dot(const Unit & U, int64_t u, bool valid, const Act & a, double * acc, int32_t * sums) {
        if (!valid) return;
        const float dw = __half2float(__ushort_as_half(U.d));
        const int ui = (int) u, K = (int) a.K;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int h = (threadIdx.x >> 2) & 1;
            const int4 * xp = reinterpret_cast<const int4 *>(a.q + c * K + ui * 32);
            const int4 x0 = xp[h], x1 = xp[1 - h];
            int s = __dp4a(U.q0.x, x0.x, 0);
            s = __dp4a(U.q0.y, x0.y, s);
            s = __dp4a(U.q0.z, x0.z, s);
            s = __dp4a(U.q0.w, x0.w, s);
            s = __dp4a(U.q1.x, x1.x, s);
            s = __dp4a(U.q1.y, x1.y, s);
            s = __dp4a(U.q1.z, x1.z, s);
            s = __dp4a(U.q1.w, x1.w, s);
            acc[c] = acc_term(acc[c], __fmul_rn(dw, a.d[c * (K / 32) + ui]), s);
            if (c == 0 && sums) sums[ui] = s;
        }
    }
};

struct TQ4_K {
    // unit = 32 bytes of qs: super-block u/4, chunk g = u%4 holding sub-blocks 2g (low nibbles) and 2g+1 (high
    // nibbles), all 32 values of each; plus the super-block's 16-byte meta. Four lanes per super-block.
    struct Unit { int4 q0; int4 q1; int4 m; };
    static constexpr int kUnroll = 2;
    static constexpr int kSmemUnroll = 2;
    __device__ static int64_t units_per_row(int64_t K) { return K / 64; }
    __device__ static int sums_per_row(int64_t K) { return (int) (2 * (K / 256)); }
    __device__ static Unit load(const WeightView & w, int64_t row, int64_t u, bool valid) {
        Unit r;
        if (valid) {
            const uint8_t * p = w.f0 + row * (w.K / 2) + u * 32;
            r.q0 = ld_stream(p);
            r.q1 = ld_stream(p + 16);
            r.m = __ldg(reinterpret_cast<const int4 *>(w.f1 + (row * (w.K / 256) + u / 4) * 16));
        } else {
            r.q0 = r.q1 = r.m = make_int4(0, 0, 0, 0);
        }
        return r;
    }
    static constexpr int kFields = 2;  // qs [rows][K/2], meta [rows][K/256][16]
    __host__ __device__ static int64_t field_row_bytes(int64_t K, int i) { return i == 0 ? K / 2 : i == 1 ? K / 16 : 0; }
    __device__ static Unit load_s(const uint8_t * const * f, int64_t K, int64_t row, int64_t u) {
        Unit r;
        const int off = (int) row * (int) (K / 2) + (int) u * 32;
        r.q0 = *reinterpret_cast<const int4 *>(f[0] + off);
        r.q1 = *reinterpret_cast<const int4 *>(f[0] + off + 16);
        r.m = *reinterpret_cast<const int4 *>(f[1] + ((int) row * (int) (K / 256) + (int) u / 4) * 16);
        return r;
    }
    // six-bit scale and min of sub-block j from the 12 scale bytes, which are bytes 4..15 of the meta value
    __device__ static void scale_min_reg(const int4 & m, int j, int & sc, int & mn) {
        if (j < 4) {
            sc = byte_of(m, 4 + j) & 63;
            mn = byte_of(m, 8 + j) & 63;
        } else {
            sc = (byte_of(m, 12 + j - 4) & 15) | ((byte_of(m, 4 + j - 4) >> 6) << 4);
            mn = (byte_of(m, 12 + j - 4) >> 4) | ((byte_of(m, 8 + j - 4) >> 6) << 4);
        }
    }
    // the same from a byte pointer (GET_ROWS)
    __device__ static void scale_min(const uint8_t * s, int j, int & sc, int & m) {
        if (j < 4) {
            sc = s[j] & 63;
            m = s[j + 4] & 63;
        } else {
            sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
            m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
    }
    // six-bit scale and min of sub-block j (0..7) from the meta words y = bytes 4..7, z = 8..11, w = 12..15
    __device__ static void scale_min_words(int y, int z, int w, int j, int & sc, int & mn) {
        const int sh = 8 * (j & 3);
        const int by = (y >> sh) & 0xFF, bz = (z >> sh) & 0xFF, bw = (w >> sh) & 0xFF;
        if (j < 4) {
            sc = by & 63;
            mn = bz & 63;
        } else {
            sc = (bw & 15) | ((by >> 6) << 4);
            mn = (bw >> 4) | ((bz >> 6) << 4);
        }
    }
    template <int NC>
    __device__ static void dot(const Unit & U, int64_t u, bool valid, const Act & a, double * acc, int32_t * sums) {
        const int ui = (int) u, K = (int) a.K;
        const int sb = ui >> 2, g = ui & 3, s0 = 2 * g, s1 = 2 * g + 1;
        int sc0 = 0, m0 = 0, sc1 = 0, m1 = 0;
        if (valid) {
            scale_min_words(U.m.y, U.m.z, U.m.w, s0, sc0, m0);
            scale_min_words(U.m.y, U.m.z, U.m.w, s1, sc1, m1);
        }
        const float dw = __half2float(__ushort_as_half((unsigned short) (U.m.x & 0xFFFF)));
        const float dmw = __half2float(__ushort_as_half((unsigned short) ((unsigned) U.m.x >> 16)));
        const int w[8] = {U.q0.x, U.q0.y, U.q0.z, U.q0.w, U.q1.x, U.q1.y, U.q1.z, U.q1.w};
#pragma unroll
        for (int c = 0; c < NC; c++) {
            int si = 0, sm = 0;
            if (valid) {
                const int8_t * xq = a.q + c * K + sb * 256;
                const int4 * xl = reinterpret_cast<const int4 *>(xq + s0 * 32);
                const int4 * xh = reinterpret_cast<const int4 *>(xq + s1 * 32);
                const int4 l0 = xl[0], l1 = xl[1], h0 = xh[0], h1 = xh[1];
                const int xlv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                const int xhv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                int il = 0, ih = 0;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    il = __dp4a(w[i] & 0x0F0F0F0F, xlv[i], il);
                    ih = __dp4a((w[i] >> 4) & 0x0F0F0F0F, xhv[i], ih);
                }
                si = sc0 * il + sc1 * ih;
                // sums of each 32 activations: bsums 2s and 2s+1 are adjacent int16, one 32-bit load each
                const int * bs2 = reinterpret_cast<const int *>(a.bs + c * (K / 16) + sb * 16);
                const int p0 = bs2[s0], p1 = bs2[s1];
                sm = m0 * ((int) (int16_t) (p0 & 0xFFFF) + (p0 >> 16)) + m1 * ((int) (int16_t) (p1 & 0xFFFF) + (p1 >> 16));
            }
            if (sums) {
                // the block-sums path forms the super-block's exact int32 sums over its four lanes
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                sm += __shfl_xor_sync(0xffffffffu, sm, 1);
                sm += __shfl_xor_sync(0xffffffffu, sm, 2);
                if (valid && g == 0 && c == 0) {
                    sums[2 * sb] = si;
                    sums[2 * sb + 1] = sm;
                }
            }
            if (valid && (!sums || g == 0)) {
                // each lane's exact partial sums, scaled in float (the super-block's scale is common to its lanes)
                const float dx = a.d[c * (K / 256) + sb];
                acc[c] = acc_term(acc[c], __fmul_rn(dx, dw), si);
                acc[c] = acc_term(acc[c], -__fmul_rn(dx, dmw), sm);
            }
        }
    }
};

struct TQ5_K {
    // unit = 32 bytes of qs (super-block u/4, chunk g = u%4: the low nibbles are the 32 values of sub-block 2g, the high
    // nibbles those of sub-block 2g+1, as in Q4_K), the super-block's 32 fifth-bit bytes (bit j of byte l: value l of
    // sub-block j) and its 16-byte meta (d, dmin, the 12 scale bytes packed as Q4_K's). Four lanes per super-block.
    struct Unit { int4 q0; int4 q1; int4 h0; int4 h1; int4 m; };
    static constexpr int kUnroll = 1;
    static constexpr int kSmemUnroll = 1;
    __device__ static int64_t units_per_row(int64_t K) { return K / 64; }
    __device__ static int sums_per_row(int64_t K) { return (int) (2 * (K / 256)); }
    __device__ static Unit load(const WeightView & w, int64_t row, int64_t u, bool valid) {
        Unit r;
        if (valid) {
            const uint8_t * p = w.f0 + row * (w.K / 2) + u * 32;
            const uint8_t * h = w.f2 + row * (w.K / 8) + (u / 4) * 32;
            r.q0 = ld_stream(p);
            r.q1 = ld_stream(p + 16);
            r.h0 = ld_stream(h);
            r.h1 = ld_stream(h + 16);
            r.m = __ldg(reinterpret_cast<const int4 *>(w.f1 + (row * (w.K / 256) + u / 4) * 16));
        } else {
            r.q0 = r.q1 = r.h0 = r.h1 = r.m = make_int4(0, 0, 0, 0);
        }
        return r;
    }
    static constexpr int kFields = 3;  // qs [rows][K/2], meta [rows][K/256][16], qh [rows][K/8]
    __host__ __device__ static int64_t field_row_bytes(int64_t K, int i) { return i == 0 ? K / 2 : i == 1 ? K / 16 : i == 2 ? K / 8 : 0; }
    __device__ static Unit load_s(const uint8_t * const * f, int64_t K, int64_t row, int64_t u) {
        Unit r;
        const uint8_t * p = f[0] + row * (K / 2) + u * 32;
        const uint8_t * h = f[2] + row * (K / 8) + (u / 4) * 32;
        r.q0 = *reinterpret_cast<const int4 *>(p);
        r.q1 = *reinterpret_cast<const int4 *>(p + 16);
        r.h0 = *reinterpret_cast<const int4 *>(h);
        r.h1 = *reinterpret_cast<const int4 *>(h + 16);
        r.m = *reinterpret_cast<const int4 *>(f[1] + (row * (K / 256) + u / 4) * 16);
        return r;
    }
    template <int NC>
    __device__ static void dot(const Unit & U, int64_t u, bool valid, const Act & a, double * acc, int32_t * sums) {
        const int ui = (int) u, K = (int) a.K;
        const int sb = ui >> 2, g = ui & 3, s0 = 2 * g, s1 = 2 * g + 1;
        int sc0 = 0, m0 = 0, sc1 = 0, m1 = 0;
        if (valid) {
            TQ4_K::scale_min_words(U.m.y, U.m.z, U.m.w, s0, sc0, m0);
            TQ4_K::scale_min_words(U.m.y, U.m.z, U.m.w, s1, sc1, m1);
        }
        const float dw = __half2float(__ushort_as_half((unsigned short) (U.m.x & 0xFFFF)));
        const float dmw = __half2float(__ushort_as_half((unsigned short) ((unsigned) U.m.x >> 16)));
        const int w[8] = {U.q0.x, U.q0.y, U.q0.z, U.q0.w, U.q1.x, U.q1.y, U.q1.z, U.q1.w};
        const int hb[8] = {U.h0.x, U.h0.y, U.h0.z, U.h0.w, U.h1.x, U.h1.y, U.h1.z, U.h1.w};
#pragma unroll
        for (int c = 0; c < NC; c++) {
            int si = 0, sm = 0;
            if (valid) {
                const int8_t * xq = a.q + c * K + sb * 256;
                const int4 * xl = reinterpret_cast<const int4 *>(xq + s0 * 32);
                const int4 * xh = reinterpret_cast<const int4 *>(xq + s1 * 32);
                const int4 l0 = xl[0], l1 = xl[1], h0 = xh[0], h1 = xh[1];
                const int xlv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                const int xhv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                int il = 0, ih = 0;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    // five-bit values of bytes 4i .. 4i+3: the nibble and the sub-block's bit of the high-bit byte
                    const int lo = (w[i] & 0x0F0F0F0F) | (((hb[i] >> s0) & 0x01010101) << 4);
                    const int hi = ((w[i] >> 4) & 0x0F0F0F0F) | (((hb[i] >> s1) & 0x01010101) << 4);
                    il = __dp4a(lo, xlv[i], il);
                    ih = __dp4a(hi, xhv[i], ih);
                }
                si = sc0 * il + sc1 * ih;
                const int * bs2 = reinterpret_cast<const int *>(a.bs + c * (K / 16) + sb * 16);
                const int p0 = bs2[s0], p1 = bs2[s1];
                sm = m0 * ((int) (int16_t) (p0 & 0xFFFF) + (p0 >> 16)) + m1 * ((int) (int16_t) (p1 & 0xFFFF) + (p1 >> 16));
            }
            if (sums) {
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                sm += __shfl_xor_sync(0xffffffffu, sm, 1);
                sm += __shfl_xor_sync(0xffffffffu, sm, 2);
                if (valid && g == 0 && c == 0) {
                    sums[2 * sb] = si;
                    sums[2 * sb + 1] = sm;
                }
            }
            if (valid && (!sums || g == 0)) {
                const float dx = a.d[c * (K / 256) + sb];
                acc[c] = acc_term(acc[c], __fmul_rn(dx, dw), si);
                acc[c] = acc_term(acc[c], -__fmul_rn(dx, dmw), sm);
            }
        }
    }
};

struct TQ6_K {
    // unit = a quarter of a super-block: half h = (u%4)/2, values l in [lq, lq+16), lq = (u%2)*16, all four t:
    // 16 bytes of ql (t = 0, 2), 16 bytes of ql (t = 1, 3), 16 bytes of qh, and the 16 scales.
    struct Unit { int4 a; int4 b; int4 h; int4 s; uint16_t d; };
    static constexpr int kUnroll = 1;
    static constexpr int kSmemUnroll = 1;
    __device__ static int64_t units_per_row(int64_t K) { return K / 64; }
    __device__ static int sums_per_row(int64_t K) { return (int) (K / 256); }
    __device__ static Unit load(const WeightView & w, int64_t row, int64_t u, bool valid) {
        Unit r;
        if (valid) {
            const int64_t sb = u / 4;
            const int j = (int) (u & 3), h = j >> 1, lq = (j & 1) * 16;
            const int64_t nsb = w.K / 256;
            const uint8_t * ql = w.f0 + row * (w.K / 2) + sb * 128 + h * 64 + lq;
            r.a = ld_stream(ql);
            r.b = ld_stream(ql + 32);
            r.h = ld_stream(w.f1 + row * (w.K / 4) + sb * 64 + h * 32 + lq);
            r.s = __ldg(reinterpret_cast<const int4 *>(w.f2 + (row * nsb + sb) * 16));
            r.d = __ldg(reinterpret_cast<const unsigned short *>(w.f3) + row * nsb + sb);
        } else {
            r.a = r.b = r.h = r.s = make_int4(0, 0, 0, 0);
            r.d = 0;
        }
        return r;
    }
    static constexpr int kFields = 4;  // ql [rows][K/2], qh [rows][K/4], sc [rows][K/256][16], d [rows][K/256]
    __host__ __device__ static int64_t field_row_bytes(int64_t K, int i) {
        return i == 0 ? K / 2 : i == 1 ? K / 4 : i == 2 ? K / 16 : K / 128;
    }
    __device__ static Unit load_s(const uint8_t * const * f, int64_t K, int64_t row, int64_t u) {
        Unit r;
        const int64_t sb = u / 4, nsb = K / 256;
        const int j = (int) (u & 3), h = j >> 1, lq = (j & 1) * 16;
        const uint8_t * ql = f[0] + row * (K / 2) + sb * 128 + h * 64 + lq;
        r.a = *reinterpret_cast<const int4 *>(ql);
        r.b = *reinterpret_cast<const int4 *>(ql + 32);
        r.h = *reinterpret_cast<const int4 *>(f[1] + row * (K / 4) + sb * 64 + h * 32 + lq);
        r.s = *reinterpret_cast<const int4 *>(f[2] + (row * nsb + sb) * 16);
        r.d = reinterpret_cast<const uint16_t *>(f[3])[row * nsb + sb];
        return r;
    }
    template <int NC>
    __device__ static void dot(const Unit & U, int64_t u, bool valid, const Act & a, double * acc, int32_t * sums) {
        const int * A = reinterpret_cast<const int *>(&U.a);
        const int * B = reinterpret_cast<const int *>(&U.b);
        const int * H = reinterpret_cast<const int *>(&U.h);
        const int64_t sb = u / 4;
        const int j = (int) (u & 3), h = j >> 1, lh = j & 1;
        const float dw = __half2float(__ushort_as_half(U.d));
#pragma unroll
        for (int c = 0; c < NC; c++) {
            int si = 0;
            if (valid) {
                const int8_t * xq = a.q + (int64_t) c * a.K + sb * 256 + h * 128 + lh * 16;
                const int16_t * bs = a.bs + (int64_t) c * (a.K / 16) + sb * 16 + h * 8 + lh;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int4 xv = *reinterpret_cast<const int4 *>(xq + t * 32);
                    const int * src = (t & 1) ? B : A;
                    const int shift = (t >> 1) * 4;
                    int s = 0;
                    const int xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int v = ((src[i] >> shift) & 0x0F0F0F0F) | (((H[i] >> (2 * t)) & 0x03030303) << 4);
                        s = __dp4a(v, xs[i], s);
                    }
                    // sum (q - 32) x = sum q x - 32 sum x; sum x over these 16 values is their q8_K bsum
                    s -= 32 * (int) bs[2 * t];
                    si += (int) (int8_t) byte_of(U.s, h * 8 + 2 * t + lh) * s;
                }
            }
            if (sums) {
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                if (valid && j == 0 && c == 0) sums[sb] = si;
            }
            if (valid && (!sums || j == 0)) {
                const float dx = a.d[(int64_t) c * (a.K / 256) + sb];
                acc[c] = acc_term(acc[c], __fmul_rn(dw, dx), si);
            }
        }
    }
};

struct TBF16 {
    struct Unit { int4 q; };
    static constexpr int kUnroll = 4;
    static constexpr int kSmemUnroll = 4;
    __device__ static int64_t units_per_row(int64_t K) { return K / 8; }
    __device__ static int sums_per_row(int64_t) { return 0; }
    __device__ static Unit load(const WeightView & w, int64_t row, int64_t u, bool valid) {
        Unit r;
        r.q = valid ? ld_stream(w.f0 + (row * w.K + u * 8) * 2) : make_int4(0, 0, 0, 0);
        return r;
    }
    static constexpr int kFields = 1;  // w [rows][K] bf16
    __host__ __device__ static int64_t field_row_bytes(int64_t K, int i) { return i == 0 ? 2 * K : 0; }
    __device__ static Unit load_s(const uint8_t * const * f, int64_t K, int64_t row, int64_t u) {
        Unit r;
        r.q = *reinterpret_cast<const int4 *>(f[0] + (row * K + u * 8) * 2);
        return r;
    }
    template <int NC>
    __device__ static void dot(const Unit & U, int64_t u, bool valid, const Act & a, double * acc, int32_t *) {
        if (!valid) return;
        const __nv_bfloat162 * wv = reinterpret_cast<const __nv_bfloat162 *>(&U.q);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int4 xr = *reinterpret_cast<const int4 *>(a.b + (int64_t) c * a.K + u * 8);
            const __nv_bfloat162 * xv = reinterpret_cast<const __nv_bfloat162 *>(&xr);
            double s = acc[c];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 wf = __bfloat1622float2(wv[i]);
                const float2 xf = __bfloat1622float2(xv[i]);
                s += (double) __fmul_rn(wf.x, xf.x);  // bf16 x bf16 is exact in f32
                s += (double) __fmul_rn(wf.y, xf.y);
            }
            acc[c] = s;
        }
    }
};

// ---------------------------------------------------------------------------------------------------------------
// The kernel: each warp walks a flat sequence of (row, unit batch) steps with a two-deep register pipeline.
// Without groups, CTAs split the N rows (grid.x); with groups (MUL_MAT_ID), grid.y is the expert and each CTA runs
// that expert's routed columns in chunks of NC against its slice of the expert's rows.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kGemvThreads = 256;

template <class T, int NC>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = (int64_t) gridDim.x * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t upr = T::units_per_row(p.w.K);
    const int64_t per_step = 32 * T::kUnroll;
    const int64_t steps_per_row = (upr + per_step - 1) / per_step;
    const int64_t my_rows = gwarp < p.N ? (p.N - gwarp + warps_total - 1) / warps_total : 0;
    const int64_t my_steps = my_rows * steps_per_row;
    const bool grouped = p.grp_off != nullptr;
    int64_t row0 = p.row0;

    typename T::Unit cur[T::kUnroll], nxt[T::kUnroll];
    auto load_step = [&](int64_t s, typename T::Unit * dst) {
        const int64_t r = gwarp + (s / steps_per_row) * warps_total;
        const int64_t u0 = (s % steps_per_row) * per_step;
#pragma unroll
        for (int i = 0; i < T::kUnroll; i++) {
            const int64_t u = u0 + i * 32 + lane;
            dst[i] = T::load(p.w, row0 + r, u, s < my_steps && u < upr);
        }
    };
    // Weight bytes depend on nothing: start streaming before waiting for the previous kernel. (With groups the
    // routing is the previous kernel's output, so the stream starts after the wait.)
    if (!grouped) load_step(0, cur);
    pdl_launch_dependents();
    pdl_wait();

    int64_t cbeg = 0, cend = p.ncols;
    if (grouped) {
        cbeg = p.grp_off[blockIdx.y];
        cend = p.grp_off[blockIdx.y + 1];
        row0 += (int64_t) blockIdx.y * p.grp_rows;
    }

    Act a;
    const int kind = act_kind(p.w.type);
    {
        const int64_t K = p.w.K;
        uint8_t * s = smem;
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
    float * xs = reinterpret_cast<float *>(smem + act_base_bytes(p.w.type, p.w.K, NC));
    const int nsums = T::sums_per_row(p.w.K);

    for (int64_t c0 = cbeg; c0 < cend; c0 += NC) {
        const int nc = (int) ((cend - c0) < NC ? (cend - c0) : NC);
        if (grouped || c0 != cbeg) {
            __syncthreads();  // the previous chunk's staging is no longer read
            load_step(0, cur);
        }
        if (NC == 1 && !p.aq && single_fast(a.K)) {
            stage_one(p, a, kind, nc > 0 ? column_src(p, c0) : p.x, xs, xs + 2 * a.K, blockDim.x);
        } else {
            stage_activations<NC>(p, a, kind, c0, nc, blockDim.x);
        }

        double acc[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) acc[c] = 0.0;
        for (int64_t s = 0; s < my_steps; s++) {
            if (s + 1 < my_steps) load_step(s + 1, nxt);
            const int64_t r = gwarp + (s / steps_per_row) * warps_total;
            const int64_t u0 = (s % steps_per_row) * per_step;
            int32_t * sums = p.sums ? p.sums + r * nsums : nullptr;
#pragma unroll
            for (int i = 0; i < T::kUnroll; i++) {
                const int64_t u = u0 + i * 32 + lane;
                T::template dot<NC>(cur[i], u, u < upr, a, acc, sums);
            }
            if (s % steps_per_row == steps_per_row - 1) {
#pragma unroll
                for (int c = 0; c < NC; c++) {
                    const float v = __double2float_rn(warp_sum_d(acc[c]));
                    if (lane == 0 && c < nc && !p.sums) {
                        const int64_t col = p.col_dst ? (int64_t) p.col_dst[c0 + c] : c0 + c;
                        float out = v;
                        if (p.res) out = __fadd_rn(p.res[col * p.ldres + r], v);
                        p.y[col * p.ldy + r] = out;
                    }
                    acc[c] = 0.0;
                }
            }
#pragma unroll
            for (int i = 0; i < T::kUnroll; i++) cur[i] = nxt[i];
        }
    }
}

}  // namespace b200
