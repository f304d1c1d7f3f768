// ops.cu — kernels of the non-GEMV ops and the GEMV launchers.
//
//  - repack_scatter / repack_gather: the weight buffer's set_tensor / get_tensor (src/common/model-file.cpp:247-268
//    uploads GGUF bytes in 16 MiB pieces at any offset). The repacked layout (common.cuh) is a byte permutation of the
//    GGUF bytes, so a piece maps byte by byte.
//  - get_rows: quantized GET_ROWS (src/families/qwen3-tts/talker.cpp:131-133, src/families/qwen3-asr/decoder.cpp:319),
//    dequantizing with the same float operations, in the same order, as the CPU dequantizers (bit-identical).
//  - quantize_act: the CPU backend's src1 quantization (q8_0 / q8_K), bit-identical to the oracle.
//  - route: MUL_MAT_ID's router sort (src/families/drama3/text-model.cpp:208-210): (token, slot) pairs grouped by
//    expert with a shared-memory histogram and scan, so each expert's rows stream once over all of its pairs.
#include "internal.h"
#include "gemv_tma.cuh"

#include <cstdlib>

namespace b200 {

// ------------------------------------------------------------------------------------------------------------------
// Layout
// ------------------------------------------------------------------------------------------------------------------
struct FieldOff {
    int64_t f[4];
};

__device__ __forceinline__ int64_t repacked_offset(int type, int64_t o, const FieldOff & fo) {
    switch (type) {
    case B200_TYPE_Q8_0: {
        const int64_t b = o / 34, w = o % 34;
        return w < 2 ? fo.f[1] + b * 2 + w : fo.f[0] + b * 32 + (w - 2);
    }
    case B200_TYPE_Q4_K: {
        const int64_t b = o / 144, w = o % 144;
        return w < 16 ? fo.f[1] + b * 16 + w : fo.f[0] + b * 128 + (w - 16);
    }
    case B200_TYPE_Q5_K: {  // d, dmin, scales (16 B) | qh (32 B) | qs (128 B)
        const int64_t b = o / 176, w = o % 176;
        if (w < 16) return fo.f[1] + b * 16 + w;
        if (w < 48) return fo.f[2] + b * 32 + (w - 16);
        return fo.f[0] + b * 128 + (w - 48);
    }
    case B200_TYPE_Q6_K: {
        const int64_t b = o / 210, w = o % 210;
        if (w < 128) return fo.f[0] + b * 128 + w;
        if (w < 192) return fo.f[1] + b * 64 + (w - 128);
        if (w < 208) return fo.f[2] + b * 16 + (w - 192);
        return fo.f[3] + b * 2 + (w - 208);
    }
    default: return o;
    }
}

__global__ void repack_kernel(int type, FieldOff fo, const uint8_t * __restrict__ src, int64_t off0, int64_t n,
                              uint8_t * __restrict__ dev, uint8_t * __restrict__ gather_dst) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t d = repacked_offset(type, off0 + i, fo);
        if (gather_dst) gather_dst[i] = dev[d];
        else dev[d] = src[i];
    }
}

cudaError_t launch_repack(int type, const b200_weight * w, const uint8_t * src, int64_t off0, int64_t n, bool to_device_layout,
                          uint8_t * gather_dst, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    FieldOff fo;
    for (int i = 0; i < 4; i++) fo.f[i] = w->field_off[i];
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads < 148 * 16 ? (n + threads - 1) / threads : 148 * 16;
    repack_kernel<<<(unsigned) blocks, threads, 0, st>>>(type, fo, src, off0, n, (uint8_t *) w->data,
                                                          to_device_layout ? nullptr : gather_dst);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// L2 prefetch of a byte range (a weight that the next kernels will read): each thread asks L2 for one 64 KB piece with
// one bulk prefetch and the kernel ends; nothing waits for the data.
// ------------------------------------------------------------------------------------------------------------------
__global__ void prefetch_l2_kernel(const uint8_t * base, size_t bytes) {
    constexpr size_t kPiece = 64 * 1024;
    const size_t n = (bytes + kPiece - 1) / kPiece;
    for (size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        const size_t off = i * kPiece;
        const uint32_t sz = (uint32_t) ((bytes - off < kPiece ? bytes - off : kPiece) & ~(size_t) 15);
        if (sz) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(sz) : "memory");
    }
}

cudaError_t launch_prefetch_l2(const void * base, size_t bytes, cudaStream_t st) {
    if (!bytes) return cudaSuccess;
    const size_t pieces = (bytes + 65535) / 65536;
    const unsigned blocks = (unsigned) ((pieces + 255) / 256 < 1024 ? (pieces + 255) / 256 : 1024);
    prefetch_l2_kernel<<<blocks, 256, 0, st>>>((const uint8_t *) base, bytes);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// GET_ROWS
// ------------------------------------------------------------------------------------------------------------------
__global__ void get_rows_kernel(WeightView w, const int32_t * __restrict__ ids, float * __restrict__ dst, unsigned * err) {
    const int64_t i = blockIdx.x;
    const int64_t r = ids[i];
    if (r < 0 || r >= w.rows) {
        if (threadIdx.x == 0) atomicOr(err, B200_DEVERR_ROWS);
        return;
    }
    const int64_t K = w.K;
    float * out = dst + i * K;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
        float v;
        switch (w.type) {
        case B200_TYPE_Q8_0: {
            const float d = __half2float(__ushort_as_half(reinterpret_cast<const uint16_t *>(w.f1)[r * (K / 32) + k / 32]));
            v = __fmul_rn((float) reinterpret_cast<const int8_t *>(w.f0)[r * K + k], d);
            break;
        }
        case B200_TYPE_Q4_K: {
            const int64_t sb = k / 256;
            const int s = (int) ((k % 256) / 32), l = (int) (k % 32);
            const uint8_t * meta = w.f1 + (r * (K / 256) + sb) * 16;
            const int q = (w.f0[r * (K / 2) + sb * 128 + (s >> 1) * 32 + l] >> ((s & 1) * 4)) & 15;
            int sc, m;
            TQ4_K::scale_min(meta + 4, s, sc, m);
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(meta)));
            const float dmin = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(meta + 2)));
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float) sc), (float) q), __fmul_rn(dmin, (float) m));
            break;
        }
        case B200_TYPE_Q5_K: {
            const int64_t sb = k / 256;
            const int s = (int) ((k % 256) / 32), l = (int) (k % 32);
            const uint8_t * meta = w.f1 + (r * (K / 256) + sb) * 16;
            const int q = ((w.f0[r * (K / 2) + sb * 128 + (s >> 1) * 32 + l] >> ((s & 1) * 4)) & 15) |
                          (((w.f2[r * (K / 8) + sb * 32 + l] >> s) & 1) << 4);
            int sc, m;
            TQ4_K::scale_min(meta + 4, s, sc, m);
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(meta)));
            const float dmin = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(meta + 2)));
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float) sc), (float) q), __fmul_rn(dmin, (float) m));
            break;
        }
        case B200_TYPE_Q6_K: {
            const int64_t sb = k / 256;
            const int vv = (int) (k % 256), h = vv >> 7, t = (vv >> 5) & 3, l = vv & 31;
            const int lo = (w.f0[r * (K / 2) + sb * 128 + h * 64 + (t & 1) * 32 + l] >> ((t >> 1) * 4)) & 15;
            const int hi = (w.f1[r * (K / 4) + sb * 64 + h * 32 + l] >> (2 * t)) & 3;
            const int q = (lo | (hi << 4)) - 32;
            const int sc = reinterpret_cast<const int8_t *>(w.f2)[(r * (K / 256) + sb) * 16 + vv / 16];
            const float d = __half2float(__ushort_as_half(reinterpret_cast<const uint16_t *>(w.f3)[r * (K / 256) + sb]));
            v = __fmul_rn(__fmul_rn(d, (float) sc), (float) q);
            break;
        }
        case B200_TYPE_BF16:
            v = __uint_as_float((unsigned) reinterpret_cast<const uint16_t *>(w.f0)[r * K + k] << 16);
            break;
        default:
            v = reinterpret_cast<const float *>(w.f0)[r * K + k];
            break;
        }
        out[k] = v;
    }
}

cudaError_t launch_get_rows(const WeightView & w, const int32_t * ids, int64_t n, float * dst, unsigned * err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    get_rows_kernel<<<(unsigned) n, 256, 0, st>>>(w, ids, dst, err);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// Activation quantization (one warp per block)
// ------------------------------------------------------------------------------------------------------------------
__global__ void quantize_act_kernel(int kind, const float * __restrict__ x, int64_t K, int64_t M, uint8_t * gguf, int8_t * q,
                                    float * d, int16_t * bs, int64_t dT_ld) {
    // launched with programmatic dependent launch: x is read after the previous kernel's writes are visible; the next
    // kernel (a tensor-core product streaming its weights) may start now
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    const int64_t bsz = kind == B200_TYPE_Q8_0 ? 32 : 256;
    const int64_t nb = K / bsz;
    for (int64_t i = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < M * nb; i += warps) {
        const int64_t r = i / nb, b = i % nb;
        const float * xb = x + r * K + b * bsz;
        if (kind == B200_TYPE_Q8_0) {
            float df;
            uint16_t dh;
            const int8_t qv = quantize_q8_0_lane(xb[lane], &df, &dh);
            if (gguf) {
                uint8_t * blk = gguf + i * 34;
                blk[2 + lane] = (uint8_t) qv;
                if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = dh;
            } else {
                q[r * K + b * 32 + lane] = qv;
                if (lane == 0) {
                    if (dT_ld) d[b * dT_ld + r] = df;  // transposed: [K/32][dT_ld]
                    else d[i] = df;
                }
            }
        } else {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = xb[lane * 8 + j];
            int8_t qv[8];
            int16_t bsum;
            float df;
            quantize_q8_K_warp(v, qv, &bsum, &df);
            if (gguf) {
                uint8_t * blk = gguf + i * 292;
#pragma unroll
                for (int j = 0; j < 8; j++) blk[4 + lane * 8 + j] = (uint8_t) qv[j];
                if ((lane & 1) == 0) reinterpret_cast<int16_t *>(blk + 260)[lane / 2] = bsum;
                if (lane == 0) *reinterpret_cast<float *>(blk) = df;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) q[r * K + b * 256 + lane * 8 + j] = qv[j];
                if ((lane & 1) == 0) bs[r * (K / 16) + b * 16 + lane / 2] = bsum;
                if (lane == 0) d[i] = df;
            }
        }
    }
}

cudaError_t launch_quantize(int kind, const float * x, int64_t K, int64_t M, uint8_t * gguf, int8_t * q, float * d, int16_t * bs,
                            cudaStream_t st, int64_t dT_ld) {
    const int64_t nb = M * (K / (kind == B200_TYPE_Q8_0 ? 32 : 256));
    if (nb <= 0) return cudaSuccess;
    const int threads = 256;
    int64_t blocks = (nb + 7) / 8;
    if (blocks > 148 * 8) blocks = 148 * 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) blocks, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quantize_act_kernel, kind, x, K, M, gguf, q, d, bs, dT_ld);
}

// ------------------------------------------------------------------------------------------------------------------
// MUL_MAT_ID routing: one CTA histograms the expert ids, scans, and places each (token, slot) pair in its expert's
// segment. Pairs of one expert are independent products, so the order inside a segment does not change any result.
// ------------------------------------------------------------------------------------------------------------------
// With expert sharding (expert parallelism), this GPU holds experts [e0, e0 + E) of `total`: pairs routed to other
// GPUs' experts are skipped; only ids outside [0, total) are errors. col_tok (optional) receives each pair's token.
__global__ void route_kernel(const int32_t * __restrict__ ids, int64_t P, int64_t top_k, int64_t nb1, int E, int e0, int total,
                             int32_t * grp_off, int32_t * col_src, int32_t * col_dst, int32_t * col_tok, unsigned * err) {
    extern __shared__ int cnt[];  // [E] counts, then [E] cursors
    int * pos = cnt + E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
        const int g = ids[p];
        if (g < 0 || g >= total) {
            atomicOr(err, B200_DEVERR_EXPERT);
            continue;
        }
        const int e = g - e0;
        if (e < 0 || e >= E) continue;
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        // warp-parallel exclusive scan over E counts, 32 at a time
        int carry = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + (int) threadIdx.x;
            const int v = e < E ? cnt[e] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if ((int) threadIdx.x >= o) incl += t;
            }
            if (e < E) {
                grp_off[e] = carry + incl - v;
                pos[e] = carry + incl - v;
            }
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (threadIdx.x == 0) grp_off[E] = carry;
    }
    __syncthreads();
    for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
        const int e = ids[p] - e0;
        if (ids[p] < 0 || ids[p] >= total || e < 0 || e >= E) continue;
        const int slot = atomicAdd(&pos[e], 1);
        const int64_t t = p / top_k, s = p % top_k;
        col_src[slot] = (int32_t) (t * nb1 + (nb1 == 1 ? 0 : s));
        col_dst[slot] = (int32_t) p;
        if (col_tok) col_tok[slot] = (int32_t) t;
    }
}

cudaError_t launch_route(const int32_t * ids, int64_t T, int64_t top_k, int64_t nb1, int64_t E, int32_t * grp_off,
                         int32_t * col_src, int32_t * col_dst, unsigned * err, cudaStream_t st, int64_t e0, int64_t total,
                         int32_t * col_tok) {
    route_kernel<<<1, 1024, (size_t) 2 * E * sizeof(int), st>>>(ids, T * top_k, top_k, nb1, (int) E, (int) e0,
                                                                 (int) (total > 0 ? total : E), grp_off, col_src, col_dst, col_tok, err);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// MoE glue (TextModel::experts, src/families/drama3/text-model.cpp:198-221): SwiGLU of each routed pair's gate|up row,
// quantized to q8_0 for the down product; and the router-weighted sum of a token's down rows, in slot order.
// ------------------------------------------------------------------------------------------------------------------
__global__ void swiglu_quant_pairs_kernel(const float * __restrict__ gu, int64_t F, const int32_t * __restrict__ col_dst,
                                          const int32_t * __restrict__ n_pairs, int8_t * q, float * d) {
    // one warp per (pair slot, 32-block); pairs come in routed order, their rows are the pair index p
    const int lane = threadIdx.x & 31;
    const int64_t nb = F / 32;
    const int64_t total = (int64_t) (*n_pairs) * nb;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += warps) {
        const int64_t p = col_dst[i / nb], b = i % nb;
        const float * row = gu + p * 2 * F;
        const float v = __fmul_rn(silu(row[b * 32 + lane]), row[F + b * 32 + lane]);
        float df;
        uint16_t dh;
        const int8_t qv = quantize_q8_0_lane(v, &df, &dh);
        q[p * F + b * 32 + lane] = qv;
        if (lane == 0) d[p * nb + b] = df;
    }
}

// The same for K-quant down experts: q8_K of each pair's SwiGLU row, one warp per (pair slot, 256-block), as
// quantize_act_kernel lays q8_K out (q [rows][F], d [rows][F/256], bs [rows][F/16]); bit-identical to
// quantize_row_q8_K of the SwiGLU row.
__global__ void swiglu_quant_pairs_k_kernel(const float * __restrict__ gu, int64_t F, const int32_t * __restrict__ col_dst,
                                            const int32_t * __restrict__ n_pairs, int8_t * q, float * d, int16_t * bs) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = F / 256;
    const int64_t total = (int64_t) (*n_pairs) * nb;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += warps) {
        const int64_t p = col_dst[i / nb], b = i % nb;
        const float * row = gu + p * 2 * F + b * 256 + lane * 8;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = __fmul_rn(silu(row[j]), row[F + j]);
        int8_t qv[8];
        int16_t bsum;
        float df;
        quantize_q8_K_warp(v, qv, &bsum, &df);
#pragma unroll
        for (int j = 0; j < 8; j++) q[p * F + b * 256 + lane * 8 + j] = qv[j];
        if ((lane & 1) == 0) bs[p * (F / 16) + b * 16 + lane / 2] = bsum;
        if (lane == 0) d[p * nb + b] = df;
    }
}

__global__ void moe_combine_kernel(const float * __restrict__ down, const float * __restrict__ w, const int32_t * __restrict__ ids,
                                   int64_t top_k, int64_t H, int e0, int E, float * __restrict__ out) {
    const int64_t t = blockIdx.x;
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
        float sum = 0.0f;
        bool any = false;
        for (int64_t s = 0; s < top_k; s++) {
            const int e = ids[t * top_k + s] - e0;
            if (e < 0 || e >= E) continue;
            const float v = __fmul_rn(down[(t * top_k + s) * H + h], w[t * top_k + s]);
            sum = any ? __fadd_rn(sum, v) : v;
            any = true;
        }
        out[t * H + h] = sum;
    }
}

cudaError_t launch_swiglu_quant_pairs(const float * gu, int64_t F, const int32_t * col_dst, const int32_t * n_pairs, int64_t max_pairs,
                                      int8_t * q, float * d, cudaStream_t st) {
    int64_t blocks = (max_pairs * (F / 32) + 7) / 8;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    swiglu_quant_pairs_kernel<<<(unsigned) blocks, 256, 0, st>>>(gu, F, col_dst, n_pairs, q, d);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_quant_pairs_k(const float * gu, int64_t F, const int32_t * col_dst, const int32_t * n_pairs, int64_t max_pairs,
                                        int8_t * q, float * d, int16_t * bs, cudaStream_t st) {
    int64_t blocks = (max_pairs * (F / 256) + 7) / 8;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    swiglu_quant_pairs_k_kernel<<<(unsigned) blocks, 256, 0, st>>>(gu, F, col_dst, n_pairs, q, d, bs);
    return cudaGetLastError();
}

cudaError_t launch_moe_combine(const float * down, const float * w, const int32_t * ids, int64_t T, int64_t top_k, int64_t H, int64_t e0,
                               int64_t E, float * out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    moe_combine_kernel<<<(unsigned) T, 256, 0, st>>>(down, w, ids, top_k, H, (int) e0, (int) E, out);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// GEMV launchers
// ------------------------------------------------------------------------------------------------------------------
template <class T, int NC>
static cudaError_t launch_one(const GemvParams & p, int grid_y, cudaStream_t st, bool pdl, int num_sms, int cap_per_sm) {
    auto kern = gemv_kernel<T, NC>;
    const size_t smem = act_smem_bytes(p.w.type, p.w.K, NC);
    static int configured_smem = 0;  // per instantiation
    static int ctas_per_sm = 0;
    if ((int) smem > configured_smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return e;
        configured_smem = (int) smem;
        ctas_per_sm = 0;
    }
    if (ctas_per_sm == 0) {
        int n = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGemvThreads, configured_smem);
        if (e != cudaSuccess) return e;
        ctas_per_sm = n > 0 ? n : 1;
    }
    const int warps_per_cta = kGemvThreads / 32;
    // expert groups: 64 rows per CTA, so one staging of an expert's activation columns serves many weight rows
    const int rows_per_cta = grid_y > 1 ? 64 : warps_per_cta;
    int64_t gx = (p.N + rows_per_cta - 1) / rows_per_cta;
    const int capped = cap_per_sm >= 3 ? 2 : cap_per_sm;  // (cap 3 is the TMA path's one-CTA-per-SM form of cap 2)
    const int per_sm = capped > 0 && capped < ctas_per_sm ? capped : ctas_per_sm;
    const int64_t cap = grid_y > 1 ? gx : (int64_t) num_sms * per_sm;
    if (gx > cap) gx = cap;
    if (gx < 1) gx = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) gx, (unsigned) grid_y, 1);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// TMA-streamed launch (gemv_tma.cuh): grid and ring geometry.
template <class T, int NC, int CW>
static cudaError_t launch_tma_cw(const GemvParams & p, int64_t gx, size_t smem, cudaStream_t st, bool pdl) {
    auto kern = gemv_tma_kernel<T, NC, CW>;
    static int configured = 0;
    if ((int) smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess) return e;
        configured = 220 * 1024;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) gx, 1, 1);
    cfg.blockDim = dim3(32 * (CW + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <class T, int NC>
static cudaError_t launch_tma(const GemvParams & p0, cudaStream_t st, bool pdl, int num_sms, int cap_per_sm) {
    GemvParams p = p0;
    const int64_t K = p.w.K;
    const int64_t row_bytes = tma_row_bytes<T>(K);
    static const int env_cta0 = [] { const char * e = getenv("B200_TMA_CTAS_PER_SM"); return e ? atoi(e) : 1; }();
    // a caller's cap (a chain of products wants two CTAs per SM, so the next product's CTA fits beside the running
    // one) wins over the default of one CTA per SM with the large ring
    // (cap 3: one CTA per SM with the two-CTA ring and 8 consumer warps, the other half of each SM left to the next
    // launch; measured 5 % faster than two CTAs per SM on chains of 3.3 MB products)
    const int per_sm = cap_per_sm > 0 ? (cap_per_sm < 2 ? cap_per_sm : 2) : env_cta0;
    const int grid_per_sm = cap_per_sm >= 3 ? 1 : per_sm;
    int64_t gx = (int64_t) num_sms * grid_per_sm;
    if (gx > p.N) gx = p.N;
    if (gx < 1) gx = 1;
    int64_t rpc = (p.N + gx - 1) / gx;
    gx = (p.N + rpc - 1) / rpc;
    // Ring geometry: 8 stages (one chunk in flight per consumer warp) of ring / 8 bytes; measured on B200 with large
    // Q8_0 / Q4_K / Q6_K products, a 192 KB ring of 24 KB stages at one CTA per SM streamed fastest.
    // B200_TMA_RING_KB / B200_TMA_STAGES / B200_TMA_CTAS_PER_SM override it: the ring-geometry tests run other
    // shapes through these (results must not change with the geometry).
    static const int64_t env_ring = [] { const char * e = getenv("B200_TMA_RING_KB"); return e ? atoll(e) * 1024 : 0; }();
    static const int64_t env_stages = [] { const char * e = getenv("B200_TMA_STAGES"); return e ? atoll(e) : 8; }();
    const size_t act = act_smem_bytes(p.w.type, K, NC) + 256;
    int64_t ring_budget = env_ring > 0 ? env_ring : (per_sm >= 2 ? 96 * 1024 : 192 * 1024);
    if ((int64_t) (ring_budget + act) > 220 * 1024) ring_budget = 220 * 1024 - (int64_t) act;
    const int64_t max_stages = env_stages < 1 ? 1 : env_stages;
    int64_t rps = (ring_budget / max_stages) / row_bytes;
    if (rps < 1) rps = 1;
    if (rps > rpc) rps = rpc;
    int64_t stages = ring_budget / (rps * row_bytes);
    const int64_t chunks = (rpc + rps - 1) / rps;
    if (stages > chunks) stages = chunks;
    if (stages > max_stages) stages = max_stages;
    if (stages < 1) stages = 1;
    // each slot must belong to one consumer warp: a multiple of the 8 warps, or fewer slots than warps
    if (stages > kTmaConsumerWarps) stages -= stages % kTmaConsumerWarps;
    p.rows_per_cta = (int) rpc;
    p.rows_per_stage = (int) rps;
    p.stages = (int) stages;
    const size_t smem = tma_smem_bytes<T, NC>(p.w.type, K, (int) rps, (int) stages);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    // one CTA per SM: 16 consumer warps (single column; measured faster for the large HBM-bound products);
    // B200_TMA_WARPS=8 keeps 8 (the geometry tests' other form)
    static const int env_warps = [] { const char * e = getenv("B200_TMA_WARPS"); return e ? atoi(e) : 16; }();
    if constexpr (NC == 1) {
        if (per_sm == 1 && env_warps == 16) return launch_tma_cw<T, NC, 2 * kTmaConsumerWarps>(p, gx, smem, st, pdl);
    }
    return launch_tma_cw<T, NC, kTmaConsumerWarps>(p, gx, smem, st, pdl);
}

template <class T, int NC>
static cudaError_t launch_pick(const GemvParams & p, int grid_y, cudaStream_t st, bool pdl, int num_sms, int cap) {
    // the TMA path needs whole 16-byte field rows, no expert groups, and its geometry must fit shared memory
    if (p.grp_off == nullptr && grid_y == 1 && p.err && tma_fits<T>(p.w.K) && tma_row_bytes<T>(p.w.K) <= 64 * 1024 &&
        p.ncols <= NC) {
        const cudaError_t e = launch_tma<T, NC>(p, st, pdl, num_sms, cap);
        if (e != cudaErrorInvalidValue) return e;
    }
    return launch_one<T, NC>(p, grid_y, st, pdl, num_sms, cap);
}

template <class T>
static cudaError_t launch_nc(const GemvParams & p, int nc, int grid_y, cudaStream_t st, bool pdl, int num_sms, int cap) {
    switch (nc) {
    case 1: return launch_pick<T, 1>(p, grid_y, st, pdl, num_sms, cap);
    case 2: return launch_pick<T, 2>(p, grid_y, st, pdl, num_sms, cap);
    case 4: return launch_pick<T, 4>(p, grid_y, st, pdl, num_sms, cap);
    case 8: return launch_pick<T, 8>(p, grid_y, st, pdl, num_sms, cap);
    case 16: return launch_pick<T, 16>(p, grid_y, st, pdl, num_sms, cap);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(const GemvParams & p, int nc, int grid_y, cudaStream_t st, bool pdl, int num_sms, int ctas_per_sm) {
    switch (p.w.type) {
    case B200_TYPE_Q8_0: return launch_nc<TQ8_0>(p, nc, grid_y, st, pdl, num_sms, ctas_per_sm);
    case B200_TYPE_Q4_K: return launch_nc<TQ4_K>(p, nc, grid_y, st, pdl, num_sms, ctas_per_sm);
    case B200_TYPE_Q5_K: return launch_nc<TQ5_K>(p, nc, grid_y, st, pdl, num_sms, ctas_per_sm);
    case B200_TYPE_Q6_K: return launch_nc<TQ6_K>(p, nc, grid_y, st, pdl, num_sms, ctas_per_sm);
    case B200_TYPE_BF16: return launch_nc<TBF16>(p, nc, grid_y, st, pdl, num_sms, ctas_per_sm);
    default: return cudaErrorInvalidValue;
    }
}

int gemv_max_columns(int wtype, int64_t K) {
    const size_t limit = 200 * 1024;
    for (int nc = 16; nc >= 1; nc >>= 1)
        if (act_smem_bytes(wtype, K, nc) <= limit) return nc;
    return 0;
}

}  // namespace b200
