// gemm_kq_tc.cu — Q4_K and Q6_K products with many activation rows (prefill) on the int8 tensor cores.
//
// ggml's CPU backend multiplies K-quant weights by q8_K activations (one float scale per 256 values, int8 values,
// int16 sums of 16) with exact integer sums per super-block of 256:
//   Q4_K: sumi = sum_s sc_s * (sum_l q_l x_l) and summ = sum_s m_s * (bsum_2s + bsum_2s+1) over the 8 sub-blocks s of
//         32 (q in 0..15, six-bit scale sc and min m), then sumf += (dx * d) * sumi - (dx * dmin) * summ;
//   Q6_K: sumi = sum_g sc_g * (sum_l (q_l - 32) x_l) over the 16 groups g of 16 (int8 scales), then
//         sumf += (d * dx) * sumi.
// Here the same integers come from the tensor cores. Each weight matrix is expanded once (on the first product with
// many rows; cached until the weight is written or freed) into int8 planes that carry the integer scales, because a
// scale times a quant does not fit int8 but the scale's digits do:
//   Q4_K: three planes, sc = 8 a + b (a, b <= 7): a * q, b * q and the min m at every value;
//         sumi = 8 A0 + A1 and summ = A2;
//   Q6_K: four planes, sc = e0 + 5 e1 + 25 e2 + 125 e3 (balanced base 5, e in -2..2): e_k * (q - 32);
//         sumi = A0 + 5 A1 + 25 A2 + 125 A3,
// where A_k is plane k's accumulator over a whole 256-value super-block: one tcgen05.mma kind::i8 per plane per
// 32-value block (M = 128 weight rows x N = 64 tokens x K = 32) accumulates in tensor memory, and the epilogue runs
// once per super-block, converting to float in super-block order (ggml's float steps). Warp 0 = TMA producer (no
// multicast), warp 1 = tensor-memory allocator and MMA issuer, warps 2..9 = epilogue; one CTA per SM with 512
// tensor-memory columns (two super-block buffers) and three shared-memory stages; every wait bounded.
#include <unordered_map>

#include "internal.h"
#include "tcgen05.cuh"

namespace b200 {

// ------------------------------------------------------------------------------------------------------------------
// Expansion
// ------------------------------------------------------------------------------------------------------------------
// Q4_K: three int8 planes q [3][rows][K] and dd float4 [rows][K/256] (d, dmin, 0, 0). With the sub-block's six-bit
// scale written in base 8, sc = 8 a + b (a, b <= 7), plane 0 holds a * q, plane 1 b * q (q the nibble, 0..15; both
// <= 105) and plane 2 the sub-block's min m (<= 63) at every value: over a super-block, 8 (plane 0 . x) + (plane 1 . x)
// is ggml's sumi = sum_s sc_s sum_l q_l x_l and (plane 2 . x) its summ = sum_s m_s sum_l x_l, exactly.
__global__ void expand_q4k_kernel(WeightView w, int8_t * q, float4 * dd) {
    const int lane = threadIdx.x & 31;
    const int64_t nsb = w.K / 256, total = w.rows * nsb, plane = w.rows * w.K;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += warps) {
        const int64_t r = i / nsb, sb = i % nsb;
        const uint8_t * qs = w.f0 + r * (w.K / 2) + sb * 128;
        const uint8_t * meta = w.f1 + (r * nsb + sb) * 16;  // d, dmin (fp16), 12 scale bytes
        const int s = lane >> 2, l0 = (lane & 3) * 8;  // this lane: values 8 lane .. 8 lane + 7 = sub-block s, l0..
        const uint8_t * src = qs + (s >> 1) * 32 + l0;
        const int shift = (s & 1) * 4;
        int sc, m;
        TQ4_K::scale_min(meta + 4, s, sc, m);
        const uint32_t da = (uint32_t) (sc >> 3), db = (uint32_t) (sc & 7);
        uint32_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t n0 = (src[j] >> shift) & 15, n1 = (src[4 + j] >> shift) & 15;
            a0 |= (da * n0) << (8 * j);
            a1 |= (da * n1) << (8 * j);
            b0 |= (db * n0) << (8 * j);
            b1 |= (db * n1) << (8 * j);
        }
        const uint32_t mm = (uint32_t) m * 0x01010101u;
        int8_t * dst = q + r * w.K + sb * 256 + lane * 8;
        *reinterpret_cast<uint2 *>(dst) = make_uint2(a0, a1);
        *reinterpret_cast<uint2 *>(dst + plane) = make_uint2(b0, b1);
        *reinterpret_cast<uint2 *>(dst + 2 * plane) = make_uint2(mm, mm);
        if (lane == 0) {
            const float d = __half2float(*reinterpret_cast<const __half *>(meta));
            const float dmin = __half2float(*reinterpret_cast<const __half *>(meta + 2));
            dd[r * nsb + sb] = make_float4(d, dmin, 0.0f, 0.0f);
        }
    }
}

// Q6_K: four int8 planes q [4][rows][K] and dd float4 [rows][K/256] (d, 0, 0, 0). The 16-value group's int8 scale is
// written in balanced base 5, sc = e0 + 5 e1 + 25 e2 + 125 e3 with every e in -2..2, and plane k holds e_k * (q - 32)
// (|.| <= 64): over a super-block, (plane 0 . x) + 5 (plane 1 . x) + 25 (plane 2 . x) + 125 (plane 3 . x) is ggml's
// sumi = sum_g sc_g sum_l (q_l - 32) x_l, exactly.
__global__ void expand_q6k_kernel(WeightView w, int8_t * q, float4 * dd) {
    const int lane = threadIdx.x & 31;
    const int64_t nsb = w.K / 256, total = w.rows * nsb, plane = w.rows * w.K;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += warps) {
        const int64_t r = i / nsb, sb = i % nsb;
        const uint8_t * ql = w.f0 + r * (w.K / 2) + sb * 128;
        const uint8_t * qh = w.f1 + r * (w.K / 4) + sb * 64;
        // this lane: values v = 8 lane .. 8 lane + 7 of the super-block: half hh, quarter t, positions l0 .. l0 + 7
        const int v0 = 8 * lane, hh = v0 >> 7, t = (v0 >> 5) & 3, l0 = v0 & 31;
        int sc = (int) reinterpret_cast<const int8_t *>(w.f2)[r * (w.K / 16) + sb * 16 + (v0 >> 4)];
        int e[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int d = ((sc % 5) + 5) % 5;  // 0..4
            if (d > 2) d -= 5;           // -2..2
            e[k] = d;
            sc = (sc - d) / 5;
        }
        uint32_t out[4][2] = {};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int l = l0 + j;
            const int lo4 = (ql[hh * 64 + (t & 1) * 32 + l] >> ((t >> 1) * 4)) & 15;
            const int hi2 = (qh[hh * 32 + l] >> (2 * t)) & 3;
            const int qv = (lo4 | (hi2 << 4)) - 32;
#pragma unroll
            for (int k = 0; k < 4; k++) out[k][j >> 2] |= (uint32_t) (uint8_t) (int8_t) (e[k] * qv) << (8 * (j & 3));
        }
        int8_t * dst = q + r * w.K + sb * 256 + v0;
#pragma unroll
        for (int k = 0; k < 4; k++) *reinterpret_cast<uint2 *>(dst + k * plane) = make_uint2(out[k][0], out[k][1]);
        if (lane == 0) dd[r * nsb + sb] = make_float4(__half2float(reinterpret_cast<const __half *>(w.f3)[r * nsb + sb]), 0.0f, 0.0f, 0.0f);
    }
}

// q8_K of M activation rows for the tensor-core products: q int8 [M][K], dxT float [K/256][ld] (transposed scales;
// the block sums that q8_K also carries are not needed: Q4_K's min term comes from its m plane). One warp per
// 256-block; bit-identical to quantize_row_q8_K.
__global__ void quantize_q8k_tc_kernel(const float * __restrict__ x, int64_t K, int64_t M, int8_t * q, float * dxT, int64_t ld) {
    const int lane = threadIdx.x & 31;
    const int64_t nsb = K / 256;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t i = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < M * nsb; i += warps) {
        const int64_t m = i / nsb, sb = i % nsb;
        const float * xb = x + m * K + sb * 256 + lane * 8;
        const float4 a = *reinterpret_cast<const float4 *>(xb), c = *reinterpret_cast<const float4 *>(xb + 4);
        const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
        int8_t qv[8];
        int16_t bsum;
        float df;
        quantize_q8_K_warp(v, qv, &bsum, &df);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            lo |= (uint32_t) (uint8_t) qv[j] << (8 * j);
            hi |= (uint32_t) (uint8_t) qv[4 + j] << (8 * j);
        }
        *reinterpret_cast<uint2 *>(q + m * K + sb * 256 + lane * 8) = make_uint2(lo, hi);
        if (lane == 0) dxT[sb * ld + m] = df;
    }
}

namespace {

constexpr int kQM = 128;       // weight rows per tile
constexpr int kQNT = 64;       // tokens per tile
constexpr int kQKB = 4;        // 32-value blocks per stage
constexpr int kQThreads = 320; // producer, MMA, 8 epilogue warps
constexpr int kQEpiWarps = 8;
constexpr int kQTmemCols = 512; // tensor memory of the one CTA per SM: two super-block buffers of planes x kQNT
constexpr unsigned kErrTimeout = 4u;

template <int KIND>
struct KqLayout {
    static constexpr int kPlanes = KIND == 6 ? 4 : 3;      // expansion planes = accumulators per super-block
    static constexpr int kA = kPlanes * kQM * 128;        // A tiles ([128 rows][128 B], swizzled), one per plane
    static constexpr int kB = kQKB * kQNT * 32;            // activations: [64 rows][128 B] swizzled
    static constexpr int kDd = kQM * 16;                   // float4 (d, dmin) per row
    static constexpr int kDx = kQNT * 4;                   // the super-block's activation scales
    static constexpr int kStage = (kA + kB + kDd + kDx + 1023) & ~1023;
    static constexpr int kStages = 3;
    static constexpr int kCtasPerSm = 1;
    static constexpr int kTotal = kStages * kStage + 1024 + 256;  // + alignment slack + barriers
    static_assert(2 * kPlanes * kQNT <= kQTmemCols, "two super-block buffers fit the tensor-memory allocation");
    static_assert(kTotal + 64 <= 227 * 1024, "shared memory of one CTA");
};

struct KqParams {
    int64_t N, K, row0;
    int64_t plane_rows;  // rows of one expansion plane (the weight's rows)
    int M;
    int tiles_m, tiles_n;
    float * y;
    int64_t ldy;
    unsigned * err;
};

// ggml's super-block integers from the accumulators A of the expansion planes (see the expansion kernels).
template <int KIND>
__device__ __forceinline__ void kq_combine(int (*A)[16], int i, int & sumi, int & summ) {
    if (KIND == 4) {
        sumi = 8 * A[0][i] + A[1][i];
        summ = A[2][i];
    } else {
        sumi = A[0][i] + 5 * A[1][i] + 25 * A[2][i] + 125 * A[3][i];
        summ = 0;
    }
}

template <int KIND>
__global__ void __launch_bounds__(kQThreads, KqLayout<KIND>::kCtasPerSm)
    gemm_kq_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmDd, const __grid_constant__ CUtensorMap tmDx, KqParams p) {
    using L = KqLayout<KIND>;
    constexpr int S = L::kStages, P = L::kPlanes;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint64_t * bars = reinterpret_cast<uint64_t *>(smem + S * L::kStage);
    uint64_t * full = bars;
    uint64_t * empty = bars + S;
    uint64_t * acc_full = bars + 2 * S;
    uint64_t * acc_empty = acc_full + 2;
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    __shared__ volatile int give_up;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nstage = (int) (p.K / 32 / kQKB);  // two per super-block
    const int items = p.tiles_m * p.tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kQEpiWarps);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kQEpiWarps);
        }
        fence_mbar_init();
        give_up = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)), "r"(kQTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // item -> (token tile, row tile): consecutive items share a weight tile (its 128 rows come from L2 for the
    // other token tiles)
    auto tile_of = [&](int it, int & m0, int & nz, int & live, int & tn) {
        const int tm = it % p.tiles_m;
        tn = it / p.tiles_m;
        m0 = tm * kQNT;
        live = p.M - m0 < kQNT ? p.M - m0 : kQNT;
        nz = (live + 15) & ~15;
    };

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            int sg = 0;
            for (int it = blockIdx.x; it < items && !give_up; it += gridDim.x) {
                int m0, nz, live, tn;
                tile_of(it, m0, nz, live, tn);
                const int arow = (int) (p.row0 + (int64_t) tn * kQM);
                const uint32_t bytes = (uint32_t) (L::kA + nz * 128 + L::kDd + L::kDx);
                for (int st = 0; st < nstage; st++, sg++) {
                    const int s = sg % S, use = sg / S;
                    if (use > 0 && !mbar_wait_sleep(&empty[s], (use - 1) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    uint8_t * base = smem + s * L::kStage;
                    mbar_arrive_expect_tx(&full[s], bytes);
                    const int kbs = st * kQKB;  // first 32-value block of the stage
                    for (int pl = 0; pl < P; pl++)
                        tma_load_2d(base + pl * kQM * 128, &tmA, kbs * 32, (int) (pl * p.plane_rows) + arow, &full[s]);
                    for (int r = 0; r < nz / 16; r++) tma_load_2d(base + L::kA + r * 16 * 128, &tmB, kbs * 32, m0 + 16 * r, &full[s]);
                    uint8_t * dd = base + L::kA + L::kB;
                    tma_load_2d(dd, &tmDd, 4 * (kbs / 8), arow, &full[s]);
                    tma_load_2d(dd + L::kDd, &tmDx, m0, kbs / 8, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: a super-block is two stages; its P accumulators take one buffer of P x 32 columns ----
        if (lane == 0) {
            int sg = 0, g2 = 0;
            for (int it = blockIdx.x; it < items && !give_up; it += gridDim.x) {
                int m0, nz, live, tn;
                tile_of(it, m0, nz, live, tn);
                const uint32_t idesc = idesc_i8_n(nz);
                for (int st = 0; st < nstage && !give_up; st++, sg++) {
                    const int s = sg % S;
                    if (!mbar_wait_sleep(&full[s], (sg / S) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
                    uint8_t * base = smem + s * L::kStage;
                    const int sbpos = st & 1, buf = g2 % 2, use = g2 / 2;
                    if (sbpos == 0 && use > 0 && !mbar_wait_sleep(&acc_empty[buf], (use - 1) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
                    for (int blk = 0; blk < kQKB; blk++) {
#pragma unroll
                        for (int pl = 0; pl < P; pl++)
                            mma_i8_acc(tmem + buf * P * kQNT + pl * kQNT, smem_desc_sw128(base + pl * kQM * 128, blk),
                                       smem_desc_sw128(base + L::kA, blk), idesc, (uint32_t) (sbpos | blk));
                    }
                    mma_commit(&empty[s]);
                    if (sbpos == 1) {
                        mma_commit(&acc_full[buf]);
                        g2++;
                    }
                }
            }
        }
    } else {
        // ---- epilogue: lane quarter q = warp % 4 owns tile rows 32 q .. 32 q + 31; warp half h the 32 tokens
        // 32 h .. 32 h + 31, read as two groups of 16. A warp without tokens in a tile still waits and arrives on
        // every barrier ----
        const int q = warp & 3, h = (warp - 2) >> 2;
        const int row = 32 * q + lane;
        int sg = 0, g2 = 0;
        for (int it = blockIdx.x; it < items && !give_up; it += gridDim.x) {
            int m0, nz, live_all, tn;
            tile_of(it, m0, nz, live_all, tn);
            const int live = live_all - 32 * h;
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; i++) acc[i] = 0.0f;
            for (int st = 0; st < nstage && !give_up; st++, sg++) {
                const int s = sg % S;
                if ((st & 1) == 1) {
                    // the super-block's (d, dmin) and dx come with its second stage: read them into registers as soon
                    // as the stage has landed and hand the stage back, so the ring is paced by the MMAs alone; then
                    // one integer and one float step on the accumulators, in super-block order
                    if (!mbar_wait_sleep(&full[s], (sg / S) & 1)) {
                        if (lane == 0) atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    const uint8_t * dd = smem + s * L::kStage + L::kA + L::kB;
                    const float4 ddv = reinterpret_cast<const float4 *>(dd)[row];
                    float dxr[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) dxr[i] = reinterpret_cast<const float *>(dd + L::kDd)[32 * h + i];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);
                    const int buf = g2 % 2, use = g2 / 2;
                    g2++;
                    if (!mbar_wait_sleep(&acc_full[buf], use & 1)) {
                        if (lane == 0) atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        if (32 * h + 16 * hf >= nz) break;  // warp-uniform
                        int A[P][16];
                        const uint32_t ta = tmem + ((uint32_t) (32 * q) << 16) + buf * P * kQNT + 32 * h + 16 * hf;
#pragma unroll
                        for (int pl = 0; pl < P; pl++) tmem_ld16(ta + pl * kQNT, A[pl]);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            if (16 * hf + i >= live) break;
                            const float dxv = dxr[16 * hf + i];
                            int sumi, summ;
                            kq_combine<KIND>(A, i, sumi, summ);
                            float & a = acc[16 * hf + i];
                            a = fmaf(__fmul_rn(dxv, ddv.x), (float) sumi, a);
                            if (KIND == 4) a = fmaf(-__fmul_rn(dxv, ddv.y), (float) summ, a);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
                    continue;
                }
                // nothing of the super-block's first stage is read here, but the warp still waits for the stage to
                // land before handing it back: a parity wait tells only one phase from the next, so an arrival
                // ahead of the landing could complete a phase that a slower warp is still reading
                if (!mbar_wait_sleep(&full[s], (sg / S) & 1)) {
                    if (lane == 0) atomicOr(p.err, kErrTimeout);
                    give_up = 1;
                    break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (give_up) break;
            if (live <= 0) continue;
            const int64_t grow = (int64_t) tn * kQM + row;
            if (grow < p.N)
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    if (i >= live) break;
                    p.y[(int64_t) (m0 + 32 * h + i) * p.ldy + grow] = acc[i];
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kQTmemCols));
    }
}

}  // namespace

// ------------------------------------------------------------------------------------------------------------------
// Host: the expansion cache and the launcher
// ------------------------------------------------------------------------------------------------------------------
bool gemm_kq_tc_supported(const WeightView & w, int64_t M) {
    return (w.type == B200_TYPE_Q4_K || w.type == B200_TYPE_Q6_K) && M >= 32 && w.K % 256 == 0 && w.K <= (int64_t) 1 << 29 &&
           4 * w.rows < ((int64_t) 1 << 31) && tensor_maps_available();
}

void kq_release(b200_context * ctx, const void * data) {
    auto it = ctx->kq.find(data);
    if (it == ctx->kq.end()) return;
    cudaFreeAsync(it->second.mem, ctx->stream);  // stream-ordered: kernels already queued still read it
    ctx->kq.erase(it);
}

void kq_release_all(b200_context * ctx) {
    for (auto & e : ctx->kq) cudaFree(e.second.mem);
    ctx->kq.clear();
}

// The expanded copy of w (created on first use, on the context stream).
static cudaError_t kq_get(b200_context * ctx, const b200_weight * wt, KqExpansion ** out) {
    auto it = ctx->kq.find(wt->data);
    if (it != ctx->kq.end()) {
        *out = &it->second;
        return cudaSuccess;
    }
    const WeightView w = view_of(wt);
    const int64_t rows = w.rows, K = w.K, nsb = K / 256;
    auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    const size_t qb = up((size_t) rows * K * (w.type == B200_TYPE_Q6_K ? 4 : 3));
    const size_t db = up((size_t) rows * nsb * 16);
    KqExpansion e;
    e.type = w.type;
    e.bytes = qb + db;
    cudaError_t err = cudaMallocAsync(&e.mem, e.bytes, ctx->stream);
    if (err != cudaSuccess) return err;
    uint8_t * m = (uint8_t *) e.mem;
    e.q = (int8_t *) m;
    e.dd = (float *) (m + qb);
    const int64_t work = rows * nsb;
    int64_t blocks = (work + 7) / 8;
    if (blocks > (int64_t) ctx->num_sms * 16) blocks = (int64_t) ctx->num_sms * 16;
    if (w.type == B200_TYPE_Q4_K) expand_q4k_kernel<<<(unsigned) blocks, 256, 0, ctx->stream>>>(w, e.q, (float4 *) e.dd);
    else expand_q6k_kernel<<<(unsigned) blocks, 256, 0, ctx->stream>>>(w, e.q, (float4 *) e.dd);
    err = cudaGetLastError();
    if (err != cudaSuccess) {
        cudaFreeAsync(e.mem, ctx->stream);
        return err;
    }
    auto ins = ctx->kq.emplace(wt->data, e);
    *out = &ins.first->second;
    return cudaSuccess;
}

template <int KIND>
static cudaError_t launch_kq(const WeightView & w, const KqExpansion & e, int64_t row0, int64_t N, const int8_t * q, const float * dxT,
                             int64_t ld, int64_t M, float * y, int64_t ldy, unsigned * err, int num_sms, cudaStream_t st) {
    using L = KqLayout<KIND>;
    const int64_t K = w.K;
    CUtensorMap ta, tb, tdd, tdx;
    const uint64_t arows = (uint64_t) L::kPlanes * (uint64_t) w.rows;  // the planes, one after the other
    bool ok = make_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, e.q, (uint64_t) K, arows, (uint64_t) K, 128, kQM, CU_TENSOR_MAP_SWIZZLE_128B) &&
              make_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, (uint64_t) K, (uint64_t) M, (uint64_t) K, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B) &&
              make_map_2d(&tdd, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, e.dd, (uint64_t) (4 * (K / 256)), (uint64_t) w.rows, (uint64_t) (K / 256) * 16, 4,
                          kQM, CU_TENSOR_MAP_SWIZZLE_NONE) &&
              make_map_2d(&tdx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dxT, (uint64_t) ld, (uint64_t) (K / 256), (uint64_t) ld * 4, kQNT, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) return cudaErrorInvalidValue;
    KqParams p;
    p.N = N;
    p.K = K;
    p.row0 = row0;
    p.plane_rows = w.rows;
    p.M = (int) M;
    p.tiles_m = (int) ((M + kQNT - 1) / kQNT);
    p.tiles_n = (int) ((N + kQM - 1) / kQM);
    p.y = y;
    p.ldy = ldy;
    p.err = err;
    static int configured = 0;
    if (!configured) {
        cudaError_t e2 = cudaFuncSetAttribute(gemm_kq_tc_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
        if (e2 != cudaSuccess) return e2;
        configured = 1;
    }
    gemm_kq_tc_kernel<KIND><<<L::kCtasPerSm * num_sms, kQThreads, L::kTotal, st>>>(ta, tb, tdd, tdx, p);
    return cudaGetLastError();
}

size_t gemm_kq_tc_act_bytes(int64_t K, int64_t M) {
    const int64_t ld = (M + 15) & ~(int64_t) 15;
    auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    return up((size_t) M * K) + up((size_t) (K / 256) * ld * 4);
}

cudaError_t launch_gemm_kq_tc(b200_context * ctx, const b200_weight * wt, int64_t row0, int64_t N, const float * x, int64_t M, float * y,
                              int64_t ldy, void * act) {
    const WeightView w = view_of(wt);
    if (!gemm_kq_tc_supported(w, M) || row0 + N > w.rows || ((uintptr_t) x & 15)) return cudaErrorInvalidValue;
    KqExpansion * e = nullptr;
    cudaError_t err = kq_get(ctx, wt, &e);
    if (err != cudaSuccess) return err;
    const int64_t K = w.K, ld = (M + 15) & ~(int64_t) 15;
    auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    uint8_t * a = (uint8_t *) act;
    int8_t * q = (int8_t *) a;
    float * dxT = (float *) (a + up((size_t) M * K));
    int64_t blocks = (M * (K / 256) + 7) / 8;
    if (blocks > (int64_t) ctx->num_sms * 8) blocks = (int64_t) ctx->num_sms * 8;
    quantize_q8k_tc_kernel<<<(unsigned) blocks, 256, 0, ctx->stream>>>(x, K, M, q, dxT, ld);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    if (w.type == B200_TYPE_Q4_K)
        return launch_kq<4>(w, *e, row0, N, q, dxT, ld, M, y, ldy, ctx->dev_err, ctx->num_sms, ctx->stream);
    return launch_kq<6>(w, *e, row0, N, q, dxT, ld, M, y, ldy, ctx->dev_err, ctx->num_sms, ctx->stream);
}

}  // namespace b200
