// gemm_tc_grouped.cu — expert-grouped Q8_0 products (MUL_MAT_ID, the MoE FFN of TextModel::experts,
// src/families/drama3/text-model.cpp:198-221) on the tensor cores.
//
// The (token, slot) pairs are sorted by expert (moe.cu): expert e's pairs occupy slots [grp_off[e], grp_off[e+1]),
// each segment padded to a multiple of 16 slots, and the pairs' activations are quantized to q8_0 in slot order
// (q [slots][K] int8, dT [K/32][ldP] float block scales, transposed). A token tile is 16 or 32 consecutive slots of
// one expert; the route kernel lists the tiles. One work item = one token tile x one 128-row tile of the expert's weight
// matrix. A dense product (MUL_MAT with many activation rows) is one expert whose tiles are 32 consecutive tokens.
// Per 32-wide K block, one tcgen05.mma kind::i8 of shape M = 128 (weight rows) x N = the tile's token count
// (16 or 32, a run-time field of the instruction descriptor) x K = 32 computes the block's exact int32 sums. Blocks go
// in pairs into one of four tensor-memory buffers (2 x 32 columns each; eight blocks in flight between the MMA and the
// epilogue), one barrier round trip per pair; epilogue warps
// read a pair's sums (tcgen05.ld), scale them by d_w[row][b] * d_x[slot][b] and add them to float32 registers in
// block order, as ggml's CPU vec_dot does. Operands come by TMA (2-D tensor maps, 128-byte swizzle, no multicast).
// The grid is persistent (two CTAs per SM) and walks the items in a fixed order; every role of
// a CTA derives the same item sequence from the tile list, so they need no other coordination than the stage and
// accumulator barriers. Warp roles: 0 = TMA producer, 1 = tensor-memory allocator and MMA issuer (one thread),
// 2..9 = epilogue. Every wait is bounded; one that gives up records B200_DEVERR_TIMEOUT and the CTA runs to its end
// (freeing its tensor memory) without further waits.
#include "internal.h"
#include "tcgen05.cuh"

namespace b200 {

namespace {

constexpr int kGM = 128;       // weight rows per tile (MMA M)
constexpr int kGKB = 8;        // 32-wide K blocks per pipeline stage
constexpr int kGStages = 2;
constexpr int kGThreads = 320; // producer, MMA, 8 epilogue warps
constexpr int kGEpiWarps = 8;
constexpr int kGBufs = 4;      // tensor-memory accumulators in flight, one K-block pair (2 x kGNT columns) each
constexpr int kGNT = 32;       // slots per token tile (largest MMA N used)
constexpr unsigned kErrTimeout = 4u;

struct GLayout {
    static constexpr int kA = kGKB * kGM * 32;   // weights: two [128 rows][128 B] swizzled tiles
    static constexpr int kB = kGKB * kGNT * 32;  // activations: two [32 rows][128 B] swizzled tiles
    static constexpr int kDw = kGM * kGKB * 2;   // fp16 weight scales [128][8]
    static constexpr int kDx = kGKB * kGNT * 4;  // f32 activation scales [8][32]
    static constexpr int kStage = kA + kB + kDw + kDx;
    static constexpr int kTotal = kGStages * kStage + 1024 + 1024;  // + barriers + alignment slack
    static_assert(kA % 1024 == 0 && kB % 1024 == 0 && kStage % 1024 == 0, "stage regions stay 1024-aligned");
};

struct GroupedParams {
    int64_t N;                // rows per expert (output width)
    int64_t K;
    int64_t row0;             // first weight row (dense products of a row range)
    int dense_m;              // > 0: one dense product of dense_m tokens in token order; tiles is null
    const int4 * tiles;       // {expert, first slot, slots (16 or 32), routed slots (the rest is padding)}
    const int * ntiles;       // number of tiles (device)
    int tiles_n;              // 128-row tiles per expert
    int ksplit;               // dense products: K ranges per output tile (partials summed in split order), else 1
    float * ws;               // split partial tiles [output tile][split][kGNT][kGM]
    unsigned * tickets;       // one per output tile, zero between launches
    const int32_t * row_map;  // output row of each slot (< 0: none); null: the slot itself
    float * y;
    int64_t ldy;
    unsigned * err;
};

// Token tile i: from the route kernel's list, or (dense products) 32 consecutive tokens.
__device__ __forceinline__ int4 g_tile(const GroupedParams & p, int i) {
    if (p.tiles) return p.tiles[i];
    const int m0 = 32 * i, rem = p.dense_m - m0;
    const int live = rem < 32 ? rem : 32;
    return make_int4(0, m0, (live + 15) & ~15, live);
}

// kSplit: K may be split across CTAs (dense products with few output tiles); the expert products compile without
// that code.
template <bool kSplit>
__global__ void __launch_bounds__(kGThreads, 2)
    gemm_q8_0_tc_grouped_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                const __grid_constant__ CUtensorMap tmDw, const __grid_constant__ CUtensorMap tmDx, GroupedParams p) {
    using L = GLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint64_t * bars = reinterpret_cast<uint64_t *>(smem + kGStages * L::kStage);
    uint64_t * full = bars;
    uint64_t * empty = bars + kGStages;
    uint64_t * acc_full = bars + 2 * kGStages;   // [bufs] a block pair's int32 sums ready in tensor memory
    uint64_t * acc_empty = acc_full + kGBufs;    // [bufs] epilogue has read them
    uint64_t * xbar = acc_empty + kGBufs;        // [2] split-K: every epilogue warp stored its partial / ticket taken
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(xbar + 2);
    __shared__ int last_split;
    __shared__ volatile int give_up;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nstage = (int) (p.K / 32 / kGKB);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kGEpiWarps);
        }
        for (int b = 0; b < kGBufs; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kGEpiWarps);
        }
        mbar_init(&xbar[0], kGEpiWarps);
        mbar_init(&xbar[1], 1);
        fence_mbar_init();
        give_up = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)), "r"(2 * kGBufs * kGNT));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // item = (output tile, K split), the split fastest: the splits of one tile run at the same time on different CTAs
    const int ksplit = kSplit ? p.ksplit : 1;
    const int spl = nstage / ksplit;  // stages per split
    // Launched with programmatic dependent launch, the producer streams the weights (and weight scales) of its first
    // item's first stages now, while the kernel before this one (activation quantization, or the SwiGLU between the
    // expert products) still runs; those stages' activation loads follow the wait below. Weight tiles depend on no
    // earlier kernel for dense products, and on the routing's tile list for expert products: the routing ran two or
    // more launches earlier and had completed before the previous kernel passed its own wait, which preceded this
    // launch; the list is read through L2.
    int pre = 0;
    const int items_early = p.tiles ? (int) __ldcg(p.ntiles) * p.tiles_n * ksplit : ((p.dense_m + 31) / 32) * p.tiles_n * ksplit;
    if (warp == 0 && lane == 0 && (int) blockIdx.x < items_early) {
        const int it = blockIdx.x;
        const int ot = kSplit ? it / ksplit : it, ks = kSplit ? it % ksplit : 0;
        const int4 t = p.tiles ? __ldcg(p.tiles + ot / p.tiles_n) : g_tile(p, ot / p.tiles_n);
        const int arow = (int) ((int64_t) t.x * p.N + p.row0 + (int64_t) (ot % p.tiles_n) * kGM);
        const uint32_t bytes = (uint32_t) (L::kA + t.z * 256 + L::kDw + L::kDx);
        for (; pre < kGStages && pre < spl; pre++) {
            uint8_t * base = smem + pre * L::kStage;
            mbar_arrive_expect_tx(&full[pre], bytes);
            const int kbs = (ks * spl + pre) * kGKB;
            for (int jj = 0; jj < 2; jj++) tma_load_2d(base + jj * kGM * 128, &tmA, (kbs + 4 * jj) * 32, arow, &full[pre]);
            tma_load_2d(base + L::kA + L::kB, &tmDw, kbs, arow, &full[pre]);
        }
    }
    // the tile list and the activations come from the kernels before this one (no-ops unless launched with
    // programmatic dependent launch); the next kernel may launch its CTAs once these have started
    pdl_wait();
    pdl_launch_dependents();
    const int items = (p.tiles ? *p.ntiles : (p.dense_m + 31) / 32) * p.tiles_n * ksplit;

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            prefetch_tensormap(&tmA);
            prefetch_tensormap(&tmB);
            prefetch_tensormap(&tmDw);
            prefetch_tensormap(&tmDx);
            int sg = 0;
            for (int it = blockIdx.x; it < items && !give_up; it += gridDim.x) {
                const int ot = kSplit ? it / ksplit : it, ks = kSplit ? it % ksplit : 0;
                const int4 t = g_tile(p, ot / p.tiles_n);
                const int arow = (int) ((int64_t) t.x * p.N + p.row0 + (int64_t) (ot % p.tiles_n) * kGM);
                const int nsub = t.z / 16;
                const uint32_t bytes = (uint32_t) (L::kA + t.z * 256 + L::kDw + L::kDx);
                for (int st = ks * spl; st < (ks + 1) * spl; st++, sg++) {
                    const int s = sg % kGStages, use = sg / kGStages;
                    const bool early = sg < pre;  // weights already issued before the wait
                    if (use > 0 && !mbar_wait_sleep(&empty[s], (use - 1) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    uint8_t * base = smem + s * L::kStage;
                    if (!early) mbar_arrive_expect_tx(&full[s], bytes);
                    const int kbs = st * kGKB;
                    for (int jj = 0; jj < 2; jj++) {
                        if (!early) tma_load_2d(base + jj * kGM * 128, &tmA, (kbs + 4 * jj) * 32, arow, &full[s]);
                        for (int r = 0; r < nsub; r++)
                            tma_load_2d(base + L::kA + jj * kGNT * 128 + r * 16 * 128, &tmB, (kbs + 4 * jj) * 32, t.y + 16 * r, &full[s]);
                    }
                    if (!early) tma_load_2d(base + L::kA + L::kB, &tmDw, kbs, arow, &full[s]);
                    tma_load_2d(base + L::kA + L::kB + L::kDw, &tmDx, t.y, kbs, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: one K block per MMA; block pair g goes to tensor-memory buffer g % 2 (columns 0..63 and
        // 64..127 of it), one commit per pair ----
        if (lane == 0) {
            int sg = 0, g2 = 0;
            for (int it = blockIdx.x; it < items && !give_up; it += gridDim.x) {
                const int4 t = g_tile(p, (kSplit ? it / ksplit : it) / p.tiles_n);
                const uint32_t idesc = idesc_i8_n(t.z);
                for (int st = 0; st < spl && !give_up; st++, sg++) {
                    const int s = sg % kGStages;
                    if (!mbar_wait_sleep(&full[s], (sg / kGStages) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
                    uint8_t * base = smem + s * L::kStage;
                    for (int j = 0; j < kGKB; j += 2, g2++) {
                        const int buf = g2 % kGBufs, use = g2 / kGBufs;
                        if (use > 0 && !mbar_wait_sleep(&acc_empty[buf], (use - 1) & 1)) {
                            atomicOr(p.err, kErrTimeout);
                            give_up = 1;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (int jj = 0; jj < 2; jj++)
                            mma_i8(tmem + buf * 2 * kGNT + jj * kGNT, smem_desc_sw128(base + ((j + jj) / 4) * kGM * 128, (j + jj) % 4),
                                   smem_desc_sw128(base + L::kA + ((j + jj) / 4) * kGNT * 128, (j + jj) % 4), idesc);
                        mma_commit(&acc_full[buf]);
                    }
                    if (give_up) break;
                    mma_commit(&empty[s]);
                }
            }
        }
    } else {
        // ---- epilogue: lane quarter q = warp % 4 owns tile rows 32 q .. 32 q + 31 (one per lane); warp half h takes
        // the tile's 16-slot column chunk h. A warp without columns (h = 1 in a tile of 16 slots) still waits and
        // arrives on every barrier, so no warp runs a phase ahead of the others: parity waits cannot tell phase n
        // from phase n + 2 ----
        const int q = warp & 3, h = (warp - 2) >> 2;
        const int row = 32 * q + lane;
        const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
        int sg = 0, g2 = 0, xi = 0;
        for (int it = blockIdx.x; it < items && !give_up; it += gridDim.x) {
            const int ot = kSplit ? it / ksplit : it, ks = kSplit ? it % ksplit : 0;
            const int4 t = g_tile(p, ot / p.tiles_n);
            const int tn = ot % p.tiles_n;
            const bool has = h < t.z / 16;
            const int live = t.w - 16 * h;  // routed slots in this warp's chunk (the rest is padding: no math)
            float2 acc[8];
#pragma unroll
            for (int i = 0; i < 8; i++) acc[i] = make_float2(0.0f, 0.0f);
            for (int st = 0; st < spl && !give_up; st++, sg++) {
                const int s = sg % kGStages;
                const uint8_t * base = smem + s * L::kStage;
                const __half2 * dw2 = reinterpret_cast<const __half2 *>(base + L::kA + L::kB) + row * (kGKB / 2);
                const float * dxT = reinterpret_cast<const float *>(base + L::kA + L::kB + L::kDw);
                for (int j = 0; j < kGKB; j += 2, g2++) {
                    const int buf = g2 % kGBufs, use = g2 / kGBufs;
                    if (!mbar_wait_sleep(&acc_full[buf], use & 1)) {
                        if (lane == 0) atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
                    if (!has) {  // no columns in this tile: only the barrier protocol
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[buf]);
                        continue;
                    }
                    // both blocks of the pair in registers, then the buffer is released
                    int v[2][16];
                    const uint32_t ta = tmem + ((uint32_t) (32 * q) << 16) + buf * 2 * kGNT + 16 * h;
                    tmem_ld16(ta, v[0]);
                    tmem_ld16(ta + kGNT, v[1]);
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
                    const float2 dwp = __half22float2(dw2[j / 2]);
                    // acc += float(sum) * (d_x * d_w), in block order; |sum| <= 32 * 127 * 128 < 2^22 converts exactly
                    // through the float 12582912 + sum (bit pattern 0x4B400000 + sum)
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        const float dwr = jj ? dwp.y : dwp.x;
                        const float2 w2 = make_float2(dwr, dwr);
                        const float4 * dx4 = reinterpret_cast<const float4 *>(dxT + (j + jj) * kGNT + 16 * h);
#pragma unroll
                        for (int t4 = 0; t4 < 4; t4++) {
                            if (4 * t4 >= live) break;
                            const float4 d = dx4[t4];
                            const int * vv = v[jj] + 4 * t4;
                            const float2 s01 = __fmul2_rn(make_float2(d.x, d.y), w2);
                            const float2 s23 = __fmul2_rn(make_float2(d.z, d.w), w2);
                            const float2 f01 = __fadd2_rn(make_float2(__int_as_float(vv[0] + 0x4B400000), __int_as_float(vv[1] + 0x4B400000)),
                                                          neg_magic);
                            const float2 f23 = __fadd2_rn(make_float2(__int_as_float(vv[2] + 0x4B400000), __int_as_float(vv[3] + 0x4B400000)),
                                                          neg_magic);
                            acc[2 * t4] = __ffma2_rn(f01, s01, acc[2 * t4]);
                            acc[2 * t4 + 1] = __ffma2_rn(f23, s23, acc[2 * t4 + 1]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (give_up) break;
            const int64_t grow = (int64_t) tn * kGM + row;
            if (kSplit && ksplit > 1) {
                // ---- split K: store this split's partial tile; the last split of the tile (an atomic ticket) adds
                // the partials in split order, so the result does not depend on timing. Every epilogue warp takes
                // part (bounded mbarrier waits, no unbounded named barrier) ----
                float * part = p.ws + ((int64_t) ot * ksplit + ks) * kGNT * kGM;
                if (has)
#pragma unroll
                    for (int i = 0; i < 16; i++) part[(16 * h + i) * kGM + row] = (i & 1) ? acc[i / 2].y : acc[i / 2].x;
                __threadfence();
                __syncwarp();
                if (lane == 0) mbar_arrive(&xbar[0]);
                if (warp == 2 && lane == 0) {
                    if (!mbar_wait_sleep(&xbar[0], xi & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                    }
                    const unsigned ticket = atomicAdd(&p.tickets[ot], 1u);
                    last_split = ticket == (unsigned) (ksplit - 1);
                    if (last_split) p.tickets[ot] = 0u;  // ready for the next launch
                    mbar_arrive(&xbar[1]);
                }
                if (!mbar_wait_sleep(&xbar[1], xi & 1)) {
                    if (lane == 0) atomicOr(p.err, kErrTimeout);
                    give_up = 1;
                }
                xi++;
                if (give_up || !last_split || !has || grow >= p.N) continue;
                __threadfence();
                // partials summed in split order; each split's 16 values are read together (one L2 round trip per
                // split, not per value)
                const float * parts = p.ws + (int64_t) ot * ksplit * kGNT * kGM + (int64_t) (16 * h) * kGM + row;
                float sum[16];
#pragma unroll
                for (int i = 0; i < 16; i++) sum[i] = 0.0f;
                for (int z = 0; z < ksplit; z++) {
                    float v[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = __ldcg(parts + ((int64_t) z * kGNT + i) * kGM);
#pragma unroll
                    for (int i = 0; i < 16; i++) sum[i] += v[i];
                }
#pragma unroll
                for (int i = 0; i < 16; i++)
                    if (i < live) p.y[(int64_t) (t.y + 16 * h + i) * p.ldy + grow] = sum[i];
                continue;
            }
            if (!has) continue;
            // ---- output: one weight row per lane, so each slot's store is one coalesced 128-byte line ----
            if (grow < p.N) {
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    if (i >= live) break;
                    const int slot = t.y + 16 * h + i;
                    const int64_t orow = p.row_map ? (int64_t) p.row_map[slot] : (int64_t) slot;
                    const float2 a = acc[i / 2];
                    if (orow >= 0) p.y[orow * p.ldy + grow] = (i & 1) ? a.y : a.x;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kGBufs * kGNT));
    }
}

}  // namespace

bool gemm_tc_grouped_supported(const WeightView & w) {
    return w.type == B200_TYPE_Q8_0 && w.K % (32 * kGKB) == 0 && w.K <= (int64_t) 1 << 30 && w.rows < ((int64_t) 1 << 31) &&
           tensor_maps_available();
}

namespace {

cudaError_t launch_grouped(const WeightView & w, int64_t N, int64_t row0, int dense_m, const int4 * tiles, const int * ntiles,
                           const int8_t * q, const float * dT, int64_t ldP, int64_t slots, const int32_t * row_map, float * y,
                           int64_t ldy, unsigned * err, int num_sms, cudaStream_t st, int ksplit = 1, float * ws = nullptr,
                           unsigned * tickets = nullptr) {
    using L = GLayout;
    const int64_t K = w.K, KB = K / 32;
    if (!gemm_tc_grouped_supported(w) || ldP % 16 || slots > ldP || slots < 1) return cudaErrorInvalidValue;
    CUtensorMap ta, tb, tdw, tdx;
    if (!make_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.f0, (uint64_t) K, (uint64_t) w.rows, (uint64_t) K, 128, kGM,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, (uint64_t) K, (uint64_t) slots, (uint64_t) K, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&tdw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.f1, (uint64_t) KB, (uint64_t) w.rows, (uint64_t) KB * 2, kGKB, kGM,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&tdx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dT, (uint64_t) ldP, (uint64_t) KB, (uint64_t) ldP * 4, kGNT, kGKB,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    GroupedParams p;
    p.N = N;
    p.K = K;
    p.row0 = row0;
    p.dense_m = dense_m;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.tiles_n = (int) ((N + kGM - 1) / kGM);
    p.ksplit = ksplit;
    p.ws = ws;
    p.tickets = tickets;
    p.row_map = row_map;
    p.y = y;
    p.ldy = ldy;
    p.err = err;
    static int configured = 0;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_0_tc_grouped_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_q8_0_tc_grouped_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
        if (e != cudaSuccess) return e;
        configured = 1;
    }
    // Programmatic dependent launch: the CTAs stream their first weight stages while the previous kernel finishes.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) (2 * num_sms), 1, 1);
    cfg.blockDim = dim3(kGThreads, 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (ksplit > 1) return cudaLaunchKernelEx(&cfg, gemm_q8_0_tc_grouped_kernel<true>, ta, tb, tdw, tdx, p);
    return cudaLaunchKernelEx(&cfg, gemm_q8_0_tc_grouped_kernel<false>, ta, tb, tdw, tdx, p);
}

}  // namespace

cudaError_t launch_gemm_tc_grouped(const WeightView & w, int64_t N, const int4 * tiles, const int * ntiles, const int8_t * q,
                                   const float * dT, int64_t ldP, int64_t slots, const int32_t * row_map, float * y, int64_t ldy,
                                   unsigned * err, int num_sms, cudaStream_t st) {
    if (slots % 16) return cudaErrorInvalidValue;
    return launch_grouped(w, N, 0, 0, tiles, ntiles, q, dT, ldP, slots, row_map, y, ldy, err, num_sms, st);
}

int gemm_tc_dense_splits(const WeightView & w, int64_t N, int64_t M, int num_sms) {
    const int64_t tiles = ((M + 31) / 32) * ((N + kGM - 1) / kGM);
    const int nstage = (int) (w.K / 32 / kGKB);
    int ks = 1;
    while (ks * 2 <= 8 && tiles * ks * 2 <= 2 * (int64_t) num_sms && nstage % (ks * 2) == 0) ks *= 2;
    return ks;
}

size_t gemm_tc_dense_ws_bytes(int64_t N, int64_t M, int ksplit) {
    return ksplit > 1 ? (size_t) ((M + 31) / 32) * ((N + kGM - 1) / kGM) * ksplit * kGNT * kGM * 4 : 0;
}

cudaError_t launch_gemm_tc_dense(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dT, int64_t ldP,
                                 int64_t M, float * y, int64_t ldy, unsigned * err, int num_sms, cudaStream_t st, int ksplit, float * ws,
                                 unsigned * tickets) {
    if (M < 1 || M > (1 << 30) || row0 + N > w.rows || ksplit < 1 || (w.K / 32 / kGKB) % ksplit || (ksplit > 1 && (!ws || !tickets)))
        return cudaErrorInvalidValue;
    return launch_grouped(w, N, row0, (int) M, nullptr, nullptr, q, dT, ldP, M, nullptr, y, ldy, err, num_sms, st, ksplit, ws, tickets);
}

}  // namespace b200
