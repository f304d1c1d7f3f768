// gemm_tc.cu — Q8_0 products with many activation rows (M >= 32: prefill, audio-encoder, multi-stream decode) on the
// 5th-generation tensor cores: tcgen05.mma kind::i8 with int32 accumulators in tensor memory, fed by TMA.
//
// ggml's CPU backend computes these as per-32-block int32 dot products of the Q8_0 weights with q8_0-quantized
// activations, each scaled by d_w * d_x and summed in float32. Here one tcgen05.mma of shape M=128 (weight rows) x
// N=NT (tokens) x K=32 computes exactly the int32 sums of ONE block for a 128 x NT tile ("swap AB": weights on the M
// side, since decode batches are small). Accumulators live in tensor memory, four deep: while later blocks multiply
// into the other buffers, eight epilogue warps read block b's int32 sums out of its buffer (tcgen05.ld), scale them
// by d_w[row][b] * d_x[token][b] and add them to float32 registers. Operands arrive by TMA (2-D tensor maps, boxes of
// 128-byte rows = four K blocks, 128-byte swizzle that the MMA's shared-memory descriptors read as is; no multicast).
// Warp roles: 0 = TMA producer, 1 = tensor-memory allocator and MMA issuer (one thread), 2..9 = epilogue.
// Split-K: with S > 1, CTAs of one tile sum disjoint K ranges; each writes its partial tile to a workspace and the
// last to finish (an atomic ticket) adds the S partials in split order, so results do not depend on timing.
// Every wait is bounded; one that gives up records B200_DEVERR_TIMEOUT and the CTA runs to its end (freeing its
// tensor memory) without further waits.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "tcgen05.cuh"

namespace b200 {

namespace {

constexpr int kTcM = 128;          // weight rows per tile (MMA M)
constexpr int kTcKB = 8;           // 32-wide K blocks per pipeline stage
constexpr int kTcStages = 2;       // two CTAs fit per SM
constexpr int kTcThreads = 320;    // 10 warps: producer, MMA, 8 epilogue
constexpr int kTcEpiWarps = 8;
constexpr int kTcAccBufs = 4;      // tensor-memory accumulators in flight (4 x NT columns; two CTAs per SM use all 512)
constexpr unsigned kErrTimeout = 4u;

template <int NT>
struct TcLayout {
    static constexpr int kA = kTcKB * kTcM * 32;       // weight int8: two [128 rows][128 B] tiles (4 K blocks each)
    static constexpr int kB = kTcKB * NT * 32;         // activation int8: two [NT rows][128 B] tiles
    static constexpr int kDw = kTcM * kTcKB * 2;       // fp16 weight scales [128][KB]
    static constexpr int kDx = kTcKB * NT * 4;         // f32 activation scales [KB][NT] (transposed)
    static constexpr int kStage = kA + kB + kDw + kDx; // multiple of 1024
    static constexpr int kBars = 1024;
    static constexpr int kTotal = kTcStages * kStage + kBars + 1024;  // + alignment slack
    static_assert(kA % 1024 == 0 && kB % 1024 == 0 && (kDw + kDx) % 1024 == 0, "stage regions stay 1024-aligned");
};

struct TcParams {
    int64_t N;      // rows of this product (weight rows row0 .. row0 + N)
    int64_t M;      // activation rows (tokens)
    int64_t K;
    int64_t row0;
    float * y;
    int64_t ldy;
    unsigned * err;
    int splits;          // K splits per tile
    int kb_per_split;    // K blocks per split (a multiple of kTcKB)
    float * ws;          // split-K partial tiles [tiles][splits][NT][128]
    unsigned * tickets;  // one per tile, zero between launches
};


template <int NT>
__global__ void __launch_bounds__(kTcThreads, 2)
    gemm_q8_0_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmDw, const __grid_constant__ CUtensorMap tmDx, TcParams p) {
    using L = TcLayout<NT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint64_t * bars = reinterpret_cast<uint64_t *>(smem + kTcStages * L::kStage);
    uint64_t * full = bars;                       // [stages] TMA landed
    uint64_t * empty = bars + kTcStages;          // [stages] MMAs done + epilogue done with the scales
    uint64_t * acc_full = bars + 2 * kTcStages;   // [bufs] block's int32 sums ready in tensor memory
    uint64_t * acc_empty = acc_full + kTcAccBufs; // [bufs] epilogue has read them
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + kTcAccBufs);
    __shared__ volatile int give_up;
    __shared__ int last_split;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
    const int kb0 = split * p.kb_per_split;
    const int nkb = p.kb_per_split;
    const int nstage = nkb / kTcKB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kTcEpiWarps);
        }
        for (int b = 0; b < kTcAccBufs; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kTcEpiWarps);
        }
        fence_mbar_init();
        give_up = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)), "r"(kTcAccBufs * NT));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer: per stage two 128-byte-row boxes of weights and of activations, and both scale tiles ----
        if (lane == 0) {
            for (int st = 0; st < nstage && !give_up; st++) {
                const int s = st % kTcStages;
                const int use = st / kTcStages;
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
                    atomicOr(p.err, kErrTimeout);
                    give_up = 1;
                    break;
                }
                uint8_t * base = smem + s * L::kStage;
                mbar_arrive_expect_tx(&full[s], (uint32_t) L::kStage);
                const int kbs = kb0 + st * kTcKB;
                for (int j = 0; j < kTcKB; j += 4) {
                    tma_load_2d(base + (j / 4) * kTcM * 128, &tmA, (kbs + j) * 32, (int) (p.row0 + (int64_t) tile_n * kTcM), &full[s]);
                    tma_load_2d(base + L::kA + (j / 4) * NT * 128, &tmB, (kbs + j) * 32, tile_m * NT, &full[s]);
                }
                tma_load_2d(base + L::kA + L::kB, &tmDw, kbs, (int) (p.row0 + (int64_t) tile_n * kTcM), &full[s]);
                tma_load_2d(base + L::kA + L::kB + L::kDw, &tmDx, tile_m * NT, kbs, &full[s]);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: one block (K = 32) per MMA, into the tensor-memory buffer b % 4 ----
        if (lane == 0) {
            const uint32_t idesc = idesc_i8<NT>();
            int b = 0;
            for (int st = 0; st < nstage && !give_up; st++) {
                const int s = st % kTcStages;
                if (!mbar_wait(&full[s], (st / kTcStages) & 1)) {
                    atomicOr(p.err, kErrTimeout);
                    give_up = 1;
                    break;
                }
                tc_fence_after();
                uint8_t * base = smem + s * L::kStage;
                for (int j = 0; j < kTcKB; j++, b++) {
                    const int buf = b % kTcAccBufs, use = b / kTcAccBufs;
                    if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
                    mma_i8(tmem + buf * NT, smem_desc_sw128(base + (j / 4) * kTcM * 128, j % 4),
                           smem_desc_sw128(base + L::kA + (j / 4) * NT * 128, j % 4), idesc);
                    mma_commit(&acc_full[buf]);
                }
                if (give_up) break;
                mma_commit(&empty[s]);  // the stage's operands are free once these MMAs complete
            }
        }
    } else {
        // ---- epilogue: warps 2..9; lane quarter q = warp % 4 gives the tile row 32 q + lane, and the two warps of a
        // quarter take token columns [32 h, 32 h + 32) ----
        constexpr int kCols = NT / 2;
        const int q = warp & 3, h = (warp - 2) >> 2;
        const int row = 32 * q + lane;
        float2 acc[kCols / 2];
#pragma unroll
        for (int t = 0; t < kCols / 2; t++) acc[t] = make_float2(0.0f, 0.0f);
        const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
        int b = 0;
        for (int st = 0; st < nstage && !give_up; st++) {
            const int s = st % kTcStages;
            const uint8_t * base = smem + s * L::kStage;
            const __half * dw = reinterpret_cast<const __half *>(base + L::kA + L::kB);
            const float * dxT = reinterpret_cast<const float *>(base + L::kA + L::kB + L::kDw);
            for (int j = 0; j < kTcKB; j++, b++) {
                const int buf = b % kTcAccBufs, use = b / kTcAccBufs;
                if (!mbar_wait(&acc_full[buf], use & 1)) {
                    if (lane == 0) atomicOr(p.err, kErrTimeout);
                    give_up = 1;
                    break;
                }
                tc_fence_after();
                int v[kCols];
                tmem_ld32(tmem + ((uint32_t) (32 * q) << 16) + buf * NT + kCols * h, v);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
                // acc += float(sum) * (d_x * d_w), two tokens per packed f32x2 op. The int32 block sums
                // (|sum| <= 32 * 127 * 128 < 2^22) convert exactly: 0x4B400000 + sum is the float 12582912 + sum.
                const float dwr = __half2float(dw[row * kTcKB + j]);
                const float2 w2 = make_float2(dwr, dwr);
                const float4 * dx4 = reinterpret_cast<const float4 *>(dxT + j * NT + kCols * h);
#pragma unroll
                for (int t4 = 0; t4 < kCols / 4; t4++) {
                    const float4 d = dx4[t4];
                    const float2 s01 = __fmul2_rn(make_float2(d.x, d.y), w2);
                    const float2 s23 = __fmul2_rn(make_float2(d.z, d.w), w2);
                    const float2 f01 = __fadd2_rn(
                        make_float2(__int_as_float(v[4 * t4] + 0x4B400000), __int_as_float(v[4 * t4 + 1] + 0x4B400000)), neg_magic);
                    const float2 f23 = __fadd2_rn(
                        make_float2(__int_as_float(v[4 * t4 + 2] + 0x4B400000), __int_as_float(v[4 * t4 + 3] + 0x4B400000)), neg_magic);
                    acc[2 * t4] = __ffma2_rn(f01, s01, acc[2 * t4]);
                    acc[2 * t4 + 1] = __ffma2_rn(f23, s23, acc[2 * t4 + 1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // ---- output (direct, or split-K partial + ordered reduction by the last split) ----
        const int64_t grow = (int64_t) tile_n * kTcM + row;  // row of this product
        const int tile = tile_m * gridDim.x + tile_n;
        const int t0 = kCols * h;
        if (p.splits == 1) {
            if (grow < p.N)
                for (int t = 0; t < kCols; t++) {
                    const int64_t m = (int64_t) tile_m * NT + t0 + t;
                    if (m < p.M) p.y[m * p.ldy + grow] = (t & 1) ? acc[t / 2].y : acc[t / 2].x;
                }
        } else {
            float * part = p.ws + ((int64_t) tile * p.splits + split) * NT * kTcM;
            for (int t = 0; t < kCols; t++) part[(t0 + t) * kTcM + row] = (t & 1) ? acc[t / 2].y : acc[t / 2].x;
            __threadfence();
            asm volatile("bar.sync 2, %0;" ::"r"(32 * kTcEpiWarps) : "memory");
            if (warp == 2 && lane == 0) {
                const unsigned ticket = atomicAdd(&p.tickets[tile], 1u);
                last_split = ticket == (unsigned) (p.splits - 1);
                if (last_split) p.tickets[tile] = 0;  // ready for the next launch
            }
            asm volatile("bar.sync 2, %0;" ::"r"(32 * kTcEpiWarps) : "memory");
            if (last_split) {
                __threadfence();
                if (grow < p.N)
                    for (int t = 0; t < kCols; t++) {
                        float sum = 0.0f;
                        for (int z = 0; z < p.splits; z++)
                            sum += __ldcg(p.ws + ((int64_t) tile * p.splits + z) * NT * kTcM + (t0 + t) * kTcM + row);
                        const int64_t m = (int64_t) tile_m * NT + t0 + t;
                        if (m < p.M) p.y[m * p.ldy + grow] = sum;
                    }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcAccBufs * NT));
    }
}

template <int NT>
cudaError_t launch_nt(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dx, int64_t dx_ld, int64_t M,
                      float * y, int64_t ldy, unsigned * err, void * ws, size_t ws_bytes, unsigned * tickets, int num_sms, cudaStream_t st) {
    using L = TcLayout<NT>;
    const int64_t K = w.K, KB = K / 32;
    CUtensorMap ta, tb, tdw, tdx;
    if (!make_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.f0, (uint64_t) K, (uint64_t) w.rows, (uint64_t) K, 128, kTcM,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, (uint64_t) K, (uint64_t) M, (uint64_t) K, 128, NT, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&tdw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.f1, (uint64_t) KB, (uint64_t) w.rows, (uint64_t) KB * 2, kTcKB, kTcM,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&tdx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dx, (uint64_t) M, (uint64_t) KB, (uint64_t) dx_ld * 4, NT, kTcKB,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    const int tn = (int) ((N + kTcM - 1) / kTcM), tm = (int) ((M + NT - 1) / NT);
    const int stages_total = (int) (KB / kTcKB);
    // split K (in whole stages, dividing them evenly) while the grid still fits one wave of two CTAs per SM
    int splits = 1;
    while (splits * 2 <= stages_total && (int64_t) tn * tm * splits * 2 <= 2 * (int64_t) num_sms && stages_total % (splits * 2) == 0)
        splits *= 2;
    const size_t ws_need = splits > 1 ? (size_t) tn * tm * splits * NT * kTcM * 4 : 0;
    if (ws_need > ws_bytes || !tickets) splits = 1;
    TcParams p;
    p.N = N;
    p.M = M;
    p.K = K;
    p.row0 = row0;
    p.y = y;
    p.ldy = ldy;
    p.err = err;
    p.splits = splits;
    p.kb_per_split = (int) (KB / splits);
    p.ws = splits > 1 ? (float *) ws : nullptr;
    p.tickets = splits > 1 ? tickets : nullptr;
    static int configured = 0;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_0_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
        if (e != cudaSuccess) return e;
        configured = 1;
    }
    gemm_q8_0_tc_kernel<NT><<<dim3(tn, tm, splits), kTcThreads, L::kTotal, st>>>(ta, tb, tdw, tdx, p);
    return cudaGetLastError();
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void * p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000) p;
    });
    return fn;
}

// Encoded maps are cached by their arguments: a product re-encodes nothing when its weight and scratch are the same.
struct MapKey {
    const void * base;
    uint64_t inner, outer, row_bytes;
    uint32_t box_inner, box_outer;
    int dt, sw;
    bool operator==(const MapKey & o) const { return std::memcmp(this, &o, sizeof o) == 0; }
};

bool make_map_2d_uncached(CUtensorMap * m, CUtensorMapDataType dt, const void * base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);

bool make_map_2d(CUtensorMap * m, CUtensorMapDataType dt, const void * base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    constexpr int kSlots = 64;
    static std::mutex mu;
    static MapKey keys[kSlots];
    static CUtensorMap maps[kSlots];
    static int used = 0, next = 0;
    MapKey k;
    std::memset(&k, 0, sizeof k);
    k.base = base;
    k.inner = inner;
    k.outer = outer;
    k.row_bytes = row_bytes;
    k.box_inner = box_inner;
    k.box_outer = box_outer;
    k.dt = (int) dt;
    k.sw = (int) sw;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; i++)
        if (keys[i] == k) {
            *m = maps[i];
            return true;
        }
    if (!make_map_2d_uncached(m, dt, base, inner, outer, row_bytes, box_inner, box_outer, sw)) return false;
    keys[next] = k;
    maps[next] = *m;
    next = (next + 1) % kSlots;
    if (used < kSlots) used++;
    return true;
}

bool make_map_2d_uncached(CUtensorMap * m, CUtensorMapDataType dt, const void * base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn || ((uintptr_t) base & 15) || row_bytes % 16) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tensor_maps_available() { return encode_fn() != nullptr; }

bool gemm_tc_supported(const WeightView & w, int64_t M) {
    return w.type == B200_TYPE_Q8_0 && M >= 32 && w.K % (32 * kTcKB) == 0 && w.K <= (int64_t) 1 << 30 && encode_fn() != nullptr;
}

int64_t gemm_tc_tiles(int64_t N, int64_t M) { return ((N + kTcM - 1) / kTcM) * ((M + 63) / 64); }

// partial tiles for up to 16 K splits
size_t gemm_tc_workspace_bytes(int64_t N, int64_t M) { return (size_t) gemm_tc_tiles(N, M) * 16 * 64 * kTcM * 4; }

int64_t gemm_tc_dx_ld(int64_t M) { return (M + 3) & ~(int64_t) 3; }

cudaError_t launch_gemm_tc(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dxT, int64_t M, float * y,
                           int64_t ldy, unsigned * err, void * ws, size_t ws_bytes, unsigned * tickets, int num_sms, cudaStream_t st) {
    return launch_nt<64>(w, row0, N, q, dxT, gemm_tc_dx_ld(M), M, y, ldy, err, ws, ws_bytes, tickets, num_sms, st);
}


}  // namespace b200
