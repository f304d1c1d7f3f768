// gemm_tc.cu — Q8_0 products with many activation rows (M >= 32: prefill, audio-encoder, multi-stream decode) on the
// 5th-generation tensor cores: tcgen05.mma kind::i8 with int32 accumulators in tensor memory, fed by TMA.
//
// ggml's CPU backend computes these as per-32-block int32 dot products of the Q8_0 weights with q8_0-quantized
// activations, each scaled by d_w * d_x and summed in float32. Here one tcgen05.mma of shape M=128 (weight rows) x
// N=NT (tokens) x K=32 computes exactly the int32 sums of ONE block for a 128 x NT tile ("swap AB": weights on the M
// side, since decode batches are small). The accumulator lives in tensor memory, double-buffered: while block b+1
// multiplies into one buffer, four epilogue warps read block b's int32 sums out of the other (tcgen05.ld), scale them
// by d_w[row][b] * d_x[token][b] and add them to float32 registers. Operands arrive by TMA (2-D tensor maps, one
// box per 32-wide K block, 32-byte swizzle that the MMA's shared-memory descriptors read as is; no multicast).
// Warp roles: 0 = TMA producer, 1 = tensor-memory allocator and MMA issuer (one thread), 2..5 = epilogue.
// Split-K: with S > 1, CTAs of one tile sum disjoint K ranges; each writes its partial tile to a workspace and the
// last to finish (an atomic ticket) adds the S partials in split order, so results do not depend on timing.
// Every wait is bounded; one that gives up records B200_DEVERR_TIMEOUT and the CTA runs to its end (freeing its
// tensor memory) without further waits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace b200 {

namespace {

constexpr int kTcM = 128;          // weight rows per tile (MMA M)
constexpr int kTcKB = 8;           // 32-wide K blocks per pipeline stage
constexpr int kTcStages = 3;
constexpr int kTcThreads = 192;    // 6 warps
constexpr unsigned kErrTimeout = 4u;

template <int NT>
struct TcLayout {
    static constexpr int kA = kTcKB * kTcM * 32;       // weight int8 tiles, one 4 KB tile per K block
    static constexpr int kB = kTcKB * NT * 32;         // activation int8 tiles
    static constexpr int kDw = kTcM * kTcKB * 2;       // fp16 weight scales [128][KB]
    static constexpr int kDx = NT * kTcKB * 4;         // f32 activation scales [NT][KB]
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

__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * map, int c0, int c1, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile of rows x 32 int8 written by TMA with 32-byte swizzle:
// start address >> 4, leading byte offset 16 B (unused by swizzled K-major layouts), stride byte offset 256 B
// (eight 32-byte rows), descriptor version 1, layout SWIZZLE_32B (6).
__device__ __forceinline__ uint64_t smem_desc_sw32(const void * tile) {
    const uint64_t a = (uint64_t) (smem_addr(tile) & 0x3FFFF) >> 4;
    return a | (1ull << 16) | (16ull << 32) | (1ull << 46) | (6ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::i8: D s32, A s8, B s8, both K-major, N = NT, M = 128.
template <int NT>
__device__ __forceinline__ uint32_t idesc_i8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (NT >> 3) << 17) | ((uint32_t) (kTcM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc)
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

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_q8_0_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmDw, const __grid_constant__ CUtensorMap tmDx, TcParams p) {
    using L = TcLayout<NT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t) 1023);
    uint64_t * bars = reinterpret_cast<uint64_t *>(smem + kTcStages * L::kStage);
    uint64_t * full = bars;                      // [stages] TMA landed
    uint64_t * empty = bars + kTcStages;         // [stages] MMAs done + epilogue done with the scales
    uint64_t * acc_full = bars + 2 * kTcStages;  // [2] block's int32 sums ready in tensor memory
    uint64_t * acc_empty = acc_full + 2;         // [2] epilogue has read them
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
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
            mbar_init(&empty[s], 1 + 4);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        fence_mbar_init();
        give_up = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)), "r"(2 * NT));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer ----
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
                for (int j = 0; j < kTcKB; j++) {
                    tma_load_2d(base + j * kTcM * 32, &tmA, (kbs + j) * 32, (int) (p.row0 + (int64_t) tile_n * kTcM), &full[s]);
                    tma_load_2d(base + L::kA + j * NT * 32, &tmB, (kbs + j) * 32, tile_m * NT, &full[s]);
                }
                tma_load_2d(base + L::kA + L::kB, &tmDw, kbs, (int) (p.row0 + (int64_t) tile_n * kTcM), &full[s]);
                tma_load_2d(base + L::kA + L::kB + L::kDw, &tmDx, kbs, tile_m * NT, &full[s]);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: one block (K = 32) per MMA, into the tensor-memory buffer b % 2 ----
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
                    const int buf = b & 1, use = b >> 1;
                    if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1)) {
                        atomicOr(p.err, kErrTimeout);
                        give_up = 1;
                        break;
                    }
                    tc_fence_after();
                    mma_i8(tmem + buf * NT, smem_desc_sw32(base + j * kTcM * 32), smem_desc_sw32(base + L::kA + j * NT * 32), idesc);
                    mma_commit(&acc_full[buf]);
                }
                if (give_up) break;
                mma_commit(&empty[s]);  // the stage's operands are free once these MMAs complete
            }
        }
    } else {
        // ---- epilogue: warps 2..5, lane quarter q = warp % 4, tile row 32 q + lane ----
        const int q = warp & 3;
        const int row = 32 * q + lane;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.0f;
        int b = 0;
        for (int st = 0; st < nstage && !give_up; st++) {
            const int s = st % kTcStages;
            const uint8_t * base = smem + s * L::kStage;
            const __half * dw = reinterpret_cast<const __half *>(base + L::kA + L::kB);
            const float * dx = reinterpret_cast<const float *>(base + L::kA + L::kB + L::kDw);
            for (int j = 0; j < kTcKB; j++, b++) {
                const int buf = b & 1, use = b >> 1;
                if (!mbar_wait(&acc_full[buf], use & 1)) {
                    if (lane == 0) atomicOr(p.err, kErrTimeout);
                    give_up = 1;
                    break;
                }
                tc_fence_after();
                int v[NT];
#pragma unroll
                for (int c = 0; c < NT; c += 32) tmem_ld32(tmem + ((uint32_t) (32 * q) << 16) + buf * NT + c, v + c);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
                const float dwr = __half2float(dw[row * kTcKB + j]);
#pragma unroll
                for (int t = 0; t < NT; t++) acc[t] = fmaf((float) v[t], __fmul_rn(dwr, dx[t * kTcKB + j]), acc[t]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // ---- output (direct, or split-K partial + ordered reduction by the last split) ----
        const int64_t grow = (int64_t) tile_n * kTcM + row;  // row of this product
        const int tiles = gridDim.x * gridDim.y;
        const int tile = tile_m * gridDim.x + tile_n;
        if (p.splits == 1) {
            if (grow < p.N)
                for (int t = 0; t < NT; t++) {
                    const int64_t m = (int64_t) tile_m * NT + t;
                    if (m < p.M) p.y[m * p.ldy + grow] = acc[t];
                }
        } else {
            float * part = p.ws + ((int64_t) tile * p.splits + split) * NT * kTcM;
            for (int t = 0; t < NT; t++) part[t * kTcM + row] = acc[t];
            __threadfence();
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (warp == 2 && lane == 0) {
                const unsigned ticket = atomicAdd(&p.tickets[tile], 1u);
                last_split = ticket == (unsigned) (p.splits - 1);
                if (last_split) p.tickets[tile] = 0;  // ready for the next launch
            }
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (last_split) {
                __threadfence();
                if (grow < p.N)
                    for (int t = 0; t < NT; t++) {
                        float sum = 0.0f;
                        for (int z = 0; z < p.splits; z++) sum += __ldcg(p.ws + ((int64_t) tile * p.splits + z) * NT * kTcM + t * kTcM + row);
                        const int64_t m = (int64_t) tile_m * NT + t;
                        if (m < p.M) p.y[m * p.ldy + grow] = sum;
                    }
            }
            (void) tiles;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NT));
    }
}

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

bool make_map_2d(CUtensorMap * m, CUtensorMapDataType dt, const void * base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn || ((uintptr_t) base & 15) || row_bytes % 16) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT>
cudaError_t launch_nt(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dx, int64_t M, float * y,
                      int64_t ldy, unsigned * err, void * ws, size_t ws_bytes, unsigned * tickets, int num_sms, cudaStream_t st) {
    using L = TcLayout<NT>;
    const int64_t K = w.K, KB = K / 32;
    CUtensorMap ta, tb, tdw, tdx;
    if (!make_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.f0, (uint64_t) K, (uint64_t) w.rows, (uint64_t) K, 32, kTcM,
                     CU_TENSOR_MAP_SWIZZLE_32B) ||
        !make_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, (uint64_t) K, (uint64_t) M, (uint64_t) K, 32, NT, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !make_map_2d(&tdw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.f1, (uint64_t) KB, (uint64_t) w.rows, (uint64_t) KB * 2, kTcKB, kTcM,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&tdx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dx, (uint64_t) KB, (uint64_t) M, (uint64_t) KB * 4, kTcKB, NT,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    const int tn = (int) ((N + kTcM - 1) / kTcM), tm = (int) ((M + NT - 1) / NT);
    const int stages_total = (int) (KB / kTcKB);
    // split K so that the grid covers the SMs, in whole stages, dividing the stages evenly
    int splits = 1;
    while (splits * 2 <= stages_total && (int64_t) tn * tm * splits < num_sms && stages_total % (splits * 2) == 0) splits *= 2;
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

bool gemm_tc_supported(const WeightView & w, int64_t M) {
    return w.type == B200_TYPE_Q8_0 && M >= 32 && w.K % (32 * kTcKB) == 0 && w.K <= (int64_t) 1 << 30 && encode_fn() != nullptr;
}

int64_t gemm_tc_tiles(int64_t N, int64_t M) { return ((N + kTcM - 1) / kTcM) * ((M + 63) / 64); }

// partial tiles for up to 16 K splits
size_t gemm_tc_workspace_bytes(int64_t N, int64_t M) { return (size_t) gemm_tc_tiles(N, M) * 16 * 64 * kTcM * 4; }

cudaError_t launch_gemm_tc(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dx, int64_t M, float * y,
                           int64_t ldy, unsigned * err, void * ws, size_t ws_bytes, unsigned * tickets, int num_sms, cudaStream_t st) {
    return launch_nt<64>(w, row0, N, q, dx, M, y, ldy, err, ws, ws_bytes, tickets, num_sms, st);
}

}  // namespace b200
