// moe.cu — routing and glue of the tensor-core expert path (TextModel::experts, src/families/drama3/text-model.cpp:198-221;
// MUL_MAT_ID, src/common/graph.h:22-26): pairs sorted by expert into 16-slot-padded segments, activations quantized in
// slot order, SwiGLU re-quantization between the two expert products, and the router-weighted combine.
#include "internal.h"

namespace b200 {

// One CTA: histogram of the local experts' pairs, exclusive scans of the counts rounded up to 16 (segment starts) and
// of the segments' tile counts, placement of every pair in its expert's segment, the padding slots marked empty, and
// the list of token tiles (16 or 32 slots each, in expert order; .w = how many of them hold routed pairs). Pair p = t * top_k + s reads activation row
// t * nb1 + (nb1 == 1 ? 0 : s). Pairs of experts outside [e0, e0 + E) are skipped (another shard's); ids outside
// [0, total) are reported. inv[p] = the pair's slot, or -1.
__global__ void moe_route_kernel(const int32_t * __restrict__ ids, int64_t P, int64_t top_k, int64_t nb1, int E, int e0, int total,
                                 int32_t * grp_off, int32_t * col_src, int32_t * col_dst, int32_t * inv, int4 * tiles, int * ntiles,
                                 unsigned * err) {
    pdl_wait();  // launched with programmatic dependent launch: the previous kernel's writes are visible after this
    pdl_launch_dependents();
    extern __shared__ int sh[];
    int * cnt = sh;            // [E] pairs
    int * pos = sh + E;        // [E] placement cursor
    int * start = sh + 2 * E;  // [E] segment start
    int * toff = sh + 3 * E;   // [E] first tile
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
        inv[p] = -1;
        const int g = ids[p];
        if (g < 0 || g >= total) {
            atomicOr(err, B200_DEVERR_EXPERT);
            continue;
        }
        const int e = g - e0;
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        int carry = 0, tcarry = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + (int) threadIdx.x;
            const int len = e < E ? (cnt[e] + 15) & ~15 : 0;
            const int nt = (len + 31) / 32;
            int incl = len, tincl = nt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, incl, o);
                const int b = __shfl_up_sync(0xffffffffu, tincl, o);
                if ((int) threadIdx.x >= o) {
                    incl += a;
                    tincl += b;
                }
            }
            if (e < E) {
                start[e] = pos[e] = grp_off[e] = carry + incl - len;
                toff[e] = tcarry + tincl - nt;
            }
            carry += __shfl_sync(0xffffffffu, incl, 31);
            tcarry += __shfl_sync(0xffffffffu, tincl, 31);
        }
        if (threadIdx.x == 0) {
            grp_off[E] = carry;
            *ntiles = tcarry;
        }
    }
    __syncthreads();
    for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
        const int g = ids[p];
        const int e = g - e0;
        if (g < 0 || g >= total || e < 0 || e >= E) continue;
        const int slot = atomicAdd(&pos[e], 1);
        const int64_t t = p / top_k, s = p % top_k;
        col_src[slot] = (int32_t) (t * nb1 + (nb1 == 1 ? 0 : s));
        col_dst[slot] = (int32_t) p;
        inv[p] = slot;
    }
    __syncthreads();
    // padding slots (pos[e] is now the end of expert e's pairs) and the expert's token tiles
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int len = (cnt[e] + 15) & ~15;
        for (int slot = pos[e]; slot < start[e] + len; slot++) {
            col_src[slot] = -1;
            col_dst[slot] = -1;
        }
        for (int o = 0, k = toff[e]; o < len; o += 32, k++)
            tiles[k] = make_int4(e, start[e] + o, min(32, len - o), max(0, min(32, cnt[e] - o)));
    }
}

// q8_0 quantization of each slot's activation row (zeros for padding), in slot order: q [slots][K], dT [K/32][ldP].
// One warp per slot row, 128 values per step (a block per 8 lanes); bit-identical to the CPU backend's
// quantize_row_q8_0 of the same row. vec: x and ldx allow 16-byte loads.
template <int U>
__global__ void moe_quant_slots_kernel(const float * __restrict__ x, int64_t K, int64_t ldx, int vec, const int32_t * __restrict__ col_src,
                                       const int32_t * __restrict__ n_slots, int8_t * q, float * dT, int64_t ldP) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int S = *n_slots;
    for (int slot = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); slot < S; slot += warps) {
        const int32_t src = col_src[slot];
        const float * xr = src >= 0 ? x + (int64_t) src * ldx : nullptr;
        for (int64_t k0 = 0; k0 < K; k0 += 128 * U) {
            float4 v[U];  // U loads in flight before any arithmetic
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t k = k0 + 128 * u + 4 * lane;
                v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (xr && k < K) v[u] = vec ? *reinterpret_cast<const float4 *>(xr + k) : make_float4(xr[k], xr[k + 1], xr[k + 2], xr[k + 3]);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t k = k0 + 128 * u + 4 * lane;
                if (k0 + 128 * u >= K) break;
                float d;
                const uint32_t packed = quantize_q8_0_quad(v[u], &d);
                if (k < K) {
                    *reinterpret_cast<uint32_t *>(q + (int64_t) slot * K + k) = packed;
                    if ((lane & 7) == 0) dT[(k >> 5) * ldP + slot] = d;
                }
            }
        }
    }
}

// SwiGLU of each slot's gate|up row (gu [slots][2F]: gate F, then up F), re-quantized to q8_0 in slot order for the
// down product: q [slots][F], dT [F/32][ldP]; zeros for padding. One warp per slot row, 128 values per step.
template <int U>
__global__ void moe_swiglu_slots_kernel(const float * __restrict__ gu, int64_t F, const int32_t * __restrict__ col_src,
                                        const int32_t * __restrict__ n_slots, int8_t * q, float * dT, int64_t ldP) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int S = *n_slots;
    for (int slot = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); slot < S; slot += warps) {
        const bool live = col_src[slot] >= 0;
        const float * row = gu + (int64_t) slot * 2 * F;
        for (int64_t k0 = 0; k0 < F; k0 += 128 * U) {
            float4 g[U], u4[U];  // U gate and up loads in flight before any arithmetic
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t k = k0 + 128 * u + 4 * lane;
                g[u] = u4[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (live && k < F) {
                    g[u] = *reinterpret_cast<const float4 *>(row + k);
                    u4[u] = *reinterpret_cast<const float4 *>(row + F + k);
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t k = k0 + 128 * u + 4 * lane;
                if (k0 + 128 * u >= F) break;
                const float4 v = make_float4(__fmul_rn(silu(g[u].x), u4[u].x), __fmul_rn(silu(g[u].y), u4[u].y),
                                             __fmul_rn(silu(g[u].z), u4[u].z), __fmul_rn(silu(g[u].w), u4[u].w));
                float d;
                const uint32_t packed = quantize_q8_0_quad(v, &d);
                if (k < F) {
                    *reinterpret_cast<uint32_t *>(q + (int64_t) slot * F + k) = packed;
                    if ((lane & 7) == 0) dT[(k >> 5) * ldP + slot] = d;
                }
            }
        }
    }
}

// out[t] = sum over s (slot order) of w[t][s] * down row of pair (t, s), over the pairs this shard computed.
// vec: out allows 16-byte stores and H % 4 == 0.
__global__ void moe_combine_slots_kernel(const float * __restrict__ down, const float * __restrict__ w, const int32_t * __restrict__ inv,
                                         int64_t top_k, int64_t H, int vec, float * __restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    extern __shared__ int cslot[];  // [top_k] slots, then [top_k] weights
    float * cw = reinterpret_cast<float *>(cslot + top_k);
    const int64_t t = blockIdx.x;
    for (int64_t s = threadIdx.x; s < top_k; s += blockDim.x) {
        cslot[s] = inv[t * top_k + s];
        cw[s] = w[t * top_k + s];
    }
    __syncthreads();
    if (vec) {
        for (int64_t h = 4 * (int64_t) threadIdx.x; h < H; h += 4 * (int64_t) blockDim.x) {
            float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            bool any = false;
            for (int64_t s0 = 0; s0 < top_k; s0 += 8) {
                float4 d[8];  // eight rows in flight
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int64_t s = s0 + u;
                    d[u] = (s < top_k && cslot[s] >= 0) ? *reinterpret_cast<const float4 *>(down + (int64_t) cslot[s] * H + h)
                                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int64_t s = s0 + u;
                    if (s >= top_k || cslot[s] < 0) continue;
                    const float ws = cw[s];
                    const float4 v = make_float4(__fmul_rn(d[u].x, ws), __fmul_rn(d[u].y, ws), __fmul_rn(d[u].z, ws), __fmul_rn(d[u].w, ws));
                    sum = any ? make_float4(__fadd_rn(sum.x, v.x), __fadd_rn(sum.y, v.y), __fadd_rn(sum.z, v.z), __fadd_rn(sum.w, v.w)) : v;
                    any = true;
                }
            }
            *reinterpret_cast<float4 *>(out + t * H + h) = sum;
        }
        return;
    }
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
        float sum = 0.0f;
        bool any = false;
        for (int64_t s = 0; s < top_k; s++) {
            const int32_t slot = cslot[s];
            if (slot < 0) continue;
            const float v = __fmul_rn(down[(int64_t) slot * H + h], cw[s]);
            sum = any ? __fadd_rn(sum, v) : v;
            any = true;
        }
        out[t * H + h] = sum;
    }
}

// Launches a kernel with programmatic dependent launch (its CTAs may start while the previous kernel finishes; every
// kernel here calls griddepcontrol.wait before reading anything a previous kernel wrote).
template <class... Params, class... Args>
static cudaError_t launch_pdl(void (*kern)(Params...), unsigned grid, unsigned block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(block, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}

int64_t moe_max_slots(int64_t P, int64_t E) { return ((P + 15 * E) + 15) & ~(int64_t) 15; }
int64_t moe_max_tiles(int64_t P, int64_t E) { return moe_max_slots(P, E) / 16 + E + 1; }

cudaError_t launch_moe_route(const int32_t * ids, int64_t T, int64_t top_k, int64_t nb1, int64_t E, int64_t e0, int64_t total,
                             int32_t * grp_off, int32_t * col_src, int32_t * col_dst, int32_t * inv, int4 * tiles, int * ntiles,
                             unsigned * err, cudaStream_t st) {
    return launch_pdl(moe_route_kernel, 1, 1024, (size_t) 4 * E * sizeof(int), st, ids, T * top_k, top_k, nb1, (int) E, (int) e0,
                      (int) (total > 0 ? total : E), grp_off, col_src, col_dst, inv, tiles, ntiles, err);
}

static unsigned glue_blocks(int64_t work_warps, int num_sms) {
    // one warp per slot row, eight warps per block
    int64_t blocks = (work_warps + 7) / 8;
    const int64_t cap = (int64_t) num_sms * 8;
    if (blocks > cap) blocks = cap;
    return (unsigned) (blocks < 1 ? 1 : blocks);
}

cudaError_t launch_moe_quant_slots(const float * x, int64_t K, int64_t ldx, const int32_t * col_src, const int32_t * n_slots,
                                   int64_t max_slots, int8_t * q, float * dT, int64_t ldP, int num_sms, cudaStream_t st) {
    const int vec = ((uintptr_t) x % 16 == 0 && ldx % 4 == 0) ? 1 : 0;
    return launch_pdl(moe_quant_slots_kernel<8>, glue_blocks(max_slots, num_sms), 256, 0, st, x, K, ldx, vec, col_src, n_slots, q, dT, ldP);
}

cudaError_t launch_moe_swiglu_slots(const float * gu, int64_t F, const int32_t * col_src, const int32_t * n_slots, int64_t max_slots,
                                    int8_t * q, float * dT, int64_t ldP, int num_sms, cudaStream_t st) {
    return launch_pdl(moe_swiglu_slots_kernel<4>, glue_blocks(max_slots, num_sms), 256, 0, st, gu, F, col_src, n_slots, q, dT, ldP);
}

cudaError_t launch_moe_combine_slots(const float * down, const float * w, const int32_t * inv, int64_t T, int64_t top_k, int64_t H,
                                     float * out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int vec = ((uintptr_t) out % 16 == 0 && H % 4 == 0) ? 1 : 0;
    return launch_pdl(moe_combine_slots_kernel, (unsigned) T, 256, (size_t) top_k * 8, st, down, w, inv, top_k, H, vec, out);
}

}  // namespace b200
