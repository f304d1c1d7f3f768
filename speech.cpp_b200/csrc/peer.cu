// peer.cu — the combine step of expert parallelism over NVLink peer memory: the router-weighted sum of this rank's
// experts (TextModel::experts, src/families/drama3/text-model.cpp:198-221) fused with a two-shot all-reduce.
//
// Every rank of an expert-parallel group holds a "mailbox" device buffer (cudaMalloc, shared with the other ranks by
// CUDA IPC handles): inbox [G][Ts][H] and final [T][H], both of tagged words. Token slice g = tokens [g Ts, (g + 1) Ts)
// belongs to rank g. One cooperative kernel per layer (one CTA per SM, all resident):
//   1. every CTA computes its tokens' partial sums over this rank's experts and stores each token's row into the
//      owner's inbox (plain stores through the peer mapping; the owner's own rows stay local);
//   2. the CTAs sum their share of this rank's slice over the G inboxes in rank order (the result does not depend on
//      timing) and store the sums into every rank's final buffer;
//   3. the CTAs copy final to the caller's output.
// Every value travels with its call's tag in one 8-byte word {float bits, tag}, written by one store: a reader polls
// the words it needs until their tags are the current call's, so a value proves its own arrival and no fence, counter
// or barrier separates the steps (the stores of one word are single-copy atomic over NVLink as in local memory). The
// tag of call k is k + 1, k the calls this CTA has completed (a per-CTA device word): every CTA of every rank takes
// part in every call, so all agree. A rank writes call k + 1's inbox words only after it has read all of call k's
// final words, each stored by its owner after that owner had read the corresponding inbox words, so no word is
// overwritten before it has been read.
// Every poll is bounded in time (the group's limit, 2 s unless set). One that gives up records B200_DEVERR_TIMEOUT
// and marks the group broken: the ranks' call counts are then out of step, so every later call on the group returns at
// once with the same error (b200_synchronize reports B200_ERR_TIMEOUT) until the group is destroyed and a new one
// created. No multicast, no NVLS: plain peer loads and stores.
#include "internal.h"

namespace b200 {

// The device side of a b200_ep_group: every rank's mailbox parts.
struct PeerGroupDev {
    unsigned long long * inbox[kEpMaxRanks];   // rank g's inbox [G][Ts][H] of {value, tag}
    unsigned long long * final_[kEpMaxRanks];  // rank g's final buffer [T][H] of {value, tag}
};

namespace {

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long tagged(float v, unsigned tag) {
    return (unsigned long long) __float_as_uint(v) | ((unsigned long long) tag << 32);
}

// Two tagged words to (possibly peer) global memory, one 16-byte store.
__device__ __forceinline__ void st_pair(unsigned long long * p, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_pair(const unsigned long long * p, unsigned long long & a, unsigned long long & b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Polls two tagged words until both carry `tag`; false once timeout_ns have passed or another thread of the CTA gave
// up (failed).
__device__ __forceinline__ bool poll_pair(const unsigned long long * p, unsigned tag, uint64_t timeout_ns, volatile int * failed,
                                          float & x, float & y) {
    unsigned long long a, b;
    ld_pair(p, a, b);
    if ((unsigned) (a >> 32) == tag && (unsigned) (b >> 32) == tag) {
        x = __uint_as_float((unsigned) a);
        y = __uint_as_float((unsigned) b);
        return true;
    }
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1; i < (1u << 26); i++) {
        if (*failed) return false;
        ld_pair(p, a, b);
        if ((unsigned) (a >> 32) == tag && (unsigned) (b >> 32) == tag) {
            x = __uint_as_float((unsigned) a);
            y = __uint_as_float((unsigned) b);
            return true;
        }
        if ((i & 63) == 63 && global_ns() - t0 > timeout_ns) break;
        if (i > 256) __nanosleep(64);
    }
    *failed = 1;
    return false;
}

// state: [1] broken (a poll gave up), [kEpStateCtas + c] the calls CTA c has completed.
__global__ void __launch_bounds__(256) moe_combine_allreduce_kernel(const float * __restrict__ down, const float * __restrict__ w,
                                                                    const int32_t * __restrict__ inv, int T, int top_k, int H,
                                                                    int rank, int G, int Ts, PeerGroupDev grp, unsigned * state,
                                                                    uint64_t timeout_ns, float * __restrict__ out, unsigned * err) {
    __shared__ volatile int failed;
    const int nct = gridDim.x, c = blockIdx.x;
    if (*reinterpret_cast<volatile unsigned *>(state + 1)) {  // a poll of an earlier call gave up: refuse at once
        if (c == 0 && threadIdx.x == 0) atomicOr(err, B200_DEVERR_TIMEOUT);
        return;
    }
    if (threadIdx.x == 0) failed = 0;
    const unsigned tag = *reinterpret_cast<volatile unsigned *>(state + kEpStateCtas + c) + 1u;
    __syncthreads();
    const int H4 = H / 4, H2 = H / 2;
    // ---- 1. partial sums of this rank's experts, pushed to each token's owner ----
    for (int t = c; t < T; t += nct) {
        const int g = t / Ts, tl = t - g * Ts;
        unsigned long long * dst = grp.inbox[g] + ((int64_t) rank * Ts + tl) * H;
        for (int h4 = threadIdx.x; h4 < H4; h4 += blockDim.x) {
            float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            bool any = false;
            for (int s = 0; s < top_k; s++) {
                const int32_t slot = inv[(int64_t) t * top_k + s];
                if (slot < 0) continue;
                const float ws = w[(int64_t) t * top_k + s];
                const float4 d = reinterpret_cast<const float4 *>(down + (int64_t) slot * H)[h4];
                const float4 v = make_float4(__fmul_rn(d.x, ws), __fmul_rn(d.y, ws), __fmul_rn(d.z, ws), __fmul_rn(d.w, ws));
                sum = any ? make_float4(__fadd_rn(sum.x, v.x), __fadd_rn(sum.y, v.y), __fadd_rn(sum.z, v.z), __fadd_rn(sum.w, v.w)) : v;
                any = true;
            }
            st_pair(dst + 4 * h4, tagged(sum.x, tag), tagged(sum.y, tag));
            st_pair(dst + 4 * h4 + 2, tagged(sum.z, tag), tagged(sum.w, tag));
        }
    }
    // ---- 2. this rank's slice: the G ranks' partials summed in rank order, stored to every rank's final buffer ----
    const int t0 = rank * Ts, t1 = min(T, t0 + Ts);
    for (int t = t0 + c; t < t1 && !failed; t += nct) {
        const int tl = t - t0;
        for (int h2 = threadIdx.x; h2 < H2 && !failed; h2 += blockDim.x) {
            float sx = 0.0f, sy = 0.0f;
            for (int g = 0; g < G; g++) {
                float x, y;
                if (!poll_pair(grp.inbox[rank] + ((int64_t) g * Ts + tl) * H + 2 * h2, tag, timeout_ns, &failed, x, y)) break;
                sx = g ? __fadd_rn(sx, x) : x;
                sy = g ? __fadd_rn(sy, y) : y;
            }
            if (failed) break;
            const unsigned long long a = tagged(sx, tag), b = tagged(sy, tag);
            for (int g = 0; g < G; g++) st_pair(grp.final_[g] + (int64_t) t * H + 2 * h2, a, b);
        }
    }
    // ---- 3. the reduced output, every token ----
    for (int t = c; t < T && !failed; t += nct) {
        for (int h2 = threadIdx.x; h2 < H2 && !failed; h2 += blockDim.x) {
            float x, y;
            if (!poll_pair(grp.final_[rank] + (int64_t) t * H + 2 * h2, tag, timeout_ns, &failed, x, y)) break;
            reinterpret_cast<float2 *>(out + (int64_t) t * H)[h2] = make_float2(x, y);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (failed) {
            atomicOr(err, B200_DEVERR_TIMEOUT);
            atomicExch(state + 1, 1u);  // the ranks' call counts are out of step from here on
        }
        state[kEpStateCtas + c] = tag;  // this CTA's call is over
    }
}

}  // namespace

size_t peer_mailbox_bytes(int G, int T_max, int H) {
    const int Ts = (T_max + G - 1) / G;
    return (((size_t) G * Ts * H * 8 + 255) & ~(size_t) 255) + (((size_t) T_max * H * 8 + 255) & ~(size_t) 255);
}

cudaError_t launch_moe_combine_allreduce(const float * down, const float * w, const int32_t * inv, int64_t T, int64_t top_k, int64_t H,
                                         const b200_ep_group * ep, float * out, unsigned * err, int num_sms, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (!ep || H % 4 || T > ep->T_max || H != ep->H || ((uintptr_t) out & 15)) return cudaErrorInvalidValue;
    PeerGroupDev grp;
    std::memset(&grp, 0, sizeof grp);
    const int Ts = (int) ((ep->T_max + ep->G - 1) / ep->G);
    for (int g = 0; g < ep->G; g++) {
        uint8_t * base = (uint8_t *) ep->peer[g];
        grp.inbox[g] = (unsigned long long *) base;
        grp.final_[g] = (unsigned long long *) (base + (((size_t) ep->G * Ts * ep->H * 8 + 255) & ~(size_t) 255));
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_combine_allreduce_kernel, 256, 0);
    if (e != cudaSuccess) return e;
    int nct = num_sms < per_sm * num_sms ? num_sms : per_sm * num_sms;  // one CTA per SM: all co-resident
    if (nct > kEpMaxCtas) nct = kEpMaxCtas;
    int Ti = (int) T, ki = (int) top_k, Hi = (int) H, r = ep->rank, G = ep->G, Tsi = Ts;
    unsigned * state = ep->calls;
    uint64_t timeout_ns = ep->timeout_ns;
    void * args[] = {(void *) &down, (void *) &w, (void *) &inv, &Ti, &ki, &Hi, &r, &G, &Tsi, &grp, &state, &timeout_ns, (void *) &out, &err};
    return cudaLaunchCooperativeKernel((const void *) moe_combine_allreduce_kernel, dim3((unsigned) nct), dim3(256), args, 0, st);
}

}  // namespace b200

using namespace b200;

extern "C" {

b200_status b200_ep_mailbox_alloc(b200_context * ctx, int world, int64_t max_tokens, int64_t hidden, void ** mailbox, void * ipc_handle) {
    if (!ctx || !mailbox || !ipc_handle || world < 1 || world > kEpMaxRanks || max_tokens < 1 || hidden < 4 || hidden % 4) {
        if (ctx) ctx->last_error = "ep_mailbox_alloc: bad arguments";
        return B200_ERR_INVALID;
    }
    *mailbox = nullptr;
    const size_t bytes = peer_mailbox_bytes(world, (int) max_tokens, (int) hidden);
    cudaError_t e = cudaMalloc(mailbox, bytes);
    if (e == cudaSuccess) e = cudaMemset(*mailbox, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *mailbox);
    if (e != cudaSuccess) {
        if (*mailbox) cudaFree(*mailbox);
        *mailbox = nullptr;
        ctx->last_error = std::string("ep_mailbox_alloc: ") + cudaGetErrorString(e);
        return e == cudaErrorMemoryAllocation ? B200_ERR_ALLOC : B200_ERR_DEVICE;
    }
    std::memcpy(ipc_handle, &h, sizeof h);
    return B200_OK;
}

b200_status b200_ep_mailbox_open(b200_context * ctx, const void * ipc_handle, void ** peer_mailbox) {
    if (!ctx || !ipc_handle || !peer_mailbox) return B200_ERR_INVALID;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof h);
    const cudaError_t e = cudaIpcOpenMemHandle(peer_mailbox, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        ctx->last_error = std::string("ep_mailbox_open: ") + cudaGetErrorString(e);
        return B200_ERR_DEVICE;
    }
    return B200_OK;
}

b200_status b200_ep_mailbox_close(b200_context * ctx, void * peer_mailbox) {
    if (!ctx || !peer_mailbox) return B200_ERR_INVALID;
    return cudaIpcCloseMemHandle(peer_mailbox) == cudaSuccess ? B200_OK : B200_ERR_DEVICE;
}

b200_status b200_ep_mailbox_free(b200_context * ctx, void * mailbox) {
    if (!ctx || !mailbox) return B200_ERR_INVALID;
    return cudaFree(mailbox) == cudaSuccess ? B200_OK : B200_ERR_DEVICE;
}

b200_status b200_ep_create(b200_context * ctx, int rank, int world, int64_t max_tokens, int64_t hidden, void * const * mailboxes,
                           b200_ep_group ** out) {
    if (!ctx || !out || !mailboxes || world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world || max_tokens < 1 || hidden % 4) {
        if (ctx) ctx->last_error = "ep_create: bad arguments";
        return B200_ERR_INVALID;
    }
    b200_ep_group * g = new b200_ep_group();
    g->rank = rank;
    g->G = world;
    g->T_max = max_tokens;
    g->H = hidden;
    for (int i = 0; i < world; i++) g->peer[i] = mailboxes[i];
    const size_t cb = (kEpStateCtas + kEpMaxCtas) * sizeof(unsigned);
    if (cudaMalloc(&g->calls, cb) != cudaSuccess || cudaMemset(g->calls, 0, cb) != cudaSuccess) {
        delete g;
        ctx->last_error = "ep_create: device allocation";
        return B200_ERR_ALLOC;
    }
    *out = g;
    return B200_OK;
}

b200_status b200_ep_set_timeout(b200_ep_group * g, uint64_t microseconds) {
    if (!g || microseconds == 0) return B200_ERR_INVALID;
    g->timeout_ns = microseconds * 1000ull;
    return B200_OK;
}

void b200_ep_destroy(b200_ep_group * g) {
    if (!g) return;
    if (g->calls) cudaFree(g->calls);
    delete g;
}

}  // extern "C"
