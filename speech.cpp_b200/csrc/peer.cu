// peer.cu — the combine step of expert parallelism over NVLink peer memory: the router-weighted sum of this rank's
// experts (TextModel::experts, src/families/drama3/text-model.cpp:198-221) fused with a two-shot all-reduce.
//
// Every rank of an expert-parallel group holds a "mailbox" device buffer (cudaMalloc, shared with the other ranks by
// CUDA IPC handles): inbox [G][Ts][H] float (partial sums of the owner's token slice from each rank), final [T][H]
// float (the reduced output), and two arrival counters. Token slice g = tokens [g Ts, (g + 1) Ts) belongs to rank g.
// One cooperative kernel per layer:
//   1. every CTA computes its tokens' partial sums over this rank's experts and stores each token's row into the
//      owner's inbox (a plain store through the peer mapping; the owner's own rows stay local);
//   2. once every CTA of every rank has stored its rows, the CTAs sum their share of this rank's slice over the G
//      inboxes in rank order (the result does not depend on timing) and store the sums into every rank's final
//      buffer;
//   3. once every rank's sums are stored, the CTAs copy final to the caller's output.
// Arrival: after a CTA barrier, one thread per CTA makes the CTA's stores visible at system scope (one fence per
// CTA) and counts the CTA in a local counter; the CTA that completes the count tells every rank with one system-scope
// release each (G remote updates per step). Counters only grow: the targets of call k are (k + 1) x CTAs locally and
// (k + 1) x G remotely, k a device word this rank advances at the end of the call, so no reset is needed between
// layers or steps (also under graph replay). A rank starts writing call k + 1 only after every rank finished reading
// call k (step 3 waits for all of step 2).
// Every wait is bounded in time (the group's limit, 2 s unless set). A wait that gives up records B200_DEVERR_TIMEOUT
// and marks the group broken: the counters of the ranks are then out of step, so every later call on the group
// returns at once with the same error (b200_synchronize reports B200_ERR_TIMEOUT) until the group is destroyed and a
// new one created. No multicast, no NVLS: plain peer loads and stores.
#include "internal.h"

namespace b200 {

// The device side of a b200_ep_group: every rank's mailbox parts.
struct PeerGroupDev {
    float * inbox[kEpMaxRanks];      // rank g's inbox
    float * final_[kEpMaxRanks];     // rank g's final buffer
    unsigned * flags[kEpMaxRanks];   // rank g's counters: [0] step 1 arrivals, [1] step 2 arrivals
};

namespace {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_sys(unsigned * p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (one thread) until *p >= target; false once timeout_ns have passed (or after 2^26 polls, whichever first).
__device__ __forceinline__ bool wait_at_least(const unsigned * p, unsigned target, uint64_t timeout_ns) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < (1u << 26); i++) {
        if ((int) (ld_acquire_sys(p) - target) >= 0) return true;
        if ((i & 63) == 63 && global_ns() - t0 > timeout_ns) return false;
        if (i > 512) __nanosleep(32);
    }
    return false;
}

// This CTA's part of a step is stored (the caller has passed a CTA barrier): one system-scope fence makes it visible
// beyond this GPU, then the CTA counts itself; the CTA that completes the count tells every rank.
__device__ __forceinline__ void arrive_all(unsigned * local, unsigned local_target, unsigned * const * flags, int G, int which) {
    __threadfence_system();
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(local), "r"(1u) : "memory");
    if (old + 1u == local_target)
        for (int g = 0; g < G; g++) red_release_sys(&flags[g][which], 1u);
}

// state: [0] calls completed (the counters' epoch), [1] [2] this rank's CTAs done with steps 1 and 2, [3] broken.
__global__ void __launch_bounds__(256) moe_combine_allreduce_kernel(const float * __restrict__ down, const float * __restrict__ w,
                                                                    const int32_t * __restrict__ inv, int T, int top_k, int H,
                                                                    int rank, int G, int Ts, PeerGroupDev grp, unsigned * state,
                                                                    uint64_t timeout_ns, float * __restrict__ out, unsigned * err) {
    __shared__ int ok;
    const int nct = gridDim.x, c = blockIdx.x;
    const unsigned k = *reinterpret_cast<volatile unsigned *>(state);
    if (*reinterpret_cast<volatile unsigned *>(state + 3)) {  // a wait of an earlier call gave up: refuse at once
        if (c == 0 && threadIdx.x == 0) atomicOr(err, B200_DEVERR_TIMEOUT);
        return;
    }
    const unsigned target = (k + 1u) * (unsigned) G;         // remote arrivals: one per rank per call
    const unsigned local_target = (k + 1u) * (unsigned) nct;  // this rank's CTAs per call
    const int H4 = H / 4;
    // ---- 1. partial sums of this rank's experts, pushed to each token's owner ----
    for (int t = c; t < T; t += nct) {
        const int g = t / Ts, tl = t - g * Ts;
        float4 * dst = reinterpret_cast<float4 *>(grp.inbox[g] + ((int64_t) rank * Ts + tl) * H);
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
            dst[h4] = sum;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        arrive_all(&state[1], local_target, grp.flags, G, 0);
        ok = wait_at_least(&grp.flags[rank][0], target, timeout_ns);
    }
    __syncthreads();
    if (ok) {
        // ---- 2. this rank's slice: sum over the G inboxes in rank order, stored to every rank's final buffer ----
        const int t0 = rank * Ts, t1 = min(T, t0 + Ts);
        for (int t = t0 + c; t < t1; t += nct) {
            const int tl = t - t0;
            for (int h4 = threadIdx.x; h4 < H4; h4 += blockDim.x) {
                // written by other GPUs since the last call: read through L2 (__ldcg), never from a stale L1 line
                float4 v[kEpMaxRanks];
#pragma unroll
                for (int g = 0; g < kEpMaxRanks; g++)
                    if (g < G) v[g] = __ldcg(reinterpret_cast<const float4 *>(grp.inbox[rank] + ((int64_t) g * Ts + tl) * H) + h4);
                float4 sum = v[0];
#pragma unroll
                for (int g = 1; g < kEpMaxRanks; g++)
                    if (g < G) sum = make_float4(__fadd_rn(sum.x, v[g].x), __fadd_rn(sum.y, v[g].y), __fadd_rn(sum.z, v[g].z), __fadd_rn(sum.w, v[g].w));
                for (int g = 0; g < G; g++) reinterpret_cast<float4 *>(grp.final_[g] + (int64_t) t * H)[h4] = sum;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            arrive_all(&state[2], local_target, grp.flags, G, 1);
            ok = wait_at_least(&grp.flags[rank][1], target, timeout_ns);
        }
        __syncthreads();
    }
    if (ok) {
        // ---- 3. the reduced output, every token ----
        for (int t = c; t < T; t += nct) {
            const float4 * src = reinterpret_cast<const float4 *>(grp.final_[rank] + (int64_t) t * H);
            float4 * o = reinterpret_cast<float4 *>(out + (int64_t) t * H);
            for (int h4 = threadIdx.x; h4 < H4; h4 += blockDim.x) o[h4] = __ldcg(src + h4);
        }
    } else if (threadIdx.x == 0) {
        atomicOr(err, B200_DEVERR_TIMEOUT);
        atomicExch(state + 3, 1u);  // the ranks' counters are out of step from here on
    }
    // the call is over for this CTA; CTA 0 advances the call count once every CTA of this rank is past step 2 (the
    // step 2 wait proves it: all CTAs of all ranks arrived there after reading k)
    if (c == 0 && threadIdx.x == 0) atomicAdd(state, 1u);
}

}  // namespace

size_t peer_mailbox_bytes(int G, int T_max, int H) {
    const int Ts = (T_max + G - 1) / G;
    return (((size_t) G * Ts * H * 4 + 255) & ~(size_t) 255) + (((size_t) T_max * H * 4 + 255) & ~(size_t) 255) + 256;
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
        grp.inbox[g] = (float *) base;
        grp.final_[g] = (float *) (base + (((size_t) ep->G * Ts * ep->H * 4 + 255) & ~(size_t) 255));
        grp.flags[g] = (unsigned *) (base + (((size_t) ep->G * Ts * ep->H * 4 + 255) & ~(size_t) 255) +
                                     (((size_t) ep->T_max * ep->H * 4 + 255) & ~(size_t) 255));
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_combine_allreduce_kernel, 256, 0);
    if (e != cudaSuccess) return e;
    const int nct = num_sms < per_sm * num_sms ? num_sms : per_sm * num_sms;  // one CTA per SM: all co-resident
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
    if (cudaMalloc(&g->calls, 4 * sizeof(unsigned)) != cudaSuccess || cudaMemset(g->calls, 0, 4 * sizeof(unsigned)) != cudaSuccess) {
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
