// internal.h — host-side declarations shared by the backend's translation units (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <unordered_map>

#include "../../include/b200.h"
#include "common.cuh"
#include "gemv.cuh"

// Device error bits, OR-ed by kernels into b200_context::dev_err and reported by b200_synchronize().
#define B200_DEVERR_ROWS 1u     // GET_ROWS id out of range
#define B200_DEVERR_EXPERT 2u   // MUL_MAT_ID id out of range
#define B200_DEVERR_TIMEOUT 4u  // a bounded wait gave up

// An expert-parallel group's view of every rank's mailbox (peer.cu): inbox [G][ceil(T_max / G)][H] float, final
// [T_max][H] float, two arrival counters; peer[g] is rank g's mailbox mapped into this process (peer[rank] its own).
constexpr int kEpMaxRanks = 8;
constexpr int kEpStateCtas = 4;    // words of an expert-parallel group's state before the per-CTA call counts
constexpr int kEpMaxCtas = 1024;   // CTAs of the combine kernel at most (one per SM)

struct b200_ep_group {
    int rank = 0, G = 1;
    int64_t T_max = 0, H = 0;
    void * peer[kEpMaxRanks] = {};
    unsigned * calls = nullptr;  // [1]: the broken flag (a poll gave up); [kEpStateCtas + c]: the calls CTA c has
                                 // completed (its tags)
    uint64_t timeout_ns = 2000000000ull;  // how long one wait of the combine may take
};

// A K-quant weight expanded to int8 for the tensor cores (gemm_kq_tc.cu): one device allocation.
struct KqExpansion {
    int type = 0;
    void * mem = nullptr;
    size_t bytes = 0;
    int8_t * q = nullptr;      // planes [P][rows][K] with the scales inside: Q4_K (P = 3) (sc / 8) q, (sc % 8) q, m;
                               // Q6_K (P = 4) e_k (q - 32), sc's balanced base-5 digits e_k
    float * dd = nullptr;      // [rows][K/256][4]: d, dmin (Q4_K) or d (Q6_K)
};

struct b200_context {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::string last_error;
    unsigned * dev_err = nullptr;     // device word of B200_DEVERR_* bits
    unsigned * host_err = nullptr;    // pinned mirror
    void * scratch = nullptr;         // per-op scratch (quantized activations, routing tables)
    size_t scratch_bytes = 0;
    void * staging = nullptr;         // device staging for weight uploads
    size_t staging_bytes = 0;
    unsigned * tickets = nullptr;     // split-K tile tickets of the tensor-core GEMM (zero between launches)
    size_t ntickets = 0;
    // The last kernel launched on the stream wrote weight bytes (an upload). A product launched with programmatic
    // dependent launch reads weights before griddepcontrol.wait, so it must not directly follow an upload.
    bool upload_pending = false;
    // Expanded copies of K-quant weights used with many activation rows, by weight data pointer; dropped when the
    // weight is written or freed.
    std::unordered_map<const void *, KqExpansion> kq;
};

namespace b200 {

WeightView view_of(const b200_weight * w);
// Records the text b200_last_error(NULL) returns on this thread (errors outside any context).
void set_thread_error(const char * what);

// Kernel launchers (ops.cu). Each returns the launch's cudaError_t.
// ctas_per_sm > 0 caps the grid at num_sms * ctas_per_sm CTAs (leaves room for a dependent launch's CTAs).
cudaError_t launch_gemv(const GemvParams & p, int nc, int grid_y, cudaStream_t st, bool pdl, int num_sms, int ctas_per_sm = 0);
int gemv_max_columns(int wtype, int64_t K);  // largest NC whose staging fits in shared memory
cudaError_t launch_repack(int type, const b200_weight * w, const uint8_t * src, int64_t off0, int64_t n, bool to_device_layout,
                          uint8_t * gather_dst, cudaStream_t st);
cudaError_t launch_prefetch_l2(const void * base, size_t bytes, cudaStream_t st);
cudaError_t launch_get_rows(const WeightView & w, const int32_t * ids, int64_t n, float * dst, unsigned * err, cudaStream_t st);
// Activation quantization: gguf != null writes GGUF blocks there; else the internal layout (q, d, bs).
cudaError_t launch_quantize(int kind, const float * x, int64_t K, int64_t M, uint8_t * gguf, int8_t * q, float * d, int16_t * bs,
                            cudaStream_t st, int64_t dT_ld = 0);
// Tensor-core Q8_0 GEMM (gemm_tc.cu): x quantized to q (int8 [M][K]) and dxT (float [K/32][gemm_tc_dx_ld(M)], the
// block scales transposed so that one block's scales of all tokens are contiguous).
int64_t gemm_tc_dx_ld(int64_t M);
bool gemm_tc_supported(const WeightView & w, int64_t M);
size_t gemm_tc_workspace_bytes(int64_t N, int64_t M);
int64_t gemm_tc_tiles(int64_t N, int64_t M);
cudaError_t launch_gemm_tc(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dx, int64_t M, float * y,
                           int64_t ldy, unsigned * err, void * ws, size_t ws_bytes, unsigned * tickets, int num_sms, cudaStream_t st);
cudaError_t launch_route(const int32_t * ids, int64_t T, int64_t top_k, int64_t nb1, int64_t E, int32_t * grp_off,
                         int32_t * col_src, int32_t * col_dst, unsigned * err, cudaStream_t st, int64_t e0 = 0, int64_t total = 0,
                         int32_t * col_tok = nullptr);
cudaError_t launch_swiglu_quant_pairs(const float * gu, int64_t F, const int32_t * col_dst, const int32_t * n_pairs, int64_t max_pairs,
                                      int8_t * q, float * d, cudaStream_t st);
// q8_K of the SwiGLU rows (K-quant down experts): q [rows][F], d [rows][F/256], bs [rows][F/16]; F % 256 == 0.
cudaError_t launch_swiglu_quant_pairs_k(const float * gu, int64_t F, const int32_t * col_dst, const int32_t * n_pairs, int64_t max_pairs,
                                        int8_t * q, float * d, int16_t * bs, cudaStream_t st);
cudaError_t launch_moe_combine(const float * down, const float * w, const int32_t * ids, int64_t T, int64_t top_k, int64_t H, int64_t e0,
                               int64_t E, float * out, cudaStream_t st);
// Tensor-core expert products (gemm_tc_grouped.cu) and their routing/glue (moe.cu). Slots: pairs sorted by expert,
// each expert's segment padded to a multiple of 16; at most moe_max_slots(P, E) slots and moe_max_tiles(P, E) tiles.
bool gemm_tc_grouped_supported(const WeightView & w);
cudaError_t launch_gemm_tc_grouped(const WeightView & w, int64_t N, const int4 * tiles, const int * ntiles, const int8_t * q,
                                   const float * dT, int64_t ldP, int64_t slots, const int32_t * row_map, float * y, int64_t ldy,
                                   unsigned * err, int num_sms, cudaStream_t st);
// A dense Q8_0 product on the same kernel: q int8 [M][K] in token order, dT [K/32][ldP] (ldP % 16 == 0, >= M).
// Split-K (ksplit > 1): partial tiles in ws (gemm_tc_dense_ws_bytes) and one zeroed ticket per output tile.
int gemm_tc_dense_splits(const WeightView & w, int64_t N, int64_t M, int num_sms);
size_t gemm_tc_dense_ws_bytes(int64_t N, int64_t M, int ksplit);
cudaError_t launch_gemm_tc_dense(const WeightView & w, int64_t row0, int64_t N, const int8_t * q, const float * dT, int64_t ldP,
                                 int64_t M, float * y, int64_t ldy, unsigned * err, int num_sms, cudaStream_t st, int ksplit = 1,
                                 float * ws = nullptr, unsigned * tickets = nullptr);
size_t peer_mailbox_bytes(int G, int T_max, int H);
cudaError_t launch_moe_combine_allreduce(const float * down, const float * w, const int32_t * inv, int64_t T, int64_t top_k, int64_t H,
                                         const b200_ep_group * ep, float * out, unsigned * err, int num_sms, cudaStream_t st);
// K-quant (Q4_K, Q6_K) products with M >= 32 on the tensor cores (gemm_kq_tc.cu). act: scratch of
// gemm_kq_tc_act_bytes(K, M) bytes (quantized activations).
bool gemm_kq_tc_supported(const WeightView & w, int64_t M);
size_t gemm_kq_tc_act_bytes(int64_t K, int64_t M);
cudaError_t launch_gemm_kq_tc(b200_context * ctx, const b200_weight * w, int64_t row0, int64_t N, const float * x, int64_t M, float * y,
                              int64_t ldy, void * act);
void kq_release(b200_context * ctx, const void * data);
void kq_release_all(b200_context * ctx);
int64_t moe_max_slots(int64_t P, int64_t E);
int64_t moe_max_tiles(int64_t P, int64_t E);
cudaError_t launch_moe_route(const int32_t * ids, int64_t T, int64_t top_k, int64_t nb1, int64_t E, int64_t e0, int64_t total,
                             int32_t * grp_off, int32_t * col_src, int32_t * col_dst, int32_t * inv, int4 * tiles, int * ntiles,
                             unsigned * err, cudaStream_t st);
cudaError_t launch_moe_quant_slots(const float * x, int64_t K, int64_t ldx, const int32_t * col_src, const int32_t * n_slots,
                                   int64_t max_slots, int8_t * q, float * dT, int64_t ldP, int num_sms, cudaStream_t st);
cudaError_t launch_moe_swiglu_slots(const float * gu, int64_t F, const int32_t * col_src, const int32_t * n_slots, int64_t max_slots,
                                    int8_t * q, float * dT, int64_t ldP, int num_sms, cudaStream_t st);
cudaError_t launch_moe_combine_slots(const float * down, const float * w, const int32_t * inv, int64_t T, int64_t top_k, int64_t H,
                                     float * out, cudaStream_t st);

}  // namespace b200
