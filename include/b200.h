/*
 * b200.h — C ABI of the B200-native backend for speech.cpp's quantized matrix products.
 *
 * speech.cpp computes every weight product as a ggml node inside a ggml backend: MUL_MAT (src/common/graph.h:15-19),
 * MUL_MAT_ID (src/common/graph.h:22-26) and quantized GET_ROWS (src/families/qwen3-tts/talker.cpp:131-133,
 * src/families/qwen3-asr/decoder.cpp:319), run by ggml_backend_graph_compute (src/common/graph.cpp:145-147). A ggml
 * backend ("ggml-b200") forwards those nodes to the functions below, its buffer type's set_tensor / get_tensor to the
 * weight functions. Everything here takes plain pointers and sizes: no C++ or torch types, no exceptions.
 *
 * Conventions
 *  - Type ids are GGUF / ggml type ids (the reference lists them in checks/compare/quantize_compare.py:27).
 *  - A matrix of `type` has ne0 = K values per row and ne1 = N rows; ne2 = E stacks E such matrices (experts).
 *  - Activations and outputs are float32, row-major: x [M][K] is M rows of K values (ggml src1 [K, M]); dst [M][N]
 *    (ggml dst [N, M]).
 *  - Pointers named dev_* or documented as device pointers live in the context's GPU memory; *_host functions take
 *    host memory and copy inside the call.
 *  - Calls are asynchronous on the context's stream unless they say otherwise. b200_synchronize() waits and reports
 *    errors found on the device (an id out of range, a bounded wait that gave up).
 *  - Results follow ggml's CPU backend: each activation row is quantized to the weight type's vec_dot type (q8_0 for
 *    Q8_0, q8_K for Q4_K / Q5_K / Q6_K, bf16 for BF16) bit-identically and each (sub-)block's int32 sum is exact. The
 *    float step is defined without an order: each block's term fl32(d_w d_x) * sum is added exactly (in double) and
 *    the total is rounded once to float32. Products of up to 31 activation rows and the decode step compute exactly
 *    that; the tensor-core products (Q8_0 / Q4_K / Q6_K weights, 32 or more rows) accumulate the same terms in float32,
 *    within 1e-4 of sum |w x|.
 */
#ifndef SPEECH_B200_H
#define SPEECH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes. A ggml adapter maps B200_ERR_ALLOC to GGML_STATUS_ALLOC_FAILED and every other error to
 * GGML_STATUS_FAILED, which speech.cpp turns into Fault::OutOfMemory / Fault::Device (src/common/graph.cpp:139-140). */
typedef enum b200_status {
    B200_OK = 0,
    B200_ERR_INVALID = -1,     /* a null pointer, a bad shape, a row length that is not whole blocks */
    B200_ERR_UNSUPPORTED = -2, /* a type or op this backend does not compute */
    B200_ERR_ALLOC = -3,       /* device memory could not be allocated */
    B200_ERR_DEVICE = -4,      /* a CUDA error (b200_last_error() has the text) */
    B200_ERR_RANGE = -5,       /* an id (row or expert) outside its table, found on the device */
    B200_ERR_TIMEOUT = -6      /* a bounded device-side wait gave up */
} b200_status;

enum {
    B200_TYPE_F32 = 0,
    B200_TYPE_F16 = 1,
    B200_TYPE_Q8_0 = 8,
    B200_TYPE_Q4_K = 12,
    B200_TYPE_Q5_K = 13,
    B200_TYPE_Q6_K = 14,
    B200_TYPE_Q8_K = 15,
    B200_TYPE_BF16 = 30
};

/* ------------------------------------------------------------------------------------------------------------
 * Devices. Replaces the ggml device registry speech.cpp enumerates once (src/common/backend.cpp:113-131) and the
 * free-memory query Drama 3's placement uses (src/engines/drama3-engine.cpp:56-58: ggml_backend_dev_memory).
 * ------------------------------------------------------------------------------------------------------------ */
int b200_device_count(void);
/* name: e.g. "B200_0" (up to name_len bytes with the NUL); free / total device bytes. Any output may be NULL. */
b200_status b200_device_info(int device, char * name, size_t name_len, size_t * free_bytes, size_t * total_bytes);

/* ------------------------------------------------------------------------------------------------------------
 * Contexts: one device, one stream, a scratch pool. Replaces ggml_backend_dev_init (src/common/backend.cpp:158-163),
 * whose NULL return speech.cpp maps to Fault::Device. One request per context at a time (include/speech.h:27).
 * ------------------------------------------------------------------------------------------------------------ */
typedef struct b200_context b200_context;

b200_status b200_context_create(int device, b200_context ** out);
void b200_context_destroy(b200_context * ctx);
/* The context's cudaStream_t. */
void * b200_context_stream(b200_context * ctx);
/* Waits for the stream; returns the first device-side error recorded since the last call (then clears it). */
b200_status b200_synchronize(b200_context * ctx);
/* Text of the last error on this context ("" when none). */
const char * b200_last_error(b200_context * ctx);
/* Device memory helpers for callers without another allocator (ggml_backend_buffer alloc / free / memset). */
b200_status b200_malloc(b200_context * ctx, size_t bytes, void ** dev_out);
b200_status b200_free(b200_context * ctx, void * dev);
b200_status b200_memcpy_h2d(b200_context * ctx, void * dev_dst, const void * host_src, size_t bytes);
b200_status b200_memcpy_d2h(b200_context * ctx, void * host_dst, const void * dev_src, size_t bytes);

/* ------------------------------------------------------------------------------------------------------------
 * Weight tensors: the backend's weight buffer type. speech.cpp allocates weights in the backend's default buffer
 * type (src/common/model-file.cpp:222-245) and uploads them with ggml_backend_tensor_set in 16 MiB pieces at any
 * byte offset (src/common/model-file.cpp:247-268). b200_weight_set / _get accept the same GGUF bytes at the same
 * offsets. On the device the blocks are stored field by field, one row-contiguous array per block field, each array
 * 256-byte aligned (Q8_0: qs int8 [R][K] | d fp16 [R][K/32]; Q4_K: qs [R][K/2] | d, dmin, scales [R][K/256][16];
 * Q5_K: qs [R][K/2] | d, dmin, scales [R][K/256][16] | qh [R][K/8];
 * Q6_K: ql [R][K/2] | qh [R][K/4] | scales [R][K/256][16] | d fp16 [R][K/256]; BF16 as is). That is a byte
 * permutation, so any piece boundary works and the device holds exactly the GGUF bytes plus alignment.
 * ------------------------------------------------------------------------------------------------------------ */
typedef struct b200_weight {
    int32_t type;   /* B200_TYPE_* */
    int32_t device;
    int64_t ne0;    /* K: values per row */
    int64_t ne1;    /* N: rows per matrix */
    int64_t ne2;    /* E: matrices (experts); 1 for a plain matrix */
    void * data;    /* device allocation holding the repacked fields */
    size_t nbytes;  /* GGUF bytes (ggml_nbytes) */
    size_t dbytes;  /* device bytes (GGUF bytes + field alignment) */
    int64_t field_off[4]; /* byte offset of each field in data */
} b200_weight;

/* GGUF bytes of a [ne0, ne1, ne2] tensor of `type` (ggml_nbytes); 0 when rows are not whole blocks. */
size_t b200_weight_nbytes(int type, int64_t ne0, int64_t ne1, int64_t ne2);
b200_status b200_weight_alloc(b200_context * ctx, int type, int64_t ne0, int64_t ne1, int64_t ne2, b200_weight * out);
b200_status b200_weight_free(b200_context * ctx, b200_weight * w);
/* Writes GGUF bytes [offset, offset + size) of the tensor from host memory (ggml_backend_tensor_set). */
b200_status b200_weight_set(b200_context * ctx, b200_weight * w, const void * host_src, size_t offset, size_t size);
/* Same, with the source bytes already in device memory. */
b200_status b200_weight_set_device(b200_context * ctx, b200_weight * w, const void * dev_src, size_t offset, size_t size);
/* Reads GGUF bytes [offset, offset + size) back into host memory (ggml_backend_tensor_get). Synchronous. */
b200_status b200_weight_get(b200_context * ctx, const b200_weight * w, void * host_dst, size_t offset, size_t size);

/* ------------------------------------------------------------------------------------------------------------
 * Ops. All pointers are device pointers. These are the nodes the ggml adapter forwards.
 * ------------------------------------------------------------------------------------------------------------ */

/* MUL_MAT (src/common/graph.h:15-19; ggml_mul_mat with GGML_PREC_F32): dst[m][n] = sum_k W[n][k] x[m][k] for
 * x [M][K], dst [M][N], W of weight matrix 0 (ne2 == 1). */
b200_status b200_mul_mat(b200_context * ctx, const b200_weight * w, const float * x, int64_t M, float * dst);

/* MUL_MAT on rows [row0, row0 + n) of W only: dst [M][n] (a column shard of the output; multi-GPU column split). */
b200_status b200_mul_mat_rows(b200_context * ctx, const b200_weight * w, int64_t row0, int64_t n, const float * x,
                              int64_t M, float * dst, int64_t ld_dst);

/* MUL_MAT_ID (src/common/graph.h:22-26, used at src/families/drama3/text-model.cpp:208-210):
 *   experts: W [E][N][K]; b [T][nb1][K] with nb1 == 1 (one row per token shared by its chosen experts) or top_k;
 *   ids [T][top_k] int32 expert numbers; dst [T][top_k][N].
 * Routes by sorting (token, slot) pairs by expert on the device, then runs each expert's rows once over all of its
 * pairs. An id outside [0, E) is skipped and reported by the next b200_synchronize() as B200_ERR_RANGE. */
b200_status b200_mul_mat_id(b200_context * ctx, const b200_weight * experts, const float * b, int64_t nb1,
                            const int32_t * ids, int64_t top_k, int64_t T, float * dst);

/* The routed-expert block of a mixture-of-experts FFN, as TextModel::experts builds it from ggml nodes
 * (src/families/drama3/text-model.cpp:198-221): for each token t and slot s with expert e = ids[t][s],
 *   out[t] = sum over s (in slot order) of w[t][s] * Wdown_e (silu(Wgate_e x_t) * Wup_e x_t),
 * with gate and up stored as one expert matrix: gate_up [H, 2F, E] (rows 0..F-1 gate, F..2F-1 up) and down [F, H, E],
 * each Q8_0, Q4_K, Q5_K or Q6_K (K-quant down experts need F % 256 == 0). Q8_0 experts with H and F multiples of 256
 * run on the tensor cores; the others on the routed GEMV. x [T][H], ids int32 [T][top_k], w float [T][top_k] (the router's softmax weights,
 * computed upstream), out [T][H]. Expert parallelism: these experts are experts [expert0, expert0 + E) of
 * n_expert_total (0: all); pairs routed to other experts are skipped, so out is this shard's partial sum, and the
 * shards' outputs add up to the full result. Ids outside [0, n_expert_total) are reported by b200_synchronize(). */
b200_status b200_moe_ffn(b200_context * ctx, const b200_weight * gate_up, const b200_weight * down, int64_t expert0,
                         int64_t n_expert_total, const float * x, const int32_t * ids, const float * w, int64_t top_k, int64_t T,
                         float * out);

/* Expert parallelism over NVLink peer memory: the combine step of b200_moe_ffn fused with a two-shot all-reduce.
 * The reference runs a layer's routed experts on one device (src/families/drama3/text-model.cpp:198-221); this is its
 * multi-GPU extension. Every rank of a group of `world` (<= 8) GPUs allocates a mailbox and shares its IPC handle
 * (64 bytes, exchanged by the caller, e.g. over torch.distributed); every rank opens the others' mailboxes and creates
 * the group with all mailbox pointers (its own at index rank). b200_moe_ffn_ep then runs the rank's experts like
 * b200_moe_ffn and leaves in `out` the FULL weighted sum over all ranks' experts (every rank gets the same out). All
 * ranks must call it in the same order with the same T (<= max_tokens) and H; the experts are Q8_0 (tensor-core path).
 * A rank that never arrives makes the
 * others give up after a bounded wait (B200_ERR_TIMEOUT from b200_synchronize; see b200_ep_set_timeout). */
typedef struct b200_ep_group b200_ep_group;
b200_status b200_ep_mailbox_alloc(b200_context * ctx, int world, int64_t max_tokens, int64_t hidden, void ** mailbox, void * ipc_handle);
b200_status b200_ep_mailbox_open(b200_context * ctx, const void * ipc_handle, void ** peer_mailbox);
b200_status b200_ep_mailbox_close(b200_context * ctx, void * peer_mailbox);
b200_status b200_ep_mailbox_free(b200_context * ctx, void * mailbox);
b200_status b200_ep_create(b200_context * ctx, int rank, int world, int64_t max_tokens, int64_t hidden, void * const * mailboxes,
                           b200_ep_group ** out);
void b200_ep_destroy(b200_ep_group * group);
/* How long one wait of the combine may take before it gives up (default 2 s). After a wait gave up the group is broken
 * (the ranks' arrival counters are out of step): every later b200_moe_ffn_ep on it reports B200_ERR_TIMEOUT without
 * running; destroy it and create a new group on every rank. */
b200_status b200_ep_set_timeout(b200_ep_group * group, uint64_t microseconds);
b200_status b200_moe_ffn_ep(b200_context * ctx, const b200_weight * gate_up, const b200_weight * down, int64_t expert0,
                            int64_t n_expert_total, const float * x, const int32_t * ids, const float * w, int64_t top_k, int64_t T,
                            float * out, b200_ep_group * group);

/* Asks L2 to fetch a weight's device bytes ahead of the kernels that will read it, on `stream` (a cudaStream_t of the
 * weight's device; NULL: the context's stream). No counterpart in the reference. Returns once the request is queued;
 * nothing waits for the data. Useful when the weight fits in L2 (126 MB on B200) and the GPU's memory would otherwise
 * sit idle, e.g. for the next layer's experts while an expert-parallel combine crosses NVLink. */
b200_status b200_weight_prefetch_l2(b200_context * ctx, const b200_weight * w, void * stream);

/* Where a mixture-of-experts model's routed experts go on the GPUs of one node. speech.cpp keeps as many layers'
 * experts on its one GPU as its free memory holds and computes the rest on the CPU (src/families/drama3/
 * placement.cpp:58-74, used by src/engines/drama3-engine.cpp:51-88); here they spread over GPUs instead: rank r of
 * `ranks` holds experts [r E/ranks, (r+1) E/ranks) of every layer (b200_moe_ffn_ep) and every rank holds the rest of
 * the model. Given the free bytes of n_devices devices (b200_device_info), each layer's routed-expert bytes (all E
 * experts) and the bytes every rank needs beside its experts (the other weights, caches and working memory), the plan
 * is the fewest ranks (a power of two dividing n_expert, at most n_devices and 8) whose share fits each of the first
 * `ranks` devices. B200_ERR_ALLOC (out->ranks 0) when no such count fits. Host only. */
typedef struct b200_ep_plan {
    int32_t ranks;             /* GPUs that share the experts (1: one GPU holds them all) */
    int32_t experts_per_rank;  /* experts of each layer a rank holds */
    uint64_t bytes_per_rank;   /* its experts plus the rest */
    uint64_t expert_bytes;     /* the routed experts of all layers */
} b200_ep_plan;
b200_status b200_ep_place(int n_devices, const size_t * free_bytes, int n_layers, const uint64_t * expert_bytes, int n_expert,
                          uint64_t rest_bytes, b200_ep_plan * out);

/* GET_ROWS of a weight table (talker.cpp:131-133, decoder.cpp:319): dst [n][K] = dequantize(row ids[i]), bit for bit
 * as ggml's CPU dequantizers. An id outside [0, N * E) is skipped (its row is left untouched) and reported by
 * b200_synchronize() as B200_ERR_RANGE. */
b200_status b200_get_rows(b200_context * ctx, const b200_weight * table, const int32_t * ids, int64_t n, float * dst);

/* The CPU backend's activation quantization (src1 -> vec_dot type): M rows of K floats -> GGUF blocks of
 * B200_TYPE_Q8_0 (34 B / 32) or B200_TYPE_Q8_K (292 B / 256), bit for bit. dst holds M * row bytes. */
b200_status b200_quantize_rows(b200_context * ctx, int type, const float * x, int64_t K, int64_t M, void * dst);

/* Test hook for the bit-exactness of integer partials: the int32 (sub-)block sums the product of W's rows with
 * activation row x forms — Q8_0: one per 32-block; Q4_K: (sum_s sc_s I_s, sum_s m_s bsum_s) per super-block; Q6_K:
 * sum_g sc_g I_g per super-block — written to sums [N][per_row]. */
b200_status b200_block_sums(b200_context * ctx, const b200_weight * w, const float * x, int32_t * sums);

/* ------------------------------------------------------------------------------------------------------------
 * Decoder step: the matmul stack of one Qwen3 decoder step for one token, as Qwen3Decoder::layers / outputs build it
 * (src/common/qwen3-decoder.cpp:350-413, 422-438) and Qwen3Decoder::step keeps it as one graph on a GPU
 * (:462-490): per layer RMSNorm * attn_norm -> q, k, v -> attention -> o (+ residual) -> RMSNorm * ffn_norm ->
 * gate, up -> SwiGLU -> down (+ residual); then RMSNorm * output_norm -> head. Attention is taken at the first
 * position of a sequence, where each query head's output is its key/value head's value row; q/k norms, RoPE and
 * the KV cache do not change that output and stay with the rest of the ggml graph. The Qwen3-TTS talker step
 * (src/families/qwen3-tts/talker.cpp:119-138) and the Qwen3-ASR decoder step (qwen3-asr/decoder.cpp:383-449) run
 * this stack. Weights are set with GGUF bytes, per tensor, like ggml_backend_tensor_set.
 * ------------------------------------------------------------------------------------------------------------ */
typedef struct b200_decoder_shape {
    int32_t n_layer;
    int32_t hidden;
    int32_t n_head;
    int32_t n_kv_head;
    int32_t head_dim;
    int32_t ffn;
    int64_t n_vocab;
    float eps;            /* rms_norm epsilon */
    int32_t type_attn;    /* q, k, v, o */
    int32_t type_ffn_up;  /* gate, up */
    int32_t type_ffn_down;
    int32_t type_head;
} b200_decoder_shape;

enum {
    B200_DEC_ATTN_Q = 0,
    B200_DEC_ATTN_K = 1,
    B200_DEC_ATTN_V = 2,
    B200_DEC_ATTN_O = 3,
    B200_DEC_FFN_GATE = 4,
    B200_DEC_FFN_UP = 5,
    B200_DEC_FFN_DOWN = 6,
    B200_DEC_ATTN_NORM = 7,   /* float32 [hidden] */
    B200_DEC_FFN_NORM = 8,    /* float32 [hidden] */
    B200_DEC_OUTPUT_NORM = 9, /* float32 [hidden], layer ignored */
    B200_DEC_OUTPUT = 10      /* head [hidden -> n_vocab], layer ignored */
};

typedef struct b200_decoder b200_decoder;

b200_status b200_decoder_create(b200_context * ctx, const b200_decoder_shape * shape, b200_decoder ** out);
void b200_decoder_destroy(b200_decoder * d);
/* Writes bytes [offset, offset + size) of tensor `which` of `layer` (GGUF blocks for matrices, float32 for norms).
 * on_device != 0: data is a device pointer. */
b200_status b200_decoder_set_tensor(b200_decoder * d, int layer, int which, const void * data, int on_device, size_t offset,
                                    size_t size);
/* One step on device buffers: x [hidden] -> logits [n_vocab] (logits may be NULL). Asynchronous; the first call
 * captures the step's launches in a CUDA graph, later calls replay it. */
b200_status b200_decoder_step(b200_decoder * d, const float * x, float * logits);
/* One step from host memory to host memory (copies in, step, copies out; synchronous). */
b200_status b200_decoder_step_host(b200_decoder * d, const float * x_host, float * logits_host);
/* Kernel launches of one step, and the GGUF weight bytes one step streams. */
int64_t b200_decoder_launches(const b200_decoder * d);
size_t b200_decoder_weight_bytes(const b200_decoder * d);
/* How a step runs. B200_DEC_MODE_CHAIN: one launch per product, chained with programmatic dependent launch
 * (pdl != 0) and ctas_per_sm CTAs per SM (0: as many as fit). B200_DEC_MODE_PERSISTENT: the whole step as one
 * persistent kernel, one CTA per SM, products separated by device-side completion counters; needs K % 1024 == 0
 * (K % 2048 for Q4_K / Q6_K) and K <= 8192 for every product. -1 (the default): persistent when every product fits,
 * else chain. */
enum { B200_DEC_MODE_CHAIN = 0, B200_DEC_MODE_PERSISTENT = 1 };
b200_status b200_decoder_set_launch(b200_decoder * d, int mode, int pdl, int ctas_per_sm);

/* ------------------------------------------------------------------------------------------------------------
 * Graph execution: the backend's graph_compute over ggml-shaped tensor records, so a whole decoder graph
 * (Qwen3Decoder::layers / outputs, src/common/qwen3-decoder.cpp:350-438) runs on this backend with no other backend
 * beside it (speech.cpp computes each graph on one backend, src/common/graph.cpp:145-147). A ggml adapter fills one
 * b200_tensor per ggml_tensor of the graph (its op, type, ne, nb and data; sources by index) and calls
 * b200_graph_compute once; b200_graph_supports answers ggml_backend_supports_op. Leaves (inputs, weights, the KV
 * cache, views, reshapes, permutes and transposes: op B200_OP_NONE) carry only their data pointer and strides.
 *
 * Arithmetic (the CPU oracle defines the same): products of quantized weights as b200_mul_mat; products of F16 / F32
 * matrices with the activations rounded to the matrix's type as ggml's CPU vec_dot does (F16 for an F16 matrix), the
 * element products summed exactly and rounded once to float32; RMS_NORM, SOFT_MAX and SiLU sums and exponentials in
 * double, rounded once; ROPE angles p * base^(-2i/n_dims) in double, their cosine and sine rounded once to float32.
 * ------------------------------------------------------------------------------------------------------------ */
enum {
    B200_TYPE_I32 = 26  /* row ids and positions (ggml's GGML_TYPE_I32) */
};

typedef enum b200_op {
    B200_OP_NONE = 0,        /* a leaf or a view: nothing to compute */
    B200_OP_GET_ROWS = 1,    /* dst[:, i, j, k] = dequantize(src0[:, src1[i, j, k], j, k]); src0 a weight or F32 / F16 */
    B200_OP_MUL_MAT = 2,     /* dst[n, m, i2, i3] = sum_k src0[k, n, i2 / r2, i3 / r3] * src1[k, m, i2, i3] */
    B200_OP_RMS_NORM = 3,    /* per row: x / sqrt(mean(x^2) + eps); params[0] = eps (float bits) */
    B200_OP_MUL = 4,         /* src0 * src1, src1 repeated to src0's shape */
    B200_OP_ADD = 5,         /* src0 + src1, src1 repeated to src0's shape */
    B200_OP_ROPE = 6,        /* NEOX rotation of src0 [head_dim, heads, tokens] at positions src1 (I32 [tokens]);
                                params: [0] n_dims, [1] mode (2 = NEOX, the only one), [2] freq_base (float bits),
                                [3] freq_scale (float bits, must be 1), [4] ext_factor (float bits, must be 0),
                                [5] attn_factor (float bits, must be 1) */
    B200_OP_SET_ROWS = 7,    /* dst (a view of the cache, F16 or F32) rows src1[i] = src0 row i (converted); dst is also
                                src[2] of the record (the tensor written in place) */
    B200_OP_CPY = 8,         /* dst = src0 element by element in row-major order (same shape), converted to dst's type;
                                dst written in place through src[1] */
    B200_OP_CONT = 9,        /* a contiguous copy of src0 (a permuted or transposed view) */
    B200_OP_SOFT_MAX = 10,   /* rows of softmax(src0 * scale + src1 (mask, F16 / F32, optional)); params[0] = scale */
    B200_OP_FLASH_ATTN = 11, /* ggml_flash_attn_ext: q src0 [D, n_q, H], k src1 [D, n_kv, H_kv] F16, v src2 [D, n_kv,
                                H_kv] F16, mask src3 [n_kv, >= n_q] F16 (optional); dst [D, H, n_q] F32; params[0] = scale */
    B200_OP_SWIGLU = 12,     /* ggml_swiglu_split: silu(src0) * src1 */
    B200_OP_ARGMAX = 13,     /* dst I32 [rows]: index of the first largest value of each row of src0 */
    B200_OP_SCALE = 14,      /* src0 * params[0] + params[1] (float bits) */
    B200_OP_FILL = 15,       /* every element of dst (a view, written in place; src0 optional, the same tensor) =
                                params[0] (float bits): ggml_fill_inplace of the KV cache's tail */
    B200_OP_CONCAT = 16      /* src0 and src1 joined along dimension params[0] (the others equal) */
} b200_op;

typedef struct b200_tensor {
    int32_t op;                 /* b200_op */
    int32_t type;               /* B200_TYPE_F32, F16, I32, or the weight's type when `weight` is set */
    int64_t ne[4];              /* elements per dimension, innermost first (ggml ne) */
    int64_t nb[4];              /* byte strides (ggml nb) */
    void * data;                /* device address of element [0, 0, 0, 0] */
    const b200_weight * weight; /* a weight in this backend's layout (MUL_MAT src0, GET_ROWS table), else NULL */
    int32_t src[4];             /* indices of the source records in the same array; -1: none */
    int32_t params[8];          /* op parameters, as listed with each op */
} b200_tensor;

/* Runs the records with an op, in array order, on the context's stream (asynchronous). A record's sources must come
 * before it. Returns B200_ERR_UNSUPPORTED for a record b200_graph_supports rejects (nothing after it is launched). */
b200_status b200_graph_compute(b200_context * ctx, const b200_tensor * tensors, int64_t n);
/* Whether record i (with its sources in the same array) can run here: ggml_backend_supports_op. */
int b200_graph_supports(const b200_tensor * tensors, int64_t n, int64_t i);

/* ------------------------------------------------------------------------------------------------------------
 * Host-buffer entry points (the end-to-end path a CPU caller takes: copies in, product, copy out, synchronous).
 * ------------------------------------------------------------------------------------------------------------ */
b200_status b200_mul_mat_host(b200_context * ctx, const b200_weight * w, const float * x_host, int64_t M, float * dst_host);

/* ------------------------------------------------------------------------------------------------------------
 * MUL_MAT_ID without allocation. No counterpart in the reference: speech.cpp's ggml backends allocate their scratch
 * themselves. This entry point is for callers that cannot call cudaMalloc — a serving runtime that owns all device
 * memory through its own arena, a latency-critical path where an allocation could synchronize the device, a process
 * whose weights already fill the GPU. It runs the grouped GEMV path of b200_mul_mat_id for every size, on `stream` (a
 * cudaStream_t of the current device, which must be the experts' device). Its results equal b200_mul_mat_id's bit for
 * bit wherever b200_mul_mat_id takes that path too (any type other than Q8_0, and Q8_0 with fewer than 128
 * (token, slot) pairs); for Q8_0 with 128 pairs or more b200_mul_mat_id runs the tensor-core grouped GEMM, and the two
 * agree within the products' tolerance, |err| <= 1e-4 * sum |w x| per element. The experts' upload must be complete
 * before the call, or ordered before it by the caller: b200_weight_set runs on the context's stream, which nothing
 * orders against `stream`. Its scratch is a static device array of B200_NOALLOC_SCRATCH_BYTES that every GPU loading
 * the library holds until exit. The first call on a device looks up that array's device address
 * (cudaGetSymbolAddress); make it before any stream capture. A call needs about T*nb1*K bytes of quantized
 * activations plus 8*T*top_k + 4*E bytes of routing tables; a call that needs more than the array returns
 * B200_ERR_INVALID. Calls share the array: two calls that overlap on the GPU race. Ids outside [0, E) are skipped
 * (their dst rows are left unchanged) and not reported.
 * ------------------------------------------------------------------------------------------------------------ */
#define B200_NOALLOC_SCRATCH_BYTES (16u << 20)
b200_status b200_mul_mat_id_noalloc(void * stream, const b200_weight * experts, const float * b, int64_t nb1,
                                    const int32_t * ids, int64_t top_k, int64_t T, float * dst);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* SPEECH_B200_H */
