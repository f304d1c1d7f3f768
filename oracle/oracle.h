/*
 * oracle.h — CPU restatement of the quantized matrix products of speech.cpp's hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the B200 kernels and the timed CPU baseline of bench.py.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs load it. The product path
 * (speech.cpp_b200/, include/b200.h) never calls it.
 *
 * What it restates. speech.cpp computes every weight product as a ggml node: mul_mat() / mul_mat_id() in
 * src/common/graph.h:15-26 (ggml_mul_mat / ggml_mul_mat_id with GGML_PREC_F32), and quantized embedding lookups with
 * ggml_get_rows (src/families/qwen3-tts/talker.cpp:131-133, src/families/qwen3-asr/decoder.cpp:319). The arithmetic of
 * those nodes lives in ggml (git submodule nyosegawa/ggml, branch speech.cpp, on upstream tag v0.27.0 — see
 * .gitmodules and docs/adr/ggml-comes-from-a-fork-...md:5), which is ABSENT from the reference checkout. This file
 * restates, in our own code, the published GGUF block formats and the CPU backend's semantics for these nodes:
 *   - weights stay in their GGUF blocks (Q8_0 34 B / 32, Q4_K 144 B / 256, Q6_K 210 B / 256, BF16 2 B);
 *   - each activation row is quantized to the weight type's "vec_dot type": q8_0 blocks for Q8_0 weights, q8_K
 *     blocks for Q4_K / Q6_K weights, bf16 for BF16 weights;
 *   - each output element is a dot product formed from exact int32 sums per (sub-)block, scaled and accumulated in
 *     float32.
 *
 * Pins. (1) Q8_0 quantization of weights follows ggml's reference quantizer, which gguf-py 0.19.0
 * (gguf/quants.py:378-394) restates bit-exactly and which the reference's checks/compare/quantize_compare.py:1-11 pins
 * against ggml; tests/golden holds gguf-py outputs. (2) Q8_0 / Q4_K / Q6_K / BF16 dequantization is pinned the same way
 * against gguf-py (quants.py:396-401, 504-527, 554-575, 204-216). (3) The activation quantizers (q8_0 for activations,
 * q8_K) and the int32 / float order of ggml's CPU vec_dot are NOT pinned: ggml is absent and no golden vectors exist.
 * The activation q8_0 quantizer is the same function as the pinned weight quantizer (ggml's reference row quantizer);
 * q8_K restates ggml's reference q8_K quantizer. The GPU must match these bit-exactly per block.
 */
#ifndef SPEECH_B200_ORACLE_H
#define SPEECH_B200_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF / ggml type ids (GGUF file format; the reference's checks/compare/quantize_compare.py:27 lists the same ids). */
enum {
    ORACLE_TYPE_F32 = 0,
    ORACLE_TYPE_F16 = 1,
    ORACLE_TYPE_Q8_0 = 8,
    ORACLE_TYPE_Q4_K = 12,
    ORACLE_TYPE_Q5_K = 13,
    ORACLE_TYPE_Q6_K = 14,
    ORACLE_TYPE_Q8_K = 15,
    ORACLE_TYPE_BF16 = 30,
};

#define ORACLE_QK8_0 32
#define ORACLE_QK_K 256

/* Block layouts, byte for byte as GGUF stores them. */
typedef struct {
    uint16_t d; /* fp16 scale */
    int8_t qs[32];
} oracle_block_q8_0; /* 34 bytes */

typedef struct {
    uint16_t d;          /* fp16 super-block scale of the sub-block scales */
    uint16_t dmin;       /* fp16 super-block scale of the sub-block mins */
    uint8_t scales[12];  /* 8 six-bit scales and 8 six-bit mins */
    uint8_t qs[128];     /* 256 four-bit values */
} oracle_block_q4_K;     /* 144 bytes */

typedef struct {
    uint16_t d;          /* fp16 super-block scale of the sub-block scales */
    uint16_t dmin;       /* fp16 super-block scale of the sub-block mins */
    uint8_t scales[12];  /* 8 six-bit scales and 8 six-bit mins, packed as Q4_K's */
    uint8_t qh[32];      /* bit j of byte l: the fifth bit of value l of sub-block j */
    uint8_t qs[128];     /* low four bits, laid out as Q4_K's values */
} oracle_block_q5_K;     /* 176 bytes */

typedef struct {
    uint8_t ql[128];     /* low four bits of 256 six-bit values */
    uint8_t qh[64];      /* high two bits */
    int8_t scales[16];   /* one signed scale per 16 values */
    uint16_t d;          /* fp16 super-block scale */
} oracle_block_q6_K;     /* 210 bytes */

typedef struct {
    float d;             /* f32 scale */
    int8_t qs[256];
    int16_t bsums[16];   /* sums of each 16 values of qs */
} oracle_block_q8_K;     /* 292 bytes */

/* Bytes of one row of `k` values of `type` (ggml_row_size). 0 for an unknown type or k not a multiple of the block. */
size_t oracle_row_size(int type, int64_t k);

/* Scalar conversions (IEEE round-to-nearest-even, as F16C / numpy astype do). */
uint16_t oracle_fp32_to_fp16(float f);
float oracle_fp16_to_fp32(uint16_t h);
uint16_t oracle_fp32_to_bf16(float f);
float oracle_bf16_to_fp32(uint16_t h);

/* Row quantizers: `k` floats -> k / block_size blocks. */
void oracle_quantize_q8_0(const float * x, void * y, int64_t k);
void oracle_quantize_q8_K(const float * x, void * y, int64_t k);
void oracle_quantize_q4_K(const float * x, void * y, int64_t k);
void oracle_quantize_q5_K(const float * x, void * y, int64_t k);
void oracle_quantize_q6_K(const float * x, void * y, int64_t k);
void oracle_quantize_bf16(const float * x, void * y, int64_t k);
/* Quantizes n rows of k values each, in parallel over rows (nthreads <= 0: all). */
int oracle_quantize_rows(int type, const float * x, void * y, int64_t k, int64_t n, int nthreads);

/* Row dequantizers: blocks -> `k` floats. */
int oracle_dequantize_row(int type, const void * x, float * y, int64_t k);

/* Dot product of one weight row (blocks of `type`) with one activation row already in the vec_dot type. */
float oracle_vec_dot(int type, const void * w_row, const void * x_row, int64_t k);

/* The vec_dot type of a weight type: Q8_0 for Q8_0, Q8_K for Q4_K / Q6_K, BF16 for BF16, F32 for F32. */
int oracle_vec_dot_type(int type);

/*
 * The int32 sums the CPU's vec_dot forms for one weight row and one quantized activation row, in block order:
 *   Q8_0: one per 32-block: sum_j qw_j * qx_j.                               (k / 32 values)
 *   Q4_K: two per super-block: sum_s sc_s * (sum over sub-block s of q4*q8), then sum_s m_s * bsum32_s.   (2 k / 256)
 *   Q6_K: one per super-block: sum_g sc_g * (sum over 16-group g of q6*q8).  (k / 256)
 * Returns the number of values written, or -1 for an unsupported type.
 */
int64_t oracle_block_sums(int type, const void * w_row, const void * x_row, int64_t k, int32_t * out);

/*
 * ggml_mul_mat on the CPU backend: dst[m][n] = sum_k W[n][k] * x[m][k], W as `type` blocks (N rows of K values),
 * x as float32 [M][K], dst float32 [M][N]. Each x row is quantized to the vec_dot type first.
 * nthreads <= 0 uses all host cores. Returns 0, or -1 for an unsupported type / shape.
 */
int oracle_mul_mat(int type, const void * w, int64_t K, int64_t N, const float * x, int64_t M, float * dst, int nthreads);

/*
 * ggml_mul_mat_id on the CPU backend (src/families/drama3/text-model.cpp:208-210):
 *   experts: E matrices of N rows x K values each (`type` blocks, expert e at byte e * N * row_size);
 *   b: float32 [T][nb1][K] with nb1 == 1 (one row shared by every chosen expert) or nb1 == top_k;
 *   ids: int32 [T][top_k] expert numbers;
 *   dst: float32 [T][top_k][N].
 * Returns 0, -1 for an unsupported type / shape, -2 for an id out of [0, E).
 */
int oracle_mul_mat_id(int type, const void * experts, int64_t K, int64_t N, int64_t E, const float * b, int64_t nb1,
                      const int32_t * ids, int64_t top_k, int64_t T, float * dst, int nthreads);

/* ggml_get_rows of a quantized / f32 table [rows][K]: dst[i] = dequantize(table row ids[i]). Returns 0, -1, or -2. */
int oracle_get_rows(int type, const void * table, int64_t K, int64_t rows, const int32_t * ids, int64_t n, float * dst);

/* Number of host threads OpenMP would use. */
int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif

#endif
