/*
 * oracle.c — CPU restatement of ggml's quantized MUL_MAT / MUL_MAT_ID / GET_ROWS for speech.cpp's hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the B200 kernels and the timed CPU baseline ("port"). The product path
 * never links it. See oracle.h for what is pinned (gguf-py golden vectors) and what is not (ggml is absent from the
 * reference checkout: the activation quantizers and ggml's float summation order are unpinned).
 *
 * Build with -ffp-contract=off: a fused multiply-add would change the float results the GPU must reproduce
 * (dequantized rows are compared bit for bit).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------------------------------------------------
 * Scalar conversions.
 * ------------------------------------------------------------------------------------------------------------- */

static uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static float u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary32 -> binary16, round to nearest even (what F16C's _cvtss_sh(x, 0) and numpy's astype(float16) do). */
uint16_t oracle_fp32_to_fp16(float f) {
    const uint32_t x = f2u(f);
    const uint16_t sign = (uint16_t) ((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t) (sign | 0x7e00u);           /* NaN -> quiet NaN */
    if (a >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u);          /* >= 65520 rounds to infinity */
    if (a >= 0x38800000u) {                                             /* normal half: 2^-14 <= |f| */
        const uint32_t r = a - 0x38000000u;                             /* rebias exponent 127 -> 15 */
        const uint32_t rounded = (r + 0x0fffu + ((r >> 13) & 1u)) >> 13;
        return (uint16_t) (sign | rounded);
    }
    if (a < 0x33000000u) return sign;                                   /* < 2^-25: rounds to zero */
    /* subnormal half: value in units of 2^-24 = m * 2^(e - 126) */
    const uint32_t e = a >> 23;
    const uint32_t m = (a & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;                                    /* 14 .. 24 */
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t) (sign | q);
}

float oracle_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = ((uint32_t) h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        /* subnormal: m * 2^-24, exact in float */
        const float v = (float) m * u2f(0x33800000u); /* 2^-24 */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* binary32 -> bfloat16 as gguf-py's BF16.quantize_blocks (quants.py:206-213): quiet NaNs, round to nearest even. */
uint16_t oracle_fp32_to_bf16(float f) {
    uint32_t n = f2u(f);
    if ((n & 0x7fffffffu) > 0x7f800000u) return (uint16_t) (((n & 0xffff0000u) | (64u << 16)) >> 16);
    const uint64_t r = ((uint64_t) n + (0x7fffu + ((n >> 16) & 1u))) >> 16;
    return (uint16_t) r;
}

float oracle_bf16_to_fp32(uint16_t h) {
    return u2f((uint32_t) h << 16);
}

size_t oracle_row_size(int type, int64_t k) {
    switch (type) {
    case ORACLE_TYPE_F32: return (size_t) k * 4;
    case ORACLE_TYPE_F16:
    case ORACLE_TYPE_BF16: return (size_t) k * 2;
    case ORACLE_TYPE_Q8_0: return k % 32 ? 0 : (size_t) (k / 32) * sizeof(oracle_block_q8_0);
    case ORACLE_TYPE_Q4_K: return k % 256 ? 0 : (size_t) (k / 256) * sizeof(oracle_block_q4_K);
    case ORACLE_TYPE_Q5_K: return k % 256 ? 0 : (size_t) (k / 256) * sizeof(oracle_block_q5_K);
    case ORACLE_TYPE_Q6_K: return k % 256 ? 0 : (size_t) (k / 256) * sizeof(oracle_block_q6_K);
    case ORACLE_TYPE_Q8_K: return k % 256 ? 0 : (size_t) (k / 256) * sizeof(oracle_block_q8_K);
    default: return 0;
    }
}

int oracle_vec_dot_type(int type) {
    switch (type) {
    case ORACLE_TYPE_Q8_0: return ORACLE_TYPE_Q8_0;
    case ORACLE_TYPE_Q4_K:
    case ORACLE_TYPE_Q5_K:
    case ORACLE_TYPE_Q6_K: return ORACLE_TYPE_Q8_K;
    case ORACLE_TYPE_BF16: return ORACLE_TYPE_BF16;
    case ORACLE_TYPE_F32: return ORACLE_TYPE_F32;
    default: return -1;
    }
}

/* Round half to even for |v| < 2^22: the value ggml's nearest_int() gives (its float-add trick rounds this way). */
static int nearest_even(float v) {
    return (int) rintf(v);
}

/* ---------------------------------------------------------------------------------------------------------------
 * Quantizers.
 * ------------------------------------------------------------------------------------------------------------- */

/*
 * Q8_0 / q8_0: per 32 values, d = amax / 127, id = 1 / d (0 when d is 0), q = round-half-away(x * id), d stored as fp16
 * of the unrounded d. This is ggml's reference row quantizer, which gguf-py's Q8_0.quantize_blocks restates
 * (gguf/quants.py:381-394, np_roundf rounds half away from zero, :43-48) and which the reference pins against ggml in
 * checks/compare/quantize_compare.py:1-11. The same function quantizes activation rows for Q8_0 weights.
 */
void oracle_quantize_q8_0(const float * x, void * vy, int64_t k) {
    oracle_block_q8_0 * y = (oracle_block_q8_0 *) vy;
    for (int64_t i = 0; i < k / 32; i++) {
        const float * xb = x + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = oracle_fp32_to_fp16(d);
        for (int j = 0; j < 32; j++) y[i].qs[j] = (int8_t) roundf(xb[j] * id);
    }
}

/*
 * q8_K (activations for K-quant weights): per 256 values, max = the value of largest magnitude (the first one on
 * ties), iscale = -127 / max, q = min(127, round-half-even(iscale * x)), d = 1 / iscale, and the sums of each 16 q.
 * A block of zeros has d = 0. Restates ggml's reference q8_K quantizer (ggml-quants.c, absent here).
 */
void oracle_quantize_q8_K(const float * x, void * vy, int64_t k) {
    oracle_block_q8_K * y = (oracle_block_q8_K *) vy;
    for (int64_t i = 0; i < k / 256; i++) {
        const float * xb = x + i * 256;
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < 256; j++) {
            const float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
                max = xb[j];
            }
        }
        if (amax == 0.0f) {
            memset(&y[i], 0, sizeof(y[i]));
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < 256; j++) {
            const int v = nearest_even(iscale * xb[j]);
            y[i].qs[j] = (int8_t) (v < 127 ? v : 127);
        }
        for (int j = 0; j < 16; j++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += y[i].qs[j * 16 + l];
            y[i].bsums[j] = (int16_t) s;
        }
        y[i].d = 1.0f / iscale;
    }
}

/*
 * Q4_K weights. speech.cpp's files are written by ggml's quantizer (src/common/quantize.cpp:164-182), whose search for
 * scales is not restated: the products only need valid blocks that the oracle and the GPU read identically, so this
 * quantizer is a plain min/max one. Layout (GGUF): d, dmin (fp16), 12 bytes holding 8 six-bit scales and 8 six-bit
 * mins (unpacked as gguf-py's Q4_K.get_scale_min, quants.py:478-502), then 128 bytes: byte g*32+l holds value
 * (2g)*32+l in its low nibble and value (2g+1)*32+l in its high nibble. Value = d*sc*q - dmin*m.
 */
void oracle_quantize_q4_K(const float * x, void * vy, int64_t k) {
    oracle_block_q4_K * y = (oracle_block_q4_K *) vy;
    for (int64_t i = 0; i < k / 256; i++) {
        const float * xb = x + i * 256;
        float scale[8], mn[8], max_scale = 0.0f, max_min = 0.0f;
        for (int s = 0; s < 8; s++) {
            float lo = xb[s * 32], hi = xb[s * 32];
            for (int l = 1; l < 32; l++) {
                const float v = xb[s * 32 + l];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            if (lo > 0.0f) lo = 0.0f;
            scale[s] = (hi - lo) / 15.0f;
            mn[s] = -lo;
            if (scale[s] > max_scale) max_scale = scale[s];
            if (mn[s] > max_min) max_min = mn[s];
        }
        const uint16_t dh = oracle_fp32_to_fp16(max_scale / 63.0f);
        const uint16_t mh = oracle_fp32_to_fp16(max_min / 63.0f);
        const float d = oracle_fp16_to_fp32(dh), dmin = oracle_fp16_to_fp32(mh);
        uint8_t sc[8], m[8];
        for (int s = 0; s < 8; s++) {
            int a = d > 0.0f ? nearest_even(scale[s] / d) : 0;
            int b = dmin > 0.0f ? nearest_even(mn[s] / dmin) : 0;
            sc[s] = (uint8_t) (a < 0 ? 0 : a > 63 ? 63 : a);
            m[s] = (uint8_t) (b < 0 ? 0 : b > 63 ? 63 : b);
        }
        y[i].d = dh;
        y[i].dmin = mh;
        for (int j = 0; j < 4; j++) {
            y[i].scales[j] = (uint8_t) ((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            y[i].scales[j + 4] = (uint8_t) ((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            y[i].scales[j + 8] = (uint8_t) ((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
        }
        uint8_t q[256];
        for (int s = 0; s < 8; s++) {
            const float ds = d * (float) sc[s], ms = dmin * (float) m[s];
            for (int l = 0; l < 32; l++) {
                int v = ds > 0.0f ? nearest_even((xb[s * 32 + l] + ms) / ds) : 0;
                q[s * 32 + l] = (uint8_t) (v < 0 ? 0 : v > 15 ? 15 : v);
            }
        }
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) y[i].qs[g * 32 + l] = (uint8_t) (q[(2 * g) * 32 + l] | (q[(2 * g + 1) * 32 + l] << 4));
    }
}

/*
 * Q5_K weights (our own plain min/max quantizer, valid blocks, as for Q4_K). Layout (GGUF, as gguf-py's
 * Q5_K.dequantize_blocks reads it, quants.py:528-551): d, dmin (fp16), the 12 scale bytes packed as Q4_K's, qh[32]
 * (bit j of byte l is the fifth bit of value l of sub-block j), qs[128] as Q4_K's four-bit values. Value =
 * d*sc*q - dmin*m with q = low | fifth << 4 in 0..31.
 */
void oracle_quantize_q5_K(const float * x, void * vy, int64_t k) {
    oracle_block_q5_K * y = (oracle_block_q5_K *) vy;
    for (int64_t i = 0; i < k / 256; i++) {
        const float * xb = x + i * 256;
        float scale[8], mn[8], max_scale = 0.0f, max_min = 0.0f;
        for (int s = 0; s < 8; s++) {
            float lo = xb[s * 32], hi = xb[s * 32];
            for (int l = 1; l < 32; l++) {
                const float v = xb[s * 32 + l];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            if (lo > 0.0f) lo = 0.0f;
            scale[s] = (hi - lo) / 31.0f;
            mn[s] = -lo;
            if (scale[s] > max_scale) max_scale = scale[s];
            if (mn[s] > max_min) max_min = mn[s];
        }
        const uint16_t dh = oracle_fp32_to_fp16(max_scale / 63.0f);
        const uint16_t mh = oracle_fp32_to_fp16(max_min / 63.0f);
        const float d = oracle_fp16_to_fp32(dh), dmin = oracle_fp16_to_fp32(mh);
        uint8_t sc[8], m[8];
        for (int s = 0; s < 8; s++) {
            int a = d > 0.0f ? nearest_even(scale[s] / d) : 0;
            int b = dmin > 0.0f ? nearest_even(mn[s] / dmin) : 0;
            sc[s] = (uint8_t) (a < 0 ? 0 : a > 63 ? 63 : a);
            m[s] = (uint8_t) (b < 0 ? 0 : b > 63 ? 63 : b);
        }
        y[i].d = dh;
        y[i].dmin = mh;
        for (int j = 0; j < 4; j++) {
            y[i].scales[j] = (uint8_t) ((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            y[i].scales[j + 4] = (uint8_t) ((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            y[i].scales[j + 8] = (uint8_t) ((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
        }
        uint8_t q[256];
        for (int s = 0; s < 8; s++) {
            const float ds = d * (float) sc[s], ms = dmin * (float) m[s];
            for (int l = 0; l < 32; l++) {
                int v = ds > 0.0f ? nearest_even((xb[s * 32 + l] + ms) / ds) : 0;
                q[s * 32 + l] = (uint8_t) (v < 0 ? 0 : v > 31 ? 31 : v);
            }
        }
        memset(y[i].qh, 0, sizeof y[i].qh);
        for (int s = 0; s < 8; s++)
            for (int l = 0; l < 32; l++) y[i].qh[l] |= (uint8_t) (((q[s * 32 + l] >> 4) & 1) << s);
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++)
                y[i].qs[g * 32 + l] = (uint8_t) ((q[(2 * g) * 32 + l] & 15) | ((q[(2 * g + 1) * 32 + l] & 15) << 4));
    }
}

/*
 * Q6_K weights (our own plain quantizer, valid blocks). Layout (GGUF, as gguf-py's Q6_K.dequantize_blocks reads it,
 * quants.py:554-575): value v = h*128 + t*32 + l (h in 0..1, t in 0..3, l in 0..31) has its low four bits in byte
 * ql[h*64 + (t&1)*32 + l] (low nibble for t < 2, high for t >= 2) and its high two bits in qh[h*32 + l] at bit 2t;
 * value = d * scales[v/16] * (q - 32).
 */
void oracle_quantize_q6_K(const float * x, void * vy, int64_t k) {
    oracle_block_q6_K * y = (oracle_block_q6_K *) vy;
    for (int64_t i = 0; i < k / 256; i++) {
        const float * xb = x + i * 256;
        float gs[16], max_gs = 0.0f;
        for (int g = 0; g < 16; g++) {
            float amax = 0.0f;
            for (int l = 0; l < 16; l++) {
                const float a = fabsf(xb[g * 16 + l]);
                if (a > amax) amax = a;
            }
            gs[g] = amax / 31.0f;
            if (gs[g] > max_gs) max_gs = gs[g];
        }
        const uint16_t dh = oracle_fp32_to_fp16(max_gs / 127.0f);
        const float d = oracle_fp16_to_fp32(dh);
        int8_t sc[16];
        for (int g = 0; g < 16; g++) {
            int a = d > 0.0f ? nearest_even(gs[g] / d) : 0;
            sc[g] = (int8_t) (a < 0 ? 0 : a > 127 ? 127 : a);
        }
        uint8_t q[256];
        for (int v = 0; v < 256; v++) {
            const float ds = d * (float) sc[v / 16];
            int t = ds > 0.0f ? nearest_even(xb[v] / ds) : 0;
            t = t < -32 ? -32 : t > 31 ? 31 : t;
            q[v] = (uint8_t) (t + 32);
        }
        memset(y[i].ql, 0, sizeof(y[i].ql));
        memset(y[i].qh, 0, sizeof(y[i].qh));
        for (int h = 0; h < 2; h++)
            for (int t = 0; t < 4; t++)
                for (int l = 0; l < 32; l++) {
                    const uint8_t v = q[h * 128 + t * 32 + l];
                    y[i].ql[h * 64 + (t & 1) * 32 + l] |= (uint8_t) ((v & 15) << ((t >> 1) * 4));
                    y[i].qh[h * 32 + l] |= (uint8_t) ((v >> 4) << (2 * t));
                }
        memcpy(y[i].scales, sc, 16);
        y[i].d = dh;
    }
}

void oracle_quantize_bf16(const float * x, void * vy, int64_t k) {
    uint16_t * y = (uint16_t *) vy;
    for (int64_t i = 0; i < k; i++) y[i] = oracle_fp32_to_bf16(x[i]);
}

int oracle_quantize_rows(int type, const float * x, void * y, int64_t k, int64_t n, int nthreads) {
    const size_t rs = oracle_row_size(type, k);
    if (!rs) return -1;
    void (*fn)(const float *, void *, int64_t) = NULL;
    switch (type) {
    case ORACLE_TYPE_Q8_0: fn = oracle_quantize_q8_0; break;
    case ORACLE_TYPE_Q8_K: fn = oracle_quantize_q8_K; break;
    case ORACLE_TYPE_Q4_K: fn = oracle_quantize_q4_K; break;
    case ORACLE_TYPE_Q5_K: fn = oracle_quantize_q5_K; break;
    case ORACLE_TYPE_Q6_K: fn = oracle_quantize_q6_K; break;
    case ORACLE_TYPE_BF16: fn = oracle_quantize_bf16; break;
    default: return -1;
    }
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
    for (int64_t r = 0; r < n; r++) fn(x + r * k, (uint8_t *) y + (size_t) r * rs, k);
    (void) nthreads;
    return 0;
}

/* ---------------------------------------------------------------------------------------------------------------
 * Dequantizers (float op order as gguf-py's, so results are bit-identical to it).
 * ------------------------------------------------------------------------------------------------------------- */

static void q4_K_scale_min(const uint8_t * s, int j, uint8_t * sc, uint8_t * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t) ((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t) ((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Value v (0..255) of a Q6_K block as the signed six-bit integer q - 32. */
static int q6_K_value(const oracle_block_q6_K * b, int v) {
    const int h = v >> 7, t = (v >> 5) & 3, l = v & 31;
    const int lo = (b->ql[h * 64 + (t & 1) * 32 + l] >> ((t >> 1) * 4)) & 15;
    const int hi = (b->qh[h * 32 + l] >> (2 * t)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* Value v (0..255) of a Q5_K block as the unsigned five-bit integer. */
static int q5_K_value(const oracle_block_q5_K * b, int v) {
    const int s = v >> 5, l = v & 31;
    return ((b->qs[(s >> 1) * 32 + l] >> ((s & 1) * 4)) & 15) | (((b->qh[l] >> s) & 1) << 4);
}

/* Value v (0..255) of a Q4_K block as the unsigned four-bit integer. */
static int q4_K_value(const oracle_block_q4_K * b, int v) {
    const int s = v >> 5, l = v & 31;
    return (b->qs[(s >> 1) * 32 + l] >> ((s & 1) * 4)) & 15;
}

int oracle_dequantize_row(int type, const void * vx, float * y, int64_t k) {
    if (!oracle_row_size(type, k)) return -1;
    switch (type) {
    case ORACLE_TYPE_F32: memcpy(y, vx, (size_t) k * 4); return 0;
    case ORACLE_TYPE_F16: {
        const uint16_t * x = (const uint16_t *) vx;
        for (int64_t i = 0; i < k; i++) y[i] = oracle_fp16_to_fp32(x[i]);
        return 0;
    }
    case ORACLE_TYPE_BF16: {
        const uint16_t * x = (const uint16_t *) vx;
        for (int64_t i = 0; i < k; i++) y[i] = oracle_bf16_to_fp32(x[i]);
        return 0;
    }
    case ORACLE_TYPE_Q8_0: {
        const oracle_block_q8_0 * x = (const oracle_block_q8_0 *) vx;
        for (int64_t i = 0; i < k / 32; i++) {
            const float d = oracle_fp16_to_fp32(x[i].d);
            for (int j = 0; j < 32; j++) y[i * 32 + j] = (float) x[i].qs[j] * d;
        }
        return 0;
    }
    case ORACLE_TYPE_Q5_K: {
        const oracle_block_q5_K * x = (const oracle_block_q5_K *) vx;
        for (int64_t i = 0; i < k / 256; i++) {
            const float d = oracle_fp16_to_fp32(x[i].d), dmin = oracle_fp16_to_fp32(x[i].dmin);
            for (int s = 0; s < 8; s++) {
                uint8_t sc, m;
                q4_K_scale_min(x[i].scales, s, &sc, &m);
                const float ds = d * (float) sc, dm = dmin * (float) m;
                for (int l = 0; l < 32; l++) y[i * 256 + s * 32 + l] = ds * (float) q5_K_value(&x[i], s * 32 + l) - dm;
            }
        }
        return 0;
    }
    case ORACLE_TYPE_Q4_K: {
        const oracle_block_q4_K * x = (const oracle_block_q4_K *) vx;
        for (int64_t i = 0; i < k / 256; i++) {
            const float d = oracle_fp16_to_fp32(x[i].d), dmin = oracle_fp16_to_fp32(x[i].dmin);
            for (int s = 0; s < 8; s++) {
                uint8_t sc, m;
                q4_K_scale_min(x[i].scales, s, &sc, &m);
                const float ds = d * (float) sc, dm = dmin * (float) m;
                for (int l = 0; l < 32; l++) y[i * 256 + s * 32 + l] = ds * (float) q4_K_value(&x[i], s * 32 + l) - dm;
            }
        }
        return 0;
    }
    case ORACLE_TYPE_Q6_K: {
        const oracle_block_q6_K * x = (const oracle_block_q6_K *) vx;
        for (int64_t i = 0; i < k / 256; i++) {
            const float d = oracle_fp16_to_fp32(x[i].d);
            for (int v = 0; v < 256; v++) y[i * 256 + v] = (d * (float) x[i].scales[v / 16]) * (float) q6_K_value(&x[i], v);
        }
        return 0;
    }
    case ORACLE_TYPE_Q8_K: {
        const oracle_block_q8_K * x = (const oracle_block_q8_K *) vx;
        for (int64_t i = 0; i < k / 256; i++)
            for (int j = 0; j < 256; j++) y[i * 256 + j] = x[i].d * (float) x[i].qs[j];
        return 0;
    }
    default: return -1;
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Dot products. Integer parts are exact. Each (super-)block contributes ggml's term: its exact int32 sum times the
 * float32 product of the two scales, formed as ggml's CPU vec_dot forms it (Q8_0: d_w * d_x; Q4_K: d_x * d and
 * d_x * dmin; Q6_K: d * d_x). ggml accumulates those terms in float32, in an order that depends on its SIMD path
 * (the generic C loop goes in block order; the AVX2, AVX-512 and NEON loops keep 8, 16 or 4 partial sums and add them
 * at the end), so no single float32 order is ggml's. The oracle takes the one order-free definition: the exact sum of
 * the terms, rounded once to float32. Each term is exact in double (a 24-bit float times an integer below 2^26) and
 * the double sum's own rounding is about 1e-16 of the sum of magnitudes, so the result is the exactly rounded sum
 * unless the true sum lies within that distance of a float32 rounding boundary. Every ggml order lies within a few
 * float32 ulps of it, inside the products' stated tolerance (1e-4 of sum |w x|).
 * ------------------------------------------------------------------------------------------------------------- */

static float dot_q8_0(const oracle_block_q8_0 * w, const oracle_block_q8_0 * x, int64_t nb) {
    double sum = 0.0;
    for (int64_t i = 0; i < nb; i++) {
        int sumi = 0;
        for (int j = 0; j < 32; j++) sumi += (int) w[i].qs[j] * (int) x[i].qs[j];
        const float d = oracle_fp16_to_fp32(w[i].d) * oracle_fp16_to_fp32(x[i].d);
        sum += (double) d * (double) sumi;
    }
    return (float) sum;
}

static void sums_q4_K(const oracle_block_q4_K * w, const oracle_block_q8_K * x, int32_t * sumi, int32_t * summ) {
    int32_t si = 0, sm = 0;
    for (int s = 0; s < 8; s++) {
        uint8_t sc, m;
        q4_K_scale_min(w->scales, s, &sc, &m);
        int32_t isum = 0;
        for (int l = 0; l < 32; l++) isum += q4_K_value(w, s * 32 + l) * (int) x->qs[s * 32 + l];
        si += (int32_t) sc * isum;
        sm += (int32_t) m * ((int32_t) x->bsums[2 * s] + (int32_t) x->bsums[2 * s + 1]);
    }
    *sumi = si;
    *summ = sm;
}

static void sums_q5_K(const oracle_block_q5_K * w, const oracle_block_q8_K * x, int32_t * sumi, int32_t * summ) {
    int32_t si = 0, sm = 0;
    for (int s = 0; s < 8; s++) {
        uint8_t sc, m;
        q4_K_scale_min(w->scales, s, &sc, &m);
        int32_t isum = 0;
        for (int l = 0; l < 32; l++) isum += q5_K_value(w, s * 32 + l) * (int) x->qs[s * 32 + l];
        si += (int32_t) sc * isum;
        sm += (int32_t) m * ((int32_t) x->bsums[2 * s] + (int32_t) x->bsums[2 * s + 1]);
    }
    *sumi = si;
    *summ = sm;
}

static int32_t sums_q6_K(const oracle_block_q6_K * w, const oracle_block_q8_K * x) {
    int32_t si = 0;
    for (int g = 0; g < 16; g++) {
        int32_t isum = 0;
        for (int l = 0; l < 16; l++) isum += q6_K_value(w, g * 16 + l) * (int) x->qs[g * 16 + l];
        si += (int32_t) w->scales[g] * isum;
    }
    return si;
}

static float dot_q4_K(const oracle_block_q4_K * w, const oracle_block_q8_K * x, int64_t nb) {
    double sum = 0.0;
    for (int64_t i = 0; i < nb; i++) {
        int32_t sumi, summ;
        sums_q4_K(&w[i], &x[i], &sumi, &summ);
        const float d = x[i].d * oracle_fp16_to_fp32(w[i].d);
        const float dmin = x[i].d * oracle_fp16_to_fp32(w[i].dmin);
        sum += (double) d * (double) sumi;
        sum -= (double) dmin * (double) summ;
    }
    return (float) sum;
}

static float dot_q5_K(const oracle_block_q5_K * w, const oracle_block_q8_K * x, int64_t nb) {
    double sum = 0.0;
    for (int64_t i = 0; i < nb; i++) {
        int32_t sumi, summ;
        sums_q5_K(&w[i], &x[i], &sumi, &summ);
        const float d = x[i].d * oracle_fp16_to_fp32(w[i].d);
        const float dmin = x[i].d * oracle_fp16_to_fp32(w[i].dmin);
        sum += (double) d * (double) sumi;
        sum -= (double) dmin * (double) summ;
    }
    return (float) sum;
}

static float dot_q6_K(const oracle_block_q6_K * w, const oracle_block_q8_K * x, int64_t nb) {
    double sum = 0.0;
    for (int64_t i = 0; i < nb; i++) {
        const float d = oracle_fp16_to_fp32(w[i].d) * x[i].d;
        sum += (double) d * (double) sums_q6_K(&w[i], &x[i]);
    }
    return (float) sum;
}

static float dot_bf16(const uint16_t * w, const uint16_t * x, int64_t k) {
    double s = 0.0;
    for (int64_t i = 0; i < k; i++) s += (double) (oracle_bf16_to_fp32(w[i]) * oracle_bf16_to_fp32(x[i]));
    return (float) s;
}

static float dot_f32(const float * w, const float * x, int64_t k) {
    double s = 0.0;
    for (int64_t i = 0; i < k; i++) s += (double) (w[i] * x[i]);
    return (float) s;
}

float oracle_vec_dot(int type, const void * w, const void * x, int64_t k) {
    switch (type) {
    case ORACLE_TYPE_Q8_0: return dot_q8_0((const oracle_block_q8_0 *) w, (const oracle_block_q8_0 *) x, k / 32);
    case ORACLE_TYPE_Q4_K: return dot_q4_K((const oracle_block_q4_K *) w, (const oracle_block_q8_K *) x, k / 256);
    case ORACLE_TYPE_Q5_K: return dot_q5_K((const oracle_block_q5_K *) w, (const oracle_block_q8_K *) x, k / 256);
    case ORACLE_TYPE_Q6_K: return dot_q6_K((const oracle_block_q6_K *) w, (const oracle_block_q8_K *) x, k / 256);
    case ORACLE_TYPE_BF16: return dot_bf16((const uint16_t *) w, (const uint16_t *) x, k);
    case ORACLE_TYPE_F32: return dot_f32((const float *) w, (const float *) x, k);
    default: return NAN;
    }
}

int64_t oracle_block_sums(int type, const void * vw, const void * vx, int64_t k, int32_t * out) {
    switch (type) {
    case ORACLE_TYPE_Q8_0: {
        const oracle_block_q8_0 * w = (const oracle_block_q8_0 *) vw;
        const oracle_block_q8_0 * x = (const oracle_block_q8_0 *) vx;
        for (int64_t i = 0; i < k / 32; i++) {
            int32_t s = 0;
            for (int j = 0; j < 32; j++) s += (int32_t) w[i].qs[j] * (int32_t) x[i].qs[j];
            out[i] = s;
        }
        return k / 32;
    }
    case ORACLE_TYPE_Q4_K: {
        const oracle_block_q4_K * w = (const oracle_block_q4_K *) vw;
        const oracle_block_q8_K * x = (const oracle_block_q8_K *) vx;
        for (int64_t i = 0; i < k / 256; i++) sums_q4_K(&w[i], &x[i], &out[2 * i], &out[2 * i + 1]);
        return 2 * (k / 256);
    }
    case ORACLE_TYPE_Q5_K: {
        const oracle_block_q5_K * w = (const oracle_block_q5_K *) vw;
        const oracle_block_q8_K * x = (const oracle_block_q8_K *) vx;
        for (int64_t i = 0; i < k / 256; i++) sums_q5_K(&w[i], &x[i], &out[2 * i], &out[2 * i + 1]);
        return 2 * (k / 256);
    }
    case ORACLE_TYPE_Q6_K: {
        const oracle_block_q6_K * w = (const oracle_block_q6_K *) vw;
        const oracle_block_q8_K * x = (const oracle_block_q8_K *) vx;
        for (int64_t i = 0; i < k / 256; i++) out[i] = sums_q6_K(&w[i], &x[i]);
        return k / 256;
    }
    default: return -1;
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Nodes.
 * ------------------------------------------------------------------------------------------------------------- */

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Quantizes each of M rows of x to the vec_dot type of `type`; returns malloc'd blocks (or x itself for F32). */
static void * quantize_activations(int type, const float * x, int64_t K, int64_t M, size_t * row_bytes, int nthreads) {
    const int vt = oracle_vec_dot_type(type);
    if (vt == ORACLE_TYPE_F32) {
        *row_bytes = (size_t) K * 4;
        return NULL;
    }
    *row_bytes = oracle_row_size(vt, K);
    void * q = malloc(*row_bytes * (size_t) (M ? M : 1));
    if (!q) return NULL;
    oracle_quantize_rows(vt, x, q, K, M, nthreads);
    return q;
}

int oracle_mul_mat(int type, const void * w, int64_t K, int64_t N, const float * x, int64_t M, float * dst, int nthreads) {
    const size_t wrs = oracle_row_size(type, K);
    if (!wrs || oracle_vec_dot_type(type) < 0 || K <= 0 || N < 0 || M < 0) return -1;
    size_t xrs = 0;
    void * xq = quantize_activations(type, x, K, M, &xrs, nthreads);
    const uint8_t * xb = xq ? (const uint8_t *) xq : (const uint8_t *) x;
    if (!xb && M > 0) return -1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for collapse(2) num_threads(nthreads) schedule(static)
#endif
    for (int64_t m = 0; m < M; m++)
        for (int64_t n = 0; n < N; n++)
            dst[m * N + n] = oracle_vec_dot(type, (const uint8_t *) w + (size_t) n * wrs, xb + (size_t) m * xrs, K);
    free(xq);
    (void) nthreads;
    return 0;
}

int oracle_mul_mat_id(int type, const void * experts, int64_t K, int64_t N, int64_t E, const float * b, int64_t nb1,
                      const int32_t * ids, int64_t top_k, int64_t T, float * dst, int nthreads) {
    const size_t wrs = oracle_row_size(type, K);
    if (!wrs || oracle_vec_dot_type(type) < 0 || (nb1 != 1 && nb1 != top_k) || top_k <= 0 || T < 0) return -1;
    for (int64_t i = 0; i < T * top_k; i++)
        if (ids[i] < 0 || ids[i] >= E) return -2;
    size_t xrs = 0;
    void * xq = quantize_activations(type, b, K, T * nb1, &xrs, nthreads);
    const uint8_t * xb = xq ? (const uint8_t *) xq : (const uint8_t *) b;
    if (!xb && T > 0) return -1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for collapse(2) num_threads(nthreads) schedule(static)
#endif
    for (int64_t t = 0; t < T; t++)
        for (int64_t s = 0; s < top_k; s++) {
            const int64_t e = ids[t * top_k + s];
            const uint8_t * ew = (const uint8_t *) experts + (size_t) e * (size_t) N * wrs;
            const uint8_t * xr = xb + (size_t) (t * nb1 + (nb1 == 1 ? 0 : s)) * xrs;
            float * o = dst + (t * top_k + s) * N;
            for (int64_t n = 0; n < N; n++) o[n] = oracle_vec_dot(type, ew + (size_t) n * wrs, xr, K);
        }
    free(xq);
    (void) nthreads;
    return 0;
}

int oracle_get_rows(int type, const void * table, int64_t K, int64_t rows, const int32_t * ids, int64_t n, float * dst) {
    const size_t rs = oracle_row_size(type, K);
    if (!rs) return -1;
    for (int64_t i = 0; i < n; i++) {
        if (ids[i] < 0 || ids[i] >= rows) return -2;
        oracle_dequantize_row(type, (const uint8_t *) table + (size_t) ids[i] * rs, dst + i * K, K);
    }
    return 0;
}
