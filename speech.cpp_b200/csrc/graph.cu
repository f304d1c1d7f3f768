// graph.cu — the backend's graph_compute: the ops of a Qwen3 decoder graph besides the quantized products
// (Qwen3Decoder::layers / outputs, src/common/qwen3-decoder.cpp:350-438; the cache's FILL at :320-321 and the talker's
// CONCAT, src/families/qwen3-tts/talker.cpp:55, 174), over ggml-shaped tensor records
// (b200_graph_compute, include/b200.h).
//
// Tensors are strided views: element [i0, i1, i2, i3] of a record lives at data + i0 nb0 + i1 nb1 + i2 nb2 + i3 nb3,
// as in ggml, so permutes, transposes and cache views need no copies. The ops are memory- or latency-bound (a decode
// step moves kilobytes through each); every kernel walks its output with a grid-stride loop, one thread per element,
// or one warp per row where a row reduces (RMS_NORM, SOFT_MAX, ARGMAX, products of plain matrices), or one CTA per
// (query, head) for attention. Reductions follow the oracle's definitions: sums and exponentials in double, rounded
// once to float32; products of F16 / F32 matrices with the activations rounded to the matrix's type first.
#include <cmath>

#include "internal.h"

using namespace b200;

namespace {

struct TView {
    uint8_t * p;
    int64_t ne[4];
    int64_t nb[4];
    int type;
};

TView view(const b200_tensor & t) {
    TView v;
    v.p = (uint8_t *) t.data;
    for (int i = 0; i < 4; i++) {
        v.ne[i] = t.ne[i];
        v.nb[i] = t.nb[i];
    }
    v.type = t.type;
    return v;
}

__device__ __forceinline__ const uint8_t * at(const TView & t, int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
    return t.p + i0 * t.nb[0] + i1 * t.nb[1] + i2 * t.nb[2] + i3 * t.nb[3];
}

__device__ __forceinline__ float ld(const TView & t, int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
    const uint8_t * q = at(t, i0, i1, i2, i3);
    return t.type == B200_TYPE_F16 ? __half2float(*reinterpret_cast<const __half *>(q)) : *reinterpret_cast<const float *>(q);
}

__device__ __forceinline__ void st(const TView & t, int64_t i0, int64_t i1, int64_t i2, int64_t i3, float v) {
    uint8_t * q = const_cast<uint8_t *>(at(t, i0, i1, i2, i3));
    if (t.type == B200_TYPE_F16) *reinterpret_cast<__half *>(q) = __float2half_rn(v);
    else *reinterpret_cast<float *>(q) = v;
}

__device__ __forceinline__ void unflat(int64_t i, const int64_t * ne, int64_t & i0, int64_t & i1, int64_t & i2, int64_t & i3) {
    i0 = i % ne[0];
    i /= ne[0];
    i1 = i % ne[1];
    i /= ne[1];
    i2 = i % ne[2];
    i3 = i / ne[2];
}

__device__ __forceinline__ int64_t n_elems(const TView & t) { return t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]; }

// ---- element-wise ----

// kind 0: ADD, 1: MUL (src1 repeated), 2: SWIGLU (silu(a) * b, same shapes), 3: SCALE (a * s + b), 4: copy / convert,
// 5: FILL (every element s; a is not read)
__global__ void k_elementwise(TView a, TView b, TView d, int kind, float s, float bias) {
    const int64_t n = n_elems(d);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t i0, i1, i2, i3;
        unflat(i, d.ne, i0, i1, i2, i3);
        if (kind == 5) {
            st(d, i0, i1, i2, i3, s);
            continue;
        }
        const float x = ld(a, i0, i1, i2, i3);
        float y;
        switch (kind) {
        case 0: y = __fadd_rn(x, ld(b, i0 % b.ne[0], i1 % b.ne[1], i2 % b.ne[2], i3 % b.ne[3])); break;
        case 1: y = __fmul_rn(x, ld(b, i0 % b.ne[0], i1 % b.ne[1], i2 % b.ne[2], i3 % b.ne[3])); break;
        case 2: y = __fmul_rn(silu_exact(x), ld(b, i0, i1, i2, i3)); break;
        case 3: y = __fadd_rn(__fmul_rn(x, s), bias); break;
        default: y = x; break;
        }
        st(d, i0, i1, i2, i3, y);
    }
}

// CONCAT along dimension `dim`: d's index there below a.ne[dim] reads a, the rest read b shifted down by a.ne[dim].
__global__ void k_concat(TView a, TView b, TView d, int dim) {
    const int64_t n = n_elems(d);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t c[4];
        unflat(i, d.ne, c[0], c[1], c[2], c[3]);
        const int64_t k = c[dim];
        float v;
        if (k < a.ne[dim]) {
            v = ld(a, c[0], c[1], c[2], c[3]);
        } else {
            c[dim] = k - a.ne[dim];
            v = ld(b, c[0], c[1], c[2], c[3]);
            c[dim] = k;
        }
        st(d, c[0], c[1], c[2], c[3], v);
    }
}

// ---- row reductions: one warp per row (dimension 0) ----

__global__ void k_rms_norm(TView x, TView y, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = x.ne[1] * x.ne[2] * x.ne[3];
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t) (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const int64_t i1 = r % x.ne[1], i2 = (r / x.ne[1]) % x.ne[2], i3 = r / (x.ne[1] * x.ne[2]);
        double sq = 0.0;
        for (int64_t i0 = lane; i0 < x.ne[0]; i0 += 32) {
            const double v = ld(x, i0, i1, i2, i3);
            sq = fma(v, v, sq);
        }
        sq = warp_sum_d(sq);
        const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean_rounded(sq, x.ne[0]), eps)));
        for (int64_t i0 = lane; i0 < x.ne[0]; i0 += 32) st(y, i0, i1, i2, i3, __fmul_rn(ld(x, i0, i1, i2, i3), scale));
    }
}

// softmax(x * scale + mask) along dimension 0: v = fl(fl(x * scale) + mask); e = fl32(exp(v - max)); s = fl32(sum e in
// double); y = fl(e / s). The mask's row is the row's i1 (broadcast over dimensions 2 and 3).
__global__ void k_soft_max(TView x, TView mask, int has_mask, TView y, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = x.ne[1] * x.ne[2] * x.ne[3];
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t) (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const int64_t i1 = r % x.ne[1], i2 = (r / x.ne[1]) % x.ne[2], i3 = r / (x.ne[1] * x.ne[2]);
        auto value = [&](int64_t i0) {
            float v = __fmul_rn(ld(x, i0, i1, i2, i3), scale);
            if (has_mask) v = __fadd_rn(v, ld(mask, i0, i1, 0, 0));
            return v;
        };
        float m = -INFINITY;
        for (int64_t i0 = lane; i0 < x.ne[0]; i0 += 32) m = fmaxf(m, value(i0));
        m = warp_max(m);
        double sum = 0.0;
        for (int64_t i0 = lane; i0 < x.ne[0]; i0 += 32) {
            const float e = __double2float_rn(exp((double) __fsub_rn(value(i0), m)));
            st(y, i0, i1, i2, i3, e);
            sum += (double) e;
        }
        const float s = __double2float_rn(warp_sum_d(sum));
        __syncwarp();
        for (int64_t i0 = lane; i0 < x.ne[0]; i0 += 32) st(y, i0, i1, i2, i3, __fdiv_rn(ld(y, i0, i1, i2, i3), s));
    }
}

__global__ void k_argmax(TView x, int32_t * out) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = x.ne[1] * x.ne[2] * x.ne[3];
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t) (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const int64_t i1 = r % x.ne[1], i2 = (r / x.ne[1]) % x.ne[2], i3 = r / (x.ne[1] * x.ne[2]);
        float best = -INFINITY;
        int64_t idx = -1;  // -1: no value seen (NaN values are never taken)
        for (int64_t i0 = lane; i0 < x.ne[0]; i0 += 32) {
            const float v = ld(x, i0, i1, i2, i3);
            if (v > best || (idx < 0 && v == best)) {  // strictly larger: a lane keeps its first of equal values
                best = v;
                idx = i0;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (oi >= 0 && (idx < 0 || ob > best || (ob == best && oi < idx))) {
                best = ob;
                idx = oi;
            }
        }
        if (lane == 0) out[r] = (int32_t) (idx >= 0 ? idx : 0);
    }
}

// ---- products of plain (F16 / F32) matrices: one warp per output element ----
// dst[n, m, i2, i3] = sum_k a[k, n, i2 / r2, i3 / r3] * b[k, m, i2, i3], b rounded to a's type first (ggml's CPU
// converts src1 to the vec_dot type of src0), each product rounded to float32 (exact for F16 x F16), summed in double.
__global__ void k_mul_mat_plain(TView a, TView b, TView d) {
    const int lane = threadIdx.x & 31;
    const int64_t outs = d.ne[0] * d.ne[1] * d.ne[2] * d.ne[3];
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    const int64_t r2 = d.ne[2] / a.ne[2], r3 = d.ne[3] / a.ne[3];
    for (int64_t o = blockIdx.x * (int64_t) (blockDim.x >> 5) + (threadIdx.x >> 5); o < outs; o += warps) {
        int64_t n, m, i2, i3;
        unflat(o, d.ne, n, m, i2, i3);
        double acc = 0.0;
        for (int64_t k = lane; k < a.ne[0]; k += 32) {
            float bv = ld(b, k, m, i2, i3);
            if (a.type == B200_TYPE_F16) bv = __half2float(__float2half_rn(bv));
            acc += (double) __fmul_rn(ld(a, k, n, i2 / r2, i3 / r3), bv);
        }
        acc = warp_sum_d(acc);
        if (lane == 0) st(d, n, m, i2, i3, __double2float_rn(acc));
    }
}

// ---- rows and positions ----

// NEOX rotation: for i < n_dims / 2 the pair (x[i], x[i + n_dims/2]) of head i1 of token i2 turns by
// theta = pos[i2] * base^(-2 i / n_dims) (double; cos and sin rounded once to float32); values past n_dims are copied.
__global__ void k_rope_neox(TView x, const int32_t * pos, TView y, int n_dims, double base) {
    const int half = n_dims / 2;
    const int64_t n = n_elems(x);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t i0, i1, i2, i3;
        unflat(i, x.ne, i0, i1, i2, i3);
        if (i0 >= n_dims) {
            st(y, i0, i1, i2, i3, ld(x, i0, i1, i2, i3));
            continue;
        }
        if (i0 >= half) continue;  // the pair's first index handles it
        const double theta = (double) pos[i2] * pow(base, -2.0 * (double) i0 / (double) n_dims);
        const float c = __double2float_rn(cos(theta)), s = __double2float_rn(sin(theta));
        const float x0 = ld(x, i0, i1, i2, i3), x1 = ld(x, i0 + half, i1, i2, i3);
        st(y, i0, i1, i2, i3, __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
        st(y, i0 + half, i1, i2, i3, __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
    }
}

// dst[:, idx[i1], i2, i3] = src[:, i1, i2, i3] (converted to dst's type); idx I32 [ne1].
__global__ void k_set_rows(TView src, const int32_t * idx, TView dst, unsigned * err) {
    const int64_t n = n_elems(src);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t i0, i1, i2, i3;
        unflat(i, src.ne, i0, i1, i2, i3);
        const int64_t r = idx[i1];
        if (r < 0 || r >= dst.ne[1]) {
            atomicOr(err, B200_DEVERR_ROWS);
            continue;
        }
        st(dst, i0, r, i2, i3, ld(src, i0, i1, i2, i3));
    }
}

// dst[:, i, j, k] = table[:, ids[i, j, k], j, k] for a plain (F32 / F16) table.
__global__ void k_get_rows_plain(TView table, TView ids, TView dst, unsigned * err) {
    const int64_t n = n_elems(dst);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t i0, i1, i2, i3;
        unflat(i, dst.ne, i0, i1, i2, i3);
        const int32_t r = *reinterpret_cast<const int32_t *>(at(ids, i1, i2, i3, 0));
        if (r < 0 || r >= table.ne[1]) {
            atomicOr(err, B200_DEVERR_ROWS);
            continue;
        }
        st(dst, i0, i1, i2, i3, ld(table, i0, r, i2, i3));
    }
}

// ---- attention: one CTA per (query row, head) ----
// Scores s_j = fl32(sum_d fp16(q_d) k_dj) * scale + mask[j, iq]; w_j = fl32(exp(s_j - max)); out = fl32(sum_j w_j v_j /
// sum_j w_j), the sums in double. Key / value head = head / (H / H_kv). Scores and weights live in shared memory.
__global__ void k_flash_attn(TView q, TView k, TView v, TView mask, int has_mask, TView out, float scale) {
    extern __shared__ float sw[];  // [n_kv] scores, then weights
    __shared__ float qh[1024];
    __shared__ double red[32];
    __shared__ float smax;
    __shared__ double ssum;
    const int64_t D = q.ne[0], nkv = k.ne[1], H = q.ne[2], Hkv = k.ne[2];
    const int64_t iq = blockIdx.x, h = blockIdx.y, hk = h / (H / Hkv);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int64_t d = threadIdx.x; d < D; d += blockDim.x) qh[d] = __half2float(__float2half_rn(ld(q, d, iq, h, 0)));
    __syncthreads();
    // scores: one warp per key
    float lmax = -INFINITY;
    for (int64_t j = warp; j < nkv; j += nw) {
        double acc = 0.0;
        for (int64_t d = lane; d < D; d += 32) acc += (double) __fmul_rn(qh[d], ld(k, d, j, hk, 0));
        acc = warp_sum_d(acc);
        float s = __fmul_rn(__double2float_rn(acc), scale);
        if (has_mask) s = __fadd_rn(s, ld(mask, j, iq, 0, 0));
        if (lane == 0) sw[j] = s;
        lmax = fmaxf(lmax, s);
    }
    if (lane == 0) red[warp] = (double) lmax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = -INFINITY;
        for (int w = 0; w < nw; w++) m = fmaxf(m, (float) red[w]);
        smax = m;
    }
    __syncthreads();
    double lsum = 0.0;
    for (int64_t j = threadIdx.x; j < nkv; j += blockDim.x) {
        const float w = __double2float_rn(exp((double) __fsub_rn(sw[j], smax)));
        sw[j] = w;
        lsum += (double) w;
    }
    lsum = warp_sum_d(lsum);
    __syncthreads();
    if (lane == 0) red[warp] = lsum;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < nw; w++) t += red[w];
        ssum = t;
    }
    __syncthreads();
    for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
        double acc = 0.0;
        for (int64_t j = 0; j < nkv; j++) acc += (double) __fmul_rn(sw[j], ld(v, d, j, hk, 0));
        st(out, d, h, iq, 0, __double2float_rn(acc / ssum));
    }
}

unsigned grid_for(int64_t n, int per_block, int num_sms) {
    int64_t b = (n + per_block - 1) / per_block;
    const int64_t cap = (int64_t) num_sms * 16;
    if (b > cap) b = cap;
    return (unsigned) (b < 1 ? 1 : b);
}

float fparam(const b200_tensor & t, int i) {
    float f;
    std::memcpy(&f, &t.params[i], sizeof f);
    return f;
}

bool plain_float(const b200_tensor & t) { return !t.weight && (t.type == B200_TYPE_F32 || t.type == B200_TYPE_F16); }

bool same_shape(const b200_tensor & a, const b200_tensor & b) {
    for (int i = 0; i < 4; i++)
        if (a.ne[i] != b.ne[i]) return false;
    return true;
}

bool repeats(const b200_tensor & a, const b200_tensor & b) {  // b can be repeated to a's shape
    for (int i = 0; i < 4; i++)
        if (b.ne[i] <= 0 || a.ne[i] % b.ne[i]) return false;
    return true;
}

bool contiguous_rows(const b200_tensor & t, int64_t elem) { return t.nb[0] == elem && t.nb[1] == t.ne[0] * elem; }

const b200_tensor * src_of(const b200_tensor * ts, int64_t n, int64_t i, int j) {
    const int32_t s = ts[i].src[j];
    return (s >= 0 && s < i && s < n) ? &ts[s] : nullptr;
}

bool supports(const b200_tensor * ts, int64_t n, int64_t i) {
    if (i < 0 || i >= n) return false;
    const b200_tensor & t = ts[i];
    const b200_tensor * a = src_of(ts, n, i, 0);
    const b200_tensor * b = src_of(ts, n, i, 1);
    for (int d = 0; d < 4; d++)
        if (t.ne[d] <= 0) return false;
    switch (t.op) {
    case B200_OP_NONE: return true;
    case B200_OP_GET_ROWS:
        if (!a || !b || b->type != B200_TYPE_I32 || t.type != B200_TYPE_F32) return false;
        if (a->weight)
            return b->ne[1] == 1 && b->ne[2] == 1 && b->ne[3] == 1 && b->nb[0] == 4 && contiguous_rows(t, 4) && t.ne[0] == a->weight->ne0 &&
                   t.ne[1] == b->ne[0];
        return plain_float(*a) && t.ne[0] == a->ne[0] && t.ne[1] == b->ne[0];
    case B200_OP_MUL_MAT:
        if (!a || !b || t.type != B200_TYPE_F32 || b->type != B200_TYPE_F32 || t.ne[0] != (a->weight ? a->weight->ne1 : a->ne[1]))
            return false;
        if (a->weight)
            return a->weight->ne2 == 1 && b->ne[0] == a->weight->ne0 && b->ne[2] == 1 && b->ne[3] == 1 && contiguous_rows(*b, 4) &&
                   contiguous_rows(t, 4) && t.ne[1] == b->ne[1];
        return plain_float(*a) && a->ne[0] == b->ne[0] && t.ne[1] == b->ne[1] && t.ne[2] == b->ne[2] && t.ne[3] == b->ne[3] &&
               b->ne[2] % a->ne[2] == 0 && b->ne[3] % a->ne[3] == 0;
    case B200_OP_RMS_NORM:
    case B200_OP_CONT:
        return a && plain_float(*a) && plain_float(t) && same_shape(*a, t);
    case B200_OP_MUL:
    case B200_OP_ADD:
        return a && b && plain_float(*a) && plain_float(*b) && plain_float(t) && same_shape(*a, t) && repeats(t, *b);
    case B200_OP_SWIGLU:
        return a && b && plain_float(*a) && plain_float(*b) && plain_float(t) && same_shape(*a, t) && same_shape(*b, t);
    case B200_OP_SCALE:
        return a && plain_float(*a) && plain_float(t) && same_shape(*a, t);
    case B200_OP_ROPE: {
        const int n_dims = t.params[0];
        return a && b && plain_float(*a) && plain_float(t) && same_shape(*a, t) && b->type == B200_TYPE_I32 && b->nb[0] == 4 &&
               b->ne[0] >= t.ne[2] && t.params[1] == 2 && n_dims > 0 && n_dims % 2 == 0 && n_dims <= t.ne[0] && fparam(t, 2) > 0.0f &&
               fparam(t, 3) == 1.0f && fparam(t, 4) == 0.0f && fparam(t, 5) == 1.0f && t.ne[3] == 1;
    }
    case B200_OP_SET_ROWS: {
        const b200_tensor * dst = src_of(ts, n, i, 2);
        return a && b && dst && plain_float(*a) && plain_float(*dst) && b->type == B200_TYPE_I32 && b->nb[0] == 4 && b->ne[0] == a->ne[1] &&
               a->ne[0] == dst->ne[0] && a->ne[2] == dst->ne[2] && a->ne[3] == dst->ne[3] && same_shape(*dst, t);
    }
    case B200_OP_CPY:
        return a && b && plain_float(*a) && plain_float(*b) && same_shape(*a, *b) && same_shape(*b, t);
    case B200_OP_SOFT_MAX:
        return a && plain_float(*a) && t.type == B200_TYPE_F32 && same_shape(*a, t) &&
               (!b || (plain_float(*b) && b->ne[0] == t.ne[0] && b->ne[1] >= t.ne[1]));
    case B200_OP_FLASH_ATTN: {
        const b200_tensor * v = src_of(ts, n, i, 2);
        const b200_tensor * m = src_of(ts, n, i, 3);
        if (!a || !b || !v || !plain_float(*a) || b->type != B200_TYPE_F16 || v->type != B200_TYPE_F16 || t.type != B200_TYPE_F32)
            return false;
        const int64_t D = a->ne[0], nq = a->ne[1], H = a->ne[2];
        return D <= 1024 && b->ne[0] == D && v->ne[0] == D && v->ne[1] == b->ne[1] && v->ne[2] == b->ne[2] && H % b->ne[2] == 0 &&
               a->ne[3] == 1 && t.ne[0] == D && t.ne[1] == H && t.ne[2] == nq && t.ne[3] == 1 && b->ne[1] <= 48 * 1024 &&
               (!m || (m->type == B200_TYPE_F16 && m->ne[0] >= b->ne[1] && m->ne[1] >= nq));
    }
    case B200_OP_ARGMAX:
        return a && plain_float(*a) && t.type == B200_TYPE_I32 && t.nb[0] == 4 && t.ne[0] == a->ne[1] * a->ne[2] * a->ne[3];
    case B200_OP_FILL:
        return plain_float(t) && (!a || same_shape(*a, t));
    case B200_OP_CONCAT: {
        const int dim = t.params[0];
        if (!a || !b || !plain_float(*a) || !plain_float(*b) || !plain_float(t) || dim < 0 || dim > 3) return false;
        for (int d = 0; d < 4; d++)
            if (d == dim ? t.ne[d] != a->ne[d] + b->ne[d] : (a->ne[d] != t.ne[d] || b->ne[d] != t.ne[d])) return false;
        return true;
    }
    default: return false;
    }
}

}  // namespace

extern "C" {

int b200_graph_supports(const b200_tensor * tensors, int64_t n, int64_t i) { return tensors && supports(tensors, n, i) ? 1 : 0; }

b200_status b200_graph_compute(b200_context * ctx, const b200_tensor * ts, int64_t n) {
    if (!ctx || (n > 0 && !ts) || n < 0) return B200_ERR_INVALID;
    cudaStream_t st = ctx->stream;
    const int sms = ctx->num_sms;
    for (int64_t i = 0; i < n; i++) {
        const b200_tensor & t = ts[i];
        if (t.op == B200_OP_NONE) continue;
        if (!supports(ts, n, i)) {
            ctx->last_error = "graph_compute: unsupported record " + std::to_string(i) + " (op " + std::to_string(t.op) + ")";
            return B200_ERR_UNSUPPORTED;
        }
        const b200_tensor * a = src_of(ts, n, i, 0);
        const b200_tensor * b = src_of(ts, n, i, 1);
        const TView d = view(t);
        const int64_t ne = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
        const TView none = view(t);
        switch (t.op) {
        case B200_OP_GET_ROWS:
            if (a->weight) {
                b200_status s = b200_get_rows(ctx, a->weight, (const int32_t *) b->data, b->ne[0], (float *) t.data);
                if (s != B200_OK) return s;
            } else {
                k_get_rows_plain<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), view(*b), d, ctx->dev_err);
            }
            break;
        case B200_OP_MUL_MAT:
            if (a->weight) {
                b200_status s = b200_mul_mat(ctx, a->weight, (const float *) b->data, b->ne[1], (float *) t.data);
                if (s != B200_OK) return s;
            } else {
                k_mul_mat_plain<<<grid_for(ne, 8, sms), 256, 0, st>>>(view(*a), view(*b), d);
            }
            break;
        case B200_OP_RMS_NORM:
            k_rms_norm<<<grid_for(ne / t.ne[0], 8, sms), 256, 0, st>>>(view(*a), d, fparam(t, 0));
            break;
        case B200_OP_ADD:
        case B200_OP_MUL:
            k_elementwise<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), view(*b), d, t.op == B200_OP_ADD ? 0 : 1, 0.0f, 0.0f);
            break;
        case B200_OP_SWIGLU:
            k_elementwise<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), view(*b), d, 2, 0.0f, 0.0f);
            break;
        case B200_OP_SCALE:
            k_elementwise<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), none, d, 3, fparam(t, 0), fparam(t, 1));
            break;
        case B200_OP_CONT:
            k_elementwise<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), none, d, 4, 0.0f, 0.0f);
            break;
        case B200_OP_CPY:
            k_elementwise<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), none, view(*b), 4, 0.0f, 0.0f);
            break;
        case B200_OP_FILL:
            k_elementwise<<<grid_for(ne, 256, sms), 256, 0, st>>>(none, none, d, 5, fparam(t, 0), 0.0f);
            break;
        case B200_OP_CONCAT:
            k_concat<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), view(*b), d, t.params[0]);
            break;
        case B200_OP_ROPE:
            k_rope_neox<<<grid_for(ne, 256, sms), 256, 0, st>>>(view(*a), (const int32_t *) b->data, d, t.params[0], (double) fparam(t, 2));
            break;
        case B200_OP_SET_ROWS: {
            const b200_tensor * dst = src_of(ts, n, i, 2);
            const int64_t ns = a->ne[0] * a->ne[1] * a->ne[2] * a->ne[3];
            k_set_rows<<<grid_for(ns, 256, sms), 256, 0, st>>>(view(*a), (const int32_t *) b->data, view(*dst), ctx->dev_err);
            break;
        }
        case B200_OP_SOFT_MAX:
            k_soft_max<<<grid_for(ne / t.ne[0], 8, sms), 256, 0, st>>>(view(*a), b ? view(*b) : none, b ? 1 : 0, d, fparam(t, 0));
            break;
        case B200_OP_FLASH_ATTN: {
            const b200_tensor * v = src_of(ts, n, i, 2);
            const b200_tensor * m = src_of(ts, n, i, 3);
            const dim3 grid((unsigned) a->ne[1], (unsigned) a->ne[2]);
            const size_t smem = (size_t) b->ne[1] * sizeof(float);
            if (smem > 48 * 1024) {
                cudaError_t e = cudaFuncSetAttribute(k_flash_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
                if (e != cudaSuccess) {
                    ctx->last_error = std::string("graph_compute: ") + cudaGetErrorString(e);
                    return B200_ERR_DEVICE;
                }
            }
            k_flash_attn<<<grid, 256, smem, st>>>(view(*a), view(*b), view(*v), m ? view(*m) : none, m ? 1 : 0, d, fparam(t, 0));
            break;
        }
        case B200_OP_ARGMAX:
            k_argmax<<<grid_for(t.ne[0], 8, sms), 256, 0, st>>>(view(*a), (int32_t *) t.data);
            break;
        default: break;
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            ctx->last_error = std::string("graph_compute: ") + cudaGetErrorString(e);
            return B200_ERR_DEVICE;
        }
    }
    return B200_OK;
}

}  // extern "C"
