// api.cu — the C ABI (include/b200.h): devices, contexts, weight buffers, and op dispatch.
#include <cstdio>
#include <cstring>

#include "internal.h"

using namespace b200;

namespace {

thread_local std::string g_error;  // errors before a context exists

b200_status fail(b200_context * ctx, b200_status s, const char * what) {
    if (ctx) ctx->last_error = what;
    else g_error = what;
    return s;
}

b200_status cuda_fail(b200_context * ctx, cudaError_t e, const char * where) {
    char buf[256];
    std::snprintf(buf, sizeof buf, "%s: %s", where, cudaGetErrorString(e));
    return fail(ctx, e == cudaErrorMemoryAllocation ? B200_ERR_ALLOC : B200_ERR_DEVICE, buf);
}

#define CK(ctx, call)                                           \
    do {                                                        \
        cudaError_t e_ = (call);                                \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
    } while (0)

bool known_weight_type(int t) {
    return t == B200_TYPE_Q8_0 || t == B200_TYPE_Q4_K || t == B200_TYPE_Q5_K || t == B200_TYPE_Q6_K || t == B200_TYPE_BF16 ||
           t == B200_TYPE_F32;
}

int64_t block_values(int t) {
    switch (t) {
    case B200_TYPE_Q8_0: return 32;
    case B200_TYPE_Q4_K:
    case B200_TYPE_Q5_K:
    case B200_TYPE_Q6_K:
    case B200_TYPE_Q8_K: return 256;
    default: return 1;
    }
}

int64_t block_bytes(int t) {
    switch (t) {
    case B200_TYPE_Q8_0: return 34;
    case B200_TYPE_Q4_K: return 144;
    case B200_TYPE_Q5_K: return 176;
    case B200_TYPE_Q6_K: return 210;
    case B200_TYPE_Q8_K: return 292;
    case B200_TYPE_BF16:
    case B200_TYPE_F16: return 2;
    case B200_TYPE_F32: return 4;
    default: return 0;
    }
}

// Grows the context's scratch to at least `bytes` (synchronizes the stream when it has to reallocate).
b200_status ensure_scratch(b200_context * ctx, size_t bytes) {
    if (ctx->scratch_bytes >= bytes) return B200_OK;
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->scratch) cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t want = bytes < ((size_t) 1 << 20) ? ((size_t) 1 << 20) : bytes;
    CK(ctx, cudaMalloc(&ctx->scratch, want));
    ctx->scratch_bytes = want;
    return B200_OK;
}

b200_status ensure_staging(b200_context * ctx, size_t bytes) {
    if (ctx->staging_bytes >= bytes) return B200_OK;
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->staging) cudaFree(ctx->staging);
    ctx->staging = nullptr;
    ctx->staging_bytes = 0;
    CK(ctx, cudaMalloc(&ctx->staging, bytes));
    ctx->staging_bytes = bytes;
    return B200_OK;
}

// Sub-allocation from scratch, 256-byte aligned.
struct Carve {
    uint8_t * base;
    size_t used = 0;
    template <class T>
    T * take(size_t count) {
        T * p = reinterpret_cast<T *>(base + used);
        used += (count * sizeof(T) + 255) & ~(size_t) 255;
        return p;
    }
};

size_t quantized_act_bytes(int kind, int64_t K, int64_t rows) {
    size_t b = (((size_t) rows * K + 255) & ~(size_t) 255);
    if (kind == B200_TYPE_Q8_0) b += (((size_t) rows * (K / 32) * 4 + 255) & ~(size_t) 255);
    else b += (((size_t) rows * (K / 256) * 4 + 255) & ~(size_t) 255) + (((size_t) rows * (K / 16) * 2 + 255) & ~(size_t) 255);
    return b;
}

bool check_weight(b200_context * ctx, const b200_weight * w) {
    return ctx && w && w->data && known_weight_type(w->type) && w->ne0 > 0 && w->ne1 > 0 && w->ne2 > 0 &&
           w->ne0 % block_values(w->type) == 0;
}

GemvParams base_params(b200_context * ctx, const b200_weight * w) {
    GemvParams p;
    std::memset(&p, 0, sizeof p);
    p.w = view_of(w);
    p.eps = 0.0f;
    p.err = ctx->dev_err;
    return p;
}

int pow2_at_least(int64_t m) {
    int nc = 1;
    while (nc < m) nc <<= 1;
    return nc;
}

// The product of rows [row0, row0 + n) of matrix 0 with M activation rows, through the GEMV kernels.
b200_status mul_mat_impl(b200_context * ctx, const b200_weight * w, int64_t row0, int64_t n, const float * x, int64_t M,
                         float * dst, int64_t ld_dst) {
    if (!check_weight(ctx, w)) return fail(ctx, B200_ERR_INVALID, "mul_mat: bad weight");
    if (w->type == B200_TYPE_F32) return fail(ctx, B200_ERR_UNSUPPORTED, "mul_mat: F32 weights are not on this path");
    if (M < 0 || row0 < 0 || n < 0 || row0 + n > w->ne1 * w->ne2 || (M > 0 && (!x || !dst)))
        return fail(ctx, B200_ERR_INVALID, "mul_mat: bad shape");
    if (M == 0 || n == 0) return B200_OK;
    const int64_t K = w->ne0;
    GemvParams p = base_params(ctx, w);
    p.N = n;
    p.row0 = row0;
    p.x = x;
    p.ldx = K;
    p.y = dst;
    p.ldy = ld_dst;
    const int maxnc = gemv_max_columns(w->type, K);
    if (maxnc == 0) return fail(ctx, B200_ERR_UNSUPPORTED, "mul_mat: rows too long for the staging buffer");
    if (M <= maxnc) {
        // Few columns: one GEMV launch. Launched with programmatic dependent launch (its CTAs start streaming weights
        // while the previous kernel finishes; activations are read after griddepcontrol.wait), except right after an
        // upload; a product of at most 64 MB of weights leaves room on every SM for the next launch's CTAs (up to 16 MB:
        // one CTA per SM with a half-size ring; up to 64 MB: two such CTAs per SM).
        p.ncols = (int) M;
        const bool pdl = !ctx->upload_pending;
        const double bytes = (double) n * (double) w->nbytes / (double) (w->ne1 * w->ne2);
        const int cap = bytes <= 16.0 * 1024 * 1024 ? 3 : bytes <= 64.0 * 1024 * 1024 ? 2 : 0;
        CK(ctx, launch_gemv(p, pow2_at_least(M), 1, ctx->stream, pdl, ctx->num_sms, cap));
        ctx->upload_pending = false;
        return B200_OK;
    }
    const int kind = act_kind(w->type);
    // Many columns of Q4_K / Q6_K: int8 tensor cores over an expanded copy of the weights (made once, cached).
    if (gemm_kq_tc_supported(p.w, M) && ((uintptr_t) x & 15) == 0) {
        b200_status s = ensure_scratch(ctx, gemm_kq_tc_act_bytes(K, M) + 256);
        if (s != B200_OK) return s;
        const cudaError_t e = launch_gemm_kq_tc(ctx, w, row0, n, x, M, dst, ld_dst, ctx->scratch);
        if (e == cudaSuccess) return B200_OK;
        if (e != cudaErrorInvalidValue) return cuda_fail(ctx, e, "launch_gemm_kq_tc");
        // a tensor map the driver refused: the GEMV path below computes the same product
    }
    // Many columns of Q8_0: int8 tensor cores (tcgen05) over the once-quantized activations: the persistent tile
    // kernel (32-token tiles x 128-row weight tiles, eight K blocks in flight) or the split-K GEMM.
    // Up to 128 rows: the persistent tile kernel, with K split across CTAs when there are few (token x row) tiles;
    // more rows run faster on the split-K GEMM below (measured on B200).
    if (M >= 32 && M <= 128 && gemm_tc_grouped_supported(p.w)) {
        const int64_t ld = (M + 15) & ~(int64_t) 15;
        const int ks = gemm_tc_dense_splits(p.w, n, M, ctx->num_sms);
        const size_t wsb = gemm_tc_dense_ws_bytes(n, M, ks);
        const int64_t out_tiles = ((M + 31) / 32) * ((n + 127) / 128);
        b200_status s = ensure_scratch(ctx, quantized_act_bytes(B200_TYPE_Q8_0, K, ld) + wsb + 1024);
        if (s != B200_OK) return s;
        if (ks > 1 && (size_t) out_tiles > ctx->ntickets) {
            CK(ctx, cudaStreamSynchronize(ctx->stream));
            if (ctx->tickets) cudaFree(ctx->tickets);
            ctx->tickets = nullptr;
            ctx->ntickets = 0;
            const size_t nt = (size_t) out_tiles < 4096 ? 4096 : (size_t) out_tiles;
            CK(ctx, cudaMalloc(&ctx->tickets, nt * sizeof(unsigned)));
            CK(ctx, cudaMemset(ctx->tickets, 0, nt * sizeof(unsigned)));
            ctx->ntickets = nt;
        }
        Carve c{(uint8_t *) ctx->scratch};
        int8_t * q = c.take<int8_t>((size_t) M * K);
        float * d = c.take<float>((size_t) ld * (K / 32));
        float * ws = ks > 1 ? c.take<float>(wsb / 4) : nullptr;
        CK(ctx, launch_quantize(kind, x, K, M, nullptr, q, d, nullptr, ctx->stream, ld));
        const cudaError_t e = launch_gemm_tc_dense(p.w, row0, n, q, d, ld, M, dst, ld_dst, ctx->dev_err, ctx->num_sms, ctx->stream, ks, ws,
                                                   ctx->tickets);
        if (e == cudaSuccess) return B200_OK;
        if (e != cudaErrorInvalidValue) return cuda_fail(ctx, e, "launch_gemm_tc_dense");
        // a tensor map the driver refused: the paths below compute the same product
    }
    if (gemm_tc_supported(p.w, M)) {
        const int64_t tiles = gemm_tc_tiles(n, M);
        const size_t qb = quantized_act_bytes(kind, K, M + 4), wsb = gemm_tc_workspace_bytes(n, M);
        b200_status s = ensure_scratch(ctx, qb + wsb + 256);
        if (s != B200_OK) return s;
        if ((size_t) tiles > ctx->ntickets) {
            CK(ctx, cudaStreamSynchronize(ctx->stream));
            if (ctx->tickets) cudaFree(ctx->tickets);
            ctx->tickets = nullptr;
            ctx->ntickets = 0;
            const size_t nt = (size_t) tiles < 4096 ? 4096 : (size_t) tiles;
            CK(ctx, cudaMalloc(&ctx->tickets, nt * sizeof(unsigned)));
            CK(ctx, cudaMemset(ctx->tickets, 0, nt * sizeof(unsigned)));
            ctx->ntickets = nt;
        }
        Carve c{(uint8_t *) ctx->scratch};
        int8_t * q = c.take<int8_t>((size_t) M * K);
        const int64_t ld = gemm_tc_dx_ld(M);
        float * d = c.take<float>((size_t) ld * (K / 32));
        void * ws = c.take<uint8_t>(wsb);
        CK(ctx, launch_quantize(kind, x, K, M, nullptr, q, d, nullptr, ctx->stream, ld));
        const cudaError_t e = launch_gemm_tc(p.w, row0, n, q, d, M, dst, ld_dst, ctx->dev_err, ws, wsb, ctx->tickets, ctx->num_sms,
                                             ctx->stream);
        if (e == cudaSuccess) return B200_OK;
        if (e != cudaErrorInvalidValue) return cuda_fail(ctx, e, "launch_gemm_tc");
        // a tensor map the driver refused: the GEMV path below computes the same product
    }
    // Many columns: quantize them once, then stream the weights once per chunk of `maxnc` columns.
    if (kind == B200_TYPE_BF16) {
        p.ncols = (int) M;
        CK(ctx, launch_gemv(p, maxnc, 1, ctx->stream, false, ctx->num_sms));
        return B200_OK;
    }
    b200_status s = ensure_scratch(ctx, quantized_act_bytes(kind, K, M));
    if (s != B200_OK) return s;
    Carve c{(uint8_t *) ctx->scratch};
    int8_t * q = c.take<int8_t>((size_t) M * K);
    float * d = c.take<float>((size_t) M * (K / (kind == B200_TYPE_Q8_0 ? 32 : 256)));
    int16_t * bs = kind == B200_TYPE_Q8_K ? c.take<int16_t>((size_t) M * (K / 16)) : nullptr;
    CK(ctx, launch_quantize(kind, x, K, M, nullptr, q, d, bs, ctx->stream));
    p.aq = q;
    p.ad = d;
    p.abs = bs;
    p.ncols = (int) M;
    CK(ctx, launch_gemv(p, maxnc, 1, ctx->stream, false, ctx->num_sms));
    return B200_OK;
}

}  // namespace

namespace b200 {

void set_thread_error(const char * what) { g_error = what; }

WeightView view_of(const b200_weight * w) {
    WeightView v;
    v.type = w->type;
    v.K = w->ne0;
    v.rows = w->ne1 * w->ne2;
    const uint8_t * base = (const uint8_t *) w->data;
    v.f0 = base + w->field_off[0];
    v.f1 = base + w->field_off[1];
    v.f2 = base + w->field_off[2];
    v.f3 = base + w->field_off[3];
    return v;
}

}  // namespace b200

extern "C" {

int b200_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

b200_status b200_device_info(int device, char * name, size_t name_len, size_t * free_bytes, size_t * total_bytes) {
    int n = b200_device_count();
    if (device < 0 || device >= n) return fail(nullptr, B200_ERR_INVALID, "device_info: no such device");
    if (name && name_len) std::snprintf(name, name_len, "B200_%d", device);
    if (free_bytes || total_bytes) {
        int prev = 0;
        cudaGetDevice(&prev);
        if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, B200_ERR_DEVICE, "device_info: cudaSetDevice");
        size_t f = 0, t = 0;
        cudaError_t e = cudaMemGetInfo(&f, &t);
        cudaSetDevice(prev);
        if (e != cudaSuccess) return fail(nullptr, B200_ERR_DEVICE, "device_info: cudaMemGetInfo");
        if (free_bytes) *free_bytes = f;
        if (total_bytes) *total_bytes = t;
    }
    return B200_OK;
}

b200_status b200_context_create(int device, b200_context ** out) {
    if (!out) return fail(nullptr, B200_ERR_INVALID, "context_create: out is NULL");
    *out = nullptr;
    if (device < 0 || device >= b200_device_count()) return fail(nullptr, B200_ERR_INVALID, "context_create: no such device");
    if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, B200_ERR_DEVICE, "context_create: cudaSetDevice");
    b200_context * ctx = new b200_context();
    ctx->device = device;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) {
        delete ctx;
        return fail(nullptr, B200_ERR_UNSUPPORTED, "context_create: the device is not sm_100 (B200)");
    }
    ctx->num_sms = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&ctx->dev_err, sizeof(unsigned)) != cudaSuccess || cudaMallocHost(&ctx->host_err, sizeof(unsigned)) != cudaSuccess ||
        cudaMemsetAsync(ctx->dev_err, 0, sizeof(unsigned), ctx->stream) != cudaSuccess) {
        b200_context_destroy(ctx);
        return fail(nullptr, B200_ERR_DEVICE, "context_create: stream / memory setup failed");
    }
    *out = ctx;
    return B200_OK;
}

void b200_context_destroy(b200_context * ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    b200::kq_release_all(ctx);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->staging) cudaFree(ctx->staging);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->tickets) cudaFree(ctx->tickets);
    if (ctx->host_err) cudaFreeHost(ctx->host_err);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

void * b200_context_stream(b200_context * ctx) { return ctx ? (void *) ctx->stream : nullptr; }

b200_status b200_synchronize(b200_context * ctx) {
    if (!ctx) return fail(nullptr, B200_ERR_INVALID, "synchronize: NULL context");
    CK(ctx, cudaMemcpyAsync(ctx->host_err, ctx->dev_err, sizeof(unsigned), cudaMemcpyDeviceToHost, ctx->stream));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    const unsigned bits = *ctx->host_err;
    if (bits) {
        CK(ctx, cudaMemsetAsync(ctx->dev_err, 0, sizeof(unsigned), ctx->stream));
        CK(ctx, cudaStreamSynchronize(ctx->stream));
        if (bits & B200_DEVERR_TIMEOUT) return fail(ctx, B200_ERR_TIMEOUT, "a bounded device wait gave up");
        if (bits & B200_DEVERR_EXPERT) return fail(ctx, B200_ERR_RANGE, "mul_mat_id: an expert id is outside [0, E)");
        return fail(ctx, B200_ERR_RANGE, "get_rows: a row id is outside the table");
    }
    return B200_OK;
}

const char * b200_last_error(b200_context * ctx) { return ctx ? ctx->last_error.c_str() : g_error.c_str(); }

b200_status b200_malloc(b200_context * ctx, size_t bytes, void ** dev_out) {
    if (!ctx || !dev_out) return fail(ctx, B200_ERR_INVALID, "malloc: NULL argument");
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaMalloc(dev_out, bytes ? bytes : 1));
    return B200_OK;
}

b200_status b200_free(b200_context * ctx, void * dev) {
    if (!ctx) return fail(ctx, B200_ERR_INVALID, "free: NULL context");
    if (dev) CK(ctx, cudaFree(dev));
    return B200_OK;
}

b200_status b200_memcpy_h2d(b200_context * ctx, void * dev_dst, const void * host_src, size_t bytes) {
    if (!ctx || (bytes && (!dev_dst || !host_src))) return fail(ctx, B200_ERR_INVALID, "memcpy_h2d: NULL argument");
    CK(ctx, cudaMemcpyAsync(dev_dst, host_src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return B200_OK;
}

b200_status b200_memcpy_d2h(b200_context * ctx, void * host_dst, const void * dev_src, size_t bytes) {
    if (!ctx || (bytes && (!dev_src || !host_dst))) return fail(ctx, B200_ERR_INVALID, "memcpy_d2h: NULL argument");
    CK(ctx, cudaMemcpyAsync(host_dst, dev_src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    return B200_OK;
}

size_t b200_weight_nbytes(int type, int64_t ne0, int64_t ne1, int64_t ne2) {
    const int64_t bv = block_values(type), bb = block_bytes(type);
    if (!bb || ne0 <= 0 || ne1 < 0 || ne2 < 0 || ne0 % bv) return 0;
    return (size_t) (ne0 / bv) * (size_t) bb * (size_t) ne1 * (size_t) ne2;
}

b200_status b200_weight_alloc(b200_context * ctx, int type, int64_t ne0, int64_t ne1, int64_t ne2, b200_weight * out) {
    if (!ctx || !out) return fail(ctx, B200_ERR_INVALID, "weight_alloc: NULL argument");
    std::memset(out, 0, sizeof *out);
    if (!known_weight_type(type)) return fail(ctx, B200_ERR_UNSUPPORTED, "weight_alloc: unsupported type");
    const size_t nbytes = b200_weight_nbytes(type, ne0, ne1, ne2);
    if (!nbytes || ne1 <= 0 || ne2 <= 0) return fail(ctx, B200_ERR_INVALID, "weight_alloc: rows are not whole blocks");
    int64_t sz[4] = {0, 0, 0, 0};
    const int nf = field_sizes(type, ne0, ne1 * ne2, sz);
    int64_t off = 0;
    for (int i = 0; i < 4; i++) {
        out->field_off[i] = off;
        if (i < nf) off += align256(sz[i]);
    }
    CK(ctx, cudaSetDevice(ctx->device));
    void * p = nullptr;
    CK(ctx, cudaMalloc(&p, (size_t) off));
    out->type = type;
    out->device = ctx->device;
    out->ne0 = ne0;
    out->ne1 = ne1;
    out->ne2 = ne2;
    out->data = p;
    out->nbytes = nbytes;
    out->dbytes = (size_t) off;
    return B200_OK;
}

b200_status b200_weight_free(b200_context * ctx, b200_weight * w) {
    if (!ctx || !w) return fail(ctx, B200_ERR_INVALID, "weight_free: NULL argument");
    if (w->data) kq_release(ctx, w->data);
    if (w->data) CK(ctx, cudaFree(w->data));
    w->data = nullptr;
    return B200_OK;
}

static const size_t kStagingPiece = (size_t) 64 << 20;

b200_status b200_weight_set(b200_context * ctx, b200_weight * w, const void * host_src, size_t offset, size_t size) {
    if (!ctx || !w || !w->data || (size && !host_src)) return fail(ctx, B200_ERR_INVALID, "weight_set: NULL argument");
    if (offset > w->nbytes || size > w->nbytes - offset) return fail(ctx, B200_ERR_INVALID, "weight_set: range outside the tensor");
    kq_release(ctx, w->data);  // an expanded copy of the old bytes is stale
    if (w->type == B200_TYPE_BF16 || w->type == B200_TYPE_F32) {
        CK(ctx, cudaMemcpyAsync((uint8_t *) w->data + offset, host_src, size, cudaMemcpyHostToDevice, ctx->stream));
        return B200_OK;
    }
    const size_t piece = size < kStagingPiece ? size : kStagingPiece;
    b200_status s = ensure_staging(ctx, piece ? piece : 1);
    if (s != B200_OK) return s;
    for (size_t done = 0; done < size;) {
        const size_t n = size - done < kStagingPiece ? size - done : kStagingPiece;
        CK(ctx, cudaMemcpyAsync(ctx->staging, (const uint8_t *) host_src + done, n, cudaMemcpyHostToDevice, ctx->stream));
        CK(ctx, launch_repack(w->type, w, (const uint8_t *) ctx->staging, (int64_t) (offset + done), (int64_t) n, true, nullptr, ctx->stream));
        ctx->upload_pending = true;
        done += n;
    }
    return B200_OK;
}

b200_status b200_weight_set_device(b200_context * ctx, b200_weight * w, const void * dev_src, size_t offset, size_t size) {
    if (!ctx || !w || !w->data || (size && !dev_src)) return fail(ctx, B200_ERR_INVALID, "weight_set_device: NULL argument");
    if (offset > w->nbytes || size > w->nbytes - offset) return fail(ctx, B200_ERR_INVALID, "weight_set_device: range outside the tensor");
    kq_release(ctx, w->data);  // an expanded copy of the old bytes is stale
    if (w->type == B200_TYPE_BF16 || w->type == B200_TYPE_F32) {
        CK(ctx, cudaMemcpyAsync((uint8_t *) w->data + offset, dev_src, size, cudaMemcpyDeviceToDevice, ctx->stream));
        return B200_OK;
    }
    CK(ctx, launch_repack(w->type, w, (const uint8_t *) dev_src, (int64_t) offset, (int64_t) size, true, nullptr, ctx->stream));
    ctx->upload_pending = true;
    return B200_OK;
}

b200_status b200_weight_get(b200_context * ctx, const b200_weight * w, void * host_dst, size_t offset, size_t size) {
    if (!ctx || !w || !w->data || (size && !host_dst)) return fail(ctx, B200_ERR_INVALID, "weight_get: NULL argument");
    if (offset > w->nbytes || size > w->nbytes - offset) return fail(ctx, B200_ERR_INVALID, "weight_get: range outside the tensor");
    if (w->type == B200_TYPE_BF16 || w->type == B200_TYPE_F32) {
        CK(ctx, cudaMemcpyAsync(host_dst, (const uint8_t *) w->data + offset, size, cudaMemcpyDeviceToHost, ctx->stream));
        CK(ctx, cudaStreamSynchronize(ctx->stream));
        return B200_OK;
    }
    const size_t piece = size < kStagingPiece ? size : kStagingPiece;
    b200_status s = ensure_staging(ctx, piece ? piece : 1);
    if (s != B200_OK) return s;
    for (size_t done = 0; done < size;) {
        const size_t n = size - done < kStagingPiece ? size - done : kStagingPiece;
        CK(ctx, launch_repack(w->type, w, nullptr, (int64_t) (offset + done), (int64_t) n, false, (uint8_t *) ctx->staging, ctx->stream));
        CK(ctx, cudaMemcpyAsync((uint8_t *) host_dst + done, ctx->staging, n, cudaMemcpyDeviceToHost, ctx->stream));
        CK(ctx, cudaStreamSynchronize(ctx->stream));
        done += n;
    }
    return B200_OK;
}

b200_status b200_mul_mat(b200_context * ctx, const b200_weight * w, const float * x, int64_t M, float * dst) {
    if (!check_weight(ctx, w)) return fail(ctx, B200_ERR_INVALID, "mul_mat: bad weight");
    if (w->ne2 != 1) return fail(ctx, B200_ERR_INVALID, "mul_mat: a stack of matrices needs mul_mat_id");
    return mul_mat_impl(ctx, w, 0, w->ne1, x, M, dst, w->ne1);
}

b200_status b200_mul_mat_rows(b200_context * ctx, const b200_weight * w, int64_t row0, int64_t n, const float * x, int64_t M,
                              float * dst, int64_t ld_dst) {
    if (ld_dst < n) return fail(ctx, B200_ERR_INVALID, "mul_mat_rows: ld_dst < n");
    return mul_mat_impl(ctx, w, row0, n, x, M, dst, ld_dst);
}

namespace {

// Pairs from which MUL_MAT_ID of Q8_0 experts runs on the tensor cores (fewer: the grouped GEMV).
constexpr int64_t kMoeTcMinPairs = 128;

// Slot-ordered scratch of the tensor-core expert path, carved in a fixed order.
struct MoeSlots {
    int32_t * grp_off;
    int32_t * col_src;
    int32_t * col_dst;
    int32_t * inv;
    int4 * tiles;
    int * ntiles;
    int64_t max_slots;
    static size_t bytes(int64_t P, int64_t E) {
        auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
        const int64_t S = moe_max_slots(P, E);
        return up((size_t) (E + 1) * 4) + 2 * up((size_t) S * 4) + up((size_t) P * 4) + up((size_t) moe_max_tiles(P, E) * 16) + 256;
    }
    void carve(Carve & c, int64_t P, int64_t E) {
        max_slots = moe_max_slots(P, E);
        grp_off = c.take<int32_t>((size_t) E + 1);
        col_src = c.take<int32_t>((size_t) max_slots);
        col_dst = c.take<int32_t>((size_t) max_slots);
        inv = c.take<int32_t>((size_t) P);
        tiles = c.take<int4>((size_t) moe_max_tiles(P, E));
        ntiles = c.take<int>(1);
    }
};

// The expert FFN on the tensor cores: route into padded slots, quantize x per slot, gate|up grouped GEMM, SwiGLU +
// re-quantization per slot, down grouped GEMM, weighted combine (over NVLink peer memory when `ep` is given). Both
// expert matrices Q8_0 with K % 256 == 0. (Fusing the route with the quantization, and the SwiGLU into the gate|up
// GEMM's epilogue, measured slower on B200: 26.7k against 29.3k tokens/s for config 5 on one GPU, equal on eight.)
b200_status moe_ffn_tc(b200_context * ctx, const b200_weight * gate_up, const b200_weight * down, int64_t expert0, int64_t total,
                       const float * x, const int32_t * ids, const float * w, int64_t top_k, int64_t T, float * out,
                       const b200_ep_group * ep = nullptr) {
    const int64_t H = gate_up->ne0, F2 = gate_up->ne1, E = gate_up->ne2, F = F2 / 2, P = T * top_k;
    const int64_t S = moe_max_slots(P, E);
    auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    const size_t need = MoeSlots::bytes(P, E) + up((size_t) S * H) + up((size_t) (H / 32) * S * 4) + up((size_t) S * F2 * 4) +
                        up((size_t) S * F) + up((size_t) (F / 32) * S * 4) + up((size_t) S * H * 4);
    b200_status s = ensure_scratch(ctx, need);
    if (s != B200_OK) return s;
    Carve c{(uint8_t *) ctx->scratch};
    MoeSlots m;
    m.carve(c, P, E);
    int8_t * q1 = c.take<int8_t>((size_t) S * H);
    float * d1 = c.take<float>((size_t) (H / 32) * S);
    float * gu = c.take<float>((size_t) S * F2);
    int8_t * q2 = c.take<int8_t>((size_t) S * F);
    float * d2 = c.take<float>((size_t) (F / 32) * S);
    float * dn = c.take<float>((size_t) S * H);
    cudaStream_t st = ctx->stream;
    CK(ctx, launch_moe_route(ids, T, top_k, 1, E, expert0, total, m.grp_off, m.col_src, m.col_dst, m.inv, m.tiles, m.ntiles,
                             ctx->dev_err, st));
    CK(ctx, launch_moe_quant_slots(x, H, H, m.col_src, m.grp_off + E, S, q1, d1, S, ctx->num_sms, st));
    cudaError_t e = launch_gemm_tc_grouped(view_of(gate_up), F2, m.tiles, m.ntiles, q1, d1, S, S, nullptr, gu, F2, ctx->dev_err,
                                           ctx->num_sms, st);
    if (e == cudaErrorInvalidValue) return B200_ERR_UNSUPPORTED;  // a tensor map the driver refused: the GEMV path runs
    if (e != cudaSuccess) return cuda_fail(ctx, e, "gemm_tc_grouped");
    CK(ctx, launch_moe_swiglu_slots(gu, F, m.col_src, m.grp_off + E, S, q2, d2, S, ctx->num_sms, st));
    e = launch_gemm_tc_grouped(view_of(down), H, m.tiles, m.ntiles, q2, d2, S, S, nullptr, dn, H, ctx->dev_err, ctx->num_sms, st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "gemm_tc_grouped");
    if (ep) {
        e = launch_moe_combine_allreduce(dn, w, m.inv, T, top_k, H, ep, out, ctx->dev_err, ctx->num_sms, st);
        if (e != cudaSuccess) return e == cudaErrorInvalidValue ? fail(ctx, B200_ERR_INVALID, "moe_ffn_ep: tokens, hidden or out do not fit the group")
                                                                : cuda_fail(ctx, e, "moe_combine_allreduce");
        return B200_OK;
    }
    CK(ctx, launch_moe_combine_slots(dn, w, m.inv, T, top_k, H, out, st));
    return B200_OK;
}

}  // namespace

b200_status b200_mul_mat_id(b200_context * ctx, const b200_weight * experts, const float * b, int64_t nb1, const int32_t * ids,
                            int64_t top_k, int64_t T, float * dst) {
    if (!check_weight(ctx, experts)) return fail(ctx, B200_ERR_INVALID, "mul_mat_id: bad experts");
    if (experts->type == B200_TYPE_F32) return fail(ctx, B200_ERR_UNSUPPORTED, "mul_mat_id: F32 experts are not on this path");
    if (top_k <= 0 || T < 0 || (nb1 != 1 && nb1 != top_k)) return fail(ctx, B200_ERR_INVALID, "mul_mat_id: bad shape");
    if (T == 0) return B200_OK;
    if (!b || !ids || !dst) return fail(ctx, B200_ERR_INVALID, "mul_mat_id: NULL argument");
    const int64_t K = experts->ne0, N = experts->ne1, E = experts->ne2, P = T * top_k;
    // Many pairs of Q8_0 experts: tensor cores over expert-sorted, slot-quantized activations.
    if (P >= kMoeTcMinPairs && gemm_tc_grouped_supported(view_of(experts))) {
        const int64_t S = moe_max_slots(P, E);
        auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
        b200_status s = ensure_scratch(ctx, MoeSlots::bytes(P, E) + up((size_t) S * K) + up((size_t) (K / 32) * S * 4));
        if (s != B200_OK) return s;
        Carve c{(uint8_t *) ctx->scratch};
        MoeSlots m;
        m.carve(c, P, E);
        int8_t * q = c.take<int8_t>((size_t) S * K);
        float * d = c.take<float>((size_t) (K / 32) * S);
        CK(ctx, launch_moe_route(ids, T, top_k, nb1, E, 0, E, m.grp_off, m.col_src, m.col_dst, m.inv, m.tiles, m.ntiles, ctx->dev_err,
                                 ctx->stream));
        CK(ctx, launch_moe_quant_slots(b, K, K, m.col_src, m.grp_off + E, S, q, d, S, ctx->num_sms, ctx->stream));
        const cudaError_t e = launch_gemm_tc_grouped(view_of(experts), N, m.tiles, m.ntiles, q, d, S, S, m.col_dst, dst, N, ctx->dev_err,
                                                     ctx->num_sms, ctx->stream);
        if (e == cudaSuccess) return B200_OK;
        if (e != cudaErrorInvalidValue) return cuda_fail(ctx, e, "gemm_tc_grouped");
        // a tensor map the driver refused: the GEMV path below computes the same product
    }
    const int kind = act_kind(experts->type);
    const int nc = gemv_max_columns(experts->type, K);
    if (nc == 0) return fail(ctx, B200_ERR_UNSUPPORTED, "mul_mat_id: rows too long for the staging buffer");
    size_t need = (((size_t) (E + 1) * 4 + 255) & ~(size_t) 255) + 2 * (((size_t) P * 4 + 255) & ~(size_t) 255);
    if (kind != B200_TYPE_BF16) need += quantized_act_bytes(kind, K, T * nb1);
    b200_status s = ensure_scratch(ctx, need);
    if (s != B200_OK) return s;
    Carve c{(uint8_t *) ctx->scratch};
    int32_t * grp_off = c.take<int32_t>((size_t) E + 1);
    int32_t * col_src = c.take<int32_t>((size_t) P);
    int32_t * col_dst = c.take<int32_t>((size_t) P);
    GemvParams p = base_params(ctx, experts);
    if (kind != B200_TYPE_BF16) {
        int8_t * q = c.take<int8_t>((size_t) T * nb1 * K);
        float * d = c.take<float>((size_t) T * nb1 * (K / (kind == B200_TYPE_Q8_0 ? 32 : 256)));
        int16_t * bs = kind == B200_TYPE_Q8_K ? c.take<int16_t>((size_t) T * nb1 * (K / 16)) : nullptr;
        CK(ctx, launch_quantize(kind, b, K, T * nb1, nullptr, q, d, bs, ctx->stream));
        p.aq = q;
        p.ad = d;
        p.abs = bs;
    }
    CK(ctx, launch_route(ids, T, top_k, nb1, E, grp_off, col_src, col_dst, ctx->dev_err, ctx->stream));
    p.N = N;
    p.row0 = 0;
    p.x = b;
    p.ldx = K;
    p.y = dst;
    p.ldy = N;
    p.col_src = col_src;
    p.col_dst = col_dst;
    p.grp_off = grp_off;
    p.grp_rows = N;
    CK(ctx, launch_gemv(p, nc, (int) E, ctx->stream, false, ctx->num_sms));
    return B200_OK;
}

b200_status b200_moe_ffn(b200_context * ctx, const b200_weight * gate_up, const b200_weight * down, int64_t expert0,
                         int64_t n_expert_total, const float * x, const int32_t * ids, const float * w, int64_t top_k, int64_t T,
                         float * out) {
    if (!check_weight(ctx, gate_up) || !check_weight(ctx, down)) return fail(ctx, B200_ERR_INVALID, "moe_ffn: bad experts");
    const int64_t H = gate_up->ne0, F2 = gate_up->ne1, E = gate_up->ne2, F = F2 / 2;
    if (F2 % 2 || down->ne0 != F || down->ne1 != H || down->ne2 != E || F % 32)
        return fail(ctx, B200_ERR_INVALID, "moe_ffn: gate_up must be [H, 2F, E] and down [F, H, E]");
    const bool kdown = down->type == B200_TYPE_Q4_K || down->type == B200_TYPE_Q5_K || down->type == B200_TYPE_Q6_K;
    if ((down->type != B200_TYPE_Q8_0 && !kdown) || gate_up->type == B200_TYPE_F32 || gate_up->type == B200_TYPE_BF16)
        return fail(ctx, B200_ERR_UNSUPPORTED, "moe_ffn: quantized experts (Q8_0, Q4_K, Q5_K or Q6_K)");
    if (kdown && F % 256)
        return fail(ctx, B200_ERR_INVALID, "moe_ffn: K-quant down experts need whole 256-value super-blocks");
    if (top_k <= 0 || T < 0 || expert0 < 0 || (n_expert_total > 0 && expert0 + E > n_expert_total))
        return fail(ctx, B200_ERR_INVALID, "moe_ffn: bad shape or expert range");
    if (T == 0) return B200_OK;
    if (!x || !ids || !w || !out) return fail(ctx, B200_ERR_INVALID, "moe_ffn: NULL argument");
    const int64_t P = T * top_k, total = n_expert_total > 0 ? n_expert_total : E;
    if (gemm_tc_grouped_supported(view_of(gate_up)) && gemm_tc_grouped_supported(view_of(down)) && F % 256 == 0) {
        b200_status s = moe_ffn_tc(ctx, gate_up, down, expert0, total, x, ids, w, top_k, T, out);
        if (s != B200_ERR_UNSUPPORTED) return s;
    }
    const int kind = act_kind(gate_up->type);
    const int nc1 = gemv_max_columns(gate_up->type, H), nc2 = gemv_max_columns(down->type, F);
    if (!nc1 || !nc2) return fail(ctx, B200_ERR_UNSUPPORTED, "moe_ffn: rows too long for the staging buffer");
    auto up = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    const int kind2 = act_kind(down->type);  // q8_0 for Q8_0 down experts, q8_K for K-quants
    const size_t need = up((size_t) (E + 1) * 4) + 3 * up((size_t) P * 4) + quantized_act_bytes(kind, H, T) + up((size_t) P * F2 * 4) +
                        quantized_act_bytes(kind2, F, P) + up((size_t) P * H * 4);
    b200_status s = ensure_scratch(ctx, need);
    if (s != B200_OK) return s;
    Carve c{(uint8_t *) ctx->scratch};
    int32_t * grp_off = c.take<int32_t>((size_t) E + 1);
    int32_t * col_src = c.take<int32_t>((size_t) P);
    int32_t * col_dst = c.take<int32_t>((size_t) P);
    int32_t * col_tok = c.take<int32_t>((size_t) P);
    int8_t * xq = c.take<int8_t>((size_t) T * H);
    float * xd = c.take<float>((size_t) T * (H / (kind == B200_TYPE_Q8_0 ? 32 : 256)));
    int16_t * xbs = kind == B200_TYPE_Q8_K ? c.take<int16_t>((size_t) T * (H / 16)) : nullptr;
    float * gu = c.take<float>((size_t) P * F2);
    int8_t * aq = c.take<int8_t>((size_t) P * F);
    float * ad = c.take<float>((size_t) P * (F / (kdown ? 256 : 32)));
    int16_t * abs = kdown ? c.take<int16_t>((size_t) P * (F / 16)) : nullptr;
    float * dn = c.take<float>((size_t) P * H);
    cudaStream_t st = ctx->stream;
    CK(ctx, launch_quantize(kind, x, H, T, nullptr, xq, xd, xbs, st));
    CK(ctx, launch_route(ids, T, top_k, top_k, E, grp_off, col_src, col_dst, ctx->dev_err, st, expert0, total, col_tok));
    // gate|up of every routed pair: rows p of gu
    GemvParams p1 = base_params(ctx, gate_up);
    p1.N = F2;
    p1.x = x;
    p1.ldx = H;
    p1.aq = xq;
    p1.ad = xd;
    p1.abs = xbs;
    p1.y = gu;
    p1.ldy = F2;
    p1.col_src = col_tok;
    p1.col_dst = col_dst;
    p1.grp_off = grp_off;
    p1.grp_rows = F2;
    CK(ctx, launch_gemv(p1, nc1, (int) E, st, false, ctx->num_sms));
    if (kdown) CK(ctx, launch_swiglu_quant_pairs_k(gu, F, col_dst, grp_off + E, P, aq, ad, abs, st));
    else CK(ctx, launch_swiglu_quant_pairs(gu, F, col_dst, grp_off + E, P, aq, ad, st));
    // down of every routed pair: rows p of dn
    GemvParams p2 = base_params(ctx, down);
    p2.N = H;
    p2.x = nullptr;
    p2.ldx = F;
    p2.aq = aq;
    p2.ad = ad;
    p2.abs = abs;
    p2.y = dn;
    p2.ldy = H;
    p2.col_src = col_dst;
    p2.col_dst = col_dst;
    p2.grp_off = grp_off;
    p2.grp_rows = H;
    CK(ctx, launch_gemv(p2, nc2, (int) E, st, false, ctx->num_sms));
    CK(ctx, launch_moe_combine(dn, w, ids, T, top_k, H, expert0, E, out, st));
    return B200_OK;
}

b200_status b200_moe_ffn_ep(b200_context * ctx, const b200_weight * gate_up, const b200_weight * down, int64_t expert0,
                            int64_t n_expert_total, const float * x, const int32_t * ids, const float * w, int64_t top_k, int64_t T,
                            float * out, b200_ep_group * group) {
    if (!group) return fail(ctx, B200_ERR_INVALID, "moe_ffn_ep: NULL group");
    if (!check_weight(ctx, gate_up) || !check_weight(ctx, down)) return fail(ctx, B200_ERR_INVALID, "moe_ffn_ep: bad experts");
    const int64_t H = gate_up->ne0, F2 = gate_up->ne1, E = gate_up->ne2, F = F2 / 2;
    if (F2 % 2 || down->ne0 != F || down->ne1 != H || down->ne2 != E)
        return fail(ctx, B200_ERR_INVALID, "moe_ffn_ep: gate_up must be [H, 2F, E] and down [F, H, E]");
    if (top_k <= 0 || T < 0 || expert0 < 0 || n_expert_total <= 0 || expert0 + E > n_expert_total || !x || !ids || !w || !out)
        return fail(ctx, B200_ERR_INVALID, "moe_ffn_ep: bad shape, expert range or NULL argument");
    if (!(gemm_tc_grouped_supported(view_of(gate_up)) && gemm_tc_grouped_supported(view_of(down)) && F % 256 == 0))
        return fail(ctx, B200_ERR_UNSUPPORTED, "moe_ffn_ep: Q8_0 experts with rows of whole 256-value groups");
    if (T == 0) return B200_OK;
    return moe_ffn_tc(ctx, gate_up, down, expert0, n_expert_total, x, ids, w, top_k, T, out, group);
}

b200_status b200_weight_prefetch_l2(b200_context * ctx, const b200_weight * w, void * stream) {
    if (!check_weight(ctx, w)) return fail(ctx, B200_ERR_INVALID, "weight_prefetch_l2: bad weight");
    const int64_t base = (int64_t) (((uintptr_t) w->data + 15) & ~(uintptr_t) 15) - (int64_t) (uintptr_t) w->data;
    if ((size_t) base >= w->dbytes) return B200_OK;
    CK(ctx, launch_prefetch_l2((const uint8_t *) w->data + base, w->dbytes - (size_t) base, stream ? (cudaStream_t) stream : ctx->stream));
    return B200_OK;
}

b200_status b200_get_rows(b200_context * ctx, const b200_weight * table, const int32_t * ids, int64_t n, float * dst) {
    if (!check_weight(ctx, table)) return fail(ctx, B200_ERR_INVALID, "get_rows: bad table");
    if (n < 0 || (n > 0 && (!ids || !dst))) return fail(ctx, B200_ERR_INVALID, "get_rows: bad arguments");
    CK(ctx, launch_get_rows(view_of(table), ids, n, dst, ctx->dev_err, ctx->stream));
    return B200_OK;
}

b200_status b200_quantize_rows(b200_context * ctx, int type, const float * x, int64_t K, int64_t M, void * dst) {
    if (!ctx || (M > 0 && (!x || !dst)) || M < 0) return fail(ctx, B200_ERR_INVALID, "quantize_rows: bad arguments");
    if (type != B200_TYPE_Q8_0 && type != B200_TYPE_Q8_K) return fail(ctx, B200_ERR_UNSUPPORTED, "quantize_rows: type must be Q8_0 or Q8_K");
    if (K <= 0 || K % block_values(type)) return fail(ctx, B200_ERR_INVALID, "quantize_rows: K is not whole blocks");
    CK(ctx, launch_quantize(type, x, K, M, (uint8_t *) dst, nullptr, nullptr, nullptr, ctx->stream));
    return B200_OK;
}

b200_status b200_block_sums(b200_context * ctx, const b200_weight * w, const float * x, int32_t * sums) {
    if (!check_weight(ctx, w) || !x || !sums) return fail(ctx, B200_ERR_INVALID, "block_sums: bad arguments");
    if (w->type != B200_TYPE_Q8_0 && w->type != B200_TYPE_Q4_K && w->type != B200_TYPE_Q5_K && w->type != B200_TYPE_Q6_K)
        return fail(ctx, B200_ERR_UNSUPPORTED, "block_sums: integer types only");
    GemvParams p = base_params(ctx, w);
    p.N = w->ne1 * w->ne2;
    p.x = x;
    p.ldx = w->ne0;
    p.sums = sums;
    p.ncols = 1;
    CK(ctx, launch_gemv(p, 1, 1, ctx->stream, false, ctx->num_sms));
    return B200_OK;
}

b200_status b200_mul_mat_host(b200_context * ctx, const b200_weight * w, const float * x_host, int64_t M, float * dst_host) {
    if (!check_weight(ctx, w) || (M > 0 && (!x_host || !dst_host))) return fail(ctx, B200_ERR_INVALID, "mul_mat_host: bad arguments");
    if (M == 0) return B200_OK;
    const size_t xb = (size_t) M * w->ne0 * 4, yb = (size_t) M * w->ne1 * 4;
    const size_t need = ((xb + 255) & ~(size_t) 255) + ((yb + 255) & ~(size_t) 255);
    b200_status s = ensure_staging(ctx, need);
    if (s != B200_OK) return s;
    float * dx = (float *) ctx->staging;
    float * dy = (float *) ((uint8_t *) ctx->staging + ((xb + 255) & ~(size_t) 255));
    CK(ctx, cudaMemcpyAsync(dx, x_host, xb, cudaMemcpyHostToDevice, ctx->stream));
    s = b200_mul_mat(ctx, w, dx, M, dy);
    if (s != B200_OK) return s;
    CK(ctx, cudaMemcpyAsync(dst_host, dy, yb, cudaMemcpyDeviceToHost, ctx->stream));
    return b200_synchronize(ctx);
}

}  // extern "C"
