// decoder.cu — the matmul stack of one Qwen3 decoder step (b200_decoder_*).
//
// Mirrors Qwen3Decoder::layers / outputs (src/common/qwen3-decoder.cpp:350-413, 422-438) for one token: per layer
//   h = rms_norm(x) * attn_norm;  q, k, v = Wq h, Wk h, Wv h;  o = attention(q, k, v);  x += Wo o;
//   h = rms_norm(x) * ffn_norm;   x += Wdown (silu(Wgate h) * Wup h)
// then logits = Whead (rms_norm(x) * output_norm). Attention is taken at the sequence's first position, where the
// softmax has one term and each query head's output is its key/value head's value row (grouped-query broadcast): the
// q/k norms, RoPE and the KV cache then do not change any output, and are left to the rest of the ggml graph.
//
// B200 design: q|k|v and gate|up are stored as one matrix each (their rows concatenated), so a layer is four
// dependent products. Each product is one GEMV launch whose prologue fuses the glue before it (RMSNorm, SwiGLU, the
// value broadcast) and whose epilogue adds the residual. Launches carry the programmatic-serialization attribute:
// a product's CTAs issue their weight loads before griddepcontrol.wait, overlapping the previous product's tail.
// The whole step is captured once in a CUDA graph and replayed.
#include <cstring>
#include <vector>

#include "internal.h"
#include "decoder_mk.cuh"

using namespace b200;


struct b200_decoder {
    b200_context * ctx = nullptr;
    b200_decoder_shape s{};
    std::vector<b200_weight> qkv, o, gu, down;
    std::vector<float *> attn_norm, ffn_norm;
    b200_weight head{};
    float * out_norm = nullptr;
    float * x_in = nullptr;     // step input (hidden)
    float * h = nullptr;        // residual stream (hidden)
    float * qkv_out = nullptr;  // (n_head + 2 n_kv_head) * head_dim
    float * gu_out = nullptr;   // 2 * ffn
    float * logits = nullptr;   // n_vocab
    float * host_io = nullptr;  // pinned: hidden + n_vocab floats
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool pdl = true;
    int cap = 2;      // CTAs per SM per product (chain mode)
    int mode = -1;    // B200_DEC_MODE_*; -1: persistent when every product fits it, else chain
    int64_t launches = 0;
    MkStage * mk_stages = nullptr;  // device table of the step's products (persistent mode)
    unsigned * mk_epoch = nullptr;     // persistent steps completed (the tags' epoch)
    unsigned * mk_finished = nullptr;  // CTAs that finished the running step
    uint2 * t_h0 = nullptr;   // tagged vectors of the persistent step: residual stream at layer inputs,
    uint2 * t_h1 = nullptr;   // residual stream after attention,
    uint2 * t_qkv = nullptr;  // q|k|v outputs,
    uint2 * t_gu = nullptr;   // gate|up outputs
    int mk_n = 0;
    bool mk_forms = false;  // some product has K-quant weights: the instantiation with their row forms
};

namespace {

b200_status dfail(b200_decoder * d, b200_status s, const char * what) {
    d->ctx->last_error = what;
    return s;
}

#define DCK(d, call)                                                                              \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) {                                                                  \
            d->ctx->last_error = std::string(#call) + ": " + cudaGetErrorString(e_);              \
            return e_ == cudaErrorMemoryAllocation ? B200_ERR_ALLOC : B200_ERR_DEVICE;            \
        }                                                                                         \
    } while (0)

int64_t qkv_rows(const b200_decoder_shape & s) { return (int64_t) (s.n_head + 2 * s.n_kv_head) * s.head_dim; }

GemvParams stage(const b200_decoder * d, const b200_weight & w, const float * x, float * y) {
    GemvParams p;
    std::memset(&p, 0, sizeof p);
    p.err = d->ctx->dev_err;
    p.w = view_of(&w);
    p.N = w.ne1;
    p.x = x;
    p.ldx = w.ne0;
    p.y = y;
    p.ldy = w.ne1;
    p.ncols = 1;
    return p;
}

// The step's products in chain order, as GemvParams (both modes are built from this one list).
std::vector<GemvParams> step_products(b200_decoder * d) {
    const b200_decoder_shape & s = d->s;
    std::vector<GemvParams> v;
    for (int l = 0; l < s.n_layer; l++) {
        const float * x = l == 0 ? d->x_in : d->h;
        GemvParams a = stage(d, d->qkv[l], x, d->qkv_out);
        a.pro = PRO_RMSNORM;
        a.norm_w = d->attn_norm[l];
        a.eps = s.eps;
        v.push_back(a);
        GemvParams b = stage(d, d->o[l], d->qkv_out + (int64_t) (s.n_head + s.n_kv_head) * s.head_dim, d->h);
        b.pro = PRO_GQA;
        b.pro_k = s.head_dim;
        b.pro_rep = s.n_head / s.n_kv_head;
        b.res = x;
        v.push_back(b);
        GemvParams c = stage(d, d->gu[l], d->h, d->gu_out);
        c.pro = PRO_RMSNORM;
        c.norm_w = d->ffn_norm[l];
        c.eps = s.eps;
        v.push_back(c);
        GemvParams e = stage(d, d->down[l], d->gu_out, d->h);
        e.pro = PRO_SWIGLU;
        e.pro_k = s.ffn;
        e.res = d->h;
        v.push_back(e);
    }
    GemvParams hd = stage(d, d->head, s.n_layer > 0 ? d->h : d->x_in, d->logits);
    hd.pro = PRO_RMSNORM;
    hd.norm_w = d->out_norm;
    hd.eps = s.eps;
    v.push_back(hd);
    return v;
}

// Whether product p can run in the persistent step (staging layout, slot size, alignment of its input).
bool mk_fits(const GemvParams & p) {
    const int64_t K = p.w.K;
    const int kind = act_kind(p.w.type);
    if (K > kMkMaxK || (kind == B200_TYPE_Q8_K ? K % 2048 : K % 1024) != 0) return false;
    if (p.pro == PRO_GQA && (p.pro_k % 4 != 0 || p.pro_rep <= 0)) return false;
    if (p.pro == PRO_SWIGLU && p.pro_k % 4 != 0) return false;
    if ((((uintptr_t) p.x) & 15) != 0) return false;
    switch (p.w.type) {
    case B200_TYPE_Q8_0: return mk_type_fits<TQ8_0>(K);
    case B200_TYPE_Q4_K: return mk_type_fits<TQ4_K>(K);
    case B200_TYPE_Q6_K: return mk_type_fits<TQ6_K>(K);
    case B200_TYPE_BF16: return mk_type_fits<TBF16>(K);
    default: return false;
    }
}

b200_status prepare_mk(b200_decoder * d, const std::vector<GemvParams> & v) {
    if (d->mk_stages) return B200_OK;
    const b200_decoder_shape & sh = d->s;
    DCK(d, cudaMalloc(&d->t_h0, sizeof(uint2) * (size_t) sh.hidden));
    DCK(d, cudaMalloc(&d->t_h1, sizeof(uint2) * (size_t) sh.hidden));
    DCK(d, cudaMalloc(&d->t_qkv, sizeof(uint2) * (size_t) qkv_rows(sh)));
    DCK(d, cudaMalloc(&d->t_gu, sizeof(uint2) * 2 * (size_t) sh.ffn));
    DCK(d, cudaMalloc(&d->mk_epoch, 2 * sizeof(unsigned)));
    d->mk_finished = d->mk_epoch + 1;
    // Tags are never zero-based stale matches: epoch starts at 1 and the tagged vectors start with tag 0.
    DCK(d, cudaMemset(d->t_h0, 0, sizeof(uint2) * (size_t) sh.hidden));
    DCK(d, cudaMemset(d->t_h1, 0, sizeof(uint2) * (size_t) sh.hidden));
    DCK(d, cudaMemset(d->t_qkv, 0, sizeof(uint2) * (size_t) qkv_rows(sh)));
    DCK(d, cudaMemset(d->t_gu, 0, sizeof(uint2) * 2 * (size_t) sh.ffn));
    const unsigned init[2] = {1u, 0u};
    DCK(d, cudaMemcpy(d->mk_epoch, init, sizeof init, cudaMemcpyHostToDevice));
    // Vectors between products, tagged. Per layer: A q|k|v (x: h0) -> qkv; B o (x: the v part of qkv, res h0) -> h1;
    // C gate|up (x: h1) -> gu, the F values silu(gate) * up (each CTA streams the gate and up rows of its own features
    // and forms their SwiGLU once); D down (x: gu, res h1) -> h0. A CTA can be one product ahead of the slowest, so no
    // product writes a vector that the product before it reads: h1 (written by B) is not read by A, and h0 (written
    // by D) is read by A and B only, which every CTA has finished before any CTA can start D (D's input gu needs
    // every CTA's C). Layer 0 reads the step input, and the head writes the logits, untagged.
    const int64_t v_off = (int64_t) (sh.n_head + sh.n_kv_head) * sh.head_dim;
    const float * h0 = reinterpret_cast<const float *>(d->t_h0);
    std::vector<MkStage> st(v.size());
    for (size_t i = 0; i < v.size(); i++) {
        const GemvParams & p = v[i];
        MkStage & m = st[i];
        std::memset(&m, 0, sizeof m);
        m.w = p.w;
        m.N = p.N;
        m.pro = p.pro;
        m.pro_k = (int) p.pro_k;
        m.pro_rep = p.pro_rep;
        m.eps = p.eps;
        m.norm_w = p.norm_w;
        const bool head = i + 1 == v.size();
        const int l = (int) (i / 4), role = (int) (i % 4);
        if (head) {
            m.x = sh.n_layer > 0 ? h0 : d->x_in;
            m.x_tagged = sh.n_layer > 0;
            m.y = d->logits;
        } else if (role == 0) {
            m.x = l == 0 ? d->x_in : h0;
            m.x_tagged = l > 0;
            m.y = reinterpret_cast<float *>(d->t_qkv);
            m.y_tagged = 1;
        } else if (role == 1) {
            m.x = reinterpret_cast<const float *>(d->t_qkv) + 2 * v_off;
            m.x_tagged = 1;
            m.res = l == 0 ? d->x_in : h0;
            m.res_tagged = l > 0;
            m.y = reinterpret_cast<float *>(d->t_h1);
            m.y_tagged = 1;
        } else if (role == 2) {
            m.x = reinterpret_cast<const float *>(d->t_h1);
            m.x_tagged = 1;
            m.y = reinterpret_cast<float *>(d->t_gu);
            m.y_tagged = 1;
            m.glu = 1;
        } else {
            m.x = reinterpret_cast<const float *>(d->t_gu);
            m.x_tagged = 1;
            m.pro = PRO_COPY;  // the SwiGLU was formed by the gate|up product
            m.pro_k = 0;
            m.res = reinterpret_cast<const float *>(d->t_h1);
            m.res_tagged = 1;
            m.y = reinterpret_cast<float *>(d->t_h0);
            m.y_tagged = 1;
        }
        if ((((uintptr_t) m.x) & 15) != 0) return dfail(d, B200_ERR_UNSUPPORTED, "decoder: persistent step input not 16-byte aligned");
        m.row_bytes = (int) mk_row_bytes(p.w.type, p.w.K);
        m.rps = kMkSlotBytes / m.row_bytes / (m.glu ? 2 : 1);  // a gate|up chunk holds its features' gate and up rows
        const int64_t units = m.glu ? p.N / 2 : p.N;         // the rows, or the features, the CTAs split
        m.slice_base = (int) (units / d->ctx->num_sms);
        m.slice_extra = (int) (units % d->ctx->num_sms);
        auto log2_exact = [](int64_t v) { int s = 0; while ((1ll << s) < v) s++; return (v > 0 && (1ll << s) == v) ? s : -1; };
        m.gqa_shift = p.pro == PRO_GQA ? log2_exact(p.pro_k * p.pro_rep) : -1;
        m.hd_shift = p.pro == PRO_GQA ? log2_exact(p.pro_k) : -1;
    }
    DCK(d, cudaMalloc(&d->mk_stages, sizeof(MkStage) * st.size()));
    DCK(d, cudaMemcpy(d->mk_stages, st.data(), sizeof(MkStage) * st.size(), cudaMemcpyHostToDevice));
    d->mk_n = (int) st.size();
    d->mk_forms = false;
    for (const GemvParams & p : v) d->mk_forms |= p.w.type == B200_TYPE_Q4_K || p.w.type == B200_TYPE_Q6_K;
    auto kern = d->mk_forms ? decoder_mk_kernel<true> : decoder_mk_kernel<false>;
    DCK(d, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kMkSmemBytes));
    return B200_OK;
}

b200_status enqueue_mk(b200_decoder * d) {
    cudaStream_t st = d->ctx->stream;
    MkParams P;
    P.stages = d->mk_stages;
    P.nstages = d->mk_n;
    P.epoch = d->mk_epoch;
    P.finished = d->mk_finished;
    P.err = d->ctx->dev_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) d->ctx->num_sms, 1, 1);
    cfg.blockDim = dim3(kMkThreads, 1, 1);
    cfg.dynamicSmemBytes = kMkSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    DCK(d, cudaLaunchKernelEx(&cfg, d->mk_forms ? decoder_mk_kernel<true> : decoder_mk_kernel<false>, P));
    d->launches = 1;
    return B200_OK;
}

// Enqueues the step's products on the context stream.
b200_status enqueue_step(b200_decoder * d) {
    std::vector<GemvParams> prods = step_products(d);
    bool persistent = d->mode == B200_DEC_MODE_PERSISTENT;
    // the gate|up products keep their features' sums in shared memory: at most kMkResRows features per CTA
    const bool glu_fits = (d->s.ffn + d->ctx->num_sms - 1) / d->ctx->num_sms <= kMkResRows;
    if (d->mode < 0) {
        persistent = glu_fits;
        for (const GemvParams & p : prods) persistent = persistent && mk_fits(p);
    }
    if (persistent) {
        for (const GemvParams & p : prods)
            if (!mk_fits(p) || !glu_fits) return dfail(d, B200_ERR_UNSUPPORTED, "decoder: a product does not fit the persistent step");
        b200_status s = prepare_mk(d, prods);
        if (s != B200_OK) return s;
        return enqueue_mk(d);
    }
    cudaStream_t st0 = d->ctx->stream;
    d->launches = 0;
    for (const GemvParams & p : prods) {
        DCK(d, launch_gemv(p, 1, 1, st0, d->pdl, d->ctx->num_sms, d->cap));
        d->launches++;
    }
    return B200_OK;
}

b200_status alloc_weight(b200_decoder * d, int type, int64_t ne0, int64_t ne1, b200_weight * w) {
    return b200_weight_alloc(d->ctx, type, ne0, ne1, 1, w);
}

}  // namespace

extern "C" {

b200_status b200_decoder_create(b200_context * ctx, const b200_decoder_shape * shape, b200_decoder ** out) {
    if (!ctx || !shape || !out) return B200_ERR_INVALID;
    *out = nullptr;
    const b200_decoder_shape & s = *shape;
    if (s.n_layer < 0 || s.hidden <= 0 || s.n_head <= 0 || s.n_kv_head <= 0 || s.n_head % s.n_kv_head || s.head_dim <= 0 ||
        s.ffn <= 0 || s.n_vocab <= 0) {
        ctx->last_error = "decoder_create: bad shape";
        return B200_ERR_INVALID;
    }
    b200_decoder * d = new b200_decoder();
    d->ctx = ctx;
    d->s = s;
    b200_status st = B200_OK;
    const int64_t attn = (int64_t) s.n_head * s.head_dim;
    d->qkv.resize(s.n_layer);
    d->o.resize(s.n_layer);
    d->gu.resize(s.n_layer);
    d->down.resize(s.n_layer);
    d->attn_norm.assign(s.n_layer, nullptr);
    d->ffn_norm.assign(s.n_layer, nullptr);
    for (int l = 0; l < s.n_layer && st == B200_OK; l++) {
        st = alloc_weight(d, s.type_attn, s.hidden, qkv_rows(s), &d->qkv[l]);
        if (st == B200_OK) st = alloc_weight(d, s.type_attn, attn, s.hidden, &d->o[l]);
        if (st == B200_OK) st = alloc_weight(d, s.type_ffn_up, s.hidden, 2 * (int64_t) s.ffn, &d->gu[l]);
        if (st == B200_OK) st = alloc_weight(d, s.type_ffn_down, s.ffn, s.hidden, &d->down[l]);
        if (st == B200_OK && cudaMalloc(&d->attn_norm[l], sizeof(float) * s.hidden) != cudaSuccess) st = B200_ERR_ALLOC;
        if (st == B200_OK && cudaMalloc(&d->ffn_norm[l], sizeof(float) * s.hidden) != cudaSuccess) st = B200_ERR_ALLOC;
    }
    if (st == B200_OK) st = alloc_weight(d, s.type_head, s.hidden, s.n_vocab, &d->head);
    if (st == B200_OK) {
        if (cudaMalloc(&d->out_norm, sizeof(float) * s.hidden) != cudaSuccess || cudaMalloc(&d->x_in, sizeof(float) * s.hidden) != cudaSuccess ||
            cudaMalloc(&d->h, sizeof(float) * s.hidden) != cudaSuccess || cudaMalloc(&d->qkv_out, sizeof(float) * qkv_rows(s)) != cudaSuccess ||
            cudaMalloc(&d->gu_out, sizeof(float) * 2 * (size_t) s.ffn) != cudaSuccess ||
            cudaMalloc(&d->logits, sizeof(float) * (size_t) s.n_vocab) != cudaSuccess ||
            cudaMallocHost(&d->host_io, sizeof(float) * ((size_t) s.hidden + (size_t) s.n_vocab)) != cudaSuccess)
            st = B200_ERR_ALLOC;
    }
    if (st != B200_OK) {
        b200_decoder_destroy(d);
        ctx->last_error = "decoder_create: device memory";
        return st;
    }
    *out = d;
    return B200_OK;
}

void b200_decoder_destroy(b200_decoder * d) {
    if (!d) return;
    cudaStreamSynchronize(d->ctx->stream);
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    for (auto * v : {&d->qkv, &d->o, &d->gu, &d->down})
        for (auto & w : *v)
            if (w.data) cudaFree(w.data);
    for (float * p : d->attn_norm) if (p) cudaFree(p);
    for (float * p : d->ffn_norm) if (p) cudaFree(p);
    if (d->head.data) cudaFree(d->head.data);
    for (float * p : {d->out_norm, d->x_in, d->h, d->qkv_out, d->gu_out, d->logits}) if (p) cudaFree(p);
    if (d->mk_stages) cudaFree(d->mk_stages);
    if (d->mk_epoch) cudaFree(d->mk_epoch);
    if (d->t_h0) cudaFree(d->t_h0);
    if (d->t_h1) cudaFree(d->t_h1);
    if (d->t_qkv) cudaFree(d->t_qkv);
    if (d->t_gu) cudaFree(d->t_gu);
    if (d->host_io) cudaFreeHost(d->host_io);
    delete d;
}

b200_status b200_decoder_set_tensor(b200_decoder * d, int layer, int which, const void * data, int on_device, size_t offset,
                                    size_t size) {
    if (!d || !data) return B200_ERR_INVALID;
    const b200_decoder_shape & s = d->s;
    const bool per_layer = which != B200_DEC_OUTPUT_NORM && which != B200_DEC_OUTPUT;
    if (per_layer && (layer < 0 || layer >= s.n_layer)) return dfail(d, B200_ERR_INVALID, "decoder_set_tensor: no such layer");
    float * vec = nullptr;
    b200_weight * w = nullptr;
    int64_t row_off = 0, rows = 0;
    switch (which) {
    case B200_DEC_ATTN_Q: w = &d->qkv[layer]; row_off = 0; rows = (int64_t) s.n_head * s.head_dim; break;
    case B200_DEC_ATTN_K: w = &d->qkv[layer]; row_off = (int64_t) s.n_head * s.head_dim; rows = (int64_t) s.n_kv_head * s.head_dim; break;
    case B200_DEC_ATTN_V: w = &d->qkv[layer]; row_off = (int64_t) (s.n_head + s.n_kv_head) * s.head_dim; rows = (int64_t) s.n_kv_head * s.head_dim; break;
    case B200_DEC_ATTN_O: w = &d->o[layer]; rows = s.hidden; break;
    case B200_DEC_FFN_GATE: w = &d->gu[layer]; row_off = 0; rows = s.ffn; break;
    case B200_DEC_FFN_UP: w = &d->gu[layer]; row_off = s.ffn; rows = s.ffn; break;
    case B200_DEC_FFN_DOWN: w = &d->down[layer]; rows = s.hidden; break;
    case B200_DEC_OUTPUT: w = &d->head; rows = s.n_vocab; break;
    case B200_DEC_ATTN_NORM: vec = d->attn_norm[layer]; break;
    case B200_DEC_FFN_NORM: vec = d->ffn_norm[layer]; break;
    case B200_DEC_OUTPUT_NORM: vec = d->out_norm; break;
    default: return dfail(d, B200_ERR_INVALID, "decoder_set_tensor: no such tensor");
    }
    if (vec) {
        if (offset + size > sizeof(float) * (size_t) s.hidden) return dfail(d, B200_ERR_INVALID, "decoder_set_tensor: range");
        DCK(d, cudaMemcpyAsync((uint8_t *) vec + offset, data, size, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                               d->ctx->stream));
        return B200_OK;
    }
    const size_t row_bytes = b200_weight_nbytes(w->type, w->ne0, 1, 1);
    if (offset + size > row_bytes * (size_t) rows) return dfail(d, B200_ERR_INVALID, "decoder_set_tensor: range");
    const size_t at = row_bytes * (size_t) row_off + offset;
    return on_device ? b200_weight_set_device(d->ctx, w, data, at, size) : b200_weight_set(d->ctx, w, data, at, size);
}

b200_status b200_decoder_step(b200_decoder * d, const float * x, float * logits) {
    if (!d || !x) return B200_ERR_INVALID;
    cudaStream_t st = d->ctx->stream;
    DCK(d, cudaMemcpyAsync(d->x_in, x, sizeof(float) * d->s.hidden, cudaMemcpyDeviceToDevice, st));
    if (!d->exec) {
        // warm the launchers (kernel attributes, occupancy) outside the capture, then capture the step once
        b200_status s0 = enqueue_step(d);
        if (s0 != B200_OK) return s0;
        DCK(d, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        b200_status s1 = enqueue_step(d);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(st, &g);
        if (s1 != B200_OK) return s1;
        if (e != cudaSuccess) return dfail(d, B200_ERR_DEVICE, "decoder_step: graph capture failed");
        d->graph = g;
        DCK(d, cudaGraphInstantiate(&d->exec, g, 0));
    }
    DCK(d, cudaGraphLaunch(d->exec, st));
    if (logits) DCK(d, cudaMemcpyAsync(logits, d->logits, sizeof(float) * (size_t) d->s.n_vocab, cudaMemcpyDeviceToDevice, st));
    return B200_OK;
}

b200_status b200_decoder_step_host(b200_decoder * d, const float * x_host, float * logits_host) {
    if (!d || !x_host || !logits_host) return B200_ERR_INVALID;
    cudaStream_t st = d->ctx->stream;
    float * hx = d->host_io;
    float * hl = d->host_io + d->s.hidden;
    std::memcpy(hx, x_host, sizeof(float) * d->s.hidden);
    DCK(d, cudaMemcpyAsync(d->x_in, hx, sizeof(float) * d->s.hidden, cudaMemcpyHostToDevice, st));
    if (!d->exec) {
        b200_status s0 = b200_decoder_step(d, d->x_in, nullptr);
        if (s0 != B200_OK) return s0;
    } else {
        DCK(d, cudaGraphLaunch(d->exec, st));
    }
    DCK(d, cudaMemcpyAsync(hl, d->logits, sizeof(float) * (size_t) d->s.n_vocab, cudaMemcpyDeviceToHost, st));
    DCK(d, cudaStreamSynchronize(st));
    std::memcpy(logits_host, hl, sizeof(float) * (size_t) d->s.n_vocab);
    return B200_OK;
}

int64_t b200_decoder_launches(const b200_decoder * d) { return d ? d->launches : 0; }

size_t b200_decoder_weight_bytes(const b200_decoder * d) {
    if (!d) return 0;
    size_t b = d->head.nbytes;
    for (int l = 0; l < d->s.n_layer; l++) b += d->qkv[l].nbytes + d->o[l].nbytes + d->gu[l].nbytes + d->down[l].nbytes;
    return b;
}

b200_status b200_decoder_set_launch(b200_decoder * d, int mode, int pdl, int ctas_per_sm) {
    if (!d || ctas_per_sm < 0 || mode < -1 || mode > 1) return B200_ERR_INVALID;
    d->mode = mode;
    d->pdl = pdl != 0;
    d->cap = ctas_per_sm;
    if (d->exec) {
        cudaStreamSynchronize(d->ctx->stream);
        cudaGraphExecDestroy(d->exec);
        cudaGraphDestroy(d->graph);
        d->exec = nullptr;
        d->graph = nullptr;
    }
    return B200_OK;
}

}  // extern "C"
