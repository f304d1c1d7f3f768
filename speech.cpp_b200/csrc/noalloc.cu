// noalloc.cu — MUL_MAT_ID for callers that cannot allocate device memory (b200_mul_mat_id_noalloc).
//
// Some callers of these products must not call cudaMalloc: a serving runtime that owns all device memory through
// its own arena and forbids allocations outside it; a latency-critical path where cudaMalloc / cudaFree could
// synchronize the device and stall the other streams; a process that already fills the GPU with weights, where a
// late allocation would fail mid-request. The regular b200_mul_mat_id takes its scratch (routing tables and the
// quantized activation rows) from the context's pool, which grows with cudaMalloc. This variant runs the same
// kernels with that scratch in one file-scope device array instead, so it allocates nothing.
//
// The array is B200_NOALLOC_SCRATCH_BYTES (16 MiB); every GPU that loads this library holds it until the process
// exits. In host code `g_noalloc_scratch` names a host-side stand-in, not device memory, so its device address is
// fetched once per device with cudaGetSymbolAddress (with that device current) and passed to the kernels. All calls
// on a device share the one array and it keeps the last call's contents: each call rewrites everything it reads
// (the error word is cleared, the routing tables and quantized rows are written before they are read), and calls that
// overlap on the GPU — on two streams at once — race on it.
#include <mutex>

#include "internal.h"

using namespace b200;

namespace {

constexpr size_t kScratchBytes = (size_t) B200_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

struct DeviceScratch {
    uint8_t * base = nullptr;  // device address of g_noalloc_scratch on this device
    int sms = 0;
    bool ready = false;
};

std::mutex g_mutex;
DeviceScratch g_devices[kMaxDevices];

// Once per device, with that device current: the array's device address and the SM count.
b200_status device_scratch(int device, DeviceScratch ** out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (device < 0 || device >= kMaxDevices) return B200_ERR_INVALID;
    DeviceScratch & d = g_devices[device];
    if (!d.ready) {
        void * p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            set_thread_error("mul_mat_id_noalloc: cudaGetSymbolAddress of the static scratch failed");
            return B200_ERR_DEVICE;
        }
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess || sms <= 0) {
            set_thread_error("mul_mat_id_noalloc: cannot read the SM count");
            return B200_ERR_DEVICE;
        }
        d.base = (uint8_t *) p;
        d.sms = sms;
        d.ready = true;
    }
    *out = &d;
    return B200_OK;
}

size_t up256(size_t v) { return (v + 255) & ~(size_t) 255; }

b200_status bad(const char * what) {
    set_thread_error(what);
    return B200_ERR_INVALID;
}

}  // namespace

extern "C" b200_status b200_mul_mat_id_noalloc(void * stream, const b200_weight * experts, const float * b, int64_t nb1,
                                               const int32_t * ids, int64_t top_k, int64_t T, float * dst) {
    if (!experts || !experts->data || experts->ne0 <= 0 || experts->ne1 <= 0 || experts->ne2 <= 0)
        return bad("mul_mat_id_noalloc: bad experts");
    const int t = experts->type;
    if (t != B200_TYPE_Q8_0 && t != B200_TYPE_Q4_K && t != B200_TYPE_Q5_K && t != B200_TYPE_Q6_K && t != B200_TYPE_BF16) {
        set_thread_error("mul_mat_id_noalloc: unsupported expert type");
        return B200_ERR_UNSUPPORTED;
    }
    const int64_t K = experts->ne0, N = experts->ne1, E = experts->ne2;
    if (K % (t == B200_TYPE_Q8_0 ? 32 : t == B200_TYPE_BF16 ? 8 : 256)) return bad("mul_mat_id_noalloc: rows are not whole blocks");
    if (top_k <= 0 || T < 0 || (nb1 != 1 && nb1 != top_k)) return bad("mul_mat_id_noalloc: bad shape");
    if (T == 0) return B200_OK;
    if (!b || !ids || !dst) return bad("mul_mat_id_noalloc: NULL argument");
    if (E > 4096) return bad("mul_mat_id_noalloc: more than 4096 experts");

    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device != experts->device)
        return bad("mul_mat_id_noalloc: the current device is not the experts' device");
    DeviceScratch * ds = nullptr;
    b200_status s = device_scratch(device, &ds);
    if (s != B200_OK) return s;

    // scratch plan: error word | grp_off [E+1] | col_src [P] | col_dst [P] | quantized rows (q, d, bs)
    const int kind = act_kind(t);
    const int64_t P = T * top_k, R = T * nb1;
    size_t need = 256 + up256((size_t) (E + 1) * 4) + 2 * up256((size_t) P * 4);
    size_t q_off = need, d_off = 0, bs_off = 0;
    if (kind != B200_TYPE_BF16) {
        need += up256((size_t) R * K);
        d_off = need;
        need += up256((size_t) R * (K / (kind == B200_TYPE_Q8_0 ? 32 : 256)) * 4);
        bs_off = need;
        if (kind == B200_TYPE_Q8_K) need += up256((size_t) R * (K / 16) * 2);
    }
    if (need > kScratchBytes) {
        set_thread_error("mul_mat_id_noalloc: this call needs more than the 16 MiB static scratch "
                         "(T * nb1 * K activation bytes + routing tables); use b200_mul_mat_id");
        return B200_ERR_INVALID;
    }
    const int nc = gemv_max_columns(t, K);
    if (nc == 0) {
        set_thread_error("mul_mat_id_noalloc: rows too long for the staging buffer");
        return B200_ERR_UNSUPPORTED;
    }

    cudaStream_t st = (cudaStream_t) stream;
    uint8_t * base = ds->base;
    unsigned * err = (unsigned *) base;
    int32_t * grp_off = (int32_t *) (base + 256);
    int32_t * col_src = (int32_t *) (base + 256 + up256((size_t) (E + 1) * 4));
    int32_t * col_dst = (int32_t *) ((uint8_t *) col_src + up256((size_t) P * 4));

    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(unsigned), st);
    GemvParams p;
    std::memset(&p, 0, sizeof p);
    p.w = view_of(experts);
    p.err = err;
    if (e == cudaSuccess && kind != B200_TYPE_BF16) {
        int8_t * q = (int8_t *) (base + q_off);
        float * d = (float *) (base + d_off);
        int16_t * bs = kind == B200_TYPE_Q8_K ? (int16_t *) (base + bs_off) : nullptr;
        e = launch_quantize(kind, b, K, R, nullptr, q, d, bs, st);
        p.aq = q;
        p.ad = d;
        p.abs = bs;
    }
    if (e == cudaSuccess) e = launch_route(ids, T, top_k, nb1, E, grp_off, col_src, col_dst, err, st);
    if (e == cudaSuccess) {
        p.N = N;
        p.x = b;
        p.ldx = K;
        p.y = dst;
        p.ldy = N;
        p.col_src = col_src;
        p.col_dst = col_dst;
        p.grp_off = grp_off;
        p.grp_rows = N;
        e = launch_gemv(p, nc, (int) E, st, false, ds->sms);
    }
    if (e != cudaSuccess) {
        set_thread_error(cudaGetErrorString(e));
        return B200_ERR_DEVICE;
    }
    return B200_OK;
}
