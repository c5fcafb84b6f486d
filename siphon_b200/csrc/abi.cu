// The extern "C" boundary of libsiphon_cuda (declared in include/siphon_cuda.h).
// Argument checks happen on the host before any CUDA call, so they behave the
// same on a machine without a GPU.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "siphon_cuda.h"
#include "common.cuh"
#include "launch.h"

using namespace sicu;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

struct DevState {
    bool ready = false;
    int sms = 0;
    int smem_optin = 0;
    int smem_per_sm = 0;
    int smem_reserved = 0;
    int *status = nullptr;      // device status word
    // growable staging for the host-buffer entry points
    void *stage = nullptr;
    size_t stage_bytes = 0;
    // growable workspace of the prefill product (token operand, f32 quantization)
    void *pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    // growable f32 activation of sicu_gemv_fused's F16 path (the step's output)
    float *pro_buf = nullptr;
    size_t pro_buf_bytes = 0;
    // growable activation records of the batch matvec
    void *bt_ws = nullptr;
    size_t bt_ws_bytes = 0;
};

constexpr int MAX_DEV = 64;
int g_overlap = 0;   // sicu_set_overlap
DevState g_dev[MAX_DEV];
std::mutex g_mu;

bool geometry(uint32_t t, uint32_t &blck, uint32_t &bytes) {
    switch (t) {
        case T_F32: blck = 1; bytes = 4; return true;
        case T_F16: blck = 1; bytes = 2; return true;
        case T_Q4_0: blck = 32; bytes = B_Q4_0; return true;
        case T_Q5_0: blck = 32; bytes = B_Q5_0; return true;
        case T_Q8_0: blck = 32; bytes = B_Q8_0; return true;
        case T_Q2_K: blck = 256; bytes = B_Q2_K; return true;
        case T_Q3_K: blck = 256; bytes = B_Q3_K; return true;
        case T_Q4_K: blck = 256; bytes = B_Q4_K; return true;
        case T_Q5_K: blck = 256; bytes = B_Q5_K; return true;
        case T_Q6_K: blck = 256; bytes = B_Q6_K; return true;
        case T_Q8_K: blck = 256; bytes = B_Q8_K; return true;
        default: return false;
    }
}

bool pair_of(uint32_t wt, uint32_t &pair) {
    switch (wt) {
        case T_F16: pair = T_F16; return true;
        case T_Q4_0: case T_Q5_0: case T_Q8_0: pair = T_Q8_0; return true;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: pair = T_Q8_K; return true;
        default: return false;
    }
}

const char *tname(uint32_t t) {
    switch (t) {
        case T_F32: return "F32"; case T_F16: return "F16"; case T_Q4_0: return "Q4_0";
        case T_Q5_0: return "Q5_0"; case T_Q8_0: return "Q8_0"; case T_Q2_K: return "Q2_K";
        case T_Q3_K: return "Q3_K"; case T_Q4_K: return "Q4_K"; case T_Q5_K: return "Q5_K";
        case T_Q6_K: return "Q6_K"; case T_Q8_K: return "Q8_K"; default: return "unknown";
    }
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int cuda_fail(cudaError_t e, const char *what) {
    return fail(SICU_EIO, "%s: %s", what, cudaGetErrorString(e));
}

// Current device's state, or an error when sicu_init was not called for it.
bool any_ready();

int current(DevState *&ds) {
    if (!any_ready()) return fail(SICU_EINVAL, "no device initialised (call sicu_init first)");
    int dev = -1;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= MAX_DEV || !g_dev[dev].ready)
        return fail(SICU_EINVAL, "device %d not initialised (call sicu_init first)", dev);
    ds = &g_dev[dev];
    return SICU_OK;
}

int current_ok() {
    DevState *ds;
    return current(ds);
}

bool any_ready() {
    for (auto &d : g_dev) if (d.ready) return true;
    return false;
}

int check_activation(uint32_t pair, const float *dx, const void *dy, int64_t n, int64_t m) {
    uint32_t blck, bytes;
    if (!geometry(pair, blck, bytes)) return fail(SICU_ENOTSUP, "no activation format %u", pair);
    if (n <= 0 || m <= 0) return fail(SICU_EINVAL, "empty activation (n=%lld, m=%lld)", (long long)n, (long long)m);
    if (n % blck) return fail(SICU_EINVAL, "%s activation length %lld is not a multiple of %u", tname(pair), (long long)n, blck);
    if (n > (int64_t)1 << 30) return fail(SICU_EINVAL, "activation length %lld too large", (long long)n);
    if (!dx || !dy) return fail(SICU_EINVAL, "null activation pointer");
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "f32 activation must be 16-byte aligned");
    if (!aligned(dy, pair == T_Q8_K ? 4 : 2)) return fail(SICU_EINVAL, "%s output misaligned", tname(pair));
    return SICU_OK;
}

int check_matvec(uint32_t wt, const void *dw, int64_t n_in, int64_t n_out, const void *dx, const float *dy,
                 int64_t m, uint32_t &pair) {
    if (!pair_of(wt, pair)) return fail(SICU_ENOTSUP, "matvec: unsupported weight type %s (%u)", tname(wt), wt);
    uint32_t blck, bytes;
    geometry(wt, blck, bytes);
    if (n_in <= 0 || n_out < 0 || m <= 0)
        return fail(SICU_EINVAL, "matvec: bad shape n_in=%lld n_out=%lld m=%lld", (long long)n_in, (long long)n_out, (long long)m);
    if (n_in % blck) return fail(SICU_EINVAL, "matvec: row length %lld of %s is not a multiple of %u", (long long)n_in, tname(wt), blck);
    if (n_in > (int64_t)1 << 24) return fail(SICU_EINVAL, "matvec: row length %lld too large", (long long)n_in);
    if (!dx) return fail(SICU_EINVAL, "matvec: null activation");
    if (n_out == 0) return SICU_OK;   // nothing is read or written
    if (!dw || !dy) return fail(SICU_EINVAL, "matvec: null pointer");
    if (!aligned(dw, 16)) return fail(SICU_EINVAL, "matvec: weight pointer must be 16-byte aligned");
    if (!aligned(dy, 4)) return fail(SICU_EINVAL, "matvec: output must be 4-byte aligned");
    return SICU_OK;
}

int64_t pair_row_bytes(uint32_t pair, int64_t n) {
    uint32_t blck, bytes;
    geometry(pair, blck, bytes);
    return n / blck * bytes;
}

GemvLaunch make_launch(const DevState &ds, const void *dw, int64_t n_in, int64_t n_out, float *dy) {
    GemvLaunch L{};
    L.w = dw;
    L.y = dy;
    L.n_out = n_out;
    L.nmat = 1;
    L.wm[0] = dw;
    L.ym[0] = dy;
    L.n_outm[0] = n_out;
    L.n_in = (int)n_in;
    L.num_sms = ds.sms;
    L.smem_limit = ds.smem_optin;
    L.smem_per_sm = ds.smem_per_sm;
    L.smem_reserved = ds.smem_reserved;
    L.overlap = g_overlap;
    int dev = 0;
    cudaGetDevice(&dev);
    L.device = dev;
    L.status = ds.status;
    return L;
}

int run_gemv(uint32_t wt, GemvLaunch &L, cudaStream_t st) {
    const int rc = (wt == T_F16) ? launch_gemv_f16(L, st) : launch_gemv(wt, L, st);
    if (rc == -1) return fail(SICU_ENOTSUP, "matvec: %s row of %d elements does not fit the kernel's shared memory", tname(wt), L.n_in);
    if (rc == -3) return fail(SICU_ENOTSUP, "matvec: no kernel for %s", tname(wt));
    if (rc != 0) return cuda_fail(cudaGetLastError(), "matvec launch");
    return SICU_OK;
}

}  // namespace

namespace sicu {
// Sets the calling thread's error message (read by sicu_last_error) from
// other translation units of the library; returns code.
int report_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}
}  // namespace sicu

extern "C" {

int sicu_init(int device) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (device < 0 || device >= MAX_DEV) return fail(SICU_EINVAL, "device %d out of range", device);
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device >= count) return fail(SICU_EINVAL, "device %d not present (%d devices)", device, count);
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    DevState &ds = g_dev[device];
    if (ds.ready) return SICU_OK;
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(SICU_ENOTSUP, "device %d is sm_%d%d; this library is built for sm_100a only", device, prop.major, prop.minor);
    ds.sms = prop.multiProcessorCount;
    ds.smem_optin = (int)prop.sharedMemPerBlockOptin;
    ds.smem_per_sm = (int)prop.sharedMemPerMultiprocessor;
    ds.smem_reserved = (int)prop.reservedSharedMemPerBlock;
    if ((e = cudaMalloc(&ds.status, sizeof(int))) != cudaSuccess) return cuda_fail(e, "cudaMalloc(status)");
    if ((e = cudaMemset(ds.status, 0, sizeof(int))) != cudaSuccess) return cuda_fail(e, "cudaMemset(status)");
    ds.ready = true;
    return SICU_OK;
}

int sicu_shutdown(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    int cur = -1;
    const bool have = cudaGetDevice(&cur) == cudaSuccess;
    for (int d = 0; d < MAX_DEV; ++d) {
        DevState &ds = g_dev[d];
        if (!ds.ready) continue;
        cudaSetDevice(d);
        cudaFree(ds.status);
        if (ds.stage) cudaFree(ds.stage);
        if (ds.pf_ws) cudaFree(ds.pf_ws);
        if (ds.pro_buf) cudaFree(ds.pro_buf);
        if (ds.bt_ws) cudaFree(ds.bt_ws);
        ds = DevState{};
    }
    if (have && cur >= 0) cudaSetDevice(cur);
    return SICU_OK;
}

int sicu_set_overlap(int on) {
    g_overlap = on ? 1 : 0;
    return SICU_OK;
}

int sicu_last_error(char *buf, size_t len) {
    const size_t n = strlen(g_err);
    if (buf && len) {
        const size_t c = n < len - 1 ? n : len - 1;
        memcpy(buf, g_err, c);
        buf[c] = '\0';
    }
    return (int)n;
}

int sicu_status(int *flags) {
    if (!flags) return fail(SICU_EINVAL, "null flags");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
    if ((e = cudaMemcpy(flags, ds->status, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "read status");
    if ((e = cudaMemset(ds->status, 0, sizeof(int))) != cudaSuccess) return cuda_fail(e, "clear status");
    return SICU_OK;
}

int sicu_malloc(void **dev, size_t bytes) {
    if (!dev) return fail(SICU_EINVAL, "null out pointer");
    if (!any_ready()) return fail(SICU_EINVAL, "no device initialised (call sicu_init first)");
    const cudaError_t e = cudaMalloc(dev, bytes ? bytes : 1);
    if (e != cudaSuccess) return e == cudaErrorMemoryAllocation ? fail(SICU_ENOMEM, "cudaMalloc(%zu) failed", bytes)
                                                                : cuda_fail(e, "cudaMalloc");
    return SICU_OK;
}

int sicu_free(void *dev) {
    if (!dev) return SICU_OK;
    const cudaError_t e = cudaFree(dev);
    return e == cudaSuccess ? SICU_OK : cuda_fail(e, "cudaFree");
}

int sicu_upload(const void *host, size_t bytes, void **dev) {
    if (!host || !dev) return fail(SICU_EINVAL, "upload: null pointer");
    if (int rc = sicu_malloc(dev, bytes)) return rc;
    const cudaError_t e = cudaMemcpy(*dev, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(*dev);
        *dev = nullptr;
        return cuda_fail(e, "upload copy");
    }
    return SICU_OK;
}

int sicu_memcpy_h2d(void *dev, const void *host, size_t bytes, void *stream) {
    if ((!dev || !host) && bytes) return fail(SICU_EINVAL, "memcpy: null pointer");
    const cudaError_t e = cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    return e == cudaSuccess ? SICU_OK : cuda_fail(e, "memcpy h2d");
}

int sicu_memcpy_d2h(void *host, const void *dev, size_t bytes, void *stream) {
    if ((!dev || !host) && bytes) return fail(SICU_EINVAL, "memcpy: null pointer");
    const cudaError_t e = cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    return e == cudaSuccess ? SICU_OK : cuda_fail(e, "memcpy d2h");
}

int sicu_stream_sync(void *stream) {
    const cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    return e == cudaSuccess ? SICU_OK : cuda_fail(e, "stream sync");
}

int sicu_quant_geometry(uint32_t type, uint32_t *blck_size, uint32_t *type_size) {
    if (!blck_size || !type_size) return fail(SICU_EINVAL, "null out pointer");
    uint32_t b, s;
    if (!geometry(type, b, s)) return fail(SICU_ENOTSUP, "unsupported type %u", type);
    *blck_size = b;
    *type_size = s;
    return SICU_OK;
}

int sicu_vec_dot_pair(uint32_t wtype, uint32_t *pair_type) {
    if (!pair_type) return fail(SICU_EINVAL, "null out pointer");
    uint32_t p;
    if (!pair_of(wtype, p)) return fail(SICU_ENOTSUP, "no dot product for type %s (%u)", tname(wtype), wtype);
    *pair_type = p;
    return SICU_OK;
}

static int quantize_common(uint32_t pair, const float *dx, void *dy, int64_t n, int64_t m, void *stream) {
    if (int rc = check_activation(pair, dx, dy, n, m)) return rc;
    DevState *ds;
    if (int rc = current(ds)) return rc;
    const int rc = launch_quantize(pair, dx, dy, n, m, (cudaStream_t)stream);
    if (rc) return cuda_fail(cudaGetLastError(), "quantize launch");
    return SICU_OK;
}

int sicu_quantize_q8_K(const float *dx, void *dy, int64_t n, int64_t m, void *stream) {
    return quantize_common(T_Q8_K, dx, dy, n, m, stream);
}
int sicu_quantize_q8_0(const float *dx, void *dy, int64_t n, int64_t m, void *stream) {
    return quantize_common(T_Q8_0, dx, dy, n, m, stream);
}
int sicu_convert_f16(const float *dx, void *dy, int64_t n, int64_t m, void *stream) {
    return quantize_common(T_F16, dx, dy, n, m, stream);
}
int sicu_quantize_pair(uint32_t wtype, const float *dx, void *dxq, int64_t n, int64_t m, void *stream) {
    uint32_t pair;
    if (!pair_of(wtype, pair)) return fail(SICU_ENOTSUP, "no dot product for type %s (%u)", tname(wtype), wtype);
    return quantize_common(pair, dx, dxq, n, m, stream);
}

int sicu_gemv(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const void *dxq, float *dy, int64_t m,
              void *stream) {
    uint32_t pair;
    if (int rc = check_matvec(wtype, dw, n_in, n_out, dxq, dy, m, pair)) return rc;
    if (!aligned(dxq, pair == T_Q8_K ? 4 : 2)) return fail(SICU_EINVAL, "matvec: activation misaligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (n_out == 0) return SICU_OK;
    const int64_t prb = pair_row_bytes(pair, n_in);
    for (int64_t i = 0; i < m; ++i) {
        GemvLaunch L = make_launch(*ds, dw, n_in, n_out, dy + i * n_out);
        L.xq = static_cast<const uint8_t *>(dxq) + i * prb;
        if (int rc = run_gemv(wtype, L, (cudaStream_t)stream)) return rc;
    }
    return SICU_OK;
}

int sicu_gemv_f32(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const float *dx, float *dy, int64_t m,
                  void *stream) {
    uint32_t pair;
    if (int rc = check_matvec(wtype, dw, n_in, n_out, dx, dy, m, pair)) return rc;
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "matvec: f32 activation must be 16-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (n_out == 0) return SICU_OK;
    for (int64_t i = 0; i < m; ++i) {
        GemvLaunch L = make_launch(*ds, dw, n_in, n_out, dy + i * n_out);
        L.xf = dx + i * n_in;
        if (int rc = run_gemv(wtype, L, (cudaStream_t)stream)) return rc;
    }
    return SICU_OK;
}

int sicu_gemv_multi(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out, int64_t n_in,
                    const float *dx, float *const *dy, void *stream) {
    if (n_mats < 1 || n_mats > MAX_MATS) return fail(SICU_EINVAL, "matvec multi: %d matrices (1..%d)", n_mats, MAX_MATS);
    if (!dw || !n_out || !dy) return fail(SICU_EINVAL, "matvec multi: null array");
    uint32_t pair;
    for (int i = 0; i < n_mats; ++i) {
        if (int rc = check_matvec(wtype, dw[i], n_in, n_out[i], dx, dy[i], 1, pair)) return rc;
        if (n_out[i] > ((int64_t)1 << 30)) return fail(SICU_EINVAL, "matvec multi: too many rows");
    }
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "matvec: f32 activation must be 16-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (wtype == T_F16) {
        for (int i = 0; i < n_mats; ++i) {
            if (n_out[i] == 0) continue;
            GemvLaunch L = make_launch(*ds, dw[i], n_in, n_out[i], dy[i]);
            L.xf = dx;
            if (int rc = run_gemv(wtype, L, (cudaStream_t)stream)) return rc;
        }
        return SICU_OK;
    }
    GemvLaunch L = make_launch(*ds, dw[0], n_in, n_out[0], dy[0]);
    L.xf = dx;
    L.nmat = n_mats;
    for (int i = 0; i < n_mats; ++i) {
        L.wm[i] = dw[i];
        L.ym[i] = dy[i];
        L.n_outm[i] = n_out[i];
    }
    return run_gemv(wtype, L, (cudaStream_t)stream);
}

int sicu_gemv_host(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const float *hx, float *hy,
                   void *stream) {
    uint32_t pair;
    if (int rc = check_matvec(wtype, dw, n_in, n_out, hx, hy, 1, pair)) return rc;
    DevState *ds;
    if (int rc = current(ds)) return rc;
    const size_t xb = ((size_t)n_in * 4 + 255) & ~size_t(255);
    const size_t need = xb + (size_t)n_out * 4;
    cudaError_t e;
    if (ds->stage_bytes < need) {
        if (ds->stage) cudaFree(ds->stage);
        ds->stage = nullptr;
        ds->stage_bytes = 0;
        if ((e = cudaMalloc(&ds->stage, need)) != cudaSuccess) return fail(SICU_ENOMEM, "staging alloc of %zu bytes", need);
        ds->stage_bytes = need;
    }
    float *dx = static_cast<float *>(ds->stage);
    float *dy = reinterpret_cast<float *>(static_cast<uint8_t *>(ds->stage) + xb);
    const cudaStream_t st = (cudaStream_t)stream;
    // page-locked x and y (and a quantized format): the GPU reads x and writes
    // y through their device views, with no copy-engine operation: a small
    // kernel copies x and the matvec, launched behind it, streams its weights
    // meanwhile (the call's latency, not its bandwidth, sets its time)
    cudaPointerAttributes ax{}, ay{};
    const bool direct = wtype != T_F16 && n_out > 0 && n_in % 4 == 0 &&
                        cudaPointerGetAttributes(&ax, hx) == cudaSuccess && ax.type == cudaMemoryTypeHost &&
                        ax.devicePointer && aligned(ax.devicePointer, 16) &&
                        cudaPointerGetAttributes(&ay, hy) == cudaSuccess && ay.type == cudaMemoryTypeHost &&
                        ay.devicePointer;
    cudaGetLastError();
    if (direct) {
        if (launch_host_copy(static_cast<const float *>(ax.devicePointer), dx, n_in, st))
            return cuda_fail(cudaGetLastError(), "gemv_host copy");
        GemvLaunch L = make_launch(*ds, dw, n_in, n_out, static_cast<float *>(ay.devicePointer));
        L.xf = dx;
        L.overlap = 1;
        if (int rc = run_gemv(wtype, L, st)) return rc;
        if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(e, "gemv_host sync");
        return SICU_OK;
    }
    if ((e = cudaMemcpyAsync(dx, hx, (size_t)n_in * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return cuda_fail(e, "gemv_host h2d");
    if (n_out > 0) {
        GemvLaunch L = make_launch(*ds, dw, n_in, n_out, dy);
        L.xf = dx;
        if (int rc = run_gemv(wtype, L, st)) return rc;
        if ((e = cudaMemcpyAsync(hy, dy, (size_t)n_out * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess)
            return cuda_fail(e, "gemv_host d2h");
    }
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(e, "gemv_host sync");
    return SICU_OK;
}

// ---- prefill product -----------------------------------------------------------
static int check_prefill(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const void *dx, int64_t m,
                         const float *dy, uint32_t &pair) {
    if (!pair_of(wtype, pair)) return fail(SICU_ENOTSUP, "prefill: unsupported weight type %s (%u)", tname(wtype), wtype);
    uint32_t blck, bytes;
    geometry(wtype, blck, bytes);
    if (n_in <= 0 || n_out < 0 || m < 0)
        return fail(SICU_EINVAL, "prefill: bad shape n_in=%lld n_out=%lld m=%lld", (long long)n_in, (long long)n_out,
                    (long long)m);
    if (n_in % blck)
        return fail(SICU_EINVAL, "prefill: row length %lld of %s is not a multiple of %u", (long long)n_in, tname(wtype), blck);
    if (n_in > (int64_t)1 << 20 || n_out > (int64_t)1 << 30 || m > 65535)
        return fail(SICU_EINVAL, "prefill: shape too large (n_in <= 2^20, n_out <= 2^30, m <= 65535)");
    if (m == 0 || n_out == 0) return SICU_OK;
    if (!dw || !dx || !dy) return fail(SICU_EINVAL, "prefill: null pointer");
    if (!aligned(dw, 16)) return fail(SICU_EINVAL, "prefill: weight pointer must be 16-byte aligned");
    if (!aligned(dy, 4)) return fail(SICU_EINVAL, "prefill: output must be 4-byte aligned");
    return SICU_OK;
}

static int grow_prefill_ws(DevState &ds, size_t need) {
    if (ds.pf_ws_bytes >= need) return SICU_OK;
    if (ds.pf_ws) cudaFree(ds.pf_ws);
    ds.pf_ws = nullptr;
    ds.pf_ws_bytes = 0;
    if (cudaMalloc(&ds.pf_ws, need) != cudaSuccess) {
        cudaGetLastError();
        return fail(SICU_ENOMEM, "prefill workspace of %zu bytes", need);
    }
    ds.pf_ws_bytes = need;
    return SICU_OK;
}

// The batch matvec (m <= 8 rows, Q4_K / Q6_K) for n_mats matrices sharing one
// activation: xf (m f32 rows) or xq (m Q8_K rows).
static int batch_common(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out, int64_t n_in,
                        const float *xf, const void *xq, int64_t m, float *const *dy, cudaStream_t st) {
    DevState *ds;
    if (int rc = current(ds)) return rc;
    const size_t need = batch_workspace_bytes(n_in);
    if (ds->bt_ws_bytes < need) {
        if (ds->bt_ws) cudaFree(ds->bt_ws);
        ds->bt_ws = nullptr;
        ds->bt_ws_bytes = 0;
        if (cudaMalloc(&ds->bt_ws, need) != cudaSuccess) {
            cudaGetLastError();
            return fail(SICU_ENOMEM, "batch workspace of %zu bytes", need);
        }
        ds->bt_ws_bytes = need;
    }
    BatchLaunch L{};
    L.nmat = n_mats;
    for (int i = 0; i < n_mats; ++i) {
        L.w[i] = dw[i];
        L.y[i] = dy[i];
        L.n_out[i] = n_out[i];
    }
    L.n_in = n_in;
    L.xf = xf;
    L.xq = xq;
    L.m = (int)m;
    L.ws = ds->bt_ws;
    L.num_sms = ds->sms;
    L.smem_per_sm = ds->smem_per_sm;
    L.smem_reserved = ds->smem_reserved;
    L.overlap = g_overlap;
    cudaGetDevice(&L.device);
    L.status = ds->status;
    const int rc = launch_batch(wtype, L, st);
    if (rc == -1) return fail(SICU_EINVAL, "batch matvec: %d matrices, %lld rows (1..16, 1..8)", n_mats, (long long)m);
    if (rc == -3) return fail(SICU_ENOTSUP, "batch matvec: no kernel for %s", tname(wtype));
    if (rc != 0) return cuda_fail(cudaGetLastError(), "batch matvec launch");
    return SICU_OK;
}

// xq: m rows of pair-format activation blocks (device), or null with xf set
static int prefill_common(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const void *xq,
                          const float *xf, int64_t m, float *dy, cudaStream_t st, const void *pack = nullptr) {
    DevState *ds;
    if (int rc = current(ds)) return rc;
    uint32_t pair;
    pair_of(wtype, pair);
    if (m <= BATCH_MAX && batch_supported(wtype)) {
        // a few tokens (a batch of decode steps): every weight block read once
        // for all of them, bit-identical with the per-token matvec
        const void *w1[1] = {dw};
        float *y1[1] = {dy};
        return batch_common(wtype, 1, w1, &n_out, n_in, xf, xq, m, y1, st);
    }
    // Q2_K, Q3_K, Q5_K have tensor-core kernels only for the prefill copy:
    // without a copy of the caller's, the product makes one in the workspace
    const bool copy_only = !prefill_supported(wtype) && prefill_pack_supported(wtype) &&
                           !(is_classic(wtype) && n_in < 128) && !(wtype == T_F16 && n_in % QK_K);
    if (!prefill_supported(wtype) && !(copy_only && m > PREFILL_PACKED_MIN_M)) {
        // formats without a tensor-core kernel (and copy-only formats for
        // blocks of at most 32 tokens): the decode matvec per token
        const int64_t prb = pair_row_bytes(pair, n_in);
        for (int64_t i = 0; i < m; ++i) {
            GemvLaunch L = make_launch(*ds, dw, n_in, n_out, dy + i * n_out);
            if (xq) L.xq = static_cast<const uint8_t *>(xq) + i * prb;
            else L.xf = xf + i * n_in;
            if (int rc = run_gemv(wtype, L, st)) return rc;
        }
        return SICU_OK;
    }
    // f32 rows are quantized inside the launch, straight into the token operand
    size_t need = prefill_workspace_bytes(wtype, n_in, n_out, m, ds->sms, pack != nullptr || copy_only);
    const size_t pack_off = (need + 255) & ~size_t(255);
    const bool own_copy = copy_only && !pack;
    if (own_copy) need = pack_off + prefill_pack_bytes(wtype, n_in, n_out);
    if (int rc = grow_prefill_ws(*ds, need)) return rc;
    if (own_copy) {
        pack = static_cast<uint8_t *>(ds->pf_ws) + pack_off;
        if (launch_prefill_pack(wtype, dw, n_in, n_out, const_cast<void *>(pack), st) != 0)
            return cuda_fail(cudaGetLastError(), "prefill pack launch");
    }
    PrefillLaunch L{};
    L.w = dw;
    L.n_in = n_in;
    L.n_out = n_out;
    L.xq = xq;
    L.xf = xq ? nullptr : xf;
    L.m = m;
    L.y = dy;
    L.ws = ds->pf_ws;
    cudaGetDevice(&L.device);
    L.num_sms = ds->sms;
    L.status = ds->status;
    L.pack = pack;
    const int rc = launch_prefill(wtype, L, st);
    if (rc == -4) return fail(SICU_EIO, "prefill: tensor map encoding failed");
    if (rc != 0) return cuda_fail(cudaGetLastError(), "prefill launch");
    return SICU_OK;
}

int sicu_gemm_prefill(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const void *dxq, int64_t m,
                      float *dy, void *stream) {
    uint32_t pair;
    if (int rc = check_prefill(wtype, dw, n_in, n_out, dxq, m, dy, pair)) return rc;
    if (m == 0 || n_out == 0) return current_ok();
    if (!aligned(dxq, pair == T_Q8_K ? 4 : 2)) return fail(SICU_EINVAL, "prefill: activation misaligned");
    return prefill_common(wtype, dw, n_in, n_out, dxq, nullptr, m, dy, (cudaStream_t)stream);
}

int sicu_gemm_prefill_f32(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const float *dx, int64_t m,
                          float *dy, void *stream) {
    uint32_t pair;
    if (int rc = check_prefill(wtype, dw, n_in, n_out, dx, m, dy, pair)) return rc;
    if (m == 0 || n_out == 0) return current_ok();
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "prefill: f32 activation must be 16-byte aligned");
    return prefill_common(wtype, dw, n_in, n_out, nullptr, dx, m, dy, (cudaStream_t)stream);
}

// ---- prefill copies of the weights ---------------------------------------------------
static int check_pack_shape(const char *what, uint32_t wtype, int64_t n_in, int64_t n_out) {
    if (!prefill_pack_supported(wtype))
        return fail(SICU_ENOTSUP, "%s: no tensor-core prefill kernel for %s (%u)", what, tname(wtype), wtype);
    // K formats: whole super-blocks; classic formats: whole 32-blocks, at least one 128-element K-step
    const bool shape_ok = is_classic(wtype) ? (n_in % 32 == 0 && n_in >= 128) : (n_in % QK_K == 0);
    if (n_in <= 0 || n_out < 0 || !shape_ok || n_in > (int64_t)1 << 20 || n_out > (int64_t)1 << 30)
        return fail(SICU_EINVAL, "%s: bad shape n_in=%lld n_out=%lld", what, (long long)n_in, (long long)n_out);
    return SICU_OK;
}

int sicu_prefill_pack_bytes(uint32_t wtype, int64_t n_in, int64_t n_out, size_t *bytes) {
    if (!bytes) return fail(SICU_EINVAL, "prefill pack: null bytes");
    *bytes = 0;
    if (int rc = check_pack_shape("prefill pack", wtype, n_in, n_out)) return rc;
    *bytes = prefill_pack_bytes(wtype, n_in, n_out);
    return SICU_OK;
}

int sicu_prefill_pack(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, void *dpack, size_t pack_bytes,
                      void *stream) {
    if (int rc = check_pack_shape("prefill pack", wtype, n_in, n_out)) return rc;
    const size_t need = prefill_pack_bytes(wtype, n_in, n_out);
    if (pack_bytes < need)
        return fail(SICU_EINVAL, "prefill pack: %zu bytes given, %zu needed", pack_bytes, need);
    if (n_out == 0) return current_ok();
    if (!dw || !dpack) return fail(SICU_EINVAL, "prefill pack: null pointer");
    if (!aligned(dw, 16) || !aligned(dpack, 16)) return fail(SICU_EINVAL, "prefill pack: pointers must be 16-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_prefill_pack(wtype, dw, n_in, n_out, dpack, (cudaStream_t)stream) != 0)
        return cuda_fail(cudaGetLastError(), "prefill pack launch");
    return SICU_OK;
}

static int check_packed(uint32_t wtype, const void *dpack) {
    if (!dpack) return SICU_OK;
    if (!prefill_pack_supported(wtype))
        return fail(SICU_EINVAL, "prefill: %s has no prefill copy (no tensor-core kernel)", tname(wtype));
    if (!aligned(dpack, 16)) return fail(SICU_EINVAL, "prefill: packed copy must be 16-byte aligned");
    return SICU_OK;
}

int sicu_gemm_prefill_packed(uint32_t wtype, const void *dw, const void *dpack, int64_t n_in, int64_t n_out,
                             const void *dxq, int64_t m, float *dy, void *stream) {
    uint32_t pair;
    if (int rc = check_prefill(wtype, dw, n_in, n_out, dxq, m, dy, pair)) return rc;
    if (int rc = check_packed(wtype, dpack)) return rc;
    if (m == 0 || n_out == 0) return current_ok();
    if (!aligned(dxq, pair == T_Q8_K ? 4 : 2)) return fail(SICU_EINVAL, "prefill: activation misaligned");
    return prefill_common(wtype, dw, n_in, n_out, dxq, nullptr, m, dy, (cudaStream_t)stream, dpack);
}

int sicu_gemm_prefill_packed_f32(uint32_t wtype, const void *dw, const void *dpack, int64_t n_in, int64_t n_out,
                                 const float *dx, int64_t m, float *dy, void *stream) {
    uint32_t pair;
    if (int rc = check_prefill(wtype, dw, n_in, n_out, dx, m, dy, pair)) return rc;
    if (int rc = check_packed(wtype, dpack)) return rc;
    if (m == 0 || n_out == 0) return current_ok();
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "prefill: f32 activation must be 16-byte aligned");
    return prefill_common(wtype, dw, n_in, n_out, nullptr, dx, m, dy, (cudaStream_t)stream, dpack);
}

int sicu_gemm_prefill_multi_f32(uint32_t wtype, int n_mats, const void *const *dw, const void *const *dpack,
                                const int64_t *n_out, int64_t n_in, const float *dx, int64_t m, float *const *dy,
                                void *stream) {
    if (n_mats < 1 || n_mats > PREFILL_MAXM)
        return fail(SICU_EINVAL, "prefill multi: %d matrices (1..%d)", n_mats, PREFILL_MAXM);
    if (!dw || !n_out || !dy) return fail(SICU_EINVAL, "prefill multi: null array");
    uint32_t pair;
    for (int i = 0; i < n_mats; ++i) {
        if (int rc = check_prefill(wtype, dw[i], n_in, n_out[i], dx, m, dy[i], pair)) return rc;
        if (dpack)
            if (int rc = check_packed(wtype, dpack[i])) return rc;
    }
    if (m == 0) return current_ok();
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "prefill multi: f32 activation must be 16-byte aligned");
    const cudaStream_t st = (cudaStream_t)stream;
    bool grouped = dpack && n_mats > 1 && m > PREFILL_PACKED_MIN_M && prefill_groupable(wtype);
    for (int i = 0; grouped && i < n_mats; ++i) grouped = dpack[i] && n_out[i] > 0;
    if (!grouped) {
        // the products one by one (a few tokens: one batch launch for all)
        if (m <= BATCH_MAX && batch_supported(wtype))
            return batch_common(wtype, n_mats, dw, n_out, n_in, dx, nullptr, m, dy, st);
        for (int i = 0; i < n_mats; ++i)
            if (n_out[i] > 0)
                if (int rc = prefill_common(wtype, dw[i], n_in, n_out[i], nullptr, dx, m, dy[i], st,
                                            dpack ? dpack[i] : nullptr))
                    return rc;
        return SICU_OK;
    }
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (int rc = grow_prefill_ws(*ds, prefill_group_workspace_bytes(wtype, n_in, n_mats, n_out, m, ds->sms)))
        return rc;
    PrefillLaunch L{};
    L.w = dw[0];
    L.n_in = n_in;
    L.n_out = n_out[0];
    L.xf = dx;
    L.m = m;
    L.y = dy[0];
    L.ws = ds->pf_ws;
    cudaGetDevice(&L.device);
    L.num_sms = ds->sms;
    L.status = ds->status;
    L.pack = dpack[0];
    L.nmat = n_mats;
    for (int i = 0; i < n_mats; ++i) {
        L.packm[i] = dpack[i];
        L.n_outm[i] = n_out[i];
        L.ym[i] = dy[i];
    }
    const int rc = launch_prefill(wtype, L, st);
    if (rc == -4) return fail(SICU_EIO, "prefill multi: tensor map encoding failed");
    if (rc != 0) return cuda_fail(cudaGetLastError(), "prefill multi launch");
    return SICU_OK;
}

int sicu_gemv_batch(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out, int64_t n_in,
                    const float *dx, int64_t m, float *const *dy, void *stream) {
    if (n_mats < 1 || n_mats > 16) return fail(SICU_EINVAL, "batch matvec: %d matrices (1..16)", n_mats);
    if (!dw || !n_out || !dy) return fail(SICU_EINVAL, "batch matvec: null array");
    if (m < 0 || m > 8) return fail(SICU_EINVAL, "batch matvec: %lld activation rows (0..8)", (long long)m);
    uint32_t pair;
    for (int i = 0; i < n_mats; ++i)
        if (int rc = check_matvec(wtype, dw[i], n_in, n_out[i], dx, dy[i], 1, pair)) return rc;
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "batch matvec: f32 activation must be 16-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (m == 0) return SICU_OK;
    const cudaStream_t st = (cudaStream_t)stream;
    if (m > 1 && batch_supported(wtype)) return batch_common(wtype, n_mats, dw, n_out, n_in, dx, nullptr, m, dy, st);
    // one activation row, or a type without a batch kernel: the matvec once per
    // row (one launch for all matrices; F16 one launch per matrix)
    for (int64_t t = 0; t < m; ++t) {
        for (int i0 = 0; i0 < n_mats; i0 = (wtype == T_F16) ? i0 + 1 : n_mats) {
            const int i1 = (wtype == T_F16) ? i0 + 1 : n_mats;
            GemvLaunch L = make_launch(*ds, dw[i0], n_in, n_out[i0], dy[i0] + t * n_out[i0]);
            L.xf = dx + t * n_in;
            L.nmat = i1 - i0;
            for (int i = i0; i < i1; ++i) {
                L.wm[i - i0] = dw[i];
                L.ym[i - i0] = dy[i] + t * n_out[i];
                L.n_outm[i - i0] = n_out[i];
            }
            if (int rc = run_gemv(wtype, L, st)) return rc;
        }
    }
    return SICU_OK;
}

// ---- fused all-reduce groups ---------------------------------------------------------
}  // extern "C"

struct sicu_ar {
    ArDev d;                       // what the kernels get (by value)
    int device = -1;
    void *own = nullptr;           // this rank's allocation
    void *peer[AR_MAX] = {};       // mapped peer allocations
    bool opened = false;
};

static_assert(sizeof(cudaIpcMemHandle_t) == SICU_AR_HANDLE_BYTES, "IPC handle size");

namespace {

int ar_current(sicu_ar *g, DevState *&ds) {
    if (!g) return fail(SICU_EINVAL, "all-reduce: null group");
    if (!g->opened) return fail(SICU_EINVAL, "all-reduce: group not opened (sicu_ar_open)");
    if (int rc = current(ds)) return rc;
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != g->device) return fail(SICU_EINVAL, "all-reduce: group belongs to device %d, current is %d", g->device, dev);
    return SICU_OK;
}

}  // namespace

extern "C" {

int sicu_ar_create(int n_ranks, int rank, int64_t len, sicu_ar **group, void *handle) {
    if (!group || !handle) return fail(SICU_EINVAL, "all-reduce: null out pointer");
    *group = nullptr;
    if (n_ranks < 1 || n_ranks > AR_MAX) return fail(SICU_EINVAL, "all-reduce: %d ranks (1..%d)", n_ranks, AR_MAX);
    if (rank < 0 || rank >= n_ranks) return fail(SICU_EINVAL, "all-reduce: rank %d of %d", rank, n_ranks);
    if (len <= 0 || len % 256 || len > ((int64_t)1 << 24))
        return fail(SICU_EINVAL, "all-reduce: length %lld (a multiple of 256, <= 2^24)", (long long)len);
    DevState *ds;
    if (int rc = current(ds)) return rc;
    sicu_ar *g = new sicu_ar;
    cudaGetDevice(&g->device);
    const size_t bytes = (size_t)ar_alloc_bytes(n_ranks, len);
    cudaError_t e = cudaMalloc(&g->own, bytes);
    if (e != cudaSuccess) {
        delete g;
        cudaGetLastError();
        return fail(SICU_ENOMEM, "all-reduce: %zu bytes", bytes);
    }
    // zeroed and complete before any peer can learn the handle
    if ((e = cudaMemset(g->own, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess ||
        (e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), g->own)) != cudaSuccess) {
        cudaFree(g->own);
        delete g;
        return cuda_fail(e, "all-reduce: create");
    }
    g->d.n = n_ranks;
    g->d.rank = rank;
    g->d.len = len;
    g->d.limit_ns = 2000000000ull;
    g->d.epoch = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(g->own) + ar_epoch_offset(n_ranks, len));
    *group = g;
    return SICU_OK;
}

int sicu_ar_open(sicu_ar *g, const void *handles) {
    if (!g || !handles) return fail(SICU_EINVAL, "all-reduce: null pointer");
    if (g->opened) return fail(SICU_EINVAL, "all-reduce: group already opened");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != g->device) return fail(SICU_EINVAL, "all-reduce: group belongs to device %d, current is %d", g->device, dev);
    const auto *h = static_cast<const cudaIpcMemHandle_t *>(handles);
    for (int q = 0; q < g->d.n; ++q) {
        void *base = g->own;
        if (q != g->d.rank) {
            const cudaError_t e = cudaIpcOpenMemHandle(&base, h[q], cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                for (int k = 0; k < q; ++k)
                    if (g->peer[k]) cudaIpcCloseMemHandle(g->peer[k]), g->peer[k] = nullptr;
                return cuda_fail(e, "all-reduce: open a peer's handle");
            }
            g->peer[q] = base;
        }
        g->d.slot[q] = static_cast<uint64_t *>(base);
    }
    g->opened = true;
    return SICU_OK;
}

int sicu_ar_set_timeout(sicu_ar *g, uint64_t ns) {
    if (!g) return fail(SICU_EINVAL, "all-reduce: null group");
    if (ns == 0) return fail(SICU_EINVAL, "all-reduce: zero timeout");
    g->d.limit_ns = ns;
    return SICU_OK;
}

int sicu_ar_destroy(sicu_ar *g) {
    if (!g) return SICU_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    if (g->device >= 0) cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    for (int q = 0; q < AR_MAX; ++q)
        if (g->peer[q]) cudaIpcCloseMemHandle(g->peer[q]);
    if (g->own) cudaFree(g->own);
    if (cur >= 0) cudaSetDevice(cur);
    delete g;
    return SICU_OK;
}

int sicu_ar_allreduce(sicu_ar *g, const float *dsrc, float *ddst, void *stream) {
    DevState *ds;
    if (int rc = ar_current(g, ds)) return rc;
    if (!dsrc || !ddst) return fail(SICU_EINVAL, "all-reduce: null vector");
    if (launch_allreduce(g->d, dsrc, ddst, ds->status, ds->sms, (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "all-reduce launch");
    return SICU_OK;
}

int sicu_gemv_ar(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, const float *dx, float *dy,
                 sicu_ar *g, void *stream) {
    if (wtype == T_F16) return fail(SICU_ENOTSUP, "matvec ar: F16 weights are not supported");
    uint32_t pair;
    if (int rc = check_matvec(wtype, dw, n_in, n_out, dx, dy, 1, pair)) return rc;
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "matvec: f32 activation must be 16-byte aligned");
    DevState *ds;
    if (int rc = ar_current(g, ds)) return rc;
    if (n_out != g->d.len)
        return fail(SICU_EINVAL, "matvec ar: %lld rows, the group reduces vectors of %lld", (long long)n_out,
                    (long long)g->d.len);
    GemvLaunch L = make_launch(*ds, dw, n_in, n_out, dy);
    L.xf = dx;
    L.ar = g->d;
    return run_gemv(wtype, L, (cudaStream_t)stream);
}

}  // extern "C"

namespace {

// [a, a + abytes) and [b, b + bbytes) share a byte (bbytes < 0: same as abytes)
bool overlaps(const void *a, const void *b, int64_t abytes, int64_t bbytes = -1) {
    if (!a || !b) return false;
    if (bbytes < 0) bbytes = abytes;
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + (uintptr_t)bbytes && y < x + (uintptr_t)abytes;
}

// Checks a step's vectors (n floats each) and turns it into the kernels' form.
int check_prologue(const sicu_prologue *pro, int64_t n, const float *dx, ProDev &pd) {
    pd = ProDev{};
    if (!pro || pro->kind == SICU_PRO_NONE) return SICU_OK;
    if (n % 4) return fail(SICU_EINVAL, "activation step: length %lld is not a multiple of 4", (long long)n);
    if (pro->kind == SICU_PRO_RMS_NORM) {
        if (!pro->weight) return fail(SICU_EINVAL, "rms norm: null weight");
        if (!aligned(pro->weight, 16) || !aligned(pro->residual, 16) || !aligned(pro->sum_out, 16))
            return fail(SICU_EINVAL, "rms norm: vectors must be 16-byte aligned");
        if (!(pro->eps >= 0.0f)) return fail(SICU_EINVAL, "rms norm: eps must be >= 0");
        if (n > INT32_MAX) return fail(SICU_EINVAL, "rms norm: row too long");
        const int64_t b = n * 4;
        if (overlaps(pro->sum_out, dx, b) || overlaps(pro->sum_out, pro->residual, b) ||
            overlaps(pro->sum_out, pro->weight, b))
            return fail(SICU_EINVAL, "rms norm: sum_out overlaps an input");
        pd.kind = PRO_RMS_NORM;
        pd.eps = pro->eps;
        pd.g = pro->weight;
        pd.res = pro->residual;
        pd.h_out = pro->sum_out;
        pd.inv_n = 1.0 / (double)n;
        return SICU_OK;
    }
    if (pro->kind == SICU_PRO_SWIGLU || pro->kind == SICU_PRO_MUL) {
        if (!pro->up) return fail(SICU_EINVAL, "swiglu: null up vector");
        if (!aligned(pro->up, 16)) return fail(SICU_EINVAL, "swiglu: up vector must be 16-byte aligned");
        if (n % 8) return fail(SICU_EINVAL, "swiglu: length %lld is not a multiple of 8", (long long)n);
        pd.kind = pro->kind == SICU_PRO_SWIGLU ? PRO_SWIGLU : PRO_MUL;
        pd.up = pro->up;
        return SICU_OK;
    }
    return fail(SICU_EINVAL, "activation step: unknown kind %d", (int)pro->kind);
}

int run_step(const ProDev &pd, const float *dx, int64_t n, float *dy, cudaStream_t st) {
    int rc;
    if (pd.kind == PRO_RMS_NORM) rc = launch_rms_norm(dx, pd.res, pd.h_out, pd.g, n, 1, pd.eps, dy, st);
    else if (pd.kind == PRO_SWIGLU) rc = launch_swiglu(dx, pd.up, n, 1, dy, st);
    else rc = launch_mul(dx, pd.up, n, dy, st);
    return rc ? cuda_fail(cudaGetLastError(), "activation step launch") : SICU_OK;
}

}  // namespace

extern "C" {

int sicu_gemv_fused(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out, int64_t n_in,
                    const float *dx, const sicu_prologue *pro, const int32_t *epi, float *const *dy, sicu_ar *group,
                    void *stream) {
    return sicu_gemv_fused_ex(wtype, n_mats, dw, n_out, n_in, dx, pro, epi, nullptr, dy, group, stream);
}

int sicu_gemv_fused_ex(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out, int64_t n_in,
                       const float *dx, const sicu_prologue *pro, const int32_t *epi, const float *const *bias,
                       float *const *dy, sicu_ar *group, void *stream) {
    if (n_mats < 1 || n_mats > MAX_MATS) return fail(SICU_EINVAL, "matvec fused: %d matrices (1..%d)", n_mats, MAX_MATS);
    if (!dw || !n_out || !dy) return fail(SICU_EINVAL, "matvec fused: null array");
    uint32_t pair;
    for (int i = 0; i < n_mats; ++i) {
        if (int rc = check_matvec(wtype, dw[i], n_in, n_out[i], dx, dy[i], 1, pair)) return rc;
        if (n_out[i] > ((int64_t)1 << 30)) return fail(SICU_EINVAL, "matvec fused: too many rows");
    }
    if (!aligned(dx, 16)) return fail(SICU_EINVAL, "matvec: f32 activation must be 16-byte aligned");
    ProDev pd;
    if (int rc = check_prologue(pro, n_in, dx, pd)) return rc;
    if (pd.h_out)
        for (int i = 0; i < n_mats; ++i)
            if (overlaps(pd.h_out, dy[i], 4 * n_in, 4 * n_out[i]))
                return fail(SICU_EINVAL, "rms norm: sum_out overlaps an output");
    uint64_t silu_mask = 0;
    if (epi)
        for (int i = 0; i < n_mats; ++i) {
            if (epi[i] == SICU_EPI_SILU) silu_mask |= 1ull << i;
            else if (epi[i] != SICU_EPI_NONE) return fail(SICU_EINVAL, "matvec fused: unknown epilogue %d", (int)epi[i]);
        }
    const float *bs[MAX_MATS] = {};
    if (bias)
        for (int i = 0; i < n_mats; ++i) {
            bs[i] = bias[i];
            if (bs[i] && !aligned(bs[i], 4)) return fail(SICU_EINVAL, "matvec fused: bias %d misaligned", i);
        }
    DevState *ds;
    const cudaStream_t st = (cudaStream_t)stream;
    if (group) {
        if (n_mats != 1) return fail(SICU_EINVAL, "matvec fused: an all-reduce group takes one matrix");
        if (wtype == T_F16) return fail(SICU_ENOTSUP, "matvec ar: F16 weights are not supported");
        if (int rc = ar_current(group, ds)) return rc;
        if (n_out[0] != group->d.len)
            return fail(SICU_EINVAL, "matvec ar: %lld rows, the group reduces vectors of %lld", (long long)n_out[0],
                        (long long)group->d.len);
        GemvLaunch L = make_launch(*ds, dw[0], n_in, n_out[0], dy[0]);
        L.xf = dx;
        L.ar = group->d;
        L.pro = pd;
        L.epi_silu = silu_mask;
        L.bias[0] = bs[0];
        return run_gemv(wtype, L, st);
    }
    if (int rc = current(ds)) return rc;
    if (wtype == T_F16) {
        const float *x = dx;
        if (pd.kind != PRO_NONE) {
            const size_t need = (size_t)n_in * 4;
            if (ds->pro_buf_bytes < need) {
                if (ds->pro_buf) cudaFree(ds->pro_buf);
                ds->pro_buf = nullptr;
                ds->pro_buf_bytes = 0;
                if (cudaMalloc(&ds->pro_buf, need) != cudaSuccess) {
                    cudaGetLastError();
                    return fail(SICU_ENOMEM, "activation step buffer");
                }
                ds->pro_buf_bytes = need;
            }
            if (int rc = run_step(pd, dx, n_in, ds->pro_buf, st)) return rc;
            x = ds->pro_buf;
        }
        for (int i = 0; i < n_mats; ++i) {
            if (n_out[i] == 0) continue;
            GemvLaunch L = make_launch(*ds, dw[i], n_in, n_out[i], dy[i]);
            L.xf = x;
            if (int rc = run_gemv(wtype, L, st)) return rc;
            if (bs[i] && launch_add_inplace(dy[i], bs[i], n_out[i], st)) return cuda_fail(cudaGetLastError(), "bias launch");
            if (((silu_mask >> i) & 1) && launch_silu_inplace(dy[i], n_out[i], st))
                return cuda_fail(cudaGetLastError(), "silu launch");
        }
        return SICU_OK;
    }
    GemvLaunch L = make_launch(*ds, dw[0], n_in, n_out[0], dy[0]);
    L.xf = dx;
    L.pro = pd;
    L.epi_silu = silu_mask;
    L.nmat = n_mats;
    for (int i = 0; i < n_mats; ++i) {
        L.wm[i] = dw[i];
        L.ym[i] = dy[i];
        L.n_outm[i] = n_out[i];
        L.bias[i] = bs[i];
    }
    return run_gemv(wtype, L, st);
}

int sicu_rms_norm(const float *dx, const float *dres, float *dsum, const float *dw, int64_t n, int64_t m, float eps,
                  float *dy, void *stream) {
    if (n <= 0 || m < 0 || m > INT32_MAX)
        return fail(SICU_EINVAL, "rms norm: bad shape n=%lld m=%lld", (long long)n, (long long)m);
    if (!dx || !dy) return fail(SICU_EINVAL, "rms norm: null pointer");
    if (!aligned(dx, 16) || !aligned(dy, 16)) return fail(SICU_EINVAL, "rms norm: rows must be 16-byte aligned");
    sicu_prologue pro{SICU_PRO_RMS_NORM, eps, dw, dres, dsum, nullptr};
    ProDev pd;
    if (int rc = check_prologue(&pro, n, dx, pd)) return rc;
    if (overlaps(dsum, dy, 4 * n * m) || overlaps(dsum, dx, 4 * n * m) || overlaps(dsum, dres, 4 * n * m))
        return fail(SICU_EINVAL, "rms norm: sum_out overlaps another row block");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (m == 0) return SICU_OK;
    if (launch_rms_norm(dx, dres, dsum, dw, n, m, eps, dy, (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "rms norm launch");
    return SICU_OK;
}

int sicu_add_bias(float *dy, const float *db, int64_t n, int64_t m, void *stream) {
    if (n <= 0 || m < 0 || n > INT64_MAX / (m > 0 ? m : 1))
        return fail(SICU_EINVAL, "add bias: bad shape n=%lld m=%lld", (long long)n, (long long)m);
    if (!dy || !db) return fail(SICU_EINVAL, "add bias: null pointer");
    if (!aligned(dy, 4) || !aligned(db, 4)) return fail(SICU_EINVAL, "add bias: rows must be 4-byte aligned");
    if (overlaps(dy, db, 4 * n * m, 4 * n)) return fail(SICU_EINVAL, "add bias: bias overlaps the rows");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (m == 0) return SICU_OK;
    if (launch_add_rows(dy, db, n, m, (cudaStream_t)stream)) return cuda_fail(cudaGetLastError(), "add bias launch");
    return SICU_OK;
}

int sicu_swiglu(const float *dx, const float *dup, int64_t n, int64_t m, float *dy, void *stream) {
    if (n <= 0 || m < 0) return fail(SICU_EINVAL, "swiglu: bad shape n=%lld m=%lld", (long long)n, (long long)m);
    if (!dx || !dy) return fail(SICU_EINVAL, "swiglu: null pointer");
    if (!aligned(dx, 16) || !aligned(dy, 16)) return fail(SICU_EINVAL, "swiglu: rows must be 16-byte aligned");
    sicu_prologue pro{SICU_PRO_SWIGLU, 0.0f, nullptr, nullptr, nullptr, dup};
    ProDev pd;
    if (int rc = check_prologue(&pro, n, dx, pd)) return rc;
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (m == 0) return SICU_OK;
    if (launch_swiglu(dx, dup, n, m, dy, (cudaStream_t)stream)) return cuda_fail(cudaGetLastError(), "swiglu launch");
    return SICU_OK;
}

int sicu_softmax(const float *dx, float *dy, int64_t n, int64_t m, void *stream) {
    if (n <= 0 || n > INT32_MAX || m < 0 || m > INT32_MAX)
        return fail(SICU_EINVAL, "softmax: bad shape n=%lld m=%lld", (long long)n, (long long)m);
    if (!dx || !dy) return fail(SICU_EINVAL, "softmax: null pointer");
    if (dx != dy && overlaps(dx, dy, 4 * n * m)) return fail(SICU_EINVAL, "softmax: rows overlap partially");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (m == 0) return SICU_OK;
    if (launch_softmax(dx, dy, n, m, (cudaStream_t)stream)) return cuda_fail(cudaGetLastError(), "softmax launch");
    return SICU_OK;
}

int sicu_rope(float *dx, int64_t n_heads, int64_t head_dim, int64_t n_rot, const float *dcos, const float *dsin,
              int neox, void *stream) {
    if (n_heads < 0 || head_dim <= 0 || n_rot < 0 || n_rot > head_dim || n_rot % 2 || (neox && head_dim % 2) ||
        n_heads * head_dim > INT32_MAX)
        return fail(SICU_EINVAL, "rope: bad shape");
    if (!dx || (n_rot && (!dcos || !dsin))) return fail(SICU_EINVAL, "rope: null pointer");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_rope(dx, (int)n_heads, (int)head_dim, (int)n_rot, dcos, dsin, neox ? 1 : 0, (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "rope launch");
    return SICU_OK;
}

int sicu_kv_store(const float *dk, const float *dv, void *dk_cache, void *dv_cache, int64_t n_head_kv,
                  int64_t head_dim, int64_t n_ctx, int64_t pos, void *stream) {
    if (n_head_kv <= 0 || head_dim <= 0 || n_ctx <= 0 || pos < 0 || pos >= n_ctx || n_head_kv * head_dim > INT32_MAX ||
        n_ctx > INT32_MAX)
        return fail(SICU_EINVAL, "kv store: bad shape or position");
    if (!dk || !dv || !dk_cache || !dv_cache) return fail(SICU_EINVAL, "kv store: null pointer");
    if (!aligned(dk_cache, 2) || !aligned(dv_cache, 2)) return fail(SICU_EINVAL, "kv store: caches must be 2-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_kv_store(dk, dv, dk_cache, dv_cache, (int)n_head_kv, (int)head_dim, (int)n_ctx, (int)pos,
                        (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "kv store launch");
    return SICU_OK;
}

int sicu_attention(const float *dq, const void *dk_cache, const void *dv_cache, int64_t n_head, int64_t n_head_kv,
                   int64_t head_dim, int64_t n_ctx, int64_t pos, float kq_scale, float *dout, void *stream) {
    if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv || head_dim <= 0 || head_dim > 1024 || n_ctx <= 0 ||
        n_ctx > INT32_MAX || pos < 0 || pos >= n_ctx || n_head * head_dim > INT32_MAX)
        return fail(SICU_EINVAL, "attention: bad shape or position");
    if (pos + 1 > 32768) return fail(SICU_EINVAL, "attention: at most 32768 positions per call");
    if (!dq || !dk_cache || !dv_cache || !dout) return fail(SICU_EINVAL, "attention: null pointer");
    if (!aligned(dk_cache, 2) || !aligned(dv_cache, 2)) return fail(SICU_EINVAL, "attention: caches must be 2-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_attention(dq, dk_cache, dv_cache, (int)n_head, (int)n_head_kv, (int)head_dim, (int)n_ctx, (int)pos,
                         kq_scale, dout, (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "attention launch");
    return SICU_OK;
}

int sicu_attention_step(const float *dq, const float *dk, const float *dv, void *dk_cache, void *dv_cache,
                        const float *dcos, const float *dsin, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                        int64_t n_rot, int neox, int64_t n_ctx, int64_t pos, float kq_scale, float *dout,
                        void *stream) {
    if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv || head_dim <= 0 || head_dim > 1024 || n_ctx <= 0 ||
        n_ctx > INT32_MAX || pos < 0 || pos >= n_ctx || n_head * head_dim > INT32_MAX || n_rot < 0 ||
        n_rot > head_dim || n_rot % 2 || (neox && head_dim % 2))
        return fail(SICU_EINVAL, "attention step: bad shape or position");
    if (pos + 1 > 30000) return fail(SICU_EINVAL, "attention step: at most 30000 positions per call");
    if (!dq || !dk || !dv || !dk_cache || !dv_cache || !dout || (n_rot && (!dcos || !dsin)))
        return fail(SICU_EINVAL, "attention step: null pointer");
    if (!aligned(dk_cache, 2) || !aligned(dv_cache, 2)) return fail(SICU_EINVAL, "attention step: caches must be 2-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_attention_step(dq, dk, dv, dk_cache, dv_cache, dcos, dsin, (int)n_head, (int)n_head_kv, (int)head_dim,
                              (int)n_rot, neox ? 1 : 0, (int)n_ctx, (int)pos, kq_scale, dout, g_overlap,
                              (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "attention step launch");
    return SICU_OK;
}

int sicu_attention_prompt(const float *dq, const float *dk, const float *dv, void *dk_cache, void *dv_cache,
                          const float *dcos, const float *dsin, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                          int64_t n_rot, int neox, int64_t n_ctx, int64_t pos0, int64_t m, float kq_scale,
                          float *dout, void *stream) {
    if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv || head_dim <= 0 || head_dim > 1024 || n_ctx <= 0 ||
        n_ctx > INT32_MAX || pos0 < 0 || m < 0 || pos0 + m > n_ctx || n_head * head_dim > INT32_MAX || n_rot < 0 ||
        n_rot > head_dim || n_rot % 2 || (neox && head_dim % 2) || n_head > 65535 || m > 65535)
        return fail(SICU_EINVAL, "attention prompt: bad shape or positions");
    if (pos0 + m > 30000) return fail(SICU_EINVAL, "attention prompt: at most 30000 positions per call");
    if (m == 0) return current_ok();
    if (!dq || !dk || !dv || !dk_cache || !dv_cache || !dout || (n_rot && (!dcos || !dsin)))
        return fail(SICU_EINVAL, "attention prompt: null pointer");
    if (!aligned(dk_cache, 2) || !aligned(dv_cache, 2))
        return fail(SICU_EINVAL, "attention prompt: caches must be 2-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_attention_prompt(dq, dk, dv, dk_cache, dv_cache, dcos, dsin, (int)n_head, (int)n_head_kv,
                                (int)head_dim, (int)n_rot, neox ? 1 : 0, (int)n_ctx, (int)pos0, (int)m, kq_scale, dout,
                                (cudaStream_t)stream))
        return cuda_fail(cudaGetLastError(), "attention prompt launch");
    return SICU_OK;
}

int sicu_row_to_f32_dev(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_rows, const int64_t *drows,
                        int64_t nrows, float *dout, void *stream) {
    uint32_t blck, bytes;
    if (!geometry(wtype, blck, bytes) || wtype == T_F32 || wtype == T_Q8_K)
        return fail(SICU_ENOTSUP, "row_to_f32: unsupported type %s (%u)", tname(wtype), wtype);
    if (n_in <= 0 || n_rows <= 0 || nrows < 0 || n_in % blck) return fail(SICU_EINVAL, "row_to_f32: bad shape");
    if (nrows > 65535) return fail(SICU_EINVAL, "row_to_f32: at most 65535 rows per call");
    if (!dw || !dout || (nrows && !drows)) return fail(SICU_EINVAL, "row_to_f32: null pointer");
    if (!aligned(drows, 8)) return fail(SICU_EINVAL, "row_to_f32: row ids must be 8-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (nrows == 0) return SICU_OK;
    if (launch_dequant(wtype, dw, n_in, drows, nrows, dout, (cudaStream_t)stream, n_rows, ds->status))
        return cuda_fail(cudaGetLastError(), "dequant launch");
    return SICU_OK;
}

int sicu_argmax(const float *dx, int64_t n, int64_t m, int64_t *dout, void *stream) {
    if (n <= 0 || m < 0 || m > INT32_MAX) return fail(SICU_EINVAL, "argmax: bad shape");
    if (!dx || !dout) return fail(SICU_EINVAL, "argmax: null pointer");
    if (!aligned(dout, 8)) return fail(SICU_EINVAL, "argmax: output must be 8-byte aligned");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (launch_argmax(dx, n, m, dout, (cudaStream_t)stream)) return cuda_fail(cudaGetLastError(), "argmax launch");
    return SICU_OK;
}

int sicu_row_to_f32(uint32_t wtype, const void *dw, int64_t n_in, const int64_t *rows, int64_t nrows, float *dout,
                    void *stream) {
    uint32_t blck, bytes;
    if (!geometry(wtype, blck, bytes) || wtype == T_F32 || wtype == T_Q8_K)
        return fail(SICU_ENOTSUP, "row_to_f32: unsupported type %s (%u)", tname(wtype), wtype);
    if (n_in <= 0 || nrows < 0 || n_in % blck) return fail(SICU_EINVAL, "row_to_f32: bad shape");
    if (nrows > 65535) return fail(SICU_EINVAL, "row_to_f32: at most 65535 rows per call");
    if (!dw || !dout || (nrows && !rows)) return fail(SICU_EINVAL, "row_to_f32: null pointer");
    DevState *ds;
    if (int rc = current(ds)) return rc;
    if (nrows == 0) return SICU_OK;
    const size_t need = (size_t)nrows * sizeof(int64_t);
    cudaError_t e;
    // the row list rides in the staging buffer's tail-free head
    if (ds->stage_bytes < need) {
        if (ds->stage) cudaFree(ds->stage);
        ds->stage = nullptr;
        ds->stage_bytes = 0;
        if ((e = cudaMalloc(&ds->stage, need)) != cudaSuccess) return fail(SICU_ENOMEM, "staging alloc");
        ds->stage_bytes = need;
    }
    const cudaStream_t st = (cudaStream_t)stream;
    if ((e = cudaMemcpyAsync(ds->stage, rows, need, cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return cuda_fail(e, "row list copy");
    const int rc = launch_dequant(wtype, dw, n_in, static_cast<const int64_t *>(ds->stage), nrows, dout, st);
    if (rc) return cuda_fail(cudaGetLastError(), "dequant launch");
    // the row list must stay put until the kernel read it
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(e, "row_to_f32 sync");
    return SICU_OK;
}

}  // extern "C"
