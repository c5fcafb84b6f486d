// sicu_gemv_host_noalloc: the host-buffer matvec of sicu_gemv_host for
// callers that cannot allocate device memory. Its device staging (the copied
// activation, the output before it goes back to the host, a status word) is a
// fixed array compiled into the library instead of memory obtained from
// cudaMalloc, so a call performs no allocation at all.
#include <cstring>
#include <mutex>

#include "siphon_cuda.h"
#include "common.cuh"
#include "launch.h"

namespace sicu {
int report_error(int code, const char *fmt, ...);
}

using namespace sicu;

namespace {

constexpr int64_t NA_MAX_IN = 65536;     // activation elements per call
constexpr int64_t NA_MAX_OUT = 262144;   // output rows per call
constexpr size_t NA_HDR = 256;           // status word, padded to 256 bytes
constexpr size_t NA_BYTES = NA_HDR + 4 * (size_t)(NA_MAX_IN + NA_MAX_OUT);

// [0, 256): status word | activation f32 [NA_MAX_IN] | output f32 [NA_MAX_OUT]
// (1.25 MiB, resident on every device that loads the library until exit)
static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

struct NaDev {
    bool ready = false;
    unsigned char *scratch = nullptr;   // device address of g_noalloc_scratch
    int sms = 0, smem_optin = 0, smem_per_sm = 0, smem_reserved = 0;
};
NaDev g_na[64];
std::mutex g_na_mu;

int na_cuda_fail(cudaError_t e, const char *what) {
    return report_error(SICU_EIO, "gemv_host_noalloc: %s: %s", what, cudaGetErrorString(e));
}

// First call on a device: with that device current, resolve the scratch
// array's device address and read the launch limits. No allocation. The
// address is kept for the life of the process: after a cudaDeviceReset the
// module loads again in a new context, and the kept address is stale.
int na_setup(int dev, NaDev *&out) {
    std::lock_guard<std::mutex> lk(g_na_mu);
    NaDev &d = g_na[dev];
    if (!d.ready) {
        int major = 0, minor = 0;
        cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        if (e != cudaSuccess) return na_cuda_fail(e, "device attributes");
        if (major != 10 || minor != 0)
            return report_error(SICU_ENOTSUP, "gemv_host_noalloc: device %d is sm_%d%d; this library is built for "
                                "sm_100a only", dev, major, minor);
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) return na_cuda_fail(e, "scratch address");
        d.scratch = static_cast<unsigned char *>(ptr);
        if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess)
            return na_cuda_fail(e, "device attributes");
        d.ready = true;
    }
    out = &d;
    return SICU_OK;
}

bool na_supported(uint32_t t, uint32_t &blck) {
    switch (t) {
        case T_F16: blck = 1; return true;
        case T_Q4_0: case T_Q5_0: case T_Q8_0: blck = 32; return true;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: blck = 256; return true;
        default: return false;
    }
}

}  // namespace

extern "C" int sicu_gemv_host_noalloc(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                                      const float *hx, float *hy, void *stream) {
    uint32_t blck = 1;
    if (!na_supported(wtype, blck))
        return report_error(SICU_ENOTSUP, "gemv_host_noalloc: unsupported weight type %u", wtype);
    if (n_in <= 0 || n_out < 0 || n_in % blck)
        return report_error(SICU_EINVAL, "gemv_host_noalloc: bad shape n_in=%lld n_out=%lld",
                            (long long)n_in, (long long)n_out);
    if (n_in > NA_MAX_IN || n_out > NA_MAX_OUT)
        return report_error(SICU_EINVAL,
                            "gemv_host_noalloc: n_in=%lld n_out=%lld exceed the fixed scratch "
                            "(at most %lld inputs and %lld outputs per call); use sicu_gemv_host",
                            (long long)n_in, (long long)n_out, (long long)NA_MAX_IN, (long long)NA_MAX_OUT);
    if (!hx || (n_out > 0 && (!dw || !hy))) return report_error(SICU_EINVAL, "gemv_host_noalloc: null pointer");
    if (n_out > 0 && (reinterpret_cast<uintptr_t>(dw) & 15))
        return report_error(SICU_EINVAL, "gemv_host_noalloc: weight pointer must be 16-byte aligned");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return na_cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return report_error(SICU_EINVAL, "gemv_host_noalloc: device %d out of range", dev);
    NaDev *d = nullptr;
    if (int rc = na_setup(dev, d)) return rc;

    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int *status = reinterpret_cast<int *>(d->scratch);
    float *dx = reinterpret_cast<float *>(d->scratch + NA_HDR);
    float *dy = dx + NA_MAX_IN;
    // the array keeps the previous call's contents: the status word must start at zero;
    // the activation and output regions are fully overwritten below
    if ((e = cudaMemsetAsync(status, 0, sizeof(int), st)) != cudaSuccess) return na_cuda_fail(e, "clear status");
    if ((e = cudaMemcpyAsync(dx, hx, (size_t)n_in * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return na_cuda_fail(e, "copy in");
    if (n_out > 0) {
        GemvLaunch L{};
        L.w = dw;
        L.xf = dx;
        L.y = dy;
        L.n_out = n_out;
        L.n_in = (int)n_in;
        L.nmat = 1;
        L.wm[0] = dw;
        L.ym[0] = dy;
        L.n_outm[0] = n_out;
        L.num_sms = d->sms;
        L.smem_limit = d->smem_optin;
        L.smem_per_sm = d->smem_per_sm;
        L.smem_reserved = d->smem_reserved;
        L.overlap = 0;
        L.device = dev;
        L.status = status;
        const int rc = (wtype == T_F16) ? launch_gemv_f16(L, st) : launch_gemv(wtype, L, st);
        if (rc == -1)
            return report_error(SICU_ENOTSUP, "gemv_host_noalloc: row of %lld elements does not fit shared memory",
                                (long long)n_in);
        if (rc == -3) return report_error(SICU_ENOTSUP, "gemv_host_noalloc: no kernel for weight type %u", wtype);
        if (rc != 0) return na_cuda_fail(cudaGetLastError(), "launch");
        if ((e = cudaMemcpyAsync(hy, dy, (size_t)n_out * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess)
            return na_cuda_fail(e, "copy out");
    }
    int flags = 0;
    if ((e = cudaMemcpyAsync(&flags, status, sizeof(int), cudaMemcpyDeviceToHost, st)) != cudaSuccess)
        return na_cuda_fail(e, "read status");
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return na_cuda_fail(e, "stream sync");
    if (flags) return report_error(SICU_EIO, "gemv_host_noalloc: kernel status %d (a bounded wait gave up)", flags);
    return SICU_OK;
}
