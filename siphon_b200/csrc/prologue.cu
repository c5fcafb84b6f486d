// The activation steps on their own (f32 rows in, f32 rows out), for
// callers that do not fuse them into a product: prompts (m rows before the
// prefill product) and F16 weights.
#include "prologue.cuh"

namespace sicu {

namespace {

// one CTA per row: scale, then h * scale * g
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *x, const float *res, float *h_out, const float *g,
                                                       int n, float eps, float *y) {
    __shared__ __align__(16) uint8_t scratch[RMS_SCRATCH];
    const int64_t off = (int64_t)blockIdx.x * n;
    const float *xr = x + off;
    const float *rr = res ? res + off : nullptr;
    const float scale = cta_rms_scale(xr, rr, h_out ? h_out + off : nullptr, n, eps, scratch);
    ProDev pro;
    pro.kind = PRO_RMS_NORM;
    pro.g = g;
    pro.res = rr;
    const ActLoad ld{xr, pro, scale};
    float4 *yr = reinterpret_cast<float4 *>(y + off);
    for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) yr[i] = ld(i);
}

// silu(x) * up, or x * up (mul)
__global__ void __launch_bounds__(256) glu_kernel(const float *x, const float *up, int64_t n4, bool mul, float *y) {
    ProDev pro;
    pro.kind = mul ? PRO_MUL : PRO_SWIGLU;
    pro.up = up;
    const ActLoad ld{x, pro, 0.0f};
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x)
        reinterpret_cast<float4 *>(y)[i] = ld(i);
}

__global__ void __launch_bounds__(256) add_kernel(float *y, const float *b, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], b[i]);
}

// y_r += b for m rows of n floats: y[i] + b[i mod n], one f32 addition each
__global__ void __launch_bounds__(256) add_rows_kernel(float *y, const float *b, int64_t n, int64_t total) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], b[i % n]);
}

__global__ void __launch_bounds__(256) silu_kernel(float *y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = silu_ref(y[i]);
}

int grid_for(int64_t n) {
    int64_t blocks = (n + 255) / 256;
    return (int)(blocks > 4096 ? 4096 : blocks);
}

int launch_glu(const float *x, const float *up, int64_t n, bool mul, float *y, cudaStream_t st) {
    const int64_t n4 = n / 4;
    if (n4 <= 0) return 0;
    glu_kernel<<<grid_for(n4), 256, 0, st>>>(x, up, n4, mul, y);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace

int launch_rms_norm(const float *x, const float *res, float *h_out, const float *g, int64_t n, int64_t m, float eps,
                    float *y, cudaStream_t st) {
    if (m <= 0) return 0;
    rms_norm_kernel<<<(unsigned)m, 256, 0, st>>>(x, res, h_out, g, (int)n, eps, y);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_swiglu(const float *x, const float *up, int64_t n, int64_t m, float *y, cudaStream_t st) {
    return launch_glu(x, up, n * m, false, y, st);
}

int launch_mul(const float *x, const float *up, int64_t n, float *y, cudaStream_t st) {
    return launch_glu(x, up, n, true, y, st);
}

int launch_add_inplace(float *y, const float *b, int64_t n, cudaStream_t st) {
    if (n <= 0) return 0;
    add_kernel<<<grid_for(n), 256, 0, st>>>(y, b, n);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_add_rows(float *y, const float *b, int64_t n, int64_t m, cudaStream_t st) {
    if (n <= 0 || m <= 0) return 0;
    add_rows_kernel<<<grid_for(n * m), 256, 0, st>>>(y, b, n, n * m);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_silu_inplace(float *y, int64_t n, cudaStream_t st) {
    if (n <= 0) return 0;
    silu_kernel<<<grid_for(n), 256, 0, st>>>(y, n);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
