// Standalone steps of the fused all-reduce group: deliver a vector that no
// matvec produced, or consume the group's sum into a vector (for work that is
// not a matvec, e.g. a residual add). The matvec kernel runs the same steps
// inside its prologue and epilogue.
#include "allreduce.cuh"
#include "launch.h"

namespace sicu {
namespace {

constexpr int AR_THREADS = 256;

__global__ void __launch_bounds__(AR_THREADS) ar_deliver_kernel(const ArDev a, const float *src, int *status) {
    __shared__ unsigned s_e;
    __shared__ int s_ok;
    if (threadIdx.x == 0) s_ok = ar_deliver_begin(a, status, s_e) ? 1 : 0;
    __syncthreads();
    if (!s_ok) return;
    const unsigned e = s_e;
    const int64_t n4 = a.len >> 2;
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = s4[i];
#pragma unroll
        for (int q = 0; q < AR_MAX; ++q)
            if (q < a.n) reinterpret_cast<float4 *>(ar_dst(a, q, e))[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) ar_deliver_arrive(a, e);
}

__global__ void __launch_bounds__(AR_THREADS) ar_reduce_kernel(const ArDev a, float *dst, int *status) {
    __shared__ unsigned s_e;
    if (threadIdx.x == 0) s_e = ar_consume_wait(a, status);
    __syncthreads();
    const int64_t n4 = a.len >> 2;
    const float4 *base = reinterpret_cast<const float4 *>(a.slot[a.rank] + (int64_t)((s_e - 1u) & 1u) * a.n * a.len);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 v = __ldcg(base + i);
        for (int r = 1; r < a.n; ++r) {
            const float4 w = __ldcg(base + r * n4 + i);
            v.x = __fadd_rn(v.x, w.x);
            v.y = __fadd_rn(v.y, w.y);
            v.z = __fadd_rn(v.z, w.z);
            v.w = __fadd_rn(v.w, w.w);
        }
        reinterpret_cast<float4 *>(dst)[i] = v;
    }
}

int grid_for(int64_t len, int num_sms) {
    const int64_t want = (len / 4 + AR_THREADS - 1) / AR_THREADS;
    return (int)(want < num_sms ? (want > 0 ? want : 1) : num_sms);
}

}  // namespace

int launch_ar_deliver(const ArDev &a, const float *src, int *status, int num_sms, cudaStream_t st) {
    ar_deliver_kernel<<<grid_for(a.len, num_sms), AR_THREADS, 0, st>>>(a, src, status);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_ar_reduce(const ArDev &a, float *dst, int *status, int num_sms, cudaStream_t st) {
    ar_reduce_kernel<<<grid_for(a.len, num_sms), AR_THREADS, 0, st>>>(a, dst, status);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
