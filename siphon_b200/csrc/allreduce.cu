// Standalone all-reduce of a vector over the group, for partial sums that no
// matvec of the library produced. The row-split matvec runs the same steps
// inside its epilogue.
#include "allreduce.cuh"
#include "launch.h"

namespace sicu {
namespace {

constexpr int AR_THREADS = 256;

// One delivery of src: every thread sends its elements to every rank, then
// sums the same elements over the ranks into dst.
__global__ void __launch_bounds__(AR_THREADS) allreduce_kernel(const __grid_constant__ ArDev a, const float *src, float *dst,
                                                                int *status) {
    __shared__ unsigned s_e, s_ok;
    if (threadIdx.x == 0) {
        const ArState st = ar_load_state(a);
        if (st.broken) atomicOr(status, STATUS_AR_TIMEOUT);
        else ar_arrive(a, st.e);
        s_e = st.e;
        s_ok = st.broken ? 0u : 1u;
    }
    __syncthreads();
    const unsigned e = s_e;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (!s_ok) {
        for (int64_t i = first; i < a.len; i += stride) dst[i] = src[i];
        return;
    }
    for (int64_t i = first; i < a.len; i += stride) ar_send(a, e, i, src[i]);
    bool live = true;
    for (int64_t i = first; i < a.len; i += stride) dst[i] = ar_sum(a, e, i, status, live);
}

int grid_for(int64_t len, int num_sms) {
    const int64_t want = (len + AR_THREADS - 1) / AR_THREADS;
    return (int)(want < num_sms ? (want > 0 ? want : 1) : num_sms);
}

}  // namespace

int launch_allreduce(const ArDev &a, const float *src, float *dst, int *status, int num_sms, cudaStream_t st) {
    allreduce_kernel<<<grid_for(a.len, num_sms), AR_THREADS, 0, st>>>(a, src, dst, status);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
