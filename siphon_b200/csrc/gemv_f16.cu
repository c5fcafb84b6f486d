// F16 weight rows (reference src/kernels.c:189-195): products of two halves are
// exact in f32 and the reference adds them into a double left to right. Here
// each warp adds its row's products into doubles in a tree; the double sums
// are exact whenever the reference's chain is (no partial sum needs more than
// 53 significant bits), so the final (float) matches it.
#include "common.cuh"
#include "launch.h"

namespace sicu {

namespace {

constexpr int F16_WARPS = 16;

__global__ void __launch_bounds__(F16_WARPS * 32) gemv_f16_kernel(const uint16_t *w, const uint16_t *xh,
                                                                  const float *xf, float *y, int64_t n_out,
                                                                  int n_in) {
    extern __shared__ __align__(16) float act[];
    for (int i = threadIdx.x; i < n_in; i += blockDim.x) act[i] = xf ? h2f(f2h(xf[i])) : h2f(xh[i]);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (n_in & 7) == 0;
    for (int64_t row = (int64_t)blockIdx.x * F16_WARPS + warp; row < n_out; row += (int64_t)gridDim.x * F16_WARPS) {
        const uint16_t *wr = w + row * n_in;
        double acc = 0.0;
        if (vec) {
            const uint4 *w4 = reinterpret_cast<const uint4 *>(wr);
            const int n8 = n_in >> 3;
#pragma unroll 4
            for (int i = lane; i < n8; i += 32) {
                const uint4 v = __ldg(w4 + i);
                const float4 a0 = reinterpret_cast<const float4 *>(act)[2 * i];
                const float4 a1 = reinterpret_cast<const float4 *>(act)[2 * i + 1];
                const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    acc += (double)__fmul_rn(h2f(hv[k] & 0xffffu), av[2 * k]);
                    acc += (double)__fmul_rn(h2f(hv[k] >> 16), av[2 * k + 1]);
                }
            }
        } else {
            for (int i = lane; i < n_in; i += 32) acc += (double)__fmul_rn(h2f(wr[i]), act[i]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) y[row] = __double2float_rn(acc);
    }
}

}  // namespace

int launch_gemv_f16(const GemvLaunch &L, cudaStream_t st) {
    const size_t smem = (size_t)L.n_in * sizeof(float);
    if (smem > (size_t)L.smem_limit) return -1;
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        cudaFuncSetAttribute(gemv_f16_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (cudaFuncSetAttribute(gemv_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_limit) != cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    int64_t grid = (L.n_out + F16_WARPS - 1) / F16_WARPS;
    if (grid > 2 * (int64_t)L.num_sms) grid = 2 * (int64_t)L.num_sms;
    if (grid < 1) grid = 1;
    gemv_f16_kernel<<<(unsigned)grid, F16_WARPS * 32, smem, st>>>(static_cast<const uint16_t *>(L.w),
                                                               static_cast<const uint16_t *>(L.xq), L.xf, L.y,
                                                               L.n_out, L.n_in);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
