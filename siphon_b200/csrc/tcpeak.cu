// Tensor-core throughput probe: the dense MMA rate this GPU sustains for the
// two operand kinds the prefill design weighs, kind::f16 (what the prefill
// kernels issue: exact f16 scale x quant operands, f32 accumulation) and
// kind::i8 (int8 operands, s32 accumulation). It gives the measured int8
// denominator of the prefill roofline in place of a "2 x bf16" estimate. No
// counterpart in the reference, which has no tensor-core code.
//
// One CTA per SM (its dynamic shared memory keeps a second one off the SM):
// both operand tiles stay in shared memory (A: 128 rows x 128 bytes, B: 256
// rows x 128 bytes, K-major, 128-byte swizzle), two 256-column accumulators in
// tensor memory, and one thread issues rounds of 64 MMAs of M = 128, N = 256
// (K = 16 f16 or 32 int8 per MMA), committing each round to an mbarrier and
// waiting (bounded) for the round before the previous one, so at most two
// rounds are in flight. Operand values are small pseudo-random numbers so the
// datapath toggles as it would on real data; results are not read.
#include "siphon_cuda.h"
#include "tc.cuh"

namespace sicu {
int report_error(int code, const char *fmt, ...);

namespace {

constexpr int TCP_ITERS = 16;                       // iterations of 4 MMAs per round
constexpr int TCP_A = 128 * 128, TCP_B = 256 * 128;  // operand tile bytes
constexpr int TCP_SMEM = 160 * 1024;                 // > half an SM's shared memory: one CTA per SM

// Instruction descriptor for kind::i8: signed int8 A and B, s32 accumulation,
// both K-major: [4,6) D format (2 = s32), [7,10) A format (1 = signed 8-bit),
// [10,13) B format (1 = signed 8-bit), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__global__ void __launch_bounds__(128, 1) tc_peak_kernel(int i8, int rounds, int *status) {
    extern __shared__ uint8_t dsm[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint32_t tbase;
    const int tid = threadIdx.x;
    // int8 in [-8, 7]; f16 in [0.5, 1) (sign 0, exponent of 0.5, random mantissa)
    uint32_t *w = reinterpret_cast<uint32_t *>(sm);
    for (int i = tid; i < (TCP_A + TCP_B) / 4; i += blockDim.x) {
        uint32_t h = (uint32_t)i * 0x9e3779b9u + (uint32_t)blockIdx.x * 0x85ebca6bu;
        h ^= h >> 15;
        h *= 0x2c1b3c6du;
        h ^= h >> 12;
        w[i] = i8 ? (h & 0x0f0f0f0fu) - 0x08080808u : ((h & 0x03ff03ffu) | 0x38003800u);
    }
    if (tid < 32) tmem_alloc(smem_addr(&tbase), 512);
    if (tid == 0) {
        mbar_init(smem_addr(&bars[0]), 1);
        mbar_init(smem_addr(&bars[1]), 1);
        fence_mbar_init();
    }
    fence_proxy_async();   // the operands' generic writes, before the tensor cores read them
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
        const uint32_t idesc = i8 ? idesc_s8_s32(128, 256) : idesc_f16_f32(128, 256);
        const uint32_t aa = smem_addr(sm), ba = smem_addr(sm + TCP_A);
        bool ok = true;
        int r = 0;
        for (; r < rounds; ++r) {
            if (r >= 2 && !(ok = mbar_wait(smem_addr(&bars[r & 1]), (uint32_t)((r - 2) >> 1) & 1u))) break;
            for (int it = 0; it < TCP_ITERS; ++it) {
                const uint32_t d = tbase + (uint32_t)(it & 1) * 256u;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    // K step k: 32 bytes further into the 128-byte swizzle atom
                    const uint64_t ad = smem_desc(aa + 32u * k, 1024, SMEM_SWZ_128B);
                    const uint64_t bd = smem_desc(ba + 32u * k, 1024, SMEM_SWZ_128B);
                    const uint32_t acc = (it >= 2 || k > 0) ? 1u : 0u;
                    if (i8) tc_mma_i8(d, ad, bd, idesc, acc);
                    else tc_mma_f16(d, ad, bd, idesc, acc);
                }
            }
            tc_commit(smem_addr(&bars[r & 1]));
        }
        // the rounds still in flight (every issued round was committed)
        for (int q = r - 2 < 0 ? 0 : r - 2; q < r; ++q)
            if (!mbar_wait(smem_addr(&bars[q & 1]), (uint32_t)(q >> 1) & 1u)) ok = false;
        if (!ok) atomicOr(status, 1);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid < 32) tmem_dealloc(tbase, 512);
}

}  // namespace
}  // namespace sicu

using namespace sicu;

extern "C" int sicu_tc_peak(int kind, int rounds, int sms, float *ms_out, double *tflops_out) {
    if ((kind != SICU_TC_F16 && kind != SICU_TC_I8) || rounds < 1 || sms < 1 || !ms_out || !tflops_out)
        return report_error(SICU_EINVAL, "tc_peak: bad arguments");
    static bool attr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return report_error(SICU_EIO, "tc_peak: no device");
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(tc_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TCP_SMEM) != cudaSuccess)
            return report_error(SICU_EIO, "tc_peak: shared memory attribute");
        attr[dev] = true;
    }
    int *status = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = SICU_OK;
    if (cudaMalloc(&status, sizeof(int)) != cudaSuccess || cudaMemset(status, 0, sizeof(int)) != cudaSuccess ||
        cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
        rc = report_error(SICU_EIO, "tc_peak: set-up: %s", cudaGetErrorString(cudaGetLastError()));
    } else {
        const int i8 = kind == SICU_TC_I8 ? 1 : 0;
        cudaEventRecord(e0);
        tc_peak_kernel<<<sms, 128, TCP_SMEM>>>(i8, rounds, status);
        cudaEventRecord(e1);
        int flag = 0;
        float ms = 0.0f;
        cudaError_t e = cudaEventSynchronize(e1);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        if (e == cudaSuccess) e = cudaMemcpy(&flag, status, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            rc = report_error(SICU_EIO, "tc_peak: %s", cudaGetErrorString(e));
        } else if (flag) {
            rc = report_error(SICU_EIO, "tc_peak: a bounded wait gave up");
        } else {
            // per MMA: 128 x 256 x K multiply-adds, K = 16 (f16) or 32 (int8)
            const double macs = (double)sms * rounds * TCP_ITERS * 4 * 128.0 * 256.0 * (i8 ? 32.0 : 16.0);
            *ms_out = ms;
            *tflops_out = 2.0 * macs / (ms * 1e-3) / 1e12;
        }
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (status) cudaFree(status);
    return rc;
}
