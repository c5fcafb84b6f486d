// Activation quantizers, byte-identical with the reference:
//   Q8_K : src/kernels.c:561-595 (the only form the reference has)
//   Q8_0 : src/kernels_avx2.c:594-645 (the form x86 hosts dispatch to)
//   F16  : element-wise RNE narrowing (src/backend.c:19-27)
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace sicu {

// One warp quantizes one 256-element block into the raw 292-byte Q8_K layout
// (d f32 @0, qs int8 @4, bsums int16 @260). Lane L owns elements 8L..8L+7.
// x must be 16-byte aligned. An all-zero block writes d = 0, qs = 0 and
// bsums = 0 (the reference leaves bsums untouched there).
__device__ __forceinline__ void q8k_block_warp(const float *x, uint8_t *dst, int lane) {
    const float4 v0 = reinterpret_cast<const float4 *>(x)[2 * lane];
    const float4 v1 = reinterpret_cast<const float4 *>(x)[2 * lane + 1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    // first element of largest magnitude: strict '>' scan keeps the earliest,
    // NaN never compares greater
    float best = 0.0f;
    int bi = 256;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fabsf(v[i]);
        if (a > best) { best = a; bi = 8 * lane + i; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    uint32_t *qw = reinterpret_cast<uint32_t *>(dst + 4);
    int16_t *bs = reinterpret_cast<int16_t *>(dst + 260);
    if (!(best > 0.0f)) {
        qw[2 * lane] = 0u;
        qw[2 * lane + 1] = 0u;
        if (lane < 16) bs[lane] = 0;
        if (lane == 0) *reinterpret_cast<float *>(dst) = 0.0f;
        return;
    }
    float own = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) if ((bi & 7) == i) own = v[i];
    const float mx = __shfl_sync(0xffffffffu, own, bi >> 3);
    const float iscale = __fdiv_rn(-127.0f, mx);
    uint32_t packed[2] = {0u, 0u};
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int q;
        if (isnan(v[i])) {
            // the reference's magic-number rounding leaves a NaN's low payload bits
            q = (int)(__float_as_uint(v[i]) & 0x3fffffu);
        } else {
            q = __float2int_rn(__fmul_rn(iscale, v[i]));
        }
        q = q < 127 ? q : 127;
        sum += q;
        packed[i / 4] |= ((uint32_t)q & 0xffu) << (8 * (i & 3));
    }
    qw[2 * lane] = packed[0];
    qw[2 * lane + 1] = packed[1];
    const int pair = sum + __shfl_xor_sync(0xffffffffu, sum, 1);
    if ((lane & 1) == 0) bs[lane >> 1] = (int16_t)pair;
    if (lane == 0) *reinterpret_cast<float *>(dst) = __fdiv_rn(1.0f, iscale);
}

__device__ __forceinline__ float vmaxps(float a, float b) { return a > b ? a : b; }

__device__ __forceinline__ int sat8_rounded(float r) {
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) return -128;
    const int i = (int)r;
    return i > 127 ? 127 : (i < -128 ? -128 : i);
}

// One thread quantizes one 32-element block (AVX2 form): v in, f16 d and
// 32 int8 quants (8 little-endian words) out.
__device__ __forceinline__ void q8_0_block(const float *x, uint32_t &d16, uint32_t qw[8]) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float4 f = reinterpret_cast<const float4 *>(x)[k];
        v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
    }
    float lane[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float m = fabsf(v[i]);
        m = vmaxps(m, fabsf(v[8 + i]));
        m = vmaxps(m, fabsf(v[16 + i]));
        m = vmaxps(m, fabsf(v[24 + i]));
        lane[i] = m;
    }
    float q4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q4[i] = vmaxps(lane[4 + i], lane[i]);
    const float top = vmaxps(vmaxps(q4[0], q4[2]), vmaxps(q4[1], q4[3]));
    d16 = f2h(__fdiv_rn(top, 127.0f));
    const float id = (top != 0.0f) ? __fdiv_rn(127.0f, top) : 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t w = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int q = sat8_rounded(rintf(__fmul_rn(v[4 * k + b], id)));
            w |= ((uint32_t)q & 0xffu) << (8 * b);
        }
        qw[k] = w;
    }
}

// Fused prologue: quantize the f32 activation straight into the prepared
// shared-memory layout. `stage` is a 292-byte per-warp scratch in shared memory.
template <int ACT>
__device__ void quantize_into_act(const ActView av, const float *xf, int n_in, uint8_t *stage) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if constexpr (ACT == 3) {
        const int nblk = n_in / 32;
        for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
            uint32_t d16, qw[8];
            q8_0_block(xf + 32 * b, d16, qw);
            int s = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) s = dp4a_ss(qw[k], 0x01010101u, s);
            const int u = b >> 3, bi = b & 7;
            uint32_t *dst = reinterpret_cast<uint32_t *>(av.aq(u)) + bi * 8;
#pragma unroll
            for (int k = 0; k < 8; ++k) dst[k] = qw[k];
            av.ad(u)[bi] = h2f(d16);
            av.ax(u)[bi] = s;
        }
    } else {
        for (int u = warp; u < n_in / 256; u += nw) {
            q8k_block_warp(xf + 256 * u, stage, lane);
            __syncwarp();
            if (lane < 8) prep_piece<ACT>(av, stage, u, lane);
            __syncwarp();
        }
    }
}

}  // namespace sicu
