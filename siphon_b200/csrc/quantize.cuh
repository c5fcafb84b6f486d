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
// records this cluster rank owns (u % nrank == rank), writing each into every
// CTA of the cluster. K formats: eight lanes per 256-element block, lane j
// owning elements 32j..32j+31, so after one 3-step max reduction every lane
// emits its own piece. Classic formats: one thread per 32-element block.
template <int ACT>
__device__ void quantize_into_act(const ActView av, const float *xf, int n_in, uint32_t rank, uint32_t nrank) {
    const RecWriter wr{nrank};
    if constexpr (ACT == 3) {
        const int nblk = n_in / 32, nu = (nblk + 7) / 8;
        const int mine = (nu - (int)rank + (int)nrank - 1) / (int)nrank;
        for (int i = threadIdx.x; i < mine * 8; i += blockDim.x) {
            const int u = (int)rank + (int)nrank * (i >> 3), b = 8 * u + (i & 7);
            if (b >= nblk) continue;
            uint32_t d16, q[8];
            q8_0_block(xf + 32 * b, d16, q);
            int s = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) s = dp4a_ss(q[k], 0x01010101u, s);
            put_block(av, wr, u, i & 7, q, h2f(d16), s);
        }
    } else {
        const int nsb = n_in / 256;
        const int lane = threadIdx.x & 31, j = lane & 7;
        const unsigned gmask = 0xffu << (lane & 24);
        const int groups = blockDim.x >> 3;
        for (int u = (int)rank + (int)nrank * (threadIdx.x >> 3); u < nsb; u += (int)nrank * groups) {
            const float4 *src = reinterpret_cast<const float4 *>(xf + 256 * u + 32 * j);
            float v[32];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 f = src[k];
                v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
            }
            // first element of largest magnitude (strict '>' keeps the earliest)
            float best = 0.0f, bval = 0.0f;
            int bi = 256;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float a = fabsf(v[i]);
                if (a > best) { best = a; bval = v[i]; bi = 32 * j + i; }
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) {
                const float ob = __shfl_xor_sync(gmask, best, off, 8);
                const float ov = __shfl_xor_sync(gmask, bval, off, 8);
                const int oi = __shfl_xor_sync(gmask, bi, off, 8);
                if (ob > best || (ob == best && oi < bi)) { best = ob; bval = ov; bi = oi; }
            }
            uint32_t q[8];
            int s0 = 0, s1 = 0;
            float d = 0.0f;
            if (best > 0.0f) {
                const float iscale = __fdiv_rn(-127.0f, bval);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    uint32_t w = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const float x = v[4 * k + b];
                        int qq = isnan(x) ? (int)(__float_as_uint(x) & 0x3fffffu) : __float2int_rn(__fmul_rn(iscale, x));
                        qq = qq < 127 ? qq : 127;
                        if (k < 4) s0 += qq; else s1 += qq;
                        w |= ((uint32_t)qq & 0xffu) << (8 * b);
                    }
                    q[k] = w;
                }
                d = __fdiv_rn(1.0f, iscale);
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) q[k] = 0u;
            }
            put_piece<ACT>(av, wr, u, j, q, s0, s1, d);
        }
    }
}

}  // namespace sicu
