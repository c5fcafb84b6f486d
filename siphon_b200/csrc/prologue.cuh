// The activation steps the reference's forward pass runs between two
// products, in its float order so results stay bit-identical:
//   RMS norm   src/engine.c:12-18 (rms_norm_mul) with the scale of
//              src/kernels.c:892-900 (si_rms_scale); the residual adds of
//              src/engine.c:369 and 379 come first
//   SwiGLU     src/engine.c:162-179 (swiglu_row): silu(x) * up, silu of
//              src/kernels.c:851-853 over the exp polynomial of
//              src/kernels.c:821-849
// Every float operation is an explicit round-to-nearest intrinsic, so the
// compiler contracts nothing into a multiply-add the reference does not have.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace sicu {

// exp(x) by ggml's vector exp polynomial (the form the reference transcribes
// to scalar code): n = round(x / ln2) through the 1.5 * 2^23 shifter, b = x -
// n ln2 with ln2 in two parts, p = b (c1 + b c2 + b^2 (c3 + b c4 + b^2 c5))
// evaluated as ((c5 b + c4) b^2 + (c3 b + c2)) b^2 + c1 b, and 2^n (1 + p)
// with 2^n built in the exponent field. |n| > 126 scales by two powers of two
// instead; |n| > 192 saturates to 0 or inf.
__device__ __forceinline__ float expf_ref(float x) {
    const float shifter = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, shifter);
    const float n = __fsub_rn(z, shifter);
    const float b = __fmaf_rn(-n, 0x1.7f7d1cp-20f, __fmaf_rn(-n, 0x1.62e4p-1f, x));
    const uint32_t e = __float_as_uint(z) << 23;
    const float k = __uint_as_float(e + 0x3f800000u);
    const float u = __fmul_rn(b, b);
    const float hi = __fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f);
    const float mid = __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f);
    const float lo = __fmul_rn(0x1.ffffecp-1f, b);
    const float p = __fmaf_rn(__fmaf_rn(hi, u, mid), u, lo);
    const float an = fabsf(n);
    if (!(an > 126.0f)) return __fmaf_rn(p, k, k);
    const uint32_t g = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = __uint_as_float(g + 0x7f000000u);
    if (an > 192.0f) return __fmul_rn(s1, s1);
    const float s2 = __uint_as_float(e - g);
    return __fmul_rn(__fmaf_rn(s2, p, s2), s1);
}

// x / (1 + exp(0 - x))
__device__ __forceinline__ float silu_ref(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, expf_ref(__fsub_rn(0.0f, x))));
}

// silu_ref as an out-of-line call, for the matvec epilogues: one call per
// output row when the epilogue is on, no silu code in the kernels' loops
static __device__ __noinline__ float silu_call(float x) { return silu_ref(x); }

__device__ __forceinline__ float4 ld_f4(const float *p, int64_t i4) { return reinterpret_cast<const float4 *>(p)[i4]; }

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Bytes of shared scratch the RMS scale needs: one double per warp and
// cluster rank (blocks of up to 8 warps, clusters of up to 8 CTAs) and the
// broadcast mean.
constexpr int RMS_SCRATCH = 8 * 64 + 16;

__device__ __forceinline__ double sq4(float4 v) {
    const double a = (double)__fmul_rn(v.x, v.x) + (double)__fmul_rn(v.y, v.y);
    const double b = (double)__fmul_rn(v.z, v.z) + (double)__fmul_rn(v.w, v.w);
    return a + b;
}

// The f32 mean of squares of h = x (+ res) over n floats the reference
// computes (src/kernels.c:892-896: f32 squares added in double in index
// order, the double mean rounded to f32), from S, the same squares added in
// any order. Adding n nonnegative doubles in any order gives the exact sum
// within a factor (1 +- gamma), gamma = (n-1) 2^-53 / (1 - (n-1) 2^-53), so S
// and the sequential sum s differ by at most 2 gamma / (1 - gamma) S < n 2^-52 S,
// and the reference's mean RN(s / n) lies within q (1 +- w) of q = S * (1/n)
// for w = n 2^-52 plus the roundings of 1/n, of q and of RN itself (each at
// most 2^-53 relative); w = n 2^-50 + 2^-49 covers them with room to spare.
// The ends of that interval, rounded outwards, are narrowed to f32
// (monotone): when they agree, the sequential sum gives the same f32 mean.
// Otherwise (a mean within about n 2^-50 of a point halfway between two
// floats: roughly one call in 10^5 on random data, every call whose mean is
// exactly halfway) the CTA's thread 0 adds the squares again in index order
// and divides as the reference does. Every thread of the CTA calls with the
// same S; inv_n = 1.0 / n; `out` is shared scratch.
__device__ __forceinline__ float rms_mean(double S, const float *x, const float *res, int n, double inv_n,
                                          float *out) {
    const double dn = (double)n;
    const double q = __dmul_rn(S, inv_n);
    const double w = dn * 0x1p-50 + 0x1p-49;
    const float lo = __double2float_rn(__dmul_rd(q, 1.0 - w));
    const float hi = __double2float_rn(__dmul_ru(q, 1.0 + w));
    if (lo == hi) return lo;
    // uniform across the CTA (same S everywhere); also every non-finite sum
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < n; ++i) {
            float h = x[i];
            if (res) h = __fadd_rn(h, res[i]);
            t = __dadd_rn(t, (double)__fmul_rn(h, h));
        }
        *out = __double2float_rn(__ddiv_rn(t, dn));
    }
    __syncthreads();
    return *out;
}

__device__ __forceinline__ float rms_scale_of(float mean, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

__device__ __forceinline__ double warp_sum(double s) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    return s;
}

// Sum over the CTA of each thread's s (every thread must call); red: 8
// doubles of shared scratch (blockDim <= 256).
__device__ __forceinline__ double cta_sum(double s, double *red) {
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    double c = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) c += red[w];
    return c;
}

// 1 / sqrtf(mean(h^2) + eps) for one row of h = x (+ res) (n a multiple of 4,
// rows 16-byte aligned) by one CTA on its own (blockDim <= 256; every thread
// calls); h_out, when given, receives h.
__device__ __forceinline__ float cta_rms_scale(const float *x, const float *res, float *h_out, int n, float eps,
                                               void *scratch) {
    double *red = reinterpret_cast<double *>(scratch);
    float *out = reinterpret_cast<float *>(red + 64);
    double s = 0.0;
    for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) {
        float4 v = ld_f4(x, i);
        if (res) v = add4(v, ld_f4(res, i));
        if (h_out) reinterpret_cast<float4 *>(h_out)[i] = v;
        s += sq4(v);
    }
    const double S = cta_sum(s, red);
    return rms_scale_of(rms_mean(S, x, res, n, 1.0 / (double)n, out), eps);
}

// Reads the activation the standalone step kernels consume, four floats at a
// time, with the step applied: x as is, the normed h, silu(x) * up or
// x * up. The scale of the norm is computed before the first read.
struct ActLoad {
    const float *x;
    ProDev pro;
    float scale;
    __device__ __forceinline__ float4 operator()(int64_t i4) const {
        float4 v = ld_f4(x, i4);
        if (pro.kind == PRO_RMS_NORM) {
            if (pro.res) v = add4(v, ld_f4(pro.res, i4));
            const float4 g = ld_f4(pro.g, i4);
            v.x = __fmul_rn(__fmul_rn(v.x, scale), g.x);
            v.y = __fmul_rn(__fmul_rn(v.y, scale), g.y);
            v.z = __fmul_rn(__fmul_rn(v.z, scale), g.z);
            v.w = __fmul_rn(__fmul_rn(v.w, scale), g.w);
        } else if (pro.kind == PRO_SWIGLU) {
            const float4 u = ld_f4(pro.up, i4);
            v.x = __fmul_rn(silu_ref(v.x), u.x);
            v.y = __fmul_rn(silu_ref(v.y), u.y);
            v.z = __fmul_rn(silu_ref(v.z), u.z);
            v.w = __fmul_rn(silu_ref(v.w), u.w);
        } else if (pro.kind == PRO_MUL) {
            const float4 u = ld_f4(pro.up, i4);
            v.x = __fmul_rn(v.x, u.x);
            v.y = __fmul_rn(v.y, u.y);
            v.z = __fmul_rn(v.z, u.z);
            v.w = __fmul_rn(v.w, u.w);
        }
        return v;
    }
};

}  // namespace sicu
