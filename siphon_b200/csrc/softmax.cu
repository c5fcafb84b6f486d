// Softmax over rows on the device, bit-identical with the reference's
// si_softmax (src/kernels.c:855-890) with the row maximum its attention code
// passes (src/engine.c:124-130): 8-element groups through the exp polynomial
// (expf_ref), each group's sum in the lane order of an 8-wide horizontal add
// added into a double, the n % 8 tail through libm's expf (restated below),
// then every element times (float)(1 / sum).
#include "prologue.cuh"

namespace sicu {

namespace {

// libm expf as this image's glibc computes it on hosts with FMA (its x86-64
// FMA build; the table-driven algorithm of ARM's optimized routines): x / ln2
// scaled by N = 32 and rounded to an integer k with the 1.5 * 2^52 shifter, the
// remainder r formed with one fused multiply-add, 2^(k/N) from a 32-entry table
// plus k's integer part in the exponent field, and 2^(r/N) by a degree-3
// polynomial, all in double, rounded to float once. Special cases as there:
// -inf -> 0, NaN -> x + x, overflow above 0x1.62e42ep6, 0 below -0x1.9fe368p6.
// Checked bit for bit against the host's expf on every float in
// [-0x1.9fe368p6, 0] (tests/test_softmax.py runs the same check on the host).
// kExp2Tab[i] = bits of 2^(i/32) rounded to the nearest double, minus i << 47.
__device__ const uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

__device__ __forceinline__ float expf_libm(float x) {
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= (__float_as_uint(88.0f) >> 20)) {
        if (ux == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8u) return __fadd_rn(x, x);
        if (x > 0x1.62e42ep6f) return __uint_as_float(0x7f800000u);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double invln2n = 0x1.71547652b82fep+0 * 32;
    const double shift = 0x1.8p+52;
    const double xd = (double)x;
    const double z = __dmul_rn(invln2n, xd);
    double kd = __dadd_rn(z, shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(invln2n, xd, -kd);
    uint64_t t = kExp2Tab[ki % 32];
    t += ki << 47;
    const double s = __longlong_as_double((long long)t);
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                 c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double p = __fma_rn(c0, r, c1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(c2, r, 1.0);
    y = __fma_rn(p, r2, y);
    return __double2float_rn(__dmul_rn(y, s));
}

// The sum of one 8-element group in the lane order of the reference's
// horizontal add: ((v4 + v0) + (v6 + v2)) + ((v5 + v1) + (v7 + v3)).
__device__ __forceinline__ float group_sum(const float v[8]) {
    const float s0 = __fadd_rn(v[4], v[0]), s1 = __fadd_rn(v[5], v[1]);
    const float s2 = __fadd_rn(v[6], v[2]), s3 = __fadd_rn(v[7], v[3]);
    return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}

// One CTA per row (blockDim 256). The reference adds the group sums and then
// the tail values into a double in index order; the CTA adds them in
// parallel. As for the RMS norm's mean, the terms are nonnegative, so any
// order lies within nt 2^-52 of the sequential sum (nt terms), and
// (float)(1 / sum) is decided when both ends of the widened interval around
// 1 / S narrow to the same float (1 / s is monotone); otherwise thread 0
// redoes the sum in the reference's order from the stored values.
// The softmax of one row by one CTA (every thread calls; blockDim <= 256;
// xr and yr may be the same row, in global or shared memory).
__device__ void softmax_row(const float *xr, float *yr, int n) {
    __shared__ double red[8];
    __shared__ float bmax[8];
    __shared__ float out[2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    // the row maximum: the largest element, NaNs never selected, -inf when
    // there is none (src/engine.c:124-128)
    float mx = -__int_as_float(0x7f800000);
    for (int i = tid; i < n; i += blockDim.x) {
        const float v = xr[i];
        if (v > mx) mx = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, mx, o);
        if (v > mx) mx = v;
    }
    if (lane == 0) bmax[warp] = mx;
    __syncthreads();
    mx = bmax[0];
    for (int w = 1; w < nw; ++w)
        if (bmax[w] > mx) mx = bmax[w];
    const int ng = n / 8, body = 8 * ng;
    double s = 0.0;
    for (int g = tid; g < ng; g += blockDim.x) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = expf_ref(__fsub_rn(xr[8 * g + k], mx));
#pragma unroll
        for (int k = 0; k < 8; ++k) yr[8 * g + k] = v[k];
        s += (double)group_sum(v);
    }
    for (int i = body + tid; i < n; i += blockDim.x) {
        const float v = expf_libm(__fsub_rn(xr[i], mx));
        yr[i] = v;
        s += (double)v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int w = 0; w < nw; ++w) S += red[w];
        const double nt = (double)(ng + (n - body));
        const double q = __ddiv_rn(1.0, S);
        const double w = nt * 0x1p-50 + 0x1p-49;
        const float lo = __double2float_rn(__dmul_rd(q, 1.0 - w));
        const float hi = __double2float_rn(__dmul_ru(q, 1.0 + w));
        float scale = lo;
        if (!(lo == hi)) {
            double t = 0.0;
            for (int g = 0; g < ng; ++g) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = yr[8 * g + k];
                t = __dadd_rn(t, (double)group_sum(v));
            }
            for (int i = body; i < n; ++i) t = __dadd_rn(t, (double)yr[i]);
            scale = __double2float_rn(__ddiv_rn(1.0, t));
        }
        out[0] = scale;
    }
    __syncthreads();
    const float scale = out[0];
    for (int i = tid; i < n; i += blockDim.x) yr[i] = __fmul_rn(yr[i], scale);
    __syncthreads();
}

__global__ void __launch_bounds__(256) softmax_kernel(const float *x, float *y, int n) {
    const int64_t off = (int64_t)blockIdx.x * n;
    softmax_row(x + off, y + off, n);
}

// Eight f16 values x[0..7]: one 16-byte load when vec (x 16-byte aligned),
// else eight 2-byte loads; the same bits either way. Lanes of a warp read
// rows a whole row apart, so the wide load cuts the cache wavefronts of a
// chunk eightfold.
__device__ __forceinline__ void ld_h8(const uint16_t *x, bool vec, uint16_t a[8]) {
    if (vec) {
        const uint4 u = *reinterpret_cast<const uint4 *>(x);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a[2 * k] = (uint16_t)(w[k] & 0xffffu);
            a[2 * k + 1] = (uint16_t)(w[k] >> 16);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = x[k];
    }
}

// ---- exactly parallel f16 dots ------------------------------------------------
// The reference adds the exact f32 products of two f16 vectors into a double
// in index order. Each product of f16 values a, b is a multiple of
// 2^(qa + qb), q the weight of a value's last mantissa bit (2^-24 for the
// smallest), so every partial sum is a multiple of 2^(qmin_a + qmin_b); a
// double holds every such multiple below 2^(53 + qmin_a + qmin_b) exactly.
// When sum |a_i b_i| <= max|a| * sum|b| stays below that, no addition rounds
// in any order, and a parallel sum gives the sequential sum's bits. The value
// dots below sum in parallel, check that bound for the head afterwards
// (max|a| over everything they read, sum|b| and qmin_b of the fixed vector)
// and redo the head sequentially when it fails.

// weight of the last mantissa bit of a finite nonzero f16, as a power of 2
__device__ __forceinline__ int h_quantum(uint32_t b) {
    const int e = (int)((b >> 10) & 31u);
    return e ? e - 25 : -24;
}

// CTA-wide reductions through shared memory (every thread calls)
__device__ __forceinline__ uint32_t cta_max_u32(uint32_t v, uint32_t *scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) *scratch = 0u;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) atomicMax(scratch, v);
    __syncthreads();
    const uint32_t r = *scratch;
    __syncthreads();
    return r;
}

// sum |x_i| (exact in double for f16 values) and the smallest last-bit
// weight among the nonzero ones (+1000 when all are zero) of n f16 values
__device__ __forceinline__ void h_abs_sum_qmin(const uint16_t *x, int n, double *sum_out, int *qmin_out,
                                               double *dscratch, int *iscratch) {
    double s = 0.0;
    int qm = 1000;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t b = x[i] & 0x7fffu;
        s += (double)h2f(b);
        if (b) qm = min(qm, h_quantum(b));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        qm = min(qm, __shfl_xor_sync(0xffffffffu, qm, o));
    }
    if (threadIdx.x == 0) {
        *dscratch = 0.0;
        *iscratch = 1000;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(dscratch, s);
        atomicMin(iscratch, qm);
    }
    __syncthreads();
    *sum_out = *dscratch;
    *qmin_out = *iscratch;
    __syncthreads();
}

// true when max|a| (as f16 bits) times sum|b| stays below 2^(29 + qmin_b):
// the parallel sums are exact (qmin_a >= -24)
__device__ __forceinline__ bool dots_exact(uint32_t amax_bits, double bsum, int bqmin) {
    if (amax_bits >= 0x7c00u || !(bsum < 1e300)) return false;
    if (bqmin >= 1000) return true;   // b all zero: every product is 0
    return __dmul_ru((double)h2f(amax_bits), bsum) < ldexp(1.0, 29 + bqmin);
}

// 64 f16 values x[0..63] into eight 16-byte registers (x 16-byte aligned):
// the eight loads are all in flight before any is used
__device__ __forceinline__ void ld_h64(const uint16_t *x, uint4 r[8]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = reinterpret_cast<const uint4 *>(x)[k];
}
__device__ __forceinline__ uint32_t h_of(const uint4 r[8], int i) {
    const uint4 v = r[i >> 3];
    const uint32_t w = ((i >> 1) & 3) == 0 ? v.x : ((i >> 1) & 3) == 1 ? v.y : ((i >> 1) & 3) == 2 ? v.z : v.w;
    return (i & 1) ? (w >> 16) : (w & 0xffffu);
}

// Scores of positions 0..n_score-1 (row j of K at kh + j * hd; the row of
// position `own` from krow_own when not null), times ks, into sc; q16 the
// head's query as f16 in shared memory. Each position's dot is the
// reference's sequential double sum (src/kernels.c:189-195, index order); a
// thread runs two positions' chains side by side, the eight loads of each
// row's chunk issued before their additions. (A parallel sum, checked against
// an exactness bound afterwards, measured no faster: both are bounded by the
// f32 -> f64 widening of every product, and the bound failed for typical
// queries, whose smallest components have small last-bit weights.)
__device__ void head_scores(const uint16_t *kh, const uint16_t *krow_own, int own, const uint16_t *q16, int hd,
                            int n_score, float ks, float *sc) {
    const int nt = blockDim.x;
    const bool vec = (reinterpret_cast<uintptr_t>(kh) & 15) == 0 && (hd & 7) == 0 &&
                     (!krow_own || (reinterpret_cast<uintptr_t>(krow_own) & 15) == 0);
    for (int j = threadIdx.x; j < n_score; j += 2 * nt) {
        const int j2 = j + nt;
        const bool two = j2 < n_score;
        const uint16_t *ra = (krow_own && j == own) ? krow_own : kh + (int64_t)j * hd;
        const uint16_t *rb = two ? ((krow_own && j2 == own) ? krow_own : kh + (int64_t)j2 * hd) : ra;
        double a = 0.0, b = 0.0;
        int d = 0;
        if (vec) {
            for (; d + 8 <= hd; d += 8) {
                uint16_t xa[8], xb[8];
                ld_h8(ra + d, true, xa);
                ld_h8(rb + d, true, xb);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float qv = h2f(q16[d + k]);
                    a = __dadd_rn(a, (double)__fmul_rn(h2f(xa[k]), qv));
                    b = __dadd_rn(b, (double)__fmul_rn(h2f(xb[k]), qv));
                }
            }
        }
        for (; d < hd; ++d) {
            const float qv = h2f(q16[d]);
            a = __dadd_rn(a, (double)__fmul_rn(h2f(ra[d]), qv));
            b = __dadd_rn(b, (double)__fmul_rn(h2f(rb[d]), qv));
        }
        sc[j] = __fmul_rn(__double2float_rn(a), ks);
        if (two) sc[j2] = __fmul_rn(__double2float_rn(b), ks);
    }
    __syncthreads();
}

// out[c] = the f16 dot of V row c (vh + c * n_ctx, positions 0..n_score-1;
// the value of position `own` from v_own[c] when v_own is not null) with the
// probabilities p16, for c < hd. Threads split each row's positions into
// blockDim / hd segments summed in parallel (two accumulators each),
// sequential when the exactness bound fails. part: blockDim doubles.
__device__ void head_values(const uint16_t *vh, int64_t n_ctx, const uint16_t *v_own, int own, const uint16_t *p16,
                            int hd, int n_score, float *out, double *part, double *dscratch, int *iscratch,
                            uint32_t *uscratch) {
    double psum;
    int pqmin;
    h_abs_sum_qmin(p16, n_score, &psum, &pqmin, dscratch, iscratch);
    const int segs = hd <= (int)blockDim.x ? (int)blockDim.x / hd : 1;
    const int len = ((n_score + segs - 1) / segs + 7) & ~7;
    uint32_t vmax = 0;
    for (int task = threadIdx.x; task < hd * segs; task += blockDim.x) {
        const int c = task % hd, sg = task / hd;
        const uint16_t *row = vh + (int64_t)c * n_ctx;
        const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
        const int j0 = sg * len, j1 = min(n_score, j0 + len);
        double a[2] = {0.0, 0.0};
        int j = j0;
        if (vec) {
            // 64 positions at a time, every load in flight before use
            for (; j + 64 <= j1; j += 64) {
                uint4 x[8];
                ld_h64(row + j, x);
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    const uint32_t xv = (v_own && j + k == own) ? (uint32_t)v_own[c] : h_of(x, k);
                    vmax = max(vmax, xv & 0x7fffu);
                    a[k & 1] = __dadd_rn(a[k & 1], (double)__fmul_rn(h2f(xv), h2f(p16[j + k])));
                }
            }
        }
        for (; j + 8 <= j1; j += 8) {
            uint16_t x[8];
            if (v_own && own >= j && own < j + 8) {
#pragma unroll
                for (int k = 0; k < 8; ++k) x[k] = (j + k == own) ? v_own[c] : row[j + k];
            } else {
                ld_h8(row + j, vec, x);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                vmax = max(vmax, (uint32_t)x[k] & 0x7fffu);
                a[k & 1] = __dadd_rn(a[k & 1], (double)__fmul_rn(h2f(x[k]), h2f(p16[j + k])));
            }
        }
        for (; j < j1; ++j) {
            const uint16_t x = (v_own && j == own) ? v_own[c] : row[j];
            vmax = max(vmax, (uint32_t)x & 0x7fffu);
            a[0] = __dadd_rn(a[0], (double)__fmul_rn(h2f(x), h2f(p16[j])));
        }
        part[task] = __dadd_rn(a[0], a[1]);
    }
    vmax = cta_max_u32(vmax, uscratch);   // also orders the partials before their use
    if (dots_exact(vmax, psum, pqmin)) {
        for (int c = threadIdx.x; c < hd; c += blockDim.x) {
            double sum = part[c];
            for (int sg = 1; sg < segs; ++sg) sum = __dadd_rn(sum, part[sg * hd + c]);
            out[c] = __double2float_rn(sum);
        }
    } else {
        for (int c = threadIdx.x; c < hd; c += blockDim.x) {
            const uint16_t *row = vh + (int64_t)c * n_ctx;
            double sum = 0.0;
            for (int j = 0; j < n_score; ++j) {
                const uint16_t x = (v_own && j == own) ? v_own[c] : row[j];
                sum = __dadd_rn(sum, (double)__fmul_rn(h2f(x), h2f(p16[j])));
            }
            out[c] = __double2float_rn(sum);
        }
    }
}

// One query head per CTA (src/engine.c:90-147, attn_head, on the scalar dot
// path): q as f16, a score per cached position 0..pos against the head's K
// rows, times kq_scale, the row's softmax, the probabilities as f16, and per
// channel the f16 dot of the head's transposed V row with them. Dynamic
// shared memory: n_score floats (scores, then probabilities) and n_score
// halves.
__global__ void __launch_bounds__(256) attention_kernel(const float *q, const uint16_t *kc, const uint16_t *vc,
                                                        int n_head, int gqa, int hd, int n_ctx, int n_score,
                                                        float ks, float *out) {
    extern __shared__ __align__(16) uint8_t sm[];
    float *sc = reinterpret_cast<float *>(sm);
    uint16_t *p16 = reinterpret_cast<uint16_t *>(sc + n_score);
    __shared__ __align__(16) uint16_t q16[1024];
    __shared__ double part[1024], dscr;
    __shared__ int iscr;
    __shared__ uint32_t uscr;
    const int h = blockIdx.x, hk = h / gqa;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) q16[d] = (uint16_t)f2h(q[(int64_t)h * hd + d]);
    __syncthreads();
    const uint16_t *kh = kc + (int64_t)hk * n_ctx * hd;
    const uint16_t *vh = vc + (int64_t)hk * hd * n_ctx;
    head_scores(kh, nullptr, -1, q16, hd, n_score, ks, sc);
    softmax_row(sc, sc, n_score);
    for (int j = threadIdx.x; j < n_score; j += blockDim.x) p16[j] = (uint16_t)f2h(sc[j]);
    __syncthreads();
    head_values(vh, n_ctx, nullptr, -1, p16, hd, n_score, out + (int64_t)h * hd, part, &dscr, &iscr, &uscr);
}

// The attention step of one layer and position in one launch, one CTA per
// query head: the head's q and its KV head's k rotated (the rotation of
// rope_kernel) in shared memory, this position's K and V stored into the
// caches (by the first CTA of each KV group; the others only read earlier
// positions), the scores of positions 0..pos (this position's from the f16 k
// in shared memory, the same bits the cache holds), softmax, f16
// probabilities and the value dots (this position's V from shared memory);
// the scores as sequential chains in the reference's order (head_scores), the
// value dots summed in parallel where that is exact (head_values).
// Same results as rope_kernel + kv_store_kernel + attention_kernel. Launched
// after the producing matvec has finished (launched early behind it, the
// decode step measured slower: 3.0 ms per TinyLlama-shape token against 1.86),
// it lets the next matvec launch early and stream its weights meanwhile.
__global__ void __launch_bounds__(256) attention_step_kernel(const float *q, const float *k, const float *v,
                                                             uint16_t *kc, uint16_t *vc, const float *cs,
                                                             const float *sn, int n_head, int gqa, int hd, int n_rot,
                                                             int neox, int n_ctx, int pos, float ks, float *out) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(16) uint8_t sm[];
    const int n_score = pos + 1;
    float *sc = reinterpret_cast<float *>(sm);
    uint16_t *p16 = reinterpret_cast<uint16_t *>(sc + n_score);
    __shared__ __align__(16) float qf[1024], kf[1024];
    __shared__ __align__(16) uint16_t q16[1024], k16[1024], v16[1024];
    __shared__ double part[1024], dscr;
    __shared__ int iscr;
    __shared__ uint32_t uscr;
    const int h = blockIdx.x, hk = h / gqa, tid = threadIdx.x;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int d = tid; d < hd; d += blockDim.x) {
        qf[d] = q[(int64_t)h * hd + d];
        kf[d] = k[(int64_t)hk * hd + d];
        v16[d] = (uint16_t)f2h(v[(int64_t)hk * hd + d]);
    }
    __syncthreads();
    const int np = n_rot / 2;
    for (int j = tid; j < np; j += blockDim.x) {
        const float c = cs[j], s = sn[j];
        const int i0 = neox ? j : 2 * j, i1 = neox ? j + hd / 2 : 2 * j + 1;
        const float q0 = qf[i0], q1 = qf[i1], k0 = kf[i0], k1 = kf[i1];
        if (!neox) {
            qf[i0] = __fmaf_rn(q0, c, -__fmul_rn(q1, s));
            qf[i1] = __fmaf_rn(q0, s, __fmul_rn(q1, c));
            kf[i0] = __fmaf_rn(k0, c, -__fmul_rn(k1, s));
            kf[i1] = __fmaf_rn(k0, s, __fmul_rn(k1, c));
        } else {
            qf[i0] = __fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s));
            qf[i1] = __fadd_rn(__fmul_rn(q0, s), __fmul_rn(q1, c));
            kf[i0] = __fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s));
            kf[i1] = __fadd_rn(__fmul_rn(k0, s), __fmul_rn(k1, c));
        }
    }
    __syncthreads();
    uint16_t *kh = kc + (int64_t)hk * n_ctx * hd;
    uint16_t *vh = vc + (int64_t)hk * hd * n_ctx;
    const bool writer = (h % gqa) == 0;
    for (int d = tid; d < hd; d += blockDim.x) {
        q16[d] = (uint16_t)f2h(qf[d]);
        k16[d] = (uint16_t)f2h(kf[d]);
        if (writer) {
            kh[(int64_t)pos * hd + d] = k16[d];
            vh[(int64_t)d * n_ctx + pos] = v16[d];
        }
    }
    __syncthreads();
    // scores and value dots: this position's k and v from shared memory (the
    // same bits the cache holds), positions 0..pos-1 from the cache
    head_scores(kh, k16, pos, q16, hd, n_score, ks, sc);
    softmax_row(sc, sc, n_score);
    for (int j = tid; j < n_score; j += blockDim.x) p16[j] = (uint16_t)f2h(sc[j]);
    __syncthreads();
    head_values(vh, n_ctx, v16, pos, p16, hd, n_score, out + (int64_t)h * hd, part, &dscr, &iscr, &uscr);
}

// RoPE in place on n_heads heads of hd floats (src/engine.c:42-75): pairs
// (2j, 2j+1) rotated as fma(x0, c, -(x1 * s)), fma(x0, s, x1 * c) (the
// interleaved form), or (j, j + hd/2) with plain products and sums (neox);
// channels from n_rot on unchanged.
__global__ void rope_kernel(float *x, int n_heads, int hd, int n_rot, const float *cs, const float *sn, int neox) {
    const int np = n_rot / 2;
    const int64_t total = (int64_t)n_heads * np;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int hh = (int)(t / np), j = (int)(t % np);
        float *v = x + (int64_t)hh * hd;
        const float c = cs[j], s = sn[j];
        if (!neox) {
            const float x0 = v[2 * j], x1 = v[2 * j + 1];
            v[2 * j] = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
            v[2 * j + 1] = __fmaf_rn(x0, s, __fmul_rn(x1, c));
        } else {
            const int half = hd / 2;
            const float x0 = v[j], x1 = v[j + half];
            v[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            v[j + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
    }
}

// K and V of one position into the f16 caches (src/engine.c:344-362): K
// position-major [h][n_ctx][hd], V transposed [h][hd][n_ctx].
__global__ void kv_store_kernel(const float *k, const float *v, uint16_t *kc, uint16_t *vc, int n_head_kv, int hd,
                                int n_ctx, int pos) {
    const int total = n_head_kv * hd;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int hh = t / hd, d = t % hd;
        kc[((int64_t)hh * n_ctx + pos) * hd + d] = (uint16_t)f2h(k[t]);
        vc[((int64_t)hh * hd + d) * n_ctx + pos] = (uint16_t)f2h(v[t]);
    }
}

// ---- a prompt's attention: m consecutive positions in two launches -------------
// The engine runs a prompt one token at a time (src/cmd_run.c:276): for token
// t at position pos0 + t, RoPE of its q and k, k and v stored at that
// position, then each head's attention over positions 0..pos0 + t
// (src/engine.c:336-366, 90-147). Here every token's k and v are rotated and
// stored first (one CTA per token), then one CTA per (head, token) rotates its
// q and attends over its prefix, which by then holds exactly what the
// token-serial engine's cache held at that token: the same computations, the
// same bits, m tokens at once.

// channel d of one head's vector after RoPE with tables c, s (n_rot / 2 pairs),
// the rotation attention_step_kernel applies
__device__ __forceinline__ float rope_channel(const float *x, int d, int hd, int n_rot, int neox, const float *c,
                                              const float *s) {
    if (!neox) {
        const int j = d >> 1;
        if (2 * j >= n_rot) return x[d];
        const float x0 = x[2 * j], x1 = x[2 * j + 1];
        return (d & 1) ? __fmaf_rn(x0, s[j], __fmul_rn(x1, c[j])) : __fmaf_rn(x0, c[j], -__fmul_rn(x1, s[j]));
    }
    const int half = hd / 2, j = d < half ? d : d - half;
    if (j >= n_rot / 2) return x[d];
    const float x0 = x[j], x1 = x[j + half];
    return d < half ? __fsub_rn(__fmul_rn(x0, c[j]), __fmul_rn(x1, s[j]))
                    : __fadd_rn(__fmul_rn(x0, s[j]), __fmul_rn(x1, c[j]));
}

// token t = blockIdx.x: its k rotated and stored (f16) at position pos0 + t
// of the K cache, its v stored at that position of the V cache
__global__ void prompt_kv_store_kernel(const float *k, const float *v, uint16_t *kc, uint16_t *vc, const float *cs,
                                       const float *sn, int n_head_kv, int hd, int n_rot, int neox, int n_ctx,
                                       int pos0) {
    const int t = blockIdx.x, pos = pos0 + t;
    const float *kt = k + (int64_t)t * n_head_kv * hd, *vt = v + (int64_t)t * n_head_kv * hd;
    const float *c = cs + (int64_t)t * (n_rot / 2), *s = sn + (int64_t)t * (n_rot / 2);
    for (int i = threadIdx.x; i < n_head_kv * hd; i += blockDim.x) {
        const int hh = i / hd, d = i - hh * hd;
        kc[((int64_t)hh * n_ctx + pos) * hd + d] = (uint16_t)f2h(rope_channel(kt + (int64_t)hh * hd, d, hd, n_rot,
                                                                               neox, c, s));
        vc[((int64_t)hh * hd + d) * n_ctx + pos] = (uint16_t)f2h(vt[i]);
    }
}

// query head h = blockIdx.x of token t = blockIdx.y: its q rotated and made
// f16, then the scores, softmax and value dots of attention_step_kernel over
// positions 0..pos0 + t of the caches. Dynamic shared memory: (pos0 + m) x 6
// bytes + 16.
__global__ void __launch_bounds__(256) prompt_attention_kernel(const float *q, const uint16_t *kc, const uint16_t *vc,
                                                               const float *cs, const float *sn, int n_head, int gqa,
                                                               int hd, int n_rot, int neox, int n_ctx, int pos0,
                                                               float ks, float *out) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int h = blockIdx.x, t = blockIdx.y, hk = h / gqa, tid = threadIdx.x;
    const int n_score = pos0 + t + 1;
    float *sc = reinterpret_cast<float *>(sm);
    uint16_t *p16 = reinterpret_cast<uint16_t *>(sc + n_score);
    __shared__ __align__(16) float qf[1024];
    __shared__ __align__(16) uint16_t q16[1024];
    __shared__ double part[1024], dscr;
    __shared__ int iscr;
    __shared__ uint32_t uscr;
    const float *qt = q + ((int64_t)t * n_head + h) * hd;
    for (int d = tid; d < hd; d += blockDim.x) qf[d] = qt[d];
    __syncthreads();
    const float *c = cs + (int64_t)t * (n_rot / 2), *s = sn + (int64_t)t * (n_rot / 2);
    for (int d = tid; d < hd; d += blockDim.x) q16[d] = (uint16_t)f2h(rope_channel(qf, d, hd, n_rot, neox, c, s));
    __syncthreads();
    const uint16_t *kh = kc + (int64_t)hk * n_ctx * hd;
    const uint16_t *vh = vc + (int64_t)hk * hd * n_ctx;
    head_scores(kh, nullptr, -1, q16, hd, n_score, ks, sc);
    softmax_row(sc, sc, n_score);
    for (int j = tid; j < n_score; j += blockDim.x) p16[j] = (uint16_t)f2h(sc[j]);
    __syncthreads();
    head_values(vh, n_ctx, nullptr, -1, p16, hd, n_score, out + ((int64_t)t * n_head + h) * hd, part, &dscr, &iscr,
                &uscr);
}

// ---- the prompt's attention per KV group ---------------------------------------
// The product of two f16 values is exact in f32 (22 significant bits) and in
// double, so the reference's s += (double)(a * b) is fma(a, b, s) with a and
// b widened to double: one rounding either way, the same bits. Widening each
// f16 once and sharing it across the query heads of a KV group replaces the
// per-product f32 -> f64 conversion (the bound of the per-head kernel) by
// double fmas.

// an f16 value as a double, exactly, with integer operations only
// (subnormals normalised, infinities and NaNs kept)
__device__ __forceinline__ double h2d_exact(uint32_t b) {
    const uint32_t s = (b & 0x8000u) << 16, e = (b >> 10) & 31u, m = b & 1023u;
    uint32_t hi;
    if (e == 31u) {
        hi = s | 0x7ff00000u | (m << 10);
    } else if (e) {
        hi = s | ((e + 1008u) << 20) | (m << 10);
    } else if (m) {
        const int p = 31 - __clz((int)m);          // leading bit of m, 0..9
        hi = s | ((uint32_t)(p + 999) << 20) | (((m << (10 - p)) & 1023u) << 10);
    } else {
        hi = s;
    }
    return __hiloint2double((int)hi, 0);
}

// softmax_row by one warp (every lane calls; xr and yr may be the same row):
// the same per-element arithmetic, the row's sum reduced across the lanes and
// decided (or redone in the reference's order) by lane 0, as softmax_row does
// across its CTA
__device__ void softmax_row_warp(const float *xr, float *yr, int n) {
    const int lane = threadIdx.x & 31;
    float mx = -__int_as_float(0x7f800000);
    for (int i = lane; i < n; i += 32) {
        const float v = xr[i];
        if (v > mx) mx = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, mx, o);
        if (v > mx) mx = v;
    }
    const int ng = n / 8, body = 8 * ng;
    double s = 0.0;
    for (int g = lane; g < ng; g += 32) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = expf_ref(__fsub_rn(xr[8 * g + k], mx));
#pragma unroll
        for (int k = 0; k < 8; ++k) yr[8 * g + k] = v[k];
        s += (double)group_sum(v);
    }
    for (int i = body + lane; i < n; i += 32) {
        const float v = expf_libm(__fsub_rn(xr[i], mx));
        yr[i] = v;
        s += (double)v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    __syncwarp();
    float scale = 0.0f;
    if (lane == 0) {
        const double nt = (double)(ng + (n - body));
        const double q = __ddiv_rn(1.0, s);
        const double w = nt * 0x1p-50 + 0x1p-49;
        const float lo = __double2float_rn(__dmul_rd(q, 1.0 - w));
        const float hi = __double2float_rn(__dmul_ru(q, 1.0 + w));
        scale = lo;
        if (!(lo == hi)) {
            double t = 0.0;
            for (int g = 0; g < ng; ++g) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = yr[8 * g + k];
                t = __dadd_rn(t, (double)group_sum(v));
            }
            for (int i = body; i < n; ++i) t = __dadd_rn(t, (double)yr[i]);
            scale = __double2float_rn(__ddiv_rn(1.0, t));
        }
    }
    scale = __shfl_sync(0xffffffffu, scale, 0);
    for (int i = lane; i < n; i += 32) yr[i] = __fmul_rn(yr[i], scale);
    __syncwarp();
}

constexpr int PA_CHUNK = 64;   // positions whose probabilities are widened at a time
constexpr int PA_GROUP_SMEM_MAX = 200 * 1024;

// KV head hk = blockIdx.x, token t = blockIdx.y, its G query heads at once
// (256 threads): the queries rotated, made f16 and widened to double in
// shared memory; a thread per position, its K row against all G queries
// (G fma chains, in index order); one warp per head for the softmax;
// the value dots as fma chains over positions in index order, a thread per
// (channel, HPT heads). Dynamic shared memory: pa_group_smem.
template <int G>
__global__ void __launch_bounds__(256) prompt_attention_group_kernel(const float *q, const uint16_t *kc,
                                                                     const uint16_t *vc, const float *cs,
                                                                     const float *sn, int n_head, int hd, int n_rot,
                                                                     int neox, int n_ctx, int pos0, int ns_max,
                                                                     float ks, float *out) {
    extern __shared__ __align__(16) uint8_t sm[];
    double *qd = reinterpret_cast<double *>(sm);                       // [G][hd]
    double *pd = qd + G * hd;                                          // [G][PA_CHUNK]
    float *sc = reinterpret_cast<float *>(pd + G * PA_CHUNK);          // [G][n_score]
    uint16_t *p16 = reinterpret_cast<uint16_t *>(sc + (size_t)G * ns_max);   // [G][n_score]
    const int hk = blockIdx.x, t = blockIdx.y, tid = threadIdx.x;
    const int n_score = pos0 + t + 1;
    const float *c = cs + (int64_t)t * (n_rot / 2), *s = sn + (int64_t)t * (n_rot / 2);
    for (int i = tid; i < G * hd; i += blockDim.x) {
        const int g = i / hd, d = i - g * hd;
        const float *qrow = q + ((int64_t)t * n_head + hk * G + g) * hd;
        qd[i] = h2d_exact(f2h(rope_channel(qrow, d, hd, n_rot, neox, c, s)));
    }
    __syncthreads();
    // scores: a position per thread at a time, its K row read 64 halves
    // (eight 16-byte loads in flight) at a time
    const uint16_t *kh = kc + (int64_t)hk * n_ctx * hd;
    const bool kvec = (reinterpret_cast<uintptr_t>(kh) & 15) == 0 && (hd & 7) == 0;
    for (int j = tid; j < n_score; j += blockDim.x) {
        const uint16_t *row = kh + (int64_t)j * hd;
        double a[G];
#pragma unroll
        for (int g = 0; g < G; ++g) a[g] = 0.0;
        for (int d0 = 0; d0 < hd; d0 += 64) {
            if (kvec && d0 + 64 <= hd) {
                uint4 xr[8];
                ld_h64(row + d0, xr);
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    const double kd = h2d_exact(h_of(xr, k));
#pragma unroll
                    for (int g = 0; g < G; ++g) a[g] = __fma_rn(kd, qd[g * hd + d0 + k], a[g]);
                }
            } else {
                for (int d = d0; d < min(hd, d0 + 64); d += 8) {
                    uint16_t x[8];
                    ld_h8(row + d, kvec, x);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const double kd = h2d_exact(x[k]);
#pragma unroll
                        for (int g = 0; g < G; ++g) a[g] = __fma_rn(kd, qd[g * hd + d + k], a[g]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) sc[(size_t)g * n_score + j] = __fmul_rn(__double2float_rn(a[g]), ks);
    }
    __syncthreads();
    // softmax and f16 probabilities, one warp per head
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < G; g += (int)(blockDim.x >> 5)) {
        float *row = sc + (size_t)g * n_score;
        softmax_row_warp(row, row, n_score);
        for (int j = lane; j < n_score; j += 32) p16[(size_t)g * n_score + j] = f2h(row[j]);
    }
    // value dots: task (channel cch, heads g0 .. g0 + hpt - 1), hpt the
    // fewest heads per task that fit hd x ceil(G / hpt) tasks in the CTA
    // (hd <= blockDim)
    int hpt = 1;
    while (hd * ((G + hpt - 1) / hpt) > (int)blockDim.x) ++hpt;
    const int ngrp = (G + hpt - 1) / hpt;
    const int cch = tid % hd, g0 = (tid / hd) * hpt;
    const bool active = tid < hd * ngrp;
    const uint16_t *vrow = vc + ((int64_t)hk * hd + cch) * n_ctx;
    const bool vvec = (reinterpret_cast<uintptr_t>(vrow) & 15) == 0;   // j0 is a multiple of 64
    double acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.0;
    for (int j0 = 0; j0 < n_score; j0 += PA_CHUNK) {
        const int jn = min(PA_CHUNK, n_score - j0);
        // a whole chunk of the V row in flight across the barriers below
        const bool full = active && vvec && jn == PA_CHUNK;
        uint4 xv[8];
        if (full) ld_h64(vrow + j0, xv);
        __syncthreads();   // the probabilities written; the previous chunk consumed
        for (int i = tid; i < G * PA_CHUNK; i += blockDim.x) {
            const int g = i / PA_CHUNK, jj = i - g * PA_CHUNK;
            pd[i] = jj < jn ? h2d_exact(p16[(size_t)g * n_score + j0 + jj]) : 0.0;
        }
        __syncthreads();
        if (full) {
#pragma unroll
            for (int k = 0; k < PA_CHUNK; ++k) {
                const double vd = h2d_exact(h_of(xv, k));
#pragma unroll
                for (int hh = 0; hh < G; ++hh)
                    if (hh < hpt && g0 + hh < G) acc[hh] = __fma_rn(vd, pd[(g0 + hh) * PA_CHUNK + k], acc[hh]);
            }
        } else if (active) {
            const uint16_t *r = vrow + j0;
            for (int jj = 0; jj < jn; jj += 8) {
                uint16_t x[8];
                if (jj + 8 <= jn) {
                    ld_h8(r + jj, vvec, x);
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) x[k] = jj + k < jn ? r[jj + k] : (uint16_t)0;
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (jj + k < jn) {
                        const double vd = h2d_exact(x[k]);
#pragma unroll
                        for (int hh = 0; hh < G; ++hh)
                            if (hh < hpt && g0 + hh < G)
                                acc[hh] = __fma_rn(vd, pd[(g0 + hh) * PA_CHUNK + jj + k], acc[hh]);
                    }
                }
            }
        }
    }
    if (active) {
#pragma unroll
        for (int hh = 0; hh < G; ++hh)
            if (hh < hpt && g0 + hh < G)
                out[((int64_t)t * n_head + hk * G + g0 + hh) * hd + cch] = __double2float_rn(acc[hh]);
    }
}

// dynamic shared memory of prompt_attention_group_kernel for G heads of hd
// channels and at most ns_max positions
size_t pa_group_smem(int G, int hd, int ns_max) {
    return (size_t)G * hd * 8 + (size_t)G * PA_CHUNK * 8 + (size_t)G * ns_max * 6 + 16;
}

template <int G>
int launch_pa_group(const float *q, const uint16_t *kc, const uint16_t *vc, const float *cs, const float *sn,
                    int n_head, int n_head_kv, int hd, int n_rot, int neox, int n_ctx, int pos0, int m, float ks,
                    float *out, size_t smem, cudaStream_t st) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(prompt_attention_group_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PA_GROUP_SMEM_MAX) != cudaSuccess)
            return -2;
        attr[dev & 63] = true;
    }
    prompt_attention_group_kernel<G><<<dim3((unsigned)n_head_kv, (unsigned)m), 256, smem, st>>>(
        q, kc, vc, cs, sn, n_head, hd, n_rot, neox, n_ctx, pos0, pos0 + m, ks, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace

int launch_attention(const float *q, const void *kc, const void *vc, int n_head, int n_head_kv, int hd, int n_ctx,
                     int pos, float ks, float *out, cudaStream_t st) {
    const int n_score = pos + 1;
    const size_t smem = (size_t)n_score * 6 + 16;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
            return -2;
        attr[dev & 63] = true;
    }
    attention_kernel<<<n_head, 256, smem, st>>>(q, static_cast<const uint16_t *>(kc), static_cast<const uint16_t *>(vc),
                                                n_head, n_head / n_head_kv, hd, n_ctx, n_score, ks, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_attention_prompt(const float *q, const float *k, const float *v, void *kc, void *vc, const float *cs,
                            const float *sn, int n_head, int n_head_kv, int hd, int n_rot, int neox, int n_ctx, int pos0,
                            int m, float ks, float *out, cudaStream_t st) {
    const int gqa = n_head / n_head_kv;
    const size_t gsmem = pa_group_smem(gqa, hd, pos0 + m);
    if (gqa <= 8 && hd <= 256 && hd % 8 == 0 && gsmem <= (size_t)PA_GROUP_SMEM_MAX) {
        prompt_kv_store_kernel<<<(unsigned)m, 256, 0, st>>>(k, v, static_cast<uint16_t *>(kc),
                                                             static_cast<uint16_t *>(vc), cs, sn, n_head_kv, hd, n_rot,
                                                             neox, n_ctx, pos0);
        if (cudaPeekAtLastError() != cudaSuccess) return -2;
        const uint16_t *kcc = static_cast<const uint16_t *>(kc), *vcc = static_cast<const uint16_t *>(vc);
        switch (gqa) {
#define PA_G(G)                                                                                                        \
    case G:                                                                                                            \
        return launch_pa_group<G>(q, kcc, vcc, cs, sn, n_head, n_head_kv, hd, n_rot, neox, n_ctx, pos0, m, ks, out,   \
                                  gsmem, st);
            PA_G(1) PA_G(2) PA_G(3) PA_G(4) PA_G(5) PA_G(6) PA_G(7) PA_G(8)
#undef PA_G
        }
    }
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(prompt_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 180 * 1024) !=
            cudaSuccess)
            return -2;
        attr[dev & 63] = true;
    }
    prompt_kv_store_kernel<<<(unsigned)m, 256, 0, st>>>(k, v, static_cast<uint16_t *>(kc), static_cast<uint16_t *>(vc),
                                                         cs, sn, n_head_kv, hd, n_rot, neox, n_ctx, pos0);
    if (cudaPeekAtLastError() != cudaSuccess) return -2;
    const size_t smem = (size_t)(pos0 + m) * 6 + 16;
    prompt_attention_kernel<<<dim3((unsigned)n_head, (unsigned)m), 256, smem, st>>>(
        q, static_cast<const uint16_t *>(kc), static_cast<const uint16_t *>(vc), cs, sn, n_head, n_head / n_head_kv, hd,
        n_rot, neox, n_ctx, pos0, ks, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_attention_step(const float *q, const float *k, const float *v, void *kc, void *vc, const float *cs,
                          const float *sn, int n_head, int n_head_kv, int hd, int n_rot, int neox, int n_ctx, int pos,
                          float ks, float *out, int overlap, cudaStream_t st) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        if (cudaFuncSetAttribute(attention_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 180 * 1024) !=
            cudaSuccess)
            return -2;
        attr[dev & 63] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)n_head);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t)(pos + 1) * 6 + 16;
    cfg.stream = st;
    cudaLaunchAttribute attr1[1];
    attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr1[0].val.programmaticStreamSerializationAllowed = 0;
    (void)overlap;
    cfg.attrs = attr1;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, attention_step_kernel, q, k, v, static_cast<uint16_t *>(kc),
                           static_cast<uint16_t *>(vc), cs, sn, n_head, n_head / n_head_kv, hd, n_rot, neox, n_ctx,
                           pos, ks, out) != cudaSuccess)
        return -2;
    return 0;
}

int launch_rope(float *x, int n_heads, int hd, int n_rot, const float *cs, const float *sn, int neox, cudaStream_t st) {
    const int64_t total = (int64_t)n_heads * (n_rot / 2);
    if (total <= 0) return 0;
    rope_kernel<<<(unsigned)((total + 255) / 256 > 1024 ? 1024 : (total + 255) / 256), 256, 0, st>>>(x, n_heads, hd, n_rot,
                                                                                                   cs, sn, neox);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_kv_store(const float *k, const float *v, void *kc, void *vc, int n_head_kv, int hd, int n_ctx, int pos,
                    cudaStream_t st) {
    const int total = n_head_kv * hd;
    kv_store_kernel<<<(total + 255) / 256, 256, 0, st>>>(k, v, static_cast<uint16_t *>(kc), static_cast<uint16_t *>(vc),
                                                         n_head_kv, hd, n_ctx, pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_softmax(const float *x, float *y, int64_t n, int64_t m, cudaStream_t st) {
    if (m <= 0 || n <= 0) return 0;
    softmax_kernel<<<(unsigned)m, 256, 0, st>>>(x, y, (int)n);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
