// Stand-alone activation quantizers and row dequantisation (row_to_f32).
#include "quantize.cuh"
#include "launch.h"

namespace sicu {

namespace {

// Q8_K: one warp per 256-element block; m rows of n floats are contiguous,
// so block g of the whole batch maps to x[256 g] and y[292 g].
__global__ void __launch_bounds__(256) quant_q8k_kernel(const float *x, uint8_t *y, int64_t nblk) {
    const int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (g >= nblk) return;
    q8k_block_warp(x + 256 * g, y + (size_t)B_Q8_K * g, threadIdx.x & 31);
}

// Q8_0 (AVX2 form): one thread per 32-element block
__global__ void __launch_bounds__(256) quant_q80_kernel(const float *x, uint8_t *y, int64_t nblk) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= nblk) return;
    uint32_t d16, qw[8];
    q8_0_block(x + 32 * g, d16, qw);
    uint16_t *o = reinterpret_cast<uint16_t *>(y + (size_t)B_Q8_0 * g);   // 2-byte aligned
    o[0] = (uint16_t)d16;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        o[1 + 2 * k] = (uint16_t)(qw[k] & 0xffffu);
        o[2 + 2 * k] = (uint16_t)(qw[k] >> 16);
    }
}

// n floats from page-locked host memory (its device view) into device
// memory, one 16-byte load per thread; lets the next kernel (programmatic
// dependent launch) start streaming its weights right away
__global__ void __launch_bounds__(256) host_copy_kernel(const float4 *src, float4 *dst, int64_t n4) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) dst[i] = src[i];
}

__global__ void __launch_bounds__(256) convert_f16_kernel(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = f2h(x[i]);
}

// ---- dequantisation, reference semantics (src/kernels.c:599-817) ----------------
__device__ __forceinline__ uint32_t b8(const uint8_t *p, int i) { return p[i]; }
__device__ __forceinline__ uint32_t h16(const uint8_t *p, int i) { return (uint32_t)p[i] | ((uint32_t)p[i + 1] << 8); }

__device__ float dequant_elem(uint32_t t, const uint8_t *row, int e) {
    switch (t) {
        case T_F16: return h2f(h16(row, 2 * e));
        case T_Q4_0: {
            const uint8_t *b = row + (e / 32) * B_Q4_0;
            const int j = e % 32;
            const int q = (j < 16 ? (int)(b8(b, 2 + j) & 15u) : (int)(b8(b, 2 + j - 16) >> 4)) - 8;
            return __fmul_rn(__int2float_rn(q), h2f(h16(b, 0)));
        }
        case T_Q5_0: {
            const uint8_t *b = row + (e / 32) * B_Q5_0;
            const int j = e % 32;
            const uint32_t qh = h16(b, 2) | (h16(b, 4) << 16);
            const int nib = j < 16 ? (int)(b8(b, 6 + j) & 15u) : (int)(b8(b, 6 + j - 16) >> 4);
            const int q = (nib | (int)(((qh >> j) & 1u) << 4)) - 16;
            return __fmul_rn(__int2float_rn(q), h2f(h16(b, 0)));
        }
        case T_Q8_0: {
            const uint8_t *b = row + (e / 32) * B_Q8_0;
            return __fmul_rn(__int2float_rn((int)(int8_t)b[2 + e % 32]), h2f(h16(b, 0)));
        }
        case T_Q2_K: {
            const uint8_t *b = row + (e / 256) * B_Q2_K;
            const int i = e % 256, k = i / 128, r = i % 128;
            const uint32_t s = b8(b, i / 16);
            const int q = (int)((b8(b, 16 + 32 * k + r % 32) >> (2 * (r / 32))) & 3u);
            const float dl = __fmul_rn(h2f(h16(b, 80)), __int2float_rn((int)(s & 15u)));
            const float ml = __fmul_rn(h2f(h16(b, 82)), __int2float_rn((int)(s >> 4)));
            return __fsub_rn(__fmul_rn(dl, __int2float_rn(q)), ml);
        }
        case T_Q3_K: {
            const uint8_t *b = row + (e / 256) * B_Q3_K;
            const int i = e % 256, h = i / 128, g = (i % 128) / 32, l = i % 32, j = i / 16;
            const int q = (int)((b8(b, 32 + 32 * h + l) >> (2 * g)) & 3u) - (((b8(b, l) >> (4 * h + g)) & 1u) ? 0 : 4);
            const uint8_t *s = b + 96;
            const uint32_t lo = j < 8 ? (b8(s, j) & 15u) : (b8(s, j - 8) >> 4);
            const uint32_t hi = (b8(s, 8 + j % 4) >> (2 * (j / 4))) & 3u;
            const float dl = __fmul_rn(h2f(h16(b, 108)), __int2float_rn((int)(lo | (hi << 4)) - 32));
            return __fmul_rn(dl, __int2float_rn(q));
        }
        case T_Q4_K:
        case T_Q5_K: {
            const bool q5 = t == T_Q5_K;
            const uint8_t *b = row + (e / 256) * (q5 ? B_Q5_K : B_Q4_K);
            const int i = e % 256, j = i / 32;
            const uint8_t *s = b + 4;
            uint32_t sc, mn;
            if (j < 4) { sc = b8(s, j) & 63u; mn = b8(s, j + 4) & 63u; }
            else { sc = (b8(s, j + 4) & 15u) | ((b8(s, j - 4) >> 6) << 4); mn = (b8(s, j + 4) >> 4) | ((b8(s, j) >> 6) << 4); }
            const uint32_t byte = b8(b, (q5 ? 48 : 16) + 32 * (i / 64) + i % 32);
            int q = (int)((i % 64) < 32 ? (byte & 15u) : (byte >> 4));
            if (q5) q += ((b8(b, 16 + i % 32) >> j) & 1u) ? 16 : 0;
            const float d1 = __fmul_rn(h2f(h16(b, 0)), __int2float_rn((int)sc));
            const float m1 = __fmul_rn(h2f(h16(b, 2)), __int2float_rn((int)mn));
            return __fsub_rn(__fmul_rn(d1, __int2float_rn(q)), m1);
        }
        case T_Q6_K: {
            const uint8_t *b = row + (e / 256) * B_Q6_K;
            const int i = e % 256, h = i / 128, g = (i % 128) / 32, l = i % 32;
            const uint32_t lo = b8(b, 64 * h + l + ((g & 1) ? 32 : 0));
            const uint32_t hi = b8(b, 128 + 32 * h + l);
            const uint32_t nib = g < 2 ? (lo & 15u) : (lo >> 4);
            const int q = (int)(nib | (((hi >> (2 * g)) & 3u) << 4)) - 32;
            const int sc = (int)(int8_t)b[192 + i / 16];
            return __fmul_rn(__fmul_rn(h2f(h16(b, 208)), __int2float_rn(sc)), __int2float_rn(q));
        }
        default: return 0.0f;
    }
}

// rows[i] outside [0, n_rows) (ids read from device memory): the output row
// is NaN and the status word gets STATUS_BAD_ROW; nothing is read
__global__ void __launch_bounds__(256) dequant_kernel(uint32_t t, const uint8_t *w, int64_t row_bytes, int n_in,
                                                    const int64_t *rows, float *out, int64_t n_rows, int *status) {
    const int64_t r = rows[blockIdx.y];
    if (r < 0 || r >= n_rows) {
        for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_in; e += gridDim.x * blockDim.x)
            out[(int64_t)blockIdx.y * n_in + e] = __uint_as_float(0x7fc00000u);
        if (status && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(status, STATUS_BAD_ROW);
        return;
    }
    const uint8_t *row = w + r * row_bytes;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_in; e += gridDim.x * blockDim.x)
        out[(int64_t)blockIdx.y * n_in + e] = dequant_elem(t, row, e);
}

// Greedy choice per row (si_sample_greedy, src/sampler.c:6-12): best = 0, then
// every later element strictly greater than the best so far takes its place;
// i.e. the first maximum among the non-NaN values, or 0 when x[0] is NaN.
__global__ void __launch_bounds__(256) argmax_kernel(const float *x, int64_t n, int64_t *out) {
    __shared__ float bv[8];
    __shared__ int64_t bi[8];
    const float *xr = x + (int64_t)blockIdx.x * n;
    float v = -__int_as_float(0x7f800000);
    int64_t idx = -1;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float a = xr[i];
        if (a > v || (idx < 0 && a == v)) { v = a; idx = i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oi >= 0 && (idx < 0 || ov > v || (ov == v && oi < idx))) { v = ov; idx = oi; }
    }
    if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = v; bi[threadIdx.x >> 5] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (bi[w] >= 0 && (idx < 0 || bv[w] > v || (bv[w] == v && bi[w] < idx))) { v = bv[w]; idx = bi[w]; }
        out[blockIdx.x] = (isnan(xr[0]) || idx < 0) ? 0 : idx;
    }
}

}  // namespace

int launch_host_copy(const float *src, float *dst, int64_t n, cudaStream_t st) {
    const int64_t n4 = n / 4;
    host_copy_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(reinterpret_cast<const float4 *>(src),
                                                                    reinterpret_cast<float4 *>(dst), n4);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_quantize(uint32_t pair, const float *x, void *y, int64_t n, int64_t m, cudaStream_t st) {
    if (pair == T_Q8_K) {
        const int64_t nblk = m * (n / 256);
        if (nblk == 0) return 0;
        quant_q8k_kernel<<<(unsigned)((nblk + 7) / 8), 256, 0, st>>>(x, static_cast<uint8_t *>(y), nblk);
    } else if (pair == T_Q8_0) {
        const int64_t nblk = m * (n / 32);
        if (nblk == 0) return 0;
        quant_q80_kernel<<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>(x, static_cast<uint8_t *>(y), nblk);
    } else if (pair == T_F16) {
        const int64_t tot = m * n;
        if (tot == 0) return 0;
        int64_t grid = (tot + 255) / 256;
        if (grid > 4096) grid = 4096;
        convert_f16_kernel<<<(unsigned)grid, 256, 0, st>>>(x, static_cast<uint16_t *>(y), tot);
    } else {
        return -3;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_argmax(const float *x, int64_t n, int64_t m, int64_t *out, cudaStream_t st) {
    if (m <= 0 || n <= 0) return 0;
    argmax_kernel<<<(unsigned)m, 256, 0, st>>>(x, n, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_dequant(uint32_t wtype, const void *w, int64_t n_in, const int64_t *rows_dev, int64_t nrows,
                   float *out, cudaStream_t st, int64_t n_rows, int *status) {
    int64_t blk = 1, bsz = 2;
    switch (wtype) {
        case T_F16: blk = 1; bsz = 2; break;
        case T_Q4_0: blk = 32; bsz = B_Q4_0; break;
        case T_Q5_0: blk = 32; bsz = B_Q5_0; break;
        case T_Q8_0: blk = 32; bsz = B_Q8_0; break;
        case T_Q2_K: blk = 256; bsz = B_Q2_K; break;
        case T_Q3_K: blk = 256; bsz = B_Q3_K; break;
        case T_Q4_K: blk = 256; bsz = B_Q4_K; break;
        case T_Q5_K: blk = 256; bsz = B_Q5_K; break;
        case T_Q6_K: blk = 256; bsz = B_Q6_K; break;
        default: return -3;
    }
    if (nrows == 0 || n_in == 0) return 0;
    const int64_t row_bytes = n_in / blk * bsz;
    int64_t gx = (n_in + 255) / 256;
    if (gx > 1024) gx = 1024;
    dim3 grid((unsigned)gx, (unsigned)nrows);
    dequant_kernel<<<grid, 256, 0, st>>>(wtype, static_cast<const uint8_t *>(w), row_bytes, (int)n_in, rows_dev, out,
                                         n_rows, status);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
