// Activation quantizers, byte-identical with the reference:
//   Q8_K : src/kernels.c:561-595 (the only form the reference has)
//   Q8_0 : src/kernels_avx2.c:594-645 (the form x86 hosts dispatch to)
//   F16  : element-wise RNE narrowing (src/backend.c:19-27)
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "prologue.cuh"

namespace sicu {

// One warp quantizes one 256-element block (src/kernels.c:561-595); lane L
// owns elements 8L..8L+7 and gets their quants q[0..7], the sum of the 16
// quants of lanes 2k and 2k+1 (bsum2: block sum k in lane 2k and 2k+1) and
// the block scale d. An all-zero block gives d = 0 and zero quants and sums.
// x must be 16-byte aligned.
__device__ __forceinline__ void q8k_quant_warp(const float *x, int lane, int (&q)[8], int &bsum2, float &d) {
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
    if (!(best > 0.0f)) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
        bsum2 = 0;
        d = 0.0f;
        return;
    }
    float own = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) if ((bi & 7) == i) own = v[i];
    const float mx = __shfl_sync(0xffffffffu, own, bi >> 3);
    const float iscale = __fdiv_rn(-127.0f, mx);
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int qi;
        if (isnan(v[i])) {
            // the reference's magic-number rounding leaves a NaN's low payload bits
            qi = (int)(__float_as_uint(v[i]) & 0x3fffffu);
        } else {
            qi = __float2int_rn(__fmul_rn(iscale, v[i]));
        }
        q[i] = qi < 127 ? qi : 127;
        sum += q[i];
    }
    bsum2 = sum + __shfl_xor_sync(0xffffffffu, sum, 1);
    d = __fdiv_rn(1.0f, iscale);
}

// One warp quantizes one 256-element block into the raw 292-byte Q8_K layout
// (d f32 @0, qs int8 @4, bsums int16 @260). Lane L owns elements 8L..8L+7.
// x must be 16-byte aligned. An all-zero block writes d = 0, qs = 0 and
// bsums = 0 (the reference leaves bsums untouched there).
__device__ __forceinline__ void q8k_block_warp(const float *x, uint8_t *dst, int lane) {
    int q[8], bsum2;
    float d;
    q8k_quant_warp(x, lane, q, bsum2, d);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) packed[i / 4] |= ((uint32_t)q[i] & 0xffu) << (8 * (i & 3));
    uint32_t *qw = reinterpret_cast<uint32_t *>(dst + 4);
    qw[2 * lane] = packed[0];
    qw[2 * lane + 1] = packed[1];
    if ((lane & 1) == 0) reinterpret_cast<int16_t *>(dst + 260)[lane >> 1] = (int16_t)bsum2;
    if (lane == 0) *reinterpret_cast<float *>(dst) = d;
}

__device__ __forceinline__ float vmaxps(float a, float b) { return a > b ? a : b; }

__device__ __forceinline__ int sat8_rounded(float r) {
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) return -128;
    const int i = (int)r;
    return i > 127 ? 127 : (i < -128 ? -128 : i);
}

// One thread quantizes one 32-element block (AVX2 form): v in, f16 d and
// 32 int8 quants (8 little-endian words) out.
__device__ __forceinline__ void q8_0_block_v(const float v[32], uint32_t &d16, uint32_t qw[8]);

__device__ __forceinline__ void q8_0_block(const float *x, uint32_t &d16, uint32_t qw[8]) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float4 f = reinterpret_cast<const float4 *>(x)[k];
        v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
    }
    q8_0_block_v(v, d16, qw);
}

__device__ __forceinline__ void q8_0_block_v(const float v[32], uint32_t &d16, uint32_t qw[8]) {
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

// Quantizes one K-format piece: lane j (of the 8-lane group owning record u)
// holds elements 32j..32j+31 of the record in v.
template <int ACT>
__device__ __forceinline__ void q8k_piece(const ActView av, const RecWriter &wr, int u, int j, unsigned gmask,
                                          const float v[32]) {
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

// Quantizes one classic-format 32-element block (unit u, block bi of it).
__device__ __forceinline__ void q80_piece(const ActView av, const RecWriter &wr, int u, int bi, const float v[32]) {
    uint32_t d16, q[8];
    q8_0_block_v(v, d16, q);
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = dp4a_ss(q[k], 0x01010101u, s);
    put_block(av, wr, u, bi, q, h2f(d16), s);
}

// Fused prologue: quantize the f32 activation straight into the prepared
// records this cluster rank owns (u % nrank == rank), writing each into every
// CTA of the cluster. K formats: eight lanes per 256-element block, lane j
// owning elements 32j..32j+31, so after one 3-step max reduction every lane
// emits its own piece. Classic formats: one thread per 32-element block.
template <int ACT>
__device__ __forceinline__ void quantize_into_act(const ActView av, const float *xf, int n_in, uint32_t rank,
                                                  uint32_t nrank) {
    const RecWriter wr{nrank};
    if constexpr (ACT == 3) {
        const int nblk = n_in / 32, nu = (nblk + 7) / 8;
        const int mine = (nu - (int)rank + (int)nrank - 1) / (int)nrank;
        for (int i = threadIdx.x; i < mine * 8; i += blockDim.x) {
            const int u = (int)rank + (int)nrank * (i >> 3), b = 8 * u + (i & 7);
            if (b >= nblk) continue;
            float v[32];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 f = ld_f4(xf, 8 * b + k);
                v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
            }
            q80_piece(av, wr, u, i & 7, v);
        }
    } else {
        const int nsb = n_in / 256;
        const int lane = threadIdx.x & 31, j = lane & 7;
        const unsigned gmask = 0xffu << (lane & 24);
        const int groups = blockDim.x >> 3;
        for (int u = (int)rank + (int)nrank * (threadIdx.x >> 3); u < nsb; u += (int)nrank * groups) {
            float v[32];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 f = ld_f4(xf, 64 * u + 8 * j + k);
                v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
            }
            q8k_piece<ACT>(av, wr, u, j, gmask, v);
        }
    }
}

// The RMS norm's scale from this thread's share s of the sum of squares:
// each warp adds its lanes' shares and writes the result into slot
// [rank][warp] of every CTA of the cluster (distributed shared memory); after
// one cluster barrier every thread adds the slots in (rank, warp) order, and
// rms_mean turns the total into the reference's mean. Every thread of every
// CTA of the cluster calls.
__device__ __forceinline__ float cluster_scale(double s, const float *x, const ProDev &pro, int n_in, uint32_t rank,
                                               uint32_t nrank, void *scratch) {
    double *part = reinterpret_cast<double *>(scratch);     // [nrank][8]
    float *out = reinterpret_cast<float *>(part + 64);
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) {
        const uint32_t a = smem_addr(&part[rank * 8 + warp]);
        const uint64_t bits = (uint64_t)__double_as_longlong(s);
        for (uint32_t r = 0; r < nrank; ++r) {
            const uint32_t ra = mapa(a, r);
            st_cluster(ra, (uint32_t)bits);
            st_cluster(ra + 4, (uint32_t)(bits >> 32));
        }
    }
    cluster_sync();
    double S = 0.0;
    for (uint32_t r = 0; r < nrank; ++r)
        for (int w = 0; w < nw; ++w) S += part[r * 8 + w];
    return rms_scale_of(rms_mean(S, x, pro.res, n_in, pro.inv_n, out), pro.eps);
}

// Eight float4s of h = x (+ res) at i4 into a, all loads issued first (the
// compiler cannot know the stores to h_out alias nothing the loads read);
// the first cluster's CTAs also store them to h_out. Returns their squares'
// sum.
__device__ __forceinline__ double load_h8(const float *x, const float *res, float *h_out, int64_t i4, float4 a[8]) {
    float4 b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = ld_f4(x, i4 + k);
    if (res) {
#pragma unroll
        for (int k = 0; k < 8; ++k) b[k] = ld_f4(res, i4 + k);
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = add4(a[k], b[k]);
    }
    if (h_out) {
#pragma unroll
        for (int k = 0; k < 8; ++k) reinterpret_cast<float4 *>(h_out)[i4 + k] = a[k];
    }
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += sq4(a[k]);
    return s;
}

// The fused quantizer of launches with an activation step (pro.kind is not
// PRO_NONE; the matvec kernels' STEPS instantiations), kept out of line:
// called once per CTA, it
// leaves the kernel's main loop its own register allocation. Same pieces as
// quantize_into_act, with pro applied to xf first (every thread of the CTA
// calls; scratch holds RMS_SCRATCH bytes of shared memory). The norm needs
// the sum of squares of the whole row before its first output: each thread
// loads its own piece of h and of the norm weight once, adds its squares, and
// keeps the piece in registers while the cluster agrees on the scale; rows
// with more pieces than the CTA has threads (groups) take two passes over
// memory instead.
template <int ACT>
__device__ __noinline__ void quantize_steps(const ActView av, const float *xf, int n_in, uint32_t rank,
                                            uint32_t nrank, const ProDev pro, void *scratch) {
    const RecWriter wr{nrank};
    const int lane = threadIdx.x & 31;
    // this CTA's pieces: K formats one per 8-lane group and record, classic
    // formats one per thread and 32-element block
    int npieces, per_pass;
    if constexpr (ACT == 3) {
        const int nu = (n_in / 32 + 7) / 8;
        npieces = 8 * ((nu - (int)rank + (int)nrank - 1) / (int)nrank);
        per_pass = blockDim.x;
    } else {
        npieces = (n_in / 256 - (int)rank + (int)nrank - 1) / (int)nrank;
        per_pass = blockDim.x >> 3;
    }
    // piece p: its unit, index inside the unit, first float4, and validity
    auto piece = [&](int p, int &u, int &jb, int64_t &i4) -> bool {
        if constexpr (ACT == 3) {
            u = (int)rank + (int)nrank * (p >> 3);
            jb = p & 7;
            const int b = 8 * u + jb;
            i4 = 8 * (int64_t)b;
            return p < npieces && b < n_in / 32;
        } else {
            u = (int)rank + (int)nrank * p;
            jb = lane & 7;
            i4 = 64 * (int64_t)u + 8 * jb;
            return p < npieces;
        }
    };
    const int first = (ACT == 3) ? (int)threadIdx.x : (int)(threadIdx.x >> 3);
    const unsigned gmask = 0xffu << (lane & 24);
    auto emit = [&](int u, int jb, const float v[32]) {
        if constexpr (ACT == 3) q80_piece(av, wr, u, jb, v);
        else q8k_piece<ACT>(av, wr, u, jb, gmask, v);
    };

    if (pro.kind == PRO_RMS_NORM) {
        float *h_out = blockIdx.x < nrank ? pro.h_out : nullptr;
        if (npieces <= per_pass) {
            int u, jb;
            int64_t i4;
            const bool have = piece(first, u, jb, i4);
            float4 a[8], g[8];
            double s = 0.0;
            if (have) {
#pragma unroll
                for (int k = 0; k < 8; ++k) g[k] = ld_f4(pro.g, i4 + k);
                s = load_h8(xf, pro.res, h_out, i4, a);
            }
            const float scale = cluster_scale(s, xf, pro, n_in, rank, nrank, scratch);
            if (have) {
                float v[32];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    v[4 * k] = __fmul_rn(__fmul_rn(a[k].x, scale), g[k].x);
                    v[4 * k + 1] = __fmul_rn(__fmul_rn(a[k].y, scale), g[k].y);
                    v[4 * k + 2] = __fmul_rn(__fmul_rn(a[k].z, scale), g[k].z);
                    v[4 * k + 3] = __fmul_rn(__fmul_rn(a[k].w, scale), g[k].w);
                }
                emit(u, jb, v);
            }
            return;
        }
        // long rows: a pass for the sum, then the quantizing pass reads again
        double s = 0.0;
        for (int p = first; p < npieces; p += per_pass) {
            int u, jb;
            int64_t i4;
            float4 a[8];
            if (piece(p, u, jb, i4)) s += load_h8(xf, pro.res, h_out, i4, a);
        }
        const float scale = cluster_scale(s, xf, pro, n_in, rank, nrank, scratch);
        const ActLoad ld{xf, pro, scale};
        for (int p = first; p < npieces; p += per_pass) {
            int u, jb;
            int64_t i4;
            if (!piece(p, u, jb, i4)) continue;
            float v[32];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 f = ld(i4 + k);
                v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
            }
            emit(u, jb, v);
        }
        return;
    }
    // SwiGLU / multiply: both operands' eight float4s in flight together
    for (int p = first; p < npieces; p += per_pass) {
        int u, jb;
        int64_t i4;
        if (!piece(p, u, jb, i4)) continue;
        float4 a[8], b[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = ld_f4(xf, i4 + k);
#pragma unroll
        for (int k = 0; k < 8; ++k) b[k] = ld_f4(pro.up, i4 + k);
        float v[32];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float4 t = a[k];
            if (pro.kind == PRO_SWIGLU) {
                t.x = silu_ref(t.x); t.y = silu_ref(t.y); t.z = silu_ref(t.z); t.w = silu_ref(t.w);
            }
            v[4 * k] = __fmul_rn(t.x, b[k].x);
            v[4 * k + 1] = __fmul_rn(t.y, b[k].y);
            v[4 * k + 2] = __fmul_rn(t.z, b[k].z);
            v[4 * k + 3] = __fmul_rn(t.w, b[k].w);
        }
        emit(u, jb, v);
    }
}

}  // namespace sicu
