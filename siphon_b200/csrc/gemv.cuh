// Batch-1 decode matvec y = W x for GGUF block formats, bit-exact with the
// reference's scalar dot products (src/kernels.c:197-523).
//
// Structure (one persistent CTA per SM, 8 warps):
//   * Work is split into tasks of R consecutive rows; long rows are streamed
//     in chunks of CU "units" (a unit is one K super-block, or eight classic
//     32-blocks = 256 elements). Tasks are dealt to CTAs in balanced
//     contiguous ranges and to warps round-robin.
//   * Each warp owns an S-slot ring in shared memory. Lane 0 fills slots with
//     1-D bulk TMA copies (cp.async.bulk + mbarrier transaction counts); the
//     raw GGUF bytes are never re-laid-out in HBM.
//   * Phase 1: lanes decode one unit each (nibbles, high bits, 6-bit scales in
//     registers), run int8 dot products (dp4a / dp2a), and emit the float
//     terms the reference's scalar loop adds per block.
//   * Phase 2: one lane per float chain adds those terms in the reference's
//     order with __fadd_rn / __fsub_rn, so every output is bit-identical.
//
// Exactness: the reference keeps, for the K formats with int8 lane
// accumulators, eight per-lane integer sums aux32[l] over elements l mod 8
// (src/kernels.c:384-409). Integer sums are order-free, so the kernel forms
// them with byte transposes (prmt) that gather same-l elements into one
// dp4a / dp2a operand; only the float chain is order-bound.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace sicu {

constexpr int GEMV_WARPS = 8;
constexpr int MAX_CHAINS = 9;
// term buffer: K formats [chain][row][unit padded to 4] with rows x units <= 32
// and rows <= 7 (<= 9 x 53 floats); classic [row][8 x unit] (<= 256 floats)
constexpr int TERM_FLOATS = 480;
constexpr int CONS_BYTES = 4 * (TERM_FLOATS + 64);   // per consumer warp: terms, chain results

constexpr int GEMV_MAX_MATS = 64;
// Ring slots each warp fills before the activation is ready (the rest after)
constexpr int GEMV_PRE_WAIT_SLOTS = 64;

struct GemvParams {
    // the matrices of one launch: same format and row length, one activation
    int nmat;
    const uint8_t *w[GEMV_MAX_MATS];   // weight blocks, row-major, 16-byte aligned
    float *y[GEMV_MAX_MATS];
    int n_out[GEMV_MAX_MATS];
    int task0[GEMV_MAX_MATS + 1];      // first task of each matrix (prefix sums)
    const uint8_t *xq;     // pair-format activation (Q8_K / Q8_0 blocks), or null
    const float *xf;       // f32 activation for the fused quantize variant, or null
    int64_t row_bytes;
    int n_in;
    int nu;                // units per row
    int cu;                // units per chunk
    int nchunks;           // chunks per row (1 unless R == 1)
    int rows_per_task;     // R
    int64_t ntasks;
    int slot_bytes;
    int nslots;            // ring slots per warp
    int act_bytes;         // prepared-activation region
    int warp_bytes;        // per-warp region: barriers, slot geometry, terms, ring
    int *status;
    ArDev ar;              // n > 0: one row-split matrix; y = the group's sum of the partial outputs
    ProDev pro;            // activation step the quantizer applies to xf first (STEPS kernels)
    uint64_t epi_silu;     // bit i: write silu(y) for matrix i (STEPS kernels)
    const float *bias[GEMV_MAX_MATS];   // add bias[i][row] to matrix i's outputs (STEPS kernels; null: none)
};

// ---------------------------------------------------------------------------
// Prepared activation layout (shared memory, one record per 256-element unit)
//   aq : 64 words of int8 quants in the order the format's unit decoder wants
//   ad : K formats: Q8_K d; classic: 8 per-block f32 scales
//   ax : K formats: extra integer sums; classic: 8 per-block quant sums
// ---------------------------------------------------------------------------
struct ActView {
    // one 368-byte record (23 x 16 B, an odd number of 16-byte units so lanes
    // reading consecutive records never share a bank group) per 256 elements:
    //   [0,256)   aq: 64 words of int8 quants in the decoder's order
    //   [256,320) ax: 16 ints (format-dependent integer sums)
    //   [320,352) ad: 8 floats (scales)
    uint8_t *base;
    int nu;
    static constexpr int STRIDE = 368;
    __device__ uint8_t *rec(int u) const { return base + (size_t)u * STRIDE; }
    __device__ uint8_t *aq(int u) const { return rec(u); }
    __device__ int *ax(int u) const { return reinterpret_cast<int *>(rec(u) + 256); }
    __device__ float *ad(int u) const { return reinterpret_cast<float *>(rec(u) + 320); }
    static __host__ __device__ int bytes(int nu) { return nu * STRIDE; }
};

// ---- format traits ----------------------------------------------------------
// kind: 0 = K format, lane sums (9 chains: 8 lanes + dmin), 1 = K format,
// lane sums without mins (8 chains), 2 = one chain per super-block (Q2_K),
// 3 = classic 32-blocks (one chain, eight terms per unit)
template <uint32_t T> struct Fmt;
template <> struct Fmt<T_Q4_K> { static constexpr int kind = 0, unit_bytes = B_Q4_K, chains = 9, tpu = 1, act = 0; };
template <> struct Fmt<T_Q5_K> { static constexpr int kind = 0, unit_bytes = B_Q5_K, chains = 9, tpu = 1, act = 0; };
template <> struct Fmt<T_Q6_K> { static constexpr int kind = 1, unit_bytes = B_Q6_K, chains = 8, tpu = 1, act = 1; };
template <> struct Fmt<T_Q3_K> { static constexpr int kind = 1, unit_bytes = B_Q3_K, chains = 8, tpu = 1, act = 1; };
template <> struct Fmt<T_Q2_K> { static constexpr int kind = 2, unit_bytes = B_Q2_K, chains = 1, tpu = 1, act = 2; };
template <> struct Fmt<T_Q4_0> { static constexpr int kind = 3, unit_bytes = 8 * B_Q4_0, chains = 1, tpu = 8, act = 3; };
template <> struct Fmt<T_Q5_0> { static constexpr int kind = 3, unit_bytes = 8 * B_Q5_0, chains = 1, tpu = 8, act = 3; };
template <> struct Fmt<T_Q8_0> { static constexpr int kind = 3, unit_bytes = 8 * B_Q8_0, chains = 1, tpu = 8, act = 3; };

// ---------------------------------------------------------------------------
// Activation preparation (every CTA builds its own copy in shared memory).
//   act 0 (Q4_K, Q5_K): per 32-element sub-block j, word l holds the quants of
//         elements l, l+8, l+16, l+24 (the reference's lane-l elements);
//         ax[k] = bsums[2k] + bsums[2k+1] (the per-32 sums the mins use).
//   act 1 (Q3_K, Q6_K): per 16-element sub-block j, word q holds elements
//         q, q+8 (dp2a.lo half) and q+4, q+12 (dp2a.hi half).
//   act 2 (Q2_K): natural order; ax = the 16 bsums.
//   act 3 (classic): natural order, ad = f16 block scale as f32, ax = sum of
//         the block's 32 quants.
// src points at the raw pair-format row (global or shared memory).
// ---------------------------------------------------------------------------
// Writes a record field into the same place of every CTA of the thread-block
// cluster (distributed shared memory), so each activation record is built once
// per cluster instead of once per CTA.
struct RecWriter {
    uint32_t nrank;
    __device__ void put4(const void *local, uint32_t a, uint32_t b, uint32_t c, uint32_t d) const {
        const uint32_t addr = smem_addr(local);
        for (uint32_t r = 0; r < nrank; ++r) st_cluster4(mapa(addr, r), a, b, c, d);
    }
    __device__ void put(const void *local, uint32_t v) const {
        const uint32_t addr = smem_addr(local);
        for (uint32_t r = 0; r < nrank; ++r) st_cluster(mapa(addr, r), v);
    }
};

// K formats: piece j (elements 32j..32j+31) of record u from 8 natural-order
// quant words, the piece's two 16-element sums, and (j == 0) the block scale.
template <int ACT>
__device__ __forceinline__ void put_piece(const ActView av, const RecWriter &wr, int u, int j, const uint32_t q[8],
                                          int s0, int s1, float d) {
    uint32_t o[8];
    if constexpr (ACT == 0) {
        transpose4(q[0], q[2], q[4], q[6], o[0], o[1], o[2], o[3]);
        transpose4(q[1], q[3], q[5], q[7], o[4], o[5], o[6], o[7]);
    } else if constexpr (ACT == 1) {
        // two 16-element sub-blocks: words (q0,q1,q2,q3) = elements 0..15
        transpose4(q[0], q[2], q[1], q[3], o[0], o[1], o[2], o[3]);
        transpose4(q[4], q[6], q[5], q[7], o[4], o[5], o[6], o[7]);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = q[k];
    }
    uint8_t *rec = av.rec(u);
    wr.put4(rec + 32 * j, o[0], o[1], o[2], o[3]);
    wr.put4(rec + 32 * j + 16, o[4], o[5], o[6], o[7]);
    if constexpr (ACT == 0) {
        wr.put(av.ax(u) + j, (uint32_t)(s0 + s1));
    } else if constexpr (ACT == 2) {
        wr.put(av.ax(u) + 2 * j, (uint32_t)s0);
        wr.put(av.ax(u) + 2 * j + 1, (uint32_t)s1);
    }
    if (j == 0) wr.put(av.ad(u), __float_as_uint(d));
}

// Classic formats: block bi of record u.
__device__ __forceinline__ void put_block(const ActView av, const RecWriter &wr, int u, int bi, const uint32_t q[8],
                                          float d, int asum) {
    uint8_t *rec = av.rec(u);
    wr.put4(rec + 32 * bi, q[0], q[1], q[2], q[3]);
    wr.put4(rec + 32 * bi + 16, q[4], q[5], q[6], q[7]);
    wr.put(av.ad(u) + bi, __float_as_uint(d));
    wr.put(av.ax(u) + bi, (uint32_t)asum);
}

// Build the records this cluster rank owns (u % nrank == rank) from the
// caller's pair-format row in global memory.
template <int ACT>
__device__ void prep_activation(const ActView av, const uint8_t *src, int n_in, uint32_t rank, uint32_t nrank) {
    const RecWriter wr{nrank};
    const int tid = threadIdx.x, nt = blockDim.x;
    if constexpr (ACT == 3) {
        const int nblk = n_in / 32, nu = (nblk + 7) / 8;
        const int mine = (nu - (int)rank + (int)nrank - 1) / (int)nrank;
        for (int i = tid; i < mine * 8; i += nt) {
            const int u = (int)rank + (int)nrank * (i >> 3), b = 8 * u + (i & 7);
            if (b >= nblk) continue;
            // qs start at byte 2 of a 34-byte block: read halves and rejoin
            const uint16_t *h = reinterpret_cast<const uint16_t *>(src + (size_t)b * B_Q8_0);
            uint32_t q[8];
            int s = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                q[k] = (uint32_t)h[1 + 2 * k] | ((uint32_t)h[2 + 2 * k] << 16);
                s = dp4a_ss(q[k], 0x01010101u, s);
            }
            put_block(av, wr, u, i & 7, q, h2f(h[0]), s);
        }
    } else {
        const int nu = n_in / 256;
        const int mine = (nu - (int)rank + (int)nrank - 1) / (int)nrank;
        for (int i = tid; i < mine * 8; i += nt) {
            const int u = (int)rank + (int)nrank * (i >> 3), j = i & 7;
            const uint8_t *blk = src + (size_t)u * B_Q8_K;
            const uint32_t *qs = reinterpret_cast<const uint32_t *>(blk + 4 + 32 * j);
            uint32_t q[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) q[k] = qs[k];
            const int16_t *bs = reinterpret_cast<const int16_t *>(blk + 260);
            put_piece<ACT>(av, wr, u, j, q, bs[2 * j], bs[2 * j + 1], *reinterpret_cast<const float *>(blk));
        }
    }
}

// ---- unit decoders ------------------------------------------------------------
// Each computes the float term(s) one super-block (or eight 32-blocks) of one
// weight row contributes, exactly as the reference computes them before the
// running sums: t[0..chains-1] (K formats) or t[0..7] (classic, per block).

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }
__device__ __forceinline__ int sbyte_of(uint32_t w, int i) { return ((int)(w << (24 - 8 * i))) >> 24; }

// Q4_K (src/kernels.c:349-410): 16-byte aligned in shared memory.
template <bool Q5>
__device__ __forceinline__ void unit_q45k(const uint8_t *wb, const uint8_t *aq, float *t) {
    const uint4 h = *reinterpret_cast<const uint4 *>(wb);
    const int4 pb0 = *reinterpret_cast<const int4 *>(aq + 256);
    const int4 pb1 = *reinterpret_cast<const int4 *>(aq + 272);
    const int pb[8] = {pb0.x, pb0.y, pb0.z, pb0.w, pb1.x, pb1.y, pb1.z, pb1.w};
    const float yd = reinterpret_cast<const float4 *>(aq + 320)->x;
    // 6-bit scales/mins (src/kernels.c:377-382 / 648-656), four per word
    const uint32_t sc_lo = h.y & 0x3f3f3f3fu;
    const uint32_t mn_lo = h.z & 0x3f3f3f3fu;
    const uint32_t sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);

    constexpr int QS = Q5 ? 48 : 16;
    uint32_t ht[8];
    if constexpr (Q5) {
        const uint4 h0 = *reinterpret_cast<const uint4 *>(wb + 16);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(wb + 32);
        transpose4(h0.x, h0.z, h1.x, h1.z, ht[0], ht[1], ht[2], ht[3]);
        transpose4(h0.y, h0.w, h1.y, h1.w, ht[4], ht[5], ht[6], ht[7]);
    }
    int aux[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) aux[l] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 qa = *reinterpret_cast<const uint4 *>(wb + QS + 32 * c);
        const uint4 qb = *reinterpret_cast<const uint4 *>(wb + QS + 32 * c + 16);
        uint32_t tq[8];
        transpose4(qa.x, qa.z, qb.x, qb.z, tq[0], tq[1], tq[2], tq[3]);
        transpose4(qa.y, qa.w, qb.y, qb.w, tq[4], tq[5], tq[6], tq[7]);
        const uint4 a0 = *reinterpret_cast<const uint4 *>(aq + 64 * c);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(aq + 64 * c + 16);
        const uint4 a2 = *reinterpret_cast<const uint4 *>(aq + 64 * c + 32);
        const uint4 a3 = *reinterpret_cast<const uint4 *>(aq + 64 * c + 48);
        const uint32_t alo[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t ahi[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
        const uint32_t scw = c < 2 ? sc_lo : sc_hi;
        // the high nibbles stay in place (16x their value); the low-nibble
        // scale carries the same factor 16, divided out exactly below
        const int s0 = 16 * (int)byte_of(scw, (2 * c) & 3), s1 = (int)byte_of(scw, (2 * c + 1) & 3);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            uint32_t lo, hi;
            if constexpr (Q5) {
                // fifth bit of sub-block 2c / 2c+1 is bit 2c / 2c+1 of qh[b]:
                // bit 4 of a low byte, bit 8 (= bit 4 of 16 x value) of a high one
                const uint32_t b0 = (c <= 2 ? (ht[l] << (4 - 2 * c)) : (ht[l] >> (2 * c - 4))) & 0x10101010u;
                const uint32_t b1 = (c <= 1 ? (ht[l] << (3 - 2 * c)) : (ht[l] >> (2 * c - 3))) & 0x10101010u;
                lo = and_or(tq[l], 0x0f0f0f0fu, b0);
                hi = ((tq[l] >> 4) & 0x0f0f0f0fu) | b1;
                aux[l] += dp4a(lo, alo[l], 0) * (s0 >> 4) + dp4a(hi, ahi[l], 0) * s1;
            } else {
                lo = tq[l] & 0x0f0f0f0fu;
                hi = tq[l] & 0xf0f0f0f0u;
                aux[l] += dp4a(lo, alo[l], 0) * s0 + dp4a(hi, ahi[l], 0) * s1;
            }
        }
    }
    if constexpr (!Q5) {
#pragma unroll
        for (int l = 0; l < 8; ++l) aux[l] >>= 4;   // exact: every term carries a factor 16
    }
    const int mins = (int)byte_of(mn_lo, 0) * pb[0] + (int)byte_of(mn_lo, 1) * pb[1] +
                     (int)byte_of(mn_lo, 2) * pb[2] + (int)byte_of(mn_lo, 3) * pb[3] +
                     (int)byte_of(mn_hi, 0) * pb[4] + (int)byte_of(mn_hi, 1) * pb[5] +
                     (int)byte_of(mn_hi, 2) * pb[6] + (int)byte_of(mn_hi, 3) * pb[7];
    const float d = __fmul_rn(h2f(h.x & 0xffffu), yd);
#pragma unroll
    for (int l = 0; l < 8; ++l) t[l] = __fmul_rn(d, __int2float_rn(aux[l]));
    // the reference subtracts this term (sumf -= dmin*sumi); a - b == a + (-b)
    // exactly in IEEE arithmetic, so it is stored negated and added like the rest
    t[8] = -__fmul_rn(__fmul_rn(h2f(h.x >> 16), yd), __int2float_rn(mins));
}

// Realigned 32-bit reads from a 2-byte aligned shared address.
struct Words {
    const uint32_t *p;
    uint32_t sh;
    __device__ Words(const uint8_t *addr) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(addr);
        p = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
        sh = (uint32_t)(a & 3) * 8;
    }
    __device__ __forceinline__ uint32_t operator[](int k) const { return funnel(p[k], p[k + 1], sh); }
};

// sign-extending pair selectors: int16 {byte b of x, byte b of y}
__device__ __forceinline__ uint32_t pair_sel(int b) {
    return (uint32_t)(b | ((b | 8) << 4) | ((4 + b) << 8) | (((4 + b) | 8) << 12));
}

// Q6_K (src/kernels.c:480-523) and Q3_K (src/kernels.c:289-347): 16-element
// sub-blocks, int8 quants built as 4*v (Q6_K) / 32*v (Q3_K) so the sign sits
// in bit 7, paired by element (e, e+8) into int16 for dp2a.
template <bool Q3>
__device__ __forceinline__ void unit_q36k(const uint8_t *wb, const uint8_t *aq, float *t) {
    const Words W(wb);
    const float yd = reinterpret_cast<const float4 *>(aq + 320)->x;
    int aux[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) aux[l] = 0;
    // scales: 16 signed values, sub-block j
    int sc[16];
    float dx;
    if constexpr (Q3) {
        const uint32_t s0 = W[24], s1 = W[25], s2 = W[26];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t lo = j < 8 ? (byte_of(j < 4 ? s0 : s1, j & 3) & 15u) : (byte_of(j < 12 ? s0 : s1, j & 3) >> 4);
            const uint32_t hi = (byte_of(s2, j & 3) >> (2 * (j / 4))) & 3u;
            sc[j] = (int)(lo | (hi << 4)) - 32;
        }
        dx = h2f(W[27] & 0xffffu);
    } else {
        const uint32_t s[4] = {W[48], W[49], W[50], W[51]};
#pragma unroll
        for (int j = 0; j < 16; ++j) sc[j] = sbyte_of(s[j / 4], j & 3);
        dx = h2f(W[52] & 0xffffu);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // element words E[g][k]: elements 128h + 32g + 4k .. +3
        uint32_t E[4][8];
        if constexpr (Q3) {
            uint32_t HM[8], QS[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) { HM[k] = W[k]; QS[k] = W[8 + 8 * h + k]; }
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int p = 4 * h + g;   // hmask bit
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint32_t qs = (5 - 2 * g) >= 0 ? (QS[k] << (5 - 2 * g)) : (QS[k] >> 1);
                    const uint32_t hb = and_xor(HM[k] << (7 - p), 0x80808080u, 0x80808080u);
                    E[g][k] = and_or(qs, 0x60606060u, hb);
                }
            }
        } else {
            uint32_t QL[16], QH[8];
#pragma unroll
            for (int k = 0; k < 16; ++k) QL[k] = W[16 * h + k];
#pragma unroll
            for (int k = 0; k < 8; ++k) QH[k] = W[32 + 8 * h + k];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint32_t ql = QL[(g & 1) ? 8 + k : k];
                    const uint32_t lo = g < 2 ? (ql << 2) : (ql >> 2);
                    const uint32_t hi = and_xor(QH[k] << (6 - 2 * g), 0xc0c0c0c0u, 0x80808080u);
                    E[g][k] = and_or(lo, 0x3c3c3c3cu, hi);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
#pragma unroll
            for (int k4 = 0; k4 < 2; ++k4) {
                const int j = 8 * h + 2 * g + k4;
                const uint4 aw = *reinterpret_cast<const uint4 *>(aq + 16 * j);
                const uint32_t awv[4] = {aw.x, aw.y, aw.z, aw.w};
                const uint32_t e0 = E[g][4 * k4], e1 = E[g][4 * k4 + 1], e2 = E[g][4 * k4 + 2], e3 = E[g][4 * k4 + 3];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint32_t plo = prmt(e0, e2, pair_sel(b));   // lane b
                    const uint32_t phi = prmt(e1, e3, pair_sel(b));   // lane 4+b
                    aux[b] += sc[j] * dp2a_lo(plo, awv[b], 0);
                    aux[4 + b] += sc[j] * dp2a_hi(phi, awv[b], 0);
                }
            }
        }
    }
    const float d = __fmul_rn(dx, yd);
#pragma unroll
    for (int l = 0; l < 8; ++l) t[l] = __fmul_rn(d, __int2float_rn(aux[l] >> (Q3 ? 5 : 2)));
}

// Q2_K (src/kernels.c:249-287): one integer sum per super-block. 4-byte aligned.
__device__ __forceinline__ void unit_q2k(const uint8_t *wb, const uint8_t *aq, float *t) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(wb);
    int bs[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int4 v = reinterpret_cast<const int4 *>(aq + 256)[k];
        bs[4 * k] = v.x; bs[4 * k + 1] = v.y; bs[4 * k + 2] = v.z; bs[4 * k + 3] = v.w;
    }
    const float yd = reinterpret_cast<const float4 *>(aq + 320)->x;
    const uint32_t scw[4] = {w[0], w[1], w[2], w[3]};
    int isum = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        uint32_t QS[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) QS[i] = w[4 + 8 * k + i];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int is = 8 * k + 2 * jj + hh;
                const uint4 a = *reinterpret_cast<const uint4 *>(aq + 4 * (32 * k + 8 * jj + 4 * hh));
                const uint32_t av[4] = {a.x, a.y, a.z, a.w};
                int s = 0;
#pragma unroll
                for (int m = 0; m < 4; ++m) s = dp4a((QS[4 * hh + m] >> (2 * jj)) & 0x03030303u, av[m], s);
                isum += (int)(byte_of(scw[is / 4], is & 3) & 15u) * s;
            }
        }
    }
    int summs = 0;
#pragma unroll
    for (int g = 0; g < 16; ++g) summs += bs[g] * (int)(byte_of(scw[g / 4], g & 3) >> 4);
    const uint32_t dd = w[20];
    const float dall = __fmul_rn(yd, h2f(dd & 0xffffu));
    const float dmin = __fmul_rn(yd, h2f(dd >> 16));
    t[0] = __fsub_rn(__fmul_rn(dall, __int2float_rn(isum)), __fmul_rn(dmin, __int2float_rn(summs)));
}

// Classic 32-blocks (src/kernels.c:197-247): up to eight blocks per unit,
// 2-byte aligned. Terms: Q4_0/Q5_0 (sumi*dx)*dy, Q8_0 sumi*(dx*dy).
template <uint32_t T>
__device__ __forceinline__ void unit_classic(const uint8_t *wb, int nblk, const uint8_t *aq, float *t) {
    const Words W(wb);
    float dy[8];
    int asum[8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float4 d = reinterpret_cast<const float4 *>(aq + 320)[k];
        const int4 a = reinterpret_cast<const int4 *>(aq + 256)[k];
        dy[4 * k] = d.x; dy[4 * k + 1] = d.y; dy[4 * k + 2] = d.z; dy[4 * k + 3] = d.w;
        asum[4 * k] = a.x; asum[4 * k + 1] = a.y; asum[4 * k + 2] = a.z; asum[4 * k + 3] = a.w;
    }
    constexpr int BW = (T == T_Q4_0) ? 9 : (T == T_Q5_0) ? 11 : 17;   // words per block pair
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int b = 2 * p + half;
            if (b < nblk) {
                const uint4 a0 = *reinterpret_cast<const uint4 *>(aq + 32 * b);
                const uint4 a1 = *reinterpret_cast<const uint4 *>(aq + 32 * b + 16);
                const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const int base = BW * p;
                uint32_t d16;
                int s = 0;
                if constexpr (T == T_Q4_0) {
                    // pair: [d0 qs0(16)] [d1 qs1(16)], 36 bytes
                    uint32_t q[4];
                    if (half == 0) {
                        const uint32_t x0 = W[base];
                        d16 = x0 & 0xffffu;
                        uint32_t prev = x0;
#pragma unroll
                        for (int m = 0; m < 4; ++m) { const uint32_t nx = W[base + 1 + m]; q[m] = funnel(prev, nx, 16); prev = nx; }
                    } else {
                        d16 = W[base + 4] >> 16;
#pragma unroll
                        for (int m = 0; m < 4; ++m) q[m] = W[base + 5 + m];
                    }
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        s = dp4a(q[m] & 0x0f0f0f0fu, av[m], s);
                        s = dp4a((q[m] >> 4) & 0x0f0f0f0fu, av[4 + m], s);
                    }
                    s -= 8 * asum[b];
                } else if constexpr (T == T_Q5_0) {
                    // pair: [d0 qh0(4) qs0(16)] [d1 qh1 qs1], 44 bytes
                    uint32_t q[4], qh;
                    if (half == 0) {
                        const uint32_t x0 = W[base], x1 = W[base + 1];
                        d16 = x0 & 0xffffu;
                        qh = funnel(x0, x1, 16);
                        uint32_t prev = x1;
#pragma unroll
                        for (int m = 0; m < 4; ++m) { const uint32_t nx = W[base + 2 + m]; q[m] = funnel(prev, nx, 16); prev = nx; }
                    } else {
                        d16 = W[base + 5] >> 16;
                        qh = W[base + 6];
#pragma unroll
                        for (int m = 0; m < 4; ++m) q[m] = W[base + 7 + m];
                    }
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        // bits 4m..4m+3 (low nibbles) and 16+4m.. (high) of qh to bit 4 of each byte
                        const uint32_t b_lo = (((qh >> (4 * m)) & 15u) * 0x02040810u) & 0x10101010u;
                        const uint32_t b_hi = (((qh >> (16 + 4 * m)) & 15u) * 0x02040810u) & 0x10101010u;
                        s = dp4a(and_or(q[m], 0x0f0f0f0fu, b_lo), av[m], s);
                        s = dp4a(and_or(q[m] >> 4, 0x0f0f0f0fu, b_hi), av[4 + m], s);
                    }
                    s -= 16 * asum[b];
                } else {
                    // Q8_0 pair: [d0 qs0(32)] [d1 qs1(32)], 68 bytes
                    uint32_t q[8];
                    if (half == 0) {
                        const uint32_t x0 = W[base];
                        d16 = x0 & 0xffffu;
                        uint32_t prev = x0;
#pragma unroll
                        for (int m = 0; m < 8; ++m) { const uint32_t nx = W[base + 1 + m]; q[m] = funnel(prev, nx, 16); prev = nx; }
                    } else {
                        d16 = W[base + 8] >> 16;
#pragma unroll
                        for (int m = 0; m < 8; ++m) q[m] = W[base + 9 + m];
                    }
#pragma unroll
                    for (int m = 0; m < 8; ++m) s = dp4a_ss(q[m], av[m], s);
                }
                const float dx = h2f(d16);
                if constexpr (T == T_Q8_0) {
                    t[b] = __fmul_rn(__int2float_rn(s), __fmul_rn(dx, dy[b]));
                } else {
                    t[b] = __fmul_rn(__fmul_rn(__int2float_rn(s), dx), dy[b]);
                }
            }
        }
    }
}

}  // namespace sicu
