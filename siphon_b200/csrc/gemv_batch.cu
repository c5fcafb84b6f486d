// Batch decode matvec: Y[n][r] = (W x_n)[r] for up to eight activation rows
// x_0..x_{m-1} (one token of each of m sequences) in ONE pass over the weight
// blocks, on the tensor cores, bit-identical with the reference's per-token
// scalar dot products (src/kernels.c:349-410 Q4_K, 480-523 Q6_K).
//
// The reference's K-quant dot keeps eight integer lane sums per super-block,
// aux32[l] = sum over the elements e = l (mod 8) of sc(e) * q(e) * a(e), and
// adds d * aux32[l] into eight float running sums (plus a dmin chain for
// Q4_K). Integer sums are order-free, float sums are not. Here:
//
//   * a CTA of four warps owns a tile of 16 weight rows and walks its
//     super-blocks in rounds of four, one super-block per warp. For half h of
//     a super-block and lane class l, one mma.sync.m16n8k16 (f16 operands, f32
//     accumulation) multiplies the 16 rows' elements e = 128h + l + 8k
//     (k = 0..15) with the same elements of the 8 activation rows: the MMA's K
//     dimension runs over one lane class, so its f32 accumulator holds the
//     exact integer lane sum (every operand and partial sum is an integer
//     below 2^24). Q4_K's min term, sum_j mins[j] * bsums, is one more MMA per
//     (h, l) with the sub-block mins as the weight operand;
//   * the weight operand is decoded in registers straight from the raw GGUF
//     bytes into exact f16 (scale x quant) values: a nibble (or 6-bit quant)
//     is OR-ed into the mantissa of 1024.0 and one half-precision FMA removes
//     the bias and applies the sub-block scale (Q4_K: sc * q <= 945; Q6_K: the
//     int8 scale split as 16 * hi + lo into two planes with separate
//     accumulators, combined exactly in f32);
//   * the activation operand (int8 Q8_K quants, exact in f16) is laid out in
//     the MMA's fragment order once per call by a small prep kernel, which
//     also quantizes f32 rows with the reference's quantizer;
//   * each warp turns its accumulators into the reference's float terms
//     (d * aux32[l], -(dmin * sumi)) in shared memory (double buffered);
//     after one CTA barrier per round, one thread per (row, token) adds the
//     round's terms to its nine float chains in super-block order with
//     __fadd_rn, exactly the reference's sequence. The barrier sits where the
//     threads have no global loads in flight (a barrier waits for them): the
//     next round's activation loads are issued after it.
//
// Weights stream through a ring of shared-memory stages (16 rows x four
// super-blocks) filled by 1-D bulk copies, one per row (rows that do not
// start on a 16-byte boundary are copied from the boundary below and read
// with funnel shifts), issued by a fifth warp that refills a stage once the
// four compute warps have released it: issuing a stage's 16 copies takes
// ~1 us, which in a compute warp held every round's barrier. The compute
// warps' round barrier is a named barrier of their 128 threads. Every wait
// is bounded and reports through the status word.
#include "common.cuh"
#include "launch.h"
#include "quantize.cuh"

namespace sicu {

namespace {

// record of one super-block's activation, for BATCH_MAX tokens
constexpr int BREC_YD = 4096;            // float yd[8]: the Q8_K block scale of each token
constexpr int BREC_BYTES = 4096 + 32;
// fragment part: [h 2][lp 4][lane 32] uint4 = {b0(l), b1(l), b0(l+1), b1(l+1)}, l = 2 lp,
// b0 = f16x2(a[e], a[e+64]), b1 = f16x2(a[e+8], a[e+72]), e = 128h + l + 16t, token g
// (lane = 4g + t): the MMA for (h, l) maps its K index 2t, 2t+1, 2t+8, 2t+9 to
// the elements e, e+64, e+8, e+72 of lane class l

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t f16x2_of_ints(int a, int b) {
    const __half2 h = __halves2half2(__int2half_rn(a), __int2half_rn(b));
    return *reinterpret_cast<const uint32_t *>(&h);
}

// One CTA per super-block u, one warp per token: quantize (f32 input, the
// reference's Q8_K quantizer) or copy (Q8_K input) the token's block, then
// write the record.
template <bool FROM_F32>
__global__ void __launch_bounds__(256) batch_prep_kernel(const float *xf, const uint8_t *xq, int n_in, int m,
                                                         uint8_t *rec) {
    __shared__ __align__(16) uint8_t q8[BATCH_MAX][304];
    const int u = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = n_in / 256;
    grid_dep_launch();   // the product kernel may start streaming its weights
    grid_dep_wait();     // x may be written by the previous kernel in the stream
    if (warp < m) {
        if constexpr (FROM_F32) {
            q8k_block_warp(xf + (size_t)warp * n_in + 256 * (size_t)u, q8[warp], lane);
        } else {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(xq + ((size_t)warp * nb + u) * B_Q8_K);
            uint32_t *dst = reinterpret_cast<uint32_t *>(q8[warp]);
            for (int i = lane; i < B_Q8_K / 4; i += 32) dst[i] = src[i];
        }
    }
    __syncthreads();
    uint8_t *r = rec + (size_t)u * BREC_BYTES;
    {
        const int i = threadIdx.x, h = i >> 7, lp = (i >> 5) & 3, ln = i & 31, g = ln >> 2, t = ln & 3;
        uint32_t v[4] = {0u, 0u, 0u, 0u};
        if (g < m) {
            const int8_t *qs = reinterpret_cast<const int8_t *>(q8[g] + 4);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int e = 128 * h + 2 * lp + k + 16 * t;
                v[2 * k] = f16x2_of_ints(qs[e], qs[e + 64]);
                v[2 * k + 1] = f16x2_of_ints(qs[e + 8], qs[e + 72]);
            }
        }
        reinterpret_cast<uint4 *>(r)[i] = make_uint4(v[0], v[1], v[2], v[3]);
    }
    if (threadIdx.x < BATCH_MAX) {
        const int n = threadIdx.x;
        reinterpret_cast<float *>(r + BREC_YD)[n] = n < m ? *reinterpret_cast<const float *>(q8[n]) : 0.0f;
    }
}

constexpr int BATCH_MATS = 16;
constexpr int BW = 4;                   // compute warps per CTA = super-blocks per round
constexpr int BT = (BW + 1) * 32;       // threads per CTA: the compute warps and the producer warp

// barrier of the compute warps' BW * 32 threads (named barrier 1), true if
// any of them passes true
__device__ __forceinline__ bool compute_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\t"
        "setp.ne.u32 a, %1, 0;\n\t"
        "bar.red.or.pred b, 1, %2, a;\n\t"
        "selp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r) : "r"((uint32_t)v), "n"(BW * 32) : "memory");
    return r != 0;
}
constexpr int NPAIR = 16 * BATCH_MAX;   // (row, token) pairs of a tile
// float terms of a round, double buffered: lane terms [buffer 2][warp][pair 128][8],
// then the dmin terms [buffer 2][warp][pair 128]
constexpr int TERMS_LANE_FLOATS = 2 * BW * NPAIR * 8;
constexpr int TERMS_BYTES = 2 * BW * NPAIR * 9 * 4;

struct BatchParams {
    int nmat;
    const uint8_t *w[BATCH_MATS];
    float *y[BATCH_MATS];                // [m][n_out] each
    int n_out[BATCH_MATS];
    int tile0[BATCH_MATS + 1];           // first tile of each matrix
    int ntiles;
    const uint8_t *rec;                  // [nb] activation records
    int64_t row_bytes;
    int nb;                              // super-blocks per row
    int rounds;                          // rounds per tile: ceil(nb / BW)
    int m;                               // tokens (1..8)
    int rs;                              // shared-memory bytes per row of a stage
    int nstages;
    int *status;
};

template <uint32_t T> struct BFmt;
template <> struct BFmt<T_Q4_K> { static constexpr int ub = B_Q4_K; };
template <> struct BFmt<T_Q6_K> { static constexpr int ub = B_Q6_K; };

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// f16x2 {v, v} of an integer v that has at most 11 significant bits (exact)
__device__ __forceinline__ uint32_t h2dup(int v) {
    const unsigned short h = __half_as_ushort(__int2half_rn(v));
    return (uint32_t)h * 0x10001u;
}
// f16x2 {v / 16, v / 16} (exact for |v| < 2^11)
__device__ __forceinline__ uint32_t h2dup_div16(int v) {
    const unsigned short h = __half_as_ushort(__float2half_rn((float)v * 0.0625f));
    return (uint32_t)h * 0x10001u;
}

// byte j of the 16 bytes x[0..3] at bytes 0 and 1, byte j of y[0..3] at bytes 2 and 3
__device__ __forceinline__ uint32_t pairxy(const uint32_t x[4], const uint32_t y[4], int j) {
    const uint32_t b = (uint32_t)(j & 3);
    const uint32_t sel = b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12);
    return prmt(x[j >> 2], y[j >> 2], sel);
}
// bytes j, j + 8, j, j + 8 of the 16 bytes x[0..3] (j < 8)
__device__ __forceinline__ uint32_t pair_j8(const uint32_t x[4], int j) {
    const uint32_t b = (uint32_t)(j & 3);
    const uint32_t sel = b | ((4 + b) << 4) | (b << 8) | ((4 + b) << 12);
    return prmt(x[j >> 2], x[(j >> 2) + 2], sel);
}
// f16x2 {byte i of w, byte k of w} for bytes holding 0..255
__device__ __forceinline__ uint32_t h2_bytes(uint32_t w, int i, int k) {
    const uint32_t v = prmt(w, 0u, (uint32_t)(i | (4 << 4) | (k << 8) | (4 << 12))) | 0x64006400u;
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64006400u));   // - 1024: exact
    return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t h2f32(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// 16 bytes at a 2-byte aligned shared address as four words
__device__ __forceinline__ void lds16_any(const uint8_t *addr, uint32_t w[4]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(addr);
    const uint32_t *p = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3) * 8;
    const uint32_t x0 = p[0], x1 = p[1], x2 = p[2], x3 = p[3], x4 = p[4];
    w[0] = funnel(x0, x1, sh);
    w[1] = funnel(x1, x2, sh);
    w[2] = funnel(x2, x3, sh);
    w[3] = funnel(x3, x4, sh);
}

__device__ __forceinline__ void lds16(const uint8_t *addr, uint32_t w[4]) {
    const uint4 v = *reinterpret_cast<const uint4 *>(addr);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
}

// Lane sums of one super-block for the warp's 16 rows x 8 tokens:
// acc[l][q] (q: d0..d3 of the MMA fragment = (row g | g + 8) x (token 2t | 2t + 1)),
// accm[q] the mins sum (Q4_K), xd / xm the rows' f16 d / dmin as f32. The
// thread's A registers hold elements (e, e + 64) and (e + 8, e + 72) of lane
// class l, e = 128h + 16t + l, i.e. sub-blocks (4h + t/2, 4h + 2 + t/2) (Q4_K)
// or (8h + t, 8h + 4 + t) (Q6_K): one f16x2 scale constant per row and half.
template <uint32_t T>
__device__ __forceinline__ void batch_superblock(const uint8_t *b0, const uint8_t *b1, const uint4 (&fc)[8], int t,
                                                 float (&acc)[8][4], float (&accm)[4], float (&xd)[2],
                                                 float (&xm)[2]) {
#pragma unroll
    for (int l = 0; l < 8; ++l)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[l][q] = 0.0f;
    if constexpr (T == T_Q4_K) {
        float am[4][4];   // mins sums, four independent accumulators (by l & 3)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) am[i][q] = 0.0f;
        // d, dmin, 12 bytes of packed 6-bit scales and mins (src/kernels.c:377-382)
        uint32_t hd[2][4];
        lds16(b0, hd[0]);
        lds16(b1, hd[1]);
        uint32_t mul[2][2], add[2][2], mnv[2][2];   // [row][h]
        const int ja = t >> 1, jb = 2 + (t >> 1);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const uint32_t y = hd[rr][1], z = hd[rr][2], wv = hd[rr][3];
            const uint32_t sc_lo = y & 0x3f3f3f3fu, mn_lo = z & 0x3f3f3f3fu;
            const uint32_t sc_hi = (wv & 0x0f0f0f0fu) | ((y >> 2) & 0x30303030u);
            const uint32_t mn_hi = ((wv >> 4) & 0x0f0f0f0fu) | ((z >> 2) & 0x30303030u);
            xd[rr] = h2f(hd[rr][0] & 0xffffu);
            xm[rr] = h2f(hd[rr][0] >> 16);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t sc = h2_bytes(h ? sc_hi : sc_lo, ja, jb);
                // low nibbles (t < 2): (1024 + q) * sc - 1024 sc; high nibbles in
                // place (1024 + 16 q): * sc / 16 - 64 sc (every value exact in f16)
                mul[rr][h] = (t < 2) ? sc : hmul2(sc, 0x2c002c00u);                // x 1/16
                add[rr][h] = hmul2(sc, (t < 2) ? 0xe400e400u : 0xd400d400u);      // x -1024 | x -64
                mnv[rr][h] = h2_bytes(h ? mn_hi : mn_lo, ja, jb);
            }
        }
        const uint32_t nmask = (t < 2) ? 0x000f000fu : 0x00f000f0u;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t x[2][2][4];   // [row][chunk 2h | 2h + 1][word]
            const int off = 16 + 64 * h + 16 * (t & 1);
            lds16(b0 + off, x[0][0]);
            lds16(b0 + off + 32, x[0][1]);
            lds16(b1 + off, x[1][0]);
            lds16(b1 + off + 32, x[1][1]);
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                uint32_t a[4];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                    for (int k = 0; k < 2; ++k) {   // k = 0: elements (e, e+64); 1: (e+8, e+72)
                        const uint32_t v = and_or(pairxy(x[rr][0], x[rr][1], l + 8 * k), nmask, 0x64006400u);
                        a[rr + 2 * k] = hfma2(v, mul[rr][h], add[rr][h]);
                    }
                const uint4 f = fc[4 * h + (l >> 1)];
                const uint32_t bb0 = (l & 1) ? f.z : f.x, bb1 = (l & 1) ? f.w : f.y;
                mma16816(acc[l], a[0], a[1], a[2], a[3], bb0, bb1);
                // sumi = sum over the elements of mins[sub-block] * a (= sum_j mins[j] * bsums)
                mma16816(am[l & 3], mnv[0][h], mnv[1][h], mnv[0][h], mnv[1][h], bb0, bb1);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) accm[q] = (am[0][q] + am[1][q]) + (am[2][q] + am[3][q]);   // exact integers
    } else {
        // Q6_K: ql[128] @0, qh[64] @128, int8 scales[16] @192, d @208 (src/kernels.c:480-523)
        float acch[8][4];
#pragma unroll
        for (int l = 0; l < 8; ++l)
#pragma unroll
            for (int q = 0; q < 4; ++q) acch[l][q] = 0.0f;
        uint32_t scw[2][4];
        lds16_any(b0 + 192, scw[0]);
        lds16_any(b1 + 192, scw[1]);
        {
            uint32_t dd[4];
            lds16_any(b0 + 196, dd);   // bytes 208, 209 = word 3's low half
            xd[0] = h2f(dd[3] & 0xffffu);
            lds16_any(b1 + 196, dd);
            xd[1] = h2f(dd[3] & 0xffffu);
        }
        xm[0] = xm[1] = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) accm[q] = 0.0f;
        const int q0 = t >> 1;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            // planes: sc = 16 hi + lo; half 0 holds 1024 + q, half 1 1024 + 16 q
            uint32_t ml[2], al[2], mh[2], ah[2];   // [row]
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int sa = sbyte_of(scw[rr][2 * h], t), sb = sbyte_of(scw[rr][2 * h + 1], t);
                const float la = (float)(sa & 15), lb = (float)(sb & 15), ha = (float)(sa >> 4), hb = (float)(sb >> 4);
                ml[rr] = h2f32(la, lb * 0.0625f);
                al[rr] = h2f32(-1056.0f * la, -96.0f * lb);
                mh[rr] = h2f32(ha, hb * 0.0625f);
                ah[rr] = h2f32(-1056.0f * ha, -96.0f * hb);
            }
            uint32_t ql[2][4], qh[2][4];
            lds16_any(b0 + 64 * h + 32 * q0 + 16 * (t & 1), ql[0]);
            lds16_any(b1 + 64 * h + 32 * q0 + 16 * (t & 1), ql[1]);
            lds16_any(b0 + 128 + 32 * h + 16 * (t & 1), qh[0]);
            lds16_any(b1 + 128 + 32 * h + 16 * (t & 1), qh[1]);
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                uint32_t alo[4], ahi[4];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    // x: ql bytes l, l+8, l, l+8; y: the same of qh. Element e: low
                    // nibble, qh bits 2 q0; element e + 64: high nibble, qh bits
                    // 2 q0 + 4, kept at 16x (src/kernels.c:497-502)
                    const uint32_t x = pair_j8(ql[rr], l), y = pair_j8(qh[rr], l);
                    const uint32_t ta = and_or(y << (4 - 2 * q0), 0x03000030u, 0x64006400u);
                    const uint32_t tb = and_or(y >> (4 + 2 * q0), 0x03000030u, 0x64006400u);
                    const uint32_t va = and_or(x, 0x00f0000fu, ta);          // (e, e + 64)
                    const uint32_t vb = and_or(x >> 8, 0x00f0000fu, tb);     // (e + 8, e + 72)
                    alo[rr] = hfma2(va, ml[rr], al[rr]);
                    alo[rr + 2] = hfma2(vb, ml[rr], al[rr]);
                    ahi[rr] = hfma2(va, mh[rr], ah[rr]);
                    ahi[rr + 2] = hfma2(vb, mh[rr], ah[rr]);
                }
                const uint4 f = fc[4 * h + (l >> 1)];
                const uint32_t bb0 = (l & 1) ? f.z : f.x, bb1 = (l & 1) ? f.w : f.y;
                mma16816(acc[l], alo[0], alo[1], alo[2], alo[3], bb0, bb1);
                mma16816(acch[l], ahi[0], ahi[1], ahi[2], ahi[3], bb0, bb1);
            }
        }
        // aux32 = lo-plane sum + 16 x hi-plane sum, exact (|result| < 2^24)
#pragma unroll
        for (int l = 0; l < 8; ++l)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[l][q] = __fmaf_rn(16.0f, acch[l][q], acc[l][q]);
    }
}

template <uint32_t T>
__global__ void __launch_bounds__(BT, 2) gemv_batch_kernel(const __grid_constant__ BatchParams p) {
    constexpr int UB = BFmt<T>::ub;
    constexpr bool Q4 = T == T_Q4_K;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int S = p.nstages, R = p.rounds;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);        // [S <= 8] stage landed (bytes)
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + 64);  // [S <= 8] stage released (BW warps)
    float *terms = reinterpret_cast<float *>(smem + 128);
    uint8_t *ring = smem + 128 + TERMS_BYTES;
    const int stage_bytes = 16 * p.rs;
    const int my_tiles = (int)blockIdx.x < p.ntiles ? (p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int Q = my_tiles * R;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(smem_addr(&full[i]), 16);
            mbar_init(smem_addr(&empty[i]), BW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const uint64_t policy = policy_evict_first();
    uint32_t tailmask = 0;

    auto tile_geom = [&](int tile, int &mat, int &row0) {
        mat = 0;
        while (mat + 1 < p.nmat && tile >= p.tile0[mat + 1]) ++mat;
        row0 = (tile - p.tile0[mat]) * 16;
    };
    // round q into stage s: lane r < 16 of warp 0 copies row r's super-blocks of the round
    auto produce = [&](int q, int s) {
        if (lane >= 16) return;
        int mat, row0;
        tile_geom((int)blockIdx.x + (q / R) * (int)gridDim.x, mat, row0);
        const int u0 = (q % R) * BW, cnt = min(BW, p.nb - u0);
        const int row = row0 + lane;
        const uint32_t bar = smem_addr(&full[s]);
        uint8_t *dst = ring + (size_t)s * stage_bytes + (size_t)lane * p.rs;
        if (tailmask & (1u << s)) {
            fence_proxy_async();
            tailmask &= ~(1u << s);
        }
        if (row >= p.n_out[mat]) {
            mbar_expect_tx(bar, 0);
            return;
        }
        const uint8_t *mend = p.w[mat] + (int64_t)p.n_out[mat] * p.row_bytes;
        const uint8_t *src = p.w[mat] + (int64_t)row * p.row_bytes + (int64_t)u0 * UB;
        const int len = cnt * UB;
        const uintptr_t a = reinterpret_cast<uintptr_t>(src);
        const uint8_t *al = reinterpret_cast<const uint8_t *>(a & ~uintptr_t(15));
        const int head = (int)(a & 15);
        int bulk = (head + len + 15) & ~15;
        if (al + bulk > mend) bulk = (int)((mend - al) & ~int64_t(15));
        const int tail = head + len - bulk;
        if (tail > 0) {
            for (int k = 0; k < tail; ++k) dst[bulk + k] = (uint8_t)ldg_u8(al + bulk + k);
            tailmask |= 1u << s;
        }
        mbar_expect_tx(bar, (uint32_t)bulk);
        if (bulk > 0) bulk_g2s_hint(smem_addr(dst), al, (uint32_t)bulk, bar, policy);
    };

    if (warp == BW) {
        // producer: the first stages right away (weights never depend on
        // earlier kernels), then each stage again once the compute warps have
        // released it
        for (int q = 0; q < Q; ++q) {
            const int s = q % S;
            if (q >= S) {
                const bool ok = mbar_wait(smem_addr(&empty[s]), (uint32_t)((q / S - 1) & 1));
                if (!__all_sync(0xffffffffu, ok)) {
                    if (lane == 0) atomicOr(p.status, STATUS_WAIT_TIMEOUT);
                    break;
                }
            }
            produce(q, s);
        }
        return;
    }
    grid_dep_wait();                                          // the activation records do

    // this warp's activation fragments for its next super-block
    uint4 fr[8];
    float yd[2];
    auto load_rec = [&](int u) {
        const uint8_t *r = p.rec + (size_t)u * BREC_BYTES;
#pragma unroll
        for (int k = 0; k < 8; ++k) fr[k] = __ldg(reinterpret_cast<const uint4 *>(r) + 32 * k + lane);
        const float2 dd = __ldg(reinterpret_cast<const float2 *>(r + BREC_YD) + t);
        yd[0] = dd.x;
        yd[1] = dd.y;
    };
    if (Q > 0 && warp < p.nb) load_rec(warp);

    // chain thread: pair tid = (row tid / 8, token tid % 8), its nine chains
    float ch[9];
    int mat = 0, row0 = 0, tile = (int)blockIdx.x;
    int r = 0, s = 0;
    uint32_t sphase = 0;
    bool failed = false;
    for (int q = 0; q < Q; ++q) {
        const int buf = q & 1;
        if (r == 0) {
            tile_geom(tile, mat, row0);
#pragma unroll
            for (int c = 0; c < 9; ++c) ch[c] = 0.0f;
        }
        const int u0 = r * BW, cnt = min(BW, p.nb - u0);
        if (warp < cnt) {
            const bool ok = mbar_wait(smem_addr(&full[s]), sphase);
            if (__all_sync(0xffffffffu, ok)) {
                uint4 fc[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) fc[k] = fr[k];
                const float ydc0 = yd[0], ydc1 = yd[1];
                const uint8_t *stage = ring + (size_t)s * stage_bytes;
                const uint8_t *w0 = p.w[mat] + (int64_t)(row0 + g) * p.row_bytes + (int64_t)u0 * UB;
                const uint8_t *w1 = w0 + 8 * p.row_bytes;
                const uint8_t *b0 = stage + (size_t)g * p.rs + (reinterpret_cast<uintptr_t>(w0) & 15) + warp * UB;
                const uint8_t *b1 = stage + (size_t)(g + 8) * p.rs + (reinterpret_cast<uintptr_t>(w1) & 15) + warp * UB;
                float acc[8][4], accm[4], xd[2], xm[2];
                batch_superblock<T>(b0, b1, fc, t, acc, accm, xd, xm);
                // the reference's float terms of this super-block (src/kernels.c:405-407)
                float *tl = terms + (size_t)(buf * BW + warp) * NPAIR * 8;
                float *tm = terms + TERMS_LANE_FLOATS + (size_t)(buf * BW + warp) * NPAIR;
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
                    for (int n = 0; n < 2; ++n) {
                        const int q4 = 2 * rr + n, pi = (g + 8 * rr) * BATCH_MAX + 2 * t + n;
                        const float ydn = n ? ydc1 : ydc0;
                        const float d = __fmul_rn(xd[rr], ydn);
                        float4 *dst = reinterpret_cast<float4 *>(tl + pi * 8);
                        dst[0] = make_float4(__fmul_rn(d, acc[0][q4]), __fmul_rn(d, acc[1][q4]),
                                             __fmul_rn(d, acc[2][q4]), __fmul_rn(d, acc[3][q4]));
                        dst[1] = make_float4(__fmul_rn(d, acc[4][q4]), __fmul_rn(d, acc[5][q4]),
                                             __fmul_rn(d, acc[6][q4]), __fmul_rn(d, acc[7][q4]));
                        // sumf -= dmin * sumi, stored negated: a - b == a + (-b) in IEEE arithmetic
                        if (Q4) tm[pi] = -__fmul_rn(__fmul_rn(xm[rr], ydn), accm[q4]);
                    }
                }
            } else {
                failed = true;
            }
        }
        // this warp is done with the stage (every compute warp releases it,
        // with or without a super-block in it)
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&empty[s]));
        // terms written by every compute warp. No load of this thread is in
        // flight here (a barrier waits for them), so the next round's loads
        // are issued after it.
        if (compute_bar_or(failed)) {
            failed = true;
            break;
        }
        {
            const int rn = r + 1 == R ? 0 : r + 1;
            const int un = rn * BW + warp;
            if (q + 1 < Q && un < p.nb) load_rec(un);
        }
        // chains: the round's super-blocks in order
        for (int w = 0; w < cnt; ++w) {
            const float4 *tl = reinterpret_cast<const float4 *>(terms + ((size_t)(buf * BW + w) * NPAIR + tid) * 8);
            const float4 v0 = tl[0], v1 = tl[1];
            ch[0] = __fadd_rn(ch[0], v0.x); ch[1] = __fadd_rn(ch[1], v0.y);
            ch[2] = __fadd_rn(ch[2], v0.z); ch[3] = __fadd_rn(ch[3], v0.w);
            ch[4] = __fadd_rn(ch[4], v1.x); ch[5] = __fadd_rn(ch[5], v1.y);
            ch[6] = __fadd_rn(ch[6], v1.z); ch[7] = __fadd_rn(ch[7], v1.w);
            if (Q4) ch[8] = __fadd_rn(ch[8], terms[TERMS_LANE_FLOATS + (size_t)(buf * BW + w) * NPAIR + tid]);
        }
        if (r == R - 1) {
            // sumf (the dmin chain; Q6_K: 0) + sums[0..7] (src/kernels.c:408, 521)
            float out = Q4 ? ch[8] : 0.0f;
#pragma unroll
            for (int l = 0; l < 8; ++l) out = __fadd_rn(out, ch[l]);
            const int row = row0 + (tid >> 3), tok = tid & 7;
            if (row < p.n_out[mat] && tok < p.m) p.y[mat][(size_t)tok * p.n_out[mat] + row] = out;
        }
        if (++s == S) {
            s = 0;
            sphase ^= 1u;
        }
        if (++r == R) {
            r = 0;
            tile += (int)gridDim.x;
        }
    }
    if (failed) {
        if (tid == 0) atomicOr(p.status, STATUS_WAIT_TIMEOUT);
        // let copies still in flight land before the CTA's memory goes away
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
    }
}

}  // namespace

bool batch_supported(uint32_t wtype) { return wtype == T_Q4_K || wtype == T_Q6_K; }

size_t batch_workspace_bytes(int64_t n_in) { return (size_t)(n_in / 256) * BREC_BYTES; }

template <uint32_t T>
static int launch_batch_t(const BatchLaunch &L, cudaStream_t st) {
    constexpr int UB = BFmt<T>::ub;
    BatchParams p{};
    p.nmat = L.nmat;
    p.rec = static_cast<const uint8_t *>(L.ws);
    p.nb = (int)(L.n_in / 256);
    p.row_bytes = (int64_t)p.nb * UB;
    p.rounds = (p.nb + BW - 1) / BW;
    p.m = L.m;
    p.status = L.status;
    int tiles = 0;
    for (int i = 0; i < L.nmat; ++i) {
        p.w[i] = static_cast<const uint8_t *>(L.w[i]);
        p.y[i] = L.y[i];
        p.n_out[i] = (int)L.n_out[i];
        p.tile0[i] = tiles;
        tiles += (int)((L.n_out[i] + 15) / 16);
    }
    p.tile0[L.nmat] = tiles;
    p.ntiles = tiles;
    if (tiles == 0) return 0;
    // a stage holds a round's four super-blocks of 16 rows, each row's piece
    // with alignment slack (Q4_K: the row size in 16-byte units kept at 2..6
    // (mod 8), so the rows' 16-byte reads fall into distinct bank groups)
    const int cu = p.nb < BW ? p.nb : BW;
    int rs = (cu * UB + 32 + 15) & ~15;
    if (T == T_Q4_K)
        while (((rs >> 4) & 7) < 2 || ((rs >> 4) & 7) > 6) rs += 16;
    p.rs = rs;
    const int stage = 16 * rs;
    // two CTAs per SM (the compute warps need ~168 registers: with the
    // producer warp, three CTAs would leave them 128 and spill), at most
    // eight stages each
    int per_sm = 2, stages = 0;
    for (; per_sm >= 2; --per_sm) {
        const int budget = L.smem_per_sm / per_sm - L.smem_reserved - 128 - TERMS_BYTES;
        stages = budget / stage;
        if (stages >= 3) break;
    }
    if (stages > 8) stages = 8;
    if (stages < 2) return -1;
    p.nstages = stages;
    const int smem = 128 + TERMS_BYTES + stages * stage;
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    auto kern = gemv_batch_kernel<T>;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
            return -2;
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        attr_set[dev] = true;
    }
    int64_t grid = (int64_t)per_sm * L.num_sms;
    if (tiles < grid) grid = tiles;

    // the prep kernel: records of the m activation rows
    {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)p.nb);
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = L.overlap ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        uint8_t *rec = static_cast<uint8_t *>(L.ws);
        const int n_in = (int)L.n_in, m = L.m;
        cudaError_t e = L.xf ? cudaLaunchKernelEx(&cfg, batch_prep_kernel<true>, L.xf, (const uint8_t *)nullptr, n_in,
                                                  m, rec)
                             : cudaLaunchKernelEx(&cfg, batch_prep_kernel<false>, (const float *)nullptr,
                                                  static_cast<const uint8_t *>(L.xq), n_in, m, rec);
        if (e != cudaSuccess) return -2;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(BT);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;   // streams weights while the prep runs
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return -2;
    return 0;
}

int launch_batch(uint32_t wtype, const BatchLaunch &L, cudaStream_t st) {
    if (L.nmat < 1 || L.nmat > BATCH_MATS || L.m < 1 || L.m > BATCH_MAX) return -1;
    switch (wtype) {
        case T_Q4_K: return launch_batch_t<T_Q4_K>(L, st);
        case T_Q6_K: return launch_batch_t<T_Q6_K>(L, st);
        default: return -3;
    }
}

}  // namespace sicu
