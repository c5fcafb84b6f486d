// Prefill matrix product on the 5th-generation tensor cores: Y = X W^T for a
// block of m >= 64 tokens, X quantized to Q8_K rows, W in its GGUF K-quant
// blocks. Y[t][r] is the reference's per-row dot product (for Q4_K,
// si_dot_q4_K_q8_K, src/kernels.c:349-410; Q6_K, si_dot_q6_K_q8_K,
// src/kernels.c:480-523) for every (token, row) pair:
//
//   Y[t][r] = sum_sb dA[t][sb] * ( d[r][sb] * S1 - dmin[r][sb] * S2 )
//   S1 = sum_k (sc * q)[r][k] * qa[t][k]                         (256 k)
//   S2 = sum_j mn[r][j] * (bsums[t][2j] + bsums[t][2j+1])         (Q4_K only)
//
// S1's factors are small integers that f16 holds exactly (sc * q <= 945 for
// Q4_K; Q6_K's (q - 32) * sc is split into two exact planes), so kind::f16
// MMAs with f32 accumulation produce the integer sums. The dmin term joins the
// same accumulator: with f = d * 2^s (s >= 0 the smallest that keeps the mins
// in f16 range) the super-block is f * (sum_k (sc q 2^-s) qa - sum_i
// (dmin / f) mn[i/2] bsums[i]), the mins factor split into two f16 parts
// (hi + lo, 22 bits). Outputs agree with the reference within a relative 1e-5
// of the L1 norm of the products.
//
// One CTA computes a 128-row x 128-token tile (one SM; 19 warps):
//   warp 0      TMA: token operand (f16, 128-byte swizzle), bsums, dA
//   warp 1      TMEM owner; lane 0 issues the MMAs
//   warp 2      TMA of raw weight super-blocks (one 128-row tile of GGUF
//               block bytes per super-block)
//   warps 3-10  weight converters: raw blocks -> f16 weights written straight
//               into tensor memory (the MMA's A operand), the mins operand
//               and the per-row scale f; thread = one row; the two groups of
//               four warps convert alternate K-steps, so two are in flight
//   warps 11-18 epilogue: per super-block, the accumulator from tensor memory,
//               scaled by f * dA and added in registers; Y written at the end
//               (two warps per 32-lane quarter of tensor memory, 64 tokens each)
// Tensor memory (512 columns): two accumulators (128 columns each), so the
// MMAs of super-block sb+1 run while the epilogue drains sb; four 32-column A
// stages (64 k each); four 16-column mins operands. Only the token operand
// and the raw blocks pass through shared memory.
#include <cudaTypedefs.h>

#include "launch.h"
#include "quantize.cuh"
#include "tc.cuh"

namespace sicu {

namespace {

constexpr int PF_BM = 128;        // weight rows per tile (MMA M)
constexpr int PF_BN = 128;        // tokens per tile (MMA N) for prompts
constexpr int PF_BN_SMALL = 32;   // tokens per tile for blocks of <= 32 tokens (batched decode)
static_assert(PF_BN_SMALL == PREFILL_PACKED_MIN_M, "blocks above one small tile read the prefill copies");
constexpr int PF_KS = 64;         // k slots per pipeline stage: one 128-byte swizzle atom of f16
constexpr int PF_STAGES = 6;     // K-steps in flight (even: each stage belongs to one converter group)
constexpr int PF_NSB = 4;         // per-super-block buffers: mins / bsums tiles, scales
// token stage: BN rows x 64 f16 (128-byte swizzle); bsums tile: BN rows x 16 f16 (32-byte swizzle)
__host__ __device__ constexpr int stage_bytes(int bn) { return bn * PF_KS * 2; }
__host__ __device__ constexpr int min_bytes(int bn) { return bn * 16 * 2; }

constexpr int W_TMA = 0, W_MMA = 1, W_RAW = 2, W_CONV = 3, N_CONV = 8, W_EPI = 11, N_EPI = 8;
constexpr int PF_WARPS = 19;

// Per-format geometry of the prefill kernel.
//   KSTEPS  64-slot K-steps per super-block (weight slots = 64 * KSTEPS)
//   RAW_ROW bytes per row of a raw weight tile (TMA box width; the 16-byte
//           aligned span that holds the row's super-block)
//   MINS    the format has a dmin * mins term (second accumulator)
template <uint32_t T> struct PfFmt;
// Q4_K: one f16 plane (sc * q); slots of K-step c = elements 64c..64c+63
template <> struct PfFmt<T_Q4_K> {
    static constexpr int BLOCK = B_Q4_K, RAW_ROW = 144, KSTEPS = 4, NRAW = 3;
    static constexpr bool MINS = true;
};
// Q6_K: (q - 32) * sc with int8 sc = 16 hi + lo is split into two exact f16
// planes, (q - 32) * lo against x and (q - 32) * hi against 16 x; K-steps 2c
// and 2c+1 hold the two planes of elements 64c..64c+63. A super-block starts
// at any even byte: the raw row is the 240-byte aligned span around it (an
// odd number of 16-byte units, so 16-byte shared loads of consecutive rows
// are free of bank conflicts).
template <> struct PfFmt<T_Q6_K> {
    static constexpr int BLOCK = B_Q6_K, RAW_ROW = 240, KSTEPS = 8, NRAW = 2;
    static constexpr bool MINS = false;
};

template <uint32_t T, int BN> struct PfLayout {
    using F = PfFmt<T>;
    static constexpr int RAW_BUF = PF_BM * F::RAW_ROW;
    static constexpr int OFF_B = 0;
    static constexpr int OFF_RAW = OFF_B + PF_STAGES * stage_bytes(BN);
    static constexpr int MINB = F::MINS ? PF_NSB * min_bytes(BN) : 0;
    static constexpr int OFF_B2 = (OFF_RAW + F::NRAW * RAW_BUF + 1023) & ~1023;
    static constexpr int OFF_DA = OFF_B2 + MINB;
    static constexpr int OFF_DW = OFF_DA + PF_NSB * BN * 4;             // per-row scale f
    static constexpr int OFF_BAR = OFF_DW + PF_NSB * PF_BM * 4;
    static constexpr int OFF_FLAGS = OFF_BAR + 8 * 64;     // abort flag, TMEM address
    static constexpr int SMEM = OFF_FLAGS + 16 + 1024;     // + alignment slack
};

// barriers
enum {
    BAR_B_FULL = 0,                          // [S] token stage landed (TMA bytes)
    BAR_A_FULL = BAR_B_FULL + PF_STAGES,     // [S] weight stage converted (the 4 warps of one group)
    BAR_ST_EMPTY = BAR_A_FULL + PF_STAGES,   // [S] stage consumed by the MMAs (commit)
    BAR_RAW_FULL = BAR_ST_EMPTY + PF_STAGES, // [3] raw super-block landed (TMA bytes)
    BAR_RAW_EMPTY = BAR_RAW_FULL + 3,        // [3] raw super-block converted (8 warps)
    BAR_SBD_FULL = BAR_RAW_EMPTY + 3,        // [4] bsums tile + dA landed (TMA bytes)
    BAR_A2_FULL = BAR_SBD_FULL + PF_NSB,     // [4] mins operand, row scales written (group 0, 4 warps)
    BAR_SB_FREE = BAR_A2_FULL + PF_NSB,      // [4] epilogue done with a super-block (8 warps)
    BAR_ACC_FULL = BAR_SB_FREE + PF_NSB,     // [2] accumulators of a super-block ready (commit)
    BAR_ACC_EMPTY = BAR_ACC_FULL + 2,        // [2] accumulators read (8 warps)
    BAR_DRAIN = BAR_ACC_EMPTY + 2,           // teardown after an abandoned wait
    NBARS = BAR_DRAIN + 1,
};
static_assert(NBARS <= 64, "barrier area");
constexpr uint32_t PF_TMEM_COLS = 512;
// tensor-memory columns
constexpr uint32_t TM_ACC = 0;      // accumulators: 128 * buf
constexpr uint32_t TM_A = 256;      // A stages: 32 * stage
constexpr uint32_t TM_MIN = TM_A + 32 * PF_STAGES;   // mins operands: 16 * (sb % PF_NSB): 8 columns hi, 8 lo
static_assert(TM_MIN + 16 * PF_NSB <= PF_TMEM_COLS, "tensor-memory columns");
static_assert(PF_STAGES % 2 == 0, "stages alternate between the two converter groups");
// pipeline stage of K-step t and the parity of its use
__device__ __forceinline__ int stage_of(int t) { return t % PF_STAGES; }
__device__ __forceinline__ uint32_t use_of(int t) { return (uint32_t)(t / PF_STAGES) & 1u; }

struct PfParams {
    int n_out;
    int nsb;              // super-blocks per row
    int nsplit;           // the row's super-blocks split into this many ranges (one CTA each)
    int sb_per_split;
    float *part;          // nsplit > 1: [nsplit][m][n_out] partial products, summed afterwards
    const float *da;      // [nsb][m_pad] token scales
    float *y;             // [m][n_out]
    int m, m_pad;
    int ntt;              // token tiles
    int *status;
};

// Bounded wait shared by all roles: gives up when another role already gave
// up, or after 2 s, recording the failure in the status word. Roles other
// than the MMA issuer wait suspended (a suspend-time hint), so they take no
// issue slots from the warps that share their scheduler (the MMA issuer's
// warp among them); the MMA issuer polls.
template <bool POLL = false>
__device__ __forceinline__ bool pf_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *status) {
    if (mbar_poll(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!(POLL ? mbar_poll(bar, parity) : mbar_try_wait(bar, parity))) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            *abort_flag = 1;
            atomicOr(status, STATUS_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}
// after an abandoned pipeline: let a copy that may still be in flight land
__device__ __forceinline__ void pf_settle(uint32_t bar, uint32_t parity) {
    (void)mbar_wait(bar, parity, 200000000ull);
}

__device__ __forceinline__ uint32_t byte_at(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }

// f16 pair (1024 + q0, 1024 + q2) from the low nibbles of bytes 0 and 2 of x
// (mask 0x000f000f) or 1024 + 16 q from the high nibbles (mask 0x00f000f0),
// then one fused multiply-add per pair removes the 1024 bias exactly:
// (1024 + q) * sc - 1024 * sc = q * sc, and (1024 + 16 q) * sc/16 - 64 * sc.
__device__ __forceinline__ uint32_t nib_f16(uint32_t x, uint32_t mask, uint32_t mul, uint32_t add) {
    return hfma2_u32(and_or(x, mask, 0x64006400u), mul, add);
}

// N words of a shared-memory span that starts at byte `head` (even, < 16)
// of 16-byte aligned address a: loads the (N + 7) / 4 aligned 16-byte units
// that cover it and funnels. head is the same for every thread of the CTA.
template <int N>
__device__ __forceinline__ void span_words(uint32_t a, int head, uint32_t (&W)[N]) {
    constexpr int U = (N + 7) / 4;
    uint32_t w[4 * U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint4 v = lds128(a + 16 * u);
        w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
    }
    const uint32_t sh = (uint32_t)(head & 2) * 8;
    switch (head >> 2) {
        case 0:
#pragma unroll
            for (int k = 0; k < N; ++k) W[k] = funnel(w[k], w[k + 1], sh);
            break;
        case 1:
#pragma unroll
            for (int k = 0; k < N; ++k) W[k] = funnel(w[k + 1], w[k + 2], sh);
            break;
        case 2:
#pragma unroll
            for (int k = 0; k < N; ++k) W[k] = funnel(w[k + 2], w[k + 3], sh);
            break;
        default:
#pragma unroll
            for (int k = 0; k < N; ++k) W[k] = funnel(w[k + 3], w[k + 4], sh);
            break;
    }
}

// Q4_K super-block header h (d, dmin, 12 bytes of packed scales and mins,
// src/kernels.c:377-382): the exponent s of the row scale f = d 2^s, s >= 0
// the smallest that keeps (dmin / f) * mn inside f16 range; keep_main is
// false when d is zero or negligible (s > 14) and only the mins term is kept.
__device__ __forceinline__ void q4k_scale_exp(const uint4 &h, int &sexp, bool &keep_main) {
    const uint32_t mn_lo = h.z & 0x3f3f3f3fu;
    const uint32_t mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
    const float d = h2f(h.x & 0xffffu), dmin = h2f(h.x >> 16);
    uint32_t mn_max = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) mn_max = max(mn_max, max(byte_at(mn_lo, j), byte_at(mn_hi, j)));
    sexp = 0;
    keep_main = d != 0.0f;
    if (keep_main) {
        const float ratio = fabsf(dmin) * (float)mn_max / (60000.0f * fabsf(d));
        if (ratio > 1.0f) sexp = ilogbf(ratio) + 1;
        if (sexp > 14) keep_main = false;
    }
}

// The row scale f and the mins operand: 16 k (the bsums index i, mn[i / 2])
// as -(hi + lo) of (dmin / f) mn, the hi parts in words 0-7, the lo parts in
// 8-15, two equal f16 per word (k = 2j, 2j + 1).
__device__ __forceinline__ void q4k_mins_words(const uint4 &h, int sexp, bool keep_main, bool valid, float &f,
                                               uint32_t (&mw)[16]) {
    const uint32_t mn_lo = h.z & 0x3f3f3f3fu;
    const uint32_t mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
    const float d = h2f(h.x & 0xffffu), dmin = h2f(h.x >> 16);
    f = keep_main ? ldexpf(d, sexp) : ldexpf(dmin, -10);
    const float mfac = f != 0.0f ? dmin / f : 0.0f;
    if (!valid) f = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float mu = mfac * (float)byte_at(c < 4 ? mn_lo : mn_hi, c & 3);
        const float hi = __half2float(__float2half_rn(mu));
        mw[c] = valid ? half2_bits(-hi, -hi) : 0u;
        mw[8 + c] = valid ? half2_bits(hi - mu, hi - mu) : 0u;
    }
}

// K-step c of a Q4_K super-block (qs[32c..32c+31] in x: low nibbles =
// sub-block 2c, high = 2c+1) as 64 f16 slots (sc q 2^-s): words 0-15 sub-block
// 2c, 16-31 sub-block 2c+1; slot order inside each group of four elements:
// 0, 2, 1, 3. on = false gives zeros.
__device__ __forceinline__ void q4k_kstep_words(const uint4 &h, const uint32_t (&x)[8], int c, int sexp, bool on,
                                                uint32_t (&w)[32]) {
    const uint32_t sc_lo = h.y & 0x3f3f3f3fu;
    const uint32_t sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t scw = c < 2 ? sc_lo : sc_hi;
    const float s0 = on ? ldexpf((float)byte_at(scw, (2 * c) & 3), -sexp) : 0.0f;
    const float s1 = on ? ldexpf((float)byte_at(scw, (2 * c + 1) & 3), -sexp) : 0.0f;
    // (1024 + q) * sc - 1024 sc for the low nibbles, (1024 + 16 q) * sc/16 -
    // 64 sc for the high ones: exact
    const uint32_t mul0 = half2_bits(s0, s0), add0 = half2_bits(-1024.0f * s0, -1024.0f * s0);
    const uint32_t mul1 = half2_bits(0.0625f * s1, 0.0625f * s1), add1 = half2_bits(-64.0f * s1, -64.0f * s1);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        w[2 * k] = nib_f16(x[k], 0x000f000fu, mul0, add0);
        w[2 * k + 1] = nib_f16(x[k] >> 8, 0x000f000fu, mul0, add0);
        w[16 + 2 * k] = nib_f16(x[k], 0x00f000f0u, mul1, add1);
        w[16 + 2 * k + 1] = nib_f16(x[k] >> 8, 0x00f000f0u, mul1, add1);
    }
}

// Quarter cq of a Q6_K super-block (src/kernels.c:480-523) as the two exact
// f16 planes, (q - 32) lo (p0) and (q - 32) hi (p1) with sc = 16 hi + lo.
// row: shared-memory address of the 16-byte aligned span holding the block
// from byte `head` on; S: its scale words (bytes 192..211). Quarter cq (h =
// cq / 2) element 32g + l (g = 0, 1; group G' = 2 (cq & 1) + g of half h):
// ql[64h + 32g + l] (low nibble for even cq, high for odd), qh[32h + l] bits
// 2G'..2G'+1, scale sc[4cq + 2g + l / 16].
__device__ __forceinline__ void q6k_quarter_words(uint32_t row, int head, const uint32_t (&S)[5], bool valid,
                                                  int cq, uint32_t (&p0)[32], uint32_t (&p1)[32]) {
    const int h = cq >> 1;
    const int nsh = (cq & 1) ? 4 : 0;
    uint32_t QH[8];
    span_words<8>(row + 128 + 32 * h, head, QH);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const int Gp = 2 * (cq & 1) + g;
        uint32_t QL[8];
        span_words<8>(row + 64 * h + 32 * g, head, QL);
        // the two 16-element sub-blocks of these 32 elements
        const int sbi = 4 * cq + 2 * g;
        const int sa = (int)(int8_t)byte_at(S[sbi >> 2], sbi & 3);
        const int sb2 = (int)(int8_t)byte_at(S[(sbi + 1) >> 2], (sbi + 1) & 3);
        const int sv[2] = {valid ? sa : 0, valid ? sb2 : 0};
        uint32_t mul0[2], add0[2], mul1[2], add1[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float lo = (float)(sv[i] & 15), hi = (float)(sv[i] >> 4);   // sc = 16 hi + lo
            mul0[i] = half2_bits(lo, lo);
            add0[i] = half2_bits(-1056.0f * lo, -1056.0f * lo);              // (1024 + q) lo - 1056 lo
            mul1[i] = half2_bits(hi, hi);
            add1[i] = half2_bits(-1056.0f * hi, -1056.0f * hi);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = k >> 2;   // sub-block of word k
            // 6-bit q of elements 4k..4k+3, one per byte
            const uint32_t q = ((QL[k] >> nsh) & 0x0f0f0f0fu) | (((QH[k] >> (2 * Gp)) & 0x03030303u) << 4);
            const uint32_t e02 = and_or(q, 0x00ff00ffu, 0x64006400u);
            const uint32_t e13 = and_or(q >> 8, 0x00ff00ffu, 0x64006400u);
            p0[16 * g + 2 * k] = hfma2_u32(e02, mul0[i], add0[i]);
            p0[16 * g + 2 * k + 1] = hfma2_u32(e13, mul0[i], add0[i]);
            p1[16 * g + 2 * k] = hfma2_u32(e02, mul1[i], add1[i]);
            p1[16 * g + 2 * k + 1] = hfma2_u32(e13, mul1[i], add1[i]);
        }
    }
}

struct PfCtx {
    uint32_t sb0;
    uint8_t *smem;
    volatile int *abort_flag;
    int *status;
};

// Q4_K converter for one super-block. Thread: tile row r (tensor-memory lane
// of this warp's quarter); converter group G converts the K-steps c with
// c % 2 == G (c: qs[32c..32c+31], low nibbles = sub-block 2c, high = 2c+1).
// Group 0 also writes the mins operand and the row scale. tl = this warp's
// lane base in tensor memory.
template <class Lay>
__device__ __forceinline__ bool convert_q4k(const PfCtx &cx, uint32_t base, uint32_t tl, int sb, int rb, int b4,
                                            int r, int G, bool valid, uint32_t barbase) {
    constexpr uint32_t FULL = 0xffffffffu;
    auto bar = [&](int i) { return barbase + 8u * (uint32_t)i; };
    const uint32_t raw = base + Lay::OFF_RAW + rb * Lay::RAW_BUF + r * B_Q4_K;
    const uint4 h = valid ? lds128(raw) : make_uint4(0, 0, 0, 0);
    int sexp;
    bool keep_main;
    q4k_scale_exp(h, sexp, keep_main);
    if (G == 0) {
        float f;
        uint32_t mw[16];
        q4k_mins_words(h, sexp, keep_main, valid, f, mw);
        reinterpret_cast<float *>(cx.smem + Lay::OFF_DW)[b4 * PF_BM + r] = f;
        tc_fence_after();
        tmem_st16(tl + TM_MIN + 16 * b4, mw);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(bar(BAR_A2_FULL + b4));
    }
    for (int c = G; c < 4; c += 2) {
        const int t = 4 * sb + c, s = stage_of(t);
        if (!__all_sync(FULL, pf_wait(bar(BAR_ST_EMPTY + s), use_of(t) ^ 1, cx.abort_flag, cx.status)))
            return false;
        const uint4 q0 = lds128(raw + 16 + 32 * c), q1 = lds128(raw + 32 + 32 * c);
        const uint32_t x[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t w[32];
        q4k_kstep_words(h, x, c, sexp, valid && keep_main, w);
        tc_fence_after();
        tmem_st32(tl + TM_A + 32 * s, w);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(bar(BAR_A_FULL + s));
    }
    return true;
}

// Q6_K converter for one super-block (src/kernels.c:480-523). Thread: tile
// row r; converter group G converts the quarters cq (64 elements, K-steps
// 2cq and 2cq+1: the two planes) with cq % 2 == G. Quarter cq (h = cq / 2)
// element 32g + l (g = 0, 1; group G' = 2 (cq & 1) + g of half h):
// ql[64h + 32g + l] (low nibble for even cq, high for odd), qh[32h + l] bits
// 2G'..2G'+1, scale sc[4cq + 2g + l / 16].
template <class Lay>
__device__ __forceinline__ bool convert_q6k(const PfCtx &cx, uint32_t base, uint32_t tl, int sb, int gsb, int rb,
                                            int b4, int r, int G, bool valid, uint32_t barbase) {
    constexpr uint32_t FULL = 0xffffffffu;
    auto bar = [&](int i) { return barbase + 8u * (uint32_t)i; };
    const int head = (int)(((int64_t)gsb * B_Q6_K) & 15);
    const uint32_t row = base + Lay::OFF_RAW + rb * Lay::RAW_BUF + r * PfFmt<T_Q6_K>::RAW_ROW;
    // scales (bytes 192..207) and d (208..209)
    uint32_t S[5];
    span_words<5>(row + 192, head, S);
    if (!valid) {
#pragma unroll
        for (int k = 0; k < 5; ++k) S[k] = 0;
    }
    if (G == 0) {
        reinterpret_cast<float *>(cx.smem + Lay::OFF_DW)[b4 * PF_BM + r] = h2f(S[4] & 0xffffu);
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(bar(BAR_A2_FULL + b4));
    }
    for (int cq = G; cq < 4; cq += 2) {
        const int t0 = 8 * sb + 2 * cq, s0 = stage_of(t0), s1 = stage_of(t0 + 1);
        if (!__all_sync(FULL, pf_wait(bar(BAR_ST_EMPTY + s0), use_of(t0) ^ 1, cx.abort_flag, cx.status) &&
                                  pf_wait(bar(BAR_ST_EMPTY + s1), use_of(t0 + 1) ^ 1, cx.abort_flag, cx.status)))
            return false;
        uint32_t p0[32], p1[32];
        q6k_quarter_words(row, head, S, valid, cq, p0, p1);
        tc_fence_after();
        tmem_st32(tl + TM_A + 32 * s0, p0);
        tmem_st32(tl + TM_A + 32 * s1, p1);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) {
            mbar_arrive(bar(BAR_A_FULL + s0));
            mbar_arrive(bar(BAR_A_FULL + s1));
        }
    }
    return true;
}

template <uint32_t T, int BN>
__global__ void __launch_bounds__(PF_WARPS * 32, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmS, const PfParams p) {
    using F = PfFmt<T>;
    using Lay = PfLayout<T, BN>;
    constexpr int KST = F::KSTEPS;
    constexpr int EPI_COLS = BN / 2;   // token columns per epilogue warp
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb0 = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // blockIdx: split-major over (row tile, token tile); this CTA's super-blocks
    // are sbb .. sbb + nsb - 1 (sb below counts from 0 within them)
    const int ntiles = (int)(gridDim.x / (unsigned)p.nsplit);
    const int split = blockIdx.x / ntiles, tile = blockIdx.x - split * ntiles;
    const int rt = tile / p.ntt, tt = tile - rt * p.ntt;
    const int row0 = rt * PF_BM, tok0 = tt * BN;
    const int rows = min(PF_BM, p.n_out - row0);
    const int sbb = split * p.sb_per_split;
    const int nsb = min(p.sb_per_split, p.nsb - sbb);
    float *const yout = p.nsplit > 1 ? p.part + (size_t)split * p.m * p.n_out : p.y;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + Lay::OFF_FLAGS);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Lay::OFF_FLAGS + 4);
    const uint32_t barbase = sb0 + Lay::OFF_BAR;
    auto bar = [&](int i) { return barbase + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STAGES; ++i) {
            mbar_init(bar(BAR_B_FULL + i), 1);
            mbar_init(bar(BAR_A_FULL + i), N_CONV / 2);
            mbar_init(bar(BAR_ST_EMPTY + i), 1);
        }
        for (int i = 0; i < F::NRAW; ++i) {
            mbar_init(bar(BAR_RAW_FULL + i), 1);
            mbar_init(bar(BAR_RAW_EMPTY + i), N_CONV);
        }
        for (int i = 0; i < PF_NSB; ++i) {
            mbar_init(bar(BAR_SBD_FULL + i), 1);
            mbar_init(bar(BAR_A2_FULL + i), N_CONV / 2);
            mbar_init(bar(BAR_SB_FREE + i), N_EPI);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(BAR_ACC_FULL + i), 1);
            mbar_init(bar(BAR_ACC_EMPTY + i), N_EPI);
        }
        mbar_init(bar(BAR_DRAIN), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) tmem_alloc(smem_addr(tmem_slot), PF_TMEM_COLS);
    if (warp == W_TMA && lane == 0) {
        tma_prefetch_map(&tmW);
        tma_prefetch_map(&tmB);
        if constexpr (F::MINS) tma_prefetch_map(&tmS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t FULL = 0xffffffffu;

    if (warp == W_TMA) {
        // ---- token operand, bsums and token scales ----
        if (lane == 0) {
            int t_issued = 0, sb_issued = 0;
            for (int sb = 0; sb < nsb; ++sb) {
                const int b4 = sb % PF_NSB;
                if (!pf_wait(bar(BAR_SB_FREE + b4), ((sb / PF_NSB) & 1) ^ 1, abort_flag, p.status)) break;
                mbar_expect_tx(bar(BAR_SBD_FULL + b4), (F::MINS ? min_bytes(BN) : 0) + BN * 4);
                if constexpr (F::MINS)
                    tma_load_2d(sb0 + Lay::OFF_B2 + b4 * min_bytes(BN), &tmS, 16 * (sbb + sb), tok0, bar(BAR_SBD_FULL + b4));
                bulk_g2s(sb0 + Lay::OFF_DA + b4 * BN * 4, p.da + (size_t)(sbb + sb) * p.m_pad + tok0, BN * 4,
                         bar(BAR_SBD_FULL + b4));
                sb_issued = sb + 1;
                bool ok = true;
                for (int c = 0; c < KST; ++c) {
                    const int t = KST * sb + c, s = stage_of(t);
                    if (!pf_wait(bar(BAR_ST_EMPTY + s), use_of(t) ^ 1, abort_flag, p.status)) { ok = false; break; }
                    mbar_expect_tx(bar(BAR_B_FULL + s), stage_bytes(BN));
                    tma_load_2d(sb0 + Lay::OFF_B + s * stage_bytes(BN), &tmB, PF_KS * (KST * sbb + t), tok0,
                                bar(BAR_B_FULL + s));
                    t_issued = t + 1;
                }
                if (!ok) break;
            }
            if (*abort_flag) {
                for (int t = max(0, t_issued - PF_STAGES); t < t_issued; ++t) pf_settle(bar(BAR_B_FULL + stage_of(t)), use_of(t));
                for (int sb = max(0, sb_issued - PF_NSB); sb < sb_issued; ++sb)
                    pf_settle(bar(BAR_SBD_FULL + sb % PF_NSB), (sb / PF_NSB) & 1);
            }
        }
    } else if (warp == W_MMA) {
        // ---- MMA issue ----
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(PF_BM, BN);
            for (int sb = 0; sb < nsb; ++sb) {
                const int buf = sb & 1;
                const uint32_t ph = (sb >> 1) & 1;
                if (!pf_wait<true>(bar(BAR_ACC_EMPTY + buf), ph ^ 1, abort_flag, p.status)) break;
                tc_fence_after();
                const uint32_t dacc = tmem + TM_ACC + (uint32_t)buf * 128u;
                bool ok = true;
                for (int c = 0; c < KST; ++c) {
                    const int t = KST * sb + c, s = stage_of(t);
                    const uint32_t sph = use_of(t);
                    if (!pf_wait<true>(bar(BAR_A_FULL + s), sph, abort_flag, p.status) ||
                        !pf_wait<true>(bar(BAR_B_FULL + s), sph, abort_flag, p.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t b = sb0 + Lay::OFF_B + s * stage_bytes(BN);
#pragma unroll
                    for (int kk = 0; kk < PF_KS / 16; ++kk)
                        tc_mma_f16_ts(dacc, tmem + TM_A + 32u * s + 8u * kk, smem_desc(b + 32 * kk, 1024, SMEM_SWZ_128B),
                                      idesc, (c | kk) != 0);
                    tc_commit(bar(BAR_ST_EMPTY + s));
                }
                if (!ok) break;
                if constexpr (F::MINS) {
                    // the mins term, into the same accumulator: -(hi + lo) x bsums
                    const int b4 = sb % PF_NSB;
                    const uint32_t ph4 = (sb / PF_NSB) & 1;
                    if (!pf_wait<true>(bar(BAR_A2_FULL + b4), ph4, abort_flag, p.status) ||
                        !pf_wait<true>(bar(BAR_SBD_FULL + b4), ph4, abort_flag, p.status)) break;
                    tc_fence_after();
                    const uint64_t bd = smem_desc(sb0 + Lay::OFF_B2 + b4 * min_bytes(BN), 256, SMEM_SWZ_32B);
                    tc_mma_f16_ts(dacc, tmem + TM_MIN + 16u * b4, bd, idesc, 1);
                    tc_mma_f16_ts(dacc, tmem + TM_MIN + 16u * b4 + 8u, bd, idesc, 1);
                }
                tc_commit(bar(BAR_ACC_FULL + buf));
            }
            if (*abort_flag) {
                tc_commit(bar(BAR_DRAIN));
                pf_settle(bar(BAR_DRAIN), 0);
            }
        }
    } else if (warp == W_RAW) {
        // ---- raw weight super-blocks: one 2-D tile (128 rows x RAW_ROW bytes) each ----
        if (lane == 0) {
            int sb_issued = 0;
            for (int sb = 0; sb < nsb; ++sb) {
                const int rb = sb % F::NRAW;
                if (!pf_wait(bar(BAR_RAW_EMPTY + rb), ((sb / F::NRAW) & 1) ^ 1, abort_flag, p.status)) break;
                mbar_expect_tx(bar(BAR_RAW_FULL + rb), Lay::RAW_BUF);
                tma_load_2d(sb0 + Lay::OFF_RAW + rb * Lay::RAW_BUF, &tmW,
                            (int)(((int64_t)(sbb + sb) * F::BLOCK) & ~int64_t(15)), row0, bar(BAR_RAW_FULL + rb));
                sb_issued = sb + 1;
            }
            if (*abort_flag)
                for (int sb = max(0, sb_issued - F::NRAW); sb < sb_issued; ++sb)
                    pf_settle(bar(BAR_RAW_FULL + sb % F::NRAW), (sb / F::NRAW) & 1);
        }
    } else if (warp < W_EPI) {
        // ---- weight converters ----
        // a warp may only address its own 32-lane quarter of tensor memory
        const int r = 32 * (warp & 3) + lane;
        const int grp = (warp - W_CONV) >> 2;   // converter group
        const bool valid = r < rows;
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const PfCtx cx{sb0, smem, abort_flag, p.status};
        for (int sb = 0; sb < nsb; ++sb) {
            const int rb = sb % F::NRAW, b4 = sb % PF_NSB;
            if (!__all_sync(FULL, pf_wait(bar(BAR_RAW_FULL + rb), (sb / F::NRAW) & 1, abort_flag, p.status))) break;
            if (!__all_sync(FULL, pf_wait(bar(BAR_SB_FREE + b4), ((sb / PF_NSB) & 1) ^ 1, abort_flag, p.status))) break;
            bool ok;
            if constexpr (T == T_Q4_K) ok = convert_q4k<Lay>(cx, sb0, tl, sb, rb, b4, r, grp, valid, barbase);
            else ok = convert_q6k<Lay>(cx, sb0, tl, sb, sbb + sb, rb, b4, r, grp, valid, barbase);
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(BAR_RAW_EMPTY + rb));
        }
    } else {
        // ---- epilogue: thread = tile row (tensor-memory lane), 64 token columns ----
        const int q = warp & 3;                       // tensor-memory quarter this warp may read
        const int c0 = ((warp - W_EPI) >> 2) * EPI_COLS;
        const int r = 32 * q + lane;
        float acc[EPI_COLS];
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int sb = 0; sb < nsb && ok; ++sb) {
            const int buf = sb & 1, b4 = sb % PF_NSB;
            const uint32_t ph = (sb >> 1) & 1, ph4 = (sb / PF_NSB) & 1;
            if (!__all_sync(FULL, pf_wait(bar(BAR_ACC_FULL + buf), ph, abort_flag, p.status) &&
                                      pf_wait(bar(BAR_A2_FULL + b4), ph4, abort_flag, p.status) &&
                                      pf_wait(bar(BAR_SBD_FULL + b4), ph4, abort_flag, p.status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float fr = reinterpret_cast<const float *>(smem + Lay::OFF_DW)[b4 * PF_BM + r];
            const float4 *da4 = reinterpret_cast<const float4 *>(smem + Lay::OFF_DA + b4 * BN * 4 + c0 * 4);
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + TM_ACC + (uint32_t)buf * 128u + (uint32_t)c0;
#pragma unroll
            for (int cc = 0; cc < EPI_COLS / 8; ++cc) {
                uint32_t v[8];
                tmem_ld8(ta + 8 * cc, v);
                tmem_wait_ld(v);
#pragma unroll
                for (int gq = 0; gq < 2; ++gq) {
                    const float4 d = da4[2 * cc + gq];
                    const float dv[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = 4 * gq + e;
                        acc[8 * cc + j] = fmaf(dv[e], fr * __uint_as_float(v[j]), acc[8 * cc + j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(BAR_ACC_EMPTY + buf));
                mbar_arrive(bar(BAR_SB_FREE + b4));
            }
        }
        if (ok && !*abort_flag && r < rows) {
            float *yr = yout + row0 + r;
#pragma unroll
            for (int j = 0; j < EPI_COLS; ++j)
                if (tok0 + c0 + j < p.m) yr[(int64_t)(tok0 + c0 + j) * p.n_out] = acc[j];
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, PF_TMEM_COLS);
    }
}

// ---- prefill copies of the weights ------------------------------------------------
// Made once when the weights are uploaded, beside the raw GGUF bytes (which
// the decode kernels keep reading): per 128-row tile and super-block one
// contiguous chunk holding exactly the shared-memory image the MMAs read, so
// the prefill kernel moves it with plain 1-D bulk copies and converts nothing:
//   [KSTEPS][128 rows][64 f16]  A operand of each K-step (sc q 2^-s, or the two
//                               Q6_K planes), K-major with the 128-byte swizzle
//                               (16-byte unit j of row r stored at j ^ (r & 7))
//   Q4_K: [2][128 rows][16 f16] the mins operand, hi then lo parts, K-major
//                               with the 32-byte swizzle (unit j of row r at
//                               j ^ ((r >> 2) & 1))
//   [128] f32                   the row scale f (Q4_K: d 2^s; Q6_K: d)
// Rows past n_out are zero. The values are those the converters of
// prefill_kernel write into tensor memory.
template <uint32_t T> struct PkFmt;
template <> struct PkFmt<T_Q4_K> {
    static constexpr int KSTEPS = 4, RAW_ROW = 144;
    static constexpr bool MINS = true;
};
template <> struct PkFmt<T_Q6_K> {
    static constexpr int KSTEPS = 8, RAW_ROW = 240;
    static constexpr bool MINS = false;
};
// Q5_K, Q3_K, Q2_K have a prefill copy but no converter kernel: their K-step
// tiles hold one exact f16 plane of integer scale x quant, in the Q4_K slot
// order, so they share the Q4_K token operand; Q5_K and Q2_K carry a mins
// operand (Q2_K: one min per 16 elements, i.e. per bsums index).
template <> struct PkFmt<T_Q5_K> {
    static constexpr int KSTEPS = 4, RAW_ROW = 176;
    static constexpr bool MINS = true;
};
template <> struct PkFmt<T_Q3_K> {
    static constexpr int KSTEPS = 4, RAW_ROW = 112;
    static constexpr bool MINS = false;
};
template <> struct PkFmt<T_Q2_K> {
    static constexpr int KSTEPS = 4, RAW_ROW = 96;
    static constexpr bool MINS = true;
};
// F16: the weights themselves, re-tiled (no scale: row scale f = 1), against
// the activation converted to f16 (the reference's F16 pair, src/backend.c:
// 19-27) with token scale 1; 256-element chunks play the super-block's part,
// so each chunk's sum is accumulated in tensor memory and the chunks are
// added in the epilogue.
template <> struct PkFmt<T_F16> {
    static constexpr int KSTEPS = 4, RAW_ROW = 16;   // the pack kernel reads the row from global memory
    static constexpr bool MINS = false;
};

// Integer main-term weight (sub-block scale x quant) of element e (0..255) of
// one super-block, as the reference's dots form it:
//   Q5_K src/kernels.c:412-478: sc (6-bit, src/kernels.c:648-656) x (nibble +
//        16 x qh bit), qs[32c + l] low nibble = element 64c + l, high nibble
//        = 64c + 32 + l, qh[l] bit 2c / 2c + 1;
//   Q3_K src/kernels.c:289-347: (sc - 32) x ((qs[32n + l] >> 2j) & 3) - (4
//        unless hmask[l] bit 4n + j), element 128n + 32j + l;
//   Q2_K src/kernels.c:249-287: (scales[e / 16] & 15) x ((qs[32n + l] >> 2j)
//        & 3), element 128n + 32j + l.
// b: the block's bytes in shared memory.
__device__ __forceinline__ int k4_scale6(const uint8_t *q, int j) {   // 6-bit scale j of the 12 packed bytes
    return j < 4 ? (q[j] & 63) : ((q[j + 4] & 0xf) | ((q[j - 4] >> 6) << 4));
}
__device__ __forceinline__ int k4_min6(const uint8_t *q, int j) {     // 6-bit min j
    return j < 4 ? (q[j + 4] & 63) : ((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
}
template <uint32_t T>
__device__ __forceinline__ int pk_int_weight(const uint8_t *b, int e) {
    if constexpr (T == T_Q5_K) {
        const int c = e >> 6, hi = (e >> 5) & 1, l = e & 31;
        const int qs = b[48 + 32 * c + l];
        const int q = (hi ? qs >> 4 : qs & 15) | (((b[16 + l] >> (2 * c + hi)) & 1) << 4);
        return k4_scale6(b + 4, e >> 5) * q;
    } else if constexpr (T == T_Q3_K) {
        const int n = e >> 7, j = (e >> 5) & 3, l = e & 31;
        const int q = ((b[32 + 32 * n + l] >> (2 * j)) & 3) - (((b[l] >> (4 * n + j)) & 1) ? 0 : 4);
        const int s = e >> 4;   // 16 6-bit scales in 12 bytes (src/kernels.c:328-333)
        const uint8_t *sc = b + 96;
        const int lo = s < 8 ? (sc[s & 7] & 15) : (sc[s & 7] >> 4);
        const int hi2 = (sc[8 + (s & 3)] >> (2 * (s >> 2))) & 3;
        return ((lo | (hi2 << 4)) - 32) * q;
    } else {
        const int n = e >> 7, j = (e >> 5) & 3, l = e & 31;
        return (b[e >> 4] & 15) * ((b[16 + 32 * n + l] >> (2 * j)) & 3);
    }
}

// The exponent s of the row scale f = d 2^s (s >= 0 the smallest keeping
// (dmin / f) x min inside f16 range), as q4k_scale_exp, for the given d, dmin
// and largest min; keep_main is false when d is zero or negligible.
__device__ __forceinline__ void pk_scale_exp(float d, float dmin, int mn_max, int &sexp, bool &keep_main) {
    sexp = 0;
    keep_main = d != 0.0f;
    if (keep_main) {
        const float ratio = fabsf(dmin) * (float)mn_max / (60000.0f * fabsf(d));
        if (ratio > 1.0f) sexp = ilogbf(ratio) + 1;
        if (sexp > 14) keep_main = false;
    }
}
constexpr int PK_ATILE = PF_BM * PF_KS * 2;   // 16 KB: one K-step of a 128-row tile
constexpr int PK_MINT = PF_BM * 16 * 2;       // 4 KB: one half of the mins operand
template <uint32_t T> __host__ __device__ constexpr int pk_off_min() { return PkFmt<T>::KSTEPS * PK_ATILE; }
template <uint32_t T> __host__ __device__ constexpr int pk_off_f() {
    return pk_off_min<T>() + (PkFmt<T>::MINS ? 2 * PK_MINT : 0);
}
template <uint32_t T> __host__ __device__ constexpr int pk_chunk() { return pk_off_f<T>() + PF_BM * 4; }

// one CTA per (row tile, super-block); thread = tile row
template <uint32_t T>
__global__ void __launch_bounds__(PF_BM) prefill_pack_kernel(const uint8_t *w, int64_t row_bytes, int n_out, int nsb,
                                                            uint8_t *pack) {
    using P = PkFmt<T>;
    __shared__ __align__(16) uint8_t raw[PF_BM * P::RAW_ROW];
    const int rt = blockIdx.x, sb = blockIdx.y, r = threadIdx.x;
    const int64_t row = (int64_t)rt * PF_BM + r;
    const bool valid = row < n_out;
    // this row's block into shared memory, 16-byte aligned (Q6_K blocks start
    // at any even byte)
    uint8_t *mine = raw + r * P::RAW_ROW;
    if constexpr (T == T_F16) {
        // 256 halves of the row straight from global memory (rows are 16-byte
        // multiples: n_in is a multiple of 256), in the Q4_K slot order
        uint8_t *chunk = pack + ((size_t)rt * nsb + sb) * (size_t)pk_chunk<T>();
        reinterpret_cast<float *>(chunk + pk_off_f<T>())[r] = valid ? 1.0f : 0.0f;
        const uint4 *src = reinterpret_cast<const uint4 *>(w + row * row_bytes + (int64_t)sb * 512);
        for (int t = 0; t < 4; ++t) {
            uint32_t h[32];   // halves 64t .. 64t + 63, two per word
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint4 u = valid ? src[8 * t + k] : make_uint4(0, 0, 0, 0);
                h[4 * k] = u.x; h[4 * k + 1] = u.y; h[4 * k + 2] = u.z; h[4 * k + 3] = u.w;
            }
            uint32_t v[32];
#pragma unroll
            for (int g = 0; g < 16; ++g) {   // elements 4g..4g+3 as slots (4g, 4g+2), (4g+1, 4g+3)
                const uint32_t a = h[2 * g], b = h[2 * g + 1];
                v[2 * g] = (a & 0xffffu) | (b << 16);
                v[2 * g + 1] = (a >> 16) | (b & 0xffff0000u);
            }
            uint8_t *dst = chunk + (size_t)t * PK_ATILE + r * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                reinterpret_cast<uint4 *>(dst)[j ^ (r & 7)] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        return;
    }
    if (T == T_Q4_K || T == T_Q5_K) {
        constexpr int BLK = T == T_Q4_K ? B_Q4_K : B_Q5_K;
        const uint4 *src = reinterpret_cast<const uint4 *>(w + row * row_bytes + (int64_t)sb * BLK);
#pragma unroll
        for (int k = 0; k < BLK / 16; ++k)
            reinterpret_cast<uint4 *>(mine)[k] = valid ? src[k] : make_uint4(0, 0, 0, 0);
    } else if (T == T_Q3_K || T == T_Q2_K) {
        // 110- and 84-byte blocks start at any even byte
        constexpr int BLK = T == T_Q3_K ? B_Q3_K : B_Q2_K;
        const uint16_t *src = reinterpret_cast<const uint16_t *>(w + row * row_bytes + (int64_t)sb * BLK);
        for (int k = 0; k < P::RAW_ROW / 2; ++k)
            reinterpret_cast<uint16_t *>(mine)[k] = (valid && k < BLK / 2) ? src[k] : (uint16_t)0;
    } else {
        const uint16_t *src = reinterpret_cast<const uint16_t *>(w + row * row_bytes + (int64_t)sb * B_Q6_K);
        for (int k = 0; k < P::RAW_ROW / 2; ++k)
            reinterpret_cast<uint16_t *>(mine)[k] = (valid && k < B_Q6_K / 2) ? src[k] : (uint16_t)0;
    }
    __syncwarp();
    uint8_t *chunk = pack + ((size_t)rt * nsb + sb) * (size_t)pk_chunk<T>();
    auto put_a = [&](int t, const uint32_t (&v)[32]) {
        uint8_t *dst = chunk + (size_t)t * PK_ATILE + r * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            reinterpret_cast<uint4 *>(dst)[j ^ (r & 7)] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    };
    float *fdst = reinterpret_cast<float *>(chunk + pk_off_f<T>());
    const uint32_t a = smem_addr(mine);
    if constexpr (T == T_Q4_K) {
        const uint4 h = lds128(a);
        int sexp;
        bool keep_main;
        q4k_scale_exp(h, sexp, keep_main);
        float f;
        uint32_t mw[16];
        q4k_mins_words(h, sexp, keep_main, valid, f, mw);
        fdst[r] = f;
        for (int half = 0; half < 2; ++half) {
            uint8_t *dst = chunk + pk_off_min<T>() + half * PK_MINT + r * 32;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t *m4 = mw + 8 * half + 4 * j;
                reinterpret_cast<uint4 *>(dst)[j ^ ((r >> 2) & 1)] = make_uint4(m4[0], m4[1], m4[2], m4[3]);
            }
        }
        for (int c = 0; c < 4; ++c) {
            const uint4 q0 = lds128(a + 16 + 32 * c), q1 = lds128(a + 32 + 32 * c);
            const uint32_t x[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            uint32_t v[32];
            q4k_kstep_words(h, x, c, sexp, valid && keep_main, v);
            put_a(c, v);
        }
    } else if constexpr (T == T_Q6_K) {
        uint32_t S[5];
        span_words<5>(a + 192, 0, S);
        fdst[r] = valid ? h2f(S[4] & 0xffffu) : 0.0f;
        for (int cq = 0; cq < 4; ++cq) {
            uint32_t p0[32], p1[32];
            q6k_quarter_words(a, 0, S, valid, cq, p0, p1);
            put_a(2 * cq, p0);
            put_a(2 * cq + 1, p1);
        }
    } else {
        // Q5_K / Q3_K / Q2_K: made once at load, so plain per-element code.
        // Main plane: (sc q) 2^-s, exact in f16 (|sc q| <= 1953, 128, 45);
        // mins (Q5_K: mn[i / 2], Q2_K: m[i] for bsums index i): -(dmin / f)
        // min as hi + lo f16 parts.
        const uint8_t *b = mine;
        float d = 0.0f, dmin = 0.0f;
        int mins[16] = {};
        int mn_max = 0;
        if constexpr (T == T_Q5_K) {
            d = h2f(b[0] | (b[1] << 8));
            dmin = h2f(b[2] | (b[3] << 8));
            for (int i = 0; i < 16; ++i) mins[i] = k4_min6(b + 4, i >> 1);
        } else if constexpr (T == T_Q2_K) {
            d = h2f(b[80] | (b[81] << 8));
            dmin = h2f(b[82] | (b[83] << 8));
            for (int i = 0; i < 16; ++i) mins[i] = b[i] >> 4;
        } else {
            d = h2f(b[108] | (b[109] << 8));
        }
        for (int i = 0; i < 16; ++i) mn_max = max(mn_max, mins[i]);
        int sexp = 0;
        bool keep_main = d != 0.0f;
        if (P::MINS) pk_scale_exp(d, dmin, mn_max, sexp, keep_main);
        const float f = !P::MINS ? d : keep_main ? ldexpf(d, sexp) : ldexpf(dmin, -10);
        fdst[r] = valid ? f : 0.0f;
        const bool on = valid && keep_main;
        const float s2 = ldexpf(1.0f, -sexp);
        for (int t = 0; t < 4; ++t) {
            uint32_t v[32];
#pragma unroll 4
            for (int wi = 0; wi < 32; ++wi) {
                // word wi: slots 2 wi, 2 wi + 1 = elements 4 (wi / 2) + (wi % 2) and that + 2
                const int e0 = 64 * t + 4 * (wi >> 1) + (wi & 1);
                const float v0 = on ? (float)pk_int_weight<T>(b, e0) * s2 : 0.0f;
                const float v1 = on ? (float)pk_int_weight<T>(b, e0 + 2) * s2 : 0.0f;
                v[wi] = half2_bits(v0, v1);
            }
            put_a(t, v);
        }
        if constexpr (P::MINS) {
            const float mfac = f != 0.0f ? dmin / f : 0.0f;
            uint32_t mw[16];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float m0 = mfac * (float)mins[2 * c], m1 = mfac * (float)mins[2 * c + 1];
                const float h0 = __half2float(__float2half_rn(m0)), h1 = __half2float(__float2half_rn(m1));
                mw[c] = valid ? half2_bits(-h0, -h1) : 0u;
                mw[8 + c] = valid ? half2_bits(h0 - m0, h1 - m1) : 0u;
            }
            for (int half = 0; half < 2; ++half) {
                uint8_t *dst = chunk + pk_off_min<T>() + half * PK_MINT + r * 32;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const uint32_t *m4 = mw + 8 * half + 4 * j;
                    reinterpret_cast<uint4 *>(dst)[j ^ ((r >> 2) & 1)] = make_uint4(m4[0], m4[1], m4[2], m4[3]);
                }
            }
        }
    }
}

// ---- prefill from the packed copy ------------------------------------------------------
// One CTA: 128 weight rows x BN tokens, one SM, 10 warps:
//   warp 0     loads: per super-block the mins operand, row scales, bsums tile
//              and token scales; per K-step the A chunk (bulk copy of 16 KB)
//              and the token operand tile (TMA, 128-byte swizzle)
//   warp 1     tensor-memory owner; lane 0 issues the MMAs, both operands
//              from shared memory
//   warps 2-9  epilogue as in prefill_kernel: per super-block the accumulator
//              scaled by f * dA and added in registers (thread = row, BN / 2
//              tokens)
// Tensor memory: two BN-column accumulators.
constexpr int PK_WARPS = 10, PK_EPI = 2, PK_NEPI = 8, PK_NSB = 2;
template <uint32_t T, int BN> struct PkLayout {
    using P = PkFmt<T>;
    static constexpr int STAGE = PK_ATILE + stage_bytes(BN);
    // per super-block buffer: mins hi / lo, bsums tile, row scales, token scales
    static constexpr int META_MIN = P::MINS ? 2 * PK_MINT : 0;
    static constexpr int META_B2 = P::MINS ? min_bytes(BN) : 0;
    static constexpr int META = (META_MIN + META_B2 + PF_BM * 4 + BN * 4 + 1023) & ~1023;
    static constexpr int BUDGET = 227 * 1024 - 2048;   // barriers, flags, alignment slack
    static constexpr int STAGES = (BUDGET - PK_NSB * META) / STAGE > 6 ? 6 : (BUDGET - PK_NSB * META) / STAGE;
    static constexpr int OFF_META = STAGES * STAGE;
    static constexpr int OFF_BAR = OFF_META + PK_NSB * META;
    static constexpr int OFF_FLAGS = OFF_BAR + 8 * 32;
    static constexpr int SMEM = OFF_FLAGS + 16 + 1024;
    static_assert(STAGES >= 2, "shared memory");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};
enum {
    PB_FULL = 0,            // [6] A chunk + token tile landed (bytes)
    PB_EMPTY = 6,           // [6] stage consumed by the MMAs (commit)
    PB_META_FULL = 12,      // [2] super-block buffer landed (bytes)
    PB_META_FREE = 14,      // [2] epilogue done with a super-block buffer (8 warps)
    PB_ACC_FULL = 16,       // [2] accumulator of a super-block ready (commit)
    PB_ACC_EMPTY = 18,      // [2] accumulator read (8 warps)
    PB_DRAIN = 20,
    PB_NBARS = 21,
};

struct PkParams {
    const uint8_t *pack;
    int n_out, nsb, nsplit, sb_per_split;
    float *part;
    const float *da;
    float *y;
    int m, m_pad, ntt;
    int *status;
};

// 32 lanes x N consecutive 32-bit columns, waited for
template <int N>
__device__ __forceinline__ void tmem_ld32x(uint32_t taddr, uint32_t (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld32x<16>(uint32_t taddr, uint32_t (&v)[16]) {
    tmem_ld16(taddr, v);
    tmem_wait_ld(v);
}
template <>
__device__ __forceinline__ void tmem_ld32x<32>(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
          "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
          "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
          "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
        :: "memory");
}

template <uint32_t T, int BN>
__global__ void __launch_bounds__(PK_WARPS * 32, 1)
prefill_packed_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmS,
                      const PkParams p) {
    using P = PkFmt<T>;
    using Lay = PkLayout<T, BN>;
    constexpr int KST = P::KSTEPS, S = Lay::STAGES;
    constexpr int EPI_COLS = BN / 2;
    constexpr uint32_t FULL = 0xffffffffu;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb0 = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (int)(gridDim.x / (unsigned)p.nsplit);
    const int split = blockIdx.x / ntiles, tile = blockIdx.x - split * ntiles;
    const int rt = tile / p.ntt, tt = tile - rt * p.ntt;
    const int row0 = rt * PF_BM, tok0 = tt * BN;
    const int rows = min(PF_BM, p.n_out - row0);
    const int sbb = split * p.sb_per_split;
    const int nsb = min(p.sb_per_split, p.nsb - sbb);
    float *const yout = p.nsplit > 1 ? p.part + (size_t)split * p.m * p.n_out : p.y;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + Lay::OFF_FLAGS);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Lay::OFF_FLAGS + 4);
    const uint32_t barbase = sb0 + Lay::OFF_BAR;
    auto bar = [&](int i) { return barbase + 8u * (uint32_t)i; };
    // shared-memory pieces
    auto stage_a = [&](int s) { return sb0 + (uint32_t)(s * Lay::STAGE); };
    auto stage_b = [&](int s) { return sb0 + (uint32_t)(s * Lay::STAGE + PK_ATILE); };
    auto meta = [&](int b) { return (uint32_t)(Lay::OFF_META + b * Lay::META); };   // offset from smem
    constexpr int M_MIN = 0, M_B2 = Lay::META_MIN, M_F = M_B2 + Lay::META_B2, M_DA = M_F + PF_BM * 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(bar(PB_FULL + i), 1);
            mbar_init(bar(PB_EMPTY + i), 1);
        }
        for (int i = 0; i < PK_NSB; ++i) {
            mbar_init(bar(PB_META_FULL + i), 1);
            mbar_init(bar(PB_META_FREE + i), PK_NEPI);
            mbar_init(bar(PB_ACC_FULL + i), 1);
            mbar_init(bar(PB_ACC_EMPTY + i), PK_NEPI);
        }
        mbar_init(bar(PB_DRAIN), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_addr(tmem_slot), 2 * BN);
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tmB);
        if constexpr (P::MINS) tma_prefetch_map(&tmS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- loads ----
        if (lane == 0) {
            const uint8_t *chunks = p.pack + ((size_t)rt * p.nsb + sbb) * (size_t)pk_chunk<T>();
            int t_issued = 0, sb_issued = 0;
            for (int sb = 0; sb < nsb; ++sb) {
                const int b = sb % PK_NSB;
                const uint8_t *ck = chunks + (size_t)sb * pk_chunk<T>();
                if (!pf_wait(bar(PB_META_FREE + b), ((sb / PK_NSB) & 1) ^ 1, abort_flag, p.status)) break;
                const uint32_t mb = sb0 + meta(b);
                mbar_expect_tx(bar(PB_META_FULL + b), (uint32_t)(Lay::META_MIN + Lay::META_B2 + PF_BM * 4 + BN * 4));
                if constexpr (P::MINS) {
                    bulk_g2s(mb + M_MIN, ck + pk_off_min<T>(), 2 * PK_MINT, bar(PB_META_FULL + b));
                    tma_load_2d(mb + M_B2, &tmS, 16 * (sbb + sb), tok0, bar(PB_META_FULL + b));
                }
                bulk_g2s(mb + M_F, ck + pk_off_f<T>(), PF_BM * 4, bar(PB_META_FULL + b));
                bulk_g2s(mb + M_DA, p.da + (size_t)(sbb + sb) * p.m_pad + tok0, BN * 4, bar(PB_META_FULL + b));
                sb_issued = sb + 1;
                bool ok = true;
                for (int c = 0; c < KST; ++c) {
                    const int t = KST * sb + c, s = t % S;
                    const uint32_t use = (uint32_t)(t / S) & 1u;
                    if (!pf_wait(bar(PB_EMPTY + s), use ^ 1, abort_flag, p.status)) { ok = false; break; }
                    mbar_expect_tx(bar(PB_FULL + s), (uint32_t)(PK_ATILE + stage_bytes(BN)));
                    bulk_g2s(stage_a(s), ck + (size_t)c * PK_ATILE, PK_ATILE, bar(PB_FULL + s));
                    tma_load_2d(stage_b(s), &tmB, PF_KS * (KST * sbb + t), tok0, bar(PB_FULL + s));
                    t_issued = t + 1;
                }
                if (!ok) break;
            }
            if (*abort_flag) {
                for (int t = max(0, t_issued - S); t < t_issued; ++t) pf_settle(bar(PB_FULL + t % S), (t / S) & 1);
                for (int sb = max(0, sb_issued - PK_NSB); sb < sb_issued; ++sb)
                    pf_settle(bar(PB_META_FULL + sb % PK_NSB), (sb / PK_NSB) & 1);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue ----
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(PF_BM, BN);
            for (int sb = 0; sb < nsb; ++sb) {
                const int buf = sb & 1;
                const uint32_t ph = (sb >> 1) & 1;
                if (!pf_wait<true>(bar(PB_ACC_EMPTY + buf), ph ^ 1, abort_flag, p.status)) break;
                tc_fence_after();
                const uint32_t dacc = tmem + (uint32_t)(buf * BN);
                bool ok = true;
                for (int c = 0; c < KST; ++c) {
                    const int t = KST * sb + c, s = t % S;
                    if (!pf_wait<true>(bar(PB_FULL + s), (uint32_t)(t / S) & 1u, abort_flag, p.status)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < PF_KS / 16; ++kk)
                        tc_mma_f16(dacc, smem_desc(stage_a(s) + 32 * kk, 1024, SMEM_SWZ_128B),
                                   smem_desc(stage_b(s) + 32 * kk, 1024, SMEM_SWZ_128B), idesc, (c | kk) != 0);
                    tc_commit(bar(PB_EMPTY + s));
                }
                if (!ok) break;
                const int b = sb % PK_NSB;
                if (!pf_wait<true>(bar(PB_META_FULL + b), (uint32_t)(sb / PK_NSB) & 1u, abort_flag, p.status)) break;
                if constexpr (P::MINS) {
                    // the mins term, into the same accumulator: -(hi + lo) x bsums
                    tc_fence_after();
                    const uint32_t mb = sb0 + meta(b);
                    const uint64_t bd = smem_desc(mb + M_B2, 256, SMEM_SWZ_32B);
                    tc_mma_f16(dacc, smem_desc(mb + M_MIN, 256, SMEM_SWZ_32B), bd, idesc, 1);
                    tc_mma_f16(dacc, smem_desc(mb + M_MIN + PK_MINT, 256, SMEM_SWZ_32B), bd, idesc, 1);
                }
                tc_commit(bar(PB_ACC_FULL + buf));
            }
            if (*abort_flag) {
                tc_commit(bar(PB_DRAIN));
                pf_settle(bar(PB_DRAIN), 0);
            }
        }
    } else {
        // ---- epilogue: thread = tile row (tensor-memory lane), BN / 2 token columns ----
        const int q = warp & 3;
        const int c0 = ((warp - PK_EPI) >> 2) * EPI_COLS;
        const int r = 32 * q + lane;
        float acc[EPI_COLS];
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int sb = 0; sb < nsb && ok; ++sb) {
            const int buf = sb & 1, b = sb % PK_NSB;
            if (!__all_sync(FULL, pf_wait(bar(PB_ACC_FULL + buf), (uint32_t)(sb >> 1) & 1u, abort_flag, p.status) &&
                                      pf_wait(bar(PB_META_FULL + b), (uint32_t)(sb / PK_NSB) & 1u, abort_flag,
                                              p.status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint8_t *mp = smem + meta(b);
            const float fr = reinterpret_cast<const float *>(mp + M_F)[r];
            const float4 *da4 = reinterpret_cast<const float4 *>(mp + M_DA + c0 * 4);
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BN + c0);
            // 10 warps leave 168 registers a thread: 128 accumulators load 16 columns at a time
            constexpr int LD = EPI_COLS > 64 ? 16 : 32;
#pragma unroll
            for (int cc = 0; cc < EPI_COLS / LD; ++cc) {
                uint32_t v[LD];
                tmem_ld32x<LD>(ta + LD * cc, v);
#pragma unroll
                for (int g4 = 0; g4 < LD / 4; ++g4) {
                    const float4 d = da4[(LD / 4) * cc + g4];
                    const float dv[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = LD * cc + 4 * g4 + e;
                        acc[j] = fmaf(dv[e], fr * __uint_as_float(v[4 * g4 + e]), acc[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(PB_ACC_EMPTY + buf));
                mbar_arrive(bar(PB_META_FREE + b));
            }
        }
        if (ok && !*abort_flag && r < rows) {
            float *yr = yout + row0 + r;
#pragma unroll
            for (int j = 0; j < EPI_COLS; ++j)
                if (tok0 + c0 + j < p.m) yr[(int64_t)(tok0 + c0 + j) * p.n_out] = acc[j];
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// ---- prefill from the packed copy on CTA pairs ------------------------------------------
// A cluster of two CTAs (two SMs) computes a 256-row x BN-token tile with
// M = 256 MMAs (cta_group::2): CTA r holds weight rows 128 r .. 128 r + 127 of
// the tile (its own 128-row tile's chunks of the prefill copy: the A operand)
// and tokens BN/2 r .. BN/2 r + BN/2 - 1 of the token operand (B); the MMAs
// read both CTAs' shared memory and leave each CTA's 128 rows x BN tokens in
// its own tensor memory. Per K-step an SM loads 16 KB of weights and BN x 64
// bytes of tokens: half the token bytes of the one-CTA tile for the same MMA
// work per SM, and shallower stages, so more of them fit.
//   warp 0     K-step loads, in both CTAs: the A tile and B half of each
//              K-step by TMA, completion counted on the leader's barrier (the
//              leader expects both CTAs' bytes)
//   warp 10    super-block loads, in both CTAs: the mins / bsums halves the
//              same way; row scales and token scales into its own CTA for its
//              epilogue (a separate warp, so the K-step ring never waits for
//              an epilogue to free a super-block buffer)
//   warp 1     tensor-memory owner in both; lane 0 of the leader (cluster
//              rank 0) issues the MMAs and commits to both CTAs' barriers
//   warps 2-9  epilogue in both, as in prefill_packed_kernel; the arrival
//              that frees an accumulator goes to the leader
// The loaders and the epilogue poll their barriers rather than suspending:
// a suspended wait measured ~1 us late waking, longer than a K-step.
// A pair whose second row tile lies past the matrix loads zeros for it (the
// tensor map's fill) and stores nothing for those rows.
constexpr int PP_NSB = 2, PP_WARPS = 11, PP_W_META = 10;
template <uint32_t T, int BN> struct PpLayout {
    using P = PkFmt<T>;
    static constexpr int HB = BN / 2;                              // tokens per CTA in B
    static constexpr int BHALF = HB * PF_KS * 2;                   // B bytes per CTA and K-step
    static constexpr int STAGE = PK_ATILE + BHALF;
    static constexpr int META_MIN = P::MINS ? 2 * PK_MINT : 0;     // mins operand hi + lo (A side)
    static constexpr int META_B2 = P::MINS ? HB * 16 * 2 : 0;      // bsums half (B side)
    static constexpr int META = (META_MIN + META_B2 + PF_BM * 4 + BN * 4 + 1023) & ~1023;
    static constexpr int BUDGET = 227 * 1024 - 2048;               // barriers, flags, alignment slack
    static constexpr int NS = (BUDGET - PP_NSB * META) / STAGE;
    static constexpr int STAGES = NS > 8 ? 8 : NS;
    static constexpr int OFF_META = STAGES * STAGE;
    static constexpr int OFF_BAR = OFF_META + PP_NSB * META;
    static constexpr int OFF_FLAGS = OFF_BAR + 8 * 32;
    static constexpr int SMEM = OFF_FLAGS + 16 + 1024;
    static_assert(STAGES >= 3, "shared memory");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(STAGE % 1024 == 0 && META % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
};
enum {
    PP_FULL = 0,           // [8] leader: A tiles + B halves of both CTAs landed (bytes)
    PP_EMPTY = 8,          // [8] both: stage consumed by the pair's MMAs (multicast commit)
    PP_MMETA = 16,         // [2] leader: mins + bsums halves of both CTAs landed (bytes)
    PP_EMETA = 18,         // [2] own: row scales + token scales landed (bytes)
    PP_META_FREE = 20,     // [2] own epilogue done with a super-block buffer (8 warps)
    PP_ACC_FULL = 22,      // [2] both: accumulator of a super-block ready (multicast commit)
    PP_ACC_EMPTY = 24,     // [2] leader: accumulator drained by both epilogues (16 warps)
    PP_DRAIN = 26,
    PP_NBARS = 27,
};
static_assert(PP_NBARS <= 32, "barrier area");

// A launch covers up to PP_MAXM matrices that read the same activation (the
// products Wq / Wk / Wv, or W_gate / W_up, of a prompt), with one shared
// token operand: pair tiles are numbered matrix by matrix.
constexpr int PP_MAXM = PREFILL_MAXM;
struct PpMaps {
    CUtensorMap a[PP_MAXM];      // each matrix's prefill copy as 128-byte rows, 128-row boxes (A tiles)
    CUtensorMap mins[PP_MAXM];   // the same, 64-row boxes (Q4_K mins operand)
};
struct PpParams {
    const uint8_t *pack[PP_MAXM];
    float *y[PP_MAXM];           // [m][n_out]
    float *part[PP_MAXM];        // nsplit > 1: [nsplit][m][n_out] partial products
    int n_out[PP_MAXM];
    int tile_end[PP_MAXM];       // pair tiles of matrices 0..i (one split)
    int nmat, nsb, nsplit, sb_per_split;
    const float *da;             // [nsb][m_pad] token scales
    int m, m_pad, ntt;
    int *status;
};

template <uint32_t T, int BN>
__global__ void __launch_bounds__(PP_WARPS * 32, 1)
prefill_pair_kernel(const __grid_constant__ PpMaps maps, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmS, const PpParams p) {
    using P = PkFmt<T>;
    using Lay = PpLayout<T, BN>;
    constexpr int KST = P::KSTEPS, S = Lay::STAGES, HB = Lay::HB;
    constexpr int CH = pk_chunk<T>() / 128;   // 128-byte rows per chunk of the prefill copy
    constexpr int EPI_COLS = BN / 2;
    constexpr uint32_t FULL = 0xffffffffu;
    static_assert(pk_chunk<T>() % 128 == 0, "chunks are whole 128-byte rows of the copy's tensor map");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb0 = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = (int)(blockIdx.x >> 1);
    const int ntiles = p.tile_end[p.nmat - 1];
    const int split = pair / ntiles;
    int tile = pair - split * ntiles, mi = 0;
    while (mi + 1 < p.nmat && tile >= p.tile_end[mi]) ++mi;
    if (mi > 0) tile -= p.tile_end[mi - 1];
    const int n_out = p.n_out[mi];
    const uint8_t *const pack = p.pack[mi];
    const CUtensorMap *const tmP = &maps.a[mi];
    const CUtensorMap *const tmM = &maps.mins[mi];
    const int prt = tile / p.ntt, tt = tile - prt * p.ntt;
    const int rt = 2 * prt + (int)rank;                  // this CTA's 128-row tile
    const int nrt = (n_out + PF_BM - 1) / PF_BM;
    const bool has_rows = rt < nrt;
    const int row0 = rt * PF_BM, tok0 = tt * BN;
    const int rows = has_rows ? min(PF_BM, n_out - row0) : 0;
    const int sbb = split * p.sb_per_split;
    const int nsb = min(p.sb_per_split, p.nsb - sbb);
    float *const yout = p.nsplit > 1 ? p.part[mi] + (size_t)split * p.m * n_out : p.y[mi];
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + Lay::OFF_FLAGS);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Lay::OFF_FLAGS + 4);
    const uint32_t barbase = sb0 + Lay::OFF_BAR;
    auto bar = [&](int i) { return barbase + 8u * (uint32_t)i; };
    auto lbar = [&](int i) { return mapa(bar(i), 0); };   // the leader's barrier (shared::cluster)
    auto stage_a = [&](int s) { return sb0 + (uint32_t)(s * Lay::STAGE); };
    auto stage_b = [&](int s) { return sb0 + (uint32_t)(s * Lay::STAGE + PK_ATILE); };
    auto meta = [&](int b) { return (uint32_t)(Lay::OFF_META + b * Lay::META); };   // offset from smem
    constexpr int M_MIN = 0, M_B2 = Lay::META_MIN, M_F = M_B2 + Lay::META_B2, M_DA = M_F + PF_BM * 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(bar(PP_FULL + i), 1);
            mbar_init(bar(PP_EMPTY + i), 1);
        }
        for (int i = 0; i < PP_NSB; ++i) {
            mbar_init(bar(PP_MMETA + i), 1);
            mbar_init(bar(PP_EMETA + i), 1);
            mbar_init(bar(PP_META_FREE + i), PK_NEPI);
            mbar_init(bar(PP_ACC_FULL + i), 1);
            mbar_init(bar(PP_ACC_EMPTY + i), 2 * PK_NEPI);
        }
        mbar_init(bar(PP_DRAIN), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc_pair(smem_addr(tmem_slot), 2 * BN);
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(tmP);
        tma_prefetch_map(&tmB);
        if constexpr (P::MINS) {
            tma_prefetch_map(tmM);
            tma_prefetch_map(&tmS);
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync();       // both CTAs' barriers initialised and tensor memory allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- K-step loads (both CTAs) ----
        if (lane == 0) {
            const int64_t chunk0 = (int64_t)rt * p.nsb + sbb;    // this CTA's first chunk of the copy
            for (int t = 0; t < KST * nsb; ++t) {
                const int sb = t / KST, c = t - sb * KST, s = t % S;
                // past the copy's end for a pair's missing row tile: zeros
                const int crow = (int)((chunk0 + sb) * CH);
                if (!pf_wait<true>(bar(PP_EMPTY + s), ((uint32_t)(t / S) & 1u) ^ 1u, abort_flag, p.status)) break;
                if (leader) mbar_expect_tx(bar(PP_FULL + s), 2u * (uint32_t)Lay::STAGE);
                tma_load_2d_pair(stage_a(s), tmP, 0, crow + c * 128, lbar(PP_FULL + s));
                tma_load_2d_pair(stage_b(s), &tmB, PF_KS * (KST * sbb + t), tok0 + (int)rank * HB, lbar(PP_FULL + s));
            }
        }
    } else if (warp == PP_W_META) {
        // ---- super-block loads (both CTAs) ----
        if (lane == 0) {
            const int64_t chunk0 = (int64_t)rt * p.nsb + sbb;
            for (int sb = 0; sb < nsb; ++sb) {
                const int b = sb % PP_NSB;
                if (!pf_wait<true>(bar(PP_META_FREE + b), ((sb / PP_NSB) & 1) ^ 1, abort_flag, p.status)) break;
                const uint32_t mb = sb0 + meta(b);
                if constexpr (P::MINS) {
                    const int crow = (int)((chunk0 + sb) * CH);
                    if (leader) mbar_expect_tx(bar(PP_MMETA + b), 2u * (uint32_t)(Lay::META_MIN + Lay::META_B2));
                    tma_load_2d_pair(mb + M_MIN, tmM, 0, crow + KST * 128, lbar(PP_MMETA + b));
                    tma_load_2d_pair(mb + M_B2, &tmS, 16 * (sbb + sb), tok0 + (int)rank * HB, lbar(PP_MMETA + b));
                }
                mbar_expect_tx(bar(PP_EMETA + b), (uint32_t)((has_rows ? PF_BM * 4 : 0) + BN * 4));
                if (has_rows)
                    bulk_g2s(mb + M_F, pack + (size_t)(chunk0 + sb) * pk_chunk<T>() + pk_off_f<T>(), PF_BM * 4,
                             bar(PP_EMETA + b));
                bulk_g2s(mb + M_DA, p.da + (size_t)(sbb + sb) * p.m_pad + tok0, BN * 4, bar(PP_EMETA + b));
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue (leader) ----
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(2 * PF_BM, BN);
            for (int sb = 0; sb < nsb; ++sb) {
                const int buf = sb & 1;
                if (!pf_wait<true>(bar(PP_ACC_EMPTY + buf), ((uint32_t)(sb >> 1) & 1u) ^ 1u, abort_flag, p.status))
                    break;
                tc_fence_after();
                const uint32_t dacc = tmem + (uint32_t)(buf * BN);
                bool ok = true;
                for (int c = 0; c < KST; ++c) {
                    const int t = KST * sb + c, s = t % S;
                    if (!pf_wait<true>(bar(PP_FULL + s), (uint32_t)(t / S) & 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < PF_KS / 16; ++kk)
                        tc_mma_f16_pair(dacc, smem_desc(stage_a(s) + 32 * kk, 1024, SMEM_SWZ_128B),
                                        smem_desc(stage_b(s) + 32 * kk, 1024, SMEM_SWZ_128B), idesc, (c | kk) != 0);
                    tc_commit_pair(bar(PP_EMPTY + s), 3);
                }
                if (!ok) break;
                if constexpr (P::MINS) {
                    // the mins term, into the same accumulator: -(hi + lo) x bsums
                    const int b = sb % PP_NSB;
                    if (!pf_wait<true>(bar(PP_MMETA + b), (uint32_t)(sb / PP_NSB) & 1u, abort_flag, p.status)) break;
                    tc_fence_after();
                    const uint32_t mb = sb0 + meta(b);
                    const uint64_t bd = smem_desc(mb + M_B2, 256, SMEM_SWZ_32B);
                    tc_mma_f16_pair(dacc, smem_desc(mb + M_MIN, 256, SMEM_SWZ_32B), bd, idesc, 1);
                    tc_mma_f16_pair(dacc, smem_desc(mb + M_MIN + PK_MINT, 256, SMEM_SWZ_32B), bd, idesc, 1);
                }
                tc_commit_pair(bar(PP_ACC_FULL + buf), 3);
            }
            if (*abort_flag) {
                tc_commit_pair(bar(PP_DRAIN), 1);
                pf_settle(bar(PP_DRAIN), 0);
            }
        }
    } else {
        // ---- epilogue (both): thread = tile row (tensor-memory lane), BN / 2 token columns ----
        const int q = warp & 3;
        const int c0 = ((warp - PK_EPI) >> 2) * EPI_COLS;
        const int r = 32 * q + lane;
        float acc[EPI_COLS];
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int sb = 0; sb < nsb && ok; ++sb) {
            const int buf = sb & 1, b = sb % PP_NSB;
            if (!__all_sync(FULL, pf_wait<true>(bar(PP_ACC_FULL + buf), (uint32_t)(sb >> 1) & 1u, abort_flag,
                                                p.status) &&
                                      pf_wait<true>(bar(PP_EMETA + b), (uint32_t)(sb / PP_NSB) & 1u, abort_flag,
                                                    p.status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint8_t *mp = smem + meta(b);
            const float fr = reinterpret_cast<const float *>(mp + M_F)[r];
            const float4 *da4 = reinterpret_cast<const float4 *>(mp + M_DA + c0 * 4);
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BN + c0);
            constexpr int LD = EPI_COLS > 64 ? 16 : 32;
#pragma unroll
            for (int cc = 0; cc < EPI_COLS / LD; ++cc) {
                uint32_t v[LD];
                tmem_ld32x<LD>(ta + LD * cc, v);
#pragma unroll
                for (int g4 = 0; g4 < LD / 4; ++g4) {
                    const float4 d = da4[(LD / 4) * cc + g4];
                    const float dv[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = LD * cc + 4 * g4 + e;
                        acc[j] = fmaf(dv[e], fr * __uint_as_float(v[4 * g4 + e]), acc[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_remote(lbar(PP_ACC_EMPTY + buf));
                mbar_arrive(bar(PP_META_FREE + b));
            }
        }
        if (ok && !*abort_flag && r < rows) {
            float *yr = yout + row0 + r;
#pragma unroll
            for (int j = 0; j < EPI_COLS; ++j)
                if (tok0 + c0 + j < p.m) yr[(int64_t)(tok0 + c0 + j) * n_out] = acc[j];
        }
    }

    if (*abort_flag && (warp == 0 || warp == PP_W_META) && lane == 0) {
        // let copies still in flight land before the CTA's shared memory goes away
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) {
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync();       // the pair's MMAs and remote arrivals are done
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 2 * BN);
    }
}

// Q8_K rows -> token operand for the MMAs: f16 quants with the slots of each
// group of four holding elements 0, 2, 1, 3 (the order the weight converters
// produce); for two-plane formats (Q6_K) each 64-element quarter is followed by
// the same quarter times 16. Also f16 bsums (formats with mins) and the block
// scales transposed to [sb][token]. Tokens m..m_pad-1 are zero.
template <int PLANES>
__global__ void prefill_prep_q8k(const uint8_t *xq, int m, int nsb, int m_pad, uint16_t *B, uint16_t *S, float *DA) {
    const int sb = blockIdx.x, t = blockIdx.y, i = threadIdx.x;   // 64 threads, 4 elements each
    const int64_t K = (int64_t)nsb * QK_K;
    uint32_t e[4] = {0, 0, 0, 0};
    if (t < m) {
        const uint8_t *blk = xq + ((int64_t)t * nsb + sb) * B_Q8_K;
        const uint32_t w = *reinterpret_cast<const uint32_t *>(blk + 4 + 4 * i);
#pragma unroll
        for (int k = 0; k < 4; ++k) e[k] = (uint32_t)(int)(int8_t)byte_at(w, k);
        if (S && i < 16) {
            const int16_t bs = *reinterpret_cast<const int16_t *>(blk + 260 + 2 * i);
            S[(int64_t)t * (K / 16) + 16 * sb + i] = __half_as_ushort(__float2half_rn((float)bs));
        }
        if (i == 0) DA[(int64_t)sb * m_pad + t] = *reinterpret_cast<const float *>(blk);
    } else {
        if (S && i < 16) S[(int64_t)t * (K / 16) + 16 * sb + i] = 0;
        if (i == 0) DA[(int64_t)sb * m_pad + t] = 0.0f;
    }
    const float a0 = (float)(int)e[0], a1 = (float)(int)e[1], a2 = (float)(int)e[2], a3 = (float)(int)e[3];
    uint16_t *row = B + (int64_t)t * K * PLANES + (int64_t)QK_K * PLANES * sb;
    if (PLANES == 1) {
        *reinterpret_cast<uint2 *>(row + 4 * i) = make_uint2(half2_bits(a0, a2), half2_bits(a1, a3));
    } else {
        const int cq = i >> 4, e64 = (4 * i) & 63;
        *reinterpret_cast<uint2 *>(row + 128 * cq + e64) = make_uint2(half2_bits(a0, a2), half2_bits(a1, a3));
        *reinterpret_cast<uint2 *>(row + 128 * cq + 64 + e64) =
            make_uint2(half2_bits(16.0f * a0, 16.0f * a2), half2_bits(16.0f * a1, 16.0f * a3));
    }
}

// f32 rows straight into the token operand, the block sums and the block
// scales, with the values and layout prefill_prep_q8k writes from the Q8_K
// rows the quantizer would make of them (the same warp quantizer,
// src/kernels.c:561-595): one warp per (token, super-block), lane L elements
// 8L..8L+7. Tokens m..m_pad-1 are zero.
template <int PLANES>
__global__ void __launch_bounds__(256) prefill_prep_f32(const float *x, int m, int nsb, int m_pad, uint16_t *B,
                                                        uint16_t *S, float *DA) {
    const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (wid >= (int64_t)m_pad * nsb) return;
    const int t = (int)(wid / nsb), sb = (int)(wid - (int64_t)t * nsb);
    const int64_t K = (int64_t)nsb * QK_K;
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0}, bsum2 = 0;
    float d = 0.0f;
    if (t < m) q8k_quant_warp(x + t * K + (int64_t)sb * QK_K, lane, q, bsum2, d);
    if (S && (lane & 1) == 0) S[(int64_t)t * (K / 16) + 16 * sb + (lane >> 1)] = __half_as_ushort(__float2half_rn((float)bsum2));
    if (lane == 0) DA[(int64_t)sb * m_pad + t] = d;
    float a[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = (float)q[i];
    // slots of each group of four hold elements 0, 2, 1, 3
    uint16_t *row = B + (int64_t)t * K * PLANES + (int64_t)QK_K * PLANES * sb;
    const uint4 v = make_uint4(half2_bits(a[0], a[2]), half2_bits(a[1], a[3]), half2_bits(a[4], a[6]),
                               half2_bits(a[5], a[7]));
    if (PLANES == 1) {
        *reinterpret_cast<uint4 *>(row + 8 * lane) = v;
    } else {
        const int cq = lane >> 3, e64 = (8 * lane) & 63;
        *reinterpret_cast<uint4 *>(row + 128 * cq + e64) = v;
        *reinterpret_cast<uint4 *>(row + 128 * cq + 64 + e64) =
            make_uint4(half2_bits(16.0f * a[0], 16.0f * a[2]), half2_bits(16.0f * a[1], 16.0f * a[3]),
                       half2_bits(16.0f * a[4], 16.0f * a[6]), half2_bits(16.0f * a[5], 16.0f * a[7]));
    }
}

// The token operand of a launch, from its f32 rows (L.xf) or its Q8_K rows.
template <int PLANES>
int launch_prep(const PrefillLaunch &L, int64_t nsb, int64_t m_pad, uint16_t *B, uint16_t *S, float *DA,
                cudaStream_t st) {
    if (L.xf) {
        const int64_t warps = m_pad * nsb;
        prefill_prep_f32<PLANES><<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(L.xf, (int)L.m, (int)nsb, (int)m_pad, B,
                                                                              S, DA);
    } else {
        prefill_prep_q8k<PLANES><<<dim3((unsigned)nsb, (unsigned)m_pad), 64, 0, st>>>(
            static_cast<const uint8_t *>(L.xq), (int)L.m, (int)nsb, (int)m_pad, B, S, DA);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// The F16 token operand: the activation as f16 (the reference's RNE
// conversion, src/kernels.c:98-176, from f32 rows, or the caller's f16 rows)
// in the slot order of the copies, token scale 1: one warp per (token,
// 256-element chunk), lane L elements 8L..8L+7. Tokens m..m_pad-1 are zero.
__global__ void __launch_bounds__(256) prefill_prep_f16(const float *xf, const uint16_t *xh, int m, int nsb,
                                                        int m_pad, uint16_t *B, float *DA) {
    const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (wid >= (int64_t)m_pad * nsb) return;
    const int t = (int)(wid / nsb), sb = (int)(wid - (int64_t)t * nsb);
    const int64_t K = (int64_t)nsb * QK_K;
    uint32_t hv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (t < m) {
        const int64_t off = t * K + (int64_t)sb * QK_K + 8 * lane;
        if (xf) {
            const float4 a = reinterpret_cast<const float4 *>(xf + off)[0];
            const float4 b = reinterpret_cast<const float4 *>(xf + off)[1];
            const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) hv[k] = f2h(v[k]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) hv[k] = xh[off + k];
        }
    }
    if (lane == 0) DA[(int64_t)sb * m_pad + t] = t < m ? 1.0f : 0.0f;
    uint16_t *row = B + t * K + (int64_t)QK_K * sb;
    *reinterpret_cast<uint4 *>(row + 8 * lane) =
        make_uint4(hv[0] | (hv[2] << 16), hv[1] | (hv[3] << 16), hv[4] | (hv[6] << 16), hv[5] | (hv[7] << 16));
}

// The token operand of a copy-reading launch for weight type T.
template <uint32_t T>
int launch_prep_t(const PrefillLaunch &L, int64_t nsb, int64_t m_pad, uint16_t *B, uint16_t *S, float *DA,
                  cudaStream_t st) {
    if constexpr (T == T_F16) {
        const int64_t warps = m_pad * nsb;
        prefill_prep_f16<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
            L.xf, static_cast<const uint16_t *>(L.xq), (int)L.m, (int)nsb, (int)m_pad, B, DA);
        return cudaGetLastError() == cudaSuccess ? 0 : -2;
    } else {
        return launch_prep<PkFmt<T>::KSTEPS / 4>(L, nsb, m_pad, B, S, DA, st);
    }
}

// Y = the splits' partial products added in split order (one f32 add per
// split, the same order on every run)
__global__ void prefill_sum_splits(const float *part, int nsplit, int64_t n, float *y) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float a = part[i];
        for (int k = 1; k < nsplit; ++k) a = __fadd_rn(a, part[(int64_t)k * n + i]);
        y[i] = a;
    }
}

// Weight rows whose byte length is not a multiple of 16 (Q6_K with a
// super-block count that is not a multiple of 8) cannot be described by a
// tensor map; they are copied to rows of `stride` bytes first.
__global__ void prefill_pad_rows(const uint16_t *src, int64_t row_bytes, int64_t n_out, uint16_t *dst, int64_t stride) {
    const int64_t hw = row_bytes / 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_out * hw; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / hw, c = i - r * hw;
        dst[r * (stride / 2) + c] = src[i];
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 2-D tensor [rows][cols] of f16 (esize 2) or bytes (esize 1), cols contiguous
// with rows `pitch` bytes apart, box {bx cols, by rows}; reads past the ends
// return zeros
bool make_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint64_t pitch, uint32_t bx,
              uint32_t by, CUtensorMapSwizzle swz, int esize) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {bx, by};
    cuuint32_t es[2] = {1, 1};
    return fn(map, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
              const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Super-block ranges per row: when a product's 128-row x token tiles fill the
// SMs in few or ragged waves (the kernel holds one SM per CTA), splitting each
// row's super-blocks over s CTAs shortens the busiest SM's work; the partial
// products then cost s x m x n_out x 8 bytes of traffic (written, read back
// and added). s minimises (waves / s) x per-tile time + that traffic, with a
// tile costing ~2.5 us per super-block and traffic at ~5 TB/s (measured
// orders of magnitude; only the comparison matters). The split changes only
// the float order in which super-blocks are added.
int split_count_tiles(int64_t tiles, int64_t nsb, int64_t m, int64_t n_out, int slots, double us_per_sb) {
    if (slots <= 0 || tiles <= 0) return 1;
    const double tile_us = us_per_sb * (double)nsb;
    auto cost = [&](int s) {
        const double waves = (double)((tiles * s + slots - 1) / slots) / s;
        const double traffic_us = s > 1 ? (double)s * m * n_out * 8.0 / 5e6 : 0.0;
        return waves * tile_us + traffic_us;
    };
    int best = 1;
    double best_c = cost(1);
    for (int s = 2; s <= 8 && nsb / s >= 4; ++s) {
        const double c = cost(s);
        if (c < best_c * 0.97) {
            best_c = c;
            best = s;
        }
    }
    return best;
}
int split_count_bn(int64_t n_in, int64_t n_out, int64_t m, int num_sms, int64_t bn, double us_per_sb) {
    const int64_t tiles = (n_out + PF_BM - 1) / PF_BM * ((m + bn - 1) / bn);
    return split_count_tiles(tiles, n_in / QK_K, m, n_out, num_sms, us_per_sb);
}
int split_count(int64_t n_in, int64_t n_out, int64_t m, int num_sms) {
    return split_count_bn(n_in, n_out, m, num_sms, m <= PF_BN_SMALL ? PF_BN_SMALL : PF_BN, 2.5);
}
// the packed kernel's token tile and its time per super-block (MMA time of a
// 128 x bn x 256 tile at ~60 % of the f16 rate; only the comparison matters)
int pk_bn(int64_t m) { return m > PF_BN ? 256 : PF_BN; }
double pk_us_per_sb(uint32_t wtype, int64_t bn) { return (bn == 256 ? 1.8 : 0.9) * (wtype == T_Q6_K ? 2.0 : 1.0); }
// Products of at least two 128-row tiles, and groups of products, run on CTA
// pairs (one 256-row tile per pair, 2 SMs); a pair's time per super-block is
// the one-CTA tile's.
bool use_pair(int64_t n_out) { return (n_out + PF_BM - 1) / PF_BM >= 2; }
struct PairPlan {
    int64_t tiles;       // pair tiles of the group (one split)
    int64_t sum_out;     // rows of the group
    int nsplit, sb_per_split;
};
PairPlan pair_plan(uint32_t wtype, int64_t n_in, int nmat, const int64_t *n_out, int64_t m, int num_sms) {
    const int64_t bn = pk_bn(m), ntt = (m + bn - 1) / bn, nsb = n_in / QK_K;
    PairPlan pl{};
    for (int i = 0; i < nmat; ++i) {
        pl.tiles += ((n_out[i] + PF_BM - 1) / PF_BM + 1) / 2 * ntt;
        pl.sum_out += n_out[i];
    }
    const int ns = split_count_tiles(pl.tiles, nsb, m, pl.sum_out, num_sms / 2, pk_us_per_sb(wtype, bn));
    pl.sb_per_split = (int)((nsb + ns - 1) / ns);
    pl.nsplit = (int)((nsb + pl.sb_per_split - 1) / pl.sb_per_split);   // no empty range
    return pl;
}

struct WsParts {
    size_t b, s, da, pad, part;
};
WsParts ws_parts(uint32_t wtype, int64_t n_in, int64_t n_out, int64_t m, int num_sms, bool packed = false) {
    const int64_t bn = packed ? pk_bn(m) : PF_BN;
    const int64_t m_pad = (m + bn - 1) / bn * bn;
    const int planes = wtype == T_Q6_K ? 2 : 1;
    const bool mins = wtype == T_Q4_K || wtype == T_Q5_K || wtype == T_Q2_K;   // PkFmt<T>::MINS
    WsParts w{};
    w.b = align256((size_t)m_pad * n_in * 2 * planes);
    w.s = mins ? align256((size_t)m_pad * (n_in / 16) * 2) : 0;
    w.da = align256((size_t)(n_in / QK_K) * m_pad * 4);
    const int64_t rb = n_in / QK_K * B_Q6_K;
    w.pad = (!packed && wtype == T_Q6_K && rb % 16) ? align256((size_t)n_out * ((rb + 15) & ~int64_t(15))) : 0;
    const int ns = !packed ? split_count(n_in, n_out, m, num_sms)
                 : use_pair(n_out) ? pair_plan(wtype, n_in, 1, &n_out, m, num_sms).nsplit
                                   : split_count_bn(n_in, n_out, m, num_sms, bn, pk_us_per_sb(wtype, bn));
    w.part = ns > 1 ? align256((size_t)ns * m * n_out * 4) : 0;
    return w;
}

template <uint32_t T, int BN>
int launch_tb(const PrefillLaunch &L, cudaStream_t st) {
    using F = PfFmt<T>;
    using Lay = PfLayout<T, BN>;
    const int64_t K = L.n_in, nsb = K / QK_K;
    const int64_t m_pad = (L.m + BN - 1) / BN * BN;
    const WsParts parts = ws_parts(T, L.n_in, L.n_out, L.m, L.num_sms);
    uint8_t *ws = static_cast<uint8_t *>(L.ws);
    uint16_t *B = reinterpret_cast<uint16_t *>(ws);
    uint16_t *S = F::MINS ? reinterpret_cast<uint16_t *>(ws + parts.b) : nullptr;
    float *DA = reinterpret_cast<float *>(ws + parts.b + parts.s);
    if (launch_prep<F::KSTEPS / 4>(L, nsb, m_pad, B, S, DA, st) != 0) return -2;

    const int64_t row_bytes = nsb * F::BLOCK;
    const void *w = L.w;
    int64_t pitch = row_bytes;
    if (row_bytes % 16 || reinterpret_cast<uintptr_t>(w) % 16) {
        pitch = (row_bytes + 15) & ~int64_t(15);
        uint16_t *dst = reinterpret_cast<uint16_t *>(ws + parts.b + parts.s + parts.da);
        prefill_pad_rows<<<1024, 256, 0, st>>>(static_cast<const uint16_t *>(w), row_bytes, L.n_out, dst, pitch);
        if (cudaGetLastError() != cudaSuccess) return -2;
        w = dst;
    }
    CUtensorMap tmW, tmB, tmS;
    if (!make_map(&tmW, w, (uint64_t)row_bytes, (uint64_t)L.n_out, (uint64_t)pitch, F::RAW_ROW, PF_BM,
                  CU_TENSOR_MAP_SWIZZLE_NONE, 1) ||
        !make_map(&tmB, B, (uint64_t)(K * F::KSTEPS / 4), (uint64_t)m_pad, (uint64_t)(K * F::KSTEPS / 4) * 2, PF_KS,
                  BN, CU_TENSOR_MAP_SWIZZLE_128B, 2))
        return -4;
    if (F::MINS) {
        if (!make_map(&tmS, S, (uint64_t)(K / 16), (uint64_t)m_pad, (uint64_t)(K / 16) * 2, 16, BN,
                      CU_TENSOR_MAP_SWIZZLE_32B, 2))
            return -4;
    } else {
        tmS = tmB;   // unused
    }
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        cudaFuncSetAttribute(prefill_kernel<T, BN>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (cudaFuncSetAttribute(prefill_kernel<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::SMEM) !=
            cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    PfParams p{};
    p.n_out = (int)L.n_out;
    p.nsb = (int)nsb;
    p.da = DA;
    p.y = L.y;
    p.m = (int)L.m;
    p.m_pad = (int)m_pad;
    p.ntt = (int)(m_pad / BN);
    p.status = L.status;
    p.nsplit = split_count(L.n_in, L.n_out, L.m, L.num_sms);
    p.sb_per_split = (int)((nsb + p.nsplit - 1) / p.nsplit);
    p.nsplit = (int)((nsb + p.sb_per_split - 1) / p.sb_per_split);   // no empty range
    p.part = p.nsplit > 1 ? reinterpret_cast<float *>(ws + parts.b + parts.s + parts.da + parts.pad) : nullptr;
    const int64_t tiles = (L.n_out + PF_BM - 1) / PF_BM * p.ntt;
    prefill_kernel<T, BN><<<(unsigned)(tiles * p.nsplit), PF_WARPS * 32, Lay::SMEM, st>>>(tmW, tmB, tmS, p);
    if (cudaGetLastError() != cudaSuccess) return -2;
    if (p.nsplit > 1) {
        const int64_t n = L.m * L.n_out;
        const int64_t blocks = (n + 255) / 256 < 4 * L.num_sms ? (n + 255) / 256 : 4 * L.num_sms;
        prefill_sum_splits<<<(unsigned)blocks, 256, 0, st>>>(p.part, p.nsplit, n, L.y);
        if (cudaGetLastError() != cudaSuccess) return -2;
    }
    return 0;
}

template <uint32_t T, int BN>
int launch_packed_tb(const PrefillLaunch &L, cudaStream_t st) {
    using P = PkFmt<T>;
    using Lay = PkLayout<T, BN>;
    const int64_t K = L.n_in, nsb = K / QK_K;
    const int64_t m_pad = (L.m + BN - 1) / BN * BN;
    const WsParts parts = ws_parts(T, L.n_in, L.n_out, L.m, L.num_sms, true);
    uint8_t *ws = static_cast<uint8_t *>(L.ws);
    uint16_t *B = reinterpret_cast<uint16_t *>(ws);
    uint16_t *S = P::MINS ? reinterpret_cast<uint16_t *>(ws + parts.b) : nullptr;
    float *DA = reinterpret_cast<float *>(ws + parts.b + parts.s);
    if (launch_prep_t<T>(L, nsb, m_pad, B, S, DA, st) != 0) return -2;
    CUtensorMap tmB, tmS;
    if (!make_map(&tmB, B, (uint64_t)(K * P::KSTEPS / 4), (uint64_t)m_pad, (uint64_t)(K * P::KSTEPS / 4) * 2, PF_KS,
                  BN, CU_TENSOR_MAP_SWIZZLE_128B, 2))
        return -4;
    if (P::MINS) {
        if (!make_map(&tmS, S, (uint64_t)(K / 16), (uint64_t)m_pad, (uint64_t)(K / 16) * 2, 16, BN,
                      CU_TENSOR_MAP_SWIZZLE_32B, 2))
            return -4;
    } else {
        tmS = tmB;   // unused
    }
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        cudaFuncSetAttribute(prefill_packed_kernel<T, BN>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (cudaFuncSetAttribute(prefill_packed_kernel<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Lay::SMEM) != cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    PkParams p{};
    p.pack = static_cast<const uint8_t *>(L.pack);
    p.n_out = (int)L.n_out;
    p.nsb = (int)nsb;
    p.da = DA;
    p.y = L.y;
    p.m = (int)L.m;
    p.m_pad = (int)m_pad;
    p.ntt = (int)(m_pad / BN);
    p.status = L.status;
    p.nsplit = split_count_bn(L.n_in, L.n_out, L.m, L.num_sms, BN, pk_us_per_sb(T, BN));
    p.sb_per_split = (int)((nsb + p.nsplit - 1) / p.nsplit);
    p.nsplit = (int)((nsb + p.sb_per_split - 1) / p.sb_per_split);   // no empty range
    p.part = p.nsplit > 1 ? reinterpret_cast<float *>(ws + parts.b + parts.s + parts.da + parts.pad) : nullptr;
    const int64_t tiles = (L.n_out + PF_BM - 1) / PF_BM * p.ntt;
    prefill_packed_kernel<T, BN><<<(unsigned)(tiles * p.nsplit), PK_WARPS * 32, Lay::SMEM, st>>>(tmB, tmS, p);
    if (cudaGetLastError() != cudaSuccess) return -2;
    if (p.nsplit > 1) {
        const int64_t n = L.m * L.n_out;
        const int64_t blocks = (n + 255) / 256 < 4 * L.num_sms ? (n + 255) / 256 : 4 * L.num_sms;
        prefill_sum_splits<<<(unsigned)blocks, 256, 0, st>>>(p.part, p.nsplit, n, L.y);
        if (cudaGetLastError() != cudaSuccess) return -2;
    }
    return 0;
}

template <uint32_t T, int BN>
int launch_pair_tb(const PrefillLaunch &L, cudaStream_t st) {
    using P = PkFmt<T>;
    using Lay = PpLayout<T, BN>;
    const int64_t K = L.n_in, nsb = K / QK_K;
    const int64_t m_pad = (L.m + BN - 1) / BN * BN;
    const int nmat = L.nmat > 1 ? L.nmat : 1;
    const int64_t *n_out = L.nmat > 1 ? L.n_outm : &L.n_out;
    const PairPlan pl = pair_plan(T, L.n_in, nmat, n_out, L.m, L.num_sms);
    const WsParts parts = ws_parts(T, L.n_in, L.n_out, L.m, L.num_sms, true);   // activation parts
    uint8_t *ws = static_cast<uint8_t *>(L.ws);
    uint16_t *B = reinterpret_cast<uint16_t *>(ws);
    uint16_t *S = P::MINS ? reinterpret_cast<uint16_t *>(ws + parts.b) : nullptr;
    float *DA = reinterpret_cast<float *>(ws + parts.b + parts.s);
    float *part = reinterpret_cast<float *>(ws + parts.b + parts.s + parts.da);
    if (launch_prep_t<T>(L, nsb, m_pad, B, S, DA, st) != 0) return -2;
    // each prefill copy as rows of 128 bytes: one K-step's A tile is 128 rows,
    // the mins operand 64 (the copy is already in the shared-memory layout, so
    // the maps do not swizzle)
    PpMaps maps;
    PpParams p{};
    int64_t tiles = 0, rows_before = 0;
    for (int i = 0; i < nmat; ++i) {
        const void *pack = L.nmat > 1 ? L.packm[i] : L.pack;
        const uint64_t copy_rows = prefill_pack_bytes(T, L.n_in, n_out[i]) / 128;
        if (!make_map(&maps.a[i], pack, 64, copy_rows, 128, 64, PF_BM, CU_TENSOR_MAP_SWIZZLE_NONE, 2) ||
            !make_map(&maps.mins[i], pack, 64, copy_rows, 128, 64, 64, CU_TENSOR_MAP_SWIZZLE_NONE, 2))
            return -4;
        p.pack[i] = static_cast<const uint8_t *>(pack);
        p.y[i] = L.nmat > 1 ? L.ym[i] : L.y;
        p.n_out[i] = (int)n_out[i];
        p.part[i] = part + (size_t)pl.nsplit * L.m * rows_before;
        tiles += ((n_out[i] + PF_BM - 1) / PF_BM + 1) / 2 * (m_pad / BN);
        p.tile_end[i] = (int)tiles;
        rows_before += n_out[i];
    }
    for (int i = nmat; i < PP_MAXM; ++i) maps.a[i] = maps.mins[i] = maps.a[0];
    CUtensorMap tmB, tmS;
    if (!make_map(&tmB, B, (uint64_t)(K * P::KSTEPS / 4), (uint64_t)m_pad, (uint64_t)(K * P::KSTEPS / 4) * 2, PF_KS,
                  Lay::HB, CU_TENSOR_MAP_SWIZZLE_128B, 2))
        return -4;
    if (P::MINS) {
        if (!make_map(&tmS, S, (uint64_t)(K / 16), (uint64_t)m_pad, (uint64_t)(K / 16) * 2, 16, Lay::HB,
                      CU_TENSOR_MAP_SWIZZLE_32B, 2))
            return -4;
    } else {
        tmS = tmB;   // unused
    }
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        cudaFuncSetAttribute(prefill_pair_kernel<T, BN>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (cudaFuncSetAttribute(prefill_pair_kernel<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Lay::SMEM) != cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    p.nmat = nmat;
    p.nsb = (int)nsb;
    p.nsplit = pl.nsplit;
    p.sb_per_split = pl.sb_per_split;
    p.da = DA;
    p.m = (int)L.m;
    p.m_pad = (int)m_pad;
    p.ntt = (int)(m_pad / BN);
    p.status = L.status;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(2 * tiles * p.nsplit));
    cfg.blockDim = dim3(PP_WARPS * 32);
    cfg.dynamicSmemBytes = Lay::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, prefill_pair_kernel<T, BN>, maps, tmB, tmS, p) != cudaSuccess) return -2;
    if (p.nsplit > 1) {
        for (int i = 0; i < nmat; ++i) {
            const int64_t n = L.m * n_out[i];
            const int64_t blocks = (n + 255) / 256 < 4 * L.num_sms ? (n + 255) / 256 : 4 * L.num_sms;
            prefill_sum_splits<<<(unsigned)blocks, 256, 0, st>>>(p.part[i], p.nsplit, n, p.y[i]);
            if (cudaGetLastError() != cudaSuccess) return -2;
        }
    }
    return 0;
}

// blocks of up to 32 tokens (batched decode) use 32-token tiles: the weights
// still stream once per token tile, with a quarter of the token-operand traffic
template <uint32_t T>
int launch_t(const PrefillLaunch &L, cudaStream_t st) {
    if (L.pack && L.m > PF_BN_SMALL) {
        if (L.nmat > 1 || use_pair(L.n_out))
            return pk_bn(L.m) == 256 ? launch_pair_tb<T, 256>(L, st) : launch_pair_tb<T, PF_BN>(L, st);
        return pk_bn(L.m) == 256 ? launch_packed_tb<T, 256>(L, st) : launch_packed_tb<T, PF_BN>(L, st);
    }
    return L.m <= PF_BN_SMALL ? launch_tb<T, PF_BN_SMALL>(L, st) : launch_tb<T, PF_BN>(L, st);
}

// formats with a prefill copy but no converter kernel: the copy only, and
// blocks of more than PF_BN_SMALL tokens
template <uint32_t T>
int launch_pk_t(const PrefillLaunch &L, cudaStream_t st) {
    if (!L.pack || L.m <= PF_BN_SMALL) return -3;
    if (L.nmat > 1 || use_pair(L.n_out))
        return pk_bn(L.m) == 256 ? launch_pair_tb<T, 256>(L, st) : launch_pair_tb<T, PF_BN>(L, st);
    return pk_bn(L.m) == 256 ? launch_packed_tb<T, 256>(L, st) : launch_packed_tb<T, PF_BN>(L, st);
}

template <uint32_t T>
constexpr int64_t block_bytes() {
    return T == T_Q4_K ? B_Q4_K : T == T_Q5_K ? B_Q5_K : T == T_Q6_K ? B_Q6_K : T == T_Q3_K ? B_Q3_K
         : T == T_F16 ? 512 : B_Q2_K;
}

template <uint32_t T>
int launch_pack_t(const void *w, int64_t n_in, int64_t n_out, void *pack, cudaStream_t st) {
    const int64_t nsb = n_in / QK_K, nrt = (n_out + PF_BM - 1) / PF_BM;
    const int64_t row_bytes = nsb * block_bytes<T>();
    prefill_pack_kernel<T><<<dim3((unsigned)nrt, (unsigned)nsb), PF_BM, 0, st>>>(
        static_cast<const uint8_t *>(w), row_bytes, (int)n_out, (int)nsb, static_cast<uint8_t *>(pack));
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---- classic formats (Q4_0, Q5_0, Q8_0) on int8 MMAs -------------------------------
// The reference's dots for these formats (src/kernels.c:197-247) form one
// exact integer sum per 32-element block, then add one float term per block
// into the row's running sum, in block order:
//   Q4_0, Q5_0: sumf += sumi * dx * dy      ((sumi dx) dy, left to right)
//   Q8_0:       sumf += sumi * (dx * dy)
// with dx, dy the blocks' f16 scales. Every quant fits int8 (Q4_0 q - 8,
// Q5_0 q - 16, Q8_0 q, the activation's Q8_0 quants), so one kind::i8 MMA of
// K = 32 gives a block's integer sums for 128 rows x 128 tokens exactly, in
// its own tensor-memory accumulator, and the epilogue replays the reference's
// float operations per block in order: the outputs are the reference's bits.
//
// Prefill copy of a classic matrix: per 128-row tile and K-step of four
// blocks (128 elements) one chunk of
//   [128 rows][128] int8   the quants, K-major, 128-byte swizzle (16-byte
//                          unit j of row r stored at j ^ (r & 7))
//   [128 rows][4] f32      the blocks' weight scales dx (0 past the row's end)
// Token operand: [m_pad][K] int8 (the activation's Q8_0 quants) and the
// blocks' activation scales dy as [nblk][m_pad] f32.
//
// One CTA: 128 rows x 128 tokens, 18 warps: warp 0 loads (bulk copies of the
// chunk and the scales, a TMA tile of the token quants), warp 1 owns tensor
// memory and issues one MMA per block into a ring of four 128-column
// accumulators, warps 2-17 are the epilogue (thread = row, 32 tokens, one
// running sum each; four warps per 32-lane quarter of tensor memory). The epilogue's five operations per (row, token, block)
// bound the kernel, about ten times the MMA time.
constexpr int I8_ATILE = PF_BM * 128;                // int8 quants of one K-step
constexpr int I8_CHUNK = I8_ATILE + PF_BM * 4 * 4;   // + the four blocks' row scales
constexpr int I8_BN = 128;                           // tokens per tile
constexpr int I8_S = 4, I8_NSC = 4, I8_NACC = 4;     // stages, scale buffers, accumulators
constexpr int I8_WARPS = 18, I8_NEPI = 16;   // loads, MMA, 16 epilogue warps (4 per lane quarter)
constexpr int I8_STAGE = I8_ATILE + I8_BN * 128;
constexpr int I8_SCBUF = PF_BM * 16 + 4 * I8_BN * 4;   // row scales [128][4], token scales [4][128]
constexpr int I8_OFF_SC = I8_S * I8_STAGE, I8_OFF_BAR = I8_OFF_SC + I8_NSC * I8_SCBUF;
constexpr int I8_SMEM = I8_OFF_BAR + 256 + 16 + 1024;
enum {
    I8B_FULL = 0, I8B_EMPTY = 4, I8B_SC_FULL = 8, I8B_SC_FREE = 12, I8B_ACC_FULL = 16, I8B_ACC_EMPTY = 20,
    I8B_DRAIN = 24, I8B_NBARS = 25,
};
static_assert(I8B_NBARS * 8 <= 256, "barrier area");

template <uint32_t T> struct I8Fmt;
template <> struct I8Fmt<T_Q8_0> { static constexpr int BLOCK = B_Q8_0; static constexpr bool SCALES_FIRST = true; };
template <> struct I8Fmt<T_Q4_0> { static constexpr int BLOCK = B_Q4_0; static constexpr bool SCALES_FIRST = false; };
template <> struct I8Fmt<T_Q5_0> { static constexpr int BLOCK = B_Q5_0; static constexpr bool SCALES_FIRST = false; };

// Instruction descriptor for kind::i8: signed int8 A and B, s32 accumulation,
// both K-major: [4,6) D format (2 = s32), [7,10) / [10,13) A / B format (1 =
// signed 8-bit), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_s8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// D[tmem] = A[smem] * B[smem]^T (the accumulator is overwritten); one thread issues
__device__ __forceinline__ void tc_mma_s8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0u)
        : "memory");
}

// Two f32 operations per instruction (sm_100 f32x2), each element rounded as
// the scalar operation rounds it. The int8 epilogue uses them for the exact
// integer-to-float conversion and the scale products; its running sums stay
// scalar additions: with packed additions after the packed products, some
// outputs differed from the reference by an ulp (measured), as a fused
// multiply-add would.
__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
    float2 r;
    asm("{.reg .b64 a_, b_, d_;\n\tmov.b64 a_, {%2, %3};\n\tmov.b64 b_, {%4, %5};\n\t"
        "mul.rn.f32x2 d_, a_, b_;\n\tmov.b64 {%0, %1}, d_;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    float2 r;
    asm("{.reg .b64 a_, b_, d_;\n\tmov.b64 a_, {%2, %3};\n\tmov.b64 b_, {%4, %5};\n\t"
        "add.rn.f32x2 d_, a_, b_;\n\tmov.b64 {%0, %1}, d_;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

// Quant e (0..31) of a classic block b (its bytes), as the reference's dots
// form it (src/kernels.c:203-205, 222-225, 241).
template <uint32_t T>
__device__ __forceinline__ int classic_quant(const uint8_t *b, int e) {
    if constexpr (T == T_Q8_0) {
        return (int)(int8_t)b[2 + e];
    } else if constexpr (T == T_Q4_0) {
        const int q = b[2 + (e & 15)];
        return (e < 16 ? (q & 15) : (q >> 4)) - 8;
    } else {
        const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        const int q = b[6 + (e & 15)];
        return (e < 16 ? ((q & 15) | (int)(((qh >> e) << 4) & 0x10u)) : ((q >> 4) | (int)((qh >> (e - 4)) & 0x10u))) - 16;
    }
}

// one CTA per (row tile, K-step); thread = row
template <uint32_t T>
__global__ void __launch_bounds__(PF_BM) prefill_pack_i8_kernel(const uint8_t *w, int64_t row_bytes, int n_out,
                                                               int nblk, uint8_t *pack) {
    const int rt = blockIdx.x, ks = blockIdx.y, nks = gridDim.y, r = threadIdx.x;
    const int64_t row = (int64_t)rt * PF_BM + r;
    const bool valid = row < n_out;
    uint8_t *chunk = pack + ((size_t)rt * nks + ks) * (size_t)I8_CHUNK;
    float *dst_d = reinterpret_cast<float *>(chunk + I8_ATILE) + 4 * r;
    uint32_t words[32];
#pragma unroll
    for (int bi = 0; bi < 4; ++bi) {
        const int b = 4 * ks + bi;
        const bool on = valid && b < nblk;
        const uint8_t *blk = w + (on ? row * row_bytes + (int64_t)b * I8Fmt<T>::BLOCK : 0);
        dst_d[bi] = on ? h2f((uint32_t)blk[0] | ((uint32_t)blk[1] << 8)) : 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t v = 0;
            if (on)
                for (int e = 0; e < 4; ++e) v |= (uint32_t)(classic_quant<T>(blk, 4 * k + e) & 0xff) << (8 * e);
            words[8 * bi + k] = v;
        }
    }
    uint8_t *dst = chunk + r * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        reinterpret_cast<uint4 *>(dst)[j ^ (r & 7)] =
            make_uint4(words[4 * j], words[4 * j + 1], words[4 * j + 2], words[4 * j + 3]);
}

// The token operand from f32 rows (the library's Q8_0 quantizer, the AVX2
// form the decode matvec uses) or from Q8_0 rows: thread = (token, block).
// Tokens m..m_pad-1 are zero.
__global__ void prefill_prep_i8(const float *xf, const uint8_t *xq, int m, int nblk, int m_pad, uint8_t *B,
                                float *DY) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)m_pad * nblk) return;
    const int t = (int)(i / nblk), b = (int)(i - (int64_t)t * nblk);
    const int64_t K = 32 * (int64_t)nblk;
    uint32_t q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float d = 0.0f;
    if (t < m) {
        if (xf) {
            uint32_t d16;
            q8_0_block(xf + t * K + 32 * (int64_t)b, d16, q);
            d = h2f(d16);
        } else {
            const uint16_t *blk = reinterpret_cast<const uint16_t *>(xq + ((int64_t)t * nblk + b) * B_Q8_0);
            d = h2f(blk[0]);
#pragma unroll
            for (int k = 0; k < 8; ++k) q[k] = (uint32_t)blk[1 + 2 * k] | ((uint32_t)blk[2 + 2 * k] << 16);
        }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(B + t * K + 32 * (int64_t)b);
    dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
    dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
    DY[(int64_t)b * m_pad + t] = d;
}

struct I8Params {
    const uint8_t *pack;
    const float *dy;
    float *y;
    int n_out, nblk, nks, m, m_pad, ntt;
    int *status;
};

template <uint32_t T>
__global__ void __launch_bounds__(I8_WARPS * 32, 1) prefill_i8_kernel(const __grid_constant__ CUtensorMap tmB,
                                                                       const I8Params p) {
    constexpr uint32_t FULL = 0xffffffffu;
    constexpr int EPI_COLS = I8_BN / (I8_NEPI / 4);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb0 = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = blockIdx.x / p.ntt, tt = blockIdx.x - rt * p.ntt;
    const int row0 = rt * PF_BM, tok0 = tt * I8_BN;
    const int rows = min(PF_BM, p.n_out - row0);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + I8_OFF_BAR + 256);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + I8_OFF_BAR + 256 + 4);
    const uint32_t barbase = sb0 + I8_OFF_BAR;
    auto bar = [&](int i) { return barbase + 8u * (uint32_t)i; };
    auto stage_a = [&](int s) { return sb0 + (uint32_t)(s * I8_STAGE); };
    auto stage_b = [&](int s) { return sb0 + (uint32_t)(s * I8_STAGE + I8_ATILE); };
    auto scbuf = [&](int b) { return (uint32_t)(I8_OFF_SC + b * I8_SCBUF); };   // offset from smem

    if (threadIdx.x == 0) {
        for (int i = 0; i < I8_S; ++i) {
            mbar_init(bar(I8B_FULL + i), 1);
            mbar_init(bar(I8B_EMPTY + i), 1);
        }
        for (int i = 0; i < I8_NSC; ++i) {
            mbar_init(bar(I8B_SC_FULL + i), 1);
            mbar_init(bar(I8B_SC_FREE + i), I8_NEPI);
        }
        for (int i = 0; i < I8_NACC; ++i) {
            mbar_init(bar(I8B_ACC_FULL + i), 1);
            mbar_init(bar(I8B_ACC_EMPTY + i), I8_NEPI);
        }
        mbar_init(bar(I8B_DRAIN), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_addr(tmem_slot), I8_NACC * I8_BN);
    if (warp == 0 && lane == 0) tma_prefetch_map(&tmB);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- loads: per K-step the scales (own ring) and the quant tiles ----
        if (lane == 0) {
            const uint8_t *chunks = p.pack + (size_t)rt * p.nks * (size_t)I8_CHUNK;
            int k_issued = 0, sc_issued = 0;
            for (int ks = 0; ks < p.nks; ++ks) {
                const int nb = min(4, p.nblk - 4 * ks);
                const uint8_t *ck = chunks + (size_t)ks * I8_CHUNK;
                const int b = ks % I8_NSC;
                if (!pf_wait(bar(I8B_SC_FREE + b), ((ks / I8_NSC) & 1) ^ 1, abort_flag, p.status)) break;
                const uint32_t sc = sb0 + scbuf(b);
                mbar_expect_tx(bar(I8B_SC_FULL + b), (uint32_t)(PF_BM * 16 + nb * I8_BN * 4));
                bulk_g2s(sc, ck + I8_ATILE, PF_BM * 16, bar(I8B_SC_FULL + b));
                for (int bi = 0; bi < nb; ++bi)
                    bulk_g2s(sc + PF_BM * 16 + bi * I8_BN * 4, p.dy + (size_t)(4 * ks + bi) * p.m_pad + tok0,
                             I8_BN * 4, bar(I8B_SC_FULL + b));
                sc_issued = ks + 1;
                const int s = ks % I8_S;
                if (!pf_wait(bar(I8B_EMPTY + s), ((ks / I8_S) & 1) ^ 1, abort_flag, p.status)) break;
                mbar_expect_tx(bar(I8B_FULL + s), (uint32_t)I8_STAGE);
                bulk_g2s(stage_a(s), ck, I8_ATILE, bar(I8B_FULL + s));
                tma_load_2d(stage_b(s), &tmB, 128 * ks, tok0, bar(I8B_FULL + s));
                k_issued = ks + 1;
            }
            if (*abort_flag) {
                for (int t = max(0, k_issued - I8_S); t < k_issued; ++t) pf_settle(bar(I8B_FULL + t % I8_S), (t / I8_S) & 1);
                for (int t = max(0, sc_issued - I8_NSC); t < sc_issued; ++t)
                    pf_settle(bar(I8B_SC_FULL + t % I8_NSC), (t / I8_NSC) & 1);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue: one K = 32 MMA per block into its own accumulator ----
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_s8(PF_BM, I8_BN);
            bool ok = true;
            for (int ks = 0; ks < p.nks && ok; ++ks) {
                const int nb = min(4, p.nblk - 4 * ks), s = ks % I8_S;
                if (!pf_wait<true>(bar(I8B_FULL + s), (uint32_t)(ks / I8_S) & 1u, abort_flag, p.status)) break;
                tc_fence_after();
                for (int bi = 0; bi < nb; ++bi) {
                    const int g = 4 * ks + bi, a = g % I8_NACC;
                    if (!pf_wait<true>(bar(I8B_ACC_EMPTY + a), ((g / I8_NACC) & 1) ^ 1, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // block bi: 32 bytes into the 128-byte swizzle atom of each row
                    tc_mma_s8(tmem + (uint32_t)(a * I8_BN), smem_desc(stage_a(s) + 32 * bi, 1024, SMEM_SWZ_128B),
                              smem_desc(stage_b(s) + 32 * bi, 1024, SMEM_SWZ_128B), idesc);
                    tc_commit(bar(I8B_ACC_FULL + a));
                }
                tc_commit(bar(I8B_EMPTY + s));
            }
            if (*abort_flag) {
                tc_commit(bar(I8B_DRAIN));
                pf_settle(bar(I8B_DRAIN), 0);
            }
        }
    } else {
        // ---- epilogue: thread = row (tensor-memory lane), EPI_COLS tokens ----
        const int q = warp & 3;
        const int c0 = ((warp - 2) >> 2) * EPI_COLS;
        const int r = 32 * q + lane;
        float sum[EPI_COLS];
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) sum[j] = 0.0f;
        bool ok = true;
        for (int ks = 0; ks < p.nks && ok; ++ks) {
            const int nb = min(4, p.nblk - 4 * ks), b = ks % I8_NSC;
            if (!__all_sync(FULL, pf_wait(bar(I8B_SC_FULL + b), (uint32_t)(ks / I8_NSC) & 1u, abort_flag, p.status))) {
                ok = false;
                break;
            }
            const uint8_t *scp = smem + scbuf(b);
            const float4 dx4 = reinterpret_cast<const float4 *>(scp)[r];
            const float dxs[4] = {dx4.x, dx4.y, dx4.z, dx4.w};
            for (int bi = 0; bi < nb; ++bi) {
                const int g = 4 * ks + bi, a = g % I8_NACC;
                if (!__all_sync(FULL, pf_wait(bar(I8B_ACC_FULL + a), (uint32_t)(g / I8_NACC) & 1u, abort_flag,
                                              p.status))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t v0[EPI_COLS];
                const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(a * I8_BN + c0);
                tmem_ld32x<EPI_COLS>(ta, v0);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(I8B_ACC_EMPTY + a));
                const float dx = dxs[bi];
                const float4 *dy4 = reinterpret_cast<const float4 *>(scp + PF_BM * 16 + bi * I8_BN * 4 + c0 * 4);
#pragma unroll
                for (int g4 = 0; g4 < EPI_COLS / 4; ++g4) {
                    const float4 dq = dy4[g4];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int j = 4 * g4 + 2 * e;   // tokens j, j + 1
                        // the blocks' integer sums (|sumi| < 2^20) to float, exactly
                        const float2 si = fadd2_rn(make_float2(__int_as_float((int)v0[j] + 0x4b400000),
                                                               __int_as_float((int)v0[j + 1] + 0x4b400000)),
                                                   make_float2(-12582912.0f, -12582912.0f));
                        const float2 dy = e ? make_float2(dq.z, dq.w) : make_float2(dq.x, dq.y);
                        const float2 dx2 = make_float2(dx, dx);
                        const float2 t = I8Fmt<T>::SCALES_FIRST ? fmul2_rn(si, fmul2_rn(dx2, dy))
                                                               : fmul2_rn(fmul2_rn(si, dx2), dy);
                        sum[j] = __fadd_rn(sum[j], t.x);
                        sum[j + 1] = __fadd_rn(sum[j + 1], t.y);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(I8B_SC_FREE + b));
        }
        if (ok && !*abort_flag && r < rows) {
            float *yr = p.y + row0 + r;
#pragma unroll
            for (int j = 0; j < EPI_COLS; ++j)
                if (tok0 + c0 + j < p.m) yr[(int64_t)(tok0 + c0 + j) * p.n_out] = sum[j];
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, I8_NACC * I8_BN);
    }
}

size_t i8_ws_b(int64_t n_in, int64_t m) { return align256((size_t)((m + I8_BN - 1) / I8_BN * I8_BN) * n_in); }
size_t i8_ws_bytes(int64_t n_in, int64_t m) {
    const int64_t m_pad = (m + I8_BN - 1) / I8_BN * I8_BN;
    return i8_ws_b(n_in, m) + align256((size_t)(n_in / 32) * m_pad * 4);
}

template <uint32_t T>
int launch_i8_t(const PrefillLaunch &L, cudaStream_t st) {
    if (!L.pack || L.m <= PF_BN_SMALL || L.nmat > 1 || L.n_in < 128) return -3;
    const int64_t K = L.n_in, nblk = K / 32, nks = (nblk + 3) / 4;
    const int64_t m_pad = (L.m + I8_BN - 1) / I8_BN * I8_BN;
    uint8_t *ws = static_cast<uint8_t *>(L.ws);
    uint8_t *B = ws;
    float *DY = reinterpret_cast<float *>(ws + i8_ws_b(L.n_in, L.m));
    const int64_t items = m_pad * nblk;
    prefill_prep_i8<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(L.xf, static_cast<const uint8_t *>(L.xq),
                                                                      (int)L.m, (int)nblk, (int)m_pad, B, DY);
    if (cudaGetLastError() != cudaSuccess) return -2;
    CUtensorMap tmB;
    if (!make_map(&tmB, B, (uint64_t)K, (uint64_t)m_pad, (uint64_t)K, 128, I8_BN, CU_TENSOR_MAP_SWIZZLE_128B, 1))
        return -4;
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        cudaFuncSetAttribute(prefill_i8_kernel<T>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (cudaFuncSetAttribute(prefill_i8_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, I8_SMEM) !=
            cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    I8Params p{};
    p.pack = static_cast<const uint8_t *>(L.pack);
    p.dy = DY;
    p.y = L.y;
    p.n_out = (int)L.n_out;
    p.nblk = (int)nblk;
    p.nks = (int)nks;
    p.m = (int)L.m;
    p.m_pad = (int)m_pad;
    p.ntt = (int)(m_pad / I8_BN);
    p.status = L.status;
    const int64_t tiles = (L.n_out + PF_BM - 1) / PF_BM * p.ntt;
    prefill_i8_kernel<T><<<(unsigned)tiles, I8_WARPS * 32, I8_SMEM, st>>>(tmB, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

template <uint32_t T>
int launch_pack_i8_t(const void *w, int64_t n_in, int64_t n_out, void *pack, cudaStream_t st) {
    const int64_t nblk = n_in / 32, nks = (nblk + 3) / 4, nrt = (n_out + PF_BM - 1) / PF_BM;
    prefill_pack_i8_kernel<T><<<dim3((unsigned)nrt, (unsigned)nks), PF_BM, 0, st>>>(
        static_cast<const uint8_t *>(w), nblk * I8Fmt<T>::BLOCK, (int)n_out, (int)nblk, static_cast<uint8_t *>(pack));
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace

bool prefill_supported(uint32_t wtype) { return wtype == T_Q4_K || wtype == T_Q6_K; }
bool is_classic(uint32_t wtype) { return wtype == T_Q4_0 || wtype == T_Q5_0 || wtype == T_Q8_0; }
bool prefill_pack_supported(uint32_t wtype) {
    return wtype == T_Q2_K || wtype == T_Q3_K || wtype == T_Q4_K || wtype == T_Q5_K || wtype == T_Q6_K ||
           wtype == T_F16 || is_classic(wtype);
}
bool prefill_groupable(uint32_t wtype) { return prefill_pack_supported(wtype) && !is_classic(wtype); }

size_t prefill_workspace_bytes(uint32_t wtype, int64_t n_in, int64_t n_out, int64_t m, int num_sms, bool packed) {
    if (is_classic(wtype)) return i8_ws_bytes(n_in, m);
    const WsParts w = ws_parts(wtype, n_in, n_out, m, num_sms, packed && m > PF_BN_SMALL);
    return w.b + w.s + w.da + w.pad + w.part;
}

size_t prefill_group_workspace_bytes(uint32_t wtype, int64_t n_in, int nmat, const int64_t *n_out, int64_t m,
                                     int num_sms) {
    const WsParts w = ws_parts(wtype, n_in, n_out[0], m, num_sms, true);
    const PairPlan pl = pair_plan(wtype, n_in, nmat, n_out, m, num_sms);
    return w.b + w.s + w.da + (pl.nsplit > 1 ? align256((size_t)pl.nsplit * m * pl.sum_out * 4) : 0);
}

size_t prefill_pack_bytes(uint32_t wtype, int64_t n_in, int64_t n_out) {
    const int64_t nsb = n_in / QK_K, nrt = (n_out + PF_BM - 1) / PF_BM;
    if (is_classic(wtype)) return (size_t)(nrt * ((n_in / 32 + 3) / 4)) * (size_t)I8_CHUNK;
    switch (wtype) {
        case T_Q4_K: return (size_t)(nrt * nsb) * (size_t)pk_chunk<T_Q4_K>();
        case T_Q6_K: return (size_t)(nrt * nsb) * (size_t)pk_chunk<T_Q6_K>();
        case T_Q5_K: return (size_t)(nrt * nsb) * (size_t)pk_chunk<T_Q5_K>();
        case T_Q3_K: return (size_t)(nrt * nsb) * (size_t)pk_chunk<T_Q3_K>();
        case T_Q2_K: return (size_t)(nrt * nsb) * (size_t)pk_chunk<T_Q2_K>();
        case T_F16: return (size_t)(nrt * nsb) * (size_t)pk_chunk<T_F16>();
        default: return 0;
    }
}

int launch_prefill_pack(uint32_t wtype, const void *w, int64_t n_in, int64_t n_out, void *pack, cudaStream_t st) {
    switch (wtype) {
        case T_Q4_K: return launch_pack_t<T_Q4_K>(w, n_in, n_out, pack, st);
        case T_Q6_K: return launch_pack_t<T_Q6_K>(w, n_in, n_out, pack, st);
        case T_Q5_K: return launch_pack_t<T_Q5_K>(w, n_in, n_out, pack, st);
        case T_Q3_K: return launch_pack_t<T_Q3_K>(w, n_in, n_out, pack, st);
        case T_Q2_K: return launch_pack_t<T_Q2_K>(w, n_in, n_out, pack, st);
        case T_F16: return launch_pack_t<T_F16>(w, n_in, n_out, pack, st);
        case T_Q8_0: return launch_pack_i8_t<T_Q8_0>(w, n_in, n_out, pack, st);
        case T_Q4_0: return launch_pack_i8_t<T_Q4_0>(w, n_in, n_out, pack, st);
        case T_Q5_0: return launch_pack_i8_t<T_Q5_0>(w, n_in, n_out, pack, st);
        default: return -3;
    }
}

int launch_prefill(uint32_t wtype, const PrefillLaunch &L, cudaStream_t st) {
    switch (wtype) {
        case T_Q4_K: return launch_t<T_Q4_K>(L, st);
        case T_Q6_K: return launch_t<T_Q6_K>(L, st);
        case T_Q5_K: return launch_pk_t<T_Q5_K>(L, st);
        case T_Q3_K: return launch_pk_t<T_Q3_K>(L, st);
        case T_Q2_K: return launch_pk_t<T_Q2_K>(L, st);
        case T_F16: return launch_pk_t<T_F16>(L, st);
        case T_Q8_0: return launch_i8_t<T_Q8_0>(L, st);
        case T_Q4_0: return launch_i8_t<T_Q4_0>(L, st);
        case T_Q5_0: return launch_i8_t<T_Q5_0>(L, st);
        default: return -3;
    }
}

}  // namespace sicu
