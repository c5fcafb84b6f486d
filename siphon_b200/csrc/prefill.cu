// Prefill matrix product on the 5th-generation tensor cores: Y = X W^T for a
// block of m >= 64 tokens, X quantized to Q8_K rows, W in its GGUF K-quant
// blocks. Y[t][r] is the reference's per-row dot product (for Q4_K,
// si_dot_q4_K_q8_K, src/kernels.c:349-410) for every (token, row) pair:
//
//   Y[t][r] = sum_sb dA[t][sb] * ( d[r][sb] * S1 - dmin[r][sb] * S2 )
//   S1 = sum_k (sc * q)[r][k] * qa[t][k]                         (256 k)
//   S2 = sum_j mn[r][j] * (bsums[t][2j] + bsums[t][2j+1])
//
// Every factor of S1 and S2 is a small integer that f16 holds exactly
// (sc * q <= 945, |qa| <= 127, |bsums| <= 2032), so kind::f16 MMAs with f32
// accumulation produce the integer sums (exactly while partial sums stay below
// 2^24), and only the float scaling per super-block rounds in a different order
// from the reference's lane sums. Outputs agree with the reference within a
// relative 1e-5 of the L1 norm of the products.
//
// One CTA computes a 128-row x 128-token tile (one SM; 15 warps):
//   warp 0      TMA: token operand (f16, 128-byte swizzle), bsums, dA
//   warp 1      TMEM owner; lane 0 issues the MMAs
//   warp 2      bulk copies of raw weight super-blocks (3 buffers)
//   warps 3-6   weight converters: raw blocks -> f16 (sc*q) tiles in the
//               swizzled K-major layout, mins tile, per-row d / dmin
//   warps 7-14  epilogue: per super-block, S1/S2 from tensor memory, scale,
//               accumulate in registers; write Y at the end (two warps per
//               32-lane quarter of tensor memory, 64 token columns each)
// Tensor memory: two accumulator sets (S1, S2: 128 columns each), so the MMAs
// of super-block sb+1 run while the epilogue drains sb.
#include <cudaTypedefs.h>

#include "launch.h"
#include "tc.cuh"

namespace sicu {

namespace {

constexpr int PF_BM = 128;        // weight rows per tile (MMA M)
constexpr int PF_BN = 128;        // tokens per tile (MMA N)
constexpr int PF_KS = 64;         // k slots per pipeline stage: one 128-byte swizzle atom of f16
constexpr int PF_STAGES = 4;
constexpr int PF_NRAW = 3;
constexpr int PF_STAGE_BYTES = PF_BM * PF_KS * 2;   // 16 KB; the token stage has the same size
constexpr int PF_MIN_BYTES = PF_BM * 16 * 2;        // 4 KB: 128 rows x 16 f16 (32-byte swizzle)

constexpr int W_TMA = 0, W_MMA = 1, W_RAW = 2, W_CONV = 3, N_CONV = 4, W_EPI = 7, N_EPI = 8;
constexpr int PF_WARPS = 15;
constexpr int EPI_COLS = PF_BN / 2;   // token columns per epilogue warp

// shared-memory map (offsets from a 1024-byte aligned base)
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + PF_STAGES * PF_STAGE_BYTES;
constexpr int OFF_RAW = OFF_B + PF_STAGES * PF_STAGE_BYTES;
constexpr int RAW_BUF = PF_BM * B_Q4_K;                                  // 18432
constexpr int OFF_A2 = (OFF_RAW + PF_NRAW * RAW_BUF + 1023) & ~1023;
constexpr int OFF_B2 = OFF_A2 + 2 * PF_MIN_BYTES;
constexpr int OFF_DA = OFF_B2 + 2 * PF_MIN_BYTES;
constexpr int OFF_DW = OFF_DA + 2 * PF_BN * 4;
constexpr int OFF_DM = OFF_DW + 2 * PF_BM * 4;
constexpr int OFF_BAR = OFF_DM + 2 * PF_BM * 4;
// barriers
enum {
    BAR_B_FULL = 0,                          // [4] token stage landed (TMA bytes)
    BAR_A_FULL = BAR_B_FULL + PF_STAGES,     // [4] weight stage converted (4 warps)
    BAR_ST_EMPTY = BAR_A_FULL + PF_STAGES,   // [4] stage consumed by the MMAs (commit)
    BAR_RAW_FULL = BAR_ST_EMPTY + PF_STAGES, // [3] raw super-block landed (bulk bytes)
    BAR_RAW_EMPTY = BAR_RAW_FULL + PF_NRAW,  // [3] raw super-block converted (4 warps)
    BAR_SBD_FULL = BAR_RAW_EMPTY + PF_NRAW,  // [2] bsums tile + dA landed (TMA bytes)
    BAR_A2_FULL = BAR_SBD_FULL + 2,          // [2] mins tile, d, dmin written (4 warps)
    BAR_SB_FREE = BAR_A2_FULL + 2,           // [2] epilogue done with a super-block (8 warps)
    BAR_ACC_FULL = BAR_SB_FREE + 2,          // [2] accumulators of a super-block ready (commit)
    BAR_ACC_EMPTY = BAR_ACC_FULL + 2,        // [2] accumulators read (8 warps)
    BAR_DRAIN = BAR_ACC_EMPTY + 2,           // teardown after an abandoned wait
    NBARS = BAR_DRAIN + 1,
};
constexpr int OFF_FLAGS = OFF_BAR + 8 * NBARS;   // abort flag, TMEM address
constexpr int PF_SMEM = OFF_FLAGS + 16 + 1024;   // + alignment slack
constexpr uint32_t PF_TMEM_COLS = 512;

struct PfParams {
    const uint8_t *w;     // weight blocks, row-major
    int64_t row_bytes;
    int n_out;
    int nsb;              // super-blocks per row
    const float *da;      // [nsb][m_pad] token scales
    float *y;             // [m][n_out]
    int m, m_pad;
    int ntt;              // token tiles
    int *status;
};

// Bounded wait shared by all roles: gives up when another role already gave
// up, or after 2 s, recording the failure in the status word.
__device__ __forceinline__ bool pf_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
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

// 128-byte swizzle, K-major: row r, 16-byte chunk j of a 128-row x 64-f16 tile
__device__ __forceinline__ uint32_t swz128(int r, int j) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}
// 32-byte swizzle, K-major: row r, chunk j (0/1) of a 128-row x 16-f16 tile
__device__ __forceinline__ uint32_t swz32(int r, int j) {
    return (uint32_t)((r >> 3) * 256 + (r & 7) * 32 + ((j ^ ((r >> 2) & 1)) << 4));
}

// f16 pair (1024 + q0, 1024 + q2) from the low nibbles of bytes 0 and 2 of x
// (mask 0x000f000f) or 1024 + 16 q from the high nibbles (mask 0x00f000f0),
// then one fused multiply-add per pair removes the 1024 bias exactly:
// (1024 + q) * sc - 1024 * sc = q * sc, and (1024 + 16 q) * sc/16 - 64 * sc.
__device__ __forceinline__ uint32_t nib_f16(uint32_t x, uint32_t mask, uint32_t mul, uint32_t add) {
    return hfma2_u32(and_or(x, mask, 0x64006400u), mul, add);
}

__global__ void __launch_bounds__(PF_WARPS * 32, 1)
prefill_q4k_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmS,
                   const PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb0 = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = blockIdx.x / p.ntt, tt = blockIdx.x - rt * p.ntt;
    const int row0 = rt * PF_BM, tok0 = tt * PF_BN;
    const int rows = min(PF_BM, p.n_out - row0);
    const int nsb = p.nsb;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_FLAGS);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_FLAGS + 4);
    auto bar = [&](int i) { return sb0 + OFF_BAR + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STAGES; ++i) {
            mbar_init(bar(BAR_B_FULL + i), 1);
            mbar_init(bar(BAR_A_FULL + i), N_CONV);
            mbar_init(bar(BAR_ST_EMPTY + i), 1);
        }
        for (int i = 0; i < PF_NRAW; ++i) {
            mbar_init(bar(BAR_RAW_FULL + i), 1);
            mbar_init(bar(BAR_RAW_EMPTY + i), N_CONV);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(BAR_SBD_FULL + i), 1);
            mbar_init(bar(BAR_A2_FULL + i), N_CONV);
            mbar_init(bar(BAR_SB_FREE + i), N_EPI);
            mbar_init(bar(BAR_ACC_FULL + i), 1);
            mbar_init(bar(BAR_ACC_EMPTY + i), N_EPI);
        }
        mbar_init(bar(BAR_DRAIN), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) tmem_alloc(smem_addr(tmem_slot), PF_TMEM_COLS);
    if (warp == W_TMA && lane == 0) {
        tma_prefetch_map(&tmB);
        tma_prefetch_map(&tmS);
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
                const int b2 = sb & 1;
                if (!pf_wait(bar(BAR_SB_FREE + b2), ((sb >> 1) & 1) ^ 1, abort_flag, p.status)) break;
                mbar_expect_tx(bar(BAR_SBD_FULL + b2), PF_MIN_BYTES + PF_BN * 4);
                tma_load_2d(sb0 + OFF_B2 + b2 * PF_MIN_BYTES, &tmS, 16 * sb, tok0, bar(BAR_SBD_FULL + b2));
                bulk_g2s(sb0 + OFF_DA + b2 * PF_BN * 4, p.da + (size_t)sb * p.m_pad + tok0, PF_BN * 4,
                         bar(BAR_SBD_FULL + b2));
                sb_issued = sb + 1;
                bool ok = true;
                for (int c = 0; c < 4; ++c) {
                    const int t = 4 * sb + c, s = t & 3;
                    if (!pf_wait(bar(BAR_ST_EMPTY + s), ((t >> 2) & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
                    mbar_expect_tx(bar(BAR_B_FULL + s), PF_STAGE_BYTES);
                    tma_load_2d(sb0 + OFF_B + s * PF_STAGE_BYTES, &tmB, PF_KS * t, tok0, bar(BAR_B_FULL + s));
                    t_issued = t + 1;
                }
                if (!ok) break;
            }
            if (*abort_flag) {
                for (int t = max(0, t_issued - PF_STAGES); t < t_issued; ++t) pf_settle(bar(BAR_B_FULL + (t & 3)), (t >> 2) & 1);
                for (int sb = max(0, sb_issued - 2); sb < sb_issued; ++sb) pf_settle(bar(BAR_SBD_FULL + (sb & 1)), (sb >> 1) & 1);
            }
        }
    } else if (warp == W_MMA) {
        // ---- MMA issue ----
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(PF_BM, PF_BN);
            for (int sb = 0; sb < nsb; ++sb) {
                const int buf = sb & 1;
                const uint32_t ph = (sb >> 1) & 1;
                if (!pf_wait(bar(BAR_ACC_EMPTY + buf), ph ^ 1, abort_flag, p.status)) break;
                tc_fence_after();
                const uint32_t d1 = tmem + (uint32_t)buf * 256u, d2 = d1 + 128u;
                bool ok = true;
                for (int c = 0; c < 4; ++c) {
                    const int t = 4 * sb + c, s = t & 3;
                    const uint32_t sph = (t >> 2) & 1;
                    if (!pf_wait(bar(BAR_A_FULL + s), sph, abort_flag, p.status) ||
                        !pf_wait(bar(BAR_B_FULL + s), sph, abort_flag, p.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = sb0 + OFF_A + s * PF_STAGE_BYTES, b = sb0 + OFF_B + s * PF_STAGE_BYTES;
#pragma unroll
                    for (int kk = 0; kk < PF_KS / 16; ++kk)
                        tc_mma_f16(d1, smem_desc(a + 32 * kk, 1024, SMEM_SWZ_128B),
                                   smem_desc(b + 32 * kk, 1024, SMEM_SWZ_128B), idesc, (c | kk) != 0);
                    tc_commit(bar(BAR_ST_EMPTY + s));
                }
                if (!ok) break;
                if (!pf_wait(bar(BAR_A2_FULL + buf), ph, abort_flag, p.status) ||
                    !pf_wait(bar(BAR_SBD_FULL + buf), ph, abort_flag, p.status)) break;
                tc_fence_after();
                tc_mma_f16(d2, smem_desc(sb0 + OFF_A2 + buf * PF_MIN_BYTES, 256, SMEM_SWZ_32B),
                           smem_desc(sb0 + OFF_B2 + buf * PF_MIN_BYTES, 256, SMEM_SWZ_32B), idesc, 0);
                tc_commit(bar(BAR_ACC_FULL + buf));
            }
            if (*abort_flag) {
                tc_commit(bar(BAR_DRAIN));
                pf_settle(bar(BAR_DRAIN), 0);
            }
        }
    } else if (warp == W_RAW) {
        // ---- raw weight super-blocks: one 144-byte bulk copy per row ----
        int sb_issued = 0;
        for (int sb = 0; sb < nsb; ++sb) {
            const int rb = sb % PF_NRAW;
            if (!__all_sync(FULL, pf_wait(bar(BAR_RAW_EMPTY + rb), ((sb / PF_NRAW) & 1) ^ 1, abort_flag, p.status)))
                break;
            if (lane == 0) mbar_expect_tx(bar(BAR_RAW_FULL + rb), (uint32_t)rows * B_Q4_K);
            __syncwarp();
            const uint8_t *src = p.w + (int64_t)row0 * p.row_bytes + (int64_t)sb * B_Q4_K;
            for (int r = lane; r < rows; r += 32)
                bulk_g2s(sb0 + OFF_RAW + rb * RAW_BUF + r * B_Q4_K, src + (int64_t)r * p.row_bytes, B_Q4_K,
                         bar(BAR_RAW_FULL + rb));
            sb_issued = sb + 1;
        }
        if (*abort_flag && lane == 0)
            for (int sb = max(0, sb_issued - PF_NRAW); sb < sb_issued; ++sb)
                pf_settle(bar(BAR_RAW_FULL + sb % PF_NRAW), (sb / PF_NRAW) & 1);
    } else if (warp < W_EPI) {
        // ---- weight converters: thread = tile row ----
        const int r = (warp - W_CONV) * 32 + lane;
        const bool valid = r < rows;
        for (int sb = 0; sb < nsb; ++sb) {
            const int rb = sb % PF_NRAW, b2 = sb & 1;
            if (!__all_sync(FULL, pf_wait(bar(BAR_RAW_FULL + rb), (sb / PF_NRAW) & 1, abort_flag, p.status))) break;
            if (!__all_sync(FULL, pf_wait(bar(BAR_SB_FREE + b2), ((sb >> 1) & 1) ^ 1, abort_flag, p.status))) break;
            const uint32_t raw = sb0 + OFF_RAW + rb * RAW_BUF + r * B_Q4_K;
            const uint4 h = valid ? lds128(raw) : make_uint4(0, 0, 0, 0);
            // 6-bit scales / mins (src/kernels.c:377-382)
            const uint32_t sc_lo = h.y & 0x3f3f3f3fu;
            const uint32_t mn_lo = h.z & 0x3f3f3f3fu;
            const uint32_t sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
            reinterpret_cast<float *>(smem + OFF_DW)[b2 * PF_BM + r] = valid ? h2f(h.x & 0xffffu) : 0.0f;
            reinterpret_cast<float *>(smem + OFF_DM)[b2 * PF_BM + r] = valid ? h2f(h.x >> 16) : 0.0f;
            // mins tile: column i (bsums index) holds mn[i / 2]
            uint32_t mw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float mv = (float)byte_at(j < 4 ? mn_lo : mn_hi, j & 3);
                mw[j] = half2_bits(mv, mv);
            }
            const uint32_t a2 = sb0 + OFF_A2 + b2 * PF_MIN_BYTES;
            sts128(a2 + swz32(r, 0), mw[0], mw[1], mw[2], mw[3]);
            sts128(a2 + swz32(r, 1), mw[4], mw[5], mw[6], mw[7]);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(BAR_A2_FULL + b2));
            bool ok = true;
            for (int c = 0; c < 4; ++c) {
                const int t = 4 * sb + c, s = t & 3;
                if (!__all_sync(FULL, pf_wait(bar(BAR_ST_EMPTY + s), ((t >> 2) & 1) ^ 1, abort_flag, p.status))) {
                    ok = false;
                    break;
                }
                const uint32_t abase = sb0 + OFF_A + s * PF_STAGE_BYTES;
                // sub-block 2c: low nibbles of qs[32c..32c+31]; 2c+1: high nibbles
                const uint4 q0 = lds128(raw + 16 + 32 * c), q1 = lds128(raw + 32 + 32 * c);
                const uint32_t x[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                const uint32_t scw = c < 2 ? sc_lo : sc_hi;
                const float slo = valid ? (float)byte_at(scw, (2 * c) & 3) : 0.0f;
                const float shi = valid ? (float)byte_at(scw, (2 * c + 1) & 3) : 0.0f;
                const uint32_t mlo = half2_bits(slo, slo), alo = half2_bits(-1024.0f * slo, -1024.0f * slo);
                const uint32_t mhi = half2_bits(0.0625f * shi, 0.0625f * shi), ahi = half2_bits(-64.0f * shi, -64.0f * shi);
                // slot order inside each group of four: elements 0, 2, 1, 3
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t u = x[2 * j], v = x[2 * j + 1];
                    sts128(abase + swz128(r, j), nib_f16(u, 0x000f000fu, mlo, alo), nib_f16(u >> 8, 0x000f000fu, mlo, alo),
                           nib_f16(v, 0x000f000fu, mlo, alo), nib_f16(v >> 8, 0x000f000fu, mlo, alo));
                    sts128(abase + swz128(r, 4 + j), nib_f16(u, 0x00f000f0u, mhi, ahi),
                           nib_f16(u >> 8, 0x00f000f0u, mhi, ahi), nib_f16(v, 0x00f000f0u, mhi, ahi),
                           nib_f16(v >> 8, 0x00f000f0u, mhi, ahi));
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(BAR_A_FULL + s));
            }
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
            const int buf = sb & 1;
            const uint32_t ph = (sb >> 1) & 1;
            if (!__all_sync(FULL, pf_wait(bar(BAR_ACC_FULL + buf), ph, abort_flag, p.status) &&
                                      pf_wait(bar(BAR_A2_FULL + buf), ph, abort_flag, p.status) &&
                                      pf_wait(bar(BAR_SBD_FULL + buf), ph, abort_flag, p.status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float dw = reinterpret_cast<const float *>(smem + OFF_DW)[buf * PF_BM + r];
            const float ndm = -reinterpret_cast<const float *>(smem + OFF_DM)[buf * PF_BM + r];
            const float4 *da4 = reinterpret_cast<const float4 *>(smem + OFF_DA + buf * PF_BN * 4 + c0 * 4);
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)buf * 256u + (uint32_t)c0;
#pragma unroll
            for (int cc = 0; cc < EPI_COLS / 16; ++cc) {
                uint32_t v1[16], v2[16];
                tmem_ld16(ta + 16 * cc, v1);
                tmem_ld16(ta + 128 + 16 * cc, v2);
                tmem_wait_ld(v1);
                tmem_wait_ld(v2);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const float4 d = da4[4 * cc + g];
                    const float dv[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = 4 * g + e;
                        const float sv = fmaf(ndm, __uint_as_float(v2[j]), dw * __uint_as_float(v1[j]));
                        acc[16 * cc + j] = fmaf(dv[e], sv, acc[16 * cc + j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(BAR_ACC_EMPTY + buf));
                mbar_arrive(bar(BAR_SB_FREE + buf));
            }
        }
        if (ok && !*abort_flag && r < rows) {
            float *yr = p.y + row0 + r;
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

// Q8_K rows -> token operand for the MMAs: f16 quants with the slots of each
// group of four holding elements 0, 2, 1, 3 (the order the weight converters
// produce), f16 bsums, and the block scales transposed to [sb][token].
// Tokens m..m_pad-1 are zero.
__global__ void prefill_prep_q8k(const uint8_t *xq, int m, int nsb, int m_pad, uint16_t *B, uint16_t *S, float *DA) {
    const int sb = blockIdx.x, t = blockIdx.y, i = threadIdx.x;   // 64 threads
    const int64_t K = (int64_t)nsb * QK_K;
    uint2 out = make_uint2(0, 0);
    if (t < m) {
        const uint8_t *blk = xq + ((int64_t)t * nsb + sb) * B_Q8_K;
        const uint32_t w = *reinterpret_cast<const uint32_t *>(blk + 4 + 4 * i);
        const float e0 = (float)(int8_t)byte_at(w, 0), e1 = (float)(int8_t)byte_at(w, 1);
        const float e2 = (float)(int8_t)byte_at(w, 2), e3 = (float)(int8_t)byte_at(w, 3);
        out.x = half2_bits(e0, e2);
        out.y = half2_bits(e1, e3);
        if (i < 16) {
            const int16_t bs = *reinterpret_cast<const int16_t *>(blk + 260 + 2 * i);
            S[(int64_t)t * (K / 16) + 16 * sb + i] = __half_as_ushort(__float2half_rn((float)bs));
        }
        if (i == 0) DA[(int64_t)sb * m_pad + t] = *reinterpret_cast<const float *>(blk);
    } else {
        if (i < 16) S[(int64_t)t * (K / 16) + 16 * sb + i] = 0;
        if (i == 0) DA[(int64_t)sb * m_pad + t] = 0.0f;
    }
    *reinterpret_cast<uint2 *>(B + (int64_t)t * K + (int64_t)QK_K * sb + 4 * i) = out;
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

// 2-D f16 tensor [rows][cols] (cols contiguous), box {bx cols, by rows}
bool make_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint32_t bx, uint32_t by,
              CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {bx, by};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

bool prefill_supported(uint32_t wtype) { return wtype == T_Q4_K; }

size_t prefill_workspace_bytes(int64_t n_in, int64_t m) {
    const int64_t m_pad = (m + PF_BN - 1) / PF_BN * PF_BN;
    return align256((size_t)m_pad * n_in * 2) + align256((size_t)m_pad * (n_in / 16) * 2) +
           align256((size_t)(n_in / QK_K) * m_pad * 4);
}

int launch_prefill(uint32_t wtype, const PrefillLaunch &L, cudaStream_t st) {
    if (wtype != T_Q4_K) return -3;
    const int64_t K = L.n_in, nsb = K / QK_K;
    const int64_t m_pad = (L.m + PF_BN - 1) / PF_BN * PF_BN;
    uint8_t *ws = static_cast<uint8_t *>(L.ws);
    uint16_t *B = reinterpret_cast<uint16_t *>(ws);
    uint16_t *S = reinterpret_cast<uint16_t *>(ws + align256((size_t)m_pad * K * 2));
    float *DA = reinterpret_cast<float *>(ws + align256((size_t)m_pad * K * 2) + align256((size_t)m_pad * (K / 16) * 2));
    prefill_prep_q8k<<<dim3((unsigned)nsb, (unsigned)m_pad), 64, 0, st>>>(static_cast<const uint8_t *>(L.xq), (int)L.m,
                                                                          (int)nsb, (int)m_pad, B, S, DA);
    if (cudaGetLastError() != cudaSuccess) return -2;

    CUtensorMap tmB, tmS;
    if (!make_map(&tmB, B, (uint64_t)K, (uint64_t)m_pad, PF_KS, PF_BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tmS, S, (uint64_t)(K / 16), (uint64_t)m_pad, 16, PF_BN, CU_TENSOR_MAP_SWIZZLE_32B))
        return -4;
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(prefill_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM) !=
            cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    PfParams p{};
    p.w = static_cast<const uint8_t *>(L.w);
    p.row_bytes = nsb * B_Q4_K;
    p.n_out = (int)L.n_out;
    p.nsb = (int)nsb;
    p.da = DA;
    p.y = L.y;
    p.m = (int)L.m;
    p.m_pad = (int)m_pad;
    p.ntt = (int)(m_pad / PF_BN);
    p.status = L.status;
    const int64_t tiles = (L.n_out + PF_BM - 1) / PF_BM * p.ntt;
    prefill_q4k_kernel<<<(unsigned)tiles, PF_WARPS * 32, PF_SMEM, st>>>(tmB, tmS, p);
    if (cudaGetLastError() != cudaSuccess) return -2;
    return 0;
}

}  // namespace sicu
