// Persistent streaming matvec driver (see gemv.cuh for the design notes).
#include "gemv.cuh"
#include "quantize.cuh"
#include "launch.h"

namespace sicu {

namespace {

struct Item {
    int64_t task, row0;
    int rows, chunk, u0, cu;
    int64_t byte_start, byte_len;
};

template <uint32_t T>
__device__ __forceinline__ Item item_of(const GemvParams &p, int64_t t0, int warp, int64_t k) {
    Item it;
    it.task = t0 + warp + (k / p.nchunks) * GEMV_WARPS;
    it.chunk = (int)(k % p.nchunks);
    it.row0 = it.task * p.rows_per_task;
    const int64_t left = p.n_out - it.row0;
    it.rows = left < p.rows_per_task ? (int)left : p.rows_per_task;
    it.u0 = it.chunk * p.cu;
    it.cu = min(p.cu, p.nu - it.u0);
    it.byte_start = it.row0 * p.row_bytes + (int64_t)it.u0 * Fmt<T>::unit_bytes;
    if (p.nchunks == 1) {
        it.byte_len = it.rows * p.row_bytes;
    } else {
        const int64_t rest = p.row_bytes - (int64_t)it.u0 * Fmt<T>::unit_bytes;
        const int64_t want = (int64_t)it.cu * Fmt<T>::unit_bytes;
        it.byte_len = want < rest ? want : rest;
    }
    return it;
}

// Fill one ring slot with an item's bytes: a 16-byte aligned bulk copy plus,
// at the very end of the matrix, up to 15 tail bytes copied by lanes.
__device__ __forceinline__ void issue_item(const GemvParams &p, const Item &it, uint8_t *slot, uint32_t bar,
                                           int lane, uint64_t policy) {
    const uint8_t *src = p.w + it.byte_start;
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    const uint8_t *al = reinterpret_cast<const uint8_t *>(a & ~uintptr_t(15));
    const int64_t head = (int64_t)(a & 15);
    const uint8_t *mend = p.w + p.n_out * p.row_bytes;
    int64_t bulk = (head + it.byte_len + 15) & ~int64_t(15);
    if (al + bulk > mend) bulk = (int64_t)(mend - al) & ~int64_t(15);
    const int64_t tail = head + it.byte_len - bulk;
    if (lane == 0) {
        fence_proxy_async();
        mbar_expect_tx(bar, (uint32_t)bulk);
        if (bulk > 0) bulk_g2s_hint(smem_addr(slot), al, (uint32_t)bulk, bar, policy);
    }
    if (tail > 0 && lane < tail) slot[bulk + lane] = (uint8_t)ldg_u8(al + bulk + lane);
}

template <uint32_t T>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 1) gemv_kernel(const GemvParams p) {
    using F = Fmt<T>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const ActView av{smem, p.nu};
    uint8_t *wreg = smem + p.act_bytes + (size_t)warp * p.warp_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(wreg);   // up to 8 slots
    float *terms = reinterpret_cast<float *>(wreg + 64);   // TERM_FLOATS
    float *fin = terms + TERM_FLOATS;                      // 64 chain results
    uint8_t *slots = wreg + WARP_HDR;

    const int64_t t0 = (int64_t)blockIdx.x * p.ntasks / gridDim.x;
    const int64_t t1 = (int64_t)(blockIdx.x + 1) * p.ntasks / gridDim.x;
    const int64_t mine = (t1 - t0 > warp) ? (t1 - t0 - warp + GEMV_WARPS - 1) / GEMV_WARPS : 0;
    const int64_t items = mine * p.nchunks;
    const uint64_t policy = policy_evict_first();

    if (lane == 0) {
        for (int s = 0; s < p.nslots; ++s) mbar_init(smem_addr(&bars[s]), 1);
        fence_mbar_init();
    }
    __syncwarp();
    for (int64_t k = 0; k < items && k < p.nslots; ++k) {
        const Item it = item_of<T>(p, t0, warp, k);
        issue_item(p, it, slots + (size_t)k * p.slot_bytes, smem_addr(&bars[k]), lane, policy);
    }

    // activation: the caller's pair-format row, or quantized here from f32
    if (p.xf) {
        // the term buffer is idle until the main loop: use it as the 292-byte stage
        quantize_into_act<F::act>(av, p.xf, p.n_in, reinterpret_cast<uint8_t *>(terms));
    } else {
        prep_activation<F::act>(av, p.xq, p.n_in);
    }
    __syncthreads();

    constexpr int CH = F::chains;
    float acc[2] = {0.f, 0.f};
    int64_t failed_at = -1;
    for (int64_t k = 0; k < items; ++k) {
        const int s = (int)(k % p.nslots);
        const uint32_t parity = (uint32_t)((k / p.nslots) & 1);
        // warp-uniform verdict: a lane that timed out takes the whole warp out
        const bool landed = mbar_wait(smem_addr(&bars[s]), parity);
        if (!__all_sync(0xffffffffu, landed)) { failed_at = k; break; }
        __syncwarp();
        const Item it = item_of<T>(p, t0, warp, k);
        uint8_t *slot = slots + (size_t)s * p.slot_bytes;
        const uint8_t *data = slot + (reinterpret_cast<uintptr_t>(p.w + it.byte_start) & 15);

        // ---- phase 1: one unit per lane ----
        const int units = it.rows * it.cu;
        for (int q = lane; q < units; q += 32) {
            const int r = q / it.cu, u = q % it.cu, ug = it.u0 + u;
            const uint8_t *wb = data + (p.nchunks == 1 ? (int64_t)r * p.row_bytes : 0) + (int64_t)u * F::unit_bytes;
            if constexpr (F::kind == 3) {
                const int nblk_row = p.n_in / 32;
                const int nb = min(8, nblk_row - ug * 8);
                float t[8];
                unit_classic<T>(wb, nb, av.aq(ug), av.ad(ug), av.ax(ug), t);
                float *dst = terms + (r * it.cu + u) * 8;
#pragma unroll
                for (int b = 0; b < 8; ++b) if (b < nb) dst[b] = t[b];
            } else {
                float t[MAX_CHAINS];
                if constexpr (T == T_Q4_K) unit_q45k<false>(wb, av.aq(ug), av.ad(ug)[0], av.ax(ug), t);
                else if constexpr (T == T_Q5_K) unit_q45k<true>(wb, av.aq(ug), av.ad(ug)[0], av.ax(ug), t);
                else if constexpr (T == T_Q6_K) unit_q36k<false>(wb, av.aq(ug), av.ad(ug)[0], t);
                else if constexpr (T == T_Q3_K) unit_q36k<true>(wb, av.aq(ug), av.ad(ug)[0], t);
                else unit_q2k(wb, av.aq(ug), av.ad(ug)[0], av.ax(ug), t);
#pragma unroll
                for (int c = 0; c < CH; ++c) terms[(r * CH + c) * it.cu + u] = t[c];
            }
        }
        __syncwarp();
        // the slot is consumed: refill it with item k + nslots
        if (k + p.nslots < items) {
            const Item nx = item_of<T>(p, t0, warp, k + p.nslots);
            issue_item(p, nx, slot, smem_addr(&bars[s]), lane, policy);
        }

        // ---- phase 2: ordered float chains, one lane per (row, chain) ----
        if (it.chunk == 0) { acc[0] = 0.f; acc[1] = 0.f; }
        const int pairs = it.rows * CH;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int q = lane + 32 * h;
            if (q < pairs) {
                float a = acc[h];
                if constexpr (F::kind == 3) {
                    const int nblk_row = p.n_in / 32;
                    const int nb = min(it.cu * 8, nblk_row - it.u0 * 8);
                    const float *src = terms + q * it.cu * 8;
                    for (int b = 0; b < nb; ++b) a = __fadd_rn(a, src[b]);
                } else {
                    const float *src = terms + q * it.cu;
                    const bool sub = (F::kind == 0) && (q % CH == 8);
                    if (sub) {
                        for (int u = 0; u < it.cu; ++u) a = __fsub_rn(a, src[u]);
                    } else {
                        for (int u = 0; u < it.cu; ++u) a = __fadd_rn(a, src[u]);
                    }
                }
                acc[h] = a;
            }
        }
        if (it.chunk == p.nchunks - 1) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int q = lane + 32 * h;
                if (q < pairs) fin[q] = acc[h];
            }
            __syncwarp();
            if (lane < it.rows) {
                float s;
                if constexpr (F::kind == 0) {
                    s = fin[lane * CH + 8];
#pragma unroll
                    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, fin[lane * CH + l]);
                } else if constexpr (F::kind == 1) {
                    s = 0.0f;
#pragma unroll
                    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, fin[lane * CH + l]);
                } else {
                    s = fin[lane];
                }
                p.y[it.row0 + lane] = s;
            }
        }
        __syncwarp();
    }
    if (failed_at >= 0) {
        if (lane == 0) atomicOr(p.status, STATUS_WAIT_TIMEOUT);
        // let the copies still in flight land before the CTA's memory goes away
        for (int64_t k = failed_at; k < items && k < failed_at + p.nslots; ++k)
            (void)mbar_wait(smem_addr(&bars[k % p.nslots]), (uint32_t)((k / p.nslots) & 1), 1u << 16);
    }
}

}  // namespace

// ---- host side ------------------------------------------------------------------

template <uint32_t T>
static int launch_gemv_t(const GemvLaunch &L, cudaStream_t st) {
    using F = Fmt<T>;
    GemvParams p{};
    p.w = static_cast<const uint8_t *>(L.w);
    p.xq = static_cast<const uint8_t *>(L.xq);
    p.xf = L.xf;
    p.y = L.y;
    p.n_out = L.n_out;
    p.n_in = L.n_in;
    p.status = L.status;
    const int nblk = (F::kind == 3) ? L.n_in / 32 : L.n_in / 256;
    p.row_bytes = (int64_t)nblk * (F::kind == 3 ? F::unit_bytes / 8 : F::unit_bytes);
    p.nu = (F::kind == 3) ? (nblk + 7) / 8 : nblk;
    // rows x units-per-chunk <= 32 (one unit per lane); rows x chains <= 64
    if (p.nu <= 32) {
        p.nchunks = 1;
        p.cu = p.nu;
        p.rows_per_task = 32 / p.nu;
        if (F::chains > 1 && p.rows_per_task > 64 / F::chains) p.rows_per_task = 64 / F::chains;
    } else {
        p.nchunks = (p.nu + 31) / 32;
        p.cu = (p.nu + p.nchunks - 1) / p.nchunks;
        p.rows_per_task = 1;
    }
    p.ntasks = (p.n_out + p.rows_per_task - 1) / p.rows_per_task;
    const int64_t item_max = (p.nchunks == 1) ? p.rows_per_task * p.row_bytes : (int64_t)p.cu * F::unit_bytes;
    p.slot_bytes = (int)((item_max + 32 + 127) & ~int64_t(127));
    p.act_bytes = (ActView::bytes(p.nu) + 127) & ~127;
    const int hdr = WARP_HDR;
    const int budget = L.smem_limit - p.act_bytes;
    int slots = (budget / GEMV_WARPS - hdr) / p.slot_bytes;
    if (slots > 4) slots = 4;
    if (slots < 2) return -1;
    p.nslots = slots;
    p.warp_bytes = (hdr + slots * p.slot_bytes + 127) & ~127;
    const int smem = p.act_bytes + GEMV_WARPS * p.warp_bytes;
    static bool attr_set[64] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(gemv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_limit) != cudaSuccess)
            return -2;
        attr_set[dev] = true;
    }
    int64_t grid = p.ntasks < L.num_sms ? p.ntasks : L.num_sms;
    if (grid < 1) grid = 1;
    gemv_kernel<T><<<(unsigned)grid, GEMV_WARPS * 32, smem, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_gemv(uint32_t wtype, const GemvLaunch &L, cudaStream_t st) {
    switch (wtype) {
        case T_Q4_K: return launch_gemv_t<T_Q4_K>(L, st);
        case T_Q5_K: return launch_gemv_t<T_Q5_K>(L, st);
        case T_Q6_K: return launch_gemv_t<T_Q6_K>(L, st);
        case T_Q3_K: return launch_gemv_t<T_Q3_K>(L, st);
        case T_Q2_K: return launch_gemv_t<T_Q2_K>(L, st);
        case T_Q4_0: return launch_gemv_t<T_Q4_0>(L, st);
        case T_Q5_0: return launch_gemv_t<T_Q5_0>(L, st);
        case T_Q8_0: return launch_gemv_t<T_Q8_0>(L, st);
        default: return -3;
    }
}

}  // namespace sicu
