// Persistent streaming matvec driver (see gemv.cuh for the design notes).
#include <map>
#include <mutex>

#include "allreduce.cuh"
#include "gemv.cuh"
#include "quantize.cuh"
#include "launch.h"

namespace sicu {

namespace {

// Producer state of one warp: its next item (task t over all matrices, the
// task's matrix, chunk) and the item's geometry, advanced incrementally.
struct Producer {
    int task, mat, chunk, row0, rows, u0, cu;
    const uint8_t *w, *mend;   // current matrix and its end
    const uint8_t *src;        // first byte of the item
    uint32_t tailmask;         // slots that received lane-written tail bytes

    template <uint32_t T>
    __device__ void locate(const GemvParams &p) {   // task/chunk -> geometry
        while (mat + 1 < p.nmat && task >= p.task0[mat + 1]) ++mat;
        w = p.w[mat];
        mend = w + (int64_t)p.n_out[mat] * p.row_bytes;
        row0 = (task - p.task0[mat]) * p.rows_per_task;
        const int left = p.n_out[mat] - row0;
        rows = left < p.rows_per_task ? left : p.rows_per_task;
        u0 = chunk * p.cu;
        cu = min(p.cu, p.nu - u0);
        src = w + (int64_t)row0 * p.row_bytes + (int64_t)u0 * Fmt<T>::unit_bytes;
    }
    template <uint32_t T>
    __device__ void next(const GemvParams &p, int step) {
        if (++chunk < p.nchunks) {
            src += (int64_t)cu * Fmt<T>::unit_bytes;
            u0 += cu;
            cu = min(p.cu, p.nu - u0);
        } else {
            chunk = 0;
            task += step;
            locate<T>(p);
        }
    }
    // Fill ring slot s with the current item: a 16-byte aligned bulk copy
    // plus, at the very end of a matrix, up to 15 tail bytes written by this
    // lane; publish the geometry next to the slot.
    template <uint32_t T>
    __device__ void produce(const GemvParams &p, int s, uint8_t *slot, int4 *info, uint32_t full, uint64_t policy) {
        int64_t len;
        if (p.nchunks == 1) {
            len = (int64_t)rows * p.row_bytes;
        } else {
            const int64_t rest = p.row_bytes - (int64_t)u0 * Fmt<T>::unit_bytes;
            const int64_t want = (int64_t)cu * Fmt<T>::unit_bytes;
            len = want < rest ? want : rest;
        }
        const uintptr_t a = reinterpret_cast<uintptr_t>(src);
        const uint8_t *al = reinterpret_cast<const uint8_t *>(a & ~uintptr_t(15));
        const int head = (int)(a & 15);
        int64_t bulk = (head + len + 15) & ~int64_t(15);
        if (al + bulk > mend) bulk = (int64_t)(mend - al) & ~int64_t(15);
        const int tail = (int)(head + len - bulk);
        // generic writes to this slot before an async-proxy write to it need a proxy fence
        if (tailmask & (1u << s)) {
            fence_proxy_async();
            tailmask &= ~(1u << s);
        }
        if (tail > 0) {
            for (int i = 0; i < tail; ++i) slot[bulk + i] = (uint8_t)ldg_u8(al + bulk + i);
            tailmask |= 1u << s;
        }
        info[0] = make_int4(row0, rows | (head << 16), u0, cu);
        info[1] = make_int4(mat, 0, 0, 0);
        mbar_expect_tx(full, (uint32_t)bulk);   // also the phase's one arrival
        if (bulk > 0) bulk_g2s_hint(smem_addr(slot), al, (uint32_t)bulk, full, policy);
    }
};

// a += src[0]; a += src[1]; ... in order, each a separate IEEE rounding.
// src is 16-byte aligned.
__device__ __forceinline__ float chain_add(float a, const float *src, int n) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    const int n4 = n >> 2;
#pragma unroll 4
    for (int g = 0; g < n4; ++g) {
        const float4 v = s4[g];
        a = __fadd_rn(a, v.x); a = __fadd_rn(a, v.y); a = __fadd_rn(a, v.z); a = __fadd_rn(a, v.w);
    }
    for (int u = n4 << 2; u < n; ++u) a = __fadd_rn(a, src[u]);
    return a;
}

// Output epilogue of the STEPS kernels: the bias add the reference runs after
// the Q, K and V products (src/engine.c:320-334: y + b, one f32 rounding),
// then silu for a gate product with the SwiGLU epilogue.
__device__ __forceinline__ float epilogue(const GemvParams &p, int mat, int64_t row, float v) {
    if (p.bias[mat]) v = __fadd_rn(v, p.bias[mat][row]);
    if ((p.epi_silu >> mat) & 1) v = silu_call(v);
    return v;
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Every warp streams and decodes its own tasks: warp w of a CTA owns the
// CTA's tasks w, w+W, ... (all chunks of a task, so a row's float chains stay
// in one warp) and a private ring of nslots shared-memory slots. Lane 0 keeps
// the ring full with bulk copies; a slot's geometry is published next to it,
// so the consuming side does no address arithmetic of its own.
// AR: a row-split product whose partial outputs are all-reduced over the
// tensor-parallel group inside the kernel. STEPS: the launch has an
// activation step or an output epilogue (p.pro, p.epi_silu). Both are
// separate instantiations, so the plain matvec carries none of their code
// (kernels that follow one another in a decode step measured ~1.5 us slower
// per launch with the step code inlined, and ~2 % slower per step with it out
// of line but still present).
template <uint32_t T, bool AR, bool STEPS>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 2) gemv_kernel(const GemvParams p) {
    using F = Fmt<T>;
    constexpr int CH = F::chains;
    const int W = (int)(blockDim.x >> 5);   // warps per CTA (<= GEMV_WARPS)
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.nslots;

    const ActView av{smem, p.nu};
    uint8_t *wreg = smem + p.act_bytes + (size_t)warp * p.warp_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(wreg);          // [S]
    int4 *info = reinterpret_cast<int4 *>(wreg + 64);              // [S][2]
    float *terms = reinterpret_cast<float *>(wreg + 192);          // TERM_FLOATS
    float *fin = terms + TERM_FLOATS;                              // 64 chain results
    uint8_t *slots = wreg + 192 + CONS_BYTES;

    const int t0 = (int)((int64_t)blockIdx.x * p.ntasks / gridDim.x);
    const int t1 = (int)((int64_t)(blockIdx.x + 1) * p.ntasks / gridDim.x);
    const int ntask = t1 - t0;
    const int items = warp < ntask ? ((ntask - warp + W - 1) / W) * p.nchunks : 0;
    grid_dep_launch();

    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(smem_addr(&full[i]), 1);
        fence_mbar_init();
    }
    __syncwarp();
    // producer: item m is task t0 + warp + (m / nchunks) * W, chunk m % nchunks
    Producer pc;
    pc.task = t0 + warp;
    pc.mat = 0;
    pc.chunk = 0;
    pc.tailmask = 0;
    int pm = 0;
    uint64_t policy = 0;
    if (lane == 0 && items > 0) {
        pc.locate<T>(p);
        // weights never depend on earlier kernels: start streaming right away
        policy = policy_evict_first();
        for (; pm < items && pm < S && pm < GEMV_PRE_WAIT_SLOTS; ++pm) {
            pc.produce<T>(p, pm, slots + (size_t)pm * p.slot_bytes, &info[2 * pm], smem_addr(&full[pm]), policy);
            pc.next<T>(p, W);
        }
    }

    // the activation may be produced by the previous kernel in the stream;
    // each CTA of the cluster builds 1/nrank of the records for every member
    grid_dep_wait();
    const uint32_t rank = cluster_rank(), nrank = cluster_size();
    // row-split product with a fused all-reduce: the delivery count and the
    // group's state, read once per CTA, live in the 16 bytes after the
    // activation records ([0] count e, [1] intact) and are re-read where used
    // (the loop below is at the launch bound's register limit)
    volatile unsigned *const ar_st = reinterpret_cast<volatile unsigned *>(smem + ActView::bytes(p.nu));
    ArState as{};
    if constexpr (AR) {
        if (threadIdx.x == 0) as = ar_load_state(p.ar);   // used after the quantizer
    }
    if (STEPS && p.pro.kind != PRO_NONE)
        quantize_steps<F::act>(av, p.xf, p.n_in, rank, nrank, p.pro, smem + ActView::bytes(p.nu) + 16);
    else if (p.xf) quantize_into_act<F::act>(av, p.xf, p.n_in, rank, nrank);
    else prep_activation<F::act>(av, p.xq, p.n_in, rank, nrank);
    if constexpr (AR) {
        if (threadIdx.x == 0) {
            if (as.broken) atomicOr(p.status, STATUS_AR_TIMEOUT);
            ar_st[0] = as.e;
            ar_st[1] = as.broken ? 0u : 1u;
            if (!as.broken) ar_arrive(p.ar, as.e);
        }
    }
    cluster_sync();   // also publishes ar_st to the CTA
    // the rest of the ring, held back so the activation's loads do not queue
    // behind the weight stream
    if (lane == 0 && items > 0) {
        for (; pm < items && pm < S; ++pm) {
            pc.produce<T>(p, pm, slots + (size_t)pm * p.slot_bytes, &info[2 * pm], smem_addr(&full[pm]), policy);
            pc.next<T>(p, W);
        }
    }

    const int r_l = p.nchunks == 1 ? lane / p.cu : 0;
    const int u_l = p.nchunks == 1 ? lane - r_l * p.cu : lane;
    // chain strides in floats: a multiple of 4 that is an odd number of
    // 16-byte units, so the chain lanes' vector loads hit distinct banks
    int cup = (p.cu + 3) & ~3;
    if (((cup >> 2) & 1) == 0) cup += 4;   // K formats: [chain][row] stride
    const int rstride = 8 * p.cu + 4;      // classic formats: row stride
    float acc[2] = {0.f, 0.f};
    int s = 0, chunk = 0;
    uint32_t parity = 0;
    for (int m = 0; m < items; ++m) {
        const bool landed = mbar_wait(smem_addr(&full[s]), parity);
        if (!__all_sync(0xffffffffu, landed)) {
            if (lane == 0) atomicOr(p.status, STATUS_WAIT_TIMEOUT);
            // let the copies still in flight land before the CTA's memory goes away
            for (int k = m; k < items && k < m + S; ++k)
                (void)mbar_wait(smem_addr(&full[k % S]), (uint32_t)((k / S) & 1), 100000000ull);
            break;
        }
        const int4 g = info[2 * s];
        const int mat = info[2 * s + 1].x;
        const int rows = g.y & 0xffff, u0 = g.z, cu = g.w;
        uint8_t *slot = slots + (size_t)s * p.slot_bytes;
        const uint8_t *data = slot + (g.y >> 16);

        // ---- phase 1: each lane decodes its unit ----
        if (r_l < rows && u_l < cu) {
            const int ug = u0 + u_l;
            const uint8_t *wb = data + (int64_t)r_l * (p.nchunks == 1 ? p.row_bytes : 0) + u_l * F::unit_bytes;
            const uint8_t *rec = av.rec(ug);
            if constexpr (F::kind == 3) {
                const int nb = min(8, p.n_in / 32 - ug * 8);
                float t[8];
                unit_classic<T>(wb, nb, rec, t);
                float *dst = terms + r_l * rstride + u_l * 8;
#pragma unroll
                for (int b = 0; b < 8; ++b) if (b < nb) dst[b] = t[b];
            } else {
                float t[MAX_CHAINS];
                if constexpr (T == T_Q4_K) unit_q45k<false>(wb, rec, t);
                else if constexpr (T == T_Q5_K) unit_q45k<true>(wb, rec, t);
                else if constexpr (T == T_Q6_K) unit_q36k<false>(wb, rec, t);
                else if constexpr (T == T_Q3_K) unit_q36k<true>(wb, rec, t);
                else unit_q2k(wb, rec, t);
#pragma unroll
                for (int ch = 0; ch < CH; ++ch) terms[(ch * p.rows_per_task + r_l) * cup + u_l] = t[ch];
            }
        }
        __syncwarp();
        // the slot is consumed: refill it with item m + S
        if (lane == 0 && pm < items) {
            pc.produce<T>(p, s, slot, &info[2 * s], smem_addr(&full[s]), policy);
            pc.next<T>(p, W);
            ++pm;
        }

        // ---- phase 2: ordered float chains, one lane per (row, chain) ----
        const int pairs = rows * CH;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int q = lane + 32 * h;
            if (q < pairs) {
                const int r = q / CH, ch = q - r * CH;
                if constexpr (F::kind == 3) {
                    const int nb = min(cu * 8, p.n_in / 32 - u0 * 8);
                    acc[h] = chain_add(acc[h], terms + r * rstride, nb);
                } else {
                    acc[h] = chain_add(acc[h], terms + (ch * p.rows_per_task + r) * cup, cu);
                }
            }
        }
        if (++chunk == p.nchunks) {
            chunk = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int q = lane + 32 * h;
                if (q < pairs) fin[q] = acc[h];
                acc[h] = 0.f;
            }
            __syncwarp();
            if (lane < rows) {
                float r;
                if constexpr (F::kind == 0) {
                    r = fin[lane * CH + 8];
#pragma unroll
                    for (int l = 0; l < 8; ++l) r = __fadd_rn(r, fin[lane * CH + l]);
                } else if constexpr (F::kind == 1) {
                    r = 0.0f;
#pragma unroll
                    for (int l = 0; l < 8; ++l) r = __fadd_rn(r, fin[lane * CH + l]);
                } else {
                    r = fin[lane];
                }
                // row-split product: the partial goes to every rank; y gets
                // the sum after the loop
                if (AR && ar_st[1]) ar_send(p.ar, ar_st[0], g.x + lane, r);
                else if (STEPS) p.y[mat][g.x + lane] = epilogue(p, mat, g.x + lane, r);
                else p.y[mat][g.x + lane] = r;
            }
        }
        __syncwarp();
        if (++s == S) { s = 0; parity ^= 1u; }
    }
    if constexpr (AR) {
        // the sums of this warp's rows: by now the other ranks' CTAs that
        // compute the same rows have usually sent their parts
        if (ar_st[1]) {
            const unsigned e = ar_st[0];
            bool live = true;
            for (int t = t0 + warp; t < t1; t += W) {
                const int64_t row = (int64_t)t * p.rows_per_task + lane;
                if (lane < p.rows_per_task && row < p.n_out[0]) {
                    const float v = ar_sum(p.ar, e, row, p.status, live);
                    p.y[0][row] = STEPS ? epilogue(p, 0, row, v) : v;
                }
            }
        }
    }
}

// ---- flattened items ------------------------------------------------------------
// When a row's unit count nu does not divide 32, whole-row items leave lanes
// idle (nu = 20: 20 of 32). Here a task is R consecutive rows of one matrix
// and its R x nu units are streamed as items of up to 32 consecutive units --
// one contiguous bulk copy, rows being back to back -- so every lane decodes a
// unit. A row whose units straddle two items continues its float chains in
// the next item of the same warp, in order (the partial chains wait in shared
// memory), so every output is bit-identical to the whole-row kernel's.

// a += src[0]; a += src[1]; ... in order; src 4-byte aligned
__device__ __forceinline__ float chain_add_any(float a, const float *src, int n) {
    int i = 0;
    const int head = min(n, (int)((4u - ((uint32_t)(reinterpret_cast<uintptr_t>(src) >> 2) & 3u)) & 3u));
    for (; i < head; ++i) a = __fadd_rn(a, src[i]);
    const float4 *s4 = reinterpret_cast<const float4 *>(src + i);
    const int n4 = (n - i) >> 2;
#pragma unroll 2
    for (int g = 0; g < n4; ++g) {
        const float4 v = s4[g];
        a = __fadd_rn(a, v.x); a = __fadd_rn(a, v.y); a = __fadd_rn(a, v.z); a = __fadd_rn(a, v.w);
    }
    for (i += n4 << 2; i < n; ++i) a = __fadd_rn(a, src[i]);
    return a;
}

// Item cursor of one warp: task (over all matrices), item k of the task.
struct FlatCursor {
    int task, k, mat, row0, units;
    __device__ void locate(const GemvParams &p) {
        while (mat + 1 < p.nmat && task >= p.task0[mat + 1]) ++mat;
        row0 = (task - p.task0[mat]) * p.rows_per_task;
        units = min(p.rows_per_task, p.n_out[mat] - row0) * p.nu;
    }
    __device__ void next(const GemvParams &p, int step) {
        if (32 * (k + 1) < units) {
            ++k;
        } else {
            k = 0;
            task += step;
            if (task < p.ntasks) locate(p);
        }
    }
};

constexpr int FLAT_TS = 36;    // terms row stride (floats): an odd number of 16-byte units

template <uint32_t T, bool STEPS>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 2) gemv_flat_kernel(const GemvParams p) {
    using F = Fmt<T>;
    constexpr int CH = F::chains;
    const int W = (int)(blockDim.x >> 5);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.nslots, nu = p.nu;

    const ActView av{smem, nu};
    uint8_t *wreg = smem + p.act_bytes + (size_t)warp * p.warp_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(wreg);          // [S]
    int4 *info = reinterpret_cast<int4 *>(wreg + 64);              // [S][2]
    float *terms = reinterpret_cast<float *>(wreg + 192);          // [CH][FLAT_TS]
    float *carry = terms + 448;                                    // [2][CH] chains continuing
    float *fin = terms + TERM_FLOATS;                              // 64 chain results
    uint8_t *slots = wreg + 192 + CONS_BYTES;

    const int t0 = (int)((int64_t)blockIdx.x * p.ntasks / gridDim.x);
    const int t1 = (int)((int64_t)(blockIdx.x + 1) * p.ntasks / gridDim.x);
    grid_dep_launch();

    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(smem_addr(&full[i]), 1);
        fence_mbar_init();
    }
    __syncwarp();
    // producer (lane 0): its own cursor, S items ahead of the consumer
    FlatCursor pc{t0 + warp, 0, 0, 0, 0};
    uint32_t tailmask = 0;
    uint64_t policy = 0;
    auto produce = [&](int s) {
        const uint8_t *w = p.w[pc.mat];
        const uint8_t *mend = w + (int64_t)p.n_out[pc.mat] * p.row_bytes;
        const int fs = 32 * pc.k, c = min(32, pc.units - fs);
        const uint8_t *src = w + (int64_t)pc.row0 * p.row_bytes + (int64_t)fs * F::unit_bytes;
        const int64_t len = (int64_t)c * F::unit_bytes;
        uint8_t *slot = slots + (size_t)s * p.slot_bytes;
        const uintptr_t a = reinterpret_cast<uintptr_t>(src);
        const uint8_t *al = reinterpret_cast<const uint8_t *>(a & ~uintptr_t(15));
        const int head = (int)(a & 15);
        int64_t bulk = (head + len + 15) & ~int64_t(15);
        if (al + bulk > mend) bulk = (int64_t)(mend - al) & ~int64_t(15);
        const int tail = (int)(head + len - bulk);
        if (tailmask & (1u << s)) {
            fence_proxy_async();
            tailmask &= ~(1u << s);
        }
        if (tail > 0) {
            for (int i = 0; i < tail; ++i) slot[bulk + i] = (uint8_t)ldg_u8(al + bulk + i);
            tailmask |= 1u << s;
        }
        info[2 * s] = make_int4(pc.row0, fs | (head << 16), c, pc.units);
        info[2 * s + 1] = make_int4(pc.mat, 0, 0, 0);
        const uint32_t bar = smem_addr(&full[s]);
        mbar_expect_tx(bar, (uint32_t)bulk);
        if (bulk > 0) bulk_g2s_hint(smem_addr(slot), al, (uint32_t)bulk, bar, policy);
    };
    int pi = 0;   // ring slots filled before the activation phase
    if (lane == 0 && pc.task < t1) {
        pc.locate(p);
        policy = policy_evict_first();
        for (; pi < S && pi < GEMV_PRE_WAIT_SLOTS && pc.task < t1; ++pi) {
            produce(pi);
            pc.next(p, W);
        }
    }

    grid_dep_wait();
    const uint32_t rank = cluster_rank(), nrank = cluster_size();
    if (STEPS && p.pro.kind != PRO_NONE)
        quantize_steps<F::act>(av, p.xf, p.n_in, rank, nrank, p.pro, smem + ActView::bytes(p.nu) + 16);
    else if (p.xf) quantize_into_act<F::act>(av, p.xf, p.n_in, rank, nrank);
    else prep_activation<F::act>(av, p.xq, p.n_in, rank, nrank);
    cluster_sync();
    if (lane == 0) {
        for (; pi < S && pc.task < t1; ++pi) {
            produce(pi);
            pc.next(p, W);
        }
    }

    int s = 0, cpar = 0;
    uint32_t parity = 0;
    bool ok = true;
    for (int task = t0 + warp; task < t1 && ok; task += W) {
        for (int k = 0;; ++k) {
            const bool landed = mbar_wait(smem_addr(&full[s]), parity);
            if (!__all_sync(0xffffffffu, landed)) {
                if (lane == 0) atomicOr(p.status, STATUS_WAIT_TIMEOUT);
                // let the copies still in flight land before the CTA's memory goes away
                for (int j = 0; j < S; ++j) {
                    const int sj = (s + j) % S;
                    (void)mbar_wait(smem_addr(&full[sj]), parity ^ (uint32_t)(sj < s), 100000000ull);
                }
                ok = false;
                break;
            }
            const int4 g = info[2 * s];
            const int mat = info[2 * s + 1].x;
            const int row0 = g.x, fs = g.y & 0xffff, c = g.z, units = g.w;
            const uint8_t *data = slots + (size_t)s * p.slot_bytes + (g.y >> 16);

            // ---- phase 1: lane l decodes unit fs + l of the task ----
            const int r_first = fs / nu, r_last = (fs + c - 1) / nu;
            if (lane < c) {
                int ug = fs - r_first * nu + lane;   // unit within its row
                while (ug >= nu) ug -= nu;
                float t[MAX_CHAINS];
                const uint8_t *wb = data + lane * F::unit_bytes;
                const uint8_t *rec = av.rec(ug);
                if constexpr (T == T_Q4_K) unit_q45k<false>(wb, rec, t);
                else if constexpr (T == T_Q5_K) unit_q45k<true>(wb, rec, t);
                else if constexpr (T == T_Q6_K) unit_q36k<false>(wb, rec, t);
                else if constexpr (T == T_Q3_K) unit_q36k<true>(wb, rec, t);
                else unit_q2k(wb, rec, t);
#pragma unroll
                for (int ch = 0; ch < CH; ++ch) terms[ch * FLAT_TS + lane] = t[ch];
            }
            __syncwarp();
            if (lane == 0 && pc.task < t1) {
                produce(s);
                pc.next(p, W);
            }

            // ---- phase 2: the rows' chains over this item's units, in order ----
            const int pairs = (r_last - r_first + 1) * CH;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int q = lane + 32 * h;
                if (q < pairs) {
                    const int kp = q / CH, ch = q - kp * CH;
                    const int r = r_first + kp;
                    const int b0 = r * nu, b1 = b0 + nu;
                    const int p0 = max(b0, fs) - fs, p1 = min(b1, fs + c) - fs;
                    float a = b0 < fs ? carry[cpar * CH + ch] : 0.0f;
                    a = chain_add_any(a, terms + ch * FLAT_TS + p0, p1 - p0);
                    if (b1 <= fs + c) fin[kp * CH + ch] = a;
                    else carry[(cpar ^ 1) * CH + ch] = a;
                }
            }
            cpar ^= 1;
            __syncwarp();
            // ---- rows completed in this item ----
            const int ncomp = (r_last - r_first + 1) - (((r_last + 1) * nu > fs + c) ? 1 : 0);
            if (lane < ncomp) {
                float r;
                if constexpr (F::kind == 0) {
                    r = fin[lane * CH + 8];
#pragma unroll
                    for (int l = 0; l < 8; ++l) r = __fadd_rn(r, fin[lane * CH + l]);
                } else if constexpr (F::kind == 1) {
                    r = 0.0f;
#pragma unroll
                    for (int l = 0; l < 8; ++l) r = __fadd_rn(r, fin[lane * CH + l]);
                } else {
                    r = fin[lane];
                }
                p.y[mat][row0 + r_first + lane] = STEPS ? epilogue(p, mat, row0 + r_first + lane, r) : r;
            }
            __syncwarp();
            if (++s == S) { s = 0; parity ^= 1u; }
            if (32 * (k + 1) >= units) break;
        }
    }
}

}  // namespace

// ---- host side ------------------------------------------------------------------

template <uint32_t T>
static int launch_gemv_t(const GemvLaunch &L, cudaStream_t st) {
    using F = Fmt<T>;
    GemvParams p{};
    p.nmat = L.nmat;
    p.xq = static_cast<const uint8_t *>(L.xq);
    p.xf = L.xf;
    p.n_in = L.n_in;
    p.status = L.status;
    p.ar = L.ar;
    const int nblk = (F::kind == 3) ? L.n_in / 32 : L.n_in / 256;
    p.row_bytes = (int64_t)nblk * (F::kind == 3 ? F::unit_bytes / 8 : F::unit_bytes);
    p.nu = (F::kind == 3) ? (nblk + 7) / 8 : nblk;
    // rows x units-per-chunk <= 32 (one unit per lane); rows x chains <= 64.
    // Whole rows when they fit (R = 32 / nu); longer rows stream in balanced
    // chunks of one row each, one contiguous bulk copy per item. (Items of
    // several rows' chunks, one bulk copy per row piece, fill the lanes left
    // idle when nu does not divide 32, but measured slower.)
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
    // flattened items (gemv_flat_kernel) when rows leave lanes idle and the
    // launch has enough rows that fewer, fuller items per warp win: compare
    // the items the busiest warp processes (grid of 2 CTAs x 8 warps per SM)
    const bool ar = L.ar.n > 0;
    bool flat = false;
    // (only when whole-row items leave a quarter of the lanes idle or more:
    // at 87.5 % lane use, e.g. 56 units in chunks of 28, the whole-row kernel's
    // aligned register-carried chains measured faster)
    const double row_lanes = p.nchunks == 1 ? (double)(p.rows_per_task * p.nu) / 32.0
                                            : (double)p.nu / (32.0 * p.nchunks);
    if (F::kind != 3 && !ar && p.nu >= 6 && row_lanes < 0.8) {
        const int64_t G = 2LL * L.num_sms;
        auto busiest = [&](int rows, int64_t items_per_task) {
            int64_t tasks = 0;
            for (int i = 0; i < L.nmat; ++i) tasks += (L.n_outm[i] + rows - 1) / rows;
            const int64_t per_cta = (tasks + G - 1) / G;
            return (per_cta + GEMV_WARPS - 1) / GEMV_WARPS * items_per_task;
        };
        int64_t best = busiest(p.rows_per_task, p.nchunks);
        for (int r = 1; r <= 8; ++r) {
            const int64_t v = busiest(r, (r * p.nu + 31) / 32);
            if (v < best) {
                best = v;
                flat = true;
                p.rows_per_task = r;
            }
        }
        if (flat) {
            p.nchunks = 1;
            p.cu = 32;
        }
    }
    int64_t tasks = 0;
    for (int i = 0; i < L.nmat; ++i) {
        p.w[i] = static_cast<const uint8_t *>(L.wm[i]);
        p.y[i] = L.ym[i];
        p.n_out[i] = (int)L.n_outm[i];
        p.task0[i] = (int)tasks;
        tasks += (L.n_outm[i] + p.rows_per_task - 1) / p.rows_per_task;
    }
    p.task0[L.nmat] = (int)tasks;
    p.ntasks = tasks;
    if (tasks == 0) return 0;
    const int64_t item_max = flat ? 32LL * F::unit_bytes
                                  : (p.nchunks == 1) ? p.rows_per_task * p.row_bytes : (int64_t)p.cu * F::unit_bytes;
    p.slot_bytes = (int)((item_max + 32 + 127) & ~int64_t(127));
    // after the records: the all-reduce state (16 bytes), then the norm's
    // reduction scratch
    p.pro = L.pro;
    p.epi_silu = L.epi_silu;
    bool any_bias = false;
    for (int i = 0; i < L.nmat; ++i) {
        p.bias[i] = L.bias[i];
        any_bias = any_bias || L.bias[i] != nullptr;
    }
    const bool rms = L.pro.kind == PRO_RMS_NORM;
    p.act_bytes = (ActView::bytes(p.nu) + (ar || rms ? 16 : 0) + (rms ? RMS_SCRATCH : 0) + 127) & ~127;
    // two CTAs per SM when each warp keeps >= 2 ring slots, with 8 warps per
    // CTA or, for large slots, down to 6 (12 warps per SM still hide more
    // latency than one CTA of 8); else one CTA of 8 warps with up to 4 slots
    int ctas = 2, slots = 0, warps = GEMV_WARPS;
    const int hdr = 192 + CONS_BYTES;
    for (bool found = false; ctas >= 1 && !found; --ctas) {
        const int per_cta = (ctas == 2) ? L.smem_per_sm / 2 - L.smem_reserved : L.smem_limit;
        for (warps = GEMV_WARPS; warps >= (ctas == 2 ? 6 : GEMV_WARPS); --warps) {
            // a 128-aligned budget per warp, so rounding the region up stays inside it
            const int per_warp = ((per_cta - p.act_bytes) / warps & ~127) - hdr;
            slots = per_warp > 0 ? per_warp / p.slot_bytes : 0;
            if (slots > 4) slots = 4;
            if (slots >= 2) { found = true; break; }
        }
        if (found) break;
    }
    if (slots < 2) return -1;
    p.nslots = slots;
    p.warp_bytes = (hdr + slots * p.slot_bytes + 127) & ~127;
    const int smem = p.act_bytes + warps * p.warp_bytes;
    const bool steps = L.pro.kind != PRO_NONE || L.epi_silu != 0 || any_bias;
    auto kern = ar ? (steps ? gemv_kernel<T, true, true> : gemv_kernel<T, true, false>)
                   : (steps ? gemv_kernel<T, false, true> : gemv_kernel<T, false, false>);
    if constexpr (F::kind != 3) {
        if (flat) kern = steps ? gemv_flat_kernel<T, true> : gemv_flat_kernel<T, false>;
    }
    const int variant = (flat ? 2 : ar ? 1 : 0) + (steps ? 3 : 0);
    static bool attr_set[64][6] = {};
    const int dev = L.device & 63;
    if (!attr_set[dev][variant]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_limit) != cudaSuccess)
            return -2;
        // every kernel of the library asks for the same (largest) shared-memory
        // carveout, so consecutive launches of different kernels never wait
        // for an SM to reconfigure its L1 / shared-memory split
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        attr_set[dev][variant] = true;
    }
    // thread-block cluster size: 2 when pairs still keep (almost) every CTA
    // slot of the launch co-resident, else 1
    const int target = ctas * L.num_sms;
    int csize = 1, capacity = target;
    {
        static std::mutex mu;
        static std::map<std::pair<int, int>, std::pair<int, int>> cache;   // (device x variant, smem x warps) -> (C, capacity)
        std::lock_guard<std::mutex> lk(mu);
        const auto key = std::make_pair(dev * 8 + variant, smem * 16 + warps);
        auto hit = cache.find(key);
        if (hit == cache.end()) {
            int best_c = 1, best_cap = target;
            // pairs of CTAs: larger clusters share the activation work further
            // but cost launch latency (in a graph-captured decode step,
            // clusters of 8 took 35 % longer per token than pairs on small
            // matrices and were no faster on large ones)
            for (int c = 2; c >= 2; c /= 2) {
                cudaLaunchConfig_t q{};
                q.gridDim = dim3((unsigned)(target / c * c));
                q.blockDim = dim3(warps * 32);
                q.dynamicSmemBytes = (size_t)smem;
                cudaLaunchAttribute ca[1];
                ca[0].id = cudaLaunchAttributeClusterDimension;
                ca[0].val.clusterDim.x = c;
                ca[0].val.clusterDim.y = 1;
                ca[0].val.clusterDim.z = 1;
                q.attrs = ca;
                q.numAttrs = 1;
                int n = 0;
                if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess) {
                    cudaGetLastError();
                    continue;
                }
                if (n * c >= target - target / 16) {
                    best_c = c;
                    best_cap = n * c < target ? n * c : target;
                    break;
                }
            }
            hit = cache.emplace(key, std::make_pair(best_c, best_cap)).first;
        }
        csize = hit->second.first;
        capacity = hit->second.second;
    }
    int64_t grid = capacity;
    if (p.ntasks < grid) grid = p.ntasks;
    if (grid < csize) csize = 1;
    grid = grid / csize * csize;
    if (grid < 1) grid = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(warps * 32);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.overlap ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = csize;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return -2;
    return 0;
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
