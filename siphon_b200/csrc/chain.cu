// A chain of dependent matvecs in one persistent launch: a decode step's
// products (Wq/Wk/Wv, Wo, W_gate/W_up, W_down per layer, then the output head)
// run as stages of one kernel instead of one launch each. Between stages
// every CTA meets at a bounded grid barrier, so a stage reads what the
// previous one wrote; the weights of the next stages keep streaming into the
// warps' rings across the barrier, because weights never depend on a stage's
// output. A stage computes exactly what the whole-row matvec kernel computes
// (same task geometry, same unit decoders, same float chains), so its outputs
// are bit-identical. A row-split stage runs the all-reduce of the tensor-
// parallel group inside, as sicu_gemv_ar does.
#include <map>
#include <mutex>

#include "allreduce.cuh"
#include "gemv.cuh"
#include "quantize.cuh"
#include "launch.h"

namespace sicu {
namespace {

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// All CTAs of the grid (co-resident by construction of the grid size):
// every CTA's writes before the call are visible to every CTA after it.
// Bounded: after 2 s the CTA goes on and the status word says so.
__device__ __forceinline__ void grid_sync(unsigned *ctr, unsigned target, int *status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
        if (ld_acquire_gpu(ctr) < target) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_gpu(ctr) < target) {
                if (globaltimer_ns() - t0 > 2000000000ull) {
                    atomicOr(status, STATUS_WAIT_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

// The warp's items of stage s: tasks t0 + warp, t0 + warp + W, ... of this
// CTA's balanced range, every chunk of each.
__device__ __forceinline__ void stage_range(const ChainStage &cs, int warp, int W, int &t0, int &t1, int &items) {
    t0 = (int)((int64_t)blockIdx.x * cs.ntasks / gridDim.x);
    t1 = (int)((int64_t)(blockIdx.x + 1) * cs.ntasks / gridDim.x);
    const int n = t1 - t0;
    items = warp < n ? ((n - warp + W - 1) / W) * cs.nchunks : 0;
}

// Producer of one warp (lane 0): walks the items of every stage in order and
// keeps the ring full, across stage boundaries.
struct ChainProducer {
    int stage, left, task, mat, chunk, row0, rows, u0, cu;
    uint32_t tailmask;
    uint64_t policy;

    __device__ void locate(const ChainParams &p, const ChainStage &cs) {
        while (mat + 1 < cs.nmat && task >= cs.task0[mat + 1]) ++mat;
        row0 = (task - cs.task0[mat]) * cs.rows_per_task;
        const int lft = cs.n_out[mat] - row0;
        rows = lft < cs.rows_per_task ? lft : cs.rows_per_task;
        u0 = chunk * cs.cu;
        cu = min(cs.cu, cs.nu - u0);
    }
    // first item of the first stage at or after `s` in which the warp has items
    __device__ void enter(const ChainParams &p, int s, int warp, int W) {
        for (stage = s; stage < p.nstages; ++stage) {
            const ChainStage &cs = p.st[stage];
            int t0, t1;
            stage_range(cs, warp, W, t0, t1, left);
            if (left > 0) {
                task = t0 + warp;
                mat = 0;
                chunk = 0;
                locate(p, cs);
                return;
            }
        }
    }
    __device__ bool more(const ChainParams &p) const { return stage < p.nstages; }
    __device__ void next(const ChainParams &p, int warp, int W) {
        if (--left == 0) {
            enter(p, stage + 1, warp, W);
            return;
        }
        const ChainStage &cs = p.st[stage];
        if (++chunk < cs.nchunks) {
            u0 += cu;
            cu = min(cs.cu, cs.nu - u0);
        } else {
            chunk = 0;
            task += W;
            locate(p, cs);
        }
    }
    __device__ void produce(const ChainParams &p, int s, uint8_t *slot, int4 *info, uint32_t full) {
        const ChainStage &cs = p.st[stage];
        const uint8_t *w = cs.w[mat];
        const uint8_t *mend = w + (int64_t)cs.n_out[mat] * cs.row_bytes;
        const uint8_t *src = w + (int64_t)row0 * cs.row_bytes + (int64_t)u0 * cs.unit_bytes;
        const int64_t len = cs.nchunks == 1 ? (int64_t)rows * cs.row_bytes
                                            : min((int64_t)cu * cs.unit_bytes, cs.row_bytes - (int64_t)u0 * cs.unit_bytes);
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
        info[0] = make_int4(row0, rows | (head << 16), u0, cu);
        info[1] = make_int4(mat, stage, 0, 0);
        mbar_expect_tx(full, (uint32_t)bulk);
        if (bulk > 0) bulk_g2s_hint(smem_addr(slot), al, (uint32_t)bulk, full, policy);
    }
};

// warp region: [0,64) ring barriers, [64,192) slot geometry, [192,256) the
// producer's state (lane 0 only; kept in shared memory, not registers),
// then terms, chain results and the ring slots
constexpr int CHAIN_HDR = 256 + CONS_BYTES;

struct Ring {
    uint64_t *full;
    int4 *info;
    float *terms, *fin;
    uint8_t *slots;
    int s;
    uint32_t parity;
    bool dead;   // a wait for the warp's own copies gave up: the warp computes nothing more
};

// The items of stage `si` for this warp (the whole-row kernel's loop body).
template <uint32_t T>
__device__ __forceinline__ void run_stage(const ChainParams &p, const ChainStage &cs, int si, const ActView av, Ring &rg,
                          ChainProducer *pc, int warp, int W, bool ar_live, unsigned ar_e) {
    using F = Fmt<T>;
    constexpr int CH = F::chains;
    const int lane = threadIdx.x & 31, S = p.nslots;
    int t0, t1, items;
    stage_range(cs, warp, W, t0, t1, items);
    const int r_l = cs.nchunks == 1 ? lane / cs.cu : 0;
    const int u_l = cs.nchunks == 1 ? lane - r_l * cs.cu : lane;
    int cup = (cs.cu + 3) & ~3;
    if (((cup >> 2) & 1) == 0) cup += 4;
    float acc[2] = {0.f, 0.f};
    int chunk = 0;
    for (int m = 0; m < items && !rg.dead; ++m) {
        const bool landed = mbar_wait(smem_addr(&rg.full[rg.s]), rg.parity);
        if (!__all_sync(0xffffffffu, landed)) {
            if (lane == 0) atomicOr(p.status, STATUS_WAIT_TIMEOUT);
            for (int j = 0; j < S; ++j) {
                const int sj = (rg.s + j) % S;
                (void)mbar_wait(smem_addr(&rg.full[sj]), rg.parity ^ (uint32_t)(sj < rg.s), 100000000ull);
            }
            rg.dead = true;
            break;
        }
        const int4 g = rg.info[2 * rg.s];
        const int mat = rg.info[2 * rg.s + 1].x;
        const int rows = g.y & 0xffff, u0 = g.z, cu = g.w;
        uint8_t *slot = rg.slots + (size_t)rg.s * p.slot_bytes;
        const uint8_t *data = slot + (g.y >> 16);

        if (r_l < rows && u_l < cu) {
            const int ug = u0 + u_l;
            const uint8_t *wb = data + (int64_t)r_l * (cs.nchunks == 1 ? cs.row_bytes : 0) + u_l * F::unit_bytes;
            float t[MAX_CHAINS];
            if constexpr (T == T_Q4_K) unit_q45k<false>(wb, av.rec(ug), t);
            else unit_q36k<false>(wb, av.rec(ug), t);
#pragma unroll
            for (int ch = 0; ch < CH; ++ch) rg.terms[(ch * cs.rows_per_task + r_l) * cup + u_l] = t[ch];
        }
        __syncwarp();
        if (lane == 0 && pc->more(p)) {
            pc->produce(p, rg.s, slot, &rg.info[2 * rg.s], smem_addr(&rg.full[rg.s]));
            pc->next(p, warp, W);
        }
        const int pairs = rows * CH;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int q = lane + 32 * h;
            if (q < pairs) {
                const int r = q / CH, ch = q - r * CH;
                const float *src = rg.terms + (ch * cs.rows_per_task + r) * cup;
                float a = acc[h];
                const float4 *s4 = reinterpret_cast<const float4 *>(src);
                const int n4 = cu >> 2;
                for (int k = 0; k < n4; ++k) {
                    const float4 v = s4[k];
                    a = __fadd_rn(a, v.x); a = __fadd_rn(a, v.y); a = __fadd_rn(a, v.z); a = __fadd_rn(a, v.w);
                }
                for (int u = n4 << 2; u < cu; ++u) a = __fadd_rn(a, src[u]);
                acc[h] = a;
            }
        }
        if (++chunk == cs.nchunks) {
            chunk = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int q = lane + 32 * h;
                if (q < pairs) rg.fin[q] = acc[h];
                acc[h] = 0.f;
            }
            __syncwarp();
            if (lane < rows) {
                float r;
                if constexpr (F::kind == 0) {
                    r = rg.fin[lane * CH + 8];
#pragma unroll
                    for (int l = 0; l < 8; ++l) r = __fadd_rn(r, rg.fin[lane * CH + l]);
                } else {
                    r = 0.0f;
#pragma unroll
                    for (int l = 0; l < 8; ++l) r = __fadd_rn(r, rg.fin[lane * CH + l]);
                }
                if (cs.ar && ar_live) ar_send(p.ar, ar_e, g.x + lane, r);
                else cs.y[mat][g.x + lane] = r;
            }
        }
        __syncwarp();
        if (++rg.s == S) { rg.s = 0; rg.parity ^= 1u; }
    }
    if (cs.ar && ar_live && !rg.dead) {
        // the sums of this warp's rows (one matrix): the other ranks' CTAs
        // computing the same rows have usually sent their parts by now
        bool live = true;
        for (int t = t0 + warp; t < t1; t += W) {
            const int64_t row = (int64_t)t * cs.rows_per_task + lane;
            if (lane < cs.rows_per_task && row < cs.n_out[0]) cs.y[0][row] = ar_sum(p.ar, ar_e, row, p.status, live);
        }
    }
}

__global__ void __launch_bounds__(GEMV_WARPS * 32, 2) gemv_chain_kernel(const __grid_constant__ ChainParams p) {
    const int W = (int)(blockDim.x >> 5);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.nslots;
    uint8_t *wreg = smem + p.act_bytes + (size_t)warp * p.warp_bytes;
    Ring rg;
    rg.full = reinterpret_cast<uint64_t *>(wreg);
    rg.info = reinterpret_cast<int4 *>(wreg + 64);
    rg.terms = reinterpret_cast<float *>(wreg + 256);
    rg.fin = rg.terms + TERM_FLOATS;
    rg.slots = wreg + CHAIN_HDR;
    rg.s = 0;
    rg.parity = 0;
    rg.dead = false;

    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(smem_addr(&rg.full[i]), 1);
        fence_mbar_init();
    }
    __syncwarp();
    ChainProducer *pc = reinterpret_cast<ChainProducer *>(wreg + 192);
    if (lane == 0) {
        pc->tailmask = 0;
        pc->policy = policy_evict_first();
        pc->enter(p, 0, warp, W);
        for (int i = 0; i < S && pc->more(p); ++i) {
            pc->produce(p, i, rg.slots + (size_t)i * p.slot_bytes, &rg.info[2 * i], smem_addr(&rg.full[i]));
            pc->next(p, warp, W);
        }
    }

    // the group's delivery count at the start of the chain; each CTA reads it
    // once, and the last CTA to have read it advances it by the chain's
    // all-reduce stages (no CTA reads it again in this launch)
    __shared__ unsigned ar_base, ar_intact;
    if (threadIdx.x == 0) {
        ar_intact = 0;
        if (p.ar.n) {
            const ArState st = ar_load_state(p.ar);
            ar_base = st.e;
            ar_intact = st.broken ? 0u : 1u;
            if (st.broken) {
                atomicOr(p.status, STATUS_AR_TIMEOUT);
            } else {
                const unsigned old = atomicAdd(p.ar.epoch + 2, 1u);
                if (old == gridDim.x - 1) {
                    st_vol(p.ar.epoch + 2, 0u);
                    st_vol(p.ar.epoch, st.e + (unsigned)p.n_ar);
                }
            }
        }
    }
    const uint32_t rank = cluster_rank(), nrank = cluster_size();
    for (int si = 0; si < p.nstages; ++si) {
        const ChainStage &cs = p.st[si];
        if (si > 0) grid_sync(p.barrier, (unsigned)si * gridDim.x, p.status);
        else __syncthreads();
        const ActView sv{smem, cs.nu};
        if (cs.type == T_Q4_K) quantize_into_act<Fmt<T_Q4_K>::act, true>(sv, cs.x, cs.n_in, rank, nrank);
        else quantize_into_act<Fmt<T_Q6_K>::act, true>(sv, cs.x, cs.n_in, rank, nrank);
        cluster_sync();
        const bool ar_live = ar_intact != 0;
        const unsigned ar_e = ar_base + (unsigned)cs.ar_index;
        if (cs.type == T_Q4_K) run_stage<T_Q4_K>(p, cs, si, sv, rg, pc, warp, W, ar_live, ar_e);
        else run_stage<T_Q6_K>(p, cs, si, sv, rg, pc, warp, W, ar_live, ar_e);
        // the next stage's grid barrier also keeps its quantizer from
        // overwriting records a cluster peer is still reading
    }
}

}  // namespace

// Geometry of one stage: the whole-row kernel's rules (launch_gemv_t).
static void stage_geometry(ChainStage &c) {
    const int chains = c.type == T_Q4_K ? Fmt<T_Q4_K>::chains : Fmt<T_Q6_K>::chains;
    c.unit_bytes = c.type == T_Q4_K ? Fmt<T_Q4_K>::unit_bytes : Fmt<T_Q6_K>::unit_bytes;
    c.nu = c.n_in / 256;
    c.row_bytes = (int64_t)c.nu * c.unit_bytes;
    if (c.nu <= 32) {
        c.nchunks = 1;
        c.cu = c.nu;
        c.rows_per_task = 32 / c.nu;
        if (c.rows_per_task > 64 / chains) c.rows_per_task = 64 / chains;
    } else {
        c.nchunks = (c.nu + 31) / 32;
        c.cu = (c.nu + c.nchunks - 1) / c.nchunks;
        c.rows_per_task = 1;
    }
    int64_t tasks = 0;
    for (int i = 0; i < c.nmat; ++i) {
        c.task0[i] = (int)tasks;
        tasks += (c.n_out[i] + c.rows_per_task - 1) / c.rows_per_task;
    }
    c.task0[c.nmat] = (int)tasks;
    c.ntasks = (int)tasks;
}

int chain_prepare(ChainStage *st, int n, ChainParams &p, ChainLaunch &L) {
    int64_t item_max = 0, act_max = 0;
    int max_nu = 0, n_ar = 0;
    for (int i = 0; i < n; ++i) {
        stage_geometry(st[i]);
        const int64_t im = st[i].nchunks == 1 ? st[i].rows_per_task * st[i].row_bytes : (int64_t)st[i].cu * st[i].unit_bytes;
        item_max = im > item_max ? im : item_max;
        max_nu = st[i].nu > max_nu ? st[i].nu : max_nu;
        if (st[i].ar) st[i].ar_index = n_ar++;
    }
    act_max = (ActView::bytes(max_nu) + 127) & ~127;
    p.nstages = n;
    p.n_ar = n_ar;
    p.max_nu = max_nu;
    p.slot_bytes = (int)((item_max + 32 + 127) & ~int64_t(127));
    p.act_bytes = (int)act_max;
    // static shared memory of the kernel (the group's state) comes off the budget
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, gemv_chain_kernel) != cudaSuccess) return -2;
    const int hdr = CHAIN_HDR;
    static_assert(sizeof(ChainProducer) <= 64, "producer state");
    int warps = GEMV_WARPS, slots = 0;
    const int per_cta = L.smem_per_sm / 2 - L.smem_reserved - (int)fa.sharedSizeBytes;
    for (warps = GEMV_WARPS; warps >= 6; --warps) {
        const int per_warp = ((per_cta - p.act_bytes) / warps & ~127) - hdr;
        slots = per_warp > 0 ? per_warp / p.slot_bytes : 0;
        if (slots > 4) slots = 4;
        if (slots >= 2) break;
    }
    if (slots < 2) return -1;
    p.nslots = slots;
    p.warp_bytes = (hdr + slots * p.slot_bytes + 127) & ~127;
    L.smem = p.act_bytes + warps * p.warp_bytes;
    L.threads = warps * 32;
    if (cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem) != cudaSuccess)
        return -2;
    cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    // every CTA must be resident at once (grid barriers): the grid is what
    // the occupancy calculator says fits, in clusters of two
    cudaLaunchConfig_t q{};
    q.gridDim = dim3((unsigned)(2 * L.num_sms));
    q.blockDim = dim3((unsigned)L.threads);
    q.dynamicSmemBytes = (size_t)L.smem;
    cudaLaunchAttribute ca[1];
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = 2;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = 1;
    q.attrs = ca;
    q.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemv_chain_kernel, &q) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        return -2;
    }
    L.grid = 2 * (clusters < L.num_sms ? clusters : L.num_sms);
    return 0;
}

int launch_chain(const ChainParams &p, const ChainLaunch &L, cudaStream_t st) {
    if (cudaMemsetAsync(p.barrier, 0, sizeof(unsigned), st) != cudaSuccess) return -2;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)L.grid);
    cfg.blockDim = dim3((unsigned)L.threads);
    cfg.dynamicSmemBytes = (size_t)L.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_chain_kernel, p) == cudaSuccess ? 0 : -2;
}

}  // namespace sicu
