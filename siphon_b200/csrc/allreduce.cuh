// Device side of the all-reduce fused into a row-split matvec (ArDev in
// launch.h): every CTA sends the partial outputs of the rows it computed to
// every rank over NVLink as tagged 64-bit peer stores, then waits for the
// other ranks' parts of the same rows (each word checked for its tag) and
// writes their sum. No fence, flag or counter is on the critical path.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace sicu {

__device__ __forceinline__ unsigned ld_vol(const unsigned *p) { return *reinterpret_cast<const volatile unsigned *>(p); }
__device__ __forceinline__ void st_vol(unsigned *p, unsigned v) { *reinterpret_cast<volatile unsigned *>(p) = v; }
// one tagged element: a single 64-bit store is single-copy atomic, so a
// reader that sees the tag sees the value stored with it
__device__ __forceinline__ void st_tagged(uint64_t *p, float v, unsigned tag) {
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(w) : "memory");
}

// ---- one delivery ----------------------------------------------------------------
// State read once per CTA (one thread, after the stream's previous kernels
// completed): e = deliveries this rank made so far (this one is e + 1), and
// whether an earlier failure broke the group.
struct ArState {
    unsigned e, broken;
};
__device__ __forceinline__ ArState ar_load_state(const ArDev &a) {
    return ArState{ld_vol(a.epoch), ld_vol(a.epoch + 3)};
}

// Where rank `from`'s part of delivery e + 1 lives in rank q's memory.
__device__ __forceinline__ uint64_t *ar_part(const ArDev &a, int q, int from, unsigned e) {
    return a.slot[q] + ((int64_t)(e & 1u) * a.n + from) * a.len;
}

// Counts the delivery once every CTA has read the count (each CTA arrives
// after its read; the last one to arrive stores e + 1).
__device__ __forceinline__ void ar_arrive(const ArDev &a, unsigned e) {
    const unsigned old = atomicAdd(a.epoch + 2, 1u);
    if (old == gridDim.x - 1) {
        st_vol(a.epoch + 2, 0u);
        st_vol(a.epoch, e + 1);
    }
}

// Sends element i of this rank's partial (delivery e + 1) to every rank.
__device__ __forceinline__ void ar_send(const ArDev &a, unsigned e, int64_t i, float v) {
#pragma unroll
    for (int q = 0; q < AR_MAX; ++q)
        if (q < a.n) st_tagged(ar_part(a, q, a.rank, e) + i, v, e + 1);
}

// Element i of the sum over ranks (rank order, f32) of delivery e + 1, from
// this rank's memory, each part read once it carries tag e + 1. The wait is
// bounded: after limit_ns, or at once when the group is already broken, the
// words are used as they are (status bit, group marked broken; `live` turns
// false so the calling thread waits no more).
__device__ __forceinline__ float ar_sum(const ArDev &a, unsigned e, int64_t i, int *status, bool &live) {
    uint64_t w[AR_MAX];
#pragma unroll
    for (int q = 0; q < AR_MAX; ++q)
        if (q < a.n) w[q] = *reinterpret_cast<const volatile uint64_t *>(ar_part(a, a.rank, q, e) + i);
    if (live) {
        uint64_t t0 = 0;
        for (;;) {
            bool ready = true;
#pragma unroll
            for (int q = 0; q < AR_MAX; ++q)
                if (q < a.n) ready &= (unsigned)(w[q] >> 32) == e + 1;
            if (ready) break;
            const uint64_t t = globaltimer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > a.limit_ns || ld_vol(a.epoch + 3)) {
                atomicOr(status, STATUS_AR_TIMEOUT);
                st_vol(a.epoch + 3, 1u);
                live = false;
                break;
            }
#pragma unroll
            for (int q = 0; q < AR_MAX; ++q)
                if (q < a.n && (unsigned)(w[q] >> 32) != e + 1)
                    w[q] = *reinterpret_cast<const volatile uint64_t *>(ar_part(a, a.rank, q, e) + i);
        }
    }
    float s = __uint_as_float((uint32_t)w[0]);
#pragma unroll
    for (int q = 1; q < AR_MAX; ++q)
        if (q < a.n) s = __fadd_rn(s, __uint_as_float((uint32_t)w[q]));
    return s;
}

}  // namespace sicu
