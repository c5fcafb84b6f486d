// Device side of the fused all-reduce of a tensor-parallel group (ArDev in
// launch.h): the partial outputs of a row-split matvec travel to every rank
// over NVLink as plain peer stores, and the consumer adds them up while it
// quantizes its activation. One thread per CTA runs the protocol steps; the
// other threads wait at a CTA barrier.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace sicu {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_vol(const unsigned *p) { return *reinterpret_cast<const volatile unsigned *>(p); }
__device__ __forceinline__ void st_vol(unsigned *p, unsigned v) { *reinterpret_cast<volatile unsigned *>(p) = v; }

// Consumption step 1 (one thread of each CTA, after the stream's previous
// kernels completed): waits until every rank's flag reached this rank's
// delivery count e and returns e; the partials to add are parity (e - 1) & 1.
// Gives up after a.limit_ns (status bit, group marked broken); a broken group
// or a consumption before any delivery returns at once with a status bit.
__device__ __forceinline__ unsigned ar_consume_wait(const ArDev &a, int *status) {
    const unsigned e = ld_vol(a.epoch);
    if (ld_vol(a.epoch + 3)) {
        atomicOr(status, STATUS_AR_TIMEOUT);
        return e;
    }
    if (e == 0) {
        atomicOr(status, STATUS_AR_ORDER);
        st_vol(a.epoch + 3, 1u);
        return e;
    }
    const unsigned *f = a.flag[a.rank];
    uint64_t t0 = 0;
    for (int q = 0; q < a.n; ++q) {
        while ((int)(ld_acquire_sys(f + q) - e) < 0) {
            const uint64_t t = globaltimer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > a.limit_ns) {
                atomicOr(status, STATUS_AR_TIMEOUT);
                st_vol(a.epoch + 3, 1u);
                return e;
            }
        }
    }
    // every CTA stores the same value: the deliveries up to e are consumed
    st_vol(a.epoch + 1, e);
    return e;
}

// Delivery step 1 (one thread of each CTA, after the stream's previous
// kernels completed): the delivery count e, or false when the group is broken
// or the previous delivery was not consumed yet (status bit, no delivery).
__device__ __forceinline__ bool ar_deliver_begin(const ArDev &a, int *status, unsigned &e) {
    e = ld_vol(a.epoch);
    if (ld_vol(a.epoch + 3)) {
        atomicOr(status, STATUS_AR_TIMEOUT);
        return false;
    }
    if (ld_vol(a.epoch + 1) != e) {
        atomicOr(status, STATUS_AR_ORDER);
        st_vol(a.epoch + 3, 1u);
        return false;
    }
    return true;
}

// Where element i of this rank's delivery e goes on rank q.
__device__ __forceinline__ float *ar_dst(const ArDev &a, int q, unsigned e) {
    return a.slot[q] + ((int64_t)(e & 1u) * a.n + a.rank) * a.len;
}

// Delivery step 2 (one thread of each CTA, after every thread of the CTA
// fenced its peer stores at system scope and met at a CTA barrier): the last
// CTA to arrive publishes the delivery: count e + 1 here, flag e + 1 on every
// rank (release, so a peer that sees the flag sees the data).
__device__ __forceinline__ void ar_deliver_arrive(const ArDev &a, unsigned e) {
    __threadfence_system();
    const unsigned old = atomicAdd(a.epoch + 2, 1u);
    if (old == gridDim.x - 1) {
        __threadfence_system();
        st_vol(a.epoch + 2, 0u);
        st_vol(a.epoch, e + 1);
#pragma unroll
        for (int q = 0; q < AR_MAX; ++q)
            if (q < a.n) st_release_sys(a.flag[q] + a.rank, e + 1);
    }
}

}  // namespace sicu
