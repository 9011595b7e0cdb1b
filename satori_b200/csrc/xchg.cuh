// xchg.cuh -- peer exchange hooks that a producing and a consuming MatVec launch of a sharded decode step
// carry, so that the all-gather of a row-sharded output needs no launch of its own.
//
// Producer: while it writes each output value, the launch also stores it into every peer's copy of the
// gathered buffer (NVLink stores into IPC-mapped memory); after its last row, every CTA fences and the
// last CTA to finish advances this rank's exchange sequence number n and release-stores n into each
// peer's flag for this rank.  Consumer: before reading the gathered vector, one thread of each CTA waits
// (bounded) until every peer's flag holds this rank's current n.
//
// Ordering (with the exchange kernel in session_sharded.cu for the exchanges a launch cannot carry): a
// rank's consumer of exchange n only runs after its producer of n completed, so the sequence numbers of
// all ranks advance in step; a peer's stores into this rank's buffer for exchange n happen after that
// peer has waited for exchange n-1, which this rank signals only after it has last read the buffer's
// remote slices.
#pragma once

#include "common.cuh"

namespace satori {

constexpr int kXchgMaxRanks = 8;

struct XPush {
    float *dst[kXchgMaxRanks];                  // peer address of the launch's output element 0 (null: self)
    unsigned long long *signal[kXchgMaxRanks];  // the peer's flag for this rank
    unsigned *ticket;                           // this rank's count of CTAs done with the running exchange
    unsigned long long *seq;                    // this rank's exchanges signalled
    int world, rank;                            // world == 0: no push
};

struct XWait {
    const unsigned long long *flags;            // this rank's flags, one per source rank
    const unsigned long long *seq;
    long long budget;                           // SM cycles
    int world, rank;                            // world == 0: no wait
};

__device__ __forceinline__ void xchg_store_release_sys(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long xchg_load_acquire_sys(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Stores one output value into every peer's copy.
__device__ __forceinline__ void xpush_value(const XPush &x, long long idx, float v)
{
    for (int p = 0; p < x.world; ++p)
        if (x.dst[p]) x.dst[p][idx] = v;
}

// One thread per CTA, after every thread of the CTA that pushed has fenced its stores system-wide.
__device__ inline void xpush_finish(const XPush &x)
{
    if (atomicAdd(x.ticket, 1u) != gridDim.x - 1) return;
    *x.ticket = 0;
    const unsigned long long n = *reinterpret_cast<volatile unsigned long long *>(x.seq) + 1;
    *x.seq = n;
    __threadfence_system();
    for (int p = 0; p < x.world; ++p)
        if (p != x.rank) xchg_store_release_sys(x.signal[p], n);
}

// One thread: wait until every peer has signalled this rank's current sequence number.  An expired wait
// (or one already recorded in this step) sets the timeout bit and returns false.
__device__ inline bool xwait_peers(const XWait &w, unsigned *err)
{
    const unsigned long long n = *reinterpret_cast<const volatile unsigned long long *>(w.seq);
    const long long start = clock64();
    for (int p = 0; p < w.world; ++p) {
        if (p == w.rank) continue;
        while (xchg_load_acquire_sys(&w.flags[p]) < n) {
            if (clock64() - start > w.budget || (*reinterpret_cast<volatile unsigned *>(err) & kDevErrTimeout)) {
                atomicOr(err, kDevErrTimeout);
                return false;
            }
        }
    }
    return true;
}

}  // namespace satori
