// Bounded grid-wide barrier of the persistent (cooperative) kernels.
//
// bar[0] counts arrivals over the whole launch (never reset within it), bar[1] is an abort word
// every waiter watches; both are zeroed before each launch. Thread 0 of each CTA arrives and
// waits; the caller brackets the call with its own CTA barrier. A wait that does not see the
// arrivals within `limit` clock cycles raises the abort word (so every other waiter gives up too),
// records `code` in *err (first failure wins) and returns false; the kernel then unwinds and the
// host reads *err after the launch. Nothing traps: the context stays usable.
#pragma once
#include <stdint.h>

namespace nb {

__device__ __forceinline__ bool grid_arrive_wait(unsigned *bar, unsigned target, int *err, int code, long long limit) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    const long long t0 = clock64();
    bool ok = true;
    // the arrival is a release (this CTA's writes, ordered before it by the caller's CTA barrier,
    // are visible to whoever observes it); one acquiring 8-byte load polls the arrival count and
    // the abort word together and orders this CTA's later reads (after the caller's CTA barrier)
    // after every arrival it observed. A relaxed poll followed by fence.acq_rel.gpu measured
    // ~500-700 cycles slower per barrier when the CTAs had stored data before arriving.
    for (;;) {
        unsigned cnt, ab;
        asm volatile("ld.acquire.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(cnt), "=r"(ab) : "l"(bar) : "memory");
        if (cnt >= target) break;
        if (ab) { ok = false; break; }
        if (clock64() - t0 > limit) {
            atomicExch(&bar[1], 1u);
            atomicCAS(err, 0, code);
            ok = false;
            break;
        }
    }
    return ok;
}

}  // namespace nb
