// common.cuh -- shared device helpers for the sm_100a decode kernels.
//
// Arithmetic helpers use the _rn intrinsics so nvcc never contracts or reorders them: the
// kernels reproduce the reference's FP32 operation order bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/satori_cuda.h"

namespace satori {

// --------------------------------------------------------------------------- error flags
// Device-side error word of a context: bit 0 = a bounded wait expired.
enum : unsigned { kDevErrTimeout = 1u };

// Spin budget for mbarrier waits: ~4e9 cycles of polling is seconds, far beyond any copy.
constexpr long long kWaitBudgetCycles = 4000000000LL;

// --------------------------------------------------------------------------- launch set-up (host)
// Opts `kernel` in to `bytes` of dynamic shared memory on the CURRENT device.  The attribute belongs to
// a device's context, so the opt-in is remembered per (kernel, device) -- a process that launches on
// several GPUs sets it on each -- under a lock, so concurrent callers on different threads are safe.
cudaError_t opt_in_smem(const void *kernel, size_t bytes);

// --------------------------------------------------------------------------- exact FP32 ops
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }

// The SSE horizontal sum every reference AVX2 kernel ends a block with
// (QuantizedKAvx2Kernel.cs:341-347): ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)).
__device__ __forceinline__ float hsum8(const float a[8])
{
    float h0 = fadd(a[0], a[4]), h1 = fadd(a[1], a[5]), h2 = fadd(a[2], a[6]), h3 = fadd(a[3], a[7]);
    return fadd(fadd(h0, h2), fadd(h1, h3));
}

// Exact small-integer -> float conversion through the 2^23 exponent trick: (float)v - bias, v < 2^23.
__device__ __forceinline__ float u8_to_f_minus(uint32_t v, float bias)
{
    return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.0f + bias);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16)
{
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

// TransformerOps.RmsNorm's sum of squares (TransformerOps.cs:13-22) in FP64, in one fixed order that
// every kernel uses, so a norm fused into a MatVec equals the standalone norm kernel bit for bit:
// 256 strided partials (partial j adds x[j]^2, x[j+256]^2, ... in index order), a shuffle-xor tree over
// each warp's 32 partials, then ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).  Threads 0..255 of the block call
// rms_partial (warp w's lane 0 stores s_w into red[w]); after a barrier any thread calls rms_scale.
__device__ __forceinline__ void rms_partial(const float *x, int n, int tid, double *red)
{
    double sum = 0;
    for (int i = tid; i < n; i += 256) sum = __dadd_rn(sum, __dmul_rn((double)x[i], (double)x[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __dadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, o));
    if ((tid & 31) == 0) red[tid >> 5] = sum;
}

// 1 / sqrt(sum / n + eps), the RmsNorm scale, from the eight warp sums.
__device__ __forceinline__ double rms_scale(const double *red, int n, float eps)
{
    const double sum = __dadd_rn(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])),
                                 __dadd_rn(__dadd_rn(red[4], red[5]), __dadd_rn(red[6], red[7])));
    return __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)n), (double)eps)));
}

// One normalised element: (float)(x * scale * w), each product rounded in FP64.
__device__ __forceinline__ float rms_apply(float x, double scale, float w)
{
    return (float)__dmul_rn(__dmul_rn((double)x, scale), (double)w);
}

// TransformerOps.SwiGlu (TransformerOps.cs:41-51) for one element: FP64 sigmoid of the gate, every
// multiply and add rounded separately, FP32 result.
__device__ __forceinline__ float swiglu_value(float gate, float up)
{
    const double x = gate;
    double sig;
    if (x >= 0) {
        sig = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
    } else {
        const double e = exp(x);
        sig = __ddiv_rn(e, __dadd_rn(1.0, e));
    }
    return (float)__dmul_rn(__dmul_rn(x, sig), (double)up);
}

// --------------------------------------------------------------------------- shared memory
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ float4 lds128f(uint32_t addr)
{
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr)
{
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts128f(uint32_t addr, float4 v)
{
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" :: "r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// --------------------------------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Non-blocking test of a phase (no suspension).
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase completes (or ~hint_ns pass)
// instead of spinning, leaving the issue slots to the warps that have work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and the caller records a timeout) if the phase never flips.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity)
{
    if (mbar_test(bar, parity)) return true;
    long long start = clock64();
    while (!mbar_try_wait_sleep(bar, parity, 100000u)) {
        if (clock64() - start > kWaitBudgetCycles) return false;
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// 2-D tiled TMA load (unicast, no multicast) of the box at (c0 = inner, c1 = outer) of `map`
// into shared memory, completing on `bar`.  `map` is the address of a __grid_constant__ kernel
// parameter; c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int c0, int c1, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const void *map)
{
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 1-D bulk copy global -> shared (TMA unicast, no multicast), completing on `bar`.
// dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// L2 prefetch of a global range (no shared-memory destination, nothing to wait for).  src and bytes must
// be multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(src), "r"(bytes) : "memory");
}

// --------------------------------------------------------------------------- PDL
// Programmatic dependent launch: wait for the producer grid's memory to be visible / let the
// next grid start its prologue.  Both are no-ops when the launch did not use PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

}  // namespace satori
