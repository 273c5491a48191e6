// Shared device helpers for the particle hot path (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace forge {

// Device status bits (mirrors FORGE_DEV_* in include/forge_sph.h).
constexpr uint32_t kDevTimeout = 0x1u;
constexpr uint32_t kDevKeyRange = 0x2u;
constexpr uint32_t kDevCapacity = 0x4u;
constexpr uint32_t kDevZone = 0x8u;  // an interior particle of a zoned force pass entered the boundary zone

// Upper bound on polls of one look-back status word before a wait gives up
// and reports kDevTimeout (~0.3 s with the back-off below). A predecessor
// tile always publishes its aggregate without waiting on anything, so this
// only triggers if the device is badly oversubscribed or something is wrong.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Programmatic dependent launch. The kernels of a step chain are launched
// with cudaLaunchAttributeProgrammaticStreamSerialization, so a kernel's
// launch is processed while its predecessor in the stream drains (its CTAs
// become eligible as the predecessor's CTAs exit). Every such kernel calls
// pdl_enter() first: griddepcontrol.wait returns once the predecessor grid
// has completed and its writes are visible (immediately for a kernel
// launched without the attribute). Nothing is read or written before the wait
// and every CTA executes it (no early return ahead of it), so a grid's
// completion still implies the completion of all work before it in the
// stream. No kernel triggers its dependents early (launch_dependents): CTAs
// parked at the wait while the predecessor still runs cost more in CUDA
// graph replays than the launch latency they hide (the 50K dam break: 58 vs
// 65 us per step).
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Streaming (evict-first) 128-bit global load for data read exactly once.
__device__ __forceinline__ float4 ld_stream_f4(const float4* p) {
    float4 v;
    asm volatile("ld.global.cs.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// Unsigned division of n < 2^31 by a fixed divisor 1 <= d < 2^31 with one
// 64-bit multiply and a shift: floor(n / d) == (n * m) >> s for
// s = 31 + ceil(log2 d), m = floor(2^s / d) + 1 (m d - 2^s <= d <= 2^(s-31)).
struct FastDiv {
    uint64_t m;
    uint32_t s;
    uint32_t d;
};

__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    FastDiv f;
    f.d = d;
    f.s = 31 + l;
    f.m = (1ull << f.s) / d + 1;
    return f;
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
    return (uint32_t)(((uint64_t)n * f.m) >> f.s);
}

// Hardware square root approximation (relative error ~2^-22; callers that
// bound a search window add a margin for it).
__device__ __forceinline__ float sqrt_approx(float x) {
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Exclusive scan of one uint32 per thread over a block of NT threads
// (NT a multiple of 32, <= 1024). `warp_tot` is shared scratch of NT/32
// words. Returns the exclusive prefix; *total receives the block sum.
template <int NT>
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_tot,
                                                         uint32_t* total) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < NW ? warp_tot[lane] : 0u;
        uint32_t wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < NW) warp_tot[lane] = wi - w;  // exclusive warp offsets
        if (lane == NW - 1) warp_tot[NW] = wi;   // block total
    }
    __syncthreads();
    uint32_t r = warp_tot[warp] + inc - v;
    *total = warp_tot[NW];
    __syncthreads();  // warp_tot may be reused by the caller
    return r;
}

}  // namespace forge
