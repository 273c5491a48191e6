// Cell-block density pass with shared-memory staging by TMA bulk copies
// (sm_100a).
//
// The per-thread walks read every candidate with its own 16-byte global
// load; the lanes of a warp read unrelated addresses, so the passes are
// bound by L1 wavefronts, not by bytes. Here a CTA owns one segment of a
// grid row: cells [x0, x0 + kTileCells) of row (cy, cz). All candidates of
// its particles lie in the 9 rows (cy + dy, cz + dz) over cells
// [x0 - 1, x0 + kTileCells + 1), and in each row they are one contiguous
// range of the cell order. So the CTA
//
//   1. loads the cell-table entries of those 9 row ranges into shared memory;
//   2. stages the 9 position ranges into shared memory with one 1-D TMA bulk
//      copy each (cp.async.bulk, completion on an mbarrier; no multicast);
//   3. walks each owned particle's trimmed windows (sph.cuh row_window) over
//      the staged rows: shared-memory loads instead of global ones.
//
// Candidates and their order are exactly those of the per-thread walk (rows
// in the reference order (dz, dy), ascending j inside a window), so the sums
// are bit-identical to it. A segment whose rows hold more than kTileCap
// particles (dense cells) walks the same windows from global memory.
//
// Measured on one B200 it is slower than the per-thread walks it replaces
// (16.4M particles, 160^3 cells: 2.38 vs 1.25 ms; the 1M dam break 0.23 vs
// 0.10 ms; two particles per thread sharing each staged candidate: 3.18 ms):
// each CTA waits for its own copies with nothing to overlap them, the rows
// are staged for 9 segments each, and 73 KiB per CTA leaves 3 CTAs per SM.
// It stays an explicit choice (FORGE_WALK_TILE, density only); AUTO never
// takes it.
#pragma once

#include "sph.cuh"

namespace forge {
namespace sph {

constexpr int kTileCells = 64;    // cells per segment
constexpr int kTileThreads = 256;
constexpr int kTileCap = 4096;    // staged particles per CTA (64 KiB of float4)
constexpr int kTileMaxSub = 2;    // x-slices per cell: at most 2^kTileMaxSub
constexpr int kTileEntries = (kTileCells + 2) * (1 << kTileMaxSub) + 1;  // cell-table entries per row
constexpr uint32_t kTileSpinLimit = 1u << 22;  // mbarrier polls before the wait gives up

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    return done != 0;
}

// Bounded wait for phase `phase` of the mbarrier; false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    for (uint32_t k = 0; k < kTileSpinLimit; ++k)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}

__global__ void __launch_bounds__(kTileThreads)
    density_tile_kernel(float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                        const uint32_t* __restrict__ sorted_idx, Geom g, SphConsts c, uint32_t segs,
                        float4* __restrict__ vel4, float2* __restrict__ aux, float* __restrict__ density_out,
                        uint32_t* __restrict__ err) {
    pdl_enter();
    extern __shared__ __align__(16) float4 s_pos[];  // kTileCap staged positions
    __shared__ uint32_t s_cs[9][kTileEntries];
    __shared__ uint32_t s_b[9], s_off[9];
    __shared__ __align__(8) uint64_t s_bar;
    __shared__ int s_staged;
    const int t = threadIdx.x;
    const uint32_t S = 1u << g.sub_bits;
    const uint32_t row0 = blockIdx.x / segs, seg = blockIdx.x - row0 * segs;
    const int cz0 = (int)(row0 / (uint32_t)g.ny), cy0 = (int)(row0 - (uint32_t)cz0 * (uint32_t)g.ny);
    const int x0 = (int)seg * kTileCells, x1 = min(x0 + kTileCells, g.nx);
    const int xa = max(x0 - 1, 0), xb = min(x1 + 1, g.nx);
    const uint32_t sa = (uint32_t)xa * S, entries = (uint32_t)(xb - xa) * S + 1;
    const uint32_t row_len = (uint32_t)g.nx * S;

    // 1. cell-table entries of the 9 row ranges (0 for rows outside the grid)
    for (uint32_t k = t; k < 9 * entries; k += kTileThreads) {
        const uint32_t r = k / entries, e = k - r * entries;
        const int z = cz0 + (int)(r / 3) - 1, y = cy0 + (int)(r % 3) - 1;
        uint32_t v = 0;
        if (z >= 0 && z < g.nz && y >= 0 && y < g.ny)
            v = __ldg(cell_start + ((uint32_t)z * (uint32_t)g.ny + (uint32_t)y) * row_len + sa + e);
        s_cs[r][e] = v;
    }
    __syncthreads();

    // 2. stage the 9 position ranges (one thread issues the bulk copies)
    const uint32_t bar = smem_u32(&s_bar);
    if (t == 0) {
        uint32_t total = 0;
        for (int r = 0; r < 9; ++r) {
            s_b[r] = s_cs[r][0];
            s_off[r] = total;
            total += s_cs[r][entries - 1] - s_cs[r][0];
        }
        const int staged = total > 0 && total <= (uint32_t)kTileCap;
        s_staged = staged;
        if (staged) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(total * 16u)
                         : "memory");
            for (int r = 0; r < 9; ++r) {
                const uint32_t cnt = s_cs[r][entries - 1] - s_cs[r][0];
                if (cnt == 0) continue;
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        smem_u32(s_pos + s_off[r])),
                    "l"(pos4 + s_b[r]), "r"(cnt * 16u), "r"(bar)
                    : "memory");
            }
        }
    }
    __syncthreads();
    bool staged = s_staged != 0;
    if (staged && !mbar_wait(bar, 0)) {
        // the copies did not complete in time: report, wait (bounded) for
        // them once more before leaving shared memory, walk from global
        if (t == 0) atomicOr(err, kDevTimeout);
        mbar_wait(bar, 0);
        staged = false;
    }

    // 3. the owned particles: row 4 (dz = dy = 0), cells [x0, x1)
    const uint32_t own_b = s_cs[4][(uint32_t)(x0 - xa) * S], own_e = s_cs[4][(uint32_t)(x1 - xa) * S];
    for (uint32_t j = own_b + t; j < own_e; j += kTileThreads) {
        const float4 p = staged ? s_pos[s_off[4] + (j - s_b[4])] : pos4[j];
        const Frame f = make_frame(p, g);
        float rho = 0.f;
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int lo, hi;
            if (!row_window(f, r, g, c.h2_skip, lo, hi)) continue;
            const uint32_t b = s_cs[r][(uint32_t)lo - sa], e = s_cs[r][(uint32_t)hi + 1 - sa];
            if (staged) {
                const float4* q = s_pos + s_off[r] - s_b[r];
#pragma unroll 4
                for (uint32_t k = b; k < e; ++k) {
                    const float d = poly6_base(p, q[k], c.h2);
                    rho = fmaf(d * d, d, rho);
                }
            } else {
                poly6_one(pos4, b, e, p, c, rho);
            }
        }
        rho *= c.mass_poly6;
        float inv_rho;
        float2 a;
        density_derived(rho, c, inv_rho, a);
        if (vel4 != nullptr) {
            vel4[j].w = inv_rho;
            aux[j] = a;
            pos4[j] = make_float4(p.x, p.y, p.z, a.x);
        }
        if (density_out != nullptr) density_out[sorted_idx[j]] = rho;
    }
}

}  // namespace sph
}  // namespace forge
