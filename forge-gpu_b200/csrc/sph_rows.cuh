// Row-parallel neighbour passes for small, sparse workloads (sm_100a).
//
// With a few particles per cell (the reference's 50K dam break: ~1.5) a
// particle has only a few dozen candidates, and the per-thread and group
// walks are bound by latency: nine rows visited one after another, each a
// dependent cell-table load and then the candidate loads. Here the nine rows
// of a particle are walked at the same time by nine threads:
//
//   block = 32 particles x 9 rows = 288 threads, thread t: particle t / 9,
//   row t % 9 (row r = (dz+1)*3 + (dy+1), as everywhere in sph.cuh)
//
// so a particle's walk costs one cell-table latency and one round of
// candidate loads. Each thread sums its row (ascending j) into a partial; the
// partials go through shared memory and thread p of the block adds particle
// p's nine in row order. The sum of a particle depends on nothing but the
// particle (no other particle shares its lanes): deterministic and the same in
// any cell order or zone list, equal to the reference's one-accumulator sum to
// fp32 rounding (the stated tolerances).
#pragma once

#include "sph.cuh"

namespace forge {
namespace sph {

constexpr int kRowsParticles = 32;
constexpr int kRowsThreads = kRowsParticles * 9;

// ---------------------------------------------------------------------------
// Density (poly6, self included).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kRowsThreads)
    density_rows_kernel(float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                        const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c,
                        float4* __restrict__ vel4, float2* __restrict__ aux, float* __restrict__ density_out) {
    pdl_enter();
    __shared__ float part[kRowsThreads];
    const int t = threadIdx.x, pl = t / 9, r = t - pl * 9;
    const uint32_t s0 = blockIdx.x * kRowsParticles;
    const uint32_t s = s0 + pl;
    float rho = 0.f;
    if (s < n) {
        const float4 p = pos4[s];
        const Frame f = make_frame(p, g);
        int lo, hi;
        if (row_window(f, r, g, c.h2_skip, lo, hi)) {
            const uint32_t row = row_base(g, f, r);
            poly6_one(pos4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), p, c, rho);
        }
    }
    part[t] = rho;
    __syncthreads();
    if (t >= kRowsParticles) return;
    const uint32_t sp = s0 + t;
    if (sp >= n) return;
    float sum = part[t * 9];
#pragma unroll
    for (int k = 1; k < 9; ++k) sum += part[t * 9 + k];
    sum *= c.mass_poly6;
    float inv_rho;
    float2 a;
    density_derived(sum, c, inv_rho, a);
    if (vel4 != nullptr) {
        vel4[sp].w = inv_rho;
        aux[sp] = a;
        const float4 q = pos4[sp];
        pos4[sp] = make_float4(q.x, q.y, q.z, a.x);
    }
    if (density_out != nullptr) density_out[sorted_idx[sp]] = sum;
}

// ---------------------------------------------------------------------------
// Force (pressure + viscosity, Jacobi) + epilogue. Each thread scans its row
// for r^2 < h^2 and evaluates the hits (sph.cuh force_one); the six partial
// sums of a particle's rows are added in row order by thread p, which then
// runs the epilogue. LIST: particle slots index a zone list.
// ---------------------------------------------------------------------------
template <int TERMS, int EPI, bool LIST>
__global__ void __launch_bounds__(kRowsThreads)
    force_rows_kernel(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                      const float2* __restrict__ aux, const uint32_t* __restrict__ cell_start,
                      const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c, StepEpi ep,
                      ForceOut out, ZoneList zl) {
    pdl_enter();
    __shared__ float part[6][kRowsThreads];
    uint32_t cnt = n;
    const uint32_t* lst = nullptr;
    if (LIST) lst = zone_begin(zl, cnt);
    const int t = threadIdx.x, pl = t / 9, r = t - pl * 9;
    const uint32_t t0 = blockIdx.x * kRowsParticles;
    if (t0 >= cnt) return;  // whole block
    const uint32_t slot = t0 + pl;
    ForceAcc A;
    A.pax = A.pay = A.paz = A.vax = A.vay = A.vaz = 0.f;
    if (slot < cnt) {
        const uint32_t s = LIST ? lst[slot] : slot;
        A = force_acc(pos4, vel4, aux, s, c, g);
        // rho < 1e-6 (1/rho stored as 0) or not updated (a ghost): no walk
        if (A.v.w != 0.f && sorted_idx[s] < out.limit) {
            const Frame f = make_frame(A.p, g);
            int lo, hi;
            if (row_window(f, r, g, c.h2_skip, lo, hi)) {
                const uint32_t row = row_base(g, f, r);
                force_one<TERMS>(pos4, vel4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), A,
                                 c);
            }
        }
    }
    part[0][t] = A.pax;
    part[1][t] = A.pay;
    part[2][t] = A.paz;
    part[3][t] = A.vax;
    part[4][t] = A.vay;
    part[5][t] = A.vaz;
    __syncthreads();
    if (t >= kRowsParticles) return;
    const uint32_t sp = t0 + t;
    if (sp >= cnt) return;
    const uint32_t s = LIST ? lst[sp] : sp;
    ForceAcc B = force_acc(pos4, vel4, aux, s, c, g);
    float acc[6];
#pragma unroll
    for (int q = 0; q < 6; ++q) {
        float v = part[q][t * 9];
#pragma unroll
        for (int k = 1; k < 9; ++k) v += part[q][t * 9 + k];
        acc[q] = v;
    }
    B.pax = acc[0];
    B.pay = acc[1];
    B.paz = acc[2];
    B.vax = acc[3];
    B.vay = acc[4];
    B.vaz = acc[5];
    force_finish<EPI>(B, sorted_idx[s], ep, out);
}

}  // namespace sph
}  // namespace forge
