// SPH neighbour passes (sm_100a): poly6 density and the fused spiky-pressure
// + viscosity-Laplacian force with the manifest step epilogue.
//
// Data layout (HBM): particles live in the caller's SoA arrays in ORIGINAL
// order. After the grid build the library holds cell-ordered copies
//   pos4[s] = (x, y, z, bits(cell key))
//   vel4[s] = (vx, vy, vz, 1/rho)       (1/rho := 0 when rho < 1e-6)
//   aux[s]  = (p/rho, rho)              p = k (rho - rho0)
// so for each (dz, dy) the three cells dx = -1..1 are ONE contiguous range
// [cell_start[row+cx-1], cell_start[row+cx+2]). Walking the rows dz-major,
// dy-minor visits neighbours in exactly the reference order (dz, dy, dx, then
// ascending particle index inside a cell), sph_density.rs:429-458.
//
// Per particle the walk is trimmed to the cells whose box can hold a point
// closer than h: a cell (or a whole row) is skipped only when the squared
// distance from the particle to the cell's box, shrunk by a rounding slack,
// exceeds h^2 (1 + 1e-4). Every pair with r^2 < h^2 is still visited, in the
// same order, so the sums are unchanged; at cell size h this removes ~24% of
// the candidates, at the reference's default cell size 2h far more.
//
// One thread per particle in cell order: consecutive lanes sit in the same or
// adjacent cells, so a warp walks (almost) the same ranges and neighbour
// loads are warp-broadcasts served by L1. Results are scattered back to the
// original order through sorted_idx.
//
// Both passes are bound by instruction issue, not HBM (a few % of DRAM
// bandwidth at these densities), so the kernels minimise instructions per
// candidate pair: the density sum is branchless, and the force pass first
// scans a chunk of 32 candidates for r^2 < h^2 (cheap) and then evaluates the
// expensive pair term only for the hits, with per-particle reciprocals
// instead of per-pair divides.
#pragma once

#include "common.cuh"

namespace forge {
namespace sph {

struct SphConsts {
    float h, h2;
    float h2_skip;     // h^2 (1 + 1e-4): cell-skip threshold
    float mass_poly6;  // mass * 315 / (64 pi h^9)     (sph_density.rs:413-416)
    float mass;
    float k, rho0, mu;
    float kp;  // -mass/2 * spiky, spiky = -45/(pi h^6)  (sph_fused.rs:552-613)
    float kv;  // mu * mass * 45/(pi h^6)                (sph_fused.rs:619-620)
};

struct Geom {
    float ox, oy, oz, cs;
    int nx, ny, nz;
};

__device__ __forceinline__ void key_to_cell(uint32_t key, const Geom& d, int& cx, int& cy, int& cz) {
    const uint32_t t = key / (uint32_t)d.nx;
    cx = (int)(key - t * (uint32_t)d.nx);
    cy = (int)(t % (uint32_t)d.ny);
    cz = (int)(t / (uint32_t)d.ny);
}

// Squared conservative gap: distance shrunk by a slack covering the rounding
// of the cell assignment and of r^2, clamped at 0 (clamped out-of-grid
// particles give negative raw gaps -> 0, i.e. never skipped).
__device__ __forceinline__ float gap2(float raw, float slack) {
    const float g = fmaxf(raw - slack, 0.f);
    return g * g;
}

// Calls f(b, e) for each trimmed contiguous candidate range of particle p
// (cell-ordered indices), in reference order.
template <class F>
__device__ __forceinline__ void for_each_range(const float4& p, const Geom& g, const uint32_t* __restrict__ cell_start,
                                               float H, F&& f) {
    int cx, cy, cz;
    key_to_cell(__float_as_uint(p.w), g, cx, cy, cz);
    const float bx = g.ox + (float)cx * g.cs, by = g.oy + (float)cy * g.cs, bz = g.oz + (float)cz * g.cs;
    const float sx = 4e-7f * (fabsf(p.x) + fabsf(bx) + g.cs);
    const float sy = 4e-7f * (fabsf(p.y) + fabsf(by) + g.cs);
    const float sz = 4e-7f * (fabsf(p.z) + fabsf(bz) + g.cs);
    const float gxl = gap2(p.x - bx, sx), gxr = gap2(bx + g.cs - p.x, sx);
    const float gyl = gap2(p.y - by, sy), gyr = gap2(by + g.cs - p.y, sy);
    const float gzl = gap2(p.z - bz, sz), gzr = gap2(bz + g.cs - p.z, sz);
    for (int dz = -1; dz <= 1; ++dz) {
        const int z = cz + dz;
        if (z < 0 || z >= g.nz) continue;
        const float gz = dz < 0 ? gzl : (dz > 0 ? gzr : 0.f);
        for (int dy = -1; dy <= 1; ++dy) {
            const int y = cy + dy;
            if (y < 0 || y >= g.ny) continue;
            const float base = gz + (dy < 0 ? gyl : (dy > 0 ? gyr : 0.f));
            if (base > H) continue;
            const int lo = (cx > 0 && base + gxl <= H) ? cx - 1 : cx;
            const int hi = (cx < g.nx - 1 && base + gxr <= H) ? cx + 2 : cx + 1;
            const uint32_t row = ((uint32_t)z * (uint32_t)g.ny + (uint32_t)y) * (uint32_t)g.nx;
            f(__ldg(cell_start + row + lo), __ldg(cell_start + row + hi));
        }
    }
}

// Per-particle data the force pass reads for a neighbour, from its density.
__device__ __forceinline__ void density_derived(float rho, const SphConsts& c, float& inv_rho, float2& aux) {
    const bool valid = !(rho < 1e-6f);
    inv_rho = valid ? 1.0f / rho : 0.f;  // 0 makes an invalid neighbour contribute nothing
    const float p = c.k * (rho - c.rho0);
    aux = make_float2(valid ? p * inv_rho : 0.f, rho);
}

// ---------------------------------------------------------------------------
// Density: rho_i = sum_{j: r2 < h2} m * poly6 * (h2 - r2)^3, self included.
// max(h2 - r2, 0)^3 adds exactly +0 for pairs outside h (and for NaN r2), so
// the sum equals the reference's branchy one. Writes 1/rho to vel4[s].w, aux[s]
// and, if given, density_out[i] (original order).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128)
    density_kernel(const float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                   const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c,
                   float4* __restrict__ vel4, float2* __restrict__ aux, float* __restrict__ density_out) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const float4 pi = pos4[s];
    float rho = 0.f;
    for_each_range(pi, g, cell_start, c.h2_skip, [&](uint32_t b, uint32_t e) {
#pragma unroll 4
        for (uint32_t j = b; j < e; ++j) {
            const float4 q = __ldg(pos4 + j);
            const float dx = pi.x - q.x, dy = pi.y - q.y, dz = pi.z - q.z;
            const float r2 = dx * dx + dy * dy + dz * dz;
            const float d = fmaxf(c.h2 - r2, 0.f);
            rho += c.mass_poly6 * d * d * d;
        }
    });
    float inv_rho;
    float2 a;
    density_derived(rho, c, inv_rho, a);
    if (vel4 != nullptr) {
        vel4[s].w = inv_rho;
        aux[s] = a;
    }
    if (density_out != nullptr) density_out[sorted_idx[s]] = rho;
}

// vel4[s] = (vx[i], vy[i], vz[i], 1/rho[i]), aux[s] = (p/rho, rho), i = svals[s]
// (forge_sph_force with a caller-supplied density).
__global__ void __launch_bounds__(256)
    gather_vel_rho_kernel(const uint32_t* __restrict__ svals, uint32_t n, const float* __restrict__ vx,
                          const float* __restrict__ vy, const float* __restrict__ vz,
                          const float* __restrict__ rho, SphConsts c, float4* __restrict__ vel4,
                          float2* __restrict__ aux) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const uint32_t i = svals[s];
    float inv_rho;
    float2 a;
    density_derived(rho[i], c, inv_rho, a);
    vel4[s] = make_float4(vx[i], vy[i], vz[i], inv_rho);
    aux[s] = a;
}

// ---------------------------------------------------------------------------
// Force pass. TERMS: 1 pressure, 2 viscosity, 3 both (fused). Jacobi: all
// neighbour data come from the cell-ordered snapshot (pos4, vel4, aux), so
// the update never races with reads (fixes the in-place vx[i] += of
// sph_fused.rs:635-637 / sph_viscosity.rs:103-105).
//
// Pair term, algebraically the reference's (sph_fused.rs:604-623):
//   f = -m (p_i + p_j) / (2 rho_j) * spiky (h-r)^2 / r
//     = kp * (p_i/rho_j + p_j/rho_j) * (h-r)^2 / r
//   v = mu m / rho_j * lap (h-r) = kv * (1/rho_j) * (h-r)
// with 1/rho_j and p_j/rho_j precomputed per particle (0 for rho_j < 1e-6,
// which reproduces the reference's skip of such neighbours). r = sqrtf of an
// uncontracted r^2 (the reference's rounding), because h - r cancels for r
// near h; 1/r uses rsqrtf (its error only scales the term).
//
// EPI == 0: write vel_out[i] = v_i + a_i dt (and accel_out[i] = a_i).
// EPI == 1: manifest step epilogue: + gravity, NaN/Inf reset + integrate,
//           box clamp/reflect; writes pos and vel in place (original order).
// ---------------------------------------------------------------------------
struct ForceOut {
    float* vx;
    float* vy;
    float* vz;
    float* ax;  // nullable
    float* ay;
    float* az;
    float* px;  // EPI == 1
    float* py;
    float* pz;
};

struct StepEpi {
    float dt;
    float gx, gy, gz;
    float bmin[3], bmax[3];
    float restitution;
    uint32_t flags;  // FORGE_STEP_* bits
};

template <int TERMS, int EPI>
__global__ void __launch_bounds__(128)
    force_kernel(const float4* __restrict__ pos4, const float4* __restrict__ vel4, const float2* __restrict__ aux,
                 const uint32_t* __restrict__ cell_start, const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g,
                 SphConsts c, StepEpi ep, ForceOut out) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const float4 pi = pos4[s];
    const float4 vi = vel4[s];
    const float rho_i = aux[s].y;
    const bool valid = !(rho_i < 1e-6f);
    const float p_i = c.k * (rho_i - c.rho0);
    const float* __restrict__ pj_over_rho = reinterpret_cast<const float*>(aux);

    float pax = 0.f, pay = 0.f, paz = 0.f;
    float vax = 0.f, vay = 0.f, vaz = 0.f;
    if (valid) {
        for_each_range(pi, g, cell_start, c.h2_skip, [&](uint32_t b, uint32_t e) {
            for (uint32_t j0 = b; j0 < e; j0 += 32) {
                const uint32_t cnt = min(32u, e - j0);
                // Phase 1: which of the next <= 32 candidates are in range.
                uint32_t hit = 0;
#pragma unroll 4
                for (uint32_t k = 0; k < cnt; ++k) {
                    const float4 q = __ldg(pos4 + j0 + k);
                    const float dx = pi.x - q.x, dy = pi.y - q.y, dz = pi.z - q.z;
                    const float r2 = dx * dx + dy * dy + dz * dz;
                    hit |= (r2 < c.h2 && r2 > 1e-12f) ? (1u << k) : 0u;
                }
                // Phase 2: pair terms for the hits, ascending j.
                while (hit) {
                    const uint32_t j = j0 + (uint32_t)(__ffs(hit) - 1);
                    hit &= hit - 1;
                    const float4 q = __ldg(pos4 + j);
                    const float4 vj = __ldg(vel4 + j);
                    const float djx = pi.x - q.x, djy = pi.y - q.y, djz = pi.z - q.z;
                    const float r2 = __fadd_rn(__fadd_rn(__fmul_rn(djx, djx), __fmul_rn(djy, djy)),
                                               __fmul_rn(djz, djz));
                    const float diff = c.h - sqrtf(r2);
                    const float inv_rho_j = vj.w;
                    if (TERMS & 1) {
                        const float pp = fmaf(p_i, inv_rho_j, __ldg(pj_over_rho + 2 * j));
                        const float f = c.kp * pp * (diff * diff) * rsqrtf(r2);
                        pax = fmaf(f, djx, pax);
                        pay = fmaf(f, djy, pay);
                        paz = fmaf(f, djz, paz);
                    }
                    if (TERMS & 2) {
                        const float v = c.kv * inv_rho_j * diff;
                        vax = fmaf(v, vj.x - vi.x, vax);
                        vay = fmaf(v, vj.y - vi.y, vay);
                        vaz = fmaf(v, vj.z - vi.z, vaz);
                    }
                }
            }
        });
    }

    // a = (a_p + a_v) / rho_i (sph_fused.rs:633-638).
    float ax = 0.f, ay = 0.f, az = 0.f;
    float vx = vi.x, vy = vi.y, vz = vi.z;
    if (valid) {
        const float inv_rho = vi.w;
        ax = (pax + vax) * inv_rho;
        ay = (pay + vay) * inv_rho;
        az = (paz + vaz) * inv_rho;
        vx += ax * ep.dt;
        vy += ay * ep.dt;
        vz += az * ep.dt;
    }
    const uint32_t i = sorted_idx[s];
    if (EPI == 0) {
        out.vx[i] = vx;
        out.vy[i] = vy;
        out.vz[i] = vz;
        if (out.ax != nullptr) {
            out.ax[i] = ax;
            out.ay[i] = ay;
            out.az[i] = az;
        }
    } else {
        // GravityModule: gravity.rs:31-34.
        if (ep.flags & 1u) {
            vx += ep.gx * ep.dt;
            vy += ep.gy * ep.dt;
            vz += ep.gz * ep.dt;
        }
        float x = pi.x, y = pi.y, z = pi.z;
        // IntegrateModule: integrate.rs:16-31.
        if (ep.flags & 2u) {
            if (!isfinite(vx)) vx = 0.f;
            if (!isfinite(vy)) vy = 0.f;
            if (!isfinite(vz)) vz = 0.f;
            x += vx * ep.dt;
            y += vy * ep.dt;
            z += vz * ep.dt;
        }
        // BoxColliderModule: box_collider.rs:36-46.
        if (ep.flags & 4u) {
            const float e = ep.restitution;
            if (x < ep.bmin[0]) { x = ep.bmin[0]; vx = fabsf(vx) * e; }
            if (x > ep.bmax[0]) { x = ep.bmax[0]; vx = -fabsf(vx) * e; }
            if (y < ep.bmin[1]) { y = ep.bmin[1]; vy = fabsf(vy) * e; }
            if (y > ep.bmax[1]) { y = ep.bmax[1]; vy = -fabsf(vy) * e; }
            if (z < ep.bmin[2]) { z = ep.bmin[2]; vz = fabsf(vz) * e; }
            if (z > ep.bmax[2]) { z = ep.bmax[2]; vz = -fabsf(vz) * e; }
        }
        out.px[i] = x;
        out.py[i] = y;
        out.pz[i] = z;
        out.vx[i] = vx;
        out.vy[i] = vy;
        out.vz[i] = vz;
    }
}

}  // namespace sph
}  // namespace forge
