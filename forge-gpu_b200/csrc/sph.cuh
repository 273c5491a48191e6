// SPH neighbour passes (sm_100a): poly6 density and the fused spiky-pressure
// + viscosity-Laplacian force with the manifest step epilogue.
//
// Data layout (HBM): particles live in the caller's SoA arrays in ORIGINAL
// order. After the grid build the library holds cell-ordered copies
//   pos4[s] = (x, y, z, bits(cell key))     vel4[s] = (vx, vy, vz, rho)
// so a neighbour is one or two 16-byte loads, and for each (dz, dy) the three
// cells dx = -1..1 are ONE contiguous range [cell_start[row+cx-1],
// cell_start[row+cx+2]). Walking the 9 rows dz-major, dy-minor therefore
// visits neighbours in exactly the reference order (dz, dy, dx, then
// ascending particle index inside a cell), sph_density.rs:429-458.
//
// One thread per particle in cell order: consecutive lanes sit in the same or
// adjacent cells, so a warp walks (almost) the same ranges and neighbour
// loads are warp-broadcasts served by L1. Results are scattered back to the
// original order through sorted_idx.
#pragma once

#include "common.cuh"

namespace forge {
namespace sph {

struct SphConsts {
    float h, h2;
    float mass_poly6;  // mass * 315 / (64 pi h^9)     (sph_density.rs:413-416)
    float mass;
    float k, rho0, mu;
    float spiky;     // -45 / (pi h^6)                 (sph_fused.rs:552-555)
    float visc_lap;  //  45 / (pi h^6)
};

struct Dims {
    int nx, ny, nz;
};

__device__ __forceinline__ void key_to_cell(uint32_t key, const Dims& d, int& cx, int& cy, int& cz) {
    const uint32_t t = key / (uint32_t)d.nx;
    cx = (int)(key - t * (uint32_t)d.nx);
    cy = (int)(t % (uint32_t)d.ny);
    cz = (int)(t / (uint32_t)d.ny);
}

// ---------------------------------------------------------------------------
// Density: rho_i = sum_{j: r2 < h2} m * poly6 * (h2 - r2)^3, self included.
// Writes rho into vel4[s].w (cell order, for the force pass) and, if given,
// density_out[i] (original order).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128)
    density_kernel(const float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                   const uint32_t* __restrict__ sorted_idx, uint32_t n, Dims dims, SphConsts c,
                   float4* __restrict__ vel4, float* __restrict__ density_out) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const float4 pi = pos4[s];
    int cx, cy, cz;
    key_to_cell(__float_as_uint(pi.w), dims, cx, cy, cz);
    const int x0 = max(cx - 1, 0), x1 = min(cx + 1, dims.nx - 1) + 1;
    float rho = 0.f;
    for (int dz = -1; dz <= 1; ++dz) {
        const int z = cz + dz;
        if (z < 0 || z >= dims.nz) continue;
        for (int dy = -1; dy <= 1; ++dy) {
            const int y = cy + dy;
            if (y < 0 || y >= dims.ny) continue;
            const uint32_t row = ((uint32_t)z * (uint32_t)dims.ny + (uint32_t)y) * (uint32_t)dims.nx;
            const uint32_t b = __ldg(cell_start + row + x0);
            const uint32_t e = __ldg(cell_start + row + x1);
            for (uint32_t j = b; j < e; ++j) {
                const float4 q = __ldg(pos4 + j);
                const float dx = pi.x - q.x, dy2 = pi.y - q.y, dz2 = pi.z - q.z;
                const float r2 = dx * dx + dy2 * dy2 + dz2 * dz2;
                if (r2 < c.h2) {
                    const float diff = c.h2 - r2;
                    rho += c.mass_poly6 * diff * diff * diff;
                }
            }
        }
    }
    if (vel4 != nullptr) vel4[s].w = rho;
    if (density_out != nullptr) density_out[sorted_idx[s]] = rho;
}

// ---------------------------------------------------------------------------
// Force pass. TERMS: 1 pressure, 2 viscosity, 3 both (fused). Jacobi: all
// neighbour data come from the cell-ordered snapshot (pos4, vel4), so the
// update never races with reads (fixes the in-place vx[i] += of
// sph_fused.rs:635-637 / sph_viscosity.rs:103-105).
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
    force_kernel(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                 const uint32_t* __restrict__ cell_start, const uint32_t* __restrict__ sorted_idx, uint32_t n,
                 Dims dims, SphConsts c, StepEpi ep, ForceOut out) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const float4 pi = pos4[s];
    const float4 vi = vel4[s];
    const float rho_i = vi.w;
    const bool valid = !(rho_i < 1e-6f);
    const float p_i = c.k * (rho_i - c.rho0);

    float pax = 0.f, pay = 0.f, paz = 0.f;
    float vax = 0.f, vay = 0.f, vaz = 0.f;
    if (valid) {
        int cx, cy, cz;
        key_to_cell(__float_as_uint(pi.w), dims, cx, cy, cz);
        const int x0 = max(cx - 1, 0), x1 = min(cx + 1, dims.nx - 1) + 1;
        for (int dz = -1; dz <= 1; ++dz) {
            const int z = cz + dz;
            if (z < 0 || z >= dims.nz) continue;
            for (int dy = -1; dy <= 1; ++dy) {
                const int y = cy + dy;
                if (y < 0 || y >= dims.ny) continue;
                const uint32_t row = ((uint32_t)z * (uint32_t)dims.ny + (uint32_t)y) * (uint32_t)dims.nx;
                const uint32_t b = __ldg(cell_start + row + x0);
                const uint32_t e = __ldg(cell_start + row + x1);
                for (uint32_t j = b; j < e; ++j) {
                    const float4 q = __ldg(pos4 + j);
                    const float djx = pi.x - q.x, djy = pi.y - q.y, djz = pi.z - q.z;
                    const float r2 = djx * djx + djy * djy + djz * djz;
                    if (r2 < c.h2 && r2 > 1e-12f) {
                        const float4 vj = __ldg(vel4 + j);
                        const float rho_j = vj.w;
                        if (rho_j < 1e-6f) continue;
                        // diff = h - r cancels for r close to h; recompute r2
                        // with the reference's rounding (no multiply-add
                        // contraction) so r and diff carry no extra error.
                        const float r2e = __fadd_rn(__fadd_rn(__fmul_rn(djx, djx), __fmul_rn(djy, djy)),
                                                    __fmul_rn(djz, djz));
                        const float r = sqrtf(r2e);
                        const float diff = c.h - r;
                        if (TERMS & 1) {
                            const float p_j = c.k * (rho_j - c.rho0);
                            const float grad_scale = c.spiky * diff * diff / r;
                            const float f_scale = -c.mass * (p_i + p_j) / (2.0f * rho_j) * grad_scale;
                            pax += f_scale * djx;
                            pay += f_scale * djy;
                            paz += f_scale * djz;
                        }
                        if (TERMS & 2) {
                            const float lap = c.visc_lap * diff;
                            const float v_scale = c.mu * c.mass / rho_j * lap;
                            vax += v_scale * (vj.x - vi.x);
                            vay += v_scale * (vj.y - vi.y);
                            vaz += v_scale * (vj.z - vi.z);
                        }
                    }
                }
            }
        }
    }

    // Acceleration as the reference applies it: the fused module multiplies
    // by 1/rho_i (sph_fused.rs:633-638); the single-term modules divide
    // (sph_pressure.rs:109-111, sph_viscosity.rs:103-105).
    float ax = 0.f, ay = 0.f, az = 0.f;
    if (valid) {
        if (TERMS == 3) {
            const float inv_rho = 1.0f / rho_i;
            ax = (pax + vax) * inv_rho;
            ay = (pay + vay) * inv_rho;
            az = (paz + vaz) * inv_rho;
        } else if (TERMS == 1) {
            ax = pax / rho_i;
            ay = pay / rho_i;
            az = paz / rho_i;
        } else {
            ax = vax / rho_i;
            ay = vay / rho_i;
            az = vaz / rho_i;
        }
    }
    float vx = vi.x, vy = vi.y, vz = vi.z;
    if (valid) {
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
