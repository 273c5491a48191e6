// SPH neighbour passes (sm_100a): poly6 density and the fused spiky-pressure
// + viscosity-Laplacian force with the manifest step epilogue.
//
// Data layout (HBM): particles live in the caller's SoA arrays in ORIGINAL
// order. The SPH grid build sorts them by key = cell << sub_bits | x-slice
// (each cell cut into 2^sub_bits slabs along x; ties in ascending particle
// index) and the library holds cell-ordered copies
//   pos4[s] = (x, y, z, bits(key))     after the build
//           = (x, y, z, p/rho)         after the density pass (a force-pass
//                                      neighbour's position and p_j/rho_j in
//                                      one 16-byte load; own keys then come
//                                      from the sorted keys)
//   vel4[s] = (vx, vy, vz, 1/rho)       (1/rho := 0 when rho < 1e-6)
//   aux[s]  = (p/rho, rho)              p = k (rho - rho0)
// so for each row (dz, dy) of the 3x3x3 cell block the candidates are ONE
// contiguous range of slices [lo, hi] along x. Rows are walked in the
// reference order (dz, dy); inside a row the candidates come in slice order
// instead of the reference's (dx, index) order, so sums agree with the
// reference to rounding, not bit for bit.
//
// Per particle and row the slice range is trimmed to the x-extent that can
// hold a point with r^2 < h^2: w = sqrt(h^2 (1 + 1e-4) - gap_y^2 - gap_z^2)
// around the particle, gaps shrunk by a rounding slack, clipped to the
// reference's 3-cell window; a row whose (y, z) gap alone exceeds h is
// skipped. Every pair with r^2 < h^2 is still visited.
//
// Two consecutive particles per thread share neighbour loads: same row ->
// one walk over the union of their windows (a candidate outside one particle's
// window is > h from it when cell size >= h, and adds nothing); otherwise two
// walks. Results are scattered back to the original order through sorted_idx.
//
// Both passes are bound by instruction issue and L1 wavefronts, not HBM, so
// the kernels minimise instructions per candidate: the density sum is
// branchless, and the force pass first scans a chunk of 32 candidates for
// r^2 < h^2 (cheap) and then evaluates the expensive pair term only for the
// hits, with per-particle reciprocals instead of per-pair divides.
#pragma once

#include "common.cuh"

namespace forge {
namespace sph {

// floorf + saturating convert (NaN -> 0), as the cell hash does.
__device__ __forceinline__ int floor_to_int_dev(float v) { return (int)floorf(v); }

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
    int sub_bits;   // x-slices per cell = 2^sub_bits (keys are cell << sub_bits | slice)
    int pairable;   // cs >= h: a walk over a same-row neighbour's window adds only r >= h pairs
    float inv_slice;   // 2^sub_bits / cs (rounded: window bounds carry a margin for it)
    int x_off;         // first slice of the grid's x-window: cx0 << sub_bits (nx is the window's width)
    FastDiv row_len;   // nx << sub_bits: key -> (row, slice in row)
    FastDiv ny_div;    // ny: row -> (cy, cz)
    const uint32_t* __restrict__ keys;  // cell keys in cell order (a particle's own key: its frame)
};

// Cell-ordered position of particle s with w = bits(its cell key), for the
// force pass. pos4.w holds the key from the grid build (the density pass
// reads its own particles' keys there) until the density pass replaces it
// with p/rho (the force pass's neighbour data: one 16-byte load gives a
// neighbour's position and p_j/rho_j), so the force pass takes a particle's
// own key from the sorted keys. Every density pass follows a build.
__device__ __forceinline__ float4 own_pos(const float4* __restrict__ pos4, const Geom& g, uint32_t s) {
    float4 p = pos4[s];
    p.w = __uint_as_float(__ldg(g.keys + s));
    return p;
}

// Squared conservative gap: distance shrunk by a slack covering the rounding
// of the cell assignment and of r^2, clamped at 0 (clamped out-of-grid
// particles give negative raw gaps -> 0, i.e. never skipped).
__device__ __forceinline__ float gap2(float raw, float slack) {
    const float g = fmaxf(raw - slack, 0.f);
    return g * g;
}

// A particle's place in the grid and what its row windows are built from.
struct Frame {
    int cy, cz;
    int fx_lo, fx_hi;   // x-slice range of the reference window: cells cx-1..cx+1, clamped to the grid
    int f_own;          // own x-slice index in the row
    float fxs;          // (x - ox) / cs * 2^sub_bits   (global slice coordinate: windows round
                        // the same whatever the grid's x-window)
    float slack;        // slice-units rounding slack
    float gyl, gyr, gzl, gzr;  // squared gaps to the neighbouring rows
};

__device__ __forceinline__ Frame make_frame(const float4& p, const Geom& g) {
    Frame f;
    const uint32_t key = __float_as_uint(p.w);
    const uint32_t S = 1u << g.sub_bits;
    const uint32_t t = fast_div(key, g.row_len);
    f.f_own = (int)(key - t * g.row_len.d);
    const uint32_t tz = fast_div(t, g.ny_div);
    f.cy = (int)(t - tz * g.ny_div.d);
    f.cz = (int)tz;
    const int cx = f.f_own >> g.sub_bits;
    f.fx_lo = max(cx - 1, 0) * (int)S;
    f.fx_hi = (min(cx + 1, g.nx - 1) + 1) * (int)S - 1;
    f.fxs = (p.x - g.ox) * g.inv_slice;
    // rounding of the cell assignment and of r^2, plus 1e-3 slices for the
    // rounded reciprocal and the approximate square root of row_window
    f.slack = 4e-7f * (fabsf(f.fxs) + 2.f * (float)S) + 1e-3f;
    const float by = g.oy + (float)f.cy * g.cs, bz = g.oz + (float)f.cz * g.cs;
    const float sy = 4e-7f * (fabsf(p.y) + fabsf(by) + g.cs);
    const float sz = 4e-7f * (fabsf(p.z) + fabsf(bz) + g.cs);
    f.gyl = gap2(p.y - by, sy);
    f.gyr = gap2(by + g.cs - p.y, sy);
    f.gzl = gap2(p.z - bz, sz);
    f.gzr = gap2(bz + g.cs - p.z, sz);
    return f;
}

// Window of row r = (dz+1)*3 + (dy+1) as an inclusive x-slice range
// [lo, hi]: the slices that can hold a point with r^2 < h^2, i.e. whose x
// lies within w = sqrt(H - gap_y^2 - gap_z^2) of the particle, clipped to the
// reference's 3-cell window and always containing the particle's own slice
// (clamped out-of-grid particles). false: the row is skipped.
__device__ __forceinline__ bool row_window(const Frame& f, int r, const Geom& g, float H, int& lo, int& hi) {
    const int dz = r / 3 - 1, dy = r % 3 - 1;
    const int z = f.cz + dz, y = f.cy + dy;
    if (z < 0 || z >= g.nz || y < 0 || y >= g.ny) return false;
    const float base = (dz < 0 ? f.gzl : (dz > 0 ? f.gzr : 0.f)) + (dy < 0 ? f.gyl : (dy > 0 ? f.gyr : 0.f));
    if (base > H) return false;
    const float w = sqrt_approx(H - base) * g.inv_slice + f.slack;
    lo = max(min(floor_to_int_dev(f.fxs - w) - g.x_off, f.f_own), f.fx_lo);
    hi = min(max(floor_to_int_dev(f.fxs + w) - g.x_off, f.f_own), f.fx_hi);
    return true;
}

__device__ __forceinline__ uint32_t row_base(const Geom& g, const Frame& f, int r) {
    const int dz = r / 3 - 1, dy = r % 3 - 1;
    return ((uint32_t)(f.cz + dz) * (uint32_t)g.ny + (uint32_t)(f.cy + dy)) * ((uint32_t)g.nx << g.sub_bits);
}

// Calls f(b, e) for each trimmed contiguous candidate range of particle p
// (cell-ordered indices), rows in the reference order (dz, dy).
template <class F>
__device__ __forceinline__ void for_each_range(const float4& p, const Geom& g, const uint32_t* __restrict__ cell_start,
                                               float H, F&& fn) {
    const Frame f = make_frame(p, g);
#pragma unroll 1
    for (int r = 0; r < 9; ++r) {
        int lo, hi;
        if (!row_window(f, r, g, H, lo, hi)) continue;
        const uint32_t row = row_base(g, f, r);
        fn(__ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1));
    }
}

// Union of two windows of the same row (either may be absent).
__device__ __forceinline__ bool union_window(bool a, int alo, int ahi, bool b, int blo, int bhi, int& lo, int& hi) {
    if (!a && !b) return false;
    lo = a ? (b ? min(alo, blo) : alo) : blo;
    hi = a ? (b ? max(ahi, bhi) : ahi) : bhi;
    return true;
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
// max(h^2 - r^2, 0) as three FMAs (h^2 - dx^2 - dy^2 - dz^2): the poly6
// base of a pair, exactly +0 outside h. The sums below accumulate base^3 and
// are scaled by m * poly6 once per particle (the reference scales each term;
// the difference is fp32 rounding, inside the density tolerance).
__device__ __forceinline__ float poly6_base(const float4& p, const float4& q, float h2) {
    const float dx = p.x - q.x, dy = p.y - q.y, dz = p.z - q.z;
    return fmaxf(fmaf(-dz, dz, fmaf(-dy, dy, fmaf(-dx, dx, h2))), 0.f);
}

// Poly6 contributions of candidates [b, e) to one or two particles.
__device__ __forceinline__ void poly6_one(const float4* __restrict__ pos4, uint32_t b, uint32_t e, const float4& p,
                                          const SphConsts& c, float& rho) {
#pragma unroll 4
    for (uint32_t j = b; j < e; ++j) {
        const float4 q = __ldg(pos4 + j);
        const float d = poly6_base(p, q, c.h2);
        rho = fmaf(d * d, d, rho);
    }
}

__device__ __forceinline__ void poly6_two(const float4* __restrict__ pos4, uint32_t b, uint32_t e, const float4& p0,
                                          const float4& p1, const SphConsts& c, float& rho0, float& rho1) {
#pragma unroll 2
    for (uint32_t j = b; j < e; ++j) {
        const float4 q = __ldg(pos4 + j);
        const float d0 = poly6_base(p0, q, c.h2);
        const float d1 = poly6_base(p1, q, c.h2);
        rho0 = fmaf(d0 * d0, d0, rho0);
        rho1 = fmaf(d1 * d1, d1, rho1);
    }
}

// Density, two consecutive cell-ordered particles per thread: each neighbour
// load feeds two pair evaluations (the one-particle walk is bound by L1
// wavefronts, not arithmetic). Same cell: walk the union of both trimmed
// windows -- every extra candidate lies in the other particle's untrimmed
// window and was trimmed only because it cannot be within h, so it adds +0,
// exactly as in the reference. Adjacent cells of one row: walk three
// segments (first only, both, second only) of their ordered ranges.
// Different rows: two single walks. Each particle's sum keeps the reference
// order.
#ifndef FORGE_DENSITY_MIN_BLOCKS
#define FORGE_DENSITY_MIN_BLOCKS 10  // 48 registers (a few spills): 10 blocks per SM
#endif
#ifndef FORGE_FORCE_MIN_BLOCKS
#define FORGE_FORCE_MIN_BLOCKS 8  // 64 registers: 8 blocks per SM (the spills cost less than the occupancy gains)
#endif

__global__ void __launch_bounds__(128, FORGE_DENSITY_MIN_BLOCKS)
    density_pair_kernel(float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                        const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c,
                        float4* __restrict__ vel4, float2* __restrict__ aux, float* __restrict__ density_out) {
    pdl_enter();
    const uint32_t s0 = 2u * (blockIdx.x * blockDim.x + threadIdx.x);
    if (s0 >= n) return;
    const bool has1 = s0 + 1 < n;
    const float4 p0 = pos4[s0];
    const float4 p1 = has1 ? pos4[s0 + 1] : p0;
    const Frame f0 = make_frame(p0, g);
    const Frame f1 = make_frame(p1, g);
    float rho0 = 0.f, rho1 = 0.f;
    if (has1 && g.pairable && f0.cy == f1.cy && f0.cz == f1.cz) {
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int l0, h0, l1, h1, lo, hi;
            const bool a = row_window(f0, r, g, c.h2_skip, l0, h0);
            const bool b = row_window(f1, r, g, c.h2_skip, l1, h1);
            if (!union_window(a, l0, h0, b, l1, h1, lo, hi)) continue;
            const uint32_t row = row_base(g, f0, r);
            poly6_two(pos4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), p0, p1, c, rho0, rho1);
        }
    } else {
        for_each_range(p0, g, cell_start, c.h2_skip,
                       [&](uint32_t b, uint32_t e) { poly6_one(pos4, b, e, p0, c, rho0); });
        if (has1)
            for_each_range(p1, g, cell_start, c.h2_skip,
                           [&](uint32_t b, uint32_t e) { poly6_one(pos4, b, e, p1, c, rho1); });
    }
    rho0 *= c.mass_poly6;
    rho1 *= c.mass_poly6;
    float inv_rho;
    float2 a;
    density_derived(rho0, c, inv_rho, a);
    if (vel4 != nullptr) {
        vel4[s0].w = inv_rho;
        aux[s0] = a;
        pos4[s0] = make_float4(p0.x, p0.y, p0.z, a.x);
    }
    if (density_out != nullptr) density_out[sorted_idx[s0]] = rho0;
    if (has1) {
        density_derived(rho1, c, inv_rho, a);
        if (vel4 != nullptr) {
            vel4[s0 + 1].w = inv_rho;
            aux[s0 + 1] = a;
            pos4[s0 + 1] = make_float4(p1.x, p1.y, p1.z, a.x);
        }
        if (density_out != nullptr) density_out[sorted_idx[s0 + 1]] = rho1;
    }
}

// Density, P consecutive cell-ordered particles per thread: when all lie in
// one grid row (and cell size >= h), one walk over the union of their
// windows feeds P pair evaluations per neighbour load (extra candidates add
// exactly +0, as in the two-particle kernel); otherwise P single walks.
#ifndef FORGE_MULTI_MIN_BLOCKS
#define FORGE_MULTI_MIN_BLOCKS 8  // at most 64 registers: 8 blocks per SM
#endif
template <int P>
__global__ void __launch_bounds__(128, FORGE_MULTI_MIN_BLOCKS)
    density_multi_kernel(float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                         const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c,
                         float4* __restrict__ vel4, float2* __restrict__ aux, float* __restrict__ density_out) {
    pdl_enter();
    const uint32_t s0 = P * (blockIdx.x * blockDim.x + threadIdx.x);
    if (s0 >= n) return;
    const uint32_t np = min((uint32_t)P, n - s0);
    float4 p[P];
    float rho[P];
    bool together = g.pairable != 0;
    const Frame f0 = make_frame(p[0] = pos4[s0], g);
#pragma unroll
    for (int k = 1; k < P; ++k) {
        p[k] = (uint32_t)k < np ? pos4[s0 + k] : p[0];
        const Frame fk = make_frame(p[k], g);
        together = together && fk.cy == f0.cy && fk.cz == f0.cz;
    }
#pragma unroll
    for (int k = 0; k < P; ++k) rho[k] = 0.f;
    if (together) {
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int lo = 0x7fffffff, hi = -1;
#pragma unroll
            for (int k = 0; k < P; ++k) {
                int l, h;
                if (row_window(make_frame(p[k], g), r, g, c.h2_skip, l, h)) {
                    lo = min(lo, l);
                    hi = max(hi, h);
                }
            }
            if (lo > hi) continue;
            const uint32_t row = row_base(g, f0, r);
            const uint32_t b = __ldg(cell_start + row + lo), e = __ldg(cell_start + row + hi + 1);
#pragma unroll 2
            for (uint32_t j = b; j < e; ++j) {
                const float4 q = __ldg(pos4 + j);
#pragma unroll
                for (int k = 0; k < P; ++k) {
                    const float d = poly6_base(p[k], q, c.h2);
                    rho[k] = fmaf(d * d, d, rho[k]);
                }
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < P; ++k)
            if ((uint32_t)k < np)
                for_each_range(p[k], g, cell_start, c.h2_skip,
                               [&](uint32_t b, uint32_t e) { poly6_one(pos4, b, e, p[k], c, rho[k]); });
    }
#pragma unroll
    for (int k = 0; k < P; ++k) {
        if ((uint32_t)k >= np) break;
        const float r = rho[k] * c.mass_poly6;
        float inv_rho;
        float2 a;
        density_derived(r, c, inv_rho, a);
        if (vel4 != nullptr) {
            vel4[s0 + k].w = inv_rho;
            aux[s0 + k] = a;
            pos4[s0 + k] = make_float4(p[k].x, p[k].y, p[k].z, a.x);
        }
        if (density_out != nullptr) density_out[sorted_idx[s0 + k]] = r;
    }
}

// vel4[s] = (vx[i], vy[i], vz[i], 1/rho[i]), aux[s] = (p/rho, rho), i = svals[s]
// (forge_sph_force with a caller-supplied density).
__global__ void __launch_bounds__(256)
    gather_vel_rho_kernel(const uint32_t* __restrict__ svals, uint32_t n, const float* __restrict__ vx,
                          const float* __restrict__ vy, const float* __restrict__ vz,
                          const float* __restrict__ rho, SphConsts c, float4* __restrict__ vel4,
                          float2* __restrict__ aux, float4* __restrict__ pos4) {
    pdl_enter();
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const uint32_t i = svals[s];
    float inv_rho;
    float2 a;
    density_derived(rho[i], c, inv_rho, a);
    vel4[s] = make_float4(vx[i], vy[i], vz[i], inv_rho);
    aux[s] = a;
    pos4[s].w = a.x;
}

// Re-derives 1/rho, p/rho and rho of the ghosts (original index >= limit)
// from density[] after their owners' values arrived.
__global__ void __launch_bounds__(256)
    ghost_rho_kernel(const uint32_t* __restrict__ svals, uint32_t n, uint32_t limit, const float* __restrict__ rho,
                     SphConsts c, float4* __restrict__ vel4, float2* __restrict__ aux, float4* __restrict__ pos4) {
    pdl_enter();
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const uint32_t i = svals[s];
    if (i < limit) return;
    float inv_rho;
    float2 a;
    density_derived(rho[i], c, inv_rho, a);
    vel4[s].w = inv_rho;
    aux[s] = a;
    pos4[s].w = a.x;
}

// ---------------------------------------------------------------------------
// Force pass. TERMS: 1 pressure, 2 viscosity, 3 both (fused). Jacobi: all
// neighbour data come from the cell-ordered snapshot (pos4 with p/rho in w,
// vel4 with 1/rho in w; aux holds each particle's own rho), so
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
    uint32_t limit;  // only particles with original index < limit are written
    // Interior pass of a zoned step (zone == 2): a particle whose x before
    // or after the step lies below glo or at/above ghi sets kDevZone in
    // *status (it is, or moved, too close to a face for the overlapped
    // exchange).
    uint32_t zone = 0;
    float glo = 0.f, ghi = 0.f;
    uint32_t* status = nullptr;
};

// Sorted positions of one zone of a zoned force pass: list `list` (1 =
// boundary, 2 = interior) of a classification [A | L | R] with device-side
// sizes counts[3].
struct ZoneList {
    const uint32_t* idx = nullptr;
    const uint32_t* counts = nullptr;
    uint32_t list = 0;
};

// Zone lists from the cell-start table. With keys cell << sub_bits | slice
// and x the fastest cell axis, each grid row (cy, cz) is one run of the
// cell order, and the interior zone -- x-slices [k_lo, k_hi) of the row --
// one contiguous piece of it: per row, boundary = [b0, i0) u [i1, e),
// interior = [i0, i1). Lists come out in the cell order (row by row), so
// consecutive entries are mostly neighbours in the same row.
constexpr int kZoneRows = 256;  // rows per block (one per thread)

struct ZoneRows {
    const uint32_t* __restrict__ cell_start;
    uint32_t rows;     // ny * nz
    uint32_t row_len;  // table entries per row: nx << sub_bits
    uint32_t k_lo, k_hi;
    __device__ __forceinline__ void seg(uint32_t r, uint32_t& b0, uint32_t& i0, uint32_t& i1, uint32_t& e) const {
        const uint32_t* t = cell_start + (size_t)r * row_len;
        b0 = __ldg(t);
        i0 = __ldg(t + k_lo);
        i1 = __ldg(t + k_hi);
        e = __ldg(t + row_len);
    }
};

// Per-tile sums of the boundary and interior lengths (tile_counts[t*3 + 1],
// [t*3 + 2]; [t*3] = 0), in the layout slab::classify_scan_kernel scans.
__global__ void __launch_bounds__(kZoneRows) zone_rows_count_kernel(ZoneRows z, uint32_t* __restrict__ tile_counts) {
    pdl_enter();
    __shared__ uint32_t s[2];
    if (threadIdx.x < 2) s[threadIdx.x] = 0;
    __syncthreads();
    const uint32_t r = blockIdx.x * kZoneRows + threadIdx.x;
    uint32_t lb = 0, li = 0;
    if (r < z.rows) {
        uint32_t b0, i0, i1, e;
        z.seg(r, b0, i0, i1, e);
        lb = (i0 - b0) + (e - i1);
        li = i1 - i0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lb += __shfl_xor_sync(0xffffffffu, lb, o);
        li += __shfl_xor_sync(0xffffffffu, li, o);
    }
    if ((threadIdx.x & 31) == 0) {
        if (lb) atomicAdd(&s[0], lb);
        if (li) atomicAdd(&s[1], li);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        tile_counts[blockIdx.x * 3 + 0] = 0;
        tile_counts[blockIdx.x * 3 + 1] = s[0];
        tile_counts[blockIdx.x * 3 + 2] = s[1];
    }
}

// Writes the lists [A (empty) | boundary | interior] of sorted positions.
__global__ void __launch_bounds__(kZoneRows)
    zone_rows_write_kernel(ZoneRows z, const uint32_t* __restrict__ tile_offsets, const uint32_t* __restrict__ counts,
                           uint32_t* __restrict__ out) {
    pdl_enter();
    __shared__ uint32_t s_scan[kZoneRows / 32 + 1];
    __shared__ uint32_t s_seg[kZoneRows][6];
    const uint32_t r = blockIdx.x * kZoneRows + threadIdx.x;
    uint32_t b0 = 0, i0 = 0, i1 = 0, e = 0;
    if (r < z.rows) z.seg(r, b0, i0, i1, e);
    uint32_t total;
    const uint32_t ob = block_exclusive_scan<kZoneRows>((i0 - b0) + (e - i1), s_scan, &total) +
                        tile_offsets[blockIdx.x * 3 + 1] + counts[0];
    const uint32_t oi = block_exclusive_scan<kZoneRows>(i1 - i0, s_scan, &total) + tile_offsets[blockIdx.x * 3 + 2] +
                        counts[0] + counts[1];
    s_seg[threadIdx.x][0] = b0;
    s_seg[threadIdx.x][1] = i0;
    s_seg[threadIdx.x][2] = i1;
    s_seg[threadIdx.x][3] = e;
    s_seg[threadIdx.x][4] = ob;
    s_seg[threadIdx.x][5] = oi;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nrows = min((uint32_t)kZoneRows, z.rows - blockIdx.x * kZoneRows);
    for (uint32_t q = warp; q < nrows; q += kZoneRows / 32) {
        const uint32_t qb0 = s_seg[q][0], qi0 = s_seg[q][1], qi1 = s_seg[q][2], qe = s_seg[q][3];
        const uint32_t qob = s_seg[q][4], qoi = s_seg[q][5];
        const uint32_t la = qi0 - qb0;
        for (uint32_t j = lane; j < la; j += 32) out[qob + j] = qb0 + j;
        for (uint32_t j = lane; j < qe - qi1; j += 32) out[qob + la + j] = qi1 + j;
        for (uint32_t j = lane; j < qi1 - qi0; j += 32) out[qoi + j] = qi0 + j;
    }
}

struct StepOp {
    uint32_t kind;  // FORGE_OP_*
    float p[7];
};

struct StepEpi {
    float dt;
    float gx, gy, gz;
    float bmin[3], bmax[3];
    float restitution;
    uint32_t flags;  // FORGE_STEP_* bits (used when n_ops == 0)
    uint32_t n_ops;
    StepOp ops[8];
};

// BoxColliderModule: box_collider.rs:36-46.
__device__ __forceinline__ void box_op(float& x, float& y, float& z, float& vx, float& vy, float& vz, const float* mn,
                                       const float* mx, float e) {
    if (x < mn[0]) { x = mn[0]; vx = fabsf(vx) * e; }
    if (x > mx[0]) { x = mx[0]; vx = -fabsf(vx) * e; }
    if (y < mn[1]) { y = mn[1]; vy = fabsf(vy) * e; }
    if (y > mx[1]) { y = mx[1]; vy = -fabsf(vy) * e; }
    if (z < mn[2]) { z = mn[2]; vz = fabsf(vz) * e; }
    if (z > mx[2]) { z = mx[2]; vz = -fabsf(vz) * e; }
}

// The manifest modules after the SPH module, in list order.
__device__ __forceinline__ void apply_ops(const StepEpi& ep, float& x, float& y, float& z, float& vx, float& vy,
                                          float& vz) {
    const float dt = ep.dt;
    for (uint32_t k = 0; k < ep.n_ops; ++k) {
        const StepOp& o = ep.ops[k];
        switch (o.kind) {
            case 1u:  // gravity.rs:31-34
                vx += o.p[0] * dt;
                vy += o.p[1] * dt;
                vz += o.p[2] * dt;
                break;
            case 2u: {  // drag.rs:18-20
                const float d = 1.0f - o.p[0] * dt;
                vx *= d;
                vy *= d;
                vz *= d;
                break;
            }
            case 3u:  // integrate.rs:16-31
                if (!isfinite(vx)) vx = 0.f;
                if (!isfinite(vy)) vy = 0.f;
                if (!isfinite(vz)) vz = 0.f;
                x += vx * dt;
                y += vy * dt;
                z += vz * dt;
                break;
            case 4u:  // ground_plane.rs:19-21
                if (y < o.p[0]) {
                    y = o.p[0];
                    vy = -vy * o.p[1];
                }
                break;
            case 5u: {  // sphere_collider.rs:22-41
                const float dx = x - o.p[0], dy = y - o.p[1], dz = z - o.p[2];
                const float dist = sqrtf(dx * dx + dy * dy + dz * dz);
                const float r = o.p[3];
                if (dist < r && dist > 1e-8f) {
                    const float inv = 1.0f / dist;
                    const float nx = dx * inv, ny = dy * inv, nz = dz * inv;
                    x = o.p[0] + nx * r;
                    y = o.p[1] + ny * r;
                    z = o.p[2] + nz * r;
                    const float vn = vx * nx + vy * ny + vz * nz;
                    if (vn < 0) {
                        vx -= (1 + o.p[4]) * vn * nx;
                        vy -= (1 + o.p[4]) * vn * ny;
                        vz -= (1 + o.p[4]) * vn * nz;
                    }
                }
                break;
            }
            case 6u:  // box_collider.rs:36-46
                box_op(x, y, z, vx, vy, vz, &o.p[0], &o.p[3], o.p[6]);
                break;
            default:
                break;
        }
    }
}

// One particle's state in the force pass.
struct ForceAcc {
    float4 p;   // position, w = bits(cell key)
    float4 v;   // velocity, w = 1/rho
    float pres; // p_i = k (rho_i - rho0)
    float pax, pay, paz, vax, vay, vaz;
};

__device__ __forceinline__ ForceAcc force_acc(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                                              const float2* __restrict__ aux, uint32_t s, const SphConsts& c,
                                              const Geom& g) {
    ForceAcc A;
    A.p = own_pos(pos4, g, s);
    A.v = vel4[s];
    A.pres = c.k * (aux[s].y - c.rho0);
    A.pax = A.pay = A.paz = A.vax = A.vay = A.vaz = 0.f;
    return A;
}

__device__ __forceinline__ uint32_t in_range_bit(const float4& p, const float4& q, const SphConsts& c, uint32_t k) {
    const float dx = p.x - q.x, dy = p.y - q.y, dz = p.z - q.z;
    const float r2 = fmaf(dz, dz, fmaf(dy, dy, dx * dx));
    return (r2 < c.h2 && r2 > 1e-12f) ? (1u << k) : 0u;
}

// Pressure and viscosity terms of one pair (neighbour position q, velocity
// and 1/rho vj, p_j/rho_j pjr) added to A.
template <int TERMS>
__device__ __forceinline__ void force_term(const float4& q, const float4& vj, float pjr, ForceAcc& A,
                                           const SphConsts& c) {
    const float djx = A.p.x - q.x, djy = A.p.y - q.y, djz = A.p.z - q.z;
    const float r2 = __fadd_rn(__fadd_rn(__fmul_rn(djx, djx), __fmul_rn(djy, djy)), __fmul_rn(djz, djz));
    const float diff = c.h - sqrtf(r2);
    const float inv_rho_j = vj.w;
    if (TERMS & 1) {
        const float pp = fmaf(A.pres, inv_rho_j, pjr);
        const float f = c.kp * pp * (diff * diff) * rsqrtf(r2);
        A.pax = fmaf(f, djx, A.pax);
        A.pay = fmaf(f, djy, A.pay);
        A.paz = fmaf(f, djz, A.paz);
    }
    if (TERMS & 2) {
        const float v = c.kv * inv_rho_j * diff;
        A.vax = fmaf(v, vj.x - A.v.x, A.vax);
        A.vay = fmaf(v, vj.y - A.v.y, A.vay);
        A.vaz = fmaf(v, vj.z - A.v.z, A.vaz);
    }
}

// Pair terms of the hits (bit k = candidate j0 + k), ascending j.
template <int TERMS>
__device__ __forceinline__ void force_hits(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                                           uint32_t j0, uint32_t hit,
                                           ForceAcc& A, const SphConsts& c) {
    while (hit) {
        const uint32_t j = j0 + (uint32_t)(__ffs(hit) - 1);
        hit &= hit - 1;
        // both loads issued together (one latency per hit)
        const float4 q = __ldg(pos4 + j);
        const float4 vj = __ldg(vel4 + j);
        force_term<TERMS>(q, vj, q.w, A, c);  // q.w = p_j / rho_j
    }
}

// Candidates [b, e) for one particle: scan 32 at a time for r^2 < h^2, then
// evaluate only the hits.
template <int TERMS>
__device__ __forceinline__ void force_one(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                                          uint32_t b, uint32_t e, ForceAcc& A,
                                          const SphConsts& c) {
    for (uint32_t j0 = b; j0 < e; j0 += 32) {
        const uint32_t cnt = min(32u, e - j0);
        uint32_t hit = 0;
#pragma unroll 4
        for (uint32_t k = 0; k < cnt; ++k) hit |= in_range_bit(A.p, __ldg(pos4 + j0 + k), c, k);
        force_hits<TERMS>(pos4, vel4, j0, hit, A, c);
    }
}

// Candidates [b, e) for two particles: one load per candidate in the scan.
template <int TERMS>
__device__ __forceinline__ void force_two(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                                          uint32_t b, uint32_t e, ForceAcc& A,
                                          ForceAcc& B, const SphConsts& c) {
    for (uint32_t j0 = b; j0 < e; j0 += 32) {
        const uint32_t cnt = min(32u, e - j0);
        uint32_t ha = 0, hb = 0;
#pragma unroll 2
        for (uint32_t k = 0; k < cnt; ++k) {
            const float4 q = __ldg(pos4 + j0 + k);
            ha |= in_range_bit(A.p, q, c, k);
            hb |= in_range_bit(B.p, q, c, k);
        }
        force_hits<TERMS>(pos4, vel4, j0, ha, A, c);
        force_hits<TERMS>(pos4, vel4, j0, hb, B, c);
    }
}

// a = (a_p + a_v) / rho_i (sph_fused.rs:633-638), then the velocity update
// or the manifest step epilogue, written in original order.
template <int EPI>
__device__ __forceinline__ void force_finish(const ForceAcc& A, uint32_t i, const StepEpi& ep, const ForceOut& out) {
    if (i >= out.limit) return;
    float ax = 0.f, ay = 0.f, az = 0.f;
    float vx = A.v.x, vy = A.v.y, vz = A.v.z;
    const float inv_rho = A.v.w;
    if (inv_rho != 0.f) {  // rho_i >= 1e-6 (sph_fused.rs:550)
        ax = (A.pax + A.vax) * inv_rho;
        ay = (A.pay + A.vay) * inv_rho;
        az = (A.paz + A.vaz) * inv_rho;
        vx += ax * ep.dt;
        vy += ay * ep.dt;
        vz += az * ep.dt;
    }
    if (EPI == 0) {
        out.vx[i] = vx;
        out.vy[i] = vy;
        out.vz[i] = vz;
        if (out.ax != nullptr) {
            out.ax[i] = ax;
            out.ay[i] = ay;
            out.az[i] = az;
        }
        return;
    }
    float x = A.p.x, y = A.p.y, z = A.p.z;
    if (ep.n_ops) {
        apply_ops(ep, x, y, z, vx, vy, vz);
    } else {
        // GravityModule: gravity.rs:31-34.
        if (ep.flags & 1u) {
            vx += ep.gx * ep.dt;
            vy += ep.gy * ep.dt;
            vz += ep.gz * ep.dt;
        }
        // IntegrateModule: integrate.rs:16-31.
        if (ep.flags & 2u) {
            if (!isfinite(vx)) vx = 0.f;
            if (!isfinite(vy)) vy = 0.f;
            if (!isfinite(vz)) vz = 0.f;
            x += vx * ep.dt;
            y += vy * ep.dt;
            z += vz * ep.dt;
        }
        if (ep.flags & 4u) box_op(x, y, z, vx, vy, vz, ep.bmin, ep.bmax, ep.restitution);
    }
    if (out.zone == 2 && (x < out.glo || x >= out.ghi || A.p.x < out.glo || A.p.x >= out.ghi))
        atomicOr(out.status, kDevZone);
    out.px[i] = x;
    out.py[i] = y;
    out.pz[i] = z;
    out.vx[i] = vx;
    out.vy[i] = vy;
    out.vz[i] = vz;
}

// Force pass, one particle per thread (dense cells, where the hit loop
// dominates and a second particle would only add divergence).
template <int TERMS, int EPI>
__device__ __forceinline__ void force_single_at(uint32_t s, const float4* __restrict__ pos4,
                                                const float4* __restrict__ vel4, const float2* __restrict__ aux,
                                                const uint32_t* __restrict__ cell_start,
                                                const uint32_t* __restrict__ sorted_idx, const Geom& g,
                                                const SphConsts& c, const StepEpi& ep, const ForceOut& out) {
    const uint32_t i = sorted_idx[s];
    if (i >= out.limit) return;  // not updated (a ghost of a sharded run)
    ForceAcc A = force_acc(pos4, vel4, aux, s, c, g);
    if (A.v.w != 0.f) {
        const Frame f = make_frame(A.p, g);
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int lo, hi;
            if (!row_window(f, r, g, c.h2_skip, lo, hi)) continue;
            const uint32_t row = row_base(g, f, r);
            force_one<TERMS>(pos4, vel4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), A, c);
        }
    }
    force_finish<EPI>(A, i, ep, out);
}

// Two cell-ordered particles s0, s1 (s1 valid if has1) with the same window
// logic as density_pair_kernel (union walk when both lie in one row, two
// single walks otherwise). NEAR: the two need not be adjacent in the cell
// order (zone lists), so the union walk also requires their cells to be at
// most two apart. A particle with rho < 1e-6 (1/rho stored as 0) walks
// nothing and keeps its velocity.
template <int TERMS, int EPI, bool NEAR>
__device__ __forceinline__ void force_pair_at(uint32_t s0, uint32_t s1, bool has1, const float4* __restrict__ pos4,
                                              const float4* __restrict__ vel4, const float2* __restrict__ aux,
                                              const uint32_t* __restrict__ cell_start,
                                              const uint32_t* __restrict__ sorted_idx, const Geom& g,
                                              const SphConsts& c, const StepEpi& ep, const ForceOut& out) {
    ForceAcc A = force_acc(pos4, vel4, aux, s0, c, g);
    ForceAcc B = force_acc(pos4, vel4, aux, has1 ? s1 : s0, c, g);
    const uint32_t i0 = sorted_idx[s0], i1 = has1 ? sorted_idx[s1] : 0xffffffffu;
    // rho < 1e-6 (1/rho stored as 0) or not updated (ghost): no walk
    const bool va = A.v.w != 0.f && i0 < out.limit, vb = has1 && B.v.w != 0.f && i1 < out.limit;
    const Frame f0 = make_frame(A.p, g);
    const Frame f1 = make_frame(B.p, g);
    const bool near = !NEAR || abs(f0.f_own - f1.f_own) <= (2 << g.sub_bits);
    if (va && vb && g.pairable && f0.cy == f1.cy && f0.cz == f1.cz && near) {
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int l0, h0, l1, h1, lo, hi;
            const bool a = row_window(f0, r, g, c.h2_skip, l0, h0);
            const bool b = row_window(f1, r, g, c.h2_skip, l1, h1);
            if (!union_window(a, l0, h0, b, l1, h1, lo, hi)) continue;
            const uint32_t row = row_base(g, f0, r);
            force_two<TERMS>(pos4, vel4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), A, B, c);
        }
    } else {
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int lo, hi;
            if (va && row_window(f0, r, g, c.h2_skip, lo, hi)) {
                const uint32_t row = row_base(g, f0, r);
                force_one<TERMS>(pos4, vel4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), A,
                                 c);
            }
        }
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            int lo, hi;
            if (vb && row_window(f1, r, g, c.h2_skip, lo, hi)) {
                const uint32_t row = row_base(g, f1, r);
                force_one<TERMS>(pos4, vel4, __ldg(cell_start + row + lo), __ldg(cell_start + row + hi + 1), B,
                                 c);
            }
        }
    }
    force_finish<EPI>(A, i0, ep, out);
    if (has1) force_finish<EPI>(B, i1, ep, out);
}

__device__ __forceinline__ const uint32_t* zone_begin(const ZoneList& z, uint32_t& cnt) {
    cnt = z.counts[z.list];
    return z.idx + z.counts[0] + (z.list == 2 ? z.counts[1] : 0u);
}

template <int TERMS, int EPI, bool LIST>
__global__ void __launch_bounds__(128)
    force_single_kernel(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                        const float2* __restrict__ aux, const uint32_t* __restrict__ cell_start,
                        const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c, StepEpi ep,
                        ForceOut out, ZoneList zl) {
    pdl_enter();
    if (!LIST) {
        const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
        if (s < n) force_single_at<TERMS, EPI>(s, pos4, vel4, aux, cell_start, sorted_idx, g, c, ep, out);
        return;
    }
    // LIST: the grid covers an upper bound of the list (its size is only on
    // the device); threads past its end leave at once
    uint32_t cnt;
    const uint32_t* lst = zone_begin(zl, cnt);
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < cnt) force_single_at<TERMS, EPI>(lst[t], pos4, vel4, aux, cell_start, sorted_idx, g, c, ep, out);
}

// Force pass, two consecutive cell-ordered particles per thread (LIST: two
// consecutive entries of a zone list).
template <int TERMS, int EPI, bool LIST>
__global__ void __launch_bounds__(128, FORGE_FORCE_MIN_BLOCKS)
    force_kernel(const float4* __restrict__ pos4, const float4* __restrict__ vel4, const float2* __restrict__ aux,
                 const uint32_t* __restrict__ cell_start, const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g,
                 SphConsts c, StepEpi ep, ForceOut out, ZoneList zl) {
    pdl_enter();
    if (!LIST) {
        const uint32_t s0 = 2u * (blockIdx.x * blockDim.x + threadIdx.x);
        if (s0 < n)
            force_pair_at<TERMS, EPI, false>(s0, s0 + 1, s0 + 1 < n, pos4, vel4, aux, cell_start, sorted_idx, g, c,
                                             ep, out);
        return;
    }
    uint32_t cnt;
    const uint32_t* lst = zone_begin(zl, cnt);
    const uint32_t t = 2u * (blockIdx.x * blockDim.x + threadIdx.x);
    if (t < cnt) {
        const bool has1 = t + 1 < cnt;
        force_pair_at<TERMS, EPI, true>(lst[t], has1 ? lst[t + 1] : 0u, has1, pos4, vel4, aux, cell_start,
                                        sorted_idx, g, c, ep, out);
    }
}

// The per-particle modules of an unfused pipeline: ep.ops[0..n_ops) in order
// on each particle, the arithmetic of the fused force epilogue.
__global__ void __launch_bounds__(256)
    apply_ops_kernel(StepEpi ep, float* __restrict__ px, float* __restrict__ py, float* __restrict__ pz,
                     float* __restrict__ vx, float* __restrict__ vy, float* __restrict__ vz, uint32_t n) {
    pdl_enter();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float x = px[i], y = py[i], z = pz[i], u = vx[i], v = vy[i], w = vz[i];
    apply_ops(ep, x, y, z, u, v, w);
    px[i] = x;
    py[i] = y;
    pz[i] = z;
    vx[i] = u;
    vy[i] = v;
    vz[i] = w;
}

}  // namespace sph
}  // namespace forge
