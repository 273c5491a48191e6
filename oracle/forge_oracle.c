/*
 * forge_oracle.c -- CPU restatement of huaying/forge-gpu's particle hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product). Built with
 * -ffp-contract=off so every float operation rounds exactly as written in the
 * reference kernel strings; the GPU build may fuse multiply-adds, which the
 * density/force tolerances absorb. Grid, sort and boundary outputs are
 * integer work and must match the GPU bit for bit.
 *
 * Parity: grid build / radix sort / find_cell_boundaries / query are pinned
 * by the reference's known-answer tests (tests/golden fixtures). SPH density
 * and force: parity unpinned by reference fixtures (the reference has no SPH
 * unit test); they restate the kernel strings cited per function and are
 * cross-checked against fp64 all-pairs evaluations of the same formulas
 * (tests/test_oracle.py).
 */
#include "forge_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Generators                                                               */
/* ------------------------------------------------------------------------ */
static uint64_t splitmix64(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct { uint32_t s[4]; } xo128;

static void xo_seed(xo128* r, uint64_t seed) {
    uint64_t sm = seed;
    uint64_t a = splitmix64(&sm), b = splitmix64(&sm);
    r->s[0] = (uint32_t)a;
    r->s[1] = (uint32_t)(a >> 32);
    r->s[2] = (uint32_t)b;
    r->s[3] = (uint32_t)(b >> 32);
    if (!(r->s[0] | r->s[1] | r->s[2] | r->s[3])) r->s[0] = 1;
}

static inline uint32_t rotl32(uint32_t x, int k) { return (x << k) | (x >> (32 - k)); }

/* xoshiro128** (Blackman & Vigna). */
static inline uint32_t xo_next(xo128* r) {
    uint32_t* s = r->s;
    const uint32_t result = rotl32(s[1] * 5u, 7) * 9u;
    const uint32_t t = s[1] << 9;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl32(s[3], 11);
    return result;
}

static inline float xo_unit(xo128* r) { return (float)(xo_next(r) >> 8) * (1.0f / 16777216.0f); }

void orc_uniform_f32(uint64_t seed, uint64_t n, float lo, float hi, float* out) {
    xo128 r;
    xo_seed(&r, seed);
    for (uint64_t i = 0; i < n; ++i) out[i] = lo + (hi - lo) * xo_unit(&r);
}

void orc_normal_f32(uint64_t seed, uint64_t n, float mean, float sigma, float* out) {
    xo128 r;
    xo_seed(&r, seed);
    for (uint64_t i = 0; i < n; i += 2) {
        double u1 = ((double)(xo_next(&r) >> 8) + 1.0) / 16777217.0; /* (0,1] */
        double u2 = (double)(xo_next(&r) >> 8) / 16777216.0;
        double rad = sqrt(-2.0 * log(u1));
        out[i] = (float)(mean + sigma * rad * cos(6.283185307179586 * u2));
        if (i + 1 < n) out[i + 1] = (float)(mean + sigma * rad * sin(6.283185307179586 * u2));
    }
}

void orc_uniform_u32(uint64_t seed, uint64_t n, uint32_t* out) {
    xo128 r;
    xo_seed(&r, seed);
    for (uint64_t i = 0; i < n; ++i) out[i] = xo_next(&r);
}

static uint32_t spread10(uint32_t v) {
    v &= 0x3ffu;
    v = (v | (v << 16)) & 0x030000FFu;
    v = (v | (v << 8)) & 0x0300F00Fu;
    v = (v | (v << 4)) & 0x030C30C3u;
    v = (v | (v << 2)) & 0x09249249u;
    return v;
}

void orc_morton30(uint64_t seed, uint64_t n, uint32_t* out) {
    xo128 r;
    xo_seed(&r, seed);
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t x = (uint32_t)floorf(xo_unit(&r) * 1024.0f);
        uint32_t y = (uint32_t)floorf(xo_unit(&r) * 1024.0f);
        uint32_t z = (uint32_t)floorf(xo_unit(&r) * 1024.0f);
        out[i] = spread10(x) | (spread10(y) << 1) | (spread10(z) << 2);
    }
}

void orc_lattice(uint32_t nx, uint32_t ny, uint32_t nz, float spacing, const float lo[3], float* px, float* py,
                 float* pz) {
    uint64_t i = 0;
    for (uint32_t z = 0; z < nz; ++z)
        for (uint32_t y = 0; y < ny; ++y)
            for (uint32_t x = 0; x < nx; ++x, ++i) {
                px[i] = lo[0] + ((float)x + 0.5f) * spacing;
                py[i] = lo[1] + ((float)y + 0.5f) * spacing;
                pz[i] = lo[2] + ((float)z + 0.5f) * spacing;
            }
}

void orc_blobs(uint64_t seed, uint64_t n, uint32_t blobs, float clo, float chi, float sigma, float* px, float* py,
               float* pz) {
    float* c = (float*)malloc(sizeof(float) * 3 * blobs);
    orc_uniform_f32(seed, 3ull * blobs, clo, chi, c);
    float* g = (float*)malloc(sizeof(float) * 3 * n);
    orc_normal_f32(seed ^ 0xB10B5ull, 3 * n, 0.0f, sigma, g);
    const uint64_t per = (n + blobs - 1) / blobs;
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t b = i / per;
        px[i] = c[3 * b + 0] + g[3 * i + 0];
        py[i] = c[3 * b + 1] + g[3 * i + 1];
        pz[i] = c[3 * b + 2] + g[3 * i + 2];
    }
    free(g);
    free(c);
}

void orc_xorshift32_keys(uint32_t seed, uint64_t n, uint32_t mask, uint32_t* out) {
    uint32_t s = seed;
    for (uint64_t i = 0; i < n; ++i) {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        out[i] = s & mask;
    }
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* Grid build                                                               */
/* ------------------------------------------------------------------------ */

/* Rust `f32 as i32`: truncate toward zero, saturate, NaN -> 0. The value is
 * already floored, so truncation is exact. */
static inline int32_t sat_f2i(float v) {
    if (v != v) return 0;
    if (v >= 2147483648.0f) return 2147483647;
    if (v < -2147483648.0f) return (-2147483647 - 1);
    return (int32_t)v;
}

/* hashgrid.rs:128-139: ((p - o) / cs).floor() as i32, clamp, x-fastest. */
uint32_t orc_cell_of(float x, float y, float z, const float origin[3], float cs, uint32_t nx, uint32_t ny,
                     uint32_t nz) {
    const float ox = origin ? origin[0] : 0.f, oy = origin ? origin[1] : 0.f, oz = origin ? origin[2] : 0.f;
    int32_t cx = sat_f2i(floorf((x - ox) / cs));
    int32_t cy = sat_f2i(floorf((y - oy) / cs));
    int32_t cz = sat_f2i(floorf((z - oz) / cs));
    if (cx < 0) cx = 0;
    if (cx > (int32_t)nx - 1) cx = (int32_t)nx - 1;
    if (cy < 0) cy = 0;
    if (cy > (int32_t)ny - 1) cy = (int32_t)ny - 1;
    if (cz < 0) cz = 0;
    if (cz > (int32_t)nz - 1) cz = (int32_t)nz - 1;
    return (uint32_t)cx + (uint32_t)cy * nx + (uint32_t)cz * nx * ny;
}

/* hashgrid.rs:82-125. */
void orc_grid_build(const float* px, const float* py, const float* pz, uint32_t stride, uint64_t n,
                    const float origin[3], float cs, uint32_t nx, uint32_t ny, uint32_t nz, uint32_t* cell_idx,
                    uint32_t* sorted_idx, uint32_t* cell_start) {
    const uint64_t C = (uint64_t)nx * ny * nz;
    for (uint64_t i = 0; i < n; ++i)
        cell_idx[i] = orc_cell_of(px[i * stride], py[i * stride], pz[i * stride], origin, cs, nx, ny, nz);
    /* counts into cell_start[1..C], then inclusive prefix -> exclusive starts */
    memset(cell_start, 0, sizeof(uint32_t) * (C + 1));
    for (uint64_t i = 0; i < n; ++i) cell_start[cell_idx[i] + 1] += 1;
    for (uint64_t c = 0; c < C; ++c) cell_start[c + 1] += cell_start[c];
    uint32_t* off = (uint32_t*)malloc(sizeof(uint32_t) * (C ? C : 1));
    memcpy(off, cell_start, sizeof(uint32_t) * C);
    for (uint64_t i = 0; i < n; ++i) sorted_idx[off[cell_idx[i]]++] = (uint32_t)i;
    free(off);
}

/* Stable LSD counting sort by 8-bit digits of key bits [begin, end): equal to
 * std::stable_sort by the masked key (and to the reference's stable 4-bit
 * LSD RadixSorter). */
void orc_sort_pairs(uint32_t* keys, uint32_t* vals, uint64_t n, uint32_t begin_bit, uint32_t end_bit) {
    if (n == 0 || begin_bit >= end_bit) return;
    uint32_t* k2 = (uint32_t*)malloc(sizeof(uint32_t) * n);
    uint32_t* v2 = (uint32_t*)malloc(sizeof(uint32_t) * n);
    uint32_t* ka = keys;
    uint32_t* va = vals;
    uint32_t* kb = k2;
    uint32_t* vb = v2;
    for (uint32_t shift = begin_bit; shift < end_bit; shift += 8) {
        const uint32_t bits = end_bit - shift < 8 ? end_bit - shift : 8;
        const uint32_t mask = (1u << bits) - 1u;
        uint64_t cnt[257];
        memset(cnt, 0, sizeof cnt);
        for (uint64_t i = 0; i < n; ++i) cnt[((ka[i] >> shift) & mask) + 1]++;
        for (int d = 0; d < 256; ++d) cnt[d + 1] += cnt[d];
        for (uint64_t i = 0; i < n; ++i) {
            const uint64_t o = cnt[(ka[i] >> shift) & mask]++;
            kb[o] = ka[i];
            vb[o] = va[i];
        }
        uint32_t* t = ka; ka = kb; kb = t;
        t = va; va = vb; vb = t;
    }
    if (ka != keys) {
        memcpy(keys, ka, sizeof(uint32_t) * n);
        memcpy(vals, va, sizeof(uint32_t) * n);
    }
    free(k2);
    free(v2);
}

/* radix_sort.rs:259-293 (fills) + :444-466 (boundary kernel). Ids >= num_cells
 * are skipped (the reference would write out of bounds). */
void orc_cell_bounds(const uint32_t* ids, uint64_t n, uint64_t num_cells, uint32_t* start, uint32_t* end) {
    for (uint64_t c = 0; c < num_cells; ++c) {
        start[c] = 0xFFFFFFFFu;
        end[c] = 0;
    }
    for (uint64_t i = 0; i < n; ++i) {
        const uint32_t cell = ids[i];
        if (cell >= num_cells) continue;
        if (i == 0 || ids[i - 1] != cell) start[cell] = (uint32_t)i;
        if (i == n - 1 || ids[i + 1] != cell) end[cell] = (uint32_t)(i + 1);
    }
}

/* hashgrid.rs:145-193. */
uint64_t orc_query(const float* px, const float* py, const float* pz, uint32_t stride, const uint32_t* cell_start,
                   const uint32_t* sorted_idx, const float origin[3], float cs, uint32_t nx, uint32_t ny,
                   uint32_t nz, float qx, float qy, float qz, float radius, uint32_t* hits, uint64_t max_hits) {
    const float ox = origin ? origin[0] : 0.f, oy = origin ? origin[1] : 0.f, oz = origin ? origin[2] : 0.f;
    const float r2 = radius * radius;
    const int64_t cx = sat_f2i(floorf((qx - ox) / cs));
    const int64_t cy = sat_f2i(floorf((qy - oy) / cs));
    const int64_t cz = sat_f2i(floorf((qz - oz) / cs));
    uint64_t cnt = 0;
    for (int dz = -1; dz <= 1; ++dz)
        for (int dy = -1; dy <= 1; ++dy)
            for (int dx = -1; dx <= 1; ++dx) {
                const int64_t x = cx + dx, y = cy + dy, z = cz + dz;
                if (x < 0 || y < 0 || z < 0) continue;
                if (x >= nx || y >= ny || z >= nz) continue;
                const uint32_t cell = (uint32_t)x + (uint32_t)y * nx + (uint32_t)z * nx * ny;
                for (uint32_t s = cell_start[cell]; s < cell_start[cell + 1]; ++s) {
                    const uint32_t j = sorted_idx[s];
                    const float ddx = px[(uint64_t)j * stride] - qx;
                    const float ddy = py[(uint64_t)j * stride] - qy;
                    const float ddz = pz[(uint64_t)j * stride] - qz;
                    const float d2 = ddx * ddx + ddy * ddy + ddz * ddz;
                    if (d2 <= r2) {
                        if (hits && cnt < max_hits) hits[cnt] = j;
                        ++cnt;
                    }
                }
            }
    return cnt;
}

/* ------------------------------------------------------------------------ */
/* SPH (parity unpinned by reference fixtures: restated kernel strings)     */
/* ------------------------------------------------------------------------ */

/* Clamped cell coordinates as the SPH kernels recompute them from the
 * position (sph_density.rs:421-426). */
static inline void sph_cell(float x, float y, float z, float cs, uint32_t nx, uint32_t ny, uint32_t nz, int* cx,
                            int* cy, int* cz) {
    int a = sat_f2i(floorf(x / cs)), b = sat_f2i(floorf(y / cs)), c = sat_f2i(floorf(z / cs));
    if (a < 0) a = 0;
    if (a >= (int)nx) a = (int)nx - 1;
    if (b < 0) b = 0;
    if (b >= (int)ny) b = (int)ny - 1;
    if (c < 0) c = 0;
    if (c >= (int)nz) c = (int)nz - 1;
    *cx = a;
    *cy = b;
    *cz = c;
}

/* sph_density.rs:401-461, for particles idx[0..count) (all n when idx is
 * NULL); out[k] is the density of particle idx[k]. */
static void density_of(const orc_sph_params* p, const float* px, const float* py, const float* pz, float cs,
                       uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                       const uint32_t* idx, uint64_t count, float* density, int threads) {
    const float h = p->h, mass = p->mass;
    const float h2 = h * h;
    const float h9 = h2 * h2 * h2 * h2 * h;
    const float poly6_coeff = 315.0f / (64.0f * 3.14159265f * h9);
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 256) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t kk = 0; kk < (int64_t)count; ++kk) {
        const uint64_t i = idx ? idx[kk] : (uint64_t)kk;
        const float xi = px[i], yi = py[i], zi = pz[i];
        float rho = 0.0f;
        int cx, cy, cz;
        sph_cell(xi, yi, zi, cs, nx, ny, nz, &cx, &cy, &cz);
        for (int dz = -1; dz <= 1; dz++) {
            const int z = cz + dz;
            if (z < 0 || z >= (int)nz) continue;
            for (int dy = -1; dy <= 1; dy++) {
                const int y = cy + dy;
                if (y < 0 || y >= (int)ny) continue;
                for (int dx = -1; dx <= 1; dx++) {
                    const int x = cx + dx;
                    if (x < 0 || x >= (int)nx) continue;
                    const uint32_t cell = (uint32_t)x + (uint32_t)y * nx + (uint32_t)z * nx * ny;
                    for (uint32_t s = cell_start[cell]; s < cell_start[cell + 1]; s++) {
                        const uint32_t j = sorted_idx[s];
                        const float dx2 = xi - px[j], dy2 = yi - py[j], dz2 = zi - pz[j];
                        const float r2 = dx2 * dx2 + dy2 * dy2 + dz2 * dz2;
                        if (r2 < h2) {
                            const float diff = h2 - r2;
                            rho += mass * poly6_coeff * diff * diff * diff;
                        }
                    }
                }
            }
        }
        density[kk] = rho;
    }
    (void)threads;
}

void orc_density(const orc_sph_params* p, const float* px, const float* py, const float* pz, uint64_t n, float cs,
                 uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                 float* density, int threads) {
    density_of(p, px, py, pz, cs, nx, ny, nz, cell_start, sorted_idx, NULL, n, density, threads);
}

void orc_density_at(const orc_sph_params* p, const float* px, const float* py, const float* pz, float cs,
                    uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                    const uint32_t* idx, uint64_t m, float* density, int threads) {
    density_of(p, px, py, pz, cs, nx, ny, nz, cell_start, sorted_idx, idx, m, density, threads);
}

/* Fused pressure + viscosity, sph_fused.rs:542-638 (terms per
 * sph_pressure.rs:28-112 / sph_viscosity.rs:27-106), Jacobi velocities. */
static void force_of(const orc_sph_params* p, uint32_t terms, const float* px, const float* py, const float* pz,
                     const float* vx, const float* vy, const float* vz, const float* density, float cs, uint32_t nx,
                     uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                     const uint32_t* idx, uint64_t count, float dt, float* vx_out, float* vy_out, float* vz_out,
                     float* ax_out, float* ay_out, float* az_out, int threads) {
    const float h = p->h, mass = p->mass, gas_constant = p->gas_constant, rest_density = p->rest_density,
                visc_coeff = p->viscosity;
    const float h2 = h * h;
    const float h6 = h2 * h2 * h2;
    const float spiky_grad_coeff = -45.0f / (3.14159265f * h6);
    const float visc_lap_coeff = 45.0f / (3.14159265f * h6);
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 256) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t kk = 0; kk < (int64_t)count; ++kk) {
        const uint64_t i = idx ? idx[kk] : (uint64_t)kk;
        const float xi = px[i], yi = py[i], zi = pz[i];
        const float vxi = vx[i], vyi = vy[i], vzi = vz[i];
        const float rho_i = density[i];
        const float p_i = gas_constant * (rho_i - rest_density);
        const int valid = !(rho_i < 1e-6f);
        float pax = 0.0f, pay = 0.0f, paz = 0.0f, vax = 0.0f, vay = 0.0f, vaz = 0.0f;
        if (valid) {
            int cx, cy, cz;
            sph_cell(xi, yi, zi, cs, nx, ny, nz, &cx, &cy, &cz);
            for (int dz = -1; dz <= 1; dz++) {
                const int z = cz + dz;
                if (z < 0 || z >= (int)nz) continue;
                for (int dy = -1; dy <= 1; dy++) {
                    const int y = cy + dy;
                    if (y < 0 || y >= (int)ny) continue;
                    for (int dx = -1; dx <= 1; dx++) {
                        const int x = cx + dx;
                        if (x < 0 || x >= (int)nx) continue;
                        const uint32_t cell = (uint32_t)x + (uint32_t)y * nx + (uint32_t)z * nx * ny;
                        for (uint32_t s = cell_start[cell]; s < cell_start[cell + 1]; s++) {
                            const uint32_t j = sorted_idx[s];
                            const float djx = xi - px[j], djy = yi - py[j], djz = zi - pz[j];
                            const float r2 = djx * djx + djy * djy + djz * djz;
                            if (r2 < h2 && r2 > 1e-12f) {
                                const float r = sqrtf(r2);
                                const float rho_j = density[j];
                                if (rho_j < 1e-6f) continue;
                                const float diff = h - r;
                                if (terms & 1u) {
                                    const float p_j = gas_constant * (rho_j - rest_density);
                                    const float grad_scale = spiky_grad_coeff * diff * diff / r;
                                    const float f_scale = -mass * (p_i + p_j) / (2.0f * rho_j) * grad_scale;
                                    if (terms & 4u) { /* magnitude scale for tolerances */
                                        pax += fabsf(f_scale * djx);
                                        pay += fabsf(f_scale * djy);
                                        paz += fabsf(f_scale * djz);
                                    } else {
                                        pax += f_scale * djx;
                                        pay += f_scale * djy;
                                        paz += f_scale * djz;
                                    }
                                }
                                if (terms & 2u) {
                                    const float lap = visc_lap_coeff * diff;
                                    const float v_scale = visc_coeff * mass / rho_j * lap;
                                    if (terms & 4u) {
                                        vax += fabsf(v_scale * (vx[j] - vxi));
                                        vay += fabsf(v_scale * (vy[j] - vyi));
                                        vaz += fabsf(v_scale * (vz[j] - vzi));
                                    } else {
                                        vax += v_scale * (vx[j] - vxi);
                                        vay += v_scale * (vy[j] - vyi);
                                        vaz += v_scale * (vz[j] - vzi);
                                    }
                                }
                            }
                        }
                    }
                }
            }
        }
        float ax = 0.0f, ay = 0.0f, az = 0.0f;
        const uint32_t t3 = terms & 3u;
        if (valid) {
            if (t3 == 3u) { /* sph_fused.rs:633-638 */
                const float inv_rho = 1.0f / rho_i;
                ax = (pax + vax) * inv_rho;
                ay = (pay + vay) * inv_rho;
                az = (paz + vaz) * inv_rho;
            } else if (t3 == 1u) { /* sph_pressure.rs:109-111 */
                ax = pax / rho_i;
                ay = pay / rho_i;
                az = paz / rho_i;
            } else { /* sph_viscosity.rs:103-105 */
                ax = vax / rho_i;
                ay = vay / rho_i;
                az = vaz / rho_i;
            }
        }
        vx_out[kk] = valid ? vxi + ax * dt : vxi;
        vy_out[kk] = valid ? vyi + ay * dt : vyi;
        vz_out[kk] = valid ? vzi + az * dt : vzi;
        if (ax_out) {
            ax_out[kk] = ax;
            ay_out[kk] = ay;
            az_out[kk] = az;
        }
    }
    (void)threads;
}

void orc_force(const orc_sph_params* p, uint32_t terms, const float* px, const float* py, const float* pz,
               const float* vx, const float* vy, const float* vz, const float* density, uint64_t n, float cs,
               uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
               float dt, float* vx_out, float* vy_out, float* vz_out, float* ax_out, float* ay_out, float* az_out,
               int threads) {
    force_of(p, terms, px, py, pz, vx, vy, vz, density, cs, nx, ny, nz, cell_start, sorted_idx, NULL, n, dt, vx_out,
             vy_out, vz_out, ax_out, ay_out, az_out, threads);
}

/* The force of particles idx[0..m) only (outputs indexed by k), against
 * all particles as neighbours: sampled checks of large configs. */
void orc_force_at(const orc_sph_params* p, uint32_t terms, const float* px, const float* py, const float* pz,
                  const float* vx, const float* vy, const float* vz, const float* density, float cs, uint32_t nx,
                  uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                  const uint32_t* idx, uint64_t m, float dt, float* vx_out, float* vy_out, float* vz_out,
                  float* ax_out, float* ay_out, float* az_out, int threads) {
    force_of(p, terms, px, py, pz, vx, vy, vz, density, cs, nx, ny, nz, cell_start, sorted_idx, idx, m, dt, vx_out,
             vy_out, vz_out, ax_out, ay_out, az_out, threads);
}

/* One per-particle module after the SPH module:
 * 1 gravity.rs:31-34, 2 drag.rs:18-20, 3 integrate.rs:16-31,
 * 4 ground_plane.rs:19-21, 5 sphere_collider.rs:22-41, 6 box_collider.rs:36-46. */
static void orc_apply_op(const orc_step_op* o, float dt, float* x, float* y, float* z, float* vx, float* vy,
                         float* vz) {
    switch (o->kind) {
        case 1:
            *vx += o->p[0] * dt;
            *vy += o->p[1] * dt;
            *vz += o->p[2] * dt;
            break;
        case 2: {
            const float d = 1.0f - o->p[0] * dt;
            *vx *= d;
            *vy *= d;
            *vz *= d;
            break;
        }
        case 3:
            if (!isfinite(*vx)) *vx = 0.0f;
            if (!isfinite(*vy)) *vy = 0.0f;
            if (!isfinite(*vz)) *vz = 0.0f;
            *x += *vx * dt;
            *y += *vy * dt;
            *z += *vz * dt;
            break;
        case 4:
            if (*y < o->p[0]) {
                *y = o->p[0];
                *vy = -*vy * o->p[1];
            }
            break;
        case 5: {
            const float dx = *x - o->p[0], dy = *y - o->p[1], dz = *z - o->p[2];
            const float dist = sqrtf(dx * dx + dy * dy + dz * dz);
            const float r = o->p[3];
            if (dist < r && dist > 1e-8f) {
                const float inv = 1.0f / dist;
                const float nx = dx * inv, ny = dy * inv, nz = dz * inv;
                *x = o->p[0] + nx * r;
                *y = o->p[1] + ny * r;
                *z = o->p[2] + nz * r;
                const float vn = *vx * nx + *vy * ny + *vz * nz;
                if (vn < 0) {
                    *vx -= (1 + o->p[4]) * vn * nx;
                    *vy -= (1 + o->p[4]) * vn * ny;
                    *vz -= (1 + o->p[4]) * vn * nz;
                }
            }
            break;
        }
        case 6: {
            const float e = o->p[6];
            if (*x < o->p[0]) { *x = o->p[0]; *vx = fabsf(*vx) * e; }
            if (*x > o->p[3]) { *x = o->p[3]; *vx = -fabsf(*vx) * e; }
            if (*y < o->p[1]) { *y = o->p[1]; *vy = fabsf(*vy) * e; }
            if (*y > o->p[4]) { *y = o->p[4]; *vy = -fabsf(*vy) * e; }
            if (*z < o->p[2]) { *z = o->p[2]; *vz = fabsf(*vz) * e; }
            if (*z > o->p[5]) { *z = o->p[5]; *vz = -fabsf(*vz) * e; }
            break;
        }
        default:
            break;
    }
}

/* manifest_runner.rs:371-541: SphFused -> Gravity (gravity.rs:31-34) ->
 * Integrate (integrate.rs:16-31) -> BoxCollider (box_collider.rs:26-47). */
/* The per-particle modules of an unfused pipeline (gravity.rs, drag.rs,
 * integrate.rs, ground_plane.rs, sphere_collider.rs, box_collider.rs): the
 * step's op list applied in order to every particle. */
void orc_apply_ops(const orc_step_params* sp, float* px, float* py, float* pz, float* vx, float* vy, float* vz,
                   uint64_t n) {
    for (uint64_t i = 0; i < n; ++i)
        for (uint32_t k = 0; k < sp->n_ops; ++k)
            orc_apply_op(&sp->ops[k], sp->dt, &px[i], &py[i], &pz[i], &vx[i], &vy[i], &vz[i]);
}

void orc_step(const orc_sph_params* p, const orc_step_params* sp, float* px, float* py, float* pz, float* vx,
              float* vy, float* vz, float* density, uint64_t n, float cs, uint32_t nx, uint32_t ny, uint32_t nz,
              uint32_t* work, int threads) {
    uint32_t* cell_idx = work;
    uint32_t* sorted_idx = work + n;
    float* rho = (float*)(work + 2 * n);
    uint32_t* cell_start = work + 4 * n; /* words [3n, 4n) are spare */
    orc_grid_build(px, py, pz, 1, n, NULL, cs, nx, ny, nz, cell_idx, sorted_idx, cell_start);
    orc_density(p, px, py, pz, n, cs, nx, ny, nz, cell_start, sorted_idx, rho, threads);
    float* nvx = (float*)malloc(sizeof(float) * (n ? 3 * n : 1));
    float* nvy = nvx + n;
    float* nvz = nvx + 2 * n;
    orc_force(p, 3u, px, py, pz, vx, vy, vz, rho, n, cs, nx, ny, nz, cell_start, sorted_idx, sp->dt, nvx, nvy, nvz,
              NULL, NULL, NULL, threads);
    const float dt = sp->dt, e = sp->restitution;
    for (uint64_t i = 0; i < n; ++i) {
        float x = px[i], y = py[i], z = pz[i];
        float u = nvx[i], v = nvy[i], w = nvz[i];
        if (sp->n_ops) {
            for (uint32_t k = 0; k < sp->n_ops; ++k) orc_apply_op(&sp->ops[k], dt, &x, &y, &z, &u, &v, &w);
        } else {
        if (sp->flags & 1u) {
            u += sp->gravity[0] * dt;
            v += sp->gravity[1] * dt;
            w += sp->gravity[2] * dt;
        }
        if (sp->flags & 2u) {
            if (!isfinite(u)) u = 0.0f;
            if (!isfinite(v)) v = 0.0f;
            if (!isfinite(w)) w = 0.0f;
            x += u * dt;
            y += v * dt;
            z += w * dt;
        }
        if (sp->flags & 4u) {
            if (x < sp->box_min[0]) { x = sp->box_min[0]; u = fabsf(u) * e; }
            if (x > sp->box_max[0]) { x = sp->box_max[0]; u = -fabsf(u) * e; }
            if (y < sp->box_min[1]) { y = sp->box_min[1]; v = fabsf(v) * e; }
            if (y > sp->box_max[1]) { y = sp->box_max[1]; v = -fabsf(v) * e; }
            if (z < sp->box_min[2]) { z = sp->box_min[2]; w = fabsf(w) * e; }
            if (z > sp->box_max[2]) { z = sp->box_max[2]; w = -fabsf(w) * e; }
        }
        }
        px[i] = x; py[i] = y; pz[i] = z;
        vx[i] = u; vy[i] = v; vz[i] = w;
        if (density) density[i] = rho[i];
    }
    free(nvx);
}
