/*
 * forge_oracle.h -- CPU restatement of huaying/forge-gpu's particle hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the parity tests, smoke()
 * and bench.py's CPU-baseline leg compare the CUDA library against. The
 * product (libforge_sph.so) never links, loads or calls it.
 *
 * Pinning: the grid-build, radix-sort and find_cell_boundaries functions are
 * checked against every known-answer test of the reference
 * (tests/radix_sort_test.rs, tests/hashgrid_test.rs). The SPH density and
 * force math has no golden vector in the reference's own tests, so that part
 * is "parity unpinned" by reference fixtures: it restates the reference's
 * kernel strings line by line (file:line cited per function).
 *
 * Paths are relative to the forge-gpu project root.
 */
#ifndef FORGE_ORACLE_H
#define FORGE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded generators shared by CPU and GPU tests ---------------------- */
/* splitmix64 seeds a xoshiro128** stream; uniforms are 24-bit floats in
 * [0,1); normals use Box-Muller. */
void orc_uniform_f32(uint64_t seed, uint64_t n, float lo, float hi, float* out);
void orc_normal_f32(uint64_t seed, uint64_t n, float mean, float sigma, float* out);
void orc_uniform_u32(uint64_t seed, uint64_t n, uint32_t* out);
/* 30-bit Morton codes (10 bits/axis, floor(x*1024)) of uniform points. */
void orc_morton30(uint64_t seed, uint64_t n, uint32_t* out);
/* Lattice of nx*ny*nz points lo + (i+0.5)*spacing, x fastest. */
void orc_lattice(uint32_t nx, uint32_t ny, uint32_t nz, float spacing, const float lo[3],
                 float* px, float* py, float* pz);
/* n points from `blobs` isotropic Gaussians, centres uniform in [clo,chi]^3,
 * n/blobs points each (blob-major order). */
void orc_blobs(uint64_t seed, uint64_t n, uint32_t blobs, float clo, float chi, float sigma,
               float* px, float* py, float* pz);
/* The reference's test PRNG (tests/radix_sort_test.rs:58-66). */
void orc_xorshift32_keys(uint32_t seed, uint64_t n, uint32_t mask, uint32_t* out);

/* ---- grid build --------------------------------------------------------- */
/* HashGrid::position_to_cell, forge-runtime/src/hashgrid.rs:128-139
 * (== compute_cell_index, sph_fused.rs:84-100, when origin is 0). */
uint32_t orc_cell_of(float x, float y, float z, const float origin[3], float cs,
                     uint32_t nx, uint32_t ny, uint32_t nz);
/* HashGrid::build, hashgrid.rs:82-125: stable counting sort.
 * stride 1 = SoA (px,py,pz), stride 3 = Vec3f AoS (px = xyz). */
void orc_grid_build(const float* px, const float* py, const float* pz, uint32_t stride, uint64_t n,
                    const float origin[3], float cs, uint32_t nx, uint32_t ny, uint32_t nz,
                    uint32_t* cell_idx, uint32_t* sorted_idx, uint32_t* cell_start /*C+1*/);
/* Stable sort of pairs by key bits [begin,end) == std::stable_sort; the
 * result of RadixSorter::sort (radix_sort.rs:79-220). In place. */
void orc_sort_pairs(uint32_t* keys, uint32_t* vals, uint64_t n, uint32_t begin_bit, uint32_t end_bit);
/* find_cell_boundaries, radix_sort.rs:229-317 / kernel :444-466. */
void orc_cell_bounds(const uint32_t* ids, uint64_t n, uint64_t num_cells, uint32_t* start, uint32_t* end);
/* HashGrid::query_neighbors, hashgrid.rs:145-193 (no clamp, `<=`).
 * Returns hit count; writes up to max_hits indices in walk order. */
uint64_t orc_query(const float* px, const float* py, const float* pz, uint32_t stride,
                   const uint32_t* cell_start, const uint32_t* sorted_idx, const float origin[3], float cs,
                   uint32_t nx, uint32_t ny, uint32_t nz, float qx, float qy, float qz, float radius,
                   uint32_t* hits, uint64_t max_hits);

/* ---- SPH ---------------------------------------------------------------- */
typedef struct orc_sph_params {
    float h, mass, gas_constant, rest_density, viscosity;
} orc_sph_params;

typedef struct orc_step_op {
    uint32_t kind; /* 1 gravity, 2 drag, 3 integrate, 4 ground, 5 sphere, 6 box */
    float p[7];
} orc_step_op;

typedef struct orc_step_params {
    float dt;
    float gravity[3];
    float box_min[3], box_max[3];
    float restitution;
    uint32_t flags; /* 1 gravity, 2 integrate, 4 box (when n_ops == 0) */
    uint32_t n_ops; /* > 0: apply ops[] in order instead */
    orc_step_op ops[8];
} orc_step_params;

/* sph_density kernel, sph_density.rs:401-461. threads > 1 uses OpenMP over
 * particles (each particle's sum keeps the reference order). */
void orc_density(const orc_sph_params* p, const float* px, const float* py, const float* pz, uint64_t n,
                 float cs, uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start,
                 const uint32_t* sorted_idx, float* density, int threads);
/* Force terms (1 pressure sph_pressure.rs:28-112, 2 viscosity
 * sph_viscosity.rs:27-106, 3 fused sph_fused.rs:518-639) with Jacobi
 * velocities: reads v_in, writes v_out and accel (nullable). terms | 4
 * accumulates |term| instead of term (the per-particle magnitude scale the
 * force tolerance is stated against). */
/* density / force of the particles idx[0..m) only, against all n as
 * neighbours (outputs indexed 0..m): sampled checks of large configs */
void orc_density_at(const orc_sph_params* p, const float* px, const float* py, const float* pz, float cs,
                    uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                    const uint32_t* idx, uint64_t m, float* density, int threads);
void orc_force_at(const orc_sph_params* p, uint32_t terms, const float* px, const float* py, const float* pz,
                  const float* vx, const float* vy, const float* vz, const float* density, float cs, uint32_t nx,
                  uint32_t ny, uint32_t nz, const uint32_t* cell_start, const uint32_t* sorted_idx,
                  const uint32_t* idx, uint64_t m, float dt, float* vx_out, float* vy_out, float* vz_out,
                  float* ax_out, float* ay_out, float* az_out, int threads);
void orc_force(const orc_sph_params* p, uint32_t terms, const float* px, const float* py, const float* pz,
               const float* vx, const float* vy, const float* vz, const float* density, uint64_t n,
               float cs, uint32_t nx, uint32_t ny, uint32_t nz, const uint32_t* cell_start,
               const uint32_t* sorted_idx, float dt, float* vx_out, float* vy_out, float* vz_out,
               float* ax, float* ay, float* az, int threads);
/* sp->ops[0..n_ops) applied in order to every particle (unfused modules). */
void orc_apply_ops(const orc_step_params* sp, float* px, float* py, float* pz, float* vx, float* vy, float* vz,
                   uint64_t n);

/* One manifest step in place: SphFused (grid rebuild, density, fused force)
 * -> Gravity -> Integrate -> BoxCollider (manifest_runner.rs:371-541).
 * `work` must hold 4*n + (C+1) uint32/float words. density nullable. */
void orc_step(const orc_sph_params* p, const orc_step_params* sp, float* px, float* py, float* pz, float* vx,
              float* vy, float* vz, float* density, uint64_t n, float cs, uint32_t nx, uint32_t ny, uint32_t nz,
              uint32_t* work, int threads);

int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
