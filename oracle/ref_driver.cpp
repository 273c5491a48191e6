/* Launch loops for the reference's kernels built on the host (test
 * infrastructure only; the product never loads this library).
 *
 * Each ref_* function runs one reference kernel (or the reference's sequence
 * of kernels) over all thread indices. The kernel bodies are the reference's
 * own strings (oracle/_ref/ref_kernels.cpp, made by ref_extract.py); only the
 * loops and the exclusive scan of the cell counts are written here.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "ref_shim.h"

thread_local ref_dim3 blockIdx = {0u, 0u, 0u};

extern "C" {
void compute_cell_index(const float*, const float*, const float*, unsigned int*, float, int, int, int, int);
void count_cells(const unsigned int*, unsigned int*, int);
void scatter_particles(const unsigned int*, const unsigned int*, unsigned int*, unsigned int*, int);
void set_last(unsigned int*, int, unsigned int);
void sph_density(const float*, const float*, const float*, float*, const unsigned int*, const unsigned int*, float,
                 float, float, int, int, int, int);
void sph_pressure(const float*, const float*, const float*, float*, float*, float*, const float*,
                  const unsigned int*, const unsigned int*, float, float, float, float, float, int, int, int, float,
                  int);
void sph_viscosity(const float*, const float*, const float*, float*, float*, float*, const float*,
                   const unsigned int*, const unsigned int*, float, float, float, float, int, int, int, float, int);
void gravity(float*, float*, float*, float, float, float, float, int);
void integrate(float*, float*, float*, float*, float*, float*, float, int);
void box_collider(float*, float*, float*, float*, float*, float*, float, float, float, float, float, float, float,
                  int);
void drag(float*, float*, float*, float, float, int);
void ground(float*, float*, float, float, int);
void sphere_collide(float*, float*, float*, float*, float*, float*, float, float, float, float, float, int);
}

#define FOR_THREADS(n, threads, body)                                   \
    _Pragma("omp parallel for schedule(dynamic, 1024) num_threads(threads)") \
    for (int i_ = 0; i_ < (int)(n); ++i_) {                             \
        blockIdx.x = (unsigned int)i_;                                  \
        body;                                                           \
    }

#define FOR_SERIAL(n, body)                         \
    for (int i_ = 0; i_ < (int)(n); ++i_) {         \
        blockIdx.x = (unsigned int)i_;              \
        body;                                       \
    }

extern "C" {

/* The unfused SphDensityModule grid build (sph_density.rs:130-380):
 * compute_cell_index, count_cells, exclusive scan, set_last(C, n) and
 * scatter_particles, each over every particle in index order. The reference
 * scans with a block-level shared-memory kernel; an exclusive scan has one
 * result, computed here directly. */
void ref_grid_build(const float* px, const float* py, const float* pz, float cs, int nx, int ny, int nz, int n,
                    uint32_t* cell_idx, uint32_t* cell_start /* C+1 */, uint32_t* sorted_idx) {
    const size_t C = (size_t)nx * ny * nz;
    uint32_t* count = (uint32_t*)calloc(C, 4);
    uint32_t* offset = (uint32_t*)calloc(C, 4);
    FOR_SERIAL(n, compute_cell_index(px, py, pz, cell_idx, cs, nx, ny, nz, n));
    FOR_SERIAL(n, count_cells(cell_idx, count, n));
    uint32_t run = 0;
    for (size_t c = 0; c < C; ++c) {
        cell_start[c] = run;
        run += count[c];
    }
    blockIdx.x = 0;
    set_last(cell_start, (int)C, (unsigned int)n);
    FOR_SERIAL(n, scatter_particles(cell_idx, cell_start, offset, sorted_idx, n));
    free(count);
    free(offset);
}

void ref_density(const float* px, const float* py, const float* pz, float* density, const uint32_t* cell_start,
                 const uint32_t* sorted_idx, float h, float mass, float cs, int nx, int ny, int nz, int n,
                 int threads) {
    FOR_THREADS(n, threads,
                sph_density(px, py, pz, density, cell_start, sorted_idx, h, mass, cs, nx, ny, nz, n));
}

/* sph_pressure / sph_viscosity update vx[i] in place while other threads
 * read vx[j] (a race on the GPU). Jacobi form, the one the parity tests
 * use: each particle's thread runs against the unmodified velocities, its
 * result is taken, and its own velocity is put back before the next thread
 * runs (serial, index order). out_* receive the updated velocities. */
static void jacobi(int which, const float* px, const float* py, const float* pz, float* vx, float* vy, float* vz,
                   const float* density, const uint32_t* cs_, const uint32_t* si, float h, float mass, float k,
                   float rho0, float mu, float cs, int nx, int ny, int nz, float dt, int n, float* ox, float* oy,
                   float* oz) {
    for (int i = 0; i < n; ++i) {
        const float sx = vx[i], sy = vy[i], sz = vz[i];
        blockIdx.x = (unsigned int)i;
        if (which == 0)
            sph_pressure(px, py, pz, vx, vy, vz, density, cs_, si, h, mass, k, rho0, cs, nx, ny, nz, dt, n);
        else
            sph_viscosity(px, py, pz, vx, vy, vz, density, cs_, si, h, mass, mu, cs, nx, ny, nz, dt, n);
        ox[i] = vx[i];
        oy[i] = vy[i];
        oz[i] = vz[i];
        vx[i] = sx;
        vy[i] = sy;
        vz[i] = sz;
    }
}

void ref_pressure_jacobi(const float* px, const float* py, const float* pz, float* vx, float* vy, float* vz,
                         const float* density, const uint32_t* cell_start, const uint32_t* sorted_idx, float h,
                         float mass, float k, float rho0, float cs, int nx, int ny, int nz, float dt, int n,
                         float* ox, float* oy, float* oz) {
    jacobi(0, px, py, pz, vx, vy, vz, density, cell_start, sorted_idx, h, mass, k, rho0, 0.f, cs, nx, ny, nz, dt,
           n, ox, oy, oz);
}

void ref_viscosity_jacobi(const float* px, const float* py, const float* pz, float* vx, float* vy, float* vz,
                          const float* density, const uint32_t* cell_start, const uint32_t* sorted_idx, float h,
                          float mass, float mu, float cs, int nx, int ny, int nz, float dt, int n, float* ox,
                          float* oy, float* oz) {
    jacobi(1, px, py, pz, vx, vy, vz, density, cell_start, sorted_idx, h, mass, 0.f, 0.f, mu, cs, nx, ny, nz, dt,
           n, ox, oy, oz);
}

/* Per-particle modules, one kernel each over all particles. */
void ref_gravity(float* vx, float* vy, float* vz, float gx, float gy, float gz, float dt, int n, int threads) {
    FOR_THREADS(n, threads, gravity(vx, vy, vz, gx, gy, gz, dt, n));
}
void ref_integrate(float* px, float* py, float* pz, float* vx, float* vy, float* vz, float dt, int n, int threads) {
    FOR_THREADS(n, threads, integrate(px, py, pz, vx, vy, vz, dt, n));
}
void ref_box_collider(float* px, float* py, float* pz, float* vx, float* vy, float* vz, const float* mn,
                      const float* mx, float e, int n, int threads) {
    FOR_THREADS(n, threads, box_collider(px, py, pz, vx, vy, vz, mn[0], mn[1], mn[2], mx[0], mx[1], mx[2], e, n));
}
void ref_drag(float* vx, float* vy, float* vz, float c, float dt, int n, int threads) {
    FOR_THREADS(n, threads, drag(vx, vy, vz, c, dt, n));
}
void ref_ground(float* py, float* vy, float y0, float rest, int n, int threads) {
    FOR_THREADS(n, threads, ground(py, vy, y0, rest, n));
}
void ref_sphere_collide(float* px, float* py, float* pz, float* vx, float* vy, float* vz, float cx, float cy,
                        float cz, float r, float rest, int n, int threads) {
    FOR_THREADS(n, threads, sphere_collide(px, py, pz, vx, vy, vz, cx, cy, cz, r, rest, n));
}

/* The reference's unfused manifest step (manifest_runner.rs:405-541 order:
 * sph_density with its grid build, sph_pressure, sph_viscosity, gravity,
 * integrate, box_collider) as the reference runs it: every kernel in place,
 * threads in parallel. pressure and viscosity race on velocities exactly as
 * the reference's kernels do on the GPU (D2); this is the timed CPU
 * baseline, not a parity source. */
void ref_manifest_step(float* px, float* py, float* pz, float* vx, float* vy, float* vz, float* density,
                       uint32_t* cell_idx, uint32_t* cell_start, uint32_t* sorted_idx, float h, float mass, float k,
                       float rho0, float mu, float cs, int nx, int ny, int nz, float dt, const float* g,
                       const float* mn, const float* mx, float e, int n, int threads) {
    ref_grid_build(px, py, pz, cs, nx, ny, nz, n, cell_idx, cell_start, sorted_idx);
    ref_density(px, py, pz, density, cell_start, sorted_idx, h, mass, cs, nx, ny, nz, n, threads);
    FOR_THREADS(n, threads,
                sph_pressure(px, py, pz, vx, vy, vz, density, cell_start, sorted_idx, h, mass, k, rho0, cs, nx, ny,
                             nz, dt, n));
    FOR_THREADS(n, threads,
                sph_viscosity(px, py, pz, vx, vy, vz, density, cell_start, sorted_idx, h, mass, mu, cs, nx, ny, nz,
                              dt, n));
    ref_gravity(vx, vy, vz, g[0], g[1], g[2], dt, n, threads);
    ref_integrate(px, py, pz, vx, vy, vz, dt, n, threads);
    ref_box_collider(px, py, pz, vx, vy, vz, mn, mx, e, n, threads);
}

}  // extern "C"
