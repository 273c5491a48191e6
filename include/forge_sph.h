/*
 * forge_sph.h -- C ABI of the B200 (sm_100a) particle hot path.
 *
 * This library replaces, for the particle hot path only, the NVRTC-compiled
 * CUDA strings that huaying/forge-gpu launches through cudarc. Every entry
 * point below names the reference interface it stands in for (paths are
 * relative to the forge-gpu project root).
 *
 * Conventions
 *  - All pointers are DEVICE pointers unless a comment says "host".
 *  - All sizes are uint64_t element counts.
 *  - `stream` is a cudaStream_t / CUstream passed as void* (NULL = legacy
 *    default stream). Every call only enqueues work on that stream: no host
 *    synchronisation and no device allocation happen inside build / sort /
 *    density / force / step calls, so they may be recorded into a CUDA graph.
 *    Temporaries are allocated once, in the *_create calls (the reference's
 *    "pre-allocated for graph capture" contract, forge-runtime/src/radix_sort.rs:10).
 *  - Return value: FORGE_OK (0) on success, a negative FORGE_ERR_* code
 *    otherwise; forge_last_error() returns the calling thread's message.
 *    Conditions the reference asserts/panics on (radix_sort.rs:86-87) are
 *    returned as FORGE_ERR_INVALID_ARG here.
 *  - A handle is used by one host thread at a time; distinct handles are
 *    independent. Each handle is bound to the device ordinal given at create
 *    (the reference pins everything to device 0, forge-runtime/src/cuda.rs:55-63).
 *  - Device-side failures (a bounded wait that gave up, an out-of-range key)
 *    are recorded in a per-handle status word and reported by *_check().
 */
#ifndef FORGE_SPH_H
#define FORGE_SPH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FORGE_SPH_ABI_VERSION 1

#if defined(__GNUC__)
#define FORGE_API __attribute__((visibility("default")))
#else
#define FORGE_API
#endif

enum forge_status {
    FORGE_OK = 0,
    FORGE_ERR_INVALID_ARG = -1, /* bad pointer / size / bit range          */
    FORGE_ERR_CAPACITY = -2,    /* n > max_n given at create                */
    FORGE_ERR_CUDA = -3,        /* a CUDA runtime call failed               */
    FORGE_ERR_TIMEOUT = -4,     /* a bounded device wait gave up            */
    FORGE_ERR_NCCL = -5,        /* reserved for the sharded path            */
    FORGE_ERR_DEVICE = -6       /* device-side check failed (e.g. key >= C) */
};

/* Device status bits written by kernels (read back by *_check). */
#define FORGE_DEV_TIMEOUT 0x1u
#define FORGE_DEV_KEY_RANGE 0x2u
#define FORGE_DEV_CAPACITY 0x4u
#define FORGE_DEV_ZONE 0x8u

/* Copy the calling thread's last error message into buf (NUL-terminated).
 * Returns the full message length. */
FORGE_API uint64_t forge_last_error(char* buf, uint64_t len);

/* ABI version of the loaded library (FORGE_SPH_ABI_VERSION). */
FORGE_API int forge_abi_version(void);

/* ------------------------------------------------------------------------ */
/* Radix sort -- replaces RadixSorter (forge-runtime/src/radix_sort.rs:26-220) */
/* ------------------------------------------------------------------------ */

typedef struct forge_sorter forge_sorter;

/* RadixSorter::new(max_n, ordinal) -- radix_sort.rs:55-70.
 * Allocates alternate key/value buffers for max_n pairs plus the Onesweep
 * histogram and look-back status tables. max_n < 2^30. */
FORGE_API int forge_sorter_create(uint64_t max_n, int device, forge_sorter** out);

/* RadixSorter::sort(keys, values, n, num_bits) -- radix_sort.rs:79-220.
 * Stable LSD sort of (keys[i], vals[i]) by key bits [begin_bit, end_bit).
 * Equal keys keep their input order (bit-exact equal to std::stable_sort by
 * (key >> begin_bit) & mask). Bits outside the range are carried, not sorted.
 * vals may be NULL: the sort then behaves as if vals[i] == i (the particle
 * index) and writes the permutation into the value output.
 *
 * Result location: if keys_alt/vals_alt are NULL the result is always left in
 * keys/vals (the sorter's own alternate buffers are used, and vals must not be
 * NULL). If the caller passes its own alternate buffers the sorter ping-pongs
 * between the pairs and reports in *result_in_alt (host, nullable) whether
 * the sorted data ended in keys_alt/vals_alt -- the caller then swaps its
 * Arrays, exactly like the reference's std::mem::swap (radix_sort.rs:215-216). */
FORGE_API int forge_sorter_sort_pairs(forge_sorter* s, uint32_t* keys, uint32_t* vals,
                            uint32_t* keys_alt, uint32_t* vals_alt, uint64_t n,
                            uint32_t begin_bit, uint32_t end_bit,
                            int* result_in_alt, void* stream);

/* Stable key/value sort that allocates nothing. No counterpart in the
 * reference: this entry point exists for callers that cannot call
 * cudaMalloc -- hosts that fix their device-memory budget at start-up,
 * plug-in hosts whose allocator belongs to someone else, and latency-critical
 * loops where an allocation's implicit device synchronisation is not
 * acceptable. Same result as forge_sorter_sort_pairs with NULL alternate
 * buffers (sorted data left in keys/vals), for n <= FORGE_STATIC_SORT_MAX_N.
 *
 * Its scratch (look-back table, digit histograms, one alternate key/value
 * pair) is a fixed ~8.3 MiB array inside the library that every GPU which
 * loads the library holds until process exit. Runs on the calling thread's
 * current device. The first call on a device (and the first after a
 * cudaDeviceReset or under another CUDA context) looks the array up: make
 * that first call before any stream capture. All calls share
 * the array, so calls whose work overlaps on the GPU (different streams, or
 * different host threads on one device) race; serialise them. A device-side
 * wait that gives up is not reported by this entry point (use the
 * handle-based sorter and forge_sorter_check when that matters).
 * Returns FORGE_ERR_CAPACITY for n > FORGE_STATIC_SORT_MAX_N. */
#define FORGE_STATIC_SORT_MAX_N (1ull << 20)
FORGE_API int forge_sort_pairs_static(uint32_t* keys, uint32_t* vals, uint64_t n, uint32_t begin_bit,
                                      uint32_t end_bit, void* stream);

/* Synchronise `stream` and report any device-side failure of this sorter
 * (FORGE_ERR_TIMEOUT if a look-back wait gave up). Clears the status. */
FORGE_API int forge_sorter_check(forge_sorter* s, void* stream);

/* Test hook for failure detection (no reference counterpart; no GPU fault
 * is involved). skip_tiles = 1 makes the first pass of the following sorts
 * never take tile id 0, so the look-back of tile 1 waits on a status word
 * that nothing writes; the wait gives up after spin_limit polls (0: the
 * default, ~0.3 s), records the timeout and returns, the sort completes
 * with unspecified output and forge_sorter_check reports FORGE_ERR_TIMEOUT.
 * skip_tiles = 0 and spin_limit = 0 restore normal sorting. */
FORGE_API int forge_sorter_set_test_fault(forge_sorter* s, uint32_t skip_tiles, uint32_t spin_limit);

FORGE_API void forge_sorter_destroy(forge_sorter* s);

/* find_cell_boundaries(sorted_ids, start, end, n, num_cells, ordinal)
 * -- radix_sort.rs:229-317, kernel :444-466.
 * start[c] = first index of cell c in sorted_ids or 0xFFFFFFFF if empty,
 * end[c]   = one past its last index, or 0 if empty. Every one of the
 * num_cells entries is written exactly once (no fill pass). Ids >= num_cells
 * are skipped. */
FORGE_API int forge_cell_bounds(const uint32_t* sorted_ids, uint32_t* start, uint32_t* end,
                      uint64_t n, uint64_t num_cells, void* stream);

/* ------------------------------------------------------------------------ */
/* Uniform hash grid -- replaces HashGrid (forge-runtime/src/hashgrid.rs)  and */
/* the GPU grid rebuild of SphFusedModule (forge-manifest/src/modules/builtins/ */
/* sph_fused.rs:36-408).                                                        */
/* ------------------------------------------------------------------------ */

typedef struct forge_grid forge_grid;

/* HashGrid::new(cell_size, (nx,ny,nz), origin, max_particles, device)
 * -- hashgrid.rs:50-72. origin is host float[3] (NULL = 0,0,0, the SPH
 * modules' convention, sph_fused.rs:91-99). nx*ny*nz < 2^31. Pre-allocates
 * every temporary for max_n particles (sort buffers, cell table, packed
 * cell-ordered particle arrays). */
FORGE_API int forge_grid_create(float cell_size, uint32_t nx, uint32_t ny, uint32_t nz,
                      const float* origin, uint64_t max_n, int device,
                      forge_grid** out);

/* GPU HashGrid::build (hashgrid.rs:82-125) from SoA positions (the manifest
 * FieldSet layout pos_x/pos_y/pos_z). Outputs (each nullable; the grid keeps
 * its own copy either way for later density/force/query calls):
 *   cell_idx[n]          cell of particle i (hashgrid.rs:128-139 / sph_fused.rs:84-100)
 *   sorted_idx[n]        particle indices ordered by cell, ascending index
 *                        within a cell (the stable order of hashgrid.rs:109-117)
 *   cell_start[C+1]      exclusive prefix of per-cell counts, cell_start[C] = n */
FORGE_API int forge_grid_build(forge_grid* g, const float* px, const float* py,
                     const float* pz, uint64_t n, uint32_t* cell_idx,
                     uint32_t* sorted_idx, uint32_t* cell_start, void* stream);

/* Same as forge_grid_build for Vec3f AoS positions (12-byte x,y,z records,
 * forge-core/src/vec.rs:137-143), the HashGrid::build input type. */
FORGE_API int forge_grid_build_aos(forge_grid* g, const float* xyz, uint64_t n,
                         uint32_t* cell_idx, uint32_t* sorted_idx,
                         uint32_t* cell_start, void* stream);

/* Batched GPU HashGrid::query_neighbors (hashgrid.rs:145-193): for each
 * query point q (SoA qx/qy/qz, nq of them) list the particles of the last
 * build within `radius` (dist^2 <= radius^2, the reference's `<=`), walking
 * the 3x3x3 cells around q in the reference order. Output is CSR:
 *   counts[nq]         number of hits per query (always written)
 *   offsets[nq+1]      exclusive prefix of counts (nullable)
 *   hits[max_hits]     hit indices, query-major, in walk order (nullable)
 * Call once with hits == NULL to size, then again with hits; if the total
 * exceeds max_hits, only counts/offsets are written and FORGE_ERR_CAPACITY
 * is returned by forge_grid_check. positions are the SoA arrays the grid was
 * built from. */
FORGE_API int forge_grid_query(forge_grid* g, const float* px, const float* py,
                     const float* pz, const float* qx, const float* qy,
                     const float* qz, uint64_t nq, float radius,
                     uint32_t* counts, uint32_t* offsets, uint32_t* hits,
                     uint64_t max_hits, void* stream);

/* Synchronise `stream`; report and clear device-side failures of this grid. */
FORGE_API int forge_grid_check(forge_grid* g, void* stream);

FORGE_API void forge_grid_destroy(forge_grid* g);

/* ------------------------------------------------------------------------ */
/* SPH passes -- replace SphDensityModule / SphPressureModule /             */
/* SphViscosityModule / SphFusedModule::execute                             */
/* (forge-manifest/src/modules/builtins/sph_*.rs)                           */
/* ------------------------------------------------------------------------ */

/* Module parameters (SphFusedModule fields, sph_fused.rs:14-22; cell size,
 * grid dims and origin live in the forge_grid). */
typedef struct forge_sph_params {
    float h;             /* smoothing_radius                 */
    float mass;          /* particle_mass                    */
    float gas_constant;  /* stiffness k, p = k (rho - rho0)  */
    float rest_density;  /* rho0                             */
    float viscosity;     /* viscosity_coefficient mu         */
} forge_sph_params;

/* Which terms forge_sph_force evaluates. */
#define FORGE_TERM_PRESSURE 0x1u  /* sph_pressure.rs:28-112   */
#define FORGE_TERM_VISCOSITY 0x2u /* sph_viscosity.rs:27-106  */

/* One per-particle module of the manifest pipeline after the SPH module,
 * applied in list order in the force kernel's epilogue (forge-manifest/src/
 * manifest_runner.rs:371-541 adds forces, then IntegrateModule, then the
 * constraints in TOML order). */
typedef struct forge_step_op {
    uint32_t kind; /* FORGE_OP_* */
    float p[7];
} forge_step_op;

#define FORGE_OP_GRAVITY 1u   /* v += g dt, p[0..2] = g            (gravity.rs:31-34)          */
#define FORGE_OP_DRAG 2u      /* v *= 1 - c dt, p[0] = c            (drag.rs:18-20)             */
#define FORGE_OP_INTEGRATE 3u /* NaN/Inf v -> 0, x += v dt          (integrate.rs:16-31)        */
#define FORGE_OP_GROUND 4u    /* y < p[0]: y = p[0], vy = -vy p[1]  (ground_plane.rs:19-21)     */
#define FORGE_OP_SPHERE 5u    /* centre p[0..2], radius p[3], restitution p[4]
                                                                    (sphere_collider.rs:22-41)  */
#define FORGE_OP_BOX 6u       /* min p[0..2], max p[3..5], restitution p[6]
                                                                    (box_collider.rs:26-47)     */
#define FORGE_STEP_MAX_OPS 8

/* Per-step epilogue after the SPH module. With n_ops == 0 the flags select
 * the common GravityModule -> IntegrateModule -> BoxColliderModule chain
 * (manifest_runner.rs:371-541); with n_ops > 0 the op list is applied
 * instead, in order. */
typedef struct forge_step_params {
    float dt;
    float gravity[3];    /* v += g dt                     (flags & FORGE_STEP_GRAVITY)   */
    float box_min[3];    /* clamp + reflect               (flags & FORGE_STEP_BOX)       */
    float box_max[3];
    float restitution;
    uint32_t flags;
    uint32_t n_ops;
    forge_step_op ops[FORGE_STEP_MAX_OPS];
} forge_step_params;

#define FORGE_STEP_GRAVITY 0x1u
#define FORGE_STEP_INTEGRATE 0x2u
#define FORGE_STEP_BOX 0x4u

/* SphDensityModule::execute (sph_density.rs:388-501): rebuilds the grid
 * from (px,py,pz) and writes the poly6 density of every particle, self
 * included, into density[n] (original particle order):
 *   rho_i = sum_{j: r2 < h2} m * 315/(64 pi h^9) * (h2 - r2)^3
 * Neighbours are summed in the reference order (dz, dy, dx from -1..1, then
 * ascending particle index within a cell). */
FORGE_API int forge_sph_density(forge_grid* g, const forge_sph_params* p,
                      const float* px, const float* py, const float* pz,
                      uint64_t n, float* density, void* stream);

/* Pressure and/or viscosity pass over the grid of the last build
 * (sph_pressure.rs:28-112, sph_viscosity.rs:27-106, fused as in
 * sph_fused.rs:518-639). Velocities are read from vel_in and written to
 * vel_out (Jacobi update: every neighbour term sees the velocities at the
 * start of the pass). vel_out may alias vel_in. accel_out (nullable, 3
 * arrays) receives (a_p + a_v) / rho_i, the per-particle acceleration
 * before the dt multiply. Particles with rho_i < 1e-6 keep their velocity
 * (accel 0). positions must be the ones the grid was last built from. */
FORGE_API int forge_sph_force(forge_grid* g, const forge_sph_params* p, uint32_t terms,
                    const float* px, const float* py, const float* pz,
                    const float* vx_in, const float* vy_in, const float* vz_in,
                    const float* density, uint64_t n, float dt,
                    float* vx_out, float* vy_out, float* vz_out,
                    float* ax_out, float* ay_out, float* az_out, void* stream);

/* The per-particle modules of an unfused pipeline on device `device`:
 * sp->ops[0..n_ops) (FORGE_OP_GRAVITY..FORGE_OP_BOX) applied in order to
 * each of the n particles in place, with the arithmetic of the fused force
 * epilogue -- GravityModule (gravity.rs:31-34), DragModule (drag.rs),
 * IntegrateModule (integrate.rs:16-31), GroundPlaneModule, SphereCollider-
 * Module, BoxColliderModule (box_collider.rs:36-46). sp->flags is ignored.
 * Capture-safe. */
FORGE_API int forge_apply_ops(const forge_step_params* sp, float* px, float* py, float* pz, float* vx, float* vy,
                              float* vz, uint64_t n, int device, void* stream);

/* One fused SPH step in place on the FieldSet arrays: grid rebuild,
 * density, pressure+viscosity (Jacobi), then the optional gravity /
 * integrate / box epilogue in pipeline order -- the work of
 * SphFusedModule::execute followed by GravityModule, IntegrateModule and
 * BoxColliderModule (manifest_runner.rs:371-541). density (nullable)
 * receives rho in original order. Capture-safe. */
FORGE_API int forge_sph_step(forge_grid* g, const forge_sph_params* p,
                   const forge_step_params* sp, float* px, float* py,
                   float* pz, float* vx, float* vy, float* vz, float* density,
                   uint64_t n, void* stream);

/* Force + step epilogue from a caller-supplied density, for a domain-
 * decomposed run (the sharded form of forge_sph_step): the grid was built by
 * forge_sph_density over n particles = owned particles first, then ghost
 * copies of neighbouring slabs' boundary particles; density[n] holds the
 * owners' exact densities (ghost entries overwritten after the exchange).
 * Pressure + viscosity (Jacobi) + gravity / integrate / box as in
 * forge_sph_step, but only particles i < n_update (the owned ones) are
 * updated in place. Same math as SphFusedModule::execute's force pass
 * (sph_fused.rs:518-639) followed by gravity.rs, integrate.rs,
 * box_collider.rs. */
FORGE_API int forge_sph_force_step(forge_grid* g, const forge_sph_params* p, const forge_step_params* sp,
                                   float* px, float* py, float* pz, float* vx, float* vy, float* vz,
                                   const float* density, uint64_t n, uint64_t n_update, void* stream);

/* Split form of forge_sph_force_step for overlapping the slab exchange with
 * the force pass. The owned particles (i < n_update) are split by grid cell
 * x-slice: the interior zone is the slices whose x-extent lies inside
 * [inner_lo, inner_hi) (+-inf for an open side), the boundary zone the rest.
 * Modes, on one grid build:
 *   FORGE_ZONE_PREPARE   gather velocities + density in cell order, list
 *                        both zones (no force kernel);
 *   FORGE_ZONE_BOUNDARY  update the boundary particles (preceded by the
 *                        prepare step if none ran; else it first re-reads
 *                        the ghosts' densities, i >= n_update, which may
 *                        have arrived since);
 *   FORGE_ZONE_INTERIOR  update the interior particles (needs a prepare or
 *                        boundary call before it).
 * BOUNDARY + INTERIOR equal one forge_sph_force_step bit for bit. Each zone
 * call waits, on its own stream, only for the prepare step, so the two
 * zones' kernels may run concurrently on two streams; interior particles
 * have no ghost neighbours, so the interior pass may also run before the
 * ghost densities arrive. Once a boundary call's work is done its particles'
 * columns are final and may be read (e.g. by forge_slab_exchange_begin
 * enqueued after it). An interior particle whose x before or after the step
 * lies outside [guard_lo, guard_hi) sets FORGE_DEV_ZONE in the grid's status
 * (forge_grid_check): it is, or moved, too close to a face for the
 * overlapped exchange to classify it safely. The first prepare on a grid
 * allocates its zone lists (4 bytes per particle). */
#define FORGE_ZONE_BOUNDARY 1u
#define FORGE_ZONE_INTERIOR 2u
#define FORGE_ZONE_PREPARE 3u
typedef struct forge_force_zone {
    uint32_t mode;
    float inner_lo, inner_hi;
    float guard_lo, guard_hi;
} forge_force_zone;

FORGE_API int forge_sph_force_step_zone(forge_grid* g, const forge_sph_params* p, const forge_step_params* sp,
                                        float* px, float* py, float* pz, float* vx, float* vy, float* vz,
                                        const float* density, uint64_t n, uint64_t n_update,
                                        const forge_force_zone* zone, void* stream);

/* ------------------------------------------------------------------------ */
/* Slab-exchange helpers for the sharded step. No counterpart in the        */
/* reference: its multi-GPU API is a stub (forge-runtime/src/cuda.rs:134-178). */
/* ------------------------------------------------------------------------ */

typedef struct forge_slab forge_slab;

/* Scratch for classifying up to max_n particles of one slab. */
FORGE_API int forge_slab_create(uint64_t max_n, int device, forge_slab** out);
FORGE_API void forge_slab_destroy(forge_slab* h);

/* Ordered selection against the slab [lo, hi). flags: 1 = has a left
 * neighbour, 2 = has a right neighbour, 4 = halo mode, 8 = (halo mode)
 * in-slab rows only.
 *   migrate mode: L = {i : x[i] < lo}, R = {i : x[i] >= hi}, A = L u R
 *   halo mode:    L = {i : x[i] < lo + reach}, R = {i : x[i] >= hi - reach}, A = {}
 *   with 8:       L = {i : lo <= x[i] < lo + reach}, R = {i : hi - reach <= x[i] < hi}
 * (L only with a left neighbour, R only with a right one). idx_out receives
 * [A | L | R], each ascending -- at most 2n entries, so it must hold 2n;
 * counts[3] (device) = |A|, |L|, |R|. */
FORGE_API int forge_slab_classify(forge_slab* h, const float* x, uint64_t n, float lo, float hi, float reach,
                                  uint32_t flags, uint32_t* idx_out, uint32_t* counts, void* stream);

/* x-histogram of n particles for load balancing (no reference
 * counterpart): out[b] (bins doubles, device) = sum of w[i] (1 when w is
 * NULL; negative weights count 0) over the particles whose x lies in bin b
 * of [lo, hi), x below/above in the end bins. Summed in 2^-16 fixed point
 * with 64-bit integer atomics: the same inputs give the same histogram
 * bit for bit. bins <= 4096. */
FORGE_API int forge_slab_x_hist(forge_slab* h, const float* x, const float* w, uint64_t n, float lo, float hi,
                                uint32_t bins, double* out, void* stream);

/* Remove the k columns gone[] (ascending, < n) from a row-major rows x ld
 * float buffer holding n live columns: surviving columns among the last k
 * move into the holes, so the live columns become [0, n - k). */
FORGE_API int forge_slab_compact(float* cols, uint64_t ld, uint32_t rows, uint64_t n, const uint32_t* gone,
                                 uint64_t k, void* stream);

/* Neighbour exchange of the sharded SPH step over the library's own NCCL
 * communicator (libnccl.so.2 is loaded at run time; single-GPU use needs no
 * NCCL). One rank per GPU owns the x-slab [lo, hi); particle state is a
 * row-major 7 x ld float buffer (rows x, y, z, vx, vy, vz, id bits), owned
 * columns first, ghosts after them. No counterpart in the reference. */
typedef struct forge_slab_comm forge_slab_comm;

/* NCCL unique id (128 bytes) made on one rank and shared by the caller. */
FORGE_API int forge_nccl_unique_id(uint8_t* out);

/* Creates the communicator (collective over all ranks) and buffers for up
 * to `capacity` particles per message / per classification. reach = halo
 * width (h, with a small margin). */
FORGE_API int forge_slab_comm_create(const uint8_t* id, int rank, int world, int device, uint64_t capacity,
                                     float lo, float hi, float reach, forge_slab_comm** out);
FORGE_API void forge_slab_comm_destroy(forge_slab_comm* c);

/* Failure detection: every host wait of the exchange (the message sizes)
 * polls with a deadline, default 60 s. Past it -- a neighbour that stopped
 * answering -- or on an asynchronous NCCL error the call aborts the
 * communicator (ending this rank's pending NCCL kernels) and returns
 * FORGE_ERR_TIMEOUT / FORGE_ERR_NCCL; every later exchange call on it fails. */
FORGE_API int forge_slab_comm_set_timeout(forge_slab_comm* c, double seconds);

/* Moves this rank's slab to [lo, hi) (load balancing). The next round 1
 * (forge_slab_exchange with migrate = 1) sends every owned particle outside
 * it to the neighbour: callers keep each new bound between the old
 * neighbouring bounds, so no particle moves more than one slab, and every
 * slab at least 2 * reach wide, so halos come from direct neighbours only. */
FORGE_API int forge_slab_comm_set_bounds(forge_slab_comm* c, float lo, float hi);

/* Round 1 (after a step's force pass, or once at start with migrate = 0):
 * migrants (x outside the slab) leave the owned columns and go to the
 * neighbour, together with the halo rows (owned particles within reach of a
 * face); arrivals are appended to the owned columns, then the ghosts.
 * Synchronises `stream` once (the exchanged message sizes). */
FORGE_API int forge_slab_exchange(forge_slab_comm* c, float* cols, uint64_t ld, uint64_t n_own, int migrate,
                                  uint64_t* n_own_out, uint64_t* n_ghost_out, void* stream);

/* Round 1 split for overlap with the interior force pass (same result as
 * forge_slab_exchange with migrate = 1, up to the order of the halo rows):
 *   stream B: forge_sph_force_step_zone(BOUNDARY)
 *             forge_slab_exchange_begin   classify + pack migrants and halo
 *                                         rows, exchange the counts
 *   stream A: forge_sph_force_step_zone(INTERIOR)
 *             forge_slab_exchange_end     wait (host) for the counts, send the
 *                                         payload on stream B, then on stream
 *                                         A: remove the migrants, append
 *                                         arrivals and ghosts.
 * Halo rows are taken among the owned particles still in the slab
 * (lo <= x < lo + reach, hi - reach <= x < hi), so begin may read the
 * columns while the interior pass writes particles at least `reach` away
 * from both faces (the zone's guard). No call on `c` may come between the
 * two; stream B should have a high priority. */
FORGE_API int forge_slab_exchange_begin(forge_slab_comm* c, const float* cols, uint64_t ld, uint64_t n_own,
                                        void* stream);
FORGE_API int forge_slab_exchange_end(forge_slab_comm* c, float* cols, uint64_t ld, uint64_t* n_own_out,
                                      uint64_t* n_ghost_out, void* stream);

/* Round 2 (after density): every ghost receives its owner's density in
 * rho[] (indexed like the columns). No host synchronisation. */
FORGE_API int forge_slab_exchange_rho(forge_slab_comm* c, float* rho, void* stream);

/* ------------------------------------------------------------------------ */
/* Field I/O (manifest_runner.rs:192-269 init_fields, :83-92 the result     */
/* gather). A handle owns a pinned host staging buffer (6 x max_n floats)   */
/* and a device one (3 x max_n): pageable host arrays are copied through    */
/* the pinned buffer, pinned ones are copied directly; Vec3f AoS <-> SoA    */
/* conversion runs on the GPU. Uploads are asynchronous on `stream` (a      */
/* pageable source may be reused when the call returns); downloads return   */
/* once the data are in the host arrays. One handle per thread at a time.   */
/* ------------------------------------------------------------------------ */
typedef struct forge_io forge_io;
FORGE_API int forge_io_create(uint64_t max_n, int device, forge_io** out);
FORGE_API void forge_io_destroy(forge_io* io);
/* nfields (<= 6) float columns of n values: host[f] -> dev[f]. Replaces the
 * per-column Array::from_vec uploads of init_fields (manifest_runner.rs:205-213). */
FORGE_API int forge_io_upload(forge_io* io, const float* const* host, float* const* dev, uint32_t nfields,
                              uint64_t n, void* stream);
/* dev[f] -> host[f] (Array::to_vec, array.rs, as the result gather uses
 * it). If every host array is page-locked the copies are only enqueued on
 * `stream` (the caller synchronises, and can overlap them with uploads on
 * another stream); otherwise the call returns when the host arrays hold the
 * data. */
FORGE_API int forge_io_download(forge_io* io, const float* const* dev, float* const* host, uint32_t nfields,
                                uint64_t n, void* stream);
/* Vec3f AoS host array (n x 3 floats, the layout init_vec3 produces,
 * manifest_runner.rs:268-310) -> x, y, z device columns. */
FORGE_API int forge_io_upload_vec3(forge_io* io, const float* xyz, float* x, float* y, float* z, uint64_t n,
                                   void* stream);
/* x, y, z device columns -> interleaved n x 3 host array (the SimResult
 * positions of manifest_runner.rs:83-92); returns when the data are there. */
FORGE_API int forge_io_download_vec3(forge_io* io, const float* x, const float* y, const float* z, float* xyz,
                                     uint64_t n, void* stream);

/* Neighbour-pass kernel family of a grid's density and force passes (no
 * reference counterpart: the reference has one thread per particle). AUTO
 * (the default) takes per-thread walks for large particle counts and row
 * walks below 2^18 particles, where per-thread walks leave most of the GPU
 * idle; the others force one family, for tests and benchmarks. Every family
 * meets the parity tolerances and is deterministic run to run. Per-thread
 * walks sum each particle's pairs in the reference's order (bit-identical
 * whatever the other particles of the thread); row walks sum each of the
 * nine rows in that order and add the nine partial sums in row order (the
 * same whatever the other particles, so bit-identical across cell orders,
 * zone lists and shards too); group walks sum a particle's lanes in a fixed
 * tree whose lane split depends on the particles that share its warp, so the
 * same particle can round differently in another cell order. */
#define FORGE_WALK_AUTO 0
#define FORGE_WALK_THREAD 1  /* one, two or four particles per thread */
#define FORGE_WALK_GROUP4 2  /* warp-cooperative: 4 particles per warp, 8 lanes each */
#define FORGE_WALK_GROUP8 3  /* 8 particles per warp, 4 lanes each */
#define FORGE_WALK_GROUP16 4 /* 16 particles per warp, 2 lanes each */
#define FORGE_WALK_ROWS 5    /* nine threads per particle, one per neighbour row */
#define FORGE_WALK_TILE 6    /* density: cell-block CTAs, neighbour rows staged in shared memory by TMA
                              * (slower than THREAD on every measured case; force passes as THREAD) */
FORGE_API int forge_grid_set_walk(forge_grid* g, int walk);

/* x-window of a grid (no reference counterpart; for a shard of an x-slab
 * decomposition): builds index only global cells [cx0, cx0 + nxw) along x,
 * so the cell-start table and its build shrink with the shard. Cells are
 * still assigned on the global grid (floor and clamp of hashgrid.rs:128-139
 * / sph_fused.rs:91-99), then shifted; neighbour windows are clipped at the
 * window's edges as at the grid's. The caller keeps every particle it builds
 * inside the window (a shard's owned particles and ghosts, plus one cell of
 * margin each side for the ghosts' neighbours). Resets the last build;
 * forge_grid_query needs the whole grid. Default: the whole grid. */
FORGE_API int forge_grid_set_x_window(forge_grid* g, uint32_t cx0, uint32_t nxw);

/* ------------------------------------------------------------------------ */
/* Benchmark aid (no reference counterpart; the reference only times the    */
/* whole run with a wall clock, manifest_runner.rs:40-80).                  */
/* ------------------------------------------------------------------------ */

/* Record CUDA events at the phase boundaries of each forge_sph_step call
 * (a ring of max_steps steps; 0 disables). Not for use under stream capture. */
FORGE_API int forge_grid_profile_enable(forge_grid* g, uint32_t max_steps);

/* Synchronise and write the phase times (ms) of the recorded steps, oldest
 * first: out[s*4 + k] with k = 0 hash + radix sort, 1 cell table + gather,
 * 2 density, 3 force + epilogue. *steps receives the count written
 * (<= cap_steps). Clears the ring. */
FORGE_API int forge_grid_profile_read(forge_grid* g, float* out, uint32_t cap_steps, uint32_t* steps);

#ifdef __cplusplus
}
#endif

#endif /* FORGE_SPH_H */
