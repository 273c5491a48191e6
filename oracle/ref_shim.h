/* Host shim for the reference's CUDA C kernel strings (test infrastructure).
 *
 * oracle/ref_extract.py copies the reference's kernels, unmodified, into the
 * git-ignored oracle/_ref/ref_kernels.cpp, which includes this header and is
 * compiled with g++ as ordinary C++ functions: one call runs one CUDA thread.
 * A launch is a loop over the thread index; the driver (ref_driver.cpp) sets
 * blockIdx.x = i with blockDim = (1,1,1) and threadIdx = (0,0,0), so
 * `blockIdx.x * blockDim.x + threadIdx.x` is i. Compiled with
 * -ffp-contract=off: every float operation rounds as written (NVRTC's default
 * would contract a*b+c into FMAs on the GPU; the difference is the ulp-level
 * rounding the parity tolerances cover).
 */
#pragma once
#include <math.h>
#include <stdint.h>

struct ref_dim3 {
    unsigned int x, y, z;
};

extern thread_local ref_dim3 blockIdx;
static const ref_dim3 blockDim = {1u, 1u, 1u};
static const ref_dim3 threadIdx = {0u, 0u, 0u};

#define __global__
#define __device__
#define __forceinline__ inline

/* Only the serial grid-build launches use it (count_cells, scatter_particles):
 * threads run one after another in index order, so a plain add is what the
 * atomic does, and the scatter comes out in ascending index within a cell. */
static inline unsigned int atomicAdd(unsigned int* p, unsigned int v) {
    const unsigned int old = *p;
    *p = old + v;
    return old;
}
