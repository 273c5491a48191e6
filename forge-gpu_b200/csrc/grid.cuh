// Uniform hash grid kernels (sm_100a): cell hashing, the cell-start table,
// the cell-ordered particle gather, find_cell_boundaries and the batched
// neighbour query.
#pragma once

#include "common.cuh"

namespace forge {
namespace grid {

struct GridGeom {
    float ox, oy, oz;  // origin (0 for the SPH modules)
    float cs;          // cell size
    int nx, ny, nz;
    // x-window of the table: global cells [cx0, cx0 + nxw) (a shard's slab;
    // the whole grid by default). Cells are assigned globally (the
    // reference's floor and clamp), then shifted into the window.
    int cx0, nxw;
};

// Saturating float -> int as Rust's `as i32` and CUDA's cvt.rzi.s32 do
// (NaN -> 0). floorf() already rounded, so this is the truncating convert.
__device__ __forceinline__ int floor_to_int(float v) { return (int)floorf(v); }

// Cell of a position: hashgrid.rs:128-139 (origin subtracted, floor, clamp,
// x-fastest linear index); with origin 0 this is sph_fused.rs:91-99 exactly,
// since (x - 0.0f) == x. The divide is IEEE (no fast-math), which keeps the
// cell index bit-exact with the CPU.
__device__ __forceinline__ uint32_t cell_of(float x, float y, float z, const GridGeom& g) {
    int cx = floor_to_int((x - g.ox) / g.cs);
    int cy = floor_to_int((y - g.oy) / g.cs);
    int cz = floor_to_int((z - g.oz) / g.cs);
    cx = cx < 0 ? 0 : (cx >= g.nx ? g.nx - 1 : cx);
    cy = cy < 0 ? 0 : (cy >= g.ny ? g.ny - 1 : cy);
    cz = cz < 0 ? 0 : (cz >= g.nz ? g.nz - 1 : cz);
    cx -= g.cx0;  // the caller keeps every particle inside the window; clamped for safety
    cx = cx < 0 ? 0 : (cx >= g.nxw ? g.nxw - 1 : cx);
    return (uint32_t)cx + (uint32_t)cy * (uint32_t)g.nxw + (uint32_t)cz * (uint32_t)g.nxw * (uint32_t)g.ny;
}

// Sub-slice of a position inside its (clamped) cell along x: the cell is cut
// into 2^sub_bits slabs. fx - cx is exact (the fractional part of a float is
// representable), so slice = floor(2^sub_bits * fx) - 2^sub_bits * cx for
// positions inside the grid; clamped positions land in the edge slice.
__device__ __forceinline__ uint32_t slice_of(float x, const GridGeom& g, uint32_t sub_bits) {
    const float fx = (x - g.ox) / g.cs;
    int cx = floor_to_int(fx);
    cx = cx < 0 ? 0 : (cx >= g.nx ? g.nx - 1 : cx);
    const int S = 1 << sub_bits;
    int s = floor_to_int((fx - (float)cx) * (float)S);
    return (uint32_t)(s < 0 ? 0 : (s >= S ? S - 1 : s));
}

// Histogram key source that hashes positions and stores the key:
// cell << sub_bits | x-slice (sub_bits = 0: the plain cell index).
// stride 1: SoA (px, py, pz separate); stride 3: Vec3f AoS (px = xyz).
struct HashKeys {
    const float* __restrict__ px;
    const float* __restrict__ py;
    const float* __restrict__ pz;
    uint32_t stride;
    GridGeom g;
    uint32_t* __restrict__ keys_out;
    uint32_t sub_bits;
    __device__ __forceinline__ uint32_t operator()(uint32_t i) const {
        const size_t o = (size_t)i * stride;
        const float x = px[o];
        uint32_t c = cell_of(x, py[o], pz[o], g);
        if (sub_bits) c = (c << sub_bits) | slice_of(x, g, sub_bits);
        keys_out[i] = c;
        return c;
    }
    // keys of particles i0 .. i0+7 (i0 a multiple of 8; missing ones 0):
    // 16-byte loads and stores for aligned SoA columns
    __device__ __forceinline__ void load8(uint32_t i0, uint32_t n, uint32_t (&k)[8]) const {
        const uintptr_t al = reinterpret_cast<uintptr_t>(px) | reinterpret_cast<uintptr_t>(py) |
                             reinterpret_cast<uintptr_t>(pz) | reinterpret_cast<uintptr_t>(keys_out);
        if (stride == 1 && i0 + 8 <= n && (al & 15u) == 0) {
            float x[8], y[8], z[8];
            *reinterpret_cast<float4*>(x) = __ldg(reinterpret_cast<const float4*>(px + i0));
            *reinterpret_cast<float4*>(x + 4) = __ldg(reinterpret_cast<const float4*>(px + i0) + 1);
            *reinterpret_cast<float4*>(y) = __ldg(reinterpret_cast<const float4*>(py + i0));
            *reinterpret_cast<float4*>(y + 4) = __ldg(reinterpret_cast<const float4*>(py + i0) + 1);
            *reinterpret_cast<float4*>(z) = __ldg(reinterpret_cast<const float4*>(pz + i0));
            *reinterpret_cast<float4*>(z + 4) = __ldg(reinterpret_cast<const float4*>(pz + i0) + 1);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t c = cell_of(x[j], y[j], z[j], g);
                if (sub_bits) c = (c << sub_bits) | slice_of(x[j], g, sub_bits);
                k[j] = c;
            }
            reinterpret_cast<uint4*>(keys_out + i0)[0] = make_uint4(k[0], k[1], k[2], k[3]);
            reinterpret_cast<uint4*>(keys_out + i0)[1] = make_uint4(k[4], k[5], k[6], k[7]);
            return;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) k[j] = i0 + j < n ? (*this)(i0 + j) : 0u;
    }
};

// Fill value `v` into table[a..b] (inclusive, empty if a > b) with the whole
// warp helping on long runs. Every lane of the warp must call this.
__device__ __forceinline__ void warp_fill_runs(uint32_t* __restrict__ table, int64_t a, int64_t b,
                                               uint32_t v) {
    const int lane = threadIdx.x & 31;
    const int64_t len = b - a + 1;
    const bool longrun = len > 8;
    if (!longrun) {
        for (int64_t c = a; c <= b; ++c) table[c] = v;
    }
    uint32_t todo = __ballot_sync(0xffffffffu, longrun);
    while (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        const int64_t la = __shfl_sync(0xffffffffu, a, src);
        const int64_t lb = __shfl_sync(0xffffffffu, b, src);
        const uint32_t lv = __shfl_sync(0xffffffffu, v, src);
        for (int64_t c = la + lane; c <= lb; c += 32) table[c] = lv;
    }
}

// cell_start[c] = first sorted position whose key >= c, for c in [0, C],
// so cell_start[C] == n (sph_fused.rs:280-390 without the scan or memsets).
// Thread s in [0, n] owns the cells (key[s-1], key[s]]. A run longer than
// two chunks of kFillChunk entries (a large empty region: the space around
// a dam-break column, the cells past the last particle) is not written by
// one warp: the thread writes its partial first chunk and the chunk holding
// key[s], and marks the whole chunks between them in chunk_val[] for
// fill_chunks_kernel, which writes them one block per chunk. Entries are
// written once, except that whole chunks of a run may be written twice with
// the same value; the table needs no clearing.
// Also zeroes the sort's histograms and tile counters for the next build.
// Optionally gathers positions (and velocities) into cell order:
//   pos4[s] = (x, y, z, bits(key)), vel4[s] = (vx, vy, vz, 0).
struct GatherSrc {
    const float* __restrict__ px;
    const float* __restrict__ py;
    const float* __restrict__ pz;
    uint32_t stride;
    const float* __restrict__ vx;  // nullable
    const float* __restrict__ vy;
    const float* __restrict__ vz;
};

constexpr uint32_t kFillChunk = 1024;
constexpr uint32_t kChunkFree = 0xffffffffu;  // chunk_val: not marked

__global__ void __launch_bounds__(256)
    cell_start_gather_kernel(const uint32_t* __restrict__ skeys, const uint32_t* __restrict__ svals,
                             uint32_t n, uint32_t C, uint32_t* __restrict__ cell_start, GatherSrc src,
                             float4* __restrict__ pos4, float4* __restrict__ vel4, uint32_t* __restrict__ chunk_val,
                             uint32_t* __restrict__ sort_meta, uint32_t sort_meta_words) {
    pdl_enter();
    // the build's sort is done with its digit histograms and tile counters:
    // zero them for the next build's sort (no memset node between builds)
    if (blockIdx.x == 0)
        for (uint32_t j = threadIdx.x; j < sort_meta_words; j += blockDim.x) sort_meta[j] = 0u;
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    int64_t a = 1, b = 0;  // empty
    uint32_t key = 0;
    if (s <= n) {
        if (s < n) key = skeys[s];
        a = (s == 0) ? 0 : (int64_t)skeys[s - 1] + 1;
        b = (s == n) ? (int64_t)C : (int64_t)key;
    }
    constexpr int64_t K = kFillChunk;
    int64_t a2 = 1, b2 = 0, ca = 1, cb = 0;  // second piece; whole chunks [ca, cb]
    if (b - a + 1 > 2 * K) {
        ca = (a + K - 1) / K;   // first whole chunk
        cb = b / K - 1;         // last whole chunk before the one holding b
        a2 = (b / K) * K;
        b2 = b;
        b = ca * K - 1;
    }
    warp_fill_runs(cell_start, a, b, s);
    warp_fill_runs(cell_start, a2, b2, s);
    warp_fill_runs(chunk_val, ca, cb, s);
    if (s < n && pos4 != nullptr) {
        const uint32_t i = svals[s];
        const size_t o = (size_t)i * src.stride;
        pos4[s] = make_float4(src.px[o], src.py[o], src.pz[o], __uint_as_float(key));
        if (vel4 != nullptr) vel4[s] = make_float4(src.vx[i], src.vy[i], src.vz[i], 0.f);
    }
}

// Whole chunks marked by cell_start_gather_kernel: block per chunk (grid-
// stride), marks cleared for the next build.
__global__ void __launch_bounds__(256)
    fill_chunks_kernel(uint32_t* __restrict__ cell_start, uint32_t* __restrict__ chunk_val, uint32_t chunks) {
    pdl_enter();
    for (uint32_t k = blockIdx.x; k < chunks; k += gridDim.x) {
        const uint32_t v = chunk_val[k];
        if (v == kChunkFree) continue;  // uniform per block
        uint4* t = reinterpret_cast<uint4*>(cell_start + (size_t)k * kFillChunk);
        for (uint32_t j = threadIdx.x; j < kFillChunk / 4; j += blockDim.x) t[j] = make_uint4(v, v, v, v);
        __syncthreads();
        if (threadIdx.x == 0) chunk_val[k] = kChunkFree;
    }
}

// find_cell_boundaries (radix_sort.rs:444-466 plus the two fills :259-293)
// in one pass: thread s in [0, n] handles the boundary between sorted
// positions s-1 and s, and the empty cells strictly between their ids.
__global__ void __launch_bounds__(256)
    cell_bounds_kernel(const uint32_t* __restrict__ ids, uint32_t n, uint32_t C,
                       uint32_t* __restrict__ start, uint32_t* __restrict__ end, uint32_t* err) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    int64_t a = 1, b = 0;
    if (s <= n) {
        int64_t prev = -1, cur = C;
        if (s > 0) prev = min((int64_t)ids[s - 1], (int64_t)C);
        if (s < n) {
            const uint32_t id = ids[s];
            if (id >= C) atomicOr(err, kDevKeyRange);
            cur = min((int64_t)id, (int64_t)C);
        }
        if (prev != cur) {
            if (prev >= 0 && prev < C) end[prev] = s;
            if (cur < C) start[cur] = s;
        }
        a = prev + 1;
        b = min(cur, (int64_t)C) - 1;
    }
    warp_fill_runs(start, a, b, 0xffffffffu);
    warp_fill_runs(end, a, b, 0u);
}

// ---------------------------------------------------------------------------
// Batched neighbour query, hashgrid.rs:145-193: cell of the query WITHOUT
// clamping, 3x3x3 walk dz, dy, dx, hits where dist^2 <= r^2 with
// diff = p - q. Pass 1 counts, pass 2 (after a scan) writes hits.
// ---------------------------------------------------------------------------
template <bool WRITE>
__global__ void __launch_bounds__(128)
    query_kernel(const float* __restrict__ px, const float* __restrict__ py, const float* __restrict__ pz,
                 const float* __restrict__ qx, const float* __restrict__ qy, const float* __restrict__ qz,
                 uint32_t nq, float r2, GridGeom g, const uint32_t* __restrict__ cell_start,
                 const uint32_t* __restrict__ sorted_idx, uint32_t* __restrict__ counts,
                 const uint32_t* __restrict__ offsets, uint32_t* __restrict__ hits, uint64_t max_hits,
                 uint32_t* err) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    const float x = qx[q], y = qy[q], z = qz[q];
    const int cx = floor_to_int((x - g.ox) / g.cs);
    const int cy = floor_to_int((y - g.oy) / g.cs);
    const int cz = floor_to_int((z - g.oz) / g.cs);
    uint64_t out = 0;
    if (WRITE) {
        out = offsets[q];
        if (out + counts[q] > max_hits) {
            atomicOr(err, kDevCapacity);
            return;
        }
    }
    uint32_t cnt = 0;
    for (int dz = -1; dz <= 1; ++dz) {
        for (int dy = -1; dy <= 1; ++dy) {
            for (int dx = -1; dx <= 1; ++dx) {
                // (int64 to avoid overflow for far-away queries)
                const int64_t nxx = (int64_t)cx + dx, nyy = (int64_t)cy + dy, nzz = (int64_t)cz + dz;
                if (nxx < 0 || nyy < 0 || nzz < 0) continue;
                if (nxx >= g.nx || nyy >= g.ny || nzz >= g.nz) continue;
                const uint32_t cell = (uint32_t)nxx + (uint32_t)nyy * (uint32_t)g.nx +
                                      (uint32_t)nzz * (uint32_t)g.nx * (uint32_t)g.ny;
                const uint32_t b = cell_start[cell], e = cell_start[cell + 1];
                for (uint32_t s = b; s < e; ++s) {
                    const uint32_t j = sorted_idx[s];
                    const float ddx = px[j] - x, ddy = py[j] - y, ddz = pz[j] - z;
                    // every product and sum rounded on its own, as hashgrid.rs:183-184
                    // evaluates it (no FMA contraction), so d2 <= r2 is decided
                    // exactly as the reference decides it, also at d2 == r2
                    const float d2 = __fadd_rn(__fadd_rn(__fmul_rn(ddx, ddx), __fmul_rn(ddy, ddy)), __fmul_rn(ddz, ddz));
                    if (d2 <= r2) {
                        if (WRITE) hits[out + cnt] = j;
                        ++cnt;
                    }
                }
            }
        }
    }
    if (!WRITE) counts[q] = cnt;
}

// Three-phase exclusive scan of u32 counts (tile sums, scan of the sums in
// one block, rescan of each tile); out[n] receives the total.
constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;

__global__ void __launch_bounds__(kScanThreads)
    scan_tile_sums_kernel(const uint32_t* __restrict__ in, uint32_t n, uint32_t* __restrict__ sums) {
    __shared__ uint32_t s_scan[kScanThreads / 32 + 1];
    const uint32_t base = blockIdx.x * kScanTile + threadIdx.x * kScanItems;
    uint32_t acc = 0;
    for (int k = 0; k < kScanItems; ++k)
        if (base + k < n) acc += in[base + k];
    uint32_t total;
    block_exclusive_scan<kScanThreads>(acc, s_scan, &total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(1024) scan_sums_kernel(uint32_t* __restrict__ sums, uint32_t m) {
    __shared__ uint32_t s_scan[1024 / 32 + 1];
    uint32_t carry = 0;
    for (uint32_t base = 0; base < m; base += 1024) {
        const uint32_t i = base + threadIdx.x;
        const uint32_t v = i < m ? sums[i] : 0u;
        uint32_t total;
        const uint32_t ex = block_exclusive_scan<1024>(v, s_scan, &total);
        if (i < m) sums[i] = carry + ex;
        carry += total;
    }
}

__global__ void __launch_bounds__(kScanThreads)
    scan_apply_kernel(const uint32_t* __restrict__ in, uint32_t n, const uint32_t* __restrict__ sums,
                      uint32_t* __restrict__ out) {
    __shared__ uint32_t s_scan[kScanThreads / 32 + 1];
    const uint32_t base = blockIdx.x * kScanTile + threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    uint32_t acc = 0;
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = (base + k < n) ? in[base + k] : 0u;
        acc += v[k];
    }
    uint32_t total;
    uint32_t run = sums[blockIdx.x] + block_exclusive_scan<kScanThreads>(acc, s_scan, &total);
    for (int k = 0; k < kScanItems; ++k) {
        if (base + k < n) out[base + k] = run;
        run += v[k];
    }
    if (base < n && base + kScanItems >= n) out[n] = run;
}

}  // namespace grid
}  // namespace forge
