// Slab-exchange helpers for the sharded SPH step (sm_100a): ordered
// selection of the particles that leave a slab or lie within h of its faces,
// and in-place removal of leaving particles from a column buffer. Integer /
// byte work, HBM-bound; deterministic (every list comes out in ascending
// particle order, no atomics on positions).
#pragma once

#include "common.cuh"

namespace forge {
namespace slab {

constexpr int kThreads = 256;
constexpr int kItems = 16;
constexpr int kTile = kThreads * kItems;
constexpr int kLists = 3;  // A (either side), L (left), R (right)

struct ClassifyArgs {
    float lo, hi, reach;
    uint32_t flags;  // 1 has left neighbour, 2 has right neighbour, 4 halo mode (else migrate mode),
                     // 8 (halo mode) in-slab rows only: lo <= x on the left, x < hi on the right
};

// Membership bits of element x in lists A, L, R.
__device__ __forceinline__ uint32_t member_bits(float x, const ClassifyArgs& a) {
    const bool halo = a.flags & 4u, in_slab = a.flags & 8u;
    const bool l = (a.flags & 1u) && (halo ? x < a.lo + a.reach && (!in_slab || x >= a.lo) : x < a.lo);
    const bool r = (a.flags & 2u) && (halo ? x >= a.hi - a.reach && (!in_slab || x < a.hi) : x >= a.hi);
    const bool all = !halo && (l || r);
    return (all ? 1u : 0u) | (l ? 2u : 0u) | (r ? 4u : 0u);
}

// Membership of element i by its x coordinate (the slab lists).
struct XMember {
    const float* __restrict__ x;
    ClassifyArgs a;
    __device__ __forceinline__ uint32_t operator()(uint32_t i) const { return member_bits(x[i], a); }
};

// Pass 1: per-tile counts of each list.
template <class M>
__global__ void __launch_bounds__(kThreads)
    classify_count_kernel(M m, uint32_t n, const uint32_t* __restrict__ n_sub, uint32_t* __restrict__ tile_counts) {
    __shared__ uint32_t s[kLists];
    if (n_sub) n -= *n_sub;  // live length known only on the device
    if (threadIdx.x < kLists) s[threadIdx.x] = 0;
    __syncthreads();
    uint32_t c[kLists] = {0, 0, 0};
    const uint32_t base = blockIdx.x * kTile;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = base + k * kThreads + threadIdx.x;
        if (i < n) {
            const uint32_t b = m(i);
#pragma unroll
            for (int l = 0; l < kLists; ++l) c[l] += (b >> l) & 1u;
        }
    }
#pragma unroll
    for (int l = 0; l < kLists; ++l) {
        uint32_t v = c[l];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((threadIdx.x & 31) == 0 && v) atomicAdd(&s[l], v);
    }
    __syncthreads();
    if (threadIdx.x < kLists) tile_counts[blockIdx.x * kLists + threadIdx.x] = s[threadIdx.x];
}

// Pass 2 (one block): exclusive scan of the tile counts per list, list totals
// to counts[0..2], and each list's start in the packed output.
__global__ void __launch_bounds__(1024)
    classify_scan_kernel(uint32_t* __restrict__ tile_counts, uint32_t tiles, uint32_t* __restrict__ counts) {
    __shared__ uint32_t s_scan[1024 / 32 + 1];
    __shared__ uint32_t s_tot[kLists];
    for (int l = 0; l < kLists; ++l) {
        uint32_t carry = 0;
        for (uint32_t b = 0; b < tiles; b += 1024) {
            const uint32_t t = b + threadIdx.x;
            const uint32_t v = t < tiles ? tile_counts[t * kLists + l] : 0u;
            uint32_t total;
            const uint32_t ex = block_exclusive_scan<1024>(v, s_scan, &total);
            if (t < tiles) tile_counts[t * kLists + l] = carry + ex;
            carry += total;
        }
        if (threadIdx.x == 0) s_tot[l] = carry;
        __syncthreads();
    }
    if (threadIdx.x < kLists) counts[threadIdx.x] = s_tot[threadIdx.x];
}

// Pass 3: write each list's element indices in ascending order, packed as
// [A | L | R].
template <class M>
__global__ void __launch_bounds__(kThreads)
    classify_write_kernel(M m, uint32_t n, const uint32_t* __restrict__ n_sub,
                          const uint32_t* __restrict__ tile_offsets, const uint32_t* __restrict__ counts,
                          uint32_t* __restrict__ out) {
    __shared__ uint32_t s_scan[kThreads / 32 + 1];
    if (n_sub) n -= *n_sub;
    const uint32_t base = blockIdx.x * kTile + threadIdx.x * kItems;  // blocked: thread owns 16 consecutive
    uint32_t bits[kItems];
    uint32_t c[kLists] = {0, 0, 0};
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = base + k;
        bits[k] = i < n ? m(i) : 0u;
#pragma unroll
        for (int l = 0; l < kLists; ++l) c[l] += (bits[k] >> l) & 1u;
    }
    uint32_t start = 0;
#pragma unroll
    for (int l = 0; l < kLists; ++l) {
        uint32_t total;
        uint32_t pos = block_exclusive_scan<kThreads>(c[l], s_scan, &total) + tile_offsets[blockIdx.x * kLists + l] +
                       start;
        start += counts[l];
#pragma unroll
        for (int k = 0; k < kItems; ++k)
            if ((bits[k] >> l) & 1u) out[pos++] = base + k;
    }
}

// Remove columns `gone` (ascending, k of them, all < n) from a row-major
// (rows x ld) buffer of n live columns: the surviving columns among the last k
// move into the holes below n - k, in ascending order. One block.
__global__ void __launch_bounds__(1024)
    compact_kernel(float* __restrict__ cols, uint64_t ld, uint32_t rows, uint32_t n, const uint32_t* __restrict__ gone,
                   uint32_t k, const uint32_t* __restrict__ k_dev) {
    __shared__ uint32_t s_scan[1024 / 32 + 1];
    if (k_dev) k = *k_dev;
    const uint32_t keep = n - k;
    uint32_t carry = 0;  // fillers ranked so far
    for (uint32_t b = 0; b < k; b += 1024) {
        const uint32_t t = keep + b + threadIdx.x;  // tail column
        bool fill = false;
        if (b + threadIdx.x < k) {
            // t is a filler unless it is in `gone` (binary search)
            uint32_t lo = 0, hi = k;
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (gone[mid] < t) lo = mid + 1;
                else hi = mid;
            }
            fill = !(lo < k && gone[lo] == t);
        }
        uint32_t total;
        const uint32_t r = carry + block_exclusive_scan<1024>(fill ? 1u : 0u, s_scan, &total);
        if (fill) {
            const uint32_t dst = gone[r];  // the r-th hole (holes are the smallest entries of gone)
            for (uint32_t row = 0; row < rows; ++row) cols[row * ld + dst] = cols[row * ld + t];
        }
        carry += total;
    }
}

}  // namespace slab
}  // namespace forge

namespace forge {
namespace slab {

// x-histogram for load balancing: out[b] += weight of each particle whose x
// falls in bin b of [lo, hi) (clamped to the end bins; weight 1 when w is
// NULL). Weights are summed as fixed point (2^-16 units) in 64-bit
// integers, so the result does not depend on the order of the atomics and
// every rank computes the same bounds from the same all-reduced histogram.
constexpr uint32_t kHistMaxBins = 4096;
constexpr double kHistScale = 65536.0;

__global__ void __launch_bounds__(256)
    x_hist_kernel(const float* __restrict__ x, const float* __restrict__ w, uint32_t n, double lo, double scale,
                  uint32_t bins, unsigned long long* __restrict__ acc) {
    __shared__ unsigned long long s[kHistMaxBins];
    for (uint32_t b = threadIdx.x; b < bins; b += blockDim.x) s[b] = 0ull;
    __syncthreads();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const double f = floor(((double)x[i] - lo) * scale);
        const uint32_t b = f < 0.0 ? 0u : (f >= (double)(bins - 1) ? bins - 1 : (uint32_t)f);
        const unsigned long long q = w ? (unsigned long long)((double)fmaxf(w[i], 0.f) * kHistScale + 0.5) : 65536ull;
        atomicAdd(&s[b], q);
    }
    __syncthreads();
    for (uint32_t b = threadIdx.x; b < bins; b += blockDim.x)
        if (s[b]) atomicAdd(&acc[b], s[b]);
}

__global__ void x_hist_finish_kernel(const unsigned long long* __restrict__ acc, uint32_t bins, double* __restrict__ out) {
    for (uint32_t b = blockIdx.x * blockDim.x + threadIdx.x; b < bins; b += gridDim.x * blockDim.x)
        out[b] = (double)acc[b] / kHistScale;
}

}  // namespace slab
}  // namespace forge

namespace forge {
namespace slab {

// Packs list `list` (1 = L, 2 = R) of a classification [A | L | R] with
// device-side sizes counts[3] into records at out + *rec0_dev (0 if null),
// optionally copying the column indices to idx_copy. Grid-stride: the sizes
// are not known on the host.
__global__ void __launch_bounds__(256)
    pack_dev_kernel(const float* __restrict__ cols, uint64_t ld, uint32_t rows, const uint32_t* __restrict__ idx,
                    const uint32_t* __restrict__ counts, int list, const uint32_t* __restrict__ rec0_dev,
                    float* __restrict__ out, uint32_t* __restrict__ idx_copy) {
    const uint32_t off = counts[0] + (list == 2 ? counts[1] : 0u);
    const uint32_t cnt = counts[list], rec0 = rec0_dev ? *rec0_dev : 0u;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < cnt * rows; t += gridDim.x * blockDim.x) {
        const uint32_t i = t / rows, r = t - i * rows;
        const uint32_t col = idx[off + i];
        out[(size_t)(rec0 + i) * rows + r] = cols[r * ld + col];
        if (idx_copy && r == 0) idx_copy[i] = col;
    }
}

// Column indices taken before compact_kernel(gone, k) -> after it: an index
// t >= keep = n - k (t not in gone) is the r-th surviving tail column, r =
// (t - keep) - |gone in [keep, t)|, and moved to the r-th hole gone[r].
// Remaps lists a (na entries) and b (nb) in place; k is read from *k_dev.
__global__ void __launch_bounds__(256)
    remap_after_compact_kernel(uint32_t* __restrict__ a, uint32_t na, uint32_t* __restrict__ b, uint32_t nb,
                               uint32_t n, const uint32_t* __restrict__ gone, const uint32_t* __restrict__ k_dev) {
    const uint32_t k = *k_dev, keep = n - k;
    auto lower = [&](uint32_t v) {  // |{gone[j] < v}|
        uint32_t lo = 0, hi = k;
        while (lo < hi) {
            const uint32_t mid = (lo + hi) >> 1;
            if (gone[mid] < v) lo = mid + 1;
            else hi = mid;
        }
        return lo;
    };
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < na + nb; i += gridDim.x * blockDim.x) {
        uint32_t* p = i < na ? a + i : b + (i - na);
        const uint32_t t = *p;
        if (t >= keep) *p = gone[(t - keep) - (lower(t) - lower(keep))];
    }
}

// The counts message and bookkeeping from the two classifications:
// mig = [A, L, R], halo = [0, L, R] -> msg[0..3] = mL, hL, mR, hR; msg[8] = A.
__global__ void counts_msg_kernel(const uint32_t* __restrict__ mig, const uint32_t* __restrict__ halo,
                                  uint64_t* __restrict__ msg) {
    msg[0] = mig[1];
    msg[1] = halo[1];
    msg[2] = mig[2];
    msg[3] = halo[2];
    msg[8] = mig[0];
}

}  // namespace slab
}  // namespace forge

namespace forge {
namespace slab {

// One-pass selection of round 1 of the overlapped exchange: for each owned
// particle, membership in five lists -- migrants A (either side), ML, MR and
// in-slab halo rows HL, HR -- counted, scanned and written (with the records
// packed straight into the two send buffers) by three kernels.
constexpr int kXLists = 5;  // A, ML, MR, HL, HR

__device__ __forceinline__ uint32_t xchg_bits(float x, float lo, float hi, float reach, uint32_t sides) {
    const bool hasl = sides & 1u, hasr = sides & 2u;
    const bool ml = hasl && x < lo, mr = hasr && x >= hi;
    const bool hl = hasl && x >= lo && x < lo + reach;
    const bool hr = hasr && x < hi && x >= hi - reach;
    return ((ml || mr) ? 1u : 0u) | (ml ? 2u : 0u) | (mr ? 4u : 0u) | (hl ? 8u : 0u) | (hr ? 16u : 0u);
}

struct XchgArgs {
    const float* cols;  // rows x, y, z, vx, vy, vz, id; row stride ld
    uint64_t ld;
    uint32_t n;
    float lo, hi, reach;
    uint32_t sides;
};

__global__ void __launch_bounds__(kThreads) xchg_count_kernel(XchgArgs a, uint32_t* __restrict__ tile_counts) {
    __shared__ uint32_t s[kXLists];
    if (threadIdx.x < kXLists) s[threadIdx.x] = 0;
    __syncthreads();
    uint32_t c[kXLists] = {0, 0, 0, 0, 0};
    const uint32_t base = blockIdx.x * kTile;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = base + k * kThreads + threadIdx.x;
        if (i < a.n) {
            const uint32_t b = xchg_bits(a.cols[i], a.lo, a.hi, a.reach, a.sides);
#pragma unroll
            for (int l = 0; l < kXLists; ++l) c[l] += (b >> l) & 1u;
        }
    }
#pragma unroll
    for (int l = 0; l < kXLists; ++l) {
        uint32_t v = c[l];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((threadIdx.x & 31) == 0 && v) atomicAdd(&s[l], v);
    }
    __syncthreads();
    if (threadIdx.x < kXLists) tile_counts[blockIdx.x * kXLists + threadIdx.x] = s[threadIdx.x];
}

// One block: tile offsets per list, totals to counts[0..3) = A, ML, MR and
// counts[4], counts[5] = HL, HR (counts[3] = 0: the layout of the two-pass
// exchange), and the counts message msg[0..3] = ML, HL, MR, HR, msg[8] = A,
// msg[4..8) (the neighbours' counts, received later) = 0.
__global__ void __launch_bounds__(1024)
    xchg_scan_kernel(uint32_t* __restrict__ tile_counts, uint32_t tiles, uint32_t* __restrict__ counts,
                     uint64_t* __restrict__ msg) {
    __shared__ uint32_t s_scan[1024 / 32 + 1];
    __shared__ uint32_t s_tot[kXLists];
    for (int l = 0; l < kXLists; ++l) {
        uint32_t carry = 0;
        for (uint32_t b = 0; b < tiles; b += 1024) {
            const uint32_t t = b + threadIdx.x;
            const uint32_t v = t < tiles ? tile_counts[t * kXLists + l] : 0u;
            uint32_t total;
            const uint32_t ex = block_exclusive_scan<1024>(v, s_scan, &total);
            if (t < tiles) tile_counts[t * kXLists + l] = carry + ex;
            carry += total;
        }
        if (threadIdx.x == 0) s_tot[l] = carry;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        counts[0] = s_tot[0];
        counts[1] = s_tot[1];
        counts[2] = s_tot[2];
        counts[3] = 0;
        counts[4] = s_tot[3];
        counts[5] = s_tot[4];
        msg[0] = s_tot[1];
        msg[1] = s_tot[3];
        msg[2] = s_tot[2];
        msg[3] = s_tot[4];
        msg[4] = msg[5] = msg[6] = msg[7] = 0;
        msg[8] = s_tot[0];
    }
}

struct XchgOut {
    uint32_t* gone;    // [A | ML | MR]
    uint32_t* halo_l;  // HL column indices
    uint32_t* halo_r;
    float* send_l;     // records: [ML | HL], 7 floats each
    float* send_r;     // [MR | HR]
};

__global__ void __launch_bounds__(kThreads)
    xchg_write_kernel(XchgArgs a, const uint32_t* __restrict__ tile_offsets, const uint32_t* __restrict__ counts,
                      XchgOut o) {
    __shared__ uint32_t s_scan[kThreads / 32 + 1];
    const uint32_t base = blockIdx.x * kTile + threadIdx.x * kItems;  // blocked: 16 consecutive per thread
    uint32_t bits[kItems];
    uint32_t c[kXLists] = {0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = base + k;
        bits[k] = i < a.n ? xchg_bits(a.cols[i], a.lo, a.hi, a.reach, a.sides) : 0u;
#pragma unroll
        for (int l = 0; l < kXLists; ++l) c[l] += (bits[k] >> l) & 1u;
    }
    const uint32_t nA = counts[0], nML = counts[1], nMR = counts[2];
#pragma unroll
    for (int l = 0; l < kXLists; ++l) {
        uint32_t total;
        uint32_t pos = block_exclusive_scan<kThreads>(c[l], s_scan, &total) + tile_offsets[blockIdx.x * kXLists + l];
        if (!c[l]) continue;
#pragma unroll
        for (int k = 0; k < kItems; ++k) {
            if (!((bits[k] >> l) & 1u)) continue;
            const uint32_t i = base + k;
            float* rec = nullptr;
            if (l == 0) {
                o.gone[pos] = i;
            } else if (l == 1) {
                o.gone[nA + pos] = i;
                rec = o.send_l + (size_t)pos * 7;
            } else if (l == 2) {
                o.gone[nA + nML + pos] = i;
                rec = o.send_r + (size_t)pos * 7;
            } else if (l == 3) {
                o.halo_l[pos] = i;
                rec = o.send_l + (size_t)(nML + pos) * 7;
            } else {
                o.halo_r[pos] = i;
                rec = o.send_r + (size_t)(nMR + pos) * 7;
            }
            if (rec)
#pragma unroll
                for (int r = 0; r < 7; ++r) rec[r] = a.cols[r * a.ld + i];
            ++pos;
        }
    }
}

}  // namespace slab
}  // namespace forge

namespace forge {
namespace slab {

// Up to six record blocks copied into the column buffer by one launch:
// block b moves cnt[b] records of 7 floats from src[b] to columns
// [dst[b], dst[b] + cnt[b]).
struct UnpackSet {
    const float* src[6];
    uint32_t cnt[6];
    uint32_t dst[6];
};

__global__ void __launch_bounds__(256)
    unpack_set_kernel(UnpackSet u, uint32_t total, float* __restrict__ cols, uint64_t ld) {
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total * 7; t += gridDim.x * blockDim.x) {
        uint32_t rec = t / 7, r = t - rec * 7;
        int b = 0;
        while (rec >= u.cnt[b]) rec -= u.cnt[b++];  // total = sum(cnt) keeps b < 6
        cols[r * ld + u.dst[b] + rec] = u.src[b][(size_t)rec * 7 + r];
    }
}

// Up to four float blocks scattered by one launch: block b moves cnt[b]
// values from src[b] to dst[b].
struct CopySet {
    const float* src[4];
    float* dst[4];
    uint32_t cnt[4];
};

__global__ void __launch_bounds__(256) copy_set_kernel(CopySet c, uint32_t total) {
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        uint32_t k = t;
        int b = 0;
        while (k >= c.cnt[b]) k -= c.cnt[b++];
        c.dst[b][k] = c.src[b][k];
    }
}

// Density messages to both neighbours by one launch: to side X, rho of
// [halo rows sent to X (list), arrivals from X (columns start..)].
struct RhoPackSet {
    const uint32_t* list[2];
    uint32_t k1[2], start[2], k2[2];
    float* out[2];
};

__global__ void __launch_bounds__(256) rho_pack_set_kernel(const float* __restrict__ rho, RhoPackSet p) {
    const uint32_t n0 = p.k1[0] + p.k2[0], n1 = p.k1[1] + p.k2[1];
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < n0 + n1; t += gridDim.x * blockDim.x) {
        const int s = t < n0 ? 0 : 1;
        const uint32_t i = s ? t - n0 : t;
        p.out[s][i] = i < p.k1[s] ? rho[p.list[s][i]] : rho[p.start[s] + i - p.k1[s]];
    }
}

}  // namespace slab
}  // namespace forge
