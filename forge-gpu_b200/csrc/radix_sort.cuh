// Onesweep-style stable LSD radix sort of (u32 key, u32 value) pairs, sm_100a.
//
// Replaces the reference's 4-bit LSD sorter (forge-runtime/src/radix_sort.rs:79-220,
// kernels radix_histogram :323-351, radix_prefix_sum :356-389, radix_scatter
// :394-440). Same result (a stable sort by the low key bits), different machine:
//
//  * 8-bit digits, ceil(bits/8) passes instead of bits/4.
//  * One up-front kernel builds the digit histograms of every pass at once
//    (one read of the keys), so each pass is a single kernel.
//  * Each pass kernel takes a tile of kTile keys, ranks them inside the tile
//    with warp-level digit matching from bit-sliced ballots (stable:
//    item-major, lane-minor order is the input order), finds the tile's global offset per digit with a
//    decoupled look-back over earlier tiles (bounded waits), stages the
//    digit-sorted tile in shared memory and writes it out coalesced.
//  * Tile ids come from an atomic counter, so every tile a CTA waits on
//    belongs to a CTA that is already running (forward progress without
//    co-residency assumptions).
#pragma once

#include "common.cuh"

namespace forge {
namespace radix {

constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kThreads = 256;  // == kRadix: one digit per thread in the look-back
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 16;
constexpr int kTile = kThreads * kItems;  // 4096 keys per tile
constexpr int kMaxPasses = 4;
constexpr int kLookBatch = 8;  // look-back status words loaded per round trip

// Look-back status word: [31] pass parity | [30:29] flag | [28:0] count.
constexpr uint32_t kFlagAgg = 1u << 29;
constexpr uint32_t kFlagPre = 2u << 29;
constexpr uint32_t kFlagMask = 3u << 29;
constexpr uint32_t kParityBit = 1u << 31;
constexpr uint32_t kCountMask = (1u << 29) - 1;
constexpr uint64_t kMaxN = (1ull << 29) - 1;

constexpr int kHistThreads = 256;

constexpr int kHistItems = 8;

__host__ __device__ constexpr uint32_t num_tiles(uint64_t n, uint32_t tile = kTile) {
    return (uint32_t)((n + tile - 1) / tile);
}

// Small sorts (at most kSmallN keys) take tiles of kSmallItems keys per
// thread: four times the CTAs, so a 50,000-key sort still spreads over the
// GPU instead of running 13 long tiles one after another.
constexpr int kSmallItems = 4;
constexpr uint32_t kSmallTile = kThreads * kSmallItems;
constexpr uint32_t kSmallN = 1u << 20;

// Lanes of the warp holding the same 8-bit digit as this lane, from eight
// ballots (bit slicing); cheaper than the MATCH instruction on this part.
// Lanes with valid == false are excluded from every lane's mask.
__device__ __forceinline__ uint32_t warp_same_digit(uint32_t d, bool valid) {
    uint32_t peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int b = 0; b < kRadixBits; ++b) {
        const bool bit = (d >> b) & 1u;
        const uint32_t v = __ballot_sync(0xffffffffu, bit);
        peers &= bit ? v : ~v;
    }
    return peers;
}

// Digit of `key` for a pass starting at `shift` with `bits` bits.
__device__ __forceinline__ uint32_t digit_of(uint32_t key, uint32_t shift, uint32_t mask) {
    return (key >> shift) & mask;
}

// ---------------------------------------------------------------------------
// Key sources for the up-front histogram kernel.
// ---------------------------------------------------------------------------
struct KeysFromArray {
    const uint32_t* __restrict__ keys;
    __device__ __forceinline__ uint32_t operator()(uint32_t i) const { return keys[i]; }
    // keys i0 .. i0+7 (i0 a multiple of 8; missing keys read as 0): two
    // 16-byte loads when the array is 16-byte aligned
    __device__ __forceinline__ void load8(uint32_t i0, uint32_t n, uint32_t (&k)[8]) const {
        if (i0 + 8 <= n && (reinterpret_cast<uintptr_t>(keys) & 15u) == 0) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(keys + i0));
            const uint4 b = __ldg(reinterpret_cast<const uint4*>(keys + i0) + 1);
            k[0] = a.x, k[1] = a.y, k[2] = a.z, k[3] = a.w, k[4] = b.x, k[5] = b.y, k[6] = b.z, k[7] = b.w;
            return;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) k[j] = i0 + j < n ? keys[i0 + j] : 0u;
    }
};

// ---------------------------------------------------------------------------
// Up-front histogram: hist[p*256 + d] += #keys whose pass-p digit is d, for
// every pass p. Also zeroes the look-back status table used by the passes.
// Each thread takes runs of kHistItems consecutive keys and counts each
// pass's digits run-length (a change of digit flushes the run with one
// shared atomic), so spatially ordered cell keys -- long runs of one digit
// in the upper passes -- cost one atomic per run, and random keys one per
// key, with no warp-wide votes. Each warp keeps its own shared histograms.
// ---------------------------------------------------------------------------
template <class Src>
__global__ void __launch_bounds__(kHistThreads)
    digit_histogram_kernel(Src src, uint32_t n, uint32_t begin_bit, uint32_t end_bit,
                           uint32_t passes, uint32_t* __restrict__ hist,
                           uint4* __restrict__ status, uint32_t status_vec4) {
    pdl_enter();
    static_assert(kHistItems == 8, "load8 runs");
    constexpr int kW = kHistThreads / 32;
    __shared__ uint32_t s_hist[kW][kMaxPasses * kRadix];
    const int warp = threadIdx.x >> 5;
    for (uint32_t j = threadIdx.x; j < kW * kMaxPasses * kRadix; j += kHistThreads) (&s_hist[0][0])[j] = 0;

    const uint32_t stride = gridDim.x * kHistThreads;
    const uint4 zero = make_uint4(0, 0, 0, 0);
    for (uint32_t j = blockIdx.x * kHistThreads + threadIdx.x; j < status_vec4; j += stride)
        status[j] = zero;
    __syncthreads();

    uint32_t* wh = s_hist[warp];
    uint32_t cur[kMaxPasses], cnt[kMaxPasses];
#pragma unroll
    for (int p = 0; p < kMaxPasses; ++p) cur[p] = 0, cnt[p] = 0;
    for (uint32_t i0 = (blockIdx.x * kHistThreads + threadIdx.x) * kHistItems; i0 < n;
         i0 += stride * kHistItems) {
        uint32_t key[kHistItems];
        src.load8(i0, n, key);
        const uint32_t m = min((uint32_t)kHistItems, n - i0);
#pragma unroll
        for (int k = 0; k < kHistItems; ++k) {
            if ((uint32_t)k >= m) break;
#pragma unroll
            for (int p = 0; p < kMaxPasses; ++p) {
                if ((uint32_t)p >= passes) break;
                const uint32_t shift = begin_bit + p * kRadixBits;
                const uint32_t bits = min((uint32_t)kRadixBits, end_bit - shift);
                const uint32_t d = digit_of(key[k], shift, (1u << bits) - 1u);
                if (d != cur[p]) {
                    if (cnt[p]) atomicAdd(&wh[p * kRadix + cur[p]], cnt[p]);
                    cur[p] = d;
                    cnt[p] = 1;
                } else {
                    ++cnt[p];
                }
            }
        }
    }
#pragma unroll
    for (int p = 0; p < kMaxPasses; ++p)
        if (cnt[p]) atomicAdd(&wh[p * kRadix + cur[p]], cnt[p]);
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < passes * kRadix; j += kHistThreads) {
        uint32_t c = 0;
#pragma unroll
        for (int w = 0; w < kW; ++w) c += s_hist[w][j];
        if (c) atomicAdd(&hist[j], c);
    }
}

// ---------------------------------------------------------------------------
// One Onesweep pass over tiles of kThreads * ITEMS keys. IOTA: the input
// values are the element indices (first pass of the grid build), vals_in is
// not read.
// ---------------------------------------------------------------------------
#ifndef FORGE_SORT_MIN_BLOCKS
#define FORGE_SORT_MIN_BLOCKS 5  // 51 registers (spills): 5 CTAs per SM, the shared-memory limit
#endif
template <bool IOTA, int ITEMS = kItems>
__global__ void __launch_bounds__(kThreads, FORGE_SORT_MIN_BLOCKS)
    onesweep_pass_kernel(const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                         uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
                         uint32_t n, uint32_t shift, uint32_t bits,
                         const uint32_t* __restrict__ pass_hist,  // [256] of this pass
                         uint32_t* status,                        // [tiles][256]
                         uint32_t* tile_counter, uint32_t parity, uint32_t* err,
                         uint32_t tile_base, uint32_t spin_limit, uint32_t ntiles) {
    pdl_enter();
    __shared__ uint32_t s_whist[kWarps][kRadix];  // per-warp digit counts, then offsets
    __shared__ uint32_t s_tile_off[kRadix];       // digit start inside the sorted tile
    __shared__ uint32_t s_base[kRadix];           // global dst = s_base[d] + tile position
    __shared__ uint32_t s_scan[kWarps + 1];
    constexpr uint32_t TILE = kThreads * ITEMS;
    __shared__ uint32_t s_exchange[TILE];  // the tile's keys, in sorted order
    __shared__ uint32_t s_vals[TILE];      // its values: input order (staged), then sorted order
    __shared__ uint32_t s_tile;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // tile_base > 0 only under the failure-detection test hook: tile ids
    // below it are never taken, so their successors' look-backs run out
    if (tid == 0) s_tile = atomicAdd(tile_counter, 1u) + tile_base;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s_whist[w][tid] = 0;
    __syncthreads();

    const uint32_t tile = s_tile;
    if (tile >= ntiles) return;  // (only with tile_base > 0) the whole block
    const uint32_t tile_start = tile * TILE;
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t warp_start = tile_start + warp * 32 * ITEMS;

    // Load: warp-striped so each load instruction is 128 contiguous bytes and
    // (item, lane) order equals input order. The values go straight to
    // shared memory (cp.async, no registers held through the ranking); they
    // are needed only once every key has its tile position.
    uint32_t key[ITEMS];
    const uint32_t wbase = (uint32_t)warp * 32u * ITEMS;  // this warp's first tile slot
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const uint32_t idx = warp_start + k * 32 + lane;
        const bool ok = idx < n;
        key[k] = ok ? keys_in[idx] : 0u;
        if (!IOTA && ok) {
            const uint32_t sa = (uint32_t)__cvta_generic_to_shared(&s_vals[wbase + k * 32 + lane]);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(vals_in + idx) : "memory");
        }
    }
    if (!IOTA) asm volatile("cp.async.commit_group;" ::: "memory");

    // Early counts: per-warp digit histograms from shared atomics (a warp
    // whose keys share one digit adds 32 once), so the tile aggregate is
    // published before the ranking and successors' look-backs do not wait
    // for it.
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const uint32_t idx = warp_start + k * 32 + lane;
        const bool ok = idx < n;
        const uint32_t d = digit_of(key[k], shift, mask);
        const uint32_t d0 = __shfl_sync(0xffffffffu, d, 0);
        if (__all_sync(0xffffffffu, ok && d == d0)) {
            if (lane == 0) s_whist[warp][d0] += 32u;
        } else if (ok) {
            atomicAdd(&s_whist[warp][d], 1u);
        }
        __syncwarp();
    }
    __syncthreads();

    // Per digit (thread tid == digit): tile count, published at once, then
    // each warp's starting position of the digit inside the sorted tile.
    uint32_t cnt = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) cnt += s_whist[w][tid];
    uint32_t* my_status = status + (size_t)tile * kRadix + tid;
    const uint32_t par = parity ? kParityBit : 0u;
    st_relaxed_u32(my_status, par | (tile == 0 ? kFlagPre : kFlagAgg) | cnt);

    uint32_t total;
    const uint32_t tile_off = block_exclusive_scan<kThreads>(cnt, s_scan, &total);
    s_tile_off[tid] = tile_off;
    {
        uint32_t run = tile_off;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const uint32_t c = s_whist[w][tid];
            s_whist[w][tid] = run;
            run += c;
        }
    }
    // (the scan's barriers also publish s_whist / s_tile_off)
    const uint32_t hist_off = block_exclusive_scan<kThreads>(pass_hist[tid], s_scan, &total);

    // Stable warp-level ranking straight to tile positions: item-major,
    // lane-minor order is the input order.
    const uint32_t lt = lanemask_lt();
    uint32_t pos[ITEMS];
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const uint32_t idx = warp_start + k * 32 + lane;
        const bool ok = idx < n;
        const uint32_t d = digit_of(key[k], shift, mask);
        const uint32_t peers = warp_same_digit(d, ok);
        uint32_t before = 0;
        if (ok) before = s_whist[warp][d];
        __syncwarp();
        if (ok && (peers & lt) == 0) s_whist[warp][d] = before + __popc(peers);
        __syncwarp();
        pos[k] = ok ? before + __popc(peers & lt) : 0xffffffffu;
        if (ok) s_exchange[pos[k]] = key[k];
    }

    // Decoupled look-back for digit tid. The nearest inclusive prefix is
    // typically ~20 tiles back with every aggregate already published, so
    // kLookBatch status words are loaded per round trip and consumed in order
    // until a prefix (a word not yet published is re-polled).
    uint32_t excl = 0;
    if (tile > 0) {
        int t = (int)tile - 1;
        uint32_t spins = 0;
        bool done = false;
        while (!done) {
            uint32_t v[kLookBatch];
#pragma unroll
            for (int q = 0; q < kLookBatch; ++q)
                v[q] = (t - q >= 0) ? ld_relaxed_u32(status + (size_t)(t - q) * kRadix + tid) : (par | kFlagPre);
            bool go = true;
            int used = 0;
#pragma unroll
            for (int q = 0; q < kLookBatch; ++q) {
                if (!go) continue;
                const bool ready = ((v[q] & kParityBit) == par) && (v[q] & kFlagMask) != 0;
                if (!ready) {
                    go = false;
                    continue;
                }
                excl += v[q] & kCountMask;
                ++used;
                if ((v[q] & kFlagMask) == kFlagPre) {
                    done = true;
                    go = false;
                }
            }
            t -= used;
            if (!done && used == 0) {
                if (++spins > spin_limit) {
                    atomicOr(err, kDevTimeout);
                    break;
                }
                if (spins > 64) __nanosleep(64);
            }
        }
        st_relaxed_u32(my_status, par | kFlagPre | ((excl + cnt) & kCountMask));
    }
    s_base[tid] = hist_off + excl - tile_off;

    // Values to their tile positions: read this thread's staged values
    // (input order), then, after a barrier, write them sorted.
    uint32_t val[ITEMS];
    if (IOTA) {
#pragma unroll
        for (int k = 0; k < ITEMS; ++k) val[k] = warp_start + k * 32 + lane;
    } else {
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // every thread's copies landed
#pragma unroll
        for (int k = 0; k < ITEMS; ++k) val[k] = s_vals[wbase + k * 32 + lane];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < ITEMS; ++k)
        if (pos[k] != 0xffffffffu) s_vals[pos[k]] = val[k];
    __syncthreads();

    // Coalesced scatter of the sorted tile: runs of one digit are contiguous.
    const uint32_t tile_n = min((uint32_t)TILE, n - tile_start);
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const uint32_t j = tid + k * kThreads;
        if (j < tile_n) {
            const uint32_t kk = s_exchange[j];
            const uint32_t dst = s_base[digit_of(kk, shift, mask)] + j;
            keys_out[dst] = kk;
            vals_out[dst] = s_vals[j];
        }
    }
}

}  // namespace radix
}  // namespace forge
