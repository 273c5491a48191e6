// Warp-cooperative neighbour passes for occupied cells (sm_100a).
//
// The per-thread passes of sph.cuh give every lane its own candidate list,
// so each candidate load is a divergent 16-byte gather and the passes are
// bound by L1 wavefronts. Here a warp takes a GROUP of G consecutive
// cell-ordered particles and walks their neighbour candidates together:
//
//   lane = ii * J + jj,  J = 32 / G
//   ii  : which particle of the group (its frame, accumulators)
//   jj  : which residue of the candidate range (j = b + jj, b + jj + J, ...)
//
// For every row (dz, dy) of the 3x3x3 block the G particles' trimmed windows
// (sph.cuh row_window) are united with two warp reductions, and the row's
// candidates [b, e) -- one contiguous range of the cell order -- are read J
// at a time: the J lanes of one ii read J consecutive float4s and the G
// lanes of one jj read the SAME float4, so each warp load is one broadcast
// L1 wavefront instead of up to 32. Per-particle sums are reduced over the
// J lanes of a particle with shuffles at the end.
//
// Members: the group's particles in the same grid row (cy, cz) as its first
// pending particle and at most one cell further in x (sorted order: x never
// decreases along a row) share one walk; the rest are walked in further
// rounds. A candidate of the union that lies outside a member's own window is
// more than h from it when cell size >= h (Geom::pairable), so it adds +0
// (density: max(h^2 - r^2, 0) = 0; force: fails r^2 < h^2), exactly as in
// the reference; with cell size < h the members must share their cell.
//
// Summation order: each particle's sum is the J lane partial sums (each in
// row order, then ascending j) added in a fixed shuffle tree, so results are
// deterministic run to run and agree with the reference to fp32 rounding
// (the stated tolerances), like the per-thread passes.
#pragma once

#include "sph.cuh"

namespace forge {
namespace sph {

template <int G>
struct GroupLanes {
    static constexpr int J = 32 / G;
    static_assert(G * J == 32, "G divides 32");
};

// Sum over the J lanes of one particle (lanes ii*J .. ii*J + J-1).
template <int J>
__device__ __forceinline__ float sum_lanes(float v) {
#pragma unroll
    for (int o = J / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One round of a group walk: picks the members (pending particles in the
// row of the first pending one, at most one cell further in x when cell size
// >= h, else in its cell) and the base of their row block. Returns false when
// no lane is pending. Warp-uniform.
__device__ __forceinline__ bool group_round(const Frame& f, bool pending, const Geom& g, bool& member,
                                            uint32_t& base0) {
    const uint32_t pend = __ballot_sync(0xffffffffu, pending);
    if (!pend) return false;
    const int leader = __ffs(pend) - 1;
    const int lcy = __shfl_sync(0xffffffffu, f.cy, leader);
    const int lcz = __shfl_sync(0xffffffffu, f.cz, leader);
    const int lcx = __shfl_sync(0xffffffffu, f.f_own, leader) >> g.sub_bits;
    const int cx = f.f_own >> g.sub_bits;
    member = pending && f.cy == lcy && f.cz == lcz && cx >= lcx && cx - lcx <= (g.pairable ? 1 : 0);
    base0 = (uint32_t)lcz * (uint32_t)g.ny + (uint32_t)lcy;
    return true;
}

// Union of the members' trimmed windows of row r (warp-uniform; false: no
// member walks the row) and the row's candidate range [b, e).
__device__ __forceinline__ bool group_row(const Frame& f, bool member, int r, const Geom& g, float H,
                                          const uint32_t* __restrict__ cell_start, uint32_t base0, uint32_t& b,
                                          uint32_t& e) {
    int lo = 0x7fffffff, hi = -1;
    if (member) {
        int l, h;
        if (row_window(f, r, g, H, l, h)) {
            lo = l;
            hi = h;
        }
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if (lo > hi) return false;
    const int dz = r / 3 - 1, dy = r % 3 - 1;
    const uint32_t row = (uint32_t)((int)base0 + dz * g.ny + dy) * ((uint32_t)g.nx << g.sub_bits);
    b = __ldg(cell_start + row + lo);
    e = __ldg(cell_start + row + hi + 1);
    return true;
}

// ---------------------------------------------------------------------------
// Density (poly6, self included), G particles per warp.
// ---------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(128)
    density_group_kernel(float4* __restrict__ pos4, const uint32_t* __restrict__ cell_start,
                         const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c,
                         float4* __restrict__ vel4, float2* __restrict__ aux, float* __restrict__ density_out) {
    pdl_enter();
    constexpr int J = GroupLanes<G>::J;
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, ii = lane / J, jj = lane % J;
    const uint32_t s0 = warp * G;
    if (s0 >= n) return;  // whole warp
    const uint32_t s = s0 + ii;
    const bool valid = s < n;
    const float4 p = pos4[valid ? s : s0];
    const Frame f = make_frame(p, g);
    float rho = 0.f;
    bool pending = valid, member;
    uint32_t base0;
    while (group_round(f, pending, g, member, base0)) {
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            uint32_t b, e;
            if (!group_row(f, member, r, g, c.h2_skip, cell_start, base0, b, e)) continue;
            float acc = 0.f;
#pragma unroll 4
            for (uint32_t j = b + jj; j < e; j += J) {
                const float4 q = __ldg(pos4 + j);
                const float dx = p.x - q.x, dy = p.y - q.y, dz = p.z - q.z;
                const float d = fmaxf(c.h2 - (dx * dx + dy * dy + dz * dz), 0.f);
                acc += d * d * d;
            }
            if (member) rho += c.mass_poly6 * acc;
        }
        pending = pending && !member;
    }
    rho = sum_lanes<J>(rho);
    if (jj == 0 && valid) {
        float inv_rho;
        float2 a;
        density_derived(rho, c, inv_rho, a);
        if (vel4 != nullptr) {
            vel4[s].w = inv_rho;
            aux[s] = a;
            pos4[s] = make_float4(p.x, p.y, p.z, a.x);
        }
        if (density_out != nullptr) density_out[sorted_idx[s]] = rho;
    }
}

// ---------------------------------------------------------------------------
// Force (pressure + viscosity, Jacobi) + epilogue, G particles per warp.
// Each lane scans up to 32 of its candidates for r^2 < h^2 into a bit mask,
// then evaluates the pair terms of its hits (sph.cuh force_hits, indices
// j0 + jj + k*J for bit k).
// ---------------------------------------------------------------------------
template <int TERMS, int J>
__device__ __forceinline__ void force_hits_strided(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                                                   uint32_t j0,
                                                   uint32_t hit, ForceAcc& A, const SphConsts& c) {
    while (hit) {
        const uint32_t j = j0 + (uint32_t)(__ffs(hit) - 1) * J;
        hit &= hit - 1;
        const float4 q = __ldg(pos4 + j);
        const float4 vj = __ldg(vel4 + j);
        const float djx = A.p.x - q.x, djy = A.p.y - q.y, djz = A.p.z - q.z;
        const float r2 = __fadd_rn(__fadd_rn(__fmul_rn(djx, djx), __fmul_rn(djy, djy)), __fmul_rn(djz, djz));
        const float diff = c.h - sqrtf(r2);
        const float inv_rho_j = vj.w;
        if (TERMS & 1) {
            const float pp = fmaf(A.pres, inv_rho_j, q.w);  // q.w = p_j / rho_j
            const float fs = c.kp * pp * (diff * diff) * rsqrtf(r2);
            A.pax = fmaf(fs, djx, A.pax);
            A.pay = fmaf(fs, djy, A.pay);
            A.paz = fmaf(fs, djz, A.paz);
        }
        if (TERMS & 2) {
            const float v = c.kv * inv_rho_j * diff;
            A.vax = fmaf(v, vj.x - A.v.x, A.vax);
            A.vay = fmaf(v, vj.y - A.v.y, A.vay);
            A.vaz = fmaf(v, vj.z - A.v.z, A.vaz);
        }
    }
}

template <int TERMS, int EPI, int G, bool LIST>
__global__ void __launch_bounds__(128)
    force_group_kernel(const float4* __restrict__ pos4, const float4* __restrict__ vel4,
                       const float2* __restrict__ aux, const uint32_t* __restrict__ cell_start,
                       const uint32_t* __restrict__ sorted_idx, uint32_t n, Geom g, SphConsts c, StepEpi ep,
                       ForceOut out, ZoneList zl) {
    pdl_enter();
    constexpr int J = GroupLanes<G>::J;
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, ii = lane / J, jj = lane % J;
    uint32_t cnt = n;
    const uint32_t* lst = nullptr;
    if (LIST) lst = zone_begin(zl, cnt);
    const uint32_t t0 = warp * G;
    if (t0 >= cnt) return;  // whole warp
    const uint32_t t = t0 + ii;
    const bool in = t < cnt;
    const uint32_t s = LIST ? lst[in ? t : t0] : (in ? t : t0);
    ForceAcc A = force_acc(pos4, vel4, aux, s, c, g);
    const uint32_t i = sorted_idx[s];
    // rho < 1e-6 (1/rho stored as 0) or not updated (a ghost): no walk
    bool pending = in && A.v.w != 0.f && i < out.limit;
    const Frame f = make_frame(A.p, g);
    bool member;
    uint32_t base0;
    while (group_round(f, pending, g, member, base0)) {
#pragma unroll 1
        for (int r = 0; r < 9; ++r) {
            uint32_t b, e;
            if (!group_row(f, member, r, g, c.h2_skip, cell_start, base0, b, e)) continue;
            for (uint32_t j0 = b + jj; j0 < e; j0 += 32u * J) {
                const uint32_t k_end = min(32u, (e - j0 + J - 1) / J);
                uint32_t hit = 0;
#pragma unroll 4
                for (uint32_t k = 0; k < k_end; ++k) hit |= in_range_bit(A.p, __ldg(pos4 + j0 + k * J), c, k);
                if (!member) hit = 0;
                force_hits_strided<TERMS, J>(pos4, vel4, j0, hit, A, c);
            }
        }
        pending = pending && !member;
    }
    A.pax = sum_lanes<J>(A.pax);
    A.pay = sum_lanes<J>(A.pay);
    A.paz = sum_lanes<J>(A.paz);
    A.vax = sum_lanes<J>(A.vax);
    A.vay = sum_lanes<J>(A.vay);
    A.vaz = sum_lanes<J>(A.vaz);
    if (jj == 0 && in) force_finish<EPI>(A, i, ep, out);
}

}  // namespace sph
}  // namespace forge
