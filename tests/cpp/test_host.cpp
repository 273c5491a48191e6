// Tests of the C++ host mirror (forge-gpu_b200/host/forge.hpp), written like
// the reference's own Rust tests (tests/radix_sort_test.rs,
// tests/hashgrid_test.rs) against the same known answers.
//   test_host cpu   host-only logic (no GPU needed)
//   test_host gpu   the reference's tests on the GPU through the C++ API
// Prints one line per test, exits non-zero on any failure.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <numeric>
#include <string>
#include <vector>

#include "forge.hpp"

using namespace forge;

static int g_failures = 0;
static std::string g_test;

#define CHECK(cond)                                                                          \
    do {                                                                                     \
        if (!(cond)) {                                                                       \
            std::printf("  FAIL %s: %s (line %d)\n", g_test.c_str(), #cond, __LINE__);      \
            ++g_failures;                                                                    \
        }                                                                                    \
    } while (0)

template <class E, class F>
static bool throws(F f) {
    try {
        f();
    } catch (const E&) {
        return true;
    } catch (...) {
        return false;
    }
    return false;
}

// xorshift32 key stream of the reference's radix tests (radix_sort_test.rs:57-66, :100-108).
static std::vector<uint32_t> xorshift_keys(uint32_t seed, size_t n, uint32_t mask) {
    std::vector<uint32_t> k(n);
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        k[i] = s & mask;
    }
    return k;
}

// Stable order of (keys, 0..n-1) by key: what every radix test compares with.
static void stable_reference(const std::vector<uint32_t>& keys, std::vector<uint32_t>& sk, std::vector<uint32_t>& sv) {
    sv.resize(keys.size());
    std::iota(sv.begin(), sv.end(), 0u);
    std::stable_sort(sv.begin(), sv.end(), [&](uint32_t a, uint32_t b) { return keys[a] < keys[b]; });
    sk.resize(keys.size());
    for (size_t i = 0; i < keys.size(); ++i) sk[i] = keys[sv[i]];
}

// ---------------------------------------------------------------------------
// host-only
// ---------------------------------------------------------------------------
static void cpu_fused_plan() {
    Pipeline p;
    p.add(std::make_unique<SphFusedModule>(0.025f, 0.025f, std::make_tuple(40u, 40u, 40u), 1.f, 3.f, 1000.f, 0.1f));
    p.add(std::make_unique<GravityModule>(0.f, -9.81f, 0.f));
    p.add(std::make_unique<DragModule>(0.5f));
    p.add(std::make_unique<IntegrateModule>());
    p.add(std::make_unique<GroundPlaneModule>(0.1f, 0.3f));
    p.add(std::make_unique<SphereColliderModule>(0.5f, 0.5f, 0.5f, 0.2f, 0.4f));
    p.add(std::make_unique<BoxColliderModule>(0.f, 0.f, 0.f, 1.f, 1.f, 1.f, 0.5f));
    forge_step_params sp{};
    CHECK(p.fused_plan(sp));
    CHECK(sp.n_ops == 6);
    const uint32_t kinds[6] = {FORGE_OP_GRAVITY, FORGE_OP_DRAG, FORGE_OP_INTEGRATE, FORGE_OP_GROUND, FORGE_OP_SPHERE,
                               FORGE_OP_BOX};
    for (int k = 0; k < 6; ++k) CHECK(sp.ops[k].kind == kinds[k]);
    CHECK(sp.ops[0].p[1] == -9.81f);
    CHECK(sp.ops[5].p[6] == 0.5f);
    Pipeline q;  // no SPH module first
    q.add(std::make_unique<GravityModule>());
    CHECK(!q.fused_plan(sp));
    Pipeline r;  // an SPH pass after the fused module: not the pattern
    r.add(std::make_unique<SphFusedModule>(0.025f, 0.025f, std::make_tuple(40u, 40u, 40u), 1.f, 3.f, 1000.f, 0.1f));
    r.add(std::make_unique<SphDensityModule>(0.025f, 0.025f, std::make_tuple(40u, 40u, 40u), 1.f));
    CHECK(!r.fused_plan(sp));
    CHECK(r.len() == 2);
}

static void cpu_cell_of() {
    const Vec3f o{0.f, 0.f, 0.f};
    CHECK(HashGrid::cell_of({5.f, 5.f, 5.f}, o, 1.f, 10, 10, 10) == 555u);
    CHECK(HashGrid::cell_of({-3.f, 0.5f, 0.5f}, o, 1.f, 10, 10, 10) == 0u);       // clamped low
    CHECK(HashGrid::cell_of({42.f, 9.99f, 0.f}, o, 1.f, 10, 10, 10) == 99u);       // clamped high
    CHECK(HashGrid::cell_of({NAN, 1.f, 2.f}, o, 1.f, 10, 10, 10) == 210u);         // NaN -> 0
    CHECK(HashGrid::cell_of({1.5f, 2.5f, 3.5f}, {1.f, 2.f, 3.f}, 0.5f, 4, 4, 4) == 1u + 4u + 16u);  // origin
}

static void cpu_abi_errors() {
    // Argument errors come back as the library's status, before any device call.
    forge_step_params sp{};
    sp.n_ops = 9;
    CHECK(forge_apply_ops(&sp, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 10, 0, nullptr) ==
          FORGE_ERR_INVALID_ARG);
    CHECK(throws<ForgeError>([] { detail::check(FORGE_ERR_CAPACITY, "x"); }));
    try {
        detail::check(FORGE_ERR_TIMEOUT, "wait");
    } catch (const ForgeError& e) {
        CHECK(e.kind() == ForgeError::Kind::LaunchFailed);
        CHECK(e.code() == FORGE_ERR_TIMEOUT);
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)  // no GPU: allocation fails as a ForgeError
        CHECK(throws<ForgeError>([] { RadixSorter s(1024, 0); }));
}

// ---------------------------------------------------------------------------
// GPU: radix_sort_test.rs
// ---------------------------------------------------------------------------
static void run_sort_case(const std::vector<uint32_t>& keys, uint32_t bits) {
    const size_t n = keys.size();
    std::vector<uint32_t> vals(n);
    std::iota(vals.begin(), vals.end(), 0u);
    const Device d = Device::Cuda(0);
    Array<uint32_t> k = Array<uint32_t>::from_vec(keys, d), v = Array<uint32_t>::from_vec(vals, d);
    RadixSorter s(n, 0);
    s.sort(k, v, n, bits);
    s.check();
    std::vector<uint32_t> sk, sv;
    stable_reference(keys, sk, sv);
    CHECK(k.to_vec() == sk);
    CHECK(v.to_vec() == sv);
}

static void gpu_radix_small() {  // radix_sort_test.rs:14-48
    run_sort_case({15, 3, 7, 1, 9, 0, 12, 5, 8, 2, 14, 6, 11, 4, 13, 10}, 4);
}

static void gpu_radix_xorshift() {  // radix_sort_test.rs:50-91 and :93-136
    auto a = xorshift_keys(12345, 10000, 0xFFFFF);
    const uint32_t head[8] = {357498, 657839, 36768, 934378, 567763, 528994, 156056, 409400};
    for (int i = 0; i < 8; ++i) CHECK(a[i] == head[i]);  // the reference's key stream
    run_sort_case(a, 20);
    run_sort_case(xorshift_keys(42, 5000, 0xFFFF), 16);
}

static void gpu_radix_reuse_and_asserts() {
    // One sorter, many sorts of shrinking sizes: the swapped-in alternates
    // stay usable (radix_sort.rs:215-216 swap semantics).
    const Device d = Device::Cuda(0);
    RadixSorter s(4096, 0);
    for (size_t n : {4096u, 3000u, 1u, 2048u}) {
        auto keys = xorshift_keys(7 + (uint32_t)n, n, 0xFFFFFFFFu);
        std::vector<uint32_t> vals(n);
        std::iota(vals.begin(), vals.end(), 0u);
        Array<uint32_t> k = Array<uint32_t>::from_vec(keys, d), v = Array<uint32_t>::from_vec(vals, d);
        s.sort(k, v, n, 32);
        std::vector<uint32_t> sk, sv;
        stable_reference(keys, sk, sv);
        CHECK(k.to_vec() == sk);
        CHECK(v.to_vec() == sv);
    }
    Array<uint32_t> k = Array<uint32_t>::zeros(8, d), v = Array<uint32_t>::zeros(8, d);
    CHECK(throws<std::logic_error>([&] { s.sort(k, v, 8, 6); }));     // num_bits % 4 != 0
    CHECK(throws<std::logic_error>([&] { s.sort(k, v, 5000, 8); }));  // n > max_n
}

static void gpu_cell_bounds() {  // radix_sort_test.rs:138-171
    const Device d = Device::Cuda(0);
    const uint32_t S = 0xFFFFFFFFu;
    Array<uint32_t> ids = Array<uint32_t>::from_vec({0, 0, 1, 1, 1, 3, 3, 5}, d);
    Array<uint32_t> start = Array<uint32_t>::zeros(8, d), end = Array<uint32_t>::zeros(8, d);
    find_cell_boundaries(ids, start, end, 8, 8, 0);
    CHECK(start.to_vec() == (std::vector<uint32_t>{0, 2, S, 5, S, 7, S, S}));
    CHECK(end.to_vec() == (std::vector<uint32_t>{2, 5, 0, 7, 0, 8, 0, 0}));
}

// ---------------------------------------------------------------------------
// GPU: hashgrid_test.rs
// ---------------------------------------------------------------------------
static bool contains(const std::vector<uint32_t>& v, uint32_t x) { return std::find(v.begin(), v.end(), x) != v.end(); }

static void gpu_hashgrid_basic() {  // hashgrid_test.rs:6-36
    std::vector<Vec3f> pos = {{5.f, 5.f, 5.f}, {5.1f, 5.f, 5.f}, {5.5f, 5.5f, 5.5f}, {9.f, 9.f, 9.f}};
    HashGrid g(1.f, {10u, 10u, 10u}, Vec3f{}, 100, Device::Cuda(0));
    g.build(pos);
    CHECK(g.num_particles == 4);
    auto hits = g.query_neighbors({5.f, 5.f, 5.f}, 1.f, pos);
    CHECK(contains(hits, 0) && contains(hits, 1) && contains(hits, 2));
    CHECK(!contains(hits, 3));
}

static void gpu_hashgrid_uniform() {  // hashgrid_test.rs:38-88
    std::vector<Vec3f> pos;
    for (int i = 0; i < 1000; ++i)
        pos.push_back({(float)(i % 10) + 0.5f, (float)((i / 10) % 10) + 0.5f, (float)(i / 100) + 0.5f});
    HashGrid g(2.f, {5u, 5u, 5u}, Vec3f{}, 1000, Device::Cuda(0));
    g.build(pos);
    const Vec3f q{5.f, 5.f, 5.f};
    const float r = 1.5f;
    auto hits = g.query_neighbors(q, r, pos);
    CHECK(hits.size() >= 4);
    // every hit within r, every point within r of q found (the 3x3x3 walk covers r <= cell size)
    size_t inside = 0;
    for (size_t i = 0; i < pos.size(); ++i) {
        const float dx = pos[i].x - q.x, dy = pos[i].y - q.y, dz = pos[i].z - q.z;
        const bool in = dx * dx + dy * dy + dz * dz <= r * r;
        inside += in;
        CHECK(in == contains(hits, (uint32_t)i));
    }
    CHECK(hits.size() == inside);
    // the build: cell_indices = position_to_cell, sorted_indices stable by cell, cell_start the prefix
    auto ci = g.cell_indices.to_vec(), si = g.sorted_indices.to_vec(), cs = g.cell_start.to_vec();
    std::vector<uint32_t> cells(pos.size());
    for (size_t i = 0; i < pos.size(); ++i) cells[i] = g.position_to_cell(pos[i]);
    CHECK(std::equal(cells.begin(), cells.end(), ci.begin()));
    std::vector<uint32_t> sk, sv;
    stable_reference(cells, sk, sv);
    CHECK(std::equal(sv.begin(), sv.end(), si.begin()));
    std::vector<uint32_t> prefix(g.num_cells() + 1, 0);
    for (uint32_t c : cells) ++prefix[c + 1];
    for (size_t c = 0; c < g.num_cells(); ++c) prefix[c + 1] += prefix[c];
    CHECK(cs == prefix);
    CHECK(throws<std::logic_error>([&] { g.query_neighbors(q, r, std::vector<Vec3f>(3)); }));
}

// ---------------------------------------------------------------------------
// GPU: the manifest pipeline
// ---------------------------------------------------------------------------
static FieldSet lattice_fields(size_t& n, Device d) {
    std::vector<float> x, y, z;
    for (int k = 0; k < 16; ++k)
        for (int j = 0; j < 32; ++j)
            for (int i = 0; i < 16; ++i) {
                x.push_back(0.1f + 0.0125f * i);
                y.push_back(0.1f + 0.0125f * j);
                z.push_back(0.1f + 0.0125f * k);
            }
    n = x.size();
    FieldSet f(n, d);
    f.add_f32("pos_x", x);
    f.add_f32("pos_y", y);
    f.add_f32("pos_z", z);
    f.add_f32_zeros("vel_x", n);
    f.add_f32_zeros("vel_y", n);
    f.add_f32_zeros("vel_z", n);
    return f;
}

static void gpu_pipeline_fused_equals_direct_step() {
    // The fused Pipeline dispatches exactly one forge_sph_step with its op
    // list: same bits as calling the C ABI directly.
    const Device d = Device::Cuda(0);
    size_t n = 0;
    FieldSet a = lattice_fields(n, d), b = lattice_fields(n, d);
    const float h = 0.025f, m = 1000.f * 0.0125f * 0.0125f * 0.0125f, dt = 1e-4f;
    Pipeline p;
    p.add(std::make_unique<SphFusedModule>(h, h, std::make_tuple(40u, 40u, 40u), m, 3.f, 1000.f, 0.1f));
    p.add(std::make_unique<GravityModule>(0.f, -9.81f, 0.f));
    p.add(std::make_unique<IntegrateModule>());
    p.add(std::make_unique<BoxColliderModule>(0.f, 0.f, 0.f, 1.f, 1.f, 1.f, 0.5f));
    p.run(a, dt, 5);
    forge_step_params sp{};
    CHECK(p.fused_plan(sp));
    sp.dt = dt;
    forge_sph_params prm{};
    prm.h = h, prm.mass = m, prm.gas_constant = 3.f, prm.rest_density = 1000.f, prm.viscosity = 0.1f;
    HashGrid g(h, {40u, 40u, 40u}, Vec3f{}, n, d);
    b.add_f32_zeros("density", n);
    for (int s = 0; s < 5; ++s)
        detail::check(forge_sph_step(g.handle(), &prm, &sp, b.need("pos_x"), b.need("pos_y"), b.need("pos_z"),
                                     b.need("vel_x"), b.need("vel_y"), b.need("vel_z"), b.need("density"), n, nullptr),
                      "forge_sph_step");
    for (const char* f : {"pos_x", "pos_y", "pos_z", "vel_x", "vel_y", "vel_z", "density"})
        CHECK(a.get_f32(f)->to_vec() == b.get_f32(f)->to_vec());
    // pressure and viscosity conserve momentum (equal masses): the mean
    // velocity change is gravity's alone, -9.81 * 5 * dt
    auto vy = a.get_f32("vel_y")->to_vec();
    double mean = 0.0;
    for (float v : vy) mean += v;
    mean /= (double)vy.size();
    CHECK(std::fabs(mean + 9.81 * 5 * 1e-4) < 1e-4);
}

static void gpu_pipeline_unfused_modules() {
    // SphDensity -> SphPressure -> SphViscosity -> Gravity -> Integrate ->
    // GroundPlane, module by module (forge_sph_density, forge_sph_force,
    // forge_apply_ops): runs, stays finite, and a module that needs the
    // density pass refuses to run first.
    const Device d = Device::Cuda(0);
    size_t n = 0;
    FieldSet f = lattice_fields(n, d);
    const float h = 0.025f, m = 1000.f * 0.0125f * 0.0125f * 0.0125f;
    Pipeline p;
    p.add(std::make_unique<SphDensityModule>(h, h, std::make_tuple(40u, 40u, 40u), m));
    p.add(std::make_unique<SphPressureModule>(h, m, 3.f, 1000.f));
    p.add(std::make_unique<SphViscosityModule>(h, m, 0.1f));
    p.add(std::make_unique<GravityModule>(0.f, -9.81f, 0.f));
    p.add(std::make_unique<IntegrateModule>());
    p.add(std::make_unique<GroundPlaneModule>(0.15f, 0.5f));
    forge_step_params sp{};
    CHECK(!p.fused_plan(sp));
    p.run(f, 1e-3f, 4);
    auto y = f.get_f32("pos_y")->to_vec();
    auto rho = f.get_f32("density")->to_vec();
    bool finite = true, above = true;
    for (size_t i = 0; i < n; ++i) {
        finite = finite && std::isfinite(y[i]) && std::isfinite(rho[i]);
        above = above && y[i] >= 0.15f;
    }
    CHECK(finite);
    CHECK(above);  // the ground plane held
    const size_t mid = 8 + 16 * (16 + 32 * 8);  // lattice point (8, 16, 8): interior
    CHECK(rho[mid] > 500.f && rho[mid] < 2000.f);  // interior lattice density near rest
    FieldSet g = lattice_fields(n, d);
    SphPressureModule alone(h, m, 3.f, 1000.f);
    CHECK(throws<ForgeError>([&] { alone.execute(g, 1e-3f); }));
    // one per-particle module on its own: v += g dt
    GravityModule grav(0.f, -10.f, 0.f);
    grav.execute(g, 0.5f);
    auto vy = g.get_f32("vel_y")->to_vec();
    CHECK(std::fabs(vy[0] + 5.f) < 1e-6f && std::fabs(vy[n - 1] + 5.f) < 1e-6f);
}

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "cpu";
    std::vector<std::pair<const char*, std::function<void()>>> tests;
    if (mode == "cpu") {
        tests = {{"cpu_fused_plan", cpu_fused_plan}, {"cpu_cell_of", cpu_cell_of}, {"cpu_abi_errors", cpu_abi_errors}};
    } else {
        tests = {{"gpu_radix_small", gpu_radix_small},
                 {"gpu_radix_xorshift", gpu_radix_xorshift},
                 {"gpu_radix_reuse_and_asserts", gpu_radix_reuse_and_asserts},
                 {"gpu_cell_bounds", gpu_cell_bounds},
                 {"gpu_hashgrid_basic", gpu_hashgrid_basic},
                 {"gpu_hashgrid_uniform", gpu_hashgrid_uniform},
                 {"gpu_pipeline_fused_equals_direct_step", gpu_pipeline_fused_equals_direct_step},
                 {"gpu_pipeline_unfused_modules", gpu_pipeline_unfused_modules}};
    }
    for (auto& t : tests) {
        g_test = t.first;
        const int before = g_failures;
        try {
            t.second();
        } catch (const std::exception& e) {
            std::printf("  FAIL %s: exception: %s\n", t.first, e.what());
            ++g_failures;
        }
        std::printf("%s %s\n", g_failures == before ? "PASS" : "FAIL", t.first);
    }
    return g_failures ? 1 : 0;
}
