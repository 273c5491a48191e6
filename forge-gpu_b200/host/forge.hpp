// C++ host side of the particle hot path over libforge_sph's C ABI,
// mirroring the reference's Rust interface (names, argument meaning and
// error behaviour) for a host written in a compiled language:
//   Array<T>                   forge-runtime/src/array.rs:102-407 (device buffer)
//   RadixSorter, find_cell_boundaries
//                              forge-runtime/src/radix_sort.rs:26-317
//   HashGrid                   forge-runtime/src/hashgrid.rs:21-193
//   FieldSet, SimModule, Pipeline
//                              forge-manifest/src/modules/mod.rs:12-117
//   Sph{Fused,Density,Pressure,Viscosity}Module, Gravity, Drag, Integrate,
//   GroundPlane, SphereCollider, BoxCollider modules
//                              forge-manifest/src/modules/builtins/*.rs
// Errors are ForgeError with the reference's kinds (error.rs:7-22); the
// reference's assert!s (radix_sort.rs:86-87) become std::logic_error. All
// work goes to the CUDA default stream of the calling thread, so to_vec()
// (a synchronous copy) sees it finished, as the reference's to_vec does.
// Header-only; link libforge_sph.so and libcudart.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "forge_sph.h"

namespace forge {

// forge-core Vec3f (12-byte AoS element).
struct Vec3f {
    float x = 0.f, y = 0.f, z = 0.f;
};

// Device (forge-runtime): CUDA ordinal.
struct Device {
    int ordinal = 0;
    static Device Cuda(int ordinal) { return Device{ordinal}; }
};

class ForgeError : public std::runtime_error {
   public:
    enum class Kind { CompilationFailed, ModuleLoadFailed, FunctionLoadFailed, LaunchFailed, SyncFailed,
                      WrongDevice, DeviceNotFound };
    ForgeError(Kind kind, int code, const std::string& msg) : std::runtime_error(msg), kind_(kind), code_(code) {}
    Kind kind() const { return kind_; }
    int code() const { return code_; }  // the C ABI status (FORGE_ERR_*), FORGE_OK for host-side errors

   private:
    Kind kind_;
    int code_;
};

namespace detail {

inline std::string last_error() {
    char buf[1024];
    forge_last_error(buf, sizeof buf);
    return buf;
}

// A failed library call: a launch-time failure in the reference's terms.
inline void check(int rc, const char* what) {
    if (rc == FORGE_OK) return;
    throw ForgeError(ForgeError::Kind::LaunchFailed, rc, std::string(what) + ": " + last_error());
}

inline void cuda_check(cudaError_t e, const char* what, ForgeError::Kind kind = ForgeError::Kind::LaunchFailed) {
    if (e == cudaSuccess) return;
    throw ForgeError(kind, FORGE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Selects `ordinal` for the scope, restoring the previous device.
class DeviceScope {
   public:
    explicit DeviceScope(int ordinal) {
        cuda_check(cudaGetDevice(&prev_), "cudaGetDevice", ForgeError::Kind::DeviceNotFound);
        if (prev_ != ordinal) cuda_check(cudaSetDevice(ordinal), "cudaSetDevice", ForgeError::Kind::WrongDevice);
    }
    ~DeviceScope() { cudaSetDevice(prev_); }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;

   private:
    int prev_ = 0;
};

}  // namespace detail

// Array<T> (array.rs): a device buffer of `len` elements on one device.
// Move-only; freed with the object.
template <class T>
class Array {
   public:
    Array() = default;
    static Array zeros(size_t len, Device device) {
        Array a;
        a.len_ = len;
        a.dev_ = device;
        if (len) {
            detail::DeviceScope s(device.ordinal);
            detail::cuda_check(cudaMalloc(reinterpret_cast<void**>(&a.p_), len * sizeof(T)), "Array::zeros");
            detail::cuda_check(cudaMemset(a.p_, 0, len * sizeof(T)), "Array::zeros");
        }
        return a;
    }
    static Array from_vec(const std::vector<T>& host, Device device) {
        Array a = zeros(host.size(), device);
        a.copy_from(host);
        return a;
    }
    void copy_from(const std::vector<T>& host) {
        if (host.size() > len_)
            throw ForgeError(ForgeError::Kind::LaunchFailed, FORGE_OK, "Array::copy_from: host data longer than the array");
        if (host.empty()) return;
        detail::DeviceScope s(dev_.ordinal);
        detail::cuda_check(cudaMemcpy(p_, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice),
                           "Array::copy_from");
    }
    std::vector<T> to_vec() const {
        std::vector<T> out(len_);
        if (len_) {
            detail::DeviceScope s(dev_.ordinal);
            detail::cuda_check(cudaMemcpy(out.data(), p_, len_ * sizeof(T), cudaMemcpyDeviceToHost), "Array::to_vec",
                               ForgeError::Kind::SyncFailed);
        }
        return out;
    }
    size_t len() const { return len_; }
    Device device() const { return dev_; }
    T* data() { return p_; }
    const T* data() const { return p_; }

    Array(Array&& o) noexcept : p_(o.p_), len_(o.len_), dev_(o.dev_) { o.p_ = nullptr, o.len_ = 0; }
    Array& operator=(Array&& o) noexcept {
        if (this != &o) {
            release();
            p_ = o.p_, len_ = o.len_, dev_ = o.dev_;
            o.p_ = nullptr, o.len_ = 0;
        }
        return *this;
    }
    Array(const Array&) = delete;
    Array& operator=(const Array&) = delete;
    ~Array() { release(); }

   private:
    void release() {
        if (!p_) return;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(dev_.ordinal);
        cudaFree(p_);
        cudaSetDevice(prev);
        p_ = nullptr;
    }
    T* p_ = nullptr;
    size_t len_ = 0;
    Device dev_{};
};

// RadixSorter (radix_sort.rs:26-220): a pre-allocated stable key/value
// sorter (capture-safe: nothing is allocated by sort()).
class RadixSorter {
   public:
    RadixSorter(size_t max_n, size_t ordinal)
        : max_n_(max_n), ordinal_((int)ordinal),
          keys_alt_(Array<uint32_t>::zeros(max_n, Device::Cuda((int)ordinal))),
          vals_alt_(Array<uint32_t>::zeros(max_n, Device::Cuda((int)ordinal))) {
        detail::check(forge_sorter_create(max_n, (int)ordinal, &h_), "RadixSorter::new");
    }
    ~RadixSorter() { forge_sorter_destroy(h_); }
    RadixSorter(const RadixSorter&) = delete;
    RadixSorter& operator=(const RadixSorter&) = delete;

    // Sorts (keys, values) by the low num_bits bits of the keys; afterwards
    // keys/values hold the result (the Arrays are swapped with the sorter's
    // alternates when the passes end there, radix_sort.rs:215-216).
    void sort(Array<uint32_t>& keys, Array<uint32_t>& values, size_t n, uint32_t num_bits) {
        if (n > max_n_)
            throw std::logic_error("n=" + std::to_string(n) + " exceeds max_n=" + std::to_string(max_n_));
        if (num_bits % 4 != 0 || num_bits > 32) throw std::logic_error("num_bits must be multiple of 4, <= 32");
        if (keys.len() < n || values.len() < n) throw std::logic_error("keys/values shorter than n");
        if (n == 0 || num_bits == 0) return;
        int in_alt = 0;
        // After a swap the alternates are the caller's old arrays; when those
        // are shorter than n the library ping-pongs through its own buffers
        // and leaves the result in keys/values.
        const bool alts = keys_alt_.len() >= n && vals_alt_.len() >= n;
        detail::check(forge_sorter_sort_pairs(h_, keys.data(), values.data(), alts ? keys_alt_.data() : nullptr,
                                              alts ? vals_alt_.data() : nullptr, n, 0, num_bits, &in_alt, nullptr),
                      "RadixSorter::sort");
        if (in_alt) {
            std::swap(keys, keys_alt_);
            std::swap(values, vals_alt_);
        }
    }

    // Device-side status of the sorts so far (bounded waits that gave up).
    void check() { detail::check(forge_sorter_check(h_, nullptr), "RadixSorter::check"); }
    size_t max_n() const { return max_n_; }

   private:
    forge_sorter* h_ = nullptr;
    size_t max_n_;
    int ordinal_;
    Array<uint32_t> keys_alt_, vals_alt_;
};

// find_cell_boundaries (radix_sort.rs:229-317): cell_start[c] = first index
// of cell c in sorted_cell_ids or 0xFFFFFFFF, cell_end[c] = one past its last
// index or 0.
inline void find_cell_boundaries(const Array<uint32_t>& sorted_cell_ids, Array<uint32_t>& cell_start,
                                 Array<uint32_t>& cell_end, size_t n, size_t num_cells, size_t ordinal) {
    if (sorted_cell_ids.len() < n || cell_start.len() < num_cells || cell_end.len() < num_cells)
        throw std::logic_error("find_cell_boundaries: arrays shorter than n / num_cells");
    detail::DeviceScope s((int)ordinal);
    detail::check(forge_cell_bounds(sorted_cell_ids.data(), cell_start.data(), cell_end.data(), n, num_cells, nullptr),
                  "find_cell_boundaries");
}

// HashGrid (hashgrid.rs:21-193), built and queried on the GPU.
class HashGrid {
   public:
    float cell_size;
    uint32_t dim_x, dim_y, dim_z;
    Vec3f origin;
    Array<uint32_t> cell_start;      // num_cells + 1
    Array<uint32_t> sorted_indices;  // max_particles
    Array<uint32_t> cell_indices;    // max_particles
    size_t num_particles = 0;

    HashGrid(float cell_size_, std::tuple<uint32_t, uint32_t, uint32_t> grid_dims, Vec3f origin_,
             size_t max_particles, Device device)
        : cell_size(cell_size_), dim_x(std::get<0>(grid_dims)), dim_y(std::get<1>(grid_dims)),
          dim_z(std::get<2>(grid_dims)), origin(origin_),
          cell_start(Array<uint32_t>::zeros(num_cells() + 1, device)),
          sorted_indices(Array<uint32_t>::zeros(max_particles, device)),
          cell_indices(Array<uint32_t>::zeros(max_particles, device)),
          px_(Array<float>::zeros(max_particles, device)), py_(Array<float>::zeros(max_particles, device)),
          pz_(Array<float>::zeros(max_particles, device)), dev_(device), max_(max_particles) {
        const float o[3] = {origin.x, origin.y, origin.z};
        detail::check(forge_grid_create(cell_size, dim_x, dim_y, dim_z, o, max_particles, device.ordinal, &h_),
                      "HashGrid::new");
    }
    ~HashGrid() { forge_grid_destroy(h_); }
    HashGrid(const HashGrid&) = delete;
    HashGrid& operator=(const HashGrid&) = delete;

    size_t num_cells() const { return (size_t)dim_x * dim_y * dim_z; }

    // HashGrid::build (hashgrid.rs:82-125): uploads the positions (kept on
    // the device for queries) and builds cell_indices, sorted_indices (stable
    // within a cell) and cell_start on the GPU.
    void build(const std::vector<Vec3f>& positions) {
        const size_t n = positions.size();
        if (n > max_)
            throw ForgeError(ForgeError::Kind::LaunchFailed, FORGE_ERR_CAPACITY,
                             "HashGrid::build: " + std::to_string(n) + " positions > max_particles " +
                                 std::to_string(max_));
        std::vector<float> x(n), y(n), z(n);
        for (size_t i = 0; i < n; ++i) x[i] = positions[i].x, y[i] = positions[i].y, z[i] = positions[i].z;
        px_.copy_from(x);
        py_.copy_from(y);
        pz_.copy_from(z);
        detail::DeviceScope s(dev_.ordinal);
        detail::check(forge_grid_build(h_, px_.data(), py_.data(), pz_.data(), n, cell_indices.data(),
                                       sorted_indices.data(), cell_start.data(), nullptr),
                      "HashGrid::build");
        num_particles = n;
    }

    // HashGrid::position_to_cell (hashgrid.rs:128-139), host arithmetic in f32.
    uint32_t position_to_cell(Vec3f pos) const { return cell_of(pos, origin, cell_size, dim_x, dim_y, dim_z); }

    // The cell hash itself: floor((p - origin) / cell_size) per axis (f32,
    // saturating to int, NaN -> 0), clamped to the grid, x fastest.
    static uint32_t cell_of(Vec3f pos, Vec3f origin, float cell_size, uint32_t nx, uint32_t ny, uint32_t nz) {
        auto axis = [&](float p, float o, uint32_t d) -> uint32_t {
            const float f = std::floor((p - o) / cell_size);
            long long v = std::isnan(f) ? 0 : (f >= 2147483647.f ? 2147483647LL
                                                                 : (f <= -2147483648.f ? -2147483648LL : (long long)f));
            if (v < 0) v = 0;
            if (v >= (long long)d) v = (long long)d - 1;
            return (uint32_t)v;
        };
        return axis(pos.x, origin.x, nx) + axis(pos.y, origin.y, ny) * nx + axis(pos.z, origin.z, nz) * nx * ny;
    }

    // HashGrid::query_neighbors (hashgrid.rs:145-193): indices within
    // `radius` (dist^2 <= radius^2) of pos, in the reference's walk order,
    // from the positions of the last build (`positions` must be those; the
    // reference passes them because its query runs on the host).
    std::vector<uint32_t> query_neighbors(Vec3f pos, float radius, const std::vector<Vec3f>& positions) const {
        if (positions.size() != num_particles)
            throw std::logic_error("HashGrid::query_neighbors: positions are not those of the last build");
        Array<float> q = Array<float>::from_vec({pos.x, pos.y, pos.z}, dev_);
        Array<uint32_t> counts = Array<uint32_t>::zeros(1, dev_), offsets = Array<uint32_t>::zeros(2, dev_);
        detail::DeviceScope s(dev_.ordinal);
        detail::check(forge_grid_query(h_, px_.data(), py_.data(), pz_.data(), q.data(), q.data() + 1, q.data() + 2,
                                       1, radius, counts.data(), offsets.data(), nullptr, 0, nullptr),
                      "HashGrid::query_neighbors");
        const uint32_t total = offsets.to_vec()[1];
        if (!total) return {};
        Array<uint32_t> hits = Array<uint32_t>::zeros(total, dev_);
        detail::check(forge_grid_query(h_, px_.data(), py_.data(), pz_.data(), q.data(), q.data() + 1, q.data() + 2,
                                       1, radius, counts.data(), offsets.data(), hits.data(), total, nullptr),
                      "HashGrid::query_neighbors");
        detail::check(forge_grid_check(h_, nullptr), "HashGrid::query_neighbors");
        return hits.to_vec();
    }

    forge_grid* handle() const { return h_; }

   private:
    forge_grid* h_ = nullptr;
    Array<float> px_, py_, pz_;
    Device dev_;
    size_t max_;
};

// ---------------------------------------------------------------------------
// Manifest modules (forge-manifest/src/modules)
// ---------------------------------------------------------------------------

// The SPH passes' grid, rebuilt by every density pass and shared with the
// force passes of the same step (the reference keeps it in u32_fields).
class SphGrid {
   public:
    SphGrid(float cell_size, const uint32_t dims[3], size_t max_n, Device d)
        : cell_size(cell_size), dims{dims[0], dims[1], dims[2]}, max_n(max_n), device(d) {
        const float o[3] = {0.f, 0.f, 0.f};
        detail::check(forge_grid_create(cell_size, dims[0], dims[1], dims[2], o, max_n, d.ordinal, &h),
                      "SphGrid::new");
    }
    ~SphGrid() { forge_grid_destroy(h); }
    SphGrid(const SphGrid&) = delete;
    SphGrid& operator=(const SphGrid&) = delete;
    bool fits(float cs, const uint32_t d[3], size_t n) const {
        return cs == cell_size && d[0] == dims[0] && d[1] == dims[1] && d[2] == dims[2] && n <= max_n;
    }
    float cell_size;
    uint32_t dims[3];
    size_t max_n;
    Device device;
    forge_grid* h = nullptr;
};

// FieldSet (modules/mod.rs:12-66): named SoA device arrays of one particle
// set (pos_x..vel_z, density, ...).
struct FieldSet {
    size_t particle_count;
    Device device;
    std::map<std::string, Array<float>> f32_fields;
    std::map<std::string, Array<uint32_t>> u32_fields;
    std::shared_ptr<SphGrid> sph_grid;

    FieldSet(size_t particle_count_, Device device_) : particle_count(particle_count_), device(device_) {}
    void add_f32(const std::string& name, const std::vector<float>& data) {
        f32_fields[name] = Array<float>::from_vec(data, device);
    }
    void add_f32_zeros(const std::string& name, size_t len) { f32_fields[name] = Array<float>::zeros(len, device); }
    Array<float>* get_f32(const std::string& name) {
        auto it = f32_fields.find(name);
        return it == f32_fields.end() ? nullptr : &it->second;
    }
    float* need(const std::string& name) {
        Array<float>* a = get_f32(name);
        if (!a || a->len() < particle_count)
            throw ForgeError(ForgeError::Kind::LaunchFailed, FORGE_OK, "FieldSet: missing field " + name);
        return a->data();
    }
};

// SimModule (modules/mod.rs:69-72). op() gives the per-particle modules'
// step op (for the fused force epilogue and forge_apply_ops).
class SimModule {
   public:
    virtual ~SimModule() = default;
    virtual std::string name() const = 0;
    virtual void execute(FieldSet& fields, float dt) = 0;
    virtual bool op(forge_step_op& /*out*/) const { return false; }
};

namespace detail {

inline forge_sph_params sph_params(float h, float mass, float gas, float rest, float visc) {
    forge_sph_params p{};
    p.h = h;
    p.mass = mass;
    p.gas_constant = gas;
    p.rest_density = rest;
    p.viscosity = visc;
    return p;
}

inline SphGrid& sph_grid(FieldSet& f, float cell_size, const uint32_t dims[3]) {
    if (!f.sph_grid || !f.sph_grid->fits(cell_size, dims, f.particle_count))
        f.sph_grid = std::make_shared<SphGrid>(cell_size, dims, f.particle_count, f.device);
    return *f.sph_grid;
}

inline float* density_field(FieldSet& f) {
    if (!f.get_f32("density")) f.add_f32_zeros("density", f.particle_count);
    return f.need("density");
}

// One per-particle module on its own (an unfused pipeline).
inline void apply_one(FieldSet& f, float dt, const forge_step_op& o) {
    forge_step_params sp{};
    sp.dt = dt;
    sp.n_ops = 1;
    sp.ops[0] = o;
    check(forge_apply_ops(&sp, f.need("pos_x"), f.need("pos_y"), f.need("pos_z"), f.need("vel_x"), f.need("vel_y"),
                          f.need("vel_z"), f.particle_count, f.device.ordinal, nullptr),
          "forge_apply_ops");
}

inline forge_step_op make_op(uint32_t kind, std::initializer_list<float> p) {
    forge_step_op o{};
    o.kind = kind;
    int k = 0;
    for (float v : p) o.p[k++] = v;
    return o;
}

}  // namespace detail

// SphFusedModule (sph_fused.rs:14-22, execute :413-733): grid rebuild,
// density, fused pressure + viscosity (Jacobi velocities).
struct SphFusedModule : SimModule {
    float smoothing_radius, cell_size;
    uint32_t grid_dims[3];
    float particle_mass, gas_constant, rest_density, viscosity_coefficient;
    SphFusedModule(float h, float cs, std::tuple<uint32_t, uint32_t, uint32_t> dims, float mass, float gas, float rest,
                   float visc)
        : smoothing_radius(h), cell_size(cs), grid_dims{std::get<0>(dims), std::get<1>(dims), std::get<2>(dims)},
          particle_mass(mass), gas_constant(gas), rest_density(rest), viscosity_coefficient(visc) {}
    std::string name() const override { return "sph_fused"; }
    forge_sph_params params() const {
        return detail::sph_params(smoothing_radius, particle_mass, gas_constant, rest_density, viscosity_coefficient);
    }
    void execute(FieldSet& f, float dt) override {
        SphGrid& g = detail::sph_grid(f, cell_size, grid_dims);
        const forge_sph_params p = params();
        float* rho = detail::density_field(f);
        detail::check(forge_sph_density(g.h, &p, f.need("pos_x"), f.need("pos_y"), f.need("pos_z"), f.particle_count,
                                        rho, nullptr),
                      "sph_fused density");
        detail::check(forge_sph_force(g.h, &p, (FORGE_TERM_PRESSURE | FORGE_TERM_VISCOSITY), f.need("pos_x"), f.need("pos_y"), f.need("pos_z"),
                                      f.need("vel_x"), f.need("vel_y"), f.need("vel_z"), rho, f.particle_count, dt,
                                      f.need("vel_x"), f.need("vel_y"), f.need("vel_z"), nullptr, nullptr, nullptr,
                                      nullptr),
                      "sph_fused force");
    }
};

// SphDensityModule (sph_density.rs:16-21, execute :385-501).
struct SphDensityModule : SimModule {
    float smoothing_radius, cell_size;
    uint32_t grid_dims[3];
    float particle_mass;
    SphDensityModule(float h, float cs, std::tuple<uint32_t, uint32_t, uint32_t> dims, float mass)
        : smoothing_radius(h), cell_size(cs), grid_dims{std::get<0>(dims), std::get<1>(dims), std::get<2>(dims)},
          particle_mass(mass) {}
    std::string name() const override { return "sph_density"; }
    void execute(FieldSet& f, float /*dt*/) override {
        SphGrid& g = detail::sph_grid(f, cell_size, grid_dims);
        const forge_sph_params p = detail::sph_params(smoothing_radius, particle_mass, 0.f, 0.f, 0.f);
        detail::check(forge_sph_density(g.h, &p, f.need("pos_x"), f.need("pos_y"), f.need("pos_z"), f.particle_count,
                                        detail::density_field(f), nullptr),
                      "sph_density");
    }
};

// The force passes of an unfused pipeline read the grid and density the
// density module left (sph_pressure.rs:20-161, sph_viscosity.rs:19-154).
struct SphForceModuleBase : SimModule {
    float smoothing_radius, particle_mass;
    SphForceModuleBase(float h, float mass) : smoothing_radius(h), particle_mass(mass) {}
    void run(FieldSet& f, float dt, uint32_t terms, const forge_sph_params& p, const char* what) {
        if (!f.sph_grid || !f.get_f32("density"))
            throw ForgeError(ForgeError::Kind::LaunchFailed, FORGE_OK,
                             std::string(what) + " needs a preceding sph_density module");
        detail::check(forge_sph_force(f.sph_grid->h, &p, terms, f.need("pos_x"), f.need("pos_y"), f.need("pos_z"),
                                      f.need("vel_x"), f.need("vel_y"), f.need("vel_z"), f.need("density"),
                                      f.particle_count, dt, f.need("vel_x"), f.need("vel_y"), f.need("vel_z"), nullptr,
                                      nullptr, nullptr, nullptr),
                      what);
    }
};

struct SphPressureModule : SphForceModuleBase {
    float gas_constant, rest_density;
    SphPressureModule(float h, float mass, float gas, float rest)
        : SphForceModuleBase(h, mass), gas_constant(gas), rest_density(rest) {}
    std::string name() const override { return "sph_pressure"; }
    void execute(FieldSet& f, float dt) override {
        run(f, dt, FORGE_TERM_PRESSURE,
            detail::sph_params(smoothing_radius, particle_mass, gas_constant, rest_density, 0.f), "sph_pressure");
    }
};

struct SphViscosityModule : SphForceModuleBase {
    float coefficient;
    SphViscosityModule(float h, float mass, float coeff) : SphForceModuleBase(h, mass), coefficient(coeff) {}
    std::string name() const override { return "sph_viscosity"; }
    void execute(FieldSet& f, float dt) override {
        run(f, dt, FORGE_TERM_VISCOSITY, detail::sph_params(smoothing_radius, particle_mass, 0.f, 0.f, coefficient),
            "sph_viscosity");
    }
};

// Per-particle modules: one forge_apply_ops call on their own, an op of the
// force epilogue inside a fused pipeline.
struct PerParticleModule : SimModule {
    void execute(FieldSet& f, float dt) override {
        forge_step_op o{};
        op(o);
        detail::apply_one(f, dt, o);
    }
};

struct GravityModule : PerParticleModule {  // gravity.rs:31-34
    float gx = 0.f, gy = -9.81f, gz = 0.f;
    GravityModule() = default;
    GravityModule(float x, float y, float z) : gx(x), gy(y), gz(z) {}
    std::string name() const override { return "gravity"; }
    bool op(forge_step_op& o) const override { return o = detail::make_op(FORGE_OP_GRAVITY, {gx, gy, gz}), true; }
};

struct DragModule : PerParticleModule {  // drag.rs: v *= 1 - coefficient * dt
    float coefficient = 0.f;
    explicit DragModule(float c) : coefficient(c) {}
    std::string name() const override { return "drag"; }
    bool op(forge_step_op& o) const override { return o = detail::make_op(FORGE_OP_DRAG, {coefficient}), true; }
};

struct IntegrateModule : PerParticleModule {  // integrate.rs:16-31
    std::string name() const override { return "integrate"; }
    bool op(forge_step_op& o) const override { return o = detail::make_op(FORGE_OP_INTEGRATE, {}), true; }
};

struct GroundPlaneModule : PerParticleModule {  // ground_plane.rs
    float y = 0.f, restitution = 0.5f;
    GroundPlaneModule(float y_, float e) : y(y_), restitution(e) {}
    std::string name() const override { return "ground_plane"; }
    bool op(forge_step_op& o) const override { return o = detail::make_op(FORGE_OP_GROUND, {y, restitution}), true; }
};

struct SphereColliderModule : PerParticleModule {  // sphere_collider.rs
    float cx, cy, cz, radius, restitution;
    SphereColliderModule(float x, float y, float z, float r, float e) : cx(x), cy(y), cz(z), radius(r), restitution(e) {}
    std::string name() const override { return "sphere_collider"; }
    bool op(forge_step_op& o) const override {
        return o = detail::make_op(FORGE_OP_SPHERE, {cx, cy, cz, radius, restitution}), true;
    }
};

struct BoxColliderModule : PerParticleModule {  // box_collider.rs:36-46
    float min_x, min_y, min_z, max_x, max_y, max_z, restitution;
    BoxColliderModule(float x0, float y0, float z0, float x1, float y1, float z1, float e)
        : min_x(x0), min_y(y0), min_z(z0), max_x(x1), max_y(y1), max_z(z1), restitution(e) {}
    std::string name() const override { return "box_collider"; }
    bool op(forge_step_op& o) const override {
        return o = detail::make_op(FORGE_OP_BOX, {min_x, min_y, min_z, max_x, max_y, max_z, restitution}), true;
    }
};

// Pipeline (modules/mod.rs:74-117). step_async recognises the manifest SPH
// pattern -- SphFusedModule followed only by per-particle modules (at most
// FORGE_STEP_MAX_OPS) -- and runs it as ONE forge_sph_step whose force
// kernel applies those modules in order; any other pipeline runs module by
// module.
class Pipeline {
   public:
    void add(std::unique_ptr<SimModule> m) { modules_.push_back(std::move(m)); }
    size_t len() const { return modules_.size(); }
    const std::vector<std::unique_ptr<SimModule>>& modules() const { return modules_; }

    // The fused plan: true and `sp` filled (ops, n_ops; dt left to the caller)
    // when the pipeline matches the pattern.
    bool fused_plan(forge_step_params& sp) const {
        if (modules_.empty() || !dynamic_cast<const SphFusedModule*>(modules_[0].get())) return false;
        if (modules_.size() - 1 > FORGE_STEP_MAX_OPS) return false;
        sp = forge_step_params{};
        for (size_t k = 1; k < modules_.size(); ++k)
            if (!modules_[k]->op(sp.ops[k - 1])) return false;
        sp.n_ops = (uint32_t)(modules_.size() - 1);
        return true;
    }

    void step_async(FieldSet& fields, float dt) {
        forge_step_params sp{};
        if (!fused_plan(sp)) {
            for (auto& m : modules_) m->execute(fields, dt);
            return;
        }
        sp.dt = dt;
        auto* sph = static_cast<SphFusedModule*>(modules_[0].get());
        SphGrid& g = detail::sph_grid(fields, sph->cell_size, sph->grid_dims);
        const forge_sph_params p = sph->params();
        detail::check(forge_sph_step(g.h, &p, &sp, fields.need("pos_x"), fields.need("pos_y"), fields.need("pos_z"),
                                     fields.need("vel_x"), fields.need("vel_y"), fields.need("vel_z"),
                                     detail::density_field(fields), fields.particle_count, nullptr),
                      "Pipeline::step_async");
    }

    void step(FieldSet& fields, float dt) {
        step_async(fields, dt);
        detail::DeviceScope s(fields.device.ordinal);
        detail::cuda_check(cudaDeviceSynchronize(), "Pipeline::step", ForgeError::Kind::SyncFailed);
    }

    void run(FieldSet& fields, float dt, size_t steps) {
        for (size_t i = 0; i < steps; ++i) step(fields, dt);
    }

   private:
    std::vector<std::unique_ptr<SimModule>> modules_;
};

}  // namespace forge
