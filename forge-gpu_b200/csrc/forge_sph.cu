// C ABI of the particle hot path: handles, launch plumbing and error
// reporting around the sm_100a kernels in radix_sort.cuh, grid.cuh, sph.cuh.
// Single translation unit -> libforge_sph.so.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "forge_sph.h"
#include "common.cuh"
#include "grid.cuh"
#include "radix_sort.cuh"
#include "sph.cuh"
#include "sph_group.cuh"
#include "sph_rows.cuh"
#include "sph_tile.cuh"
#include "slab.cuh"

using namespace forge;

namespace {

thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define FORGE_CUDA(call)                                                                              \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess)                                                                        \
            return set_error(FORGE_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                             __FILE__, __LINE__);                                                     \
    } while (0)

#define FORGE_LAUNCHED()                                                                              \
    do {                                                                                              \
        cudaError_t e_ = cudaGetLastError();                                                          \
        if (e_ != cudaSuccess)                                                                        \
            return set_error(FORGE_ERR_CUDA, "kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), \
                             __FILE__, __LINE__);                                                     \
    } while (0)

// Makes `dev` current for the scope of one API call and restores the caller's.
struct DeviceScope {
    int prev = -1;
    int dev;
    cudaError_t status = cudaSuccess;
    explicit DeviceScope(int d) : dev(d) {
        status = cudaGetDevice(&prev);
        if (status == cudaSuccess && prev != dev) status = cudaSetDevice(dev);
    }
    ~DeviceScope() {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    }
};

#define FORGE_DEVICE_SCOPE(d)                                                                         \
    DeviceScope scope_(d);                                                                            \
    if (scope_.status != cudaSuccess)                                                                 \
        return set_error(FORGE_ERR_CUDA, "cannot select device %d: %s", (d), cudaGetErrorString(scope_.status))

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

template <class T>
cudaError_t dalloc(T** p, size_t count) {
    return cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 16);
}

uint32_t grid_blocks(uint64_t work, uint32_t threads) { return (uint32_t)((work + threads - 1) / threads); }

// Launches a kernel of a step chain with programmatic dependent launch: its
// launch overlaps the previous kernel's drain, and its CTAs wait in
// pdl_enter() (common.cuh) until that kernel has completed. Errors
// surface through cudaGetLastError like a <<<>>> launch.
template <typename... KArgs, typename... Args>
void launch_pdl_smem(void (*kernel)(KArgs...), uint32_t grid, uint32_t block, uint32_t smem, cudaStream_t st,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), uint32_t grid, uint32_t block, cudaStream_t st, Args&&... args) {
    launch_pdl_smem(kernel, grid, block, 0, st, std::forward<Args>(args)...);
}

int num_sms(int device) {
    int v = 148;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    return v;
}

// Radix-sort scratch shared by the standalone sorter and the grid build:
// meta = [kMaxPasses x 256 digit histograms][kMaxPasses tile counters][status word].
// x-slices per cell (as bits) of the SPH passes' internal ordering.
constexpr uint32_t kSphSubBits = 2;

constexpr size_t kMetaHist = radix::kMaxPasses * radix::kRadix;
constexpr size_t kMetaCounters = kMetaHist;
constexpr size_t kMetaErr = kMetaHist + radix::kMaxPasses;
constexpr size_t kMetaWords = kMetaErr + 1;

struct SortScratch {
    uint32_t* meta = nullptr;    // kMetaWords
    uint32_t* status = nullptr;  // tiles * 256 (+pad to uint4)
    uint32_t max_tiles = 0;
    int sms = 148;
    // failure-detection test hook (forge_sorter_set_test_fault): the first
    // pass skips tile ids below skip_tiles; look-back waits give up after
    // spin_limit polls
    uint32_t skip_tiles = 0;
    uint32_t spin_limit = kSpinLimit;
};

int scratch_alloc(SortScratch& s, uint64_t max_n, int device) {
    const uint64_t m = max_n > 0 ? max_n : 1;
    s.max_tiles = std::max(radix::num_tiles(m), radix::num_tiles(std::min<uint64_t>(m, radix::kSmallN),
                                                                 radix::kSmallTile));
    FORGE_CUDA(dalloc(&s.meta, kMetaWords));
    FORGE_CUDA(cudaMemset(s.meta, 0, kMetaWords * sizeof(uint32_t)));
    FORGE_CUDA(dalloc(&s.status, (size_t)s.max_tiles * radix::kRadix));
    s.sms = num_sms(device);
    return FORGE_OK;
}

void scratch_free(SortScratch& s) {
    cudaFree(s.meta);
    cudaFree(s.status);
    s.meta = nullptr;
    s.status = nullptr;
}

// Runs histogram + passes. The histogram kernel reads keys through `src`.
// Pass 0 reads keys0 (vals0, or iota if vals0 == nullptr) and writes
// (ka, va); later passes ping-pong between (ka, va) and (kb, vb).
// Returns 0 if the result is in (ka, va), 1 if in (kb, vb).
template <class Src>
int run_onesweep(const SortScratch& s, Src src, const uint32_t* keys0, const uint32_t* vals0, uint32_t* ka,
                 uint32_t* va, uint32_t* kb, uint32_t* vb, uint32_t n, uint32_t begin_bit, uint32_t end_bit,
                 cudaStream_t st, int* where, bool meta_zeroed = false) {
    const uint32_t passes = (end_bit - begin_bit + radix::kRadixBits - 1) / radix::kRadixBits;
    const bool small = n <= radix::kSmallN && s.max_tiles >= radix::num_tiles(n, radix::kSmallTile);
    const uint32_t tiles = small ? radix::num_tiles(n, radix::kSmallTile) : radix::num_tiles(n);
    // histograms and tile counters start at zero (meta_zeroed: the caller's
    // previous use left them so)
    if (!meta_zeroed) FORGE_CUDA(cudaMemsetAsync(s.meta, 0, kMetaErr * sizeof(uint32_t), st));
    const uint32_t status_vec4 = (uint32_t)(((size_t)tiles * radix::kRadix + 3) / 4);
    const uint32_t hblocks =
        std::max(1u, std::min(grid_blocks(n, radix::kHistThreads * radix::kHistItems), (uint32_t)s.sms * 8u));
    launch_pdl(radix::digit_histogram_kernel<Src>, hblocks, radix::kHistThreads, st,
        src, n, begin_bit, end_bit, passes, s.meta, reinterpret_cast<uint4*>(s.status), status_vec4);
    FORGE_LAUNCHED();
    const uint32_t* kin = keys0;
    const uint32_t* vin = vals0;
    int cur = -1;
    for (uint32_t p = 0; p < passes; ++p) {
        uint32_t* kout = (p % 2 == 0) ? ka : kb;
        uint32_t* vout = (p % 2 == 0) ? va : vb;
        const uint32_t shift = begin_bit + p * radix::kRadixBits;
        const uint32_t bits = std::min((uint32_t)radix::kRadixBits, end_bit - shift);
        const uint32_t skip = p == 0 ? s.skip_tiles : 0u;
        uint32_t* hist = s.meta + p * radix::kRadix;
        uint32_t* counter = s.meta + kMetaCounters + p;
        uint32_t* err = s.meta + kMetaErr;
        const bool iota = p == 0 && vin == nullptr;
        if (small && iota)
            launch_pdl(radix::onesweep_pass_kernel<true, radix::kSmallItems>, tiles, radix::kThreads, st,
                kin, nullptr, kout, vout, n, shift, bits, hist, s.status, counter, p & 1u, err, skip, s.spin_limit,
                tiles);
        else if (small)
            launch_pdl(radix::onesweep_pass_kernel<false, radix::kSmallItems>, tiles, radix::kThreads, st,
                kin, vin, kout, vout, n, shift, bits, hist, s.status, counter, p & 1u, err, skip, s.spin_limit,
                tiles);
        else if (iota)
            launch_pdl(radix::onesweep_pass_kernel<true>, tiles, radix::kThreads, st,
                kin, nullptr, kout, vout, n, shift, bits, hist, s.status, counter, p & 1u, err, skip, s.spin_limit,
                tiles);
        else
            launch_pdl(radix::onesweep_pass_kernel<false>, tiles, radix::kThreads, st,
                kin, vin, kout, vout, n, shift, bits, hist, s.status, counter, p & 1u, err, skip, s.spin_limit,
                tiles);
        FORGE_LAUNCHED();
        kin = kout;
        vin = vout;
        cur = (int)(p % 2);
    }
    *where = cur;
    return FORGE_OK;
}

int check_status_word(uint32_t* word, cudaStream_t st, const char* what) {
    FORGE_CUDA(cudaStreamSynchronize(st));
    uint32_t v = 0;
    FORGE_CUDA(cudaMemcpy(&v, word, sizeof v, cudaMemcpyDeviceToHost));
    if (v == 0) return FORGE_OK;
    FORGE_CUDA(cudaMemset(word, 0, sizeof v));
    if (v & kDevTimeout) return set_error(FORGE_ERR_TIMEOUT, "%s: a look-back wait on the device gave up", what);
    if (v & kDevCapacity) return set_error(FORGE_ERR_CAPACITY, "%s: output capacity exceeded on the device", what);
    if (v & kDevKeyRange) return set_error(FORGE_ERR_DEVICE, "%s: device-side range check failed", what);
    return set_error(FORGE_ERR_DEVICE, "%s: device status 0x%x", what, v);
}

}  // namespace

// ===========================================================================
// Errors / version
// ===========================================================================
extern "C" uint64_t forge_last_error(char* buf, uint64_t len) {
    const std::string& m = g_last_error;
    if (buf && len) {
        const size_t c = std::min<size_t>(m.size(), len - 1);
        memcpy(buf, m.data(), c);
        buf[c] = 0;
    }
    return m.size();
}

extern "C" int forge_abi_version(void) { return FORGE_SPH_ABI_VERSION; }

// ===========================================================================
// Standalone sorter
// ===========================================================================
struct forge_sorter {
    int device = 0;
    uint64_t max_n = 0;
    uint32_t* keys_alt = nullptr;
    uint32_t* vals_alt = nullptr;
    SortScratch scratch;
};

extern "C" int forge_sorter_create(uint64_t max_n, int device, forge_sorter** out) {
    if (!out) return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_create: out is NULL");
    *out = nullptr;
    if (max_n > radix::kMaxN)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_create: max_n=%llu exceeds %llu",
                         (unsigned long long)max_n, (unsigned long long)radix::kMaxN);
    FORGE_DEVICE_SCOPE(device);
    forge_sorter* s = new forge_sorter;
    s->device = device;
    s->max_n = max_n;
    int rc = FORGE_OK;
    if (cudaMalloc(&s->keys_alt, (max_n ? max_n : 1) * 4) != cudaSuccess ||
        cudaMalloc(&s->vals_alt, (max_n ? max_n : 1) * 4) != cudaSuccess) {
        rc = set_error(FORGE_ERR_CUDA, "forge_sorter_create: cudaMalloc of %llu pairs failed",
                       (unsigned long long)max_n);
    } else {
        rc = scratch_alloc(s->scratch, max_n, device);
    }
    if (rc != FORGE_OK) {
        cudaFree(s->keys_alt);
        cudaFree(s->vals_alt);
        scratch_free(s->scratch);
        delete s;
        return rc;
    }
    *out = s;
    return FORGE_OK;
}

extern "C" int forge_sorter_sort_pairs(forge_sorter* s, uint32_t* keys, uint32_t* vals, uint32_t* keys_alt,
                                       uint32_t* vals_alt, uint64_t n, uint32_t begin_bit, uint32_t end_bit,
                                       int* result_in_alt, void* stream) {
    if (result_in_alt) *result_in_alt = 0;
    if (!s) return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_sort_pairs: sorter is NULL");
    if (n > s->max_n)
        return set_error(FORGE_ERR_CAPACITY, "forge_sorter_sort_pairs: n=%llu exceeds max_n=%llu",
                         (unsigned long long)n, (unsigned long long)s->max_n);
    if (begin_bit >= end_bit || end_bit > 32 || end_bit - begin_bit > 8 * radix::kMaxPasses)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_sort_pairs: bad bit range [%u, %u)", begin_bit,
                         end_bit);
    if ((keys_alt == nullptr) != (vals_alt == nullptr))
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_sort_pairs: pass both alt buffers or neither");
    if (n == 0) return FORGE_OK;
    if (!keys || !vals) return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_sort_pairs: keys/vals NULL");
    FORGE_DEVICE_SCOPE(s->device);
    cudaStream_t st = as_stream(stream);
    const bool own_alt = keys_alt == nullptr;
    uint32_t* ka = own_alt ? s->keys_alt : keys_alt;
    uint32_t* va = own_alt ? s->vals_alt : vals_alt;
    int where = 0;
    radix::KeysFromArray src{keys};
    int rc = run_onesweep(s->scratch, src, keys, vals, ka, va, keys, vals, (uint32_t)n, begin_bit, end_bit, st,
                          &where);
    if (rc != FORGE_OK) return rc;
    if (where == 0) {  // result in (ka, va)
        if (own_alt) {
            FORGE_CUDA(cudaMemcpyAsync(keys, ka, n * 4, cudaMemcpyDeviceToDevice, st));
            FORGE_CUDA(cudaMemcpyAsync(vals, va, n * 4, cudaMemcpyDeviceToDevice, st));
        } else if (result_in_alt) {
            *result_in_alt = 1;
        }
    }
    return FORGE_OK;
}

// ===========================================================================
// Allocation-free sort: scratch in a file-scope device array
// ===========================================================================
namespace {

constexpr uint64_t kStaticMaxN = FORGE_STATIC_SORT_MAX_N;
constexpr size_t kStaticTiles = (kStaticMaxN + radix::kTile - 1) / radix::kTile;
// [meta | look-back status | alternate keys | alternate values], in words;
// each part starts on a 16-byte boundary (kMetaWords rounded up to 4).
constexpr size_t kStaticMetaWords = (kMetaWords + 3) / 4 * 4;
constexpr size_t kStaticStatusWords = kStaticTiles * radix::kRadix;
constexpr size_t kStaticWords = kStaticMetaWords + kStaticStatusWords + 2 * kStaticMaxN;

static __device__ __align__(256) uint32_t g_static_sort_scratch[kStaticWords];

// Device address of g_static_sort_scratch per device ordinal. In host code the
// symbol's name is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress (with that device current). The lookup is cached
// together with the unique id of the CUDA context it was made in: after a
// cudaDeviceReset, or under another context, the module (and the array) may
// be loaded again at another address, and the next call looks it up anew.
std::mutex g_static_mu;
struct StaticAddr {
    uint32_t* addr = nullptr;
    unsigned long long ctx_id = 0;
};
StaticAddr g_static_addr[64];

// Unique id of the calling thread's current context (cuCtxGetCurrent +
// cuCtxGetId through the runtime's driver entry points, so the library need
// not link libcuda); 0 if unavailable.
unsigned long long current_ctx_id() {
    using GetCurrent = int (*)(void**);
    using GetId = int (*)(void*, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
    return 0;
}

int static_scratch(int dev, uint32_t** out) {
    if (dev < 0 || dev >= 64) return set_error(FORGE_ERR_INVALID_ARG, "forge_sort_pairs_static: device %d", dev);
    const unsigned long long ctx = current_ctx_id();
    std::lock_guard<std::mutex> lock(g_static_mu);
    StaticAddr& a = g_static_addr[dev];
    if (!a.addr || ctx == 0 || a.ctx_id != ctx) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_sort_scratch);
        if (e != cudaSuccess)
            return set_error(FORGE_ERR_CUDA, "forge_sort_pairs_static: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        a.addr = static_cast<uint32_t*>(p);
        a.ctx_id = ctx;
    }
    *out = a.addr;
    return FORGE_OK;
}

}  // namespace

extern "C" int forge_sort_pairs_static(uint32_t* keys, uint32_t* vals, uint64_t n, uint32_t begin_bit,
                                       uint32_t end_bit, void* stream) {
    if (n > kStaticMaxN)
        return set_error(FORGE_ERR_CAPACITY, "forge_sort_pairs_static: n=%llu exceeds the static maximum %llu",
                         (unsigned long long)n, (unsigned long long)kStaticMaxN);
    if (begin_bit >= end_bit || end_bit > 32)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sort_pairs_static: bad bit range [%u, %u)", begin_bit,
                         end_bit);
    if (n == 0) return FORGE_OK;
    if (!keys || !vals) return set_error(FORGE_ERR_INVALID_ARG, "forge_sort_pairs_static: keys/vals NULL");
    int dev = 0;
    FORGE_CUDA(cudaGetDevice(&dev));
    uint32_t* base = nullptr;
    int rc = static_scratch(dev, &base);
    if (rc != FORGE_OK) return rc;
    SortScratch s;
    s.meta = base;
    s.status = base + kStaticMetaWords;
    s.max_tiles = (uint32_t)kStaticTiles;
    s.sms = num_sms(dev);
    uint32_t* ka = s.status + kStaticStatusWords;
    uint32_t* va = ka + kStaticMaxN;
    cudaStream_t st = as_stream(stream);
    int where = 0;
    // run_onesweep clears the histograms and tile counters (memset) and the
    // look-back table (histogram kernel) left by the previous call.
    rc = run_onesweep(s, radix::KeysFromArray{keys}, keys, vals, ka, va, keys, vals, (uint32_t)n, begin_bit,
                      end_bit, st, &where);
    if (rc != FORGE_OK) return rc;
    if (where == 0) {  // odd pass count: result is in the static alternate pair
        FORGE_CUDA(cudaMemcpyAsync(keys, ka, n * 4, cudaMemcpyDeviceToDevice, st));
        FORGE_CUDA(cudaMemcpyAsync(vals, va, n * 4, cudaMemcpyDeviceToDevice, st));
    }
    return FORGE_OK;
}

extern "C" int forge_sorter_check(forge_sorter* s, void* stream) {
    if (!s) return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_check: sorter is NULL");
    FORGE_DEVICE_SCOPE(s->device);
    return check_status_word(s->scratch.meta + kMetaErr, as_stream(stream), "radix sort");
}

extern "C" int forge_sorter_set_test_fault(forge_sorter* s, uint32_t skip_tiles, uint32_t spin_limit) {
    if (!s) return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_set_test_fault: sorter is NULL");
    if (skip_tiles > 1) return set_error(FORGE_ERR_INVALID_ARG, "forge_sorter_set_test_fault: skip_tiles is 0 or 1");
    s->scratch.skip_tiles = skip_tiles;
    s->scratch.spin_limit = spin_limit ? spin_limit : kSpinLimit;
    return FORGE_OK;
}

extern "C" void forge_sorter_destroy(forge_sorter* s) {
    if (!s) return;
    DeviceScope scope(s->device);
    cudaFree(s->keys_alt);
    cudaFree(s->vals_alt);
    scratch_free(s->scratch);
    delete s;
}

extern "C" int forge_cell_bounds(const uint32_t* sorted_ids, uint32_t* start, uint32_t* end, uint64_t n,
                                 uint64_t num_cells, void* stream) {
    if (num_cells == 0) return FORGE_OK;
    if (!start || !end || (n && !sorted_ids))
        return set_error(FORGE_ERR_INVALID_ARG, "forge_cell_bounds: NULL pointer");
    if (n >= 0xffffffffull || num_cells >= 0xffffffffull)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_cell_bounds: sizes must be < 2^32-1");
    cudaStream_t st = as_stream(stream);
    grid::cell_bounds_kernel<<<grid_blocks(n + 1, 256), 256, 0, st>>>(sorted_ids, (uint32_t)n, (uint32_t)num_cells,
                                                                       start, end, nullptr);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

// ===========================================================================
// Grid
// ===========================================================================
struct forge_grid {
    int device = 0;
    uint64_t max_n = 0;
    grid::GridGeom geom{};
    uint32_t C = 0;
    uint32_t key_bits = 1;
    uint32_t* cell_idx = nullptr;  // hash output, original order
    uint32_t* kb = nullptr;
    uint32_t* vb = nullptr;
    uint32_t* kc = nullptr;
    uint32_t* vc = nullptr;
    uint32_t* cell_start = nullptr;  // (C << kSphSubBits) + 1
    uint32_t* chunk_val = nullptr;   // marks of whole table chunks to fill (grid::kFillChunk entries each)
    uint32_t sub_bits = 0;           // x-slices of the last build (0: plain cells)
    int walk = FORGE_WALK_AUTO;      // neighbour-pass kernel family (forge_grid_set_walk)
    float4* pos4 = nullptr;          // cell-ordered (x, y, z, key)
    float4* vel4 = nullptr;          // cell-ordered (vx, vy, vz, 1/rho)
    float2* aux = nullptr;           // cell-ordered (p/rho, rho)
    uint32_t* scan_sums = nullptr;   // query scan tile sums
    uint32_t* q_offsets = nullptr;   // max_n + 1
    SortScratch scratch;
    // State of the last build.
    uint32_t* sorted_keys = nullptr;
    uint32_t* sorted_idx = nullptr;
    uint64_t n = 0;
    bool built = false;
    bool force_gathered = false;  // a zone prepare step gathered velocities + density of this build
    // Zone lists of a zoned force pass (allocated by the first one).
    uint32_t* zone_idx = nullptr;     // [A (empty) | boundary | interior] sorted positions, max_n
    uint32_t* zone_tiles = nullptr;   // classification tile counts
    uint32_t* zone_counts = nullptr;  // list sizes A (0), boundary, interior
    cudaEvent_t ev_zone = nullptr;  // gather + zone lists of the last boundary pass done
    // Phase-event ring for forge_grid_profile_* (5 events per step).
    std::vector<cudaEvent_t> prof_events;
    uint32_t prof_cap = 0, prof_next = 0, prof_count = 0;
};

namespace {
void prof_mark(forge_grid* g, int k, cudaStream_t st) {
    if (g->prof_cap) cudaEventRecord(g->prof_events[(size_t)g->prof_next * 5 + k], st);
}
void prof_step_done(forge_grid* g) {
    if (!g->prof_cap) return;
    g->prof_next = (g->prof_next + 1) % g->prof_cap;
    if (g->prof_count < g->prof_cap) ++g->prof_count;
}
void prof_free(forge_grid* g) {
    for (cudaEvent_t e : g->prof_events) cudaEventDestroy(e);
    g->prof_events.clear();
    g->prof_cap = g->prof_next = g->prof_count = 0;
}
}  // namespace

extern "C" int forge_grid_create(float cell_size, uint32_t nx, uint32_t ny, uint32_t nz, const float* origin,
                                 uint64_t max_n, int device, forge_grid** out) {
    if (!out) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_create: out is NULL");
    *out = nullptr;
    if (!(cell_size > 0.f)) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_create: cell_size must be > 0");
    const uint64_t C = (uint64_t)nx * ny * nz;
    if (nx == 0 || ny == 0 || nz == 0 || C >= (1ull << (31 - kSphSubBits)))
        return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_create: grid %ux%ux%u must be non-empty and < 2^29 cells",
                         nx, ny, nz);
    if (max_n > radix::kMaxN)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_create: max_n exceeds %llu",
                         (unsigned long long)radix::kMaxN);
    FORGE_DEVICE_SCOPE(device);
    forge_grid* g = new forge_grid;
    g->device = device;
    g->max_n = max_n;
    g->geom.ox = origin ? origin[0] : 0.f;
    g->geom.oy = origin ? origin[1] : 0.f;
    g->geom.oz = origin ? origin[2] : 0.f;
    g->geom.cs = cell_size;
    g->geom.nx = (int)nx;
    g->geom.ny = (int)ny;
    g->geom.nz = (int)nz;
    g->geom.cx0 = 0;
    g->geom.nxw = (int)nx;
    g->C = (uint32_t)C;
    uint32_t kb = 1;
    while (kb < 32 && (1ull << kb) < C) ++kb;
    g->key_bits = kb;
    const size_t m = max_n ? max_n : 1;
    int rc = FORGE_OK;
    bool ok = dalloc(&g->cell_idx, m) == cudaSuccess && dalloc(&g->kb, m) == cudaSuccess &&
              dalloc(&g->vb, m) == cudaSuccess && dalloc(&g->kc, m) == cudaSuccess &&
              dalloc(&g->vc, m) == cudaSuccess && dalloc(&g->cell_start, (C << kSphSubBits) + 1) == cudaSuccess &&
              dalloc(&g->chunk_val, (C << kSphSubBits) / grid::kFillChunk + 1) == cudaSuccess &&
              cudaMemset(g->chunk_val, 0xff, ((C << kSphSubBits) / grid::kFillChunk + 1) * sizeof(uint32_t)) ==
                  cudaSuccess &&
              dalloc(&g->pos4, m) == cudaSuccess && dalloc(&g->vel4, m) == cudaSuccess &&
              dalloc(&g->aux, m) == cudaSuccess &&
              dalloc(&g->scan_sums, m / grid::kScanTile + 1) == cudaSuccess &&
              dalloc(&g->q_offsets, m + 1) == cudaSuccess;
    if (!ok) rc = set_error(FORGE_ERR_CUDA, "forge_grid_create: cudaMalloc failed (max_n=%llu, cells=%llu)",
                            (unsigned long long)max_n, (unsigned long long)C);
    if (rc == FORGE_OK) rc = scratch_alloc(g->scratch, max_n, device);
    // the cell-block density pass stages up to kTileCap positions (64 KiB)
    if (rc == FORGE_OK && cudaFuncSetAttribute(sph::density_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)(sph::kTileCap * sizeof(float4))) != cudaSuccess)
        rc = set_error(FORGE_ERR_CUDA, "forge_grid_create: shared-memory attribute of the tile pass");
    if (rc != FORGE_OK) {
        forge_grid_destroy(g);
        return rc;
    }
    *out = g;
    return FORGE_OK;
}

extern "C" void forge_grid_destroy(forge_grid* g) {
    if (!g) return;
    DeviceScope scope(g->device);
    cudaFree(g->cell_idx);
    cudaFree(g->kb);
    cudaFree(g->vb);
    cudaFree(g->kc);
    cudaFree(g->vc);
    cudaFree(g->cell_start);
    cudaFree(g->chunk_val);
    cudaFree(g->pos4);
    cudaFree(g->vel4);
    cudaFree(g->aux);
    cudaFree(g->scan_sums);
    cudaFree(g->q_offsets);
    cudaFree(g->zone_idx);
    cudaFree(g->zone_tiles);
    cudaFree(g->zone_counts);
    if (g->ev_zone) cudaEventDestroy(g->ev_zone);
    scratch_free(g->scratch);
    prof_free(g);
    delete g;
}

namespace {

// Cells of the grid's x-window (the table's extent) and the key bits that
// index them.
uint32_t cells_w(const forge_grid* g) {
    return (uint32_t)g->geom.nxw * (uint32_t)g->geom.ny * (uint32_t)g->geom.nz;
}
uint32_t key_bits_w(const forge_grid* g) {
    const uint32_t C = cells_w(g);
    uint32_t kb = 1;
    while (kb < 32 && (1ull << kb) < C) ++kb;
    return kb;
}

// Hash + sort + cell-start table (+ optional cell-ordered gather).
// sub_bits > 0 (the SPH passes): keys are cell << sub_bits | x-slice, so the
// cell-ordered arrays are also ordered by x-slice inside each cell and the
// table has (C << sub_bits) + 1 entries.
int grid_build_impl(forge_grid* g, const float* px, const float* py, const float* pz, uint32_t stride, uint64_t n,
                    uint32_t* cell_idx_out, bool gather_pos, const float* vx, const float* vy, const float* vz,
                    cudaStream_t st, uint32_t sub_bits = 0) {
    if (n > g->max_n)
        return set_error(FORGE_ERR_CAPACITY, "grid build: n=%llu exceeds max_n=%llu", (unsigned long long)n,
                         (unsigned long long)g->max_n);
    if (n && (!px || !py || !pz)) return set_error(FORGE_ERR_INVALID_ARG, "grid build: NULL positions");
    uint32_t* keys = cell_idx_out ? cell_idx_out : g->cell_idx;
    const uint32_t nn = (uint32_t)n;
    if (n > 0) {
        grid::HashKeys src{px, py, pz, stride, g->geom, keys, sub_bits};
        int where = 0;
        int rc = run_onesweep(g->scratch, src, keys, nullptr, g->kb, g->vb, g->kc, g->vc, nn, 0,
                              key_bits_w(g) + sub_bits, st, &where, true);
        if (rc != FORGE_OK) return rc;
        g->sorted_keys = where == 0 ? g->kb : g->kc;
        g->sorted_idx = where == 0 ? g->vb : g->vc;
    } else {
        g->sorted_keys = g->kb;
        g->sorted_idx = g->vb;
    }
    prof_mark(g, 1, st);
    grid::GatherSrc gs{px, py, pz, stride, vx, vy, vz};
    const uint32_t table = cells_w(g) << sub_bits;  // entries [0, table]
    launch_pdl(grid::cell_start_gather_kernel, grid_blocks(n + 1, 256), 256, st,
        g->sorted_keys, g->sorted_idx, nn, table, g->cell_start, gs, gather_pos ? g->pos4 : nullptr,
        (gather_pos && vx) ? g->vel4 : nullptr, g->chunk_val, g->scratch.meta, (uint32_t)kMetaErr);
    const uint32_t chunks = table / grid::kFillChunk;  // whole chunks below entry `table`
    if (chunks)
        launch_pdl(grid::fill_chunks_kernel, std::min(chunks, (uint32_t)g->scratch.sms * 8u), 256, st, g->cell_start,
                                                                                                g->chunk_val, chunks);
    FORGE_LAUNCHED();
    prof_mark(g, 2, st);
    g->n = n;
    g->built = true;
    g->force_gathered = false;
    g->sub_bits = sub_bits;
    return FORGE_OK;
}

int grid_export(forge_grid* g, uint32_t* sorted_idx, uint32_t* cell_start, cudaStream_t st) {
    if (sorted_idx && g->n)
        FORGE_CUDA(cudaMemcpyAsync(sorted_idx, g->sorted_idx, g->n * 4, cudaMemcpyDeviceToDevice, st));
    if (cell_start)
        FORGE_CUDA(cudaMemcpyAsync(cell_start, g->cell_start, ((size_t)cells_w(g) + 1) * 4, cudaMemcpyDeviceToDevice,
                                   st));
    return FORGE_OK;
}

sph::SphConsts make_consts(const forge_sph_params* p) {
    // Same float expressions as the reference kernels (sph_density.rs:413-416,
    // sph_fused.rs:552-555); products/quotients only, so host == device bits.
    sph::SphConsts c;
    const float h = p->h;
    const float h2 = h * h;
    const float h9 = h2 * h2 * h2 * h2 * h;
    const float poly6 = 315.0f / (64.0f * 3.14159265f * h9);
    const float h6 = h2 * h2 * h2;
    const float spiky = -45.0f / (3.14159265f * h6);
    const float visc_lap = 45.0f / (3.14159265f * h6);
    c.h = h;
    c.h2 = h2;
    c.h2_skip = h2 * (1.0f + 1e-4f);
    c.mass_poly6 = p->mass * poly6;
    c.mass = p->mass;
    c.k = p->gas_constant;
    c.rho0 = p->rest_density;
    c.mu = p->viscosity;
    c.kp = -0.5f * p->mass * spiky;
    c.kv = p->viscosity * p->mass * visc_lap;
    return c;
}

sph::Geom geom_of(const forge_grid* g, float h) {
    sph::Geom G{g->geom.ox, g->geom.oy, g->geom.oz, g->geom.cs, g->geom.nxw, g->geom.ny, g->geom.nz,
                (int)g->sub_bits, g->geom.cs >= h ? 1 : 0};
    G.inv_slice = (float)(1u << g->sub_bits) / g->geom.cs;
    G.x_off = (int)((uint32_t)g->geom.cx0 << g->sub_bits);
    G.row_len = make_fastdiv((uint32_t)g->geom.nxw << g->sub_bits);
    G.ny_div = make_fastdiv((uint32_t)g->geom.ny);
    G.keys = g->sorted_keys;
    return G;
}

constexpr uint32_t kSphThreads = 128;

// Two particles per thread pay off when cells are sparse (the candidate scan
// dominates); with dense cells the per-hit work dominates and one particle
// per thread diverges less. Mean occupancy n / C selects the kernel.
constexpr double kPairMaxOccupancy = 8.0;

// Neighbour-pass kernel family of a build. Per-thread walks (one, two or
// four particles per thread) need many particles to fill the GPU: below
// kSmallWalkMaxN particles, row-parallel walks (sph_rows.cuh) give every
// particle nine threads instead, one per neighbour row (the reference's 50K
// dam break: 101 -> 60 us per step against the group walks; 65,536 uniform
// particles: 0.16 -> 0.10 ms against per-thread walks).
#ifndef FORGE_SMALL_WALK_MAX_N
#define FORGE_SMALL_WALK_MAX_N (1u << 18)
#endif
constexpr uint64_t kSmallWalkMaxN = FORGE_SMALL_WALK_MAX_N;

int walk_of(const forge_grid* g) {
    if (g->walk != FORGE_WALK_AUTO) return g->walk;
    return g->n < kSmallWalkMaxN ? FORGE_WALK_ROWS : FORGE_WALK_THREAD;
}

template <int G>
uint32_t group_blocks(uint64_t n) {
    return grid_blocks((n + G - 1) / G * 32, kSphThreads);
}

uint32_t rows_blocks(uint64_t n) {
    return (uint32_t)((n + sph::kRowsParticles - 1) / sph::kRowsParticles);
}

int launch_density(forge_grid* g, const forge_sph_params* p, float* density, cudaStream_t st) {
    if (g->n == 0) return FORGE_OK;
    const sph::Geom G = geom_of(g, p->h);
    const sph::SphConsts c = make_consts(p);
    const uint32_t n = (uint32_t)g->n;
    switch (walk_of(g)) {
        case FORGE_WALK_GROUP4:
            launch_pdl(sph::density_group_kernel<4>, group_blocks<4>(n), kSphThreads, st,
                g->pos4, g->cell_start, g->sorted_idx, n, G, c, g->vel4, g->aux, density);
            break;
        case FORGE_WALK_GROUP8:
            launch_pdl(sph::density_group_kernel<8>, group_blocks<8>(n), kSphThreads, st,
                g->pos4, g->cell_start, g->sorted_idx, n, G, c, g->vel4, g->aux, density);
            break;
        case FORGE_WALK_GROUP16:
            launch_pdl(sph::density_group_kernel<16>, group_blocks<16>(n), kSphThreads, st,
                g->pos4, g->cell_start, g->sorted_idx, n, G, c, g->vel4, g->aux, density);
            break;
        case FORGE_WALK_TILE:
            if (g->sub_bits <= (uint32_t)sph::kTileMaxSub) {
                const uint32_t segs = (uint32_t)((G.nx + sph::kTileCells - 1) / sph::kTileCells);
                launch_pdl_smem(sph::density_tile_kernel, (uint32_t)G.ny * (uint32_t)G.nz * segs, sph::kTileThreads,
                                (uint32_t)(sph::kTileCap * sizeof(float4)), st, g->pos4, g->cell_start, g->sorted_idx,
                                G, c, segs, g->vel4, g->aux, density, g->scratch.meta + kMetaErr);
                break;
            }
            [[fallthrough]];
        case FORGE_WALK_ROWS:
            launch_pdl(sph::density_rows_kernel, rows_blocks(n), sph::kRowsThreads, st,
                g->pos4, g->cell_start, g->sorted_idx, n, G, c, g->vel4, g->aux, density);
            break;
        default:
            // Four particles per thread share each neighbour load where cells
            // hold a few particles (cfg3: 1.41 -> 1.25 ms); with dense cells
            // the union of four windows adds more evaluations than it saves
            // loads: two per thread.
            if ((double)n / (double)cells_w(g) < kPairMaxOccupancy)
                launch_pdl(sph::density_multi_kernel<4>, grid_blocks((n + 3) / 4, kSphThreads), kSphThreads, st,
                    g->pos4, g->cell_start, g->sorted_idx, n, G, c, g->vel4, g->aux, density);
            else
                launch_pdl(sph::density_pair_kernel, grid_blocks((n + 1) / 2, kSphThreads), kSphThreads, st,
                    g->pos4, g->cell_start, g->sorted_idx, n, G, c, g->vel4, g->aux, density);
    }
    FORGE_LAUNCHED();
    return FORGE_OK;
}

// One force pass over all particles (LIST false) or a zone list (the grid
// covers an upper bound of the list; warps past its end leave at once).
template <int TERMS, int EPI, bool LIST>
void launch_force_k(forge_grid* g, const sph::SphConsts& c, const sph::StepEpi& ep, const sph::ForceOut& o,
                    const sph::ZoneList& zl, cudaStream_t st) {
    const sph::Geom G = geom_of(g, c.h);
    const uint32_t n = (uint32_t)g->n;
    switch (walk_of(g)) {
        case FORGE_WALK_GROUP4:
            launch_pdl(sph::force_group_kernel<TERMS, EPI, 4, LIST>, group_blocks<4>(n), kSphThreads, st,
                g->pos4, g->vel4, g->aux, g->cell_start, g->sorted_idx, n, G, c, ep, o, zl);
            break;
        case FORGE_WALK_GROUP8:
            launch_pdl(sph::force_group_kernel<TERMS, EPI, 8, LIST>, group_blocks<8>(n), kSphThreads, st,
                g->pos4, g->vel4, g->aux, g->cell_start, g->sorted_idx, n, G, c, ep, o, zl);
            break;
        case FORGE_WALK_GROUP16:
            launch_pdl(sph::force_group_kernel<TERMS, EPI, 16, LIST>, group_blocks<16>(n), kSphThreads, st,
                g->pos4, g->vel4, g->aux, g->cell_start, g->sorted_idx, n, G, c, ep, o, zl);
            break;
        case FORGE_WALK_ROWS:
            launch_pdl(sph::force_rows_kernel<TERMS, EPI, LIST>, rows_blocks(n), sph::kRowsThreads, st,
                g->pos4, g->vel4, g->aux, g->cell_start, g->sorted_idx, n, G, c, ep, o, zl);
            break;
        default:
            if ((double)n / (double)cells_w(g) < kPairMaxOccupancy)
                launch_pdl(sph::force_kernel<TERMS, EPI, LIST>, grid_blocks((n + 1) / 2, kSphThreads), kSphThreads, st,
                    g->pos4, g->vel4, g->aux, g->cell_start, g->sorted_idx, n, G, c, ep, o, zl);
            else
                launch_pdl(sph::force_single_kernel<TERMS, EPI, LIST>, grid_blocks(n, kSphThreads), kSphThreads, st,
                    g->pos4, g->vel4, g->aux, g->cell_start, g->sorted_idx, n, G, c, ep, o, zl);
    }
}

template <int TERMS, int EPI>
void launch_force_t(forge_grid* g, const sph::SphConsts& c, const sph::StepEpi& ep, const sph::ForceOut& o,
                    cudaStream_t st) {
    launch_force_k<TERMS, EPI, false>(g, c, ep, o, {}, st);
}

// One zone of a zoned force step: the same kernels over a zone list; short-
// lived blocks leave room for concurrent work (the other zone, the exchange
// kernels, NCCL).
int launch_force_zone(forge_grid* g, const sph::SphConsts& c, const sph::StepEpi& ep, const sph::ForceOut& o,
                      uint32_t list, cudaStream_t st) {
    const sph::ZoneList zl{g->zone_idx, g->zone_counts, list};
    launch_force_k<3, 1, true>(g, c, ep, o, zl, st);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

// First zoned pass on a grid: zone lists and their event.
int zone_setup(forge_grid* g) {
    if (g->zone_idx) return FORGE_OK;
    const uint64_t rows = (uint64_t)g->geom.ny * g->geom.nz;
    const uint64_t tiles = (rows + sph::kZoneRows - 1) / sph::kZoneRows;
    FORGE_CUDA(dalloc(&g->zone_idx, std::max<uint64_t>(g->max_n, 1)));
    FORGE_CUDA(dalloc(&g->zone_tiles, std::max<uint64_t>(tiles, 1) * slab::kLists));
    FORGE_CUDA(dalloc(&g->zone_counts, slab::kLists));
    FORGE_CUDA(cudaEventCreateWithFlags(&g->ev_zone, cudaEventDisableTiming));
    return FORGE_OK;
}

// Splits the built grid's particles into the boundary and interior zone
// lists by x-slice: interior = slices whose x-extent lies inside
// [inner_lo, inner_hi). Ghosts fall in the boundary list (skipped there).
int zone_classify(forge_grid* g, float inner_lo, float inner_hi, cudaStream_t st) {
    const grid::GridGeom& G = g->geom;
    const uint32_t row_len = (uint32_t)G.nxw << g->sub_bits;
    const double w = (double)G.cs / (double)(1u << g->sub_bits);  // slice width
    auto edge = [&](float x, bool up) -> uint32_t {
        if (std::isinf(x)) return x < 0 ? 0u : row_len;
        if (!(x == x)) return 0u;
        const double f = ((double)x - (double)G.ox) / w - (double)((uint64_t)G.cx0 << g->sub_bits);
        const double e = up ? std::ceil(f) : std::floor(f);
        return (uint32_t)std::min<double>(std::max<double>(e, 0.0), (double)row_len);
    };
    // interior slices [k_lo, k_hi): lower edge >= inner_lo, upper edge <=
    // inner_hi (a particle hashed into a slice by a rounded divide may sit a
    // few ulps outside it; the guard check of the interior pass sees that)
    const uint32_t k_lo = edge(inner_lo, true);
    const uint32_t k_hi = std::max(k_lo, edge(inner_hi, false));
    const sph::ZoneRows z{g->cell_start, (uint32_t)G.ny * (uint32_t)G.nz, row_len, k_lo, k_hi};
    const uint32_t tiles = grid_blocks(z.rows, sph::kZoneRows);
    launch_pdl(sph::zone_rows_count_kernel, tiles, sph::kZoneRows, st, z, g->zone_tiles);
    slab::classify_scan_kernel<<<1, 1024, 0, st>>>(g->zone_tiles, tiles, g->zone_counts);
    launch_pdl(sph::zone_rows_write_kernel, tiles, sph::kZoneRows, st, z, g->zone_tiles, g->zone_counts, g->zone_idx);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

}  // namespace

extern "C" int forge_grid_build(forge_grid* g, const float* px, const float* py, const float* pz, uint64_t n,
                                uint32_t* cell_idx, uint32_t* sorted_idx, uint32_t* cell_start, void* stream) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_build: grid is NULL");
    FORGE_DEVICE_SCOPE(g->device);
    cudaStream_t st = as_stream(stream);
    int rc = grid_build_impl(g, px, py, pz, 1, n, cell_idx, true, nullptr, nullptr, nullptr, st);
    if (rc != FORGE_OK) return rc;
    return grid_export(g, sorted_idx, cell_start, st);
}

extern "C" int forge_grid_build_aos(forge_grid* g, const float* xyz, uint64_t n, uint32_t* cell_idx,
                                    uint32_t* sorted_idx, uint32_t* cell_start, void* stream) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_build_aos: grid is NULL");
    if (n && !xyz) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_build_aos: xyz is NULL");
    FORGE_DEVICE_SCOPE(g->device);
    cudaStream_t st = as_stream(stream);
    int rc = grid_build_impl(g, xyz, xyz ? xyz + 1 : nullptr, xyz ? xyz + 2 : nullptr, 3, n, cell_idx, true, nullptr,
                             nullptr, nullptr, st);
    if (rc != FORGE_OK) return rc;
    return grid_export(g, sorted_idx, cell_start, st);
}

extern "C" int forge_grid_query(forge_grid* g, const float* px, const float* py, const float* pz, const float* qx,
                                const float* qy, const float* qz, uint64_t nq, float radius, uint32_t* counts,
                                uint32_t* offsets, uint32_t* hits, uint64_t max_hits, void* stream) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_query: grid is NULL");
    if (!g->built || g->sub_bits != 0)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_query: build the grid with forge_grid_build first");
    if (g->geom.cx0 != 0 || g->geom.nxw != g->geom.nx)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_query: the grid has an x-window; queries need the whole grid");
    if (nq > g->max_n)
        return set_error(FORGE_ERR_CAPACITY, "forge_grid_query: nq=%llu exceeds max_n=%llu",
                         (unsigned long long)nq, (unsigned long long)g->max_n);
    if (!counts) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_query: counts is NULL");
    if (nq && (!qx || !qy || !qz)) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_query: NULL queries");
    if (g->n && (!px || !py || !pz)) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_query: NULL positions");
    FORGE_DEVICE_SCOPE(g->device);
    cudaStream_t st = as_stream(stream);
    uint32_t* offs = offsets ? offsets : g->q_offsets;
    if (nq == 0) {
        FORGE_CUDA(cudaMemsetAsync(offs, 0, 4, st));
        return FORGE_OK;
    }
    const float r2 = radius * radius;
    uint32_t* err = g->scratch.meta + kMetaErr;
    const uint32_t nb = grid_blocks(nq, 128);
    grid::query_kernel<false><<<nb, 128, 0, st>>>(px, py, pz, qx, qy, qz, (uint32_t)nq, r2, g->geom, g->cell_start,
                                                  g->sorted_idx, counts, nullptr, nullptr, 0, err);
    FORGE_LAUNCHED();
    if (!offsets && !hits) return FORGE_OK;
    const uint32_t tiles = grid_blocks(nq, grid::kScanTile);
    grid::scan_tile_sums_kernel<<<tiles, grid::kScanThreads, 0, st>>>(counts, (uint32_t)nq, g->scan_sums);
    grid::scan_sums_kernel<<<1, 1024, 0, st>>>(g->scan_sums, tiles);
    grid::scan_apply_kernel<<<tiles, grid::kScanThreads, 0, st>>>(counts, (uint32_t)nq, g->scan_sums, offs);
    FORGE_LAUNCHED();
    if (hits) {
        grid::query_kernel<true><<<nb, 128, 0, st>>>(px, py, pz, qx, qy, qz, (uint32_t)nq, r2, g->geom,
                                                     g->cell_start, g->sorted_idx, counts, offs, hits, max_hits, err);
        FORGE_LAUNCHED();
    }
    return FORGE_OK;
}

extern "C" int forge_grid_check(forge_grid* g, void* stream) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_check: grid is NULL");
    FORGE_DEVICE_SCOPE(g->device);
    return check_status_word(g->scratch.meta + kMetaErr, as_stream(stream), "grid");
}

// ===========================================================================
// SPH
// ===========================================================================
extern "C" int forge_sph_density(forge_grid* g, const forge_sph_params* p, const float* px, const float* py,
                                 const float* pz, uint64_t n, float* density, void* stream) {
    if (!g || !p) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_density: NULL grid or params");
    if (n && !density) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_density: density is NULL");
    FORGE_DEVICE_SCOPE(g->device);
    cudaStream_t st = as_stream(stream);
    int rc = grid_build_impl(g, px, py, pz, 1, n, nullptr, true, nullptr, nullptr, nullptr, st, kSphSubBits);
    if (rc != FORGE_OK) return rc;
    return launch_density(g, p, density, st);
}

extern "C" int forge_sph_force(forge_grid* g, const forge_sph_params* p, uint32_t terms, const float* px,
                               const float* py, const float* pz, const float* vx_in, const float* vy_in,
                               const float* vz_in, const float* density, uint64_t n, float dt, float* vx_out,
                               float* vy_out, float* vz_out, float* ax_out, float* ay_out, float* az_out,
                               void* stream) {
    (void)px;
    (void)py;
    (void)pz;
    if (!g || !p) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_force: NULL grid or params");
    if (terms == 0 || terms > 3) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_force: terms must be 1, 2 or 3");
    if (!g->built || g->n != n)
        return set_error(FORGE_ERR_INVALID_ARG,
                         "forge_sph_force: the grid was not built for these %llu particles (last build: %llu)",
                         (unsigned long long)n, (unsigned long long)g->n);
    if (n == 0) return FORGE_OK;
    if (!vx_in || !vy_in || !vz_in || !density || !vx_out || !vy_out || !vz_out)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_force: NULL velocity/density pointer");
    if ((ax_out == nullptr) != (ay_out == nullptr) || (ax_out == nullptr) != (az_out == nullptr))
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_force: pass all three accel arrays or none");
    FORGE_DEVICE_SCOPE(g->device);
    cudaStream_t st = as_stream(stream);
    const sph::SphConsts c = make_consts(p);
    launch_pdl(sph::gather_vel_rho_kernel, grid_blocks(n, 256), 256, st, g->sorted_idx, (uint32_t)n, vx_in, vy_in,
                                                                    vz_in, density, c, g->vel4, g->aux, g->pos4);
    FORGE_LAUNCHED();
    sph::StepEpi ep{};
    ep.dt = dt;
    sph::ForceOut o{vx_out, vy_out, vz_out, ax_out, ay_out, az_out, nullptr, nullptr, nullptr, 0xffffffffu};
    if (terms == 3) launch_force_t<3, 0>(g, c, ep, o, st);
    else if (terms == 1) launch_force_t<1, 0>(g, c, ep, o, st);
    else launch_force_t<2, 0>(g, c, ep, o, st);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

namespace {
sph::StepEpi epi_of(const forge_step_params* sp) {
    sph::StepEpi ep{};
    ep.dt = sp->dt;
    ep.gx = sp->gravity[0];
    ep.gy = sp->gravity[1];
    ep.gz = sp->gravity[2];
    for (int a = 0; a < 3; ++a) {
        ep.bmin[a] = sp->box_min[a];
        ep.bmax[a] = sp->box_max[a];
    }
    ep.restitution = sp->restitution;
    ep.flags = sp->flags;
    ep.n_ops = sp->n_ops;
    for (uint32_t k = 0; k < ep.n_ops; ++k) {
        ep.ops[k].kind = sp->ops[k].kind;
        for (int q = 0; q < 7; ++q) ep.ops[k].p[q] = sp->ops[k].p[q];
    }
    return ep;
}
}  // namespace

namespace {

int force_step_impl(const char* fn, forge_grid* g, const forge_sph_params* p, const forge_step_params* sp, float* px,
                    float* py, float* pz, float* vx, float* vy, float* vz, const float* density, uint64_t n,
                    uint64_t n_update, const forge_force_zone* zone, cudaStream_t st) {
    if (!g || !p || !sp) return set_error(FORGE_ERR_INVALID_ARG, "%s: NULL grid or params", fn);
    if (sp->n_ops > FORGE_STEP_MAX_OPS) return set_error(FORGE_ERR_INVALID_ARG, "%s: n_ops > 8", fn);
    if (!g->built || g->n != n)
        return set_error(FORGE_ERR_INVALID_ARG, "%s: the grid was not built for these %llu particles (last build: %llu)",
                         fn, (unsigned long long)n, (unsigned long long)g->n);
    if (n_update > n) return set_error(FORGE_ERR_INVALID_ARG, "%s: n_update > n", fn);
    const uint32_t mode = zone ? zone->mode : 0u;
    if (mode > FORGE_ZONE_PREPARE) return set_error(FORGE_ERR_INVALID_ARG, "%s: bad zone mode %u", fn, mode);
    if (mode == FORGE_ZONE_INTERIOR && !g->force_gathered)
        return set_error(FORGE_ERR_INVALID_ARG,
                         "%s: an interior pass must follow a prepare or boundary pass of the same build", fn);
    if (n == 0) return FORGE_OK;
    if (!px || !py || !pz || !vx || !vy || !vz || !density)
        return set_error(FORGE_ERR_INVALID_ARG, "%s: NULL array", fn);
    FORGE_DEVICE_SCOPE(g->device);
    const sph::SphConsts c = make_consts(p);
    sph::ForceOut o{vx, vy, vz, nullptr, nullptr, nullptr, px, py, pz, (uint32_t)n_update};
    if (!mode) {
        launch_pdl(sph::gather_vel_rho_kernel, grid_blocks(n, 256), 256, st, g->sorted_idx, (uint32_t)n, vx, vy, vz,
                                                                        density, c, g->vel4, g->aux, g->pos4);
        g->force_gathered = false;
        launch_force_t<3, 1>(g, c, epi_of(sp), o, st);
        FORGE_LAUNCHED();
        return FORGE_OK;
    }
    int rc;
    const bool prepared = g->force_gathered;
    if (mode == FORGE_ZONE_PREPARE || (mode == FORGE_ZONE_BOUNDARY && !prepared)) {
        // cell-ordered velocities + density, both zone lists: what the two
        // zones' kernels read (the boundary particles' columns are updated
        // in place afterwards, so this is done once per build)
        launch_pdl(sph::gather_vel_rho_kernel, grid_blocks(n, 256), 256, st, g->sorted_idx, (uint32_t)n, vx, vy, vz,
                                                                        density, c, g->vel4, g->aux, g->pos4);
        FORGE_LAUNCHED();
        if ((rc = zone_setup(g)) != FORGE_OK) return rc;
        if ((rc = zone_classify(g, zone->inner_lo, zone->inner_hi, st)) != FORGE_OK) return rc;
        FORGE_CUDA(cudaEventRecord(g->ev_zone, st));
        g->force_gathered = true;
        if (mode == FORGE_ZONE_PREPARE) return FORGE_OK;
    } else {
        // the zone passes need the gather and the lists, not each other: on
        // two streams their kernels run concurrently
        FORGE_CUDA(cudaStreamWaitEvent(st, g->ev_zone, 0));
        if (mode == FORGE_ZONE_BOUNDARY && n_update < n) {
            // ghost densities may have arrived since the prepare pass
            launch_pdl(sph::ghost_rho_kernel, grid_blocks(n, 256), 256, st, g->sorted_idx, (uint32_t)n,
                                                                       (uint32_t)n_update, density, c, g->vel4,
                                                                       g->aux, g->pos4);
            FORGE_LAUNCHED();
        }
    }
    o.zone = mode;
    o.glo = zone->guard_lo;
    o.ghi = zone->guard_hi;
    o.status = g->scratch.meta + kMetaErr;
    return launch_force_zone(g, c, epi_of(sp), o, mode, st);
}

}  // namespace

extern "C" int forge_sph_force_step(forge_grid* g, const forge_sph_params* p, const forge_step_params* sp,
                                    float* px, float* py, float* pz, float* vx, float* vy, float* vz,
                                    const float* density, uint64_t n, uint64_t n_update, void* stream) {
    return force_step_impl("forge_sph_force_step", g, p, sp, px, py, pz, vx, vy, vz, density, n, n_update, nullptr,
                           as_stream(stream));
}

extern "C" int forge_sph_force_step_zone(forge_grid* g, const forge_sph_params* p, const forge_step_params* sp,
                                         float* px, float* py, float* pz, float* vx, float* vy, float* vz,
                                         const float* density, uint64_t n, uint64_t n_update,
                                         const forge_force_zone* zone, void* stream) {
    if (!zone) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_force_step_zone: zone is NULL");
    return force_step_impl("forge_sph_force_step_zone", g, p, sp, px, py, pz, vx, vy, vz, density, n, n_update, zone,
                           as_stream(stream));
}

extern "C" int forge_apply_ops(const forge_step_params* sp, float* px, float* py, float* pz, float* vx, float* vy,
                               float* vz, uint64_t n, int device, void* stream) {
    if (!sp) return set_error(FORGE_ERR_INVALID_ARG, "forge_apply_ops: params are NULL");
    if (sp->n_ops > FORGE_STEP_MAX_OPS) return set_error(FORGE_ERR_INVALID_ARG, "forge_apply_ops: n_ops > 8");
    if (n >= 0xffffffffull) return set_error(FORGE_ERR_INVALID_ARG, "forge_apply_ops: n too large");
    if (n == 0 || sp->n_ops == 0) return FORGE_OK;
    if (!px || !py || !pz || !vx || !vy || !vz)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_apply_ops: NULL position/velocity pointer");
    FORGE_DEVICE_SCOPE(device);
    launch_pdl(sph::apply_ops_kernel, grid_blocks(n, 256), 256, as_stream(stream), epi_of(sp), px, py, pz, vx, vy, vz,
                                                                            (uint32_t)n);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

extern "C" int forge_sph_step(forge_grid* g, const forge_sph_params* p, const forge_step_params* sp, float* px,
                              float* py, float* pz, float* vx, float* vy, float* vz, float* density, uint64_t n,
                              void* stream) {
    if (!g || !p || !sp) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_step: NULL grid or params");
    if (sp->n_ops > FORGE_STEP_MAX_OPS) return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_step: n_ops > 8");
    if (n && (!px || !py || !pz || !vx || !vy || !vz))
        return set_error(FORGE_ERR_INVALID_ARG, "forge_sph_step: NULL position/velocity pointer");
    FORGE_DEVICE_SCOPE(g->device);
    cudaStream_t st = as_stream(stream);
    prof_mark(g, 0, st);
    int rc = grid_build_impl(g, px, py, pz, 1, n, nullptr, true, vx, vy, vz, st, kSphSubBits);
    if (rc != FORGE_OK) return rc;
    if (n == 0) return FORGE_OK;
    rc = launch_density(g, p, density, st);
    if (rc != FORGE_OK) return rc;
    prof_mark(g, 3, st);
    const sph::StepEpi ep = epi_of(sp);
    sph::ForceOut o{vx, vy, vz, nullptr, nullptr, nullptr, px, py, pz, 0xffffffffu};
    launch_force_t<3, 1>(g, make_consts(p), ep, o, st);
    FORGE_LAUNCHED();
    prof_mark(g, 4, st);
    prof_step_done(g);
    return FORGE_OK;
}

extern "C" int forge_grid_set_walk(forge_grid* g, int walk) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_set_walk: grid is NULL");
    if (walk < FORGE_WALK_AUTO || walk > FORGE_WALK_TILE)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_set_walk: unknown walk %d", walk);
    g->walk = walk;
    return FORGE_OK;
}

extern "C" int forge_grid_set_x_window(forge_grid* g, uint32_t cx0, uint32_t nxw) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_set_x_window: grid is NULL");
    if (nxw == 0 || (uint64_t)cx0 + nxw > (uint64_t)g->geom.nx)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_set_x_window: cells [%u, %u) outside the grid's %d",
                         cx0, cx0 + nxw, g->geom.nx);
    g->geom.cx0 = (int)cx0;
    g->geom.nxw = (int)nxw;
    g->built = false;  // the table of the last build no longer matches
    return FORGE_OK;
}

extern "C" int forge_grid_profile_enable(forge_grid* g, uint32_t max_steps) {
    if (!g) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_profile_enable: grid is NULL");
    FORGE_DEVICE_SCOPE(g->device);
    prof_free(g);
    if (max_steps == 0) return FORGE_OK;
    g->prof_events.resize((size_t)max_steps * 5);
    for (auto& e : g->prof_events) FORGE_CUDA(cudaEventCreate(&e));
    g->prof_cap = max_steps;
    return FORGE_OK;
}

extern "C" int forge_grid_profile_read(forge_grid* g, float* out, uint32_t cap_steps, uint32_t* steps) {
    if (!g || !steps) return set_error(FORGE_ERR_INVALID_ARG, "forge_grid_profile_read: NULL argument");
    *steps = 0;
    if (!g->prof_cap) return FORGE_OK;
    FORGE_DEVICE_SCOPE(g->device);
    const uint32_t cnt = std::min(g->prof_count, cap_steps);
    const uint32_t first = (g->prof_next + g->prof_cap - g->prof_count) % g->prof_cap;
    for (uint32_t i = 0; i < cnt; ++i) {
        const size_t b = (size_t)((first + i) % g->prof_cap) * 5;
        FORGE_CUDA(cudaEventSynchronize(g->prof_events[b + 4]));
        for (int k = 0; k < 4; ++k)
            FORGE_CUDA(cudaEventElapsedTime(&out[i * 4 + k], g->prof_events[b + k], g->prof_events[b + k + 1]));
    }
    *steps = cnt;
    g->prof_count = 0;
    return FORGE_OK;
}

// ===========================================================================
// Slab-exchange helpers
// ===========================================================================
struct forge_slab {
    int device = 0;
    int sms = 148;
    uint64_t max_n = 0;
    uint32_t* tile_counts = nullptr;
    uint32_t* hist_acc = nullptr;  // 2 x kHistMaxBins words: 64-bit fixed-point bins of forge_slab_x_hist
};

extern "C" int forge_slab_create(uint64_t max_n, int device, forge_slab** out) {
    if (!out) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_create: out is NULL");
    *out = nullptr;
    if (max_n >= 0xffffffffull) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_create: max_n must be < 2^32-1");
    FORGE_DEVICE_SCOPE(device);
    forge_slab* h = new forge_slab;
    h->device = device;
    h->max_n = max_n;
    h->sms = num_sms(device);
    const size_t tiles = (max_n + slab::kTile - 1) / slab::kTile + 1;
    if (dalloc(&h->tile_counts, tiles * slab::kLists) != cudaSuccess ||
        dalloc(&h->hist_acc, 2 * (size_t)slab::kHistMaxBins) != cudaSuccess) {
        cudaFree(h->tile_counts);
        delete h;
        return set_error(FORGE_ERR_CUDA, "forge_slab_create: cudaMalloc failed");
    }
    *out = h;
    return FORGE_OK;
}

extern "C" void forge_slab_destroy(forge_slab* h) {
    if (!h) return;
    DeviceScope scope(h->device);
    cudaFree(h->tile_counts);
    cudaFree(h->hist_acc);
    delete h;
}

extern "C" int forge_slab_classify(forge_slab* h, const float* x, uint64_t n, float lo, float hi, float reach,
                                   uint32_t flags, uint32_t* idx_out, uint32_t* counts, void* stream) {
    if (!h || !counts) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_classify: NULL handle or counts");
    if (n > h->max_n)
        return set_error(FORGE_ERR_CAPACITY, "forge_slab_classify: n=%llu exceeds max_n=%llu", (unsigned long long)n,
                         (unsigned long long)h->max_n);
    if (n && (!x || !idx_out)) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_classify: NULL array");
    FORGE_DEVICE_SCOPE(h->device);
    cudaStream_t st = as_stream(stream);
    if (n == 0) {
        FORGE_CUDA(cudaMemsetAsync(counts, 0, slab::kLists * sizeof(uint32_t), st));
        return FORGE_OK;
    }
    const slab::ClassifyArgs a{lo, hi, reach, flags};
    const uint32_t tiles = grid_blocks(n, slab::kTile);
    slab::classify_count_kernel<<<tiles, slab::kThreads, 0, st>>>(slab::XMember{x, a}, (uint32_t)n,
                                                                  nullptr, h->tile_counts);
    slab::classify_scan_kernel<<<1, 1024, 0, st>>>(h->tile_counts, tiles, counts);
    slab::classify_write_kernel<<<tiles, slab::kThreads, 0, st>>>(slab::XMember{x, a}, (uint32_t)n,
                                                                  nullptr, h->tile_counts,
                                                                  counts, idx_out);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

extern "C" int forge_slab_x_hist(forge_slab* h, const float* x, const float* w, uint64_t n, float lo, float hi,
                                 uint32_t bins, double* out, void* stream) {
    if (!h || !out || (n && !x)) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_x_hist: NULL argument");
    if (bins == 0 || bins > slab::kHistMaxBins || !(lo < hi) || n >= 0xffffffffull)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_x_hist: bins in [1, %u], lo < hi", slab::kHistMaxBins);
    FORGE_DEVICE_SCOPE(h->device);
    cudaStream_t st = as_stream(stream);
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(h->hist_acc);
    FORGE_CUDA(cudaMemsetAsync(acc, 0, bins * sizeof(unsigned long long), st));
    if (n) {
        const uint32_t blocks = std::min(grid_blocks(n, 256), (uint32_t)h->sms * 2u);
        slab::x_hist_kernel<<<blocks, 256, 0, st>>>(x, w, (uint32_t)n, (double)lo,
                                                    (double)bins / ((double)hi - (double)lo), bins, acc);
    }
    slab::x_hist_finish_kernel<<<grid_blocks(bins, 256), 256, 0, st>>>(acc, bins, out);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

extern "C" int forge_slab_compact(float* cols, uint64_t ld, uint32_t rows, uint64_t n, const uint32_t* gone,
                                  uint64_t k, void* stream) {
    if (k == 0) return FORGE_OK;
    if (!cols || !gone || k > n || n >= 0xffffffffull)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_compact: bad arguments");
    slab::compact_kernel<<<1, 1024, 0, as_stream(stream)>>>(cols, ld, rows, (uint32_t)n, gone, (uint32_t)k, nullptr);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

#include "field_io.cuh"
#include "slab_comm.cuh"
