// Host side of the sharded SPH step's neighbour exchange, over the library's
// own NCCL communicator (NCCL 2.x, loaded at run time with dlopen so that
// single-GPU users need no NCCL). Included at the end of forge_sph.cu.
//
// Per step and rank (x-slab [lo, hi), one neighbour on each side at most):
//   forge_slab_exchange  (round 1, after the force pass of the previous step)
//     classify migrants (x outside the slab)   -> pack their records
//     remove them from the owned columns        (compact, tail into holes)
//     classify halo rows (x within reach)      -> pack their records
//     send [migrants | halo] to each neighbour, counts first, then payload
//     append arrivals as owned, then ghosts: halo from L, halo from R,
//     our migrants to L, our migrants to R (they sit just across the face)
//   forge_slab_exchange_rho (round 2, after density; sizes known, no sync)
//     send rho of [halo sent to X, arrivals from X] to X; X's values land in
//     [halo from X, our migrants to X].
// Round 1 split for overlap with the interior force pass:
//   forge_slab_exchange_begin (after the boundary force, on the caller's
//     side stream) one-pass selection of migrants and in-slab halo rows from
//     the uncompacted columns, records packed as listed, counts exchanged
//   forge_slab_exchange_end   (host waits for the counts) payload on the side
//     stream; on the main stream, after it: compaction, remap of the halo
//     lists to the compacted columns, arrivals and ghosts in one launch.
// One host wait per round 1 (after the count exchange: NCCL needs the payload
// sizes on the host); every list size before it stays on the device. Host
// waits have a deadline: past it, or on an asynchronous NCCL error, the
// communicator is aborted and every later call fails (failure detection).
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>

namespace {

struct NcclApi {
    bool loaded = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

int nccl_load() {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.loaded) return FORGE_OK;
    // Prefer a libnccl already in the process (e.g. the one torch loaded).
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return set_error(FORGE_ERR_NCCL, "libnccl.so.2 not found: %s", dlerror());
#define FORGE_NCCL_SYM(name)                                                                        \
    *reinterpret_cast<void**>(&g_nccl.name) = dlsym(h, "nccl" #name);                               \
    if (!g_nccl.name) return set_error(FORGE_ERR_NCCL, "libnccl.so.2 lacks nccl" #name);
    FORGE_NCCL_SYM(GetUniqueId)
    FORGE_NCCL_SYM(CommInitRank)
    FORGE_NCCL_SYM(CommDestroy)
    FORGE_NCCL_SYM(GroupStart)
    FORGE_NCCL_SYM(GroupEnd)
    FORGE_NCCL_SYM(Send)
    FORGE_NCCL_SYM(Recv)
    FORGE_NCCL_SYM(GetErrorString)
    FORGE_NCCL_SYM(CommAbort)
    FORGE_NCCL_SYM(CommGetAsyncError)
#undef FORGE_NCCL_SYM
    g_nccl.loaded = true;
    return FORGE_OK;
}

#define FORGE_NCCL(call)                                                                            \
    do {                                                                                            \
        ncclResult_t r_ = (call);                                                                   \
        if (r_ != ncclSuccess)                                                                      \
            return set_error(FORGE_ERR_NCCL, "%s failed: %s", #call, g_nccl.GetErrorString(r_));    \
    } while (0)

constexpr uint32_t kSlabRows = 7;  // x, y, z, vx, vy, vz, id bits

}  // namespace

struct forge_slab_comm {
    int device = 0, rank = 0, world = 1;
    int sms = 148;
    int left = -1, right = -1;
    uint64_t cap = 0;
    float lo = 0.f, hi = 0.f, reach = 0.f;
    ncclComm_t comm = nullptr;
    forge_slab* sel = nullptr;
    uint32_t* idx = nullptr;       // migrant classification [A | L | R], 2 cap
    uint32_t* idx_h = nullptr;     // halo classification [L | R], 2 cap
    uint32_t* counts = nullptr;    // 6 device words: migrant sizes A, L, R; halo sizes 0, L, R
    uint32_t* hcounts = nullptr;   // 3 pinned host words
    uint32_t* halo_l = nullptr;    // halo lists of the last round (cap each)
    uint32_t* halo_r = nullptr;
    float* send_l = nullptr;       // records, cap x 7 each
    float* send_r = nullptr;
    float* recv_l = nullptr;
    float* recv_r = nullptr;
    float* rho_send_l = nullptr;   // cap each
    float* rho_send_r = nullptr;
    float* rho_recv_l = nullptr;
    float* rho_recv_r = nullptr;
    uint64_t* dcount = nullptr;    // [send l(2) | send r(2) | recv l(2) | recv r(2) | migrants A]
    uint64_t* hcount = nullptr;    // pinned mirror
    // bookkeeping of the last round 1
    uint32_t n_hl = 0, n_hr = 0;          // halo rows sent left / right
    uint32_t n_ml = 0, n_mr = 0;          // migrants sent left / right
    uint32_t arr_l = 0, n_arr_l = 0;      // arrivals from left: columns [arr_l, arr_l + n_arr_l)
    uint32_t arr_r = 0, n_arr_r = 0;
    uint32_t g_hl = 0, n_ghl = 0;         // ghost blocks: halo from left
    uint32_t g_hr = 0, n_ghr = 0;         // halo from right
    uint32_t g_ml = 0, g_mr = 0;          // our migrants to left / right
    bool have_round = false;
    // split round 1 (forge_slab_exchange_begin / _end)
    uint32_t* xtiles = nullptr;          // tile counts of the one-pass selection
    cudaStream_t pend_stream = nullptr;  // begin's stream
    cudaEvent_t ev_counts = nullptr, ev_payload = nullptr;
    bool pending = false;
    uint64_t pend_n_own = 0;
    // failure detection: host waits give up after `timeout_s`, abort the
    // communicator and fail every later call
    double timeout_s = 60.0;
    cudaEvent_t ev_sync = nullptr;
    bool aborted = false;
};

namespace {

void slab_comm_free(forge_slab_comm* c) {
    DeviceScope scope(c->device);
    if (c->comm) (c->aborted ? g_nccl.CommAbort : g_nccl.CommDestroy)(c->comm);
    forge_slab_destroy(c->sel);
    for (void* p : {(void*)c->idx, (void*)c->idx_h, (void*)c->counts, (void*)c->halo_l, (void*)c->halo_r, (void*)c->send_l,
                    (void*)c->send_r, (void*)c->recv_l, (void*)c->recv_r, (void*)c->rho_send_l,
                    (void*)c->rho_send_r, (void*)c->rho_recv_l, (void*)c->rho_recv_r, (void*)c->dcount, (void*)c->xtiles})
        cudaFree(p);
    cudaFreeHost(c->hcounts);
    cudaFreeHost(c->hcount);
    for (cudaEvent_t e : {c->ev_counts, c->ev_payload, c->ev_sync})
        if (e) cudaEventDestroy(e);
    delete c;
}

// Enqueues a classification of x[0, n - *n_sub) into idx/counts (no sync).
int classify_async(forge_slab_comm* c, const float* x, uint64_t n, const uint32_t* n_sub, uint32_t flags,
                   uint32_t* idx, uint32_t* counts, cudaStream_t st) {
    if (n == 0) {
        FORGE_CUDA(cudaMemsetAsync(counts, 0, 3 * sizeof(uint32_t), st));
        return FORGE_OK;
    }
    const slab::ClassifyArgs a{c->lo, c->hi, c->reach, flags};
    const uint32_t tiles = grid_blocks(n, slab::kTile);
    slab::classify_count_kernel<<<tiles, slab::kThreads, 0, st>>>(slab::XMember{x, a}, (uint32_t)n,
                                                                  n_sub, c->sel->tile_counts);
    slab::classify_scan_kernel<<<1, 1024, 0, st>>>(c->sel->tile_counts, tiles, counts);
    slab::classify_write_kernel<<<tiles, slab::kThreads, 0, st>>>(slab::XMember{x, a}, (uint32_t)n,
                                                                  n_sub, c->sel->tile_counts,
                                                                  counts, idx);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

int pack_list(forge_slab_comm* c, const float* cols, uint64_t ld, const uint32_t* idx, const uint32_t* counts,
              int list, const uint32_t* rec0, float* out, uint32_t* idx_copy, cudaStream_t st) {
    slab::pack_dev_kernel<<<(uint32_t)c->sms * 4, 256, 0, st>>>(cols, ld, kSlabRows, idx, counts, list,
                                                                             rec0, out, idx_copy);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

}  // namespace

extern "C" int forge_nccl_unique_id(uint8_t* out) {
    if (!out) return set_error(FORGE_ERR_INVALID_ARG, "forge_nccl_unique_id: out is NULL");
    int rc = nccl_load();
    if (rc != FORGE_OK) return rc;
    ncclUniqueId id;
    FORGE_NCCL(g_nccl.GetUniqueId(&id));
    memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return FORGE_OK;
}

extern "C" int forge_slab_comm_create(const uint8_t* id, int rank, int world, int device, uint64_t capacity,
                                      float lo, float hi, float reach, forge_slab_comm** out) {
    if (!out || !id) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_comm_create: NULL argument");
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world || capacity == 0 || capacity >= 0x7fffffffull)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_comm_create: bad rank/world/capacity");
    int rc = nccl_load();
    if (rc != FORGE_OK) return rc;
    FORGE_DEVICE_SCOPE(device);
    forge_slab_comm* c = new forge_slab_comm;
    c->device = device;
    c->sms = num_sms(device);
    c->rank = rank;
    c->world = world;
    c->left = rank > 0 ? rank - 1 : -1;
    c->right = rank < world - 1 ? rank + 1 : -1;
    c->cap = capacity;
    c->lo = lo;
    c->hi = hi;
    c->reach = reach;
    const size_t m = capacity;
    bool ok = dalloc(&c->idx, 2 * m) == cudaSuccess && dalloc(&c->idx_h, 2 * m) == cudaSuccess &&
              dalloc(&c->counts, 6) == cudaSuccess &&
              dalloc(&c->halo_l, m) == cudaSuccess && dalloc(&c->halo_r, m) == cudaSuccess &&
              dalloc(&c->send_l, m * kSlabRows) == cudaSuccess && dalloc(&c->send_r, m * kSlabRows) == cudaSuccess &&
              dalloc(&c->recv_l, m * kSlabRows) == cudaSuccess && dalloc(&c->recv_r, m * kSlabRows) == cudaSuccess &&
              dalloc(&c->rho_send_l, m) == cudaSuccess && dalloc(&c->rho_send_r, m) == cudaSuccess &&
              dalloc(&c->rho_recv_l, m) == cudaSuccess && dalloc(&c->rho_recv_r, m) == cudaSuccess &&
              dalloc(&c->dcount, 9) == cudaSuccess &&
              dalloc(&c->xtiles, (m + slab::kTile - 1) / slab::kTile * slab::kXLists) == cudaSuccess &&
              cudaMallocHost(&c->hcounts, 3 * sizeof(uint32_t)) == cudaSuccess &&
              cudaMallocHost(&c->hcount, 9 * sizeof(uint64_t)) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&c->ev_counts, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&c->ev_sync, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&c->ev_payload, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        slab_comm_free(c);
        return set_error(FORGE_ERR_CUDA, "forge_slab_comm_create: allocation failed (capacity %llu)",
                         (unsigned long long)capacity);
    }
    rc = forge_slab_create(capacity, device, &c->sel);
    if (rc != FORGE_OK) {
        slab_comm_free(c);
        return rc;
    }
    ncclUniqueId uid;
    memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclResult_t r = g_nccl.CommInitRank(&c->comm, world, uid, rank);
    if (r != ncclSuccess) {
        c->comm = nullptr;
        slab_comm_free(c);
        return set_error(FORGE_ERR_NCCL, "ncclCommInitRank failed: %s", g_nccl.GetErrorString(r));
    }
    *out = c;
    return FORGE_OK;
}

extern "C" int forge_slab_comm_set_timeout(forge_slab_comm* c, double seconds) {
    if (!c || !(seconds > 0)) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_comm_set_timeout: bad argument");
    c->timeout_s = seconds;
    return FORGE_OK;
}

extern "C" int forge_slab_comm_set_bounds(forge_slab_comm* c, float lo, float hi) {
    if (!c) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_comm_set_bounds: NULL communicator");
    if (c->pending) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_comm_set_bounds: a split round is open");
    if (!(lo < hi)) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_comm_set_bounds: lo >= hi");
    c->lo = lo;
    c->hi = hi;
    return FORGE_OK;
}

extern "C" void forge_slab_comm_destroy(forge_slab_comm* c) {
    if (c) slab_comm_free(c);
}

namespace {

// Host wait for `ev` with failure detection: polls the event and the
// communicator's asynchronous error; past the deadline (a neighbour that
// stopped answering) or on an NCCL error it aborts the communicator, which
// ends this rank's pending NCCL kernels, and fails.
int wait_event(forge_slab_comm* c, cudaEvent_t ev, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t k = 0;; ++k) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return FORGE_OK;
        if (e != cudaErrorNotReady) return set_error(FORGE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
        ncclResult_t ae = ncclSuccess;
        if (g_nccl.CommGetAsyncError(c->comm, &ae) != ncclSuccess || ae != ncclSuccess) {
            c->aborted = true;
            g_nccl.CommAbort(c->comm);
            c->comm = nullptr;
            return set_error(FORGE_ERR_NCCL, "%s: NCCL error %s; communicator aborted", what,
                             g_nccl.GetErrorString(ae));
        }
        const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (waited > c->timeout_s) {
            c->aborted = true;
            g_nccl.CommAbort(c->comm);
            c->comm = nullptr;
            return set_error(FORGE_ERR_TIMEOUT,
                             "%s: no progress for %.1f s (a neighbour stopped answering); communicator aborted", what,
                             waited);
        }
        if (k > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

uint32_t slab_sides(const forge_slab_comm* c) { return (c->left >= 0 ? 1u : 0u) | (c->right >= 0 ? 2u : 0u); }

// Sends the counts message of the two classifications (migrant sizes in
// counts[0..3), halo sizes in counts[3..6)) to the neighbours, receives
// theirs and copies everything to the pinned host mirror, on `st`.
int exchange_counts(forge_slab_comm* c, cudaStream_t st, bool make_msg = true) {
    if (make_msg) {  // else the selection wrote the message (and zeroed the receive words)
        slab::counts_msg_kernel<<<1, 1, 0, st>>>(c->counts, c->counts + 3, c->dcount);
        FORGE_LAUNCHED();
        FORGE_CUDA(cudaMemsetAsync(c->dcount + 4, 0, 4 * sizeof(uint64_t), st));
    }
    FORGE_NCCL(g_nccl.GroupStart());
    if (c->left >= 0) {
        FORGE_NCCL(g_nccl.Send(c->dcount + 0, 2, ncclUint64, c->left, c->comm, st));
        FORGE_NCCL(g_nccl.Recv(c->dcount + 4, 2, ncclUint64, c->left, c->comm, st));
    }
    if (c->right >= 0) {
        FORGE_NCCL(g_nccl.Send(c->dcount + 2, 2, ncclUint64, c->right, c->comm, st));
        FORGE_NCCL(g_nccl.Recv(c->dcount + 6, 2, ncclUint64, c->right, c->comm, st));
    }
    FORGE_NCCL(g_nccl.GroupEnd());
    FORGE_CUDA(cudaMemcpyAsync(c->hcount, c->dcount, 9 * sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
    return FORGE_OK;
}

// Message sizes of the round, from the host mirror of the counts.
struct RoundSizes {
    uint32_t ml, hl, mr, hr;      // sent: migrants / halo rows, left and right
    uint64_t aml, ahl, amr, ahr;  // received
    uint32_t keep;                // owned columns left after the migrants
};

int round_sizes(const forge_slab_comm* c, uint64_t n_own, uint64_t ld, RoundSizes& z) {
    const uint64_t* h = c->hcount;
    z = RoundSizes{(uint32_t)h[0], (uint32_t)h[1], (uint32_t)h[2], (uint32_t)h[3], h[4], h[5], h[6], h[7],
                   (uint32_t)(n_own - h[8])};
    if ((uint64_t)z.ml + z.hl > c->cap || (uint64_t)z.mr + z.hr > c->cap || z.aml + z.ahl > c->cap ||
        z.amr + z.ahr > c->cap)
        return set_error(FORGE_ERR_CAPACITY, "forge_slab_exchange: message exceeds capacity");
    const uint64_t n_new = z.keep + z.aml + z.amr, ng = z.ahl + z.ahr + z.ml + z.mr;
    if (n_new + ng > ld) return set_error(FORGE_ERR_CAPACITY, "forge_slab_exchange: owned + ghosts exceed ld");
    return FORGE_OK;
}

int send_payload(forge_slab_comm* c, const RoundSizes& z, cudaStream_t st) {
    FORGE_NCCL(g_nccl.GroupStart());
    if (c->left >= 0) {
        if (z.ml + z.hl) FORGE_NCCL(g_nccl.Send(c->send_l, (z.ml + z.hl) * kSlabRows, ncclFloat32, c->left, c->comm, st));
        if (z.aml + z.ahl)
            FORGE_NCCL(g_nccl.Recv(c->recv_l, (z.aml + z.ahl) * kSlabRows, ncclFloat32, c->left, c->comm, st));
    }
    if (c->right >= 0) {
        if (z.mr + z.hr)
            FORGE_NCCL(g_nccl.Send(c->send_r, (z.mr + z.hr) * kSlabRows, ncclFloat32, c->right, c->comm, st));
        if (z.amr + z.ahr)
            FORGE_NCCL(g_nccl.Recv(c->recv_r, (z.amr + z.ahr) * kSlabRows, ncclFloat32, c->right, c->comm, st));
    }
    FORGE_NCCL(g_nccl.GroupEnd());
    return FORGE_OK;
}

// Arrivals after the kept owned columns, then the ghosts: halo from left,
// halo from right, our migrants to left, to right. Records the layout for
// the density round.
int place_arrivals(forge_slab_comm* c, float* cols, uint64_t ld, const RoundSizes& z, uint64_t* n_own_out,
                   uint64_t* n_ghost_out, cudaStream_t st) {
    // layout: kept | arrivals from L | from R | ghosts: halo from L | halo
    // from R | our migrants to L | to R
    const uint32_t aml = (uint32_t)z.aml, amr = (uint32_t)z.amr, ahl = (uint32_t)z.ahl, ahr = (uint32_t)z.ahr;
    c->arr_l = z.keep;
    c->n_arr_l = aml;
    c->arr_r = c->arr_l + aml;
    c->n_arr_r = amr;
    c->g_hl = c->arr_r + amr;
    c->n_ghl = ahl;
    c->g_hr = c->g_hl + ahl;
    c->n_ghr = ahr;
    c->g_ml = c->g_hr + ahr;
    c->g_mr = c->g_ml + z.ml;
    const slab::UnpackSet u{{c->recv_l, c->recv_r, c->recv_l + (size_t)aml * kSlabRows,
                             c->recv_r + (size_t)amr * kSlabRows, c->send_l, c->send_r},
                            {aml, amr, ahl, ahr, z.ml, z.mr},
                            {c->arr_l, c->arr_r, c->g_hl, c->g_hr, c->g_ml, c->g_mr}};
    const uint32_t total = aml + amr + ahl + ahr + z.ml + z.mr;
    if (total) {
        slab::unpack_set_kernel<<<std::min(grid_blocks((uint64_t)total * kSlabRows, 256), (uint32_t)c->sms * 8), 256,
                                  0, st>>>(u, total, cols, ld);
        FORGE_LAUNCHED();
    }
    c->n_hl = z.hl;
    c->n_hr = z.hr;
    c->n_ml = z.ml;
    c->n_mr = z.mr;
    c->have_round = true;
    *n_own_out = z.keep + z.aml + z.amr;
    *n_ghost_out = z.ahl + z.ahr + z.ml + z.mr;
    return FORGE_OK;
}

}  // namespace

extern "C" int forge_slab_exchange(forge_slab_comm* c, float* cols, uint64_t ld, uint64_t n_own, int migrate,
                                   uint64_t* n_own_out, uint64_t* n_ghost_out, void* stream) {
    if (!c || !cols || !n_own_out || !n_ghost_out)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange: NULL argument");
    if (n_own > c->cap || ld < c->cap)
        return set_error(FORGE_ERR_CAPACITY, "forge_slab_exchange: n_own or ld does not fit the capacity");
    if (c->pending) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange: a split round is open");
    if (c->aborted) return set_error(FORGE_ERR_NCCL, "slab exchange: communicator aborted by an earlier failure");
    FORGE_DEVICE_SCOPE(c->device);
    cudaStream_t st = as_stream(stream);
    const uint32_t sides = slab_sides(c);
    uint32_t* cm = c->counts;      // migrant list sizes A, L, R
    uint32_t* ch = c->counts + 3;  // halo list sizes 0, L, R
    int rc;
    // All list sizes stay on the device until the count exchange below: one
    // host synchronisation per round.
    // 1. migrants: classify, pack (before the compaction moves columns), remove
    if (migrate) {
        if ((rc = classify_async(c, cols, n_own, nullptr, sides, c->idx, cm, st)) != FORGE_OK) return rc;
        if ((rc = pack_list(c, cols, ld, c->idx, cm, 1, nullptr, c->send_l, nullptr, st)) != FORGE_OK) return rc;
        if ((rc = pack_list(c, cols, ld, c->idx, cm, 2, nullptr, c->send_r, nullptr, st)) != FORGE_OK) return rc;
        if (n_own) {
            slab::compact_kernel<<<1, 1024, 0, st>>>(cols, ld, kSlabRows, (uint32_t)n_own, c->idx, 0u, cm);
            FORGE_LAUNCHED();
        }
    } else {
        FORGE_CUDA(cudaMemsetAsync(cm, 0, 3 * sizeof(uint32_t), st));
    }
    // 2. halo rows of the remaining owned particles, after the migrants
    if ((rc = classify_async(c, cols, n_own, cm, sides | 4u, c->idx_h, ch, st)) != FORGE_OK) return rc;
    if ((rc = pack_list(c, cols, ld, c->idx_h, ch, 1, cm + 1, c->send_l, c->halo_l, st)) != FORGE_OK) return rc;
    if ((rc = pack_list(c, cols, ld, c->idx_h, ch, 2, cm + 2, c->send_r, c->halo_r, st)) != FORGE_OK) return rc;
    // 3. counts: ours to the neighbours, theirs back, everything to the host
    if ((rc = exchange_counts(c, st)) != FORGE_OK) return rc;
    FORGE_CUDA(cudaEventRecord(c->ev_sync, st));
    if ((rc = wait_event(c, c->ev_sync, "forge_slab_exchange")) != FORGE_OK) return rc;
    RoundSizes z;
    if ((rc = round_sizes(c, n_own, ld, z)) != FORGE_OK) return rc;
    // 4. payload, 5. arrivals, then ghosts
    if ((rc = send_payload(c, z, st)) != FORGE_OK) return rc;
    return place_arrivals(c, cols, ld, z, n_own_out, n_ghost_out, st);
}

extern "C" int forge_slab_exchange_begin(forge_slab_comm* c, const float* cols, uint64_t ld, uint64_t n_own,
                                         void* stream) {
    if (!c || !cols) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_begin: NULL argument");
    if (n_own > c->cap || ld < c->cap)
        return set_error(FORGE_ERR_CAPACITY, "forge_slab_exchange_begin: n_own or ld does not fit the capacity");
    if (c->pending) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_begin: a split round is open");
    if (c->aborted) return set_error(FORGE_ERR_NCCL, "slab exchange: communicator aborted by an earlier failure");
    FORGE_DEVICE_SCOPE(c->device);
    cudaStream_t sd = as_stream(stream);
    // Migrants and in-slab halo rows (disjoint) from one read of the
    // uncompacted columns, records packed as they are listed; the halo lists
    // keep the uncompacted indices until _end remaps them.
    if (n_own) {
        const slab::XchgArgs a{cols, ld, (uint32_t)n_own, c->lo, c->hi, c->reach, slab_sides(c)};
        const uint32_t tiles = grid_blocks(n_own, slab::kTile);
        slab::xchg_count_kernel<<<tiles, slab::kThreads, 0, sd>>>(a, c->xtiles);
        slab::xchg_scan_kernel<<<1, 1024, 0, sd>>>(c->xtiles, tiles, c->counts, c->dcount);
        slab::xchg_write_kernel<<<tiles, slab::kThreads, 0, sd>>>(
            a, c->xtiles, c->counts, slab::XchgOut{c->idx, c->halo_l, c->halo_r, c->send_l, c->send_r});
        FORGE_LAUNCHED();
    } else {
        FORGE_CUDA(cudaMemsetAsync(c->counts, 0, 6 * sizeof(uint32_t), sd));
        FORGE_CUDA(cudaMemsetAsync(c->dcount, 0, 9 * sizeof(uint64_t), sd));
    }
    int rc;
    if ((rc = exchange_counts(c, sd, false)) != FORGE_OK) return rc;
    FORGE_CUDA(cudaEventRecord(c->ev_counts, sd));
    c->pend_stream = sd;
    c->pending = true;
    c->pend_n_own = n_own;
    return FORGE_OK;
}

extern "C" int forge_slab_exchange_end(forge_slab_comm* c, float* cols, uint64_t ld, uint64_t* n_own_out,
                                       uint64_t* n_ghost_out, void* stream) {
    if (!c || !cols || !n_own_out || !n_ghost_out)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_end: NULL argument");
    if (!c->pending) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_end: no forge_slab_exchange_begin");
    if (ld < c->cap) return set_error(FORGE_ERR_CAPACITY, "forge_slab_exchange_end: ld does not fit the capacity");
    c->pending = false;
    if (c->aborted) return set_error(FORGE_ERR_NCCL, "slab exchange: communicator aborted by an earlier failure");
    FORGE_DEVICE_SCOPE(c->device);
    cudaStream_t st = as_stream(stream), sd = c->pend_stream;
    const uint64_t n_own = c->pend_n_own;
    int rc;
    // the interior pass keeps running meanwhile
    if ((rc = wait_event(c, c->ev_counts, "forge_slab_exchange_end")) != FORGE_OK) return rc;
    RoundSizes z;
    if ((rc = round_sizes(c, n_own, ld, z)) != FORGE_OK) return rc;
    if ((rc = send_payload(c, z, sd)) != FORGE_OK) return rc;
    FORGE_CUDA(cudaEventRecord(c->ev_payload, sd));
    FORGE_CUDA(cudaStreamWaitEvent(st, c->ev_payload, 0));
    if (n_own - z.keep) {
        uint32_t* cm = c->counts;
        slab::compact_kernel<<<1, 1024, 0, st>>>(cols, ld, kSlabRows, (uint32_t)n_own, c->idx, 0u, cm);
        if (z.hl + z.hr)
            slab::remap_after_compact_kernel<<<std::min(grid_blocks(z.hl + z.hr, 256), (uint32_t)c->sms * 2), 256, 0,
                                               st>>>(c->halo_l, z.hl, c->halo_r, z.hr, (uint32_t)n_own, c->idx, cm);
        FORGE_LAUNCHED();
    }
    return place_arrivals(c, cols, ld, z, n_own_out, n_ghost_out, st);
}

extern "C" int forge_slab_exchange_rho(forge_slab_comm* c, float* rho, void* stream) {
    if (!c || !rho) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_rho: NULL argument");
    if (c->pending) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_rho: a split round is open");
    if (!c->have_round) return set_error(FORGE_ERR_INVALID_ARG, "forge_slab_exchange_rho: no exchange round yet");
    if (c->aborted) return set_error(FORGE_ERR_NCCL, "slab exchange: communicator aborted by an earlier failure");
    FORGE_DEVICE_SCOPE(c->device);
    cudaStream_t st = as_stream(stream);
    const uint32_t kl = c->n_hl + c->n_arr_l, kr = c->n_hr + c->n_arr_r;
    if (kl + kr) {
        const slab::RhoPackSet pk{{c->halo_l, c->halo_r},
                                  {c->n_hl, c->n_hr},
                                  {c->arr_l, c->arr_r},
                                  {c->n_arr_l, c->n_arr_r},
                                  {c->rho_send_l, c->rho_send_r}};
        slab::rho_pack_set_kernel<<<std::min(grid_blocks(kl + kr, 256), (uint32_t)c->sms * 4), 256, 0, st>>>(rho, pk);
        FORGE_LAUNCHED();
    }
    // from X: [X's halo rows to us | our migrants to X]
    const uint32_t il = c->n_ghl + c->n_ml, ir = c->n_ghr + c->n_mr;
    FORGE_NCCL(g_nccl.GroupStart());
    if (c->left >= 0) {
        if (kl) FORGE_NCCL(g_nccl.Send(c->rho_send_l, kl, ncclFloat32, c->left, c->comm, st));
        if (il) FORGE_NCCL(g_nccl.Recv(c->rho_recv_l, il, ncclFloat32, c->left, c->comm, st));
    }
    if (c->right >= 0) {
        if (kr) FORGE_NCCL(g_nccl.Send(c->rho_send_r, kr, ncclFloat32, c->right, c->comm, st));
        if (ir) FORGE_NCCL(g_nccl.Recv(c->rho_recv_r, ir, ncclFloat32, c->right, c->comm, st));
    }
    FORGE_NCCL(g_nccl.GroupEnd());
    if (il + ir) {
        const slab::CopySet cp{{c->rho_recv_l, c->rho_recv_l + c->n_ghl, c->rho_recv_r, c->rho_recv_r + c->n_ghr},
                               {rho + c->g_hl, rho + c->g_ml, rho + c->g_hr, rho + c->g_mr},
                               {c->n_ghl, c->n_ml, c->n_ghr, c->n_mr}};
        slab::copy_set_kernel<<<std::min(grid_blocks(il + ir, 256), (uint32_t)c->sms * 4), 256, 0, st>>>(cp, il + ir);
        FORGE_LAUNCHED();
    }
    return FORGE_OK;
}
