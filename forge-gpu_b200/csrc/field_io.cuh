// Field I/O: the host <-> device moves either side of the hot path
// (manifest_runner.rs:192-269 init_fields uploads each SoA column built on
// the host; :83-92 gathers pos_x/y/z back and interleaves them into the
// result's Vec3f positions). Here the AoS <-> SoA conversion runs on the
// GPU (one contiguous copy per direction instead of three, then one
// coalesced pass), and pageable host buffers go through a pinned staging
// buffer owned by the handle, so every copy is a DMA transfer.
// Included by forge_sph.cu.
#pragma once

namespace forge {
namespace io {

// xyz (Vec3f AoS, n x 12 bytes) -> x, y, z columns. Thread per particle;
// the loads are 12-byte strided but every 128-byte line is used in full.
__global__ void __launch_bounds__(256)
    aos_to_soa_kernel(const float* __restrict__ xyz, uint32_t n, float* __restrict__ x, float* __restrict__ y,
                      float* __restrict__ z) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    x[i] = xyz[3 * (size_t)i];
    y[i] = xyz[3 * (size_t)i + 1];
    z[i] = xyz[3 * (size_t)i + 2];
}

__global__ void __launch_bounds__(256)
    soa_to_aos_kernel(const float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ z,
                      uint32_t n, float* __restrict__ xyz) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    xyz[3 * (size_t)i] = x[i];
    xyz[3 * (size_t)i + 1] = y[i];
    xyz[3 * (size_t)i + 2] = z[i];
}

}  // namespace io
}  // namespace forge

struct forge_io {
    int device = 0;
    uint64_t max_n = 0;
    float* pinned = nullptr;   // kIoStageFields x max_n floats (host, page-locked)
    float* dstage = nullptr;   // 3 x max_n floats (device): the AoS image
    cudaEvent_t ev = nullptr;  // last use of the pinned staging
};

namespace {

constexpr uint32_t kIoStageFields = 6;

bool host_pinned(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // pageable memory may report an error on some drivers: clear it
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// The pinned staging may be refilled once its previous copies are done.
int io_reuse(forge_io* io) {
    FORGE_CUDA(cudaEventSynchronize(io->ev));
    return FORGE_OK;
}

}  // namespace

extern "C" int forge_io_create(uint64_t max_n, int device, forge_io** out) {
    if (!out) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_create: out is NULL");
    *out = nullptr;
    if (max_n == 0 || max_n >= 0xffffffffull)
        return set_error(FORGE_ERR_INVALID_ARG, "forge_io_create: max_n must be in [1, 2^32)");
    FORGE_DEVICE_SCOPE(device);
    forge_io* io = new forge_io;
    io->device = device;
    io->max_n = max_n;
    const bool ok = cudaMallocHost(&io->pinned, kIoStageFields * max_n * sizeof(float)) == cudaSuccess &&
                    dalloc(&io->dstage, 3 * max_n) == cudaSuccess &&
                    cudaEventCreateWithFlags(&io->ev, cudaEventDisableTiming) == cudaSuccess &&
                    cudaEventRecord(io->ev, 0) == cudaSuccess;
    if (!ok) {
        forge_io_destroy(io);
        return set_error(FORGE_ERR_CUDA, "forge_io_create: allocation failed (max_n=%llu)", (unsigned long long)max_n);
    }
    *out = io;
    return FORGE_OK;
}

extern "C" void forge_io_destroy(forge_io* io) {
    if (!io) return;
    DeviceScope scope(io->device);
    if (io->ev) {
        cudaEventSynchronize(io->ev);
        cudaEventDestroy(io->ev);
    }
    cudaFreeHost(io->pinned);
    cudaFree(io->dstage);
    delete io;
}

extern "C" int forge_io_upload(forge_io* io, const float* const* host, float* const* dev, uint32_t nfields, uint64_t n,
                               void* stream) {
    if (!io || (nfields && (!host || !dev))) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_upload: NULL argument");
    if (n > io->max_n) return set_error(FORGE_ERR_CAPACITY, "forge_io_upload: n=%llu > max_n", (unsigned long long)n);
    if (nfields > kIoStageFields) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_upload: at most 6 fields");
    if (n == 0 || nfields == 0) return FORGE_OK;
    FORGE_DEVICE_SCOPE(io->device);
    cudaStream_t st = as_stream(stream);
    bool staged = false;
    for (uint32_t f = 0; f < nfields; ++f) {
        if (!host[f] || !dev[f]) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_upload: field %u is NULL", f);
        const float* src = host[f];
        if (!host_pinned(src)) {
            if (!staged) {
                int rc = io_reuse(io);
                if (rc != FORGE_OK) return rc;
                staged = true;
            }
            float* s = io->pinned + (size_t)f * io->max_n;
            memcpy(s, src, n * sizeof(float));
            src = s;
        }
        FORGE_CUDA(cudaMemcpyAsync(dev[f], src, n * sizeof(float), cudaMemcpyHostToDevice, st));
    }
    FORGE_CUDA(cudaEventRecord(io->ev, st));
    return FORGE_OK;
}

extern "C" int forge_io_download(forge_io* io, const float* const* dev, float* const* host, uint32_t nfields,
                                 uint64_t n, void* stream) {
    if (!io || (nfields && (!host || !dev))) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_download: NULL argument");
    if (n > io->max_n) return set_error(FORGE_ERR_CAPACITY, "forge_io_download: n=%llu > max_n", (unsigned long long)n);
    if (nfields > kIoStageFields) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_download: at most 6 fields");
    if (n == 0 || nfields == 0) return FORGE_OK;
    FORGE_DEVICE_SCOPE(io->device);
    cudaStream_t st = as_stream(stream);
    bool any_staged = false;
    for (uint32_t f = 0; f < nfields; ++f) {
        if (!host[f] || !dev[f]) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_download: field %u is NULL", f);
        any_staged |= !host_pinned(host[f]);
    }
    if (!any_staged) {  // all pinned: DMA straight into them, asynchronously
        for (uint32_t f = 0; f < nfields; ++f)
            FORGE_CUDA(cudaMemcpyAsync(host[f], dev[f], n * sizeof(float), cudaMemcpyDeviceToHost, st));
        return FORGE_OK;
    }
    int rc = io_reuse(io);
    if (rc != FORGE_OK) return rc;
    for (uint32_t f = 0; f < nfields; ++f) {
        const bool direct = host_pinned(host[f]);
        float* dst = direct ? host[f] : io->pinned + (size_t)f * io->max_n;
        FORGE_CUDA(cudaMemcpyAsync(dst, dev[f], n * sizeof(float), cudaMemcpyDeviceToHost, st));
    }
    FORGE_CUDA(cudaEventRecord(io->ev, st));
    FORGE_CUDA(cudaEventSynchronize(io->ev));
    if (any_staged)
        for (uint32_t f = 0; f < nfields; ++f)
            if (!host_pinned(host[f])) memcpy(host[f], io->pinned + (size_t)f * io->max_n, n * sizeof(float));
    return FORGE_OK;
}

extern "C" int forge_io_upload_vec3(forge_io* io, const float* xyz, float* x, float* y, float* z, uint64_t n,
                                    void* stream) {
    if (!io) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_upload_vec3: NULL handle");
    if (n > io->max_n) return set_error(FORGE_ERR_CAPACITY, "forge_io_upload_vec3: n=%llu > max_n",
                                        (unsigned long long)n);
    if (n == 0) return FORGE_OK;
    if (!xyz || !x || !y || !z) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_upload_vec3: NULL array");
    FORGE_DEVICE_SCOPE(io->device);
    cudaStream_t st = as_stream(stream);
    const float* src = xyz;
    if (!host_pinned(xyz)) {
        int rc = io_reuse(io);
        if (rc != FORGE_OK) return rc;
        memcpy(io->pinned, xyz, 3 * n * sizeof(float));
        src = io->pinned;
    }
    FORGE_CUDA(cudaMemcpyAsync(io->dstage, src, 3 * n * sizeof(float), cudaMemcpyHostToDevice, st));
    FORGE_CUDA(cudaEventRecord(io->ev, st));
    io::aos_to_soa_kernel<<<grid_blocks(n, 256), 256, 0, st>>>(io->dstage, (uint32_t)n, x, y, z);
    FORGE_LAUNCHED();
    return FORGE_OK;
}

extern "C" int forge_io_download_vec3(forge_io* io, const float* x, const float* y, const float* z, float* xyz,
                                      uint64_t n, void* stream) {
    if (!io) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_download_vec3: NULL handle");
    if (n > io->max_n) return set_error(FORGE_ERR_CAPACITY, "forge_io_download_vec3: n=%llu > max_n",
                                        (unsigned long long)n);
    if (n == 0) return FORGE_OK;
    if (!xyz || !x || !y || !z) return set_error(FORGE_ERR_INVALID_ARG, "forge_io_download_vec3: NULL array");
    FORGE_DEVICE_SCOPE(io->device);
    cudaStream_t st = as_stream(stream);
    int rc = io_reuse(io);
    if (rc != FORGE_OK) return rc;
    io::soa_to_aos_kernel<<<grid_blocks(n, 256), 256, 0, st>>>(x, y, z, (uint32_t)n, io->dstage);
    FORGE_LAUNCHED();
    const bool direct = host_pinned(xyz);
    FORGE_CUDA(cudaMemcpyAsync(direct ? xyz : io->pinned, io->dstage, 3 * n * sizeof(float), cudaMemcpyDeviceToHost,
                               st));
    FORGE_CUDA(cudaEventRecord(io->ev, st));
    FORGE_CUDA(cudaEventSynchronize(io->ev));
    if (!direct) memcpy(xyz, io->pinned, 3 * n * sizeof(float));
    return FORGE_OK;
}
