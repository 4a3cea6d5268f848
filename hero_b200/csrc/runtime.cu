// runtime.cu -- error reporting and per-device scratch/flag management.
#include <mutex>
#include <stdarg.h>
#include <stdio.h>
#include <string>
#include <vector>

#include "common.cuh"

namespace nmg {

namespace {
thread_local char g_last_error[1024] = "";

struct Pool {
    void* ptr = nullptr;
    size_t bytes = 0;
};
struct DeviceResources {
    Pool scratch, staging, tickets;
    int* error_flag = nullptr;
};
std::mutex g_mu;
std::vector<DeviceResources> g_dev;

DeviceResources& resources(int device) {
    if ((int)g_dev.size() <= device) g_dev.resize(device + 1);
    return g_dev[device];
}
}  // namespace

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int grow(int device, Pool& p, size_t bytes, void** ptr) {
    if (p.bytes < bytes) {
        int prev = 0;
        NMG_CUDA_TRY(cudaGetDevice(&prev));
        NMG_CUDA_TRY(cudaSetDevice(device));
        if (p.ptr) {
            // The old block may still be read by queued work on any stream.
            NMG_CUDA_TRY(cudaDeviceSynchronize());
            NMG_CUDA_TRY(cudaFree(p.ptr));
            p.ptr = nullptr;
            p.bytes = 0;
        }
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        want = (want + 0xFFFFF) & ~size_t(0xFFFFF);
        NMG_CUDA_TRY(cudaMalloc(&p.ptr, want));
        NMG_CUDA_TRY(cudaMemset(p.ptr, 0, want));
        p.bytes = want;
        NMG_CUDA_TRY(cudaSetDevice(prev));
    }
    *ptr = p.ptr;
    return NMG_OK;
}

int device_scratch(int device, size_t bytes, void** ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    return grow(device, resources(device).scratch, bytes, ptr);
}

int device_tickets(int device, size_t bytes, void** ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    return grow(device, resources(device).tickets, bytes, ptr);
}

int device_staging(int device, size_t bytes, void** ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    return grow(device, resources(device).staging, bytes, ptr);
}

int device_error_flag(int device, int** flag) {
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceResources& r = resources(device);
    if (!r.error_flag) {
        int prev = 0;
        NMG_CUDA_TRY(cudaGetDevice(&prev));
        NMG_CUDA_TRY(cudaSetDevice(device));
        NMG_CUDA_TRY(cudaMalloc(&r.error_flag, sizeof(int)));
        NMG_CUDA_TRY(cudaMemset(r.error_flag, 0, sizeof(int)));
        NMG_CUDA_TRY(cudaSetDevice(prev));
    }
    *flag = r.error_flag;
    return NMG_OK;
}

int check_device_flag(int device, cudaStream_t stream) {
    int* flag = nullptr;
    int st = device_error_flag(device, &flag);
    if (st != NMG_OK) return st;
    int host = 0;
    NMG_CUDA_TRY(cudaMemcpyAsync(&host, flag, sizeof(int), cudaMemcpyDeviceToHost, stream));
    NMG_CUDA_TRY(cudaStreamSynchronize(stream));
    if (host != 0) {
        NMG_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), stream));
        return set_error(NMG_DEVICE_TIMEOUT, "a device-side wait gave up (code %d)", host);
    }
    return NMG_OK;
}

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

}  // namespace nmg

extern "C" const char* nmg_last_error(void) { return nmg::g_last_error; }
extern "C" const char* nmg_version(void) { return "nmg 0.1 sm_100a"; }

extern "C" int nmg_device_status(int device, void* stream) {
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) NMG_CUDA_TRY(cudaSetDevice(device));
    const int st = nmg::check_device_flag(device, (cudaStream_t)stream);
    if (prev != device) cudaSetDevice(prev);
    return st;
}
