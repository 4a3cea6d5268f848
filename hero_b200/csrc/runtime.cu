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
    Pool scratch, staging, tickets, weight_act;
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

int weight_act_scratch(int device, size_t bytes, void** ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    return grow(device, resources(device).weight_act, bytes, ptr);
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
    int* lib_flag = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((int)g_dev.size() > device) lib_flag = g_dev[device].error_flag;
    }
    int* words[2] = {lib_flag, noalloc_error_word(device)};
    int raised = 0;
    for (int* w : words) {
        if (!w) continue;  // never created: nothing on this device could have raised it
        int host = 0;
        NMG_CUDA_TRY(cudaMemcpyAsync(&host, w, sizeof(int), cudaMemcpyDeviceToHost, stream));
        NMG_CUDA_TRY(cudaStreamSynchronize(stream));
        if (host != 0) NMG_CUDA_TRY(cudaMemsetAsync(w, 0, sizeof(int), stream));
        raised |= host;
    }
    if (raised) NMG_CUDA_TRY(cudaStreamSynchronize(stream));
    if (raised & dev::kErrWaitTimeout)
        return set_error(NMG_DEVICE_TIMEOUT, "a device-side wait gave up (flags 0x%x)", raised);
    if (raised & dev::kErrF16Overflow)
        return set_error(NMG_VALUE_OVERFLOW,
                         "a V value beyond fp16's range (bf16 magnitude >= 65536) was appended to a bf16 cache, which keeps V as "
                         "fp16; it was stored as +-inf");
    if (raised) return set_error(NMG_RUNTIME_ERROR, "device flag 0x%x", raised);
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

namespace {

// Waits on an mbarrier that nothing arrives on, with a short poll limit: the
// wait gives up, raises the timeout bit of `flag` and the kernel returns,
// exactly as a kernel whose producer stalled would.  No copy is in flight.
__global__ void wait_timeout_selftest_kernel(int* flag) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        dev::mbar_init(&bar, 1);
        dev::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) dev::mbar_wait_n<4096>(&bar, 0, flag);
}

}  // namespace

}  // namespace nmg

extern "C" int nmg_selftest_wait_timeout(int device, int target, void* stream) {
    if (target != 0 && target != 1) return nmg::set_error(NMG_INVALID_ARGUMENT, "nmg_selftest_wait_timeout: target %d", target);
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) NMG_CUDA_TRY(cudaSetDevice(device));
    int* flag = nullptr;
    int st = target == 0 ? nmg::device_error_flag(device, &flag) : nmg::noalloc_error_word_init(device, &flag);
    if (st == NMG_OK) {
        nmg::wait_timeout_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flag);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) st = nmg::set_error(NMG_CUDA_ERROR, "nmg_selftest_wait_timeout: %s", cudaGetErrorString(e));
    }
    if (prev != device) cudaSetDevice(prev);
    return st;
}

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
