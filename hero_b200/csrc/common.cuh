// common.cuh -- shared device/host helpers for the nmg CUDA library (sm_100a).
//
// Status plumbing, dtype conversions that reproduce the reference engine's
// fp32->bf16 / fp32->fp16 rounding bit for bit (nm/src/core.hpp:61-100), and
// thin inline-PTX wrappers for mbarriers, bulk/tensor TMA copies and tcgen05.
// Every spin wait is bounded: it gives up after a fixed number of polls,
// records an error code in a device flag and lets the kernel return.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

#include "../../include/nmg.h"

// ---------------------------------------------------------------- host side

namespace nmg {

// Records the message for nmg_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...);

#define NMG_CUDA_TRY(expr)                                                                 \
    do {                                                                                   \
        cudaError_t err__ = (expr);                                                        \
        if (err__ != cudaSuccess)                                                          \
            return ::nmg::set_error(NMG_CUDA_ERROR, "%s: %s (%s:%d)", #expr,               \
                                    cudaGetErrorString(err__), __FILE__, __LINE__);        \
    } while (0)

inline int dtype_size(int dtype) { return dtype == NMG_F32 ? 4 : 2; }
inline bool dtype_valid(int dtype) { return dtype == NMG_F32 || dtype == NMG_F16 || dtype == NMG_BF16; }

// Per-device scratch owned by the library: grows on demand, never shrinks.
// Kernels that need it take a pointer; callers that cannot allocate use the
// entry points that take caller memory instead.
int device_scratch(int device, size_t bytes, void** ptr);
// A second, independent pool for staging copies (never the same memory as
// device_scratch, so a kernel may use both).
int device_staging(int device, size_t bytes, void** ptr);
// Zero-initialised int32 counters (the split-KV merge tickets).  Every kernel
// that takes a ticket returns it to zero before it exits, so the pool is all
// zeros between launches; nothing else may write it.
int device_tickets(int device, size_t bytes, void** ptr);
// A zero-initialised int32 error flag per device.  Kernels OR bits into it
// (dev::kErrWaitTimeout, dev::kErrF16Overflow); nmg_device_status reports them.
int device_error_flag(int device, int** flag);
// Copies the device error flags back (synchronising `stream`), clears them,
// and turns a raised bit into NMG_DEVICE_TIMEOUT or NMG_VALUE_OVERFLOW.  Reads
// only flags that already exist: it allocates nothing.
int check_device_flag(int device, cudaStream_t stream);
// The no-allocation decode path's own error word (inside its fixed device
// array), or null when that path never ran on `device`; _init looks it up
// (no allocation) with `device` current.
int* noalloc_error_word(int device);
int noalloc_error_word_init(int device, int** word);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per device and kernel;
// `done` holds one bit per device (devices 64 and up set it on every call).
// Safe to call from several host threads.
template <typename Kernel>
int set_smem_once(Kernel kern, int bytes, std::atomic<uint64_t>& done) {
    int dev_id = 0;
    NMG_CUDA_TRY(cudaGetDevice(&dev_id));
    const uint64_t bit = dev_id < 64 ? (uint64_t(1) << dev_id) : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return NMG_OK;
    NMG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    if (bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return NMG_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda);
// null when the driver does not provide it.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

}  // namespace nmg

// -------------------------------------------------------------- device side

namespace nmg {
namespace dev {

// Bits of the device error flag.
constexpr int kErrWaitTimeout = 1;  // a bounded wait gave up
constexpr int kErrF16Overflow = 2;  // a finite bf16 V value beyond fp16's range reached a bf16 cache
constexpr long long kMaxPolls = 1ll << 22;  // ~ a second or so of polling before giving up

// fp32 -> bf16, round to nearest even, quiet NaN (core.hpp:92-100).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    uint32_t bits = __float_as_uint(f);
    if ((bits & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

// fp32 -> fp16 with the reference's own rounding (core.hpp:61-79): the
// normal range rounds on bit 12 alone, subnormals round half up, and
// anything below 2^-25 flushes to signed zero.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t m = x & 0x7FFFFFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const uint32_t shift = (uint32_t)(14 - e);
        uint32_t r = m >> shift;
        if ((m >> (shift - 1)) & 1u) ++r;
        return (uint16_t)(sign | r);
    }
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    uint16_t h = (uint16_t)(sign | ((uint32_t)e << 10) | (m >> 13));
    if (m & 0x1000u) ++h;
    return h;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

template <int DT>
struct Elem;
template <>
struct Elem<NMG_F32> {
    using T = float;
    static __device__ __forceinline__ float load(const float* p) { return *p; }
};
template <>
struct Elem<NMG_F16> {
    using T = uint16_t;
    static __device__ __forceinline__ float load(const uint16_t* p) { return f16_bits_to_f32(*p); }
};
template <>
struct Elem<NMG_BF16> {
    using T = uint16_t;
    static __device__ __forceinline__ float load(const uint16_t* p) { return bf16_bits_to_f32(*p); }
};

__device__ __forceinline__ float load_as_f32(const void* base, int dtype, int64_t i) {
    if (dtype == NMG_F32) return ((const float*)base)[i];
    const uint16_t b = ((const uint16_t*)base)[i];
    return dtype == NMG_BF16 ? bf16_bits_to_f32(b) : f16_bits_to_f32(b);
}

__device__ __forceinline__ void store_from_f32(void* base, int dtype, int64_t i, float v) {
    if (dtype == NMG_F32)
        ((float*)base)[i] = v;
    else if (dtype == NMG_BF16)
        ((uint16_t*)base)[i] = f32_to_bf16_bits(v);
    else
        ((uint16_t*)base)[i] = f32_to_f16_bits(v);
}

// ---- shared-memory addresses, mbarriers, bulk copies (PTX ISA 8.x) ----------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe: has the phase with `parity` completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with `parity` to complete.  Returns false (and
// raises the kernel's error flag) when it gives up; callers then skip the
// remaining work and fall through to their normal exit.  A phase that has
// already completed is seen by the non-blocking probe, which costs far less
// than a try_wait.
template <long long kPolls>
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bar, uint32_t parity, int* err_flag) {
    if (mbar_test_wait(bar, parity)) return true;
    for (long long i = 0; i < kPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err_flag) atomicOr(err_flag, kErrWaitTimeout);
    return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err_flag) {
    return mbar_wait_n<kMaxPolls>(bar, parity, err_flag);
}

// Untiled bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled TMA load into this CTA's shared memory.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Prefetch one tile of a 3-D tensor map into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int32_t x, int32_t y, int32_t z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(x), "r"(y),
                 "r"(z)
                 : "memory");
}

// Prefetch `bytes` of global memory into L2 (address 16-byte aligned, size a
// multiple of 16).  Only a hint: L2 is where device memory is kept coherent,
// so a later read still sees whatever a kernel writes there in between.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem), "r"(bytes) : "memory");
}

// Untiled bulk copy shared -> global in the thread's bulk group; both
// addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// All but the most recent bulk group have finished reading their sources.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace dev
}  // namespace nmg
