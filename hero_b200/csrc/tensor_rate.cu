// tensor_rate.cu -- issue-loop measurement of the tcgen05 tensor-core rate,
// built into its own library (libnmg_rate.so) for bench.py's roofline
// denominators; nothing on the product path calls it.
//
// One CTA per SM; its thread 0 issues `reps` back-to-back tcgen05.mma of
// shape M = 128 x N x K into one TMEM accumulator (kind::tf32, K = 8, or
// kind::f16 with bf16 operands, K = 16), both operands in shared memory
// (zeros, K-major, 128-byte swizzle -- the forms the chunked delta rule and
// the prefill kernels issue), then waits for the last one through
// tcgen05.commit.  clock64 over the loop gives cycles per MMA; clock64
// against %globaltimer over the same interval gives the SM clock, so
//   TFLOP/s = 2 M N K / (cycles per MMA) x clock x SMs.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace nmg {
namespace {

struct RateOut {
    long long cycles;
    long long ns;
    int err;
    int pad;
};

__global__ void __launch_bounds__(128, 1) tensor_rate_kernel(int kind, int n, int reps, RateOut* out) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char* a_tile = smem;            // 128 rows x 128 B
    unsigned char* b_tile = smem + 16384;    // n rows x 128 B (n <= 256)
    uint64_t* bar = (uint64_t*)(smem + 16384 + 32768);
    uint32_t* slot = (uint32_t*)(bar + 1);
    int* err = (int*)(slot + 1);
    for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x) ((uint4*)smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        dev::mbar_init(bar, 1);
        dev::fence_mbar_init();
        *err = 0;
    }
    dev::fence_proxy_async_smem();  // the zeros, written by the generic proxy, before the MMAs read them
    if (threadIdx.x < 32) {
        tc::tmem_alloc(slot, 256);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *slot;
    if (threadIdx.x == 0) {
        const uint64_t ad = tc::smem_desc_sw128(dev::smem_u32(a_tile), 16, 1024);
        const uint64_t bd = tc::smem_desc_sw128(dev::smem_u32(b_tile), 16, 1024);
        const uint32_t id = kind == 0 ? tc::idesc_tf32(128, n, 0, 0) : tc::idesc_f16(128, n, 1, 0, 0);
        long long g0, g1;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
        const long long c0 = clock64();
        for (int r = 0; r < reps; ++r) {
            if (kind == 0)
                tc::mma_tf32_ss(tmem, ad, bd, id, r > 0);
            else
                tc::mma_f16_ss(tmem, ad, bd, id, r > 0);
        }
        tc::commit(bar);
        const bool ok = dev::mbar_wait(bar, 0, err);
        const long long c1 = clock64();
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));
        out[blockIdx.x] = RateOut{c1 - c0, g1 - g0, ok ? 0 : 1, 0};
    }
    tc::fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 256);
    }
}

}  // namespace
}  // namespace nmg

// kind 0: tf32 (K = 8), 1: bf16 (K = 16); n: the MMA's N (16..256, a multiple
// of 16); reps: MMAs per SM.  Writes the mean cycles per MMA, the SM clock in
// GHz and the number of SMs measured.  Returns 0, or a CUDA error code.
extern "C" __attribute__((visibility("default"))) int nmg_rate_tensor(int kind, int n, int reps, double* cycles_per_mma,
                                                                      double* ghz, int* sms) {
    if ((kind != 0 && kind != 1) || n < 16 || n > 256 || n % 16 != 0 || reps < 1) return (int)cudaErrorInvalidValue;
    int dev = 0, nsm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    const int smem = 1024 + 16384 + 32768 + 64;
    e = cudaFuncSetAttribute(nmg::tensor_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    nmg::RateOut* d_out = nullptr;
    e = cudaMalloc(&d_out, sizeof(nmg::RateOut) * nsm);
    if (e != cudaSuccess) return (int)e;
    nmg::tensor_rate_kernel<<<nsm, 128, smem>>>(kind, n, reps, d_out);
    e = cudaGetLastError();
    nmg::RateOut* h = new nmg::RateOut[nsm];
    if (e == cudaSuccess) e = cudaMemcpy(h, d_out, sizeof(nmg::RateOut) * nsm, cudaMemcpyDeviceToHost);
    cudaFree(d_out);
    if (e == cudaSuccess) {
        double cyc = 0, ns = 0;
        int bad = 0;
        for (int i = 0; i < nsm; ++i) {
            cyc += (double)h[i].cycles;
            ns += (double)h[i].ns;
            bad += h[i].err;
        }
        if (bad) e = cudaErrorLaunchTimeout;
        *cycles_per_mma = cyc / nsm / reps;
        *ghz = ns > 0 ? cyc / ns : 0.0;
        *sms = nsm;
    }
    delete[] h;
    return (int)e;
}

// The warp-level integer MMA rate: every warp of 16 per SM issues `reps`
// rounds of 8 independent mma.sync m16n8k32 s8 x s8 -> s32 on register
// operands (the instruction the quantised projection GEMM issues).  Timed with
// CUDA events around one launch; returns tera-ops per second.
namespace nmg {
namespace {

__global__ void __launch_bounds__(512) imma_rate_kernel(int reps, int* sink) {
    int c[8][4] = {};
    const uint32_t a0 = threadIdx.x, a1 = a0 * 3u, a2 = a0 * 5u, a3 = a0 * 7u, b0 = a0 * 11u, b1 = a0 * 13u;
    for (int i = 0; i < reps; ++i) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                : "+r"(c[j][0]), "+r"(c[j][1]), "+r"(c[j][2]), "+r"(c[j][3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
    int s = 0;
    for (int j = 0; j < 8; ++j) s += c[j][0] ^ c[j][3];
    if (s == 0x7fffffff) sink[0] = s;  // keeps the loop live
}

}  // namespace
}  // namespace nmg

extern "C" __attribute__((visibility("default"))) int nmg_rate_imma(int reps, double* tops) {
    if (reps < 1 || !tops) return (int)cudaErrorInvalidValue;
    int dev = 0, nsm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    int* sink = nullptr;
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    e = cudaMalloc(&sink, sizeof(int));
    if (e == cudaSuccess) e = cudaEventCreate(&t0);
    if (e == cudaSuccess) e = cudaEventCreate(&t1);
    if (e == cudaSuccess) {
        nmg::imma_rate_kernel<<<nsm, 512>>>(reps, sink);  // warm-up
        cudaEventRecord(t0);
        nmg::imma_rate_kernel<<<nsm, 512>>>(reps, sink);
        cudaEventRecord(t1);
        e = cudaEventSynchronize(t1);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t0, t1);
    if (e == cudaSuccess) *tops = (double)nsm * 16 * reps * 8 * (2.0 * 16 * 8 * 32) / (ms * 1e-3) / 1e12;
    if (t0) cudaEventDestroy(t0);
    if (t1) cudaEventDestroy(t1);
    if (sink) cudaFree(sink);
    return (int)e;
}
