// attn_io.cu -- the steps either side of the attention reduction, on the
// device (HBM-bound elementwise kernels).
//
// Before, Qwen 3.5 gated attention (nm/src/qwen35.hpp:343-352, :386):
//   [Q | G] = the head-major pairs of the query projection (attention.hpp:31-57)
//   Q = rope(rmsnorm_per_head(Q)),  K = rope(rmsnorm_per_head(K))
//   cache <- (K, V)
// and Gemma 4 (gemma4.hpp:206-209, :676-680): the same without the gate, and
// V = rmsnorm_no_scale_per_head(V) (components.hpp:204-215).  RMSNorm<HeadDim>
// (components.hpp:167-180) walked over the heads (:248-281); half-split
// ("NEOX") RoPE with inv_freq_i = Base^(-2i/HeadDim) for the first
// RotaryNum/RotaryDen of the planes and 0 for the rest (attention.hpp:68-101).
// After (qwen35.hpp:390-393): A *= sigmoid(G).
//
// One warp per (token, head) row: a lane holds the row's elements lane + 32 e,
// so a RoPE pair (i, i + HeadDim/2) sits in one lane and the norm is one warp
// reduction.  A grid of a few CTAs per SM strides over the rows; each CTA
// copies the frequency table into shared memory once.  The rotated K (and a
// normed V) go through nmg_kv_append (positions, ring and dtype handling of
// the cache) from a staging buffer.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kv_cache.cuh"

namespace nmg {
namespace {

constexpr int kMaxPlanes = 256;  // HeadDim / 2 up to 512

struct QkArgs {
    const float* q;        // [T][Hq Dh], or [T][2 Hq Dh] as q_0 | g_0 | q_1 | g_1 ... when gated
    const float* k;        // [T][Hkv Dh]
    const float* v;        // [T][Hkv Dh] (read only when normed here)
    const float* q_gamma;  // [Dh]
    const float* k_gamma;  // [Dh]
    void* q_out;           // [T][Hq Dh] in q_dtype
    float* k_out;          // [T][Hkv Dh] fp32
    float* v_out;          // [T][Hkv Dh] fp32, when v_norm
    int64_t T, position, rows;
    int hq, hkv, dh, q_dtype, q_pair;  // q_pair = 2 for the gated layout, 1 otherwise
    float eps;
    float inv_freq[kMaxPlanes];
};

template <int PER>  // PER = Dh / 32 elements per lane
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const __grid_constant__ QkArgs a) {
    __shared__ float freq[kMaxPlanes];
    for (int i = threadIdx.x; i < a.dh / 2; i += blockDim.x) freq[i] = a.inv_freq[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t nq = a.T * a.hq, nk = a.T * a.hkv;
    const int64_t stride = (int64_t)gridDim.x * 8;
    for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < a.rows; r += stride) {
        // rows: Q (t, h) for r < nq, then K (t, h), then V (t, h) when normed
        const int kind = r < nq ? 0 : r < nq + nk ? 1 : 2;
        const int64_t rr = kind == 0 ? r : kind == 1 ? r - nq : r - nq - nk;
        const int hn = kind == 0 ? a.hq : a.hkv;
        const int64_t t = rr / hn;
        const float* src = kind == 0 ? a.q + rr * a.q_pair * a.dh : (kind == 1 ? a.k : a.v) + rr * a.dh;
        float x[PER];
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            x[e] = src[lane + 32 * e];
            ss = fmaf(x[e], x[e], ss);
        }
        ss = dev::warp_sum(ss);
        const float inv = 1.f / sqrtf(ss / (float)a.dh + a.eps);  // components.hpp:174, :212
        if (kind == 2) {
            float* o = a.v_out + rr * a.dh;
#pragma unroll
            for (int e = 0; e < PER; ++e) o[lane + 32 * e] = x[e] * inv;
            continue;
        }
        const float* gamma = kind == 0 ? a.q_gamma : a.k_gamma;
#pragma unroll
        for (int e = 0; e < PER; ++e) x[e] = gamma[lane + 32 * e] * x[e] * inv;
        const float pos = (float)(a.position + t);  // Position -> Scalar, attention.hpp:85
#pragma unroll
        for (int e = 0; e < PER / 2; ++e) {  // plane i = lane + 32 e pairs with i + Dh/2 (attention.hpp:84-91)
            float s, c;
            sincosf(pos * freq[lane + 32 * e], &s, &c);
            const float xi = x[e], yi = x[e + PER / 2];
            x[e] = xi * c - yi * s;
            x[e + PER / 2] = yi * c + xi * s;
        }
        if (kind == 0) {
            const int64_t o = rr * a.dh;
#pragma unroll
            for (int e = 0; e < PER; ++e) dev::store_from_f32(a.q_out, a.q_dtype, o + lane + 32 * e, x[e]);
        } else {
            float* o = a.k_out + rr * a.dh;
#pragma unroll
            for (int e = 0; e < PER; ++e) o[lane + 32 * e] = x[e];
        }
    }
}

// a[t][h][i] *= sigmoid(g[t][h][i]), g the second half of each head pair of
// qg: for row r = t * Hq + h of a, the gate row starts at (2 r + 1) * Dh.
// VEC consecutive elements per thread (VEC divides Dh, so they share a row).
template <int DT, int VEC>
__global__ void __launch_bounds__(256) gate_kernel(const float* __restrict__ qg, typename dev::Elem<DT>::T* __restrict__ a,
                                                   int64_t n, int dh) {
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * VEC; i < n; i += (int64_t)gridDim.x * blockDim.x * VEC) {
        const int64_t r = i / dh;
        const float* g = qg + (2 * r + 1) * dh + (i - r * dh);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const float v = dev::Elem<DT>::load(a + i + j) * (1.f / (1.f + expf(-g[j])));  // sigmoid, core.hpp:579
            dev::store_from_f32(a, DT, i + j, v);
        }
    }
}

}  // namespace
}  // namespace nmg

using namespace nmg;

namespace nmg {
namespace {

// Validates, fills the frequency table and launches the row kernel on the
// current device; K (and V when v_norm) land in k_out / v_out as fp32.
int launch_prepare(const char* who, int hq, int hkv, int dh, int64_t position, int64_t T, const float* q, int q_gated,
                   const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm, float eps,
                   double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype, float* k_out,
                   float* v_out, cudaStream_t stream) {
    if (hq <= 0 || hkv <= 0 || hq % hkv != 0) return set_error(NMG_INVALID_ARGUMENT, "%s: Hq must be a multiple of Hkv", who);
    if (dh <= 0 || dh % 64 != 0 || dh > 2 * kMaxPlanes)
        return set_error(NMG_UNSUPPORTED, "%s: head_dim must be a multiple of 64 up to %d", who, 2 * kMaxPlanes);
    if (rotary_den <= 0 || rotary_num < 0 || rotary_num > rotary_den || !(rope_base > 0))
        return set_error(NMG_INVALID_ARGUMENT, "%s: RoPE fraction or base out of range", who);
    if (T < 0 || position < 0) return set_error(NMG_INVALID_ARGUMENT, "%s: negative rows or position", who);
    if (!dtype_valid(q_dtype)) return set_error(NMG_INVALID_ARGUMENT, "%s: bad q dtype", who);
    if (T == 0) return NMG_OK;
    if (!q || !k || !v || !q_gamma || !k_gamma || !q_out || !k_out || (v_norm && !v_out))
        return set_error(NMG_INVALID_ARGUMENT, "%s: null argument", who);
    QkArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.q_gamma = q_gamma;
    a.k_gamma = k_gamma;
    a.q_out = q_out;
    a.k_out = k_out;
    a.v_out = v_norm ? v_out : nullptr;
    a.T = T;
    a.position = position;
    a.hq = hq;
    a.hkv = hkv;
    a.dh = dh;
    a.q_dtype = q_dtype;
    a.q_pair = q_gated ? 2 : 1;
    a.eps = eps;
    a.rows = T * (int64_t)(hq + (v_norm ? 2 : 1) * hkv);
    // RotaryEmbedding's table (attention.hpp:76-80): double pow, then fp32.
    const int planes = dh / 2, rotary = (int)((int64_t)rotary_num * dh / rotary_den / 2);
    for (int i = 0; i < kMaxPlanes; ++i)
        a.inv_freq[i] = i < planes && i < rotary ? (float)pow(rope_base, -(double)(2 * i) / (double)dh) : 0.f;
    int device = 0, sms = 148;
    NMG_CUDA_TRY(cudaGetDevice(&device));
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const unsigned grid = (unsigned)std::min<int64_t>((a.rows + 7) / 8, (int64_t)sms * 8);
    switch (dh / 32) {
        case 2: qk_norm_rope_kernel<2><<<grid, 256, 0, stream>>>(a); break;
        case 4: qk_norm_rope_kernel<4><<<grid, 256, 0, stream>>>(a); break;
        case 6: qk_norm_rope_kernel<6><<<grid, 256, 0, stream>>>(a); break;
        case 8: qk_norm_rope_kernel<8><<<grid, 256, 0, stream>>>(a); break;
        case 10: qk_norm_rope_kernel<10><<<grid, 256, 0, stream>>>(a); break;
        case 12: qk_norm_rope_kernel<12><<<grid, 256, 0, stream>>>(a); break;
        case 14: qk_norm_rope_kernel<14><<<grid, 256, 0, stream>>>(a); break;
        case 16: qk_norm_rope_kernel<16><<<grid, 256, 0, stream>>>(a); break;
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(NMG_CUDA_ERROR, "%s: launch: %s", who, cudaGetErrorString(e));
    return NMG_OK;
}

}  // namespace
}  // namespace nmg

extern "C" int nmg_attn_prepare(int hq, int hkv, int head_dim, int64_t position, int64_t T, const float* q, int q_gated,
                                const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm,
                                float eps, double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype,
                                float* k_out, float* v_out, void* stream) {
    return launch_prepare("nmg_attn_prepare", hq, hkv, head_dim, position, T, q, q_gated, k, v, q_gamma, k_gamma,
                          v_norm, eps, rope_base, rotary_num, rotary_den, q_out, q_dtype, k_out, v_out,
                          (cudaStream_t)stream);
}

extern "C" int nmg_attn_prologue(nmg_kv_cache* cache, int hq, int64_t position, int64_t T, const float* q, int q_gated,
                                 const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm,
                                 float eps, double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype,
                                 void* stream) {
    if (!cache) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_prologue: null cache");
    if (T <= 0)
        return T < 0 ? set_error(NMG_INVALID_ARGUMENT, "nmg_attn_prologue: negative rows") : NMG_OK;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != cache->device) NMG_CUDA_TRY(cudaSetDevice(cache->device));
    const size_t kv_bytes = (size_t)T * cache->hkv * cache->dh * sizeof(float);
    void* tmp = nullptr;
    int st = device_staging(cache->device, v_norm ? 2 * kv_bytes : kv_bytes, &tmp);
    float* k_out = (float*)tmp;
    float* v_out = v_norm && tmp ? (float*)((char*)tmp + kv_bytes) : nullptr;
    if (st == NMG_OK)
        st = launch_prepare("nmg_attn_prologue", hq, cache->hkv, cache->dh, position, T, q, q_gated, k, v, q_gamma,
                            k_gamma, v_norm, eps, rope_base, rotary_num, rotary_den, q_out, q_dtype, k_out, v_out,
                            (cudaStream_t)stream);
    if (st == NMG_OK) st = nmg_kv_append(cache, position, k_out, v_norm ? v_out : v, T, NMG_F32, stream);
    if (prev != cache->device) cudaSetDevice(prev);
    return st;
}

extern "C" int nmg_attn_gate(int64_t T, int hq, int dh, const float* qg, void* a, int a_dtype, void* stream) {
    if (T < 0 || hq <= 0 || dh <= 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_gate: bad dimensions");
    if (!dtype_valid(a_dtype)) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_gate: bad dtype");
    if (T == 0) return NMG_OK;
    if (!qg || !a) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_gate: null argument");
    const int64_t n = T * hq * dh;
    const int vec = dh % 4 == 0 ? 4 : 1;
    const unsigned blocks = (unsigned)std::min<int64_t>((n / vec + 255) / 256, 148 * 16);
    const cudaStream_t s = (cudaStream_t)stream;
    if (a_dtype == NMG_F32) {
        if (vec == 4) gate_kernel<NMG_F32, 4><<<blocks, 256, 0, s>>>(qg, (float*)a, n, dh);
        else gate_kernel<NMG_F32, 1><<<blocks, 256, 0, s>>>(qg, (float*)a, n, dh);
    } else if (a_dtype == NMG_BF16) {
        if (vec == 4) gate_kernel<NMG_BF16, 4><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
        else gate_kernel<NMG_BF16, 1><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
    } else {
        if (vec == 4) gate_kernel<NMG_F16, 4><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
        else gate_kernel<NMG_F16, 1><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
    }
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}
