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
// One warp per (token, head) row.  A lane holds VW consecutive elements in
// each of 2M chunks (element 32 VW j + VW lane + w), VW the widest of 4, 2, 1
// with 64 VW | HeadDim, so loads and stores are 16/8/4-byte vectors and the
// RoPE partner of chunk j < M is chunk j + M in the same lane.  The norm is
// one warp reduction.  One wave of CTAs (as many per SM as fit) strides over
// items of 8 rows of one token, each warp loading its next row before
// finishing the current one, so a token's angles are evaluated once per item
// rather than once per head; each CTA copies the frequency table into shared
// memory once.  K and V rows go
// straight to their cache slots in the cache's dtype (the ring layout of
// kv_cache.cuh); rows a batch evicts before it ends are never written.
#include <math.h>

#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "kv_cache.cuh"

namespace nmg {
namespace {

constexpr int kMaxPlanes = 256;  // HeadDim / 2 up to 512

struct QkArgs {
    const float* q;        // [T][Hq Dh], or [T][2 Hq Dh] as q_0 | g_0 | q_1 | g_1 ... when gated
    const float* k;        // [T][Hkv Dh]
    const float* v;        // [T][Hkv Dh]
    const float* q_gamma;  // [Dh]
    const float* k_gamma;  // [Dh]
    void* q_out;           // [T][Hq Dh] in q_dtype
    // K/V destination: a cache ([Hkv][slots][Dh], kv_dtype with V per store_cache_v)
    // or, with slots == 0, fp32 rows [T][Hkv Dh].
    void* k_dst;
    void* v_dst;
    int64_t slots, slot0, row0, kv_rows;  // tokens row0 .. kv_rows-1 are written, token row0 to slot0
    int64_t T, position, rows;
    int hq, hkv, dh, q_dtype, kv_dtype, q_pair, v_norm;
    int* err;  // device error flag: a bf16 cache's V overflowing fp16
    int idx32;  // row and slot arithmetic fits 32 bits (one divide instead of a 64-bit sequence)
    float eps;
    float inv_freq[kMaxPlanes];
};

template <int VW>
__device__ __forceinline__ void load_vec(const float* p, float* x) {
    if constexpr (VW == 4) {
        const float4 v = *reinterpret_cast<const float4*>(p);
        x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
    } else if constexpr (VW == 2) {
        const float2 v = *reinterpret_cast<const float2*>(p);
        x[0] = v.x, x[1] = v.y;
    } else {
        x[0] = *p;
    }
}

// VW values to element i.. of a row buffer of dtype dt (v_cache: the V rule of
// a bf16 cache, bf16-rounded values stored as fp16).  Returns true when such a
// V value overflowed fp16.
template <int VW>
__device__ __forceinline__ bool store_vec(void* base, int dt, int64_t i, const float* x, bool v_cache) {
    bool overflow = false;
    if (dt == NMG_F32) {
        float* p = (float*)base + i;
        if constexpr (VW == 4) *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
        else if constexpr (VW == 2) *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
        else *p = x[0];
        return overflow;
    }
    uint32_t b[VW];
    if (dt == NMG_BF16 && !v_cache && VW >= 2) {
        // Hardware round-to-nearest-even equals core.hpp:92-100 for every
        // non-NaN input; a NaN takes the reference's own quieting.
#pragma unroll
        for (int w = 0; w < VW; w += 2) {
            uint32_t r;
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x[w + 1]), "f"(x[w]));
            if (x[w] != x[w] || x[w + 1] != x[w + 1])
                r = (uint32_t)dev::f32_to_bf16_bits(x[w]) | ((uint32_t)dev::f32_to_bf16_bits(x[w + 1]) << 16);
            b[w] = r & 0xFFFFu;
            b[w + 1] = r >> 16;
        }
    } else {
#pragma unroll
        for (int w = 0; w < VW; ++w) {
            if (dt == NMG_BF16)
                b[w] = v_cache ? cache_v_bits(x[w], overflow) : dev::f32_to_bf16_bits(x[w]);
            else
                b[w] = dev::f32_to_f16_bits(x[w]);
        }
    }
    uint16_t* p = (uint16_t*)base + i;
    if constexpr (VW == 4) *reinterpret_cast<uint2*>(p) = make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
    else if constexpr (VW == 2) *reinterpret_cast<uint32_t*>(p) = b[0] | (b[1] << 16);
    else *p = (uint16_t)b[0];
    return overflow;
}

// The row space is token-major: token t's rows are its Hq Q heads, its Hkv K
// heads, then (when V is written here) its Hkv V heads.
struct Row {
    int kind;  // 0 Q, 1 K, 2 V; -1: nothing to do
    int64_t rr, t, dst;  // rr: the row's index in its own tensor ([T][heads])
    const float* src;
};

// Row c of token t (c < per_token); t >= T means no row.
__device__ __forceinline__ Row row_at(const QkArgs& a, int64_t t, int c) {
    Row w{-1, 0, t, 0, nullptr};
    if (t >= a.T) return w;
    w.kind = c < a.hq ? 0 : c < a.hq + a.hkv ? 1 : 2;
    const int h = w.kind == 0 ? c : w.kind == 1 ? c - a.hq : c - a.hq - a.hkv;
    w.rr = t * (w.kind == 0 ? a.hq : a.hkv) + h;
    if (w.kind != 0) {
        if (t < a.row0 || t >= a.kv_rows) {  // evicted within the batch, or refused
            w.kind = -1;
            return w;
        }
        if (a.slots) {
            const int64_t ring = a.slot0 + (t - a.row0);
            const int64_t slot = a.idx32 ? (int64_t)((uint32_t)ring % (uint32_t)a.slots) : ring % a.slots;
            w.dst = ((int64_t)h * a.slots + slot) * a.dh;
        } else {
            w.dst = w.rr * a.dh;
        }
    }
    w.src = w.kind == 0 ? a.q + w.rr * a.q_pair * a.dh : (w.kind == 1 ? a.k : a.v) + w.rr * a.dh;
    return w;
}

// (token, row-in-token) of global row r.
__device__ __forceinline__ void token_of(const QkArgs& a, int64_t r, int per_token, int64_t* t, int* c) {
    *t = a.idx32 ? (int64_t)((uint32_t)r / (uint32_t)per_token) : r / per_token;
    *c = (int)(r - *t * per_token);
}

template <int VW, int M>
__device__ __forceinline__ void finish_row(const QkArgs& a, const Row& w, float (&x)[2 * M][VW],
                                           const float (&cs)[M][VW], const float (&sn)[M][VW], int lane) {
    constexpr int J = 2 * M;
    const int kv_dt = a.slots ? a.kv_dtype : NMG_F32;
    if (w.kind == 2 && !a.v_norm) {
        bool overflow = false;
#pragma unroll
        for (int j = 0; j < J; ++j)
            overflow |= store_vec<VW>(a.v_dst, kv_dt, w.dst + 32 * VW * j + VW * lane, x[j], true);
        if (overflow && a.err) atomicOr(a.err, dev::kErrF16Overflow);
        return;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int e = 0; e < VW; ++e) ss = fmaf(x[j][e], x[j][e], ss);
    ss = dev::warp_sum(ss);
    const float inv = 1.f / sqrtf(ss / (float)a.dh + a.eps);  // components.hpp:174, :212
    if (w.kind == 2) {
        bool overflow = false;
#pragma unroll
        for (int j = 0; j < J; ++j) {
#pragma unroll
            for (int e = 0; e < VW; ++e) x[j][e] *= inv;
            overflow |= store_vec<VW>(a.v_dst, kv_dt, w.dst + 32 * VW * j + VW * lane, x[j], true);
        }
        if (overflow && a.err) atomicOr(a.err, dev::kErrF16Overflow);
        return;
    }
    const float* gamma = w.kind == 0 ? a.q_gamma : a.k_gamma;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        float g[VW];
        load_vec<VW>(gamma + 32 * VW * j + VW * lane, g);
#pragma unroll
        for (int e = 0; e < VW; ++e) x[j][e] = g[e] * x[j][e] * inv;
    }
#pragma unroll
    for (int j = 0; j < M; ++j) {  // plane i pairs with i + Dh/2 (attention.hpp:84-91)
#pragma unroll
        for (int e = 0; e < VW; ++e) {
            const float xi = x[j][e], yi = x[j + M][e];
            x[j][e] = xi * cs[j][e] - yi * sn[j][e];
            x[j + M][e] = yi * cs[j][e] + xi * sn[j][e];
        }
    }
    void* out = w.kind == 0 ? a.q_out : a.k_dst;
    const int dt = w.kind == 0 ? a.q_dtype : kv_dt;
    const int64_t o = w.kind == 0 ? w.rr * a.dh : w.dst;
#pragma unroll
    for (int j = 0; j < J; ++j) store_vec<VW>(out, dt, o + 32 * VW * j + VW * lane, x[j], false);
}

constexpr int kRowsPerItem = 8;

// Warps take items of kRowsPerItem consecutive rows (items w, w + warps, ...)
// and walk their rows with the next row's loads issued before the current
// row's arithmetic.  cos/sin of the lane's planes are computed once per token
// a warp meets (rotating planes only: the rest keep cos 1, sin 0, whose
// product is the reference's own angle-0 rotation).
template <int VW, int M>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const __grid_constant__ QkArgs a) {
    constexpr int J = 2 * M;
    __shared__ __align__(16) float freq[kMaxPlanes];
    for (int i = threadIdx.x; i < a.dh / 2; i += blockDim.x) freq[i] = a.inv_freq[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int per_token = a.hq + a.hkv + (a.v_dst ? a.hkv : 0);
    const int64_t total = a.T * per_token;
    const int64_t items = (total + kRowsPerItem - 1) / kRowsPerItem;
    const int64_t warps = (int64_t)gridDim.x * 8;
    int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    int k = 0;
    // (nt, nc): token and row-in-token of the row being fetched; one division
    // when a warp moves to its next item, increments within an item.
    int64_t nt = 0;
    int nc = 0;
    if (item < items) token_of(a, item * kRowsPerItem, per_token, &nt, &nc);
    Row cur = item < items && item * kRowsPerItem < total ? row_at(a, nt, nc) : Row{-1, 0, 0, 0, nullptr};
    float x[J][VW];
    if (cur.kind >= 0) {
#pragma unroll
        for (int j = 0; j < J; ++j) load_vec<VW>(cur.src + 32 * VW * j + VW * lane, x[j]);
    }
    float cs[M][VW], sn[M][VW];
    int64_t trig_t = -1;
    while (item < items) {
        int64_t nitem = item;
        int nk = k + 1;
        if (nk == kRowsPerItem) {
            nitem += warps, nk = 0;
            if (nitem < items) token_of(a, nitem * kRowsPerItem, per_token, &nt, &nc);
        } else if (++nc == per_token) {
            ++nt, nc = 0;
        }
        const bool more = nitem < items && nitem * kRowsPerItem + nk < total;
        const Row nxt = more ? row_at(a, nt, nc) : Row{-1, 0, 0, 0, nullptr};
        float y[J][VW];
        if (nxt.kind >= 0) {
#pragma unroll
            for (int j = 0; j < J; ++j) load_vec<VW>(nxt.src + 32 * VW * j + VW * lane, y[j]);
        }
        if (cur.kind >= 0) {
            if (cur.kind < 2 && cur.t != trig_t) {
                const float pos = (float)(a.position + cur.t);  // Position -> Scalar, attention.hpp:85
#pragma unroll
                for (int j = 0; j < M; ++j) {
                    float f[VW];
                    load_vec<VW>(freq + 32 * VW * j + VW * lane, f);
#pragma unroll
                    for (int e = 0; e < VW; ++e) {
                        cs[j][e] = 1.f, sn[j][e] = 0.f;
                        if (f[e] != 0.f) sincosf(pos * f[e], &sn[j][e], &cs[j][e]);
                    }
                }
                trig_t = cur.t;
            }
            finish_row<VW, M>(a, cur, x, cs, sn, lane);
        }
        cur = nxt;
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int e = 0; e < VW; ++e) x[j][e] = y[j][e];
        item = nitem, k = nk;
    }
}

// a[t][h][i] *= sigmoid(g[t][h][i]), g the second half of each head pair of
// qg: for row r = t * Hq + h of a, the gate row starts at (2 r + 1) * Dh.
// VEC consecutive elements per thread (VEC divides Dh, so they share a row);
// with VEC = 8 the gate and a move as 16-byte vectors.
template <int DT, int VEC>
__global__ void __launch_bounds__(256) gate_kernel(const float* __restrict__ qg, typename dev::Elem<DT>::T* __restrict__ a,
                                                   int64_t n, int dh) {
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * VEC; i < n; i += (int64_t)gridDim.x * blockDim.x * VEC) {
        const int64_t r = i / dh;
        const float* g = qg + (2 * r + 1) * dh + (i - r * dh);
        float gv[VEC], av[VEC];
        if constexpr (VEC == 8) {
            const float4 g0 = reinterpret_cast<const float4*>(g)[0], g1 = reinterpret_cast<const float4*>(g)[1];
            gv[0] = g0.x, gv[1] = g0.y, gv[2] = g0.z, gv[3] = g0.w, gv[4] = g1.x, gv[5] = g1.y, gv[6] = g1.z, gv[7] = g1.w;
            if constexpr (DT == NMG_F32) {
                const float4 a0 = reinterpret_cast<const float4*>(a + i)[0], a1 = reinterpret_cast<const float4*>(a + i)[1];
                av[0] = a0.x, av[1] = a0.y, av[2] = a0.z, av[3] = a0.w, av[4] = a1.x, av[5] = a1.y, av[6] = a1.z, av[7] = a1.w;
            } else {
                const uint4 w = *reinterpret_cast<const uint4*>(a + i);
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint16_t lo = (uint16_t)(u[j] & 0xFFFFu), hi = (uint16_t)(u[j] >> 16);
                    av[2 * j] = dev::Elem<DT>::load(&lo);
                    av[2 * j + 1] = dev::Elem<DT>::load(&hi);
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) gv[j] = g[j], av[j] = dev::Elem<DT>::load(a + i + j);
        }
#pragma unroll
        for (int j = 0; j < VEC; ++j) av[j] *= 1.f / (1.f + expf(-gv[j]));  // sigmoid, core.hpp:579
        if constexpr (VEC == 8 && DT == NMG_F32) {
            reinterpret_cast<float4*>(a + i)[0] = make_float4(av[0], av[1], av[2], av[3]);
            reinterpret_cast<float4*>(a + i)[1] = make_float4(av[4], av[5], av[6], av[7]);
        } else if constexpr (VEC == 8) {
            uint32_t u[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t lo = DT == NMG_BF16 ? dev::f32_to_bf16_bits(av[2 * j]) : dev::f32_to_f16_bits(av[2 * j]);
                const uint32_t hi = DT == NMG_BF16 ? dev::f32_to_bf16_bits(av[2 * j + 1]) : dev::f32_to_f16_bits(av[2 * j + 1]);
                u[j] = lo | (hi << 16);
            }
            *reinterpret_cast<uint4*>(a + i) = make_uint4(u[0], u[1], u[2], u[3]);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) dev::store_from_f32(a, DT, i + j, av[j]);
        }
    }
}

}  // namespace
}  // namespace nmg

using namespace nmg;

namespace nmg {
namespace {

// Where K and V go: a cache's slots (slots > 0), or fp32 rows.
struct KvDst {
    void* k = nullptr;
    void* v = nullptr;  // null: V is left to the caller (prepare without v_norm)
    int dtype = NMG_F32;
    int64_t slots = 0, slot0 = 0, row0 = 0, rows = 0;
    int* err = nullptr;  // the device error flag (a cache destination)
};

template <int VW, int M>
void launch_rows(const QkArgs& a, int sms, cudaStream_t s) {
    // Resident CTAs per SM at this variant's register count (one full wave), asked once.
    static const int per_sm = [] {
        int n = 0;
        return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qk_norm_rope_kernel<VW, M>, 256, 0) == cudaSuccess &&
                       n > 0
                   ? n
                   : 4;
    }();
    const int64_t items = (a.rows + kRowsPerItem - 1) / kRowsPerItem;
    const unsigned grid = (unsigned)std::min<int64_t>((items + 7) / 8, (int64_t)sms * per_sm);
    qk_norm_rope_kernel<VW, M><<<grid, 256, 0, s>>>(a);
}

// Validates, fills the frequency table and launches the row kernel on the
// current device.
int launch_prepare(const char* who, int hq, int hkv, int dh, int64_t position, int64_t T, const float* q, int q_gated,
                   const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm, float eps,
                   double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype, const KvDst& d,
                   cudaStream_t stream) {
    if (hq <= 0 || hkv <= 0 || hq % hkv != 0) return set_error(NMG_INVALID_ARGUMENT, "%s: Hq must be a multiple of Hkv", who);
    if (dh <= 0 || dh % 64 != 0 || dh > 2 * kMaxPlanes)
        return set_error(NMG_UNSUPPORTED, "%s: head_dim must be a multiple of 64 up to %d", who, 2 * kMaxPlanes);
    if (rotary_den <= 0 || rotary_num < 0 || rotary_num > rotary_den || !(rope_base > 0))
        return set_error(NMG_INVALID_ARGUMENT, "%s: RoPE fraction or base out of range", who);
    if (T < 0 || position < 0) return set_error(NMG_INVALID_ARGUMENT, "%s: negative rows or position", who);
    if (!dtype_valid(q_dtype)) return set_error(NMG_INVALID_ARGUMENT, "%s: bad q dtype", who);
    if (T == 0) return NMG_OK;
    if (!q || !k || !v || !q_gamma || !k_gamma || !q_out || !d.k)
        return set_error(NMG_INVALID_ARGUMENT, "%s: null argument", who);
    QkArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.q_gamma = q_gamma;
    a.k_gamma = k_gamma;
    a.q_out = q_out;
    a.k_dst = d.k;
    a.v_dst = d.v;
    a.slots = d.slots;
    a.slot0 = d.slot0;
    a.row0 = d.row0;
    a.kv_rows = d.rows;
    a.T = T;
    a.position = position;
    a.hq = hq;
    a.hkv = hkv;
    a.dh = dh;
    a.q_dtype = q_dtype;
    a.kv_dtype = d.dtype;
    a.q_pair = q_gated ? 2 : 1;
    a.v_norm = v_norm ? 1 : 0;
    a.eps = eps;
    a.err = d.err;
    a.rows = T * (int64_t)(hq + (d.v ? 2 : 1) * hkv);
    a.idx32 = a.rows < (1ll << 31) && d.slot0 + T < (1ll << 31) && d.slots < (1ll << 31) ? 1 : 0;
    // RotaryEmbedding's table (attention.hpp:76-80): double pow, then fp32;
    // the last table built on this thread is reused (a layer stack repeats one).
    struct Table {
        int dh = 0, num = 0, den = 0;
        double base = 0;
        float f[kMaxPlanes];
    };
    static thread_local Table last;
    if (last.dh != dh || last.num != rotary_num || last.den != rotary_den || last.base != rope_base) {
        const int planes = dh / 2, rotary = (int)((int64_t)rotary_num * dh / rotary_den / 2);
        for (int i = 0; i < kMaxPlanes; ++i)
            last.f[i] = i < planes && i < rotary ? (float)pow(rope_base, -(double)(2 * i) / (double)dh) : 0.f;
        last.dh = dh, last.num = rotary_num, last.den = rotary_den, last.base = rope_base;
    }
    memcpy(a.inv_freq, last.f, sizeof(a.inv_freq));
    int device = 0, sms = 148;
    NMG_CUDA_TRY(cudaGetDevice(&device));
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    // Vector width: the widest of 4, 2, 1 dividing Dh/64 that every row pointer's alignment allows.
    int vw = (dh / 64) % 4 == 0 ? 4 : (dh / 64) % 2 == 0 ? 2 : 1;
    const uintptr_t ptrs = (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)q_gamma | (uintptr_t)k_gamma |
                           (uintptr_t)q_out | (uintptr_t)d.k | (uintptr_t)d.v;
    while (vw > 1 && (ptrs % (4u * vw)) != 0) vw /= 2;
    const int m = dh / (64 * vw);
    switch (vw * 16 + m) {
        case 4 * 16 + 1: launch_rows<4, 1>(a, sms, stream); break;
        case 4 * 16 + 2: launch_rows<4, 2>(a, sms, stream); break;
        case 2 * 16 + 1: launch_rows<2, 1>(a, sms, stream); break;
        case 2 * 16 + 2: launch_rows<2, 2>(a, sms, stream); break;
        case 2 * 16 + 3: launch_rows<2, 3>(a, sms, stream); break;
        case 2 * 16 + 4: launch_rows<2, 4>(a, sms, stream); break;
        case 16 + 1: launch_rows<1, 1>(a, sms, stream); break;
        case 16 + 2: launch_rows<1, 2>(a, sms, stream); break;
        case 16 + 3: launch_rows<1, 3>(a, sms, stream); break;
        case 16 + 4: launch_rows<1, 4>(a, sms, stream); break;
        case 16 + 5: launch_rows<1, 5>(a, sms, stream); break;
        case 16 + 6: launch_rows<1, 6>(a, sms, stream); break;
        case 16 + 7: launch_rows<1, 7>(a, sms, stream); break;
        case 16 + 8: launch_rows<1, 8>(a, sms, stream); break;
        default: return set_error(NMG_UNSUPPORTED, "%s: head_dim %d", who, dh);
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
    if (v_norm && !v_out && T > 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_prepare: null v_out");
    KvDst d;
    d.k = k_out;
    d.v = v_norm ? v_out : nullptr;
    d.rows = T;
    return launch_prepare("nmg_attn_prepare", hq, hkv, head_dim, position, T, q, q_gated, k, v, q_gamma, k_gamma,
                          v_norm, eps, rope_base, rotary_num, rotary_den, q_out, q_dtype, d, (cudaStream_t)stream);
}

extern "C" int nmg_attn_prologue(nmg_kv_cache* cache, int hq, int64_t position, int64_t T, const float* q, int q_gated,
                                 const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm,
                                 float eps, double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype,
                                 void* stream) {
    if (!cache) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_prologue: null cache");
    if (T <= 0) return T < 0 ? set_error(NMG_INVALID_ARGUMENT, "nmg_attn_prologue: negative rows") : NMG_OK;
    if (!q || !k || !v || !q_gamma || !k_gamma || !q_out)  // before the cache's bookkeeping moves
        return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_prologue: null argument");
    if (cache->dtype == NMG_Q8_0) {
        // A Q8_0 cache quantises whole rows on append: prepare K (and V) in
        // fp32 staging, then append them through the quantiser.
        const int64_t n = T * cache->hkv * cache->dh;
        void* stage = nullptr;
        int st = device_staging(cache->device, (size_t)n * 4 * (v_norm ? 2 : 1), &stage);
        if (st != NMG_OK) return st;
        float* ks = (float*)stage;
        float* vs = v_norm ? ks + n : nullptr;
        st = nmg_attn_prepare(hq, cache->hkv, cache->dh, position, T, q, q_gated, k, v, q_gamma, k_gamma, v_norm, eps,
                              rope_base, rotary_num, rotary_den, q_out, q_dtype, ks, vs, stream);
        if (st != NMG_OK) return st;
        return nmg_kv_append(cache, position, ks, v_norm ? (const void*)vs : (const void*)v, T, NMG_F32, stream);
    }
    int* err = nullptr;  // made with the cache, so no allocation here
    int st = device_error_flag(cache->device, &err);
    if (st != NMG_OK) return st;
    int64_t accepted = 0;
    int deferred = NMG_OK;
    st = kv_append_begin(cache, position, T, &accepted, &deferred);
    if (st != NMG_OK) return st;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != cache->device) NMG_CUDA_TRY(cudaSetDevice(cache->device));
    KvDst d;
    d.k = cache->k;
    d.v = cache->v;
    d.dtype = cache->dtype;
    d.slots = cache->slots;
    d.err = err;
    d.rows = accepted;
    kv_append_slots(cache, position, accepted, &d.row0, &d.slot0);
    st = launch_prepare("nmg_attn_prologue", hq, cache->hkv, cache->dh, position, T, q, q_gated, k, v, q_gamma, k_gamma,
                        v_norm, eps, rope_base, rotary_num, rotary_den, q_out, q_dtype, d, (cudaStream_t)stream);
    if (st == NMG_OK) kv_append_commit(cache, position, accepted);
    if (prev != cache->device) cudaSetDevice(prev);
    return st == NMG_OK ? deferred : st;
}

extern "C" int nmg_attn_gate(int64_t T, int hq, int dh, const float* qg, void* a, int a_dtype, void* stream) {
    if (T < 0 || hq <= 0 || dh <= 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_gate: bad dimensions");
    if (!dtype_valid(a_dtype)) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_gate: bad dtype");
    if (T == 0) return NMG_OK;
    if (!qg || !a) return set_error(NMG_INVALID_ARGUMENT, "nmg_attn_gate: null argument");
    const int64_t n = T * hq * dh;
    const bool v8 = dh % 8 == 0 && ((uintptr_t)qg % 16) == 0 && ((uintptr_t)a % 16) == 0;
    const int vec = v8 ? 8 : 1;
    const unsigned blocks = (unsigned)std::min<int64_t>((n / vec + 255) / 256, 148 * 16);
    const cudaStream_t s = (cudaStream_t)stream;
    if (a_dtype == NMG_F32) {
        if (v8) gate_kernel<NMG_F32, 8><<<blocks, 256, 0, s>>>(qg, (float*)a, n, dh);
        else gate_kernel<NMG_F32, 1><<<blocks, 256, 0, s>>>(qg, (float*)a, n, dh);
    } else if (a_dtype == NMG_BF16) {
        if (v8) gate_kernel<NMG_BF16, 8><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
        else gate_kernel<NMG_BF16, 1><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
    } else {
        if (v8) gate_kernel<NMG_F16, 8><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
        else gate_kernel<NMG_F16, 1><<<blocks, 256, 0, s>>>(qg, (uint16_t*)a, n, dh);
    }
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}
