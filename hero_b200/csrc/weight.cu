// weight.cu -- the engine's quantised projections on the device:
// Weight<In,Out>::matvec / matmul / gather_rows (src/quant.hpp:439-487,
// src/quant_i8.hpp:351-514) over GGUF Q4_0 / Q8_0 / Q4_K / Q5_K / Q6_K blocks
// and F32 rows.
//
// Storage.  nmg_weight_create takes the GGUF bytes (one row per output,
// quant.hpp:479 `qp_ + o * row_bytes`) and re-lays them once into planes whose
// rows start on 16-byte boundaries, so a warp streams a row with 16-byte loads:
//   Q8_0  quants int8 [out][in]        + fp16 block scales [out][in/32]
//   Q4_0  nibbles [out][in/2] (a block's 16 bytes as stored) + fp16 scales
//   Q4_K  nibbles [out][in/2] + 16 B per superblock (d, dmin, 12 scale bytes)
//   Q5_K  as Q4_K + the high-bit plane [out][in/8]
//   Q6_K  low nibbles [out][in/2] + high pairs [out][in/4] + 16 int8 scales per
//         superblock + fp16 d [out][in/256]
// The bytes per weight are the GGUF ones; nothing is dequantised at rest.
//
// Products.  The reference's default path (quant_i8.hpp:351-392) quantises the
// activation row once (Q8_0 blocks for Q8_0/Q4_0 weights, Q8_K for Q4_K/Q6_K)
// and takes integer dot products per block; act_quant_* below reproduce those
// quantisers bit for bit and the product kernels form the same integer block
// sums with dp4a (exact), scaling them in fp32 per block as the reference does,
// so only the fp32 summation order differs.  Q5_K (no integer kernel in the
// reference, has_i8_kernel :325), F32 weights and the NM_FP32_ACT mode take the
// fp32-activation path: dequantise in registers, fp32 FMAs (quant.hpp:130-289).
//
// The matvec kernels are HBM-bound on the weight bytes: one warp per output row
// streams it with 16-byte loads, up to 8 activation rows reuse each loaded word
// (the reference's "stream W once per batch", quant_i8.hpp:420-425), and the
// activation quantiser runs as a programmatic dependent launch ahead of them so
// the weight loads start before the activations exist.
#include <stdint.h>

#include <algorithm>

#include "weight.cuh"

namespace nmg {
namespace {
using namespace wq;

// ---- re-lay the GGUF blocks into planes (one thread per block) ------------
__global__ void repack_kernel(const uint8_t* __restrict__ src, int type, int64_t out, int64_t nb, int64_t src_row,
                              uint8_t* qs, uint8_t* hi, uint32_t* meta, uint16_t* dp, uint32_t* ddp, int64_t qs_row,
                              int64_t hi_row, int64_t meta_row, int64_t d_row, int64_t dd_row) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= out * nb) return;
    const int64_t o = i / nb, b = i % nb;
    const uint8_t* s = src + o * src_row + b * block_bytes(type);
    auto u16 = [&](int off) { return (uint16_t)(s[off] | (s[off + 1] << 8)); };
    switch (type) {
        case GT_Q8_0:
            dp[o * d_row + b] = u16(0);
            for (int j = 0; j < 32; ++j) qs[o * qs_row + 32 * b + j] = s[2 + j];
            break;
        case GT_Q4_0:
            dp[o * d_row + b] = u16(0);
            for (int j = 0; j < 16; ++j) qs[o * qs_row + 16 * b + j] = s[2 + j];
            break;
        case GT_Q4_K:
        case GT_Q5_K: {
            // get_scale_min_k4 (quant.hpp:154-162) once, at rest
            const uint8_t* q = s + 4;
            int sc[8], mn[8];
            for (int j = 0; j < 8; ++j) {
                if (j < 4) {
                    sc[j] = q[j] & 63;
                    mn[j] = q[j + 4] & 63;
                } else {
                    sc[j] = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
                    mn[j] = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
                }
            }
            for (int g = 0; g < 4; ++g)
                meta[o * meta_row + 4 * b + g] = (uint32_t)sc[2 * g] | ((uint32_t)sc[2 * g + 1] << 8) |
                                                 ((uint32_t)mn[2 * g] << 16) | ((uint32_t)mn[2 * g + 1] << 24);
            ddp[o * dd_row + b] = (uint32_t)u16(0) | ((uint32_t)u16(2) << 16);
            const int qoff = type == GT_Q5_K ? 48 : 16;
            if (type == GT_Q5_K)
                for (int j = 0; j < 32; ++j) hi[o * hi_row + 32 * b + j] = s[16 + j];
            for (int j = 0; j < 128; ++j) qs[o * qs_row + 128 * b + j] = s[qoff + j];
            break;
        }
        case GT_Q6_K:
            for (int j = 0; j < 128; ++j) qs[o * qs_row + 128 * b + j] = s[j];
            for (int j = 0; j < 64; ++j) hi[o * hi_row + 64 * b + j] = s[128 + j];
            for (int hk = 0; hk < 4; ++hk) {
                const int h = hk >> 1, k = hk & 1;
                uint32_t wv = 0;
                for (int r = 0; r < 4; ++r) wv |= (uint32_t)s[192 + 8 * h + 2 * r + k] << (8 * r);
                meta[o * meta_row + 4 * b + hk] = wv;
            }
            dp[o * d_row + b] = u16(208);
            break;
    }
}

// F32 / F16 / BF16 rows widened to fp32 (the loader dequantises 16-bit
// tensors at load, quant.hpp:6-9).
__global__ void widen_kernel(const uint8_t* __restrict__ src, int type, int64_t n, float* dst) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (type == GT_F32) dst[i] = ((const float*)src)[i];
    else if (type == GT_F16) dst[i] = dev::f16_bits_to_f32(((const uint16_t*)src)[i]);
    else dst[i] = dev::bf16_bits_to_f32(((const uint16_t*)src)[i]);
}

// ---- activation quantisers ------------------------------------------------
// quantize_row_q8_0 (quant_i8.hpp:69-81) of one block of 32 by one warp, a
// value per lane.  d = amax / 127 and 1 / d are IEEE divisions; the scale is
// kept as fp16 (core.hpp:61-79 rounding, f32_to_f16_bits); q = roundf(x * id).
// `packed` (optional) receives the reference's 34-byte block.
__device__ __forceinline__ void quant_block_q8_0(float v, int lane, int8_t* qs, float* d, uint8_t* packed) {
    const float amax = dev::warp_max(fabsf(v));
    const float dd = amax / 127.f;
    const float id = dd != 0.f ? 1.f / dd : 0.f;
    const uint16_t h = dev::f32_to_f16_bits(dd);
    const int8_t q = (int8_t)roundf(v * id);
    qs[lane] = q;
    if (lane == 0) *d = dev::f16_bits_to_f32(h);
    if (packed) {
        packed[2 + lane] = (uint8_t)q;
        if (lane < 2) packed[lane] = (uint8_t)(h >> (8 * lane));
    }
}

// ggml's nearest_int (quant_i8.hpp:30-36) as the reference build evaluates
// it: the product and the 1.5 * 2^23 bias in one fused multiply-add (its
// release flags contract `iscale * x + bias`), i.e. the exact product rounded
// to nearest even.
__device__ __forceinline__ int nearest_int_fma(float iscale, float x) {
    const float s = __fmaf_rn(iscale, x, 12582912.f);
    return (__float_as_int(s) & 0x007fffff) - 0x00400000;
}

// quantize_row_q8_K (quant_i8.hpp:38-67) of one block of 256 by one warp,
// eight consecutive values per lane.  The value of largest magnitude is the
// first one on ties (strict > in index order); iscale = -127 / max; q =
// min(127, nearest(iscale * x)); d = 1 / iscale; bsums over 16-value groups.
__device__ __forceinline__ void quant_block_q8_k(float4 x0, float4 x1, int lane, int8_t* qs, float* d, int16_t* bsums,
                                                 uint8_t* packed) {
    const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    float amax = 0.f, mx = 0.f;
    int idx = 1 << 30;
    for (int i = 0; i < 8; ++i) {
        const float ax = fabsf(v[i]);
        if (ax > amax) {
            amax = ax;
            mx = v[i];
            idx = 8 * lane + i;
        }
    }
    for (int s = 16; s; s >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, s);
        const float om = __shfl_xor_sync(0xffffffffu, mx, s);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, s);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            mx = om;
            idx = oi;
        }
    }
    int8_t q[8];
    float dd = 0.f;
    if (amax != 0.f) {
        const float iscale = -127.f / mx;
        for (int i = 0; i < 8; ++i) {
            const int t = nearest_int_fma(iscale, v[i]);
            q[i] = (int8_t)(t < 127 ? t : 127);
        }
        dd = 1.f / iscale;
    } else {
        for (int i = 0; i < 8; ++i) q[i] = 0;
    }
    int sum = 0;
    for (int i = 0; i < 8; ++i) sum += q[i];
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    uint32_t lo = 0, hi = 0;
    for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(uint8_t)q[i] << (8 * i);
        hi |= (uint32_t)(uint8_t)q[4 + i] << (8 * i);
    }
    reinterpret_cast<uint2*>(qs)[lane] = make_uint2(lo, hi);
    if (lane == 0) *d = dd;
    if (!(lane & 1)) bsums[lane >> 1] = (int16_t)sum;
    if (packed) {
        for (int i = 0; i < 8; ++i) packed[4 + 8 * lane + i] = (uint8_t)q[i];
        if (lane < 4) packed[lane] = (uint8_t)(__float_as_uint(dd) >> (8 * lane));
        if (!(lane & 1)) {
            packed[260 + lane] = (uint8_t)(sum & 0xFF);
            packed[261 + lane] = (uint8_t)((sum >> 8) & 0xFF);
        }
    }
}

// Activation rows quantised to global planes: a warp per block.
__global__ void act_q8_0_kernel(const float* __restrict__ x, int64_t blocks, ActPlanes a, uint8_t* packed) {
    const int lane = threadIdx.x & 31;
    const int64_t w0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int64_t b = w0; b < blocks; b += nw)
        quant_block_q8_0(x[b * 32 + lane], lane, a.qs + b * 32, a.d + b, packed ? packed + b * 34 : nullptr);
}

__global__ void act_q8_k_kernel(const float* __restrict__ x, int64_t blocks, ActPlanes a, uint8_t* packed) {
    const int lane = threadIdx.x & 31;
    const int64_t w0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int64_t b = w0; b < blocks; b += nw) {
        const float4* xp = reinterpret_cast<const float4*>(x + b * 256 + 8 * lane);
        quant_block_q8_k(xp[0], xp[1], lane, a.qs + b * 256, a.d + b, a.bsums + b * 16,
                         packed ? packed + b * 292 : nullptr);
    }
}

// ---- the products ---------------------------------------------------------
struct MvArgs {
    Planes w;
    int64_t in, out;
    int rows;               // activation rows in this launch (<= the kernel's T)
    const int8_t* aq;       // integer path: quants [rows][in]
    const float* ad;        //               block scales [rows][in/block]
    const int16_t* ab;      //               Q8_K 16-value sums [rows][in/16]
    const float* x;         // fp32 path: activations [rows][in]
    float* y;               // [rows][out]
};

__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }
__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint4 ld16_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float h2f(uint32_t bits) { return dev::f16_bits_to_f32(bits & 0xFFFF); }

// Chunks: the unit one lane takes per step.  Q8_0 16 values (16 B), Q4_0 a
// block of 32 (16 B of nibbles), Q4_K/Q5_K 32 values (16 B of nibbles: 16 of
// sub-block 2g, 16 of 2g+1), Q6_K 64 values (16 B from each half of the low
// plane and 16 B of high pairs), F32 4 values.
template <int TYPE>
__host__ __device__ constexpr int chunk_values() {
    return TYPE == GT_Q8_0 ? 16 : TYPE == GT_Q6_K ? 64 : TYPE == GT_F32 ? 4 : 32;
}

template <int TYPE>
struct WChunk {
    uint4 q, q2, h;
    uint32_t m, d;  // the lane's scale word and block scale(s)
};

// One output row's plane pointers (64-bit arithmetic once per row; the
// chunk offsets inside a row are 32-bit).
struct RowPtr {
    const uint8_t* qs;
    const uint8_t* hi;
    const uint32_t* meta;
    const uint16_t* d;
    const uint32_t* dd;
};

__device__ __forceinline__ RowPtr row_ptr(const Planes& P, int64_t o) {
    return {P.qs + o * P.qs_row, P.hi + o * P.hi_row, P.meta + o * P.meta_row, P.d + o * P.d_row, P.dd + o * P.dd_row};
}

template <int TYPE>
__device__ __forceinline__ WChunk<TYPE> load_chunk(const RowPtr& r, int c) {
    WChunk<TYPE> w;
    if constexpr (TYPE == GT_Q8_0 || TYPE == GT_Q4_0) {
        w.q = ld16_stream(r.qs + 16 * c);
        w.d = r.d[TYPE == GT_Q8_0 ? (c >> 1) : c];
    } else if constexpr (TYPE == GT_Q4_K || TYPE == GT_Q5_K) {
        w.q = ld16_stream(r.qs + 16 * c);
        w.m = r.meta[4 * (c >> 3) + ((c >> 1) & 3)];
        w.d = r.dd[c >> 3];
        if constexpr (TYPE == GT_Q5_K) w.h = ld16_stream(r.hi + 32 * (c >> 3) + 16 * (c & 1));
    } else if constexpr (TYPE == GT_Q6_K) {
        const int sb = c >> 2, h = (c >> 1) & 1, k = c & 1;
        const uint8_t* ql = r.qs + 128 * sb + 64 * h + 16 * k;
        w.q = ld16_stream(ql);
        w.q2 = ld16_stream(ql + 32);
        w.h = ld16_stream(r.hi + 64 * sb + 32 * h + 16 * k);
        w.m = r.meta[4 * sb + (c & 3)];
        w.d = r.d[sb];
    } else {
        w.q = ld16_stream(r.qs + 16 * c);
    }
    return w;
}

__device__ __forceinline__ int dot16(const uint32_t (&wq)[4], const uint4& a) {
    int s = dp4(wq[0], a.x, 0);
    s = dp4(wq[1], a.y, s);
    s = dp4(wq[2], a.z, s);
    return dp4(wq[3], a.w, s);
}

// Integer path: the chunk's exact block sums against each activation row,
// scaled in fp32 as the reference's vec_dot_* does per block.
template <int TYPE, int T>
__device__ __forceinline__ void i8_chunk(const WChunk<TYPE>& w, int c, const MvArgs& a, float (&acc)[T]) {
    const int in = (int)a.in;
    if constexpr (TYPE == GT_Q8_0) {
        const uint32_t wq[4] = {w.q.x, w.q.y, w.q.z, w.q.w};
        const float dw = h2f(w.d);
#pragma unroll
        for (int t = 0; t < T; ++t) {
            if (t >= a.rows) break;
            const int s = dot16(wq, ld16(a.aq + t * in + 16 * c));
            acc[t] += (float)s * (dw * a.ad[t * (in >> 5) + (c >> 1)]);
        }
    } else if constexpr (TYPE == GT_Q4_0) {
        const uint32_t lo[4] = {__vsub4(w.q.x & 0x0F0F0F0Fu, 0x08080808u), __vsub4(w.q.y & 0x0F0F0F0Fu, 0x08080808u),
                                __vsub4(w.q.z & 0x0F0F0F0Fu, 0x08080808u), __vsub4(w.q.w & 0x0F0F0F0Fu, 0x08080808u)};
        const uint32_t hi[4] = {__vsub4((w.q.x >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                __vsub4((w.q.y >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                __vsub4((w.q.z >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                __vsub4((w.q.w >> 4) & 0x0F0F0F0Fu, 0x08080808u)};
        const float dw = h2f(w.d);
#pragma unroll
        for (int t = 0; t < T; ++t) {
            if (t >= a.rows) break;
            const int8_t* aq = a.aq + t * in + 32 * c;
            const int s = dot16(lo, ld16(aq)) + dot16(hi, ld16(aq + 16));
            acc[t] += (float)s * dw * a.ad[t * (in >> 5) + c];
        }
    } else if constexpr (TYPE == GT_Q4_K) {
        const int sb = c >> 3;
        const int g = (c >> 1) & 3, h = c & 1;
        const int e0 = 256 * sb + 64 * g + 16 * h;
        const int sc1 = w.m & 0xFF, sc2 = (w.m >> 8) & 0xFF, m1 = (w.m >> 16) & 0xFF, m2 = w.m >> 24;
        const float dd = h2f(w.d), dm = h2f(w.d >> 16);
        const uint32_t lo[4] = {w.q.x & 0x0F0F0F0Fu, w.q.y & 0x0F0F0F0Fu, w.q.z & 0x0F0F0F0Fu, w.q.w & 0x0F0F0F0Fu};
        const uint32_t hi[4] = {(w.q.x >> 4) & 0x0F0F0F0Fu, (w.q.y >> 4) & 0x0F0F0F0Fu, (w.q.z >> 4) & 0x0F0F0F0Fu,
                                (w.q.w >> 4) & 0x0F0F0F0Fu};
#pragma unroll
        for (int t = 0; t < T; ++t) {
            if (t >= a.rows) break;
            const int8_t* aq = a.aq + t * in + e0;
            const int isum = sc1 * dot16(lo, ld16(aq)) + sc2 * dot16(hi, ld16(aq + 32));
            const int16_t* bs = a.ab + t * (in >> 4) + (e0 >> 4);
            const int msum = m1 * bs[0] + m2 * bs[2];
            const float dx = a.ad[t * (in >> 8) + sb];
            acc[t] += (dd * dx) * (float)isum - (dm * dx) * (float)msum;
        }
    } else if constexpr (TYPE == GT_Q6_K) {
        const int sb = c >> 2;
        const int h = (c >> 1) & 1, k = c & 1;
        const uint32_t qa[4] = {w.q.x, w.q.y, w.q.z, w.q.w}, qb[4] = {w.q2.x, w.q2.y, w.q2.z, w.q2.w};
        const uint32_t qh[4] = {w.h.x, w.h.y, w.h.z, w.h.w};
        uint32_t u[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            u[0][i] = (qa[i] & 0x0F0F0F0Fu) | ((qh[i] << 4) & 0x30303030u);
            u[1][i] = (qb[i] & 0x0F0F0F0Fu) | ((qh[i] << 2) & 0x30303030u);
            u[2][i] = ((qa[i] >> 4) & 0x0F0F0F0Fu) | (qh[i] & 0x30303030u);
            u[3][i] = ((qb[i] >> 4) & 0x0F0F0F0Fu) | ((qh[i] >> 2) & 0x30303030u);
        }
        int sc[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) sc[r] = (int)(int8_t)((w.m >> (8 * r)) & 0xFF);
        const float dw = h2f(w.d);
        const int e0 = 256 * sb + 128 * h + 16 * k;
#pragma unroll
        for (int t = 0; t < T; ++t) {
            if (t >= a.rows) break;
            const int8_t* aq = a.aq + t * in + e0;
            const int16_t* bs = a.ab + t * (in >> 4) + (e0 >> 4);
            int isum = 0;
#pragma unroll
            for (int r = 0; r < 4; ++r) isum += sc[r] * (dot16(u[r], ld16(aq + 32 * r)) - 32 * bs[2 * r]);
            acc[t] += (dw * a.ad[t * (in >> 8) + sb]) * (float)isum;
        }
    }
}

__device__ __forceinline__ float4 ldx4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// The chunk's values dequantised in registers with the dequant_to_f32
// arithmetic (quant.hpp:291-400; every product there is exact in fp32 except
// Q6_K's (d * scale) * q, which is evaluated in that order).  Returns the
// element index of v[0]; chunk_off gives the others.
template <int TYPE>
__device__ __forceinline__ int dequant_chunk(const WChunk<TYPE>& w, int c, float (&v)[chunk_values<TYPE>()]) {
    int e0 = c * chunk_values<TYPE>();
    if constexpr (TYPE == GT_F32) {
        v[0] = __uint_as_float(w.q.x), v[1] = __uint_as_float(w.q.y), v[2] = __uint_as_float(w.q.z);
        v[3] = __uint_as_float(w.q.w);
    } else if constexpr (TYPE == GT_Q8_0) {
        const uint32_t q[4] = {w.q.x, w.q.y, w.q.z, w.q.w};
        const float dw = h2f(w.d);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = dw * (float)(int8_t)((q[i >> 2] >> (8 * (i & 3))) & 0xFF);
    } else if constexpr (TYPE == GT_Q4_0) {
        const uint32_t q[4] = {w.q.x, w.q.y, w.q.z, w.q.w};
        const float dw = h2f(w.d);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int b = (q[i >> 2] >> (8 * (i & 3))) & 0xFF;
            v[i] = dw * (float)((b & 0xF) - 8);
            v[i + 16] = dw * (float)((b >> 4) - 8);
        }
    } else if constexpr (TYPE == GT_Q4_K || TYPE == GT_Q5_K) {
        const int sb = c >> 3;
        const int g = (c >> 1) & 3, h = c & 1;
        e0 = 256 * sb + 64 * g + 16 * h;
        const int sc1 = w.m & 0xFF, sc2 = (w.m >> 8) & 0xFF, m1 = (w.m >> 16) & 0xFF, m2 = w.m >> 24;
        const float dd = h2f(w.d), dm = h2f(w.d >> 16);
        const float d1 = dd * (float)sc1, f1 = dm * (float)m1, d2 = dd * (float)sc2, f2 = dm * (float)m2;
        const uint32_t q[4] = {w.q.x, w.q.y, w.q.z, w.q.w};
        const uint32_t hb[4] = {w.h.x, w.h.y, w.h.z, w.h.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int b = (q[i >> 2] >> (8 * (i & 3))) & 0xFF;
            int lo = b & 0xF, hi = b >> 4;
            if constexpr (TYPE == GT_Q5_K) {
                const int hbyte = (hb[i >> 2] >> (8 * (i & 3))) & 0xFF;
                lo += ((hbyte >> (2 * g)) & 1) * 16;
                hi += ((hbyte >> (2 * g + 1)) & 1) * 16;
            }
            v[i] = d1 * (float)lo - f1;       // elements e0 + i        (sub-block 2g)
            v[i + 16] = d2 * (float)hi - f2;  // elements e0 + 32 + i   (sub-block 2g+1)
        }
    } else if constexpr (TYPE == GT_Q6_K) {
        const int sb = c >> 2;
        const int h = (c >> 1) & 1, k = c & 1;
        e0 = 256 * sb + 128 * h + 16 * k;
        const uint32_t qa[4] = {w.q.x, w.q.y, w.q.z, w.q.w}, qb[4] = {w.q2.x, w.q2.y, w.q2.z, w.q2.w};
        const uint32_t qh[4] = {w.h.x, w.h.y, w.h.z, w.h.w};
        const float dw = h2f(w.d);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float ds = dw * (float)(int8_t)((w.m >> (8 * r)) & 0xFF);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t lw = (r & 1) ? qb[i >> 2] : qa[i >> 2];
                const int nib = (lw >> (8 * (i & 3) + ((r & 2) ? 4 : 0))) & 0xF;
                const int two = (qh[i >> 2] >> (8 * (i & 3) + 2 * r)) & 3;
                v[16 * r + i] = ds * (float)((nib | (two << 4)) - 32);
            }
        }
    }
    return e0;
}

// Element index of v[i] relative to v[0]: runs of 16 values, the second run of
// a Q4_K/Q5_K chunk 32 values on (sub-block 2g+1), Q6_K's quarters 32 apart;
// Q8_0, Q4_0 and F32 chunks are contiguous.
template <int TYPE>
__host__ __device__ constexpr int chunk_off(int i) {
    return (TYPE == GT_Q4_K || TYPE == GT_Q5_K) ? (i < 16 ? i : 16 + i)
           : TYPE == GT_Q6_K                    ? 32 * (i >> 4) + (i & 15)
                                                : i;
}

// fp32-activation path: dequantised chunk values times each activation row.
template <int TYPE, int T>
__device__ __forceinline__ void f32_chunk(const WChunk<TYPE>& w, int c, const MvArgs& a, float (&acc)[T]) {
    constexpr int NV = chunk_values<TYPE>();
    float v[NV];
    const int e0 = dequant_chunk<TYPE>(w, c, v);
#pragma unroll
    for (int t = 0; t < T; ++t) {
        if (t >= a.rows) break;
        const float* xr = a.x + t * (int)a.in + e0;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i += 4) {
            const float4 xv = ldx4(xr + chunk_off<TYPE>(i));
            s = fmaf(v[i], xv.x, s);
            s = fmaf(v[i + 1], xv.y, s);
            s = fmaf(v[i + 2], xv.z, s);
            s = fmaf(v[i + 3], xv.w, s);
        }
        acc[t] += s;
    }
}

// Persistent product kernel.  Warp w of CTA b takes output rows
// o = b * 8 + w + k * (8 * gridDim.x) and streams each row in groups of 32 * U
// chunks (lane-consecutive 16-byte loads); the group stream runs on across
// the warp's rows with a register double buffer, so the next group's loads
// (of this row or the next) are in flight while the current one is reduced.
// The first group is requested before griddepcontrol.wait: under a
// programmatic launch the weight stream starts while the previous kernel
// finishes.  Up to T activation rows reuse every loaded chunk.  With FUSE the
// CTA quantises its activation rows into shared memory itself (no separate
// quantiser launch); otherwise they come quantised from global planes.
constexpr int kMvWarps = 8;

template <int TYPE, int T, bool I8>
__host__ __device__ constexpr int mv_unroll() {
    return (T >= 8 || (!I8 && TYPE == GT_Q6_K && T > 1)) ? 1 : (T >= 4 || TYPE == GT_Q6_K || TYPE == GT_Q5_K) ? 2 : 4;
}

template <int TYPE>
__host__ __device__ constexpr int act_block() {
    return (TYPE == GT_Q4_K || TYPE == GT_Q6_K) ? 256 : 32;
}

__host__ __device__ constexpr int64_t align16(int64_t v) { return (v + 15) & ~int64_t(15); }

// Shared-memory bytes of `rows` quantised activation rows of `in` values.
template <int TYPE>
__host__ __device__ constexpr int64_t fused_act_bytes(int rows, int64_t in) {
    return align16(rows * in) + align16(4 * rows * (in / act_block<TYPE>())) +
           (act_block<TYPE>() == 256 ? align16(2 * rows * (in / 16)) : 0);
}

template <int TYPE, int T, bool I8, bool FUSE>
__global__ void __launch_bounds__(kMvWarps * 32, (TYPE == GT_Q6_K || TYPE == GT_Q5_K || T > 1) ? 2 : 3)
    mv_kernel(MvArgs a) {
    constexpr int U = mv_unroll<TYPE, T, I8>();
    extern __shared__ __align__(16) uint8_t act_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = (int)(a.in / chunk_values<TYPE>());
    const int G = (nch + 32 * U - 1) / (32 * U);
    const int64_t stride = (int64_t)gridDim.x * kMvWarps;
    const int64_t o0 = (int64_t)blockIdx.x * kMvWarps + warp;
    const int nrows = o0 < a.out ? (int)((a.out - o0 + stride - 1) / stride) : 0;
    WChunk<TYPE> w[U], wn[U];
    auto load_group = [&](int row, int grp, WChunk<TYPE>(&dst)[U]) {
        const RowPtr rp = row_ptr(a.w, o0 + row * stride);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = grp * (32 * U) + lane + 32 * u;
            if (c < nch) dst[u] = load_chunk<TYPE>(rp, c);
        }
    };
    if (nrows > 0) load_group(0, 0, w);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the next kernel may be scheduled as this one's CTAs retire; it still
    // waits for all of this grid before reading what it wrote
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    MvArgs b = a;
    if constexpr (FUSE) {
        constexpr int BL = act_block<TYPE>();
        int8_t* qs = (int8_t*)act_smem;
        float* d = (float*)(act_smem + align16(T * a.in));
        int16_t* bs = (int16_t*)(act_smem + align16(T * a.in) + align16(4 * T * (a.in / BL)));
        // each warp takes NB consecutive blocks per step with all their loads
        // issued before the first reduction (the loads are L2 round trips)
        const int blocks = (int)(a.rows * (a.in / BL));
        constexpr int NB = BL == 256 ? 4 : 8;
        for (int b0 = warp * NB; b0 < blocks; b0 += kMvWarps * NB) {
            if constexpr (BL == 256) {
                float4 xv[NB][2];
#pragma unroll
                for (int k = 0; k < NB; ++k)
                    if (b0 + k < blocks) {
                        const float4* xp = reinterpret_cast<const float4*>(a.x + (int64_t)(b0 + k) * 256 + 8 * lane);
                        xv[k][0] = xp[0], xv[k][1] = xp[1];
                    }
#pragma unroll
                for (int k = 0; k < NB; ++k)
                    if (b0 + k < blocks)
                        quant_block_q8_k(xv[k][0], xv[k][1], lane, qs + (b0 + k) * 256, d + b0 + k, bs + (b0 + k) * 16,
                                         nullptr);
            } else {
                float xv[NB];
#pragma unroll
                for (int k = 0; k < NB; ++k)
                    if (b0 + k < blocks) xv[k] = a.x[(int64_t)(b0 + k) * 32 + lane];
#pragma unroll
                for (int k = 0; k < NB; ++k)
                    if (b0 + k < blocks) quant_block_q8_0(xv[k], lane, qs + (b0 + k) * 32, d + b0 + k, nullptr);
            }
        }
        __syncthreads();
        b.aq = qs, b.ad = d, b.ab = bs;
    }
    float acc[T];
#pragma unroll
    for (int t = 0; t < T; ++t) acc[t] = 0.f;
    int row = 0, grp = 0;
    while (row < nrows) {
        int nrow = row, ngrp = grp + 1;
        if (ngrp == G) ngrp = 0, ++nrow;
        if (nrow < nrows) load_group(nrow, ngrp, wn);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = grp * (32 * U) + lane + 32 * u;
            if (c < nch) {
                if constexpr (I8) i8_chunk<TYPE, T>(w[u], c, b, acc);
                else f32_chunk<TYPE, T>(w[u], c, b, acc);
            }
        }
        if (ngrp == 0) {
            const int64_t o = o0 + row * stride;
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const float sum = dev::warp_sum(acc[t]);
                if (lane == 0 && t < a.rows) a.y[t * a.out + o] = sum;
                acc[t] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) w[u] = wn[u];
        row = nrow, grp = ngrp;
    }
}

// gather_rows / dequant_row (quant.hpp:469-487): rows dequantised to fp32, one
// thread per chunk, bit-identical to dequant_to_f32.
template <int TYPE>
__global__ void dequant_rows_kernel(Planes P, int64_t in, const int32_t* __restrict__ ids, int64_t n, float* out) {
    const int64_t nch = in / chunk_values<TYPE>();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n * nch) return;
    const int64_t r = i / nch;
    const int c = (int)(i % nch);
    const WChunk<TYPE> w = load_chunk<TYPE>(row_ptr(P, ids[r]), c);
    float v[chunk_values<TYPE>()];
    const int e0 = dequant_chunk<TYPE>(w, c, v);
    float* dst = out + r * in + e0;
#pragma unroll
    for (int j = 0; j < chunk_values<TYPE>(); ++j) dst[chunk_off<TYPE>(j)] = v[j];
}

#define NMG_WEIGHT_TYPES(X) X(GT_F32) X(GT_Q8_0) X(GT_Q4_0) X(GT_Q4_K) X(GT_Q5_K) X(GT_Q6_K)

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int TYPE, int T, bool I8, bool FUSE>
cudaError_t launch_mv_k(const MvArgs& a, cudaStream_t st) {
    auto kern = mv_kernel<TYPE, T, I8, FUSE>;
    const int smem = FUSE ? (int)fused_act_bytes<TYPE>(T, a.in) : 0;
    static int cached_smem = -1, cached_blocks = 0;  // per instantiation
    if (cached_smem != smem) {
        int nb = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kMvWarps * 32, smem);
        if (e != cudaSuccess) return e;
        cached_blocks = nb > 0 ? nb : 1;
        cached_smem = smem;
    }
    const int64_t want = (a.out + kMvWarps - 1) / kMvWarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<int64_t>(want, (int64_t)cached_blocks * sm_count()));
    cfg.blockDim = dim3(kMvWarps * 32);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// Activation rows quantised inside every CTA: Q8_K rows (one warp reduction
// per 256 values) of at most 4096 values, one or two rows.  Longer rows, and
// Q8_0's reduction per 32 values, cost every CTA more up front than the
// separate quantiser launch does.
template <int TYPE>
bool fuse_activations(int rows, int64_t in) {
    return act_block<TYPE>() == 256 && rows <= 2 && in <= 4096;
}

template <int TYPE, int T>
cudaError_t launch_mv_t(const MvArgs& a, bool i8, bool fuse, cudaStream_t st) {
    if constexpr (TYPE == GT_Q8_0 || TYPE == GT_Q4_0 || TYPE == GT_Q4_K || TYPE == GT_Q6_K) {
        if (i8) {
            if constexpr (T <= 2) {
                if (fuse) return launch_mv_k<TYPE, T, true, true>(a, st);
            }
            return launch_mv_k<TYPE, T, true, false>(a, st);
        }
    }
    return launch_mv_k<TYPE, T, false, false>(a, st);
}

template <int TYPE>
cudaError_t launch_mv(const MvArgs& a, bool i8, cudaStream_t st) {
    const bool fuse = i8 && fuse_activations<TYPE>(a.rows, a.in);
    if (a.rows <= 1) return launch_mv_t<TYPE, 1>(a, i8, fuse, st);
    if (a.rows <= 2) return launch_mv_t<TYPE, 2>(a, i8, fuse, st);
    if (a.rows <= 4) return launch_mv_t<TYPE, 4>(a, i8, false, st);
    return launch_mv_t<TYPE, 8>(a, i8, false, st);
}

template <int TYPE>
bool fuses(int64_t rows, int64_t in, bool i8) {
    return i8 && rows <= 2 && fuse_activations<TYPE>((int)rows, in);
}

}  // namespace

// Scratch for one call's quantised activations (a pool of its own, so a
// product never shares bytes with an attention call's split partials).
int weight_act_scratch(int device, size_t bytes, void** ptr);

}  // namespace nmg

using namespace nmg;
using namespace nmg::wq;

namespace {

bool type_known(int t) {
    return t == GT_F32 || t == GT_F16 || t == GT_BF16 || t == GT_Q4_0 || t == GT_Q8_0 || t == GT_Q4_K || t == GT_Q5_K ||
           t == GT_Q6_K;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct DeviceGuard {
    int prev = 0;
    bool ok = false;
    explicit DeviceGuard(int device) {
        ok = cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (ok) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" int nmg_weight_row_bytes(int type, int64_t in, int64_t* bytes) {
    if (!bytes) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_row_bytes: null out");
    if (!type_known(type) && type != GT_Q8_K) return set_error(NMG_INVALID_ARGUMENT, "type_size_bytes: unknown type %d", type);
    const int bl = block_len(type);
    if (in <= 0 || in % bl) return set_error(NMG_INVALID_ARGUMENT, "row of %lld elements is not whole blocks of %d",
                                             (long long)in, bl);
    *bytes = in / bl * block_bytes(type);
    return NMG_OK;
}

extern "C" int nmg_weight_create(int type, int64_t in, int64_t out, const void* data, int data_on_device, int device,
                                 nmg_weight** result) {
    if (!result) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_create: null out");
    *result = nullptr;
    if (!data) return set_error(NMG_INVALID_ARGUMENT, "Weight: null quantised data");
    if (!type_known(type)) return set_error(NMG_INVALID_ARGUMENT, "Weight: type %d is not a weight type", type);
    int64_t src_row = 0;
    if (int rc = nmg_weight_row_bytes(type, in, &src_row)) return rc;
    if (out <= 0) return set_error(NMG_INVALID_ARGUMENT, "Weight: %lld output rows", (long long)out);
    const bool wide = type == GT_F32 || type == GT_F16 || type == GT_BF16;
    if (wide && in % 4) return set_error(NMG_UNSUPPORTED, "Weight: fp32 rows of %lld values (not a multiple of 4)", (long long)in);
    nmg_weight* w = new nmg_weight();
    w->type = wide ? GT_F32 : type;
    w->in = in;
    w->out = out;
    w->device = device;
    // plane sizes (bytes per row)
    int64_t qs_row = 0, hi_row = 0, meta_row = 0, d_row = 0, dd_row = 0;
    switch (w->type) {
        case GT_F32: qs_row = 4 * in; break;
        case GT_Q8_0: qs_row = in, d_row = in / 32; break;
        case GT_Q4_0: qs_row = in / 2, d_row = in / 32; break;
        case GT_Q4_K: qs_row = in / 2, meta_row = in / 64, dd_row = in / 256; break;
        case GT_Q5_K: qs_row = in / 2, hi_row = in / 8, meta_row = in / 64, dd_row = in / 256; break;
        case GT_Q6_K: qs_row = in / 2, hi_row = in / 4, meta_row = in / 64, d_row = in / 256; break;
    }
    const size_t o_qs = 0, o_hi = align256(o_qs + (size_t)(qs_row * out)), o_meta = align256(o_hi + (size_t)(hi_row * out)),
                 o_d = align256(o_meta + (size_t)(4 * meta_row * out)), o_dd = align256(o_d + (size_t)(2 * d_row * out)),
                 total = align256(o_dd + (size_t)(4 * dd_row * out));
    DeviceGuard g(device);
    cudaError_t e = g.ok ? cudaSuccess : cudaErrorInvalidDevice;
    if (e == cudaSuccess) e = cudaMalloc(&w->base, total);
    const uint8_t* src = (const uint8_t*)data;
    void* staged = nullptr;
    if (e == cudaSuccess && !data_on_device) {
        e = cudaMalloc(&staged, (size_t)(src_row * out));
        if (e == cudaSuccess) e = cudaMemcpy(staged, data, (size_t)(src_row * out), cudaMemcpyHostToDevice);
        src = (const uint8_t*)staged;
    }
    if (e == cudaSuccess) {
        uint8_t* b = (uint8_t*)w->base;
        w->p.qs = b + o_qs, w->p.hi = b + o_hi, w->p.meta = (const uint32_t*)(b + o_meta);
        w->p.d = (const uint16_t*)(b + o_d), w->p.dd = (const uint32_t*)(b + o_dd);
        w->p.qs_row = qs_row, w->p.hi_row = hi_row, w->p.meta_row = meta_row, w->p.d_row = d_row, w->p.dd_row = dd_row;
        if (wide) {
            const int64_t n = in * out;
            widen_kernel<<<(unsigned)((n + 255) / 256), 256>>>(src, type, n, (float*)b);
        } else {
            const int64_t nb = in / block_len(type), jobs = nb * out;
            repack_kernel<<<(unsigned)((jobs + 255) / 256), 256>>>(
                src, type, out, nb, src_row, b + o_qs, b + o_hi, (uint32_t*)(b + o_meta), (uint16_t*)(b + o_d),
                (uint32_t*)(b + o_dd), qs_row, hi_row, meta_row, d_row, dd_row);
        }
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    if (staged) cudaFree(staged);
    if (e != cudaSuccess) {
        if (w->base) cudaFree(w->base);
        delete w;
        return set_error(NMG_CUDA_ERROR, "nmg_weight_create: %s", cudaGetErrorString(e));
    }
    *result = w;
    return NMG_OK;
}

extern "C" int nmg_weight_destroy(nmg_weight* w) {
    if (!w) return NMG_OK;
    DeviceGuard g(w->device);
    cudaFree(w->base);
    delete w;
    return NMG_OK;
}

extern "C" int nmg_weight_info(const nmg_weight* w, int* type, int64_t* in, int64_t* out) {
    if (!w) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_info: null weight");
    if (type) *type = w->type;
    if (in) *in = w->in;
    if (out) *out = w->out;
    return NMG_OK;
}

namespace {

// Quantised activation planes for `rows` rows in the product scratch, plus
// `extra` bytes after them (returned in *extra_ptr).
int act_planes(int device, int atype, int64_t rows, int64_t in, ActPlanes* ap, size_t extra = 0,
               void** extra_ptr = nullptr) {
    const int bl = atype == GT_Q8_K ? 256 : 32;
    const size_t qs = align256((size_t)(rows * in)), ds = align256((size_t)(rows * (in / bl) * 4)),
                 bs = atype == GT_Q8_K ? align256((size_t)(rows * (in / 16) * 2)) : 0;
    void* p = nullptr;
    if (int rc = weight_act_scratch(device, qs + ds + bs + extra, &p)) return rc;
    ap->qs = (int8_t*)p;
    ap->d = (float*)((uint8_t*)p + qs);
    ap->bsums = atype == GT_Q8_K ? (int16_t*)((uint8_t*)p + qs + ds) : nullptr;
    if (extra_ptr) *extra_ptr = (uint8_t*)p + qs + ds + bs;
    return NMG_OK;
}

cudaError_t launch_act(int atype, const float* x, int64_t rows, int64_t in, const ActPlanes& ap, uint8_t* packed,
                       cudaStream_t st) {
    const int bl = atype == GT_Q8_K ? 256 : 32;
    const int64_t blocks = rows * (in / bl);
    const unsigned grid = (unsigned)std::min<int64_t>((blocks + 7) / 8, 148 * 16);
    if (atype == GT_Q8_K) act_q8_k_kernel<<<grid, 256, 0, st>>>(x, blocks, ap, packed);
    else act_q8_0_kernel<<<grid, 256, 0, st>>>(x, blocks, ap, packed);
    return cudaGetLastError();
}

}  // namespace

// Weight::matmul (rows >= 1; matvec is rows == 1): y[rows][out] from
// x[rows][in], both device fp32.  act = NMG_ACT_DEFAULT quantises the
// activations (Q8_0 / Q8_K) for the four types with an integer kernel, as the
// reference does unless NM_FP32_ACT is set; NMG_ACT_FP32 is that variable's
// fp32-activation path.
extern "C" int nmg_weight_matmul(const nmg_weight* w, int64_t rows, const float* x, float* y, int act, void* stream) {
    if (!w) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_matmul: null weight");
    if (rows < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_matmul: %lld rows", (long long)rows);
    if (rows == 0) return NMG_OK;
    if (!x || !y) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_matmul: null activations or output");
    if (((uintptr_t)x & 15) != 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_matmul: activations not 16-byte aligned");
    if (act != NMG_ACT_DEFAULT && act != NMG_ACT_FP32) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_matmul: act %d", act);
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(w->device);
    const bool i8 = act == NMG_ACT_DEFAULT && has_i8(w->type);
    MvArgs a = {};
    a.w = w->p;
    a.in = w->in;
    a.out = w->out;
    bool fused = false;
#define NMG_FUSES(T) \
    if (w->type == T) fused = fuses<T>(rows, w->in, i8);
    NMG_WEIGHT_TYPES(NMG_FUSES)
#undef NMG_FUSES
    const bool mm = i8 && rows > 8 && mm_supported(w->type);
    const int splits = mm ? mm_splits(w, rows) : 1;
    void* part = nullptr;
    if (i8 && !fused) {
        const int atype = (w->type == GT_Q4_K || w->type == GT_Q6_K) ? GT_Q8_K : GT_Q8_0;
        ActPlanes ap;
        const size_t extra = splits > 1 ? (size_t)splits * rows * w->out * 4 : 0;
        if (int rc = act_planes(w->device, atype, rows, w->in, &ap, extra, &part)) return rc;
        NMG_CUDA_TRY(launch_act(atype, x, rows, w->in, ap, nullptr, st));
        a.aq = ap.qs, a.ad = ap.d, a.ab = ap.bsums;
    }
    const int bl = (w->type == GT_Q4_K || w->type == GT_Q6_K) ? 256 : 32;
    if (mm) {
        // long batches: int8 tensor-core tiles over the quantised activations
        ActPlanes ap = {const_cast<int8_t*>(a.aq), const_cast<float*>(a.ad), const_cast<int16_t*>(a.ab)};
        cudaError_t e = launch_mm(w, rows, ap, (float*)part, y, st);
        if (e != cudaSuccess) return set_error(NMG_CUDA_ERROR, "nmg_weight_matmul: %s", cudaGetErrorString(e));
        return NMG_OK;
    }
    for (int64_t r0 = 0; r0 < rows; r0 += 8) {
        MvArgs b = a;
        b.rows = (int)std::min<int64_t>(8, rows - r0);
        b.x = x + r0 * w->in;
        b.y = y + r0 * w->out;
        if (i8 && !fused) {
            b.aq = a.aq + r0 * w->in;
            b.ad = a.ad + r0 * (w->in / bl);
            if (a.ab) b.ab = a.ab + r0 * (w->in / 16);
        }
        cudaError_t e = cudaErrorInvalidValue;
#define NMG_MV(T) \
    if (w->type == T) e = launch_mv<T>(b, i8, st);
        NMG_WEIGHT_TYPES(NMG_MV)
#undef NMG_MV
        if (e != cudaSuccess) return set_error(NMG_CUDA_ERROR, "nmg_weight_matmul: %s", cudaGetErrorString(e));
    }
    return NMG_OK;
}

extern "C" int nmg_weight_matvec(const nmg_weight* w, const float* x, float* y, int act, void* stream) {
    return nmg_weight_matmul(w, 1, x, y, act, stream);
}

// gather_rows: `n` rows (indices in host memory, checked against the output
// count) dequantised to fp32 [n][in] on the device.
extern "C" int nmg_weight_gather_rows(const nmg_weight* w, const int32_t* rows, int64_t n, float* out, void* stream) {
    if (!w) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_gather_rows: null weight");
    if (n < 0 || (n && (!rows || !out))) return set_error(NMG_INVALID_ARGUMENT, "nmg_weight_gather_rows: bad arguments");
    if (n == 0) return NMG_OK;
    for (int64_t i = 0; i < n; ++i)
        if (rows[i] < 0 || rows[i] >= w->out)
            return set_error(NMG_OUT_OF_RANGE, "gather_rows: row %d of a %lld-row weight", rows[i], (long long)w->out);
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(w->device);
    void* p = nullptr;
    if (int rc = weight_act_scratch(w->device, (size_t)n * 4, &p)) return rc;
    NMG_CUDA_TRY(cudaMemcpyAsync(p, rows, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    cudaError_t e = cudaErrorInvalidValue;
#define NMG_DQ(T)                                                                                           \
    if (w->type == T) {                                                                                     \
        const int64_t jobs = n * (w->in / chunk_values<T>());                                               \
        dequant_rows_kernel<T><<<(unsigned)((jobs + 255) / 256), 256, 0, st>>>(w->p, w->in, (const int32_t*)p, n, out); \
        e = cudaGetLastError();                                                                             \
    }
    NMG_WEIGHT_TYPES(NMG_DQ)
#undef NMG_DQ
    if (e != cudaSuccess) return set_error(NMG_CUDA_ERROR, "nmg_weight_gather_rows: %s", cudaGetErrorString(e));
    // the index copy reads host memory the caller may reuse once this returns
    NMG_CUDA_TRY(cudaStreamSynchronize(st));
    return NMG_OK;
}

// The activation quantisers alone, writing the reference's packed blocks
// (34-byte block_q8_0 or 292-byte block_q8_K) for `rows` rows of `n` values.
extern "C" int nmg_quantize_activations(int act_type, int64_t rows, int64_t n, const float* x, void* blocks, void* stream) {
    if (act_type != GT_Q8_0 && act_type != GT_Q8_K)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_quantize_activations: type %d is not Q8_0 or Q8_K", act_type);
    const int bl = act_type == GT_Q8_K ? 256 : 32;
    if (rows < 0 || n <= 0 || n % bl) return set_error(NMG_INVALID_ARGUMENT, "nmg_quantize_activations: bad shape");
    if (rows == 0) return NMG_OK;
    if (!x || !blocks || ((uintptr_t)x & 15)) return set_error(NMG_INVALID_ARGUMENT, "nmg_quantize_activations: bad pointers");
    int device = 0;
    NMG_CUDA_TRY(cudaGetDevice(&device));
    ActPlanes ap;
    if (int rc = act_planes(device, act_type, rows, n, &ap)) return rc;
    NMG_CUDA_TRY(launch_act(act_type, x, rows, n, ap, (uint8_t*)blocks, (cudaStream_t)stream));
    return NMG_OK;
}
