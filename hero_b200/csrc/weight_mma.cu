// weight_mma.cu -- Weight<In,Out>::matmul for long activation batches on the
// tensor cores: the reference's integer path (src/quant_i8.hpp:430-514,
// activations quantised once per row, integer block dots, fp32 block scaling)
// as int8 mma.sync tiles.
//
// A CTA computes a 128 (activation rows) x 128 (outputs) tile of y, walking
// the reduction one 256-value superblock per stage (two stages in shared
// memory).  Per stage: the activation quants (A, int8 [rows][256]) arrive by
// cp.async; the weight block (B, [outputs][256]) by cp.async for Q8_0 or
// through registers for the 4- and 6-bit types, unpacked to int8 (Q4_0: q - 8,
// Q4_K: q, Q6_K: q - 32) so one int8 MMA shape serves them all.  Eight warps,
// each a 64 x 32 sub-tile: per 32-value step 4 x 4 m16n8k32 MMAs (Q6_K: two
// m16n8k16 per tile, its scales cover 16 values) whose int32 results are
// exactly the reference's block sums.  Their scaling follows the reference:
//   Q8_0 / Q4_0   acc += sum * (d_w * d_x) per 32-value block (vec_dot :84-127)
//   Q4_K          isum += sc_j * sum_j per sub-block, then per superblock
//                 acc += (d_w d_x) isum - (dmin_w d_x) sum_j m_j bsum_j (:144-187)
//   Q6_K          isum += sc_j * sum_j per 16 values, acc += (d_w d_x) isum (:232-274)
// so the integer parts are exact and only the fp32 order of the block sums
// differs.  The per-block fp32 scaling (one conversion and two multiply-adds
// per output per 32 values) is CUDA-core work beside each MMA, which is why
// this is an mma.sync kernel: a tcgen05 MMA accumulating in tensor memory
// would have to be read back after every 32-value block for the same scaling.
#include <stdint.h>

#include <algorithm>

#include "weight.cuh"

namespace nmg {
namespace wq {
namespace {

constexpr int kBM = 128, kBN = 128, kKS = 256;
constexpr int kMT = 2;                            // m16 tiles per warp: warp tile 32 x 32
constexpr int kThreads = 32 * (kBM / (16 * kMT)) * 4;  // 4 x 4 warps
constexpr int kMetaN = (kBM * 9 + kThreads - 1) / kThreads;
constexpr int kTile = kBM * kKS;                 // bytes of one int8 operand tile
constexpr int kAMeta = kBM * 9 * 4;              // per row: 8 block scales (Q8_0) or d + 8 bsum pairs (Q8_K)
constexpr int kBMeta = kBN * 9 * 4;              // per output: 8 block scales, or packed scales + d (+ dmin)
constexpr int kStage = 2 * kTile + kAMeta + kBMeta;
constexpr int kSmem = 2 * kStage;

struct MmArgs {
    Planes w;
    int64_t in, out, rows;
    const int8_t* aq;
    const float* ad;
    const int16_t* ab;
    float* y;
    int kps;      // superblocks per split (grid.z splits of the reduction)
    float* part;  // with more than one split: partial sums [split][rows][out]
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte chunk cc of row r of a 256-byte-row tile, XOR-swizzled over the
// low three chunk bits so the eight rows an ldmatrix phase reads sit in
// different bank groups.
__device__ __forceinline__ int swz(int r, int cc) { return r * kKS + ((cc ^ (r & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void mma_k32(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_k16(uint32_t a0, uint32_t a1, uint32_t b0, int (&c)[4]) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                 : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ float h2f(uint32_t bits) { return dev::f16_bits_to_f32(bits & 0xFFFF); }

// Paired fp32 arithmetic (Blackwell's two-wide FMA path) on float2 values
// held as 64-bit registers.
__device__ __forceinline__ uint64_t f2(float x, float y) {
    return (uint64_t)__float_as_uint(x) | ((uint64_t)__float_as_uint(y) << 32);
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Two int32 block sums (|s| < 2^22: at most 32 * 127 * 127) as exact fp32
// values: the integer added to the bit pattern of 1.5 * 2^23, then that
// bias subtracted, two full-rate operations in place of a conversion.
__device__ __forceinline__ uint64_t i2f2(int a, int b) {
    const uint64_t biased = (uint64_t)(uint32_t)(a + 0x4B400000) | ((uint64_t)(uint32_t)(b + 0x4B400000) << 32);
    return add2(biased, f2(-12582912.f, -12582912.f));
}

// Weight-side staging of one superblock: what a thread loads into registers
// (one 16-byte unit per task, 4 tasks per thread) before unpacking it.
template <int TYPE>
struct BRegs {
    uint4 q[1024 / kThreads], q2[1024 / kThreads], h[1024 / kThreads];
};

// Number of register-staged 16-byte weight units a thread carries per stage.
template <int TYPE>
__host__ __device__ constexpr int b_tasks() {
    return TYPE == GT_Q6_K ? 512 / kThreads : TYPE == GT_Q8_0 ? 0 : 1024 / kThreads;
}

// Fetch this thread's weight units of superblock kb into registers.
//   Q4_0: unit = block j (16 nibble bytes) of row r      (128 rows x 8)
//   Q4_K: unit = bytes 32g + 16h of the row's 128         (128 rows x 8)
//   Q6_K: unit = (hh, k): ql 64hh + 16k, ql + 32, qh 32hh + 16k   (128 rows x 4)
// Rows past the end load values that unpack to zero.
template <int TYPE>
__device__ __forceinline__ void b_fetch(const MmArgs& a, int64_t o0, int kb, int tid, BRegs<TYPE>& R) {
    const Planes& P = a.w;
#pragma unroll
    for (int i = 0; i < b_tasks<TYPE>(); ++i) {
        const int id = tid + kThreads * i;
        if constexpr (TYPE == GT_Q6_K) {
            const int r = id >> 2, u = id & 3, hh = u >> 1, k = u & 1;
            const int64_t o = o0 + r;
            if (o < a.out) {
                const uint8_t* ql = P.qs + o * P.qs_row + 128 * (int64_t)kb + 64 * hh + 16 * k;
                R.q[i] = *reinterpret_cast<const uint4*>(ql);
                R.q2[i] = *reinterpret_cast<const uint4*>(ql + 32);
                R.h[i] = *reinterpret_cast<const uint4*>(P.hi + o * P.hi_row + 64 * (int64_t)kb + 32 * hh + 16 * k);
            } else {  // nibble 0, high pair 2: 0 | 32 -> 32 - 32 = 0
                R.q[i] = make_uint4(0, 0, 0, 0);
                R.q2[i] = R.q[i];
                R.h[i] = make_uint4(0xAAAAAAAAu, 0xAAAAAAAAu, 0xAAAAAAAAu, 0xAAAAAAAAu);
            }
        } else {
            const int r = id >> 3, u = id & 7;
            const int64_t o = o0 + r;
            bool ok = o < a.out;
            if constexpr (TYPE == GT_Q4_0) ok = ok && (int64_t)kb * 8 + u < a.in / 32;
            constexpr uint32_t zero = TYPE == GT_Q4_0 ? 0x88888888u : 0u;  // unpacks to 0
            R.q[i] = ok ? *reinterpret_cast<const uint4*>(P.qs + o * P.qs_row + 128 * (int64_t)kb + 16 * u)
                        : make_uint4(zero, zero, zero, zero);
        }
    }
}

// Unpack the fetched units to int8 and store them into the B tile.
template <int TYPE>
__device__ __forceinline__ void b_store(uint8_t* Bs, int tid, const BRegs<TYPE>& R) {
#pragma unroll
    for (int i = 0; i < b_tasks<TYPE>(); ++i) {
        const int id = tid + kThreads * i;
        if constexpr (TYPE == GT_Q6_K) {
            const int r = id >> 2, u = id & 3, hh = u >> 1, k = u & 1;
            const uint32_t qa[4] = {R.q[i].x, R.q[i].y, R.q[i].z, R.q[i].w};
            const uint32_t qb[4] = {R.q2[i].x, R.q2[i].y, R.q2[i].z, R.q2[i].w};
            const uint32_t qh[4] = {R.h[i].x, R.h[i].y, R.h[i].z, R.h[i].w};
            uint32_t v[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[0][j] = __vsub4((qa[j] & 0x0F0F0F0Fu) | ((qh[j] << 4) & 0x30303030u), 0x20202020u);
                v[1][j] = __vsub4((qb[j] & 0x0F0F0F0Fu) | ((qh[j] << 2) & 0x30303030u), 0x20202020u);
                v[2][j] = __vsub4(((qa[j] >> 4) & 0x0F0F0F0Fu) | (qh[j] & 0x30303030u), 0x20202020u);
                v[3][j] = __vsub4(((qb[j] >> 4) & 0x0F0F0F0Fu) | ((qh[j] >> 2) & 0x30303030u), 0x20202020u);
            }
            // quarter q of half hh: values 128hh + 32q + 16k + 0..15
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
                *reinterpret_cast<uint4*>(Bs + swz(r, 8 * hh + 2 * qq + k)) =
                    make_uint4(v[qq][0], v[qq][1], v[qq][2], v[qq][3]);
        } else {
            const int r = id >> 3, u = id & 7;
            const uint32_t w[4] = {R.q[i].x, R.q[i].y, R.q[i].z, R.q[i].w};
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                lo[j] = w[j] & 0x0F0F0F0Fu;
                hi[j] = (w[j] >> 4) & 0x0F0F0F0Fu;
                if constexpr (TYPE == GT_Q4_0) lo[j] = __vsub4(lo[j], 0x08080808u), hi[j] = __vsub4(hi[j], 0x08080808u);
            }
            // Q4_0 block u: values 32u + 0..15 (low), 32u + 16..31 (high);
            // Q4_K unit (g, h) = u: values 64g + 16h + 0..15 (low), + 32 (high)
            const int c_lo = TYPE == GT_Q4_0 ? 2 * u : 4 * (u >> 1) + (u & 1);
            const int c_hi = TYPE == GT_Q4_0 ? 2 * u + 1 : c_lo + 2;
            *reinterpret_cast<uint4*>(Bs + swz(r, c_lo)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<uint4*>(Bs + swz(r, c_hi)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
    }
}

// Issue the cp.async copies of superblock kb: the activation tile, and the
// weight tile itself for Q8_0.  Rows or values past the end are zero-filled.
template <int TYPE>
__device__ __forceinline__ void ab_async(const MmArgs& a, int64_t t0, int64_t o0, int kb, int tid, uint8_t* As,
                                         uint8_t* Bs) {
    const int64_t k0 = (int64_t)kb * kKS;
#pragma unroll
    for (int i = 0; i < kTile / 16 / kThreads; ++i) {
        const int id = tid + kThreads * i, r = id >> 4, cc = id & 15;
        const int64_t t = t0 + r;
        const bool ok = t < a.rows && k0 + 16 * cc < a.in;
        cp_async16(smem_addr(As + swz(r, cc)), ok ? (const void*)(a.aq + t * a.in + k0 + 16 * cc) : (const void*)a.aq,
                   ok ? 16 : 0);
        if constexpr (TYPE == GT_Q8_0) {
            const int64_t o = o0 + r;
            const bool okb = o < a.out && k0 + 16 * cc < a.in;
            cp_async16(smem_addr(Bs + swz(r, cc)),
                       okb ? (const void*)(a.w.qs + o * a.w.qs_row + k0 + 16 * cc) : (const void*)a.w.qs, okb ? 16 : 0);
        }
    }
}

// Scales of superblock kb for the stage's metadata: fetched into registers
// ahead of the stage's compute, stored after it.
//   am[r][0..8]: Q8_0 activations: the 8 block scales; Q8_K: d, then the 8
//                sub-block quant sums (bsums pairs) as int bits
//   bm[o][0..8]: Q8_0/Q4_0: the 8 block scales; Q4_K: the 4 scale words, d,
//                dmin; Q6_K: the 4 scale words, d
template <int TYPE>
struct MetaRegs {
    float a[kMetaN], b[kMetaN];
};

template <int TYPE>
__device__ __forceinline__ void meta_fetch(const MmArgs& a, int64_t t0, int64_t o0, int kb, int tid, MetaRegs<TYPE>& M) {
    constexpr bool K = TYPE == GT_Q4_K || TYPE == GT_Q6_K;
#pragma unroll
    for (int i = 0; i < kMetaN; ++i) {
        const int id = tid + kThreads * i;
        float va = 0.f, vb = 0.f;
        if (id < kBM * 9) {
            const int r = id / 9, j = id % 9;
            const int64_t t = t0 + r, o = o0 + r;
            if (t < a.rows) {
                if constexpr (K) {
                    if (j == 0) {
                        va = a.ad[t * (a.in / 256) + kb];
                    } else {
                        const int16_t* bs = a.ab + t * (a.in / 16) + 16 * (int64_t)kb + 2 * (j - 1);
                        va = __int_as_float((int)bs[0] + (int)bs[1]);
                    }
                } else if (j < 8 && (int64_t)kb * 8 + j < a.in / 32) {
                    va = a.ad[t * (a.in / 32) + 8 * (int64_t)kb + j];
                }
            }
            if (o < a.out) {
                if constexpr (TYPE == GT_Q8_0 || TYPE == GT_Q4_0) {
                    if (j < 8 && (int64_t)kb * 8 + j < a.in / 32) vb = h2f(a.w.d[o * a.w.d_row + 8 * (int64_t)kb + j]);
                } else if (j < 4) {
                    vb = __uint_as_float(a.w.meta[o * a.w.meta_row + 4 * (int64_t)kb + j]);
                } else if (TYPE == GT_Q4_K && j < 6) {
                    const uint32_t dd = a.w.dd[o * a.w.dd_row + kb];
                    vb = h2f(j == 4 ? dd : dd >> 16);
                } else if (TYPE == GT_Q6_K && j == 4) {
                    vb = h2f(a.w.d[o * a.w.d_row + kb]);
                }
            }
        }
        M.a[i] = va, M.b[i] = vb;
    }
}

template <int TYPE>
__device__ __forceinline__ void meta_store(int tid, const MetaRegs<TYPE>& M, float* am, float* bm) {
#pragma unroll
    for (int i = 0; i < kMetaN; ++i) {
        const int id = tid + kThreads * i;
        if (id < kBM * 9) am[id] = M.a[i], bm[id] = M.b[i];
    }
}

}  // namespace
}  // namespace wq
}  // namespace nmg

namespace nmg {
namespace wq {
namespace {

template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1) mm_kernel(MmArgs a) {
    constexpr bool K = TYPE == GT_Q4_K || TYPE == GT_Q6_K;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;  // 4 x 4 warps, 32 x 32 each
    const int g = lane >> 2, q = lane & 3;
    const int64_t o0 = (int64_t)blockIdx.x * kBN, t0 = (int64_t)blockIdx.y * kBM;
    const int nk_all = (int)((a.in + kKS - 1) / kKS);
    const int kb0 = blockIdx.z * a.kps;
    const int nk = min(nk_all - kb0, a.kps);  // this split's superblocks kb0 .. kb0 + nk - 1
    auto As = [&](int s) { return smem + s * kStage; };
    auto Bs = [&](int s) { return smem + s * kStage + kTile; };
    auto Am = [&](int s) { return reinterpret_cast<float*>(smem + s * kStage + 2 * kTile); };
    auto Bm = [&](int s) { return reinterpret_cast<float*>(smem + s * kStage + 2 * kTile + kAMeta); };

    // acc2[mt][nt][h]: the pair (cols 2q, 2q+1) of row g + 8h, as float2 bits
    uint64_t acc2[kMT][4][2];
    int isum[kMT][4][4];
#pragma unroll
    for (int i = 0; i < kMT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc2[i][j][0] = acc2[i][j][1] = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) isum[i][j][e] = 0;
        }

    BRegs<TYPE> R;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    ab_async<TYPE>(a, t0, o0, kb0, tid, As(0), Bs(0));
    cp_commit();
    if constexpr (b_tasks<TYPE>() > 0) {
        b_fetch<TYPE>(a, o0, kb0, tid, R);
        b_store<TYPE>(Bs(0), tid, R);
    }
    MetaRegs<TYPE> M;
    meta_fetch<TYPE>(a, t0, o0, kb0, tid, M);
    meta_store<TYPE>(tid, M, Am(0), Bm(0));
    cp_wait_all();
    __syncthreads();

    for (int kb = 0; kb < nk; ++kb) {
        const int s = kb & 1, sn = s ^ 1;
        const bool more = kb + 1 < nk;
        if (more) {
            ab_async<TYPE>(a, t0, o0, kb0 + kb + 1, tid, As(sn), Bs(sn));
            cp_commit();
            if constexpr (b_tasks<TYPE>() > 0) b_fetch<TYPE>(a, o0, kb0 + kb + 1, tid, R);
            if constexpr (K) meta_fetch<TYPE>(a, t0, o0, kb0 + kb + 1, tid, M);  // Q8_0/Q4_0: no registers to spare
        }
        const uint32_t abase = smem_addr(As(s)), bbase = smem_addr(Bs(s));
        const float* am = Am(s);
        const float* bm = Bm(s);
        // one 32-value step; Q4_K overlaps two steps (its epilogue is the
        // lightest, so the registers allow it)
        auto step = [&](int kk) {
            uint32_t af[kMT][4], bf[2][4];
#pragma unroll
            for (int mt = 0; mt < kMT; ++mt) {
                const int r = wm * (16 * kMT) + mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                ldsm4(abase + swz(r, 2 * kk + (lane >> 4)), af[mt]);
            }
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                const int r = wn * 32 + np * 16 + (lane & 7) + 8 * (lane >> 4);
                ldsm4(bbase + swz(r, 2 * kk + ((lane >> 3) & 1)), bf[np]);
            }
            // per-column factors of this 32-value step
            float cs[4][2];
            int sc_lo[4][2], sc_hi[4][2];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float* b = bm + (wn * 32 + nt * 8 + 2 * q + e) * 9;
                    cs[nt][e] = 0.f, sc_lo[nt][e] = 0, sc_hi[nt][e] = 0;
                    if constexpr (TYPE == GT_Q8_0 || TYPE == GT_Q4_0) {
                        cs[nt][e] = b[kk];
                    } else if constexpr (TYPE == GT_Q4_K) {
                        sc_lo[nt][e] = (__float_as_uint(b[kk >> 1]) >> (8 * (kk & 1))) & 0xFF;
                    } else {
                        // 16-value groups 2kk, 2kk+1 -> word 2(gi>>3) + (gi&1), byte (gi>>1)&3
                        const int g0 = 2 * kk, g1 = 2 * kk + 1;
                        sc_lo[nt][e] =
                            (int)(int8_t)((__float_as_uint(b[2 * (g0 >> 3) + (g0 & 1)]) >> (8 * ((g0 >> 1) & 3))) & 0xFF);
                        sc_hi[nt][e] =
                            (int)(int8_t)((__float_as_uint(b[2 * (g1 >> 3) + (g1 & 1)]) >> (8 * ((g1 >> 1) & 3))) & 0xFF);
                    }
                }
#pragma unroll
            for (int mt = 0; mt < kMT; ++mt) {
                float rs[2] = {0.f, 0.f};
                if constexpr (!K) {
                    rs[0] = am[(wm * (16 * kMT) + mt * 16 + g) * 9 + kk];
                    rs[1] = am[(wm * (16 * kMT) + mt * 16 + g + 8) * 9 + kk];
                }
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const uint32_t b0 = bf[nt >> 1][2 * (nt & 1)], b1 = bf[nt >> 1][2 * (nt & 1) + 1];
                    if constexpr (TYPE == GT_Q6_K) {
                        int c0[4], c1[4];
                        mma_k16(af[mt][0], af[mt][1], b0, c0);
                        mma_k16(af[mt][2], af[mt][3], b1, c1);
#pragma unroll
                        for (int e = 0; e < 4; ++e) isum[mt][nt][e] += sc_lo[nt][e & 1] * c0[e] + sc_hi[nt][e & 1] * c1[e];
                    } else {
                        int c[4];
                        mma_k32(af[mt], b0, b1, c);
                        if constexpr (TYPE == GT_Q4_K) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) isum[mt][nt][e] += sc_lo[nt][e & 1] * c[e];
                        } else {
                            const uint64_t csp = f2(cs[nt][0], cs[nt][1]);
#pragma unroll
                            for (int h = 0; h < 2; ++h)
                                acc2[mt][nt][h] = fma2(i2f2(c[2 * h], c[2 * h + 1]), mul2(csp, f2(rs[h], rs[h])),
                                                       acc2[mt][nt][h]);
                        }
                    }
                }
            }
                };
        if constexpr (TYPE == GT_Q4_K) {
#pragma unroll 2
            for (int kk = 0; kk < 8; ++kk) step(kk);
        } else {
#pragma unroll 1
            for (int kk = 0; kk < 8; ++kk) step(kk);
        }
        if constexpr (K) {
            // superblock end: (d_w d_x) isum, minus (dmin_w d_x) sum_j m_j bsum_j
            // for Q4_K; the mins sum is four dp2a per output (int16 pairs of
            // row sums against the column's packed 6-bit mins).
            float cd[4][2], cm[4][2];
            uint32_t mp[4][2][2];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float* b = bm + (wn * 32 + nt * 8 + 2 * q + e) * 9;
                    cd[nt][e] = b[4];
                    if constexpr (TYPE == GT_Q4_K) {
                        cm[nt][e] = b[5];
                        // mins m_0..m_7 sit in bytes 2 and 3 of words 0..3
                        const uint32_t w0 = __float_as_uint(b[0]), w1 = __float_as_uint(b[1]);
                        const uint32_t w2 = __float_as_uint(b[2]), w3 = __float_as_uint(b[3]);
                        mp[nt][e][0] = __byte_perm(w0, w1, 0x7632);
                        mp[nt][e][1] = __byte_perm(w2, w3, 0x7632);
                    }
                }
#pragma unroll
            for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const float* ar = am + (wm * (16 * kMT) + mt * 16 + g + 8 * hf) * 9;
                    const float dx = ar[0];
                    uint32_t bp[4] = {0, 0, 0, 0};
                    if constexpr (TYPE == GT_Q4_K) {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            bp[j] = (uint32_t)(__float_as_int(ar[1 + 2 * j]) & 0xFFFF) |
                                    ((uint32_t)__float_as_int(ar[2 + 2 * j]) << 16);
                    }
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) {
                        float v[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int idx = 2 * hf + e;
                            v[e] = (cd[nt][e] * dx) * (float)isum[mt][nt][idx];  // |isum| may pass 2^22
                            if constexpr (TYPE == GT_Q4_K) {
                                int msum = __dp2a_lo((int)bp[0], (int)mp[nt][e][0], 0);
                                msum = __dp2a_hi((int)bp[1], (int)mp[nt][e][0], msum);
                                msum = __dp2a_lo((int)bp[2], (int)mp[nt][e][1], msum);
                                msum = __dp2a_hi((int)bp[3], (int)mp[nt][e][1], msum);
                                v[e] -= (cm[nt][e] * dx) * (float)msum;
                            }
                            isum[mt][nt][idx] = 0;
                        }
                        acc2[mt][nt][hf] = add2(acc2[mt][nt][hf], f2(v[0], v[1]));
                    }
                }
        }
        if (more) {
            if constexpr (b_tasks<TYPE>() > 0) b_store<TYPE>(Bs(sn), tid, R);
            if constexpr (!K) meta_fetch<TYPE>(a, t0, o0, kb0 + kb + 1, tid, M);
            meta_store<TYPE>(tid, M, Am(sn), Bm(sn));
            cp_wait_all();
        }
        __syncthreads();
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int64_t t = t0 + wm * (16 * kMT) + mt * 16 + g + 8 * hf;
            if (t >= a.rows) continue;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int64_t o = o0 + wn * 32 + nt * 8 + 2 * q;
                float* yp = (a.part ? a.part + (int64_t)blockIdx.z * a.rows * a.out : a.y) + t * a.out + o;
                const uint64_t pr = acc2[mt][nt][hf];
                if (o < a.out) yp[0] = __uint_as_float((uint32_t)pr);
                if (o + 1 < a.out) yp[1] = __uint_as_float((uint32_t)(pr >> 32));
            }
        }
}

// Sum of the split partials, in split order.
__global__ void split_sum_kernel(const float* __restrict__ part, int splits, int64_t n, float* y) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (i >= n) return;
    float s = part[i];
    for (int z = 1; z < splits; ++z) s += part[z * n + i];
    y[i] = s;
}

template <int TYPE>
cudaError_t launch_mm_t(const MmArgs& a, int splits, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(mm_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.out + kBN - 1) / kBN), (unsigned)((a.rows + kBM - 1) / kBM), (unsigned)splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, mm_kernel<TYPE>, a);
    if (e != cudaSuccess || splits == 1) return e;
    const int64_t n = a.rows * a.out;
    cfg.gridDim = dim3((unsigned)((n + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, split_sum_kernel, (const float*)a.part, splits, n, a.y);
}

}  // namespace

bool mm_supported(int type) { return type == GT_Q8_0 || type == GT_Q4_0 || type == GT_Q4_K || type == GT_Q6_K; }

int mm_splits(const nmg_weight* w, int64_t rows) {
    const int64_t tiles = ((w->out + kBN - 1) / kBN) * ((rows + kBM - 1) / kBM);
    const int nk = (int)((w->in + kKS - 1) / kKS);
    if (tiles >= 148 || nk < 4) return 1;
    int s = (int)std::min<int64_t>((2 * 148 + tiles - 1) / tiles, std::min(nk / 2, 16));
    const int kps = (nk + s - 1) / s;
    return (nk + kps - 1) / kps;
}

cudaError_t launch_mm(const nmg_weight* w, int64_t rows, const ActPlanes& act, float* part, float* y, cudaStream_t st) {
    const int splits = mm_splits(w, rows);
    const int nk = (int)((w->in + kKS - 1) / kKS);
    MmArgs a;
    a.kps = (nk + splits - 1) / splits;
    a.part = splits > 1 ? part : nullptr;
    a.w = w->p;
    a.in = w->in;
    a.out = w->out;
    a.rows = rows;
    a.aq = act.qs;
    a.ad = act.d;
    a.ab = act.bsums;
    a.y = y;
    switch (w->type) {
        case GT_Q8_0: return launch_mm_t<GT_Q8_0>(a, splits, st);
        case GT_Q4_0: return launch_mm_t<GT_Q4_0>(a, splits, st);
        case GT_Q4_K: return launch_mm_t<GT_Q4_K>(a, splits, st);
        case GT_Q6_K: return launch_mm_t<GT_Q6_K>(a, splits, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace wq
}  // namespace nmg
