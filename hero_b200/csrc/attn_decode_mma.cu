// attn_decode_mma.cu -- split-KV decode on tensor cores for 16-bit caches (K2, K3).
//
// Decode reads every visible K/V row once and does ~8-16 flops per byte
// (query heads per KV head x 2 x 2), which at HBM speed is more than the CUDA
// cores can issue comfortably; warp-level mma.sync keeps the math off the
// critical path so the kernel is bound by the bytes it streams.
//
// One CTA owns (query row, KV head, 16-head subgroup, key split).  Key tiles
// of 64 positions (64-aligned in slot space, so a tile never straddles the
// ring end) arrive by 2-D TMA with the 128-byte swizzle into a 2-3 stage ring.
// Each of the 4 warps takes 16 keys of a tile:
//   S^T-free form: S[16 heads x 16 keys] = Q[16 x D] K^T   (m16n8k16, A = Q
//                  fragments held in registers, B = K via ldmatrix)
//   online softmax on the accumulator fragments (rows = query heads; heads
//                  beyond the group are zero rows), P -> fp16 A fragments
//   O[16 x D] += P V                                        (B = V via ldmatrix.trans)
// Warps merge through shared memory; rows with several splits merge their
// partials in the last CTA of the row (atomic ticket), as the CUDA-core kernel.
// The reduction is the reference's (nm/src/qwen35.hpp:360-382,
// nm/src/gemma4.hpp:211-235 ...): [scale *] dot(q, k), softmax, sum alpha v.
#include <algorithm>
#include <math.h>
#include <vector>

#include "attn.cuh"

namespace nmg {
namespace {

constexpr int kMmaMaxBatch = 48;  // sequences per launch (tensor maps ride in the parameter block)
constexpr int KT = 64;            // keys per tile (4 warps x 16)

struct MmaSeq {
    int64_t base, slots, lo, hi;  // visible positions [lo, hi]
    int32_t work_first, nsplit, qrow, map;
};

// A Q8_0 cache's int8 quants [hkv][slots][DH] and fp16 scales [hkv][slots][DH / 32].
struct Q8Src {
    const int8_t* k;
    const int8_t* v;
    const uint16_t* ks;  // scale row of slot s of head h: h * sstride + s
    const uint16_t* vs;
    int64_t sstride;
};

struct MmaArgs {
    CUtensorMap tm_k[kMmaMaxBatch];  // K of each distinct cache, (d, hkv*slots)
    CUtensorMap tm_v[kMmaMaxBatch];
    Q8Src q8[kMmaMaxBatch];          // the same caches when they are Q8_0 (tensor maps of the quants at head_dim 128)
    int q_dtype;                     // Q8_0 caches: the query's dtype, staged as fp16
    int hn;                          // 1: heads in the MMA's N (subgroups of 8 heads), 0: in M (16)
    int cl;                          // > 1: every row has cl splits, one thread-block cluster, merged
                                     // through distributed shared memory; 0: ticket merge
    int mode;  // 0: one cache, rows first_query..; 1: table
    int hkv, hq, gtot, zdim;
    int64_t blocks_per_split;
    // mode 0
    int64_t base, slots, rows, first_query, window, floor_pos, newest;
    int32_t max_splits;
    // mode 1
    int nseq;
    MmaSeq seq[kMmaMaxBatch];
    // common
    const void* q;
    void* out;
    int out_dtype;
    float scale_log2;
    float* part;
    int* counters;
    int* err;
};

struct MmaRow {
    int64_t base, slots, lo, hi, work_first, nsplit, qrow, s;
    int map;
};

__device__ __forceinline__ bool mma_row(const MmaArgs& a, int64_t w, MmaRow& r) {
    if (a.mode == 0) {
        const int64_t row = w / a.max_splits;
        r.s = w % a.max_splits;
        const int64_t q = a.first_query + row;
        int64_t lo = a.floor_pos;
        if (a.window > 0 && q - a.window + 1 > lo) lo = q - a.window + 1;
        r.lo = lo;
        r.hi = q < a.newest ? q : a.newest;
        r.base = a.base;
        r.slots = a.slots;
        const int64_t nblk = (r.hi - r.base) / KT - (r.lo - r.base) / KT + 1;
        r.nsplit = (nblk + a.blocks_per_split - 1) / a.blocks_per_split;
        r.work_first = row * a.max_splits;
        r.qrow = row;
        r.map = 0;
        return r.s < r.nsplit;
    }
    int b = 0;
    while (b + 1 < a.nseq && a.seq[b + 1].work_first <= w) ++b;
    const MmaSeq& e = a.seq[b];
    r.base = e.base;
    r.slots = e.slots;
    r.lo = e.lo;
    r.hi = e.hi;
    r.nsplit = e.nsplit;
    r.work_first = e.work_first;
    r.qrow = e.qrow;
    r.map = e.map;
    r.s = w - e.work_first;
    return r.s < r.nsplit;
}

// Q8_0 tiles at head_dim 128 and 256 with the heads in N become MMA fragments
// in registers, straight from the quants (no fp16 copy of the tile).
constexpr bool q8_in_registers(int dh, bool q8, bool hn) { return q8 && hn && (dh == 128 || dh == 256); }

template <int DH, bool Q8 = false, bool Q8R = false, bool HN = false>
struct MmaCfg {
    // head_dim 256: one stage, so several CTAs fit an SM and overlap each
    // other's loads (measured: sliding-window decode 24.8 -> 18.6 us, global
    // 372 -> 362 us against two stages at one CTA per SM; heads in N, whose
    // merge records and staged query need half the rows, fit three: global
    // 336 -> 324 us).  Q8_0 tiles read in registers:
    // two stages, so four CTAs (128 registers each) share an SM (config-5
    // shape: 2.16 ms with four stages at three CTAs per SM, 1.92 ms with two
    // at four, 2.03 ms with five at 96 registers)
    static constexpr int STAGES = Q8R ? 2 : Q8 ? (DH <= 128 ? 4 : 2) : (DH <= 128 ? 3 : 1);
    static constexpr int TILE_BYTES = KT * DH * 2;  // one of K or V as fp16 / bf16
    // Q8_0: a stage holds the raw tile (K quants, V quants, K scales, V scales);
    // the fp16 K and V tiles the MMAs read are one buffer after the stages.
    static constexpr int Q8_QBYTES = KT * DH, Q8_SBYTES = KT * (DH / 32) * 2;
    static constexpr int STAGE_BYTES = Q8 ? 2 * (Q8_QBYTES + Q8_SBYTES) : 2 * TILE_BYTES;
    static constexpr int F16_OFF = STAGES * STAGE_BYTES;  // Q8_0 converted through shared memory only
    static constexpr int LOAD_END = Q8 && !Q8R ? F16_OFF + 2 * TILE_BYTES : STAGES * STAGE_BYTES;
    // Query heads per subgroup: rows of the staged query and of each warp's merge record.
    static constexpr int QR = HN ? 8 : 16;
    // The warp merge ([4][QR][DH + 2] fp32) and, heads in N, the cluster-merge
    // partial ([8][DH + 2] fp32, at XP_OFF) reuse the stage memory, idle by then.
    static constexpr int XP_OFF = 4 * QR * (DH + 2) * 4;
    static constexpr int MERGE_BYTES = (XP_OFF + (HN ? 8 * (DH + 2) * 4 : 0) + 1023) / 1024 * 1024;
    static constexpr int Q_OFF = LOAD_END > MERGE_BYTES ? LOAD_END : MERGE_BYTES;  // QR x DH query rows
    static constexpr int Q_PITCH = DH * 2 + 16;                 // bytes per staged query row
    static constexpr int C_OFF = 0;
    static constexpr int BAR_OFF = Q_OFF + QR * Q_PITCH;
    static constexpr int SMEM = BAR_OFF + 64 + 1024;            // + alignment slack
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(!Q8 || (Q8_QBYTES % 16 == 0 && Q8_SBYTES % 16 == 0 && F16_OFF % 1024 == 0),
                  "bulk copies move 16-byte multiples; the fp16 tiles keep the 128-byte swizzle atoms aligned");
    static_assert(!Q8R || (DH % 128 == 0 && Q8_QBYTES % 1024 == 0 && STAGE_BYTES % 1024 == 0),
                  "the swizzled quant tiles start on 1024-byte boundaries, 128-byte rows per key and box");
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (BF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte chunk `chunk` (8 elements of d) of tile row `key` in
// a K or V tile stored as DH/64 swizzled boxes of [64 keys][128 B].
template <int DH>
__device__ __forceinline__ uint32_t tile_off(int key, int chunk) {
    return (uint32_t)((chunk >> 3) * (KT * 128) + key * 128 + (((chunk & 7) ^ (key & 7)) << 4));
}

// HN (heads in N, groups of at most 8): S^T = K Q^T with the keys in the
// MMA's M rows and the group's heads in its N = 8 columns, O^T += V^T P^T the
// same way, so a group of 8 or fewer wastes at most 7 of 8 columns instead of
// 15 of 16 rows and the O accumulator is half the size.
template <int DH, bool BF16, bool Q8 = false, bool HN = false>
__global__ void __launch_bounds__(128) attn_decode_mma_kernel(const __grid_constant__ MmaArgs a) {
    constexpr bool Q8R = q8_in_registers(DH, Q8, HN);
    using C = MmaCfg<DH, Q8, Q8R, HN>;
    constexpr int ST = C::STAGES;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = (uint64_t*)(smem + C::BAR_OFF);
    float* cs = (float*)(smem + C::C_OFF);
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int h = blockIdx.y, z = blockIdx.z;
    MmaRow r;
    // Under the cluster merge the host gives every row exactly a.cl splits,
    // so every CTA of the grid has work and reaches the cluster barriers.
    if (!mma_row(a, blockIdx.x, r)) return;
    constexpr int GZ = HN ? 8 : 16;  // query heads per subgroup
    const int G = a.gtot - z * GZ < GZ ? a.gtot - z * GZ : GZ;  // valid query heads of this subgroup
    const int qh0 = h * a.gtot + z * GZ;
    const int64_t u_lo = r.lo - r.base, u_hi = r.hi - r.base;
    const int64_t jb = u_lo / KT + r.s * a.blocks_per_split;
    const int64_t je = min(u_lo / KT + (r.s + 1) * a.blocks_per_split, u_hi / KT + 1);
    const int ntiles = (int)(je - jb);
    const CUtensorMap* tmk = &a.tm_k[r.map];
    const CUtensorMap* tmv = &a.tm_v[r.map];

    // One stage (head_dim 256): K and V land on barriers of their own, so the
    // next tile's K loads while this tile's softmax and P.V run.
    constexpr bool SPLIT = ST == 1 && !Q8;
    if (tid == 0) {
        for (int s = 0; s < (SPLIT ? 2 : ST); ++s) dev::mbar_init(&full[s], 1);
        dev::fence_mbar_init();
        if constexpr (!Q8 || Q8R) {
            dev::prefetch_tensormap(tmk);
            dev::prefetch_tensormap(tmv);
        }
    }
    // Launched with programmatic stream serialisation: the set-up above
    // overlaps the previous kernel's tail; q, the cache, the scratch partials
    // and the tickets are touched only after its results are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    auto issue = [&](int t, int st) {
        if (tid == 0) {
            const int64_t u0 = (jb + t) * KT;
            const int32_t row = (int32_t)(h * r.slots + u0 % r.slots);
            dev::fence_proxy_async_smem();
            dev::mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
            if constexpr (Q8) {
                // 64 consecutive slots of the head: contiguous quant rows and scales
                // (the buffers carry 64 spare rows past the last head).
                const Q8Src& q8 = a.q8[r.map];
                unsigned char* dst = smem + st * C::STAGE_BYTES;
                if constexpr (Q8R) {  // quants through the 128-byte swizzle: boxes of 128 dims, a 128-byte row per key
#pragma unroll
                    for (int c = 0; c < DH / 128; ++c) {
                        dev::tma_load_2d(dst + c * KT * 128, tmk, c * 128, row, &full[st]);
                        dev::tma_load_2d(dst + C::Q8_QBYTES + c * KT * 128, tmv, c * 128, row, &full[st]);
                    }
                } else {
                    dev::bulk_g2s(dst, q8.k + (int64_t)row * DH, C::Q8_QBYTES, &full[st]);
                    dev::bulk_g2s(dst + C::Q8_QBYTES, q8.v + (int64_t)row * DH, C::Q8_QBYTES, &full[st]);
                }
                const int64_t srow = (int64_t)h * q8.sstride + u0 % r.slots;
                dev::bulk_g2s(dst + 2 * C::Q8_QBYTES, q8.ks + srow * (DH / 32), C::Q8_SBYTES, &full[st]);
                dev::bulk_g2s(dst + 2 * C::Q8_QBYTES + C::Q8_SBYTES, q8.vs + srow * (DH / 32), C::Q8_SBYTES, &full[st]);
            } else {
#pragma unroll
                for (int c = 0; c < DH / 64; ++c) {
                    dev::tma_load_2d(smem + st * C::STAGE_BYTES + c * KT * 128, tmk, c * 64, row, &full[st]);
                    dev::tma_load_2d(smem + st * C::STAGE_BYTES + C::TILE_BYTES + c * KT * 128, tmv, c * 64, row,
                                     &full[st]);
                }
            }
        }
    };

    auto issue_half = [&](int t, int which) {  // SPLIT: K (0) or V (1) of tile t
        if (tid == 0) {
            const int64_t u0 = (jb + t) * KT;
            const int32_t row = (int32_t)(h * r.slots + u0 % r.slots);
            dev::fence_proxy_async_smem();
            dev::mbar_arrive_expect_tx(&full[which], C::TILE_BYTES);
#pragma unroll
            for (int c = 0; c < DH / 64; ++c)
                dev::tma_load_2d(smem + which * C::TILE_BYTES + c * KT * 128, which ? tmv : tmk, c * 64, row,
                                 &full[which]);
        }
    };

    // The first tiles' copies go out before the query is staged, so their
    // latency overlaps the query loads (thread 0 initialised the barriers).
    for (int t = 0; t < ST - 1 && t < ntiles; ++t) issue(t, t);
    if (SPLIT && ntiles > 0) {
        issue_half(0, 0);
        issue_half(0, 1);
    }
    // Stage the query heads as 16-bit rows (rows past the group are zero).
    for (int i = tid; i < C::QR * (DH / 8); i += 128) {
        const int g = i / (DH / 8), c8 = i % (DH / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if constexpr (Q8) {  // the query as fp16, from whatever dtype it came in
            if (g < G) {
                const int64_t q0 = (r.qrow * (int64_t)a.hq + qh0 + g) * DH + c8 * 8;
                uint32_t w[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    w[u] = pack_h2(dev::load_as_f32(a.q, a.q_dtype, q0 + 2 * u), dev::load_as_f32(a.q, a.q_dtype, q0 + 2 * u + 1));
                v = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else if (g < G) {
            v = *(const uint4*)((const uint16_t*)a.q + (r.qrow * (int64_t)a.hq + qh0 + g) * DH + c8 * 8);
        }
        *(uint4*)(smem + C::Q_OFF + g * C::Q_PITCH + c8 * 16) = v;
    }
    __syncthreads();

    // Q fragments.  Rows form: A fragments (m16k16 per 16 columns of d), rows
    // g = lane/4 (+8).  HN: B fragments (k16 x n8), head lane/4, dims
    // 2*(lane%4) (+1, +8, +9) -- straight 32-bit reads of the staged rows.
    uint32_t qa[DH / 16][4];
    uint32_t qb[DH / 16][2];
    if constexpr (Q8R) {
        // The K fragments below take each lane's 8 consecutive quants of a
        // 32-value block as MMA columns 2q, 2q+1, 2q+8, 2q+9 of two k16 steps
        // (q = lane % 4): the query's dimensions are permuted to match, one
        // 16-byte read per block.
        const unsigned char* qrow = smem + C::Q_OFF + (lane >> 2) * C::Q_PITCH;
#pragma unroll
        for (int b = 0; b < DH / 32; ++b) {
            const uint4 w = *(const uint4*)(qrow + (32 * b + 8 * (lane & 3)) * 2);
            qb[2 * b][0] = w.x;
            qb[2 * b][1] = w.y;
            qb[2 * b + 1][0] = w.z;
            qb[2 * b + 1][1] = w.w;
        }
    } else if constexpr (HN) {
        const unsigned char* qrow = smem + C::Q_OFF + (lane >> 2) * C::Q_PITCH;
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
            qb[kk][0] = *(const uint32_t*)(qrow + (kk * 16 + 2 * (lane & 3)) * 2);
            qb[kk][1] = *(const uint32_t*)(qrow + (kk * 16 + 8 + 2 * (lane & 3)) * 2);
        }
    } else {
        const uint32_t qbase = dev::smem_u32(smem + C::Q_OFF);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
            // matrices: (rows 0-7, k 0-7), (rows 8-15, k 0-7), (rows 0-7, k 8-15), (rows 8-15, k 8-15)
            const int mrow = (lane & 7) + ((lane >> 3) & 1) * 8;
            const int kc = kk * 2 + (lane >> 4);
            ldsm_x4(qbase + mrow * C::Q_PITCH + kc * 16, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
        }
    }

    // O accumulators: rows form O[16 heads x DH] as DH / 8 n8 tiles; HN
    // O^T[DH x 8 heads] as DH / 16 m16 tiles.
    constexpr int NO = HN ? DH / 16 : DH / 8;
    float o[NO][4];
#pragma unroll
    for (int n = 0; n < NO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    // rows form: rows lane/4 and lane/4 + 8; HN: heads 2*(lane%4) and 2*(lane%4) + 1
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

    bool aborted = false;
    for (int t = 0; t < ntiles; ++t) {
        const int st = t % ST;
        if (!SPLIT && t + ST - 1 < ntiles) issue(t + ST - 1, (t + ST - 1) % ST);
        const bool ok = dev::mbar_wait(&full[st], SPLIT ? (t & 1) : ((t / ST) & 1), a.err);
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        uint32_t kbase = dev::smem_u32(smem + st * C::STAGE_BYTES);
        if constexpr (Q8 && !Q8R) {
            // scale * quant of every K and V value of the tile, as fp16 into the
            // swizzled layout the MMA loop reads; 8 values (one 16-byte chunk)
            // at a time, consecutive threads on consecutive chunks of a row.
            // A quant q becomes the fp16 1152 + q by placing q ^ 0x80 under
            // the exponent byte 0x64 (exact), the bias comes off exactly, and
            // the multiply by the fp16 scale rounds the exact product once.
            const unsigned char* raw = smem + st * C::STAGE_BYTES;
            unsigned char* f16 = smem + C::F16_OFF;
            const __half2 bias = __float2half2_rn(1152.f);
#pragma unroll 4
            for (int i = tid; i < 2 * KT * (DH / 8); i += 128) {
                const int mat = i / (KT * (DH / 8)), rem = i % (KT * (DH / 8));
                const int key = rem / (DH / 8), c8 = rem % (DH / 8);
                const uint2 q = *(const uint2*)(raw + mat * C::Q8_QBYTES + key * DH + c8 * 8);
                const uint16_t sb = *(const uint16_t*)(raw + 2 * C::Q8_QBYTES + mat * C::Q8_SBYTES +
                                                       (key * (DH / 32) + c8 / 4) * 2);
                const __half2 sc = __halves2half2(__ushort_as_half(sb), __ushort_as_half(sb));
                const uint32_t qw[2] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u};
                uint32_t w[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t biased = __byte_perm(qw[u >> 1], 0x64646464u, (u & 1) ? 0x4342u : 0x4140u);
                    const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&biased), bias), sc);
                    w[u] = *reinterpret_cast<const uint32_t*>(&v);
                }
                *(uint4*)(f16 + mat * C::TILE_BYTES + tile_off<DH>(key, c8)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            __syncthreads();
            kbase = dev::smem_u32(f16);
        }
        const uint32_t vbase = kbase + C::TILE_BYTES;
        const int key0 = wid * 16;  // this warp's keys within the tile

        float st4[4] = {0.f, 0.f, 0.f, 0.f};  // HN: S^T[16 keys x 8 heads]
        [[maybe_unused]] const __half2 q8_bias = __float2half2_rn(1152.f);
        if constexpr (Q8R) {
            // A = K[16 keys x 16 dims] from the quants: lane (g, q) reads 8
            // quants of keys g and g + 8 per 32-value block (one 8-byte load
            // each, conflict-free under the swizzle), turns them into fp16
            // scale * quant exactly as the shared-memory conversion does, and
            // feeds two k16 steps.
            const unsigned char* stg = smem + st * C::STAGE_BYTES;
            const unsigned char* ksc = stg + 2 * C::Q8_QBYTES;
            const int g = lane >> 2, qd = lane & 3, ra = key0 + g;
            uint32_t sa[DH / 64], sb[DH / 64];  // the fp16 scales of keys ra and ra + 8, two per word
#pragma unroll
            for (int i = 0; i < DH / 64; ++i) {
                sa[i] = *(const uint32_t*)(ksc + ra * (DH / 32) * 2 + 4 * i);
                sb[i] = *(const uint32_t*)(ksc + (ra + 8) * (DH / 32) * 2 + 4 * i);
            }
#pragma unroll
            for (int b = 0; b < DH / 32; ++b) {
                // block b: box b / 4 (128 dims), 16-byte chunk 2 (b % 4) + q / 2 of the key's row
                const uint32_t off = (uint32_t)(b >> 2) * (KT * 128) + (uint32_t)ra * 128 +
                                     ((((2 * (b & 3) + (qd >> 1)) ^ (ra & 7))) << 4) + (qd & 1) * 8;
                const uint2 wa = *(const uint2*)(stg + off), wb = *(const uint2*)(stg + off + 8 * 128);
                const uint32_t sel = (b & 1) ? 0x3232u : 0x1010u;
                const uint32_t s2a = __byte_perm(sa[b >> 1], 0, sel);
                const uint32_t s2b = __byte_perm(sb[b >> 1], 0, sel);
                const __half2 sca = *reinterpret_cast<const __half2*>(&s2a);
                const __half2 scb = *reinterpret_cast<const __half2*>(&s2b);
                auto deq = [&](uint32_t x, uint32_t pick, __half2 sc) -> uint32_t {
                    const uint32_t biased = __byte_perm(x, 0x64646464u, pick);
                    const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&biased), q8_bias), sc);
                    return *reinterpret_cast<const uint32_t*>(&v);
                };
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {  // k16 steps 2b and 2b + 1
                    const uint32_t xa = (h2 ? wa.y : wa.x) ^ 0x80808080u, xb = (h2 ? wb.y : wb.x) ^ 0x80808080u;
                    uint32_t ka[4];
                    ka[0] = deq(xa, 0x4140u, sca);  // key g,     columns 2q, 2q+1
                    ka[1] = deq(xb, 0x4140u, scb);  // key g + 8
                    ka[2] = deq(xa, 0x4342u, sca);  // key g,     columns 2q+8, 2q+9
                    ka[3] = deq(xb, 0x4342u, scb);  // key g + 8
                    mma_16816<false>(st4, ka, qb[2 * b + h2][0], qb[2 * b + h2][1]);
                }
            }
        } else if constexpr (HN) {
#pragma unroll
            for (int kk = 0; kk < DH / 16; ++kk) {
                // A = K[16 keys x 16 dims]: (keys 0-7, d lo), (keys 8-15, d lo), (keys 0-7, d hi), (keys 8-15, d hi)
                const int key = key0 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int chunk = kk * 2 + (lane >> 4);
                uint32_t ka[4];
                ldsm_x4(kbase + tile_off<DH>(key, chunk), ka[0], ka[1], ka[2], ka[3]);
                mma_16816<BF16>(st4, ka, qb[kk][0], qb[kk][1]);
            }
        }
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if constexpr (!HN) {
            // S = Q K^T over this warp's 16 keys: two n8 tiles.
    #pragma unroll
            for (int kk = 0; kk < DH / 16; ++kk) {
                // matrices: (keys 0-7, d lo), (keys 0-7, d hi), (keys 8-15, d lo), (keys 8-15, d hi)
                const int key = key0 + (lane & 7) + (lane >> 4) * 8;
                const int chunk = kk * 2 + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kbase + tile_off<DH>(key, chunk), b0, b1, b2, b3);
                mma_16816<BF16>(sc[0], qa[kk], b0, b1);
                mma_16816<BF16>(sc[1], qa[kk], b2, b3);
            }
        }
        if constexpr (SPLIT) {  // every warp is done with K(t): fetch K(t + 1)
            __syncthreads();
            if (t + 1 < ntiles) issue_half(t + 1, 0);
        }
        uint32_t pfrag[4];  // rows form: the P A fragment; HN: [0], [1] the P^T B fragment
        if constexpr (HN) {
            // mask + scale: st4[e] is (key lane/4 (+8 for e >= 2), head 2*(lane%4) + (e & 1))
            const int64_t p_key = r.base + (jb + t) * KT + key0 + (lane >> 2);
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int64_t pos = p_key + (e >> 1) * 8;
                float x = st4[e] * a.scale_log2;
                if (pos < r.lo || pos > r.hi) x = -INFINITY;
                st4[e] = x;
                mx[e & 1] = fmaxf(mx[e & 1], x);
            }
            float alpha[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {  // over the 8 lanes that share the head pair
                mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 4));
                mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 8));
                mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 16));
                const float m_new = fmaxf(m_r[hh], mx[hh]);
                alpha[hh] = (m_new == -INFINITY) ? 1.f : ex2f(m_r[hh] - m_new);
                m_r[hh] = m_new;
            }
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float m = m_r[e & 1];
                p[e] = (m == -INFINITY) ? 0.f : ex2f(st4[e] - m);
            }
            l_r[0] = l_r[0] * alpha[0] + (p[0] + p[2]);
            l_r[1] = l_r[1] * alpha[1] + (p[1] + p[3]);
            // P^T as the B operand (k16 keys x n8 heads): lane L needs head
            // n = L/4 at keys 2q, 2q+1 (+8, +9), q = L%4, which lanes 8q + n/2
            // and 8q + 4 + n/2 hold (the n-th half of their packed pair).
            const uint32_t pk01 = pack_h2(p[0], p[1]), pk23 = pack_h2(p[2], p[3]);
            const int n = lane >> 2, q = lane & 3;
            const int sa = 8 * q + (n >> 1), sb = sa + 4;
            const uint32_t v0 = __shfl_sync(0xffffffffu, pk01, sa), v1 = __shfl_sync(0xffffffffu, pk01, sb);
            const uint32_t v2 = __shfl_sync(0xffffffffu, pk23, sa), v3 = __shfl_sync(0xffffffffu, pk23, sb);
            const uint32_t sel = (n & 1) ? 0x7632u : 0x5410u;
            pfrag[0] = __byte_perm(v0, v1, sel);
            pfrag[1] = __byte_perm(v2, v3, sel);
            pfrag[2] = pfrag[3] = 0u;
#pragma unroll
            for (int dd = 0; dd < NO; ++dd) {  // o[dd][e] is (dim row, head 2*(lane%4) + (e & 1))
                o[dd][0] *= alpha[0];
                o[dd][1] *= alpha[1];
                o[dd][2] *= alpha[0];
                o[dd][3] *= alpha[1];
            }
        }
        if constexpr (!HN) {
            // mask + scale: accumulator element (row, key) with key = 8n + 2*(lane%4) + {0,1}
            const int64_t p_tile = r.base + (jb + t) * KT + key0;
            float mx[2] = {-INFINITY, -INFINITY};
    #pragma unroll
            for (int n = 0; n < 2; ++n)
    #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int64_t pos = p_tile + 8 * n + 2 * (lane & 3) + (e & 1);
                    float x = sc[n][e] * a.scale_log2;
                    if (pos < r.lo || pos > r.hi) x = -INFINITY;
                    sc[n][e] = x;
                    mx[e >> 1] = fmaxf(mx[e >> 1], x);
                }
            float alpha[2];
    #pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
                mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
                const float m_new = fmaxf(m_r[hr], mx[hr]);
                alpha[hr] = (m_new == -INFINITY) ? 1.f : ex2f(m_r[hr] - m_new);  // ex2(-inf) = 0 for the first block
                m_r[hr] = m_new;
            }
            float ps[2] = {0.f, 0.f};
            uint32_t pa[4];
    #pragma unroll
            for (int n = 0; n < 2; ++n) {
                float p[4];
    #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float m = m_r[e >> 1];
                    p[e] = (m == -INFINITY) ? 0.f : ex2f(sc[n][e] - m);
                    ps[e >> 1] += p[e];
                }
                pa[2 * n] = pack_h2(p[0], p[1]);      // row g, keys of n-tile n
                pa[2 * n + 1] = pack_h2(p[2], p[3]);  // row g + 8
            }
            l_r[0] = l_r[0] * alpha[0] + ps[0];
            l_r[1] = l_r[1] * alpha[1] + ps[1];
            // A operand order for m16k16: a0 (g, k0-7) a1 (g+8, k0-7) a2 (g, k8-15) a3 (g+8, k8-15)
            pfrag[0] = pa[0], pfrag[1] = pa[1], pfrag[2] = pa[2], pfrag[3] = pa[3];
    #pragma unroll
            for (int n = 0; n < DH / 8; ++n) {
                o[n][0] *= alpha[0];
                o[n][1] *= alpha[0];
                o[n][2] *= alpha[1];
                o[n][3] *= alpha[1];
            }
        }
        if constexpr (SPLIT) {
            const bool okv = dev::mbar_wait(&full[1], t & 1, a.err);
            if (__syncthreads_or(!okv)) {
                aborted = true;
                break;
            }
        }
        if constexpr (Q8R) {
            // A = V^T[16 dims x 16 keys] from the quants.  Lane (g, q) reads the
            // 4 quants at dims 32p + 4g .. + 3 of keys 2q, 2q+1, 2q+8, 2q+9 (one
            // 32-bit load each, conflict-free under the swizzle): bytes 0 and 1
            // are rows g and g + 8 of dim tile 2p, bytes 2 and 3 those of tile
            // 2p + 1 -- the O^T rows carry that dimension order into the merge.
            const unsigned char* stg = smem + st * C::STAGE_BYTES;
            const unsigned char* vqt = stg + C::Q8_QBYTES;
            const unsigned char* vsc = stg + 2 * C::Q8_QBYTES + C::Q8_SBYTES;
            const int g = lane >> 2, k0 = key0 + 2 * (lane & 3);
            uint32_t s4[4][DH / 64];  // the fp16 scales of keys k0, k0 + 1, k0 + 8, k0 + 9, two per word
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int w2 = 0; w2 < DH / 64; ++w2)
                    s4[i][w2] = *(const uint32_t*)(vsc + (k0 + (i & 1) + 8 * (i >> 1)) * (DH / 32) * 2 + 4 * w2);
#pragma unroll
            for (int p = 0; p < DH / 32; ++p) {
                // dims 32p + 4g: box p / 4 (128 dims), 16-byte chunk 2 (p % 4) + g / 4 of the key's row
                const int c = 2 * (p & 3) + (g >> 2);
                const uint32_t box = (uint32_t)(p >> 2) * (KT * 128);
                const uint32_t o0 = box + (uint32_t)k0 * 128 + ((c ^ (k0 & 7)) << 4) + (g & 3) * 4;
                const uint32_t o1 = box + (uint32_t)(k0 + 1) * 128 + ((c ^ ((k0 + 1) & 7)) << 4) + (g & 3) * 4;
                const uint32_t x0 = *(const uint32_t*)(vqt + o0) ^ 0x80808080u;
                const uint32_t x1 = *(const uint32_t*)(vqt + o1) ^ 0x80808080u;
                const uint32_t x2 = *(const uint32_t*)(vqt + o0 + 8 * 128) ^ 0x80808080u;
                const uint32_t x3 = *(const uint32_t*)(vqt + o1 + 8 * 128) ^ 0x80808080u;
                const uint32_t ssel = (p & 1) ? 0x7632u : 0x5410u;
                const uint32_t s01 = __byte_perm(s4[0][p >> 1], s4[1][p >> 1], ssel);
                const uint32_t s23 = __byte_perm(s4[2][p >> 1], s4[3][p >> 1], ssel);
                const __half2 sc01 = *reinterpret_cast<const __half2*>(&s01);
                const __half2 sc23 = *reinterpret_cast<const __half2*>(&s23);
                auto deq = [&](uint32_t x, uint32_t pick, __half2 sc) -> uint32_t {
                    const uint32_t biased = __byte_perm(x, 0x64646464u, pick);
                    const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&biased), q8_bias), sc);
                    return *reinterpret_cast<const uint32_t*>(&v);
                };
#pragma unroll
                for (int j = 0; j < 2; ++j) {  // dim tiles 2p (bytes 0, 1) and 2p + 1 (bytes 2, 3)
                    // the two keys of a pair side by side: byte i of key k0 next to byte i of key k0 + 1
                    const uint32_t i01 = __byte_perm(x0, x1, j ? 0x7362u : 0x5140u);
                    const uint32_t i23 = __byte_perm(x2, x3, j ? 0x7362u : 0x5140u);
                    uint32_t va[4];
                    va[0] = deq(i01, 0x4140u, sc01);  // row g,     keys 2q, 2q+1
                    va[1] = deq(i01, 0x4342u, sc01);  // row g + 8
                    va[2] = deq(i23, 0x4140u, sc23);  // row g,     keys 2q+8, 2q+9
                    va[3] = deq(i23, 0x4342u, sc23);  // row g + 8
                    mma_16816<false>(o[2 * p + j], va, pfrag[0], pfrag[1]);
                }
            }
        } else if constexpr (HN) {
            // O^T += V^T P^T: per 16 dims one ldmatrix.trans (x4) of V and one MMA.
#pragma unroll
            for (int dd = 0; dd < NO; ++dd) {
                // A = V^T[16 dims x 16 keys]: (d lo, keys 0-7), (d hi, keys 0-7), (d lo, keys 8-15), (d hi, keys 8-15)
                const int key = key0 + (lane & 7) + (lane >> 4) * 8;
                const int chunk = dd * 2 + ((lane >> 3) & 1);
                uint32_t va[4];
                ldsm_x4_t(vbase + tile_off<DH>(key, chunk), va[0], va[1], va[2], va[3]);
                mma_16816<false>(o[dd], va, pfrag[0], pfrag[1]);
            }
        } else {
            // O += P V: per 16 columns of d one ldmatrix.trans (x4) and two MMAs.
    #pragma unroll
            for (int dd = 0; dd < DH / 16; ++dd) {
                // matrices: (keys 0-7, d lo), (keys 8-15, d lo), (keys 0-7, d hi), (keys 8-15, d hi)
                const int key = key0 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int chunk = dd * 2 + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vbase + tile_off<DH>(key, chunk), b0, b1, b2, b3);
                mma_16816<false>(o[2 * dd], pfrag, b0, b1);
                mma_16816<false>(o[2 * dd + 1], pfrag, b2, b3);
            }
        }
        __syncthreads();  // the stage is refilled next iteration
        if (SPLIT && t + 1 < ntiles) issue_half(t + 1, 1);
    }
    if (aborted) {
        if (!a.cl) return;
        // the cluster's other CTAs wait at its barriers: offer an empty partial
#pragma unroll
        for (int n = 0; n < NO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m_r[0] = m_r[1] = -INFINITY;
        l_r[0] = l_r[1] = 0.f;
    }

    // ---- merge the 4 warps: row sums over the lanes that share a row (head),
    // then through shared memory as [head][DH + 2] per warp
    float* cw = cs + wid * C::QR * (DH + 2);
    if constexpr (HN) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            l_r[hh] += __shfl_xor_sync(0xffffffffu, l_r[hh], 4);
            l_r[hh] += __shfl_xor_sync(0xffffffffu, l_r[hh], 8);
            l_r[hh] += __shfl_xor_sync(0xffffffffu, l_r[hh], 16);
        }
        const int h0 = 2 * (lane & 3), d0 = lane >> 2;
#pragma unroll
        for (int dd = 0; dd < NO; ++dd) {
            // dims of rows d0 and d0 + 8 of tile dd (Q8R: 32p + 4 d0 + 2j (+1), dd = 2p + j)
            const int dlo = Q8R ? 32 * (dd >> 1) + 4 * d0 + 2 * (dd & 1) : 16 * dd + d0;
            const int dhi = Q8R ? dlo + 1 : dlo + 8;
            cw[h0 * (DH + 2) + dlo] = o[dd][0];
            cw[(h0 + 1) * (DH + 2) + dlo] = o[dd][1];
            cw[h0 * (DH + 2) + dhi] = o[dd][2];
            cw[(h0 + 1) * (DH + 2) + dhi] = o[dd][3];
        }
        if (d0 == 0) {
            cw[h0 * (DH + 2) + DH] = m_r[0];
            cw[h0 * (DH + 2) + DH + 1] = l_r[0];
            cw[(h0 + 1) * (DH + 2) + DH] = m_r[1];
            cw[(h0 + 1) * (DH + 2) + DH + 1] = l_r[1];
        }
    } else {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
            l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
        }
        const int g0 = lane >> 2;
#pragma unroll
        for (int n = 0; n < NO; ++n) {
            const int c0 = 8 * n + 2 * (lane & 3);
            cw[g0 * (DH + 2) + c0] = o[n][0];
            cw[g0 * (DH + 2) + c0 + 1] = o[n][1];
            cw[(g0 + 8) * (DH + 2) + c0] = o[n][2];
            cw[(g0 + 8) * (DH + 2) + c0 + 1] = o[n][3];
        }
        if ((lane & 3) == 0) {
            cw[g0 * (DH + 2) + DH] = m_r[0];
            cw[g0 * (DH + 2) + DH + 1] = l_r[0];
            cw[(g0 + 8) * (DH + 2) + DH] = m_r[1];
            cw[(g0 + 8) * (DH + 2) + DH + 1] = l_r[1];
        }
    }
    __syncthreads();

    const bool single = r.nsplit == 1;
    const bool clm = a.cl > 1;  // cluster merge
    float* xp = (float*)(smem + C::XP_OFF);  // cluster merge (heads in N): this CTA's partial [G][DH + 2]
    const int64_t cnt_idx = (r.qrow * (int64_t)a.hkv + h) * a.zdim + z;
    float* my_part = a.part + ((((int64_t)blockIdx.x) * a.hkv + h) * a.zdim + z) * (int64_t)(16 * (DH + 2));
    for (int i = tid; i < G * DH; i += 128) {
        const int g = i / DH, d = i % DH;
        float M = -INFINITY;
        for (int w2 = 0; w2 < 4; ++w2) M = fmaxf(M, cs[(w2 * C::QR + g) * (DH + 2) + DH]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w2 = 0; w2 < 4; ++w2) {
                const float* c = cs + (w2 * C::QR + g) * (DH + 2);
                if (c[DH] == -INFINITY) continue;
                const float f = ex2f(c[DH] - M);
                L += c[DH + 1] * f;
                O += c[d] * f;
            }
        }
        if (single) {
            dev::store_from_f32(a.out, a.out_dtype, (r.qrow * (int64_t)a.hq + qh0 + g) * DH + d, O / L);
        } else {
            float* dst = clm ? xp : my_part;
            dst[g * (DH + 2) + d] = O;
            if (d == 0) {
                dst[g * (DH + 2) + DH] = M;
                dst[g * (DH + 2) + DH + 1] = L;
            }
        }
    }
    if (single) return;
    if (clm) {
        // every split's partial is in its CTA's shared memory: CTA s of the
        // cluster combines items [s * share, ...) of the G x DH over the splits
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        uint32_t rank;
        asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
        const int ncl = a.cl, items = G * DH, share = (items + ncl - 1) / ncl;
        const uint32_t xbase = dev::smem_u32(xp);
        for (int i = (int)rank * share + tid; i < min(items, ((int)rank + 1) * share); i += 128) {
            const int g = i / DH, d = i % DH;
            float Ms[8], Ls[8], Os[8], M = -INFINITY;
#pragma unroll
            for (int sp = 0; sp < 8; ++sp) {
                Ms[sp] = -INFINITY, Ls[sp] = 0.f, Os[sp] = 0.f;
                if (sp < ncl) {
                    uint32_t ra;
                    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(xbase), "r"((uint32_t)sp));
                    const uint32_t rg = ra + (uint32_t)(g * (DH + 2)) * 4u;
                    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(Ms[sp]) : "r"(rg + DH * 4) : "memory");
                    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(Ls[sp]) : "r"(rg + (DH + 1) * 4) : "memory");
                    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(Os[sp]) : "r"(rg + d * 4) : "memory");
                    M = fmaxf(M, Ms[sp]);
                }
            }
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int sp = 0; sp < 8; ++sp)
                if (Ms[sp] != -INFINITY) {
                    const float f = ex2f(Ms[sp] - M);
                    L = fmaf(Ls[sp], f, L);
                    O = fmaf(Os[sp], f, O);
                }
            dev::store_from_f32(a.out, a.out_dtype, (r.qrow * (int64_t)a.hq + qh0 + g) * DH + d,
                                L > 0.f ? O / L : 0.f);
        }
        // no CTA leaves while another may still read its partial
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        return;
    }

    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counters[cnt_idx], 1) == (int)r.nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    {
        __shared__ float red[4], wbuf[kMergeChunk];
        const float* first = a.part + (((r.work_first) * a.hkv + h) * a.zdim + z) * (int64_t)(16 * (DH + 2));
        merge_partials<128, DH, true>(first, (int64_t)a.hkv * a.zdim * (16 * (DH + 2)), r.nsplit, G, red, wbuf,
                                      [&](int g, int d, float v) {
                                          dev::store_from_f32(a.out, a.out_dtype,
                                                              (r.qrow * (int64_t)a.hq + qh0 + g) * DH + d, v);
                                      });
    }
    if (tid == 0) a.counters[cnt_idx] = 0;
}

template <int DH, bool BF16, bool Q8, bool HN>
int launch_mma_hn(const MmaArgs& a, dim3 grid, cudaStream_t s) {
    using C = MmaCfg<DH, Q8, q8_in_registers(DH, Q8, HN), HN>;
    auto kern = attn_decode_mma_kernel<DH, BF16, Q8, HN>;
    static std::atomic<uint64_t> attr_set{0};  // one bit per device
    const int st = set_smem_once(kern, C::SMEM, attr_set);
    if (st != NMG_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a.cl > 1) {  // the splits of a row as one cluster
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)a.cl;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    NMG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
    return NMG_OK;
}

template <int DH, bool BF16, bool Q8 = false>
int launch_mma(const MmaArgs& a, dim3 grid, cudaStream_t s) {
    return a.hn ? launch_mma_hn<DH, BF16, Q8, true>(a, grid, s) : launch_mma_hn<DH, BF16, Q8, false>(a, grid, s);
}

int dispatch_mma(const nmg_kv_cache* c, const MmaArgs& a, dim3 grid, cudaStream_t s) {
    const bool bf = c->dtype == NMG_BF16;
    if (c->dtype == NMG_Q8_0) {
        switch (c->dh) {
            case 64: return launch_mma<64, false, true>(a, grid, s);
            case 128: return launch_mma<128, false, true>(a, grid, s);
            case 256: return launch_mma<256, false, true>(a, grid, s);
        }
        return set_error(NMG_UNSUPPORTED, "Q8_0 decode: head_dim %d", c->dh);
    }
    switch (c->dh) {
        case 64: return bf ? launch_mma<64, true>(a, grid, s) : launch_mma<64, false>(a, grid, s);
        case 128: return bf ? launch_mma<128, true>(a, grid, s) : launch_mma<128, false>(a, grid, s);
        case 256: return bf ? launch_mma<256, true>(a, grid, s) : launch_mma<256, false>(a, grid, s);
    }
    return set_error(NMG_UNSUPPORTED, "tensor-core decode: head_dim %d", c->dh);
}

// Groups of at most 8 query heads put the heads in the MMA's N dimension.
int mma_heads_in_n(int gtot) { return gtot <= 8 ? 1 : 0; }

int64_t mma_blocks_per_split(int64_t total_blocks, int dh) {
    // About 6 CTAs per SM of work, at most 128 tiles (8192 keys) per split.
    // Small launches (a sliding window, a short cache) still give each CTA up
    // to 4 tiles while that leaves a CTA per SM (two at head_dim 256, where
    // three CTAs share an SM and a launch of one per SM would leave SMs idle:
    // config-4 window decode 15.8 us at 4 tiles per CTA, 14.7 at 3, 19.6 at 2,
    // which no longer fits one wave): a CTA of
    // one tile pays its load latency with nothing to overlap it and adds a
    // split to merge.
    int64_t b = total_blocks / (148 * 6);
    b = std::max<int64_t>(b, std::min<int64_t>(4, total_blocks / (148 * (dh == 256 ? 2 : 1))));
    return std::max<int64_t>(1, std::min<int64_t>(128, b));
}

int mma_scratch(int device, int64_t work, int hkv, int zdim, int dh, int64_t counter_rows, float** part,
                int** counters) {
    const int64_t part_floats = work * hkv * zdim * 16 * (int64_t)(dh + 2);
    const int64_t cnt_ints = counter_rows * hkv * zdim;
    void* tickets = nullptr;
    void* base = nullptr;
    int st = device_tickets(device, (size_t)cnt_ints * 4, &tickets);
    if (st == NMG_OK) st = device_scratch(device, (size_t)part_floats * 4, &base);
    if (st != NMG_OK) return st;
    *counters = (int*)tickets;
    *part = (float*)base;
    return NMG_OK;
}

}  // namespace

bool decode_mma_supported(const nmg_kv_cache* c, int q_dtype) {
    if (c->dtype != NMG_Q8_0 && (c->dtype == NMG_F32 || q_dtype != c->dtype)) return false;
    if (c->dh != 64 && c->dh != 128 && c->dh != 256) return false;
    if (c->window > 0 && c->slots % KT != 0) return false;  // a tile must not straddle the ring end
    if ((int64_t)c->hkv * c->slots > 0x7FFFFFFF) return false;
    return true;
}

// Tensor maps of a Q8_0 cache's quants at head_dim 128 or 256: rows of dh
// int8 (the 64 spare rows included), boxes of 128 x 64 rows under the
// 128-byte swizzle.
static int make_q8_tensor_maps(const nmg_kv_cache* c, CUtensorMap* k, CUtensorMap* v) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(NMG_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)c->k & 15) || ((uintptr_t)c->v & 15)) return set_error(NMG_UNSUPPORTED, "unaligned cache");
    cuuint64_t dims[2] = {(cuuint64_t)c->dh, (cuuint64_t)c->hkv * (cuuint64_t)c->slots + 64};
    cuuint64_t strides[1] = {(cuuint64_t)c->dh};
    cuuint32_t box[2] = {128u, (cuuint32_t)KT};
    cuuint32_t estr[2] = {1, 1};
    for (int which = 0; which < 2; ++which) {
        const CUresult r = enc(which ? v : k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, which ? c->v : c->k, dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(NMG_CUDA_ERROR, "Q8_0 quant tensor map (%d)", (int)r);
    }
    return NMG_OK;
}

// Where the kernel reads cache i: tensor maps of a 16-bit cache, raw pointers of a Q8_0 one.
static int kv_sources(const nmg_kv_cache* c, MmaArgs* a, int i) {
    if (c->dtype == NMG_Q8_0) {
        a->q8[i] = Q8Src{(const int8_t*)c->k, (const int8_t*)c->v, (const uint16_t*)c->ks, (const uint16_t*)c->vs,
                         c->sstride};
        return c->dh == 128 || c->dh == 256 ? make_q8_tensor_maps(c, &a->tm_k[i], &a->tm_v[i]) : NMG_OK;
    }
    return make_kv_tensor_maps(c, KT, &a->tm_k[i], &a->tm_v[i]);
}

int attend_rows_mma(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                    int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                    cudaStream_t stream) {
    MmaArgs* a = new MmaArgs();
    int st = kv_sources(c, a, 0);
    const int gtot = hq / c->hkv;
    const int hn = mma_heads_in_n(gtot);
    const int zdim = hn ? 1 : (gtot + 15) / 16;
    a->hn = hn;
    int64_t longest = 0, total_blocks = 0;
    for (int64_t t = 0; st == NMG_OK && t < rows; ++t) {
        const VisibleSpan sp = visible_span(first_query + t, window, floor_pos, newest);
        const int64_t nb = (sp.hi - c->base) / KT - (sp.lo - c->base) / KT + 1;
        longest = std::max(longest, nb);
        total_blocks += nb;
    }
    const int64_t bps = mma_blocks_per_split(total_blocks * c->hkv * zdim, c->dh);
    const int64_t max_splits = (longest + bps - 1) / bps;
    const int64_t work = rows * max_splits;
    // every row with the same split count (2..8), heads in N: merge through a cluster
    bool uniform = hn && max_splits >= 2 && max_splits <= 8;
    for (int64_t t = 0; uniform && t < rows; ++t) {
        const VisibleSpan sp = visible_span(first_query + t, window, floor_pos, newest);
        const int64_t nb = (sp.hi - c->base) / KT - (sp.lo - c->base) / KT + 1;
        uniform = (nb + bps - 1) / bps == max_splits;
    }
    a->cl = uniform ? (int)max_splits : 0;
    if (st == NMG_OK && work > 0x7FFFFFFF) st = set_error(NMG_UNSUPPORTED, "decode: too many work items");
    if (st == NMG_OK) st = mma_scratch(c->device, work, c->hkv, zdim, c->dh, rows, &a->part, &a->counters);
    if (st == NMG_OK) st = device_error_flag(c->device, &a->err);
    if (st == NMG_OK) {
        a->mode = 0;
        a->hkv = c->hkv;
        a->hq = hq;
        a->gtot = gtot;
        a->zdim = zdim;
        a->blocks_per_split = bps;
        a->base = c->base;
        a->slots = c->slots;
        a->rows = rows;
        a->first_query = first_query;
        a->window = window;
        a->floor_pos = floor_pos;
        a->newest = newest;
        a->max_splits = (int32_t)max_splits;
        a->nseq = 0;
        a->q = q;
        a->q_dtype = q_dtype;
        a->out = out;
        a->out_dtype = out_dtype;
        a->scale_log2 = scale * 1.4426950408889634f;
        st = dispatch_mma(c, *a, dim3((unsigned)work, c->hkv, zdim), stream);
    }
    delete a;
    return st;
}

int attend_batch_mma(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq, const void* q,
                     int q_dtype, float scale, void* out, int out_dtype, cudaStream_t stream) {
    const nmg_kv_cache* c0 = caches[0];
    const int gtot = hq / c0->hkv;
    const int hn = mma_heads_in_n(gtot);
    const int zdim = hn ? 1 : (gtot + 15) / 16;
    std::vector<VisibleSpan> spans(batch);
    int64_t total_blocks = 0;
    for (int b = 0; b < batch; ++b) {
        const nmg_kv_cache* c = caches[b];
        const int64_t qpos = queries_at ? queries_at[b] : c->newest();
        spans[b] = visible_span(qpos, c->window, c->oldest, c->newest());
        total_blocks += (spans[b].hi - c->base) / KT - (spans[b].lo - c->base) / KT + 1;
    }
    const int64_t bps = mma_blocks_per_split(total_blocks * c0->hkv * zdim, c0->dh);
    int64_t all_work = 0;
    std::vector<int32_t> nsplit(batch);
    for (int b = 0; b < batch; ++b) {
        const nmg_kv_cache* c = caches[b];
        const int64_t nb = (spans[b].hi - c->base) / KT - (spans[b].lo - c->base) / KT + 1;
        nsplit[b] = (int32_t)((nb + bps - 1) / bps);
        all_work += nsplit[b];
    }
    // every sequence with the same split count (2..8), heads in N: merge through a cluster
    bool uniform = hn && nsplit[0] >= 2 && nsplit[0] <= 8;
    for (int b = 1; uniform && b < batch; ++b) uniform = nsplit[b] == nsplit[0];
    const int cl = uniform ? nsplit[0] : 0;
    float* part = nullptr;
    int* counters = nullptr;
    int st = mma_scratch(c0->device, all_work, c0->hkv, zdim, c0->dh, batch, &part, &counters);
    int* err = nullptr;
    if (st == NMG_OK) st = device_error_flag(c0->device, &err);
    MmaArgs* a = new MmaArgs();
    int64_t work_base = 0;
    for (int b0 = 0; st == NMG_OK && b0 < batch; b0 += kMmaMaxBatch) {
        const int nb = std::min(kMmaMaxBatch, batch - b0);
        int64_t w = 0;
        for (int i = 0; st == NMG_OK && i < nb; ++i) {
            const nmg_kv_cache* c = caches[b0 + i];
            st = kv_sources(c, a, i);
            MmaSeq& e = a->seq[i];
            e.base = c->base;
            e.slots = c->slots;
            e.lo = spans[b0 + i].lo;
            e.hi = spans[b0 + i].hi;
            e.nsplit = nsplit[b0 + i];
            e.work_first = (int32_t)w;
            e.qrow = b0 + i;
            e.map = i;
            w += e.nsplit;
        }
        if (st != NMG_OK) break;
        a->mode = 1;
        a->hn = hn;
        a->cl = cl;
        a->hkv = c0->hkv;
        a->hq = hq;
        a->gtot = gtot;
        a->zdim = zdim;
        a->blocks_per_split = bps;
        a->nseq = nb;
        a->q = q;
        a->q_dtype = q_dtype;
        a->out = out;
        a->out_dtype = out_dtype;
        a->scale_log2 = scale * 1.4426950408889634f;
        a->part = part + work_base * c0->hkv * zdim * 16 * (int64_t)(c0->dh + 2);
        a->counters = counters;
        a->err = err;
        st = dispatch_mma(c0, *a, dim3((unsigned)w, c0->hkv, zdim), stream);
        work_base += w;
    }
    delete a;
    return st;
}

}  // namespace nmg
