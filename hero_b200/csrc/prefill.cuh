// prefill.cuh -- pieces shared by the tcgen05 flash-attention prefill kernels
// (attn_prefill_sm100.cu: one query head a unit; attn_prefill_pair.cu: two
// query heads of one GQA group a unit): the argument block, the unit list
// walk, output rounding, and the epilogue's row stores and split merges.
#pragma once
#include <math.h>

#include "attn.cuh"
#include "tcgen05.cuh"

namespace nmg {
namespace pf {

constexpr int kMaxFanout = 8;
constexpr int kMaxItems = 2048;  // work items of a split launch
constexpr int kMaxTiles = 1024;  // query tiles of a split launch

struct PrefillArgs {
    CUtensorMap tm_q;  // (d, head, row) over q [rows][hq*DH]
    CUtensorMap tm_k;  // (d, hkv*slots) over the cache
    CUtensorMap tm_v;
    int64_t rows, first_query, window, floor_pos, newest, base, slots;
    int hq, hkv, g;
    int hunits;  // head units per tile item: hq (one head a unit) or hq / 2 (head pairs)
    float scale_log2;
    // Output row t of this call goes to outs[i] + t * out_row_elems + out_col0
    // (elements) for every i < nout: the caller's buffer and, when the heads
    // are sharded across GPUs, the other GPUs' buffers (peer pointers), so
    // the gather of head outputs rides on the epilogue's stores.
    void* outs[kMaxFanout];
    int nout;
    int64_t out_row_elems, out_col0;
    int out_dtype;
    int* err;
    // Work list: n_work = (n_items or ntiles) * hunits units, heaviest first,
    // head unit fastest.  Key splits (n_items > 0): unit u takes items[u / hq] =
    // tile << 12 | split << 6 | nsplit, key blocks [split * split_blocks,
    // +split_blocks) of the tile's range.  A split tile's units leave (O, m,
    // l) partials in part (slot part_base[tile] + split of head h: [BM][DH +
    // 4] fp32, O then m, l, with rows padded to 16 bytes) and the last one to
    // finish (ticket per head and tile) merges them.  n_items == 0: one unit
    // per (tile, head), unit u = tile ntiles - 1 - u / hq of head u % hq.
    int64_t n_work;
    int n_items, split_blocks, nparts, ntiles;
    float* part;
    int* tickets;
    uint32_t items[kMaxItems];
    uint32_t part_base[kMaxTiles];
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
    if (bf16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Output conversions with the reference's rounding (dev::f32_to_bf16_bits,
// dev::f32_to_f16_bits), for two values packed low first.
__device__ __forceinline__ uint32_t pack_out(float lo, float hi, int dtype) {
    if (dtype == NMG_BF16) return (uint32_t)dev::f32_to_bf16_bits(lo) | ((uint32_t)dev::f32_to_bf16_bits(hi) << 16);
    return (uint32_t)dev::f32_to_f16_bits(lo) | ((uint32_t)dev::f32_to_f16_bits(hi) << 16);
}
// The same without branches for the values the epilogue meets almost
// always; a warp with any other value takes pack_out instead.
//   bf16: round to nearest even, which the hardware conversion gives for
//         every value but NaN (the reference quiets NaN its own way).
//   f16:  results in the normal range (fp32 exponent 113..142), where the
//         reference rounds half up on bit 12 of the mantissa.
__device__ __forceinline__ bool bf16_fast_ok(float x) { return x == x; }
__device__ __forceinline__ bool f16_fast_ok(float x) { return ((__float_as_uint(x) >> 23) & 0xFFu) - 113u <= 29u; }
__device__ __forceinline__ uint32_t pack_bf16_fast(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t f16_fast(float x) {
    const uint32_t b = __float_as_uint(x);
    const uint32_t h = ((b >> 16) & 0x8000u) | ((((b >> 23) & 0xFFu) - 112u) << 10) | ((b >> 13) & 0x3FFu);
    return h + ((b >> 12) & 1u);
}
__device__ __forceinline__ uint32_t pack_f16_fast(float lo, float hi) { return f16_fast(lo) | (f16_fast(hi) << 16); }

// AND of `v` over the `count` threads that meet on named barrier `id`.
__device__ __forceinline__ bool bar_and(int id, int count, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ int64_t vis_lo(const PrefillArgs& a, int64_t q) {
    int64_t lo = a.floor_pos;
    if (a.window > 0 && q - a.window + 1 > lo) lo = q - a.window + 1;
    return lo;
}
__device__ __forceinline__ int64_t vis_hi(const PrefillArgs& a, int64_t q) { return q < a.newest ? q : a.newest; }

// One unit of work: a query tile (or a key split of one) of one head unit
// (h: a head, or a pair of heads 2h, 2h + 1 of one GQA group).
struct Work {
    int h, tile, split, nsplit, nblk;
    int64_t t0, t_last, j_begin, full_lo, full_hi;
};

// The k-th unit of this CTA.  CTAs walk the heavy-first list in snake order
// (k even: unit k * G + b, k odd: k * G + G - 1 - b), which evens out the
// per-CTA totals of a list sorted by decreasing work.  Every role of the CTA
// decodes the same sequence.
template <int BM, int BN>
__device__ __forceinline__ bool decode_work(const PrefillArgs& a, int k, Work& w) {
    const int G = gridDim.x, b = blockIdx.x;
    const int64_t idx = (int64_t)k * G + ((k & 1) ? G - 1 - b : b);
    if (idx >= a.n_work) return false;
    w.h = (int)(idx % a.hunits);
    const int it = (int)(idx / a.hunits);
    if (a.n_items > 0) {
        const uint32_t item = a.items[it];
        w.tile = (int)(item >> 12);
        w.split = (int)((item >> 6) & 63u);
        w.nsplit = (int)(item & 63u);
    } else {
        w.tile = a.ntiles - 1 - it;
        w.split = 0;
        w.nsplit = 1;
    }
    w.t0 = (int64_t)w.tile * BM;
    w.t_last = (w.t0 + BM < a.rows ? w.t0 + BM : a.rows) - 1;
    const int64_t q_first = a.first_query + w.t0, q_last = a.first_query + w.t_last;
    const int64_t u_lo = vis_lo(a, q_first) - a.base, u_hi = vis_hi(a, q_last) - a.base;
    const int nblk_all = (int)(u_hi / BN + 1 - u_lo / BN);
    w.j_begin = u_lo / BN + (int64_t)w.split * a.split_blocks;
    w.nblk = w.nsplit == 1 ? nblk_all : min(a.split_blocks, nblk_all - w.split * a.split_blocks);
    // A block needs no mask when every row of the tile sees all of it.
    w.full_lo = vis_lo(a, q_last);
    w.full_hi = vis_hi(a, q_first);
    return true;
}


// ---- epilogue pieces shared by the prefill kernels ------------------------
//
// One warp per TMEM lane quadrant (128 threads): `quad` and `lane` name the
// row (quad * 32 + lane) of the unit's tile, t_lane the quadrant's TMEM base.

// Normalise one head's finished O rows (TMEM columns o_col..) by 1 / l_row,
// stage the warp's 32 rows 128 bytes at a time, then store whole 128-byte row
// pieces (four rows per instruction) to every output.  Arrives on o_free once
// the last TMEM read is done.
template <int DH>
__device__ __forceinline__ void store_rows(const PrefillArgs& a, const Work& w, int head, uint32_t t_lane,
                                           uint32_t o_col, float l_row, int quad, int lane, uint4* stage,
                                           uint64_t* o_free) {
    const int oes = a.out_dtype == NMG_F32 ? 4 : 2;
    const int cpc = 128 / oes;  // output columns per 128-byte row piece
    const int valid_rows = (int)(w.t_last - w.t0 + 1);
    const float inv = 1.f / l_row;
    const int64_t row_bytes = a.out_row_elems * oes;
    const int64_t base_off =
        ((w.t0 + quad * 32 + (lane >> 3)) * a.out_row_elems + a.out_col0 + (int64_t)head * DH) * oes + (lane & 7) * 16;
#pragma unroll 1
    for (int c0 = 0; c0 < DH; c0 += cpc) {
        // 32 columns per TMEM load: 8 stage chunks of fp32, or 4 of 16-bit values.
#pragma unroll 1
        for (int h = 0; h < cpc / 32; ++h) {
            uint32_t r[32];
            tc::ld_32x32b_x32(t_lane + o_col + c0 + 32 * h, r);
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * inv);
            auto f = [&](int e) { return __uint_as_float(r[e]); };
            if (oes == 4) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    stage[lane * 8 + (j ^ (lane & 7))] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            } else {
                const bool bf = a.out_dtype == NMG_BF16;
                bool fast = true;
#pragma unroll
                for (int e = 0; e < 32; ++e) fast &= bf ? bf16_fast_ok(f(e)) : f16_fast_ok(f(e));
                const bool all_fast = __all_sync(0xffffffffu, fast);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int chunk = 4 * h + j;
                    uint4 v;
                    if (!all_fast)
                        v = make_uint4(pack_out(f(8 * j), f(8 * j + 1), a.out_dtype), pack_out(f(8 * j + 2), f(8 * j + 3), a.out_dtype),
                                       pack_out(f(8 * j + 4), f(8 * j + 5), a.out_dtype), pack_out(f(8 * j + 6), f(8 * j + 7), a.out_dtype));
                    else if (bf)
                        v = make_uint4(pack_bf16_fast(f(8 * j), f(8 * j + 1)), pack_bf16_fast(f(8 * j + 2), f(8 * j + 3)),
                                       pack_bf16_fast(f(8 * j + 4), f(8 * j + 5)), pack_bf16_fast(f(8 * j + 6), f(8 * j + 7)));
                    else
                        v = make_uint4(pack_f16_fast(f(8 * j), f(8 * j + 1)), pack_f16_fast(f(8 * j + 2), f(8 * j + 3)),
                                       pack_f16_fast(f(8 * j + 4), f(8 * j + 5)), pack_f16_fast(f(8 * j + 6), f(8 * j + 7)));
                    stage[lane * 8 + (chunk ^ (lane & 7))] = v;
                }
            }
        }
        if (c0 + cpc >= DH) {  // O and the statistics are read: the buffer is free
            tc::fence_before_sync();
            dev::mbar_arrive(o_free);
        }
        __syncwarp();
        uint4 v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int rr = m * 4 + (lane >> 3);
            v[m] = stage[rr * 8 + ((lane & 7) ^ (rr & 7))];
        }
        __syncwarp();
        for (int o = 0; o < a.nout; ++o) {
            unsigned char* p = (unsigned char*)a.outs[o] + base_off + c0 * oes;
#pragma unroll
            for (int m = 0; m < 8; ++m)
                if (quad * 32 + m * 4 + (lane >> 3) < valid_rows) *(uint4*)(p + m * 4 * row_bytes) = v[m];
        }
    }
    // No fence: a caller that reads the rows on another GPU orders these
    // stores with a stream-ordered barrier (nmg_comm_barrier), which starts
    // only after this grid, stores included, has completed.
}

// A split of a tile: leave one head's unnormalised O row with its m and l
// (base-2 units) in the partials, then arrive on o_free.
template <int DH>
__device__ __forceinline__ void store_partial(const PrefillArgs& a, const Work& w, int head, int row, uint32_t t_lane,
                                              uint32_t o_col, float m_run, float l_row, uint64_t* o_free) {
    float* mine = a.part + (((int64_t)head * a.nparts + a.part_base[w.tile] + w.split) * 128 + row) * (DH + 4);
#pragma unroll 1
    for (int c = 0; c < DH / 32; ++c) {
        uint32_t r[32];
        tc::ld_32x32b_x32(t_lane + o_col + c * 32, r);
        float4* dst = (float4*)(mine + c * 32);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]), __uint_as_float(r[4 * e + 2]),
                                 __uint_as_float(r[4 * e + 3]));
    }
    mine[DH] = m_run;
    mine[DH + 1] = l_row;
    tc::fence_before_sync();
    dev::mbar_arrive(o_free);
}

// Row rr of one head of a split tile, merged over all of the tile's splits
// and written to every output: the row's maximum and sum over the splits
// first, then 16-column chunks in which every split's loads are independent
// of its weight, so each split costs about one L2 round trip per chunk.
template <int DH>
__device__ __forceinline__ void merge_row(const PrefillArgs& a, const Work& w, int head, int rr) {
    const int oes = a.out_dtype == NMG_F32 ? 4 : 2;
    const float* base = a.part + ((int64_t)head * a.nparts + a.part_base[w.tile]) * 128 * (DH + 4);
    const int64_t slot = (int64_t)128 * (DH + 4);
    const float* rowp = base + rr * (DH + 4);
    float M = -INFINITY;
#pragma unroll 4
    for (int sp = 0; sp < w.nsplit; ++sp) M = fmaxf(M, __ldcg(rowp + sp * slot + DH));
    float L = 0.f;
#pragma unroll 4
    for (int sp = 0; sp < w.nsplit; ++sp) {
        const float m = __ldcg(rowp + sp * slot + DH);
        if (m != -INFINITY) L = fmaf(ex2(m - M), __ldcg(rowp + sp * slot + DH + 1), L);
    }
    const float inv = 1.f / L;
    const int64_t off0 = ((w.t0 + rr) * a.out_row_elems + a.out_col0 + (int64_t)head * DH) * oes;
#pragma unroll 1
    for (int c = 0; c < DH / 16; ++c) {
        float o[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) o[e] = 0.f;
#pragma unroll 1
        for (int sp = 0; sp < w.nsplit; ++sp) {
            const float* rp = rowp + sp * slot;
            float4 v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = __ldcg((const float4*)(rp + c * 16) + e);
            const float m = __ldcg(rp + DH);
            const float wgt = m == -INFINITY ? 0.f : ex2(m - M);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                o[4 * e] = fmaf(wgt, v[e].x, o[4 * e]), o[4 * e + 1] = fmaf(wgt, v[e].y, o[4 * e + 1]);
                o[4 * e + 2] = fmaf(wgt, v[e].z, o[4 * e + 2]), o[4 * e + 3] = fmaf(wgt, v[e].w, o[4 * e + 3]);
            }
        }
        const int64_t off = off0 + (int64_t)c * 16 * oes;
        for (int oi = 0; oi < a.nout; ++oi) {
            unsigned char* dst = (unsigned char*)a.outs[oi] + off;
            if (a.out_dtype == NMG_F32) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    ((float4*)dst)[e] = make_float4(o[4 * e] * inv, o[4 * e + 1] * inv, o[4 * e + 2] * inv, o[4 * e + 3] * inv);
            } else {
#pragma unroll
                for (int e = 0; e < 2; ++e)
                    ((uint4*)dst)[e] = make_uint4(pack_out(o[8 * e] * inv, o[8 * e + 1] * inv, a.out_dtype),
                                                  pack_out(o[8 * e + 2] * inv, o[8 * e + 3] * inv, a.out_dtype),
                                                  pack_out(o[8 * e + 4] * inv, o[8 * e + 5] * inv, a.out_dtype),
                                                  pack_out(o[8 * e + 6] * inv, o[8 * e + 7] * inv, a.out_dtype));
            }
        }
    }
}

}  // namespace pf

// Launches the two-head prefill kernel for head_dim `dh` (attn_prefill_pair.cu);
// NMG_UNSUPPORTED for head dims it is not built for.
int launch_prefill_pair(const pf::PrefillArgs& a, int dh, bool bf16, dim3 grid, cudaStream_t s);

}  // namespace nmg
