// attn_decode_cluster.cu -- split-KV decode over fp32 caches (head_dim 128,
// 256) on 8-warp CTAs, the splits of a row merged across a thread-block
// cluster when the decode is short.
//
// A decode over a short fp32 cache (a few MB) is bound by latency, not by
// bandwidth: a chain of tile load -> scores -> partial write -> fence ->
// atomic ticket -> merge pass runs in series.  Here the CL CTAs that share one
// (query row, K/V head, head subgroup) form one cluster:
//
//   * thread 0 issues the bulk copies of the CTA's first key tiles before
//     anything else, so the query load and set-up hide under them;
//   * 8 warps share a tile; a key's dot products are spread over LPK lanes
//     that hold DH / LPK query dims each in registers (G heads x DH / LPK = 64
//     values at most), reduced by xor shuffles; each warp keeps its own
//     online-softmax state (base 2, scale folded into q) for the keys it owns
//     and accumulates P.V with lane = value column;
//   * the warps merge through shared memory into one partial (m, l, o) per
//     head; the partial stays in shared memory, a cluster barrier publishes it,
//     and CTA r of the cluster combines columns [r * G*DH/CL, ...) of every
//     split's partial with distributed-shared-memory loads and writes them;
//   * a second cluster barrier keeps each CTA's shared memory alive until the
//     others have read it.
//
// So a short decode is one launch that touches only the cache, q and out:
// no global scratch, fence or ticket.  Every CTA reaches both cluster
// barriers (there is no early return), and each bulk-copy wait is bounded.
//
// A long decode over few (row, head) units needs more splits than a cluster
// holds; then the same CTAs run as an ordinary grid, write their partials to
// global scratch and the last CTA of the unit (atomic ticket) merges them.
//
// The reduction is the reference's (nm/src/qwen35.hpp:360-382,
// nm/src/gemma4.hpp:593-615): [scale *] dot(q, k_j), softmax over the visible
// rows, sum of alpha_j * v_j, GQA group head / (Hq / Hkv).
#include <algorithm>
#include <math.h>
#include <vector>

#include "attn.cuh"

namespace nmg {
namespace {

constexpr int kClBatch = 64;    // sequences per launch in the parameter block
// CTAs per cluster: the portable limit.  Wider (non-portable) clusters were
// measured slower on B200: a GPC held few 16-CTA clusters at a time, so a
// config-1 decode ran in two rounds (10.9 us against 7.1 us at 8).
constexpr int kClMax = 8;

struct ClRow {
    const float* k;
    const float* v;
    int64_t slots, base, lo, hi, qrow;
};

struct ClCommon {
    const void* q;
    void* out;
    int q_dtype, out_dtype, hq, hkv, gtot, zdim;
    float scale_log2;  // scale * log2(e): scores in base 2
    int* err;
    // ticket merge only: splits per row, partials [unit][split][G][DH+2], a ticket per unit
    int splits;
    float* gpart;
    int* tickets;
};

// One cache, query rows first_query.. (row r sees [max(q-window+1, floor), min(q, newest)]).
struct ClRowsArgs {
    ClCommon c;
    const float* k;
    const float* v;
    int64_t slots, base, first_query, window, floor_pos, newest;
    __device__ __forceinline__ ClRow row(int64_t r) const {
        const int64_t qpos = first_query + r;
        int64_t lo = floor_pos;
        if (window > 0 && qpos - window + 1 > lo) lo = qpos - window + 1;
        return ClRow{k, v, slots, base, lo, qpos < newest ? qpos : newest, r};
    }
};

struct ClSeq {
    const float* k;
    const float* v;
    int64_t slots, base, lo, hi;
};

// A table of caches, one query row each (row b of q / out is sequence b + row0).
struct ClBatchArgs {
    ClCommon c;
    int64_t row0;
    ClSeq seq[kClBatch];
    __device__ __forceinline__ ClRow row(int64_t b) const {
        const ClSeq& e = seq[b];
        return ClRow{e.k, e.v, e.slots, e.base, e.lo, e.hi, row0 + b};
    }
};

template <int DH, int G>
struct ClCfg {
    static constexpr int WARPS = 8, NT = WARPS * 32;
    // lanes per key: enough that a lane holds at most 64 query values and a
    // key tile of one of K or V stays within 32 KB
    static constexpr int LPK_Q = DH * G / 64, LPK_T = DH / 32;
    static constexpr int LPK = LPK_Q > LPK_T ? LPK_Q : LPK_T;
    static constexpr int DPL = DH / LPK;  // query dims per lane
    static constexpr int NCL = DPL / 4;   // 16-byte chunks per lane
    static constexpr int KPW = 32 / LPK;  // keys per warp per tile
    static constexpr int TK = WARPS * KPW;
    static constexpr int ROWB = DH * 4;
    static constexpr int TILE = TK * ROWB;  // one of K or V
    static constexpr int STAGE = 2 * TILE;
    // the CTA's exchange region: under the cluster merge the partials pushed
    // to this CTA, one record per (split, warp): (m, l) [R][G][2], then o
    // [R][share] with share <= G*DH/S rounded up to 4; under the ticket merge
    // the CTA's own partial [G][DH + 2]
    static constexpr int XR_FLOATS = WARPS * (G * DH + 4 * kClMax) + kClMax * WARPS * 2 * G;
    static constexpr int PART_BYTES = (XR_FLOATS * 4 + 15) / 16 * 16;
    // stages that fit beside it within the 227 KB a CTA may hold
    static constexpr int FIT = (232448 - PART_BYTES - 2048) / STAGE;
    static constexpr int MAX_STAGES = FIT < 8 ? FIT : 8;
    // rotate each lane's chunk order by its key so the 8 lanes of a shared
    // memory phase hit 8 distinct 16-byte bank groups
    static constexpr int ROT = LPK < 8 ? 8 / LPK : 1;
    static constexpr int PVC = DH / 128;  // 16-byte value chunks per lane
    // after the key loop: each warp's o [WARPS][G][DH], then its (m, l) [WARPS][G][2]
    static constexpr int CW_BYTES = WARPS * G * (DH + 2) * 4;
    static_assert(LPK <= 32 && DH % (4 * LPK) == 0 && NCL >= 1, "lane split");
    static_assert(DH % 128 == 0, "value columns: whole 16-byte chunks per lane");
    static_assert(ROWB % 16 == 0 && TILE % 16 == 0, "bulk copies move 16-byte multiples");
    static_assert(MAX_STAGES >= 1 && XR_FLOATS >= G * (DH + 2), "shared memory plan");
    static_assert(G * 64 * 4 <= STAGE, "merge weights fit the stage memory");
    static int smem(int stages) {
        const int body = stages * STAGE > CW_BYTES ? stages * STAGE : CW_BYTES;
        return body + PART_BYTES + 8 * MAX_STAGES;
    }
};

// 2^x by the hardware approximation (relative error ~2^-22; subnormal
// results flush to zero, far below the tolerance of the softmax weights).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split phase of a cluster barrier with no memory ordering: arrive early,
// wait later (here: every CTA of the cluster has started, so its shared
// memory may be written).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(dev::smem_u32(p)), "r"(rank));
    return d;
}
__device__ __forceinline__ void dsmem_st(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st4(uint32_t addr, float x, float y, float z, float w) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(x), "f"(y), "f"(z), "f"(w)
                 : "memory");
}

// GM = false: the CTAs of a row form a cluster and merge in distributed
// shared memory.  GM = true: an ordinary grid of `splits` CTAs per row that
// write their partials to global scratch; the last one (atomic ticket) merges.
template <int DH, int G, bool GM, class Args>
__global__ void __launch_bounds__(256, 1) attn_cluster_kernel(const __grid_constant__ Args a, int stages) {
    using C = ClCfg<DH, G>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int body = stages * C::STAGE > C::CW_BYTES ? stages * C::STAGE : C::CW_BYTES;
    float* part = (float*)(smem + body);  // this CTA's [G][DH+2]
    uint64_t* full = (uint64_t*)((unsigned char*)part + C::PART_BYTES);

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t rank = GM ? blockIdx.x % (uint32_t)a.c.splits : cluster_rank();
    const uint32_t ncl = GM ? (uint32_t)a.c.splits : cluster_size();
    const int64_t rowi = blockIdx.x / ncl;
    const int h = blockIdx.y, z = blockIdx.z;
    const ClRow r = a.row(rowi);
    const int qh0 = h * a.c.gtot + z * G;

    // This CTA's keys: split `rank` of the row, whole tiles except the last.
    const int64_t n = r.hi - r.lo + 1;
    const int64_t per = ((n + ncl - 1) / ncl + C::TK - 1) / C::TK * C::TK;
    const int64_t k_begin = r.lo + rank * per;
    const int64_t k_end = min(k_begin + per, r.hi + 1);
    const int ntiles = k_end > k_begin ? (int)((k_end - k_begin + C::TK - 1) / C::TK) : 0;
    const float* kh = r.k + (int64_t)h * r.slots * DH;
    const float* vh = r.v + (int64_t)h * r.slots * DH;

    auto stage_k = [&](int st) { return (float*)(smem + st * C::STAGE); };
    auto stage_v = [&](int st) { return (float*)(smem + st * C::STAGE + C::TILE); };
    // Slots run contiguously from the split's first slot, wrapping once at
    // the ring's end at most (a split never spans more than the ring).
    const int64_t slot_begin = (k_begin - r.base) % r.slots;
    auto issue = [&](int t) {  // thread 0: tile t into stage t % stages
        const int st = t % stages;
        const int64_t p0 = k_begin + (int64_t)t * C::TK;
        const int nt = (int)min((int64_t)C::TK, k_end - p0);
        int64_t slot0 = slot_begin + (int64_t)t * C::TK;
        if (slot0 >= r.slots) slot0 -= r.slots;
        const int run1 = (int)min((int64_t)nt, r.slots - slot0);
        const int run2 = nt - run1;
        // a refill follows generic reads of the stage: order them before the copy
        if (t >= stages) dev::fence_proxy_async_smem();
        dev::mbar_arrive_expect_tx(&full[st], 2u * nt * C::ROWB);
        dev::bulk_g2s(stage_k(st), kh + slot0 * DH, run1 * C::ROWB, &full[st]);
        dev::bulk_g2s(stage_v(st), vh + slot0 * DH, run1 * C::ROWB, &full[st]);
        if (run2 > 0) {
            dev::bulk_g2s(stage_k(st) + (int64_t)run1 * DH, kh, run2 * C::ROWB, &full[st]);
            dev::bulk_g2s(stage_v(st) + (int64_t)run1 * DH, vh, run2 * C::ROWB, &full[st]);
        }
    };
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) dev::mbar_init(&full[s], 1);
        dev::fence_mbar_init();
        // This split's K and V rows towards L2 while the previous kernel
        // finishes: a hint only (a row that kernel still writes is read again
        // after the wait below, from L2, where the write lands).
        if (k_end > k_begin) {
            const int64_t nk = k_end - k_begin;
            const int64_t run1 = min(nk, r.slots - slot_begin);
            dev::bulk_prefetch_l2(kh + slot_begin * DH, (uint32_t)(run1 * C::ROWB));
            dev::bulk_prefetch_l2(vh + slot_begin * DH, (uint32_t)(run1 * C::ROWB));
            if (nk > run1) {
                dev::bulk_prefetch_l2(kh, (uint32_t)((nk - run1) * C::ROWB));
                dev::bulk_prefetch_l2(vh, (uint32_t)((nk - run1) * C::ROWB));
            }
        }
    }
    // Launched with programmatic stream serialisation: everything above
    // overlaps the previous kernel's tail; no input (cache, q) is read before
    // its results are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0)
        for (int t = 0; t < ntiles && t < stages; ++t) issue(t);

    // Lane roles for the scores: key kk of the warp's KPW, query dims of part p.
    const int kk = lane / C::LPK, p = lane % C::LPK, rot = kk % C::ROT;
    float qv[G][C::NCL][4];
#pragma unroll
    for (int c = 0; c < C::NCL; ++c) {
        const int d0 = 4 * (p + C::LPK * ((c + rot) % C::NCL));
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int64_t qi = (r.qrow * (int64_t)a.c.hq + qh0 + g) * DH + d0;
#pragma unroll
            for (int e = 0; e < 4; ++e) qv[g][c][e] = dev::load_as_f32(a.c.q, a.c.q_dtype, qi + e) * a.c.scale_log2;
        }
    }
    __syncthreads();  // barrier initialisation visible to every waiter
    if constexpr (!GM) cluster_arrive_relaxed();  // waited on before the first remote store

    float m[G], l[G], o[G][C::PVC][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int c = 0; c < C::PVC; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[g][c][e] = 0.f;
    }

    bool aborted = false;
    for (int t = 0; t < ntiles; ++t) {
        const int st = t % stages;
        const bool ok = dev::mbar_wait(&full[st], (t / stages) & 1, a.c.err);
        if (__syncthreads_or(!ok)) {  // every thread gets here: waits are bounded
            aborted = true;
            break;
        }
        const int64_t p0 = k_begin + (int64_t)t * C::TK;
        const int nt = (int)min((int64_t)C::TK, k_end - p0);
        const int j = wid * C::KPW + kk;  // this lane's key within the tile
        const bool valid = j < nt;
        const float* krow = stage_k(st) + j * DH;
        float sc[G], sc2[G];  // two chains per head halve the dependent FMA depth
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = sc2[g] = 0.f;
#pragma unroll
        for (int c = 0; c < C::NCL; ++c) {
            const float4 kx = *(const float4*)(krow + 4 * (p + C::LPK * ((c + rot) % C::NCL)));
#pragma unroll
            for (int g = 0; g < G; ++g) {
                sc[g] = fmaf(qv[g][c][0], kx.x, sc[g]);
                sc2[g] = fmaf(qv[g][c][1], kx.y, sc2[g]);
                sc[g] = fmaf(qv[g][c][2], kx.z, sc[g]);
                sc2[g] = fmaf(qv[g][c][3], kx.w, sc2[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] += sc2[g];
        const int nk = min((int)C::KPW, nt - wid * C::KPW);  // warp-uniform
        float pj[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float s = sc[g];
#pragma unroll
            for (int off = 1; off < C::LPK; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            s = valid ? s : -INFINITY;
            float tmax = s;
#pragma unroll
            for (int off = C::LPK; off < 32; off <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(m[g], tmax);
            float alpha = 1.f, pe = 0.f;
            if (mnew != -INFINITY) {
                alpha = ex2(m[g] - mnew);  // m = -inf gives 0
                pe = valid ? ex2(s - mnew) : 0.f;
            }
            m[g] = mnew;
            l[g] = l[g] * alpha + (p == 0 ? pe : 0.f);
#pragma unroll
            for (int c = 0; c < C::PVC; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[g][c][e] *= alpha;
            pj[g] = pe;
        }
        const float* vbase = stage_v(st) + (wid * C::KPW) * DH;
        auto pv_key = [&](int jj) {
            float pw[G];
#pragma unroll
            for (int g = 0; g < G; ++g) pw[g] = __shfl_sync(0xffffffffu, pj[g], jj * C::LPK);
#pragma unroll
            for (int c = 0; c < C::PVC; ++c) {
                const float4 vx = *(const float4*)(vbase + jj * DH + 4 * (lane + 32 * c));
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    o[g][c][0] = fmaf(pw[g], vx.x, o[g][c][0]);
                    o[g][c][1] = fmaf(pw[g], vx.y, o[g][c][1]);
                    o[g][c][2] = fmaf(pw[g], vx.z, o[g][c][2]);
                    o[g][c][3] = fmaf(pw[g], vx.w, o[g][c][3]);
                }
            }
        };
        if (nk == C::KPW) {  // a full share: unrolled, the value loads issue together
#pragma unroll
            for (int jj = 0; jj < C::KPW; ++jj) pv_key(jj);
        } else {  // the tile's ragged end (value rows past it hold stale data)
            for (int jj = 0; jj < nk; ++jj) pv_key(jj);
        }
        __syncthreads();  // every warp is done with stage st
        if (tid == 0 && t + stages < ntiles) issue(t + stages);
    }

    const bool has = !aborted && ntiles > 0;
    if (!has) {  // an aborted or keyless CTA offers empty partials
#pragma unroll
        for (int g = 0; g < G; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int c = 0; c < C::PVC; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[g][c][e] = 0.f;
        }
    }
    float* xr = part;  // the exchange region

    if constexpr (GM) {
        // Merge the warps through shared memory (stage memory, idle now): each
        // warp's o, m, l, then thread i combines item i = (g, d) over the warps.
        float* cw = (float*)smem;
        float* wml = cw + C::WARPS * G * DH;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float lsum = dev::warp_sum(l[g]);
            if (lane == 0) {
                wml[(wid * G + g) * 2] = m[g];
                wml[(wid * G + g) * 2 + 1] = lsum;
            }
#pragma unroll
            for (int c = 0; c < C::PVC; ++c)
                *(float4*)(cw + (wid * G + g) * DH + 4 * (lane + 32 * c)) =
                    make_float4(o[g][c][0], o[g][c][1], o[g][c][2], o[g][c][3]);
        }
        __syncthreads();
        for (int i = tid; i < G * DH; i += C::NT) {
            const int g = i / DH, d = i % DH;
            float M = -INFINITY;
#pragma unroll
            for (int w2 = 0; w2 < C::WARPS; ++w2) M = fmaxf(M, wml[(w2 * G + g) * 2]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < C::WARPS; ++w2) {
                const float mw = wml[(w2 * G + g) * 2];
                const float f = mw == -INFINITY ? 0.f : ex2(mw - M);
                L = fmaf(wml[(w2 * G + g) * 2 + 1], f, L);
                O = fmaf(cw[(w2 * G + g) * DH + d], f, O);
            }
            xr[g * (DH + 2) + d] = O;
            if (d == 0) {
                xr[g * (DH + 2) + DH] = M;
                xr[g * (DH + 2) + DH + 1] = L;
            }
        }
        __shared__ int s_last;
        __syncthreads();
        const int64_t unit = (rowi * a.c.hkv + h) * a.c.zdim + z;
        float* mine = a.c.gpart + (unit * ncl + rank) * (int64_t)(G * (DH + 2));
        for (int i = tid; i < G * (DH + 2); i += C::NT) mine[i] = xr[i];
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&a.c.tickets[unit], 1) == (int)ncl - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        __shared__ float red[C::WARPS], wbuf[kMergeChunk];
        merge_partials<C::NT, DH, true>(a.c.gpart + unit * ncl * (int64_t)(G * (DH + 2)), G * (DH + 2), ncl, G, red,
                                        wbuf, [&](int g, int d, float v) {
                                            dev::store_from_f32(a.c.out, a.c.out_dtype,
                                                                (r.qrow * (int64_t)a.c.hq + qh0 + g) * DH + d, v);
                                        });
        if (tid == 0) a.c.tickets[unit] = 0;  // ready for the next launch
        return;
    } else {
        // Each warp pushes its partial straight from registers to the CTAs
        // that own its columns (CTA r owns items [r * share, (r+1) * share) of
        // the G*DH, share a multiple of 4 so a lane's float4 has one owner).
        // Receiver: record rec = rank * WARPS + warp, (m, l) [R][G][2], then
        // o [R][share].
        const int S = (int)ncl, R = S * C::WARPS, items = G * DH;
        const int share = ((items + S - 1) / S + 3) / 4 * 4;
        float* rml = xr;
        float* ro = xr + R * G * 2;
        const int rec = (int)rank * C::WARPS + wid;
        float lsum[G];
#pragma unroll
        for (int g = 0; g < G; ++g) lsum[g] = dev::warp_sum(l[g]);
        cluster_wait();  // every CTA of the cluster has started
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (lane < S) {
                const uint32_t dst = dsmem_addr(rml + (rec * G + g) * 2, lane);
                dsmem_st(dst, m[g]);
                dsmem_st(dst + 4, lsum[g]);
            }
#pragma unroll
            for (int c = 0; c < C::PVC; ++c) {
                const int i = g * DH + 4 * (lane + 32 * c);
                const int owner = i / share;
                dsmem_st4(dsmem_addr(ro + rec * share + (i - owner * share), owner), o[g][c][0], o[g][c][1],
                          o[g][c][2], o[g][c][3]);
            }
        }
        cluster_sync_all();  // every push has landed; no remote access follows

        // Weights per (group, record), normalised: warp g reduces group g.
        float* fn = (float*)smem;  // [G][64], stage memory (idle now)
        for (int g = wid; g < G; g += C::WARPS) {
            const float m0 = lane < R ? rml[(lane * G + g) * 2] : -INFINITY;
            const float m1 = lane + 32 < R ? rml[((lane + 32) * G + g) * 2] : -INFINITY;
            const float M = dev::warp_max(fmaxf(m0, m1));
            const float f0 = m0 == -INFINITY ? 0.f : ex2(m0 - M);
            const float f1 = m1 == -INFINITY ? 0.f : ex2(m1 - M);
            const float l0 = lane < R ? rml[(lane * G + g) * 2 + 1] : 0.f;
            const float l1 = lane + 32 < R ? rml[((lane + 32) * G + g) * 2 + 1] : 0.f;
            const float L = dev::warp_sum(f0 * l0 + f1 * l1);
            const float inv = L > 0.f ? 1.f / L : 0.f;
            fn[g * 64 + lane] = f0 * inv;
            fn[g * 64 + lane + 32] = f1 * inv;
        }
        __syncthreads();
        // This CTA's items: TPI threads per item, each over every TPI-th record.
        const int i0 = (int)rank * share, n_it = min(items, i0 + share) - i0;
        const int TPI = share * 8 <= C::NT ? 8 : share * 4 <= C::NT ? 4 : share * 2 <= C::NT ? 2 : 1;
        const int sub = tid % TPI;
        for (int base = 0; base < share; base += C::NT / TPI) {
            const int j = base + tid / TPI;
            const bool ok = j < n_it;
            const int g = (i0 + j) / DH, d = (i0 + j) % DH;
            float O = 0.f;
            if (ok)
                for (int r2 = sub; r2 < R; r2 += TPI) O = fmaf(ro[r2 * share + j], fn[g * 64 + r2], O);
            for (int off = 1; off < TPI; off <<= 1) O += __shfl_xor_sync(0xffffffffu, O, off);
            if (ok && sub == 0)
                dev::store_from_f32(a.c.out, a.c.out_dtype, (r.qrow * (int64_t)a.c.hq + qh0 + g) * DH + d, O);
        }
    }
}

// ---------------------------------------------------------------- host side

struct ClPlan {
    int ncl;     // cluster merge: splits per row (CTAs per cluster); 0 under the ticket merge
    int splits;  // ticket merge: splits per row; 0 under the cluster merge
    int stages;  // key tiles in flight per CTA
};

template <int DH, int G, class Args>
int launch_cluster(const Args& a, int rows, int hkv, int zdim, ClPlan pl, cudaStream_t s) {
    using C = ClCfg<DH, G>;
    if (a.c.splits > 0) {  // ticket merge: an ordinary grid
        auto kern = attn_cluster_kernel<DH, G, true, Args>;
        static std::atomic<uint64_t> attr_gm{0};
        const int st = set_smem_once(kern, C::smem(C::MAX_STAGES), attr_gm);
        if (st != NMG_OK) return st;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((int64_t)rows * a.c.splits), (unsigned)hkv, (unsigned)zdim);
        cfg.blockDim = dim3(C::NT, 1, 1);
        cfg.dynamicSmemBytes = C::smem(pl.stages);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        NMG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, pl.stages));
        return NMG_OK;
    }
    auto kern = attn_cluster_kernel<DH, G, false, Args>;
    static std::atomic<uint64_t> attr_set{0};
    const int st = set_smem_once(kern, C::smem(C::MAX_STAGES), attr_set);  // covers any stage count
    if (st != NMG_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * pl.ncl), (unsigned)hkv, (unsigned)zdim);
    cfg.blockDim = dim3(C::NT, 1, 1);
    cfg.dynamicSmemBytes = C::smem(pl.stages);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)pl.ncl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    NMG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, pl.stages));
    return NMG_OK;
}

int pick_group(int gtot) {
    for (int g : {8, 4, 2, 1})
        if (gtot % g == 0) return g;
    return 1;
}

template <int DH>
int tile_keys_dh(int gt) {
    return gt == 8 ? ClCfg<DH, 8>::TK : gt == 4 ? ClCfg<DH, 4>::TK : gt == 2 ? ClCfg<DH, 2>::TK : ClCfg<DH, 1>::TK;
}
template <int DH>
int max_stages_dh(int gt) {
    return gt == 8   ? ClCfg<DH, 8>::MAX_STAGES
           : gt == 4 ? ClCfg<DH, 4>::MAX_STAGES
           : gt == 2 ? ClCfg<DH, 2>::MAX_STAGES
                     : ClCfg<DH, 1>::MAX_STAGES;
}

// Cluster merge while (row, head, subgroup) units x at most kClMax splits
// still cover the SMs or the decode moves under 16 MB (latency-bound, where
// no scratch round trip is worth paying); otherwise enough ticket-merged
// splits for about four CTAs per SM, each of at least two tiles.
ClPlan plan_decode(int64_t units, int64_t longest, int64_t bytes, int dh, int gt) {
    const int tk = dh == 128 ? tile_keys_dh<128>(gt) : tile_keys_dh<256>(gt);
    const int smax = dh == 128 ? max_stages_dh<128>(gt) : max_stages_dh<256>(gt);
    const int64_t tiles = (longest + tk - 1) / tk;
    ClPlan pl{0, 0, 1};
    int64_t sp;
    if (units * kClMax >= 148 || bytes <= (16ll << 20)) {
        sp = std::min<int64_t>((2 * 148 + units - 1) / units, kClMax);
        sp = std::max<int64_t>(1, std::min<int64_t>(sp, tiles));
        pl.ncl = (int)sp;
    } else {
        sp = (4 * 148 + units - 1) / units;
        sp = std::max<int64_t>(1, std::min<int64_t>(sp, (tiles + 1) / 2));
        sp = std::min<int64_t>(sp, 4096);
        pl.splits = (int)sp;
    }
    pl.stages = (int)std::max<int64_t>(1, std::min<int64_t>((tiles + sp - 1) / sp, smax));
    return pl;
}

template <int DH, class Args>
int dispatch_g(int gt, const Args& a, int rows, int hkv, int zdim, const ClPlan& pl, cudaStream_t s) {
    switch (gt) {
        case 8: return launch_cluster<DH, 8>(a, rows, hkv, zdim, pl, s);
        case 4: return launch_cluster<DH, 4>(a, rows, hkv, zdim, pl, s);
        case 2: return launch_cluster<DH, 2>(a, rows, hkv, zdim, pl, s);
        default: return launch_cluster<DH, 1>(a, rows, hkv, zdim, pl, s);
    }
}

template <class Args>
int dispatch(int dh, int gt, const Args& a, int rows, int hkv, int zdim, const ClPlan& pl, cudaStream_t s) {
    if (dh == 128) return dispatch_g<128>(gt, a, rows, hkv, zdim, pl, s);
    return dispatch_g<256>(gt, a, rows, hkv, zdim, pl, s);
}

int fill_common(ClCommon& cm, const nmg_kv_cache* c, int hq, const void* q, int q_dtype, float scale, void* out,
                int out_dtype, int zdim, int gt, int64_t rows, const ClPlan& pl) {
    cm.q = q;
    cm.out = out;
    cm.q_dtype = q_dtype;
    cm.out_dtype = out_dtype;
    cm.hq = hq;
    cm.hkv = c->hkv;
    cm.gtot = hq / c->hkv;
    cm.zdim = zdim;
    cm.scale_log2 = scale * 1.4426950408889634f;
    cm.splits = pl.splits;
    cm.gpart = nullptr;
    cm.tickets = nullptr;
    if (pl.splits > 0) {  // scratch of the ticket merge (tickets stay zero between launches)
        const int64_t units = rows * c->hkv * zdim;
        void* p = nullptr;
        int st = device_scratch(c->device, (size_t)(units * pl.splits * gt * (int64_t)(c->dh + 2) * 4), &p);
        if (st != NMG_OK) return st;
        cm.gpart = (float*)p;
        st = device_tickets(c->device, (size_t)units * 4, &p);
        if (st != NMG_OK) return st;
        cm.tickets = (int*)p;
    }
    return device_error_flag(c->device, &cm.err);
}

}  // namespace

// fp32 caches at head_dim 128 / 256 decode here (either merge form).
bool fp32_decode_fits(const nmg_kv_cache* c) { return c->dtype == NMG_F32 && (c->dh == 128 || c->dh == 256); }

int attend_rows_cluster(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                        int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                        cudaStream_t stream) {
    int64_t longest = 0, total = 0;
    for (int64_t t = 0; t < rows; ++t) {
        const VisibleSpan sp = visible_span(first_query + t, window, floor_pos, newest);
        longest = std::max(longest, sp.hi - sp.lo + 1);
        total += sp.hi - sp.lo + 1;
    }
    const int gt = pick_group(hq / c->hkv);
    const int zdim = hq / c->hkv / gt;
    const int64_t units = rows * c->hkv * zdim;
    const ClPlan pl = plan_decode(units, longest, total * c->hkv * c->dh * 8, c->dh, gt);
    if (rows * std::max(pl.ncl, pl.splits) > 0x7FFFFFFF) return set_error(NMG_UNSUPPORTED, "attention: too many query rows");
    ClRowsArgs a{};
    int st = fill_common(a.c, c, hq, q, q_dtype, scale, out, out_dtype, zdim, gt, rows, pl);
    if (st != NMG_OK) return st;
    a.k = (const float*)c->k;
    a.v = (const float*)c->v;
    a.slots = c->slots;
    a.base = c->base;
    a.first_query = first_query;
    a.window = window;
    a.floor_pos = floor_pos;
    a.newest = newest;
    return dispatch(c->dh, gt, a, (int)rows, c->hkv, zdim, pl, stream);
}

int attend_batch_cluster(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq,
                         const void* q, int q_dtype, float scale, void* out, int out_dtype, cudaStream_t stream) {
    const nmg_kv_cache* c0 = caches[0];
    std::vector<VisibleSpan> spans(batch);
    int64_t longest = 0, total = 0;
    for (int b = 0; b < batch; ++b) {
        const nmg_kv_cache* c = caches[b];
        const int64_t qpos = queries_at ? queries_at[b] : c->newest();
        spans[b] = visible_span(qpos, c->window, c->oldest, c->newest());
        longest = std::max(longest, spans[b].hi - spans[b].lo + 1);
        total += spans[b].hi - spans[b].lo + 1;
    }
    const int gt = pick_group(hq / c0->hkv);
    const int zdim = hq / c0->hkv / gt;
    const int nb0 = std::min(kClBatch, batch);
    const ClPlan pl = plan_decode((int64_t)nb0 * c0->hkv * zdim, longest, total * c0->hkv * c0->dh * 8, c0->dh, gt);
    ClBatchArgs* a = new ClBatchArgs();
    int st = fill_common(a->c, c0, hq, q, q_dtype, scale, out, out_dtype, zdim, gt, nb0, pl);
    for (int b0 = 0; b0 < batch && st == NMG_OK; b0 += kClBatch) {
        const int nb = std::min(kClBatch, batch - b0);
        a->row0 = b0;
        for (int i = 0; i < nb; ++i) {
            const nmg_kv_cache* c = caches[b0 + i];
            a->seq[i] = ClSeq{(const float*)c->k, (const float*)c->v, c->slots, c->base, spans[b0 + i].lo,
                              spans[b0 + i].hi};
        }
        st = dispatch(c0->dh, gt, *a, nb, c0->hkv, zdim, pl, stream);
    }
    delete a;
    return st;
}

}  // namespace nmg
