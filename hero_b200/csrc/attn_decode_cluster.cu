// attn_decode_cluster.cu -- low-latency split-KV decode over fp32 caches,
// the splits of a row merged across a thread-block cluster.
//
// A decode over a short fp32 cache (a few MB) is bound by latency, not by
// bandwidth: the split kernel's chain of tile load -> scores -> partial write
// -> fence -> atomic ticket -> merge pass runs in series.  Here the CL CTAs
// that share one (query row, K/V head, head subgroup) form one cluster:
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
// No global scratch, fence or ticket: a decode is one launch that touches
// only the cache, q and out.  Every CTA reaches both cluster barriers (there
// is no early return), and each bulk-copy wait is bounded.
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

constexpr int kClBatch = 64;  // sequences per launch in the parameter block
constexpr int kClMax = 8;     // CTAs per cluster (the portable limit)

struct ClRow {
    const float* k;
    const float* v;
    int64_t slots, base, lo, hi, qrow;
};

struct ClCommon {
    const void* q;
    void* out;
    int q_dtype, out_dtype, hq, hkv, gtot;
    float scale_log2;  // scale * log2(e): scores in base 2
    int* err;
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
    static constexpr int MAX_STAGES = (196608 / STAGE) < 8 ? 196608 / STAGE : 8;
    // rotate each lane's chunk order by its key so the 8 lanes of a shared
    // memory phase hit 8 distinct 16-byte bank groups
    static constexpr int ROT = LPK < 8 ? 8 / LPK : 1;
    static constexpr int PVC = DH / 128;  // 16-byte value chunks per lane
    static constexpr int CW_BYTES = WARPS * G * (DH + 2) * 4;
    static constexpr int PART_BYTES = (G * (DH + 2) * 4 + 15) / 16 * 16;
    static_assert(LPK <= 32 && DH % (4 * LPK) == 0 && NCL >= 1, "lane split");
    static_assert(DH % 128 == 0, "value columns: whole 16-byte chunks per lane");
    static_assert(ROWB % 16 == 0 && TILE % 16 == 0, "bulk copies move 16-byte multiples");
    static int smem(int stages) {
        const int body = stages * STAGE > CW_BYTES ? stages * STAGE : CW_BYTES;
        return body + PART_BYTES + 8 * MAX_STAGES;
    }
};

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
// Address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(dev::smem_u32(p)), "r"(rank));
    return d;
}
__device__ __forceinline__ float dsmem_ld(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

template <int DH, int G, class Args>
__global__ void __launch_bounds__(256, 1) attn_cluster_kernel(const __grid_constant__ Args a, int stages) {
    using C = ClCfg<DH, G>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int body = stages * C::STAGE > C::CW_BYTES ? stages * C::STAGE : C::CW_BYTES;
    float* part = (float*)(smem + body);  // this CTA's [G][DH+2]
    uint64_t* full = (uint64_t*)((unsigned char*)part + C::PART_BYTES);

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t rank = cluster_rank(), ncl = cluster_size();
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
    auto issue = [&](int t) {  // thread 0: tile t into stage t % stages
        const int st = t % stages;
        const int64_t p0 = k_begin + (int64_t)t * C::TK;
        const int nt = (int)min((int64_t)C::TK, k_end - p0);
        const int64_t slot0 = (p0 - r.base) % r.slots;
        const int run1 = (int)min((int64_t)nt, r.slots - slot0);
        const int run2 = nt - run1;
        dev::fence_proxy_async_smem();
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
        for (int t = 0; t < ntiles && t < stages; ++t) issue(t);
    }

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
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = 0.f;
#pragma unroll
        for (int c = 0; c < C::NCL; ++c) {
            const float4 kx = *(const float4*)(krow + 4 * (p + C::LPK * ((c + rot) % C::NCL)));
#pragma unroll
            for (int g = 0; g < G; ++g) {
                sc[g] = fmaf(qv[g][c][0], kx.x, sc[g]);
                sc[g] = fmaf(qv[g][c][1], kx.y, sc[g]);
                sc[g] = fmaf(qv[g][c][2], kx.z, sc[g]);
                sc[g] = fmaf(qv[g][c][3], kx.w, sc[g]);
            }
        }
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
                alpha = exp2f(m[g] - mnew);  // m = -inf gives 0
                pe = valid ? exp2f(s - mnew) : 0.f;
            }
            m[g] = mnew;
            l[g] = l[g] * alpha + (p == 0 ? pe : 0.f);
#pragma unroll
            for (int c = 0; c < C::PVC; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[g][c][e] *= alpha;
            pj[g] = pe;
        }
        if (nk > 0) {
            const float* vbase = stage_v(st) + (wid * C::KPW) * DH;
            for (int jj = 0; jj < nk; ++jj) {
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
            }
        }
        __syncthreads();  // every warp is done with stage st
        if (tid == 0 && t + stages < ntiles) issue(t + stages);
    }

    // Merge the warps into this CTA's partial; an aborted CTA offers an empty one.
    if (!aborted && ntiles > 0) {
        float* cw = (float*)smem;  // stage memory, idle now
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float lsum = dev::warp_sum(l[g]);
            float* w = cw + (wid * G + g) * (DH + 2);
            if (lane == 0) {
                w[DH] = m[g];
                w[DH + 1] = lsum;
            }
#pragma unroll
            for (int c = 0; c < C::PVC; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) w[4 * (lane + 32 * c) + e] = o[g][c][e];
        }
        __syncthreads();
        for (int i = tid; i < G * DH; i += C::NT) {
            const int g = i / DH, d = i % DH;
            float M = -INFINITY;
#pragma unroll
            for (int w2 = 0; w2 < C::WARPS; ++w2) M = fmaxf(M, cw[(w2 * G + g) * (DH + 2) + DH]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < C::WARPS; ++w2) {
                const float* w = cw + (w2 * G + g) * (DH + 2);
                const float f = w[DH] == -INFINITY ? 0.f : exp2f(w[DH] - M);
                L = fmaf(w[DH + 1], f, L);
                O = fmaf(w[d], f, O);
            }
            part[g * (DH + 2) + d] = O;
            if (d == 0) {
                part[g * (DH + 2) + DH] = M;
                part[g * (DH + 2) + DH + 1] = L;
            }
        }
    } else {
        for (int i = tid; i < G; i += C::NT) {
            part[i * (DH + 2) + DH] = -INFINITY;
            part[i * (DH + 2) + DH + 1] = 0.f;
        }
    }

    cluster_sync_all();  // every split's partial is published

    // CTA `rank` combines its share of the G*DH output columns over the splits.
    const int items = G * DH;
    const int share = (items + (int)ncl - 1) / (int)ncl;
    const int i0 = (int)rank * share, i1 = min(items, i0 + share);
    for (int i = i0 + tid; i < i1; i += C::NT) {
        const int g = i / DH, d = i % DH;
        float Ms[kClMax], Ls[kClMax], Os[kClMax];
        float M = -INFINITY;
#pragma unroll
        for (int s = 0; s < kClMax; ++s) {
            Ms[s] = -INFINITY;
            Ls[s] = 0.f;
            Os[s] = 0.f;
            if (s < (int)ncl) {
                const uint32_t base = dsmem_addr(part + g * (DH + 2), s);
                Ms[s] = dsmem_ld(base + DH * 4);
                Ls[s] = dsmem_ld(base + (DH + 1) * 4);
                Os[s] = dsmem_ld(base + d * 4);
                M = fmaxf(M, Ms[s]);
            }
        }
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int s = 0; s < kClMax; ++s) {
            if (Ms[s] != -INFINITY) {
                const float f = exp2f(Ms[s] - M);
                L = fmaf(Ls[s], f, L);
                O = fmaf(Os[s], f, O);
            }
        }
        dev::store_from_f32(a.c.out, a.c.out_dtype, (r.qrow * (int64_t)a.c.hq + qh0 + g) * DH + d,
                            L > 0.f ? O / L : 0.f);
    }

    cluster_sync_all();  // no CTA leaves while another may still read its partial
}

// ---------------------------------------------------------------- host side

template <int DH, int G, class Args>
int launch_cluster(const Args& a, int rows, int hkv, int zdim, int ncl, int stages, cudaStream_t s) {
    using C = ClCfg<DH, G>;
    auto kern = attn_cluster_kernel<DH, G, Args>;
    static std::atomic<uint64_t> attr_set{0};
    const int st = set_smem_once(kern, C::smem(C::MAX_STAGES), attr_set);  // covers any stage count
    if (st != NMG_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * ncl), (unsigned)hkv, (unsigned)zdim);
    cfg.blockDim = dim3(C::NT, 1, 1);
    cfg.dynamicSmemBytes = C::smem(stages);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ncl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NMG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, stages));
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

struct ClPlan {
    int ncl;     // splits per row (CTAs per cluster)
    int stages;  // key tiles in flight per CTA
};

ClPlan plan_cluster(int64_t units, int64_t longest, int dh, int gt) {
    // Enough CTAs to cover the SMs about twice, at most kClMax splits, and no
    // split without a whole tile.
    const int tk = dh == 128 ? tile_keys_dh<128>(gt) : tile_keys_dh<256>(gt);
    const int smax = dh == 128 ? max_stages_dh<128>(gt) : max_stages_dh<256>(gt);
    int64_t ncl = (2 * 148 + units - 1) / units;
    ncl = std::min<int64_t>(ncl, kClMax);
    ncl = std::min<int64_t>(ncl, (longest + tk - 1) / tk);
    ncl = std::max<int64_t>(ncl, 1);
    const int64_t per = ((longest + ncl - 1) / ncl + tk - 1) / tk;  // tiles of the longest split
    return ClPlan{(int)ncl, (int)std::max<int64_t>(1, std::min<int64_t>(per, smax))};
}

template <int DH, class Args>
int dispatch_g(int gt, const Args& a, int rows, int hkv, int zdim, const ClPlan& pl, cudaStream_t s) {
    switch (gt) {
        case 8: return launch_cluster<DH, 8>(a, rows, hkv, zdim, pl.ncl, pl.stages, s);
        case 4: return launch_cluster<DH, 4>(a, rows, hkv, zdim, pl.ncl, pl.stages, s);
        case 2: return launch_cluster<DH, 2>(a, rows, hkv, zdim, pl.ncl, pl.stages, s);
        default: return launch_cluster<DH, 1>(a, rows, hkv, zdim, pl.ncl, pl.stages, s);
    }
}

template <class Args>
int dispatch(int dh, int gt, const Args& a, int rows, int hkv, int zdim, const ClPlan& pl, cudaStream_t s) {
    if (dh == 128) return dispatch_g<128>(gt, a, rows, hkv, zdim, pl, s);
    return dispatch_g<256>(gt, a, rows, hkv, zdim, pl, s);
}

int fill_common(ClCommon& cm, const nmg_kv_cache* c, int hq, const void* q, int q_dtype, float scale, void* out,
                int out_dtype) {
    cm.q = q;
    cm.out = out;
    cm.q_dtype = q_dtype;
    cm.out_dtype = out_dtype;
    cm.hq = hq;
    cm.hkv = c->hkv;
    cm.gtot = hq / c->hkv;
    cm.scale_log2 = scale * 1.4426950408889634f;
    return device_error_flag(c->device, &cm.err);
}

}  // namespace

// The cluster path serves fp32 caches at head_dim 128 / 256 when its CTAs
// (units x at most kClMax splits) still fill the GPU, or when the whole
// decode moves under 16 MB and latency, not bandwidth, bounds it.
bool cluster_decode_fits(const nmg_kv_cache* c, int64_t units, int64_t total_keys) {
    if (c->dtype != NMG_F32 || (c->dh != 128 && c->dh != 256)) return false;
    const int64_t bytes = total_keys * c->hkv * c->dh * 4 * 2;
    return units * kClMax >= 148 || bytes <= (16ll << 20);
}

int attend_rows_cluster(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                        int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                        cudaStream_t stream) {
    const int gt = pick_group(hq / c->hkv);
    const int zdim = hq / c->hkv / gt;
    int64_t longest = 0;
    for (int64_t t = 0; t < rows; ++t) {
        const VisibleSpan sp = visible_span(first_query + t, window, floor_pos, newest);
        longest = std::max(longest, sp.hi - sp.lo + 1);
    }
    if (rows > 0x7FFFFFFF / kClMax) return set_error(NMG_UNSUPPORTED, "attention: too many query rows");
    const ClPlan pl = plan_cluster(rows * c->hkv * zdim, longest, c->dh, gt);
    ClRowsArgs a{};
    int st = fill_common(a.c, c, hq, q, q_dtype, scale, out, out_dtype);
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
    const int gt = pick_group(hq / c0->hkv);
    const int zdim = hq / c0->hkv / gt;
    std::vector<VisibleSpan> spans(batch);
    int64_t longest = 0;
    for (int b = 0; b < batch; ++b) {
        const nmg_kv_cache* c = caches[b];
        const int64_t qpos = queries_at ? queries_at[b] : c->newest();
        spans[b] = visible_span(qpos, c->window, c->oldest, c->newest());
        longest = std::max(longest, spans[b].hi - spans[b].lo + 1);
    }
    const ClPlan pl = plan_cluster((int64_t)batch * c0->hkv * zdim, longest, c0->dh, gt);
    ClBatchArgs* a = new ClBatchArgs();
    int st = fill_common(a->c, c0, hq, q, q_dtype, scale, out, out_dtype);
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
