// attn_decode.cu -- split-KV attention over the device cache (K2/K3), and the
// host dispatch of every attention entry point.
//
// One CTA owns (query row, kv head, q-head subgroup, key split).  Key tiles of
// 32*WARPS consecutive positions arrive in shared memory by bulk TMA copies
// (cp.async.bulk, one CTA per copy) into a 2-stage ring; each warp takes 32 keys
// of a tile: lane = key for the scores (q rows broadcast from shared memory,
// 16-byte chunks read in a lane-rotated order so the 32 key rows hit distinct
// banks), an online softmax per query head, then lane = value column for P.V.
// Warps merge through shared memory.  When a row's keys span several splits,
// each CTA writes an unnormalised partial (m, l, o) to scratch and the last
// CTA of the row (atomic ticket) merges them and writes the output, so decode
// is one launch.
//
// This is the reduction the reference writes inline per layer
// (nm/src/qwen35.hpp:360-382, nm/src/gemma4.hpp:211-235, :302-321, :593-615,
// :687-709): scores = [scale *] dot(q, k_j), softmax over the visible rows,
// sum of alpha_j * v_j, with GQA group head / (Hq / Hkv).
#include <algorithm>
#include <math.h>
#include <mutex>
#include <stdio.h>
#include <vector>

#include "attn.cuh"
#include "kv_cache.cuh"

namespace nmg {
namespace {

constexpr int kMaxBatch = 96;  // sequences per launch carried in the parameter block

struct SeqEntry {
    const void* k;  // head 0, slot 0
    const void* v;
    int64_t slots, base;
    int64_t lo, hi;      // visible positions, inclusive
    int32_t work_first;  // first work item (blockIdx.x) of this sequence
    int32_t nsplit;
    int32_t qrow;
};

struct SplitArgs {
    int mode;  // 0: one cache, `rows` query rows; 1: table of sequences
    int hkv, hq, gtot, zdim;
    int64_t split_len;
    // mode 0
    const void* k;
    const void* v;
    int64_t slots, base, rows, first_query, window, floor_pos, newest;
    int32_t max_splits;
    // mode 1
    int nseq;
    SeqEntry seq[kMaxBatch];
    int32_t row_offset;  // counter/qrow offset of this launch within the batch
    // common
    const void* q;
    int q_dtype;
    void* out;
    int out_dtype;
    float scale;
    float* part;      // partials [work][hkv][zdim][G*(DH+2)]
    int* counters;    // [row][hkv][zdim]
    int* err;
};

struct RowInfo {
    const void* k;
    const void* v;
    int64_t slots, base, lo, hi;
    int64_t work_first, nsplit, qrow, s;
};

__device__ __forceinline__ bool decode_row(const SplitArgs& a, int64_t w, RowInfo& r) {
    if (a.mode == 0) {
        const int64_t row = w / a.max_splits;
        r.s = w % a.max_splits;
        const int64_t qpos = a.first_query + row;
        int64_t lo = a.floor_pos;
        if (a.window > 0 && qpos - a.window + 1 > lo) lo = qpos - a.window + 1;
        const int64_t hi = qpos < a.newest ? qpos : a.newest;
        r.k = a.k;
        r.v = a.v;
        r.slots = a.slots;
        r.base = a.base;
        r.lo = lo;
        r.hi = hi;
        r.nsplit = (hi - lo + a.split_len) / a.split_len;
        r.work_first = row * a.max_splits;
        r.qrow = row;
        return r.s < r.nsplit;
    }
    int b = 0;
    while (b + 1 < a.nseq && a.seq[b + 1].work_first <= w) ++b;
    const SeqEntry& e = a.seq[b];
    r.k = e.k;
    r.v = e.v;
    r.slots = e.slots;
    r.base = e.base;
    r.lo = e.lo;
    r.hi = e.hi;
    r.nsplit = e.nsplit;
    r.work_first = e.work_first;
    r.qrow = e.qrow;
    r.s = w - e.work_first;
    return r.s < r.nsplit;
}

template <int KVDT, int DH, int G, int WARPS>
struct SplitCfg {
    using KT = typename dev::Elem<KVDT>::T;
    static constexpr int ES = sizeof(KT);
    static constexpr int TK = 32 * WARPS;
    static constexpr int ROWB = DH * ES;
    static constexpr bool BULK = (ROWB % 16) == 0;
    static constexpr int PER = (DH + 31) / 32;
    static constexpr int TILE_BYTES = TK * ROWB;
    static constexpr int STAGE_BYTES = 2 * ((TILE_BYTES + 127) / 128) * 128;
    static constexpr int Q_OFF = 2 * STAGE_BYTES;
    static constexpr int P_OFF = Q_OFF + G * DH * 4;
    static constexpr int C_OFF = P_OFF + WARPS * G * 32 * 4;
    static constexpr int BAR_OFF = ((C_OFF + WARPS * G * (DH + 2) * 4) + 15) / 16 * 16;
    static constexpr int SMEM = BAR_OFF + 64;
    // dynamic plus the kernel's static arrays (ticket flag, merge scratch) within 227 KB
    static_assert(SMEM + 4 * (WARPS + 256 + 1) <= 232448, "shared memory budget");
    static_assert(!BULK || (ROWB % 16 == 0 && (Q_OFF % 16) == 0), "bulk copies move 16-byte multiples");
};

template <int KVDT, int DH, int G, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) attn_split_kernel(const __grid_constant__ SplitArgs a) {
    using C = SplitCfg<KVDT, DH, G, WARPS>;
    using KT = typename C::KT;
    // V buffer element type (a bf16 cache keeps V as fp16; same width).
    constexpr int VDT = KVDT == NMG_BF16 ? NMG_F16 : KVDT;
    extern __shared__ __align__(128) unsigned char smem[];
    float* qs = (float*)(smem + C::Q_OFF);
    float* ps = (float*)(smem + C::P_OFF);
    float* cs = (float*)(smem + C::C_OFF);
    uint64_t* full = (uint64_t*)(smem + C::BAR_OFF);
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int h = blockIdx.y, z = blockIdx.z;
    RowInfo r;
    if (!decode_row(a, blockIdx.x, r)) return;

    const int64_t k_begin = r.lo + r.s * a.split_len;
    const int64_t k_end = min(r.lo + (r.s + 1) * a.split_len, r.hi + 1);
    const int64_t nkeys = k_end - k_begin;
    const int ntiles = (int)((nkeys + C::TK - 1) / C::TK);
    const KT* kh = (const KT*)r.k + (int64_t)h * r.slots * DH;
    const KT* vh = (const KT*)r.v + (int64_t)h * r.slots * DH;
    const int qh0 = h * a.gtot + z * G;

    if (tid == 0) mbar_init_pair(full);
    for (int i = tid; i < G * DH; i += WARPS * 32) {
        const int g = i / DH, d = i % DH;
        qs[i] = dev::load_as_f32(a.q, a.q_dtype, (r.qrow * (int64_t)a.hq + qh0 + g) * DH + d);
    }
    __syncthreads();

    auto stage_k = [&](int st) { return (KT*)(smem + st * C::STAGE_BYTES); };
    auto stage_v = [&](int st) { return (KT*)(smem + st * C::STAGE_BYTES + C::STAGE_BYTES / 2); };

    // Fill stage `st` with tile t (bulk copies issued by thread 0, or a
    // cooperative copy when a head row is not a multiple of 16 bytes).
    auto issue = [&](int t, int st) {
        const int64_t p0 = k_begin + (int64_t)t * C::TK;
        const int n = (int)min((int64_t)C::TK, k_end - p0);
        const int64_t slot0 = (p0 - r.base) % r.slots;
        const int run1 = (int)min((int64_t)n, r.slots - slot0);
        const int run2 = n - run1;
        if constexpr (C::BULK) {
            if (tid == 0) {
                dev::fence_proxy_async_smem();
                dev::mbar_arrive_expect_tx(&full[st], 2u * n * C::ROWB);
                dev::bulk_g2s(stage_k(st), kh + slot0 * DH, run1 * C::ROWB, &full[st]);
                dev::bulk_g2s(stage_v(st), vh + slot0 * DH, run1 * C::ROWB, &full[st]);
                if (run2 > 0) {
                    dev::bulk_g2s(stage_k(st) + (int64_t)run1 * DH, kh, run2 * C::ROWB, &full[st]);
                    dev::bulk_g2s(stage_v(st) + (int64_t)run1 * DH, vh, run2 * C::ROWB, &full[st]);
                }
            }
        } else {
            for (int i = tid; i < n * DH; i += WARPS * 32) {
                const int row = i / DH, d = i % DH;
                const int64_t slot = row < run1 ? slot0 + row : row - run1;
                stage_k(st)[i] = kh[slot * DH + d];
                stage_v(st)[i] = vh[slot * DH + d];
            }
        }
    };

    float m[G], l[G], o[G][C::PER];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < C::PER; ++e) o[g][e] = 0.f;
    }

    bool aborted = false;
    issue(0, 0);
    for (int t = 0; t < ntiles; ++t) {
        const int st = t & 1;
        if (t + 1 < ntiles) issue(t + 1, st ^ 1);
        bool ok = true;
        if constexpr (C::BULK) ok = dev::mbar_wait(&full[st], (t >> 1) & 1, a.err);
        // Every thread reaches this barrier (waits are bounded), so a timeout
        // anywhere ends the loop uniformly.
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        const KT* ks = stage_k(st);
        const KT* vs = stage_v(st);
        const int64_t p0 = k_begin + (int64_t)t * C::TK;
        const int n = (int)min((int64_t)C::TK, k_end - p0);
        const int key = wid * 32 + lane;
        const bool valid = key < n;

        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = 0.f;
        if (valid) {
            const KT* krow = ks + key * DH;
            if constexpr (C::BULK) {
                constexpr int E = 16 / C::ES;  // elements per 16-byte chunk
                constexpr int NCH = DH / E;
#pragma unroll 4
                for (int c = 0; c < NCH; ++c) {
                    const int cc = (c + lane) % NCH;
                    const uint4 raw = *(const uint4*)(krow + cc * E);
                    float kv[E];
                    unpack16<KVDT>(raw, kv);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float* qg = qs + g * DH + cc * E;
#pragma unroll
                        for (int e = 0; e < E; ++e) sc[g] = fmaf(qg[e], kv[e], sc[g]);
                    }
                }
            } else {
                for (int d = 0; d < DH; ++d) {
                    const float kf = dev::Elem<KVDT>::load(krow + d);
#pragma unroll
                    for (int g = 0; g < G; ++g) sc[g] = fmaf(qs[g * DH + d], kf, sc[g]);
                }
            }
        }
        float* pw = ps + wid * G * 32;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float s = valid ? a.scale * sc[g] : -INFINITY;
            const float tmax = dev::warp_max(s);
            const float mnew = fmaxf(m[g], tmax);
            float alpha = 1.f, p = 0.f;
            if (mnew != -INFINITY) {
                alpha = (m[g] == -INFINITY) ? 0.f : __expf(m[g] - mnew);
                p = valid ? __expf(s - mnew) : 0.f;
            }
            l[g] = l[g] * alpha + p;
#pragma unroll
            for (int e = 0; e < C::PER; ++e) o[g][e] *= alpha;
            m[g] = mnew;
            pw[g * 32 + lane] = p;
        }
        __syncwarp();
        const int nk = min(32, n - wid * 32);
        for (int j = 0; j < nk; ++j) {
            const KT* vrow = vs + (wid * 32 + j) * DH;
            float vv[C::PER];
            load_row_chunk<VDT, DH, C::PER>(vrow, lane, vv);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float p = pw[g * 32 + j];
#pragma unroll
                for (int e = 0; e < C::PER; ++e) o[g][e] = fmaf(p, vv[e], o[g][e]);
            }
        }
        __syncthreads();
    }
    if (aborted) return;

    // Merge the warps of this CTA.
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float lsum = dev::warp_sum(l[g]);
        float* cw = cs + (wid * G + g) * (DH + 2);
        if (lane == 0) {
            cw[DH] = m[g];
            cw[DH + 1] = lsum;
        }
#pragma unroll
        for (int e = 0; e < C::PER; ++e) {
            const int d = lane * C::PER + e;
            if (d < DH) cw[d] = o[g][e];
        }
    }
    __syncthreads();

    const bool single = r.nsplit == 1;
    const int64_t cnt_idx = ((r.qrow + a.row_offset) * (int64_t)a.hkv + h) * a.zdim + z;
    float* my_part = a.part + ((((int64_t)blockIdx.x) * a.hkv + h) * a.zdim + z) * (int64_t)(G * (DH + 2));
    for (int i = tid; i < G * DH; i += WARPS * 32) {
        const int g = i / DH, d = i % DH;
        float M = -INFINITY;
        for (int w2 = 0; w2 < WARPS; ++w2) M = fmaxf(M, cs[(w2 * G + g) * (DH + 2) + DH]);
        float L = 0.f, O = 0.f;
        for (int w2 = 0; w2 < WARPS; ++w2) {
            const float* cw = cs + (w2 * G + g) * (DH + 2);
            if (cw[DH] == -INFINITY) continue;
            const float f = __expf(cw[DH] - M);
            L += cw[DH + 1] * f;
            O += cw[d] * f;
        }
        if (single) {
            dev::store_from_f32(a.out, a.out_dtype, (r.qrow * (int64_t)a.hq + qh0 + g) * DH + d, O / L);
        } else {
            my_part[g * (DH + 2) + d] = O;
            if (d == 0) {
                my_part[g * (DH + 2) + DH] = M;
                my_part[g * (DH + 2) + DH + 1] = L;
            }
        }
    }
    if (single) return;

    // Last CTA of the row merges every split.
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int old = atomicAdd(&a.counters[cnt_idx], 1);
        s_last = (old == (int)r.nsplit - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    {
        __shared__ float red[WARPS], wbuf[kMergeChunk];
        const float* first = a.part + (((r.work_first) * a.hkv + h) * a.zdim + z) * (int64_t)(G * (DH + 2));
        merge_partials<WARPS * 32, DH, false>(
            first, (int64_t)a.hkv * a.zdim * (G * (DH + 2)), r.nsplit, G, red, wbuf, [&](int g, int d, float v) {
                dev::store_from_f32(a.out, a.out_dtype, (r.qrow * (int64_t)a.hq + qh0 + g) * DH + d, v);
            });
    }
    if (tid == 0) a.counters[cnt_idx] = 0;  // ready for the next launch
}

// ---------------------------------------------------------------- dispatch

template <int KVDT, int DH, int G>
constexpr int warps_for() {
    constexpr int rowb = DH * (KVDT == NMG_F32 ? 4 : 2);
    return rowb <= 256 ? 4 : (rowb <= 512 ? 2 : 1);
}

template <int KVDT, int DH, int G>
int launch_split(const SplitArgs& a, dim3 grid, cudaStream_t s) {
    constexpr int W = warps_for<KVDT, DH, G>();
    using C = SplitCfg<KVDT, DH, G, W>;
    auto kern = attn_split_kernel<KVDT, DH, G, W>;
    static std::atomic<uint64_t> attr_set{0};  // one bit per device
    const int st = set_smem_once(kern, C::SMEM, attr_set);
    if (st != NMG_OK) return st;
    kern<<<grid, W * 32, C::SMEM, s>>>(a);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

template <int KVDT, int DH>
int dispatch_g(int gt, const SplitArgs& a, dim3 grid, cudaStream_t s) {
    switch (gt) {
        case 8: return launch_split<KVDT, DH, 8>(a, grid, s);
        case 4: return launch_split<KVDT, DH, 4>(a, grid, s);
        case 2: return launch_split<KVDT, DH, 2>(a, grid, s);
        default: return launch_split<KVDT, DH, 1>(a, grid, s);
    }
}

int dispatch_split(int kvdt, int dh, int gt, const SplitArgs& a, dim3 grid, cudaStream_t s) {
    if (kvdt == NMG_Q8_0) return set_error(NMG_UNSUPPORTED, "split-KV attention: Q8_0 caches are not built");
    if (kvdt == NMG_F32) {
        switch (dh) {
            case 1: return dispatch_g<NMG_F32, 1>(gt, a, grid, s);
            case 2: return dispatch_g<NMG_F32, 2>(gt, a, grid, s);
            case 4: return dispatch_g<NMG_F32, 4>(gt, a, grid, s);
            case 8: return dispatch_g<NMG_F32, 8>(gt, a, grid, s);
            case 16: return dispatch_g<NMG_F32, 16>(gt, a, grid, s);
            case 32: return dispatch_g<NMG_F32, 32>(gt, a, grid, s);
            case 64: return dispatch_g<NMG_F32, 64>(gt, a, grid, s);
            case 128: return dispatch_g<NMG_F32, 128>(gt, a, grid, s);
            case 256: return dispatch_g<NMG_F32, 256>(gt, a, grid, s);
        }
    } else if (kvdt == NMG_F16) {
        switch (dh) {
            case 64: return dispatch_g<NMG_F16, 64>(gt, a, grid, s);
            case 128: return dispatch_g<NMG_F16, 128>(gt, a, grid, s);
            case 256: return dispatch_g<NMG_F16, 256>(gt, a, grid, s);
            case 512: return dispatch_g<NMG_F16, 512>(gt, a, grid, s);
        }
    } else {
        switch (dh) {
            case 64: return dispatch_g<NMG_BF16, 64>(gt, a, grid, s);
            case 128: return dispatch_g<NMG_BF16, 128>(gt, a, grid, s);
            case 256: return dispatch_g<NMG_BF16, 256>(gt, a, grid, s);
            case 512: return dispatch_g<NMG_BF16, 512>(gt, a, grid, s);
        }
    }
    return set_error(NMG_UNSUPPORTED, "attention: head_dim %d with cache dtype %d is not built", dh, kvdt);
}

int pick_gt(int gtot) {
    for (int g : {8, 4, 2, 1})
        if (gtot % g == 0) return g;
    return 1;
}

int64_t pick_split_len(int64_t key_heads, int warps) {
    const int64_t tk = 32 * warps;
    int64_t target = key_heads / (148 * 6);
    if (target < tk) target = tk;
    if (target > 8192) target = 8192;
    return (target + tk - 1) / tk * tk;
}

int warps_runtime(int kvdt, int dh) {
    const int rowb = dh * dtype_size(kvdt);
    return rowb <= 256 ? 4 : (rowb <= 512 ? 2 : 1);
}

int scratch_for(int device, int64_t work, int hkv, int zdim, int gt, int dh, int64_t counter_rows, float** part,
                int** counters, void* caller_scratch, int64_t caller_bytes) {
    const int64_t part_floats = work * hkv * zdim * (int64_t)gt * (dh + 2);
    const int64_t cnt_ints = counter_rows * hkv * zdim;
    if (caller_scratch) {  // the caller zeroes the tickets at the start of its memory
        const size_t bytes = (size_t)cnt_ints * 4 + 256 + (size_t)part_floats * 4;
        if ((int64_t)bytes > caller_bytes)
            return set_error(NMG_LENGTH_ERROR, "attention needs %zu bytes of scratch, %lld given", bytes,
                             (long long)caller_bytes);
        *counters = (int*)caller_scratch;
        *part = (float*)((char*)caller_scratch + ((size_t)cnt_ints * 4 + 255) / 256 * 256);
        return NMG_OK;
    }
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

// Rows of one cache: positions first_query.., visible [max(q-window+1, floor), min(q, newest)].
int attend_rows_split(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                      int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                      cudaStream_t stream, void* caller_scratch, int64_t caller_bytes) {
    const int gtot = hq / c->hkv;
    const int gt = pick_gt(gtot);
    const int zdim = gtot / gt;
    // Longest visible span over the rows (the last row sees the most keys in
    // a full cache; any row can be longest under a window).
    int64_t longest = 0, total_keys = 0;
    for (int64_t t = 0; t < rows; ++t) {
        const VisibleSpan sp = visible_span(first_query + t, window, floor_pos, newest);
        const int64_t n = sp.hi - sp.lo + 1;
        if (n > longest) longest = n;
        total_keys += n;
    }
    if (!caller_scratch && fp32_decode_fits(c))
        return attend_rows_cluster(c, hq, q, q_dtype, rows, first_query, window, floor_pos, newest, scale, out,
                                   out_dtype, stream);
    const int warps = warps_runtime(c->dtype, c->dh);
    const int64_t split_len = pick_split_len(total_keys * c->hkv * zdim, warps);
    const int64_t max_splits = (longest + split_len - 1) / split_len;
    const int64_t work = rows * max_splits;
    if (work > (int64_t)0x7FFFFFFF) return set_error(NMG_UNSUPPORTED, "attention: too many work items");
    SplitArgs* a = new SplitArgs();
    a->mode = 0;
    a->hkv = c->hkv;
    a->hq = hq;
    a->gtot = gtot;
    a->zdim = zdim;
    a->split_len = split_len;
    a->k = c->k;
    a->v = c->v;
    a->slots = c->slots;
    a->base = c->base;
    a->rows = rows;
    a->first_query = first_query;
    a->window = window;
    a->floor_pos = floor_pos;
    a->newest = newest;
    a->max_splits = (int32_t)max_splits;
    a->nseq = 0;
    a->row_offset = 0;
    a->q = q;
    a->q_dtype = q_dtype;
    a->out = out;
    a->out_dtype = out_dtype;
    a->scale = scale;
    int st = scratch_for(c->device, work, c->hkv, zdim, gt, c->dh, rows, &a->part, &a->counters, caller_scratch,
                         caller_bytes);
    if (st == NMG_OK) st = device_error_flag(c->device, &a->err);
    if (st == NMG_OK) st = dispatch_split(c->dtype, c->dh, gt, *a, dim3((unsigned)work, c->hkv, zdim), stream);
    delete a;
    return st;
}

int attend_batch_split(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq, const void* q,
                       int q_dtype, float scale, void* out, int out_dtype, cudaStream_t stream) {
    const nmg_kv_cache* c0 = caches[0];
    const int gtot = hq / c0->hkv;
    const int gt = pick_gt(gtot);
    const int zdim = gtot / gt;
    int64_t total_keys = 0;
    std::vector<VisibleSpan> spans(batch);
    for (int b = 0; b < batch; ++b) {
        const nmg_kv_cache* c = caches[b];
        const int64_t qpos = queries_at ? queries_at[b] : c->newest();
        spans[b] = visible_span(qpos, c->window, c->oldest, c->newest());
        total_keys += spans[b].hi - spans[b].lo + 1;
    }
    if (fp32_decode_fits(c0))
        return attend_batch_cluster(caches, batch, queries_at, hq, q, q_dtype, scale, out, out_dtype, stream);
    const int warps = warps_runtime(c0->dtype, c0->dh);
    const int64_t split_len = pick_split_len(total_keys * c0->hkv * zdim, warps);
    int64_t all_work = 0;
    for (int b = 0; b < batch; ++b) all_work += (spans[b].hi - spans[b].lo + split_len) / split_len;
    float* part = nullptr;
    int* counters = nullptr;
    int st = scratch_for(c0->device, all_work, c0->hkv, zdim, gt, c0->dh, batch, &part, &counters, nullptr, 0);
    if (st != NMG_OK) return st;
    int* err = nullptr;
    st = device_error_flag(c0->device, &err);
    if (st != NMG_OK) return st;
    SplitArgs* a = new SplitArgs();
    int64_t work_base = 0;
    for (int b0 = 0; b0 < batch && st == NMG_OK; b0 += kMaxBatch) {
        const int nb = std::min(kMaxBatch, batch - b0);
        a->mode = 1;
        a->hkv = c0->hkv;
        a->hq = hq;
        a->gtot = gtot;
        a->zdim = zdim;
        a->split_len = split_len;
        a->nseq = nb;
        a->row_offset = 0;
        int64_t w = 0;
        for (int i = 0; i < nb; ++i) {
            const nmg_kv_cache* c = caches[b0 + i];
            SeqEntry& e = a->seq[i];
            e.k = c->k;
            e.v = c->v;
            e.slots = c->slots;
            e.base = c->base;
            e.lo = spans[b0 + i].lo;
            e.hi = spans[b0 + i].hi;
            e.nsplit = (int32_t)((e.hi - e.lo + split_len) / split_len);
            e.work_first = (int32_t)w;
            e.qrow = b0 + i;
            w += e.nsplit;
        }
        a->q = q;
        a->q_dtype = q_dtype;
        a->out = out;
        a->out_dtype = out_dtype;
        a->scale = scale;
        // Partials of this launch start after the previous launches' work items.
        a->part = part + work_base * c0->hkv * zdim * (int64_t)gt * (c0->dh + 2);
        a->counters = counters;
        a->err = err;
        st = dispatch_split(c0->dtype, c0->dh, gt, *a, dim3((unsigned)w, c0->hkv, zdim), stream);
        work_base += w;
    }
    delete a;
    return st;
}

}  // namespace nmg

// ------------------------------------------------ no-allocation decode entry
//
// Some callers cannot call cudaMalloc at all: an engine whose device memory
// is carved out by its own arena allocator and may not be grown behind its
// back, or a serving loop that must never hit the device-wide synchronisation
// cudaMalloc/cudaFree can cause.  nmg_attend_noalloc serves them: the same
// split-KV attention as nmg_attend's decode path, but its scratch (row
// tickets and per-split partial results) lives in the fixed array below, so
// no call allocates device memory.  The caller still owns q and out.
//
// The array is shared by every call in the process on a given device and keeps
// what the last call left; calls whose kernels overlap on that device (two
// streams, two host threads) race on it and must be serialised by the caller.
//
// Layout: [0, 256) the path's error word (a wait that gave up raises it; only
// nmg_device_status reads and clears it), then the row tickets (cleared by
// every call), then the split partials.
namespace nmg {
namespace {

constexpr size_t kNoallocScratchBytes = size_t(4) << 20;  // 4 MiB per device, held until exit
constexpr size_t kNoallocFlagBytes = 256;                   // the error word, then the tickets

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Host code may not use the array's name as a device address; look it up once
// per device with that device current.
int noalloc_scratch(int device, void** ptr) {
    if (device < 0 || device >= 64) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_noalloc: device %d", device);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(NMG_CUDA_ERROR, "nmg_attend_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_noalloc_addr[device] = p;
    }
    *ptr = g_noalloc_addr[device];
    return NMG_OK;
}

}  // namespace

int* noalloc_error_word(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    return (int*)g_noalloc_addr[device];
}

int noalloc_error_word_init(int device, int** word) {
    void* base = nullptr;
    const int st = noalloc_scratch(device, &base);
    *word = (int*)base;
    return st;
}

}  // namespace nmg

extern "C" int nmg_attend_noalloc(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows,
                                  int64_t first_query, float scale, int use_scale, void* out, int out_dtype,
                                  void* stream) {
    using namespace nmg;
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_noalloc: null cache");
    if (c->dtype == NMG_Q8_0) return set_error(NMG_UNSUPPORTED, "nmg_attend_noalloc: Q8_0 caches are not supported");
    if (hq <= 0 || hq % c->hkv != 0)
        return set_error(NMG_INVALID_ARGUMENT, "attention: %d query heads is not a multiple of %d K/V heads", hq, c->hkv);
    if (!dtype_valid(q_dtype) || !dtype_valid(out_dtype)) return set_error(NMG_INVALID_ARGUMENT, "attention: bad dtype");
    if (rows < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_noalloc: negative row count");
    if (rows == 0) return NMG_OK;
    if (!q || !out) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_noalloc: null tensor");
    if (c->size == 0 && c->total == 0)
        return set_error(NMG_RUNTIME_ERROR, "%s: query has no visible keys", c->window ? "LocalAttentionCache" : "FullAttentionCache");
    const int64_t newest = c->newest();
    for (int64_t t : {(int64_t)0, rows - 1}) {
        const VisibleSpan sp = visible_span(first_query + t, c->window, c->oldest, newest);
        if (sp.lo > sp.hi)
            return set_error(NMG_RUNTIME_ERROR, "%s: query has no visible keys",
                             c->window ? "LocalAttentionCache" : "FullAttentionCache");
    }
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != c->device) NMG_CUDA_TRY(cudaSetDevice(c->device));
    void* base = nullptr;
    int st = noalloc_scratch(c->device, &base);
    if (st == NMG_OK) {
        const int gtot = hq / c->hkv, gt = pick_gt(gtot), zdim = gtot / gt;
        int64_t longest = 0, total_keys = 0;
        for (int64_t t = 0; t < rows; ++t) {
            const VisibleSpan sp = visible_span(first_query + t, c->window, c->oldest, newest);
            longest = std::max(longest, sp.hi - sp.lo + 1);
            total_keys += sp.hi - sp.lo + 1;
        }
        // Work items the fixed array holds after the error word and the
        // tickets; nmg_attend's split length when they fit, otherwise longer
        // splits (fewer partials) so that every row's splits fit.
        const int warps = warps_runtime(c->dtype, c->dh);
        const int64_t tile = 32 * warps;
        const int64_t cnt_bytes = rows * c->hkv * zdim * 4;
        const int64_t cnt_span = (cnt_bytes + 255) / 256 * 256;
        const int64_t item_bytes = (int64_t)c->hkv * zdim * gt * (c->dh + 2) * 4;
        const int64_t avail = (int64_t)kNoallocScratchBytes - (int64_t)kNoallocFlagBytes - cnt_span;
        const int64_t max_items = avail > 0 ? avail / item_bytes : 0;
        const int64_t splits_cap = max_items / rows;
        int64_t split_len = pick_split_len(total_keys * c->hkv * zdim, warps);
        if (splits_cap >= 1 && (longest + split_len - 1) / split_len > splits_cap)
            split_len = ((longest + splits_cap - 1) / splits_cap + tile - 1) / tile * tile;
        const int64_t max_splits = (longest + split_len - 1) / split_len;
        const int64_t work = rows * max_splits;
        if (splits_cap < 1 || work > max_items || work > (int64_t)0x7FFFFFFF) {
            st = set_error(NMG_LENGTH_ERROR,
                           "nmg_attend_noalloc: %lld query rows need more scratch than the fixed %zu bytes hold "
                           "(at most %lld rows of %d query heads at head_dim %d); use nmg_attend or fewer rows",
                           (long long)rows, kNoallocScratchBytes, (long long)max_items, hq, c->dh);
        } else {
            SplitArgs a;  // on the stack: nothing is allocated
            a.mode = 0;
            a.hkv = c->hkv;
            a.hq = hq;
            a.gtot = gtot;
            a.zdim = zdim;
            a.split_len = split_len;
            a.k = c->k;
            a.v = c->v;
            a.slots = c->slots;
            a.base = c->base;
            a.rows = rows;
            a.first_query = first_query;
            a.window = c->window;
            a.floor_pos = c->oldest;
            a.newest = newest;
            a.max_splits = (int32_t)max_splits;
            a.nseq = 0;
            a.row_offset = 0;
            a.q = q;
            a.q_dtype = q_dtype;
            a.out = out;
            a.out_dtype = out_dtype;
            a.scale = use_scale ? scale : 1.f;
            a.err = (int*)base;  // never cleared here: nmg_device_status reports it
            a.counters = (int*)((char*)base + kNoallocFlagBytes);
            a.part = (float*)((char*)base + kNoallocFlagBytes + cnt_span);
            // The row tickets must start at zero; a kernel that gave up a
            // wait may have left some set, so clear them (not the error word).
            cudaError_t e = cudaMemsetAsync(a.counters, 0, (size_t)cnt_bytes, (cudaStream_t)stream);
            if (e != cudaSuccess)
                st = set_error(NMG_CUDA_ERROR, "nmg_attend_noalloc: cudaMemsetAsync: %s", cudaGetErrorString(e));
            else
                st = dispatch_split(c->dtype, c->dh, gt, a, dim3((unsigned)work, c->hkv, zdim), (cudaStream_t)stream);
        }
    }
    if (prev != c->device) cudaSetDevice(prev);
    return st;
}
