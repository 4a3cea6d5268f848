// attn_prefill_sm100.cu -- causal / sliding-window GQA flash attention on the
// 5th-generation tensor cores (K4).
//
// One CTA computes a 128-row query tile of one query head against the key
// blocks its rows can see, reading K/V straight out of the device cache:
//
//   warp 0      TMA producer for Q (once) and K blocks (3-stage ring; a K
//               stage is released as soon as its S MMA completes)
//   warp 2      TMA producer for V blocks (2-stage ring, released after P.V)
//               (cp.async.bulk.tensor, 128-byte swizzle, one CTA per copy)
//   warp 1      allocates TMEM and issues tcgen05.mma from one thread:
//                 S_j = Q K_j^T  (M=128, N=BN, K=DH)  into TMEM (two S buffers)
//                 O  += P_j V_j  (M=128, N=DH, K=BN)  A = P_j read from TMEM
//   warps 3..   softmax: PARTS warps (4 for head_dim 128, 2 for 256) share
//               each 32-row TMEM lane quadrant and split every S row into
//               PARTS column ranges; they swap their block maxima through
//               shared memory, so all apply the same running max (four warps
//               per scheduler hide each other's TMEM and barrier latency).
//               Each thread reads its part of the row from TMEM, applies the
//               causal/window mask, an online softmax in base 2
//               (rescaling O in TMEM only when the running max grows by more
//               than 2^8), writes P as packed fp16 pairs into TMEM over the
//               S buffer it came from (V is fp16 in every 16-bit cache, so
//               P.V is an fp16 MMA with 11-bit probabilities), and at the end
//               normalises O and stores the row.
//
// The equation is the reference reduction (nm/src/qwen35.hpp:360-382,
// nm/src/gemma4.hpp:593-615, :687-709): softmax over visible rows of
// scale * q.k, then the alpha-weighted sum of values; visibility is
// CausalWindow (nm/src/attention.hpp:154-176) in closed form per row.
#include <math.h>
#include <algorithm>
#include <vector>
#include <stdio.h>

#include "attn.cuh"
#include "tcgen05.cuh"

namespace nmg {
namespace {

template <int DH>
struct PfCfg {
    static constexpr int BM = 128;
    static constexpr int BN = DH == 128 ? 128 : 64;
    static constexpr int KST = DH == 128 ? 3 : 2;  // K stages (K is released as soon as S is computed)
    static constexpr int VST = 2;  // V stages (released after P.V)
    static constexpr int Q_BYTES = BM * DH * 2;
    static constexpr int K_BYTES = BN * DH * 2;
    static constexpr int V_BYTES = BN * DH * 2;
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + Q_BYTES;
    static constexpr int V_OFF = K_OFF + KST * K_BYTES;
    static constexpr int BAR_OFF = V_OFF + VST * V_BYTES;
    // q_full, k_full/k_empty[KST], v_full/v_empty[VST], s_full[2], p_full[2], o_done, quad[4]
    static constexpr int NBARS = 1 + 2 * KST + 2 * VST + 2 + 2 + 1 + 4;
    static constexpr int TMEMPTR_OFF = BAR_OFF + NBARS * 8;
    // Softmax warps per TMEM lane quadrant: each owns PART_N keys of a score
    // row and PART_D columns of its output row.
    static constexpr int PARTS = DH == 128 ? 4 : 2;
    static constexpr int RED_OFF = TMEMPTR_OFF + 16;                  // float [2 parity][PARTS][BM]
    static constexpr int SMEM = RED_OFF + 2 * PARTS * BM * 4 + 1024;  // + slack to align the base to 1024
    static constexpr int SOFTMAX_THREADS = 128 * PARTS;
    static constexpr int THREADS = 96 + SOFTMAX_THREADS;  // K producer, MMA, V producer, softmax warps
    static constexpr int PART_N = BN / PARTS, PART_D = DH / PARTS;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t O_COL = 2 * BN;
    static_assert(O_COL + DH <= 512, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory budget");
};

constexpr int kMaxFanout = 8;
constexpr int kMaxItems = 2048;  // work items of a split launch
constexpr int kMaxTiles = 1024;  // query tiles of a split launch

struct PrefillArgs {
    CUtensorMap tm_q;  // (d, head, row) over q [rows][hq*DH]
    CUtensorMap tm_k;  // (d, hkv*slots) over the cache
    CUtensorMap tm_v;
    int64_t rows, first_query, window, floor_pos, newest, base, slots;
    int hq, hkv, g;
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
    // Key splits (n_items > 0): CTA x takes items[x] = tile << 12 | split << 6 |
    // nsplit, keys blocks [split * split_blocks, +split_blocks) of the tile's
    // range.  A split tile's CTAs leave (O, m, l) partials in part (slot
    // part_base[tile] + split of head h: [BM][DH + 4] fp32, O then m, l, with
    // rows padded to 16 bytes) and the last one
    // to finish (ticket per head and tile) merges them.  n_items == 0: one
    // CTA per tile, heaviest tile first.
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

__device__ __forceinline__ int64_t vis_lo(const PrefillArgs& a, int64_t q) {
    int64_t lo = a.floor_pos;
    if (a.window > 0 && q - a.window + 1 > lo) lo = q - a.window + 1;
    return lo;
}
__device__ __forceinline__ int64_t vis_hi(const PrefillArgs& a, int64_t q) { return q < a.newest ? q : a.newest; }

template <int DH, bool BF16>
__global__ void __launch_bounds__(PfCfg<DH>::THREADS, 1) attn_prefill_kernel(const __grid_constant__ PrefillArgs a) {
    using C = PfCfg<DH>;
    constexpr int BM = C::BM, BN = C::BN, KST = C::KST, VST = C::VST;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::BAR_OFF);
    uint64_t* q_full = bars;
    uint64_t* k_full = q_full + 1;
    uint64_t* k_empty = k_full + KST;
    uint64_t* v_full = k_empty + KST;
    uint64_t* v_empty = v_full + VST;
    uint64_t* s_full = v_empty + VST;  // [2]
    // p_full[b] completes once per block of parity b: the softmax can never be
    // two phases ahead of the MMA thread's wait on it.
    uint64_t* p_full = s_full + 2;  // [2]
    uint64_t* o_done = p_full + 2;
    uint64_t* quad_bar = o_done + 1;  // [4], one arrival per softmax thread of the quadrant
    uint32_t* tmem_slot = (uint32_t*)(smem + C::TMEMPTR_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The grid is (head, work item) with the head fastest, so CTAs start in
    // order of decreasing work over all heads (longest-first balancing).
    int tile, split = 0, nsplit = 1;
    if (a.n_items > 0) {
        const uint32_t it = a.items[blockIdx.y];
        tile = (int)(it >> 12);
        split = (int)((it >> 6) & 63u);
        nsplit = (int)(it & 63u);
    } else {
        tile = gridDim.y - 1 - blockIdx.y;  // heaviest tiles first
    }
    const int h = blockIdx.x;
    const int hk = h / a.g;
    const int64_t t0 = (int64_t)tile * BM;
    const int64_t t_last = (t0 + BM < a.rows ? t0 + BM : a.rows) - 1;
    const int64_t q_first = a.first_query + t0, q_last = a.first_query + t_last;
    const int64_t u_lo = vis_lo(a, q_first) - a.base;
    const int64_t u_hi = vis_hi(a, q_last) - a.base;
    const int nblk_all = (int)(u_hi / BN + 1 - u_lo / BN);
    const int64_t j_begin = u_lo / BN + (int64_t)split * a.split_blocks;
    const int nblk = nsplit == 1 ? nblk_all : min(a.split_blocks, nblk_all - split * a.split_blocks);
    // A block needs no mask when every row of the tile sees all of it.
    const int64_t full_lo = vis_lo(a, q_last), full_hi = vis_hi(a, q_first);

    if (threadIdx.x == 0) {
        dev::mbar_init(q_full, 1);
        for (int s = 0; s < KST; ++s) {
            dev::mbar_init(&k_full[s], 1);
            dev::mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VST; ++s) {
            dev::mbar_init(&v_full[s], 1);
            dev::mbar_init(&v_empty[s], 1);
        }
        dev::mbar_init(&s_full[0], 1);
        dev::mbar_init(&s_full[1], 1);
        dev::mbar_init(&p_full[0], C::SOFTMAX_THREADS);
        dev::mbar_init(&p_full[1], C::SOFTMAX_THREADS);
        dev::mbar_init(o_done, 1);
        for (int q = 0; q < 4; ++q) dev::mbar_init(&quad_bar[q], 32 * C::PARTS);
        dev::fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    auto kv_row = [&](int i) -> int32_t {
        const int64_t u0 = (j_begin + i) * BN;
        return (int32_t)(hk * a.slots + u0 % a.slots);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ Q and K producer
            dev::prefetch_tensormap(&a.tm_q);
            dev::prefetch_tensormap(&a.tm_k);
            dev::mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
            for (int c = 0; c < DH / 64; ++c)
                dev::tma_load_3d(smem + C::Q_OFF + c * BM * 128, &a.tm_q, c * 64, h, (int32_t)t0, q_full);
            for (int i = 0; i < nblk; ++i) {
                const int s = i % KST;
                if (i >= KST && !dev::mbar_wait(&k_empty[s], ((i / KST) - 1) & 1, a.err)) break;
                dev::mbar_arrive_expect_tx(&k_full[s], C::K_BYTES);
                const int32_t row = kv_row(i);
#pragma unroll
                for (int c = 0; c < DH / 64; ++c)
                    dev::tma_load_2d(smem + C::K_OFF + s * C::K_BYTES + c * BN * 128, &a.tm_k, c * 64, row, &k_full[s]);
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ------------------------------------------------ V producer
            dev::prefetch_tensormap(&a.tm_v);
            for (int i = 0; i < nblk; ++i) {
                const int s = i % VST;
                if (i >= VST && !dev::mbar_wait(&v_empty[s], ((i / VST) - 1) & 1, a.err)) break;
                dev::mbar_arrive_expect_tx(&v_full[s], C::V_BYTES);
                const int32_t row = kv_row(i);
#pragma unroll
                for (int c = 0; c < DH / 64; ++c)
                    dev::tma_load_2d(smem + C::V_OFF + s * C::V_BYTES + c * BN * 128, &a.tm_v, c * 64, row, &v_full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc_s = tc::idesc_f16(128, BN, BF16 ? 1 : 0, 0, 0);
            // P.V runs fp16 x fp16 (V of a 16-bit cache is stored fp16), A = P from TMEM.
            constexpr uint32_t idesc_o = tc::idesc_f16(128, DH, 0, 0, 1);
            const uint32_t sbase = dev::smem_u32(smem);
            // Descriptors are built once; each MMA only advances a start address.
            const uint64_t q_desc = tc::smem_desc_sw128(sbase + C::Q_OFF, 16, 1024);
            const uint64_t k_desc = tc::smem_desc_sw128(sbase + C::K_OFF, 16, 1024);
            const uint64_t v_desc = tc::smem_desc_sw128(sbase + C::V_OFF, BN * 128, 1024);
            bool ok = dev::mbar_wait(q_full, 0, a.err);
            auto issue_pv = [&](int i) -> bool {
                const int s = i % VST;
                if (!dev::mbar_wait(&p_full[i & 1], (i >> 1) & 1, a.err)) return false;
                if (!dev::mbar_wait(&v_full[s], (i / VST) & 1, a.err)) return false;
                tc::fence_after_sync();
                const uint32_t p_tmem = tmem + (i & 1) * BN;  // P_i overwrote S_i, 2 values per column
                const uint64_t vs = tc::desc_advance(v_desc, s * C::V_BYTES);
#pragma unroll
                for (int k = 0; k < BN / 16; ++k)
                    tc::mma_f16_ts(tmem + C::O_COL, p_tmem + k * 8, tc::desc_advance(vs, k * 2048), idesc_o,
                                   (i > 0 || k > 0) ? 1u : 0u);
                tc::commit(o_done);
                tc::commit(&v_empty[s]);
                return true;
            };
            for (int i = 0; ok && i < nblk; ++i) {
                const int s = i % KST, sb = i & 1;
                if (!dev::mbar_wait(&k_full[s], (i / KST) & 1, a.err)) break;
                tc::fence_after_sync();
                // S_i overwrites buffer sb, which held P_{i-2}; P_{i-2}.V was issued
                // earlier and the tensor pipe executes in order.
                const uint64_t ks = tc::desc_advance(k_desc, s * C::K_BYTES);
#pragma unroll
                for (int k = 0; k < DH / 16; ++k)
                    tc::mma_f16_ss(tmem + sb * BN, tc::desc_advance(q_desc, (k / 4) * BM * 128 + (k % 4) * 32),
                                   tc::desc_advance(ks, (k / 4) * BN * 128 + (k % 4) * 32), idesc_s, k > 0 ? 1u : 0u);
                tc::commit(&s_full[sb]);
                tc::commit(&k_empty[s]);
                if (i >= 1 && !issue_pv(i - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && nblk > 0) issue_pv(nblk - 1);
        }
    } else {
        // ---------------------------------------------------- softmax warps
        const int quad = warp & 3;          // TMEM lane quadrant this warp may access
        const int part = (warp - 3) >> 2;   // which PART_N keys / PART_D output columns of the row
        const int row = quad * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        const int64_t qpos = a.first_query + t0 + row;
        const int64_t lo = vis_lo(a, qpos), hi = vis_hi(a, qpos);
        float* red = (float*)(smem + C::RED_OFF);  // [parity][part][row]
        const int col0 = part * C::PART_N;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        // The PARTS warps of one quadrant exchange through red[] and meet on
        // their quadrant mbarrier (completion k = exchange k; bounded wait).
        int quad_phase = 0;
        // The fences order this warp's TMEM reads before the other warps'
        // TMEM writes (P of one part lands on S columns of another).
        auto quad_sync = [&]() -> bool {
            tc::fence_before_sync();
            dev::mbar_arrive(&quad_bar[quad]);
            const bool done = __all_sync(0xffffffffu, dev::mbar_wait(&quad_bar[quad], quad_phase & 1, a.err));
            tc::fence_after_sync();
            ++quad_phase;
            return done;
        };

        for (int i = 0; i < nblk; ++i) {
            const int sb = i & 1;
            // Waits are voted warp-wide so the .sync.aligned TMEM accesses
            // below always see a converged warp.  S_i complete also means
            // P_{i-2}.V is complete (issued before it, in order).
            if (!__all_sync(0xffffffffu, dev::mbar_wait(&s_full[sb], (i >> 1) & 1, a.err))) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            // Raw scores: the maximum is taken before scaling (scale_log2 > 0)
            // and the scale is folded into the exponent's FFMA below.
            float x[C::PART_N];
#pragma unroll
            for (int c = 0; c < C::PART_N / 32; ++c) {
                uint32_t r[32];
                tc::ld_32x32b_x32(t_lane + sb * BN + col0 + c * 32, r);
#pragma unroll
                for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(r[e]);
            }

            const int64_t p0 = a.base + (j_begin + i) * BN + col0;
            if (!(p0 - col0 >= full_lo && p0 - col0 + BN - 1 <= full_hi)) {
#pragma unroll
                for (int e = 0; e < C::PART_N; ++e) {
                    const int64_t pos = p0 + e;
                    if (pos < lo || pos > hi) x[e] = -INFINITY;
                }
            }
            float mb = x[0];
#pragma unroll
            for (int e = 1; e < C::PART_N; ++e) mb = fmaxf(mb, x[e]);
            mb *= a.scale_log2;
            red[(sb * C::PARTS + part) * BM + row] = mb;
            if (!quad_sync()) {
                ok = false;
                break;
            }
#pragma unroll
            for (int q2 = 0; q2 < C::PARTS; ++q2) mb = fmaxf(mb, red[(sb * C::PARTS + q2) * BM + row]);
            const float m_new = fmaxf(m_run, mb);
            const bool rescale = m_new > m_run + 8.0f;  // also true for the first finite block
            float alpha = 1.f;
            if (rescale) {
                alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_new);
                m_run = m_new;
            }
            const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
            float sum = 0.f;
            uint32_t pk[C::PART_N / 2];
#pragma unroll
            for (int e = 0; e < C::PART_N; e += 2) {
                const float p0v = ex2(fmaf(x[e], a.scale_log2, -m_use)), p1v = ex2(fmaf(x[e + 1], a.scale_log2, -m_use));
                sum += p0v + p1v;
                pk[e / 2] = pack2(p0v, p1v, false);
            }
            l_run = l_run * alpha + sum;

            // Every o_done phase is waited for, in order: a parity wait only
            // tells the current phase from the previous one, so a waiter that
            // skipped a phase could mistake an unfinished P.V for a finished
            // one.  P_{i-1}.V is normally long done by now.
            if (i >= 1 && !__all_sync(0xffffffffu, dev::mbar_wait(o_done, (i - 1) & 1, a.err))) {
                ok = false;
                break;
            }
            // O is rescaled only after P_{i-1}.V has landed in it.
            if (i >= 1 && __any_sync(0xffffffffu, rescale)) {
                tc::fence_after_sync();
#pragma unroll 1
                for (int c = 0; c < C::PART_D / 32; ++c) {
                    uint32_t r[32];
                    const uint32_t col = C::O_COL + part * C::PART_D + c * 32;
                    tc::ld_32x32b_x32(t_lane + col, r);
#pragma unroll
                    for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
                    tc::st_32x32b_x32(t_lane + col, r);
                }
            }
            // P_i (fp16 pairs) over the first half of S_i's columns: this
            // part's keys [col0, col0 + PART_N) -> columns [col0/2, col0/2 + PART_N/2).
            const uint32_t pcol = t_lane + sb * BN + col0 / 2;
            if constexpr (C::PART_N / 2 == 32) {
                tc::st_32x32b_x32(pcol, *reinterpret_cast<const uint32_t(*)[32]>(pk));
            } else {
                tc::st_32x32b_x16(pcol, pk);
            }
            tc::wait_st();
            tc::fence_before_sync();
            dev::mbar_arrive(&p_full[sb]);
        }

        // Row sum = the parts' partial sums.  The slot of parity nblk & 1 was
        // last read for block nblk - 2, which every part is past.
        const int ls = nblk & 1;
        red[(ls * C::PARTS + part) * BM + row] = l_run;
        if (ok) ok = quad_sync();
        float l_row = 0.f;
#pragma unroll
        for (int q2 = 0; q2 < C::PARTS; ++q2) l_row += red[(ls * C::PARTS + q2) * BM + row];
        // Epilogue: normalise O.  With one local output every thread stores
        // its own row part.  With several (other GPUs' memory among them) the
        // tile is staged in shared memory (the Q and K stages are idle now:
        // every MMA has completed) and all softmax threads copy whole row
        // segments (DH * out_es contiguous bytes per row) to each output, so
        // a warp writes two or more full segments per store instead of 32
        // rows' 16-byte pieces, which NVLink carries far less efficiently.
        const bool have_o = ok && nblk > 0 && __all_sync(0xffffffffu, dev::mbar_wait(o_done, (nblk - 1) & 1, a.err));
        if (nsplit > 1) {
            // A split of a tile: leave the unnormalised O with its m and l
            // (base-2 units), and the last split of the tile merges them.
            float* mine = a.part + (((int64_t)h * a.nparts + a.part_base[tile] + split) * BM + row) * (DH + 4);
            if (have_o) {
                tc::fence_after_sync();
#pragma unroll 1
                for (int c = 0; c < C::PART_D / 32; ++c) {
                    uint32_t r[32];
                    tc::ld_32x32b_x32(t_lane + C::O_COL + part * C::PART_D + c * 32, r);
                    float4* dst = (float4*)(mine + part * C::PART_D + c * 32);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                             __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
                }
                if (part == 0) {
                    mine[DH] = m_run;
                    mine[DH + 1] = l_row;
                }
            }
            __threadfence();
            asm volatile("bar.sync 2, %0;" ::"r"(C::SOFTMAX_THREADS) : "memory");
            int* last_flag = (int*)(smem + C::RED_OFF);  // red[] is no longer read
            if (threadIdx.x == 96) {
                int* ticket = a.tickets + (int64_t)h * a.ntiles + tile;
                const int prev = atomicAdd(ticket, 1);
                const bool last = prev == nsplit - 1;
                if (last) *ticket = 0;  // ready for the next launch
                *last_flag = last;
            }
            asm volatile("bar.sync 2, %0;" ::"r"(C::SOFTMAX_THREADS) : "memory");
            if (*last_flag) {
                __threadfence();
                const int sid = threadIdx.x - 96;
                const int valid_rows = (int)(t_last - t0 + 1);
                const float* base = a.part + ((int64_t)h * a.nparts + a.part_base[tile]) * BM * (DH + 4);
                const int64_t slot = (int64_t)BM * (DH + 4);
                const int oes = a.out_dtype == NMG_F32 ? 4 : 2;
                // 4 output columns per work unit
                for (int idx = sid; idx < valid_rows * (DH / 4); idx += C::SOFTMAX_THREADS) {
                    const int rr = idx / (DH / 4), d0 = (idx - rr * (DH / 4)) * 4;
                    float M = -INFINITY;
                    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(base + sp * slot + rr * (DH + 4) + DH));
                    float L = 0.f, o4[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int sp = 0; sp < nsplit; ++sp) {
                        const float* rp = base + sp * slot + rr * (DH + 4);
                        const float m = __ldcg(rp + DH);
                        if (m == -INFINITY) continue;
                        const float w = ex2(m - M);
                        L = fmaf(w, __ldcg(rp + DH + 1), L);
                        const float4 v = __ldcg((const float4*)(rp + d0));
                        o4[0] = fmaf(w, v.x, o4[0]), o4[1] = fmaf(w, v.y, o4[1]);
                        o4[2] = fmaf(w, v.z, o4[2]), o4[3] = fmaf(w, v.w, o4[3]);
                    }
                    const float inv = 1.f / L;
                    const int64_t off = ((t0 + rr) * a.out_row_elems + a.out_col0 + (int64_t)h * DH + d0) * oes;
                    if (a.out_dtype == NMG_F32) {
                        const float4 v = make_float4(o4[0] * inv, o4[1] * inv, o4[2] * inv, o4[3] * inv);
                        for (int o = 0; o < a.nout; ++o) *(float4*)((unsigned char*)a.outs[o] + off) = v;
                    } else {
                        const bool obf = a.out_dtype == NMG_BF16;
                        uint32_t w[2];
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            const float f0 = o4[2 * t] * inv, f1 = o4[2 * t + 1] * inv;
                            const uint32_t b0 = obf ? dev::f32_to_bf16_bits(f0) : dev::f32_to_f16_bits(f0);
                            const uint32_t b1 = obf ? dev::f32_to_bf16_bits(f1) : dev::f32_to_f16_bits(f1);
                            w[t] = b0 | (b1 << 16);
                        }
                        for (int o = 0; o < a.nout; ++o) *(uint2*)((unsigned char*)a.outs[o] + off) = make_uint2(w[0], w[1]);
                    }
                }
            }
        }
        const int oes = a.out_dtype == NMG_F32 ? 4 : 2;
        const int cpr = DH * oes / 16;  // 16-byte chunks per row: 16, 32 or 64
        unsigned char* stage = smem + C::Q_OFF;
        if (nsplit == 1 && have_o && a.nout == 1) {  // one local output: each thread stores its own row part
            tc::fence_after_sync();
            const float inv = 1.f / l_row;
            const bool row_valid = t0 + row < a.rows;
            const int64_t obase = (t0 + row) * a.out_row_elems + a.out_col0 + (int64_t)h * DH + part * C::PART_D;
#pragma unroll 1
            for (int c = 0; c < C::PART_D / 32; ++c) {
                uint32_t r[32];
                tc::ld_32x32b_x32(t_lane + C::O_COL + part * C::PART_D + c * 32, r);
                if (!row_valid) continue;
                if (a.out_dtype == NMG_F32) {
                    uint4* dst = (uint4*)((float*)a.outs[0] + obase + c * 32);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        dst[e] = make_uint4(__float_as_uint(__uint_as_float(r[4 * e]) * inv),
                                            __float_as_uint(__uint_as_float(r[4 * e + 1]) * inv),
                                            __float_as_uint(__uint_as_float(r[4 * e + 2]) * inv),
                                            __float_as_uint(__uint_as_float(r[4 * e + 3]) * inv));
                } else {
                    const bool obf = a.out_dtype == NMG_BF16;
                    uint4* dst = (uint4*)((uint16_t*)a.outs[0] + obase + c * 32);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        uint32_t w[4];
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float f0 = __uint_as_float(r[8 * e + 2 * t]) * inv;
                            const float f1 = __uint_as_float(r[8 * e + 2 * t + 1]) * inv;
                            const uint32_t b0 = obf ? dev::f32_to_bf16_bits(f0) : dev::f32_to_f16_bits(f0);
                            const uint32_t b1 = obf ? dev::f32_to_bf16_bits(f1) : dev::f32_to_f16_bits(f1);
                            w[t] = b0 | (b1 << 16);
                        }
                        dst[e] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        } else if (nsplit == 1 && have_o) {
            tc::fence_after_sync();
            const float inv = 1.f / l_row;
#pragma unroll 1
            for (int c = 0; c < C::PART_D / 32; ++c) {
                uint32_t r[32];
                tc::ld_32x32b_x32(t_lane + C::O_COL + part * C::PART_D + c * 32, r);
                const int col = part * C::PART_D + c * 32;  // first of this thread's 32 columns
                if (a.out_dtype == NMG_F32) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int ch = col / 4 + e;
                        *(uint4*)(stage + row * cpr * 16 + ((ch ^ (row & 15)) << 4)) =
                            make_uint4(__float_as_uint(__uint_as_float(r[4 * e]) * inv),
                                       __float_as_uint(__uint_as_float(r[4 * e + 1]) * inv),
                                       __float_as_uint(__uint_as_float(r[4 * e + 2]) * inv),
                                       __float_as_uint(__uint_as_float(r[4 * e + 3]) * inv));
                    }
                } else {
                    const bool obf = a.out_dtype == NMG_BF16;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        uint32_t w[4];
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float f0 = __uint_as_float(r[8 * e + 2 * t]) * inv;
                            const float f1 = __uint_as_float(r[8 * e + 2 * t + 1]) * inv;
                            const uint32_t b0 = obf ? dev::f32_to_bf16_bits(f0) : dev::f32_to_f16_bits(f0);
                            const uint32_t b1 = obf ? dev::f32_to_bf16_bits(f1) : dev::f32_to_f16_bits(f1);
                            w[t] = b0 | (b1 << 16);
                        }
                        const int ch = col / 8 + e;
                        *(uint4*)(stage + row * cpr * 16 + ((ch ^ (row & 15)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
        // Every softmax thread reaches this barrier (have_o is uniform across
        // the CTA: the o_done wait is the same for all, and a timeout sets the
        // error flag but still arrives here).
        if (nsplit == 1) asm volatile("bar.sync 2, %0;" ::"r"(C::SOFTMAX_THREADS) : "memory");
        if (nsplit == 1 && have_o && a.nout > 1) {
            const int sid = threadIdx.x - 96;  // 0 .. SOFTMAX_THREADS - 1
            const int valid_rows = (int)(t_last - t0 + 1);
            const int64_t col_base = a.out_col0 + (int64_t)h * DH;
            for (int idx = sid; idx < valid_rows * cpr; idx += C::SOFTMAX_THREADS) {
                const int rr = idx / cpr, ch = idx - rr * cpr;
                const uint4 val = *(const uint4*)(stage + rr * cpr * 16 + ((ch ^ (rr & 15)) << 4));
                const int64_t off = ((t0 + rr) * a.out_row_elems + col_base) * oes + ch * 16;
                for (int o = 0; o < a.nout; ++o) *(uint4*)((unsigned char*)a.outs[o] + off) = val;
            }
            // No fence here: the caller orders these stores before any read of
            // the rows with a stream-ordered barrier (nmg_comm_barrier), which
            // starts only after this grid, stores included, has completed.
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side


template <int DH, bool BF16>
int launch_prefill(const PrefillArgs& a, dim3 grid, cudaStream_t s) {
    using C = PfCfg<DH>;
    auto kern = attn_prefill_kernel<DH, BF16>;
    static unsigned attr_set = 0;
    int dev_id = 0;
    NMG_CUDA_TRY(cudaGetDevice(&dev_id));
    if (!(attr_set & (1u << (dev_id & 31)))) {
        NMG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_set |= 1u << (dev_id & 31);
    }
    kern<<<grid, C::THREADS, C::SMEM, s>>>(a);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace

int make_kv_tensor_maps(const nmg_kv_cache* c, int box_rows, CUtensorMap* k, CUtensorMap* v) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(NMG_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)c->k & 15) || ((uintptr_t)c->v & 15)) return set_error(NMG_UNSUPPORTED, "unaligned cache");
    for (int which = 0; which < 2; ++which) {
        const int dt = which ? c->vdtype : c->dtype;
        const CUtensorMapDataType t = dt == NMG_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : dt == NMG_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        const int es = dtype_size(dt);
        cuuint64_t dims[2] = {(cuuint64_t)c->dh, (cuuint64_t)c->hkv * (cuuint64_t)c->slots};
        cuuint64_t strides[1] = {(cuuint64_t)c->dh * es};
        cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
        cuuint32_t estr[2] = {1, 1};
        const CUresult r = enc(which ? v : k, t, 2, which ? c->v : c->k, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(NMG_CUDA_ERROR, "K/V tensor map (%d)", (int)r);
    }
    return NMG_OK;
}

bool prefill_supported(const nmg_kv_cache* c, int hq, int q_dtype, int64_t rows) {
    if (c->dtype == NMG_F32 || q_dtype != c->dtype) return false;
    if (c->dh != 128 && c->dh != 256) return false;
    const int bn = c->dh == 128 ? 128 : 64;
    if (c->slots % bn != 0) return false;
    if (rows < 64 || (rows + 127) / 128 > 65535) return false;  // query tiles index the grid's y
    if ((int64_t)c->hkv * c->slots > 0x7FFFFFFF) return false;
    return encode_tiled_fn() != nullptr;
}

int attend_rows_prefill(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                        int64_t window, int64_t floor_pos, int64_t newest, float scale, void* const* outs, int nout,
                        int64_t out_row_elems, int64_t out_col0, int out_dtype, cudaStream_t stream) {
    if (nout < 1 || nout > kMaxFanout) return set_error(NMG_INVALID_ARGUMENT, "prefill: %d outputs (1..%d)", nout, kMaxFanout);
    const int es = dtype_size(out_dtype);
    if (((out_row_elems * es) | (out_col0 * es)) & 15)
        return set_error(NMG_UNSUPPORTED, "prefill: output rows and column offset must be 16-byte multiples");
    for (int i = 0; i < nout; ++i)
        if (!outs[i] || ((uintptr_t)outs[i] & 15)) return set_error(NMG_INVALID_ARGUMENT, "prefill: output %d unaligned", i);
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(NMG_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)q & 15) || ((uintptr_t)c->k & 15) || ((uintptr_t)c->v & 15))
        return set_error(NMG_UNSUPPORTED, "prefill: 16-byte aligned tensors required");
    const int dh = c->dh;
    const CUtensorMapDataType dt = c->dtype == NMG_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    PrefillArgs* a = new PrefillArgs();
    {
        cuuint64_t dims[3] = {(cuuint64_t)dh, (cuuint64_t)hq, (cuuint64_t)rows};
        cuuint64_t strides[2] = {(cuuint64_t)dh * 2, (cuuint64_t)hq * dh * 2};
        cuuint32_t box[3] = {64, 1, 128};
        cuuint32_t es[3] = {1, 1, 1};
        CUresult r = enc(&a->tm_q, dt, 3, (void*)q, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            delete a;
            return set_error(NMG_CUDA_ERROR, "prefill: Q tensor map (%d)", (int)r);
        }
    }
    const int bn = dh == 128 ? 128 : 64;
    for (int which = 0; which < 2; ++which) {
        cuuint64_t dims[2] = {(cuuint64_t)dh, (cuuint64_t)c->hkv * (cuuint64_t)c->slots};
        cuuint64_t strides[1] = {(cuuint64_t)dh * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)bn};
        cuuint32_t es[2] = {1, 1};
        const CUtensorMapDataType wdt = which ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : dt;
        CUresult r = enc(which ? &a->tm_v : &a->tm_k, wdt, 2, which ? c->v : c->k, dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            delete a;
            return set_error(NMG_CUDA_ERROR, "prefill: K/V tensor map (%d)", (int)r);
        }
    }
    a->rows = rows;
    a->first_query = first_query;
    a->window = window;
    a->floor_pos = floor_pos;
    a->newest = newest;
    a->base = c->base;
    a->slots = c->slots;
    a->hq = hq;
    a->hkv = c->hkv;
    a->g = hq / c->hkv;
    a->scale_log2 = scale * 1.4426950408889634f;
    // Key splits when one CTA per query tile would leave the GPU's 148 SMs
    // waiting on the heaviest tiles (a causal tile sees as many key blocks
    // as its index): under two waves of CTAs, cut the tiles into pieces for
    // about two waves.  With more CTAs the heavy-first order already
    // balances the grid and the partials' round trip would only cost.
    const int ntiles = (int)((rows + 127) / 128);
    a->n_items = 0;
    a->split_blocks = 0;
    a->nparts = 0;
    a->ntiles = ntiles;
    a->part = nullptr;
    a->tickets = nullptr;
    if (ntiles <= kMaxTiles && (int64_t)ntiles * hq < 2 * 148) {
        std::vector<int> nb(ntiles);
        int64_t total = 0;
        int maxb = 0;
        for (int t = 0; t < ntiles; ++t) {
            const int64_t qf = first_query + (int64_t)t * 128, ql = first_query + std::min<int64_t>((int64_t)t * 128 + 128, rows) - 1;
            int64_t lo = floor_pos;
            if (window > 0 && qf - window + 1 > lo) lo = qf - window + 1;
            const int64_t hi = ql < newest ? ql : newest;
            nb[t] = (int)((hi - c->base) / bn + 1 - (lo - c->base) / bn);
            total += (int64_t)nb[t] * hq;
            maxb = std::max(maxb, nb[t]);
        }
        int sb = (int)std::max<int64_t>(8, (total + 2 * 148 - 1) / (2 * 148));
        sb = std::max(sb, (maxb + 62) / 63);  // at most 63 splits per tile
        if (maxb > sb) {
            std::vector<std::pair<int, uint32_t>> items;  // (blocks, packed item)
            int parts = 0;
            for (int t = 0; t < ntiles; ++t) {
                const int ns = (nb[t] + sb - 1) / sb;
                a->part_base[t] = (uint32_t)parts;
                parts += ns;
                for (int sp = 0; sp < ns; ++sp)
                    items.push_back({std::min(sb, nb[t] - sp * sb), ((uint32_t)t << 12) | ((uint32_t)sp << 6) | (uint32_t)ns});
            }
            if ((int)items.size() <= kMaxItems) {
                std::stable_sort(items.begin(), items.end(), [](const std::pair<int, uint32_t>& x, const std::pair<int, uint32_t>& y) { return x.first > y.first; });
                for (size_t i = 0; i < items.size(); ++i) a->items[i] = items[i].second;
                void* part = nullptr;
                void* tickets = nullptr;
                int st = device_scratch(c->device, (size_t)hq * parts * 128 * (dh + 4) * sizeof(float), &part);
                if (st == NMG_OK) st = device_tickets(c->device, (size_t)hq * ntiles * sizeof(int), &tickets);
                if (st != NMG_OK) {
                    delete a;
                    return st;
                }
                a->n_items = (int)items.size();
                a->split_blocks = sb;
                a->nparts = parts;
                a->part = (float*)part;
                a->tickets = (int*)tickets;
            }
        }
    }
    for (int i = 0; i < nout; ++i) a->outs[i] = outs[i];
    a->nout = nout;
    a->out_row_elems = out_row_elems;
    a->out_col0 = out_col0;
    a->out_dtype = out_dtype;
    int st = device_error_flag(c->device, &a->err);
    if (st == NMG_OK) {
        dim3 grid((unsigned)hq, a->n_items > 0 ? (unsigned)a->n_items : (unsigned)ntiles);
        if (dh == 128)
            st = c->dtype == NMG_BF16 ? launch_prefill<128, true>(*a, grid, stream) : launch_prefill<128, false>(*a, grid, stream);
        else
            st = c->dtype == NMG_BF16 ? launch_prefill<256, true>(*a, grid, stream) : launch_prefill<256, false>(*a, grid, stream);
    }
    delete a;
    return st;
}

}  // namespace nmg
