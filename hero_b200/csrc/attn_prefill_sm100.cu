// attn_prefill_sm100.cu -- causal / sliding-window GQA flash attention on the
// 5th-generation tensor cores (K4).
//
// A persistent kernel: one CTA per SM walks a list of units -- a 128-row
// query tile of one query head (or a key split of one) against the key
// blocks its rows can see -- heaviest first, reading K/V straight out of the
// device cache:
//
//   warp 0      TMA producer for Q (one tile per unit; the next unit's tile
//               is prefetched into L2) and K blocks (3-stage ring; a K stage
//               is released as soon as its S MMA completes; at head_dim 256
//               a ring of four 64-dimension pieces, one block)
//   warp 2      TMA producer for V blocks (2-stage ring, released after P.V;
//               at head_dim 256 two 64-key pieces, one block)
//               (cp.async.bulk.tensor, 128-byte swizzle, one CTA per copy)
//   warp 1      allocates TMEM and issues tcgen05.mma from one thread, one
//               stream over all units:
//                 S_g = Q K_g^T  (M=128, N=BN, K=DH)  into TMEM (two S buffers)
//                 O  += P_g V_g  (M=128, N=DH, K=BN)  A = P_g read from TMEM,
//                 O one of two accumulators by unit parity (head_dim 128)
//   warps 3..   softmax: two warps share each 32-row TMEM lane quadrant and
//               split every S row into two column ranges; they swap their
//               block maxima through shared memory, so both apply the same
//               running max.  Each thread reads its part of the row from
//               TMEM, applies the causal/window mask, an online softmax in
//               base 2 (rescaling O in TMEM only when the running max grows
//               by more than 2^8), writes P as packed fp16 pairs into TMEM
//               over the S buffer it came from (V is fp16 in every 16-bit
//               cache, so P.V is an fp16 MMA with 11-bit probabilities), and
//               leaves each unit's row sum and max for the epilogue.
//   last 4      epilogue: one warp per quadrant normalises a finished unit's
//               O and stores the rows (or split partials) while the softmax
//               works on the next unit.
//
// The equation is the reference reduction (nm/src/qwen35.hpp:360-382,
// nm/src/gemma4.hpp:593-615, :687-709): softmax over visible rows of
// scale * q.k, then the alpha-weighted sum of values; visibility is
// CausalWindow (nm/src/attention.hpp:154-176) in closed form per row.
#include <math.h>
#include <algorithm>
#include <functional>
#include <queue>
#include <vector>
#include <stdio.h>

#include "prefill.cuh"

namespace nmg {
namespace {

using namespace pf;

template <int DH, int BN_>
struct PfCfg {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    // K and V stream through shared memory in pieces, each with its own full
    // and empty barrier.  At head_dim 256 with 128-key blocks a block's K is
    // four pieces of 64 dimensions (an S MMA group frees each as it
    // completes) and its V two pieces of 64 keys, so a ring of one block each
    // still overlaps the loads with the MMAs; otherwise a piece is a block.
    static constexpr bool WIDE = DH == 256 && BN == 128;
    static constexpr int KP = WIDE ? 4 : 1;             // K pieces per block
    static constexpr int KRING = WIDE ? 4 : (DH == 256 ? 2 : 3);  // K ring, in pieces
    static constexpr int VP = WIDE ? 2 : 1;             // V pieces per block
    static constexpr int VRING = 2;                     // V ring, in pieces
    static constexpr int KDIMS = DH / KP;               // dimensions of a K piece
    static constexpr int VROWS = BN / VP;               // keys of a V piece
    static constexpr int Q_BYTES = BM * DH * 2;
    static constexpr int K_BYTES = BN * KDIMS * 2;      // one K piece
    static constexpr int V_BYTES = VROWS * DH * 2;      // one V piece
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + Q_BYTES;
    static constexpr int V_OFF = K_OFF + KRING * K_BYTES;
    static constexpr int BAR_OFF = V_OFF + VRING * V_BYTES;
    // q_full, q_empty, k_full/k_empty[KRING], v_full/v_empty[VRING], s_full[2], p_full[2], o_done,
    // o_final[2], o_free[2], l_full[2], quad[4]
    static constexpr int NBARS = 2 + 2 * KRING + 2 * VRING + 2 + 2 + 1 + 2 + 2 + 2 + 4;
    static constexpr int FLAGS_OFF = BAR_OFF + NBARS * 8;  // TMEM address, abort flag, last-split flag
    // Softmax warps per TMEM lane quadrant: each owns PART_N keys of a score
    // row and PART_D columns of its output row.
    static constexpr int PARTS = 2;
    static constexpr int RED_OFF = FLAGS_OFF + 16;                  // float [3][PARTS][BM]: max (2 parities), sum
    static constexpr int STATS_OFF = RED_OFF + 3 * PARTS * BM * 4;  // float2 [2][BM]: a work's (l, m) per row
    static constexpr int STAGE_OFF = (STATS_OFF + 2 * BM * 8 + 127) / 128 * 128;  // 4 epilogue warps x 32 rows x 128 B
    static constexpr int SMEM = STAGE_OFF + 4 * 32 * 128 + 1024;    // + slack to align the base to 1024
    static constexpr int SOFTMAX_THREADS = 128 * PARTS;
    static constexpr int EPI_WARP0 = 3 + SOFTMAX_THREADS / 32;
    static constexpr int THREADS = 96 + SOFTMAX_THREADS + 128;  // K producer, MMA, V producer, softmax, epilogue
    static constexpr int PART_N = BN / PARTS, PART_D = DH / PARTS;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t O_COL = 2 * BN;
    // Two O accumulators when TMEM has room: the epilogue of one work reads
    // one while the next work's P.V accumulates into the other.
    static constexpr int OBUF = O_COL + 2 * DH <= 512 ? 2 : 1;
    static_assert(O_COL + OBUF * DH <= 512, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(STATS_OFF % 8 == 0 && STAGE_OFF % 16 == 0, "vector accesses");
    static_assert(KDIMS % 64 == 0 && VROWS % 16 == 0 && K_BYTES % 1024 == 0 && V_BYTES % 1024 == 0, "pieces");
};

template <int DH, int BN_, bool BF16>
__global__ void __launch_bounds__(PfCfg<DH, BN_>::THREADS, 1) attn_prefill_kernel(const __grid_constant__ PrefillArgs a) {
    using C = PfCfg<DH, BN_>;
    constexpr int BM = C::BM, BN = C::BN, KRING = C::KRING, VRING = C::VRING, OBUF = C::OBUF;
    constexpr int KP = C::KP, VP = C::VP;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::BAR_OFF);
    uint64_t* q_full = bars;
    uint64_t* q_empty = q_full + 1;  // completes once per unit: its last S has read Q
    uint64_t* k_full = q_empty + 1;
    uint64_t* k_empty = k_full + KRING;
    uint64_t* v_full = k_empty + KRING;
    uint64_t* v_empty = v_full + VRING;
    uint64_t* s_full = v_empty + VRING;  // [2]
    // p_full[b] completes once per block of parity b: the softmax can never be
    // two phases ahead of the MMA thread's wait on it.
    uint64_t* p_full = s_full + 2;    // [2]
    uint64_t* o_done = p_full + 2;    // P.V of every block but a unit's last
    uint64_t* o_final = o_done + 1;   // [OBUF] a unit's last P.V
    uint64_t* o_free = o_final + 2;   // [OBUF] the epilogue has read O and the row statistics
    uint64_t* l_full = o_free + 2;    // [OBUF] the softmax has left a unit's (l, m)
    uint64_t* quad_bar = l_full + 2;  // [4], one arrival per softmax thread of the quadrant
    uint32_t* tmem_slot = (uint32_t*)(smem + C::FLAGS_OFF);
    volatile int* abort_flag = (volatile int*)(smem + C::FLAGS_OFF + 4);
    volatile int* last_flag = (volatile int*)(smem + C::FLAGS_OFF + 8);
    float2* stats = (float2*)(smem + C::STATS_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        dev::mbar_init(q_full, 1);
        dev::mbar_init(q_empty, 1);
        for (int s = 0; s < KRING; ++s) {
            dev::mbar_init(&k_full[s], 1);
            dev::mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VRING; ++s) {
            dev::mbar_init(&v_full[s], 1);
            dev::mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            dev::mbar_init(&s_full[b], 1);
            dev::mbar_init(&p_full[b], C::SOFTMAX_THREADS);
            dev::mbar_init(&o_final[b], 1);
            dev::mbar_init(&o_free[b], 128);
            dev::mbar_init(&l_full[b], 128);
        }
        dev::mbar_init(o_done, 1);
        for (int q = 0; q < 4; ++q) dev::mbar_init(&quad_bar[q], 32 * C::PARTS);
        *abort_flag = 0;
        *last_flag = 0;
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

    // Bounded wait; once any role gave up, every later wait that would block
    // returns at once (a completed phase is taken without reading the flag).
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (dev::mbar_test_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (dev::mbar_wait(bar, parity, a.err)) return true;
        *abort_flag = 1;
        return false;
    };
    auto kv_row = [&](const Work& w, int i) -> int32_t {
        const int64_t u0 = (w.j_begin + i) * BN;
        return (int32_t)((w.h / a.g) * a.slots + u0 % a.slots);
    };

    Work w;
    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ Q and K producer
            dev::prefetch_tensormap(&a.tm_q);
            dev::prefetch_tensormap(&a.tm_k);
            uint32_t g = 0;  // key blocks loaded so far (all units)
            int kn = 0;      // units with key blocks so far
            bool ok = true;
            for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
                if (w.nblk <= 0) continue;
                if (kn >= 1 && !wait(q_empty, (kn - 1) & 1)) break;  // the previous unit's S MMAs are done with Q
                dev::mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
                for (int c = 0; c < DH / 64; ++c)
                    dev::tma_load_3d(smem + C::Q_OFF + c * BM * 128, &a.tm_q, c * 64, w.h, (int32_t)w.t0, q_full);
                {
                    // The next unit's Q tile comes from HBM once: start it towards
                    // L2 now, so its load after this unit's last S finds it there.
                    Work nx;
                    if (decode_work<BM, BN>(a, k + 1, nx) && nx.nblk > 0)
#pragma unroll
                        for (int c = 0; c < DH / 64; ++c) dev::tma_prefetch_3d(&a.tm_q, c * 64, nx.h, (int32_t)nx.t0);
                }
                for (int i = 0; ok && i < w.nblk; ++i, ++g) {
                    const int32_t row = kv_row(w, i);
#pragma unroll 1
                    for (int p = 0; p < KP; ++p) {
                        const uint32_t gp = g * KP + p;  // K pieces loaded so far
                        const int s = gp % KRING;
                        if (gp >= KRING && !wait(&k_empty[s], ((gp / KRING) - 1) & 1)) {
                            ok = false;
                            break;
                        }
                        dev::mbar_arrive_expect_tx(&k_full[s], C::K_BYTES);
#pragma unroll
                        for (int c = 0; c < C::KDIMS / 64; ++c)
                            dev::tma_load_2d(smem + C::K_OFF + s * C::K_BYTES + c * BN * 128, &a.tm_k,
                                             p * C::KDIMS + c * 64, row, &k_full[s]);
                    }
                }
                ++kn;
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ------------------------------------------------ V producer
            dev::prefetch_tensormap(&a.tm_v);
            uint32_t g = 0;
            bool ok = true;
            for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
                for (int i = 0; ok && i < w.nblk; ++i, ++g) {
                    const int32_t row = kv_row(w, i);
#pragma unroll 1
                    for (int p = 0; p < VP; ++p) {
                        const uint32_t gp = g * VP + p;  // V pieces loaded so far
                        const int s = gp % VRING;
                        if (gp >= VRING && !wait(&v_empty[s], ((gp / VRING) - 1) & 1)) {
                            ok = false;
                            break;
                        }
                        dev::mbar_arrive_expect_tx(&v_full[s], C::V_BYTES);
#pragma unroll
                        for (int c = 0; c < DH / 64; ++c)
                            dev::tma_load_2d(smem + C::V_OFF + s * C::V_BYTES + c * C::VROWS * 128, &a.tm_v, c * 64,
                                             row + p * C::VROWS, &v_full[s]);
                    }
                }
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
            const uint64_t v_desc = tc::smem_desc_sw128(sbase + C::V_OFF, C::VROWS * 128, 1024);
            // P_gg . V_gg into O buffer ob; `first` starts the accumulator, the
            // unit's last P.V completes o_final[ob] instead of o_done.
            auto issue_pv = [&](uint32_t gg, bool first, bool last, int ob, int use) -> bool {
                if (!wait(&p_full[gg & 1], (gg >> 1) & 1)) return false;
                // the epilogue of the buffer's previous unit has read O
                if (first && use >= 1 && !wait(&o_free[ob], (use - 1) & 1)) return false;
                const uint32_t p_tmem = tmem + (gg & 1) * BN;  // P overwrote S, 2 values per column
#pragma unroll
                for (int p = 0; p < VP; ++p) {
                    const uint32_t gp = gg * VP + p;
                    const int s = gp % VRING;
                    if (!wait(&v_full[s], (gp / VRING) & 1)) return false;
                    tc::fence_after_sync();
                    const uint64_t vs = tc::desc_advance(v_desc, s * C::V_BYTES);
#pragma unroll
                    for (int kq = 0; kq < C::VROWS / 16; ++kq) {
                        const int k = p * (C::VROWS / 16) + kq;  // 16-key step of the block
                        tc::mma_f16_ts(tmem + C::O_COL + ob * DH, p_tmem + k * 8, tc::desc_advance(vs, kq * 2048),
                                       idesc_o, (!first || k > 0) ? 1u : 0u);
                    }
                    tc::commit(&v_empty[s]);
                }
                tc::commit(last ? &o_final[ob] : o_done);
                return true;
            };
            // One stream over all units: S_g, then P_{g-1}.V, so the next
            // unit's first S runs while the softmax finishes this unit's last
            // block (Q of the next unit is loaded once this unit's last S is done).
            uint32_t g = 0;
            int kn = 0;
            bool ok = true;
            bool pend = false;  // P_{g-1}.V still to issue, with its flags:
            bool pv_first = false, pv_last = false;
            int pv_ob = 0, pv_use = 0;
            for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
                if (w.nblk <= 0) continue;
                const int ob = kn % OBUF, use = kn / OBUF;
                if (!wait(q_full, kn & 1)) break;
                for (int i = 0; ok && i < w.nblk; ++i, ++g) {
                    const int sb = g & 1;
                    // S_g overwrites buffer sb, which held P_{g-2}; P_{g-2}.V was issued
                    // earlier and the tensor pipe executes in order.
#pragma unroll
                    for (int p = 0; p < KP; ++p) {
                        const uint32_t gp = g * KP + p;
                        const int s = gp % KRING;
                        if (!wait(&k_full[s], (gp / KRING) & 1)) {
                            ok = false;
                            break;
                        }
                        tc::fence_after_sync();
                        const uint64_t ks = tc::desc_advance(k_desc, s * C::K_BYTES);
#pragma unroll
                        for (int kq = 0; kq < C::KDIMS / 16; ++kq) {
                            const int kk = p * (C::KDIMS / 16) + kq;  // 16-dimension step of the head
                            tc::mma_f16_ss(tmem + sb * BN, tc::desc_advance(q_desc, (kk / 4) * BM * 128 + (kk % 4) * 32),
                                           tc::desc_advance(ks, (kq / 4) * BN * 128 + (kq % 4) * 32), idesc_s,
                                           kk > 0 ? 1u : 0u);
                        }
                        tc::commit(&k_empty[s]);
                    }
                    if (!ok) break;
                    tc::commit(&s_full[sb]);
                    if (i == w.nblk - 1) tc::commit(q_empty);
                    if (pend && !issue_pv(g - 1, pv_first, pv_last, pv_ob, pv_use)) {
                        ok = false;
                        break;
                    }
                    pend = true;
                    pv_first = i == 0;
                    pv_last = i == w.nblk - 1;
                    pv_ob = ob;
                    pv_use = use;
                }
                ++kn;
            }
            if (ok && pend) issue_pv(g - 1, pv_first, pv_last, pv_ob, pv_use);
        }
    } else if (warp < C::EPI_WARP0) {
        // ---------------------------------------------------- softmax warps
        const int quad = warp & 3;          // TMEM lane quadrant this warp may access
        const int part = (warp - 3) >> 2;   // which PART_N keys / PART_D output columns of the row
        const int row = quad * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        float* red = (float*)(smem + C::RED_OFF);  // [slot][part][row]; slots 0, 1: block maxima by parity, 2: sums
        const int col0 = part * C::PART_N;
        // The PARTS warps of one quadrant exchange through red[] and meet on
        // their quadrant mbarrier (completion k = exchange k; bounded wait).
        int quad_phase = 0;
        // The fences order this warp's TMEM reads before the other warps'
        // TMEM writes (P of one part lands on S columns of another).
        auto quad_sync = [&]() -> bool {
            tc::fence_before_sync();
            dev::mbar_arrive(&quad_bar[quad]);
            const bool done = __all_sync(0xffffffffu, wait(&quad_bar[quad], quad_phase & 1));
            tc::fence_after_sync();
            ++quad_phase;
            return done;
        };
        uint32_t g = 0, od = 0;
        int kn = 0;
        bool ok = true;
        for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
            if (w.nblk <= 0) continue;
            const int ob = kn % OBUF, use = kn / OBUF;
            const uint32_t o_col = C::O_COL + ob * DH;
            const int64_t qpos = a.first_query + w.t0 + row;
            const int64_t lo = vis_lo(a, qpos), hi = vis_hi(a, qpos);
            float m_run = -INFINITY, l_run = 0.f;
            for (int i = 0; i < w.nblk; ++i, ++g) {
                const int sb = g & 1;
                // Waits are voted warp-wide so the .sync.aligned TMEM accesses
                // below always see a converged warp.  S_g complete also means
                // P_{g-2}.V is complete (issued before it, in order).
                if (!__all_sync(0xffffffffu, wait(&s_full[sb], (g >> 1) & 1))) {
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
                const int64_t p0 = a.base + (w.j_begin + i) * BN + col0;
                if (!(p0 - col0 >= w.full_lo && p0 - col0 + BN - 1 <= w.full_hi)) {
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
                // one.  The MMA thread completes o_done for every P.V but a
                // unit's last, exactly the ones waited for here.
                if (i >= 1) {
                    if (!__all_sync(0xffffffffu, wait(o_done, od & 1))) {
                        ok = false;
                        break;
                    }
                    ++od;
                }
                // O is rescaled only after the previous P.V has landed in it.
                if (i >= 1 && __any_sync(0xffffffffu, rescale)) {
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < C::PART_D / 32; ++c) {
                        uint32_t r[32];
                        const uint32_t col = o_col + part * C::PART_D + c * 32;
                        tc::ld_32x32b_x32(t_lane + col, r);
#pragma unroll
                        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
                        tc::st_32x32b_x32(t_lane + col, r);
                    }
                }
                // P (fp16 pairs) over the first half of S's columns: this
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
            if (!ok) break;
            // Row sum = the parts' partial sums (slot 2; the previous unit's
            // readers are past a block exchange since).
            red[(2 * C::PARTS + part) * BM + row] = l_run;
            if (!quad_sync()) break;
            float l_row = 0.f;
#pragma unroll
            for (int q2 = 0; q2 < C::PARTS; ++q2) l_row += red[(2 * C::PARTS + q2) * BM + row];
            // The epilogue of the buffer's previous unit has read its statistics.
            if (use >= 1 && !__all_sync(0xffffffffu, wait(&o_free[ob], (use - 1) & 1))) break;
            if (part == 0) {
                stats[ob * BM + row] = make_float2(l_row, m_run);
                dev::mbar_arrive(&l_full[ob]);
            }
            ++kn;
        }
    } else {
        // ---------------------------------------------------- epilogue warps
        // One warp per TMEM lane quadrant: normalise a unit's O rows and store
        // them (or leave split partials and merge), while the softmax warps
        // already work on the next unit.
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int eid = threadIdx.x - 32 * C::EPI_WARP0;  // 0 .. 127
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        uint4* stage = (uint4*)(smem + C::STAGE_OFF + (warp - C::EPI_WARP0) * 4096);  // [32 rows][8 chunks]
        int kn = 0;
        for (int k = 0; decode_work<BM, BN>(a, k, w); ++k) {
            if (w.nblk <= 0) continue;
            const int ob = kn % OBUF, use = kn / OBUF;
            const uint32_t o_col = C::O_COL + ob * DH;
            // Waits are bounded, so all four warps reach the vote; a unit is
            // skipped by all of them or by none (the split path meets on
            // named barrier 1 below).
            bool have = wait(&l_full[ob], use & 1);
            have = wait(&o_final[ob], use & 1) && have;
            if (!bar_and(1, 128, __all_sync(0xffffffffu, have))) break;
            tc::fence_after_sync();
            const float2 st = stats[ob * BM + row];
            const float l_row = st.x, m_run = st.y;
            const int valid_rows = (int)(w.t_last - w.t0 + 1);
            if (w.nsplit == 1) {
                store_rows<DH>(a, w, w.h, t_lane, o_col, l_row, quad, lane, stage, &o_free[ob]);
            } else {
                store_partial<DH>(a, w, w.h, row, t_lane, o_col, m_run, l_row, &o_free[ob]);
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (eid == 0) {
                    int* ticket = a.tickets + (int64_t)w.h * a.ntiles + w.tile;
                    const int prev = atomicAdd(ticket, 1);
                    const bool last = prev == w.nsplit - 1;
                    if (last) *ticket = 0;  // ready for the next launch
                    *last_flag = last;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                const bool last = *last_flag;
                asm volatile("bar.sync 1, 128;" ::: "memory");  // every thread has read the flag
                if (last) {
                    __threadfence();
                    if (eid < valid_rows) merge_row<DH>(a, w, w.h, eid);
                }
            }
            ++kn;
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


template <int DH, int BN, bool BF16>
int launch_prefill(const PrefillArgs& a, dim3 grid, cudaStream_t s) {
    using C = PfCfg<DH, BN>;
    auto kern = attn_prefill_kernel<DH, BN, BF16>;
    static std::atomic<uint64_t> attr_set{0};  // one bit per device
    const int st = set_smem_once(kern, C::SMEM, attr_set);
    if (st != NMG_OK) return st;
    kern<<<grid, C::THREADS, C::SMEM, s>>>(a);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace

// A split item's partial store and merge, in key blocks of the same CTA's
// time: measured on 480 split items of a 12-head, 2520-token dense launch
// (78 us split against 60 us whole, 34 against 40 blocks of makespan).
constexpr double kSplitItemBlocks = 5.0;

// Makespan, in key blocks, of placing unit loads longest first on `ctas` CTAs,
// each on the least loaded one.
static int64_t lpt_makespan(std::vector<int> loads, int ctas) {
    std::sort(loads.begin(), loads.end(), std::greater<int>());
    std::priority_queue<int64_t, std::vector<int64_t>, std::greater<int64_t>> q;
    for (int i = 0; i < ctas; ++i) q.push(0);
    int64_t mk = 0;
    for (int l : loads) {
        const int64_t t = q.top() + l;
        q.pop();
        mk = std::max(mk, t);
        q.push(t);
    }
    return mk;
}

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

// Keys per block of the one-head kernel: 128, or 64 at head_dim 256 when the
// cache's slots are not a multiple of 128 (a block never straddles a head).
static int prefill_block_keys(const nmg_kv_cache* c) { return c->dh == 256 && c->slots % 128 != 0 ? 64 : 128; }

bool prefill_supported(const nmg_kv_cache* c, int hq, int q_dtype, int64_t rows) {
    if (c->dtype == NMG_F32 || q_dtype != c->dtype) return false;
    if (c->dh != 64 && c->dh != 128 && c->dh != 256) return false;
    if (c->slots % prefill_block_keys(c) != 0) return false;
    if (rows < 64) return false;
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
    // Two query heads of one GQA group a unit (they share every K/V block)
    // where the group is even; one head a unit otherwise.
    // Two heads per unit when the pair units alone fill the GPU; with fewer
    // (a sharded launch's few heads) a pair unit's two heads would run in
    // series on one SM, so the heaviest causal tile takes twice as long as
    // with one head per unit.
    const bool pair = dh == 128 && (hq / c->hkv) % 2 == 0 && (rows + 127) / 128 * (hq / 2) >= 148;
    const int bn = pair ? 128 : prefill_block_keys(c);
    // Rows per V copy: a V piece is half a 128-key block at head_dim 256.
    const int v_rows = !pair && dh == 256 && bn == 128 ? 64 : bn;
    for (int which = 0; which < 2; ++which) {
        cuuint64_t dims[2] = {(cuuint64_t)dh, (cuuint64_t)c->hkv * (cuuint64_t)c->slots};
        cuuint64_t strides[1] = {(cuuint64_t)dh * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)(which ? v_rows : bn)};
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
    a->hunits = pair ? hq / 2 : hq;
    a->scale_log2 = scale * 1.4426950408889634f;
    // Key splits when one CTA per query tile would leave the GPU's 148 SMs
    // idle: under two waves of CTAs, cut the tiles into pieces for about two
    // waves.  With more CTAs the heavy-first order already balances the grid
    // and the partials' round trip would only cost.
    const int ntiles = (int)((rows + 127) / 128);
    a->n_items = 0;
    a->split_blocks = 0;
    a->nparts = 0;
    a->ntiles = ntiles;
    a->part = nullptr;
    a->tickets = nullptr;
    if (ntiles <= kMaxTiles && (int64_t)ntiles * a->hunits < 2 * 148) {
        std::vector<int> nb(ntiles);
        int64_t total = 0;
        int maxb = 0, minb = 1 << 30;
        for (int t = 0; t < ntiles; ++t) {
            const int64_t qf = first_query + (int64_t)t * 128, ql = first_query + std::min<int64_t>((int64_t)t * 128 + 128, rows) - 1;
            int64_t lo = floor_pos;
            if (window > 0 && qf - window + 1 > lo) lo = qf - window + 1;
            const int64_t hi = ql < newest ? ql : newest;
            nb[t] = (int)((hi - c->base) / bn + 1 - (lo - c->base) / bn);
            total += (int64_t)nb[t] * a->hunits;
            maxb = std::max(maxb, nb[t]);
            minb = std::min(minb, nb[t]);
        }
        int sb = (int)std::max<int64_t>(8, (total + 2 * 148 - 1) / (2 * 148));
        sb = std::max(sb, (maxb + 62) / 63);  // at most 63 splits per tile
        // Only tiles that all see the same keys (dense attention) are split:
        // under a causal mask with few heads per GPU (sharded launches), split
        // pieces and their merges ran slower than whole tiles, e.g. 4 query
        // heads over 4096 tokens 99 against 75 us, head_dim 256 with one
        // head over 8192 tokens 262 against 120 us.
        if (maxb > sb && minb == maxb) {
            std::vector<std::pair<int, uint32_t>> items;  // (blocks, packed item)
            int parts = 0;
            for (int t = 0; t < ntiles; ++t) {
                const int ns = (nb[t] + sb - 1) / sb;
                a->part_base[t] = (uint32_t)parts;
                parts += ns;
                for (int sp = 0; sp < ns; ++sp)
                    items.push_back({std::min(sb, nb[t] - sp * sb), ((uint32_t)t << 12) | ((uint32_t)sp << 6) | (uint32_t)ns});
            }
            // Split only when it shortens the launch: greedy longest-first
            // makespans in key blocks (the unit order the CTAs walk), the
            // split plan charged kSplitItemBlocks per item for its partial
            // store and merge.
            std::vector<int> whole, pieces;
            for (int t = 0; t < ntiles; ++t) whole.insert(whole.end(), a->hunits, nb[t]);
            for (const auto& it : items) pieces.insert(pieces.end(), a->hunits, it.first);
            const double m0 = (double)lpt_makespan(whole, 148);
            const double m1 = (double)lpt_makespan(pieces, 148) + kSplitItemBlocks * (double)pieces.size() / 148.0;
            if ((int)items.size() <= kMaxItems && m1 < m0) {
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
        // Persistent CTAs, one per SM, walk the unit list (heaviest first).
        a->n_work = (int64_t)(a->n_items > 0 ? a->n_items : ntiles) * a->hunits;
        int nsm = 148;
        if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, c->device) != cudaSuccess) nsm = 148;
        const dim3 grid((unsigned)std::min<int64_t>(a->n_work, nsm));
        if (pair)
            st = launch_prefill_pair(*a, dh, c->dtype == NMG_BF16, grid, stream);
        else if (dh == 64)
            st = c->dtype == NMG_BF16 ? launch_prefill<64, 128, true>(*a, grid, stream)
                                      : launch_prefill<64, 128, false>(*a, grid, stream);
        else if (dh == 128)
            st = c->dtype == NMG_BF16 ? launch_prefill<128, 128, true>(*a, grid, stream)
                                      : launch_prefill<128, 128, false>(*a, grid, stream);
        else if (bn == 128)
            st = c->dtype == NMG_BF16 ? launch_prefill<256, 128, true>(*a, grid, stream)
                                      : launch_prefill<256, 128, false>(*a, grid, stream);
        else
            st = c->dtype == NMG_BF16 ? launch_prefill<256, 64, true>(*a, grid, stream)
                                      : launch_prefill<256, 64, false>(*a, grid, stream);
    }
    delete a;
    return st;
}

}  // namespace nmg
