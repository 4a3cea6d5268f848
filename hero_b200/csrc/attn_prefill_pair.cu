// attn_prefill_pair.cu -- causal / sliding-window GQA flash attention on the
// 5th-generation tensor cores, two query heads of one GQA group per unit
// (K4, head_dim 128).
//
// Query heads 2p and 2p + 1 read the same K/V head whenever the GQA group is
// even (head h reads K/V head h / (Hq / Hkv)), so one unit takes the same
// 128-row query tile of both heads (tiles A and B) against the key blocks the
// tile's rows can see: every K and V block staged in shared memory feeds two
// S MMAs and two P.V MMAs, and the two tiles' softmax steps run side by side
// on separate warps, each overlapping the other tile's MMAs.  A persistent
// kernel: one CTA per SM walks the unit list heaviest first.
//
//   warp 0      TMA producer for Q (both heads' tiles per unit; the next
//               unit's tiles are prefetched into L2) and K blocks (2 stages,
//               a stage released once both S MMAs have read it)
//   warp 1      allocates TMEM and issues tcgen05.mma from one thread:
//                 per key block g:  P_A(g-1).V, S_A(g), P_B(g-1).V, S_B(g)
//                 S_t = Q_t K^T (M=128, N=128, K=128) into TMEM S_t,
//                 O_t += P_t V  (M=128, N=128, K=128), A = P_t from TMEM
//   warp 2      TMA producer for V blocks (2 stages, released after P_B.V)
//   warp 3      idle (the next warps start on TMEM lane quadrant 0)
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B: one thread
//               per row, all 128 keys of a block (maximum over both column
//               halves, then base-2 exponentials, P as packed fp16 over the
//               first half of the S columns), rescaling O in TMEM only when
//               the running max grows by more than 2^8
//   warps 12-15 epilogue: normalise and store each finished unit's rows of
//               both heads (or leave key-split partials and merge them)
//
// TMEM: S_A, S_B, O_A, O_B, 128 columns each.  S_t(g) is issued after
// P_t(g-1).V, so its completion also means the previous P.V into O_t has
// landed: the softmax may rescale O_t as soon as it sees S_t(g).
//
// The equation is the reference reduction (nm/src/qwen35.hpp:360-382,
// nm/src/gemma4.hpp:593-615, :687-709): softmax over visible rows of
// scale * q.k, then the alpha-weighted sum of values; visibility is
// CausalWindow (nm/src/attention.hpp:154-176) in closed form per row.
#include <type_traits>

#include "prefill.cuh"

namespace nmg {
namespace {

using namespace pf;

struct PairCfg {
    static constexpr int DH = 128, BM = 128, BN = 128;
    static constexpr int KST = 2, VST = 2;
    static constexpr int Q_BYTES = BM * DH * 2;  // one head's tile
    static constexpr int K_BYTES = BN * DH * 2;
    static constexpr int V_BYTES = BN * DH * 2;
    static constexpr int Q_OFF = 0;  // tile A, then tile B
    static constexpr int K_OFF = Q_OFF + 2 * Q_BYTES;
    static constexpr int V_OFF = K_OFF + KST * K_BYTES;
    static constexpr int STAGE_OFF = V_OFF + VST * V_BYTES;  // 4 epilogue warps x 32 rows x 128 B
    static constexpr int BAR_OFF = STAGE_OFF + 4 * 32 * 128;
    // q_full, q_empty, k_full/k_empty[KST], v_full/v_empty[VST],
    // per tile: s_full, p_full, o_final, o_free, l_full
    static constexpr int NBARS = 2 + 2 * KST + 2 * VST + 2 * 5;
    static constexpr int FLAGS_OFF = BAR_OFF + NBARS * 8;  // TMEM address, abort flag, last-split flag
    static constexpr int STATS_OFF = FLAGS_OFF + 16;       // float2 [2][BM]: a unit's (l, m) per row and tile
    static constexpr int SMEM = STATS_OFF + 2 * BM * 8 + 1024;  // + slack to align the base to 1024
    static constexpr int THREADS = 512;
    static constexpr int SOFTMAX_WARP0 = 4, EPI_WARP0 = 12;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t O_COL = 2 * BN;  // O_t at O_COL + t * DH; S_t at t * BN
    static_assert(O_COL + 2 * DH <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(Q_OFF % 1024 == 0 && K_OFF % 1024 == 0 && V_OFF % 1024 == 0, "128-byte swizzle atoms");
    static_assert(STATS_OFF % 8 == 0 && STAGE_OFF % 16 == 0, "vector accesses");
};

template <bool BF16>
__global__ void __launch_bounds__(PairCfg::THREADS, 1) attn_prefill_pair_kernel(const __grid_constant__ PrefillArgs a) {
    using C = PairCfg;
    constexpr int BM = C::BM, BN = C::BN, DH = C::DH, KST = C::KST, VST = C::VST;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::BAR_OFF);
    uint64_t* q_full = bars;
    uint64_t* q_empty = q_full + 1;  // completes once per unit: its last S MMAs have read both Q tiles
    uint64_t* k_full = q_empty + 1;
    uint64_t* k_empty = k_full + KST;
    uint64_t* v_full = k_empty + KST;
    uint64_t* v_empty = v_full + VST;
    uint64_t* s_full = v_empty + VST;  // [2] per tile, once per key block
    uint64_t* p_full = s_full + 2;     // [2] per tile, once per key block (128 softmax threads)
    uint64_t* o_final = p_full + 2;    // [2] a unit's last P.V of the tile
    uint64_t* o_free = o_final + 2;    // [2] the epilogue has read the tile's O and statistics
    uint64_t* l_full = o_free + 2;     // [2] the softmax has left the tile's (l, m)
    uint32_t* tmem_slot = (uint32_t*)(smem + C::FLAGS_OFF);
    volatile int* abort_flag = (volatile int*)(smem + C::FLAGS_OFF + 4);
    volatile int* last_flag = (volatile int*)(smem + C::FLAGS_OFF + 8);
    float2* stats = (float2*)(smem + C::STATS_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        dev::mbar_init(q_full, 1);
        dev::mbar_init(q_empty, 1);
        for (int s = 0; s < KST; ++s) {
            dev::mbar_init(&k_full[s], 1);
            dev::mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VST; ++s) {
            dev::mbar_init(&v_full[s], 1);
            dev::mbar_init(&v_empty[s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            dev::mbar_init(&s_full[t], 1);
            dev::mbar_init(&p_full[t], 128);
            dev::mbar_init(&o_final[t], 1);
            dev::mbar_init(&o_free[t], 128);
            dev::mbar_init(&l_full[t], 128);
        }
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
    // Cache row of key block i of a unit (both heads of the pair read K/V head 2h / g).
    auto kv_row = [&](const Work& w, int i) -> int32_t {
        const int64_t u0 = (w.j_begin + i) * BN;
        return (int32_t)(((2 * w.h) / a.g) * a.slots + u0 % a.slots);
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
                dev::mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
#pragma unroll
                for (int t = 0; t < 2; ++t)
#pragma unroll
                    for (int c = 0; c < DH / 64; ++c)
                        dev::tma_load_3d(smem + C::Q_OFF + t * C::Q_BYTES + c * BM * 128, &a.tm_q, c * 64, 2 * w.h + t,
                                         (int32_t)w.t0, q_full);
                {
                    // The next unit's Q tiles come from HBM once: start them towards
                    // L2 now, so their load after this unit's last S finds them there.
                    Work nx;
                    if (decode_work<BM, BN>(a, k + 1, nx) && nx.nblk > 0)
#pragma unroll
                        for (int t = 0; t < 2; ++t)
#pragma unroll
                            for (int c = 0; c < DH / 64; ++c)
                                dev::tma_prefetch_3d(&a.tm_q, c * 64, 2 * nx.h + t, (int32_t)nx.t0);
                }
                for (int i = 0; i < w.nblk; ++i, ++g) {
                    const int s = g % KST;
                    if (g >= KST && !wait(&k_empty[s], ((g / KST) - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    dev::mbar_arrive_expect_tx(&k_full[s], C::K_BYTES);
                    const int32_t row = kv_row(w, i);
#pragma unroll
                    for (int c = 0; c < DH / 64; ++c)
                        dev::tma_load_2d(smem + C::K_OFF + s * C::K_BYTES + c * BN * 128, &a.tm_k, c * 64, row, &k_full[s]);
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
                for (int i = 0; i < w.nblk; ++i, ++g) {
                    const int s = g % VST;
                    if (g >= VST && !wait(&v_empty[s], ((g / VST) - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    dev::mbar_arrive_expect_tx(&v_full[s], C::V_BYTES);
                    const int32_t row = kv_row(w, i);
#pragma unroll
                    for (int c = 0; c < DH / 64; ++c)
                        dev::tma_load_2d(smem + C::V_OFF + s * C::V_BYTES + c * BN * 128, &a.tm_v, c * 64, row, &v_full[s]);
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
            const uint64_t q_desc = tc::smem_desc_sw128(sbase + C::Q_OFF, 16, 1024);
            const uint64_t k_desc = tc::smem_desc_sw128(sbase + C::K_OFF, 16, 1024);
            const uint64_t v_desc = tc::smem_desc_sw128(sbase + C::V_OFF, BN * 128, 1024);
            // P_t(gg) . V(gg) into O_t; `first` starts the accumulator (after the
            // epilogue has read the tile's previous unit), `last` completes o_final.
            auto issue_pv = [&](int t, uint32_t gg, bool first, bool last, int use) -> bool {
                const int s = gg % VST;
                if (!wait(&p_full[t], gg & 1)) return false;
                if (t == 0 && !wait(&v_full[s], (gg / VST) & 1)) return false;
                if (first && use >= 1 && !wait(&o_free[t], (use - 1) & 1)) return false;
                tc::fence_after_sync();
                const uint64_t vs = tc::desc_advance(v_desc, s * C::V_BYTES);
                const uint32_t p_tmem = tmem + t * BN;  // P overwrote S, 2 values per column
#pragma unroll
                for (int k = 0; k < BN / 16; ++k)
                    tc::mma_f16_ts(tmem + C::O_COL + t * DH, p_tmem + k * 8, tc::desc_advance(vs, k * 2048), idesc_o,
                                   (!first || k > 0) ? 1u : 0u);
                if (last) tc::commit(&o_final[t]);
                if (t == 1) tc::commit(&v_empty[s]);
                return true;
            };
            // S_t(gg) = Q_t . K(gg)^T into S_t (which held P_t(gg-1), already
            // issued to the in-order tensor pipe).
            auto issue_s = [&](int t, uint32_t gg) {
                const int s = gg % KST;
                const uint64_t ks = tc::desc_advance(k_desc, s * C::K_BYTES);
                const uint64_t qs = tc::desc_advance(q_desc, t * C::Q_BYTES);
#pragma unroll
                for (int kk = 0; kk < DH / 16; ++kk)
                    tc::mma_f16_ss(tmem + t * BN, tc::desc_advance(qs, (kk / 4) * BM * 128 + (kk % 4) * 32),
                                   tc::desc_advance(ks, (kk / 4) * BN * 128 + (kk % 4) * 32), idesc_s, kk > 0 ? 1u : 0u);
                tc::commit(&s_full[t]);
            };
            uint32_t g = 0;
            int kn = 0;
            bool ok = true;
            bool pend = false;  // P(g-1).V of both tiles still to issue, with its flags:
            bool pv_first = false, pv_last = false;
            int pv_use = 0;
            for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
                if (w.nblk <= 0) continue;
                if (!wait(q_full, kn & 1)) break;
                for (int i = 0; i < w.nblk; ++i, ++g) {
                    const int s = g % KST;
                    if (!wait(&k_full[s], (g / KST) & 1)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    for (int t = 0; t < 2 && ok; ++t) {
                        if (pend && !issue_pv(t, g - 1, pv_first, pv_last, pv_use)) {
                            ok = false;
                            break;
                        }
                        issue_s(t, g);
                    }
                    if (!ok) break;
                    tc::commit(&k_empty[s]);
                    if (i == w.nblk - 1) tc::commit(q_empty);
                    pend = true;
                    pv_first = i == 0;
                    pv_last = i == w.nblk - 1;
                    pv_use = kn;
                }
                ++kn;
            }
            if (ok && pend)
                for (int t = 0; t < 2; ++t)
                    if (!issue_pv(t, g - 1, pv_first, pv_last, pv_use)) break;
        }
    } else if (warp == 3) {
        // idle: keeps the softmax and epilogue warps aligned to TMEM lane quadrants
    } else if (warp < C::EPI_WARP0) {
        // ---------------------------------------------------- softmax warps
        const int t = (warp - C::SOFTMAX_WARP0) >> 2;  // tile A (0) or B (1)
        const int quad = warp & 3;                     // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t s_col = t * BN, o_col = C::O_COL + t * DH;
        uint32_t g = 0;
        int kn = 0;
        bool ok = true;
        for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
            if (w.nblk <= 0) continue;
            const int use = kn;
            const int64_t qpos = a.first_query + w.t0 + row;
            const int64_t lo = vis_lo(a, qpos), hi = vis_hi(a, qpos);
            float m_run = -INFINITY, l_run = 0.f;
            for (int i = 0; i < w.nblk; ++i, ++g) {
                // Waits are voted warp-wide so the .sync.aligned TMEM accesses
                // below always see a converged warp.
                if (!__all_sync(0xffffffffu, wait(&s_full[t], g & 1))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const int64_t p0 = a.base + (w.j_begin + i) * BN;  // position of the block's key 0
                // Keys [k_lo, k_hi) of the block are visible to this row; the
                // mask is applied only on blocks some row of the tile cannot
                // fully see (a warp-uniform branch).
                const bool masked = !(p0 >= w.full_lo && p0 + BN - 1 <= w.full_hi);
                int k_lo = 0, k_hi = BN;
                if (masked) {
                    k_lo = (int)max((int64_t)0, min((int64_t)BN, lo - p0));
                    k_hi = (int)max((int64_t)0, min((int64_t)BN, hi - p0 + 1));
                }
                // Raw scores: the maximum is taken before scaling (scale_log2 > 0)
                // and the scale is folded into the exponent's FFMA below.  Keys
                // 64..127 first (32 at a time, for the maximum only), then 0..63,
                // which stay in registers.  Four independent max chains.
                float x[64];
                float mb4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                auto scores = [&](auto mask_tag) {
                    constexpr bool M = decltype(mask_tag)::value;
#pragma unroll
                    for (int c = 2; c < 4; ++c) {
                        uint32_t r[32];
                        tc::ld_32x32b_x32(t_lane + s_col + c * 32, r);
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            float v = __uint_as_float(r[e]);
                            if (M && (c * 32 + e < k_lo || c * 32 + e >= k_hi)) v = -INFINITY;
                            mb4[e & 3] = fmaxf(mb4[e & 3], v);
                        }
                    }
                    uint32_t r[64];
                    tc::ld_32x32b_x64(t_lane + s_col, r);
#pragma unroll
                    for (int e = 0; e < 64; ++e) {
                        x[e] = __uint_as_float(r[e]);
                        if (M && (e < k_lo || e >= k_hi)) x[e] = -INFINITY;
                        mb4[e & 3] = fmaxf(mb4[e & 3], x[e]);
                    }
                };
                if (masked)
                    scores(std::true_type{});
                else
                    scores(std::false_type{});
                float mb = fmaxf(fmaxf(mb4[0], mb4[1]), fmaxf(mb4[2], mb4[3]));
                mb *= a.scale_log2;
                const float m_new = fmaxf(m_run, mb);
                const bool rescale = m_new > m_run + 8.0f;  // also true for the first finite block
                float alpha = 1.f;
                if (rescale) {
                    alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_new);
                    m_run = m_new;
                }
                const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
                // O_t holds the blocks before this one (S_t(g) completing means
                // P_t(g-1).V has landed); within a unit it is rescaled only when
                // the running max grew by more than 2^8.
                if (i >= 1 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
                    for (int c = 0; c < DH / 32; ++c) {
                        uint32_t r[32];
                        tc::ld_32x32b_x32(t_lane + o_col + c * 32, r);
#pragma unroll
                        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
                        tc::st_32x32b_x32(t_lane + o_col + c * 32, r);
                    }
                }
                // P as fp16 pairs: keys 2j, 2j + 1 -> column j of S_t, over
                // columns whose scores were read already.  Keys 0..63 from
                // registers, then 64..127 again from TMEM, 32 at a time.  Four
                // independent sum chains.
                float sum4[4] = {0.f, 0.f, 0.f, 0.f};
                const float sl2 = a.scale_log2;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float pa = ex2(fmaf(x[c * 32 + e], sl2, -m_use));
                        const float pb = ex2(fmaf(x[c * 32 + e + 1], sl2, -m_use));
                        sum4[(e >> 1) & 3] += pa + pb;
                        pk[e / 2] = pack2(pa, pb, false);
                    }
                    tc::st_32x32b_x16(t_lane + s_col + c * 16, pk);
                }
                auto exps_hi = [&](auto mask_tag) {
                    constexpr bool M = decltype(mask_tag)::value;
#pragma unroll
                    for (int c = 2; c < 4; ++c) {
                        uint32_t r[32];
                        tc::ld_32x32b_x32(t_lane + s_col + c * 32, r);
                        uint32_t pk[16];
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            float va = __uint_as_float(r[e]), vb = __uint_as_float(r[e + 1]);
                            if (M && (c * 32 + e < k_lo || c * 32 + e >= k_hi)) va = -INFINITY;
                            if (M && (c * 32 + e + 1 < k_lo || c * 32 + e + 1 >= k_hi)) vb = -INFINITY;
                            const float pa = ex2(fmaf(va, sl2, -m_use)), pb = ex2(fmaf(vb, sl2, -m_use));
                            sum4[(e >> 1) & 3] += pa + pb;
                            pk[e / 2] = pack2(pa, pb, false);
                        }
                        tc::st_32x32b_x16(t_lane + s_col + c * 16, pk);
                    }
                };
                if (masked)
                    exps_hi(std::true_type{});
                else
                    exps_hi(std::false_type{});
                const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
                l_run = l_run * alpha + sum;
                tc::wait_st();
                tc::fence_before_sync();
                dev::mbar_arrive(&p_full[t]);
            }
            if (!ok) break;
            // The epilogue has read the tile's statistics of the previous unit.
            if (use >= 1 && !__all_sync(0xffffffffu, wait(&o_free[t], (use - 1) & 1))) break;
            stats[t * BM + row] = make_float2(l_run, m_run);
            dev::mbar_arrive(&l_full[t]);
            ++kn;
        }
    } else {
        // ---------------------------------------------------- epilogue warps
        // One warp per TMEM lane quadrant: normalise a unit's O rows of both
        // heads and store them (or leave split partials and merge), while the
        // softmax warps already work on the next unit.
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int eid = threadIdx.x - 32 * C::EPI_WARP0;  // 0 .. 127
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        uint4* stage = (uint4*)(smem + C::STAGE_OFF + (warp - C::EPI_WARP0) * 4096);  // [32 rows][8 chunks]
        int kn = 0;
        bool ok = true;
        for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
            if (w.nblk <= 0) continue;
            const int use = kn;
            for (int t = 0; t < 2; ++t) {
                // Waits are bounded, so all four warps reach the vote; a tile is
                // skipped by all of them or by none.
                bool have = wait(&l_full[t], use & 1);
                have = wait(&o_final[t], use & 1) && have;
                if (!bar_and(1, 128, __all_sync(0xffffffffu, have))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const float2 st = stats[t * BM + row];
                const uint32_t o_col = C::O_COL + t * DH;
                if (w.nsplit == 1)
                    store_rows<DH>(a, w, 2 * w.h + t, t_lane, o_col, st.x, quad, lane, stage, &o_free[t]);
                else
                    store_partial<DH>(a, w, 2 * w.h + t, row, t_lane, o_col, st.y, st.x, &o_free[t]);
            }
            if (!ok) break;
            if (w.nsplit > 1) {
                // The last split of the tile (ticket per head pair and tile) merges both heads.
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
                    const int valid_rows = (int)(w.t_last - w.t0 + 1);
                    if (eid < valid_rows) {
                        merge_row<DH>(a, w, 2 * w.h, eid);
                        merge_row<DH>(a, w, 2 * w.h + 1, eid);
                    }
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

template <bool BF16>
int launch_pair(const PrefillArgs& a, dim3 grid, cudaStream_t s) {
    auto kern = attn_prefill_pair_kernel<BF16>;
    static std::atomic<uint64_t> attr_set{0};  // one bit per device
    const int st = set_smem_once(kern, PairCfg::SMEM, attr_set);
    if (st != NMG_OK) return st;
    kern<<<grid, PairCfg::THREADS, PairCfg::SMEM, s>>>(a);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace

int launch_prefill_pair(const pf::PrefillArgs& a, int dh, bool bf16, dim3 grid, cudaStream_t s) {
    if (dh != 128) return set_error(NMG_UNSUPPORTED, "prefill: the two-head kernel is built for head_dim 128");
    return bf16 ? launch_pair<true>(a, grid, s) : launch_pair<false>(a, grid, s);
}

}  // namespace nmg
