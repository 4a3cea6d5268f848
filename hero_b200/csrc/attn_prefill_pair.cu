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
//   warps 4-7   tile A, warps 8-11 tile B, one thread per row: the softmax
//               of every key block (all 128 scores of the row in registers
//               from one TMEM load, the block maximum, base-2 exponentials,
//               P as packed fp16 over the first half of the S columns, O in
//               TMEM rescaled only when the running max grows by more than
//               2^8), then the unit's epilogue: normalise and store the
//               tile's rows (or leave key-split partials and merge them).
//               The other tile's softmax keeps the tensor core busy meanwhile.
//
// 384 threads, so each holds 168 registers: a whole score row fits.
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
    static constexpr int STAGE_OFF = V_OFF + VST * V_BYTES;  // 2 tiles x 4 warps x 32 rows x 128 B
    static constexpr int BAR_OFF = STAGE_OFF + 2 * 4 * 32 * 128;
    // q_full, q_empty, k_full/k_empty[KST], v_full/v_empty[VST],
    // per tile: s_full, p_full, o_final, o_free
    static constexpr int NBARS = 2 + 2 * KST + 2 * VST + 2 * 4;
    static constexpr int FLAGS_OFF = BAR_OFF + NBARS * 8;  // TMEM address, abort flag, last-split flags [2]
    static constexpr int SMEM = FLAGS_OFF + 16 + 1024;     // + slack to align the base to 1024
    static constexpr int THREADS = 384;
    static constexpr int SOFTMAX_WARP0 = 4;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t O_COL = 2 * BN;  // O_t at O_COL + t * DH; S_t at t * BN
    static_assert(O_COL + 2 * DH <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(Q_OFF % 1024 == 0 && K_OFF % 1024 == 0 && V_OFF % 1024 == 0, "128-byte swizzle atoms");
    static_assert(STAGE_OFF % 16 == 0 && BAR_OFF % 8 == 0, "vector and mbarrier accesses");
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
    uint64_t* o_free = o_final + 2;    // [2] the tile's epilogue has read O (128 threads)
    uint32_t* tmem_slot = (uint32_t*)(smem + C::FLAGS_OFF);
    volatile int* abort_flag = (volatile int*)(smem + C::FLAGS_OFF + 4);
    volatile int* last_flag = (volatile int*)(smem + C::FLAGS_OFF + 8);  // [2] per tile

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
            last_flag[t] = 0;
        }
        *abort_flag = 0;
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
    } else if (warp >= C::SOFTMAX_WARP0) {
        // ------------------------------------------- softmax + epilogue warps
        const int t = (warp - C::SOFTMAX_WARP0) >> 2;  // tile A (0) or B (1)
        const int quad = warp & 3;                     // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        const int gid = row;                           // 0 .. 127 within the tile's warps
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t s_col = t * BN, o_col = C::O_COL + t * DH;
        uint4* stage = (uint4*)(smem + C::STAGE_OFF + (warp - C::SOFTMAX_WARP0) * 4096);  // [32 rows][8 chunks]
        const float sl2 = a.scale_log2;
        uint32_t g = 0;
        int kn = 0;
        bool ok = true;
        for (int k = 0; ok && decode_work<BM, BN>(a, k, w); ++k) {
            if (w.nblk <= 0) continue;
            const int use = kn;
            // This row's visible keys, relative to the unit's first key block
            // (clamped: only comparisons against 0 .. nblk * BN matter), and
            // the blocks [i_full0, i_full1] every row of the tile sees whole.
            int lo_rel, hi_rel, i_full0, i_full1;
            {
                const int64_t qpos = a.first_query + w.t0 + row;
                const int64_t p_first = a.base + w.j_begin * BN;
                const int64_t span = (int64_t)w.nblk * BN + 1;
                lo_rel = (int)max((int64_t)-1, min(span, vis_lo(a, qpos) - p_first));
                hi_rel = (int)max((int64_t)-1, min(span, vis_hi(a, qpos) - p_first));
                i_full0 = (int)min((int64_t)w.nblk, max((int64_t)0, (w.full_lo - p_first + BN - 1) / BN));
                i_full1 = (int)max((int64_t)-1, min((int64_t)w.nblk, (w.full_hi - p_first + 1) / BN) - 1);
            }
            float m_run = -INFINITY, l_run = 0.f;
            for (int i = 0; i < w.nblk; ++i, ++g) {
                // Waits are voted warp-wide so the .sync.aligned TMEM accesses
                // below always see a converged warp.
                if (!__all_sync(0xffffffffu, wait(&s_full[t], g & 1))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                // The row's 128 raw scores, one TMEM load.  The maximum is
                // taken before scaling (scale_log2 > 0); the scale is folded
                // into each exponent's FFMA.
                float x[BN];
                {
                    uint32_t r[BN];
                    tc::ld_32x32b_x128(t_lane + s_col, r);
#pragma unroll
                    for (int e = 0; e < BN; ++e) x[e] = __uint_as_float(r[e]);
                }
                // Keys [k_lo, k_hi) of the block are visible to this row; the
                // mask applies only on blocks some row of the tile cannot fully
                // see (a warp-uniform branch).
                if (i < i_full0 || i > i_full1) {
                    const int k_lo = max(0, min(BN, lo_rel - i * BN));
                    const int k_hi = max(0, min(BN, hi_rel - i * BN + 1));
#pragma unroll
                    for (int e = 0; e < BN; ++e)
                        if (e < k_lo || e >= k_hi) x[e] = -INFINITY;
                }
                float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int e = 0; e < BN; ++e) mx[e & 3] = fmaxf(mx[e & 3], x[e]);
                const float mb = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
                const float m_new = fmaxf(m_run, mb);
                const bool rescale = m_new > m_run + 8.0f;  // also true for the first finite block
                float alpha = 1.f;
                if (rescale) {
                    alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_new);
                    m_run = m_new;
                }
                const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
                // P as fp16 pairs: keys 2j, 2j + 1 -> column j of S_t (every
                // score is in registers), 32 keys per store; four sum chains.
                float sm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float pa = ex2(fmaf(x[c * 32 + e], sl2, -m_use));
                        const float pb = ex2(fmaf(x[c * 32 + e + 1], sl2, -m_use));
                        sm[(e >> 1) & 3] += pa + pb;
                        pk[e / 2] = pack2(pa, pb, false);
                    }
                    tc::st_32x32b_x16(t_lane + s_col + c * 16, pk);
                }
                l_run = l_run * alpha + ((sm[0] + sm[1]) + (sm[2] + sm[3]));
                // O_t holds the blocks before this one (S_t(g) completing means
                // P_t(g-1).V has landed); within a unit it is rescaled only when
                // the running max grew by more than 2^8, after the scores are
                // consumed and before P_t(g).V may start.
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
                tc::wait_st();
                tc::fence_before_sync();
                dev::mbar_arrive(&p_full[t]);
            }
            if (!ok) break;
            // ---- the unit's epilogue for this tile, once its last P.V is in O_t.
            // Waits are bounded, so the four warps reach the vote together and
            // skip the tile together (the split path meets on named barriers).
            const int bar_id = 1 + t;
            if (!bar_and(bar_id, 128, __all_sync(0xffffffffu, wait(&o_final[t], use & 1)))) break;
            tc::fence_after_sync();
            const int head = 2 * w.h + t;
            if (w.nsplit == 1) {
                store_rows<DH>(a, w, head, t_lane, o_col, l_run, quad, lane, stage, &o_free[t]);
            } else {
                store_partial<DH>(a, w, head, row, t_lane, o_col, m_run, l_run, &o_free[t]);
                __threadfence();
                asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
                if (gid == 0) {
                    int* ticket = a.tickets + (int64_t)head * a.ntiles + w.tile;
                    const int prev = atomicAdd(ticket, 1);
                    const bool last = prev == w.nsplit - 1;
                    if (last) *ticket = 0;  // ready for the next launch
                    last_flag[t] = last;
                }
                asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
                const bool last = last_flag[t];
                asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");  // every thread has read the flag
                if (last) {
                    __threadfence();
                    if (gid <= (int)(w.t_last - w.t0)) merge_row<DH>(a, w, head, gid);
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
