// ref_shim.cpp -- a C entry layer over the reference engine's OWN headers.
//
// TEST INFRASTRUCTURE ONLY.  This file is compiled against the reference
// sources where they lie (include path to the reference's nm/src, plus its
// core.cpp for the par_for pool) by oracle/Makefile into oracle/_ref/.  It
// is used to pin oracle/nm_oracle.c, to write tests/golden fixtures, and as
// the timed CPU baseline (bench.py --impl reference).  It copies no reference
// code: it instantiates the reference's FullAttentionCache, LocalAttentionCache,
// CausalWindow, Softmax, dot, DeltaNetState, gated_delta_step, l2_normalize and
// softplus directly.
//
// The softmax reduction itself exists in the reference only as a lambda inside
// each model layer (src/qwen35.hpp:360-382, src/gemma4.hpp:211-235 ...), which
// cannot be instantiated without a model config.  The reference's own tests
// therefore mirror it (tests/property_tests.cpp:33-56 with a score scale,
// tests/gemma4_tests.cpp:34-57 without).  `reduce` below is that same equation
// over the reference types: visible_rows per query, then per (row, head) task
// on par_for: scores = [scale *] dot(q, key(j, head / group)), Softmax, and
// scaled_add of value(j, head / group).
#include "attention.hpp"
#include "components.hpp"
#include "recurrent.hpp"
#include "quant_i8.hpp"

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <stdexcept>
#include <vector>

namespace {

enum Status { OK = 0, INVALID_ARGUMENT = 1, OUT_OF_RANGE = 2, RUNTIME_ERROR = 3, LENGTH_ERROR = 4, LOGIC_ERROR = 5 };

template <size_t N>
Vec<N> vec_from(const float* p) {
    Vec<N> v;
    for (size_t i = 0; i < N; ++i) v[i] = p[i];
    return v;
}

// The mirrored reduction over a reference cache.  q is [qrows][hq*Dh].
template <size_t Hkv, size_t Dh, class Cache>
void reduce(const Cache& cache, const float* q, size_t qrows, size_t hq, Position at, float scale, bool use_scale,
            float* out) {
    std::vector<VisibleRows> visible;
    visible.reserve(qrows);
    for (size_t row = 0; row < qrows; ++row) visible.push_back(cache.visible_rows(at + row));

    par_for(qrows * hq, [&](size_t task) {
        const size_t row = task / hq, head = task % hq;
        const Vec<Dh> query = vec_from<Dh>(q + (row * hq + head) * Dh);
        const KVHead group{head / (hq / Hkv)};
        const VisibleRows rows = visible[row];

        std::vector<Scalar> alpha;
        alpha.reserve(rows.count());
        for (size_t j = rows.first; j < rows.end; ++j) {
            const Scalar d = dot(VecView<Dh>(query), cache.key(j, group));
            alpha.push_back(use_scale ? scale * d : d);
        }
        alpha = Softmax{}(std::move(alpha));

        Vec<Dh> head_output;
        for (size_t n = 0; n < alpha.size(); ++n) head_output.scaled_add(cache.value(rows.first + n, group), alpha[n]);
        for (size_t i = 0; i < Dh; ++i) out[(row * hq + head) * Dh + i] = head_output[i];
    });
}

// The reduction with a causal window applied to a full cache's rows:
// CausalWindow{window}.visible_rows over the cache's positions.
template <size_t Hkv, size_t Dh, class Cache>
void reduce_window(const Cache& cache, size_t window, const float* q, size_t qrows, size_t hq, Position at, float scale,
                   bool use_scale, float* out) {
    std::vector<VisibleRows> visible;
    visible.reserve(qrows);
    for (size_t row = 0; row < qrows; ++row)
        visible.push_back(CausalWindow{window}.visible_rows(at + row, cache.position(0), cache.size()));
    par_for(qrows * hq, [&](size_t task) {
        const size_t row = task / hq, head = task % hq;
        const Vec<Dh> query = vec_from<Dh>(q + (row * hq + head) * Dh);
        const KVHead group{head / (hq / Hkv)};
        const VisibleRows rows = visible[row];
        std::vector<Scalar> alpha;
        alpha.reserve(rows.count());
        for (size_t j = rows.first; j < rows.end; ++j) {
            const Scalar d = dot(VecView<Dh>(query), cache.key(j, group));
            alpha.push_back(use_scale ? scale * d : d);
        }
        alpha = Softmax{}(std::move(alpha));
        Vec<Dh> head_output;
        for (size_t n = 0; n < alpha.size(); ++n) head_output.scaled_add(cache.value(rows.first + n, group), alpha[n]);
        for (size_t i = 0; i < Dh; ++i) out[(row * hq + head) * Dh + i] = head_output[i];
    });
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return OK;
    } catch (const std::invalid_argument&) {
        return INVALID_ARGUMENT;
    } catch (const std::out_of_range&) {
        return OUT_OF_RANGE;
    } catch (const std::length_error&) {
        return LENGTH_ERROR;
    } catch (const std::logic_error&) {
        return LOGIC_ERROR;
    } catch (const std::runtime_error&) {
        return RUNTIME_ERROR;
    }
}

// Append `rows` K/V rows at positions first.. and reduce `qrows` queries at
// positions first_query.. over a FullAttentionCache (qwen35.hpp:386-387).
template <size_t Hkv, size_t Dh>
int attend_full(const float* k, const float* v, size_t rows, size_t first, const float* q, size_t qrows, size_t hq,
                size_t first_query, float scale, bool use_scale, float* out) {
    constexpr size_t W = Hkv * Dh;
    return guarded([&] {
        if (hq % Hkv != 0) throw std::invalid_argument("hq is not a multiple of Hkv");
        FullAttentionCache<Hkv, Dh> cache;
        for (size_t r = 0; r < rows; ++r) cache.append(Position{first + r}, vec_from<W>(k + r * W), vec_from<W>(v + r * W));
        reduce<Hkv, Dh>(cache, q, qrows, hq, Position{first_query}, scale, use_scale, out);
    });
}

// The Gemma local-layer path (gemma4.hpp:617-630): the whole batch when the
// ring has room, otherwise append one row and reduce one query at a time.
// Rows [0, rows - qrows) are history appended before the queried batch.
template <size_t Hkv, size_t Dh>
int attend_local(size_t window, const float* k, const float* v, size_t rows, size_t first, const float* q,
                 size_t qrows, size_t hq, float scale, bool use_scale, float* out) {
    constexpr size_t W = Hkv * Dh;
    return guarded([&] {
        if (qrows > rows) throw std::invalid_argument("more queries than rows");
        if (hq % Hkv != 0) throw std::invalid_argument("hq is not a multiple of Hkv");
        LocalAttentionCache<Hkv, Dh> cache(window);
        const size_t history = rows - qrows;
        for (size_t r = 0; r < history; ++r) cache.append(Position{first + r}, vec_from<W>(k + r * W), vec_from<W>(v + r * W));
        const Position at{first + history};
        if (cache.can_append_without_eviction(qrows)) {
            for (size_t r = history; r < rows; ++r) cache.append(Position{first + r}, vec_from<W>(k + r * W), vec_from<W>(v + r * W));
            reduce<Hkv, Dh>(cache, q, qrows, hq, at, scale, use_scale, out);
        } else {
            for (size_t t = 0; t < qrows; ++t) {
                const size_t r = history + t;
                cache.append(Position{first + r}, vec_from<W>(k + r * W), vec_from<W>(v + r * W));
                reduce<Hkv, Dh>(cache, q + t * hq * Dh, 1, hq, at + t, scale, use_scale, out + t * hq * Dh);
            }
        }
    });
}

// A scripted LocalAttentionCache<1,1>: ops are (code, arg) pairs; code 0 =
// append one row at position arg, 1 = begin_batch_retention(arg), 2 =
// end_batch_retention().  Afterwards size, window and every chronological
// row's position are reported (gemma4_tests.cpp:153-172 is one such script).
int local_script(size_t window, const int64_t* ops, size_t nops, int64_t* size_out, int64_t* positions_out,
                 size_t max_positions, int64_t* first_failed_op) {
    *first_failed_op = -1;
    std::unique_ptr<LocalAttentionCache<1, 1>> cache;
    int status = guarded([&] { cache = std::make_unique<LocalAttentionCache<1, 1>>(window); });
    if (status != OK) return status;
    for (size_t i = 0; i < nops; ++i) {
        const int64_t code = ops[2 * i], arg = ops[2 * i + 1];
        status = guarded([&] {
            if (code == 0) {
                Vec<1> row;
                row[0] = float(arg);
                cache->append(Position{size_t(arg)}, row, row);
            } else if (code == 1) {
                cache->begin_batch_retention(size_t(arg));
            } else if (code == 2) {
                cache->end_batch_retention();
            } else {
                throw std::invalid_argument("unknown op");
            }
        });
        if (status != OK) {
            *first_failed_op = int64_t(i);
            return status;
        }
    }
    *size_out = int64_t(cache->size());
    for (size_t r = 0; r < cache->size() && r < max_positions; ++r) {
        // position() is a Position; its only numeric face is Position - Position.
        positions_out[r] = int64_t(cache->position(r) - Position{0});
    }
    return OK;
}

template <size_t Hv, size_t Dk, size_t Dv>
int delta_run(float* state_io, size_t T, size_t hk, const float* q, const float* k, const float* v, const float* g,
              const float* beta, float* out) {
    return guarded([&] {
        DeltaNetState<Hv, Dk, Dv> state;
        for (size_t h = 0; h < Hv; ++h)
            for (size_t i = 0; i < Dk * Dv; ++i) state.head(h)[i] = state_io[h * Dk * Dv + i];
        for (size_t t = 0; t < T; ++t) {
            for (size_t h = 0; h < Hv; ++h) {
                const size_t kh = h % hk;  // qwen35.hpp:172 (tiled key heads)
                const Vec<Dk> qv = vec_from<Dk>(q + (t * hk + kh) * Dk);
                const Vec<Dk> kv = vec_from<Dk>(k + (t * hk + kh) * Dk);
                const Vec<Dv> vv = vec_from<Dv>(v + (t * Hv + h) * Dv);
                const Vec<Dv> o = gated_delta_step<Dk, Dv>(state.head(h), VecView<Dk>(qv), VecView<Dk>(kv), VecView<Dv>(vv),
                                                           g[t * Hv + h], beta[t * Hv + h]);
                for (size_t j = 0; j < Dv; ++j) out[(t * Hv + h) * Dv + j] = o[j];
            }
        }
        for (size_t h = 0; h < Hv; ++h)
            for (size_t i = 0; i < Dk * Dv; ++i) state_io[h * Dk * Dv + i] = state.head(h)[i];
    });
}

// Timed sample of a prefill: the cache is filled untimed, then the reduction
// runs for each block [start, start+len) of query rows; only the reductions
// are timed (seconds_out).  q is the full [rows][hq*Dh] query matrix.
template <size_t Hkv, size_t Dh>
int prefill_sample(const float* k, const float* v, size_t rows, const float* q, size_t hq, const int64_t* blocks,
                   size_t nblocks, float scale, bool use_scale, size_t window, float* out, double* seconds_out) {
    constexpr size_t W = Hkv * Dh;
    return guarded([&] {
        FullAttentionCache<Hkv, Dh> cache;
        for (size_t r = 0; r < rows; ++r) cache.append(Position{r}, vec_from<W>(k + r * W), vec_from<W>(v + r * W));
        double total = 0;
        for (size_t b = 0; b < nblocks; ++b) {
            const size_t start = size_t(blocks[2 * b]), len = size_t(blocks[2 * b + 1]);
            const auto t0 = std::chrono::steady_clock::now();
            if (window == 0) {
                reduce<Hkv, Dh>(cache, q + start * hq * Dh, len, hq, Position{start}, scale, use_scale, out + start * hq * Dh);
            } else {
                // A window only narrows each row's visible interval; the same
                // reduction over a LocalAttentionCache view is what the Gemma
                // local layers run (gemma4.hpp:593-615).
                reduce_window<Hkv, Dh>(cache, window, q + start * hq * Dh, len, hq, Position{start}, scale, use_scale,
                                       out + start * hq * Dh);
            }
            total += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        }
        *seconds_out = total;
    });
}

// Timed sample of single-token decode: the cache is filled with `rows` rows
// (untimed), then one query at position rows - 1 is reduced `reps` times
// (timed, seconds_out = the total); window > 0 narrows the visible rows as a
// Gemma local layer's ring does.  q / out are one [hq*Dh] row.
template <size_t Hkv, size_t Dh>
int decode_sample(const float* k, const float* v, size_t rows, const float* q, size_t hq, float scale, bool use_scale,
                  size_t window, size_t reps, float* out, double* seconds_out) {
    constexpr size_t W = Hkv * Dh;
    return guarded([&] {
        FullAttentionCache<Hkv, Dh> cache;
        for (size_t r = 0; r < rows; ++r) cache.append(Position{r}, vec_from<W>(k + r * W), vec_from<W>(v + r * W));
        const Position at{rows - 1};
        const auto t0 = std::chrono::steady_clock::now();
        for (size_t i = 0; i < reps; ++i) {
            if (window == 0)
                reduce<Hkv, Dh>(cache, q, 1, hq, at, scale, use_scale, out);
            else
                reduce_window<Hkv, Dh>(cache, window, q, 1, hq, at, scale, use_scale, out);
        }
        *seconds_out = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    });
}

}  // namespace

#define NMREF_ATTN_SHAPES(X) \
    X(1, 1)                  \
    X(1, 2)                  \
    X(1, 4)                  \
    X(2, 4)                  \
    X(1, 16)                 \
    X(2, 16)                 \
    X(2, 32)                 \
    X(4, 32)                 \
    X(1, 64)                 \
    X(2, 64)                 \
    X(4, 64)                 \
    X(1, 128)                \
    X(2, 128)                \
    X(4, 128)                \
    X(8, 128)                \
    X(1, 256)                \
    X(2, 256)                \
    X(4, 256)                \
    X(1, 512)                \
    X(2, 512)

#define NMREF_DELTA_SHAPES(X) \
    X(1, 2, 2)                \
    X(2, 2, 2)                \
    X(4, 16, 16)              \
    X(4, 32, 32)              \
    X(8, 64, 64)              \
    X(2, 128, 128)            \
    X(4, 128, 128)            \
    X(8, 128, 128)            \
    X(32, 128, 128)

extern "C" {

// Status codes: 0 ok, 1 invalid_argument, 2 out_of_range, 3 runtime_error,
// 4 length_error, 5 logic_error, 100 shape not instantiated here.
int nmref_attend_full(int hkv, int dh, const float* k, const float* v, int64_t rows, int64_t first, const float* q,
                      int64_t qrows, int hq, int64_t first_query, float scale, int use_scale, float* out) {
#define X(H, D) \
    if (hkv == H && dh == D) return attend_full<H, D>(k, v, rows, first, q, qrows, hq, first_query, scale, use_scale != 0, out);
    NMREF_ATTN_SHAPES(X)
#undef X
    return 100;
}

int nmref_attend_local(int hkv, int dh, int64_t window, const float* k, const float* v, int64_t rows, int64_t first,
                       const float* q, int64_t qrows, int hq, float scale, int use_scale, float* out) {
#define X(H, D)                       \
    if (hkv == H && dh == D)          \
        return attend_local<H, D>(window, k, v, rows, first, q, qrows, hq, scale, use_scale != 0, out);
    NMREF_ATTN_SHAPES(X)
#undef X
    return 100;
}

int nmref_prefill_sample(int hkv, int dh, const float* k, const float* v, int64_t rows, const float* q, int hq,
                         const int64_t* blocks, int64_t nblocks, float scale, int use_scale, int64_t window, float* out,
                         double* seconds) {
#define X(H, D)                                                                                                   \
    if (hkv == H && dh == D)                                                                                      \
        return prefill_sample<H, D>(k, v, size_t(rows), q, size_t(hq), blocks, size_t(nblocks), scale, use_scale != 0, \
                                    size_t(window), out, seconds);
    NMREF_ATTN_SHAPES(X)
#undef X
    return 100;
}

int nmref_decode_sample(int hkv, int dh, const float* k, const float* v, int64_t rows, const float* q, int hq,
                        float scale, int use_scale, int64_t window, int64_t reps, float* out, double* seconds) {
    if (rows <= 0 || reps <= 0) return 1;
#define X(H, D)                                                                                                     \
    if (hkv == H && dh == D)                                                                                        \
        return decode_sample<H, D>(k, v, size_t(rows), q, size_t(hq), scale, use_scale != 0, size_t(window), size_t(reps), \
                                   out, seconds);
    NMREF_ATTN_SHAPES(X)
#undef X
    return 100;
}

int nmref_local_script(int64_t window, const int64_t* ops, int64_t nops, int64_t* size_out, int64_t* positions_out,
                       int64_t max_positions, int64_t* first_failed_op) {
    return local_script(size_t(window), ops, size_t(nops), size_out, positions_out, size_t(max_positions), first_failed_op);
}

int nmref_visible_rows(int64_t width, int64_t query, int64_t oldest, int64_t rows, int64_t* first, int64_t* end) {
    const VisibleRows r = CausalWindow{size_t(width)}.visible_rows(Position{size_t(query)}, Position{size_t(oldest)}, size_t(rows));
    *first = int64_t(r.first);
    *end = int64_t(r.end);
    return 0;
}

int nmref_contains(int64_t width, int64_t key, int64_t query) {
    return CausalWindow{size_t(width)}.contains(Position{size_t(key)}, Position{size_t(query)}) ? 1 : 0;
}

int nmref_delta_run(int hv, int dk, int dv, float* state, int64_t T, int hk, const float* q, const float* k, const float* v,
                    const float* g, const float* beta, float* out) {
#define X(H, DK, DV) \
    if (hv == H && dk == DK && dv == DV) return delta_run<H, DK, DV>(state, T, hk, q, k, v, g, beta, out);
    NMREF_DELTA_SHAPES(X)
#undef X
    return 100;
}

int nmref_delta_timed(int hv, int dk, int dv, float* state, int64_t T, int hk, const float* q, const float* k,
                      const float* v, const float* g, const float* beta, float* out, double* seconds) {
    const auto t0 = std::chrono::steady_clock::now();
    const int st = nmref_delta_run(hv, dk, dv, state, T, hk, q, k, v, g, beta, out);
    *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return st;
}

float nmref_softplus(float x) { return softplus(x); }
float nmref_sigmoid(float x) { return sigmoid(x); }

int nmref_l2_normalize(int n, const float* x, float* y) {
    if (n == 2) {
        const Vec<2> r = l2_normalize<2>(VecView<2>(vec_from<2>(x)));
        for (int i = 0; i < 2; ++i) y[i] = r[i];
        return 0;
    }
    if (n == 128) {
        const Vec<128> r = l2_normalize<128>(VecView<128>(vec_from<128>(x)));
        for (int i = 0; i < 128; ++i) y[i] = r[i];
        return 0;
    }
    return 100;
}

// CausalConv1dState<C, W>::step over T tokens from a fresh (zero) state.
int nmref_conv_run(int channels, int width, const float* weights, const float* x, int64_t T, float* y) {
#define X(C, W)                                                                              \
    if (channels == C && width == W) {                                                       \
        Matrix<W> taps;                                                                      \
        taps.reserve(C);                                                                     \
        for (int c = 0; c < C; ++c) taps.append(VecView<W>(vec_from<W>(weights + (size_t)c * W))); \
        auto conv = std::make_unique<CausalConv1dState<C, W>>();                             \
        for (int64_t t = 0; t < T; ++t) {                                                    \
            const Vec<C> out = conv->step(VecView<C>(vec_from<C>(x + (size_t)t * C)), taps);   \
            for (int c = 0; c < C; ++c) y[(size_t)t * C + c] = out[c];                       \
        }                                                                                    \
        return 0;                                                                            \
    }
    X(2, 3) X(24, 4) X(1024, 4) X(8192, 4)
#undef X
    return 100;
}

// Silu (components.hpp:102-105), one element at a time through the reference type.
void nmref_silu(int64_t n, const float* x, float* y) {
    for (int64_t i = 0; i < n; ++i) {
        Vec<1> v;
        v[0] = x[i];
        Silu{}(MutVecView<1>(v));
        y[i] = v[0];
    }
}

// RMSNorm<N> (components.hpp:167-180) of each of `rows` rows.
int nmref_rmsnorm(int n, int64_t rows, const float* gamma, float eps, const float* x, float* y) {
#define X(N)                                                                   \
    if (n == N) {                                                              \
        const RMSNorm<N> norm(vec_from<N>(gamma), eps);                        \
        for (int64_t r = 0; r < rows; ++r) {                                   \
            const Vec<N> out = norm(VecView<N>(vec_from<N>(x + (size_t)r * N))); \
            for (int i = 0; i < N; ++i) y[(size_t)r * N + i] = out[i];         \
        }                                                                      \
        return 0;                                                              \
    }
    X(2) X(64) X(128)
#undef X
    return 100;
}

// RotaryEmbedding<HeadDim, Base, Num, Den> (attention.hpp:68-101) applied to
// each head of each row of x [rows][heads*HeadDim] at position first + row,
// through the reference's own Matrix overload.
int nmref_rope(int head_dim, int64_t base, int num, int den, int heads, int64_t rows, int64_t first, float* x) {
#define X(DH, B, N, D, H)                                                                       \
    if (head_dim == DH && base == B && num == N && den == D && heads == H) {                    \
        Matrix<DH * H> m = Matrix<DH * H>::from_row_major(std::vector<Scalar>(x, x + (size_t)rows * DH * H)); \
        m = RotaryEmbedding<DH, B, N, D>{}(std::move(m), Position{(size_t)first});              \
        for (int64_t r = 0; r < rows; ++r)                                                      \
            for (int i = 0; i < DH * H; ++i) x[(size_t)r * DH * H + i] = m.row((size_t)r)[i];   \
        return 0;                                                                               \
    }
    X(8, 10000, 1, 2, 1) X(8, 10000, 1, 1, 1) X(256, 10000000, 1, 4, 2) X(256, 10000, 1, 1, 2) X(512, 1000000, 1, 4, 1)
    X(64, 10000, 1, 1, 3)
#undef X
    return 100;
}

// PerHeadNorm<RMSNorm<N>> (gamma given) or PerHeadNorm<RMSNormNoScale<N>>
// (gamma null) over `heads` heads of each row (components.hpp:167-215, :248-281).
int nmref_head_norm(int n, int heads, int64_t rows, const float* gamma, float eps, const float* x, float* y) {
#define X(N, H)                                                                                  \
    if (n == N && heads == H) {                                                                  \
        for (int64_t r = 0; r < rows; ++r) {                                                     \
            const Vec<N * H> row = vec_from<N * H>(x + (size_t)r * N * H);                       \
            const Vec<N * H> out = gamma ? PerHeadNorm<RMSNorm<N>>(RMSNorm<N>(vec_from<N>(gamma), eps))(VecView<N * H>(row)) \
                                         : PerHeadNorm<RMSNormNoScale<N>>(RMSNormNoScale<N>(eps))(VecView<N * H>(row));      \
            for (int i = 0; i < N * H; ++i) y[(size_t)r * N * H + i] = out[i];                   \
        }                                                                                        \
        return 0;                                                                                \
    }
    X(256, 2) X(512, 1) X(64, 3) X(4, 1)
#undef X
    return 100;
}

// scaled_dot_product_attention<Heads, D, D> (attention.hpp:124-139): dense,
// unmasked, Q [tq][Heads*D], K/V [tk][Heads*D]; the vision ViT's call
// (gemma4_vision.hpp:167) is <12, 64, 64> with scale 1.
int nmref_sdpa(int heads, int d, int64_t tq, int64_t tk, const float* q, const float* k, const float* v, float scale,
               float* out) {
#define X(H, D)                                                                                               \
    if (heads == H && d == D) {                                                                               \
        const auto Q = Matrix<H * D>::from_row_major(std::vector<Scalar>(q, q + (size_t)tq * H * D));        \
        const auto K = Matrix<H * D>::from_row_major(std::vector<Scalar>(k, k + (size_t)tk * H * D));        \
        const auto V = Matrix<H * D>::from_row_major(std::vector<Scalar>(v, v + (size_t)tk * H * D));        \
        const auto A = scaled_dot_product_attention<H, D, D>(Q.view(), K.view(), V.view(), scale);           \
        for (int64_t r = 0; r < tq; ++r)                                                                      \
            for (int i = 0; i < H * D; ++i) out[(size_t)r * H * D + i] = A.row((size_t)r)[i];               \
        return 0;                                                                                             \
    }
    X(12, 64) X(4, 64)
#undef X
    return 100;
}

// sigmoid (core.hpp:579) of each element.
void nmref_sigmoid_n(int64_t n, const float* x, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = sigmoid(x[i]);
}

uint16_t nmref_fp32_to_bf16(float f) { return fp32_to_bf16(f); }
uint16_t nmref_fp32_to_fp16(float f) { return fp32_to_fp16(f); }
float nmref_bf16_to_fp32(uint16_t b) { return bf16_to_fp32(b); }
float nmref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }

int nmref_threads(void) { return int(nm_num_threads()); }

// quantize_row_q8_0 (quant_i8.hpp:69-81) over n values (a multiple of 32):
// int8 quants and the fp16 bit pattern of each 32-value block's scale.
void nmref_quantize_q8_0(const float* x, int64_t n, int8_t* qs, uint16_t* d) {
    std::vector<block_q8_0> blocks((size_t)n / QK8_0);
    quantize_row_q8_0(x, blocks.data(), (size_t)n);
    for (size_t b = 0; b < blocks.size(); ++b) {
        d[b] = blocks[b].d;
        for (int j = 0; j < QK8_0; ++j) qs[b * QK8_0 + j] = blocks[b].qs[j];
    }
}


// ---- quantised weights (quant.hpp, quant_i8.hpp) -------------------------
// Packed activation blocks as the reference lays them out: quantize_row_q8_0
// (34-byte block_q8_0) and quantize_row_q8_K (292-byte block_q8_K).
void nmref_quantize_row_q8_0_blocks(const float* x, int64_t n, void* out) {
    quantize_row_q8_0(x, static_cast<block_q8_0*>(out), (size_t)n);
}
void nmref_quantize_row_q8_K(const float* x, int64_t n, void* out) {
    quantize_row_q8_K(x, static_cast<block_q8_K*>(out), (size_t)n);
}
// The weight-side quantisers the reference's tests build fixtures with.
void nmref_quantize_q8_0_weights(const float* x, int64_t n, void* out) {
    quantize_q8_0(x, static_cast<block_q8_0*>(out), (size_t)n);
}
void nmref_quantize_q4_0_weights(const float* x, int64_t n, void* out) {
    quantize_q4_0(x, static_cast<block_q4_0*>(out), (size_t)n);
}

// One weight row's integer dot against a quantised activation row, through
// the reference's own vec_dot_* (the scalar ggml-generic clones on hosts
// without ARM dotprod).
float nmref_vec_dot_i8(int type, int64_t n, const void* w, const void* act) {
    switch (GT(type)) {
        case GT::Q8_0:
            return vec_dot_q8_0_q8_0((size_t)n, (const block_q8_0*)w, (const block_q8_0*)act);
        case GT::Q4_0:
            return vec_dot_q4_0_q8_0((size_t)n, (const block_q4_0*)w, (const block_q8_0*)act);
        case GT::Q4_K:
            return vec_dot_q4_K_q8_K((size_t)n, (const block_q4_K*)w, (const block_q8_K*)act);
        case GT::Q6_K:
            return vec_dot_q6_K_q8_K((size_t)n, (const block_q6_K*)w, (const block_q8_K*)act);
        default:
            return NAN;
    }
}

// One weight row against fp32 activations: the dot_block_* sum of
// Weight::matvec's fp32-activation branch (quant_i8.hpp:394-427).
float nmref_dot_fp32(int type, int64_t n, const void* w, const float* x) {
    Scalar acc = 0;
    switch (GT(type)) {
        case GT::Q8_0:
            for (size_t i = 0; i < (size_t)n / QK8_0; ++i) acc += dot_block_q8_0(((const block_q8_0*)w)[i], x + i * QK8_0);
            break;
        case GT::Q4_0:
            for (size_t i = 0; i < (size_t)n / QK4_0; ++i) acc += dot_block_q4_0(((const block_q4_0*)w)[i], x + i * QK4_0);
            break;
        case GT::Q4_K:
            for (size_t i = 0; i < (size_t)n / QK_K; ++i) acc += dot_block_q4_K(((const block_q4_K*)w)[i], x + i * QK_K);
            break;
        case GT::Q5_K:
            for (size_t i = 0; i < (size_t)n / QK_K; ++i) acc += dot_block_q5_K(((const block_q5_K*)w)[i], x + i * QK_K);
            break;
        case GT::Q6_K:
            for (size_t i = 0; i < (size_t)n / QK_K; ++i) acc += dot_block_q6_K(((const block_q6_K*)w)[i], x + i * QK_K);
            break;
        default:
            return NAN;
    }
    return acc;
}

int nmref_dequant(int type, const void* src, float* dst, int64_t n) {
    return guarded([&] { dequant_to_f32(GT(type), src, dst, (size_t)n); });
}

}  // extern "C"

namespace {
template <size_t In, size_t Out>
int weight_product(int type, const void* w, int64_t rows, const float* x, float* y) {
    return guarded([&] {
        const Weight<In, Out> weight(GT(type), w, std::shared_ptr<const void>());
        if (rows == 1) {
            const Vec<In> v = vec_from<In>(x);
            const Vec<Out> r = weight.matvec(VecView<In>(v));
            for (size_t o = 0; o < Out; ++o) y[o] = r[o];
            return;
        }
        const Matrix<In> m = Matrix<In>::from_row_major(std::vector<Scalar>(x, x + (size_t)rows * In));
        const Matrix<Out> r = weight.matmul(m.view());
        for (size_t i = 0; i < (size_t)rows; ++i)
            for (size_t o = 0; o < Out; ++o) y[i * Out + o] = r.row(i)[o];
    });
}
}  // namespace

extern "C" {

// Weight<In,Out>::matvec (rows == 1) or ::matmul itself, for the shapes the
// tests use; 100 for a shape that is not instantiated here.  Which activation
// path runs is the reference's own choice (NM_FP32_ACT, read once).
int nmref_weight_product(int type, int64_t in, int64_t out, const void* w, int64_t rows, const float* x, float* y) {
#define X(I, O) \
    if (in == I && out == O) return weight_product<I, O>(type, w, rows, x, y);
    X(256, 40) X(512, 24) X(1024, 16) X(2048, 8)
#undef X
    return 100;
}

}  // extern "C"
