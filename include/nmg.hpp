// nmg.hpp -- C++ face of the nmg C ABI with the nm engine's own names.
//
// Header-only.  A maintainer of the nm engine swaps
//   FullAttentionCache<Hkv, HeadDim>       (nm/src/attention.hpp:201-250)
//   LocalAttentionCache<Hkv, HeadDim>      (nm/src/attention.hpp:252-395)
//   the per-layer softmax reduction         (nm/src/qwen35.hpp:360-382, nm/src/gemma4.hpp:211-235, ...)
//   DeltaNetState<Heads, Dk, Dv>, gated_delta_step (nm/src/recurrent.hpp:117-177)
//   scaled_dot_product_attention<Heads, Dqk, Dv>  (nm/src/attention.hpp:123-139)
//   Qwen35State<C>, Gemma4_12BCache / Gemma4E4BCache (nm/src/qwen35.hpp:206-241,
//                                                     nm/src/gemma4.hpp:343-378, :734-762)
// for the types below, which keep the method names and throw the same
// exception types; storage and arithmetic live on the GPU behind include/nmg.h.
// The per-layer state owners need C++20 (the reference engine's language level).
// Rows are device pointers in the reference's token-major layout
// [rows][heads * head_dim]; every call takes the CUDA stream it runs on.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>
#include <variant>
#include <vector>

#include "nmg.h"

namespace nmg {

enum class Dtype : int { f32 = NMG_F32, f16 = NMG_F16, bf16 = NMG_BF16, q8_0 = NMG_Q8_0 };  // q8_0: cache storage only

// Status -> the exception type the reference throws in the same situation.
inline void check(int status) {
    if (status == NMG_OK) return;
    const std::string msg = nmg_last_error();
    switch (status) {
        case NMG_INVALID_ARGUMENT: throw std::invalid_argument(msg);
        case NMG_OUT_OF_RANGE: throw std::out_of_range(msg);
        case NMG_LENGTH_ERROR: throw std::length_error(msg);
        case NMG_LOGIC_ERROR: throw std::logic_error(msg);
        case NMG_VALUE_OVERFLOW: throw std::overflow_error(msg);
        default: throw std::runtime_error(msg);  // no visible key, CUDA, NCCL, device timeout
    }
}

struct VisibleRows {  // attention.hpp:144-150
    size_t first;
    size_t end;
    bool empty() const { return first == end; }
    size_t count() const { return end - first; }
};

namespace detail {

class Cache {
public:
    Cache(const Cache&) = delete;
    Cache& operator=(const Cache&) = delete;
    Cache(Cache&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    ~Cache() { nmg_kv_destroy(h_); }

    size_t size() const {
        int64_t v = 0;
        check(nmg_kv_size(h_, &v));
        return size_t(v);
    }
    size_t position(size_t chronological_row) const {
        int64_t p = 0;
        check(nmg_kv_position(h_, int64_t(chronological_row), &p));
        return size_t(p);
    }
    bool can_append_without_eviction(size_t rows) const {
        int yes = 0;
        check(nmg_kv_can_append_without_eviction(h_, int64_t(rows), &yes));
        return yes != 0;
    }
    // append() for one row or a batch of consecutive rows.
    void append(size_t position, const void* keys, const void* values, size_t rows, Dtype src, void* stream) {
        check(nmg_kv_append(h_, int64_t(position), keys, values, int64_t(rows), int(src), stream));
    }
    VisibleRows visible_rows(size_t query) const {
        int64_t f = 0, e = 0;
        check(nmg_kv_visible_rows(h_, int64_t(query), &f, &e));
        return VisibleRows{size_t(f), size_t(e)};
    }
    // key()/value() as a synchronous copy-back (debug only).
    void read_row(size_t chronological_row, size_t kv_head, float* key, float* value, void* stream) const {
        check(nmg_kv_read_row(h_, int64_t(chronological_row), int(kv_head), key, value, stream));
    }
    void reset() { check(nmg_kv_reset(h_)); }
    nmg_kv_cache* handle() const { return h_; }

protected:
    Cache(int hkv, int head_dim, Dtype dtype, size_t window, size_t capacity, int device) {
        check(nmg_kv_create(hkv, head_dim, int(dtype), int64_t(window), int64_t(capacity), device, &h_));
    }
    nmg_kv_cache* h_ = nullptr;
};

}  // namespace detail

template <size_t Hkv, size_t HeadDim>
class FullAttentionCache : public detail::Cache {
public:
    static constexpr size_t kv_heads = Hkv, head_dim = HeadDim;
    explicit FullAttentionCache(size_t capacity, Dtype dtype = Dtype::f32, int device = 0)
        : Cache(int(Hkv), int(HeadDim), dtype, 0, capacity, device) {}
};

template <size_t Hkv, size_t HeadDim>
class LocalAttentionCache : public detail::Cache {
public:
    static constexpr size_t kv_heads = Hkv, head_dim = HeadDim;
    // `capacity` physical rows >= window; one batch of up to
    // capacity - window + 1 rows is attended as a whole.
    LocalAttentionCache(size_t window, size_t capacity, Dtype dtype = Dtype::f32, int device = 0)
        : Cache(int(Hkv), int(HeadDim), dtype, window, capacity, device) {}
    size_t window() const {
        int64_t w = 0;
        check(nmg_kv_window(h_, &w));
        return size_t(w);
    }
    void begin_batch_retention(size_t appended_rows) { check(nmg_kv_begin_batch_retention(h_, int64_t(appended_rows))); }
    void end_batch_retention() { check(nmg_kv_end_batch_retention(h_)); }
};

// The layer reduction over `rows` queries at positions at.. (qwen35.hpp:360-382
// with a score scale; pass no scale for the Gemma form, gemma4.hpp:211-235).
template <size_t Hq, class Cache>
void attend(const Cache& cache, const void* queries, Dtype q_dtype, size_t rows, size_t at, void* out, Dtype out_dtype,
            void* stream) {
    static_assert(Hq % Cache::kv_heads == 0, "query heads must be a whole number of GQA groups");
    check(nmg_attend(cache.handle(), int(Hq), queries, int(q_dtype), int64_t(rows), int64_t(at), 1.f, 0, out,
                     int(out_dtype), stream));
}
template <size_t Hq, class Cache>
void attend(const Cache& cache, const void* queries, Dtype q_dtype, size_t rows, size_t at, float score_scale,
            void* out, Dtype out_dtype, void* stream) {
    static_assert(Hq % Cache::kv_heads == 0, "query heads must be a whole number of GQA groups");
    check(nmg_attend(cache.handle(), int(Hq), queries, int(q_dtype), int64_t(rows), int64_t(at), score_scale, 1, out,
                     int(out_dtype), stream));
}

// A layer's append-then-reduce, including the local ring's token-by-token
// windows when the batch would evict (gemma4.hpp:237-253, :617-630).
template <size_t Hq, class Cache>
void append_attend(Cache& cache, size_t position, const void* keys, const void* values, Dtype kv_dtype,
                   const void* queries, Dtype q_dtype, size_t rows, const float* score_scale, void* out,
                   Dtype out_dtype, void* stream) {
    check(nmg_append_attend(cache.handle(), int64_t(position), keys, values, int(kv_dtype), int(Hq), queries,
                            int(q_dtype), int64_t(rows), score_scale ? *score_scale : 1.f, score_scale ? 1 : 0, out,
                            int(out_dtype), stream));
}

template <size_t Heads, size_t Dk, size_t Dv>
class DeltaNetState {  // recurrent.hpp:117-138, fp32 [head][Dk][Dv] on the device
public:
    static constexpr size_t floats_per_head = Dk * Dv;
    static constexpr size_t floats = Heads * floats_per_head;
    explicit DeltaNetState(int device = 0) { check(nmg_delta_create(int(Heads), int(Dk), int(Dv), device, &h_)); }
    DeltaNetState(const DeltaNetState&) = delete;
    DeltaNetState& operator=(const DeltaNetState&) = delete;
    ~DeltaNetState() { nmg_delta_destroy(h_); }
    void clear(void* stream) { check(nmg_delta_clear(h_, stream)); }
    float* head(size_t h) {  // device pointer; out_of_range like recurrent.hpp:128
        float* p = nullptr;
        check(nmg_delta_head(h_, int(h), &p));
        return p;
    }
    // One token through every value head; value head h reads key head h % Hk.
    void step(size_t hk, const float* q, const float* k, const float* v, const float* gate, const float* beta,
              float* out, void* stream) {
        check(nmg_delta_step(h_, int(hk), q, k, v, gate, beta, out, stream));
    }
    void prefill(size_t hk, size_t tokens, const float* q, const float* k, const float* v, const float* gate,
                 const float* beta, float* out, int chunk, void* stream) {
        check(nmg_delta_prefill(h_, int(hk), int64_t(tokens), q, k, v, gate, beta, out, chunk, stream));
    }
    nmg_delta_state* handle() const { return h_; }

private:
    nmg_delta_state* h_ = nullptr;
};

// One decode token for each of `batch` sequences, each with its own state
// (the head loop of qwen35.hpp:449-454 run for a batch of sequences at once).
template <size_t Heads, size_t Dk, size_t Dv>
void delta_step_batch(DeltaNetState<Heads, Dk, Dv>* const* states, size_t batch, size_t hk, const float* q,
                      const float* k, const float* v, const float* gate, const float* beta, float* out, void* stream) {
    std::vector<nmg_delta_state*> hs(batch);
    for (size_t b = 0; b < batch; ++b) hs[b] = states[b]->handle();
    check(nmg_delta_step_batch(hs.data(), int(batch), int(hk), q, k, v, gate, beta, out, stream));
}

// CausalConv1dState<Channels, Width> (recurrent.hpp:63-110): the carried last
// Width - 1 inputs of the depthwise causal conv, on the device.
template <size_t Channels, size_t Width>
class CausalConv1dState {
public:
    explicit CausalConv1dState(int device = 0) { check(nmg_conv_create(int(Channels), int(Width), device, &h_)); }
    CausalConv1dState(const CausalConv1dState&) = delete;
    CausalConv1dState& operator=(const CausalConv1dState&) = delete;
    ~CausalConv1dState() { nmg_conv_destroy(h_); }
    void clear(void* stream) { check(nmg_conv_clear(h_, stream)); }
    // step() over `tokens` rows: x, y [tokens][Channels]; weights [Channels][Width].
    void step(const float* weights, const float* x, size_t tokens, float* y, bool silu, void* stream) {
        check(nmg_conv_step(h_, weights, x, int64_t(tokens), y, silu ? 1 : 0, stream));
    }
    nmg_conv_state* handle() const { return h_; }

private:
    nmg_conv_state* h_ = nullptr;
};

// The delta-net prologue of qwen35.hpp:396-446 (conv + SiLU over the packed
// [q | k | v] projection, per-head L2 norms, gates) into the layouts
// DeltaNetState::prefill takes, and the gated RMS norm of qwen35.hpp:458-460.
template <size_t Hk, size_t Hv, size_t Dk, size_t Dv, size_t Width>
void delta_prologue(CausalConv1dState<2 * Hk * Dk + Hv * Dv, Width>& conv, const float* conv_weights, size_t tokens,
                    const float* qkv, const float* beta_raw, const float* alpha_raw, const float* dt_bias,
                    const float* decay_scale, float* q, float* k, float* v, float* beta, float* gate, void* stream) {
    check(nmg_delta_prologue(conv.handle(), conv_weights, int(Hk), int(Hv), int(Dk), int(Dv), int64_t(tokens), qkv,
                             beta_raw, alpha_raw, dt_bias, decay_scale, q, k, v, beta, gate, stream));
}
template <size_t Hv, size_t Dv>
void delta_epilogue(size_t tokens, const float* o, const float* z, const float* gamma, float eps, float* out,
                    void* stream) {
    check(nmg_delta_epilogue(int(Hv), int(Dv), int64_t(tokens), o, z, gamma, eps, out, stream));
}
// One decode token of the layer core (qwen35.hpp:396-461 at T = 1): the
// prologue, the recurrent step and the gated output norm in one launch.
template <size_t Hk, size_t Hv, size_t Dk, size_t Dv, size_t Width>
void delta_decode_token(DeltaNetState<Hv, Dk, Dv>& state, CausalConv1dState<2 * Hk * Dk + Hv * Dv, Width>& conv,
                        const float* conv_weights, const float* qkv, const float* beta_raw, const float* alpha_raw,
                        const float* dt_bias, const float* decay_scale, const float* z, const float* gamma, float eps,
                        float* out, void* stream) {
    check(nmg_delta_decode_token(state.handle(), conv.handle(), conv_weights, int(Hk), qkv, beta_raw, alpha_raw,
                                 dt_bias, decay_scale, z, gamma, eps, out, stream));
}

// Before an attention reduction: Q = rope(rmsnorm_per_head(q)) into q_out,
// K = rope(rmsnorm_per_head(k)) and V (scale-free per-head RMS norm when
// v_norm, Gemma 4) appended at position.. , with RotaryEmbedding<HeadDim, Base,
// RotaryNum, RotaryDen> (attention.hpp:68-101).  gated: q is the Qwen 3.5
// query projection in head-major [q | gate] pairs (qwen35.hpp:343-352);
// otherwise plain [tokens][Hq * HeadDim] (gemma4.hpp:206-209, :676-680).
template <size_t Hq, size_t Base, size_t RotaryNum = 1, size_t RotaryDen = 1, class Cache>
void attention_prologue(Cache& cache, size_t position, size_t tokens, const float* q, bool gated, const float* k,
                        const float* v, const float* q_gamma, const float* k_gamma, bool v_norm, float eps, void* q_out,
                        Dtype q_dtype, void* stream) {
    static_assert(Hq % Cache::kv_heads == 0, "query heads must be a whole number of GQA groups");
    static_assert(RotaryDen != 0 && RotaryNum <= RotaryDen, "the rotary fraction is at most one");
    check(nmg_attn_prologue(cache.handle(), int(Hq), int64_t(position), int64_t(tokens), q, gated ? 1 : 0, k, v,
                            q_gamma, k_gamma, v_norm ? 1 : 0, eps, double(Base), int(RotaryNum), int(RotaryDen), q_out,
                            int(q_dtype), stream));
}
// The same preparation without a cache: K (and V when v_norm) to fp32 rows
// [tokens][Hkv * HeadDim], for append_attend (a Gemma sliding-window layer
// whose batch would evict, gemma4.hpp:617-630).
template <size_t Hq, size_t Hkv, size_t HeadDim, size_t Base, size_t RotaryNum = 1, size_t RotaryDen = 1>
void attention_prepare(size_t position, size_t tokens, const float* q, bool gated, const float* k, const float* v,
                       const float* q_gamma, const float* k_gamma, bool v_norm, float eps, void* q_out, Dtype q_dtype,
                       float* k_out, float* v_out, void* stream) {
    static_assert(Hq % Hkv == 0, "query heads must be a whole number of GQA groups");
    static_assert(RotaryDen != 0 && RotaryNum <= RotaryDen, "the rotary fraction is at most one");
    check(nmg_attn_prepare(int(Hq), int(Hkv), int(HeadDim), int64_t(position), int64_t(tokens), q, gated ? 1 : 0, k, v,
                           q_gamma, k_gamma, v_norm ? 1 : 0, eps, double(Base), int(RotaryNum), int(RotaryDen), q_out,
                           int(q_dtype), k_out, v_out, stream));
}
// After it: attended *= sigmoid(gate), the gates the second halves of the
// [q | gate] pairs (qwen35.hpp:390-393).
template <size_t Hq, size_t HeadDim>
void attention_gate(size_t tokens, const float* query_gate, void* attended, Dtype dtype, void* stream) {
    check(nmg_attn_gate(int64_t(tokens), int(Hq), int(HeadDim), query_gate, attended, int(dtype), stream));
}

// One decode query per cache -- the reference keeps one cache per sequence,
// so a batch is a list of caches of one shape.  queries [batch][Hq * HeadDim];
// queries_at[b] is query b's position (nullptr: each cache's newest row);
// score_scale nullptr is the Gemma form.
template <size_t Hq, class Cache>
void attend_batch(const Cache* const* caches, size_t batch, const size_t* queries_at, const void* queries,
                  Dtype q_dtype, const float* score_scale, void* out, Dtype out_dtype, void* stream) {
    static_assert(Hq % Cache::kv_heads == 0, "query heads must be a whole number of GQA groups");
    std::vector<const nmg_kv_cache*> handles(batch);
    std::vector<int64_t> at(queries_at ? batch : 0);
    for (size_t b = 0; b < batch; ++b) {
        handles[b] = caches[b]->handle();
        if (queries_at) at[b] = int64_t(queries_at[b]);
    }
    check(nmg_attend_batch(handles.data(), int(batch), queries_at ? at.data() : nullptr, int(Hq), queries,
                           int(q_dtype), score_scale ? *score_scale : 1.f, score_scale ? 1 : 0, out, int(out_dtype),
                           stream));
}

// softmax_rows(scale * Q K^T) V per head with no mask (the vision tower's
// attention): queries [tq][Heads * Dqk], keys / values [tk][Heads * Dqk], all
// in `dtype`; out [tq][Heads * Dv].  The K/V row mismatch the reference
// checks cannot arise here (one tk for both); tk == 0 is invalid_argument.
template <size_t Heads, size_t QueryKeyDim, size_t ValueDim>
void scaled_dot_product_attention(const void* queries, const void* keys, const void* values, Dtype dtype, size_t tq,
                                  size_t tk, float scale, void* out, Dtype out_dtype, void* stream) {
    static_assert(QueryKeyDim == ValueDim, "the device kernel takes equal query/key and value widths");
    check(nmg_sdpa(int(Heads), int(QueryKeyDim), queries, keys, values, int(dtype), int64_t(tq), int64_t(tk), scale,
                   out, int(out_dtype), stream));
}

// Waits for `stream` and throws std::runtime_error if a kernel since the last
// call gave up a bounded device-side wait.
inline void device_status(int device, void* stream) { check(nmg_device_status(device, stream)); }

// GGUF tensor types (quant.hpp:18-27).
enum class GT : uint32_t {
    F32 = NMG_GT_F32,
    F16 = NMG_GT_F16,
    Q4_0 = NMG_GT_Q4_0,
    Q8_0 = NMG_GT_Q8_0,
    Q4_K = NMG_GT_Q4_K,
    Q5_K = NMG_GT_Q5_K,
    Q6_K = NMG_GT_Q6_K,
    BF16 = NMG_GT_BF16,
};

inline size_t type_size_bytes(GT t, size_t nelem) {  // quant.hpp:89-108
    int64_t b = 0;
    check(nmg_weight_row_bytes(int(t), int64_t(nelem), &b));
    return size_t(b);
}

// Weight<In,Out> (quant.hpp:439-487) with its GGUF bytes resident on the
// device.  matvec / matmul take device fp32 activations and write device fp32
// outputs; fp32_act selects the NM_FP32_ACT path (the default follows that
// environment variable, as the reference reads it, quant_i8.hpp:343-349).
template <size_t In, size_t Out>
class Weight {
public:
    Weight(GT type, const void* host_data, int device = 0) : type_(type) {
        check(nmg_weight_create(int(type), int64_t(In), int64_t(Out), host_data, 0, device, &h_));
        const char* e = std::getenv("NM_FP32_ACT");
        fp32_act_ = e && e[0] && e[0] != '0';
    }
    Weight(const Weight&) = delete;
    Weight& operator=(const Weight&) = delete;
    ~Weight() { nmg_weight_destroy(h_); }
    GT type() const { return type_; }
    size_t row_bytes() const { return type_size_bytes(type_, In); }
    void set_fp32_act(bool on) { fp32_act_ = on; }
    // y[Out] = W x
    void matvec(const float* x, float* y, void* stream) const {
        check(nmg_weight_matvec(h_, x, y, fp32_act_ ? NMG_ACT_FP32 : NMG_ACT_DEFAULT, stream));
    }
    // y[rows][Out] for x[rows][In]
    void matmul(const float* x, size_t rows, float* y, void* stream) const {
        check(nmg_weight_matmul(h_, int64_t(rows), x, y, fp32_act_ ? NMG_ACT_FP32 : NMG_ACT_DEFAULT, stream));
    }
    // rows dequantised to fp32 [rows.size()][In] on the device
    void gather_rows(const std::vector<int32_t>& rows, float* out, void* stream) const {
        check(nmg_weight_gather_rows(h_, rows.data(), int64_t(rows.size()), out, stream));
    }
    nmg_weight* handle() const { return h_; }

private:
    GT type_;
    bool fp32_act_ = false;
    nmg_weight* h_ = nullptr;
};

// gated_delta_step<Dk, Dv> (recurrent.hpp:146-177) on one device head block;
// gate and beta are device scalars.
template <size_t Dk, size_t Dv>
void gated_delta_step(float* state, const float* q, const float* k, const float* v, const float* gate,
                      const float* beta, float* out, void* stream) {
    check(nmg_gated_delta_step(state, int(Dk), int(Dv), q, k, v, gate, beta, out, stream));
}

#if __cplusplus >= 202002L
// ---- per-layer state owners ---------------------------------------------------
//
// The reference's prefix states hold every layer's carried state in one
// object whose token count the model advances.  Here each entry is device
// memory allocated once, at construction: attention caches get `capacity`
// rows (the reference's full caches grow without bound up to C::CTX; a device
// cache is sized up front), local caches `local_capacity` physical rows
// (>= the window; one batch of up to local_capacity - window + 1 rows is
// attended as a whole).  clear() forgets everything derived, in place, where
// the reference's PrefixCache::clear (transformer.hpp:154-160) assigns a
// fresh state; the device memory is kept.

// Qwen35State<C> (qwen35.hpp:206-241) for a Qwen 3.5 config type C (the
// reference's Qwen35_4BConfig, ...): attention layers own a
// FullAttentionCache<Hkv, HEAD_DIM>, recurrent layers (C::is_recurrent) a
// causal-conv history over the packed [q | k | v] channels and a DeltaNetState.
template <class C>
class Qwen35State {
public:
    static constexpr size_t conv_channels = 2 * C::KEY_HEADS * C::KEY_HEAD_DIM + C::VALUE_HEADS * C::VALUE_HEAD_DIM;
    using AttentionEntry = FullAttentionCache<C::Hkv, C::HEAD_DIM>;
    struct RecurrentEntry {
        CausalConv1dState<conv_channels, C::CONV_WIDTH> conv;
        DeltaNetState<C::VALUE_HEADS, C::KEY_HEAD_DIM, C::VALUE_HEAD_DIM> delta;
        explicit RecurrentEntry(int device) : conv(device), delta(device) {}
    };

    explicit Qwen35State(size_t capacity = C::CTX, Dtype kv_dtype = Dtype::bf16, int device = 0) {
        for (size_t layer = 0; layer < C::L; ++layer) {
            if (C::is_recurrent(layer))
                entries_[layer].template emplace<RecurrentEntry>(device);
            else
                entries_[layer].template emplace<AttentionEntry>(capacity, kv_dtype, device);
        }
    }
    Qwen35State(const Qwen35State&) = delete;
    Qwen35State& operator=(const Qwen35State&) = delete;

    size_t tokens() const { return tokens_; }
    void advance(size_t count) {
        if (count > C::CTX - tokens_) throw std::length_error("Qwen35State: context exhausted");
        tokens_ += count;
    }
    // std::bad_variant_access for a layer of the other kind, as in the reference.
    AttentionEntry& attention(size_t layer) { return std::get<AttentionEntry>(entries_.at(layer)); }
    RecurrentEntry& recurrent(size_t layer) { return std::get<RecurrentEntry>(entries_.at(layer)); }

    void clear(void* stream) {
        for (auto& e : entries_) {
            if (auto* a = std::get_if<AttentionEntry>(&e)) a->reset();
            if (auto* r = std::get_if<RecurrentEntry>(&e)) {
                r->conv.clear(stream);
                r->delta.clear(stream);
            }
        }
        tokens_ = 0;
    }

    static constexpr size_t recurrent_floats_per_layer() {
        return DeltaNetState<C::VALUE_HEADS, C::KEY_HEAD_DIM, C::VALUE_HEAD_DIM>::floats;
    }
    static constexpr size_t attention_floats_per_token_per_layer() { return 2 * C::Hkv * C::HEAD_DIM; }

private:
    std::array<std::variant<std::monostate, AttentionEntry, RecurrentEntry>, C::L> entries_;
    size_t tokens_ = 0;
};

namespace detail {
template <class C>
constexpr size_t local_kv_heads() {
    if constexpr (requires { C::LOCAL_HKV; }) return C::LOCAL_HKV;
    else return C::Hkv;
}
template <class C>
constexpr size_t full_kv_heads() {
    if constexpr (requires { C::FULL_HKV; }) return C::FULL_HKV;
    else return C::Hkv;
}
template <class C>
constexpr bool is_full(size_t layer) {
    return C::attention_type(layer) == decltype(C::attention_type(layer))::Full;
}
// The layer whose cache a shared-KV layer reads: the last layer of the same
// attention type that owns its cache (Gemma 4 E4B: 22 for local layers, 23 for
// full ones, gemma4.hpp:371-374).
template <class C>
constexpr size_t kv_source(size_t layer) {
    if (!C::uses_shared_kv(layer)) return layer;
    for (size_t s = layer; s-- > 0;)
        if (!C::uses_shared_kv(s) && is_full<C>(s) == is_full<C>(layer)) return s;
    return layer;
}
}  // namespace detail

// Gemma4_12BCache (gemma4.hpp:734-762) and Gemma4E4BCache (gemma4.hpp:343-378)
// for a Gemma 4 text config type C: local layers own a sliding-window ring of
// C::LOCAL_WINDOW, full layers an append-only cache; layers that read another
// layer's K/V (C::uses_shared_kv) own nothing and resolve to their source.
// K/V heads per kind come from C::LOCAL_HKV / C::FULL_HKV (12B) or C::Hkv (E4B).
template <class C>
class Gemma4Cache {
public:
    using Local = LocalAttentionCache<detail::local_kv_heads<C>(), C::LOCAL_HEAD_DIM>;
    using Full = FullAttentionCache<detail::full_kv_heads<C>(), C::FULL_HEAD_DIM>;

    explicit Gemma4Cache(size_t capacity = C::CTX, size_t local_capacity = 2 * C::LOCAL_WINDOW,
                         Dtype kv_dtype = Dtype::bf16, int device = 0) {
        for (size_t layer = 0; layer < C::L; ++layer) {
            if (C::uses_shared_kv(layer)) continue;
            if (detail::is_full<C>(layer))
                entries_[layer].template emplace<Full>(capacity, kv_dtype, device);
            else
                entries_[layer].template emplace<Local>(C::LOCAL_WINDOW, local_capacity, kv_dtype, device);
        }
    }
    Gemma4Cache(const Gemma4Cache&) = delete;
    Gemma4Cache& operator=(const Gemma4Cache&) = delete;

    size_t tokens() const { return tokens_; }
    void advance(size_t count) {
        if (count > C::CTX - tokens_) throw std::length_error("Gemma4Cache: context exhausted");
        tokens_ += count;
    }
    Local& local(size_t layer) { return std::get<Local>(entries_.at(detail::kv_source<C>(layer))); }
    const Local& local(size_t layer) const { return std::get<Local>(entries_.at(detail::kv_source<C>(layer))); }
    Full& full(size_t layer) { return std::get<Full>(entries_.at(detail::kv_source<C>(layer))); }
    const Full& full(size_t layer) const { return std::get<Full>(entries_.at(detail::kv_source<C>(layer))); }

    void clear() {
        for (auto& e : entries_) {
            if (auto* l = std::get_if<Local>(&e)) l->reset();
            if (auto* f = std::get_if<Full>(&e)) f->reset();
        }
        tokens_ = 0;
    }

private:
    std::array<std::variant<std::monostate, Local, Full>, C::L> entries_;
    size_t tokens_ = 0;
};
#endif  // C++20

}  // namespace nmg
