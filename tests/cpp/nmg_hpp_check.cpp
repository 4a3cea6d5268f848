// Compiles the C++ face of the C ABI and checks its error mapping on argument
// validation, which runs before any device work (so this needs no GPU).
#include <cstdio>
#include <stdexcept>

#include "nmg.hpp"

// The delta-net prologue/epilogue templates instantiate at a Qwen 3.5 shape
// (only compiled here: running them needs a GPU).
[[maybe_unused]] static auto* const prologue_fn = &nmg::delta_prologue<16, 32, 128, 128, 4>;
[[maybe_unused]] static auto* const epilogue_fn = &nmg::delta_epilogue<32, 128>;
[[maybe_unused]] static auto* const attn_prologue_fn =
    &nmg::attention_prologue<16, 10000000, 1, 4, nmg::FullAttentionCache<4, 256>>;
[[maybe_unused]] static auto* const attn_gate_fn = &nmg::attention_gate<16, 256>;
[[maybe_unused]] static auto* const attn_prepare_fn = &nmg::attention_prepare<8, 4, 256, 10000>;
[[maybe_unused]] static void (nmg::CausalConv1dState<8192, 4>::*const conv_step_fn)(const float*, const float*, size_t,
                                                                                    float*, bool, void*) =
    &nmg::CausalConv1dState<8192, 4>::step;

[[maybe_unused]] static void (*const sdpa_fn)(const void*, const void*, const void*, nmg::Dtype, size_t, size_t, float,
                                                void*, nmg::Dtype, void*) =
    &nmg::scaled_dot_product_attention<12, 64, 64>;
[[maybe_unused]] static auto* const attend_batch_fn = &nmg::attend_batch<64, nmg::FullAttentionCache<8, 128>>;

// Config types shaped like the reference's (only the members the state owners read).
enum class AttentionType { Local, Full };
struct QwenLike {  // Qwen35_4BConfig's layer schedule and recurrent shapes, 8 layers
    static constexpr size_t L = 8, CTX = 262144, Hkv = 4, HEAD_DIM = 256;
    static constexpr size_t KEY_HEADS = 16, VALUE_HEADS = 32, KEY_HEAD_DIM = 128, VALUE_HEAD_DIM = 128, CONV_WIDTH = 4;
    static constexpr bool is_recurrent(size_t layer) { return (layer + 1) % 4 != 0; }
};
struct NoLayers : QwenLike {  // no device state at all: the token bookkeeping alone
    static constexpr size_t L = 0, CTX = 10;
};
struct E4BLike {  // Gemma4E4BTextConfig's schedule: 42 layers, the last 18 read shared K/V
    static constexpr size_t L = 42, CTX = 131072, Hkv = 2, LOCAL_HEAD_DIM = 256, FULL_HEAD_DIM = 512;
    static constexpr size_t LOCAL_WINDOW = 512;
    static constexpr AttentionType attention_type(size_t layer) {
        return layer % 6 == 5 ? AttentionType::Full : AttentionType::Local;
    }
    static constexpr bool uses_shared_kv(size_t layer) { return layer >= 24; }
};
struct Gemma12BLike {  // Gemma4_12BTextConfig: per-kind K/V head counts, no shared layers
    static constexpr size_t L = 48, CTX = 262144, LOCAL_HKV = 8, FULL_HKV = 1, LOCAL_HEAD_DIM = 256, FULL_HEAD_DIM = 512;
    static constexpr size_t LOCAL_WINDOW = 1024;
    static constexpr AttentionType attention_type(size_t layer) {
        return layer % 6 == 5 ? AttentionType::Full : AttentionType::Local;
    }
    static constexpr bool uses_shared_kv(size_t) { return false; }
};
// The shared-KV sources the reference hard-codes (gemma4.hpp:371-374).
static_assert(nmg::detail::kv_source<E4BLike>(24) == 22 && nmg::detail::kv_source<E4BLike>(29) == 23 &&
              nmg::detail::kv_source<E4BLike>(41) == 23 && nmg::detail::kv_source<E4BLike>(10) == 10);
static_assert(nmg::detail::kv_source<Gemma12BLike>(47) == 47);
static_assert(nmg::Gemma4Cache<Gemma12BLike>::Full::kv_heads == 1 && nmg::Gemma4Cache<Gemma12BLike>::Local::kv_heads == 8);
static_assert(nmg::Gemma4Cache<E4BLike>::Full::head_dim == 512 && nmg::Gemma4Cache<E4BLike>::Local::kv_heads == 2);
static_assert(nmg::Qwen35State<QwenLike>::conv_channels == 8192);
static_assert(nmg::Qwen35State<QwenLike>::recurrent_floats_per_layer() == 32 * 128 * 128);
static_assert(nmg::Qwen35State<QwenLike>::attention_floats_per_token_per_layer() == 2 * 4 * 256);

int main() {
    int failures = 0;
    {
        nmg::Qwen35State<NoLayers> s;
        s.advance(4);
        s.advance(6);
        try {
            s.advance(1);
            std::puts("FAIL: advance past the context");
            ++failures;
        } catch (const std::length_error&) {
            std::puts(s.tokens() == 10 ? "PASS: advance past CTX is std::length_error" : "FAIL: token count");
            failures += s.tokens() != 10;
        }
    }
    // Device state: without a GPU the first allocation fails as std::runtime_error;
    // with one, the layer kinds resolve as in the reference.
    try {
        nmg::Qwen35State<QwenLike> s(64);
        s.attention(3);
        s.recurrent(0);
        try {
            s.attention(0);
            ++failures;
        } catch (const std::bad_variant_access&) {
        }
        nmg::Gemma4Cache<E4BLike> g(64, 1024);
        failures += &g.local(30) != &g.local(22) || &g.full(41) != &g.full(23);
        std::puts("PASS: state owners build on the device");
    } catch (const std::runtime_error&) {
        std::puts("PASS: state owners report a missing device as std::runtime_error");
    }
    try {
        nmg::LocalAttentionCache<1, 2> bad(/*window*/ 4, /*capacity*/ 2);  // capacity < window
        std::puts("FAIL: no exception");
        ++failures;
    } catch (const std::invalid_argument&) {
        std::puts("PASS: capacity below the window is std::invalid_argument");
    }
    try {
        nmg::check(NMG_OUT_OF_RANGE);
        ++failures;
    } catch (const std::out_of_range&) {
        std::puts("PASS: NMG_OUT_OF_RANGE is std::out_of_range");
    }
    try {
        nmg::check(NMG_RUNTIME_ERROR);
        ++failures;
    } catch (const std::runtime_error&) {
        std::puts("PASS: NMG_RUNTIME_ERROR is std::runtime_error");
    }
    return failures;
}
