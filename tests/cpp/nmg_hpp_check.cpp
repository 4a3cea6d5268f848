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

int main() {
    int failures = 0;
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
