// Compiles the C++ face of the C ABI and checks its error mapping on argument
// validation, which runs before any device work (so this needs no GPU).
#include <cstdio>
#include <stdexcept>

#include "nmg.hpp"

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
