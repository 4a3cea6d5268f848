// delta_chunked.cu -- chunked WY-form gated delta-rule prefill (K5).
#include "common.cuh"

struct nmg_delta_state;

namespace nmg {

int delta_prefill_chunked(nmg_delta_state*, int, int64_t, const float*, const float*, const float*, const float*,
                          const float*, float*, int, cudaStream_t) {
    return set_error(NMG_UNSUPPORTED, "chunked delta-rule prefill is not built yet");
}

}  // namespace nmg
