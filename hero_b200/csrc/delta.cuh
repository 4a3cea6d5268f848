// delta.cuh -- the device-resident gated delta-rule state shared by the
// sequential (delta.cu) and chunked (delta_chunked.cu) kernels.
#pragma once
#include "common.cuh"

struct nmg_delta_state {
    int heads = 0, dk = 0, dv = 0, device = 0;
    float* data = nullptr;  // [heads][dk][dv], fp32, DeltaNetState's layout (recurrent.hpp:117-138)
};

namespace nmg {

// Chunked WY-form prefill (chunk 64, tcgen05 tf32).  NMG_UNSUPPORTED for
// shapes it is not built for (Dk != 128 or Dv not a multiple of 32).
bool delta_chunked_supported(const nmg_delta_state* st);
int delta_prefill_chunked(nmg_delta_state* st, int hk, int64_t T, const float* q, const float* k, const float* v,
                          const float* gate, const float* beta, float* out, int chunk, cudaStream_t stream);

}  // namespace nmg
