// weight.cuh -- device layout of the quantised projections shared by the
// weight-streaming products (weight.cu) and the tensor-core products
// (weight_mma.cu).
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace nmg {
namespace wq {

enum : int { GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q5_K = 13, GT_Q6_K = 14, GT_Q8_K = 15, GT_BF16 = 30 };

__host__ __device__ inline int block_len(int t) {
    switch (t) {
        case GT_F32:
        case GT_F16:
        case GT_BF16: return 1;
        case GT_Q4_0:
        case GT_Q8_0: return 32;
        case GT_Q4_K:
        case GT_Q5_K:
        case GT_Q6_K:
        case GT_Q8_K: return 256;
    }
    return 0;
}

__host__ __device__ inline int block_bytes(int t) {
    switch (t) {
        case GT_F32: return 4;
        case GT_F16:
        case GT_BF16: return 2;
        case GT_Q4_0: return 18;
        case GT_Q8_0: return 34;
        case GT_Q4_K: return 144;
        case GT_Q5_K: return 176;
        case GT_Q6_K: return 210;
        case GT_Q8_K: return 292;
    }
    return 0;
}

inline bool has_i8(int t) { return t == GT_Q8_0 || t == GT_Q4_0 || t == GT_Q4_K || t == GT_Q6_K; }

// Device planes of one weight (row strides in bytes / elements).
struct Planes {
    const uint8_t* qs;    // quants / nibbles / low nibbles; F32: the fp32 rows
    const uint8_t* hi;    // Q5_K high bits, Q6_K high pairs
    const uint32_t* meta; // per superblock 4 words: Q4_K/Q5_K word g = the 6-bit scales and
                          // mins of sub-blocks 2g, 2g+1 (sc lo, sc hi, m lo, m hi bytes);
                          // Q6_K word 2h+k = the int8 scales 8h+k, 8h+2+k, 8h+4+k, 8h+6+k
    const uint16_t* d;    // Q8_0/Q4_0 block scales, Q6_K superblock d (fp16 bits)
    const uint32_t* dd;   // Q4_K/Q5_K superblock d | dmin << 16 (fp16 bits)
    int64_t qs_row, hi_row, meta_row, d_row, dd_row;  // bytes / words / elements per row
};

}  // namespace wq
}  // namespace nmg

struct nmg_weight {
    int type = 0, device = 0;
    int64_t in = 0, out = 0;
    void* base = nullptr;
    nmg::wq::Planes p{};
};


namespace nmg {
namespace wq {

// Device form of a quantised activation row: int8 quants [rows][in], the fp32
// value of each block's scale [rows][in/block] (the fp16-rounded d for Q8_0,
// as its dot reads it back; the fp32 d for Q8_K), and for Q8_K the int16 sums
// of each 16 quants [rows][in/16].
struct ActPlanes {
    int8_t* qs;
    float* d;
    int16_t* bsums;
};

// Tensor-core product for long activation batches (weight_mma.cu): y[rows][out]
// from activations already quantised into `act` (Q8_0 planes for Q8_0/Q4_0
// weights, Q8_K planes for Q4_K/Q6_K).  Returns false when the type has no
// tensor-core kernel.
bool mm_supported(int type);
// Splits of the reduction for a batch of `rows` (more than one when the output
// tiles alone would leave SMs idle); each needs rows * out floats of `part`.
int mm_splits(const nmg_weight* w, int64_t rows);
cudaError_t launch_mm(const nmg_weight* w, int64_t rows, const ActPlanes& act, float* part, float* y, cudaStream_t st);

}  // namespace wq
}  // namespace nmg
