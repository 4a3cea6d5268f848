// attn.cuh -- helpers shared by the attention kernels.
#pragma once
#include "common.cuh"
#include "kv_cache.cuh"

namespace nmg {

// Two single-arrival mbarriers (stage 0 and 1), made visible to the async proxy.
__device__ __forceinline__ void mbar_init_pair(uint64_t* bars) {
    dev::mbar_init(&bars[0], 1);
    dev::mbar_init(&bars[1], 1);
    dev::fence_mbar_init();
}

// 16 bytes of cache elements -> fp32.
template <int DT>
__device__ __forceinline__ void unpack16(const uint4& raw, float* out);

template <>
__device__ __forceinline__ void unpack16<NMG_F32>(const uint4& raw, float* out) {
    out[0] = __uint_as_float(raw.x);
    out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z);
    out[3] = __uint_as_float(raw.w);
}

template <>
__device__ __forceinline__ void unpack16<NMG_BF16>(const uint4& raw, float* out) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

template <>
__device__ __forceinline__ void unpack16<NMG_F16>(const uint4& raw, float* out) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        const float2 f = __half22float2(h);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// The PER consecutive elements lane*PER .. of one cached row, as fp32
// (elements past DH read as zero).
template <int DT, int DH, int PER>
__device__ __forceinline__ void load_row_chunk(const typename dev::Elem<DT>::T* row, int lane, float* out) {
    constexpr int ES = DT == NMG_F32 ? 4 : 2;
    if constexpr (PER * ES == 16) {
        unpack16<DT>(*(const uint4*)(row + lane * PER), out);
    } else if constexpr (DT == NMG_F32 && PER == 8) {
        unpack16<DT>(*(const uint4*)(row + lane * PER), out);
        unpack16<DT>(*(const uint4*)(row + lane * PER + 4), out + 4);
    } else if constexpr (DT != NMG_F32 && PER == 4) {
        const uint2 raw = *(const uint2*)(row + lane * PER);
        float tmp[8];
        unpack16<DT>(make_uint4(raw.x, raw.y, 0u, 0u), tmp);
#pragma unroll
        for (int e = 0; e < 4; ++e) out[e] = tmp[e];
    } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            const int d = lane * PER + e;
            out[e] = d < DH ? dev::Elem<DT>::load(row + d) : 0.f;
        }
    }
}

// Split-KV launcher over one cache: rows first_query.. with visible positions
// [max(q - window + 1, floor), min(q, newest)].  caller_scratch/bytes: when
// non-null the kernel uses that memory instead of the library's scratch.
int attend_rows_split(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                      int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                      cudaStream_t stream, void* caller_scratch, int64_t caller_bytes);

int attend_batch_split(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq, const void* q,
                       int q_dtype, float scale, void* out, int out_dtype, cudaStream_t stream);

// 2-D TMA maps over a cache's K and V buffers, (d, hkv*slots), boxes of
// 64 elements x box_rows rows with the 128-byte swizzle (attn_prefill_sm100.cu).
int make_kv_tensor_maps(const nmg_kv_cache* c, int box_rows, CUtensorMap* k, CUtensorMap* v);

// Tensor-core (mma.sync) split-KV decode for 16-bit caches (attn_decode_mma.cu).
bool decode_mma_supported(const nmg_kv_cache* c, int q_dtype);
int attend_rows_mma(const nmg_kv_cache* c, int hq, const void* q, int64_t rows, int64_t first_query, int64_t window,
                    int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype, cudaStream_t stream);
int attend_batch_mma(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq, const void* q,
                     float scale, void* out, int out_dtype, cudaStream_t stream);

// tcgen05 flash prefill (attn_prefill_sm100.cu).  Returns NMG_UNSUPPORTED
// when the shape is not one it was built for.
bool prefill_supported(const nmg_kv_cache* c, int hq, int q_dtype, int64_t rows);
int attend_rows_prefill(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                        int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                        cudaStream_t stream);

}  // namespace nmg
