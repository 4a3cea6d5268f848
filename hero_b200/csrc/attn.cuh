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
    } else if constexpr (DT != NMG_F32 && PER == 16) {
        unpack16<DT>(*(const uint4*)(row + lane * PER), out);
        unpack16<DT>(*(const uint4*)(row + lane * PER + 8), out + 8);
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

// ---- merging split-KV partials -------------------------------------------
// Block-wide max / sum over NT threads; `red` holds NT / 32 floats.
template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
    v = dev::warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < NT / 32; ++i) r = fmaxf(r, red[i]);
    return r;
}
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = dev::warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < NT / 32; ++i) r += red[i];
    return r;
}

constexpr int kMergeChunk = 256;  // split weights staged per pass

// The last CTA of a query row combines the row's split partials.  Split sp's
// record for group g sits at part + sp * sp_stride + g * (DH + 2): DH
// weighted sums, then the split's running max m and sum l (natural-log units,
// or base-2 units when LOG2).  Weights go through shared memory in chunks so
// the loads of each pass are independent of one another (a serial walk over
// the splits pays the L2 latency once per split).  `red` holds NT / 32
// floats, `wbuf` kMergeChunk floats; store(g, d, value) writes the result.
template <int NT, int DH, bool LOG2, class Store>
__device__ void merge_partials(const float* part, int64_t sp_stride, int64_t nsplit, int ng, float* red, float* wbuf,
                               Store&& store) {
    constexpr int PER = (DH + NT - 1) / NT;
    const int tid = threadIdx.x;
    for (int g = 0; g < ng; ++g) {
        const float* pg = part + g * (DH + 2);
        float mx = -INFINITY;
        for (int64_t sp = tid; sp < nsplit; sp += NT) mx = fmaxf(mx, __ldcg(pg + sp * sp_stride + DH));
        const float M = block_max<NT>(mx, red);
        float acc[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) acc[k] = 0.f;
        float lsum = 0.f;
        for (int64_t base = 0; base < nsplit; base += kMergeChunk) {
            const int cnt = (int)(nsplit - base < kMergeChunk ? nsplit - base : kMergeChunk);
            __syncthreads();
            for (int i = tid; i < cnt; i += NT) {
                const float* pp = pg + (base + i) * sp_stride;
                const float m = __ldcg(pp + DH);
                float w = 0.f;
                if (m != -INFINITY) w = LOG2 ? exp2f(m - M) : __expf(m - M);
                wbuf[i] = w;
                lsum = fmaf(w, __ldcg(pp + DH + 1), lsum);
            }
            __syncthreads();
#pragma unroll 4
            for (int i = 0; i < cnt; ++i) {
                const float w = wbuf[i];
                const float* pp = pg + (base + i) * sp_stride;
#pragma unroll
                for (int k = 0; k < PER; ++k) {
                    const int d = tid + k * NT;
                    if (d < DH) acc[k] = fmaf(w, __ldcg(pp + d), acc[k]);
                }
            }
        }
        const float L = block_sum<NT>(lsum, red);
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int d = tid + k * NT;
            if (d < DH) store(g, d, acc[k] / L);
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

// Decode over fp32 caches at head_dim 128 / 256 (attn_decode_cluster.cu):
// 8-warp CTAs whose key splits merge across a thread-block cluster (short
// decodes) or through global partials and a ticket (long ones).  The two
// functions above hand these caches over when fp32_decode_fits says so.
bool fp32_decode_fits(const nmg_kv_cache* c);
int attend_rows_cluster(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                        int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                        cudaStream_t stream);
int attend_batch_cluster(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq,
                         const void* q, int q_dtype, float scale, void* out, int out_dtype, cudaStream_t stream);

// 2-D TMA maps over a cache's K and V buffers, (d, hkv*slots), boxes of
// 64 elements x box_rows rows with the 128-byte swizzle (attn_prefill_sm100.cu).
int make_kv_tensor_maps(const nmg_kv_cache* c, int box_rows, CUtensorMap* k, CUtensorMap* v);

// Tensor-core (mma.sync) split-KV decode for 16-bit caches with a query of the
// cache's dtype, and for Q8_0 caches with any query dtype (attn_decode_mma.cu).
bool decode_mma_supported(const nmg_kv_cache* c, int q_dtype);
int attend_rows_mma(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                    int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                    cudaStream_t stream);
int attend_batch_mma(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq, const void* q,
                     int q_dtype, float scale, void* out, int out_dtype, cudaStream_t stream);

// tcgen05 flash prefill (attn_prefill_sm100.cu).  Returns NMG_UNSUPPORTED
// when the shape is not one it was built for.
bool prefill_supported(const nmg_kv_cache* c, int hq, int q_dtype, int64_t rows);
// Row t's hq*dh outputs go to outs[i] + t * out_row_elems + out_col0 for
// every i < nout (at most 8; the caller's buffer and, for head-sharded
// multi-GPU runs, peer buffers).
int attend_rows_prefill(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                        int64_t window, int64_t floor_pos, int64_t newest, float scale, void* const* outs, int nout,
                        int64_t out_row_elems, int64_t out_col0, int out_dtype, cudaStream_t stream);

}  // namespace nmg
