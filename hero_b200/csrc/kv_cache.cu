// kv_cache.cu -- device KV cache: creation, append (K1), bookkeeping.
//
// The bookkeeping restates nm/src/attention.hpp:201-395 on the host:
//   append            :215-220 (full), :320-345 (local ring / retention)
//   visible_rows      :222-226, :347-351 (CausalWindow::visible_rows :170-176)
//   position          :208-211, :264-267
//   can_append...     :213, :315-318
//   batch retention   :274-313
// The device holds the rows; the kernel below writes a batch of appended rows
// into their ring slots, converting to the cache dtype with the reference's
// rounding (core.hpp:61-100).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

#include "kv_cache.cuh"

namespace nmg {
namespace {

// One thread per (row, head, 8-element chunk); rows are the last `rows`
// appended positions, row r going to slot (slot0 + r) mod slots.
template <int SRC, int DST>
__global__ void kv_append_kernel(const void* __restrict__ keys, const void* __restrict__ values, void* __restrict__ kc,
                                 void* __restrict__ vc, int64_t rows, int64_t src_row0, int hkv, int dh, int64_t slots,
                                 int64_t slot0, int* __restrict__ err) {
    const int chunks = (dh + 7) / 8;
    bool overflow = false;
    const int64_t total = rows * hkv * chunks;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(t % chunks);
        const int64_t rh = t / chunks;
        const int h = (int)(rh % hkv);
        const int64_t r = rh / hkv;
        const int64_t slot = (slot0 + r) % slots;
        const int64_t src = (src_row0 + r) * (int64_t)hkv * dh + (int64_t)h * dh;
        const int64_t dst = ((int64_t)h * slots + slot) * dh;
        const int d0 = c * 8;
        const int n = dh - d0 < 8 ? dh - d0 : 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            if (e < n) {
                const float kf = dev::load_as_f32(keys, SRC, src + d0 + e);
                const float vf = dev::load_as_f32(values, SRC, src + d0 + e);
                dev::store_from_f32(kc, DST, dst + d0 + e, kf);
                store_cache_v(vc, DST, dst + d0 + e, vf, overflow);
            }
        }
    }
    if (overflow) atomicOr(err, dev::kErrF16Overflow);
}

// Same-dtype fast path: 16-byte vector copies when a head row is a multiple of
// 16 bytes; V_TO_F16 converts bf16 V rows to the fp16 V buffer on the way.
template <bool V_TO_F16>
__global__ void kv_append_copy16_kernel(const uint4* __restrict__ keys, const uint4* __restrict__ values,
                                        uint4* __restrict__ kc, uint4* __restrict__ vc, int64_t rows, int64_t src_row0,
                                        int hkv, int vecs_per_head, int64_t slots, int64_t slot0,
                                        int* __restrict__ err) {
    const int64_t total = rows * hkv * vecs_per_head;
    bool overflow = false;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(t % vecs_per_head);
        const int64_t rh = t / vecs_per_head;
        const int h = (int)(rh % hkv);
        const int64_t r = rh / hkv;
        const int64_t slot = (slot0 + r) % slots;
        const int64_t src = ((src_row0 + r) * hkv + h) * vecs_per_head + c;
        const int64_t dst = ((int64_t)h * slots + slot) * vecs_per_head + c;
        kc[dst] = __ldg(keys + src);
        uint4 v = __ldg(values + src);
        if constexpr (V_TO_F16) {
            uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t lo = cache_v_from_bf16(w[i] & 0xFFFFu, overflow);
                const uint32_t hi = cache_v_from_bf16(w[i] >> 16, overflow);
                w[i] = lo | (hi << 16);
            }
            v = make_uint4(w[0], w[1], w[2], w[3]);
        }
        vc[dst] = v;
    }
    if (V_TO_F16 && overflow) atomicOr(err, dev::kErrF16Overflow);
}

// Q8_0 append: one warp per (row, head); lane l takes values 4l .. 4l + 3 of
// each 128-value group, so a 32-value block is 8 lanes and its maximum three
// xor-shuffles.  quantize_row_q8_0 (nm/src/quant_i8.hpp:69-81) exactly:
// d = amax / 127, id = d ? 1 / d : 0, the scale stored as fp16 with the
// reference's rounding, q = roundf(x * id).
template <int SRC>
__global__ void kv_append_q8_kernel(const void* __restrict__ keys, const void* __restrict__ values,
                                    int8_t* __restrict__ kq, int8_t* __restrict__ vq, uint16_t* __restrict__ ks,
                                    uint16_t* __restrict__ vs, int64_t rows, int64_t src_row0, int hkv, int dh,
                                    int64_t slots, int64_t sstride, int64_t slot0, int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    bool overflow = false;
    for (int64_t wi = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); wi < rows * hkv; wi += nwarps) {
        const int h = (int)(wi % hkv);
        const int64_t r = wi / hkv;
        const int64_t slot = (slot0 + r) % slots;
        const int64_t src = (src_row0 + r) * (int64_t)hkv * dh + (int64_t)h * dh;
        const int64_t dst = (int64_t)h * slots + slot, sdst = (int64_t)h * sstride + slot;
        for (int g0 = 0; g0 < dh; g0 += 128) {
            const int e0 = g0 + 4 * lane;
            const bool in = e0 < dh;
#pragma unroll
            for (int which = 0; which < 2; ++which) {
                const void* in_rows = which ? values : keys;
                float x[4];
                float amax = 0.f;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    x[u] = in ? dev::load_as_f32(in_rows, SRC, src + e0 + u) : 0.f;
                    amax = fmaxf(amax, fabsf(x[u]));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
                if (!in) continue;
                const float d = amax / 127.f;
                const float id = d != 0.f ? 1.f / d : 0.f;
                uint32_t packed = 0;
#pragma unroll
                for (int u = 0; u < 4; ++u) packed |= ((uint32_t)(uint8_t)(int8_t)(int)roundf(x[u] * id)) << (8 * u);
                int8_t* q = which ? vq : kq;
                uint16_t* sc = which ? vs : ks;
                *(uint32_t*)(q + dst * dh + e0) = packed;
                if ((lane & 7) == 0) sc[sdst * (dh / 32) + e0 / 32] = dev::f32_to_f16_bits(d);
                overflow |= amax > 65504.f;  // the attention kernels take scale * quant as fp16
            }
        }
    }
    if (overflow) atomicOr(err, dev::kErrF16Overflow);
}

template <int SRC>
int launch_append(int dst, const void* k, const void* v, void* kc, void* vc, int64_t rows, int64_t row0, int hkv,
                  int dh, int64_t slots, int64_t slot0, cudaStream_t s, int blocks, int* err) {
    if (dst == NMG_F32)
        kv_append_kernel<SRC, NMG_F32><<<blocks, 256, 0, s>>>(k, v, kc, vc, rows, row0, hkv, dh, slots, slot0, err);
    else if (dst == NMG_F16)
        kv_append_kernel<SRC, NMG_F16><<<blocks, 256, 0, s>>>(k, v, kc, vc, rows, row0, hkv, dh, slots, slot0, err);
    else
        kv_append_kernel<SRC, NMG_BF16><<<blocks, 256, 0, s>>>(k, v, kc, vc, rows, row0, hkv, dh, slots, slot0, err);
    return NMG_OK;
}

}  // namespace

int kv_append_device(nmg_kv_cache* c, int64_t first_position, const void* keys, const void* values, int64_t rows,
                     int src_dtype, cudaStream_t stream) {
    if (rows <= 0) return NMG_OK;
    // Only the newest `slots` rows of a batch can survive in the ring; writing
    // just those keeps one launch free of same-slot write races.
    int64_t row0 = 0, slot0 = 0;
    kv_append_slots(c, first_position, rows, &row0, &slot0);
    const int64_t write = rows - row0;
    // Created with the cache (nmg_kv_create), so this never allocates.
    int* err = nullptr;
    const int fst = device_error_flag(c->device, &err);
    if (fst != NMG_OK) return fst;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != c->device) NMG_CUDA_TRY(cudaSetDevice(c->device));
    if (c->dtype == NMG_Q8_0) {
        const int64_t warps = write * c->hkv;
        const int blocks = (int)((warps + 7) / 8 < 148 * 16 ? (warps + 7) / 8 : 148 * 16);
        int8_t *kq = (int8_t*)c->k, *vq = (int8_t*)c->v;
        uint16_t *ks = (uint16_t*)c->ks, *vs = (uint16_t*)c->vs;
        if (src_dtype == NMG_F32)
            kv_append_q8_kernel<NMG_F32><<<blocks, 256, 0, stream>>>(keys, values, kq, vq, ks, vs, write, row0, c->hkv,
                                                                      c->dh, c->slots, c->sstride, slot0, err);
        else if (src_dtype == NMG_F16)
            kv_append_q8_kernel<NMG_F16><<<blocks, 256, 0, stream>>>(keys, values, kq, vq, ks, vs, write, row0, c->hkv,
                                                                      c->dh, c->slots, c->sstride, slot0, err);
        else
            kv_append_q8_kernel<NMG_BF16><<<blocks, 256, 0, stream>>>(keys, values, kq, vq, ks, vs, write, row0,
                                                                       c->hkv, c->dh, c->slots, c->sstride, slot0, err);
        NMG_CUDA_TRY(cudaGetLastError());
        if (prev != c->device) NMG_CUDA_TRY(cudaSetDevice(prev));
        return NMG_OK;
    }
    const int es = dtype_size(c->dtype);
    if (src_dtype == c->dtype && (c->dh * es) % 16 == 0 && ((uintptr_t)keys % 16) == 0 && ((uintptr_t)values % 16) == 0) {
        const int vecs = c->dh * es / 16;
        const int64_t work = write * c->hkv * vecs;
        const int blocks = (int)((work + 255) / 256 < 148 * 16 ? (work + 255) / 256 : 148 * 16);
        if (c->vdtype != c->dtype)
            kv_append_copy16_kernel<true><<<blocks, 256, 0, stream>>>((const uint4*)keys, (const uint4*)values,
                                                                      (uint4*)c->k, (uint4*)c->v, write, row0, c->hkv,
                                                                      vecs, c->slots, slot0, err);
        else
            kv_append_copy16_kernel<false><<<blocks, 256, 0, stream>>>((const uint4*)keys, (const uint4*)values,
                                                                       (uint4*)c->k, (uint4*)c->v, write, row0, c->hkv,
                                                                       vecs, c->slots, slot0, err);
    } else {
        const int64_t work = write * c->hkv * ((c->dh + 7) / 8);
        const int blocks = (int)((work + 255) / 256 < 148 * 16 ? (work + 255) / 256 : 148 * 16);
        if (src_dtype == NMG_F32)
            launch_append<NMG_F32>(c->dtype, keys, values, c->k, c->v, write, row0, c->hkv, c->dh, c->slots, slot0,
                                   stream, blocks, err);
        else if (src_dtype == NMG_F16)
            launch_append<NMG_F16>(c->dtype, keys, values, c->k, c->v, write, row0, c->hkv, c->dh, c->slots, slot0,
                                   stream, blocks, err);
        else
            launch_append<NMG_BF16>(c->dtype, keys, values, c->k, c->v, write, row0, c->hkv, c->dh, c->slots, slot0,
                                    stream, blocks, err);
    }
    NMG_CUDA_TRY(cudaGetLastError());
    if (prev != c->device) NMG_CUDA_TRY(cudaSetDevice(prev));
    return NMG_OK;
}

}  // namespace nmg

using nmg::set_error;

extern "C" int nmg_kv_create(int hkv, int head_dim, int dtype, int64_t window, int64_t capacity, int device,
                             nmg_kv_cache** out) {
    if (!out) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_create: null out");
    *out = nullptr;
    if (hkv <= 0 || head_dim <= 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_create: hkv and head_dim must be positive");
    if (!nmg::cache_dtype_valid(dtype)) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_create: bad dtype %d", dtype);
    if (dtype == NMG_Q8_0 && head_dim % 32 != 0)
        return set_error(NMG_UNSUPPORTED, "nmg_kv_create: a Q8_0 cache needs head_dim a multiple of 32");
    if (window < 0) return set_error(NMG_INVALID_ARGUMENT, "LocalAttentionCache: window must be positive");
    if (capacity <= 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_create: capacity must be positive");
    if (window > 0 && capacity < window)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_create: a local cache needs capacity >= window");
    nmg_kv_cache* c = new nmg_kv_cache();
    c->hkv = hkv;
    c->dh = head_dim;
    c->dtype = dtype;
    c->device = device;
    c->vdtype = nmg::v_dtype_for(dtype);
    c->window = window;
    c->slots = capacity;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    // A Q8_0 cache's kernels stream whole 64-row tiles with bulk copies, so its
    // buffers carry 64 zeroed rows past the last head's slots.
    const size_t rows_alloc = (size_t)hkv * (size_t)capacity + (dtype == NMG_Q8_0 ? 64 : 0);
    const size_t bytes = rows_alloc * (size_t)head_dim * nmg::cache_elem_size(dtype);
    if (e == cudaSuccess) e = cudaMalloc(&c->k, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&c->v, bytes);
    // Zeroed like the reference's ring storage (attention.hpp:363-372).
    if (e == cudaSuccess) e = cudaMemset(c->k, 0, bytes);
    if (e == cudaSuccess) e = cudaMemset(c->v, 0, bytes);
    if (dtype == NMG_Q8_0) {
        c->sstride = (capacity + 63) / 64 * 64;
        const size_t sbytes = ((size_t)hkv * (size_t)c->sstride + 64) * (size_t)(head_dim / 32) * 2;
        if (e == cudaSuccess) e = cudaMalloc(&c->ks, sbytes);
        if (e == cudaSuccess) e = cudaMalloc(&c->vs, sbytes);
        if (e == cudaSuccess) e = cudaMemset(c->ks, 0, sbytes);
        if (e == cudaSuccess) e = cudaMemset(c->vs, 0, sbytes);
    }
    // The device's error flag, which appends raise on fp16 overflow of V:
    // created here so that no later call (possibly under stream capture)
    // has to allocate it.
    int* flag = nullptr;
    if (e == cudaSuccess && nmg::device_error_flag(device, &flag) != NMG_OK) e = cudaErrorMemoryAllocation;
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (c->k) cudaFree(c->k);
        if (c->v) cudaFree(c->v);
        if (c->ks) cudaFree(c->ks);
        if (c->vs) cudaFree(c->vs);
        delete c;
        return set_error(NMG_CUDA_ERROR, "nmg_kv_create: %s", cudaGetErrorString(e));
    }
    *out = c;
    return NMG_OK;
}

extern "C" int nmg_kv_destroy(nmg_kv_cache* c) {
    if (!c) return NMG_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    cudaFree(c->k);
    cudaFree(c->v);
    if (c->ks) cudaFree(c->ks);
    if (c->vs) cudaFree(c->vs);
    cudaSetDevice(prev);
    delete c;
    return NMG_OK;
}

namespace nmg {

int kv_append_begin(nmg_kv_cache* c, int64_t first, int64_t rows, int64_t* accepted, int* deferred) {
    *accepted = 0;
    *deferred = NMG_OK;
    const char* kind = c->window ? "LocalAttentionCache" : "FullAttentionCache";
    if (first < 0) return set_error(NMG_INVALID_ARGUMENT, "%s: negative position", kind);
    if (c->size == 0 && c->total == 0) {
        c->base = first;
        c->oldest = first;
    } else if (first != c->oldest + c->size) {
        return set_error(NMG_INVALID_ARGUMENT, "%s: positions must be consecutive", kind);
    }
    int64_t take = rows;
    if (c->window == 0) {
        if (c->total + rows > c->slots)
            return set_error(NMG_LENGTH_ERROR, "FullAttentionCache: device capacity of %lld rows exhausted",
                             (long long)c->slots);
    } else if (c->retaining) {
        if (rows > c->batch_remaining) {
            take = c->batch_remaining;  // the reference appends these, then throws
            *deferred = set_error(NMG_LENGTH_ERROR, "LocalAttentionCache: retained batch received too many rows");
        }
    }
    *accepted = take;
    return NMG_OK;
}

void kv_append_commit(nmg_kv_cache* c, int64_t first, int64_t accepted) {
    if (accepted <= 0) return;
    if (c->window == 0) {
        c->size += accepted;
    } else if (c->retaining) {
        c->size += accepted;
        c->batch_remaining -= accepted;
    } else {
        const int64_t newest = first + accepted - 1;
        c->size = c->size + accepted < c->window ? c->size + accepted : c->window;
        c->oldest = newest - c->size + 1;
    }
    c->total += accepted;
}

}  // namespace nmg

extern "C" int nmg_kv_append(nmg_kv_cache* c, int64_t first, const void* keys, const void* values, int64_t rows,
                             int src_dtype, void* stream) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_append: null cache");
    if (rows < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_append: negative row count");
    if (rows == 0) return NMG_OK;
    if (!keys || !values) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_append: null rows");
    if (!nmg::dtype_valid(src_dtype)) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_append: bad dtype");
    int64_t accepted = 0;
    int deferred = NMG_OK;
    int st = nmg::kv_append_begin(c, first, rows, &accepted, &deferred);
    if (st != NMG_OK) return st;
    if (accepted > 0) {
        st = nmg::kv_append_device(c, first, keys, values, accepted, src_dtype, (cudaStream_t)stream);
        if (st != NMG_OK) return st;
        nmg::kv_append_commit(c, first, accepted);
    }
    return deferred;
}

extern "C" int nmg_kv_size(const nmg_kv_cache* c, int64_t* size) {
    if (!c || !size) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_size: null argument");
    *size = c->size;
    return NMG_OK;
}

extern "C" int nmg_kv_window(const nmg_kv_cache* c, int64_t* window) {
    if (!c || !window) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_window: null argument");
    *window = c->window;
    return NMG_OK;
}

extern "C" int nmg_kv_position(const nmg_kv_cache* c, int64_t row, int64_t* position) {
    if (!c || !position) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_position: null argument");
    if (row < 0 || row >= c->size)
        return set_error(NMG_OUT_OF_RANGE, "%s: row out of range", c->window ? "LocalAttentionCache" : "FullAttentionCache");
    *position = c->oldest + row;
    return NMG_OK;
}

extern "C" int nmg_kv_can_append_without_eviction(const nmg_kv_cache* c, int64_t rows, int* answer) {
    if (!c || !answer) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_can_append_without_eviction: null argument");
    if (c->window == 0)
        *answer = 1;
    else if (c->retaining)
        *answer = rows <= c->batch_remaining;
    else
        *answer = rows <= c->window - c->size;
    return NMG_OK;
}

extern "C" int nmg_kv_visible_rows(const nmg_kv_cache* c, int64_t query, int64_t* first, int64_t* end) {
    if (!c || !first || !end) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_visible_rows: null argument");
    // CausalWindow{window}.visible_rows(query, oldest, size) (attention.hpp:170-176).
    int64_t f = 0, e = 0;
    if (query >= c->oldest) {
        const int64_t distance = query - c->oldest;
        e = c->size < distance + 1 ? c->size : distance + 1;
        const int64_t b = (c->window == 0 || distance < c->window) ? 0 : distance + 1 - c->window;
        f = b < e ? b : e;
    }
    *first = f;
    *end = e;
    if (f == e)
        return set_error(NMG_RUNTIME_ERROR, "%s: query has no visible keys",
                         c->window ? "LocalAttentionCache" : "FullAttentionCache");
    return NMG_OK;
}

extern "C" int nmg_kv_begin_batch_retention(nmg_kv_cache* c, int64_t appended_rows) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_begin_batch_retention: null cache");
    if (c->window == 0) return set_error(NMG_LOGIC_ERROR, "batch retention applies to a local cache only");
    if (c->retaining) return set_error(NMG_LOGIC_ERROR, "LocalAttentionCache: batch retention already active");
    if (appended_rows <= 1) return NMG_OK;
    if (c->size + appended_rows > c->slots)
        return set_error(NMG_LENGTH_ERROR,
                         "LocalAttentionCache: retaining %lld rows needs a device capacity of at least %lld slots",
                         (long long)(c->size + appended_rows), (long long)(c->size + appended_rows));
    c->retaining = true;
    c->batch_remaining = appended_rows;
    return NMG_OK;
}

extern "C" int nmg_kv_end_batch_retention(nmg_kv_cache* c) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_end_batch_retention: null cache");
    if (!c->retaining) return NMG_OK;
    if (c->batch_remaining != 0)
        return set_error(NMG_LOGIC_ERROR, "LocalAttentionCache: retained batch was not fully appended");
    const int64_t kept = c->size < c->window ? c->size : c->window;
    c->oldest += c->size - kept;
    c->size = kept;
    c->retaining = false;
    return NMG_OK;
}

extern "C" int nmg_kv_read_row(const nmg_kv_cache* c, int64_t row, int head, float* key_out, float* value_out,
                               void* stream) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_read_row: null cache");
    const char* who = c->window ? "LocalAttentionCache" : "FullAttentionCache";
    if (head < 0 || head >= c->hkv) return set_error(NMG_OUT_OF_RANGE, "%s: K/V head out of range", who);
    if (row < 0 || row >= c->size) return set_error(NMG_OUT_OF_RANGE, "%s: row out of range", who);
    const int es = nmg::cache_elem_size(c->dtype);
    const int64_t slot = c->slot_of(c->oldest + row);
    const size_t off = ((size_t)head * c->slots + slot) * c->dh * es;
    if (c->dtype == NMG_Q8_0) {  // key(row, head) of a Q8_0 cache: scale * quant, exactly
        const int nb = c->dh / 32;
        std::vector<int8_t> kq(c->dh), vq(c->dh);
        std::vector<uint16_t> kd(nb), vd(nb);
        const size_t soff = ((size_t)head * c->sstride + slot) * nb * 2;
        int prev = 0;
        NMG_CUDA_TRY(cudaGetDevice(&prev));
        NMG_CUDA_TRY(cudaSetDevice(c->device));
        cudaStream_t s = (cudaStream_t)stream;
        NMG_CUDA_TRY(cudaMemcpyAsync(kq.data(), (const char*)c->k + off, c->dh, cudaMemcpyDeviceToHost, s));
        NMG_CUDA_TRY(cudaMemcpyAsync(vq.data(), (const char*)c->v + off, c->dh, cudaMemcpyDeviceToHost, s));
        NMG_CUDA_TRY(cudaMemcpyAsync(kd.data(), (const char*)c->ks + soff, nb * 2, cudaMemcpyDeviceToHost, s));
        NMG_CUDA_TRY(cudaMemcpyAsync(vd.data(), (const char*)c->vs + soff, nb * 2, cudaMemcpyDeviceToHost, s));
        NMG_CUDA_TRY(cudaStreamSynchronize(s));
        NMG_CUDA_TRY(cudaSetDevice(prev));
        for (int d = 0; d < c->dh; ++d) {
            if (key_out) key_out[d] = __half2float(__ushort_as_half(kd[d / 32])) * (float)kq[d];
            if (value_out) value_out[d] = __half2float(__ushort_as_half(vd[d / 32])) * (float)vq[d];
        }
        return NMG_OK;
    }
    std::vector<unsigned char> kb((size_t)c->dh * es), vb((size_t)c->dh * es);
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    NMG_CUDA_TRY(cudaSetDevice(c->device));
    NMG_CUDA_TRY(cudaMemcpyAsync(kb.data(), (const char*)c->k + off, kb.size(), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    NMG_CUDA_TRY(cudaMemcpyAsync(vb.data(), (const char*)c->v + off, vb.size(), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    NMG_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    NMG_CUDA_TRY(cudaSetDevice(prev));
    for (int d = 0; d < c->dh; ++d) {
        float kf, vf;
        if (c->dtype == NMG_F32) {
            memcpy(&kf, kb.data() + 4 * d, 4);
            memcpy(&vf, vb.data() + 4 * d, 4);
        } else {
            uint16_t kh, vh;
            memcpy(&kh, kb.data() + 2 * d, 2);
            memcpy(&vh, vb.data() + 2 * d, 2);
            if (c->dtype == NMG_BF16) {
                uint32_t kbits = (uint32_t)kh << 16;
                memcpy(&kf, &kbits, 4);
            } else {
                kf = __half2float(__ushort_as_half(kh));
            }
            vf = __half2float(__ushort_as_half(vh));  // V of a 16-bit cache is fp16
        }
        if (key_out) key_out[d] = kf;
        if (value_out) value_out[d] = vf;
    }
    return NMG_OK;
}

extern "C" int nmg_kv_reset(nmg_kv_cache* c) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_reset: null cache");
    c->size = c->oldest = c->base = c->total = 0;
    c->retaining = false;
    c->batch_remaining = 0;
    return NMG_OK;
}

extern "C" int nmg_kv_storage(const nmg_kv_cache* c, void** keys, void** values, int64_t* slots) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_storage: null cache");
    if (keys) *keys = c->k;
    if (values) *values = c->v;
    if (slots) *slots = c->slots;
    return NMG_OK;
}

extern "C" int nmg_kv_scales(const nmg_kv_cache* c, void** key_scales, void** value_scales, int64_t* rows_per_head) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_scales: null cache");
    if (c->dtype != NMG_Q8_0) return set_error(NMG_INVALID_ARGUMENT, "nmg_kv_scales: not a Q8_0 cache");
    if (key_scales) *key_scales = c->ks;
    if (value_scales) *value_scales = c->vs;
    if (rows_per_head) *rows_per_head = c->sstride;
    return NMG_OK;
}
