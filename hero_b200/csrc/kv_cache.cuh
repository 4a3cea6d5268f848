// kv_cache.cuh -- the device KV cache object shared by the cache and attention code.
#pragma once
#include "common.cuh"

// Device-resident replacement for FullAttentionCache / LocalAttentionCache
// (nm/src/attention.hpp:201-395).  Storage is head-major, [hkv][slots][dh]
// for K and for V, so one head's keys for consecutive positions are one
// contiguous run (a single bulk copy per tile) and a KV-head group shards by
// pointer offset.  Position p lives in slot (p - base) mod slots.
//
// The logical fields (size, oldest, retention) follow the reference's
// bookkeeping exactly and are kept on the host, so size()/position()/
// visible_rows() never touch the device.
struct nmg_kv_cache {
    int hkv = 0, dh = 0, dtype = NMG_F32, device = 0;
    // Element type of the V buffer.  A bf16 cache keeps V as fp16: a bf16
    // value in fp16's normal range (magnitude 2^-14 .. 65504) is exactly
    // representable in fp16 (smaller ones round to its subnormal grid, error
    // <= 2^-25), and fp16 V lets P.V run fp16 x fp16 with 11-bit probabilities
    // (bf16 P would carry 8).
    int vdtype = NMG_F32;
    int64_t window = 0;  // 0: full (append-only) cache
    int64_t slots = 0;   // physical rows per head
    void* k = nullptr;
    void* v = nullptr;
    // NMG_Q8_0: fp16 block scales [hkv][slots][dh / 32] of K and V (k, v hold
    // the int8 quants [hkv][slots][dh]).
    void* ks = nullptr;
    void* vs = nullptr;
    // Scale rows per head (slots rounded up to 64): every 64-row tile of
    // scales starts 512-byte aligned and stays inside its head.
    int64_t sstride = 0;

    int64_t size = 0;    // logical rows (reference size())
    int64_t oldest = 0;  // position of chronological row 0
    int64_t base = 0;    // first position ever appended (slot origin)
    int64_t total = 0;   // rows ever appended
    bool retaining = false;
    int64_t batch_remaining = 0;

    int64_t newest() const { return oldest + size - 1; }
    // Slot of a position that is physically present.
    int64_t slot_of(int64_t position) const { return (position - base) % slots; }
};

namespace nmg {

inline int v_dtype_for(int dtype) { return dtype == NMG_BF16 ? NMG_F16 : dtype; }
inline bool cache_dtype_valid(int dtype) { return dtype_valid(dtype) || dtype == NMG_Q8_0; }
// Bytes of one cached element (the int8 quants of a Q8_0 cache).
inline int cache_elem_size(int dtype) { return dtype == NMG_Q8_0 ? 1 : dtype_size(dtype); }

// Half-open visible position range of a query for a cache as it stands:
// [max(q - window + 1, floor), min(q, newest)] in positions.
struct VisibleSpan {
    int64_t lo, hi;  // inclusive positions; empty when lo > hi
};

inline VisibleSpan visible_span(int64_t query, int64_t window, int64_t floor_pos, int64_t newest) {
    int64_t lo = floor_pos;
    if (window > 0 && query - window + 1 > lo) lo = query - window + 1;
    int64_t hi = query < newest ? query : newest;
    return VisibleSpan{lo, hi};
}

// Append kernel launcher (kv_cache.cu).
int kv_append_device(nmg_kv_cache* c, int64_t first_position, const void* keys, const void* values, int64_t rows,
                     int src_dtype, cudaStream_t stream);

// nmg_kv_append in two halves for kernels that write the rows themselves.
// kv_append_begin validates an append of `rows` rows at `first` (setting the
// first position of an empty cache) and returns how many rows the cache
// takes (*accepted; fewer than rows only for an overfull retained batch, whose
// error *deferred carries, as the reference appends those rows then throws).
// The accepted rows' device writes go to kv_append_slots' slots, then
// kv_append_commit updates size/oldest/retention.
int kv_append_begin(nmg_kv_cache* c, int64_t first, int64_t rows, int64_t* accepted, int* deferred);
void kv_append_commit(nmg_kv_cache* c, int64_t first, int64_t accepted);
// Of `rows` rows appended at `first`, rows row0.. survive in the ring (at
// most `slots` of them); row row0 + i goes to slot (slot0 + i) % slots.
inline void kv_append_slots(const nmg_kv_cache* c, int64_t first, int64_t rows, int64_t* row0, int64_t* slot0) {
    const int64_t write = rows < c->slots ? rows : c->slots;
    *row0 = rows - write;
    *slot0 = ((first + *row0 - c->base) % c->slots + c->slots) % c->slots;
}

// A bf16 cache's V element: x rounded to bf16, then held as fp16 (exact for
// magnitudes in fp16's normal range).  `overflow` is set when a finite value
// lands on +-inf (bf16 magnitude 65536 or more; fp16's largest is 65504).
__device__ __forceinline__ uint16_t cache_v_from_bf16(uint32_t b, bool& overflow) {
    const uint16_t h = dev::f32_to_f16_bits(dev::bf16_bits_to_f32(b));
    overflow |= (h & 0x7FFFu) == 0x7C00u && (b & 0x7F80u) != 0x7F80u;
    return h;
}
__device__ __forceinline__ uint16_t cache_v_bits(float x, bool& overflow) {
    return cache_v_from_bf16(dev::f32_to_bf16_bits(x), overflow);
}

// A value stored into a V buffer of a cache of dtype `cache_dtype`.
__device__ __forceinline__ void store_cache_v(void* vc, int cache_dtype, int64_t i, float x, bool& overflow) {
    if (cache_dtype == NMG_BF16)
        ((uint16_t*)vc)[i] = cache_v_bits(x, overflow);
    else
        dev::store_from_f32(vc, cache_dtype, i, x);
}

}  // namespace nmg
