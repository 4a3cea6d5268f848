// attn_api.cu -- C ABI for the attention entry points; validation mirrors the
// reference's exceptions, dispatch picks the tensor-core flash kernel or the
// split-KV kernel.
#include <algorithm>
#include <vector>

#include "attn.cuh"

using nmg::set_error;

namespace {

const char* cache_name(const nmg_kv_cache* c) { return c->window ? "LocalAttentionCache" : "FullAttentionCache"; }

// Every query row first_query.. must see a key; the reference asks the cache
// for visible_rows() of every row before it reduces any (qwen35.hpp:360-363).
int check_visible(const nmg_kv_cache* c, int64_t rows, int64_t first_query, int64_t window, int64_t floor_pos,
                  int64_t newest) {
    if (c->size == 0 && c->total == 0)
        return set_error(NMG_RUNTIME_ERROR, "%s: query has no visible keys", cache_name(c));
    // lo rises and hi rises with the query, so only the two ends can be empty
    // ... except a window past the newest row, which grows with the query.
    for (int64_t t : {(int64_t)0, rows - 1}) {
        const nmg::VisibleSpan sp = nmg::visible_span(first_query + t, window, floor_pos, newest);
        if (sp.lo > sp.hi) return set_error(NMG_RUNTIME_ERROR, "%s: query has no visible keys", cache_name(c));
    }
    return NMG_OK;
}

int dispatch_rows(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                  int64_t window, int64_t floor_pos, int64_t newest, float scale, void* out, int out_dtype,
                  cudaStream_t stream) {
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != c->device) NMG_CUDA_TRY(cudaSetDevice(c->device));
    int st;
    if (nmg::prefill_supported(c, hq, q_dtype, rows))
        st = nmg::attend_rows_prefill(c, hq, q, q_dtype, rows, first_query, window, floor_pos, newest, scale, &out, 1,
                                      (int64_t)hq * c->dh, 0, out_dtype, stream);
    else if (nmg::decode_mma_supported(c, q_dtype))
        st = nmg::attend_rows_mma(c, hq, q, q_dtype, rows, first_query, window, floor_pos, newest, scale, out, out_dtype,
                                  stream);
    else if (c->dtype == NMG_Q8_0)
        st = set_error(NMG_UNSUPPORTED, "attention over a Q8_0 cache: head_dim %d is not built", c->dh);
    else
        st = nmg::attend_rows_split(c, hq, q, q_dtype, rows, first_query, window, floor_pos, newest, scale, out,
                                    out_dtype, stream, nullptr, 0);
    if (prev != c->device) cudaSetDevice(prev);
    return st;
}

int validate_heads(const nmg_kv_cache* c, int hq, int q_dtype, int out_dtype) {
    if (hq <= 0 || hq % c->hkv != 0)
        return set_error(NMG_INVALID_ARGUMENT, "attention: %d query heads is not a multiple of %d K/V heads", hq, c->hkv);
    if (!nmg::dtype_valid(q_dtype) || !nmg::dtype_valid(out_dtype))
        return set_error(NMG_INVALID_ARGUMENT, "attention: bad dtype");
    return NMG_OK;
}

}  // namespace

extern "C" int nmg_attend(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
                          float scale, int use_scale, void* out, int out_dtype, void* stream) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend: null cache");
    int st = validate_heads(c, hq, q_dtype, out_dtype);
    if (st != NMG_OK) return st;
    if (rows < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend: negative row count");
    if (rows == 0) return NMG_OK;
    if (!q || !out) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend: null tensor");
    const int64_t newest = c->newest();
    st = check_visible(c, rows, first_query, c->window, c->oldest, newest);
    if (st != NMG_OK) return st;
    return dispatch_rows(c, hq, q, q_dtype, rows, first_query, c->window, c->oldest, newest, use_scale ? scale : 1.f,
                         out, out_dtype, (cudaStream_t)stream);
}

extern "C" int nmg_attend_fanout(const nmg_kv_cache* c, int hq, const void* q, int q_dtype, int64_t rows,
                                 int64_t first_query, float scale, int use_scale, void* const* outs, int nout,
                                 int64_t out_row_elems, int64_t out_col0, int out_dtype, void* stream) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_fanout: null cache");
    int st = validate_heads(c, hq, q_dtype, out_dtype);
    if (st != NMG_OK) return st;
    if (rows < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_fanout: negative row count");
    if (rows == 0) return NMG_OK;
    if (!q || !outs || nout < 1 || nout > 8) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_fanout: 1..8 outputs");
    for (int i = 0; i < nout; ++i)
        if (!outs[i]) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_fanout: null output %d", i);
    const int64_t width = (int64_t)hq * c->dh;
    if (out_col0 < 0 || out_row_elems < out_col0 + width)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_fanout: %lld output columns at %lld do not fit rows of %lld",
                         (long long)width, (long long)out_col0, (long long)out_row_elems);
    const int64_t newest = c->newest();
    st = check_visible(c, rows, first_query, c->window, c->oldest, newest);
    if (st != NMG_OK) return st;
    const float sc = use_scale ? scale : 1.f;
    cudaStream_t s = (cudaStream_t)stream;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != c->device) NMG_CUDA_TRY(cudaSetDevice(c->device));
    const int es = nmg::dtype_size(out_dtype);
    const bool aligned = !(((out_row_elems * es) | (out_col0 * es)) & 15);
    if (aligned && nmg::prefill_supported(c, hq, q_dtype, rows)) {
        st = nmg::attend_rows_prefill(c, hq, q, q_dtype, rows, first_query, c->window, c->oldest, newest, sc, outs,
                                      nout, out_row_elems, out_col0, out_dtype, s);
    } else {
        // Other shapes: reduce into staging, then one strided copy per output.
        void* tmp = nullptr;
        st = nmg::device_staging(c->device, (size_t)rows * width * es, &tmp);
        if (st == NMG_OK)
            st = dispatch_rows(c, hq, q, q_dtype, rows, first_query, c->window, c->oldest, newest, sc, tmp, out_dtype, s);
        for (int i = 0; st == NMG_OK && i < nout; ++i) {
            const cudaError_t e = cudaMemcpy2DAsync((char*)outs[i] + out_col0 * es, (size_t)out_row_elems * es, tmp,
                                                    (size_t)width * es, (size_t)width * es, (size_t)rows,
                                                    cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) st = set_error(NMG_CUDA_ERROR, "nmg_attend_fanout: copy: %s", cudaGetErrorString(e));
        }
    }
    if (prev != c->device) cudaSetDevice(prev);
    return st;
}

extern "C" int nmg_append_attend(nmg_kv_cache* c, int64_t first, const void* keys, const void* values, int kv_dtype,
                                 int hq, const void* q, int q_dtype, int64_t rows, float scale, int use_scale, void* out,
                                 int out_dtype, void* stream) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_append_attend: null cache");
    int st = validate_heads(c, hq, q_dtype, out_dtype);
    if (st != NMG_OK) return st;
    if (rows <= 0) return rows == 0 ? NMG_OK : set_error(NMG_INVALID_ARGUMENT, "nmg_append_attend: negative rows");
    // The floor of every query's window is the oldest row before this batch:
    // the batch path never evicts, and the token-by-token path (one append,
    // one reduce) gives row t exactly [max(p_t - W + 1, oldest_before), p_t].
    const bool empty = c->size == 0 && c->total == 0;
    const int64_t floor_pos = empty ? first : c->oldest;
    if (c->window > 0 && c->retaining && rows > c->batch_remaining) {
        // The reference appends what the retained batch admits, then throws.
        return nmg_kv_append(c, first, keys, values, rows, kv_dtype, stream);
    }
    // A ring can only serve queries whose keys are all still in it: chunk the
    // batch so no chunk overwrites a key its own first query needs.
    int64_t chunk = rows;
    if (c->window > 0 && !c->retaining) chunk = std::min<int64_t>(rows, c->slots - c->window + 1);
    const int es_kv = nmg::dtype_size(kv_dtype), es_q = nmg::dtype_size(q_dtype), es_o = nmg::dtype_size(out_dtype);
    const int64_t kv_row = (int64_t)c->hkv * c->dh, q_row = (int64_t)hq * c->dh;
    for (int64_t done = 0; done < rows; done += chunk) {
        const int64_t n = std::min(chunk, rows - done);
        st = nmg_kv_append(c, first + done, (const char*)keys + done * kv_row * es_kv,
                           (const char*)values + done * kv_row * es_kv, n, kv_dtype, stream);
        if (st != NMG_OK) return st;
        st = dispatch_rows(c, hq, (const char*)q + done * q_row * es_q, q_dtype, n, first + done, c->window, floor_pos,
                           first + done + n - 1, use_scale ? scale : 1.f, (char*)out + done * q_row * es_o, out_dtype,
                           (cudaStream_t)stream);
        if (st != NMG_OK) return st;
    }
    return NMG_OK;
}

extern "C" int nmg_attend_batch(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq,
                                const void* q, int q_dtype, float scale, int use_scale, void* out, int out_dtype,
                                void* stream) {
    if (!caches || batch < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_batch: bad batch");
    if (batch == 0) return NMG_OK;
    const nmg_kv_cache* c0 = caches[0];
    if (!c0) return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_batch: null cache");
    int st = validate_heads(c0, hq, q_dtype, out_dtype);
    if (st != NMG_OK) return st;
    for (int b = 0; b < batch; ++b) {
        const nmg_kv_cache* c = caches[b];
        if (!c || c->hkv != c0->hkv || c->dh != c0->dh || c->dtype != c0->dtype || c->device != c0->device)
            return set_error(NMG_INVALID_ARGUMENT, "nmg_attend_batch: caches differ in shape, dtype or device");
        const int64_t qpos = queries_at ? queries_at[b] : c->newest();
        st = check_visible(c, 1, qpos, c->window, c->oldest, c->newest());
        if (st != NMG_OK) return st;
    }
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != c0->device) NMG_CUDA_TRY(cudaSetDevice(c0->device));
    bool mma = true;
    for (int b = 0; b < batch; ++b) mma = mma && nmg::decode_mma_supported(caches[b], q_dtype);
    if (mma)
        st = nmg::attend_batch_mma(caches, batch, queries_at, hq, q, q_dtype, use_scale ? scale : 1.f, out, out_dtype,
                                   (cudaStream_t)stream);
    else if (c0->dtype == NMG_Q8_0)
        st = set_error(NMG_UNSUPPORTED, "attention over Q8_0 caches: head_dim %d is not built", c0->dh);
    else
        st = nmg::attend_batch_split(caches, batch, queries_at, hq, q, q_dtype, use_scale ? scale : 1.f, out, out_dtype,
                                     (cudaStream_t)stream);
    if (prev != c0->device) cudaSetDevice(prev);
    return st;
}

extern "C" int nmg_sdpa(int heads, int head_dim, const void* q, const void* k, const void* v, int dtype, int64_t tq,
                        int64_t tk, float scale, void* out, int out_dtype, void* stream) {
    if (heads <= 0 || head_dim <= 0 || tq < 0 || tk <= 0)
        return set_error(NMG_INVALID_ARGUMENT, "scaled_dot_product_attention: bad shape");
    if (!nmg::dtype_valid(dtype) || !nmg::dtype_valid(out_dtype))
        return set_error(NMG_INVALID_ARGUMENT, "scaled_dot_product_attention: bad dtype");
    if (tq == 0) return NMG_OK;
    int device = 0;
    NMG_CUDA_TRY(cudaGetDevice(&device));
    // Stage K/V head-major in a transient cache view so both attention kernels
    // apply unchanged: every query sits at the newest position, so no key is masked.
    int64_t slots = (tk + 127) / 128 * 128;
    nmg_kv_cache view;
    view.hkv = heads;
    view.dh = head_dim;
    view.dtype = dtype;
    view.vdtype = nmg::v_dtype_for(dtype);
    view.device = device;
    view.window = 0;
    view.slots = slots;
    const size_t bytes = (size_t)heads * slots * head_dim * nmg::dtype_size(dtype);
    void* buf = nullptr;
    int st = nmg::device_staging(device, 2 * bytes, &buf);
    if (st != NMG_OK) return st;
    view.k = buf;
    view.v = (char*)buf + bytes;
    view.base = 0;
    view.oldest = 0;
    view.size = 0;
    view.total = 0;
    st = nmg::kv_append_device(&view, 0, k, v, tk, dtype, (cudaStream_t)stream);
    if (st != NMG_OK) return st;
    view.size = tk;
    view.total = tk;
    return dispatch_rows(&view, heads, q, dtype, tq, tk - 1, 0, 0, tk - 1, scale, out, out_dtype, (cudaStream_t)stream);
}
