/*
 * nmg.h -- C ABI of the B200 (sm_100a) attention / KV-cache / gated delta-rule
 * path for the nm engine.
 *
 * Plain pointers and sizes only.  Every function returns an int status:
 *
 *   NMG_OK                 0
 *   NMG_INVALID_ARGUMENT   1  std::invalid_argument (non-consecutive position, bad shape)
 *   NMG_OUT_OF_RANGE       2  std::out_of_range     (row or head index)
 *   NMG_RUNTIME_ERROR      3  std::runtime_error    (a query with no visible key)
 *   NMG_LENGTH_ERROR       4  std::length_error     (capacity exhausted)
 *   NMG_LOGIC_ERROR        5  std::logic_error      (batch-retention misuse)
 *   NMG_CUDA_ERROR         6  a CUDA runtime call failed
 *   NMG_DEVICE_TIMEOUT     7  a bounded device-side wait gave up
 *   NMG_COMM_ERROR         8  an NCCL call failed
 *   NMG_UNSUPPORTED        9  shape / dtype combination not built
 *   NMG_VALUE_OVERFLOW    10  std::overflow_error    (a V value a bf16 cache cannot hold)
 *
 * nmg_last_error() returns the message of the last failure on this thread.
 * The exception types are the ones the reference throws at the cited lines;
 * include/nmg.hpp maps the codes back onto them.
 *
 * Device pointers are raw device addresses; `stream` is a cudaStream_t (NULL =
 * legacy default stream).  Nothing here synchronises the stream unless it says
 * so.  A handle is used from one host thread and one stream at a time, like the
 * reference's caches, which are owned by one model thread (src/core.cpp:30-54
 * runs one par_for job at a time).
 *
 * Reference paths are relative to the nm/ project root.
 */
#ifndef NMG_H
#define NMG_H

#include <stdint.h>

#if defined(__GNUC__)
#define NMG_API __attribute__((visibility("default")))
#else
#define NMG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define NMG_OK 0
#define NMG_INVALID_ARGUMENT 1
#define NMG_OUT_OF_RANGE 2
#define NMG_RUNTIME_ERROR 3
#define NMG_LENGTH_ERROR 4
#define NMG_LOGIC_ERROR 5
#define NMG_CUDA_ERROR 6
#define NMG_DEVICE_TIMEOUT 7
#define NMG_COMM_ERROR 8
#define NMG_UNSUPPORTED 9
#define NMG_VALUE_OVERFLOW 10

/* Element types.  The reference computes in fp32 (Scalar = float,
 * src/core.hpp:31) and rounds to fp16/bf16 with src/core.hpp:61-100; the
 * device rounds with the same bit-exact rules. */
#define NMG_F32 0
#define NMG_F16 1
#define NMG_BF16 2
/* Cache storage only: K and V as Q8_0 blocks (32 int8 quants and an fp16
 * scale), the format the reference plans behind its append / key / value
 * seam (INFERENCE_PLAN.md, P1.3), quantised as quantize_row_q8_0
 * (src/quant_i8.hpp:69-81).  Queries, inputs and outputs stay F32/F16/BF16. */
#define NMG_Q8_0 3

NMG_API const char* nmg_last_error(void);
NMG_API const char* nmg_version(void);

/* Synchronises `stream` (the legacy default stream when NULL) and reports
 * what kernels on `device` flagged since the last call, then clears it:
 *   NMG_DEVICE_TIMEOUT  a kernel gave up a bounded device-side wait (it
 *                       returned early instead of hanging; its output is not
 *                       valid), including kernels of nmg_attend_noalloc;
 *   NMG_VALUE_OVERFLOW  a finite V value whose bf16 rounding has magnitude
 *                       65536 or more was appended to a bf16 cache, which
 *                       keeps V as fp16 (largest finite 65504): the stored
 *                       value became +-inf.
 * Allocates nothing. */
NMG_API int nmg_device_status(int device, void* stream);

/* Diagnostic (no counterpart in the reference): launches one kernel that waits
 * on a barrier nothing completes, with a short poll limit, so the wait gives up
 * and raises the timeout flag exactly as a stalled kernel would; target 0 is
 * the library's flag, target 1 the no-allocation path's.  The kernel returns;
 * nmg_device_status then reports NMG_DEVICE_TIMEOUT. */
NMG_API int nmg_selftest_wait_timeout(int device, int target, void* stream);

/* ---- device KV cache -------------------------------------------------------
 *
 * Replaces FullAttentionCache<Hkv,HeadDim> (src/attention.hpp:201-250) when
 * window == 0, and LocalAttentionCache<Hkv,HeadDim>(window)
 * (src/attention.hpp:252-395) when window > 0.
 *
 * Device layout: K and V are separate buffers [hkv][slots][head_dim] in
 * `dtype` (NMG_Q8_0: int8 quants, plus fp16 scales, one per 32 values, and
 * head_dim a multiple of 32); the position p lives in slot (p - first position ever appended)
 * mod slots.  `capacity` is the number of slots.  A full cache fails with
 * NMG_LENGTH_ERROR once more than `capacity` rows were appended.  A local
 * cache keeps logical rows exactly as the reference (window-sized ring, batch
 * retention) while physically holding the last `capacity` rows, so one batch
 * of up to capacity - window + 1 rows can be attended as a whole.
 */
typedef struct nmg_kv_cache nmg_kv_cache;

NMG_API int nmg_kv_create(int hkv, int head_dim, int dtype, int64_t window, int64_t capacity, int device, nmg_kv_cache** out);
NMG_API int nmg_kv_destroy(nmg_kv_cache* cache);

/* FullAttentionCache::append / LocalAttentionCache::append, for `rows`
 * consecutive positions first_position.. at once (attention.hpp:215-220,
 * :320-345).  keys/values: device [rows][hkv*head_dim] in src_dtype (the
 * reference's token-major row layout); converted to the cache dtype on the
 * way in.  Positions must continue the cache (NMG_INVALID_ARGUMENT). */
NMG_API int nmg_kv_append(nmg_kv_cache* cache, int64_t first_position, const void* keys, const void* values, int64_t rows,
                  int src_dtype, void* stream);

/* size() / position(row) / window() / can_append_without_eviction(rows)
 * (attention.hpp:207-213, :262-267, :315-318).  Host-side state, no sync. */
NMG_API int nmg_kv_size(const nmg_kv_cache* cache, int64_t* size);
NMG_API int nmg_kv_position(const nmg_kv_cache* cache, int64_t chronological_row, int64_t* position);
NMG_API int nmg_kv_window(const nmg_kv_cache* cache, int64_t* window);
NMG_API int nmg_kv_can_append_without_eviction(const nmg_kv_cache* cache, int64_t rows, int* answer);

/* visible_rows(query) (attention.hpp:222-226, :347-351): the half-open
 * chronological row interval; NMG_RUNTIME_ERROR when it is empty. */
NMG_API int nmg_kv_visible_rows(const nmg_kv_cache* cache, int64_t query_position, int64_t* first, int64_t* end);

/* LocalAttentionCache::begin_batch_retention / end_batch_retention
 * (attention.hpp:274-313).  NMG_LOGIC_ERROR as the reference throws. */
NMG_API int nmg_kv_begin_batch_retention(nmg_kv_cache* cache, int64_t appended_rows);
NMG_API int nmg_kv_end_batch_retention(nmg_kv_cache* cache);

/* key(row, KVHead) / value(row, KVHead) (attention.hpp:228-237, :353-360) as a
 * synchronous copy-back to host fp32 [head_dim]; a debug accessor. */
NMG_API int nmg_kv_read_row(const nmg_kv_cache* cache, int64_t chronological_row, int kv_head, float* key_out, float* value_out,
                    void* stream);

/* Forget every row (a new sequence on the same device storage), the device
 * counterpart of dropping a PrefixState's carried caches
 * (src/transformer.hpp:154-160).  No device work. */
NMG_API int nmg_kv_reset(nmg_kv_cache* cache);

/* Raw device storage, for callers that fuse their own producer. */
NMG_API int nmg_kv_storage(const nmg_kv_cache* cache, void** keys, void** values, int64_t* slots);

/* The block scales of an NMG_Q8_0 cache: fp16 bit patterns
 * [hkv][rows_per_head][head_dim/32] (rows_per_head = slots rounded up to 64;
 * slot s of head h is row h * rows_per_head + s) beside the int8 quants of
 * nmg_kv_storage ([hkv][slots][head_dim]); a cached value is scale * quant
 * (fp16_to_fp32(d) * qs, src/quant.hpp:59-62).  NMG_INVALID_ARGUMENT for other
 * cache dtypes. */
NMG_API int nmg_kv_scales(const nmg_kv_cache* cache, void** key_scales, void** value_scales, int64_t* rows_per_head);

/* ---- attention ---------------------------------------------------------------
 *
 * The softmax reduction the reference writes inline per layer
 * (src/qwen35.hpp:360-382; src/gemma4.hpp:211-235, :302-321, :593-615,
 * :687-709): for every query row t (position first_query + t) and query head h,
 *   out[t,h] = sum_j softmax_j(s_j) * V[j, h/(hq/hkv)],
 *   s_j = scale * dot(q[t,h], K[j, h/(hq/hkv)])        (use_scale != 0, Qwen)
 *   s_j =         dot(q[t,h], K[j, h/(hq/hkv)])        (use_scale == 0, Gemma)
 * over the cache's visible_rows(first_query + t) as the cache stands now.
 * q: device [rows][hq*head_dim] in q_dtype; out: device [rows][hq*head_dim] in
 * out_dtype.  Dispatches to the tcgen05 flash kernel for 16-bit caches with
 * head_dim 64/128/256 and many rows, and to the split-KV decode kernels
 * otherwise (head_dim 1..256 in powers of two for fp32 caches; 64, 128, 256
 * and 512 for 16-bit caches; NMG_UNSUPPORTED for any other).
 * NMG_RUNTIME_ERROR if any query sees no key (checked on the host first). */
NMG_API int nmg_attend(const nmg_kv_cache* cache, int hq, const void* q, int q_dtype, int64_t rows, int64_t first_query,
               float scale, int use_scale, void* out, int out_dtype, void* stream);

/* The append-then-reduce step of a layer in one call.  Equivalent to the
 * reference's own choice (gemma4.hpp:237-253, :617-630): when the batch fits
 * without eviction it appends and reduces the batch; otherwise it gives every
 * query the keys the token-by-token path would (append one row, reduce one
 * query), computed as one batched kernel, chunking batches larger than the
 * ring's spare capacity. */
NMG_API int nmg_append_attend(nmg_kv_cache* cache, int64_t first_position, const void* keys, const void* values, int kv_dtype,
                      int hq, const void* q, int q_dtype, int64_t rows, float scale, int use_scale, void* out,
                      int out_dtype, void* stream);

/* Batched single-token decode over `batch` independent caches (one reference
 * cache per sequence), query b at position queries_at[b] (host array; pass
 * NULL for "each cache's newest position").  q: device [batch][hq*head_dim];
 * out: device [batch][hq*head_dim].  All caches share hkv/head_dim/dtype. */
NMG_API int nmg_attend_batch(const nmg_kv_cache* const* caches, int batch, const int64_t* queries_at, int hq, const void* q,
                     int q_dtype, float scale, int use_scale, void* out, int out_dtype, void* stream);

/* nmg_attend for callers that cannot allocate device memory (no counterpart in
 * the reference: its CPU path never allocates device memory).  Same result as
 * nmg_attend on the split-KV decode kernel, with that kernel's scratch in a
 * fixed 4 MiB device array per device instead of library-allocated memory;
 * nothing is allocated on any call.  Calls needing more scratch than that
 * fail with NMG_LENGTH_ERROR (one decode row over a long cache needs well
 * under 1 MiB).  The first call on a device looks the array up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * The array is shared by all calls on a device: calls whose kernels overlap
 * on the GPU race on it and must be serialised by the caller. */
NMG_API int nmg_attend_noalloc(const nmg_kv_cache* cache, int hq, const void* q, int q_dtype, int64_t rows,
                               int64_t first_query, float scale, int use_scale, void* out, int out_dtype, void* stream);

/* Dense, unmasked attention scaled_dot_product_attention<Heads,Dqk,Dv>
 * (src/attention.hpp:124-139) over plain device tensors q [tq][heads*d],
 * k/v [tk][heads*d] (no cache, no mask; heads == kv heads). */
NMG_API int nmg_sdpa(int heads, int head_dim, const void* q, const void* k, const void* v, int dtype, int64_t tq, int64_t tk,
             float scale, void* out, int out_dtype, void* stream);

/* ---- gated delta-rule state -------------------------------------------------
 *
 * DeltaNetState<Heads,Dk,Dv> (src/recurrent.hpp:117-138): device fp32
 * [heads][dk][dv], row i = key dim, column j = value dim, zero-initialised. */
typedef struct nmg_delta_state nmg_delta_state;

NMG_API int nmg_delta_create(int heads, int dk, int dv, int device, nmg_delta_state** out);
NMG_API int nmg_delta_destroy(nmg_delta_state* state);
NMG_API int nmg_delta_clear(nmg_delta_state* state, void* stream);
/* head(h) (recurrent.hpp:127-134): device pointer to the [dk][dv] block. */
NMG_API int nmg_delta_head(nmg_delta_state* state, int head, float** head_ptr);

/* gated_delta_step<Dk,Dv> (recurrent.hpp:146-177) for one head and one token:
 * decay = exp(gate); S *= decay; pred = S^T k; d = (v - pred) * beta;
 * S += k (x) d; out = S^T q (read after the write).  All device fp32;
 * gate/beta are device scalars so a graph can replay the step. */
NMG_API int nmg_gated_delta_step(float* state_head, int dk, int dv, const float* q, const float* k, const float* v,
                         const float* gate, const float* beta, float* out, void* stream);

/* One token through every value head: the loop of src/qwen35.hpp:449-454.
 * q,k: [hk][dk] (L2-normalised, q pre-scaled, as recurrent.hpp:144-145
 * requires), v: [heads][dv], gate/beta: [heads], out: [heads][dv]; value head
 * h reads key head h % hk (qwen35.hpp:172). */
NMG_API int nmg_delta_step(nmg_delta_state* state, int hk, const float* q, const float* k, const float* v, const float* gate,
                   const float* beta, float* out, void* stream);

/* One decode token for each of `batch` sequences, each with its own state
 * (the reference keeps one DeltaNetState per sequence's PrefixState and runs
 * the head loop of qwen35.hpp:449-454 per sequence; this is that loop over a
 * batch of sequences in one launch).  states[b]: handles of equal shape on one
 * device; q,k: [batch][hk][dk]; v: [batch][heads][dv]; gate/beta:
 * [batch][heads]; out: [batch][heads][dv].  Dk = 128 with Dv a multiple of 64
 * (16-byte aligned v and out) streams the states in one kernel; other shapes
 * run nmg_delta_step per sequence. */
NMG_API int nmg_delta_step_batch(nmg_delta_state* const* states, int batch, int hk, const float* q, const float* k,
                                 const float* v, const float* gate, const float* beta, float* out, void* stream);

/* T tokens of the same recurrence (qwen35.hpp:436-456 over a prefill batch):
 * q,k: [T][hk][dk], v: [T][heads][dv], gate/beta: [T][heads],
 * out: [T][heads][dv].  chunk = 0 runs the token-sequential kernel; chunk = 64
 * runs the chunked WY-form tensor-core kernel where it is built (Dk = 128, Dv a
 * multiple of 32, q/k/v/out 16-byte aligned) and the token-sequential kernel
 * for other shapes.  Both compute the same recurrence; the chunked one
 * multiplies tf32-rounded operands with fp32 sums (relative L2 error against
 * the fp32 recurrence of a few 1e-4 over 8192 tokens). */
NMG_API int nmg_delta_prefill(nmg_delta_state* state, int hk, int64_t T, const float* q, const float* k, const float* v,
                      const float* gate, const float* beta, float* out, int chunk, void* stream);

/* ---- the steps either side of the attention reduction -------------------------
 *
 * Before the reduction (replaces the Q/K/V preparation of qwen35.hpp:343-352 and
 * gemma4.hpp:206-209, :676-680):
 *   Q = rope(rmsnorm_per_head(q; q_gamma, eps)) written to q_out [T][hq*head_dim]
 *       in q_dtype (the reference's fp32 -> bf16/fp16 rounding);
 *   K = rope(rmsnorm_per_head(k; k_gamma, eps)) and V (v_norm = 0), or
 *   V = rmsnorm_no_scale_per_head(v; eps) (v_norm = 1, Gemma 4, components.hpp:204-215)
 *       appended to the cache at position.. (nmg_kv_append's rules).
 * q is [T][hq*head_dim], or with q_gated = 1 the Qwen 3.5 query projection
 * [T][2*hq*head_dim] in head-major pairs q_0 | gate_0 | q_1 | gate_1 ...
 * (attention.hpp:31-57); k and v are [T][hkv*head_dim] fp32 (k == v is allowed,
 * Gemma's unified projection).  RMSNorm<HeadDim> per head (components.hpp:167-180,
 * :248-281); RoPE half-split, inv_freq_i = rope_base^(-2i/head_dim) rounded from
 * double for the first rotary_num/rotary_den of the planes and 0 for the rest,
 * angle = float(position + t) * inv_freq_i (RotaryEmbedding<HeadDim,Base,Num,Den>,
 * attention.hpp:68-101).  head_dim a multiple of 64 up to 512.  Uses the
 * library's staging memory: calls on one GPU are ordered by their stream. */
NMG_API int nmg_attn_prologue(nmg_kv_cache* cache, int hq, int64_t position, int64_t T, const float* q, int q_gated,
                              const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm,
                              float eps, double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype,
                              void* stream);
/* The same preparation without a cache: K (rotated) to k_out and, with v_norm, V
 * (normed) to v_out, both fp32 [T][hkv*head_dim]; v_out is unused (may be NULL)
 * without v_norm.  For callers that append through nmg_append_attend, e.g. a
 * Gemma 4 sliding-window layer whose batch would evict (gemma4.hpp:237-253). */
NMG_API int nmg_attn_prepare(int hq, int hkv, int head_dim, int64_t position, int64_t T, const float* q, int q_gated,
                             const float* k, const float* v, const float* q_gamma, const float* k_gamma, int v_norm,
                             float eps, double rope_base, int rotary_num, int rotary_den, void* q_out, int q_dtype,
                             float* k_out, float* v_out, void* stream);
/* After the reduction (qwen35.hpp:390-393): a[t][h*head_dim + i] *= sigmoid(gate_h[i]),
 * the gates the second halves of qg's [T][2*hq*head_dim] head pairs; a [T][hq*head_dim]
 * in a_dtype, in place. */
NMG_API int nmg_attn_gate(int64_t T, int hq, int head_dim, const float* qg, void* a, int a_dtype, void* stream);

/* ---- the steps either side of the recurrence ---------------------------------
 *
 * A Qwen 3.5 recurrent layer around gated_delta_step (src/qwen35.hpp:420-461).
 *
 * CausalConv1dState<Channels,Width> (src/recurrent.hpp:63-110): the last
 * width - 1 inputs of a depthwise causal conv, zero-initialised (the causal
 * pad), on the device as [width - 1][channels] fp32, oldest row first. */
typedef struct nmg_conv_state nmg_conv_state;

NMG_API int nmg_conv_create(int channels, int width, int device, nmg_conv_state** out);
NMG_API int nmg_conv_destroy(nmg_conv_state* state);
NMG_API int nmg_conv_clear(nmg_conv_state* state, void* stream);
/* Device pointer to the history rows (for inspection and tests). */
NMG_API int nmg_conv_history(const nmg_conv_state* state, float** hist);
/* CausalConv1dState::step (recurrent.hpp:76-88) over T tokens:
 * y[t][c] = sum_i w[c][i] x[c][t - (W-1) + i], x/y: [T][channels] fp32,
 * weights: [channels][width] (one row of taps per channel, tap 0 oldest);
 * silu != 0 applies x / (1 + e^-x) to y (Silu, src/components.hpp:102-105).
 * The history advances by the T inputs.  At most 65535 * 16 tokens a call. */
NMG_API int nmg_conv_step(nmg_conv_state* state, const float* weights, const float* x, int64_t T, float* y, int silu,
                          void* stream);

/* The delta-net prologue of T tokens (qwen35.hpp:396-415, :436-446): the
 * packed projection qkv [T][2*hk*dk + hv*dv] ([q | k | v] channels) through
 * the conv state and SiLU; q and k L2-normalised per key head (eps 1e-6,
 * recurrent.hpp:40-48) and q scaled by 1/sqrt(dk); beta = sigmoid(beta_raw),
 * gate = decay_scale[h] * softplus(alpha_raw + dt_bias[h]) (recurrent.hpp:35,
 * core.hpp:579).  Outputs in the layouts nmg_delta_prefill takes: q,k
 * [T][hk][dk], v [T][hv][dv], beta/gate [T][hv].  dk and dv multiples of 32
 * up to 1024; at most 65535 * 16 tokens a call. */
NMG_API int nmg_delta_prologue(nmg_conv_state* conv, const float* conv_weights, int hk, int hv, int dk, int dv, int64_t T,
                               const float* qkv, const float* beta_raw, const float* alpha_raw, const float* dt_bias,
                               const float* decay_scale, float* q, float* k, float* v, float* beta, float* gate,
                               void* stream);
/* The gated output norm (qwen35.hpp:458-460): out[t][h][j] =
 * gamma[j] * o[t][h][j] * inv_rms(o[t][h]) * SiLU(z[t][h][j]) with
 * inv_rms = 1 / sqrt(mean(o^2) + eps) (RMSNorm, components.hpp:167-180, per
 * head, :248-281).  o, z, out: [T][hv][dv]; gamma: [dv]. */
NMG_API int nmg_delta_epilogue(int hv, int dv, int64_t T, const float* o, const float* z, const float* gamma, float eps,
                               float* out, void* stream);

/* One decode token of the linear-attention layer core in one launch
 * (qwen35.hpp:396-461 at T = 1): the prologue of nmg_delta_prologue (conv +
 * SiLU, per-key-head L2 norms, q's 1/sqrt(Dk), beta and the decay gate), the
 * recurrent step of nmg_delta_step over every value head and the gated output
 * norm of nmg_delta_epilogue, replacing those three launches per layer and
 * token.  qkv: [2*Hk*Dk + Hv*Dv] ([q | k | v] channels); beta_raw, alpha_raw,
 * dt_bias, decay_scale: [Hv]; z, out: [Hv][Dv]; gamma: [Dv].  The conv
 * history and the state advance by the token.  Hv is the state's head count.
 * Built for Dk = 128, Dv a multiple of 32 and (Hv/Hk) x (Dv/32) <= 8 (Qwen
 * 3.5's 32 value / 16 key heads at 128); other shapes return NMG_UNSUPPORTED
 * and take the three calls. */
NMG_API int nmg_delta_decode_token(nmg_delta_state* state, nmg_conv_state* conv, const float* conv_weights, int hk,
                                   const float* qkv, const float* beta_raw, const float* alpha_raw,
                                   const float* dt_bias, const float* decay_scale, const float* z, const float* gamma,
                                   float eps, float* out, void* stream);

/* ---- multi-GPU: KV-head-group sharding + one all-gather --------------------
 *
 * The reference has no distributed backend (it runs par_for on one host).
 * These sit outside it: one process per GPU, NCCL over NVLink.  The unique id
 * (128 bytes) is made on rank 0 and shipped to the others by the caller. */
typedef struct nmg_comm nmg_comm;

NMG_API int nmg_comm_unique_id(void* id128);
NMG_API int nmg_comm_init(const void* id128, int rank, int world, int device, nmg_comm** out);
NMG_API int nmg_comm_destroy(nmg_comm* comm);
/* All-gather of equal byte-sized blocks: recv[world][bytes_per_rank]. */
NMG_API int nmg_allgather(nmg_comm* comm, const void* send, void* recv, int64_t bytes_per_rank, void* stream);
/* Scatter the gathered per-rank head blocks [world][rows][hq_local*d] into
 * the reference row layout [rows][world*hq_local*d] (elem_bytes per value). */
NMG_API int nmg_gather_heads_to_rows(const void* gathered, void* out, int world, int64_t rows, int64_t row_bytes_per_rank,
                             void* stream);
/* Stream-ordered barrier: completes on each rank once every rank's earlier
 * work on its stream has completed (used after nmg_attend_fanout wrote into
 * the other ranks' buffers). */
NMG_API int nmg_comm_barrier(nmg_comm* comm, void* stream);

/* ---- the gather fused into the attention epilogue ---------------------------
 *
 * No reference counterpart (the reference is single-process).  Each rank
 * allocates its output buffer with nmg_shared_alloc and ships the 64-byte
 * handle to the other ranks of the node, which map it with nmg_ipc_open.
 * nmg_attend_fanout then writes this rank's heads of every output row into
 * all mapped buffers at once (NVLink stores from the epilogue), so the
 * reference's [rows][H*D] rows assemble on every GPU without a separate
 * all-gather; nmg_comm_barrier orders the stores before the rows are read. */
NMG_API int nmg_shared_alloc(int64_t bytes, int device, void** ptr, void* handle64);
NMG_API int nmg_shared_free(void* ptr);
NMG_API int nmg_ipc_open(const void* handle64, int device, void** ptr);
NMG_API int nmg_ipc_close(void* ptr);
/* nmg_attend for the cache's heads, each output row t (hq*head_dim values)
 * written to outs[i] + t*out_row_elems + out_col0 (elements) for i < nout
 * (1..8 device pointers, this GPU's or mapped peers'). */
NMG_API int nmg_attend_fanout(const nmg_kv_cache* cache, int hq, const void* q, int q_dtype, int64_t rows,
                              int64_t first_query, float scale, int use_scale, void* const* outs, int nout,
                              int64_t out_row_elems, int64_t out_col0, int out_dtype, void* stream);

/* ---- quantised projections (src/quant.hpp, src/quant_i8.hpp) ----------------
 *
 * Weight<In,Out> over GGUF tensors (quant.hpp:439-487): one row of `in`
 * values per output, stored as GGUF blocks.  Type codes are GGUF's
 * (quant.hpp:18-27).  F16 and BF16 rows are widened to fp32 at creation, as
 * the reference's loader does; everything else stays in its block format. */
#define NMG_GT_F32 0
#define NMG_GT_F16 1
#define NMG_GT_Q4_0 2
#define NMG_GT_Q8_0 8
#define NMG_GT_Q4_K 12
#define NMG_GT_Q5_K 13
#define NMG_GT_Q6_K 14
#define NMG_GT_Q8_K 15 /* activation blocks only */
#define NMG_GT_BF16 30
/* Activation handling of a product: the reference's default (activations
 * quantised to Q8_0 / Q8_K once per row and integer block dots, for Q8_0,
 * Q4_0, Q4_K and Q6_K; fp32 otherwise) or its NM_FP32_ACT path (fp32
 * activations against blocks dequantised inside the dot, every type). */
#define NMG_ACT_DEFAULT 0
#define NMG_ACT_FP32 1
typedef struct nmg_weight nmg_weight;
/* type_size_bytes (quant.hpp:89-108): bytes of one row of `in` values;
 * NMG_INVALID_ARGUMENT for an unknown type or a row that is not whole blocks. */
NMG_API int nmg_weight_row_bytes(int type, int64_t in, int64_t* bytes);
/* The Weight(GT, data, keepalive) constructor (quant.hpp:456-460): `data`
 * holds out * row_bytes GGUF bytes, on the host or (data_on_device != 0) on
 * `device`; the weight keeps its own device copy.  NMG_UNSUPPORTED for fp32
 * rows whose length is not a multiple of 4. */
NMG_API int nmg_weight_create(int type, int64_t in, int64_t out, const void* data, int data_on_device, int device,
                              nmg_weight** w);
NMG_API int nmg_weight_destroy(nmg_weight* w);
/* type() (F16/BF16 report NMG_GT_F32, as stored), In, Out. */
NMG_API int nmg_weight_info(const nmg_weight* w, int* type, int64_t* in, int64_t* out);
/* Weight::matvec (quant_i8.hpp:351-428): y[out] = W x, device fp32 x[in]
 * (16-byte aligned) and y[out]. */
NMG_API int nmg_weight_matvec(const nmg_weight* w, const float* x, float* y, int act, void* stream);
/* Weight::matmul (quant_i8.hpp:430-514): y[rows][out] for x[rows][in]. */
NMG_API int nmg_weight_matmul(const nmg_weight* w, int64_t rows, const float* x, float* y, int act, void* stream);
/* Weight::gather_rows (quant.hpp:469-475): rows[0..n) (host indices, each
 * < out, else NMG_OUT_OF_RANGE) dequantised to device fp32 out[n][in], bit
 * for bit dequant_to_f32.  Returns once the indices were consumed. */
NMG_API int nmg_weight_gather_rows(const nmg_weight* w, const int32_t* rows, int64_t n, float* out, void* stream);
/* quantize_row_q8_0 / quantize_row_q8_K (quant_i8.hpp:38-81) of rows x n
 * device fp32 values into the reference's packed blocks (34-byte block_q8_0,
 * 292-byte block_q8_K) at device `blocks`. */
NMG_API int nmg_quantize_activations(int act_type, int64_t rows, int64_t n, const float* x, void* blocks, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NMG_H */
