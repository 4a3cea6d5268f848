/*
 * nm_oracle.c -- CPU restatement of the nm engine's attention / KV-cache /
 * gated delta-rule arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path under hero_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  Nothing in the product links it.
 *
 * Every function restates one piece of the reference (paths relative to the
 * nm/ project root) and keeps its floating-point operation order, so that the
 * result matches the reference's own fp32 code up to FMA contraction:
 *
 *   nmo_visible_rows        src/attention.hpp:170-176   CausalWindow::visible_rows
 *   nmo_contains            src/attention.hpp:159-162   CausalWindow::contains
 *   nmo_attend              src/qwen35.hpp:360-382, src/gemma4.hpp:211-235,
 *                           tests/property_tests.cpp:33-56 (the reduction:
 *                           dot -> scale -> Softmax -> scaled_add)
 *   nmo_softmax_inplace     src/components.hpp:131-141
 *   nmo_dot                 src/core.hpp:495-500 (sequential fp32 accumulate)
 *   nmo_gated_delta_step    src/recurrent.hpp:146-177
 *   nmo_delta_run           src/qwen35.hpp:449-454 (head loop, key head h % Hk)
 *   nmo_l2_normalize        src/recurrent.hpp:40-48
 *   nmo_softplus            src/recurrent.hpp:35
 *   nmo_sigmoid             src/core.hpp:579
 *   nmo_conv_run            src/recurrent.hpp:63-110 (CausalConv1dState::step over T tokens)
 *   nmo_silu                src/components.hpp:102-105
 *   nmo_delta_prologue      src/qwen35.hpp:396-415, :436-446 (conv, SiLU, L2 norms, gates)
 *   nmo_delta_epilogue      src/qwen35.hpp:458-460, src/components.hpp:167-180, :248-281
 *   nmo_rope_freqs, nmo_rope src/attention.hpp:68-92 (RotaryEmbedding table, one head)
 *   nmo_rmsnorm             src/components.hpp:167-180 (RMSNorm), :204-215 (RMSNormNoScale)
 *   nmo_attn_prologue       src/qwen35.hpp:343-352, src/gemma4.hpp:206-209, :676-680
 *   nmo_attn_gate           src/qwen35.hpp:390-393
 *   nmo_fp32_to_bf16 etc.   src/core.hpp:34-100
 *   nmo_quantize_q8_0       src/quant_i8.hpp:69-81 (quantize_row_q8_0: Q8_0 blocks of 32)
 *
 * Inputs are plain row-major fp32 arrays in the reference's own layouts:
 * activations [rows][heads*dim] (heads contiguous inside a row), cached K/V
 * [chronological row][Hkv*HeadDim], delta state [head][Dk][Dv].
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define NMO_OK 0
#define NMO_INVALID_ARGUMENT 1
#define NMO_OUT_OF_RANGE 2
#define NMO_RUNTIME_ERROR 3

/* ---- fp16 / bf16 conversions: src/core.hpp:34-100 ------------------------ */

float nmo_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            /* subnormal: normalise the mantissa, counting the shifts */
            int shifts = -1;
            do {
                m <<= 1;
                ++shifts;
            } while ((m & 0x400u) == 0);
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(112 - shifts) << 23) | (m << 13);
        }
    } else if (e == 0x1F) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t nmo_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t m = x & 0x7FFFFFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t r = m >> shift;
        if ((m >> (shift - 1)) & 1u) ++r; /* the reference rounds half up here */
        return (uint16_t)(sign | r);
    }
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    uint16_t h = (uint16_t)(sign | ((uint32_t)e << 10) | (m >> 13));
    if (m & 0x1000u) ++h;
    return h;
}

float nmo_bf16_to_fp32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t nmo_fp32_to_bf16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    if ((bits & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

void nmo_round_bf16(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = nmo_bf16_to_fp32(nmo_fp32_to_bf16(x[i]));
}
void nmo_round_fp16(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = nmo_fp16_to_fp32(nmo_fp32_to_fp16(x[i]));
}
void nmo_to_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = nmo_fp32_to_bf16(x[i]);
}
void nmo_to_fp16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = nmo_fp32_to_fp16(x[i]);
}

/* ---- seeded input generator ------------------------------------------------
 * SplitMix64 counter stream + Box-Muller.  Element i of stream (seed, stream)
 * is a pure function of (seed, stream, i), so any slice can be regenerated
 * independently (the GPU bench uses the same construction on the device). */

static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static double unit_open(uint64_t bits) { /* (0, 1], 53 bits */
    return ((double)(bits >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}

void nmo_normal(uint64_t seed, uint64_t stream, uint64_t first, int64_t n, float* out) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
    for (int64_t j = 0; j < n; ++j) {
        uint64_t i = first + (uint64_t)j;
        uint64_t pair = i >> 1;
        double u1 = unit_open(splitmix64(key + 2 * pair));
        double u2 = unit_open(splitmix64(key + 2 * pair + 1));
        double r = sqrt(-2.0 * log(u1));
        double a = 6.283185307179586 * u2;
        out[j] = (float)((i & 1) ? r * sin(a) : r * cos(a));
    }
}

void nmo_uniform_int(uint64_t seed, uint64_t stream, int64_t n, int64_t lo, int64_t hi, int64_t* out) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
    const uint64_t span = (uint64_t)(hi - lo + 1);
    for (int64_t j = 0; j < n; ++j) out[j] = lo + (int64_t)(splitmix64(key + (uint64_t)j) % span);
}

/* ---- mask: src/attention.hpp:154-176 -------------------------------------- */

int nmo_contains(int64_t width, int64_t key, int64_t query) {
    if (key > query) return 0;
    return width == 0 || query - key < width;
}

void nmo_visible_rows(int64_t width, int64_t query, int64_t oldest, int64_t rows, int64_t* first, int64_t* end) {
    if (query < oldest) {
        *first = 0;
        *end = 0;
        return;
    }
    int64_t distance = query - oldest;
    int64_t e = rows < distance + 1 ? rows : distance + 1;
    int64_t b = (width == 0 || distance < width) ? 0 : distance + 1 - width;
    *first = b < e ? b : e;
    *end = e;
}

/* ---- the reduction --------------------------------------------------------- */

float nmo_dot(const float* a, const float* b, int64_t n) {
    float s = 0.f;
    for (int64_t i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

void nmo_softmax_inplace(float* v, int64_t n) {
    float largest = v[0];
    for (int64_t i = 1; i < n; ++i)
        if (v[i] > largest) largest = v[i];
    float total = 0.f;
    for (int64_t i = 0; i < n; ++i) {
        v[i] = expf(v[i] - largest);
        total += v[i];
    }
    for (int64_t i = 0; i < n; ++i) v[i] /= total;
}

typedef struct {
    const float* keys;   /* [rows][hkv*dh], chronological */
    const float* values; /* [rows][hkv*dh] */
    int64_t rows, oldest, window;
    int hkv, dh, hq;
    const float* q; /* [qrows][hq*dh] */
    int64_t qrows, first_query;
    float scale;
    int use_scale; /* 0: Gemma form (no multiply), 1: Qwen form (scale * dot) */
    float* out;    /* [qrows][hq*dh] */
    int64_t next_task;
    pthread_mutex_t lock;
} attend_job;

static void attend_task(attend_job* J, int64_t task, float* alpha) {
    const int64_t row = task / J->hq;
    const int head = (int)(task % J->hq);
    const int group = head / (J->hq / J->hkv);
    const int width = J->hkv * J->dh;
    int64_t first, end;
    nmo_visible_rows(J->window, J->first_query + row, J->oldest, J->rows, &first, &end);
    const float* query = J->q + row * (int64_t)J->hq * J->dh + (int64_t)head * J->dh;
    const int64_t count = end - first;
    for (int64_t j = first; j < end; ++j) {
        float d = nmo_dot(query, J->keys + j * width + (int64_t)group * J->dh, J->dh);
        alpha[j - first] = J->use_scale ? J->scale * d : d;
    }
    nmo_softmax_inplace(alpha, count);
    float* o = J->out + row * (int64_t)J->hq * J->dh + (int64_t)head * J->dh;
    for (int i = 0; i < J->dh; ++i) o[i] = 0.f;
    for (int64_t n = 0; n < count; ++n) {
        const float* v = J->values + (first + n) * width + (int64_t)group * J->dh;
        const float a = alpha[n];
        for (int i = 0; i < J->dh; ++i) o[i] += a * v[i];
    }
}

static void* attend_worker(void* arg) {
    attend_job* J = (attend_job*)arg;
    float* alpha = (float*)malloc(sizeof(float) * (size_t)(J->rows > 0 ? J->rows : 1));
    for (;;) {
        pthread_mutex_lock(&J->lock);
        int64_t t = J->next_task;
        J->next_task += 1;
        pthread_mutex_unlock(&J->lock);
        if (t >= J->qrows * J->hq) break;
        attend_task(J, t, alpha);
    }
    free(alpha);
    return NULL;
}

/* Attention of `qrows` query rows at positions first_query.. over a cache whose
 * `rows` chronological rows start at position `oldest`, visible through a
 * causal window of `window` (0 = full).  Returns NMO_RUNTIME_ERROR when some
 * query sees no key (attention.hpp:224, :349) and NMO_INVALID_ARGUMENT for a
 * head count that is not a whole GQA group. */
int nmo_attend(const float* keys, const float* values, int64_t rows, int64_t oldest, int64_t window, int hkv, int dh,
               const float* q, int64_t qrows, int hq, int64_t first_query, float scale, int use_scale, float* out,
               int threads) {
    if (hkv <= 0 || dh <= 0 || hq <= 0 || hq % hkv != 0) return NMO_INVALID_ARGUMENT;
    for (int64_t r = 0; r < qrows; ++r) {
        int64_t f, e;
        nmo_visible_rows(window, first_query + r, oldest, rows, &f, &e);
        if (f == e) return NMO_RUNTIME_ERROR;
    }
    attend_job J;
    J.keys = keys;
    J.values = values;
    J.rows = rows;
    J.oldest = oldest;
    J.window = window;
    J.hkv = hkv;
    J.dh = dh;
    J.hq = hq;
    J.q = q;
    J.qrows = qrows;
    J.first_query = first_query;
    J.scale = scale;
    J.use_scale = use_scale;
    J.out = out;
    J.next_task = 0;
    pthread_mutex_init(&J.lock, NULL);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, attend_worker, &J);
    attend_worker(&J);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
    pthread_mutex_destroy(&J.lock);
    return NMO_OK;
}

/* ---- the gated delta rule: src/recurrent.hpp:146-177 ----------------------- */

void nmo_gated_delta_step(float* state, const float* q, const float* k, const float* v, float gate, float beta,
                          float* out, int dk, int dv, float* scratch /* [2*dv] */) {
    const float decay = expf(gate);
    float* predicted = scratch;
    float* delta = scratch + dv;
    for (int j = 0; j < dv; ++j) predicted[j] = 0.f;
    for (int i = 0; i < dk; ++i) {
        float* row = state + (int64_t)i * dv;
        const float ki = k[i];
        for (int j = 0; j < dv; ++j) {
            row[j] *= decay;
            predicted[j] += row[j] * ki;
        }
    }
    for (int j = 0; j < dv; ++j) delta[j] = (v[j] - predicted[j]) * beta;
    for (int j = 0; j < dv; ++j) out[j] = 0.f;
    for (int i = 0; i < dk; ++i) {
        float* row = state + (int64_t)i * dv;
        const float ki = k[i], qi = q[i];
        for (int j = 0; j < dv; ++j) {
            row[j] += ki * delta[j];
            out[j] += row[j] * qi;
        }
    }
}

/* The per-token head loop of src/qwen35.hpp:436-456 after the conv/normalise
 * prologue: q,k are [T][hk][dk] (already L2-normalised, q already scaled),
 * v is [T][hv][dv], gate/beta are [T][hv], state is [hv][dk][dv] (in/out),
 * out is [T][hv][dv].  Value head h reads key head h % hk (qwen35.hpp:172). */
void nmo_delta_run(float* state, int64_t T, int hk, int hv, int dk, int dv, const float* q, const float* k,
                   const float* v, const float* gate, const float* beta, float* out) {
    float* scratch = (float*)malloc(sizeof(float) * 2 * (size_t)dv);
    for (int64_t t = 0; t < T; ++t) {
        for (int h = 0; h < hv; ++h) {
            const int kh = h % hk;
            nmo_gated_delta_step(state + (int64_t)h * dk * dv, q + (t * hk + kh) * (int64_t)dk,
                                 k + (t * hk + kh) * (int64_t)dk, v + (t * hv + h) * (int64_t)dv, gate[t * hv + h],
                                 beta[t * hv + h], out + (t * hv + h) * (int64_t)dv, dk, dv, scratch);
        }
    }
    free(scratch);
}

/* ---- small pieces: src/recurrent.hpp:35-48, src/core.hpp:579 --------------- */

float nmo_softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
float nmo_sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

void nmo_l2_normalize(const float* x, float* y, int n, float eps) {
    float ss = 0.f;
    for (int i = 0; i < n; ++i) ss += x[i] * x[i];
    float norm = sqrtf(ss);
    const float scale = 1.f / (norm < eps ? eps : norm); /* std::max(norm, eps) */
    for (int i = 0; i < n; ++i) y[i] = x[i] * scale;
}

/* ---- the steps either side of the recurrence ----------------------------- */

/* CausalConv1dState<C,W>::step over T tokens (recurrent.hpp:76-104).  hist
 * [W-1][C] holds the carried inputs, oldest first, and is advanced in place;
 * per channel the current sample's tap comes first, then taps 0 .. W-2
 * (recurrent.hpp:80-83). */
void nmo_conv_run(const float* w, int C, int W, const float* x, int64_t T, float* hist, float* y) {
    const int H = W - 1;
    float* win = (float*)malloc(sizeof(float) * (size_t)(H > 0 ? H : 1));
    for (int c = 0; c < C; ++c) {
        for (int i = 0; i < H; ++i) win[i] = hist[(size_t)i * C + c];
        for (int64_t t = 0; t < T; ++t) {
            const float xin = x[(size_t)t * C + c];
            float sum = w[(size_t)c * W + H] * xin;
            for (int tap = 0; tap < H; ++tap) sum += w[(size_t)c * W + tap] * win[tap];
            y[(size_t)t * C + c] = sum;
            for (int i = 0; i + 1 < H; ++i) win[i] = win[i + 1];
            if (H > 0) win[H - 1] = xin;
        }
        for (int i = 0; i < H; ++i) hist[(size_t)i * C + c] = win[i];
    }
    free(win);
}

float nmo_silu(float x) { return x / (1.f + expf(-x)); } /* not x * sigmoid(x): components.hpp:104 */

/* The delta-net prologue of T tokens: conv + SiLU over the packed [q | k | v]
 * channels, q and k L2-normalised per key head (q then scaled by 1/sqrt(dk),
 * qwen35.hpp:427, :443-445), beta = sigmoid, gate = decay_scale * softplus(a +
 * dt_bias) (qwen35.hpp:400-415). */
void nmo_delta_prologue(const float* w, int W, int hk, int hv, int dk, int dv, int64_t T, const float* qkv, float* hist,
                        const float* beta_raw, const float* alpha_raw, const float* dt_bias, const float* decay_scale,
                        float* q, float* k, float* v, float* beta, float* gate) {
    const int C = 2 * hk * dk + hv * dv;
    float* y = (float*)malloc(sizeof(float) * (size_t)T * C);
    nmo_conv_run(w, C, W, qkv, T, hist, y);
    const float q_scale = 1.f / sqrtf((float)dk);
    for (int64_t t = 0; t < T; ++t) {
        float* row = y + (size_t)t * C;
        for (int c = 0; c < C; ++c) row[c] = nmo_silu(row[c]);
        for (int h = 0; h < hk; ++h) {
            float* qo = q + ((size_t)t * hk + h) * dk;
            float* ko = k + ((size_t)t * hk + h) * dk;
            nmo_l2_normalize(row + (size_t)h * dk, qo, dk, 1e-6f);
            for (int i = 0; i < dk; ++i) qo[i] *= q_scale;
            nmo_l2_normalize(row + (size_t)hk * dk + (size_t)h * dk, ko, dk, 1e-6f);
        }
        memcpy(v + (size_t)t * hv * dv, row + (size_t)2 * hk * dk, sizeof(float) * (size_t)hv * dv);
        for (int h = 0; h < hv; ++h) {
            const size_t i = (size_t)t * hv + h;
            beta[i] = nmo_sigmoid(beta_raw[i]);
            gate[i] = decay_scale[h] * nmo_softplus(alpha_raw[i] + dt_bias[h]);
        }
    }
    free(y);
}

/* out = RMSNorm(o; gamma, eps) per head, times SiLU(z) (qwen35.hpp:458-460):
 * inverse_rms = 1 / sqrt(dot(o, o) / dv + eps), out = gamma * o * inverse_rms
 * * silu(z) (components.hpp:174-176). */
void nmo_delta_epilogue(int64_t rows, int dv, const float* o, const float* z, const float* gamma, float eps, float* out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* x = o + (size_t)r * dv;
        float ss = 0.f;
        for (int i = 0; i < dv; ++i) ss += x[i] * x[i];
        const float inv = 1.f / sqrtf(ss / (float)dv + eps);
        for (int i = 0; i < dv; ++i) out[(size_t)r * dv + i] = gamma[i] * x[i] * inv * nmo_silu(z[(size_t)r * dv + i]);
    }
}

/* ---- the steps either side of the attention reduction ------------------- */

/* RotaryEmbedding<dh, base, num, den>'s table (attention.hpp:76-80): planes
 * below num*dh/den/2 get float(base^(-2i/dh)) computed in double, the rest 0. */
void nmo_rope_freqs(int dh, double base, int num, int den, float* inv_freq) {
    const int rotary = (int)((int64_t)num * dh / den / 2);
    for (int i = 0; i < dh / 2; ++i) inv_freq[i] = i < rotary ? (float)pow(base, -(double)(2 * i) / (double)dh) : 0.f;
}

/* One head rotated at `position` (attention.hpp:82-92): plane i couples
 * (i, i + dh/2); the angle is float(position) * inv_freq_i. */
void nmo_rope(float* x, int dh, const float* inv_freq, int64_t position) {
    const int planes = dh / 2;
    for (int i = 0; i < planes; ++i) {
        const float angle = (float)position * inv_freq[i];
        const float c = cosf(angle), s = sinf(angle);
        const float a = x[i], b = x[i + planes];
        x[i] = a * c - b * s;
        x[i + planes] = b * c + a * s;
    }
}

/* RMSNorm<n> (components.hpp:174-176) of one row, or RMSNormNoScale<n>
 * (:212-213) when gamma is NULL. */
void nmo_rmsnorm(int n, const float* gamma, float eps, const float* x, float* y) {
    float ss = 0.f;
    for (int i = 0; i < n; ++i) ss += x[i] * x[i];
    const float inv = 1.f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; ++i) y[i] = gamma ? gamma[i] * x[i] * inv : x[i] * inv;
}

/* Q, K and V of an attention layer for T tokens at position.. (qwen35.hpp:343-352,
 * gemma4.hpp:206-209, :676-680): q_out = rope(rmsnorm(q head; q_gamma)) with q
 * the head-major [q | gate] pairs when q_gated, k_out = rope(rmsnorm(k head;
 * k_gamma)), v_out = rmsnorm_no_scale(v head) when v_norm, else v. */
void nmo_attn_prologue(int64_t T, int hq, int hkv, int dh, int64_t position, const float* q, int q_gated, const float* k,
                       const float* v, const float* q_gamma, const float* k_gamma, int v_norm, float eps, double base,
                       int num, int den, float* q_out, float* k_out, float* v_out) {
    float* freqs = (float*)malloc(sizeof(float) * (size_t)(dh / 2));
    nmo_rope_freqs(dh, base, num, den, freqs);
    const int qstride = (q_gated ? 2 : 1) * dh;
    for (int64_t t = 0; t < T; ++t) {
        for (int h = 0; h < hq; ++h) {
            float* y = q_out + ((size_t)t * hq + h) * dh;
            nmo_rmsnorm(dh, q_gamma, eps, q + ((size_t)t * hq + h) * qstride, y);
            nmo_rope(y, dh, freqs, position + t);
        }
        for (int h = 0; h < hkv; ++h) {
            const size_t o = ((size_t)t * hkv + h) * dh;
            nmo_rmsnorm(dh, k_gamma, eps, k + o, k_out + o);
            nmo_rope(k_out + o, dh, freqs, position + t);
            if (v_norm)
                nmo_rmsnorm(dh, NULL, eps, v + o, v_out + o);
            else
                memcpy(v_out + o, v + o, sizeof(float) * (size_t)dh);
        }
    }
    free(freqs);
}

/* a *= sigmoid(gate) (qwen35.hpp:390-393), the gate of row r = t*hq + h being
 * the second half of qg's head pair r. */
void nmo_attn_gate(int64_t T, int hq, int dh, const float* qg, float* a) {
    for (int64_t r = 0; r < T * hq; ++r)
        for (int i = 0; i < dh; ++i) a[(size_t)r * dh + i] *= nmo_sigmoid(qg[((size_t)2 * r + 1) * dh + i]);
}

/* quantize_row_q8_0 (src/quant_i8.hpp:69-81) over n values, n a multiple of 32:
 * per block amax = max |x|, d = amax / 127, id = d ? 1 / d : 0, the scale kept
 * as fp16 (core.hpp:61-79 rounding), q = roundf(x * id) as int8. */
void nmo_quantize_q8_0(const float* x, int64_t n, int8_t* qs, uint16_t* dbits) {
    for (int64_t b = 0; b < n / 32; ++b) {
        float amax = 0.f;
        for (int j = 0; j < 32; ++j) {
            const float ax = fabsf(x[b * 32 + j]);
            amax = amax < ax ? ax : amax; /* std::max(amax, ax) */
        }
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.f / d : 0.f;
        dbits[b] = nmo_fp32_to_fp16(d);
        for (int j = 0; j < 32; ++j) qs[b * 32 + j] = (int8_t)roundf(x[b * 32 + j] * id);
    }
}
