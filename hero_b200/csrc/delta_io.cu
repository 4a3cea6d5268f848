// delta_io.cu -- the steps either side of the gated delta rule in a Qwen 3.5
// recurrent layer, on the device (HBM-bound elementwise kernels).
//
// Prologue, per token t (nm/src/qwen35.hpp:420-446, :396-415):
//   stream = SiLU(conv1d(qkv_t))        depthwise causal conv of width W over
//                                        the packed [q | k | v] channels, its
//                                        last W - 1 inputs carried between calls
//                                        (CausalConv1dState, recurrent.hpp:63-110)
//   q_hk = l2_normalize(stream[q slice hk]) / sqrt(Dk),  k_hk = l2_normalize(...)
//                                        (recurrent.hpp:40-48, eps 1e-6)
//   v_h  = stream[v slice h]
//   beta_h = sigmoid(b_t,h)              (core.hpp:579)
//   gate_h = decay_scale_h * softplus(a_t,h + dt_bias_h)   (recurrent.hpp:35)
// Epilogue (qwen35.hpp:458-461): out = RMSNorm_per_head(o; gamma, eps) (.) SiLU(z)
// (components.hpp:102-105, :167-180, :248-281).
//
// One CTA takes one head slice of the packed channels (Dk or Dv threads, one
// channel each) over 16 consecutive tokens: each thread walks its channel in
// time with the conv window in registers, so every input value is read once,
// and the per-token L2 norm of a q or k head is one block reduction.
#include <math.h>

#include "common.cuh"
#include "delta.cuh"

struct nmg_conv_state {
    int channels = 0, width = 0, device = 0;
    float* hist = nullptr;  // [width - 1][channels] fp32, the oldest input row first; zero = causal pad
};

namespace nmg {
namespace {

constexpr int kMaxWidth = 8;   // conv taps a thread keeps in registers
constexpr int kTokens = 8;     // tokens per CTA (16 measured slower: 149 against 138 us at config 3)

__device__ __forceinline__ float silu_ref(float x) { return x / (1.f + expf(-x)); }  // components.hpp:104
// The same with the hardware exponential and division (a few ulp apart): the
// prologue's SiLU over every conv output, where the accurate pair made the
// kernel instruction-bound.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_ref(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float softplus_ref(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// The window of channel c just before token t0: inputs t0 - (W-1) .. t0 - 1,
// from x where t >= 0 and from the carried history before the first token.
template <int W>
__device__ __forceinline__ void load_window(const float* x, const float* hist, int64_t C, int64_t c, int64_t t0,
                                            float (&h)[kMaxWidth]) {
#pragma unroll
    for (int i = 0; i < W - 1; ++i) {
        const int64_t t = t0 - (W - 1) + i;
        h[i] = t >= 0 ? x[t * C + c] : hist[(W - 1 + t) * C + c];
    }
}

// One conv output: taps[W-1] * current sample first, then taps 0 (oldest) ..
// W-2, the reference's order (recurrent.hpp:80-83); the window then shifts.
template <int W>
__device__ __forceinline__ float conv_step(const float (&w)[kMaxWidth], float (&h)[kMaxWidth], float xin) {
    float sum = w[W - 1] * xin;
#pragma unroll
    for (int i = 0; i < W - 1; ++i) sum = fmaf(w[i], h[i], sum);
#pragma unroll
    for (int i = 0; i + 1 < W - 1; ++i) h[i] = h[i + 1];
    if constexpr (W > 1) h[W - 2] = xin;
    return sum;
}

struct ConvArgs {
    const float* x;        // [T][C]
    const float* weights;  // [C][W]
    const float* hist;     // [W - 1][C]
    float* y;              // [T][C]
    int64_t T, C;
    int silu;
};

template <int W>
__global__ void __launch_bounds__(128) conv_kernel(const ConvArgs a) {
    const int64_t c = (int64_t)blockIdx.x * 128 + threadIdx.x;
    if (c >= a.C) return;
    const int64_t t0 = (int64_t)blockIdx.y * kTokens;
    float w[kMaxWidth], h[kMaxWidth];
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = a.weights[c * W + i];
    load_window<W>(a.x, a.hist, a.C, c, t0, h);
    for (int tt = 0; tt < kTokens && t0 + tt < a.T; ++tt) {
        const int64_t t = t0 + tt;
        const float s = conv_step<W>(w, h, a.x[t * a.C + c]);
        a.y[t * a.C + c] = a.silu ? silu_ref(s) : s;
    }
}

// The carried history after T inputs: the last W - 1 of [history | x].  One
// thread per channel reads its old column before writing it.
template <int W>
__global__ void __launch_bounds__(128) conv_history_kernel(const float* x, float* hist, int64_t T, int64_t C) {
    const int64_t c = (int64_t)blockIdx.x * 128 + threadIdx.x;
    if (c >= C || W < 2) return;
    float old[kMaxWidth];
#pragma unroll
    for (int i = 0; i < W - 1; ++i) old[i] = hist[i * C + c];
#pragma unroll
    for (int r = 0; r < W - 1; ++r) {
        const int64_t idx = T + r;  // position in [history (W-1) | x (T)]
        hist[r * C + c] = idx < W - 1 ? old[idx] : x[(idx - (W - 1)) * C + c];
    }
}

struct PrologueArgs {
    const float* qkv;      // [T][C], C = 2 Hk Dk + Hv Dv, packed [q | k | v]
    const float* weights;  // [C][W]
    const float* hist;     // [W - 1][C]
    const float* beta_raw, *alpha_raw, *dt_bias, *decay_scale;
    float *q, *k, *v, *beta, *gate;
    int64_t T, C;
    int hk, hv, dk, dv;
    float q_scale;
};

template <int W>
__global__ void __launch_bounds__(1024) prologue_kernel(const PrologueArgs a) {
    __shared__ float red[32][kTokens];
    const int slice = blockIdx.x;  // q slices 0..Hk-1, k slices Hk..2Hk-1, v slices 2Hk..
    const int kind = slice < a.hk ? 0 : (slice < 2 * a.hk ? 1 : 2);
    const int width = kind == 2 ? a.dv : a.dk;
    const int64_t c0 = kind == 0 ? (int64_t)slice * a.dk
                     : kind == 1 ? (int64_t)a.hk * a.dk + (int64_t)(slice - a.hk) * a.dk
                                 : 2ll * a.hk * a.dk + (int64_t)(slice - 2 * a.hk) * a.dv;
    const int j = threadIdx.x, lane = j & 31, wid = j >> 5;
    const bool on = j < width;
    const int64_t c = c0 + (on ? j : 0);
    const int64_t t0 = (int64_t)blockIdx.y * kTokens;
    const int nt = a.T - t0 < kTokens ? (int)(a.T - t0) : kTokens;  // uniform over the CTA
    float w[kMaxWidth], h[kMaxWidth], y[kTokens];
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = on ? a.weights[c * W + i] : 0.f;
    if (on) load_window<W>(a.qkv, a.hist, a.C, c, t0, h);
    // every token's input first (independent loads in flight), then the conv
    const float* xp = a.qkv + t0 * a.C + c;
#pragma unroll
    for (int tt = 0; tt < kTokens; ++tt, xp += a.C) y[tt] = (on && tt < nt) ? *xp : 0.f;
#pragma unroll
    for (int tt = 0; tt < kTokens; ++tt) {
        const float cv = conv_step<W>(w, h, y[tt]);
        y[tt] = on ? silu_fast(cv) : 0.f;
    }
    if (kind == 2) {
        float* vp = a.v + (t0 * a.hv + (slice - 2 * a.hk)) * (int64_t)a.dv + j;
        const int64_t vstep = (int64_t)a.hv * a.dv;
#pragma unroll
        for (int tt = 0; tt < kTokens; ++tt, vp += vstep)
            if (on && tt < nt) *vp = y[tt];
        if (j < nt) {  // this value head's write strength and decay gate
            const int hh = slice - 2 * a.hk;
            const int64_t i = (t0 + j) * a.hv + hh;
            a.beta[i] = sigmoid_ref(a.beta_raw[i]);
            a.gate[i] = a.decay_scale[hh] * softplus_ref(a.alpha_raw[i] + a.dt_bias[hh]);
        }
        return;
    }
    // Per-token L2 norms of this q or k head.  The warp's kTokens sums of
    // squares by a transposing butterfly: each xor step (16, 8, ...) halves
    // the tokens a lane carries until one is left, then plain steps finish
    // the sum, so lane l ends with the warp sum of token tok(l) after
    // (kTokens - 1) + (5 - log2 kTokens) shuffles instead of kTokens x 5.  One
    // thread per token then forms the scale (the IEEE square root and
    // division once per token, not once per element: 211 -> 138 us at
    // config 3).
    static_assert(kTokens >= 2 && kTokens <= 32 && (kTokens & (kTokens - 1)) == 0, "tokens per CTA: a power of 2");
    float s[kTokens];
#pragma unroll
    for (int tt = 0; tt < kTokens; ++tt) s[tt] = y[tt] * y[tt];
    int tok = 0;
#pragma unroll
    for (int step = 0; step < 5; ++step) {
        const int off = 16 >> step;
        const int cnt = kTokens >> (step + 1);  // tokens kept after this step; 0: a plain step
        if (cnt >= 1) {
            const bool hi = lane & off;
#pragma unroll
            for (int i = 0; i < kTokens / 2; ++i)
                if (i < cnt) {
                    const float keep = hi ? s[i + cnt] : s[i];
                    const float give = hi ? s[i] : s[i + cnt];
                    s[i] = keep + __shfl_xor_sync(0xffffffffu, give, off);
                }
            tok += hi ? cnt : 0;
        } else {
            s[0] += __shfl_xor_sync(0xffffffffu, s[0], off);
        }
    }
    if ((lane & (32 / kTokens - 1)) == 0) red[wid][tok] = s[0];
    __syncthreads();
    __shared__ float tscale[kTokens];
    if (j < kTokens) {
        const int nw = blockDim.x >> 5;
        float ss = 0.f;
        for (int i = 0; i < nw; ++i) ss += red[i][j];
        tscale[j] = 1.f / fmaxf(sqrtf(ss), 1e-6f);
    }
    __syncthreads();
    const int head = kind == 0 ? slice : slice - a.hk;
    float* dst = (kind == 0 ? a.q : a.k) + (t0 * a.hk + head) * (int64_t)a.dk + j;
    const int64_t dstep = (int64_t)a.hk * a.dk;
    const float post = kind == 0 ? a.q_scale : 1.f;  // q's 1/sqrt(Dk) after the norm (qwen35.hpp:445)
#pragma unroll
    for (int tt = 0; tt < kTokens; ++tt, dst += dstep) {
        const float scale = tscale[tt];
        if (on && tt < nt) *dst = kind == 0 ? (y[tt] * scale) * post : y[tt] * scale;
    }
}

// out[t][h][:] = ((gamma * o) * inv_rms(o[t][h])) * SiLU(z[t][h][:]), one warp per
// (t, h); each lane holds its PER values of the row (4 consecutive ones per
// 16-byte access when dv is a multiple of 128), so o is read once.
template <int PER>
__global__ void __launch_bounds__(256) epilogue_kernel(const float* o, const float* z, const float* gamma, float eps,
                                                        float* out, int64_t rows, int dv) {
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float* orow = o + r * dv;
    const float* zrow = z + r * dv;
    float* orow_out = out + r * dv;
    float x[PER], zz[PER];
    float ss = 0.f;
    if constexpr (PER % 4 == 0) {
#pragma unroll
        for (int q = 0; q < PER / 4; ++q) {
            const int jj = (q * 32 + lane) * 4;
            const float4 a4 = *(const float4*)(orow + jj), z4 = *(const float4*)(zrow + jj);
            x[4 * q] = a4.x, x[4 * q + 1] = a4.y, x[4 * q + 2] = a4.z, x[4 * q + 3] = a4.w;
            zz[4 * q] = z4.x, zz[4 * q + 1] = z4.y, zz[4 * q + 2] = z4.z, zz[4 * q + 3] = z4.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            const int jj = e * 32 + lane;
            x[e] = jj < dv ? orow[jj] : 0.f;
            zz[e] = jj < dv ? zrow[jj] : 0.f;
        }
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) ss = fmaf(x[e], x[e], ss);
    ss = dev::warp_sum(ss);
    const float inv = 1.f / sqrtf(ss / (float)dv + eps);
    if constexpr (PER % 4 == 0) {
#pragma unroll
        for (int q = 0; q < PER / 4; ++q) {
            const int jj = (q * 32 + lane) * 4;
            const float4 g4 = *(const float4*)(gamma + jj);
            const float g[4] = {g4.x, g4.y, g4.z, g4.w};
            float r4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) r4[e] = ((g[e] * x[4 * q + e]) * inv) * silu_ref(zz[4 * q + e]);
            *(float4*)(orow_out + jj) = make_float4(r4[0], r4[1], r4[2], r4[3]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            const int jj = e * 32 + lane;
            if (jj < dv) orow_out[jj] = ((gamma[jj] * x[e]) * inv) * silu_ref(zz[e]);
        }
    }
}

#define NMG_CONV_WIDTHS(W, CALL) \
    switch (W) {                 \
        case 1: CALL(1); break;  \
        case 2: CALL(2); break;  \
        case 3: CALL(3); break;  \
        case 4: CALL(4); break;  \
        case 5: CALL(5); break;  \
        case 6: CALL(6); break;  \
        case 7: CALL(7); break;  \
        case 8: CALL(8); break;  \
    }

// ---- one decode token of a whole layer core in one launch -----------------
// The prologue (conv + SiLU + L2 norms + gates), the recurrent step and the
// gated output norm of qwen35.hpp:396-461 at T = 1.  One thread-block
// cluster per key head kh: its CTAs are the (value head h = kh + r * Hk,
// 32-column block) pairs that read that key head, so
//   * every CTA forms q and k of kh itself (256 conv channels: cheap) and its
//     own 32 v channels, from the conv history;
//   * a cluster barrier orders every CTA's history reads before the history
//     is advanced (q and k channels by ranks 0 and 1, v channels by their CTA);
//   * the step runs as delta_step_kernel's (4 warps x 8 columns, 4 row groups
//     of 32 key rows per column);
//   * the per-head sum of squares of o meets across the head's CTAs through
//     distributed shared memory (plain remote stores), then each CTA writes
//     its 32 gated outputs.
// Numerics follow the three separate kernels: the prologue's hardware-exp
// SiLU and per-head norm, the step's __expf decay, the epilogue's IEEE SiLU.
struct DecodeArgs {
    float* state;             // [hv][128][dv]
    float* hist;              // [W - 1][C]
    const float* weights;     // [C][W]
    const float* qkv;         // [C]
    const float* beta_raw, *alpha_raw, *dt_bias, *decay_scale;  // [hv]
    const float* z;           // [hv][dv]
    const float* gamma;       // [dv]
    float* out;               // [hv][dv]
    int hk, hv, dv, cb;       // cb: 32-column blocks per value head
    int64_t C;
    float q_scale, eps;
};

__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int W>
__global__ void __launch_bounds__(128) delta_decode_kernel(const __grid_constant__ DecodeArgs a) {
    constexpr int DK = 128, RPT = DK / 4;
    __shared__ float qs[DK], ks[DK], vs[32], red[2][4], part[8];
    __shared__ float gb[2];  // decay, beta
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    uint32_t rank, ncl;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(ncl));
    const int kh = blockIdx.x / ncl;
    const int hr = rank / a.cb, cb = rank % a.cb;
    const int h = kh + hr * a.hk;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;

    // prologue: q and k of key head kh (channel t of each), v channel t < 32
    const int64_t cq = (int64_t)kh * DK + t, ck = (int64_t)a.hk * DK + kh * DK + t;
    const int64_t cvc = 2ll * a.hk * DK + (int64_t)h * a.dv + cb * 32 + t;
    float hq[kMaxWidth], hk_[kMaxWidth], hv_[kMaxWidth], wq[kMaxWidth], wk[kMaxWidth], wv[kMaxWidth];
#pragma unroll
    for (int i = 0; i < W; ++i) {
        wq[i] = a.weights[cq * W + i];
        wk[i] = a.weights[ck * W + i];
        wv[i] = t < 32 ? a.weights[cvc * W + i] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < W - 1; ++i) {
        hq[i] = a.hist[i * a.C + cq];
        hk_[i] = a.hist[i * a.C + ck];
        hv_[i] = t < 32 ? a.hist[i * a.C + cvc] : 0.f;
    }
    const float xq = a.qkv[cq], xk = a.qkv[ck], xv = t < 32 ? a.qkv[cvc] : 0.f;
    float hq2[kMaxWidth], hk2[kMaxWidth], hv2[kMaxWidth];  // copies conv_step shifts; the originals are written back
#pragma unroll
    for (int i = 0; i < W - 1; ++i) hq2[i] = hq[i], hk2[i] = hk_[i], hv2[i] = hv_[i];
    const float yq = silu_fast(conv_step<W>(wq, hq2, xq));
    const float yk = silu_fast(conv_step<W>(wk, hk2, xk));
    if (t < 32) vs[t] = silu_fast(conv_step<W>(wv, hv2, xv));
    if (t == 0) {
        gb[0] = __expf(a.decay_scale[h] * softplus_ref(a.alpha_raw[h] + a.dt_bias[h]));
        gb[1] = sigmoid_ref(a.beta_raw[h]);
    }
    const float sq = dev::warp_sum(yq * yq), sk = dev::warp_sum(yk * yk);
    if (lane == 0) red[0][w] = sq, red[1][w] = sk;
    __syncthreads();
    const float nq = 1.f / fmaxf(sqrtf(red[0][0] + red[0][1] + red[0][2] + red[0][3]), 1e-6f);
    const float nk = 1.f / fmaxf(sqrtf(red[1][0] + red[1][1] + red[1][2] + red[1][3]), 1e-6f);
    qs[t] = (yq * nq) * a.q_scale;
    ks[t] = yk * nk;

    // every CTA of the cluster has read the history: advance it
    cl_sync();
    if (W > 1) {
        auto put = [&](int64_t c, const float* old, float x) {
#pragma unroll
            for (int i = 0; i + 1 < W - 1; ++i) a.hist[i * a.C + c] = old[i + 1];
            a.hist[(int64_t)(W - 2) * a.C + c] = x;
        };
        if (t < 32) put(cvc, hv_, xv);
        if (rank == 0) put(cq, hq, xq);
        if (rank == (ncl > 1 ? 1u : 0u)) put(ck, hk_, xk);
    }
    __syncthreads();

    // the recurrent step over this CTA's 32 columns
    const int cg = lane & 7, rg = lane >> 3;
    const int jl = w * 8 + cg, j = cb * 32 + jl;
    const int i0 = rg * RPT;
    float* S = a.state + ((int64_t)h * DK + i0) * a.dv + j;
    const float decay = gb[0], b = gb[1], vj = vs[jl];
    float s[RPT], part_s = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        s[r] = S[(int64_t)r * a.dv] * decay;
        part_s = fmaf(s[r], ks[i0 + r], part_s);
    }
    part_s += __shfl_xor_sync(0xffffffffu, part_s, 8);
    part_s += __shfl_xor_sync(0xffffffffu, part_s, 16);
    const float d = (vj - part_s) * b;
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        s[r] = fmaf(ks[i0 + r], d, s[r]);
        o = fmaf(s[r], qs[i0 + r], o);
        S[(int64_t)r * a.dv] = s[r];
    }
    o += __shfl_xor_sync(0xffffffffu, o, 8);
    o += __shfl_xor_sync(0xffffffffu, o, 16);

    // gated RMS norm over the head's dv columns, spread over a.cb CTAs
    float ss = rg == 0 ? o * o : 0.f;
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    __syncthreads();
    if (lane == 0) red[0][w] = ss;
    __syncthreads();
    if (t < a.cb) {  // push this CTA's partial to slot cb of every CTA of the head
        const float mine = red[0][0] + red[0][1] + red[0][2] + red[0][3];
        uint32_t dst;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                     : "=r"(dst)
                     : "r"(dev::smem_u32(&part[cb])), "r"((uint32_t)(hr * a.cb + t)));
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(mine) : "memory");
    }
    cl_sync();
    float tot = 0.f;
    for (int i = 0; i < a.cb; ++i) tot += part[i];
    const float inv = 1.f / sqrtf(tot / (float)a.dv + a.eps);
    if (rg == 0) {
        const int64_t oi = (int64_t)h * a.dv + j;
        a.out[oi] = ((a.gamma[j] * o) * inv) * silu_ref(a.z[oi]);
    }
}

int update_history(nmg_conv_state* s, const float* x, int64_t T, cudaStream_t stream) {
    if (s->width < 2) return NMG_OK;
    const dim3 grid((unsigned)((s->channels + 127) / 128));
#define NMG_HIST(WW) conv_history_kernel<WW><<<grid, 128, 0, stream>>>(x, s->hist, T, s->channels)
    NMG_CONV_WIDTHS(s->width, NMG_HIST)
#undef NMG_HIST
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace
}  // namespace nmg

using namespace nmg;

extern "C" int nmg_conv_create(int channels, int width, int device, nmg_conv_state** out) {
    if (!out) return set_error(NMG_INVALID_ARGUMENT, "nmg_conv_create: null out");
    *out = nullptr;
    if (channels <= 0 || width < 1) return set_error(NMG_INVALID_ARGUMENT, "CausalConv1dState: channels and width must be positive");
    if (width > kMaxWidth) return set_error(NMG_UNSUPPORTED, "CausalConv1dState: width %d is not built (at most %d)", width, kMaxWidth);
    nmg_conv_state* s = new nmg_conv_state();
    s->channels = channels;
    s->width = width;
    s->device = device;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    const size_t bytes = (size_t)(width > 1 ? width - 1 : 1) * channels * sizeof(float);
    if (e == cudaSuccess) e = cudaMalloc(&s->hist, bytes);
    if (e == cudaSuccess) e = cudaMemset(s->hist, 0, bytes);  // the causal zero pad (recurrent.hpp:70-73)
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (s->hist) cudaFree(s->hist);
        delete s;
        return set_error(NMG_CUDA_ERROR, "nmg_conv_create: %s", cudaGetErrorString(e));
    }
    *out = s;
    return NMG_OK;
}

extern "C" int nmg_conv_destroy(nmg_conv_state* s) {
    if (!s) return NMG_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaFree(s->hist);
    cudaSetDevice(prev);
    delete s;
    return NMG_OK;
}

extern "C" int nmg_conv_clear(nmg_conv_state* s, void* stream) {
    if (!s) return set_error(NMG_INVALID_ARGUMENT, "nmg_conv_clear: null state");
    const size_t bytes = (size_t)(s->width > 1 ? s->width - 1 : 1) * s->channels * sizeof(float);
    NMG_CUDA_TRY(cudaMemsetAsync(s->hist, 0, bytes, (cudaStream_t)stream));
    return NMG_OK;
}

extern "C" int nmg_conv_history(const nmg_conv_state* s, float** hist) {
    if (!s || !hist) return set_error(NMG_INVALID_ARGUMENT, "nmg_conv_history: null argument");
    *hist = s->hist;
    return NMG_OK;
}

extern "C" int nmg_conv_step(nmg_conv_state* s, const float* weights, const float* x, int64_t T, float* y, int silu,
                             void* stream) {
    if (!s) return set_error(NMG_INVALID_ARGUMENT, "nmg_conv_step: null state");
    if (T < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_conv_step: negative token count");
    if (T == 0) return NMG_OK;
    if (!weights || !x || !y) return set_error(NMG_INVALID_ARGUMENT, "nmg_conv_step: null argument");
    if (T > 65535ll * kTokens) return set_error(NMG_LENGTH_ERROR, "nmg_conv_step: too many tokens for one call");
    const cudaStream_t st = (cudaStream_t)stream;
    ConvArgs a{x, weights, s->hist, y, T, s->channels, silu ? 1 : 0};
    const dim3 grid((unsigned)((s->channels + 127) / 128), (unsigned)((T + kTokens - 1) / kTokens));
#define NMG_CONV(WW) conv_kernel<WW><<<grid, 128, 0, st>>>(a)
    NMG_CONV_WIDTHS(s->width, NMG_CONV)
#undef NMG_CONV
    NMG_CUDA_TRY(cudaGetLastError());
    return update_history(s, x, T, st);
}

extern "C" int nmg_delta_prologue(nmg_conv_state* s, const float* weights, int hk, int hv, int dk, int dv, int64_t T,
                                  const float* qkv, const float* beta_raw, const float* alpha_raw, const float* dt_bias,
                                  const float* decay_scale, float* q, float* k, float* v, float* beta, float* gate,
                                  void* stream) {
    if (!s) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prologue: null conv state");
    if (hk <= 0 || hv <= 0 || dk <= 0 || dv <= 0 || hv % hk != 0)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prologue: heads and dims must be positive, Hv a multiple of Hk");
    if ((int64_t)2 * hk * dk + (int64_t)hv * dv != s->channels)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prologue: conv state has %d channels, 2*Hk*Dk + Hv*Dv = %lld",
                         s->channels, (long long)(2ll * hk * dk + (int64_t)hv * dv));
    if (dk % 32 || dv % 32 || dk > 1024 || dv > 1024)
        return set_error(NMG_UNSUPPORTED, "nmg_delta_prologue: Dk and Dv must be multiples of 32 up to 1024");
    if (T < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prologue: negative token count");
    if (T == 0) return NMG_OK;
    if (!weights || !qkv || !beta_raw || !alpha_raw || !dt_bias || !decay_scale || !q || !k || !v || !beta || !gate)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prologue: null argument");
    if (T > 65535ll * kTokens) return set_error(NMG_LENGTH_ERROR, "nmg_delta_prologue: too many tokens for one call");
    const cudaStream_t st = (cudaStream_t)stream;
    PrologueArgs a;
    a.qkv = qkv;
    a.weights = weights;
    a.hist = s->hist;
    a.beta_raw = beta_raw;
    a.alpha_raw = alpha_raw;
    a.dt_bias = dt_bias;
    a.decay_scale = decay_scale;
    a.q = q;
    a.k = k;
    a.v = v;
    a.beta = beta;
    a.gate = gate;
    a.T = T;
    a.C = s->channels;
    a.hk = hk;
    a.hv = hv;
    a.dk = dk;
    a.dv = dv;
    a.q_scale = 1.f / sqrtf((float)dk);  // qwen35.hpp:427
    const dim3 grid((unsigned)(2 * hk + hv), (unsigned)((T + kTokens - 1) / kTokens));
    const int threads = dk > dv ? dk : dv;
#define NMG_PRO(WW) prologue_kernel<WW><<<grid, threads, 0, st>>>(a)
    NMG_CONV_WIDTHS(s->width, NMG_PRO)
#undef NMG_PRO
    NMG_CUDA_TRY(cudaGetLastError());
    return update_history(s, qkv, T, st);
}

extern "C" int nmg_delta_epilogue(int hv, int dv, int64_t T, const float* o, const float* z, const float* gamma,
                                  float eps, float* out, void* stream) {
    if (hv <= 0 || dv <= 0 || T < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_epilogue: bad dimensions");
    if (T == 0) return NMG_OK;
    if (!o || !z || !gamma || !out) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_epilogue: null argument");
    const int64_t rows = T * hv;
    if ((rows + 7) / 8 > 0x7FFFFFFFll) return set_error(NMG_LENGTH_ERROR, "nmg_delta_epilogue: too many rows");
    if (dv > 1024) return set_error(NMG_UNSUPPORTED, "nmg_delta_epilogue: Dv up to 1024");
    const dim3 grid((unsigned)((rows + 7) / 8));
    const cudaStream_t st = (cudaStream_t)stream;
    const bool vec = dv % 128 == 0 && !(((uintptr_t)o | (uintptr_t)z | (uintptr_t)gamma | (uintptr_t)out) & 15);
    if (vec && dv == 128)
        epilogue_kernel<4><<<grid, 256, 0, st>>>(o, z, gamma, eps, out, rows, dv);
    else if (vec && dv == 256)
        epilogue_kernel<8><<<grid, 256, 0, st>>>(o, z, gamma, eps, out, rows, dv);
    else if (dv <= 128)
        epilogue_kernel<5><<<grid, 256, 0, st>>>(o, z, gamma, eps, out, rows, dv);  // PER not a multiple of 4: scalar path
    else
        epilogue_kernel<33><<<grid, 256, 0, st>>>(o, z, gamma, eps, out, rows, dv);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

extern "C" int nmg_delta_decode_token(nmg_delta_state* st, nmg_conv_state* conv, const float* weights, int hk,
                                      const float* qkv, const float* beta_raw, const float* alpha_raw,
                                      const float* dt_bias, const float* decay_scale, const float* z,
                                      const float* gamma, float eps, float* out, void* stream) {
    if (!st || !conv) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_decode_token: null state");
    const int hv = st->heads, dk = st->dk, dv = st->dv;
    if (hk <= 0 || hv % hk != 0)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_decode_token: Hv = %d is not a multiple of Hk = %d", hv, hk);
    if ((int64_t)2 * hk * dk + (int64_t)hv * dv != conv->channels)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_decode_token: conv state has %d channels, 2*Hk*Dk + Hv*Dv = %lld",
                         conv->channels, (long long)(2ll * hk * dk + (int64_t)hv * dv));
    if (!weights || !qkv || !beta_raw || !alpha_raw || !dt_bias || !decay_scale || !z || !gamma || !out)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_decode_token: null argument");
    if (conv->device != st->device) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_decode_token: states on two devices");
    const int ratio = hv / hk, cbs = dv / 32;
    if (dk != 128 || dv % 32 != 0 || ratio * cbs > 8)
        return set_error(NMG_UNSUPPORTED,
                         "nmg_delta_decode_token: built for Dk = 128 and (Hv/Hk) x (Dv/32) <= 8 (Dk %d, Dv %d, Hv/Hk %d)", dk,
                         dv, ratio);
    DecodeArgs a;
    a.state = st->data;
    a.hist = conv->hist;
    a.weights = weights;
    a.qkv = qkv;
    a.beta_raw = beta_raw;
    a.alpha_raw = alpha_raw;
    a.dt_bias = dt_bias;
    a.decay_scale = decay_scale;
    a.z = z;
    a.gamma = gamma;
    a.out = out;
    a.hk = hk;
    a.hv = hv;
    a.dv = dv;
    a.cb = cbs;
    a.C = conv->channels;
    a.q_scale = 1.f / sqrtf((float)dk);  // qwen35.hpp:427
    a.eps = eps;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != st->device) NMG_CUDA_TRY(cudaSetDevice(st->device));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(hk * ratio * cbs), 1, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)(ratio * cbs);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaErrorInvalidValue;
#define NMG_DEC(WW) e = cudaLaunchKernelEx(&cfg, delta_decode_kernel<WW>, a)
    NMG_CONV_WIDTHS(conv->width, NMG_DEC)
#undef NMG_DEC
    if (prev != st->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(NMG_CUDA_ERROR, "nmg_delta_decode_token: %s", cudaGetErrorString(e));
    return NMG_OK;
}
