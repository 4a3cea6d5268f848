// delta.cu -- gated delta-rule state, the per-token recurrent step (K6) and
// the token-sequential prefill; the chunked WY-form prefill (K5) is in
// delta_chunked.cu.
//
// Reference: nm/src/recurrent.hpp:117-177 (DeltaNetState, gated_delta_step)
// and the head loop of nm/src/qwen35.hpp:436-456 (value head h reads key head
// h % Hk, qwen35.hpp:172).  Per head and token, with S in R^{Dk x Dv}:
//     S *= exp(g);  pred = S^T k;  d = (v - pred) * beta;  S += k d^T;  o = S^T q
// Columns of S evolve independently (column j only needs v_j and column j of
// S), which is how both kernels split a head across threads and CTAs.
#include <math.h>

#include <algorithm>

#include "delta.cuh"

namespace nmg {
namespace {

// ---- one token, every head ---------------------------------------------------
// grid (heads, ceil(dv/32)); 4 warps, each owning 8 value columns.  Lane =
// (column cg = lane & 7) x (row group rg = lane >> 3): a thread holds rows
// [rg * RPT, (rg + 1) * RPT) of one state column in registers, so both
// reductions over the Dk rows are two xor-shuffles (no shared memory, no
// block barrier).  Launched with programmatic stream serialisation: the wait
// below lets the launch overlap the previous kernel's tail, and no input is
// read before it (the previous kernel may be the one producing q, k, v).
template <int DK>
__global__ void __launch_bounds__(128) delta_step_kernel(float* __restrict__ state, int dv, int hk,
                                                         const float* __restrict__ q, const float* __restrict__ k,
                                                         const float* __restrict__ v, const float* __restrict__ gate,
                                                         const float* __restrict__ beta, float* __restrict__ out,
                                                         int64_t head_stride_q) {
    constexpr int RPT = (DK + 3) / 4;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int h = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int cg = lane & 7, rg = lane >> 3;
    const int j = blockIdx.y * 32 + w * 8 + cg;
    const bool cv = j < dv;
    const int kh = h % hk;
    const int i0 = rg * RPT;
    const float* kk = k + kh * head_stride_q + i0;
    const float* qq = q + kh * head_stride_q + i0;
    float* S = state + ((int64_t)h * DK + i0) * dv + j;
    const float decay = __expf(gate[h]);
    const float b = beta[h];
    const float vj = cv ? v[(int64_t)h * dv + j] : 0.f;

    float kr[RPT], qr[RPT], s[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const bool in = i0 + r < DK;
        kr[r] = in ? __ldg(kk + r) : 0.f;
        qr[r] = in ? __ldg(qq + r) : 0.f;
        s[r] = (in && cv) ? S[(int64_t)r * dv] : 0.f;
    }
    float part = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        s[r] *= decay;
        part = fmaf(s[r], kr[r], part);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 8);
    part += __shfl_xor_sync(0xffffffffu, part, 16);
    const float d = (vj - part) * b;
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        s[r] = fmaf(kr[r], d, s[r]);
        o = fmaf(s[r], qr[r], o);
        if (cv && i0 + r < DK) S[(int64_t)r * dv] = s[r];
    }
    o += __shfl_xor_sync(0xffffffffu, o, 8);
    o += __shfl_xor_sync(0xffffffffu, o, 16);
    if (rg == 0 && cv) out[(int64_t)h * dv + j] = o;
}

// ---- one token of many sequences ---------------------------------------------
// The decode step of a batch of sequences, each with its own state (one
// DeltaNetState per sequence, as the reference keeps one per PrefixState).
// grid (dv / 64, heads, sequences); 128 threads; CTA = 64 value columns of
// one head of one sequence.  Warp w owns columns 16w .. 16w + 15; lane =
// (4-column group cg = lane & 3) x (row group rg = lane >> 2, 16 key rows), so
// each thread streams 16 float4 of state (64 B runs per row, 8 rows per warp
// instruction) and both reductions over the 128 key rows are three
// xor-shuffles.  The state is read and written once: HBM-bound when the
// batch's states exceed L2.
constexpr int kMaxStepBatch = 128;  // sequences per launch carried in the parameter block

struct StepBatchArgs {
    float* state[kMaxStepBatch];  // [heads][128][dv] per sequence
    const float* q;               // [B][hk][128]
    const float* k;
    const float* v;               // [B][heads][dv]
    const float* gate;            // [B][heads]
    const float* beta;
    float* out;                   // [B][heads][dv]
    int heads, hk, dv, seq0;      // seq0: this launch's first sequence within the batch
};

__global__ void __launch_bounds__(128) delta_step_batch_kernel(const __grid_constant__ StepBatchArgs a) {
    constexpr int DK = 128, RPT = 16;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ float ks[DK], qs[DK];
    const int h = blockIdx.y, bl = blockIdx.z, b = a.seq0 + bl;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int cg = lane & 3, rg = lane >> 2;
    const int j0 = blockIdx.x * 64 + w * 16 + cg * 4;  // first of this thread's 4 value columns
    const int kh = h % a.hk;
    const int64_t hb = (int64_t)b * a.heads + h;
    {
        const int64_t qk = ((int64_t)b * a.hk + kh) * DK + threadIdx.x;
        ks[threadIdx.x] = __ldg(a.k + qk);
        qs[threadIdx.x] = __ldg(a.q + qk);
    }
    float* S = a.state[bl] + ((int64_t)h * DK + rg * RPT) * a.dv + j0;
    float4 s[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) s[r] = __ldcs((const float4*)(S + (int64_t)r * a.dv));
    const float decay = __expf(__ldg(a.gate + hb));
    const float bt = __ldg(a.beta + hb);
    const float4 vj = __ldg((const float4*)(a.v + hb * a.dv + j0));
    __syncthreads();
    float4 part = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const float kr = ks[rg * RPT + r];
        s[r].x *= decay, s[r].y *= decay, s[r].z *= decay, s[r].w *= decay;
        part.x = fmaf(s[r].x, kr, part.x), part.y = fmaf(s[r].y, kr, part.y);
        part.z = fmaf(s[r].z, kr, part.z), part.w = fmaf(s[r].w, kr, part.w);
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        part.x += __shfl_xor_sync(0xffffffffu, part.x, o), part.y += __shfl_xor_sync(0xffffffffu, part.y, o);
        part.z += __shfl_xor_sync(0xffffffffu, part.z, o), part.w += __shfl_xor_sync(0xffffffffu, part.w, o);
    }
    const float4 d = make_float4((vj.x - part.x) * bt, (vj.y - part.y) * bt, (vj.z - part.z) * bt, (vj.w - part.w) * bt);
    float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const float kr = ks[rg * RPT + r], qr = qs[rg * RPT + r];
        s[r].x = fmaf(kr, d.x, s[r].x), s[r].y = fmaf(kr, d.y, s[r].y);
        s[r].z = fmaf(kr, d.z, s[r].z), s[r].w = fmaf(kr, d.w, s[r].w);
        o4.x = fmaf(s[r].x, qr, o4.x), o4.y = fmaf(s[r].y, qr, o4.y);
        o4.z = fmaf(s[r].z, qr, o4.z), o4.w = fmaf(s[r].w, qr, o4.w);
        __stcs((float4*)(S + (int64_t)r * a.dv), s[r]);
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        o4.x += __shfl_xor_sync(0xffffffffu, o4.x, o), o4.y += __shfl_xor_sync(0xffffffffu, o4.y, o);
        o4.z += __shfl_xor_sync(0xffffffffu, o4.z, o), o4.w += __shfl_xor_sync(0xffffffffu, o4.w, o);
    }
    if (rg == 0) *(float4*)(a.out + hb * a.dv + j0) = o4;
}

// Launch with programmatic stream serialisation (the kernel waits on its
// predecessor with griddepcontrol.wait before reading anything).
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---- T tokens, state held in registers ---------------------------------------
// grid (heads, ceil(dv/16)); 128 threads; warp w owns columns 4w..4w+3 of the
// CTA's 16, lane = (column-in-warp (4) x row group (8)); a row group holds
// DK/8 rows.  Row reductions are 3 xor-shuffles inside the 8-lane group.
template <int DK>
__global__ void __launch_bounds__(128) delta_seq_kernel(float* __restrict__ state, int dv, int hk, int heads, int64_t T,
                                                        const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, const float* __restrict__ gate,
                                                        const float* __restrict__ beta, float* __restrict__ out) {
    constexpr int RPG = (DK + 7) / 8;  // rows per group
    constexpr int TB = 8;              // tokens staged per refill
    __shared__ __align__(16) float ks[TB][DK];
    __shared__ __align__(16) float qs[TB][DK];
    const int h = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int grp = lane & 7;
    const int j = blockIdx.y * 16 + w * 4 + (lane >> 3);
    const bool cv = j < dv;
    const int kh = h % hk;
    float* S = state + (int64_t)h * DK * dv;

    float s[RPG];
#pragma unroll
    for (int r = 0; r < RPG; ++r) {
        const int i = grp * RPG + r;
        s[r] = (cv && i < DK) ? S[(int64_t)i * dv + j] : 0.f;
    }
    for (int64_t t0 = 0; t0 < T; t0 += TB) {
        const int nt = (int)(T - t0 < TB ? T - t0 : TB);
        __syncthreads();
        for (int x = threadIdx.x; x < nt * DK; x += 128) {
            const int tt = x / DK, i = x % DK;
            ks[tt][i] = k[((t0 + tt) * hk + kh) * (int64_t)DK + i];
            qs[tt][i] = q[((t0 + tt) * hk + kh) * (int64_t)DK + i];
        }
        __syncthreads();
        for (int tt = 0; tt < nt; ++tt) {
            const int64_t t = t0 + tt;
            const float decay = __expf(gate[t * heads + h]);
            const float b = beta[t * heads + h];
            const float vj = cv ? v[(t * heads + h) * (int64_t)dv + j] : 0.f;
            float part = 0.f;
#pragma unroll
            for (int r = 0; r < RPG; ++r) {
                const int i = grp * RPG + r;
                s[r] *= decay;
                if (i < DK) part = fmaf(s[r], ks[tt][i], part);
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            part += __shfl_xor_sync(0xffffffffu, part, 4);
            const float d = (vj - part) * b;
            float o = 0.f;
#pragma unroll
            for (int r = 0; r < RPG; ++r) {
                const int i = grp * RPG + r;
                if (i < DK) {
                    s[r] = fmaf(ks[tt][i], d, s[r]);
                    o = fmaf(s[r], qs[tt][i], o);
                }
            }
            o += __shfl_xor_sync(0xffffffffu, o, 1);
            o += __shfl_xor_sync(0xffffffffu, o, 2);
            o += __shfl_xor_sync(0xffffffffu, o, 4);
            if (cv && grp == 0) out[(t * heads + h) * (int64_t)dv + j] = o;
        }
    }
#pragma unroll
    for (int r = 0; r < RPG; ++r) {
        const int i = grp * RPG + r;
        if (cv && i < DK) S[(int64_t)i * dv + j] = s[r];
    }
}

#define NMG_DK_CASES(KERNEL, GRID, BLOCK, STREAM, ...)                                    \
    switch (dk) {                                                                         \
        case 2: KERNEL<2><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;               \
        case 4: KERNEL<4><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;               \
        case 8: KERNEL<8><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;               \
        case 16: KERNEL<16><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;             \
        case 32: KERNEL<32><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;             \
        case 64: KERNEL<64><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;             \
        case 128: KERNEL<128><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;           \
        case 256: KERNEL<256><<<GRID, BLOCK, 0, STREAM>>>(__VA_ARGS__); break;           \
        default: return set_error(NMG_UNSUPPORTED, "delta rule: Dk=%d is not built", dk); \
    }

#define NMG_DK_CASES_PDL(KERNEL, GRID, BLOCK, STREAM, ...)                                 \
    switch (dk) {                                                                           \
        case 2: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<2>, GRID, BLOCK, STREAM, __VA_ARGS__)); break;     \
        case 4: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<4>, GRID, BLOCK, STREAM, __VA_ARGS__)); break;     \
        case 8: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<8>, GRID, BLOCK, STREAM, __VA_ARGS__)); break;     \
        case 16: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<16>, GRID, BLOCK, STREAM, __VA_ARGS__)); break;   \
        case 32: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<32>, GRID, BLOCK, STREAM, __VA_ARGS__)); break;   \
        case 64: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<64>, GRID, BLOCK, STREAM, __VA_ARGS__)); break;   \
        case 128: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<128>, GRID, BLOCK, STREAM, __VA_ARGS__)); break; \
        case 256: NMG_CUDA_TRY(::nmg::launch_pdl(KERNEL<256>, GRID, BLOCK, STREAM, __VA_ARGS__)); break; \
        default: return set_error(NMG_UNSUPPORTED, "delta rule: Dk=%d is not built", dk);   \
    }

bool dk_supported(int dk) { return dk == 2 || dk == 4 || dk == 8 || dk == 16 || dk == 32 || dk == 64 || dk == 128 || dk == 256; }

}  // namespace

int delta_prefill_sequential(nmg_delta_state* st, int hk, int64_t T, const float* q, const float* k, const float* v,
                             const float* gate, const float* beta, float* out, cudaStream_t stream) {
    const int dk = st->dk;
    dim3 grid(st->heads, (st->dv + 15) / 16);
    NMG_DK_CASES(delta_seq_kernel, grid, 128, stream, st->data, st->dv, hk, st->heads, T, q, k, v, gate, beta, out)
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace nmg

using nmg::set_error;

extern "C" int nmg_delta_create(int heads, int dk, int dv, int device, nmg_delta_state** out) {
    if (!out) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_create: null out");
    *out = nullptr;
    if (heads <= 0 || dk <= 0 || dv <= 0) return set_error(NMG_INVALID_ARGUMENT, "DeltaNetState: dimensions must be positive");
    if (!nmg::dk_supported(dk)) return set_error(NMG_UNSUPPORTED, "DeltaNetState: Dk=%d is not built", dk);
    nmg_delta_state* s = new nmg_delta_state();
    s->heads = heads;
    s->dk = dk;
    s->dv = dv;
    s->device = device;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    const size_t bytes = (size_t)heads * dk * dv * sizeof(float);
    if (e == cudaSuccess) e = cudaMalloc(&s->data, bytes);
    if (e == cudaSuccess) e = cudaMemset(s->data, 0, bytes);  // DeltaNetState() zero-fills (recurrent.hpp:123)
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (s->data) cudaFree(s->data);
        delete s;
        return set_error(NMG_CUDA_ERROR, "nmg_delta_create: %s", cudaGetErrorString(e));
    }
    *out = s;
    return NMG_OK;
}

extern "C" int nmg_delta_destroy(nmg_delta_state* s) {
    if (!s) return NMG_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaFree(s->data);
    cudaSetDevice(prev);
    delete s;
    return NMG_OK;
}

extern "C" int nmg_delta_clear(nmg_delta_state* s, void* stream) {
    if (!s) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_clear: null state");
    NMG_CUDA_TRY(cudaMemsetAsync(s->data, 0, (size_t)s->heads * s->dk * s->dv * sizeof(float), (cudaStream_t)stream));
    return NMG_OK;
}

extern "C" int nmg_delta_head(nmg_delta_state* s, int head, float** ptr) {
    if (!s || !ptr) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_head: null argument");
    if (head < 0 || head >= s->heads) return set_error(NMG_OUT_OF_RANGE, "DeltaNetState: head out of range");
    *ptr = s->data + (size_t)head * s->dk * s->dv;
    return NMG_OK;
}

extern "C" int nmg_gated_delta_step(float* state_head, int dk, int dv, const float* q, const float* k, const float* v,
                                    const float* gate, const float* beta, float* out, void* stream) {
    if (!state_head || !q || !k || !v || !gate || !beta || !out)
        return set_error(NMG_INVALID_ARGUMENT, "gated_delta_step: null argument");
    if (dv <= 0 || !nmg::dk_supported(dk)) return set_error(NMG_UNSUPPORTED, "gated_delta_step: Dk=%d is not built", dk);
    dim3 grid(1, (dv + 31) / 32);
    cudaStream_t s = (cudaStream_t)stream;
    NMG_DK_CASES_PDL(nmg::delta_step_kernel, grid, dim3(128), s, state_head, dv, 1, q, k, v, gate, beta, out, (int64_t)dk)
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

extern "C" int nmg_delta_step(nmg_delta_state* st, int hk, const float* q, const float* k, const float* v,
                              const float* gate, const float* beta, float* out, void* stream) {
    if (!st) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step: null state");
    if (hk <= 0 || hk > st->heads) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step: bad key-head count %d", hk);
    const int dk = st->dk;
    dim3 grid(st->heads, (st->dv + 31) / 32);
    cudaStream_t s = (cudaStream_t)stream;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != st->device) NMG_CUDA_TRY(cudaSetDevice(st->device));
    NMG_DK_CASES_PDL(nmg::delta_step_kernel, grid, dim3(128), s, st->data, st->dv, hk, q, k, v, gate, beta, out, (int64_t)dk)
    NMG_CUDA_TRY(cudaGetLastError());
    if (prev != st->device) NMG_CUDA_TRY(cudaSetDevice(prev));
    return NMG_OK;
}

extern "C" int nmg_delta_prefill(nmg_delta_state* st, int hk, int64_t T, const float* q, const float* k, const float* v,
                                 const float* gate, const float* beta, float* out, int chunk, void* stream) {
    if (!st) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prefill: null state");
    if (hk <= 0 || hk > st->heads) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prefill: bad key-head count %d", hk);
    if (T < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prefill: negative length");
    if (T == 0) return NMG_OK;
    if (chunk != 0 && chunk != 64) return set_error(NMG_UNSUPPORTED, "nmg_delta_prefill: chunk must be 0 or 64");
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != st->device) NMG_CUDA_TRY(cudaSetDevice(st->device));
    int r;
    const bool aligned = !(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15);
    if (chunk == 0 || !aligned || !nmg::delta_chunked_supported(st))
        r = nmg::delta_prefill_sequential(st, hk, T, q, k, v, gate, beta, out, (cudaStream_t)stream);
    else
        r = nmg::delta_prefill_chunked(st, hk, T, q, k, v, gate, beta, out, chunk, (cudaStream_t)stream);
    if (prev != st->device) cudaSetDevice(prev);
    return r;
}

extern "C" int nmg_delta_step_batch(nmg_delta_state* const* states, int batch, int hk, const float* q, const float* k,
                                    const float* v, const float* gate, const float* beta, float* out, void* stream) {
    if (!states || batch < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step_batch: bad batch");
    if (batch == 0) return NMG_OK;
    const nmg_delta_state* s0 = states[0];
    if (!s0) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step_batch: null state");
    if (hk <= 0 || hk > s0->heads) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step_batch: bad key-head count %d", hk);
    if (!q || !k || !v || !gate || !beta || !out) return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step_batch: null tensor");
    for (int b = 0; b < batch; ++b) {
        const nmg_delta_state* st = states[b];
        if (!st || st->heads != s0->heads || st->dk != s0->dk || st->dv != s0->dv || st->device != s0->device)
            return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_step_batch: states differ in shape or device");
    }
    const int heads = s0->heads, dk = s0->dk, dv = s0->dv;
    cudaStream_t s = (cudaStream_t)stream;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != s0->device) NMG_CUDA_TRY(cudaSetDevice(s0->device));
    int st = NMG_OK;
    const bool vec = dk == 128 && dv % 64 == 0 && !(((uintptr_t)v | (uintptr_t)out) & 15);
    if (vec) {
        nmg::StepBatchArgs* a = new nmg::StepBatchArgs();
        a->q = q, a->k = k, a->v = v, a->gate = gate, a->beta = beta, a->out = out;
        a->heads = heads, a->hk = hk, a->dv = dv;
        for (int b0 = 0; b0 < batch && st == NMG_OK; b0 += nmg::kMaxStepBatch) {
            const int nb = std::min(nmg::kMaxStepBatch, batch - b0);
            for (int i = 0; i < nb; ++i) a->state[i] = states[b0 + i]->data;
            a->seq0 = b0;
            const cudaError_t e = nmg::launch_pdl(nmg::delta_step_batch_kernel, dim3(dv / 64, heads, nb), dim3(128), s, *a);
            if (e != cudaSuccess) st = set_error(NMG_CUDA_ERROR, "nmg_delta_step_batch: launch: %s", cudaGetErrorString(e));
        }
        delete a;
    } else {
        // Other shapes: the one-sequence step per sequence.
        for (int b = 0; b < batch && st == NMG_OK; ++b) {
            const int64_t qo = (int64_t)b * hk * dk, vo = (int64_t)b * heads * dv, go = (int64_t)b * heads;
            st = nmg_delta_step(states[b], hk, q + qo, k + qo, v + vo, gate + go, beta + go, out + vo, stream);
        }
    }
    if (prev != s0->device) cudaSetDevice(prev);
    return st;
}
