// delta_chunked.cu -- chunked (WY / UT form) gated delta-rule prefill on the
// sm_100a tensor cores: tcgen05.mma kind::tf32, fp32 accumulators in TMEM.
//
// The reference runs the recurrence one token at a time (nm/src/qwen35.hpp:436-456
// calling gated_delta_step, nm/src/recurrent.hpp:146-177), state S [Dk][Dv]:
//   S <- exp(g_t) S;   d_t = beta_t (v_t - S^T k_t);   S <- S + k_t d_t^T;   o_t = S^T q_t
// For a chunk of C = 64 tokens that starts from state S0, with G the inclusive
// cumulative sum of g inside the chunk, e = exp(G) and f = exp(G_last - G):
//   A_ts = beta_t exp(G_t - G_s) (k_t . k_s)   for s < t,     T = (I + A)^-1
//   M_ts = exp(G_t - G_s) (q_t . k_s)           for s <= t
//   R = beta (V - e (K S0)),   D = T R          (D's rows are the chunk's d_t)
//   O = e (Q S0) + (M T) R
//   S_C = exp(G_last) S0 + K^T (f D)
// which is the same recurrence reassociated over the chunk.
//
// Phase 1, delta_wy_kernel: one CTA per (value head, chunk), all in parallel.
//   [K;Q] K^T on the tensor core; A and M on the CUDA cores; T by fp32 forward
//   substitution (one column per thread); [I;M] T = [T;MT] on the tensor core.
//   Writes the [T;MT] tile, the chunk's (beta, e, f, exp(G_last)) and, once per
//   key head, the [K;Q] tile and its K^T, rounded to tf32 -- each as the exact
//   shared-memory image phase 2 multiplies from, so phase 2 fetches it with one
//   bulk copy.
// Phase 2, delta_scan_kernel: one CTA per (value head, 32 state columns); walks
//   the chunks in order with its state slice in registers:
//     MMA1 [K;Q] S -> (K S, Q S);  R -> smem;  MMA2 [T;MT] R -> (D, M T R);
//     O -> global;  f D -> smem;  MMA3 K^T (f D);  S <- exp(G_last) S + that.
//   A producer warp streams the next chunk's tiles meanwhile.
//
// Operand layouts: every tensor-core operand is K-major with the 128-byte
// swizzle (a tf32 operand stored MN-major in that swizzle is not multiplied by
// this hardware), so the contraction over the chunk's tokens reads K^T, and
// the state, R and f D images are written transposed (column per thread).
// Precision: each operand is rounded to the nearest tf32 value (10-bit
// mantissa) before it is multiplied; every sum is fp32 and the state stays fp32.
#include "delta.cuh"
#include "tcgen05.cuh"

namespace nmg {
namespace {

constexpr int kC = 64;                         // tokens per chunk
constexpr int kDK = 128;                       // key dimension the images are laid out for
constexpr int kSlice = 32;                     // state columns per phase-2 CTA
constexpr uint32_t kKQBytes = 65536;           // [K;Q]: 4 boxes (32 d each) x 128 rows x 128 B
constexpr uint32_t kKTBytes = 32768;           // K^T: 2 boxes (32 tokens each) x 128 rows (d) x 128 B
constexpr uint32_t kTMBytes = 32768;           // [T;MT]: 2 boxes (32 tokens each) x 128 rows x 128 B
constexpr uint32_t kAuxBytes = 1024;           // beta[64], e[64], f[64], exp(G_last), zero pad
constexpr uint32_t kVBytes = kC * kSlice * 4;  // one chunk of one value-column slice

__device__ __forceinline__ float tf32r(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Byte offset of 16-byte chunk `q` (0..7) of row `row` in a 128-byte-swizzled
// tile whose rows are 128 bytes (the layout TMA writes with SWIZZLE_128B).
__device__ __forceinline__ uint32_t sw_chunk(uint32_t row, uint32_t q) { return row * 128u + ((q ^ (row & 7u)) << 4); }
// Byte offset of element `col` (< 32) of row `row` in such a tile.
__device__ __forceinline__ uint32_t sw_elem(uint32_t row, uint32_t col) {
    return sw_chunk(row, col >> 2) + ((col & 3u) << 2);
}

__device__ __forceinline__ float4 tf32r4(float a, float b, float c, float d) {
    return make_float4(tf32r(a), tf32r(b), tf32r(c), tf32r(d));
}

// Barrier over the 128 compute threads (named barrier 1) that also returns
// whether any of them passed `pred`.
__device__ __forceinline__ bool bar_any_128(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

// K-major, 128-byte-swizzle descriptor for k-step `kk` (8 tf32 values) of an
// image whose 32-column boxes sit `box_bytes` apart.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk, uint32_t box_bytes) {
    return tc::smem_desc_sw128(base + (uint32_t)(kk >> 2) * box_bytes + (uint32_t)(kk & 3) * 32, 16, 1024);
}

// ------------------------------------------------------------ phase 1

struct WyArgs {
    CUtensorMap tm_q, tm_k;  // (dk, hk, T) fp32, box {32, 1, 64}, 128-byte swizzle
    const float* gate;       // [T][hv]
    const float* beta;       // [T][hv]
    float* kq_img;           // [hk][nchunks][kKQBytes / 4]
    float* kt_img;           // [hk][nchunks][kKTBytes / 4]
    float* tm_img;           // [hv][nchunks][kTMBytes / 4]
    float* aux;              // [hv][nchunks][kAuxBytes / 4]
    int64_t T;
    int hv, hk, nchunks;
    int* err;
};

// Shared memory: region 0 (64 KB) holds the [K;Q] image; once the first MMA
// and the image's store are done it is reused for A (rows of 64 floats, chunk
// q of row i at q ^ (i & 15)), the [I;M] image (later the [T;MT] image) and the
// T^T image (row j = column j of T).  K^T is built beside it.
constexpr uint32_t P1_A = 0, P1_IM = 16384, P1_TI = 49152, P1_KT = 65536, P1_G = P1_KT + kKTBytes,
                   P1_AUX = P1_G + 256, P1_BAR = P1_AUX + kAuxBytes, P1_END = P1_BAR + 64;
constexpr uint32_t P1_SMEM = 1024 + P1_END;

__global__ void __launch_bounds__(128) delta_wy_kernel(const __grid_constant__ WyArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* G_s = (float*)(smem + P1_G);
    float* aux_s = (float*)(smem + P1_AUX);
    uint64_t* bars = (uint64_t*)(smem + P1_BAR);  // 0: [K;Q] landed, 1: first MMA, 2: second MMA
    uint32_t* tmem_slot = (uint32_t*)(bars + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, h = blockIdx.y, kh = h % a.hk;
    const bool publish = h < a.hk;  // value head h == its key head: writes the K images once
    const int64_t t0 = (int64_t)c * kC;

    if (tid == 0) {
        dev::prefetch_tensormap(&a.tm_q);
        dev::prefetch_tensormap(&a.tm_k);
        for (int i = 0; i < 3; ++i) dev::mbar_init(&bars[i], 1);
        dev::fence_mbar_init();
        dev::mbar_arrive_expect_tx(&bars[0], kKQBytes);
        // box b of the image: K rows 0..63 then Q rows 0..63 for d in [32b, 32b+32)
        for (int b = 0; b < 4; ++b) {
            dev::tma_load_3d(smem + b * 16384, &a.tm_k, b * 32, kh, (int32_t)t0, &bars[0]);
            dev::tma_load_3d(smem + b * 16384 + 8192, &a.tm_q, b * 32, kh, (int32_t)t0, &bars[0]);
        }
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 128);
        tc::tmem_relinquish();
    }

    // Gate and beta of the chunk's tokens (zero past the end), inclusive scan of the gate.
    float gsum = 0.f, bt = 0.f;
    if (tid < kC) {
        const int64_t t = t0 + tid;
        if (t < a.T) {
            gsum = a.gate[t * a.hv + h];
            bt = a.beta[t * a.hv + h];
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float n = __shfl_up_sync(0xffffffffu, gsum, o);
            if (lane >= o) gsum += n;
        }
        if (tid == 31) G_s[0] = gsum;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    if (tid >= 32 && tid < kC) gsum += G_s[0];
    __syncthreads();
    if (tid < kC) G_s[tid] = gsum;
    __syncthreads();
    if (tid < kC) {
        aux_s[tid] = bt;
        aux_s[64 + tid] = expf(gsum);
        aux_s[128 + tid] = expf(G_s[kC - 1] - gsum);
    } else {
        aux_s[128 + tid] = tid == kC ? expf(G_s[kC - 1]) : 0.f;  // [192] = exp(G_last), then zeros
    }

    // Round the [K;Q] tile to tf32 in place.
    dev::mbar_wait(&bars[0], 0, a.err);
    {
        float4* kq4 = (float4*)smem;
#pragma unroll 4
        for (int i = tid; i < (int)(kKQBytes / 16); i += 128) {
            const float4 x = kq4[i];
            kq4[i] = tf32r4(x.x, x.y, x.z, x.w);
        }
    }
    dev::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t base = dev::smem_u32(smem);
        constexpr uint32_t id = tc::idesc_tf32(128, 64, 0, 0);
#pragma unroll
        for (int kk = 0; kk < kDK / 8; ++kk) {  // [K;Q] x K^T: B is the K rows of the same image
            const uint64_t d = kmajor_desc(base, kk, 16384);
            tc::mma_tf32_ss(tmem, d, d, id, kk > 0);
        }
        tc::commit(&bars[1]);
    }
    if (publish) {
        // K^T image: row d holds K[0..63][d] (two boxes of 32 tokens).
        uint8_t* KT = smem + P1_KT;
        const int d = tid;
        const uint8_t* kcol = smem + (d >> 5) * 16384;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            float x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = 4 * q + e;
                x[e] = *(const float*)(kcol + sw_elem(t, d & 31));
            }
            *(float4*)(KT + (q >> 3) * 16384 + sw_chunk(d, q & 7)) = make_float4(x[0], x[1], x[2], x[3]);
        }
        dev::fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            const int64_t rec = (int64_t)kh * a.nchunks + c;
            dev::bulk_s2g(a.kq_img + rec * (kKQBytes / 4), smem, kKQBytes);
            dev::bulk_s2g(a.kt_img + rec * (kKTBytes / 4), KT, kKTBytes);
            dev::bulk_commit();
            dev::bulk_wait_read();
        }
    }
    dev::mbar_wait(&bars[1], 0, a.err);
    tc::fence_after_sync();
    uint32_t r[64];  // row tid: (K K^T) row for tid < 64, (Q K^T) row tid - 64 otherwise
    {
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        tc::ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tc::ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
    }
    __syncthreads();  // region 0 is free from here on (thread 0 waited for the stores to read it)

    float* A_s = (float*)(smem + P1_A);
    uint8_t* IM = smem + P1_IM;
    uint8_t* TI = smem + P1_TI;
    if (tid < kC) {
        const int i = tid;
        const float gi = G_s[i];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * q + e;
                o[e] = j < i ? bt * __expf(gi - G_s[j]) * __uint_as_float(r[j]) : 0.f;
            }
            *(float4*)(A_s + i * 64 + ((q ^ (i & 15)) << 2)) = make_float4(o[0], o[1], o[2], o[3]);
            // identity row i of the [I;M] image
            const int j0 = 4 * q;
            *(float4*)(IM + (q >> 3) * 16384 + sw_chunk(i, q & 7)) =
                make_float4(j0 == i ? 1.f : 0.f, j0 + 1 == i ? 1.f : 0.f, j0 + 2 == i ? 1.f : 0.f, j0 + 3 == i ? 1.f : 0.f);
        }
    } else {
        const int i = tid - kC;
        const float gi = G_s[i];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * q + e;
                o[e] = j <= i ? __expf(gi - G_s[j]) * __uint_as_float(r[j]) : 0.f;
            }
            *(float4*)(IM + (q >> 3) * 16384 + sw_chunk(tid, q & 7)) = tf32r4(o[0], o[1], o[2], o[3]);
        }
    }
    __syncthreads();

    // T = (I + A)^-1 by forward substitution; thread j < 64 owns column j:
    // T_ij = [i == j] - sum_{k < i} A_ik T_kj (zero above the diagonal).
    if (tid < kC) {
        const int j = tid;
        float t[kC];
#pragma unroll
        for (int i = 0; i < kC; ++i) {
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
            for (int q = 0; q < (i + 3) / 4; ++q) {
                const float4 av = *(const float4*)(A_s + i * 64 + ((q ^ (i & 15)) << 2));
                if (4 * q + 0 < i) s0 = fmaf(av.x, t[4 * q + 0], s0);
                if (4 * q + 1 < i) s1 = fmaf(av.y, t[4 * q + 1], s1);
                if (4 * q + 2 < i) s2 = fmaf(av.z, t[4 * q + 2], s2);
                if (4 * q + 3 < i) s3 = fmaf(av.w, t[4 * q + 3], s3);
            }
            t[i] = i == j ? 1.f : -((s0 + s1) + (s2 + s3));
        }
        // column j of T is row j of the K-major B operand (two boxes of 32 k)
#pragma unroll
        for (int q = 0; q < 16; ++q)
            *(float4*)(TI + (q >> 3) * 8192 + sw_chunk(j, q & 7)) =
                tf32r4(t[4 * q], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
    }
    dev::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t im = dev::smem_u32(IM), ti = dev::smem_u32(TI);
        constexpr uint32_t id = tc::idesc_tf32(128, 64, 0, 0);
#pragma unroll
        for (int kk = 0; kk < kC / 8; ++kk)  // [I;M] x T
            tc::mma_tf32_ss(tmem + 64, kmajor_desc(im, kk, 16384), kmajor_desc(ti, kk, 8192), id, kk > 0);
        tc::commit(&bars[2]);
    }
    dev::mbar_wait(&bars[2], 0, a.err);
    tc::fence_after_sync();
    {
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + 64;
        tc::ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tc::ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
    }
    // row tid of [T;MT], rounded, over the consumed [I;M] image
#pragma unroll
    for (int q = 0; q < 16; ++q)
        *(float4*)(IM + (q >> 3) * 16384 + sw_chunk(tid, q & 7)) =
            tf32r4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                   __uint_as_float(r[4 * q + 3]));
    dev::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
        const int64_t rec = (int64_t)h * a.nchunks + c;
        dev::bulk_s2g(a.tm_img + rec * (kTMBytes / 4), IM, kTMBytes);
        dev::bulk_s2g(a.aux + rec * (kAuxBytes / 4), aux_s, kAuxBytes);
        dev::bulk_commit();
        dev::bulk_wait_all();
    }
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 128);
    }
}

// ------------------------------------------------------------ phase 2

struct ScanArgs {
    CUtensorMap tm_v;  // (dv, hv, T) fp32, box {32, 1, 64}, 128-byte swizzle
    const float* kq_img;
    const float* kt_img;
    const float* tm_img;
    const float* aux;
    float* state;  // [hv][128][dv]
    float* out;    // [T][hv][dv]
    int64_t T;
    int hv, hk, dv, nchunks;
    int* err;
};

// Shared memory.  The three big tiles are single-buffered (each is refilled as
// soon as its MMA of the current chunk completes, a whole chunk before its next
// use); V and aux are double-buffered.  The state image is S^T (row j = column
// j of the slice, 4 boxes of 32 k); the R image holds R^T, later (f D)^T (row j,
// 2 boxes of 32 tokens).
constexpr uint32_t P2_KQ = 0,                //
    P2_KT = P2_KQ + kKQBytes,                //
    P2_TM = P2_KT + kKTBytes,                //
    P2_V = P2_TM + kTMBytes,                 // 2 stages
    P2_S = P2_V + 2 * kVBytes,               // 4 boxes x 32 rows x 128 B
    P2_R = P2_S + kDK * kSlice * 4,          // 2 boxes x 32 rows x 128 B
    P2_AUX = P2_R + kC * kSlice * 4,         // 2 stages
    P2_BAR = P2_AUX + 2 * kAuxBytes, P2_END = P2_BAR + 128;
constexpr uint32_t P2_SMEM = 1024 + P2_END;
static_assert(P2_SMEM <= 227 * 1024, "phase-2 shared memory");

// Column `col` (a k index) of a transposed 32-row image: element j of `v`
// goes to row j, column col; boxes of 32 columns `box_bytes` apart.
__device__ __forceinline__ void store_col_image(uint8_t* img, int col, uint32_t box_bytes, const float (&v)[kSlice]) {
    uint8_t* base = img + (col >> 5) * box_bytes;
#pragma unroll
    for (int j = 0; j < kSlice; ++j) *(float*)(base + sw_elem(j, col & 31)) = tf32r(v[j]);
}

__global__ void __launch_bounds__(160, 1) delta_scan_kernel(const __grid_constant__ ScanArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + P2_BAR);
    uint64_t* kq_full = bars + 0;
    uint64_t* kq_empty = bars + 1;
    uint64_t* kt_full = bars + 2;
    uint64_t* kt_empty = bars + 3;
    uint64_t* tm_full = bars + 4;
    uint64_t* tm_empty = bars + 5;
    uint64_t* va_full = bars + 6;   // [2]: V and aux of a chunk landed
    uint64_t* va_empty = bars + 8;  // [2]: the chunk's V and aux were read
    uint64_t* mma_done = bars + 10;  // [3]
    uint32_t* tmem_slot = (uint32_t*)(bars + 13);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, kh = h % a.hk;
    const int col0 = blockIdx.x * kSlice;

    if (tid == 0) {
        for (int i = 0; i < 13; ++i) dev::mbar_init(&bars[i], 1);
        dev::fence_mbar_init();
        dev::prefetch_tensormap(&a.tm_v);
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 128);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            const int64_t krec = (int64_t)kh * a.nchunks, rec = (int64_t)h * a.nchunks;
            for (int c = 0; c < a.nchunks; ++c) {
                const int s = c & 1;
                if (c >= 2 && !dev::mbar_wait(&va_empty[s], ((c >> 1) - 1) & 1, a.err)) break;
                dev::mbar_arrive_expect_tx(&va_full[s], kAuxBytes + kVBytes);
                dev::bulk_g2s(smem + P2_AUX + s * kAuxBytes, a.aux + (rec + c) * (kAuxBytes / 4), kAuxBytes,
                              &va_full[s]);
                dev::tma_load_3d(smem + P2_V + s * kVBytes, &a.tm_v, col0, h, c * kC, &va_full[s]);
                const uint32_t prev = (uint32_t)(c - 1) & 1u;
                if (c >= 1 && !dev::mbar_wait(kq_empty, prev, a.err)) break;
                dev::mbar_arrive_expect_tx(kq_full, kKQBytes);
                dev::bulk_g2s(smem + P2_KQ, a.kq_img + (krec + c) * (kKQBytes / 4), kKQBytes, kq_full);
                if (c >= 1 && !dev::mbar_wait(tm_empty, prev, a.err)) break;
                dev::mbar_arrive_expect_tx(tm_full, kTMBytes);
                dev::bulk_g2s(smem + P2_TM, a.tm_img + (rec + c) * (kTMBytes / 4), kTMBytes, tm_full);
                if (c >= 1 && !dev::mbar_wait(kt_empty, prev, a.err)) break;
                dev::mbar_arrive_expect_tx(kt_full, kKTBytes);
                dev::bulk_g2s(smem + P2_KT, a.kt_img + (krec + c) * (kKTBytes / 4), kKTBytes, kt_full);
            }
        }
    } else {
        const uint32_t lanes = (uint32_t)(warp * 32) << 16;
        uint8_t* Simg = smem + P2_S;
        uint8_t* Rimg = smem + P2_R;
        const uint32_t s_addr = dev::smem_u32(Simg), r_addr = dev::smem_u32(Rimg);
        const uint32_t kq_addr = dev::smem_u32(smem + P2_KQ), kt_addr = dev::smem_u32(smem + P2_KT),
                       tm_addr = dev::smem_u32(smem + P2_TM);
        constexpr uint32_t id = tc::idesc_tf32(128, kSlice, 0, 0);
        float S[kSlice];  // state row k = tid, columns col0..col0+31
        float* srow = a.state + ((int64_t)h * kDK + tid) * a.dv + col0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 x = ((const float4*)srow)[q];
            S[4 * q] = x.x, S[4 * q + 1] = x.y, S[4 * q + 2] = x.z, S[4 * q + 3] = x.w;
        }
        store_col_image(Simg, tid, 4096, S);
        dev::fence_proxy_async_smem();
        tc::fence_before_sync();
        bool failed = false;
        bar_any_128(false);

        for (int c = 0; c < a.nchunks; ++c) {
            const int s = c & 1;
            const uint32_t ph = (uint32_t)c & 1u;
            const float* AUX = (const float*)(smem + P2_AUX + s * kAuxBytes);
            const uint8_t* V = smem + P2_V + s * kVBytes;
            failed |= !dev::mbar_wait(&va_full[s], (uint32_t)(c >> 1) & 1u, a.err);
            if (tid == 0) {  // MMA1: [K;Q] x S -> columns 0..31
                tc::fence_after_sync();
                failed |= !dev::mbar_wait(kq_full, ph, a.err);
#pragma unroll
                for (int kk = 0; kk < kDK / 8; ++kk)
                    tc::mma_tf32_ss(tmem, kmajor_desc(kq_addr, kk, 16384), kmajor_desc(s_addr, kk, 4096), id, kk > 0);
                tc::commit(&mma_done[0]);
                tc::commit(kq_empty);
            }
            failed |= !dev::mbar_wait(&mma_done[0], ph, a.err);
            tc::fence_after_sync();
            uint32_t x[32];  // (K S) row tid, or (Q S) row tid - 64
            tc::ld_32x32b_x32(tmem + lanes, x);
            const float gamma = AUX[192];
            if (tid < kC) {
                const float bt = AUX[tid], et = AUX[64 + tid];
                float rr[kSlice];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 vv = *(const float4*)(V + sw_chunk(tid, q));
                    rr[4 * q + 0] = bt * (vv.x - et * __uint_as_float(x[4 * q + 0]));
                    rr[4 * q + 1] = bt * (vv.y - et * __uint_as_float(x[4 * q + 1]));
                    rr[4 * q + 2] = bt * (vv.z - et * __uint_as_float(x[4 * q + 2]));
                    rr[4 * q + 3] = bt * (vv.w - et * __uint_as_float(x[4 * q + 3]));
                }
                store_col_image(Rimg, tid, 4096, rr);
            }
            dev::fence_proxy_async_smem();
            tc::fence_before_sync();
            if (bar_any_128(failed)) break;

            if (tid == 0) {  // MMA2: [T;MT] x R -> columns 32..63
                tc::fence_after_sync();
                failed |= !dev::mbar_wait(tm_full, ph, a.err);
#pragma unroll
                for (int kk = 0; kk < kC / 8; ++kk)
                    tc::mma_tf32_ss(tmem + 32, kmajor_desc(tm_addr, kk, 16384), kmajor_desc(r_addr, kk, 4096), id,
                                    kk > 0);
                tc::commit(&mma_done[1]);
                tc::commit(tm_empty);
            }
            failed |= !dev::mbar_wait(&mma_done[1], ph, a.err);
            tc::fence_after_sync();
            uint32_t y[32];  // D row tid, or (M T R) row tid - 64
            tc::ld_32x32b_x32(tmem + lanes + 32, y);
            if (tid < kC) {
                const float ft = AUX[128 + tid];
                float dd[kSlice];
#pragma unroll
                for (int j = 0; j < kSlice; ++j) dd[j] = ft * __uint_as_float(y[j]);
                store_col_image(Rimg, tid, 4096, dd);
            } else {
                const int t = tid - kC;
                const int64_t row = (int64_t)c * kC + t;
                const float et = AUX[64 + t];
                if (row < a.T) {
                    float4* o = (float4*)(a.out + (row * a.hv + h) * a.dv + col0);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        o[q] = make_float4(fmaf(et, __uint_as_float(x[4 * q + 0]), __uint_as_float(y[4 * q + 0])),
                                           fmaf(et, __uint_as_float(x[4 * q + 1]), __uint_as_float(y[4 * q + 1])),
                                           fmaf(et, __uint_as_float(x[4 * q + 2]), __uint_as_float(y[4 * q + 2])),
                                           fmaf(et, __uint_as_float(x[4 * q + 3]), __uint_as_float(y[4 * q + 3])));
                }
            }
            dev::fence_proxy_async_smem();
            tc::fence_before_sync();
            if (bar_any_128(failed)) break;

            if (tid == 0) {  // MMA3: K^T x (f D) -> columns 64..95
                tc::fence_after_sync();
                dev::mbar_arrive(&va_empty[s]);
                failed |= !dev::mbar_wait(kt_full, ph, a.err);
#pragma unroll
                for (int kk = 0; kk < kC / 8; ++kk)
                    tc::mma_tf32_ss(tmem + 64, kmajor_desc(kt_addr, kk, 16384), kmajor_desc(r_addr, kk, 4096), id,
                                    kk > 0);
                tc::commit(&mma_done[2]);
                tc::commit(kt_empty);
            }
            failed |= !dev::mbar_wait(&mma_done[2], ph, a.err);
            tc::fence_after_sync();
            uint32_t u[32];
            tc::ld_32x32b_x32(tmem + lanes + 64, u);
#pragma unroll
            for (int j = 0; j < kSlice; ++j) S[j] = fmaf(gamma, S[j], __uint_as_float(u[j]));
            store_col_image(Simg, tid, 4096, S);
            dev::fence_proxy_async_smem();
            tc::fence_before_sync();
            if (bar_any_128(failed)) break;
        }
        if (!failed) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
                ((float4*)srow)[q] = make_float4(S[4 * q], S[4 * q + 1], S[4 * q + 2], S[4 * q + 3]);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 128);
    }
}

int encode_f32_3d(EncodeTiledFn enc, CUtensorMap* map, const float* base, int inner, int mid, int64_t outer) {
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)mid, (cuuint64_t)outer};
    cuuint64_t strides[2] = {(cuuint64_t)inner * 4, (cuuint64_t)inner * mid * 4};
    cuuint32_t box[3] = {32, 1, (cuuint32_t)kC};
    cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(NMG_CUDA_ERROR, "chunked delta prefill: tensor map (%d)", (int)r);
    return NMG_OK;
}

}  // namespace

bool delta_chunked_supported(const nmg_delta_state* st) { return st->dk == kDK && st->dv % kSlice == 0; }

int delta_prefill_chunked(nmg_delta_state* st, int hk, int64_t T, const float* q, const float* k, const float* v,
                          const float* gate, const float* beta, float* out, int chunk, cudaStream_t stream) {
    if (chunk != kC) return set_error(NMG_UNSUPPORTED, "chunked delta prefill: chunk must be %d", kC);
    if (!delta_chunked_supported(st))
        return set_error(NMG_UNSUPPORTED, "chunked delta prefill: built for Dk=%d and Dv a multiple of %d (got %d, %d)",
                         kDK, kSlice, st->dk, st->dv);
    if (!q || !k || !v || !gate || !beta || !out)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_delta_prefill: null argument");
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15)
        return set_error(NMG_INVALID_ARGUMENT, "chunked delta prefill: q, k, v and out must be 16-byte aligned");
    if (T > 0x7FFFFFFFll - kC) return set_error(NMG_LENGTH_ERROR, "chunked delta prefill: too many tokens");
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(NMG_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    const int hv = st->heads, dv = st->dv;
    const int nchunks = (int)((T + kC - 1) / kC);
    const size_t kq_bytes = (size_t)hk * nchunks * kKQBytes;
    const size_t kt_bytes = (size_t)hk * nchunks * kKTBytes;
    const size_t tm_bytes = (size_t)hv * nchunks * kTMBytes;
    const size_t aux_bytes = (size_t)hv * nchunks * kAuxBytes;
    void* scratch = nullptr;
    int rc = device_scratch(st->device, kq_bytes + kt_bytes + tm_bytes + aux_bytes, &scratch);
    if (rc != NMG_OK) return rc;
    int* err = nullptr;
    if ((rc = device_error_flag(st->device, &err)) != NMG_OK) return rc;

    WyArgs wa;
    if ((rc = encode_f32_3d(enc, &wa.tm_q, q, kDK, hk, T)) != NMG_OK) return rc;
    if ((rc = encode_f32_3d(enc, &wa.tm_k, k, kDK, hk, T)) != NMG_OK) return rc;
    wa.gate = gate;
    wa.beta = beta;
    wa.kq_img = (float*)scratch;
    wa.kt_img = (float*)((char*)scratch + kq_bytes);
    wa.tm_img = (float*)((char*)scratch + kq_bytes + kt_bytes);
    wa.aux = (float*)((char*)scratch + kq_bytes + kt_bytes + tm_bytes);
    wa.T = T;
    wa.hv = hv;
    wa.hk = hk;
    wa.nchunks = nchunks;
    wa.err = err;

    ScanArgs sa;
    if ((rc = encode_f32_3d(enc, &sa.tm_v, v, dv, hv, T)) != NMG_OK) return rc;
    sa.kq_img = wa.kq_img;
    sa.kt_img = wa.kt_img;
    sa.tm_img = wa.tm_img;
    sa.aux = wa.aux;
    sa.state = st->data;
    sa.out = out;
    sa.T = T;
    sa.hv = hv;
    sa.hk = hk;
    sa.dv = dv;
    sa.nchunks = nchunks;
    sa.err = err;

    static unsigned attr_set = 0;
    const unsigned dbit = 1u << (st->device & 31);
    if (!(attr_set & dbit)) {
        NMG_CUDA_TRY(cudaFuncSetAttribute(delta_wy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P1_SMEM));
        NMG_CUDA_TRY(cudaFuncSetAttribute(delta_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P2_SMEM));
        attr_set |= dbit;
    }
    delta_wy_kernel<<<dim3(nchunks, hv), 128, P1_SMEM, stream>>>(wa);
    NMG_CUDA_TRY(cudaGetLastError());
    delta_scan_kernel<<<dim3(dv / kSlice, hv), 160, P2_SMEM, stream>>>(sa);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace nmg
