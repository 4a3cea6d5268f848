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
// Phase 1, delta_wy_kernel: one CTA per (key head, chunk), all in parallel.
//   [K;Q] K^T on the tensor core once for the value heads that share the key
//   head; per value head, A and M on the CUDA cores, T by a blocked fp32
//   triangular inverse and [I;M] T = [T;MT] on the tensor core.  Writes the
//   [K;Q] tile and its K^T, and per value head the [T;MT] tile and the
//   chunk's (beta, e, f, exp(G_last)), rounded to tf32 -- each as the exact
//   shared-memory image phase 2 multiplies from, so phase 2 fetches it with
//   one bulk copy.
// Phase 2, delta_scan_kernel: one CTA per (value head, 128 value columns);
//   walks the chunks in order with the state (transposed) resident in TMEM:
//     MMA1 S^T [K;Q]^T -> (K S | Q S)^T;  R^T -> TMEM;  MMA2 R^T [T;MT]^T ->
//     (D | M T R)^T;  (f D)^T -> TMEM;  MMA3 S^T += (f D)^T K  (S^T rescaled by
//     exp(G_last) beforehand);  O = e (Q S) + M T R -> global.
//   A producer warp streams the next chunk's tiles meanwhile.
//
// Operand layouts: every shared-memory operand is K-major with the 128-byte
// swizzle (a tf32 operand stored MN-major in that swizzle is not multiplied by
// this hardware), so the contraction over the chunk's tokens reads K^T.
// Precision: each operand is rounded to the nearest tf32 value (10-bit
// mantissa) before it is multiplied; every sum is fp32 and the state stays fp32.
#include "delta.cuh"
#include "tcgen05.cuh"

namespace nmg {
namespace {

constexpr int kC = 64;                         // tokens per chunk
constexpr int kDK = 128;                       // key dimension the images are laid out for
constexpr uint32_t kKQBytes = 65536;           // [K;Q]: 4 boxes (32 d each) x 128 rows x 128 B
constexpr uint32_t kKTBytes = 32768;           // K^T: 2 boxes (32 tokens each) x 128 rows (d) x 128 B
constexpr uint32_t kTMBytes = 32768;           // [T;MT]: 2 boxes (32 tokens each) x 128 rows x 128 B
constexpr uint32_t kAuxBytes = 1024;           // beta[64], e[64], f[64], exp(G_last), zero pad

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

// Shared memory of one (key head, chunk) CTA.  R0 (64 KB) holds the [K;Q]
// image and R1 (32 KB) its K^T until their stores have read them; then R0
// holds A (fp32 rows of 64, chunk q of row i at q ^ (i & 15)), the T^T image
// (row j = column j of T, fp32 while T is solved, then rounded) and the [I;M]
// image of even value heads, R1 the [I;M] image of odd ones, so the store of
// one head's [T;MT] overlaps the next head's work.  G holds the chunk's 64
// cumulative gates and, at [64], the first warp's total for the scan; D the
// four 16 x 16 diagonal blocks of T row-major, for the block products.
constexpr uint32_t P1_A = 0, P1_TI = 16384, P1_IM0 = 32768, P1_R1 = 65536, P1_IM1 = P1_R1,
                   P1_Y = P1_R1 + kKTBytes, P1_G = P1_Y + 3 * 1024, P1_AUX = P1_G + 512,
                   P1_D = P1_AUX + 2 * kAuxBytes, P1_BAR = P1_D + 4096, P1_END = P1_BAR + 64;
constexpr uint32_t P1_SMEM = 1024 + P1_END;

// Byte offset of T[i][j] .. T[i + 3][j] (i a multiple of 4) in the T^T image:
// row j, K-major over i in two boxes of 32.
__device__ __forceinline__ uint32_t ti_off4(uint32_t i, uint32_t j) { return (i >> 5) * 8192u + sw_chunk(j, (i & 31u) >> 2); }
__device__ __forceinline__ uint32_t ti_off(uint32_t i, uint32_t j) { return (i >> 5) * 8192u + sw_elem(j, i & 31u); }
// Float index of A[i][4 q .. 4 q + 3].
__device__ __forceinline__ int a_idx4(int i, int q) { return i * 64 + ((q ^ (i & 15)) << 2); }

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, fmaf(a.x, b.x, acc))));
}

// T = (I + A)^-1 for the strictly lower triangular 64 x 64 A, by 16 x 16
// blocks: the diagonal blocks by forward substitution (one column per
// thread), then the off-diagonal blocks one block diagonal at a time,
//   T_ij = -T_ii sum_{j <= k < i} A_ik T_kj,
// with all 128 threads on each step.  fp32 throughout; T lands in the T^T
// image unrounded.  Y holds 3 blocks of partial sums, D the diagonal blocks
// T_ii row-major ([4][16][16]).
__device__ __forceinline__ void wy_invert(const float* A, uint8_t* TI, float* Y, float* D, int tid) {
    if (tid < 64) {
        const int b = tid >> 4, c = tid & 15, j = 16 * b + c;
        float t[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (4 * q < r) {
                    const float4 av = *(const float4*)(A + a_idx4(16 * b + r, 4 * b + q));
                    if (4 * q + 0 < r) s0 = fmaf(av.x, t[4 * q + 0], s0);
                    if (4 * q + 1 < r) s1 = fmaf(av.y, t[4 * q + 1], s1);
                    if (4 * q + 2 < r) s0 = fmaf(av.z, t[4 * q + 2], s0);
                    if (4 * q + 3 < r) s1 = fmaf(av.w, t[4 * q + 3], s1);
                }
            }
            t[r] = r == c ? 1.f : (r < c ? 0.f : -(s0 + s1));
        }
        for (int i = 0; i < 16 * b; i += 4) *(float4*)(TI + ti_off4(i, j)) = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < 16; ++r) D[(b * 16 + r) * 16 + c] = t[r];
#pragma unroll
        for (int m = 0; m < 4; ++m)
            *(float4*)(TI + ti_off4(16 * b + 4 * m, j)) = make_float4(t[4 * m], t[4 * m + 1], t[4 * m + 2], t[4 * m + 3]);
    }
#pragma unroll 1
    for (int L = 1; L < 4; ++L) {
        const int pairs = (4 - L) * 128;  // (block, row r and r + 8, column) per thread
        __syncthreads();
        for (int p = tid; p < pairs; p += 128) {
            const int blk = p >> 7, r = (p >> 4) & 7, c = p & 15;
            const int bi = blk + L, j = 16 * blk + c;
            float y0 = 0.f, y1 = 0.f;
#pragma unroll 1
            for (int k = blk; k < bi; ++k) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 tv = *(const float4*)(TI + ti_off4(16 * k + 4 * u, j));
                    y0 = dot4(*(const float4*)(A + a_idx4(16 * bi + r, 4 * k + u)), tv, y0);
                    y1 = dot4(*(const float4*)(A + a_idx4(16 * bi + r + 8, 4 * k + u)), tv, y1);
                }
            }
            Y[(blk * 16 + r) * 16 + c] = y0;
            Y[(blk * 16 + r + 8) * 16 + c] = y1;
        }
        __syncthreads();
        for (int p = tid; p < pairs; p += 128) {
            const int blk = p >> 7, r = (p >> 4) & 7, c = p & 15;
            const int bi = blk + L, j = 16 * blk + c;
            float z0 = 0.f, z1 = 0.f;
            const float4* d0 = (const float4*)(D + (bi * 16 + r) * 16);
            const float4* d1 = (const float4*)(D + (bi * 16 + r + 8) * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // T_ii is lower triangular: its upper entries are stored zeros
                const float4 t0 = d0[q], t1 = d1[q];
                const float y0 = Y[(blk * 16 + 4 * q) * 16 + c], y1 = Y[(blk * 16 + 4 * q + 1) * 16 + c];
                const float y2 = Y[(blk * 16 + 4 * q + 2) * 16 + c], y3 = Y[(blk * 16 + 4 * q + 3) * 16 + c];
                z0 = fmaf(t0.w, y3, fmaf(t0.z, y2, fmaf(t0.y, y1, fmaf(t0.x, y0, z0))));
                z1 = fmaf(t1.w, y3, fmaf(t1.z, y2, fmaf(t1.y, y1, fmaf(t1.x, y0, z1))));
            }
            *(float*)(TI + ti_off(16 * bi + r, j)) = -z0;
            *(float*)(TI + ti_off(16 * bi + r + 8, j)) = -z1;
        }
    }
    __syncthreads();
    float4* ti4 = (float4*)TI;
#pragma unroll
    for (int i = tid; i < 1024; i += 128) {
        const float4 x = ti4[i];
        ti4[i] = tf32r4(x.x, x.y, x.z, x.w);
    }
}

// One CTA per (key head, chunk): the value heads kh, kh + hk, ... share the
// chunk's [K;Q] K^T product, so it is loaded, rounded and multiplied once.
__global__ void __launch_bounds__(128) delta_wy_kernel(const __grid_constant__ WyArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* A_s = (float*)(smem + P1_A);
    uint8_t* TI = smem + P1_TI;
    float* Y_s = (float*)(smem + P1_Y);
    float* G_s = (float*)(smem + P1_G);
    float* D_s = (float*)(smem + P1_D);
    uint64_t* bars = (uint64_t*)(smem + P1_BAR);  // 0: [K;Q] landed, 1: first MMA, 2: second MMA (once per value head)
    uint32_t* tmem_slot = (uint32_t*)(bars + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kh = (int)(blockIdx.x % (unsigned)a.hk), c = (int)(blockIdx.x / (unsigned)a.hk);
    const int64_t t0 = (int64_t)c * kC;
    const int64_t rec_k = (int64_t)kh * a.nchunks + c;

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
    // gate and beta of the first value head's tokens (zero past the end)
    const bool tok = tid < kC && t0 + tid < a.T;
    float g_raw = tok ? a.gate[(t0 + tid) * a.hv + kh] : 0.f;
    float b_raw = tok ? a.beta[(t0 + tid) * a.hv + kh] : 0.f;
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

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
    {
        // K^T image: row d holds K[0..63][d] (two boxes of 32 tokens).
        uint8_t* KT = smem + P1_R1;
        const int d = tid;
        const uint8_t* kcol = smem + (d >> 5) * 16384;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            float x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = *(const float*)(kcol + sw_elem(4 * q + e, d & 31));
            *(float4*)(KT + (q >> 3) * 16384 + sw_chunk(d, q & 7)) = make_float4(x[0], x[1], x[2], x[3]);
        }
        dev::fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            dev::bulk_s2g(a.kq_img + rec_k * (kKQBytes / 4), smem, kKQBytes);
            dev::bulk_s2g(a.kt_img + rec_k * (kKTBytes / 4), KT, kKTBytes);
            dev::bulk_commit();
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
    if (tid == 0) dev::bulk_wait_read();  // R0 and R1 are free once the image stores have read them
    __syncthreads();

    int gi = 0;
    for (int h = kh; h < a.hv; h += a.hk, ++gi) {
        uint8_t* IM = smem + ((gi & 1) ? P1_IM1 : P1_IM0);
        float* aux_s = (float*)(smem + P1_AUX + (gi & 1) * kAuxBytes);
        // Inclusive scan of the gate over the chunk.
        float gsum = g_raw;
        const float bt = b_raw;
        if (tid < kC) {
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float n = __shfl_up_sync(0xffffffffu, gsum, o);
                if (lane >= o) gsum += n;
            }
            if (tid == 31) G_s[64] = gsum;
        }
        // The next value head's gate and beta, in flight meanwhile.
        const int hn = h + a.hk;
        if (tok && hn < a.hv) {
            g_raw = a.gate[(t0 + tid) * a.hv + hn];
            b_raw = a.beta[(t0 + tid) * a.hv + hn];
        }
        // The buffers of head gi - 2 must have been read by their stores.
        if (tid == 0) dev::bulk_wait_read1();
        __syncthreads();
        if (tid >= 32 && tid < kC) gsum += G_s[64];
        if (tid < kC) G_s[tid] = gsum;
        __syncthreads();
        if (tid < kC) {
            aux_s[tid] = bt;
            aux_s[64 + tid] = expf(gsum);
            aux_s[128 + tid] = expf(G_s[kC - 1] - gsum);
        } else {
            aux_s[128 + tid] = tid == kC ? expf(G_s[kC - 1]) : 0.f;  // [192] = exp(G_last), then zeros
        }
        if (tid < kC) {
            const int i = tid;
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * q + e;
                    o[e] = j < i ? bt * __expf(gsum - G_s[j]) * __uint_as_float(r[j]) : 0.f;
                }
                *(float4*)(A_s + a_idx4(i, q)) = make_float4(o[0], o[1], o[2], o[3]);
                // identity row i of the [I;M] image
                const int j0 = 4 * q;
                *(float4*)(IM + (q >> 3) * 16384 + sw_chunk(i, q & 7)) =
                    make_float4(j0 == i ? 1.f : 0.f, j0 + 1 == i ? 1.f : 0.f, j0 + 2 == i ? 1.f : 0.f, j0 + 3 == i ? 1.f : 0.f);
            }
        } else {
            const int i = tid - kC;
            const float gq = G_s[i];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * q + e;
                    o[e] = j <= i ? __expf(gq - G_s[j]) * __uint_as_float(r[j]) : 0.f;
                }
                *(float4*)(IM + (q >> 3) * 16384 + sw_chunk(tid, q & 7)) = tf32r4(o[0], o[1], o[2], o[3]);
            }
        }
        __syncthreads();
        wy_invert(A_s, TI, Y_s, D_s, tid);
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
        dev::mbar_wait(&bars[2], gi & 1, a.err);
        tc::fence_after_sync();
        uint32_t y[64];
        {
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + 64;
            tc::ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&y[0]));
            tc::ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&y[32]));
        }
        // row tid of [T;MT], rounded, over the consumed [I;M] image
#pragma unroll
        for (int q = 0; q < 16; ++q)
            *(float4*)(IM + (q >> 3) * 16384 + sw_chunk(tid, q & 7)) =
                tf32r4(__uint_as_float(y[4 * q]), __uint_as_float(y[4 * q + 1]), __uint_as_float(y[4 * q + 2]),
                       __uint_as_float(y[4 * q + 3]));
        dev::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            const int64_t rec = (int64_t)h * a.nchunks + c;
            dev::bulk_s2g(a.tm_img + rec * (kTMBytes / 4), IM, kTMBytes);
            dev::bulk_s2g(a.aux + rec * (kAuxBytes / 4), aux_s, kAuxBytes);
            dev::bulk_commit();
        }
    }
    if (tid == 0) dev::bulk_wait_read();  // the stores are complete for the next kernel once this grid ends
    tc::fence_before_sync();
    __syncthreads();
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

// The scan works in the transposed orientation: TMEM lane j is value column
// j (128 per CTA) and every product is a TS-form MMA (A in TMEM) with N = 128.
//   MMA1  P    = S^T [K;Q]^T        A = S^T (TMEM),  B = [K;Q] image   -> (K S)^T | (Q S)^T
//   MMA2  D2   = R^T [T;MT]^T       A = R^T (TMEM),  B = [T;MT] image  -> D^T | (M T R)^T
//   MMA3  S^T += (f D)^T K          A = (f D)^T,     B = K^T image     (S^T pre-scaled by exp(G_last))
// Warpgroup 0 runs the chain (R, f D, MMA issue); warpgroup 1 rescales the
// state between MMA1 and MMA3 and forms O = e (Q S) + M T R, reading M T R
// before it lets MMA3 / MMA1 run; warp 8 loads.
constexpr int kCols = 128;  // value columns per CTA (TMEM lanes)
constexpr uint32_t kVTile = kC * kCols * 4;  // 4 boxes of 32 columns x 64 tokens
constexpr uint32_t TM_S = 0, TM_P = 128, TM_RD = 256, TM_D2 = 320;  // TMEM columns
constexpr uint32_t P2_KQ = 0,                //
    P2_KT = P2_KQ + kKQBytes,                //
    P2_TM = P2_KT + kKTBytes,                //
    P2_V = P2_TM + kTMBytes,                 // 2 stages
    P2_AUX = P2_V + 2 * kVTile,              // 2 stages
    P2_BAR = P2_AUX + 2 * kAuxBytes, P2_END = P2_BAR + 256;
constexpr uint32_t P2_SMEM = 1024 + P2_END;
static_assert(P2_SMEM <= 227 * 1024, "phase-2 shared memory");

enum : int {
    B_KQ_FULL, B_KQ_EMPTY, B_KT_FULL, B_KT_EMPTY, B_TM_FULL, B_TM_EMPTY, B_VA_FULL0, B_VA_FULL1, B_VA_EMPTY0,
    B_VA_EMPTY1, B_MMA1, B_MMA2, B_MMA3, B_SCALED, B_COUNT
};

__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__global__ void __launch_bounds__(288, 1) delta_scan_kernel(const __grid_constant__ ScanArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bar = (uint64_t*)(smem + P2_BAR);
    uint32_t* tmem_slot = (uint32_t*)(bar + B_COUNT);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, kh = h % a.hk;
    const int col0 = blockIdx.x * kCols;
    const int n = a.nchunks;

    if (tid == 0) {
        for (int i = 0; i < B_COUNT; ++i) dev::mbar_init(&bar[i], 1);
        dev::mbar_init(&bar[B_VA_EMPTY0], 2);
        dev::mbar_init(&bar[B_VA_EMPTY1], 2);
        dev::mbar_init(&bar[B_SCALED], 4);
        *abort_flag = 0;
        dev::fence_mbar_init();
        dev::prefetch_tensormap(&a.tm_v);
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    int* err = a.err;
    auto wait = [&](int b, uint32_t parity) -> bool {
        if (dev::mbar_wait(&bar[b], parity, err)) return true;
        *abort_flag = 1;
        return false;
    };

    if (warp == 8) {  // ---------------------------------------------- producer
        if (lane == 0) {
            const int64_t krec = (int64_t)kh * n, rec = (int64_t)h * n;
            for (int c = 0; c < n && !*abort_flag; ++c) {
                const int s = c & 1;
                const uint32_t prev = (uint32_t)(c - 1) & 1u;
                if (c >= 2 && !wait(B_VA_EMPTY0 + s, (uint32_t)((c >> 1) - 1) & 1u)) break;
                dev::mbar_arrive_expect_tx(&bar[B_VA_FULL0 + s], kAuxBytes + kVTile);
                dev::bulk_g2s(smem + P2_AUX + s * kAuxBytes, a.aux + (rec + c) * (kAuxBytes / 4), kAuxBytes,
                              &bar[B_VA_FULL0 + s]);
                for (int b = 0; b < 4; ++b)
                    dev::tma_load_3d(smem + P2_V + s * kVTile + b * 8192, &a.tm_v, col0 + 32 * b, h, c * kC,
                                     &bar[B_VA_FULL0 + s]);
                if (c >= 1 && !wait(B_KQ_EMPTY, prev)) break;
                dev::mbar_arrive_expect_tx(&bar[B_KQ_FULL], kKQBytes);
                dev::bulk_g2s(smem + P2_KQ, a.kq_img + (krec + c) * (kKQBytes / 4), kKQBytes, &bar[B_KQ_FULL]);
                if (c >= 1 && !wait(B_TM_EMPTY, prev)) break;
                dev::mbar_arrive_expect_tx(&bar[B_TM_FULL], kTMBytes);
                dev::bulk_g2s(smem + P2_TM, a.tm_img + (rec + c) * (kTMBytes / 4), kTMBytes, &bar[B_TM_FULL]);
                if (c >= 1 && !wait(B_KT_EMPTY, prev)) break;
                dev::mbar_arrive_expect_tx(&bar[B_KT_FULL], kKTBytes);
                dev::bulk_g2s(smem + P2_KT, a.kt_img + (krec + c) * (kKTBytes / 4), kKTBytes, &bar[B_KT_FULL]);
            }
        }
    } else {
        const int j = tid & 127;                     // value column (TMEM lane)
        const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
        const bool col_ok = col0 + j < a.dv;
        const uint32_t kq_addr = dev::smem_u32(smem + P2_KQ), kt_addr = dev::smem_u32(smem + P2_KT),
                       tm_addr = dev::smem_u32(smem + P2_TM);
        constexpr uint32_t id = tc::idesc_tf32(128, 128, 0, 0);
        float* scol = a.state + (int64_t)h * kDK * a.dv + col0 + j;  // state column j, stride dv

        if (warp < 4) {  // initial state: S^T row j <- state column j
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                uint32_t v[32];
#pragma unroll
                for (int d = 0; d < 32; ++d) v[d] = __float_as_uint(col_ok ? scol[(int64_t)(32 * b + d) * a.dv] : 0.f);
                tc::st_32x32b_x32(tmem + lanes + TM_S + 32 * b, v);
            }
            tc::wait_st();
        }
        tc::fence_before_sync();
        named_bar(2, 256);
        tc::fence_after_sync();

        if (warp < 4) {  // ------------------------------------- chain warpgroup
            // The tensor pipe runs one thread's MMAs in order and an M = 128
            // MMA costs about the same for any N up to 128, so each product is
            // one N = 128 sequence: X | QS, then D | M T R, then the state.
            auto issue_mma1 = [&](int c) {
                if (!wait(B_KQ_FULL, (uint32_t)c & 1u)) return;
#pragma unroll
                for (int kk = 0; kk < kDK / 8; ++kk)
                    tc::mma_tf32_ts(tmem + TM_P, tmem + TM_S + 8 * kk, kmajor_desc(kq_addr, kk, 16384), id, kk > 0);
                tc::commit(&bar[B_MMA1]);
                tc::commit(&bar[B_KQ_EMPTY]);
            };
            if (tid == 0) issue_mma1(0);
            for (int c = 0; c < n; ++c) {
                if (*abort_flag) break;
                const int s = c & 1;
                const uint32_t ph = (uint32_t)c & 1u;
                const float4* AUX4 = (const float4*)(smem + P2_AUX + s * kAuxBytes);
                const uint8_t* V = smem + P2_V + s * kVTile + (j >> 5) * 8192;
                wait(B_VA_FULL0 + s, (uint32_t)(c >> 1) & 1u);
                wait(B_MMA1, ph);
                tc::fence_after_sync();
                // R^T row j: beta_t (V[t][j] - e_t X[t][j])
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t x[32];
                    tc::ld_32x32b_x32(tmem + lanes + TM_P + 32 * half, x);
#pragma unroll
                    for (int i4 = 0; i4 < 8; ++i4) {
                        const float4 b4 = AUX4[8 * half + i4], e4 = AUX4[16 + 8 * half + i4];
                        const float bb[4] = {b4.x, b4.y, b4.z, b4.w}, ee[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int i = 4 * i4 + u, t = 32 * half + i;
                            const float vt = *(const float*)(V + sw_elem(t, j & 31));
                            x[i] = __float_as_uint(tf32r(bb[u] * (vt - ee[u] * __uint_as_float(x[i]))));
                        }
                    }
                    tc::st_32x32b_x32(tmem + lanes + TM_RD + 32 * half, x);
                }
                tc::wait_st();
                tc::fence_before_sync();
                named_bar(1, 128);
                if (tid == 0) {  // MMA2 (warpgroup 1 read the previous M T R before the state went on)
                    tc::fence_after_sync();
                    wait(B_TM_FULL, ph);
#pragma unroll
                    for (int kk = 0; kk < kC / 8; ++kk)
                        tc::mma_tf32_ts(tmem + TM_D2, tmem + TM_RD + 8 * kk, kmajor_desc(tm_addr, kk, 16384), id,
                                        kk > 0);
                    tc::commit(&bar[B_MMA2]);
                    tc::commit(&bar[B_TM_EMPTY]);
                }
                wait(B_MMA2, ph);
                tc::fence_after_sync();
                // (f D)^T row j, over R^T
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t y[32];
                    tc::ld_32x32b_x32(tmem + lanes + TM_D2 + 32 * half, y);
#pragma unroll
                    for (int i4 = 0; i4 < 8; ++i4) {
                        const float4 f4 = AUX4[32 + 8 * half + i4];
                        const float ff[4] = {f4.x, f4.y, f4.z, f4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            y[4 * i4 + u] = __float_as_uint(tf32r(ff[u] * __uint_as_float(y[4 * i4 + u])));
                    }
                    tc::st_32x32b_x32(tmem + lanes + TM_RD + 32 * half, y);
                }
                tc::wait_st();
                tc::fence_before_sync();
                named_bar(1, 128);
                if (tid == 0) {  // MMA3 (onto the rescaled state), then the next chunk's MMA1
                    tc::fence_after_sync();
                    dev::mbar_arrive(&bar[B_VA_EMPTY0 + s]);
                    wait(B_SCALED, ph);  // warpgroup 1: state rescaled and M T R read
                    wait(B_KT_FULL, ph);
#pragma unroll
                    for (int kk = 0; kk < kC / 8; ++kk)
                        tc::mma_tf32_ts(tmem + TM_S, tmem + TM_RD + 8 * kk, kmajor_desc(kt_addr, kk, 16384), id, 1);
                    tc::commit(&bar[B_KT_EMPTY]);
                    if (c + 1 < n)
                        issue_mma1(c + 1);
                    else
                        tc::commit(&bar[B_MMA3]);
                }
            }
        } else {  // --------------------------------------- state / output warpgroup
            for (int c = 0; c < n; ++c) {
                if (*abort_flag) break;
                const int s = c & 1;
                const uint32_t ph = (uint32_t)c & 1u;
                const float* AUX = (const float*)(smem + P2_AUX + s * kAuxBytes);
                wait(B_VA_FULL0 + s, (uint32_t)(c >> 1) & 1u);
                wait(B_MMA1, ph);
                tc::fence_after_sync();
                const float gamma = AUX[192];
#pragma unroll
                for (int b = 0; b < 4; ++b) {  // S^T <- exp(G_last) S^T before MMA3 adds the chunk
                    uint32_t v[32];
                    tc::ld_32x32b_x32(tmem + lanes + TM_S + 32 * b, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(gamma * __uint_as_float(v[i]));
                    tc::st_32x32b_x32(tmem + lanes + TM_S + 32 * b, v);
                }
                float o[kC];  // e_t (Q S)[t][j], then + (M T R)[t][j]
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t x[32];
                    tc::ld_32x32b_x32(tmem + lanes + TM_P + 64 + 32 * half, x);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[32 * half + i] = AUX[64 + 32 * half + i] * __uint_as_float(x[i]);
                }
                wait(B_MMA2, ph);
                tc::fence_after_sync();
                // M T R, read before MMA3 / MMA1 run: a TMEM load queued behind
                // those MMAs waits for them, and the next chunk's MMA2 rewrites it
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t y[32];
                    tc::ld_32x32b_x32(tmem + lanes + TM_D2 + 64 + 32 * half, y);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[32 * half + i] += __uint_as_float(y[i]);
                }
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(&bar[B_SCALED]);
                if (tid == 128) dev::mbar_arrive(&bar[B_VA_EMPTY0 + s]);
                if (col_ok) {
                    const int64_t t0 = (int64_t)c * kC;
                    const int tn = a.T - t0 < kC ? (int)(a.T - t0) : kC;
                    float* op = a.out + (t0 * a.hv + h) * (int64_t)a.dv + col0 + j;
                    const int64_t step = (int64_t)a.hv * a.dv;
#pragma unroll
                    for (int t = 0; t < kC; ++t)
                        if (t < tn) op[t * step] = o[t];
                }
            }
        }
        // final state: S^T row j -> state column j
        if (warp < 4) {
            if (!*abort_flag && wait(B_MMA3, 0)) {
                tc::fence_after_sync();
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    uint32_t v[32];
                    tc::ld_32x32b_x32(tmem + lanes + TM_S + 32 * b, v);
                    if (col_ok)
#pragma unroll
                        for (int d = 0; d < 32; ++d) scol[(int64_t)(32 * b + d) * a.dv] = __uint_as_float(v[d]);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
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

bool delta_chunked_supported(const nmg_delta_state* st) { return st->dk == kDK && st->dv % 32 == 0; }

int delta_prefill_chunked(nmg_delta_state* st, int hk, int64_t T, const float* q, const float* k, const float* v,
                          const float* gate, const float* beta, float* out, int chunk, cudaStream_t stream) {
    if (chunk != kC) return set_error(NMG_UNSUPPORTED, "chunked delta prefill: chunk must be %d", kC);
    if (!delta_chunked_supported(st))
        return set_error(NMG_UNSUPPORTED, "chunked delta prefill: built for Dk=%d and Dv a multiple of %d (got %d, %d)",
                         kDK, 32, st->dk, st->dv);
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

    static std::atomic<uint64_t> wy_set{0}, scan_set{0};  // one bit per device
    if ((rc = set_smem_once(delta_wy_kernel, P1_SMEM, wy_set)) != NMG_OK) return rc;
    if ((rc = set_smem_once(delta_scan_kernel, P2_SMEM, scan_set)) != NMG_OK) return rc;
    // one CTA per (key head, chunk), the key heads of a chunk side by side
    delta_wy_kernel<<<(unsigned)((int64_t)nchunks * hk), 128, P1_SMEM, stream>>>(wa);
    NMG_CUDA_TRY(cudaGetLastError());
    delta_scan_kernel<<<dim3((dv + kCols - 1) / kCols, hv), 288, P2_SMEM, stream>>>(sa);
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}

}  // namespace nmg
