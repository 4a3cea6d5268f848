/*
 * nm_quant_oracle.c -- CPU restatement of the nm engine's quantised weight
 * products (Weight<In,Out>::matvec / matmul over GGUF block formats).
 *
 * TEST INFRASTRUCTURE ONLY.  Part of the parity checker for the CUDA path
 * under hero_b200/ (built into the same libnm_oracle.so as nm_oracle.c).
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.
 *
 * Each function restates one piece of the reference (paths relative to the
 * nm/ project root) in the same operation order as its scalar (non-NEON)
 * build, which is the build this container's x86 hosts run:
 *
 *   GGUF type codes, block layouts     src/quant.hpp:18-27, :52-85
 *   nmq_row_bytes                       src/quant.hpp:89-108  type_size_bytes
 *   nmq_scale_min_k4                    src/quant.hpp:154-162 get_scale_min_k4
 *   nmq_dequant_row                     src/quant.hpp:291-400 dequant_to_f32
 *   nmq_dot_fp32 (fp32 activations)     src/quant.hpp:130-289 dot_block_* summed
 *                                       per row as Weight::matvec's NM_FP32_ACT
 *                                       branch does (src/quant_i8.hpp:394-427)
 *   nmq_quantize_row_q8_0               src/quant_i8.hpp:69-81  quantize_row_q8_0
 *   nmq_quantize_row_q8_K               src/quant_i8.hpp:38-67  quantize_row_q8_K
 *                                       (nearest_int :30-36)
 *   nmq_vec_dot_i8                      src/quant_i8.hpp:84-101 (Q8_0), :102-127
 *                                       (Q4_0), :144-187 (Q4_K), :232-274 (Q6_K)
 *   nmq_matmul                          src/quant_i8.hpp:351-392 (matvec) and
 *                                       :430-514 (matmul): activations quantised
 *                                       once per row, then one integer dot per
 *                                       (row, output); Q5_K and fp32_act take the
 *                                       fp32-activation path (has_i8_kernel :325).
 *
 * Block bytes are the GGUF layouts, packed (no padding): Q4_0 18 B, Q8_0 34 B,
 * Q4_K 144 B, Q5_K 176 B, Q6_K 210 B per block; the activation blocks are
 * Q8_0 (34 B) and Q8_K (4 B fp32 d + 256 int8 + 16 int16 bsums = 292 B).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

float nmo_fp16_to_fp32(uint16_t h);
uint16_t nmo_fp32_to_fp16(float f);
float nmo_dot(const float* a, const float* b, int64_t n);

enum { GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q5_K = 13, GT_Q6_K = 14, GT_Q8_K = 15 };
enum { Q4_0_B = 18, Q8_0_B = 34, Q4_K_B = 144, Q5_K_B = 176, Q6_K_B = 210, Q8_K_B = 292 };

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static float rdf(const uint8_t* p) {
    float f;
    memcpy(&f, p, 4);
    return f;
}
static int16_t rds16(const uint8_t* p) {
    int16_t v;
    memcpy(&v, p, 2);
    return v;
}

/* elements per block; 0 for an unknown type */
int64_t nmq_block_len(int type) {
    switch (type) {
        case GT_F32: return 1;
        case GT_Q4_0:
        case GT_Q8_0: return 32;
        case GT_Q4_K:
        case GT_Q5_K:
        case GT_Q6_K:
        case GT_Q8_K: return 256;
    }
    return 0;
}

/* bytes of one row of n elements, 0 for an unknown type or a ragged row */
int64_t nmq_row_bytes(int type, int64_t n) {
    const int64_t bl = nmq_block_len(type);
    if (!bl || n % bl) return 0;
    switch (type) {
        case GT_F32: return 4 * n;
        case GT_Q4_0: return n / 32 * Q4_0_B;
        case GT_Q8_0: return n / 32 * Q8_0_B;
        case GT_Q4_K: return n / 256 * Q4_K_B;
        case GT_Q5_K: return n / 256 * Q5_K_B;
        case GT_Q6_K: return n / 256 * Q6_K_B;
        case GT_Q8_K: return n / 256 * Q8_K_B;
    }
    return 0;
}

/* 6-bit (scale, min) pair j of a K-quant superblock's 12 packed bytes:
 * pairs 0-3 sit in the low six bits of bytes j and j+4; pairs 4-7 take their
 * low four bits from byte j+4's nibbles and their top two from the spare high
 * bits of bytes j-4 and j. */
void nmq_scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Q6_K value (0..63) minus 32 of element l (0..31) in quarter r (0..3) of a
 * 128-element half: low nibble of ql[l] (r 0), ql[l+32] (r 1), high nibble of
 * ql[l] (r 2), ql[l+32] (r 3); the top two bits from qh[l] at bit 2r. */
static int q6_value(const uint8_t* ql, const uint8_t* qh, int l, int r) {
    const int nib = (r & 1) ? ql[l + 32] : ql[l];
    const int lo = (r & 2) ? (nib >> 4) : (nib & 0xF);
    return (lo | (((qh[l] >> (2 * r)) & 3) << 4)) - 32;
}

/* ---- dequantisation of one row (dequant_to_f32) ------------------------- */
int nmq_dequant_row(int type, const uint8_t* src, float* y, int64_t n) {
    switch (type) {
        case GT_F32:
            memcpy(y, src, (size_t)n * 4);
            return 0;
        case GT_Q8_0:
            for (int64_t b = 0; b < n / 32; ++b, src += Q8_0_B) {
                const float d = nmo_fp16_to_fp32(rd16(src));
                for (int j = 0; j < 32; ++j) *y++ = d * (int8_t)src[2 + j];
            }
            return 0;
        case GT_Q4_0:
            for (int64_t b = 0; b < n / 32; ++b, src += Q4_0_B, y += 32) {
                const float d = nmo_fp16_to_fp32(rd16(src));
                for (int j = 0; j < 16; ++j) {
                    y[j] = d * ((src[2 + j] & 0xF) - 8);
                    y[j + 16] = d * ((src[2 + j] >> 4) - 8);
                }
            }
            return 0;
        case GT_Q4_K:
        case GT_Q5_K: {
            const int five = type == GT_Q5_K;
            const int bytes = five ? Q5_K_B : Q4_K_B;
            for (int64_t b = 0; b < n / 256; ++b, src += bytes) {
                const float d = nmo_fp16_to_fp32(rd16(src)), mn = nmo_fp16_to_fp32(rd16(src + 2));
                const uint8_t* scales = src + 4;
                const uint8_t* qh = src + 16;                /* Q5_K only */
                const uint8_t* q = src + (five ? 48 : 16);
                for (int g = 0; g < 4; ++g, q += 32) {
                    uint8_t sc, m;
                    nmq_scale_min_k4(2 * g, scales, &sc, &m);
                    const float d1 = d * sc, m1 = mn * m;
                    nmq_scale_min_k4(2 * g + 1, scales, &sc, &m);
                    const float d2 = d * sc, m2 = mn * m;
                    for (int l = 0; l < 32; ++l) {
                        const int hi = five ? ((qh[l] >> (2 * g)) & 1) * 16 : 0;
                        *y++ = d1 * ((q[l] & 0xF) + hi) - m1;
                    }
                    for (int l = 0; l < 32; ++l) {
                        const int hi = five ? ((qh[l] >> (2 * g + 1)) & 1) * 16 : 0;
                        *y++ = d2 * ((q[l] >> 4) + hi) - m2;
                    }
                }
            }
            return 0;
        }
        case GT_Q6_K:
            for (int64_t b = 0; b < n / 256; ++b, src += Q6_K_B) {
                const float d = nmo_fp16_to_fp32(rd16(src + 208));
                for (int h = 0; h < 2; ++h, y += 128) {
                    const uint8_t* ql = src + 64 * h;
                    const uint8_t* qh = src + 128 + 32 * h;
                    const int8_t* sc = (const int8_t*)(src + 192 + 8 * h);
                    for (int l = 0; l < 32; ++l)
                        for (int r = 0; r < 4; ++r) y[l + 32 * r] = d * sc[l / 16 + 2 * r] * q6_value(ql, qh, l, r);
                }
            }
            return 0;
    }
    return 1;
}

/* ---- fp32-activation products (dot_block_*, summed per row) ------------- */
static float dot_q8_0_f32(const uint8_t* b, const float* x) {
    const float d = nmo_fp16_to_fp32(rd16(b));
    float s = 0;
    for (int i = 0; i < 32; ++i) s += (float)(int8_t)b[2 + i] * x[i];
    return d * s;
}
static float dot_q4_0_f32(const uint8_t* b, const float* x) {
    const float d = nmo_fp16_to_fp32(rd16(b));
    float s = 0;
    for (int j = 0; j < 16; ++j) {
        const int lo = (b[2 + j] & 0x0F) - 8, hi = (b[2 + j] >> 4) - 8;
        s += (float)lo * x[j] + (float)hi * x[j + 16];
    }
    return d * s;
}
static float dot_q45_K_f32(const uint8_t* b, const float* x, int five) {
    const float d = nmo_fp16_to_fp32(rd16(b)), mn = nmo_fp16_to_fp32(rd16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* q = b + (five ? 48 : 16);
    float acc = 0;
    for (int g = 0; g < 4; ++g, q += 32) {
        uint8_t sc, m;
        nmq_scale_min_k4(2 * g, scales, &sc, &m);
        const float d1 = d * sc, m1 = mn * m;
        nmq_scale_min_k4(2 * g + 1, scales, &sc, &m);
        const float d2 = d * sc, m2 = mn * m;
        for (int l = 0; l < 32; ++l) {
            const int hi = five ? ((qh[l] >> (2 * g)) & 1) * 16 : 0;
            acc += (d1 * (float)((q[l] & 0xF) + hi) - m1) * *x++;
        }
        for (int l = 0; l < 32; ++l) {
            const int hi = five ? ((qh[l] >> (2 * g + 1)) & 1) * 16 : 0;
            acc += (d2 * (float)((q[l] >> 4) + hi) - m2) * *x++;
        }
    }
    return acc;
}
static float dot_q6_K_f32(const uint8_t* b, const float* x) {
    const float d = nmo_fp16_to_fp32(rd16(b + 208));
    float acc = 0;
    for (int h = 0; h < 2; ++h, x += 128) {
        const uint8_t* ql = b + 64 * h;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t* sc = (const int8_t*)(b + 192 + 8 * h);
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            for (int r = 0; r < 4; ++r) acc += d * sc[is + 2 * r] * q6_value(ql, qh, l, r) * x[l + 32 * r];
        }
    }
    return acc;
}

/* one weight row (n elements) against fp32 activations x */
float nmq_dot_fp32(int type, int64_t n, const uint8_t* w, const float* x) {
    float acc = 0;
    switch (type) {
        case GT_F32: return nmo_dot((const float*)w, x, n);
        case GT_Q8_0:
            for (int64_t b = 0; b < n / 32; ++b) acc += dot_q8_0_f32(w + b * Q8_0_B, x + b * 32);
            break;
        case GT_Q4_0:
            for (int64_t b = 0; b < n / 32; ++b) acc += dot_q4_0_f32(w + b * Q4_0_B, x + b * 32);
            break;
        case GT_Q4_K:
            for (int64_t b = 0; b < n / 256; ++b) acc += dot_q45_K_f32(w + b * Q4_K_B, x + b * 256, 0);
            break;
        case GT_Q5_K:
            for (int64_t b = 0; b < n / 256; ++b) acc += dot_q45_K_f32(w + b * Q5_K_B, x + b * 256, 1);
            break;
        case GT_Q6_K:
            for (int64_t b = 0; b < n / 256; ++b) acc += dot_q6_K_f32(w + b * Q6_K_B, x + b * 256);
            break;
    }
    return acc;
}

/* ---- activation quantisers ----------------------------------------------- */
/* Q8_0 blocks of 32: d = amax / 127 kept as fp16, q = roundf(x * (1 / d)). */
void nmq_quantize_row_q8_0(const float* x, int64_t n, uint8_t* out) {
    for (int64_t b = 0; b < n / 32; ++b, x += 32, out += Q8_0_B) {
        float amax = 0;
        for (int j = 0; j < 32; ++j) {
            const float ax = fabsf(x[j]);
            amax = amax < ax ? ax : amax;
        }
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.f / d : 0.f;
        const uint16_t h = nmo_fp32_to_fp16(d);
        out[0] = (uint8_t)h;
        out[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 32; ++j) out[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
    }
}

/* round to nearest, ties to even, through the 1.5 * 2^23 bias */
static int nearest_int(float v) {
    float s = v + 12582912.f;
    int32_t i;
    memcpy(&i, &s, 4);
    return (i & 0x007fffff) - 0x00400000;
}

/* Q8_K blocks of 256: the signed value of largest magnitude (the first one on
 * ties) sets iscale = -127 / max; q = min(127, nearest(iscale * x)); d = 1 /
 * iscale in fp32; bsums = sums of the 16 groups of 16 quants. */
void nmq_quantize_row_q8_K(const float* x, int64_t n, uint8_t* out) {
    for (int64_t b = 0; b < n / 256; ++b, x += 256, out += Q8_K_B) {
        float max = 0, amax = 0;
        for (int j = 0; j < 256; ++j) {
            const float ax = fabsf(x[j]);
            if (ax > amax) {
                amax = ax;
                max = x[j];
            }
        }
        if (amax == 0.f) {
            memset(out, 0, Q8_K_B);
            continue;
        }
        const float iscale = -127.f / max;
        int8_t* qs = (int8_t*)(out + 4);
        for (int j = 0; j < 256; ++j) {
            const int v = nearest_int(iscale * x[j]);
            qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; ++g) {
            int sum = 0;
            for (int l = 0; l < 16; ++l) sum += qs[16 * g + l];
            const int16_t s16 = (int16_t)sum;
            memcpy(out + 260 + 2 * g, &s16, 2);
        }
        const float d = 1 / iscale;
        memcpy(out, &d, 4);
    }
}

/* ---- integer dots: one weight row against a quantised activation row ---- */
static float vdot_q8_0(int64_t n, const uint8_t* w, const uint8_t* a) {
    float sumf = 0;
    for (int64_t b = 0; b < n / 32; ++b, w += Q8_0_B, a += Q8_0_B) {
        int sumi = 0;
        for (int j = 0; j < 32; ++j) sumi += (int8_t)w[2 + j] * (int8_t)a[2 + j];
        sumf += sumi * (nmo_fp16_to_fp32(rd16(w)) * nmo_fp16_to_fp32(rd16(a)));
    }
    return sumf;
}
static float vdot_q4_0(int64_t n, const uint8_t* w, const uint8_t* a) {
    float sumf = 0;
    for (int64_t b = 0; b < n / 32; ++b, w += Q4_0_B, a += Q8_0_B) {
        int s0 = 0, s1 = 0;
        for (int j = 0; j < 16; ++j) {
            s0 += ((w[2 + j] & 0x0F) - 8) * (int8_t)a[2 + j];
            s1 += ((w[2 + j] >> 4) - 8) * (int8_t)a[2 + j + 16];
        }
        const int sumi = s0 + s1;
        sumf += sumi * nmo_fp16_to_fp32(rd16(w)) * nmo_fp16_to_fp32(rd16(a));
    }
    return sumf;
}
/* Q4_K and Q6_K share the per-superblock shape of the generic kernels: eight
 * int32 lanes accumulate scale * (q8 * q) over the superblock's groups of 8,
 * eight float lanes take d * lane per superblock, summed once at the end. */
static float vdot_q4_K(int64_t n, const uint8_t* w, const uint8_t* a) {
    float sums[8] = {0}, sumf = 0;
    for (int64_t b = 0; b < n / 256; ++b, w += Q4_K_B, a += Q8_K_B) {
        const int8_t* q8 = (const int8_t*)(a + 4);
        const uint8_t* q4 = w + 16;
        int8_t vals[256];
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l) {
                vals[64 * g + l] = (int8_t)(q4[32 * g + l] & 0xF);
                vals[64 * g + 32 + l] = (int8_t)(q4[32 * g + l] >> 4);
            }
        uint8_t sc[8], mins[8];
        for (int j = 0; j < 8; ++j) nmq_scale_min_k4(j, w + 4, &sc[j], &mins[j]);
        int sumi = 0;
        for (int j = 0; j < 16; ++j) sumi += rds16(a + 260 + 2 * j) * mins[j / 2];
        int32_t lane[8] = {0};
        for (int j = 0; j < 8; ++j)
            for (int rep = 0; rep < 4; ++rep)
                for (int l = 0; l < 8; ++l) {
                    const int e = 32 * j + 8 * rep + l;
                    lane[l] += sc[j] * (int16_t)(q8[e] * vals[e]);
                }
        const float d = nmo_fp16_to_fp32(rd16(w)) * rdf(a);
        for (int l = 0; l < 8; ++l) sums[l] += d * lane[l];
        const float dmin = nmo_fp16_to_fp32(rd16(w + 2)) * rdf(a);
        sumf -= dmin * sumi;
    }
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}
static float vdot_q6_K(int64_t n, const uint8_t* w, const uint8_t* a) {
    float sums[8] = {0}, sumf = 0;
    for (int64_t b = 0; b < n / 256; ++b, w += Q6_K_B, a += Q8_K_B) {
        const int8_t* q8 = (const int8_t*)(a + 4);
        const int8_t* sc = (const int8_t*)(w + 192);
        int8_t vals[256];
        for (int h = 0; h < 2; ++h)
            for (int l = 0; l < 32; ++l)
                for (int r = 0; r < 4; ++r) vals[128 * h + 32 * r + l] = (int8_t)q6_value(w + 64 * h, w + 128 + 32 * h, l, r);
        int32_t lane[8] = {0};
        for (int j = 0; j < 16; ++j)
            for (int rep = 0; rep < 2; ++rep)
                for (int l = 0; l < 8; ++l) {
                    const int e = 16 * j + 8 * rep + l;
                    lane[l] += sc[j] * (int16_t)(q8[e] * vals[e]);
                }
        const float d = nmo_fp16_to_fp32(rd16(w + 208)) * rdf(a);
        for (int l = 0; l < 8; ++l) sums[l] += d * lane[l];
    }
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}

/* Which weight types have an integer-activation kernel (Q5_K does not). */
int nmq_has_i8(int type) { return type == GT_Q8_0 || type == GT_Q4_0 || type == GT_Q4_K || type == GT_Q6_K; }
/* The activation block type a weight type's integer dot takes. */
int nmq_act_type(int type) { return (type == GT_Q4_K || type == GT_Q6_K) ? GT_Q8_K : GT_Q8_0; }

float nmq_vec_dot_i8(int type, int64_t n, const uint8_t* w, const uint8_t* act) {
    switch (type) {
        case GT_Q8_0: return vdot_q8_0(n, w, act);
        case GT_Q4_0: return vdot_q4_0(n, w, act);
        case GT_Q4_K: return vdot_q4_K(n, w, act);
        case GT_Q6_K: return vdot_q6_K(n, w, act);
    }
    return NAN;
}

/* ---- the products: y[rows][out] = x[rows][in] . W[out][in]^T ------------ */
typedef struct {
    int type, i8;
    int64_t in, out, rows, wrow, arow;
    const uint8_t* w;
    const float* x;
    const uint8_t* act;
    float* y;
    int threads, t;
} mm_job;

static void* mm_worker(void* p) {
    mm_job* J = (mm_job*)p;
    const int64_t lo = J->out * J->t / J->threads, hi = J->out * (J->t + 1) / J->threads;
    for (int64_t o = lo; o < hi; ++o) {
        const uint8_t* wr = J->w + o * J->wrow;
        for (int64_t r = 0; r < J->rows; ++r)
            J->y[r * J->out + o] = J->i8 ? nmq_vec_dot_i8(J->type, J->in, wr, J->act + r * J->arow)
                                         : nmq_dot_fp32(J->type, J->in, wr, J->x + r * J->in);
    }
    return NULL;
}

/* Weight::matmul (rows >= 1; matvec is rows == 1).  fp32_act selects the
 * NM_FP32_ACT path; Q5_K and F32 always take the fp32 path.  Returns 1 for an
 * unknown type or a row length that is not a whole number of blocks. */
int nmq_matmul(int type, int64_t in, int64_t out, const uint8_t* w, int64_t rows, const float* x, float* y, int fp32_act,
               int threads) {
    const int64_t wrow = nmq_row_bytes(type, in);
    if (!wrow || out <= 0 || rows < 0) return 1;
    if (rows == 0) return 0;
    mm_job J = {type, !fp32_act && nmq_has_i8(type), in, out, rows, wrow, 0, w, x, NULL, y, threads < 1 ? 1 : threads, 0};
    if (J.threads > 256) J.threads = 256;
    uint8_t* act = NULL;
    if (J.i8) {
        const int at = nmq_act_type(type);
        J.arow = nmq_row_bytes(at, in);
        act = (uint8_t*)malloc((size_t)(J.arow * rows));
        for (int64_t r = 0; r < rows; ++r) {
            if (at == GT_Q8_K) nmq_quantize_row_q8_K(x + r * in, in, act + r * J.arow);
            else nmq_quantize_row_q8_0(x + r * in, in, act + r * J.arow);
        }
        J.act = act;
    }
    mm_job jobs[256];
    pthread_t tid[256];
    for (int t = 0; t < J.threads; ++t) {
        jobs[t] = J;
        jobs[t].t = t;
        if (t) pthread_create(&tid[t], NULL, mm_worker, &jobs[t]);
    }
    mm_worker(&jobs[0]);
    for (int t = 1; t < J.threads; ++t) pthread_join(tid[t], NULL);
    free(act);
    return 0;
}
