/* TEST INFRASTRUCTURE ONLY -- the parity checker, never shipped or measured as the product.
 *
 * Plain-C restatement of the reference decode path (astrowar/MiniCPM5.cpp).  Compiled
 * without fast-math and without FP contraction, so each fp32 operation happens as written.
 * Integer block sums are exact by construction; where the reference's fp32 order is
 * known (the AVX2 eight-lane accumulators) it is reproduced on request.
 */
#include "mcpm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct { uint16_t d; int8_t qs[32]; } __attribute__((packed)) blk_q8_0;
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; } __attribute__((packed)) blk_q4_K;
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } __attribute__((packed)) blk_q6_K;
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } __attribute__((packed)) blk_q8_K;

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0");
_Static_assert(sizeof(blk_q4_K) == 144, "q4_K");
_Static_assert(sizeof(blk_q6_K) == 210, "q6_K");
_Static_assert(sizeof(blk_q8_K) == 292, "q8_K");

/* include/ops.h:14-31: exact IEEE half -> single, subnormals included. */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t exp = (h >> 10) & 0x1f;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* normalise the subnormal */
            int e = -1;
            do { mant <<= 1; e++; } while (!(mant & 0x400u));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
        }
    } else {
        bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* include/ops.h:77-97 (six-bit scale/min unpacking of block_q4_K.scales). */
void orc_q4k_scales_mins(const uint8_t q[12], uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; ++j) {
        sc[j] = q[j] & 63;
        mn[j] = q[j + 4] & 63;
        sc[j + 4] = (uint8_t)((q[j + 8] & 0x0f) | ((q[j] >> 6) << 4));
        mn[j + 4] = (uint8_t)((q[j + 8] >> 4) | ((q[j + 4] >> 6) << 4));
    }
}

/* Block maximum of |y| over 256 values as the reference build evaluates it: eight
 * lanes (lane k scans elements k, k+8, ... in order) with the SSE max rule
 * acc = (acc > e) ? acc : e, which returns e whenever either side is NaN; then the
 * horizontal steps m_i = hi_i > lo_i ? hi_i : lo_i (i < 4), n0 = m2 > m0 ? m2 : m0,
 * n1 = m3 > m1 ? m3 : m1, amax = n1 > n0 ? n1 : n0 (ops.cpp:705-709 / 737-742 as
 * compiled).  Identical to the plain maximum when no value is NaN. */
float orc_block_amax(const float* y) {
    float lane[8] = {0};
    for (int i = 0; i < 256; ++i) {
        const float e = fabsf(y[i]);
        lane[i & 7] = (lane[i & 7] > e) ? lane[i & 7] : e;
    }
    float m[4];
    for (int i = 0; i < 4; ++i) m[i] = (lane[i + 4] > lane[i]) ? lane[i + 4] : lane[i];
    const float n0 = (m[2] > m[0]) ? m[2] : m[0];
    const float n1 = (m[3] > m[1]) ? m[3] : m[1];
    return (n1 > n0) ? n1 : n0;
}

/* lround as the reference build inlines it (trunc(v + copysign(0.49999997, v)) through a
 * 64-bit conversion) followed by its clamp: NaN and |v| >= 2^63 give the conversion's
 * "indefinite" value and end at -127. */
static int32_t quant_away(float v) {
    const float a = v + copysignf(0.4999999701976776f, v);
    if (!(a < 9223372036854775808.0f && a >= -9223372036854775808.0f)) return -127;
    const float t = truncf(a);
    if (t >= 127.0f) return 127;
    if (t > -127.0f) return (int32_t)t;
    return -127;
}

/* _mm256_cvtps_epi32 (ties-to-even) + clamp to [-127, 127] (ops_avx2.cpp:118-121):
 * NaN and out-of-range values convert to INT_MIN and clamp to -127. */
static int32_t quant_even(float v) {
    if (!(v < 2147483648.0f && v >= -2147483648.0f)) return -127;
    const float t = rintf(v);
    if (t >= 127.0f) return 127;
    if (t <= -127.0f) return -127;
    return (int32_t)t;
}

/* One 256-block of fp32 -> Q8_K.  Restates quantize_row_q8_K_avx2 (ops_avx2.cpp:85-144,
 * ties-to-even) and the lround quantisers of ops.cpp:702-722 / 744-764 (ties-away).
 * A block whose amax is 0 or NaN is stored as zeros (the build's amax == 0 test is an
 * unordered compare).  d = amax * (1/127): the build multiplies by the reciprocal. */
static void quant_block(const float* x, blk_q8_K* dst, int rounding, int recip_d) {
    const float amax = orc_block_amax(x);
    if (amax == 0.0f || amax != amax) {
        memset(dst, 0, sizeof(*dst));
        return;
    }
    dst->d = recip_d ? amax * (1.0f / 127.0f) : amax / 127.0f;
    const float mul = 127.0f / amax;
    for (int g = 0; g < 16; ++g) {
        int32_t s = 0;
        for (int i = 0; i < 16; ++i) {
            const float v = x[16 * g + i] * mul;
            const int32_t q = rounding == ORC_ROUND_AWAY ? quant_away(v) : quant_even(v);
            dst->qs[16 * g + i] = (int8_t)q;
            s += q;
        }
        dst->bsums[g] = (int16_t)s;
    }
}

void orc_quantize_q8k(const float* x, int n, void* y, int rounding, int recip_d) {
    blk_q8_K* out = (blk_q8_K*)y;
    for (int b = 0; b < n / 256; ++b) quant_block(x + 256 * b, out + b, rounding, recip_d);
}

/* dot_row_q4_K_q8_K_scalar (ops_scalar_optimized.cpp:139-225), integer part of one block. */
void orc_q4k_block_sums(const void* wblk, const void* xblk, int32_t* isum, int32_t* minsum) {
    const blk_q4_K* w = (const blk_q4_K*)wblk;
    const blk_q8_K* a = (const blk_q8_K*)xblk;
    uint8_t sc[8], mn[8];
    orc_q4k_scales_mins(w->scales, sc, mn);
    int32_t s = 0;
    for (int j = 0; j < 4; ++j) {
        int32_t lo = 0, hi = 0;
        for (int i = 0; i < 32; ++i) {
            lo += (w->qs[32 * j + i] & 15) * a->qs[64 * j + i];
            hi += (w->qs[32 * j + i] >> 4) * a->qs[64 * j + 32 + i];
        }
        s += sc[2 * j] * lo + sc[2 * j + 1] * hi;
    }
    int32_t m = 0;
    for (int g = 0; g < 8; ++g) m += mn[g] * (a->bsums[2 * g] + a->bsums[2 * g + 1]);
    *isum = s;
    *minsum = m;
}

/* Q6_K element q (unsigned, 0..63) for half h, quarter k, lane l (include/ops.h:51-56 layout). */
static inline int q6_val(const blk_q6_K* w, int h, int k, int l) {
    const uint8_t* ql = w->ql + 64 * h;
    const uint8_t qh = w->qh[32 * h + l];
    int lo = (k & 1) ? ql[l + 32] : ql[l];
    lo = (k & 2) ? (lo >> 4) : (lo & 15);
    return lo | (((qh >> (2 * k)) & 3) << 4);
}

/* dot_row_q6_K_q8_K_scalar (ops_scalar_optimized.cpp:312-404), integer part of one block. */
void orc_q6k_block_sums(const void* wblk, const void* xblk, int32_t* isum, int32_t* offset) {
    const blk_q6_K* w = (const blk_q6_K*)wblk;
    const blk_q8_K* a = (const blk_q8_K*)xblk;
    int32_t s = 0;
    for (int h = 0; h < 2; ++h)
        for (int k = 0; k < 4; ++k)
            for (int l = 0; l < 32; ++l)
                s += w->scales[8 * h + 2 * k + (l >= 16)] * q6_val(w, h, k, l) * a->qs[128 * h + 32 * k + l];
    int32_t o = 0;
    for (int g = 0; g < 16; ++g) o += w->scales[g] * a->bsums[g];
    *isum = s;
    *offset = 32 * o;
}

void orc_blocksums(int type, const void* w, const void* xq, int rows, int cols, int32_t* isum, int32_t* aux) {
    const int nb = cols / 256;
    const blk_q8_K* x = (const blk_q8_K*)xq;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < nb; ++b) {
            size_t i = (size_t)r * nb + b;
            if (type == ORC_Q4_K)
                orc_q4k_block_sums((const blk_q4_K*)w + i, x + b, isum + i, aux + i);
            else
                orc_q6k_block_sums((const blk_q6_K*)w + i, x + b, isum + i, aux + i);
        }
    }
}

/* Horizontal sum of eight lanes in the order of hsum_f32_8 (ops_avx2.cpp:43-48). */
static float hsum8(const float a[8]) {
    float t0 = a[0] + a[4], t1 = a[1] + a[5], t2 = a[2] + a[6], t3 = a[3] + a[7];
    float u0 = t0 + t2, u1 = t1 + t3;
    return u0 + u1;
}

static float dot_q4k_row(const blk_q4_K* w, const blk_q8_K* a, int nb, int order, int fused_min) {
    if (order == ORC_ORDER_SCALAR) {
        float result = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int32_t isum, minsum;
            orc_q4k_block_sums(w + b, a + b, &isum, &minsum);
            const float wd = orc_fp16_to_fp32(w[b].d), wm = orc_fp16_to_fp32(w[b].dmin);
            result += a[b].d * (wd * (float)isum - wm * (float)minsum);
        }
        return result;
    }
    if (order == ORC_ORDER_BATCH) {   /* groups of 4 blocks, one fma per block (k_b_gemm_tc) */
        float row = 0.0f;
        for (int g0 = 0; g0 < nb; g0 += 4) {
            float acc = 0.0f, accm = 0.0f;
            for (int b = g0; b < g0 + 4 && b < nb; ++b) {
                int32_t isum, minsum;
                orc_q4k_block_sums(w + b, a + b, &isum, &minsum);
                acc = fmaf(a[b].d * orc_fp16_to_fp32(w[b].d), (float)isum, acc);
                accm = fmaf(-(a[b].d * orc_fp16_to_fp32(w[b].dmin)), (float)minsum, accm);
            }
            const float g = acc + accm;
            row = g0 == 0 ? g : row + g;
        }
        return row;
    }
    /* AVX2 order (ops_avx2.cpp:153-196): lane k holds bytes 4k..4k+3 of each 32-byte qs group. */
    float acc[8] = {0};
    float acc_min = 0.0f;
    for (int b = 0; b < nb; ++b) {
        uint8_t sc[8], mn[8];
        orc_q4k_scales_mins(w[b].scales, sc, mn);
        int32_t lane[8] = {0};
        for (int j = 0; j < 4; ++j)
            for (int k = 0; k < 8; ++k) {
                int32_t lo = 0, hi = 0;
                for (int i = 4 * k; i < 4 * k + 4; ++i) {
                    lo += (w[b].qs[32 * j + i] & 15) * a[b].qs[64 * j + i];
                    hi += (w[b].qs[32 * j + i] >> 4) * a[b].qs[64 * j + 32 + i];
                }
                lane[k] += sc[2 * j] * lo + sc[2 * j + 1] * hi;
            }
        const float ds = a[b].d * orc_fp16_to_fp32(w[b].d);
        for (int k = 0; k < 8; ++k) acc[k] = fmaf(ds, (float)lane[k], acc[k]);
        int32_t minsum = 0;
        for (int g = 0; g < 8; ++g) minsum += mn[g] * (a[b].bsums[2 * g] + a[b].bsums[2 * g + 1]);
        const float dm = a[b].d * orc_fp16_to_fp32(w[b].dmin);
        if (fused_min)
            acc_min = fmaf(-dm, (float)minsum, acc_min);
        else
            acc_min -= dm * (float)minsum;
    }
    return hsum8(acc) + acc_min;
}

static float dot_q6k_row(const blk_q6_K* w, const blk_q8_K* a, int nb, int order) {
    if (order == ORC_ORDER_SCALAR) {
        float result = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int32_t isum, off;
            orc_q6k_block_sums(w + b, a + b, &isum, &off);
            const float d = orc_fp16_to_fp32(w[b].d) * a[b].d;
            result += d * (float)(isum - off);
        }
        return result;
    }
    if (order == ORC_ORDER_BATCH) {   /* groups of 4 blocks, one fma per block (k_b_gemm_tc) */
        float row = 0.0f;
        for (int g0 = 0; g0 < nb; g0 += 4) {
            float acc = 0.0f;
            for (int b = g0; b < g0 + 4 && b < nb; ++b) {
                int32_t isum, off;
                orc_q6k_block_sums(w + b, a + b, &isum, &off);
                acc = fmaf(a[b].d * orc_fp16_to_fp32(w[b].d), (float)(isum - off), acc);
            }
            row = g0 == 0 ? acc : row + acc;
        }
        return row;
    }
    /* AVX2 order (ops_avx2.cpp:201-276): lane k holds l in [4k, 4k+4) of every quarter. */
    float acc[8] = {0};
    for (int b = 0; b < nb; ++b) {
        int32_t lane[8];
        for (int k = 0; k < 8; ++k)
            lane[k] = -32 * (a[b].bsums[2 * k] * w[b].scales[2 * k] + a[b].bsums[2 * k + 1] * w[b].scales[2 * k + 1]);
        for (int h = 0; h < 2; ++h)
            for (int kk = 0; kk < 4; ++kk)
                for (int l = 0; l < 32; ++l)
                    lane[l / 4] += w[b].scales[8 * h + 2 * kk + (l >= 16)] * q6_val(&w[b], h, kk, l) *
                                   a[b].qs[128 * h + 32 * kk + l];
        const float ds = a[b].d * orc_fp16_to_fp32(w[b].d);
        for (int k = 0; k < 8; ++k) acc[k] = fmaf(ds, (float)lane[k], acc[k]);
    }
    return hsum8(acc);
}

void orc_gemv_q4k_q8k(const void* w, const void* xq, float* y, int rows, int cols, int order, int fused_min) {
    const int nb = cols / 256;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        y[r] = dot_q4k_row((const blk_q4_K*)w + (size_t)r * nb, (const blk_q8_K*)xq, nb, order, fused_min);
}

void orc_gemv_q6k_q8k(const void* w, const void* xq, float* y, int rows, int cols, int order) {
    const int nb = cols / 256;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        y[r] = dot_q6k_row((const blk_q6_K*)w + (size_t)r * nb, (const blk_q8_K*)xq, nb, order);
}

/* gemv_q8_0 (ops.cpp:58-79). */
/* gemv_q8_0 (src/ops/ops.cpp:58-79) as the reference build evaluates it (-O3 -ffast-math
 * -mavx2 -mfma; verified bit for bit against that build): per 32-block, eight fp32 lanes
 * k: A_k = fma(q[k], x[k], q[k+8]*x[k+8]), B_k = fma(q[k+16], x[k+16], q[k+24]*x[k+24]),
 * v_k = B_k + A_k; c_k = v_{k+4} + v_k, e_k = c_{k+2} + c_k, local = e_1 + e_0;
 * row = fma(fp16(d), local, row) over the blocks in order. */
void orc_gemv_q8_0(const void* w, const float* x, float* y, int rows, int cols) {
    const int nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const blk_q8_0* row = (const blk_q8_0*)w + (size_t)r * nb;
        float sum = 0.0f;
        for (int b = 0; b < nb; ++b) {
            const int8_t* q = row[b].qs;
            const float* xb = x + 32 * b;
            float v[8];
            for (int k = 0; k < 8; ++k) {
                const float a = fmaf((float)q[k], xb[k], (float)q[k + 8] * xb[k + 8]);
                const float bb = fmaf((float)q[k + 16], xb[k + 16], (float)q[k + 24] * xb[k + 24]);
                v[k] = bb + a;
            }
            float c[4], e[2];
            for (int k = 0; k < 4; ++k) c[k] = v[k + 4] + v[k];
            for (int k = 0; k < 2; ++k) e[k] = c[k + 2] + c[k];
            const float local = e[1] + e[0];
            sum = fmaf(orc_fp16_to_fp32(row[b].d), local, sum);
        }
        y[r] = sum;
    }
}

/* ------------------------------------------------------------------------------------
 * Canonical numerics.  Where the reference's fp32 order depends on the OpenMP thread
 * count or on CPU-specific estimate instructions (rsqrtss/rcpps, libmvec), this project
 * fixes one order that a GPU evaluates efficiently; the CUDA kernels follow it bit for
 * bit.  Each function states the order.
 * ------------------------------------------------------------------------------------ */

/* Butterfly over 32 lanes: for s = 16, 8, 4, 2, 1: v[l] = v[l] + v[l ^ s]. */
static void butterfly32(float* v) {
    for (int s = 16; s >= 1; s >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ s];
        memcpy(v, t, sizeof(t));
    }
}

/* sum of squares of n = 256*m values: 256 lanes, lane l = fma chain over x[l + 256 i];
 * a 32-lane butterfly inside each of the 8 warps; warps combined as
 * ((w0+w1)+(w2+w3)) + ((w4+w5)+(w6+w7)). */
float orc_sumsq(const float* x, int n) {
    float lane[256];
    for (int l = 0; l < 256; ++l) {
        float a = 0.0f;
        for (int i = l; i < n; i += 256) a = fmaf(x[i], x[i], a);
        lane[l] = a;
    }
    float w[8];
    for (int g = 0; g < 8; ++g) {
        butterfly32(lane + 32 * g);
        w[g] = lane[32 * g];
    }
    return ((w[0] + w[1]) + (w[2] + w[3])) + ((w[4] + w[5]) + (w[6] + w[7]));
}

/* rms = 1/sqrt(sum/n + eps), IEEE sqrt and division. */
float orc_rms_scale(const float* x, int n, float eps) {
    return 1.0f / sqrtf(orc_sumsq(x, n) / (float)n + eps);
}

/* exp(x): x = k ln2 + r (k = rint(x log2 e), two-constant Cody-Waite reduction), e^r by
 * the degree-7 Taylor polynomial in Horner form (fused multiply-adds), then 2^k applied
 * as two exact power-of-two factors so the only rounding of the scaling is the last one. */
float orc_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float kf = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-kf, 0.693145751953125f, x);
    r = fmaf(-kf, 1.428606765330187045e-06f, r);
    float p = 1.98412701138295233250e-04f;            /* 1/5040 */
    p = fmaf(p, r, 1.38888892251998186111e-03f);      /* 1/720  */
    p = fmaf(p, r, 8.33333376795053482056e-03f);      /* 1/120  */
    p = fmaf(p, r, 4.16666679084300994873e-02f);      /* 1/24   */
    p = fmaf(p, r, 1.66666671633720397949e-01f);      /* 1/6    */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = (int)kf;
    const int k1 = k / 2, k2 = k - k1;
    float s1, s2;
    uint32_t b1 = (uint32_t)(k1 + 127) << 23, b2 = (uint32_t)(k2 + 127) << 23;
    memcpy(&s1, &b1, 4);
    memcpy(&s2, &b2, 4);
    return (p * s1) * s2;
}

/* rmsnorm_and_quantize_q8k (ops.cpp:676-723): y = (x*w)*rms (the reference build's
 * evaluation order), lround quantisation, d = amax*(1/127). */
void orc_rmsnorm_q8k(const float* x, const float* w, int n, float eps, void* out) {
    const float rms = orc_rms_scale(x, n, eps);
    float* y = (float*)malloc(sizeof(float) * n);
    for (int i = 0; i < n; ++i) y[i] = (x[i] * w[i]) * rms;
    orc_quantize_q8k(y, n, out, ORC_ROUND_AWAY, 1);
    free(y);
}

/* rmsnorm (ops.cpp:468-481), same order. */
void orc_rmsnorm(const float* x, const float* w, int n, float eps, float* out) {
    const float rms = orc_rms_scale(x, n, eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * w[i]) * rms;
}

/* silu(g)*u = (g * (1/(1+exp(-g)))) * u: the reference build forms the reciprocal with
 * an rcpps estimate and one Newton step, then multiplies (ops.cpp:447-449, 738-741).
 * The Newton step turns 1/inf into 0*inf = NaN, so when exp(-g) overflows the build's
 * silu is NaN; this restatement keeps that, with an IEEE reciprocal otherwise. */
float orc_silu_mul(float g, float u) {
    const float y = 1.0f + orc_expf(-g);
    const float r = isinf(y) ? NAN : 1.0f / y;
    return (g * r) * u;
}

/* swiglu_and_quantize_q8k (ops.cpp:725-765). */
void orc_swiglu_q8k(const float* g, const float* u, int n, void* out) {
    float* y = (float*)malloc(sizeof(float) * n);
    for (int i = 0; i < n; ++i) y[i] = orc_silu_mul(g[i], u[i]);
    orc_quantize_q8k(y, n, out, ORC_ROUND_AWAY, 1);
    free(y);
}

/* RoPE factor table for one position: theta_i = base^(-(i * (1/head_dim))) (the reference
 * build evaluates 1/pow(base, i/head_dim) as pow(base, -(i*(1/head_dim)))), angle =
 * theta*pos, c/s from the C library.  cs[2*(i/2)] = cos, cs[2*(i/2)+1] = sin. */
void orc_rope_row(int pos, int head_dim, float base, float* cs) {
    const float inv = 1.0f / (float)head_dim;
    for (int i = 0; i < head_dim; i += 2) {
        const float theta = powf(base, -((float)i * inv));
        const float ang = theta * (float)pos;
        cs[i] = cosf(ang);
        cs[i + 1] = sinf(ang);
    }
}

/* apply_rope (ops.cpp:502-516): interleaved pairs (2i, 2i+1) of each head, rotated as
 * v0' = fma(c, v0, -(s*v1)), v1' = fma(s, v0, c*v1) (the reference build's contraction). */
void orc_rope(float* v, int n_heads, int head_dim, int pos, float base) {
    float cs[512];
    orc_rope_row(pos, head_dim, base, cs);
    for (int h = 0; h < n_heads; ++h)
        for (int i = 0; i < head_dim; i += 2) {
            float* p = v + h * head_dim + i;
            const float c = cs[i], s = cs[i + 1], v0 = p[0], v1 = p[1];
            p[0] = fmaf(c, v0, -(s * v1));
            p[1] = fmaf(s, v0, c * v1);
        }
}

/* Attention chunk length for a context of n positions: 32 * ceil(n / 2048), so at most 64
 * chunks per head. */
int orc_attn_chunk(int n) { return 32 * ((n + 2047) / 2048); }

/* q.k over head_dim = 128: eight lanes, lane j = fma chain over dims 4j+32i+c
 * (i = 0..3, c = 0..3), then the butterfly v[j] += v[j^4], v[j] += v[j^2], v[j] += v[j^1]. */
static float dot128(const float* q, const float* k) {
    float p[8];
    for (int j = 0; j < 8; ++j) {
        float a = 0.0f;
        for (int i = 0; i < 4; ++i)
            for (int c = 0; c < 4; ++c) a = fmaf(q[4 * j + 32 * i + c], k[4 * j + 32 * i + c], a);
        p[j] = a;
    }
    for (int s = 4; s >= 1; s >>= 1) {
        float t[8];
        for (int j = 0; j < 8; ++j) t[j] = p[j] + p[j ^ s];
        memcpy(p, t, sizeof(t));
    }
    return p[0];
}

/* execute_attention (ops.cpp:537-628): appends k, v at pos, then softmax(q.k/sqrt(d)).V
 * per head over positions 0..pos in chunks of orc_attn_chunk(pos+1):
 *   per chunk: m = max s, p_t = exp(s_t - m), l = sum p_t (32 lane sums over
 *              t = lane mod 32 in position order, then a 32-lane butterfly),
 *              o[d] = fma chain over t of p_t*v_t[d];
 *   combine:   M = max m_c, w_c = exp(m_c - M), L = fma chain of w_c*l_c,
 *              O[d] = fma chain of w_c*o_c[d] (chunk order), out = O * (1/L). */
int orc_attention(float* out, const float* q, const float* k, const float* v, float* kc, float* vc,
                  int pos, int max_seq, int n_head, int n_kv, int head_dim) {
    if (pos >= max_seq || pos < 0 || head_dim != 128) return -1;
    const int kvd = n_kv * head_dim, n = pos + 1;
    memcpy(kc + (size_t)pos * kvd, k, sizeof(float) * kvd);
    memcpy(vc + (size_t)pos * kvd, v, sizeof(float) * kvd);
    const float scale = 1.0f / sqrtf((float)head_dim);
    const int group = n_head / n_kv, P = orc_attn_chunk(n), C = (n + P - 1) / P;
    float* cm = (float*)malloc(sizeof(float) * C);
    float* cl = (float*)malloc(sizeof(float) * C);
    float* co = (float*)malloc(sizeof(float) * C * 128);
    float* pt = (float*)malloc(sizeof(float) * P);
    for (int h = 0; h < n_head; ++h) {
        const int g = h / group;
        const float* qh = q + h * head_dim;
        for (int c = 0; c < C; ++c) {
            const int t0 = c * P, t1 = (t0 + P < n) ? t0 + P : n;
            float m = -INFINITY;
            for (int t = t0; t < t1; ++t) {
                pt[t - t0] = dot128(qh, kc + (size_t)t * kvd + g * head_dim) * scale;
                if (pt[t - t0] > m) m = pt[t - t0];
            }
            for (int t = t0; t < t1; ++t) pt[t - t0] = orc_expf(pt[t - t0] - m);
            /* chunk sum: 32 lane sums over positions t = lane (mod 32) in order, then a
               butterfly over lane bits 4..0 (every lane ends with the same value) */
            float lane_sum[32];
            for (int ln = 0; ln < 32; ++ln) {
                float a = 0.0f;
                for (int t = t0 + ln; t < t1; t += 32) a = a + pt[t - t0];
                lane_sum[ln] = a;
            }
            for (int o = 16; o >= 1; o >>= 1) {
                float nx[32];
                for (int ln = 0; ln < 32; ++ln) nx[ln] = lane_sum[ln] + lane_sum[ln ^ o];
                memcpy(lane_sum, nx, sizeof(nx));
            }
            const float l = lane_sum[0];
            for (int d = 0; d < 128; ++d) {
                float o = 0.0f;
                for (int t = t0; t < t1; ++t) o = fmaf(pt[t - t0], vc[(size_t)t * kvd + g * head_dim + d], o);
                co[c * 128 + d] = o;
            }
            cm[c] = m;
            cl[c] = l;
        }
        float M = cm[0];
        for (int c = 1; c < C; ++c)
            if (cm[c] > M) M = cm[c];
        float L = 0.0f;
        for (int c = 0; c < C; ++c) L = fmaf(orc_expf(cm[c] - M), cl[c], L);
        const float inv = 1.0f / L;
        for (int d = 0; d < 128; ++d) {
            float O = 0.0f;
            for (int c = 0; c < C; ++c) O = fmaf(orc_expf(cm[c] - M), co[c * 128 + d], O);
            out[h * head_dim + d] = O * inv;
        }
    }
    free(cm); free(cl); free(co); free(pt);
    return 0;
}

void orc_embedding(const void* w, int type, int token, int dim, float* out) {
    if (type == ORC_Q8_0) {
        const blk_q8_0* row = (const blk_q8_0*)w + (size_t)token * (dim / 32);
        for (int b = 0; b < dim / 32; ++b) {
            const float d = orc_fp16_to_fp32(row[b].d);
            for (int i = 0; i < 32; ++i) out[32 * b + i] = d * (float)row[b].qs[i];
        }
        return;
    }
    const blk_q4_K* row = (const blk_q4_K*)w + (size_t)token * (dim / 256);
    for (int b = 0; b < dim / 256; ++b) {
        uint8_t sc[8], mn[8];
        orc_q4k_scales_mins(row[b].scales, sc, mn);
        const float d = orc_fp16_to_fp32(row[b].d), dmin = orc_fp16_to_fp32(row[b].dmin);
        for (int j = 0; j < 4; ++j) {
            const float d1 = d * (float)sc[2 * j], m1 = dmin * (float)mn[2 * j];
            const float d2 = d * (float)sc[2 * j + 1], m2 = dmin * (float)mn[2 * j + 1];
            for (int l = 0; l < 32; ++l) {
                const uint8_t q = row[b].qs[32 * j + l];
                out[256 * b + 64 * j + l] = d1 * (float)(q & 15) - m1;
                out[256 * b + 64 * j + 32 + l] = d2 * (float)(q >> 4) - m2;
            }
        }
    }
}

/* ---------------- whole-model forward (src/model.cpp:142-242) ---------------- */
enum { T_K = 0, T_ANORM, T_O, T_Q, T_V, T_DOWN, T_GATE, T_FNORM, T_UP };

struct orc_state {
    orc_model_desc d;
    int max_seq;
    float *x, *xn, *q, *k, *v, *att, *o, *gate, *up, *h, *ffo, *logits;
    float **kc, **vc;
    blk_q8_K *xq, *hq;
    int order;   /* ORC_ORDER_AVX2 or ORC_ORDER_BATCH for the K-quant projections */
};

void orc_set_order(orc_state* s, int order) { s->order = order; }

orc_state* orc_create(const orc_model_desc* d, int max_seq) {
    orc_state* s = (orc_state*)calloc(1, sizeof(orc_state));
    s->d = *d;
    s->max_seq = max_seq;
    s->order = ORC_ORDER_AVX2;
    const int E = d->n_embd, F = d->n_ff, kvd = d->n_head_kv * (E / d->n_head);
    s->x = calloc(E, 4); s->xn = calloc(E, 4); s->q = calloc(E, 4);
    s->k = calloc(kvd, 4); s->v = calloc(kvd, 4); s->att = calloc(E, 4); s->o = calloc(E, 4);
    s->gate = calloc(F, 4); s->up = calloc(F, 4); s->h = calloc(F, 4); s->ffo = calloc(E, 4);
    s->logits = calloc(d->n_vocab, 4);
    s->xq = calloc(E / 256, sizeof(blk_q8_K));
    s->hq = calloc(F / 256, sizeof(blk_q8_K));
    s->kc = calloc(d->n_layer, sizeof(float*));
    s->vc = calloc(d->n_layer, sizeof(float*));
    for (int l = 0; l < d->n_layer; ++l) {
        s->kc[l] = calloc((size_t)max_seq * kvd, 4);
        s->vc[l] = calloc((size_t)max_seq * kvd, 4);
    }
    return s;
}

void orc_destroy(orc_state* s) {
    if (!s) return;
    for (int l = 0; l < s->d.n_layer; ++l) { free(s->kc[l]); free(s->vc[l]); }
    free(s->kc); free(s->vc);
    free(s->x); free(s->xn); free(s->q); free(s->k); free(s->v); free(s->att); free(s->o);
    free(s->gate); free(s->up); free(s->h); free(s->ffo); free(s->logits); free(s->xq); free(s->hq);
    free(s);
}

/* matmul_q8k / matmul (ops.cpp:264-349): K-quant tensors take the Q8_K activation,
 * Q8_0 tensors the fp32 one. */
static void project(const orc_state* s, uint64_t off, int type, int rows, int cols,
                    const void* xq, const float* xf, float* y) {
    const uint8_t* w = s->d.base + off;
    if (type == ORC_Q4_K)
        orc_gemv_q4k_q8k(w, xq, y, rows, cols, s->order, 1);
    else if (type == ORC_Q6_K)
        orc_gemv_q6k_q8k(w, xq, y, rows, cols, s->order);
    else
        orc_gemv_q8_0(w, xf, y, rows, cols);
}

int orc_forward(orc_state* s, int token, int pos, float* logits) {
    const orc_model_desc* d = &s->d;
    const int E = d->n_embd, F = d->n_ff, hd = E / d->n_head, kvd = d->n_head_kv * hd;
    if (pos >= s->max_seq || pos < 0 || token < 0 || token >= d->n_vocab) return -1;
    orc_embedding(d->base + d->tok_embd, d->tok_embd_type, token, E, s->x);
    for (int l = 0; l < d->n_layer; ++l) {
        const uint64_t* t = d->layer[l];
        const int* ty = d->layer_type[l];
        const float* anorm = (const float*)(d->base + t[T_ANORM]);
        const float* fnorm = (const float*)(d->base + t[T_FNORM]);
        /* attention block */
        if (ty[T_Q] == ORC_Q8_0)
            orc_rmsnorm(s->x, anorm, E, d->eps, s->xn);
        else
            orc_rmsnorm_q8k(s->x, anorm, E, d->eps, s->xq);
        project(s, t[T_Q], ty[T_Q], E, E, s->xq, s->xn, s->q);
        project(s, t[T_K], ty[T_K], kvd, E, s->xq, s->xn, s->k);
        project(s, t[T_V], ty[T_V], kvd, E, s->xq, s->xn, s->v);
        orc_rope(s->q, d->n_head, hd, pos, d->rope_base);
        orc_rope(s->k, d->n_head_kv, hd, pos, d->rope_base);
        if (d->kv_f16)
            for (int i = 0; i < kvd; ++i) {   /* the cache holds half-precision K/V rows */
                s->k[i] = (float)(_Float16)s->k[i];
                s->v[i] = (float)(_Float16)s->v[i];
            }
        orc_attention(s->att, s->q, s->k, s->v, s->kc[l], s->vc[l], pos, s->max_seq, d->n_head, d->n_head_kv, hd);
        if (ty[T_O] != ORC_Q8_0) orc_quantize_q8k(s->att, E, s->xq, ORC_ROUND_EVEN, 1);
        project(s, t[T_O], ty[T_O], E, E, s->xq, s->att, s->o);
        for (int i = 0; i < E; ++i) s->x[i] = s->x[i] + s->o[i];
        /* feed-forward block */
        if (ty[T_GATE] == ORC_Q8_0)
            orc_rmsnorm(s->x, fnorm, E, d->eps, s->xn);
        else
            orc_rmsnorm_q8k(s->x, fnorm, E, d->eps, s->xq);
        project(s, t[T_GATE], ty[T_GATE], F, E, s->xq, s->xn, s->gate);
        project(s, t[T_UP], ty[T_UP], F, E, s->xq, s->xn, s->up);
        if (ty[T_DOWN] == ORC_Q8_0) {
            for (int i = 0; i < F; ++i) s->h[i] = orc_silu_mul(s->gate[i], s->up[i]);
        } else {
            orc_swiglu_q8k(s->gate, s->up, F, s->hq);
        }
        project(s, t[T_DOWN], ty[T_DOWN], E, F, s->hq, s->h, s->ffo);
        for (int i = 0; i < E; ++i) s->x[i] = s->x[i] + s->ffo[i];
    }
    orc_rmsnorm(s->x, (const float*)(d->base + d->out_norm), E, d->eps, s->xn);
    if (d->output_type != ORC_Q8_0) orc_quantize_q8k(s->xn, E, s->xq, ORC_ROUND_EVEN, 1);
    project(s, d->output, d->output_type, d->n_vocab, E, s->xq, s->xn, s->logits);
    int best = 0;
    for (int i = 1; i < d->n_vocab; ++i)
        if (s->logits[i] > s->logits[best]) best = i;
    if (logits) memcpy(logits, s->logits, sizeof(float) * d->n_vocab);
    return best;
}

void orc_get_x(const orc_state* s, float* x) { memcpy(x, s->x, sizeof(float) * s->d.n_embd); }

void orc_get_kv(const orc_state* s, int layer, float* k, float* v, int n_pos) {
    const int kvd = s->d.n_head_kv * (s->d.n_embd / s->d.n_head);
    memcpy(k, s->kc[layer], sizeof(float) * (size_t)n_pos * kvd);
    memcpy(v, s->vc[layer], sizeof(float) * (size_t)n_pos * kvd);
}

void orc_set_kv(orc_state* s, int layer, const float* k, const float* v, int n_pos) {
    const int kvd = s->d.n_head_kv * (s->d.n_embd / s->d.n_head);
    memcpy(s->kc[layer], k, sizeof(float) * (size_t)n_pos * kvd);
    memcpy(s->vc[layer], v, sizeof(float) * (size_t)n_pos * kvd);
}

/* ---------------------------------------------------------------- top-p sampler */
/* Blocked running sums over a[0..m): 1024 ranges of L = ceil(m/1024) positions; range c is
 * summed sequentially from 0 (T_c), the prefix E_c of the T's is sequential, and the running
 * value at position k of range c is E_c + a[cL] + ... + a[k], added in order. */
static void blocked_running(const float* a, int m, float* run) {
    const int L = (m + 1023) / 1024;
    float E = 0.0f;
    for (int c = 0; c < 1024 && c * L < m; ++c) {
        const int b = c * L, e = b + L < m ? b + L : m;
        float T = 0.0f;
        for (int k = b; k < e; ++k) T += a[k];
        float cur = E;
        for (int k = b; k < e; ++k) {
            cur += a[k];
            run[k] = cur;
        }
        E += T;
    }
}

typedef struct {
    float p;
    int i;
} orc_pi;

static int cmp_pi(const void* x, const void* y) {   /* p descending, index ascending */
    const orc_pi* a = (const orc_pi*)x;
    const orc_pi* b = (const orc_pi*)y;
    if (a->p > b->p) return -1;
    if (a->p < b->p) return 1;
    return (a->i > b->i) - (a->i < b->i);
}

int orc_sample_top_p(const float* logits, int n, float temperature, float top_p, float r, int* kept) {
    const float inv_temp = temperature > 0.0f ? 1.0f / temperature : 1.0f;
    const int apply = temperature != 1.0f && temperature > 0.0f;
    float* v = (float*)malloc(sizeof(float) * n);
    float* run = (float*)malloc(sizeof(float) * n);
    orc_pi* pi = (orc_pi*)malloc(sizeof(orc_pi) * n);
    float mx = -1e9f;
    for (int i = 0; i < n; ++i) {
        v[i] = apply ? logits[i] * inv_temp : logits[i];
        if (v[i] > mx) mx = v[i];
    }
    for (int i = 0; i < n; ++i) v[i] = orc_expf(v[i] - mx);   /* e_i */
    blocked_running(v, n, run);
    const float S = run[n - 1];   /* the last range's running value is the blocked total */
    float* p = run;               /* reuse: p_i = e_i / S */
    for (int i = 0; i < n; ++i) p[i] = v[i] / S;
    int result, K = n;
    if (top_p > 0.0f && top_p < 1.0f) {
        for (int i = 0; i < n; ++i) pi[i].p = p[i], pi[i].i = i;
        qsort(pi, n, sizeof(orc_pi), cmp_pi);
        for (int k = 0; k < n; ++k) v[k] = pi[k].p;
        blocked_running(v, n, run);
        K = n;
        for (int k = 0; k < n; ++k)
            if (run[k] >= top_p) {
                K = k + 1;
                break;
            }
        const float C = run[K - 1];
        for (int k = 0; k < K; ++k) v[k] = v[k] / C;
        blocked_running(v, K, run);   /* ranges over the kept prefix */
        result = pi[K - 1].i;
        for (int k = 0; k < K; ++k)
            if (r <= run[k]) {
                result = pi[k].i;
                break;
            }
    } else {
        for (int i = 0; i < n; ++i) v[i] = p[i];
        blocked_running(v, n, run);
        result = n - 1;
        for (int i = 0; i < n; ++i)
            if (r <= run[i]) {
                result = i;
                break;
            }
    }
    if (kept) *kept = K;
    free(v);
    free(run);
    free(pi);
    return result;
}
