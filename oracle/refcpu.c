/*
 * refcpu.c -- CPU restatement of the M=1 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity oracle and the timed CPU baseline.
 * The product library never links or calls this file.  Every function names
 * the reference behaviour it restates (see refcpu.h for the list).
 *
 * Build (oracle/Makefile): gcc -O3 -march=x86-64-v3 -fopenmp -ffp-contract=off.
 * -ffp-contract=off matters: the Q4_0 quantiser computes x*id + 8.5f with two
 * roundings, exactly as gguf-py and ggml-quants.c do.
 */
#include "refcpu.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ fp16 */

float ref_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { mant <<= 1; ++e; } while ((mant & 0x400u) == 0);
            mant &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t ref_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0));
    }
    if (absx >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx < 0x38800000u) { /* below the smallest normal half: subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to 0 */
        const uint32_t e = absx >> 23;
        const uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e; /* 14 + (113 - e) - 1 */
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((absx >> 13) - (112u << 10));
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
}

static float g_f16_table[65536];
static int g_f16_table_ready = 0;

static void f16_table_init(void) {
    if (g_f16_table_ready) return;
#pragma omp critical(refcpu_f16_table)
    {
        if (!g_f16_table_ready) {
            for (uint32_t i = 0; i < 65536; ++i) g_f16_table[i] = ref_f16_to_f32((uint16_t)i);
            __atomic_store_n(&g_f16_table_ready, 1, __ATOMIC_RELEASE);
        }
    }
}

static inline float h2f(uint16_t h) { return g_f16_table[h]; }

void ref_f32_to_f16_row(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = ref_f32_to_f16(x[i]);
}

void ref_f16_to_f32_row(const uint16_t *x, float *y, int64_t n) {
    f16_table_init();
    for (int64_t i = 0; i < n; ++i) y[i] = h2f(x[i]);
}

/* ------------------------------------------------------- block quantisers */

/* ggml-quants.c quantize_row_q8_0_ref: d = amax/127, q = roundf(x * (1/d)),
 * round half away from zero (gguf-py quants.py:378-392, np_roundf at 41-45). */
void ref_quantize_q8_0(const float *x, ref_block_q8_0 *y, int64_t k) {
    const int64_t nb = k / REF_QK;
    for (int64_t i = 0; i < nb; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < REF_QK; ++j) {
            const float v = fabsf(x[i * REF_QK + j]);
            if (v > amax) amax = v;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = ref_f32_to_f16(d);
        for (int j = 0; j < REF_QK; ++j) {
            const float x0 = x[i * REF_QK + j] * id;
            y[i].qs[j] = (int8_t)roundf(x0);
        }
    }
}

/* ggml-quants.c quantize_row_q4_0_ref: the signed value of largest magnitude
 * (first occurrence) sets d = max / -8; q = min(15, (int8)(x*id + 8.5f));
 * element j in the low nibble of byte j, element j+16 in the high nibble
 * (gguf-py quants.py:220-237). */
void ref_quantize_q4_0(const float *x, ref_block_q4_0 *y, int64_t k) {
    const int64_t nb = k / REF_QK;
    for (int64_t i = 0; i < nb; ++i) {
        const float *xb = x + i * REF_QK;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < REF_QK; ++j) {
            const float v = xb[j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = ref_f32_to_f16(d);
        for (int j = 0; j < REF_QK / 2; ++j) {
            const float x0 = xb[j] * id;
            const float x1 = xb[REF_QK / 2 + j] * id;
            const float s0 = x0 + 8.5f;
            const float s1 = x1 + 8.5f;
            int q0 = (int)(int8_t)s0;
            int q1 = (int)(int8_t)s1;
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            y[i].qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void ref_dequantize_q8_0(const ref_block_q8_0 *x, float *y, int64_t k) {
    f16_table_init();
    for (int64_t i = 0; i < k / REF_QK; ++i) {
        const float d = h2f(x[i].d);
        for (int j = 0; j < REF_QK; ++j) y[i * REF_QK + j] = (float)x[i].qs[j] * d;
    }
}

void ref_dequantize_q4_0(const ref_block_q4_0 *x, float *y, int64_t k) {
    f16_table_init();
    for (int64_t i = 0; i < k / REF_QK; ++i) {
        const float d = h2f(x[i].d);
        for (int j = 0; j < REF_QK / 2; ++j) {
            y[i * REF_QK + j] = (float)((int)(x[i].qs[j] & 0x0f) - 8) * d;
            y[i * REF_QK + j + 16] = (float)((int)(x[i].qs[j] >> 4) - 8) * d;
        }
    }
}

int32_t ref_dot_block_q4_0_q8_0(const ref_block_q4_0 *w, const ref_block_q8_0 *x) {
    int32_t s = 0;
    for (int j = 0; j < REF_QK / 2; ++j) {
        s += ((int)(w->qs[j] & 0x0f) - 8) * (int)x->qs[j];
        s += ((int)(w->qs[j] >> 4) - 8) * (int)x->qs[j + 16];
    }
    return s;
}

int32_t ref_dot_block_q8_0_q8_0(const ref_block_q8_0 *w, const ref_block_q8_0 *x) {
    int32_t s = 0;
    for (int j = 0; j < REF_QK; ++j) s += (int)w->qs[j] * (int)x->qs[j];
    return s;
}

/* ----------------------------------------------------------------- mul_mat */

/* Accumulation order of the block-dot sums in the quantised MUL_MATs:
 * 0 = fp64 accumulator (default), 1 = fp32 sequential accumulator.  Both are
 * valid ggml-cpu semantics (ggml's own order depends on the SIMD width); the
 * switch exists to measure how far two valid orders drift apart downstream of
 * the discontinuous Q8_0 activation quantisation. */
static int g_accum_mode = 0;
void ref_set_accum_mode(int mode) { g_accum_mode = mode; }

static int pick_threads(int nthreads) {
#ifdef _OPENMP
    return nthreads > 0 ? nthreads : omp_get_max_threads();
#else
    (void)nthreads;
    return 1;
#endif
}

/* ggml-cpu F16 x F32: src1 is converted to F16 (vec_dot_type), the dot is
 * taken over f32 products; accumulated here in double. */
void ref_mul_mat_f16(const uint16_t *w, const float *x, float *y, int64_t n, int64_t k, int nthreads) {
    f16_table_init();
    float *xh = (float *)malloc(sizeof(float) * (size_t)k);
    for (int64_t i = 0; i < k; ++i) xh[i] = h2f(ref_f32_to_f16(x[i]));
    const int nt = pick_threads(nthreads);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const uint16_t *row = w + r * k;
        double acc = 0.0;
        float part = 0.0f;
        for (int64_t i = 0; i < k; ++i) {
            part += h2f(row[i]) * xh[i];
            if ((i & 31) == 31) { acc += part; part = 0.0f; }
        }
        y[r] = (float)(acc + part);
    }
    free(xh);
}

/* ggml-cpu Q4_0 x F32 after src1 has been converted to Q8_0 blocks (the
 * vec_dot_type of Q4_0): y[r] = sum_b d_w * d_x * dot_b.  Takes the Q8_0
 * activation as given, so a test can feed the bytes a GPU kernel used. */
void ref_mul_mat_q4_0_xq(const void *wv, const void *xqv, float *y, int64_t n, int64_t k, int nthreads) {
    f16_table_init();
    const ref_block_q4_0 *w = (const ref_block_q4_0 *)wv;
    const ref_block_q8_0 *xq = (const ref_block_q8_0 *)xqv;
    const int64_t nb = k / REF_QK;
    const int nt = pick_threads(nthreads);
    float *xd = (float *)malloc(sizeof(float) * (size_t)nb);
    for (int64_t b = 0; b < nb; ++b) xd[b] = h2f(xq[b].d);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const ref_block_q4_0 *row = w + r * nb;
        double acc = 0.0;
        float accf = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            const int32_t s = ref_dot_block_q4_0_q8_0(row + b, xq + b);
            if (g_accum_mode == 0)
                acc += (double)(h2f(row[b].d) * xd[b]) * (double)s;
            else
                accf += (h2f(row[b].d) * xd[b]) * (float)s;
        }
        y[r] = g_accum_mode == 0 ? (float)acc : accf;
    }
    free(xd);
}

void ref_mul_mat_q4_0(const void *wv, const float *x, float *y, int64_t n, int64_t k, int mode, int nthreads) {
    f16_table_init();
    const ref_block_q4_0 *w = (const ref_block_q4_0 *)wv;
    const int64_t nb = k / REF_QK;
    const int nt = pick_threads(nthreads);
    if (mode == 0) {
        ref_block_q8_0 *xq = (ref_block_q8_0 *)malloc(sizeof(ref_block_q8_0) * (size_t)nb);
        ref_quantize_q8_0(x, xq, k);
        ref_mul_mat_q4_0_xq(wv, xq, y, n, k, nthreads);
        free(xq);
    } else {
        float *xh = (float *)malloc(sizeof(float) * (size_t)k);
        for (int64_t i = 0; i < k; ++i) xh[i] = h2f(ref_f32_to_f16(x[i]));
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int64_t r = 0; r < n; ++r) {
            const ref_block_q4_0 *row = w + r * nb;
            double acc = 0.0;
            for (int64_t b = 0; b < nb; ++b) {
                const float d = h2f(row[b].d);
                float part = 0.0f;
                for (int j = 0; j < 16; ++j) {
                    part += (float)((int)(row[b].qs[j] & 0x0f) - 8) * xh[b * REF_QK + j];
                    part += (float)((int)(row[b].qs[j] >> 4) - 8) * xh[b * REF_QK + 16 + j];
                }
                acc += (double)d * (double)part;
            }
            y[r] = (float)acc;
        }
        free(xh);
    }
}

void ref_mul_mat_q8_0(const void *wv, const float *x, float *y, int64_t n, int64_t k, int nthreads) {
    f16_table_init();
    const ref_block_q8_0 *w = (const ref_block_q8_0 *)wv;
    const int64_t nb = k / REF_QK;
    ref_block_q8_0 *xq = (ref_block_q8_0 *)malloc(sizeof(ref_block_q8_0) * (size_t)nb);
    ref_quantize_q8_0(x, xq, k);
    float *xd = (float *)malloc(sizeof(float) * (size_t)nb);
    for (int64_t b = 0; b < nb; ++b) xd[b] = h2f(xq[b].d);
    const int nt = pick_threads(nthreads);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const ref_block_q8_0 *row = w + r * nb;
        double acc = 0.0;
        for (int64_t b = 0; b < nb; ++b) {
            const int32_t s = ref_dot_block_q8_0_q8_0(row + b, xq + b);
            acc += (double)(h2f(row[b].d) * xd[b]) * (double)s;
        }
        y[r] = (float)acc;
    }
    free(xd);
    free(xq);
}

/* Per-(row, 32-block) int32 dots of Q4_0 rows with given Q8_0 blocks. */
void ref_block_dots_q4_0_xq(const void *wv, const void *xqv, int32_t *dots, int64_t n, int64_t k) {
    const ref_block_q4_0 *w = (const ref_block_q4_0 *)wv;
    const ref_block_q8_0 *xq = (const ref_block_q8_0 *)xqv;
    const int64_t nb = k / REF_QK;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r)
        for (int64_t b = 0; b < nb; ++b) dots[r * nb + b] = ref_dot_block_q4_0_q8_0(w + r * nb + b, xq + b);
}

void ref_block_dots_q4_0(const void *wv, const float *x, int32_t *dots, int64_t n, int64_t k) {
    const int64_t nb = k / REF_QK;
    ref_block_q8_0 *xq = (ref_block_q8_0 *)malloc(sizeof(ref_block_q8_0) * (size_t)nb);
    ref_quantize_q8_0(x, xq, k);
    ref_block_dots_q4_0_xq(wv, xq, dots, n, k);
    free(xq);
}

void ref_block_dots_q8_0(const void *wv, const float *x, int32_t *dots, int64_t n, int64_t k) {
    const ref_block_q8_0 *w = (const ref_block_q8_0 *)wv;
    const int64_t nb = k / REF_QK;
    ref_block_q8_0 *xq = (ref_block_q8_0 *)malloc(sizeof(ref_block_q8_0) * (size_t)nb);
    ref_quantize_q8_0(x, xq, k);
    for (int64_t r = 0; r < n; ++r)
        for (int64_t b = 0; b < nb; ++b) dots[r * nb + b] = ref_dot_block_q8_0_q8_0(w + r * nb + b, xq + b);
    free(xq);
}

/* ---------------------------------------------------------- flash attention */

static int effective_ctx(const int32_t *kv_len, int n_kv) {
    /* attention_step_custom.cpp:110-113 */
    if (kv_len && kv_len[0] > 0 && kv_len[0] < n_kv) return kv_len[0];
    return n_kv;
}

void ref_flash_attn_ext_decode(const float *q, const uint16_t *k, const uint16_t *v,
                               const uint16_t *mask, const int32_t *kv_len, float *out,
                               int D, int Hq, int Hkv, int n_kv,
                               int64_t k_row, int64_t k_head, int64_t v_row, int64_t v_head,
                               float scale, int mode) {
    f16_table_init();
    const int ctx = effective_ctx(kv_len, n_kv);
    const int group = Hq / Hkv;
    float *qh = (float *)malloc(sizeof(float) * (size_t)D);
    double *sc = (double *)malloc(sizeof(double) * (size_t)(ctx > 0 ? ctx : 1));
    double *acc = (double *)malloc(sizeof(double) * (size_t)D);
    uint16_t *acc16 = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)D);
    float *acc32 = (float *)malloc(sizeof(float) * (size_t)D);
    for (int h = 0; h < Hq; ++h) {
        const int hk = h / group;
        for (int d = 0; d < D; ++d) qh[d] = h2f(ref_f32_to_f16(q[(int64_t)h * D + d]));
        float *o = out + (int64_t)h * D;
        if (mode == 0) {
            double m = -INFINITY;
            for (int t = 0; t < ctx; ++t) {
                const double mv = mask ? (double)h2f(mask[t]) : 0.0;
                if (mv == -INFINITY) { sc[t] = -INFINITY; continue; }
                const uint16_t *kr = k + (int64_t)t * k_row + (int64_t)hk * k_head;
                double s = 0.0;
                for (int d = 0; d < D; ++d) s += (double)qh[d] * (double)h2f(kr[d]);
                s = s * (double)scale + mv;
                sc[t] = s;
                if (s > m) m = s;
            }
            for (int d = 0; d < D; ++d) acc[d] = 0.0;
            double S = 0.0;
            if (m != -INFINITY) {
                for (int t = 0; t < ctx; ++t) {
                    if (sc[t] == -INFINITY) continue;
                    const double p = exp(sc[t] - m);
                    S += p;
                    const uint16_t *vr = v + (int64_t)t * v_row + (int64_t)hk * v_head;
                    for (int d = 0; d < D; ++d) acc[d] += p * (double)h2f(vr[d]);
                }
            }
            for (int d = 0; d < D; ++d) o[d] = S > 0.0 ? (float)(acc[d] / S) : 0.0f;
        } else if (mode == 1) {
            /* ggml-cpu flash_attn_ext_f16 one-chunk loop with F16 V: the V
             * accumulator is kept in f16 and rescaled/updated in place. */
            float M = -INFINITY, S = 0.0f;
            for (int d = 0; d < D; ++d) acc16[d] = 0;
            for (int t = 0; t < ctx; ++t) {
                const float mv = mask ? h2f(mask[t]) : 0.0f;
                if (mv == -INFINITY) continue;
                const uint16_t *kr = k + (int64_t)t * k_row + (int64_t)hk * k_head;
                double sd = 0.0;
                for (int d = 0; d < D; ++d) sd += (double)(qh[d] * h2f(kr[d]));
                float s = (float)sd;
                s = s * scale;
                s += mv;
                const float Mold = M;
                float ms = 1.0f, vs = 1.0f;
                if (s > M) {
                    M = s;
                    ms = expf(Mold - M);
                    for (int d = 0; d < D; ++d) acc16[d] = ref_f32_to_f16(h2f(acc16[d]) * ms);
                } else {
                    vs = expf(s - M);
                }
                const uint16_t *vr = v + (int64_t)t * v_row + (int64_t)hk * v_head;
                for (int d = 0; d < D; ++d) acc16[d] = ref_f32_to_f16(h2f(acc16[d]) + h2f(vr[d]) * vs);
                S = S * ms + vs;
            }
            const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
            for (int d = 0; d < D; ++d) o[d] = h2f(acc16[d]) * S_inv;
        } else {
            /* reference AttentionStepCustom: 240-row tiles, f32 online softmax
             * (attention_step_custom.cpp:143-269), output rounded to f16 RINT
             * (attention_step_custom.cpp:272) then cast back to f32 (P:1426). */
            const int TILE = 240;
            float mx = -2.0e38f, sum = 0.0f;
            for (int d = 0; d < D; ++d) acc32[d] = 0.0f;
            float *p = (float *)malloc(sizeof(float) * TILE);
            for (int t0 = 0; t0 < ctx; t0 += TILE) {
                const int ts = ctx - t0 < TILE ? ctx - t0 : TILE;
                float tmax = -INFINITY;
                for (int i = 0; i < ts; ++i) {
                    const int t = t0 + i;
                    const uint16_t *kr = k + (int64_t)t * k_row + (int64_t)hk * k_head;
                    float s = 0.0f;
                    for (int d = 0; d < D; ++d) s += qh[d] * h2f(kr[d]);
                    s = s * scale;
                    s = s + (mask ? h2f(mask[t]) : 0.0f);
                    p[i] = s;
                    if (s > tmax) tmax = s;
                }
                const float nmax = tmax > mx ? tmax : mx;
                const float ef = expf(mx - nmax);
                float tsum = 0.0f;
                for (int i = 0; i < ts; ++i) { p[i] = expf(p[i] - nmax); tsum += p[i]; }
                sum = sum * ef + tsum;
                mx = nmax;
                for (int d = 0; d < D; ++d) acc32[d] *= ef;
                for (int i = 0; i < ts; ++i) {
                    const uint16_t *vr = v + (int64_t)(t0 + i) * v_row + (int64_t)hk * v_head;
                    for (int d = 0; d < D; ++d) acc32[d] += p[i] * h2f(vr[d]);
                }
            }
            free(p);
            for (int d = 0; d < D; ++d) o[d] = h2f(ref_f32_to_f16(acc32[d] / sum));
        }
    }
    free(acc32);
    free(acc16);
    free(acc);
    free(sc);
    free(qh);
}

void ref_kv_lengths_from_mask_f16(const uint16_t *mask, int64_t n_kv, int64_t n_rows, int32_t *out) {
    f16_table_init();
    for (int64_t r = 0; r < n_rows; ++r) {
        int64_t len = n_kv;
        while (len > 0 && !isfinite(h2f(mask[r * n_kv + len - 1]))) --len;
        out[r] = (int32_t)(len > 1 ? len : 1);
    }
}

/* --------------------------------------------------------- reference A8W8 */

/* w8a8_quantize_custom_vector.cpp:35-64: amax over the f16 row, clamped to
 * >= 1.27e-6; scale = amax/127 stored as f16; q = rint(x * (127/amax)). */
void ref_a8w8_quantize_token(const uint16_t *x_f16, int8_t *xq, uint16_t *scale_f16, int64_t k) {
    f16_table_init();
    float amax = 0.0f;
    for (int64_t i = 0; i < k; ++i) {
        const float a = fabsf(h2f(x_f16[i]));
        if (a > amax) amax = a;
    }
    if (amax < 0.00000127f) amax = 0.00000127f;
    const float scale = amax / 127.0f;
    const float inv = 127.0f / amax;
    *scale_f16 = ref_f32_to_f16(scale);
    for (int64_t i = 0; i < k; ++i) {
        const float v = h2f(x_f16[i]) * inv;
        xq[i] = (int8_t)nearbyintf(v); /* default rounding mode: half to even */
    }
}

static inline size_t nz_index(int64_t kk, int64_t nn, int64_t k) {
    /* patch P:1690-1691: int8 NZ 16(K) x 32(N) */
    return ((((size_t)nn / 32) * ((size_t)k / 16) + (size_t)kk / 16) * 16 + (size_t)kk % 16) * 32 + (size_t)nn % 32;
}

/* patch P:1674-1695 ggml_backend_cann_transform_f16_a8w8 */
void ref_a8w8_transform_weight(const uint16_t *w_f16, int8_t *q_nz, uint16_t *scales, int64_t k, int64_t n) {
    f16_table_init();
    for (int64_t c = 0; c < n; ++c) {
        float max_abs = 0.0f;
        for (int64_t r = 0; r < k; ++r) {
            const float a = fabsf(h2f(w_f16[c * k + r]));
            if (a > max_abs) max_abs = a;
        }
        float scale = max_abs / 127.0f;
        if (scale < 1.0e-8f) scale = 1.0e-8f;
        scales[c] = ref_f32_to_f16(scale);
        for (int64_t r = 0; r < k; ++r) {
            const float value = h2f(w_f16[c * k + r]) / scale;
            float q = roundf(value);
            if (q > 127.0f) q = 127.0f;
            if (q < -127.0f) q = -127.0f;
            q_nz[nz_index(r, c, k)] = (int8_t)q;
        }
    }
}

void ref_a8w8_matmul_i32(const int8_t *xq, const int8_t *w_nz, int32_t *acc, int64_t k, int64_t n) {
    for (int64_t c = 0; c < n; ++c) {
        int32_t s = 0;
        for (int64_t r = 0; r < k; ++r) s += (int32_t)xq[r] * (int32_t)w_nz[nz_index(r, c, k)];
        acc[c] = s;
    }
}

/* W8a8DequantCustom (source not shipped; call sites P:1269-1270): the output
 * is acc * s_x * s_w[col] rounded to f16. */
void ref_a8w8_dequant(const int32_t *acc, uint16_t x_scale, const uint16_t *w_scales, uint16_t *out, int64_t n) {
    f16_table_init();
    const float xs = h2f(x_scale);
    for (int64_t c = 0; c < n; ++c) out[c] = ref_f32_to_f16(((float)acc[c] * xs) * h2f(w_scales[c]));
}

/* --------------------------------------------------- reference W4A16 probe */

/* gen_data.py:17-39: packed[tile][group][32][tile/2] with the low nibble from
 * output column j and the high nibble from column j + tile/2 (stored +8);
 * scale_layout[tile][group][tile].  Golden: f16 sequential accumulation over k
 * of f16(f16(q*s) * x[k]). */
void ref_w4a16_probe(const uint16_t *x_f16, const uint8_t *packed, const uint16_t *scale_layout,
                     uint16_t *y_f16, int64_t k, int64_t n, int64_t tile) {
    f16_table_init();
    const int64_t groups = k / REF_QK;
    const int64_t half = tile / 2;
    for (int64_t c = 0; c < n; ++c) {
        const int64_t t = c / tile, j = c % tile;
        const int hi = j >= half;
        const int64_t jj = hi ? j - half : j;
        uint16_t acc = 0;
        for (int64_t kk = 0; kk < k; ++kk) {
            const int64_t g = kk / REF_QK, r = kk % REF_QK;
            const uint8_t byte = packed[((t * groups + g) * REF_QK + r) * half + jj];
            const int q = (int)(hi ? (byte >> 4) : (byte & 0x0f)) - 8;
            const float s = h2f(scale_layout[(t * groups + g) * tile + j]);
            const uint16_t wgt = ref_f32_to_f16((float)q * s);
            const uint16_t prod = ref_f32_to_f16(h2f(wgt) * h2f(x_f16[kk]));
            acc = ref_f32_to_f16(h2f(acc) + h2f(prod));
        }
        y_f16[c] = acc;
    }
}

/* ------------------------------------------------------------ synthetic data */

static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* The synthetic-data generator of the GPU path (not a reference
 * behaviour: the benchmark's own seeded data), restated step for step so
 * that the CPU arm regenerates the device's weights and KV cache bit for
 * bit.  ln u: u = m 2^e, m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh(s) with
 * s = (m-1)/(m+1) by its series through s^10/11; cos(2 pi t): folded to
 * [0, 1/4], Taylor series of cos through x^16.  Only correctly rounded f32
 * operations (compiled with -ffp-contract=off; fmaf is a single rounding). */
static inline float synth_ln(float u) {
    union { float f; uint32_t b; } v = {u}, mv;
    mv.b = (v.b & 0x7fffffu) | 0x3f800000u;
    /* branch-free (vectorisable) form of: if m > sqrt(2): m /= 2, e += 1 */
    const int big = mv.f > 1.41421356f;
    const int e = (int)((v.b >> 23) & 0xffu) - 127 + big;
    const float m = mv.f * (big ? 0.5f : 1.0f);
    const float s = (m - 1.0f) / (m + 1.0f);
    const float s2 = s * s;
    float p = fmaf(s2, 0.0909090909f, 0.111111111f);
    p = fmaf(s2, p, 0.142857143f);
    p = fmaf(s2, p, 0.2f);
    p = fmaf(s2, p, 0.333333333f);
    p = fmaf(s2, p, 1.0f);
    return fmaf((float)e, 0.693147181f, (2.0f * s) * p);
}

static inline float synth_cos2pi(float t) {
    /* t > 1/2: 1 - t (exact); then a > 1/4: 1/2 - a (exact), negated result.
     * fminf picks the same operand as those comparisons do. */
    const float t1 = 1.0f - t;
    const float a0 = t < t1 ? t : t1;
    const float sign = a0 > 0.25f ? -1.0f : 1.0f;
    const float a1 = 0.5f - a0;
    const float a = a0 < a1 ? a0 : a1;
    const float x = a * 6.28318531f;
    const float x2 = x * x;
    float p = fmaf(x2, 4.77947733e-14f, -1.14707456e-11f);
    p = fmaf(x2, p, 2.08767570e-9f);
    p = fmaf(x2, p, -2.75573192e-7f);
    p = fmaf(x2, p, 2.48015873e-5f);
    p = fmaf(x2, p, -1.38888889e-3f);
    p = fmaf(x2, p, 4.16666667e-2f);
    p = fmaf(x2, p, -0.5f);
    p = fmaf(x2, p, 1.0f);
    return p * sign;
}

/* Box-Muller on two 24-bit uniforms drawn from splitmix64(seed, index). */
static inline float synth_normal_mixed(uint64_t seed_mixed, uint64_t index) {
    const uint64_t h = splitmix64(seed_mixed ^ (index * 0xD1B54A32D192ED03ull));
    /* both values are below 2^24: exact through a signed conversion */
    const float u1 = ((float)(int32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)(int32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * synth_ln(u1));
    return r * synth_cos2pi(u2);
}

float ref_synth_normal(uint64_t seed, uint64_t index) { return synth_normal_mixed(splitmix64(seed), index); }

/* Rows [0, nrows) of f16 N(0,1) values: element (r, c) takes stream index
 * base + r * rg + col0 + c (the device's KV-cache fill). */
void ref_synth_rows_f16(uint64_t seed, uint64_t base, int64_t nrows, int64_t rl, int64_t rg, int64_t col0,
                        uint16_t *out, int nthreads) {
    const int nt = pick_threads(nthreads);
    const uint64_t sm = splitmix64(seed);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < nrows; ++r)
        for (int64_t c = 0; c < rl; ++c)
            out[r * rl + c] = ref_f32_to_f16(synth_normal_mixed(sm, base + (uint64_t)(r * rg + col0 + c)));
}

void ref_synth_q4_0(uint64_t seed, float sigma, int64_t row0, int64_t nrows, int64_t k, ref_block_q4_0 *out, int nthreads) {
    const int nt = pick_threads(nthreads);
    const int64_t nb = k / REF_QK;
    const uint64_t sm = splitmix64(seed);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < nrows; ++r) {
        float buf[REF_QK];
        for (int64_t b = 0; b < nb; ++b) {
            const uint64_t base = (uint64_t)(row0 + r) * (uint64_t)k + (uint64_t)(b * REF_QK);
#pragma omp simd
            for (int j = 0; j < REF_QK; ++j) buf[j] = sigma * synth_normal_mixed(sm, base + (uint64_t)j);
            ref_quantize_q4_0(buf, out + r * nb + b, REF_QK);
        }
    }
}

/* ------------------------------------------------------------- llama decode */

/* ggml rms_norm (sum of squares in double, scale = 1/sqrtf(mean + eps)) then
 * ggml_mul by the norm weight. */
void ref_rms_norm_mul(const float *x, const float *w, float *y, int64_t n, float eps) {
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; ++i) y[i] = (x[i] * scale) * w[i];
}

/* ggml rope, NORM mode (adjacent pairs), no scaling: theta_i = pos *
 * theta_scale^i built by repeated f32 multiplication with theta_scale =
 * powf(base, -2/head_dim). */
void ref_rope_norm(float *x, int n_heads, int head_dim, int pos, float theta_base) {
    const float theta_scale = powf(theta_base, -2.0f / (float)head_dim);
    float cache[1024];
    float theta = (float)pos;
    for (int i0 = 0; i0 < head_dim; i0 += 2) {
        cache[i0] = cosf(theta);
        cache[i0 + 1] = sinf(theta);
        theta *= theta_scale;
    }
    for (int h = 0; h < n_heads; ++h) {
        float *v = x + (int64_t)h * head_dim;
        for (int i0 = 0; i0 < head_dim; i0 += 2) {
            const float c = cache[i0], s = cache[i0 + 1];
            const float x0 = v[i0], x1 = v[i0 + 1];
            v[i0] = x0 * c - x1 * s;
            v[i0 + 1] = x0 * s + x1 * c;
        }
    }
}

int64_t ref_argmax(const float *x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

int64_t ref_llama_step(const ref_llama *m, int32_t token, int32_t pos, float *x, float *logits,
                       int l0, int l1, int do_head, int nthreads) {
    f16_table_init();
    const ref_llama_cfg *c = &m->cfg;
    const int d = c->d_model, D = c->head_dim, Hq = c->n_head, Hkv = c->n_kv_head, F = c->d_ff;
    const int kvd = Hkv * D;
    float *xn = (float *)malloc(sizeof(float) * (size_t)d);
    float *q = (float *)malloc(sizeof(float) * (size_t)Hq * D);
    float *kk = (float *)malloc(sizeof(float) * (size_t)kvd);
    float *vv = (float *)malloc(sizeof(float) * (size_t)kvd);
    float *att = (float *)malloc(sizeof(float) * (size_t)Hq * D);
    float *y = (float *)malloc(sizeof(float) * (size_t)d);
    float *g = (float *)malloc(sizeof(float) * (size_t)F);
    float *u = (float *)malloc(sizeof(float) * (size_t)F);

    if (l0 == 0) ref_dequantize_q4_0(m->tok_embd + (int64_t)token * (d / REF_QK), x, d);
    for (int l = l0; l < l1; ++l) {
        ref_rms_norm_mul(x, m->attn_norm[l], xn, d, c->eps);
        ref_mul_mat_q4_0(m->wq[l], xn, q, (int64_t)Hq * D, d, 0, nthreads);
        ref_mul_mat_q4_0(m->wk[l], xn, kk, kvd, d, 0, nthreads);
        ref_mul_mat_q4_0(m->wv[l], xn, vv, kvd, d, 0, nthreads);
        ref_rope_norm(q, Hq, D, pos, c->rope_theta);
        ref_rope_norm(kk, Hkv, D, pos, c->rope_theta);
        uint16_t *kc = m->k_cache[l] + (int64_t)pos * kvd;
        uint16_t *vc = m->v_cache[l] + (int64_t)pos * kvd;
        ref_f32_to_f16_row(kk, kc, kvd);
        ref_f32_to_f16_row(vv, vc, kvd);
        ref_flash_attn_ext_decode(q, m->k_cache[l], m->v_cache[l], NULL, NULL, att, D, Hq, Hkv, pos + 1,
                                  kvd, D, kvd, D, 1.0f / sqrtf((float)D), 0);
        ref_mul_mat_q4_0(m->wo[l], att, y, d, (int64_t)Hq * D, 0, nthreads);
        for (int i = 0; i < d; ++i) x[i] = x[i] + y[i];
        ref_rms_norm_mul(x, m->ffn_norm[l], xn, d, c->eps);
        ref_mul_mat_q4_0(m->wgate[l], xn, g, F, d, 0, nthreads);
        ref_mul_mat_q4_0(m->wup[l], xn, u, F, d, 0, nthreads);
        for (int i = 0; i < F; ++i) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
        ref_mul_mat_q4_0(m->wdown[l], g, y, d, F, 0, nthreads);
        for (int i = 0; i < d; ++i) x[i] = x[i] + y[i];
    }
    int64_t best = -1;
    if (do_head) {
        ref_rms_norm_mul(x, m->out_norm, xn, d, c->eps);
        ref_mul_mat_q4_0(m->lm_head, xn, logits, c->vocab, d, 0, nthreads);
        best = ref_argmax(logits, c->vocab);
    }
    free(u); free(g); free(y); free(att); free(vv); free(kk); free(q); free(xn);
    return best;
}
