/*
 * quant_oracle.c -- CPU restatement of quantr-in-c's quantized GEMV path.
 *
 * TEST INFRASTRUCTURE ONLY (see quant_oracle.h): the checker for the CUDA
 * path, never part of the shipped library.
 *
 * Build flags matter: oracle/Makefile compiles this file with
 * -O3 -std=c99 -ffp-contract=off, the reference's own scalar-build semantics
 * (Makefile:3), so every float expression below rounds after each operation in
 * the written order, exactly like the reference's scalar code.
 */
#include "quant_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- fp16 ---- */

/* include/quant.h:53-66.  The bit recipe does not renormalise subnormal
 * halves; that quirk is kept because weight scales are decoded with it. */
float qo_fp16_to_fp32(uint16_t h)
{
    uint32_t mag = (uint32_t)(h & 0x7FFFu) << 13;
    uint32_t e = (h >> 10) & 0x1Fu;
    if (e == 0x1Fu)
        mag |= 0x7F800000u;
    else if (e != 0)
        mag += 0x38000000u;
    uint32_t bits = mag | ((uint32_t)(h & 0x8000u) << 16);
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* include/quant.h:68-77.  Truncates the mantissa, flushes anything below the
 * smallest normal half to signed zero, saturates to signed infinity. */
uint16_t qo_fp32_to_fp16(float f)
{
    uint32_t bits;
    memcpy(&bits, &f, sizeof bits);
    uint16_t s = (uint16_t)((bits >> 16) & 0x8000u);
    int e = (int)((bits >> 23) & 0xFFu) - 112; /* rebias 127 -> 15 */
    if (e <= 0) return s;
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    return (uint16_t)(s | (uint16_t)(e << 10) | (uint16_t)((bits >> 13) & 0x3FFu));
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ---------------------------------------------------------- row sizes ---- */

/* src/quant.c:477-484 (and src/model.c:20-30): floor(d/32) Q8_0 blocks or
 * floor(d/256) super-blocks per row; columns past the last block are ignored. */
long qo_row_bytes(uint32_t type, int d)
{
    switch (type) {
    case QO_Q8_0: return (long)(d / 32) * 34;
    case QO_Q4_K: return (long)(d / 256) * 144;
    case QO_Q5_K: return (long)(d / 256) * 176;
    case QO_Q6_K: return (long)(d / 256) * 210;
    default:      return (long)d * 4;
    }
}

/* ------------------------------------------------ activation quantizer ---- */

/* src/quant.c:143-158.  Scale d = amax/127 is stored through the truncating
 * fp32->fp16 conversion, but the quants use the fp32 reciprocal of the
 * unrounded d; lrintf rounds half to even.  A tail of k%32 is ignored. */
void qo_quantize_row_q8_0(const float* x, qo_block_q8_0* y, int k)
{
    int nblk = k / 32;
    for (int b = 0; b < nblk; b++) {
        const float* v = x + 32 * b;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(v[i]);
            if (a > amax) amax = a;
        }
        float scale = amax / 127.0f;
        float inv = (scale != 0.0f) ? 1.0f / scale : 0.0f;
        y[b].d = qo_fp32_to_fp16(scale);
        for (int i = 0; i < 32; i++)
            y[b].qs[i] = (int8_t)lrintf(v[i] * inv);
    }
}

/* ------------------------------------------------- element decoders ---- */
/* Element e (0..255) of a K-quant super-block.  Nibbles are interleaved: the
 * low nibble of byte (e/2) holds even elements of the 32-element sub-block,
 * the high nibble odd ones (src/quant.c:190). */

static int q4_nib(const uint8_t* qs, int e) { return (qs[e / 2] >> ((e & 1) * 4)) & 0xF; }

static int q4k_q(const uint8_t* sb, int e) { return q4_nib(sb + 16, e); }          /* :190 */

static int q5k_q(const uint8_t* sb, int e)                                          /* :207-209 */
{
    int hi = (sb[16 + e / 8] >> (e % 8)) & 1;
    return q4_nib(sb + 48, e) | (hi << 4);
}

static int q6k_q(const uint8_t* sb, int e)                                          /* :230-232 */
{
    int lo = q4_nib(sb, e);
    int hi = (sb[128 + e / 4] >> ((e % 4) * 2)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* ------------------------------------------------------- dequantizer ---- */

/* src/quant.c:160-240.  Unknown types and NULL sources give zeros. */
void qo_dequantize_row(float* out, const void* src, uint32_t type, int n)
{
    const uint8_t* p = (const uint8_t*)src;
    if (!src) { memset(out, 0, (size_t)n * sizeof(float)); return; }
    if (type == QO_F32) { memcpy(out, src, (size_t)n * sizeof(float)); return; }
    if (type == QO_Q8_0) {
        for (int b = 0; b < n / 32; b++) {
            const uint8_t* blk = p + 34 * b;
            float d = qo_fp16_to_fp32(rd16(blk));
            for (int i = 0; i < 32; i++) out[32 * b + i] = (float)(int8_t)blk[2 + i] * d;
        }
        return;
    }
    if (type == QO_Q4_K || type == QO_Q5_K) {
        long sbb = (type == QO_Q4_K) ? 144 : 176;
        for (int s = 0; s < n / 256; s++) {
            const uint8_t* sb = p + sbb * s;
            float d = qo_fp16_to_fp32(rd16(sb));
            float dmin = qo_fp16_to_fp32(rd16(sb + 2));
            for (int j = 0; j < 8; j++) {
                float sc = (float)(sb[4 + j] & 63) * d;
                float m = (float)(sb[4 + j] >> 6) * dmin;
                for (int l = 0; l < 32; l++) {
                    int e = 32 * j + l;
                    int q = (type == QO_Q4_K) ? q4k_q(sb, e) : q5k_q(sb, e);
                    out[256 * s + e] = (float)q * sc - m;
                }
            }
        }
        return;
    }
    if (type == QO_Q6_K) {
        for (int s = 0; s < n / 256; s++) {
            const uint8_t* sb = p + 210 * s;
            float d = qo_fp16_to_fp32(rd16(sb + 208));
            for (int j = 0; j < 8; j++) {
                float sc = (float)(int8_t)sb[192 + j] * d;
                for (int l = 0; l < 32; l++) {
                    int e = 32 * j + l;
                    out[256 * s + e] = (float)q6k_q(sb, e) * sc;
                }
            }
        }
        return;
    }
    memset(out, 0, (size_t)n * sizeof(float));
}

/* ----------------------------------------------------- unit partials ---- */

/* Integer part of one unit: isum = sum q_w*q_x, bsum = sum q_x. */
static void unit_ints(const uint8_t* sb, uint32_t type, int j, const qo_block_q8_0* xb,
                      int32_t* isum, int32_t* bsum)
{
    int32_t is = 0, bs = 0;
    for (int l = 0; l < 32; l++) {
        int q;
        int e = 32 * j + l;
        switch (type) {
        case QO_Q8_0: q = (int8_t)sb[2 + l]; break;
        case QO_Q4_K: q = q4k_q(sb, e); break;
        case QO_Q5_K: q = q5k_q(sb, e); break;
        default:      q = q6k_q(sb, e); break;
        }
        is += q * (int32_t)xb->qs[l];
        bs += xb->qs[l];
    }
    *isum = is;
    *bsum = bs;
}

/* --------------------------------------------------------- dot kernels ---- */

/* src/quant.c:279-285 (scalar branch): per block, ((float)isum * d_w) * d_x,
 * accumulated in block order. */
float qo_vec_dot_q8_0_q8_0(const void* a, const qo_block_q8_0* b, int k)
{
    const uint8_t* w = (const uint8_t*)a;
    float acc = 0.0f;
    for (int blk = 0; blk < k / 32; blk++) {
        int32_t is, bs;
        unit_ints(w + 34 * blk, QO_Q8_0, 0, &b[blk], &is, &bs);
        acc += (float)is * qo_fp16_to_fp32(rd16(w + 34 * blk)) * qo_fp16_to_fp32(b[blk].d);
    }
    return acc;
}

/* Shared body of the Q4_K / Q5_K dots: src/quant.c:372-403 (Q5_K, verbatim
 * semantics) and the restated Q4_K (decode :180-195, combine as :399). */
static float dot_k45(const void* a, const qo_block_q8_0* b, int k, uint32_t type)
{
    const uint8_t* w = (const uint8_t*)a;
    long sbb = (type == QO_Q4_K) ? 144 : 176;
    float acc = 0.0f;
    for (int s = 0; s < k / 256; s++) {
        const uint8_t* sb = w + sbb * s;
        float d = qo_fp16_to_fp32(rd16(sb));
        float dmin = qo_fp16_to_fp32(rd16(sb + 2));
        for (int j = 0; j < 8; j++) {
            float sc = (float)(sb[4 + j] & 63) * d;
            float m = (float)(sb[4 + j] >> 6) * dmin;
            int32_t is, bs;
            const qo_block_q8_0* xb = &b[8 * s + j];
            unit_ints(sb, type, j, xb, &is, &bs);
            float bd = qo_fp16_to_fp32(xb->d);
            acc += (sc * (float)is - m * (float)bs) * bd;
        }
    }
    return acc;
}

float qo_vec_dot_q4K_q8_0(const void* a, const qo_block_q8_0* b, int k) { return dot_k45(a, b, k, QO_Q4_K); }
float qo_vec_dot_q5K_q8_0(const void* a, const qo_block_q8_0* b, int k) { return dot_k45(a, b, k, QO_Q5_K); }

/* src/quant.c:406-437: signed 6-bit quants, int8 sub-block scales, the term
 * evaluated as (sc * (float)isum) * bd. */
float qo_vec_dot_q6K_q8_0(const void* a, const qo_block_q8_0* b, int k)
{
    const uint8_t* w = (const uint8_t*)a;
    float acc = 0.0f;
    for (int s = 0; s < k / 256; s++) {
        const uint8_t* sb = w + 210 * s;
        float d = qo_fp16_to_fp32(rd16(sb + 208));
        for (int j = 0; j < 8; j++) {
            float sc = (float)(int8_t)sb[192 + j] * d;
            int32_t is, bs;
            const qo_block_q8_0* xb = &b[8 * s + j];
            unit_ints(sb, QO_Q6_K, j, xb, &is, &bs);
            acc += sc * (float)is * qo_fp16_to_fp32(xb->d);
        }
    }
    return acc;
}

/* ------------------------------------------------------ fused matmul ---- */

static float row_dot(const uint8_t* row, const qo_block_q8_0* xq, uint32_t type, int d)
{
    switch (type) {
    case QO_Q8_0: return qo_vec_dot_q8_0_q8_0(row, xq, d);
    case QO_Q4_K: return qo_vec_dot_q4K_q8_0(row, xq, d);
    case QO_Q5_K: return qo_vec_dot_q5K_q8_0(row, xq, d);
    default:      return qo_vec_dot_q6K_q8_0(row, xq, d);
    }
}

/* src/quant.c:441-523.  NULL weights -> zeros; F32 -> sequential row dots;
 * quantized -> quantize x once then one fused dot per row; any other type ->
 * dequantize (zeros for unknown types) and a plain dot. */
void qo_matmul_q_fused(float* out, const float* x, const void* w, uint32_t type,
                       int n, int d, int threads)
{
    if (!w) { memset(out, 0, (size_t)n * sizeof(float)); return; }
    if (type == QO_F32) {
        const float* wf = (const float*)w;
        for (int r = 0; r < n; r++) {
            float acc = 0.0f;
            for (int c = 0; c < d; c++) acc += wf[(size_t)r * d + c] * x[c];
            out[r] = acc;
        }
        return;
    }
    int nx = d / 32 > 0 ? d / 32 : 1;
    qo_block_q8_0* xq = (qo_block_q8_0*)malloc((size_t)nx * sizeof *xq);
    if (!xq) { memset(out, 0, (size_t)n * sizeof(float)); return; }
    qo_quantize_row_q8_0(x, xq, d);
    long rb = qo_row_bytes(type, d);
    int known = type == QO_Q8_0 || type == QO_Q4_K || type == QO_Q5_K || type == QO_Q6_K;
    float* tmp = known ? NULL : (float*)malloc((size_t)d * sizeof(float));
    if (known && threads > 1) {
        /* rows are independent (the reference's OpenMP row loop, src/quant.c:489) */
        int r;
#pragma omp parallel for num_threads(threads) schedule(static)
        for (r = 0; r < n; r++) out[r] = row_dot((const uint8_t*)w + (size_t)r * (size_t)rb, xq, type, d);
        free(xq);
        return;
    }
    for (int r = 0; r < n; r++) {
        const uint8_t* row = (const uint8_t*)w + (size_t)r * (size_t)rb;
        if (known) {
            out[r] = row_dot(row, xq, type, d);
        } else if (tmp) {
            qo_dequantize_row(tmp, row, type, d);
            float acc = 0.0f;
            for (int c = 0; c < d; c++) acc += tmp[c] * x[c];
            out[r] = acc;
        } else {
            out[r] = 0.0f;
        }
    }
    free(tmp);
    free(xq);
}

void qo_matmul_q_fused_batch(float* out, const float* x, const void* w, uint32_t type,
                             int n, int d, int B, int threads)
{
    for (int t = 0; t < B; t++)
        qo_matmul_q_fused(out + (size_t)t * n, x + (size_t)t * d, w, type, n, d, threads);
}

int qo_unit_partials(int32_t* isum, int32_t* bsum, const void* w, uint32_t type,
                     int n, int d, const qo_block_q8_0* xq)
{
    long rb = qo_row_bytes(type, d);
    int per_blk = (type == QO_Q8_0) ? 1 : 8;
    long blk_bytes = (type == QO_Q8_0) ? 34 : (type == QO_Q4_K ? 144 : (type == QO_Q5_K ? 176 : 210));
    int nblk = (type == QO_Q8_0) ? d / 32 : d / 256;
    if (type != QO_Q8_0 && type != QO_Q4_K && type != QO_Q5_K && type != QO_Q6_K) return -1;
    int U = nblk * per_blk;
    for (int r = 0; r < n; r++) {
        const uint8_t* row = (const uint8_t*)w + (size_t)r * (size_t)rb;
        for (int u = 0; u < U; u++) {
            const uint8_t* blk = row + blk_bytes * (u / per_blk);
            unit_ints(blk, type, u % per_blk, &xq[u], &isum[(size_t)r * U + u], &bsum[(size_t)r * U + u]);
        }
    }
    return U;
}

/* ----------------------------------------------------------- F32 + MoE ---- */

/* src/kernels.c:18-28 (matmul_ref). */
void qo_matmul_f32(float* out, const float* x, const float* w, int n, int d)
{
    for (int r = 0; r < n; r++) {
        float acc = 0.0f;
        for (int c = 0; c < d; c++) acc += w[(size_t)r * d + c] * x[c];
        out[r] = acc;
    }
}

/* src/kernels.c:191-207 (softmax_ref). */
void qo_softmax(float* x, int size)
{
    float mx = x[0];
    for (int i = 1; i < size; i++) if (x[i] > mx) mx = x[i];
    float tot = 0.0f;
    for (int i = 0; i < size; i++) { x[i] = expf(x[i] - mx); tot += x[i]; }
    float inv = 1.0f / tot;
    for (int i = 0; i < size; i++) x[i] *= inv;
}

/* src/runtime.c:15-17. */
static float qo_silu(float v) { return v / (1.0f + expf(-v)); }

/* src/runtime.c:202-269, one token.  Router GEMV (or injected logits),
 * softmax, k passes of strict-greater argmax (lowest index wins ties, picked
 * entries masked to -1e9), renormalise by the sum in selection order, then per
 * selected expert in that order: hb = W1.xb, hb2 = W3.xb, hb = silu(hb)*hb2,
 * o = W2.hb, out += o*ew.  W1 is the tensor the reference binds to ffn_up
 * (src/model.c:401-418), so SiLU applies to W1's output as written. */
int qo_moe_token(float* out, int* sel, float* wts, const float* xb,
                 const float* router, const float* logits, int E, int k,
                 const void* w1, uint32_t t1, long w1_bytes,
                 const void* w3, uint32_t t3, long w3_bytes,
                 const void* w2, uint32_t t2, long w2_bytes,
                 int dim, int hidden)
{
    float prob[256];
    if (E > 256 || k > 16 || k > E) return -1;
    if (router) qo_matmul_f32(prob, xb, router, E, dim);
    else memcpy(prob, logits, (size_t)E * sizeof(float));
    qo_softmax(prob, E);
    for (int t = 0; t < k; t++) {
        float best = -1e9f;
        int arg = -1;
        for (int e = 0; e < E; e++)
            if (prob[e] > best) { best = prob[e]; arg = e; }
        sel[t] = arg;
        wts[t] = best;
        prob[arg] = -1e9f;
    }
    float tot = 0.0f;
    for (int t = 0; t < k; t++) tot += wts[t];
    for (int t = 0; t < k; t++) wts[t] /= tot;

    float* hb = (float*)malloc((size_t)hidden * sizeof(float));
    float* hb2 = (float*)malloc((size_t)hidden * sizeof(float));
    float* o = (float*)malloc((size_t)dim * sizeof(float));
    if (!hb || !hb2 || !o) { free(hb); free(hb2); free(o); return -1; }
    memset(out, 0, (size_t)dim * sizeof(float));
    for (int t = 0; t < k; t++) {
        int e = sel[t];
        qo_matmul_q_fused(hb, xb, (const uint8_t*)w1 + (size_t)e * w1_bytes, t1, hidden, dim, 1);
        qo_matmul_q_fused(hb2, xb, (const uint8_t*)w3 + (size_t)e * w3_bytes, t3, hidden, dim, 1);
        for (int i = 0; i < hidden; i++) hb[i] = qo_silu(hb[i]) * hb2[i];
        qo_matmul_q_fused(o, hb, (const uint8_t*)w2 + (size_t)e * w2_bytes, t2, dim, hidden, 1);
        for (int i = 0; i < dim; i++) out[i] += o[i] * wts[t];
    }
    free(hb); free(hb2); free(o);
    return 0;
}

/* Number of i < n where got[i] differs from the C library's expf of the float
 * with bit pattern first + i (NaN results compare equal to any NaN).  Used to
 * check the device's exponential over every float. */
long qo_expf_mismatches(const float* got, uint32_t first, long n)
{
    long bad = 0;
    long i;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (i = 0; i < n; i++) {
        uint32_t u = first + (uint32_t)i, ua, ub;
        float x, a;
        memcpy(&x, &u, 4);
        a = expf(x);
        memcpy(&ua, &a, 4);
        memcpy(&ub, &got[i], 4);
        if (ua != ub && !(a != a && got[i] != got[i])) bad++;
    }
    return bad;
}
