/*
 * forward_oracle.c -- CPU restatement of the reference's decoder step,
 * forward_runtime (src/runtime.c:94-289), for the device decoder's parity
 * tests.  TEST INFRASTRUCTURE ONLY: imported by tests/ and bench.py's CPU
 * baseline leg, never by the product library.
 *
 * It follows the reference statement for statement, in the same operation
 * order, compiled like the reference's scalar build (-O3 -std=c99
 * -ffp-contract=off), with the C library's expf/powf/cosf/sinf:
 *   embedding   dequantize_row of the token's row (src/runtime.c:108-113)
 *   rmsnorm     src/kernels.c:179-189 (sequential sum of squares, eps 1e-5)
 *   Q/K/V       matmul_q -> matmul_q_fused (src/runtime.c:58-70, 124-126)
 *   RoPE        src/runtime.c:19-41: adjacent pairs (i, i+1), frequency
 *               base^(-i/head_dim) with i running over the whole query
 *   KV store    src/runtime.c:74-92, 129-132 (fp32, or fp16 through the
 *               reference's truncating fp32_to_fp16)
 *   attention   src/runtime.c:135-194 (dot_ref * 1/sqrt(head_dim), softmax_ref,
 *               value rows accumulated position by position)
 *   FFN         dense (src/runtime.c:270-284) or the routed MoE block
 *               (src/runtime.c:202-269, W1 = the tensor the loader binds to
 *               ffn_up)
 *   head        final rmsnorm + matmul_q (src/runtime.c:286-287)
 *
 * Two generalisations, both identities on every model the reference can load:
 *   - head_dim may be given explicitly (the reference derives dim / n_heads,
 *     src/runtime.c:102); the query then has q_dim = n_heads*head_dim
 *     elements, Wq is q_dim x dim, Wo dim x q_dim, and RoPE runs over q_dim;
 *   - an optional shared expert with a sigmoid gate (Qwen1.5-MoE; the
 *     reference loads none, src/model.c:401-446): after the routed experts,
 *     hb = silu(Ws1.xb) * (Ws3.xb), o = Ws2.hb (the dense FFN's binding,
 *     W1 = gate), g = 1/(1 + expf(-(gate . xb))) with gate . xb in
 *     matmul_ref order, and xb2[i] += o[i]*g before x += xb2.
 * tests/test_forward_oracle.py pins this file against the reference's own
 * forward_runtime (oracle/_ref/libquantr_ref_forward_scalar.so) bit for bit.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "quant_oracle.h"

struct qo_state {
    qo_model m;
    int head_dim, q_dim, kv_dim, kv_mul, threads;
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits, *sh;
    void *key_cache, *value_cache;
};

/* src/kernels.c:179-189 */
static void rmsnorm(float* o, const float* x, const float* w, int size)
{
    float ss = 0.0f;
    for (int i = 0; i < size; i++) ss += x[i] * x[i];
    ss = ss / (float)size + 1e-5f;
    float scale = 1.0f / sqrtf(ss);
    for (int i = 0; i < size; i++) o[i] = w[i] * (x[i] * scale);
}

/* src/kernels.c:171-177 */
static float dot(const float* a, const float* b, int n)
{
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

static float silu(float x) { return x / (1.0f + expf(-x)); } /* src/runtime.c:15-17 */

/* src/runtime.c:58-70 (F32 weights through KernelOps.matmul = matmul_ref order). */
static void matmul_q(float* out, const float* x, const void* w, uint32_t type, int n, int d, int threads)
{
    if (!w) {
        memset(out, 0, (size_t)n * sizeof(float));
        return;
    }
    if (type == QO_F32) {
        qo_matmul_f32(out, x, (const float*)w, n, d);
        return;
    }
    qo_matmul_q_fused(out, x, w, type, n, d, threads);
}

/* src/runtime.c:19-41 over the whole query (q_dim) and the first kv_dim key
 * elements. */
static void rope(float* q, float* k, int q_dim, int kv_dim, int head_dim, int pos, float base_in)
{
    if (kv_dim > q_dim) kv_dim = q_dim;
    float base = base_in > 0.0f ? base_in : 10000.0f;
    for (int i = 0; i < q_dim; i += 2) {
        float freq = powf(base, -((float)i / (float)head_dim));
        float theta = (float)pos * freq;
        float c = cosf(theta);
        float s = sinf(theta);
        float q0 = q[i], q1 = q[i + 1];
        q[i] = q0 * c - q1 * s;
        q[i + 1] = q0 * s + q1 * c;
        if (i < kv_dim) {
            float k0 = k[i], k1 = k[i + 1];
            k[i] = k0 * c - k1 * s;
            k[i + 1] = k0 * s + k1 * c;
        }
    }
}

/* src/runtime.c:74-92 */
static void kv_store(void* cache, int kv_type, size_t off, const float* src, int n)
{
    if (kv_type == 1) {
        uint16_t* d = (uint16_t*)cache + off;
        for (int i = 0; i < n; i++) d[i] = qo_fp32_to_fp16(src[i]);
    } else {
        memcpy((float*)cache + off, src, (size_t)n * sizeof(float));
    }
}
static float kv_get(const void* cache, int kv_type, size_t idx)
{
    return kv_type == 1 ? qo_fp16_to_fp32(((const uint16_t*)cache)[idx]) : ((const float*)cache)[idx];
}

qo_state* qo_open(const qo_model* m, int threads)
{
    qo_state* s = (qo_state*)calloc(1, sizeof(qo_state));
    if (!s) return NULL;
    s->m = *m;
    s->head_dim = m->head_dim > 0 ? m->head_dim : m->dim / (m->n_heads > 0 ? m->n_heads : 1);
    s->q_dim = m->n_heads * s->head_dim;
    s->kv_dim = m->n_kv_heads * s->head_dim;
    s->kv_mul = m->n_heads / (m->n_kv_heads > 0 ? m->n_kv_heads : 1);
    s->threads = threads > 0 ? threads : 1;
    const int hid = m->hidden_dim > m->shexp_hidden_dim ? m->hidden_dim : m->shexp_hidden_dim;
    const int wide = s->q_dim > m->dim ? s->q_dim : m->dim;
    s->x = (float*)calloc((size_t)m->dim, sizeof(float));
    s->xb = (float*)calloc((size_t)wide, sizeof(float));
    s->xb2 = (float*)calloc((size_t)m->dim, sizeof(float));
    s->hb = (float*)calloc((size_t)hid + 1, sizeof(float));
    s->hb2 = (float*)calloc((size_t)hid + 1, sizeof(float));
    s->q = (float*)calloc((size_t)wide, sizeof(float));
    s->k = (float*)calloc((size_t)s->kv_dim, sizeof(float));
    s->v = (float*)calloc((size_t)s->kv_dim, sizeof(float));
    s->sh = (float*)calloc((size_t)m->dim, sizeof(float));
    s->att = (float*)calloc((size_t)m->n_heads * m->seq_len, sizeof(float));
    s->logits = (float*)calloc((size_t)m->vocab_size, sizeof(float));
    const size_t kv = (size_t)m->n_layers * m->seq_len * s->kv_dim;
    const size_t es = m->kv_type == 1 ? 2 : 4;
    s->key_cache = calloc(kv, es);
    s->value_cache = calloc(kv, es);
    if (!s->x || !s->xb || !s->xb2 || !s->hb || !s->hb2 || !s->q || !s->k || !s->v || !s->sh || !s->att ||
        !s->logits || !s->key_cache || !s->value_cache) {
        qo_close(s);
        return NULL;
    }
    return s;
}

void qo_close(qo_state* s)
{
    if (!s) return;
    free(s->x); free(s->xb); free(s->xb2); free(s->hb); free(s->hb2); free(s->q); free(s->k); free(s->v);
    free(s->sh); free(s->att); free(s->logits); free(s->key_cache); free(s->value_cache);
    free(s);
}

/* The routed MoE branch of src/runtime.c:202-269 for layer l (xb2 = routed
 * sum), then the optional shared expert. */
static void moe(qo_state* s, int l)
{
    const qo_model* m = &s->m;
    const int dim = m->dim, hidden = m->hidden_dim, E = m->expert_count, K = m->expert_used_count;
    float router_logits[256];
    int active[16];
    float ew[16];
    qo_matmul_f32(router_logits, s->xb, m->ffn_gate_inp[l], E, dim);
    qo_softmax(router_logits, E);
    for (int ki = 0; ki < K; ki++) {
        float max_val = -1e9f;
        int max_idx = -1;
        for (int e = 0; e < E; e++)
            if (router_logits[e] > max_val) {
                max_val = router_logits[e];
                max_idx = e;
            }
        active[ki] = max_idx;
        ew[ki] = max_val;
        router_logits[max_idx] = -1e9f;
    }
    float wsum = 0.0f;
    for (int ki = 0; ki < K; ki++) wsum += ew[ki];
    for (int ki = 0; ki < K; ki++) ew[ki] /= wsum;
    memset(s->xb2, 0, (size_t)dim * sizeof(float));
    for (int ki = 0; ki < K; ki++) {
        const int e = active[ki];
        matmul_q(s->hb, s->xb, m->expert_w1[l][e], m->exp_w1_type[l], hidden, dim, s->threads);
        matmul_q(s->hb2, s->xb, m->expert_w3[l][e], m->exp_w3_type[l], hidden, dim, s->threads);
        for (int i = 0; i < hidden; i++) s->hb[i] = silu(s->hb[i]) * s->hb2[i];
        matmul_q(s->q, s->hb, m->expert_w2[l][e], m->exp_w2_type[l], dim, hidden, s->threads);
        for (int i = 0; i < dim; i++) s->xb2[i] += s->q[i] * ew[ki];
    }
    if (m->shexp_hidden_dim > 0 && m->shexp_w1)
        qo_shared_expert(s->xb2, s->xb, m->shexp_gate[l], m->shexp_w1[l], m->shexp_w1_type[l], m->shexp_w3[l],
                         m->shexp_w3_type[l], m->shexp_w2[l], m->shexp_w2_type[l], dim, m->shexp_hidden_dim,
                         s->threads);
}

/* Shared expert (restated from the dense FFN, src/runtime.c:270-284, plus the
 * sigmoid gate): out[i] += (W2.(silu(W1.xb) * W3.xb))[i] * g,
 * g = 1/(1 + expf(-(gate . xb))) with gate . xb in matmul_ref order. */
void qo_shared_expert(float* out, const float* xb, const float* gate, const void* w1, uint32_t t1, const void* w3,
                      uint32_t t3, const void* w2, uint32_t t2, int dim, int hidden, int threads)
{
    float* h1 = (float*)malloc((size_t)hidden * sizeof(float));
    float* h3 = (float*)malloc((size_t)hidden * sizeof(float));
    float* o = (float*)malloc((size_t)dim * sizeof(float));
    if (!h1 || !h3 || !o) {
        free(h1); free(h3); free(o);
        return;
    }
    matmul_q(h1, xb, w1, t1, hidden, dim, threads);
    matmul_q(h3, xb, w3, t3, hidden, dim, threads);
    for (int i = 0; i < hidden; i++) h1[i] = silu(h1[i]) * h3[i];
    matmul_q(o, h1, w2, t2, dim, hidden, threads);
    float g = 0.0f;
    qo_matmul_f32(&g, xb, gate, 1, dim);
    g = 1.0f / (1.0f + expf(-g));
    for (int i = 0; i < dim; i++) out[i] += o[i] * g;
    free(h1); free(h3); free(o);
}

const float* qo_forward(qo_state* s, int token, int pos)
{
    const qo_model* m = &s->m;
    const int dim = m->dim, hidden = m->hidden_dim, hd = s->head_dim, q_dim = s->q_dim, kv_dim = s->kv_dim;
    const int kv_mul = s->kv_mul, seq = m->seq_len, kvt = m->kv_type;
    const float inv_sqrt = 1.0f / sqrtf((float)hd);

    if (m->token_embd_row_bytes > 0)
        qo_dequantize_row(s->x, (const uint8_t*)m->token_embd + (size_t)token * m->token_embd_row_bytes,
                          m->token_embd_type, dim);
    else
        memcpy(s->x, (const float*)m->token_embd + (size_t)token * dim, (size_t)dim * sizeof(float));

    for (int l = 0; l < m->n_layers; l++) {
        rmsnorm(s->xb, s->x, m->rms_att[l], dim);
        matmul_q(s->q, s->xb, m->wq[l], m->wq_type[l], q_dim, dim, s->threads);
        matmul_q(s->k, s->xb, m->wk[l], m->wk_type[l], kv_dim, dim, s->threads);
        matmul_q(s->v, s->xb, m->wv[l], m->wv_type[l], kv_dim, dim, s->threads);
        rope(s->q, s->k, q_dim, kv_dim, hd, pos, m->rope_freq_base);

        const size_t base = ((size_t)l * seq) * kv_dim;
        kv_store(s->key_cache, kvt, base + (size_t)pos * kv_dim, s->k, kv_dim);
        kv_store(s->value_cache, kvt, base + (size_t)pos * kv_dim, s->v, kv_dim);

        float kh[512];
        for (int kvh = 0; kvh < m->n_kv_heads; kvh++) {
            for (int t = 0; t <= pos; t++) {
                const size_t ko = base + (size_t)t * kv_dim + (size_t)kvh * hd;
                for (int i = 0; i < hd; i++) kh[i] = kv_get(s->key_cache, kvt, ko + i);
                for (int mm = 0; mm < kv_mul; mm++) {
                    const int h = kvh * kv_mul + mm;
                    s->att[(size_t)h * seq + t] = dot(s->q + (size_t)h * hd, kh, hd) * inv_sqrt;
                }
            }
        }
        for (int h = 0; h < m->n_heads; h++) qo_softmax(s->att + (size_t)h * seq, pos + 1);
        for (int kvh = 0; kvh < m->n_kv_heads; kvh++) {
            for (int mm = 0; mm < kv_mul; mm++)
                memset(s->xb + (size_t)(kvh * kv_mul + mm) * hd, 0, (size_t)hd * sizeof(float));
            for (int t = 0; t <= pos; t++) {
                const size_t vo = base + (size_t)t * kv_dim + (size_t)kvh * hd;
                for (int mm = 0; mm < kv_mul; mm++) {
                    const int h = kvh * kv_mul + mm;
                    const float a = s->att[(size_t)h * seq + t];
                    float* out = s->xb + (size_t)h * hd;
                    for (int i = 0; i < hd; i++) out[i] += a * kv_get(s->value_cache, kvt, vo + i);
                }
            }
        }

        matmul_q(s->xb2, s->xb, m->wo[l], m->wo_type[l], dim, q_dim, s->threads);
        for (int i = 0; i < dim; i++) s->x[i] += s->xb2[i];
        rmsnorm(s->xb, s->x, m->rms_ffn[l], dim);

        if (m->expert_count > 0) {
            moe(s, l);
            for (int i = 0; i < dim; i++) s->x[i] += s->xb2[i];
        } else {
            matmul_q(s->hb, s->xb, m->w1[l], m->w1_type[l], hidden, dim, s->threads);
            matmul_q(s->hb2, s->xb, m->w3[l], m->w3_type[l], hidden, dim, s->threads);
            for (int i = 0; i < hidden; i++) s->hb[i] = silu(s->hb[i]) * s->hb2[i];
            matmul_q(s->xb, s->hb, m->w2[l], m->w2_type[l], dim, hidden, s->threads);
            for (int i = 0; i < dim; i++) s->x[i] += s->xb[i];
        }
    }
    rmsnorm(s->xb, s->x, m->rms_final, dim);
    matmul_q(s->logits, s->xb, m->wcls, m->wcls_type, m->vocab_size, dim, s->threads);
    return s->logits;
}

/* Greedy pick of src/sampling.c:125-131 (the first maximum; the penalties
 * at repetition 1.0 / frequency 0.0 leave every logit unchanged). */
static int argmax(const float* l, int n)
{
    int best = 0;
    for (int i = 1; i < n; i++)
        if (l[i] > l[best]) best = i;
    return best;
}

/* The reference CLI's loop (src/main.c:305-317): sequential prefill
 * (src/runtime.c:294-304), then the last prompt token again at position
 * n_prompt, `steps` greedy tokens. */
void qo_generate(qo_state* s, const int* prompt, int n_prompt, int steps, int* out_tokens, float* logits)
{
    const int vocab = s->m.vocab_size;
    int token = 0, pos = 0;
    for (int i = 0; i < n_prompt; i++) qo_forward(s, prompt[i], i);
    if (n_prompt > 0) {
        token = prompt[n_prompt - 1];
        pos = n_prompt;
    }
    for (int i = 0; i < steps; i++) {
        const float* l = qo_forward(s, token, pos++ % s->m.seq_len);
        if (logits) memcpy(logits + (size_t)i * vocab, l, (size_t)vocab * sizeof(float));
        token = argmax(l, vocab);
        out_tokens[i] = token;
    }
}
