/*
 * ref_forward.c -- drives the reference's own forward pass for the decode
 * parity tests.  TEST INFRASTRUCTURE ONLY: compiled by oracle/Makefile into
 * oracle/_ref/libquantr_ref_forward_*.so next to the reference's unmodified
 * src/runtime.c, src/kernels.c, src/quant.c, src/model.c, src/gguf.c,
 * src/sampling.c and src/threadpool.c (read in place), never into the product.
 *
 * The harness builds a Transformer (include/types.h:135-146) around caller
 * buffers instead of a GGUF mapping (src/model.c:253-449 does the same with
 * pointers into the file), allocates the reference RunState with its own
 * malloc_run_state_kv (src/model.c:101-150), and then calls the reference's
 * forward_runtime / prefill_runtime / sample_next exactly as its CLI does
 * (src/main.c:305-317): prefill the prompt, feed the last prompt token again
 * at position n_prompt, and take `steps` greedy tokens.
 *
 * In the "scalar" build the reference's vec_dot_q4K_q8_0 (src/quant.c:291-369,
 * which reads fp16 scales as integers) is interposed at link time by the
 * restated Q4_K dot product (ref_q4k.c); everything else is the reference's
 * own code.  The "avx512" build links the reference unmodified and is only
 * timed (the CPU baseline), never compared.
 */
#include <stdlib.h>
#include <string.h>

#include "model.h"
#include "runtime.h"
#include "sampling.h"

/* Mirror of the model description the tests fill (one layer entry per
 * pointer-array element). */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
    float rope_freq_base;
    int expert_count, expert_used_count;
    int kv_type;
    const void* token_embd;
    uint32_t token_embd_type;
    size_t token_embd_row_bytes;
    const float** rms_att;
    const float** rms_ffn;
    const void** wq;
    const void** wk;
    const void** wv;
    const void** wo;
    const void** w1;
    const void** w2;
    const void** w3;
    const uint32_t* wq_type;
    const uint32_t* wk_type;
    const uint32_t* wv_type;
    const uint32_t* wo_type;
    const uint32_t* w1_type;
    const uint32_t* w2_type;
    const uint32_t* w3_type;
    const float* rms_final;
    const void* wcls;
    uint32_t wcls_type;
    const float** ffn_gate_inp;
    const void*** expert_w1;
    const void*** expert_w2;
    const void*** expert_w3;
    const uint32_t* exp_w1_type;
    const uint32_t* exp_w2_type;
    const uint32_t* exp_w3_type;
} ref_model;

typedef struct {
    Transformer t;
    RuntimeContext rt;
} ref_handle;

ref_handle* ref_open(const ref_model* m, int backend, int threads)
{
    ref_handle* h = (ref_handle*)calloc(1, sizeof(ref_handle));
    if (!h) return NULL;
    Config* c = &h->t.config;
    c->dim = m->dim;
    c->hidden_dim = m->hidden_dim;
    c->n_layers = m->n_layers;
    c->n_heads = m->n_heads;
    c->n_kv_heads = m->n_kv_heads;
    c->vocab_size = m->vocab_size;
    c->seq_len = m->seq_len;
    c->rope_freq_base = m->rope_freq_base;
    c->expert_count = m->expert_count;
    c->expert_used_count = m->expert_used_count;

    TransformerWeights* w = &h->t.weights;
    /* The reference stores weight pointers as float* whatever their type. */
    w->token_embedding_table = (float*)m->token_embd;
    w->token_embd_type = m->token_embd_type;
    w->token_embd_row_bytes = m->token_embd_row_bytes;
    w->rms_att_weight = (float**)m->rms_att;
    w->rms_ffn_weight = (float**)m->rms_ffn;
    w->wq = (float**)m->wq;
    w->wk = (float**)m->wk;
    w->wv = (float**)m->wv;
    w->wo = (float**)m->wo;
    w->w1 = (float**)m->w1;
    w->w2 = (float**)m->w2;
    w->w3 = (float**)m->w3;
    w->wq_type = (uint32_t*)m->wq_type;
    w->wk_type = (uint32_t*)m->wk_type;
    w->wv_type = (uint32_t*)m->wv_type;
    w->wo_type = (uint32_t*)m->wo_type;
    w->w1_type = (uint32_t*)m->w1_type;
    w->w2_type = (uint32_t*)m->w2_type;
    w->w3_type = (uint32_t*)m->w3_type;
    w->rms_final_weight = (float*)m->rms_final;
    w->wcls = (float*)m->wcls;
    w->wcls_type = m->wcls_type;
    w->ffn_gate_inp = (float**)m->ffn_gate_inp;
    w->expert_w1 = (float***)m->expert_w1;
    w->expert_w2 = (float***)m->expert_w2;
    w->expert_w3 = (float***)m->expert_w3;
    w->exp_w1_type = (uint32_t*)m->exp_w1_type;
    w->exp_w2_type = (uint32_t*)m->exp_w2_type;
    w->exp_w3_type = (uint32_t*)m->exp_w3_type;

    malloc_run_state_kv(&h->t.state, c, m->kv_type);

    RuntimeOptions o;
    memset(&o, 0, sizeof(o));
    o.backend = (KernelBackend)backend;
    o.num_threads = threads > 0 ? threads : 1;
    o.deterministic = 1;
    o.temperature = 0.0f;         /* greedy (src/sampling.c:125-131) */
    o.repetition_penalty = 1.0f;  /* penalties are identities */
    o.frequency_penalty = 0.0f;
    o.kv_cache_quant = m->kv_type;
    runtime_init(&h->rt, o);
    return h;
}

void ref_close(ref_handle* h)
{
    if (!h) return;
    free_run_state(&h->t.state);
    free(h);
}

/* One forward_runtime call; copies the logits out. */
void ref_forward(ref_handle* h, int token, int pos, float* logits)
{
    const float* l = forward_runtime(&h->rt, &h->t, token, pos);
    if (logits) memcpy(logits, l, (size_t)h->t.config.vocab_size * sizeof(float));
}

void ref_prefill(ref_handle* h, const int* tokens, int n) { prefill_runtime(&h->rt, &h->t, tokens, n); }

/* The reference CLI's generation loop (src/main.c:305-317) with greedy
 * sampling.  out_tokens: `steps` ids.  logits (optional): steps x vocab, the
 * logits each sampled token was chosen from. */
void ref_generate(ref_handle* h, const int* prompt, int n_prompt, int steps, int* out_tokens, float* logits)
{
    SamplingState s;
    sampling_state_init(&s, 128);
    const int vocab = h->t.config.vocab_size;
    int token = 0, pos = 0;
    if (n_prompt > 0) {
        prefill_runtime(&h->rt, &h->t, prompt, n_prompt);
        for (int i = 0; i < n_prompt; i++) sampling_state_push(&s, prompt[i]);
        token = prompt[n_prompt - 1];
        pos = n_prompt;
    }
    for (int i = 0; i < steps; i++) {
        float* l = forward_runtime(&h->rt, &h->t, token, pos++ % h->t.config.seq_len);
        if (logits) memcpy(logits + (size_t)i * vocab, l, (size_t)vocab * sizeof(float));
        int next = sample_next(l, vocab, &h->rt.options, &s);
        sampling_state_push(&s, next);
        token = next;
        out_tokens[i] = token;
    }
    sampling_state_free(&s);
}
