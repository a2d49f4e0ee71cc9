/*
 * quant_oracle.h -- CPU restatement of quantr-in-c's quantized GEMV path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA path is compared
 * against; it is never linked into, loaded by, or called from the product
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg use it.
 *
 * Every function restates one reference function (cited per function in
 * quant_oracle.c) with the reference's exact floating-point evaluation order,
 * so that it is bit-identical to the reference's scalar build (Makefile:3 flags:
 * -O3 -std=c99, no -mavx2, which implies -ffp-contract=off).  Parity pin: the
 * fixtures in tests/golden/ were produced by the reference's own quant.c
 * compiled from its sources (oracle/Makefile -> oracle/_ref/), and
 * tests/test_oracle.py checks this restatement against them bit for bit.
 *
 * One deliberate divergence: vec_dot_q4K_q8_0 in the reference
 * (src/quant.c:291-369) reads the fp16 fields d, dmin and the activation d as
 * raw integers, so its outputs are not a dot product.  qo_vec_dot_q4K_q8_0 is
 * the restated semantics: the Q4_K decode of src/quant.c:180-195 combined per
 * sub-block as (sc*isum - m*bsum)*bd, the same expression the reference's
 * Q5_K kernel uses (src/quant.c:399).
 */
#ifndef QUANT_ORACLE_H
#define QUANT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids used by the reference (include/gguf.h:28-42). */
enum { QO_F32 = 0, QO_Q8_0 = 8, QO_Q4_K = 12, QO_Q5_K = 13, QO_Q6_K = 14 };

/* Packed Q8_0 block, 34 bytes (include/quant.h:28-33). */
#pragma pack(push, 1)
typedef struct { uint16_t d; int8_t qs[32]; } qo_block_q8_0;
#pragma pack(pop)

float    qo_fp16_to_fp32(uint16_t h);
uint16_t qo_fp32_to_fp16(float f);

/* Bytes of one packed row of `d` columns (src/quant.c:477-484). */
long     qo_row_bytes(uint32_t type, int d);

void  qo_quantize_row_q8_0(const float* x, qo_block_q8_0* y, int k);
void  qo_dequantize_row(float* out, const void* src, uint32_t type, int n);
float qo_vec_dot_q8_0_q8_0(const void* a, const qo_block_q8_0* b, int k);
float qo_vec_dot_q4K_q8_0(const void* a, const qo_block_q8_0* b, int k);
float qo_vec_dot_q5K_q8_0(const void* a, const qo_block_q8_0* b, int k);
float qo_vec_dot_q6K_q8_0(const void* a, const qo_block_q8_0* b, int k);

void  qo_matmul_q_fused(float* out, const float* x, const void* w, uint32_t type,
                        int n, int d, int threads);
/* B independent matmul_q_fused calls: out is B x n, x is B x d (row-major). */
void  qo_matmul_q_fused_batch(float* out, const float* x, const void* w, uint32_t type,
                              int n, int d, int B, int threads);

/* Per-unit int32 partial sums of one GEMV (unit = one Q8_0 block for type 8,
 * one 32-element sub-block for the K-quants).  isum[r*U + u] = sum of
 * weight_q * x_q over the unit (Q6_K: weight_q already offset by -32);
 * bsum[r*U + u] = sum of x_q over the unit.  U = units per row. */
int   qo_unit_partials(int32_t* isum, int32_t* bsum, const void* w, uint32_t type,
                       int n, int d, const qo_block_q8_0* xq);

/* MoE block of forward_runtime (src/runtime.c:202-269), one token.
 *   xb       : [dim] normalised activation
 *   router   : [E x dim] fp32 router weights, or NULL when `logits` is given
 *   logits   : [E] precomputed router logits (used when router == NULL)
 *   w1/w2/w3 : expert weight bases; expert e starts at base + e * bytes
 *   out      : [dim] the accumulated xb2 (the residual add is the caller's)
 *   sel/wts  : [k] selected experts (selection order) and renormalised weights
 * Returns 0, or -1 when k or E exceed the reference's fixed buffers. */
int   qo_moe_token(float* out, int* sel, float* wts, const float* xb,
                   const float* router, const float* logits, int E, int k,
                   const void* w1, uint32_t t1, long w1_bytes,
                   const void* w3, uint32_t t3, long w3_bytes,
                   const void* w2, uint32_t t2, long w2_bytes,
                   int dim, int hidden);

/* Reference F32 kernels the MoE block uses (src/kernels.c:18-28, :191-207). */
void  qo_matmul_f32(float* out, const float* x, const float* w, int n, int d);
void  qo_softmax(float* x, int size);

/* Mismatches of got[i] against the C library's expf(bits first + i). */
long  qo_expf_mismatches(const float* got, uint32_t first, long n);

/* ---- decoder step (forward_oracle.c) ------------------------------------ */

/* Model description: the reference's Config + TransformerWeights
 * (include/types.h:19-71) as plain arrays indexed by layer (experts: per layer
 * an array of expert_count pointers).  The fields up to exp_w3_type are laid
 * out exactly like oracle/ref_forward.c's ref_model, so one struct drives both
 * the restatement and the reference.  head_dim = 0 means dim / n_heads. */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
    float rope_freq_base;
    int expert_count, expert_used_count;
    int kv_type;                       /* 0 = fp32, 1 = fp16 (src/runtime.c:74-92) */
    const void* token_embd;
    uint32_t token_embd_type;
    size_t token_embd_row_bytes;       /* 0: F32 table of dim floats per token */
    const float* const* rms_att;
    const float* const* rms_ffn;
    const void* const* wq;
    const void* const* wk;
    const void* const* wv;
    const void* const* wo;
    const void* const* w1;
    const void* const* w2;
    const void* const* w3;
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
    const float* const* ffn_gate_inp;  /* router, expert_count x dim F32 */
    const void* const* const* expert_w1;
    const void* const* const* expert_w2;
    const void* const* const* expert_w3;
    const uint32_t* exp_w1_type;
    const uint32_t* exp_w2_type;
    const uint32_t* exp_w3_type;
    /* restatement-only extensions */
    int head_dim;
    int shexp_hidden_dim;              /* shared expert (0 = none) */
    const void* const* shexp_w1;       /* gate: shexp_hidden x dim */
    const void* const* shexp_w2;       /* down: dim x shexp_hidden */
    const void* const* shexp_w3;       /* up:   shexp_hidden x dim */
    const uint32_t* shexp_w1_type;
    const uint32_t* shexp_w2_type;
    const uint32_t* shexp_w3_type;
    const float* const* shexp_gate;    /* dim F32 per layer */
} qo_model;

/* Shared expert + sigmoid gate added to out (a Qwen1.5-MoE block's tail). */
void qo_shared_expert(float* out, const float* xb, const float* gate, const void* w1, uint32_t t1,
                      const void* w3, uint32_t t3, const void* w2, uint32_t t2, int dim, int hidden,
                      int threads);

typedef struct qo_state qo_state;
qo_state*    qo_open(const qo_model* m, int threads);
void         qo_close(qo_state* s);
/* forward_runtime(token, pos): returns the state's logits (vocab floats). */
const float* qo_forward(qo_state* s, int token, int pos);
/* src/main.c:305-317 with greedy sampling; logits optional (steps x vocab). */
void         qo_generate(qo_state* s, const int* prompt, int n_prompt, int steps, int* out_tokens,
                         float* logits);

#ifdef __cplusplus
}
#endif
#endif
