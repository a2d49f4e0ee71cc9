/*
 * quantr_cuda.h -- C ABI of the B200 (sm_100a) quantized-GEMV library
 * libquantr_cuda.so.
 *
 * Part 1 is a drop-in for the reference's hot-path API: the same symbol names,
 * argument types and meanings as quantr-in-c's include/quant.h:84-92, so the
 * reference's runtime (src/runtime.c:58-70 matmul_q -> matmul_q_fused) links
 * against this library instead of src/quant.o unchanged.  These calls take
 * HOST pointers and are synchronous, exactly like the CPU versions: results are
 * in `out` when the call returns.  Weights passed as `w` are served from a
 * device-resident copy when the host range was registered with
 * quantr_gpu_register_weights(), otherwise they are copied up on every call.
 *
 * Part 2 is additive: device selection, weight registration, a sticky error
 * code (the reference's entry points return void), a batched variant, and a
 * stream-ordered device-pointer API for callers that keep activations in HBM.
 *
 * Numerics: every output is bit-identical to the reference's scalar build of
 * src/quant.c (quantized activations, int32 unit sums and fp32 outputs), with
 * one documented exception: for Q4_K the reference's vec_dot_q4K_q8_0
 * (src/quant.c:291-369) reads fp16 scales as raw integers; this library
 * computes the Q4_K dot product that the reference's dequantize_row defines
 * (src/quant.c:180-195), combined per 32-element sub-block as
 * (sc*isum - m*bsum)*d_x like its Q5_K kernel (src/quant.c:399).
 */
#ifndef QUANTR_CUDA_H
#define QUANTR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is
 * exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Block layouts, identical to include/quant.h:28-50 (packed, little-endian).
 * Skipped when the reference's quant.h was included first. */
#ifndef QUANT_H
#define QK8_0 32
#define QK_K 256
#define K_SCALE_SIZE 12
#pragma pack(push, 1)
typedef struct { uint16_t d; int8_t qs[QK8_0]; } block_q8_0;
typedef struct { uint16_t d; uint16_t dmin; uint8_t scales[K_SCALE_SIZE]; uint8_t qs[QK_K / 2]; } block_q4_K;
typedef struct {
    uint16_t d; uint16_t dmin; uint8_t scales[K_SCALE_SIZE]; uint8_t qh[QK_K / 8]; uint8_t qs[QK_K / 2];
} block_q5_K;
#pragma pack(pop)
#endif

/* GGML type ids accepted as `type` (reference include/gguf.h:28-42). */
#define QUANTR_TYPE_F32  0u
#define QUANTR_TYPE_Q8_0 8u
#define QUANTR_TYPE_Q4_K 12u
#define QUANTR_TYPE_Q5_K 13u
#define QUANTR_TYPE_Q6_K 14u

/* ---------------------------------------------------------------------------
 * Part 1: reference-compatible entry points (host pointers, synchronous).
 * -------------------------------------------------------------------------*/

/* Replaces src/quant.c:143 quantize_row_q8_0 (include/quant.h:84).  x: k
 * floats; y: k/32 blocks; a tail of k%32 elements is ignored. */
void quantize_row_q8_0(const float* x, block_q8_0* y, int k);

/* Replaces src/quant.c:160 dequantize_row (include/quant.h:85).  NULL src or
 * an unknown type writes zeros, as the reference does. */
void dequantize_row(float* out, const void* src, uint32_t type, int n);

/* Replace src/quant.c:242/291/372/406 (include/quant.h:86-89).  `a` is one
 * packed weight row of k columns, `b` k/32 Q8_0 activation blocks. */
float vec_dot_q4K_q8_0(const block_q4_K* a, const block_q8_0* b, int k);
float vec_dot_q5K_q8_0(const block_q5_K* a, const block_q8_0* b, int k);
float vec_dot_q6K_q8_0(const void* a, const block_q8_0* b, int k);
float vec_dot_q8_0_q8_0(const block_q8_0* a, const block_q8_0* b, int k);

/* Replaces src/quant.c:441 matmul_q_fused (include/quant.h:91-92):
 * out[i] = row_i(w) . x for n rows of d columns.  NULL w writes zeros; type 0
 * is an fp32 GEMV; Q8_0/Q4_K/Q5_K/Q6_K quantize x to Q8_0 on the device and
 * run the fused integer GEMV; any other type writes zeros (the reference's
 * dequantize fallback yields zeros for types it cannot decode).  `threads` is
 * accepted for signature compatibility and ignored. */
void matmul_q_fused(float* out, const float* x, const void* w, uint32_t type, int n, int d, int threads);

/* ---------------------------------------------------------------------------
 * Part 2: additive API.
 * -------------------------------------------------------------------------*/

/* Error codes.  The reference-compatible calls return void and keep the
 * reference's degrade-to-zeros behaviour; the first failure since the last
 * quantr_gpu_clear_error() is kept and readable here. */
enum {
    QUANTR_OK = 0,
    QUANTR_ERR_CUDA = 1,             /* a CUDA runtime call failed */
    QUANTR_ERR_NO_DEVICE = 2,        /* no usable CUDA device */
    QUANTR_ERR_BAD_ARG = 3,          /* NULL pointer / negative size / bad stride */
    QUANTR_ERR_UNSUPPORTED_TYPE = 4, /* type is not F32/Q8_0/Q4_K/Q5_K/Q6_K */
    QUANTR_ERR_OOM = 5,              /* device or pinned allocation failed */
    QUANTR_ERR_DEVICE_TIMEOUT = 6,   /* a bounded in-kernel wait gave up */
    QUANTR_ERR_TOO_LARGE = 7,        /* shape exceeds a kernel limit */
    QUANTR_ERR_WORKSPACE = 8,        /* caller workspace too small */
    QUANTR_ERR_ROUTING = 9,          /* a token's router probabilities were not finite */
    QUANTR_ERR_UNREGISTERED = 10     /* host weights not covered by quantr_gpu_register_weights */
};
int quantr_gpu_last_error(void);
void quantr_gpu_clear_error(void);
const char* quantr_gpu_error_string(int code);

/* Selects the CUDA device used by the Part 1 calls (default: device 0, or
 * $QUANTR_DEVICE).  Idempotent; Part 1 calls initialise lazily. */
int quantr_gpu_init(int device);
/* Releases device buffers, registrations and the stream. */
void quantr_gpu_shutdown(void);
/* Number of kernel launches this library has issued (all devices). */
uint64_t quantr_gpu_launch_count(void);

/* Uploads `bytes` of read-only weights at host address `host` (e.g. the whole
 * GGUF mapping, src/model.c:451-482) once; later Part 1 calls whose `w` lies
 * inside a registered range read the device copy.  Overlapping ranges are
 * rejected.  The host bytes must not change while registered. */
int quantr_gpu_register_weights(const void* host, size_t bytes);
int quantr_gpu_unregister_weights(const void* host);
/* Device address backing host address `host`, or NULL if unregistered. */
void* quantr_gpu_device_ptr(const void* host);

/* B independent matmul_q_fused calls sharing the weights: out is B x n and x
 * is B x d, both row-major host arrays.  Oracle: B separate reference calls. */
void matmul_q_fused_batch(float* out, const float* x, const void* w, uint32_t type, int n, int d, int B);

/* ---- stream-ordered device API (all pointers are device pointers) ------ */

/* Workspace bytes quantr_gemv_dev needs for B tokens of d columns. */
size_t quantr_gemv_workspace_bytes(int d, int B);

/* out[t*ldo + r] = row_r(w) . x[t*ldx ...] for t < B, r < n, with on-device Q8_0
 * quantization of x into `workspace`.  Asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream).  Launches use programmatic
 * dependent launch, so the weight stream of this GEMV overlaps the kernel that
 * produced x.  With B >= 2 (16-byte aligned quantized weights) the GEMV runs
 * on the tensor cores: the first call for a given (w, type, n, d, B, x, ldx,
 * out, ldo) plans it and allocates its activation tiles (up to 64 such plans
 * are kept per process); later calls allocate nothing.  Returns a QUANTR_*
 * code. */
int quantr_gemv_dev(float* out, long long ldo, const float* x, long long ldx, const void* w, uint32_t type,
                    int n, int d, int B, void* workspace, size_t workspace_bytes, void* stream);

/* Q8_0 quantization of B rows of k floats into packed block_q8_0 arrays
 * (B * (k/32) blocks), bit-identical to the reference quantize_row_q8_0. */
int quantr_quantize_q8_0_dev(block_q8_0* y, const float* x, long long ldx, int k, int B, void* stream);

/* dequantize_row (src/quant.c:160-240) of `rows` packed rows of n elements,
 * row r at src + r*src_stride bytes, into out[r*ldo ...]; elements past the
 * last whole block are left untouched, as in the reference.  Q8_0/Q4_K/Q5_K/
 * Q6_K.  (The expert-parallel MoE dequantizes the Q8_0 activation rows it
 * receives with it; re-quantizing them reproduces the sender's blocks.) */
int quantr_dequantize_rows_dev(float* out, long long ldo, const void* src, long long src_stride, uint32_t type, int n,
                               int rows, void* stream);

/* GEMV over already-quantized activations given as packed block_q8_0 rows
 * (B rows of d/32 blocks): the device counterpart of B vec_dot calls per row. */
int quantr_gemv_q8act_dev(float* out, long long ldo, const block_q8_0* xq, const void* w, uint32_t type,
                          int n, int d, int B, void* workspace, size_t workspace_bytes, void* stream);

/* Debug variant of quantr_gemv_dev that also writes the int32 partial sums of
 * every 32-element unit: isum/bsum[(t*n + r)*U + u], U = units per row
 * (d/32 for Q8_0, 8*(d/256) for the K types).  isum is sum(w_q * x_q) (Q6_K:
 * w_q already offset by -32), bsum is sum(x_q).  Used by the parity tests to
 * pin the integer stage bit for bit. */
int quantr_gemv_partials_dev(float* out, int32_t* isum, int32_t* bsum, const float* x, const void* w,
                             uint32_t type, int n, int d, int B, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Device error word of the current device (DEVICE_TIMEOUT if any bounded
 * in-kernel wait gave up since the last reset, including waits of
 * quantr_gemv_noalloc_dev calls); synchronises `stream`.  reset != 0 clears
 * the recorded error. */
int quantr_gpu_device_status(void* stream, int reset);

/* ---- GEMV programs: many independent GEMVs per launch ------------------ */

/* One GEMV of a program: out[t*ldo + r] = row_r(w) . x[t*ldx ...] for t < B,
 * with the reference's numerics (the same as matmul_q_fused per token).  All pointers are device pointers; w must be 16-byte aligned and
 * readable up to the next 16-byte boundary past its last row (every cudaMalloc
 * allocation and registered range is).  Jobs of one token run on the dp4a
 * engine, jobs of 2..64 tokens on the tensor cores (tcgen05 kind::i8), wider
 * jobs (a prefill chunk) as 64-token slices on the tensor cores. */
typedef struct {
    const void* w;
    uint32_t type;       /* QUANTR_TYPE_Q8_0 / Q4_K / Q5_K / Q6_K */
    int n, d, B;
    const float* x;
    long long ldx;
    float* out;
    long long ldo;
} quantr_gemv_job;

typedef struct quantr_program quantr_program;

/* Plans a program on the current device: tiles every job, lays out the
 * quantized activations (inputs shared by several jobs are quantized once)
 * and uploads the job table.  The jobs are independent: no job may read
 * another job's output within one run (chain dependent GEMVs as separate
 * runs, or separate programs, on one stream).  This call allocates; runs do
 * not.  No counterpart in the reference, whose runtime issues one
 * matmul_q_fused per GEMV (src/runtime.c:124-287); a program is the batched
 * device form of such a sequence. */
int quantr_program_create(quantr_program** prog, const quantr_gemv_job* jobs, int njobs);
/* Runs the program on `stream` (per kernel kind used: an activation quantizer
 * launch, then the persistent GEMV kernel; programmatic dependent launch
 * between them). */
int quantr_program_run(quantr_program* prog, void* stream);
void quantr_program_destroy(quantr_program* prog);
/* Work items (row tiles), persistent CTAs and shared memory per CTA. */
int quantr_program_info(const quantr_program* prog, int* items, int* grid, int* smem_bytes);

/* ---- routed mixture-of-experts FFN block -------------------------------- */

/* One expert projection: E matrices of one type and shape.  Expert e lives at
 * base + e*stride (the merged *_exps tensors, src/model.c:409-419) or, when
 * table is non-NULL, at table[e] (a device array of E device pointers: the
 * per-expert tensors of src/model.c:421-435). */
typedef struct {
    const void* base;
    long long stride;
    const void* const* table;
    uint32_t type; /* QUANTR_TYPE_Q8_0 / Q4_K / Q5_K / Q6_K */
} quantr_expert_weights;

/* Workspace bytes quantr_moe_dev needs (also enough for the three stage calls
 * below with the same T, E, k, dim, hidden; the experts stage may pass its
 * local expert count as E). */
size_t quantr_moe_workspace_bytes(int T, int E, int k, int dim, int hidden);

/* The reference's routed-MoE branch (src/runtime.c:202-269) for T tokens, each
 * as one forward_runtime call would compute it: router logits (F32 matmul of
 * `router`, E x dim, in matmul_ref order; or the given T x E `logits` when
 * router is NULL), softmax, top-k by repeated strict arg-max, renormalised
 * weights, and per selected expert in order hb = W1.xb, hb2 = W3.xb,
 * hb = silu(hb)*hb2, o = W2.hb, out += o*ew from out = 0.  W1 is the tensor
 * the reference binds to ffn_up; W1/W3 are hidden x dim, W2 dim x hidden.
 * out is T x dim (out[t*ldo + i]); the caller adds the residual (x += out).
 * sel / wts (T x k, optional) receive the routing.  E <= 256, k <= 16
 * (the reference's fixed buffers), k <= E.  All expert GEMVs are bit-identical
 * to matmul_q_fused; softmax and silu use correctly rounded expf, which can
 * differ from glibc's expf in the last bit.  A token whose probabilities are
 * not finite (NaN logits) gets no experts and out = 0, and the device status
 * reports QUANTR_ERR_ROUTING.  The workspace must be 256-byte aligned.
 * Asynchronous on `stream`.  From 16 tokens on the expert GEMVs run on the
 * tensor cores: the first call with a given configuration (shapes, weight
 * descriptors, xb, workspace and output pointers) plans those launches, which
 * allocates their job tables and, for a pointer table of experts, reads the
 * table once; make that first call before any stream capture.  Later calls
 * with the same configuration allocate nothing. */
int quantr_moe_dev(float* out, long long ldo, const float* xb, long long ldx, int T, const float* router,
                   const float* logits, long long ldl, int E, int k, const quantr_expert_weights* w1,
                   const quantr_expert_weights* w3, const quantr_expert_weights* w2, int dim, int hidden, int* sel,
                   float* wts, void* workspace, size_t workspace_bytes, void* stream);

/* The same block as three stream-ordered stages, for expert-parallel use
 * (each rank routes every token identically, computes only its experts, and
 * the per-pair outputs are exchanged before the combine):
 *   route:   sel/wts (T x k) from router weights or logits, as above;
 *   experts: for every pair p = t*k + s with sel[p] in [e0, e0 + E_local),
 *            o[p*dim + i] = (W2.(silu(W1.xb_t) * (W3.xb_t)))_i of expert
 *            sel[p] (w1/w3/w2 describe the E_local local experts, expert
 *            sel[p] - e0); rows of o of other pairs are left untouched;
 *   combine: out[t*ldo + i] = sum over s in selection order of
 *            o[(t*k+s)*dim + i] * wts[t*k+s] from +0.0, skipping sel < 0
 *            (src/runtime.c:241, 262-264). */
int quantr_moe_route_dev(int* sel, float* wts, const float* xb, long long ldx, int T, const float* router,
                         const float* logits, long long ldl, int E, int k, int dim, void* workspace,
                         size_t workspace_bytes, void* stream);
int quantr_moe_experts_dev(float* o, const float* xb, long long ldx, int T, const int* sel, int k, int e0, int E_local,
                           const quantr_expert_weights* w1, const quantr_expert_weights* w3,
                           const quantr_expert_weights* w2, int dim, int hidden, void* workspace,
                           size_t workspace_bytes, void* stream);
int quantr_moe_combine_dev(float* out, long long ldo, const float* o, const int* sel, const float* wts, int T, int k,
                           int dim, void* stream);

/* The shared expert of a Qwen1.5-MoE-style block, added after the routed
 * experts (no counterpart in the reference, which loads no shared expert,
 * src/model.c:401-446; restated from its dense FFN, src/runtime.c:270-284):
 * for every token t, out[t*ldo + i] += o_i * g with
 * o = W2.(silu(W1.xb_t) * (W3.xb_t)) (W1 the gate projection, hidden x dim;
 * W3 up, hidden x dim; W2 down, dim x hidden; the same GEMVs and SwiGLU as
 * the dense FFN) and g = 1/(1 + expf(-(gate . xb_t))), gate . xb_t in
 * matmul_ref order, the add a single fp32 add after the routed sum.  ldo must
 * equal dim.  Device pointers, asynchronous on `stream`; the first call with
 * a configuration (pointers, T, shapes) plans the GEMVs and allocates their
 * buffers - make it before any stream capture - later calls allocate
 * nothing. */
int quantr_moe_shared_dev(float* out, long long ldo, const float* xb, long long ldx, int T, const float* gate,
                          const void* w1, uint32_t t1, const void* w3, uint32_t t3, const void* w2, uint32_t t2,
                          int dim, int hidden, void* stream);

/* Host-pointer, synchronous form for the reference's runtime: w1/w3/w2 are the
 * per-layer arrays of E expert pointers (w->expert_w1[l], ..., include/types.h:
 * 68-70), each inside a range registered with quantr_gpu_register_weights
 * (else QUANTR_ERR_UNREGISTERED); router is w->ffn_gate_inp[l] (E x dim F32,
 * registered or not) or NULL with `logits` given.  On failure out is zeroed and
 * the sticky error is set.  Returns a QUANTR_* code. */
int quantr_moe_layer(float* out, const float* xb, int T, const float* router, const float* logits, int E, int k,
                     const void* const* w1, uint32_t t1, const void* const* w3, uint32_t t3, const void* const* w2,
                     uint32_t t2, int dim, int hidden, int* sel, float* wts);

/* ---- device-resident decoder (forward_runtime on the GPU) -------------- */

/* A decoder model: the reference's Config and TransformerWeights
 * (include/types.h:19-71) flattened into per-layer arrays.  Every tensor
 * pointer is a HOST address inside a range registered with
 * quantr_gpu_register_weights (the GGUF mapping, the normal case: resolved to
 * the device copy), a device address, or any other host address (uploaded
 * once into memory the decoder owns).  Weight tensors must be 16-byte aligned
 * (GGUF aligns tensors to 32 bytes, src/gguf.c:130-140).  Types are GGML ids;
 * linears may be Q8_0/Q4_K/Q5_K/Q6_K, the router and norms F32, the embedding
 * any type dequantize_row reads (row bytes token_embd_row_bytes; 0 = an F32
 * table).  The reference's fields come first in its own order; head_dim and
 * the shared expert are additions with no counterpart in the reference:
 *   head_dim          0 = dim / n_heads (src/runtime.c:102); otherwise the
 *                     query has n_heads*head_dim elements (Wq is that x dim,
 *                     Wo dim x that) and RoPE runs over all of them;
 *   shexp_*           a shared expert after the routed ones (Qwen1.5-MoE):
 *                     xb2 += (Ws2.(silu(Ws1.xb) * Ws3.xb)) * sigmoid(gate.xb),
 *                     Ws1 the gate projection like the dense FFN's W1. */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
    float rope_freq_base;                   /* <= 0: 10000 (src/runtime.c:24) */
    int expert_count, expert_used_count;    /* 0 experts: dense SwiGLU FFN */
    int kv_type;                            /* 0 = fp32 KV cache, 1 = fp16 (src/runtime.c:74-92) */
    const void* token_embd;
    uint32_t token_embd_type;
    size_t token_embd_row_bytes;
    const float* const* rms_att;
    const float* const* rms_ffn;
    const void* const* wq;
    const void* const* wk;
    const void* const* wv;
    const void* const* wo;
    const void* const* w1;                  /* dense FFN gate (SiLU side) */
    const void* const* w2;                  /* dense FFN down */
    const void* const* w3;                  /* dense FFN up */
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
    const float* const* ffn_gate_inp;       /* router, expert_count x dim F32 */
    const void* const* const* expert_w1;    /* [layer][expert]: the loader's ffn_up (SiLU side) */
    const void* const* const* expert_w2;
    const void* const* const* expert_w3;
    const uint32_t* exp_w1_type;
    const uint32_t* exp_w2_type;
    const uint32_t* exp_w3_type;
    int head_dim;
    int shexp_hidden_dim;                   /* 0 = no shared expert */
    const void* const* shexp_w1;
    const void* const* shexp_w2;
    const void* const* shexp_w3;
    const uint32_t* shexp_w1_type;
    const uint32_t* shexp_w2_type;
    const uint32_t* shexp_w3_type;
    const float* const* shexp_gate;         /* dim F32 per layer */
} quantr_model;

typedef struct quantr_decoder quantr_decoder;

/* Builds a decoder for `batch` independent sequences on the current device:
 * resolves or uploads every weight, allocates the KV caches
 * (n_layers x batch x seq_len x n_kv_heads*head_dim, fp32 or fp16) and the
 * activations, plans every GEMV, computes the RoPE cos/sin table with the
 * host C library's powf/cosf/sinf exactly as src/runtime.c:19-41 does per
 * call, and captures one decode step and one prefill step as CUDA graphs.
 * Every later call allocates nothing.  No counterpart in the reference (its
 * RunState is malloc_run_state, src/model.c:101-150). */
int quantr_decoder_create(quantr_decoder** dec, const quantr_model* m, int batch);
void quantr_decoder_destroy(quantr_decoder* dec);

/* forward_runtime (src/runtime.c:94-289) for every sequence b < batch:
 * token tokens[b] at position pos[b] (0 <= pos < seq_len; the KV cache of
 * sequence b), logits[b*ldl + v] (may be NULL) and the greedy next token
 * next[b] (src/sampling.c:125-131; may be NULL).  Device pointers,
 * asynchronous on `stream`.  Results are bit-identical to the reference's
 * scalar build. */
int quantr_decoder_step_dev(quantr_decoder* dec, const int* tokens, const int* pos, float* logits, long long ldl,
                            int* next, void* stream);

/* The reference CLI's generation loop (src/main.c:305-317) for every sequence
 * at once, on the device: sequential prefill of the n_prompt prompt tokens
 * (prompt[b*n_prompt + i]; src/runtime.c:294-304), then the last prompt token
 * again at position n_prompt and `steps` greedy tokens (out[b*steps + i]),
 * positions wrapping at seq_len.  Host arrays; synchronous.  One CUDA-graph
 * replay per position, no host round trip between steps. */
int quantr_decoder_generate(quantr_decoder* dec, const int* prompt, int n_prompt, int steps, int* out);

/* quantr_decoder_generate with device arrays, asynchronous on `stream`:
 * prompt is batch x n_prompt, out receives the greedy tokens step-major
 * (out[i*batch + b]); steps <= max(seq_len, 4096). */
int quantr_decoder_generate_dev(quantr_decoder* dec, const int* prompt, int n_prompt, int steps, int* out,
                                void* stream);
/* Kernel launches (graph nodes) of one decode step and one prefill step. */
int quantr_decoder_launches(const quantr_decoder* dec, int* decode_step, int* prefill_step);

/* Drop-in shapes of the reference's runtime calls for sequence 0 (host
 * values, synchronous): forward_runtime's logits (vocab floats, valid until
 * the next call) and prefill_runtime. */
const float* quantr_forward_runtime(quantr_decoder* dec, int token, int pos);
void quantr_prefill_runtime(quantr_decoder* dec, const int* tokens, int n_tokens);

/* The decoder's KV caches (device memory, `bytes` each): element i of head h
 * at position t of sequence b in layer l is at
 * (((l*batch + b)*n_kv_heads + h)*seq_len + t)*head_dim + i, fp32 or fp16
 * per kv_type.  For restoring a saved context (the reference keeps its cache
 * in RunState, src/model.c:128-137) or seeding one. */
int quantr_decoder_kv(const quantr_decoder* dec, void** key_cache, void** value_cache, size_t* bytes);

/* Bytes the decode step reads that do not depend on the position (weights of
 * one token: every linear, the head, the norms, one embedding row) and the
 * KV-cache bytes it reads per position, per sequence. */
int quantr_decoder_info(const quantr_decoder* dec, size_t* weight_bytes_per_step, size_t* kv_bytes_per_position,
                        size_t* device_bytes);

/* Test hook: out[i] = the device's expf (the C library's method, used by the
 * decoder's softmax and silu and by the MoE block) of the float whose bit
 * pattern is first + i, for i < n.  Lets a test compare it with the host C
 * library's expf over every float.  Asynchronous on `stream`. */
int quantr_debug_expf_dev(float* out, uint32_t first, long long n, void* stream);

/* Allocation-free quantized GEMV.  No counterpart in the reference: an
 * addition for callers that cannot call cudaMalloc - embedders whose own
 * memory manager owns all device memory, plugin hosts that pass only input and
 * output buffers, and latency-critical paths that cannot take cudaMalloc's
 * implicit synchronisation.  Same arguments and results as quantr_gemv_dev
 * (Q8_0/Q4_K/Q5_K/Q6_K only), but the quantized activations live in a fixed
 * scratch array inside the library (QUANTR_NOALLOC_SCRATCH_BYTES, held by every
 * GPU that loads the library until exit) and nothing is allocated or freed.
 * Limit: 256 + quantr_gemv_workspace_bytes(d, B) must not exceed
 * QUANTR_NOALLOC_SCRATCH_BYTES (1 MiB: B * (d/32) up to 26,180 activation
 * blocks, e.g. d up to 52,360 at B = 16); larger shapes return
 * QUANTR_ERR_TOO_LARGE.  The
 * first call on each device looks up the scratch address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls on a device share the one array: calls that overlap on the GPU
 * (different streams, or other threads) race, so serialise them.  The call is
 * asynchronous and returns QUANTR_OK once its launches are queued; a bounded
 * in-kernel wait that gave up is recorded in the array's error word and stays
 * recorded until quantr_gpu_device_status(stream, 1) reports and clears it
 * (QUANTR_ERR_DEVICE_TIMEOUT), as for quantr_gemv_dev.  The cached scratch
 * address belongs to the device's primary context: do not call this entry
 * point after cudaDeviceReset in the same process.  It always runs the
 * one-launch-per-GEMV kernel (the persistent engine that quantr_gemv_dev uses
 * for aligned decode shapes keeps a cached plan in allocated memory), so it is
 * slower than quantr_gemv_dev at batch 1-16, with identical results. */
#define QUANTR_NOALLOC_SCRATCH_BYTES (1u << 20)
int quantr_gemv_noalloc_dev(float* out, long long ldo, const float* x, long long ldx, const void* w,
                            uint32_t type, int n, int d, int B, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* QUANTR_CUDA_H */
