// kernels.cuh -- launch interface of the quantized-GEMV kernels (internal; the
// public C ABI is include/quantr_cuda.h).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <vector>

#include "quantr_cuda.h"

namespace qr {

// Quantized activations in the layout the GEMV kernels read: for token t and
// 32-element block b, q[(t*nbx + b)*32 .. +31] are the int8 quants (natural
// element order), d[t*nbx + b] the fp32 decode of the block's fp16 scale and
// s[t*nbx + b] the int32 sum of its quants (the K-quant min term needs it).
struct ActQ {
    int8_t* q;
    float* d;
    int32_t* s;
    int nbx;  // blocks per token
};

// Bytes of workspace an ActQ for B tokens of d columns needs (40 per block).
size_t actq_bytes(int d, int B);
ActQ actq_carve(void* ws, int d, int B);

// Device error word written by kernels whose bounded waits give up.
enum : int { DEV_OK = 0, DEV_ERR_WAIT_TIMEOUT = 1, DEV_ERR_ROUTING = 2 };

struct LaunchCfg {
    cudaStream_t stream = nullptr;
    bool pdl = true;  // programmatic dependent launch on this stream
};

// x: B rows of ldx floats -> ActQ (skipped when a.q is null) and, if blocks
// is non-null, the reference's packed block_q8_0 array (B*nbx blocks of 34
// bytes).  If err_reset is non-null the kernel zeroes that error word first,
// so a following GEMV on the same stream reports only its own timeouts.
cudaError_t launch_quantize(const float* x, long long ldx, int d, int B, ActQ a,
                            uint8_t* blocks, int* err_reset, const LaunchCfg& c);

// Packed block_q8_0 activations (B*nbx blocks) -> ActQ.
cudaError_t launch_repack(const uint8_t* blocks, int nbx, int B, ActQ a, const LaunchCfg& c);

struct GemvArgs {
    const uint8_t* w = nullptr;  // packed rows, n * row_bytes(type, d)
    uint32_t type = 0;
    int n = 0, d = 0;
    ActQ x{};
    float* out = nullptr;
    long long ldo = 0;  // out[t*ldo + r]
    int B = 1;
    int32_t* dbg_isum = nullptr;  // optional per-unit partials, [B][n][U]
    int32_t* dbg_bsum = nullptr;
    int* err = nullptr;           // device error word (may be null)
};

// Quantized GEMV over already-quantized activations.
cudaError_t launch_gemv(const GemvArgs& g, const LaunchCfg& c);

// F32 weights (type 0): out[t*ldo + r] = sequential sum_j w[r*d+j]*x[t*ldx+j].
cudaError_t launch_gemv_f32(const float* w, const float* x, long long ldx, float* out,
                            long long ldo, int n, int d, int B, const LaunchCfg& c);

// Reference dequantize_row on device (src/quant.c:160-240).
cudaError_t launch_dequantize(float* out, const uint8_t* src, uint32_t type, int n,
                              const LaunchCfg& c);

// dequantize_row of `rows` packed rows (row r at src + r*src_stride) into
// out[r*ldo ...] (elements past the last whole block are left untouched).
cudaError_t launch_dequantize_rows(float* out, long long ldo, const uint8_t* src, long long src_stride, uint32_t type,
                                   int n, int rows, const LaunchCfg& c);

int device_sm_count();

// Kernel launches issued by this library since load.
unsigned long long launch_count();

// Per-device error word that kernels launched through the device API report
// bounded-wait timeouts into (allocated on first use; api.cu).
int* device_error_word();

// Error word of the allocation-free GEMV (noalloc.cu) on the current device;
// reset != 0 clears a recorded error.  DEV_OK if that path never ran here.
int noalloc_device_error(int reset);

// Single GEMV through the persistent engine (engine.cu): x is quantized into
// `ws` (engine_act_bytes of it) and the engine program runs one job.  Returns
// cudaErrorNotSupported when the engine cannot take the call (unaligned
// weights, B > 16, workspace too small, shape too large), so the caller can
// use launch_quantize + launch_gemv instead.
cudaError_t launch_gemv_engine(const uint8_t* w, uint32_t type, int n, int d, int B, const float* x,
                               long long ldx, float* out, long long ldo, void* ws, size_t ws_bytes, int* err,
                               cudaStream_t stream);
size_t engine_act_bytes(uint32_t type, int d, int B);

// ---- tensor-core GEMV programs for batched tokens (tc.cu) ----

// One GEMV: out[t*ldo + r] = row_r(w) . x[t*ldx ...] for t < B, r < n.
struct GemvJobIn {
    const uint8_t* w;  // 16-byte aligned packed rows
    uint32_t type;
    int n, d, B;
    const float* x;
    long long ldx;
    float* out;
    long long ldo;
    // Gathered job (the pairs routed to one MoE expert; tensor-core path
    // only): counts[e] live columns (a device value an earlier launch
    // writes), processed B = 16 at a time; column i stands for the pair
    // list[offsets[e] + i], its output row.  Its activations are operand
    // tiles (act/ds), one set of U units per 16 columns.  Null counts: all B
    // columns live, output row = column.
    const int* g_counts = nullptr;
    const int* g_offsets = nullptr;
    const int* g_list = nullptr;
    int g_e = 0;
    // Activations already quantized into operand tiles ([U] x N x 32 bytes)
    // and records ([U] x N x 16 bytes, tensor-core layout): x is unused.
    const uint8_t* act = nullptr;
    const uint8_t* ds = nullptr;
    // Non-null: the GEMV input is silu(x) * xmul elementwise (the reference's
    // SwiGLU product feeding the down projection), formed by the quantizer.
    const float* xmul = nullptr;
};

// Plans a tensor-core program (B <= kTcMaxB per job, at most kTcMaxJobs
// jobs): allocates the activation operand buffer and the device job table.
// Runs are two launches (quantizer, persistent tcgen05 kernel) and allocate
// nothing.
struct TcPlan;
constexpr int kTcMaxB = 64;
constexpr int kTcMaxJobs = 128;
int tc_plan_create(const GemvJobIn* jobs, int njobs, TcPlan** out);
// A tensor-core job list with fewer 128-row tiles than SMs leaves most SMs
// idle while a few run long epilogues: splits the widest job's tokens in two
// (16-aligned) until every SM has a tile (results do not change).
void tc_split_narrow(std::vector<GemvJobIn>& jobs, int sms);
// One GEMV of 2+ tokens on the tensor cores, planned (and its activation
// tiles allocated) on the first call for these arguments and cached;
// cudaErrorNotSupported for shapes the tensor-core kernel does not take.
cudaError_t launch_gemv_tc(const uint8_t* w, uint32_t type, int n, int d, int B, const float* x, long long ldx,
                           float* out, long long ldo, int* err, cudaStream_t stream);
cudaError_t tc_plan_run(TcPlan* plan, int* err, cudaStream_t stream);
void tc_plan_destroy(TcPlan* plan);
void tc_plan_info(const TcPlan* plan, int* items, int* grid, int* smem);

// Where a program's persistent-engine jobs expect one input's quantized
// activations: the engine layout of k_quant_tasks (int8 quants of unit u of
// token t at act[(t*U + u)*32 + perm(type, e)], records (fp32 decoded scale,
// fp32 quant sum) at act + ds_off, K-quant units stored sub-block-major).
struct ActTarget {
    uint8_t* act;
    uint32_t ds_off;
    int U, B, type;
};
// Targets of input x (one per element order the jobs reading x need); returns
// how many (<= max).  0 when x is not an engine input of the program.
int program_act_targets(const quantr_program* p, const float* x, ActTarget* out, int max);
// When on, quantr_program_run skips the engine's activation quantizer: the
// caller's kernel writes every target before the program runs.  Only for
// programs whose every job runs on the engine (one token, no SwiGLU input).
int program_external_quant(quantr_program* p, bool on);

// quantr_program_create with, per job, an optional second input: a non-null
// xmul[j] makes job j's input silu(x) * xmul (same shape and strides as x),
// formed inside the activation quantizer.  xmul may be null (no job has one).
int program_create_ex(quantr_program** out, const quantr_gemv_job* jobs, const float* const* xmul, int njobs);

// ---- routed MoE block (moe.cu) ----

// The reference's fixed routing buffers: router_logits[256], active_experts[16]
// (src/runtime.c:204, 210).
constexpr int kMoeMaxExperts = 256;
constexpr int kMoeMaxK = 16;

// E matrices of one expert projection: expert e at base + e*stride, or
// table[e] (a device array of device pointers) when table is non-null.
struct ExpertMats {
    const uint8_t* base = nullptr;
    long long stride = 0;
    const uint8_t* const* table = nullptr;
    uint32_t type = 0;
};

// Routing for T tokens: logits = router.xb (F32, matmul_ref order) or the
// given logits; softmax, strict arg-max top-k, renormalisation -> sel/wts
// (T x k; a token with non-finite probabilities gets sel = -1, wts = 0 and the
// error word DEV_ERR_ROUTING).
struct MoeRoute {
    int* sel = nullptr;
    float* wts = nullptr;
    const float* xb = nullptr;
    long long ldx = 0;
    int T = 0;
    const float* router = nullptr;
    const float* logits = nullptr;
    long long ldl = 0;
    int E = 0, k = 0, dim = 0;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int* err = nullptr;
};

// Expert FFNs of the pairs p = t*k + s with sel[p] in [e0, e0 + El):
// o[p*dim + i] = (W2_e . (silu(W1_e.xb_t) * (W3_e.xb_t)))_i for local expert
// e = sel[p] - e0.  Rows of o for other pairs are not written.
struct MoeExperts {
    float* o = nullptr;  // (T*k) x dim
    const float* xb = nullptr;
    long long ldx = 0;
    int T = 0;
    const int* sel = nullptr;
    int k = 0, e0 = 0, El = 0, dim = 0, hidden = 0;
    ExpertMats w1, w3, w2;  // local experts 0..El-1; w1/w3 hidden x dim, w2 dim x hidden
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int* err = nullptr;
};

// Workspace bytes for T tokens, E experts (route: E = all experts; experts
// stage: E = local experts; the full-E figure covers both).
size_t moe_workspace_bytes(int T, int E, int k, int dim, int hidden);
cudaError_t launch_moe_route(const MoeRoute& r, const LaunchCfg& c);
cudaError_t launch_moe_experts(const MoeExperts& a, const LaunchCfg& c);
// out[t*ldo + i] = sum over s in order of o[(t*k+s)*dim + i] * wts[t*k+s]
// from +0.0, skipping slots with sel < 0 (src/runtime.c:241, 262-264).
cudaError_t launch_moe_combine(float* out, long long ldo, const float* o, const int* sel, const float* wts, int T,
                               int k, int dim, const LaunchCfg& c);

} // namespace qr
