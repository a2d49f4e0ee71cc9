// decode_persist.cuh -- parameters of the persistent one-token decode kernel
// (decode_persist.cu), shared with the decoder's host code (decode.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace qr {
namespace dp {

constexpr int kPersistThreads = 512;
// Longest activation vector the kernel's quantizers take (12 blocks of 32 per warp).
constexpr int kPersistMaxVec = 12 * (kPersistThreads / 32) * 32;

// One GEMV stage of a layer: up to three matrices of one type and width
// whose rows are concatenated (Wq|Wk|Wv, Wo, W1|W3, W2); rows are split
// evenly over the CTAs.
struct Stage {
    int nmat;
    const uint8_t* w[3];  // device, 16-byte aligned, rb % 16 == 0
    int rows[3];
    float* out[3];        // output vector of each matrix
    int rb;               // bytes per row
    int U;                // 32-element units per row
    long long total;      // rows of all matrices
};

struct LayerW {
    const float* rms_att;
    const float* rms_ffn;
};

// Shared-memory carve-up (byte offsets).
struct SmemLayout {
    uint32_t bar, xs, xq, xd, xsum, terms, r0, r1;
};

struct Params {
    const LayerW* layers;  // device [L]
    const Stage* stages;   // device [L][4]
    int L;
    int dim, q_dim, kv_dim, hd, n_heads, n_kv, kv_mul, hidden, seq_len, vocab, kv_type;
    float inv_sqrt;
    const int* tok;
    const int* pos;
    const uint8_t* embd;
    uint32_t embd_type;
    long long embd_rb;  // 0: F32 table
    float* X[2];        // residual stream ping-pong; X[0] holds it after the last layer
    float* q;
    float* kc;
    float* vc;
    float* xa;
    float* delta;  // branch output (O, then W2); the caller adds the last one
    float* h1;
    float* h3;
    void* kcache;
    void* vcache;
    long long layer_kv;  // cache elements per layer (head-major rows)
    const float2* rope;
    unsigned* bar;  // grid-barrier counter, zeroed before every launch
    int* err;
    SmemLayout sm;
};

} // namespace dp

// Shared memory the kernel needs for these stages at `grid` CTAs (fills
// p.sm); QUANTR_ERR_TOO_LARGE if above the per-CTA limit.
int persist_layout(dp::Params& p, uint32_t type, int grid, size_t* smem);
cudaError_t persist_set_smem(uint32_t type, int kv_type, size_t smem);
// The kernel for a linear type and KV type (for occupancy queries).
const void* persist_kernel(uint32_t type, int kv_type);
// Zeroes the barrier counter and launches the kernel (cooperative, `grid`
// CTAs of kPersistThreads) on s.
cudaError_t launch_persist(const dp::Params& p, uint32_t type, int grid, size_t smem, cudaStream_t s);

} // namespace qr
