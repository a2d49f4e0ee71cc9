// decode.cu -- the reference's decoder step, forward_runtime
// (src/runtime.c:94-289), resident on the device, for `batch` independent
// sequences, and its generation loop (src/main.c:305-317).
//
// One step is a fixed sequence of stream-ordered launches, captured once as a
// CUDA graph and replayed per position; token ids, positions and the step
// counters live in device memory, so prefill and greedy decoding run without
// a host round trip between positions.  Per layer:
//   rmsnorm       x += delta (the previous residual branch), xb = rmsnorm(x)
//                 (src/kernels.c:179-189: sequential sum of squares)
//   Q/K/V         one GEMV program over xb (csrc/engine.cu for one token,
//                 csrc/tc.cu tensor cores for 2-64)
//   scores        RoPE (adjacent pairs, cos/sin table; src/runtime.c:19-41)
//                 fused with the K/V store (:74-92, 129-132) and q.k per
//                 (head, position) * 1/sqrt(head_dim) (:139-157)
//   softmax + V   per KV head: max, expf, sequential sum, normalise, value
//                 rows accumulated position by position (:159-194)
//   O             GEMV program -> delta; rmsnorm (x += delta)
//   FFN           dense: W1/W3 program, W2 program whose activation quantizer
//                 forms silu(h1)*h3 -> delta (:270-284); MoE: route/experts/
//                 combine stages
//                 (csrc/moe.cu, :202-269), plus the optional shared expert
// then the final rmsnorm, the head GEMV (:286-287) and the greedy pick
// (src/sampling.c:125-131).  Every floating-point operation is the
// reference's, in its order and rounding (explicit __f*_rn intrinsics; expf
// from libm_ref.cuh), so the logits are bit-identical to its scalar build.
//
// The RoPE cos/sin values depend only on (position, index): they are
// computed once per decoder on the host with the C library's powf/cosf/sinf,
// the functions the reference calls per token, and read from a table.
#include "quantr_cuda.h"

#include "decode_persist.cuh"
#include "device_common.cuh"
#include "engine_act.cuh"
#include "formats.cuh"
#include "kernels.cuh"
#include "launch_util.cuh"
#include "libm_ref.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace qr {
namespace dec {

constexpr int kMaxBatch = 1024;
constexpr size_t kSmemMax = 227 * 1024;

enum : int { MODE_EXPLICIT = 0, MODE_PREFILL = 1, MODE_DECODE = 2, MODE_PREFILL_CHUNK = 3 };

// Device control block: what the feed kernel at the start of each step does.
struct Ctl {
    int mode;
    int n_prompt;
    int step;   // next prefill position
    int dstep;  // decode steps taken
    int ring;   // capacity (steps) of the output ring
};

// Up to three engine activation layouts to write an output into (one per
// element order the next program's weight types need); n = 0: none, the next
// program quantizes its input itself.
struct Tgts {
    int n;
    ActTarget t[3];
};

// Block b (32 elements, one warp, lane = element) of token t of an output
// that feeds a GEMV program: quantized straight into the program's layout.
__device__ __forceinline__ void tgts_write(const Tgts& tg, int t, int b, int lane, float v)
{
    for (int k = 0; k < tg.n; ++k)
        if (b < tg.t[k].U) act_write_block(tg.t[k].act, tg.t[k].ds_off, tg.t[k].U, tg.t[k].type, t, b, lane, v);
}

struct Dims {
    int B, dim, q_dim, kv_dim, hd, n_heads, n_kv, kv_mul, seq_len, hidden, vocab, kv_type;
    int vst;   // value-row stages of the attention kernel's ring (set with its shared-memory size)
    int vsth;  // the same for the one-head-per-CTA variant
    float inv_sqrt;
    int kv_B;        // sequences the KV cache holds
    int seq_stride;  // KV-cache sequence of step row b = b * seq_stride (0: every row is one sequence's position)
};

// ------------------------------------------------------------- kernels --

// Token and position of every sequence for this step (src/main.c:305-317).
__global__ void k_feed(Ctl* ctl, int* tok, int* pos, const int* prompt, const int* next, int B, int seq_len)
{
    pdl_wait();
    const int b = threadIdx.x;
    const int mode = ctl->mode, n = ctl->n_prompt;
    const int s = ctl->step, i = ctl->dstep;
    if (b < B) {
        if (mode == MODE_PREFILL) {
            tok[b] = prompt[(long long)b * n + s];
            pos[b] = s % seq_len;
        } else if (mode == MODE_DECODE) {
            tok[b] = i == 0 ? prompt[(long long)b * n + n - 1] : next[b];
            pos[b] = (n + i) % seq_len;
        } else if (mode == MODE_PREFILL_CHUNK) {
            // Rows are consecutive prompt positions of one sequence; rows
            // past the prompt get position -1 and are skipped.
            const int idx = s * B + b;
            tok[b] = idx < n ? prompt[idx] : 0;
            pos[b] = idx < n ? idx : -1;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (mode == MODE_PREFILL || mode == MODE_PREFILL_CHUNK) ctl->step = s + 1;
        if (mode == MODE_DECODE) ctl->dstep = i + 1;
    }
    pdl_trigger();
}

// x[b] = row tok[b] of the embedding table (src/runtime.c:108-113).  A token
// outside [0, vocab) reads row 0 (the reference would read out of bounds).
__global__ void k_embed(float* __restrict__ x, const int* __restrict__ tok, const uint8_t* __restrict__ table,
                        uint32_t type, long long row_bytes, int dim, int vocab)
{
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= dim) return;
    int t = tok[b];
    if (t < 0 || t >= vocab) t = 0;
    if (row_bytes == 0) {
        x[(long long)b * dim + e] = reinterpret_cast<const float*>(table)[(long long)t * dim + e];
    } else if (e < dequant_extent(type, dim)) {
        x[(long long)b * dim + e] = dequant_elem(table + (long long)t * row_bytes, type, e);
    }
}

// s = ((s + p[0]) + p[1]) + ... in fp32, left to right: the reference's
// accumulation order.  The additions form one dependent chain.
__device__ __forceinline__ float chain_sum(const float* __restrict__ p, int n, float s = 0.0f)
{
    // 32 loads in flight, then 32 dependent adds: one load latency per 32 terms.
    int i = 0;
    for (; i + 32 <= n; i += 32) {
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = p[i + k];
#pragma unroll
        for (int k = 0; k < 32; ++k) s = __fadd_rn(s, v[k]);
    }
    for (; i < n; ++i) s = __fadd_rn(s, p[i]);
    return s;
}

// x += delta (if given), out = rmsnorm(x) * w, per sequence (one CTA each).
// src/kernels.c:179-189: ss accumulated left to right, ss/size + 1e-5,
// 1/sqrtf, o = w * (x * scale).  dim % 4 == 0.  Every global access is
// issued in one round (float4, all threads) and the rest runs out of shared
// memory: the weight vector before the dependency wait, x (+ delta) after it;
// one thread then walks the sum of squares while the others wait.
constexpr int kNormThreads = 1024;  // 32 warps: the quantization tail is 2 blocks per warp at dim 2048
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm(float* __restrict__ x, const float* __restrict__ delta,
                                                 const float* __restrict__ w, float* __restrict__ out, int dim,
                                                 const __grid_constant__ Tgts tg)
{
    extern __shared__ float4 sm4[];  // xs[dim] | ws[dim]
    __shared__ float s_scale;
    const int n4 = dim >> 2;
    float4* xs4 = sm4;
    float4* ws4 = sm4 + n4;
    const float* xs = reinterpret_cast<const float*>(xs4);
    const float* wsm = reinterpret_cast<const float*>(ws4);
    const int b = blockIdx.x;
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll 4
    for (int k = threadIdx.x; k < n4; k += blockDim.x) ws4[k] = w4[k];
    pdl_wait();
    pdl_trigger();
    float4* x4 = reinterpret_cast<float4*>(x + (long long)b * dim);
    const float4* d4 = reinterpret_cast<const float4*>(delta + (long long)b * dim);
#pragma unroll 4
    for (int k = threadIdx.x; k < n4; k += blockDim.x) {
        float4 v = x4[k];
        if (delta) {
            const float4 dv = d4[k];
            v.x = __fadd_rn(v.x, dv.x);
            v.y = __fadd_rn(v.y, dv.y);
            v.z = __fadd_rn(v.z, dv.z);
            v.w = __fadd_rn(v.w, dv.w);
            x4[k] = v;
        }
        xs4[k] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = 0.0f;
        int k = 0;
        for (; k + 8 <= n4; k += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = xs4[k + u];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                ss = __fadd_rn(ss, __fmul_rn(v[u].x, v[u].x));
                ss = __fadd_rn(ss, __fmul_rn(v[u].y, v[u].y));
                ss = __fadd_rn(ss, __fmul_rn(v[u].z, v[u].z));
                ss = __fadd_rn(ss, __fmul_rn(v[u].w, v[u].w));
            }
        }
        for (int i = 4 * k; i < dim; ++i) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
        ss = __fadd_rn(__fdiv_rn(ss, (float)dim), 1e-5f);
        s_scale = __fdiv_rn(1.0f, __fsqrt_rn(ss));
    }
    __syncthreads();
    const float sc = s_scale;
    if (tg.n == 0) {
        for (int i = threadIdx.x; i < dim; i += blockDim.x)
            out[(long long)b * dim + i] = __fmul_rn(wsm[i], __fmul_rn(xs[i], sc));
        return;
    }
    // Warp per 32-element block: the normalised values also go, quantized,
    // into the next program's activation layout.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int blk = warp; blk < (dim + 31) / 32; blk += nw) {
        const int i = blk * 32 + lane;
        const float v = i < dim ? __fmul_rn(wsm[i], __fmul_rn(xs[i], sc)) : 0.0f;
        if (i < dim) out[(long long)b * dim + i] = v;
        if (blk < dim / 32) tgts_write(tg, b, blk, lane, v);
    }
}

__device__ __forceinline__ void kv_put(void* cache, int kv_type, long long idx, float v)
{
    if (kv_type == 1)
        reinterpret_cast<uint16_t*>(cache)[idx] = (uint16_t)f2h_ref(v);
    else
        reinterpret_cast<float*>(cache)[idx] = v;
}
// The value a cache of this type returns for v (the fp16 cache stores the
// reference's truncated half, src/runtime.c:74-92).
__device__ __forceinline__ float kv_round(int kv_type, float v) { return kv_type == 1 ? h2f_ref(f2h_ref(v)) : v; }
__device__ __forceinline__ float kv_get(const void* cache, int kv_type, long long idx)
{
    return kv_type == 1 ? h2f_ref(reinterpret_cast<const uint16_t*>(cache)[idx])
                        : reinterpret_cast<const float*>(cache)[idx];
}

constexpr int kScoreTile = 32;  // positions per CTA

__device__ __forceinline__ void rot(float a, float b, float2 cs, float& o0, float& o1)
{
    o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

// KV cache layout (head-major): element i of head kh at position t of
// sequence b in layer l is at layer_off + ((b*n_kv + kh)*seq_len + t)*hd + i,
// so the rows of one head are contiguous across positions (one bulk copy per
// tile of positions).  Values match the reference's cache element for
// element (src/runtime.c:129-132, 143, 181), only the addresses differ.
__device__ __forceinline__ long long kv_head_base(const Dims& D, long long layer_off, int b, int kh)
{
    return layer_off + ((long long)b * D.seq_stride * D.n_kv + kh) * D.seq_len * D.hd;
}

// K (rotated) and V rows of every step row's position into the cache, for
// steps whose rows are positions of one sequence (chunked prefill): all rows
// are stored before any row's scores read them.  Rows with pos < 0 skip.
template <int KVT>
__global__ void k_rope_store_rows(const float* __restrict__ kc, const float* __restrict__ vc,
                                  const float2* __restrict__ rope, void* kcache, void* vcache, long long layer_off,
                                  const int* __restrict__ pos, Dims D)
{
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;  // pair index within kv_dim
    const int p = pos[b];
    if (p < 0 || 2 * j >= D.kv_dim) return;
    const int i = 2 * j, kh = i / D.hd, ii = i - kh * D.hd;
    const float2 cs = rope[(long long)p * (D.q_dim / 2) + j];
    const long long kb = (long long)b * D.kv_dim;
    const long long row = kv_head_base(D, layer_off, b, kh) + (long long)p * D.hd + ii;
    const float k0 = kc[kb + i], k1 = kc[kb + i + 1];
    kv_put(kcache, KVT, row, __fsub_rn(__fmul_rn(k0, cs.x), __fmul_rn(k1, cs.y)));
    kv_put(kcache, KVT, row + 1, __fadd_rn(__fmul_rn(k0, cs.y), __fmul_rn(k1, cs.x)));
    kv_put(vcache, KVT, row, vc[kb + i]);
    kv_put(vcache, KVT, row + 1, vc[kb + i + 1]);
}

// RoPE (src/runtime.c:19-41) fused with the scores (:139-157): each CTA
// rotates the kv_mul query heads of its KV head (the whole query is rotated,
// adjacent pairs, cos/sin from the table), loads 32 cached key rows, and the
// CTA whose tile holds the current position rotates that position's key and
// stores the key and value rows into the cache (:129-132).  Then
// att[b][h][t] = dot_ref(q_h, k_t) * (1/sqrt(head_dim)).  Threads: x = position
// in the tile, y = query head of the group.
template <int KVT, bool FUSED>
__global__ void k_att_scores(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                             const float2* __restrict__ rope, void* kcache, void* vcache, long long layer_off,
                             const int* __restrict__ pos, float* __restrict__ att, Dims D)
{
    extern __shared__ float sm[];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x / D.n_kv, kh = blockIdx.x % D.n_kv;
    const int t0 = blockIdx.y * kScoreTile;
    const int p = pos[b];
    if (p < 0 || t0 > p) return;
    // Rows padded to hd + 4 floats: 16-byte aligned, and the 128-bit reads of
    // 8 consecutive rows (one per lane) hit distinct banks (hd % 32 == 0).
    const int hd = D.hd, ld = hd + 4;
    float* Ks = sm;
    float* Qs = sm + kScoreTile * ld;
    const int nthr = blockDim.x * blockDim.y, tid = threadIdx.y * blockDim.x + threadIdx.x;
    const int nt = min(kScoreTile, p - t0 + 1);
    const float2* rp = rope + (long long)p * (D.q_dim / 2);
    const long long q0 = (long long)b * D.q_dim + (long long)kh * D.kv_mul * hd;
    const bool here = FUSED && p < t0 + kScoreTile;  // this tile holds the current position (stored here)
    const long long hb = kv_head_base(D, layer_off, b, kh);
    // Cached rows t0 .. (here ? p-1 : t0+nt-1): contiguous, 16-byte words.
    const int ncached = nt - (here ? 1 : 0);
    constexpr int EPW = KVT ? 8 : 4;  // elements per 16-byte word
    const int words = ncached * hd / EPW;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(kcache) +
                                                      (hb + (long long)t0 * hd) * (KVT ? 2 : 4));
#pragma unroll 4
    for (int wd = tid; wd < words; wd += nthr) {
        const uint4 v = src[wd];
        const int e = wd * EPW, tt = e / hd, i = e % hd;
        float4* dst = reinterpret_cast<float4*>(Ks + tt * ld + i);
        if (KVT) {
            dst[0] = make_float4(h2f_ref(v.x & 0xFFFFu), h2f_ref(v.x >> 16), h2f_ref(v.y & 0xFFFFu), h2f_ref(v.y >> 16));
            dst[1] = make_float4(h2f_ref(v.z & 0xFFFFu), h2f_ref(v.z >> 16), h2f_ref(v.w & 0xFFFFu), h2f_ref(v.w >> 16));
        } else {
            dst[0] = make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
        }
    }
    for (int e = 2 * tid; e < D.kv_mul * hd; e += 2 * nthr) {
        float o0, o1;
        rot(q[q0 + e], q[q0 + e + 1], rp[(kh * D.kv_mul * hd + e) >> 1], o0, o1);
        Qs[e] = o0;
        Qs[e + 1] = o1;
    }
    if (here) {
        const long long kb = (long long)b * D.kv_dim + (long long)kh * hd;
        const long long row = hb + (long long)p * hd;
        for (int i = 2 * tid; i < hd; i += 2 * nthr) {
            float o0, o1;
            rot(kc[kb + i], kc[kb + i + 1], rp[(kh * hd + i) >> 1], o0, o1);
            Ks[(p - t0) * ld + i] = kv_round(KVT, o0);
            Ks[(p - t0) * ld + i + 1] = kv_round(KVT, o1);
            kv_put(kcache, KVT, row + i, o0);
            kv_put(kcache, KVT, row + i + 1, o1);
            kv_put(vcache, KVT, row + i, vc[kb + i]);
            kv_put(vcache, KVT, row + i + 1, vc[kb + i + 1]);
        }
    }
    __syncthreads();
    const int tt = threadIdx.x, m = threadIdx.y;
    if (tt < nt && m < D.kv_mul) {
        // dot_ref order: element 0, 1, 2, ... (4 per 128-bit load; hd % 8 == 0)
        const float4* kr = reinterpret_cast<const float4*>(Ks + tt * ld);
        const float4* qh = reinterpret_cast<const float4*>(Qs + m * hd);
        float s = 0.0f;
#pragma unroll 4
        for (int i4 = 0; i4 < hd / 4; ++i4) {
            const float4 a = qh[i4], k = kr[i4];
            const float p0 = __fmul_rn(a.x, k.x), p1 = __fmul_rn(a.y, k.y), p2 = __fmul_rn(a.z, k.z),
                        p3 = __fmul_rn(a.w, k.w);
            s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, p0), p1), p2), p3);
        }
        const int h = kh * D.kv_mul + m;
        att[((long long)b * D.n_heads + h) * D.seq_len + t0 + tt] = __fmul_rn(s, D.inv_sqrt);
    }
}

constexpr int kVTile = 32;       // value rows per pipeline stage
constexpr int kVMaxStages = 64;  // most stages of the ring (Dims::vst)
constexpr int kVHThreads = 256;  // threads of the one-head-per-CTA kernel's softmax

// Score rows in shared memory: seq_len rounded up to 32, plus 4 floats, so
// rows are 16-byte aligned and two heads' rows start in different banks.
__host__ __device__ inline int att_sstride(int seq_len) { return ((seq_len + 31) & ~31) + 4; }
// Threads: one per 4 consecutive output elements of the kv_mul heads, and at
// least one warp per head (the softmax runs a head per warp), in whole warps.
__host__ __device__ inline int att_v_threads_of(int kv_mul, int hd)
{
    const int t = (kv_mul * hd / 4 + 31) / 32 * 32;
    return t > 32 * kv_mul ? t : 32 * kv_mul;
}

// Per (sequence, KV head): softmax_ref of each query head's scores
// (src/kernels.c:191-207) and out_h[i] = sum over positions, in order, of
// att_h[t] * v_t[i] from 0 (src/runtime.c:171-194).  The kv_mul heads share
// the value rows, which stream through a ring of shared-memory stages (one
// bulk copy per tile of rows, mbarrier completion; the first stages are in
// flight while the softmax runs), so the rows are read from memory once per
// KV head.  Each thread owns 4 consecutive elements of one head's output:
// four independent running sums that advance position by position, fed by
// 128-bit reads of 4 scores and of each row's 4 elements.
template <int KVT>
__global__ void k_att_softmax_v(const float* __restrict__ att, const void* __restrict__ vcache, long long layer_off,
                                const int* __restrict__ pos, float* __restrict__ xa, int* err, Dims D,
                                const __grid_constant__ Tgts tg)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ __align__(8) uint64_t bars[kVMaxStages];
    __shared__ int s_abort;
    constexpr int ES = KVT ? 2 : 4;
    const int hd = D.hd;
    const int row_bytes = hd * ES;
    const int stage_bytes = kVTile * row_bytes;
    const int ss = att_sstride(D.seq_len);
    const int NS = D.vst;  // stages in flight
    unsigned char* vring = smraw;                                  // [NS][kVTile][hd]
    float* S = reinterpret_cast<float*>(smraw + NS * stage_bytes);  // [kv_mul][ss]
    const int b = blockIdx.x / D.n_kv, kh = blockIdx.x % D.n_kv;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
        s_abort = 0;
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int p = pos[b], np = p + 1;
    if (p < 0) return;
    const int ntiles = (np + kVTile - 1) / kVTile;
    // The head's value rows are contiguous: one bulk copy per tile.
    const unsigned char* vrow0 =
        static_cast<const unsigned char*>(vcache) + kv_head_base(D, layer_off, b, kh) * ES;
    auto issue = [&](int j) {  // one thread: tile j's rows into stage j % NS
        const int st = j % NS, t0 = j * kVTile, nt = min(kVTile, np - t0);
        mbar_arrive_expect_tx(&bars[st], (uint32_t)(nt * row_bytes));
        bulk_g2s(vring + st * stage_bytes, vrow0 + (long long)t0 * row_bytes, (uint32_t)(nt * row_bytes), &bars[st]);
    };
    if (tid == 0)
        for (int j = 0; j < min(NS, ntiles); ++j) issue(j);

    for (int m = warp; m < D.kv_mul; m += nwarps) {
        // Warp m copies head m's scores into shared memory and takes their
        // maximum: x[0], then any strictly greater value (a NaN at 0 sticks).
        float* s = S + m * ss;
        const float* a = att + ((long long)b * D.n_heads + kh * D.kv_mul + m) * D.seq_len;
        const float a0 = a[0];
        float mx = a0;
#pragma unroll 4
        for (int t = lane; t < np; t += 32) {
            const float v = a[t];
            s[t] = v;
            mx = fmaxf(mx, v);
        }
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (a0 != a0) mx = a0;
        __syncwarp();
        for (int t = lane; t < np; t += 32) s[t] = libm::expf_ref(__fsub_rn(s[t], mx));
        __syncwarp();
        float inv = 0.0f;
        if (lane == 0) inv = __fdiv_rn(1.0f, chain_sum(s, np));
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int t = lane; t < np; t += 32) s[t] = __fmul_rn(s[t], inv);
    }
    __syncthreads();

    // Thread (m, q): outputs 4q .. 4q+3 of head m.
    const int nq = hd / 4, nout = D.kv_mul * hd;
    const bool live = tid < D.kv_mul * nq;
    const int m = live ? tid / nq : 0, q = live ? tid % nq : 0;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int issued = min(NS, ntiles);  // meaningful in thread 0
    int j = 0;
    for (; j < ntiles; ++j) {
        const int st = j % NS;
        // Every thread waits on the same stage; a wait that gives up (250 ms)
        // raises the CTA's abort flag, which the barrier makes uniform.
        if (!mbar_wait_bounded(&bars[st], (uint32_t)((j / NS) & 1), err, &s_abort)) s_abort = 1;
        __syncthreads();
        if (s_abort) break;
        const int t0 = j * kVTile, nt = min(kVTile, np - t0);
        const unsigned char* vt = vring + st * stage_bytes + (KVT ? 8 : 16) * q;
        auto vrow = [&](int r) {
            if (KVT) {
                const uint2 h = *reinterpret_cast<const uint2*>(vt + r * row_bytes);
                return make_float4(h2f_ref(h.x & 0xFFFFu), h2f_ref(h.x >> 16), h2f_ref(h.y & 0xFFFFu),
                                   h2f_ref(h.y >> 16));
            }
            return *reinterpret_cast<const float4*>(vt + r * row_bytes);
        };
        const float* sp = S + m * ss + t0;
        if (live) {
            int r = 0;
            for (; r + 4 <= nt; r += 4) {
                const float4 s4 = *reinterpret_cast<const float4*>(sp + r);
                const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 v = vrow(r + k);
                    a0 = __fadd_rn(a0, __fmul_rn(sv[k], v.x));
                    a1 = __fadd_rn(a1, __fmul_rn(sv[k], v.y));
                    a2 = __fadd_rn(a2, __fmul_rn(sv[k], v.z));
                    a3 = __fadd_rn(a3, __fmul_rn(sv[k], v.w));
                }
            }
            for (; r < nt; ++r) {
                const float sc = sp[r];
                const float4 v = vrow(r);
                a0 = __fadd_rn(a0, __fmul_rn(sc, v.x));
                a1 = __fadd_rn(a1, __fmul_rn(sc, v.y));
                a2 = __fadd_rn(a2, __fmul_rn(sc, v.z));
                a3 = __fadd_rn(a3, __fmul_rn(sc, v.w));
            }
        }
        __syncthreads();  // stage st is free again
        if (tid == 0 && j + NS < ntiles) {
            issue(j + NS);
            issued = j + NS + 1;
        }
    }
    if (j < ntiles) {
        // Gave up: drain this CTA's copies still in flight (bounded) before
        // its shared memory is released; the output is not written.
        if (tid == 0)
            for (int jj = j; jj < issued; ++jj)
                mbar_wait_bounded(&bars[jj % NS], (uint32_t)((jj / NS) & 1), err, nullptr);
        return;
    }
    if (live)
        *reinterpret_cast<float4*>(xa + (long long)b * D.q_dim + (long long)(kh * D.kv_mul + m) * hd + 4 * q) =
            make_float4(a0, a1, a2, a3);
    // With head_dim a multiple of 32, warp w holds output elements
    // [128w, 128w + 128) of this KV head: four whole 32-element blocks of the
    // attention output, quantized here for the O projection (element l of a
    // block comes from lane 8*block + l/4, component l % 4).
    if (tg.n) {
        const int g0 = kh * D.kv_mul * hd;  // first output element of this KV head
#pragma unroll
        for (int bq = 0; bq < 4; ++bq) {
            const int src = 8 * bq + (lane >> 2);
            const float c0 = __shfl_sync(0xffffffffu, a0, src), c1 = __shfl_sync(0xffffffffu, a1, src);
            const float c2 = __shfl_sync(0xffffffffu, a2, src), c3 = __shfl_sync(0xffffffffu, a3, src);
            const int c = lane & 3;
            const float v = c == 0 ? c0 : c == 1 ? c1 : c == 2 ? c2 : c3;
            const int e = 128 * warp + 32 * bq;
            if (e < nout) tgts_write(tg, b, (g0 + e) >> 5, lane, v);
        }
    }
}

// The same for steps with few KV heads (one sequence): one CTA per
// (sequence, query head), so 8x more SMs share the work.  All kVHThreads
// threads form the head's softmax exactly as above (copies, maximum and
// exponentials shared; one thread keeps the left-to-right sum); then only the
// warps that own output elements stay: thread i owns output element i and its
// running sum over the positions, in order; each CTA streams its KV head's
// value rows through its own ring (the other query heads of the group read
// the same rows from L2).  With head_dim a multiple of 32, warp w holds
// elements [32w, 32w + 32) of the head: one block of the O projection's input.
template <int KVT>
__global__ void k_att_softmax_v_head(const float* __restrict__ att, const void* __restrict__ vcache,
                                     long long layer_off, const int* __restrict__ pos, float* __restrict__ xa,
                                     int* err, Dims D, const __grid_constant__ Tgts tg)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ __align__(8) uint64_t bars[kVMaxStages];
    __shared__ int s_abort;
    constexpr int ES = KVT ? 2 : 4;
    const int hd = D.hd;
    const int row_bytes = hd * ES;
    const int stage_bytes = kVTile * row_bytes;
    const int NS = D.vsth;
    unsigned char* vring = smraw;                                   // [NS][kVTile][hd]
    float* S = reinterpret_cast<float*>(smraw + NS * stage_bytes);  // this head's scores
    const int b = blockIdx.x / D.n_heads, h = blockIdx.x % D.n_heads, kh = h / D.kv_mul;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int vthreads = (hd + 31) / 32 * 32;  // the value loop's threads (whole warps)
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
        s_abort = 0;
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int p = pos[b], np = p + 1;
    if (p < 0) return;
    const int ntiles = (np + kVTile - 1) / kVTile;
    const unsigned char* vrow0 =
        static_cast<const unsigned char*>(vcache) + kv_head_base(D, layer_off, b, kh) * ES;
    auto issue = [&](int j) {  // one thread: tile j's rows into stage j % NS
        const int st = j % NS, t0 = j * kVTile, nt = min(kVTile, np - t0);
        mbar_arrive_expect_tx(&bars[st], (uint32_t)(nt * row_bytes));
        bulk_g2s(vring + st * stage_bytes, vrow0 + (long long)t0 * row_bytes, (uint32_t)(nt * row_bytes), &bars[st]);
    };
    if (tid == 0)
        for (int j = 0; j < min(NS, ntiles); ++j) issue(j);
    {
        // softmax_ref of this head's scores: max from x[0] (a NaN at 0
        // sticks), expf, left-to-right sum (one thread), scale.  Every thread
        // of the CTA copies and exponentiates its share.
        __shared__ float s_red[32];
        const int nthr = blockDim.x, nw = nthr >> 5;
        const float* a = att + ((long long)b * D.n_heads + h) * D.seq_len;
        const float a0 = a[0];
        float mx = a0;
#pragma unroll 8
        for (int t = tid; t < np; t += nthr) {
            const float v = a[t];
            S[t] = v;
            mx = fmaxf(mx, v);
        }
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) s_red[warp] = mx;
        __syncthreads();
        mx = s_red[0];
        for (int w = 1; w < nw; ++w) mx = fmaxf(mx, s_red[w]);
        if (a0 != a0) mx = a0;
        for (int t = tid; t < np; t += nthr) S[t] = libm::expf_ref(__fsub_rn(S[t], mx));
        __syncthreads();
        if (tid == 0) s_red[0] = __fdiv_rn(1.0f, chain_sum(S, np));
        __syncthreads();
        const float inv = s_red[0];
        for (int t = tid; t < np; t += nthr) S[t] = __fmul_rn(S[t], inv);
    }
    __syncthreads();
    if (tid >= vthreads) return;  // the value loop synchronises its own warps only (barrier 1)
    const bool live = tid < hd;
    float acc = 0.0f;
    int issued = min(NS, ntiles);  // meaningful in thread 0
    int j = 0;
    for (; j < ntiles; ++j) {
        const int st = j % NS;
        if (!mbar_wait_bounded(&bars[st], (uint32_t)((j / NS) & 1), err, &s_abort)) s_abort = 1;
        bar_sync_n(1, vthreads);
        if (s_abort) break;
        const int t0 = j * kVTile, nt = min(kVTile, np - t0);
        const unsigned char* vt = vring + st * stage_bytes + ES * (live ? tid : 0);
        auto vat = [&](int r) {
            return KVT ? h2f_ref(*reinterpret_cast<const uint16_t*>(vt + r * row_bytes))
                       : *reinterpret_cast<const float*>(vt + r * row_bytes);
        };
        const float* sp = S + t0;
        if (live && nt == kVTile) {
            // The tile's 32 scores and values into registers first, then the
            // 32 dependent adds in position order.
            float sv[kVTile], vv[kVTile];
#pragma unroll
            for (int q = 0; q < kVTile / 4; ++q) {
                const float4 s4 = *reinterpret_cast<const float4*>(sp + 4 * q);
                sv[4 * q] = s4.x;
                sv[4 * q + 1] = s4.y;
                sv[4 * q + 2] = s4.z;
                sv[4 * q + 3] = s4.w;
            }
#pragma unroll
            for (int r = 0; r < kVTile; ++r) vv[r] = vat(r);
#pragma unroll
            for (int r = 0; r < kVTile; ++r) acc = __fadd_rn(acc, __fmul_rn(sv[r], vv[r]));
        } else if (live) {
            for (int r = 0; r < nt; ++r) acc = __fadd_rn(acc, __fmul_rn(sp[r], vat(r)));
        }
        bar_sync_n(1, vthreads);  // stage st is free again
        if (tid == 0 && j + NS < ntiles) {
            issue(j + NS);
            issued = j + NS + 1;
        }
    }
    if (j < ntiles) {
        if (tid == 0)
            for (int jj = j; jj < issued; ++jj)
                mbar_wait_bounded(&bars[jj % NS], (uint32_t)((jj / NS) & 1), err, nullptr);
        return;
    }
    if (live) xa[(long long)b * D.q_dim + (long long)h * hd + tid] = acc;
    if (tg.n && 32 * warp < hd) tgts_write(tg, b, (h * hd + 32 * warp) >> 5, lane, acc);
}

// delta += sh * sigmoid(g) per sequence (the shared expert's gated add).
__global__ void k_shexp_add(float* __restrict__ delta, const float* __restrict__ sh, const float* __restrict__ g,
                            int dim)
{
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    const float gv = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm::expf_ref(-g[b])));
    delta[(long long)b * dim + i] = __fadd_rn(delta[(long long)b * dim + i], __fmul_rn(sh[(long long)b * dim + i], gv));
}

// Greedy pick (src/sampling.c:125-131): best = 0, then every later index whose
// logit is strictly greater.  So: the first maximum among non-NaN logits,
// and 0 when logits[0] is NaN.  Records the token in the decode ring.
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ logits, long long ldl, int vocab,
                                                 int* __restrict__ next, const Ctl* __restrict__ ctl,
                                                 int* __restrict__ ring, int B)
{
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x;
    const float* l = logits + (long long)b * ldl;
    float bv = 0.0f;
    int bi = -1;
    // Each thread visits its logits in increasing index order (so among equal
    // values it keeps the first); 16-byte loads, eight in flight per thread.
    auto see = [&](float v, int i) {
        if (v == v && (bi < 0 || v > bv)) {
            bv = v;
            bi = i;
        }
    };
    int i0 = 0;
    if ((reinterpret_cast<uintptr_t>(l) & 15) == 0) {
        const int n4 = vocab >> 2;
        const float4* l4 = reinterpret_cast<const float4*>(l);
        for (int k0 = threadIdx.x; k0 < n4; k0 += 8 * blockDim.x) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int k = k0 + u * blockDim.x;
                v[u] = k < n4 ? l4[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int k = k0 + u * blockDim.x;
                if (k < n4) {
                    see(v[u].x, 4 * k);
                    see(v[u].y, 4 * k + 1);
                    see(v[u].z, 4 * k + 2);
                    see(v[u].w, 4 * k + 3);
                }
            }
        }
        i0 = 4 * n4;
    }
    for (int i = i0 + threadIdx.x; i < vocab; i += blockDim.x) see(l[i], i);
    auto better = [](float v2, int i2, float v1, int i1) {
        if (i2 < 0) return false;
        if (i1 < 0) return true;
        if (v2 > v1) return true;
        if (v1 > v2) return false;
        return i2 < i1;
    };
    for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(v2, i2, bv, bi)) {
            bv = v2;
            bi = i2;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : 0.0f;
        bi = lane < nw ? si[lane] : -1;
        for (int o = 16; o; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(v2, i2, bv, bi)) {
                bv = v2;
                bi = i2;
            }
        }
        if (lane == 0) {
            const float l0 = l[0];
            const int pick = (l0 != l0 || bi < 0) ? 0 : bi;
            next[b] = pick;
            if (ctl->mode == MODE_DECODE && ctl->dstep >= 1)
                ring[(long long)((ctl->dstep - 1) % ctl->ring) * B + b] = pick;
        }
    }
}

// Test hook: out[i] = expf_ref of the float with bit pattern first + i.
__global__ void k_debug_expf(float* __restrict__ out, uint32_t first, long long n)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = libm::expf_ref(__uint_as_float(first + (uint32_t)i));
}

__global__ void k_ctl_set(Ctl* ctl, int mode, int n_prompt, int ring)
{
    ctl->mode = mode;
    ctl->n_prompt = n_prompt;
    ctl->step = 0;
    ctl->dstep = 0;
    ctl->ring = ring;
}

} // namespace dec
} // namespace qr

using namespace qr;
using namespace qr::dec;

struct quantr_decoder {
    int device = 0;
    Dims D{};
    int n_layers = 0, E = 0, K = 0, shexp = 0;
    float rope_base = 10000.0f;
    // resolved device pointers
    const uint8_t* embd = nullptr;
    uint32_t embd_type = 0;
    long long embd_rb = 0;
    std::vector<const float*> rms_att, rms_ffn, router, sh_gate;
    const float* rms_final = nullptr;
    std::vector<ExpertMats> ew1, ew2, ew3;  // per layer
    // owned device memory
    std::vector<void*> owned;
    uint8_t* arena = nullptr;
    float *x = nullptr, *xb = nullptr, *xa = nullptr, *q = nullptr, *kc = nullptr, *vc = nullptr, *att = nullptr;
    float *hb = nullptr, *hb2 = nullptr, *delta = nullptr, *logits = nullptr, *sh = nullptr, *gdot = nullptr;
    float *moe_o = nullptr, *wts = nullptr;
    int* sel = nullptr;
    void *kcache = nullptr, *vcache = nullptr;
    float2* rope = nullptr;
    int *tok = nullptr, *pos = nullptr, *next = nullptr, *prompt = nullptr, *ring = nullptr;
    int prompt_cap = 0, ring_cap = 0;
    Ctl* ctl = nullptr;
    void* moe_ws = nullptr;
    size_t moe_ws_bytes = 0;
    // plans
    std::vector<quantr_program*> p_qkv, p_o, p_ffn13, p_w2, p_sh13, p_sh2;
    quantr_program* p_head = nullptr;
    // Activation layouts the norm / attention kernels quantize into directly
    // (one-token decoders; n = 0 where the program quantizes its own input).
    std::vector<Tgts> t_qkv, t_o, t_ffn;
    Tgts t_head{};
    // One-token dense models: every layer in one persistent kernel per step
    // (decode_persist.cu); the head and the greedy pick follow as kernels.
    bool child = false;          // a chunked-prefill decoder sharing its parent's KV cache
    quantr_decoder* pf = nullptr;  // this decoder's chunked-prefill child (one-sequence decoders)
    bool persist = false;
    uint32_t persist_type = 0;
    int persist_grid = 0;
    size_t persist_smem = 0;
    dp::Params pp{};
    cudaStream_t stream = nullptr;
    cudaGraphExec_t g_decode = nullptr, g_prefill = nullptr;
    int nodes_decode = 0, nodes_prefill = 0;
    float* host_logits = nullptr;  // pinned, forward_runtime's return
    size_t weight_bytes = 0, kv_pos_bytes = 0, device_bytes = 0;
    double load_ms = 0.0;
};

namespace {

int code_of(cudaError_t e)
{
    if (e == cudaSuccess) return QUANTR_OK;
    cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? QUANTR_ERR_OOM : QUANTR_ERR_CUDA;
}

template <typename T>
cudaError_t dev_alloc(quantr_decoder* d, T** p, size_t count)
{
    void* v = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess) return e;
    d->owned.push_back(v);
    d->device_bytes += bytes;
    *p = static_cast<T*>(v);
    return cudaMemset(v, 0, bytes);
}

// Device address of a model tensor: a registered host range's copy, a device
// pointer as is, or (other host memory) a copy in the decoder's arena.
struct Resolver {
    struct Up {
        const void* host;
        size_t bytes;
        size_t off;
    };
    std::vector<Up> ups;
    size_t arena_bytes = 0;
    const uint8_t* arena = nullptr;
    bool planning = true;

    const uint8_t* get(const void* p, size_t bytes)
    {
        if (!p) return nullptr;
        if (void* r = quantr_gpu_device_ptr(p)) return static_cast<const uint8_t*>(r);
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, p) == cudaSuccess &&
            (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged))
            return static_cast<const uint8_t*>(p);
        cudaGetLastError();
        for (const Up& u : ups)
            if (u.host == p) return planning ? nullptr : arena + u.off;
        if (!planning) return nullptr;
        ups.push_back(Up{p, bytes, arena_bytes});
        arena_bytes += (bytes + 255) / 256 * 256 + 256;  // +16 readable bytes past each tensor, 256-aligned
        return nullptr;
    }
};

size_t tensor_bytes(uint32_t type, long long rows, int cols)
{
    return (size_t)(rows * row_bytes(type, cols));
}

struct ProgJob {
    const void* w;
    uint32_t type;
    int n, d;
    const float* x;
    long long ldx;
    float* out;
    long long ldo;
    const float* xmul = nullptr;  // input silu(x) * xmul (the down projection's SwiGLU)
};

// Threads of the softmax/value kernel: each owns one or two running sums.
int att_v_threads(const Dims& D) { return att_v_threads_of(D.kv_mul, D.hd); }
size_t att_v_smem(const Dims& D)
{
    return (size_t)D.vst * kVTile * D.hd * (D.kv_type ? 2 : 4) + (size_t)D.kv_mul * att_sstride(D.seq_len) * 4;
}
// Stages of the value ring: with at least one CTA per SM (batched steps) as
// many as leave room for two CTAs per SM; with fewer CTAs (one sequence) as
// many as fit, up to every tile of the context, so the copies of a whole head
// are in flight at once.
// The one-head-per-CTA variant: its own score row and as many stages as fit.
size_t att_vh_smem(const Dims& D)
{
    return (size_t)D.vsth * kVTile * D.hd * (D.kv_type ? 2 : 4) + (size_t)att_sstride(D.seq_len) * 4;
}
int att_vh_stages(const Dims& D)
{
    const size_t stage = (size_t)kVTile * D.hd * (D.kv_type ? 2 : 4);
    const size_t budget = kSmemMax - 1024 - (size_t)att_sstride(D.seq_len) * 4;
    const int tiles = (D.seq_len + kVTile - 1) / kVTile;
    return (int)std::max<long long>(2, std::min<long long>({(long long)(budget / stage), (long long)tiles,
                                                            (long long)kVMaxStages}));
}
// Steps with few KV heads in flight (one sequence) take the one-head-per-CTA
// variant.
bool att_per_head(const Dims& D, int sms) { return D.B * D.n_kv * 4 <= sms; }

int att_v_stages(const Dims& D, int sms)
{
    const size_t stage = (size_t)kVTile * D.hd * (D.kv_type ? 2 : 4);
    const size_t scores = (size_t)D.kv_mul * att_sstride(D.seq_len) * 4;
    const size_t budget = (D.B * D.n_kv >= sms ? kSmemMax / 2 : kSmemMax) - 1024;
    const long long fit = budget > scores ? (long long)((budget - scores) / stage) : 0;
    const int tiles = (D.seq_len + kVTile - 1) / kVTile;
    return (int)std::max<long long>(2, std::min<long long>({fit, (long long)tiles, (long long)kVMaxStages}));
}

int make_program(quantr_decoder* d, const std::vector<ProgJob>& js, quantr_program** out)
{
    std::vector<quantr_gemv_job> jobs;
    std::vector<const float*> xm;
    for (const ProgJob& j : js) {
        jobs.push_back(quantr_gemv_job{j.w, j.type, j.n, j.d, d->D.B, j.x, j.ldx, j.out, j.ldo});
        xm.push_back(j.xmul);
    }
    return program_create_ex(out, jobs.data(), xm.data(), (int)jobs.size());
}

// Enqueues one step on `s`.  with_head: final norm, head GEMV and greedy pick.
int enqueue_step(quantr_decoder* d, cudaStream_t s, bool with_head)
{
    const Dims& D = d->D;
    LaunchCfg c;
    c.stream = s;
    cudaError_t e = launch_ex(&k_feed, dim3(1), dim3(std::max(32, (D.B + 31) / 32 * 32)), 0, c, d->ctl, d->tok,
                              d->pos, (const int*)d->prompt, (const int*)d->next, D.B, D.seq_len);
    if (e == cudaSuccess && !d->persist)
        e = launch_ex(&k_embed, dim3((D.dim + 255) / 256, D.B), dim3(256), 0, c, d->x, (const int*)d->tok, d->embd,
                      d->embd_type, d->embd_rb, D.dim, D.vocab);
    const size_t norm_smem = (size_t)2 * D.dim * sizeof(float);
    const long long layer_kv = (long long)D.kv_B * D.seq_len * D.kv_dim;
    const bool chunk = D.seq_stride == 0;  // rows are positions of one sequence (chunked prefill)
    if (e == cudaSuccess && d->persist) e = launch_persist(d->pp, d->persist_type, d->persist_grid, d->persist_smem, s);
    for (int l = 0; l < d->n_layers && e == cudaSuccess && !d->persist; ++l) {
        const long long loff = (long long)l * layer_kv;
        e = launch_ex(&k_rmsnorm, dim3(D.B), dim3(kNormThreads), norm_smem, c, d->x, (const float*)(l ? d->delta : nullptr),
                      d->rms_att[l], d->xb, D.dim, d->t_qkv[l]);
        if (e != cudaSuccess) break;
        if (quantr_program_run(d->p_qkv[l], s) != QUANTR_OK) return QUANTR_ERR_CUDA;
        const size_t ssm = (size_t)(kScoreTile * (D.hd + 4) + D.kv_mul * D.hd) * sizeof(float);
        if (chunk) {
            e = launch_ex(D.kv_type ? &k_rope_store_rows<1> : &k_rope_store_rows<0>,
                          dim3((D.kv_dim / 2 + 127) / 128, D.B), dim3(128), 0, c, (const float*)d->kc,
                          (const float*)d->vc, (const float2*)d->rope, d->kcache, d->vcache, loff, (const int*)d->pos, D);
            if (e != cudaSuccess) break;
        }
        e = launch_ex(D.kv_type ? (chunk ? &k_att_scores<1, false> : &k_att_scores<1, true>)
                                : (chunk ? &k_att_scores<0, false> : &k_att_scores<0, true>),
                      dim3(D.B * D.n_kv, (D.seq_len + kScoreTile - 1) / kScoreTile),
                      dim3(kScoreTile, D.kv_mul), ssm, c, (const float*)d->q, (const float*)d->kc,
                      (const float*)d->vc, (const float2*)d->rope, d->kcache, d->vcache, loff, (const int*)d->pos,
                      d->att, D);
        if (e != cudaSuccess) break;
        if (att_per_head(D, device_sm_count()))
            e = launch_ex(D.kv_type ? &k_att_softmax_v_head<1> : &k_att_softmax_v_head<0>, dim3(D.B * D.n_heads),
                          dim3(std::max(kVHThreads, (D.hd + 31) / 32 * 32)), att_vh_smem(D), c, (const float*)d->att,
                          (const void*)d->vcache, loff, (const int*)d->pos, d->xa, device_error_word(), D, d->t_o[l]);
        else
            e = launch_ex(D.kv_type ? &k_att_softmax_v<1> : &k_att_softmax_v<0>, dim3(D.B * D.n_kv),
                          dim3(att_v_threads(D)), att_v_smem(D), c, (const float*)d->att, (const void*)d->vcache,
                          loff, (const int*)d->pos, d->xa, device_error_word(), D, d->t_o[l]);
        if (e != cudaSuccess) break;
        if (quantr_program_run(d->p_o[l], s) != QUANTR_OK) return QUANTR_ERR_CUDA;
        e = launch_ex(&k_rmsnorm, dim3(D.B), dim3(kNormThreads), norm_smem, c, d->x, (const float*)d->delta, d->rms_ffn[l],
                      d->xb, D.dim, d->t_ffn[l]);
        if (e != cudaSuccess) break;
        if (d->E == 0) {
            if (quantr_program_run(d->p_ffn13[l], s) != QUANTR_OK) return QUANTR_ERR_CUDA;
            // W2's activation quantizer forms silu(h1) * h3 itself.
            if (quantr_program_run(d->p_w2[l], s) != QUANTR_OK) return QUANTR_ERR_CUDA;
        } else {
            int* err = device_error_word();
            MoeRoute r;
            r.sel = d->sel;
            r.wts = d->wts;
            r.xb = d->xb;
            r.ldx = D.dim;
            r.T = D.B;
            r.router = d->router[l];
            r.E = d->E;
            r.k = d->K;
            r.dim = D.dim;
            r.ws = d->moe_ws;
            r.ws_bytes = d->moe_ws_bytes;
            r.err = err;
            e = launch_moe_route(r, c);
            if (e != cudaSuccess) break;
            MoeExperts a;
            a.o = d->moe_o;
            a.xb = d->xb;
            a.ldx = D.dim;
            a.T = D.B;
            a.sel = d->sel;
            a.k = d->K;
            a.e0 = 0;
            a.El = d->E;
            a.dim = D.dim;
            a.hidden = D.hidden;
            a.w1 = d->ew1[l];
            a.w3 = d->ew3[l];
            a.w2 = d->ew2[l];
            a.ws = d->moe_ws;
            a.ws_bytes = d->moe_ws_bytes;
            a.err = err;
            e = launch_moe_experts(a, c);
            if (e != cudaSuccess) break;
            e = launch_moe_combine(d->delta, D.dim, d->moe_o, d->sel, d->wts, D.B, d->K, D.dim, c);
            if (e != cudaSuccess) break;
            if (d->shexp) {
                if (quantr_program_run(d->p_sh13[l], s) != QUANTR_OK) return QUANTR_ERR_CUDA;
                if (quantr_program_run(d->p_sh2[l], s) != QUANTR_OK) return QUANTR_ERR_CUDA;
                e = launch_gemv_f32(d->sh_gate[l], d->xb, D.dim, d->gdot, 1, 1, D.dim, D.B, c);
                if (e != cudaSuccess) break;
                e = launch_ex(&k_shexp_add, dim3((D.dim + 255) / 256, D.B), dim3(256), 0, c, d->delta,
                              (const float*)d->sh, (const float*)d->gdot, D.dim);
                if (e != cudaSuccess) break;
            }
        }
    }
    if (e == cudaSuccess && with_head) {
        e = launch_ex(&k_rmsnorm, dim3(D.B), dim3(kNormThreads), norm_smem, c, d->x, (const float*)d->delta, d->rms_final,
                      d->xb, D.dim, d->t_head);
        if (e == cudaSuccess && quantr_program_run(d->p_head, s) != QUANTR_OK) return QUANTR_ERR_CUDA;
        if (e == cudaSuccess)
            e = launch_ex(&k_argmax, dim3(D.B), dim3(1024), 0, c, (const float*)d->logits, (long long)D.vocab,
                          D.vocab, d->next, (const Ctl*)d->ctl, d->ring, D.B);
    }
    // A prefill step stops after the last layer: the reference's x there only
    // feeds the head, and the next position's embedding overwrites it.
    return code_of(e);
}

int capture(quantr_decoder* d, bool with_head, cudaGraphExec_t* out, int* nodes)
{
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return code_of(e);
    const int rc = enqueue_step(d, d->stream, with_head);
    e = cudaStreamEndCapture(d->stream, &g);
    if (rc != QUANTR_OK || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return rc != QUANTR_OK ? rc : code_of(e);
    }
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    *nodes = (int)n;
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return code_of(e);
}

void destroy(quantr_decoder* d)
{
    if (!d) return;
    if (d->pf) {
        destroy(d->pf);
        d->pf = nullptr;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d->device);
    if (d->stream) cudaStreamSynchronize(d->stream);
    if (d->g_decode) cudaGraphExecDestroy(d->g_decode);
    if (d->g_prefill) cudaGraphExecDestroy(d->g_prefill);
    for (auto* v : {&d->p_qkv, &d->p_o, &d->p_ffn13, &d->p_w2, &d->p_sh13, &d->p_sh2})
        for (quantr_program* p : *v) quantr_program_destroy(p);
    quantr_program_destroy(d->p_head);
    for (void* p : d->owned) cudaFree(p);
    if (d->host_logits) cudaFreeHost(d->host_logits);
    if (d->stream) cudaStreamDestroy(d->stream);
    if (prev >= 0) cudaSetDevice(prev);
    delete d;
}

// RoPE table: (cos, sin) of theta = pos * powf(base, -(i/head_dim)) for every
// position and even index i < q_dim, with the C library's functions
// (src/runtime.c:24-29).
void rope_table(std::vector<float2>& t, int seq_len, int q_dim, int head_dim, float base_in)
{
    const float base = base_in > 0.0f ? base_in : 10000.0f;
    const int half = q_dim / 2;
    std::vector<float> freq(half);
    for (int j = 0; j < half; ++j) freq[j] = ::powf(base, -((float)(2 * j) / (float)head_dim));
    t.resize((size_t)seq_len * half);
    for (int p = 0; p < seq_len; ++p)
        for (int j = 0; j < half; ++j) {
            volatile float theta = (float)p * freq[j];
            const float th = theta;
            t[(size_t)p * half + j] = make_float2(::cosf(th), ::sinf(th));
        }
}

} // namespace

extern "C" {

} // extern "C"

namespace {
constexpr int kPrefillChunk = 64;  // prompt positions per chunked-prefill step

// parent != null: a chunked-prefill decoder for parent's single sequence: its
// `batch` rows are consecutive prompt positions, it shares the parent's KV
// cache, and it only has a prefill graph.
int create_impl(quantr_decoder** out, const quantr_model* m, int batch, quantr_decoder* parent)
{
    if (!out || !m) return QUANTR_ERR_BAD_ARG;
    *out = nullptr;
    if (batch < 1 || batch > kMaxBatch || m->dim <= 0 || m->n_layers <= 0 || m->n_heads <= 0 ||
        m->n_kv_heads <= 0 || m->vocab_size <= 0 || m->seq_len <= 0 || m->hidden_dim < 0)
        return QUANTR_ERR_BAD_ARG;
    const int hd = m->head_dim > 0 ? m->head_dim : m->dim / m->n_heads;
    if (hd <= 0 || (hd & 1) || m->n_heads % m->n_kv_heads) return QUANTR_ERR_BAD_ARG;
    if (m->expert_count < 0 || m->expert_count > kMoeMaxExperts || m->expert_used_count > kMoeMaxK ||
        (m->expert_count > 0 && (m->expert_used_count < 1 || m->expert_used_count > m->expert_count)))
        return QUANTR_ERR_BAD_ARG;
    const auto t0 = std::chrono::steady_clock::now();
    quantr_decoder* d = new (std::nothrow) quantr_decoder();
    if (!d) return QUANTR_ERR_OOM;
    cudaGetDevice(&d->device);
    Dims& D = d->D;
    D.B = batch;
    D.dim = m->dim;
    D.hd = hd;
    D.n_heads = m->n_heads;
    D.n_kv = m->n_kv_heads;
    D.kv_mul = m->n_heads / m->n_kv_heads;
    D.q_dim = m->n_heads * hd;
    D.kv_dim = m->n_kv_heads * hd;
    D.seq_len = m->seq_len;
    D.hidden = m->hidden_dim;
    D.vocab = m->vocab_size;
    D.kv_type = m->kv_type == 1 ? 1 : 0;
    D.inv_sqrt = 1.0f / std::sqrt((float)hd);
    D.kv_B = parent ? parent->D.kv_B : batch;
    D.seq_stride = parent ? 0 : 1;
    D.vst = att_v_stages(D, device_sm_count());
    D.vsth = att_vh_stages(D);
    d->child = parent != nullptr;
    d->n_layers = m->n_layers;
    d->E = m->expert_count;
    d->K = m->expert_used_count;
    d->shexp = m->expert_count > 0 && m->shexp_w1 ? m->shexp_hidden_dim : 0;
    if (D.kv_mul > 32 || att_v_smem(D) > kSmemMax || D.kv_mul * hd > 2048 || (hd * (D.kv_type ? 2 : 4)) % 16 || hd % 8 ||
        (size_t)(kScoreTile * (hd + 4) + D.kv_mul * hd) * 4 > kSmemMax || (size_t)2 * D.dim * 4 > 48 * 1024 || D.dim % 4) {
        delete d;
        return QUANTR_ERR_TOO_LARGE;
    }
    auto fail = [&](int rc) {
        destroy(d);
        return rc;
    };
    if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(QUANTR_ERR_CUDA);

    // ---- weights: resolve (registered / device / upload), two passes ----
    const int L = m->n_layers;
    const int hid = m->hidden_dim;
    Resolver R;
    auto lin = [&](const void* const* arr, const uint32_t* ty, int l, int rows, int cols) -> const uint8_t* {
        if (!arr || !ty || !arr[l]) return nullptr;
        return R.get(arr[l], tensor_bytes(ty[l], rows, cols));
    };
    std::vector<const uint8_t*> wq(L), wk(L), wv(L), wo(L), w1(L), w2(L), w3(L), s1(L), s2(L), s3(L);
    std::vector<std::vector<const uint8_t*>> e1(L), e2(L), e3(L);
    const uint8_t* wcls = nullptr;
    for (int pass = 0; pass < 2; ++pass) {
        if (pass == 1) {
            if (R.arena_bytes) {
                uint8_t* a = nullptr;
                if (dev_alloc(d, &a, R.arena_bytes) != cudaSuccess) return fail(QUANTR_ERR_OOM);
                R.arena = a;
                for (const auto& u : R.ups)
                    if (cudaMemcpy(a + u.off, u.host, u.bytes, cudaMemcpyHostToDevice) != cudaSuccess)
                        return fail(QUANTR_ERR_CUDA);
            }
            R.planning = false;
        }
        const size_t erb = m->token_embd_row_bytes;
        d->embd = R.get(m->token_embd, erb ? erb * m->vocab_size : (size_t)m->vocab_size * m->dim * 4);
        d->embd_type = m->token_embd_type;
        d->embd_rb = (long long)erb;
        d->rms_att.assign(L, nullptr);
        d->rms_ffn.assign(L, nullptr);
        d->router.assign(L, nullptr);
        d->sh_gate.assign(L, nullptr);
        for (int l = 0; l < L; ++l) {
            d->rms_att[l] = (const float*)R.get(m->rms_att ? m->rms_att[l] : nullptr, (size_t)m->dim * 4);
            d->rms_ffn[l] = (const float*)R.get(m->rms_ffn ? m->rms_ffn[l] : nullptr, (size_t)m->dim * 4);
            wq[l] = lin(m->wq, m->wq_type, l, D.q_dim, m->dim);
            wk[l] = lin(m->wk, m->wk_type, l, D.kv_dim, m->dim);
            wv[l] = lin(m->wv, m->wv_type, l, D.kv_dim, m->dim);
            wo[l] = lin(m->wo, m->wo_type, l, m->dim, D.q_dim);
            if (d->E == 0) {
                w1[l] = lin(m->w1, m->w1_type, l, hid, m->dim);
                w3[l] = lin(m->w3, m->w3_type, l, hid, m->dim);
                w2[l] = lin(m->w2, m->w2_type, l, m->dim, hid);
            } else {
                d->router[l] = (const float*)R.get(m->ffn_gate_inp ? m->ffn_gate_inp[l] : nullptr,
                                                   (size_t)d->E * m->dim * 4);
                e1[l].assign(d->E, nullptr);
                e2[l].assign(d->E, nullptr);
                e3[l].assign(d->E, nullptr);
                for (int x = 0; x < d->E; ++x) {
                    e1[l][x] = R.get(m->expert_w1[l][x], tensor_bytes(m->exp_w1_type[l], hid, m->dim));
                    e3[l][x] = R.get(m->expert_w3[l][x], tensor_bytes(m->exp_w3_type[l], hid, m->dim));
                    e2[l][x] = R.get(m->expert_w2[l][x], tensor_bytes(m->exp_w2_type[l], m->dim, hid));
                }
                if (d->shexp) {
                    s1[l] = lin(m->shexp_w1, m->shexp_w1_type, l, d->shexp, m->dim);
                    s3[l] = lin(m->shexp_w3, m->shexp_w3_type, l, d->shexp, m->dim);
                    s2[l] = lin(m->shexp_w2, m->shexp_w2_type, l, m->dim, d->shexp);
                    d->sh_gate[l] = (const float*)R.get(m->shexp_gate ? m->shexp_gate[l] : nullptr, (size_t)m->dim * 4);
                }
            }
        }
        d->rms_final = (const float*)R.get(m->rms_final, (size_t)m->dim * 4);
        wcls = R.get(m->wcls, tensor_bytes(m->wcls_type, m->vocab_size, m->dim));
    }
    // Everything the step reads must exist (the reference would crash on a
    // NULL norm; a NULL linear there gives zeros, which this decoder rejects).
    bool ok = d->embd && d->rms_final && wcls;
    for (int l = 0; l < L && ok; ++l) {
        ok = d->rms_att[l] && d->rms_ffn[l] && wq[l] && wk[l] && wv[l] && wo[l];
        if (d->E == 0) ok = ok && w1[l] && w2[l] && w3[l];
        else {
            ok = ok && d->router[l];
            for (int x = 0; x < d->E && ok; ++x) ok = e1[l][x] && e2[l][x] && e3[l][x];
            if (d->shexp) ok = ok && s1[l] && s2[l] && s3[l] && d->sh_gate[l];
        }
    }
    // The norm kernels read the norm weights as 16-byte words.
    for (int l = 0; l < L && ok; ++l)
        ok = !((uintptr_t)d->rms_att[l] & 15) && !((uintptr_t)d->rms_ffn[l] & 15);
    ok = ok && !((uintptr_t)d->rms_final & 15);
    if (!ok) return fail(QUANTR_ERR_BAD_ARG);

    // ---- activations, caches, tables ----
    const int B = batch;
    const int wide = std::max(D.q_dim, m->dim);
    const int hmax = std::max(hid, d->shexp);
    cudaError_t e = cudaSuccess;
    auto A = [&](auto** p, size_t n) {
        if (e == cudaSuccess) e = dev_alloc(d, p, n);
    };
    A(&d->x, (size_t)B * m->dim);
    A(&d->xb, (size_t)B * wide);
    A(&d->xa, (size_t)B * D.q_dim);
    A(&d->q, (size_t)B * D.q_dim);
    A(&d->kc, (size_t)B * D.kv_dim);
    A(&d->vc, (size_t)B * D.kv_dim);
    A(&d->att, (size_t)B * D.n_heads * D.seq_len);
    A(&d->hb, (size_t)B * std::max(hmax, 1));
    A(&d->hb2, (size_t)B * std::max(hmax, 1));
    A(&d->delta, (size_t)B * m->dim);
    A(&d->logits, (size_t)B * D.vocab);
    A(&d->tok, (size_t)B);
    A(&d->pos, (size_t)B);
    A(&d->next, (size_t)B);
    d->prompt_cap = D.seq_len;
    A(&d->prompt, (size_t)B * d->prompt_cap);
    d->ring_cap = std::max(D.seq_len, 4096);
    A(&d->ring, (size_t)B * d->ring_cap);
    A(&d->ctl, 1);
    const size_t kv_elems = (size_t)L * D.kv_B * D.seq_len * D.kv_dim;
    if (parent) {
        d->kcache = parent->kcache;
        d->vcache = parent->vcache;
    } else {
        uint8_t *kcb = nullptr, *vcb = nullptr;
        A(&kcb, kv_elems * (D.kv_type ? 2 : 4));
        A(&vcb, kv_elems * (D.kv_type ? 2 : 4));
        d->kcache = kcb;
        d->vcache = vcb;
    }
    if (d->E) {
        A(&d->moe_o, (size_t)B * d->K * m->dim);
        A(&d->sel, (size_t)B * d->K);
        A(&d->wts, (size_t)B * d->K);
        d->moe_ws_bytes = moe_workspace_bytes(B, d->E, d->K, m->dim, hid);
        uint8_t* ws = nullptr;
        A(&ws, d->moe_ws_bytes);
        d->moe_ws = ws;
        if (d->shexp) {
            A(&d->sh, (size_t)B * m->dim);
            A(&d->gdot, (size_t)B);
        }
    }
    std::vector<float2> rt;
    rope_table(rt, D.seq_len, D.q_dim, hd, m->rope_freq_base);
    A(&d->rope, rt.size());
    if (e == cudaSuccess) e = cudaMemcpy(d->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMallocHost((void**)&d->host_logits, (size_t)D.vocab * 4);
    if (e != cudaSuccess) return fail(code_of(e));
    // Expert pointer tables (device arrays of device pointers).
    if (d->E) {
        d->ew1.resize(L);
        d->ew2.resize(L);
        d->ew3.resize(L);
        for (int l = 0; l < L; ++l) {
            const uint8_t** tb = nullptr;
            A(&tb, (size_t)3 * d->E);
            if (e != cudaSuccess) return fail(code_of(e));
            std::vector<const uint8_t*> h(3 * (size_t)d->E);
            for (int x = 0; x < d->E; ++x) {
                h[x] = e1[l][x];
                h[d->E + x] = e3[l][x];
                h[2 * d->E + x] = e2[l][x];
            }
            e = cudaMemcpy(tb, h.data(), h.size() * sizeof(void*), cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return fail(code_of(e));
            d->ew1[l] = ExpertMats{nullptr, 0, tb, m->exp_w1_type[l]};
            d->ew3[l] = ExpertMats{nullptr, 0, tb + d->E, m->exp_w3_type[l]};
            d->ew2[l] = ExpertMats{nullptr, 0, tb + 2 * d->E, m->exp_w2_type[l]};
        }
    }

    // ---- GEMV programs ----
    for (int l = 0; l < L; ++l) {
        quantr_program* p = nullptr;
        int rc = make_program(d, {{wq[l], m->wq_type[l], D.q_dim, m->dim, d->xb, m->dim, d->q, D.q_dim},
                                  {wk[l], m->wk_type[l], D.kv_dim, m->dim, d->xb, m->dim, d->kc, D.kv_dim},
                                  {wv[l], m->wv_type[l], D.kv_dim, m->dim, d->xb, m->dim, d->vc, D.kv_dim}},
                              &p);
        if (rc) return fail(rc);
        d->p_qkv.push_back(p);
        rc = make_program(d, {{wo[l], m->wo_type[l], m->dim, D.q_dim, d->xa, D.q_dim, d->delta, m->dim}}, &p);
        if (rc) return fail(rc);
        d->p_o.push_back(p);
        if (d->E == 0) {
            rc = make_program(d, {{w1[l], m->w1_type[l], hid, m->dim, d->xb, m->dim, d->hb, hid},
                                  {w3[l], m->w3_type[l], hid, m->dim, d->xb, m->dim, d->hb2, hid}},
                              &p);
            if (rc) return fail(rc);
            d->p_ffn13.push_back(p);
            rc = make_program(d, {{w2[l], m->w2_type[l], m->dim, hid, d->hb, hid, d->delta, m->dim, d->hb2}}, &p);
            if (rc) return fail(rc);
            d->p_w2.push_back(p);
        } else if (d->shexp) {
            const int sh = d->shexp;
            rc = make_program(d, {{s1[l], m->shexp_w1_type[l], sh, m->dim, d->xb, m->dim, d->hb, sh},
                                  {s3[l], m->shexp_w3_type[l], sh, m->dim, d->xb, m->dim, d->hb2, sh}},
                              &p);
            if (rc) return fail(rc);
            d->p_sh13.push_back(p);
            rc = make_program(d, {{s2[l], m->shexp_w2_type[l], m->dim, sh, d->hb, sh, d->sh, m->dim, d->hb2}}, &p);
            if (rc) return fail(rc);
            d->p_sh2.push_back(p);
        }
    }
    if (!parent) {
        int rc = make_program(d, {{wcls, m->wcls_type, D.vocab, m->dim, d->xb, m->dim, d->logits, D.vocab}},
                              &d->p_head);
        if (rc) return fail(rc);
    }
    // One-token decoders: the kernels producing the inputs of the Q/K/V, O,
    // W1/W3 and head programs quantize them straight into the engine's
    // layout, and those programs skip their own quantizer launch.
    auto external = [&](quantr_program* p, const float* x) {
        Tgts t{};
        if (B != 1 || !p) return t;
        const int n = program_act_targets(p, x, t.t, 3);
        if (n > 0 && program_external_quant(p, true) == QUANTR_OK) t.n = n;
        return t;
    };
    d->t_qkv.assign(L, Tgts{});
    d->t_o.assign(L, Tgts{});
    d->t_ffn.assign(L, Tgts{});
    for (int l = 0; l < L; ++l) {
        d->t_qkv[l] = external(d->p_qkv[l], d->xb);
        if (hd % 32 == 0) d->t_o[l] = external(d->p_o[l], d->xa);
        if (d->E == 0) d->t_ffn[l] = external(d->p_ffn13[l], d->xb);
    }
    if (!parent) d->t_head = external(d->p_head, d->xb);

    // Persistent one-token path (decode_persist.cu): dense layers whose
    // linears share one type with 16-byte multiple row sizes.  Bit-identical
    // to the launch-per-stage step but measured slower on B200 (its per-CTA
    // stages are latency-bound), so it runs only when QUANTR_DECODE_PERSIST=1
    // is set when the decoder is created.
    const char* pe = std::getenv("QUANTR_DECODE_PERSIST");
    if (B == 1 && d->E == 0 && pe && pe[0] == '1') {
        const uint32_t T = m->wq_type[0];
        bool elig = type_supported(T) && m->dim % 256 == 0 && D.q_dim % 256 == 0 && hid % 256 == 0 &&
                    D.kv_dim % 32 == 0 && hd <= dp::kPersistThreads && D.n_heads <= device_sm_count() &&
                    std::max({m->dim, D.q_dim, hid}) <= dp::kPersistMaxVec;
        for (int l = 0; l < L && elig; ++l)
            elig = m->wq_type[l] == T && m->wk_type[l] == T && m->wv_type[l] == T && m->wo_type[l] == T &&
                   m->w1_type[l] == T && m->w2_type[l] == T && m->w3_type[l] == T;
        for (int dd : {m->dim, D.q_dim, hid})
            if (elig) elig = row_bytes(T, dd) % 16 == 0;
        if (elig) elig = d->embd_rb == 0 || dequant_extent_host(d->embd_type, m->dim) == m->dim;
        int dev = 0, coop = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
        if (elig && coop) {
            const int grid = device_sm_count();
            std::vector<dp::Stage> st((size_t)L * 4);
            std::vector<dp::LayerW> lw((size_t)L);
            auto units = [&](int dd) { return (int)((dd / block_elems(T)) * block_units(T)); };
            for (int l = 0; l < L; ++l) {
                lw[l] = dp::LayerW{d->rms_att[l], d->rms_ffn[l]};
                dp::Stage& a = st[(size_t)l * 4 + 0];
                a.nmat = 3;
                a.w[0] = wq[l]; a.w[1] = wk[l]; a.w[2] = wv[l];
                a.rows[0] = D.q_dim; a.rows[1] = D.kv_dim; a.rows[2] = D.kv_dim;
                a.out[0] = d->q; a.out[1] = d->kc; a.out[2] = d->vc;
                a.rb = (int)row_bytes(T, m->dim); a.U = units(m->dim); a.total = D.q_dim + 2LL * D.kv_dim;
                dp::Stage& o = st[(size_t)l * 4 + 1];
                o.nmat = 1; o.w[0] = wo[l]; o.rows[0] = m->dim; o.out[0] = d->delta;
                o.rb = (int)row_bytes(T, D.q_dim); o.U = units(D.q_dim); o.total = m->dim;
                dp::Stage& f = st[(size_t)l * 4 + 2];
                f.nmat = 2; f.w[0] = w1[l]; f.w[1] = w3[l]; f.rows[0] = hid; f.rows[1] = hid;
                f.out[0] = d->hb; f.out[1] = d->hb2;
                f.rb = (int)row_bytes(T, m->dim); f.U = units(m->dim); f.total = 2LL * hid;
                dp::Stage& w = st[(size_t)l * 4 + 3];
                w.nmat = 1; w.w[0] = w2[l]; w.rows[0] = m->dim; w.out[0] = d->delta;
                w.rb = (int)row_bytes(T, hid); w.U = units(hid); w.total = m->dim;
            }
            dp::Params& P = d->pp;
            P.L = L;
            P.dim = m->dim; P.q_dim = D.q_dim; P.kv_dim = D.kv_dim; P.hd = hd; P.n_heads = D.n_heads;
            P.n_kv = D.n_kv; P.kv_mul = D.kv_mul; P.hidden = hid; P.seq_len = D.seq_len; P.vocab = D.vocab;
            P.kv_type = D.kv_type; P.inv_sqrt = D.inv_sqrt;
            P.tok = d->tok; P.pos = d->pos;
            P.embd = d->embd; P.embd_type = d->embd_type; P.embd_rb = d->embd_rb;
            P.q = d->q; P.kc = d->kc; P.vc = d->vc; P.xa = d->xa; P.delta = d->delta; P.h1 = d->hb; P.h3 = d->hb2;
            P.kcache = d->kcache; P.vcache = d->vcache; P.layer_kv = (long long)B * D.seq_len * D.kv_dim;
            P.rope = d->rope; P.err = device_error_word();
            P.stages = st.data();  // host copy while sizing
            size_t smem = 0;
            int rc2 = persist_layout(P, T, grid, &smem);
            float* x1 = nullptr;
            dp::Stage* dst = nullptr;
            dp::LayerW* dlw = nullptr;
            unsigned* bar = nullptr;
            if (rc2 == QUANTR_OK) {
                cudaError_t e2 = dev_alloc(d, &x1, (size_t)m->dim);
                if (e2 == cudaSuccess) e2 = dev_alloc(d, &dst, st.size());
                if (e2 == cudaSuccess) e2 = dev_alloc(d, &dlw, lw.size());
                if (e2 == cudaSuccess) e2 = dev_alloc(d, &bar, 4);
                if (e2 == cudaSuccess)
                    e2 = cudaMemcpy(dst, st.data(), st.size() * sizeof(dp::Stage), cudaMemcpyHostToDevice);
                if (e2 == cudaSuccess)
                    e2 = cudaMemcpy(dlw, lw.data(), lw.size() * sizeof(dp::LayerW), cudaMemcpyHostToDevice);
                if (e2 == cudaSuccess) e2 = persist_set_smem(T, D.kv_type, smem);
                int per_sm = 0;
                if (e2 == cudaSuccess)
                    e2 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                        &per_sm, (const void*)persist_kernel(T, D.kv_type), dp::kPersistThreads, smem);
                if (e2 == cudaSuccess && per_sm >= 1) {
                    P.stages = dst;
                    P.layers = dlw;
                    P.X[0] = d->x;
                    P.X[1] = x1;
                    P.bar = bar;
                    d->persist = true;
                    d->persist_type = T;
                    d->persist_grid = grid;
                    d->persist_smem = smem;
                } else {
                    cudaGetLastError();
                }
            }
        }
    }

    // Per-step bytes: every linear once, norms, one embedding row per sequence.
    size_t wb = 0;
    for (int l = 0; l < L; ++l) {
        wb += tensor_bytes(m->wq_type[l], D.q_dim, m->dim) + tensor_bytes(m->wk_type[l], D.kv_dim, m->dim) +
              tensor_bytes(m->wv_type[l], D.kv_dim, m->dim) + tensor_bytes(m->wo_type[l], m->dim, D.q_dim) +
              (size_t)2 * m->dim * 4;
        if (d->E == 0)
            wb += tensor_bytes(m->w1_type[l], hid, m->dim) + tensor_bytes(m->w3_type[l], hid, m->dim) +
                  tensor_bytes(m->w2_type[l], m->dim, hid);
    }
    wb += tensor_bytes(m->wcls_type, D.vocab, m->dim) + (size_t)m->dim * 4 +
          (size_t)B * (m->token_embd_row_bytes ? m->token_embd_row_bytes : (size_t)m->dim * 4);
    d->weight_bytes = wb;
    d->kv_pos_bytes = (size_t)L * 2 * D.kv_dim * (D.kv_type ? 2 : 4);

    // Dynamic shared memory of the attention kernels beyond the default 48 KB:
    // raised to what this decoder needs, never lowered (another decoder's
    // captured steps may need more).
    {
        const int ssm = (kScoreTile * (hd + 4) + D.kv_mul * hd) * 4;
        const int vsm = (int)att_v_smem(D);
        auto raise = [](const void* f, int bytes) {
            cudaFuncAttributes fa{};
            if (cudaFuncGetAttributes(&fa, f) != cudaSuccess) return false;
            if (fa.maxDynamicSharedSizeBytes >= bytes) return true;
            return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
        };
        if (!raise((const void*)k_att_scores<0, true>, ssm) || !raise((const void*)k_att_scores<1, true>, ssm) ||
            !raise((const void*)k_att_scores<0, false>, ssm) || !raise((const void*)k_att_scores<1, false>, ssm) ||
            !raise((const void*)k_att_softmax_v<0>, vsm) || !raise((const void*)k_att_softmax_v<1>, vsm) ||
            !raise((const void*)k_att_softmax_v_head<0>, (int)att_vh_smem(D)) ||
            !raise((const void*)k_att_softmax_v_head<1>, (int)att_vh_smem(D)))
            return fail(QUANTR_ERR_CUDA);
    }

    // ---- warm-up (MoE tensor-core plans are made on their first call), then
    // clean caches and the two graphs ----
    k_ctl_set<<<1, 1, 0, d->stream>>>(d->ctl, MODE_EXPLICIT, 0, d->ring_cap);
    int rc = enqueue_step(d, d->stream, !parent);
    if (rc) return fail(rc);
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return fail(QUANTR_ERR_CUDA);
    // The warm-up wrote garbage rows; the cache starts zeroed like the
    // reference's calloc'd one (src/model.c:128-137).
    if (cudaMemsetAsync(d->kcache, 0, kv_elems * (D.kv_type ? 2 : 4), d->stream) != cudaSuccess ||
        cudaMemsetAsync(d->vcache, 0, kv_elems * (D.kv_type ? 2 : 4), d->stream) != cudaSuccess)
        return fail(QUANTR_ERR_CUDA);
    if (!parent) rc = capture(d, true, &d->g_decode, &d->nodes_decode);
    if (!rc) rc = capture(d, false, &d->g_prefill, &d->nodes_prefill);
    if (rc) return fail(rc);
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return fail(QUANTR_ERR_CUDA);
    d->load_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    *out = d;
    return QUANTR_OK;
}

} // namespace

extern "C" {

int quantr_decoder_create(quantr_decoder** out, const quantr_model* m, int batch)
{
    int rc = create_impl(out, m, batch, nullptr);
    if (rc || batch != 1) return rc;
    // One sequence: prompts are prefilled kPrefillChunk positions per step
    // (the tokens' GEMVs as tensor-core jobs), which needs the whole prompt
    // within seq_len.  Without the chunked decoder prefill is per position.
    quantr_decoder* d = *out;
    quantr_decoder* pf = nullptr;
    if (m->seq_len >= 2 && create_impl(&pf, m, std::min(kPrefillChunk, m->seq_len), d) == QUANTR_OK) {
        d->pf = pf;
        d->device_bytes += pf->device_bytes;
        const size_t kv = (size_t)m->n_layers * d->D.kv_B * d->D.seq_len * d->D.kv_dim * (d->D.kv_type ? 2 : 4);
        if (cudaMemset(d->kcache, 0, kv) != cudaSuccess || cudaMemset(d->vcache, 0, kv) != cudaSuccess) {
            cudaGetLastError();
            destroy(d);
            *out = nullptr;
            return QUANTR_ERR_CUDA;
        }
    }
    cudaGetLastError();
    return QUANTR_OK;
}

void quantr_decoder_destroy(quantr_decoder* d) { destroy(d); }

int quantr_decoder_step_dev(quantr_decoder* d, const int* tokens, const int* pos, float* logits, long long ldl,
                            int* next, void* stream)
{
    if (!d || !tokens || !pos || (logits && ldl < d->D.vocab)) return QUANTR_ERR_BAD_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t nb = (size_t)d->D.B * sizeof(int);
    cudaError_t e = cudaMemcpyAsync(d->tok, tokens, nb, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->pos, pos, nb, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) {
        k_ctl_set<<<1, 1, 0, s>>>(d->ctl, MODE_EXPLICIT, 0, d->ring_cap);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaGraphLaunch(d->g_decode, s);
    if (e == cudaSuccess && logits)
        e = cudaMemcpy2DAsync(logits, (size_t)ldl * 4, d->logits, (size_t)d->D.vocab * 4, (size_t)d->D.vocab * 4,
                              d->D.B, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess && next) e = cudaMemcpyAsync(next, d->next, nb, cudaMemcpyDeviceToDevice, s);
    return code_of(e);
}

} // extern "C"

namespace {
// Prefill of the n_prompt positions whose tokens are in d->prompt (and, for a
// chunked prefill, in d->pf->prompt): chunked-prefill graph replays when the
// decoder has one, else one prefill-graph replay per position.
cudaError_t enqueue_prefill(quantr_decoder* d, int n_prompt, cudaStream_t s)
{
    cudaError_t e = cudaSuccess;
    if (d->pf && n_prompt <= d->D.seq_len) {
        quantr_decoder* c = d->pf;
        k_ctl_set<<<1, 1, 0, s>>>(c->ctl, MODE_PREFILL_CHUNK, n_prompt, c->ring_cap);
        e = cudaGetLastError();
        for (int i = 0; i * c->D.B < n_prompt && e == cudaSuccess; ++i) e = cudaGraphLaunch(c->g_prefill, s);
        return e;
    }
    k_ctl_set<<<1, 1, 0, s>>>(d->ctl, MODE_PREFILL, n_prompt, d->ring_cap);
    e = cudaGetLastError();
    for (int i = 0; i < n_prompt && e == cudaSuccess; ++i) e = cudaGraphLaunch(d->g_prefill, s);
    return e;
}

// Copies a prompt into the decoder's (and its chunked child's) prompt buffer.
cudaError_t put_prompt(quantr_decoder* d, const int* prompt, size_t bytes, cudaMemcpyKind kind, cudaStream_t s)
{
    cudaError_t e = cudaMemcpyAsync(d->prompt, prompt, bytes, kind, s);
    if (e == cudaSuccess && d->pf) e = cudaMemcpyAsync(d->pf->prompt, prompt, bytes, kind, s);
    return e;
}
} // namespace

extern "C" {

int quantr_decoder_generate(quantr_decoder* d, const int* prompt, int n_prompt, int steps, int* out)
{
    if (!d || !prompt || n_prompt < 1 || n_prompt > d->prompt_cap || steps < 0 || (steps && !out))
        return QUANTR_ERR_BAD_ARG;
    const int B = d->D.B;
    for (long long i = 0; i < (long long)B * n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= d->D.vocab) return QUANTR_ERR_BAD_ARG;
    cudaStream_t s = d->stream;
    cudaError_t e = put_prompt(d, prompt, (size_t)B * n_prompt * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = enqueue_prefill(d, n_prompt, s);
    if (e == cudaSuccess) {
        k_ctl_set<<<1, 1, 0, s>>>(d->ctl, MODE_DECODE, n_prompt, d->ring_cap);
        e = cudaGetLastError();
    }
    std::vector<int> ring;
    for (int done = 0; done < steps && e == cudaSuccess;) {
        const int chunk = std::min(steps - done, d->ring_cap);
        for (int i = 0; i < chunk && e == cudaSuccess; ++i) e = cudaGraphLaunch(d->g_decode, s);
        ring.resize((size_t)chunk * B);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(ring.data(), d->ring + (size_t)(done % d->ring_cap) * B, ring.size() * 4,
                                cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        for (int i = 0; i < chunk && e == cudaSuccess; ++i)
            for (int b = 0; b < B; ++b) out[(size_t)b * steps + done + i] = ring[(size_t)i * B + b];
        done += chunk;
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    const int rc = code_of(e);
    if (rc) return rc;
    const int dv = quantr_gpu_device_status(s, 0);
    return dv == QUANTR_ERR_ROUTING ? QUANTR_OK : dv;
}

int quantr_decoder_generate_dev(quantr_decoder* d, const int* prompt, int n_prompt, int steps, int* out, void* stream)
{
    if (!d || !prompt || n_prompt < 1 || n_prompt > d->prompt_cap || steps < 0 || steps > d->ring_cap ||
        (steps && !out))
        return QUANTR_ERR_BAD_ARG;
    const int B = d->D.B;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = put_prompt(d, prompt, (size_t)B * n_prompt * 4, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = enqueue_prefill(d, n_prompt, s);
    if (e == cudaSuccess && steps) {
        k_ctl_set<<<1, 1, 0, s>>>(d->ctl, MODE_DECODE, n_prompt, d->ring_cap);
        e = cudaGetLastError();
        for (int i = 0; i < steps && e == cudaSuccess; ++i) e = cudaGraphLaunch(d->g_decode, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(out, d->ring, (size_t)steps * B * 4, cudaMemcpyDeviceToDevice, s);
    }
    return code_of(e);
}

int quantr_decoder_launches(const quantr_decoder* d, int* decode_step, int* prefill_step)
{
    if (!d) return QUANTR_ERR_BAD_ARG;
    if (decode_step) *decode_step = d->nodes_decode;
    if (prefill_step) *prefill_step = d->nodes_prefill;
    return QUANTR_OK;
}

const float* quantr_forward_runtime(quantr_decoder* d, int token, int pos)
{
    if (!d || d->D.B != 1 || token < 0 || token >= d->D.vocab || pos < 0 || pos >= d->D.seq_len) return nullptr;
    cudaStream_t s = d->stream;
    const int tp[2] = {token, pos};
    cudaError_t e = cudaMemcpyAsync(d->tok, &tp[0], 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->pos, &tp[1], 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        k_ctl_set<<<1, 1, 0, s>>>(d->ctl, MODE_EXPLICIT, 0, d->ring_cap);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaGraphLaunch(d->g_decode, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d->host_logits, d->logits, (size_t)d->D.vocab * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return d->host_logits;
}

void quantr_prefill_runtime(quantr_decoder* d, const int* tokens, int n)
{
    if (!d || d->D.B != 1 || !tokens || n <= 0 || n > d->prompt_cap) return;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= d->D.vocab) return;
    cudaStream_t s = d->stream;
    cudaError_t e = put_prompt(d, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = enqueue_prefill(d, n, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) cudaGetLastError();
}

int quantr_debug_expf_dev(float* out, uint32_t first, long long n, void* stream)
{
    if (!out || n < 0) return QUANTR_ERR_BAD_ARG;
    if (n == 0) return QUANTR_OK;
    k_debug_expf<<<(unsigned)std::min<long long>((n + 255) / 256, 148 * 64), 256, 0,
                   static_cast<cudaStream_t>(stream)>>>(out, first, n);
    return code_of(cudaGetLastError());
}

} // extern "C"

namespace {
// Plans of quantr_moe_shared_dev, one per configuration (first call plans).
struct SharedPlan {
    quantr_program* p13 = nullptr;
    quantr_program* p2 = nullptr;
    float *h1 = nullptr, *h3 = nullptr, *o = nullptr, *g = nullptr;
};
std::mutex g_shared_mu;
std::map<std::tuple<int, const void*, const void*, const void*, const float*, const float*, float*, int, int, int,
                    long long, long long>,
         SharedPlan>
    g_shared;
} // namespace

extern "C" {

int quantr_moe_shared_dev(float* out, long long ldo, const float* xb, long long ldx, int T, const float* gate,
                          const void* w1, uint32_t t1, const void* w3, uint32_t t3, const void* w2, uint32_t t2,
                          int dim, int hidden, void* stream)
{
    if (T <= 0) return QUANTR_OK;
    if (!out || !xb || !gate || !w1 || !w2 || !w3 || dim <= 0 || hidden <= 0 || ldo < dim || ldx < dim ||
        T > kMaxBatch)
        return QUANTR_ERR_BAD_ARG;
    if (!type_supported(t1) || !type_supported(t2) || !type_supported(t3)) return QUANTR_ERR_UNSUPPORTED_TYPE;
    int dev = 0;
    cudaGetDevice(&dev);
    SharedPlan* P = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_shared_mu);
        auto key = std::make_tuple(dev, w1, w3, w2, xb, gate, out, T, dim, hidden, ldo, ldx);
        auto it = g_shared.find(key);
        if (it == g_shared.end()) {
            SharedPlan sp;
            cudaError_t e = cudaMalloc(&sp.h1, (size_t)T * hidden * 4);
            if (e == cudaSuccess) e = cudaMalloc(&sp.h3, (size_t)T * hidden * 4);
            if (e == cudaSuccess) e = cudaMalloc(&sp.o, (size_t)T * dim * 4);
            if (e == cudaSuccess) e = cudaMalloc(&sp.g, (size_t)T * 4);
            int rc = e == cudaSuccess ? QUANTR_OK : QUANTR_ERR_OOM;
            if (!rc) {
                quantr_gemv_job j13[2] = {{w1, t1, hidden, dim, T, xb, ldx, sp.h1, hidden},
                                          {w3, t3, hidden, dim, T, xb, ldx, sp.h3, hidden}};
                rc = quantr_program_create(&sp.p13, j13, 2);
            }
            if (!rc) {
                quantr_gemv_job j2 = {w2, t2, dim, hidden, T, sp.h1, hidden, sp.o, dim};
                const float* xm = sp.h3;
                rc = program_create_ex(&sp.p2, &j2, &xm, 1);
            }
            if (rc) {
                cudaGetLastError();
                quantr_program_destroy(sp.p13);
                quantr_program_destroy(sp.p2);
                cudaFree(sp.h1);
                cudaFree(sp.h3);
                cudaFree(sp.o);
                cudaFree(sp.g);
                return rc;
            }
            it = g_shared.emplace(key, sp).first;
        }
        P = &it->second;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    LaunchCfg c;
    c.stream = s;
    if (quantr_program_run(P->p13, s) != QUANTR_OK || quantr_program_run(P->p2, s) != QUANTR_OK)
        return QUANTR_ERR_CUDA;
    cudaError_t e = launch_gemv_f32(gate, xb, ldx, P->g, 1, 1, dim, T, c);
    if (e == cudaSuccess) {
        if (ldo == dim)
            e = launch_ex(&k_shexp_add, dim3((dim + 255) / 256, T), dim3(256), 0, c, out, (const float*)P->o,
                          (const float*)P->g, dim);
        else
            e = cudaErrorInvalidValue;
    }
    return code_of(e);
}

int quantr_decoder_kv(const quantr_decoder* d, void** key_cache, void** value_cache, size_t* bytes)
{
    if (!d) return QUANTR_ERR_BAD_ARG;
    if (key_cache) *key_cache = d->kcache;
    if (value_cache) *value_cache = d->vcache;
    if (bytes)
        *bytes = (size_t)d->n_layers * d->D.kv_B * d->D.seq_len * d->D.kv_dim * (d->D.kv_type ? 2 : 4);
    return QUANTR_OK;
}

int quantr_decoder_info(const quantr_decoder* d, size_t* weight_bytes, size_t* kv_bytes_per_position,
                        size_t* device_bytes)
{
    if (!d) return QUANTR_ERR_BAD_ARG;
    if (weight_bytes) *weight_bytes = d->weight_bytes;
    if (kv_bytes_per_position) *kv_bytes_per_position = d->kv_pos_bytes;
    if (device_bytes) *device_bytes = d->device_bytes;
    return QUANTR_OK;
}

} // extern "C"
