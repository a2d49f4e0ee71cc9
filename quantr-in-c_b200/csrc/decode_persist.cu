// decode_persist.cu -- the one-token decode step (forward_runtime,
// src/runtime.c:94-285) for dense models as ONE persistent kernel.
//
// At batch 1 every phase of a layer is latency-bound: the weights of a whole
// layer (25 MB for TinyLlama) stream in ~4 us, but the step has ~10 dependent
// stages per layer, and as separate kernels each dependency costs a launch,
// a ramp and a drain.  Here one cooperative launch of one CTA per SM runs all
// layers; the stages are separated by grid barriers:
//   NORM+QKV  every CTA: x += delta, rmsnorm (its own copy; no barrier needed),
//             Q8_0-quantize xb into shared memory, then its slice of the
//             Wq|Wk|Wv rows -> q, k, v
//   ATTN      one CTA per KV head: RoPE, K/V rows into the cache, scores,
//             softmax, value rows (src/runtime.c:19-41, 129-194)
//   O         every CTA: quantize the attention output, its Wo rows -> delta
//   NORM+W13  every CTA: x += delta, rmsnorm, quantize, its W1|W3 rows -> h1, h3
//   W2        every CTA: quantize silu(h1)*h3, its W2 rows -> delta
// Weights do not depend on activations, so each CTA's rows for a GEMV stage
// are bulk-copied into shared memory (two regions, alternating) one stage
// ahead and are resident when the stage's input arrives.  Every value is the
// reference's: exact per-unit terms (quant_decode.cuh), left-to-right sums,
// explicitly rounded fp32 (and fp64 inside expf), as in decode.cu.
//
// Bounded everywhere: grid barriers and mbarrier waits give up after 250 ms,
// record DEV_ERR_WAIT_TIMEOUT, drain this CTA's copies in flight (bounded) and
// return.
#include "quantr_cuda.h"

#include "decode_persist.cuh"
#include "device_common.cuh"
#include "formats.cuh"
#include "launch_util.cuh"
#include "libm_ref.cuh"
#include "quant_decode.cuh"

#include <algorithm>

namespace qr {
namespace dp {

constexpr int kWarps = kPersistThreads / 32;
constexpr int kKVTile = 128;  // cached key/value rows per stage of the attention ring
constexpr int kCopyChunk = 8192;  // bytes per bulk copy: many copies in flight per SM

__device__ __forceinline__ float kvr(int kvt, float v) { return kvt ? h2f_ref(f2h_ref(v)) : v; }
__device__ __forceinline__ void kv_store(void* c, int kvt, long long i, float v)
{
    if (kvt)
        reinterpret_cast<uint16_t*>(c)[i] = (uint16_t)f2h_ref(v);
    else
        reinterpret_cast<float*>(c)[i] = v;
}

// Grid barrier: every CTA arrives once per call; `target` counts arrivals.
// Gives up after kWaitNs (error word + CTA abort flag).
__device__ __forceinline__ bool grid_sync(const Params& p, unsigned& target, int* s_abort)
{
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0 && !*s_abort) {
        __threadfence();
        atomicAdd(p.bar, 1u);
        const unsigned long long t0 = gtimer();
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
            if (v >= target) break;
            if (gtimer() - t0 > kWaitNs) {
                atomicExch(p.err, DEV_ERR_WAIT_TIMEOUT);
                *s_abort = 1;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
    }
    __syncthreads();
    return !*s_abort;
}

// Rows [r0, r1) of a stage's concatenated matrices (all rb bytes per row,
// rb % 16 == 0) into shared memory at dst, consecutive.  One thread.
__device__ __forceinline__ uint32_t issue_rows(uint8_t* dst, const Stage& st, int r0, int r1, uint64_t* bar)
{
    uint32_t bytes = 0;
    int base = 0;
    for (int m = 0; m < st.nmat; ++m) {
        const int a = max(r0, base), b = min(r1, base + st.rows[m]);
        if (a < b) bytes += (uint32_t)(b - a) * (uint32_t)st.rb;
        base += st.rows[m];
    }
    mbar_arrive_expect_tx(bar, bytes);
    base = 0;
    for (int m = 0; m < st.nmat; ++m) {
        const int a = max(r0, base), b = min(r1, base + st.rows[m]);
        if (a < b) {
            const uint8_t* src = st.w[m] + (long long)(a - base) * st.rb;
            uint8_t* d = dst + (long long)(a - r0) * st.rb;
            long long n = (long long)(b - a) * st.rb;
            for (long long off = 0; off < n; off += kCopyChunk)
                bulk_g2s(d + off, src + off, (uint32_t)min((long long)kCopyChunk, n - off), bar);
        }
        base += st.rows[m];
    }
    return bytes;
}

__device__ __forceinline__ void stage_rows(const Stage& st, int& r0, int& r1)
{
    const long long R = st.total;
    r0 = (int)(R * blockIdx.x / gridDim.x);
    r1 = (int)(R * (blockIdx.x + 1) / gridDim.x);
}

// Q8_0 quantization (quantize_row_q8_0, src/quant.c:143-158) of n values into
// shared memory, natural order: q[u*32 + e], dx[u] (decoded fp16 scale),
// sx[u] (quant sum).  Warp per block, lane = element; get(i) supplies element
// i.  A warp's blocks are u = warp + k*kWarps; every input of a thread is
// fetched (k = 0..NB-1) before the first block is quantized, so the global
// loads behind get() cost one round trip.
template <int NB, typename F>
__device__ __forceinline__ void quant_act(int n, int8_t* q, float* dx, int* sx, F get)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = n / 32;
    float v[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        const int u = warp + k * kWarps;
        v[k] = u < nb ? get(u * 32 + lane) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        const int u = warp + k * kWarps;
        if (u < nb) {
            uint32_t h;
            int sum;
            q[u * 32 + lane] = q8_block_warp(v[k], h, sum);
            if (lane == 0) {
                dx[u] = h2f_ref(h);
                sx[u] = sum;
            }
        }
    }
}
// Blocks per warp the quantizers are compiled for (inputs of up to
// kQuantNB * kWarps * 32 elements).
constexpr int kQuantNB = 12;

// out = rows [r0, r1) of the stage's matrices . activations, rows resident at
// w_sm (consecutive, rb bytes each).  Exact per-unit terms into terms[row][u]
// (padded rows), then one thread per row sums its terms left to right.
template <uint32_t T>
__device__ __forceinline__ void gemv_rows(const uint8_t* sm, uint32_t w_off, int nrows, int rb, int U,
                                          const int8_t* xq, const float* xd, const int* xs, float* terms,
                                          int r0, const Stage& st)
{
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sm);
    const int G = U / 8;  // 8-unit groups per row
    const int ld = U + 1;
    for (int it = threadIdx.x; it < nrows * G; it += kPersistThreads) {
        const int r = it / G, g = it - r * G;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int u = g * 8 + k;
            Unit o;
            decode_unit<T>(s32, sm, w_off + (uint32_t)(r * rb), u, o);
            const uint4* xv = reinterpret_cast<const uint4*>(xq + u * 32);
            int isum = dot8(o.wq, permute_x16<T>(xv[0]), permute_x16<T>(xv[1]));
            const int bsum = xs[u];
            if (T == T_Q6_K) isum -= 32 * bsum;  // quants stored with +32 offset
            terms[r * ld + u] = unit_term<T>(o.a, o.b, isum, bsum, xd[u]);
        }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < nrows; r += kPersistThreads) {
        const float* tp = terms + r * ld;
        float s = 0.0f;
        int u = 0;
        for (; u + 8 <= U; u += 8) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = tp[u + k];
#pragma unroll
            for (int k = 0; k < 8; ++k) s = __fadd_rn(s, v[k]);
        }
        for (; u < U; ++u) s = __fadd_rn(s, tp[u]);
        // row r0 + r of the concatenation -> its matrix's output
        int row = r0 + r, m = 0;
        while (m + 1 < st.nmat && row >= st.rows[m]) row -= st.rows[m++];
        st.out[m][row] = s;
    }
}

// rmsnorm (src/kernels.c:179-189) of xs[0..dim) with weights w: one thread
// walks the sum of squares, returns the scale to every thread.
__device__ __forceinline__ float rms_scale(const float* xs, int dim, float* s_scale)
{
    if (threadIdx.x == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        float ss = 0.0f;
        int k = 0;
        for (; 4 * (k + 8) <= dim; k += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = x4[k + u];
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
        *s_scale = __fdiv_rn(1.0f, __fsqrt_rn(ss));
    }
    __syncthreads();
    return *s_scale;
}

// xs = x + delta elementwise (the residual add, src/runtime.c:197-199,
// 281-283), float4 words, every load of a thread issued before its adds.
__device__ __forceinline__ void add4(float* xs, const float* x, const float* delta, int dim)
{
    const float4* a = reinterpret_cast<const float4*>(x);
    const float4* b = reinterpret_cast<const float4*>(delta);
    float4* o = reinterpret_cast<float4*>(xs);
#pragma unroll 4
    for (int k = threadIdx.x; k < dim / 4; k += kPersistThreads) {
        const float4 u = a[k], v = b[k];
        o[k] = make_float4(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y), __fadd_rn(u.z, v.z), __fadd_rn(u.w, v.w));
    }
}

struct Smem {
    uint8_t* base;
    uint64_t* bar;  // [2] weight regions, [2] attention ring
    float* xs;      // dim
    int8_t* xq;     // Umax * 32
    float* xd;      // Umax
    int* xsum;      // Umax
    float* terms;   // rows_max * (Umax + 1)
    uint32_t r_off[2];
};

// The attention of query head h = kh*kv_mul + m (B = 1) at position `pos`
// (src/runtime.c:139-194), one CTA, scratch in region 0: RoPE of the head's
// query and of its KV head's key (src/runtime.c:19-41), the K/V rows of this
// position into the cache (stored by the group's first head, m == 0; the
// others use the same values from registers), scores against the cached
// keys (tiles through a 2-stage bulk-copy ring, converted into padded rows),
// softmax_ref, and the value rows accumulated position by position.
template <int KVT>
__device__ void attn_head(const Params& p, const Smem& S, int l, int kh, int m, int pos, uint32_t* ring_uses,
                          int* s_abort)
{
    const int hd = p.hd, np = pos + 1;
    constexpr int ES = KVT ? 2 : 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* scr = S.base + S.r_off[0];
    float* Qs = reinterpret_cast<float*>(scr);     // hd
    float* Kc = Qs + hd;                           // hd (current key, as the cache returns it)
    float* Vc = Kc + hd;                           // hd
    float* Sc = Vc + hd;                           // seq_len scores / probabilities
    float* red = Sc + p.seq_len;                   // kWarps reduction slots
    float* Kp = red + 32;                          // kKVTile * (hd + 1) padded key rows
    uint8_t* ring = reinterpret_cast<uint8_t*>(Kp + kKVTile * (hd + 1));
    ring = reinterpret_cast<uint8_t*>(((uintptr_t)ring + 127) & ~(uintptr_t)127);
    const int tile_bytes = kKVTile * hd * ES;
    uint64_t* rbar = S.bar + 2;
    const long long hbase = (long long)l * p.layer_kv + (long long)kh * p.seq_len * hd;
    const float2* rp = p.rope + (long long)pos * (p.q_dim / 2);
    const int h = kh * p.kv_mul + m;

    const int nt = (pos + kKVTile - 1) / kKVTile;  // tiles of cached rows (0 .. pos-1)
    const uint8_t* ksrc = static_cast<const uint8_t*>(p.kcache) + hbase * ES;
    const uint8_t* vsrc = static_cast<const uint8_t*>(p.vcache) + hbase * ES;
    auto issue = [&](int j) {  // j < nt: K tile j; nt <= j < 2nt: V tile j - nt
        const int st = j & 1, t0 = (j % nt) * kKVTile, n = min(kKVTile, pos - t0);
        mbar_arrive_expect_tx(&rbar[st], (uint32_t)(n * hd * ES));
        bulk_g2s(ring + st * tile_bytes, (j < nt ? ksrc : vsrc) + (long long)t0 * hd * ES, (uint32_t)(n * hd * ES),
                 &rbar[st]);
    };
    auto wait = [&](int j) {
        const int st = j & 1;
        const uint32_t par = (ring_uses[st] + (uint32_t)(j >> 1)) & 1u;
        if (!mbar_wait_bounded(&rbar[st], par, p.err, s_abort)) *s_abort = 1;
    };
    if (tid == 0) {
        // generic writes of the previous stage to this region precede the
        // async-proxy copies into it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int jj = 0; jj < min(2, 2 * nt); ++jj) issue(jj);
    }
    for (int i = 2 * tid; i < hd; i += 2 * kPersistThreads) {
        const int gq = h * hd + i;
        const float2 cq = rp[gq >> 1];
        const float a = p.q[gq], b = p.q[gq + 1];
        Qs[i] = __fsub_rn(__fmul_rn(a, cq.x), __fmul_rn(b, cq.y));
        Qs[i + 1] = __fadd_rn(__fmul_rn(a, cq.y), __fmul_rn(b, cq.x));
        const int gk = kh * hd + i;
        const float2 ck = rp[gk >> 1];
        const float ka = p.kc[gk], kb = p.kc[gk + 1];
        const float k0 = __fsub_rn(__fmul_rn(ka, ck.x), __fmul_rn(kb, ck.y));
        const float k1 = __fadd_rn(__fmul_rn(ka, ck.y), __fmul_rn(kb, ck.x));
        if (m == 0) {
            kv_store(p.kcache, KVT, hbase + (long long)pos * hd + i, k0);
            kv_store(p.kcache, KVT, hbase + (long long)pos * hd + i + 1, k1);
            kv_store(p.vcache, KVT, hbase + (long long)pos * hd + i, p.vc[gk]);
            kv_store(p.vcache, KVT, hbase + (long long)pos * hd + i + 1, p.vc[gk + 1]);
        }
        Kc[i] = kvr(KVT, k0);
        Kc[i + 1] = kvr(KVT, k1);
        Vc[i] = kvr(KVT, p.vc[gk]);
        Vc[i + 1] = kvr(KVT, p.vc[gk + 1]);
    }
    __syncthreads();
    auto dot_q = [&](const float* kr) {
        float s = 0.0f;
        int i = 0;
        for (; i + 8 <= hd; i += 8) {
            float pr[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) pr[k] = __fmul_rn(Qs[i + k], kr[i + k]);
#pragma unroll
            for (int k = 0; k < 8; ++k) s = __fadd_rn(s, pr[k]);
        }
        for (; i < hd; ++i) s = __fadd_rn(s, __fmul_rn(Qs[i], kr[i]));
        return __fmul_rn(s, p.inv_sqrt);
    };
    int j = 0;
    for (; j < nt; ++j) {  // scores of the cached positions, a tile at a time
        wait(j);
        __syncthreads();
        if (*s_abort) break;
        const int t0 = j * kKVTile, n = min(kKVTile, pos - t0);
        const uint8_t* tile = ring + (j & 1) * tile_bytes;
        for (int e = tid; e < n * hd; e += kPersistThreads) {
            const int r = e / hd, i = e - r * hd;
            Kp[r * (hd + 1) + i] = KVT ? h2f_ref(reinterpret_cast<const uint16_t*>(tile)[e])
                                       : reinterpret_cast<const float*>(tile)[e];
        }
        __syncthreads();
        if (tid == 0 && j + 2 < 2 * nt) issue(j + 2);
        for (int r = tid; r < n; r += kPersistThreads) Sc[t0 + r] = dot_q(Kp + r * (hd + 1));
        __syncthreads();
    }
    if (!*s_abort) {
        if (tid == 0) Sc[pos] = dot_q(Kc);
        __syncthreads();
        // softmax_ref (src/kernels.c:191-207): max from x[0] (a NaN there
        // sticks), expf, a left-to-right sum by one thread, 1/sum, scale.
        float mx = Sc[0];
        const bool nan0 = mx != mx;
        for (int t = tid; t < np; t += kPersistThreads) mx = fmaxf(mx, Sc[t]);
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = red[0];
        for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, red[w]);
        if (nan0) mx = Sc[0];
        for (int t = tid; t < np; t += kPersistThreads) Sc[t] = libm::expf_ref(__fsub_rn(Sc[t], mx));
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            int t = 0;
            for (; t + 8 <= np; t += 8) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = Sc[t + k];
#pragma unroll
                for (int k = 0; k < 8; ++k) sum = __fadd_rn(sum, v[k]);
            }
            for (; t < np; ++t) sum = __fadd_rn(sum, Sc[t]);
            red[kWarps] = __fdiv_rn(1.0f, sum);
        }
        __syncthreads();
        const float inv = red[kWarps];
        for (int t = tid; t < np; t += kPersistThreads) Sc[t] = __fmul_rn(Sc[t], inv);
        __syncthreads();
    }
    // Values: thread i < hd sums att[t] * v_t[i] over t in order.
    float acc = 0.0f;
    for (; j < 2 * nt && !*s_abort; ++j) {
        wait(j);
        __syncthreads();
        if (*s_abort) break;
        const int t0 = (j - nt) * kKVTile, n = min(kKVTile, pos - t0);
        const uint8_t* tile = ring + (j & 1) * tile_bytes;
        if (tid < hd) {
            const float* sp = Sc + t0;
            int r = 0;
            for (; r + 8 <= n; r += 8) {
                float pr[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float v = KVT ? h2f_ref(reinterpret_cast<const uint16_t*>(tile)[(r + k) * hd + tid])
                                        : reinterpret_cast<const float*>(tile)[(r + k) * hd + tid];
                    pr[k] = __fmul_rn(sp[r + k], v);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) acc = __fadd_rn(acc, pr[k]);
            }
            for (; r < n; ++r) {
                const float v = KVT ? h2f_ref(reinterpret_cast<const uint16_t*>(tile)[r * hd + tid])
                                    : reinterpret_cast<const float*>(tile)[r * hd + tid];
                acc = __fadd_rn(acc, __fmul_rn(sp[r], v));
            }
        }
        __syncthreads();
        if (tid == 0 && j + 2 < 2 * nt) issue(j + 2);
    }
    if (*s_abort) {
        // drain what this CTA still has in flight on the ring (bounded)
        if (tid == 0)
            for (int jj = j; jj < min(2 * nt, j + 2); ++jj) {
                const int st = jj & 1;
                mbar_wait_bounded(&rbar[st], (ring_uses[st] + (uint32_t)(jj >> 1)) & 1u, nullptr);
            }
        return;
    }
    if (tid < hd) p.xa[(long long)h * hd + tid] = __fadd_rn(acc, __fmul_rn(Sc[pos], Vc[tid]));
    // ring stage use counts advance by the tiles this call consumed
    if (tid == 0) {
        ring_uses[0] += (uint32_t)nt;
        ring_uses[1] += (uint32_t)nt;
    }
}

template <uint32_t T, int KVT>
__global__ void __launch_bounds__(kPersistThreads, 1) k_decode_persist(const __grid_constant__ Params p)
{
    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ int s_abort;
    __shared__ float s_scale;
    __shared__ uint32_t s_ring_uses[2];
    Smem S;
    S.base = smraw;
    S.bar = reinterpret_cast<uint64_t*>(smraw + p.sm.bar);
    S.xs = reinterpret_cast<float*>(smraw + p.sm.xs);
    S.xq = reinterpret_cast<int8_t*>(smraw + p.sm.xq);
    S.xd = reinterpret_cast<float*>(smraw + p.sm.xd);
    S.xsum = reinterpret_cast<int*>(smraw + p.sm.xsum);
    S.terms = reinterpret_cast<float*>(smraw + p.sm.terms);
    S.r_off[0] = p.sm.r0;
    S.r_off[1] = p.sm.r1;
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(&S.bar[i], 1);
        mbar_fence_init();
        s_abort = 0;
        s_ring_uses[0] = s_ring_uses[1] = 0;
    }
    __syncthreads();
    // Region r (0, 1) receives weights for every other GEMV stage; its
    // mbarrier completes once per load (parity = loads so far & 1).
    uint32_t issued[2] = {0, 0}, waited[2] = {0, 0};
    auto load = [&](int reg, const Stage& st) {
        // Every thread has finished with the region (a CTA or grid barrier
        // separates the stage that last read it); its generic accesses are
        // ordered before the async-proxy copies.
        if (tid == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            int r0, r1;
            stage_rows(st, r0, r1);
            issue_rows(S.base + S.r_off[reg], st, r0, r1, &S.bar[reg]);
        }
        ++issued[reg];
    };
    auto wait_reg = [&](int reg) {
        if (!mbar_wait_bounded(&S.bar[reg], waited[reg] & 1u, p.err, &s_abort)) s_abort = 1;
        ++waited[reg];
    };
    const int dim = p.dim;
    const int pos = p.pos[0];
    int tok = p.tok[0];
    if (tok < 0 || tok >= p.vocab) tok = 0;
    unsigned target = 0;
    int par = 0;  // X[par] holds the current residual stream

    load(0, p.stages[0 * 4 + 0]);  // layer 0 Q/K/V rows
    for (int l = 0; l < p.L; ++l) {
        const LayerW& W = p.layers[l];
        const Stage* st = p.stages + l * 4;
        // ---- NORM + QKV ----
        load(1, st[1]);  // O rows, needed two stages on
        if (l == 0) {
            const uint8_t* row = p.embd + (long long)tok * p.embd_rb;
            for (int i = tid; i < dim; i += kPersistThreads)
                S.xs[i] = p.embd_rb ? dequant_elem(row, p.embd_type, i) : reinterpret_cast<const float*>(p.embd)[(long long)tok * dim + i];
        } else {
            add4(S.xs, p.X[par], p.delta, dim);
        }
        __syncthreads();
        {  // this CTA's slice of the new residual stream
            const int a = (int)((long long)dim * blockIdx.x / gridDim.x), b = (int)((long long)dim * (blockIdx.x + 1) / gridDim.x);
            for (int i = a + tid; i < b; i += kPersistThreads) p.X[par ^ 1][i] = S.xs[i];
            par ^= 1;
        }
        float sc = rms_scale(S.xs, dim, &s_scale);
        quant_act<kQuantNB>(dim, S.xq, S.xd, S.xsum,
                            [&](int i) { return __fmul_rn(W.rms_att[i], __fmul_rn(S.xs[i], sc)); });
        wait_reg(0);
        __syncthreads();
        if (s_abort) break;
        {
            int r0, r1;
            stage_rows(st[0], r0, r1);
            gemv_rows<T>(S.base, S.r_off[0], r1 - r0, st[0].rb, st[0].U, S.xq, S.xd, S.xsum, S.terms, r0, st[0]);
        }
        if (!grid_sync(p, target, &s_abort)) break;
        // ---- ATTN ----
        if ((int)blockIdx.x < p.n_heads)
            attn_head<KVT>(p, S, l, blockIdx.x / p.kv_mul, blockIdx.x % p.kv_mul, pos, s_ring_uses, &s_abort);
        if (!grid_sync(p, target, &s_abort)) break;
        // ---- O ----
        load(0, st[2]);  // W1|W3 rows
        quant_act<kQuantNB>(p.q_dim, S.xq, S.xd, S.xsum, [&](int i) { return p.xa[i]; });
        wait_reg(1);
        __syncthreads();
        if (s_abort) break;
        {
            int r0, r1;
            stage_rows(st[1], r0, r1);
            gemv_rows<T>(S.base, S.r_off[1], r1 - r0, st[1].rb, st[1].U, S.xq, S.xd, S.xsum, S.terms, r0, st[1]);
        }
        if (!grid_sync(p, target, &s_abort)) break;
        // ---- NORM + W1|W3 ----
        load(1, st[3]);  // W2 rows
        add4(S.xs, p.X[par], p.delta, dim);
        __syncthreads();
        {
            const int a = (int)((long long)dim * blockIdx.x / gridDim.x), b = (int)((long long)dim * (blockIdx.x + 1) / gridDim.x);
            for (int i = a + tid; i < b; i += kPersistThreads) p.X[par ^ 1][i] = S.xs[i];
            par ^= 1;
        }
        sc = rms_scale(S.xs, dim, &s_scale);
        quant_act<kQuantNB>(dim, S.xq, S.xd, S.xsum,
                            [&](int i) { return __fmul_rn(W.rms_ffn[i], __fmul_rn(S.xs[i], sc)); });
        wait_reg(0);
        __syncthreads();
        if (s_abort) break;
        {
            int r0, r1;
            stage_rows(st[2], r0, r1);
            gemv_rows<T>(S.base, S.r_off[0], r1 - r0, st[2].rb, st[2].U, S.xq, S.xd, S.xsum, S.terms, r0, st[2]);
        }
        if (!grid_sync(p, target, &s_abort)) break;
        // ---- W2 ----
        if (l + 1 < p.L) load(0, p.stages[(l + 1) * 4 + 0]);  // next layer's Q/K/V rows
        quant_act<kQuantNB>(p.hidden, S.xq, S.xd, S.xsum,
                            [&](int i) { return libm::swiglu_ref(p.h1[i], p.h3[i]); });
        wait_reg(1);
        __syncthreads();
        if (s_abort) break;
        {
            int r0, r1;
            stage_rows(st[3], r0, r1);
            gemv_rows<T>(S.base, S.r_off[1], r1 - r0, st[3].rb, st[3].U, S.xq, S.xd, S.xsum, S.terms, r0, st[3]);
        }
        if (!grid_sync(p, target, &s_abort)) break;
    }
    if (s_abort && tid == 0) {
        // drain this CTA's weight copies still in flight (bounded)
        for (int reg = 0; reg < 2; ++reg)
            while (waited[reg] < issued[reg]) {
                mbar_wait_bounded(&S.bar[reg], waited[reg] & 1u, nullptr);
                ++waited[reg];
            }
    }
}

} // namespace dp

// ---------------------------------------------------------------- host --

namespace {
template <uint32_t T>
void* kernel_for(int kvt)
{
    return kvt ? (void*)&dp::k_decode_persist<T, 1> : (void*)&dp::k_decode_persist<T, 0>;
}
void* kernel_of(uint32_t type, int kvt)
{
    switch (type) {
    case T_Q8_0: return kernel_for<T_Q8_0>(kvt);
    case T_Q4_K: return kernel_for<T_Q4_K>(kvt);
    case T_Q5_K: return kernel_for<T_Q5_K>(kvt);
    case T_Q6_K: return kernel_for<T_Q6_K>(kvt);
    default: return nullptr;
    }
}
} // namespace

int persist_layout(dp::Params& p, uint32_t type, int grid, size_t* smem_out)
{
    using namespace dp;
    // largest per-CTA row slice of each region and the largest unit count
    size_t reg[2] = {0, 0}, terms = 0;
    int umax = 0;
    for (int l = 0; l < p.L; ++l)
        for (int s = 0; s < 4; ++s) {
            const Stage& st = p.stages[l * 4 + s];
            const int rows = (int)((st.total + grid - 1) / grid) + 1;
            reg[s & 1] = std::max(reg[s & 1], (size_t)rows * st.rb);
            terms = std::max(terms, (size_t)rows * (st.U + 1) * 4);
            umax = std::max(umax, st.U);
        }
    // attention scratch lives in region 0
    const int ES = p.kv_type ? 2 : 4;
    const size_t att = (size_t)(3 * p.hd + (size_t)p.seq_len + 32 + dp::kKVTile * (p.hd + 1)) * 4 + 128 +
                       2 * (size_t)dp::kKVTile * p.hd * ES;
    reg[0] = std::max(reg[0], att);
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) {
        off = (off + align - 1) / align * align;
        const size_t o = off;
        off += bytes;
        return (uint32_t)o;
    };
    p.sm.bar = take(4 * 8, 16);
    p.sm.xs = take((size_t)std::max(p.dim, p.q_dim) * 4, 16);
    p.sm.xq = take((size_t)umax * 32, 16);
    p.sm.xd = take((size_t)umax * 4, 16);
    p.sm.xsum = take((size_t)umax * 4, 16);
    p.sm.terms = take(terms, 16);
    p.sm.r0 = take(reg[0], 128);
    p.sm.r1 = take(reg[1], 128);
    *smem_out = off;
    (void)type;
    return off <= 227 * 1024 - 2048 ? QUANTR_OK : QUANTR_ERR_TOO_LARGE;
}

cudaError_t launch_persist(const dp::Params& p, uint32_t type, int grid, size_t smem, cudaStream_t s)
{
    void* k = kernel_of(type, p.kv_type);
    if (!k) return cudaErrorNotSupported;
    cudaError_t e = cudaMemsetAsync(p.bar, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(dp::kPersistThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    void* args[] = {const_cast<dp::Params*>(&p)};
    return cudaLaunchKernelExC(&cfg, k, args);
}

const void* persist_kernel(uint32_t type, int kvt) { return kernel_of(type, kvt); }

cudaError_t persist_set_smem(uint32_t type, int kvt, size_t smem)
{
    void* k = kernel_of(type, kvt);
    if (!k) return cudaErrorNotSupported;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

} // namespace qr
