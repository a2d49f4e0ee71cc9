// moe.cu -- the routed mixture-of-experts FFN block on the device: router
// softmax / top-k / renormalisation and the grouped expert GEMVs of the
// reference's MoE branch (src/runtime.c:202-269), applied to T tokens at once.
//
// Per token the reference computes, with F32 router weights R (E x dim):
//   logits = R.xb (KernelOps matmul), softmax (src/kernels.c:191-207), k
//   passes of arg-max with strict '>' from -1e9 (lowest index wins ties, the
//   winner masked to -1e9), weights renormalised by their left-to-right sum;
//   then for each selected expert in selection order
//   hb = W1.xb, hb2 = W3.xb, hb = silu(hb)*hb2, o = W2.hb, xb2 += o*ew
//   (W1 is the tensor the reference binds to ffn_up, src/model.c:401-418).
//
// Three stages (all launches stream-ordered, programmatic dependent launch),
// so that expert-parallel ranks can run the middle one on their own experts:
//   route:   [router logits: F32 GEMV, one thread per (expert, token)], then
//            one thread per token: softmax, top-k, renormalisation;
//   experts: one CTA groups the (token, slot) pairs whose expert is local, by
//            expert (pair id ascending within each expert); xb is quantized
//            once (the reference quantizes the same xb for every W1/W3 call,
//            src/quant.c:466-474, so one quantization is bit-identical);
//            grouped GEMVs: CTA (row tile, expert) streams its expert's rows
//            once and serves every pair routed to that expert (experts nobody
//            chose are never read); silu(h1)*h3 fused with the Q8_0
//            quantization of hb per pair; grouped GEMV for W2 -> o per pair;
//   combine: out = sum over slots in selection order of o*ew, from +0.0.
// Every GEMV output is bit-identical to the reference's matmul_q_fused for
// that (row, pair).  expf is evaluated correctly rounded (through double
// precision), which differs from glibc's expf in rare last-bit cases.
#include "device_common.cuh"
#include "formats.cuh"
#include "kernels.cuh"
#include "launch_util.cuh"
#include "quant_decode.cuh"

#include <algorithm>
#include <cuda_runtime.h>

namespace qr {
namespace {

constexpr int kThreads = 256;
constexpr int kBT = 8;             // pairs per pass over a staged weight tile
constexpr uint32_t kChunk = 16384; // bytes per bulk copy
constexpr size_t kSmemMax = 227 * 1024;

__device__ __forceinline__ float expf_cr(float x) { return __double2float_rn(exp((double)x)); }

// src/runtime.c:15-17: x / (1.0f + expf(-x)).
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf_cr(-x))); }

// ------------------------------------------------------- route and group --

// Thread t routes token t, working on its row of `probs` (T x E in the
// workspace; logits may alias it).
__global__ void __launch_bounds__(128)
    k_moe_route(const float* logits, long long ldl, float* probs, int T, int E, int k, int* __restrict__ sel,
                float* __restrict__ wts, int* err)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    float* p = probs + (long long)t * E;
    const float* lg = logits + (long long)t * ldl;
    // softmax_ref (src/kernels.c:191-207)
    float m = lg[0];
    for (int e = 1; e < E; ++e)
        if (lg[e] > m) m = lg[e];
    float sum = 0.0f;
    for (int e = 0; e < E; ++e) {
        const float v = expf_cr(__fsub_rn(lg[e], m));
        p[e] = v;
        sum = __fadd_rn(sum, v);
    }
    const float inv = __fdiv_rn(1.0f, sum);
    for (int e = 0; e < E; ++e) p[e] = __fmul_rn(p[e], inv);
    // top-k (src/runtime.c:208-221)
    float w[kMoeMaxK];
    int s_[kMoeMaxK];
    bool bad = false;
    for (int s = 0; s < k; ++s) {
        float best = -1e9f;
        int arg = -1;
        for (int e = 0; e < E; ++e) {
            const float v = p[e];
            if (v > best) {
                best = v;
                arg = e;
            }
        }
        if (arg < 0) {  // non-finite probabilities: the reference would index [-1]
            bad = true;
            break;
        }
        s_[s] = arg;
        w[s] = best;
        p[arg] = -1e9f;
    }
    // renormalisation (src/runtime.c:223-229)
    float tot = 0.0f;
    if (!bad)
        for (int s = 0; s < k; ++s) tot = __fadd_rn(tot, w[s]);
    for (int s = 0; s < k; ++s) {
        sel[t * k + s] = bad ? -1 : s_[s];
        wts[t * k + s] = bad ? 0.0f : __fdiv_rn(w[s], tot);
    }
    if (bad && err) atomicExch(err, DEV_ERR_ROUTING);
}

// One CTA: lists the pairs p = t*k + s whose expert lies in [e0, e0 + El),
// per local expert in pair order (warp ballots), with counts and offsets.
__global__ void __launch_bounds__(1024)
    k_moe_group(const int* __restrict__ sel, int P, int e0, int El, int* __restrict__ counts,
                int* __restrict__ offsets, int* __restrict__ list)
{
    __shared__ int cnt[kMoeMaxExperts];
    __shared__ int off[kMoeMaxExperts + 1];
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int e = warp; e < El; e += nw) {
        int c = 0;
        for (int p0 = 0; p0 < P; p0 += 32) {
            const int q = p0 + lane;
            c += __popc(__ballot_sync(0xffffffffu, q < P && sel[q] == e0 + e));
        }
        if (lane == 0) cnt[e] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0;
        for (int e = 0; e < El; ++e) {
            off[e] = a;
            a += cnt[e];
        }
        off[El] = a;
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= El; e += blockDim.x) {
        offsets[e] = off[e];
        if (e < El) counts[e] = cnt[e];
    }
    for (int e = warp; e < El; e += nw) {
        int o = off[e];
        for (int p0 = 0; p0 < P; p0 += 32) {
            const int q = p0 + lane;
            const bool hit = q < P && sel[q] == e0 + e;
            const unsigned mk = __ballot_sync(0xffffffffu, hit);
            if (hit) list[o + __popc(mk & ((1u << lane) - 1u))] = q;
            o += __popc(mk);
        }
    }
}

// ------------------------------------------------------- grouped GEMV --

struct MoeGemvParams {
    const uint8_t* base[2];
    long long stride[2];
    const uint8_t* const* table[2];
    float* out[2];  // out[z][pair * n + r]
    long long rb;   // row bytes
    int n, U, G, TS;
    const int8_t* xq;
    const float* xd;
    const int32_t* xs;
    int nbx;
    int in_div;  // activation row of pair p is p / in_div
    const int* counts;
    const int* offsets;
    const int* list;
    int* err;
    uint32_t w_off, x_off, xd_off, xs_off, t_off;
};

// CTA (row tile, expert e, matrix z): stages G rows of expert e's matrix z in
// shared memory once, then serves the pairs routed to e kBT at a time.  Each
// (row, pair) output is the reference's left-to-right sum of exact unit terms.
template <uint32_t TYPE>
__global__ void __launch_bounds__(kThreads) k_moe_gemv(const __grid_constant__ MoeGemvParams p)
{
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sm);
    const int tid = threadIdx.x;
    const int e = blockIdx.y, z = blockIdx.z;
    pdl_trigger();
    pdl_wait();  // counts / list / activations come from earlier launches
    const int cnt = p.counts[e];
    if (cnt == 0) return;
    const int first = p.offsets[e];
    const int r0 = blockIdx.x * p.G;
    const int gcnt = min(p.G, p.n - r0);
    const uint8_t* mat = p.table[z] ? p.table[z][e] : p.base[z] + (long long)e * p.stride[z];
    const uint8_t* src = mat + (long long)r0 * p.rb;
    const long long nbytes = (long long)gcnt * p.rb;

    const uint32_t mis = (uint32_t)((uintptr_t)src & 15u);
    const uint32_t wb_off = p.w_off + mis;
    uint8_t* wb = sm + wb_off;
    const long long head = min((long long)((16u - mis) & 15u), nbytes);
    const long long body = (nbytes - head) & ~15LL;
    const long long tail0 = head + body;
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, (uint32_t)body);
        for (long long o = 0; o < body; o += kChunk) {
            const uint32_t sz = (uint32_t)min((long long)kChunk, body - o);
            bulk_g2s(wb + head + o, src + head + o, sz, bar);
        }
    }
    for (long long i = tid; i < head; i += kThreads) wb[i] = src[i];
    for (long long i = tail0 + tid; i < nbytes; i += kThreads) wb[i] = src[i];

    const int U = p.U;
    int8_t* xq = reinterpret_cast<int8_t*>(sm + p.x_off);
    float* xd = reinterpret_cast<float*>(sm + p.xd_off);
    int32_t* xs = reinterpret_cast<int32_t*>(sm + p.xs_off);
    float* terms = reinterpret_cast<float*>(sm + p.t_off);
    const int TS = p.TS;
    float* out = p.out[z];

    const bool ok = mbar_wait_bounded(bar, 0, p.err);
    if (!__syncthreads_and(ok)) {
        mbar_wait_bounded(bar, 0, nullptr);
        return;
    }
    for (int c0 = 0; c0 < cnt; c0 += kBT) {
        const int nb = min(kBT, cnt - c0);
        const int* pl = p.list + first + c0;
        for (int i = tid; i < nb * U * 2; i += kThreads) {
            const int j = i / (2 * U);
            const int r = i - j * 2 * U;
            const long long row = pl[j] / p.in_div;
            const uint4 v = *reinterpret_cast<const uint4*>(p.xq + (row * p.nbx + (r >> 1)) * 32 + (r & 1) * 16);
            *reinterpret_cast<uint4*>(xq + (j * U + (r >> 1)) * 32 + (r & 1) * 16) = permute_x16<TYPE>(v);
        }
        for (int i = tid; i < nb * U; i += kThreads) {
            const int j = i / U, u = i - j * U;
            const long long row = pl[j] / p.in_div;
            xd[i] = p.xd[row * p.nbx + u];
            xs[i] = p.xs[row * p.nbx + u];
        }
        __syncthreads();
        for (int it = tid; it < gcnt * U; it += kThreads) {
            const int g = it / U, u = it - g * U;
            Unit o;
            decode_unit<TYPE>(s32, sm, wb_off + (uint32_t)(g * p.rb), u, o);
#pragma unroll
            for (int t = 0; t < kBT; ++t) {
                if (t < nb) {
                    const uint4* xv = reinterpret_cast<const uint4*>(xq + (t * U + u) * 32);
                    int isum = dot8(o.wq, xv[0], xv[1]);
                    const int bsum = xs[t * U + u];
                    if (TYPE == T_Q6_K) isum -= 32 * bsum;
                    terms[u * TS + g * kBT + t] = unit_term<TYPE>(o.a, o.b, isum, bsum, xd[t * U + u]);
                }
            }
        }
        __syncthreads();
        for (int i = tid; i < gcnt * nb; i += kThreads) {
            const int g = i / nb, t = i - g * nb;
            const float* tp = terms + g * kBT + t;
            float s = 0.0f;
            for (int u = 0; u < U; ++u) s = __fadd_rn(s, tp[u * TS]);
            out[(long long)pl[t] * p.n + r0 + g] = s;
        }
        __syncthreads();
    }
}

// ---------------------------------------------- activation and combine --

// hb = silu(h1)*h3 per pair (src/runtime.c:254-256), quantized to Q8_0 in the
// same step (the reference's matmul_q on W2 quantizes hb, src/quant.c:466-474).
__global__ void __launch_bounds__(kThreads)
    k_moe_act(const float* __restrict__ h1, const float* __restrict__ h3, int hidden, int P,
              const int* __restrict__ sel, int e0, int El, int8_t* __restrict__ q, float* __restrict__ dq,
              int32_t* __restrict__ sq)
{
    pdl_trigger();
    pdl_wait();
    const int nbh = hidden / 32;
    const int lane = threadIdx.x & 31;
    const long long total = (long long)P * nbh;
    const long long step = (long long)gridDim.x * (kThreads / 32);
    for (long long wb = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); wb < total; wb += step) {
        const int pr = (int)(wb / nbh);
        const int b = (int)(wb - (long long)pr * nbh);
        const int se = sel[pr];
        if (se < e0 || se >= e0 + El) continue;  // not a local pair (warp-uniform)
        const long long i = (long long)pr * hidden + b * 32 + lane;
        const float v = __fmul_rn(silu_ref(h1[i]), h3[i]);
        uint32_t h;
        int sum;
        const int8_t qq = q8_block_warp(v, h, sum);
        q[wb * 32 + lane] = qq;
        if (lane == 0) {
            dq[wb] = h2f_ref(h);
            sq[wb] = sum;
        }
    }
}

// out[t][i] = ((0 + o[t,0][i]*w[t,0]) + o[t,1][i]*w[t,1]) + ... in selection
// order (src/runtime.c:241, 262-264).
__global__ void __launch_bounds__(kThreads)
    k_moe_combine(const float* __restrict__ o, int dim, int T, int k, const int* __restrict__ sel,
                  const float* __restrict__ wts, float* __restrict__ out, long long ldo)
{
    pdl_trigger();
    pdl_wait();
    const long long total = (long long)T * dim;
    for (long long idx = (long long)blockIdx.x * kThreads + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * kThreads) {
        const int t = (int)(idx / dim);
        const int i = (int)(idx - (long long)t * dim);
        float acc = 0.0f;
        for (int s = 0; s < k; ++s) {
            const int pr = t * k + s;
            if (sel[pr] < 0) continue;
            acc = __fadd_rn(acc, __fmul_rn(o[(long long)pr * dim + i], wts[pr]));
        }
        out[(long long)t * ldo + i] = acc;
    }
}

// Rows of o for local pairs when W2 has fewer columns than one block (the
// reference's empty sum, 0.0f).
__global__ void __launch_bounds__(kThreads)
    k_moe_zero_rows(float* __restrict__ o, int dim, int P, const int* __restrict__ sel, int e0, int El)
{
    pdl_trigger();
    pdl_wait();
    const long long total = (long long)P * dim;
    for (long long idx = (long long)blockIdx.x * kThreads + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * kThreads) {
        const int se = sel[idx / dim];
        if (se >= e0 && se < e0 + El) o[idx] = 0.0f;
    }
}

// ------------------------------------------------------------- host side --

// Workspace: probs (route) | counts | offsets | list | xb quants | h1 | h3 |
// hb quants (experts).  One layout serves every stage.
struct MoeWs {
    size_t probs, counts, offsets, list, actx, h1, h3, acth, total;
};

size_t a256(size_t v) { return (v + 255) & ~size_t(255); }

MoeWs moe_layout(int T, int E, int k, int dim, int hidden)
{
    const size_t P = (size_t)T * k;
    MoeWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += a256(bytes);
        return at;
    };
    w.probs = take((size_t)T * E * 4);
    w.counts = take((size_t)E * 4);
    w.offsets = take((size_t)(E + 1) * 4);
    w.list = take(P * 4);
    w.actx = take(actq_bytes(dim, T));
    w.h1 = take(P * hidden * 4);
    w.h3 = take(P * hidden * 4);
    w.acth = take(actq_bytes(hidden, (int)P));
    w.total = off;
    return w;
}

template <uint32_t TYPE>
cudaError_t launch_grouped(const ExpertMats* mats, int nmat, float* const* outs, int n, int d, ActQ x, int in_div,
                           const int* counts, const int* offsets, const int* list, int E, int* err,
                           const LaunchCfg& c)
{
    const long long rb = row_bytes(TYPE, d);
    const int U = (d / block_elems(TYPE)) * block_units(TYPE);
    MoeGemvParams p{};
    auto smem_for = [&](int G) {
        p.TS = G * kBT;
        if ((p.TS & 1) == 0) p.TS += 1;
        size_t off = 128;
        p.w_off = (uint32_t)off;
        off += ((size_t)G * rb + 32 + 15) & ~size_t(15);
        p.x_off = (uint32_t)off;
        off += (size_t)kBT * U * 32;
        p.xd_off = (uint32_t)off;
        off += (size_t)kBT * U * 4;
        p.xs_off = (uint32_t)off;
        off += (size_t)kBT * U * 4;
        p.t_off = (uint32_t)off;
        off += (size_t)U * p.TS * 4;
        return off;
    };
    // About 24 KB of weights per CTA (two or three CTAs per SM).
    int G = (int)std::max(1LL, std::min<long long>(n, 24576 / std::max(rb, 1LL)));
    size_t smem = smem_for(G);
    while (G > 1 && smem > kSmemMax / 2) smem = smem_for(--G);
    if (smem > kSmemMax) return cudaErrorInvalidConfiguration;
    for (int z = 0; z < nmat; ++z) {
        p.base[z] = mats[z].base;
        p.stride[z] = mats[z].stride;
        p.table[z] = mats[z].table;
        p.out[z] = outs[z];
    }
    p.rb = rb;
    p.n = n;
    p.U = U;
    p.G = G;
    p.xq = x.q;
    p.xd = x.d;
    p.xs = x.s;
    p.nbx = x.nbx;
    p.in_div = in_div;
    p.counts = counts;
    p.offsets = offsets;
    p.list = list;
    p.err = err;
    auto kern = &k_moe_gemv<TYPE>;
    static int configured_dev = -1;
    cudaError_t e = ensure_smem_attr(kern, (int)kSmemMax, configured_dev);
    if (e != cudaSuccess) return e;
    return launch_ex(kern, dim3((n + G - 1) / G, E, nmat), dim3(kThreads), smem, c, p);
}

cudaError_t launch_grouped_rt(uint32_t type, const ExpertMats* mats, int nmat, float* const* outs, int n, int d,
                              ActQ x, int in_div, const int* counts, const int* offsets, const int* list, int E,
                              int* err, const LaunchCfg& c)
{
    // Fewer columns than one block: every sum is empty; the caller zero-fills.
    if (row_bytes(type, d) == 0) return cudaErrorNotSupported;
    switch (type) {
    case T_Q8_0: return launch_grouped<T_Q8_0>(mats, nmat, outs, n, d, x, in_div, counts, offsets, list, E, err, c);
    case T_Q4_K: return launch_grouped<T_Q4_K>(mats, nmat, outs, n, d, x, in_div, counts, offsets, list, E, err, c);
    case T_Q5_K: return launch_grouped<T_Q5_K>(mats, nmat, outs, n, d, x, in_div, counts, offsets, list, E, err, c);
    case T_Q6_K: return launch_grouped<T_Q6_K>(mats, nmat, outs, n, d, x, in_div, counts, offsets, list, E, err, c);
    default: return cudaErrorInvalidValue;
    }
}

int grid_for(long long items, int per_cta)
{
    const long long cap = (long long)device_sm_count() * 8;
    return (int)std::max(1LL, std::min((items + per_cta - 1) / per_cta, cap));
}

} // namespace

size_t moe_workspace_bytes(int T, int E, int k, int dim, int hidden)
{
    return moe_layout(std::max(T, 1), std::max(E, 1), std::max(k, 1), std::max(dim, 1), std::max(hidden, 1)).total;
}

cudaError_t launch_moe_route(const MoeRoute& r, const LaunchCfg& c)
{
    if (r.T <= 0) return cudaSuccess;
    const MoeWs L = moe_layout(r.T, r.E, r.k, r.dim, 1);
    if (r.ws_bytes < L.probs + (size_t)r.T * r.E * 4) return cudaErrorInvalidValue;
    float* probs = reinterpret_cast<float*>(static_cast<uint8_t*>(r.ws) + L.probs);
    const float* lg = r.logits;
    long long ldl = r.ldl;
    cudaError_t e = cudaSuccess;
    if (r.router) {
        e = launch_gemv_f32(r.router, r.xb, r.ldx, probs, r.E, r.E, r.dim, r.T, c);
        lg = probs;
        ldl = r.E;
    }
    if (e == cudaSuccess)
        e = launch_ex(&k_moe_route, dim3((r.T + 127) / 128), dim3(128), 0, c, lg, ldl, probs, r.T, r.E, r.k, r.sel,
                      r.wts, r.err);
    return e;
}

cudaError_t launch_moe_experts(const MoeExperts& a, const LaunchCfg& c)
{
    if (a.T <= 0 || a.El <= 0) return cudaSuccess;
    const MoeWs L = moe_layout(a.T, a.El, a.k, a.dim, a.hidden);
    if (a.ws_bytes < L.total) return cudaErrorInvalidValue;
    uint8_t* ws = static_cast<uint8_t*>(a.ws);
    int* counts = reinterpret_cast<int*>(ws + L.counts);
    int* offsets = reinterpret_cast<int*>(ws + L.offsets);
    int* list = reinterpret_cast<int*>(ws + L.list);
    ActQ ax = actq_carve(ws + L.actx, a.dim, a.T);
    float* h1 = reinterpret_cast<float*>(ws + L.h1);
    float* h3 = reinterpret_cast<float*>(ws + L.h3);
    const int P = a.T * a.k;
    ActQ ah = actq_carve(ws + L.acth, a.hidden, P);

    cudaError_t e = launch_ex(&k_moe_group, dim3(1), dim3(1024), 0, c, a.sel, P, a.e0, a.El, counts, offsets, list);
    if (e == cudaSuccess) e = launch_quantize(a.xb, a.ldx, a.dim, a.T, ax, nullptr, nullptr, c);
    if (e != cudaSuccess) return e;

    auto grouped = [&](const ExpertMats* m, int nmat, float* const* outs, int n, int d, ActQ x, int in_div,
                       size_t zero_bytes) -> cudaError_t {
        cudaError_t r = launch_grouped_rt(m[0].type, m, nmat, outs, n, d, x, in_div, counts, offsets, list, a.El,
                                          a.err, c);
        if (r != cudaErrorNotSupported) return r;
        for (int z = 0; z < nmat; ++z) {
            r = cudaMemsetAsync(outs[z], 0, zero_bytes, c.stream);
            if (r != cudaSuccess) return r;
        }
        return cudaSuccess;
    };
    // W1 and W3 read the same activations: one launch when their types match.
    const size_t hbytes = (size_t)P * a.hidden * 4;
    if (a.w1.type == a.w3.type) {
        const ExpertMats m[2] = {a.w1, a.w3};
        float* const outs[2] = {h1, h3};
        e = grouped(m, 2, outs, a.hidden, a.dim, ax, a.k, hbytes);
    } else {
        float* const o1[1] = {h1};
        float* const o3[1] = {h3};
        e = grouped(&a.w1, 1, o1, a.hidden, a.dim, ax, a.k, hbytes);
        if (e == cudaSuccess) e = grouped(&a.w3, 1, o3, a.hidden, a.dim, ax, a.k, hbytes);
    }
    if (e == cudaSuccess && a.hidden / 32 > 0)
        e = launch_ex(&k_moe_act, dim3(grid_for((long long)P * (a.hidden / 32), kThreads / 32)), dim3(kThreads), 0,
                      c, (const float*)h1, (const float*)h3, a.hidden, P, a.sel, a.e0, a.El, ah.q, ah.d, ah.s);
    if (e == cudaSuccess) {
        if (row_bytes(a.w2.type, a.hidden) == 0) {
            // Empty W2 sums: zero only the local pairs' rows.
            e = launch_ex(&k_moe_zero_rows, dim3(grid_for((long long)P * a.dim, kThreads)), dim3(kThreads), 0, c,
                          a.o, a.dim, P, a.sel, a.e0, a.El);
        } else {
            float* const oo[1] = {a.o};
            e = grouped(&a.w2, 1, oo, a.dim, a.hidden, ah, 1, 0);
        }
    }
    return e;
}

cudaError_t launch_moe_combine(float* out, long long ldo, const float* o, const int* sel, const float* wts, int T,
                               int k, int dim, const LaunchCfg& c)
{
    if (T <= 0 || dim <= 0) return cudaSuccess;
    return launch_ex(&k_moe_combine, dim3(grid_for((long long)T * dim, kThreads)), dim3(kThreads), 0, c, o, dim, T,
                     k, sel, wts, out, ldo);
}

} // namespace qr
