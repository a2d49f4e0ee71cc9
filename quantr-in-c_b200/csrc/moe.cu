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
// From kMoeTcMinT tokens on, the experts stage runs on the tensor cores
// instead: each local pair's xb (and later hb) is quantized into its expert's
// operand tiles (16 pairs per chunk), and every (expert, matrix) is one
// gathered tcgen05 GEMV job over its pairs (tc.cu; counts and pair lists stay
// on the device).
// Every GEMV output is bit-identical to the reference's matmul_q_fused for
// that (row, pair), and expf (softmax, silu) is the host C library's own
// method evaluated step for step (libm_ref.cuh), so the whole block is
// bit-identical to the reference's scalar build.
#include "device_common.cuh"
#include "formats.cuh"
#include "kernels.cuh"
#include "launch_util.cuh"
#include "libm_ref.cuh"
#include "quant_decode.cuh"

#include <algorithm>
#include <cuda_runtime.h>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace qr {
namespace {

constexpr int kThreads = 256;
constexpr int kBT = 8;             // pairs per pass over a staged weight tile
constexpr uint32_t kChunk = 16384; // bytes per bulk copy
constexpr size_t kSmemMax = 227 * 1024;

// src/runtime.c:15-17: x / (1.0f + expf(-x)).
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, libm::expf_ref(-x))); }

// ------------------------------------------------------- route and group --

// Warp w routes token w, working on its row of `probs` (T x E in the
// workspace; logits may alias it): lane l takes experts l, l+32, ...  Every
// value is computed as the reference computes it; only the independent
// per-expert steps run in parallel, and the two left-to-right sums (softmax
// denominator, renormalisation) stay sequential in one lane.
__global__ void __launch_bounds__(128)
    k_moe_route(const float* logits, long long ldl, float* probs, int T, int E, int k, int* __restrict__ sel,
                float* __restrict__ wts, int* err)
{
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;  // warp-uniform
    float* p = probs + (long long)t * E;
    const float* lg = logits + (long long)t * ldl;
    // softmax_ref (src/kernels.c:191-207).  The running maximum with a strict
    // '>' from lg[0] is lg[0] when that is NaN, else the largest non-NaN value
    // (which of +0/-0 it keeps does not change lg[e] - m).
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e]);  // fmaxf skips NaN
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float l0 = lg[0];
    if (l0 != l0) m = l0;
    for (int e = lane; e < E; e += 32) p[e] = libm::expf_ref(__fsub_rn(lg[e], m));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0)
        for (int e = 0; e < E; ++e) sum = __fadd_rn(sum, p[e]);
    const float inv = __fdiv_rn(1.0f, __shfl_sync(0xffffffffu, sum, 0));
    for (int e = lane; e < E; e += 32) p[e] = __fmul_rn(p[e], inv);
    __syncwarp();
    // top-k (src/runtime.c:208-221): k passes of the first strict maximum
    // above -1e9 (the lowest index among equal values), then masked to -1e9.
    float w[kMoeMaxK];
    int s_[kMoeMaxK];
    bool bad = false;
    for (int s = 0; s < k; ++s) {
        float best = -1e9f;
        int arg = -1;
        for (int e = lane; e < E; e += 32) {
            const float v = p[e];
            if (v > best) {
                best = v;
                arg = e;
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
            if (oa >= 0 && (arg < 0 || ob > best || (ob == best && oa < arg))) {
                best = ob;
                arg = oa;
            }
        }
        if (arg < 0) {  // non-finite probabilities: the reference would index [-1]
            bad = true;
            break;
        }
        s_[s] = arg;
        w[s] = best;
        if (lane == (arg & 31)) p[arg] = -1e9f;
        __syncwarp();
    }
    if (lane != 0) return;
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
                int* __restrict__ offsets, int* __restrict__ list, int* __restrict__ pos)
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
            if (hit) {
                const int r = o + __popc(mk & ((1u << lane) - 1u));
                list[r] = q;
                pos[q] = r - off[e];  // the pair's place among its expert's pairs
            }
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

// Position of element e (0..31) of a unit in the tensor-core operand row for
// a weight type (the element order its decoder produces).
__device__ __forceinline__ int tc_elem_pos(uint32_t type, int e)
{
    if (type == T_Q4_K || type == T_Q5_K) return (e & ~7) + ((e & 1) << 2) + ((e & 7) >> 1);
    if (type == T_Q6_K) return (e & ~15) + ((e & 3) << 2) + ((e & 15) >> 2);
    return e;
}

// Tensor-core operand tiles of the pairs routed to each local expert: the
// pairs of local expert e, in list order (pos[p] = place of pair p), in chunks
// of 16 columns; chunk c of expert e holds U units of 16 x 32 quant bytes at
// tiles + ((e*nch + c)*U + u)*512 (column i%16 at (i/8)*256 + (i%8)*16 + (k/16)*128
// + k%16 for element order position k) and records (dx | bsum | 32*bsum, 16
// floats each) at recs + ((e*nch + c)*U + u)*256.
__device__ __forceinline__ void put_tile_block(uint8_t* tiles, uint8_t* recs, int e, int nch, int U, int u, int i,
                                               int kk, int lane, int8_t qq, uint32_t h, int sum)
{
    const long long unit = ((long long)e * nch + (i >> 4)) * U + u;
    const int c = i & 15;
    tiles[unit * 512 + (c >> 3) * 256 + (c & 7) * 16 + (kk >> 4) * 128 + (kk & 15)] = (uint8_t)qq;
    if (lane == 0) {
        float* rec = reinterpret_cast<float*>(recs + unit * 256);
        rec[c] = h2f_ref(h);
        rec[16 + c] = (float)sum;
        rec[32 + c] = __int_as_float(32 * sum);
    }
}

// xb of each local pair's token, quantized (quantize_row_q8_0, as every path)
// into W1's operand tiles and, when W3's element order or unit count differ,
// W3's.
__global__ void __launch_bounds__(kThreads)
    k_moe_x_tc(const float* __restrict__ xb, long long ldx, int P, int k, const int* __restrict__ sel,
               const int* __restrict__ pos, int e0, int El, int nch, int U1, uint32_t type1, uint8_t* tiles1,
               uint8_t* recs1, int U3, uint32_t type3, uint8_t* tiles3, uint8_t* recs3)
{
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int Um = max(U1, tiles3 ? U3 : 0);
    const long long total = (long long)P * Um;
    const long long step = (long long)gridDim.x * (kThreads / 32);
    const int k1 = tc_elem_pos(type1, lane), k3 = tc_elem_pos(type3, lane);
    for (long long wb = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); wb < total; wb += step) {
        const int pr = (int)(wb / Um);
        const int b = (int)(wb - (long long)pr * Um);
        const int se = sel[pr];
        if (se < e0 || se >= e0 + El) continue;  // not a local pair (warp-uniform)
        const float v = xb[(long long)(pr / k) * ldx + b * 32 + lane];
        uint32_t h;
        int sum;
        const int8_t qq = q8_block_warp(v, h, sum);
        if (b < U1) put_tile_block(tiles1, recs1, se - e0, nch, U1, b, pos[pr], k1, lane, qq, h, sum);
        if (tiles3 && b < U3) put_tile_block(tiles3, recs3, se - e0, nch, U3, b, pos[pr], k3, lane, qq, h, sum);
    }
}

// hb = silu(h1)*h3 per local pair (src/runtime.c:254-256), quantized (the
// same arithmetic as k_moe_act) into W2's operand tiles.
__global__ void __launch_bounds__(kThreads)
    k_moe_act_tc(const float* __restrict__ h1, const float* __restrict__ h3, int hidden, int P,
                 const int* __restrict__ sel, const int* __restrict__ pos, int e0, int El, int nch, int U2,
                 uint32_t type2, uint8_t* __restrict__ tiles, uint8_t* __restrict__ recs)
{
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long total = (long long)P * U2;
    const long long step = (long long)gridDim.x * (kThreads / 32);
    const int kk = tc_elem_pos(type2, lane);
    for (long long wb = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); wb < total; wb += step) {
        const int pr = (int)(wb / U2);
        const int b = (int)(wb - (long long)pr * U2);
        const int se = sel[pr];
        if (se < e0 || se >= e0 + El) continue;  // not a local pair (warp-uniform)
        const long long x = (long long)pr * hidden + b * 32 + lane;
        const float v = __fmul_rn(silu_ref(h1[x]), h3[x]);
        uint32_t h;
        int sum;
        const int8_t qq = q8_block_warp(v, h, sum);
        put_tile_block(tiles, recs, se - e0, nch, U2, b, pos[pr], kk, lane, qq, h, sum);
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
    size_t probs, counts, offsets, list, pos, actx, h1, h3, acth, t1, r1, t3, r3, t2, r2, total;
};

// Chunks of 16 pairs per local expert on the tensor-core path (an expert has
// at most T pairs: a token picks an expert once).  The path takes T <=
// kMoeTcMaxT: its operand tiles are laid out for that worst case per expert
// (the workspace grows with T; about 0.5 GB at T = 512 with 128 experts of
// the c5 shape).
constexpr int kMoeTcMaxT = 1024;
int moe_tc_chunks(int T) { return (T + 15) / 16; }

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
    w.pos = take(P * 4);
    w.actx = take(actq_bytes(dim, T));
    w.h1 = take(P * hidden * 4);
    w.h3 = take(P * hidden * 4);
    w.acth = take(actq_bytes(hidden, (int)P));
    // Operand tiles per local expert for the tensor-core path (W1, W3 when its
    // element order differs, W2): up to d/32 units x 16 columns x (32 quant +
    // 16 record bytes) per chunk.
    const size_t ch = T <= kMoeTcMaxT ? (size_t)E * moe_tc_chunks(T) : 0;
    w.t1 = take(ch * (dim / 32) * 512);
    w.r1 = take(ch * (dim / 32) * 256);
    w.t3 = take(ch * (dim / 32) * 512);
    w.r3 = take(ch * (dim / 32) * 256);
    w.t2 = take(ch * (hidden / 32) * 512);
    w.r2 = take(ch * (hidden / 32) * 256);
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
        e = launch_ex(&k_moe_route, dim3((r.T + 3) / 4), dim3(128), 0, c, lg, ldl, probs, r.T, r.E, r.k, r.sel,
                      r.wts, r.err);
    return e;
}

namespace {

// Tensor-core path of the experts stage: the W1/W3 GEMVs of every local
// expert as gathered jobs over all T tokens' quantized xb (each expert's live
// columns = the tokens of its pairs, outputs to the pairs' rows of h1/h3), and
// W2 as gathered jobs over per-expert operand tiles of hb (k_moe_act_tc).
struct MoeTcPlans {
    std::vector<TcPlan*> a, b;
};

// Fewest tokens for the tensor-core path.  Measured on B200 (us per layer,
// tensor cores / dp4a): c4 shapes T = 1: 83 / 57, T = 16: 212 / 212, T = 32:
// 250 / 302, T = 64: 261 / 433; c5 T = 8: 187 / 163, T = 16: 234 / 252,
// T = 64: 303 / 501.  With about one pair per expert the dp4a kernel, which
// stages each chosen expert's rows once with no pipeline to fill, is faster.
#ifndef QR_MOE_TC_MIN_T
#define QR_MOE_TC_MIN_T 16
#endif
constexpr int kMoeTcMinT = QR_MOE_TC_MIN_T;

bool tc_type(uint32_t t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K; }

// 32-element units of a row of d columns (whole blocks only, src/quant.c:477-484).
int units_of_type(uint32_t t, int d) { return (d / block_elems(t)) * block_units(t); }

// Device pointers of the local experts' matrices (a pointer table is read
// once, here).
bool expert_ptrs(const ExpertMats& m, int El, std::vector<const uint8_t*>& out)
{
    out.resize((size_t)El);
    if (m.table) {
        if (cudaMemcpy(out.data(), m.table, sizeof(void*) * (size_t)El, cudaMemcpyDeviceToHost) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
    } else {
        for (int e = 0; e < El; ++e) out[(size_t)e] = m.base + (long long)e * m.stride;
    }
    for (auto* q : out)
        if (!q || ((uintptr_t)q & 15)) return false;
    return true;
}

void destroy_plans(MoeTcPlans& P)
{
    for (auto* t : P.a) tc_plan_destroy(t);
    for (auto* t : P.b) tc_plan_destroy(t);
    P.a.clear();
    P.b.clear();
}

// Plans (cached per configuration and buffers) or nullptr when the tensor-core
// path does not take this configuration.
// W3 needs operand tiles of its own when its element order or its unit count
// differs from W1's.
bool w3_own_tiles(const MoeExperts& a)
{
    auto perm = [](uint32_t t) { return t == T_Q8_0 ? 0 : (t == T_Q6_K ? 2 : 1); };
    return perm(a.w1.type) != perm(a.w3.type) || units_of_type(a.w1.type, a.dim) != units_of_type(a.w3.type, a.dim);
}

const MoeTcPlans* moe_tc_plans(const MoeExperts& a, const MoeWs& L)
{
    if (a.T < kMoeTcMinT || a.T > kMoeTcMaxT || !tc_type(a.w1.type) || !tc_type(a.w3.type) || !tc_type(a.w2.type) ||
        row_bytes(a.w1.type, a.dim) <= 0 || row_bytes(a.w3.type, a.dim) <= 0 || row_bytes(a.w2.type, a.hidden) <= 0 ||
        ((uintptr_t)a.xb & 3))
        return nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    using MKey = std::tuple<const uint8_t*, long long, const uint8_t* const*, uint32_t>;
    auto mk = [](const ExpertMats& m) { return MKey{m.base, m.stride, m.table, m.type}; };
    using Key = std::tuple<int, int, int, int, int, int, int, MKey, MKey, MKey, const float*, long long, void*, float*>;
    const Key key{dev, a.T, a.k, a.e0, a.El, a.dim, a.hidden, mk(a.w1), mk(a.w3), mk(a.w2), a.xb, a.ldx, a.ws, a.o};
    static std::mutex mu;
    static std::map<Key, MoeTcPlans> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second.a.empty() ? nullptr : &it->second;
    MoeTcPlans P;
    std::vector<const uint8_t*> p1, p3, p2;
    uint8_t* ws = static_cast<uint8_t*>(a.ws);
    const int* counts = reinterpret_cast<const int*>(ws + L.counts);
    const int* offsets = reinterpret_cast<const int*>(ws + L.offsets);
    const int* list = reinterpret_cast<const int*>(ws + L.list);
    float* h1 = reinterpret_cast<float*>(ws + L.h1);
    float* h3 = reinterpret_cast<float*>(ws + L.h3);
    const int nch = moe_tc_chunks(a.T);
    const int U1 = units_of_type(a.w1.type, a.dim), U3 = units_of_type(a.w3.type, a.dim);
    const int U2 = units_of_type(a.w2.type, a.hidden);
    const bool own3 = w3_own_tiles(a);
    bool ok = expert_ptrs(a.w1, a.El, p1) && expert_ptrs(a.w3, a.El, p3) && expert_ptrs(a.w2, a.El, p2);
    std::vector<GemvJobIn> ja, jb;
    // One gathered job per (expert, matrix): 16 of the expert's pairs per pass.
    auto job = [&](const uint8_t* w, uint32_t type, int n, int d, size_t t_off, size_t r_off, int U, int e,
                   float* out) {
        GemvJobIn j{};
        j.w = w;
        j.type = type;
        j.n = n;
        j.d = d;
        j.B = 16;
        j.act = ws + t_off + (size_t)e * nch * U * 512;
        j.ds = ws + r_off + (size_t)e * nch * U * 256;
        j.out = out;
        j.ldo = n;
        j.g_counts = counts;
        j.g_offsets = offsets;
        j.g_list = list;
        j.g_e = e;
        return j;
    };
    for (int e = 0; ok && e < a.El; ++e) {
        ja.push_back(job(p1[(size_t)e], a.w1.type, a.hidden, a.dim, L.t1, L.r1, U1, e, h1));
        ja.push_back(own3 ? job(p3[(size_t)e], a.w3.type, a.hidden, a.dim, L.t3, L.r3, U3, e, h3)
                          : job(p3[(size_t)e], a.w3.type, a.hidden, a.dim, L.t1, L.r1, U1, e, h3));
        jb.push_back(job(p2[(size_t)e], a.w2.type, a.dim, a.hidden, L.t2, L.r2, U2, e, a.o));
    }
    auto plan = [&](std::vector<GemvJobIn>& jobs, std::vector<TcPlan*>& out) {
        for (size_t j0 = 0; ok && j0 < jobs.size(); j0 += kTcMaxJobs) {
            TcPlan* t = nullptr;
            if (tc_plan_create(jobs.data() + j0, (int)std::min<size_t>(kTcMaxJobs, jobs.size() - j0), &t) != 0) {
                ok = false;
                break;
            }
            out.push_back(t);
        }
    };
    plan(ja, P.a);
    plan(jb, P.b);
    if (!ok) destroy_plans(P);  // an empty entry: this configuration takes the dp4a path
    if (cache.size() >= 64) {
        for (auto& kv : cache) destroy_plans(kv.second);
        cache.clear();
    }
    auto& slot = cache[key];
    slot = P;
    return slot.a.empty() ? nullptr : &slot;
}

} // namespace

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

    int* pos = reinterpret_cast<int*>(ws + L.pos);

    cudaError_t e =
        launch_ex(&k_moe_group, dim3(1), dim3(1024), 0, c, a.sel, P, a.e0, a.El, counts, offsets, list, pos);
    if (e != cudaSuccess) return e;
    if (const MoeTcPlans* tp = moe_tc_plans(a, L)) {
        // Tensor cores: each pair's xb into its expert's W1 (and W3) operand
        // tiles, W1/W3 over each expert's pairs, hb into W2's tiles, W2.
        const int nch = moe_tc_chunks(a.T);
        const int U1 = units_of_type(a.w1.type, a.dim), U3 = units_of_type(a.w3.type, a.dim);
        const int U2 = units_of_type(a.w2.type, a.hidden);
        const bool own3 = w3_own_tiles(a);
        e = launch_ex(&k_moe_x_tc, dim3(grid_for((long long)P * std::max(U1, U3), kThreads / 32)), dim3(kThreads), 0,
                      c, a.xb, a.ldx, P, a.k, a.sel, (const int*)pos, a.e0, a.El, nch, U1, a.w1.type, ws + L.t1,
                      ws + L.r1, U3, a.w3.type, own3 ? ws + L.t3 : nullptr, own3 ? ws + L.r3 : nullptr);
        for (auto* t : tp->a)
            if (e == cudaSuccess) e = tc_plan_run(t, a.err, c.stream);
        if (e == cudaSuccess)
            e = launch_ex(&k_moe_act_tc, dim3(grid_for((long long)P * U2, kThreads / 32)), dim3(kThreads), 0, c,
                          (const float*)h1, (const float*)h3, a.hidden, P, a.sel, (const int*)pos, a.e0, a.El, nch, U2,
                          a.w2.type, ws + L.t2, ws + L.r2);
        for (auto* t : tp->b)
            if (e == cudaSuccess) e = tc_plan_run(t, a.err, c.stream);
        return e;
    }
    e = launch_quantize(a.xb, a.ldx, a.dim, a.T, ax, nullptr, nullptr, c);
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
