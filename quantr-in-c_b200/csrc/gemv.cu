// gemv.cu -- activation quantizer and the per-call fused quantized GEMV.
//
// Parity design.  The reference (src/quant.c:242-437, scalar build) computes
// every output row as a left-to-right fp32 sum over 32-element units of a term
// that is itself a fixed sequence of rounded fp32 operations on the unit's
// int32 dot product.  These kernels reproduce that exactly:
//   * int32 unit sums come from dp4a (order-free, so bit-exact);
//   * each term is evaluated with explicitly rounded __fmul_rn/__fsub_rn in the
//     reference's operand order (no FMA contraction);
//   * the per-row sum adds the terms in unit order with __fadd_rn.
// The result is bit-identical to the reference's scalar build; the parity
// tests assert that, which is stronger than the 1e-5 rel / 1e-6 abs bar.
//
// k_gemv is the general kernel (any weight alignment, any shape that fits one
// row group in shared memory).  A CTA owns G consecutive rows.  Their packed
// bytes are one contiguous range, staged into shared memory with
// cp.async.bulk (the 16-byte aligned body) plus plain loads for the <16-byte
// head and tail.  The bulk copies are issued before griddepcontrol.wait, so
// under programmatic dependent launch the weight stream overlaps the tail of
// the kernel that produces x.  The persistent engine (engine.cu) is the fast
// path for 16-byte aligned weights.
#include "device_common.cuh"
#include "formats.cuh"
#include "kernels.cuh"
#include "launch_util.cuh"
#include "quant_decode.cuh"

#include <algorithm>
#include <cuda_runtime.h>

namespace qr {

std::atomic<unsigned long long> g_launches{0};

unsigned long long launch_count() { return g_launches.load(); }

namespace {

constexpr int kThreads = 256;
constexpr uint32_t kChunk = 16384;  // bytes per bulk copy

// --------------------------------------------------------------- quantizer --

// One warp per 32-element block: reference quantize_row_q8_0
// (src/quant.c:143-158) with IEEE division, the fp32 reciprocal of the
// unrounded scale, round-half-even and the truncating fp16 store.
template <bool EMIT_BLOCKS>
__global__ void __launch_bounds__(kThreads)
    k_quantize(const float* __restrict__ x, long long ldx, int nbx, int B, int8_t* __restrict__ q,
               float* __restrict__ dq, int32_t* __restrict__ sq, uint8_t* __restrict__ blocks, int* err_reset)
{
    pdl_trigger();
    pdl_wait();
    if (err_reset && blockIdx.x == 0 && threadIdx.x == 0) *err_reset = DEV_OK;
    const bool act = q != nullptr;
    const int lane = threadIdx.x & 31;
    const long long total = (long long)B * nbx;
    const long long step = (long long)gridDim.x * (kThreads / 32);
    for (long long wb = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); wb < total; wb += step) {
        const int t = (int)(wb / nbx);
        const int b = (int)(wb - (long long)t * nbx);
        const float v = x[(long long)t * ldx + (long long)b * 32 + lane];
        uint32_t h;
        int sum;
        const int8_t qq = q8_block_warp(v, h, sum);
        if (act) q[wb * 32 + lane] = qq;
        if (lane == 0) {
            if (act) {
                dq[wb] = h2f_ref(h);
                sq[wb] = sum;
            }
            if (EMIT_BLOCKS) {
                blocks[wb * 34] = (uint8_t)(h & 0xFF);
                blocks[wb * 34 + 1] = (uint8_t)(h >> 8);
            }
        }
        if (EMIT_BLOCKS) blocks[wb * 34 + 2 + lane] = (uint8_t)qq;
    }
}

// Packed block_q8_0 (34 B) -> ActQ, one warp per block.
__global__ void __launch_bounds__(kThreads)
    k_repack(const uint8_t* __restrict__ blocks, long long total, int8_t* __restrict__ q,
             float* __restrict__ dq, int32_t* __restrict__ sq)
{
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long step = (long long)gridDim.x * (kThreads / 32);
    for (long long wb = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); wb < total; wb += step) {
        const int8_t qq = (int8_t)blocks[wb * 34 + 2 + lane];
        const int sum = __reduce_add_sync(0xffffffffu, (int)qq);
        q[wb * 32 + lane] = qq;
        if (lane == 0) {
            const uint32_t h = (uint32_t)blocks[wb * 34] | ((uint32_t)blocks[wb * 34 + 1] << 8);
            dq[wb] = h2f_ref(h);
            sq[wb] = sum;
        }
    }
}

// ----------------------------------------------------------------- GEMV --

struct KParams {
    const uint8_t* w;
    long long rb;  // row bytes
    int n, U, G, TS;
    const int8_t* xq;
    const float* xd;
    const int32_t* xs;
    int nbx;
    float* out;
    long long ldo;
    int B;
    int32_t* dbg_isum;
    int32_t* dbg_bsum;
    int* err;
    uint32_t w_off, x_off, xd_off, xs_off, t_off;  // shared-memory carve-up
};

template <uint32_t TYPE, int BT, bool DBG>
__global__ void __launch_bounds__(kThreads) k_gemv(KParams p)
{
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sm);
    const int tid = threadIdx.x;
    const int r0 = blockIdx.x * p.G;
    const int gcnt = min(p.G, p.n - r0);
    const uint8_t* src = p.w + (long long)r0 * p.rb;
    const long long nbytes = (long long)gcnt * p.rb;

    // Stage this CTA's rows: wb[i] == src[i].  The 16-byte aligned body goes
    // through the bulk-copy engine, the ragged head and tail through threads.
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
        for (long long off = 0; off < body; off += kChunk) {
            const uint32_t sz = (uint32_t)min((long long)kChunk, body - off);
            bulk_g2s(wb + head + off, src + head + off, sz, bar);
        }
    }
    for (long long i = tid; i < head; i += kThreads) wb[i] = src[i];
    for (long long i = tail0 + tid; i < nbytes; i += kThreads) wb[i] = src[i];

    pdl_trigger();
    // Everything below reads x or writes out: wait for the producer grid.
    pdl_wait();

    const int U = p.U;
    int8_t* xq = reinterpret_cast<int8_t*>(sm + p.x_off);
    float* xd = reinterpret_cast<float*>(sm + p.xd_off);
    int32_t* xs = reinterpret_cast<int32_t*>(sm + p.xs_off);
    for (int i = tid; i < p.B * U * 2; i += kThreads) {
        const int t = i / (2 * U);
        const int r = i - t * 2 * U;
        const uint4 v = *reinterpret_cast<const uint4*>(p.xq + ((long long)t * p.nbx + (r >> 1)) * 32 + (r & 1) * 16);
        *reinterpret_cast<uint4*>(xq + (t * U + (r >> 1)) * 32 + (r & 1) * 16) = permute_x16<TYPE>(v);
    }
    for (int i = tid; i < p.B * U; i += kThreads) {
        const int t = i / U, u = i - t * U;
        xd[i] = p.xd[(long long)t * p.nbx + u];
        xs[i] = p.xs[(long long)t * p.nbx + u];
    }

    const bool ok = mbar_wait_bounded(bar, 0, p.err);
    if (!__syncthreads_and(ok)) {
        // Give the copies in flight a second bounded chance to land before the
        // CTA exits; the host sees the error word either way.
        mbar_wait_bounded(bar, 0, nullptr);
        return;
    }

    float* terms = reinterpret_cast<float*>(sm + p.t_off);
    const int TS = p.TS;
    for (int it = tid; it < gcnt * U; it += kThreads) {
        const int g = it / U, u = it - g * U;
        Unit o;
        decode_unit<TYPE>(s32, sm, wb_off + (uint32_t)(g * p.rb), u, o);
#pragma unroll
        for (int t = 0; t < BT; ++t) {
            if (t < p.B) {
                const uint4* xv = reinterpret_cast<const uint4*>(xq + (t * U + u) * 32);
                int isum = dot8(o.wq, xv[0], xv[1]);
                const int bsum = xs[t * U + u];
                if (TYPE == T_Q6_K) isum -= 32 * bsum;  // quants stored with +32 offset
                terms[u * TS + g * BT + t] = unit_term<TYPE>(o.a, o.b, isum, bsum, xd[t * U + u]);
                if (DBG) {
                    const long long k = ((long long)t * p.n + r0 + g) * U + u;
                    p.dbg_isum[k] = isum;
                    p.dbg_bsum[k] = bsum;
                }
            }
        }
    }
    __syncthreads();
    // Left-to-right sum over units per (row, token): the reference's order.
    for (int i = tid; i < gcnt * p.B; i += kThreads) {
        const int g = i / p.B, t = i - g * p.B;
        const float* tp = terms + g * BT + t;
        float s = 0.0f;
        for (int u = 0; u < U; ++u) s = __fadd_rn(s, tp[u * TS]);
        p.out[(long long)t * p.ldo + r0 + g] = s;
    }
}

// F32 weights (reference src/quant.c:455-461, which is KernelOps matmul_ref,
// src/kernels.c:18-28): one thread per (row, token) summing row[j]*x[j] left
// to right.  A CTA covers RT rows x TT tokens; KT-column tiles of the weights
// and of x stream through a 3-stage shared-memory ring (16-byte cp.async when
// rows are 16-byte aligned, plain loads otherwise), so two tiles are in
// flight while one is summed.  Tile rows have a stride of KT + 4 floats, so
// the 128-bit reads of 8 consecutive rows hit distinct banks.
constexpr int kF32Stages = 3;

template <int RT, int TT, int KT>
constexpr size_t f32_smem() { return (size_t)kF32Stages * (RT + TT) * (KT + 4) * sizeof(float); }

template <int RT, int TT, int KT>
__global__ void __launch_bounds__(RT * TT)
    k_gemv_f32(const float* __restrict__ w, const float* __restrict__ x, long long ldx, float* __restrict__ out,
               long long ldo, int n, int d, int B)
{
    constexpr int NT = RT * TT, KS = KT + 4, S = kF32Stages, WS = RT * KS, XS = TT * KS;
    extern __shared__ __align__(16) float fsm[];
    pdl_trigger();
    const int r0 = blockIdx.x * RT, t0 = blockIdx.y * TT, tid = threadIdx.x;
    const int rr = tid % RT, tt = tid / RT;
    const int ntile = (d + KT - 1) / KT;
    const bool wal = ((uintptr_t)w & 15) == 0 && (d & 3) == 0;
    const bool xal = ((uintptr_t)x & 15) == 0 && (ldx & 3) == 0;
    // Tile c of `rows` rows starting at g0 of src (row stride ld) -> dst.
    auto load = [&](float* dst, const float* src, long long ld, int g0, int rows, int lim, bool al, int c) {
        const int c0 = c * KT;
        for (int q = tid; q < rows * (KT / 4); q += NT) {
            const int r = q / (KT / 4), k = 4 * (q - r * (KT / 4));
            const int g = g0 + r, col = c0 + k;
            if (g >= lim || col >= d) continue;
            float* sd = dst + r * KS + k;
            const float* gs = src + (long long)g * ld + col;
            if (al) {
                cp16(sptr(sd), gs);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (col + e < d) sd[e] = gs[e];
            }
        }
    };
    auto stage = [&](int c) { return fsm + (c % S) * (WS + XS); };
#pragma unroll
    for (int c = 0; c < S - 1; ++c)
        if (c < ntile) load(stage(c), w, d, r0, RT, n, wal, c);  // weights never depend on the previous kernel
    pdl_wait();
#pragma unroll
    for (int c = 0; c < S - 1; ++c) {
        if (c < ntile) load(stage(c) + WS, x, ldx, t0, TT, B, xal, c);
        cp_commit();
    }
    float acc = 0.0f;
    for (int c = 0; c < ntile; ++c) {
        __syncthreads();  // the stage refilled next was read in the previous iteration
        const int cn = c + S - 1;
        if (cn < ntile) {
            load(stage(cn), w, d, r0, RT, n, wal, cn);
            load(stage(cn) + WS, x, ldx, t0, TT, B, xal, cn);
        }
        cp_commit();
        cp_wait<S - 1>();
        __syncthreads();
        const float* wt = stage(c) + rr * KS;
        const float* xt = stage(c) + WS + tt * KS;
        const int cw = min(KT, d - c * KT);
        int j = 0;
        for (; j + 4 <= cw; j += 4) {
            const float4 a = *reinterpret_cast<const float4*>(wt + j);
            const float4 b = *reinterpret_cast<const float4*>(xt + j);
            acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
            acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
            acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
            acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
        }
        for (; j < cw; ++j) acc = __fadd_rn(acc, __fmul_rn(wt[j], xt[j]));
    }
    cp_wait<0>();
    if (r0 + rr < n && t0 + tt < B) out[(long long)(t0 + tt) * ldo + r0 + rr] = acc;
}

// Reference dequantize_row (src/quant.c:160-240), one thread per element.
__global__ void k_dequantize(float* __restrict__ out, const uint8_t* __restrict__ src, uint32_t type, int n)
{
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e < dequant_extent(type, n)) out[e] = dequant_elem(src, type, e);
}

// dequantize_row of `rows` rows: out[r*ldo + e] from src + r*src_stride.
__global__ void k_dequantize_rows(float* __restrict__ out, long long ldo, const uint8_t* __restrict__ src,
                                  long long src_stride, uint32_t type, int n, int rows)
{
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.y;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows && e < dequant_extent(type, n)) out[(long long)r * ldo + e] = dequant_elem(src + r * src_stride, type, e);
}

int grid_for_warps(long long warps)
{
    const long long per = kThreads / 32;
    long long blocks = (warps + per - 1) / per;
    const long long cap = (long long)device_sm_count() * 8;
    return (int)std::max(1LL, std::min(blocks, cap));
}

constexpr size_t kSmemMax = 227 * 1024;

template <uint32_t TYPE, int BT, bool DBG>
cudaError_t gemv_typed(const GemvArgs& g, const LaunchCfg& c, int B0, int nb)
{
    const long long rb = row_bytes(TYPE, g.d);
    const int U = (g.d / block_elems(TYPE)) * block_units(TYPE);
    const int sms = device_sm_count();
    auto smem_for = [&](int G, int& TS, KParams& kp) {
        TS = G * BT;
        if ((TS & 1) == 0) TS += 1;
        size_t off = 128;  // mbarrier + padding
        kp.w_off = (uint32_t)off;
        off += ((size_t)G * rb + 32 + 15) & ~size_t(15);
        kp.x_off = (uint32_t)off;
        off += (size_t)BT * U * 32;
        kp.xd_off = (uint32_t)off;
        off += (size_t)BT * U * 4;
        kp.xs_off = (uint32_t)off;
        off += (size_t)BT * U * 4;
        kp.t_off = (uint32_t)off;
        off += (size_t)U * TS * 4;
        return off;
    };
    KParams kp{};
    // Rows per CTA: about two CTAs per SM over the matrix, at most 48 KB of
    // weights and whatever fits the shared-memory budget.
    int G = (int)std::max(1LL, std::min<long long>((g.n + 2LL * sms - 1) / (2LL * sms), std::max(1LL, 49152 / rb)));
    int TS = 0;
    size_t smem = smem_for(G, TS, kp);
    while (G > 1 && smem > kSmemMax) smem = smem_for(--G, TS, kp);
    if (smem > kSmemMax) return cudaErrorInvalidConfiguration;
    kp.w = g.w;
    kp.rb = rb;
    kp.n = g.n;
    kp.U = U;
    kp.G = G;
    kp.TS = TS;
    kp.xq = g.x.q + (long long)B0 * g.x.nbx * 32;
    kp.xd = g.x.d + (long long)B0 * g.x.nbx;
    kp.xs = g.x.s + (long long)B0 * g.x.nbx;
    kp.nbx = g.x.nbx;
    kp.out = g.out + (long long)B0 * g.ldo;
    kp.ldo = g.ldo;
    kp.B = nb;
    kp.dbg_isum = g.dbg_isum ? g.dbg_isum + (long long)B0 * g.n * U : nullptr;
    kp.dbg_bsum = g.dbg_bsum ? g.dbg_bsum + (long long)B0 * g.n * U : nullptr;
    kp.err = g.err;
    auto kern = &k_gemv<TYPE, BT, DBG>;
    static int configured_dev = -1;
    cudaError_t e = ensure_smem_attr(kern, (int)kSmemMax, configured_dev);
    if (e != cudaSuccess) return e;
    const int grid = (g.n + G - 1) / G;
    return launch_ex(kern, dim3(grid), dim3(kThreads), smem, c, kp);
}

template <uint32_t TYPE, bool DBG>
cudaError_t gemv_dispatch_bt(const GemvArgs& g, const LaunchCfg& c)
{
    for (int b0 = 0; b0 < g.B; b0 += 16) {
        const int nb = std::min(16, g.B - b0);
        cudaError_t e;
        if (nb == 1) e = gemv_typed<TYPE, 1, DBG>(g, c, b0, nb);
        else if (nb == 2) e = gemv_typed<TYPE, 2, DBG>(g, c, b0, nb);
        else if (nb <= 4) e = gemv_typed<TYPE, 4, DBG>(g, c, b0, nb);
        else if (nb <= 8) e = gemv_typed<TYPE, 8, DBG>(g, c, b0, nb);
        else e = gemv_typed<TYPE, 16, DBG>(g, c, b0, nb);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <bool DBG>
cudaError_t gemv_dispatch(const GemvArgs& g, const LaunchCfg& c)
{
    switch (g.type) {
    case T_Q8_0: return gemv_dispatch_bt<T_Q8_0, DBG>(g, c);
    case T_Q4_K: return gemv_dispatch_bt<T_Q4_K, DBG>(g, c);
    case T_Q5_K: return gemv_dispatch_bt<T_Q5_K, DBG>(g, c);
    case T_Q6_K: return gemv_dispatch_bt<T_Q6_K, DBG>(g, c);
    default: return cudaErrorInvalidValue;
    }
}

} // namespace

int device_sm_count()
{
    static int cached_dev = -1, cached = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != cached_dev) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cached = v > 0 ? v : 1;
        cached_dev = dev;
    }
    return cached;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

size_t actq_bytes(int d, int B)
{
    const size_t nbx = (size_t)std::max(d / 32, 1);
    return align256((size_t)B * nbx * 32) + 2 * align256((size_t)B * nbx * 4);
}

ActQ actq_carve(void* ws, int d, int B)
{
    const size_t nbx = (size_t)std::max(d / 32, 1);
    uint8_t* p = static_cast<uint8_t*>(ws);
    ActQ a;
    a.nbx = (int)nbx;
    a.q = reinterpret_cast<int8_t*>(p);
    p += align256((size_t)B * nbx * 32);
    a.d = reinterpret_cast<float*>(p);
    p += align256((size_t)B * nbx * 4);
    a.s = reinterpret_cast<int32_t*>(p);
    return a;
}

cudaError_t launch_quantize(const float* x, long long ldx, int d, int B, ActQ a, uint8_t* blocks,
                            int* err_reset, const LaunchCfg& c)
{
    const int nbx = d / 32;
    if (nbx <= 0 || B <= 0) {
        if (err_reset) return cudaMemsetAsync(err_reset, 0, sizeof(int), c.stream);
        return cudaSuccess;
    }
    const int grid = grid_for_warps((long long)B * nbx);
    if (blocks)
        return launch_ex(&k_quantize<true>, dim3(grid), dim3(kThreads), 0, c, x, ldx, nbx, B, a.q, a.d, a.s,
                         blocks, err_reset);
    return launch_ex(&k_quantize<false>, dim3(grid), dim3(kThreads), 0, c, x, ldx, nbx, B, a.q, a.d, a.s,
                     (uint8_t*)nullptr, err_reset);
}

cudaError_t launch_repack(const uint8_t* blocks, int nbx, int B, ActQ a, const LaunchCfg& c)
{
    const long long total = (long long)nbx * B;
    if (total <= 0) return cudaSuccess;
    return launch_ex(&k_repack, dim3(grid_for_warps(total)), dim3(kThreads), 0, c, blocks, total, a.q, a.d, a.s);
}

cudaError_t launch_gemv(const GemvArgs& g, const LaunchCfg& c)
{
    if (g.n <= 0 || g.B <= 0) return cudaSuccess;
    if (!type_supported(g.type)) return cudaErrorInvalidValue;
    if (row_bytes(g.type, g.d) == 0)  // fewer columns than one block: the reference sums nothing
        return cudaMemset2DAsync(g.out, (size_t)g.ldo * 4, 0, (size_t)g.n * 4, (size_t)g.B, c.stream);
    if (g.dbg_isum || g.dbg_bsum) return gemv_dispatch<true>(g, c);
    return gemv_dispatch<false>(g, c);
}

cudaError_t launch_gemv_f32(const float* w, const float* x, long long ldx, float* out, long long ldo, int n,
                            int d, int B, const LaunchCfg& c)
{
    if (n <= 0 || B <= 0) return cudaSuccess;
    static int dev1 = -1, dev4 = -1;
    if (B == 1) {
        constexpr size_t sm = f32_smem<128, 1, 64>();
        cudaError_t e = ensure_smem_attr(&k_gemv_f32<128, 1, 64>, (int)sm, dev1);
        if (e != cudaSuccess) return e;
        return launch_ex(&k_gemv_f32<128, 1, 64>, dim3((n + 127) / 128), dim3(128), sm, c, w, x, ldx, out, ldo, n, d,
                         B);
    }
    constexpr size_t sm = f32_smem<32, 4, 128>();
    cudaError_t e = ensure_smem_attr(&k_gemv_f32<32, 4, 128>, (int)sm, dev4);
    if (e != cudaSuccess) return e;
    return launch_ex(&k_gemv_f32<32, 4, 128>, dim3((n + 31) / 32, (B + 3) / 4), dim3(128), sm, c, w, x, ldx, out, ldo,
                     n, d, B);
}

cudaError_t launch_dequantize_rows(float* out, long long ldo, const uint8_t* src, long long src_stride, uint32_t type,
                                   int n, int rows, const LaunchCfg& c)
{
    if (n <= 0 || rows <= 0) return cudaSuccess;
    return launch_ex(&k_dequantize_rows, dim3((n + 255) / 256, rows), dim3(256), 0, c, out, ldo, src, src_stride,
                     type, n, rows);
}

cudaError_t launch_dequantize(float* out, const uint8_t* src, uint32_t type, int n, const LaunchCfg& c)
{
    if (n <= 0) return cudaSuccess;
    return launch_ex(&k_dequantize, dim3((n + 255) / 256), dim3(256), 0, c, out, src, type, n);
}

} // namespace qr
