// gemv.cu -- activation quantizer and fused quantized GEMV for sm_100a.
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
// Data movement.  A CTA owns G consecutive rows.  Their packed bytes are one
// contiguous range, staged into shared memory with cp.async.bulk (the 16-byte
// aligned body) plus plain loads for the <16-byte head and tail, so every
// block layout (34/144/176/210-byte blocks, any row alignment) streams from
// HBM with full coalescing.  The bulk copies are issued before
// griddepcontrol.wait, so under programmatic dependent launch the weight
// stream of this GEMV overlaps the tail of the kernel that produces x.
#include "formats.cuh"
#include "kernels.cuh"

#include <algorithm>
#include <atomic>
#include <utility>
#include <cuda_runtime.h>

namespace qr {

static std::atomic<unsigned long long> g_launches{0};

unsigned long long launch_count() { return g_launches.load(); }

namespace {

constexpr int kThreads = 256;
constexpr uint32_t kChunk = 16384;               // bytes per bulk copy
constexpr unsigned long long kWaitNs = 250000000ull;  // bounded waits: 250 ms

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t sptr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long gtimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sptr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sptr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sptr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the barrier phase; gives up after kWaitNs and records the timeout
// in *err (when given).  Never spins unboundedly.
__device__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > kWaitNs) {
            if (err) atomicExch(err, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            sptr(dst)),
        "l"(src), "r"(bytes), "r"(sptr(bar))
        : "memory");
}

// 32-bit word starting at an arbitrary shared-memory byte offset `off`.
__device__ __forceinline__ uint32_t ld_u32(const uint32_t* s32, uint32_t off)
{
    const uint32_t a = s32[off >> 2], b = s32[(off >> 2) + 1];
    return __funnelshift_r(a, b, (off & 3) * 8);
}

// N consecutive 32-bit words starting at an arbitrary byte offset.
template <int N>
__device__ __forceinline__ void ld_words(const uint32_t* s32, uint32_t off, uint32_t* out)
{
    uint32_t r[N + 1];
    const uint32_t base = off >> 2, sh = (off & 3) * 8;
#pragma unroll
    for (int k = 0; k <= N; ++k) r[k] = s32[base + k];
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = __funnelshift_r(r[k], r[k + 1], sh);
}

// --------------------------------------------------------------- quantizer --

// (int8_t)lrintf(v) as the x86-64 reference computes it: lrintf converts to a
// 64-bit long (cvtss2si), and a NaN or |v| >= 2^63 yields the "integer
// indefinite" 0x8000000000000000, whose low byte is 0.  CUDA's conversions
// saturate instead, so out-of-range values are mapped explicitly.  (Reached
// when a denormal block scale makes 1/d overflow to infinity.)
__device__ __forceinline__ int8_t lrintf_to_i8(float v)
{
    return fabsf(v) < 9.2233720368547758e18f ? (int8_t)__float2ll_rn(v) : (int8_t)0;
}

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
        const float a = fabsf(v);
        // The reference skips NaN when taking the max (v > amax is false).
        const uint32_t abits = (a == a) ? __float_as_uint(a) : 0u;
        const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, abits));
        const float dd = __fdiv_rn(amax, 127.0f);
        const float id = (dd != 0.0f) ? __fdiv_rn(1.0f, dd) : 0.0f;
        const int8_t qq = lrintf_to_i8(__fmul_rn(v, id));
        const int sum = __reduce_add_sync(0xffffffffu, (int)qq);
        if (act) q[wb * 32 + lane] = qq;
        if (lane == 0) {
            const uint32_t h = f2h_ref(dd);
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

// Activation words are stored in shared memory in the order the weight
// decoder produces its operands, so one dp4a pairs matching elements:
//   Q8_0      natural order;
//   Q4_K/Q5_K per 8 elements: [even 4 | odd 4] (nibble-interleaved weights);
//   Q6_K      per 16 elements: 4x4 byte transpose (lane k of operand m is
//             element 4k+m, matching the 2-bit qh fields of one byte).
template <uint32_t TYPE>
__device__ __forceinline__ uint4 permute_x16(uint4 v)
{
    if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        return make_uint4(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.x, v.y, 0x7531),
                          __byte_perm(v.z, v.w, 0x6420), __byte_perm(v.z, v.w, 0x7531));
    } else if (TYPE == T_Q6_K) {
        const uint32_t p01l = __byte_perm(v.x, v.y, 0x5140), p01h = __byte_perm(v.x, v.y, 0x7362);
        const uint32_t p23l = __byte_perm(v.z, v.w, 0x5140), p23h = __byte_perm(v.z, v.w, 0x7362);
        return make_uint4(__byte_perm(p01l, p23l, 0x5410), __byte_perm(p01l, p23l, 0x7632),
                          __byte_perm(p01h, p23h, 0x5410), __byte_perm(p01h, p23h, 0x7632));
    }
    return v;
}

// Spreads bits 0,2,4,6 of a byte to bit 4 of byte lanes 0..3.  Collisions of
// the multiply only carry into bits 11, 17 and 23, which the mask drops.
__device__ __forceinline__ uint32_t spread_even_bits_to_b4(uint32_t hb)
{
    return ((hb & 0x55u) * 0x410410u) & 0x10101010u;
}

// Decoded unit: 8 dp4a operands plus the per-unit scale data.
struct Unit {
    uint32_t wq[8];
    float a, b;   // Q8_0: a = d_w | K4/K5: a = sc, b = m | Q6_K: a = sc
};

template <uint32_t TYPE>
__device__ __forceinline__ void decode_unit(const uint32_t* s32, const uint8_t* s8, uint32_t row_off, int u,
                                            Unit& o)
{
    if (TYPE == T_Q8_0) {
        const uint32_t blk = row_off + 34u * u;
        o.a = h2f_ref(ld_u32(s32, blk) & 0xFFFFu);
        ld_words<8>(s32, blk + 2, o.wq);
    } else if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        const int j = u & 7;
        const uint32_t sb = row_off + (uint32_t)block_bytes(TYPE) * (uint32_t)(u >> 3);
        const uint32_t hdr = ld_u32(s32, sb);
        const uint32_t sc = s8[sb + 4 + j];
        // src/quant.c:385-386: sc = (scales[j]&63)*d, m = (scales[j]>>6)*dmin.
        o.a = __fmul_rn((float)(sc & 63u), h2f_ref(hdr & 0xFFFFu));
        o.b = __fmul_rn((float)(sc >> 6), h2f_ref(hdr >> 16));
        uint32_t qw[4];
        ld_words<4>(s32, sb + (TYPE == T_Q4_K ? 16u : 48u) + 16u * j, qw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o.wq[2 * i] = qw[i] & 0x0F0F0F0Fu;
            o.wq[2 * i + 1] = (qw[i] >> 4) & 0x0F0F0F0Fu;
        }
        if (TYPE == T_Q5_K) {
            const uint32_t H = ld_u32(s32, sb + 16u + 4u * j);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t hb = (H >> (8 * i)) & 0xFFu;
                o.wq[2 * i] |= spread_even_bits_to_b4(hb);
                o.wq[2 * i + 1] |= spread_even_bits_to_b4(hb >> 1);
            }
        }
    } else {  // Q6_K
        const int j = u & 7;
        const uint32_t sb = row_off + 210u * (uint32_t)(u >> 3);
        const float d = h2f_ref(ld_u32(s32, sb + 208) & 0xFFFFu);
        o.a = __fmul_rn((float)(int8_t)s8[sb + 192 + j], d);  // src/quant.c:423
        uint32_t ql[4], qh[2];
        ld_words<4>(s32, sb + 16u * j, ql);
        ld_words<2>(s32, sb + 128u + 8u * j, qh);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t s0 = __byte_perm(ql[2 * h], ql[2 * h + 1], 0x6420);
            const uint32_t s1 = __byte_perm(ql[2 * h], ql[2 * h + 1], 0x7531);
            const uint32_t nib[4] = {s0 & 0x0F0F0F0Fu, (s0 >> 4) & 0x0F0F0F0Fu, s1 & 0x0F0F0F0Fu,
                                     (s1 >> 4) & 0x0F0F0F0Fu};
#pragma unroll
            for (int m = 0; m < 4; ++m) o.wq[4 * h + m] = nib[m] | (((qh[h] >> (2 * m)) & 0x03030303u) << 4);
        }
    }
}

// The reference's per-unit term, operation for operation.
template <uint32_t TYPE>
__device__ __forceinline__ float unit_term(const Unit& o, int isum, int bsum, float dx)
{
    if (TYPE == T_Q8_0)  // src/quant.c:284: (float)isum * d_w * d_x
        return __fmul_rn(__fmul_rn((float)isum, o.a), dx);
    if (TYPE == T_Q6_K)  // src/quant.c:433: sc * (float)isum * bd
        return __fmul_rn(__fmul_rn(o.a, (float)isum), dx);
    // src/quant.c:399: (sc*(float)isum - m*(float)bsum) * bd
    return __fmul_rn(__fsub_rn(__fmul_rn(o.a, (float)isum), __fmul_rn(o.b, (float)bsum)), dx);
}

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
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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
                const uint4 xa = xv[0], xb = xv[1];
                int isum = 0;
                isum = __dp4a((int)o.wq[0], (int)xa.x, isum);
                isum = __dp4a((int)o.wq[1], (int)xa.y, isum);
                isum = __dp4a((int)o.wq[2], (int)xa.z, isum);
                isum = __dp4a((int)o.wq[3], (int)xa.w, isum);
                isum = __dp4a((int)o.wq[4], (int)xb.x, isum);
                isum = __dp4a((int)o.wq[5], (int)xb.y, isum);
                isum = __dp4a((int)o.wq[6], (int)xb.z, isum);
                isum = __dp4a((int)o.wq[7], (int)xb.w, isum);
                const int bsum = xs[t * U + u];
                if (TYPE == T_Q6_K) isum -= 32 * bsum;  // quants stored with +32 offset
                terms[u * TS + g * BT + t] = unit_term<TYPE>(o, isum, bsum, xd[t * U + u]);
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

// F32 weights: 128 rows per CTA, 32-column tiles through shared memory, one
// thread per row summing sequentially (reference src/quant.c:455-461).
__global__ void __launch_bounds__(128)
    k_gemv_f32(const float* __restrict__ w, const float* __restrict__ x, long long ldx, float* __restrict__ out,
               long long ldo, int n, int d, int B)
{
    __shared__ float tile[128][33];
    __shared__ float xt[32];
    pdl_trigger();
    pdl_wait();
    const int r0 = blockIdx.x * 128;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    for (int t = 0; t < B; ++t) {
        float acc = 0.0f;
        for (int c0 = 0; c0 < d; c0 += 32) {
            const int cw = min(32, d - c0);
            __syncthreads();
            for (int rr = warp; rr < 128; rr += 4) {
                const int r = r0 + rr;
                tile[rr][lane] = (r < n && lane < cw) ? w[(long long)r * d + c0 + lane] : 0.0f;
            }
            if (tid < 32) xt[tid] = tid < cw ? x[(long long)t * ldx + c0 + tid] : 0.0f;
            __syncthreads();
            for (int c = 0; c < cw; ++c) acc = __fadd_rn(acc, __fmul_rn(tile[tid][c], xt[c]));
        }
        if (r0 + tid < n) out[(long long)t * ldo + r0 + tid] = acc;
    }
}

// Reference dequantize_row (src/quant.c:160-240), one thread per element.
__global__ void k_dequantize(float* __restrict__ out, const uint8_t* __restrict__ src, uint32_t type, int n)
{
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    auto rd16 = [&](long long off) { return (uint32_t)src[off] | ((uint32_t)src[off + 1] << 8); };
    if (type == T_Q8_0) {
        if (e >= (n / 32) * 32) return;
        const long long blk = 34LL * (e / 32);
        out[e] = __fmul_rn((float)(int8_t)src[blk + 2 + (e & 31)], h2f_ref(rd16(blk)));
    } else if (type == T_Q4_K || type == T_Q5_K || type == T_Q6_K) {
        if (e >= (n / 256) * 256) return;
        const int l = e & 255, j = l >> 5;
        const long long sb = (long long)block_bytes(type) * (e >> 8);
        if (type == T_Q6_K) {
            const int lo = (src[sb + l / 2] >> ((l & 1) * 4)) & 0xF;
            const int hi = (src[sb + 128 + l / 4] >> ((l % 4) * 2)) & 3;
            const float sc = __fmul_rn((float)(int8_t)src[sb + 192 + j], h2f_ref(rd16(sb + 208)));
            out[e] = __fmul_rn((float)((lo | (hi << 4)) - 32), sc);
        } else {
            const uint32_t sc8 = src[sb + 4 + j];
            const float sc = __fmul_rn((float)(sc8 & 63u), h2f_ref(rd16(sb)));
            const float m = __fmul_rn((float)(sc8 >> 6), h2f_ref(rd16(sb + 2)));
            const long long qs = sb + (type == T_Q4_K ? 16 : 48);
            int q = (src[qs + l / 2] >> ((l & 1) * 4)) & 0xF;
            if (type == T_Q5_K) q |= ((src[sb + 16 + l / 8] >> (l % 8)) & 1) << 4;
            out[e] = __fsub_rn(__fmul_rn((float)q, sc), m);
        }
    }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, const LaunchCfg& c,
                      Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = c.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
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
    static int configured_dev = -1;  // one attribute call per device is enough
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax);
        if (e != cudaSuccess) return e;
        configured_dev = dev;
    }
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
    return launch_ex(&k_gemv_f32, dim3((n + 127) / 128), dim3(128), 0, c, w, x, ldx, out, ldo, n, d, B);
}

cudaError_t launch_dequantize(float* out, const uint8_t* src, uint32_t type, int n, const LaunchCfg& c)
{
    if (n <= 0) return cudaSuccess;
    return launch_ex(&k_dequantize, dim3((n + 255) / 256), dim3(256), 0, c, out, src, type, n);
}

} // namespace qr
