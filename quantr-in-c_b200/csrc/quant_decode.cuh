// quant_decode.cuh -- per-type decode of packed weight blocks in shared memory
// into dp4a operands, and the reference's per-unit term.
//
// A "unit" is 32 consecutive elements: one Q8_0 block or one sub-block of a
// K-quant super-block; every unit pairs with one Q8_0 activation block.
//
// Activation bytes are stored in shared memory permuted to match each weight
// layout, so one dp4a pairs matching elements without shuffling weights:
//   Q8_0      natural order;
//   Q4_K/Q5_K per 8 elements [even 4 | odd 4] (the low nibble of qs byte k is
//             element 2k, the high nibble element 2k+1, src/quant.c:190);
//   Q6_K      per 16 elements a 4x4 byte transpose (lane k of operand m is
//             element 4k+m), matching the element-linear 2-bit qh fields
//             (src/quant.c:231).
#pragma once
#include <cstdint>

#include "device_common.cuh"
#include "formats.cuh"

namespace qr {

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

// Runtime-type variant (the program quantizer serves jobs of any type).
__device__ __forceinline__ uint4 permute_x16_rt(uint32_t type, uint4 v)
{
    if (type == T_Q4_K || type == T_Q5_K) return permute_x16<T_Q4_K>(v);
    if (type == T_Q6_K) return permute_x16<T_Q6_K>(v);
    return v;
}

// The reference's per-unit term, operation for operation (explicit rounding,
// no contraction):
//   Q8_0  ((float)isum * d_w) * d_x                  src/quant.c:284
//   Q6_K  (sc * (float)isum) * d_x                   src/quant.c:433
//   Q4_K/Q5_K ((sc*(float)isum) - (m*(float)bsum)) * d_x   src/quant.c:399
template <uint32_t TYPE>
__device__ __forceinline__ float unit_term(float a, float b, int isum, int bsum, float dx)
{
    if (TYPE == T_Q8_0) return __fmul_rn(__fmul_rn((float)isum, a), dx);
    if (TYPE == T_Q6_K) return __fmul_rn(__fmul_rn(a, (float)isum), dx);
    return __fmul_rn(__fsub_rn(__fmul_rn(a, (float)isum), __fmul_rn(b, (float)bsum)), dx);
}

// --------------------------------------------- generic (any alignment) ----

// Decoded unit: 8 dp4a operands plus the per-unit scale data.
struct Unit {
    uint32_t wq[8];
    float a, b;  // Q8_0: a = d_w | K4/K5: a = sc, b = m | Q6_K: a = sc
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
        o.a = __fmul_rn((float)(sc & 63u), h2f_ref(hdr & 0xFFFFu));  // src/quant.c:385
        o.b = __fmul_rn((float)(sc >> 6), h2f_ref(hdr >> 16));       // src/quant.c:386
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

__device__ __forceinline__ int dot8_from(const uint32_t* wq, uint4 xa, uint4 xb, int s)
{
    s = __dp4a((int)wq[0], (int)xa.x, s);
    s = __dp4a((int)wq[1], (int)xa.y, s);
    s = __dp4a((int)wq[2], (int)xa.z, s);
    s = __dp4a((int)wq[3], (int)xa.w, s);
    s = __dp4a((int)wq[4], (int)xb.x, s);
    s = __dp4a((int)wq[5], (int)xb.y, s);
    s = __dp4a((int)wq[6], (int)xb.z, s);
    s = __dp4a((int)wq[7], (int)xb.w, s);
    return s;
}

__device__ __forceinline__ int dot8(const uint32_t* wq, uint4 xa, uint4 xb) { return dot8_from(wq, xa, xb, 0); }

// One Q8_0 block per warp, lane = element: reference quantize_row_q8_0
// (src/quant.c:143-158) with IEEE division, the fp32 reciprocal of the
// unrounded scale, round-half-even and the truncating fp16 store.  Returns the
// lane's quant; h (fp16 bits of the scale) and sum (int sum of the block's
// quants) are valid in every lane.  NaN is skipped when taking the maximum,
// as the reference's `v > amax` test skips it.
__device__ __forceinline__ int8_t q8_block_warp(float v, uint32_t& h, int& sum)
{
    const float a = fabsf(v);
    const uint32_t abits = (a == a) ? __float_as_uint(a) : 0u;
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, abits));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = (dd != 0.0f) ? __fdiv_rn(1.0f, dd) : 0.0f;
    const int8_t qq = lrintf_to_i8(__fmul_rn(v, id));
    sum = __reduce_add_sync(0xffffffffu, (int)qq);
    h = f2h_ref(dd);
    return qq;
}

} // namespace qr
