// formats.cuh -- packed block layouts and the reference's bit-level fp16
// conversions, device side.
//
// Layouts (all little-endian, packed; reference include/quant.h:28-50,
// src/quant.c:216-236):
//   Q8_0  34 B : u16 d | i8 qs[32]
//   Q4_K 144 B : u16 d | u16 dmin | u8 scales[12] | u8 qs[128]
//   Q5_K 176 B : u16 d | u16 dmin | u8 scales[12] | u8 qh[32] | u8 qs[128]
//   Q6_K 210 B : u8 ql[128] | u8 qh[64] | i8 scales[16] | u16 d
// Only scales[0..7] are read for every K type (one per 32-element sub-block).
#pragma once
#include <cstdint>

namespace qr {

enum : uint32_t { T_F32 = 0, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

// Bytes of one block and elements covered by it.
__host__ __device__ constexpr int block_bytes(uint32_t t)
{
    return t == T_Q8_0 ? 34 : t == T_Q4_K ? 144 : t == T_Q5_K ? 176 : t == T_Q6_K ? 210 : 4;
}
__host__ __device__ constexpr int block_elems(uint32_t t) { return t == T_Q8_0 ? 32 : t == T_F32 ? 1 : 256; }
// 32-element units (the granularity of one activation scale) per block.
__host__ __device__ constexpr int block_units(uint32_t t) { return t == T_Q8_0 ? 1 : 8; }

__host__ __device__ inline bool type_supported(uint32_t t)
{
    return t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

// Bytes of one packed row of d columns: floor(d/32) Q8_0 blocks or floor(d/256)
// super-blocks; trailing columns are ignored (reference src/quant.c:477-484).
__host__ __device__ inline long long row_bytes(uint32_t t, int d)
{
    if (t == T_F32) return 4LL * d;
    return (long long)(d / block_elems(t)) * block_bytes(t);
}

// fp16 -> fp32 with the reference's recipe (include/quant.h:53-66): exponent
// rebias by adding 0x38000000, infinities/NaNs widened, subnormal halves NOT
// renormalised.  Must stay a pure bit recipe so device and host agree.
__host__ __device__ __forceinline__ float h2f_ref(uint32_t h)
{
    uint32_t mag = (h & 0x7FFFu) << 13;
    uint32_t e = (h >> 10) & 0x1Fu;
    mag = (e == 0x1Fu) ? (mag | 0x7F800000u) : (e != 0 ? mag + 0x38000000u : mag);
    uint32_t bits = mag | ((h & 0x8000u) << 16);
#ifdef __CUDA_ARCH__
    return __uint_as_float(bits);
#else
    float f;
    __builtin_memcpy(&f, &bits, 4);
    return f;
#endif
}

// fp32 -> fp16 with the reference's recipe (include/quant.h:68-77): mantissa
// truncated, flush to signed zero below the smallest normal half, saturate to
// signed infinity.
__host__ __device__ __forceinline__ uint32_t f2h_ref(float f)
{
#ifdef __CUDA_ARCH__
    uint32_t x = __float_as_uint(f);
#else
    uint32_t x;
    __builtin_memcpy(&x, &f, 4);
#endif
    uint32_t s = (x >> 16) & 0x8000u;
    int e = (int)((x >> 23) & 0xFFu) - 112;
    if (e <= 0) return s;
    if (e >= 31) return s | 0x7C00u;
    return s | ((uint32_t)e << 10) | ((x >> 13) & 0x3FFu);
}

// Elements of an n-element row that dequantize_row defines (whole blocks).
__host__ __device__ inline int dequant_extent_host(uint32_t type, int n)
{
    return type == T_Q8_0 ? (n / 32) * 32 : (type == T_Q4_K || type == T_Q5_K || type == T_Q6_K) ? (n / 256) * 256 : 0;
}

#ifdef __CUDACC__
// Element e of a packed row, decoded as the reference's dequantize_row does
// (src/quant.c:160-240): Q8_0 q*d; K types q*sc - m (Q4_K/Q5_K) or
// (q-32)*(scale*d) (Q6_K), every product explicitly rounded.  Only elements
// below dequant_extent(type, n) are defined (whole blocks; the reference
// leaves a ragged tail untouched).
__device__ __forceinline__ int dequant_extent(uint32_t type, int n)
{
    return type == T_Q8_0 ? (n / 32) * 32 : (type == T_Q4_K || type == T_Q5_K || type == T_Q6_K) ? (n / 256) * 256 : 0;
}
__device__ __forceinline__ float dequant_elem(const uint8_t* __restrict__ src, uint32_t type, int e)
{
    auto rd16 = [&](long long off) { return (uint32_t)src[off] | ((uint32_t)src[off + 1] << 8); };
    if (type == T_Q8_0) {
        const long long blk = 34LL * (e / 32);
        return __fmul_rn((float)(int8_t)src[blk + 2 + (e & 31)], h2f_ref(rd16(blk)));
    }
    const int l = e & 255, j = l >> 5;
    const long long sb = (long long)block_bytes(type) * (e >> 8);
    if (type == T_Q6_K) {
        const int lo = (src[sb + l / 2] >> ((l & 1) * 4)) & 0xF;
        const int hi = (src[sb + 128 + l / 4] >> ((l % 4) * 2)) & 3;
        const float sc = __fmul_rn((float)(int8_t)src[sb + 192 + j], h2f_ref(rd16(sb + 208)));
        return __fmul_rn((float)((lo | (hi << 4)) - 32), sc);
    }
    const uint32_t sc8 = src[sb + 4 + j];
    const float sc = __fmul_rn((float)(sc8 & 63u), h2f_ref(rd16(sb)));
    const float m = __fmul_rn((float)(sc8 >> 6), h2f_ref(rd16(sb + 2)));
    const long long qs = sb + (type == T_Q4_K ? 16 : 48);
    int q = (src[qs + l / 2] >> ((l & 1) * 4)) & 0xF;
    if (type == T_Q5_K) q |= ((src[sb + 16 + l / 8] >> (l % 8)) & 1) << 4;
    return __fsub_rn(__fmul_rn((float)q, sc), m);
}
#endif

} // namespace qr
