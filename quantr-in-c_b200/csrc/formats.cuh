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

} // namespace qr
