// libm_ref.cuh -- the host C library's expf, reproduced bit for bit on the GPU.
//
// The reference evaluates every exponential of its forward pass with the C
// library's expf: softmax (src/kernels.c:191-207) for attention and the MoE
// router, and silu (src/runtime.c:15-17) in every FFN.  That expf is not
// correctly rounded (on this platform about 1 in 13,000 arguments in
// (-110, 90) is off by one ulp), and a one-ulp difference in an activation is
// amplified by the next Q8_0 re-quantization into a different int8 code.  So
// the device evaluates the same method the host library uses, step for step:
//
//   exp(x) = 2^(k/32) * 2^(r/32),  z = x * 32/ln2,  k = nearest integer to z,
//   r = z - k in [-1/2, 1/2] (the product x * 32/ln2 fused into the
//   subtraction), 2^(k/32) = table[k mod 32] with k div 32 added to the
//   exponent field, and 2^(r/32) ~ 1 + c2 r + c1 r^2 + c0 r^3 evaluated in
//   double precision with fused multiply-adds, then rounded once to float.
//
// This is the published table-driven expf of Szabolcs Nagy (ARM
// optimized-routines, used by glibc since 2.28); the coefficients are that
// method's cubic for 2^(r/32) and the table holds RN(2^(i/32)) with i << 47
// subtracted from its bit pattern (so adding k << 47 scales it by 2^(k div 32)).
// Bit-exactness against this platform's glibc expf was measured over all 2^32
// float arguments (tests/test_libm_ref.py repeats that check on the host build
// of this header; the GPU tests compare the device build against glibc).
//
// The header compiles as CUDA (device and host) and as plain C++ (the host
// test), with every double operation explicitly rounded and never contracted.
#pragma once
#include <cstdint>
#include <cstring>
#include <cmath>

#ifdef __CUDACC__
#define QR_HD __host__ __device__ __forceinline__
#else
#define QR_HD inline
#endif

namespace qr {
namespace libm {

// RN(2^(i/32)) as IEEE-754 bits, minus i << 47.  The device copy lives in
// global (not __constant__) memory: lanes index it divergently, which the
// constant cache would serialise.
#define QR_EXP2_TAB_VALUES \
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull, \
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, \
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull, \
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull, \
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull, \
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull, \
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull, \
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
static const uint64_t kExp2TabHost[32] = {QR_EXP2_TAB_VALUES};
#ifdef __CUDACC__
__device__ static const uint64_t kExp2TabDev[32] = {QR_EXP2_TAB_VALUES};
#endif
#undef QR_EXP2_TAB_VALUES

// Cubic for 2^(r/32), r in [-1/2, 1/2]: coefficients of r^3, r^2, r (the
// method's 2^t polynomial, t = r/32, pre-scaled by 32^-3, 32^-2, 32^-1).
constexpr double kC0 = 0x1.c6af84b912394p-5 / 32768.0;
constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / 1024.0;
constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
constexpr double kInvLn2x32 = 0x1.71547652b82fep+0 * 32.0;
constexpr double kRoundShift = 0x1.8p+52;  // adding it rounds to an integer (ties to even)

QR_HD uint32_t f2u(float f)
{
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
#endif
}
QR_HD uint64_t d2u(double d)
{
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u;
    std::memcpy(&u, &d, 8);
    return u;
#endif
}
QR_HD double u2d(uint64_t u)
{
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)u);
#else
    double d;
    std::memcpy(&d, &u, 8);
    return d;
#endif
}
QR_HD double dmul(double a, double b)
{
#ifdef __CUDA_ARCH__
    return __dmul_rn(a, b);
#else
    volatile double r = a * b;  // never contracted into a neighbouring add
    return r;
#endif
}
QR_HD double dadd(double a, double b)
{
#ifdef __CUDA_ARCH__
    return __dadd_rn(a, b);
#else
    volatile double r = a + b;
    return r;
#endif
}
QR_HD double dfma(double a, double b, double c)
{
#ifdef __CUDA_ARCH__
    return __fma_rn(a, b, c);
#else
    return std::fma(a, b, c);
#endif
}
QR_HD float d2f(double d)
{
#ifdef __CUDA_ARCH__
    return __double2float_rn(d);
#else
    return (float)d;
#endif
}
QR_HD float fmul(float a, float b)
{
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    volatile float r = a * b;
    return r;
#endif
}

// expf exactly as the host C library computes it (all 2^32 arguments).
QR_HD float expf_ref(float x)
{
    const uint32_t ux = f2u(x);
    const uint32_t top = (ux >> 20) & 0x7ffu;  // |x| >= 88 (or not finite) iff top >= 0x42b
    if (top >= 0x42bu) {
        if (ux == 0xff800000u) return 0.0f;               // exp(-inf) = +0
        if (top >= 0x7f8u) return x + x;                  // +inf, NaN
        if (x > 0x1.62e42ep6f) return fmul(0x1p97f, 0x1p97f);     // overflows to +inf
        if (x < -0x1.9fe368p6f) return fmul(0x1p-95f, 0x1p-95f);  // underflows to +0
    }
    const double xd = (double)x;
    const double z = dmul(kInvLn2x32, xd);
    double kd = dadd(z, kRoundShift);
    const uint64_t ki = d2u(kd);
    kd = dadd(kd, -kRoundShift);
    const double r = dfma(kInvLn2x32, xd, -kd);
#ifdef __CUDA_ARCH__
    const uint64_t t = __ldg(&kExp2TabDev[ki & 31u]) + (ki << 47);
#else
    const uint64_t t = kExp2TabHost[ki & 31u] + (ki << 47);
#endif
    const double s = u2d(t);
    const double p = dfma(kC0, r, kC1);
    const double r2 = dmul(r, r);
    double y = dfma(kC2, r, 1.0);
    y = dfma(p, r2, y);
    y = dmul(y, s);
    return d2f(y);
}

#ifdef __CUDACC__
// silu of the reference's runtime (src/runtime.c:15-17): x / (1 + expf(-x)).
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf_ref(-x))); }
// The reference's SwiGLU input to the down projection: silu(h1) * h3
// (src/runtime.c:254-256, 277-279).
__device__ __forceinline__ float swiglu_ref(float h1, float h3) { return __fmul_rn(silu_ref(h1), h3); }
#endif

} // namespace libm
} // namespace qr
