// engine_act.cuh -- the persistent engine's quantized-activation layout and
// the warp-level writer of one 32-element block into it (shared by the
// engine's own quantizer and the decoder kernels that quantize their outputs
// for the next GEMV program directly).
#pragma once
#include <cstdint>

#include "device_common.cuh"
#include "formats.cuh"
#include "kernels.cuh"

namespace qr {

// Position of element e (0..31) of a unit in the permuted activation layout
// (the element order each weight type's decode produces).
__device__ __forceinline__ int perm_pos(uint32_t type, int e)
{
    if (type == T_Q4_K || type == T_Q5_K) return (e & ~7) + ((e & 1) << 2) + ((e & 7) >> 1);
    if (type == T_Q6_K) return (e & ~15) + ((e & 3) << 2) + ((e & 15) >> 2);
    return e;
}

// Reference quantize_row_q8_0 (src/quant.c:143-158) of block b (32 elements)
// of token t, one warp: lane holds element `lane` (value v).  Writes the int8
// quants in the type's element order at unit u (K-quant activations go
// sub-block-major: block 8s+j of the row -> unit j*(U/8) + s, so consumer
// lanes on neighbouring super-blocks read neighbouring units; Q8_0 keeps
// block order) and the record (fp32 decode of the stored fp16 scale, fp32
// quant sum).  All 32 lanes must call it.
__device__ __forceinline__ void act_write_block(uint8_t* act, uint32_t ds_off, int U, int type, int t, int b,
                                                int lane, float v)
{
    const int u = type == T_Q8_0 ? b : (b & 7) * (U >> 3) + (b >> 3);
    const float a = fabsf(v);
    const uint32_t abits = (a == a) ? __float_as_uint(a) : 0u;  // the reference skips NaN
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, abits));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = (dd != 0.0f) ? __fdiv_rn(1.0f, dd) : 0.0f;
    const int8_t qq = lrintf_to_i8(__fmul_rn(v, id));
    const int sum = __reduce_add_sync(0xffffffffu, (int)qq);
    act[((long long)t * U + u) * 32 + perm_pos((uint32_t)type, lane)] = (uint8_t)qq;
    if (lane == 0)
        reinterpret_cast<uint2*>(act + ds_off)[t * U + u] =
            make_uint2(__float_as_uint(h2f_ref(f2h_ref(dd))), __float_as_uint((float)sum));
}

} // namespace qr
