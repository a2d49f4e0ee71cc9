/*
 * ref_shim.c -- exports the reference's header-inline fp16 helpers
 * (include/quant.h:53-77) and its KernelOps F32 matmul / softmax
 * (src/kernels.c:18-28, :191-207, selected through kernels_for_backend,
 * src/kernels.c:293-306) from the reference-built oracle library, so tests can
 * call the reference's own code.  Compiled only into oracle/_ref/, next to the
 * reference's src/quant.c and src/kernels.c.  TEST INFRASTRUCTURE ONLY.
 */
#include "kernels.h"
#include "quant.h"

float ref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }
uint16_t ref_fp32_to_fp16(float f) { return fp32_to_fp16(f); }

/* backend: 0 = BACKEND_REF (scalar matmul_ref), 1 = AVX2, 2 = AVX-512
 * (matmul_omp as compiled into this variant of the library). */
void ref_matmul_f32(float* out, const float* x, const float* w, int n, int d, int backend)
{
    kernels_for_backend((KernelBackend)backend)->matmul(out, x, w, n, d, 1);
}

void ref_softmax(float* x, int size) { kernels_for_backend(BACKEND_REF)->softmax(x, size); }
