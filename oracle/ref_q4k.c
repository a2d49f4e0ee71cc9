/*
 * ref_q4k.c -- the restated Q4_K dot product, interposed at link time over
 * the reference's vec_dot_q4K_q8_0 (src/quant.c:291-369, which reads the fp16
 * fields d, dmin and the activation scale as raw integers).  oracle/Makefile
 * weakens the reference's definition in its quant.o, so its matmul_q_fused
 * (whose call goes through the PLT) binds to this one.  The arithmetic is
 * quant_oracle.c's restatement: the decode of src/quant.c:180-195 combined
 * per sub-block as (sc*isum - m*bsum)*bd, the Q5_K kernel's expression
 * (src/quant.c:399).  TEST INFRASTRUCTURE ONLY.
 */
#include "quant.h"
#include "quant_oracle.h"

float vec_dot_q4K_q8_0(const block_q4_K* a, const block_q8_0* b, int k)
{
    return qo_vec_dot_q4K_q8_0(a, (const qo_block_q8_0*)b, k);
}
