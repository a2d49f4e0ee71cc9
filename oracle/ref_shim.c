/*
 * ref_shim.c -- exports the reference's header-inline fp16 helpers
 * (include/quant.h:53-77) from the reference-built oracle library, so tests can
 * call the reference's own conversions.  Compiled only into oracle/_ref/, next
 * to the reference's src/quant.c.  TEST INFRASTRUCTURE ONLY.
 */
#include "quant.h"

float ref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }
uint16_t ref_fp32_to_fp16(float f) { return fp32_to_fp16(f); }
