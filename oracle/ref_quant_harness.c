/*
 * Exposes the reference quantizer's quantize_buffer() (quantize.c:59-109)
 * as a shared-library symbol -- TEST INFRASTRUCTURE ONLY.  Built by
 * oracle/Makefile from the reference's quantize.c, included unmodified with
 * its main() renamed; the reference source is never copied here.
 */
#define main aion_reference_quantize_main
#include "quantize.c"
#undef main

__attribute__((visibility("default")))
void ref_quantize_buffer(const float* in, uint8_t* packed, float* scales, int n) {
    quantize_buffer(in, packed, scales, n);
}
