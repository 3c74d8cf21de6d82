/*
 * Scalar stand-in for <arm_neon.h>, test infrastructure only.
 *
 * The reference engine (src/kernel_simd.c) includes <arm_neon.h> and so does
 * not build on an x86 host.  This header restates, in plain C with the lane
 * semantics of the Arm ACLE documentation, exactly the intrinsics that file
 * uses, so the unmodified reference compiles here and can serve as the
 * oracle's second witness.  Nothing in the product includes this file.
 *
 * Semantics that matter for bit-exactness:
 *   vfmaq_f32   fused multiply-add per lane (FMLA)          -> fmaf
 *   vmlaq_f32   multiply then add, two roundings (FMUL+FADD)
 *   vaddvq_f32  pairwise reduction (a0+a1)+(a2+a3)          (FADDP, FADDP)
 *   vcvtaq_s32  round to nearest, ties away from zero       (FCVTAS)
 *   vdotq_s32   per 32-bit lane, sum of four int8 products  (SDOT)
 * Build with -ffp-contract=off so the plain C products are not fused.
 *
 * The reference spin barrier issues `asm volatile("yield")`, an AArch64
 * hint; the assembler macro below maps it to the x86 `pause` hint.  The
 * macro must precede its use in the assembly output, hence the
 * -fno-toplevel-reorder build flag.
 */
#ifndef AION_ORACLE_ARM_NEON_SHIM_H
#define AION_ORACLE_ARM_NEON_SHIM_H

#include <math.h>
#include <stdint.h>

#if defined(__x86_64__) || defined(__i386__)
__asm__(".macro yield\n\tpause\n\t.endm\n");
#endif

#ifndef __ARM_FEATURE_DOTPROD
#define __ARM_FEATURE_DOTPROD 1
#endif

typedef struct { float v[4]; } float32x4_t;
typedef struct { int32_t v[4]; } int32x4_t;
typedef struct { int16_t v[8]; } int16x8_t;
typedef struct { int16_t v[4]; } int16x4_t;
typedef struct { int8_t v[16]; } int8x16_t;
typedef struct { int8_t v[8]; } int8x8_t;
typedef struct { uint8_t v[16]; } uint8x16_t;
typedef struct { uint8_t v[8]; } uint8x8_t;
typedef struct { int8x8_t val[2]; } int8x8x2_t;

#define SHIM static inline

/* ---- float32x4 ---------------------------------------------------------- */
SHIM float32x4_t vdupq_n_f32(float a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a; return r; }
SHIM float32x4_t vld1q_f32(const float* p) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = p[i]; return r; }
SHIM void vst1q_f32(float* p, float32x4_t a) { for (int i = 0; i < 4; i++) p[i] = a.v[i]; }
SHIM float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = fmaf(b.v[i], c.v[i], a.v[i]); return r;
}
SHIM float32x4_t vmlaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r;
    for (int i = 0; i < 4; i++) { float p = b.v[i] * c.v[i]; r.v[i] = a.v[i] + p; }
    return r;
}
SHIM float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i] * b.v[i]; return r; }
SHIM float32x4_t vmulq_n_f32(float32x4_t a, float b) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i] * b; return r; }
SHIM float32x4_t vabsq_f32(float32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = fabsf(a.v[i]); return r; }
SHIM float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r;
    for (int i = 0; i < 4; i++) r.v[i] = (isnan(a.v[i]) || isnan(b.v[i])) ? NAN : (a.v[i] > b.v[i] ? a.v[i] : b.v[i]);
    return r;
}
SHIM float vaddvq_f32(float32x4_t a) { float lo = a.v[0] + a.v[1]; float hi = a.v[2] + a.v[3]; return lo + hi; }
SHIM float vmaxvq_f32(float32x4_t a) {
    float lo = a.v[0] > a.v[1] ? a.v[0] : a.v[1];
    float hi = a.v[2] > a.v[3] ? a.v[2] : a.v[3];
    return lo > hi ? lo : hi;
}
SHIM float32x4_t vcvtq_f32_s32(int32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = (float)a.v[i]; return r; }
SHIM int32x4_t vcvtaq_s32_f32(float32x4_t a) {
    int32x4_t r;
    for (int i = 0; i < 4; i++) {
        float x = roundf(a.v[i]);               /* ties away from zero */
        if (isnan(x)) r.v[i] = 0;
        else if (x >= 2147483648.0f) r.v[i] = INT32_MAX;
        else if (x < -2147483648.0f) r.v[i] = INT32_MIN;
        else r.v[i] = (int32_t)x;
    }
    return r;
}

/* ---- int32x4 ------------------------------------------------------------ */
SHIM int32x4_t vdupq_n_s32(int32_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a; return r; }
SHIM int32_t vaddvq_s32(int32x4_t a) { return (int32_t)((uint32_t)a.v[0] + (uint32_t)a.v[1] + (uint32_t)a.v[2] + (uint32_t)a.v[3]); }
#define vgetq_lane_s32(a, lane) ((a).v[(lane)])
SHIM int32x4_t vdotq_s32(int32x4_t acc, int8x16_t a, int8x16_t b) {
    int32x4_t r;
    for (int i = 0; i < 4; i++) {
        int32_t s = 0;
        for (int j = 0; j < 4; j++) s += (int32_t)a.v[4 * i + j] * (int32_t)b.v[4 * i + j];
        r.v[i] = (int32_t)((uint32_t)acc.v[i] + (uint32_t)s);
    }
    return r;
}

/* ---- widening ----------------------------------------------------------- */
SHIM int16x4_t vget_low_s16(int16x8_t a) { int16x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i]; return r; }
SHIM int16x4_t vget_high_s16(int16x8_t a) { int16x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[4 + i]; return r; }
SHIM int32x4_t vmovl_s16(int16x4_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i]; return r; }
SHIM int8x8_t vget_low_s8(int8x16_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[i]; return r; }
SHIM int8x8_t vget_high_s8(int8x16_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[8 + i]; return r; }
SHIM int16x8_t vmovl_s8(int8x8_t a) { int16x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[i]; return r; }
SHIM int8x16_t vcombine_s8(int8x8_t lo, int8x8_t hi) {
    int8x16_t r; for (int i = 0; i < 8; i++) { r.v[i] = lo.v[i]; r.v[8 + i] = hi.v[i]; } return r;
}

/* ---- 8-bit lanes -------------------------------------------------------- */
SHIM uint8x16_t vld1q_u8(const uint8_t* p) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = p[i]; return r; }
SHIM uint8x8_t vld1_u8(const uint8_t* p) { uint8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = p[i]; return r; }
SHIM int8x16_t vld1q_s8(const int8_t* p) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = p[i]; return r; }
SHIM uint8x16_t vdupq_n_u8(uint8_t a) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a; return r; }
SHIM uint8x8_t vdup_n_u8(uint8_t a) { uint8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a; return r; }
SHIM int8x16_t vdupq_n_s8(int8_t a) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a; return r; }
SHIM int8x8_t vdup_n_s8(int8_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a; return r; }
SHIM uint8x16_t vandq_u8(uint8x16_t a, uint8x16_t b) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a.v[i] & b.v[i]; return r; }
SHIM uint8x8_t vand_u8(uint8x8_t a, uint8x8_t b) { uint8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = a.v[i] & b.v[i]; return r; }
#define vshrq_n_u8(a, n) aion_shim_vshrq_n_u8((a), (n))
#define vshr_n_u8(a, n) aion_shim_vshr_n_u8((a), (n))
SHIM uint8x16_t aion_shim_vshrq_n_u8(uint8x16_t a, int n) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (uint8_t)(a.v[i] >> n); return r; }
SHIM uint8x8_t aion_shim_vshr_n_u8(uint8x8_t a, int n) { uint8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = (uint8_t)(a.v[i] >> n); return r; }
SHIM int8x16_t vreinterpretq_s8_u8(uint8x16_t a) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (int8_t)a.v[i]; return r; }
SHIM int8x8_t vreinterpret_s8_u8(uint8x8_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = (int8_t)a.v[i]; return r; }
SHIM int8x16_t vsubq_s8(int8x16_t a, int8x16_t b) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (int8_t)(a.v[i] - b.v[i]); return r; }
SHIM int8x8_t vsub_s8(int8x8_t a, int8x8_t b) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = (int8_t)(a.v[i] - b.v[i]); return r; }
SHIM int8x16_t vzip1q_s8(int8x16_t a, int8x16_t b) {
    int8x16_t r; for (int i = 0; i < 8; i++) { r.v[2 * i] = a.v[i]; r.v[2 * i + 1] = b.v[i]; } return r;
}
SHIM int8x16_t vzip2q_s8(int8x16_t a, int8x16_t b) {
    int8x16_t r; for (int i = 0; i < 8; i++) { r.v[2 * i] = a.v[8 + i]; r.v[2 * i + 1] = b.v[8 + i]; } return r;
}
SHIM int8x8x2_t vzip_s8(int8x8_t a, int8x8_t b) {
    int8x8x2_t r;
    for (int i = 0; i < 4; i++) {
        r.val[0].v[2 * i] = a.v[i];     r.val[0].v[2 * i + 1] = b.v[i];
        r.val[1].v[2 * i] = a.v[4 + i]; r.val[1].v[2 * i + 1] = b.v[4 + i];
    }
    return r;
}

#undef SHIM
#endif
