/* A scalar x86-64 stand-in for <arm_neon.h> (TEST INFRASTRUCTURE ONLY), so that the reference's own C sources compile
 * and run on this host unmodified as the parity oracle's reference build (oracle/ref.mk -> oracle/_ref/).
 *
 * Only tests/ and bench.py's reference arm load what this builds; the product library never does.
 *
 * Each intrinsic is written from its definition in the Arm Architecture Reference Manual (AArch64 Advanced SIMD), for
 * the subset the reference uses, with the Linux user-space FPCR defaults (round to nearest even, FZ = 0, DN = 0,
 * AH = 0):
 *   - fp32 lanes: IEEE single operations (x86-64 SSE arithmetic is the same IEEE operation); FMLA / FMLS as fmaf
 *     (one rounding); FMIN / FMAX NaN-propagating with -0 < +0; FADDP reductions pairwise.
 *   - FRECPE / FRECPS: the Arm ARM pseudocode (FPRecipEstimate, FPRecipStepFused), single and half precision.
 *   - conversions: FCVTZS / FCVTNS / FCVTAS saturating, NaN -> 0; SCVTF round to nearest even.
 *   - integer lanes wrap modulo 2^n (computed in unsigned arithmetic); SQXTN saturates; XTN truncates.
 *   - fp16 lanes: every operation rounded once to IEEE half (sums and products are exact in double; the fused
 *     multiply-add is rounded to odd in double first, which makes the final rounding to half correct).
 * Vectors are GCC vector types, as in GCC's own arm_neon.h, so that the reference's vector expressions and lane
 * indexing keep their meaning. NaN payloads are not modelled. */
#ifndef BNN_ORACLE_NEON_STANDIN_H
#define BNN_ORACLE_NEON_STANDIN_H
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../arm_emu.h"

typedef _Float16 float16_t;
typedef float float32_t;
typedef double float64_t;

#define NV_VEC(name, elem, bytes) typedef elem name __attribute__((vector_size(bytes), may_alias))
NV_VEC(int8x8_t, int8_t, 8);
NV_VEC(int8x16_t, int8_t, 16);
NV_VEC(uint8x8_t, uint8_t, 8);
NV_VEC(uint8x16_t, uint8_t, 16);
NV_VEC(int16x4_t, int16_t, 8);
NV_VEC(int16x8_t, int16_t, 16);
NV_VEC(uint16x4_t, uint16_t, 8);
NV_VEC(uint16x8_t, uint16_t, 16);
NV_VEC(int32x2_t, int32_t, 8);
NV_VEC(int32x4_t, int32_t, 16);
NV_VEC(uint32x2_t, uint32_t, 8);
NV_VEC(uint32x4_t, uint32_t, 16);
NV_VEC(int64x2_t, int64_t, 16);
NV_VEC(uint64x2_t, uint64_t, 16);
NV_VEC(float16x4_t, _Float16, 8);
NV_VEC(float16x8_t, _Float16, 16);
NV_VEC(float32x2_t, float, 8);
NV_VEC(float32x4_t, float, 16);
NV_VEC(float64x2_t, double, 16);
#undef NV_VEC
typedef struct { float32x4_t val[2]; } float32x4x2_t;
typedef struct { uint8x16_t val[2]; } uint8x16x2_t;
typedef struct { int8x16_t val[2]; } int8x16x2_t;
typedef struct { float16x8_t val[2]; } float16x8x2_t;

#define NV static inline __attribute__((always_inline, unused))
#define NV_LANES(v) ((int)(sizeof(v) / sizeof((v)[0])))

/* ------------------------------------------------------------------ reinterpretation (same 64 or 128 bits) */
#define NV_RI(dt, st, DT) \
  NV DT vreinterpretq_##dt##_##st(__typeof__(((DT *)0)[0]) *unused_);
#define vreinterpretq_f32_s32(x) ((float32x4_t)(x))
#define vreinterpretq_f32_u32(x) ((float32x4_t)(x))
#define vreinterpretq_f32_f64(x) ((float32x4_t)(x))
#define vreinterpretq_f32_s8(x) ((float32x4_t)(x))
#define vreinterpretq_f32_u8(x) ((float32x4_t)(x))
#define vreinterpretq_f32_s16(x) ((float32x4_t)(x))
#define vreinterpretq_f32_f16(x) ((float32x4_t)(x))
#define vreinterpretq_s32_f32(x) ((int32x4_t)(x))
#define vreinterpretq_s32_u32(x) ((int32x4_t)(x))
#define vreinterpretq_s32_s8(x) ((int32x4_t)(x))
#define vreinterpretq_s32_u8(x) ((int32x4_t)(x))
#define vreinterpretq_s32_s16(x) ((int32x4_t)(x))
#define vreinterpretq_s32_f64(x) ((int32x4_t)(x))
#define vreinterpretq_u32_f32(x) ((uint32x4_t)(x))
#define vreinterpretq_u32_s32(x) ((uint32x4_t)(x))
#define vreinterpretq_u32_u8(x) ((uint32x4_t)(x))
#define vreinterpretq_f64_f32(x) ((float64x2_t)(x))
#define vreinterpretq_f64_s32(x) ((float64x2_t)(x))
#define vreinterpretq_s8_u8(x) ((int8x16_t)(x))
#define vreinterpretq_s8_s32(x) ((int8x16_t)(x))
#define vreinterpretq_s8_s16(x) ((int8x16_t)(x))
#define vreinterpretq_s8_f32(x) ((int8x16_t)(x))
#define vreinterpretq_u8_s8(x) ((uint8x16_t)(x))
#define vreinterpretq_u8_s16(x) ((uint8x16_t)(x))
#define vreinterpretq_u8_u16(x) ((uint8x16_t)(x))
#define vreinterpretq_u8_s32(x) ((uint8x16_t)(x))
#define vreinterpretq_u8_u32(x) ((uint8x16_t)(x))
#define vreinterpretq_u8_f16(x) ((uint8x16_t)(x))
#define vreinterpretq_u8_f32(x) ((uint8x16_t)(x))
#define vreinterpretq_s16_f16(x) ((int16x8_t)(x))
#define vreinterpretq_s16_u16(x) ((int16x8_t)(x))
#define vreinterpretq_s16_u8(x) ((int16x8_t)(x))
#define vreinterpretq_s16_s8(x) ((int16x8_t)(x))
#define vreinterpretq_s16_s32(x) ((int16x8_t)(x))
#define vreinterpretq_u16_s16(x) ((uint16x8_t)(x))
#define vreinterpretq_u16_u8(x) ((uint16x8_t)(x))
#define vreinterpretq_u16_f16(x) ((uint16x8_t)(x))
#define vreinterpretq_f16_s16(x) ((float16x8_t)(x))
#define vreinterpretq_f16_u16(x) ((float16x8_t)(x))
#define vreinterpretq_f16_u8(x) ((float16x8_t)(x))
#define vreinterpretq_f16_f32(x) ((float16x8_t)(x))
#define vreinterpret_f32_s32(x) ((float32x2_t)(x))
#define vreinterpret_s32_f32(x) ((int32x2_t)(x))
#define vreinterpret_s8_u8(x) ((int8x8_t)(x))
#define vreinterpret_u8_s8(x) ((uint8x8_t)(x))
#define vreinterpret_s16_f16(x) ((int16x4_t)(x))
#define vreinterpret_f16_s16(x) ((float16x4_t)(x))
#undef NV_RI

/* ------------------------------------------------------------------ loads, stores, lanes, halves */
#define NV_LDST(sfx, T, E)                                                              \
  NV T vld1##sfx(const E *p) { T v; memcpy(&v, p, sizeof v); return v; }                 \
  NV void vst1##sfx(E *p, T v) { memcpy(p, &v, sizeof v); }                               \
  NV T vdup##sfx##_unused_(void) { T v = {0}; return v; }
NV_LDST(q_f32, float32x4_t, float)
NV_LDST(_f32, float32x2_t, float)
NV_LDST(q_f64, float64x2_t, double)
NV_LDST(q_s8, int8x16_t, int8_t)
NV_LDST(_s8, int8x8_t, int8_t)
NV_LDST(q_u8, uint8x16_t, uint8_t)
NV_LDST(_u8, uint8x8_t, uint8_t)
NV_LDST(q_s16, int16x8_t, int16_t)
NV_LDST(_s16, int16x4_t, int16_t)
NV_LDST(q_u16, uint16x8_t, uint16_t)
NV_LDST(q_s32, int32x4_t, int32_t)
NV_LDST(_s32, int32x2_t, int32_t)
NV_LDST(q_u32, uint32x4_t, uint32_t)
NV_LDST(q_f16, float16x8_t, _Float16)
NV_LDST(_f16, float16x4_t, _Float16)
#undef NV_LDST

#define NV_DUP(name, T, E)                                                 \
  NV T name(E x) { T v; for (int i = 0; i < NV_LANES(v); i++) v[i] = x; return v; }
NV_DUP(vdupq_n_f32, float32x4_t, float)
NV_DUP(vdup_n_f32, float32x2_t, float)
NV_DUP(vdupq_n_f64, float64x2_t, double)
NV_DUP(vdupq_n_s8, int8x16_t, int8_t)
NV_DUP(vdup_n_s8, int8x8_t, int8_t)
NV_DUP(vdupq_n_u8, uint8x16_t, uint8_t)
NV_DUP(vdupq_n_s16, int16x8_t, int16_t)
NV_DUP(vdupq_n_u16, uint16x8_t, uint16_t)
NV_DUP(vdupq_n_s32, int32x4_t, int32_t)
NV_DUP(vdup_n_s32, int32x2_t, int32_t)
NV_DUP(vdupq_n_u32, uint32x4_t, uint32_t)
NV_DUP(vdupq_n_f16, float16x8_t, _Float16)
NV_DUP(vdup_n_f16, float16x4_t, _Float16)
#undef NV_DUP
#define vmovq_n_f32 vdupq_n_f32
#define vmovq_n_s32 vdupq_n_s32

NV float32x4x2_t vld2q_f32(const float *p) {
  float32x4x2_t r;
  for (int i = 0; i < 4; i++) { r.val[0][i] = p[2 * i]; r.val[1][i] = p[2 * i + 1]; }
  return r;
}
NV void vst2q_f32(float *p, float32x4x2_t v) {
  for (int i = 0; i < 4; i++) { p[2 * i] = v.val[0][i]; p[2 * i + 1] = v.val[1][i]; }
}
NV uint8x16x2_t vld1q_u8_x2(const uint8_t *p) { uint8x16x2_t r; memcpy(&r, p, 32); return r; }

#define vgetq_lane_f32(v, i) ((float)(v)[(i)])
#define vget_lane_f32(v, i) ((float)(v)[(i)])
#define vgetq_lane_s32(v, i) ((int32_t)(v)[(i)])
#define vgetq_lane_u32(v, i) ((uint32_t)(v)[(i)])
#define vgetq_lane_f16(v, i) ((_Float16)(v)[(i)])
NV float32x4_t vsetq_lane_f32(float x, float32x4_t v, int i) { v[i] = x; return v; }
NV int32x4_t vsetq_lane_s32(int32_t x, int32x4_t v, int i) { v[i] = x; return v; }
NV float32x4_t vdupq_laneq_f32(float32x4_t v, int i) { return vdupq_n_f32(v[i]); }
NV float32x4_t vdupq_lane_f32(float32x2_t v, int i) { return vdupq_n_f32(v[i]); }

#define NV_HALVES(sfx, T, H)                                                                \
  NV H vget_low_##sfx(T v) { H h; memcpy(&h, &v, sizeof h); return h; }                     \
  NV H vget_high_##sfx(T v) { H h; memcpy(&h, (const char *)&v + sizeof h, sizeof h); return h; } \
  NV T vcombine_##sfx(H lo, H hi) { T v; memcpy(&v, &lo, sizeof lo); memcpy((char *)&v + sizeof lo, &hi, sizeof hi); return v; }
NV_HALVES(f32, float32x4_t, float32x2_t)
NV_HALVES(s8, int8x16_t, int8x8_t)
NV_HALVES(u8, uint8x16_t, uint8x8_t)
NV_HALVES(s16, int16x8_t, int16x4_t)
NV_HALVES(u16, uint16x8_t, uint16x4_t)
NV_HALVES(s32, int32x4_t, int32x2_t)
NV_HALVES(f16, float16x8_t, float16x4_t)
#undef NV_HALVES

/* ------------------------------------------------------------------ fp32 arithmetic */
#define NV_MAP2(name, T, expr)                                                           \
  NV T name(T a, T b) { T r; for (int i = 0; i < NV_LANES(r); i++) r[i] = (expr); return r; }
#define NV_MAP1(name, T, expr)                                                           \
  NV T name(T a) { T r; for (int i = 0; i < NV_LANES(r); i++) r[i] = (expr); return r; }
NV_MAP2(vaddq_f32, float32x4_t, a[i] + b[i])
NV_MAP2(vadd_f32, float32x2_t, a[i] + b[i])
NV_MAP2(vsubq_f32, float32x4_t, a[i] - b[i])
NV_MAP2(vmulq_f32, float32x4_t, a[i] * b[i])
NV_MAP2(vdivq_f32, float32x4_t, a[i] / b[i])
NV_MAP2(vmaxq_f32, float32x4_t, emu_fmax(a[i], b[i]))
NV_MAP2(vminq_f32, float32x4_t, emu_fmin(a[i], b[i]))
NV_MAP2(vrecpsq_f32, float32x4_t, emu_frecps(a[i], b[i]))
NV_MAP1(vnegq_f32, float32x4_t, -a[i])
NV_MAP1(vabsq_f32, float32x4_t, fabsf(a[i]))
NV_MAP1(vsqrtq_f32, float32x4_t, sqrtf(a[i]))
NV_MAP1(vrndnq_f32, float32x4_t, rintf(a[i]))
NV_MAP1(vrecpeq_f32, float32x4_t, emu_frecpe(a[i]))
NV_MAP2(vaddq_f64, float64x2_t, a[i] + b[i])
NV_MAP2(vmulq_f64, float64x2_t, a[i] * b[i])

NV float32x4_t vmulq_n_f32(float32x4_t a, float s) { return vmulq_f32(a, vdupq_n_f32(s)); }
NV float32x4_t vmulq_laneq_f32(float32x4_t a, float32x4_t v, int l) { return vmulq_n_f32(a, v[l]); }
/* FMLA / FMLS: a + b * c (a - b * c), one rounding */
NV float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
  float32x4_t r; for (int i = 0; i < 4; i++) r[i] = fmaf(b[i], c[i], a[i]); return r;
}
NV float32x2_t vfma_f32(float32x2_t a, float32x2_t b, float32x2_t c) {
  float32x2_t r; for (int i = 0; i < 2; i++) r[i] = fmaf(b[i], c[i], a[i]); return r;
}
NV float32x4_t vfmsq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
  float32x4_t r; for (int i = 0; i < 4; i++) r[i] = fmaf(-b[i], c[i], a[i]); return r;
}
NV float32x4_t vfmaq_n_f32(float32x4_t a, float32x4_t b, float n) { return vfmaq_f32(a, b, vdupq_n_f32(n)); }
NV float32x4_t vfmsq_n_f32(float32x4_t a, float32x4_t b, float n) { return vfmsq_f32(a, b, vdupq_n_f32(n)); }
NV float32x4_t vfmaq_laneq_f32(float32x4_t a, float32x4_t b, float32x4_t v, int l) { return vfmaq_n_f32(a, b, v[l]); }
NV float32x4_t vfmaq_lane_f32(float32x4_t a, float32x4_t b, float32x2_t v, int l) { return vfmaq_n_f32(a, b, v[l]); }
NV float32x4_t vfmsq_laneq_f32(float32x4_t a, float32x4_t b, float32x4_t v, int l) { return vfmsq_n_f32(a, b, v[l]); }
/* FADDP: pairwise; the across-vector forms reduce the two halves' pairs last */
NV float32x4_t vpaddq_f32(float32x4_t a, float32x4_t b) {
  float32x4_t r = {a[0] + a[1], a[2] + a[3], b[0] + b[1], b[2] + b[3]}; return r;
}
NV float vaddvq_f32(float32x4_t a) { return (a[0] + a[1]) + (a[2] + a[3]); }
NV float vmaxvq_f32(float32x4_t a) { return emu_fmax(emu_fmax(a[0], a[1]), emu_fmax(a[2], a[3])); }
NV float vminvq_f32(float32x4_t a) { return emu_fmin(emu_fmin(a[0], a[1]), emu_fmin(a[2], a[3])); }
/* FCMLE: all ones where a <= b (false for NaN) */
NV uint32x4_t vcleq_f32(float32x4_t a, float32x4_t b) {
  uint32x4_t r; for (int i = 0; i < 4; i++) r[i] = a[i] <= b[i] ? 0xffffffffu : 0u; return r;
}
NV uint32x4_t vcgtq_f32(float32x4_t a, float32x4_t b) {
  uint32x4_t r; for (int i = 0; i < 4; i++) r[i] = a[i] > b[i] ? 0xffffffffu : 0u; return r;
}
NV float32x4_t vbslq_f32(uint32x4_t m, float32x4_t a, float32x4_t b) {
  return (float32x4_t)((m & (uint32x4_t)a) | (~m & (uint32x4_t)b));
}

/* permutes */
NV float32x4_t vzip1q_f32(float32x4_t a, float32x4_t b) { float32x4_t r = {a[0], b[0], a[1], b[1]}; return r; }
NV float32x4_t vzip2q_f32(float32x4_t a, float32x4_t b) { float32x4_t r = {a[2], b[2], a[3], b[3]}; return r; }
NV float32x4_t vtrn1q_f32(float32x4_t a, float32x4_t b) { float32x4_t r = {a[0], b[0], a[2], b[2]}; return r; }
NV float32x4_t vtrn2q_f32(float32x4_t a, float32x4_t b) { float32x4_t r = {a[1], b[1], a[3], b[3]}; return r; }
NV float32x4_t vuzp1q_f32(float32x4_t a, float32x4_t b) { float32x4_t r = {a[0], a[2], b[0], b[2]}; return r; }
NV float32x4_t vuzp2q_f32(float32x4_t a, float32x4_t b) { float32x4_t r = {a[1], a[3], b[1], b[3]}; return r; }
NV float64x2_t vzip1q_f64(float64x2_t a, float64x2_t b) { float64x2_t r = {a[0], b[0]}; return r; }
NV float64x2_t vzip2q_f64(float64x2_t a, float64x2_t b) { float64x2_t r = {a[1], b[1]}; return r; }
NV float64x2_t vtrn1q_f64(float64x2_t a, float64x2_t b) { float64x2_t r = {a[0], b[0]}; return r; }
NV float64x2_t vtrn2q_f64(float64x2_t a, float64x2_t b) { float64x2_t r = {a[1], b[1]}; return r; }
NV int8x16_t vuzp1q_s8(int8x16_t a, int8x16_t b) {
  int8x16_t r; for (int i = 0; i < 8; i++) { r[i] = a[2 * i]; r[8 + i] = b[2 * i]; } return r;
}
NV float32x4_t vextq_f32(float32x4_t a, float32x4_t b, int n) {
  float32x4_t r; for (int i = 0; i < 4; i++) r[i] = i + n < 4 ? a[i + n] : b[i + n - 4]; return r;
}

/* ------------------------------------------------------------------ conversions */
NV float32x4_t vcvtq_f32_s32(int32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r[i] = (float)a[i]; return r; }
NV float32x4_t vcvtq_f32_u32(uint32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r[i] = (float)a[i]; return r; }
NV int32x4_t vcvtq_s32_f32(float32x4_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r[i] = emu_cvtzs(a[i]); return r; }
NV int32x4_t vcvtnq_s32_f32(float32x4_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r[i] = emu_cvtns(a[i]); return r; }
NV int32x4_t vcvtaq_s32_f32(float32x4_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r[i] = emu_cvtas(a[i]); return r; }
NV float32x4_t vcvt_f32_f16(float16x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r[i] = (float)a[i]; return r; }
NV float32x4_t vcvt_high_f32_f16(float16x8_t a) {
  float32x4_t r; for (int i = 0; i < 4; i++) r[i] = (float)a[4 + i]; return r;
}
/* FCVTN: single to half, round to nearest even (one rounding: the float -> _Float16 conversion) */
NV float16x4_t vcvt_f16_f32(float32x4_t a) { float16x4_t r; for (int i = 0; i < 4; i++) r[i] = (_Float16)a[i]; return r; }
NV float16x8_t vcvt_high_f16_f32(float16x4_t lo, float32x4_t a) { return vcombine_f16(lo, vcvt_f16_f32(a)); }

/* ------------------------------------------------------------------ integer lanes (wrap modulo 2^n) */
#define NV_IMAP2(name, T, U, expr)                                                       \
  NV T name(T a_, T b_) { U a = (U)a_, b = (U)b_, r; for (int i = 0; i < NV_LANES(r); i++) r[i] = (expr); return (T)r; }
NV_IMAP2(vaddq_s32, int32x4_t, uint32x4_t, a[i] + b[i])
NV_IMAP2(vsubq_s32, int32x4_t, uint32x4_t, a[i] - b[i])
NV_IMAP2(vmulq_s32, int32x4_t, uint32x4_t, a[i] * b[i])
NV_IMAP2(vaddq_s16, int16x8_t, uint16x8_t, (uint16_t)(a[i] + b[i]))
NV_IMAP2(vsubq_s16, int16x8_t, uint16x8_t, (uint16_t)(a[i] - b[i]))
NV_IMAP2(vaddq_u16, uint16x8_t, uint16x8_t, (uint16_t)(a[i] + b[i]))
NV_IMAP2(vaddq_u32, uint32x4_t, uint32x4_t, a[i] + b[i])
NV_IMAP2(vorrq_u16, uint16x8_t, uint16x8_t, a[i] | b[i])
NV_IMAP2(vorrq_u32, uint32x4_t, uint32x4_t, a[i] | b[i])
NV_IMAP2(vandq_u32, uint32x4_t, uint32x4_t, a[i] & b[i])
#undef NV_IMAP2
NV uint32x4_t vmvnq_u32(uint32x4_t a) { return ~a; }
NV int32x4_t vmulq_n_s32(int32x4_t a, int32_t n) { return vmulq_s32(a, vdupq_n_s32(n)); }
NV int32x4_t vshlq_n_s32(int32x4_t a, int n) { return (int32x4_t)((uint32x4_t)a << n); }
NV int16x8_t vshlq_n_s16(int16x8_t a, int n) { return (int16x8_t)((uint16x8_t)a << n); }
NV int32x4_t vshrq_n_s32(int32x4_t a, int n) { return a >> n; } /* arithmetic (GCC: signed >> is arithmetic) */
NV int16x8_t vshrq_n_s16(int16x8_t a, int n) { return a >> n; }
#define NV_MINMAX(sfx, T)                                                                                  \
  NV T vmaxq_##sfx(T a, T b) { T r; for (int i = 0; i < NV_LANES(r); i++) r[i] = a[i] > b[i] ? a[i] : b[i]; return r; } \
  NV T vminq_##sfx(T a, T b) { T r; for (int i = 0; i < NV_LANES(r); i++) r[i] = a[i] < b[i] ? a[i] : b[i]; return r; }
NV_MINMAX(s32, int32x4_t)
NV_MINMAX(s16, int16x8_t)
NV_MINMAX(u16, uint16x8_t)
NV_MINMAX(s8, int8x16_t)
#undef NV_MINMAX
NV int8x8_t vmax_s8(int8x8_t a, int8x8_t b) { int8x8_t r; for (int i = 0; i < 8; i++) r[i] = a[i] > b[i] ? a[i] : b[i]; return r; }
NV int8x16_t vabsq_s8(int8x16_t a) { /* ABS wraps: |-128| = -128 */
  int8x16_t r; for (int i = 0; i < 16; i++) r[i] = (int8_t)(uint8_t)(a[i] < 0 ? -(unsigned)a[i] : (unsigned)a[i]); return r;
}
NV uint16_t vmaxvq_u16(uint16x8_t a) { uint16_t m = a[0]; for (int i = 1; i < 8; i++) m = a[i] > m ? a[i] : m; return m; }
NV uint32_t vmaxvq_u32(uint32x4_t a) { uint32_t m = a[0]; for (int i = 1; i < 4; i++) m = a[i] > m ? a[i] : m; return m; }
NV int32_t vaddvq_s32(int32x4_t a) { return (int32_t)((uint32_t)a[0] + (uint32_t)a[1] + (uint32_t)a[2] + (uint32_t)a[3]); }
NV uint16x8_t vcgtq_u16(uint16x8_t a, uint16x8_t b) {
  uint16x8_t r; for (int i = 0; i < 8; i++) r[i] = a[i] > b[i] ? 0xffff : 0; return r;
}
/* widening / narrowing */
NV uint16x8_t vaddl_u8(uint8x8_t a, uint8x8_t b) {
  uint16x8_t r; for (int i = 0; i < 8; i++) r[i] = (uint16_t)(a[i] + b[i]); return r;
}
NV int16x8_t vmull_s8(int8x8_t a, int8x8_t b) {
  int16x8_t r; for (int i = 0; i < 8; i++) r[i] = (int16_t)(a[i] * b[i]); return r;
}
NV int16x8_t vmull_high_s8(int8x16_t a, int8x16_t b) { return vmull_s8(vget_high_s8(a), vget_high_s8(b)); }
NV int16x8_t vmlal_s8(int16x8_t acc, int8x8_t a, int8x8_t b) { return vaddq_s16(acc, vmull_s8(a, b)); }
NV int16x8_t vmlal_high_s8(int16x8_t acc, int8x16_t a, int8x16_t b) { return vaddq_s16(acc, vmull_high_s8(a, b)); }
/* SADALP: acc + pairwise sums of the int16 lanes, widened */
NV int32x4_t vpadalq_s16(int32x4_t acc, int16x8_t b) {
  int32x4_t r;
  for (int i = 0; i < 4; i++) r[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)((int32_t)b[2 * i] + (int32_t)b[2 * i + 1]));
  return r;
}
NV int32x4_t vpaddlq_s16(int16x8_t b) { return vpadalq_s16(vdupq_n_s32(0), b); }
/* ADDP: [a0 + a1, a2 + a3, b0 + b1, b2 + b3] */
NV int32x4_t vpaddq_s32(int32x4_t a, int32x4_t b) {
  int32x4_t r = {(int32_t)((uint32_t)a[0] + (uint32_t)a[1]), (int32_t)((uint32_t)a[2] + (uint32_t)a[3]),
                 (int32_t)((uint32_t)b[0] + (uint32_t)b[1]), (int32_t)((uint32_t)b[2] + (uint32_t)b[3])};
  return r;
}
/* SQXTN (saturating) and XTN (truncating) */
NV int16x4_t vqmovn_s32(int32x4_t a) {
  int16x4_t r; for (int i = 0; i < 4; i++) r[i] = a[i] > 32767 ? 32767 : a[i] < -32768 ? -32768 : (int16_t)a[i]; return r;
}
NV int8x8_t vqmovn_s16(int16x8_t a) {
  int8x8_t r; for (int i = 0; i < 8; i++) r[i] = a[i] > 127 ? 127 : a[i] < -128 ? -128 : (int8_t)a[i]; return r;
}
NV int16x4_t vmovn_s32(int32x4_t a) { int16x4_t r; for (int i = 0; i < 4; i++) r[i] = (int16_t)(uint16_t)(uint32_t)a[i]; return r; }
NV int8x8_t vmovn_s16(int16x8_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r[i] = (int8_t)(uint8_t)(uint16_t)a[i]; return r; }
/* SDOT by element: acc[i] + sum over j < 4 of a[4i + j] * b[4 l + j] */
NV int32x4_t vdotq_laneq_s32(int32x4_t acc, int8x16_t a, int8x16_t b, int l) {
  int32x4_t r;
  for (int i = 0; i < 4; i++) {
    int32_t s = 0;
    for (int j = 0; j < 4; j++) s += (int32_t)a[4 * i + j] * (int32_t)b[4 * l + j];
    r[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)s);
  }
  return r;
}
NV int32x4_t vdotq_s32(int32x4_t acc, int8x16_t a, int8x16_t b) {
  int32x4_t r;
  for (int i = 0; i < 4; i++) {
    int32_t s = 0;
    for (int j = 0; j < 4; j++) s += (int32_t)a[4 * i + j] * (int32_t)b[4 * i + j];
    r[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)s);
  }
  return r;
}
/* TBL: out-of-range indices give 0 */
NV uint8x16_t vqtbl1q_u8(uint8x16_t t, uint8x16_t idx) {
  uint8x16_t r; for (int i = 0; i < 16; i++) r[i] = idx[i] < 16 ? t[idx[i]] : 0; return r;
}
NV uint8x16_t vqtbl2q_u8(uint8x16x2_t t, uint8x16_t idx) {
  uint8x16_t r; for (int i = 0; i < 16; i++) r[i] = idx[i] < 32 ? t.val[idx[i] >> 4][idx[i] & 15] : 0; return r;
}

/* ------------------------------------------------------------------ fp16 lanes: one rounding per operation */
NV _Float16 nv_h_round_odd_sum(double p, double c) {
  /* p + c rounded to odd in double (TwoSum gives the exact error), then once to half: the same as rounding the exact
   * sum to half, since double keeps more than two bits beyond half's 11 */
  double s = p + c, bp = s - c, e = (p - bp) + (c - (s - bp));
  if (e != 0 && isfinite(s)) {
    uint64_t u; memcpy(&u, &s, 8);
    if (!(u & 1)) { s = nextafter(s, e > 0 ? INFINITY : -INFINITY); }
  }
  return (_Float16)s;
}
NV _Float16 nv_h_add(_Float16 a, _Float16 b) { return (_Float16)((double)a + (double)b); }
NV _Float16 nv_h_sub(_Float16 a, _Float16 b) { return (_Float16)((double)a - (double)b); }
NV _Float16 nv_h_mul(_Float16 a, _Float16 b) { return (_Float16)((double)a * (double)b); }
NV _Float16 nv_h_fma(_Float16 a, _Float16 b, _Float16 c) { /* a * b + c */
  const double p = (double)a * (double)b; /* exact: 22 significant bits */
  if (!isfinite(p) || !isfinite((double)c)) return (_Float16)(p + (double)c);
  return nv_h_round_odd_sum(p, (double)c);
}
NV _Float16 nv_h_max(_Float16 a, _Float16 b) { return (_Float16)emu_fmax((float)a, (float)b); }
NV _Float16 nv_h_min(_Float16 a, _Float16 b) { return (_Float16)emu_fmin((float)a, (float)b); }
/* FRECPE, half precision (FPRecipEstimate with N = 16: 5 exponent bits, bias 15) */
NV _Float16 nv_h_frecpe(_Float16 x) {
  uint16_t u; memcpy(&u, &x, 2);
  const uint16_t sign = u & 0x8000u, e = (u >> 10) & 0x1fu, frac = u & 0x3ffu;
  uint16_t r;
  if (e == 0x1f && frac) r = u | 0x200u;
  else if (e == 0x1f) r = sign;
  else if (e == 0 && frac == 0) r = sign | 0x7c00u;
  else if (fabsf((float)x) < 0x1p-16f) r = sign | 0x7c00u;
  else {
    int32_t exp = e;
    uint64_t f52 = (uint64_t)frac << 42;
    if (exp == 0) {
      if (!((f52 >> 51) & 1)) { exp = -1; f52 = (f52 << 2) & ((1ull << 52) - 1); }
      else f52 = (f52 << 1) & ((1ull << 52) - 1);
    }
    const uint32_t est = emu_recip_estimate(256u | (uint32_t)(f52 >> 44));
    int32_t rexp = 29 - exp;
    uint64_t rf = (uint64_t)(est & 0xffu) << 44;
    if (rexp == 0) rf = (1ull << 51) | (rf >> 1);
    else if (rexp == -1) { rf = (1ull << 50) | (rf >> 2); rexp = 0; }
    r = sign | (uint16_t)((uint32_t)rexp << 10) | (uint16_t)(rf >> 42);
  }
  _Float16 y; memcpy(&y, &r, 2);
  return y;
}
NV _Float16 nv_h_frecps(_Float16 a, _Float16 b) {
  if ((isinf((float)a) && (float)b == 0.f) || ((float)a == 0.f && isinf((float)b))) return (_Float16)2.f;
  return nv_h_fma((_Float16)-a, b, (_Float16)2.f);
}
#define NV_HMAP2(name, T, expr)                                                          \
  NV T name(T a, T b) { T r; for (int i = 0; i < NV_LANES(r); i++) r[i] = (expr); return r; }
NV_HMAP2(vaddq_f16, float16x8_t, nv_h_add(a[i], b[i]))
NV_HMAP2(vsubq_f16, float16x8_t, nv_h_sub(a[i], b[i]))
NV_HMAP2(vmulq_f16, float16x8_t, nv_h_mul(a[i], b[i]))
NV_HMAP2(vmaxq_f16, float16x8_t, nv_h_max(a[i], b[i]))
NV_HMAP2(vminq_f16, float16x8_t, nv_h_min(a[i], b[i]))
NV_HMAP2(vrecpsq_f16, float16x8_t, nv_h_frecps(a[i], b[i]))
NV_HMAP2(vadd_f16, float16x4_t, nv_h_add(a[i], b[i]))
NV_HMAP2(vmul_f16, float16x4_t, nv_h_mul(a[i], b[i]))
#undef NV_HMAP2
NV float16x8_t vabsq_f16(float16x8_t a) {
  uint16x8_t u = (uint16x8_t)a; return (float16x8_t)(u & (uint16_t)0x7fff);
}
NV float16x8_t vrecpeq_f16(float16x8_t a) { float16x8_t r; for (int i = 0; i < 8; i++) r[i] = nv_h_frecpe(a[i]); return r; }
NV float16x8_t vmulq_n_f16(float16x8_t a, _Float16 n) { return vmulq_f16(a, vdupq_n_f16(n)); }
NV float16x8_t vfmaq_f16(float16x8_t a, float16x8_t b, float16x8_t c) {
  float16x8_t r; for (int i = 0; i < 8; i++) r[i] = nv_h_fma(b[i], c[i], a[i]); return r;
}
NV float16x4_t vfma_f16(float16x4_t a, float16x4_t b, float16x4_t c) {
  float16x4_t r; for (int i = 0; i < 4; i++) r[i] = nv_h_fma(b[i], c[i], a[i]); return r;
}
NV float16x8_t vfmsq_f16(float16x8_t a, float16x8_t b, float16x8_t c) {
  float16x8_t r; for (int i = 0; i < 8; i++) r[i] = nv_h_fma((_Float16)-b[i], c[i], a[i]); return r;
}
NV float16x8_t vfmaq_n_f16(float16x8_t a, float16x8_t b, _Float16 n) { return vfmaq_f16(a, b, vdupq_n_f16(n)); }
NV float16x8_t vfmaq_laneq_f16(float16x8_t a, float16x8_t b, float16x8_t v, int l) { return vfmaq_n_f16(a, b, v[l]); }
NV _Float16 vfmah_f16(_Float16 a, _Float16 b, _Float16 c) { return nv_h_fma(b, c, a); }
NV _Float16 vmaxvq_f16(float16x8_t a) {
  _Float16 l0 = nv_h_max(nv_h_max(a[0], a[1]), nv_h_max(a[2], a[3]));
  _Float16 l1 = nv_h_max(nv_h_max(a[4], a[5]), nv_h_max(a[6], a[7]));
  return nv_h_max(l0, l1);
}
NV _Float16 vminvq_f16(float16x8_t a) {
  _Float16 l0 = nv_h_min(nv_h_min(a[0], a[1]), nv_h_min(a[2], a[3]));
  _Float16 l1 = nv_h_min(nv_h_min(a[4], a[5]), nv_h_min(a[6], a[7]));
  return nv_h_min(l0, l1);
}

#undef NV_MAP1
#undef NV_MAP2
#endif
