/* CPU restatement of the AArch64 NEON arithmetic the reference's int8 path relies on (TEST INFRASTRUCTURE ONLY).
 *
 * This header belongs to the parity oracle: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load anything under oracle/. It is never part of the product path.
 *
 * What is emulated, and from where:
 *   - FRECPE (reciprocal estimate) and FRECPS (fused reciprocal step): Arm Architecture Reference Manual pseudocode
 *     FPRecipEstimate / RecipEstimate / FPRecipStepFused, with the Linux user-space FPCR defaults (FZ = 0, DN = 0,
 *     AH = 0, round to nearest). Used by rcp_f32x4 / silu_f32x4 / sigmoid_f32x4 (src/gemm_f32.h:87-118).
 *   - FMIN/FMAX (vminq_f32/vmaxq_f32, vminvq/vmaxvq): NaN in either operand gives NaN; min(-0, +0) = -0.
 *   - FCVTNS (vcvtnq_s32_f32): round to nearest even, saturating, NaN -> 0. FCVTZS (vcvtq_s32_f32): truncating.
 *   - FADDP reduction (vaddvq_f32): (x0 + x1) + (x2 + x3).
 * NaN payloads are not modelled (the parity tests compare NaN as NaN). */
#ifndef BNN_ORACLE_ARM_EMU_H
#define BNN_ORACLE_ARM_EMU_H
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint32_t emu_bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float emu_float(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* FMIN / FMAX (NEON): NaN-propagating, -0 < +0 */
static inline float emu_fmin(float a, float b) {
  if (a != a || b != b) return NAN;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}
static inline float emu_fmax(float a, float b) {
  if (a != a || b != b) return NAN;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

/* FCVTNS: nearest-even, saturating to int32, NaN -> 0 */
static inline int32_t emu_cvtns(float x) {
  if (x != x) return 0;
  float r = rintf(x); /* the default rounding mode is round-to-nearest-even */
  if (r >= 2147483648.0f) return INT32_MAX;
  if (r < -2147483648.0f) return INT32_MIN;
  return (int32_t)r;
}
/* FCVTZS: toward zero, saturating, NaN -> 0 */
static inline int32_t emu_cvtzs(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483904.0f) return INT32_MIN;
  return (int32_t)x;
}
/* FCVTAS (vcvtaq_s32_f32): nearest with ties away from zero, saturating to int32, NaN -> 0 */
static inline int32_t emu_cvtas(float x) {
  if (x != x) return 0;
  float r = roundf(x); /* C roundf: halfway cases away from zero */
  if (r >= 2147483648.0f) return INT32_MAX;
  if (r < -2147483648.0f) return INT32_MIN;
  return (int32_t)r;
}
/* glibc lrintf on AArch64 (FRINTX + FCVTZS to 64 bits), then the C conversion to int32_t (modulo 2^32). The
 * reference only reaches values well inside int64. */
static inline int32_t emu_lrintf_i32(float x) {
  if (x != x) return 0;
  double r = rint((double)x);
  if (r >= 9223372036854775808.0) return (int32_t)(uint32_t)0xffffffffu; /* INT64_MAX mod 2^32 */
  if (r < -9223372036854775808.0) return 0;                              /* INT64_MIN mod 2^32 */
  return (int32_t)(uint32_t)(uint64_t)(int64_t)r;
}

/* RecipEstimate(a), a in [256, 512): the 8-bit estimate of 1/a in [256, 512) */
static inline uint32_t emu_recip_estimate(uint32_t a) {
  a = a * 2 + 1;
  uint32_t b = (1u << 19) / a;
  return (b + 1) / 2;
}

/* FRECPE, single precision */
static inline float emu_frecpe(float x) {
  uint32_t u = emu_bits(x), sign = u & 0x80000000u;
  uint32_t e = (u >> 23) & 0xffu, frac = u & 0x7fffffu;
  if (e == 0xffu && frac) return emu_float(u | 0x400000u);          /* NaN: quieted */
  if (e == 0xffu) return emu_float(sign);                           /* infinity -> signed zero */
  if (e == 0 && frac == 0) return emu_float(sign | 0x7f800000u);    /* zero -> signed infinity */
  if (fabsf(x) < 0x1p-128f) return emu_float(sign | 0x7f800000u);  /* overflow, round to nearest -> infinity */
  int32_t exp = (int32_t)e;
  uint64_t f52 = (uint64_t)frac << 29; /* the 52-bit fraction of the pseudocode */
  if (exp == 0) {
    if (!((f52 >> 51) & 1)) { exp = -1; f52 = (f52 << 2) & ((1ull << 52) - 1); }
    else f52 = (f52 << 1) & ((1ull << 52) - 1);
  }
  uint32_t scaled = 256u | (uint32_t)(f52 >> 44);
  int32_t rexp = 253 - exp;
  uint32_t est = emu_recip_estimate(scaled);
  uint64_t rf = (uint64_t)(est & 0xffu) << 44;
  if (rexp == 0) rf = (1ull << 51) | (rf >> 1);
  else if (rexp == -1) { rf = (1ull << 50) | (rf >> 2); rexp = 0; }
  return emu_float(sign | ((uint32_t)rexp << 23) | (uint32_t)(rf >> 29));
}

/* FRECPS(a, b) = 2 - a * b, fused; infinity x zero gives 2 */
static inline float emu_frecps(float a, float b) {
  if ((isinf(a) && b == 0.f) || (a == 0.f && isinf(b))) return 2.f;
  return fmaf(-a, b, 2.f);
}

/* vaddvq_f32: pairwise */
static inline float emu_addv4(const float v[4]) { return (v[0] + v[1]) + (v[2] + v[3]); }

#endif
