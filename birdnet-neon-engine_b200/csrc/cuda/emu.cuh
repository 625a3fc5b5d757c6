// Device arithmetic that reproduces the reference's AArch64 results bit for bit.
//
// Every floating-point step is an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn, ...) and the
// translation units build with -fmad=false -ftz=false -prec-div=true -prec-sqrt=true, so nothing is contracted or
// flushed behind our back.
//   * FRECPE / FRECPS: the Arm ARM pseudocode (FPRecipEstimate, RecipEstimate, FPRecipStepFused) with the Linux FPCR
//     defaults (FZ = 0, AH = 0): the reciprocal estimate and Newton step of the reference's SiLU and sigmoid
//     (src/gemm_f32.h:87-118).
//   * FMIN / FMAX: NaN-propagating (PTX min.NaN / max.NaN), as NEON vminq_f32 / vmaxq_f32.
//   * FCVTNS: cvt.rni.s32.f32 saturates and maps NaN to 0, as NEON does.
//   * glibc expf (the SE block's SiLU calls libm expf, src/v24_f32.c:160): the published table-driven algorithm of
//     glibc >= 2.27 (ARM optimized-routines: k = round(x N / ln 2), N = 32, 2^(k/N) from a 32-entry table, a cubic in
//     r for 2^(r/N), evaluated in double), with the products fused as the FMA build of glibc fuses them. The table is
//     computed on the host from libm exp2 and uploaded once per device. Host tests compare this against libm expf.
#pragma once
#include <stdint.h>

namespace bnn {

// Per translation unit (the kernels build without relocatable device code, so each .cu file holds its own copy and
// fills it in its *_tables_init): the glibc expf table and the FRECPE estimate table (est(256 + i) << 15).
static __constant__ unsigned long long c_expf_tab[32];
static __device__ uint32_t g_frecpe_lut[256];

__device__ __forceinline__ float fmin_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// FCVTNS: nearest-even, saturating, NaN -> 0
__device__ __forceinline__ int32_t cvtns(float x) {
  int32_t r;
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// FCVTZS: toward zero, saturating, NaN -> 0
__device__ __forceinline__ int32_t cvtzs(float x) {
  int32_t r;
  asm("cvt.rzi.s32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// glibc lrintf on AArch64 (nearest-even to 64 bits, saturating), then the C conversion to int32_t (modulo 2^32)
__device__ __forceinline__ int32_t lrintf_i32(float x) {
  long long r;
  asm("cvt.rni.s64.f32 %0, %1;" : "=l"(r) : "f"(x));
  return (int32_t)(uint32_t)(unsigned long long)r;
}

// s8n_quant_rows' per-row parameters (gemm_s8n.c:15-63) from the row's min lo and max hi: a constant row (range
// not above 1e-30 of its magnitude) is quantized symmetrically (zero point 0), else asymmetrically into [-127, 127]
__device__ __forceinline__ void quant_params(float lo, float hi, float &inv, int32_t &z, float &s) {
  const float d = __fsub_rn(hi, lo);
  if (!(d > __fmul_rn(1e-30f, fmaxf(fabsf(hi), fabsf(lo)))) || !(d > 0.f)) {
    const float a = fmaxf(fabsf(hi), 1e-30f);
    inv = __fdiv_rn(127.f, a);
    z = 0;
    s = __fdiv_rn(a, 127.f);
  } else {
    inv = __fdiv_rn(254.f, d);
    z = (int32_t)(0u - 127u - (uint32_t)lrintf_i32(__fmul_rn(lo, inv)));
    s = __fdiv_rn(d, 254.f);
  }
}
// four quantized values packed little-endian: clamp(round(t) + z, -127, 127); the 8-wide part rounds with FCVTNS,
// the tail (columns past the last multiple of 8) with lrintf
__device__ __forceinline__ uint32_t quant_word(float t0, float t1, float t2, float t3, int32_t z, bool eight_wide) {
  int32_t qi[4];
  if (eight_wide) {
    qi[0] = cvtns(t0); qi[1] = cvtns(t1); qi[2] = cvtns(t2); qi[3] = cvtns(t3);
  } else {
    qi[0] = lrintf_i32(t0); qi[1] = lrintf_i32(t1); qi[2] = lrintf_i32(t2); qi[3] = lrintf_i32(t3);
  }
#pragma unroll
  for (int t = 0; t < 4; t++) qi[t] = min(max((int32_t)((uint32_t)qi[t] + (uint32_t)z), -127), 127);
  return __byte_perm(__byte_perm(qi[0], qi[1], 0x0040), __byte_perm(qi[2], qi[3], 0x0040), 0x5410);
}

// The same for a row whose scaled values all lie below 2^22 in magnitude (quant_fast): t + 1.5 * 2^23 falls in
// (2^23, 2^24), where the fp32 grid is the integers, so the one rounded add rounds t to nearest-even, as FCVTNS and
// lrintf do there, and its bits are 0x4B400000 + round(t). The products x * inv feed that add, so they stay scalar
// (__fmul_rn: never contracted). Rows with larger values, NaN or infinities keep the conversions above.
constexpr float kRoundMagic = 12582912.f;  // 1.5 * 2^23
constexpr uint32_t kRoundBits = 0x4B400000u;
__device__ __forceinline__ bool quant_fast(float lo, float hi, float inv) {
  return __fmul_rn(fmaxf(fabsf(lo), fabsf(hi)), inv) < 4194304.f;  // false for NaN / infinite lo, hi
}
__device__ __forceinline__ uint32_t quant_word_fast(float4 v, float inv, uint32_t zz) {  // zz = z - kRoundBits
  const int32_t q0 = min(max((int32_t)(__float_as_uint(__fadd_rn(__fmul_rn(v.x, inv), kRoundMagic)) + zz), -127), 127);
  const int32_t q1 = min(max((int32_t)(__float_as_uint(__fadd_rn(__fmul_rn(v.y, inv), kRoundMagic)) + zz), -127), 127);
  const int32_t q2 = min(max((int32_t)(__float_as_uint(__fadd_rn(__fmul_rn(v.z, inv), kRoundMagic)) + zz), -127), 127);
  const int32_t q3 = min(max((int32_t)(__float_as_uint(__fadd_rn(__fmul_rn(v.w, inv), kRoundMagic)) + zz), -127), 127);
  return __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
}

// RecipEstimate of the Arm ARM for a in [256, 512): ((2^19 / (2a + 1)) + 1) / 2
__device__ __forceinline__ uint32_t recip_estimate(uint32_t a) {
  uint32_t b = (1u << 19) / (2u * a + 1u);
  return (b + 1u) >> 1;
}

// FRECPE (single precision), the whole pseudocode: special values, denormal inputs and outputs
__device__ __forceinline__ float frecpe(float x) {
  uint32_t u = __float_as_uint(x), sign = u & 0x80000000u;
  uint32_t e = (u >> 23) & 0xffu, frac = u & 0x7fffffu;
  if (e == 0xffu) return frac ? __uint_as_float(u | 0x400000u) : __uint_as_float(sign);
  if (e == 0 && frac == 0) return __uint_as_float(sign | 0x7f800000u);
  if (fabsf(x) < 0x1p-128f) return __uint_as_float(sign | 0x7f800000u);
  int32_t ex = (int32_t)e;
  uint32_t f = frac << 9;  // the pseudocode's 52-bit fraction, top 32 bits (bits 51..20)
  if (ex == 0) {
    if (!(f >> 31)) { ex = -1; f <<= 2; }
    else f <<= 1;
  }
  uint32_t est = recip_estimate(256u | (f >> 24)) & 0xffu;
  int32_t rexp = 253 - ex;
  uint32_t m;
  if (rexp > 0) m = est << 15;
  else if (rexp == 0) m = (1u << 22) | (est << 14);
  else { m = (1u << 21) | (est << 13); rexp = 0; }
  return __uint_as_float(sign | ((uint32_t)rexp << 23) | m);
}

// FRECPE for a normal d in [1, 2^126) (the SiLU denominators): exponent 253 - e, 8-bit estimate from the table
// (lut[i] = estimate(256 + i) << 15). The estimate bits and the exponent bits do not overlap, so the pseudocode's
// OR is an add (one three-input integer add), and the table is read at a byte offset cut straight from the mantissa.
__device__ __forceinline__ float frecpe_ge1(float d, const uint32_t *lut) {
  const uint32_t u = __float_as_uint(d);
  const uint32_t est = *reinterpret_cast<const uint32_t *>(reinterpret_cast<const char *>(lut) + ((u >> 13) & 0x3fcu));
  return __uint_as_float(0x7e800000u - (u & 0x7f800000u) + est);
}

// FRECPS(a, b) = 2 - a * b fused (finite operands: the infinity x zero case cannot arise here)
__device__ __forceinline__ float frecps(float a, float b) { return __fmaf_rn(-a, b, 2.f); }

// silu_f32x4 / SILU_N_F32X4 (src/gemm_f32.h:102-144)
template <bool kLut>
__device__ __forceinline__ float silu(float x, const uint32_t *lut) {
  const float magic = 0x1.8p+23f;
  float t = __fmul_rn(x, -0x1.715476p+0f);
  t = fmin_nan(fmax_nan(t, -60.f), 60.f);
  float tm = __fadd_rn(t, magic);
  float f = __fsub_rn(t, __fsub_rn(tm, magic));
  float p = __fmaf_rn(0x1.5d87fep-10f, f, 0x1.3b2ab6p-7f);
  p = __fmaf_rn(p, f, 0x1.c6b08ep-5f);
  p = __fmaf_rn(p, f, 0x1.ebfbep-3f);
  p = __fmaf_rn(p, f, 0x1.62e43p-1f);
  p = __fmaf_rn(p, f, 1.0f);
  uint32_t ni = __float_as_uint(tm) << 23;
  float d = __fadd_rn(1.f, __uint_as_float(__float_as_uint(p) + ni));
  float r = kLut ? frecpe_ge1(d, lut) : frecpe(d);
  r = __fmul_rn(r, frecps(d, r));
  return __fmul_rn(x, r);
}

// sm_100's paired fp32 instructions (each half an IEEE fp32 operation). Measured with this toolchain: a paired
// multiply whose result feeds a paired add comes out fused into one rounding although both carry .rn, while the
// scalar forms never are. So the paired forms serve only chains in which no product feeds an add or a
// subtraction (a product into a multiply, an fma, a min / max or a store); products that feed an add stay scalar.
__device__ __forceinline__ unsigned long long pk2(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 up2(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return up2(d);
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return up2(d);
}
__device__ __forceinline__ float2 sub2_rn(float2 a, float2 b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return up2(d);
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
  return up2(d);
}
__device__ __forceinline__ float2 neg2(float2 v) { return make_float2(-v.x, -v.y); }
__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }

// The SiLU above on two lanes (a - b is a + (-b), exactly). Its one product that meets an add, x * -log2(e), is
// clamped by the scalar min / max first; the result x * r is a product, so callers add to it with scalar __fadd_rn.
__device__ __forceinline__ float2 silu2(float2 x, const uint32_t *lut) {
  const float magic = 0x1.8p+23f;
  float2 t = mul2_rn(x, splat2(-0x1.715476p+0f));
  t.x = fmin_nan(fmax_nan(t.x, -60.f), 60.f);
  t.y = fmin_nan(fmax_nan(t.y, -60.f), 60.f);
  const float2 tm = add2_rn(t, splat2(magic));
  const float2 f = sub2_rn(t, add2_rn(tm, splat2(-magic)));
  float2 p = fma2_rn(splat2(0x1.5d87fep-10f), f, splat2(0x1.3b2ab6p-7f));
  p = fma2_rn(p, f, splat2(0x1.c6b08ep-5f));
  p = fma2_rn(p, f, splat2(0x1.ebfbep-3f));
  p = fma2_rn(p, f, splat2(0x1.62e43p-1f));
  p = fma2_rn(p, f, splat2(1.0f));
  const float2 e = make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(tm.x) << 23)),
                               __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(tm.y) << 23)));
  const float2 d = add2_rn(splat2(1.f), e);
  const float2 dn = sub2_rn(splat2(-1.f), e);  // -d exactly: rounding to nearest is symmetric in sign
  float2 r = make_float2(frecpe_ge1(d.x, lut), frecpe_ge1(d.y, lut));
  r = mul2_rn(r, fma2_rn(dn, r, splat2(2.f)));  // FRECPS(d, r) = 2 - d r fused
  return mul2_rn(x, r);
}

// exp2_f32x4 (src/gemm_f32.h:74-85)
__device__ __forceinline__ float exp2_poly(float t) {
  t = fmin_nan(fmax_nan(t, -126.f), 126.f);
  float n = rintf(t), f = __fsub_rn(t, n);
  float p = 0x1.430912p-13f;
  p = __fmaf_rn(p, f, 0x1.5d87fep-10f);
  p = __fmaf_rn(p, f, 0x1.3b2ab6p-7f);
  p = __fmaf_rn(p, f, 0x1.c6b08ep-5f);
  p = __fmaf_rn(p, f, 0x1.ebfbep-3f);
  p = __fmaf_rn(p, f, 0x1.62e43p-1f);
  p = __fmaf_rn(p, f, 1.f);
  return __uint_as_float(__float_as_uint(p) + ((uint32_t)cvtzs(n) << 23));
}
// sigmoid_f32x4 (src/gemm_f32.h:93-96): FRECPE + two fused Newton steps
__device__ __forceinline__ float sigmoid(float x) {
  float d = __fadd_rn(1.f, exp2_poly(__fmul_rn(x, -0x1.715476p+0f)));
  float r = frecpe(d);
  r = __fmul_rn(r, frecps(d, r));
  r = __fmul_rn(r, frecps(d, r));
  return r;
}

// log2_acc_f32x4 (src/gemm_f32.h:57-71)
__device__ __forceinline__ float log2_acc(float x) {
  uint32_t xi = __float_as_uint(x);
  int32_t e = ((int32_t)(xi - 0x3f3504f3u)) >> 23;
  float z = __fsub_rn(__uint_as_float(xi - ((uint32_t)e << 23)), 1.f);
  float p = __fmaf_rn(z, 0x1.f0a97ep-4f, -0x1.a6c552p-3f);
  p = __fmaf_rn(z, p, 0x1.bcc44cp-3f);
  p = __fmaf_rn(z, p, -0x1.e9aef8p-3f);
  p = __fmaf_rn(z, p, 0x1.26a67p-2f);
  p = __fmaf_rn(z, p, -0x1.7159ccp-2f);
  p = __fmaf_rn(z, p, 0x1.ec75e6p-2f);
  p = __fmaf_rn(z, p, -0x1.715476p-1f);
  p = __fmaf_rn(z, p, 0x1.715474p+0f);
  return __fmaf_rn(z, p, __int2float_rn(e));
}
// exp2_acc (src/v24_fe.c:109-123): exp2_poly without the upper clamp
__device__ __forceinline__ float exp2_acc(float t) {
  t = fmax_nan(t, -126.f);
  float n = rintf(t), f = __fsub_rn(t, n);
  float p = 0x1.430912p-13f;
  p = __fmaf_rn(p, f, 0x1.5d87fep-10f);
  p = __fmaf_rn(p, f, 0x1.3b2ab6p-7f);
  p = __fmaf_rn(p, f, 0x1.c6b08ep-5f);
  p = __fmaf_rn(p, f, 0x1.ebfbep-3f);
  p = __fmaf_rn(p, f, 0x1.62e43p-1f);
  p = __fmaf_rn(p, f, 1.f);
  return __uint_as_float(__float_as_uint(p) + ((uint32_t)cvtzs(n) << 23));
}

// glibc expf (see the header comment). tab[i] = bits(2^(i/32)) - (i << 47).
__device__ __forceinline__ float glibc_expf(float x, const unsigned long long *tab) {
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32, c2 = 0x1.62e42ff0c52d6p-1 / 32;
  uint32_t ux = __float_as_uint(x), abstop = (ux >> 20) & 0x7ffu;
  if (abstop >= 0x42bu) {  // |x| >= 88 (top 12 bits of 88.0f), infinities and NaN
    if (ux == 0xff800000u) return 0.f;
    if (abstop >= 0x7f8u) return __fadd_rn(x, x);
    if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
    if (x < -0x1.9fe368p6f) return 0.f;
  }
  double xd = (double)x;
  double kd = __fma_rn(inv_ln2_n, xd, shift);
  unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, shift);
  double r = __fma_rn(inv_ln2_n, xd, -kd);
  double s = __longlong_as_double((long long)(tab[ki & 31] + (ki << 47)));
  double z = __fma_rn(c0, r, c1), r2 = __dmul_rn(r, r), y = __fma_rn(c2, r, 1.0);
  y = __fma_rn(z, r2, y);
  return __double2float_rn(__dmul_rn(y, s));
}

}  // namespace bnn
