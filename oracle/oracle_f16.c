/* bnn oracle, neon-fp16 path: a CPU restatement of the reference's fp16 kernels for the v2.4 architecture (TEST
 * INFRASTRUCTURE ONLY: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it).
 *
 * The reference runs these kernels with ARMv8.2 fp16 arithmetic (FMLA .8h and friends) under the Linux FPCR
 * defaults: round to nearest even, fp16 subnormals kept (FZ16 = 0). Each of its fp16 operations rounds once, so the
 * oracle computes every operation exactly and rounds once:
 *   - add, sub, mul: the exact sum / product of two fp16 values fits a double (at most 40 / 22 significant bits), so
 *     one double operation followed by one rounding to fp16 is exact-then-round;
 *   - fused multiply-add a * b + c: the product is exact in a double; the sum is formed in a double with round to
 *     odd (the TwoSum error decides the sticky bit), then rounded once to fp16. Rounding to odd at 53 bits followed
 *     by rounding to nearest at 11 bits gives the correctly rounded result (Boldo and Melquiond, "When double rounding
 *     is odd", 2005).
 * NaN results are the default NaN (0x7e00); payloads are not modelled (the parity tests compare NaN as NaN).
 *
 * Ops and their reference sources:
 *   GEMM (PW f16, the pc conv): src/gemm_f16.c:52-169 -- K in balanced blocks of <= FLUSH_K = 128 k-steps (a
 *     multiple of 8), one fp16 FMA chain per output and block from +0 in k order, blocks summed in fp32 from 0 when
 *     there are two or more; bias: fp16 add of b16 (one block) or fp32 add of b32 then one rounding (several);
 *     epilogue: SiLU table (src/silu_lut.h) or FMAX(x, 0), then the fp16 residual add, stored at the padded row.
 *   C0POOL f16: src/v24_fast.c:150-164 + gemm_f16_rows (src/gemm_f16.c:171-207): the image rounded to fp16 in a
 *     zero border, one chain over K = 64 in (ky, kx, ci) order, + b16, ReLU, [max | avg] of pixel pairs.
 *   DW3 f16: src/kern_f16.c:83-155 (two FMA chains per tap row set, SiLU, fp16 row sums flushed to fp32).
 *   SE f16: src/v24_fast.c:186-235 (the fp32 gate with the degree-6 exp2 sigmoid and an IEEE division, rounded to
 *     fp16; the activation scaled in place by an fp16 multiply).
 *   POSTPC f16: src/v24_fast.c:273-311. DENSE f16: src/v24_fast.c:237-270. DENSE f32: src/v24_f32.c:213-243. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "arm_emu.h"
#include "oracle.h"

typedef uint16_t h16;

/* ------------------------------------------------------------------ fp16 arithmetic */

static double h2d_calc(h16 h) {
  const int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  double v;
  if (e == 31) v = m ? NAN : INFINITY;
  else if (e == 0) v = ldexp((double)m, -24);
  else v = ldexp((double)(m | 1024), e - 25);
  return s ? -v : v;
}
/* every fp16 value as a double (exact), filled once when the library loads */
static double H2D[65536];
__attribute__((constructor)) static void h2d_init(void) {
  for (int i = 0; i < 65536; i++) H2D[i] = h2d_calc((h16)i);
}
double bnno_h2d(h16 h) { return H2D[h]; }
float bnno_h2f(h16 h) { return (float)bnno_h2d(h); }

/* one rounding of a double to fp16, nearest even; overflow to infinity; NaN -> the default NaN */
h16 bnno_d2h(double x) {
  uint64_t u;
  memcpy(&u, &x, 8);
  const h16 s = (h16)((u >> 48) & 0x8000);
  const uint64_t a = u & 0x7fffffffffffffffull;
  if (a >= 0x7ff0000000000000ull) return a > 0x7ff0000000000000ull ? 0x7e00 : (h16)(s | 0x7c00);
  if (a == 0) return s;
  const int e = (int)(a >> 52) - 1023;           /* |x| in [2^e, 2^(e+1)) (a double subnormal is far below fp16) */
  if (e >= 16) return (h16)(s | 0x7c00);
  if (e < -25) return s;                         /* below half the smallest subnormal */
  const uint64_t m = (a & ((1ull << 52) - 1)) | (1ull << 52);
  const int E = e < -14 ? -14 : e;               /* the fp16 exponent whose ulp is 2^(E - 10) */
  const int sh = 42 + (E - e);                   /* m * 2^(e - 52) in units of 2^(E - 10) */
  uint64_t q = m >> sh;
  const uint64_t rem = m & ((1ull << sh) - 1), half = 1ull << (sh - 1);
  if (rem > half || (rem == half && (q & 1))) q++;
  return (h16)(s | (h16)(((E + 14) << 10) + (int)q)); /* q = 2^11 carries into the exponent; E = 15 -> infinity */
}
h16 bnno_f2h(float x) { return bnno_d2h((double)x); }

h16 bnno_h_add(h16 a, h16 b) { return bnno_d2h(bnno_h2d(a) + bnno_h2d(b)); }
h16 bnno_h_mul(h16 a, h16 b) { return bnno_d2h(bnno_h2d(a) * bnno_h2d(b)); }
static h16 h_sub(h16 a, h16 b) { return bnno_h_add(a, (h16)(b ^ 0x8000)); }

/* a * b + c, one rounding */
h16 bnno_h_fma(h16 a, h16 b, h16 c) {
  const double p = bnno_h2d(a) * bnno_h2d(b), cc = bnno_h2d(c);
  double s = p + cc;
  if (!isfinite(p) || !isfinite(cc) || !isfinite(s)) return bnno_d2h(s);
  const double bb = s - p, err = (p - (s - bb)) + (cc - bb); /* TwoSum: p + cc = s + err exactly */
  if (err != 0) {
    uint64_t u;
    memcpy(&u, &s, 8);
    if (!(u & 1)) u += ((err > 0) == (s > 0)) ? 1 : (uint64_t)-1; /* to the odd neighbour on err's side */
    memcpy(&s, &u, 8);
  }
  return bnno_d2h(s);
}

static int h_nan(h16 x) { return (x & 0x7c00) == 0x7c00 && (x & 1023); }
/* FMAX / FMIN (fp16): NaN-propagating, -0 < +0 */
static h16 h_max(h16 a, h16 b) {
  if (h_nan(a) || h_nan(b)) return 0x7e00;
  const double x = bnno_h2d(a), y = bnno_h2d(b);
  if (x == y) return (a & 0x8000) ? b : a;
  return x > y ? a : b;
}
static h16 h_min(h16 a, h16 b) {
  if (h_nan(a) || h_nan(b)) return 0x7e00;
  const double x = bnno_h2d(a), y = bnno_h2d(b);
  if (x == y) return (a & 0x8000) ? a : b;
  return x < y ? a : b;
}

/* The SiLU of the fp16 kernels, src/silu_lut.h:23-38: silu(x) = FMAX(x, 0) - |x| q(|x|) with q(u) ~ sigmoid(-u) a
 * quadratic per unit segment n = round(min(|x|, 15.4)) (16 segments), coefficients c0[n] + c1[n] f + c2[n] f^2 at
 * f = u - n. The coefficient table is the reference's (src/silu_lut_tables_deg2.h: the low and high bytes of each
 * fp16 value, for its 2-register TBL), here as whole fp16 values. */
const h16 BNNO_SILU_C0[16] = {0x3800, 0x344e, 0x2fa1, 0x2a12, 0x249a, 0x1ed9, 0x1910, 0x1375,
                              0x0d7e, 0x080a, 0x02f9, 0x0118, 0x0067, 0x0026, 0x000e, 0x0005};
const h16 BNNO_SILU_C1[16] = {0xb40b, 0xb242, 0xaecc, 0xa9ea, 0xa4a6, 0x9f03, 0x9935, 0x93b1,
                              0x8daa, 0x882c, 0x8312, 0x8121, 0x806a, 0x8027, 0x800e, 0x8005};
const h16 BNNO_SILU_C2[16] = {0x23bd, 0x299d, 0x2915, 0x254c, 0x2073, 0x1ae1, 0x1528, 0x0fa3,
                              0x09a2, 0x0426, 0x0187, 0x0090, 0x0035, 0x0013, 0x0007, 0x0003};

h16 bnno_h_silu(h16 x) {
  const h16 magic = 0x6600 /* 1536 */, umax = 0x4bb3 /* (fp16)15.4 */;
  const h16 u = (h16)(x & 0x7fff);                 /* FABS */
  const h16 uc = h_min(u, umax);
  const h16 tm = bnno_h_add(uc, magic);            /* 1536 + round(uc): the low byte of its bits is the segment */
  const h16 f = h_sub(uc, h_sub(tm, magic));
  const int n = tm & 0xff;                         /* TBL: an index past the 32 table bytes reads 0 */
  const h16 c0 = n < 16 ? BNNO_SILU_C0[n] : 0, c1 = n < 16 ? BNNO_SILU_C1[n] : 0, c2 = n < 16 ? BNNO_SILU_C2[n] : 0;
  h16 p = bnno_h_fma(c2, f, c1);
  p = bnno_h_fma(p, f, c0);
  return bnno_h_fma((h16)(u ^ 0x8000), p, h_max(x, 0)); /* FMLS: FMAX(x, 0) - u * p, one rounding */
}

/* ------------------------------------------------------------------ GEMM (src/gemm_f16.c) */

/* hp_pack panels: [Np/16][Kp][16], then for Np % 16 a [Kp][8] tail panel */
static inline h16 hp_w(const h16 *w, int Kp, int Np, int n, int k) {
  const int n16 = Np / 16, nb = n / 16;
  return nb < n16 ? w[((size_t)nb * Kp + k) * 16 + n % 16] : w[(size_t)n16 * Kp * 16 + (size_t)k * 8 + n % 16];
}

/* kblocks (src/gemm_f16.c:58-62) */
static void kblocks(int Kp, int *nblk, int *bs) {
  *nblk = (Kp + 127) / 128;
  *bs = ((Kp + *nblk - 1) / *nblk + 7) & ~7;
}

/* the pre-activation values of R outputs of one column from their input rows a[r] and the weight column wc [Kp]:
 * K blocks, fp16 chains, fp32 flushes, bias (the R chains are independent: computed side by side for speed) */
#define GEMM_R 4
static void gemm_pre(const h16 *const *a, int R, const h16 *wc, float b32, h16 b16, int Kp, h16 *v) {
  int nblk, bs;
  kblocks(Kp, &nblk, &bs);
  float fb[GEMM_R] = {0.f, 0.f, 0.f, 0.f};
  h16 cb[GEMM_R] = {0, 0, 0, 0};
  for (int kb = 0; kb < Kp; kb += bs) {
    const int kn = Kp - kb < bs ? Kp - kb : bs;
    for (int r = 0; r < GEMM_R; r++) cb[r] = 0;
    if (R == GEMM_R)
      for (int k = kb; k < kb + kn; k++) {
        const h16 wk = wc[k];
        for (int r = 0; r < GEMM_R; r++) cb[r] = bnno_h_fma(wk, a[r][k], cb[r]);
      }
    else
      for (int r = 0; r < R; r++)
        for (int k = kb; k < kb + kn; k++) cb[r] = bnno_h_fma(wc[k], a[r][k], cb[r]);
    if (nblk > 1)
      for (int r = 0; r < R; r++) fb[r] = fb[r] + bnno_h2f(cb[r]);
  }
  for (int r = 0; r < R; r++) v[r] = nblk > 1 ? bnno_f2h(fb[r] + b32) : bnno_h_add(cb[r], b16);
}

void bnno_gemm_f16(const h16 *A, int lda, int M, const h16 *w, const float *b32, const h16 *b16, int Kp, int Np,
                   int act, h16 *out, int ldo, int ow, int opad, const h16 *res, int ldr) {
  h16 *wc = malloc(sizeof(h16) * (size_t)Kp);
  if (!wc) return;
  for (int n = 0; n < Np; n++) { /* every output is computed on its own: column by column */
    for (int k = 0; k < Kp; k++) wc[k] = hp_w(w, Kp, Np, n, k);
    for (int m0 = 0; m0 < M; m0 += GEMM_R) {
      const int R = M - m0 < GEMM_R ? M - m0 : GEMM_R;
      const h16 *rows[GEMM_R];
      h16 vv[GEMM_R];
      for (int r = 0; r < R; r++) rows[r] = A + (size_t)(m0 + r) * lda;
      gemm_pre(rows, R, wc, b32[n], b16[n], Kp, vv);
      for (int r = 0; r < R; r++) {
        const int m = m0 + r;
        const size_t orow = opad ? (size_t)((m / ow) + opad) * (ow + 2 * opad) + (m % ow) + opad : (size_t)m;
        h16 v = vv[r];
        if (act == 1) v = bnno_h_silu(v);
        else if (act == 2) v = h_max(v, 0);
        if (res) v = bnno_h_add(v, res[(size_t)m * ldr + n]);
        out[orow * ldo + n] = v;
      }
    }
  }
  free(wc);
}

/* ------------------------------------------------------------------ C0POOL f16 */

void bnno_c0pool_f16(const float *img, const h16 *w, const h16 *b16, h16 *pin) {
  const int PW_ = 518, PH = 98;
  h16 *im = calloc((size_t)PH * PW_ * 2, sizeof(h16));
  for (int y = 0; y < 96; y++)
    for (int i = 0; i < 511 * 2; i++) im[((size_t)(y + 1) * PW_ + 3) * 2 + i] = bnno_f2h(img[(size_t)y * 511 * 2 + i]);
  h16 v[2][24];
  for (int oy = 0; oy < 48; oy++)
    for (int ox = 0; ox < 256; ox++) {
      for (int n = 0; n < 24; n++) {
        h16 acc = 0;
        for (int ky = 0; ky < 4; ky++) {
          const h16 *r = im + ((size_t)(2 * oy + ky) * PW_ + 2 * ox) * 2;
          for (int j = 0; j < 16; j++) acc = bnno_h_fma(hp_w(w, 64, 24, n, ky * 16 + j), r[j], acc);
        }
        v[ox & 1][n] = bnno_h_add(acc, b16[n]);
      }
      if (ox & 1) {
        h16 *o = pin + ((size_t)oy * 128 + ox / 2) * 48;
        for (int n = 0; n < 24; n++) {
          const h16 a = h_max(v[0][n], 0), b = h_max(v[1][n], 0);
          o[n] = h_max(a, b);
          o[24 + n] = bnno_h_mul(bnno_h_add(a, b), 0x3800 /* 0.5 */);
        }
      }
    }
  free(im);
}

/* ------------------------------------------------------------------ DW3 f16 */

void bnno_dw3_f16(const h16 *xp, int H, int W, int C, int s, int pt, int pl, const h16 *w, const h16 *b, h16 *out,
                  int Ho, int Wo, float *chsum) {
  (void)H;
  const int Wp = W + 2;
  h16 *rs = malloc(sizeof(h16) * (size_t)C);
  for (int c = 0; c < C; c++) chsum[c] = 0.f;
  for (int oy = 0; oy < Ho; oy++) {
    const int iy0 = oy * s - pt + 1;
    for (int c = 0; c < C; c++) rs[c] = 0;
    for (int ox = 0; ox < Wo; ox++) {
      const int ix0 = ox * s - pl + 1;
      const h16 *r0 = xp + ((size_t)iy0 * Wp + ix0) * C, *r1 = r0 + (size_t)Wp * C, *r2 = r1 + (size_t)Wp * C;
      for (int c = 0; c < C; c++) {
        h16 a = bnno_h_fma(r0[c], w[c], b[c]);
        h16 a2 = bnno_h_mul(r0[C + c], w[C + c]);
        a = bnno_h_fma(r0[2 * C + c], w[2 * C + c], a);
        a2 = bnno_h_fma(r1[c], w[3 * C + c], a2);
        a = bnno_h_fma(r1[C + c], w[4 * C + c], a);
        a2 = bnno_h_fma(r1[2 * C + c], w[5 * C + c], a2);
        a = bnno_h_fma(r2[c], w[6 * C + c], a);
        a2 = bnno_h_fma(r2[C + c], w[7 * C + c], a2);
        a = bnno_h_fma(r2[2 * C + c], w[8 * C + c], a);
        const h16 y = bnno_h_silu(bnno_h_add(a, a2));
        out[((size_t)oy * Wo + ox) * C + c] = y;
        rs[c] = bnno_h_add(rs[c], y);
      }
    }
    for (int c = 0; c < C; c++) chsum[c] = chsum[c] + bnno_h2f(rs[c]);
  }
  free(rs);
}

/* ------------------------------------------------------------------ SE f16 */

/* sigm4 (src/v24_fast.c:173-185): 1 / (1 + 2^t), t = -a log2 e clamped to [-126, 126], 2^t as a degree-6 polynomial
 * of the fraction (FMA chain) with the integer part added to the exponent bits */
float bnno_sigm_f16path(float a) {
  float t = a * -1.44269504f;
  t = emu_fmin(emu_fmax(t, -126.f), 126.f);
  const float n = rintf(t), f = t - n;
  float p = 1.5403530e-4f;
  p = fmaf(p, f, 1.3333558e-3f);
  p = fmaf(p, f, 9.6181291e-3f);
  p = fmaf(p, f, 5.5504109e-2f);
  p = fmaf(p, f, 2.4022651e-1f);
  p = fmaf(p, f, 6.9314718e-1f);
  p = fmaf(p, f, 1.f);
  const float e = emu_float(emu_bits(p) + ((uint32_t)emu_cvtzs(n) << 23));
  return 1.f / (1.f + e);
}

void bnno_se_f16(int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                 const float *chsum, int P, h16 *D) {
  float *g = malloc(sizeof(float) * (size_t)C);
  h16 *g16 = malloc(sizeof(h16) * (size_t)C);
  bnno_se_fc(C, rd, w1, b1, w2t, b2, chsum, P, g);
  for (int c = 0; c < C; c++) g16[c] = bnno_f2h(bnno_sigm_f16path(g[c]));
  for (int p = 0; p < P; p++)
    for (int c = 0; c < C; c++) D[(size_t)p * C + c] = bnno_h_mul(D[(size_t)p * C + c], g16[c]);
  free(g);
  free(g16);
}

/* ------------------------------------------------------------------ POSTPC f16, DENSE */

int bnno_postpc_f16(const h16 *X, const float *ps, const float *pb, const h16 *w, const float *b32, const h16 *b16,
                    float *feat) {
  h16 *post = malloc(sizeof(h16) * 24 * 192), *pcin = malloc(sizeof(h16) * 6 * 1728),
      *pcout = malloc(sizeof(h16) * 6 * 1024);
  for (int p = 0; p < 24; p++)
    for (int c = 0; c < 192; c++)
      post[p * 192 + c] = bnno_f2h(emu_fmax(fmaf(bnno_h2f(X[p * 192 + c]), ps[c], pb[c]), 0.f));
  for (int ox = 0; ox < 6; ox++)
    for (int ky = 0; ky < 3; ky++)
      for (int kx = 0; kx < 3; kx++)
        memcpy(pcin + (size_t)ox * 1728 + (ky * 3 + kx) * 192, post + (ky * 8 + ox + kx) * 192, 192 * sizeof(h16));
  bnno_gemm_f16(pcin, 1728, 6, w, b32, b16, 1728, 1024, 2, pcout, 1024, 0, 0, NULL, 0);
  int bad = 0;
  for (int c = 0; c < 1024; c++) {
    float s = 0.f;
    for (int ox = 0; ox < 6; ox++) s = s + bnno_h2f(pcout[ox * 1024 + c]);
    feat[c] = s * (1.f / 6.f);
    if (!(fabsf(feat[c]) <= 3.0e38f)) bad = 1;
  }
  free(post);
  free(pcin);
  free(pcout);
  return bad ? -2 : 0;
}

void bnno_dense_f16(const h16 *W, const float *bias, int N, const float *feat, float *out) {
  h16 x[1024];
  for (int k = 0; k < 1024; k++) x[k] = bnno_f2h(feat[k]);
  const int n4 = N & ~3;
  for (int o = 0; o < N; o++) {
    const h16 *w = W + (size_t)o * 1024;
    if (o < n4) { /* the 4-row path: 8 fp16 lanes per 128-k block, flushed to fp32 lanes */
      float s[8] = {0};
      for (int k0 = 0; k0 < 1024; k0 += 128) {
        h16 a[8] = {0};
        for (int k = k0; k < k0 + 128; k += 8)
          for (int j = 0; j < 8; j++) a[j] = bnno_h_fma(w[k + j], x[k + j], a[j]);
        for (int j = 0; j < 8; j++) s[j] = s[j] + bnno_h2f(a[j]);
      }
      const float v[4] = {s[0] + s[4], s[1] + s[5], s[2] + s[6], s[3] + s[7]};
      out[o] = emu_addv4(v) + bias[o];
    } else { /* the scalar tail: fp32 products and sums, in k order */
      float s = 0.f;
      for (int k = 0; k < 1024; k++) s = s + bnno_h2f(w[k]) * bnno_h2f(x[k]);
      out[o] = s + bias[o];
    }
  }
}

void bnno_dense_f32(const float *W, const float *bias, int N, const float *feat, float *out) {
  for (int o = 0; o < N; o++) {
    const float *w = W + (size_t)o * 1024;
    float a[4] = {0}, c[4] = {0};
    for (int k = 0; k < 1024; k += 8)
      for (int l = 0; l < 4; l++) {
        a[l] = fmaf(w[k + l], feat[k + l], a[l]);
        c[l] = fmaf(w[k + 4 + l], feat[k + 4 + l], c[l]);
      }
    const float v[4] = {a[0] + c[0], a[1] + c[1], a[2] + c[2], a[3] + c[3]};
    out[o] = emu_addv4(v) + bias[o];
  }
}
