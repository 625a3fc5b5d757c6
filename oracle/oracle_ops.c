/* bnn oracle: the per-op CPU restatement (TEST INFRASTRUCTURE ONLY; see oracle.h). Compiled with
 * -ffp-contract=off: every fused multiply-add below is an explicit fmaf, every other product and sum rounds. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "arm_emu.h"
#include "oracle.h"

/* ------------------------------------------------------------------ elementwise (src/gemm_f32.h:57-145) */

/* silu_f32x4 / SILU_N_F32X4 (src/gemm_f32.h:102-144): x * 1 / (1 + 2^(-x log2 e)), exp2 by the 1.5 * 2^23 split with
 * a degree-5 polynomial (fused), reciprocal FRECPE + one fused FRECPS step */
float bnno_silu(float x) {
  const float magic = 0x1.8p+23f;
  float t = x * -0x1.715476p+0f;
  t = emu_fmin(emu_fmax(t, -60.f), 60.f);
  float tm = t + magic;
  float f = t - (tm - magic);
  float p = fmaf(0x1.5d87fep-10f, f, 0x1.3b2ab6p-7f);
  p = fmaf(p, f, 0x1.c6b08ep-5f);
  p = fmaf(p, f, 0x1.ebfbep-3f);
  p = fmaf(p, f, 0x1.62e43p-1f);
  p = fmaf(p, f, 1.0f);
  uint32_t ni = emu_bits(tm) << 23;
  float d = 1.f + emu_float(emu_bits(p) + ni);
  float r = emu_frecpe(d);
  r = r * emu_frecps(d, r);
  return x * r;
}

/* exp2_f32x4 (src/gemm_f32.h:74-85) */
static float o_exp2(float t) {
  t = emu_fmin(emu_fmax(t, -126.f), 126.f);
  float n = rintf(t), f = t - n;
  float p = 0x1.430912p-13f;
  p = fmaf(p, f, 0x1.5d87fep-10f);
  p = fmaf(p, f, 0x1.3b2ab6p-7f);
  p = fmaf(p, f, 0x1.c6b08ep-5f);
  p = fmaf(p, f, 0x1.ebfbep-3f);
  p = fmaf(p, f, 0x1.62e43p-1f);
  p = fmaf(p, f, 1.f);
  return emu_float(emu_bits(p) + ((uint32_t)emu_cvtzs(n) << 23));
}
/* sigmoid_f32x4 = rcp_f32x4(1 + exp2_f32x4(x * -log2 e)), two fused Newton steps (src/gemm_f32.h:86-96) */
float bnno_sigmoid(float x) {
  float e = o_exp2(x * -0x1.715476p+0f);
  float d = 1.f + e;
  float r = emu_frecpe(d);
  r = r * emu_frecps(d, r);
  r = r * emu_frecps(d, r);
  return r;
}
float bnno_frecpe(float x) { return emu_frecpe(x); }

/* log2_acc_f32x4 (src/gemm_f32.h:57-71) */
float bnno_log2_acc(float x) {
  int32_t xi = (int32_t)emu_bits(x);
  int32_t t = (int32_t)((uint32_t)xi - 0x3f3504f3u);
  int32_t e = t >> 23; /* arithmetic shift (vshrq_n_s32) */
  float z = emu_float((uint32_t)xi - ((uint32_t)e << 23)) - 1.f;
  float p = fmaf(z, 0x1.f0a97ep-4f, -0x1.a6c552p-3f);
  p = fmaf(z, p, 0x1.bcc44cp-3f);
  p = fmaf(z, p, -0x1.e9aef8p-3f);
  p = fmaf(z, p, 0x1.26a67p-2f);
  p = fmaf(z, p, -0x1.7159ccp-2f);
  p = fmaf(z, p, 0x1.ec75e6p-2f);
  p = fmaf(z, p, -0x1.715476p-1f);
  p = fmaf(z, p, 0x1.715474p+0f);
  return fmaf(z, p, (float)e);
}
/* exp2_acc (src/v24_fe.c:109-123): exp2_f32x4 without the upper clamp */
float bnno_exp2_acc(float t) {
  t = emu_fmax(t, -126.f);
  float n = rintf(t), f = t - n;
  float p = 0x1.430912p-13f;
  p = fmaf(p, f, 0x1.5d87fep-10f);
  p = fmaf(p, f, 0x1.3b2ab6p-7f);
  p = fmaf(p, f, 0x1.c6b08ep-5f);
  p = fmaf(p, f, 0x1.ebfbep-3f);
  p = fmaf(p, f, 0x1.62e43p-1f);
  p = fmaf(p, f, 1.f);
  return emu_float(emu_bits(p) + ((uint32_t)emu_cvtzs(n) << 23));
}
float bnno_expf(float x) { return expf(x); }

/* ------------------------------------------------------------------ int8 path (src/gemm_s8n.c) */

/* s8n_quant_rows (src/gemm_s8n.c:15-51) for one row r of K values. The 4-wide min/max part uses NEON FMIN/FMAX
 * (NaN-propagating), the scalar tail fminf/fmaxf; the 8-wide quantization loop FCVTNS, the tail lrintf. */
static void quant_row(const float *r, int K, int Kp, int8_t *o, float *sa, int32_t *za) {
  float lo, hi;
  int k = 0;
  if (K >= 4) {
    float mn[4], mx[4];
    for (int l = 0; l < 4; l++) mn[l] = INFINITY, mx[l] = -INFINITY;
    for (; k + 4 <= K; k += 4)
      for (int l = 0; l < 4; l++) { mn[l] = emu_fmin(mn[l], r[k + l]); mx[l] = emu_fmax(mx[l], r[k + l]); }
    lo = emu_fmin(emu_fmin(mn[0], mn[1]), emu_fmin(mn[2], mn[3]));
    hi = emu_fmax(emu_fmax(mx[0], mx[1]), emu_fmax(mx[2], mx[3]));
  } else {
    lo = INFINITY; hi = -INFINITY;
  }
  for (; k < K; k++) { lo = fminf(lo, r[k]); hi = fmaxf(hi, r[k]); }
  float inv;
  int32_t z;
  if (!(hi - lo > 1e-30f * fmaxf(fabsf(hi), fabsf(lo))) || !(hi - lo > 0.f)) {
    float a = fmaxf(fabsf(hi), 1e-30f);
    inv = 127.f / a; z = 0; *sa = a / 127.f;
  } else {
    inv = 254.f / (hi - lo);
    z = (int32_t)((uint32_t)-127 - (uint32_t)emu_lrintf_i32(lo * inv));
    *sa = (hi - lo) / 254.f;
  }
  *za = z;
  k = 0;
  for (; k + 8 <= K; k += 8)
    for (int l = 0; l < 8; l++) {
      int32_t v = (int32_t)((uint32_t)emu_cvtns(r[k + l] * inv) + (uint32_t)z);
      o[k + l] = (int8_t)(v < -127 ? -127 : v > 127 ? 127 : v);
    }
  for (; k < K; k++) {
    int32_t v = (int32_t)((uint32_t)emu_lrintf_i32(r[k] * inv) + (uint32_t)z);
    o[k] = (int8_t)(v < -127 ? -127 : v > 127 ? 127 : v);
  }
  for (; k < Kp; k++) o[k] = (int8_t)z;
}

void bnno_quant_rows(const float *x, int ld, int M, int K, int Kp, const float *gate, int8_t *q, float *sa, int32_t *za) {
  float *t = gate ? malloc(sizeof(float) * (size_t)K) : NULL;
  for (int m = 0; m < M; m++) {
    const float *r = x + (size_t)m * ld;
    if (gate) { /* s8n_quant_rows_gate (src/gemm_s8n.c:55-63): one product per element, then the same quantizer */
      for (int k = 0; k < K; k++) t[k] = r[k] * gate[k];
      r = t;
    }
    quant_row(r, K, Kp, q + (size_t)m * Kp, sa + m, za + m);
  }
  free(t);
}

static size_t pad_row(int m, int w, int pad) {
  if (!pad) return (size_t)m;
  return (size_t)((m / w) + pad) * (w + 2 * pad) + (m % w) + pad;
}

void bnno_s8_gemm(const int8_t *q, const float *sa, const int32_t *za, int M, int N, int Kp, int Np, const int8_t *w,
                  const float *sw, const int32_t *cs, const float *b, int act, float *out, int ldo, int ow, int opad,
                  const float *res, int ldr, int rpad, int rw) {
  (void)N;
  /* unpack [Np/4][Kp/16][4][16] -> [Np][Kp] */
  int8_t *wt = malloc((size_t)Np * Kp);
  for (int n = 0; n < Np; n++)
    for (int k = 0; k < Kp; k++) wt[(size_t)n * Kp + k] = w[(((size_t)(n / 4) * (Kp / 16) + k / 16) * 4 + n % 4) * 16 + k % 16];
  int32_t *acc = malloc(sizeof(int32_t) * (size_t)Np);
  for (int m = 0; m < M; m++) {
    const int8_t *a = q + (size_t)m * Kp;
    for (int n = 0; n < Np; n++) {
      const int8_t *wr = wt + (size_t)n * Kp;
      int32_t s = 0;
      for (int k = 0; k < Kp; k++) s += (int32_t)a[k] * (int32_t)wr[k];
      acc[n] = s;
    }
    float *o = out + pad_row(m, ow, opad) * ldo;
    const float *rr = res ? res + pad_row(m, rw, rpad) * ldr : NULL;
    for (int n = 0; n < Np; n++) {
      /* deq4 (src/gemm_s8n.c:105-114): int32 wrap, exact conversion to fp32, sw * sa rounded first, mul then add */
      float f = (float)(int32_t)((uint32_t)acc[n] - (uint32_t)cs[n] * (uint32_t)za[m]);
      float y = f * (sw[n] * sa[m]) + b[n];
      if (act == 1) y = bnno_silu(y);
      else if (act == 2) y = emu_fmax(y, 0.f);
      if (rr) y = y + rr[n];
      o[n] = y;
    }
  }
  free(acc);
  free(wt);
}

/* rt_zero_halo (src/rt_pkg.c:194-203) of a [H + 2h][W + 2h][C] fp32 buffer */
static void zero_halo(float *x, int H, int W, int C, int h) {
  size_t rowl = (size_t)(W + 2 * h) * C;
  memset(x, 0, rowl * h * 4);
  memset(x + (size_t)(H + h) * rowl, 0, rowl * h * 4);
  for (int y = h; y < H + h; y++) {
    memset(x + (size_t)y * rowl, 0, (size_t)C * h * 4);
    memset(x + (size_t)y * rowl + (size_t)(W + h) * C, 0, (size_t)C * h * 4);
  }
}

void bnno_pw_s8(const float *x, int lda, int M, int N, int K, int Kp, int Np, const float *gate, const int8_t *w,
                const float *sw, const int32_t *cs, const float *b, int act, float *out, int ldo, int ow, int opad,
                int out_h, const float *res, int ldr, int rpad, int rw, int8_t *q, float *sa, int32_t *za) {
  if (opad) zero_halo(out, out_h, ow, ldo, opad);
  bnno_quant_rows(x, lda, M, K, Kp, gate, q, sa, za);
  bnno_s8_gemm(q, sa, za, M, N, Kp, Np, w, sw, cs, b, act, out, ldo, ow, opad, res, ldr, rpad, rw);
}

/* ------------------------------------------------------------------ depthwise (src/gemm_f32.c:214-440) */

/* per output: three column partial sums (DW_ACC, :221-225), SiLU, channel sums added pixel by pixel in raster order
 * (silu_rows_f32 :303-328, dw_silu_row16 :342-365: both add the pixels one at a time from 0) */
void bnno_dw3(const float *xp, int H, int W, int C, int s, const float *w, const float *b, float *out, int Ho, int Wo,
              float *chsum) {
  (void)H;
  const int Wp = W + 2;
  for (int c = 0; c < C; c++) chsum[c] = 0.f;
  for (int oy = 0; oy < Ho; oy++)
    for (int ox = 0; ox < Wo; ox++) {
      const float *q = xp + ((size_t)(oy * s) * Wp + (size_t)ox * s) * C;
      float *o = out + ((size_t)oy * Wo + ox) * C;
      for (int c = 0; c < C; c++) {
#define X(ky, kx) q[((size_t)(ky) * Wp + (kx)) * C + c]
#define WT(t) w[(size_t)(t) * C + c]
        float acc = fmaf(WT(0), X(0, 0), b[c]);
        float acb = WT(1) * X(0, 1);
        float acd = WT(2) * X(0, 2);
        acc = fmaf(WT(3), X(1, 0), acc);
        acb = fmaf(WT(4), X(1, 1), acb);
        acd = fmaf(WT(5), X(1, 2), acd);
        acc = fmaf(WT(6), X(2, 0), acc);
        acb = fmaf(WT(7), X(2, 1), acb);
        acd = fmaf(WT(8), X(2, 2), acd);
        acc = acc + (acb + acd);
#undef X
#undef WT
        float v = bnno_silu(acc);
        o[c] = v;
        chsum[c] = chsum[c] + v;
      }
    }
}

/* ------------------------------------------------------------------ squeeze-excitation gate */

/* v24k32_se_fc1 (src/v24_f32.c:164-179) then se_gate_range (src/rt_ops_f32.c:272-283) */
/* the SE's two fully connected layers (v24k32_se_fc1, src/v24_f32.c:164-179, and se_gate_range, src/rt_ops_f32.c:
 * 272-283): g [C] before the sigmoid. Shared by SE_GATE and the fp16 path's SE (src/v24_fast.c:188-210). */
void bnno_se_fc(int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2, const float *chsum,
                int P, float *g) {
  float *mean = malloc(sizeof(float) * (size_t)C), *s1 = malloc(sizeof(float) * (size_t)rd);
  const float inv = 1.f / (float)P;
  for (int c = 0; c < C; c++) mean[c] = chsum[c] * inv;
  for (int r = 0; r < rd; r++) {
    const float *wr = w1 + (size_t)r * C;
    float a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
    int c = 0;
    for (; c + 8 <= C; c += 8)
      for (int l = 0; l < 4; l++) {
        a0[l] = fmaf(wr[c + l], mean[c + l], a0[l]);
        a1[l] = fmaf(wr[c + 4 + l], mean[c + 4 + l], a1[l]);
      }
    for (; c < C; c += 4)
      for (int l = 0; l < 4; l++) a0[l] = fmaf(wr[c + l], mean[c + l], a0[l]);
    float v[4];
    for (int l = 0; l < 4; l++) v[l] = a0[l] + a1[l];
    float xr = emu_addv4(v) + b1[r];
    s1[r] = xr / (1.f + expf(-xr)); /* silu_s (src/v24_f32.c:160): libm expf, IEEE division */
  }
  for (int c = 0; c < C; c++) {
    float a = b2[c];
    for (int r = 0; r < rd; r++) a = fmaf(w2t[(size_t)r * C + c], s1[r], a);
    g[c] = a;
  }
  free(mean);
  free(s1);
}

void bnno_se_gate(int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                  const float *chsum, int P, float *gate) {
  bnno_se_fc(C, rd, w1, b1, w2t, b2, chsum, P, gate);
  for (int c = 0; c < C; c++) gate[c] = bnno_sigmoid(gate[c]);
}

/* ------------------------------------------------------------------ c0 conv + pool */

/* v24k32_c0_pool (src/v24_f32.c:139-147): the image in a zero border [98][518][2] (1 row top, 3 columns left); output
 * pixel (oy, ox) = patch rows 2oy..2oy+3, columns 2ox..2ox+7; K = 64 in (ky, kx, ci) order, one accumulator from 0,
 * fused multiply-adds in k order (gemm_f32_kblock.h). Epilogue ACT32_RELU_POOL2 (src/gemm_f32.c:60-70): a = max(u + b,
 * 0), c = max(v + b, 0) for the pixel pair, max(a, c) into channels 0-23 and (a + c) * 0.5 into 24-47. */
void bnno_c0pool(const float *img, const float *w, const float *b, float *pin) {
  const int PW_ = 518, PH = 98;
  float *imgp = calloc((size_t)PH * PW_ * 2 + 64, sizeof(float));
  for (int y = 0; y < 96; y++) memcpy(imgp + ((size_t)(y + 1) * PW_ + 3) * 2, img + (size_t)y * 511 * 2, sizeof(float) * 511 * 2);
  for (int oy = 0; oy < 48; oy++)
    for (int qx = 0; qx < 128; qx++) {
      float acc[2][24];
      for (int pix = 0; pix < 2; pix++) {
        int ox = 2 * qx + pix;
        for (int n = 0; n < 24; n++) {
          float a = 0.f;
          for (int ky = 0; ky < 4; ky++) {
            const float *row = imgp + ((size_t)(2 * oy + ky) * PW_ + 2 * ox) * 2;
            for (int kk = 0; kk < 16; kk++) {
              int k = ky * 16 + kk;
              a = fmaf(w[((size_t)(n / 8) * 64 + k) * 8 + n % 8], row[kk], a);
            }
          }
          acc[pix][n] = a;
        }
      }
      float *o = pin + ((size_t)oy * 128 + qx) * 48;
      for (int n = 0; n < 24; n++) {
        float a = emu_fmax(acc[0][n] + b[n], 0.f), c = emu_fmax(acc[1][n] + b[n], 0.f);
        o[n] = emu_fmax(a, c);
        o[24 + n] = (a + c) * 0.5f;
      }
    }
  free(imgp);
}

/* ------------------------------------------------------------------ post BN + ReLU + pc conv + mean */

/* v24k32_postpc (src/v24_f32.c:245-266) */
void bnno_postpc(const float *X, const float *post_s, const float *post_b, const float *w, const float *b, float *feat) {
  float *post = malloc(sizeof(float) * 24 * 192), *pcin = malloc(sizeof(float) * 6 * 1728);
  for (int p = 0; p < 24; p++)
    for (int c = 0; c < 192; c++) post[p * 192 + c] = emu_fmax(fmaf(X[p * 192 + c], post_s[c], post_b[c]), 0.f);
  for (int ox = 0; ox < 6; ox++)
    for (int ky = 0; ky < 3; ky++)
      for (int kx = 0; kx < 3; kx++)
        memcpy(pcin + (size_t)ox * 1728 + (ky * 3 + kx) * 192, post + (ky * 8 + ox + kx) * 192, 192 * 4);
  for (int n = 0; n < 1024; n++) {
    float s = 0.f;
    for (int ox = 0; ox < 6; ox++) {
      float a = 0.f;
      for (int k = 0; k < 1728; k++) a = fmaf(w[((size_t)(n / 8) * 1728 + k) * 8 + n % 8], pcin[(size_t)ox * 1728 + k], a);
      float y = emu_fmax(a + b[n], 0.f);
      s = s + y;
    }
    feat[n] = s * 0x1.555556p-3f; /* 1.f / 6.f */
  }
  free(post);
  free(pcin);
}

/* ------------------------------------------------------------------ v2.4 front end (src/v24_fe.c, src/fft_tab.h) */

#define FE_NSAMP 144000
#define FE_NFR 511
#define FE_NMEL 96

typedef struct {
  int N, M, hop, lg, klo, khi;
  float *tw_re, *tw_im, *pc, *ps, *win;
  int *rev;
  int mel_off[FE_NMEL + 1];
  int *mel_k;
  float *mel_w;
  float pw2, bn_s, bn_b;
} fe_spec;
struct bnno_fe { fe_spec s[2]; };

static void fe_spec_init(fe_spec *s, int which, const float *win, const float *mel, float pw, float bs, float bb) {
  s->N = which ? 1024 : 2048;
  s->hop = which ? 280 : 278;
  s->M = s->N / 2;
  s->lg = 0;
  while ((1 << s->lg) < s->M) s->lg++;
  int bins = s->N / 2 + 1, lo[FE_NMEL], hi[FE_NMEL];
  /* nz_range (src/rt_ops_f32.c:16-24): first and one-past-last nonzero weight of each mel row */
  for (int j = 0; j < FE_NMEL; j++) {
    const float *f = mel + (size_t)j * bins;
    int l = 0, h = 0;
    for (int k = 0; k < bins; k++)
      if (f[k] != 0.f) { if (h == 0) l = k; h = k + 1; }
    lo[j] = l; hi[j] = h;
  }
  s->klo = bins; s->khi = 0;
  for (int j = 0; j < FE_NMEL; j++)
    if (hi[j] > lo[j]) { if (lo[j] < s->klo) s->klo = lo[j]; if (hi[j] > s->khi) s->khi = hi[j]; }
  /* fft_twiddles (src/fft_tab.h:9-14) and the real-split tables (src/v24_fe.c:63-66): double, rounded once */
  s->tw_re = malloc(sizeof(float) * s->M / 2);
  s->tw_im = malloc(sizeof(float) * s->M / 2);
  for (int k = 0; k < s->M / 2; k++) {
    double a = -2 * M_PI * k / s->M;
    s->tw_re[k] = (float)cos(a); s->tw_im[k] = (float)sin(a);
  }
  s->pc = malloc(sizeof(float) * (s->khi + 1));
  s->ps = malloc(sizeof(float) * (s->khi + 1));
  for (int k = 0; k < s->khi; k++) {
    double a = 2 * M_PI * k / s->N;
    s->pc[k] = (float)cos(a); s->ps[k] = (float)sin(a);
  }
  s->rev = malloc(sizeof(int) * s->M);
  for (int i = 0; i < s->M; i++) {
    int r = 0;
    for (int bt = 0; bt < s->lg; bt++) r |= ((i >> bt) & 1) << (s->lg - 1 - bt);
    s->rev[i] = r;
  }
  s->win = malloc(sizeof(float) * s->N);
  memcpy(s->win, win, sizeof(float) * s->N);
  int nnz = 0;
  for (int j = 0; j < FE_NMEL; j++) nnz += hi[j] - lo[j];
  s->mel_k = malloc(sizeof(int) * (nnz + 1));
  s->mel_w = malloc(sizeof(float) * (nnz + 1));
  nnz = 0;
  for (int j = 0; j < FE_NMEL; j++) {
    s->mel_off[j] = nnz;
    for (int k = lo[j]; k < hi[j]; k++) { s->mel_k[nnz] = k; s->mel_w[nnz] = mel[(size_t)j * bins + k]; nnz++; }
  }
  s->mel_off[FE_NMEL] = nnz;
  s->pw2 = 2.f * pw;
  s->bn_s = bs;
  s->bn_b = bb;
}

bnno_fe *bnno_fe_new(const float *win1, const float *win2, const float *mel1, const float *mel2, float pow1,
                     float pow2, const float bn_s[2], const float bn_b[2]) {
  bnno_fe *f = calloc(1, sizeof *f);
  fe_spec_init(&f->s[0], 0, win1, mel1, pow1, bn_s[0], bn_b[0]);
  fe_spec_init(&f->s[1], 1, win2, mel2, pow2, bn_s[1], bn_b[1]);
  return f;
}
void bnno_fe_free(bnno_fe *f) {
  if (!f) return;
  for (int i = 0; i < 2; i++) {
    fe_spec *s = &f->s[i];
    free(s->tw_re); free(s->tw_im); free(s->pc); free(s->ps); free(s->rev); free(s->win); free(s->mel_k); free(s->mel_w);
  }
  free(f);
}

/* fft_dit_x4 (src/fft_tab.h:25-77) on one transform: the first two levels fused without twiddles, then radix-2^2
 * passes, then a last radix-2 level when log2 M is odd. Complex products as the reference forms them:
 * (x w)_r = fma(-x_i, w_i, x_r w_r), (x w)_i = fma(x_i, w_r, x_r w_i). */
static void fft_dit(float *re, float *im, int M, const float *twr, const float *twi) {
  for (int i = 0; i < M; i += 4) {
    float ar = re[i], ai = im[i], br = re[i + 1], bi = im[i + 1], cr = re[i + 2], ci = im[i + 2], dr = re[i + 3], di = im[i + 3];
    float s0r = ar + br, s0i = ai + bi, d0r = ar - br, d0i = ai - bi;
    float s1r = cr + dr, s1i = ci + di, d1r = cr - dr, d1i = ci - di;
    re[i] = s0r + s1r; im[i] = s0i + s1i;
    re[i + 2] = s0r - s1r; im[i + 2] = s0i - s1i;
    re[i + 1] = d0r + d1i; im[i + 1] = d0i - d1r;
    re[i + 3] = d0r - d1i; im[i + 3] = d0i + d1r;
  }
  int len = 8;
  for (; 2 * len <= M; len <<= 2) {
    int h = len / 2, st1 = M / len, st2 = M / (2 * len);
    for (int i = 0; i < M; i += 2 * len)
      for (int j = 0; j < h; j++) {
        float w1r = twr[j * st1], w1i = twi[j * st1], w2r = twr[j * st2], w2i = twi[j * st2];
        float *pr = re + i + j, *pi = im + i + j;
        float ar = pr[0], ai = pi[0], br = pr[h], bi = pi[h], cr = pr[2 * h], ci = pi[2 * h], dr = pr[3 * h], di = pi[3 * h];
        float tr = fmaf(-bi, w1i, br * w1r), ti = fmaf(bi, w1r, br * w1i);
        float a1r = ar + tr, a1i = ai + ti, b1r = ar - tr, b1i = ai - ti;
        tr = fmaf(-di, w1i, dr * w1r); ti = fmaf(di, w1r, dr * w1i);
        float c1r = cr + tr, c1i = ci + ti, d1r = cr - tr, d1i = ci - ti;
        tr = fmaf(-c1i, w2i, c1r * w2r); ti = fmaf(c1i, w2r, c1r * w2i);
        pr[0] = a1r + tr; pi[0] = a1i + ti;
        pr[2 * h] = a1r - tr; pi[2 * h] = a1i - ti;
        float ur = fmaf(-d1i, w2i, d1r * w2r), ui = fmaf(d1i, w2r, d1r * w2i);
        pr[h] = b1r + ui; pi[h] = b1i - ur;
        pr[3 * h] = b1r - ui; pi[3 * h] = b1i + ur;
      }
  }
  for (; len <= M; len <<= 1) {
    int half = len / 2, step = M / len;
    for (int i = 0; i < M; i += len)
      for (int j = 0; j < half; j++) {
        float wr = twr[j * step], wi = twi[j * step];
        float xr = re[i + j + half], xi = im[i + j + half];
        float vr = fmaf(-xi, wi, xr * wr), vi = fmaf(xi, wr, xr * wi);
        float ur = re[i + j], ui = im[i + j];
        re[i + j] = ur + vr; im[i + j] = ui + vi;
        re[i + j + half] = ur - vr; im[i + j + half] = ui - vi;
      }
  }
}

/* one frame t of one spectrogram (spec_group, src/v24_fe.c:127-190, one lane) -> P[96] */
static void fe_frame(const fe_spec *s, const float *y, int t, float *re, float *im, float *R, float *P) {
  const int M = s->M;
  int st = t * s->hop;
  for (int n = 0; n < M; n++) {
    re[s->rev[n]] = y[st + 2 * n] * s->win[2 * n];
    im[s->rev[n]] = y[st + 2 * n + 1] * s->win[2 * n + 1];
  }
  fft_dit(re, im, M, s->tw_re, s->tw_im);
  /* Re X_k = 1/2 [(Zr_k + Zr_{M-k}) + c (Zi_k + Zi_{M-k}) - s (Zr_k - Zr_{M-k})]. The reference's k = M (Nyquist)
   * would index one past its FFT buffer; here Z_M = Z_0 (the DFT's period), which the v2.4 filter banks never use. */
  for (int k = s->klo; k < s->khi; k++) {
    int k2 = k == 0 ? 0 : M - k, k1 = k == M ? 0 : k;
    float zr = re[k1], zi = im[k1], yr = re[k2], yi = im[k2];
    float v = zr + yr;
    v = fmaf(zi + yi, s->pc[k], v);
    v = fmaf(-(zr - yr), s->ps[k], v);
    R[k] = v * 0.5f;
  }
  for (int j = 0; j < FE_NMEL; j++) {
    float a0 = 0.f, a1 = 0.f;
    int e = s->mel_off[j], e1 = s->mel_off[j + 1];
    for (; e + 2 <= e1; e += 2) {
      a0 = fmaf(R[s->mel_k[e]], s->mel_w[e], a0);
      a1 = fmaf(R[s->mel_k[e + 1]], s->mel_w[e + 1], a1);
    }
    if (e < e1) a0 = fmaf(R[s->mel_k[e]], s->mel_w[e], a0);
    float m = emu_fmax(fabsf(a0 + a1), 1e-30f);
    float l = bnno_log2_acc(m);
    float p = bnno_exp2_acc(s->pw2 * l);
    P[j] = fmaf(p, s->bn_s, s->bn_b);
  }
}

/* ------------------------------------------------------------------ FE_LOGMEL (src/pc_kern_f32.c:14-149) */

struct bnno_logmel {
  int nsamp, frame, hop, pad, nfft, M, lg, nmel, nfr, klo, khi;
  float *win, *tw_re, *tw_im, *pc, *ps;
  int *rev, *mel_off, *mel_k;
  float *mel_w;
  float floor_, scale;
};

/* pc_logmel_new (src/pc_kern_f32.c:28-72): frames nfr = (nsamp + 2 pad - frame) / hop + 1 (C division); the window
 * zero past frame; twiddles and the real-split cos / sin in double, rounded once; the sparse mel as the NONZERO
 * entries of each row in bin order (zeros inside a row are skipped); [klo, khi) the bins any row uses */
bnno_logmel *bnno_logmel_new(int nsamp, int frame, int hop, int pad, int nfft, int nmel, const float *window,
                             const float *mel, float floor_, float scale) {
  if (nfft < 16 || nfft > 2048 || (nfft & (nfft - 1)) || frame > nfft || hop <= 0 || pad < 0 || nmel < 1 || nmel > 512)
    return NULL;
  bnno_logmel *f = calloc(1, sizeof *f);
  f->nsamp = nsamp; f->frame = frame; f->hop = hop; f->pad = pad; f->nfft = nfft; f->M = nfft / 2; f->nmel = nmel;
  f->nfr = (nsamp + 2 * pad - frame) / hop + 1;
  while ((1 << f->lg) < f->M) f->lg++;
  const int bins = nfft / 2 + 1;
  f->klo = bins; f->khi = 0;
  int nnz = 0;
  for (int j = 0; j < nmel; j++)
    for (int k = 0; k < bins; k++)
      if (mel[(size_t)j * bins + k] != 0.f) { nnz++; if (k < f->klo) f->klo = k; if (k + 1 > f->khi) f->khi = k + 1; }
  if (f->khi == 0) f->klo = 0;
  f->win = calloc(nfft, sizeof(float));
  memcpy(f->win, window, sizeof(float) * frame);
  f->tw_re = malloc(sizeof(float) * (f->M / 2 + 1)); f->tw_im = malloc(sizeof(float) * (f->M / 2 + 1));
  for (int k = 0; k < f->M / 2; k++) {
    double a = -2 * M_PI * k / f->M;
    f->tw_re[k] = (float)cos(a); f->tw_im[k] = (float)sin(a);
  }
  f->pc = malloc(sizeof(float) * (f->khi + 1)); f->ps = malloc(sizeof(float) * (f->khi + 1));
  for (int k = 0; k < f->khi; k++) {
    double a = 2 * M_PI * k / nfft;
    f->pc[k] = (float)cos(a); f->ps[k] = (float)sin(a);
  }
  f->rev = malloc(sizeof(int) * f->M);
  for (int i = 0; i < f->M; i++) {
    int r = 0;
    for (int bt = 0; bt < f->lg; bt++) r |= ((i >> bt) & 1) << (f->lg - 1 - bt);
    f->rev[i] = r;
  }
  f->mel_off = malloc(sizeof(int) * (nmel + 1));
  f->mel_k = malloc(sizeof(int) * (nnz + 1)); f->mel_w = malloc(sizeof(float) * (nnz + 1));
  nnz = 0;
  for (int j = 0; j < nmel; j++) {
    f->mel_off[j] = nnz;
    for (int k = 0; k < bins; k++)
      if (mel[(size_t)j * bins + k] != 0.f) { f->mel_k[nnz] = k; f->mel_w[nnz] = mel[(size_t)j * bins + k]; nnz++; }
  }
  f->mel_off[nmel] = nnz;
  f->floor_ = floor_; f->scale = scale;
  return f;
}
int bnno_logmel_frames(const bnno_logmel *f) { return f->nfr; }
void bnno_logmel_free(bnno_logmel *f) {
  if (!f) return;
  free(f->win); free(f->tw_re); free(f->tw_im); free(f->pc); free(f->ps); free(f->rev); free(f->mel_off);
  free(f->mel_k); free(f->mel_w); free(f);
}

/* pc_logmel_run / group (src/pc_kern_f32.c:85-149), one frame at a time: y = pad zeros, pcm, zeros;
 * z[n] = w[2n] y[st + 2n] + i w[2n + 1] y[st + 2n + 1] for n < (frame + 1) / 2, else 0, in bit-reversed order; the
 * DIT transform; |X_k| = sqrt(Xr Xr + Xi Xi) (the square of Xr rounded, Xi Xi fused) from the real split
 * Xr = fma(Oi, s, fma(Or, c, Er)), Xi = fma(-Or, s, fma(Oi, c, Ei)) with E = (A + B) / 2, O = (A - B) / (2i),
 * A = Z_k, B = conj Z_{M-k}; mel over the nonzero weights with two alternating fused accumulators;
 * spec = (log2_acc(max(a0 + a1, floor)) * 0.69314718) * scale (FMAX NaN-propagating). spec [nfr][nmel]. */
void bnno_logmel_run(const bnno_logmel *f, const float *pcm, float *spec) {
  const int M = f->M, nz = (f->frame + 1) / 2;
  const size_t ylen = (size_t)(f->nfr > 0 ? f->nfr - 1 : 0) * f->hop + f->nfft + (size_t)f->nsamp + 2 * f->pad + 64;
  float *y = calloc(ylen, sizeof(float));
  memcpy(y + f->pad, pcm, sizeof(float) * f->nsamp);
  float *re = malloc(sizeof(float) * M), *im = malloc(sizeof(float) * M), *mag = malloc(sizeof(float) * (M + 2));
  for (int t = 0; t < f->nfr; t++) {
    const int st = t * f->hop;
    for (int n = 0; n < M; n++) {
      if (n >= nz) { re[f->rev[n]] = 0.f; im[f->rev[n]] = 0.f; continue; }
      re[f->rev[n]] = y[st + 2 * n] * f->win[2 * n];
      im[f->rev[n]] = y[st + 2 * n + 1] * f->win[2 * n + 1];
    }
    fft_dit(re, im, M, f->tw_re, f->tw_im);
    for (int k = f->klo; k < f->khi; k++) {
      const int k2 = (k == 0 || k == M) ? 0 : M - k, ka = k == M ? 0 : k;
      const float Ar = re[ka], Ai = im[ka], Br = re[k2], Bi = -im[k2];
      const float Er = (Ar + Br) * 0.5f, Ei = (Ai + Bi) * 0.5f;
      const float Or = (Ai - Bi) * 0.5f, Oi = (Br - Ar) * 0.5f;
      const float c = f->pc[k], s = f->ps[k];
      const float Xr = fmaf(Oi, s, fmaf(Or, c, Er));
      const float Xi = fmaf(-Or, s, fmaf(Oi, c, Ei));
      mag[k] = sqrtf(fmaf(Xi, Xi, Xr * Xr));
    }
    for (int j = 0; j < f->nmel; j++) {
      float a0 = 0.f, a1 = 0.f;
      int e = f->mel_off[j], e1 = f->mel_off[j + 1];
      for (; e + 2 <= e1; e += 2) {
        a0 = fmaf(mag[f->mel_k[e]], f->mel_w[e], a0);
        a1 = fmaf(mag[f->mel_k[e + 1]], f->mel_w[e + 1], a1);
      }
      if (e < e1) a0 = fmaf(mag[f->mel_k[e]], f->mel_w[e], a0);
      spec[(size_t)t * f->nmel + j] = (bnno_log2_acc(emu_fmax(a0 + a1, f->floor_)) * 0.69314718f) * f->scale;
    }
  }
  free(y); free(re); free(im); free(mag);
}

/* b24_fe_run (src/v24_fe.c:192-224) */
void bnno_fe_run(const bnno_fe *f, const float *pcm, float *img) {
  float mn = pcm[0], mx = pcm[0];
  float mn4[4], mx4[4];
  for (int l = 0; l < 4; l++) mn4[l] = mx4[l] = pcm[l];
  for (int i = 0; i < FE_NSAMP; i += 4)
    for (int l = 0; l < 4; l++) { mn4[l] = emu_fmin(mn4[l], pcm[i + l]); mx4[l] = emu_fmax(mx4[l], pcm[i + l]); }
  mn = emu_fmin(emu_fmin(mn4[0], mn4[1]), emu_fmin(mn4[2], mn4[3]));
  mx = emu_fmax(emu_fmax(mx4[0], mx4[1]), emu_fmax(mx4[2], mx4[3])) - mn;
  float den = mx + 1e-6f;
  float *y = calloc(FE_NSAMP + 64, sizeof(float));
  for (int i = 0; i < FE_NSAMP; i++) y[i] = ((pcm[i] - mn) / den - 0.5f) * 2.f;
  float *re = malloc(sizeof(float) * 1024), *im = malloc(sizeof(float) * 1024), *R = malloc(sizeof(float) * 1028);
  float P[FE_NMEL];
  for (int b = 0; b < 2; b++)
    for (int t = 0; t < FE_NFR; t++) {
      fe_frame(&f->s[b], y, t, re, im, R, P);
      for (int j = 0; j < FE_NMEL; j++) img[((size_t)(FE_NMEL - 1 - j) * FE_NFR + t) * 2 + b] = P[j];
    }
  free(y); free(re); free(im); free(R);
}
