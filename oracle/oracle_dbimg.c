/* CPU restatement of the reference's dB-image front end FE_DBIMG (TEST INFRASTRUCTURE ONLY: the parity oracle; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs load it; the product never does).
 *
 * Follows src/fe_dbimg.c, one frame at a time (the reference's four frames per vector are independent lanes):
 *   fe_db_new (:49-107): twiddles e^{-2 pi i k / NC} (k < NC / 2) and the real-split factors e^{-2 pi i k / N}
 *     (k <= NC) computed in double and rounded once, bit reversal over NC = N / 2, the mel as the nonzero entries of
 *     each row in bin order, [klo, khi) the bins any row uses, ONNX Runtime's half-pixel resize coordinates
 *     (axis_setup :37-47);
 *   fe_db_frames (:142-226): frame t starts at t hop - pad; samples outside [0, nsamp) reflect (padmode 1) or read
 *     zero (src_index :109-115); z[n] = x[2n] w[2n] + i x[2n + 1] w[2n + 1] in bit-reversed order; the radix-2 DIT
 *     of fft4 (:117-133: b w as fms(bi, wi, br wr) and fma(br, wi, bi wr), the products of wr rounded first); the
 *     real split (:195-204) and the power re^2 + im^2 (each square rounded, then added); the mel as one fused
 *     accumulator from +0 in entry order; Clip(floor) (v < floor ? floor : v); ln; up to three scalar ops;
 *   fe_db_image (:229-258): the top-db floor from the fmaxf of every dB value, the selected rows with fmaxf against
 *     it, their fminf / fmaxf, the min/max normalisation with IEEE divisions, the bilinear resize
 *     ((dx2 dy2) r1[x1] + (dx1 dy2) r1[x2] + (dx2 dy1) r2[x1] + (dx1 dy1) r2[x2], left to right, each product
 *     rounded), the two per-channel ops, zero pad channels and a zero halo.
 * The natural logarithm: the reference calls libm logf. log_mode 0 calls this host's logf (the reference build on
 * this host calls the same function); log_mode 1 rounds the double-precision log once to float (correctly rounded,
 * the B200 kernel's choice: glibc's logf is not correctly rounded on 416,909 of the 2^31 - 2^23 positive finite
 * floats, by one unit in the last place). */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

struct bnno_dbimg {
  int nsamp, N, NC, F, hop, pad, padmode, nfr, nmel, R, has_top_db, norm, post[3], Ho, Wo, C, chan[2], ld, halo;
  float floor_, top_db, eps, postv[3];
  float *win, *tw_re, *tw_im, *sp_re, *sp_im, *mel_w, *chv;
  int *rev, *mel_off, *mel_k, *rows, klo, khi;
  int *ry1, *ry2, *rx1, *rx2;
  float *dy1, *dy2, *dx1, *dx2;
};

static void axis_setup(int nin, int nout, int *i1, int *i2, float *d1, float *d2) {
  const float scale = (float)nout / (float)nin;
  for (int o = 0; o < nout; o++) {
    float x = ((float)o + 0.5f) / scale - 0.5f;
    if (x > (float)(nin - 1)) x = (float)(nin - 1);
    if (x < 0.f) x = 0.f;
    const int a = (int)x < nin - 1 ? (int)x : nin - 1;
    const int b = a + 1 < nin - 1 ? a + 1 : nin - 1;
    i1[o] = a;
    i2[o] = b;
    d1[o] = fabsf(x - (float)a);
    d2[o] = fabsf(x - (float)b);
    if (a == b) { d1[o] = 0.5f; d2[o] = 0.5f; }
  }
}

/* p = the record's ints [nsamp N hop pad padmode nfr nmel R has_top_db norm post0 post1 post2 resize Ho Wo C chan0
 * chan1 ld h]; consts = {floor, top_db, eps, postv[3], chan0[C], chan1[C]} (src/rt_ops_f32x.c:15-17) */
bnno_dbimg *bnno_dbimg_new(const int32_t *p, const float *window, const float *mel, const int32_t *rows,
                           const float *consts) {
  bnno_dbimg *f = calloc(1, sizeof *f);
  f->nsamp = p[0]; f->N = p[1]; f->hop = p[2]; f->pad = p[3]; f->padmode = p[4]; f->nfr = p[5]; f->nmel = p[6];
  f->R = p[7]; f->has_top_db = p[8]; f->norm = p[9]; f->post[0] = p[10]; f->post[1] = p[11]; f->post[2] = p[12];
  f->Ho = p[14]; f->Wo = p[15]; f->C = p[16]; f->chan[0] = p[17]; f->chan[1] = p[18]; f->ld = p[19]; f->halo = p[20];
  f->floor_ = consts[0]; f->top_db = consts[1]; f->eps = consts[2];
  for (int u = 0; u < 3; u++) f->postv[u] = consts[3 + u];
  const int N = f->N, NC = N / 2, F = NC + 1;
  f->NC = NC; f->F = F;
  f->win = malloc(sizeof(float) * N);
  memcpy(f->win, window, sizeof(float) * N);
  f->tw_re = malloc(sizeof(float) * (NC / 2 + 1)); f->tw_im = malloc(sizeof(float) * (NC / 2 + 1));
  for (int k = 0; k < NC / 2; k++) {
    const double a = -2 * M_PI * k / NC;
    f->tw_re[k] = (float)cos(a); f->tw_im[k] = (float)sin(a);
  }
  f->sp_re = malloc(sizeof(float) * (NC + 1)); f->sp_im = malloc(sizeof(float) * (NC + 1));
  for (int k = 0; k <= NC; k++) {
    const double a = -2 * M_PI * k / N;
    f->sp_re[k] = (float)cos(a); f->sp_im[k] = (float)sin(a);
  }
  int bits = 0;
  while ((1 << bits) < NC) bits++;
  f->rev = malloc(sizeof(int) * NC);
  for (int i = 0; i < NC; i++) {
    int r = 0;
    for (int b = 0; b < bits; b++) r |= ((i >> b) & 1) << (bits - 1 - b);
    f->rev[i] = r;
  }
  int nnz = 0;
  for (size_t i = 0; i < (size_t)f->nmel * F; i++) nnz += mel[i] != 0.f;
  f->mel_off = malloc(sizeof(int) * (f->nmel + 1));
  f->mel_k = malloc(sizeof(int) * (nnz + 1)); f->mel_w = malloc(sizeof(float) * (nnz + 1));
  int q = 0, klo = F, khi = 0;
  for (int j = 0; j < f->nmel; j++) {
    f->mel_off[j] = q;
    for (int k = 0; k < F; k++) {
      const float w = mel[(size_t)j * F + k];
      if (w != 0.f) {
        f->mel_k[q] = k; f->mel_w[q] = w; q++;
        if (k < klo) klo = k;
        if (k + 1 > khi) khi = k + 1;
      }
    }
  }
  f->mel_off[f->nmel] = q;
  f->klo = klo < khi ? klo : 0;
  f->khi = khi;
  f->rows = malloc(sizeof(int) * f->R);
  for (int r = 0; r < f->R; r++) f->rows[r] = rows[r];
  f->chv = malloc(sizeof(float) * 2 * f->C);
  memcpy(f->chv, consts + 6, sizeof(float) * 2 * f->C);
  f->ry1 = malloc(sizeof(int) * f->Ho); f->ry2 = malloc(sizeof(int) * f->Ho);
  f->dy1 = malloc(sizeof(float) * f->Ho); f->dy2 = malloc(sizeof(float) * f->Ho);
  f->rx1 = malloc(sizeof(int) * f->Wo); f->rx2 = malloc(sizeof(int) * f->Wo);
  f->dx1 = malloc(sizeof(float) * f->Wo); f->dx2 = malloc(sizeof(float) * f->Wo);
  axis_setup(f->R, f->Ho, f->ry1, f->ry2, f->dy1, f->dy2);
  axis_setup(f->nfr, f->Wo, f->rx1, f->rx2, f->dx1, f->dx2);
  return f;
}

void bnno_dbimg_free(bnno_dbimg *f) {
  if (!f) return;
  void *ps[] = {f->win, f->tw_re, f->tw_im, f->sp_re, f->sp_im, f->mel_w, f->chv, f->rev, f->mel_off, f->mel_k,
                f->rows, f->ry1, f->ry2, f->rx1, f->rx2, f->dy1, f->dy2, f->dx1, f->dx2};
  for (size_t i = 0; i < sizeof ps / sizeof *ps; i++) free(ps[i]);
  free(f);
}

float bnno_logf_cr(float x) { return (float)log((double)x); }
void bnno_log_n(const float *x, float *y, long n, int log_mode) {
  for (long i = 0; i < n; i++) y[i] = log_mode ? bnno_logf_cr(x[i]) : logf(x[i]);
}

static float post_op(float v, int code, float c) {
  switch (code) {
  case 1: return v * c;
  case 2: return v / c;
  case 3: return v + c;
  case 4: return v - c;
  default: return v;
  }
}

static int src_index(int i, int n, int mode) {
  if (i >= 0 && i < n) return i;
  if (mode != 1) return -1;
  if (i < 0) i = -i;
  if (i >= n) i = 2 * n - 2 - i;
  return i >= 0 && i < n ? i : -1;
}

/* the dB rows db [nmel][nfr] of one window */
void bnno_dbimg_frames(const bnno_dbimg *f, const float *pcm, float *db, int log_mode) {
  const int NC = f->NC, nfr = f->nfr;
  float *re = malloc(sizeof(float) * NC), *im = malloc(sizeof(float) * NC), *pw = malloc(sizeof(float) * (NC + 1));
  for (int t = 0; t < nfr; t++) {
    const int base = t * f->hop - f->pad;
    for (int n = 0; n < NC; n++) {
      const int i0 = src_index(base + 2 * n, f->nsamp, f->padmode), i1 = src_index(base + 2 * n + 1, f->nsamp, f->padmode);
      re[f->rev[n]] = (i0 < 0 ? 0.f : pcm[i0]) * f->win[2 * n];
      im[f->rev[n]] = (i1 < 0 ? 0.f : pcm[i1]) * f->win[2 * n + 1];
    }
    for (int len = 2, tws = NC / 2; len <= NC; len <<= 1, tws >>= 1) {
      const int h = len / 2;
      for (int i = 0; i < NC; i += len)
        for (int k = 0; k < h; k++) {
          const float wr = f->tw_re[k * tws], wi = f->tw_im[k * tws];
          const float br = re[i + k + h], bi = im[i + k + h];
          const float vr = fmaf(-bi, wi, br * wr), vi = fmaf(br, wi, bi * wr);
          const float ur = re[i + k], ui = im[i + k];
          re[i + k] = ur + vr; im[i + k] = ui + vi;
          re[i + k + h] = ur - vr; im[i + k + h] = ui - vi;
        }
    }
    for (int k = f->klo; k < f->khi; k++) {
      const int k1 = k & (NC - 1), k2 = (NC - k) & (NC - 1);
      const float zr = re[k1], zi = im[k1], cr = re[k2], ci = -im[k2];
      const float er = (zr + cr) * 0.5f, ei = (zi + ci) * 0.5f;
      const float dr = zr - cr, di = zi - ci;
      const float or_ = di * 0.5f, oi = dr * -0.5f;
      const float wr = f->sp_re[k], wi = f->sp_im[k];
      const float xr = er + fmaf(-oi, wi, or_ * wr), xi = ei + fmaf(or_, wi, oi * wr);
      pw[k] = xr * xr + xi * xi;
    }
    for (int j = 0; j < f->nmel; j++) {
      float acc = 0.f;
      for (int q = f->mel_off[j]; q < f->mel_off[j + 1]; q++) acc = fmaf(pw[f->mel_k[q]], f->mel_w[q], acc);
      const float x = acc < f->floor_ ? f->floor_ : acc;
      float y = log_mode ? bnno_logf_cr(x) : logf(x);
      for (int u = 0; u < 3; u++) y = post_op(y, f->post[u], f->postv[u]);
      db[(size_t)j * nfr + t] = y;
    }
  }
  free(re); free(im); free(pw);
}

/* the image of one window from its dB rows: img [(Ho + 2 halo)][(Wo + 2 halo)][ld] */
void bnno_dbimg_image(const bnno_dbimg *f, const float *db, float *img) {
  const int nfr = f->nfr, R = f->R, h = f->halo, ld = f->ld, Wp = f->Wo + 2 * h;
  float *sp = malloc(sizeof(float) * (size_t)R * nfr);
  float fl = -FLT_MAX;
  if (f->has_top_db) {
    float mx = -FLT_MAX;
    for (size_t i = 0; i < (size_t)f->nmel * nfr; i++) mx = fmaxf(mx, db[i]);
    fl = mx - f->top_db;
  }
  float mn = FLT_MAX, mx = -FLT_MAX;
  for (int r = 0; r < R; r++)
    for (int t = 0; t < nfr; t++) {
      const float s = db[(size_t)f->rows[r] * nfr + t];
      const float v = f->has_top_db ? fmaxf(s, fl) : s;
      sp[(size_t)r * nfr + t] = v;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  if (f->norm) {
    const float den = (mx - mn) + f->eps;
    for (size_t i = 0; i < (size_t)R * nfr; i++) sp[i] = f->norm == 2 ? (mx - sp[i]) / den : (sp[i] - mn) / den;
  }
  memset(img, 0, sizeof(float) * (size_t)(f->Ho + 2 * h) * Wp * ld);
  const float *c0 = f->chv, *c1 = f->chv + f->C;
  for (int oy = 0; oy < f->Ho; oy++) {
    const float *r1 = sp + (size_t)f->ry1[oy] * nfr, *r2 = sp + (size_t)f->ry2[oy] * nfr;
    const float dy1 = f->dy1[oy], dy2 = f->dy2[oy];
    float *o = img + ((size_t)(oy + h) * Wp + h) * ld;
    for (int ox = 0; ox < f->Wo; ox++) {
      const int x1 = f->rx1[ox], x2 = f->rx2[ox];
      const float dx1 = f->dx1[ox], dx2 = f->dx2[ox];
      const float v = dx2 * dy2 * r1[x1] + dx1 * dy2 * r1[x2] + dx2 * dy1 * r2[x1] + dx1 * dy1 * r2[x2];
      float *px = o + (size_t)ox * ld;
      for (int c = 0; c < f->C; c++) px[c] = post_op(post_op(v, f->chan[0], c0[c]), f->chan[1], c1[c]);
    }
  }
  free(sp);
}

int bnno_dbimg_frames_count(const bnno_dbimg *f) { return f->nfr; }

void bnno_dbimg_run(const bnno_dbimg *f, const float *pcm, float *img, int log_mode) {
  float *db = malloc(sizeof(float) * (size_t)f->nmel * f->nfr);
  bnno_dbimg_frames(f, pcm, db, log_mode);
  bnno_dbimg_image(f, db, img);
  free(db);
}
