/* bnn oracle, the ops of compiled models' neon-fp16 bodies (Perch v2): a CPU restatement of the reference's kernels
 * (TEST INFRASTRUCTURE ONLY: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it).
 *
 * fp16 arithmetic is the exact-then-round emulation of oracle_f16.c (bnno_h_fma, bnno_h_add, bnno_h_silu); fp32
 * arithmetic is the host's IEEE single precision with fmaf for the fused steps.
 *
 * Ops and their reference sources:
 *   STEM f32 -> f16: src/rt_ops_f16.c:175-190 (rt_stem_f32_tmp, src/rt_ops_f32.c:426-432: pc_im2col1
 *     src/pc_kern_f32.c:151-161, gemm_f32 src/gemm_f32.c:100-132 + src/gemm_f32_kblock.h, then pc_cvt_pad_f16
 *     src/pc_kern_f16.c:104-113 into the zero-haloed output).
 *   DWK f16: pc_dwk_f16_cr, src/pc_kern_f16.c:16-96.
 *   PAD f16: pc_pad_f16, src/pc_kern_f16.c:98-102 (halo zeroed by rt_zero_halo, src/rt_pkg.c:194-202).
 *   MEAN f16: pc_mean_f16, src/pc_kern_f16.c:115-121. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "arm_emu.h"
#include "oracle.h"

typedef uint16_t h16;

/* im2col of the 1-channel image with the taps (ky, kx) in order and zeros up to Kp, one fp32 accumulator per output
 * from +0 over all Kp taps (fused multiply-adds, k ascending), + bias, activation (1 SiLU polynomial, 2 FMAX(x, 0)),
 * rounded to fp16 (nearest even) at the padded position; weights in the fp32 GEMM panels [Np/8][Kp][8] */
void bnno_stem_f16(const float *img, int H, int W, int k, int s, int Ho, int Wo, const float *w, const float *b, int N,
                   int Kp, int act, h16 *out, int ldo, int opad) {
  (void)H;
  float *col = malloc(sizeof(float) * (size_t)Kp);
  if (!col) return;
  for (int oy = 0; oy < Ho; oy++)
    for (int ox = 0; ox < Wo; ox++) {
      int q = 0;
      for (int ky = 0; ky < k; ky++)
        for (int kx = 0; kx < k; kx++) col[q++] = img[(size_t)(oy * s + ky) * W + ox * s + kx];
      for (; q < Kp; q++) col[q] = 0.f;
      h16 *o = out + ((size_t)(oy + opad) * (Wo + 2 * opad) + ox + opad) * ldo;
      for (int n = 0; n < N; n++) {
        const float *wp = w + (size_t)(n / 8) * Kp * 8 + n % 8;
        float acc = 0.f;
        for (int t = 0; t < Kp; t++) acc = fmaf(col[t], wp[(size_t)t * 8], acc);
        float y = acc + b[n];
        if (act == 1) y = bnno_silu(y);
        else if (act == 2) y = emu_fmax(y, 0.f);
        o[n] = bnno_f2h(y);
      }
    }
  free(col);
}

/* depthwise k x k on the input zero-haloed by h = (k - 1) / 2, output pixel (oy, ox) reading rows oy*s - pt + h + ky
 * and columns ox*s - pl + h + kx. Per output row: groups of four pixels (two chains each from the bias and from +0,
 * even taps into the first and odd taps into the second in (ky, kx) order, then one fp16 add), then a pair, then a
 * single pixel (one chain from the bias); activation 1 = the SiLU table; the group's pixels summed in fp16
 * ((v0 + v1) + (v2 + v3), or v0 + v1) and that sum added to the fp32 channel sum */
void bnno_dwk_f16(const h16 *xp, int H, int W, int C, int k, int s, int pt, int pl, const h16 *w, const h16 *b, int act,
                  h16 *out, int Ho, int Wo, float *chsum) {
  (void)H;
  const int h = (k - 1) / 2, Wp = W + 2 * h;
  for (int c = 0; c < C; c++) chsum[c] = 0.f;
  for (int oy = 0; oy < Ho; oy++) {
    int ox = 0;
    while (ox < Wo) {
      const int g = Wo - ox >= 4 ? 4 : Wo - ox >= 2 ? 2 : 1;
      for (int c = 0; c < C; c++) {
        h16 v[4];
        for (int q = 0; q < g; q++) {
          const h16 *x0 = xp + ((size_t)(oy * s - pt + h) * Wp + (size_t)((ox + q) * s - pl + h)) * C + c;
          h16 a = b[c], e = 0;
          int t = 0;
          for (int ky = 0; ky < k; ky++)
            for (int kx = 0; kx < k; kx++, t++) {
              const h16 xv = x0[((size_t)ky * Wp + kx) * C], wv = w[(size_t)(ky * k + kx) * C + c];
              if (g == 4 && (t & 1)) e = bnno_h_fma(xv, wv, e);
              else a = bnno_h_fma(xv, wv, a);
            }
          v[q] = g == 4 ? bnno_h_add(a, e) : a;
          if (act == 1) v[q] = bnno_h_silu(v[q]);
          out[((size_t)oy * Wo + ox + q) * C + c] = v[q];
        }
        h16 sm = g == 4 ? bnno_h_add(bnno_h_add(v[0], v[1]), bnno_h_add(v[2], v[3])) : g == 2 ? bnno_h_add(v[0], v[1]) : v[0];
        chsum[c] += bnno_h2f(sm);
      }
      ox += g;
    }
  }
}

/* a copy of x [H][W] (channel stride ld, C channels) into the zero-haloed xp [H+2h][W+2h][C] */
void bnno_pad_f16(const h16 *x, int H, int W, int C, int ld, int h, h16 *xp) {
  const size_t Wp = (size_t)W + 2 * (size_t)h;
  memset(xp, 0, sizeof(h16) * (size_t)(H + 2 * h) * Wp * C);
  for (int y = 0; y < H; y++)
    for (int xx = 0; xx < W; xx++)
      memcpy(xp + ((size_t)(y + h) * Wp + xx + h) * C, x + ((size_t)y * W + xx) * ld, sizeof(h16) * (size_t)C);
}

/* per channel: the pixels converted to fp32 and summed in pixel order from +0, then one IEEE division by P */
void bnno_mean_f16(const h16 *x, int P, int C, int ld, float *out) {
  for (int c = 0; c < C; c++) {
    float s = 0.f;
    for (int p = 0; p < P; p++) s += bnno_h2f(x[(size_t)p * ld + c]);
    out[c] = s / (float)P;
  }
}
