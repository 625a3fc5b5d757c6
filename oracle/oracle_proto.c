/* bnn oracle: the int8 prototype head PROTO_S8 (TEST INFRASTRUCTURE ONLY; see oracle.h). A plain-C restatement of
 * src/proto_s8n.c and src/pc_kern_f32.c:364-376 with the NEON arithmetic emulated per element (-ffp-contract=off:
 * every fused step below is an explicit fmaf). */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "arm_emu.h"
#include "oracle.h"

/* pc_quant_cells_f32 (src/proto_s8n.c:28-52). Per cell: the sums of squares in two 4-lane fused accumulators over
 * 8-channel steps (lane l of step c holds channel c + l), reduced as vaddvq_f32(s0 + s1) = pairwise; the NaN-propagating
 * maximum of |x| (vmaxq_f32 / vmaxvq_f32); den = sqrtf(sum) + eps; mx = 1e-30 unless mx > 0; sx = mx / (127 den);
 * q = FCVTAS(x * (127 / mx)) narrowed with saturation to int8 (vqmovn twice) and raised to -127; zero past C. */
void bnno_proto_quant_cells(const float *x, int P, int C, int ld, float eps, int8_t *qa, int Kp, float *sx) {
  for (int p = 0; p < P; p++) {
    const float *r = x + (size_t)p * ld;
    float s[8] = {0}, m[8] = {0};
    for (int c = 0; c < C; c += 8)
      for (int l = 0; l < 8; l++) {
        const float u = r[c + l];
        s[l] = fmaf(u, u, s[l]);
        m[l] = emu_fmax(m[l], fabsf(u));
      }
    const float v[4] = {s[0] + s[4], s[1] + s[5], s[2] + s[6], s[3] + s[7]};
    const float den = sqrtf(emu_addv4(v)) + eps;
    float mx = emu_fmax(emu_fmax(emu_fmax(m[0], m[4]), emu_fmax(m[1], m[5])),
                        emu_fmax(emu_fmax(m[2], m[6]), emu_fmax(m[3], m[7])));
    if (!(mx > 0)) mx = 1e-30f;
    sx[p] = mx / (127.f * den);
    const float inv = 127.f / mx;
    int8_t *q = qa + (size_t)p * Kp;
    for (int c = 0; c < C; c++) {
      int32_t i = emu_cvtas(r[c] * inv);
      if (i > 127) i = 127;
      if (i < -127) i = -127; /* saturating narrow to [-128, 127], then vmax_s8 with -127 */
      q[c] = (int8_t)i;
    }
    memset(q + C, 0, (size_t)(Kp - C));
  }
}

/* an IEEE half (fp16 bits) as a float: exact (vcvt_f32_f16); a NaN keeps its payload, quieted */
static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t u;
  if (e == 0x1f) u = sign | 0x7f800000u | (m << 13) | (m ? 0x400000u : 0u);
  else if (e) u = sign | ((e + 112u) << 23) | (m << 13);
  else if (!m) u = sign;
  else { /* subnormal: normalise */
    int sh = 0;
    uint32_t mm = m;
    while (!(mm & 0x400u)) { mm <<= 1; sh++; }
    u = sign | ((uint32_t)(113 - sh) << 23) | ((mm & 0x3ffu) << 13);
  }
  return emu_float(u);
}

/* pc_quant_cells_f16 (src/pc_proto_s8.c:13-45): as the fp32 quantizer on the fp16 cells converted exactly to fp32,
 * but the bytes are only narrowed with saturation (no clamp to -127: an infinite cell value gives -128); rows qa [P][K]
 * (the reference packs them [P/8][K/4][8][4] for SDOT; the bytes are the same) */
void bnno_proto_quant_cells_f16(const uint16_t *x, int P, int C, int ld, float eps, int8_t *qa, float *sx) {
  for (int p = 0; p < P; p++) {
    const uint16_t *r = x + (size_t)p * ld;
    float s[8] = {0}, m[8] = {0};
    for (int c = 0; c < C; c += 8)
      for (int l = 0; l < 8; l++) {
        const float u = half_to_float(r[c + l]);
        s[l] = fmaf(u, u, s[l]);
        m[l] = emu_fmax(m[l], fabsf(u));
      }
    const float v[4] = {s[0] + s[4], s[1] + s[5], s[2] + s[6], s[3] + s[7]};
    const float den = sqrtf(emu_addv4(v)) + eps;
    float mx = emu_fmax(emu_fmax(emu_fmax(m[0], m[4]), emu_fmax(m[1], m[5])),
                        emu_fmax(emu_fmax(m[2], m[6]), emu_fmax(m[3], m[7])));
    if (!(mx > 0)) mx = 1e-30f;
    sx[p] = mx / (127.f * den);
    const float inv = 127.f / mx;
    for (int c = 0; c < C; c++) {
      int32_t i = emu_cvtas(half_to_float(r[c]) * inv);
      if (i > 127) i = 127;
      if (i < -128) i = -128;
      qa[(size_t)p * C + c] = (int8_t)i;
    }
  }
}

/* the SDOT head's prototype panels [Np/12][K/4][12][4] (python/bnneon/compiler/lower.py proto_s8) -> rows [Np][K] */
void bnno_proto_unpack12(const int8_t *qw, int Np, int K, int8_t *rows) {
  for (int j = 0; j < Np; j++)
    for (int k = 0; k < K; k++)
      rows[(size_t)j * K + k] = qw[(((size_t)(j / 12) * (size_t)(K / 4) + (size_t)(k / 4)) * 12 + (size_t)(j % 12)) * 4 + (size_t)(k % 4)];
}

/* the byte of prototype j, channel k in the package layout [Np/4][Kp/16][4][16] (python/bnneon/compiler/lower.py
 * proto_s8n: rows of 4-prototype panels, 16 channels per step) */
static inline int8_t wbyte(const int8_t *qw, int Kp, int j, int k) {
  return qw[(((size_t)(j / 4) * (size_t)(Kp / 16) + (size_t)(k / 16)) * 4 + (size_t)(j % 4)) * 16 + (size_t)(k % 16)];
}

void bnno_proto_unpack(const int8_t *qw, int Np, int Kp, int8_t *rows) {
  for (int j = 0; j < Np; j++)
    for (int k = 0; k < Kp; k++) rows[(size_t)j * Kp + k] = wbyte(qw, Kp, j, k);
}

/* pc_proto_colmax_s8n (src/proto_s8n.c:130-164, tiles :80-108) on unpacked prototype rows [Np][Kp]: exact int32 sums
 * (the n2 and n4 K loops add the same integers), then per prototype j, over the cells in order from -inf:
 * mx = vmaxq(mx, (float)acc * sx[p]) (vcvtq_f32_s32 rounds to nearest even, vmulq_n_f32), colmax[j] = mx * sw[j]. */
void bnno_proto_colmax_rows(const int8_t *qa, int Kp, const float *sx, int P, const int8_t *rows, const float *sw,
                            int Np, float *colmax) {
  for (int j = 0; j < Np; j++) {
    const int8_t *w = rows + (size_t)j * Kp;
    float mx = -INFINITY;
    for (int p = 0; p < P; p++) {
      const int8_t *a = qa + (size_t)p * Kp;
      int32_t acc = 0;
      for (int k = 0; k < Kp; k++) acc += (int32_t)a[k] * (int32_t)w[k];
      mx = emu_fmax(mx, (float)acc * sx[p]);
    }
    colmax[j] = mx * sw[j];
  }
}

void bnno_proto_colmax(const int8_t *qa, int Kp, const float *sx, int P, const int8_t *qw, const float *sw, int Np,
                       float *colmax) {
  int8_t *rows = malloc((size_t)Np * Kp);
  if (!rows) return;
  bnno_proto_unpack(qw, Np, Kp, rows);
  bnno_proto_colmax_rows(qa, Kp, sx, P, rows, sw, Np, colmax);
  free(rows);
}

/* pc_proto_logits (src/pc_kern_f32.c:364-376): per class, s = sum over its ppc prototypes in order of colmax * w
 * (product and sum each rounded), logits = s + b; -2 when a logit is not finite or above 3e38 in magnitude */
int bnno_proto_logits(const float *colmax, const float *w, const float *b, int nc, int ppc, float *logits) {
  int bad = 0;
  for (int c = 0; c < nc; c++) {
    float s = 0.f;
    for (int q = 0; q < ppc; q++) s += colmax[(size_t)c * ppc + q] * w[(size_t)c * ppc + q];
    const float v = s + b[c];
    logits[c] = v;
    bad |= !(fabsf(v) <= 3.0e38f);
  }
  return bad ? -2 : 0;
}

/* pc_proto_n4_check (src/proto_s8n.c:110-128): the first flagged panel with an int16 lane whose 4 weights have
 * sum |w| > 258 (|w| as vabsq_s8 then unsigned: -128 counts 128), -1 if none (or Kp % 32 != 0) */
int bnno_proto_n4_check(const int8_t *qw, int Kp, const uint8_t *n4, int npanels) {
  if (Kp % 32) return -1;
  for (int pn = 0; pn < npanels; pn++) {
    if (!n4[pn]) continue;
    const int8_t *w = qw + (size_t)pn * Kp * 4;
    for (int k = 0; k < Kp; k += 32, w += 128)
      for (int ch = 0; ch < 4; ch++)
        for (int l = 0; l < 8; l++) {
          const int8_t *a = w + 16 * ch, *b = w + 64 + 16 * ch;
          const unsigned s = (uint8_t)abs(a[l]) + (uint8_t)abs(a[l + 8]) + (uint8_t)abs(b[l]) + (uint8_t)abs(b[l + 8]);
          if (s > 258) return pn;
        }
  }
  return -1;
}

/* PROTO_S8 run (src/rt_ops_s8n.c:243-250): quantizer, column maxima, logits of one window */
int bnno_proto_s8(const float *x, int P, int C, int ld, float eps, const int8_t *rows, const float *sw, int Np, int Kp,
                  const float *cls_w, const float *cls_b, int nc, int ppc, int8_t *qa, float *sx, float *colmax,
                  float *logits) {
  bnno_proto_quant_cells(x, P, C, ld, eps, qa, Kp, sx);
  bnno_proto_colmax_rows(qa, Kp, sx, P, rows, sw, Np, colmax);
  return bnno_proto_logits(colmax, cls_w, cls_b, nc, ppc, logits);
}

typedef struct {
  int n, threads, k, P, C, ld, Np, Kp, nc, ppc, rc;
  long long xws;
  float eps;
  const float *x, *sw, *cls_w, *cls_b;
  const int8_t *rows;
  float *logits;
} proto_job;

static void *proto_worker(void *arg) {
  proto_job *j = arg;
  int8_t *qa = malloc((size_t)j->P * j->Kp);
  float *sx = malloc(sizeof(float) * (size_t)j->P), *cm = malloc(sizeof(float) * (size_t)j->Np);
  if (!qa || !sx || !cm) { j->rc = -1; free(qa); free(sx); free(cm); return NULL; }
  for (int w = j->k; w < j->n; w += j->threads)
    if (bnno_proto_s8(j->x + (size_t)w * j->xws, j->P, j->C, j->ld, j->eps, j->rows, j->sw, j->Np, j->Kp, j->cls_w,
                      j->cls_b, j->nc, j->ppc, qa, sx, cm, j->logits + (size_t)w * j->nc))
      j->rc = -2;
  free(qa); free(sx); free(cm);
  return NULL;
}

/* n windows (x at window stride xws floats) on `threads` threads, each window independent: logits [n][nc]; -2 if any
 * window's logits failed the finite check */
int bnno_proto_s8_many(int n, int threads, const float *x, long long xws, int P, int C, int ld, float eps,
                       const int8_t *rows, const float *sw, int Np, int Kp, const float *cls_w, const float *cls_b,
                       int nc, int ppc, float *logits) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t th[256];
  proto_job jobs[256];
  for (int k = 0; k < threads; k++) {
    jobs[k] = (proto_job){n, threads, k, P, C, ld, Np, Kp, nc, ppc, 0, xws, eps, x, sw, cls_w, cls_b, rows, logits};
    pthread_create(&th[k], NULL, proto_worker, &jobs[k]);
  }
  int rc = 0;
  for (int k = 0; k < threads; k++) {
    pthread_join(th[k], NULL);
    if (jobs[k].rc && !rc) rc = jobs[k].rc;
  }
  return rc;
}
