/* bnn oracle: a .bnpk package executed on the CPU one window at a time (TEST INFRASTRUCTURE ONLY; see oracle.h).
 *
 * Reads the package format the reference compiler writes (python/bnneon/compiler/pkgfmt.py:1-22) and runs the op
 * list in order (rt_run, src/rt_pkg.c:528-542) with the oracle's per-op restatements. Buffers get memory of their
 * own instead of the reference's shared slots: no op of the v2.4 int8 and fp16 paths reads a value it did not write
 * in the same window (halos are re-zeroed by the producing PW, every other buffer is written in full), so the results
 * are the same. Package validation is minimal here; the product loader does the full checks. */
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

typedef struct { uint32_t dtype, H, W, C, ld, halo, slot, reserved; uint64_t elems; } o_buf;
typedef struct { char name[48]; uint32_t dtype, ndim, dims[4]; uint64_t offset, nbytes, reserved; } o_ten;
typedef struct { int code, nb, nt, ni; const int32_t *b, *t, *p; } o_op;

struct bnno_pkg {
  uint8_t *file;
  size_t size;
  uint32_t n_ten, n_buf, n_ops, in_buf, out_buf, emb_buf;
  const o_ten *ten;
  o_buf *bufd;
  o_op *ops;
  void **buf;
  bnno_fe *fe;
  bnno_logmel **logmel; /* per op: the FE_LOGMEL state (NULL for other ops) */
  bnno_dbimg **dbimg;   /* per op: the FE_DBIMG state (NULL for other ops) */
  int n_classes, emb_dim;
};

static int meta_i64(const uint8_t *m, size_t mbytes, uint32_t n, const char *key, int64_t *v) {
  const uint8_t *q = m, *end = m + mbytes;
  size_t kl = strlen(key);
  for (uint32_t i = 0; i < n && q + 8 <= end; i++) {
    uint16_t h[2];
    uint32_t vl;
    memcpy(h, q, 4);
    memcpy(&vl, q + 4, 4);
    size_t rec = (8 + (size_t)h[0] + vl + 7) & ~(size_t)7;
    if (h[0] == kl && !memcmp(q + 8, key, kl) && h[1] == 1 && vl == 8) { memcpy(v, q + 8 + h[0], 8); return 0; }
    q += rec;
  }
  return -1;
}

/* the natural logarithm of FE_DBIMG in package runs: 0 this host's libm logf (the reference's), 1 correctly rounded */
static int g_log_mode;
void bnno_pkg_set_log_mode(int mode) { g_log_mode = mode; }

static const void *tdata(const bnno_pkg *p, const o_op *op, int i) {
  if (i >= op->nt || op->t[i] < 0 || (uint32_t)op->t[i] >= p->n_ten) return NULL;
  return p->file + p->ten[op->t[i]].offset;
}
static void *bptr(const bnno_pkg *p, const o_op *op, int i) {
  return i >= op->nb || op->b[i] < 0 ? NULL : p->buf[op->b[i]];
}
static const o_buf *bdesc(const bnno_pkg *p, const o_op *op, int i) {
  return i >= op->nb || op->b[i] < 0 ? NULL : &p->bufd[op->b[i]];
}
static size_t dsz(uint32_t dt) { return dt == 1 ? 2 : dt == 2 ? 1 : 4; }

bnno_pkg *bnno_pkg_open(const char *path, const char *path_name, char *err, size_t errlen) {
  FILE *f = fopen(path, "rb");
  if (!f) { snprintf(err, errlen, "cannot open %s", path); return NULL; }
  bnno_pkg *p = calloc(1, sizeof *p);
  fseek(f, 0, SEEK_END);
  p->size = (size_t)ftell(f);
  fseek(f, 0, SEEK_SET);
  p->file = malloc(p->size + 64);
  if (fread(p->file, 1, p->size, f) != p->size) { fclose(f); snprintf(err, errlen, "read failed"); bnno_pkg_close(p); return NULL; }
  fclose(f);
  const uint8_t *m = p->file;
  if (p->size < 64 || memcmp(m, "BNNPKG01", 8)) { snprintf(err, errlen, "not a package"); bnno_pkg_close(p); return NULL; }
  uint32_t cnt[4];
  uint64_t off[4];
  memcpy(cnt, m + 16, 16);
  memcpy(off, m + 32, 32);
  p->n_ten = cnt[1];
  p->ten = (const o_ten *)(m + off[1]);
  int pi = -1;
  for (uint32_t i = 0; i < cnt[2]; i++)
    if (!strncmp((const char *)(m + off[2] + 72 * i), path_name, 24)) { pi = (int)i; break; }
  if (pi < 0) { snprintf(err, errlen, "no path %s", path_name); bnno_pkg_close(p); return NULL; }
  const uint8_t *pd = m + off[2] + 72 * (size_t)pi;
  uint32_t pv[8];
  uint64_t po[2];
  memcpy(pv, pd + 24, 32);
  memcpy(po, pd + 56, 16);
  p->n_buf = pv[1]; p->n_ops = pv[2]; p->in_buf = pv[4]; p->out_buf = pv[5]; p->emb_buf = pv[6];
  p->bufd = malloc(sizeof(o_buf) * p->n_buf);
  memcpy(p->bufd, m + po[0], sizeof(o_buf) * p->n_buf);
  p->ops = calloc(p->n_ops, sizeof(o_op));
  const uint8_t *q = m + po[1];
  for (uint32_t i = 0; i < p->n_ops; i++) {
    uint16_t h[6];
    memcpy(h, q, 12);
    o_op *op = &p->ops[i];
    op->code = h[0]; op->nb = h[2]; op->nt = h[3]; op->ni = h[4];
    op->b = (const int32_t *)(q + 12);
    op->t = op->b + op->nb;
    op->p = op->t + op->nt;
    q += h[1];
  }
  p->buf = calloc(p->n_buf, sizeof(void *));
  for (uint32_t i = 0; i < p->n_buf; i++)
    if (i != p->in_buf) p->buf[i] = calloc(p->bufd[i].elems * dsz(p->bufd[i].dtype) + 64, 1);
  int64_t v;
  p->n_classes = meta_i64(m + off[0], off[1] - off[0], cnt[0], "n_classes", &v) ? 0 : (int)v;
  p->emb_dim = meta_i64(m + off[0], off[1] - off[0], cnt[0], "emb_dim", &v) ? 0 : (int)v;
  p->logmel = calloc(p->n_ops, sizeof(bnno_logmel *));
  p->dbimg = calloc(p->n_ops, sizeof(bnno_dbimg *));
  for (uint32_t i = 0; i < p->n_ops; i++) {
    const o_op *op = &p->ops[i];
    if (op->code == 16) /* FE_DBIMG: t = window, mel, rows, consts; p = 21 ints */
      p->dbimg[i] = bnno_dbimg_new(op->p, tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3));
    if (op->code == 8) { /* FE_LOGMEL: t = window, mel, consts {floor, scale}; p = nsamp frame hop pad nfft nmel */
      const float *k = tdata(p, op, 2);
      p->logmel[i] = bnno_logmel_new(op->p[0], op->p[1], op->p[2], op->p[3], op->p[4], op->p[5], tdata(p, op, 0),
                                     tdata(p, op, 1), k[0], k[1]);
    }
    if ((op->code & 0xff) == 1) { /* FE_STFT2: t = win1 win2 mel1 mel2 pow1 pow2 bn_s bn_b */
      const float *pw1 = tdata(p, op, 4), *pw2 = tdata(p, op, 5);
      p->fe = bnno_fe_new(tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3), pw1[0], pw2[0],
                          tdata(p, op, 6), tdata(p, op, 7));
    }
  }
  return p;
}

void bnno_pkg_close(bnno_pkg *p) {
  if (!p) return;
  if (p->buf)
    for (uint32_t i = 0; i < p->n_buf; i++)
      if (i != p->in_buf) free(p->buf[i]);
  free(p->buf);
  free(p->bufd);
  if (p->logmel)
    for (uint32_t i = 0; i < p->n_ops; i++) bnno_logmel_free(p->logmel[i]);
  free(p->logmel);
  if (p->dbimg)
    for (uint32_t i = 0; i < p->n_ops; i++) bnno_dbimg_free(p->dbimg[i]);
  free(p->dbimg);
  free(p->ops);
  bnno_fe_free(p->fe);
  free(p->file);
  free(p);
}

int bnno_pkg_n_ops(const bnno_pkg *p) { return (int)p->n_ops; }
int bnno_pkg_n_bufs(const bnno_pkg *p) { return (int)p->n_buf; }
int bnno_pkg_op_code(const bnno_pkg *p, int i) { return i >= 0 && (uint32_t)i < p->n_ops ? p->ops[i].code : -1; }
long bnno_pkg_buf_elems(const bnno_pkg *p, int i, int *dtype) {
  if (i < 0 || (uint32_t)i >= p->n_buf) return -1;
  if (dtype) *dtype = (int)p->bufd[i].dtype;
  return (long)p->bufd[i].elems;
}
int bnno_pkg_out_elems(const bnno_pkg *p) { return p->n_classes; }
int bnno_pkg_emb_elems(const bnno_pkg *p) { return p->emb_dim; }

static int run_op(bnno_pkg *p, const o_op *op) {
  const int *P = op->p;
  switch (op->code) {
  case 1: /* FE_STFT2 */
    bnno_fe_run(p->fe, bptr(p, op, 0), bptr(p, op, 1));
    return 0;
  case 2: /* C0POOL */
    bnno_c0pool(bptr(p, op, 0), tdata(p, op, 0), tdata(p, op, 1), bptr(p, op, 1));
    return 0;
  case 22: { /* PW_S8: b = [in, out, res|-1, q, sa, za (, gate)]; p = [N K Kp Np M lda act ldo ow opad ldr] */
    const o_buf *o = bdesc(p, op, 1), *r = bdesc(p, op, 2);
    const float *gate = op->nb == 7 ? bptr(p, op, 6) : NULL;
    bnno_pw_s8(bptr(p, op, 0), P[5], P[4], P[0], P[1], P[2], P[3], gate, tdata(p, op, 0), tdata(p, op, 1),
               tdata(p, op, 2), tdata(p, op, 3), P[6], bptr(p, op, 1), P[7], P[8], P[9], (int)o->H, bptr(p, op, 2),
               P[10], r && r->halo ? (int)r->halo : 0, r && r->halo ? (int)r->W : 0, bptr(p, op, 3), bptr(p, op, 4),
               bptr(p, op, 5));
    return 0;
  }
  case 23: { /* GEMV_S8: b = [x, out, q, sa, za]; p = [N K Kp Np act] */
    int8_t *q = bptr(p, op, 2);
    float *sa = bptr(p, op, 3);
    int32_t *za = bptr(p, op, 4);
    bnno_quant_rows(bptr(p, op, 0), P[1], 1, P[1], P[2], NULL, q, sa, za);
    bnno_s8_gemm(q, sa, za, 1, P[0], P[2], P[3], tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3),
                 P[4], bptr(p, op, 1), P[3], 0, 0, NULL, 0, 0, 0);
    return 0;
  }
  case 4: /* DW3: b = [xp, out, chsum]; p = [H W C s Ho Wo] */
    bnno_dw3(bptr(p, op, 0), P[0], P[1], P[2], P[3], tdata(p, op, 0), tdata(p, op, 1), bptr(p, op, 1), P[4], P[5],
             bptr(p, op, 2));
    return 0;
  case 25: /* SE_GATE: b = [chsum, gate]; p = [C rd P] */
    bnno_se_gate(P[0], P[1], tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3), bptr(p, op, 0), P[2],
                 bptr(p, op, 1));
    return 0;
  case 6: /* POSTPC: b = [X, feat, pcin, pcout] */
    bnno_postpc(bptr(p, op, 0), tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3), bptr(p, op, 1));
    return 0;
  case 16: { /* FE_DBIMG: b = [pcm, img] */
    const bnno_dbimg *f = p->dbimg[op - p->ops];
    if (!f) return -1;
    bnno_dbimg_run(f, bptr(p, op, 0), bptr(p, op, 1), g_log_mode);
    return 0;
  }
  case 8: { /* FE_LOGMEL: b = [pcm, spec] */
    const bnno_logmel *f = p->logmel[op - p->ops];
    if (!f) return -1;
    bnno_logmel_run(f, bptr(p, op, 0), bptr(p, op, 1));
    return 0;
  }
  case 35: { /* PROTO_S8: b = [x, logits, qa, colmax]; t = [qw, sw, n4, cls w, cls b, eps];
             * p = [N K Kp Np P C ld nc ppc] */
    float *sx = malloc(sizeof(float) * (size_t)P[4]);
    if (!sx) return -1;
    const float *eps = tdata(p, op, 5);
    bnno_proto_quant_cells(bptr(p, op, 0), P[4], P[5], P[6], eps[0], bptr(p, op, 2), P[2], sx);
    bnno_proto_colmax(bptr(p, op, 2), P[2], sx, P[4], tdata(p, op, 0), tdata(p, op, 1), P[3], bptr(p, op, 3));
    free(sx);
    return bnno_proto_logits(bptr(p, op, 3), tdata(p, op, 3), tdata(p, op, 4), P[7], P[8], bptr(p, op, 1));
  }
  case 0x102: /* C0POOL f16: b = [img f32, pin f16]; t = [w b32 b16] */
    bnno_c0pool_f16(bptr(p, op, 0), tdata(p, op, 0), tdata(p, op, 2), bptr(p, op, 1));
    return 0;
  case 0x103: /* PW f16: b = [in, out, res|-1]; t = [w b32 b16]; p = [N K Kp Np M lda act ldo ow opad ldr] */
    bnno_gemm_f16(bptr(p, op, 0), P[5], P[4], tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), P[2], P[3], P[6],
                  bptr(p, op, 1), P[7], P[8], P[9], bptr(p, op, 2), P[10]);
    return 0;
  case 0x104: /* DW3 f16: b = [xp, out, chsum]; p = [H W C s Ho Wo pt pl] */
    bnno_dw3_f16(bptr(p, op, 0), P[0], P[1], P[2], P[3], P[6], P[7], tdata(p, op, 0), tdata(p, op, 1), bptr(p, op, 1),
                 P[4], P[5], bptr(p, op, 2));
    return 0;
  case 0x105: /* SE f16: b = [D, chsum]; p = [C rd P] */
    bnno_se_f16(P[0], P[1], tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3), bptr(p, op, 1), P[2],
                bptr(p, op, 0));
    return 0;
  case 0x106: /* POSTPC f16: b = [X, feat, pcin, pcout]; t = [post_s post_b w b32 b16] */
    return bnno_postpc_f16(bptr(p, op, 0), tdata(p, op, 0), tdata(p, op, 1), tdata(p, op, 2), tdata(p, op, 3),
                           tdata(p, op, 4), bptr(p, op, 1));
  case 0x107: /* DENSE f16: b = [feat, out]; t = [w f16 [N][1024], b]; p = [N] */
    bnno_dense_f16(tdata(p, op, 0), tdata(p, op, 1), P[0], bptr(p, op, 0), bptr(p, op, 1));
    return 0;
  case 7: /* DENSE f32 */
    bnno_dense_f32(tdata(p, op, 0), tdata(p, op, 1), P[0], bptr(p, op, 0), bptr(p, op, 1));
    return 0;
  case 0x109: /* STEM f32 -> f16: b = [img, out, col, tmp]; t = [w, b]; p = [N K Kp Np H W Ho Wo k s act ldo opad] */
    bnno_stem_f16(bptr(p, op, 0), P[4], P[5], P[8], P[9], P[6], P[7], tdata(p, op, 0), tdata(p, op, 1), P[0], P[2],
                  P[10], bptr(p, op, 1), P[11], P[12]);
    return 0;
  case 0x10a: /* DWK f16: b = [xp, out, chsum]; t = [w, b]; p = [H W C k s pt pl Ho Wo act] */
    bnno_dwk_f16(bptr(p, op, 0), P[0], P[1], P[2], P[3], P[4], P[5], P[6], tdata(p, op, 0), tdata(p, op, 1), P[9],
                 bptr(p, op, 1), P[7], P[8], bptr(p, op, 2));
    return 0;
  case 0x10b: /* PAD f16: b = [x, xp]; p = [H W C ld h] */
    bnno_pad_f16(bptr(p, op, 0), P[0], P[1], P[2], P[3], P[4], bptr(p, op, 1));
    return 0;
  case 0x10c: /* MEAN f16: b = [x, out f32]; p = [P C ld] */
    bnno_mean_f16(bptr(p, op, 0), P[0], P[1], P[2], bptr(p, op, 1));
    return 0;
  case 0x20d: { /* PROTO, int8 SDOT head of the fp16 path: b = [x f16, logits, qa, colmax];
                 * t = [qw [Np/12][K/4][12][4], sw, cls w, cls b, eps]; p = [N K Np, P C ld nc ppc] */
    float *sx = malloc(sizeof(float) * (size_t)P[3]);
    int8_t *rows = malloc((size_t)P[2] * (size_t)P[1]);
    if (!sx || !rows) { free(sx); free(rows); return -1; }
    const float *eps = tdata(p, op, 4);
    bnno_proto_quant_cells_f16(bptr(p, op, 0), P[3], P[4], P[5], eps[0], bptr(p, op, 2), sx);
    bnno_proto_unpack12(tdata(p, op, 0), P[2], P[1], rows);
    bnno_proto_colmax_rows(bptr(p, op, 2), P[1], sx, P[3], rows, tdata(p, op, 1), P[2], bptr(p, op, 3));
    free(sx);
    free(rows);
    return bnno_proto_logits(bptr(p, op, 3), tdata(p, op, 2), tdata(p, op, 3), P[6], P[7], bptr(p, op, 1));
  }
  default:
    return -1;
  }
}

int bnno_pkg_run_range(bnno_pkg *p, const float *pcm, int op0, int op1) {
  p->buf[p->in_buf] = (void *)pcm;
  for (int i = op0; i < op1 && (uint32_t)i < p->n_ops; i++)
    if (run_op(p, &p->ops[i])) return -(i + 1);
  return 0;
}

int bnno_pkg_run(bnno_pkg *p, const float *pcm, float *out, float *emb) {
  int r = bnno_pkg_run_range(p, pcm, 0, (int)p->n_ops);
  if (r) return r;
  memcpy(out, p->buf[p->out_buf], sizeof(float) * (size_t)p->n_classes);
  if (emb && p->emb_buf != 0xffffffffu) memcpy(emb, p->buf[p->emb_buf], sizeof(float) * (size_t)p->emb_dim);
  return 0;
}

int bnno_pkg_get_buf(const bnno_pkg *p, int i, void *dst, size_t bytes) {
  if (i < 0 || (uint32_t)i >= p->n_buf || !p->buf[i]) return -1;
  size_t have = p->bufd[i].elems * dsz(p->bufd[i].dtype);
  memcpy(dst, p->buf[i], bytes < have ? bytes : have);
  return 0;
}
int bnno_pkg_set_buf(bnno_pkg *p, int i, const void *src, size_t bytes) {
  if (i < 0 || (uint32_t)i >= p->n_buf || (uint32_t)i == p->in_buf) return -1;
  size_t have = p->bufd[i].elems * dsz(p->bufd[i].dtype);
  memcpy(p->buf[i], src, bytes < have ? bytes : have);
  return 0;
}

typedef struct {
  const char *path, *path_name;
  int n, threads, k, ns, nc, ne, rc;
  const float *pcm;
  float *out, *emb;
} many_job;

static void *many_worker(void *a) {
  many_job *j = a;
  char err[256];
  bnno_pkg *p = bnno_pkg_open(j->path, j->path_name, err, sizeof err);
  if (!p) { j->rc = -1; return NULL; }
  for (int w = j->k; w < j->n; w += j->threads)
    if (bnno_pkg_run(p, j->pcm + (size_t)w * j->ns, j->out + (size_t)w * j->nc, j->emb ? j->emb + (size_t)w * j->ne : NULL)) {
      j->rc = -1;
      break;
    }
  bnno_pkg_close(p);
  return NULL;
}

int bnno_pkg_run_many(const char *path, const char *path_name, int n, const float *pcm, float *out, float *emb,
                      int threads) {
  char err[256];
  bnno_pkg *p = bnno_pkg_open(path, path_name, err, sizeof err);
  if (!p) return -1;
  int ns = (int)p->bufd[p->in_buf].elems, nc = p->n_classes, ne = p->emb_dim;
  bnno_pkg_close(p);
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t th[256];
  many_job jobs[256];
  for (int k = 0; k < threads; k++) {
    jobs[k] = (many_job){path, path_name, n, threads, k, ns, nc, ne, 0, pcm, out, emb};
    pthread_create(&th[k], NULL, many_worker, &jobs[k]);
  }
  int rc = 0;
  for (int k = 0; k < threads; k++) {
    pthread_join(th[k], NULL);
    if (jobs[k].rc) rc = -1;
  }
  return rc;
}
