/* The package runtime on B200: op-list decoding and validation, per-device weights and activation arena, and the
 * launch sequence of one batch.
 *
 * Replaces src/rt_pkg.c:168-542 (executor, arena, registry) and the inits / runs of the registry kernels the v2.4
 * neon-int8 package uses (src/rt_ops_f32.c FE_STFT2 / C0POOL / DW3 / SE_GATE / POSTPC / DENSE, src/rt_ops_s8n.c
 * PW_S8 / GEMV_S8 / PROTO_S8, FE_LOGMEL) and the v2.4 neon-fp16 package uses (src/rt_ops_f16.c C0POOL / PW / DW3 / SE
 * / POSTPC / DENSE). The validation is the reference's: the same records are accepted and refused with the same messages
 * (op index, kernel, source node, expected and found values, hint), so a package that loads on the reference loads
 * here and a bad one fails the same way.
 *
 * Device layout of a context (per GPU, for `batch` windows):
 *  - every package buffer keeps its per-window layout; a batch holds its windows at a fixed window stride;
 *  - buffers with a zero halo (the pw outputs a depthwise conv reads) get memory of their own, zeroed once: no op
 *    writes a halo, so it stays zero and needs no per-window clearing (the reference re-zeroes it in every PW run
 *    because its slot memory is shared, src/rt_ops_s8n.c:125);
 *  - the other buffers share memory by the package's slot plan (the compiler gave a slot's buffers disjoint
 *    lifetimes), scaled by the batch;
 *  - the int8 row buffers of PW_S8 / GEMV_S8 (q, sa, za) are replaced by one device scratch in the GEMM's layout
 *    (rows of Kq = K rounded up to 32 bytes);
 *  - weights are uploaded once per device in the kernels' layouts (int8 [N][Kq] rows for the tensor-core GEMM,
 *    k-major fp32 for the CUDA-core convs). */
#define _GNU_SOURCE
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "bnn_internal.h"

#define R8(x) (((x) + 7) & ~7)
#define R16(x) (((x) + 15) & ~15)
#define R32(x) (((x) + 31) & ~31)

/* ------------------------------------------------------------------ validation (the reference's rt_need* family) */

typedef struct {
  bnn_ctx *c;
  int i;               /* op index */
  const bnn_op *op;
  char *err;
  size_t errlen;
  int set;
} vctx;

static int vbad(vctx *v, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
static int vbad(vctx *v, const char *fmt, ...) {
  if (v->set) return -1;
  char msg[320], src[160] = "", params[160] = "";
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof msg, fmt, ap);
  va_end(ap);
  /* the op's source node: metadata "src_nodes/<path>", one line per op */
  char key[64];
  uint16_t ty;
  uint32_t vl;
  snprintf(key, sizeof key, "src_nodes/%.24s", v->c->path->name);
  const uint8_t *s = bnn_meta_raw(v->c->pkg, key, &ty, &vl);
  if (s && (ty == 0 || ty == 3)) {
    const char *p = (const char *)s, *end = p + vl;
    for (int k = 0; k < v->i && p < end; k++) {
      const char *nl = memchr(p, '\n', (size_t)(end - p));
      p = nl ? nl + 1 : end;
    }
    if (p < end) {
      const char *nl = memchr(p, '\n', (size_t)(end - p));
      size_t l = (size_t)((nl ? nl : end) - p);
      if (l > sizeof src - 1) l = sizeof src - 1;
      memcpy(src, p, l);
      src[l] = 0;
      if (strlen(src) > 96) strcpy(src + 93, "...'");
    }
  }
  size_t k = 0;
  for (int j = 0; j < v->op->ni && k + 16 < sizeof params; j++)
    k += (size_t)snprintf(params + k, sizeof params - k, "%s%d", j ? " " : "", v->op->p[j]);
  char pfx[256];
  if (src[0]) snprintf(pfx, sizeof pfx, "op %d %s (ONNX node %s)", v->i, v->op->kname, src);
  else snprintf(pfx, sizeof pfx, "op %d %s (no source node names in the package: compile with bnc 2 or newer)", v->i,
                v->op->kname);
  int n = snprintf(v->err, v->errlen,
                   "%s: %s; hint: package/library mismatch or a lowering bug: recompile with this checkout's "
                   "compiler/bnc.py; if it reproduces, report this message", pfx, msg);
  if (n > 0 && (size_t)n + 24 < v->errlen && params[0]) snprintf(v->err + n, v->errlen - (size_t)n, " (int params: [%s])", params);
  v->set = 1;
  return -1;
}
#define VREQ(v, cond) do { if (!(cond)) return vbad(v, "parameter check failed: %s", #cond); } while (0)

static const bnn_buf_rec *vbd(vctx *v, int a) {
  return a >= v->op->nb || v->op->b[a] < 0 ? NULL : &v->c->bufd[v->op->b[a]];
}
static size_t dsize(uint32_t dt) { return dt == BNN_F16 ? 2 : dt == BNN_I8 ? 1 : 4; }

static int vneed(vctx *v, int a, int dt, size_t elems) {
  const bnn_buf_rec *d = vbd(v, a);
  if (!d) return vbad(v, "buffer argument %d is absent (the op record has %d buffer arguments)", a, v->op->nb);
  if ((int)d->dtype == dt && d->elems >= elems) return 0;
  return vbad(v, "buffer argument %d (buffer #%d): expected dtype %s with >= %zu elements, found dtype %s [%ux%ux%u ld "
              "%u halo %u] with %llu elements", a, v->op->b[a], bnn_dtype_name((uint32_t)dt), elems,
              bnn_dtype_name(d->dtype), d->H, d->W, d->C, d->ld, d->halo, (unsigned long long)d->elems);
}
static int vneed_haloed(vctx *v, int a, int dt, int H, int W, int ld, int h) {
  if (vneed(v, a, dt, ((size_t)H + 2 * (size_t)h) * ((size_t)W + 2 * (size_t)h) * (size_t)ld)) return -1;
  const bnn_buf_rec *d = vbd(v, a);
  if ((int)d->halo != h || (int)d->ld != ld)
    return vbad(v, "buffer argument %d (buffer #%d): expected halo %d and channel stride %d, found halo %u and stride %u",
                a, v->op->b[a], h, ld, d->halo, d->ld);
  return 0;
}
static int vneed_nohalo(vctx *v, int a, int dt, size_t elems) {
  if (vneed(v, a, dt, elems)) return -1;
  const bnn_buf_rec *d = vbd(v, a);
  if (d->halo) return vbad(v, "buffer argument %d (buffer #%d, input): expected no halo, found halo %u", a, v->op->b[a], d->halo);
  return 0;
}
static const void *vt(vctx *v, int a, size_t *nbytes) {
  if (a >= v->op->nt || v->op->t[a] < 0) return NULL;
  const bnn_tensor_rec *t = &v->c->pkg->tensors[v->op->t[a]];
  if (nbytes) *nbytes = t->nbytes;
  return v->c->pkg->map + t->offset;
}
static int vneed_t(vctx *v, int a, size_t nbytes, int atleast) {
  size_t nb = 0;
  if (!vt(v, a, &nb)) return vbad(v, "tensor argument %d is absent (the op record has %d tensor arguments)", a, v->op->nt);
  if (atleast ? nb >= nbytes : nb == nbytes) return 0;
  const bnn_tensor_rec *t = &v->c->pkg->tensors[v->op->t[a]];
  return vbad(v, "tensor argument %d (tensor #%d '%.48s' %s [%u %u %u %u]): expected %s%zu bytes, found %llu bytes", a,
              v->op->t[a], t->name, bnn_dtype_name(t->dtype), t->dims[0], t->dims[1], t->dims[2], t->dims[3],
              atleast ? ">= " : "", nbytes, (unsigned long long)t->nbytes);
}
static int vneed_args(vctx *v, int nb, int nt, int ni) {
  const bnn_op *op = v->op;
  if ((nb < 0 || op->nb == nb) && (nt < 0 || op->nt == nt) && (ni < 0 || op->ni == ni)) return 0;
  return vbad(v, "op record shape: expected %d buffer, %d tensor and %d int arguments, found %d, %d and %d", nb, nt, ni,
              op->nb, op->nt, op->ni);
}

/* [N K Kp Np] of an int8 GEMM at int params po, tensors w sw cs b at ti (s8_view, src/rt_ops_s8n.c:13-25) */
static int v_s8(vctx *v, int ti, int po) {
  const int *p = v->op->p;
  if (v->op->ni < po + 4) return vbad(v, "int8 GEMM shape [N K Kp Np] expected at int params %d..%d", po, po + 3);
  const int N = p[po], K = p[po + 1], Kp = p[po + 2], Np = p[po + 3];
  if (N <= 0 || K <= 0 || Np != R8(N) || Kp != R16(K))
    return vbad(v, "int8 GEMM shape N %d K %d Kp %d Np %d: expected Np = N rounded up to 8, Kp = K rounded up to 16", N,
                K, Kp, Np);
  if (vneed_t(v, ti, (size_t)Np * Kp, 0) || vneed_t(v, ti + 1, (size_t)Np * 4, 1) || vneed_t(v, ti + 2, (size_t)Np * 4, 1) ||
      vneed_t(v, ti + 3, (size_t)Np * 4, 1))
    return -1;
  return 0;
}
/* fp32 GEMM panels (rt_fpack_view, src/rt_ops_f32.c:49-59) */
static int v_fpack(vctx *v, int ti, int po) {
  const int *p = v->op->p;
  if (v->op->ni < po + 4)
    return vbad(v, "GEMM shape [N K Kp Np] expected at int params %d..%d, the op has %d ints", po, po + 3, v->op->ni);
  const int N = p[po], K = p[po + 1], Kp = p[po + 2], Np = p[po + 3];
  if (N <= 0 || K <= 0 || Np != R8(N) || Kp < K || Kp % 4)
    return vbad(v, "GEMM shape N %d K %d Kp %d Np %d: expected Np = N rounded up to 8, Kp >= K, Kp %% 4 == 0", N, K, Kp, Np);
  return vneed_t(v, ti, (size_t)Np * Kp * 4, 1) || vneed_t(v, ti + 1, (size_t)Np * 4, 1) ? -1 : 0;
}
/* the output of a 1x1 conv (rt_pw_out_check, src/rt_ops_f32.c:115-128) */
static int v_pw_out(vctx *v, int dt) {
  const int *p = v->op->p;
  const int M = p[4], ldo = p[7], ow = p[8], opad = p[9];
  const bnn_buf_rec *o = vbd(v, 1);
  if (!o) return vbad(v, "buffer argument 1 (output) is absent");
  if ((int)o->dtype != dt || o->ld != (uint32_t)ldo || o->halo != (uint32_t)opad)
    return vbad(v, "buffer argument 1 (buffer #%d, output): expected dtype %s ld %d halo %d, found dtype %s ld %u halo %u",
                v->op->b[1], bnn_dtype_name((uint32_t)dt), ldo, opad, bnn_dtype_name(o->dtype), o->ld, o->halo);
  if (!opad) return vneed(v, 1, dt, (size_t)M * ldo);
  VREQ(v, ow > 0 && M % ow == 0);
  if (o->W != (uint32_t)ow || (size_t)o->H * o->W != (size_t)M)
    return vbad(v, "buffer argument 1 (buffer #%d, padded output): expected %d x %d rows, found %u x %u", v->op->b[1],
                M / ow, ow, o->H, o->W);
  return vneed(v, 1, dt, (size_t)(M / ow + 2 * opad) * (ow + 2 * opad) * ldo);
}

static int init_pw_s8(vctx *v) { /* pw8_init, src/rt_ops_s8n.c:94-118 */
  const bnn_op *op = v->op;
  if (vneed_args(v, op->nb == 7 ? 7 : 6, 4, 11) || v_s8(v, 0, 0)) return -1;
  const int *p = op->p;
  const int K = p[1], Np = p[3];
  if (op->nb == 7 && op->b[6] >= 0) {
    VREQ(v, K % 4 == 0 && K <= 4096);
    if (vneed(v, 6, BNN_F32, (size_t)K)) return -1;
  }
  const int M = p[4], lda = p[5], act = p[6], ldo = p[7], opad = p[9], ldr = p[10];
  const size_t M4 = ((size_t)M + 3) & ~(size_t)3;
  VREQ(v, M > 0 && lda >= K && act >= 0 && act <= 2 && ldo >= Np && opad >= 0 && opad <= 3);
  const bnn_buf_rec *r = vbd(v, 2);
  if (vneed_nohalo(v, 0, BNN_F32, (size_t)M * lda) || v_pw_out(v, BNN_F32)) return -1;
  if (r) {
    VREQ(v, ldr >= Np && r->dtype == BNN_F32 && r->ld == (uint32_t)ldr);
    if (r->halo) {
      VREQ(v, (size_t)r->H * r->W == (size_t)M && r->W > 0);
      if (vneed(v, 2, BNN_F32, (size_t)(r->H + 2 * r->halo) * (r->W + 2 * r->halo) * ldr)) return -1;
    } else if (vneed(v, 2, BNN_F32, (size_t)M * ldr))
      return -1;
  }
  return vneed(v, 3, BNN_I8, M4 * p[2]) || vneed(v, 4, BNN_F32, M4) || vneed(v, 5, BNN_I32, M4) ? -1 : 0;
}
static int init_gemv_s8(vctx *v) { /* gemv8_init, src/rt_ops_s8n.c:138-148 */
  if (vneed_args(v, 5, 4, 5) || v_s8(v, 0, 0)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[4] == BNN_ACT_NONE || p[4] == BNN_ACT_RELU);
  return vneed(v, 0, BNN_F32, (size_t)p[1]) || vneed(v, 1, BNN_F32, (size_t)p[3]) || vneed(v, 2, BNN_I8, (size_t)4 * p[2]) ||
                 vneed(v, 3, BNN_F32, 4) || vneed(v, 4, BNN_I32, 4)
             ? -1
             : 0;
}
static int init_dw3(vctx *v) { /* dw3_init + rt_dw3_check, src/rt_ops_f32.c:216-233 */
  if (vneed_args(v, 3, 2, 6)) return -1;
  const int *p = v->op->p;
  const int H = p[0], W = p[1], C = p[2], s = p[3], Ho = p[4], Wo = p[5];
  VREQ(v, H > 0 && W > 0 && Ho > 0 && Wo > 0 && C > 0);
  VREQ(v, C % 8 == 0);
  VREQ(v, s == 1 || s == 2);
  if (vneed_t(v, 0, (size_t)9 * C * 4, 0) || vneed_t(v, 1, (size_t)C * 4, 0)) return -1;
  VREQ(v, (Ho - 1) * s - 1 + 1 + 3 <= H + 2);
  VREQ(v, (Wo - 1) * s - 1 + 1 + 3 <= W + 2);
  if (vneed_haloed(v, 0, BNN_F32, H, W, C, 1)) return -1;
  return vneed(v, 1, BNN_F32, (size_t)Ho * Wo * C) || vneed(v, 2, BNN_F32, (size_t)C) ? -1 : 0;
}
static int init_se_gate(vctx *v) { /* rt_se_check(gate), src/rt_ops_f32.c:256-266 */
  if (vneed_args(v, 2, 4, 3)) return -1;
  const int C = v->op->p[0], rd = v->op->p[1], P = v->op->p[2];
  VREQ(v, C > 0 && C % 8 == 0 && C <= 4096);
  VREQ(v, rd > 0 && rd <= 512);
  VREQ(v, P > 0);
  const size_t want[4] = {(size_t)rd * C, (size_t)rd, (size_t)rd * C, (size_t)C};
  for (int i = 0; i < 4; i++)
    if (vneed_t(v, i, want[i] * 4, 0)) return -1;
  return vneed(v, 0, BNN_F32, (size_t)C) || vneed(v, 1, BNN_F32, (size_t)C) ? -1 : 0;
}
static int init_c0pool(vctx *v) { /* c0_init, src/rt_ops_f32.c:63-72 */
  if (vneed_args(v, 2, 2, 4) || v_fpack(v, 0, 0)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[0] == 24 && p[1] == 64 && p[2] == 64);
  return vneed(v, 0, BNN_F32, (size_t)96 * 511 * 2) || vneed(v, 1, BNN_F32, (size_t)48 * 128 * 48) ? -1 : 0;
}
static int init_postpc(vctx *v) { /* postpc_init + rt_postpc_check, src/rt_ops_f32.c:329-343 */
  if (vneed_args(v, 4, 4, 4) || v_fpack(v, 2, 0)) return -1;
  VREQ(v, v->op->p[0] == 1024 && v->op->p[1] == 1728);
  if (vneed_t(v, 0, 192 * 4, 1) || vneed_t(v, 1, 192 * 4, 1)) return -1;
  return vneed(v, 0, BNN_F32, 24 * 192) || vneed(v, 1, BNN_F32, 1024) || vneed(v, 2, BNN_F32, 8 * 1728) ||
                 vneed(v, 3, BNN_F32, 8 * 1024)
             ? -1
             : 0;
}
static int init_fe_stft2(vctx *v) { /* fe_stft2_init, src/rt_ops_f32.c:25-40 */
  const size_t want[8] = {2048, 1024, (size_t)96 * 1025, (size_t)96 * 513, 1, 1, 2, 2};
  if (vneed_args(v, 2, 8, -1)) return -1;
  for (int i = 0; i < 8; i++)
    if (vneed_t(v, i, want[i] * 4, 0)) return -1;
  return vneed(v, 0, BNN_F32, 144000) || vneed(v, 1, BNN_F32, (size_t)96 * 511 * 2) ? -1 : 0;
}

/* pc_proto_n4_check (src/proto_s8n.c:110-128): the first 4-prototype panel flagged for 4 products per int16 lane in
 * which some lane's 4 weights (bytes l, l + 8 of two consecutive 16-byte steps of one prototype) have sum |w| > 258
 * (|w| as an unsigned byte: -128 counts 128); -1 if none or Kp % 32 != 0 */
int bnn_proto_n4_check(const int8_t *qw, int Kp, const uint8_t *n4, int npanels) {
  if (Kp % 32) return -1;
  for (int pn = 0; pn < npanels; pn++) {
    if (!n4[pn]) continue;
    const int8_t *w = qw + (size_t)pn * Kp * 4;
    for (int k = 0; k < Kp; k += 32, w += 128)
      for (int ch = 0; ch < 4; ch++)
        for (int l = 0; l < 8; l++) {
          const int8_t *a = w + 16 * ch, *b = w + 64 + 16 * ch;
          const unsigned sum = (uint8_t)abs(a[l]) + (uint8_t)abs(a[l + 8]) + (uint8_t)abs(b[l]) + (uint8_t)abs(b[l + 8]);
          if (sum > 258) return pn;
        }
  }
  return -1;
}

static int init_fe_logmel(vctx *v) { /* logmel_init (src/rt_ops_f32.c:364-380) */
  if (vneed_args(v, 2, 3, 6)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[0] > 0 && p[1] > 0 && p[2] > 0 && p[3] >= 0 && p[4] >= p[1] && p[5] > 0);
  if (vneed_t(v, 0, (size_t)p[1] * 4, 0) || vneed_t(v, 1, (size_t)p[5] * (p[4] / 2 + 1) * 4, 0) || vneed_t(v, 2, 8, 0))
    return -1;
  if (vneed(v, 0, BNN_F32, (size_t)p[0]) || vneed(v, 1, BNN_F32, 1)) return -1;
  /* the FFT's limits (pc_kern_f32.c pc_logmel_new): nfft a power of two in 16..2048, frame <= nfft, nmel <= 512 */
  VREQ(v, (p[4] & (p[4] - 1)) == 0 && p[4] >= 16 && p[4] <= 2048); /* nfft */
  VREQ(v, p[1] <= p[4] && p[5] <= 512);                            /* frame, nmel */
  const int nfr = (p[0] + 2 * p[3] - p[1]) / p[2] + 1;
  return vneed(v, 1, BNN_F32, (size_t)nfr * p[5]);
}

static int init_fe_dbimg(vctx *v) { /* fe_db_init (src/rt_ops_f32x.c:18-56), the same checks in the same order */
  if (vneed_args(v, 2, 4, 21)) return -1;
  const int *p = v->op->p;
  const int N = p[1], F = N / 2 + 1, nsamp = p[0], hop = p[2], pad = p[3], padmode = p[4], nfr = p[5], nmel = p[6];
  const int R = p[7], Ho = p[14], Wo = p[15], C = p[16], ld = p[19], h = p[20];
  VREQ(v, N >= 64 && N <= 8192 && (N & (N - 1)) == 0);
  VREQ(v, hop > 0 && pad >= 0 && padmode >= 0 && padmode <= 2 && (padmode || !pad));
  VREQ(v, padmode != 1 || pad < nsamp);
  VREQ(v, nfr > 0 && nfr == (nsamp + 2 * pad - N) / hop + 1 && nsamp + 2 * pad >= N);
  VREQ(v, nmel > 0 && R > 0 && nmel <= 4096);
  VREQ(v, p[8] == 0 || p[8] == 1);
  VREQ(v, p[9] >= 0 && p[9] <= 2);
  VREQ(v, p[10] >= 0 && p[10] <= 4 && p[11] >= 0 && p[11] <= 4 && p[12] >= 0 && p[12] <= 4 && p[13] == 1);
  VREQ(v, Ho > 0 && Wo > 0 && C > 0 && C <= 64 && ld >= C && h >= 0 && h <= 3);
  VREQ(v, p[17] >= 0 && p[17] <= 4 && p[18] >= 0 && p[18] <= 4);
  if (vneed_t(v, 0, (size_t)N * 4, 0) || vneed_t(v, 1, (size_t)nmel * F * 4, 0) || vneed_t(v, 2, (size_t)R * 4, 0) ||
      vneed_t(v, 3, (size_t)(6 + 2 * C) * 4, 0))
    return -1;
  const int32_t *rows = vt(v, 2, NULL);
  for (int r = 0; r < R; r++)
    if (rows[r] < 0 || rows[r] >= nmel) return vbad(v, "row table entry %d = %d outside 0..%d", r, rows[r], nmel - 1);
  if (vneed(v, 0, BNN_F32, (size_t)nsamp)) return -1;
  const bnn_buf_rec *o = vbd(v, 1);
  if (!o) return vbad(v, "buffer argument 1 (image) is absent");
  if (o->halo != (uint32_t)h || o->ld != (uint32_t)ld || o->H != (uint32_t)Ho || o->W != (uint32_t)Wo)
    return vbad(v, "buffer argument 1 (buffer #%d, image): expected %d x %d, ld %d, halo %d; found %u x %u, ld %u, halo %u",
                v->op->b[1], Ho, Wo, ld, h, o->H, o->W, o->ld, o->halo);
  return vneed(v, 1, BNN_F32, (size_t)(Ho + 2 * h) * (Wo + 2 * h) * ld);
}

static int init_proto_s8(vctx *v) { /* proto8n_init (src/rt_ops_s8n.c:220-240) after rt_proto_geom / rt_proto_io
                                     * (src/rt_ops_f32.c:525-545) */
  if (vneed_args(v, 4, 6, 9)) return -1;
  const int *p = v->op->p;
  const int N = p[0], K = p[1], Kp = p[2], Np = p[3], P = p[4], C = p[5], ld = p[6], nc = p[7], ppc = p[8];
  VREQ(v, P > 0 && P <= 65536 && nc > 0 && ppc >= 1);
  VREQ(v, N > 0 && N <= (1 << 26) && K > 0 && K <= (1 << 17));
  VREQ(v, K == C);
  VREQ(v, ld >= C);
  VREQ(v, (size_t)nc * ppc == (size_t)N);
  VREQ(v, C % 8 == 0 && Kp == ((K + 15) & ~15));
  VREQ(v, P % 4 == 0 && Np == ((N + 3) & ~3));
  if (vneed_t(v, 0, (size_t)Np * Kp, 0) || vneed_t(v, 1, (size_t)Np * 4, 1) || vneed_t(v, 2, (size_t)Np / 4, 1))
    return -1;
  if (vneed_t(v, 3, (size_t)N * 4, 0) || vneed_t(v, 4, (size_t)nc * 4, 0) || vneed_t(v, 5, 4, 0)) return -1;
  if (vneed_nohalo(v, 0, BNN_F32, (size_t)P * ld) || vneed(v, 1, BNN_F32, (size_t)nc)) return -1;
  if (vneed(v, 2, BNN_I8, (size_t)P * Kp) || vneed(v, 3, BNN_F32, (size_t)Np)) return -1;
  const int bad = bnn_proto_n4_check(vt(v, 0, NULL), Kp, vt(v, 2, NULL), Np / 4);
  if (bad >= 0)
    return vbad(v, "prototype panel %d is flagged for 4 products per int16 lane, but a lane's 4 weights sum to more "
                "than 258 (the sums could wrap)", bad);
  if (P > 256) v->c->launches += 1; /* the chunk maxima */
  return 0;
}

/* ---- the neon-fp16 path (src/rt_ops_f16.c, with the shared checks of src/rt_ops_f32.c) */

/* packed fp16 GEMM weights (hpack_view, src/rt_ops_f16.c:14-27): t = [w (panels), b32, b16], p = [N K Kp Np] at po */
static int v_hpack(vctx *v, int ti, int po) {
  const int *p = v->op->p;
  if (v->op->ni < po + 4)
    return vbad(v, "GEMM shape [N K Kp Np] expected at int params %d..%d, the op has %d ints", po, po + 3, v->op->ni);
  const int N = p[po], K = p[po + 1], Kp = p[po + 2], Np = p[po + 3];
  if (N <= 0 || K <= 0 || Np != R8(N) || Kp < K || Kp % 8)
    return vbad(v, "GEMM shape N %d K %d Kp %d Np %d: expected Np = N rounded up to 8, Kp >= K, Kp %% 8 == 0", N, K, Kp, Np);
  return vneed_t(v, ti, (size_t)Np * Kp * 2, 1) || vneed_t(v, ti + 1, ((size_t)Np + 16) * 4, 1) ||
                 vneed_t(v, ti + 2, ((size_t)Np + 16) * 2, 1)
             ? -1
             : 0;
}
static int init_c0pool_f16(vctx *v) { /* c0_init, src/rt_ops_f16.c:31-42 */
  if (vneed_args(v, 2, 3, 4) || v_hpack(v, 0, 0)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[0] == 24 && p[1] == 64 && p[2] == 64);
  return vneed(v, 0, BNN_F32, (size_t)96 * 511 * 2) || vneed(v, 1, BNN_F16, (size_t)48 * 128 * 48) ? -1 : 0;
}
static int init_pw_f16(vctx *v) { /* pw_init + rt_pw_check, src/rt_ops_f16.c:54-61, src/rt_ops_f32.c:129-150 */
  if (vneed_args(v, 3, 3, 11) || v_hpack(v, 0, 0)) return -1;
  const int *p = v->op->p;
  const int Kp = p[2], Np = p[3], M = p[4], lda = p[5], act = p[6], ldo = p[7], opad = p[9], ldr = p[10];
  VREQ(v, M > 0);
  VREQ(v, lda >= Kp);
  VREQ(v, ldo >= Np);
  VREQ(v, act >= 0 && act <= 2);
  VREQ(v, opad >= 0 && opad <= 3);
  if (vneed(v, 0, BNN_F16, (size_t)R8(M) * lda) || v_pw_out(v, BNN_F16)) return -1;
  const bnn_buf_rec *r = vbd(v, 2);
  if (r) {
    VREQ(v, ldr >= Np);
    if (r->halo)
      return vbad(v, "buffer argument 2 (buffer #%d, residual): halo %u needs an fp32 buffer with ld %d and H x W = %d "
                  "rows, found %s ld %u %ux%u", v->op->b[2], r->halo, ldr, M, bnn_dtype_name(r->dtype), r->ld, r->H, r->W);
    if (vneed(v, 2, BNN_F16, (size_t)M * ldr)) return -1;
  }
  /* this library's GEMM reads 8 fp16 channels and writes 4 at a time (every compiled package's strides qualify) */
  if (lda % 8 || ldo % 4 || (r && ldr % 4))
    return vbad(v, "channel strides lda %d, ldo %d, ldr %d: the B200 fp16 GEMM needs lda a multiple of 8 and ldo, ldr "
                "multiples of 4", lda, ldo, ldr);
  return 0;
}
static int init_dw3_f16(vctx *v) { /* dw3_init + rt_dw3_check, src/rt_ops_f16.c:64-68, src/rt_ops_f32.c:216-230 */
  if (vneed_args(v, 3, 2, 8)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[2] <= 2048);
  const int H = p[0], W = p[1], C = p[2], s = p[3], Ho = p[4], Wo = p[5], pt = p[6], pl = p[7];
  VREQ(v, H > 0 && W > 0 && Ho > 0 && Wo > 0 && C > 0);
  VREQ(v, C % 8 == 0);
  VREQ(v, s == 1 || s == 2);
  VREQ(v, pt >= 0 && pt <= 1 && pl >= 0 && pl <= 1);
  if (vneed_t(v, 0, (size_t)9 * C * 2, 0) || vneed_t(v, 1, (size_t)C * 2, 0)) return -1;
  VREQ(v, (Ho - 1) * s - pt + 1 + 3 <= H + 2);
  VREQ(v, (Wo - 1) * s - pl + 1 + 3 <= W + 2);
  if (vneed_haloed(v, 0, BNN_F16, H, W, C, 1)) return -1;
  if (vneed(v, 1, BNN_F16, (size_t)Ho * Wo * C) || vneed(v, 2, BNN_F32, (size_t)C)) return -1;
  if (Ho > 12288) return vbad(v, "%d output rows: the B200 fp16 depthwise kernel takes at most 12288", Ho);
  return 0;
}
static int init_se_f16(vctx *v) { /* se_init = rt_se_check(F16), src/rt_ops_f16.c:115, src/rt_ops_f32.c:256-266 */
  if (vneed_args(v, 2, 4, 3)) return -1;
  const int C = v->op->p[0], rd = v->op->p[1], P = v->op->p[2];
  VREQ(v, C > 0 && C % 8 == 0 && C <= 4096);
  VREQ(v, rd > 0 && rd <= 512);
  VREQ(v, P > 0);
  const size_t want[4] = {(size_t)rd * C, (size_t)rd, (size_t)rd * C, (size_t)C};
  for (int i = 0; i < 4; i++)
    if (vneed_t(v, i, want[i] * 4, 0)) return -1;
  return vneed(v, 0, BNN_F16, (size_t)P * C) || vneed(v, 1, BNN_F32, (size_t)C) ? -1 : 0;
}
static int init_postpc_f16(vctx *v) { /* postpc_init + rt_postpc_check, src/rt_ops_f16.c:136-143, rt_ops_f32.c:329-336 */
  if (vneed_args(v, 4, 5, 4) || v_hpack(v, 2, 0)) return -1;
  VREQ(v, v->op->p[0] == 1024 && v->op->p[1] == 1728);
  if (vneed_t(v, 0, 192 * 4, 1) || vneed_t(v, 1, 192 * 4, 1)) return -1;
  if (vneed(v, 0, BNN_F16, 24 * 192) || vneed(v, 1, BNN_F32, 1024) || vneed(v, 2, BNN_F16, 8 * 1728) ||
      vneed(v, 3, BNN_F16, 8 * 1024))
    return -1;
  VREQ(v, v->op->p[2] == 1728); /* im2col rows of 1728 (v24k16_postpc): the GEMM's K is the row */
  return 0;
}
static int init_dense(vctx *v, size_t wsize) { /* dense_init, src/rt_ops_f16.c:156-161, src/rt_ops_f32.c:351-356 */
  if (vneed_args(v, 2, 2, 1)) return -1;
  const int N = v->op->p[0];
  VREQ(v, N > 0);
  if (vneed(v, 0, BNN_F32, 1024) || vneed(v, 1, BNN_F32, (size_t)N)) return -1;
  if (vneed_t(v, 0, (size_t)N * 1024 * wsize, 0) || vneed_t(v, 1, (size_t)N * 4, 0)) return -1;
  return 0;
}
static int init_dense_f16(vctx *v) {
  if (init_dense(v, 2)) return -1;
  if (v->op->p[0] % 4) v->c->launches += 1; /* the scalar tail */
  return 0;
}
static int init_dense_f32(vctx *v) { return init_dense(v, 4); }

/* ---- compiled models' fp16 bodies (src/rt_ops_f16.c:175-218, with the shared checks of src/rt_ops_f32.c) */

static int init_stem_f16(vctx *v) { /* stem_init + rt_stem_f32_check, src/rt_ops_f16.c:175-181, src/rt_ops_f32.c:390-408 */
  if (vneed_args(v, 4, -1, -1) || vneed_args(v, -1, 2, 13) || v_fpack(v, 0, 0)) return -1;
  const int *p = v->op->p;
  const int K = p[1], Kp = p[2], Np = p[3], H = p[4], W = p[5], Ho = p[6], Wo = p[7], k = p[8], s = p[9];
  const int ldo = p[11], h = p[12];
  VREQ(v, k >= 1 && s >= 1 && Ho > 0 && Wo > 0);
  VREQ(v, (Ho - 1) * s + k <= H && (Wo - 1) * s + k <= W); /* VALID conv */
  VREQ(v, K == k * k);
  VREQ(v, ldo >= Np);
  VREQ(v, h >= 0 && h <= 3);
  VREQ(v, p[10] >= 0 && p[10] <= 2);
  if (vneed(v, 0, BNN_F32, (size_t)H * W) || vneed(v, 2, BNN_F32, (size_t)R8(Ho * Wo) * Kp)) return -1;
  const bnn_buf_rec *o = vbd(v, 1);
  if (!o) return vbad(v, "buffer argument 1 (output) is absent");
  if (o->halo != (uint32_t)h || o->ld != (uint32_t)ldo || (h && (o->W != (uint32_t)Wo || o->H != (uint32_t)Ho)))
    return vbad(v, "buffer argument 1 (buffer #%d, output): expected %d x %d, halo %d, ld %d; found %u x %u, halo %u, ld %u",
                v->op->b[1], Ho, Wo, h, ldo, o->H, o->W, o->halo, o->ld);
  if (vneed(v, 1, (int)o->dtype, (size_t)(Ho + 2 * h) * (Wo + 2 * h) * ldo) || vneed(v, 1, BNN_F16, 1)) return -1;
  if (vneed(v, 3, BNN_F32, (size_t)Ho * Wo * Np)) return -1;
  if (((size_t)Np * Kp + Np) * 4 > 48 * 1024)
    return vbad(v, "stem GEMM %d x %d: the B200 stem kernel keeps the weights in 48 KB of shared memory", Np, Kp);
  return 0;
}
static int init_dwk_f16(vctx *v) { /* dwk_init = rt_dwk_check(2), src/rt_ops_f16.c:192, src/rt_ops_f32.c:435-451 */
  if (vneed_args(v, 3, 2, 10)) return -1;
  const int *p = v->op->p;
  const int H = p[0], W = p[1], C = p[2], k = p[3], s = p[4], pt = p[5], pl = p[6], Ho = p[7], Wo = p[8];
  const int h = (k - 1) / 2;
  VREQ(v, H > 0 && W > 0 && Ho > 0 && Wo > 0 && C > 0);
  VREQ(v, C % 8 == 0);
  VREQ(v, k % 2 == 1 && k >= 1 && k <= 7);
  VREQ(v, s >= 1 && s <= 2);
  VREQ(v, pt >= 0 && pt <= h && pl >= 0 && pl <= h);
  VREQ(v, p[9] >= 0 && p[9] <= 1);
  if (vneed_t(v, 0, (size_t)k * k * C * 2, 0) || vneed_t(v, 1, (size_t)C * 2, 0)) return -1;
  /* the last tap of the last output stays inside the haloed input */
  VREQ(v, (Ho - 1) * s - pt + k <= H + 2 * h - h);
  VREQ(v, (Wo - 1) * s - pl + k <= W + 2 * h - h);
  if (vneed_haloed(v, 0, BNN_F16, H, W, C, h)) return -1;
  if (vneed(v, 1, BNN_F16, (size_t)Ho * Wo * C) || vneed(v, 2, BNN_F32, (size_t)C)) return -1;
  const int groups = Wo / 4 + (Wo % 4 >= 2) + Wo % 2;
  if (groups > 768)
    return vbad(v, "%d output columns (%d pixel groups): the B200 depthwise kernel takes at most 768 groups per row", Wo,
                groups);
  return 0;
}
/* PAD and MEAN of variant 1 take the shared checks as the reference registers them (rt_pad_check, rt_mean_check):
 * sizes are checked in the buffers' own dtypes and the dtype itself is not pinned, while the kernels read 16-bit
 * elements, as pc_pad_f16 / pc_mean_f16 do; the compiler only emits them on fp16 buffers */
static int init_pad(vctx *v) { /* rt_pad_check, src/rt_ops_f32.c:474-492 (pad_f16: src/rt_ops_f16.c:204-208) */
  if (vneed_args(v, 2, -1, 5)) return -1;
  const int *p = v->op->p;
  const bnn_buf_rec *x = vbd(v, 0), *o = vbd(v, 1);
  if (!x || !o) return vbad(v, "buffer argument %d is absent", x ? 1 : 0);
  VREQ(v, p[0] > 0 && p[1] > 0 && p[2] > 0);
  VREQ(v, p[4] >= 1 && p[4] <= 3);
  VREQ(v, p[3] >= p[2]);
  if (x->dtype != o->dtype)
    return vbad(v, "buffer argument 0 (buffer #%d, input) is %s but buffer argument 1 (buffer #%d, output) is %s",
                v->op->b[0], bnn_dtype_name(x->dtype), v->op->b[1], bnn_dtype_name(o->dtype));
  if (x->halo) return vbad(v, "buffer argument 0 (buffer #%d, input): expected no halo, found halo %u", v->op->b[0], x->halo);
  if (o->ld != (uint32_t)p[2] || o->halo != (uint32_t)p[4])
    return vbad(v, "buffer argument 1 (buffer #%d, output): expected ld %d halo %d, found ld %u halo %u", v->op->b[1],
                p[2], p[4], o->ld, o->halo);
  return vneed(v, 0, (int)x->dtype, (size_t)p[0] * p[1] * p[3]) ||
                 vneed(v, 1, (int)o->dtype, (size_t)(p[0] + 2 * p[4]) * (p[1] + 2 * p[4]) * p[2])
             ? -1
             : 0;
}
static int init_mean(vctx *v) { /* rt_mean_check, src/rt_ops_f32.c:501-513 (mean_f16: src/rt_ops_f16.c:210-213) */
  if (vneed_args(v, 2, -1, 3)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[0] > 0 && p[1] > 0);
  VREQ(v, p[1] % 4 == 0);
  VREQ(v, p[2] >= p[1]);
  const bnn_buf_rec *x = vbd(v, 0);
  if (!x) return vbad(v, "buffer argument 0 (input) is absent");
  if (x->halo) return vbad(v, "buffer argument 0 (buffer #%d, input): expected no halo, found halo %u", v->op->b[0], x->halo);
  return vneed(v, 0, (int)x->dtype, (size_t)p[0] * p[2]) || vneed(v, 1, BNN_F32, (size_t)p[1]) ? -1 : 0;
}
/* ---- fp32 bodies beyond v2.4: Perch's STEM / DWK (src/rt_ops_f32.c:387-472) and v3.0's CONVK, GEM, SED, VADD,
 * CONVW (src/rt_ops_f32x.c:88-436); the same checks in the same order, with the reference's messages */

static int init_pw_f32(vctx *v) { /* pw_init + rt_pw_check, src/rt_ops_f32.c:115-165 */
  const bnn_op *op = v->op;
  if (vneed_args(v, op->nb == 4 ? 4 : 3, 2, 11) || v_fpack(v, 0, 0)) return -1;
  const int *p = op->p;
  const int K = p[1], Kp = p[2], Np = p[3], M = p[4], lda = p[5], act = p[6], ldo = p[7], opad = p[9], ldr = p[10];
  if (op->nb == 4 && op->b[3] >= 0) {
    VREQ(v, K == Kp);
    if (vneed(v, 3, BNN_F32, (size_t)K)) return -1;
  }
  VREQ(v, M > 0);
  VREQ(v, lda >= Kp);
  VREQ(v, ldo >= Np);
  VREQ(v, act >= 0 && act <= 2);
  VREQ(v, opad >= 0 && opad <= 3);
  if (vneed(v, 0, BNN_F32, (size_t)R8(M) * lda)) return -1;
  if (v_pw_out(v, BNN_F32)) return -1;
  if (op->b[2] >= 0) {
    VREQ(v, ldr >= Np);
    const bnn_buf_rec *r = vbd(v, 2);
    if (r->halo) {
      if (r->ld != (uint32_t)ldr || (size_t)r->H * r->W != (size_t)M || !r->W)
        return vbad(v, "buffer argument 2 (buffer #%d, residual): halo %u needs an fp32 buffer with ld %d and H x W = "
                    "%d rows, found %s ld %u %ux%u", op->b[2], r->halo, ldr, M, bnn_dtype_name(r->dtype), r->ld, r->H,
                    r->W);
      if (vneed(v, 2, BNN_F32, (size_t)(r->H + 2 * r->halo) * (r->W + 2 * r->halo) * ldr)) return -1;
    } else if (vneed(v, 2, BNN_F32, (size_t)M * ldr))
      return -1;
  }
  if (opad) v->c->launches += 1; /* the zero halo */
  return 0;
}
static int init_stem_f32(vctx *v) { /* stem_init + rt_stem_f32_check, src/rt_ops_f32.c:390-415 */
  if (vneed_args(v, 3, -1, -1) || vneed_args(v, -1, 2, 13) || v_fpack(v, 0, 0)) return -1;
  const int *p = v->op->p;
  const int K = p[1], Kp = p[2], Np = p[3], H = p[4], W = p[5], Ho = p[6], Wo = p[7], k = p[8], s = p[9];
  const int ldo = p[11], h = p[12];
  VREQ(v, k >= 1 && s >= 1 && Ho > 0 && Wo > 0);
  VREQ(v, (Ho - 1) * s + k <= H && (Wo - 1) * s + k <= W); /* VALID conv */
  VREQ(v, K == k * k);
  VREQ(v, ldo >= Np);
  VREQ(v, h >= 0 && h <= 3);
  VREQ(v, p[10] >= 0 && p[10] <= 2);
  if (vneed(v, 0, BNN_F32, (size_t)H * W) || vneed(v, 2, BNN_F32, (size_t)R8(Ho * Wo) * Kp)) return -1;
  const bnn_buf_rec *o = vbd(v, 1);
  if (!o) return vbad(v, "buffer argument 1 (output) is absent");
  if (o->halo != (uint32_t)h || o->ld != (uint32_t)ldo || (h && (o->W != (uint32_t)Wo || o->H != (uint32_t)Ho)))
    return vbad(v, "buffer argument 1 (buffer #%d, output): expected %d x %d, halo %d, ld %d; found %u x %u, halo %u, ld %u",
                v->op->b[1], Ho, Wo, h, ldo, o->H, o->W, o->halo, o->ld);
  if (vneed(v, 1, (int)o->dtype, (size_t)(Ho + 2 * h) * (Wo + 2 * h) * ldo) || vneed(v, 1, BNN_F32, 1)) return -1;
  if (h) v->c->launches += 1; /* the zero halo */
  return 0;
}
static int init_dwk_f32(vctx *v) { /* dwk_init = rt_dwk_check(4), src/rt_ops_f32.c:435-453 */
  if (vneed_args(v, 3, 2, 10)) return -1;
  const int *p = v->op->p;
  const int H = p[0], W = p[1], C = p[2], k = p[3], s = p[4], pt = p[5], pl = p[6], Ho = p[7], Wo = p[8];
  const int h = (k - 1) / 2;
  VREQ(v, H > 0 && W > 0 && Ho > 0 && Wo > 0 && C > 0);
  VREQ(v, C % 8 == 0);
  VREQ(v, k % 2 == 1 && k >= 1 && k <= 7);
  VREQ(v, s >= 1 && s <= 2);
  VREQ(v, pt >= 0 && pt <= h && pl >= 0 && pl <= h);
  VREQ(v, p[9] >= 0 && p[9] <= 1);
  if (vneed_t(v, 0, (size_t)k * k * C * 4, 0) || vneed_t(v, 1, (size_t)C * 4, 0)) return -1;
  VREQ(v, (Ho - 1) * s - pt + k <= H + 2 * h - h);
  VREQ(v, (Wo - 1) * s - pl + k <= W + 2 * h - h);
  if (vneed_haloed(v, 0, BNN_F32, H, W, C, h)) return -1;
  return vneed(v, 1, BNN_F32, (size_t)Ho * Wo * C) || vneed(v, 2, BNN_F32, (size_t)C) ? -1 : 0;
}
static int init_pad_f32(vctx *v) { /* rt_pad_check; the run zeroes the halo and copies */
  return init_pad(v);
}
static int init_convk(vctx *v) { /* convk_init, src/rt_ops_f32x.c:91-129 */
  if (vneed_args(v, 3, 2, 16) || v_fpack(v, 0, 0)) return -1;
  const int *p = v->op->p;
  const int K = p[1], Kp = p[2], Np = p[3], H = p[4], W = p[5], Ho = p[6], Wo = p[7], kh = p[8], kw = p[9], st = p[10];
  const int oy0 = p[11], ox0 = p[12], act = p[13], ldo = p[14], opad = p[15];
  VREQ(v, H > 0 && W > 0 && Ho > 0 && Wo > 0 && kh >= 1 && kh <= 7 && kw >= 1 && kw <= 7 && st >= 1 && st <= 2);
  VREQ(v, act >= 0 && act <= 2 && opad >= 0 && opad <= 3 && oy0 >= 0 && ox0 >= 0);
  const bnn_buf_rec *x = vbd(v, 0), *o = vbd(v, 1);
  if (!x || !o) return vbad(v, "buffer argument %d is absent", x ? 1 : 0);
  const int h = (int)x->halo, ld = (int)x->ld, Wp = W + 2 * h;
  if (x->dtype != BNN_F32 || x->H != (uint32_t)H || x->W != (uint32_t)W || ld % 4)
    return vbad(v, "buffer argument 0 (buffer #%d, input): expected fp32 %d x %d with ld a multiple of 4, found %s %u x %u ld %u",
                v->op->b[0], H, W, bnn_dtype_name(x->dtype), x->H, x->W, x->ld);
  VREQ(v, K == kh * kw * ld && Kp == K);
  VREQ(v, oy0 + (Ho - 1) * st + kh <= H + 2 * h && ox0 + (Wo - 1) * st + kw <= W + 2 * h);
  const size_t last = ((size_t)(oy0 + (Ho - 1) * st + kh - 1) * Wp + ox0 + (size_t)(((Wo + 7) & ~7) - 1) * st + kw) * ld + 4;
  if (vneed(v, 0, BNN_F32, last)) return -1;
  if (o->dtype != BNN_F32 || o->H != (uint32_t)Ho || o->W != (uint32_t)Wo || o->ld != (uint32_t)ldo ||
      o->halo != (uint32_t)opad || ldo < Np)
    return vbad(v, "buffer argument 1 (buffer #%d, output): expected fp32 %d x %d ld %d (>= %d) halo %d, found %s %u x %u ld %u halo %u",
                v->op->b[1], Ho, Wo, ldo, Np, opad, bnn_dtype_name(o->dtype), o->H, o->W, o->ld, o->halo);
  if (vneed(v, 1, BNN_F32, (size_t)(Ho + 2 * opad) * (Wo + 2 * opad) * ldo)) return -1;
  const bnn_buf_rec *r = vbd(v, 2);
  if (r) {
    if (r->dtype != BNN_F32 || r->H != (uint32_t)Ho || r->W != (uint32_t)Wo || r->ld < (uint32_t)Np)
      return vbad(v, "buffer argument 2 (buffer #%d, residual): expected fp32 %d x %d with ld >= %d, found %s %u x %u ld %u",
                  v->op->b[2], Ho, Wo, Np, bnn_dtype_name(r->dtype), r->H, r->W, r->ld);
    if (vneed(v, 2, BNN_F32, (size_t)(Ho + 2 * r->halo) * (Wo + 2 * r->halo) * r->ld)) return -1;
  }
  if (opad) v->c->launches += 1; /* the zero halo */
  return 0;
}
static int init_gem(vctx *v) { /* gem_init, src/rt_ops_f32x.c:168-176 */
  if (vneed_args(v, 2, 1, 3)) return -1;
  const int P = v->op->p[0], C = v->op->p[1], ld = v->op->p[2];
  VREQ(v, P > 0 && C > 0 && C % 4 == 0 && ld >= C);
  if (vneed_t(v, 0, 12, 0)) return -1;
  const float *k = vt(v, 0, NULL);
  VREQ(v, k[0] > 0.f && k[1] > 0.f);
  return vneed_nohalo(v, 0, BNN_F32, (size_t)P * ld) || vneed(v, 1, BNN_F32, (size_t)C) ? -1 : 0;
}
static int init_vadd(vctx *v) { /* vadd_init, src/rt_ops_f32x.c:352-357 */
  if (vneed_args(v, 3, 0, 1)) return -1;
  VREQ(v, v->op->p[0] > 0);
  const size_t n = (size_t)v->op->p[0];
  return vneed(v, 0, BNN_F32, n) || vneed(v, 1, BNN_F32, n) || vneed(v, 2, BNN_F32, n) ? -1 : 0;
}
/* rt_sed_geom (src/rt_ops_f32x.c:207-236): what SED and SED_S8 check alike after their three GEMM views; kt = the consts
 * tensor, Cp = the channel stride of s and pooled */
static int sed_geom(vctx *v, int kt, int Cp) {
  const int *p = v->op->p;
  const int fcN = p[0], fcK = p[1], fcNp = p[3], atN = p[4], atK = p[5], atNp = p[7], clN = p[8], clK = p[9];
  const int clNp = p[11];
  const int red = p[12], H = p[13], W = p[14], C = p[15], ld = p[16], L = p[17], pk = p[18], dk = p[19], hc = p[20];
  const int L8 = (L + 7) & ~7;
  VREQ(v, red == 2 || red == 3);
  VREQ(v, H > 0 && W > 0 && C > 0 && C % 4 == 0 && ld >= C && L == (red == 3 ? H : W));
  VREQ(v, pk >= 0 && pk <= 15 && (pk == 0 || pk % 2) && dk >= 0 && dk <= 15 && (dk == 0 || dk % 2) && (pk || dk));
  VREQ(v, hc == 0 || hc == 1);
  VREQ(v, L <= 64);
  VREQ(v, fcK == C && atK == fcN && clK == fcN && atN == clN);
  if (vneed_t(v, 0, (size_t)(dk ? dk : 1) * C * 4, 0) || vneed_t(v, 1, (size_t)C * 4, 0) || vneed_t(v, kt, 12, 0))
    return -1;
  const bnn_buf_rec *x = vbd(v, 0);
  if (!x || x->halo || x->dtype != BNN_F32 || x->H != (uint32_t)H || x->W != (uint32_t)W)
    return vbad(v, "buffer argument 0: expected an unpadded fp32 activation %d x %d", H, W);
  return vneed(v, 0, BNN_F32, (size_t)H * W * ld) || vneed(v, 1, BNN_F32, (size_t)atN) ||
                 vneed(v, 2, BNN_F32, (size_t)L8 * Cp) || vneed(v, 3, BNN_F32, (size_t)L8 * Cp) ||
                 vneed(v, 4, BNN_F32, (size_t)L8 * fcNp) || vneed(v, 5, BNN_F32, (size_t)L8 * atNp) ||
                 vneed(v, 6, BNN_F32, (size_t)L8 * clNp)
             ? -1
             : 0;
}
static int init_sed(vctx *v) { /* sed_init, src/rt_ops_f32x.c:237-248 */
  if (vneed_args(v, 7, 9, 21) || v_fpack(v, 2, 0) || v_fpack(v, 4, 4) || v_fpack(v, 6, 8)) return -1;
  const int *p = v->op->p;
  VREQ(v, p[2] % 8 == 0 && p[6] == p[3] && p[10] == p[3]);
  return sed_geom(v, 8, p[2]);
}
static int init_sed_s8(vctx *v) { /* sed8_init, src/rt_ops_s8n.c:163-174 */
  if (vneed_args(v, 10, 15, 21) || v_s8(v, 2, 0) || v_s8(v, 6, 4) || v_s8(v, 10, 8)) return -1;
  const int *p = v->op->p;
  const int Cp = R8(p[15]);
  if (sed_geom(v, 14, Cp)) return -1;
  const size_t L8 = (size_t)R8(p[17]), Kq = (size_t)(p[2] > p[6] ? p[2] : p[6]);
  return vneed(v, 7, BNN_I8, L8 * Kq) || vneed(v, 8, BNN_F32, L8) || vneed(v, 9, BNN_I32, L8) ? -1 : 0;
}
static int init_convw(vctx *v) { /* convw_init, src/rt_ops_f32x.c:370-412 */
  if (vneed_args(v, 3, 2, 10)) return -1;
  const int *p = v->op->p;
  const int C = p[0], N = p[1], Np = p[2], H = p[3], W = p[4], act = p[5], ldo = p[6], opad = p[7], S = p[8], Nb = p[9];
  VREQ(v, C > 0 && C % 4 == 0 && N > 0 && Np == ((N + 7) & ~7) && H > 0 && W > 0);
  VREQ(v, act >= 0 && act <= 2 && opad >= 0 && opad <= 3 && ldo >= Np);
  VREQ(v, S >= 1 && S <= 256 && Nb >= 8 && Nb % 8 == 0);
  const bnn_buf_rec *x = vbd(v, 0), *o = vbd(v, 1);
  if (!x || !o) return vbad(v, "buffer argument %d is absent", x ? 1 : 0);
  if (x->dtype != BNN_F32 || x->H != (uint32_t)H || x->W != (uint32_t)W || x->ld != (uint32_t)C || x->halo < 1)
    return vbad(v, "buffer argument 0 (buffer #%d, input): expected fp32 %d x %d ld %d with a halo, found %s %u x %u ld %u halo %u",
                v->op->b[0], H, W, C, bnn_dtype_name(x->dtype), x->H, x->W, x->ld, x->halo);
  const int h = (int)x->halo;
  if (vneed(v, 0, BNN_F32, (size_t)(H + 2 * h) * (W + 2 * h) * C)) return -1;
  if (o->dtype != BNN_F32 || o->H != (uint32_t)H || o->W != (uint32_t)W || o->ld != (uint32_t)ldo || o->halo != (uint32_t)opad)
    return vbad(v, "buffer argument 1 (buffer #%d, output): expected fp32 %d x %d ld %d halo %d", v->op->b[1], H, W, ldo, opad);
  if (vneed(v, 1, BNN_F32, (size_t)(H + 2 * opad) * (W + 2 * opad) * ldo)) return -1;
  if (vneed_t(v, 0, (size_t)36 * Np * C * 4, 1) || vneed_t(v, 1, (size_t)Np * 4, 1)) return -1;
  const bnn_buf_rec *r = vbd(v, 2);
  if (r) {
    if (r->dtype != BNN_F32 || r->H != (uint32_t)H || r->W != (uint32_t)W || r->ld < (uint32_t)Np)
      return vbad(v, "buffer argument 2 (buffer #%d, residual): expected fp32 %d x %d with ld >= %d", v->op->b[2], H, W, Np);
    if (vneed(v, 2, BNN_F32, (size_t)(H + 2 * r->halo) * (W + 2 * r->halo) * r->ld)) return -1;
  }
  if (opad) v->c->launches += 1; /* the zero halo */
  return 0;
}

static int init_proto_f16s8(vctx *v) { /* proto8_init (src/rt_ops_f16.c:254-267) after rt_proto_geom / rt_proto_io
                                        * (src/rt_ops_f32.c:525-545) */
  if (vneed_args(v, 4, 5, 8)) return -1;
  const int *p = v->op->p;
  const int N = p[0], K = p[1], Np = p[2], P = p[3], C = p[4], ld = p[5], nc = p[6], ppc = p[7];
  VREQ(v, P > 0 && P <= 65536 && nc > 0 && ppc >= 1);
  VREQ(v, N > 0 && N <= (1 << 26) && K > 0 && K <= (1 << 17));
  VREQ(v, K == C);
  VREQ(v, ld >= C);
  VREQ(v, (size_t)nc * ppc == (size_t)N);
  VREQ(v, K % 8 == 0);
  VREQ(v, P % 8 == 0 && Np % 12 == 0 && Np >= N);
  if (vneed_t(v, 0, (size_t)Np * K, 1) || vneed_t(v, 1, (size_t)Np * 4, 1)) return -1;
  if (vneed_t(v, 2, (size_t)N * 4, 0) || vneed_t(v, 3, (size_t)nc * 4, 0) || vneed_t(v, 4, 4, 0)) return -1;
  if (vneed_nohalo(v, 0, BNN_F16, (size_t)P * ld) || vneed(v, 1, BNN_F32, (size_t)nc)) return -1;
  if (vneed(v, 2, BNN_I8, (size_t)P * K) || vneed(v, 3, BNN_F32, (size_t)Np)) return -1;
  if (P > 256) v->c->launches += 1; /* the chunk maxima */
  return 0;
}

/* the registry of this library: opcode (base | variant << 8) -> kernel; outmask / optmask as the reference's
 * (src/rt_ops_f32.c:620-637, src/rt_ops_s8n.c:255-260, src/rt_ops_f16.c:280-299). Variant 0: the neon-int8 path's
 * ops (and the fp32 head of small models); variant 1: the neon-fp16 path's; variant 2: the int8 prototype head of
 * the neon-fp16 path (the reference's SDOT head, rt_k_f16_s8). */
typedef struct {
  int code;
  const char *name;
  int (*init)(vctx *);
  uint32_t outmask, optmask;
  int launches;  /* kernel launches per run */
} kdesc;
static const kdesc KERNELS[] = {
    {BNN_OP_FE_STFT2, "fe_stft2", init_fe_stft2, 0x2, 0, 2},
    {BNN_OP_C0POOL, "c0pool_f32", init_c0pool, 0x2, 0, 1},
    {BNN_OP_DW3, "dw3_f32", init_dw3, 0x6, 0, 1},
    {BNN_OP_POSTPC, "postpc_f32", init_postpc, 0xe, 0, 2},
    {BNN_OP_SE_GATE, "se_gate_f32", init_se_gate, 0x2, 0, 1},
    {BNN_OP_PW_S8, "pw_s8n", init_pw_s8, 0x3a, 0x44, 2},
    {BNN_OP_GEMV_S8, "gemv_s8n", init_gemv_s8, 0x1e, 0, 2},
    {BNN_OP_PROTO_S8, "proto_s8n", init_proto_s8, 0xe, 0, 3},
    {BNN_OP_FE_LOGMEL, "fe_logmel", init_fe_logmel, 0x2, 0, 1},
    {BNN_OP_FE_DBIMG, "fe_dbimg", init_fe_dbimg, 0x2, 0, 3},
    {BNN_OP_DENSE, "dense_f32", init_dense_f32, 0x2, 0, 1},
    {BNN_OP_C0POOL_F16, "c0pool_f16", init_c0pool_f16, 0x2, 0, 1},
    {BNN_OP_PW_F16, "pw_f16", init_pw_f16, 0x2, 0x4, 1},
    {BNN_OP_DW3_F16, "dw3_f16", init_dw3_f16, 0x6, 0, 1},
    {BNN_OP_SE_F16, "se_f16", init_se_f16, 0x1, 0, 2},
    {BNN_OP_POSTPC_F16, "postpc_f16", init_postpc_f16, 0xe, 0, 3},
    {BNN_OP_DENSE_F16, "dense_f16", init_dense_f16, 0x2, 0, 1},
    {BNN_OP_STEM_F16, "stem_f32to16", init_stem_f16, 0xe, 0, 1},
    {BNN_OP_DWK_F16, "dwk_f16", init_dwk_f16, 0x6, 0, 1},
    {BNN_OP_PAD_F16, "pad_f16", init_pad, 0x2, 0, 1},
    {BNN_OP_MEAN_F16, "mean_f16", init_mean, 0x2, 0, 1},
    {BNN_OP_PROTO_F16S8, "proto_s8", init_proto_f16s8, 0xe, 0, 3},
    {BNN_OP_PW, "pw_f32", init_pw_f32, 0x2, 0xc, 1},
    {BNN_OP_STEM, "stem_f32", init_stem_f32, 0x6, 0, 2},
    {BNN_OP_DWK, "dwk_f32", init_dwk_f32, 0x6, 0, 1},
    {BNN_OP_PAD, "pad_f32", init_pad_f32, 0x2, 0, 2},
    {BNN_OP_MEAN, "mean_f32", init_mean, 0x2, 0, 1},
    {BNN_OP_CONVK, "convk_f32", init_convk, 0x2, 0x4, 1},
    {BNN_OP_GEM, "gem_f32", init_gem, 0x2, 0, 1},
    {BNN_OP_SED, "sed_f32", init_sed, 0x7e, 0, 5},
    {BNN_OP_SED_S8, "sed_s8n", init_sed_s8, 0x3fe, 0, 7},
    {BNN_OP_VADD, "vadd_f32", init_vadd, 0x4, 0, 1},
    {BNN_OP_CONVW, "convw_f32", init_convw, 0x2, 0x4, 3},
};
static const kdesc *kernel_for(int code) {
  for (size_t i = 0; i < sizeof KERNELS / sizeof KERNELS[0]; i++)
    if (KERNELS[i].code == code) return &KERNELS[i];
  return NULL;
}

/* ------------------------------------------------------------------ op list decoding (src/rt_pkg.c:349-509) */

#define HINT_PKG "hint: package/library mismatch or a lowering bug: recompile with this checkout's compiler/bnc.py; if it " \
                 "reproduces, report this message"

int bnn_rt_open(bnn_ctx *c, char *err, size_t errlen, int *kind) {
  *kind = BNN_ERR_PACKAGE;
  const bnn_path_rec *d = c->path;
  const uint8_t *m = c->pkg->map;
  c->bufd = bnn_fail_host_alloc() ? NULL : malloc(sizeof(bnn_buf_rec) * d->n_buf);
  c->ops = calloc(d->n_ops, sizeof(bnn_op));
  if (!c->bufd || !c->ops) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (op list)"); return -1; }
  memcpy(c->bufd, m + d->buf_off, sizeof(bnn_buf_rec) * d->n_buf);
  const bnn_buf_rec *bd = c->bufd;
  size_t *slot_sz = calloc(d->n_buf, sizeof(size_t)), total = 0;
  if (!slot_sz) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (slot table)"); return -1; }
  for (uint32_t i = 0; i < d->n_buf; i++) {
    if (bd[i].dtype > BNN_I32 || bd[i].elems > ((size_t)1 << 30) || bd[i].slot >= d->n_buf) {
      snprintf(err, errlen, "path %.24s buffer #%u: bad descriptor (dtype %u, %llu elements, slot %u of %u); " HINT_PKG,
               d->name, i, bd[i].dtype, (unsigned long long)bd[i].elems, bd[i].slot, d->n_buf);
      free(slot_sz);
      return -1;
    }
    if ((i == d->in_buf) != (bd[i].slot == bd[d->in_buf].slot)) {
      snprintf(err, errlen, "path %.24s buffer #%u shares the input window's memory slot %u; " HINT_PKG, d->name, i, bd[i].slot);
      free(slot_sz);
      return -1;
    }
    const size_t b = ((size_t)bd[i].elems * dsize(bd[i].dtype) + 64 + 63) & ~(size_t)63;
    if (b > slot_sz[bd[i].slot]) slot_sz[bd[i].slot] = b;
  }
  for (uint32_t s = 0; s < d->n_buf; s++) {
    if (s == bd[d->in_buf].slot) continue;
    total += slot_sz[s];
    if (total > ((size_t)1 << 30)) {
      snprintf(err, errlen, "path %.24s needs more than 1 GB of activation buffers; hint: the package is corrupt or the "
               "model is far larger than this runtime is built for", d->name);
      free(slot_sz);
      return -1;
    }
  }
  free(slot_sz);
  for (uint32_t i = 0; i < d->n_buf; i++)
    if (i != d->out_buf && (bd[i].slot == bd[d->out_buf].slot ||
                            (d->emb_buf != 0xffffffffu && i != d->emb_buf && bd[i].slot == bd[d->emb_buf].slot))) {
      snprintf(err, errlen, "path %.24s buffer #%u shares memory slot %u with the output buffer (#%u / #%u); " HINT_PKG,
               d->name, i, bd[i].slot, d->out_buf, d->emb_buf);
      return -1;
    }
  const uint8_t *q = m + d->ops_off, *end = q + d->ops_bytes;
  for (uint32_t i = 0; i < d->n_ops; i++) {
    uint16_t h[6];
    if (q + 12 > end) {
      snprintf(err, errlen, "op %u: truncated op list (%u ops declared, %u bytes); " HINT_PKG, i, d->n_ops, d->ops_bytes);
      return -1;
    }
    memcpy(h, q, 12);
    const size_t need = 12 + 4 * ((size_t)h[2] + h[3] + h[4]);
    if (h[1] < need || q + h[1] > end || ((uintptr_t)(q - m) % 4)) {
      snprintf(err, errlen, "op %u: bad op record (%u bytes for %u buffer, %u tensor, %u int arguments); " HINT_PKG, i,
               h[1], h[2], h[3], h[4]);
      return -1;
    }
    bnn_op *op = &c->ops[i];
    op->code = h[0];
    op->nb = h[2];
    op->nt = h[3];
    op->ni = h[4];
    op->b = (const int32_t *)(q + 12);
    op->t = op->b + op->nb;
    op->p = op->t + op->nt;
    op->kname = "?";
    c->n_ops = (int)i + 1;
    vctx v = {c, (int)i, op, err, errlen, 0};
    for (int k = 0; k < op->nb; k++)
      if (op->b[k] >= (int32_t)d->n_buf || op->b[k] < -1)
        return vbad(&v, "buffer argument %d names buffer #%d but the path has %u buffers", k, op->b[k], d->n_buf);
    for (int k = 0; k < op->nt; k++)
      if (op->t[k] >= (int32_t)c->pkg->n_tensors)
        return vbad(&v, "tensor argument %d names tensor #%d but the package has %u tensors", k, op->t[k],
                    c->pkg->n_tensors);
    const int var = op->code >> 8;
    if (var && !(d->hwcap & 1))
      return vbad(&v, "fp16 kernel (opcode 0x%x) in path %.24s, which does not declare the fp16 requirement", op->code,
                  d->name);
    if (var == 2 && !(d->hwcap & 2))
      return vbad(&v, "dotprod kernel (opcode 0x%x) in path %.24s, which does not declare the dotprod requirement",
                  op->code, d->name);
    const kdesc *k = kernel_for(op->code);
    if (!k) {
      char comp[48];
      if (bnn_meta_str(c->pkg, "compiler", comp, sizeof comp) < 0) snprintf(comp, sizeof comp, "unknown");
      *kind = BNN_ERR_CPU;
      return vbad(&v, "opcode 0x%x (base %d variant %d) has no B200 kernel in this library (it runs the neon-int8 ops "
                  "FE_STFT2, C0POOL, PW_S8, DW3, SE_GATE, POSTPC, GEMV_S8, PROTO_S8, FE_LOGMEL, FE_DBIMG and DENSE, and the "
                  "neon-fp16 ops C0POOL, PW, DW3, SE, POSTPC and DENSE of variant 1; the package was written by "
                  "compiler '%s')",
                  op->code, op->code & 0xff, var, comp);
    }
    op->kname = k->name;
    for (int a = 0; a < op->nb; a++) {
      if (op->b[a] < 0 && !(a < 32 && (k->optmask >> a & 1)))
        return vbad(&v, "buffer argument %d is required by the kernel but absent (-1) in the op record", a);
      if (op->b[a] == (int32_t)d->in_buf && a < 32 && (k->outmask >> a & 1))
        return vbad(&v, "buffer argument %d is the input window (#%u) but the kernel writes it", a, d->in_buf);
    }
    for (int a = 0; a < op->nb; a++)
      for (int b2 = 0; b2 < op->nb; b2++)
        if (a != b2 && op->b[a] >= 0 && op->b[b2] >= 0 && a < 32 && (k->outmask >> a & 1) &&
            (op->b[a] == op->b[b2] || bd[op->b[a]].slot == bd[op->b[b2]].slot))
          return vbad(&v, "buffer arguments %d (#%d, written) and %d (#%d) share memory slot %u", a, op->b[a], b2,
                      op->b[b2], bd[op->b[a]].slot);
    if (k->init(&v)) return -1;
    c->launches += k->launches;
    q += h[1];
  }
  for (int i = 0; i + 1 < c->n_ops; i++)  /* quantizers done by the launch before */
    if (c0_quantizes_next(c, i)) c->launches -= 1;
  return 0;
}

/* ------------------------------------------------------------------ device state */

static int cerr(char *err, size_t errlen, int *kind, cudaError_t e, const char *what) {
  *kind = e == cudaErrorMemoryAllocation ? BNN_ERR_OOM : BNN_ERR_CPU;
  snprintf(err, errlen, "%s: CUDA error %d (%s); hint: %s", what, (int)e, cudaGetErrorString(e),
           e == cudaErrorMemoryAllocation ? "free GPU memory or lower the batch (bnn_set_batch, BNN_BATCH)"
                                          : "check the GPU and the driver (nvidia-smi)");
  return -1;
}
#define CK(call, what)                                                  \
  do {                                                                  \
    cudaError_t e_ = (cudaError_t)(call);                               \
    if (e_ != cudaSuccess) return cerr(err, errlen, kind, e_, (what));  \
  } while (0)

/* every device allocation of the runtime: cudaMalloc, unless the test hook (bnn_debug_fail_alloc) fails this one */
static cudaError_t dmalloc(void **p, size_t bytes) {
  if (bnn_fail_dev_alloc()) return cudaErrorMemoryAllocation;
  return cudaMalloc(p, bytes);
}

static const void *tptr(const bnn_ctx *c, const bnn_op *op, int a) {
  return c->pkg->map + c->pkg->tensors[op->t[a]].offset;
}
static int upload(void **dst, const void *src, size_t bytes, char *err, size_t errlen, int *kind) {
  CK(dmalloc(dst, bytes ? bytes : 16), "weight upload (cudaMalloc)");
  if (bytes) CK(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice), "weight upload (cudaMemcpy)");
  return 0;
}
/* the buffer arguments [lo, lo + n) of an op that the device scratch replaces or that its kernels never touch:
 * PW_S8 b[3..5], GEMV_S8 b[2..4] (q, sa, za), PROTO_S8 and PROTO variant 2 b[2] (the quantized cells), STEM f16 b[2..3]
 * (the im2col rows and the fp32 GEMM output: the kernel reads the image and writes fp16 directly) */
static void scratch_args(const bnn_op *op, int *lo, int *n) {
  const int proto = op->code == BNN_OP_PROTO_S8 || op->code == BNN_OP_PROTO_F16S8;
  *lo = op->code == BNN_OP_PW_S8 ? 3 : op->code == BNN_OP_GEMV_S8 || proto || op->code == BNN_OP_STEM_F16 ? 2
        : op->code == BNN_OP_SED_S8 ? 7 : -1;
  *n = proto ? 1 : op->code == BNN_OP_STEM_F16 ? 2 : 3;
}
static int is_scratch(const bnn_ctx *c, int buf) {
  for (int i = 0; i < c->n_ops; i++) {
    const bnn_op *op = &c->ops[i];
    int lo, n;
    scratch_args(op, &lo, &n);
    for (int a = 0; a < op->nb; a++) {
      if (op->b[a] != buf) continue;
      if (lo < 0 || a < lo || a >= lo + n) return 0;
    }
  }
  for (int i = 0; i < c->n_ops; i++) {
    const bnn_op *op = &c->ops[i];
    int lo, n;
    scratch_args(op, &lo, &n);
    if (lo >= 0)
      for (int a = lo; a < lo + n; a++)
        if (op->b[a] == buf) return 1;
  }
  return 0;
}

/* FE_STFT2 tables (spec_init, src/v24_fe.c:45-84; fft_twiddles / fft_bitrev, src/fft_tab.h:9-21): twiddles and the
 * real-split cos / sin in double, rounded once; the sparse mel as the nonzero range of each filter row
 * (nz_range, src/rt_ops_f32.c:16-24) */
static int fe_tables(bnn_ctx *c, bnn_dev *dv, const bnn_op *op, char *err, size_t errlen, int *kind) {
  bnnk_fe_tables *t = &dv->fe;
  for (int br = 0; br < 2; br++) {
    const int N = br ? 1024 : 2048, M = N / 2, bins = M + 1;
    int lg = 0;
    while ((1 << lg) < M) lg++;
    const float *win = tptr(c, op, br), *mel = tptr(c, op, 2 + br);
    const float pw = ((const float *)tptr(c, op, 4 + br))[0];
    int lo[96], hi[96], klo = bins, khi = 0, nnz = 0;
    for (int j = 0; j < 96; j++) {
      const float *f = mel + (size_t)j * bins;
      int l = 0, h = 0;
      for (int k = 0; k < bins; k++)
        if (f[k] != 0.f) { if (h == 0) l = k; h = k + 1; }
      lo[j] = l;
      hi[j] = h;
      if (h > l) { if (l < klo) klo = l; if (h > khi) khi = h; }
      nnz += h - l;
    }
    if (khi <= klo) { klo = 0; khi = 0; }
    float *twr = malloc(sizeof(float) * M / 2), *twi = malloc(sizeof(float) * M / 2);
    float *pcv = malloc(sizeof(float) * (khi + 1)), *psv = malloc(sizeof(float) * (khi + 1));
    int *rev = malloc(sizeof(int) * M), *off = malloc(sizeof(int) * 97), *mk = malloc(sizeof(int) * (nnz + 1));
    float *mw = malloc(sizeof(float) * (nnz + 1));
    if (!twr || !twi || !pcv || !psv || !rev || !off || !mk || !mw) {
      *kind = BNN_ERR_OOM;
      snprintf(err, errlen, "out of memory (front-end tables)");
      return -1;
    }
    for (int k = 0; k < M / 2; k++) {
      const double a = -2 * M_PI * k / M;
      twr[k] = (float)cos(a);
      twi[k] = (float)sin(a);
    }
    for (int k = 0; k < khi; k++) {
      const double a = 2 * M_PI * k / N;
      pcv[k] = (float)cos(a);
      psv[k] = (float)sin(a);
    }
    for (int i = 0; i < M; i++) {
      int r = 0;
      for (int b = 0; b < lg; b++) r |= ((i >> b) & 1) << (lg - 1 - b);
      rev[i] = r;
    }
    nnz = 0;
    for (int j = 0; j < 96; j++) {
      off[j] = nnz;
      for (int k = lo[j]; k < hi[j]; k++) { mk[nnz] = k; mw[nnz] = mel[(size_t)j * bins + k]; nnz++; }
    }
    off[96] = nnz;
    void *d;
    int rc = 0;
#define UP(field, src, bytes)                                     \
    if (!rc) {                                                    \
      rc = upload(&d, (src), (bytes), err, errlen, kind);         \
      if (!rc) { t->field[br] = d; dv->fe_mem[dv->n_fe_mem++] = d; } \
    }
    /* the window in the gather order of the spectrogram kernel: thread l of a frame reads bit-reversed positions
     * 16 l .. 16 l + 15, its e-th pair stored at e * (M / 16) + l */
    float *wg = malloc(sizeof(float) * N);
    if (!wg) {
      free(twr); free(twi); free(pcv); free(psv); free(rev); free(off); free(mk); free(mw);
      *kind = BNN_ERR_OOM;
      snprintf(err, errlen, "out of memory (front-end tables)");
      return -1;
    }
    for (int p = 0; p < M; p++) {
      const int r = rev[p], e = p % 16, l = p / 16;
      wg[2 * (e * (M / 16) + l)] = win[2 * r];
      wg[2 * (e * (M / 16) + l) + 1] = win[2 * r + 1];
    }
    UP(win, wg, sizeof(float) * N);
    free(wg);
    UP(tw_re, twr, sizeof(float) * M / 2);
    UP(tw_im, twi, sizeof(float) * M / 2);
    {  /* the stage table: stages of length 8, 32, 128, 512 hold 4, 16, 64, 256 groups (the last only for M = 1024) */
      float st[(4 + 16 + 64 + 256) * 4];
      memset(st, 0, sizeof st);
      static const int lens[4] = {8, 32, 128, 512}, base[4] = {0, 4, 20, 84};
      for (int g = 0; g < 4; g++) {
        if (2 * lens[g] > M) continue; /* a stage of length 512 only runs when M = 1024 */
        for (int j = 0; j < lens[g] / 2; j++) {
          const int i1 = j * (M / lens[g]), i2 = j * (M / (2 * lens[g]));
          float *e = st + 4 * (base[g] + j);
          e[0] = twr[i1]; e[1] = twi[i1]; e[2] = twr[i2]; e[3] = twi[i2];
        }
      }
      UP(tw_st, st, sizeof st);
    }
    UP(pc, pcv, sizeof(float) * (khi + 1));
    UP(ps, psv, sizeof(float) * (khi + 1));
    UP(rev, rev, sizeof(int) * M);
    UP(mel_off, off, sizeof(int) * 97);
    UP(mel_k, mk, sizeof(int) * (nnz + 1));
#undef UP
    if (!rc) {
      rc = upload(&d, mw, sizeof(float) * (nnz + 1), err, errlen, kind);
      if (!rc) { t->mel_w[br] = d; dv->fe_mem[dv->n_fe_mem++] = d; }
    }
    free(twr); free(twi); free(pcv); free(psv); free(rev); free(off); free(mk); free(mw);
    if (rc) return rc;
    t->klo[br] = klo;
    t->khi[br] = khi;
    t->pw2[br] = 2.f * pw;
    t->bn_s[br] = ((const float *)tptr(c, op, 6))[br];
    t->bn_b[br] = ((const float *)tptr(c, op, 7))[br];
  }
  return 0;
}

/* int8 GEMM weights in the GEMM's layout: the package's panels [Np/4][Kp/16][4][16] (lower.py:883-914) as rows
 * [n_tiles * bn][Kq] (Kq = K rounded up to 32), zero beyond N and K; scales, column sums and biases padded with zeros */
int bnn_s8_weights(bnn_devop *d, int N, int K, int Kp, int Np, const int8_t *src, const float *sw_src,
                   const int32_t *cs_src, const float *b_src, int rows_cap, char *err, size_t errlen, int *kind) {
  (void)N;
  const int kq = R32(K), rows = bnnk_gemm_weight_rows(Np, rows_cap);
  d->kq = kq;
  int8_t *w = calloc((size_t)rows * kq, 1);
  float *sw = calloc(rows, sizeof(float)), *b = calloc(rows, sizeof(float));
  int32_t *cs = calloc(rows, sizeof(int32_t));
  if (!w || !sw || !b || !cs) {
    free(w); free(sw); free(b); free(cs);
    *kind = BNN_ERR_OOM;
    snprintf(err, errlen, "out of memory (int8 weights, %d x %d)", rows, kq);
    return -1;
  }
  for (int n = 0; n < Np; n++)
    for (int k = 0; k < Kp; k++)
      w[(size_t)n * kq + k] = src[(((size_t)(n / 4) * (Kp / 16) + k / 16) * 4 + n % 4) * 16 + k % 16];
  memcpy(sw, sw_src, sizeof(float) * Np);
  memcpy(cs, cs_src, sizeof(int32_t) * Np);
  memcpy(b, b_src, sizeof(float) * Np);
  int rc = upload((void **)&d->w, w, (size_t)rows * kq, err, errlen, kind);
  if (!rc) rc = upload((void **)&d->sw, sw, sizeof(float) * rows, err, errlen, kind);
  if (!rc) rc = upload((void **)&d->cs, cs, sizeof(int32_t) * rows, err, errlen, kind);
  if (!rc) rc = upload((void **)&d->bias, b, sizeof(float) * rows, err, errlen, kind);
  free(w); free(sw); free(b); free(cs);
  return rc;
}

/* PROTO_S8 tensors in the kernels' layouts: the package's prototype panels [Np/4][Kp/16][4][16] (lower.py
 * proto_s8n) as rows [Np][Kp]; sw [Np]; class weights [N], biases [nc]; eps */
int bnn_proto_weights(bnn_devop *d, int N, int Kp, int Np, const int8_t *src, const float *sw_src, const float *cw,
                      const float *cb, int nc, float eps, char *err, size_t errlen, int *kind) {
  return bnn_proto_weights_l(d, 0, N, Kp, Kp, Np, src, sw_src, cw, cb, nc, eps, err, errlen, kind);
}

/* layout 0: the neon-int8 head's panels [Np/4][Kp/16][4][16] (K = Kp); layout 1: the SDOT head's [Np/12][K/4][12][4]
 * (python/bnneon/compiler/lower.py proto_s8). Rows [Np][Kq], Kq >= K a multiple of 16, zero past K. */
int bnn_proto_weights_l(bnn_devop *d, int layout, int N, int K, int Kq, int Np, const int8_t *src, const float *sw_src,
                        const float *cw, const float *cb, int nc, float eps, char *err, size_t errlen, int *kind) {
  const int Kp = Kq;
  int8_t *w = calloc((size_t)Np * Kq, 1);
  if (!w) {
    *kind = BNN_ERR_OOM;
    snprintf(err, errlen, "out of memory (prototypes, %d x %d)", Np, Kq);
    return -1;
  }
  for (int j = 0; j < Np; j++)
    for (int k = 0; k < K; k++)
      w[(size_t)j * Kq + k] = layout == 0 ? src[(((size_t)(j / 4) * (Kp / 16) + k / 16) * 4 + j % 4) * 16 + k % 16]
                                          : src[(((size_t)(j / 12) * (K / 4) + k / 4) * 12 + j % 12) * 4 + k % 4];
  int rc = upload((void **)&d->w, w, (size_t)Np * Kq, err, errlen, kind);
  free(w);
  if (!rc) rc = upload((void **)&d->sw, sw_src, sizeof(float) * Np, err, errlen, kind);
  if (!rc) rc = upload((void **)&d->f[1], cw, sizeof(float) * N, err, errlen, kind);
  if (!rc) rc = upload((void **)&d->f[2], cb, sizeof(float) * nc, err, errlen, kind);
  d->kq = Kq;
  d->eps = eps;
  return rc;
}

/* pc_logmel_new (src/pc_kern_f32.c:28-72): the window zero past frame; twiddles e^{-2 pi i k / M} and the real-split
 * cos / sin (2 pi k / nfft) in double, rounded once; the sparse mel as each row's nonzero entries in bin order; [klo,
 * khi) the bins any row uses (0, 0 when none) */
int bnn_logmel_build(bnn_devop *d, int nsamp, int frame, int hop, int pad, int nfft, int nmel, const float *window,
                     const float *mel, float floor_, float scale, char *err, size_t errlen, int *kind) {
  bnnk_logmel_tables *t = &d->lm;
  memset(t, 0, sizeof *t);
  const int M = nfft / 2, bins = nfft / 2 + 1;
  t->nsamp = nsamp; t->frame = frame; t->hop = hop; t->pad = pad; t->nfft = nfft; t->M = M; t->nmel = nmel;
  t->nfr = (nsamp + 2 * pad - frame) / hop + 1;
  while ((1 << t->lg) < M) t->lg++;
  t->nz = (frame + 1) / 2;
  t->floor_ = floor_;
  t->scale = scale;
  t->klo = bins;
  int nnz = 0;
  for (int j = 0; j < nmel; j++)
    for (int k = 0; k < bins; k++)
      if (mel[(size_t)j * bins + k] != 0.f) { nnz++; if (k < t->klo) t->klo = k; if (k + 1 > t->khi) t->khi = k + 1; }
  if (t->khi == 0) t->klo = 0;
  float *win = calloc((size_t)nfft, sizeof(float)), *twr = malloc(sizeof(float) * (size_t)(M / 2 + 1)),
        *twi = malloc(sizeof(float) * (size_t)(M / 2 + 1)), *pc = malloc(sizeof(float) * (size_t)(t->khi + 1)),
        *ps = malloc(sizeof(float) * (size_t)(t->khi + 1)), *mw = malloc(sizeof(float) * (size_t)(nnz + 1));
  int *moff = malloc(sizeof(int) * (size_t)(nmel + 1)), *mk = malloc(sizeof(int) * (size_t)(nnz + 1));
  int rc = 0;
  if (!win || !twr || !twi || !pc || !ps || !mw || !moff || !mk) {
    *kind = BNN_ERR_OOM;
    snprintf(err, errlen, "out of memory (log-mel tables)");
    rc = -1;
  } else {
    memcpy(win, window, sizeof(float) * (size_t)frame);
    for (int k = 0; k < M / 2; k++) {
      const double a = -2 * M_PI * k / M;
      twr[k] = (float)cos(a); twi[k] = (float)sin(a);
    }
    for (int k = 0; k < t->khi; k++) {
      const double a = 2 * M_PI * k / nfft;
      pc[k] = (float)cos(a); ps[k] = (float)sin(a);
    }
    nnz = 0;
    for (int j = 0; j < nmel; j++) {
      moff[j] = nnz;
      for (int k = 0; k < bins; k++)
        if (mel[(size_t)j * bins + k] != 0.f) { mk[nnz] = k; mw[nnz] = mel[(size_t)j * bins + k]; nnz++; }
    }
    moff[nmel] = nnz;
    const void *src[8] = {win, twr, twi, pc, ps, mw, moff, mk};
    const size_t sz[8] = {sizeof(float) * (size_t)nfft, sizeof(float) * (size_t)(M / 2 + 1),
                          sizeof(float) * (size_t)(M / 2 + 1), sizeof(float) * (size_t)(t->khi + 1),
                          sizeof(float) * (size_t)(t->khi + 1), sizeof(float) * (size_t)(nnz + 1),
                          sizeof(int) * (size_t)(nmel + 1), sizeof(int) * (size_t)(nnz + 1)};
    for (int i = 0; i < 8 && !rc; i++) rc = upload(&d->lm_mem[i], src[i], sz[i], err, errlen, kind);
    if (!rc) {
      t->win = d->lm_mem[0]; t->tw_re = d->lm_mem[1]; t->tw_im = d->lm_mem[2]; t->pc = d->lm_mem[3];
      t->ps = d->lm_mem[4]; t->mel_w = d->lm_mem[5]; t->mel_off = d->lm_mem[6]; t->mel_k = d->lm_mem[7];
    }
  }
  free(win); free(twr); free(twi); free(pc); free(ps); free(mw); free(moff); free(mk);
  return rc;
}
void bnn_logmel_release(bnn_devop *d) {
  for (int i = 0; i < 8; i++) {
    cudaFree(d->lm_mem[i]);
    d->lm_mem[i] = NULL;
  }
}

/* fe_db_new (src/fe_dbimg.c:49-107): twiddles e^{-2 pi i k / NC} (k < NC / 2) and the real-split factors
 * e^{-2 pi i k / N} (k <= NC) in double, rounded once; the sparse mel as each row's nonzero entries in bin order,
 * [klo, khi) the bins any row uses; ONNX Runtime's half-pixel resize coordinates (axis_setup :37-47). All tables in one
 * device allocation; the scratch for batch windows in another. */
static void db_axis(int nin, int nout, int *i1, int *i2, float *d1, float *d2) {
  const float scale = (float)nout / (float)nin;
  for (int o = 0; o < nout; o++) {
    float x = ((float)o + 0.5f) / scale - 0.5f;
    if (x > (float)(nin - 1)) x = (float)(nin - 1);
    if (x < 0.f) x = 0.f;
    const int a = (int)x < nin - 1 ? (int)x : nin - 1;
    const int b = a + 1 < nin - 1 ? a + 1 : nin - 1;
    i1[o] = a; i2[o] = b;
    d1[o] = fabsf(x - (float)a); d2[o] = fabsf(x - (float)b);
    if (a == b) { d1[o] = 0.5f; d2[o] = 0.5f; }
  }
}
int bnn_dbimg_build(bnn_devop *d, const int32_t *p, const float *window, const float *mel, const int32_t *rows,
                    const float *consts, int batch, char *err, size_t errlen, int *kind) {
  bnnk_dbimg_tables *t = &d->db;
  memset(t, 0, sizeof *t);
  t->nsamp = p[0]; t->nfft = p[1]; t->hop = p[2]; t->pad = p[3]; t->padmode = p[4]; t->nfr = p[5]; t->nmel = p[6];
  t->R = p[7]; t->has_top_db = p[8]; t->norm = p[9]; t->post[0] = p[10]; t->post[1] = p[11]; t->post[2] = p[12];
  t->Ho = p[14]; t->Wo = p[15]; t->C = p[16]; t->chan[0] = p[17]; t->chan[1] = p[18]; t->ld = p[19]; t->halo = p[20];
  t->floor_ = consts[0]; t->top_db = consts[1]; t->eps = consts[2];
  for (int u = 0; u < 3; u++) t->postv[u] = consts[3 + u];
  const int N = t->nfft, NC = N / 2, F = NC + 1;
  while ((1 << t->lg) < NC) t->lg++;
  int nnz = 0, klo = F, khi = 0;
  for (int j = 0; j < t->nmel; j++)
    for (int k = 0; k < F; k++)
      if (mel[(size_t)j * F + k] != 0.f) { nnz++; if (k < klo) klo = k; if (k + 1 > khi) khi = k + 1; }
  t->klo = klo < khi ? klo : 0;
  t->khi = khi;
  /* sections of 4-byte elements, each starting on 64 elements */
  const size_t cnt[18] = {(size_t)N, (size_t)NC / 2 + 1, (size_t)NC / 2 + 1, (size_t)F, (size_t)F, (size_t)nnz + 1,
                          2 * (size_t)t->C, (size_t)t->Ho, (size_t)t->Ho, (size_t)t->Wo, (size_t)t->Wo,
                          (size_t)t->nmel + 1, (size_t)nnz + 1, (size_t)t->R, (size_t)t->Ho, (size_t)t->Ho,
                          (size_t)t->Wo, (size_t)t->Wo};
  size_t off[18], total = 0;
  for (int i = 0; i < 18; i++) { off[i] = total; total += (cnt[i] + 63) & ~(size_t)63; }
  uint32_t *h = calloc(total, 4);
  if (!h) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (dB-image tables)"); return -1; }
  float *win = (float *)(h + off[0]), *twr = (float *)(h + off[1]), *twi = (float *)(h + off[2]);
  float *spr = (float *)(h + off[3]), *spi = (float *)(h + off[4]), *mw = (float *)(h + off[5]);
  float *chv = (float *)(h + off[6]), *dy1 = (float *)(h + off[7]), *dy2 = (float *)(h + off[8]);
  float *dx1 = (float *)(h + off[9]), *dx2 = (float *)(h + off[10]);
  int *moff = (int *)(h + off[11]), *mk = (int *)(h + off[12]), *rw = (int *)(h + off[13]);
  int *ry1 = (int *)(h + off[14]), *ry2 = (int *)(h + off[15]), *rx1 = (int *)(h + off[16]), *rx2 = (int *)(h + off[17]);
  memcpy(win, window, sizeof(float) * (size_t)N);
  for (int k = 0; k < NC / 2; k++) {
    const double a = -2 * M_PI * k / NC;
    twr[k] = (float)cos(a); twi[k] = (float)sin(a);
  }
  for (int k = 0; k <= NC; k++) {
    const double a = -2 * M_PI * k / N;
    spr[k] = (float)cos(a); spi[k] = (float)sin(a);
  }
  int q = 0;
  for (int j = 0; j < t->nmel; j++) {
    moff[j] = q;
    for (int k = 0; k < F; k++)
      if (mel[(size_t)j * F + k] != 0.f) { mk[q] = k; mw[q] = mel[(size_t)j * F + k]; q++; }
  }
  moff[t->nmel] = q;
  memcpy(rw, rows, sizeof(int) * (size_t)t->R);
  memcpy(chv, consts + 6, sizeof(float) * 2 * (size_t)t->C);
  db_axis(t->R, t->Ho, ry1, ry2, dy1, dy2);
  db_axis(t->nfr, t->Wo, rx1, rx2, dx1, dx2);
  int rc = upload(&d->db_mem, h, total * 4, err, errlen, kind);
  free(h);
  if (rc) return rc;
  uint32_t *g = d->db_mem;
  t->win = (const float *)(g + off[0]); t->tw_re = (const float *)(g + off[1]); t->tw_im = (const float *)(g + off[2]);
  t->sp_re = (const float *)(g + off[3]); t->sp_im = (const float *)(g + off[4]); t->mel_w = (const float *)(g + off[5]);
  t->chv = (const float *)(g + off[6]); t->dy1 = (const float *)(g + off[7]); t->dy2 = (const float *)(g + off[8]);
  t->dx1 = (const float *)(g + off[9]); t->dx2 = (const float *)(g + off[10]);
  t->mel_off = (const int *)(g + off[11]); t->mel_k = (const int *)(g + off[12]); t->rows = (const int *)(g + off[13]);
  t->ry1 = (const int *)(g + off[14]); t->ry2 = (const int *)(g + off[15]); t->rx1 = (const int *)(g + off[16]);
  t->rx2 = (const int *)(g + off[17]);
  CK(dmalloc((void **)&d->db_scratch, sizeof(float) * bnnk_dbimg_scratch_floats(t, batch)), "dB-image scratch");
  return 0;
}
void bnn_dbimg_release(bnn_devop *d) {
  cudaFree(d->db_mem);
  cudaFree(d->db_scratch);
  d->db_mem = NULL;
  d->db_scratch = NULL;
}

/* hp_pack panels (src/gemm_f16.c:17-40: [Np/16][Kp][16], then a [Kp][8] tail panel when Np % 16) as the k-major
 * [Kp][Np] matrix of the B200 fp16 GEMM, each weight in both halves of a 32-bit word (dup != 0, to d->hwd) or plain
 * fp16 (to d->hw); b16 [Np] to d->hb; b32 [Np] to *b32 unless NULL */
int bnn_hpack_weights(bnn_devop *d, int dup, const uint16_t *panels, const float *b32src, const uint16_t *b16src,
                      int Kp, int Np, float **b32, char *err, size_t errlen, int *kind) {
  const size_t es = dup ? 4 : 2;
  uint8_t *wt = malloc(es * (size_t)Kp * Np);
  if (!wt) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (fp16 weights, %d x %d)", Kp, Np); return -1; }
  const int n16 = Np / 16;
  for (int n = 0; n < Np; n++)
    for (int k = 0; k < Kp; k++) {
      const uint16_t h = n / 16 < n16 ? panels[((size_t)(n / 16) * Kp + k) * 16 + n % 16]
                                      : panels[(size_t)n16 * Kp * 16 + (size_t)k * 8 + n % 16];
      if (dup) ((uint32_t *)wt)[(size_t)k * Np + n] = (uint32_t)h | ((uint32_t)h << 16);
      else ((uint16_t *)wt)[(size_t)k * Np + n] = h;
    }
  int rc = upload(dup ? (void **)&d->hwd : (void **)&d->hw, wt, es * (size_t)Kp * Np, err, errlen, kind);
  free(wt);
  if (!rc) rc = upload((void **)&d->hb, b16src, sizeof(uint16_t) * (size_t)Np, err, errlen, kind);
  if (!rc && b32) rc = upload((void **)b32, b32src, sizeof(float) * (size_t)Np, err, errlen, kind);
  return rc;
}

/* hp_pack panels as the tensor mode's K-major [Np][Kp] fp16 rows (to d->hwk) */
int bnn_hpack_kmajor(bnn_devop *d, const uint16_t *panels, int Kp, int Np, char *err, size_t errlen, int *kind) {
  uint16_t *wt = malloc(sizeof(uint16_t) * (size_t)Kp * Np);
  if (!wt) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (fp16 weights, %d x %d)", Np, Kp); return -1; }
  const int n16 = Np / 16;
  for (int n = 0; n < Np; n++)
    for (int k = 0; k < Kp; k++)
      wt[(size_t)n * Kp + k] = n / 16 < n16 ? panels[((size_t)(n / 16) * Kp + k) * 16 + n % 16]
                                            : panels[(size_t)n16 * Kp * 16 + (size_t)k * 8 + n % 16];
  const int rc = upload((void **)&d->hwk, wt, sizeof(uint16_t) * (size_t)Kp * Np, err, errlen, kind);
  free(wt);
  return rc;
}

/* the weights of op i in the kernels' layouts */
static int op_weights(bnn_ctx *c, bnn_dev *dv, int i, char *err, size_t errlen, int *kind) {
  const bnn_op *op = &c->ops[i];
  bnn_devop *d = &dv->ops[i];
  const int *p = op->p;
  switch (op->code) {
  case BNN_OP_PW_S8:
  case BNN_OP_GEMV_S8:
    return bnn_s8_weights(d, p[0], p[1], p[2], p[3], tptr(c, op, 0), tptr(c, op, 1), tptr(c, op, 2), tptr(c, op, 3),
                          c->batch * (op->code == BNN_OP_PW_S8 ? p[4] : 1),
                          err, errlen, kind);
  case BNN_OP_DW3: {
    const int C = p[2];
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * 9 * C, err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * C, err, errlen, kind);
  }
  case BNN_OP_SE_GATE: {
    const int C = p[0], rd = p[1];
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * rd * C, err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * rd, err, errlen, kind) ||
           upload((void **)&d->f[2], tptr(c, op, 2), sizeof(float) * rd * C, err, errlen, kind) ||
           upload((void **)&d->f[3], tptr(c, op, 3), sizeof(float) * C, err, errlen, kind);
  }
  case BNN_OP_C0POOL: { /* panels [Np/8][64][8] -> k-major [64][24] */
    const float *src = tptr(c, op, 0);
    float wt[64 * 24];
    for (int k = 0; k < 64; k++)
      for (int n = 0; n < 24; n++) wt[k * 24 + n] = src[((size_t)(n / 8) * 64 + k) * 8 + n % 8];
    return upload((void **)&d->f[0], wt, sizeof wt, err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * 24, err, errlen, kind);
  }
  case BNN_OP_POSTPC: { /* panels [128][1728][8] -> k-major [1728][1024] */
    const float *src = tptr(c, op, 2);
    float *wt = malloc(sizeof(float) * 1728 * 1024);
    if (!wt) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (pc weights)"); return -1; }
    for (int n = 0; n < 1024; n++)
      for (int k = 0; k < 1728; k++) wt[(size_t)k * 1024 + n] = src[((size_t)(n / 8) * 1728 + k) * 8 + n % 8];
    int rc = upload((void **)&d->f[0], wt, sizeof(float) * 1728 * 1024, err, errlen, kind);
    free(wt);
    return rc || upload((void **)&d->f[1], tptr(c, op, 3), sizeof(float) * 1024, err, errlen, kind) ||
           upload((void **)&d->f[2], tptr(c, op, 0), sizeof(float) * 192, err, errlen, kind) ||
           upload((void **)&d->f[3], tptr(c, op, 1), sizeof(float) * 192, err, errlen, kind);
  }
  case BNN_OP_FE_STFT2:
    return fe_tables(c, dv, op, err, errlen, kind);
  case BNN_OP_FE_LOGMEL: {
    const float *k = tptr(c, op, 2);
    return bnn_logmel_build(d, p[0], p[1], p[2], p[3], p[4], p[5], tptr(c, op, 0), tptr(c, op, 1), k[0], k[1], err,
                            errlen, kind);
  }
  case BNN_OP_FE_DBIMG:
    return bnn_dbimg_build(d, p, tptr(c, op, 0), tptr(c, op, 1), tptr(c, op, 2), tptr(c, op, 3), c->batch, err, errlen,
                           kind);
  case BNN_OP_PROTO_S8:
    return bnn_proto_weights(d, p[0], p[2], p[3], tptr(c, op, 0), tptr(c, op, 1), tptr(c, op, 3), tptr(c, op, 4),
                             p[7], ((const float *)tptr(c, op, 5))[0], err, errlen, kind);
  case BNN_OP_C0POOL_F16: /* t = [w b32 b16]; p = [24 64 64 24] */
    return bnn_hpack_weights(d, 0, tptr(c, op, 0), tptr(c, op, 1), tptr(c, op, 2), 64, 24, NULL, err, errlen, kind);
  case BNN_OP_PW_F16: {
    int rc = bnn_hpack_weights(d, 1, tptr(c, op, 0), tptr(c, op, 1), tptr(c, op, 2), p[2], p[3], &d->f[0], err, errlen,
                               kind);
    if (!rc && c->f16_tensor) rc = bnn_hpack_kmajor(d, tptr(c, op, 0), p[2], p[3], err, errlen, kind);
    return rc;
  }
  case BNN_OP_DW3_F16: {
    const int C = p[2];
    return upload((void **)&d->hw, tptr(c, op, 0), sizeof(uint16_t) * 9 * C, err, errlen, kind) ||
           upload((void **)&d->hb, tptr(c, op, 1), sizeof(uint16_t) * C, err, errlen, kind);
  }
  case BNN_OP_SE_F16: {
    const int C = p[0], rd = p[1];
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * rd * C, err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * rd, err, errlen, kind) ||
           upload((void **)&d->f[2], tptr(c, op, 2), sizeof(float) * rd * C, err, errlen, kind) ||
           upload((void **)&d->f[3], tptr(c, op, 3), sizeof(float) * C, err, errlen, kind);
  }
  case BNN_OP_POSTPC_F16: /* t = [post_s post_b w b32 b16] */
    return bnn_hpack_weights(d, 1, tptr(c, op, 2), tptr(c, op, 3), tptr(c, op, 4), 1728, 1024, &d->f[1], err, errlen, kind) ||
           upload((void **)&d->f[2], tptr(c, op, 0), sizeof(float) * 192, err, errlen, kind) ||
           upload((void **)&d->f[3], tptr(c, op, 1), sizeof(float) * 192, err, errlen, kind);
  case BNN_OP_DENSE_F16:
    return upload((void **)&d->hw, tptr(c, op, 0), sizeof(uint16_t) * 1024 * (size_t)p[0], err, errlen, kind) ||
           upload((void **)&d->f[0], tptr(c, op, 1), sizeof(float) * (size_t)p[0], err, errlen, kind);
  case BNN_OP_STEM_F16: /* t = [w panels [Np/8][Kp][8], b [Np]] fp32, used as they are */
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * (size_t)p[3] * p[2], err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * (size_t)p[3], err, errlen, kind);
  case BNN_OP_PW:
  case BNN_OP_STEM:  /* t = [w panels [Np/8][Kp][8], b [Np]] */
  case BNN_OP_CONVK:
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * (size_t)p[3] * p[2], err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * (size_t)p[3], err, errlen, kind);
  case BNN_OP_DWK: {
    const int C = p[2], k = p[3];
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * (size_t)k * k * C, err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * C, err, errlen, kind);
  }
  case BNN_OP_GEM:
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * 3, err, errlen, kind);
  case BNN_OP_SED: { /* t = [dw, db, fc w b, att w b, cla w b, consts]; p = [fc, att, cla shapes, red H W C ld L pk dk hc] */
    const int C = p[15], dk = p[19];
    const size_t sz[9] = {(size_t)(dk ? dk : 1) * C, (size_t)C, (size_t)p[3] * p[2], (size_t)p[3], (size_t)p[7] * p[6],
                          (size_t)p[7], (size_t)p[11] * p[10], (size_t)p[11], 3};
    for (int i = 0; i < 9; i++)
      if (upload((void **)&d->f[i], tptr(c, op, i), sizeof(float) * sz[i], err, errlen, kind)) return -1;
    return 0;
  }
  case BNN_OP_SED_S8: { /* t = [dw, db, fc (w sw cs b), att (4), cla (4), consts]; p as SED */
    const int C = p[15], dk = p[19];
    if (upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * (size_t)(dk ? dk : 1) * C, err, errlen, kind) ||
        upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * C, err, errlen, kind) ||
        upload((void **)&d->f[2], tptr(c, op, 14), sizeof(float) * 3, err, errlen, kind))
      return -1;
    bnn_devop *sub = calloc(3, sizeof(bnn_devop));
    if (!sub) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (SED int8 GEMMs)"); return -1; }
    d->sub = sub;
    for (int g = 0; g < 3; g++) {
      const int *q = p + 4 * g, t0 = 2 + 4 * g;
      if (bnn_s8_weights(&sub[g], q[0], q[1], q[2], q[3], tptr(c, op, t0), tptr(c, op, t0 + 1), tptr(c, op, t0 + 2),
                         tptr(c, op, t0 + 3), c->batch * p[17], err, errlen, kind))
        return -1;
    }
    return 0;
  }
  case BNN_OP_CONVW: { /* t = [U [36][Np/8][C][8], bias [Np]]; the transform scratch of the batch */
    const int C = p[0], Np = p[2], H = p[3], W = p[4];
    if (upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * 36 * (size_t)Np * C, err, errlen, kind) ||
        upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * (size_t)Np, err, errlen, kind))
      return -1;
    CK(dmalloc((void **)&d->f[2], sizeof(float) * bnnk_convw_scratch_floats(H, W, C, Np) * (size_t)c->batch),
       "Winograd scratch");
    return 0;
  }
  case BNN_OP_DWK_F16: {
    const int C = p[2], k = p[3];
    return upload((void **)&d->hw, tptr(c, op, 0), sizeof(uint16_t) * (size_t)k * k * C, err, errlen, kind) ||
           upload((void **)&d->hb, tptr(c, op, 1), sizeof(uint16_t) * C, err, errlen, kind);
  }
  case BNN_OP_PROTO_F16S8: /* t = [qw [Np/12][K/4][12][4], sw, cls w, cls b, eps]; p = [N K Np, P C ld nc ppc] */
    return bnn_proto_weights_l(d, 1, p[0], p[1], R16(p[1]), p[2], tptr(c, op, 0), tptr(c, op, 1), tptr(c, op, 2),
                               tptr(c, op, 3), p[6], ((const float *)tptr(c, op, 4))[0], err, errlen, kind);
  case BNN_OP_DENSE:
    return upload((void **)&d->f[0], tptr(c, op, 0), sizeof(float) * 1024 * (size_t)p[0], err, errlen, kind) ||
           upload((void **)&d->f[1], tptr(c, op, 1), sizeof(float) * (size_t)p[0], err, errlen, kind);
  default:
    return 0;
  }
}

/* ops i and i + 1 are a PW_S8 pair whose quantizer the GEMM of op i can run: op i + 1 is ungated and reads op i's
 * output rows (same rows per window, its lda op i's ldo, no halo) over K columns, K % 4 == 0, K <= 256, K <= op i's N.
 * (Whether op i's GEMM holds whole rows per tile depends on the batch: the set-up checks its plan.) */
static int pw_pair(const bnn_ctx *c, int i) {
  if (i < 0 || i + 1 >= c->n_ops) return 0;
  const bnn_op *a = &c->ops[i], *b = &c->ops[i + 1];
  if (a->code != BNN_OP_PW_S8 || b->code != BNN_OP_PW_S8 || (b->nb == 7 && b->b[6] >= 0)) return 0;
  if (a->nb < 2 || a->b[1] < 0 || b->b[0] != a->b[1] || c->bufd[a->b[1]].halo) return 0;
  const int *pa = a->p, *pb = b->p;
  return pb[4] == pa[4] && pb[5] == pa[7] && pa[9] == 0 && pb[1] > 0 && pb[1] % 4 == 0 && pb[1] <= 256 &&
         pb[1] <= pa[0];
}

int bnn_rt_device(bnn_ctx *c, int di, char *err, size_t errlen, int *kind) {
  *kind = BNN_ERR_CPU;
  bnn_dev *dv = calloc(1, sizeof *dv);
  if (!dv) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory (device state)"); return -1; }
  c->dev[di] = dv;
  dv->dev = c->dev_ids[di];
  const bnn_path_rec *d = c->path;
  const int B = c->batch;
  CK(cudaSetDevice(dv->dev), "cudaSetDevice");
  int major = 0, minor = 0;
  CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dv->dev), "device query");
  CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dv->dev), "device query");
  if (major != 10 || minor != 0) {
    *kind = BNN_ERR_CPU;
    snprintf(err, errlen, "GPU %d has compute capability %d.%d, this library is built for sm_100a (B200) only; hint: "
             "run on a B200", dv->dev, major, minor);
    return -1;
  }
  CK(cudaStreamCreateWithFlags((cudaStream_t *)&dv->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  CK(bnnk_device_init(), "device tables");
  dv->buf = calloc(d->n_buf, sizeof(void *));
  dv->priv = calloc(d->n_buf, sizeof(void *));
  dv->ws = calloc(d->n_buf, sizeof(long long));
  dv->ops = calloc(c->n_ops, sizeof(bnn_devop));
  if (!dv->buf || !dv->priv || !dv->ws || !dv->ops) { *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory"); return -1; }
  /* activation memory */
  size_t *slot_bytes = calloc(d->n_buf, sizeof(size_t));
  size_t *slot_off = calloc(d->n_buf, sizeof(size_t));
  if (!slot_bytes || !slot_off) { free(slot_bytes); free(slot_off); *kind = BNN_ERR_OOM; snprintf(err, errlen, "out of memory"); return -1; }
  for (uint32_t i = 0; i < d->n_buf; i++) {
    const bnn_buf_rec *b = &c->bufd[i];
    if (i == d->in_buf || b->halo || is_scratch(c, (int)i)) continue;
    const size_t bytes = ((size_t)b->elems * dsize(b->dtype) + 255) & ~(size_t)255;
    if (bytes > slot_bytes[b->slot]) slot_bytes[b->slot] = bytes;
  }
  size_t total = 0;
  for (uint32_t s = 0; s < d->n_buf; s++) { slot_off[s] = total; total += slot_bytes[s] * (size_t)B; }
  cudaError_t e = dmalloc(&dv->arena, total ? total : 256);
  if (!e) e = cudaMemset(dv->arena, 0, total ? total : 256);
  if (e) { free(slot_bytes); free(slot_off); return cerr(err, errlen, kind, e, "activation arena"); }
  for (uint32_t i = 0; i < d->n_buf; i++) {
    const bnn_buf_rec *b = &c->bufd[i];
    const size_t es = dsize(b->dtype);
    if (i == d->in_buf) {
      dv->ws[i] = (long long)b->elems;
      e = dmalloc(&dv->priv[i], (size_t)b->elems * es * B + 256);
      dv->buf[i] = dv->priv[i];
    } else if (b->halo) {
      dv->ws[i] = (long long)(((size_t)b->elems * es + 255) / 256 * 256 / es);
      e = dmalloc(&dv->priv[i], (size_t)dv->ws[i] * es * B);
      if (!e) e = cudaMemset(dv->priv[i], 0, (size_t)dv->ws[i] * es * B);
      dv->buf[i] = dv->priv[i];
    } else if (!is_scratch(c, (int)i)) {
      dv->ws[i] = (long long)(slot_bytes[b->slot] / es);
      dv->buf[i] = (uint8_t *)dv->arena + slot_off[b->slot];
    }
    if (e) { free(slot_bytes); free(slot_off); return cerr(err, errlen, kind, e, "activation buffers"); }
  }
  free(slot_bytes);
  free(slot_off);
  /* int8 scratch, front-end and post-conv scratch, error word */
  size_t qbytes = 256, rows = 8;
  for (int i = 0; i < c->n_ops; i++) {
    const bnn_op *op = &c->ops[i];
    if (op->code == BNN_OP_PROTO_F16S8) { /* p = [N K Np, P C ld nc ppc]: cells of K rounded up to 16 */
      const size_t r = (size_t)B * op->p[3], qb = r * (size_t)R16(op->p[1]);
      if (qb > qbytes) qbytes = qb;
      if (r > rows) rows = r;
      continue;
    }
    if (op->code == BNN_OP_SED_S8) { /* rows = B x L; the fc rows (K = C) and the att / cla rows (K = fc N) */
      const size_t r = (size_t)B * op->p[17], qb = r * (size_t)(R32(op->p[1]) > R32(op->p[5]) ? R32(op->p[1]) : R32(op->p[5]));
      if (qb > qbytes) qbytes = qb;
      if (r > rows) rows = r;
      continue;
    }
    if (op->code != BNN_OP_PW_S8 && op->code != BNN_OP_GEMV_S8 && op->code != BNN_OP_PROTO_S8) continue;
    const size_t r = (size_t)B * (op->code == BNN_OP_GEMV_S8 ? 1 : (size_t)op->p[4]);
    const size_t qb = r * (op->code == BNN_OP_PROTO_S8 ? (size_t)op->p[2] : (size_t)R32(op->p[1]));
    if (qb > qbytes) qbytes = qb;
    if (r > rows) rows = r;
  }
  /* the second scratch: the expand layers of PW_S8 pairs, whose rows the pwl GEMM before quantizes when
   * BNN_PW_FUSE=1. Off by default: on the v2.4 package at batch 256 the 13 fused pwl epilogues took longer than the
   * 13 quantizer launches they replace (PW_S8 class 2.41 ms per step fused, 2.37 ms separate) */
  size_t qbytes2 = 0, rows2 = 0;
  if (getenv("BNN_PW_FUSE") && !strcmp(getenv("BNN_PW_FUSE"), "1"))
    for (int i = 0; i + 1 < c->n_ops; i++)
      if (pw_pair(c, i)) {
        const bnn_op *op = &c->ops[i + 1];
        const size_t r = (size_t)B * (size_t)op->p[4], qb = r * (size_t)R32(op->p[1]);
        if (qb > qbytes2) qbytes2 = qb;
        if (r > rows2) rows2 = r;
      }
  CK(dmalloc((void **)&dv->q, qbytes), "int8 row scratch");
  CK(cudaMemset(dv->q, 0, qbytes), "int8 row scratch");
  CK(dmalloc((void **)&dv->sa, sizeof(float) * rows), "int8 scale scratch");
  CK(dmalloc((void **)&dv->za, sizeof(int32_t) * rows), "int8 zero-point scratch");
  if (qbytes2) {
    CK(dmalloc((void **)&dv->q2, qbytes2), "int8 row scratch");
    CK(cudaMemset(dv->q2, 0, qbytes2), "int8 row scratch");
    CK(dmalloc((void **)&dv->sa2, sizeof(float) * rows2), "int8 scale scratch");
    CK(dmalloc((void **)&dv->za2, sizeof(int32_t) * rows2), "int8 zero-point scratch");
  }
  CK(dmalloc((void **)&dv->fe_minmax, sizeof(float) * 2 * B), "front-end scratch");
  CK(dmalloc((void **)&dv->pcin, sizeof(float) * 6 * 1728 * B), "post-conv scratch");
  size_t gate_elems = 8;
  for (int i = 0; i < c->n_ops; i++)
    if (c->ops[i].code == BNN_OP_SE_F16 && (size_t)B * c->ops[i].p[0] > gate_elems) gate_elems = (size_t)B * c->ops[i].p[0];
  CK(dmalloc((void **)&dv->g16, sizeof(uint16_t) * gate_elems), "SE gate scratch");
  CK(dmalloc((void **)&dv->err, 2 * sizeof(int)), "error word");
  CK(cudaMemset(dv->err, 0, sizeof(int)), "error word");
  CK(cudaMemset(dv->err + 1, 0x7f, sizeof(int)), "error word");
  CK(cudaMallocHost((void **)&dv->err_host, 2 * sizeof(int)), "error word (host)");
  dv->err_host[0] = 0;
  dv->err_host[1] = BNNK_NO_FAIL;
  /* weights and GEMM plans */
  for (int i = 0; i < c->n_ops; i++) {
    if (op_weights(c, dv, i, err, errlen, kind)) return -1;
    const bnn_op *op = &c->ops[i];
    if (op->code == BNN_OP_PW_S8 || op->code == BNN_OP_GEMV_S8) {
      bnn_devop *o = &dv->ops[i];
      const int r = B * (op->code == BNN_OP_PW_S8 ? op->p[4] : 1);
      /* the expand of a pair whose pwl GEMM holds whole rows (one N tile) and stores 16-byte aligned rows: its rows
       * come quantized from that GEMM into the second scratch */
      if (dv->q2 && pw_pair(c, i - 1) && bnnk_gemm_n_tiles(&dv->ops[i - 1].plan) == 1) {
        const bnn_op *pl = &c->ops[i - 1];
        const uint32_t ob = (uint32_t)pl->b[1];
        if (((uintptr_t)dv->buf[ob] & 15) == 0 && dv->ws[ob] % 4 == 0 && pl->p[7] % 4 == 0) {
          o->qsel = 1;
          dv->ops[i - 1].qnext = 1;
          dv->fused_q++;
        }
      }
      if (bnnk_gemm_plan_init(&o->plan, o->qsel ? dv->q2 : dv->q, r, o->kq, o->w, op->p[0], op->p[3])) {
        *kind = BNN_ERR_CPU;
        snprintf(err, errlen, "op %d %s: TMA descriptors could not be made (driver too old?)", i, op->kname);
        return -1;
      }
    }
    if (op->code == BNN_OP_SED_S8) {
      bnn_devop *sub = dv->ops[i].sub;
      for (int g = 0; g < 3; g++)
        if (bnnk_gemm_plan_init(&sub[g].plan, dv->q, B * op->p[17], sub[g].kq, sub[g].w, op->p[4 * g], op->p[4 * g + 3])) {
          *kind = BNN_ERR_CPU;
          snprintf(err, errlen, "op %d %s: TMA descriptors could not be made (driver too old?)", i, op->kname);
          return -1;
        }
    }
    if (op->code == BNN_OP_PROTO_S8 || op->code == BNN_OP_PROTO_F16S8) {
      bnn_devop *o = &dv->ops[i];
      const int v2 = op->code == BNN_OP_PROTO_F16S8;
      const int np = v2 ? op->p[2] : op->p[3], kp = v2 ? R16(op->p[1]) : op->p[2], P = v2 ? op->p[3] : op->p[4];
      if (bnnk_proto_plan_init(&o->pplan, o->w, np, kp, dv->q, B, P)) {
        *kind = BNN_ERR_CPU;
        snprintf(err, errlen, "op %d %s: TMA descriptors could not be made (driver too old?)", i, op->kname);
        return -1;
      }
      if (!o->pplan.wt)
        CK(dmalloc((void **)&o->f[0], sizeof(float) * (size_t)B * o->pplan.nch * np), "prototype scratch");
    }
  }
  c->launches_fused = dv->fused_q;
  CK(cudaDeviceSynchronize(), "device set-up");
  return 0;
}

void bnn_rt_device_free(bnn_ctx *c, int di) {
  bnn_dev *dv = c->dev[di];
  if (!dv) return;
  cudaSetDevice(dv->dev);
  if (dv->stream) cudaStreamSynchronize((cudaStream_t)dv->stream);
  if (dv->ops)
    for (int i = 0; i < c->n_ops; i++) {
      bnn_devop *o = &dv->ops[i];
      cudaFree(o->w); cudaFree(o->sw); cudaFree(o->bias); cudaFree(o->cs);
      for (int k = 0; k < 10; k++) cudaFree(o->f[k]);
      if (o->sub) {
        bnn_devop *sub = o->sub;
        for (int g = 0; g < 3; g++) { cudaFree(sub[g].w); cudaFree(sub[g].sw); cudaFree(sub[g].bias); cudaFree(sub[g].cs); }
        free(sub);
        o->sub = NULL;
      }
      cudaFree(o->hw); cudaFree(o->hb); cudaFree(o->hwd); cudaFree(o->hwk);
      bnn_logmel_release(o);
      bnn_dbimg_release(o);
    }
  for (int k = 0; k < dv->n_fe_mem; k++) cudaFree(dv->fe_mem[k]);
  if (dv->events)
    for (int k = 0; k < 2 * c->n_ops; k++)
      if (dv->events[k]) cudaEventDestroy((cudaEvent_t)dv->events[k]);
  free(dv->events);
  free(dv->op_ms);
  if (dv->priv)
    for (uint32_t i = 0; i < c->path->n_buf; i++) cudaFree(dv->priv[i]);
  cudaFree(dv->arena);
  cudaFree(dv->q); cudaFree(dv->sa); cudaFree(dv->za); cudaFree(dv->fe_minmax); cudaFree(dv->pcin); cudaFree(dv->err);
  cudaFree(dv->q2); cudaFree(dv->sa2); cudaFree(dv->za2);
  cudaFree(dv->g16);
  if (dv->err_host) cudaFreeHost(dv->err_host);
  cudaFree(dv->up[0]); cudaFree(dv->up[1]);
  for (int k = 0; k < 2; k++) {
    if (dv->up_ready[k]) cudaEventDestroy((cudaEvent_t)dv->up_ready[k]);
    if (dv->up_free[k]) cudaEventDestroy((cudaEvent_t)dv->up_free[k]);
    if (dv->up_half[k]) cudaEventDestroy((cudaEvent_t)dv->up_half[k]);
  }
  for (int k = 0; k < dv->n_graphs; k++)
    if (dv->graphs[k].exec) cudaGraphExecDestroy((cudaGraphExec_t)dv->graphs[k].exec);
  if (dv->up_stream) cudaStreamDestroy((cudaStream_t)dv->up_stream);
  if (dv->up_stream2) cudaStreamDestroy((cudaStream_t)dv->up_stream2);
  if (dv->stream) cudaStreamDestroy((cudaStream_t)dv->stream);
  free(dv->buf); free(dv->priv); free(dv->ws); free(dv->ops);
  free(dv);
  c->dev[di] = NULL;
}

/* ------------------------------------------------------------------ one batch */

#define B_(a) (op->b[a] < 0 ? NULL : dv->buf[op->b[a]])
#define WS(a) (op->b[a] < 0 ? 0 : dv->ws[op->b[a]])

/* op i is a C0POOL whose output rows the ungated PW_S8 op i + 1 quantizes (K = 48): the C0POOL launch quantizes
 * them itself */
int c0_quantizes_next(const bnn_ctx *c, int i) {
  if (i + 1 >= c->n_ops) return 0;
  const bnn_op *a = &c->ops[i], *b = &c->ops[i + 1];
  return a->code == BNN_OP_C0POOL && b->code == BNN_OP_PW_S8 && a->nb > 1 && a->b[1] >= 0 && b->b[0] == a->b[1] &&
         !(b->nb == 7 && b->b[6] >= 0) && b->p[1] == 48 && b->p[5] == 48 && b->p[4] == 6144;
}

/* buffer buf is an argument of some op other than i and j */
static int used_elsewhere(const bnn_ctx *c, int buf, int i, int j) {
  for (int k = 0; k < c->n_ops; k++)
    if (k != i && k != j)
      for (int a = 0; a < c->ops[k].nb; a++)
        if (c->ops[k].b[a] == buf) return 1;
  return 0;
}

int bnn_rt_launch(bnn_ctx *c, int di, int n, const float *d_pcm, int op0, int op1, void *stream) {
  bnn_dev *dv = c->dev[di];
  bnn_stream_t st = (bnn_stream_t)stream;
  const uint32_t in = c->path->in_buf;
  if (dv->prof_on) {
    dv->prof_op0 = op0;
    dv->prof_op1 = op1 < c->n_ops ? op1 : c->n_ops;
  }
  int pre_q = 0;  /* this op's input rows were quantized by the launch of the op before */
  int n_fq = 0;   /* PW_S8 ops run as one launch */
  for (int i = op0; i < op1 && i < c->n_ops; i++) {
    const bnn_op *op = &c->ops[i];
    const bnn_devop *o = &dv->ops[i];
    const int *p = op->p;
    int rc = 0, next_q = 0;
    if (dv->prof_on) cudaEventRecord((cudaEvent_t)dv->events[2 * i], (cudaStream_t)st);
#define IN_(a) ((uint32_t)op->b[a] == in ? (const float *)d_pcm : (const float *)B_(a))
#define INWS(a) ((uint32_t)op->b[a] == in ? (long long)c->bufd[in].elems : WS(a))
    switch (op->code) {
    case BNN_OP_FE_STFT2:
      rc = bnnk_fe_stft2(n, IN_(0), INWS(0), &dv->fe, dv->fe_minmax, B_(1), WS(1), st);
      break;
    case BNN_OP_C0POOL: {
      bnnk_qrows qr = {dv->q, dv->sa, dv->za, 0, 1};
      if (i + 1 < op1 && c0_quantizes_next(c, i)) {
        qr.kq = dv->ops[i + 1].kq;
        qr.keep = used_elsewhere(c, op->b[1], i, i + 1);
        next_q = 1;
      }
      rc = bnnk_c0pool(n, IN_(0), INWS(0), o->f[0], o->f[1], B_(1), WS(1), next_q ? &qr : NULL, st);
      break;
    }
    case BNN_OP_PW_S8: {
      const int M = p[4];
      const float *gate = op->nb == 7 && op->b[6] >= 0 ? B_(6) : NULL;
      int8_t *qq = o->qsel ? dv->q2 : dv->q;
      float *qs = o->qsel ? dv->sa2 : dv->sa;
      int32_t *qz = o->qsel ? dv->za2 : dv->za;
      const bnn_buf_rec *r = op->b[2] >= 0 ? &c->bufd[op->b[2]] : NULL;
      bnnk_epilogue e = {p[6], B_(1), WS(1), p[7], p[8], p[9], B_(2), WS(2), p[10],
                         r && r->halo ? (int)r->W : 0, r && r->halo ? (int)r->halo : 0, o->sw, o->bias, o->cs,
                         NULL, NULL, NULL, 0, 0};
      if (!pre_q && !gate && !(o->qnext && i + 1 < op1)) {  /* one launch: the quantizer inside the GEMM */
        rc = bnnk_pw_s8_fq(&o->plan, n * M, M, IN_(0), INWS(0), p[5], p[1], &e, dv->err, st);
        if (rc != BNNK_NOT_FUSED) {
          n_fq++;
          break;
        }
        rc = 0;
      }
      if (!pre_q)
        rc = bnnk_quant(n * M, M, IN_(0), INWS(0), p[5], p[1], o->kq, gate, gate ? WS(6) : 0, qq, qs, qz, dv->err, st);
      if (!rc) {
        if (o->qnext && i + 1 < op1) {  /* this GEMM quantizes its rows for the expand after it */
          e.qo = dv->q2;
          e.qsa = dv->sa2;
          e.qza = dv->za2;
          e.qk = c->ops[i + 1].p[1];
          e.qkq = dv->ops[i + 1].kq;
          next_q = 1;
        }
        rc = bnnk_gemm(&o->plan, n * M, M, qs, qz, &e, dv->err, st);
      }
      break;
    }
    case BNN_OP_GEMV_S8: {
      rc = bnnk_quant(n, 1, IN_(0), INWS(0), p[1], p[1], o->kq, NULL, 0, dv->q, dv->sa, dv->za, dv->err, st);
      if (!rc) {
        bnnk_epilogue e = {p[4], B_(1), WS(1), p[3], 0, 0, NULL, 0, 0, 0, 0, o->sw, o->bias, o->cs, NULL, NULL, NULL, 0, 0};
        rc = bnnk_gemm(&o->plan, n, 1, dv->sa, dv->za, &e, dv->err, st);
      }
      break;
    }
    case BNN_OP_DW3: { /* channel sums that no op reads are not formed in a whole-package run (debug ranges keep them) */
      const int sums = !(op0 == 0 && op1 >= c->n_ops) || used_elsewhere(c, op->b[2], i, i);
      rc = bnnk_dw3(n, IN_(0), INWS(0), p[0], p[1], p[2], p[3], o->f[0], o->f[1], B_(1), WS(1), p[4], p[5],
                    sums ? B_(2) : NULL, WS(2), dv->err, st);
      break;
    }
    case BNN_OP_SE_GATE:
      rc = bnnk_se_gate(n, p[0], p[1], o->f[0], o->f[1], o->f[2], o->f[3], IN_(0), INWS(0), p[2], B_(1), WS(1), st);
      break;
    case BNN_OP_POSTPC:
      rc = bnnk_postpc(n, IN_(0), INWS(0), o->f[2], o->f[3], o->f[0], o->f[1], dv->pcin, B_(1), WS(1), st);
      break;
    case BNN_OP_FE_DBIMG:
      rc = bnnk_dbimg(n, IN_(0), INWS(0), &o->db, o->db_scratch, B_(1), WS(1), st);
      break;
    case BNN_OP_FE_LOGMEL:
      rc = bnnk_logmel(n, IN_(0), INWS(0), &o->lm, B_(1), WS(1), st);
      break;
    case BNN_OP_PROTO_S8:
      rc = bnnk_proto_quant(n, p[4], IN_(0), INWS(0), p[6], p[5], p[2], o->eps, dv->q, dv->sa, st);
      if (!rc) rc = bnnk_proto_colmax(&o->pplan, n, dv->sa, o->sw, B_(3), WS(3), o->f[0], dv->err, st);
      if (!rc)
        rc = bnnk_proto_logits(n, p[7], p[8], B_(3), WS(3), o->f[1], o->f[2], B_(1), WS(1), NULL, dv->err + 1,
                               dv->w_base, st);
      break;
    case BNN_OP_C0POOL_F16:
      rc = bnnk_c0pool_f16(n, IN_(0), INWS(0), o->hw, o->hb, B_(1), WS(1), st);
      break;
    case BNN_OP_PW_F16: {
      const int M = p[4];
      if (o->hwk) { /* the tensor mode */
        rc = bnnk_gemm_tc16(n, M, B_(0), WS(0), p[5], o->hwk, p[2], p[3], o->f[0], p[6], B_(1), WS(1), p[7], p[8], p[9],
                            B_(2), WS(2), p[10], dv->err, st);
        break;
      }
      rc = bnnk_gemm_f16(n * M, M, B_(0), WS(0), p[5], o->hwd, p[2], p[3], o->hb, o->f[0], p[6], B_(1), WS(1), p[7],
                         p[8], p[9], B_(2), WS(2), p[10], st);
      break;
    }
    case BNN_OP_DW3_F16:
      rc = bnnk_dw3_f16(n, B_(0), WS(0), p[0], p[1], p[2], p[3], p[6], p[7], o->hw, o->hb, B_(1), WS(1), p[4], p[5],
                        B_(2), WS(2), dv->err, st);
      break;
    case BNN_OP_SE_F16:
      rc = bnnk_se_f16(n, p[0], p[1], o->f[0], o->f[1], o->f[2], o->f[3], B_(1), WS(1), p[2], B_(0), WS(0), dv->g16,
                       st);
      break;
    case BNN_OP_POSTPC_F16:
      rc = bnnk_postpc_f16(n, B_(0), WS(0), o->f[2], o->f[3], o->hwd, o->hb, o->f[1], B_(2), WS(2), B_(3), WS(3), B_(1),
                           WS(1), dv->err + 1, dv->w_base, st);
      break;
    case BNN_OP_DENSE_F16:
      rc = bnnk_dense_f16(n, p[0], B_(0), WS(0), o->hw, o->f[0], B_(1), WS(1), st);
      break;
    case BNN_OP_DENSE:
      rc = bnnk_dense_f32(n, p[0], B_(0), WS(0), o->f[0], o->f[1], B_(1), WS(1), st);
      break;
    case BNN_OP_PW: { /* pw_run (src/rt_ops_f32.c:193-206) */
      const bnn_buf_rec *ob = &c->bufd[op->b[1]], *r = op->b[2] >= 0 ? &c->bufd[op->b[2]] : NULL;
      const float *gate = op->nb == 4 && op->b[3] >= 0 ? IN_(3) : NULL;
      rc = bnnk_pw_f32(n, IN_(0), INWS(0), p[5], p[4], gate, gate ? INWS(3) : 0, o->f[0], o->f[1], p[2], p[3], p[6],
                       B_(1), WS(1), p[7], p[8], p[9], (int)ob->H, (int)ob->W, r ? IN_(2) : NULL, r ? INWS(2) : 0,
                       p[10], r && r->halo ? (int)r->W : 0, r ? (int)r->halo : 0, st);
      break;
    }
    case BNN_OP_STEM: /* the GEMM reads the image itself: the im2col rows are written only for another op */
      rc = bnnk_stem_f32(n, IN_(0), INWS(0), p[5], p[8], p[9], p[6], p[7], o->f[0], o->f[1], p[2], p[3], p[10], B_(1),
                         WS(1), p[11], p[12], used_elsewhere(c, op->b[2], i, i) ? B_(2) : NULL, WS(2), st);
      break;
    case BNN_OP_DWK:
      rc = bnnk_dwk_f32(n, IN_(0), INWS(0), p[0], p[1], p[2], p[3], p[4], p[5], p[6], o->f[0], o->f[1], p[9], B_(1),
                        WS(1), p[7], p[8], B_(2), WS(2), st);
      break;
    case BNN_OP_PAD:
      rc = bnnk_pad_f32(n, p[0], p[1], p[2], p[3], p[4], IN_(0), INWS(0), B_(1), WS(1), st);
      break;
    case BNN_OP_MEAN:
      rc = bnnk_mean_f32(n, p[0], p[1], p[2], IN_(0), INWS(0), B_(1), WS(1), st);
      break;
    case BNN_OP_CONVK: {
      const bnn_buf_rec *x = &c->bufd[op->b[0]], *r = op->b[2] >= 0 ? &c->bufd[op->b[2]] : NULL;
      rc = bnnk_convk(n, IN_(0), INWS(0), p[4], p[5], (int)x->halo, (int)x->ld, p[6], p[7], p[8], p[9], p[10], p[11],
                      p[12], o->f[0], o->f[1], p[2], p[3], p[13], B_(1), WS(1), p[14], p[15], r ? IN_(2) : NULL,
                      r ? INWS(2) : 0, r ? (int)r->ld : 0, r ? (int)r->halo : 0, st);
      break;
    }
    case BNN_OP_GEM:
      rc = bnnk_gem(n, p[0], p[1], p[2], IN_(0), INWS(0), o->f[0], B_(1), WS(1), st);
      break;
    case BNN_OP_VADD:
      rc = bnnk_vadd(n, p[0], IN_(0), INWS(0), IN_(1), INWS(1), B_(2), WS(2), st);
      break;
    case BNN_OP_SED: {
      bnnk_sed_args a = {p[12], p[13], p[14], p[15], p[16], p[17], p[18], p[19], p[20], p[2], IN_(0), INWS(0),
                         o->f[0], o->f[1], o->f[8],
                         {p[0], p[1], p[2], p[3], o->f[2], o->f[3]}, {p[4], p[5], p[6], p[7], o->f[4], o->f[5]},
                         {p[8], p[9], p[10], p[11], o->f[6], o->f[7]},
                         B_(1), B_(2), B_(3), B_(4), B_(5), B_(6), WS(1), WS(2), WS(3), WS(4), WS(5), WS(6)};
      rc = bnnk_sed(n, &a, st);
      break;
    }
    case BNN_OP_SED_S8: { /* sed8_run (src/rt_ops_s8n.c:186-210): pool, quantize, fc + ReLU, quantize, att, cla, out */
      bnn_devop *sub = o->sub;
      const int L = p[17], C = p[15], Cp = R8(C);
      bnnk_sed_args a = {p[12], p[13], p[14], p[15], p[16], p[17], p[18], p[19], p[20], Cp, IN_(0), INWS(0),
                         o->f[0], o->f[1], o->f[2],
                         {p[0], p[1], p[2], p[3], NULL, NULL}, {p[4], p[5], p[6], p[7], NULL, NULL},
                         {p[8], p[9], p[10], p[11], NULL, NULL},
                         B_(1), B_(2), B_(3), B_(4), B_(5), B_(6), WS(1), WS(2), WS(3), WS(4), WS(5), WS(6)};
      rc = bnnk_sed_pool(n, &a, st);
      if (!rc) rc = bnnk_quant(n * L, L, B_(3), WS(3), Cp, C, sub[0].kq, NULL, 0, dv->q, dv->sa, dv->za, dv->err, st);
      if (!rc) {
        bnnk_epilogue e = {2, B_(4), WS(4), p[3], 0, 0, NULL, 0, 0, 0, 0, sub[0].sw, sub[0].bias, sub[0].cs,
                           NULL, NULL, NULL, 0, 0};
        rc = bnnk_gemm(&sub[0].plan, n * L, L, dv->sa, dv->za, &e, dv->err, st);
      }
      if (!rc) rc = bnnk_quant(n * L, L, B_(4), WS(4), p[3], p[0], sub[1].kq, NULL, 0, dv->q, dv->sa, dv->za, dv->err, st);
      for (int g = 1; g < 3 && !rc; g++) {
        bnnk_epilogue e = {0, B_(4 + g), WS(4 + g), p[4 * g + 3], 0, 0, NULL, 0, 0, 0, 0, sub[g].sw, sub[g].bias,
                           sub[g].cs, NULL, NULL, NULL, 0, 0};
        rc = bnnk_gemm(&sub[g].plan, n * L, L, dv->sa, dv->za, &e, dv->err, st);
      }
      if (!rc) rc = bnnk_sed_out(n, &a, st);
      break;
    }
    case BNN_OP_CONVW: {
      const bnn_buf_rec *x = &c->bufd[op->b[0]], *r = op->b[2] >= 0 ? &c->bufd[op->b[2]] : NULL;
      rc = bnnk_convw(n, IN_(0), INWS(0), p[3], p[4], (int)x->halo, p[0], o->f[0], o->f[1], p[2], p[5], B_(1), WS(1),
                      p[6], p[7], r ? IN_(2) : NULL, r ? INWS(2) : 0, r ? (int)r->halo : 0, r ? (int)r->ld : 0, o->f[2],
                      st);
      break;
    }
    case BNN_OP_STEM_F16:
      rc = bnnk_stem_f16(n, B_(0), WS(0), p[5], p[8], p[9], p[6], p[7], o->f[0], o->f[1], p[0], p[2], p[3], p[10],
                         B_(1), WS(1), p[11], p[12], st);
      break;
    case BNN_OP_DWK_F16:
      rc = bnnk_dwk_f16(n, B_(0), WS(0), p[1], p[2], p[3], p[4], p[5], p[6], o->hw, o->hb, p[9], B_(1), WS(1), p[7],
                        p[8], B_(2), WS(2), st);
      break;
    case BNN_OP_PAD_F16:
      rc = bnnk_pad_f16(n, p[0], p[1], p[2], p[3], p[4], B_(0), WS(0), B_(1), WS(1), st);
      break;
    case BNN_OP_MEAN_F16:
      rc = bnnk_mean_f16(n, p[0], p[1], p[2], B_(0), WS(0), B_(1), WS(1), st);
      break;
    case BNN_OP_PROTO_F16S8:
      rc = bnnk_proto_quant_h(n, p[3], B_(0), WS(0), p[5], p[1], R16(p[1]), o->eps, dv->q, dv->sa, st);
      if (!rc) rc = bnnk_proto_colmax(&o->pplan, n, dv->sa, o->sw, B_(3), WS(3), o->f[0], dv->err, st);
      if (!rc)
        rc = bnnk_proto_logits(n, p[6], p[7], B_(3), WS(3), o->f[1], o->f[2], B_(1), WS(1), NULL, dv->err + 1,
                               dv->w_base, st);
      break;
    default:
      rc = cudaErrorNotSupported;
    }
#undef IN_
#undef INWS
    if (dv->prof_on) cudaEventRecord((cudaEvent_t)dv->events[2 * i + 1], (cudaStream_t)st);
    if (rc) {
      bnn_set_error(BNN_ERR_WINDOW, "window not scored: op %d %s could not be launched (CUDA error %d: %s); hint: check "
                    "the GPU (nvidia-smi) and retry", i, op->kname, rc, cudaGetErrorString((cudaError_t)rc));
      return -1;
    }
    pre_q = next_q;
  }
  if (op0 == 0 && op1 >= c->n_ops) dv->launches_fq = n_fq;
  return 0;
}

/* Whole launch sequences as CUDA graphs. A 16-window sequence costs 1.4 ms against 5.2 ms for 256 windows: most of
 * it is the host side of 101 kernel launches, which a graph replays in one call. The graph bakes in every pointer,
 * grid and parameter of the sequence, so it is keyed by the window count, the input buffer and (for packages with an
 * op that reports failed windows relative to the call: a prototype head, the fp16 post conv) the first window of the
 * chunk.
 * The first run of a key is eager (it also sets the kernels' shared-memory attributes outside any capture); the
 * second is captured on the context's own stream, thread-locally, then launched on the caller's stream. */
int bnn_window_fail_op(const bnn_ctx *c) {
  for (int i = 0; i < c->n_ops; i++)
    if (c->ops[i].code == BNN_OP_PROTO_S8 || c->ops[i].code == BNN_OP_PROTO_F16S8 || c->ops[i].code == BNN_OP_POSTPC_F16)
      return i;
  return -1;
}

int bnn_rt_run(bnn_ctx *c, int di, int n, const float *d_pcm, void *stream) {
  bnn_dev *dv = c->dev[di];
  static int env = -1;
  if (env < 0) {
    const char *e = getenv("BNN_GRAPHS");
    env = !(e && atoi(e) == 0);
  }
  if (!env || dv->graphs_off || dv->prof_on) return bnn_rt_launch(c, di, n, d_pcm, 0, c->n_ops, stream);
  const int wb = bnn_window_fail_op(c) >= 0 ? dv->w_base : 0;
  int k = 0;
  while (k < dv->n_graphs && !(dv->graphs[k].n == n && dv->graphs[k].in == d_pcm && dv->graphs[k].w_base == wb)) k++;
  if (k == dv->n_graphs) {
    if (k == (int)(sizeof dv->graphs / sizeof dv->graphs[0])) { /* full: drop the oldest */
      if (dv->graphs[0].exec) cudaGraphExecDestroy((cudaGraphExec_t)dv->graphs[0].exec);
      memmove(dv->graphs, dv->graphs + 1, sizeof dv->graphs[0] * (size_t)(k - 1));
      k--;
    } else {
      dv->n_graphs++;
    }
    dv->graphs[k].n = n;
    dv->graphs[k].in = d_pcm;
    dv->graphs[k].w_base = wb;
    dv->graphs[k].seen = 0;
    dv->graphs[k].exec = NULL;
  }
  if (!dv->graphs[k].exec && !dv->graphs[k].seen++) return bnn_rt_launch(c, di, n, d_pcm, 0, c->n_ops, stream);
  if (!dv->graphs[k].exec) {
    cudaStream_t cs = (cudaStream_t)dv->stream;
    cudaGraph_t g = NULL;
    cudaGraphExec_t ex = NULL;
    if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      cudaGetLastError();
      dv->graphs_off = 1;
      return bnn_rt_launch(c, di, n, d_pcm, 0, c->n_ops, stream);
    }
    const int rc = bnn_rt_launch(c, di, n, d_pcm, 0, c->n_ops, cs);
    cudaError_t e = cudaStreamEndCapture(cs, &g);
    if (rc || e || !g || cudaGraphInstantiate(&ex, g, 0) != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      dv->graphs_off = 1; /* run eagerly from now on */
      return bnn_rt_launch(c, di, n, d_pcm, 0, c->n_ops, stream);
    }
    cudaGraphDestroy(g);
    dv->graphs[k].exec = ex;
  }
  const cudaError_t e = cudaGraphLaunch((cudaGraphExec_t)dv->graphs[k].exec, (cudaStream_t)stream);
  if (e) {
    bnn_set_error(BNN_ERR_WINDOW, "window not scored: the op list's CUDA graph could not be launched (CUDA error %d: "
                  "%s); hint: check the GPU (nvidia-smi) and retry", (int)e, cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

void bnn_rt_close(bnn_ctx *c) {
  for (int i = 0; i < 64; i++)
    if (c->dev[i]) bnn_rt_device_free(c, i);
  free(c->bufd);
  free(c->ops);
}
