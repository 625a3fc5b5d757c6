/* Launchers of the sm_100a kernels (C ABI, device pointers, one CUDA stream each). Called by the host runtime
 * (bnn_rt.c) and by the per-op entry points of include/bnneon_cuda.h. Every launcher returns 0 or a cudaError_t.
 *
 * Batched layout: a per-window buffer of the package (an activation, a vector) holds B windows at a fixed window
 * stride (elements). Rows of a 1x1 conv are the Mw pixels of each window; the GEMM works on all B * Mw rows at
 * once. */
#ifndef BNN_KERNELS_H
#define BNN_KERNELS_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *bnn_stream_t;

/* device-side error word written by kernels whose bounded waits time out (0 = none) */
enum { BNNK_ERR_NONE = 0, BNNK_ERR_TMA_WAIT = 1, BNNK_ERR_MMA_WAIT = 2, BNNK_ERR_EPI_WAIT = 3, BNNK_ERR_DW3_WAIT = 4,
       BNNK_ERR_QUANT_WAIT = 5 };
/* the failed-window word beside it: the smallest failed window index, or BNNK_NO_FAIL (every byte 0x7f, so that a
 * byte memset restores it) */
#define BNNK_NO_FAIL 0x7f7f7f7f

/* per device, once: the glibc expf table (computed on the host) and the FRECPE estimate table */
int bnnk_device_init(void);

/* ---- int8 1x1 conv / dense layer (PW_S8, GEMV_S8) */

/* per-row dynamic quantization (s8n_quant_rows, optionally gated): rows r = w * Mw + m of x (window stride xws,
 * row stride lda; gate [B][K] at window stride gws or NULL) -> q [rows][Kq] (Kq >= K, pads = zero point), sa, za.
 * err: the device error word for the forms with bounded waits (NULL: those forms are not used) */
int bnnk_quant(int rows, int Mw, const float *x, long long xws, int lda, int K, int Kq, const float *gate,
               long long gws, int8_t *q, float *sa, int32_t *za, int *err, bnn_stream_t st);

/* The GEMM of one layer: weights [Nrows][Kq] int8 (row n = output channel, zero beyond N and K), q [rows_cap][Kq].
 * The plan holds the TMA descriptors (opaque, 64-byte aligned) and the tiling. */
typedef struct {
  unsigned char tma_a[128] __attribute__((aligned(64)));
  unsigned char tma_b[128] __attribute__((aligned(64)));
  int kq, sw, nkb, stages, bn, n_tiles, n, np, tmem_cols;
  int ne, nh, sp;  /* TMEM accumulators, epilogue warps per lane quarter, parameters staged in shared memory */
  unsigned int idesc;
  size_t smem;
} bnnk_gemm_plan;
int bnnk_gemm_plan_init(bnnk_gemm_plan *p, const int8_t *q, int rows_cap, int kq, const int8_t *w, int n, int np);
/* rows of the weight buffer the plan of a layer with np (padded) output channels and rows_cap rows reads:
 * n_tiles * bn */
int bnnk_gemm_weight_rows(int np, int rows_cap);
/* N tiles of the plan's GEMM (1: each tile holds whole rows, so its epilogue can quantize them for the next layer) */
int bnnk_gemm_n_tiles(const bnnk_gemm_plan *p);
/* test hook: the next GEMM launch in this process issues no loads and its waits give up after 200 us */
void bnnk_debug_stall_next_gemm(void);

/* epilogue of PW_S8 (gemm_s8n.c:105-135): y = (float)(acc - za * cs) * (sw * sa) + b, act (0 none, 1 SiLU,
 * 2 ReLU), + residual, stored at the padded row of each pixel (ow / opad) of each window */
typedef struct {
  int act;
  float *out;
  long long ows;
  int ldo, ow, opad;
  const float *res;
  long long rws;
  int ldr, rw, rpad;
  const float *sw, *bias;
  const int32_t *cs;
  /* optional: the stored rows quantized for the ungated PW_S8 that reads them next (s8n_quant_rows over their first
   * qk columns, qk % 4 == 0, qk <= 256): q [rows][qkq], sa, za [rows]. Needs one N tile (every CTA tile holds whole
   * rows), an unpadded output (opad 0) with 16-byte aligned rows, and q distinct from this GEMM's own rows. */
  int8_t *qo;
  float *qsa;
  int32_t *qza;
  int qk, qkq;
} bnnk_epilogue;
int bnnk_gemm(const bnnk_gemm_plan *p, int rows, int Mw, const float *sa, const int32_t *za, const bnnk_epilogue *e,
              int *err, bnn_stream_t st);
/* the ungated PW_S8 in one launch, the quantizer inside the GEMM: x [B Mw][lda] fp32 rows (xws == Mw lda), K values
 * a row; BNNK_NOT_FUSED (nothing launched) when the layer is outside the form's limits */
#define BNNK_NOT_FUSED (-4242)
int bnnk_pw_s8_fq(const bnnk_gemm_plan *p, int rows, int Mw, const float *x, long long xws, int lda, int K,
                  const bnnk_epilogue *e, int *err, bnn_stream_t st);

/* the GEMM of a planned layer on quantized rows the caller holds: q [rows][ldq] (ldq % 16 == 0, the first kp bytes
 * of each row are the row, kp <= the plan's kq), sa, za [rows] */
int bnnk_gemm_q(const bnnk_gemm_plan *p, const int8_t *q, long long ldq, int kp, int rows, int Mw, const float *sa,
                const int32_t *za, const bnnk_epilogue *e, int *err, bnn_stream_t st);

/* quantizer + GEMM of a planned layer with q / sa / za in the file-scope static array of k_int8.cu instead of the
 * layer's own scratch; allocates nothing. At most BNNK_STATIC_ROWS rows and rows * kq <= BNNK_STATIC_QBYTES
 * (cudaErrorInvalidValue beyond). The first call on a device (rows = 0 does only this) looks up the array's address
 * there. Calls on one device share the array. */
#define BNNK_STATIC_ROWS 32768
#define BNNK_STATIC_QBYTES (4 << 20)
int bnnk_pw_s8_static(const bnnk_gemm_plan *p, int rows, int Mw, const float *x, long long xws, int lda, int K,
                      const float *gate, long long gws, const bnnk_epilogue *e, int *err, bnn_stream_t st);

/* ---- depthwise 3x3 + SiLU + channel sums (DW3): xp [B][(H+2)(W+2)][C] haloed, out [B][Ho Wo][C], chsum [B][C].
 * err: the device error word a timed-out input wait is reported in (NULL: not reported) */
int bnnk_dw3(int B, const float *xp, long long xws, int H, int W, int C, int s, const float *w, const float *b,
             float *out, long long ows, int Ho, int Wo, float *chsum, long long cws, int *err, bnn_stream_t st);

/* ---- SE gate (SE_GATE): chsum [B][C] -> gate [B][C] */
int bnnk_se_gate(int B, int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                 const float *chsum, long long cws, int P, float *gate, long long gws, bnn_stream_t st);

/* a producer kernel's quantization of its output rows for the PW_S8 that reads them next (s8n_quant_rows): q
 * [rows][kq], sa, za; keep = 0: the fp32 rows are not written (no other op reads them) */
typedef struct {
  int8_t *q;
  float *sa;
  int32_t *za;
  int kq, keep;
} bnnk_qrows;

/* ---- c0 conv 4x8 s2 + ReLU + max|avg pool (C0POOL): img [B][96][511][2] -> pin [B][6144][48];
 * wt: the weights k-major [64][24], b [24]; qr (or NULL): the rows quantized for the next op too */
int bnnk_c0pool(int B, const float *img, long long iws, const float *wt, const float *b, float *pin, long long pws,
                const bnnk_qrows *qr, bnn_stream_t st);

/* ---- post BN + ReLU + pc 3x3 conv + ReLU + mean (POSTPC): X [B][24][192] -> feat [B][1024];
 * wt: pc weights k-major [1728][1024]; pcin: scratch [B][6][1728] */
int bnnk_postpc(int B, const float *X, long long xws, const float *post_s, const float *post_b, const float *wt,
                const float *b, float *pcin, float *feat, long long fws, bnn_stream_t st);

/* ---- the v2.4 front end (FE_STFT2): pcm [B][144000] -> img [B][96][511][2] */
typedef struct {
  const float *win[2];        /* [M][2]: the window pairs (w[2n], w[2n+1]) in gather order: entry e * (M / 16) + l
                               * holds bit-reversed position p = 16 l + e, n = rev(p) */
  const float *tw_re[2], *tw_im[2]; /* [M / 2] */
  const float *tw_st[2];      /* [4 + 16 + 64 + 256][4]: per radix-2^2 stage (len 8, 32, 128, 512) and group index j,
                               * (w1, w2) = (tw[j M / len], tw[j M / (2 len)]) as (re, im, re, im) */
  const float *pc[2], *ps[2]; /* [khi] */
  const int *rev[2];          /* [M] */
  const int *mel_off[2];      /* [97] */
  const int *mel_k[2];
  const float *mel_w[2];
  int klo[2], khi[2];
  float pw2[2], bn_s[2], bn_b[2];
} bnnk_fe_tables;
int bnnk_fe_stft2(int B, const float *pcm, long long pws, const bnnk_fe_tables *t, float *minmax, float *img,
                  long long iws, bnn_stream_t st);

/* ---- the framed log-mel front end (FE_LOGMEL): pcm [B][nsamp] -> spec [B][nfr][nmel]. Device tables: window
 * [nfft] (zero past frame), twiddles [M / 2], real-split cos / sin [khi], the sparse mel (row offsets [nmel + 1],
 * bins and weights of the nonzero entries) */
typedef struct {
  int nsamp, frame, hop, pad, nfft, M, lg, nmel, nfr, klo, khi, nz;
  float floor_, scale;
  const float *win, *tw_re, *tw_im, *pc, *ps, *mel_w;
  const int *mel_off, *mel_k;
} bnnk_logmel_tables;
int bnnk_logmel(int B, const float *pcm, long long pws, const bnnk_logmel_tables *t, float *spec, long long sws,
                bnn_stream_t st);

/* ---- the fp32 ops beyond v2.4 (k_v3.cu): v3.0's CONVK, CONVW, GEM, SED, VADD (src/rt_ops_f32x.c) and Perch's fp32
 * body ops STEM, DWK, PAD, MEAN (src/rt_ops_f32.c); per-window strides in floats */
typedef struct {
  int N, K, Kp, Np;
  const float *w; /* [Np/8][Kp][8] */
  const float *b; /* [Np] */
} bnnk_fpack;
typedef struct {
  int red, H, W, C, ld, L, pk, dk, hc, Cp;
  const float *x;
  long long xws;
  const float *dw, *db, *consts;
  bnnk_fpack fc, at, cl;
  float *out, *s, *pl, *h, *att, *cla;
  long long ows, sws, pws, hws, aws, clws;
} bnnk_sed_args;
int bnnk_v3_tables_init(const unsigned long long *tab, const uint32_t *lut);
int bnnk_vadd(int B, int n, const float *a, long long aws, const float *b, long long bws, float *o, long long ows,
              bnn_stream_t st);
int bnnk_gem(int B, int P, int C, int ld, const float *x, long long xws, const float *consts, float *out,
             long long ows, bnn_stream_t st);
int bnnk_mean_f32(int B, int P, int C, int ld, const float *x, long long xws, float *out, long long ows,
                  bnn_stream_t st);
int bnnk_pad_f32(int B, int H, int W, int C, int ld, int h, const float *x, long long xws, float *xp, long long pws,
                 bnn_stream_t st);
int bnnk_dwk_f32(int B, const float *xp, long long xws, int H, int W, int C, int k, int s, int pt, int pl,
                 const float *w, const float *b, int act, float *out, long long ows, int Ho, int Wo, float *chsum,
                 long long cws, bnn_stream_t st);
/* PW (fp32 1x1 conv, src/rt_ops_f32.c:110-206): rows [M][lda] of each window, optional SE gate [Kp]; output rows at
 * their padded position (ow, opad; the halo of the oH x oW output zeroed), optional residual (rw, rpad) */
int bnnk_pw_f32(int B, const float *x, long long xws, int lda, int M, const float *gate, long long gws, const float *w,
                const float *bias, int Kp, int Np, int act, float *out, long long ows, int ldo, int ow, int opad, int oH,
                int oW, const float *res, long long rws, int ldr, int rw, int rpad, bnn_stream_t st);
int bnnk_stem_f32(int B, const float *img, long long iws, int W, int k, int s, int Ho, int Wo, const float *w,
                  const float *bias, int Kp, int Np, int act, float *out, long long ows, int ldo, int opad, float *col,
                  long long cws, bnn_stream_t st);
int bnnk_convk(int B, const float *x, long long xws, int H, int W, int h, int ld, int Ho, int Wo, int kh, int kw, int s,
               int oy0, int ox0, const float *w, const float *bias, int Kp, int Np, int act, float *out, long long ows,
               int ldo, int opad, const float *res, long long rws, int ldr, int rh, bnn_stream_t st);
size_t bnnk_convw_scratch_floats(int H, int W, int C, int Np); /* per window */
int bnnk_convw(int B, const float *x, long long xws, int H, int W, int h, int C, const float *U, const float *bias,
               int Np, int act, float *out, long long ows, int ldo, int opad, const float *res, long long rws, int rh,
               int rld, float *scratch, bnn_stream_t st);
int bnnk_sed(int B, const bnnk_sed_args *a, bnn_stream_t st);
/* SED's first and last stages alone (SED_S8 runs its GEMMs on the int8 path between them) */
int bnnk_sed_pool(int B, const bnnk_sed_args *a, bnn_stream_t st);
int bnnk_sed_out(int B, const bnnk_sed_args *a, bnn_stream_t st);

/* ---- the dB-image front end (FE_DBIMG): pcm [B][nsamp] -> image [B][(Ho + 2 halo)(Wo + 2 halo)][ld]. Device tables:
 * window [nfft], twiddles [nfft / 4], real-split factors [nfft / 2 + 1], the sparse mel (row offsets [nmel + 1], bins
 * and weights of the nonzero entries), rows [R], channel values [2][C], the resize coordinates [Ho], [Wo]; the scratch
 * holds bnnk_dbimg_scratch_floats(t, B) floats (the dB rows, the selected rows, the blocks' maxima) */
typedef struct {
  int nsamp, nfft, lg, hop, pad, padmode, nfr, nmel, R, has_top_db, norm, post[3], Ho, Wo, C, chan[2], ld, halo, klo, khi;
  float floor_, top_db, eps, postv[3];
  const float *win, *tw_re, *tw_im, *sp_re, *sp_im, *mel_w, *chv, *dy1, *dy2, *dx1, *dx2;
  const int *mel_off, *mel_k, *rows, *ry1, *ry2, *rx1, *rx2;
} bnnk_dbimg_tables;
size_t bnnk_dbimg_scratch_floats(const bnnk_dbimg_tables *t, int B);
int bnnk_dbimg(int B, const float *pcm, long long pws, const bnnk_dbimg_tables *t, float *scratch, float *img,
               long long iws, bnn_stream_t st);
/* ---- the int8 prototype head (PROTO_S8) */

/* per-cell quantization (pc_quant_cells_f32): cells r = w * P + p of x (window stride xws, row stride ld floats;
 * C % 8 == 0) -> qa [B * P][Kq] int8 (Kq % 8 == 0, zero from C), sx [B * P] */
int bnnk_proto_quant(int B, int P, const float *x, long long xws, int ld, int C, int Kq, float eps, int8_t *qa,
                     float *sx, bnn_stream_t st);

/* the same on IEEE-half cells (PROTO variant 2, pc_quant_cells_f16): bytes saturated to [-128, 127] */
int bnnk_proto_quant_h(int B, int P, const uint16_t *x, long long xws, int ld, int C, int Kq, float eps, int8_t *qa,
                       float *sx, bnn_stream_t st);

/* the column-maximum GEMM of one head: prototypes w [np][kp] int8 (row j = prototype j, zero from K), cells qa
 * [batch_cap * P][kp]. Cell tiles hold wt = floor(256 / P) whole windows when P <= 256 (bn = wt P rounded up to 16
 * MMA columns), else chunks of cs cells (nch per window) whose partial maxima go through scratch. */
typedef struct {
  unsigned char tma_w[128] __attribute__((aligned(64)));
  unsigned char tma_q[128] __attribute__((aligned(64)));
  int np, kp, P, batch_cap;
  int wt, nch, cs, bn, unit, acc_cols, mh, nkb, stages;
  unsigned int idesc;
  size_t smem;
} bnnk_proto_plan;
int bnnk_proto_plan_init(bnnk_proto_plan *p, const int8_t *w, int np, int kp, const int8_t *qa, int batch_cap, int P);
/* colmax [batch][cws] = sw[j] * max over the window's cells of (float)acc * sx[cell]; part: scratch of
 * batch * nch * np floats when the plan has wt == 0 (else NULL) */
int bnnk_proto_colmax(const bnnk_proto_plan *p, int batch, const float *sx, const float *sw, float *colmax,
                      long long cws, float *part, int *err, bnn_stream_t st);
/* logits [batch][lws] from colmax [batch][cws], class weights [nc][ppc], biases [nc]. A window with a logit that is not
 * finite or above 3e38 in magnitude failed: status [batch] (or NULL) gets -2 for it (else 0), and *fail (or NULL) is
 * lowered to w_base + its index (atomic minimum) */
int bnnk_proto_logits(int batch, int nc, int ppc, const float *colmax, long long cws, const float *cw, const float *cb,
                      float *logits, long long lws, int *status, int *fail, int w_base, bnn_stream_t st);

/* ---- elementwise functions for the unit tests */
int bnnk_test_fn(int fn, int n, const float *x, float *y, bnn_stream_t st);

/* ---- the neon-fp16 path's kernels (k_f16.cu): fp16 buffers are IEEE half bits (uint16_t), window strides in
 * elements. Every fp16 operation is the reference's, in its order (src/gemm_f16.c, src/kern_f16.c, src/v24_fast.c). */
/* the glibc expf table of k_f16.cu's SE gate (per device, once) */
int bnnk_f16_tables_init(const unsigned long long *tab);
/* PW f16 / any hp_pack GEMM: rows r = w * Mw + m of A (window stride aws, row stride lda); Wd [Kp][Np] k-major, each
 * weight duplicated into both halves of a 32-bit word;
 * K blocks of <= 128 (fp16 chains, fp32 flushes), bias b16 / b32, act (0 none, 1 SiLU, 2 ReLU), + residual, stored
 * at the padded row (ow, opad). Kp, Np, lda and aws multiples of 8, ldo / ldr and their window strides of 4; A and Wd
 * 16-byte aligned, out and res 8. */
int bnnk_gemm_f16(int rows, int Mw, const uint16_t *A, long long aws, int lda, const uint32_t *Wd, int Kp, int Np,
                  const uint16_t *b16, const float *b32, int act, uint16_t *out, long long ows, int ldo, int ow,
                  int opad, const uint16_t *res, long long rws, int ldr, bnn_stream_t st);
/* PW f16 in the tensor mode: a tcgen05 kind::f16 GEMM with fp32 accumulators (not the reference's fp16 chains: within
 * a tolerance of them), then + b32, one rounding to fp16, act, the fp16 residual add, the padded row. B windows of Mw
 * rows (window stride aws, row stride lda); Wk [Np][Kp] fp16 K-major. Kp, Np, lda, aws multiples of 8; A and Wk
 * 16-byte aligned, out / res 8; err: the device error word of the bounded waits */
int bnnk_gemm_tc16(int B, int Mw, const uint16_t *A, long long aws, int lda, const uint16_t *Wk, int Kp, int Np,
                   const float *b32, int act, uint16_t *out, long long ows, int ldo, int ow, int opad,
                   const uint16_t *res, long long rws, int ldr, int *err, bnn_stream_t st);
/* C0POOL f16: img [B][96][511][2] fp32 -> pin [B][48 * 128][48] fp16; W [64][24] k-major, b16 [24] */
int bnnk_c0pool_f16(int B, const float *img, long long iws, const uint16_t *W, const uint16_t *b16, uint16_t *pin,
                    long long pws, bnn_stream_t st);
/* DW3 f16: xp [B][(H+2)(W+2)][C] haloed -> out [B][Ho Wo][C], chsum [B][C]; w [9][C], b [C] fp16; err: the device
 * error word a timed-out input wait is reported in (NULL: not reported) */
int bnnk_dw3_f16(int B, const uint16_t *xp, long long xws, int H, int W, int C, int s, int pt, int pl,
                 const uint16_t *w, const uint16_t *b, uint16_t *out, long long ows, int Ho, int Wo, float *chsum,
                 long long cws, int *err, bnn_stream_t st);
/* SE f16: the gate from chsum [B][C] (fp32 FCs, sigm4, rounded to fp16 into g16 [B][C]), D [B][P][C] scaled in place */
int bnnk_se_f16(int B, int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                const float *chsum, long long cws, int P, uint16_t *D, long long dws, uint16_t *g16, bnn_stream_t st);
/* POSTPC f16: X [B][24][192] -> pcin [B][6][1728] -> pcout [B][6][1024] -> feat [B][1024]; a window whose features
 * are not finite sets fail (atomic minimum of w_base + window) */
int bnnk_postpc_f16(int B, const uint16_t *X, long long xws, const float *ps, const float *pb, const uint32_t *W,
                    const uint16_t *b16, const float *b32, uint16_t *pcin, long long pinws, uint16_t *pcout,
                    long long poutws, float *feat, long long fws, int *fail, int w_base, bnn_stream_t st);
/* DENSE f16 (v24k16_head): feat [B][1024] fp32, W [N][1024] fp16, bias [N] -> out [B][N] */
int bnnk_dense_f16(int B, int N, const float *feat, long long fws, const uint16_t *W, const float *bias, float *out,
                   long long ows, bnn_stream_t st);
/* the fp16 FMA pipe's peak for the roofline: blocks x 256 threads x iters x 16 fp16 FMAs (out: one word, kept live) */
int bnnk_peak_hfma2(int blocks, int iters, uint32_t *out, bnn_stream_t st);
/* DENSE variant 0 (v24k32_head): W [N][1024] fp32 */
int bnnk_dense_f32(int B, int N, const float *feat, long long fws, const float *W, const float *bias, float *out,
                   long long ows, bnn_stream_t st);

/* ---- compiled models' fp16 bodies (Perch v2) */
/* STEM f32 -> f16: img [B][H][W] fp32 (window stride iws), w the fp32 GEMM panels [Np/8][Kp][8], b [Np]; out fp16
 * at the padded position (halo opad, channel stride ldo, window stride ows) */
int bnnk_stem_f16(int B, const float *img, long long iws, int W, int k, int s, int Ho, int Wo, const float *w,
                  const float *b, int N, int Kp, int Np, int act, uint16_t *out, long long ows, int ldo, int opad,
                  bnn_stream_t st);
/* DWK f16: xp [B] zero-haloed by (k - 1) / 2 with channel stride C, w [k*k][C], b [C] fp16 -> out [B][Ho][Wo][C],
 * chsum [B][C] fp32 */
int bnnk_dwk_f16(int B, const uint16_t *xp, long long xws, int W, int C, int k, int s, int pt, int pl,
                 const uint16_t *w, const uint16_t *b, int act, uint16_t *out, long long ows, int Ho, int Wo,
                 float *chsum, long long cws, bnn_stream_t st);
/* PAD f16: x [B][H][W] (channel stride ld) into the interior of xp [B][H+2h][W+2h][C] */
int bnnk_pad_f16(int B, int H, int W, int C, int ld, int h, const uint16_t *x, long long xws, uint16_t *xp,
                 long long pws, bnn_stream_t st);
/* MEAN f16: x [B][P][ld] -> out [B][C] fp32 */
int bnnk_mean_f16(int B, int P, int C, int ld, const uint16_t *x, long long xws, float *out, long long ows,
                  bnn_stream_t st);

#ifdef __cplusplus
}
#endif
#endif
