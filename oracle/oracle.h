/* bnn oracle: a plain-C CPU restatement of the reference's BirdNET v2.4 neon-int8 hot path (TEST INFRASTRUCTURE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg may load liboracle.so; the
 * product library (libbnneon.so) never links or calls it. Every function restates one reference routine with the
 * same per-element arithmetic (the NEON order of operations, FMA where the reference fuses, no FMA where it does
 * not), so its outputs are the reference's outputs bit for bit wherever the reference's AArch64 arithmetic is
 * emulated exactly (arm_emu.h). Layouts are the reference's (per window, NHWC fp32 activations, packed weights as
 * stored in the .bnpk package).
 *
 * Parity pins: the int8 packing tests of the reference (tests/test_lower_units.py:139-156,
 * tests/test_lower_s8.py:38-53) and packages written by the reference compiler (tests/golden). The per-op outputs
 * have no reference fixtures (the reference ships none for PW_S8 / GEMV_S8 / DW3 / SE / FE_STFT2; its NEON build
 * does not compile on x86): for those ops parity rests on this restatement. */
#ifndef BNN_ORACLE_H
#define BNN_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* elementwise helpers (src/gemm_f32.h, src/v24_fe.c, src/v24_f32.c:160) */
float bnno_silu(float x);      /* silu_f32x4 / SILU_N_F32X4 */
float bnno_sigmoid(float x);   /* sigmoid_f32x4 */
float bnno_frecpe(float x);    /* FRECPE */
float bnno_log2_acc(float x);  /* log2_acc_f32x4 */
float bnno_exp2_acc(float x);  /* v24_fe.c exp2_acc */
float bnno_expf(float x);      /* the host libm expf the reference calls (SE fc1) */

/* s8n_quant_rows / s8n_quant_rows_gate (src/gemm_s8n.c:15-63): rows [0, M) of x (row stride ld) -> q [M][Kp] */
void bnno_quant_rows(const float *x, int ld, int M, int K, int Kp, const float *gate, int8_t *q, float *sa, int32_t *za);

/* int8 GEMM + epilogue (src/gemm_s8n.c:82-190) on quantized rows; w is the package tensor [Np/4][Kp/16][4][16].
 * act: 0 none, 1 SiLU, 2 ReLU. opad/ow: padded output rows; rpad/rw: residual in a haloed buffer; res may be NULL. */
void bnno_s8_gemm(const int8_t *q, const float *sa, const int32_t *za, int M, int N, int Kp, int Np, const int8_t *w,
                  const float *sw, const int32_t *cs, const float *b, int act, float *out, int ldo, int ow, int opad,
                  const float *res, int ldr, int rpad, int rw);

/* PW_S8 run (src/rt_ops_s8n.c:119-134): halo zeroing of a padded output, quantization (optionally gated), GEMM */
void bnno_pw_s8(const float *x, int lda, int M, int N, int K, int Kp, int Np, const float *gate, const int8_t *w,
                const float *sw, const int32_t *cs, const float *b, int act, float *out, int ldo, int ow, int opad,
                int out_h, const float *res, int ldr, int rpad, int rw, int8_t *q, float *sa, int32_t *za);

/* DW3 (src/gemm_f32.c:214-440): depthwise 3x3 pad 1 stride s + SiLU + channel sums */
void bnno_dw3(const float *xp, int H, int W, int C, int s, const float *w, const float *b, float *out, int Ho, int Wo,
              float *chsum);

/* SE_GATE (src/rt_ops_f32.c:314-325 = v24k32_se_fc1 + se_gate_range) */
void bnno_se_gate(int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                  const float *chsum, int P, float *gate);

/* C0POOL (src/v24_f32.c:139-147, src/gemm_f32.c:60-70, :199-212): img [96][511][2] -> pin [48*128][48];
 * w: fp32 panels [Np/8][Kp][8] (Np 24, Kp 64), b [>= 24] */
void bnno_c0pool(const float *img, const float *w, const float *b, float *pin);

/* POSTPC (src/v24_f32.c:245-266): X [24][192] -> feat [1024]; w: panels [128][1728][8], b [>= 1024] */
void bnno_postpc(const float *X, const float *post_s, const float *post_b, const float *w, const float *b, float *feat);

/* FE_STFT2 (src/v24_fe.c:127-224, src/fft_tab.h): pcm [144000] -> img [96][511][2] */
typedef struct bnno_fe bnno_fe;
bnno_fe *bnno_fe_new(const float *win1, const float *win2, const float *mel1, const float *mel2, float pow1,
                     float pow2, const float bn_s[2], const float bn_b[2]);
void bnno_fe_run(const bnno_fe *f, const float *pcm, float *img);
void bnno_fe_free(bnno_fe *f);

/* ---- FE_LOGMEL, the framed log-mel front end (src/pc_kern_f32.c:14-149, record src/rt_ops_f32.c:362-385) */
/* FE_DBIMG (src/fe_dbimg.c), oracle_dbimg.c: p = the record's 21 ints, consts {floor, top_db, eps, postv[3], chan0[C],
 * chan1[C]}; log_mode 0 = this host's libm logf (as the reference build here), 1 = correctly rounded (the GPU's) */
typedef struct bnno_dbimg bnno_dbimg;
bnno_dbimg *bnno_dbimg_new(const int32_t *p, const float *window, const float *mel, const int32_t *rows,
                           const float *consts);
void bnno_dbimg_free(bnno_dbimg *f);
int bnno_dbimg_frames_count(const bnno_dbimg *f);
void bnno_dbimg_frames(const bnno_dbimg *f, const float *pcm, float *db, int log_mode);
void bnno_dbimg_image(const bnno_dbimg *f, const float *db, float *img);
void bnno_dbimg_run(const bnno_dbimg *f, const float *pcm, float *img, int log_mode);
float bnno_logf_cr(float x);
/* y[i] = the logarithm of x[i] for i < n: log_mode 0 this host's logf, 1 bnno_logf_cr */
void bnno_log_n(const float *x, float *y, long n, int log_mode);
/* FE_DBIMG's logarithm in package runs (bnno_pkg_*): 0 libm logf (default), 1 correctly rounded */
void bnno_pkg_set_log_mode(int mode);
typedef struct bnno_logmel bnno_logmel;
/* NULL when the geometry is outside pc_logmel_new's limits (nfft a power of two in 16..2048, frame <= nfft, hop > 0,
 * pad >= 0, 1 <= nmel <= 512); window [frame], mel [nmel][nfft / 2 + 1] */
bnno_logmel *bnno_logmel_new(int nsamp, int frame, int hop, int pad, int nfft, int nmel, const float *window,
                             const float *mel, float floor_, float scale);
int bnno_logmel_frames(const bnno_logmel *f);
/* pcm [nsamp] -> spec [nfr][nmel] */
void bnno_logmel_run(const bnno_logmel *f, const float *pcm, float *spec);
void bnno_logmel_free(bnno_logmel *f);

/* ---- the int8 prototype head PROTO_S8 (src/proto_s8n.c, src/rt_ops_s8n.c:212-250, src/pc_kern_f32.c:364-376) */
/* pc_quant_cells_f32: x [P][ld] -> qa [P][Kp] (ties away, never -128, zero past C), sx [P]; C % 8 == 0 */
void bnno_proto_quant_cells(const float *x, int P, int C, int ld, float eps, int8_t *qa, int Kp, float *sx);
/* pc_quant_cells_f16 (PROTO variant 2, the SDOT head of the neon-fp16 path): fp16 cells x [P][ld] (IEEE half bits)
 * -> rows qa [P][C] (saturated to [-128, 127], no -127 clamp), sx [P]; C % 8 == 0 */
void bnno_proto_quant_cells_f16(const uint16_t *x, int P, int C, int ld, float eps, int8_t *qa, float *sx);
/* the SDOT head's prototype panels [Np/12][K/4][12][4] -> rows [Np][K] */
void bnno_proto_unpack12(const int8_t *qw, int Np, int K, int8_t *rows);
/* the package's prototype bytes [Np/4][Kp/16][4][16] -> rows [Np][Kp] */
void bnno_proto_unpack(const int8_t *qw, int Np, int Kp, int8_t *rows);
/* pc_proto_colmax_s8n: colmax[j] = sw[j] * max_p (float)(qa[p] . w[j]) * sx[p]; packed or unpacked prototypes */
void bnno_proto_colmax(const int8_t *qa, int Kp, const float *sx, int P, const int8_t *qw, const float *sw, int Np,
                       float *colmax);
void bnno_proto_colmax_rows(const int8_t *qa, int Kp, const float *sx, int P, const int8_t *rows, const float *sw,
                            int Np, float *colmax);
/* pc_proto_logits: 0, or -2 when a logit is not finite or above 3e38 in magnitude */
int bnno_proto_logits(const float *colmax, const float *w, const float *b, int nc, int ppc, float *logits);
/* pc_proto_n4_check: the first flagged 4-prototype panel whose int16 lanes could wrap, or -1 */
int bnno_proto_n4_check(const int8_t *qw, int Kp, const uint8_t *n4, int npanels);
/* the whole op on one window (prototype rows unpacked); 0 or -2 */
int bnno_proto_s8(const float *x, int P, int C, int ld, float eps, const int8_t *rows, const float *sw, int Np, int Kp,
                  const float *cls_w, const float *cls_b, int nc, int ppc, int8_t *qa, float *sx, float *colmax,
                  float *logits);
/* n windows at window stride xws on `threads` threads: logits [n][nc]; 0 or -2 */
int bnno_proto_s8_many(int n, int threads, const float *x, long long xws, int P, int C, int ld, float eps,
                       const int8_t *rows, const float *sw, int Np, int Kp, const float *cls_w, const float *cls_b,
                       int nc, int ppc, float *logits);

/* ---- the neon-fp16 path's ops (variant 1; oracle_f16.c). fp16 values are IEEE half bits (uint16_t). */
double bnno_h2d(uint16_t h);
float bnno_h2f(uint16_t h);
uint16_t bnno_d2h(double x);          /* one rounding, nearest even */
uint16_t bnno_f2h(float x);
uint16_t bnno_h_add(uint16_t a, uint16_t b);
uint16_t bnno_h_mul(uint16_t a, uint16_t b);
uint16_t bnno_h_fma(uint16_t a, uint16_t b, uint16_t c); /* a * b + c, one rounding */
uint16_t bnno_h_silu(uint16_t x);     /* src/silu_lut.h */
extern const uint16_t BNNO_SILU_C0[16], BNNO_SILU_C1[16], BNNO_SILU_C2[16];
float bnno_sigm_f16path(float a);     /* sigm4, src/v24_fast.c:173-185 */
/* the SE's two FCs before the sigmoid: g [C] */
void bnno_se_fc(int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2, const float *chsum,
                int P, float *g);
/* PW f16 / any hp_pack GEMM (src/gemm_f16.c): A [M][lda] -> out (padded rows when opad); act 0 none, 1 SiLU, 2 ReLU;
 * w: panels [Np/16][Kp][16] + tail [Kp][8]; b32 / b16 [>= Np] */
void bnno_gemm_f16(const uint16_t *A, int lda, int M, const uint16_t *w, const float *b32, const uint16_t *b16, int Kp,
                   int Np, int act, uint16_t *out, int ldo, int ow, int opad, const uint16_t *res, int ldr);
/* C0POOL f16: img [96][511][2] fp32 -> pin [48*128][48] fp16 (w: panels Kp 64 Np 24, b16) */
void bnno_c0pool_f16(const float *img, const uint16_t *w, const uint16_t *b16, uint16_t *pin);
/* DW3 f16: xp haloed [H+2][W+2][C] -> out [Ho][Wo][C], chsum [C] */
void bnno_dw3_f16(const uint16_t *xp, int H, int W, int C, int s, int pt, int pl, const uint16_t *w, const uint16_t *b,
                  uint16_t *out, int Ho, int Wo, float *chsum);
/* SE f16: D [P][C] scaled in place */
void bnno_se_f16(int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                 const float *chsum, int P, uint16_t *D);
/* POSTPC f16: X [24][192] -> feat [1024]; 0, or -2 when a feature is not finite (src/v24_fast.c:305-310) */
int bnno_postpc_f16(const uint16_t *X, const float *post_s, const float *post_b, const uint16_t *w, const float *b32,
                    const uint16_t *b16, float *feat);
/* DENSE f16 (W fp16 [N][1024]) and DENSE f32 (W fp32 [N][1024]): feat [1024] -> out [N] */
void bnno_dense_f16(const uint16_t *W, const float *bias, int N, const float *feat, float *out);
void bnno_dense_f32(const float *W, const float *bias, int N, const float *feat, float *out);

/* ---- compiled models' fp16 bodies (oracle_perch.c) */
void bnno_stem_f16(const float *img, int H, int W, int k, int s, int Ho, int Wo, const float *w, const float *b, int N,
                   int Kp, int act, uint16_t *out, int ldo, int opad);
void bnno_dwk_f16(const uint16_t *xp, int H, int W, int C, int k, int s, int pt, int pl, const uint16_t *w,
                  const uint16_t *b, int act, uint16_t *out, int Ho, int Wo, float *chsum);
void bnno_pad_f16(const uint16_t *x, int H, int W, int C, int ld, int h, uint16_t *xp);
void bnno_mean_f16(const uint16_t *x, int P, int C, int ld, float *out);

/* ---- a .bnpk package run on the CPU, window by window (the executor of src/rt_pkg.c:528-542) */
typedef struct bnno_pkg bnno_pkg;
/* path: the package; path_name: the package path to run ("neon-int8"). NULL on failure (err filled). */
bnno_pkg *bnno_pkg_open(const char *path, const char *path_name, char *err, size_t errlen);
void bnno_pkg_close(bnno_pkg *p);
int bnno_pkg_n_ops(const bnno_pkg *p);
int bnno_pkg_n_bufs(const bnno_pkg *p);
int bnno_pkg_op_code(const bnno_pkg *p, int i);
/* elements of buffer i (its descriptor's elems) and its dtype (0 f32, 1 f16, 2 i8, 3 i32) */
long bnno_pkg_buf_elems(const bnno_pkg *p, int i, int *dtype);
int bnno_pkg_out_elems(const bnno_pkg *p); /* n_classes (metadata) */
int bnno_pkg_emb_elems(const bnno_pkg *p); /* emb_dim (metadata) */
/* ops [op0, op1) on the buffers as they are (buffer 0 = pcm): a whole window is bnno_pkg_run_range(p, pcm, 0, n) */
int bnno_pkg_run_range(bnno_pkg *p, const float *pcm, int op0, int op1);
/* one window: out [n_classes], emb [emb_dim] (may be NULL) */
int bnno_pkg_run(bnno_pkg *p, const float *pcm, float *out, float *emb);
/* copy buffer i out of / into the executor (bytes = elems * dtype size) */
int bnno_pkg_get_buf(const bnno_pkg *p, int i, void *dst, size_t bytes);
int bnno_pkg_set_buf(bnno_pkg *p, int i, const void *src, size_t bytes);
/* n windows [n][n_samples] on `threads` threads (each window independent): out [n][n_classes], emb [n][emb_dim] */
int bnno_pkg_run_many(const char *path, const char *path_name, int n, const float *pcm, float *out, float *emb,
                      int threads);

#ifdef __cplusplus
}
#endif
#endif
