/* B200 additions to the bnneon API (additive: the reference's bnneon.h is unchanged; hosts check for these symbols
 * with dlsym, as they do for bnn_set_threads, src/bnneon.h:94-98).
 *
 * Batching: the reference scores one window per bnn_infer call (src/bnneon.h:78-80, src/bnneon.c:310-330). A GPU
 * needs many windows per launch, so bnn_infer_batch scores n windows per call; the results are bit-identical to n
 * calls of bnn_infer (every op is per window).
 *
 * Per-op entry points: the kernel-level interface of the reference's int8 GEMM and depthwise routines
 * (src/gemm_s8n.h:16-23 s8n_quant_rows / s8n_gemm_range, src/gemm_f32.h:46-51 dw3x3_f32), batched over windows and
 * taking device pointers, for hosts that run their own graphs and for the parity tests.
 *
 * Pointers named d_* are device pointers on the current CUDA device; `stream` is a cudaStream_t (NULL = the legacy
 * default stream). Functions return 0 on success, else -1 with bnn_last_error / bnn_last_error_kind set.
 *
 * Device reset: the library keeps per-device state for the life of the process (kernels' shared-memory limits, the
 * address of bnn_pw_s8_run_static's array, every context's and op's device memory). cudaDeviceReset destroys all of
 * it on the CUDA side, so a host that resets a device must not use this library on that device afterwards. */
#ifndef BNNEON_CUDA_H
#define BNNEON_CUDA_H
#include <stddef.h>
#include <stdint.h>

#include "bnneon.h"
#ifdef __cplusplus
extern "C" {
#endif

/* ---- batched inference */

/* n windows of host memory: pcm [n][n_samples] -> out [n][n_classes], emb [n][emb_dim] (emb may be NULL). The
 * windows are split into contiguous slices over the context's GPUs (bnn_set_threads) and into chunks of the batch
 * capacity (bnn_set_batch). Synchronous. Returns -2 (kind BNN_ERR_WINDOW, as bnn_infer on a failed window,
 * src/bnneon.c:313-325) when an op reported a failed window (the prototype head's non-finite logits); the message
 * names the first such window, and the other windows' outputs are still written. */
int bnn_infer_batch(bnn_ctx *ctx, int n, const float *pcm, float *out, float *emb);
/* the same with device-resident buffers on the context's first GPU (n <= the batch capacity); asynchronous on
 * `stream` (NULL = the context's own stream, synchronized before return, failed windows reported as above; with a
 * caller's stream they are reported by the context's next synchronous call) */
int bnn_infer_device(bnn_ctx *ctx, int n, const float *d_pcm, float *d_out, float *d_emb, void *stream);
/* windows per launch sequence on each GPU (default 256, or the BNN_BATCH environment variable): sizes the device
 * arena; 0 on success */
int bnn_set_batch(bnn_ctx *ctx, int batch);
int bnn_get_batch(const bnn_ctx *ctx);
/* No counterpart in the reference: the neon-fp16 path's 1x1 convs (PW f16) on the tensor cores (tcgen05 kind::f16,
 * fp32 accumulation) instead of the reference's fp16 FMA chains (src/gemm_f16.c:109-169), which the default mode
 * reproduces bit for bit on the CUDA cores. Outputs then agree with the reference within a tolerance, not exactly.
 * on = 1 selects it (default 0, or the BNN_F16_TENSOR environment variable at bnn_init); re-creates the context's
 * device state (weights in both layouts), so call it before inference. 0 on success. */
int bnn_set_fp16_tensor(bnn_ctx *ctx, int on);
int bnn_get_fp16_tensor(const bnn_ctx *ctx);
/* kernels launched by one bnn_infer_device call of n windows (the op list's launches) */
int bnn_launches_per_batch(const bnn_ctx *ctx);

/* ---- per-op profile on the first GPU (the reference's BNN_PROF per-op times, src/rt_pkg.c:558-625, measured with
 * CUDA events on the launching stream): begin clears the totals and brackets every op of later launches with
 * events; collect waits for the last launch and adds its op times; op_ms reads the totals (milliseconds). */
int bnn_profile_begin(bnn_ctx *ctx);
int bnn_profile_collect(bnn_ctx *ctx);
double bnn_profile_op_ms(const bnn_ctx *ctx, int op);
int bnn_profile_end(bnn_ctx *ctx);

/* ---- op-level debugging (the reference's BNN_DUMP bisection, src/rt_pkg.c:512-526) on the first GPU:
 * buffers are addressed by their package buffer id and hold n windows [n][elems] (elems from the package) */
int bnn_debug_n_ops(const bnn_ctx *ctx);
int bnn_debug_op_code(const bnn_ctx *ctx, int op);
/* buffer 0 (the input window) <- pcm [n][n_samples] (host), then ops [op0, op1) on n windows */
int bnn_debug_run_ops(bnn_ctx *ctx, int n, const float *pcm, int op0, int op1);
int bnn_debug_get_buffer(bnn_ctx *ctx, int buf, int n, void *dst);
int bnn_debug_set_buffer(bnn_ctx *ctx, int buf, int n, const void *src);

/* ---- per-op entry points */

/* loads the device tables (expf table, reciprocal-estimate table) on the current device; the context does this
 * itself, the per-op entry points below need it once per device */
int bnn_cuda_device_init(void);

/* s8n_quant_rows (src/gemm_s8n.c:15-63), batched: rows r = w * Mw + m of d_x (window stride xws, row stride lda,
 * floats), optionally times d_gate [B][K] (window stride gws) -> d_q [rows][Kq] int8 (Kq >= K; pads = zero point),
 * d_sa, d_za [rows] */
int bnn_cuda_quant_rows(int rows, int Mw, const float *d_x, long long xws, int lda, int K, int Kq,
                        const float *d_gate, long long gws, int8_t *d_q, float *d_sa, int32_t *d_za, void *stream);

/* PW_S8 / GEMV_S8 (src/rt_ops_s8n.c:92-158): an int8 1x1 conv built from the package's tensors (host pointers:
 * w [Np/4][Kp/16][4][16], sw / cs / b [>= Np]) for up to rows_cap rows (windows x pixels) per run */
typedef struct bnn_pw_s8 bnn_pw_s8;
bnn_pw_s8 *bnn_pw_s8_new(int N, int K, int Kp, int Np, const int8_t *w, const float *sw, const int32_t *cs,
                         const float *b, int rows_cap);
/* B windows of Mw rows: quantize (gated if d_gate), GEMM, epilogue act (0 none, 1 SiLU, 2 ReLU) + residual, stored
 * at the padded row of each pixel (ow / opad, as epi32, src/gemm_f32.h:15-24); window strides in floats. A padded
 * output's halo is not written. */
int bnn_pw_s8_run(bnn_pw_s8 *op, int B, int Mw, const float *d_x, long long xws, int lda, const float *d_gate,
                  long long gws, int act, float *d_out, long long ows, int ldo, int ow, int opad, const float *d_res,
                  long long rws, int ldr, int rw, int rpad, void *stream);
/* s8n_gemm_range (src/gemm_s8n.c:176-190 with its tiles :82-175, declared src/gemm_s8n.h:22) on quantized rows the
 * caller holds, as s8n_quant_rows / bnn_cuda_quant_rows write them: d_q [B * Mw][ldq] int8 (ldq >= Kp, a multiple of
 * 16; the row's first Kp bytes are used), d_sa, d_za [B * Mw]; then the same epilogue and store as bnn_pw_s8_run */
int bnn_pw_s8_gemm(bnn_pw_s8 *op, int B, int Mw, const int8_t *d_q, long long ldq, const float *d_sa,
                   const int32_t *d_za, int act, float *d_out, long long ows, int ldo, int ow, int opad,
                   const float *d_res, long long rws, int ldr, int rw, int rpad, void *stream);
/* No counterpart in the reference: bnn_pw_s8_run for hosts that must not allocate device memory while they run (a
 * live-audio loop, where cudaMalloc / cudaFree may synchronise the device and take unbounded time; a server whose
 * device memory was sized at start-up). The quantized activations and their per-row scale / zero point go to one
 * file-scope static device array instead of the op's own buffers, and the call allocates nothing. Limits:
 * B * Mw <= BNN_PW_S8_STATIC_MAX_ROWS and B * Mw * Kq <= BNN_PW_S8_STATIC_MAX_QBYTES (Kq = K rounded up to 32);
 * larger calls fail with BNN_ERR_USAGE. The first call on each device, with that device current, looks up the array's
 * address there (B = 0 does only this); make it before any stream capture. Every call on a device uses the same
 * array, so calls whose work may overlap in time (different streams, or host threads, with no ordering between them)
 * race on it: serialise them. Nothing in the array has to start at zero. Results equal bnn_pw_s8_run's; the op's
 * error word (bnn_pw_s8_error) is shared by both calls. */
#define BNN_PW_S8_STATIC_MAX_ROWS 32768
#define BNN_PW_S8_STATIC_MAX_QBYTES (4 << 20)
int bnn_pw_s8_run_static(bnn_pw_s8 *op, int B, int Mw, const float *d_x, long long xws, int lda,
                         const float *d_gate, long long gws, int act, float *d_out, long long ows, int ldo, int ow,
                         int opad, const float *d_res, long long rws, int ldr, int rw, int rpad, void *stream);
/* the device error word of the op's GEMM (0 = no bounded wait ran out) */
int bnn_pw_s8_error(bnn_pw_s8 *op);
void bnn_pw_s8_free(bnn_pw_s8 *op);

/* FE_LOGMEL, the framed log-mel front end of compiled models such as Perch (src/pc_kern_f32.c:14-149 driven by
 * src/rt_ops_f32.c:362-385), batched: the package's tensors (host pointers) window [frame], mel [nmel][nfft / 2 + 1],
 * floor, scale; nfft a power of two in 16..2048, frame <= nfft, nmel <= 512. A window of nsamp samples gives
 * bnn_logmel_frames() = (nsamp + 2 pad - frame) / hop + 1 frames of nmel log-mel values. */
typedef struct bnn_logmel bnn_logmel;
bnn_logmel *bnn_logmel_new(int nsamp, int frame, int hop, int pad, int nfft, int nmel, const float *window,
                           const float *mel, float floor_, float scale);
int bnn_logmel_frames(const bnn_logmel *op);
/* d_pcm [B][nsamp] (window stride pws floats) -> d_spec [B][frames][nmel] (window stride sws floats) */
int bnn_logmel_run(bnn_logmel *op, int B, const float *d_pcm, long long pws, float *d_spec, long long sws,
                   void *stream);
void bnn_logmel_free(bnn_logmel *op);

/* FE_DBIMG, the dB-image front end of the v3.0 models (src/fe_dbimg.c:49-235 driven by src/rt_ops_f32x.c:15-86),
 * batched: p = the op record's 21 ints [nsamp N hop pad padmode nfr nmel R has_top_db norm post0 post1 post2 1 Ho Wo C
 * chan0 chan1 ld halo] and its tensors (host pointers) window [N], mel [nmel][N / 2 + 1], rows [R],
 * consts {floor, top_db, eps, post[3], chan0[C], chan1[C]}, checked as fe_db_init checks them; batch = the most
 * windows one bnn_dbimg_run call takes (it sizes the device scratch). The log is the correctly rounded logf (the
 * reference calls the C library's); see bnn_dbimg_run. */
typedef struct bnn_dbimg bnn_dbimg;
bnn_dbimg *bnn_dbimg_new(const int32_t *p, int np, const float *window, const float *mel, const int32_t *rows,
                         const float *consts, int batch);
/* floats in one window's image: (Ho + 2 halo) (Wo + 2 halo) ld, the halo zero */
long long bnn_dbimg_image_elems(const bnn_dbimg *op);
/* d_pcm [B][nsamp] (window stride pws floats) -> d_img [B][image] (window stride iws floats); 0 <= B <= batch */
int bnn_dbimg_run(bnn_dbimg *op, int B, const float *d_pcm, long long pws, float *d_img, long long iws, void *stream);
void bnn_dbimg_free(bnn_dbimg *op);

/* PROTO_S8, the int8 prototype head (src/rt_ops_s8n.c:212-250: pc_quant_cells_f32 and pc_proto_colmax_s8n,
 * src/proto_s8n.c:28-164, then pc_proto_logits, src/pc_kern_f32.c:364-376), batched. The package's tensors (host
 * pointers): prototypes qw [Np/4][Kp/16][4][16] int8, sw [Np], n4 [Np/4] (checked as pc_proto_n4_check does; the GPU
 * sums never wrap, so the flags only gate loading), class weights cls_w [N = nc x ppc], biases cls_b [nc], eps; P
 * cells of K = C channels per window (K % 8 == 0, P % 4 == 0), up to batch_cap windows per run. */
typedef struct bnn_proto_s8 bnn_proto_s8;
bnn_proto_s8 *bnn_proto_s8_new(int N, int K, int Kp, int Np, const int8_t *qw, const float *sw, const uint8_t *n4,
                               const float *cls_w, const float *cls_b, int nc, int ppc, float eps, int P,
                               int batch_cap);
/* B windows of cells d_x [B][P][ld] (window stride xws floats) -> d_colmax [B][cws] (the column maxima, Np per
 * window) and d_logits [B][lws] (nc per window). d_status [B] (or NULL): -2 for a window whose logits failed the
 * finite check (where pc_proto_logits returns -2), else 0. */
int bnn_proto_s8_run(bnn_proto_s8 *op, int B, const float *d_x, long long xws, int ld, float *d_logits, long long lws,
                     float *d_colmax, long long cws, int *d_status, void *stream);
/* PROTO variant 2 (the neon-fp16 path's SDOT head, src/rt_ops_f16.c:252-283: pc_quant_cells_f16, src/pc_proto_s8.c:
 * 13-45, pc_proto_colmax_s8, then pc_proto_logits), batched: prototypes qw [Np/12][K/4][12][4] int8 (Np % 12 == 0,
 * Np >= N, K % 8 == 0), sw [Np], cls_w, cls_b, eps as above; P % 8 == 0 cells of IEEE-half channels per window. Run
 * with bnn_proto_s8h_run (fp16 cells d_x [B][P][ld], as uint16 bits); the rest of the API (read_scratch, error, free)
 * is shared. The quantized bytes saturate to [-128, 127] (the fp16 quantizer has no -127 clamp). */
bnn_proto_s8 *bnn_proto_s8h_new(int N, int K, int Np, const int8_t *qw, const float *sw, const float *cls_w,
                                const float *cls_b, int nc, int ppc, float eps, int P, int batch_cap);
int bnn_proto_s8h_run(bnn_proto_s8 *op, int B, const uint16_t *d_x, long long xws, int ld, float *d_logits,
                      long long lws, float *d_colmax, long long cws, int *d_status, void *stream);
/* copies the op's own device scratch as the last run of B windows left it to host memory (synchronous; either pointer
 * may be NULL): the quantized cells qa [B * P][Kp] int8 (for a variant-2 head [B * P][K rounded up to 16], zero past
 * K) and their scales sx [B * P] (the reference's qa buffer and per-cell scale state) */
int bnn_proto_s8_read_scratch(bnn_proto_s8 *op, int B, int8_t *qa, float *sx);
/* the device error word of the op's GEMM (0 = no bounded wait ran out) */
int bnn_proto_s8_error(bnn_proto_s8 *op);
void bnn_proto_s8_free(bnn_proto_s8 *op);

/* ---- PW f16: the neon-fp16 path's 1x1 conv (gemm_f16, src/gemm_f16.c:109-169; record src/rt_ops_f16.c:53-82).
 * Weights as the package stores them: hp_pack panels [Np/16][Kp][16] then, when Np % 16, a [Kp][8] tail panel, b32
 * [Np] and b16 [Np] (fp16 values are IEEE half bits); Np = N rounded up to 8, Kp >= K a multiple of 8. A run scores B
 * windows of Mw rows: d_x rows of Kp fp16 values at row stride lda (a multiple of 8, >= Kp; window stride xws, a
 * multiple of 8; 16-byte aligned) -> d_out fp16 rows of Np values at stride ldo (>= Np, a multiple of 4; window stride
 * ows), stored at the padded row when opad (ow pixels a row, zero halo opad: the buffer's halo is not written);
 * act 0 none, 1 SiLU (the reference's table form), 2 ReLU; d_res (or NULL): fp16 rows at stride ldr added after
 * the activation. Bit-identical to the reference's fp16 arithmetic (fp16 FMA chains over K blocks of <= 128,
 * fp32 flushes). */
typedef struct bnn_pw_f16 bnn_pw_f16;
bnn_pw_f16 *bnn_pw_f16_new(int N, int K, int Kp, int Np, const uint16_t *panels, const float *b32,
                           const uint16_t *b16);
int bnn_pw_f16_run(bnn_pw_f16 *op, int B, int Mw, const void *d_x, long long xws, int lda, int act, void *d_out,
                   long long ows, int ldo, int ow, int opad, const void *d_res, long long rws, int ldr, void *stream);
void bnn_pw_f16_free(bnn_pw_f16 *op);

/* DW3 (src/gemm_f32.c:398-411, dw3x3_f32), batched: d_xp [B][(H+2)(W+2)][C] (zero halo 1), d_w [9][C], d_b [C] ->
 * d_out [B][Ho Wo][C], d_chsum [B][C] (NULL: the channel sums are not formed, and the rows of a window are spread
 * over several CTAs). A bounded device wait that ran out is reported by bnn_cuda_op_error. */
int bnn_cuda_dw3(int B, const float *d_xp, long long xws, int H, int W, int C, int s, const float *d_w,
                 const float *d_b, float *d_out, long long ows, int Ho, int Wo, float *d_chsum, long long cws,
                 void *stream);

/* DW3 f16 (dw3x3_f16_cr, src/kern_f16.c:83-155; record src/rt_ops_f16.c:64-103), batched: d_xp [B][(H+2)(W+2)][C]
 * fp16 (zero halo 1; window stride xws), d_w [9][C], d_b [C] fp16 -> d_out [B][Ho Wo][C] fp16, d_chsum [B][C] fp32;
 * stride s 1 | 2, output pixel (oy, ox) reads input rows oy s - pt + 1 .. + 2 and columns ox s - pl + 1 .. + 2 of the
 * haloed image (pt, pl in {0, 1}); Ho <= 12288. A bounded device wait that ran out is reported by bnn_cuda_op_error. */
int bnn_cuda_dw3_f16(int B, const void *d_xp, long long xws, int H, int W, int C, int s, int pt, int pl,
                     const void *d_w, const void *d_b, void *d_out, long long ows, int Ho, int Wo, float *d_chsum,
                     long long cws, void *stream);

/* DWK f16 (pc_dwk_f16_cr, src/pc_kern_f16.c:16-96; record src/rt_ops_f16.c:192-202, checks src/rt_ops_f32.c:435-451),
 * batched: d_xp [B][(H+2h)(W+2h)][C] fp16 zero-haloed by h = (k - 1) / 2 (window stride xws), d_w [k*k][C], d_b [C]
 * fp16 -> d_out [B][Ho Wo][C] fp16, d_chsum [B][C] fp32; k odd 1..7, stride s 1 | 2, output pixel (oy, ox) reads
 * rows oy s - pt + h + ky and columns ox s - pl + h + kx (pt, pl in 0..h); act 0 none | 1 the SiLU table; at most 768
 * pixel groups (Wo / 4 fours, then a pair, then a single pixel) per output row. */
int bnn_cuda_dwk_f16(int B, const void *d_xp, long long xws, int H, int W, int C, int k, int s, int pt, int pl,
                     const void *d_w, const void *d_b, int act, void *d_out, long long ows, int Ho, int Wo,
                     float *d_chsum, long long cws, void *stream);

/* STEM f32 -> f16 (stem_run, src/rt_ops_f16.c:175-190: pc_im2col1 + gemm_f32 + pc_cvt_pad_f16), batched: the VALID
 * k x k stride-s conv of the 1-channel image d_img [B][H][W] fp32 (window stride iws) with the package's fp32 GEMM
 * panels d_w [Np/8][Kp][8] and bias d_b [Np] (Np = N rounded up to 8, Kp >= k k, a multiple of 4): one fp32
 * accumulator per output over all Kp taps, + bias, act 0 none | 1 SiLU | 2 ReLU, rounded to fp16 into d_out at the
 * padded position ((Ho + 2 opad) (Wo + 2 opad) pixels of ldo channels per window, window stride ows; channels N..ldo
 * and the halo are not written). (Np Kp + Np) fp32 weights at most 48 KB. */
int bnn_cuda_stem_f16(int B, const float *d_img, long long iws, int H, int W, int k, int s, int Ho, int Wo,
                      const float *d_w, const float *d_b, int N, int Kp, int act, void *d_out, long long ows, int ldo,
                      int opad, void *stream);

/* the current device's error word of the per-op entry points (0 = no bounded device wait ran out; then reset to 0;
 * -1 if it cannot be read); synchronous */
int bnn_cuda_op_error(void);

/* Failure-path hooks for tests.
 * bnn_debug_fail_alloc: the host_k-th host allocation and the dev_k-th device allocation the library makes from now
 * on fail as if memory had run out (0 = none); the call that makes it fails with BNN_ERR_OOM and frees what it had.
 * bnn_debug_stall_next_gemm: the next int8 GEMM launch in this process issues no TMA load and no MMA, and every wait
 * of its warps gives up after 200 us (nothing is in flight when they do); the call that launched it fails with
 * BNN_ERR_WINDOW ("a GPU kernel's bounded wait ran out") and the context stays usable. */
int bnn_debug_fail_alloc(int host_k, int dev_k);
void bnn_debug_stall_next_gemm(void);

/* elementwise functions of the int8 path, for tests: 0 SiLU, 1 SiLU (table estimate), 2 sigmoid, 3 FRECPE,
 * 4 log2 polynomial, 5 exp2 polynomial (front end), 6 glibc expf, 7 SiLU on paired fp32 lanes (table estimate),
 * 8 fma(x, 1.7f, 0.3f) on paired fp32 lanes, 9 the dB-image front end's logarithm (double log rounded to float) */
int bnn_cuda_fn(int fn, int n, const float *d_x, float *d_y, void *stream);

/* the fp16 FMA pipe's throughput, for a roofline: blocks x 256 threads each run iters x 16 fp16 FMAs (8 chains of
 * fma.rn.f16x2); d_word: one device word the result is kept live in. Time it with events on the stream. */
int bnn_cuda_peak_hfma2(int blocks, int iters, void *d_word, void *stream);

#ifdef __cplusplus
}
#endif
#endif
