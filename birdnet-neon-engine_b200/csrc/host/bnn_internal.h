/* Internal types of the B200 bnneon runtime (host side, C11). */
#ifndef BNN_INTERNAL_H
#define BNN_INTERNAL_H
#include <stddef.h>
#include <stdint.h>

#include "../../../include/bnneon.h"
#include "../cuda/bnn_kernels.h"

/* ---- the .bnpk format (python/bnneon/compiler/pkgfmt.py:1-22; the same byte layout, read-only here) */
enum { BNN_F32 = 0, BNN_F16 = 1, BNN_I8 = 2, BNN_I32 = 3 };
typedef struct {
  char name[48];
  uint32_t dtype, ndim, dims[4];
  uint64_t offset, nbytes, reserved;
} bnn_tensor_rec; /* 96 bytes */
typedef struct {
  uint32_t dtype, H, W, C, ld, halo, slot, reserved;
  uint64_t elems;
} bnn_buf_rec; /* 40 bytes */
typedef struct {
  char name[24];
  uint32_t hwcap, n_buf, n_ops, ops_bytes, in_buf, out_buf, emb_buf, reserved;
  uint64_t buf_off, ops_off;
} bnn_path_rec; /* 72 bytes */

typedef struct bnn_pkg {
  uint8_t *map;
  size_t size;
  uint32_t n_meta, n_tensors, n_paths;
  int version;
  const uint8_t *meta;
  size_t meta_bytes;
  bnn_tensor_rec *tensors;
  bnn_path_rec *paths;
} bnn_pkg;

bnn_pkg *bnn_pkg_open(const char *path, char *err, size_t errlen);
void bnn_pkg_close(bnn_pkg *p);
int bnn_meta_str(const bnn_pkg *p, const char *key, char *buf, size_t n);
int bnn_meta_i64(const bnn_pkg *p, const char *key, int64_t *v);
int bnn_meta_f64(const bnn_pkg *p, const char *key, double *v);
/* the raw value of a metadata record (type 0 string or 3 bytes): NULL if absent */
const uint8_t *bnn_meta_raw(const bnn_pkg *p, const char *key, uint16_t *type, uint32_t *len);
const char *bnn_dtype_name(uint32_t dt);

/* ---- opcodes of the registry (src/rt.h:170-208; append-only, the same numbers) */
enum {
  BNN_OP_FE_STFT2 = 1, BNN_OP_C0POOL = 2, BNN_OP_PW = 3, BNN_OP_DW3 = 4, BNN_OP_SE = 5, BNN_OP_POSTPC = 6,
  BNN_OP_DENSE = 7, BNN_OP_FE_LOGMEL = 8, BNN_OP_STEM = 9, BNN_OP_DWK = 10, BNN_OP_PAD = 11, BNN_OP_MEAN = 12,
  BNN_OP_FE_DBIMG = 16, BNN_OP_CONVK = 17, BNN_OP_GEM = 18, BNN_OP_SED = 19, BNN_OP_VADD = 20, BNN_OP_CONVW = 21,
  BNN_OP_SED_S8 = 24, BNN_OP_PW_S8 = 22, BNN_OP_GEMV_S8 = 23, BNN_OP_SE_GATE = 25, BNN_OP_PROTO_S8 = 35, BNN_OP_N = 36
};
/* the fp16 kernels of the neon-fp16 path: base | variant 1 << 8 (src/rt_pkg.c:320-331, src/rt_ops_f16.c:286-299) */
enum {
  BNN_OP_C0POOL_F16 = 0x102, BNN_OP_PW_F16 = 0x103, BNN_OP_DW3_F16 = 0x104, BNN_OP_SE_F16 = 0x105,
  BNN_OP_POSTPC_F16 = 0x106, BNN_OP_DENSE_F16 = 0x107,
  /* compiled models' fp16 bodies (Perch): STEM = 9, DWK = 10, PAD = 11, MEAN = 12 (src/rt.h:179-182) */
  BNN_OP_STEM_F16 = 0x109, BNN_OP_DWK_F16 = 0x10a, BNN_OP_PAD_F16 = 0x10b, BNN_OP_MEAN_F16 = 0x10c,
  /* PROTO = 13 variant 2: the int8 prototype head of the fp16 path (src/rt_ops_f16.c:280-283) */
  BNN_OP_PROTO_F16S8 = 0x20d
};
enum { BNN_ACT_NONE = 0, BNN_ACT_SILU = 1, BNN_ACT_RELU = 2 };

/* one decoded op record (pointers into the package) */
typedef struct {
  uint16_t code, nb, nt, ni;
  const int32_t *b, *t, *p;
  const char *kname;
} bnn_op;

/* per device, per op: the weights in the kernels' layouts */
typedef struct {
  /* PW_S8 / GEMV_S8 */
  int8_t *w;
  float *sw, *bias;
  int32_t *cs;
  bnnk_gemm_plan plan;
  int kq;
  /* PW_S8 pairs (pwl, then the ungated expand that reads its rows): qnext = this op's GEMM epilogue quantizes its
   * stored rows for op i + 1; qsel = this op's quantized rows live in the second scratch (q2, sa2, za2), which the
   * op before writes while its own GEMM still reads the first */
  int qnext, qsel;
  /* SED_S8: its three int8 GEMMs (fc, att, cla), each with its weights and plan as a PW_S8 op has them */
  void *sub;
  /* DW3, SE_GATE, C0POOL, POSTPC; PROTO_S8: f[0] chunk maxima scratch, f[1] class weights, f[2] class biases */
  float *f[10];
  /* PROTO_S8: prototype rows w [Np][Kp], sw, the GEMM plan, eps */
  bnnk_proto_plan pplan;
  float eps;
  /* FE_LOGMEL: the device tables and their allocations */
  bnnk_logmel_tables lm;
  void *lm_mem[8];
  /* FE_DBIMG: the device tables (one allocation) and the scratch for the batch */
  bnnk_dbimg_tables db;
  void *db_mem;
  float *db_scratch;
  /* fp16 ops: hw the fp16 weights (C0POOL k-major [64][24], DW3 [9][C], DENSE [N][1024]), hwd the GEMM weights
   * k-major [Kp][Np] with each weight in both halves of a word, hb the fp16 bias */
  uint16_t *hw, *hb;
  uint32_t *hwd;
  /* PW f16 in the tensor mode: the weights K-major, [Np][Kp] fp16 (row n = output channel n) */
  uint16_t *hwk;
} bnn_devop;

typedef struct {
  int dev;
  void *stream; /* cudaStream_t */
  int owns_tables;
  void **buf;           /* device pointer per package buffer (NULL for the int8 scratch buffers) */
  long long *ws;        /* window stride per buffer (elements) */
  void *arena;          /* shared-slot memory */
  void **priv;          /* per-buffer private allocations (halos, input) */
  bnn_devop *ops;
  int8_t *q;            /* int8 GEMM scratch: [batch * rows][kq] */
  int8_t *q2;           /* the second int8 scratch (sa2, za2): rows quantized by a pwl GEMM for the expand after it */
  float *sa2;
  int32_t *za2;
  int fused_q;          /* PW_S8 quantizer launches this device's set-up folded into the GEMM before */
  int launches_fq;      /* PW_S8 ops of the last whole-package launch sequence that ran as one launch (kFQ) */
  float *sa, *fe_minmax, *pcin;
  int32_t *za;
  uint16_t *g16;        /* SE f16: the fp16 gates [batch][C] */
  int *err;             /* device words: [0] the error word of the bounded waits, [1] the smallest failed window index
                         * of the call (BNNK_NO_FAIL if none; set by PROTO_S8's logits and POSTPC f16's features) */
  int *err_host;        /* pinned copy of both */
  int w_base;           /* index of the launch's first window in the caller's call (failed-window reports) */
  bnnk_fe_tables fe;
  void *fe_mem[32];     /* the front-end tables: 9 per spectrogram */
  int n_fe_mem;
  /* bnn_infer_batch's upload pipeline: two device input buffers of up_cap windows (outside the slot plan, whose
   * input slot later ops may reuse), a copy stream, and per buffer an upload-done and a compute-done event */
  float *up[2];
  int up_cap;
  void *up_stream, *up_stream2;  /* two copy streams: each chunk's upload is split between them (one host-to-device
                                  * copy reaches ~29 GB/s on PCIe Gen5 x16, two concurrent ones ~39 GB/s) */
  void *up_ready[2], *up_free[2], *up_half[2];
  /* CUDA graphs of whole launch sequences (bnn_rt_run): one per (windows, input buffer, first window of the call);
   * a key seen once runs eagerly, the second time it is captured. graphs_off: capture failed or BNN_GRAPHS=0. */
  struct { int n, w_base, seen; const void *in; void *exec; } graphs[8];
  int n_graphs, graphs_off;
  /* per-op CUDA-event profile (bnn_profile_*): events[2 i], events[2 i + 1] bracket op i of the last launch */
  void **events;
  double *op_ms;
  int prof_on, prof_op0, prof_op1;
} bnn_dev;

struct bnn_ctx {
  bnn_pkg *pkg;
  int path_index;
  const bnn_path_rec *path;
  bnn_buf_rec *bufd;
  bnn_op *ops;
  int n_ops;
  bnn_info info;
  int batch;      /* windows per launch sequence and device */
  int n_dev;      /* devices in use */
  int dev_ids[64];
  bnn_dev *dev[64];
  int launches;   /* kernel launches per batch, before the set-up's PW_S8 pair fusion */
  int launches_fused; /* launches the pair fusion of the devices' set-up removed (the same on every device) */
  int prof;       /* BNN_PROF */
  int f16_tensor; /* the neon-fp16 path's 1x1 convs on the tensor cores (bnn_set_fp16_tensor, BNN_F16_TENSOR) */
};

/* the runtime (bnn_rt.c) */
/* decodes and validates the path's op list; 0 or -1 with err set (kind: BNN_ERR_*) */
int bnn_rt_open(bnn_ctx *c, char *err, size_t errlen, int *kind);
/* device state for c->dev_ids[i]: weights, arena for c->batch windows */
int bnn_rt_device(bnn_ctx *c, int i, char *err, size_t errlen, int *kind);
void bnn_rt_device_free(bnn_ctx *c, int i);
/* n <= batch windows on device i: pcm at d_pcm (window stride n_samples); outputs stay in the arena */
int bnn_rt_launch(bnn_ctx *c, int i, int n, const float *d_pcm, int op0, int op1, void *stream);
/* the whole op list on n windows, replayed from a CUDA graph when the same (n, d_pcm, w_base) ran before */
int bnn_rt_run(bnn_ctx *c, int i, int n, const float *d_pcm, void *stream);
int c0_quantizes_next(const bnn_ctx *c, int i);
int bnn_hpack_kmajor(bnn_devop *d, const uint16_t *panels, int Kp, int Np, char *err, size_t errlen, int *kind);
/* the op that reports failed windows (-2) through the failed-window word (PROTO_S8, POSTPC f16), or -1 */
int bnn_window_fail_op(const bnn_ctx *c);
void bnn_rt_close(bnn_ctx *c);
int bnn_s8_weights(bnn_devop *d, int N, int K, int Kp, int Np, const int8_t *src, const float *sw_src,
                   const int32_t *cs_src, const float *b_src, int rows_cap, char *err, size_t errlen, int *kind);
int bnn_proto_weights(bnn_devop *d, int N, int Kp, int Np, const int8_t *src, const float *sw_src, const float *cw,
                      const float *cb, int nc, float eps, char *err, size_t errlen, int *kind);
int bnn_proto_weights_l(bnn_devop *d, int layout, int N, int K, int Kq, int Np, const int8_t *src, const float *sw_src,
                        const float *cw, const float *cb, int nc, float eps, char *err, size_t errlen, int *kind);
int bnn_proto_n4_check(const int8_t *qw, int Kp, const uint8_t *n4, int npanels);
/* hp_pack panels as the fp16 GEMM's k-major [Kp][Np] weights (dup: each in both halves of a word, to d->hwd; else
 * plain fp16, to d->hw), b16 to d->hb, b32 to *b32 unless NULL */
int bnn_hpack_weights(bnn_devop *d, int dup, const uint16_t *panels, const float *b32src, const uint16_t *b16src,
                      int Kp, int Np, float **b32, char *err, size_t errlen, int *kind);
/* pc_logmel_new's tables on the current device (t points into d->lm_mem); -1 with err set on failure */
int bnn_logmel_build(bnn_devop *d, int nsamp, int frame, int hop, int pad, int nfft, int nmel, const float *window,
                     const float *mel, float floor_, float scale, char *err, size_t errlen, int *kind);
void bnn_logmel_release(bnn_devop *d);
/* allocation-failure injection for tests (bnn_debug_fail_alloc): 1 when this host / device allocation is to fail */
int bnn_fail_host_alloc(void);
int bnn_fail_dev_alloc(void);

/* FE_DBIMG tables (fe_db_new, src/fe_dbimg.c:49-107) from the record's 21 ints and its tensors, and a scratch for
 * batch windows */
int bnn_dbimg_build(bnn_devop *d, const int32_t *p, const float *window, const float *mel, const int32_t *rows,
                    const float *consts, int batch, char *err, size_t errlen, int *kind);
void bnn_dbimg_release(bnn_devop *d);

/* errors (bnn_api.c): thread-local message and kind */
void bnn_set_error(int kind, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

/* sha256 (sha256.c) */
typedef struct {
  uint32_t h[8];
  uint64_t len;
  uint8_t buf[64];
  size_t fill;
} bnn_sha256;
void bnn_sha256_init(bnn_sha256 *s);
void bnn_sha256_update(bnn_sha256 *s, const void *data, size_t n);
void bnn_sha256_final(bnn_sha256 *s, uint8_t out[32]);

#endif
