/* bnneon API v2 on NVIDIA B200 (sm_100a): the drop-in replacement of libbnneon's public C interface.
 *
 * Replaces src/bnneon.h:22-99 of the reference (cdw9bf/birdnet-neon-engine) symbol for symbol: the same functions,
 * enums, error kinds and bnn_info layout (fields are only ever appended; struct_size handshake), so hosts that bind
 * the reference library (BirdNET-Go through cgo + dlopen, python/bnneon/binding.py through ctypes, bench/cli.c) load
 * this libbnneon.so unchanged. The weights file is a compiled .bnpk package (magic BNNPKG01); its op list runs on the
 * GPU with hand-written sm_100a kernels whose outputs equal the reference's AArch64 outputs bit for bit on the
 * neon-int8 path.
 *
 * What differs, by design:
 *  - "path" names stay the package's ("neon-int8"): the package format and its paths are unchanged. Modes 0 and 4
 *    select the neon-int8 path; the fp16 / fp32 paths have no GPU kernels yet and are refused with BNN_ERR_CPU
 *    ("no path this device can run"), as the reference refuses a path its CPU cannot run. Legacy .bn24 / .bnv3 files
 *    are refused with BNN_ERR_PACKAGE.
 *  - bnn_set_threads(ctx, n) sets how many GPUs the context spreads a batch over (1..the visible devices; at most
 *    64). The outputs are bit-identical for every count, as the reference guarantees for its thread counts.
 *  - bnn_infer is bnn_infer_batch (bnneon_cuda.h) with one window.
 * Thread safety as before: one context per host thread; contexts share nothing. */
#ifndef BNNEON_H
#define BNNEON_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define BNN_API_VERSION 2

/* model family codes (informational) */
enum { BNN_MODEL_V24 = 24, BNN_MODEL_V30 = 30, BNN_MODEL_PERCH_V2 = 120, BNN_MODEL_BAT_V24 = 224 };
/* what bnn_infer writes: always raw logits from this library */
enum { BNN_OUT_LOGITS = 0, BNN_OUT_SIGMOID = 1 };
/* what the host applies to the logits */
enum { BNN_POST_NONE = 0, BNN_POST_SIGMOID = 1, BNN_POST_SOFTMAX = 2 };
/* bnn_init modes: 0 the best path of the package this device runs, 1 the fp32 reference engine of legacy files
 * (refused for packages), 2 the "neon-fp32" path, 3 the "neon-fp16" path, 4 the "neon-int8" path */
enum { BNN_MODE_DEFAULT = 0, BNN_MODE_REFERENCE = 1, BNN_MODE_FP32 = 2, BNN_MODE_FP16 = 3, BNN_MODE_INT8 = 4 };

typedef struct {
  uint32_t struct_size;  /* in: the caller's sizeof(bnn_info); out: the bytes the library filled (the smaller) */
  int model;             /* BNN_MODEL_* */
  int format_version;    /* >= 1 for a .bnpk */
  int sample_rate;       /* Hz */
  int n_samples;         /* samples per window */
  int hop_samples;       /* default hop between windows (0 = the caller's choice) */
  int n_classes;         /* outputs per window */
  int output_kind;       /* BNN_OUT_* */
  int post;              /* BNN_POST_* */
  float logit_scale;     /* applied by the host before post */
  int emb_dim;           /* embedding length (0 = none) */
  int has_labels_sha;
  unsigned char labels_sha256[32];
  char model_id[64];
  char path[32];         /* after init: the chosen package path; after probe: the best runnable path ("" = none) */
  const char *precision; /* static text ("" after probe) */
} bnn_info;

typedef struct bnn_ctx bnn_ctx;

int bnn_api_version(void);
/* legacy engines' family check (src/bnneon.c:51-54 answers): 1 for V24, PERCH_V2, BAT_V24; V30 answers 0 here (its
 * legacy engine needs fp16 + dotprod NEON); packages are judged by bnn_probe's info.path */
int bnn_cpu_supported(int model);
/* header and metadata only: fills info or returns -1 */
int bnn_probe(const char *weights_path, bnn_info *info);
/* a metadata string by key (numbers as decimal text; "license" and "licence" are one key): copies at most n - 1
 * bytes + NUL, returns the full length or -1 when absent */
int bnn_probe_meta(const char *weights_path, const char *key, char *buf, size_t n);
int bnn_meta(const bnn_ctx *ctx, const char *key, char *buf, size_t n);
bnn_ctx *bnn_init(const char *weights_path, int mode);
int bnn_get_info(const bnn_ctx *ctx, bnn_info *info);
/* one window of info.n_samples floats -> info.n_classes logits (+ the embedding when emb != NULL); 0 on success */
int bnn_infer(bnn_ctx *ctx, const float *pcm, float *out, float *emb);
/* 0 if labels_path is byte for byte the label file the package was compiled with, else -1 (BNN_ERR_LABELS) */
int bnn_verify_labels(const char *weights_path, const char *labels_path);
/* the last failure of this thread: "<what failed>: <expected> vs <found>; hint: <what to do>" (<= 511 bytes) */
const char *bnn_last_error(void);
enum { BNN_ERR_NONE = 0, BNN_ERR_PACKAGE = 1, BNN_ERR_OOM = 2, BNN_ERR_CPU = 3, BNN_ERR_WINDOW = 4,
       BNN_ERR_LABELS = 5, BNN_ERR_USAGE = 6 };
int bnn_last_error_kind(void);
/* the number of GPUs this context uses (1..64, at most the visible devices); 0 on success */
int bnn_set_threads(bnn_ctx *ctx, int threads);
void bnn_free(bnn_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif
