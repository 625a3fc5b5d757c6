/* The public C API (include/bnneon.h, include/bnneon_cuda.h) over the B200 package runtime.
 *
 * Replaces src/bnneon.c:30-387 of the reference for compiled packages: probe / metadata / labels answer from the
 * package exactly as there (the same keys, the same license-key alias, the same struct_size handshake and error
 * texts); bnn_init picks the package path by name for the mode and builds the GPU context; bnn_infer runs the op list
 * on the GPU. Legacy .bn24 / .bnv3 files (the hand-written NEON engines) are refused: there is no GPU engine for
 * them. */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "../../../include/bnneon_cuda.h"
#include "bnn_internal.h"

static __thread char g_err[512];
static __thread int g_kind;

void bnn_set_error(int kind, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  g_kind = kind;
}
#define ERR(kind, ...) bnn_set_error((kind), __VA_ARGS__)

const char *bnn_last_error(void) { return g_err; }
int bnn_last_error_kind(void) { return g_kind; }
int bnn_api_version(void) { return BNN_API_VERSION; }

int bnn_cpu_supported(int model) {
  return model == BNN_MODEL_V24 || model == BNN_MODEL_PERCH_V2 || model == BNN_MODEL_BAT_V24;
}

static const char *base_name(const char *path) {
  const char *s = strrchr(path, '/');
  return s ? s + 1 : path;
}

/* the package paths a mode names (src/bnneon.c:73-78: mode -> path name, precision text) */
static const struct { int mode; const char *name, *precision; } PATHS[] = {
    {BNN_MODE_FP16, "neon-fp16", "fp16"},
    {BNN_MODE_INT8, "neon-int8", "int8 GEMMs, fp32 elsewhere"},
    {BNN_MODE_FP32, "neon-fp32", "fp32"},
};

/* 1 when every op of path i has a GPU kernel here (the neon-int8 path's ops, variant 0, and the neon-fp16 path's,
 * variant 1) */
static int path_runs_here(const bnn_pkg *p, int i) {
  static const int codes[] = {BNN_OP_FE_STFT2, BNN_OP_C0POOL, BNN_OP_PW_S8, BNN_OP_DW3, BNN_OP_SE_GATE,
                              BNN_OP_POSTPC, BNN_OP_GEMV_S8, BNN_OP_PROTO_S8, BNN_OP_FE_LOGMEL, BNN_OP_FE_DBIMG, BNN_OP_DENSE,
                              BNN_OP_C0POOL_F16, BNN_OP_PW_F16, BNN_OP_DW3_F16, BNN_OP_SE_F16, BNN_OP_POSTPC_F16,
                              BNN_OP_DENSE_F16, BNN_OP_STEM_F16, BNN_OP_DWK_F16, BNN_OP_PAD_F16, BNN_OP_MEAN_F16,
                              BNN_OP_PROTO_F16S8, BNN_OP_STEM, BNN_OP_DWK, BNN_OP_PAD, BNN_OP_MEAN, BNN_OP_CONVK,
                              BNN_OP_GEM, BNN_OP_SED, BNN_OP_VADD, BNN_OP_CONVW, BNN_OP_SED_S8, BNN_OP_PW};
  const bnn_path_rec *d = &p->paths[i];
  const uint8_t *q = p->map + d->ops_off, *end = q + d->ops_bytes;
  for (uint32_t k = 0; k < d->n_ops; k++) {
    if (q + 12 > end) return 0;
    uint16_t h[6];
    memcpy(h, q, 12);
    int ok = 0;
    for (size_t j = 0; j < sizeof codes / sizeof codes[0]; j++) ok |= h[0] == codes[j];
    if (!ok || h[1] < 12) return 0;
    q += h[1];
  }
  return 1;
}

/* the first path (paths are stored fastest first) this library runs; want: a path name, "" = any */
static int pick_path(const bnn_pkg *p, const char *want) {
  for (uint32_t i = 0; i < p->n_paths; i++) {
    if (want[0] && strncmp(p->paths[i].name, want, sizeof p->paths[i].name)) continue;
    if (path_runs_here(p, (int)i)) return (int)i;
  }
  return -1;
}

static void no_path_error(const char *path, const bnn_pkg *p, const char *want) {
  char list[256] = "";
  size_t k = 0;
  int present = 0;
  for (uint32_t i = 0; i < p->n_paths && k + 64 < sizeof list; i++) {
    if (want[0] && !strncmp(p->paths[i].name, want, 24)) present = 1;
    k += (size_t)snprintf(list + k, sizeof list - k, "%s%.24s", i ? ", " : "", p->paths[i].name);
  }
  char id[64] = "";
  bnn_meta_str(p, "model_id", id, sizeof id);
  if (want[0] && !present)
    ERR(BNN_ERR_CPU, "%s: path %s is not in this package (it has: %s); hint: use mode 0 to let the library pick, or a "
        "package of this model compiled for %s (%s-%s.bnpk)", path, want, list, want, id[0] ? id : "<model_id>", want);
  else
    ERR(BNN_ERR_CPU, "%s: this GPU library runs none of the package's paths%s%s (it has: %s; B200 kernels exist for the "
        "neon-int8 and neon-fp16 paths); hint: use the neon-int8 package of this model (%s-neon-int8.bnpk) or compile "
        "one with --paths neon-int8", path, want[0] ? " named " : "", want, list, id[0] ? id : "<model_id>");
}

static void pkg_info(const bnn_pkg *p, int pi, bnn_info *info) {
  int64_t v;
  double x;
#define I_(key, fld) do { if (!bnn_meta_i64(p, key, &v)) info->fld = (int)v; } while (0)
  I_("family", model); I_("sample_rate", sample_rate); I_("n_samples", n_samples); I_("hop_samples", hop_samples);
  I_("n_classes", n_classes); I_("post", post); I_("emb_dim", emb_dim);
#undef I_
  info->format_version = p->version;
  info->output_kind = BNN_OUT_LOGITS;
  info->logit_scale = bnn_meta_f64(p, "logit_scale", &x) ? 1.f : (float)x;
  char sha[40];
  if (bnn_meta_str(p, "labels_sha256", sha, sizeof sha) == 32) { memcpy(info->labels_sha256, sha, 32); info->has_labels_sha = 1; }
  bnn_meta_str(p, "model_id", info->model_id, sizeof info->model_id);
  if (pi >= 0) snprintf(info->path, sizeof info->path, "%.24s", p->paths[pi].name);
}

static void copy_info(bnn_info *dst, const bnn_info *src) {
  uint32_t n = dst->struct_size;
  if (n > sizeof *src) n = sizeof *src;
  bnn_info tmp = *src;
  tmp.struct_size = n;
  memcpy(dst, &tmp, n);
}

/* header / metadata of a weights file; keep: receives the open package */
static int probe_full(const char *path, bnn_info *info, bnn_pkg **keep) {
  memset(info, 0, sizeof *info);
  info->struct_size = sizeof *info;
  info->logit_scale = 1.f;
  info->precision = "";
  FILE *f = fopen(path, "rb");
  if (!f) { ERR(BNN_ERR_PACKAGE, "cannot open %s; hint: check the path and permissions", path); return -1; }
  char magic[8];
  const int ok = fread(magic, 1, 8, f) == 8;
  fclose(f);
  if (!ok) { ERR(BNN_ERR_PACKAGE, "%s: shorter than 8 bytes; hint: incomplete download or the wrong file", path); return -1; }
  if (!memcmp(magic, "BNNPKG01", 8)) {
    bnn_pkg *p = bnn_pkg_open(path, g_err, sizeof g_err);
    if (!p) { g_kind = BNN_ERR_PACKAGE; return -1; }
    pkg_info(p, pick_path(p, ""), info);
    if (keep) *keep = p;
    else bnn_pkg_close(p);
    return 0;
  }
  if (!memcmp(magic, "BN24ENG1", 8) || !memcmp(magic, "BNV3ENG1", 8)) {
    ERR(BNN_ERR_PACKAGE, "%s: a legacy %s file for the hand-written NEON engine, which this GPU library does not run; "
        "hint: use the model's compiled package (.bnpk, neon-int8 path)", path,
        magic[2] == '2' ? "BirdNET v2.4 .bn24" : "BirdNET v3.0 .bnv3");
    return -1;
  }
  ERR(BNN_ERR_PACKAGE, "%s: not a bnneon weights file (magic '%.8s'; expected BNNPKG01 for a compiled package, "
      "BN24ENG1 for a legacy BirdNET v2.4 file); hint: compile the model with compiler/bnc.py, or check the download "
      "(sha256)", path, magic);
  return -1;
}

int bnn_probe(const char *path, bnn_info *info) {
  if (!info || info->struct_size < 8) { ERR(BNN_ERR_USAGE, "bnn_probe: bnn_info.struct_size not set"); return -1; }
  bnn_info full;
  if (probe_full(path, &full, NULL)) return -1;
  copy_info(info, &full);
  return 0;
}

static int is_license_key(const char *key) { return !strcmp(key, "license") || !strcmp(key, "licence"); }
static int pkg_meta(const bnn_pkg *p, const char *key, char *buf, size_t n) {
  int r = bnn_meta_str(p, key, buf, n);
  if (r < 0 && is_license_key(key)) r = bnn_meta_str(p, strcmp(key, "licence") ? "licence" : "license", buf, n);
  return r;
}

int bnn_probe_meta(const char *path, const char *key, char *buf, size_t n) {
  bnn_info info;
  bnn_pkg *p = NULL;
  if (probe_full(path, &info, &p)) return -1;
  const int r = pkg_meta(p, key, buf, n);
  bnn_pkg_close(p);
  return r;
}

int bnn_meta(const bnn_ctx *c, const char *key, char *buf, size_t n) {
  if (!c) return -1;
  return pkg_meta(c->pkg, key, buf, n);
}

/* ------------------------------------------------------------------ contexts */

static int visible_devices(int *ids, int max) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) return 0;
  const char *env = getenv("BNN_DEVICES");
  int k = 0;
  if (env && *env) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s", env);
    for (char *t = strtok(buf, ","); t && k < max; t = strtok(NULL, ",")) {
      const int d = atoi(t);
      if (d >= 0 && d < n) ids[k++] = d;
    }
    return k;
  }
  for (int d = 0; d < n && k < max; d++) ids[k++] = d;
  return k;
}

static int make_devices(bnn_ctx *c, int n_dev) {
  char err[512];
  int kind = BNN_ERR_CPU;
  for (int i = 0; i < n_dev; i++)
    if (!c->dev[i] && bnn_rt_device(c, i, err, sizeof err, &kind)) {
      ERR(kind, "%s path %.24s: %s", c->info.model_id, c->path->name, err);
      return -1;
    }
  c->n_dev = n_dev;
  return 0;
}

/* allocation-failure injection: the k-th host / device allocation from now fails (0 = none) */
static int g_fail_host, g_fail_dev;
static int count_down(int *k) {
  int v = __atomic_load_n(k, __ATOMIC_RELAXED);
  while (v > 0)
    if (__atomic_compare_exchange_n(k, &v, v - 1, 0, __ATOMIC_RELAXED, __ATOMIC_RELAXED)) return v == 1;
  return 0;
}
int bnn_fail_host_alloc(void) { return count_down(&g_fail_host); }
int bnn_fail_dev_alloc(void) { return count_down(&g_fail_dev); }
int bnn_debug_fail_alloc(int host_k, int dev_k) {
  if (host_k < 0 || dev_k < 0) { ERR(BNN_ERR_USAGE, "bnn_debug_fail_alloc: %d %d", host_k, dev_k); return -1; }
  __atomic_store_n(&g_fail_host, host_k, __ATOMIC_RELAXED);
  __atomic_store_n(&g_fail_dev, dev_k, __ATOMIC_RELAXED);
  return 0;
}

void bnn_debug_stall_next_gemm(void) { bnnk_debug_stall_next_gemm(); }

bnn_ctx *bnn_init(const char *path, int mode) {
  bnn_info pi;
  bnn_pkg *pkg = NULL;
  if (probe_full(path, &pi, &pkg)) return NULL;
  bnn_ctx *c = bnn_fail_host_alloc() ? NULL : calloc(1, sizeof *c);
  if (!c) { bnn_pkg_close(pkg); ERR(BNN_ERR_OOM, "out of memory (%zu bytes for the context)", sizeof *c); return NULL; }
  c->pkg = pkg;
  c->info = pi;
  if (mode == BNN_MODE_REFERENCE || mode < 0 || mode > BNN_MODE_INT8) {
    ERR(BNN_ERR_USAGE, "%s: mode %d is not available for compiled packages; hint: use mode 0 (best path for this "
        "device), 2 (the neon-fp32 path), 3 (the neon-fp16 path) or 4 (the neon-int8 path); mode 1 (fp32 reference) "
        "exists for the legacy .bn24 files only", path, mode);
    bnn_free(c);
    return NULL;
  }
  const char *want = "";
  for (size_t i = 0; i < sizeof PATHS / sizeof PATHS[0]; i++)
    if (PATHS[i].mode == mode) want = PATHS[i].name;
  c->path_index = pick_path(pkg, want);
  if (c->path_index < 0) { no_path_error(path, pkg, want); bnn_free(c); return NULL; }
  c->path = &pkg->paths[c->path_index];
  const char *eb = getenv("BNN_BATCH");
  c->batch = eb && atoi(eb) > 0 ? atoi(eb) : 64;
  const char *ep = getenv("BNN_PROF");
  c->prof = ep ? atoi(ep) : 0;
  const char *et = getenv("BNN_F16_TENSOR");
  c->f16_tensor = et && atoi(et) > 0;
  char rerr[512];
  int kind = BNN_ERR_PACKAGE;
  if (bnn_rt_open(c, rerr, sizeof rerr, &kind)) {
    ERR(kind, "%s path %.24s: %s", base_name(path), c->path->name, rerr);
    bnn_free(c);
    return NULL;
  }
  pkg_info(pkg, c->path_index, &c->info);
  /* the metadata must agree with the buffers the outputs are read from (src/bnneon.c:255-274) */
  const bnn_path_rec *d = c->path;
  const bnn_buf_rec *ib = &c->bufd[d->in_buf], *ob = &c->bufd[d->out_buf];
  const bnn_buf_rec *ebd = d->emb_buf == 0xffffffffu ? NULL : &c->bufd[d->emb_buf];
#define META_HINT "; hint: the package is inconsistent: recompile it (compiler/bnc.py) and check its 'compiler' metadata"
  if (c->info.n_samples <= 0 || ib->dtype != BNN_F32 || ib->elems != (uint64_t)c->info.n_samples) {
    ERR(BNN_ERR_PACKAGE, "%s: metadata n_samples = %d but the input buffer is %s with %llu elements" META_HINT, path,
        c->info.n_samples, bnn_dtype_name(ib->dtype), (unsigned long long)ib->elems);
    bnn_free(c);
    return NULL;
  }
  if (c->info.n_classes <= 0 || ob->dtype != BNN_F32 || ob->elems < (uint64_t)c->info.n_classes) {
    ERR(BNN_ERR_PACKAGE, "%s: metadata n_classes = %d but the output buffer is %s with %llu elements" META_HINT, path,
        c->info.n_classes, bnn_dtype_name(ob->dtype), (unsigned long long)ob->elems);
    bnn_free(c);
    return NULL;
  }
  if (c->info.emb_dim < 0 || (c->info.emb_dim && (!ebd || ebd->dtype != BNN_F32 || ebd->elems < (uint64_t)c->info.emb_dim))) {
    ERR(BNN_ERR_PACKAGE, "%s: metadata emb_dim = %d but the path's embedding buffer is %s" META_HINT, path,
        c->info.emb_dim, !ebd ? "absent" : bnn_dtype_name(ebd->dtype));
    bnn_free(c);
    return NULL;
  }
  c->info.precision = "int8 GEMMs, fp32 elsewhere";
  for (size_t i = 0; i < sizeof PATHS / sizeof PATHS[0]; i++)
    if (!strncmp(d->name, PATHS[i].name, 24)) c->info.precision = PATHS[i].precision;
  /* the package is valid: now the GPU side (on a machine without one, the validation above still runs) */
  int ids[64];
  const int nvis = visible_devices(ids, 64);
  if (nvis == 0) {
    ERR(BNN_ERR_CPU, "%s: no CUDA device is visible (this library runs packages on NVIDIA B200 GPUs); hint: check "
        "nvidia-smi, CUDA_VISIBLE_DEVICES and BNN_DEVICES", path);
    bnn_free(c);
    return NULL;
  }
  memcpy(c->dev_ids, ids, sizeof(int) * nvis);
  if (make_devices(c, 1)) { bnn_free(c); return NULL; }
  return c;
}

int bnn_get_info(const bnn_ctx *c, bnn_info *info) {
  if (!c || !info || info->struct_size < 8) { ERR(BNN_ERR_USAGE, "bnn_get_info: no context or struct_size"); return -1; }
  copy_info(info, &c->info);
  return 0;
}

void bnn_free(bnn_ctx *c) {
  if (!c) return;
  bnn_rt_close(c);
  bnn_pkg_close(c->pkg);
  free(c);
}

int bnn_set_threads(bnn_ctx *c, int threads) {
  if (!c) { ERR(BNN_ERR_USAGE, "bnn_set_threads: NULL context"); return -1; }
  if (threads < 1 || threads > 64) {
    ERR(BNN_ERR_USAGE, "bnn_set_threads: %d threads; hint: pass 1..64 (a host's 0 = all CPUs must be resolved by the host)",
        threads);
    return -1;
  }
  int ids[64];
  const int nvis = visible_devices(ids, 64);
  const int want = threads < nvis ? threads : nvis;
  for (int i = want; i < 64; i++)
    if (c->dev[i]) bnn_rt_device_free(c, i);
  return make_devices(c, want);
}

int bnn_set_batch(bnn_ctx *c, int batch) {
  if (!c || batch < 1 || batch > 65536) {
    ERR(BNN_ERR_USAGE, "bnn_set_batch: batch %d; hint: pass 1..65536 windows", batch);
    return -1;
  }
  if (batch == c->batch) return 0;
  const int n = c->n_dev;
  for (int i = 0; i < 64; i++)
    if (c->dev[i]) bnn_rt_device_free(c, i);
  c->batch = batch;
  return make_devices(c, n);
}
int bnn_get_batch(const bnn_ctx *c) { return c ? c->batch : 0; }

int bnn_set_fp16_tensor(bnn_ctx *c, int on) {
  if (!c) { ERR(BNN_ERR_USAGE, "bnn_set_fp16_tensor: NULL context"); return -1; }
  on = on != 0;
  if (on == c->f16_tensor) return 0;
  const int n = c->n_dev;
  for (int i = 0; i < 64; i++)
    if (c->dev[i]) bnn_rt_device_free(c, i);
  c->f16_tensor = on;
  return make_devices(c, n);
}
int bnn_get_fp16_tensor(const bnn_ctx *c) { return c ? c->f16_tensor : 0; }
int bnn_launches_per_batch(const bnn_ctx *c) {
  return c ? c->launches - c->launches_fused - (c->dev[0] ? c->dev[0]->launches_fq : 0) : 0;
}

/* ------------------------------------------------------------------ inference */

typedef struct {
  bnn_ctx *c;
  int di, w0, w1, rc;
  const float *pcm;
  float *out, *emb;
  char err[512];
  int kind;
} dev_job;

/* after a call's copy of the device words to err_host: a bounded wait that ran out (-1), a window that an op reported
 * as failed (-2: PROTO_S8's non-finite logits, as rt_run / bnn_infer report it, src/bnneon.c:313-325), else 0; both
 * words are reset */
static int check_err_word(bnn_ctx *c, int di) {
  bnn_dev *dv = c->dev[di];
  if (dv->err_host[1] != BNNK_NO_FAIL) {
    const int w = dv->err_host[1];
    dv->err_host[1] = BNNK_NO_FAIL;
    cudaMemsetAsync(dv->err + 1, 0x7f, sizeof(int), (cudaStream_t)dv->stream);
    const int i = bnn_window_fail_op(c);
    ERR(BNN_ERR_WINDOW, "window not scored: op %d %s reported a failed window (code -2: non-finite values on the %s "
        "path) for window %d of the call; hint: skip this window (the input itself is probably non-finite or extreme)",
        i, i >= 0 ? c->ops[i].kname : "?", c->info.path, w);
    return -2;
  }
  if (*dv->err_host) {
    const int code = *dv->err_host;
    *dv->err_host = 0;
    cudaMemsetAsync(dv->err, 0, sizeof(int), (cudaStream_t)dv->stream);
    ERR(BNN_ERR_WINDOW, "window not scored: a GPU kernel's bounded wait ran out (code %d: %s) on GPU %d; hint: the GPU "
        "is stalled or shared with a long job: retry, and check nvidia-smi", code,
        code == BNNK_ERR_TMA_WAIT ? "TMA load" : code == BNNK_ERR_MMA_WAIT ? "tensor-core operands"
        : code == BNNK_ERR_EPI_WAIT ? "GEMM result" : code == BNNK_ERR_DW3_WAIT ? "depthwise row ring"
        : code == BNNK_ERR_QUANT_WAIT ? "quantizer row copy" : "other",
        dv->dev);
    return -1;
  }
  return 0;
}

/* the upload pipeline's buffers, stream and events on the current device, sized for the context's batch */
static cudaError_t upload_setup(bnn_ctx *c, bnn_dev *dv) {
  cudaError_t e = cudaSuccess;
  if (dv->up_cap < c->batch) {
    if (dv->up_stream) e = cudaStreamSynchronize((cudaStream_t)dv->up_stream);
    if (!e && dv->up_stream2) e = cudaStreamSynchronize((cudaStream_t)dv->up_stream2);
    cudaFree(dv->up[0]); cudaFree(dv->up[1]);
    dv->up[0] = dv->up[1] = NULL;
    dv->up_cap = 0;
    const size_t bytes = sizeof(float) * (size_t)c->batch * c->info.n_samples;
    if (!e) e = cudaMalloc((void **)&dv->up[0], bytes);
    if (!e) e = cudaMalloc((void **)&dv->up[1], bytes);
    if (e) return e;
    dv->up_cap = c->batch;
  }
  if (!dv->up_stream) {
    e = cudaStreamCreateWithFlags((cudaStream_t *)&dv->up_stream, cudaStreamNonBlocking);
    if (!e) e = cudaStreamCreateWithFlags((cudaStream_t *)&dv->up_stream2, cudaStreamNonBlocking);
    for (int k = 0; k < 2 && !e; k++) {
      e = cudaEventCreateWithFlags((cudaEvent_t *)&dv->up_ready[k], cudaEventDisableTiming);
      if (!e) e = cudaEventCreateWithFlags((cudaEvent_t *)&dv->up_free[k], cudaEventDisableTiming);
      if (!e) e = cudaEventCreateWithFlags((cudaEvent_t *)&dv->up_half[k], cudaEventDisableTiming);
    }
  }
  return e;
}

/* windows per pipeline chunk: the first is a quarter of min(call, batch) (from 64 windows on; smaller calls run in one
 * chunk), the next ones a full batch, and a tail shorter than half a chunk joins its predecessor. The first upload is
 * the only one not hidden behind kernels, while every chunk pays the op list's fixed GPU latencies (~1 ms per launch
 * sequence even for one window): at batch 256 a first chunk of 64 measured best (37.5k windows/s end to end against
 * 34.9k for 128 and 34.4k for 32). BNN_CHUNK0 sets the first chunk (tuning sweeps). */
static int chunk0_env = -1;
static int next_chunk(int rem, int batch, int prev) {
  if (chunk0_env < 0) {
    const char *e0 = getenv("BNN_CHUNK0");
    chunk0_env = e0 && atoi(e0) >= 1 ? atoi(e0) : 0;
  }
  const int first = rem < batch ? rem : batch;
  int s = prev ? batch : chunk0_env ? chunk0_env : first >= 64 ? (first / 4 + 7) / 8 * 8 : first;
  if (s > rem) s = rem;
  if (rem - s > 0 && rem - s < s / 2 && rem <= batch) s = rem;
  return s;
}

/* one device's share [w0, w1) of a bnn_infer_batch call: chunk i is uploaded into buffer i % 2 by two copies in
 * parallel on the two copy streams (after chunk i - 2's kernels have finished reading it) while chunk i - 1 computes
 * on the context's stream */
static void *dev_worker(void *a) {
  dev_job *j = a;
  bnn_ctx *c = j->c;
  bnn_dev *dv = c->dev[j->di];
  const bnn_path_rec *d = c->path;
  const int ns = c->info.n_samples, nc = c->info.n_classes, ne = c->info.emb_dim;
  cudaStream_t st = (cudaStream_t)dv->stream;
  cudaError_t e = cudaSetDevice(dv->dev);
  if (!e) e = upload_setup(c, dv);
  cudaStream_t cs = (cudaStream_t)dv->up_stream, cs2 = (cudaStream_t)dv->up_stream2;
  for (int w = j->w0, k = 0, nb = 0; w < j->w1 && !e && !j->rc; w += nb, k ^= 1) {
    nb = next_chunk(j->w1 - w, c->batch, nb);
    dv->w_base = w;
    float *buf = dv->up[k];
    const int na = (nb + 1) / 2;  /* windows of the first copy */
    e = cudaStreamWaitEvent(cs, (cudaEvent_t)dv->up_free[k], 0);
    if (!e) e = cudaStreamWaitEvent(cs2, (cudaEvent_t)dv->up_free[k], 0);
    if (!e) e = cudaMemcpyAsync(buf, j->pcm + (size_t)w * ns, sizeof(float) * (size_t)na * ns,
                                cudaMemcpyHostToDevice, cs);
    if (!e && nb > na)
      e = cudaMemcpyAsync(buf + (size_t)na * ns, j->pcm + (size_t)(w + na) * ns, sizeof(float) * (size_t)(nb - na) * ns,
                          cudaMemcpyHostToDevice, cs2);
    if (!e) e = cudaEventRecord((cudaEvent_t)dv->up_half[k], cs2);
    if (!e) e = cudaStreamWaitEvent(cs, (cudaEvent_t)dv->up_half[k], 0);
    if (!e) e = cudaEventRecord((cudaEvent_t)dv->up_ready[k], cs);
    if (!e) e = cudaStreamWaitEvent(st, (cudaEvent_t)dv->up_ready[k], 0);
    if (e) break;
    if (bnn_rt_run(c, j->di, nb, buf, st)) {
      j->rc = -1;
      snprintf(j->err, sizeof j->err, "%s", g_err);
      j->kind = g_kind;
      break;
    }
    e = cudaEventRecord((cudaEvent_t)dv->up_free[k], st);
    if (!e)
      e = cudaMemcpy2DAsync(j->out + (size_t)w * nc, sizeof(float) * nc, dv->buf[d->out_buf],
                            sizeof(float) * dv->ws[d->out_buf], sizeof(float) * nc, nb, cudaMemcpyDeviceToHost, st);
    if (!e && j->emb && ne)
      e = cudaMemcpy2DAsync(j->emb + (size_t)w * ne, sizeof(float) * ne, dv->buf[d->emb_buf],
                            sizeof(float) * dv->ws[d->emb_buf], sizeof(float) * ne, nb, cudaMemcpyDeviceToHost, st);
  }
  if (!e) e = cudaMemcpyAsync(dv->err_host, dv->err, 2 * sizeof(int), cudaMemcpyDeviceToHost, st);
  if (!e) e = cudaStreamSynchronize(st);
  if (!e && cs) e = cudaStreamSynchronize(cs);
  if (!e && cs2) e = cudaStreamSynchronize(cs2);
  if (e && !j->rc) {
    j->rc = -1;
    j->kind = BNN_ERR_WINDOW;
    snprintf(j->err, sizeof j->err, "window not scored: CUDA error %d (%s) on GPU %d; hint: check the GPU (nvidia-smi)",
             (int)e, cudaGetErrorString(e), dv->dev);
  }
  if (!j->rc) {
    const int r = check_err_word(c, j->di);
    if (r) {
      j->rc = r;
      snprintf(j->err, sizeof j->err, "%s", g_err);
      j->kind = g_kind;
    }
  }
  return NULL;
}

int bnn_infer_batch(bnn_ctx *c, int n, const float *pcm, float *out, float *emb) {
  if (!c || !pcm || !out || n < 0) { ERR(BNN_ERR_USAGE, "bnn_infer_batch: NULL context, pcm or out, or n < 0"); return -1; }
  if (n == 0) return 0;
  dev_job jobs[64];
  pthread_t th[64];
  char started[64] = {0};
  const int nd = c->n_dev < n ? c->n_dev : n;
  for (int i = 0; i < nd; i++) {
    jobs[i] = (dev_job){c, i, (int)((long long)n * i / nd), (int)((long long)n * (i + 1) / nd), 0, pcm, out, emb, "", 0};
    /* one host thread per further GPU; a GPU whose thread cannot be created is driven from this thread instead, so
     * every window is still scored */
    if (i > 0 && nd > 1 && pthread_create(&th[i], NULL, dev_worker, &jobs[i]) == 0) started[i] = 1;
  }
  for (int i = 0; i < nd; i++)
    if (!started[i]) dev_worker(&jobs[i]);
  for (int i = 1; i < nd; i++)
    if (started[i]) pthread_join(th[i], NULL);
  for (int i = 0; i < nd; i++)
    if (jobs[i].rc) {
      ERR(jobs[i].kind ? jobs[i].kind : BNN_ERR_WINDOW, "%s", jobs[i].err);
      return jobs[i].rc == -2 ? -2 : -1;
    }
  return 0;
}

int bnn_infer(bnn_ctx *c, const float *pcm, float *out, float *emb) {
  if (!c || !pcm || !out) { ERR(BNN_ERR_USAGE, "bnn_infer: NULL context, pcm or out"); return -1; }
  return bnn_infer_batch(c, 1, pcm, out, emb);
}

int bnn_infer_device(bnn_ctx *c, int n, const float *d_pcm, float *d_out, float *d_emb, void *stream) {
  if (!c || !d_pcm || !d_out || n < 0 || n > c->batch) {
    ERR(BNN_ERR_USAGE, "bnn_infer_device: NULL context / pointers or n %d outside 0..%d (the batch capacity)", n,
        c ? c->batch : 0);
    return -1;
  }
  if (n == 0) return 0;
  bnn_dev *dv = c->dev[0];
  const bnn_path_rec *d = c->path;
  const int nc = c->info.n_classes, ne = c->info.emb_dim;
  cudaStream_t st = stream ? (cudaStream_t)stream : (cudaStream_t)dv->stream;
  cudaSetDevice(dv->dev);
  dv->w_base = 0;
  if (bnn_rt_run(c, 0, n, d_pcm, st)) return -1;
  cudaError_t e = cudaMemcpy2DAsync(d_out, sizeof(float) * nc, dv->buf[d->out_buf], sizeof(float) * dv->ws[d->out_buf],
                                    sizeof(float) * nc, n, cudaMemcpyDeviceToDevice, st);
  if (!e && d_emb && ne)
    e = cudaMemcpy2DAsync(d_emb, sizeof(float) * ne, dv->buf[d->emb_buf], sizeof(float) * dv->ws[d->emb_buf],
                          sizeof(float) * ne, n, cudaMemcpyDeviceToDevice, st);
  if (!e && !stream) {
    e = cudaMemcpyAsync(dv->err_host, dv->err, 2 * sizeof(int), cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaStreamSynchronize(st);
    if (!e) {
      const int r = check_err_word(c, 0);
      if (r) return r;
    }
  }
  if (e) {
    ERR(BNN_ERR_WINDOW, "window not scored: CUDA error %d (%s); hint: check the GPU (nvidia-smi)", (int)e, cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

int bnn_verify_labels(const char *weights_path, const char *labels_path) {
  bnn_info info;
  if (probe_full(weights_path, &info, NULL)) return -1;
  if (!info.has_labels_sha) {
    ERR(BNN_ERR_LABELS, "%s carries no label hash (legacy file or package compiled without --labels)", weights_path);
    return -1;
  }
  FILE *f = fopen(labels_path, "rb");
  if (!f) { ERR(BNN_ERR_LABELS, "cannot open label file %s", labels_path); return -1; }
  unsigned char buf[65536];
  size_t n, total = 0;
  int lines = 0;
  bnn_sha256 h;
  bnn_sha256_init(&h);
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) {
    bnn_sha256_update(&h, buf, n);
    for (size_t i = 0; i < n; i++) lines += buf[i] == '\n';
    total += n;
  }
  fclose(f);
  unsigned char sum[32];
  bnn_sha256_final(&h, sum);
  if (!memcmp(sum, info.labels_sha256, 32)) return 0;
  char a[17], b[17];
  for (int i = 0; i < 8; i++) { snprintf(a + 2 * i, 3, "%02x", sum[i]); snprintf(b + 2 * i, 3, "%02x", info.labels_sha256[i]); }
  ERR(BNN_ERR_LABELS, "label file %s (sha256 %s..., %d lines, %zu bytes) is not the label file %s was compiled with "
      "(sha256 %s..., %d classes); hint: use the label file inside the package (bnn_probe_meta \"labels\", or `cli <pkg> "
      "--labels`) or recompile the package with --labels %s", labels_path, a, lines, total, weights_path, b,
      info.n_classes, labels_path);
  return -1;
}

/* ------------------------------------------------------------------ per-op profile */

int bnn_profile_begin(bnn_ctx *c) {
  if (!c || !c->dev[0]) { ERR(BNN_ERR_USAGE, "bnn_profile_begin: no context"); return -1; }
  bnn_dev *dv = c->dev[0];
  cudaSetDevice(dv->dev);
  if (!dv->events) {
    dv->events = calloc(2 * (size_t)c->n_ops, sizeof(void *));
    dv->op_ms = calloc((size_t)c->n_ops, sizeof(double));
    if (!dv->events || !dv->op_ms) { ERR(BNN_ERR_OOM, "bnn_profile_begin: out of memory"); return -1; }
    for (int k = 0; k < 2 * c->n_ops; k++)
      if (cudaEventCreate((cudaEvent_t *)&dv->events[k])) {
        ERR(BNN_ERR_CPU, "bnn_profile_begin: cudaEventCreate failed");
        return -1;
      }
  }
  memset(dv->op_ms, 0, sizeof(double) * (size_t)c->n_ops);
  dv->prof_on = 1;
  dv->prof_op0 = dv->prof_op1 = 0;
  return 0;
}

int bnn_profile_collect(bnn_ctx *c) {
  if (!c || !c->dev[0] || !c->dev[0]->prof_on) { ERR(BNN_ERR_USAGE, "bnn_profile_collect: profile not begun"); return -1; }
  bnn_dev *dv = c->dev[0];
  cudaSetDevice(dv->dev);
  for (int i = dv->prof_op0; i < dv->prof_op1; i++) {
    float ms = 0.f;
    if (cudaEventSynchronize((cudaEvent_t)dv->events[2 * i + 1]) ||
        cudaEventElapsedTime(&ms, (cudaEvent_t)dv->events[2 * i], (cudaEvent_t)dv->events[2 * i + 1])) {
      ERR(BNN_ERR_CPU, "bnn_profile_collect: event query failed for op %d", i);
      return -1;
    }
    dv->op_ms[i] += ms;
  }
  dv->prof_op0 = dv->prof_op1 = 0;
  return 0;
}

double bnn_profile_op_ms(const bnn_ctx *c, int op) {
  if (!c || !c->dev[0] || !c->dev[0]->op_ms || op < 0 || op >= c->n_ops) return -1.0;
  return c->dev[0]->op_ms[op];
}

int bnn_profile_end(bnn_ctx *c) {
  if (!c || !c->dev[0]) return -1;
  c->dev[0]->prof_on = 0;
  return 0;
}

/* ------------------------------------------------------------------ op-level debugging */

int bnn_debug_n_ops(const bnn_ctx *c) { return c ? c->n_ops : 0; }
int bnn_debug_op_code(const bnn_ctx *c, int i) { return c && i >= 0 && i < c->n_ops ? c->ops[i].code : -1; }

static int dbg_check(bnn_ctx *c, int buf, int n) {
  if (!c || n < 1 || n > c->batch || buf < 0 || (uint32_t)buf >= c->path->n_buf) {
    ERR(BNN_ERR_USAGE, "bnn_debug: buffer %d / %d windows out of range", buf, n);
    return -1;
  }
  if (!c->dev[0]->buf[buf]) {
    ERR(BNN_ERR_USAGE, "bnn_debug: buffer %d is an int8 row buffer, which this runtime keeps in its own scratch layout", buf);
    return -1;
  }
  return 0;
}

int bnn_debug_run_ops(bnn_ctx *c, int n, const float *pcm, int op0, int op1) {
  if (dbg_check(c, 0, n)) return -1;
  bnn_dev *dv = c->dev[0];
  cudaStream_t st = (cudaStream_t)dv->stream;
  cudaSetDevice(dv->dev);
  const uint32_t in = c->path->in_buf;
  if (pcm && cudaMemcpyAsync(dv->buf[in], pcm, sizeof(float) * (size_t)n * c->bufd[in].elems, cudaMemcpyHostToDevice, st)) {
    ERR(BNN_ERR_WINDOW, "bnn_debug_run_ops: input copy failed");
    return -1;
  }
  dv->w_base = 0;
  if (bnn_rt_launch(c, 0, n, dv->buf[in], op0, op1, st)) return -1;
  cudaError_t e = cudaMemcpyAsync(dv->err_host, dv->err, 2 * sizeof(int), cudaMemcpyDeviceToHost, st);
  if (!e) e = cudaStreamSynchronize(st);
  if (e) { ERR(BNN_ERR_WINDOW, "bnn_debug_run_ops: CUDA error %d (%s)", (int)e, cudaGetErrorString(e)); return -1; }
  return check_err_word(c, 0);
}

static int dbg_copy(bnn_ctx *c, int buf, int n, void *host, int to_host) {
  if (dbg_check(c, buf, n)) return -1;
  bnn_dev *dv = c->dev[0];
  const bnn_buf_rec *b = &c->bufd[buf];
  const size_t es = b->dtype == BNN_F16 ? 2 : b->dtype == BNN_I8 ? 1 : 4, row = es * b->elems;
  cudaSetDevice(dv->dev);
  cudaError_t e = to_host ? cudaMemcpy2D(host, row, dv->buf[buf], es * dv->ws[buf], row, n, cudaMemcpyDeviceToHost)
                          : cudaMemcpy2D(dv->buf[buf], es * dv->ws[buf], host, row, row, n, cudaMemcpyHostToDevice);
  if (e) { ERR(BNN_ERR_WINDOW, "bnn_debug buffer copy: CUDA error %d (%s)", (int)e, cudaGetErrorString(e)); return -1; }
  return 0;
}
int bnn_debug_get_buffer(bnn_ctx *c, int buf, int n, void *dst) { return dbg_copy(c, buf, n, dst, 1); }
int bnn_debug_set_buffer(bnn_ctx *c, int buf, int n, const void *src) { return dbg_copy(c, buf, n, (void *)src, 0); }

/* ------------------------------------------------------------------ per-op entry points */

/* per device: the error word of the per-op entry points (bnn_cuda_op_error) */
static int *g_op_err[64];
static pthread_mutex_t g_op_err_mu = PTHREAD_MUTEX_INITIALIZER;

static int *op_err_word(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) || dev < 0 || dev >= 64) return NULL;
  pthread_mutex_lock(&g_op_err_mu);
  if (!g_op_err[dev] && !cudaMalloc((void **)&g_op_err[dev], sizeof(int)) &&
      cudaMemset(g_op_err[dev], 0, sizeof(int))) {
    cudaFree(g_op_err[dev]);
    g_op_err[dev] = NULL;
  }
  int *w = g_op_err[dev];
  pthread_mutex_unlock(&g_op_err_mu);
  return w;
}

int bnn_cuda_device_init(void) {
  int e = bnnk_device_init();
  if (!e && !op_err_word()) e = cudaErrorMemoryAllocation;
  if (e) { ERR(BNN_ERR_CPU, "bnn_cuda_device_init: CUDA error %d (%s)", e, cudaGetErrorString((cudaError_t)e)); return -1; }
  return 0;
}

int bnn_cuda_op_error(void) {
  int *w = op_err_word(), v = 0;
  if (!w || cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost)) return -1;
  if (v) cudaMemset(w, 0, sizeof(int));
  return v;
}

static int launch_rc(const char *what, int e) {
  if (!e) return 0;
  ERR(BNN_ERR_WINDOW, "%s: CUDA error %d (%s)", what, e, cudaGetErrorString((cudaError_t)e));
  return -1;
}

int bnn_cuda_quant_rows(int rows, int Mw, const float *d_x, long long xws, int lda, int K, int Kq, const float *d_gate,
                        long long gws, int8_t *d_q, float *d_sa, int32_t *d_za, void *stream) {
  if (rows < 0 || Mw < 1 || K < 1 || Kq < K || Kq % 4) {
    ERR(BNN_ERR_USAGE, "bnn_cuda_quant_rows: rows %d Mw %d K %d Kq %d (need Mw >= 1, Kq >= K, Kq %% 4 == 0)", rows, Mw, K, Kq);
    return -1;
  }
  return launch_rc("bnn_cuda_quant_rows",
                   bnnk_quant(rows, Mw, d_x, xws, lda, K, Kq, d_gate, gws, d_q, d_sa, d_za, NULL, (bnn_stream_t)stream));
}

struct bnn_pw_s8 {
  bnn_devop op;
  int N, K, Kp, Np, rows_cap;
  int8_t *q;
  float *sa;
  int32_t *za;
  int *err;
};

bnn_pw_s8 *bnn_pw_s8_new(int N, int K, int Kp, int Np, const int8_t *w, const float *sw, const int32_t *cs,
                         const float *b, int rows_cap) {
  if (N <= 0 || K <= 0 || Np != ((N + 7) & ~7) || Kp != ((K + 15) & ~15) || rows_cap <= 0 || !w || !sw || !cs || !b) {
    ERR(BNN_ERR_USAGE, "bnn_pw_s8_new: N %d K %d Kp %d Np %d rows %d (expected Np = N rounded up to 8, Kp = K rounded up "
        "to 16)", N, K, Kp, Np, rows_cap);
    return NULL;
  }
  bnn_pw_s8 *o = calloc(1, sizeof *o);
  if (!o) { ERR(BNN_ERR_OOM, "out of memory"); return NULL; }
  o->N = N; o->K = K; o->Kp = Kp; o->Np = Np; o->rows_cap = rows_cap;
  char err[512];
  int kind = BNN_ERR_CPU;
  if (bnn_s8_weights(&o->op, N, K, Kp, Np, w, sw, cs, b, rows_cap, err, sizeof err, &kind)) {
    ERR(kind, "bnn_pw_s8_new: %s", err);
    bnn_pw_s8_free(o);
    return NULL;
  }
  cudaError_t e = cudaMalloc((void **)&o->q, (size_t)rows_cap * o->op.kq);
  if (!e) e = cudaMemset(o->q, 0, (size_t)rows_cap * o->op.kq);
  if (!e) e = cudaMalloc((void **)&o->sa, sizeof(float) * rows_cap);
  if (!e) e = cudaMalloc((void **)&o->za, sizeof(int32_t) * rows_cap);
  if (!e) e = cudaMalloc((void **)&o->err, sizeof(int));
  if (!e) e = cudaMemset(o->err, 0, sizeof(int));
  if (!e) e = (cudaError_t)bnnk_gemm_plan_init(&o->op.plan, o->q, rows_cap, o->op.kq, o->op.w, N, Np);
  if (e) {
    ERR(e == cudaErrorMemoryAllocation ? BNN_ERR_OOM : BNN_ERR_CPU, "bnn_pw_s8_new: CUDA error %d (%s)", (int)e,
        cudaGetErrorString(e));
    bnn_pw_s8_free(o);
    return NULL;
  }
  return o;
}

int bnn_pw_s8_run(bnn_pw_s8 *o, int B, int Mw, const float *d_x, long long xws, int lda, const float *d_gate,
                  long long gws, int act, float *d_out, long long ows, int ldo, int ow, int opad, const float *d_res,
                  long long rws, int ldr, int rw, int rpad, void *stream) {
  if (!o || B < 0 || Mw < 1 || (long long)B * Mw > o->rows_cap || lda < o->K || ldo < o->Np || act < 0 || act > 2 ||
      (opad && (ow <= 0 || Mw % ow)) || (rpad && (rw <= 0 || Mw % rw)) || (d_res && ldr < o->Np)) {
    ERR(BNN_ERR_USAGE, "bnn_pw_s8_run: B %d Mw %d lda %d ldo %d act %d ow %d opad %d (capacity %d rows)", B, Mw, lda, ldo,
        act, ow, opad, o ? o->rows_cap : 0);
    return -1;
  }
  bnn_stream_t st = (bnn_stream_t)stream;
  const int rows = B * Mw;
  bnnk_epilogue ep = {act, d_out, ows, ldo, ow, opad, d_res, rws, ldr, rw, rpad, o->op.sw, o->op.bias, o->op.cs,
                      NULL, NULL, NULL, 0, 0};
  if (!d_gate && rows > 0) {  /* one launch where the layer allows it: the quantizer inside the GEMM */
    const int f = bnnk_pw_s8_fq(&o->op.plan, rows, Mw, d_x, xws, lda, o->K, &ep, o->err, st);
    if (f != BNNK_NOT_FUSED) return launch_rc("bnn_pw_s8_run", f);
  }
  int e = bnnk_quant(rows, Mw, d_x, xws, lda, o->K, o->op.kq, d_gate, gws, o->q, o->sa, o->za, o->err, st);
  if (!e) {
    e = bnnk_gemm(&o->op.plan, rows, Mw, o->sa, o->za, &ep, o->err, st);
  }
  return launch_rc("bnn_pw_s8_run", e);
}

_Static_assert(BNN_PW_S8_STATIC_MAX_ROWS == BNNK_STATIC_ROWS && BNN_PW_S8_STATIC_MAX_QBYTES == BNNK_STATIC_QBYTES,
               "the public limits of bnn_pw_s8_run_static are the static array's");

int bnn_pw_s8_run_static(bnn_pw_s8 *o, int B, int Mw, const float *d_x, long long xws, int lda, const float *d_gate,
                         long long gws, int act, float *d_out, long long ows, int ldo, int ow, int opad,
                         const float *d_res, long long rws, int ldr, int rw, int rpad, void *stream) {
  if (!o || B < 0 || Mw < 1 || lda < o->K || ldo < o->Np || act < 0 || act > 2 || (opad && (ow <= 0 || Mw % ow)) ||
      (rpad && (rw <= 0 || Mw % rw)) || (d_res && ldr < o->Np)) {
    ERR(BNN_ERR_USAGE, "bnn_pw_s8_run_static: B %d Mw %d lda %d ldo %d act %d ow %d opad %d", B, Mw, lda, ldo, act, ow,
        opad);
    return -1;
  }
  const long long rows = (long long)B * Mw;
  if (rows > BNN_PW_S8_STATIC_MAX_ROWS || rows * o->op.kq > BNN_PW_S8_STATIC_MAX_QBYTES) {
    ERR(BNN_ERR_USAGE, "bnn_pw_s8_run_static: %lld rows of %d quantized bytes exceed the static scratch (at most %d "
        "rows and %d bytes); use bnn_pw_s8_run", rows, o->op.kq, BNN_PW_S8_STATIC_MAX_ROWS,
        BNN_PW_S8_STATIC_MAX_QBYTES);
    return -1;
  }
  bnnk_epilogue ep = {act, d_out, ows, ldo, ow, opad, d_res, rws, ldr, rw, rpad, o->op.sw, o->op.bias, o->op.cs,
                      NULL, NULL, NULL, 0, 0};
  return launch_rc("bnn_pw_s8_run_static", bnnk_pw_s8_static(&o->op.plan, (int)rows, Mw, d_x, xws, lda, o->K, d_gate,
                                                             gws, &ep, o->err, (bnn_stream_t)stream));
}

int bnn_pw_s8_gemm(bnn_pw_s8 *o, int B, int Mw, const int8_t *d_q, long long ldq, const float *d_sa,
                   const int32_t *d_za, int act, float *d_out, long long ows, int ldo, int ow, int opad,
                   const float *d_res, long long rws, int ldr, int rw, int rpad, void *stream) {
  if (!o || B < 0 || Mw < 1 || !d_q || !d_sa || !d_za || ldq < o->Kp || ldq % 16 || ((uintptr_t)d_q & 15) ||
      ldo < o->Np || act < 0 || act > 2 || (opad && (ow <= 0 || Mw % ow)) || (rpad && (rw <= 0 || Mw % rw)) ||
      (d_res && ldr < o->Np)) {
    ERR(BNN_ERR_USAGE, "bnn_pw_s8_gemm: B %d Mw %d ldq %lld (>= Kp %d, a multiple of 16, 16-byte aligned rows) ldo %d "
        "act %d ow %d opad %d", B, Mw, ldq, o ? o->Kp : 0, ldo, act, ow, opad);
    return -1;
  }
  bnnk_epilogue ep = {act, d_out, ows, ldo, ow, opad, d_res, rws, ldr, rw, rpad, o->op.sw, o->op.bias, o->op.cs,
                      NULL, NULL, NULL, 0, 0};
  return launch_rc("bnn_pw_s8_gemm", bnnk_gemm_q(&o->op.plan, d_q, ldq, o->Kp, B * Mw, Mw, d_sa, d_za, &ep, o->err,
                                                 (bnn_stream_t)stream));
}

int bnn_pw_s8_error(bnn_pw_s8 *o) {
  int v = 0;
  if (o && o->err) cudaMemcpy(&v, o->err, sizeof v, cudaMemcpyDeviceToHost);
  return v;
}

void bnn_pw_s8_free(bnn_pw_s8 *o) {
  if (!o) return;
  cudaFree(o->op.w); cudaFree(o->op.sw); cudaFree(o->op.bias); cudaFree(o->op.cs);
  cudaFree(o->q); cudaFree(o->sa); cudaFree(o->za); cudaFree(o->err);
  free(o);
}

/* ---- FE_LOGMEL (src/rt_ops_f32.c:362-385, src/pc_kern_f32.c:14-149) */

struct bnn_logmel {
  bnn_devop op;
};

bnn_logmel *bnn_logmel_new(int nsamp, int frame, int hop, int pad, int nfft, int nmel, const float *window,
                           const float *mel, float floor_, float scale) {
  /* logmel_init's and pc_logmel_new's limits */
  if (!window || !mel || nsamp <= 0 || frame <= 0 || hop <= 0 || pad < 0 || nfft < frame || nmel <= 0 ||
      (nfft & (nfft - 1)) || nfft < 16 || nfft > 2048 || nmel > 512) {
    ERR(BNN_ERR_USAGE, "bnn_logmel_new: nsamp %d frame %d hop %d pad %d nfft %d nmel %d (expected nfft a power of two "
        "in 16..2048, 0 < frame <= nfft, hop > 0, pad >= 0, 1 <= nmel <= 512)", nsamp, frame, hop, pad, nfft, nmel);
    return NULL;
  }
  bnn_logmel *o = calloc(1, sizeof *o);
  if (!o) { ERR(BNN_ERR_OOM, "out of memory"); return NULL; }
  char err[512];
  int kind = BNN_ERR_CPU;
  if (bnn_logmel_build(&o->op, nsamp, frame, hop, pad, nfft, nmel, window, mel, floor_, scale, err, sizeof err, &kind)) {
    ERR(kind, "bnn_logmel_new: %s", err);
    bnn_logmel_free(o);
    return NULL;
  }
  return o;
}

int bnn_logmel_frames(const bnn_logmel *o) { return o ? o->op.lm.nfr : -1; }

int bnn_logmel_run(bnn_logmel *o, int B, const float *d_pcm, long long pws, float *d_spec, long long sws,
                   void *stream) {
  if (!o || B < 0 || B > 65535 || !d_pcm || !d_spec || (B > 1 && (pws < o->op.lm.nsamp ||
                                                                  sws < (long long)o->op.lm.nfr * o->op.lm.nmel))) {
    ERR(BNN_ERR_USAGE, "bnn_logmel_run: B %d window strides %lld / %lld (expected 0 <= B <= 65535, strides >= nsamp "
        "and >= frames x mel bins)", B, pws, sws);
    return -1;
  }
  return launch_rc("bnn_logmel_run", bnnk_logmel(B, d_pcm, pws, &o->op.lm, d_spec, sws, (bnn_stream_t)stream));
}

void bnn_logmel_free(bnn_logmel *o) {
  if (!o) return;
  bnn_logmel_release(&o->op);
  free(o);
}

/* ---- FE_DBIMG (src/rt_ops_f32x.c:15-86, src/fe_dbimg.c:49-235) */

struct bnn_dbimg {
  bnn_devop op;
  int batch;
};

bnn_dbimg *bnn_dbimg_new(const int32_t *p, int np, const float *window, const float *mel, const int32_t *rows,
                         const float *consts, int batch) {
  if (!p || np != 21 || !window || !mel || !rows || !consts || batch < 1 || batch > 65535) {
    ERR(BNN_ERR_USAGE, "bnn_dbimg_new: expected the op record's 21 ints, its four tensors and 1 <= batch <= 65535 "
        "(np %d, batch %d)", np, batch);
    return NULL;
  }
  /* fe_db_init's checks (src/rt_ops_f32x.c:24-40) */
  const int N = p[1], nsamp = p[0], hop = p[2], pad = p[3], pm = p[4], nfr = p[5], nmel = p[6], R = p[7];
  const int ok = N >= 64 && N <= 8192 && !(N & (N - 1)) && hop > 0 && pad >= 0 && pm >= 0 && pm <= 2 && (pm || !pad) &&
                 (pm != 1 || pad < nsamp) && nfr > 0 && nsamp + 2 * pad >= N && nfr == (nsamp + 2 * pad - N) / hop + 1 &&
                 nmel > 0 && nmel <= 4096 && R > 0 && (p[8] == 0 || p[8] == 1) && p[9] >= 0 && p[9] <= 2 &&
                 p[10] >= 0 && p[10] <= 4 && p[11] >= 0 && p[11] <= 4 && p[12] >= 0 && p[12] <= 4 && p[13] == 1 &&
                 p[14] > 0 && p[15] > 0 && p[16] > 0 && p[16] <= 64 && p[19] >= p[16] && p[20] >= 0 && p[20] <= 3 &&
                 p[17] >= 0 && p[17] <= 4 && p[18] >= 0 && p[18] <= 4;
  if (!ok) {
    ERR(BNN_ERR_USAGE, "bnn_dbimg_new: parameters [%d %d %d %d %d %d %d %d ...] fail fe_db_init's checks", p[0], p[1],
        p[2], p[3], p[4], p[5], p[6], p[7]);
    return NULL;
  }
  for (int r = 0; r < R; r++)
    if (rows[r] < 0 || rows[r] >= nmel) {
      ERR(BNN_ERR_USAGE, "bnn_dbimg_new: row table entry %d = %d outside 0..%d", r, rows[r], nmel - 1);
      return NULL;
    }
  bnn_dbimg *o = calloc(1, sizeof *o);
  if (!o) { ERR(BNN_ERR_OOM, "out of memory"); return NULL; }
  o->batch = batch;
  char err[512];
  int kind = BNN_ERR_CPU;
  if (bnn_dbimg_build(&o->op, p, window, mel, rows, consts, batch, err, sizeof err, &kind)) {
    ERR(kind, "bnn_dbimg_new: %s", err);
    bnn_dbimg_free(o);
    return NULL;
  }
  return o;
}

long long bnn_dbimg_image_elems(const bnn_dbimg *o) {
  if (!o) return -1;
  const bnnk_dbimg_tables *t = &o->op.db;
  return (long long)(t->Ho + 2 * t->halo) * (t->Wo + 2 * t->halo) * t->ld;
}

int bnn_dbimg_run(bnn_dbimg *o, int B, const float *d_pcm, long long pws, float *d_img, long long iws, void *stream) {
  if (!o || B < 0 || B > o->batch || !d_pcm || !d_img ||
      (B > 1 && (pws < o->op.db.nsamp || iws < bnn_dbimg_image_elems(o)))) {
    ERR(BNN_ERR_USAGE, "bnn_dbimg_run: B %d window strides %lld / %lld (expected 0 <= B <= %d, strides >= nsamp and "
        ">= the image's floats)", B, pws, iws, o ? o->batch : 0);
    return -1;
  }
  return launch_rc("bnn_dbimg_run", bnnk_dbimg(B, d_pcm, pws, &o->op.db, o->op.db_scratch, d_img, iws,
                                               (bnn_stream_t)stream));
}

void bnn_dbimg_free(bnn_dbimg *o) {
  if (!o) return;
  bnn_dbimg_release(&o->op);
  free(o);
}

/* ---- PROTO_S8 (src/rt_ops_s8n.c:212-250) */

struct bnn_proto_s8 {
  bnn_devop op;
  int N, K, Kp, Np, nc, ppc, P, batch_cap;
  int half;  /* PROTO variant 2: fp16 cells, SDOT panels, no -127 clamp (bnn_proto_s8h_*) */
  int8_t *qa;
  float *sx;
  int *err;
};

bnn_proto_s8 *bnn_proto_s8_new(int N, int K, int Kp, int Np, const int8_t *qw, const float *sw, const uint8_t *n4,
                               const float *cls_w, const float *cls_b, int nc, int ppc, float eps, int P,
                               int batch_cap) {
  /* the checks of proto8n_init and rt_proto_geom on the record's numbers (src/rt_ops_s8n.c:220-240,
   * src/rt_ops_f32.c:525-535) */
  if (!qw || !sw || !n4 || !cls_w || !cls_b || P <= 0 || P > 65536 || P % 4 || nc <= 0 || ppc < 1 || N <= 0 ||
      N > (1 << 26) || K <= 0 || K > (1 << 17) || K % 8 || (long long)nc * ppc != N || Kp != ((K + 15) & ~15) ||
      Np != ((N + 3) & ~3) || batch_cap <= 0) {
    ERR(BNN_ERR_USAGE, "bnn_proto_s8_new: N %d K %d Kp %d Np %d P %d classes %d x %d batch %d (expected K %% 8 == 0, "
        "K <= 2^17, Kp = K rounded up to 16, Np = N rounded up to 4, N = classes x prototypes per class, P %% 4 == 0)",
        N, K, Kp, Np, P, nc, ppc, batch_cap);
    return NULL;
  }
  const int bad = bnn_proto_n4_check(qw, Kp, n4, Np / 4);
  if (bad >= 0) {
    ERR(BNN_ERR_PACKAGE, "bnn_proto_s8_new: prototype panel %d is flagged for 4 products per int16 lane, but a lane's 4 "
        "weights sum to more than 258 (the sums could wrap)", bad);
    return NULL;
  }
  bnn_proto_s8 *o = calloc(1, sizeof *o);
  if (!o) { ERR(BNN_ERR_OOM, "out of memory"); return NULL; }
  o->N = N; o->K = K; o->Kp = Kp; o->Np = Np; o->nc = nc; o->ppc = ppc; o->P = P; o->batch_cap = batch_cap;
  char err[512];
  int kind = BNN_ERR_CPU;
  if (bnn_proto_weights(&o->op, N, Kp, Np, qw, sw, cls_w, cls_b, nc, eps, err, sizeof err, &kind)) {
    ERR(kind, "bnn_proto_s8_new: %s", err);
    bnn_proto_s8_free(o);
    return NULL;
  }
  const size_t cells = (size_t)batch_cap * P;
  cudaError_t e = cudaMalloc((void **)&o->qa, cells * Kp);
  if (!e) e = cudaMemset(o->qa, 0, cells * Kp);
  if (!e) e = cudaMalloc((void **)&o->sx, sizeof(float) * cells);
  if (!e) e = cudaMalloc((void **)&o->err, sizeof(int));
  if (!e) e = cudaMemset(o->err, 0, sizeof(int));
  if (!e) e = (cudaError_t)bnnk_proto_plan_init(&o->op.pplan, o->op.w, Np, Kp, o->qa, batch_cap, P);
  if (!e && !o->op.pplan.wt)
    e = cudaMalloc((void **)&o->op.f[0], sizeof(float) * (size_t)batch_cap * o->op.pplan.nch * Np);
  if (e) {
    ERR(e == cudaErrorMemoryAllocation ? BNN_ERR_OOM : BNN_ERR_CPU, "bnn_proto_s8_new: CUDA error %d (%s)", (int)e,
        cudaGetErrorString(e));
    bnn_proto_s8_free(o);
    return NULL;
  }
  return o;
}

/* PROTO variant 2 (proto8_init, src/rt_ops_f16.c:252-271, after rt_proto_geom): K % 8 == 0, P % 8 == 0,
 * Np % 12 == 0 and Np >= N, K <= 2^17 */
bnn_proto_s8 *bnn_proto_s8h_new(int N, int K, int Np, const int8_t *qw, const float *sw, const float *cls_w,
                                const float *cls_b, int nc, int ppc, float eps, int P, int batch_cap) {
  if (!qw || !sw || !cls_w || !cls_b || P <= 0 || P > 65536 || P % 8 || nc <= 0 || ppc < 1 || N <= 0 ||
      N > (1 << 26) || K <= 0 || K > (1 << 17) || K % 8 || (long long)nc * ppc != N || Np % 12 || Np < N ||
      batch_cap <= 0) {
    ERR(BNN_ERR_USAGE, "bnn_proto_s8h_new: N %d K %d Np %d P %d classes %d x %d batch %d (expected K %% 8 == 0, "
        "K <= 2^17, Np %% 12 == 0, Np >= N = classes x prototypes per class, P %% 8 == 0)", N, K, Np, P, nc, ppc,
        batch_cap);
    return NULL;
  }
  bnn_proto_s8 *o = calloc(1, sizeof *o);
  if (!o) { ERR(BNN_ERR_OOM, "out of memory"); return NULL; }
  const int Kq = (K + 15) & ~15;
  o->N = N; o->K = K; o->Kp = Kq; o->Np = Np; o->nc = nc; o->ppc = ppc; o->P = P; o->batch_cap = batch_cap;
  o->half = 1;
  char err[512];
  int kind = BNN_ERR_CPU;
  if (bnn_proto_weights_l(&o->op, 1, N, K, Kq, Np, qw, sw, cls_w, cls_b, nc, eps, err, sizeof err, &kind)) {
    ERR(kind, "bnn_proto_s8h_new: %s", err);
    bnn_proto_s8_free(o);
    return NULL;
  }
  const size_t cells = (size_t)batch_cap * P;
  cudaError_t e = cudaMalloc((void **)&o->qa, cells * Kq);
  if (!e) e = cudaMemset(o->qa, 0, cells * Kq);
  if (!e) e = cudaMalloc((void **)&o->sx, sizeof(float) * cells);
  if (!e) e = cudaMalloc((void **)&o->err, sizeof(int));
  if (!e) e = cudaMemset(o->err, 0, sizeof(int));
  if (!e) e = (cudaError_t)bnnk_proto_plan_init(&o->op.pplan, o->op.w, Np, Kq, o->qa, batch_cap, P);
  if (!e && !o->op.pplan.wt)
    e = cudaMalloc((void **)&o->op.f[0], sizeof(float) * (size_t)batch_cap * o->op.pplan.nch * Np);
  if (e) {
    ERR(e == cudaErrorMemoryAllocation ? BNN_ERR_OOM : BNN_ERR_CPU, "bnn_proto_s8h_new: CUDA error %d (%s)", (int)e,
        cudaGetErrorString(e));
    bnn_proto_s8_free(o);
    return NULL;
  }
  return o;
}

int bnn_proto_s8h_run(bnn_proto_s8 *o, int B, const uint16_t *d_x, long long xws, int ld, float *d_logits,
                      long long lws, float *d_colmax, long long cws, int *d_status, void *stream) {
  if (!o || !o->half || B < 0 || B > o->batch_cap || !d_x || !d_logits || !d_colmax || ld < o->K || lws < o->nc ||
      cws < o->Np || (B > 1 && xws < (long long)o->P * ld)) {
    ERR(BNN_ERR_USAGE, "bnn_proto_s8h_run: not a variant-2 head, or B %d (capacity %d) ld %d logits stride %lld "
        "colmax stride %lld (expected ld >= K, strides >= classes / Np, window stride >= P ld)", B,
        o ? o->batch_cap : 0, ld, lws, cws);
    return -1;
  }
  bnn_stream_t st = (bnn_stream_t)stream;
  int e = bnnk_proto_quant_h(B, o->P, d_x, xws, ld, o->K, o->Kp, o->op.eps, o->qa, o->sx, st);
  if (!e) e = bnnk_proto_colmax(&o->op.pplan, B, o->sx, o->op.sw, d_colmax, cws, o->op.f[0], o->err, st);
  if (!e) e = bnnk_proto_logits(B, o->nc, o->ppc, d_colmax, cws, o->op.f[1], o->op.f[2], d_logits, lws, d_status, NULL, 0,
                                st);
  return launch_rc("bnn_proto_s8h_run", e);
}

int bnn_proto_s8_run(bnn_proto_s8 *o, int B, const float *d_x, long long xws, int ld, float *d_logits, long long lws,
                     float *d_colmax, long long cws, int *d_status, void *stream) {
  if (!o || o->half || B < 0 || B > o->batch_cap || !d_x || !d_logits || !d_colmax || ld < o->K || lws < o->nc ||
      cws < o->Np || (B > 1 && xws < (long long)o->P * ld)) {
    ERR(BNN_ERR_USAGE, "bnn_proto_s8_run: B %d (capacity %d) ld %d logits stride %lld colmax stride %lld (expected "
        "ld >= K, strides >= classes / Np, window stride >= P ld)", B, o ? o->batch_cap : 0, ld, lws, cws);
    return -1;
  }
  bnn_stream_t st = (bnn_stream_t)stream;
  int e = bnnk_proto_quant(B, o->P, d_x, xws, ld, o->K, o->Kp, o->op.eps, o->qa, o->sx, st);
  if (!e) e = bnnk_proto_colmax(&o->op.pplan, B, o->sx, o->op.sw, d_colmax, cws, o->op.f[0], o->err, st);
  if (!e) e = bnnk_proto_logits(B, o->nc, o->ppc, d_colmax, cws, o->op.f[1], o->op.f[2], d_logits, lws, d_status, NULL, 0,
                                st);
  return launch_rc("bnn_proto_s8_run", e);
}

int bnn_proto_s8_read_scratch(bnn_proto_s8 *o, int B, int8_t *qa, float *sx) {
  if (!o || B < 0 || B > o->batch_cap) {
    ERR(BNN_ERR_USAGE, "bnn_proto_s8_read_scratch: NULL op or B %d outside 0..%d", B, o ? o->batch_cap : 0);
    return -1;
  }
  const size_t cells = (size_t)B * o->P;
  cudaError_t e = cudaDeviceSynchronize();
  if (!e && qa) e = cudaMemcpy(qa, o->qa, cells * o->Kp, cudaMemcpyDeviceToHost);
  if (!e && sx) e = cudaMemcpy(sx, o->sx, sizeof(float) * cells, cudaMemcpyDeviceToHost);
  return launch_rc("bnn_proto_s8_read_scratch", e);
}

int bnn_proto_s8_error(bnn_proto_s8 *o) {
  int v = 0;
  if (o && o->err) cudaMemcpy(&v, o->err, sizeof v, cudaMemcpyDeviceToHost);
  return v;
}

void bnn_proto_s8_free(bnn_proto_s8 *o) {
  if (!o) return;
  cudaFree(o->op.w); cudaFree(o->op.sw);
  for (int k = 0; k < 6; k++) cudaFree(o->op.f[k]);
  cudaFree(o->qa); cudaFree(o->sx); cudaFree(o->err);
  free(o);
}

/* ------------------------------------------------------------------ PW f16 */

struct bnn_pw_f16 {
  bnn_devop op;
  int N, K, Kp, Np;
};

bnn_pw_f16 *bnn_pw_f16_new(int N, int K, int Kp, int Np, const uint16_t *panels, const float *b32,
                           const uint16_t *b16) {
  if (N <= 0 || K <= 0 || Np != ((N + 7) & ~7) || Kp < K || Kp % 8 || !panels || !b32 || !b16) {
    ERR(BNN_ERR_USAGE, "bnn_pw_f16_new: N %d K %d Kp %d Np %d (expected Np = N rounded up to 8, Kp >= K, Kp %% 8 == 0)",
        N, K, Kp, Np);
    return NULL;
  }
  bnn_pw_f16 *o = calloc(1, sizeof *o);
  if (!o) { ERR(BNN_ERR_OOM, "out of memory"); return NULL; }
  o->N = N; o->K = K; o->Kp = Kp; o->Np = Np;
  char err[512];
  int kind = BNN_ERR_CPU;
  if (bnn_hpack_weights(&o->op, 1, panels, b32, b16, Kp, Np, &o->op.f[0], err, sizeof err, &kind)) {
    ERR(kind, "bnn_pw_f16_new: %s", err);
    bnn_pw_f16_free(o);
    return NULL;
  }
  return o;
}

int bnn_pw_f16_run(bnn_pw_f16 *o, int B, int Mw, const void *d_x, long long xws, int lda, int act, void *d_out,
                   long long ows, int ldo, int ow, int opad, const void *d_res, long long rws, int ldr, void *stream) {
  if (!o || B < 0 || Mw < 1 || (long long)B * Mw >= (1ll << 31) || !d_x || !d_out || lda < o->Kp || lda % 8 ||
      xws % 8 || ldo < o->Np || ldo % 4 || ows % 4 || act < 0 || act > 2 || opad < 0 ||
      (opad && (ow <= 0 || Mw % ow)) || (d_res && (ldr < o->Np || ldr % 4 || rws % 4)) || ((uintptr_t)d_x & 15) ||
      ((uintptr_t)d_out & 7) || ((uintptr_t)d_res & 7)) {
    ERR(BNN_ERR_USAGE, "bnn_pw_f16_run: B %d Mw %d lda %d (>= Kp %d, a multiple of 8) xws %lld ldo %d (>= Np %d, a "
        "multiple of 4) act %d ow %d opad %d ldr %d, or a misaligned pointer", B, Mw, lda, o ? o->Kp : 0, xws, ldo,
        o ? o->Np : 0, act, ow, opad, ldr);
    return -1;
  }
  if (B == 0) return 0;
  return launch_rc("bnn_pw_f16_run", bnnk_gemm_f16(B * Mw, Mw, d_x, xws, lda, o->op.hwd, o->Kp, o->Np, o->op.hb,
                                                   o->op.f[0], act, d_out, ows, ldo, ow, opad, d_res, rws, ldr,
                                                   (bnn_stream_t)stream));
}

void bnn_pw_f16_free(bnn_pw_f16 *o) {
  if (!o) return;
  cudaFree(o->op.hwd);
  cudaFree(o->op.hb);
  cudaFree(o->op.f[0]);
  free(o);
}

int bnn_cuda_dw3(int B, const float *d_xp, long long xws, int H, int W, int C, int s, const float *d_w, const float *d_b,
                 float *d_out, long long ows, int Ho, int Wo, float *d_chsum, long long cws, void *stream) {
  if (B < 0 || H <= 0 || W <= 0 || C <= 0 || C % 8 || (s != 1 && s != 2) || Ho <= 0 || Wo <= 0 ||
      (Ho - 1) * s + 3 > H + 2 || (Wo - 1) * s + 3 > W + 2) {
    ERR(BNN_ERR_USAGE, "bnn_cuda_dw3: H %d W %d C %d s %d Ho %d Wo %d (C %% 8 == 0, s 1|2, taps inside the halo)", H, W, C,
        s, Ho, Wo);
    return -1;
  }
  return launch_rc("bnn_cuda_dw3", bnnk_dw3(B, d_xp, xws, H, W, C, s, d_w, d_b, d_out, ows, Ho, Wo, d_chsum, cws,
                                             op_err_word(), (bnn_stream_t)stream));
}

int bnn_cuda_dw3_f16(int B, const void *d_xp, long long xws, int H, int W, int C, int s, int pt, int pl,
                     const void *d_w, const void *d_b, void *d_out, long long ows, int Ho, int Wo, float *d_chsum,
                     long long cws, void *stream) {
  if (B < 0 || H <= 0 || W <= 0 || C <= 0 || C % 8 || C > 2048 || (s != 1 && s != 2) || pt < 0 || pt > 1 || pl < 0 ||
      pl > 1 || Ho <= 0 || Wo <= 0 || Ho > 12288 || (Ho - 1) * s - pt + 1 + 3 > H + 2 ||
      (Wo - 1) * s - pl + 1 + 3 > W + 2 || xws % 2 || ows % 2 || cws % 2 || !d_xp || !d_w || !d_b || !d_out ||
      !d_chsum) {
    ERR(BNN_ERR_USAGE, "bnn_cuda_dw3_f16: H %d W %d C %d s %d pt %d pl %d Ho %d Wo %d (C %% 8 == 0 and <= 2048, s 1|2, "
        "pt and pl 0|1, Ho <= 12288, taps inside the halo, even strides)", H, W, C, s, pt, pl, Ho, Wo);
    return -1;
  }
  return launch_rc("bnn_cuda_dw3_f16", bnnk_dw3_f16(B, d_xp, xws, H, W, C, s, pt, pl, d_w, d_b, d_out, ows, Ho, Wo,
                                                    d_chsum, cws, op_err_word(), (bnn_stream_t)stream));
}

/* DWK f16 with the checks of rt_dwk_check (src/rt_ops_f32.c:435-451) and this library's limit of 768 pixel groups
 * per output row */
int bnn_cuda_dwk_f16(int B, const void *d_xp, long long xws, int H, int W, int C, int k, int s, int pt, int pl,
                     const void *d_w, const void *d_b, int act, void *d_out, long long ows, int Ho, int Wo,
                     float *d_chsum, long long cws, void *stream) {
  const int h = (k - 1) / 2, groups = Wo / 4 + (Wo % 4 >= 2) + Wo % 2;
  if (B < 0 || H <= 0 || W <= 0 || Ho <= 0 || Wo <= 0 || C <= 0 || C % 8 || k < 1 || k > 7 || k % 2 == 0 ||
      (s != 1 && s != 2) || pt < 0 || pt > h || pl < 0 || pl > h || act < 0 || act > 1 ||
      (Ho - 1) * s - pt + k > H + h || (Wo - 1) * s - pl + k > W + h || groups > 768 || xws % 2 || ows % 2 ||
      (B > 1 && (xws < (long long)(H + 2 * h) * (W + 2 * h) * C || ows < (long long)Ho * Wo * C || cws < C)) ||
      !d_xp || !d_w || !d_b || !d_out || !d_chsum) {
    ERR(BNN_ERR_USAGE, "bnn_cuda_dwk_f16: H %d W %d C %d k %d s %d pt %d pl %d act %d Ho %d Wo %d (C %% 8 == 0, k odd "
        "1..7, s 1|2, pt and pl <= (k - 1) / 2, taps inside the halo, at most 768 pixel groups per row, even window "
        "strides of at least one window)", H, W, C, k, s, pt, pl, act, Ho, Wo);
    return -1;
  }
  return launch_rc("bnn_cuda_dwk_f16", bnnk_dwk_f16(B, d_xp, xws, W, C, k, s, pt, pl, d_w, d_b, act, d_out, ows, Ho,
                                                    Wo, d_chsum, cws, (bnn_stream_t)stream));
}

/* STEM f32 -> f16 with the checks of rt_stem_f32_check (src/rt_ops_f32.c:390-408) and this library's 48 KB limit */
int bnn_cuda_stem_f16(int B, const float *d_img, long long iws, int H, int W, int k, int s, int Ho, int Wo,
                      const float *d_w, const float *d_b, int N, int Kp, int act, void *d_out, long long ows, int ldo,
                      int opad, void *stream) {
  const int Np = (N + 7) & ~7;
  if (B < 0 || k < 1 || s < 1 || Ho <= 0 || Wo <= 0 || N <= 0 || (Ho - 1) * s + k > H || (Wo - 1) * s + k > W ||
      Kp < k * k || Kp % 4 || ldo < Np || opad < 0 || opad > 3 || act < 0 || act > 2 ||
      ((size_t)Np * Kp + Np) * 4 > 48 * 1024 ||
      (B > 1 && (iws < (long long)H * W || ows < (long long)(Ho + 2 * opad) * (Wo + 2 * opad) * ldo)) || !d_img ||
      !d_w || !d_b || !d_out) {
    ERR(BNN_ERR_USAGE, "bnn_cuda_stem_f16: H %d W %d k %d s %d Ho %d Wo %d N %d Kp %d act %d ldo %d opad %d (VALID "
        "conv, Kp >= k k and a multiple of 4, ldo >= N rounded up to 8, opad 0..3, act 0..2, weights within 48 KB, "
        "window strides of at least one window)", H, W, k, s, Ho, Wo, N, Kp, act, ldo, opad);
    return -1;
  }
  return launch_rc("bnn_cuda_stem_f16", bnnk_stem_f16(B, d_img, iws, W, k, s, Ho, Wo, d_w, d_b, N, Kp, Np, act, d_out,
                                                      ows, ldo, opad, (bnn_stream_t)stream));
}

int bnn_cuda_peak_hfma2(int blocks, int iters, void *d_word, void *stream) {
  if (blocks <= 0 || iters <= 0 || !d_word) {
    ERR(BNN_ERR_USAGE, "bnn_cuda_peak_hfma2: blocks %d iters %d word %p", blocks, iters, d_word);
    return -1;
  }
  return launch_rc("bnn_cuda_peak_hfma2", bnnk_peak_hfma2(blocks, iters, d_word, (bnn_stream_t)stream));
}

int bnn_cuda_fn(int fn, int n, const float *d_x, float *d_y, void *stream) {
  if (fn < 0 || fn > 9 || n < 0) { ERR(BNN_ERR_USAGE, "bnn_cuda_fn: fn %d n %d", fn, n); return -1; }
  return launch_rc("bnn_cuda_fn", bnnk_test_fn(fn, n, d_x, d_y, (bnn_stream_t)stream));
}
