/* .bnpk reader: mmap, header / table bounds checks, metadata records.
 *
 * Follows the checks and the error contract of the reference loader (src/rt_pkg.c:30-166): the same limits, the
 * same order of checks and messages of the form "<what>: <expected> vs <found>; hint: <what to do>", so a host that
 * surfaces bnn_last_error shows the same diagnosis for a bad file. */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "bnn_internal.h"

#define FAIL(...)                          \
  do {                                     \
    snprintf(err, errlen, __VA_ARGS__);    \
    bnn_pkg_close(p);                      \
    return NULL;                           \
  } while (0)

bnn_pkg *bnn_pkg_open(const char *path, char *err, size_t errlen) {
  bnn_pkg *p = calloc(1, sizeof *p);
  if (!p) { snprintf(err, errlen, "out of memory"); return NULL; }
  int fd = open(path, O_RDONLY);
  if (fd < 0) FAIL("cannot open %s (%s)", path, strerror(errno));
  struct stat sb;
  const int no_stat = fstat(fd, &sb) != 0;
  if (no_stat || sb.st_size < 64) {
    close(fd);
    FAIL("%s: %lld bytes, smaller than a package header (64); hint: incomplete download or the wrong file", path,
         no_stat ? -1LL : (long long)sb.st_size);
  }
  p->size = (size_t)sb.st_size;
  void *m = mmap(NULL, p->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED)
    FAIL("%s: mmap of %zu bytes failed (%s); hint: memory or a filesystem that cannot map files", path, p->size,
         strerror(errno));
  p->map = m;
  const uint8_t *b = p->map;
  if (memcmp(b, "BNNPKG01", 8))
    FAIL("%s: not a .bnpk package (magic '%.8s', expected BNNPKG01); hint: the file is not a compiled model package: "
         "compile the model with compiler/bnc.py, or check the download (sha256)", path, (const char *)b);
  uint32_t bom;
  uint16_t ver[2];
  memcpy(&bom, b + 8, 4);
  memcpy(ver, b + 12, 4);
  if (bom != 0x01020304u) FAIL("%s: byte-order mark 0x%08x, expected 0x01020304 (little endian); hint: corrupt file", path, bom);
  p->version = ver[0];
  if (ver[1] > 1)
    FAIL("%s: the package needs reader version %u, this library reads format version 1; hint: update libbnneon, or "
         "recompile the model with the compiler that matches this library", path, ver[1]);
  uint32_t cnt[4];
  uint64_t off[4];
  memcpy(cnt, b + 16, 16);
  memcpy(off, b + 32, 32);
  p->n_meta = cnt[0];
  p->n_tensors = cnt[1];
  p->n_paths = cnt[2];
  if (off[3] != p->size)
    FAIL("%s: package truncated (size %zu, header says %llu); hint: incomplete download or copy; compare the sha256",
         path, p->size, (unsigned long long)off[3]);
  if (p->n_tensors > 65536 || p->n_paths < 1 || p->n_paths > 8 || p->n_meta > 4096)
    FAIL("%s: corrupt header (%u metadata records, %u tensors, %u paths; limits 4096 / 65536 / 1..8); hint: corrupt "
         "file or not a package", path, p->n_meta, p->n_tensors, p->n_paths);
  if (off[0] > p->size || off[1] > p->size || off[2] > p->size || off[1] < off[0] ||
      off[1] + (uint64_t)p->n_tensors * sizeof(bnn_tensor_rec) > p->size ||
      off[2] + (uint64_t)p->n_paths * sizeof(bnn_path_rec) > p->size)
    FAIL("%s: table offsets outside the file (meta %llu, tensors %llu, paths %llu, size %zu); hint: corrupt file", path,
         (unsigned long long)off[0], (unsigned long long)off[1], (unsigned long long)off[2], p->size);
  p->meta = b + off[0];
  p->meta_bytes = off[1] - off[0];
  p->tensors = malloc(sizeof(bnn_tensor_rec) * (p->n_tensors ? p->n_tensors : 1));
  p->paths = malloc(sizeof(bnn_path_rec) * p->n_paths);
  if (!p->tensors || !p->paths) FAIL("out of memory");
  memcpy(p->tensors, b + off[1], sizeof(bnn_tensor_rec) * p->n_tensors);
  memcpy(p->paths, b + off[2], sizeof(bnn_path_rec) * p->n_paths);
  for (uint32_t i = 0; i < p->n_tensors; i++) {
    const bnn_tensor_rec *t = &p->tensors[i];
    if (t->offset % 64 || t->offset > p->size || t->nbytes > p->size - t->offset || t->offset + t->nbytes + 64 > p->size)
      FAIL("%s: tensor %u (%.48s) lies outside the file (offset %llu, %llu bytes, file %zu); hint: truncated or corrupt "
           "file", path, i, t->name, (unsigned long long)t->offset, (unsigned long long)t->nbytes, p->size);
  }
  for (uint32_t i = 0; i < p->n_paths; i++) {
    const bnn_path_rec *d = &p->paths[i];
    if (d->n_buf == 0 || d->n_buf > 4096 || d->n_ops == 0 || d->n_ops > 4096 || d->buf_off % 8 || d->ops_off % 8 ||
        d->buf_off + (uint64_t)d->n_buf * sizeof(bnn_buf_rec) > p->size || d->ops_off + d->ops_bytes > p->size ||
        d->in_buf >= d->n_buf || d->out_buf >= d->n_buf || (d->emb_buf != 0xffffffffu && d->emb_buf >= d->n_buf))
      FAIL("%s: path %u (%.24s) has corrupt tables (%u buffers, %u ops, in %u out %u emb %u); hint: corrupt file", path,
           i, d->name, d->n_buf, d->n_ops, d->in_buf, d->out_buf, d->emb_buf);
  }
  return p;
}

void bnn_pkg_close(bnn_pkg *p) {
  if (!p) return;
  if (p->map) munmap(p->map, p->size);
  free(p->tensors);
  free(p->paths);
  free(p);
}

/* metadata record: u16 key_len, u16 type (0 str, 1 i64, 2 f64, 3 bytes), u32 val_len, key, value, pad to 8 */
const uint8_t *bnn_meta_raw(const bnn_pkg *p, const char *key, uint16_t *type, uint32_t *len) {
  const uint8_t *q = p->meta, *end = p->meta + p->meta_bytes;
  const size_t kl = strlen(key);
  for (uint32_t i = 0; i < p->n_meta && q + 8 <= end; i++) {
    uint16_t h[2];
    uint32_t vl;
    memcpy(h, q, 4);
    memcpy(&vl, q + 4, 4);
    const size_t rec = (8 + (size_t)h[0] + vl + 7) & ~(size_t)7;
    if ((size_t)(end - q) < rec) return NULL;
    if (h[0] == kl && !memcmp(q + 8, key, kl)) {
      *type = h[1];
      *len = vl;
      return q + 8 + h[0];
    }
    q += rec;
  }
  return NULL;
}

int bnn_meta_str(const bnn_pkg *p, const char *key, char *buf, size_t n) {
  uint16_t ty;
  uint32_t vl;
  const uint8_t *v = bnn_meta_raw(p, key, &ty, &vl);
  if (!v) return -1;
  char tmp[64];
  if (ty == 1 || ty == 2) { /* numbers as decimal text */
    if (ty == 1) {
      int64_t x;
      memcpy(&x, v, 8);
      snprintf(tmp, sizeof tmp, "%lld", (long long)x);
    } else {
      double x;
      memcpy(&x, v, 8);
      snprintf(tmp, sizeof tmp, "%.17g", x);
    }
    v = (const uint8_t *)tmp;
    vl = (uint32_t)strlen(tmp);
  }
  if (buf && n) {
    const size_t k = vl < n - 1 ? vl : n - 1;
    memcpy(buf, v, k);
    buf[k] = 0;
  }
  return (int)vl;
}

static int meta_num(const bnn_pkg *p, const char *key, uint16_t type, void *x) {
  uint16_t ty;
  uint32_t vl;
  const uint8_t *v = bnn_meta_raw(p, key, &ty, &vl);
  if (!v || ty != type || vl != 8) return -1;
  memcpy(x, v, 8);
  return 0;
}
int bnn_meta_i64(const bnn_pkg *p, const char *key, int64_t *v) { return meta_num(p, key, 1, v); }
int bnn_meta_f64(const bnn_pkg *p, const char *key, double *v) { return meta_num(p, key, 2, v); }

const char *bnn_dtype_name(uint32_t dt) {
  static const char *nm[] = {"f32", "f16", "i8", "i32"};
  return dt < 4 ? nm[dt] : "?";
}
