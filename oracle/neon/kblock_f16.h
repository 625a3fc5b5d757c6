/* Scalar restatement of the reference's fp16 GEMM K-blocks (src/gemm_f16_kblock.h: kblock_8x16, kblock0_8x16,
 * kblock_8x8, kblock0_8x8, AArch64 inline assembly) for the x86 reference build of the parity oracle (TEST
 * INFRASTRUCTURE ONLY; oracle/ref.mk force-includes this file and defines GEMM_F16_KBLOCK_H so that the assembly
 * header is skipped).
 *
 * What the assembly computes (read from src/gemm_f16_kblock.h:4-592): 8 rows p0..p7 of fp16 activations x 16 (or 8)
 * channels; accumulators acc[r][c] in fp16, loaded from cb [8][16] (or [8][8]) or started at +0 (the kblock0 forms);
 * n8 steps of 8 k; at each k one FMLA by element (fp16, fused, one rounding) per accumulator:
 * acc = fma(w[k][c], p_r[k], acc), k ascending, 16 (or 8) weights per k, consecutive; the result is stored to cb. */
#ifndef BNN_ORACLE_KBLOCK_F16_H
#define BNN_ORACLE_KBLOCK_F16_H
#include "arm_neon.h"

static inline __attribute__((unused)) void nv_kblock_f16(const _Float16 *const p[8], const _Float16 *w, long n8,
                                                         _Float16 *cb, int nc, int zero) {
  _Float16 acc[8][16];
  for (int r = 0; r < 8; r++)
    for (int c = 0; c < nc; c++) acc[r][c] = zero ? (_Float16)0.f : cb[r * nc + c];
  for (long k = 0; k < 8 * n8; k++, w += nc)
    for (int r = 0; r < 8; r++)
      for (int c = 0; c < nc; c++) acc[r][c] = nv_h_fma(w[c], p[r][k], acc[r][c]);
  for (int r = 0; r < 8; r++)
    for (int c = 0; c < nc; c++) cb[r * nc + c] = acc[r][c];
}

#define NV_KBLOCK_F16(name, nc, zero)                                                                              \
  static inline __attribute__((unused)) void name(const _Float16 *p0, const _Float16 *p1, const _Float16 *p2,     \
                                                  const _Float16 *p3, const _Float16 *p4, const _Float16 *p5,     \
                                                  const _Float16 *p6, const _Float16 *p7, const _Float16 *w,      \
                                                  long n8, _Float16 *cb) {                                        \
    const _Float16 *const p[8] = {p0, p1, p2, p3, p4, p5, p6, p7};                                               \
    nv_kblock_f16(p, w, n8, cb, nc, zero);                                                                        \
  }
NV_KBLOCK_F16(kblock_8x16, 16, 0)
NV_KBLOCK_F16(kblock0_8x16, 16, 1)
NV_KBLOCK_F16(kblock_8x8, 8, 0)
NV_KBLOCK_F16(kblock0_8x8, 8, 1)
#undef NV_KBLOCK_F16
#endif
