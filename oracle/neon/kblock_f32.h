/* Scalar restatement of the reference's fp32 GEMM K-block (src/gemm_f32_kblock.h: KB8X8F / KB8X8F_PF, AArch64 inline
 * assembly) for the x86 reference build of the parity oracle (TEST INFRASTRUCTURE ONLY; oracle/ref.mk force-includes
 * this file and defines GEMM_F32_KBLOCK_H so that the assembly header is skipped).
 *
 * What the assembly computes (read from src/gemm_f32_kblock.h:5-136):
 *   - 8 rows at A + r * LDA bytes (r < 8) x 8 channels; the accumulators A(2r) (channels 0-3 of row r) and A(2r+1)
 *     (channels 4-7) start at +0;
 *   - NSEG segments of N4 steps of 4 k; at each k one FMLA by element per accumulator: acc = fma(w[c], a[r][k], acc),
 *     k ascending, weights 8 floats per k, consecutive across segments;
 *   - the row pointer advances (N4 + 1) * 16 + SKIP bytes per segment (its post-incremented loads run one vector
 *     ahead), the weight pointer N4 * 128 bytes per segment; both are outputs of the block.
 * KB8X8F_PF only adds prefetches, which change no result. */
#ifndef BNN_ORACLE_KBLOCK_F32_H
#define BNN_ORACLE_KBLOCK_F32_H
#include "arm_neon.h"

static inline __attribute__((unused)) void nv_kb8x8f(const char **pa, long lda, const float **pw, long n4, long nseg,
                                                     long skip, float32x4_t acc[16]) {
  const char *a = *pa;
  const float *w = *pw;
  for (int i = 0; i < 16; i++) acc[i] = vdupq_n_f32(0.f);
  for (long s = 0; s < nseg; s++) {
    for (long j = 0; j < 4 * n4; j++, w += 8) {
      for (int r = 0; r < 8; r++) {
        float x;
        memcpy(&x, a + r * lda + 4 * j, 4);
        for (int c = 0; c < 4; c++) {
          acc[2 * r][c] = fmaf(w[c], x, acc[2 * r][c]);
          acc[2 * r + 1][c] = fmaf(w[4 + c], x, acc[2 * r + 1][c]);
        }
      }
    }
    a += (n4 + 1) * 16 + skip;
  }
  *pa = a;
  *pw = w;
}

#define KB8X8F(A, LDA, W, N4, NSEG, SKIP, A0, A1, A2, A3, A4, A5, A6, A7, A8, A9, A10, A11, A12, A13, A14, A15) \
  do {                                                                                                          \
    float32x4_t nv_acc_[16];                                                                                    \
    const char *nv_a_ = (const char *)(A);                                                                      \
    const float *nv_w_ = (const float *)(W);                                                                    \
    nv_kb8x8f(&nv_a_, (long)(LDA), &nv_w_, (long)(N4), (long)(NSEG), (long)(SKIP), nv_acc_);                    \
    (A) = (__typeof__(A))(const void *)nv_a_;                                                                   \
    (W) = (__typeof__(W))(const void *)nv_w_;                                                                   \
    A0 = nv_acc_[0]; A1 = nv_acc_[1]; A2 = nv_acc_[2]; A3 = nv_acc_[3];                                         \
    A4 = nv_acc_[4]; A5 = nv_acc_[5]; A6 = nv_acc_[6]; A7 = nv_acc_[7];                                         \
    A8 = nv_acc_[8]; A9 = nv_acc_[9]; A10 = nv_acc_[10]; A11 = nv_acc_[11];                                     \
    A12 = nv_acc_[12]; A13 = nv_acc_[13]; A14 = nv_acc_[14]; A15 = nv_acc_[15];                                 \
  } while (0)
#define KB8X8F_PF(A, LDA, W, N4, NSEG, SKIP, A0, A1, A2, A3, A4, A5, A6, A7, A8, A9, A10, A11, A12, A13, A14, A15, \
                  PFD)                                                                                          \
  KB8X8F(A, LDA, W, N4, NSEG, SKIP, A0, A1, A2, A3, A4, A5, A6, A7, A8, A9, A10, A11, A12, A13, A14, A15)
#endif
