// FE_DBIMG, the dB-image front end of compiled models (BirdNET v3.0), on sm_100a: src/fe_dbimg.c (fe_db_frames
// :142-226, fe_db_image :229-258) batched over windows in three kernels.
//
//   k_dbimg_frames: one CTA per (group of FG frames, window). The frames' samples (reflect or zero padding outside the
//     window) times the window go into shared memory in bit-reversed order as NC = N / 2 complex points; the radix-2
//     DIT runs stage by stage with the reference's butterfly (b w = (fms(bi, wi, br wr), fma(br, wi, bi wr)), the
//     wr products rounded first); the real split and the power per bin; the sparse mel with one fused accumulator in
//     entry order; Clip(floor), the natural logarithm, up to three scalar ops -> dB rows [nmel][nfr] in a scratch;
//     and the block's maximum (fmaxf: NaN ignored) for the top-db floor.
//   k_dbimg_rows: one CTA per window. The top-db floor from the blocks' maxima, the selected rows (fmaxf against it)
//     into a second scratch, their minimum and maximum, then the min/max normalisation in place (IEEE divisions).
//   k_dbimg_image: a thread per image pixel (halo included): the half-pixel bilinear resize in the reference's
//     product and sum order, the two per-channel ops, zero pad channels and a zero halo.
//
// The logarithm: the reference calls libm logf; here the double-precision log rounded once to float (correctly
// rounded). glibc's logf differs from the correctly rounded result on 416,909 of the 2^31 - 2^23 positive finite
// floats, by one unit in the last place, so images agree with the reference within that tolerance; with a
// correctly rounded logarithm in the oracle they agree bit for bit. All other arithmetic is the reference's.
#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "bnn_kernels.h"
#include "ln_cr.cuh"

namespace bnn {

__device__ __forceinline__ float post_op(float v, int code, float c) {
  switch (code) {
  case 1: return __fmul_rn(v, c);
  case 2: return __fdiv_rn(v, c);
  case 3: return __fadd_rn(v, c);
  case 4: return __fsub_rn(v, c);
  default: return v;
  }
}

// C fmaxf / fminf: a NaN operand yields the other operand
__device__ __forceinline__ float fmax_c(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ float fmin_c(float a, float b) { return fminf(a, b); }

__device__ __forceinline__ int src_index(int i, int n, int mode) {
  if (i >= 0 && i < n) return i;
  if (mode != 1) return -1;
  if (i < 0) i = -i;
  if (i >= n) i = 2 * n - 2 - i;
  return i >= 0 && i < n ? i : -1;
}

constexpr int kDbThreads = 256;

template <int FG>
__global__ void __launch_bounds__(kDbThreads) k_dbimg_frames(const bnnk_dbimg_tables t, const float *__restrict__ pcm,
                                                            long long pws, float *__restrict__ db,
                                                            float *__restrict__ pmax) {
  extern __shared__ float sm[];  // re [FG][NC], im [FG][NC], pw [FG][NC + 1]
  __shared__ float red[kDbThreads / 32];
  const int NC = t.nfft >> 1, lg = t.lg, tid = threadIdx.x;
  float *re = sm, *im = sm + FG * NC, *pw = sm + 2 * FG * NC;
  const int w = blockIdx.y, t0 = blockIdx.x * FG, nblk = gridDim.x;
  const float *x = pcm + w * pws;
  // samples x window, bit-reversed
  for (int idx = tid; idx < FG * NC; idx += kDbThreads) {
    const int f = idx >> lg, n = idx & (NC - 1);
    const int tf = t0 + f < t.nfr ? t0 + f : t.nfr - 1;
    const int base = tf * t.hop - t.pad;
    const int i0 = src_index(base + 2 * n, t.nsamp, t.padmode), i1 = src_index(base + 2 * n + 1, t.nsamp, t.padmode);
    const int r = (int)(__brev((unsigned)n) >> (32 - lg));
    re[f * NC + r] = __fmul_rn(i0 < 0 ? 0.f : __ldg(x + i0), __ldg(t.win + 2 * n));
    im[f * NC + r] = __fmul_rn(i1 < 0 ? 0.f : __ldg(x + i1), __ldg(t.win + 2 * n + 1));
  }
  __syncthreads();
  // radix-2 DIT (fft4, src/fe_dbimg.c:117-133)
  for (int len = 2, tws = NC / 2, lh = 0; len <= NC; len <<= 1, tws >>= 1, lh++) {
    const int h = len >> 1;
    for (int idx = tid; idx < FG * (NC >> 1); idx += kDbThreads) {
      const int f = idx >> (lg - 1), bidx = idx & ((NC >> 1) - 1);
      const int k = bidx & (h - 1), i = (bidx >> lh) << (lh + 1);
      const float wr = __ldg(t.tw_re + k * tws), wi = __ldg(t.tw_im + k * tws);
      float *pr = re + f * NC + i + k, *pi = im + f * NC + i + k;
      const float br = pr[h], bi = pi[h];
      const float vr = __fmaf_rn(-bi, wi, __fmul_rn(br, wr)), vi = __fmaf_rn(br, wi, __fmul_rn(bi, wr));
      const float ur = pr[0], ui = pi[0];
      pr[0] = __fadd_rn(ur, vr); pi[0] = __fadd_rn(ui, vi);
      pr[h] = __fsub_rn(ur, vr); pi[h] = __fsub_rn(ui, vi);
    }
    __syncthreads();
  }
  // real split and power (src/fe_dbimg.c:195-204)
  const int nk = t.khi - t.klo;
  for (int idx = tid; idx < FG * nk; idx += kDbThreads) {
    const int f = idx / nk, k = t.klo + (idx - f * nk);
    const int k1 = k & (NC - 1), k2 = (NC - k) & (NC - 1);
    const float zr = re[f * NC + k1], zi = im[f * NC + k1], cr = re[f * NC + k2], ci = -im[f * NC + k2];
    const float er = __fmul_rn(__fadd_rn(zr, cr), 0.5f), ei = __fmul_rn(__fadd_rn(zi, ci), 0.5f);
    const float dr = __fsub_rn(zr, cr), di = __fsub_rn(zi, ci);
    const float or_ = __fmul_rn(di, 0.5f), oi = __fmul_rn(dr, -0.5f);
    const float wr = __ldg(t.sp_re + k), wi = __ldg(t.sp_im + k);
    const float xr = __fadd_rn(er, __fmaf_rn(-oi, wi, __fmul_rn(or_, wr)));
    const float xi = __fadd_rn(ei, __fmaf_rn(or_, wi, __fmul_rn(oi, wr)));
    pw[f * (NC + 1) + k] = __fadd_rn(__fmul_rn(xr, xr), __fmul_rn(xi, xi));
  }
  __syncthreads();
  // sparse mel, Clip, ln, scalar ops; frames fastest so that a row's frames are stored together
  float mx = -FLT_MAX;
  for (int idx = tid; idx < FG * t.nmel; idx += kDbThreads) {
    const int j = idx / FG, f = idx - j * FG;
    if (t0 + f >= t.nfr) continue;
    float acc = 0.f;
    const int e1 = __ldg(t.mel_off + j + 1);
    for (int e = __ldg(t.mel_off + j); e < e1; e++)
      acc = __fmaf_rn(pw[f * (NC + 1) + __ldg(t.mel_k + e)], __ldg(t.mel_w + e), acc);
    const float xv = acc < t.floor_ ? t.floor_ : acc;
    float y = ln_cr(xv);
    y = post_op(y, t.post[0], t.postv[0]);
    y = post_op(y, t.post[1], t.postv[1]);
    y = post_op(y, t.post[2], t.postv[2]);
    db[((long long)w * t.nmel + j) * t.nfr + t0 + f] = y;
    mx = fmax_c(mx, y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmax_c(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    for (int i = 1; i < kDbThreads / 32; i++) m = fmax_c(m, red[i]);
    pmax[(long long)w * nblk + blockIdx.x] = m;
  }
}

constexpr int kRowThreads = 1024;

__global__ void __launch_bounds__(kRowThreads) k_dbimg_rows(const bnnk_dbimg_tables t, const float *__restrict__ db,
                                                           const float *__restrict__ pmax, int nblk,
                                                           float *__restrict__ sp) {
  __shared__ float r0[kRowThreads / 32], r1[kRowThreads / 32];
  __shared__ float s_fl, s_mn, s_mx;
  const int w = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const float *dbw = db + (long long)w * t.nmel * t.nfr;
  float *spw = sp + (long long)w * t.R * t.nfr;
  if (t.has_top_db) {
    float m = -FLT_MAX;
    for (int i = tid; i < nblk; i += kRowThreads) m = fmax_c(m, pmax[(long long)w * nblk + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax_c(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) r0[wp] = m;
    __syncthreads();
    if (tid == 0) {
      float mm = r0[0];
      for (int i = 1; i < kRowThreads / 32; i++) mm = fmax_c(mm, r0[i]);
      s_fl = __fsub_rn(mm, t.top_db);
    }
    __syncthreads();
  }
  const float fl = t.has_top_db ? s_fl : -FLT_MAX;
  float mn = FLT_MAX, mx = -FLT_MAX;
  const int n = t.R * t.nfr;
  for (int i = tid; i < n; i += kRowThreads) {
    const int r = i / t.nfr, tt = i - r * t.nfr;
    const float s = dbw[(long long)__ldg(t.rows + r) * t.nfr + tt];
    const float v = t.has_top_db ? fmax_c(s, fl) : s;
    spw[i] = v;
    mn = fmin_c(mn, v);
    mx = fmax_c(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fmin_c(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmax_c(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) { r0[wp] = mn; r1[wp] = mx; }
  __syncthreads();
  if (tid == 0) {
    float a = r0[0], b = r1[0];
    for (int i = 1; i < kRowThreads / 32; i++) { a = fmin_c(a, r0[i]); b = fmax_c(b, r1[i]); }
    s_mn = a;
    s_mx = b;
  }
  __syncthreads();
  if (t.norm) {
    const float lo = s_mn, hi = s_mx, den = __fadd_rn(__fsub_rn(hi, lo), t.eps);
    for (int i = tid; i < n; i += kRowThreads)
      spw[i] = t.norm == 2 ? __fdiv_rn(__fsub_rn(hi, spw[i]), den) : __fdiv_rn(__fsub_rn(spw[i], lo), den);
  }
}

__global__ void __launch_bounds__(256) k_dbimg_image(const bnnk_dbimg_tables t, const float *__restrict__ sp,
                                                     float *__restrict__ img, long long iws) {
  const int h = t.halo, Wp = t.Wo + 2 * h, Hp = t.Ho + 2 * h;
  const int pix = blockIdx.x * blockDim.x + threadIdx.x, w = blockIdx.y;
  if (pix >= Hp * Wp) return;
  const int py = pix / Wp, px = pix - py * Wp, oy = py - h, ox = px - h;
  float *o = img + w * iws + (long long)pix * t.ld;
  if (oy < 0 || oy >= t.Ho || ox < 0 || ox >= t.Wo) {
    for (int c = 0; c < t.ld; c++) o[c] = 0.f;
    return;
  }
  const float *spw = sp + (long long)w * t.R * t.nfr;
  const float *r1 = spw + (long long)__ldg(t.ry1 + oy) * t.nfr, *r2 = spw + (long long)__ldg(t.ry2 + oy) * t.nfr;
  const float dy1 = __ldg(t.dy1 + oy), dy2 = __ldg(t.dy2 + oy);
  const int x1 = __ldg(t.rx1 + ox), x2 = __ldg(t.rx2 + ox);
  const float dx1 = __ldg(t.dx1 + ox), dx2 = __ldg(t.dx2 + ox);
  float v = __fmul_rn(__fmul_rn(dx2, dy2), r1[x1]);
  v = __fadd_rn(v, __fmul_rn(__fmul_rn(dx1, dy2), r1[x2]));
  v = __fadd_rn(v, __fmul_rn(__fmul_rn(dx2, dy1), r2[x1]));
  v = __fadd_rn(v, __fmul_rn(__fmul_rn(dx1, dy1), r2[x2]));
  for (int c = 0; c < t.C; c++)
    o[c] = post_op(post_op(v, t.chan[0], __ldg(t.chv + c)), t.chan[1], __ldg(t.chv + t.C + c));
  for (int c = t.C; c < t.ld; c++) o[c] = 0.f;
}

}  // namespace bnn

using namespace bnn;

// frames per CTA: FG x NC complex points in shared memory, at least 2048 of them where NC allows
static int dbimg_fg(int NC) { return NC >= 2048 ? 1 : NC >= 1024 ? 2 : NC >= 512 ? 4 : 8; }

extern "C" size_t bnnk_dbimg_scratch_floats(const bnnk_dbimg_tables *t, int B) {
  const int nblk = (t->nfr + dbimg_fg(t->nfft / 2) - 1) / dbimg_fg(t->nfft / 2);
  return (size_t)B * ((size_t)t->nmel * t->nfr + (size_t)t->R * t->nfr + (size_t)nblk);
}

extern "C" int bnnk_dbimg(int B, const float *pcm, long long pws, const bnnk_dbimg_tables *t, float *scratch,
                          float *img, long long iws, bnn_stream_t st) {
  if (B <= 0) return 0;
  const int NC = t->nfft / 2, fg = dbimg_fg(NC), nblk = (t->nfr + fg - 1) / fg;
  float *db = scratch, *sp = db + (size_t)B * t->nmel * t->nfr, *pmax = sp + (size_t)B * t->R * t->nfr;
  const size_t smem = sizeof(float) * (size_t)fg * (3 * NC + 1);
  const dim3 g1((unsigned)nblk, (unsigned)B);
#define BNN_DBF(FG)                                                                                           \
  do {                                                                                                       \
    cudaError_t e_ = cudaFuncSetAttribute(k_dbimg_frames<FG>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                          (int)smem);                                                        \
    if (e_) return e_;                                                                                       \
    k_dbimg_frames<FG><<<g1, kDbThreads, smem, st>>>(*t, pcm, pws, db, pmax);                               \
  } while (0)
  switch (fg) {
  case 1: BNN_DBF(1); break;
  case 2: BNN_DBF(2); break;
  case 4: BNN_DBF(4); break;
  default: BNN_DBF(8); break;
  }
#undef BNN_DBF
  k_dbimg_rows<<<B, kRowThreads, 0, st>>>(*t, db, pmax, nblk, sp);
  const int npix = (t->Ho + 2 * t->halo) * (t->Wo + 2 * t->halo);
  k_dbimg_image<<<dim3((unsigned)((npix + 255) / 256), (unsigned)B), 256, 0, st>>>(*t, sp, img, iws);
  return cudaGetLastError();
}
