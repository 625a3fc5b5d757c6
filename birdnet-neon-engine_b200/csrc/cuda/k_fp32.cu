// The fp32 ops of the v2.4 int8 package on CUDA cores: depthwise 3x3 + SiLU + channel sums (DW3), the SE gate
// (SE_GATE), the c0 conv + pool (C0POOL), the post BN + pc conv + mean (POSTPC) and the two-spectrogram front end
// (FE_STFT2). Each output is computed with the reference's operations in the reference's order (fused where the
// NEON code fuses, rounded where it rounds), so the values are bit-identical; the parallel schedule is free because
// no reference reduction is split across threads except where its order is restated exactly.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bnn_kernels.h"
#include "emu.cuh"

namespace bnn {

// ------------------------------------------------------------------ DW3 (src/gemm_f32.c:214-440)

// One CTA per (window, slab of SC channels): threads compute TP-pixel tiles of outputs in raster order, then SC
// threads add the tile's values into their channel sums pixel by pixel (the reference's sequential order).
template <int SC>
__global__ void __launch_bounds__(256) k_dw3(const float *__restrict__ xp, long long xws, int W, int C, int s,
                                             const float *__restrict__ wt, const float *__restrict__ bias,
                                             float *__restrict__ out, long long ows, int Ho, int Wo,
                                             float *__restrict__ chsum, long long cws) {
  constexpr int PPT = 256 / SC;  // pixels per pass
  constexpr int TP = PPT * 8;    // pixels per tile
  __shared__ float tile[TP][SC];
  __shared__ uint32_t lut[256];
  const int tid = threadIdx.x, c_l = tid % SC, pp = tid / SC;
  const int c = blockIdx.x * SC + c_l, win = blockIdx.y;
  const bool act = pp < PPT;
  for (int i = tid; i < 256; i += 256) lut[i] = g_frecpe_lut[i];
  const int Wp = W + 2;
  const float *x = xp + win * xws;
  float *o = out + win * ows;
  float wv[9], b = 0.f;
  if (act) {
#pragma unroll
    for (int t = 0; t < 9; t++) wv[t] = wt[t * C + c];
    b = bias[c];
  }
  float cs = 0.f;
  const int P = Ho * Wo;
  __syncthreads();
  for (int p0 = 0; p0 < P; p0 += TP) {
    if (act) {
#pragma unroll 2
      for (int i = 0; i < 8; i++) {
        const int p = p0 + pp + i * PPT;
        if (p < P) {
          const int oy = p / Wo, ox = p - oy * Wo;
          const float *q = x + ((long long)(oy * s) * Wp + (long long)ox * s) * C + c;
#define X_(ky, kx) q[((long long)(ky) * Wp + (kx)) * C]
          float acc = __fmaf_rn(wv[0], X_(0, 0), b);
          float acb = __fmul_rn(wv[1], X_(0, 1));
          float acd = __fmul_rn(wv[2], X_(0, 2));
          acc = __fmaf_rn(wv[3], X_(1, 0), acc);
          acb = __fmaf_rn(wv[4], X_(1, 1), acb);
          acd = __fmaf_rn(wv[5], X_(1, 2), acd);
          acc = __fmaf_rn(wv[6], X_(2, 0), acc);
          acb = __fmaf_rn(wv[7], X_(2, 1), acb);
          acd = __fmaf_rn(wv[8], X_(2, 2), acd);
#undef X_
          acc = __fadd_rn(acc, __fadd_rn(acb, acd));
          const float v = silu<true>(acc, lut);
          o[(long long)p * C + c] = v;
          tile[pp + i * PPT][c_l] = v;
        }
      }
    }
    __syncthreads();
    if (tid < SC) {
      const int n = min(TP, P - p0);
      for (int i = 0; i < n; i++) cs = __fadd_rn(cs, tile[i][tid]);
    }
    __syncthreads();
  }
  if (tid < SC) chsum[win * cws + blockIdx.x * SC + tid] = cs;
}

// ------------------------------------------------------------------ SE_GATE (src/v24_f32.c:164-179, rt_ops_f32.c:272-283)

// One CTA per window. fc1 row r: 8 threads hold the 8 NEON accumulator lanes (a0 lanes 0-3, a1 lanes 0-3) over
// c = 8i + lane, then (a0 + a1) lane-wise and the FADDP reduction (v0 + v1) + (v2 + v3); SiLU with libm expf and an
// IEEE division. fc2 per channel from the bias, one FMA per r in order, then the sigmoid.
__global__ void __launch_bounds__(256) k_se_gate(int C, int rd, const float *__restrict__ w1, const float *__restrict__ b1,
                                                 const float *__restrict__ w2t, const float *__restrict__ b2,
                                                 const float *__restrict__ chsum, long long cws, int P,
                                                 float *__restrict__ gate, long long gws) {
  extern __shared__ float sm[];
  float *mean = sm, *s1 = sm + C;
  const int win = blockIdx.x, tid = threadIdx.x;
  const float inv = __fdiv_rn(1.f, __int2float_rn(P));
  for (int c = tid; c < C; c += 256) mean[c] = __fmul_rn(chsum[win * cws + c], inv);
  __syncthreads();
  const int lane8 = tid & 7;
  for (int r0 = 0; r0 < rd; r0 += 32) {
    const int r = r0 + tid / 8;
    float a = 0.f;
    if (r < rd) {
      const float *wr = w1 + (long long)r * C;
      for (int c = lane8; c + (8 - lane8) <= C; c += 8) a = __fmaf_rn(wr[c], mean[c], a);
    }
    // lanes l and l + 4 hold a0[l] and a1[l]
    const float other = __shfl_down_sync(0xffffffffu, a, 4, 8);
    float v = __fadd_rn(a, other);  // v[l] for l < 4
    const float v1 = __shfl_down_sync(0xffffffffu, v, 1, 8), v2 = __shfl_down_sync(0xffffffffu, v, 2, 8),
                v3 = __shfl_down_sync(0xffffffffu, v, 3, 8);
    if (r < rd && lane8 == 0) {
      const float xr = __fadd_rn(__fadd_rn(__fadd_rn(v, v1), __fadd_rn(v2, v3)), b1[r]);
      s1[r] = __fdiv_rn(xr, __fadd_rn(1.f, glibc_expf(-xr, c_expf_tab)));
    }
  }
  __syncthreads();
  for (int c = tid; c < C; c += 256) {
    float g = b2[c];
    for (int r = 0; r < rd; r++) g = __fmaf_rn(w2t[(long long)r * C + c], s1[r], g);
    gate[win * gws + c] = sigmoid(g);
  }
}

// ------------------------------------------------------------------ C0POOL (src/v24_f32.c:139-147, gemm_f32.c:60-70)

// One CTA per (output row oy, window); thread qx computes the pooled pixel qx: conv pixels 2qx and 2qx + 1, 24
// channels each, K = 64 fused multiply-adds in (ky, kx, ci) order from 0, bias added after, ReLU, max | average.
__global__ void __launch_bounds__(128) k_c0pool(const float *__restrict__ img, long long iws, const float *__restrict__ wt,
                                                const float *__restrict__ bias, float *__restrict__ pin, long long pws) {
  constexpr int PWD = 518;  // padded width: 3 + 511 + 4
  __shared__ float rows[4][PWD * 2];
  __shared__ float ws[64][24];
  __shared__ float bs[24];
  const int oy = blockIdx.x, win = blockIdx.y, tid = threadIdx.x;
  const float *im = img + win * iws;
  for (int i = tid; i < 4 * PWD * 2; i += 128) {
    const int r = i / (PWD * 2), cidx = i - r * PWD * 2;
    const int y = 2 * oy + r - 1, xcol = cidx / 2 - 3, ch = cidx & 1;
    rows[r][cidx] = (y >= 0 && y < 96 && xcol >= 0 && xcol < 511) ? im[((long long)y * 511 + xcol) * 2 + ch] : 0.f;
  }
  for (int i = tid; i < 64 * 24; i += 128) ws[i / 24][i % 24] = wt[i];
  if (tid < 24) bs[tid] = bias[tid];
  __syncthreads();
  const int qx = tid;
  float res[2][24];
#pragma unroll
  for (int pix = 0; pix < 2; pix++) {
    const int ox = 2 * qx + pix;
    float acc[24];
#pragma unroll
    for (int n = 0; n < 24; n++) acc[n] = 0.f;
    for (int ky = 0; ky < 4; ky++)
#pragma unroll 4
      for (int kk = 0; kk < 16; kk++) {
        const float a = rows[ky][2 * ox * 2 + kk];
        const float *wr = ws[ky * 16 + kk];
#pragma unroll
        for (int n = 0; n < 24; n++) acc[n] = __fmaf_rn(wr[n], a, acc[n]);
      }
#pragma unroll
    for (int n = 0; n < 24; n++) res[pix][n] = fmax_nan(__fadd_rn(acc[n], bs[n]), 0.f);
  }
  float *o = pin + win * pws + ((long long)oy * 128 + qx) * 48;
#pragma unroll
  for (int n = 0; n < 24; n++) {
    o[n] = fmax_nan(res[0][n], res[1][n]);
    o[24 + n] = __fmul_rn(__fadd_rn(res[0][n], res[1][n]), 0.5f);
  }
}

// ------------------------------------------------------------------ POSTPC (src/v24_f32.c:245-266)

// post BN + ReLU and the 3x3 valid im2col: pcin [B][6][1728]
__global__ void k_postpc_im2col(const float *__restrict__ X, long long xws, const float *__restrict__ ps,
                                const float *__restrict__ pb, float *__restrict__ pcin) {
  const int win = blockIdx.x;
  for (int i = threadIdx.x; i < 6 * 1728; i += blockDim.x) {
    const int ox = i / 1728, k = i - ox * 1728, tap = k / 192, c = k - tap * 192;
    const int ky = tap / 3, kx = tap - ky * 3;
    const float v = X[win * xws + (long long)(ky * 8 + ox + kx) * 192 + c];
    pcin[(long long)win * 6 * 1728 + i] = fmax_nan(__fmaf_rn(v, ps[c], pb[c]), 0.f);
  }
}

// pc GEMM + ReLU + mean: thread = output channel n, WG windows x 6 rows of sequential fused multiply-adds from 0 over
// k (the reference's K loop), bias after, ReLU, then the 6 rows added in order and scaled by 1/6
constexpr int kPcWG = 8, kPcKC = 64;
__global__ void __launch_bounds__(128) k_postpc_gemm(int B, const float *__restrict__ pcin, const float *__restrict__ wt,
                                                     const float *__restrict__ bias, float *__restrict__ feat,
                                                     long long fws) {
  __shared__ float a_s[kPcWG][6][kPcKC];
  const int n = blockIdx.x * 128 + threadIdx.x, w0 = blockIdx.y * kPcWG;
  float acc[kPcWG][6];
#pragma unroll
  for (int j = 0; j < kPcWG; j++)
#pragma unroll
    for (int r = 0; r < 6; r++) acc[j][r] = 0.f;
  for (int k0 = 0; k0 < 1728; k0 += kPcKC) {
    __syncthreads();
    for (int i = threadIdx.x; i < kPcWG * 6 * kPcKC; i += 128) {
      const int j = i / (6 * kPcKC), rem = i - j * 6 * kPcKC, r = rem / kPcKC, kk = rem - r * kPcKC;
      a_s[j][r][kk] = (w0 + j < B) ? pcin[((long long)(w0 + j) * 6 + r) * 1728 + k0 + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kPcKC; kk++) {
      const float wv = wt[(long long)(k0 + kk) * 1024 + n];
#pragma unroll
      for (int j = 0; j < kPcWG; j++)
#pragma unroll
        for (int r = 0; r < 6; r++) acc[j][r] = __fmaf_rn(a_s[j][r][kk], wv, acc[j][r]);
    }
  }
  const float b = bias[n];
#pragma unroll
  for (int j = 0; j < kPcWG; j++) {
    if (w0 + j >= B) break;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < 6; r++) s = __fadd_rn(s, fmax_nan(__fadd_rn(acc[j][r], b), 0.f));
    feat[(long long)(w0 + j) * fws + n] = __fmul_rn(s, 0x1.555556p-3f);
  }
}

// ------------------------------------------------------------------ FE_STFT2 (src/v24_fe.c:127-224, fft_tab.h)

constexpr int kNsamp = 144000, kNfr = 511, kNmel = 96;

// per window: mn = min, den = (max - mn) + 1e-6 (NaN-propagating NEON min/max)
__global__ void __launch_bounds__(512) k_fe_minmax(const float *__restrict__ pcm, long long pws, float *__restrict__ mm) {
  __shared__ float smn[16], smx[16];
  const float *x = pcm + blockIdx.x * pws;
  float mn = x[0], mx = x[0];
  for (int i = threadIdx.x; i < kNsamp / 4; i += 512) {
    const float4 v = reinterpret_cast<const float4 *>(x)[i];
    mn = fmin_nan(mn, fmin_nan(fmin_nan(v.x, v.y), fmin_nan(v.z, v.w)));
    mx = fmax_nan(mx, fmax_nan(fmax_nan(v.x, v.y), fmax_nan(v.z, v.w)));
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (threadIdx.x % 32 == 0) { smn[threadIdx.x / 32] = mn; smx[threadIdx.x / 32] = mx; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < 16; i++) { mn = fmin_nan(mn, smn[i]); mx = fmax_nan(mx, smx[i]); }
    mm[2 * blockIdx.x] = mn;
    mm[2 * blockIdx.x + 1] = __fadd_rn(__fsub_rn(mx, mn), 1e-6f);
  }
}

// complex product as the reference forms it: (x w)_r = fma(-x_i, w_i, x_r w_r), (x w)_i = fma(x_i, w_r, x_r w_i)
__device__ __forceinline__ void cmul(float xr, float xi, float wr, float wi, float &pr, float &pi) {
  pr = __fmaf_rn(-xi, wi, __fmul_rn(xr, wr));
  pi = __fmaf_rn(xi, wr, __fmul_rn(xr, wi));
}

// One CTA per (4 frames, spectrogram, window): normalized, windowed samples in bit-reversed order into shared
// memory, the reference's DIT passes (two fused levels, radix-2^2 passes, a last radix-2 level when log2 M is odd),
// the real part of the half-size transform, sparse mel, |m|^(2p) by the log2 / exp2 polynomials, BN, reversed rows.
constexpr int kFeF = 4;
__global__ void __launch_bounds__(256) k_fe_spec(const float *__restrict__ pcm, long long pws,
                                                 const float *__restrict__ mm, const bnnk_fe_tables t,
                                                 float *__restrict__ img, long long iws) {
  extern __shared__ float sm[];
  const int br = blockIdx.y, win = blockIdx.z, t0 = blockIdx.x * kFeF;
  const int M = br ? 512 : 1024, hop = br ? 280 : 278;
  float *re = sm, *im = sm + kFeF * M, *R = sm + 2 * kFeF * M;  // R: [kFeF][M + 1]
  const float mn = mm[2 * win], den = mm[2 * win + 1];
  const float *x = pcm + win * pws;
  const float *wv = t.win[br];
  const int *rev = t.rev[br];
  const float *twr = t.tw_re[br], *twi = t.tw_im[br];
  const int tid = threadIdx.x;
  for (int i = tid; i < kFeF * M; i += 256) {
    const int f = i / M, n = i - f * M;
    const int fr = min(t0 + f, kNfr - 1), st = fr * hop;
    const float y0 = __fmul_rn(__fsub_rn(__fdiv_rn(__fsub_rn(x[st + 2 * n], mn), den), 0.5f), 2.f);
    const float y1 = __fmul_rn(__fsub_rn(__fdiv_rn(__fsub_rn(x[st + 2 * n + 1], mn), den), 0.5f), 2.f);
    re[f * M + rev[n]] = __fmul_rn(y0, wv[2 * n]);
    im[f * M + rev[n]] = __fmul_rn(y1, wv[2 * n + 1]);
  }
  __syncthreads();
  // levels 1-2 fused, no twiddles
  for (int g = tid; g < kFeF * M / 4; g += 256) {
    const int f = g / (M / 4), i = (g - f * (M / 4)) * 4;
    float *pr = re + f * M + i, *pi = im + f * M + i;
    const float ar = pr[0], ai = pi[0], brr = pr[1], bi = pi[1], cr = pr[2], ci = pi[2], dr = pr[3], di = pi[3];
    const float s0r = __fadd_rn(ar, brr), s0i = __fadd_rn(ai, bi), d0r = __fsub_rn(ar, brr), d0i = __fsub_rn(ai, bi);
    const float s1r = __fadd_rn(cr, dr), s1i = __fadd_rn(ci, di), d1r = __fsub_rn(cr, dr), d1i = __fsub_rn(ci, di);
    pr[0] = __fadd_rn(s0r, s1r); pi[0] = __fadd_rn(s0i, s1i);
    pr[2] = __fsub_rn(s0r, s1r); pi[2] = __fsub_rn(s0i, s1i);
    pr[1] = __fadd_rn(d0r, d1i); pi[1] = __fsub_rn(d0i, d1r);
    pr[3] = __fsub_rn(d0r, d1i); pi[3] = __fadd_rn(d0i, d1r);
  }
  __syncthreads();
  int len = 8;
  for (; 2 * len <= M; len <<= 2) {
    const int h = len / 2, st1 = M / len, st2 = M / (2 * len);
    for (int g = tid; g < kFeF * M / 4; g += 256) {
      const int f = g / (M / 4), gg = g - f * (M / 4), i = (gg / h) * 2 * len, j = gg % h;
      float *pr = re + f * M + i + j, *pi = im + f * M + i + j;
      const float w1r = twr[j * st1], w1i = twi[j * st1], w2r = twr[j * st2], w2i = twi[j * st2];
      const float ar = pr[0], ai = pi[0], brr = pr[h], bi = pi[h], cr = pr[2 * h], ci = pi[2 * h], dr = pr[3 * h],
                  di = pi[3 * h];
      float tr, ti;
      cmul(brr, bi, w1r, w1i, tr, ti);
      const float a1r = __fadd_rn(ar, tr), a1i = __fadd_rn(ai, ti), b1r = __fsub_rn(ar, tr), b1i = __fsub_rn(ai, ti);
      cmul(dr, di, w1r, w1i, tr, ti);
      const float c1r = __fadd_rn(cr, tr), c1i = __fadd_rn(ci, ti), d1r = __fsub_rn(cr, tr), d1i = __fsub_rn(ci, ti);
      cmul(c1r, c1i, w2r, w2i, tr, ti);
      pr[0] = __fadd_rn(a1r, tr); pi[0] = __fadd_rn(a1i, ti);
      pr[2 * h] = __fsub_rn(a1r, tr); pi[2 * h] = __fsub_rn(a1i, ti);
      float ur, ui;
      cmul(d1r, d1i, w2r, w2i, ur, ui);
      pr[h] = __fadd_rn(b1r, ui); pi[h] = __fsub_rn(b1i, ur);
      pr[3 * h] = __fsub_rn(b1r, ui); pi[3 * h] = __fadd_rn(b1i, ur);
    }
    __syncthreads();
  }
  for (; len <= M; len <<= 1) {
    const int half = len / 2, step = M / len;
    for (int g = tid; g < kFeF * M / 2; g += 256) {
      const int f = g / (M / 2), gg = g - f * (M / 2), i = (gg / half) * len, j = gg % half;
      float *pr = re + f * M + i + j, *pi = im + f * M + i + j;
      float vr, vi;
      cmul(pr[half], pi[half], twr[j * step], twi[j * step], vr, vi);
      const float ur = pr[0], ui = pi[0];
      pr[0] = __fadd_rn(ur, vr); pi[0] = __fadd_rn(ui, vi);
      pr[half] = __fsub_rn(ur, vr); pi[half] = __fsub_rn(ui, vi);
    }
    __syncthreads();
  }
  // real part: Re X_k = 1/2 [(Zr_k + Zr_{M-k}) + c (Zi_k + Zi_{M-k}) - s (Zr_k - Zr_{M-k})]; Z_M = Z_0
  const int klo = t.klo[br], khi = t.khi[br], nk = khi - klo;
  for (int i = tid; i < kFeF * nk; i += 256) {
    const int f = i / nk, k = klo + (i - f * nk);
    const int k1 = k == M ? 0 : k, k2 = k == 0 ? 0 : M - k;
    const float zr = re[f * M + k1], zi = im[f * M + k1], yr = re[f * M + k2], yi = im[f * M + k2];
    float v = __fadd_rn(zr, yr);
    v = __fmaf_rn(__fadd_rn(zi, yi), t.pc[br][k], v);
    v = __fmaf_rn(-__fsub_rn(zr, yr), t.ps[br][k], v);
    R[f * (M + 1) + k] = __fmul_rn(v, 0.5f);
  }
  __syncthreads();
  const int *moff = t.mel_off[br], *mk = t.mel_k[br];
  const float *mw = t.mel_w[br];
  const float pw2 = t.pw2[br], bs = t.bn_s[br], bb = t.bn_b[br];
  for (int i = tid; i < kFeF * kNmel; i += 256) {
    const int f = i / kNmel, j = i - f * kNmel, fr = t0 + f;
    if (fr >= kNfr) continue;
    const float *Rf = R + f * (M + 1);
    float a0 = 0.f, a1 = 0.f;
    int e = moff[j];
    const int e1 = moff[j + 1];
    for (; e + 2 <= e1; e += 2) {
      a0 = __fmaf_rn(Rf[mk[e]], mw[e], a0);
      a1 = __fmaf_rn(Rf[mk[e + 1]], mw[e + 1], a1);
    }
    if (e < e1) a0 = __fmaf_rn(Rf[mk[e]], mw[e], a0);
    const float m = fmax_nan(fabsf(__fadd_rn(a0, a1)), 1e-30f);
    const float p = exp2_acc(__fmul_rn(pw2, log2_acc(m)));
    img[win * iws + ((long long)(kNmel - 1 - j) * kNfr + fr) * 2 + br] = __fmaf_rn(p, bs, bb);
  }
}

}  // namespace bnn

using namespace bnn;

// ------------------------------------------------------------------ launchers

extern "C" int bnnk_fp32_tables_init(const unsigned long long *tab, const uint32_t *lut) {
  cudaError_t e = cudaMemcpyToSymbol(c_expf_tab, tab, sizeof(unsigned long long) * 32);
  if (e) return e;
  return cudaMemcpyToSymbol(g_frecpe_lut, lut, sizeof(uint32_t) * 256);
}

extern "C" int bnnk_dw3(int B, const float *xp, long long xws, int H, int W, int C, int s, const float *w,
                        const float *b, float *out, long long ows, int Ho, int Wo, float *chsum, long long cws,
                        bnn_stream_t st) {
  (void)H;
  if (B <= 0) return 0;
  if (C % 32 == 0) k_dw3<32><<<dim3(C / 32, B), 256, 0, st>>>(xp, xws, W, C, s, w, b, out, ows, Ho, Wo, chsum, cws);
  else if (C % 24 == 0) k_dw3<24><<<dim3(C / 24, B), 256, 0, st>>>(xp, xws, W, C, s, w, b, out, ows, Ho, Wo, chsum, cws);
  else if (C % 16 == 0) k_dw3<16><<<dim3(C / 16, B), 256, 0, st>>>(xp, xws, W, C, s, w, b, out, ows, Ho, Wo, chsum, cws);
  else k_dw3<8><<<dim3(C / 8, B), 256, 0, st>>>(xp, xws, W, C, s, w, b, out, ows, Ho, Wo, chsum, cws);
  return cudaGetLastError();
}

extern "C" int bnnk_se_gate(int B, int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                            const float *chsum, long long cws, int P, float *gate, long long gws, bnn_stream_t st) {
  if (B <= 0) return 0;
  const size_t smem = sizeof(float) * (size_t)(C + rd);
  k_se_gate<<<B, 256, smem, st>>>(C, rd, w1, b1, w2t, b2, chsum, cws, P, gate, gws);
  return cudaGetLastError();
}

extern "C" int bnnk_c0pool(int B, const float *img, long long iws, const float *wt, const float *b, float *pin,
                           long long pws, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_c0pool<<<dim3(48, B), 128, 0, st>>>(img, iws, wt, b, pin, pws);
  return cudaGetLastError();
}

extern "C" int bnnk_postpc(int B, const float *X, long long xws, const float *post_s, const float *post_b,
                           const float *wt, const float *b, float *pcin, float *feat, long long fws, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_postpc_im2col<<<B, 256, 0, st>>>(X, xws, post_s, post_b, pcin);
  k_postpc_gemm<<<dim3(1024 / 128, (B + kPcWG - 1) / kPcWG), 128, 0, st>>>(B, pcin, wt, b, feat, fws);
  return cudaGetLastError();
}

extern "C" int bnnk_fe_stft2(int B, const float *pcm, long long pws, const bnnk_fe_tables *t, float *minmax,
                             float *img, long long iws, bnn_stream_t st) {
  if (B <= 0) return 0;
  static bool attr = false;
  const size_t smem = sizeof(float) * (size_t)(2 * kFeF * 1024 + kFeF * 1025);
  if (!attr) {
    cudaFuncSetAttribute(k_fe_spec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  k_fe_minmax<<<B, 512, 0, st>>>(pcm, pws, minmax);
  k_fe_spec<<<dim3((kNfr + kFeF - 1) / kFeF, 2, B), 256, smem, st>>>(pcm, pws, minmax, *t, img, iws);
  return cudaGetLastError();
}
