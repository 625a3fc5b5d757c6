// FE_STFT2 on B200: the BirdNET v2.4 two-spectrogram front end (src/v24_fe.c:127-224, src/fft_tab.h:25-77).
//
// Arithmetic is the reference's, element for element: y = ((x - mn) / den - 0.5) * 2 per sample; z[n] = y[2n] w[2n]
// + i y[2n+1] w[2n+1] in bit-reversed order; the DIT transform with the first two levels fused (no twiddles), then
// radix-2^2 passes over level pairs (len, 2 len) with twiddles w1 = tw[j M/len], w2 = tw[j M/(2 len)], then one
// radix-2 level when log2 M is odd; complex products formed as (x w)_r = fma(-x_i, w_i, x_r w_r),
// (x w)_i = fma(x_i, w_r, x_r w_i); the real part of the half-size transform; the sparse mel with two alternating
// accumulators; max(|.|, 1e-30); |m|^(2p) by the log2 / exp2 polynomials; BN as one fma; rows written reversed.
//
// Schedule (ours): one CTA per (8 frames, spectrogram, window). The frames' samples are normalized once into a
// shared segment. A frame of M points is owned by M/16 threads holding 16 points each in registers; the 16-point
// sets are chosen so that two consecutive passes close over them (levels 1-4: 16 consecutive bit-reversed
// positions; levels 5-8: the points j + 16a + 64b of a 256-block; levels 9-10: four points 256 apart), so a frame
// makes 3 round trips through shared memory instead of one per pass. Points are stored as (re, im) pairs, their
// shared indices padded (p + p/16) so the 16-strided accesses do not collide in banks.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bnn_kernels.h"
#include "smem_attr.cuh"
#include "emu.cuh"

namespace bnn {

constexpr int kNsamp = 144000, kNfr = 511, kNmel = 96, kFG = 8;

__device__ __forceinline__ int sx(int p) { return p + (p >> 4); }
// the sample segment's padded index (one word per 32): the bit-reversed gathers, 4 words apart across a warp, then
// fall in distinct banks
__device__ __forceinline__ int sg(int i) { return i + (i >> 5); }

// the 4-bit reverse of e (levels 1-4 gather their 16 points in bit-reversed order)
__host__ __device__ constexpr int rev4(int e) { return ((e & 1) << 3) | ((e & 2) << 1) | ((e & 4) >> 1) | ((e & 8) >> 3); }

struct cpx {
  float r, i;
};
// x * w as the reference forms it
__device__ __forceinline__ cpx cmul(cpx x, float wr, float wi) {
  return {__fmaf_rn(-x.i, wi, __fmul_rn(x.r, wr)), __fmaf_rn(x.i, wr, __fmul_rn(x.r, wi))};
}

// one radix-2^2 butterfly group (fft_tab.h:51-62): a, b, c, d = points i+j, +h, +2h, +3h. On paired fp32 lanes:
// x w = fma2((x_i, x_i), (-w_i, w_r), (x_r, x_r) (w_r, w_i)) gives (fma(-x_i, w_i, x_r w_r), fma(x_i, w_r, x_r w_i)),
// each lane rounded as the scalar form; the leg b1 + (-i) u uses u' = d1 (-i w2) = -i u exactly (the negations and
// swaps are exact), so both legs are paired sums.
__device__ __forceinline__ float2 cmul2(float2 x, float2 w, float2 wn) {  // wn = (-w_i, w_r)
  return fma2_rn(splat2(x.y), wn, mul2_rn(splat2(x.x), w));
}
__device__ __forceinline__ void r22(cpx &a, cpx &b, cpx &c, cpx &d, float w1r, float w1i, float w2r, float w2i) {
  const float2 w1 = make_float2(w1r, w1i), w1n = make_float2(-w1i, w1r);
  const float2 w2 = make_float2(w2r, w2i), w2n = make_float2(-w2i, w2r), w2m = make_float2(w2i, -w2r);  // -i w2
  const float2 A = make_float2(a.r, a.i), B = make_float2(b.r, b.i), C = make_float2(c.r, c.i),
               D = make_float2(d.r, d.i);
  float2 t = cmul2(B, w1, w1n);
  const float2 a1 = add2_rn(A, t), b1 = sub2_rn(A, t);
  t = cmul2(D, w1, w1n);
  const float2 c1 = add2_rn(C, t), d1 = sub2_rn(C, t);
  t = cmul2(c1, w2, w2n);
  const float2 ao = add2_rn(a1, t), co = sub2_rn(a1, t);
  const float2 u = cmul2(d1, w2m, w2);  // -i (d1 w2): its (-w_i, w_r) is (w2r, w2i)
  const float2 bo = add2_rn(b1, u), dd = sub2_rn(b1, u);
  a = {ao.x, ao.y};
  b = {bo.x, bo.y};
  c = {co.x, co.y};
  d = {dd.x, dd.y};
}

// the first two levels fused, without twiddles (fft_tab.h:28-38)
__device__ __forceinline__ void r4first(cpx &a, cpx &b, cpx &c, cpx &d) {
  const cpx s0 = {__fadd_rn(a.r, b.r), __fadd_rn(a.i, b.i)}, d0 = {__fsub_rn(a.r, b.r), __fsub_rn(a.i, b.i)};
  const cpx s1 = {__fadd_rn(c.r, d.r), __fadd_rn(c.i, d.i)}, d1 = {__fsub_rn(c.r, d.r), __fsub_rn(c.i, d.i)};
  a = {__fadd_rn(s0.r, s1.r), __fadd_rn(s0.i, s1.i)};
  c = {__fsub_rn(s0.r, s1.r), __fsub_rn(s0.i, s1.i)};
  b = {__fadd_rn(d0.r, d1.i), __fsub_rn(d0.i, d1.r)};
  d = {__fsub_rn(d0.r, d1.i), __fadd_rn(d0.i, d1.r)};
}

template <int LG>
__device__ __forceinline__ void spec(const float *__restrict__ x, float mn, float den, const bnnk_fe_tables &t,
                                     float *__restrict__ img, int t0, float *sm) {
  constexpr int M = 1 << LG, BR = LG == 10 ? 0 : 1, HOP = BR ? 280 : 278, TPF = M / 16, FF = 256 / TPF;
  constexpr int SEG = (((kFG - 1) * HOP + 2 * M) * 33 / 32 + 2) & ~1, MP = M + M / 16;  // SEG even: pts 8-byte aligned
  float *seg = sm;
  float2 *pts = reinterpret_cast<float2 *>(sm + SEG);  // [FF][MP] (re, im)
  float *R = reinterpret_cast<float *>(pts + FF * MP);
  const int tid = threadIdx.x, fl = tid / TPF, lt = tid % TPF;
  const float *__restrict__ win = t.win[BR];
  const float *__restrict__ twr = t.tw_re[BR];
  const float *__restrict__ twi = t.tw_im[BR];
  // the radix-2^2 stages' twiddle pairs (w1, w2) in the order the stages read them
  const float4 *__restrict__ tws = reinterpret_cast<const float4 *>(t.tw_st[BR]);
  const int nfr = min(kFG, kNfr - t0);
  const int start = t0 * HOP, len = (nfr - 1) * HOP + 2 * M;
  for (int i0 = 0; i0 < len; i0 += 256 * 8) {  // 8 loads in flight per thread before the divisions
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * 256 + tid;
      v[u] = i < len ? __ldg(x + start + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * 256 + tid;
      if (i < len) seg[sg(i)] = __fmul_rn(__fsub_rn(__fdiv_rn(__fsub_rn(v[u], mn), den), 0.5f), 2.f);
    }
  }
  const int klo = t.klo[BR], nk = t.khi[BR] - klo;
  __syncthreads();
  for (int f0 = 0; f0 < nfr; f0 += FF) {
    const int f = f0 + fl;  // this thread's frame within the CTA's group
    const bool live = f < nfr;
    float2 *fp = pts + fl * MP;
    if (live) {
      // levels 1-4 on the 16 consecutive bit-reversed positions 16 lt .. 16 lt + 15
      cpx z[16];
      const int st = f * HOP;
      // the bit reverse of 16 lt + e in LG bits is rev(16 lt) + rev4(e) 2^(LG-4): one base per thread, compile-time
      // offsets per point. st + 2 n is even, so sample 2 n + 1 sits one word after sample 2 n in the padded segment,
      // and the offsets 2 rev4(e) 2^(LG-4) are multiples of 32, so they pass through sg() unchanged plus 1/32.
      const float *sb = seg + sg(st + 2 * (int)(__brev((unsigned)(16 * lt)) >> (32 - LG)));
      const float2 *wb = reinterpret_cast<const float2 *>(win) + lt;
#pragma unroll
      for (int e = 0; e < 16; e++) {
        constexpr int kSh = LG - 3;
        const int ce = rev4(e) << kSh;
        const float2 w = wb[e * TPF];  // (w[2n], w[2n+1]), lanes adjacent
        z[e] = {__fmul_rn(sb[ce + (ce >> 5)], w.x), __fmul_rn(sb[ce + (ce >> 5) + 1], w.y)};
      }
#pragma unroll
      for (int g = 0; g < 4; g++) r4first(z[4 * g], z[4 * g + 1], z[4 * g + 2], z[4 * g + 3]);
#pragma unroll
      for (int j = 0; j < 4; j++)  // len 8: h 4, st1 = M / 8, st2 = M / 16
      {
        const float4 w = __ldg(tws + j);  // stage 0 (len 8): w1 = tw[j M / 8], w2 = tw[j M / 16]
        r22(z[j], z[j + 4], z[j + 8], z[j + 12], w.x, w.y, w.z, w.w);
      }
      float2 *fo = fp + 17 * lt;  // sx(16 lt + e) = 17 lt + e
#pragma unroll
      for (int e = 0; e < 16; e++) fo[e] = make_float2(z[e].r, z[e].i);
    }
    __syncthreads();
    if (live) {
      // levels 5-8 on the points base + 16 a + 64 b of a 256-block
      const int j = lt & 15, base = (lt >> 4) * 256 + j;
      // base has j < 16 in its low four bits, so sx(base + 16 a + 64 b) = sx(base) + 17 a + 68 b
      float2 *fb = fp + sx(base);
      cpx z[16];
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
          const float2 v = fb[17 * a + 68 * b];
          z[a + 4 * b] = {v.x, v.y};
        }
      {  // len 32: h 16, groups (a = 0..3) for each b, twiddle index j
        const float4 w = __ldg(tws + 4 + j);  // stage 1 (len 32): w1 = tw[j M / 32], w2 = tw[j M / 64]
        const float w1r = w.x, w1i = w.y, w2r = w.z, w2i = w.w;
#pragma unroll
        for (int b = 0; b < 4; b++) r22(z[4 * b], z[4 * b + 1], z[4 * b + 2], z[4 * b + 3], w1r, w1i, w2r, w2i);
      }
#pragma unroll
      for (int a = 0; a < 4; a++) {  // len 128: h 64, groups (b = 0..3) for each a, twiddle index j + 16 a
        const int jj = j + 16 * a;
        const float4 w = __ldg(tws + 20 + jj);  // stage 2 (len 128): w1 = tw[jj M / 128], w2 = tw[jj M / 256]
        r22(z[a], z[a + 4], z[a + 8], z[a + 12], w.x, w.y, w.z, w.w);
      }
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) fb[17 * a + 68 * b] = make_float2(z[a + 4 * b].r, z[a + 4 * b].i);
    }
    __syncthreads();
    if (live) {
      if (LG == 10) {  // levels 9-10: len 512, h 256, st1 2, st2 1
        float2 *fq = fp + sx(lt);  // lt < 64: sx(lt + 64 c + 256 d) = sx(lt) + 68 c + 272 d
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int jj = lt + 64 * c;
          const float2 va = fq[68 * c], vb = fq[68 * c + 272], vc = fq[68 * c + 544], vd = fq[68 * c + 816];
          cpx a = {va.x, va.y}, b = {vb.x, vb.y}, cc = {vc.x, vc.y}, d = {vd.x, vd.y};
          const float4 w = __ldg(tws + 84 + jj);  // stage 3 (len 512): w1 = tw[2 jj], w2 = tw[jj]
          r22(a, b, cc, d, w.x, w.y, w.z, w.w);
          fq[68 * c] = make_float2(a.r, a.i);
          fq[68 * c + 272] = make_float2(b.r, b.i);
          fq[68 * c + 544] = make_float2(cc.r, cc.i);
          fq[68 * c + 816] = make_float2(d.r, d.i);
        }
      } else {  // level 9 alone (radix 2): len 512, half 256, step 1 (fft_tab.h:64-76)
        float2 *fq = fp + sx(lt);  // lt < 32: sx(lt + 32 c + 256 d) = sx(lt) + 34 c + 272 d
        const float *tr = twr + lt, *ti = twi + lt;
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const float2 hv = fq[34 * c + 272], uv = fq[34 * c];
          const cpx v = cmul({hv.x, hv.y}, tr[32 * c], ti[32 * c]);
          fq[34 * c] = make_float2(__fadd_rn(uv.x, v.r), __fadd_rn(uv.y, v.i));
          fq[34 * c + 272] = make_float2(__fsub_rn(uv.x, v.r), __fsub_rn(uv.y, v.i));
        }
      }
    }
    __syncthreads();
    // real part of X_k for the bins the filters use: 1/2 [(Zr_k + Zr_{M-k}) + c (Zi_k + Zi_{M-k}) - s (Zr_k - Zr_{M-k})]
    // bin-major: a bin's coefficients are loaded once for all the group's frames
    const int nff = min(FF, nfr - f0);
    for (int kk = tid; kk < nk; kk += 256) {
      const int k = klo + kk;
      const int k1 = k == M ? 0 : k, k2 = k == 0 ? 0 : M - k;  // Z_M = Z_0 (the reference reads past its buffer)
      const int o1 = sx(k1), o2 = sx(k2);
      const float pc = t.pc[BR][k], ps = t.ps[BR][k];
      for (int ff = 0; ff < nff; ff++) {
        const float2 *g = pts + ff * MP;
        const float2 zv = g[o1], yv = g[o2];
        const float zr = zv.x, zi = zv.y, yr = yv.x, yi = yv.y;
        float v = __fadd_rn(zr, yr);
        v = __fmaf_rn(__fadd_rn(zi, yi), pc, v);
        v = __fmaf_rn(-__fsub_rn(zr, yr), ps, v);
        R[ff * nk + kk] = __fmul_rn(v, 0.5f);
      }
    }
    __syncthreads();
    const int *__restrict__ moff = t.mel_off[BR];
    const int *__restrict__ mk = t.mel_k[BR];
    const float *__restrict__ mw = t.mel_w[BR];
    const float pw2 = t.pw2[BR], bs = t.bn_s[BR], bb = t.bn_b[BR];
    // a thread takes one filter for FB of the group's frames: each weight is loaded once and feeds FB frames' chains
    // (two alternating accumulators per frame, taps in order, as the reference forms them)
    constexpr int FB = FF / 2;
    for (int i = tid; i < 2 * kNmel; i += 256) {
      const int fb = i / kNmel, j = i - fb * kNmel, ffb = fb * FB;
      if (f0 + ffb >= nfr) continue;
      // a filter's taps are the consecutive bins lo .. lo + n - 1 (its nonzero range), so only the weights are
      // loaded per tap
      const int e0 = moff[j], n = moff[j + 1] - e0;
      const float *Rf = R + ffb * nk - klo + (n > 0 ? mk[e0] : klo);
      const float *wf = mw + e0;
      float a0[FB], a1[FB];
#pragma unroll
      for (int q = 0; q < FB; q++) a0[q] = a1[q] = 0.f;
      int e = 0;
      for (; e + 8 <= n; e += 8) {
        float wv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) wv[u] = __ldg(wf + e + u);
#pragma unroll
        for (int q = 0; q < FB; q++)
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            a0[q] = __fmaf_rn(Rf[q * nk + e + u], wv[u], a0[q]);
            a1[q] = __fmaf_rn(Rf[q * nk + e + u + 1], wv[u + 1], a1[q]);
          }
      }
      for (; e + 2 <= n; e += 2) {
        const float w0 = __ldg(wf + e), w1 = __ldg(wf + e + 1);
#pragma unroll
        for (int q = 0; q < FB; q++) {
          a0[q] = __fmaf_rn(Rf[q * nk + e], w0, a0[q]);
          a1[q] = __fmaf_rn(Rf[q * nk + e + 1], w1, a1[q]);
        }
      }
      if (e < n) {
        const float w0 = __ldg(wf + e);
#pragma unroll
        for (int q = 0; q < FB; q++) a0[q] = __fmaf_rn(Rf[q * nk + e], w0, a0[q]);
      }
#pragma unroll
      for (int q = 0; q < FB; q++) {
        const int fi2 = f0 + ffb + q;
        if (fi2 >= nfr) break;
        const float m = fmax_nan(fabsf(__fadd_rn(a0[q], a1[q])), 1e-30f);
        const float p = exp2_acc(__fmul_rn(pw2, log2_acc(m)));
        img[((long long)(kNmel - 1 - j) * kNfr + t0 + fi2) * 2 + BR] = __fmaf_rn(p, bs, bb);
      }
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(256) k_fe_spec(const float *__restrict__ pcm, long long pws,
                                                 const float *__restrict__ mm, const bnnk_fe_tables t,
                                                 float *__restrict__ img, long long iws) {
  extern __shared__ float sm[];
  const int win = blockIdx.z, t0 = blockIdx.x * kFG;
  const float *x = pcm + win * pws;
  float *imgw = img + win * iws;
  if (blockIdx.y == 0) spec<10>(x, mm[2 * win], mm[2 * win + 1], t, imgw, t0, sm);
  else spec<9>(x, mm[2 * win], mm[2 * win + 1], t, imgw, t0, sm);
}

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

// ------------------------------------------------------------------ FE_LOGMEL (src/pc_kern_f32.c:85-149)
// The framed log-mel front end of compiled models (Perch): any power-of-two nfft from 16 to 2048. The arithmetic is
// the reference's, element for element (group(), one lane per frame): windowed samples in bit-reversed order, the
// same DIT transform as FE_STFT2 (the butterflies above), |X_k| from the real split, the sparse mel over the nonzero
// weights with two alternating accumulators, ln = log2_acc * 0.69314718, times scale. Schedule (ours): one CTA per
// (kLmFrames frames, window); each frame's M points live in shared memory and kLmThreads threads run the passes
// over them (first two levels fused, radix-2^2 level pairs, a last radix-2 level when log2 M is odd).

constexpr int kLmFrames = 2, kLmThreads = 128;

// the points' shared-memory index, one pad word per 32: the butterfly passes' short strides and the 4-point groups
// of the first pass fall in distinct banks
__device__ __forceinline__ int lp(int i) { return i + (i >> 5); }

__global__ void __launch_bounds__(kLmFrames * kLmThreads) k_logmel(const float *__restrict__ pcm, long long pws,
                                                                 const bnnk_logmel_tables t, float *__restrict__ spec,
                                                                 long long sws) {
  extern __shared__ float lsm[];
  const int M = t.M, lg = t.lg, MP = M + M / 32;
  const int fl = threadIdx.x / kLmThreads, lt = threadIdx.x % kLmThreads;
  const int f = blockIdx.x * kLmFrames + fl, win = blockIdx.y;
  float *re = lsm + fl * (2 * MP + M + 2), *im = re + MP, *mag = im + MP;
  const float *x = pcm + win * pws;
  const bool live = f < t.nfr;
  {
    // levels 1-2 (fft_tab.h:28-38) on the 4 consecutive bit-reversed positions 4g .. 4g + 3, gathered straight from
    // the samples: z[n] = w[2n] y[st + 2n] + i w[2n + 1] y[st + 2n + 1] (y: pad zeros, the window's samples, zeros),
    // 0 past the frame's (frame + 1) / 2 points
    const int st = f * t.hop - t.pad;
    for (int g = lt; g < M / 4; g += kLmThreads) {
      cpx z[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int n = (int)(__brev((unsigned)(4 * g + e)) >> (32 - lg));
        float vr = 0.f, vi = 0.f;
        if (live && n < t.nz) {
          const int i0 = st + 2 * n, i1 = i0 + 1;
          const float y0 = (i0 >= 0 && i0 < t.nsamp) ? __ldg(x + i0) : 0.f;
          const float y1 = (i1 >= 0 && i1 < t.nsamp) ? __ldg(x + i1) : 0.f;
          vr = __fmul_rn(y0, __ldg(t.win + 2 * n));
          vi = __fmul_rn(y1, __ldg(t.win + 2 * n + 1));
        }
        z[e] = {vr, vi};
      }
      r4first(z[0], z[1], z[2], z[3]);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        re[lp(4 * g + e)] = z[e].r;
        im[lp(4 * g + e)] = z[e].i;
      }
    }
  }
  __syncthreads();
  int len = 8;
  for (; 2 * len <= M; len <<= 2) {  // radix-2^2 over the level pair (len, 2 len) (fft_tab.h:40-64)
    const int h = len / 2, st1 = M / len, st2 = M / (2 * len);
    for (int q = lt; q < M / 4; q += kLmThreads) {
      const int j = q % h, i = (q / h) * 2 * len + j;
      const int ia = lp(i), ib = lp(i + h), ic = lp(i + 2 * h), id = lp(i + 3 * h);
      cpx a = {re[ia], im[ia]}, b = {re[ib], im[ib]}, c = {re[ic], im[ic]}, d = {re[id], im[id]};
      r22(a, b, c, d, __ldg(t.tw_re + j * st1), __ldg(t.tw_im + j * st1), __ldg(t.tw_re + j * st2),
          __ldg(t.tw_im + j * st2));
      re[ia] = a.r; im[ia] = a.i; re[ib] = b.r; im[ib] = b.i;
      re[ic] = c.r; im[ic] = c.i; re[id] = d.r; im[id] = d.i;
    }
    __syncthreads();
  }
  for (; len <= M; len <<= 1) {  // a last radix-2 level (fft_tab.h:65-76)
    const int half = len / 2, step = M / len;
    for (int q = lt; q < M / 2; q += kLmThreads) {
      const int j = q % half, i = (q / half) * len + j;
      const int iu = lp(i), iv = lp(i + half);
      const cpx v = cmul({re[iv], im[iv]}, __ldg(t.tw_re + j * step), __ldg(t.tw_im + j * step));
      const float ur = re[iu], ui = im[iu];
      re[iu] = __fadd_rn(ur, v.r); im[iu] = __fadd_rn(ui, v.i);
      re[iv] = __fsub_rn(ur, v.r); im[iv] = __fsub_rn(ui, v.i);
    }
    __syncthreads();
  }
  // |X_k|: A = Z_k, B = conj Z_{M-k}; E = (A + B) / 2, O = (A - B) / (2i); X = E + W^k O
  for (int k = t.klo + lt; k < t.khi; k += kLmThreads) {
    const int k2 = (k == 0 || k == M) ? 0 : M - k, ka = k == M ? 0 : k;
    const float Ar = re[lp(ka)], Ai = im[lp(ka)], Br = re[lp(k2)], Bi = -im[lp(k2)];
    const float Er = __fmul_rn(__fadd_rn(Ar, Br), 0.5f), Ei = __fmul_rn(__fadd_rn(Ai, Bi), 0.5f);
    const float Or = __fmul_rn(__fsub_rn(Ai, Bi), 0.5f), Oi = __fmul_rn(__fsub_rn(Br, Ar), 0.5f);
    const float c = __ldg(t.pc + k), sn = __ldg(t.ps + k);
    const float Xr = __fmaf_rn(Oi, sn, __fmaf_rn(Or, c, Er));
    const float Xi = __fmaf_rn(-Or, sn, __fmaf_rn(Oi, c, Ei));
    mag[k] = __fsqrt_rn(__fmaf_rn(Xi, Xi, __fmul_rn(Xr, Xr)));
  }
  __syncthreads();
  if (!live) return;
  float *out = spec + win * sws + (long long)f * t.nmel;
  for (int j = lt; j < t.nmel; j += kLmThreads) {
    float a0 = 0.f, a1 = 0.f;
    int e = __ldg(t.mel_off + j);
    const int e1 = __ldg(t.mel_off + j + 1);
    for (; e + 2 <= e1; e += 2) {
      a0 = __fmaf_rn(mag[__ldg(t.mel_k + e)], __ldg(t.mel_w + e), a0);
      a1 = __fmaf_rn(mag[__ldg(t.mel_k + e + 1)], __ldg(t.mel_w + e + 1), a1);
    }
    if (e < e1) a0 = __fmaf_rn(mag[__ldg(t.mel_k + e)], __ldg(t.mel_w + e), a0);
    out[j] = __fmul_rn(__fmul_rn(log2_acc(fmax_nan(__fadd_rn(a0, a1), t.floor_)), 0.69314718f), t.scale);
  }
}

}  // namespace bnn

using namespace bnn;

extern "C" int bnnk_fe_stft2(int B, const float *pcm, long long pws, const bnnk_fe_tables *t, float *minmax,
                             float *img, long long iws, bnn_stream_t st) {
  if (B <= 0) return 0;
  // shared memory: the larger of the two spectrograms' layouts
  auto need = [&](int lg, int br) {
    const int M = 1 << lg, hop = br ? 280 : 278, tpf = M / 16, ff = 256 / tpf;
    return sizeof(float) * (size_t)(((((kFG - 1) * hop + 2 * M) * 33 / 32 + 2) & ~1) + 2 * ff * (M + M / 16) +
                                    ff * (t->khi[br] - t->klo[br]));
  };
  const size_t smem = need(10, 0) > need(9, 1) ? need(10, 0) : need(9, 1);
  static SmemAttr attr;
  const cudaError_t e = attr.ensure(k_fe_spec, smem);
  if (e) return e;
  k_fe_minmax<<<B, 512, 0, st>>>(pcm, pws, minmax);
  k_fe_spec<<<dim3((kNfr + kFG - 1) / kFG, 2, B), 256, smem, st>>>(pcm, pws, minmax, *t, img, iws);
  return cudaGetLastError();
}

extern "C" int bnnk_logmel(int B, const float *pcm, long long pws, const bnnk_logmel_tables *t, float *spec,
                           long long sws, bnn_stream_t st) {
  if (B <= 0 || t->nfr <= 0) return 0;
  if (B > 65535) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float) * (size_t)kLmFrames * (2 * (t->M + t->M / 32) + t->M + 2);
  const dim3 grid((t->nfr + kLmFrames - 1) / kLmFrames, B);
  k_logmel<<<grid, kLmFrames * kLmThreads, smem, st>>>(pcm, pws, *t, spec, sws);
  return cudaGetLastError();
}
