// The fp32 ops of compiled models' neon-int8 paths beyond v2.4 on sm_100a: the BirdNET v3.0 ops (src/rt_ops_f32x.c:
// CONVK, CONVW, GEM, SED, VADD) and the fp32 bodies of Perch (src/rt_ops_f32.c: STEM, DWK, PAD, MEAN).
//
// Every output is the reference's chain of fp32 operations in the reference's order (the same rule as k_conv.cu):
//   * the fp32 GEMM (gemm_f32_kblock.h) is one accumulator per output from +0, k ascending, fused multiply-add, then
//     + bias, the activation (SiLU of silu_f32x4, ReLU = FMAX with +0) and the residual; CONVK feeds it the k x k
//     patches segment by segment (gemm_f32_seg), STEM the im2col rows, SED its pooled rows;
//   * Winograd F(4x4, 3x3) (wino_f32.c) transforms each 6x6 patch with B^T . B in the reference's operation order,
//     multiplies in the transform domain with the same GEMM K loop (+0.0 after it, as pt_tile adds), and transforms
//     back with A^T . A, then bias, activation and residual;
//   * the depthwise k x k (pc_kern_f32.c:163-335): four-pixel blocks keep two tap chains (even taps from the bias,
//     odd taps from zero) and the row's last Wo % 4 pixels one chain; the channel sums add ((v0 + v1) + (v2 + v3))
//     per block and v per tail pixel, in pixel order;
//   * GEM: log2 by the atanh series of rt_ops_f32x.c (an IEEE division), exp2_f32x4 (the polynomial of gemm_f32.h),
//     the mean as an IEEE division, then powf; SED: the axis mean and pooling in the reference's scalar order, the
//     three GEMMs, the attention softmax with libm expf (the glibc algorithm restated in emu.cuh).
// The one call out of reach is powf (GEM's final power, one per channel): the device uses the double-precision pow
// rounded once to float; results agree with glibc powf within one unit in the last place.
#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdint.h>

#include "bnn_kernels.h"
#include "emu.cuh"
#include "smem_attr.cuh"

namespace bnn {

// ------------------------------------------------------------------ shared pieces

__device__ __forceinline__ float act32(float v, int act, const uint32_t *lut) {
  if (act == 1) return silu<true>(v, lut);
  if (act == 2) return (v > 0.f || v != v) ? v : 0.f;  // vmaxq_f32(x, +0): NaN stays NaN, -0 -> +0
  return v;
}

// the zero halo ring of out [Ho + 2 h][Wo + 2 h][ld] (rt_zero_halo): only the ring's pixels are visited, the h top
// rows, then 2 h pixels of each interior row, then the h bottom rows; thread (ring pixel, channel)
__global__ void k_zero_halo(float *out, long long ows, int Ho, int Wo, int ld, int h) {
  const int Wp = Wo + 2 * h;
  const int top = h * Wp, mid = Ho * 2 * h, ring = 2 * top + mid;
  float *o = out + blockIdx.y * ows;
  const long long n = (long long)ring * ld;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(i / ld), c = (int)(i - (long long)p * ld);
    int y, x;
    if (p < top) {
      y = p / Wp; x = p - y * Wp;
    } else if (p < top + mid) {
      const int q = p - top, side = q % (2 * h);
      y = h + q / (2 * h);
      x = side < h ? side : Wo + side;
    } else {
      const int q = p - top - mid;
      y = h + Ho + q / Wp;
      x = q - (y - h - Ho) * Wp;
    }
    o[((long long)y * Wp + x) * ld + c] = 0.f;
  }
}

static int zero_halo(int B, float *out, long long ows, int Ho, int Wo, int ld, int h, bnn_stream_t st) {
  if (!h || B <= 0) return 0;
  const long long n = ((long long)2 * h * (Wo + 2 * h) + (long long)Ho * 2 * h) * ld;
  const int blocks = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
  k_zero_halo<<<dim3(blocks, B), 256, 0, st>>>(out, ows, Ho, Wo, ld, h);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ VADD (rt_ops_f32x.c:351-362)

__global__ void k_vadd(int n, const float *__restrict__ a, long long aws, const float *__restrict__ b, long long bws,
                       float *__restrict__ o, long long ows) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, w = blockIdx.y;
  if (i < n) o[w * ows + i] = __fadd_rn(a[w * aws + i], b[w * bws + i]);
}

// ------------------------------------------------------------------ GEM (rt_ops_f32x.c:150-198)

__device__ __forceinline__ float log2_atanh(float x) {
  const int32_t xi = __float_as_int(x);
  const int32_t e = (int32_t)((uint32_t)xi - 0x3f3504f3u) >> 23;
  const float m = __int_as_float((int32_t)((uint32_t)xi - ((uint32_t)e << 23)));
  const float s = __fdiv_rn(__fsub_rn(m, 1.f), __fadd_rn(m, 1.f));
  const float s2 = __fmul_rn(s, s);
  float q = __fmaf_rn(s2, 1.f / 11.f, 1.f / 9.f);
  q = __fmaf_rn(s2, q, 1.f / 7.f);
  q = __fmaf_rn(s2, q, 1.f / 5.f);
  q = __fmaf_rn(s2, q, 1.f / 3.f);
  q = __fmaf_rn(s2, q, 1.f);
  const float ln = __fmul_rn(__fmul_rn(s, 2.f), q);
  return __fmaf_rn(ln, 1.4426950408889634f, __int2float_rn(e));
}

__global__ void k_gem(int B, int P, int C, int ld, const float *__restrict__ x, long long xws,
                      const float *__restrict__ k, float *__restrict__ out, long long ows) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)B * C) return;
  const int w = (int)(i / C), c = (int)(i - (long long)w * C);
  const float eps = k[0], pp = k[1], qq = k[2];
  const float *xr = x + w * xws + c;
  float acc = 0.f;
  for (int p = 0; p < P; p++) {
    const float v = fmax_nan(__ldg(xr + (long long)p * ld), eps);
    acc = __fadd_rn(acc, exp2_poly(__fmul_rn(log2_atanh(v), pp)));
  }
  const float a = __fdiv_rn(acc, (float)P);
  out[w * ows + c] = __double2float_rn(pow((double)a, (double)qq));
}

// ------------------------------------------------------------------ MEAN, PAD (pc_kern_f32.c:336-349)

__global__ void k_mean_f32(int B, int P, int C, int ld, const float *__restrict__ x, long long xws,
                           float *__restrict__ out, long long ows) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)B * C) return;
  const int w = (int)(i / C), c = (int)(i - (long long)w * C);
  const float *xr = x + w * xws + c;
  float s = 0.f;
  for (int p = 0; p < P; p++) s = __fadd_rn(s, __ldg(xr + (long long)p * ld));
  out[w * ows + c] = __fdiv_rn(s, (float)P);
}

// V: channels in groups of 4 (C, ld and both window strides multiples of 4, 16-byte aligned buffers)
template <int V>
__global__ void k_pad_f32(int H, int W, int C, int ld, int h, const float *__restrict__ x, long long xws,
                          float *__restrict__ xp, long long pws) {
  const int CV = C / V;
  const long long n = (long long)H * W * CV;
  const int w = blockIdx.y;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int px = (int)(i / CV), c = (int)(i - (long long)px * CV) * V, y = px / W, xx = px - y * W;
    const float *src = x + w * xws + (long long)px * ld + c;
    float *dst = xp + w * pws + ((long long)(y + h) * (W + 2 * h) + xx + h) * C + c;
    if (V == 4) *reinterpret_cast<float4 *>(dst) = __ldg(reinterpret_cast<const float4 *>(src));
    else *dst = __ldg(src);
  }
}

// ------------------------------------------------------------------ DWK f32 (pc_kern_f32.c:163-335)

// The general form (any k and stride, unaligned buffers): one thread per (window, channel), the pixels in raster
// order, so that the channel sum is added in the reference's order; consecutive threads take consecutive channels
__global__ void k_dwk_f32(int B, int W, int C, int k, int s, int pt, int pl, const float *__restrict__ xp,
                          long long xws, const float *__restrict__ wt, const float *__restrict__ bias, int act,
                          float *__restrict__ out, long long ows, int Ho, int Wo, float *__restrict__ chsum,
                          long long cws) {
  __shared__ uint32_t lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = g_frecpe_lut[i];
  __syncthreads();
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)B * C) return;
  const int win = (int)(i / C), c = (int)(i - (long long)win * C);
  const int h = (k - 1) / 2, Wp = W + 2 * h, kk = k * k;
  const float *xw = xp + win * xws + c;
  float *ow = out + win * ows + c;
  const float b = __ldg(bias + c);
  float cs = 0.f;
  for (int oy = 0; oy < Ho; oy++) {
    const int iy0 = oy * s - pt + h;
    int ox = 0;
    for (; ox + 4 <= Wo; ox += 4) {
      float a[4] = {b, b, b, b}, e[4] = {0.f, 0.f, 0.f, 0.f};
      for (int t = 0; t < kk; t++) {
        const int ky = t / k, kx = t - ky * k;
        const float wv = __ldg(wt + (long long)t * C + c);
        const float *r = xw + ((long long)(iy0 + ky) * Wp + (ox * s - pl + h + kx)) * C;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float xv = __ldg(r + (long long)q * s * C);
          if (t & 1) e[q] = __fmaf_rn(xv, wv, e[q]);
          else a[q] = __fmaf_rn(xv, wv, a[q]);
        }
      }
      float v[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        v[q] = __fadd_rn(a[q], e[q]);
        if (act == 1) v[q] = silu<true>(v[q], lut);
        ow[(long long)(oy * Wo + ox + q) * C] = v[q];
      }
      cs = __fadd_rn(cs, __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])));
    }
    for (; ox < Wo; ox++) {
      float a = b;
      for (int t = 0; t < kk; t++) {
        const int ky = t / k, kx = t - ky * k;
        a = __fmaf_rn(__ldg(xw + ((long long)(iy0 + ky) * Wp + (ox * s - pl + h + kx)) * C),
                      __ldg(wt + (long long)t * C + c), a);
      }
      if (act == 1) a = silu<true>(a, lut);
      ow[(long long)(oy * Wo + ox) * C] = a;
      cs = __fadd_rn(cs, a);
    }
  }
  chsum[win * cws + c] = cs;
}

// The same op with a channel pair per thread and the map's rows over the CTA's thread rows: CTA (Lc channel pairs,
// window) of Lc x (Ry + 1) threads. Thread (lane, y < Ry) computes RT consecutive output rows of each chunk of Ry RT
// rows (RT > 1 on short rows) of its pair, unit by unit in the reference's order (blocks of four pixels, then the tail
// pixels), stores them
// and leaves each unit's addend in a double-buffered shared tile; thread row Ry adds the previous chunk's addends in
// row, then unit order (the raster order of the reference's channel sums) while the others compute the next chunk.
// The tap weights sit in shared memory; a block reads each tap row's 3 s + K inputs once. The tap chains are paired
// fused multiply-adds (each lane an IEEE FMA); the addends, sums of SiLU products, are scalar adds.
template <int K, int S, int G>
__device__ __forceinline__ float2 dwk2_unit(const float2 *xr, int rs, int cs, const float2 *ws, int wl, float2 b,
                                           int act, const uint32_t *lut, float2 *o, int os) {
  constexpr int NX = (G - 1) * S + K;
  float2 a[G], e[G];
#pragma unroll
  for (int q = 0; q < G; q++) { a[q] = b; e[q] = make_float2(0.f, 0.f); }
#pragma unroll
  for (int ky = 0; ky < K; ky++, xr += rs) {  // 32-bit offsets inside a window's rows
    float2 xv[NX];
#pragma unroll
    for (int j = 0; j < NX; j++) xv[j] = __ldg(xr + j * cs);
#pragma unroll
    for (int kx = 0; kx < K; kx++) {
      const int t = ky * K + kx;
      const float2 w = ws[t * wl];
#pragma unroll
      for (int q = 0; q < G; q++) {
        if (G == 4 && (t & 1)) e[q] = fma2_rn(xv[q * S + kx], w, e[q]);
        else a[q] = fma2_rn(xv[q * S + kx], w, a[q]);
      }
    }
  }
  float2 v[G];
#pragma unroll
  for (int q = 0; q < G; q++) {
    v[q] = G == 4 ? make_float2(__fadd_rn(a[q].x, e[q].x), __fadd_rn(a[q].y, e[q].y)) : a[q];
    if (act == 1) v[q] = silu2(v[q], lut);
    o[q * os] = v[q];
  }
  if (G == 4)
    return make_float2(__fadd_rn(__fadd_rn(v[0].x, v[1].x), __fadd_rn(v[2].x, v[3].x)),
                       __fadd_rn(__fadd_rn(v[0].y, v[1].y), __fadd_rn(v[2].y, v[3].y)));
  return v[0];
}

template <int K, int S>
__global__ void __launch_bounds__(256, 3) k_dwk2_f32(const float *__restrict__ xp, long long xws, int W, int C, int pt,
                                                  int pl, const float *__restrict__ wt, const float *__restrict__ bias,
                                                  int act, float *__restrict__ out, long long ows, int Ho, int Wo,
                                                  int nu, int RT, float *__restrict__ chsum, long long cws) {
  // RT: consecutive rows per thread and chunk (short rows: more work between the chunk barriers)
  extern __shared__ float2 sd2[];  // [K K][Lc] tap weights, then [2][Ry RT nu][Lc] unit addends of two chunks
  __shared__ uint32_t lut[256];
  constexpr int KK = K * K, h = (K - 1) / 2;
  const int Lc = blockDim.x, Ry = blockDim.y - 1, lane = threadIdx.x, win = blockIdx.y;
  const int tid = threadIdx.y * Lc + lane, nthr = Lc * blockDim.y;
  const int c2 = blockIdx.x * Lc + lane, C2 = C / 2;
  const bool on = c2 < C2, summer = threadIdx.y == Ry;
  float2 *ws = sd2, *sg = sd2 + KK * Lc;
  const int CR = Ry * RT, tile = CR * nu * Lc;  // rows per chunk
  for (int i = tid; i < 256; i += nthr) lut[i] = g_frecpe_lut[i];
  for (int t = threadIdx.y; t < KK; t += blockDim.y)
    ws[t * Lc + lane] = on ? __ldg(reinterpret_cast<const float2 *>(wt) + (long long)t * C2 + c2) : make_float2(0.f, 0.f);
  const float2 b = on ? __ldg(reinterpret_cast<const float2 *>(bias) + c2) : make_float2(0.f, 0.f);
  __syncthreads();
  const float2 *x = reinterpret_cast<const float2 *>(xp + win * xws) + c2;
  float2 *o = reinterpret_cast<float2 *>(out + win * ows) + c2;
  const int cs = C2, rs = (W + 2 * h) * C2;  // pair strides of a pixel and an input row
  float sm0 = 0.f, sm1 = 0.f;
  const int nch = (Ho + CR - 1) / CR;
  for (int ci = 0; ci <= nch; ci++) {
    if (!summer) {
      for (int r = 0; r < RT; r++) {
        const int yl = threadIdx.y * RT + r, oy = ci * CR + yl;  // row yl of the chunk
        if (ci < nch && on && oy < Ho) {
          const float2 *xr = x + (long long)(oy * S - pt + h) * rs;
          float2 *orow = o + (long long)oy * Wo * cs;
          float2 *g = sg + (ci & 1) * tile + yl * nu * Lc + lane;
          int ox = 0, gi = 0;
          for (; ox + 4 <= Wo; ox += 4, gi++)
            g[gi * Lc] = dwk2_unit<K, S, 4>(xr + (long long)(ox * S - pl + h) * cs, rs, cs, ws + lane, Lc, b, act, lut,
                                            orow + ox * cs, cs);
          for (; ox < Wo; ox++, gi++)
            g[gi * Lc] = dwk2_unit<K, S, 1>(xr + (long long)(ox * S - pl + h) * cs, rs, cs, ws + lane, Lc, b, act, lut,
                                            orow + ox * cs, cs);
        }
      }
    } else if (ci > 0 && on) {  // the previous chunk's addends, row order then unit order
      const float2 *gs = sg + ((ci - 1) & 1) * tile + lane;
      const int n = min(CR, Ho - (ci - 1) * CR) * nu;
      for (int i = 0; i < n; i++) {
        const float2 r = gs[i * Lc];
        sm0 = __fadd_rn(sm0, r.x);
        sm1 = __fadd_rn(sm1, r.y);
      }
    }
    __syncthreads();
  }
  if (summer && on) {
    chsum[win * cws + 2 * c2] = sm0;
    chsum[win * cws + 2 * c2 + 1] = sm1;
  }
}

// ------------------------------------------------------------------ the fp32 GEMM with a patch source

// Rows of A: PLAIN, row m of window w at A + w aws + m lda; PATCH (CONVK / gemm_f32_seg), output pixel m = (oy, ox)
// reads nseg segments of segk floats, segment g at A + w aws + ((oy s + oy0 + g) Wp + ox0 + ox s) ld; IM2COL (STEM),
// k x k taps of a 1-channel image [H][W] (zero past K up to Kp).
enum { kSrcPlain = 0, kSrcPatch = 1, kSrcIm2col = 2, kSrcGated = 3 };
struct F32GemmArgs {
  const float *A;
  long long aws;
  int lda, M;
  // patch / im2col geometry
  int Wo, s, oy0, ox0, Wp, ld, nseg, segk, k, Wimg;
  // the SE gate of a gated 1x1 conv: gate + w gws [Kp], applied to A as the GEMM reads it (one rounded product)
  const float *gate;
  long long gws;
  // weights [Np/8][Kp][8], bias [Np]
  const float *w, *bias;
  int Kp, Np;
  // epilogue (epi32): act, output rows at out + w ows + orow(m) ldo, residual rows at res + w rws + rrow(m) ldr
  int act;
  float *out;
  long long ows;
  int ldo, ow, opad;
  const float *res;
  long long rws;
  int ldr, rw, rpad;
  int vec;  // the tiled form's output (and residual) rows take VW-float vector accesses
};

__device__ __forceinline__ long long pad_row(int m, int w, int pad) {
  return pad ? (long long)((m / w) + pad) * (w + 2 * pad) + (m % w) + pad : (long long)m;
}

// thread (row m, panel p): the panel's 8 accumulators over k ascending. A warp takes 32 consecutive rows of one panel
// (the panel's weights are the same address across the warp).
template <int SRC>
__global__ void __launch_bounds__(256) k_gemm_f32(const F32GemmArgs g) {
  __shared__ uint32_t lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = g_frecpe_lut[i];
  __syncthreads();
  const int npan = g.Np >> 3;
  const int m = blockIdx.x * 32 + (threadIdx.x & 31);
  const int p = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int w = blockIdx.z;
  if (m >= g.M || p >= npan) return;
  const float *wp = g.w + (long long)p * g.Kp * 8;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; j++) acc[j] = 0.f;
  auto step = [&](float a, int kidx) {
    const float4 w0 = __ldg(reinterpret_cast<const float4 *>(wp + (long long)kidx * 8));
    const float4 w1 = __ldg(reinterpret_cast<const float4 *>(wp + (long long)kidx * 8 + 4));
    acc[0] = __fmaf_rn(w0.x, a, acc[0]); acc[1] = __fmaf_rn(w0.y, a, acc[1]);
    acc[2] = __fmaf_rn(w0.z, a, acc[2]); acc[3] = __fmaf_rn(w0.w, a, acc[3]);
    acc[4] = __fmaf_rn(w1.x, a, acc[4]); acc[5] = __fmaf_rn(w1.y, a, acc[5]);
    acc[6] = __fmaf_rn(w1.z, a, acc[6]); acc[7] = __fmaf_rn(w1.w, a, acc[7]);
  };
  const float *Aw = g.A + w * g.aws;
  if (SRC == kSrcPlain) {
    const float *ar = Aw + (long long)m * g.lda;
    for (int kk = 0; kk < g.Kp; kk++) step(__ldg(ar + kk), kk);
  } else if (SRC == kSrcGated) {
    const float *ar = Aw + (long long)m * g.lda, *gr = g.gate + w * g.gws;
    for (int kk = 0; kk < g.Kp; kk++) step(__fmul_rn(__ldg(ar + kk), __ldg(gr + kk)), kk);
  } else if (SRC == kSrcPatch) {
    const int oy = m / g.Wo, ox = m - oy * g.Wo;
    int kk = 0;
    for (int sg = 0; sg < g.nseg; sg++) {
      const float *ar = Aw + ((long long)(oy * g.s + g.oy0 + sg) * g.Wp + g.ox0 + ox * g.s) * g.ld;
      for (int r = 0; r < g.segk; r++, kk++) step(__ldg(ar + r), kk);
    }
  } else {  // im2col of a 1-channel image, zero past the k x k taps
    const int oy = m / g.Wo, ox = m - oy * g.Wo;
    for (int kk = 0; kk < g.Kp; kk++) {
      float a = 0.f;
      if (kk < g.k * g.k) {
        const int ky = kk / g.k, kx = kk - ky * g.k;
        a = __ldg(Aw + (long long)(oy * g.s + ky) * g.Wimg + ox * g.s + kx);
      }
      step(a, kk);
    }
  }
  float *o = g.out + w * g.ows + pad_row(m, g.ow, g.opad) * g.ldo + 8 * p;
  const float *rr = g.res ? g.res + w * g.rws + pad_row(m, g.rw, g.rpad) * g.ldr + 8 * p : nullptr;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    float y = act32(__fadd_rn(acc[j], __ldg(g.bias + 8 * p + j)), g.act, lut);
    if (rr) y = __fadd_rn(y, __ldg(rr + j));
    o[j] = y;
  }
}

template <int SRC>
static int launch_gemm_f32(int B, const F32GemmArgs &g, bnn_stream_t st) {
  if (B <= 0 || g.M <= 0) return 0;
  const dim3 grid((unsigned)((g.M + 31) / 32), (unsigned)((g.Np / 8 + 7) / 8), (unsigned)B);
  k_gemm_f32<SRC><<<grid, 256, 0, st>>>(g);
  return cudaGetLastError();
}

// Register-tiled form of the same product for row-major sources (PLAIN, GATED) and STEM's im2col rows (read from the
// image tap by tap, zero past the k x k taps): the B windows' rows are one [B M] x Np product; a CTA of 256 threads computes BM = 16 TM rows x BN = 16 TN columns of it. Thread (ty, tx) =
// (tid / 16, tid % 16) holds rows ty 4 + 64 i + r (i < TM / 4, r < 4) and columns tx 4 + 64 j + c (j < TN / 4,
// c < 4; TN = 2: columns 2 tx, 2 tx + 1), so that a warp's shared-memory reads of A are broadcasts and its reads of
// B cover contiguous 16-byte chunks. K advances in steps of 16 through two shared-memory stages: the next step's
// global loads are in flight while the current one is multiplied; A is stored k-major (the SE gate applied as it is
// staged: one rounded product per element, as the reference forms it). Every accumulator still starts at +0 and
// takes its Kp fused multiply-adds in k order, so the results equal the per-thread form's bit for bit.
constexpr int kTK = 16;

template <int TM, int TN, int SRC>
__global__ void __launch_bounds__(256, TM == 4 ? 4 : 2) k_gemm_f32t(const F32GemmArgs g, int rows, int n_tiles) {
  constexpr bool GATED = SRC == kSrcGated, IM2COL = SRC == kSrcIm2col;
  constexpr int BM = 16 * TM, BN = 16 * TN, AP = BM + 4;
  constexpr int AV = BM / 64;                   // float4 loads of A (and of the gate) per thread per step
  constexpr int BV = BN / 64 > 0 ? BN / 64 : 1;  // float4 loads of B per thread per step (BN = 32: threads < 128)
  __shared__ __align__(16) float As[2][kTK][AP];
  __shared__ __align__(16) float Bs[2][kTK][BN];
  __shared__ uint32_t lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = g_frecpe_lut[i];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int nt = blockIdx.x % n_tiles, mt = blockIdx.x / n_tiles;
  const int n0 = nt * BN;
  const long long r0 = (long long)mt * BM;
  const int Kp = g.Kp;

  // this thread's A rows for staging: row r0 + tid / 4 + 64 v, k quad tid % 4
  const float *arow[AV];  // nullptr past the last row
  int awin[GATED ? AV : 1];
#pragma unroll
  for (int v = 0; v < AV; v++) {
    const long long r = r0 + tid / 4 + 64 * v;
    arow[v] = nullptr;
    if (r < rows) {
      const int w = (int)(r / g.M), m = (int)(r - (long long)w * g.M);
      if (IM2COL) {  // the patch's first tap of the 1-channel image
        const int oy = m / g.Wo, ox = m - oy * g.Wo;
        arow[v] = g.A + w * g.aws + (long long)(oy * g.s) * g.Wimg + ox * g.s;
      } else {
        arow[v] = g.A + w * g.aws + (long long)m * g.lda + 4 * (tid % 4);
      }
      if (GATED) awin[v] = w;
    }
  }
  // this thread's B quads: k = q / (BN / 4), column n0 + 4 (q % (BN / 4)) for q = tid + 256 v
  const float *bsrc = g.w + (long long)((n0 + 4 * (tid % (BN / 4))) / 8) * Kp * 8 + (long long)(tid / (BN / 4)) * 8 +
                      (4 * (tid % (BN / 4))) % 8;
  const bool bon = tid < kTK * BN / 4 / BV && n0 + 4 * (tid % (BN / 4)) < g.Np;
  float4 ra[AV], rg[GATED ? AV : 1], rb[BV];
  auto load = [&](int k0) {
    const int ka = k0 + 4 * (tid % 4);
#pragma unroll
    for (int v = 0; v < AV; v++) {
      const bool on = arow[v] && ka < Kp;
      if (IM2COL) {  // taps ka .. ka + 3 of the k x k patch, zero past them
        float t[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int kk = ka + j, ky = kk / g.k;
          t[j] = on && kk < g.k * g.k ? __ldg(arow[v] + (long long)ky * g.Wimg + (kk - ky * g.k)) : 0.f;
        }
        ra[v] = make_float4(t[0], t[1], t[2], t[3]);
        continue;
      }
      ra[v] = on ? __ldg(reinterpret_cast<const float4 *>(arow[v] + k0)) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (GATED)
        rg[v] = on ? __ldg(reinterpret_cast<const float4 *>(g.gate + awin[v] * g.gws + ka))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int v = 0; v < BV; v++) {  // quad q = tid + 256 v: k row q / (BN / 4) = tid / (BN / 4) + 256 v / (BN / 4)
      const int kk = tid / (BN / 4) + 256 * v / (BN / 4);
      rb[v] = bon && k0 + kk < Kp ? __ldg(reinterpret_cast<const float4 *>(bsrc + (long long)(k0 + 256 * v / (BN / 4)) * 8))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stage = [&](int s) {
#pragma unroll
    for (int v = 0; v < AV; v++) {
      float4 t = ra[v];
      if (GATED) {
        t.x = __fmul_rn(t.x, rg[v].x); t.y = __fmul_rn(t.y, rg[v].y);
        t.z = __fmul_rn(t.z, rg[v].z); t.w = __fmul_rn(t.w, rg[v].w);
      }
      const int m = tid / 4 + 64 * v, k = 4 * (tid % 4);
      As[s][k][m] = t.x; As[s][k + 1][m] = t.y; As[s][k + 2][m] = t.z; As[s][k + 3][m] = t.w;
    }
#pragma unroll
    for (int v = 0; v < BV; v++) {
      const int q = tid + 256 * v;
      if (q < kTK * BN / 4) *reinterpret_cast<float4 *>(&Bs[s][q / (BN / 4)][4 * (q % (BN / 4))]) = rb[v];
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

  const int nk = (Kp + kTK - 1) / kTK;
  load(0);
  stage(0);
  __syncthreads();
  for (int kt = 0; kt < nk; kt++) {
    const int s = kt & 1;
    if (kt + 1 < nk) load((kt + 1) * kTK);
    const int kn = Kp - kt * kTK < kTK ? Kp - kt * kTK : kTK;  // block-uniform: only the last step can be short
    auto body = [&](int kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM / 4; i++) {
        const float4 t = *reinterpret_cast<const float4 *>(&As[s][kk][4 * ty + 64 * i]);
        a[4 * i] = t.x; a[4 * i + 1] = t.y; a[4 * i + 2] = t.z; a[4 * i + 3] = t.w;
      }
      if (TN == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(&Bs[s][kk][2 * tx]);
        b[0] = t.x; b[TN - 1] = t.y;
      } else {
#pragma unroll
        for (int j = 0; j < TN / 4; j++) {
          const float4 t = *reinterpret_cast<const float4 *>(&Bs[s][kk][4 * tx + 64 * j]);
          b[4 * j] = t.x; b[4 * j + 1] = t.y; b[4 * j + 2] = t.z; b[4 * j + 3] = t.w;
        }
      }
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = __fmaf_rn(b[j], a[i], acc[i][j]);
    };
    if (kn == kTK) {
#pragma unroll
      for (int kk = 0; kk < kTK; kk++) body(kk);
    } else {
      for (int kk = 0; kk < kn; kk++) body(kk);
    }
    if (kt + 1 < nk) stage(s ^ 1);
    __syncthreads();
  }

  // epilogue (epi32): + bias, activation, residual, the padded output row
  // a thread's columns come in runs of VW (2 for TN = 2, else 4) that are stored (and read from the residual) as one
  // vector when g.vec allows it (rows, window strides and base pointers aligned to VW floats)
  constexpr int VW = TN == 2 ? 2 : TN == 8 ? 1 : 4;
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const long long r = r0 + 4 * ty + 64 * (i / 4) + (i % 4);
    if (r >= rows) continue;
    const int w = (int)(r / g.M), m = (int)(r - (long long)w * g.M);
    float *orow = g.out + w * g.ows + pad_row(m, g.ow, g.opad) * g.ldo;
    const float *rrow = g.res ? g.res + w * g.rws + pad_row(m, g.rw, g.rpad) * g.ldr : nullptr;
#pragma unroll
    for (int jg = 0; jg < TN / VW; jg++) {
      const int n = TN == 2 ? n0 + 2 * tx : VW == 1 ? n0 + 4 * tx + 64 * (jg / 4) + (jg % 4) : n0 + 4 * tx + 64 * jg;
      if (n >= g.Np) continue;  // Np % 8 == 0: a run is wholly inside or outside
      float y[VW], rv[VW];
#pragma unroll
      for (int v = 0; v < VW; v++) y[v] = act32(__fadd_rn(acc[i][VW * jg + v], __ldg(g.bias + n + v)), g.act, lut);
      if (rrow) {
        if (g.vec && VW == 2) {
          const float2 t = __ldg(reinterpret_cast<const float2 *>(rrow + n));
          rv[0] = t.x; rv[VW - 1] = t.y;
        } else if (g.vec) {
          const float4 t = __ldg(reinterpret_cast<const float4 *>(rrow + n));
          rv[0] = t.x; rv[1 % VW] = t.y; rv[2 % VW] = t.z; rv[3 % VW] = t.w;
        } else {
#pragma unroll
          for (int v = 0; v < VW; v++) rv[v] = __ldg(rrow + n + v);
        }
#pragma unroll
        for (int v = 0; v < VW; v++) y[v] = __fadd_rn(y[v], rv[v]);
      }
      if (g.vec && VW == 2) {
        *reinterpret_cast<float2 *>(orow + n) = make_float2(y[0], y[VW - 1]);
      } else if (g.vec) {
        *reinterpret_cast<float4 *>(orow + n) = make_float4(y[0], y[1 % VW], y[2 % VW], y[3 % VW]);
      } else {
#pragma unroll
        for (int v = 0; v < VW; v++) orow[n + v] = y[v];
      }
    }
  }
}

// the tile width with the least padded work, counting the narrower tiles' extra shared-memory reads per FMA: a
// 128-wide tile (8 x 8 per thread) at full rate, 64 (8 x 4) at 0.8, 32 (16 x 2) at 0.6 (a 96-channel layer on
// 32-wide tiles ran at half the FMA rate of the 128-wide ones)
template <int SRC>
static int launch_gemm_f32t(int B, const F32GemmArgs &g, bnn_stream_t st) {
  const long long rows = (long long)B * g.M;
  const double c128 = (g.Np + 127) / 128 * 128, c64 = (g.Np + 63) / 64 * 64 / 0.8, c32 = (g.Np + 31) / 32 * 32 / 0.6;
  const int bn = c128 <= c64 && c128 <= c32 ? 128 : c64 <= c32 ? 64 : 32;
  // narrow layers with short rows (K <= 64: a few multiply-adds per loaded byte) are bound by memory latency, not
  // by the FMA pipe: 64-row tiles, few registers, many CTAs per SM
  const bool small = bn == 32 && g.Kp <= 64;
  const int bm = small ? 64 : bn == 32 ? 256 : 128;
  const int nt = (g.Np + bn - 1) / bn;
  const long long blocks = (rows + bm - 1) / bm * nt;
  if (rows > 0x7fffffffLL || blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  const int vw = bn == 32 ? 2 : 4;  // the epilogue's run of columns per thread
  auto al = [vw](const void *p, long long ws, int ld) { return ((uintptr_t)p & (4 * vw - 1)) == 0 && ws % vw == 0 && ld % vw == 0; };
  F32GemmArgs gv = g;
  // (the 128-wide tile keeps scalar accesses: its 64 accumulators leave no registers for vectors)
  gv.vec = bn < 128 && al(g.out, g.ows, g.ldo) && (!g.res || al(g.res, g.rws, g.ldr));
  if (small) k_gemm_f32t<4, 2, SRC><<<(unsigned)blocks, 256, 0, st>>>(gv, (int)rows, nt);
  else if (bn == 128) k_gemm_f32t<8, 8, SRC><<<(unsigned)blocks, 256, 0, st>>>(gv, (int)rows, nt);
  else if (bn == 64) k_gemm_f32t<8, 4, SRC><<<(unsigned)blocks, 256, 0, st>>>(gv, (int)rows, nt);
  else k_gemm_f32t<16, 2, SRC><<<(unsigned)blocks, 256, 0, st>>>(gv, (int)rows, nt);
  return cudaGetLastError();
}

// row-major sources take the tiled form when its 16-byte loads are aligned
static bool f32t_ok(const F32GemmArgs &g) {
  return ((uintptr_t)g.A & 15) == 0 && g.aws % 4 == 0 && g.lda % 4 == 0 && ((uintptr_t)g.w & 15) == 0 &&
         g.Np % 8 == 0 && g.Kp % 4 == 0 && (!g.gate || (((uintptr_t)g.gate & 15) == 0 && g.gws % 4 == 0));
}

// STEM's im2col rows (pc_im2col1), written to the op's column buffer as the reference writes them
__global__ void k_im2col1(int W, int k, int s, int Ho, int Wo, int Kp, const float *__restrict__ img, long long iws,
                          float *__restrict__ col, long long cws) {
  const long long n = (long long)Ho * Wo * Kp;
  const int w = blockIdx.y;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / Kp;
    const int q = (int)(i - m * Kp), oy = (int)(m / Wo), ox = (int)(m - (long long)oy * Wo);
    float v = 0.f;
    if (q < k * k) {
      const int ky = q / k, kx = q - ky * k;
      v = img[w * iws + (long long)(oy * s + ky) * W + ox * s + kx];
    }
    col[w * cws + i] = v;
  }
}

// ------------------------------------------------------------------ CONVW: Winograd F(4x4, 3x3) (wino_f32.c)

// B^T applied to a column of 6 values (BT_COL)
__device__ __forceinline__ void bt_col(const float d[6], float o[6]) {
  const float t4 = __fsub_rn(d[4], __fmul_rn(d[2], 4.f)), t3 = __fsub_rn(d[3], __fmul_rn(d[1], 4.f));
  const float u4 = __fsub_rn(d[4], d[2]), u3 = __fmul_rn(__fsub_rn(d[3], d[1]), 2.f);
  o[0] = __fadd_rn(__fsub_rn(__fmul_rn(d[0], 4.f), __fmul_rn(d[2], 5.f)), d[4]);
  o[1] = __fadd_rn(t4, t3);
  o[2] = __fsub_rn(t4, t3);
  o[3] = __fadd_rn(u4, u3);
  o[4] = __fsub_rn(u4, u3);
  o[5] = __fadd_rn(__fsub_rn(__fmul_rn(d[1], 4.f), __fmul_rn(d[3], 5.f)), d[5]);
}
// A^T applied to 6 values (AT_COL)
__device__ __forceinline__ void at_col(const float m[6], float y[4]) {
  const float a12 = __fadd_rn(m[1], m[2]), s12 = __fsub_rn(m[1], m[2]);
  const float a34 = __fadd_rn(m[3], m[4]), s34 = __fsub_rn(m[3], m[4]);
  y[0] = __fadd_rn(__fadd_rn(m[0], a12), a34);
  y[1] = __fadd_rn(s12, __fmul_rn(s34, 2.f));
  y[2] = __fadd_rn(a12, __fmul_rn(a34, 4.f));
  y[3] = __fadd_rn(__fadd_rn(s12, __fmul_rn(s34, 8.f)), m[5]);
}

// V [window][tile][36][C]: thread (window, tile, channel); the 6x6 patch at (4 ty - 1 + h, 4 tx - 1 + h) of the haloed
// input, zero outside the buffer
__global__ void k_wino_in(int H, int W, int C, int h, int TW, int T, const float *__restrict__ xp, long long xws,
                          float *__restrict__ V) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const int win = blockIdx.y;
  if (i >= (long long)T * C) return;
  const int tile = (int)(i / C), c = (int)(i - (long long)tile * C);
  const int ty = tile / TW, tx = tile - ty * TW, Wp = W + 2 * h, Hp = H + 2 * h;
  const int y0 = 4 * ty - 1 + h, x0 = 4 * tx - 1 + h;
  float d[6][6], t[6][6];
  for (int a = 0; a < 6; a++)
    for (int b = 0; b < 6; b++) {
      const int y = y0 + a, x = x0 + b;
      d[a][b] = (y >= 0 && y < Hp && x >= 0 && x < Wp) ? __ldg(xp + win * xws + ((long long)y * Wp + x) * C + c) : 0.f;
    }
  for (int j = 0; j < 6; j++) {  // columns: t = B^T d
    float col[6], o[6];
    for (int a = 0; a < 6; a++) col[a] = d[a][j];
    bt_col(col, o);
    for (int a = 0; a < 6; a++) t[a][j] = o[a];
  }
  float *v = V + ((long long)win * T + tile) * 36 * C + c;
  for (int a = 0; a < 6; a++) {  // rows: V = t B
    float o[6];
    bt_col(t[a], o);
    for (int b = 0; b < 6; b++) v[(long long)(a * 6 + b) * C] = o[b];
  }
}

// M [window][tile][36][Np]: thread (window, tile, point, panel) with the panel's 8 accumulators over the channels, then
// + 0.0 (pt_tile); U [36][Np/8][C][8]
__global__ void k_wino_gemm(int C, int Np, int T, const float *__restrict__ V, const float *__restrict__ U,
                            float *__restrict__ Mb) {
  const int npan = Np >> 3;
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const int win = blockIdx.y;
  if (i >= (long long)T * 36 * npan) return;
  const int p = (int)(i % npan);
  const long long r = i / npan;
  const int xi = (int)(r % 36), tile = (int)(r / 36);
  const float *v = V + ((long long)win * T + tile) * 36 * C + (long long)xi * C;
  const float *u = U + ((long long)xi * npan + p) * C * 8;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; j++) acc[j] = 0.f;
  for (int c = 0; c < C; c++) {
    const float a = __ldg(v + c);
    const float4 w0 = __ldg(reinterpret_cast<const float4 *>(u + (long long)c * 8));
    const float4 w1 = __ldg(reinterpret_cast<const float4 *>(u + (long long)c * 8 + 4));
    acc[0] = __fmaf_rn(w0.x, a, acc[0]); acc[1] = __fmaf_rn(w0.y, a, acc[1]);
    acc[2] = __fmaf_rn(w0.z, a, acc[2]); acc[3] = __fmaf_rn(w0.w, a, acc[3]);
    acc[4] = __fmaf_rn(w1.x, a, acc[4]); acc[5] = __fmaf_rn(w1.y, a, acc[5]);
    acc[6] = __fmaf_rn(w1.z, a, acc[6]); acc[7] = __fmaf_rn(w1.w, a, acc[7]);
  }
  float *m = Mb + (((long long)win * T + tile) * 36 + xi) * Np + 8 * p;
#pragma unroll
  for (int j = 0; j < 8; j++) m[j] = __fadd_rn(acc[j], 0.f);
}

// the output tile (out_tile): thread (window, tile, channel n < Np)
__global__ void k_wino_out(int Ho, int Wo, int Np, int TW, int T, const float *__restrict__ Mb,
                           const float *__restrict__ bias, int act, const float *__restrict__ res, long long rws,
                           int rh, int rld, float *__restrict__ out, long long ows, int ldo, int opad) {
  __shared__ uint32_t lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = g_frecpe_lut[i];
  __syncthreads();
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const int win = blockIdx.y;
  if (i >= (long long)T * Np) return;
  const int tile = (int)(i / Np), n = (int)(i - (long long)tile * Np);
  const int ty = tile / TW, tx = tile - ty * TW;
  const int ny = Ho - 4 * ty < 4 ? Ho - 4 * ty : 4, nx = Wo - 4 * tx < 4 ? Wo - 4 * tx : 4;
  const float *m = Mb + ((long long)win * T + tile) * 36 * Np + n;
  float t[4][6];
  for (int j = 0; j < 6; j++) {
    float col[6], y[4];
    for (int a = 0; a < 6; a++) col[a] = m[(long long)(a * 6 + j) * Np];
    at_col(col, y);
    for (int a = 0; a < 4; a++) t[a][j] = y[a];
  }
  const float bv = __ldg(bias + n);
  const int Wop = Wo + 2 * opad;
  for (int a = 0; a < ny; a++) {
    float y[4];
    at_col(t[a], y);
    for (int b = 0; b < nx; b++) {
      float v = act32(__fadd_rn(y[b], bv), act, lut);
      if (res) v = __fadd_rn(v, __ldg(res + win * rws + ((long long)(4 * ty + a + rh) * (Wo + 2 * rh) + 4 * tx + b + rh) * rld + n));
      out[win * ows + ((long long)(4 * ty + a + opad) * Wop + 4 * tx + b + opad) * ldo + n] = v;
    }
  }
}

// ------------------------------------------------------------------ SED (rt_ops_f32x.c:200-349)

// axis mean and pooling (rt_sed_pool) for one window: thread per channel; s and pooled [L8][Cp], their pad channels
// [C, Cp) zero for the L rows (sed_run)
__global__ void k_sed_pool(int red, int H, int W, int C, int ld, int L, int pk, int dk, int Cp,
                           const float *__restrict__ x, long long xws, const float *__restrict__ dw,
                           const float *__restrict__ db, float *__restrict__ s, long long sws, float *__restrict__ pl,
                           long long pws) {
  const int w = blockIdx.y;
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= Cp) return;
  float *sw = s + w * sws, *pw = pl + w * pws;
  if (ch >= C) {
    for (int t = 0; t < L; t++) { sw[(long long)t * Cp + ch] = 0.f; pw[(long long)t * Cp + ch] = 0.f; }
    return;
  }
  const int n = red == 3 ? W : H;
  const float *xw = x + w * xws;
  for (int t = 0; t < L; t++) {
    float a = 0.f;
    for (int u = 0; u < n; u++)
      a = __fadd_rn(a, __ldg(xw + (red == 3 ? ((long long)t * W + u) : ((long long)u * W + t)) * ld + ch));
    sw[(long long)t * Cp + ch] = __fdiv_rn(a, (float)n);
  }
  for (int t = 0; t < L; t++) {
    float m = -INFINITY, cv = 0.f;
    for (int d = 0; d < pk; d++) {
      const int u = t + d - pk / 2;
      if (u >= 0 && u < L) m = fmaxf(m, sw[(long long)u * Cp + ch]);
    }
    for (int d = 0; d < dk; d++) {
      const int u = t + d - dk / 2;
      if (u >= 0 && u < L) cv = __fadd_rn(cv, __fmul_rn(__ldg(dw + (long long)d * C + ch), sw[(long long)u * Cp + ch]));
    }
    if (dk) cv = __fadd_rn(cv, __ldg(db + ch));
    pw[(long long)t * Cp + ch] = pk && dk ? __fadd_rn(m, cv) : pk ? m : cv;
  }
}

// the attention softmax over time and the weighted class sum (rt_sed_out): thread per (window, class)
__global__ void k_sed_out(int B, int NC, int L, int hc, const float *__restrict__ kk, const float *__restrict__ att,
                          long long aws, int ldn, const float *__restrict__ cla, long long cws, int ldc,
                          float *__restrict__ out, long long ows) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)B * NC) return;
  const int w = (int)(i / NC), k = (int)(i - (long long)w * NC);
  const float lo = kk[0], hi = kk[1], sc = kk[2];
  const float *aw = att + w * aws + k, *cw = cla + w * cws + k;
  auto val = [&](int t) {
    float v = aw[(long long)t * ldn];
    if (hc) v = v < lo ? lo : v > hi ? hi : v;
    return v;
  };
  float mx = -INFINITY, z = 0.f, acc = 0.f;
  for (int t = 0; t < L; t++) mx = fmaxf(mx, val(t));
  for (int t = 0; t < L; t++) z = __fadd_rn(z, glibc_expf(__fsub_rn(val(t), mx), c_expf_tab));
  for (int t = 0; t < L; t++) {
    const float a = glibc_expf(__fsub_rn(val(t), mx), c_expf_tab);
    acc = __fadd_rn(acc, __fmul_rn(__fdiv_rn(a, z), cw[(long long)t * ldc]));
  }
  out[w * ows + k] = __fmul_rn(acc, sc);
}

}  // namespace bnn

using namespace bnn;

extern "C" int bnnk_v3_tables_init(const unsigned long long *tab, const uint32_t *lut) {
  cudaError_t e = cudaMemcpyToSymbol(c_expf_tab, tab, sizeof(unsigned long long) * 32);
  if (e) return e;
  return cudaMemcpyToSymbol(g_frecpe_lut, lut, sizeof(uint32_t) * 256);
}

static unsigned cdiv(long long n, int d) { return (unsigned)((n + d - 1) / d); }

extern "C" int bnnk_vadd(int B, int n, const float *a, long long aws, const float *b, long long bws, float *o,
                         long long ows, bnn_stream_t st) {
  if (B <= 0 || n <= 0) return 0;
  k_vadd<<<dim3(cdiv(n, 256), (unsigned)B), 256, 0, st>>>(n, a, aws, b, bws, o, ows);
  return cudaGetLastError();
}

extern "C" int bnnk_gem(int B, int P, int C, int ld, const float *x, long long xws, const float *consts, float *out,
                        long long ows, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_gem<<<cdiv((long long)B * C, 128), 128, 0, st>>>(B, P, C, ld, x, xws, consts, out, ows);
  return cudaGetLastError();
}

extern "C" int bnnk_mean_f32(int B, int P, int C, int ld, const float *x, long long xws, float *out, long long ows,
                             bnn_stream_t st) {
  if (B <= 0) return 0;
  k_mean_f32<<<cdiv((long long)B * C, 128), 128, 0, st>>>(B, P, C, ld, x, xws, out, ows);
  return cudaGetLastError();
}

extern "C" int bnnk_pad_f32(int B, int H, int W, int C, int ld, int h, const float *x, long long xws, float *xp,
                            long long pws, bnn_stream_t st) {
  if (B <= 0) return 0;
  int rc = zero_halo(B, xp, pws, H, W, C, h, st);
  if (rc) return rc;
  const bool v4 = C % 4 == 0 && ld % 4 == 0 && xws % 4 == 0 && pws % 4 == 0 && ((uintptr_t)x & 15) == 0 &&
                  ((uintptr_t)xp & 15) == 0;
  const long long n = (long long)H * W * C / (v4 ? 4 : 1);
  const dim3 grid(cdiv(n, 256) < 1024 ? cdiv(n, 256) : 1024, (unsigned)B);
  if (v4) k_pad_f32<4><<<grid, 256, 0, st>>>(H, W, C, ld, h, x, xws, xp, pws);
  else k_pad_f32<1><<<grid, 256, 0, st>>>(H, W, C, ld, h, x, xws, xp, pws);
  return cudaGetLastError();
}

extern "C" int bnnk_dwk_f32(int B, const float *xp, long long xws, int H, int W, int C, int k, int s, int pt, int pl,
                            const float *w, const float *b, int act, float *out, long long ows, int Ho, int Wo,
                            float *chsum, long long cws, bnn_stream_t st) {
  (void)H;
  if (B <= 0) return 0;
  if ((k == 3 || k == 5 || k == 7) && (s == 1 || s == 2) && C % 2 == 0 && xws % 2 == 0 && ows % 2 == 0 &&
      ((uintptr_t)xp & 7) == 0 && ((uintptr_t)out & 7) == 0 && ((uintptr_t)w & 7) == 0 && ((uintptr_t)b & 7) == 0) {
    // the channel-pair form: up to 32 pairs per CTA, as many thread rows as fit 256 threads (one of them the summer)
    const int C2 = C / 2, Lc = C2 < 32 ? C2 : 32, nu = Wo / 4 + Wo % 4;
    int Ry = 256 / Lc - 1;
    if (Ry > Ho) Ry = Ho;
    if (Ry < 1) Ry = 1;
    // rows per thread and chunk: about 8 units of work between the chunk barriers, no more rows than the map has
    int RT = (8 + nu - 1) / nu;
    while (RT > 1 && Ry * RT > Ho + Ry - 1) RT--;
    auto smem_of = [&](int ry, int rt) { return (size_t)(k * k + 2 * ry * rt * nu) * Lc * 8; };
    while (RT > 1 && smem_of(Ry, RT) > 48 * 1024) RT--;
    while (Ry > 1 && smem_of(Ry, RT) > 48 * 1024) Ry--;
    const size_t smem = smem_of(Ry, RT);
    if (smem <= 96 * 1024) {
      const dim3 grid((unsigned)((C2 + Lc - 1) / Lc), (unsigned)B), blk((unsigned)Lc, (unsigned)(Ry + 1));
#define BNN_DWK2(KK, SS)                                                                                        \
  do {                                                                                                          \
    static SmemAttr attr_;                                                                                      \
    const cudaError_t e_ = attr_.ensure(k_dwk2_f32<KK, SS>, smem);                                             \
    if (e_) return e_;                                                                                          \
    k_dwk2_f32<KK, SS><<<grid, blk, smem, st>>>(xp, xws, W, C, pt, pl, w, b, act, out, ows, Ho, Wo, nu, RT, chsum,  \
                                               cws);                                                            \
  } while (0)
      if (k == 3) { if (s == 1) BNN_DWK2(3, 1); else BNN_DWK2(3, 2); }
      else if (k == 5) { if (s == 1) BNN_DWK2(5, 1); else BNN_DWK2(5, 2); }
      else { if (s == 1) BNN_DWK2(7, 1); else BNN_DWK2(7, 2); }
#undef BNN_DWK2
      return cudaGetLastError();
    }
  }
  k_dwk_f32<<<cdiv((long long)B * C, 128), 128, 0, st>>>(B, W, C, k, s, pt, pl, xp, xws, w, b, act, out, ows, Ho, Wo,
                                                         chsum, cws);
  return cudaGetLastError();
}

extern "C" int bnnk_pw_f32(int B, const float *x, long long xws, int lda, int M, const float *gate, long long gws,
                           const float *w, const float *bias, int Kp, int Np, int act, float *out, long long ows,
                           int ldo, int ow, int opad, int oH, int oW, const float *res, long long rws, int ldr, int rw,
                           int rpad, bnn_stream_t st) {
  if (B <= 0) return 0;
  int rc = zero_halo(B, out, ows, oH, oW, ldo, opad, st);
  if (rc) return rc;
  F32GemmArgs g = {};
  g.A = x; g.aws = xws; g.lda = lda; g.M = M; g.gate = gate; g.gws = gws;
  g.w = w; g.bias = bias; g.Kp = Kp; g.Np = Np;
  g.act = act; g.out = out; g.ows = ows; g.ldo = ldo; g.ow = ow; g.opad = opad;
  g.res = res; g.rws = rws; g.ldr = ldr; g.rw = rw; g.rpad = rpad;
  if (f32t_ok(g)) return gate ? launch_gemm_f32t<kSrcGated>(B, g, st) : launch_gemm_f32t<kSrcPlain>(B, g, st);
  return gate ? launch_gemm_f32<kSrcGated>(B, g, st) : launch_gemm_f32<kSrcPlain>(B, g, st);
}

extern "C" int bnnk_stem_f32(int B, const float *img, long long iws, int W, int k, int s, int Ho, int Wo,
                             const float *w, const float *bias, int Kp, int Np, int act, float *out, long long ows,
                             int ldo, int opad, float *col, long long cws, bnn_stream_t st) {
  if (B <= 0) return 0;
  const long long n = (long long)Ho * Wo * Kp;
  if (col)  // the reference's im2col rows (pc_im2col1), for an op that reads them; the GEMM below reads the image
    k_im2col1<<<dim3(cdiv(n, 256) < 1024 ? cdiv(n, 256) : 1024, (unsigned)B), 256, 0, st>>>(W, k, s, Ho, Wo, Kp, img,
                                                                                           iws, col, cws);
  int rc = cudaGetLastError();
  if (!rc) rc = zero_halo(B, out, ows, Ho, Wo, ldo, opad, st);
  if (rc) return rc;
  F32GemmArgs g = {};
  g.A = img; g.aws = iws; g.M = Ho * Wo; g.Wo = Wo; g.s = s; g.k = k; g.Wimg = W;
  g.w = w; g.bias = bias; g.Kp = Kp; g.Np = Np;
  g.act = act; g.out = out; g.ows = ows; g.ldo = ldo; g.ow = Wo; g.opad = opad;
  if (((uintptr_t)w & 15) == 0 && Np % 8 == 0 && Kp % 4 == 0) return launch_gemm_f32t<kSrcIm2col>(B, g, st);
  return launch_gemm_f32<kSrcIm2col>(B, g, st);
}

extern "C" int bnnk_convk(int B, const float *x, long long xws, int H, int W, int h, int ld, int Ho, int Wo, int kh,
                          int kw, int s, int oy0, int ox0, const float *w, const float *bias, int Kp, int Np, int act,
                          float *out, long long ows, int ldo, int opad, const float *res, long long rws, int ldr, int rh,
                          bnn_stream_t st) {
  (void)H;
  if (B <= 0) return 0;
  int rc = zero_halo(B, out, ows, Ho, Wo, ldo, opad, st);
  if (rc) return rc;
  F32GemmArgs g = {};
  g.A = x; g.aws = xws; g.M = Ho * Wo; g.Wo = Wo; g.s = s; g.oy0 = oy0; g.ox0 = ox0; g.Wp = W + 2 * h; g.ld = ld;
  g.nseg = kh; g.segk = kw * ld;
  g.w = w; g.bias = bias; g.Kp = Kp; g.Np = Np;
  g.act = act; g.out = out; g.ows = ows; g.ldo = ldo; g.ow = Wo; g.opad = opad;
  g.res = res; g.rws = rws; g.ldr = ldr; g.rw = Wo; g.rpad = rh;
  return launch_gemm_f32<kSrcPatch>(B, g, st);
}

extern "C" size_t bnnk_convw_scratch_floats(int H, int W, int C, int Np) {
  const long long T = (long long)((H + 3) / 4) * ((W + 3) / 4);
  return (size_t)(T * 36 * C + T * 36 * Np);
}

extern "C" int bnnk_convw(int B, const float *x, long long xws, int H, int W, int h, int C, const float *U,
                          const float *bias, int Np, int act, float *out, long long ows, int ldo, int opad,
                          const float *res, long long rws, int rh, int rld, float *scratch, bnn_stream_t st) {
  if (B <= 0) return 0;
  const int TW = (W + 3) / 4, T = TW * ((H + 3) / 4);
  float *V = scratch, *Mb = scratch + (size_t)B * T * 36 * C;
  int rc = zero_halo(B, out, ows, H, W, ldo, opad, st);
  if (rc) return rc;
  k_wino_in<<<dim3(cdiv((long long)T * C, 128), (unsigned)B), 128, 0, st>>>(H, W, C, h, TW, T, x, xws, V);
  k_wino_gemm<<<dim3(cdiv((long long)T * 36 * (Np / 8), 128), (unsigned)B), 128, 0, st>>>(C, Np, T, V, U, Mb);
  k_wino_out<<<dim3(cdiv((long long)T * Np, 128), (unsigned)B), 128, 0, st>>>(H, W, Np, TW, T, Mb, bias, act, res,
                                                                               rws, rh, rld, out, ows, ldo, opad);
  return cudaGetLastError();
}

extern "C" int bnnk_sed_pool(int B, const bnnk_sed_args *a, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_sed_pool<<<dim3(cdiv(a->Cp, 128), (unsigned)B), 128, 0, st>>>(a->red, a->H, a->W, a->C, a->ld, a->L, a->pk, a->dk,
                                                                  a->Cp, a->x, a->xws, a->dw, a->db, a->s, a->sws,
                                                                  a->pl, a->pws);
  return cudaGetLastError();
}

extern "C" int bnnk_sed_out(int B, const bnnk_sed_args *a, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_sed_out<<<cdiv((long long)B * a->at.N, 128), 128, 0, st>>>(B, a->at.N, a->L, a->hc, a->consts, a->att, a->aws,
                                                                a->at.Np, a->cla, a->clws, a->cl.Np, a->out, a->ows);
  return cudaGetLastError();
}

extern "C" int bnnk_sed(int B, const bnnk_sed_args *a, bnn_stream_t st) {
  if (B <= 0) return 0;
  int rc = bnnk_sed_pool(B, a, st);
  if (rc) return rc;
  // the three GEMMs on the L rows of every window (rows past L of the 8-row tiles are neither read nor written)
  const float *src[3] = {a->pl, a->h, a->h};
  const long long sws[3] = {a->pws, a->hws, a->hws};
  const int lda[3] = {a->Cp, a->fc.Np, a->fc.Np};
  const bnnk_fpack *fp[3] = {&a->fc, &a->at, &a->cl};
  float *dst[3] = {a->h, a->att, a->cla};
  const long long dws[3] = {a->hws, a->aws, a->clws};
  for (int i = 0; i < 3 && !rc; i++) {
    F32GemmArgs g = {};
    g.A = src[i]; g.aws = sws[i]; g.lda = lda[i]; g.M = a->L;
    g.w = fp[i]->w; g.bias = fp[i]->b; g.Kp = fp[i]->Kp; g.Np = fp[i]->Np;
    g.act = i == 0 ? 2 : 0; g.out = dst[i]; g.ows = dws[i]; g.ldo = fp[i]->Np;
    rc = launch_gemm_f32<kSrcPlain>(B, g, st);
  }
  return rc ? rc : bnnk_sed_out(B, a, st);
}
