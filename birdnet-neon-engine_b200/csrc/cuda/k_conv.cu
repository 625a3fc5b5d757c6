// The fp32 ops of the v2.4 int8 package on CUDA cores: depthwise 3x3 + SiLU + channel sums (DW3), the SE gate
// (SE_GATE), the c0 conv + pool (C0POOL) and the post BN + pc conv + mean (POSTPC); the front end is in k_fe.cu. Also
// the fp32 stem of compiled models' fp16 path (STEM f16: fp32 math, fp16 output).
// Each output is computed with the reference's operations in the reference's order (fused where the NEON code fuses,
// rounded where it rounds), so the values are bit-identical; only the parallel schedule is ours, and no reference
// reduction is split across threads except where its order is restated exactly.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdlib.h>

#include "bnn_kernels.h"
#include "emu.cuh"
#include "smem_attr.cuh"
#include "sync.cuh"
#include "tc.cuh"

namespace bnn {

// ------------------------------------------------------------------ DW3 (src/gemm_f32.c:214-440)

// Depthwise 3x3 (pad 1, stride S) + SiLU + channel sums, one kernel. Per channel the three column partial sums of
// DW_ACC (gemm_f32.c:221-225): acc = b + w0 A0 + w3 A1 + w6 A2 (fused, in that order), acb = w1 B0 + w4 B1 + w7 B2,
// acd = w2 C0 + w5 C1 + w8 C2, out = SiLU(acc + (acb + acd)); then chsum[c] = ((0 + v_0) + v_1) + ... over the
// output pixels in raster order (silu_rows_f32, gemm_f32.c:303-328; dw_silu_row16 :342-365).
//
// One CTA per (window, group of 4 * cg4 channels) walks the output pixels in raster order, a chunk of nl * R pixels
// at a time: thread (lane, c4) computes R consecutive pixels of one output row for 4 channels (R > 1 shares the
// input columns of neighbouring taps; channel pairs go through sm_100's paired fp32 FMA and the paired SiLU), stores
// them, and leaves them in shared memory; after the barrier one thread per channel continues its channel's sum over
// the chunk in pixel order while the others compute the next chunk into the other buffer.
constexpr int kDwThreads = 256;

template <int S, int R>
__global__ void __launch_bounds__(kDwThreads) k_dw3(const float *__restrict__ xp, long long xws, int W, int C, int cg4,
                                                    int nl, const float *__restrict__ wt,
                                                    const float *__restrict__ bias, float *__restrict__ out,
                                                    long long ows, int Wo, int P, float *__restrict__ chsum,
                                                    long long cws) {
  extern __shared__ float sb[];  // [2][nl * R][4 * cg4]
  __shared__ uint32_t lut[256];
  const int tid = threadIdx.x;
  lut[tid] = g_frecpe_lut[tid];
  const int CG = 4 * cg4, ngroups = (C >> 2) / cg4;
  const int win = blockIdx.x / ngroups, grp = blockIdx.x - win * ngroups;
  const int c4l = tid % cg4, lane = tid / cg4;
  const bool comp = lane < nl;
  const int c = grp * CG + 4 * c4l, Wp = W + 2, chunk = nl * R;
  float2 w[9][2], b[2];
  if (comp) {
#pragma unroll
    for (int t = 0; t < 9; t++) {
      const float4 v = __ldg(reinterpret_cast<const float4 *>(wt + t * C + c));
      w[t][0] = make_float2(v.x, v.y);
      w[t][1] = make_float2(v.z, v.w);
    }
    const float4 v = __ldg(reinterpret_cast<const float4 *>(bias + c));
    b[0] = make_float2(v.x, v.y);
    b[1] = make_float2(v.z, v.w);
  }
  const float *xw = xp + win * xws + c;
  float *ow = out + win * ows + c;
  float cs = 0.f;
  __syncthreads();
  for (int k = 0, p0c = 0; p0c < P; k++, p0c += chunk) {
    float *buf = sb + (k & 1) * chunk * CG;
    const int p0 = p0c + lane * R;
    if (comp && p0 < P) {
      const int oy = p0 / Wo, ox = p0 - oy * Wo;  // R pixels of one row (Wo % R == 0)
      const float *q = xw + ((long long)(oy * S) * Wp + (long long)ox * S) * C;
      constexpr int NX = (R - 1) * S + 3;  // input columns the R pixels read
      float2 acc[R][2], acb[R][2], acd[R][2];
#pragma unroll
      for (int ky = 0; ky < 3; ky++) {
        float2 xin[NX][2];
#pragma unroll
        for (int j = 0; j < NX; j++) {
          const float4 v = __ldg(reinterpret_cast<const float4 *>(q + ((long long)ky * Wp + j) * C));
          xin[j][0] = make_float2(v.x, v.y);
          xin[j][1] = make_float2(v.z, v.w);
        }
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const float2 A = xin[r * S][h], Bv = xin[r * S + 1][h], Cv = xin[r * S + 2][h];
            if (ky == 0) {
              acc[r][h] = fma2_rn(w[0][h], A, b[h]);
              acb[r][h] = mul2_rn(w[1][h], Bv);
              acd[r][h] = mul2_rn(w[2][h], Cv);
            } else {
              acc[r][h] = fma2_rn(w[3 * ky][h], A, acc[r][h]);
              acb[r][h] = fma2_rn(w[3 * ky + 1][h], Bv, acb[r][h]);
              acd[r][h] = fma2_rn(w[3 * ky + 2][h], Cv, acd[r][h]);
            }
          }
      }
#pragma unroll
      for (int r = 0; r < R; r++) {
        const float2 y0 = silu2(add2_rn(acc[r][0], add2_rn(acb[r][0], acd[r][0])), lut);
        const float2 y1 = silu2(add2_rn(acc[r][1], add2_rn(acb[r][1], acd[r][1])), lut);
        const float4 v = make_float4(y0.x, y0.y, y1.x, y1.y);
        *reinterpret_cast<float4 *>(ow + (long long)(p0 + r) * C) = v;
        *reinterpret_cast<float4 *>(buf + (lane * R + r) * CG + 4 * c4l) = v;
      }
    }
    __syncthreads();
    if (tid < CG) {
      const int n = min(chunk, P - p0c);
      int i = 0;
      for (; i + 8 <= n; i += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = buf[(i + j) * CG + tid];
#pragma unroll
        for (int j = 0; j < 8; j++) cs = __fadd_rn(cs, v[j]);
      }
      for (; i < n; i++) cs = __fadd_rn(cs, buf[i * CG + tid]);
    }
  }
  if (chsum && tid < CG) chsum[win * cws + grp * CG + tid] = cs;
}

// The same DW3 with the input streamed by TMA. One CTA per (window, group of CG channels) walks the output rows:
// the haloed input rows (W + 2 pixels x CG channels each, one 3-D tensor-map box) pass through a ring of nr slots in
// shared memory (nr >= S + 3: the 3 rows of this step plus the S new rows of the next; every slot beyond those is
// one more row of lookahead, and a ring as deep as the window's rows loads them all up front), so every input byte
// is read from HBM once and no thread waits on a global load. Thread (lane, channel quad) keeps its
// quad's weights in registers and computes pixel groups lane, lane + NL, ... of the row (R consecutive pixels per
// group share their input columns), stores them and leaves them in a double-buffered row tile; after the step's
// barrier the first CG threads continue their channel's sum over the row in pixel order.
// Without the channel sums (kSum false: no op reads them in a whole-package run) the rows of a window are cut into
// nband bands of consecutive output rows, one CTA each, so that small batches still fill the GPU.
constexpr int kDw3MaxRing = 32;
template <int S, int R, bool kSum>
__global__ void __launch_bounds__(256) k_dw3t(const __grid_constant__ CUtensorMap tmx, int W, int C, int CG, int Ho,
                                              int Wo, int NR, const float *__restrict__ wt,
                                              const float *__restrict__ bias, float *__restrict__ out, long long ows,
                                              float *__restrict__ chsum, long long cws, int *err, int nband) {
  constexpr int NX = (R - 1) * S + 3;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) unsigned long long bar[kDw3MaxRing];
  __shared__ uint32_t lut[256];
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int i = tid; i < 256; i += nt) lut[i] = g_frecpe_lut[i];
  const int ngroups = C / CG;
  const int band = blockIdx.x % nband, wg = blockIdx.x / nband;
  const int win = wg / ngroups, grp = wg - win * ngroups;
  const int hb = (Ho + nband - 1) / nband, oy0 = band * hb, oy1 = min(Ho, oy0 + hb);
  if (oy0 >= oy1) return;  // an empty last band (the whole CTA leaves before any barrier)
  const int Wp = W + 2, Q = CG >> 2, NL = nt / Q, ngrp = Wo / R;
  const uint32_t row_bytes = (uint32_t)Wp * CG * 4, row_stride = (row_bytes + 127u) & ~127u;
  const uint32_t ring = smem_u32(dsm);
  const float *ringf = reinterpret_cast<const float *>(dsm);
  float *obuf = reinterpret_cast<float *>(dsm + NR * row_stride);  // [2][Wo][CG]
  const int q = tid % Q, lane = tid / Q;  // lanes >= NL (the last nt % Q threads) only sum
  const bool comp = lane < NL;
  const int c = grp * CG + 4 * q;
  float2 w[9][2], b[2];
#pragma unroll
  for (int t = 0; t < 9; t++) {
    const float4 v = comp ? __ldg(reinterpret_cast<const float4 *>(wt + t * C + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    w[t][0] = make_float2(v.x, v.y);
    w[t][1] = make_float2(v.z, v.w);
  }
  {
    const float4 v = comp ? __ldg(reinterpret_cast<const float4 *>(bias + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    b[0] = make_float2(v.x, v.y);
    b[1] = make_float2(v.z, v.w);
  }
  if (tid == 0) {
    for (int i = 0; i < NR; i++) mbar_init(smem_u32(&bar[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // ring rows are counted from the band's first input row iy0: local row l is input row iy0 + l
  const int iy0 = oy0 * S, rows_in = (oy1 - 1 - oy0) * S + 3;  // input rows the band's outputs read
  int issued = 0;                        // local rows whose load thread 0 has issued
  auto issue_to = [&](int last) {        // thread 0: load local rows issued .. last
    for (; issued <= last && issued < rows_in; issued++) {
      const int sl = issued % NR;
      mbar_expect_tx(smem_u32(&bar[sl]), row_bytes);
      tma_load_3d(ring + sl * row_stride, &tmx, smem_u32(&bar[sl]), grp * CG, (iy0 + issued) * Wp, win);
    }
  };
  if (tid == 0) issue_to(NR - 1);  // as many rows as the ring holds
  float cs = 0.f;
  int oy = oy0;
  for (; oy < oy1; oy++) {
    bool ok = true;
    int slot[3];
#pragma unroll
    for (int ky = 0; ky < 3; ky++) {
      const int iy = (oy - oy0) * S + ky;
      slot[ky] = iy % NR;
      ok = ok && mbar_wait(smem_u32(&bar[slot[ky]]), (uint32_t)(iy / NR) & 1u);
    }
    float *ob = obuf + (oy & 1) * Wo * CG;
    if (comp) {
      // groups in reverse lane order: when they do not divide evenly, the extra ones go to the high lanes, not to
      // the low threads that also add the row sums after the barrier
      for (int g = NL - 1 - lane; g < ngrp; g += NL) {
        const int x0 = g * R;
        float2 acc[R][2], acb[R][2], acd[R][2];
#pragma unroll
        for (int ky = 0; ky < 3; ky++) {
          const float *rw = ringf + slot[ky] * (row_stride >> 2) + (x0 * S) * CG + 4 * q;
          float4 xin[NX];
#pragma unroll
          for (int j = 0; j < NX; j++) xin[j] = *reinterpret_cast<const float4 *>(rw + j * CG);
#pragma unroll
          for (int r = 0; r < R; r++) {
            const float4 A4 = xin[r * S], B4 = xin[r * S + 1], C4 = xin[r * S + 2];
            const float2 A[2] = {make_float2(A4.x, A4.y), make_float2(A4.z, A4.w)};
            const float2 Bv[2] = {make_float2(B4.x, B4.y), make_float2(B4.z, B4.w)};
            const float2 Cv[2] = {make_float2(C4.x, C4.y), make_float2(C4.z, C4.w)};
#pragma unroll
            for (int h = 0; h < 2; h++) {
              if (ky == 0) {
                acc[r][h] = fma2_rn(w[0][h], A[h], b[h]);
                acb[r][h] = mul2_rn(w[1][h], Bv[h]);
                acd[r][h] = mul2_rn(w[2][h], Cv[h]);
              } else {
                acc[r][h] = fma2_rn(w[3 * ky][h], A[h], acc[r][h]);
                acb[r][h] = fma2_rn(w[3 * ky + 1][h], Bv[h], acb[r][h]);
                acd[r][h] = fma2_rn(w[3 * ky + 2][h], Cv[h], acd[r][h]);
              }
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float2 y0 = silu2(add2_rn(acc[r][0], add2_rn(acb[r][0], acd[r][0])), lut);
          const float2 y1 = silu2(add2_rn(acc[r][1], add2_rn(acb[r][1], acd[r][1])), lut);
          const float4 v = make_float4(y0.x, y0.y, y1.x, y1.y);
          *reinterpret_cast<float4 *>(out + win * ows + (long long)(oy * Wo + x0 + r) * C + c) = v;
          if (kSum) *reinterpret_cast<float4 *>(ob + (x0 + r) * CG + 4 * q) = v;
        }
      }
    }
    if (!__syncthreads_and(ok)) break;  // every thread has left this step's rows and written its outputs
    if (tid == 0) issue_to((oy - oy0 + 1) * S + NR - 1);  // local rows below (oy - oy0 + 1) S are free
    if (kSum && tid < CG) {
      int x = 0;
      for (; x + 8 <= Wo; x += 8) {
        float u[8];
#pragma unroll
        for (int j = 0; j < 8; j++) u[j] = ob[(x + j) * CG + tid];
#pragma unroll
        for (int j = 0; j < 8; j++) cs = __fadd_rn(cs, u[j]);
      }
      for (; x < Wo; x++) cs = __fadd_rn(cs, ob[x * CG + tid]);
    }
  }
  if (oy < oy1) {  // a load never arrived: report it, then let the loads still in flight land before leaving
    if (tid == 0) {
      if (err) atomicExch(err, BNNK_ERR_DW3_WAIT);
      for (int iy = (oy - oy0) * S; iy < issued; iy++) mbar_wait(smem_u32(&bar[iy % NR]), (uint32_t)(iy / NR) & 1u);
    }
    __syncthreads();
    return;
  }
  if (kSum && tid < CG) chsum[win * cws + grp * CG + tid] = cs;
}

// ------------------------------------------------------------------ SE_GATE (src/v24_f32.c:164-179, rt_ops_f32.c:272-283)

// One CTA per WB windows (the weights are read once for all of them). fc1 row r: 8 threads hold the 8 NEON
// accumulator lanes (a0 lanes 0-3, a1 lanes 0-3) over c = 8i + lane, then (a0 + a1) lane-wise and the FADDP reduction
// (v0 + v1) + (v2 + v3); SiLU with libm expf and an IEEE division. fc2 per channel from the bias, one FMA per r in
// order, then the sigmoid. Each window keeps its own chains, in the same order as alone; their weight loads are
// shared and issued in batches ahead of the FMAs.
constexpr int kSeThreads = 512;
template <int WB>
__global__ void __launch_bounds__(kSeThreads) k_se_gate(int B, int C, int rd, const float *__restrict__ w1,
                                                        const float *__restrict__ b1, const float *__restrict__ w2t,
                                                        const float *__restrict__ b2, const float *__restrict__ chsum,
                                                        long long cws, int P, float *__restrict__ gate, long long gws) {
  extern __shared__ float sm[];
  float *mean = sm, *s1 = sm + WB * C;  // [WB][C], [WB][rd]
  const int w0 = blockIdx.x * WB, tid = threadIdx.x;
  const float inv = __fdiv_rn(1.f, __int2float_rn(P));
  for (int j = 0; j < WB; j++)
    for (int c = tid; c < C; c += kSeThreads)
      mean[j * C + c] = w0 + j < B ? __fmul_rn(chsum[(w0 + j) * cws + c], inv) : 0.f;
  __syncthreads();
  const int lane8 = tid & 7, C8 = C >> 3;
  for (int r0 = 0; r0 < rd; r0 += kSeThreads / 8) {
    const int r = r0 + tid / 8;
    float a[WB];
#pragma unroll
    for (int j = 0; j < WB; j++) a[j] = 0.f;
    if (r < rd) {
      const float *wr = w1 + (long long)r * C + lane8;
      const float *mr = mean + lane8;
      int i = 0;
      // the next batch of 8 weights is loaded while the current one is multiplied (the chain waits on L2 otherwise)
      float wn[8];
      if (C8 >= 8) {
#pragma unroll
        for (int u = 0; u < 8; u++) wn[u] = __ldg(wr + 8 * u);
      }
      for (; i + 8 <= C8; i += 8) {
        float wv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) wv[u] = wn[u];
        if (i + 16 <= C8) {
#pragma unroll
          for (int u = 0; u < 8; u++) wn[u] = __ldg(wr + 8 * (i + 8 + u));
        }
#pragma unroll
        for (int u = 0; u < 8; u++)
#pragma unroll
          for (int j = 0; j < WB; j++) a[j] = __fmaf_rn(wv[u], mr[j * C + 8 * (i + u)], a[j]);
      }
      for (; i < C8; i++) {
        const float wv = __ldg(wr + 8 * i);
#pragma unroll
        for (int j = 0; j < WB; j++) a[j] = __fmaf_rn(wv, mr[j * C + 8 * i], a[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < WB; j++) {
      // lanes l and l + 4 hold a0[l] and a1[l]
      const float other = __shfl_down_sync(0xffffffffu, a[j], 4, 8);
      const float v = __fadd_rn(a[j], other);  // v[l] for l < 4
      const float v1 = __shfl_down_sync(0xffffffffu, v, 1, 8), v2 = __shfl_down_sync(0xffffffffu, v, 2, 8),
                  v3 = __shfl_down_sync(0xffffffffu, v, 3, 8);
      if (r < rd && lane8 == 0) {
        const float xr = __fadd_rn(__fadd_rn(__fadd_rn(v, v1), __fadd_rn(v2, v3)), b1[r]);
        s1[j * rd + r] = __fdiv_rn(xr, __fadd_rn(1.f, glibc_expf(-xr, c_expf_tab)));
      }
    }
  }
  __syncthreads();
  for (int c = tid; c < C; c += kSeThreads) {
    float g[WB];
#pragma unroll
    for (int j = 0; j < WB; j++) g[j] = b2[c];
    int r = 0;
    float wn[16];  // the next batch of 16 weights in flight while the current one is multiplied
    if (rd >= 16) {
#pragma unroll
      for (int u = 0; u < 16; u++) wn[u] = __ldg(w2t + (long long)u * C + c);
    }
    for (; r + 16 <= rd; r += 16) {
      float wv[16];
#pragma unroll
      for (int u = 0; u < 16; u++) wv[u] = wn[u];
      if (r + 32 <= rd) {
#pragma unroll
        for (int u = 0; u < 16; u++) wn[u] = __ldg(w2t + (long long)(r + 16 + u) * C + c);
      }
#pragma unroll
      for (int u = 0; u < 16; u++)
#pragma unroll
        for (int j = 0; j < WB; j++) g[j] = __fmaf_rn(wv[u], s1[j * rd + r + u], g[j]);
    }
    for (; r < rd; r++) {
      const float wv = __ldg(w2t + (long long)r * C + c);
#pragma unroll
      for (int j = 0; j < WB; j++) g[j] = __fmaf_rn(wv, s1[j * rd + r], g[j]);
    }
#pragma unroll
    for (int j = 0; j < WB; j++)
      if (w0 + j < B) gate[(w0 + j) * gws + c] = sigmoid(g[j]);
  }
}

// ------------------------------------------------------------------ C0POOL (src/v24_f32.c:139-147, gemm_f32.c:60-70)

// One CTA per (output row oy, window); thread qx computes the pooled pixel qx: conv pixels 2qx and 2qx + 1, 24
// channels each, K = 64 fused multiply-adds in (ky, kx, ci) order from 0, bias added after, ReLU, max | average.
// The 4 padded input rows sit in shared memory transposed by 8-float phase (float 8i + r at [r][i]) so that the 32
// threads of a warp, whose patches start 8 floats apart, read consecutive words.
// kQ: also quantize each output row (48 channels, s8n_quant_rows) for the PW_S8 that reads it: q [rows][kq] (pads =
// zero point), sa, za; wpin = 0 leaves the fp32 output unwritten (no other op reads it)
template <bool kQ>
__global__ void __launch_bounds__(128) k_c0pool(const float *__restrict__ img, long long iws, const float *__restrict__ wt,
                                                const float *__restrict__ bias, float *__restrict__ pin, long long pws,
                                                int8_t *__restrict__ q, float *__restrict__ qsa,
                                                int32_t *__restrict__ qza, int kq, int wpin) {
  constexpr int PWD = 518, RF = PWD * 2, NI = (RF + 7) / 8 + 1;  // padded width: 3 + 511 + 4 pixels
  __shared__ float rows[4][8][NI];
  __shared__ __align__(16) float ws[64][24];
  __shared__ float bs[24];
  const int oy = blockIdx.x, win = blockIdx.y, tid = threadIdx.x;
  const float *im = img + win * iws;
  // per row, padded float index cidx = 8 ii + ph (shifts only); the row's sample cidx / 2 - 3, channel cidx & 1
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int y = 2 * oy + r - 1;
    const bool yin = y >= 0 && y < 96;
    const float *imr = im + (long long)(yin ? y : 0) * 511 * 2 - 6;  // cidx 6 is the row's first sample
    for (int cidx = tid; cidx < 8 * NI; cidx += 128) {
      const int xcol = (cidx >> 1) - 3;
      rows[r][cidx & 7][cidx >> 3] = (yin && cidx < RF && xcol >= 0 && xcol < 511) ? imr[cidx] : 0.f;
    }
  }
  for (int i = tid; i < 64 * 24; i += 128) (&ws[0][0])[i] = wt[i];
  if (tid < 24) bs[tid] = bias[tid];
  __syncthreads();
  const int qx = tid;
  float2 acc0[12], acc1[12];  // channel pairs (paired fp32 FMA: each lane one fused multiply-add)
#pragma unroll
  for (int n = 0; n < 12; n++) acc0[n] = acc1[n] = make_float2(0.f, 0.f);
  for (int ky = 0; ky < 4; ky++) {
#pragma unroll 4
    for (int kk = 0; kk < 16; kk++) {
      const int c0 = kk, c1 = kk + 4;  // float offsets of the two pixels' patches from 8 qx
      const float2 a0 = splat2(rows[ky][c0 & 7][qx + (c0 >> 3)]), a1 = splat2(rows[ky][c1 & 7][qx + (c1 >> 3)]);
      const float4 *wr = reinterpret_cast<const float4 *>(ws[ky * 16 + kk]);
#pragma unroll
      for (int n4 = 0; n4 < 6; n4++) {
        const float4 w = wr[n4];
        const float2 wl = make_float2(w.x, w.y), wh = make_float2(w.z, w.w);
        acc0[2 * n4] = fma2_rn(wl, a0, acc0[2 * n4]);
        acc0[2 * n4 + 1] = fma2_rn(wh, a0, acc0[2 * n4 + 1]);
        acc1[2 * n4] = fma2_rn(wl, a1, acc1[2 * n4]);
        acc1[2 * n4 + 1] = fma2_rn(wh, a1, acc1[2 * n4 + 1]);
      }
    }
  }
  float *o = pin + win * pws + ((long long)oy * 128 + qx) * 48;
  float y[48];  // [0, 24): max pool, [24, 48): average pool
#pragma unroll
  for (int n = 0; n < 24; n++) {
    const float c0v = (n & 1) ? acc0[n >> 1].y : acc0[n >> 1].x, c1v = (n & 1) ? acc1[n >> 1].y : acc1[n >> 1].x;
    const float u = fmax_nan(__fadd_rn(c0v, bs[n]), 0.f), v = fmax_nan(__fadd_rn(c1v, bs[n]), 0.f);
    y[n] = fmax_nan(u, v);
    y[24 + n] = __fmul_rn(__fadd_rn(u, v), 0.5f);
  }
  if (!kQ || wpin) {
#pragma unroll
    for (int i = 0; i < 48; i += 4) *reinterpret_cast<float4 *>(o + i) = make_float4(y[i], y[i + 1], y[i + 2], y[i + 3]);
  }
  if (kQ) {
    float lo = __int_as_float(0x7f800000), hi = __int_as_float(0xff800000);
#pragma unroll
    for (int i = 0; i < 48; i++) { lo = fmin_nan(lo, y[i]); hi = fmax_nan(hi, y[i]); }  // 48 = the 4-wide part
    float inv, s;
    int32_t z;
    quant_params(lo, hi, inv, z, s);
    const long long row = (long long)win * 6144 + oy * 128 + qx;
    qsa[row] = s;
    qza[row] = z;
    uint32_t wd[12];
#pragma unroll
    for (int i = 0; i < 12; i++)  // 48 columns: all in the 8-wide part
      wd[i] = quant_word(__fmul_rn(y[4 * i], inv), __fmul_rn(y[4 * i + 1], inv), __fmul_rn(y[4 * i + 2], inv),
                         __fmul_rn(y[4 * i + 3], inv), z, true);
    uint4 *qr = reinterpret_cast<uint4 *>(q + row * kq);
    const uint32_t zp = ((uint32_t)z & 0xffu) * 0x01010101u;
    qr[0] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    qr[1] = make_uint4(wd[4], wd[5], wd[6], wd[7]);
    qr[2] = make_uint4(wd[8], wd[9], wd[10], wd[11]);
    for (int i = 3; i < kq / 16; i++) qr[i] = make_uint4(zp, zp, zp, zp);
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

// pc GEMM + ReLU + mean. Each output (row m = 6 w + r, column n) is one sequential chain of fused multiply-adds from
// 0 over k = 0 .. 1727 (the reference's K loop), so only the schedule around the chains is free: a CTA owns 16
// windows (96 rows) x 64 columns, its 256 threads 6 rows x 4 columns each (two paired-fp32 FMA chains per row, each
// lane rounded once as fmaf), with 32-k slices of both operands double-buffered in shared memory by cp.async. The
// epilogue adds the bias, applies ReLU and sums the window's 6 rows in order, scaled by 1/6.
constexpr int kPcM = 96, kPcN = 64, kPcK = 32, kPcKs = kPcK + 4, kPcThreads = 256, kPcKTot = 1728;

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  const int n = valid ? 16 : 0;  // zero fill past the last row
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

__global__ void __launch_bounds__(kPcThreads) k_postpc_gemm(int B, const float *__restrict__ pcin,
                                                            const float *__restrict__ wt,
                                                            const float *__restrict__ bias, float *__restrict__ feat,
                                                            long long fws) {
  __shared__ __align__(16) float a_s[2][kPcM][kPcKs];
  __shared__ __align__(16) float w_s[2][kPcK][kPcN];
  const int tid = threadIdx.x, wl = tid / 16, cg = tid % 16;
  const int m0 = blockIdx.y * kPcM, n0 = blockIdx.x * kPcN, rows = min(kPcM, 6 * B - m0);
  auto load = [&](int st, int k0) {
    for (int i = tid; i < kPcM * kPcK / 4; i += kPcThreads) {
      const int m = i / (kPcK / 4), kq = i - m * (kPcK / 4);
      const bool ok = m < rows;
      cp_async16(&a_s[st][m][4 * kq], pcin + (long long)(m0 + (ok ? m : 0)) * kPcKTot + k0 + 4 * kq, ok);
    }
    for (int i = tid; i < kPcK * kPcN / 4; i += kPcThreads) {
      const int kk = i / (kPcN / 4), nq = i - kk * (kPcN / 4);
      cp_async16(&w_s[st][kk][4 * nq], wt + (long long)(k0 + kk) * 1024 + n0 + 4 * nq, true);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float2 acc[6][2];
#pragma unroll
  for (int r = 0; r < 6; r++) acc[r][0] = acc[r][1] = make_float2(0.f, 0.f);
  constexpr int kChunks = kPcKTot / kPcK;
  load(0, 0);
  for (int c = 0; c < kChunks; c++) {
    if (c + 1 < kChunks) {
      load((c + 1) & 1, (c + 1) * kPcK);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int st = c & 1;
#pragma unroll
    for (int kk = 0; kk < kPcK; kk += 4) {
      float4 a[6];
#pragma unroll
      for (int r = 0; r < 6; r++) a[r] = *reinterpret_cast<const float4 *>(&a_s[st][wl * 6 + r][kk]);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float4 w4 = *reinterpret_cast<const float4 *>(&w_s[st][kk + u][4 * cg]);
        const float2 w01 = make_float2(w4.x, w4.y), w23 = make_float2(w4.z, w4.w);
#pragma unroll
        for (int r = 0; r < 6; r++) {
          const float av = u == 0 ? a[r].x : u == 1 ? a[r].y : u == 2 ? a[r].z : a[r].w;
          acc[r][0] = fma2_rn(splat2(av), w01, acc[r][0]);
          acc[r][1] = fma2_rn(splat2(av), w23, acc[r][1]);
        }
      }
    }
    __syncthreads();
  }
  if (wl * 6 >= rows) return;
  const int n = n0 + 4 * cg;
  const float4 b4 = *reinterpret_cast<const float4 *>(bias + n);
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < 6; r++) {
    s[0] = __fadd_rn(s[0], fmax_nan(__fadd_rn(acc[r][0].x, b4.x), 0.f));
    s[1] = __fadd_rn(s[1], fmax_nan(__fadd_rn(acc[r][0].y, b4.y), 0.f));
    s[2] = __fadd_rn(s[2], fmax_nan(__fadd_rn(acc[r][1].x, b4.z), 0.f));
    s[3] = __fadd_rn(s[3], fmax_nan(__fadd_rn(acc[r][1].y, b4.w), 0.f));
  }
  const float k6 = 0x1.555556p-3f;
  *reinterpret_cast<float4 *>(feat + (long long)(m0 / 6 + wl) * fws + n) =
      make_float4(__fmul_rn(s[0], k6), __fmul_rn(s[1], k6), __fmul_rn(s[2], k6), __fmul_rn(s[3], k6));
}

// ------------------------------------------------------------------ STEM, fp32 math to fp16 (src/rt_ops_f16.c:175-190)
//
// The dense k x k VALID conv of compiled models on a 1-channel fp32 image (Perch's stem): the reference builds the
// im2col rows (taps (ky, kx) in order, zeros up to Kp; src/pc_kern_f32.c:151-161) and runs its fp32 GEMM (one
// accumulator per output from +0, fused multiply-adds over all Kp taps in order, + bias, SiLU polynomial or FMAX(x, 0);
// src/gemm_f32.c:100-132), then rounds the outputs to fp16 into the zero-haloed buffer (pc_cvt_pad_f16,
// src/pc_kern_f16.c:104-113). Thread (pixel, 8-channel panel): the taps are read from the image as the GEMM consumes
// them (no im2col buffer), the panel's weights and bias sit in shared memory.
template <int KS>  // KS > 0: the kernel size known at compile time (taps unrolled); 0: any k
__global__ void __launch_bounds__(256) k_stem_f16(const float *__restrict__ img, long long iws, int W, int k, int s,
                                                  int Ho, int Wo, const float *__restrict__ wt,
                                                  const float *__restrict__ bias, int N, int Kp, int Np, int act,
                                                  uint16_t *__restrict__ out, long long ows, int ldo, int opad,
                                                  int st16) {
  extern __shared__ float sw[];  // [Kp][Np] weights (channel fastest: the panels of a warp hit distinct banks), [Np] bias
  __shared__ uint32_t lut[256];
  const int tid = threadIdx.x;
  for (int i = tid; i < 256; i += blockDim.x) lut[i] = g_frecpe_lut[i];
  for (int i = tid; i < Np * Kp; i += blockDim.x) {  // from the package's panels [Np/8][Kp][8]
    const int nb = i / (Kp * 8), r = i - nb * Kp * 8, t = r / 8, j = r - t * 8;
    sw[t * Np + nb * 8 + j] = wt[i];
  }
  for (int i = tid; i < Np; i += blockDim.x) sw[Np * Kp + i] = bias[i];
  __syncthreads();
  const int npan = Np / 8, M = Ho * Wo, kk = KS > 0 ? KS : k, K = kk * kk;
  const long long win = blockIdx.y;
  const int item = blockIdx.x * blockDim.x + tid;
  if (item >= M * npan) return;
  const int m = item / npan, nb = item - m * npan;
  const int oy = m / Wo, ox = m - oy * Wo;
  const float *x = img + win * iws + (long long)(oy * s) * W + ox * s;
  const float *wp = sw + nb * 8;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; j++) acc[j] = 0.f;
  if constexpr (KS > 0) {
    constexpr int KP = ((KS * KS + 3) & ~3);
    float v[KP];
#pragma unroll
    for (int t = 0; t < KP; t++) v[t] = t < KS * KS ? __ldg(x + (t / KS) * W + t % KS) : 0.f;
#pragma unroll
    for (int t = 0; t < KP; t++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] = __fmaf_rn(v[t], wp[t * Np + j], acc[j]);
  } else {
    int ky = 0, kx = 0;
    for (int t = 0; t < Kp; t++) {
      float v = 0.f;
      if (t < K) {
        v = __ldg(x + ky * W + kx);
        if (++kx == kk) { kx = 0; ky++; }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] = __fmaf_rn(v, wp[t * Np + j], acc[j]);
    }
  }
  uint16_t *o = out + win * ows + ((long long)(oy + opad) * (Wo + 2 * opad) + ox + opad) * ldo + nb * 8;
  uint32_t hv[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    float y = __fadd_rn(acc[j], sw[Np * Kp + nb * 8 + j]);
    if (act == 1) y = silu<true>(y, lut);
    else if (act == 2) y = fmax_nan(y, 0.f);
    hv[j] = __half_as_ushort(__float2half_rn(y));
  }
  if (st16 && nb * 8 + 8 <= N) {  // a whole panel: one 16-byte store
    *reinterpret_cast<uint4 *>(o) = make_uint4(hv[0] | hv[1] << 16, hv[2] | hv[3] << 16, hv[4] | hv[5] << 16,
                                               hv[6] | hv[7] << 16);
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (nb * 8 + j < N) o[j] = (uint16_t)hv[j];
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

template <int S, int R>
static int launch_dw3(int B, int cg4, const float *xp, long long xws, int W, int C, const float *w, const float *b,
                      float *out, long long ows, int Wo, int P, float *chsum, long long cws, bnn_stream_t st) {
  const int nl = kDwThreads / cg4;
  const size_t smem = sizeof(float) * 2 * nl * R * 4 * cg4;
  const unsigned grid = (unsigned)B * (unsigned)((C / 4) / cg4);
  k_dw3<S, R><<<grid, kDwThreads, smem, st>>>(xp, xws, W, C, cg4, nl, w, b, out, ows, Wo, P, chsum, cws);
  return cudaGetLastError();
}

static PFN_cuTensorMapEncodeTiled_v12000 conv_encode_fn(void) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  }
  return fn;
}

// shared memory of the TMA form for CG channels: the ring of nr input rows and the two output-row tiles
static size_t dw3t_smem(int W, int Wo, int nr, int cg) {
  const size_t row_stride = ((size_t)(W + 2) * cg * 4 + 127) & ~(size_t)127;
  return (size_t)nr * row_stride + sizeof(float) * 2 * Wo * cg;
}

// channels per CTA for the TMA form: the largest multiple of 4 dividing C, at most 256 (one box dimension), whose
// minimal ring of S + 3 rows leaves two CTAs per SM (budget: the dynamic shared memory each may use); 0 if none.
// BNN_DW3_CG overrides it (a divisor of C, a multiple of 4, that fits).
static int dw3t_group(int C, int W, int Wo, int s, size_t budget) {
  int best = 0;
  for (int cg = 4; cg <= C && cg <= 256; cg += 4)
    if (C % cg == 0 && dw3t_smem(W, Wo, s + 3, cg) <= budget) best = cg;
  const char *e = getenv("BNN_DW3_CG");
  const int want = e ? atoi(e) : 0;
  if (want >= 4 && want <= 256 && want % 4 == 0 && C % want == 0 && dw3t_smem(W, Wo, s + 3, want) <= budget)
    best = want;
  return best;
}

// ring depth: S + 3 (one row step of lookahead, which measured as fast as deeper rings on every v2.4 layer);
// BNN_DW3_NR asks for a deeper one (at most the rows the outputs read, kDw3MaxRing and the budget)
static int dw3t_ring(int W, int Wo, int s, int cg, int rows_in, size_t budget) {
  const char *e = getenv("BNN_DW3_NR");
  int cap = e ? atoi(e) : 0;
  if (cap > rows_in) cap = rows_in;
  if (cap > kDw3MaxRing) cap = kDw3MaxRing;
  int nr = s + 3;
  while (nr < cap && dw3t_smem(W, Wo, nr + 1, cg) <= budget) nr++;
  return nr;
}

extern "C" int bnnk_dw3(int B, const float *xp, long long xws, int H, int W, int C, int s, const float *w,
                        const float *b, float *out, long long ows, int Ho, int Wo, float *chsum, long long cws,
                        int *err, bnn_stream_t st) {
  if (B <= 0) return 0;
  const int P = Ho * Wo, C4 = C / 4;
  const size_t budget = smem_budget(k_dw3t<1, 2, true>, 2);  // every instance has the same static shared memory
  const int cg = dw3t_group(C, W, Wo, s, budget);
  PFN_cuTensorMapEncodeTiled_v12000 enc = conv_encode_fn();
  if (cg && enc && ((uintptr_t)xp & 15) == 0 && (xws * 4) % 16 == 0 && W + 2 <= 256 && (s == 1 || s == 2) &&
      (Ho - 1) * s + 3 <= H + 2 && ((uintptr_t)out & 15) == 0 && ows % 4 == 0) {
    CUtensorMap map;
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)(H + 2) * (W + 2), (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)C * 4, (cuuint64_t)xws * 4};
    cuuint32_t box[3] = {(cuuint32_t)cg, (cuuint32_t)(W + 2), 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(xp), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
      // without channel sums (chsum NULL): bands of at least 4 output rows, as many as fill the two CTAs per SM
      // that the shared memory allows in one wave (more waves of shorter bands measured no faster)
      const bool sum = chsum != nullptr;
      int nband = 1;
      if (!sum) {
        const long long ctas = (long long)B * (C / cg);
        nband = (int)((2LL * num_sms()) / ctas);
        if (nband > Ho / 4) nband = Ho / 4;
        if (nband < 1) nband = 1;
      }
      const int hb = (Ho + nband - 1) / nband;
      const int nr = dw3t_ring(W, Wo, s, cg, (hb - 1) * s + 3, budget);
      const size_t smem = dw3t_smem(W, Wo, nr, cg);
      const unsigned grid = (unsigned)B * (unsigned)(C / cg) * (unsigned)nband;
      // threads: whole channel quads up to 256, at least the CG summing threads
      const int Q = cg / 4;
      int nt = (256 / Q) * Q;
      if (nt < cg) nt = cg;
      nt = (nt + 31) / 32 * 32;
      const bool pair = Wo % 2 == 0;
#define BNN_DW3T_(SS, RR, KS)                                                                                     \
  do {                                                                                                             \
    cudaFuncSetAttribute(k_dw3t<SS, RR, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);              \
    k_dw3t<SS, RR, KS><<<grid, nt, smem, st>>>(map, W, C, cg, Ho, Wo, nr, w, b, out, ows, chsum, cws, err, nband); \
  } while (0)
#define BNN_DW3T(SS, RR) \
  do {                    \
    if (sum) BNN_DW3T_(SS, RR, true); else BNN_DW3T_(SS, RR, false); \
  } while (0)
      if (s == 1) { if (pair) BNN_DW3T(1, 2); else BNN_DW3T(1, 1); }
      else { if (pair) BNN_DW3T(2, 2); else BNN_DW3T(2, 1); }
#undef BNN_DW3T
#undef BNN_DW3T_
      return cudaGetLastError();
    }
  }
  // general strides: the form that loads its taps directly
  int cg4 = 1;
  for (int d = 1; d <= 32 && d <= C4; d++)
    if (C4 % d == 0 && (d == 1 || (long long)B * (C4 / d) >= 4 * 148)) cg4 = d;
  if (cg4 == 1)
    for (int d = 2; d <= 32 && d <= C4; d++)
      if (C4 % d == 0 && d <= 8) cg4 = d;
  const bool pair = Wo % 2 == 0;
  if (s == 1) return pair ? launch_dw3<1, 2>(B, cg4, xp, xws, W, C, w, b, out, ows, Wo, P, chsum, cws, st)
                          : launch_dw3<1, 1>(B, cg4, xp, xws, W, C, w, b, out, ows, Wo, P, chsum, cws, st);
  return pair ? launch_dw3<2, 2>(B, cg4, xp, xws, W, C, w, b, out, ows, Wo, P, chsum, cws, st)
              : launch_dw3<2, 1>(B, cg4, xp, xws, W, C, w, b, out, ows, Wo, P, chsum, cws, st);
}

extern "C" int bnnk_se_gate(int B, int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                            const float *chsum, long long cws, int P, float *gate, long long gws, bnn_stream_t st) {
  if (B <= 0) return 0;
  // windows per CTA: two from 512 windows on (the weights are read once per CTA; measured: Perch's 26 SE at batch
  // 512 0.85 -> 0.65 ms, while v2.4's 13 at batch 256 went 0.26 -> 0.32 ms with 128 CTAs, so they keep one)
  const int wb = B >= 512 ? 2 : 1;
  const size_t smem = sizeof(float) * (size_t)wb * (C + rd);
  if (smem > 48 * 1024) {  // wide layers: one window per CTA
    k_se_gate<1><<<B, kSeThreads, sizeof(float) * (size_t)(C + rd), st>>>(B, C, rd, w1, b1, w2t, b2, chsum, cws, P,
                                                                          gate, gws);
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)((B + wb - 1) / wb);
  if (wb == 2) k_se_gate<2><<<grid, kSeThreads, smem, st>>>(B, C, rd, w1, b1, w2t, b2, chsum, cws, P, gate, gws);
  else k_se_gate<1><<<grid, kSeThreads, smem, st>>>(B, C, rd, w1, b1, w2t, b2, chsum, cws, P, gate, gws);
  return cudaGetLastError();
}

extern "C" int bnnk_c0pool(int B, const float *img, long long iws, const float *wt, const float *b, float *pin,
                           long long pws, const bnnk_qrows *qr, bnn_stream_t st) {
  if (B <= 0) return 0;
  if (qr && qr->kq >= 48 && qr->kq % 16 == 0)
    k_c0pool<true><<<dim3(48, B), 128, 0, st>>>(img, iws, wt, b, pin, pws, qr->q, qr->sa, qr->za, qr->kq, qr->keep);
  else
    k_c0pool<false><<<dim3(48, B), 128, 0, st>>>(img, iws, wt, b, pin, pws, nullptr, nullptr, nullptr, 0, 1);
  return cudaGetLastError();
}

extern "C" int bnnk_postpc(int B, const float *X, long long xws, const float *post_s, const float *post_b,
                           const float *wt, const float *b, float *pcin, float *feat, long long fws, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_postpc_im2col<<<B, 256, 0, st>>>(X, xws, post_s, post_b, pcin);
  k_postpc_gemm<<<dim3(1024 / kPcN, (6 * B + kPcM - 1) / kPcM), kPcThreads, 0, st>>>(B, pcin, wt, b, feat, fws);
  return cudaGetLastError();
}

extern "C" int bnnk_stem_f16(int B, const float *img, long long iws, int W, int k, int s, int Ho, int Wo,
                             const float *w, const float *b, int N, int Kp, int Np, int act, uint16_t *out,
                             long long ows, int ldo, int opad, bnn_stream_t st) {
  if (B <= 0) return 0;
  const size_t smem = sizeof(float) * ((size_t)Np * Kp + Np);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  const long long items = (long long)Ho * Wo * (Np / 8);
  const int st16 = ldo % 8 == 0 && ows % 8 == 0 && ((uintptr_t)out & 15) == 0;
  const dim3 grid((unsigned)((items + 255) / 256), (unsigned)B);
  if (k == 3 && Kp == 12)
    k_stem_f16<3><<<grid, 256, smem, st>>>(img, iws, W, k, s, Ho, Wo, w, b, N, Kp, Np, act, out, ows, ldo, opad, st16);
  else
    k_stem_f16<0><<<grid, 256, smem, st>>>(img, iws, W, k, s, Ho, Wo, w, b, N, Kp, Np, act, out, ows, ldo, opad, st16);
  return cudaGetLastError();
}
