// int8 1x1 conv / dense layer on sm_100a: the per-row dynamic quantizer and a persistent tcgen05 kind::i8 GEMM with
// the fused dequant / activation / residual / padded-store epilogue.
//
// Reference: src/gemm_s8n.c (s8n_quant_rows :15-63, acc4x4 / tile4x4 / s8n_gemm_range :82-190) driven by PW_S8 and
// GEMV_S8 (src/rt_ops_s8n.c:92-158). The int32 sums are exact in both (|q|, |w| <= 127, K <= 4096), so the tensor
// cores' summation order cannot change them; everything after the sum repeats the reference's fp32 steps.
//
// GEMM: one persistent CTA per SM walks the 128-row x BN-column tiles (N tiles inner, so consecutive tiles reuse the
// same rows of A from L2). Warp 0 lane 0 streams K blocks of A (quantized rows) and B (weights [Nrows][Kq], K-major)
// into a ring of shared-memory stages with 2-D TMA loads (128-byte K blocks, swizzle 128 B; a ragged last block reads
// zero fill; every CTA loads its own tiles). Warp 1 lane 0 issues tcgen05.mma.cta_group::1.kind::i8 (M 128, N BN,
// K 32 per instruction) into one of NE TMEM accumulators (tile i uses accumulator i mod NE) and releases stages and
// finished accumulators with tcgen05.commit. Each accumulator has an epilogue group of 4 NH warps: the warps of a
// TMEM lane quarter (= 32 rows) split the tile's 8-column units round robin, read them with tcgen05.ld, free the
// accumulator and run the fp32 epilogue while the MMA warp fills the other one. Every mbarrier wait is bounded by a
// %globaltimer deadline; a timeout sets the error word, the CTA stops and still frees its TMEM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "bnn_kernels.h"
#include "smem_attr.cuh"
#include "emu.cuh"
#include "ln_cr.cuh"
#include "sync.cuh"
#include "tc.cuh"

namespace bnn {

// ------------------------------------------------------------------ quantizer

// L lanes per row; lane l owns the 16-element chunks ch = l + i L (i < NC) of the quantized row (Kq / 16 chunks:
// 64 contiguous input bytes, 16 contiguous output bytes each), held in registers across both passes: the row's
// NaN-propagating min / max (the 4-wide part of s8n_quant_rows; K % 4 == 0 here, so there is no scalar tail),
// reduced over the lanes, then the quantized bytes (pads past K = the zero point), one 16-byte store per chunk.
// Gate and scale multiplies run paired (each lane an IEEE multiply; their products feed no add).
template <int L, int NC>
__global__ void __launch_bounds__(256) k_quant(int rows, int Mw, const float *__restrict__ x, long long xws, int lda,
                                               int K, int Kq, const float *__restrict__ gate, long long gws,
                                               int8_t *__restrict__ q, float *__restrict__ sa,
                                               int32_t *__restrict__ za) {
  const int lane = threadIdx.x % L;
  const int row = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) / L);
  const bool valid = row < rows;
  const int r = valid ? row : rows - 1;
  const int w = r / Mw, m = r - w * Mw;
  const float *xr = x + w * xws + (long long)m * lda;
  const float *gr = gate ? gate + w * gws : nullptr;
  const int K4 = K >> 2, nch = Kq >> 4;
  float4 v[NC][4];
  float lo = __int_as_float(0x7f800000), hi = __int_as_float(0xff800000);
#pragma unroll
  for (int i = 0; i < NC; i++) {
    const int ch = lane + i * L;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int g = 4 * ch + e;  // float4 group
      if (ch < nch && g < K4) {
        float4 t = __ldg(reinterpret_cast<const float4 *>(xr + 4 * g));
        if (gr) {
          const float4 gg = __ldg(reinterpret_cast<const float4 *>(gr + 4 * g));
          const float2 p0 = mul2_rn(make_float2(t.x, t.y), make_float2(gg.x, gg.y));
          const float2 p1 = mul2_rn(make_float2(t.z, t.w), make_float2(gg.z, gg.w));
          t = make_float4(p0.x, p0.y, p1.x, p1.y);
        }
        v[i][e] = t;
        lo = fmin_nan(lo, fmin_nan(fmin_nan(t.x, t.y), fmin_nan(t.z, t.w)));
        hi = fmax_nan(hi, fmax_nan(fmax_nan(t.x, t.y), fmax_nan(t.z, t.w)));
      }
    }
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) {
    lo = fmin_nan(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmax_nan(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  float inv, s;
  int32_t z;
  quant_params(lo, hi, inv, z, s);
  if (!valid) return;
  if (lane == 0) { sa[row] = s; za[row] = z; }
  const int K8 = K & ~7;
  uint4 *qr = reinterpret_cast<uint4 *>(q + (long long)r * Kq);
  const float2 inv2 = splat2(inv);
  const uint32_t zp = ((uint32_t)z & 0xffu) * 0x01010101u;  // a pad word: the zero point
  const uint32_t zz = (uint32_t)z - kRoundBits;
  const bool fast = quant_fast(lo, hi, inv);
#pragma unroll
  for (int i = 0; i < NC; i++) {
    const int ch = lane + i * L;
    if (ch >= nch) break;
    uint32_t wd[4];
    if (fast) {
#pragma unroll
      for (int e = 0; e < 4; e++) wd[e] = 4 * ch + e < K4 ? quant_word_fast(v[i][e], inv, zz) : zp;
    } else {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int g = 4 * ch + e;
        if (g < K4) {
          const float2 p0 = mul2_rn(make_float2(v[i][e].x, v[i][e].y), inv2);
          const float2 p1 = mul2_rn(make_float2(v[i][e].z, v[i][e].w), inv2);
          wd[e] = quant_word(p0.x, p0.y, p1.x, p1.y, z, 4 * g < K8);
        } else {
          wd[e] = zp;
        }
      }
    }
    qr[ch] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

// The second half of a warp-per-row quantizer: the row's gated values v (lane l holds the float4 groups l + 32 i;
// NG = ceil(K / 128), so only the last group can fall past K) and the lane's partial min / max in, the row's
// parameters and its quantized bytes (4-byte words, pads past K = the zero point) out.
template <int NG>
__device__ __forceinline__ void quant_row_out(const float4 (&v)[NG], float lo, float hi, int lane, int K4, int Kq4,
                                              int K8, int r, int8_t *__restrict__ q, int Kq, float *__restrict__ sa,
                                              int32_t *__restrict__ za) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fmin_nan(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmax_nan(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  float inv, s;
  int32_t z;
  quant_params(lo, hi, inv, z, s);
  if (lane == 0) { sa[r] = s; za[r] = z; }
  uint32_t *qr = reinterpret_cast<uint32_t *>(q + (long long)r * Kq);
  const uint32_t zp = ((uint32_t)z & 0xffu) * 0x01010101u;  // a pad word: the zero point
  if (quant_fast(lo, hi, inv)) {
    const uint32_t zz = (uint32_t)z - kRoundBits;
#pragma unroll
    for (int i = 0; i < NG; i++) {
      const int g = lane + 32 * i;
      if (i < NG - 1 || g < K4) qr[g] = quant_word_fast(v[i], inv, zz);
      else if (g < Kq4) qr[g] = zp;
    }
  } else {
    const float2 inv2 = splat2(inv);
#pragma unroll
    for (int i = 0; i < NG; i++) {
      const int g = lane + 32 * i;
      if (i < NG - 1 || g < K4) {
        const float2 p0 = mul2_rn(make_float2(v[i].x, v[i].y), inv2);
        const float2 p1 = mul2_rn(make_float2(v[i].z, v[i].w), inv2);
        qr[g] = quant_word(p0.x, p0.y, p1.x, p1.y, z, 4 * g < K8);
      } else if (g < Kq4) {
        qr[g] = zp;
      }
    }
  }
  if (Kq4 > 32 * NG)  // pads beyond the register groups (never for Kq = K rounded up to 32)
    for (int g = 32 * NG + lane; g < Kq4; g += 32) qr[g] = zp;
}

// The row's values times the gate (paired multiplies: their products feed no add) and the lane's NaN-propagating
// min / max over them (the 4-wide part of s8n_quant_rows; K % 4 == 0 here, so there is no scalar tail).
template <int NG, bool kGate>
__device__ __forceinline__ void quant_row_in(float4 (&v)[NG], const float4 (&gv)[kGate ? NG : 1], int lane, int K4,
                                             float &lo, float &hi) {
  lo = __int_as_float(0x7f800000);
  hi = __int_as_float(0xff800000);
#pragma unroll
  for (int i = 0; i < NG; i++) {
    const int g = lane + 32 * i;
    if (i < NG - 1 || g < K4) {
      float4 t = v[i];
      if (kGate) {
        const float2 p0 = mul2_rn(make_float2(t.x, t.y), make_float2(gv[i].x, gv[i].y));
        const float2 p1 = mul2_rn(make_float2(t.z, t.w), make_float2(gv[i].z, gv[i].w));
        t = make_float4(p0.x, p0.y, p1.x, p1.y);
      }
      v[i] = t;
      lo = fmin_nan(lo, fmin_nan(fmin_nan(t.x, t.y), fmin_nan(t.z, t.w)));
      hi = fmax_nan(hi, fmax_nan(fmax_nan(t.x, t.y), fmax_nan(t.z, t.w)));
    }
  }
}

// Rows of 128-1536 (K % 4 == 0, 16-byte aligned rows), a warp per row: 512-byte coalesced loads, a contiguous run of
// rpw rows per warp with D rows in flight behind the one being quantized (D + 1 register buffers rotated by a fully
// unrolled loop, so no values move between registers). The window of a row is tracked by counting (no division per
// row); the SE gate, one row of K per window, sits in registers and is reloaded when the window changes.
template <int NG, bool kGate, int D>
__global__ void __launch_bounds__(256) k_quant_w(int rows, int Mw, const float *__restrict__ x, long long xws, int lda,
                                                 int K, int Kq, const float *__restrict__ gate, long long gws,
                                                 int8_t *__restrict__ q, float *__restrict__ sa,
                                                 int32_t *__restrict__ za, int rpw) {
  const int lane = threadIdx.x % 32;
  const int wrp = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) / 32);
  const int r0 = wrp * rpw, r1 = min(rows, r0 + rpw);
  if (r0 >= r1) return;
  const int K4 = K >> 2, Kq4 = Kq >> 2, K8 = K & ~7;
  int wl = r0 / Mw, ml = r0 - wl * Mw;  // the next row to load
  int wc = wl, mc = ml;                 // the next row to quantize
  float4 gv[kGate ? NG : 1];
  int gw = -1;
  auto load = [&](float4 (&dst)[NG]) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + wl * xws + (long long)ml * lda);
#pragma unroll
    for (int i = 0; i < NG; i++) {
      const int g = lane + 32 * i;
      if (i < NG - 1 || g < K4) dst[i] = __ldg(xr + g);
    }
    if (++ml == Mw) { ml = 0; wl++; }
  };
  auto process = [&](float4 (&v)[NG], int r) {
    if (kGate && wc != gw) {
      gw = wc;
      const float4 *gp = reinterpret_cast<const float4 *>(gate + wc * gws);
#pragma unroll
      for (int i = 0; i < NG; i++) {
        const int g = lane + 32 * i;
        gv[i] = (i < NG - 1 || g < K4) ? __ldg(gp + g) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float lo, hi;
    quant_row_in<NG, kGate>(v, gv, lane, K4, lo, hi);
    quant_row_out<NG>(v, lo, hi, lane, K4, Kq4, K8, r, q, Kq, sa, za);
    if (++mc == Mw) { mc = 0; wc++; }
  };
  float4 buf[D + 1][NG];
#pragma unroll
  for (int d = 0; d < D; d++)
    if (r0 + d < r1) load(buf[d]);
  for (int r = r0; r < r1; r += D + 1) {
#pragma unroll
    for (int u = 0; u <= D; u++) {
      const int rr = r + u;
      if (rr < r1) {
        if (rr + D < r1) load(buf[(u + D) % (D + 1)]);
        process(buf[u], rr);
      }
    }
  }
}

// Wide rows (K = 128 .. 1536, 16-byte aligned) with the row data staged in shared memory: each warp owns a ring of
// kQBD row slots that lane 0 fills by bulk copies (cp.async.bulk, one per row, completion counted on the slot's
// mbarrier), so kQBD rows per warp are in flight without holding registers. A warp takes a contiguous run of rows
// (the SE gate, one row of K per window, is re-read only when the window changes) and quantizes each as k_quant_w
// does: the row's NaN-propagating min / max, reduced over the lanes, then 4-byte words of quantized bytes. A wait that
// runs out records BNNK_ERR_QUANT_WAIT, waits (bounded) for the warp's other copies and leaves.
constexpr int kQBD = 4, kQBWarps = 8;
template <int NG, bool kGate>
__global__ void __launch_bounds__(32 * kQBWarps) k_quant_b(int rows, int Mw, const float *__restrict__ x, long long xws,
                                                           int lda, int K, int Kq, const float *__restrict__ gate,
                                                           long long gws, int8_t *__restrict__ q,
                                                           float *__restrict__ sa, int32_t *__restrict__ za, int rpw,
                                                           int *err) {
  extern __shared__ __align__(128) unsigned char qb_sm[];
  __shared__ __align__(8) uint64_t bar[kQBWarps][kQBD];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const uint32_t rb = (uint32_t)K * 4u;  // row bytes, a multiple of 16
  const float4 *slot0 = reinterpret_cast<const float4 *>(qb_sm + (size_t)wid * kQBD * rb);
  const int r0 = (int)(((long long)blockIdx.x * kQBWarps + wid) * rpw), r1 = min(rows, r0 + rpw);
  if (lane == 0) {
    for (int d = 0; d < kQBD; d++) mbar_init(smem_u32(&bar[wid][d]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  int wl = r0 / Mw, ml = r0 - wl * Mw;  // the next row to copy (lane 0's count)
  int wc = wl, mc = ml;                 // the next row to quantize
  auto issue = [&](int d) {             // lane 0: the next row into slot d
    const float *src = x + wl * xws + (long long)ml * lda;
    if (++ml == Mw) { ml = 0; wl++; }
    const uint32_t b = smem_u32(&bar[wid][d]);
    mbar_expect_tx(b, rb);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(qb_sm + ((size_t)wid * kQBD + d) * rb)),
                 "l"(src), "r"(rb), "r"(b)
                 : "memory");
  };
  if (lane == 0)
    for (int d = 0; d < kQBD && r0 + d < r1; d++) issue(d);
  const int K4 = K >> 2, Kq4 = Kq >> 2, K8 = K & ~7;
  float4 gv[kGate ? NG : 1];
  int gw = -1;
  for (int r = r0; r < r1; r++) {
    const int j = r - r0, d = j % kQBD;
    const bool ok = __all_sync(0xffffffffu, mbar_wait_ns(smem_u32(&bar[wid][d]), (j / kQBD) & 1, kWaitNs));
    if (!ok) {  // record, let the copies still in flight into this warp's slots land, leave
      if (lane == 0) {
        atomicExch(err, BNNK_ERR_QUANT_WAIT);
        for (int t = 0; t < kQBD && r + t < r1; t++)
          mbar_wait_ns(smem_u32(&bar[wid][(j + t) % kQBD]), ((j + t) / kQBD) & 1, kWaitNs);
      }
      __syncwarp();
      return;
    }
    if (kGate && wc != gw) {
      gw = wc;
      const float4 *gp = reinterpret_cast<const float4 *>(gate + wc * gws);
#pragma unroll
      for (int i = 0; i < NG; i++) {
        const int g = lane + 32 * i;
        gv[i] = (i < NG - 1 || g < K4) ? __ldg(gp + g) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (++mc == Mw) { mc = 0; wc++; }
    const float4 *sl = slot0 + (size_t)d * (rb >> 4);
    float4 v[NG];
#pragma unroll
    for (int i = 0; i < NG; i++) {
      const int g = lane + 32 * i;
      if (i < NG - 1 || g < K4) v[i] = sl[g];
    }
    float lo, hi;
    quant_row_in<NG, kGate>(v, gv, lane, K4, lo, hi);
    // every lane's reads of the slot are done (their values are in use above): refill it with row r + kQBD
    __syncwarp();
    if (lane == 0 && r + kQBD < r1) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(d);
    }
    quant_row_out<NG>(v, lo, hi, lane, K4, Kq4, K8, r, q, Kq, sa, za);
  }
}

// The general form (any K, any lda): one thread per row, the reference's loops as written.
__global__ void k_quant_scalar(int rows, int Mw, const float *__restrict__ x, long long xws, int lda, int K, int Kq,
                               const float *__restrict__ gate, long long gws, int8_t *__restrict__ q,
                               float *__restrict__ sa, int32_t *__restrict__ za) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int w = row / Mw, m = row - w * Mw;
  const float *xr = x + w * xws + (long long)m * lda;
  const float *gr = gate ? gate + w * gws : nullptr;
  auto val = [&](int k) { return gr ? __fmul_rn(xr[k], gr[k]) : xr[k]; };
  float lo = __int_as_float(0x7f800000), hi = __int_as_float(0xff800000);
  int k = 0;
  for (; k < (K & ~3); k++) { lo = fmin_nan(lo, val(k)); hi = fmax_nan(hi, val(k)); }  // the 4-wide NEON part
  for (; k < K; k++) { lo = fminf(lo, val(k)); hi = fmaxf(hi, val(k)); }                // the scalar tail
  float inv, s;
  int32_t z;
  quant_params(lo, hi, inv, z, s);
  sa[row] = s;
  za[row] = z;
  int8_t *qr = q + (long long)row * Kq;
  const int K8 = K & ~7;
  for (k = 0; k < K; k++) {
    float t = __fmul_rn(val(k), inv);
    int32_t qi = (int32_t)((uint32_t)(k < K8 ? cvtns(t) : lrintf_i32(t)) + (uint32_t)z);
    qr[k] = (int8_t)(qi < -127 ? -127 : qi > 127 ? 127 : qi);
  }
  for (; k < Kq; k++) qr[k] = (int8_t)z;
}

// ------------------------------------------------------------------ tcgen05 GEMM

constexpr int kMaxStages = 8, kMaxEpi = 4;
constexpr int kMaxThreads = 832;  // 2 + 24 warps: 64 + 128 * ne * nh with ne * nh <= 6
constexpr int kSPMax = 1536;      // widest layer whose epilogue parameters are staged in shared memory

constexpr int kEpiUnits = 3;  // 8-column TMEM loads in flight per epilogue warp (832-thread blocks; 576: kEpiUnits2)
constexpr int kEpiUnits2 = 3;  // (5 measured slower: 2357 -> 2470 µs per v2.4 step)
// the epilogue's per-row partial (min, max) for the next layer's quantizer: 2 tile parities x 6 warps of 128 rows
constexpr size_t kQPartBytes = 2 * 6 * 128 * sizeof(float2);
// wait for this thread's TMEM loads; the registers they fill are operands of the wait, so no use moves above it
#define BNN_R8(u) "+r"(r[u][0]), "+r"(r[u][1]), "+r"(r[u][2]), "+r"(r[u][3]), "+r"(r[u][4]), "+r"(r[u][5]), \
                  "+r"(r[u][6]), "+r"(r[u][7])
__device__ __forceinline__ void tmem_wait(uint32_t (&r)[3][8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : BNN_R8(0), BNN_R8(1), BNN_R8(2)::"memory");
}
__device__ __forceinline__ void tmem_wait(uint32_t (&r)[5][8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : BNN_R8(0), BNN_R8(1), BNN_R8(2), BNN_R8(3), BNN_R8(4)::"memory");
}
#undef BNN_R8
__device__ __forceinline__ void ld8_global(const float *p, float (&v)[8]) {
  asm volatile("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p));
}
__device__ __forceinline__ void st8_global(float *p, const float (&v)[8]) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]),
               "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

struct GemmArgs {
  int rows, Mw, nkb, stages, bn, np, n_tiles, tiles, acc_cols, ne, nh;
  int tmem_alloc;  // TMEM columns allocated: ne * acc_cols rounded up to a power of two (tcgen05.alloc's rule)
  int vec_out, vec_res;  // output / residual rows start on 32-byte boundaries: 8-float stores / loads
  uint32_t idesc;
  const float *sa;
  const int32_t *za;
  bnnk_epilogue e;
  int *err;
  unsigned long long wait_ns;  // the limit of every mbarrier wait (kWaitNs; shorter in the stall test)
  int stall;                   // test hook: the producer issues no load, so every consumer's wait runs out
  // kFQ (the quantizer in the GEMM): fp32 rows of K (a multiple of 4, at most kFQMaxK) arrive by TMA in fs slots of
  // fp32_bytes; the A operand's K block is Kq bytes wide (one block, nkb = 1)
  int K, fs, fp32_bytes, kqz;
};
constexpr int kFQMaxK = 72, kFQSlots = 2, kFQRing = kMaxStages + kMaxEpi;  // K, fp32 slots, sa / za ring

__device__ __forceinline__ long long padded_row(int m, int w, int pad) {
  return pad ? (long long)((m / w) + pad) * (w + 2 * pad) + (m % w) + pad : (long long)m;
}

// The epilogue of NU 8-column units of one row (gemm_s8n.c:105-135): unit k covers the columns c_k .. c_k + 7, c_k =
// 8 (u0 + k nh) from the tile's first column. Dequantize, bias, activation ACT (0 none, 1 SiLU, 2 ReLU), residual
// (RES), store; VEC: 32-byte aligned rows (8-float loads and stores). Branch-free for fixed template arguments, so
// the units' independent chains can overlap. psw / pb / pcs point at the tile's first column of the per-column
// parameters (shared or global memory).
template <int ACT, bool RES, bool VEC, int NU, bool kQ, int EU>
__device__ __forceinline__ void epilogue_units(const uint32_t (&acc)[EU][8], int kofs, int u0, int nh, float sa,
                                               int32_t za, const float *psw, const float *pb, const int32_t *pcs,
                                               float *orow, const float *rrow, const uint32_t *lut, float &lo,
                                               float &hi, int qk) {
  const float2 sa2 = splat2(sa);
  const uint32_t nza = 0u - (uint32_t)za;  // acc - za cs = acc + (-za) cs, one integer multiply-add (mod 2^32)
#pragma unroll
  for (int k = 0; k < NU; k++) {
    const int c = 8 * (u0 + k * nh);
    float rv[8];
    if (RES) {
      if (VEC) {
        ld8_global(rrow + c, rv);
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) rv[j] = __ldg(rrow + c + j);
      }
    }
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float2 sw = *reinterpret_cast<const float2 *>(psw + c + j), bb = *reinterpret_cast<const float2 *>(pb + c + j);
      const int2 cs = *reinterpret_cast<const int2 *>(pcs + c + j);
      // deq4 (gemm_s8n.c:105-114): int32 wrap, exact int -> fp32, sw * sa first, multiply then add (no FMA)
      const float f0 = __int2float_rn((int32_t)(acc[kofs + k][j] + (uint32_t)cs.x * nza));
      const float f1 = __int2float_rn((int32_t)(acc[kofs + k][j + 1] + (uint32_t)cs.y * nza));
      const float2 sc = mul2_rn(sw, sa2);
      float2 v = make_float2(__fadd_rn(__fmul_rn(f0, sc.x), bb.x), __fadd_rn(__fmul_rn(f1, sc.y), bb.y));
      if (ACT == 1) {
        v = silu2(v, lut);
      } else if (ACT == 2) {  // FMAX(v, +0): NaN stays NaN, -0 -> +0
        v.x = (v.x > 0.f || v.x != v.x) ? v.x : 0.f;
        v.y = (v.y > 0.f || v.y != v.y) ? v.y : 0.f;
      }
      y[j] = RES ? __fadd_rn(v.x, rv[j]) : v.x;
      y[j + 1] = RES ? __fadd_rn(v.y, rv[j + 1]) : v.y;
    }
    if (kQ) {  // the row's NaN-propagating min / max over the next layer's K columns (s8n_quant_rows)
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (c + j < qk) { lo = fmin_nan(lo, y[j]); hi = fmax_nan(hi, y[j]); }
    }
    if (VEC) {
      st8_global(orow + c, y);
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) orow[c + j] = y[j];
    }
  }
}

template <int NU, bool kQ, int EU>
__device__ __forceinline__ void epilogue_act(const GemmArgs &a, const uint32_t (&acc)[EU][8], int kofs, int u0,
                                             int nh, float sa, int32_t za, const float *psw, const float *pb,
                                             const int32_t *pcs, float *orow, const float *rrow, const uint32_t *lut,
                                             float &lo, float &hi) {
#define BNN_E(ACT, RES, VEC) \
  epilogue_units<ACT, RES, VEC, NU, false, EU>(acc, kofs, u0, nh, sa, za, psw, pb, pcs, orow, rrow, lut, lo, hi, 0)
  const bool vec = a.vec_out && (!rrow || a.vec_res);
  if (kQ) {  // the rows also quantized for the next layer: linear layers (the host's rule)
    if (rrow && vec) epilogue_units<0, true, true, NU, true, EU>(acc, kofs, u0, nh, sa, za, psw, pb, pcs, orow, rrow, lut,
                                                             lo, hi, a.e.qk);
    else if (rrow) epilogue_units<0, true, false, NU, true, EU>(acc, kofs, u0, nh, sa, za, psw, pb, pcs, orow, rrow, lut,
                                                            lo, hi, a.e.qk);
    else if (vec) epilogue_units<0, false, true, NU, true, EU>(acc, kofs, u0, nh, sa, za, psw, pb, pcs, orow, rrow, lut,
                                                           lo, hi, a.e.qk);
    else epilogue_units<0, false, false, NU, true, EU>(acc, kofs, u0, nh, sa, za, psw, pb, pcs, orow, rrow, lut, lo, hi,
                                                   a.e.qk);
    return;
  }
  if (!vec) {  // rows off 32-byte boundaries (per-op API callers): one general form
    if (rrow) {
      if (a.e.act == 1) BNN_E(1, true, false); else if (a.e.act == 2) BNN_E(2, true, false); else BNN_E(0, true, false);
    } else {
      if (a.e.act == 1) BNN_E(1, false, false); else if (a.e.act == 2) BNN_E(2, false, false); else BNN_E(0, false, false);
    }
    return;
  }
  if (rrow) {
    if (a.e.act == 1) BNN_E(1, true, true); else if (a.e.act == 2) BNN_E(2, true, true); else BNN_E(0, true, true);
  } else {
    if (a.e.act == 1) BNN_E(1, false, true); else if (a.e.act == 2) BNN_E(2, false, true); else BNN_E(0, false, true);
  }
#undef BNN_E
}

// named barrier over nthreads threads with an AND of their predicates (bar.red.and): every thread of the group arrives,
// so a group whose wait failed in some warps still leaves the barrier together
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// The next layer's quantized row from this tile's stored row (s8n_quant_rows): the thread that stored units u0, u0 + nh,
// ... of the row reads them back (its own stores, in order) and writes their quantized bytes; columns from qk on are
// the zero point; the thread of the quarter's first warp also writes the pads past the last unit.
__device__ __forceinline__ void quant_units(const GemmArgs &a, int row, const float *orow, int units, int u0, int nh,
                                            float lo, float hi, bool first) {
  const int qk = a.e.qk, K8 = qk & ~7;
  float inv, s;
  int32_t z;
  quant_params(lo, hi, inv, z, s);
  if (first) { a.e.qsa[row] = s; a.e.qza[row] = z; }
  uint2 *qr = reinterpret_cast<uint2 *>(a.e.qo + (long long)row * a.e.qkq);
  const float2 inv2 = splat2(inv);
  const uint32_t zp = ((uint32_t)z & 0xffu) * 0x01010101u;
  for (int u = u0; u < units; u += nh) {
    const int c = 8 * u;
    if (c >= a.e.qkq) break;
    uint32_t wd[2] = {zp, zp};
    if (c < qk) {
      const float4 t0 = __ldcg(reinterpret_cast<const float4 *>(orow + c));
      const float4 t1 = __ldcg(reinterpret_cast<const float4 *>(orow + c + 4));
      const float2 p0 = mul2_rn(make_float2(t0.x, t0.y), inv2), p1 = mul2_rn(make_float2(t0.z, t0.w), inv2);
      wd[0] = quant_word(p0.x, p0.y, p1.x, p1.y, z, c < K8);
      if (c + 4 < qk) {
        const float2 p2 = mul2_rn(make_float2(t1.x, t1.y), inv2), p3 = mul2_rn(make_float2(t1.z, t1.w), inv2);
        wd[1] = quant_word(p2.x, p2.y, p3.x, p3.y, z, c + 4 < K8);
      }
    }
    qr[u] = make_uint2(wd[0], wd[1]);
  }
  if (first)
    for (int c = 8 * units; c < a.e.qkq; c += 8) qr[c / 8] = make_uint2(zp, zp);
}

// kSP: the per-column parameters (sw, bias, cs; np <= kSPMax columns) are staged in shared memory once per CTA;
// kQ: the epilogue also quantizes the stored rows for the next layer (a.e.qo); kThreads: the block size the registers
// are budgeted for (832: 72 registers a thread; 576, two epilogue warps per TMEM lane quarter and accumulator: 112)
// kFQ: four quantizer warps (warps 2-5, one thread per tile row) turn the fp32 rows, staged by TMA (tma_a is then
// the fp32 map), into the tile's int8 A operand in its shared-memory stage (in the layout that TMA's SW-byte swizzle
// gives a loaded tile), with the rows' scales and zero points in a shared ring for the epilogue
template <int SW, bool kSP, bool kQ, int kThreads = kMaxThreads, bool kFQ = false>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_s8(const __grid_constant__ CUtensorMap tma_a,
                                                           const __grid_constant__ CUtensorMap tma_b,
                                                           const GemmArgs a) {
  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) unsigned long long bar_full[kMaxStages], bar_empty[kMaxStages];
  __shared__ __align__(8) unsigned long long bar_acc_full[kMaxEpi], bar_acc_empty[kMaxEpi];
  __shared__ __align__(8) unsigned long long bar_ffull[kFQ ? kFQSlots : 1], bar_fempty[kFQ ? kFQSlots : 1];
  __shared__ __align__(8) unsigned long long bar_qdone[kFQ ? kFQRing : 1];
  __shared__ float s_qsa[kFQ ? kFQRing : 1][kFQ ? 128 : 1];
  __shared__ int32_t s_qza[kFQ ? kFQRing : 1][kFQ ? 128 : 1];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;
  __shared__ uint32_t s_lut[256];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t base = (smem_u32(dsmem) + 1023u) & ~1023u;
  const uint32_t a_bytes = 128u * SW, stage_bytes = (128u + a.bn) * SW;
  const int S = a.stages;
  // parameters after the stage ring: sw [np], bias [np], cs [np]
  uint8_t *par = dsmem + (base - smem_u32(dsmem)) + (size_t)S * stage_bytes;
  float *p_sw = reinterpret_cast<float *>(par), *p_b = p_sw + a.np;
  int32_t *p_cs = reinterpret_cast<int32_t *>(p_b + a.np);
  // the epilogue threads' partial (min, max) of their rows, per tile parity, group and warp: [2][ne][nh][128]
  float2 *q_part = reinterpret_cast<float2 *>(par + (kSP ? (size_t)12 * a.np : 0));
  // kFQ: the fp32 row slots (128-byte aligned) after the partials
  const uint32_t fbase = (smem_u32(par) + (kSP ? 12u * a.np : 0u) + (uint32_t)kQPartBytes + 127u) & ~127u;
  if (kSP) {
    for (int i = threadIdx.x; i < a.np; i += blockDim.x) {
      p_sw[i] = __ldg(a.e.sw + i);
      p_b[i] = __ldg(a.e.bias + i);
      p_cs[i] = __ldg(a.e.cs + i);
    }
  }

  for (int i = threadIdx.x; i < 256; i += blockDim.x) s_lut[i] = g_frecpe_lut[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(smem_u32(&bar_full[s]), kFQ ? 1 + 4 : 1);  // kFQ: the B load and the four quantizer warps
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    for (int g = 0; g < a.ne; g++) {
      mbar_init(smem_u32(&bar_acc_full[g]), 1);
      mbar_init(smem_u32(&bar_acc_empty[g]), 4 * a.nh);
    }
    if (kFQ) {
      for (int f = 0; f < kFQSlots; f++) { mbar_init(smem_u32(&bar_ffull[f]), 1); mbar_init(smem_u32(&bar_fempty[f]), 4); }
      for (int r = 0; r < kFQRing; r++) mbar_init(smem_u32(&bar_qdone[r]), 4);
    }
    abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(a.tmem_alloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0 && !a.stall) {  // TMA producer
      int it = 0;
      for (int t = blockIdx.x; t < a.tiles && !abort_s; t += gridDim.x) {
        const int m0 = (t / a.n_tiles) * 128, n0 = (t % a.n_tiles) * a.bn;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % S;
          if (it >= S && !mbar_wait_ns(smem_u32(&bar_empty[s]), ((it / S) - 1) & 1, a.wait_ns)) {
            atomicExch(a.err, BNNK_ERR_TMA_WAIT);
            abort_s = 1;
            break;
          }
          const uint32_t st = base + s * stage_bytes, bar = smem_u32(&bar_full[s]);
          if (kFQ) {  // the tile's fp32 rows into their slot, B into the stage (nkb = 1: it counts tiles); both waits
                      // come first, so a wait that runs out leaves no copy in flight
            const int f = it % kFQSlots;
            if (it >= kFQSlots && !mbar_wait_ns(smem_u32(&bar_fempty[f]), ((it / kFQSlots) - 1) & 1, a.wait_ns)) {
              atomicExch(a.err, BNNK_ERR_TMA_WAIT);
              abort_s = 1;
              break;
            }
            mbar_expect_tx(smem_u32(&bar_ffull[f]), (uint32_t)a.fp32_bytes);  // rows past the last read zero
            tma_load_2d(fbase + f * (uint32_t)a.fp32_bytes, &tma_a, smem_u32(&bar_ffull[f]), 0, m0);
            mbar_expect_tx(bar, stage_bytes - a_bytes);
            tma_load_2d(st + a_bytes, &tma_b, bar, 0, n0);
            continue;
          }
          mbar_expect_tx(bar, stage_bytes);  // the full boxes: bytes past Kq arrive as zero fill
          tma_load_2d(st, &tma_a, bar, kb * SW, m0);
          tma_load_2d(st + a_bytes, &tma_b, bar, kb * SW, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < a.tiles && !abort_s; t += gridDim.x, lt++) {
        const int g = lt % a.ne, use = lt / a.ne;
        if (use > 0 && !mbar_wait_ns(smem_u32(&bar_acc_empty[g]), (use - 1) & 1, a.wait_ns)) {
          atomicExch(a.err, BNNK_ERR_MMA_WAIT);
          abort_s = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tacc = tmem + (uint32_t)(g * a.acc_cols);
        bool ok = true;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % S;
          if (!mbar_wait_ns(smem_u32(&bar_full[s]), (it / S) & 1, a.wait_ns)) {
            atomicExch(a.err, BNNK_ERR_MMA_WAIT);
            abort_s = 1;
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = base + s * stage_bytes;
#pragma unroll
          for (int kk = 0; kk < SW / 32; kk++)
            mma_i8(tacc, smem_desc<SW>(st + kk * 32), smem_desc<SW>(st + a_bytes + kk * 32), a.idesc, (kb | kk) != 0);
          mma_commit(smem_u32(&bar_empty[s]));
        }
        if (!ok) break;
        mma_commit(smem_u32(&bar_acc_full[g]));  // arrives when this tile's MMAs have completed
      }
    }
  } else if (kFQ && warp < 6) {
    // quantizer: thread r = row r of each tile, s8n_quant_rows on the row's K fp32 values as k_quant does (the
    // NaN-propagating min / max, the row parameters, FCVTNS on the 8-wide part and lrintf past it, pads = the zero
    // point), the Kq bytes written to the stage in 16-byte chunks at their swizzled places
    const int r = threadIdx.x - 64;
    const int K = a.K, K4 = K >> 2, K8 = K & ~7, nch = SW / 16;
    int lt = 0;
    for (int t = blockIdx.x; t < a.tiles && !abort_s; t += gridDim.x, lt++) {
      const int s = lt % S, f = lt % kFQSlots, rs = lt % kFQRing;
      bool ok = mbar_wait_ns(smem_u32(&bar_ffull[f]), (lt / kFQSlots) & 1, a.wait_ns);
      if (ok && lt >= S) ok = mbar_wait_ns(smem_u32(&bar_empty[s]), ((lt / S) - 1) & 1, a.wait_ns);
      ok = __all_sync(0xffffffffu, ok && !abort_s);
      if (!ok) {
        if (lane == 0) { atomicExch(a.err, BNNK_ERR_TMA_WAIT); abort_s = 1; }
        break;
      }
      const float4 *xr = reinterpret_cast<const float4 *>(dsmem + (fbase + f * (uint32_t)a.fp32_bytes - smem_u32(dsmem))) +
                         (size_t)r * K4;
      float lo = __int_as_float(0x7f800000), hi = __int_as_float(0xff800000);
      for (int g4 = 0; g4 < K4; g4++) {
        const float4 v = xr[g4];
        lo = fmin_nan(lo, fmin_nan(fmin_nan(v.x, v.y), fmin_nan(v.z, v.w)));
        hi = fmax_nan(hi, fmax_nan(fmax_nan(v.x, v.y), fmax_nan(v.z, v.w)));
      }
      float inv, sc;
      int32_t z;
      quant_params(lo, hi, inv, z, sc);
      s_qsa[rs][r] = sc;
      s_qza[rs][r] = z;
      const uint32_t zp = ((uint32_t)z & 0xffu) * 0x01010101u;
      uint8_t *arow = dsmem + (base + s * stage_bytes - smem_u32(dsmem)) + (size_t)r * SW;
      for (int c = 0; c < nch; c++) {  // 16-byte chunk c of the row: 16 values, 4 words
        uint32_t wd[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int g4 = 4 * c + j;
          if (g4 < K4) {
            const float4 v = xr[g4];
            wd[j] = quant_word(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv), __fmul_rn(v.w, inv), z,
                               4 * g4 < K8);
          } else {
            wd[j] = zp;  // pads past K (to the block's SW bytes): the zero point
          }
        }
        // the swizzle of a TMA-written K-major tile: chunk c of row r sits at chunk c ^ (row bits) of its row
        const int pc = SW == 128 ? (c ^ (r & 7)) : SW == 64 ? (c ^ ((r >> 1) & 3)) : (c ^ ((r >> 2) & 1));
        *reinterpret_cast<uint4 *>(arow + 16 * pc) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the stores, seen by the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&bar_full[s]));
        mbar_arrive(smem_u32(&bar_fempty[f]));
        mbar_arrive(smem_u32(&bar_qdone[rs]));
      }
    }
  } else if (warp - 2 - (kFQ ? 4 : 0) < 4 * a.ne * a.nh) {
    // epilogue: group g drains accumulator g; its 4 * nh warps split the 8-column units of a tile round robin, the
    // warp's TMEM lane quarter q (= warp % 4) fixing its 32 rows
    const int e = warp - 2 - (kFQ ? 4 : 0), g = e / (4 * a.nh), h = (e % (4 * a.nh)) / 4, q = warp % 4;
    constexpr bool fq = kQ;  // the tile's rows are quantized for the next layer after its epilogue
    int use = 0;
    for (int t = blockIdx.x + g * gridDim.x; t < a.tiles; t += a.ne * gridDim.x, use++) {
      const int m0 = (t / a.n_tiles) * 128, n0 = (t % a.n_tiles) * a.bn;
      const int row = m0 + q * 32 + lane;
      const bool live = row < a.rows;
      int w = 0, mm = 0;
      float sa = 0.f;
      int32_t za = 0;
      if (live) {
        w = row / a.Mw;
        mm = row - w * a.Mw;
        if (!kFQ) {
          sa = __ldg(a.sa + row);
          za = __ldg(a.za + row);
        }
      }
      bool ok = mbar_wait_ns(smem_u32(&bar_acc_full[g]), use & 1, a.wait_ns);
      if (kFQ) {  // the tile's row parameters, from the quantizer warps
        const int lt = g + use * a.ne;
        ok = ok && mbar_wait_ns(smem_u32(&bar_qdone[lt % kFQRing]), (lt / kFQRing) & 1, a.wait_ns);
        sa = s_qsa[lt % kFQRing][q * 32 + lane];
        za = s_qza[lt % kFQRing][q * 32 + lane];
      }
      ok = __all_sync(0xffffffffu, ok && !abort_s);  // one outcome per warp (abort_s may change between lanes' reads)
      if (!ok) {
        if (lane == 0) { atomicExch(a.err, BNNK_ERR_EPI_WAIT); abort_s = 1; }
        if (!fq) break;
        bar_and(1 + g, 128 * a.nh, false);  // the group's other warps leave with this one
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int units = (min(a.bn, a.np - n0) + 7) / 8;  // np is a multiple of 8
      float *orow = a.e.out + (long long)w * a.e.ows + padded_row(mm, a.e.ow, a.e.opad) * a.e.ldo + n0;
      const float *rrow = a.e.res ? a.e.res + (long long)w * a.e.rws + padded_row(mm, a.e.rw, a.e.rpad) * a.e.ldr + n0
                                  : nullptr;
      const float *qsw = kSP ? p_sw + n0 : a.e.sw + n0, *qb = kSP ? p_b + n0 : a.e.bias + n0;
      const int32_t *qcs = kSP ? p_cs + n0 : a.e.cs + n0;
      const uint32_t tq = tmem + (uint32_t)(g * a.acc_cols) + ((uint32_t)(q * 32) << 16);
      float lo = __uint_as_float(0x7f800000u), hi = __uint_as_float(0xff800000u);
      // a tile whose units take one pass frees its accumulator as soon as the loads are in registers, so the next
      // tile's MMAs overlap the arithmetic
      constexpr int EU = kThreads == kMaxThreads ? kEpiUnits : kEpiUnits2;  // units in flight
      const bool single = units <= EU * a.nh;
      for (int u0 = h; u0 < units; u0 += EU * a.nh) {
        uint32_t acc[EU][8];
#pragma unroll
        for (int k = 0; k < EU; k++) {
          const int u = u0 + k * a.nh;
          if (u < units) tmem_ld8(tq + (uint32_t)(8 * u), acc[k]);
        }
        tmem_wait(acc);
        if (single) {
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[g]));
        }
        if (live) {
          if (u0 + (EU - 1) * a.nh < units) {  // every unit of the batch is a real column block
            epilogue_act<EU, kQ, EU>(a, acc, 0, u0, a.nh, sa, za, qsw, qb, qcs, orow, rrow, s_lut, lo, hi);
          } else {
#pragma unroll
            for (int k = 0; k < EU; k++)
              if (u0 + k * a.nh < units)
                epilogue_act<1, kQ, EU>(a, acc, k, u0 + k * a.nh, a.nh, sa, za, qsw, qb, qcs, orow, rrow, s_lut, lo, hi);
          }
        }
      }
      if (!single || h >= units) {  // after the last pass, or a warp with no unit in this tile
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[g]));
      }
      if (fq) {
        // the row's min / max from its nh threads' partials (the barrier orders their shared stores before the reads;
        // a warp whose wait failed arrives with false and all leave), then this thread's units quantized
        float2 *pp = q_part + ((size_t)((use & 1) * a.ne + g) * a.nh) * 128 + q * 32 + lane;
        pp[h * 128] = make_float2(lo, hi);
        if (!bar_and(1 + g, 128 * a.nh, true)) break;
        if (live) {
          for (int hh = 0; hh < a.nh; hh++) {
            const float2 v = pp[hh * 128];
            lo = fmin_nan(lo, v.x);
            hi = fmax_nan(hi, v.y);
          }
          quant_units(a, row, orow, units, h, a.nh, lo, hi, h == 0);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_alloc));
}

// ------------------------------------------------------------------ elementwise test kernel

__global__ void k_test_fn(int fn, int n, const float *x, float *y) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = x[i], r;
  switch (fn) {
  case 0: r = silu<false>(v, nullptr); break;
  case 1: r = silu<true>(v, g_frecpe_lut); break;
  case 2: r = sigmoid(v); break;
  case 3: r = frecpe(v); break;
  case 4: r = log2_acc(v); break;
  case 5: r = exp2_acc(v); break;
  case 6: r = glibc_expf(v, c_expf_tab); break;
  case 7: r = silu2(make_float2(v, -v), g_frecpe_lut).x; break;
  case 8: r = fma2_rn(make_float2(v, -v), splat2(1.7f), splat2(0.3f)).x; break;
  case 9: r = ln_cr(v); break;
  default: r = 0.f;
  }
  y[i] = r;
}

}  // namespace bnn

using namespace bnn;

// ------------------------------------------------------------------ launchers

extern "C" int bnnk_fp32_tables_init(const unsigned long long *tab, const uint32_t *lut);

extern "C" int bnnk_device_init(void) {
  unsigned long long tab[32];
  for (int i = 0; i < 32; i++) {
    double v = exp2((double)i / 32);  // host libm, as glibc's table
    unsigned long long u;
    memcpy(&u, &v, 8);
    tab[i] = u - ((unsigned long long)i << 47);
  }
  cudaError_t e = cudaMemcpyToSymbol(c_expf_tab, tab, sizeof tab);
  if (e) return e;
  uint32_t lut[256];
  for (uint32_t i = 0; i < 256; i++) {
    uint32_t a = 256 + i, b = (1u << 19) / (2 * a + 1);
    lut[i] = (((b + 1) >> 1) & 0xffu) << 15;
  }
  e = cudaMemcpyToSymbol(g_frecpe_lut, lut, sizeof lut);
  if (e) return e;
  e = (cudaError_t)bnnk_fp32_tables_init(tab, lut);
  if (!e) e = (cudaError_t)bnnk_v3_tables_init(tab, lut);
  return e ? e : bnnk_f16_tables_init(tab);
}

// k_quant_b's launch: 8 warps a block, the blocks that the slots' shared memory lets one SM hold on every SM, and a
// contiguous run of rows per warp
template <int NG>
static int launch_quant_b_t(int rows, int Mw, const float *x, long long xws, int lda, int K, int Kq, const float *gate,
                            long long gws, int8_t *q, float *sa, int32_t *za, int *err, bnn_stream_t st) {
  const size_t smem = (size_t)kQBWarps * kQBD * K * 4;
  static SmemAttr attr_g, attr_u;
  const cudaError_t e = gate ? attr_g.ensure(k_quant_b<NG, true>, smem) : attr_u.ensure(k_quant_b<NG, false>, smem);
  if (e) return e;
  int per_sm = (int)((227 * 1024) / (smem + kQBWarps * kQBD * 8 + 1024));
  per_sm = per_sm < 1 ? 1 : per_sm > 8 ? 8 : per_sm;
  const long long warps_max = (long long)num_sms() * per_sm * kQBWarps;
  const int rpw = (int)((rows + warps_max - 1) / warps_max);
  const long long warps = (rows + rpw - 1) / rpw;
  const unsigned grid = (unsigned)((warps + kQBWarps - 1) / kQBWarps);
  if (gate) k_quant_b<NG, true><<<grid, 32 * kQBWarps, smem, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, rpw, err);
  else k_quant_b<NG, false><<<grid, 32 * kQBWarps, smem, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, rpw, err);
  return cudaGetLastError();
}
static int launch_quant_b(int rows, int Mw, const float *x, long long xws, int lda, int K, int Kq, const float *gate,
                          long long gws, int8_t *q, float *sa, int32_t *za, int *err, bnn_stream_t st) {
  switch ((K / 4 + 31) / 32) {  // float4 groups per lane
#define BNN_QB(N) \
  case N: return launch_quant_b_t<N>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, err, st)
    BNN_QB(1); BNN_QB(2); BNN_QB(3); BNN_QB(4); BNN_QB(5); BNN_QB(6);
    BNN_QB(7); BNN_QB(8); BNN_QB(9); BNN_QB(10); BNN_QB(11); BNN_QB(12);
#undef BNN_QB
  default: return BNNK_NOT_FUSED;
  }
}

extern "C" int bnnk_quant(int rows, int Mw, const float *x, long long xws, int lda, int K, int Kq, const float *gate,
                          long long gws, int8_t *q, float *sa, int32_t *za, int *err, bnn_stream_t st) {
  if (rows <= 0) return 0;
  const bool vec = K % 4 == 0 && lda % 4 == 0 && xws % 4 == 0 && (!gate || gws % 4 == 0) && Kq % 4 == 0 &&
                   ((uintptr_t)x & 15) == 0 && (!gate || ((uintptr_t)gate & 15) == 0);
  const int nch = Kq / 16;  // 16-byte chunks of a quantized row
  const int K4 = K / 4, ng = (K4 + 31) / 32;
  // tuning overrides (sweeps): BNN_QUANT_W=0 keeps wide rows on the lane-group form; BNN_QUANT_RPW=n rows per warp
  const char *ew = getenv("BNN_QUANT_W"), *er = getenv("BNN_QUANT_RPW"), *ev = getenv("BNN_QUANT_V");
  // rows of 128-1536 with an error word for the bounded waits: staged by bulk copies (k_quant_b; measured on the v2.4
  // step's gated layers: K 288 74 -> 66 µs per op, K 864 48 -> 44, K 1536 37.4 -> 33.3; BNN_QUANT_V=0 turns it off)
  if (err && vec && K >= 128 && K <= 1536 && Kq % 4 == 0 && ((uintptr_t)q & 3) == 0 && !(ev && ev[0] == '0')) {
    const int rc = launch_quant_b(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, err, st);
    if (rc != BNNK_NOT_FUSED) return rc;
  }
  if (vec && K >= 128 && K <= 1024 && Kq % 4 == 0 && ((uintptr_t)q & 3) == 0 && !(ew && ew[0] == '0')) {
    // wide rows, a warp per row; rows per warp from a sweep (98k rows of 288: 4 best, 25k of 864: 2, 256 of 1024: 1;
    // rows of 1536 were faster in the lane-group form)
    int rpw = rows / (num_sms() * 64);
    rpw = rpw < 1 ? 1 : rpw > 4 ? 4 : rpw;
    if (er && atoi(er) >= 1) rpw = atoi(er);
    const int warps = (rows + rpw - 1) / rpw;
    const unsigned grid = (unsigned)((warps + 7) / 8);
#define BNN_QW(NGV)                                                                                           \
  if (gate && NGV == 3) k_quant_w<3, true, 2><<<grid, 256, 0, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, rpw); \
  else if (gate) k_quant_w<NGV, true, 1><<<grid, 256, 0, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, rpw); \
  else k_quant_w<NGV, false, 1><<<grid, 256, 0, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za, rpw)
    switch (ng) {  // K in [128, 1024]: 1 .. 8 float4 groups per lane
    case 1: BNN_QW(1); break;
    case 2: BNN_QW(2); break;
    case 3: BNN_QW(3); break;
    case 4: BNN_QW(4); break;
    case 5: BNN_QW(5); break;
    case 6: BNN_QW(6); break;
    case 7: BNN_QW(7); break;
    default: BNN_QW(8); break;
    }
#undef BNN_QW
    return cudaGetLastError();
  }
  if (!vec || Kq % 16 || nch > 32 * 3) {
    k_quant_scalar<<<(rows + 127) / 128, 128, 0, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za);
    return cudaGetLastError();
  }
  // lanes per row: the largest power of two up to 32 that is not above the chunk count; chunks per lane from that
  int L = 1;
  while (L < 32 && 2 * L <= nch) L *= 2;
  const int NC = (nch + L - 1) / L;
  const unsigned grid = (unsigned)(((long long)rows * L + 255) / 256);
#define BNN_Q(LL, NN) k_quant<LL, NN><<<grid, 256, 0, st>>>(rows, Mw, x, xws, lda, K, Kq, gate, gws, q, sa, za)
#define BNN_QL(LL) \
  if (NC == 1) BNN_Q(LL, 1); else if (NC == 2) BNN_Q(LL, 2); else BNN_Q(LL, 3)
  switch (L) {
  case 1: BNN_QL(1); break;
  case 2: BNN_QL(2); break;
  case 4: BNN_QL(4); break;
  case 8: BNN_QL(8); break;
  case 16: BNN_QL(16); break;
  default: BNN_QL(32); break;
  }
#undef BNN_QL
#undef BNN_Q
  return cudaGetLastError();
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode(void) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  }
  return fn;
}

int bnn::encode_2d_ld(void *map, const void *base, int inner, long long ld, int rows, int box_inner, int box_rows,
                      int sw) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUtensorMapSwizzle swz = sw == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : sw == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                                             : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc((CUtensorMap *)map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : cudaErrorInvalidValue;
}
static int encode_2d(void *map, const void *base, int inner, int rows, int box_inner, int box_rows, int sw) {
  return encode_2d_ld(map, base, inner, inner, rows, box_inner, box_rows, sw);
}

// N tiling: as few tiles of at most 256 columns as possible, equal widths rounded up to 16; then, while the tiles of
// rows_cap rows (128 each) do not give every SM one and tiles stay at least 32 columns wide, one N tile more (a small
// GEMM is latency bound: narrower tiles spread it over more SMs, the extra reads of A come from L2)
static void n_tiling(int np, int rows_cap, int *n_tiles, int *bn) {
  const int n16 = (np + 15) & ~15, m_tiles = (rows_cap + 127) / 128, sms = 148;
  int t = (n16 + 255) / 256;
  while ((long long)m_tiles * t < sms && ((n16 + t) / (t + 1) + 15) / 16 * 16 >= 32) t++;
  *n_tiles = t;
  const int b = (n16 + t - 1) / t;
  *bn = (b + 15) & ~15;
}

extern "C" int bnnk_gemm_n_tiles(const bnnk_gemm_plan *p) { return p->n_tiles; }

extern "C" int bnnk_gemm_weight_rows(int np, int rows_cap) {
  int t, bn;
  n_tiling(np, rows_cap, &t, &bn);
  return t * bn;
}

static int g_num_sms = 0;
int bnn::num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

// tcgen05.alloc takes a power of two from 32 to 512 columns
static int tmem_pow2(int cols) {
  int c = 32;
  while (c < cols) c *= 2;
  return c;
}

// epilogue shape: two accumulators (the MMAs of the next tile overlap the epilogue of the last) with two warps per
// TMEM lane quarter each: 576 threads, whose 112 registers a thread keep the epilogue's values and parameters in
// registers (at three warps, 832 threads and 72 registers, it spilled and reloaded kernel parameters: the v2.4 step's
// PW_S8 ops measured 2390 -> 2357 µs with two)
static void epi_shape(int tmem_cols, int *ne, int *nh) {
  const int e = 2;  // tmem_cols <= 256: two accumulators always fit the 512 columns
  const int h = 2;
  const char *env = getenv("BNN_GEMM_EPI");  // "ne,nh" override for tuning sweeps
  int ee = 0, hh = 0;
  if (env && sscanf(env, "%d,%d", &ee, &hh) == 2 && ee >= 1 && ee <= kMaxEpi && tmem_pow2(ee * tmem_cols) <= 512 &&
      hh >= 1 && 64 + 128 * ee * hh <= kMaxThreads) {
    *ne = ee;
    *nh = hh;
    return;
  }
  *ne = e;
  *nh = h;
}

extern "C" int bnnk_gemm_plan_init(bnnk_gemm_plan *p, const int8_t *q, int rows_cap, int kq, const int8_t *w, int n,
                                   int np) {
  memset(p, 0, sizeof *p);
  if (kq % 32 || rows_cap <= 0 || n <= 0 || np < n) return cudaErrorInvalidValue;
  p->kq = kq;
  // K blocks of 128 bytes (the widest swizzle); a ragged last block reads TMA zero fill past Kq on both operands,
  // which adds nothing to the sums. K of 32 or 64 bytes: one block of exactly that width.
  p->sw = kq <= 32 ? 32 : kq <= 64 ? 64 : 128;
  p->nkb = (kq + p->sw - 1) / p->sw;
  p->n = n;
  p->np = np;
  n_tiling(np, rows_cap, &p->n_tiles, &p->bn);
  p->tmem_cols = p->bn <= 32 ? 32 : p->bn <= 64 ? 64 : p->bn <= 128 ? 128 : 256;
  epi_shape(p->tmem_cols, &p->ne, &p->nh);
  p->sp = np <= kSPMax;
  const size_t par = p->sp ? (size_t)12 * np : 0;
  const size_t stage = (size_t)(128 + p->bn) * p->sw;
  int s = (int)((200 * 1024 - par) / stage);
  p->stages = s < 2 ? 2 : s > kMaxStages ? kMaxStages : s;
  p->smem = (size_t)p->stages * stage + 1024 + par + kQPartBytes;
  p->idesc = idesc_i8(p->bn);
  const int wrows = p->n_tiles * p->bn;  // the weight buffer holds n_tiles * bn rows (zero beyond n)
  int e = encode_2d(p->tma_a, q, kq, rows_cap, p->sw, 128, p->sw);
  if (!e) e = encode_2d(p->tma_b, w, kq, wrows, p->sw, p->bn, p->sw);
  return e;
}

template <int SW, bool kSP, bool kQ, int kThreads>
static int launch_gemm_t(const bnnk_gemm_plan *p, const GemmArgs &a, bnn_stream_t st) {
  // the dynamic shared memory this instantiation may use so far, per device (static + dynamic <= 227 KB)
  static SmemAttr attr;
  const cudaError_t e = attr.ensure(k_gemm_s8<SW, kSP, kQ, kThreads>, p->smem);
  if (e) return e;
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  k_gemm_s8<SW, kSP, kQ, kThreads><<<grid, 64 + 128 * a.ne * a.nh, p->smem, st>>>(
      *(const CUtensorMap *)p->tma_a, *(const CUtensorMap *)p->tma_b, a);
  return cudaGetLastError();
}
template <int SW, bool kSP, bool kQ>
static int launch_gemm_q(const bnnk_gemm_plan *p, const GemmArgs &a, bnn_stream_t st) {
  if (!kQ && 64 + 128 * a.ne * a.nh <= 576) return launch_gemm_t<SW, kSP, false, 576>(p, a, st);
  return launch_gemm_t<SW, kSP, kQ, kMaxThreads>(p, a, st);
}
template <int SW, bool kSP>
static int launch_gemm(const bnnk_gemm_plan *p, const GemmArgs &a, bnn_stream_t st) {
  return a.e.qo ? launch_gemm_q<SW, kSP, true>(p, a, st) : launch_gemm_q<SW, kSP, false>(p, a, st);
}

static bool aligned32(const float *ptr, long long ws, int ld) {
  return ((uintptr_t)ptr & 31) == 0 && ws % 8 == 0 && ld % 8 == 0;
}

// test hook: the next GEMM launch of this process stalls (bnnk_debug_stall_next_gemm)
static int g_stall_next = 0;
extern "C" void bnnk_debug_stall_next_gemm(void) { __atomic_store_n(&g_stall_next, 1, __ATOMIC_RELAXED); }

extern "C" int bnnk_gemm(const bnnk_gemm_plan *p, int rows, int Mw, const float *sa, const int32_t *za,
                         const bnnk_epilogue *e, int *err, bnn_stream_t st) {
  if (rows <= 0) return 0;
  GemmArgs a;
  a.stall = __atomic_exchange_n(&g_stall_next, 0, __ATOMIC_RELAXED);
  a.wait_ns = a.stall ? 200000ull : kWaitNs;  // a stalled launch gives up after 200 us
  a.rows = rows;
  a.Mw = Mw;
  a.nkb = p->nkb;
  a.stages = p->stages;
  a.bn = p->bn;
  a.np = p->np;
  a.n_tiles = p->n_tiles;
  a.tiles = ((rows + 127) / 128) * p->n_tiles;
  a.acc_cols = p->tmem_cols;
  a.ne = p->ne;
  a.nh = p->nh;
  a.tmem_alloc = tmem_pow2(p->ne * p->tmem_cols);
  if (a.tmem_alloc > 512) return cudaErrorInvalidValue;
  if (e->qo && (p->n_tiles != 1 || e->opad || e->qk <= 0 || e->qk % 4 || e->qk > 256 || e->qk > p->n ||
                e->qkq < e->qk || e->qkq % 4 || ((uintptr_t)e->out & 15) || e->ldo % 4 || e->ows % 4 ||
                ((uintptr_t)e->qo & 3) || !e->qsa || !e->qza))
    return cudaErrorInvalidValue;
  a.vec_out = aligned32(e->out, e->ows, e->ldo);
  a.vec_res = e->res ? aligned32(e->res, e->rws, e->ldr) : 0;
  a.idesc = p->idesc;
  a.sa = sa;
  a.za = za;
  a.e = *e;
  a.err = err;
  if (p->sp) {
    switch (p->sw) {
    case 128: return launch_gemm<128, true>(p, a, st);
    case 64: return launch_gemm<64, true>(p, a, st);
    default: return launch_gemm<32, true>(p, a, st);
    }
  }
  switch (p->sw) {
  case 128: return launch_gemm<128, false>(p, a, st);
  case 64: return launch_gemm<64, false>(p, a, st);
  default: return launch_gemm<32, false>(p, a, st);
  }
}

// The ungated PW_S8 with its quantizer inside the GEMM (kFQ): one launch, the fp32 rows read once by TMA, no int8
// round trip through global memory. For one K block (Kq <= 128), K % 4 == 0 and K <= kFQMaxK, rows of lda floats
// (lda % 4 == 0) stored back to back over the windows (xws == Mw lda), 16-byte aligned, and a linear epilogue: on the
// SiLU layers the quantizer warps take issue slots from an epilogue that is already issue-bound (measured: b1.1's
// expansion 220 -> 254 µs fused, the 1x1 layers with a residual 91 -> 80 µs). BNNK_NOT_FUSED when a layer is outside
// that (the caller then quantizes and multiplies in two launches); BNN_FQ=0 turns the form off, BNN_FQ=2 admits SiLU
// layers too (tuning).
template <int SW, bool kSP>
static int launch_fq(const bnnk_gemm_plan *p, const GemmArgs &a, const CUtensorMap &map, size_t smem,
                     bnn_stream_t st) {
  constexpr int kT = 64 + 128 + 128 * 2 * 2;  // producer + MMA warps, 4 quantizer warps, two groups of 8
  static SmemAttr attr;
  const cudaError_t e = attr.ensure(k_gemm_s8<SW, kSP, false, kT, true>, smem);
  if (e) return e;
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  k_gemm_s8<SW, kSP, false, kT, true><<<grid, kT, smem, st>>>(map, *(const CUtensorMap *)p->tma_b, a);
  return cudaGetLastError();
}

extern "C" int bnnk_pw_s8_fq(const bnnk_gemm_plan *p, int rows, int Mw, const float *x, long long xws, int lda, int K,
                             const bnnk_epilogue *e, int *err, bnn_stream_t st) {
  static int env = -1;
  if (env < 0) {
    const char *s = getenv("BNN_FQ");
    env = s ? atoi(s) : 1;
  }
  if (!env || (env == 1 && e->act != 0) || rows <= 0 || p->nkb != 1 || K % 4 || K < 4 || K > kFQMaxK || lda % 4 ||
      lda < K || xws != (long long)Mw * lda || ((uintptr_t)x & 15) || e->qo)
    return BNNK_NOT_FUSED;
  GemmArgs a;
  a.stall = __atomic_exchange_n(&g_stall_next, 0, __ATOMIC_RELAXED);  // the test hook, as for bnnk_gemm
  a.wait_ns = a.stall ? 200000ull : kWaitNs;
  a.rows = rows;
  a.Mw = Mw;
  a.nkb = 1;
  a.bn = p->bn;
  a.np = p->np;
  a.n_tiles = p->n_tiles;
  a.tiles = ((rows + 127) / 128) * p->n_tiles;
  a.acc_cols = p->tmem_cols;
  a.ne = 2;
  a.nh = 2;
  a.tmem_alloc = tmem_pow2(a.ne * p->tmem_cols);
  if (a.tmem_alloc > 512) return BNNK_NOT_FUSED;
  a.vec_out = aligned32(e->out, e->ows, e->ldo);
  a.vec_res = e->res ? aligned32(e->res, e->rws, e->ldr) : 0;
  a.idesc = p->idesc;
  a.sa = nullptr;
  a.za = nullptr;
  a.e = *e;
  a.err = err;
  a.K = K;
  a.fs = kFQSlots;
  a.fp32_bytes = 128 * K * 4;
  a.kqz = p->kq;
  // shared memory: the stage ring, the parameters, the partials, the fp32 slots (the static arrays need ~13 KB)
  const size_t stage = (size_t)(128 + p->bn) * p->sw, par = p->sp ? (size_t)12 * p->np : 0;
  const size_t fixed = 1024 + par + kQPartBytes + 128 + (size_t)kFQSlots * a.fp32_bytes;
  const size_t dyn_max = 227 * 1024 - 16 * 1024;
  if (fixed + 2 * stage > dyn_max) return BNNK_NOT_FUSED;
  int s = (int)((dyn_max - fixed) / stage);
  a.stages = s > kMaxStages ? kMaxStages : s;
  const size_t smem = fixed + (size_t)a.stages * stage;
  // the fp32 rows: [rows][K] floats at row stride lda, boxes of 128 rows (rows past the last read zero)
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode();
  if (!enc) return BNNK_NOT_FUSED;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)lda * 4};
  cuuint32_t box[2] = {(cuuint32_t)K, 128}, es[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(x), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return BNNK_NOT_FUSED;
  if (p->sp) {
    switch (p->sw) {
    case 128: return launch_fq<128, true>(p, a, map, smem, st);
    case 64: return launch_fq<64, true>(p, a, map, smem, st);
    default: return launch_fq<32, true>(p, a, map, smem, st);
    }
  }
  switch (p->sw) {
  case 128: return launch_fq<128, false>(p, a, map, smem, st);
  case 64: return launch_fq<64, false>(p, a, map, smem, st);
  default: return launch_fq<32, false>(p, a, map, smem, st);
  }
}

// ------------------------------------------------------------------ PW_S8 on file-scope scratch
// Some hosts must not allocate device memory once they run: a live-audio loop scoring each 3 s window as it
// arrives cannot absorb cudaMalloc / cudaFree, which may synchronise the whole device and take unbounded time, and a
// server that sized its device memory at start-up for a fixed set of streams must not grow on the first use of an
// op. For them the quantized activations of a PW_S8 run (q, and the per-row scale sa and zero point za) live in this
// one static array, which exists as soon as the module is loaded. Layout: sa [BNNK_STATIC_ROWS] f32, then za
// [BNNK_STATIC_ROWS] i32, then q: rows of kq int8 bytes, at most BNNK_STATIC_QBYTES in all. Nothing in it has to start
// at zero: the quantizer writes every q byte (pads included), sa and za of each row the GEMM's stored rows read; rows
// of a tile past the call's last row only feed accumulator rows that the epilogue does not store.
static __device__ __align__(256) unsigned char g_pw_scratch[8 * BNNK_STATIC_ROWS + BNNK_STATIC_QBYTES];

constexpr int kScratchDevices = 64;
static unsigned char *g_pw_scratch_at[kScratchDevices];  // the array's device address, per device (set-up)
static std::mutex g_pw_scratch_mu;

// set-up, once per device, with that device current: the address of the array on it
static int pw_scratch(unsigned char **at) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e) return e;
  if (dev < 0 || dev >= kScratchDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_pw_scratch_mu);
  if (!g_pw_scratch_at[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_pw_scratch);
    if (e) return e;
    g_pw_scratch_at[dev] = (unsigned char *)p;
  }
  *at = g_pw_scratch_at[dev];
  return 0;
}

extern "C" int bnnk_pw_s8_static(const bnnk_gemm_plan *p, int rows, int Mw, const float *x, long long xws, int lda,
                                 int K, const float *gate, long long gws, const bnnk_epilogue *e, int *err,
                                 bnn_stream_t st) {
  unsigned char *at = nullptr;
  int rc = pw_scratch(&at);
  if (rc || rows <= 0) return rc;
  if (rows > BNNK_STATIC_ROWS || (long long)rows * p->kq > BNNK_STATIC_QBYTES) return cudaErrorInvalidValue;
  float *sa = (float *)at;
  int32_t *za = (int32_t *)(at + 4 * BNNK_STATIC_ROWS);
  int8_t *q = (int8_t *)(at + 8 * BNNK_STATIC_ROWS);
  // the op's plan with its A operand moved onto the q region (a host-side encode: no device memory)
  bnnk_gemm_plan pl = *p;
  rc = encode_2d(pl.tma_a, q, p->kq, (int)(BNNK_STATIC_QBYTES / p->kq), p->sw, 128, p->sw);
  if (!rc) rc = bnnk_quant(rows, Mw, x, xws, lda, K, p->kq, gate, gws, q, sa, za, err, st);
  if (!rc) rc = bnnk_gemm(&pl, rows, Mw, sa, za, e, err, st);
  return rc;
}

// the GEMM of a planned layer on quantized rows the caller holds: q [rows][ldq] (the first kp bytes of a row used,
// TMA zero fill past them), sa, za [rows] (s8n_gemm_range on the rows s8n_quant_rows wrote)
extern "C" int bnnk_gemm_q(const bnnk_gemm_plan *p, const int8_t *q, long long ldq, int kp, int rows, int Mw,
                           const float *sa, const int32_t *za, const bnnk_epilogue *e, int *err, bnn_stream_t st) {
  if (rows <= 0) return 0;
  bnnk_gemm_plan pl = *p;
  const int rc = encode_2d_ld(pl.tma_a, q, kp, ldq, rows, p->sw, 128, p->sw);
  return rc ? rc : bnnk_gemm(&pl, rows, Mw, sa, za, e, err, st);
}

extern "C" int bnnk_test_fn(int fn, int n, const float *x, float *y, bnn_stream_t st) {
  if (n <= 0) return 0;
  k_test_fn<<<(n + 255) / 256, 256, 0, st>>>(fn, n, x, y);
  return cudaGetLastError();
}
