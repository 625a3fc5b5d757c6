// The int8 prototype head (PROTO_S8) on sm_100a: per-cell symmetric quantizer, a persistent tcgen05 kind::i8 GEMM
// whose epilogue takes each prototype's maximum over a window's cells, and the per-class logits.
//
// Reference: src/proto_s8n.c (pc_quant_cells_f32 :28-52, pc_proto_colmax_s8n :130-164) driven by PROTO_S8
// (src/rt_ops_s8n.c:212-250), logits pc_proto_logits (src/pc_kern_f32.c:364-376).
//   colmax[w][j] = sw[j] * max over the cells p of window w of (float)(sum_k qa[p][k] qw[j][k]) * sx[p]
// The int32 sums are exact in both (|q| <= 127, K <= 2^17), so the tensor cores' summation order cannot change them;
// the conversion, scale, maximum and final scale repeat the reference's fp32 steps (max is exact, so the order in
// which cells are visited does not matter; NaN propagates, -0 < +0 as in FMAX).
//
// GEMM orientation: the prototypes are the MMA's M side (128 per tile, TMEM lanes) and the cells its N side (TMEM
// columns), so one epilogue thread owns one prototype and reduces over cells along its own TMEM row, with no
// exchange between threads. A cell tile holds whole windows (floor(256 / P) of them) when P <= 256; longer windows
// are split into chunks of at most 256 cells whose partial maxima a second kernel combines.
//
// Pipeline (as the 1x1-conv GEMM): warp 0 lane 0 streams 128-byte K blocks of prototypes and cells into a ring of
// shared-memory stages with 2-D TMA loads (swizzle 128 B, zero fill past K); warp 1 lane 0 issues
// tcgen05.mma.cta_group::1.kind::i8 (M 128, N = the cell tile, K 32 per instruction) into one of two TMEM
// accumulators; each accumulator has an epilogue group of 4 NH warps that split the tile's windows. Tiles run
// prototype-tile major with the cell tiles inner, so the prototypes stream from HBM once while the (smaller) cell
// matrix stays in L2. Every mbarrier wait is bounded; a timeout sets the error word and the CTA winds down, still
// freeing its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "bnn_kernels.h"
#include "smem_attr.cuh"
#include "emu.cuh"
#include "sync.cuh"
#include "tc.cuh"

namespace bnn {

// ------------------------------------------------------------------ per-cell quantizer

// FCVTAS (nearest, ties away from zero, saturating, NaN -> 0) narrowed with saturation to int8, raised to -127 (the
// fp32 cells' bytes, src/proto_s8n.c:44-48) or not (LO = -128: the fp16 cells', src/pc_proto_s8.c:33-37). trunc(v)
// and v - trunc(v) are exact, so the tie test is exact.
template <int LO = -127>
__device__ __forceinline__ int q_ties_away(float v) {
  float t = truncf(v);
  const float d = __fsub_rn(v, t);
  if (fabsf(d) >= 0.5f) t = __fadd_rn(t, copysignf(1.f, v));
  const int i = cvtzs(t);
  return i > 127 ? 127 : i < LO ? LO : i;
}

// the cells' element type: fp32, or IEEE half (exact conversion to fp32)
__device__ __forceinline__ float load_cell(const float *p) { return __ldg(p); }
__device__ __forceinline__ float load_cell(const __half *p) { return __half2float(__ldg(p)); }

constexpr int kQCells = 8;  // cells per quantizer block: their rows are re-read from L2 right after the reduction

// cells r = w * P + p of x (window stride xws, row stride ld floats) -> qa [cells][Kq] (zero from C to Kq), sx [cells].
// Reduction: 8 threads per cell, thread l holding the reference's accumulator lane l (lanes 0-3 of s0, 4-7 of s1):
// channel c + l of each 8-channel step, fused x x + s in channel order; then vaddvq_f32(s0 + s1) = (v0 + v1) + (v2 + v3)
// with v_l = s0_l + s1_l, by shuffles in that order. Quantization: each warp takes cells of the block, a lane 8
// channels (two 16-byte loads, one 8-byte store) at a time.
// T: float or __half cells (the half form narrows without the -127 clamp)
template <typename T, bool VEC>
__global__ void __launch_bounds__(128) k_proto_quant(int cells, int P, const T *__restrict__ x, long long xws,
                                                     int ld, int C, int Kq, float eps, int8_t *__restrict__ qa,
                                                     float *__restrict__ sx) {
  constexpr bool kHalf = sizeof(T) == 2;
  __shared__ float s_inv[kQCells];
  const int c0 = blockIdx.x * kQCells;
  {
    const int cl = threadIdx.x >> 3, l = threadIdx.x & 7, cell = c0 + cl;
    float s = 0.f, m = 0.f;
    if (cl < kQCells && cell < cells) {
      const int w = cell / P, p = cell - w * P;
      const T *r = x + (long long)w * xws + (long long)p * ld + l;
#pragma unroll 8
      for (int c = 0; c < C; c += 8) {
        const float u = load_cell(r + c);
        s = __fmaf_rn(u, u, s);
        m = fmax_nan(m, fabsf(u));
      }
    }
    const float v = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 4, 8));  // lanes 0-3: v_l = s0_l + s1_l
    const float a = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 8));  // lane 0: v0 + v1, lane 2: v2 + v3
    const float sum = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 2, 8));
    float mx = fmax_nan(m, __shfl_down_sync(0xffffffffu, m, 4, 8));
    mx = fmax_nan(mx, __shfl_down_sync(0xffffffffu, mx, 2, 8));
    mx = fmax_nan(mx, __shfl_down_sync(0xffffffffu, mx, 1, 8));
    if (l == 0 && cl < kQCells && cell < cells) {
      const float den = __fadd_rn(__fsqrt_rn(sum), eps);
      if (!(mx > 0.f)) mx = 1e-30f;
      sx[cell] = __fdiv_rn(mx, __fmul_rn(127.f, den));
      s_inv[cl] = __fdiv_rn(127.f, mx);
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunk = Kq / 8;
  for (int cl = warp; cl < kQCells; cl += 4) {
    const int cell = c0 + cl;
    if (cell >= cells) break;
    const int w = cell / P, p = cell - w * P;
    const T *r = x + (long long)w * xws + (long long)p * ld;
    const float inv = s_inv[cl];
    int8_t *qrow = qa + (long long)cell * Kq;
    for (int ch = lane; ch < nchunk; ch += 32) {
      uint32_t lo = 0, hi = 0;
      if (8 * ch < C) {  // C % 8 == 0: a chunk is all inside or all outside the row
        float u[8];
        if constexpr (VEC && !kHalf) {
          const float4 a = __ldg(reinterpret_cast<const float4 *>(r + 8 * ch));
          const float4 b = __ldg(reinterpret_cast<const float4 *>(r + 8 * ch + 4));
          u[0] = a.x; u[1] = a.y; u[2] = a.z; u[3] = a.w; u[4] = b.x; u[5] = b.y; u[6] = b.z; u[7] = b.w;
        } else if constexpr (VEC) {  // 8 halves in one 16-byte load
          const uint4 a = __ldg(reinterpret_cast<const uint4 *>(r + 8 * ch));
          const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wv[k]));
            u[2 * k] = f.x;
            u[2 * k + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; k++) u[k] = load_cell(r + 8 * ch + k);
        }
        int b[8];
#pragma unroll
        for (int k = 0; k < 8; k++) b[k] = q_ties_away<kHalf ? -128 : -127>(__fmul_rn(u[k], inv));
        lo = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
        hi = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
      }
      *reinterpret_cast<uint2 *>(qrow + 8 * ch) = make_uint2(lo, hi);
    }
  }
}

// ------------------------------------------------------------------ the column-maximum GEMM

constexpr int kPMaxStages = 8;
constexpr int kPMaxThreads = 64 + 128 * 2 * 2;  // 2 accumulators x 4 lane quarters x up to 2 warps
// TMEM loads in flight per epilogue thread (24 or 16 columns per wait; more would spill at the 576-thread register
// budget)
template <int U>
constexpr int kPLoads = U == 8 ? 3 : 4;

struct ProtoArgs {
  int np;             // prototypes (rows of A, columns of colmax)
  int batch, P;       // windows, cells per window
  int wt;             // windows per cell tile (P <= 256), else 0
  int nch, cs;        // P > 256: chunks per window, cells per chunk
  int n_ct, tiles;    // cell tiles, all tiles (prototype tiles x cell tiles)
  int nkb, stages, bn, acc_cols, ne, nh, tmem_alloc;
  uint32_t idesc;
  const float *sx, *sw;
  float *out;         // colmax [batch][ows] (wt > 0) or partial maxima [batch * nch][np]
  long long ows;
  int *err;
};

// the maximum over tile columns [col0, col0 + n) of (float)acc * sx[cell0 + col] for this thread's prototype: U
// columns per TMEM load (8, or 4 when windows start on odd multiples of 4), kPLoads<U> loads in flight. Four running
// maxima (column mod 4) break the dependency chain; max is exact, so combining them at the end gives the maximum in
// any order (NaN-propagating, +0 above -0). The products run paired: each lane is one IEEE multiply, and none feeds
// an add.
template <int U>
__device__ __forceinline__ float col_max(uint32_t trow, int col0, int n, const float *__restrict__ sxc) {
  float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
  for (int c = col0; c < col0 + n; c += U * kPLoads<U>) {
    uint32_t acc[kPLoads<U>][U];
#pragma unroll
    for (int k = 0; k < kPLoads<U>; k++) {
      if (c + k * U < col0 + n) {
        if constexpr (U == 8) tmem_ld8(trow + (uint32_t)(c + k * U), acc[k]);
        else tmem_ld4(trow + (uint32_t)(c + k * U), acc[k]);
      }
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    // the loaded registers pass through an empty asm after the wait, so that no use of them moves above it
#pragma unroll
    for (int k = 0; k < kPLoads<U>; k++)
#pragma unroll
      for (int v = 0; v < U; v++) asm volatile("" : "+r"(acc[k][v]));
#pragma unroll
    for (int k = 0; k < kPLoads<U>; k++) {
      if (c + k * U < col0 + n) {
#pragma unroll
        for (int v = 0; v < U; v += 4) {
          const float4 s = __ldg(reinterpret_cast<const float4 *>(sxc + c + k * U + v));
          const float2 p01 = mul2_rn(make_float2(__int2float_rn((int)acc[k][v + 0]), __int2float_rn((int)acc[k][v + 1])),
                                     make_float2(s.x, s.y));
          const float2 p23 = mul2_rn(make_float2(__int2float_rn((int)acc[k][v + 2]), __int2float_rn((int)acc[k][v + 3])),
                                     make_float2(s.z, s.w));
          m0 = fmax_nan(m0, p01.x);
          m1 = fmax_nan(m1, p01.y);
          m2 = fmax_nan(m2, p23.x);
          m3 = fmax_nan(m3, p23.y);
        }
      }
    }
  }
  return fmax_nan(fmax_nan(m0, m1), fmax_nan(m2, m3));
}

// MH prototype halves of 128 rows per tile: with MH = 2 a tile is 256 prototypes x bn cells, two MMAs per K step
// share the stage's cell block (a third less operand traffic per MAC than 128-row tiles)
template <int U, int MH>
__global__ void __launch_bounds__(kPMaxThreads, 1) k_proto_colmax(const __grid_constant__ CUtensorMap tma_w,
                                                                 const __grid_constant__ CUtensorMap tma_q,
                                                                 const ProtoArgs a) {
  constexpr int SW = 128;
  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) unsigned long long bar_full[kPMaxStages], bar_empty[kPMaxStages];
  __shared__ __align__(8) unsigned long long bar_acc_full[2], bar_acc_empty[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t base = (smem_u32(dsmem) + 1023u) & ~1023u;
  const uint32_t a_bytes = 128u * MH * SW, stage_bytes = (128u * MH + a.bn) * SW;
  const int S = a.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) { mbar_init(smem_u32(&bar_full[s]), 1); mbar_init(smem_u32(&bar_empty[s]), 1); }
    for (int g = 0; g < a.ne; g++) {
      mbar_init(smem_u32(&bar_acc_full[g]), 1);
      mbar_init(smem_u32(&bar_acc_empty[g]), 4 * a.nh);
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
    if (lane == 0) {  // TMA producer
      int it = 0;
      for (int t = blockIdx.x; t < a.tiles && !abort_s; t += gridDim.x) {
        const int m0 = (t / a.n_ct) * 128 * MH, ct = t % a.n_ct;
        const int n0 = a.wt ? ct * a.wt * a.P : (ct / a.nch) * a.P + (ct % a.nch) * a.cs;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % S;
          if (it >= S && !mbar_wait(smem_u32(&bar_empty[s]), ((it / S) - 1) & 1)) {
            atomicExch(a.err, BNNK_ERR_TMA_WAIT);
            abort_s = 1;
            break;
          }
          const uint32_t st = base + s * stage_bytes, bar = smem_u32(&bar_full[s]);
          mbar_expect_tx(bar, stage_bytes);  // full boxes: rows and bytes out of bounds arrive as zero fill
#pragma unroll
          for (int hm = 0; hm < MH; hm++) tma_load_2d(st + hm * 128u * SW, &tma_w, bar, kb * SW, m0 + 128 * hm);
          tma_load_2d(st + a_bytes, &tma_q, bar, kb * SW, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < a.tiles && !abort_s; t += gridDim.x, lt++) {
        const int g = lt % a.ne, use = lt / a.ne;
        if (use > 0 && !mbar_wait(smem_u32(&bar_acc_empty[g]), (use - 1) & 1)) {
          atomicExch(a.err, BNNK_ERR_MMA_WAIT);
          abort_s = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tacc = tmem + (uint32_t)(g * MH * a.acc_cols);
        bool ok = true;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % S;
          if (!mbar_wait(smem_u32(&bar_full[s]), (it / S) & 1)) {
            atomicExch(a.err, BNNK_ERR_MMA_WAIT);
            abort_s = 1;
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = base + s * stage_bytes;
#pragma unroll
          for (int kk = 0; kk < SW / 32; kk++)
#pragma unroll
            for (int hm = 0; hm < MH; hm++)
              mma_i8(tacc + (uint32_t)(hm * a.acc_cols), smem_desc<SW>(st + hm * 128u * SW + kk * 32),
                     smem_desc<SW>(st + a_bytes + kk * 32), a.idesc, (kb | kk) != 0);
          mma_commit(smem_u32(&bar_empty[s]));
        }
        if (!ok) break;
        mma_commit(smem_u32(&bar_acc_full[g]));
      }
    }
  } else if (warp - 2 < 4 * a.ne * a.nh) {
    // epilogue: group g drains accumulator g; warp h of lane quarter q takes the tile's units (prototype half, window)
    // h, h + nh, ...
    const int e = warp - 2, g = e / (4 * a.nh), h = (e % (4 * a.nh)) / 4, q = warp % 4;
    int use = 0;
    for (int t = blockIdx.x + g * gridDim.x; t < a.tiles; t += a.ne * gridDim.x, use++) {
      const int m0 = (t / a.n_ct) * 128 * MH, ct = t % a.n_ct;
      bool ok = mbar_wait(smem_u32(&bar_acc_full[g]), use & 1);
      ok = __all_sync(0xffffffffu, ok && !abort_s);  // one outcome per warp
      if (!ok) {
        if (lane == 0) { atomicExch(a.err, BNNK_ERR_EPI_WAIT); abort_s = 1; }
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t tq = tmem + (uint32_t)(g * MH * a.acc_cols) + ((uint32_t)(q * 32) << 16);
      if (a.wt) {
        const int w0 = ct * a.wt, nw = min(a.wt, a.batch - w0);
        const float *sxc = a.sx + (long long)w0 * a.P;
        for (int u = h; u < MH * nw; u += a.nh) {
          const int hm = u / nw, wi = u - hm * nw, j = m0 + 128 * hm + q * 32 + lane;
          const float mx = col_max<U>(tq + (uint32_t)(hm * a.acc_cols), wi * a.P, a.P, sxc);
          if (j < a.np) a.out[(long long)(w0 + wi) * a.ows + j] = __fmul_rn(mx, __ldg(a.sw + j));
        }
      } else if (h < MH) {
        const int w = ct / a.nch, k = ct % a.nch, cell0 = w * a.P + k * a.cs;
        const int n = min(a.cs, a.P - k * a.cs), j = m0 + 128 * h + q * 32 + lane;
        const float mx = col_max<U>(tq + (uint32_t)(h * a.acc_cols), 0, n, a.sx + cell0);
        if (j < a.np) a.out[(long long)ct * a.np + j] = mx;
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[g]));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_alloc));
}

// windows longer than one cell tile: colmax[w][j] = sw[j] * the maximum of the chunks' partial maxima
__global__ void k_proto_chunks(int batch, int np, int nch, const float *__restrict__ part, const float *__restrict__ sw,
                               float *__restrict__ out, long long ows) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, w = blockIdx.y;
  if (j >= np) return;
  float mx = -INFINITY;
  for (int k = 0; k < nch; k++) mx = fmax_nan(mx, part[((long long)w * nch + k) * np + j]);
  out[(long long)w * ows + j] = __fmul_rn(mx, __ldg(sw + j));
}

// ------------------------------------------------------------------ logits

// one block per window: logits[c] = (sum over q < ppc, in order, of colmax[c ppc + q] * w[c ppc + q]) + b[c], each
// product and sum rounded. A window with a logit that is not finite or above 3e38 in magnitude failed
// (pc_proto_logits returns -2): status[w] = -2 (else 0), and fail holds the smallest failed w_base + w. V4: ppc == 4
// with 16-byte aligned rows (one 16-byte load of each operand per class).
template <bool V4>
__global__ void __launch_bounds__(1024) k_proto_logits(int nc, int ppc, const float *__restrict__ colmax,
                                                       long long cws, const float *__restrict__ cw,
                                                       const float *__restrict__ cb, float *__restrict__ logits,
                                                       long long lws, int *__restrict__ status, int *fail, int w_base) {
  const int w = blockIdx.x;
  const float *cm = colmax + (long long)w * cws;
  int bad = 0;
  for (int c = threadIdx.x; c < nc; c += blockDim.x) {
    float s = 0.f;
    if (V4) {
      const float4 a = __ldg(reinterpret_cast<const float4 *>(cm) + c);
      const float4 b = __ldg(reinterpret_cast<const float4 *>(cw) + c);
      s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, __fmul_rn(a.x, b.x)), __fmul_rn(a.y, b.y)), __fmul_rn(a.z, b.z)),
                    __fmul_rn(a.w, b.w));
    } else {
      for (int q = 0; q < ppc; q++) {
        const long long i = (long long)c * ppc + q;
        s = __fadd_rn(s, __fmul_rn(__ldg(cm + i), __ldg(cw + i)));
      }
    }
    const float v = __fadd_rn(s, __ldg(cb + c));
    logits[(long long)w * lws + c] = v;
    bad |= !(fabsf(v) <= 3.0e38f);
  }
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    if (status) status[w] = bad ? -2 : 0;
    if (bad && fail) atomicMin(fail, w_base + w);
  }
}

}  // namespace bnn

using namespace bnn;

// ------------------------------------------------------------------ launchers

extern "C" int bnnk_proto_quant(int batch, int P, const float *x, long long xws, int ld, int C, int Kq, float eps,
                                int8_t *qa, float *sx, bnn_stream_t st) {
  const int cells = batch * P;
  if (cells <= 0) return 0;
  const bool vec = ((uintptr_t)x & 15) == 0 && xws % 4 == 0 && ld % 4 == 0;
  const int grid = (cells + kQCells - 1) / kQCells;
  if (vec) k_proto_quant<float, true><<<grid, 128, 0, st>>>(cells, P, x, xws, ld, C, Kq, eps, qa, sx);
  else k_proto_quant<float, false><<<grid, 128, 0, st>>>(cells, P, x, xws, ld, C, Kq, eps, qa, sx);
  return cudaGetLastError();
}

extern "C" int bnnk_proto_quant_h(int batch, int P, const uint16_t *x, long long xws, int ld, int C, int Kq, float eps,
                                  int8_t *qa, float *sx, bnn_stream_t st) {
  const int cells = batch * P;
  if (cells <= 0) return 0;
  const __half *xh = reinterpret_cast<const __half *>(x);
  const bool vec = ((uintptr_t)x & 15) == 0 && xws % 8 == 0 && ld % 8 == 0;
  const int grid = (cells + kQCells - 1) / kQCells;
  if (vec) k_proto_quant<__half, true><<<grid, 128, 0, st>>>(cells, P, xh, xws, ld, C, Kq, eps, qa, sx);
  else k_proto_quant<__half, false><<<grid, 128, 0, st>>>(cells, P, xh, xws, ld, C, Kq, eps, qa, sx);
  return cudaGetLastError();
}

extern "C" int bnnk_proto_plan_init(bnnk_proto_plan *p, const int8_t *w, int np, int kp, const int8_t *qa,
                                    int batch_cap, int P) {
  memset(p, 0, sizeof *p);
  if (np <= 0 || np % 4 || kp <= 0 || kp % 16 || batch_cap <= 0 || P <= 0 || P % 4) return cudaErrorInvalidValue;
  p->np = np;
  p->kp = kp;
  p->P = P;
  p->batch_cap = batch_cap;
  p->nkb = (kp + 127) / 128;
  if (P <= 256) {
    p->wt = 256 / P;
    if (p->wt > batch_cap) p->wt = batch_cap;
    p->bn = (p->wt * P + 15) & ~15;
    p->nch = 1;
    p->cs = P;
  } else {
    p->wt = 0;
    p->nch = (P + 255) / 256;
    p->cs = ((P + p->nch - 1) / p->nch + 15) & ~15;
    if (p->cs > 256) p->cs = 256;
    p->nch = (P + p->cs - 1) / p->cs;
    p->bn = p->cs;
  }
  p->unit = (P % 8 == 0 && p->cs % 8 == 0) ? 8 : 4;
  p->acc_cols = p->bn <= 32 ? 32 : p->bn <= 64 ? 64 : p->bn <= 128 ? 128 : 256;
  // 256-prototype tiles (two 128-row halves sharing each cell block) when there are at least two prototype tiles
  // of 128; BNN_PROTO_MH=1 forces 128-row tiles (tuning sweeps)
  const char *env = getenv("BNN_PROTO_MH");
  p->mh = np > 128 && !(env && atoi(env) == 1) ? 2 : 1;
  const size_t stage = (size_t)(128 * p->mh + p->bn) * 128;
  int s = (int)((200 * 1024) / stage);
  p->stages = s < 2 ? 2 : s > kPMaxStages ? kPMaxStages : s;
  p->smem = (size_t)p->stages * stage + 1024;
  p->idesc = idesc_i8(p->bn);
  // prototypes [np][kp] (row stride kp), cells [batch_cap * P][kp]
  int e = encode_2d_ld(p->tma_w, w, kp, kp, np, 128, 128, 128);
  if (!e) e = encode_2d_ld(p->tma_q, qa, kp, kp, batch_cap * P, 128, p->bn, 128);
  return e;
}

template <int U, int MH>
static int launch_colmax(const bnnk_proto_plan *p, const ProtoArgs &a, bnn_stream_t st) {
  static SmemAttr attr;
  const cudaError_t e = attr.ensure(k_proto_colmax<U, MH>, p->smem);
  if (e) return e;
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  k_proto_colmax<U, MH><<<grid, 64 + 128 * a.ne * a.nh, p->smem, st>>>(*(const CUtensorMap *)p->tma_w,
                                                                      *(const CUtensorMap *)p->tma_q, a);
  return cudaGetLastError();
}

extern "C" int bnnk_proto_colmax(const bnnk_proto_plan *p, int batch, const float *sx, const float *sw, float *colmax,
                                 long long cws, float *part, int *err, bnn_stream_t st) {
  if (batch <= 0) return 0;
  if (batch > p->batch_cap || (!p->wt && (!part || batch > 65535))) return cudaErrorInvalidValue;
  ProtoArgs a;
  a.np = p->np;
  a.batch = batch;
  a.P = p->P;
  a.wt = p->wt;
  a.nch = p->nch;
  a.cs = p->cs;
  a.n_ct = p->wt ? (batch + p->wt - 1) / p->wt : batch * p->nch;
  a.tiles = ((p->np + 128 * p->mh - 1) / (128 * p->mh)) * a.n_ct;
  a.nkb = p->nkb;
  a.stages = p->stages;
  a.bn = p->bn;
  a.acc_cols = p->acc_cols;
  // two accumulators (the MMA of the next tile overlaps the epilogue of the last) when they fit the 512 TMEM columns
  a.ne = 2 * p->mh * p->acc_cols <= 512 ? 2 : 1;
  a.tmem_alloc = a.ne * p->mh * p->acc_cols;  // a power of two: acc_cols is one, mh and ne are 1 or 2
  // epilogue warps per lane quarter: one per unit (prototype half, window) of a tile, 16 warps at most
  const int units = p->mh * (p->wt ? p->wt : 1), hmax = 4 / a.ne;
  a.nh = units < hmax ? units : hmax;
  a.idesc = p->idesc;
  a.sx = sx;
  a.sw = sw;
  a.out = p->wt ? colmax : part;
  a.ows = cws;
  a.err = err;
  int e = p->mh == 2 ? (p->unit == 8 ? launch_colmax<8, 2>(p, a, st) : launch_colmax<4, 2>(p, a, st))
                     : (p->unit == 8 ? launch_colmax<8, 1>(p, a, st) : launch_colmax<4, 1>(p, a, st));
  if (e || p->wt) return e;
  const dim3 grid((p->np + 255) / 256, batch);
  k_proto_chunks<<<grid, 256, 0, st>>>(batch, p->np, p->nch, part, sw, colmax, cws);
  return cudaGetLastError();
}

extern "C" int bnnk_proto_logits(int batch, int nc, int ppc, const float *colmax, long long cws, const float *cw,
                                 const float *cb, float *logits, long long lws, int *status, int *fail, int w_base,
                                 bnn_stream_t st) {
  if (batch <= 0) return 0;
  const bool v4 = ppc == 4 && ((uintptr_t)colmax & 15) == 0 && cws % 4 == 0 && ((uintptr_t)cw & 15) == 0;
  if (v4) k_proto_logits<true><<<batch, 1024, 0, st>>>(nc, ppc, colmax, cws, cw, cb, logits, lws, status, fail, w_base);
  else k_proto_logits<false><<<batch, 1024, 0, st>>>(nc, ppc, colmax, cws, cw, cb, logits, lws, status, fail, w_base);
  return cudaGetLastError();
}
