// The neon-fp16 path's kernels (the variant-1 ops of src/rt_ops_f16.c: those of the v2.4 architecture and the DWK,
// PAD and MEAN of compiled models such as Perch v2), bit for bit.
//
// The reference computes these layers with ARMv8.2 fp16 arithmetic in a fixed order: every multiply-add of its GEMMs
// and depthwise convs is one fused fp16 FMLA lane operation, rounded once (src/gemm_f16.c, src/gemm_f16_kblock.h,
// src/kern_f16.c, src/v24_fast.c). The B200's fp16 pipe executes exactly that operation -- PTX fma.rn.f16x2: fused,
// round to nearest even, fp16 subnormals kept -- two lanes per instruction, so these kernels run the reference's
// chains as they are, on CUDA cores. (The tensor cores accumulate in another order and precision and cannot reproduce
// an fp16 FMA chain.) Every fp16 add, subtract, multiply and FMA is explicit PTX with .rn, which is never contracted;
// the fp32 steps use the __f*_rn intrinsics. NaN results are the canonical NaN; payloads are not modelled.
//
// Layouts: activations are the package's fp16 NHWC buffers, B windows at a fixed window stride (elements). GEMM
// weights are uploaded k-major, [Kp][Np] fp16 (row k holds the Np output channels), from the package's hp_pack panels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "bnn_kernels.h"
#include "emu.cuh"
#include "smem_attr.cuh"
#include "sync.cuh"
#include "tc.cuh"

namespace bnn {

// ------------------------------------------------------------------ fp16 pairs (two IEEE halves in a 32-bit word)

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {  // a * b + c, lane-wise
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float h_lo(uint32_t x) { return __half2float(__ushort_as_half((unsigned short)(x & 0xffffu))); }
__device__ __forceinline__ float h_hi(uint32_t x) { return __half2float(__ushort_as_half((unsigned short)(x >> 16))); }
// fp32 -> fp16, nearest even (cvt.rn.f16.f32)
__device__ __forceinline__ uint32_t f2h(float x) { return __half_as_ushort(__float2half_rn(x)); }
__device__ __forceinline__ uint32_t pack2(uint32_t lo, uint32_t hi) { return lo | (hi << 16); }

// FMAX(x, +0) lane-wise, as NEON vmaxq_f16(x, 0): negative values and -0 give +0, NaN stays NaN
__device__ __forceinline__ uint32_t relu2(uint32_t x) {
  const uint32_t nan = __vcmpgtu2(x & 0x7fff7fffu, 0x7c007c00u), neg = __vcmpgeu2(x, 0x80008000u);
  return x & ~(neg & ~nan);
}

// The SiLU of the fp16 kernels (src/silu_lut.h:23-38): silu(x) = FMAX(x, 0) - |x| q(|x|), q a quadratic per unit
// segment n = round(min(|x|, 15.4)) of the reference's coefficient table, at f = u - n. The clamp is an unsigned
// lane minimum, which equals FMIN for the non-negative |x| except that a NaN lane becomes 15.4: its result is NaN
// all the same, through FMAX(x, 0). tab01[n] = c0 | c1 << 16, tab2[n] = c2 (in shared memory).
__device__ __forceinline__ uint32_t silu2(uint32_t x, const uint32_t *tab01, const uint32_t *tab2) {
  const uint32_t u = x & 0x7fff7fffu;
  const uint32_t uc = __vminu2(u, 0x4bb34bb3u);      // (fp16)15.4
  const uint32_t tm = hadd2(uc, 0x66006600u);        // 1536 + round(uc): its low byte is the segment
  const uint32_t f = hsub2(uc, hsub2(tm, 0x66006600u));
  const uint32_t n0 = tm & 15u, n1 = (tm >> 16) & 15u;
  const uint32_t t0 = tab01[n0], t1 = tab01[n1];
  const uint32_t c0 = __byte_perm(t0, t1, 0x5410), c1 = __byte_perm(t0, t1, 0x7632);
  const uint32_t c2 = __byte_perm(tab2[n0], tab2[n1], 0x5410);
  uint32_t p = hfma2(c2, f, c1);
  p = hfma2(p, f, c0);
  return hfma2(u ^ 0x80008000u, p, relu2(x));  // FMLS: FMAX(x, 0) - u * p, one rounding
}

// The coefficient table of src/silu_lut_tables_deg2.h (there split into low and high bytes for a 2-register TBL):
// c0 | c1 << 16 and c2, per segment n = 0..15.
__constant__ uint32_t c_silu01[16] = {
    0xb40b3800u, 0xb242344eu, 0xaecc2fa1u, 0xa9ea2a12u, 0xa4a6249au, 0x9f031ed9u, 0x99351910u, 0x93b11375u,
    0x8daa0d7eu, 0x882c080au, 0x831202f9u, 0x81210118u, 0x806a0067u, 0x80270026u, 0x800e000eu, 0x80050005u};
__constant__ uint32_t c_silu2[16] = {0x23bd, 0x299d, 0x2915, 0x254c, 0x2073, 0x1ae1, 0x1528, 0x0fa3,
                                     0x09a2, 0x0426, 0x0187, 0x0090, 0x0035, 0x0013, 0x0007, 0x0003};

__device__ __forceinline__ void load_silu_tab(uint32_t *tab01, uint32_t *tab2) {
  for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < 16; i += blockDim.x * blockDim.y) {
    tab01[i] = c_silu01[i];
    tab2[i] = c_silu2[i];
  }
}

// ------------------------------------------------------------------ GEMM (PW f16, the pc conv)
//
// gemm_f16_range (src/gemm_f16.c:109-169) per output (row m, channel n): K in blocks of bs k-steps (kblocks: as few
// blocks of <= 128 as possible, balanced, multiples of 8), in each block one fp16 FMA chain from +0 in k order; with
// two or more blocks the chains are summed in fp32 from 0 and the bias is added in fp32 (b32) before one rounding to
// fp16, else the bias is an fp16 add (b16). Epilogue: SiLU (table) or FMAX(x, 0), then the fp16 residual add, stored
// at the pixel's padded row.
//
// CTA tile: BM = 8 RT rows x BN = TN NT channels (NT threads across the channels, RT across the rows); each thread
// holds 8 rows x TN channels (TN = 4 or 8) as 4 TN fp16 pairs, a pair being two ROWS of one channel, so that an FMA
// takes the rows' activations as they lie in the transposed shared tile and the channel's weight duplicated into both
// lanes (the weights are uploaded duplicated, [Kp][Np] words). Per k a thread issues 1 + TN / 4 16-byte shared loads
// for 4 TN fp16x2 FMAs, which occupy the FMA pipe twice as many cycles (fp16x2 issues at half rate).
//
// The CTAs are persistent, as many as fit on the GPU at once: CTA b takes tiles b, b + grid, ... of the (M tile,
// channel tile) space, channel tile fastest (neighbouring CTAs share the activation rows); a tile is ceil(Kp / kGS) stages of
// kGS k-steps, and the (tile, stage) steps run as one pipeline over two shared-memory buffers: while step j is
// computed, step j + 1's weights arrive by cp.async and its activations are loaded into registers, then stored
// transposed into the other buffer; one barrier per step.
constexpr int kGS = 32;

// n / d for 0 <= n < 2^31 and 1 <= d < 2^31 by a multiply-high and a shift (Granlund and Montgomery, "Division by
// invariant integers using multiplication", 1994): with l = ceil(log2 d), mul = ceil(2^(31 + l) / d) < 2^32 and
// n / d = (n mul) >> (31 + l), exact because n (mul - 2^(31 + l) / d) / 2^(31 + l) < 2^-l <= 1 / d; d = 1 is mul = 0
struct FastDiv {
  uint32_t d, mul, shr;
};
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) { return f.mul ? __umulhi(n, f.mul) >> f.shr : n; }
static FastDiv make_fastdiv(uint32_t d) {
  FastDiv f = {d, 0u, 0u};
  if (d > 1) {
    uint32_t l = 0;
    while ((1u << l) < d) l++;
    f.mul = (uint32_t)(((1ull << (31 + l)) + d - 1) / d);
    f.shr = l - 1;  // the multiply-high already divides by 2^32
  }
  return f;
}

struct GemmF16Args {
  const uint16_t *A;
  long long aws;
  int lda, Mw, rows, n_mtiles;
  const uint32_t *Wd;  // [Kp][Np], each weight in both halves
  int Kp, Np, bs;
  const uint16_t *b16;
  const float *b32;
  int act;
  uint16_t *out;
  long long ows;
  int ldo, ow, opad;
  const uint16_t *res;
  long long rws;
  int ldr;
  int NT, RT;
  int ntn;               // channel tiles: the CTAs take the tiles (M tile, channel tile) in M-major order
  FastDiv mw, owd, ntd;  // rows per window, padded output width, channel tiles
  int st16;  // the output rows are 16-byte aligned (out, ldo and ows): 8-channel groups store in one instruction
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gmem), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// kA: activation chunks (16 bytes) per thread per stage, >= ceil(32 / NT); TN: channels per thread
template <bool kFlush, int kA, int TN>
__global__ void __launch_bounds__(256, TN == 8 ? 2 : kA > 4 ? 2 : 4) k_gemm_f16(const GemmF16Args g) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int NT = g.NT, RT = g.RT, BM = 8 * RT, BN = TN * NT, nthr = NT * RT;
  uint16_t *At = reinterpret_cast<uint16_t *>(sm);                                    // [2][kGS][BM]
  uint32_t *Ws = reinterpret_cast<uint32_t *>(sm + (size_t)2 * kGS * BM * 2);         // [2][kGS][BN]
  uint32_t *tab01 = Ws + (size_t)2 * kGS * BN, *tab2 = tab01 + 16;
  float *fbs = reinterpret_cast<float *>(tab2 + 16);  // kFlush: the 8 TN fp32 block sums of each thread, [8 TN][nthr]
  const int tid = threadIdx.x, tn = tid % NT, tr = tid / NT;
  const int nst = (g.Kp + kGS - 1) / kGS;
  const int mine = (g.n_mtiles * g.ntn - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nsteps = mine * nst;
  load_silu_tab(tab01, tab2);

  // this thread's activation chunks of a stage: chunk i is (row ml[i], 8 k-steps c[i]) of the tile
  int cml[kA], cc[kA];
#pragma unroll
  for (int i = 0; i < kA; i++) {
    const int idx = tid + i * nthr;
    cml[i] = idx % BM;
    cc[i] = idx / BM;
  }
  uint4 pa[kA];
  // issue step j's loads: weights by cp.async into buffer j & 1, activations into registers
  auto issue = [&](int j) {
    const int tf = blockIdx.x + (j / nst) * gridDim.x, ks = (j % nst) * kGS;
    const int t = (int)fdiv((uint32_t)tf, g.ntd), n0 = (tf - t * g.ntn) * BN;
    const int kn = min(kGS, g.Kp - ks), kc = kn / 8;
    uint32_t *W = Ws + (size_t)(j & 1) * kGS * BN;
#pragma unroll
    for (int h = 0; h < TN / 4; h++) {
      const int n = n0 + TN * tn + 4 * h;
      const uint32_t *src = g.Wd + (size_t)ks * g.Np + (n < g.Np ? n : 0);
      for (int kk = tr; kk < kn; kk += RT)
        cp_async16(W + (size_t)kk * BN + TN * tn + 4 * h, src + (size_t)kk * g.Np, n < g.Np);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
#pragma unroll
    for (int i = 0; i < kA; i++) {
      pa[i] = make_uint4(0u, 0u, 0u, 0u);
      const int r = t * BM + cml[i];
      if (cc[i] < kc && r < g.rows) {
        const int w = (int)fdiv((uint32_t)r, g.mw), m = r - w * g.Mw;
        pa[i] = __ldg(reinterpret_cast<const uint4 *>(g.A + (size_t)w * g.aws + (size_t)m * g.lda + ks + 8 * cc[i]));
      }
    }
  };
  // store the registers of step j transposed into buffer j & 1 (a warp: 32 consecutive rows of one chunk column)
  auto store = [&](int j) {
    const int ks = (j % nst) * kGS, kc = min(kGS, g.Kp - ks) / 8;
    uint16_t *A = At + (size_t)(j & 1) * kGS * BM;
#pragma unroll
    for (int i = 0; i < kA; i++) {
      if (cc[i] < kc) {
        uint16_t *d = A + (size_t)(8 * cc[i]) * BM + cml[i];
        const uint32_t vv[4] = {pa[i].x, pa[i].y, pa[i].z, pa[i].w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          d[(2 * q) * BM] = (uint16_t)(vv[q] & 0xffffu);
          d[(2 * q + 1) * BM] = (uint16_t)(vv[q] >> 16);
        }
      }
    }
  };

  uint32_t acc[4][TN];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int q = 0; q < TN; q++) acc[i][q] = 0u;
  if (kFlush)
    for (int e = 0; e < 8 * TN; e++) fbs[e * nthr + tid] = 0.f;

  if (nsteps > 0) {
    issue(0);
    store(0);
    cp_async_wait_all();
  }
  __syncthreads();
  for (int j = 0; j < nsteps; j++) {
    if (j + 1 < nsteps) issue(j + 1);
    const int tf = blockIdx.x + (j / nst) * gridDim.x, st = j % nst, ks = st * kGS;
    const int t = (int)fdiv((uint32_t)tf, g.ntd), n0 = (tf - t * g.ntn) * BN;
    const int kn = min(kGS, g.Kp - ks);
    const uint16_t *A = At + (size_t)(j & 1) * kGS * BM;
    const uint32_t *W = Ws + (size_t)(j & 1) * kGS * BN;
    for (int kk = 0; kk < kn; kk += 8) {
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const uint4 a = *reinterpret_cast<const uint4 *>(A + (size_t)(kk + u) * BM + tr * 8);
        uint32_t wv[TN];
#pragma unroll
        for (int h = 0; h < TN / 4; h++) {
          const uint4 w = *reinterpret_cast<const uint4 *>(W + (size_t)(kk + u) * BN + tn * TN + 4 * h);
          wv[4 * h] = w.x; wv[4 * h + 1] = w.y; wv[4 * h + 2] = w.z; wv[4 * h + 3] = w.w;
        }
        const uint32_t av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int q = 0; q < TN; q++) acc[i][q] = hfma2(av[i], wv[q], acc[i][q]);
      }
      if (kFlush) {
        const int kg = ks + kk + 8;
        if (kg % g.bs == 0 || kg == g.Kp) {  // the end of a K block: flush the chains to fp32, restart from +0
#pragma unroll
          for (int i = 0; i < 4; i++)
#pragma unroll
            for (int q = 0; q < TN; q++) {
              float *f = fbs + (size_t)((i * TN + q) * 2) * nthr + tid;
              f[0] = __fadd_rn(f[0], h_lo(acc[i][q]));
              f[nthr] = __fadd_rn(f[nthr], h_hi(acc[i][q]));
              acc[i][q] = 0u;
            }
        }
      }
    }
    if (st == nst - 1) {  // the tile's epilogue
      const int nb = n0 + tn * TN;
      if (nb < g.Np) {
        uint32_t bias16[TN / 2];
        float bias32[TN];
#pragma unroll
        for (int h = 0; h < TN / 4; h++) {
          const uint2 b = __ldg(reinterpret_cast<const uint2 *>(g.b16 + nb + 4 * h));
          const float4 b32 = __ldg(reinterpret_cast<const float4 *>(g.b32 + nb + 4 * h));
          bias16[2 * h] = b.x; bias16[2 * h + 1] = b.y;
          bias32[4 * h] = b32.x; bias32[4 * h + 1] = b32.y; bias32[4 * h + 2] = b32.z; bias32[4 * h + 3] = b32.w;
        }
        int r = t * BM + tr * 8;
        int w = (int)fdiv((uint32_t)r, g.mw), m = r - w * g.Mw;  // the row's window and pixel, advanced row by row
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int l = 0; l < 2; l++) {
            if (r < g.rows) {
              uint32_t v[TN / 2];
#pragma unroll
              for (int q = 0; q < TN / 2; q++) {
                if (kFlush) {
                  const float x0 = fbs[(size_t)((i * TN + 2 * q) * 2 + l) * nthr + tid],
                              x1 = fbs[(size_t)((i * TN + 2 * q + 1) * 2 + l) * nthr + tid];
                  v[q] = pack2(f2h(__fadd_rn(x0, bias32[2 * q])), f2h(__fadd_rn(x1, bias32[2 * q + 1])));
                } else {
                  v[q] = hadd2(__byte_perm(acc[i][2 * q], acc[i][2 * q + 1], l ? 0x7632 : 0x5410), bias16[q]);
                }
                if (g.act == 1) v[q] = silu2(v[q], tab01, tab2);
                else if (g.act == 2) v[q] = relu2(v[q]);
              }
              if (g.res) {
#pragma unroll
                for (int h = 0; h < TN / 4; h++) {
                  const uint2 rv = __ldg(
                      reinterpret_cast<const uint2 *>(g.res + (size_t)w * g.rws + (size_t)m * g.ldr + nb + 4 * h));
                  v[2 * h] = hadd2(v[2 * h], rv.x);
                  v[2 * h + 1] = hadd2(v[2 * h + 1], rv.y);
                }
              }
              int orow = m;
              if (g.opad) {
                const int y = (int)fdiv((uint32_t)m, g.owd);
                orow = (y + g.opad) * (g.ow + 2 * g.opad) + (m - y * g.ow) + g.opad;
              }
              uint16_t *o = g.out + (size_t)w * g.ows + (size_t)orow * g.ldo + nb;
              if (TN == 8 && g.st16) {  // 16-byte rows: one store
                *reinterpret_cast<uint4 *>(o) = make_uint4(v[0], v[1], v[2 % (TN / 2)], v[3 % (TN / 2)]);
              } else {  // 8-byte aligned rows
#pragma unroll
                for (int h = 0; h < TN / 4; h++)
                  *reinterpret_cast<uint2 *>(o + 4 * h) = make_uint2(v[2 * h], v[2 * h + 1]);
              }
            }
            r++;
            if (++m == g.Mw) { m = 0; w++; }
          }
      }
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int q = 0; q < TN; q++) acc[i][q] = 0u;
      if (kFlush)
        for (int e = 0; e < 8 * TN; e++) fbs[e * nthr + tid] = 0.f;
    }
    if (j + 1 < nsteps) {
      store(j + 1);
      cp_async_wait_all();
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ PW f16 on the tensor cores (tensor mode)

// The fp16 1x1 conv as a tcgen05 kind::f16 GEMM: fp16 activations and weights, fp32 accumulators in TMEM. This is the
// path's optional tensor mode, not the reference's arithmetic: the products are exact and summed in fp32 (the
// reference sums them in fp16 chains of <= 128 k-steps, flushed to fp32), so outputs agree with the CUDA-core form
// within a tolerance, not bit for bit. The steps after the sum are the flush form's: + the fp32 bias, one rounding to
// fp16, SiLU (the table) or FMAX(x, 0), the fp16 residual add, the pixel's padded row.
//
// One persistent CTA per SM walks the (128-row tile, BN-column tile) space, column tiles fastest. Warp 0 lane 0
// streams 64-half (128-byte) K blocks of A and B into a ring of shared-memory stages with TMA (A by a 3-D map over
// [windows][rows][K], so a tile never crosses a window and rows past a window's last read zero; B [Nrows][Kp] K-major;
// 128-byte swizzle; no multicast); warp 1 lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N BN, K 16 per
// instruction) into one of two TMEM accumulators; each accumulator has an epilogue group of 4 NH warps that read
// 8-column units with tcgen05.ld. Every mbarrier wait is bounded; a timeout sets the error word and the CTA winds down,
// still freeing its TMEM.
constexpr int kT16MaxStages = 8;
constexpr int kT16Threads = 64 + 128 * 2 * 3;  // 2 accumulators x 3 warps per TMEM lane quarter

struct Tc16Args {
  int rows_w, mt_w;  // rows of one TMA window and its 128-row tiles
  int Mw, rows;      // rows per package window (epilogue mapping) and in all
  int nkb, stages, bn, np, n_tiles, tiles, acc_cols, nh, tmem_alloc;
  uint32_t idesc;
  const float *b32;
  int act;
  uint16_t *out;
  long long ows;
  int ldo, ow, opad;
  const uint16_t *res;
  long long rws;
  int ldr;
  int vec;  // out and res rows (and window strides) 16-byte aligned: one 16-byte access per 8-column unit
  int *err;
};

constexpr int kT16Units = 3;  // 8-column TMEM loads in flight per epilogue thread
// wait for this thread's TMEM loads; the registers they fill are operands of the wait, so no use moves above it
__device__ __forceinline__ void tmem_wait3(uint32_t (&r)[kT16Units][8]) {
#define BNN_R8(u) "+r"(r[u][0]), "+r"(r[u][1]), "+r"(r[u][2]), "+r"(r[u][3]), "+r"(r[u][4]), "+r"(r[u][5]), \
                  "+r"(r[u][6]), "+r"(r[u][7])
  asm volatile("tcgen05.wait::ld.sync.aligned;" : BNN_R8(0), BNN_R8(1), BNN_R8(2)::"memory");
#undef BNN_R8
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
// instruction descriptor of kind::f16: fp16 A and B, fp32 D, both K-major, M 128, N n (a multiple of 16, <= 256)
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

template <int kThreads>  // 64 + 256 nh: the registers a thread may use follow the block size
__global__ void __launch_bounds__(kThreads, 1) k_gemm_tc16(const __grid_constant__ CUtensorMap tma_a,
                                                              const __grid_constant__ CUtensorMap tma_b,
                                                              const Tc16Args a) {
  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) unsigned long long bar_full[kT16MaxStages], bar_empty[kT16MaxStages];
  __shared__ __align__(8) unsigned long long bar_acc_full[2], bar_acc_empty[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;
  __shared__ uint32_t tab01[16], tab2[16];
  __shared__ float s_b32[1024];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t base = (smem_u32(dsmem) + 1023u) & ~1023u;
  const uint32_t a_bytes = 128u * 128u, stage_bytes = (128u + a.bn) * 128u;
  const int S = a.stages;
  load_silu_tab(tab01, tab2);
  const bool sb = a.np <= 1024;  // the fp32 bias staged in shared memory
  if (sb)
    for (int i = threadIdx.x; i < a.np; i += blockDim.x) s_b32[i] = __ldg(a.b32 + i);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) { mbar_init(smem_u32(&bar_full[s]), 1); mbar_init(smem_u32(&bar_empty[s]), 1); }
    for (int g = 0; g < 2; g++) {
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
        const int mt = t / a.n_tiles, n0 = (t % a.n_tiles) * a.bn;
        const int z = mt / a.mt_w, y0 = (mt - z * a.mt_w) * 128;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % S;
          if (it >= S && !mbar_wait(smem_u32(&bar_empty[s]), ((it / S) - 1) & 1)) {
            atomicExch(a.err, BNNK_ERR_TMA_WAIT);
            abort_s = 1;
            break;
          }
          const uint32_t st = base + s * stage_bytes, bar = smem_u32(&bar_full[s]);
          mbar_expect_tx(bar, stage_bytes);  // the full boxes: elements out of bounds arrive as zero fill
          tma_load_3d(st, &tma_a, bar, kb * 64, y0, z);
          tma_load_2d(st + a_bytes, &tma_b, bar, kb * 64, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < a.tiles && !abort_s; t += gridDim.x, lt++) {
        const int g = lt % 2, use = lt / 2;
        if (use > 0 && !mbar_wait(smem_u32(&bar_acc_empty[g]), (use - 1) & 1)) {
          atomicExch(a.err, BNNK_ERR_MMA_WAIT);
          abort_s = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tacc = tmem + (uint32_t)(g * a.acc_cols);
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
          for (int kk = 0; kk < 4; kk++)
            mma_f16(tacc, smem_desc<128>(st + kk * 32), smem_desc<128>(st + a_bytes + kk * 32), a.idesc, (kb | kk) != 0);
          mma_commit(smem_u32(&bar_empty[s]));
        }
        if (!ok) break;
        mma_commit(smem_u32(&bar_acc_full[g]));
      }
    }
  } else if (warp - 2 < 8 * a.nh) {
    // epilogue: group g drains accumulator g; its 4 nh warps split the 8-column units of a tile round robin, the
    // warp's TMEM lane quarter q (= warp % 4) fixing its 32 rows
    const int e = warp - 2, g = e / (4 * a.nh), h = (e % (4 * a.nh)) / 4, q = warp % 4;
    int use = 0;
    for (int t = blockIdx.x + g * gridDim.x; t < a.tiles; t += 2 * gridDim.x, use++) {
      const int mt = t / a.n_tiles, n0 = (t % a.n_tiles) * a.bn;
      const int z = mt / a.mt_w, y = (mt - z * a.mt_w) * 128 + q * 32 + lane;
      const bool live = y < a.rows_w;
      const long long r = (long long)z * a.rows_w + y;  // the row over all windows
      const int w = live ? (int)(r / a.Mw) : 0, m = live ? (int)(r - (long long)w * a.Mw) : 0;
      bool ok = mbar_wait(smem_u32(&bar_acc_full[g]), use & 1);
      ok = __all_sync(0xffffffffu, ok && !abort_s);
      if (!ok) {
        if (lane == 0) { atomicExch(a.err, BNNK_ERR_EPI_WAIT); abort_s = 1; }
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int units = (min(a.bn, a.np - n0) + 7) / 8;
      const long long orow = a.opad ? (long long)((m / a.ow) + a.opad) * (a.ow + 2 * a.opad) + (m % a.ow) + a.opad
                                    : (long long)m;
      uint16_t *op = a.out + (long long)w * a.ows + orow * a.ldo + n0;
      const uint16_t *rp = a.res ? a.res + (long long)w * a.rws + (long long)m * a.ldr + n0 : nullptr;
      const uint32_t tq = tmem + (uint32_t)(g * a.acc_cols) + ((uint32_t)(q * 32) << 16);
      for (int u0 = h; u0 < units; u0 += kT16Units * a.nh) {
        uint32_t accs[kT16Units][8];  // up to three units' loads in flight behind one wait
#pragma unroll
        for (int k = 0; k < kT16Units; k++)
          if (u0 + k * a.nh < units) tmem_ld8(tq + (uint32_t)(8 * (u0 + k * a.nh)), accs[k]);
        tmem_wait3(accs);
#pragma unroll
        for (int k = 0; k < kT16Units; k++) {
        const int u = u0 + k * a.nh;
        if (!live || u >= units) continue;
        const uint32_t *acc = accs[k];
        const int c = 8 * u;
        uint32_t v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float b0 = sb ? s_b32[n0 + c + 2 * j] : __ldg(a.b32 + n0 + c + 2 * j);
          const float b1 = sb ? s_b32[n0 + c + 2 * j + 1] : __ldg(a.b32 + n0 + c + 2 * j + 1);
          v[j] = pack2(f2h(__fadd_rn(__uint_as_float(acc[2 * j]), b0)), f2h(__fadd_rn(__uint_as_float(acc[2 * j + 1]), b1)));
          if (a.act == 1) v[j] = silu2(v[j], tab01, tab2);
          else if (a.act == 2) v[j] = relu2(v[j]);
        }
        if (rp) {
          if (a.vec) {
            const uint4 rv = __ldg(reinterpret_cast<const uint4 *>(rp + c));
            v[0] = hadd2(v[0], rv.x); v[1] = hadd2(v[1], rv.y); v[2] = hadd2(v[2], rv.z); v[3] = hadd2(v[3], rv.w);
          } else {
            const uint2 r0 = __ldg(reinterpret_cast<const uint2 *>(rp + c)), r1 = __ldg(reinterpret_cast<const uint2 *>(rp + c + 4));
            v[0] = hadd2(v[0], r0.x); v[1] = hadd2(v[1], r0.y); v[2] = hadd2(v[2], r1.x); v[3] = hadd2(v[3], r1.y);
          }
        }
        if (a.vec) {
          *reinterpret_cast<uint4 *>(op + c) = make_uint4(v[0], v[1], v[2], v[3]);
        } else {
          *reinterpret_cast<uint2 *>(op + c) = make_uint2(v[0], v[1]);
          *reinterpret_cast<uint2 *>(op + c + 4) = make_uint2(v[2], v[3]);
        }
        }
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

// ------------------------------------------------------------------ C0POOL f16 (src/v24_fast.c:150-164)
//
// One CTA per (output row oy, window), thread qx = the pooled pixel: conv pixels 2qx and 2qx + 1 as the two lanes of
// 24 fp16 pairs (one per channel), K = 64 FMAs in (ky, kx, ci) order from +0 (gemm_f16_rows: the 4 segments continue
// one chain), + b16, ReLU, [max | avg] of the pair. The 4 padded image rows are staged in shared memory as fp16
// (the reference rounds the image to fp16 first), pre-paired: word (ky, ci, col) = (img16[col], img16[col + 2]),
// stored by col % 4 so that the 32 threads of a warp (columns 4 qx + kx) read consecutive words.
__global__ void __launch_bounds__(128) k_c0pool_f16(const float *__restrict__ img, long long iws,
                                                    const uint16_t *__restrict__ W /* [64][24] */,
                                                    const uint16_t *__restrict__ b16, uint16_t *__restrict__ pin,
                                                    long long pws) {
  constexpr int NJ = 130;  // words per (ky, ci, col % 4) run: columns 0..519
  __shared__ uint32_t P[4][2][4][NJ];
  __shared__ __align__(16) uint32_t wd[64][24];
  __shared__ uint16_t sh[4][520][2];
  const int oy = blockIdx.x, win = blockIdx.y, tid = threadIdx.x;
  const float *im = img + (long long)win * iws;
  for (int i = tid; i < 4 * 520 * 2; i += 128) {
    const int ky = i / 1040, col = (i / 2) % 520, ci = i & 1;
    const int y = 2 * oy + ky - 1, x = col - 3;
    sh[ky][col][ci] = (y >= 0 && y < 96 && x >= 0 && x < 511) ? (uint16_t)f2h(im[(y * 511 + x) * 2 + ci]) : 0;
  }
  for (int i = tid; i < 64 * 24; i += 128) {
    const uint32_t h = __ldg(W + i);
    wd[i / 24][i % 24] = h | (h << 16);
  }
  __syncthreads();
  for (int i = tid; i < 4 * 2 * 518; i += 128) {
    const int ky = i / (2 * 518), ci = (i / 518) & 1, col = i % 518;
    P[ky][ci][col & 3][col >> 2] = pack2(sh[ky][col][ci], sh[ky][col + 2][ci]);
  }
  __syncthreads();
  const int qx = tid;
  uint32_t acc[24];
#pragma unroll
  for (int n = 0; n < 24; n++) acc[n] = 0u;
#pragma unroll 1
  for (int ky = 0; ky < 4; ky++)
#pragma unroll
    for (int kx = 0; kx < 8; kx++)
#pragma unroll
      for (int ci = 0; ci < 2; ci++) {
        const uint32_t a = P[ky][ci][kx & 3][qx + (kx >> 2)];
        const uint4 *wr = reinterpret_cast<const uint4 *>(wd[ky * 16 + kx * 2 + ci]);
#pragma unroll
        for (int q = 0; q < 6; q++) {
          const uint4 w = wr[q];
          acc[4 * q] = hfma2(a, w.x, acc[4 * q]);
          acc[4 * q + 1] = hfma2(a, w.y, acc[4 * q + 1]);
          acc[4 * q + 2] = hfma2(a, w.z, acc[4 * q + 2]);
          acc[4 * q + 3] = hfma2(a, w.w, acc[4 * q + 3]);
        }
      }
  uint32_t mx[12], av[12];
#pragma unroll
  for (int q = 0; q < 12; q++) {
    uint32_t m[2], a[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t b = __ldg(b16 + 2 * q + h);
      const uint32_t v = relu2(hadd2(acc[2 * q + h], b | (b << 16)));  // lanes: the two conv pixels
      m[h] = max(v & 0xffffu, v >> 16);                                 // FMAX of values >= +0 (or NaN): bit order
      a[h] = hmul2(hadd2(v, __byte_perm(v, 0, 0x1032)), 0x38003800u) & 0xffffu;  // (a + b) * 0.5
    }
    mx[q] = pack2(m[0], m[1]);
    av[q] = pack2(a[0], a[1]);
  }
  uint4 *o = reinterpret_cast<uint4 *>(pin + (long long)win * pws + ((long long)oy * 128 + qx) * 48);
  o[0] = make_uint4(mx[0], mx[1], mx[2], mx[3]);
  o[1] = make_uint4(mx[4], mx[5], mx[6], mx[7]);
  o[2] = make_uint4(mx[8], mx[9], mx[10], mx[11]);
  o[3] = make_uint4(av[0], av[1], av[2], av[3]);
  o[4] = make_uint4(av[4], av[5], av[6], av[7]);
  o[5] = make_uint4(av[8], av[9], av[10], av[11]);
}

// ------------------------------------------------------------------ DW3 f16 (src/kern_f16.c:83-155)
//
// Thread (channel pair, output row): the row's pixels in order, per pixel two FMA chains over the taps (a from the
// bias: taps 0, 2, 4, 6, 8; a2 from the product of tap 1: taps 3, 5, 7), y = SiLU(a + a2), the fp16 row sum of y in
// pixel order; then one thread per pair adds the row sums in row order in fp32 (chsum).
__global__ void __launch_bounds__(1024) k_dw3_f16(const uint16_t *__restrict__ xp, long long xws, int W, int C, int s,
                                                  int pt, int pl, const uint16_t *__restrict__ wt,
                                                  const uint16_t *__restrict__ bt, uint16_t *__restrict__ out,
                                                  long long ows, int Ho, int Wo, float *__restrict__ chsum,
                                                  long long cws) {
  extern __shared__ uint32_t srs[];  // [Ho][Lc] row sums
  __shared__ uint32_t tab01[16], tab2[16];
  const int Lc = blockDim.x, lane = threadIdx.x, win = blockIdx.y;
  const int c2 = blockIdx.x * Lc + lane, C2 = C / 2;
  load_silu_tab(tab01, tab2);
  __syncthreads();
  const bool on = c2 < C2;
  uint32_t w[9], b = 0;
  if (on) {
    const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wt);
#pragma unroll
    for (int t = 0; t < 9; t++) w[t] = __ldg(w32 + t * C2 + c2);
    b = __ldg(reinterpret_cast<const uint32_t *>(bt) + c2);
  }
  const uint32_t *x = reinterpret_cast<const uint32_t *>(xp + (long long)win * xws);
  uint32_t *o = reinterpret_cast<uint32_t *>(out + (long long)win * ows);
  const int Wp = W + 2;
  for (int oy = threadIdx.y; oy < Ho; oy += blockDim.y) {
    uint32_t rs = 0u;
    if (on) {
      const int iy0 = oy * s - pt + 1;
      for (int ox = 0; ox < Wo; ox++) {
        const int ix0 = ox * s - pl + 1;
        const uint32_t *r0 = x + ((long long)iy0 * Wp + ix0) * C2 + c2, *r1 = r0 + (long long)Wp * C2,
                       *r2 = r1 + (long long)Wp * C2;
        const uint32_t x00 = __ldg(r0), x01 = __ldg(r0 + C2), x02 = __ldg(r0 + 2 * C2);
        const uint32_t x10 = __ldg(r1), x11 = __ldg(r1 + C2), x12 = __ldg(r1 + 2 * C2);
        const uint32_t x20 = __ldg(r2), x21 = __ldg(r2 + C2), x22 = __ldg(r2 + 2 * C2);
        uint32_t a = hfma2(x00, w[0], b);
        uint32_t a2 = hmul2(x01, w[1]);
        a = hfma2(x02, w[2], a);
        a2 = hfma2(x10, w[3], a2);
        a = hfma2(x11, w[4], a);
        a2 = hfma2(x12, w[5], a2);
        a = hfma2(x20, w[6], a);
        a2 = hfma2(x21, w[7], a2);
        a = hfma2(x22, w[8], a);
        const uint32_t y = silu2(hadd2(a, a2), tab01, tab2);
        o[((long long)oy * Wo + ox) * C2 + c2] = y;
        rs = hadd2(rs, y);
      }
    }
    srs[oy * Lc + lane] = rs;
  }
  __syncthreads();
  if (threadIdx.y == 0 && on) {
    float s0 = 0.f, s1 = 0.f;
    for (int oy = 0; oy < Ho; oy++) {
      const uint32_t r = srs[oy * Lc + lane];
      s0 = __fadd_rn(s0, h_lo(r));
      s1 = __fadd_rn(s1, h_hi(r));
    }
    *reinterpret_cast<float2 *>(chsum + (long long)win * cws + 2 * c2) = make_float2(s0, s1);
  }
}

// The same DW3 with the input streamed by TMA (the fp32 path's k_dw3t schedule in fp16 arithmetic). One CTA per
// (window, group of CG channels) walks the output rows: the haloed input rows (W + 2 pixels x CG channels, one 3-D
// tensor-map box) pass through a ring of NR = S + 3 slots in shared memory, loaded one row step ahead, so every
// input byte is read from HBM once and no thread waits on a global load. Thread (lane, channel octet) keeps its
// octet's weights in registers and computes pixel groups lane, lane + NL, ... of the row (R consecutive pixels per
// group share their input columns) with the reference's two tap chains, stores them and leaves them in a
// double-buffered row tile; after the step's barrier the first CG / 2 threads add their channel pair's outputs over
// the row in pixel order (the fp16 row sum) and flush it to their fp32 channel sums. Row v of the ring is input row
// v + 1 - pt; pixel x of an output group reads input columns x S + 1 - pl ...
template <int S, int R, bool kSum>
__global__ void __launch_bounds__(256) k_dw3t_f16(const __grid_constant__ CUtensorMap tmx, int W, int C, int CG,
                                                  int pt, int pl, int Ho, int Wo, const uint16_t *__restrict__ wt,
                                                  const uint16_t *__restrict__ bt, uint16_t *__restrict__ out,
                                                  long long ows, float *__restrict__ chsum, long long cws, int *err,
                                                  int SB) {
  constexpr int NR = S + 3, NX = (R - 1) * S + 3;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) unsigned long long bar[NR];
  __shared__ uint32_t tab01[16], tab2[16];
  // kSum: threads SB.. (whole warps) only sum, one step behind the others (row oy - 1 while row oy is computed);
  // threads below SB compute (those past the last whole channel octet of lanes idle). Otherwise the first CG / 2
  // threads also sum, after each step's barrier.
  const int tid = threadIdx.x, nt = kSum ? SB : (int)blockDim.x;
  const bool summer = kSum && tid >= SB;
  const int sp = tid - SB;  // a summer's channel pair
  load_silu_tab(tab01, tab2);
  const int ngroups = C / CG;
  const int win = blockIdx.x / ngroups, grp = blockIdx.x - win * ngroups;
  const int Wp = W + 2, Q = CG >> 3, NL = nt / Q, ngrp = Wo / R, ro = 1 - pt, co = 1 - pl;
  const uint32_t row_bytes = (uint32_t)Wp * CG * 2, row_stride = (row_bytes + 127u) & ~127u;
  const uint32_t ring = smem_u32(dsm);
  uint16_t *obuf = reinterpret_cast<uint16_t *>(dsm + NR * row_stride);  // [2][Wo][CG]
  const int q = tid % Q, lane = tid / Q;  // lanes >= NL (the last nt % Q threads) do not compute
  const bool comp = !summer && lane < NL;
  const int c = grp * CG + 8 * q;
  uint32_t w[9][4], b[4];
#pragma unroll
  for (int t = 0; t < 9; t++) {
    const uint4 v = comp ? __ldg(reinterpret_cast<const uint4 *>(wt + (size_t)t * C + c)) : make_uint4(0u, 0u, 0u, 0u);
    w[t][0] = v.x; w[t][1] = v.y; w[t][2] = v.z; w[t][3] = v.w;
  }
  {
    const uint4 v = comp ? __ldg(reinterpret_cast<const uint4 *>(bt + c)) : make_uint4(0u, 0u, 0u, 0u);
    b[0] = v.x; b[1] = v.y; b[2] = v.z; b[3] = v.w;
  }
  if (tid == 0) {
    for (int i = 0; i < NR; i++) mbar_init(smem_u32(&bar[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int rows_in = (Ho - 1) * S + 3;  // ring rows the outputs read
  int issued = 0;                        // ring rows whose load thread 0 has issued
  auto issue_to = [&](int last) {        // thread 0: load ring rows issued .. last
    for (; issued <= last && issued < rows_in; issued++) {
      const int sl = issued % NR;
      mbar_expect_tx(smem_u32(&bar[sl]), row_bytes);
      tma_load_3d(ring + sl * row_stride, &tmx, smem_u32(&bar[sl]), grp * CG, (issued + ro) * Wp, win);
    }
  };
  if (tid == 0) issue_to(S + 2);  // the rows of steps 0 and 1
  float2 cs = make_float2(0.f, 0.f);
  int oy = 0;
  for (; oy < Ho; oy++) {
    bool ok = true;
    if (!summer) {
#pragma unroll
      for (int ky = 0; ky < 3; ky++) {
        const int iy = oy * S + ky;
        ok = ok && mbar_wait(smem_u32(&bar[iy % NR]), (uint32_t)(iy / NR) & 1u);
      }
    }
    uint16_t *ob = obuf + (size_t)(oy & 1) * Wo * CG;
    if (kSum && summer) {  // the previous row's fp16 row sum in pixel order, then the fp32 channel sums
      if (oy > 0 && sp < CG / 2) {
        const uint32_t *o32 = reinterpret_cast<const uint32_t *>(obuf + (size_t)((oy - 1) & 1) * Wo * CG);
        uint32_t rs = 0u;
        for (int x = 0; x < Wo; x++) rs = hadd2(rs, o32[(size_t)x * (CG / 2) + sp]);
        cs.x = __fadd_rn(cs.x, h_lo(rs));
        cs.y = __fadd_rn(cs.y, h_hi(rs));
      }
    } else if (comp) {
      // groups in reverse lane order: when they do not divide evenly, the extra ones go to the high lanes, not to
      // the low threads that also add the row sums after the barrier
      for (int g = NL - 1 - lane; g < ngrp; g += NL) {
        const int x0 = g * R;
        uint32_t a[R][4], a2[R][4];
#pragma unroll
        for (int ky = 0; ky < 3; ky++) {
          const uint16_t *rw = reinterpret_cast<const uint16_t *>(dsm + ((oy * S + ky) % NR) * row_stride) +
                               (size_t)(x0 * S + co) * CG + 8 * q;
          uint4 xin[NX];
#pragma unroll
          for (int j = 0; j < NX; j++) xin[j] = *reinterpret_cast<const uint4 *>(rw + (size_t)j * CG);
#pragma unroll
          for (int r = 0; r < R; r++) {
#pragma unroll
            for (int kx = 0; kx < 3; kx++) {
              const uint4 xv = xin[r * S + kx];
              const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
              const int t = 3 * ky + kx;  // taps 0, 2, 4, 6, 8 chain a (from the bias), 1, 3, 5, 7 chain a2
#pragma unroll
              for (int h = 0; h < 4; h++) {
                if (t == 0) a[r][h] = hfma2(xs[h], w[0][h], b[h]);
                else if (t == 1) a2[r][h] = hmul2(xs[h], w[1][h]);
                else if (t % 2 == 0) a[r][h] = hfma2(xs[h], w[t][h], a[r][h]);
                else a2[r][h] = hfma2(xs[h], w[t][h], a2[r][h]);
              }
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
          uint32_t y[4];
#pragma unroll
          for (int h = 0; h < 4; h++) y[h] = silu2(hadd2(a[r][h], a2[r][h]), tab01, tab2);
          const uint4 v = make_uint4(y[0], y[1], y[2], y[3]);
          *reinterpret_cast<uint4 *>(out + (size_t)win * ows + ((size_t)oy * Wo + x0 + r) * C + c) = v;
          *reinterpret_cast<uint4 *>(ob + (size_t)(x0 + r) * CG + 8 * q) = v;
        }
      }
    }
    if (!__syncthreads_and(ok)) break;  // every thread has left this step's rows and written its outputs
    if (tid == 0) issue_to((oy + 2) * S + 2);
    if (!kSum && tid < CG / 2) {  // channel pair tid: the fp16 row sum in pixel order, then fp32
      const uint32_t *o32 = reinterpret_cast<const uint32_t *>(ob);
      uint32_t rs = 0u;
      for (int x = 0; x < Wo; x++) rs = hadd2(rs, o32[(size_t)x * (CG / 2) + tid]);
      cs.x = __fadd_rn(cs.x, h_lo(rs));
      cs.y = __fadd_rn(cs.y, h_hi(rs));
    }
  }
  if (oy < Ho) {  // a load never arrived: report it, then let the loads still in flight land before leaving
    if (tid == 0) {
      if (err) atomicExch(err, BNNK_ERR_DW3_WAIT);
      for (int iy = oy * S; iy < issued; iy++) mbar_wait(smem_u32(&bar[iy % NR]), (uint32_t)(iy / NR) & 1u);
    }
    __syncthreads();
    return;
  }
  if (kSum) {  // the summers add the last row (the compute threads are done with the tile)
    if (summer && sp < CG / 2) {
      const uint32_t *o32 = reinterpret_cast<const uint32_t *>(obuf + (size_t)((Ho - 1) & 1) * Wo * CG);
      uint32_t rs = 0u;
      for (int x = 0; x < Wo; x++) rs = hadd2(rs, o32[(size_t)x * (CG / 2) + sp]);
      cs.x = __fadd_rn(cs.x, h_lo(rs));
      cs.y = __fadd_rn(cs.y, h_hi(rs));
      *reinterpret_cast<float2 *>(chsum + (size_t)win * cws + grp * CG + 2 * sp) = cs;
    }
  } else if (tid < CG / 2) {
    *reinterpret_cast<float2 *>(chsum + (size_t)win * cws + grp * CG + 2 * tid) = cs;
  }
}

// ------------------------------------------------------------------ SE f16 (src/v24_fast.c:186-235)

// sigm4 (src/v24_fast.c:173-185): 1 / (1 + 2^t), t = -a log2 e clamped to [-126, 126], 2^t as a degree-6 polynomial
// of the fraction (FMA chain) with the integer part added to the exponent bits, an IEEE division
__device__ __forceinline__ float sigm_f16path(float a) {
  float t = __fmul_rn(a, -1.44269504f);
  t = fmin_nan(fmax_nan(t, -126.f), 126.f);
  const float n = rintf(t), f = __fsub_rn(t, n);
  float p = 1.5403530e-4f;
  p = __fmaf_rn(p, f, 1.3333558e-3f);
  p = __fmaf_rn(p, f, 9.6181291e-3f);
  p = __fmaf_rn(p, f, 5.5504109e-2f);
  p = __fmaf_rn(p, f, 2.4022651e-1f);
  p = __fmaf_rn(p, f, 6.9314718e-1f);
  p = __fmaf_rn(p, f, 1.f);
  const float e = __int_as_float((int)((uint32_t)__float_as_int(p) + ((uint32_t)cvtzs(n) << 23)));
  return __fdiv_rn(1.f, __fadd_rn(1.f, e));
}

// One CTA per window: the gate as SE_GATE computes it (mean, fc1 in the NEON lane order, SiLU with glibc expf, fc2
// from the bias in r order), then sigm4, rounded to fp16 -> g16 [C]
constexpr int kSe16Threads = 512;
__global__ void __launch_bounds__(kSe16Threads) k_se_gate_f16(int C, int rd, const float *__restrict__ w1,
                                                              const float *__restrict__ b1,
                                                              const float *__restrict__ w2t,
                                                              const float *__restrict__ b2,
                                                              const float *__restrict__ chsum, long long cws, int P,
                                                              uint16_t *__restrict__ g16) {
  extern __shared__ float sm_se[];
  float *mean = sm_se, *s1 = sm_se + C;
  const int win = blockIdx.x, tid = threadIdx.x;
  const float inv = __fdiv_rn(1.f, __int2float_rn(P));
  for (int c = tid; c < C; c += kSe16Threads) mean[c] = __fmul_rn(chsum[win * cws + c], inv);
  __syncthreads();
  const int lane8 = tid & 7, C8 = C >> 3;
  for (int r0 = 0; r0 < rd; r0 += kSe16Threads / 8) {
    const int r = r0 + tid / 8;
    float a = 0.f;
    if (r < rd) {
      const float *wr = w1 + (long long)r * C + lane8;
      const float *mr = mean + lane8;
      // batches of 8 weights, the next batch in flight while the current one is multiplied (same FMA order)
      int i = 0;
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
        for (int u = 0; u < 8; u++) a = __fmaf_rn(wv[u], mr[8 * (i + u)], a);
      }
      for (; i < C8; i++) a = __fmaf_rn(__ldg(wr + 8 * i), mr[8 * i], a);
    }
    const float other = __shfl_down_sync(0xffffffffu, a, 4, 8);
    const float v = __fadd_rn(a, other);
    const float v1 = __shfl_down_sync(0xffffffffu, v, 1, 8), v2 = __shfl_down_sync(0xffffffffu, v, 2, 8),
                v3 = __shfl_down_sync(0xffffffffu, v, 3, 8);
    if (r < rd && lane8 == 0) {
      const float xr = __fadd_rn(__fadd_rn(__fadd_rn(v, v1), __fadd_rn(v2, v3)), b1[r]);
      s1[r] = __fdiv_rn(xr, __fadd_rn(1.f, glibc_expf(-xr, c_expf_tab)));
    }
  }
  __syncthreads();
  for (int c = tid; c < C; c += kSe16Threads) {
    float gv = b2[c];
    int r = 0;
    for (; r + 8 <= rd; r += 8) {  // the batch's 8 loads issued ahead of its FMAs (same order)
      float wv[8];
#pragma unroll
      for (int u = 0; u < 8; u++) wv[u] = __ldg(w2t + (long long)(r + u) * C + c);
#pragma unroll
      for (int u = 0; u < 8; u++) gv = __fmaf_rn(wv[u], s1[r + u], gv);
    }
    for (; r < rd; r++) gv = __fmaf_rn(__ldg(w2t + (long long)r * C + c), s1[r], gv);
    g16[(long long)win * C + c] = (uint16_t)f2h(sigm_f16path(gv));
  }
}

// D [P][C] *= g16 [C] in place (an fp16 multiply per element), 8 halves per thread
__global__ void k_se_scale_f16(int B, int P, int C, uint16_t *__restrict__ D, long long dws,
                               const uint16_t *__restrict__ g16) {
  const long long per = (long long)P * (C / 8), total = per * B;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long win = i / per, rem = i - win * per;
    const int c8 = (int)(rem % (C / 8));
    uint4 *d = reinterpret_cast<uint4 *>(D + win * dws) + rem;
    const uint4 g = __ldg(reinterpret_cast<const uint4 *>(g16 + win * C) + c8);
    uint4 v = *d;
    v.x = hmul2(v.x, g.x); v.y = hmul2(v.y, g.y); v.z = hmul2(v.z, g.z); v.w = hmul2(v.w, g.w);
    *d = v;
  }
}

// ------------------------------------------------------------------ POSTPC f16 (src/v24_fast.c:273-311)

// post = fp16(FMAX(fma(X, s, b), 0)) and the 3x3 valid im2col: pcin [6][1728] per window, k = (ky 3 + kx) 192 + c
__global__ void k_postpc_f16_im2col(const uint16_t *__restrict__ X, long long xws, const float *__restrict__ ps,
                                    const float *__restrict__ pb, uint16_t *__restrict__ pcin, long long pws) {
  const int win = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 6 * 1728; i += gridDim.x * blockDim.x) {
    const int ox = i / 1728, k = i % 1728, t = k / 192, c = k % 192, ky = t / 3, kx = t % 3;
    const int p = ky * 8 + ox + kx;
    const float x = __half2float(__ushort_as_half(X[(long long)win * xws + p * 192 + c]));
    pcin[(long long)win * pws + i] = (uint16_t)f2h(fmax_nan(__fmaf_rn(x, ps[c], pb[c]), 0.f));
  }
}

// feat [1024] = (sum of the 6 positions in fp32, in order) * (1 / 6); a window with a feature that is not finite or
// above 3e38 in magnitude failed (v24k16_postpc returns -2): fail holds the smallest failed w_base + window
__global__ void k_postpc_f16_mean(const uint16_t *__restrict__ pcout, long long pws, float *__restrict__ feat,
                                  long long fws, int *fail, int w_base) {
  const int win = blockIdx.x;
  bool bad = false;
  for (int c = threadIdx.x; c < 1024; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int ox = 0; ox < 6; ox++)
      s = __fadd_rn(s, __half2float(__ushort_as_half(pcout[(long long)win * pws + ox * 1024 + c])));
    const float v = __fmul_rn(s, 1.f / 6.f);
    feat[(long long)win * fws + c] = v;
    bad |= !(fabsf(v) <= 3.0e38f);
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0 && fail) atomicMin(fail, w_base + win);
}

// ------------------------------------------------------------------ DENSE f16 (src/v24_fast.c:237-270)
//
// The 4-row path of v24k16_head for every class o < N & ~3: x = fp16(feat); per 128-k block 8 fp16 lanes, lane j
// the FMA chain over k = j mod 8 from +0; the lanes flushed into 8 fp32 sums; out = FADDP((s_j + s_{j+4})_j) + b.
// A thread holds 2 windows x 4 classes (tc, tc + 16, tc + 32, tc + 48 of the CTA's 64: a warp's weight rows are then
// consecutive, 4 banks apart); a lane pair (2q, 2q + 1) is one fp16x2 chain over k-step pairs. Shared tiles per
// block: X [32 windows][128 + 8] and W [64 classes][128 + 8] fp16 (rows padded against bank conflicts).
constexpr int kDnW = 32, kDnC = 64, kDnLd = 136;
__global__ void __launch_bounds__(256) k_dense_f16(int B, int N4, const float *__restrict__ feat, long long fws,
                                                   const uint16_t *__restrict__ W, const float *__restrict__ bias,
                                                   float *__restrict__ out, long long ows) {
  __shared__ __align__(16) uint16_t xs[kDnW][kDnLd];
  __shared__ __align__(16) uint16_t ws[kDnC][kDnLd];
  const int tid = threadIdx.x, tw = tid / 16, tc = tid % 16;
  const int w0 = blockIdx.y * kDnW, c0 = blockIdx.x * kDnC;
  uint32_t acc[2][4][4];
  float fs[2][4][8];
#pragma unroll
  for (int a = 0; a < 2; a++)
#pragma unroll
    for (int b = 0; b < 4; b++)
#pragma unroll
      for (int j = 0; j < 8; j++) fs[a][b][j] = 0.f;
  for (int kb = 0; kb < 1024; kb += 128) {
    __syncthreads();
    for (int i = tid; i < kDnW * 32; i += 256) {  // 4 features per step
      const int r = i / 32, k4 = i % 32;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (w0 + r < B) f = *reinterpret_cast<const float4 *>(feat + (long long)(w0 + r) * fws + kb + 4 * k4);
      *reinterpret_cast<uint2 *>(&xs[r][4 * k4]) = make_uint2(pack2(f2h(f.x), f2h(f.y)), pack2(f2h(f.z), f2h(f.w)));
    }
    for (int i = tid; i < kDnC * 16; i += 256) {
      const int r = i / 16, k8 = i % 16;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (c0 + r < N4) v = __ldg(reinterpret_cast<const uint4 *>(W + (long long)(c0 + r) * 1024 + kb + 8 * k8));
      *reinterpret_cast<uint4 *>(&ws[r][8 * k8]) = v;
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 2; a++)
#pragma unroll
      for (int b = 0; b < 4; b++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[a][b][q] = 0u;
#pragma unroll 4
    for (int k = 0; k < 128; k += 8) {
      uint4 xv[2], wv[4];
#pragma unroll
      for (int a = 0; a < 2; a++) xv[a] = *reinterpret_cast<const uint4 *>(&xs[tw * 2 + a][k]);
#pragma unroll
      for (int b = 0; b < 4; b++) wv[b] = *reinterpret_cast<const uint4 *>(&ws[tc + 16 * b][k]);
#pragma unroll
      for (int a = 0; a < 2; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
          acc[a][b][0] = hfma2(wv[b].x, xv[a].x, acc[a][b][0]);
          acc[a][b][1] = hfma2(wv[b].y, xv[a].y, acc[a][b][1]);
          acc[a][b][2] = hfma2(wv[b].z, xv[a].z, acc[a][b][2]);
          acc[a][b][3] = hfma2(wv[b].w, xv[a].w, acc[a][b][3]);
        }
    }
#pragma unroll
    for (int a = 0; a < 2; a++)
#pragma unroll
      for (int b = 0; b < 4; b++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
          fs[a][b][2 * q] = __fadd_rn(fs[a][b][2 * q], h_lo(acc[a][b][q]));
          fs[a][b][2 * q + 1] = __fadd_rn(fs[a][b][2 * q + 1], h_hi(acc[a][b][q]));
        }
  }
#pragma unroll
  for (int a = 0; a < 2; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const int w = w0 + tw * 2 + a, o = c0 + tc + 16 * b;
      if (w >= B || o >= N4) continue;
      float v[4];
#pragma unroll
      for (int l = 0; l < 4; l++) v[l] = __fadd_rn(fs[a][b][l], fs[a][b][l + 4]);
      out[(long long)w * ows + o] = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])), bias[o]);
    }
}

// the scalar tail of v24k16_head (classes N & ~3 .. N - 1): fp32 products and sums in k order, + b
__global__ void k_dense_f16_tail(int B, int N4, int N, const float *__restrict__ feat, long long fws,
                                 const uint16_t *__restrict__ W, const float *__restrict__ bias,
                                 float *__restrict__ out, long long ows) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, nt = N - N4;
  if (i >= B * nt) return;
  const int w = i / nt, o = N4 + i % nt;
  float s = 0.f;
  for (int k = 0; k < 1024; k++) {
    const float x = __half2float(__float2half_rn(feat[(long long)w * fws + k]));
    s = __fadd_rn(s, __fmul_rn(__half2float(__ushort_as_half(W[(long long)o * 1024 + k])), x));
  }
  out[(long long)w * ows + o] = __fadd_rn(s, bias[o]);
}

// DENSE variant 0 (v24k32_head, src/v24_f32.c:213-243; the head of small models on every path): per class 8 fp32
// FMA chains over k = j mod 8, out = FADDP((a_l + c_l)_l) + b
__global__ void k_dense_f32(int B, int N, const float *__restrict__ feat, long long fws, const float *__restrict__ W,
                            const float *__restrict__ bias, float *__restrict__ out, long long ows) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * N) return;
  const int w = i / N, o = i % N;
  const float *x = feat + (long long)w * fws, *wr = W + (long long)o * 1024;
  float a[4] = {0.f, 0.f, 0.f, 0.f}, c[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < 1024; k += 8)
#pragma unroll
    for (int l = 0; l < 4; l++) {
      a[l] = __fmaf_rn(wr[k + l], x[k + l], a[l]);
      c[l] = __fmaf_rn(wr[k + 4 + l], x[k + 4 + l], c[l]);
    }
  float v[4];
#pragma unroll
  for (int l = 0; l < 4; l++) v[l] = __fadd_rn(a[l], c[l]);
  out[(long long)w * ows + o] = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])), bias[o]);
}

// The fp16 FMA pipe's throughput, for the roofline of the kernels above: every thread runs 8 independent
// fma.rn.f16x2 chains for iters rounds (16 fp16 FMAs per thread per round); out keeps the chains live.
__global__ void __launch_bounds__(256) k_peak_hfma2(int iters, uint32_t seed, uint32_t *out) {
  uint32_t a[8];
#pragma unroll
  for (int j = 0; j < 8; j++) a[j] = 0x3c003c00u ^ (seed + j + threadIdx.x);
  const uint32_t m = 0x3bff3bffu, c = 0x1c001c00u;  // x * (1 - 2^-11) + 2^-8: stays finite
  for (int i = 0; i < iters; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) a[j] = hfma2(a[j], m, c);
  uint32_t r = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) r ^= a[j];
  if (r == 0x12345678u) out[0] = r;
}

// ------------------------------------------------------------------ DWK f16 (pc_dwk_f16_cr, src/pc_kern_f16.c:16-96)
//
// Depthwise k x k (k odd <= 7) on the input zero-haloed by h = (k - 1) / 2, output pixel (oy, ox) reading rows
// oy s - pt + h + ky and columns ox s - pl + h + kx. The reference walks each output row in groups: four pixels (two
// chains per pixel, even taps from the bias and odd taps from +0 in (ky, kx) order, then one fp16 add), then a pair,
// then a single pixel (one chain from the bias); activation 1 = the SiLU table; the group's fp16 sum ((v0 + v1) +
// (v2 + v3), v0 + v1 or v0) is added to the fp32 channel sum in group order.
// Thread (channel pair, output row): the row's groups in order, each group's fp16 sum kept in shared memory; the
// block walks the rows in chunks of one row per thread row, and after each chunk's barrier one thread per pair adds
// the chunk's group sums in row order, then group order, to its fp32 sums.
template <int K, int G>
__device__ __forceinline__ uint32_t dwk_group(const uint32_t *xr, long long rs, long long cs, int s, const uint32_t *w,
                                              uint32_t b, int act, const uint32_t *tab01, const uint32_t *tab2,
                                              uint32_t *o, long long os) {
  uint32_t a[G], e[G];
#pragma unroll
  for (int q = 0; q < G; q++) { a[q] = b; e[q] = 0u; }
#pragma unroll
  for (int ky = 0; ky < K; ky++)
#pragma unroll
    for (int kx = 0; kx < K; kx++) {
      const int t = ky * K + kx;
#pragma unroll
      for (int q = 0; q < G; q++) {
        const uint32_t xv = __ldg(xr + ky * rs + ((long long)q * s + kx) * cs);
        if (G == 4 && (t & 1)) e[q] = hfma2(xv, w[t], e[q]);
        else a[q] = hfma2(xv, w[t], a[q]);
      }
    }
  uint32_t v[G];
#pragma unroll
  for (int q = 0; q < G; q++) {
    v[q] = G == 4 ? hadd2(a[q], e[q]) : a[q];
    if (act == 1) v[q] = silu2(v[q], tab01, tab2);
    o[q * os] = v[q];
  }
  if (G == 4) return hadd2(hadd2(v[0], v[1]), hadd2(v[2], v[3]));
  if (G == 2) return hadd2(v[0], v[1]);
  return v[0];
}

template <int K>
__global__ void __launch_bounds__(256) k_dwk_f16(const uint16_t *__restrict__ xp, long long xws, int W, int C, int s,
                                                 int pt, int pl, const uint16_t *__restrict__ wt,
                                                 const uint16_t *__restrict__ bt, int act, uint16_t *__restrict__ out,
                                                 long long ows, int Ho, int Wo, int ngr, float *__restrict__ chsum,
                                                 long long cws) {
  extern __shared__ uint32_t sgs[];  // [Ry * ngr][Lc] group sums of the current chunk of rows
  __shared__ uint32_t tab01[16], tab2[16];
  constexpr int KK = K * K, h = (K - 1) / 2;
  const int Lc = blockDim.x, Ry = blockDim.y, lane = threadIdx.x, win = blockIdx.y;
  const int c2 = blockIdx.x * Lc + lane, C2 = C / 2;
  load_silu_tab(tab01, tab2);
  __syncthreads();
  const bool on = c2 < C2;
  uint32_t w[KK], b = 0u;
  if (on) {
    const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wt);
#pragma unroll
    for (int t = 0; t < KK; t++) w[t] = __ldg(w32 + t * C2 + c2);
    b = __ldg(reinterpret_cast<const uint32_t *>(bt) + c2);
  }
  const uint32_t *x = reinterpret_cast<const uint32_t *>(xp + (long long)win * xws) + c2;
  uint32_t *o = reinterpret_cast<uint32_t *>(out + (long long)win * ows) + c2;
  const long long cs = C2, rs = (long long)(W + 2 * h) * C2;
  float s0 = 0.f, s1 = 0.f;  // the channel pair's sums (kept by the threads of row 0 of the block)
  for (int oy0 = 0; oy0 < Ho; oy0 += Ry) {
    const int oy = oy0 + threadIdx.y;
    if (on && oy < Ho) {
      const uint32_t *xr = x + (long long)(oy * s - pt + h) * rs;
      uint32_t *orow = o + (long long)oy * Wo * cs;
      uint32_t *g = sgs + threadIdx.y * ngr * Lc + lane;
      int ox = 0, gi = 0;
      for (; ox + 4 <= Wo; ox += 4, gi++)
        g[gi * Lc] = dwk_group<K, 4>(xr + (long long)(ox * s - pl + h) * cs, rs, cs, s, w, b, act, tab01, tab2,
                                     orow + ox * cs, cs);
      if (ox + 2 <= Wo) {
        g[gi * Lc] = dwk_group<K, 2>(xr + (long long)(ox * s - pl + h) * cs, rs, cs, s, w, b, act, tab01, tab2,
                                     orow + ox * cs, cs);
        ox += 2;
        gi++;
      }
      if (ox < Wo)
        g[gi * Lc] = dwk_group<K, 1>(xr + (long long)(ox * s - pl + h) * cs, rs, cs, s, w, b, act, tab01, tab2,
                                     orow + ox * cs, cs);
    }
    __syncthreads();
    if (threadIdx.y == 0 && on) {  // the chunk's group sums in row order, then group order
      const int n = min(Ry, Ho - oy0) * ngr;
      for (int i = 0; i < n; i++) {
        const uint32_t r = sgs[i * Lc + lane];
        s0 = __fadd_rn(s0, h_lo(r));
        s1 = __fadd_rn(s1, h_hi(r));
      }
    }
    __syncthreads();
  }
  if (threadIdx.y == 0 && on) {
    chsum[(long long)win * cws + 2 * c2] = s0;
    chsum[(long long)win * cws + 2 * c2 + 1] = s1;
  }
}

// The same DWK for channel quads (C % 4 == 0 with 8-byte aligned rows: every package buffer qualifies): a thread
// holds 4 channels (two fp16 pairs, one 8-byte load per tap column), and with the stride S a template parameter the
// NX = (G - 1) S + k input columns of a G-pixel group are loaded once per tap row and shared by the group's pixels.
// The tap weights sit in shared memory (one 8-byte load feeds the group's 2 G fp16-pair FMAs of a tap), which keeps
// the kernel near 70 registers. Thread rows 0 .. Ry - 1 compute a chunk of Ry output rows into one of two group-sum
// tiles; the last thread row only adds the previous chunk's group sums (row order, then group order) into the fp32
// channel sums, so the compute rows pass one barrier per chunk and never wait for the sums.
template <int K, int S, int G>
__device__ __forceinline__ uint2 dwk4_group(const uint2 *xr, long long rs, long long cs, const uint2 *ws, int wl,
                                            uint2 b, int act, const uint32_t *tab01, const uint32_t *tab2, uint2 *o,
                                            long long os) {
  constexpr int NX = (G - 1) * S + K;
  uint32_t a[G][2], e[G][2];
#pragma unroll
  for (int q = 0; q < G; q++) { a[q][0] = b.x; a[q][1] = b.y; e[q][0] = 0u; e[q][1] = 0u; }
#pragma unroll
  for (int ky = 0; ky < K; ky++) {
    uint2 xv[NX];
#pragma unroll
    for (int j = 0; j < NX; j++) xv[j] = __ldg(xr + ky * rs + j * cs);
#pragma unroll
    for (int kx = 0; kx < K; kx++) {
      const int t = ky * K + kx;
      const uint2 wt = ws[t * wl];
#pragma unroll
      for (int q = 0; q < G; q++) {
        const uint2 v = xv[q * S + kx];
        if (G == 4 && (t & 1)) {
          e[q][0] = hfma2(v.x, wt.x, e[q][0]);
          e[q][1] = hfma2(v.y, wt.y, e[q][1]);
        } else {
          a[q][0] = hfma2(v.x, wt.x, a[q][0]);
          a[q][1] = hfma2(v.y, wt.y, a[q][1]);
        }
      }
    }
  }
  uint2 v[G];
#pragma unroll
  for (int q = 0; q < G; q++) {
    v[q] = G == 4 ? make_uint2(hadd2(a[q][0], e[q][0]), hadd2(a[q][1], e[q][1])) : make_uint2(a[q][0], a[q][1]);
    if (act == 1) v[q] = make_uint2(silu2(v[q].x, tab01, tab2), silu2(v[q].y, tab01, tab2));
    o[q * os] = v[q];
  }
  if (G == 4)
    return make_uint2(hadd2(hadd2(v[0].x, v[1].x), hadd2(v[2].x, v[3].x)),
                      hadd2(hadd2(v[0].y, v[1].y), hadd2(v[2].y, v[3].y)));
  if (G == 2) return make_uint2(hadd2(v[0].x, v[1].x), hadd2(v[0].y, v[1].y));
  return v[0];
}

template <int K, int S>
__global__ void __launch_bounds__(256, 3) k_dwk4_f16(const uint16_t *__restrict__ xp, long long xws, int W, int C, int pt,
                                                  int pl, const uint16_t *__restrict__ wt,
                                                  const uint16_t *__restrict__ bt, int act, uint16_t *__restrict__ out,
                                                  long long ows, int Ho, int Wo, int ngr, float *__restrict__ chsum,
                                                  long long cws) {
  extern __shared__ uint2 sd4[];  // [K * K][Lc] tap weights, then [2][Ry * ngr][Lc] group sums of two chunks
  __shared__ uint32_t tab01[16], tab2[16];
  constexpr int KK = K * K, h = (K - 1) / 2;
  const int Lc = blockDim.x, Ry = blockDim.y - 1, lane = threadIdx.x, win = blockIdx.y;
  const int c4 = blockIdx.x * Lc + lane, C4 = C / 4;
  const bool on = c4 < C4, summer = threadIdx.y == Ry;
  uint2 *ws = sd4, *sg = sd4 + KK * Lc;
  const int tile = Ry * ngr * Lc;
  load_silu_tab(tab01, tab2);
  for (int t = threadIdx.y; t < KK; t += blockDim.y)
    ws[t * Lc + lane] = on ? __ldg(reinterpret_cast<const uint2 *>(wt) + t * C4 + c4) : make_uint2(0u, 0u);
  const uint2 b = on ? __ldg(reinterpret_cast<const uint2 *>(bt) + c4) : make_uint2(0u, 0u);
  __syncthreads();
  const uint2 *x = reinterpret_cast<const uint2 *>(xp + (long long)win * xws) + c4;
  uint2 *o = reinterpret_cast<uint2 *>(out + (long long)win * ows) + c4;
  const long long cs = C4, rs = (long long)(W + 2 * h) * C4;
  float sm[4] = {0.f, 0.f, 0.f, 0.f};
  const int nch = (Ho + Ry - 1) / Ry;
  for (int ci = 0; ci <= nch; ci++) {
    if (!summer) {
      const int oy = ci * Ry + threadIdx.y;
      if (ci < nch && on && oy < Ho) {
        const uint2 *xr = x + (long long)(oy * S - pt + h) * rs;
        uint2 *orow = o + (long long)oy * Wo * cs;
        uint2 *g = sg + (ci & 1) * tile + threadIdx.y * ngr * Lc + lane;
        int ox = 0, gi = 0;
        for (; ox + 4 <= Wo; ox += 4, gi++)
          g[gi * Lc] = dwk4_group<K, S, 4>(xr + (long long)(ox * S - pl + h) * cs, rs, cs, ws + lane, Lc, b, act,
                                           tab01, tab2, orow + ox * cs, cs);
        if (ox + 2 <= Wo) {
          g[gi * Lc] = dwk4_group<K, S, 2>(xr + (long long)(ox * S - pl + h) * cs, rs, cs, ws + lane, Lc, b, act,
                                           tab01, tab2, orow + ox * cs, cs);
          ox += 2;
          gi++;
        }
        if (ox < Wo)
          g[gi * Lc] = dwk4_group<K, S, 1>(xr + (long long)(ox * S - pl + h) * cs, rs, cs, ws + lane, Lc, b, act,
                                           tab01, tab2, orow + ox * cs, cs);
      }
    } else if (ci > 0 && on) {  // the previous chunk's group sums, row order then group order
      const uint2 *gs = sg + ((ci - 1) & 1) * tile + lane;
      const int n = min(Ry, Ho - (ci - 1) * Ry) * ngr;
      for (int i = 0; i < n; i++) {
        const uint2 r = gs[i * Lc];
        sm[0] = __fadd_rn(sm[0], h_lo(r.x));
        sm[1] = __fadd_rn(sm[1], h_hi(r.x));
        sm[2] = __fadd_rn(sm[2], h_lo(r.y));
        sm[3] = __fadd_rn(sm[3], h_hi(r.y));
      }
    }
    __syncthreads();
  }
  if (summer && on)
    for (int j = 0; j < 4; j++) chsum[(long long)win * cws + 4 * c4 + j] = sm[j];
}

// ------------------------------------------------------------------ PAD f16 (pc_pad_f16, src/pc_kern_f16.c:98-102)
// x [H][W] (channel stride ld) into the interior of the zero-haloed xp [H + 2h][W + 2h][C]; the halo is never written
// (the buffer is zeroed once when it is allocated).
template <int V>  // V fp16 values per thread (8: 16-byte copies, for aligned rows)
__global__ void k_pad_f16(int H, int W, int C, int ld, int h, const uint16_t *__restrict__ x, long long xws,
                          uint16_t *__restrict__ xp, long long pws) {
  const int CV = C / V;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x, n = (long long)H * W * CV;
  if (i >= n) return;
  const int c = (int)(i % CV) * V;
  const long long pix = i / CV;
  const int y = (int)(pix / W), xx = (int)(pix - (long long)y * W);
  uint16_t *d = xp + (long long)blockIdx.y * pws + ((long long)(y + h) * (W + 2 * h) + xx + h) * C + c;
  const uint16_t *src = x + (long long)blockIdx.y * xws + pix * ld + c;
  if (V == 8) *reinterpret_cast<uint4 *>(d) = __ldg(reinterpret_cast<const uint4 *>(src));
  else *d = *src;
}

// ------------------------------------------------------------------ MEAN f16 (pc_mean_f16, src/pc_kern_f16.c:115-121)
// per channel: the P pixels converted to fp32 and summed in pixel order from +0, then one IEEE division by P.
__global__ void k_mean_f16(int P, int C, int ld, const uint16_t *__restrict__ x, long long xws,
                           float *__restrict__ out, long long ows) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const uint16_t *xr = x + (long long)blockIdx.y * xws + c;
  float s = 0.f;
  for (int p = 0; p < P; p++) s = __fadd_rn(s, __half2float(__ushort_as_half(xr[(long long)p * ld])));
  out[(long long)blockIdx.y * ows + c] = __fdiv_rn(s, (float)P);
}

}  // namespace bnn

using namespace bnn;

// ------------------------------------------------------------------ launchers

extern "C" int bnnk_f16_tables_init(const unsigned long long *tab) {
  return cudaMemcpyToSymbol(c_expf_tab, tab, sizeof(unsigned long long) * 32);
}

// K blocks (kblocks, src/gemm_f16.c:58-62)
static void kblocks(int Kp, int *nblk, int *bs) {
  *nblk = (Kp + 127) / 128;
  *bs = ((Kp + *nblk - 1) / *nblk + 7) & ~7;
}

// the channel tile: all of Np up to 128 (at least 16), else the widest multiple of 8 up to 128 that divides Np (else
// 128); columns past Np are zero-filled and not stored
// the channel tile: all Np channels up to 128; else the widest multiple of 8 in 64..128 that divides Np (576 -> 96);
// else the width whose tiles cover Np with the fewest padded channels, if that saves at least 15 % of the 128-wide
// tiles' width (136 -> 2 x 72 instead of 2 x 128), else 128 (816 and 232 ran 5-12 % slower on 104- and 120-wide
// tiles than on 128-wide ones with a partly empty last tile)
static int gemm_bn(int Np) {
  if (Np <= 128) return Np < 16 ? 16 : Np;
  for (int bn = 128; bn >= 64; bn -= 8)
    if (Np % bn == 0) return bn;
  const long long c128 = (long long)((Np + 127) / 128) * 128;
  int best = 128;
  long long cover = c128;
  for (int bn = 120; bn >= 64; bn -= 8) {
    const long long c = (long long)((Np + bn - 1) / bn) * bn;
    if (c < cover) { best = bn; cover = c; }
  }
  return cover * 100 <= c128 * 85 ? best : 128;
}

extern "C" int bnnk_gemm_f16(int rows, int Mw, const uint16_t *A, long long aws, int lda, const uint32_t *Wd, int Kp,
                             int Np, const uint16_t *b16, const float *b32, int act, uint16_t *out, long long ows,
                             int ldo, int ow, int opad, const uint16_t *res, long long rws, int ldr, bnn_stream_t st) {
  if (rows <= 0) return 0;
  if (Kp % 8 || Np % 8 || lda % 8 || aws % 8 || ldo % 4 || ows % 4 || (res && (ldr % 4 || rws % 4)) ||
      ((uintptr_t)A & 15) || ((uintptr_t)Wd & 15) || ((uintptr_t)out & 7) || (res && ((uintptr_t)res & 7)) ||
      ((uintptr_t)b32 & 15) || ((uintptr_t)b16 & 7))
    return cudaErrorInvalidValue;
  int nblk, bs;
  kblocks(Kp, &nblk, &bs);
  GemmF16Args g;
  g.A = A; g.aws = aws; g.lda = lda; g.Mw = Mw; g.rows = rows;
  g.Wd = Wd; g.Kp = Kp; g.Np = Np; g.bs = bs; g.b16 = b16; g.b32 = b32; g.act = act;
  g.out = out; g.ows = ows; g.ldo = ldo; g.ow = ow; g.opad = opad; g.res = res; g.rws = rws; g.ldr = ldr;
  g.st16 = ((uintptr_t)out & 15) == 0 && ldo % 8 == 0 && ows % 8 == 0;
  g.mw = make_fastdiv((uint32_t)Mw);
  g.owd = make_fastdiv((uint32_t)(ow > 0 ? ow : 1));
  // the channel tile and the channels per thread: 8 when the tile has at least 64 channels, else 4
  const int BN = gemm_bn(Np), TN = BN >= 64 && BN % 8 == 0 ? 8 : 4;
  g.NT = BN / TN;
  g.RT = 256 / g.NT < 32 ? 256 / g.NT : 32;
  const int BM = 8 * g.RT, threads = g.NT * g.RT;
  const int ka = (32 + g.NT - 1) / g.NT;  // activation chunks per thread per stage (NT >= 4: at most 8)
  g.n_mtiles = (int)((rows + BM - 1) / BM);
  const int ntn = (Np + BN - 1) / BN;
  const size_t smem = (size_t)2 * kGS * BM * 2 + (size_t)2 * kGS * BN * 4 + 32 * 4 +
                      (nblk > 1 ? sizeof(float) * 8 * TN * (size_t)threads : 0);
  void (*kern)(GemmF16Args);
  if (TN == 8)
    kern = nblk > 1 ? (ka <= 2 ? k_gemm_f16<true, 2, 8> : ka <= 4 ? k_gemm_f16<true, 4, 8> : k_gemm_f16<true, 8, 8>)
                    : (ka <= 2 ? k_gemm_f16<false, 2, 8> : ka <= 4 ? k_gemm_f16<false, 4, 8> : k_gemm_f16<false, 8, 8>);
  else
    kern = nblk > 1 ? (ka <= 2 ? k_gemm_f16<true, 2, 4> : ka <= 4 ? k_gemm_f16<true, 4, 4> : k_gemm_f16<true, 8, 4>)
                    : (ka <= 2 ? k_gemm_f16<false, 2, 4> : ka <= 4 ? k_gemm_f16<false, 4, 4> : k_gemm_f16<false, 8, 4>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int per_sm = 0;
  if (!e) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e) return e;
  g.ntn = ntn;
  g.ntd = make_fastdiv((uint32_t)ntn);
  const long long tiles = (long long)g.n_mtiles * ntn;
  long long gx = (long long)(per_sm > 0 ? per_sm : 1) * num_sms();  // resident CTAs only: none waits for a slot
  if (gx > tiles) gx = tiles;
  kern<<<(unsigned)gx, threads, smem, st>>>(g);
  return cudaGetLastError();
}

extern "C" int bnnk_c0pool_f16(int B, const float *img, long long iws, const uint16_t *W, const uint16_t *b16,
                               uint16_t *pin, long long pws, bnn_stream_t st) {
  if (B <= 0) return 0;
  if (pws % 8 || ((uintptr_t)pin & 15)) return cudaErrorInvalidValue;
  k_c0pool_f16<<<dim3(48, B), 128, 0, st>>>(img, iws, W, b16, pin, pws);
  return cudaGetLastError();
}

static PFN_cuTensorMapEncodeTiled_v12000 f16_encode_fn(void) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult qr;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// The tensor-mode PW f16: Wk [Np][Kp] fp16 K-major (row n holds output channel n's weights), b32 [Np]. Kp, Np, lda
// and aws multiples of 8 (the TMA row strides are multiples of 16 bytes); A and Wk 16-byte aligned, out / res 8.
extern "C" int bnnk_gemm_tc16(int B, int Mw, const uint16_t *A, long long aws, int lda, const uint16_t *Wk, int Kp,
                              int Np, const float *b32, int act, uint16_t *out, long long ows, int ldo, int ow, int opad,
                              const uint16_t *res, long long rws, int ldr, int *err, bnn_stream_t st) {
  if (B <= 0 || Mw <= 0) return 0;
  if (Kp % 8 || Np % 8 || Np <= 0 || lda % 8 || lda < Kp || aws % 8 || ((uintptr_t)A & 15) || ((uintptr_t)Wk & 15) ||
      ((uintptr_t)out & 7) || ldo % 4 || ows % 4 || (res && (((uintptr_t)res & 7) || ldr % 4 || rws % 4)) ||
      (opad && ow <= 0) || !err)
    return cudaErrorInvalidValue;
  PFN_cuTensorMapEncodeTiled_v12000 enc = f16_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  Tc16Args a;
  // windows stored back to back are one tall matrix (tiles cross window boundaries; the epilogue maps each row)
  const bool flat = aws == (long long)Mw * lda && (long long)B * Mw < (1ll << 31);
  const int nwin = flat ? 1 : B;
  a.rows_w = flat ? B * Mw : Mw;
  a.mt_w = (a.rows_w + 127) / 128;
  a.Mw = Mw;
  a.rows = B * Mw;
  a.nkb = (Kp + 63) / 64;
  // N tiles: as few of at most 256 columns as possible (equal widths rounded up to 16), then narrower (down to 32)
  // while the row tiles alone leave SMs idle
  const int n16 = (Np + 15) & ~15;
  const long long mtiles = (long long)nwin * a.mt_w;
  int nt = (n16 + 255) / 256;
  while (mtiles * nt < num_sms() && ((n16 + nt) / (nt + 1) + 15) / 16 * 16 >= 32) nt++;
  a.bn = ((n16 + nt - 1) / nt + 15) & ~15;
  a.n_tiles = (Np + a.bn - 1) / a.bn;
  a.np = Np;
  if (mtiles * a.n_tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  a.tiles = (int)(mtiles * a.n_tiles);
  a.acc_cols = a.bn <= 32 ? 32 : a.bn <= 64 ? 64 : a.bn <= 128 ? 128 : 256;
  a.tmem_alloc = 2 * a.acc_cols < 32 ? 32 : 2 * a.acc_cols;
  const char *enh = getenv("BNN_TC16_NH");  // epilogue warps per TMEM lane quarter and accumulator (tuning: 2 or 3)
  a.nh = enh && atoi(enh) == 2 ? 2 : 3;
  a.idesc = idesc_f16(a.bn);
  a.b32 = b32;
  a.act = act;
  a.out = out; a.ows = ows; a.ldo = ldo; a.ow = ow; a.opad = opad;
  a.res = res; a.rws = rws; a.ldr = ldr;
  a.vec = ((uintptr_t)out & 15) == 0 && ldo % 8 == 0 && ows % 8 == 0 &&
          (!res || (((uintptr_t)res & 15) == 0 && ldr % 8 == 0 && rws % 8 == 0));
  a.err = err;
  const size_t stage = (size_t)(128 + a.bn) * 128;
  int s = (int)((200 * 1024) / stage);
  a.stages = s < 2 ? 2 : s > kT16MaxStages ? kT16MaxStages : s;
  const size_t smem = (size_t)a.stages * stage + 1024;

  CUtensorMap ma, mb;
  {
    cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)a.rows_w, (cuuint64_t)nwin};
    cuuint64_t strides[2] = {(cuuint64_t)lda * 2, (cuuint64_t)(flat ? (long long)a.rows_w * lda : aws) * 2};
    cuuint32_t box[3] = {64, 128, 1}, es[3] = {1, 1, 1};
    if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t *>(A), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)Np};
    cuuint64_t strides[1] = {(cuuint64_t)Kp * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)a.bn}, es[2] = {1, 1};
    if (enc(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t *>(Wk), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  static SmemAttr attr3, attr2;
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  if (a.nh == 2) {
    const cudaError_t e = attr2.ensure(k_gemm_tc16<64 + 128 * 2 * 2>, smem);
    if (e) return e;
    k_gemm_tc16<64 + 128 * 2 * 2><<<grid, 64 + 128 * 2 * 2, smem, st>>>(ma, mb, a);
  } else {
    const cudaError_t e = attr3.ensure(k_gemm_tc16<kT16Threads>, smem);
    if (e) return e;
    k_gemm_tc16<kT16Threads><<<grid, kT16Threads, smem, st>>>(ma, mb, a);
  }
  return cudaGetLastError();
}

// shared memory of the TMA form for CG channels: the ring of S + 3 input rows and the two output-row tiles
static size_t dw3t_f16_smem(int W, int Wo, int s, int cg) {
  const size_t row_stride = ((size_t)(W + 2) * cg * 2 + 127) & ~(size_t)127;
  return (size_t)(s + 3) * row_stride + 2 * 2 * (size_t)Wo * cg;
}

extern "C" int bnnk_dw3_f16(int B, const uint16_t *xp, long long xws, int H, int W, int C, int s, int pt, int pl,
                            const uint16_t *w, const uint16_t *b, uint16_t *out, long long ows, int Ho, int Wo,
                            float *chsum, long long cws, int *err, bnn_stream_t st) {
  if (B <= 0) return 0;
  // the TMA form: channels per CTA the largest multiple of 8 dividing C, at most 256 (one box dimension), with the
  // shared memory of two CTAs per SM
  const size_t budget = smem_budget(k_dw3t_f16<1, 2, false>, 2);
  int cg = 0;
  for (int g = 8; g <= C && g <= 256; g += 8)
    if (C % g == 0 && dw3t_f16_smem(W, Wo, s, g) <= budget) cg = g;
  PFN_cuTensorMapEncodeTiled_v12000 enc = f16_encode_fn();
  if (cg && enc && ((uintptr_t)xp & 15) == 0 && xws % 8 == 0 && W + 2 <= 256 && (s == 1 || s == 2) &&
      ((uintptr_t)out & 15) == 0 && ows % 8 == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)b & 15) == 0 &&
      cws % 2 == 0 && (Ho - 1) * s - pt + 1 + 3 <= H + 2 && (Wo - 1) * s - pl + 1 + 3 <= W + 2) {
    CUtensorMap map;
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)(H + 2) * (W + 2), (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)xws * 2};
    cuuint32_t box[3] = {(cuuint32_t)cg, (cuuint32_t)(W + 2), 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t *>(xp), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
      const size_t smem = dw3t_f16_smem(W, Wo, s, cg);
      const unsigned grid = (unsigned)B * (unsigned)(C / cg);
      const int Q = cg / 8;  // threads: whole channel octets up to 256, at least the CG / 2 summing threads
      int nt = (256 / Q) * Q;
      if (nt < cg / 2) nt = cg / 2;
      nt = (nt + 31) / 32 * 32;
      int sb = nt;
      // rows of 16+ pixels: summer warps, one row behind (the row sum is a chain of Wo dependent adds, which on the
      // computing threads delayed every step: Perch's 40-channel 249 x 63 layer 0.95 -> 0.77 ms per 512 windows,
      // v2.4's 72-channel 24 x 64 layers 0.244 -> 0.206 ms per 1024), the computing threads within the rest of 256;
      // only where the summers take at most two warps and leave the passes over a row's pixel groups as they were
      // (144 and 192 channels, with three summer warps, ran 8-10 % slower)
      const int ns = 32 * ((cg / 2 + 31) / 32), ngrp = Wo / (Wo % 2 == 0 ? 2 : 1);
      const int sbc = ((256 - ns) / Q) * Q, nl_old = (256 / Q) * Q / Q, nl_new = sbc / Q;
      if (Wo >= 16 && ns <= 64 && nl_new >= 1 &&
          (ngrp + nl_new - 1) / nl_new == (ngrp + nl_old - 1) / nl_old) {
        sb = (sbc + 31) / 32 * 32;
        nt = sb + ns;
      }
      const bool pair = Wo % 2 == 0;
#define BNN_DW3T16_(SS, RR, KS)                                                                                \
  do {                                                                                                        \
    cudaError_t e_ = cudaFuncSetAttribute(k_dw3t_f16<SS, RR, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          (int)smem);                                                         \
    if (e_) return e_;                                                                                        \
    k_dw3t_f16<SS, RR, KS><<<grid, nt, smem, st>>>(map, W, C, cg, pt, pl, Ho, Wo, w, b, out, ows, chsum, cws,  \
                                                   err, sb);                                                  \
  } while (0)
#define BNN_DW3T16(SS, RR) \
  do { if (sb < nt) BNN_DW3T16_(SS, RR, true); else BNN_DW3T16_(SS, RR, false); } while (0)
      if (s == 1) { if (pair) BNN_DW3T16(1, 2); else BNN_DW3T16(1, 1); }
      else { if (pair) BNN_DW3T16(2, 2); else BNN_DW3T16(2, 1); }
#undef BNN_DW3T16
#undef BNN_DW3T16_
      return cudaGetLastError();
    }
  }
  // the general form: taps loaded straight from global memory
  if (C % 2 || xws % 2 || ows % 2 || cws % 2) return cudaErrorInvalidValue;
  const int C2 = C / 2;
  int Lc = C2 <= 64 ? C2 : 64;
  for (int l = 64; l >= 32; l -= 8)  // a lane count that divides the channel pairs, if there is one
    if (C2 > 64 && C2 % l == 0) { Lc = l; break; }
  while (Lc > 1 && sizeof(uint32_t) * (size_t)Ho * Lc > 48 * 1024) Lc = (Lc + 1) / 2;  // tall maps: fewer lanes
  const int Ry = Ho < 1024 / Lc ? Ho : 1024 / Lc;
  const size_t smem = sizeof(uint32_t) * (size_t)Ho * Lc;
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  k_dw3_f16<<<dim3((C2 + Lc - 1) / Lc, B), dim3(Lc, Ry), smem, st>>>(xp, xws, W, C, s, pt, pl, w, b, out, ows, Ho,
                                                                     Wo, chsum, cws);
  return cudaGetLastError();
}

extern "C" int bnnk_se_f16(int B, int C, int rd, const float *w1, const float *b1, const float *w2t, const float *b2,
                           const float *chsum, long long cws, int P, uint16_t *D, long long dws, uint16_t *g16,
                           bnn_stream_t st) {
  if (B <= 0) return 0;
  if (C % 8 || dws % 8 || ((uintptr_t)D & 15) || ((uintptr_t)g16 & 15)) return cudaErrorInvalidValue;
  k_se_gate_f16<<<B, kSe16Threads, sizeof(float) * (size_t)(C + rd), st>>>(C, rd, w1, b1, w2t, b2, chsum, cws, P, g16);
  cudaError_t e = cudaGetLastError();
  if (e) return e;
  const long long total = (long long)B * P * (C / 8);
  const int blocks = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
  k_se_scale_f16<<<blocks, 256, 0, st>>>(B, P, C, D, dws, g16);
  return cudaGetLastError();
}

extern "C" int bnnk_postpc_f16(int B, const uint16_t *X, long long xws, const float *ps, const float *pb,
                               const uint32_t *W, const uint16_t *b16, const float *b32, uint16_t *pcin,
                               long long pinws, uint16_t *pcout, long long poutws, float *feat, long long fws,
                               int *fail, int w_base, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_postpc_f16_im2col<<<dim3(12, B), 256, 0, st>>>(X, xws, ps, pb, pcin, pinws);
  cudaError_t e = cudaGetLastError();
  if (e) return e;
  e = (cudaError_t)bnnk_gemm_f16(6 * B, 6, pcin, pinws, 1728, W, 1728, 1024, b16, b32, 2, pcout, poutws, 1024, 0, 0,
                                 NULL, 0, 0, st);
  if (e) return e;
  k_postpc_f16_mean<<<B, 256, 0, st>>>(pcout, poutws, feat, fws, fail, w_base);
  return cudaGetLastError();
}

extern "C" int bnnk_dense_f16(int B, int N, const float *feat, long long fws, const uint16_t *W, const float *bias,
                              float *out, long long ows, bnn_stream_t st) {
  if (B <= 0) return 0;
  if (fws % 4 || ((uintptr_t)feat & 15) || ((uintptr_t)W & 15)) return cudaErrorInvalidValue;
  const int N4 = N & ~3;
  if (N4)
    k_dense_f16<<<dim3((N4 + kDnC - 1) / kDnC, (B + kDnW - 1) / kDnW), 256, 0, st>>>(B, N4, feat, fws, W, bias, out,
                                                                                    ows);
  cudaError_t e = cudaGetLastError();
  if (e || N4 == N) return e;
  k_dense_f16_tail<<<(B * (N - N4) + 127) / 128, 128, 0, st>>>(B, N4, N, feat, fws, W, bias, out, ows);
  return cudaGetLastError();
}

extern "C" int bnnk_peak_hfma2(int blocks, int iters, uint32_t *out, bnn_stream_t st) {
  k_peak_hfma2<<<blocks, 256, 0, st>>>(iters, 0x9e37u, out);
  return cudaGetLastError();
}

extern "C" int bnnk_dense_f32(int B, int N, const float *feat, long long fws, const float *W, const float *bias,
                              float *out, long long ows, bnn_stream_t st) {
  if (B <= 0) return 0;
  k_dense_f32<<<(B * N + 127) / 128, 128, 0, st>>>(B, N, feat, fws, W, bias, out, ows);
  return cudaGetLastError();
}

// groups per output row of the DWK walk: fours, then a pair, then a single pixel
static int dwk_groups(int Wo) { return Wo / 4 + (Wo % 4 >= 2) + (Wo % 2); }

extern "C" int bnnk_dwk_f16(int B, const uint16_t *xp, long long xws, int W, int C, int k, int s, int pt, int pl,
                            const uint16_t *w, const uint16_t *b, int act, uint16_t *out, long long ows, int Ho, int Wo,
                            float *chsum, long long cws, bnn_stream_t st) {
  if (B <= 0) return 0;
  const int ngr = dwk_groups(Wo);
  // the channel-quad form: 8-byte aligned rows, windows, weights and bias
  if (C % 4 == 0 && xws % 4 == 0 && ows % 4 == 0 && ((uintptr_t)xp & 7) == 0 && ((uintptr_t)out & 7) == 0 &&
      ((uintptr_t)w & 7) == 0 && ((uintptr_t)b & 7) == 0 && (s == 1 || s == 2) && (k == 3 || k == 5 || k == 7)) {
    const int C4 = C / 4;
    const int Lc = C4 < 32 ? C4 : 32;
    int Ry = 256 / Lc - 1;  // computing thread rows; one more row adds the group sums
    if (Ry > Ho) Ry = Ho;
    if (Ry < 1) Ry = 1;
    auto smem_of = [&](int ry) { return (size_t)(k * k + 2 * ry * ngr) * Lc * 8; };
    while (Ry > 1 && smem_of(Ry) > 48 * 1024) Ry--;
    const size_t smem = smem_of(Ry);
    if (smem <= 96 * 1024 && (Ry + 1) * Lc <= 256) {
      const dim3 grid((C4 + Lc - 1) / Lc, B), blk(Lc, Ry + 1);
#define BNN_DWK4(KK, SS)                                                                                         \
  do {                                                                                                           \
    cudaError_t e_ = cudaFuncSetAttribute(k_dwk4_f16<KK, SS>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                          (int)smem);                                                           \
    if (e_) return e_;                                                                                           \
    k_dwk4_f16<KK, SS><<<grid, blk, smem, st>>>(xp, xws, W, C, pt, pl, w, b, act, out, ows, Ho, Wo, ngr, chsum,  \
                                                cws);                                                            \
  } while (0)
      if (k == 3) { if (s == 1) BNN_DWK4(3, 1); else BNN_DWK4(3, 2); }
      else if (k == 5) { if (s == 1) BNN_DWK4(5, 1); else BNN_DWK4(5, 2); }
      else { if (s == 1) BNN_DWK4(7, 1); else BNN_DWK4(7, 2); }
#undef BNN_DWK4
      return cudaGetLastError();
    }
  }
  // the channel-pair form (any stride and k, 4-byte alignment)
  if (C % 2 || xws % 2 || ows % 2 || ((uintptr_t)xp & 3) || ((uintptr_t)out & 3) || ((uintptr_t)w & 3) ||
      ((uintptr_t)b & 3))
    return cudaErrorInvalidValue;
  const int C2 = C / 2;
  const int Lc = C2 < 32 ? C2 : 32;
  int Ry = Ho < 256 / Lc ? Ho : 256 / Lc;  // rows per chunk: one per thread row
  while (Ry > 1 && (size_t)Ry * ngr * Lc * 4 > 48 * 1024) Ry--;
  const size_t smem = (size_t)Ry * ngr * Lc * 4;
  if (smem > 96 * 1024) return cudaErrorInvalidValue;
  const dim3 grid((C2 + Lc - 1) / Lc, B), blk(Lc, Ry);
#define BNN_DWK(KK)                                                                                              \
  do {                                                                                                           \
    cudaError_t e_ = cudaFuncSetAttribute(k_dwk_f16<KK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e_) return e_;                                                                                           \
    k_dwk_f16<KK><<<grid, blk, smem, st>>>(xp, xws, W, C, s, pt, pl, w, b, act, out, ows, Ho, Wo, ngr, chsum, cws); \
  } while (0)
  switch (k) {
  case 1: BNN_DWK(1); break;
  case 3: BNN_DWK(3); break;
  case 5: BNN_DWK(5); break;
  case 7: BNN_DWK(7); break;
  default: return cudaErrorInvalidValue;
  }
#undef BNN_DWK
  return cudaGetLastError();
}

extern "C" int bnnk_pad_f16(int B, int H, int W, int C, int ld, int h, const uint16_t *x, long long xws, uint16_t *xp,
                            long long pws, bnn_stream_t st) {
  if (B <= 0) return 0;
  if (C % 8 == 0 && ld % 8 == 0 && xws % 8 == 0 && pws % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)xp & 15) == 0) {
    const long long n = (long long)H * W * (C / 8);
    k_pad_f16<8><<<dim3((unsigned)((n + 255) / 256), (unsigned)B), 256, 0, st>>>(H, W, C, ld, h, x, xws, xp, pws);
  } else {
    const long long n = (long long)H * W * C;
    k_pad_f16<1><<<dim3((unsigned)((n + 255) / 256), (unsigned)B), 256, 0, st>>>(H, W, C, ld, h, x, xws, xp, pws);
  }
  return cudaGetLastError();
}

extern "C" int bnnk_mean_f16(int B, int P, int C, int ld, const uint16_t *x, long long xws, float *out, long long ows,
                             bnn_stream_t st) {
  if (B <= 0) return 0;
  k_mean_f16<<<dim3((unsigned)((C + 127) / 128), (unsigned)B), 128, 0, st>>>(P, C, ld, x, xws, out, ows);
  return cudaGetLastError();
}
