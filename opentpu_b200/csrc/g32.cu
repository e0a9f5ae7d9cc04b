// The reference's 4-bit group-32 fp16-scale weight format (its survey quantizer,
// opentpu/quant.py:225-227 -> 132-170): the quantizer, bit-exact in float64 as the reference
// computes it, and the weight-only linear layer over it (fp32 activations, fp32 accumulation;
// the reference's `deq @ x`, tests/test_quant.py:276-287).
//
// Packed layout in HBM: codes [N, K/2] (two's-complement nibbles, element 2i in the low
// nibble), scales [N, K/32] fp16 -- 4.5 bits a weight, streamed once per call.
#include <cuda_runtime.h>

#include <cstdint>

#include "mm_common.cuh"
#include "otq_internal.h"

namespace otq {
namespace {

constexpr int kThreads = 256;

// double -> IEEE binary16 bits, round to nearest even, for 0 <= v <= 65504 (written from the
// format's definition: 10 fraction bits, exponent bias 15, subnormal quantum 2^-24).
__device__ __forceinline__ uint16_t f64_to_f16_bits(double v) {
  if (!(v > 0.0)) return 0;
  if (v < 6.103515625e-05) {                          // below 2^-14: the subnormal grid
    const double r = rint(v * 16777216.0);            // exact scaling by 2^24, then RNE
    return static_cast<uint16_t>(r);                  // 1024 becomes the smallest normal
  }
  int e;
  const double m = frexp(v, &e);                      // v = m 2^e, m in [0.5, 1)
  double frac = rint((m * 2.0 - 1.0) * 1024.0);       // exact, then RNE to 10 bits
  int ex = e - 1;
  if (frac >= 1024.0) {
    frac = 0.0;
    ++ex;
  }
  return static_cast<uint16_t>(((ex + 15) << 10) | static_cast<int>(frac));
}

__device__ __forceinline__ double f16_bits_to_f64(uint16_t h) {
  const int ex = (h >> 10) & 31;
  const int fr = h & 1023;
  if (ex == 0) return ldexp(static_cast<double>(fr), -24);
  return ldexp(1.0 + fr / 1024.0, ex - 15);
}

// One warp per (row, group of 32): lane l holds element l.
__global__ void __launch_bounds__(kThreads) pack_g32_kernel(const float* __restrict__ W,
                                                            int64_t N, int64_t K, int64_t ldw,
                                                            uint8_t* __restrict__ codes,
                                                            uint16_t* __restrict__ scales) {
  const int64_t ng = K / 32;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (task >= N * ng) return;
  const int lane = threadIdx.x & 31;
  const int64_t n = task / ng, g = task % ng;
  const double x = static_cast<double>(W[n * ldw + g * 32 + lane]);
  double amax = fabs(x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmax(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  double s = fmin(amax * 1.0 / 7.0, 65504.0);
  const uint16_t hb = f64_to_f16_bits(s);
  s = f16_bits_to_f64(hb);
  if (amax == 0.0 || s == 0.0) s = 1.0;
  double c = rint(x / s);
  c = fmin(fmax(c, -7.0), 7.0);
  const int nib = static_cast<int>(c) & 15;
  const int other = __shfl_down_sync(0xFFFFFFFFu, nib, 1);
  if ((lane & 1) == 0) codes[n * (K / 2) + g * 16 + (lane >> 1)] =
      static_cast<uint8_t>(nib | (other << 4));
  if (lane == 0) scales[n * ng + g] = (amax == 0.0 || hb == 0) ? static_cast<uint16_t>(0x3C00) : hb;
}

// Both GEMV kernels launch with programmatic dependent launch: a CTA prefetches its first
// weight rows into L2 before griddepcontrol.wait, and reads x and writes y only after it. The
// next launch is released at exit (releasing it after x is staged, or at the start, measured
// slower: its waiting CTAs then hold SM slots this launch's CTAs need). 4-bit Qwen3-0.6B step
// 0.667 -> 0.600 ms.
constexpr bool kG32Pdl = true;

struct G32Params {
  const uint8_t* codes;
  const uint16_t* scales;
  int64_t N;
  int K;
  const float* x;
  int64_t ldx;
  int M;
  int accumulate;
  float* y;
  int64_t ldy;
};

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  float f;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
  return f;
}

// Weight rows [row0, row0 + rows) (clipped to N): codes and scales into L2, a hint issued before
// griddepcontrol.wait (weights never depend on the kernel launched before). Whole 16-byte
// pieces of 16-byte aligned ranges only.
__device__ __forceinline__ void prefetch_rows_l2(const G32Params& p, int64_t row0, int rows) {
  const int64_t n = p.N - row0 < rows ? p.N - row0 : rows;
  const uint8_t* c = p.codes + row0 * (p.K / 2);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(p.scales + row0 * (p.K / 32));
  const uint32_t cb = static_cast<uint32_t>(n * (p.K / 2)) & ~15u;
  const uint32_t sb = static_cast<uint32_t>(n * (p.K / 32) * 2) & ~15u;
  if ((reinterpret_cast<uintptr_t>(c) & 15u) == 0 && cb > 0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(cb) : "memory");
  if ((reinterpret_cast<uintptr_t>(s) & 15u) == 0 && sb > 0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(s), "r"(sb) : "memory");
}

// LPR lanes per weight row, one 16-byte chunk (a whole group) per lane step; activations of
// MT rows in shared memory as fp32. Signed nibbles become exact floats by the 2^23 + u trick.
// The lanes of a row read different groups at once, 128 bytes apart: the same banks. So each
// group's eight float4 are stored rotated by the group's index (float4 v of group c at slot
// (v + c) % 8), and the eight lanes of a quarter warp, reading consecutive groups, hit eight
// different slots: conflict-free (8-way conflicted unrotated).
template <int MT, int LPR>
__global__ void __launch_bounds__(kThreads) linear_g32_kernel(const G32Params p) {
  extern __shared__ __align__(16) float xs[];   // [MT][K]
  constexpr int R = 32 / LPR;
  constexpr int U = 4;
  const int K = p.K;
  const int NC = K >> 5;
  const int lane = threadIdx.x & 31;
  const int li = lane % LPR;
  const int r = lane / LPR;
  const int64_t ntasks = (p.N + R - 1) / R;
  const int64_t wstride = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  const int64_t wfirst = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (lane == 0 && wfirst < ntasks) prefetch_rows_l2(p, wfirst * R, R);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int m0 = 0; m0 < p.M; m0 += MT) {
    const int mt = min(MT, p.M - m0);
    if ((reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 && (p.ldx & 3) == 0) {
      // 16-byte loads, every one of the block's loads issued before the shared-memory stores
      for (int j = 0; j < mt; ++j) {
        const float4* xr = reinterpret_cast<const float4*>(p.x + static_cast<int64_t>(m0 + j) * p.ldx);
        for (int i = threadIdx.x; i < (K >> 2); i += kThreads)
          reinterpret_cast<float4*>(xs + j * K)[(i & ~7) | (((i & 7) + (i >> 3)) & 7)] =
              __ldcg(xr + i);
      }
    } else {
      for (int j = 0; j < mt; ++j)
        for (int i = threadIdx.x; i < K; i += kThreads)
          xs[j * K + ((i & ~31) | (((((i >> 2) & 7) + (i >> 5)) & 7) << 2) | (i & 3))] =
              __ldcg(p.x + static_cast<int64_t>(m0 + j) * p.ldx + i);
    }
    __syncthreads();
    for (int64_t t = wfirst; t < ntasks; t += wstride) {
      const int64_t n = t * R + r;
      const bool valid = n < p.N;
      const uint8_t* crow = p.codes + (valid ? n : 0) * (K / 2);
      const uint16_t* srow = p.scales + (valid ? n : 0) * NC;
      float acc[MT];
#pragma unroll
      for (int j = 0; j < MT; ++j) acc[j] = 0.0f;
      for (int c0 = li; c0 < NC; c0 += LPR * U) {
        uint4 wv[U];
        float sc[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + u * LPR;
          const bool ok = valid && c < NC;
          wv[u] = ok ? ld_stream(crow + static_cast<int64_t>(c) * 16) : make_uint4(0, 0, 0, 0);
          sc[u] = ok ? half_bits_to_float(__ldg(srow + c)) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + u * LPR;
          if (!valid || c >= NC) continue;
          const uint32_t ww[4] = {wv[u].x ^ 0x88888888u, wv[u].y ^ 0x88888888u,
                                  wv[u].z ^ 0x88888888u, wv[u].w ^ 0x88888888u};
          float wf[32];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t bitsv = ((ww[q] >> (4 * e)) & 0xFu) | 0x4B000000u;   // 2^23 + u
              wf[q * 8 + e] = __fsub_rn(__uint_as_float(bitsv), 8388616.0f);     // u - 8
            }
          }
#pragma unroll
          for (int j = 0; j < MT; ++j) {
            if (j < mt) {
              const float4* xp = reinterpret_cast<const float4*>(xs + j * K + c * 32);
              float part = 0.0f;
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const float4 xv = xp[(v + c) & 7];
                part = __fmaf_rn(wf[4 * v + 0], xv.x, part);
                part = __fmaf_rn(wf[4 * v + 1], xv.y, part);
                part = __fmaf_rn(wf[4 * v + 2], xv.z, part);
                part = __fmaf_rn(wf[4 * v + 3], xv.w, part);
              }
              acc[j] = __fmaf_rn(sc[u], part, acc[j]);
            }
          }
        }
      }
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) {
#pragma unroll
        for (int j = 0; j < MT; ++j) acc[j] += __shfl_xor_sync(0xFFFFFFFFu, acc[j], off);
      }
      if (valid) {
#pragma unroll
        for (int j = 0; j < MT; ++j) {
          if (j < mt && (j % LPR) == li) {
            float* yp = p.y + static_cast<int64_t>(m0 + j) * p.ldy + n;
            *yp = p.accumulate ? *yp + acc[j] : acc[j];
          }
        }
      }
    }
    __syncthreads();
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One activation row (decode): one weight row a lane, 32 rows a CTA, the row's groups split over
// the 8 warps, so every lane of a warp reads the same activations (shared-memory broadcasts).
// x is staged as x'[k] = x[k] * 2^(-4 (k % 4)) (exact): nibble p of a half-word, masked in place
// under the exponent of 2^23, is u * 16^p after one subtraction, and its product with x' is
// u * x. With u = code ^ 8 = w + 8, a group adds s * (sum u x - 8 * sum x), the group sums of x
// staged beside x'. Warps' partial sums meet in shared memory in a fixed order.

__global__ void __launch_bounds__(kThreads) linear_g32_row_kernel(const G32Params p) {
  extern __shared__ __align__(16) float sm[];
  const int K = p.K, G = K >> 5;
  float* const xs = sm;            // [K]  x'
  float* const gsum = sm + K;      // [G]  sum of x over each group
  float* const part = gsum + G;    // [8][32] the warps' partial sums
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0 && static_cast<int64_t>(blockIdx.x) * 32 < p.N)
    prefetch_rows_l2(p, static_cast<int64_t>(blockIdx.x) * 32, 32);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if ((reinterpret_cast<uintptr_t>(p.x) & 15u) == 0) {
    // one pass over x, four elements a thread: x' and, over the 8 lanes holding a group, the
    // group's sum (x is read from L2 once; K is a multiple of 32, so groups never straddle a
    // warp and the loop bound is warp-uniform)
    const int K4 = K >> 2;
    for (int base = 0; base < K4; base += kThreads) {
      const int i = base + threadIdx.x;
      const bool in = i < K4;
      const float4 v = in ? __ldcg(reinterpret_cast<const float4*>(p.x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      float sum = __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, 1));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, 2));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, 4));
      if (in) {
        *reinterpret_cast<float4*>(xs + 4 * i) =
            make_float4(v.x, __fmul_rn(v.y, 0.0625f), __fmul_rn(v.z, 0.00390625f),
                        __fmul_rn(v.w, 0.000244140625f));   // x * 2^(-4 (k % 4)), exact
        if ((lane & 7) == 0) gsum[i >> 3] = sum;
      }
    }
  } else {
    for (int i = threadIdx.x; i < K; i += kThreads) {
      const float v = __ldcg(p.x + i);
      xs[i] = __fmul_rn(v, __int_as_float((127 - 4 * (i & 3)) << 23));   // x * 2^(-4 (i % 4))
    }
    for (int g = warp; g < G; g += kThreads / 32) {
      float v = __ldcg(p.x + g * 32 + lane);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
      if (lane == 0) gsum[g] = v;
    }
  }
  __syncthreads();
  const int g0 = warp * G / 8, g1 = (warp + 1) * G / 8;
  const int64_t nblocks = (p.N + 31) / 32;
  constexpr int U = 8;
  for (int64_t rb = blockIdx.x; rb < nblocks; rb += gridDim.x) {   // persistent: x staged once
  const int64_t row = rb * 32 + lane;
  const bool valid = row < p.N;
  const uint8_t* crow = p.codes + (valid ? row : 0) * (K / 2);
  const uint16_t* srow = p.scales + (valid ? row : 0) * G;
  float acc = 0.0f;
  for (int g = g0; g < g1; g += U) {
    uint4 w[U];
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool ok = valid && g + u < g1;
      w[u] = ok ? ld_stream(crow + static_cast<int64_t>(g + u) * 16) : make_uint4(0, 0, 0, 0);
      sc[u] = ok ? half_bits_to_float(__ldg(srow + g + u)) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (g + u >= g1) break;
      const float* xg = xs + (g + u) * 32;
      const uint32_t ws[4] = {w[u].x ^ 0x88888888u, w[u].y ^ 0x88888888u, w[u].z ^ 0x88888888u,
                              w[u].w ^ 0x88888888u};
      float pa = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 x0 = *reinterpret_cast<const float4*>(xg + 8 * q);
        const float4 x1 = *reinterpret_cast<const float4*>(xg + 8 * q + 4);
        const uint32_t lo = ws[q], hi = ws[q] >> 16;
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t h = e < 4 ? lo : hi;
          const uint32_t bitsv = (h & (0xFu << (4 * (e & 3)))) | 0x4B000000u;   // 2^23 + u 16^p
          pa = __fmaf_rn(__fsub_rn(__uint_as_float(bitsv), 8388608.0f), xv[e], pa);
        }
      }
      acc = __fmaf_rn(sc[u], __fmaf_rn(-8.0f, gsum[g + u], pa), acc);
    }
  }
  part[warp * 32 + lane] = acc;
  __syncthreads();
  if (warp == 0 && valid) {
    float v = part[lane];
#pragma unroll
    for (int w2 = 1; w2 < kThreads / 32; ++w2) v = __fadd_rn(v, part[w2 * 32 + lane]);
    float* yp = p.y + row;
    *yp = p.accumulate ? __fadd_rn(*yp, v) : v;
  }
  __syncthreads();   // part is rewritten by the next row block
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One activation row on the tensor pipe (K a multiple of 256). Per 32-element group g, x becomes
// the fixed-point integer xi = rint(x * 2^e_g), |xi| < 2^30 (e_g from the group's largest |x|:
// at most 2^-30 of it is lost), split into four signed base-256 digits (limbs). A code (a
// code plus 8 (u in 0..15) times a limb summed over the group is an exact int32: one mma.sync
// m16n8k32 (u8 x s8) gives, for 16 weight rows, the group's four limb sums D_j (the MMA's
// columns 0-3), and sum_k w_k x_k = 2^-e_g (sum_j 256^j D_j - 8 sum_k xi_k). A thread holds two
// adjacent limbs of a row, P = D_2t + 256 D_2t+1 - C_t (|P| < 2^24, exact in fp32; C_t the
// limbs' share of 8 sum xi), and adds s_g 2^-e_g P into a fp32 sum (the limb weight 1 or 2^16
// applied once at the end): every integer product is exact and the fp32 sums round like the FMA
// form's, within the 4-bit tolerance.
//
// A CTA (8 warps; two an SM for K up to about 5000) takes a block of 16 weight rows at a time and splits its K chunks (8 groups,
// 128 bytes of codes a row) over the warps (chunk c to warp c % 8, every warp one at least);
// each warp streams its chunks of the CTA's row blocks through a cp.async ring (piece q of row r
// at q ^ (r % 8): conflict-free fragment reads, rows r and r + 8 one address apart; the 16 rows'
// 8 fp16 scales),
// and the warps' row sums meet in shared memory in a fixed order. x's limbs (in the MMA's K
// order), 2^-e_g and the corrections C are built once a CTA.
constexpr int kMmaStages = 4;
constexpr int kChunkGroups = 8;                       // groups a K chunk (128 bytes of codes)
constexpr int kStageCodes = 16 * 128;                 // 16 rows x 128 bytes
constexpr int kStageBytes = kStageCodes + 16 * 16;    // + 16 rows x 8 fp16 scales

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}

// The two halves of a word of two fp16 -> fp32.
__device__ __forceinline__ float half_lo(uint32_t w) {
  float f;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, l; }" : "=f"(f) : "r"(w));
  return f;
}
__device__ __forceinline__ float half_hi(uint32_t w) {
  float f;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, h; }" : "=f"(f) : "r"(w));
  return f;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

size_t g32_mma_smem(int K) {
  return static_cast<size_t>(K / 32) * 140 + 2 * 8 * 16 * 4 +
         static_cast<size_t>(8) * kMmaStages * kStageBytes;
}

__global__ void __launch_bounds__(kThreads, 2) linear_g32_mma_kernel(const G32Params p) {
  extern __shared__ __align__(16) unsigned char gsm[];
  const int K = p.K, G = K >> 5, nch = G / kChunkGroups;
  // [G][4 limbs][32 K slots] limbs; [G] 2^-e_g; [G][2] corrections; [2][8 warps][16 rows]
  // partial sums; the rings
  uint8_t* const xl = gsm;
  float* const xf = reinterpret_cast<float*>(gsm + G * 128);
  int* const corr = reinterpret_cast<int*>(xf + G);
  float* const part = reinterpret_cast<float*>(corr + 2 * G);
  unsigned char* const ring = gsm + G * 140 + 2 * 8 * 16 * 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int64_t nblocks = (p.N + 15) / 16;
  if (threadIdx.x == 0 && static_cast<int64_t>(blockIdx.x) * 16 < p.N)
    prefetch_rows_l2(p, static_cast<int64_t>(blockIdx.x) * 16, 16);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // x -> limbs: a warp a group at a time, lane l holding element l, stored at the K slot s
  // whose element is l (slots 4t + i hold elements 8t + 2i, slots 16 + 4t + i elements 8t + 2i + 1)
  const int slot = (lane & 1) ? 16 + 4 * (lane >> 3) + ((lane >> 1) & 3)
                              : 4 * (lane >> 3) + ((lane >> 1) & 3);
  for (int g = warp; g < G; g += kThreads / 32) {
    const float v = __ldcg(p.x + g * 32 + lane);
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    // e = 29 - exponent(m), at most 126 (|x| tiny or zero): m 2^e in [2^29, 2^30)
    const int e = m > 0.0f ? min(126, 156 - static_cast<int>((__float_as_uint(m) >> 23) & 255u))
                           : 0;
    int r = __float2int_rn(__fmul_rn(v, __int_as_float((127 + e) << 23)));
    int lj[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lj[j] = j < 3 ? ((r + 128) & 255) - 128 : r;   // |r| <= 64 for the last
      xl[g * 128 + j * 32 + slot] = static_cast<uint8_t>(lj[j]);
      r = (r - lj[j]) >> 8;
    }
    // C_t = 8 (sum_k l_2t + 256 sum_k l_2t+1): the bias of u = code + 8 in limbs 2t, 2t + 1
    int c01 = lj[0] + 256 * lj[1], c23 = lj[2] + 256 * lj[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      c01 += __shfl_xor_sync(0xFFFFFFFFu, c01, o);
      c23 += __shfl_xor_sync(0xFFFFFFFFu, c23, o);
    }
    if (lane == 0) {
      xf[g] = __int_as_float((127 - e) << 23);
      corr[2 * g] = 8 * c01;
      corr[2 * g + 1] = 8 * c23;
    }
  }
  __syncthreads();

  // this warp's items: for each of the CTA's row blocks, its chunks warp, warp + 8, ...
  const int per_block = (nch - 1 - warp) / 8 + 1;   // nch >= 8: at least one
  const int64_t my_blocks = nblocks > blockIdx.x ? (nblocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total = my_blocks * per_block;
  const uint32_t wbase = static_cast<uint32_t>(__cvta_generic_to_shared(ring)) +
                         static_cast<uint32_t>(warp * kMmaStages * kStageBytes);
  // the copy side's position (row block, chunk, stage), advanced one item a call; a lane's
  // sources (its 4 code pieces, lanes 0-15 a scale row) advance 8 chunks a step within a row
  // block and are recomputed at the next row block (a row past N copies zeros)
  int64_t irb = blockIdx.x;
  int ici = 0, ist = 0;
  int64_t issued = 0;
  const uint8_t* csrc[4];
  uint32_t cbytes[4], cdst[4];
  const uint16_t* ssrc = p.scales;
  uint32_t sbytes = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int pc = lane + 32 * i, r = pc >> 3, q = pc & 7;
    cdst[i] = static_cast<uint32_t>(r * 128 + ((q ^ (r & 7)) * 16));
  }
  auto set_rows = [&]() {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pc = lane + 32 * i, r = pc >> 3, q = pc & 7;
      const int64_t row = irb * 16 + r;
      const bool ok = row < p.N;
      csrc[i] = p.codes + (ok ? row : 0) * (K / 2) + warp * 128 + q * 16;
      cbytes[i] = ok ? 16u : 0u;
    }
    const int64_t row = irb * 16 + (lane & 15);
    const bool ok = row < p.N && lane < 16;
    ssrc = p.scales + (ok ? row : 0) * G + warp * kChunkGroups;
    sbytes = ok ? 16u : 0u;
  };
  set_rows();
  auto issue = [&]() {
    if (issued < total) {
      const uint32_t st = wbase + static_cast<uint32_t>(ist * kStageBytes);
#pragma unroll
      for (int i = 0; i < 4; ++i) cp_async16(st + cdst[i], csrc[i], cbytes[i]);
      if (lane < 16) cp_async16(st + kStageCodes + lane * 16, ssrc, sbytes);
      ++issued;
      if (++ici == per_block) {
        ici = 0;
        irb += gridDim.x;
        set_rows();
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) csrc[i] += 8 * 128;
        ssrc += 8 * kChunkGroups;
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (++ist == kMmaStages) ist = 0;
  };
  for (int i = 0; i < kMmaStages - 1; ++i) issue();
  float a0s = 0.f, a1s = 0.f;   // rows gid, gid + 8: this thread's limb pair
  const float wt = tig == 0 ? 1.0f : 65536.0f;
  // the compute side's position: row block (its index among this CTA's), chunk, stage; the
  // fragment reads through 32-bit shared addresses
  int64_t blk = 0;
  int ci = 0, cst = 0;
  const uint32_t xl_s = static_cast<uint32_t>(__cvta_generic_to_shared(xl)) + gid * 32 + 4 * tig;
  const uint32_t xf_s = static_cast<uint32_t>(__cvta_generic_to_shared(xf));
  const uint32_t cr_s = static_cast<uint32_t>(__cvta_generic_to_shared(corr)) + 4 * (tig & 1);
  for (int64_t it = 0; it < total; ++it) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kMmaStages - 2) : "memory");
    __syncwarp();
    const uint32_t st = wbase + static_cast<uint32_t>(cst * kStageBytes);
    const int c = warp + 8 * ci;
    // the chunk's 8 scales of rows gid and gid + 8, its 2^-e_g
    const uint4 s0 = lds128(st + kStageCodes + gid * 16);
    const uint4 s1 = lds128(st + kStageCodes + (gid + 8) * 16);
    const uint4 f0 = lds128(xf_s + c * kChunkGroups * 4);
    const uint4 f1 = lds128(xf_s + c * kChunkGroups * 4 + 16);
    const uint32_t sw0[4] = {s0.x, s0.y, s0.z, s0.w}, sw1[4] = {s1.x, s1.y, s1.z, s1.w};
    const uint32_t fv[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
    const uint32_t arow = st + gid * 128 + 4 * tig;
    const uint32_t xlc = xl_s + c * kChunkGroups * 128;
    const uint32_t cc = cr_s + c * kChunkGroups * 8;
#pragma unroll
    for (int q = 0; q < kChunkGroups; ++q) {
      const uint32_t ap = arow + ((q ^ gid) * 16);
      const uint32_t wa = lds32(ap);
      const uint32_t wb = lds32(ap + 8 * 128);
      uint32_t a0, a1, a2, a3;
      int4_bytes(wa, a0, a2);
      int4_bytes(wb, a1, a3);
      uint32_t b0 = 0u, b1 = 0u;   // columns 4-7 stay zero
      if (gid < 4) {
        b0 = lds32(xlc + q * 128);
        b1 = lds32(xlc + q * 128 + 16);
      }
      int d[4];
      asm volatile(
          "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%10,%10,%10,%10};"
          : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
      const int cq = static_cast<int>(lds32(cc + q * 8));
      const float sc0 = (q & 1) ? half_hi(sw0[q >> 1]) : half_lo(sw0[q >> 1]);
      const float sc1 = (q & 1) ? half_hi(sw1[q >> 1]) : half_lo(sw1[q >> 1]);
      const float fq = __uint_as_float(fv[q]);
      const float p0 = static_cast<float>(d[0] + 256 * d[1] - cq);
      const float p1 = static_cast<float>(d[2] + 256 * d[3] - cq);
      a0s = __fmaf_rn(__fmul_rn(sc0, fq), p0, a0s);
      a1s = __fmaf_rn(__fmul_rn(sc1, fq), p1, a1s);
    }
    __syncwarp();
    issue();
    if (++cst == kMmaStages) cst = 0;
    if (++ci == per_block) {
      // this warp's last chunk of the row block: its rows' sums, then every warp's in order
      ci = 0;
      float v0 = tig < 2 ? __fmul_rn(a0s, wt) : 0.0f;
      float v1 = tig < 2 ? __fmul_rn(a1s, wt) : 0.0f;
      v0 = __fadd_rn(v0, __shfl_xor_sync(0xFFFFFFFFu, v0, 1));
      v1 = __fadd_rn(v1, __shfl_xor_sync(0xFFFFFFFFu, v1, 1));
      float* const pb = part + (blk & 1) * 128;
      if (tig == 0) {
        pb[warp * 16 + gid] = v0;
        pb[warp * 16 + gid + 8] = v1;
      }
      a0s = a1s = 0.f;
      __syncthreads();   // every warp calls it once a row block, in the same order
      if (threadIdx.x < 16) {
        const int64_t row = (blockIdx.x + blk * gridDim.x) * 16 + threadIdx.x;
        float v = pb[threadIdx.x];
#pragma unroll
        for (int w2 = 1; w2 < kThreads / 32; ++w2) v = __fadd_rn(v, pb[w2 * 16 + threadIdx.x]);
        if (row < p.N) {
          float* yp = p.y + row;
          *yp = p.accumulate ? __fadd_rn(*yp, v) : v;
        }
      }
      ++blk;
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

int launch_g32_mma(const G32Params& p, cudaStream_t stream) {
  const size_t smem = g32_mma_smem(p.K);
  static size_t configured[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (configured[dev] < smem) {
    if (cudaFuncSetAttribute(linear_g32_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = smem;
  }
  static int occ_cache[kMaxDevices] = {0};
  static size_t occ_smem[kMaxDevices] = {0};
  if (occ_cache[dev] == 0 || occ_smem[dev] != smem) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, linear_g32_mma_kernel, kThreads,
                                                      smem) != cudaSuccess)
      return kErrCuda;
    occ_cache[dev] = occ > 0 ? occ : 1;
    occ_smem[dev] = smem;
  }
  const int64_t blocks = (p.N + 15) / 16;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * occ_cache[dev];
  return launch_kernel(reinterpret_cast<const void*>(linear_g32_mma_kernel),
                       static_cast<int>(blocks < cap ? blocks : cap), kThreads, smem, stream,
                       kG32Pdl, p);
}

int launch_g32_row(const G32Params& p, cudaStream_t stream) {
  const size_t smem = (static_cast<size_t>(p.K) + p.K / 32 + kThreads) * 4;
  static size_t configured[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (smem > 48 * 1024 && configured[dev] < smem) {
    if (cudaFuncSetAttribute(linear_g32_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = smem;
  }
  static int occ_cache[kMaxDevices] = {0};
  if (occ_cache[dev] == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, linear_g32_row_kernel, kThreads,
                                                      smem) != cudaSuccess)
      return kErrCuda;
    occ_cache[dev] = occ > 0 ? occ : 1;
  }
  const int64_t blocks = (p.N + 31) / 32;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * occ_cache[dev];
  return launch_kernel(reinterpret_cast<const void*>(linear_g32_row_kernel),
                       static_cast<int>(blocks < cap ? blocks : cap), kThreads, smem, stream, kG32Pdl,
                       p);
}

template <int MT, int LPR>
int launch_g32(const G32Params& p, cudaStream_t stream) {
  auto kern = linear_g32_kernel<MT, LPR>;
  const size_t smem = static_cast<size_t>(MT) * p.K * 4;
  static int configured[kMaxDevices] = {0};
  static int occ_cache[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (smem > 48 * 1024 && configured[dev] < static_cast<int>(smem)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = static_cast<int>(smem);
    occ_cache[dev] = 0;
  }
  if (occ_cache[dev] == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess)
      return kErrCuda;
    occ_cache[dev] = occ > 0 ? occ : 1;
  }
  constexpr int R = 32 / LPR;
  const int64_t ntasks = (p.N + R - 1) / R;
  const int64_t want = (ntasks + 7) / 8;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * occ_cache[dev];
  return launch_kernel(reinterpret_cast<const void*>(kern), static_cast<int>(want < cap ? want : cap),
                       kThreads, smem, stream, kG32Pdl, p);
}

template <int MT>
int launch_g32_lpr(const G32Params& p, cudaStream_t stream, int lpr) {
  switch (lpr) {
    case 4: return launch_g32<MT, 4>(p, stream);
    case 8: return launch_g32<MT, 8>(p, stream);
    case 16: return launch_g32<MT, 16>(p, stream);
    default: return launch_g32<MT, 32>(p, stream);
  }
}

}  // namespace

int pack_g32_launch(const float* W, int64_t N, int64_t K, int64_t ldw, uint8_t* codes,
                    uint16_t* scales, cudaStream_t stream) {
  const int64_t tasks = N * (K / 32);
  if (tasks == 0) return kOk;
  const int64_t blocks = (tasks + 7) / 8;
  if (blocks > 0x7FFFFFFF) return kErrArg;
  pack_g32_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(W, N, K, ldw, codes,
                                                                          scales);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int linear_g32_launch(const uint8_t* codes, const uint16_t* scales, int64_t N, int K,
                      const float* x, int64_t ldx, int M, int accumulate, float* y, int64_t ldy,
                      cudaStream_t stream) {
  G32Params p{codes, scales, N, K, x, ldx, M, accumulate, y, ldy};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  // one activation row: 16-row blocks on the tensor pipe when K is whole 8-group chunks, at
  // least 8 of them (one a warp), the fixed-point limbs fit shared memory and the codes and
  // scales are 16-byte aligned (cp.async); else a weight row a lane, once there are enough
  // 32-row blocks to fill the GPU
  const bool al16 = (reinterpret_cast<uintptr_t>(codes) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(scales) & 15u) == 0;
  if (M == 1 && al16 && K % 256 == 0 && K >= 2048 && g32_mma_smem(K) <= 220 * 1024)
    return launch_g32_mma(p, stream);
  if (M == 1 && (N + 31) / 32 >= 64) return launch_g32_row(p, stream);
  const int nc = K / 32;
  int lpr = 4;
  while (lpr < 32 && nc / lpr > 8) lpr *= 2;
  while (lpr < 32 && N * lpr / 32 < static_cast<int64_t>(sm_count(dev)) * 16) lpr *= 2;
  if (M <= 1) return launch_g32_lpr<1>(p, stream, lpr);
  if (M <= 2 || static_cast<int64_t>(K) * 4 * 4 > 200 * 1024) return launch_g32_lpr<2>(p, stream, lpr);
  return launch_g32_lpr<4>(p, stream, lpr);
}

}  // namespace otq
