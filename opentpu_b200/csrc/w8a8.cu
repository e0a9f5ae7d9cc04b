// The exact int8 linear layer on the tensor cores: QACT activations x int8-row weights with
// tcgen05.mma kind::i8, for M > 1 (prefill, batched decode), bit-identical to the reference's MM.
//
// The reference's MM (opentpu/isasim.py:749-910, docs/isa.md "MM") for int8 weights with one
// scale a row (RSC) or none (UNIT) and QACT activations (q int8, S, an offset d per 32
// elements, opentpu/fp32.py:321-343) computes for output (m, n)
//     acc = sum over groups g with d(m,g) <= 16 of 2^(16 - d(m,g)) * sum_{k in g} q[m,k] w[n,k]
//     y   = (i2f(acc) * Sw[n]) * (S[m] * 2^-16)            (RNE, flushed: mm_epilogue)
// The shift depends on the row m and the group g, so it cannot be applied to one int32
// accumulator after a K-long MMA. It is folded into the activations instead: with D(m) the
// largest kept offset of row m, every kept element becomes the integer
//     a'[m,k] = q[m,k] * 2^(D(m) - d(m,g))                 (|a'| <= 127 * 2^16)
// and acc = 2^(16 - D(m)) * sum_k a'[m,k] w[n,k]. a' is split into signed base-256 digits,
// the planes: a' = p0 + 256 p1 + 65536 p2, p0 and p1 balanced residues in [-128, 127], p2 in
// [-127, 127]. Each plane is an int8 matrix and its product with the weights an exact int32 MMA
// (|p w| K <= 128 * 127 * K < 2^31 for K < 2^17); the epilogue recombines
//     acc = (c0 + 256 c1 + 65536 c2) << (16 - D(m))
// in 64-bit integers -- the reference's integer -- so y is bit-identical. A row needs 1 plane
// when D(m) = 0 (every group at the row's scale; QACT ROW mode), 2 when D(m) <= 8, else 3; a
// projection runs as many planes as its rows need at most. (N(0, 1) rows mostly have D = 1:
// two planes.)
//
// Two kernels:
//   qact_planes_kernel  one CTA a row: QACT (the arithmetic of qact.cuh), D(m), the planes,
//                       S[m], the shift 16 - D(m) and the row's plane count (the "planes"
//                       buffer, otq_qact_planes);
//   w8a8_kernel         a persistent CTA an SM over tiles of 128 weight rows x NT tokens
//                       (NT = 16 .. 128): the weight rows are the MMA's A (M = 128,
//                       tensor-memory lanes), the planes of NT tokens its B, stacked along N
//                       (plane j's tokens at columns j NT ..), so one MMA (N = planes x NT <= 256,
//                       else 256 + the rest) does every plane of a K step.
//     warp 0        TMA producer: per K chunk of 128 bytes, the weight box (128 rows) and one
//                   box of NT rows a plane (128-byte swizzle, the K-major layout the MMA reads)
//                   into a ring of stages (full / empty mbarriers);
//     warp 1        allocates the 512 tensor-memory columns; lane 0 issues the MMAs (K 32 each,
//                   four a chunk) into one of two accumulator slots, commits the stage back to
//                   the producer and, after the tile's last chunk, the slot to the epilogue;
//     warps 2-9     epilogue: warp w reads lanes 32 (w % 4) .. (its 32 weight rows) and half of
//                   the tile's tokens, recombines the planes' int32 columns in 64 bits, shifts,
//                   and writes y[m, n] = mm_epilogue(acc, Sw[n], S[m], 16) (fadd into the old y
//                   with ACC): a token's 32 outputs of a warp are one 128-byte store. Two slots
//                   let the epilogue of one tile run under the next tile's MMAs.
// Every mbarrier wait is bounded (mm_common.cuh): a wait that runs out sets bit 0 of the
// library's status word and the CTA stops, letting its copies and MMAs finish (bounded) before
// it frees tensor memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <queue>
#include <vector>

#include "mm_common.cuh"
#include "otq_fp32.cuh"
#include "otq_internal.h"
#include "qact.cuh"
#include "tcgen05.cuh"

namespace otq {
namespace {

// ------------------------------------------------------------------ the planes buffer
// For M rows of K (Mp = M rounded up to 128; rows M .. Mp - 1 are zero):
//   [0, 4 Mp)          S       fp32, the row's QACT scale
//   [4 Mp, 8 Mp)       shift   int32, 16 - D(m)
//   [8 Mp, 9 Mp)       planes  uint8, the row's plane count (1 .. 3)
//   [9 Mp, ...)        plane j, row m at 9 Mp + (j Mp + m) K: int8 [3][Mp][K]
struct PlanesView {
  float* S;
  int* shift;
  uint8_t* count;
  int8_t* data;
};

__host__ __device__ inline int64_t rows_padded(int64_t M) { return (M + 127) / 128 * 128; }

__host__ __device__ inline PlanesView planes_view(void* base, int64_t M) {
  const int64_t Mp = rows_padded(M);
  uint8_t* b = static_cast<uint8_t*>(base);
  return PlanesView{reinterpret_cast<float*>(b), reinterpret_cast<int*>(b + 4 * Mp), b + 8 * Mp,
                    reinterpret_cast<int8_t*>(b + 9 * Mp)};
}

constexpr int kQThreads = 512;
constexpr int kQWarps = kQThreads / 32;

struct PlanesParams {
  const float* x;
  int64_t ldx;
  int64_t M;
  int K;
  int row_mode;
  void* planes;
};

// One signed base-256 digit of v (balanced: [-128, 127]) and the rest (v - digit) / 256.
__device__ __forceinline__ int digit(int v, int& rest) {
  const int p = ((v + 128) & 255) - 128;
  rest = (v - p) >> 8;   // exact: v - p is a multiple of 256
  return p;
}

// QACT of one row (the reference's quantize_mx with 32-element groups: the arithmetic of
// qact.cuh's qact_row, step for step) written as planes. A group's offset d depends only on the
// row's and the group's magnitude maxima, so D, the largest kept offset, is known after the
// first pass, and the second pass writes each element's planes straight away.
__global__ void __launch_bounds__(kQThreads) qact_planes_kernel(const PlanesParams p) {
  extern __shared__ __align__(16) uint32_t qsm[];
  const int K = p.K, G = K >> 5;
  const int64_t Mp = rows_padded(p.M);
  const int64_t row = blockIdx.x;
  const PlanesView v = planes_view(p.planes, p.M);
  int8_t* const out0 = v.data + row * K;
  int8_t* const out1 = out0 + Mp * K;
  int8_t* const out2 = out1 + Mp * K;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (row >= p.M) {   // padding rows: zero planes (read by the MMA, never stored)
    for (int i = threadIdx.x * 4; i < K; i += kQThreads * 4) {
      *reinterpret_cast<uint32_t*>(out0 + i) = 0u;
      *reinterpret_cast<uint32_t*>(out1 + i) = 0u;
      *reinterpret_cast<uint32_t*>(out2 + i) = 0u;
    }
    if (threadIdx.x == 0) {
      v.S[row] = 0.0f;
      v.shift[row] = 0;
      v.count[row] = 1;
    }
    return;
  }
  float* xs = reinterpret_cast<float*>(qsm);
  uint32_t* seg = qsm + K;        // [G] group magnitude maxima (bit patterns)
  uint32_t* red = seg + G;        // [kQWarps + 3] the reductions
  const ThreadGroup<kQThreads> grp{static_cast<int>(threadIdx.x)};
  stage_row(grp, p.x + row * p.ldx, xs, K);
  // pass 1: group maxima and the row maximum (amax by bit pattern after the flush)
  uint32_t tmax = 0u;
  for (int g = warp; g < G; g += kQWarps) {
    const uint32_t mb = __float_as_uint(otq_flush(xs[(g << 5) + lane])) & 0x7FFFFFFFu;
    const uint32_t gm = __reduce_max_sync(0xFFFFFFFFu, mb);
    if (lane == 0) seg[g] = gm;
    tmax = gm > tmax ? gm : tmax;
  }
  if (lane == 0) red[warp] = tmax;
  __syncthreads();
  if (warp == 0) {
    uint32_t m = lane < kQWarps ? red[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0) {
      float S = 0.0f, inv = 0.0f;
      if (m != 0u) {
        const float amax = __uint_as_float(m);
        S = fmul(amax, __uint_as_float(kInv127Bits));
        inv = fmul(127.0f, recip(amax));
      }
      red[kQWarps] = __float_as_uint(S);
      red[kQWarps + 1] = __float_as_uint(inv);
      red[kQWarps + 2] = m;
    }
  }
  __syncthreads();
  const float S = __uint_as_float(red[kQWarps]);
  const float inv = __uint_as_float(red[kQWarps + 1]);
  const uint32_t amax_bits = red[kQWarps + 2];
  const bool row_mode = p.row_mode != 0;
  // D = the largest kept offset (groups with d > 16 are dropped by MM)
  int dl = 0;
  if (!row_mode)
    for (int g = threadIdx.x; g < G; g += kQThreads) {
      const int d = group_offset(seg[g], amax_bits);
      if (d <= 16) dl = max(dl, d);
    }
  dl = __reduce_max_sync(0xFFFFFFFFu, dl);
  __syncthreads();   // red[0 .. kQWarps) is read above by warp 0 only; reuse it now
  if (lane == 0) red[warp] = static_cast<uint32_t>(dl);
  __syncthreads();
  int D = 0;
#pragma unroll
  for (int w = 0; w < kQWarps; ++w) D = max(D, static_cast<int>(red[w]));
  // pass 2: q = q8(x * (inv * 2^d)), a' = q * 2^(D - d) (0 for a dropped group), its digits
  for (int g = warp; g < G; g += kQWarps) {
    const int d = row_mode ? 0 : group_offset(seg[g], amax_bits);
    const int i = (g << 5) + lane;
    int a = 0;
    if (d <= 16) a = q8(fmul(xs[i], fmul(inv, pow2i(d)))) * (1 << (D - d));
    int r1, r2;
    const int p0 = digit(a, r1);
    const int p1 = digit(r1, r2);
    out0[i] = static_cast<int8_t>(p0);
    out1[i] = static_cast<int8_t>(p1);
    out2[i] = static_cast<int8_t>(r2);
  }
  if (threadIdx.x == 0) {
    v.S[row] = S;
    v.shift[row] = 16 - D;
    v.count[row] = static_cast<uint8_t>(D == 0 ? 1 : (D <= 8 ? 2 : 3));
  }
}

// ------------------------------------------------------------------ the tensor-core MM
constexpr int kWR = 128;                 // weight rows a tile: the MMA's M, tensor-memory lanes
constexpr int kKC = 128;                 // K a chunk: one 128-byte swizzle row of int8
constexpr int kUK = 32;                  // K of one kind::i8 MMA
constexpr int kWBytes = kWR * kKC;       // 16 KB of weights a stage
constexpr int kEpi0 = 2;                 // first epilogue warp
constexpr int kEpiWarps = 8;             // two a tensor-memory lane quarter
constexpr int kThreads = 32 * (kEpi0 + kEpiWarps);
constexpr int kMaxStages = 8;
constexpr int kStageBudget = 200 * 1024;
constexpr uint32_t kTmemCols = 512;
constexpr int kSlotCols = 256;           // an accumulator slot (two when planes x NT <= 256)
constexpr int kMaxUnits = 2048;
constexpr int kMaxCtas = 256;

struct alignas(64) G8Proj {
  CUtensorMap wmap;   // rows [N, K] int8: box 128 bytes x 128 rows, 128-byte swizzle
  CUtensorMap pmap;   // planes [3 Mp, K] int8: box 128 bytes x NT rows, 128-byte swizzle
  const uint8_t* srows;
  float* y;
  const float* S;
  const int* shift;
  const uint8_t* count;
  int64_t srs, ldy, M, N, Mp;
  int nk, tiles_t, tile0, flags;
};

struct G8Args {
  G8Proj proj[kW8A8MaxGroup];
  uint32_t units[kMaxUnits];   // projection (3 bits) | token tile (8 bits) << 3 | row tile << 11
  uint16_t first[kMaxCtas + 1];
  int count, nunits, table, nt;
  int* status;
};

struct Bars {
  uint64_t full[kMaxStages], empty[kMaxStages], acc_full[2], acc_empty[2], drain;
  uint32_t tmem;
  int bad;
  int planes[kW8A8MaxGroup];   // planes a projection runs (its rows' largest count)
};

// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), signed A and B (bits 7,
// 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t idesc_s8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 8 consecutive int32 columns of this warp's 32 lanes from `np` planes `stride` columns apart
// (the wait in the same statement: no use of r moves above it).
__device__ __forceinline__ void tmem_planes8(uint32_t taddr, int stride, int np, uint32_t (&r)[3][8]) {
  if (np == 1) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]),
          "=r"(r[0][5]), "=r"(r[0][6]), "=r"(r[0][7])
        : "r"(taddr)
        : "memory");
  } else if (np == 2) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]),
          "=r"(r[0][5]), "=r"(r[0][6]), "=r"(r[0][7]), "=r"(r[1][0]), "=r"(r[1][1]),
          "=r"(r[1][2]), "=r"(r[1][3]), "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]), "=r"(r[1][7])
        : "r"(taddr), "r"(taddr + stride)
        : "memory");
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%24];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%25];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%26];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]),
          "=r"(r[0][5]), "=r"(r[0][6]), "=r"(r[0][7]), "=r"(r[1][0]), "=r"(r[1][1]),
          "=r"(r[1][2]), "=r"(r[1][3]), "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]), "=r"(r[1][7]),
          "=r"(r[2][0]), "=r"(r[2][1]), "=r"(r[2][2]), "=r"(r[2][3]), "=r"(r[2][4]),
          "=r"(r[2][5]), "=r"(r[2][6]), "=r"(r[2][7])
        : "r"(taddr), "r"(taddr + stride), "r"(taddr + 2 * stride)
        : "memory");
  }
}

struct Unit8 {
  int p, t0, n0;
};

__device__ __forceinline__ Unit8 unit8_at(const G8Args& g, int j) {
  uint32_t e;
  if (g.table) {
    e = g.units[j];
  } else {   // round robin: the token tiles of a row tile are consecutive units
    int p = 0;
    while (p + 1 < g.count && j >= g.proj[p + 1].tile0) ++p;
    const int r = j - g.proj[p].tile0, tt = g.proj[p].tiles_t;
    e = static_cast<uint32_t>(p) | (static_cast<uint32_t>(r % tt) << 3) |
        (static_cast<uint32_t>(r / tt) << 11);
  }
  Unit8 u;
  u.p = static_cast<int>(e & 7u);
  u.t0 = static_cast<int>((e >> 3) & 0xFFu) * g.nt;
  u.n0 = static_cast<int>(e >> 11) * kWR;
  return u;
}

struct Span8 {
  int begin, end, step;
};
__device__ __forceinline__ Span8 my_units8(const G8Args& g) {
  if (g.table) return Span8{g.first[blockIdx.x], g.first[blockIdx.x + 1], 1};
  return Span8{static_cast<int>(blockIdx.x), g.nunits, static_cast<int>(gridDim.x)};
}

__global__ void __launch_bounds__(kThreads, 1) w8a8_kernel(const __grid_constant__ G8Args g) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ Bars bars;
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* const status = g.status;
  const int NT = g.nt;

  // the planes each projection runs: warp p reads projection p's row counts
  if (warp < g.count) {
    const uint8_t* cnt = g.proj[warp].count;
    const int64_t M = g.proj[warp].M;
    uint32_t mx = 1u;
    for (int64_t m = lane; m < M; m += 32) mx = max(mx, static_cast<uint32_t>(cnt[m]));
    mx = __reduce_max_sync(0xFFFFFFFFu, mx);
    if (lane == 0) bars.planes[warp] = static_cast<int>(min(mx, 3u));
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(smem_addr(&bars.full[i]), 1);
      mbar_init(smem_addr(&bars.empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&bars.acc_full[i]), 1);
      mbar_init(smem_addr(&bars.acc_empty[i]), kEpiWarps);   // one arrival an epilogue warp
    }
    mbar_init(smem_addr(&bars.drain), 1);
    bars.bad = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane < g.count) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.proj[lane].wmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.proj[lane].pmap)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&bars.tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;
  int pmax = 1;
  for (int p = 0; p < g.count; ++p) pmax = max(pmax, bars.planes[p]);
  // the stage ring and the accumulator slots for the largest plane count of the launch
  const uint32_t stage_bytes = kWBytes + static_cast<uint32_t>(pmax * NT * kKC);
  const int nstage = min(kMaxStages, static_cast<int>(kStageBudget / stage_bytes));
  const int nslot = pmax * NT <= kSlotCols ? 2 : 1;
  const Span8 sp = my_units8(g);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, c = 0;
      bool ok = true;
      for (int j = sp.begin; j < sp.end && ok; j += sp.step) {
        const Unit8 u = unit8_at(g, j);
        const G8Proj& P = g.proj[u.p];
        const int np = bars.planes[u.p], nk = P.nk;
        const int64_t Mp = P.Mp;
        const uint32_t bytes = kWBytes + static_cast<uint32_t>(np * NT * kKC);
        for (int kb = 0; kb < nk; ++kb) {
          if (c >= static_cast<uint32_t>(nstage) &&
              !mbar_wait(smem_addr(&bars.empty[s]), ph ^ 1u, status)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_addr(&bars.full[s]);
          const uint32_t st = sbase + static_cast<uint32_t>(s) * stage_bytes;
          mbar_arrive_expect_tx(full, bytes);
          tma_2d(st, &P.wmap, kb * kKC, u.n0, full);
          for (int pl = 0; pl < np; ++pl)
            tma_2d(st + kWBytes + static_cast<uint32_t>(pl * NT * kKC), &P.pmap, kb * kKC,
                   static_cast<int>(pl * Mp + u.t0), full);
          ++c;
          if (++s == nstage) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        atomicOr(&bars.bad, 1);
        // the copies still in flight land before the shared memory is given up
        const uint32_t n = static_cast<uint32_t>(nstage);
        for (uint32_t i = c > n ? c - n : 0; i < c; ++i)
          mbar_wait(smem_addr(&bars.full[i % n]), (i / n) & 1u, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, slot = 0;
      uint32_t ph = 0, sph = 0, it = 0;
      bool ok = true, issued = false;
      for (int j = sp.begin; j < sp.end && ok; j += sp.step, ++it) {
        const Unit8 u = unit8_at(g, j);
        const int np = bars.planes[u.p], nk = g.proj[u.p].nk;
        const int ncols = np * NT;
        const uint32_t id0 = idesc_s8(kWR, min(ncols, 256));
        const uint32_t id1 = idesc_s8(kWR, max(ncols - 256, 16));
        if (it >= static_cast<uint32_t>(nslot) &&
            !mbar_wait(smem_addr(&bars.acc_empty[slot]), sph ^ 1u, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(slot * kSlotCols);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(smem_addr(&bars.full[s]), ph, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + static_cast<uint32_t>(s) * stage_bytes;
#pragma unroll
          for (int k = 0; k < kKC / kUK; ++k) {
            const uint64_t da = umma_desc(st + k * 32);
            const uint32_t acc = (kb != 0 || k != 0) ? 1u : 0u;
            umma_i8(d, da, umma_desc(st + kWBytes + k * 32), id0, acc);
            if (ncols > 256)   // the third plane of 128 tokens: columns 256 .. 383
              umma_i8(d + 256, da, umma_desc(st + kWBytes + 256 * kKC + k * 32), id1, acc);
          }
          issued = true;
          umma_commit(smem_addr(&bars.empty[s]));
          if (++s == nstage) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_addr(&bars.acc_full[slot]));
        if (++slot == nslot) {
          slot = 0;
          sph ^= 1u;
        }
      }
      if (!ok) {
        atomicOr(&bars.bad, 1);
        if (issued) {   // the MMAs in flight complete before tensor memory is freed
          umma_commit(smem_addr(&bars.drain));
          mbar_wait(smem_addr(&bars.drain), 0, nullptr);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3, h = (warp - kEpi0) >> 2;
    const int half = NT >> 1;
    int slot = 0;
    uint32_t sph = 0;
    bool ok = true;
    for (int j = sp.begin; j < sp.end; j += sp.step) {
      const Unit8 u = unit8_at(g, j);
      const G8Proj& P = g.proj[u.p];
      const int np = bars.planes[u.p];
      const int64_t M = P.M, N = P.N, ldy = P.ldy;
      const int flags = P.flags;
      float* const Y = P.y;
      const float* const S = P.S;
      const int* const shift = P.shift;
      const int64_t n = u.n0 + q * 32 + lane;
      const bool nok = n < N;
      float sw = 1.0f;
      if (!(flags & kMmUnit) && nok) sw = __ldg(reinterpret_cast<const float*>(P.srows + n * P.srs));
      if (!mbar_wait(smem_addr(&bars.acc_full[slot]), sph, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(slot * kSlotCols);
      const bool accum = (flags & kMmAcc) != 0;
      for (int tb = h * half; tb < (h + 1) * half && u.t0 + tb < M; tb += 8) {
        uint32_t r[3][8];
        tmem_planes8(taddr + tb, NT, np, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t m = u.t0 + tb + i;
          if (m >= M) break;
          long long a = static_cast<long long>(static_cast<int>(r[0][i]));
          if (np > 1) a += static_cast<long long>(static_cast<int>(r[1][i])) * 256;
          if (np > 2) a += static_cast<long long>(static_cast<int>(r[2][i])) * 65536;
          a *= static_cast<long long>(1) << __ldg(shift + m);
          if (nok) {
            float* dst = Y + m * ldy + n;
            float v = mm_epilogue(a, sw, __ldg(S + m), 16);
            if (accum) v = fadd(*dst, v);
            *dst = v;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&bars.acc_empty[slot]));
      if (++slot == nslot) {
        slot = 0;
        sph ^= 1u;
      }
    }
    if (!ok) atomicOr(&bars.bad, 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host: the schedule
// Units are (projection, row tile, token tile). When the projections' K differ (a layer's
// q/k/v/o/gate/up/down at prefill), each CTA gets a list from a longest-first (LPT) assignment
// of units costing their K chunks (+1 for the epilogue); units of equal cost keep the order
// row tile, token tile, so the token tiles of one row tile run at the same time on different
// SMs and its weights cross HBM once. Equal K (or more units than the table holds): round robin.
struct Plan8 {
  int key[3 + 3 * kW8A8MaxGroup];
  int table, nunits, grid;
  uint32_t units[kMaxUnits];
  uint16_t first[kMaxCtas + 1];
};

void make_plan8(Plan8& pl, const int* tiles, const int* tiles_t, const int* nk, int count, int sms) {
  int64_t total = 0;
  bool uniform = true;
  for (int p = 0; p < count; ++p) {
    total += tiles[p];
    uniform = uniform && nk[p] == nk[0];
  }
  pl.nunits = static_cast<int>(total);
  pl.grid = static_cast<int>(std::min<int64_t>(total, sms));
  if (uniform || total > kMaxUnits) {
    pl.table = 0;
    return;
  }
  struct U {
    int64_t cost;
    uint32_t code;
  };
  std::vector<U> u;
  u.reserve(total);
  for (int p = 0; p < count; ++p)
    for (int t = 0; t < tiles[p]; ++t)
      u.push_back({nk[p] + 1, static_cast<uint32_t>(p) |
                                  (static_cast<uint32_t>(t % tiles_t[p]) << 3) |
                                  (static_cast<uint32_t>(t / tiles_t[p]) << 11)});
  std::stable_sort(u.begin(), u.end(), [](const U& a, const U& b) { return a.cost > b.cost; });
  using Load = std::pair<int64_t, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < pl.grid; ++c) heap.push({0, c});
  std::vector<int> owner(u.size());
  for (size_t i = 0; i < u.size(); ++i) {
    Load l = heap.top();
    heap.pop();
    l.first += u[i].cost;
    owner[i] = l.second;
    heap.push(l);
  }
  std::vector<int> fill(pl.grid + 1, 0);
  for (int c : owner) ++fill[c + 1];
  for (int c = 0; c < pl.grid; ++c) fill[c + 1] += fill[c];
  for (int c = 0; c <= pl.grid; ++c) pl.first[c] = static_cast<uint16_t>(fill[c]);
  for (size_t i = 0; i < u.size(); ++i) pl.units[fill[owner[i]]++] = u[i].code;
  pl.table = 1;
}

// The last few plans (a model's layers repeat the same shapes). Called under launch_mu.
const Plan8* plan_for8(const int* tiles, const int* tiles_t, const int* nk, int count, int sms) {
  static Plan8 cache[4];
  static int used = 0, next = 0;
  int key[3 + 3 * kW8A8MaxGroup] = {count, sms, 0};
  for (int p = 0; p < count; ++p) {
    key[3 + 3 * p] = tiles[p];
    key[4 + 3 * p] = tiles_t[p];
    key[5 + 3 * p] = nk[p];
  }
  for (int i = 0; i < used; ++i)
    if (std::memcmp(cache[i].key, key, sizeof(key)) == 0) return &cache[i];
  Plan8& pl = cache[next];
  next = (next + 1) % 4;
  used = std::max(used, next == 0 ? 4 : next);
  std::memcpy(pl.key, key, sizeof(key));
  make_plan8(pl, tiles, tiles_t, nk, count, sms);
  return &pl;
}

}  // namespace

int64_t qact_planes_bytes(int64_t M, int64_t K) {
  const int64_t Mp = rows_padded(M);
  return 9 * Mp + 3 * Mp * K;
}

int qact_planes_launch(const float* x, int64_t ldx, int64_t M, int64_t K, int row_mode,
                       void* planes, cudaStream_t stream) {
  if (M == 0) return kOk;
  const int64_t Mp = rows_padded(M);
  const size_t smem = (static_cast<size_t>(K) * 4 + static_cast<size_t>(K / 32) * 4 +
                       4 * (kQWarps + 3) + 15) & ~static_cast<size_t>(15);
  if (Mp > 0x7FFFFFFF || K > 0x7FFFFFFF || smem > 227 * 1024) return kErrArg;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrCuda;
  static size_t configured[kMaxDevices] = {0};
  if (smem > 48 * 1024 && configured[dev] < smem) {
    if (cudaFuncSetAttribute(qact_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = smem;
  }
  const PlanesParams p{x, ldx, M, static_cast<int>(K), row_mode, planes};
  return launch_kernel(reinterpret_cast<const void*>(qact_planes_kernel), static_cast<int>(Mp),
                       kQThreads, smem, stream, false, p);
}

int w8a8_launch(const W8A8Proj* projs, int count, cudaStream_t stream) {
  if (count < 1 || count > kW8A8MaxGroup) return kErrArg;
  const EncodeFn enc = encoder();
  if (enc == nullptr) return kErrCuda;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrCuda;
  const int sms = std::min(sm_count(dev), kMaxCtas);
  if (sms <= 0) return kErrCuda;
  int64_t maxM = 1;
  for (int i = 0; i < count; ++i) maxM = std::max(maxM, projs[i].M);
  int nt = 16;   // tokens a tile: the power of two from 16 to 128 that covers M
  while (nt < 128 && nt < maxM) nt *= 2;

  static G8Args g;   // ~11 KB of kernel parameters, filled under launch_mu
  static std::mutex launch_mu;
  std::lock_guard<std::mutex> lock(launch_mu);
  int tiles[kW8A8MaxGroup], tiles_t[kW8A8MaxGroup], nk[kW8A8MaxGroup];
  for (int i = 0; i < count; ++i) {
    const W8A8Proj& w = projs[i];
    const int64_t tt = (w.M + nt - 1) / nt, tr = (w.N + kWR - 1) / kWR;
    if (tt > 256 || tt * tr > (int64_t{1} << 20) || 3 * rows_padded(w.M) > 0x7FFFFFFF)
      return kErrArg;
    tiles_t[i] = static_cast<int>(tt);
    tiles[i] = static_cast<int>(tt * tr);
    nk[i] = static_cast<int>((w.K + kKC - 1) / kKC);
  }
  const Plan8* pl = plan_for8(tiles, tiles_t, nk, count, sms);
  int tile0 = 0;
  for (int i = 0; i < count; ++i) {
    const W8A8Proj& w = projs[i];
    G8Proj& P = g.proj[i];
    const int64_t Mp = rows_padded(w.M);
    const PlanesView v = planes_view(const_cast<void*>(w.planes), w.M);
    if (!encode_2d(enc, &P.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.rows, w.K, w.N, w.rs,
                   CU_TENSOR_MAP_SWIZZLE_128B, kKC, kWR) ||
        !encode_2d(enc, &P.pmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, v.data, w.K, 3 * Mp, w.K,
                   CU_TENSOR_MAP_SWIZZLE_128B, kKC, nt))
      return kErrArg;
    P.srows = w.srows;
    P.y = w.y;
    P.S = v.S;
    P.shift = v.shift;
    P.count = v.count;
    P.srs = w.srs;
    P.ldy = w.ldy;
    P.M = w.M;
    P.N = w.N;
    P.Mp = Mp;
    P.nk = nk[i];
    P.tiles_t = tiles_t[i];
    P.tile0 = tile0;
    P.flags = w.flags;
    tile0 += tiles[i];
  }
  g.count = count;
  g.nt = nt;
  g.table = pl->table;
  g.nunits = pl->nunits;
  if (pl->table) {
    std::memcpy(g.units, pl->units, sizeof(uint32_t) * pl->nunits);
    std::memcpy(g.first, pl->first, sizeof(uint16_t) * (pl->grid + 1));
  }
  g.status = status_word();

  const size_t smem = kStageBudget + 1024;
  static bool configured[kMaxDevices] = {false};
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(w8a8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = true;
  }
  w8a8_kernel<<<pl->grid, kThreads, smem, stream>>>(g);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace otq
