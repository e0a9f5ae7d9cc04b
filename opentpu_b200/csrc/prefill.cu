// Prefill: the weight-only int8 linear layer as a tcgen05 tensor-core GEMM (BASELINE
// configuration 4: int8 per-row weights, bf16 activations, 512 tokens).
//
//   y[m, n] = Sw[n] * sum_k x[m, k] * q[n, k]      x bf16 [M, K]; q int8 [N, K], the int8-row
//                                                  bytes; Sw fp32, the first word of scale row n
// which is the reference's `quant.quantize(W, "int8", g=K).deq @ x` (opentpu/quant.py:218-224,
// opentpu/reference.py:14-17) with bf16 activations: every int8 is exact in bf16, every product
// of two bf16 is exact in fp32, and the sums are fp32 (tensor-core order), so results match a
// float64 evaluation to a relative tolerance, not bit for bit.
//
// A CTA tile is 256 tokens x 256 weight rows; the work units are tiles, or K slices of tiles,
// of up to kW8A16MaxGroup independent projections (a layer's q/k/v/o/gate/up/down at prefill),
// and a persistent CTA (one an SM) runs the units the host assigned it, longest first. A K
// slice adds its share into y (tensor reduce-add, or vector float atomics; y zeroed first, or
// the old y with ACC), so split tiles are summed in arrival order: still within the stated
// tolerance, but not bit-reproducible from run to run; unsplit tiles are. K goes in chunks of
// 64 through two shared-memory rings:
//   warp 0      TMA: x's 256 x 64 bf16 box (128-byte swizzle: the K-major layout tcgen05.mma
//               reads) and the weight tile's 256 x 64 int8 box into a load stage (lfull);
//   warps 12-19 dequant prologue: int8 -> bf16 (exact) into a B stage in the same swizzled
//               K-major layout, fence.proxy.async, then bconv;
//   warp 1      allocates all 512 tensor-memory columns; lane 0 issues tcgen05.mma kind::f16
//               (M 128, N 256, K 16) for the two 128-token halves and four K steps a chunk;
//               tcgen05.commit frees the stages (lempty, bempty) and, after the tile's last
//               chunk, hands the two fp32 accumulators (2 x 256 columns) to the epilogue;
//   warps 4-11  scale epilogue: tcgen05.ld of their 32 tensor-memory lanes (tokens), half the
//               columns each, times Sw, staged 32 x 8 at a time in shared memory and written by
//               tensor bulk stores (bulk reduce-adds for K slices and ACC); when y does not
//               suit the tensor engine (alignment), a transpose and coalesced fp32 stores. Then
//               the accumulators are free again.
// Every mbarrier wait is bounded (mm_common.cuh): a wait that runs out sets bit 0 of the
// library's status word, and the CTA stops, letting the copies and MMAs it issued finish
// (bounded) before it frees tensor memory.
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
#include "tcgen05.cuh"
#include "otq_internal.h"

namespace otq {
namespace {

constexpr int kEpiWarp0 = 4;             // first epilogue warp
constexpr int kEpiWarps = 8;             // two a tensor-memory lane quarter (32 (w % 4) ..)
constexpr int kConvWarp0 = kEpiWarp0 + kEpiWarps;   // first dequant warp
constexpr int kConvWarps = 8;            // dequant warps (two an SM sub-partition)
constexpr int kThreads = 32 * (kConvWarp0 + kConvWarps);
constexpr int kBM = 128;               // tokens of one MMA (its M)
constexpr int kMT = 2;                   // MMA token halves of a tile
constexpr int kTM = kBM * kMT;           // 256 tokens a tile
constexpr int kTN = 256;                 // weight rows a tile (the MMA's N)
constexpr int kBK = 64;                  // K of a chunk: 128 bytes of bf16, one swizzle row
constexpr int kUK = 16;                  // K of one MMA
constexpr int kNL = 3;                   // load stages (x + int8)
constexpr int kNB = 2;                   // bf16 weight stages
constexpr int kABytes = kTM * kBK * 2;   // 32 KB
constexpr int kIBytes = kTN * kBK;       // 16 KB
constexpr int kBBytes = kTN * kBK * 2;   // 32 KB
constexpr uint32_t kTmemCols = 512;

struct Smem {
  uint8_t a[kNL][kABytes];   // 1024-aligned (128-byte swizzle atoms)
  uint8_t b[kNB][kBBytes];
  uint8_t i8[kNL][kIBytes];
  // epilogue staging, 2 KB an epilogue warp: a 32 x 16 transpose block, or two 32 x 8 blocks
  // (32-byte swizzle) that tensor stores read
  float stage[kEpiWarps][32 * 16];
  float sw[kTN];
  uint64_t lfull[kNL], lempty[kNL], bconv[kNB], bempty[kNB], acc_full, acc_empty, drain;
  uint32_t tmem;
  int bad;
};

struct alignas(64) GProj {
  CUtensorMap amap;   // x [M, K] bf16: box 64 x 256, 128-byte swizzle
  CUtensorMap bmap;   // rows [N, K] int8: box 64 x 256
  const uint8_t* srows;
  float* y;
  int64_t srs, ldy, M, N;
  int tiles_m, tile0;   // token tiles; first unit of this projection (round-robin mode)
  int nk, cps, splits;  // K chunks; chunks a K slice; K slices a tile (> 1: partial sums added)
  int flags;
  int vec;     // y 16-byte aligned and ldy a multiple of 4: float4 stores
  int tma_y;   // ymap describes y: the epilogue writes (or adds) through the tensor engine
  CUtensorMap ymap;   // y [M, N] fp32: box 8 columns x 32 rows, 32-byte swizzle
};

// Work units: a tile of one projection and one K slice of it. With a table, CTA b runs units
// units[first[b] .. first[b + 1]) (the host's longest-first assignment); without one, CTA b runs
// units b, b + grid, ... of the projections' tiles in order, whole K.
constexpr int kMaxUnits = 1536;
constexpr int kMaxCtas = 256;

struct GroupArgs {
  GProj proj[kW8A16MaxGroup];
  uint32_t units[kMaxUnits];    // projection (3 bits) | K slice (8 bits) << 3 | tile << 11
  uint16_t first[kMaxCtas + 1];
  int count, nunits, table;
  int* status;
};

struct Unit {
  int p, m0, n0, kb0, kb1;
  bool split;
};

// A value the compiler must keep in a register: a field read from the parameter block through a
// runtime index is a load through a generic address into parameter space, which the compiler
// would otherwise repeat at every use (it treats parameters as free to reload), each one slow.
__device__ __forceinline__ int opaque(int v) {
  asm volatile("" : "+r"(v));
  return v;
}
__device__ __forceinline__ int64_t opaque(int64_t v) {
  asm volatile("" : "+l"(v));
  return v;
}
template <class T>
__device__ __forceinline__ T* opaque(T* p) {
  uint64_t v = reinterpret_cast<uint64_t>(p);
  asm volatile("" : "+l"(v));
  return reinterpret_cast<T*>(v);
}

__device__ __forceinline__ Unit unit_at(const GroupArgs& g, int j) {
  uint32_t e;
  if (g.table) {
    e = g.units[j];
  } else {
    int p = 0;
    while (p + 1 < g.count && j >= g.proj[p + 1].tile0) ++p;
    e = static_cast<uint32_t>(p) | (static_cast<uint32_t>(j - g.proj[p].tile0) << 11);
  }
  Unit w;
  w.p = static_cast<int>(e & 7u);
  const int sl = static_cast<int>((e >> 3) & 0xFFu), t = static_cast<int>(e >> 11);
  const GProj& P = g.proj[w.p];
  const int tm = opaque(P.tiles_m), cps = opaque(P.cps), nk = opaque(P.nk);
  w.m0 = (t % tm) * kTM;
  w.n0 = (t / tm) * kTN;
  w.kb0 = sl * cps;
  w.kb1 = min(nk, w.kb0 + cps);
  w.split = opaque(P.splits) > 1;
  return w;
}

// This CTA's units: [begin, end) with stride `step`.
struct Span {
  int begin, end, step;
};
__device__ __forceinline__ Span my_units(const GroupArgs& g) {
  if (g.table) return Span{g.first[blockIdx.x], g.first[blockIdx.x + 1], 1};
  return Span{static_cast<int>(blockIdx.x), g.nunits, static_cast<int>(gridDim.x)};
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A and B (bits 7-9,
// 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 consecutive fp32 columns of this warp's 32 tensor-memory lanes (one lane a thread); the
// wait is in the same statement so that no use of r can move above it.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// 8 consecutive fp32 columns of this warp's 32 tensor-memory lanes (the wait included).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
}

// A 32-row x 8-column fp32 block from shared memory into y at (column x, row y): a store, or an
// element-wise add (K slices, ACC). Out-of-range rows and columns are clipped by the engine.
__device__ __forceinline__ void tma_store_y(const CUtensorMap* map, uint32_t src, int x, int y, bool add) {
  if (add)
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::
                     "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src)
                 : "memory");
  else
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::
                     "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src)
                 : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// At most N of this thread's bulk stores still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void epi_sync() {   // the epilogue warps
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
}

// Byte sel & 3 of x (x = int8 bytes ^ 0x80, i.e. v + 128) as the fp32 v: the word 0x4B0000uu is
// 2^23 + u exactly, and subtracting 2^23 + 128 is exact.
__device__ __forceinline__ uint32_t i8_f32(uint32_t x, uint32_t sel) {
  return __float_as_uint(__fsub_rn(__uint_as_float(prmt(x, 0x4B000000u, sel)), 8388736.0f));
}
// Eight int8 -> eight bf16 (element 0 in the low half of .x). |v| <= 128 has at most 8
// significant bits, so the upper half of its fp32 is its exact bf16.
__device__ __forceinline__ uint4 i8x8_bf16(uint2 w) {
  const uint32_t x0 = w.x ^ 0x80808080u, x1 = w.y ^ 0x80808080u;
  uint4 o;
  o.x = prmt(i8_f32(x0, 0x7650u), i8_f32(x0, 0x7651u), 0x7632u);
  o.y = prmt(i8_f32(x0, 0x7652u), i8_f32(x0, 0x7653u), 0x7632u);
  o.z = prmt(i8_f32(x1, 0x7650u), i8_f32(x1, 0x7651u), 0x7632u);
  o.w = prmt(i8_f32(x1, 0x7652u), i8_f32(x1, 0x7653u), 0x7632u);
  return o;
}

__global__ void __launch_bounds__(kThreads, 1) w8a16_kernel(const __grid_constant__ GroupArgs g) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = g.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNL; ++i) {
      mbar_init(smem_addr(&s.lfull[i]), 1);
      mbar_init(smem_addr(&s.lempty[i]), 1);
    }
    for (int i = 0; i < kNB; ++i) {
      mbar_init(smem_addr(&s.bconv[i]), kConvWarps);   // one arrival a dequant warp
      mbar_init(smem_addr(&s.bempty[i]), 1);
    }
    mbar_init(smem_addr(&s.acc_full), 1);
    mbar_init(smem_addr(&s.acc_empty), kEpiWarps);   // one arrival an epilogue warp
    mbar_init(smem_addr(&s.drain), 1);
    s.bad = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane < g.count) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.proj[lane].amap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.proj[lane].bmap)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&s.tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t c = 0;   // chunks issued (all tiles)
      bool ok = true;
      const Span sp = my_units(g);
      for (int j = sp.begin; j < sp.end && ok; j += sp.step) {
        const Unit t = unit_at(g, j);
        const CUtensorMap* am = &g.proj[t.p].amap;
        const CUtensorMap* bm = &g.proj[t.p].bmap;
        for (int kb = t.kb0; kb < t.kb1; ++kb, ++c) {
          const uint32_t ls = c % kNL;
          if (c >= kNL && !mbar_wait(smem_addr(&s.lempty[ls]), ((c / kNL) - 1) & 1, status)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_addr(&s.lfull[ls]);
          mbar_arrive_expect_tx(full, kABytes + kIBytes);
          tma_2d(smem_addr(s.a[ls]), am, kb * kBK, t.m0, full);
          tma_2d(smem_addr(s.i8[ls]), bm, kb * kBK, t.n0, full);
        }
      }
      if (!ok) {
        atomicOr(&s.bad, 1);
        // the copies still in flight land before the shared memory is given up
        for (uint32_t j = c > kNL ? c - kNL : 0; j < c; ++j)
          mbar_wait(smem_addr(&s.lfull[j % kNL]), (j / kNL) & 1, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, kTN);
      uint32_t c = 0, it = 0;
      bool ok = true, issued = false;
      const Span sp = my_units(g);
      for (int j = sp.begin; j < sp.end && ok; j += sp.step, ++it) {
        const Unit t = unit_at(g, j);
        if (it > 0 && !mbar_wait(smem_addr(&s.acc_empty), (it - 1) & 1, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = t.kb0; kb < t.kb1; ++kb, ++c) {
          const uint32_t ls = c % kNL, bs = c % kNB;
          if (!mbar_wait(smem_addr(&s.bconv[bs]), (c / kNB) & 1, status) ||
              !mbar_wait(smem_addr(&s.lfull[ls]), (c / kNL) & 1, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_addr(s.a[ls]), b0 = smem_addr(s.b[bs]);
#pragma unroll
          for (int h = 0; h < kMT; ++h) {
#pragma unroll
            for (int k = 0; k < kBK / kUK; ++k) {
              umma(tmem + h * kTN, umma_desc(a0 + h * kBM * 128 + k * 32), umma_desc(b0 + k * 32),
                   idesc, (kb != t.kb0 || k != 0) ? 1u : 0u);
            }
          }
          issued = true;
          umma_commit(smem_addr(&s.lempty[ls]));
          umma_commit(smem_addr(&s.bempty[bs]));
        }
        if (!ok) break;
        umma_commit(smem_addr(&s.acc_full));
      }
      if (!ok) {
        atomicOr(&s.bad, 1);
        if (issued) {   // the MMAs in flight complete before tensor memory is freed
          umma_commit(smem_addr(&s.drain));
          mbar_wait(smem_addr(&s.drain), 0, nullptr);
        }
      }
    }
    __syncwarp();
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ dequant prologue
    const int ct = threadIdx.x - kConvWarp0 * 32;   // 0 .. 32 kConvWarps - 1
    uint32_t c = 0;
    bool ok = true;
    const Span sp = my_units(g);
    for (int j = sp.begin; j < sp.end && ok; j += sp.step) {
      const Unit t = unit_at(g, j);
      for (int kb = t.kb0; kb < t.kb1; ++kb, ++c) {
        const uint32_t ls = c % kNL, bs = c % kNB;
        if (!mbar_wait(smem_addr(&s.lfull[ls]), (c / kNL) & 1, status) ||
            (c >= kNB && !mbar_wait(smem_addr(&s.bempty[bs]), ((c / kNB) - 1) & 1, status))) {
          ok = false;
          break;
        }
        const uint8_t* src = s.i8[ls];
        uint8_t* dst = s.b[bs];
        // 256 rows x four 16-byte pieces; a warp takes 8 whole rows at a time: 16-byte loads
        // of 512 contiguous bytes, and the two 16-byte stores of a piece land in bf16 slots
        // 2pc, 2pc + 1 (XOR row % 8) of the row, conflict-free across the 8 rows
        constexpr int kPer = kTN * 4 / (32 * kConvWarps);
        uint4 w[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int p = ct + 32 * kConvWarps * i;
          w[i] = *reinterpret_cast<const uint4*>(src + p * 16);
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int p = ct + 32 * kConvWarps * i, row = p >> 2, pc = p & 3;
          uint8_t* d = dst + row * 128;
          *reinterpret_cast<uint4*>(d + 16 * ((2 * pc) ^ (row & 7))) = i8x8_bf16(make_uint2(w[i].x, w[i].y));
          *reinterpret_cast<uint4*>(d + 16 * ((2 * pc + 1) ^ (row & 7))) = i8x8_bf16(make_uint2(w[i].z, w[i].w));
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // seen by the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&s.bconv[bs]));
      }
    }
    if (!ok) atomicOr(&s.bad, 1);
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------------ scale epilogue
    // warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (tokens) and columns
    // [128 hc, 128 hc + 128) of each token half's accumulator, 16 columns at a time
    const int q = warp & 3, hc = (warp - kEpiWarp0) >> 2;
    const int et = threadIdx.x - kEpiWarp0 * 32;
    const int c4 = lane & 3, rl = lane >> 2;   // store phase: rows 8i + rl, columns 4 c4 ..
    float* const st = s.stage[warp - kEpiWarp0];
    uint32_t it = 0;
    bool ok = true;
    const Span sp = my_units(g);
    for (int j = sp.begin; j < sp.end && ok; j += sp.step, ++it) {
      const Unit t = unit_at(g, j);
      // the projection's fields, once, in registers (opaque)
      float* const Y = opaque(g.proj[t.p].y);
      const int64_t ldy = opaque(g.proj[t.p].ldy), Mr = opaque(g.proj[t.p].M),
                    Nc = opaque(g.proj[t.p].N);
      const int flags = opaque(g.proj[t.p].flags);
      const bool vec = opaque(g.proj[t.p].vec) != 0;
      const uint8_t* const srows = opaque(g.proj[t.p].srows);
      const int64_t srs = opaque(g.proj[t.p].srs);
      epi_sync();   // the previous tile's scales are no longer read
      {
        const int64_t n = t.n0 + et;
        float v = 0.0f;
        if (n < Nc) v = (flags & OTQ_MM_UNIT) ? 1.0f : __ldg(reinterpret_cast<const float*>(srows + n * srs));
        s.sw[et] = v;
      }
      epi_sync();
      if (!mbar_wait(smem_addr(&s.acc_full), it & 1, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool acc = (flags & OTQ_MM_ACC) != 0;
      if (opaque(g.proj[t.p].tma_y)) {
        // through the tensor engine: 32 x 8 blocks scaled in registers, staged (two buffers a
        // warp, 32-byte swizzle), then one bulk store (or add: K slices, ACC) by lane 0
        const CUtensorMap* ymap = &g.proj[t.p].ymap;
        const bool add = t.split || acc;
        const uint32_t buf0 = smem_addr(st);
#pragma unroll 1
        for (int h = 0; h < kMT; ++h) {
          const int row0 = t.m0 + h * kBM + q * 32;
#pragma unroll 1
          for (int cb = 0; cb < 128; cb += 8) {
            uint32_t r[8];
            tmem_ld8(tmem + (static_cast<uint32_t>(q * 32) << 16) + h * kTN + hc * 128 + cb, r);
            const float4 s0 = *reinterpret_cast<const float4*>(&s.sw[hc * 128 + cb]);
            const float4 s1 = *reinterpret_cast<const float4*>(&s.sw[hc * 128 + cb + 4]);
            const int blk = (h * 16 + cb / 8) & 1;
            if (lane == 0) bulk_wait_read<1>();   // the store from this buffer two blocks ago
            __syncwarp();
            float* b = st + blk * 256 + lane * 8;
            const int sx = (lane >> 2) & 1;   // 32-byte swizzle: chunk c of row r at c ^ (r / 4 % 2)
            *reinterpret_cast<float4*>(b + 4 * sx) =
                make_float4(__uint_as_float(r[0]) * s0.x, __uint_as_float(r[1]) * s0.y,
                            __uint_as_float(r[2]) * s0.z, __uint_as_float(r[3]) * s0.w);
            *reinterpret_cast<float4*>(b + 4 * (sx ^ 1)) =
                make_float4(__uint_as_float(r[4]) * s1.x, __uint_as_float(r[5]) * s1.y,
                            __uint_as_float(r[6]) * s1.z, __uint_as_float(r[7]) * s1.w);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // seen by the engine
            __syncwarp();
            if (lane == 0) tma_store_y(ymap, buf0 + blk * 1024, t.n0 + hc * 128 + cb, row0, add);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&s.acc_empty));
        continue;
      }
      if (lane == 0) bulk_wait_read<0>();   // no tensor store still reads the staging block
      __syncwarp();
      for (int h = 0; h < kMT; ++h) {
        const int64_t row0 = t.m0 + h * kBM + q * 32;   // this warp's 32 tokens
        const int64_t col0 = t.n0 + hc * 128;
        // the plain case: every row and column of this warp's block in range, no K slice,
        // no ACC, float4 stores; one pointer a lane, advanced by 8 rows a store
        const bool fast = !t.split && !acc && vec && row0 + 32 <= Mr && col0 + 128 <= Nc;
        float* const base = Y + (row0 + rl) * ldy + col0 + 4 * c4;
#pragma unroll 1
        for (int cb = 0; cb < 128; cb += 16) {
          uint32_t r[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + h * kTN + hc * 128 + cb, r);
          // transpose through shared memory: 64-byte rows, 16-byte chunk c of row r at
          // c ^ ((r / 2) % 4) (conflict-free both ways)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(st + lane * 16 + 4 * (c ^ ((lane >> 1) & 3))) =
                make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
          __syncwarp();
          const float4 sc = *reinterpret_cast<const float4*>(&s.sw[hc * 128 + cb + 4 * c4]);
          float4 v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 8 * i + rl;
            v[i] = *reinterpret_cast<const float4*>(st + rr * 16 + 4 * (c4 ^ ((rr >> 1) & 3)));
            v[i].x *= sc.x;
            v[i].y *= sc.y;
            v[i].z *= sc.z;
            v[i].w *= sc.w;
          }
          __syncwarp();
          if (fast) {
#pragma unroll
            for (int i = 0; i < 4; ++i) *reinterpret_cast<float4*>(base + 8 * i * ldy + cb) = v[i];
            continue;
          }
          const int64_t n = col0 + cb + 4 * c4;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int64_t m = row0 + 8 * i + rl;
            if (m >= Mr) continue;
            float* dst = Y + m * ldy + n;
            if (t.split) {   // a K slice: its share added into y (zeroed, or the old y with ACC)
              if (vec && n + 3 < Nc) {
                atomicAdd(reinterpret_cast<float4*>(dst), v[i]);
              } else {
                const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
                for (int k = 0; k < 4 && n + k < Nc; ++k) atomicAdd(dst + k, e[k]);
              }
            } else if (vec && n + 3 < Nc) {
              float4 w = v[i];
              if (acc) {
                const float4 o = *reinterpret_cast<const float4*>(dst);
                w.x += o.x;
                w.y += o.y;
                w.z += o.z;
                w.w += o.w;
              }
              *reinterpret_cast<float4*>(dst) = w;
            } else {
              const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
              for (int k = 0; k < 4 && n + k < Nc; ++k) dst[k] = acc ? dst[k] + e[k] : e[k];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&s.acc_empty));
    }
    if (lane == 0) bulk_wait_all();   // this warp's tensor stores complete before the CTA exits
    if (!ok) atomicOr(&s.bad, 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace

namespace {

// The host's schedule. A unit's cost is its K chunks plus its epilogue (reading the 512
// tensor-memory columns and writing 256 KB of fp32), measured on B200 at about 7 us against
// 0.74 us a chunk: kEpiChunks chunk times. K slices are at least kMinSlice chunks; the slice
// length is searched over the longest projection's nk / S, S = 1 .. kMaxSlices, for the
// smallest longest-first (LPT) makespan over the SMs.
constexpr int kEpiChunks = 10;
constexpr int kMinSlice = 4;
constexpr int kMaxSlices = 16;

struct Plan {
  int key[2 + 2 * kW8A16MaxGroup];   // count, sms, then (tiles, nk) a projection
  int splits[kW8A16MaxGroup], cps[kW8A16MaxGroup];
  int table, nunits, grid;
  uint32_t units[kMaxUnits];
  uint16_t first[kMaxCtas + 1];
};

struct UnitCost {
  int64_t cost;
  uint32_t code;
};

// LPT over `ctas` CTAs of units sorted by decreasing cost: each goes to the least-loaded CTA
// (ties to the lower index). Returns the makespan; with `owner`, each unit's CTA.
int64_t lpt(const std::vector<UnitCost>& u, int ctas, std::vector<int>* owner) {
  using Load = std::pair<int64_t, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < ctas; ++c) heap.push({0, c});
  int64_t span = 0;
  if (owner) owner->resize(u.size());
  for (size_t i = 0; i < u.size(); ++i) {
    Load l = heap.top();
    heap.pop();
    l.first += u[i].cost;
    span = std::max(span, l.first);
    if (owner) (*owner)[i] = l.second;
    heap.push(l);
  }
  return span;
}

void units_for(const int* tiles, const int* nk, const int* splits, const int* cps, int count,
               std::vector<UnitCost>* out) {
  out->clear();
  for (int p = 0; p < count; ++p)
    for (int t = 0; t < tiles[p]; ++t)
      for (int sl = 0; sl < splits[p]; ++sl) {
        const int len = std::min(nk[p], (sl + 1) * cps[p]) - sl * cps[p];
        out->push_back({len + kEpiChunks, static_cast<uint32_t>(p) |
                                              (static_cast<uint32_t>(sl) << 3) |
                                              (static_cast<uint32_t>(t) << 11)});
      }
  std::stable_sort(out->begin(), out->end(),
                   [](const UnitCost& a, const UnitCost& b) { return a.cost > b.cost; });
}

void make_plan(Plan& pl, const int* tiles, const int* nk, int count, int sms) {
  int nkmax = 1;
  int64_t total = 0;
  for (int p = 0; p < count; ++p) {
    nkmax = std::max(nkmax, nk[p]);
    total += tiles[p];
  }
  std::vector<UnitCost> u;
  int64_t best = INT64_MAX;
  int best_units = 0;
  for (int S = 1; S <= kMaxSlices; ++S) {
    const int T = (nkmax + S - 1) / S;
    if (S > 1 && T < kMinSlice) break;
    int sp[kW8A16MaxGroup], cp[kW8A16MaxGroup];
    int64_t n = 0;
    for (int p = 0; p < count; ++p) {
      int k = (nk[p] + T - 1) / T;
      k = std::max(1, std::min(k, nk[p] / kMinSlice));
      cp[p] = (nk[p] + k - 1) / k;
      sp[p] = (nk[p] + cp[p] - 1) / cp[p];
      n += static_cast<int64_t>(tiles[p]) * sp[p];
    }
    if (n > kMaxUnits) continue;
    units_for(tiles, nk, sp, cp, count, &u);
    const int64_t span = lpt(u, static_cast<int>(std::min<int64_t>(n, sms)), nullptr);
    if (span < best || (span == best && n < best_units)) {
      best = span;
      best_units = static_cast<int>(n);
      for (int p = 0; p < count; ++p) {
        pl.splits[p] = sp[p];
        pl.cps[p] = cp[p];
      }
    }
  }
  if (best == INT64_MAX) {   // more tiles than the table holds: round robin, whole K
    pl.table = 0;
    pl.nunits = static_cast<int>(total);
    pl.grid = static_cast<int>(std::min<int64_t>(total, sms));
    for (int p = 0; p < count; ++p) {
      pl.splits[p] = 1;
      pl.cps[p] = nk[p];
    }
    return;
  }
  units_for(tiles, nk, pl.splits, pl.cps, count, &u);
  pl.table = 1;
  pl.nunits = static_cast<int>(u.size());
  pl.grid = std::min(pl.nunits, sms);
  std::vector<int> owner;
  lpt(u, pl.grid, &owner);
  std::vector<int> fill(pl.grid + 1, 0);
  for (int c : owner) ++fill[c + 1];
  for (int c = 0; c < pl.grid; ++c) fill[c + 1] += fill[c];
  for (int c = 0; c <= pl.grid; ++c) pl.first[c] = static_cast<uint16_t>(fill[c]);
  for (size_t i = 0; i < u.size(); ++i) pl.units[fill[owner[i]]++] = u[i].code;
}

// The last few plans (a model's layers repeat the same shapes).
const Plan* plan_for(const int* tiles, const int* nk, int count, int sms) {
  static std::mutex mu;
  static Plan cache[4];
  static int used = 0, next = 0;
  int key[2 + 2 * kW8A16MaxGroup] = {count, sms};
  for (int p = 0; p < count; ++p) {
    key[2 + 2 * p] = tiles[p];
    key[3 + 2 * p] = nk[p];
  }
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (std::memcmp(cache[i].key, key, sizeof(key)) == 0) return &cache[i];
  Plan& pl = cache[next];
  next = (next + 1) % 4;
  used = std::max(used, next == 0 ? 4 : next);
  std::memcpy(pl.key, key, sizeof(key));
  make_plan(pl, tiles, nk, count, sms);
  return &pl;
}

}  // namespace

int w8a16_launch(const W8A16Proj* projs, int count, cudaStream_t stream) {
  if (count < 1 || count > kW8A16MaxGroup) return kErrArg;
  const EncodeFn enc = encoder();
  if (enc == nullptr) return kErrCuda;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrCuda;
  const int sms = std::min(sm_count(dev), kMaxCtas);
  if (sms <= 0) return kErrCuda;

  static GroupArgs g;   // ~9 KB of kernel parameters, filled under launch_mu
  static std::mutex launch_mu;
  std::lock_guard<std::mutex> lock(launch_mu);
  int tiles[kW8A16MaxGroup], nk[kW8A16MaxGroup];
  for (int i = 0; i < count; ++i) {
    const W8A16Proj& w = projs[i];
    const int64_t t = ((w.M + kTM - 1) / kTM) * ((w.N + kTN - 1) / kTN);
    if (t > (int64_t{1} << 20)) return kErrArg;
    tiles[i] = static_cast<int>(t);
    nk[i] = static_cast<int>((w.K + kBK - 1) / kBK);
  }
  const Plan* pl = plan_for(tiles, nk, count, sms);
  int tile0 = 0;
  for (int i = 0; i < count; ++i) {
    const W8A16Proj& w = projs[i];
    GProj& P = g.proj[i];
    if (!encode_2d(enc, &P.amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w.x, w.K, w.M, w.ldx * 2,
                   CU_TENSOR_MAP_SWIZZLE_128B, kBK, 256) ||
        !encode_2d(enc, &P.bmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.rows, w.K, w.N, w.rs,
                   CU_TENSOR_MAP_SWIZZLE_NONE, kBK, 256))
      return kErrArg;
    P.srows = w.srows;
    P.y = w.y;
    P.srs = w.srs;
    P.ldy = w.ldy;
    P.M = w.M;
    P.N = w.N;
    P.tiles_m = static_cast<int>((w.M + kTM - 1) / kTM);
    P.tile0 = tile0;
    tile0 += tiles[i];
    P.nk = nk[i];
    P.cps = pl->cps[i];
    P.splits = pl->splits[i];
    P.flags = w.flags;
    P.vec = (reinterpret_cast<uintptr_t>(w.y) % 16 == 0 && w.ldy % 4 == 0) ? 1 : 0;
    P.tma_y = P.vec && encode_2d(enc, &P.ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.y, w.N, w.M,
                                 w.ldy * 4, CU_TENSOR_MAP_SWIZZLE_32B, 8, 32)
                  ? 1
                  : 0;
    // K slices add into y: start from zero unless ACC asks to add to the old values
    if (P.splits > 1 && !(w.flags & OTQ_MM_ACC) &&
        cudaMemset2DAsync(w.y, static_cast<size_t>(w.ldy) * 4, 0, static_cast<size_t>(w.N) * 4,
                          static_cast<size_t>(w.M), stream) != cudaSuccess)
      return kErrCuda;
  }
  g.count = count;
  g.table = pl->table;
  g.nunits = pl->nunits;
  if (pl->table) {
    std::memcpy(g.units, pl->units, sizeof(uint32_t) * pl->nunits);
    std::memcpy(g.first, pl->first, sizeof(uint16_t) * (pl->grid + 1));
  }
  g.status = status_word();

  const size_t smem = sizeof(Smem) + 1024;
  static bool configured[kMaxDevices] = {false};
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(w8a16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = true;
  }
  w8a16_kernel<<<pl->grid, kThreads, smem, stream>>>(g);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace otq
