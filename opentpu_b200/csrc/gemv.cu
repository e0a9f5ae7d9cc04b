// MM for decode (up to 8 activation rows a pass): the weight-streaming GEMV over openTPU's MX
// formats, with exact integer accumulation (reference docs/isa.md "MM";
// opentpu/isasim.py:749-910; scalar model tests/test_mx.py:131-151).
//
//   acc = sum over 32-element groups of (m << sh) * c,  c = the group's exact int dot product,
//         sh = W - dw - da (the group is dropped where sh < 0)
//   y   = (i2f(acc) * Sw[n]) * (Sa[j] * 2^-W)      -- otq_fp32.cuh mm_epilogue
//
// Streaming. Each warp owns a contiguous range of weight rows (ranges balanced by rows) and walks
// it in blocks of R rows, 128-byte chunks of K at a time. The chunks go through a ring of NS
// shared-memory stages with cp.async (16 bytes a lane, 512 contiguous bytes a warp instruction,
// nothing held in registers while in flight; cp.async.wait_group is a hardware wait), so each warp
// keeps NS - 1 chunks of R rows in flight. Stage rows are padded to 160 bytes, which makes the
// fragment reads below conflict free. The first stages are issued before griddepcontrol.wait:
// weights never depend on the kernel launched before this one.
//
// Dot products: one mma.sync m16n8k32 (s8 x s8 -> s32) takes one 32-element group of 8 weight
// rows (B, one row a column: lane (g, t) supplies row g's bytes [8t, 8t+8) of the group) against
// 16 rows of A. 4-bit elements are decoded in registers to exact bytes (int4 as 16x its value, so
// no bias term is needed; E2M1 doubled).
//
// Class path (RSC / UNIT rows, one activation row, every group's offset representable): a
// group's multiplier 2^(W - da) depends on the activation alone, so A row c carries the bytes of
// the groups whose offset da is c (zeros elsewhere) and the MMA accumulates every group of a row
// exactly in int32 (|sum| < 2^31 for K <= 32640). At the end of a row block each class is scaled
// once by 2^(W - c) into int64 and the 8 class rows are summed across lanes. Groups below the
// window (sh < 0) are in no class: they are dropped.
//
// General path (MX rows with per-block weight offsets, several activation rows, or an int8 row
// whose offset 16 has no class row): A row j is activation row j; each group's int32 result is
// scaled by its own multiplier (m << sh) into int64 accumulators, one per (activation row,
// weight row) and lane, so no cross-lane reduction is needed.
//
// Rows with few outputs split K: S warps of a CTA take the same rows, each a range of chunks,
// and add their int64 partials through shared memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "mm_common.cuh"
#include "otq_fp32.cuh"
#include "otq_internal.h"
#include "qact.cuh"

namespace otq {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 128;           // bytes of a weight row in one stage
constexpr int kPitch = kChunk + 32;   // a stage row: conflict-free 8-row fragment reads

template <int FMT>
struct GF {
  static constexpr int kW = (FMT == kFmtInt8) ? 16 : (FMT == kFmtNvfp4 ? 13 : 11);
  static constexpr int kElems = (FMT == kFmtInt8) ? 128 : 256;   // elements of a chunk
  static constexpr int kGroups = kElems / 32;
  static constexpr int kGroupBytes = (FMT == kFmtInt8) ? 32 : 16;
  static constexpr int kBlocks = kElems / 128;
};

// A stage: R rows x kPitch, then (MX rows) 16 bytes of scale data a row.
template <int R, bool PLAIN>
struct Stage {
  static constexpr int kScaleOff = R * kPitch;
  static constexpr int kBytes = kScaleOff + (PLAIN ? 0 : R * 16);
};

struct GSmem {
  uint8_t* act;      // [MT][KP] activation bytes (int4: each run of 8 as evens, then odds)
  int* term;         // [MT][KG] general path: a group's activation-side term (group_term)
  uint8_t* cls;      // [KG] class path: the group's class (its offset), 255 = dropped
  float* Sa;         // [MT]
  int* flag;         // [1] 1: some group of activation row 0 has no class
  long long* red;    // [kWarps][32][VPL] K-split partials
  float* xs;         // [K] the fp32 row being quantized (fused QACT)
  uint32_t* seg;     // [K / 32]
  uint32_t* qred;    // [40]
  uint8_t* ring;     // [kWarps][NS][stage]
};

__host__ __device__ inline size_t gemv_layout(int MT, int K, int kp, bool fused, int vpl, int S,
                                              int stage_bytes, int ns, size_t* offs) {
  const size_t KG = K / 32;
  size_t off = 0;
  auto take = [&](int i, size_t bytes) {
    off = (off + 15) & ~size_t(15);
    if (offs) offs[i] = off;
    off += bytes;
  };
  take(0, static_cast<size_t>(MT) * kp);
  take(1, static_cast<size_t>(MT) * KG * 4);
  take(2, KG);
  take(3, MT * 4);
  take(4, 16);
  take(5, S > 1 ? static_cast<size_t>(kWarps) * 32 * vpl * 8 : 0);
  take(6, fused ? static_cast<size_t>(K) * 4 : 0);
  take(7, KG * 4);
  take(8, 40 * 4);
  take(9, static_cast<size_t>(kWarps) * ns * stage_bytes);
  return off;
}

__device__ __forceinline__ GSmem gemv_carve(unsigned char* base, int MT, int K, int kp, bool fused,
                                            int vpl, int S, int stage_bytes, int ns) {
  size_t o[10];
  gemv_layout(MT, K, kp, fused, vpl, S, stage_bytes, ns, o);
  GSmem s;
  s.act = base + o[0];
  s.term = reinterpret_cast<int*>(base + o[1]);
  s.cls = base + o[2];
  s.Sa = reinterpret_cast<float*>(base + o[3]);
  s.flag = reinterpret_cast<int*>(base + o[4]);
  s.red = reinterpret_cast<long long*>(base + o[5]);
  s.xs = reinterpret_cast<float*>(base + o[6]);
  s.seg = reinterpret_cast<uint32_t*>(base + o[7]);
  s.qred = reinterpret_cast<uint32_t*>(base + o[8]);
  s.ring = base + o[9];
  return s;
}

// Element i of an activation row -> its byte (int4: the order in which a word's low and high
// nibbles come out of the decoder).
template <int FMT>
__device__ __forceinline__ int act_pos(int i) {
  if constexpr (FMT == kFmtInt4) {
    const int r = i & 7;
    return (i & ~7) | ((r & 1) ? 4 + (r >> 1) : (r >> 1));
  }
  return i;
}

// General path term of a group: 2^(W - da) (0 below the window) where the multiplier is that
// power of two, or a shift of it (int8 MX: >> dw); W - da for 4-bit MX rows (shifted()).
template <int FMT, bool PLAIN>
__device__ __forceinline__ int group_term(int da) {
  const int sh = GF<FMT>::kW - da;
  if constexpr (FMT == kFmtInt8 || PLAIN) {
    return sh >= 0 ? (1 << sh) : 0;
  } else {
    return sh;
  }
}

template <int FMT, int MT, bool PLAIN>
__device__ __forceinline__ void put_group(const GSmem& s, int KG, int j, int G, int da) {
  s.term[j * KG + G] = group_term<FMT, PLAIN>(da);
  if (j == 0) {
    const int W = GF<FMT>::kW;
    int c = da <= W ? da : 255;   // above W: below the window, dropped
    if (c == 16) {                // int8 offset 16 (multiplier 1): no class row for it
      c = 255;
      *s.flag = 1;
    }
    s.cls[G] = static_cast<uint8_t>(c);
  }
}

// Activation rows [m0, m0 + mt) into shared memory (QACT of fp32 x, or copied bytes). Bytes past
// K, and rows mt..MT-1, are zeros.
template <int FMT, int MT, bool PLAIN>
__device__ void gemv_load_activations(const MMParams& p, const GSmem& s, int m0, int mt, int kp) {
  const int K = p.K, KG = K / 32;
  if (threadIdx.x == 0) *s.flag = 0;
  for (int j = 0; j < MT; ++j) {
    const int from = j < mt ? K : 0;
    uint32_t* aw = reinterpret_cast<uint32_t*>(s.act + static_cast<size_t>(j) * kp);
    for (int i = (from >> 2) + threadIdx.x; i < (kp >> 2); i += kThreads) aw[i] = 0u;
    if (j >= mt)
      for (int G = threadIdx.x; G < KG; G += kThreads) s.term[j * KG + G] = 0;
  }
  if (threadIdx.x < MT && static_cast<int>(threadIdx.x) >= mt) s.Sa[threadIdx.x] = 0.0f;
  __syncthreads();   // flag cleared before any group can set it
  if (p.x != nullptr) {
    const ThreadGroup<kThreads> grp{static_cast<int>(threadIdx.x)};
    for (int j = 0; j < mt; ++j) {
      stage_row(grp, p.x + static_cast<int64_t>(m0 + j) * p.ldx, s.xs, K);
      uint8_t* arow = s.act + static_cast<size_t>(j) * kp;
      QactRowResult r = qact_row(grp, s.xs, K, 32, p.row_mode != 0, s.seg, s.qred,
                                 [&](int i, int qv, int d) {
                                   arow[act_pos<FMT>(i)] = static_cast<uint8_t>(static_cast<int8_t>(qv));
                                   if ((threadIdx.x & 31) == 0) put_group<FMT, MT, PLAIN>(s, KG, j, i >> 5, d);
                                 });
      if (threadIdx.x == 0) s.Sa[j] = r.S;
    }
  } else {
    for (int j = 0; j < mt; ++j) {
      const int8_t* qr = p.q + static_cast<int64_t>(m0 + j) * p.ldq;
      const uint8_t* dr = p.da + static_cast<int64_t>(m0 + j) * p.ldd;
      uint8_t* arow = s.act + static_cast<size_t>(j) * kp;
      for (int i = threadIdx.x; i < K; i += kThreads)
        arow[act_pos<FMT>(i)] = static_cast<uint8_t>(__ldcg(qr + i));
      for (int G = threadIdx.x; G < KG; G += kThreads) put_group<FMT, MT, PLAIN>(s, KG, j, G, __ldcg(dr + G));
      if (threadIdx.x == 0) s.Sa[j] = __ldcg(p.Sa + m0 + j);
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(dst), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copy chunk kc of rows [row0, row0 + nrows) (nrows <= R) into a stage (shared address st).
// Rows past nrows and the part of a chunk past K are not copied: the stage keeps stale bytes
// there, which meet zero activation bytes or are never stored.
template <int FMT, int R, bool PLAIN>
__device__ __forceinline__ void gemv_issue(uint32_t st, const MMParams& p, int64_t row0, int nrows,
                                           int kc, int lane) {
  using F = GF<FMT>;
  const int c = lane & 7, sub = lane >> 3;   // 16-byte piece c of row sub (+ 4i)
  if (kc * F::kElems + c * (F::kElems / 8) < p.K) {
    const uint8_t* src = p.rows + (row0 + sub) * p.rs + static_cast<int64_t>(kc) * kChunk + 16 * c;
    const uint32_t dst = st + sub * kPitch + 16 * c;
#pragma unroll
    for (int i = 0; i < R / 4; ++i)
      if (4 * i + sub < nrows) cp_async16(dst + 4 * i * kPitch, src + 4 * i * p.rs);
  }
  if constexpr (!PLAIN) {
#pragma unroll
    for (int r0 = 0; r0 < R; r0 += 32) {
      const int r = r0 + lane;
      if (r < R && r < nrows) {
        const uint8_t* srow = p.srows + (row0 + r) * p.srs;
        const uint32_t dst = st + Stage<R, PLAIN>::kScaleOff + r * 16;
        const int KB = p.K / 128;
        if constexpr (FMT == kFmtInt8) {
          cp_async4(dst, srow + ((4 + p.k0 + kc) & ~3));
        } else {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const int blk = 2 * kc + b;
            if (blk < KB) {
              if constexpr (FMT == kFmtNvfp4) {
                cp_async8(dst + 8 * b, srow + 16 + 8 * (p.k0 + blk));
              } else {
                cp_async4(dst + 4 * b, srow + 8 + 4 * (p.k0 + blk));
              }
            }
          }
        }
      }
    }
  }
}

// Row g's bytes of group s of a stage for lane (g, t), as the B fragment of one MMA (two for
// nvfp4, whose 16-element sub-blocks are lanes t < 2 and t >= 2).
template <int FMT>
__device__ __forceinline__ void b_frag(const uint8_t* row, int s, int t, uint32_t& b0, uint32_t& b1) {
  if constexpr (FMT == kFmtInt8) {
    const uint2 v = *reinterpret_cast<const uint2*>(row + 32 * s + 8 * t);
    b0 = v.x;
    b1 = v.y;
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 16 * s + 4 * t);
    if constexpr (FMT == kFmtInt4) {
      b0 = (w << 4) & 0xF0F0F0F0u;   // even elements, 16x
      b1 = w & 0xF0F0F0F0u;          // odd elements, 16x
    } else {
      fp4_bytes(w, b0, b1);
    }
  }
}

// Sum over lanes of the class path: v[o][h] is this lane's share (classes g and g + 8) of row
// 8o + 2t + h. The first step keeps h by lane bit 4, the next ones split the octets by lane bits
// 3 and 2 (plain butterflies where there is nothing left to split). Returns the total of row
// 8 * oct + 2t + (lane bit 4), where oct is set by lane bits 3, 2.
template <int NO>
__device__ __forceinline__ long long class_reduce(long long (&v)[NO][2], int lane) {
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0, b2 = (lane & 4) != 0;
  long long u[NO];
#pragma unroll
  for (int o = 0; o < NO; ++o) {
    const long long send = b4 ? v[o][0] : v[o][1];
    const long long keep = b4 ? v[o][1] : v[o][0];
    u[o] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 16);
  }
  if constexpr (NO >= 2) {
#pragma unroll
    for (int o = 0; o < NO / 2; ++o) {
      const long long send = b3 ? u[o] : u[o + NO / 2];
      const long long keep = b3 ? u[o + NO / 2] : u[o];
      u[o] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 8);
    }
  } else {
    u[0] += __shfl_xor_sync(0xFFFFFFFFu, u[0], 8);
  }
  if constexpr (NO >= 4) {
    const long long send = b2 ? u[0] : u[1];
    const long long keep = b2 ? u[1] : u[0];
    u[0] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 4);
  } else {
    u[0] += __shfl_xor_sync(0xFFFFFFFFu, u[0], 4);
  }
  return u[0];
}

// The multiplier of (weight row, group s of the chunk) for the general path: ta is the
// activation-side term, sc the row's scale data in the stage.
template <int FMT, bool PLAIN>
__device__ __forceinline__ void general_mult(const uint8_t* sc, int s, int k0, int kc, int ta,
                                             int& m0, int& m1) {
  if constexpr (PLAIN) {
    m0 = m1 = ta;
  } else if constexpr (FMT == kFmtInt8) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(sc);
    const int dw = min(static_cast<int>((w >> (8 * ((4 + k0 + kc) & 3))) & 0xFFu), 31);
    m0 = m1 = ta >> dw;   // ta < 2^17: shifts of 17 or more give 0
  } else if constexpr (FMT == kFmtInt4 || FMT == kFmtFp4) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(sc + 4 * (s >> 2));
    const int sub = s & 3;
    m0 = m1 = shifted(static_cast<int>((w >> (8 + 6 * sub)) & 63u), ta, static_cast<int>(w & 0xFFu));
  } else {
    const uint32_t e = *reinterpret_cast<const uint16_t*>(sc + 8 * (s >> 2) + 2 * (s & 3));
    int mm, dw;
    e4m3_term(e & 0xFFu, mm, dw);
    m0 = shifted(mm, ta, dw);
    e4m3_term(e >> 8, mm, dw);
    m1 = shifted(mm, ta, dw);
  }
}

template <int FMT, int MT, int R, int S, int NS, bool PLAIN>
__global__ void __launch_bounds__(kThreads, R == 32 ? 1 : 2) gemv_kernel(const MMParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using F = GF<FMT>;
  using ST = Stage<R, PLAIN>;
  constexpr int NO = R / 8;                  // row octets of a block
  constexpr int TPC = kWarps / S;            // row workers of a CTA
  constexpr int VPL = 2 * NO;                // general-path values a lane
  const int K = p.K, KG = K / 32;
  const int KCH = (K + F::kElems - 1) / F::kElems;   // chunks a row
  const int kp = KCH * F::kElems;
  GSmem s = gemv_carve(smem_raw, MT, K, kp, p.x != nullptr, VPL, S, ST::kBytes, NS);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int slice = warp % S;
  const int c0 = (KCH * slice) / S, c1 = (KCH * (slice + 1)) / S;   // this warp's chunks
  const int NSL = c1 - c0;
  const int NIT = (KCH + S - 1) / S;   // items a row block: the same in every warp of the CTA
  const bool unit = (p.flags & kMmUnit) != 0;
  // this worker's rows: [rb, re), balanced by rows over all workers
  const int64_t nworkers = static_cast<int64_t>(gridDim.x) * TPC;
  const int64_t worker = static_cast<int64_t>(blockIdx.x) * TPC + warp / S;
  const int64_t rb = p.N * worker / nworkers, re = p.N * (worker + 1) / nworkers;
  const int64_t most = (p.N + nworkers - 1) / nworkers;
  const int NBLK = static_cast<int>((most + R - 1) / R);   // blocks: the same in every CTA
  uint8_t* const ring = s.ring + warp * NS * ST::kBytes;
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));

  for (int m0 = 0; m0 < p.M; m0 += MT) {
    const int mt = min(MT, p.M - m0);
    // Item (b, k): row block b of this worker, chunk c0 + k; items go through the warp's ring
    // in order, NS - 1 of them in flight ahead of the one computed.
    int bi = 0, ki = 0;   // the next item to issue
    auto issue_next = [&](int slot) {
      const int64_t r0 = rb + static_cast<int64_t>(bi) * R;
      const int nrows = static_cast<int>(min(static_cast<int64_t>(R), re - r0));
      if (bi < NBLK && ki < NSL && nrows > 0)
        gemv_issue<FMT, R, PLAIN>(ring_s + slot * ST::kBytes, p, r0, nrows, c0 + ki, lane);
      cp_async_commit();
      if (++ki == NIT) {
        ki = 0;
        ++bi;
      }
    };
#pragma unroll
    for (int q = 0; q < NS - 1; ++q) issue_next(q);
    if (m0 == 0) pdl_wait();   // the activations may come from the kernel launched before
    gemv_load_activations<FMT, MT, PLAIN>(p, s, m0, mt, kp);
    if (m0 + mt >= p.M) pdl_launch();
    const bool use_class = MT == 1 && PLAIN && *s.flag == 0;

    int D[NO][4];
    long long acc[NO][2];
#pragma unroll
    for (int o = 0; o < NO; ++o) {
#pragma unroll
      for (int i = 0; i < 4; ++i) D[o][i] = 0;
      acc[o][0] = acc[o][1] = 0;
    }
    int slot = 0;
    for (int b = 0; b < NBLK; ++b) {
      for (int k = 0; k < NIT; ++k) {
        __syncwarp();   // every lane is done with the stage that the next issue overwrites
        issue_next(slot == 0 ? NS - 1 : slot - 1);
        cp_async_wait<NS - 1>();   // this lane's copies of item (b, k) have landed
        __syncwarp();              // ... and every other lane's
        const uint8_t* st = ring + slot * ST::kBytes;
        slot = slot == NS - 1 ? 0 : slot + 1;
        if (k >= NSL) continue;
        const int kc = c0 + k;
        if (use_class) {
#pragma unroll
          for (int sg = 0; sg < F::kGroups; ++sg) {
            const int G = kc * F::kGroups + sg;
            const uint2 q = *reinterpret_cast<const uint2*>(s.act + 32 * G + 8 * t);
            const int c = s.cls[G];
            const uint32_t a0 = c == g ? q.x : 0u, a2 = c == g ? q.y : 0u;
            const uint32_t a1 = c == g + 8 ? q.x : 0u, a3 = c == g + 8 ? q.y : 0u;
#pragma unroll
            for (int o = 0; o < NO; ++o) {
              uint32_t b0, b1;
              b_frag<FMT>(st + (8 * o + g) * kPitch, sg, t, b0, b1);
              imma_acc(a0, a1, a2, a3, b0, b1, D[o]);
            }
          }
        } else {
#pragma unroll
          for (int sg = 0; sg < F::kGroups; ++sg) {
            const int G = kc * F::kGroups + sg;
            const uint2 q = *reinterpret_cast<const uint2*>(s.act + static_cast<size_t>(g < MT ? g : 0) * kp + 32 * G + 8 * t);
            const uint32_t a0 = g < MT ? q.x : 0u, a2 = g < MT ? q.y : 0u;
            const int ta = g < MT ? s.term[(g < MT ? g : 0) * KG + G] : 0;
#pragma unroll
            for (int o = 0; o < NO; ++o) {
              uint32_t b0, b1;
              b_frag<FMT>(st + (8 * o + g) * kPitch, sg, t, b0, b1);
              int d[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0};
              if constexpr (FMT == kFmtNvfp4) {
                imma_acc(a0, 0u, a2, 0u, t < 2 ? b0 : 0u, t < 2 ? b1 : 0u, d);
                imma_acc(a0, 0u, a2, 0u, t < 2 ? 0u : b0, t < 2 ? 0u : b1, e);
              } else {
                imma_acc(a0, 0u, a2, 0u, b0, b1, d);
              }
              if constexpr (FMT == kFmtInt4) {
                d[0] >>= 4;   // exact: every product was 16x
                d[1] >>= 4;
              }
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                int mA, mB;
                general_mult<FMT, PLAIN>(st + ST::kScaleOff + (8 * o + 2 * t + h) * 16, sg, p.k0, kc, ta, mA, mB);
                acc[o][h] += static_cast<long long>(d[h]) * mA;
                if constexpr (FMT == kFmtNvfp4) acc[o][h] += static_cast<long long>(e[h]) * mB;
              }
            }
          }
        }
      }
      // the row block is complete: its totals, then the S warps' partials, then the epilogue
      const int64_t r0 = rb + static_cast<int64_t>(b) * R;
      const int nrows = static_cast<int>(max(static_cast<int64_t>(0), min(static_cast<int64_t>(R), re - r0)));
      if (use_class) {
        constexpr int W = F::kW;
        const long long mlo = 1ll << (W - g);                        // class g
        const long long mhi = g + 8 <= W ? (1ll << (W - g - 8)) : 0;   // class g + 8
        long long v[NO][2];
#pragma unroll
        for (int o = 0; o < NO; ++o) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int lo = D[o][h], hi = D[o][2 + h];
            if constexpr (FMT == kFmtInt4) {
              lo >>= 4;
              hi >>= 4;
            }
            v[o][h] = lo * mlo + hi * mhi;
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) D[o][i] = 0;
        }
        long long tot = class_reduce<NO>(v, lane);
        const int oct = NO >= 4 ? (lane >> 2) & 3 : (NO >= 2 ? (lane >> 3) & 1 : 0);
        const int rr = 8 * oct + 2 * t + ((lane >> 4) & 1);
        const bool owner = NO >= 4 ? true : (NO >= 2 ? (lane & 4) == 0 : (lane & 12) == 0);
        if constexpr (S > 1) {
          if (owner) s.red[warp * 32 + lane] = tot;
          __syncthreads();
          if (slice == 0 && owner)
            for (int o = 1; o < S; ++o) tot += s.red[(warp + o) * 32 + lane];
        }
        if (slice == 0 && owner && rr < nrows) {
          const int64_t row = r0 + rr;
          const float Sw = unit ? 1.0f : __ldg(reinterpret_cast<const float*>(p.srows + row * p.srs));
          float yv = mm_epilogue(tot, Sw, s.Sa[0], W);
          float* yp = p.y + static_cast<int64_t>(m0) * p.ldy + row;
          if (p.flags & kMmAscale) {
            yv = fadd(fmul(*yp, __ldg(p.alpha + m0)), yv);
          } else if (p.flags & kMmAcc) {
            yv = fadd(*yp, yv);
          }
          *yp = yv;
        }
        if constexpr (S > 1) __syncthreads();   // red is reused by the next row block
      } else {
        if constexpr (S > 1) {
#pragma unroll
          for (int o = 0; o < NO; ++o)
#pragma unroll
            for (int h = 0; h < 2; ++h) s.red[(warp * 32 + lane) * VPL + 2 * o + h] = acc[o][h];
          __syncthreads();
          if (slice == 0)
            for (int w2 = 1; w2 < S; ++w2)
#pragma unroll
              for (int o = 0; o < NO; ++o)
#pragma unroll
                for (int h = 0; h < 2; ++h) acc[o][h] += s.red[((warp + w2) * 32 + lane) * VPL + 2 * o + h];
        }
        if (slice == 0 && g < mt) {
#pragma unroll
          for (int o = 0; o < NO; ++o)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rr = 8 * o + 2 * t + h;
              if (rr < nrows) {
                const int64_t row = r0 + rr;
                const float Sw = unit ? 1.0f : __ldg(reinterpret_cast<const float*>(p.srows + row * p.srs));
                float yv = mm_epilogue(acc[o][h], Sw, s.Sa[g], F::kW);
                float* yp = p.y + static_cast<int64_t>(m0 + g) * p.ldy + row;
                if (p.flags & kMmAscale) {
                  yv = fadd(fmul(*yp, __ldg(p.alpha + m0 + g)), yv);
                } else if (p.flags & kMmAcc) {
                  yv = fadd(*yp, yv);
                }
                *yp = yv;
              }
            }
        }
#pragma unroll
        for (int o = 0; o < NO; ++o) acc[o][0] = acc[o][1] = 0;
        if constexpr (S > 1) __syncthreads();
      }
    }
    cp_async_wait<0>();
    __syncthreads();   // the next activation rows and ring contents overwrite shared memory
  }
}

template <int FMT, int MT, int R, int S, int NS, bool PLAIN>
size_t gemv_smem(int K, bool fused) {
  using F = GF<FMT>;
  const int kp = ((K + F::kElems - 1) / F::kElems) * F::kElems;
  return gemv_layout(MT, K, kp, fused, 2 * (R / 8), S, Stage<R, PLAIN>::kBytes, NS, nullptr);
}

template <int FMT, int MT, int R, int S, int NS, bool PLAIN>
int gemv_cfg(const MMParams& p, cudaStream_t stream, bool pdl) {
  const size_t smem = gemv_smem<FMT, MT, R, S, NS, PLAIN>(p.K, p.x != nullptr);
  if (smem > 227 * 1024) return kErrArg;
  auto kern = gemv_kernel<FMT, MT, R, S, NS, PLAIN>;
  static size_t configured_smem[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (smem > 48 * 1024 && configured_smem[dev] < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured_smem[dev] = smem;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess)
    return kErrCuda;
  if (occ < 1) occ = 1;
  constexpr int TPC = kWarps / S;
  const int64_t want = (p.N + static_cast<int64_t>(R) * TPC - 1) / (static_cast<int64_t>(R) * TPC);
  const int64_t grid = min(want, static_cast<int64_t>(sm_count(dev)) * occ);
  return launch_kernel(reinterpret_cast<const void*>(kern), static_cast<int>(grid), kThreads, smem,
                       stream, pdl, p);
}

// (rows a block, K split): 32 rows a warp and no split for tall matrices; 8 rows with the split
// that keeps about 8 warps on every SM for short ones.
template <int FMT, int MT, bool PLAIN>
int gemv_split(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  const bool fused = p.x != nullptr;
  switch (split) {
    case 1:
      if (gemv_smem<FMT, MT, 32, 1, 4, PLAIN>(p.K, fused) <= 227 * 1024)
        return gemv_cfg<FMT, MT, 32, 1, 4, PLAIN>(p, stream, pdl);
      if (gemv_smem<FMT, MT, 32, 1, 2, PLAIN>(p.K, fused) <= 227 * 1024)
        return gemv_cfg<FMT, MT, 32, 1, 2, PLAIN>(p, stream, pdl);
      return gemv_cfg<FMT, MT, 8, 1, 4, PLAIN>(p, stream, pdl);
    case 2: return gemv_cfg<FMT, MT, 8, 2, 4, PLAIN>(p, stream, pdl);
    case 4: return gemv_cfg<FMT, MT, 8, 4, 4, PLAIN>(p, stream, pdl);
    default: return gemv_cfg<FMT, MT, 8, 8, 4, PLAIN>(p, stream, pdl);
  }
}

template <int FMT>
int gemv_fmt(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  const bool plain = (p.flags & (kMmUnit | kMmRsc)) != 0;
  if (p.M <= 1) {
    return plain ? gemv_split<FMT, 1, true>(p, stream, pdl, split)
                 : gemv_split<FMT, 1, false>(p, stream, pdl, split);
  }
  return plain ? gemv_split<FMT, 8, true>(p, stream, pdl, split)
               : gemv_split<FMT, 8, false>(p, stream, pdl, split);
}

}  // namespace

// Split: none while 32-row blocks give every SM eight warps; else as many warps a row as keep
// the SMs busy, each with at least one chunk.
int gemv_pick_split(int fmt, int64_t N, int K, int dev) {
  const int64_t workers = static_cast<int64_t>(sm_count(dev)) * kWarps;
  if (N >= 32 * workers) return 1;
  const int elems = fmt == kFmtInt8 ? 128 : 256;
  const int KCH = (K + elems - 1) / elems;
  int split = 1;
  while (split < 8 && (N / 8) * split < workers && KCH / (split * 2) >= 1) split *= 2;
  return split;
}

int gemv_launch(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  if (split == 0) split = gemv_pick_split(p.fmt, p.N, p.K, dev);
  switch (p.fmt) {
    case kFmtInt8: return gemv_fmt<kFmtInt8>(p, stream, pdl, split);
    case kFmtInt4: return gemv_fmt<kFmtInt4>(p, stream, pdl, split);
    case kFmtFp4: return gemv_fmt<kFmtFp4>(p, stream, pdl, split);
    case kFmtNvfp4: return gemv_fmt<kFmtNvfp4>(p, stream, pdl, split);
    default: return kErrFormat;
  }
}

}  // namespace otq
