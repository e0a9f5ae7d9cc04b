// MM for few activation rows (decode): a weight-streaming GEMV over openTPU's MX formats with
// exact integer accumulation (reference docs/isa.md "MM"; opentpu/isasim.py:749-910; scalar
// model tests/test_mx.py:131-151).
//
// Per output (activation row j, weight row n):
//   acc = sum over groups of (m << sh) * c,  c = the group's exact int dot product,
//         sh = W - dw - da (the group is dropped where sh < 0)
//   y   = (i2f(acc) * Sw[n]) * (Sa[j] * 2^-W)      -- otq_fp32.cuh mm_epilogue
//   ACC: y = y_old + y;  ASCALE: y = y_old * alpha[j] + y
//
// Engine: the integer tensor pipe as an exact dot-product unit. One mma.sync m16n8k32 (s8 x s8
// -> s32) takes one 32-element group of 16 weight rows against the same group of up to 8
// activation rows; its int32 result is exact (|c| < 2^19) and lives in registers, so each
// group's result is scaled by its own power of two (m << sh) and added into int64
// accumulators right away -- the per-group shift that keeps this from being one long MMA
// accumulation costs four integer multiply-adds. (A CUDA-core dp4a formulation runs on the
// narrow XU pipe on sm_100a; measured, it bound the kernel.)
//
// Operand layout: within a group, lane (g = lane/4, t = lane%4) supplies the weight bytes
// [8t, 8t+8) of rows g and g+8 (4-bit: the 4 bytes [4t, 4t+4) = elements 8t..8t+7) and the
// activation bytes [8t, 8t+8) of activation row g. Both operands use the same k permutation, so
// the dot product is unchanged. Weights stream straight from HBM in the reference's own row
// layout with L1-bypassing loads; activations (QACT bytes) sit in shared memory laid out
// [group][activation row][32 bytes], which makes each lane's fragment one conflict-free 8-byte
// shared load.
//
// Work split: a CTA of 8 warps takes 8/S tiles of 16 weight rows; the S warps of a tile split
// its K groups (S > 1 for matrices with few rows, so that every SM streams) and add their int64
// partials through shared memory before the epilogue. Each warp keeps U groups of loads in
// flight per lane (chunk-granular software pipelining).
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

template <int FMT>
struct Fmt {
  static constexpr int kW = (FMT == kFmtInt8) ? 16 : (FMT == kFmtNvfp4 ? 13 : 11);
  static constexpr int kGroupBytes = (FMT == kFmtInt8) ? 32 : 16;   // a 32-element group of a row
  static constexpr int kLaneBytes = (FMT == kFmtInt8) ? 8 : 4;      // what one lane reads of it
  static constexpr int kU = (FMT == kFmtInt8) ? 4 : 8;              // groups in flight per lane
};

// Shared memory of a CTA.
struct Smem {
  uint8_t* act;   // [KG][MT][32] QACT bytes (int4: each run of 8 stored evens then odds)
  int* gB;        // [KG][MT] activation side of the group multiplier (see group_terms)
  int* gA;        // [KG][MT] 4-bit formats: W - da
  int* gC;        // [KG][MT] int4: 8 * sum(q)
  float* Sa;      // [MT]
  long long* red; // [kWarps][32][4] K-split partials
  float* xs;      // [K] the fp32 row being quantized (fused QACT)
  uint32_t* seg;  // [KG]
  uint32_t* qred; // [40]
};

__host__ __device__ inline size_t smem_layout(int MT, int K, bool fused, size_t* offs) {
  const size_t KG = K / 32;
  size_t off = 0;
  auto take = [&](int i, size_t bytes) {
    off = (off + 15) & ~size_t(15);
    if (offs) offs[i] = off;
    off += bytes;
  };
  take(0, KG * MT * 32);
  take(1, KG * MT * 4);
  take(2, KG * MT * 4);
  take(3, KG * MT * 4);
  take(4, MT * 4);
  take(5, static_cast<size_t>(kWarps) * 32 * 4 * 8);
  take(6, fused ? static_cast<size_t>(K) * 4 : 0);
  take(7, KG * 4);
  take(8, 40 * 4);
  return off;
}

template <int MT>
__device__ __forceinline__ Smem carve(unsigned char* base, int K, bool fused) {
  size_t o[9];
  smem_layout(MT, K, fused, o);
  Smem s;
  s.act = base + o[0];
  s.gB = reinterpret_cast<int*>(base + o[1]);
  s.gA = reinterpret_cast<int*>(base + o[2]);
  s.gC = reinterpret_cast<int*>(base + o[3]);
  s.Sa = reinterpret_cast<float*>(base + o[4]);
  s.red = reinterpret_cast<long long*>(base + o[5]);
  s.xs = reinterpret_cast<float*>(base + o[6]);
  s.seg = reinterpret_cast<uint32_t*>(base + o[7]);
  s.qred = reinterpret_cast<uint32_t*>(base + o[8]);
  return s;
}

// Element i of activation row j -> its byte in shared memory ([group][row][32]); int4 stores
// each run of 8 as evens then odds, the order in which a packed word's low and high nibbles
// come out.
template <int FMT, int MT>
__device__ __forceinline__ int act_index(int j, int i) {
  int e = i & 31;
  if constexpr (FMT == kFmtInt4) {
    const int r = e & 7;
    e = (e & ~7) | ((r & 1) ? 4 + (r >> 1) : (r >> 1));
  }
  return ((i >> 5) * MT + j) * 32 + e;
}

// The activation side of a group's shift, once per (row, group): sh = W - dw - da. int8:
// gB = 2^(16 - da) (0 if da > 16), so the multiplier is gB >> dw -- the shift right drops
// exactly the groups with dw + da > 16. 4-bit: gA = W - da, gB = 2^gA (0 if negative) for rows
// without offsets (RSC / UNIT). int4: gC = 8 * sum(q), the bias of nibbles read as value + 8.
template <int FMT, int MT>
__device__ __forceinline__ void group_terms(const Smem& s, int j, int g, int da, int qsum) {
  constexpr int W = Fmt<FMT>::kW;
  const int sh = W - da;
  s.gB[g * MT + j] = sh >= 0 ? (1 << sh) : 0;
  s.gA[g * MT + j] = sh;
  s.gC[g * MT + j] = 8 * qsum;
}

// Activation rows [m0, m0 + mt) into shared memory (QACT of fp32 x, or copied bytes); rows
// mt..MT-1 of the tile are zeros.
template <int FMT, int MT>
__device__ void load_activations(const MMParams& p, const Smem& s, int m0, int mt) {
  const int K = p.K;
  const int KG = K >> 5;
  if (mt < MT) {
    for (int i = threadIdx.x; i < KG * MT * 8; i += kThreads) {
      const int g = i / (MT * 8), rem = i % (MT * 8), j = rem / 8;
      if (j >= mt) reinterpret_cast<uint32_t*>(s.act)[i] = 0u;
      if (rem % 8 == 0 && j >= mt) {
        s.gB[g * MT + j] = 0;
        s.gA[g * MT + j] = -1;
        s.gC[g * MT + j] = 0;
      }
    }
    if (threadIdx.x < MT && static_cast<int>(threadIdx.x) >= mt) s.Sa[threadIdx.x] = 0.0f;
  }
  if (p.x != nullptr) {
    const ThreadGroup<kThreads> grp{static_cast<int>(threadIdx.x)};
    for (int j = 0; j < mt; ++j) {
      stage_row(grp, p.x + static_cast<int64_t>(m0 + j) * p.ldx, s.xs, K);
      QactRowResult r = qact_row(
          grp, s.xs, K, 32, p.row_mode != 0, s.seg, s.qred, [&](int i, int qv, int d) {
            s.act[act_index<FMT, MT>(j, i)] = static_cast<uint8_t>(static_cast<int8_t>(qv));
            const int sum = (FMT == kFmtInt4) ? __reduce_add_sync(0xFFFFFFFFu, qv) : 0;
            if ((threadIdx.x & 31) == 0) group_terms<FMT, MT>(s, j, i >> 5, d, sum);
          });
      if (threadIdx.x == 0) s.Sa[j] = r.S;
    }
  } else {
    for (int j = 0; j < mt; ++j) {
      const int8_t* qr = p.q + static_cast<int64_t>(m0 + j) * p.ldq;
      const uint8_t* dr = p.da + static_cast<int64_t>(m0 + j) * p.ldd;
      for (int i = threadIdx.x; i < K; i += kThreads) {   // K % 32 == 0: warps stay whole
        const int qv = __ldcg(qr + i);
        s.act[act_index<FMT, MT>(j, i)] = static_cast<uint8_t>(static_cast<int8_t>(qv));
        const int sum = (FMT == kFmtInt4) ? __reduce_add_sync(0xFFFFFFFFu, qv) : 0;
        if ((threadIdx.x & 31) == 0) group_terms<FMT, MT>(s, j, i >> 5, __ldcg(dr + (i >> 5)), sum);
      }
      if (threadIdx.x == 0) s.Sa[j] = __ldcg(p.Sa + m0 + j);
    }
  }
  __syncthreads();
}

// The scale data of (row, group G): int8 the block's dw byte, int4 / fp4 the block's word,
// nvfp4 the sub-block's two E4M3 bytes.
template <int FMT>
__device__ __forceinline__ uint32_t load_scale(const uint8_t* srow, int k0, int G) {
  if constexpr (FMT == kFmtInt8) {
    return __ldg(srow + 4 + k0 + (G >> 2));
  } else if constexpr (FMT == kFmtInt4 || FMT == kFmtFp4) {
    return __ldg(reinterpret_cast<const uint32_t*>(srow + 8 + 4 * (k0 + (G >> 2))));
  } else {
    return __ldg(reinterpret_cast<const uint16_t*>(srow + 16 + 8 * (k0 + (G >> 2)) + 2 * (G & 3)));
  }
}

// One lane's registers for one group: weight words of rows g and g+8, and their scale data.
template <int FMT>
struct Slot {
  uint32_t w[Fmt<FMT>::kLaneBytes / 2];   // int8: row g (2 words), row g+8 (2); 4-bit: 1 + 1
  uint32_t sc[2];
};

template <int FMT, bool PLAIN>
__device__ __forceinline__ void load_slot(Slot<FMT>& sl, const uint8_t* rg, const uint8_t* rh,
                                          const uint8_t* sg, const uint8_t* sh, int k0, int G,
                                          int t, bool okg, bool okh) {
  constexpr int GB = Fmt<FMT>::kGroupBytes, LB = Fmt<FMT>::kLaneBytes;
  const int off = G * GB + t * LB;
  if constexpr (FMT == kFmtInt8) {
    const uint2 a = okg ? ld_stream8(rg + off) : make_uint2(0u, 0u);
    const uint2 b = okh ? ld_stream8(rh + off) : make_uint2(0u, 0u);
    sl.w[0] = a.x;
    sl.w[1] = a.y;
    sl.w[2] = b.x;
    sl.w[3] = b.y;
  } else {
    sl.w[0] = okg ? ld_stream4(rg + off) : 0u;
    sl.w[1] = okh ? ld_stream4(rh + off) : 0u;
  }
  if constexpr (!PLAIN) {
    sl.sc[0] = okg ? load_scale<FMT>(sg, k0, G) : 0u;
    sl.sc[1] = okh ? load_scale<FMT>(sh, k0, G) : 0u;
  }
}

// acc (rows g, g+8 x activation rows 2t, 2t+1) += the exact contribution of group G.
template <int FMT, int MT, bool PLAIN>
__device__ __forceinline__ void mma_group(const Smem& s, int G, int lane, const Slot<FMT>& sl,
                                          long long (&acc)[4]) {
  const int g = lane >> 2, t = lane & 3;
  uint32_t b0 = 0u, b1 = 0u;
  if (g < MT) {
    const uint2 bv = *reinterpret_cast<const uint2*>(s.act + (G * MT + g) * 32 + 8 * t);
    b0 = bv.x;
    b1 = bv.y;
  }
  const int c0 = 2 * t, c1 = 2 * t + 1;
  const int cc0 = c0 < MT ? c0 : 0, cc1 = c1 < MT ? c1 : 0;   // columns past MT read col 0 (d is 0)
  if constexpr (FMT == kFmtInt8) {
    int d[4];
    imma(sl.w[0], sl.w[2], sl.w[1], sl.w[3], b0, b1, d);
    const int B0 = s.gB[G * MT + cc0], B1 = s.gB[G * MT + cc1];
    if constexpr (PLAIN) {
      acc[0] += static_cast<long long>(d[0]) * B0;
      acc[1] += static_cast<long long>(d[1]) * B1;
      acc[2] += static_cast<long long>(d[2]) * B0;
      acc[3] += static_cast<long long>(d[3]) * B1;
    } else {
      // dw is a byte; B0 < 2^17, so any shift of 17 or more gives 0 (clamped below 32)
      const int dwg = min(static_cast<int>(sl.sc[0]), 31), dwh = min(static_cast<int>(sl.sc[1]), 31);
      acc[0] += static_cast<long long>(d[0]) * (B0 >> dwg);
      acc[1] += static_cast<long long>(d[1]) * (B1 >> dwg);
      acc[2] += static_cast<long long>(d[2]) * (B0 >> dwh);
      acc[3] += static_cast<long long>(d[3]) * (B1 >> dwh);
    }
  } else if constexpr (FMT == kFmtInt4 || FMT == kFmtFp4) {
    uint32_t glo, ghi, hlo, hhi;
    if constexpr (FMT == kFmtInt4) {
      int4_bytes(sl.w[0], glo, ghi);
      int4_bytes(sl.w[1], hlo, hhi);
    } else {
      fp4_bytes(sl.w[0], glo, ghi);
      fp4_bytes(sl.w[1], hlo, hhi);
    }
    int d[4];
    imma(glo, hlo, ghi, hhi, b0, b1, d);
    if constexpr (FMT == kFmtInt4) {
      const int C0 = s.gC[G * MT + cc0], C1 = s.gC[G * MT + cc1];
      d[0] -= C0;
      d[1] -= C1;
      d[2] -= C0;
      d[3] -= C1;
    }
    if constexpr (PLAIN) {
      const int B0 = s.gB[G * MT + cc0], B1 = s.gB[G * MT + cc1];
      acc[0] += static_cast<long long>(d[0]) * B0;
      acc[1] += static_cast<long long>(d[1]) * B1;
      acc[2] += static_cast<long long>(d[2]) * B0;
      acc[3] += static_cast<long long>(d[3]) * B1;
    } else {
      const int A0 = s.gA[G * MT + cc0], A1 = s.gA[G * MT + cc1];
      const int sub = G & 3;
      const int dwg = static_cast<int>(sl.sc[0] & 0xFFu), dwh = static_cast<int>(sl.sc[1] & 0xFFu);
      const int mg = static_cast<int>((sl.sc[0] >> (8 + 6 * sub)) & 63u);
      const int mh = static_cast<int>((sl.sc[1] >> (8 + 6 * sub)) & 63u);
      acc[0] += static_cast<long long>(d[0]) * shifted(mg, A0, dwg);
      acc[1] += static_cast<long long>(d[1]) * shifted(mg, A1, dwg);
      acc[2] += static_cast<long long>(d[2]) * shifted(mh, A0, dwh);
      acc[3] += static_cast<long long>(d[3]) * shifted(mh, A1, dwh);
    }
  } else {   // nvfp4: the sub-block's two groups of 16 (lanes t < 2 hold the first) in two MMAs
    uint32_t glo, ghi, hlo, hhi;
    fp4_bytes(sl.w[0], glo, ghi);
    fp4_bytes(sl.w[1], hlo, hhi);
    const bool first = t < 2;
    int d0[4], d1[4];
    imma(first ? glo : 0u, first ? hlo : 0u, first ? ghi : 0u, first ? hhi : 0u, b0, b1, d0);
    imma(first ? 0u : glo, first ? 0u : hlo, first ? 0u : ghi, first ? 0u : hhi, b0, b1, d1);
    const int A0 = s.gA[G * MT + cc0], A1 = s.gA[G * MT + cc1];
    int mg0 = 1, mg1 = 1, mh0 = 1, mh1 = 1, dg0 = 0, dg1 = 0, dh0 = 0, dh1 = 0;
    if constexpr (!PLAIN) {
      e4m3_term(sl.sc[0] & 0xFFu, mg0, dg0);
      e4m3_term((sl.sc[0] >> 8) & 0xFFu, mg1, dg1);
      e4m3_term(sl.sc[1] & 0xFFu, mh0, dh0);
      e4m3_term((sl.sc[1] >> 8) & 0xFFu, mh1, dh1);
    }
    acc[0] += static_cast<long long>(d0[0]) * shifted(mg0, A0, dg0) +
              static_cast<long long>(d1[0]) * shifted(mg1, A0, dg1);
    acc[1] += static_cast<long long>(d0[1]) * shifted(mg0, A1, dg0) +
              static_cast<long long>(d1[1]) * shifted(mg1, A1, dg1);
    acc[2] += static_cast<long long>(d0[2]) * shifted(mh0, A0, dh0) +
              static_cast<long long>(d1[2]) * shifted(mh1, A0, dh1);
    acc[3] += static_cast<long long>(d0[3]) * shifted(mh0, A1, dh0) +
              static_cast<long long>(d1[3]) * shifted(mh1, A1, dh1);
  }
}

template <int FMT, int MT, int S, bool PLAIN>
__global__ void __launch_bounds__(kThreads, (MT <= 2 && S == 1) ? (PLAIN ? 4 : 3) : 2) mm_tile_kernel(const MMParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using F = Fmt<FMT>;
  constexpr int U = F::kU;
  constexpr int TPC = kWarps / S;                 // row tiles per CTA iteration
  const int K = p.K;
  const int KG = K >> 5;
  Smem s = carve<MT>(smem_raw, K, p.x != nullptr);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int slice = warp % S, tw = warp / S;
  const int G0 = (KG * slice) / S, G1 = (KG * (slice + 1)) / S;   // this warp's groups
  const int NGS = G1 - G0;
  // batches of U groups per tile: the same count in every warp of the CTA (slices can differ by
  // a group), so the CTA-wide barriers of the K-split reduction are reached together
  const int NBT = ((KG + S - 1) / S + U - 1) / U;
  const bool unit = (p.flags & kMmUnit) != 0;
  const int64_t ntiles = (p.N + 15) / 16;
  const int64_t cstride = static_cast<int64_t>(gridDim.x) * TPC;
  const int64_t ctile0 = static_cast<int64_t>(blockIdx.x) * TPC;   // this CTA's first tile

  // The weights never depend on the kernel launched before this one: pull this warp's first
  // tile (its K slice) into L2 before waiting for that kernel (programmatic dependent launch).
  {
    const int64_t tile = ctile0 + tw;
    const int64_t row = tile * 16 + lane;
    if (lane < 16 && tile < ntiles && row < p.N && NGS > 0)
      prefetch_l2(p.rows + row * p.rs + G0 * F::kGroupBytes,
                  static_cast<uint32_t>(NGS * F::kGroupBytes));
  }
  pdl_wait();   // the activations may come from the kernel launched before this one

  for (int m0 = 0; m0 < p.M; m0 += MT) {
    const int mt = min(MT, p.M - m0);
    load_activations<FMT, MT>(p, s, m0, mt);
    if (m0 + mt >= p.M) pdl_launch();

    // Item (it, k): CTA iteration it (row tile ctile0 + it*cstride + tw), batch k of U groups
    // of this warp's slice. As slot u of batch k is consumed it is refilled with slot u of the
    // next item, so U groups of loads per lane stay in flight.
    auto rows_of = [&](int64_t it, const uint8_t*& rg, const uint8_t*& rh, const uint8_t*& sg,
                       const uint8_t*& sh, bool& okg, bool& okh) {
      const int64_t tile = ctile0 + it * cstride + tw;
      const int64_t r0 = tile * 16 + g, r1 = r0 + 8;
      okg = tile < ntiles && r0 < p.N;
      okh = tile < ntiles && r1 < p.N;
      rg = p.rows + (okg ? r0 : 0) * p.rs;
      rh = p.rows + (okh ? r1 : 0) * p.rs;
      sg = unit ? nullptr : p.srows + (okg ? r0 : 0) * p.srs;
      sh = unit ? nullptr : p.srows + (okh ? r1 : 0) * p.srs;
    };
    Slot<FMT> slot[U];
    long long acc[4] = {0, 0, 0, 0};
    int64_t it = 0;
    int k = 0;
    bool active = ctile0 < ntiles;
    const uint8_t *rg, *rh, *sg, *sh;
    bool okg, okh;
    rows_of(0, rg, rh, sg, sh, okg, okh);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool in = u < NGS;
      load_slot<FMT, PLAIN>(slot[u], rg, rh, sg, sh, p.k0, G0 + u, t, okg && in, okh && in);
    }
    while (active) {
      int64_t itn = it;
      int kn = k + 1;
      if (kn == NBT) {
        kn = 0;
        ++itn;
      }
      const bool active_n = ctile0 + itn * cstride < ntiles;
      const uint8_t *rgn = rg, *rhn = rh, *sgn = sg, *shn = sh;
      bool okgn = okg, okhn = okh;
      if (itn != it) rows_of(itn, rgn, rhn, sgn, shn, okgn, okhn);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const Slot<FMT> cur = slot[u];
        const int Gn = kn * U + u;
        const bool inn = active_n && Gn < NGS;
        load_slot<FMT, PLAIN>(slot[u], rgn, rhn, sgn, shn, p.k0, G0 + Gn, t, okgn && inn,
                              okhn && inn);
        if (k * U + u < NGS) mma_group<FMT, MT, PLAIN>(s, G0 + k * U + u, lane, cur, acc);
      }
      if (k == NBT - 1) {
        // the S warps of a tile add their partials; the tile's first warp runs the epilogue
        if constexpr (S > 1) {
          long long* mine = s.red + (warp * 32 + lane) * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i) mine[i] = acc[i];
          __syncthreads();
          if (slice == 0) {
            for (int o = 1; o < S; ++o) {
              const long long* other = s.red + ((warp + o) * 32 + lane) * 4;
#pragma unroll
              for (int i = 0; i < 4; ++i) acc[i] += other[i];
            }
          }
        }
        if (slice == 0) {
          const int64_t tile = ctile0 + it * cstride + tw;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int64_t row = tile * 16 + g + (i >= 2 ? 8 : 0);
            const int col = 2 * t + (i & 1);
            if (tile < ntiles && row < p.N && col < mt) {
              const float Sw =
                  unit ? 1.0f : __ldg(reinterpret_cast<const float*>(p.srows + row * p.srs));
              float yv = mm_epilogue(acc[i], Sw, s.Sa[col], F::kW);
              float* yp = p.y + static_cast<int64_t>(m0 + col) * p.ldy + row;
              if (p.flags & kMmAscale) {
                yv = fadd(fmul(*yp, __ldg(p.alpha + m0 + col)), yv);
              } else if (p.flags & kMmAcc) {
                yv = fadd(*yp, yv);
              }
              *yp = yv;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = 0;
        if constexpr (S > 1) __syncthreads();   // red is reused by the next iteration
      }
      it = itn;
      k = kn;
      active = active_n;
      rg = rgn;
      rh = rhn;
      sg = sgn;
      sh = shn;
      okg = okgn;
      okh = okhn;
    }
    __syncthreads();   // the next activation tile overwrites shared memory
  }
}

template <int FMT, int MT, int S, bool PLAIN>
int launch_cfg(const MMParams& p, cudaStream_t stream, bool pdl) {
  const size_t smem = smem_layout(MT, p.K, p.x != nullptr, nullptr);
  auto kern = mm_tile_kernel<FMT, MT, S, PLAIN>;
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
  // One wave at most; within it as few CTAs as give every CTA the same number of iterations.
  constexpr int TPC = kWarps / S;
  const int64_t ntiles = (p.N + 15) / 16;
  const int64_t ctas_needed = (ntiles + TPC - 1) / TPC;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * occ;
  const int64_t iters = (ctas_needed + cap - 1) / cap;
  const int64_t grid = (ctas_needed + iters - 1) / iters;
  return launch_kernel(reinterpret_cast<const void*>(kern), static_cast<int>(grid), kThreads, smem,
                       stream, pdl, p);
}

template <int FMT, int MT, bool PLAIN>
int launch_split(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  switch (split) {
    case 1: return launch_cfg<FMT, MT, 1, PLAIN>(p, stream, pdl);
    case 2: return launch_cfg<FMT, MT, 2, PLAIN>(p, stream, pdl);
    case 4: return launch_cfg<FMT, MT, 4, PLAIN>(p, stream, pdl);
    default: return launch_cfg<FMT, MT, 8, PLAIN>(p, stream, pdl);
  }
}

template <int FMT, int MT>
int launch_plain(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  if (p.flags & (kMmUnit | kMmRsc)) return launch_split<FMT, MT, true>(p, stream, pdl, split);
  return launch_split<FMT, MT, false>(p, stream, pdl, split);
}

template <int FMT>
int launch_fmt(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  if (p.M <= 1) return launch_plain<FMT, 1>(p, stream, pdl, split);
  if (p.M <= 2) return launch_plain<FMT, 2>(p, stream, pdl, split);
  if (p.M <= 4) return launch_plain<FMT, 4>(p, stream, pdl, split);
  return launch_plain<FMT, 8>(p, stream, pdl, split);
}

}  // namespace

size_t mm_smem_bytes(int fmt, int mt, int K, bool fused) {
  (void)fmt;
  return smem_layout(mt, K, fused, nullptr);
}

// K-split: as many warps per 16-row tile as keep every SM streaming when the matrix has few
// rows, while each warp keeps at least a few groups to stream.
int mm_pick_split(int fmt, int64_t N, int K, int dev) {
  (void)fmt;
  const int64_t tiles = (N + 15) / 16;
  const int64_t want_warps = static_cast<int64_t>(sm_count(dev)) * 16;
  const int KG = K / 32;
  int split = 1;
  while (split < 8 && tiles * split < want_warps && KG / (split * 2) >= 4) split *= 2;
  return split;
}

int mm_launch(const MMParams& p0, cudaStream_t stream, bool pdl) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  MMParams p = p0;
  p.status = status_word();
  const bool fused = p.x != nullptr;
  int kernel = p.kernel;
  if (kernel == kKernelAuto) {
    // one or two activation rows: row spans (contiguous loads, few instructions a byte); more:
    // 16-row tiles, whose MMA serves up to 8 activation rows at once
    kernel = (p.M <= 2 && rows_smem_bytes(p.M, p.K, fused) <= 227 * 1024) ? kKernelRows
                                                                            : kKernelTile;
  }
  if (kernel == kKernelGemv) return gemv_launch(p, stream, pdl, p.split);
  if (kernel == kKernelRows) {
    if (rows_smem_bytes(p.M <= 1 ? 1 : 2, p.K, fused) > 227 * 1024) return kErrArg;
    return mm_rows_launch(p, stream, pdl, p.split);
  }
  if (kernel == kKernelRing) {
    if (ring_smem_bytes(p.fmt, p.K, p.M, fused) > 227 * 1024) return kErrArg;
    return mm_ring_launch(p, stream, pdl);
  }
  const int mt = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
  if (mm_smem_bytes(p.fmt, mt, p.K, fused) > 227 * 1024) return kErrArg;
  const int split = p.split > 0 ? p.split : mm_pick_split(p.fmt, p.N, p.K, dev);
  switch (p.fmt) {
    case kFmtInt8: return launch_fmt<kFmtInt8>(p, stream, pdl, split);
    case kFmtInt4: return launch_fmt<kFmtInt4>(p, stream, pdl, split);
    case kFmtFp4: return launch_fmt<kFmtFp4>(p, stream, pdl, split);
    case kFmtNvfp4: return launch_fmt<kFmtNvfp4>(p, stream, pdl, split);
    default: return kErrFormat;
  }
}

}  // namespace otq
