// MM for one or two activation rows (decode): the row-streaming GEMV over openTPU's MX formats,
// with exact integer accumulation (reference docs/isa.md "MM"; opentpu/isasim.py:749-910;
// scalar model tests/test_mx.py:131-151).
//
//   acc = sum over 32-element groups of (m << sh) * c,  c = the group's exact int dot product,
//         sh = W - dw - da (the group is dropped where sh < 0)
//   y   = (i2f(acc) * Sw[n]) * (Sa[j] * 2^-W)      -- otq_fp32.cuh mm_epilogue
//
// Loads: a warp reads a "span" of one weight row -- 512 elements, 16 groups -- with every lane
// taking 16 contiguous elements (int8: 16 bytes, 4-bit: 8 bytes), so one load instruction moves
// 512 (256) contiguous bytes. Quad g of the warp (lanes 4g..4g+3) holds groups 2g (lanes t = 0, 1)
// and 2g+1 (t = 2, 3) of the span.
//
// Dot products: one mma.sync m16n8k32 (s8 x s8 -> s32) per 8 elements a lane holds. Its B
// operand is the weights as loaded: column n is quad n's data. Its A operand is the activation
// bytes that match each lane's weight bytes, placed in row g when the lane's data is group 2g
// (t < 2) and in row g + 8 when it is group 2g+1, zeros elsewhere. Row g of A and column g of
// B both live in quad g, so D[g][g] is exactly group 2g's dot product and D[g+8][g] group
// 2g+1's -- a "diagonal" use of the MMA that needs no data movement between lanes. Both come out
// in lane (g, t = g/2); that lane scales them by their group multipliers into int64
// accumulators. (nvfp4 has a scale per 16 elements, one lane's share: two MMAs with different
// lane masks keep the four sub-blocks of a quad apart.)
//
// Work split: a warp takes R rows at a time, so each span's activation fragments are read from
// shared memory once for R rows. For matrices with few rows, S warps of a CTA split a row's
// spans and add their partials through shared memory.
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
constexpr int kSpan = 512;   // elements of a row that a warp reads at once

template <int FMT>
struct RF {
  static constexpr int kW = (FMT == kFmtInt8) ? 16 : (FMT == kFmtNvfp4 ? 13 : 11);
  static constexpr int kLaneBytes = (FMT == kFmtInt8) ? 16 : 8;
  static constexpr int kSpanBytes = 32 * kLaneBytes;
  static constexpr int kLaneWords = kLaneBytes / 4;
};

// Shared memory of a CTA.
struct RSmem {
  uint8_t* act;     // [MR][KS * 512] activation bytes (int4: each run of 8 as evens, then odds)
  int4* terms;      // [MR][KS * 8] per pair of groups: {xA, cA, xB, cB}, see group_term
  float* Sa;        // [MR]
  long long* red;   // [kWarps][R * MR] span-split partials
  float* xs;        // [K] the fp32 row being quantized (fused QACT)
  uint32_t* seg;    // [K / 32]
  uint32_t* qred;   // [40]
  uint8_t* ring;    // [kWarps][NS] stages of each warp's weight ring
};

// slot_bytes: one stage of a warp's ring (R rows of a span, and their scale words).
__host__ __device__ inline size_t rows_layout(int MR, int R, int K, bool fused, int slot_bytes,
                                              int ns, size_t* offs) {
  const size_t KS = (K + kSpan - 1) / kSpan;
  size_t off = 0;
  auto take = [&](int i, size_t bytes) {
    off = (off + 15) & ~size_t(15);
    if (offs) offs[i] = off;
    off += bytes;
  };
  take(0, MR * KS * kSpan);
  take(1, MR * KS * 8 * sizeof(int4));
  take(2, MR * 4);
  take(3, static_cast<size_t>(kWarps) * R * MR * 8);
  take(4, fused ? static_cast<size_t>(K) * 4 : 0);
  take(5, static_cast<size_t>(K / 32) * 4);
  take(6, 40 * 4);
  take(7, static_cast<size_t>(kWarps) * ns * slot_bytes);
  return off;
}

__device__ __forceinline__ RSmem rows_carve(unsigned char* base, int MR, int R, int K, bool fused,
                                            int slot_bytes, int ns) {
  size_t o[8];
  rows_layout(MR, R, K, fused, slot_bytes, ns, o);
  RSmem s;
  s.act = base + o[0];
  s.terms = reinterpret_cast<int4*>(base + o[1]);
  s.Sa = reinterpret_cast<float*>(base + o[2]);
  s.red = reinterpret_cast<long long*>(base + o[3]);
  s.xs = reinterpret_cast<float*>(base + o[4]);
  s.seg = reinterpret_cast<uint32_t*>(base + o[5]);
  s.qred = reinterpret_cast<uint32_t*>(base + o[6]);
  s.ring = base + o[7];
  return s;
}

// Element i of an activation row -> its byte in the row's span layout.
template <int FMT>
__device__ __forceinline__ int act_pos(int i) {
  if constexpr (FMT == kFmtInt4) {
    const int r = i & 7;
    return (i & ~7) | ((r & 1) ? 4 + (r >> 1) : (r >> 1));
  }
  return i;
}

// A group's activation-side terms. x: int8, and 4-bit rows without per-block scales (PLAIN):
// 2^(W - da), 0 where that is below 1 -- the group multiplier itself, or (int8 MX) the value
// that a shift right by dw turns into it; 4-bit MX: W - da. c: int4, 8 * sum(q), the bias of
// nibbles read as value + 8.
template <int FMT, bool PLAIN>
__device__ __forceinline__ int2 group_term(int da, int qsum) {
  constexpr int W = RF<FMT>::kW;
  const int sh = W - da;
  int x;
  if constexpr (FMT == kFmtInt8 || PLAIN) {
    x = sh >= 0 ? (1 << sh) : 0;
  } else {
    x = sh;
  }
  return make_int2(x, FMT == kFmtInt4 ? 8 * qsum : 0);
}

template <int FMT, int MR, bool PLAIN>
__device__ __forceinline__ void put_term(const RSmem& s, int KS, int j, int G, int da, int qsum) {
  int2* t = reinterpret_cast<int2*>(s.terms + static_cast<size_t>(j) * KS * 8);
  t[G] = group_term<FMT, PLAIN>(da, qsum);
}

// Activation rows [m0, m0 + mt) into shared memory (QACT of fp32 x, or copied bytes). Bytes and
// terms past K, and rows mt..MR-1, are zeros.
template <int FMT, int MR, bool PLAIN>
__device__ void rows_load_activations(const MMParams& p, const RSmem& s, int m0, int mt, int KS) {
  const int K = p.K;
  const int KP = KS * kSpan;
  for (int j = 0; j < MR; ++j) {
    const int from = j < mt ? K : 0;
    uint32_t* aw = reinterpret_cast<uint32_t*>(s.act + static_cast<size_t>(j) * KP);
    for (int i = (from >> 2) + threadIdx.x; i < (KP >> 2); i += kThreads) aw[i] = 0u;
    int2* tw = reinterpret_cast<int2*>(s.terms + static_cast<size_t>(j) * KS * 8);
    for (int G = (from >> 5) + threadIdx.x; G < KS * 16; G += kThreads) tw[G] = make_int2(0, 0);
  }
  if (threadIdx.x < MR && static_cast<int>(threadIdx.x) >= mt) s.Sa[threadIdx.x] = 0.0f;
  if (p.x != nullptr) {
    const ThreadGroup<kThreads> grp{static_cast<int>(threadIdx.x)};
    for (int j = 0; j < mt; ++j) {
      stage_row(grp, p.x + static_cast<int64_t>(m0 + j) * p.ldx, s.xs, K);
      uint8_t* arow = s.act + static_cast<size_t>(j) * KP;
      QactRowResult r = qact_row(
          grp, s.xs, K, 32, p.row_mode != 0, s.seg, s.qred, [&](int i, int qv, int d) {
            arow[act_pos<FMT>(i)] = static_cast<uint8_t>(static_cast<int8_t>(qv));
            const int sum = (FMT == kFmtInt4) ? __reduce_add_sync(0xFFFFFFFFu, qv) : 0;
            if ((threadIdx.x & 31) == 0) put_term<FMT, MR, PLAIN>(s, KS, j, i >> 5, d, sum);
          });
      if (threadIdx.x == 0) s.Sa[j] = r.S;
    }
  } else {
    for (int j = 0; j < mt; ++j) {
      const int8_t* qr = p.q + static_cast<int64_t>(m0 + j) * p.ldq;
      const uint8_t* dr = p.da + static_cast<int64_t>(m0 + j) * p.ldd;
      uint8_t* arow = s.act + static_cast<size_t>(j) * KP;
      for (int i = threadIdx.x; i < K; i += kThreads) {   // K % 32 == 0: warps stay whole
        const int qv = __ldcg(qr + i);
        arow[act_pos<FMT>(i)] = static_cast<uint8_t>(static_cast<int8_t>(qv));
        const int sum = (FMT == kFmtInt4) ? __reduce_add_sync(0xFFFFFFFFu, qv) : 0;
        if ((threadIdx.x & 31) == 0) put_term<FMT, MR, PLAIN>(s, KS, j, i >> 5, __ldcg(dr + (i >> 5)), sum);
      }
      if (threadIdx.x == 0) s.Sa[j] = __ldcg(p.Sa + m0 + j);
    }
  }
  __syncthreads();
}

// A warp's weight ring: stage = R rows x one span (kSpanBytes each), then (MX rows) R x 8 scale
// words, one for each quad. The copies are cp.async (16 bytes a lane, straight to shared memory,
// nothing held in registers while in flight), so a warp keeps NS - 1 spans of R rows in flight
// whatever its register budget; cp.async.wait_group is a hardware wait.
template <int FMT, int R, bool PLAIN>
struct Ring {
  static constexpr int kSpanBytes = RF<FMT>::kSpanBytes;
  static constexpr int kScaleOff = R * kSpanBytes;
  static constexpr int kSlotBytes = kScaleOff + (PLAIN ? 0 : R * 8 * 4);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(dst), "l"(src)
               : "memory");
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

// Byte offset of the scale word that (row, 128-element block blk) needs, within the scale row:
// int8 the aligned word holding the block's dw byte, int4 / fp4 the block's word, nvfp4 the
// four sub-block bytes of quad g.
template <int FMT>
__device__ __forceinline__ int scale_word_offset(int k0, int blk, int g) {
  if constexpr (FMT == kFmtInt8) {
    return (4 + k0 + blk) & ~3;
  } else if constexpr (FMT == kFmtInt4 || FMT == kFmtFp4) {
    return 8 + 4 * (k0 + blk);
  } else {
    return 16 + 8 * (k0 + blk) + 4 * (g & 1);
  }
}

// Issue the copies of one item (rows row0.. row0+R-1, span) into a stage (shared address st).
// Rows past N and the part of a span past K are not copied: the stage keeps stale bytes there,
// which meet zero activations (or are never stored).
template <int FMT, int R, bool PLAIN>
__device__ __forceinline__ void rows_issue(uint32_t st, const MMParams& p, int64_t row0, int span,
                                           int lane, bool valid) {
  using F = RF<FMT>;
  using G = Ring<FMT, R, PLAIN>;
  constexpr int CPR = F::kSpanBytes / 16;   // 16-byte copies a row
  constexpr int RPI = 32 / CPR;             // rows a warp copies at once
  const int sub = lane / CPR, c = lane % CPR;
  const int64_t left = p.N - row0;          // rows of the block that exist
  if (valid && span * kSpan + c * (kSpan / CPR) < p.K) {
    const uint8_t* src = p.rows + (row0 + sub) * p.rs + static_cast<int64_t>(span) * F::kSpanBytes + 16 * c;
    const uint32_t dst = st + sub * F::kSpanBytes + 16 * c;
#pragma unroll
    for (int r0 = 0; r0 < R; r0 += RPI)
      if (r0 + sub < R && r0 + sub < left)
        cp_async16(dst + r0 * F::kSpanBytes, src + r0 * p.rs);
  }
  if constexpr (!PLAIN) {
    const int g = lane >> 2, t = lane & 3;
    const int blk = 4 * span + (g >> 1);   // the block of the quad's two groups
    if (valid && t == (g >> 1) && blk < p.K / 128) {
      const uint8_t* src = p.srows + row0 * p.srs + scale_word_offset<FMT>(p.k0, blk, g);
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < left) cp_async4(st + G::kScaleOff + (r * 8 + g) * 4, src + r * p.srs);
    }
  }
}

// Sum v[i] over the 32 lanes for V = R * MR values at once: each step halves the values a lane
// carries (the lanes of one half keep the upper half of the indices, their partners the lower)
// until one is left, then the lanes that share it finish with plain butterflies. Value i's sum
// ends in lanes i * 32/V .. (i + 1) * 32/V - 1.
template <int V>
__device__ __forceinline__ long long transpose_reduce(long long (&v)[V], int lane) {
  int o = 16;
#pragma unroll
  for (int n = V; n > 1; n >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const long long send = upper ? v[i] : v[i + n / 2];
      const long long keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
    }
  }
  long long s = v[0];
#pragma unroll
  for (; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  return s;
}

// One lane's registers for one span of R rows: the weight words, and (MX rows) the scale data
// of the lane's quad: int8 the block's dw byte, int4 / fp4 the block's word, nvfp4 the quad's
// four sub-block bytes.
template <int FMT, int R, bool PLAIN>
struct RSlot {
  uint32_t w[R][RF<FMT>::kLaneWords];
  uint32_t sc[PLAIN ? 1 : R];
};

template <int FMT, int R, bool PLAIN>
__device__ __forceinline__ void rows_read(RSlot<FMT, R, PLAIN>& sl, const uint8_t* st, int k0,
                                          int span, int lane) {
  using F = RF<FMT>;
  using G = Ring<FMT, R, PLAIN>;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if constexpr (FMT == kFmtInt8) {
      const uint4 v = *reinterpret_cast<const uint4*>(st + r * F::kSpanBytes + 16 * lane);
      sl.w[r][0] = v.x;
      sl.w[r][1] = v.y;
      sl.w[r][2] = v.z;
      sl.w[r][3] = v.w;
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(st + r * F::kSpanBytes + 8 * lane);
      sl.w[r][0] = v.x;
      sl.w[r][1] = v.y;
    }
  }
  if constexpr (!PLAIN) {
    const int g = lane >> 2;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint32_t v = *reinterpret_cast<const uint32_t*>(st + G::kScaleOff + (r * 8 + g) * 4);
      if constexpr (FMT == kFmtInt8) v = (v >> (8 * ((4 + k0 + 4 * span + (g >> 1)) & 3))) & 0xFFu;
      sl.sc[r] = v;
    }
  }
}

template <int FMT>
__device__ __forceinline__ void unpack(uint32_t w, uint32_t& lo, uint32_t& hi) {
  if constexpr (FMT == kFmtInt4) {
    int4_bytes(w, lo, hi);
  } else {
    fp4_bytes(w, lo, hi);
  }
}

// acc[r][j] += the exact contribution of this span (lane (g, g/2) of each quad holds it; the
// other lanes' accumulators are ignored).
template <int FMT, int MR, int R, bool PLAIN>
__device__ __forceinline__ void rows_span(const RSmem& s, int KS, int span, int lane,
                                          const RSlot<FMT, R, PLAIN>& sl, long long (&acc)[R][MR]) {
  const int g = lane >> 2, t = lane & 3;
  const bool odd = (g & 1) != 0;
  const bool lo = t < 2;
#pragma unroll
  for (int j = 0; j < MR; ++j) {
    const uint4 xv = *reinterpret_cast<const uint4*>(s.act + static_cast<size_t>(j) * KS * kSpan +
                                                     span * kSpan + 16 * lane);
    const int4 tv = s.terms[static_cast<size_t>(j) * KS * 8 + span * 8 + g];
    if constexpr (FMT != kFmtNvfp4) {
      const uint32_t a0 = lo ? xv.x : 0u, a1 = lo ? 0u : xv.x;
      const uint32_t a2 = lo ? xv.y : 0u, a3 = lo ? 0u : xv.y;
      const uint32_t e0 = lo ? xv.z : 0u, e1 = lo ? 0u : xv.z;
      const uint32_t e2 = lo ? xv.w : 0u, e3 = lo ? 0u : xv.w;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        uint32_t b0, b1, b2, b3;
        if constexpr (FMT == kFmtInt8) {
          b0 = sl.w[r][0];
          b1 = sl.w[r][1];
          b2 = sl.w[r][2];
          b3 = sl.w[r][3];
        } else {
          unpack<FMT>(sl.w[r][0], b0, b1);
          unpack<FMT>(sl.w[r][1], b2, b3);
        }
        int d[4] = {0, 0, 0, 0};
        imma_acc(a0, a1, a2, a3, b0, b1, d);
        imma_acc(e0, e1, e2, e3, b2, b3, d);
        int cA = odd ? d[1] : d[0];
        int cB = odd ? d[3] : d[2];
        if constexpr (FMT == kFmtInt4) {
          cA -= tv.y;
          cB -= tv.w;
        }
        int mA, mB;
        if constexpr (PLAIN) {
          mA = tv.x;
          mB = tv.z;
        } else if constexpr (FMT == kFmtInt8) {
          // dw is a byte; x < 2^17, so any shift of 17 or more gives 0 (clamped below 32)
          const int dw = min(static_cast<int>(sl.sc[r]), 31);
          mA = tv.x >> dw;
          mB = tv.z >> dw;
        } else {
          const uint32_t w = sl.sc[r];
          const int dw = static_cast<int>(w & 0xFFu);
          const int sub = odd ? 2 : 0;   // the groups' positions in their block
          mA = shifted(static_cast<int>((w >> (8 + 6 * sub)) & 63u), tv.x, dw);
          mB = shifted(static_cast<int>((w >> (14 + 6 * sub)) & 63u), tv.z, dw);
        }
        acc[r][j] += static_cast<long long>(cA) * mA + static_cast<long long>(cB) * mB;
      }
    } else {
      // set a: lane t = 0 -> row g, t = 2 -> row g + 8; set b: t = 1 -> row g, t = 3 -> row g + 8
      const bool sa = (t & 1) == 0;
      const uint32_t pa0 = (sa && lo) ? xv.x : 0u, pa1 = (sa && !lo) ? xv.x : 0u;
      const uint32_t pa2 = (sa && lo) ? xv.y : 0u, pa3 = (sa && !lo) ? xv.y : 0u;
      const uint32_t qa0 = (sa && lo) ? xv.z : 0u, qa1 = (sa && !lo) ? xv.z : 0u;
      const uint32_t qa2 = (sa && lo) ? xv.w : 0u, qa3 = (sa && !lo) ? xv.w : 0u;
      const uint32_t pb0 = (!sa && lo) ? xv.x : 0u, pb1 = (!sa && !lo) ? xv.x : 0u;
      const uint32_t pb2 = (!sa && lo) ? xv.y : 0u, pb3 = (!sa && !lo) ? xv.y : 0u;
      const uint32_t qb0 = (!sa && lo) ? xv.z : 0u, qb1 = (!sa && !lo) ? xv.z : 0u;
      const uint32_t qb2 = (!sa && lo) ? xv.w : 0u, qb3 = (!sa && !lo) ? xv.w : 0u;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        uint32_t b0, b1, b2, b3;
        fp4_bytes(sl.w[r][0], b0, b1);
        fp4_bytes(sl.w[r][1], b2, b3);
        int da_[4] = {0, 0, 0, 0}, db_[4] = {0, 0, 0, 0};
        imma_acc(pa0, pa1, pa2, pa3, b0, b1, da_);
        imma_acc(qa0, qa1, qa2, qa3, b2, b3, da_);
        imma_acc(pb0, pb1, pb2, pb3, b0, b1, db_);
        imma_acc(qb0, qb1, qb2, qb3, b2, b3, db_);
        // sub-blocks: t = 0 (group A, scale byte 0), 1 (A, byte 1), 2 (B, byte 2), 3 (B, byte 3)
        const int c0 = odd ? da_[1] : da_[0], c2 = odd ? da_[3] : da_[2];
        const int c1 = odd ? db_[1] : db_[0], c3 = odd ? db_[3] : db_[2];
        int m0 = tv.x, m1 = tv.x, m2 = tv.z, m3 = tv.z;
        if constexpr (!PLAIN) {
          const uint32_t w = sl.sc[r];
          int mm, dw;
          e4m3_term(w & 0xFFu, mm, dw);
          m0 = shifted(mm, tv.x, dw);
          e4m3_term((w >> 8) & 0xFFu, mm, dw);
          m1 = shifted(mm, tv.x, dw);
          e4m3_term((w >> 16) & 0xFFu, mm, dw);
          m2 = shifted(mm, tv.z, dw);
          e4m3_term(w >> 24, mm, dw);
          m3 = shifted(mm, tv.z, dw);
        }
        acc[r][j] += static_cast<long long>(c0) * m0 + static_cast<long long>(c1) * m1 +
                     static_cast<long long>(c2) * m2 + static_cast<long long>(c3) * m3;
      }
    }
  }
}

template <int FMT, int MR, int R, int S, int NS, bool PLAIN, int MINB = 2>
__global__ void __launch_bounds__(kThreads, MINB) mm_rows_kernel(const MMParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using F = RF<FMT>;
  using G = Ring<FMT, R, PLAIN>;
  constexpr int TPC = kWarps / S;   // row blocks per CTA iteration
  const int K = p.K;
  const int KS = (K + kSpan - 1) / kSpan;
  RSmem s = rows_carve(smem_raw, MR, R, K, p.x != nullptr, G::kSlotBytes, NS);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int slice = warp % S, bw = warp / S;
  const int s0 = (KS * slice) / S, s1 = (KS * (slice + 1)) / S;   // this warp's spans
  const int NSL = s1 - s0;
  const int NIT = (KS + S - 1) / S;   // items per row block: the same in every warp of the CTA
  const bool unit = (p.flags & kMmUnit) != 0;
  const int64_t NB = (p.N + R - 1) / R;
  const int64_t cstride = static_cast<int64_t>(gridDim.x) * TPC;
  const int64_t cb0 = static_cast<int64_t>(blockIdx.x) * TPC;   // this CTA's first row block
  uint8_t* const ring = s.ring + warp * NS * G::kSlotBytes;
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));

  // The weights never depend on the kernel launched before this one: pull this warp's first rows
  // (its span slice) into L2 before waiting for that kernel (programmatic dependent launch).
  {
    const int64_t row = (cb0 + bw) * R + lane;
    const int64_t used = FMT == kFmtInt8 ? K : K / 2;
    const int64_t off = static_cast<int64_t>(s0) * F::kSpanBytes;
    const int64_t len = min(static_cast<int64_t>(NSL) * F::kSpanBytes, used - off);
    if (lane < R && cb0 + bw < NB && row < p.N && len > 0)
      prefetch_l2(p.rows + row * p.rs + off, static_cast<uint32_t>(len));
  }
  pdl_wait();   // the activations may come from the kernel launched before this one

  for (int m0 = 0; m0 < p.M; m0 += MR) {
    const int mt = min(MR, p.M - m0);
    // Item (it, k): CTA iteration it (row block cb0 + it * cstride + bw), span s0 + k; items go
    // through the warp's ring in order, NS - 1 of them in flight ahead of the one computed.
    int64_t iti = 0;   // the next item to issue
    int ki = 0;
    auto issue_next = [&](int slot) {
      const bool valid = cb0 + iti * cstride < NB && ki < NSL;
      rows_issue<FMT, R, PLAIN>(ring_s + slot * G::kSlotBytes, p, (cb0 + iti * cstride + bw) * R,
                                s0 + ki, lane, valid);
      cp_async_commit();
      if (++ki == NIT) {
        ki = 0;
        ++iti;
      }
    };
#pragma unroll
    for (int q = 0; q < NS - 1; ++q) issue_next(q);   // the weights do not wait for QACT
    rows_load_activations<FMT, MR, PLAIN>(p, s, m0, mt, KS);
    if (m0 + mt >= p.M) pdl_launch();

    long long acc[R][MR];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < MR; ++j) acc[r][j] = 0;
    int64_t it = 0;
    int k = 0;
    int slot = 0;
    bool active = cb0 < NB;
    while (active) {
      __syncwarp();   // every lane is done with the stage that the next issue overwrites
      issue_next(slot == 0 ? NS - 1 : slot - 1);
      cp_async_wait<NS - 1>();   // this lane's copies of item (it, k) have landed
      __syncwarp();              // ... and every other lane's
      if (k < NSL) {
        RSlot<FMT, R, PLAIN> cur;
        rows_read<FMT, R, PLAIN>(cur, ring + slot * G::kSlotBytes, p.k0, s0 + k, lane);
        rows_span<FMT, MR, R, PLAIN>(s, KS, s0 + k, lane, cur, acc);
      }
      if (k == NIT - 1) {
        // the row block is complete: sum the useful lanes, then the S warps of the block
        constexpr int V = R * MR;
        constexpr int LPV = 32 / V;   // lanes that end up holding each value
        const bool useful = t == (g >> 1);
        long long v[V];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int j = 0; j < MR; ++j) {
            v[r * MR + j] = useful ? acc[r][j] : 0;
            acc[r][j] = 0;
          }
        long long mine = transpose_reduce<V>(v, lane);
        const int idx = lane / LPV;
        const bool owner = lane % LPV == 0;
        if constexpr (S > 1) {
          if (owner) s.red[warp * V + idx] = mine;
          __syncthreads();
          if (slice == 0 && owner)
            for (int o = 1; o < S; ++o) mine += s.red[(warp + o) * V + idx];
        }
        const int64_t rb = cb0 + it * cstride + bw;
        if (slice == 0 && owner && rb < NB) {
          const int r = idx / MR, j = idx % MR;
          const int64_t row = rb * R + r;
          if (row < p.N && j < mt) {
            const float Sw = unit ? 1.0f : __ldg(reinterpret_cast<const float*>(p.srows + row * p.srs));
            float yv = mm_epilogue(mine, Sw, s.Sa[j], F::kW);
            float* yp = p.y + static_cast<int64_t>(m0 + j) * p.ldy + row;
            if (p.flags & kMmAscale) {
              yv = fadd(fmul(*yp, __ldg(p.alpha + m0 + j)), yv);
            } else if (p.flags & kMmAcc) {
              yv = fadd(*yp, yv);
            }
            *yp = yv;
          }
        }
        if constexpr (S > 1) __syncthreads();   // red is reused by the next row block
      }
      slot = slot == NS - 1 ? 0 : slot + 1;
      if (++k == NIT) {
        k = 0;
        ++it;
        active = cb0 + it * cstride < NB;
      }
    }
    cp_async_wait<0>();
    __syncthreads();   // the next activation rows and ring contents overwrite shared memory
  }
}

template <int FMT, int MR, int R, int S, int NS, bool PLAIN, int MINB = 2>
int rows_cfg(const MMParams& p, cudaStream_t stream, bool pdl) {
  const size_t smem =
      rows_layout(MR, R, p.K, p.x != nullptr, Ring<FMT, R, PLAIN>::kSlotBytes, NS, nullptr);
  auto kern = mm_rows_kernel<FMT, MR, R, S, NS, PLAIN, MINB>;
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
  const int64_t nb = (p.N + R - 1) / R;
  const int64_t ctas_needed = (nb + TPC - 1) / TPC;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * occ;
  const int64_t iters = (ctas_needed + cap - 1) / cap;
  const int64_t grid = (ctas_needed + iters - 1) / iters;
  return launch_kernel(reinterpret_cast<const void*>(kern), static_cast<int>(grid), kThreads, smem,
                       stream, pdl, p);
}

// R rows per warp: 8 (4 for two activation rows) for tall matrices, the activation fragments
// shared by all of them; 1 with a span split for short ones.
template <int FMT, int MR, bool PLAIN>
int rows_split(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  // four-row rings that do not fit beside a long activation row: one-row rings, spans split
  constexpr int RT = MR == 1 ? 8 : 4;   // rows a warp for tall matrices
  if (split == 1 && rows_layout(MR, RT, p.K, p.x != nullptr, Ring<FMT, RT, PLAIN>::kSlotBytes, 3,
                                nullptr) > 227 * 1024)
    split = 2;
  switch (split) {   // ring stages: 3 of RT rows, 8 of one
    case 101: return rows_cfg<FMT, MR, 4, 1, 3, PLAIN, 4>(p, stream, pdl);
    case 102: return rows_cfg<FMT, MR, 4, 1, 4, PLAIN, 3>(p, stream, pdl);
    case 103: return rows_cfg<FMT, MR, 2, 1, 4, PLAIN, 4>(p, stream, pdl);
    case 104: return rows_cfg<FMT, MR, 8, 1, 4, PLAIN, 1>(p, stream, pdl);
    case 105: return rows_cfg<FMT, MR, 4, 1, 6, PLAIN, 2>(p, stream, pdl);
    case 106: return rows_cfg<FMT, MR, 2, 1, 8, PLAIN, 3>(p, stream, pdl);
    case 1: return rows_cfg<FMT, MR, RT, 1, 3, PLAIN>(p, stream, pdl);
    case 2: return rows_cfg<FMT, MR, 1, 2, 8, PLAIN>(p, stream, pdl);
    case 4: return rows_cfg<FMT, MR, 1, 4, 8, PLAIN>(p, stream, pdl);
    default: return rows_cfg<FMT, MR, 1, 8, 8, PLAIN>(p, stream, pdl);
  }
}

template <int FMT, int MR>
int rows_plain(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  if (p.flags & (kMmUnit | kMmRsc)) return rows_split<FMT, MR, true>(p, stream, pdl, split);
  return rows_split<FMT, MR, false>(p, stream, pdl, split);
}

template <int FMT>
int rows_fmt(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  if (p.M <= 1) return rows_plain<FMT, 1>(p, stream, pdl, split);
  return rows_plain<FMT, 2>(p, stream, pdl, split);
}

}  // namespace

size_t rows_smem_bytes(int mr, int K, bool fused) {
  // the smallest configuration: one-row rings of int8 spans with scale words, 8 stages
  return rows_layout(mr, 1, K, fused, Ring<kFmtInt8, 1, false>::kSlotBytes, 8, nullptr);
}

// Span split: 1 (eight rows a warp) while the matrix has enough rows to give every SM sixteen
// warps; else as many warps per row as keep the SMs busy, each with at least one span.
int rows_pick_split(int64_t N, int K, int dev) {
  const int64_t want_warps = static_cast<int64_t>(sm_count(dev)) * 16;
  if ((N + 7) / 8 >= want_warps) return 1;
  const int KS = (K + kSpan - 1) / kSpan;
  int split = 2;
  while (split < 8 && N * split < want_warps && KS / (split * 2) >= 1) split *= 2;
  return split;
}

int mm_rows_launch(const MMParams& p, cudaStream_t stream, bool pdl, int split) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  if (split == 0) split = rows_pick_split(p.N, p.K, dev);
  switch (p.fmt) {
    case kFmtInt8: return rows_fmt<kFmtInt8>(p, stream, pdl, split);
    case kFmtInt4: return rows_fmt<kFmtInt4>(p, stream, pdl, split);
    case kFmtFp4: return rows_fmt<kFmtFp4>(p, stream, pdl, split);
    case kFmtNvfp4: return rows_fmt<kFmtNvfp4>(p, stream, pdl, split);
    default: return kErrFormat;
  }
}

}  // namespace otq
