// MM for decode (up to 8 activation rows a pass): the weight-streaming GEMV over openTPU's MX
// formats, with exact integer accumulation (reference docs/isa.md "MM";
// opentpu/isasim.py:749-910; scalar model tests/test_mx.py:131-151).
//
//   acc = sum over 32-element groups of (m << sh) * c,  c = the group's exact int dot product,
//         sh = W - dw - da (the group is dropped where sh < 0)
//   y   = (i2f(acc) * Sw[n]) * (Sa[j] * 2^-W)      -- otq_fp32.cuh mm_epilogue
//
// Streaming. Each warp owns a contiguous range of weight rows (ranges balanced by rows) and walks
// it in blocks of R rows, one 128-byte chunk of K at a time. A chunk of the block's rows moves
// into one stage of the warp's ring of NS shared-memory stages by 2-D tensor copies (the TMA
// engine, one instruction for 8 rows x 128 bytes, 128-byte swizzle so that the 8-row fragment
// reads below are free of bank conflicts), completing on the stage's mbarrier; NS - 1 chunks stay
// in flight while one is computed. The first stages are issued before griddepcontrol.wait:
// weights never depend on the kernel launched before this one. MX scale data (a few bytes a row
// and chunk) comes with cp.async. Every mbarrier wait is bounded (mm_common.cuh).
//
// Dot products: one mma.sync m16n8k32 (s8 x s8 -> s32) takes one 32-element group of 8 weight
// rows (B, one row a column: lane (g, t) supplies row g's bytes [8t, 8t+8) of the group) against
// 16 rows of A. 4-bit elements are decoded in registers to exact bytes (int4 as 16x its value, so
// no bias term is needed; E2M1 doubled).
//
// Class path (RSC / UNIT rows, one activation row, every group's offset representable): a
// group's multiplier 2^(W - da) depends on the activation alone, so A row c carries the bytes of
// the groups whose offset da is c (zeros elsewhere) and the MMA accumulates every group of a row
// exactly in int32 (|sum| < 2^31 for K <= 32640). The A fragments are built once per CTA. At the
// end of a row block each class is scaled once by 2^(W - c) into int64 and the 8 class rows are
// summed across lanes. Groups below the window (sh < 0) are in no class: they are dropped.
//
// General path (MX rows with per-block weight offsets, several activation rows, or an int8 row
// whose offset 16 has no class row): A row j is activation row j; each group's int32 result is
// scaled by its own multiplier (m << sh) into int64 accumulators, one per (activation row,
// weight row) and lane, so no cross-lane reduction is needed.
//
// Rows with few outputs split K: S warps of a CTA take the same rows, each a range of chunks,
// and add their int64 partials through shared memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>

#include "mm_common.cuh"
#include "otq_fp32.cuh"
#include "otq_internal.h"
#include "qact.cuh"

namespace otq {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 128;   // bytes of a weight row in one stage
constexpr int kBox = 8;       // rows of one tensor copy (8 x 128 bytes: one swizzle atom)
constexpr int kActPad = 16;   // activation row pitch = K (padded) + 16: conflict-free 8-row reads

template <int FMT>
struct GF {
  static constexpr int kW = (FMT == kFmtInt8) ? 16 : (FMT == kFmtNvfp4 ? 13 : 11);
  static constexpr int kElems = (FMT == kFmtInt8) ? 128 : 256;   // elements of a chunk
  static constexpr int kGroups = kElems / 32;
};

// A stage: R rows x 128 bytes (1024-byte aligned, 128-byte swizzle), and (MX rows) a scale stage
// of 16 bytes a row.
template <int R, bool PLAIN>
struct Stage {
  static constexpr int kBytes = R * kChunk;
  static constexpr int kScaleBytes = PLAIN ? 0 : R * 16;
};

struct GSmem {
  uint8_t* act;      // [MT][ap] activation bytes (int4: each run of 8 as evens, then odds)
  int* term;         // [KG][MT] general path: a group's activation-side term (group_term)
  uint8_t* cls;      // [KG] class path: the group's class (its offset), 255 = dropped
  uint4* afrag;      // [KG][32] class path: each lane's A fragment of each group
  float* Sa;         // [MT]
  int* flag;         // [1] 1: some group of activation row 0 has no class
  long long* red;    // [kWarps][32][VPL] K-split partials
  float* xs;         // [K] the fp32 row being quantized (fused QACT)
  uint32_t* seg;     // [K / 32]
  uint32_t* qred;    // [40]
  uint64_t* bar;     // [kWarps][NS] stage barriers
  uint8_t* sring;    // [kWarps][NS][scale stage]
  uint8_t* ring;     // [kWarps][NS][stage], 1024-byte aligned
};

struct GLayout {
  int MT, K, ap, vpl, S, stage_bytes, scale_bytes, ns;
  bool fused, frag;
};

// Work decompositions of a projection: 32-row blocks, or 8-row blocks with S warps sharing a
// row's K (S = 1, 2, 4, 8).
enum { kCfgR32 = 0, kCfgS1 = 1, kCfgS2 = 2, kCfgS4 = 3, kCfgS8 = 4 };

// One projection (QACT + MM) of a launch: its operands and the tensor map of its weight rows.
struct alignas(64) Proj {
  CUtensorMap map;
  const uint8_t* rows;   // what the map describes (for L2 prefetches)
  const uint8_t* srows;
  const float* x;        // fp32 activations (QACT in the kernel), or null: q / Sa / da given
  float* y;
  const float* alpha;
  const int8_t* q;
  const float* Sa;
  const uint8_t* da;
  int64_t N;
  int rs, srs, ldx, ldy, ldq, ldd;   // strides (the entry points keep them below 2^31)
  int K, flags, k0, row_mode, M, cfg;
};
static_assert(sizeof(Proj) == 256, "a projection is 256 bytes of kernel parameters");

// A projection's scalars, copied out of the kernel parameters once per projection (reads
// through a pointer into parameter space cost a memory round trip each); map stays the
// address of the tensor map in parameter space, which is what a tensor copy takes.
struct PArgs {
  const CUtensorMap* map;
  const uint8_t* rows;
  const uint8_t* srows;
  const float* x;
  float* y;
  const float* alpha;
  const int8_t* q;
  const float* Sa;
  const uint8_t* da;
  int64_t N;
  int rs, srs, ldx, ldy, ldq, ldd;
  int K, flags, k0, row_mode, M, cfg;
};

__device__ __forceinline__ PArgs load_args(const Proj& d) {
  PArgs a;
  a.map = &d.map;
  a.rows = d.rows;
  a.srows = d.srows;
  a.x = d.x;
  a.y = d.y;
  a.alpha = d.alpha;
  a.q = d.q;
  a.Sa = d.Sa;
  a.da = d.da;
  a.N = d.N;
  a.rs = d.rs;
  a.srs = d.srs;
  a.ldx = d.ldx;
  a.ldy = d.ldy;
  a.ldq = d.ldq;
  a.ldd = d.ldd;
  a.K = d.K;
  a.flags = d.flags;
  a.k0 = d.k0;
  a.row_mode = d.row_mode;
  a.M = d.M;
  a.cfg = d.cfg;
  return a;
}

// The projections of one launch, run in order; from the second on, each starts after a grid
// barrier (its x may be an earlier projection's y).
// A row-sharded projection's output fan-out over NVLink (world > 0, single-projection launches).
// Output rows are tagged: element i is one 8-byte word, the fp32 value in the low half and a tag
// in the high half, stored single-copy atomically. The rank that owns a row stores its word into
// every rank's copy of the output row (symmetric buffers, delta[r] bytes from this rank's) with
// tag = this rank's projection count + 1; a launch whose x is such a row (wait != 0) reads each
// element until its tag has reached this rank's count, so it starts on every rank's previous
// output without a fence or a flag. The launch's last CTA advances the count (device scope).
constexpr int kMaxPeers = 8;
struct PeerArgs {
  int rank, world, wait, tags;
  int64_t delta[kMaxPeers];
  int* seq;     // counted tags: launches this rank has completed; stepped: steps completed
  int* done;    // CTAs of the current launch that have finished (zero between launches)
  int step_pos, step_last;
};

constexpr uint32_t kStepTags = 1024;   // stepped tags: s * 1024 + position + 1

template <int MAXP>
struct Chain {
  Proj proj[MAXP];
  int count;
  int* status;
  PeerArgs peer;
};

struct Fan {
  int world, rank;
  uint32_t tag;            // 0: plain fp32 output; else the tag of this launch's output words
  const int64_t* delta;    // shared-memory copy of PeerArgs::delta
};

__device__ __forceinline__ void st_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Output element idx of y: a plain store, or the tagged word here and on every other rank.
__device__ __forceinline__ void put_out(float* y, int64_t idx, float v, const Fan& fan) {
  if (fan.tag == 0) {
    y[idx] = v;
    return;
  }
  const unsigned long long w = __float_as_uint(v) | (static_cast<unsigned long long>(fan.tag) << 32);
  unsigned long long* p = reinterpret_cast<unsigned long long*>(y) + idx;
  st_sys_u64(p, w);
  for (int r = 0; r < fan.world; ++r)
    if (r != fan.rank)
      st_sys_u64(reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(p) + fan.delta[r]), w);
}

// A warp's share of one projection: rows [rb, re) in NBLK blocks of R, chunks [c0, c0 + NSL)
// of each (NIT items a block, the same in every warp of the CTA).
struct Geo {
  int R, S, c0, NSL, NIT, NBLK, total;
  int64_t rb, re;
};

__host__ __device__ inline size_t gemv_layout(const GLayout& L, size_t* offs) {
  const size_t KG = L.K / 32;
  size_t off = 0;
  auto take = [&](int i, size_t bytes) {
    off = (off + 15) & ~size_t(15);
    if (offs) offs[i] = off;
    off += bytes;
  };
  take(0, static_cast<size_t>(L.MT) * L.ap);
  take(1, static_cast<size_t>(L.MT) * KG * 4);
  take(2, KG);
  take(3, L.frag ? KG * 32 * 16 : 0);
  take(4, L.MT * 4);
  take(5, 16);
  take(6, L.S > 1 ? static_cast<size_t>(kWarps) * 32 * L.vpl * 8 : 0);
  take(7, L.fused ? static_cast<size_t>(L.K) * 4 : 0);
  take(8, KG * 4);
  take(9, 40 * 4);
  take(10, static_cast<size_t>(kWarps) * L.ns * 8);
  take(11, static_cast<size_t>(kWarps) * L.ns * L.scale_bytes);
  take(12, static_cast<size_t>(kWarps) * L.ns * L.stage_bytes + 1024);   // + alignment slack
  return off;
}

__device__ __forceinline__ GSmem gemv_carve(unsigned char* base, const GLayout& L) {
  size_t o[13];
  gemv_layout(L, o);
  GSmem s;
  s.act = base + o[0];
  s.term = reinterpret_cast<int*>(base + o[1]);
  s.cls = base + o[2];
  s.afrag = reinterpret_cast<uint4*>(base + o[3]);
  s.Sa = reinterpret_cast<float*>(base + o[4]);
  s.flag = reinterpret_cast<int*>(base + o[5]);
  s.red = reinterpret_cast<long long*>(base + o[6]);
  s.xs = reinterpret_cast<float*>(base + o[7]);
  s.seg = reinterpret_cast<uint32_t*>(base + o[8]);
  s.qred = reinterpret_cast<uint32_t*>(base + o[9]);
  s.bar = reinterpret_cast<uint64_t*>(base + o[10]);
  s.sring = base + o[11];
  const uint32_t r = smem_addr(base + o[12]);
  s.ring = base + o[12] + (((r + 1023u) & ~1023u) - r);
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

// Class path: a group's class (its offset), or 255 where it has none: above W it is below the
// window (dropped); the int8 offset 16 (multiplier 1) has no class row.
template <int FMT>
__device__ __forceinline__ int class_of(int da) {
  return (da <= GF<FMT>::kW && da < 16) ? da : 255;
}

template <int FMT, int MT, bool PLAIN>
__device__ __forceinline__ void put_group(const GSmem& s, int j, int G, int da) {
  s.term[G * MT + j] = group_term<FMT, PLAIN>(da);
  if (j == 0) {
    if (da == 16 && FMT == kFmtInt8) *s.flag = 1;
    s.cls[G] = static_cast<uint8_t>(class_of<FMT>(da));
  }
}

// The zeros the activation rows start from: bytes past K, rows mt..MT-1, the class flag and
// (QACT of fp32 x on the class path) the A fragments. Touches shared memory only, so a launch
// runs it before griddepcontrol.wait. Ends with a barrier.
template <int FMT, int MT, bool PLAIN>
__device__ __forceinline__ void gemv_clear_activations(const PArgs& p, const GSmem& s, int mt, int kp,
                                                       int ap, bool frag) {
  const int K = p.K, KG = K / 32;
  if (threadIdx.x == 0) *s.flag = 0;
  for (int j = 0; j < MT; ++j) {
    const int from = j < mt ? K : 0;
    uint32_t* aw = reinterpret_cast<uint32_t*>(s.act + static_cast<size_t>(j) * ap);
    for (int i = (from >> 2) + threadIdx.x; i < (kp >> 2); i += kThreads) aw[i] = 0u;
    if (j >= mt)
      for (int G = threadIdx.x; G < KG; G += kThreads) s.term[G * MT + j] = 0;
  }
  if (threadIdx.x < MT && static_cast<int>(threadIdx.x) >= mt) s.Sa[threadIdx.x] = 0.0f;
  if (p.x != nullptr && frag)
    for (int i = threadIdx.x; i < KG * 32; i += kThreads) s.afrag[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();   // flag and fragments cleared before any group can set them
}

// Activation rows [m0, m0 + mt) into shared memory (QACT of fp32 x, or copied bytes). Bytes past
// K, and rows mt..MT-1, are zeros. With `frag`, the class path's A fragments as well. cleared:
// gemv_clear_activations already ran for this projection.
template <int FMT, int MT, bool PLAIN>
__device__ __forceinline__ void gemv_load_activations(const PArgs& p, const GSmem& s, int mt, int kp, int ap,
                                      bool frag, bool cleared, bool tagged = false, uint32_t expect = 0,
                                      int* status = nullptr, uint32_t limit = 1u << 22) {
  const int K = p.K, KG = K / 32;
  if (!cleared) gemv_clear_activations<FMT, MT, PLAIN>(p, s, mt, kp, ap, frag);
  if (p.x != nullptr) {
    for (int j = 0; j < mt; ++j) {
      const float* xr = p.x + static_cast<int64_t>(j) * p.ldx;
      const bool x4 = (reinterpret_cast<uintptr_t>(xr) & 15u) == 0;
      uint8_t* arow = s.act + static_cast<size_t>(j) * ap;
      qact_row4<kThreads>(
          xr, x4, s.xs, K, p.row_mode != 0, s.seg, s.qred,
          [&](int i, int q0, int q1, int q2, int q3, int d) {
            const int G = i >> 3;
            if ((threadIdx.x & 7) == 0) put_group<FMT, MT, PLAIN>(s, j, G, d);
            const uint32_t packed = (q0 & 0xFFu) | ((q1 & 0xFFu) << 8) | ((q2 & 0xFFu) << 16) |
                                    (static_cast<uint32_t>(q3 & 0xFF) << 24);
            const int c = class_of<FMT>(d);
            // lane (g, t) of the group holds its bytes [8t, 8t+8) in A row g (class g) or g + 8
            uint8_t* fb = reinterpret_cast<uint8_t*>(s.afrag + G * 32);
            const int cg = 4 * (c & 7), ch = c >= 8 ? 4 : 0;
            if constexpr (FMT == kFmtInt4) {
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int pos = act_pos<FMT>(4 * i + k);
                const uint8_t b = static_cast<uint8_t>((packed >> (8 * k)) & 0xFFu);
                arow[pos] = b;
                if (frag && j == 0 && c != 255) {
                  const int e = pos & 31;
                  fb[(cg + (e >> 3)) * 16 + ((e & 7) >= 4 ? 8 : 0) + ch + (e & 3)] = b;
                }
              }
            } else {
              *reinterpret_cast<uint32_t*>(arow + 4 * i) = packed;
              if (frag && j == 0 && c != 255) {
                const int e = (4 * i) & 31;   // a whole aligned word of lane t = e / 8
                *reinterpret_cast<uint32_t*>(fb + (cg + (e >> 3)) * 16 + ((e & 7) >= 4 ? 8 : 0) + ch) = packed;
              }
            }
          },
          tagged ? reinterpret_cast<const unsigned long long*>(xr) : nullptr, expect, status,
          s.Sa + j, limit);
    }
    return;   // qact_row4 ends with a barrier, after every write above (Sa included)
  } else {
    for (int j = 0; j < mt; ++j) {
      const int8_t* qr = p.q + static_cast<int64_t>(j) * p.ldq;
      const uint8_t* dr = p.da + static_cast<int64_t>(j) * p.ldd;
      uint8_t* arow = s.act + static_cast<size_t>(j) * ap;
      for (int i = threadIdx.x; i < K; i += kThreads)
        arow[act_pos<FMT>(i)] = static_cast<uint8_t>(__ldcg(qr + i));
      for (int G = threadIdx.x; G < KG; G += kThreads) put_group<FMT, MT, PLAIN>(s, j, G, __ldcg(dr + G));
      if (threadIdx.x == 0) s.Sa[j] = __ldcg(p.Sa + j);
    }
  }
  __syncthreads();
  if (frag && p.x == nullptr) {
    // lane (g, t) of group G: the 8 bytes it holds of the group in row g (class g) or row g + 8
    for (int i = threadIdx.x; i < KG * 32; i += kThreads) {
      const int G = i >> 5, lane = i & 31, g = lane >> 2, t = lane & 3;
      const uint2 q = *reinterpret_cast<const uint2*>(s.act + 32 * G + 8 * t);
      const int c = s.cls[G];
      uint4 a;
      a.x = c == g ? q.x : 0u;
      a.y = c == g + 8 ? q.x : 0u;
      a.z = c == g ? q.y : 0u;
      a.w = c == g + 8 ? q.y : 0u;
      s.afrag[i] = a;
    }
    __syncthreads();
  }
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

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Issue chunk kc of rows [row0, row0 + nrows) (0 <= nrows <= R) into a stage (shared address st,
// barrier bar): lane 0 arrives announcing the bytes, then lane j copies the box of rows
// row0 + 8j .. + 7 (rows past the matrix and columns past the row's bytes read as zeros; rows
// of the next worker are loaded and never stored). MX scale data goes by cp.async into the scale
// stage sst, one commit group per issue.
template <int FMT, bool PLAIN>
__device__ __forceinline__ void gemv_issue(uint32_t st, uint32_t sst, uint32_t bar, const PArgs& p,
                                           int64_t row0, int nrows, int kc, int lane, int bh) {
  // bh: rows of the map's box. Launches use 8: a warp's partial last block then reads no rows
  // past its range (a 32-row box needs a quarter of the issues but reads up to 31 rows of the
  // next warp's range from DRAM a second time)
  const int boxes = nrows > 0 ? (nrows + bh - 1) / bh : 0;
  if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(boxes * bh * kChunk));
  __syncwarp();
  if (lane < boxes)
    tma_load_2d(st + lane * bh * kChunk, p.map, kc * kChunk, static_cast<int>(row0) + bh * lane, bar);
  if constexpr (!PLAIN) {
    if (lane < nrows) {
      const uint8_t* srow = p.srows + (row0 + lane) * p.srs;
      const uint32_t dst = sst + lane * 16;
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
    cp_async_commit();
  }
}

// Row g's bytes of group s of a stage for lane (g, t), as the B fragment of one MMA (two for
// nvfp4, whose 16-element sub-blocks are lanes t < 2 and t >= 2).
// row: the row's 128 bytes in a stage, whose 16-byte pieces are swizzled by g (the row's index
// in its 8-row box).
template <int FMT>
__device__ __forceinline__ void b_frag(const uint8_t* row, int s, int g, int t, uint32_t& b0,
                                       uint32_t& b1) {
  if constexpr (FMT == kFmtInt8) {
    const int piece = (2 * s + (t >> 1)) ^ g;
    const uint2 v = *reinterpret_cast<const uint2*>(row + 16 * piece + 8 * (t & 1));
    b0 = v.x;
    b1 = v.y;
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 16 * (s ^ g) + 4 * t);
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

// Scale data of one weight row for one chunk (general path, MX rows), decoded per group.
template <int FMT>
struct RowScale {
  uint32_t w[FMT == kFmtInt8 ? 1 : (FMT == kFmtNvfp4 ? 4 : 2)];
};

template <int FMT>
__device__ __forceinline__ void read_row_scale(RowScale<FMT>& r, const uint8_t* sc, int k0, int kc) {
  if constexpr (FMT == kFmtInt8) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(sc);
    r.w[0] = min((w >> (8 * ((4 + k0 + kc) & 3))) & 0xFFu, 31u);   // dw, clamped below 32
  } else if constexpr (FMT == kFmtNvfp4) {
    const uint4 v = *reinterpret_cast<const uint4*>(sc);
    r.w[0] = v.x;
    r.w[1] = v.y;
    r.w[2] = v.z;
    r.w[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(sc);
    r.w[0] = v.x;
    r.w[1] = v.y;
  }
}

// The multipliers of (weight row, group s of the chunk): ta the activation-side term; m1 is the
// second sub-block's (nvfp4).
template <int FMT, bool PLAIN>
__device__ __forceinline__ void general_mult(const RowScale<FMT>& r, int s, int ta, int& m0, int& m1) {
  if constexpr (PLAIN) {
    m0 = m1 = ta;
  } else if constexpr (FMT == kFmtInt8) {
    m0 = m1 = ta >> r.w[0];   // ta < 2^17: shifts of 17 or more give 0
  } else if constexpr (FMT == kFmtInt4 || FMT == kFmtFp4) {
    const uint32_t w = r.w[s >> 2];
    m0 = m1 = shifted(static_cast<int>((w >> (8 + 6 * (s & 3))) & 63u), ta, static_cast<int>(w & 0xFFu));
  } else {
    const uint32_t e = (r.w[2 * (s >> 2) + ((s & 3) >> 1)] >> (16 * (s & 1))) & 0xFFFFu;
    int mm, dw;
    e4m3_term(e & 0xFFu, mm, dw);
    m0 = shifted(mm, ta, dw);
    e4m3_term(e >> 8, mm, dw);
    m1 = shifted(mm, ta, dw);
  }
}

template <int FMT>
__device__ __forceinline__ Geo geometry(const PArgs& d, int warp) {
  Geo q;
  q.R = d.cfg == kCfgR32 ? 32 : 8;
  q.S = d.cfg <= kCfgS1 ? 1 : (1 << (d.cfg - 1));
  const int KCH = (d.K + GF<FMT>::kElems - 1) / GF<FMT>::kElems;   // chunks a row
  const int slice = warp % q.S;
  q.c0 = (KCH * slice) / q.S;
  q.NSL = (KCH * (slice + 1)) / q.S - q.c0;
  q.NIT = (KCH + q.S - 1) / q.S;
  const int tpc = kWarps / q.S;   // row workers of a CTA
  const int64_t nw = static_cast<int64_t>(gridDim.x) * tpc;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * tpc + warp / q.S;
  q.rb = d.N * w / nw;
  q.re = d.N * (w + 1) / nw;
  const int64_t most = (d.N + nw - 1) / nw;
  q.NBLK = static_cast<int>((most + q.R - 1) / q.R);
  q.total = q.NBLK * q.NIT;
  return q;
}

// Polls a wait on tagged input words makes before it gives up and records kStatusTimeout
// (otq_set_wait_limit); 2^22 by default, about a quarter of a second with the back-off.
__device__ uint32_t g_tag_wait_limit = 1u << 22;

__device__ unsigned int g_bar_count;   // CTAs arrived at the current grid barrier
__device__ unsigned int g_bar_gen;     // grid barriers completed (wraps)

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// All CTAs of the grid (co-resident: cooperative launch) meet; every global write before the
// barrier is visible to every CTA after it. The last CTA to arrive resets the count and bumps
// the generation; the others wait (bounded: after kSpinLimit polls the status word records
// kStatusTimeout and the CTA goes on, so the kernel always ends).
__device__ __forceinline__ void grid_barrier(int* status) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int gen = ld_acquire(&g_bar_gen);
    __threadfence();
    const unsigned int arrived = atomicAdd(&g_bar_count, 1u) + 1u;
    if (arrived == gridDim.x) {
      atomicExch(&g_bar_count, 0u);
      __threadfence();
      atomicAdd(&g_bar_gen, 1u);
    } else {
      uint32_t i = 0;
      while (ld_acquire(&g_bar_gen) == gen) {
        if (++i > kSpinLimit) {
          if (status != nullptr) atomicOr(status, kStatusTimeout);
          break;
        }
        if (i > 32) __nanosleep(32);
      }
    }
    __threadfence();
  }
  __syncthreads();
}

// The warp's weight ring over all projections of the launch: items are issued in order
// (projection, row block, chunk), NS - 1 ahead of the one computed, across projection boundaries
// (weights never depend on activations).
template <int FMT, bool PLAIN, int NS, int MAXP>
struct RingIssue {
  const Chain<MAXP>* C;
  uint32_t ring_s, sring_s, bar0;
  int stage_bytes, scale_bytes, lane, warp;
  int count;
  int p, i, issued;   // next item: projection p, item i of it; items issued so far
  PArgs a;            // projection p
  Geo q;

  __device__ __forceinline__ bool next() {
    while (p < count && i >= q.total) {
      ++p;
      i = 0;
      if (p < count) {
        a = load_args(C->proj[p]);
        q = geometry<FMT>(a, warp);
      }
    }
    if (p >= count) return false;
    const PArgs& d = a;
    const int b = i / q.NIT, k = i % q.NIT;
    const int64_t r0 = q.rb + static_cast<int64_t>(b) * q.R;
    int nrows = static_cast<int>(min(static_cast<int64_t>(q.R), q.re - r0));
    if (k >= q.NSL || nrows < 0) nrows = 0;
    const int st = issued % NS;
    gemv_issue<FMT, PLAIN>(ring_s + st * stage_bytes, sring_s + st * scale_bytes, bar0 + 8 * st, d,
                           r0, nrows, q.c0 + k, lane, kBox);
    ++issued;
    ++i;
    return true;
  }
};

// This warp's items of projection d (geometry q), consumed in order from the ring; f counts the
// items consumed so far (stage f % NS, parity (f / NS) & 1).
template <int FMT, int MT, bool PLAIN, int NS, int MAXP, int R, int S>
__device__ __forceinline__ void run_proj(const PArgs& d, const Geo& q, const GSmem& s,
                                         RingIssue<FMT, PLAIN, NS, MAXP>& iss, int& f, bool& ok,
                                         int* status, const GLayout& L, uint8_t* ring,
                                         uint8_t* sring, int mt, const Fan& fan) {
  using F = GF<FMT>;
  constexpr int NO = R / 8;     // row octets (tensor-copy boxes) of a block
  constexpr int VPL = 2 * NO;   // general-path values a lane
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int slice = warp % S;
  const bool unit = (d.flags & kMmUnit) != 0;
  const bool use_class = MT == 1 && PLAIN && *s.flag == 0;
  const uint32_t bar0 = iss.bar0;

  int D[NO][4];
  long long acc[NO][2];
#pragma unroll
  for (int o = 0; o < NO; ++o) {
#pragma unroll
    for (int i = 0; i < 4; ++i) D[o][i] = 0;
    acc[o][0] = acc[o][1] = 0;
  }
  for (int b = 0; b < q.NBLK; ++b) {
    for (int k = 0; k < q.NIT; ++k, ++f) {
      __syncwarp();   // every lane is done with the stage that the next issue overwrites
      const bool more = iss.next();
      const int stn = f % NS;
      if (!mbar_wait(bar0 + 8 * stn, static_cast<uint32_t>((f / NS) & 1), status)) ok = false;
      if constexpr (!PLAIN) {
        if (more) cp_async_wait<NS - 1>(); else cp_async_wait<0>();
        __syncwarp();
      }
      if (k >= q.NSL || !ok) continue;
      const uint8_t* st = ring + stn * L.stage_bytes;
      const int kc = q.c0 + k;
      if (use_class) {
#pragma unroll
        for (int sg = 0; sg < F::kGroups; ++sg) {
          const int G = kc * F::kGroups + sg;
          uint4 a;
          if (L.frag) {
            a = s.afrag[G * 32 + lane];
          } else {
            const uint2 qv = *reinterpret_cast<const uint2*>(s.act + 32 * G + 8 * t);
            const int c = s.cls[G];
            a.x = c == g ? qv.x : 0u;
            a.y = c == g + 8 ? qv.x : 0u;
            a.z = c == g ? qv.y : 0u;
            a.w = c == g + 8 ? qv.y : 0u;
          }
#pragma unroll
          for (int o = 0; o < NO; ++o) {
            uint32_t b0, b1;
            b_frag<FMT>(st + (8 * o + g) * kChunk, sg, g, t, b0, b1);
            imma_acc(a.x, a.y, a.z, a.w, b0, b1, D[o]);
          }
        }
      } else {
        RowScale<FMT> rsc[NO][2];
        if constexpr (!PLAIN) {
#pragma unroll
          for (int o = 0; o < NO; ++o)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              read_row_scale<FMT>(rsc[o][h], sring + stn * L.scale_bytes + (8 * o + 2 * t + h) * 16, d.k0, kc);
        }
        const int gm = g < MT ? g : 0;
#pragma unroll
        for (int sg = 0; sg < F::kGroups; ++sg) {
          const int G = kc * F::kGroups + sg;
          const uint2 qv = *reinterpret_cast<const uint2*>(s.act + static_cast<size_t>(gm) * L.ap + 32 * G + 8 * t);
          const uint32_t a0 = g < MT ? qv.x : 0u, a2 = g < MT ? qv.y : 0u;
          const int ta = g < MT ? s.term[G * MT + gm] : 0;
#pragma unroll
          for (int o = 0; o < NO; ++o) {
            uint32_t b0, b1;
            b_frag<FMT>(st + (8 * o + g) * kChunk, sg, g, t, b0, b1);
            int dd[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0};
            if constexpr (FMT == kFmtNvfp4) {
              imma_acc(a0, 0u, a2, 0u, t < 2 ? b0 : 0u, t < 2 ? b1 : 0u, dd);
              imma_acc(a0, 0u, a2, 0u, t < 2 ? 0u : b0, t < 2 ? 0u : b1, e);
            } else {
              imma_acc(a0, 0u, a2, 0u, b0, b1, dd);
            }
            if constexpr (FMT == kFmtInt4) {
              dd[0] >>= 4;   // exact: every product was 16x
              dd[1] >>= 4;
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              int mA, mB;
              general_mult<FMT, PLAIN>(rsc[o][h], sg, ta, mA, mB);
              acc[o][h] += static_cast<long long>(dd[h]) * mA;
              if constexpr (FMT == kFmtNvfp4) acc[o][h] += static_cast<long long>(e[h]) * mB;
            }
          }
        }
      }
    }
    // the row block is complete: its totals, then the S warps' partials, then the epilogue
    const int64_t r0 = q.rb + static_cast<int64_t>(b) * R;
    const int nrows = static_cast<int>(max(static_cast<int64_t>(0), min(static_cast<int64_t>(R), q.re - r0)));
    if (use_class) {
      constexpr int W = F::kW;
      const long long mlo = 1ll << (W - g);                          // class g
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
      if (slice == 0 && owner && rr < nrows && ok) {
        const int64_t row = r0 + rr;
        const float Sw = unit ? 1.0f : __ldg(reinterpret_cast<const float*>(d.srows + row * d.srs));
        float yv = mm_epilogue(tot, Sw, s.Sa[0], W);
        if (d.flags & kMmAscale) {
          yv = fadd(fmul(d.y[row], __ldg(d.alpha)), yv);
        } else if (d.flags & kMmAcc) {
          yv = fadd(d.y[row], yv);
        }
        put_out(d.y, row, yv, fan);
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
      if (slice == 0 && g < mt && ok) {
#pragma unroll
        for (int o = 0; o < NO; ++o)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int rr = 8 * o + 2 * t + h;
            if (rr < nrows) {
              const int64_t row = r0 + rr;
              const float Sw = unit ? 1.0f : __ldg(reinterpret_cast<const float*>(d.srows + row * d.srs));
              float yv = mm_epilogue(acc[o][h], Sw, s.Sa[g], F::kW);
              const int64_t idx = static_cast<int64_t>(g) * d.ldy + row;
              if (d.flags & kMmAscale) {
                yv = fadd(fmul(d.y[idx], __ldg(d.alpha + g)), yv);
              } else if (d.flags & kMmAcc) {
                yv = fadd(d.y[idx], yv);
              }
              put_out(d.y, idx, yv, fan);
            }
          }
      }
#pragma unroll
      for (int o = 0; o < NO; ++o) acc[o][0] = acc[o][1] = 0;
      if constexpr (S > 1) __syncthreads();
    }
  }
}

// QACT + MM over the projections of C in order (M <= MT activation rows each). RMAX: the
// largest row block the launch uses (the ring's stage size).
template <int FMT, int MT, int NS, bool PLAIN, int MAXP, int RMAX, int FIXED>
// One activation row, 8-row blocks: three CTAs' registers fit an SM (76-80 a thread, no spills),
// so the next launch's CTAs start on SMs where two of this launch still run and issue their
// first weight copies early (griddepcontrol). Measured 4-6 % off the Qwen3-0.6B step.
__global__ void __launch_bounds__(kThreads, (FIXED < 0 || FIXED == kCfgR32) ? 1 : (MT == 1 ? 3 : 2))
    gemv_kernel(const __grid_constant__ Chain<MAXP> C, const GLayout L) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using F = GF<FMT>;
  GSmem s = gemv_carve(smem_raw, L);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t* const ring = s.ring + warp * NS * L.stage_bytes;
  uint8_t* const sring = s.sring + warp * NS * L.scale_bytes;
  const uint32_t bar0 = smem_addr(s.bar + warp * NS);
  bool ok = true;   // false once a wait ran out: the remaining items are drained, not computed

  if (lane == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(bar0 + 8 * i, 1);
    mbar_init_fence();
  }
  if (MAXP == 1 ? lane == 0 : lane < C.count)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&C.proj[MAXP == 1 ? 0 : lane].map))
                 : "memory");
  __syncwarp();

  RingIssue<FMT, PLAIN, NS, MAXP> iss;
  iss.C = &C;
  iss.ring_s = smem_addr(ring);
  iss.sring_s = smem_addr(sring);
  iss.bar0 = bar0;
  iss.stage_bytes = L.stage_bytes;
  iss.scale_bytes = L.scale_bytes;
  iss.lane = lane;
  iss.warp = warp;
  const int count = MAXP == 1 ? 1 : C.count;
  PArgs d = load_args(C.proj[0]);   // the projection computed next, and its geometry
  Geo q = geometry<FMT>(d, warp);
  iss.count = count;
  iss.p = 0;
  iss.i = 0;
  iss.issued = 0;
  iss.a = d;
  iss.q = q;
#pragma unroll 1
  for (int q = 0; q < NS - 1; ++q) iss.next();
  // the row scales the epilogue reads (4 bytes a row, RSC): into L1 now, so that their memory
  // latency is not paid at the end of the critical path (they never depend on the previous
  // kernel)
  if (MAXP == 1 && PLAIN && !(d.flags & kMmUnit) && lane < q.R) {
    for (int b = 0; b < q.NBLK; ++b) {
      const int64_t row = q.rb + static_cast<int64_t>(b) * q.R + lane;
      if (row < q.re) asm volatile("prefetch.global.L1 [%0];" ::"l"(d.srows + row * d.srs));
    }
  }
  // shared memory only: ahead of the wait
  constexpr bool kCleared = MAXP == 1;
  if (kCleared)
    gemv_clear_activations<FMT, MT, PLAIN>(d, s, min(MT, d.M),
                                           ((d.K + F::kElems - 1) / F::kElems) * F::kElems, L.ap, L.frag);
  // Stepped tags with a tagged input: the input's tags alone order this launch after the one
  // before (whose CTAs all run: this launch started after each of them released it), so the
  // kernel does not wait for that launch to finish. Otherwise the activations may come from the
  // kernel launched before.
  const bool stepped = MAXP == 1 && C.peer.world > 0 && C.peer.tags != 0;
  if (!(stepped && C.peer.wait)) pdl_wait();

  // output fan-out (single-projection launches of a decode step): tagged output words, and the
  // tag a tagged input must carry. Counted tags: this rank's count of completed launches (read
  // after the wait above); stepped tags: the count of completed steps and this launch's position
  // in the step (the count only changes at the end of a step's last launch, which starts after
  // every other launch of the step has read it)
  __shared__ int64_t peer_delta[kMaxPeers];
  __shared__ int peer_count;
  Fan fan{0, 0, 0u, peer_delta};
  bool tagged_in = false;
  uint32_t expect = 0;
  if (MAXP == 1 && C.peer.world > 0) {
    if (threadIdx.x < kMaxPeers) peer_delta[threadIdx.x] = C.peer.delta[threadIdx.x];
    if (threadIdx.x == 0) peer_count = *reinterpret_cast<volatile int*>(C.peer.seq);
    __syncthreads();
    fan.world = C.peer.world;
    fan.rank = C.peer.rank;
    const uint32_t base = stepped ? static_cast<uint32_t>(peer_count) * kStepTags +
                                        static_cast<uint32_t>(C.peer.step_pos)
                                  : static_cast<uint32_t>(peer_count);
    fan.tag = base + 1u;
    tagged_in = C.peer.wait != 0;
    expect = base;
  }

  int f = 0;
  for (int pi = 0; pi < count; ++pi) {
    if (pi > 0) grid_barrier(C.status);   // projection pi may read what pi - 1 wrote
    const int KCH = (d.K + F::kElems - 1) / F::kElems;
    gemv_load_activations<FMT, MT, PLAIN>(d, s, min(MT, d.M), KCH * F::kElems, L.ap, L.frag,
                                          kCleared && pi == 0, pi == 0 && tagged_in, expect, C.status,
                                          tagged_in ? g_tag_wait_limit : 0u);
    // the next launch starts here: earlier (before the wait) or later (at exit) measured slower
    if (pi == count - 1) pdl_launch();
    const int mt = min(MT, d.M);
    // Keep HBM busy past the grid barriers: this warp's rows of the next two projections into
    // L2 (at most 64 KB a warp), and their tensor maps into the descriptor cache.
    if (MAXP > 1 && lane == 0) {
#pragma unroll 1
      for (int a = 1; a <= 2 && pi + a < count; ++a) {
        const PArgs n = load_args(C.proj[pi + a]);
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(n.map)) : "memory");
        const Geo nq = geometry<FMT>(n, warp);
        if (warp % nq.S == 0 && nq.re > nq.rb) {
          const int64_t row_bytes = FMT == kFmtInt8 ? n.K : n.K / 2;
          int64_t len = (nq.re - nq.rb - 1) * n.rs + row_bytes;
          len = (len < 64 * 1024 ? len : 64 * 1024) & ~int64_t(15);
          const uint8_t* base = reinterpret_cast<const uint8_t*>(n.rows) + nq.rb * n.rs;
          if (len > 0) prefetch_l2(base, static_cast<uint32_t>(len));
        }
      }
    }
    switch (FIXED >= 0 ? FIXED : d.cfg) {   // FIXED: one decomposition (a single projection)
      case kCfgR32:
        if constexpr (RMAX == 32 && (FIXED < 0 || FIXED == kCfgR32)) run_proj<FMT, MT, PLAIN, NS, MAXP, 32, 1>(d, q, s, iss, f, ok, C.status, L, ring, sring, mt, fan);
        break;
      case kCfgS1:
        if constexpr (FIXED < 0 || FIXED == kCfgS1) run_proj<FMT, MT, PLAIN, NS, MAXP, 8, 1>(d, q, s, iss, f, ok, C.status, L, ring, sring, mt, fan);
        break;
      case kCfgS2:
        if constexpr (FIXED < 0 || FIXED == kCfgS2) run_proj<FMT, MT, PLAIN, NS, MAXP, 8, 2>(d, q, s, iss, f, ok, C.status, L, ring, sring, mt, fan);
        break;
      case kCfgS4:
        if constexpr (FIXED < 0 || FIXED == kCfgS4) run_proj<FMT, MT, PLAIN, NS, MAXP, 8, 4>(d, q, s, iss, f, ok, C.status, L, ring, sring, mt, fan);
        break;
      default:
        if constexpr (FIXED < 0 || FIXED == kCfgS8) run_proj<FMT, MT, PLAIN, NS, MAXP, 8, 8>(d, q, s, iss, f, ok, C.status, L, ring, sring, mt, fan);
        break;
    }
    if (pi + 1 < count) {   // ahead of the barrier, off the critical path
      d = load_args(C.proj[pi + 1]);
      q = geometry<FMT>(d, warp);
    }
    if (MAXP > 1) __syncthreads();   // the next projection's activations overwrite shared memory
  }
  // the last CTA advances this rank's count (stepped tags: at the end of the step only)
  if (MAXP == 1 && C.peer.world > 0 && (!stepped || C.peer.step_last)) {
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(C.peer.done, 1) == static_cast<int>(gridDim.x) - 1) {
      *C.peer.done = 0;
      *reinterpret_cast<volatile int*>(C.peer.seq) = peer_count + 1;
    }
  }
}
// The weight rows as a 2-D tensor of bytes: [N][row_bytes] with rows rs bytes apart, copied in
// boxes of 8 rows x 128 bytes with the 128-byte swizzle. cuTensorMapEncodeTiled comes from the
// driver through the runtime's entry-point query (nothing links libcuda).
bool encode_rows_map(CUtensorMap* map, const uint8_t* rows, int row_bytes, int64_t N, int64_t rs,
                     int box_rows = kBox) {
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(N)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(rs)};
  const cuuint32_t box[2] = {kChunk, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(rows), dims, strides, box,
                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kMaxChain = 120;   // projections of one launch (kernel parameters under 32 KB)

int cfg_rows(int cfg) { return cfg == kCfgR32 ? 32 : 8; }
int cfg_split(int cfg) { return cfg <= kCfgS1 ? 1 : (1 << (cfg - 1)); }

// Work decomposition: 32-row blocks while they give every warp of the grid work; else 8-row
// blocks with as many warps a row as keep every warp busy, each with at least one chunk.
int pick_cfg(int fmt, int64_t N, int K, int64_t warps) {
  if (N >= 32 * warps) return kCfgR32;
  const int elems = fmt == kFmtInt8 ? 128 : 256;
  const int KCH = (K + elems - 1) / elems;
  int split = 1;
  while (split < 8 && (N / 8) * split < warps && KCH / (split * 2) >= 1) split *= 2;
  return split == 1 ? kCfgS1 : split == 2 ? kCfgS2 : split == 4 ? kCfgS4 : kCfgS8;
}

template <int FMT, bool PLAIN>
GLayout launch_layout(int MT, int kmax, bool fused, bool frag, int smax, int rmax, int ns) {
  using F = GF<FMT>;
  GLayout L;
  L.MT = MT;
  L.K = kmax;
  const int kp = ((kmax + F::kElems - 1) / F::kElems) * F::kElems;
  L.ap = kp + kActPad;
  L.vpl = 2;   // K-split blocks are 8 rows
  L.S = smax;
  L.stage_bytes = rmax * kChunk;
  L.scale_bytes = PLAIN ? 0 : rmax * 16;
  L.ns = ns;
  L.fused = fused;
  L.frag = frag && MT == 1 && PLAIN;
  return L;
}

template <int FMT, int MT, int NS, bool PLAIN, int MAXP, int RMAX, int FIXED>
int launch_chain(const Chain<MAXP>& C, const GLayout& L, int grid, bool coop, cudaStream_t stream,
                 bool pdl) {
  const size_t smem = gemv_layout(L, nullptr);
  if (smem > 227 * 1024) return kErrArg;
  auto kern = gemv_kernel<FMT, MT, NS, PLAIN, MAXP, RMAX, FIXED>;
  static size_t configured_smem[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (smem > 48 * 1024 && configured_smem[dev] < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured_smem[dev] = smem;
  }
  // every instantiation asks for the same (largest) shared-memory carveout, so a dependent
  // launch's CTAs can join an SM that still runs the previous kernel without reconfiguring it
  static bool carveout[kMaxDevices] = {false};
  if (!carveout[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return kErrCuda;
    carveout[dev] = true;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess)
    return kErrCuda;
  if (occ < 1) return kErrArg;
  const int cap = sm_count(dev) * occ;
  if (coop) grid = cap;   // every CTA resident: the grid barriers need it
  grid = max(1, min(grid, cap));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (coop) {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = (coop || pdl) ? 1 : 0;
  void* args[] = {const_cast<Chain<MAXP>*>(&C), const_cast<GLayout*>(&L)};
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kern), args) == cudaSuccess ? kOk
                                                                                          : kErrCuda;
}

// Choose the ring depth and whether the class path's A fragments fit beside it, then launch.
// FIXED >= 0: a single projection of that decomposition; -1: a chain (decomposition per
// projection).
template <int FMT, int MT, bool PLAIN, int MAXP, int FIXED>
int launch_fit(const Chain<MAXP>& C, int kmax, bool fused, int smax, int rmax, int grid, bool coop,
               cudaStream_t stream, bool pdl) {
  auto fits = [&](bool frag, int r, int ns) {
    return gemv_layout(launch_layout<FMT, PLAIN>(MT, kmax, fused, frag, smax, r, ns), nullptr) <=
           227 * 1024;
  };
  if constexpr (FIXED < 0 || FIXED == kCfgR32) {
    if (rmax == 32) {
      for (bool frag : {true, false}) {
        if (fits(frag, 32, 5))
          return launch_chain<FMT, MT, 5, PLAIN, MAXP, 32, FIXED>(
              C, launch_layout<FMT, PLAIN>(MT, kmax, fused, frag, smax, 32, 5), grid, coop, stream, pdl);
      }
      if (fits(false, 32, 3))
        return launch_chain<FMT, MT, 3, PLAIN, MAXP, 32, FIXED>(
            C, launch_layout<FMT, PLAIN>(MT, kmax, fused, false, smax, 32, 3), grid, coop, stream, pdl);
      return kErrArg;   // the caller retries with 8-row blocks
    }
  }
  if constexpr (FIXED != kCfgR32) {
    for (bool frag : {true, false}) {
      if (fits(frag, 8, 4))
        return launch_chain<FMT, MT, 4, PLAIN, MAXP, 8, FIXED>(
            C, launch_layout<FMT, PLAIN>(MT, kmax, fused, frag, smax, 8, 4), grid, coop, stream, pdl);
    }
  }
  return kErrArg;
}

void fill_proj(Proj& d, const MMParams& p, int64_t m0, int mt) {
  d.rows = p.rows;
  d.rs = static_cast<int>(p.rs);
  d.srows = p.srows;
  d.srs = static_cast<int>(p.srs);
  d.x = p.x != nullptr ? p.x + m0 * p.ldx : nullptr;
  d.ldx = static_cast<int>(p.ldx);
  d.q = p.q != nullptr ? p.q + m0 * p.ldq : nullptr;
  d.ldq = static_cast<int>(p.ldq);
  d.Sa = p.Sa != nullptr ? p.Sa + m0 : nullptr;
  d.da = p.da != nullptr ? p.da + m0 * p.ldd : nullptr;
  d.ldd = static_cast<int>(p.ldd);
  d.y = p.y + m0 * p.ldy;
  d.ldy = static_cast<int>(p.ldy);
  d.alpha = p.alpha != nullptr ? p.alpha + m0 : nullptr;
  d.N = p.N;
  d.K = p.K;
  d.flags = p.flags;
  d.k0 = p.k0;
  d.row_mode = p.row_mode;
  d.M = mt;
}

template <int FMT, bool PLAIN>
int single_fmt(const MMParams& p, cudaStream_t stream, bool pdl, int dev) {
  const int warps = sm_count(dev) * kWarps;
  int cfg = p.split == 0 ? pick_cfg(FMT, p.N, p.K, warps)
            : p.split == 32 ? kCfgR32
            : p.split == 1 ? kCfgS1
            : p.split == 2 ? kCfgS2
            : p.split == 4 ? kCfgS4 : kCfgS8;
  const int row_bytes = FMT == kFmtInt8 ? p.K : p.K / 2;
  for (int64_t m0 = 0; m0 < p.M; m0 += 8) {   // passes of up to 8 activation rows
    const int mt = static_cast<int>(p.M - m0 < 8 ? p.M - m0 : 8);
    Chain<1> C;
    std::memset(&C, 0, sizeof(C));
    fill_proj(C.proj[0], p, m0, mt);
    C.count = 1;
    C.status = p.status;
    if (p.peer != nullptr) {   // a row-sharded decode projection (M = 1: one pass)
      C.peer.rank = p.peer->rank;
      C.peer.world = p.peer->world;
      C.peer.wait = p.peer->wait;
      for (int r = 0; r < kMaxPeers; ++r) C.peer.delta[r] = r < p.peer->world ? p.peer->delta[r] : 0;
      C.peer.seq = p.peer->seq;
      C.peer.done = p.peer->done;
      C.peer.tags = p.peer->tags;
      C.peer.step_pos = p.peer->step_pos;
      C.peer.step_last = p.peer->step_last;
    }
    for (int attempt = 0; attempt < 2; ++attempt) {
      C.proj[0].cfg = cfg;
      if (!encode_rows_map(&C.proj[0].map, p.rows, row_bytes, p.N, p.rs)) return kErrCuda;
      const int R = cfg_rows(cfg), S = cfg_split(cfg);
      const int64_t grid = (p.N + static_cast<int64_t>(R) * (kWarps / S) - 1) / (static_cast<int64_t>(R) * (kWarps / S));
      const int g = static_cast<int>(grid < (1 << 20) ? grid : (1 << 20));
      int st;
      const bool fused = p.x != nullptr;
      switch (cfg) {
#define OTQ_SINGLE(CFG)                                                                       \
  st = mt == 1 ? launch_fit<FMT, 1, PLAIN, 1, CFG>(C, p.K, fused, S, R, g, false, stream, pdl) \
               : launch_fit<FMT, 8, PLAIN, 1, CFG>(C, p.K, fused, S, R, g, false, stream, pdl)
        case kCfgR32: OTQ_SINGLE(kCfgR32); break;
        case kCfgS1: OTQ_SINGLE(kCfgS1); break;
        case kCfgS2: OTQ_SINGLE(kCfgS2); break;
        case kCfgS4: OTQ_SINGLE(kCfgS4); break;
        default: OTQ_SINGLE(kCfgS8); break;
#undef OTQ_SINGLE
      }
      if (st == kErrArg && cfg == kCfgR32) {   // no room beside a long activation row
        cfg = kCfgS2;
        continue;
      }
      if (st != kOk) return st;
      break;
    }
  }
  return kOk;
}

template <int FMT, bool PLAIN>
int chain_fmt(const otq_proj* pr, int count, int* status, cudaStream_t stream, int dev) {
  const int warps = sm_count(dev) * kWarps;
  Chain<kMaxChain>* C = new Chain<kMaxChain>;
  std::memset(C, 0, sizeof(*C));
  int kmax = 0, smax = 1, rmax = 8;
  for (int i = 0; i < count; ++i) {
    MMParams p{};
    p.fmt = pr[i].fmt;
    p.flags = pr[i].flags;
    p.rows = pr[i].rows;
    p.rs = pr[i].rs;
    p.srows = pr[i].srows;
    p.srs = pr[i].srs;
    p.k0 = pr[i].k0;
    p.N = pr[i].N;
    p.K = static_cast<int>(pr[i].K);
    p.x = pr[i].x;
    p.ldx = pr[i].K;
    p.row_mode = pr[i].row_mode;
    p.M = 1;
    p.y = pr[i].y;
    p.ldy = pr[i].N;
    fill_proj(C->proj[i], p, 0, 1);
    const int row_bytes = FMT == kFmtInt8 ? p.K : p.K / 2;
    if (!encode_rows_map(&C->proj[i].map, pr[i].rows, row_bytes, p.N, pr[i].rs)) {
      delete C;
      return kErrCuda;
    }
    C->proj[i].cfg = pick_cfg(FMT, p.N, p.K, warps);
    kmax = max(kmax, p.K);
    smax = max(smax, cfg_split(C->proj[i].cfg));
    if (C->proj[i].cfg == kCfgR32) rmax = 32;
  }
  C->count = count;
  C->status = status;
  int st = launch_fit<FMT, 1, PLAIN, kMaxChain, -1>(*C, kmax, true, smax, rmax, 0, true, stream, false);
  if (st == kErrArg && rmax == 32) {   // no room for 32-row stages: 8-row blocks everywhere
    for (int i = 0; i < count; ++i)
      if (C->proj[i].cfg == kCfgR32) C->proj[i].cfg = kCfgS1;
    st = launch_fit<FMT, 1, PLAIN, kMaxChain, -1>(*C, kmax, true, smax, 8, 0, true, stream, false);
  }
  delete C;
  return st;
}

}  // namespace

int mm_launch(const MMParams& p0, cudaStream_t stream, bool pdl) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  MMParams p = p0;
  p.status = status_word();
  const bool plain = (p.flags & (kMmUnit | kMmRsc)) != 0;
  switch (p.fmt) {
    case kFmtInt8: return plain ? single_fmt<kFmtInt8, true>(p, stream, pdl, dev) : single_fmt<kFmtInt8, false>(p, stream, pdl, dev);
    case kFmtInt4: return plain ? single_fmt<kFmtInt4, true>(p, stream, pdl, dev) : single_fmt<kFmtInt4, false>(p, stream, pdl, dev);
    case kFmtFp4: return plain ? single_fmt<kFmtFp4, true>(p, stream, pdl, dev) : single_fmt<kFmtFp4, false>(p, stream, pdl, dev);
    case kFmtNvfp4: return plain ? single_fmt<kFmtNvfp4, true>(p, stream, pdl, dev) : single_fmt<kFmtNvfp4, false>(p, stream, pdl, dev);
    default: return kErrFormat;
  }
}

// Consecutive projections of one format and kind go in one launch (at most kMaxChain).
int chain_launch(const otq_proj* pr, int count, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  int* status = status_word();
  for (int i = 0; i < count;) {
    const int fmt = pr[i].fmt;
    const bool plain = (pr[i].flags & (kMmUnit | kMmRsc)) != 0;
    int j = i + 1;
    while (j < count && j - i < kMaxChain && pr[j].fmt == fmt &&
           ((pr[j].flags & (kMmUnit | kMmRsc)) != 0) == plain)
      ++j;
    int st;
    switch (fmt) {
      case kFmtInt8: st = plain ? chain_fmt<kFmtInt8, true>(pr + i, j - i, status, stream, dev) : chain_fmt<kFmtInt8, false>(pr + i, j - i, status, stream, dev); break;
      case kFmtInt4: st = plain ? chain_fmt<kFmtInt4, true>(pr + i, j - i, status, stream, dev) : chain_fmt<kFmtInt4, false>(pr + i, j - i, status, stream, dev); break;
      case kFmtFp4: st = plain ? chain_fmt<kFmtFp4, true>(pr + i, j - i, status, stream, dev) : chain_fmt<kFmtFp4, false>(pr + i, j - i, status, stream, dev); break;
      case kFmtNvfp4: st = plain ? chain_fmt<kFmtNvfp4, true>(pr + i, j - i, status, stream, dev) : chain_fmt<kFmtNvfp4, false>(pr + i, j - i, status, stream, dev); break;
      default: st = kErrFormat;
    }
    if (st != kOk) return st;
    i = j;
  }
  return kOk;
}

// The polls of a tagged-input wait on the current device (0: the default).
int set_tag_wait_limit(uint32_t polls) {
  const uint32_t v = polls == 0 ? (1u << 22) : polls;
  return cudaMemcpyToSymbol(g_tag_wait_limit, &v, sizeof(v)) == cudaSuccess ? kOk : kErrCuda;
}

// The grid barrier's words back to zero (after a launch whose barrier wait ran out).
int chain_reset() {
  const unsigned int zero = 0;
  if (cudaMemcpyToSymbol(g_bar_count, &zero, sizeof(zero)) != cudaSuccess) return kErrCuda;
  return kOk;
}

}  // namespace otq
