// MM for few activation rows over large weight matrices: a persistent, warp-specialized
// weight-streaming GEMV (same arithmetic and results as mm_gemv.cu; reference docs/isa.md
// "MM", opentpu/isasim.py:749-910).
//
// One CTA per SM slot walks its share of 16-row weight tiles (tile b, b + grid, ...), so the
// imbalance between CTAs is at most one tile. Warp 0 is the producer: it streams each tile, in
// row chunks of up to 2 KiB, into a ring of shared-memory stages with bulk asynchronous copies
// (cp.async.bulk ... mbarrier::complete_tx, no multicast) -- the bytes in flight are set by
// the ring, not by registers. It starts before griddepcontrol.wait: weights never depend on the
// kernel launched before this one, so under programmatic dependent launch the first stages
// fill while that kernel finishes. Warps 1..4 are consumers: after the wait they quantize the
// activations (QACT, qact.cuh) into shared memory, then all four consume every stage in order,
// each taking every fourth group of it, with the exact MMA-per-group arithmetic of mm_gemv.cu
// (weight fragments read from the stage, rows padded so the reads are bank-conflict free);
// each releases the stage to the producer, and at the end of a tile they add their int64
// partials through shared memory. Because every consumer waits for every stage in order, no
// waiter is ever two phases away from a barrier's current phase, which parity waits require.
// Every mbarrier wait is bounded; a wait that runs out records kStatusTimeout in the status
// word and the CTA returns.
#include <cuda_runtime.h>

#include <cstdint>

#include "otq_fp32.cuh"
#include "otq_internal.h"
#include "qact.cuh"

namespace otq {
namespace {

constexpr int kConsumers = 4;
constexpr int kThreads = 32 * (1 + kConsumers);
constexpr int kCThreads = 32 * kConsumers;
constexpr uint32_t kSpinLimit = 1u << 22;   // ~0.5 s of polling with the back-off below

template <int FMT>
struct Fmt {
  static constexpr int kW = (FMT == kFmtInt8) ? 16 : (FMT == kFmtNvfp4 ? 13 : 11);
  static constexpr int kGroupBytes = (FMT == kFmtInt8) ? 32 : 16;
  static constexpr int kPad = (FMT == kFmtInt8) ? 32 : 16;   // row padding in a stage
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of `bar` with parity `parity`; false after kSpinLimit polls (the status
// word records it).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 16) __nanosleep(100);
  }
  if (status != nullptr) atomicOr(status, kStatusTimeout);
  return false;
}
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst), "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ void imma(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1, int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void fp4_bytes(uint32_t w, uint32_t& lo, uint32_t& hi) {
  constexpr uint32_t kPosLo = 0x03020100u, kPosHi = 0x0C080604u;   // +0 +1 +2 +3 | +4 +6 +8 +12
  constexpr uint32_t kNegLo = 0xFDFEFF00u, kNegHi = 0xF4F8FAFCu;   // -0 -1 -2 -3 | -4 -6 -8 -12
  const uint32_t sel_lo = w & 0x7777u, sel_hi = (w >> 16) & 0x7777u;
  const uint32_t w4 = w << 4;
  const uint32_t s_lo = prmt(w4, w, 0xD9C8u);
  const uint32_t s_hi = prmt(w4, w, 0xFBEAu);
  lo = (prmt(kPosLo, kPosHi, sel_lo) & ~s_lo) | (prmt(kNegLo, kNegHi, sel_lo) & s_lo);
  hi = (prmt(kPosLo, kPosHi, sel_hi) & ~s_hi) | (prmt(kNegLo, kNegHi, sel_hi) & s_hi);
}

__device__ __forceinline__ void int4_bytes(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x8 = w ^ 0x88888888u;
  lo = x8 & 0x0F0F0F0Fu;
  hi = (x8 >> 4) & 0x0F0F0F0Fu;
}

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

__device__ __forceinline__ int shifted(int m, int shA, int dw) {
  const int sh = shA - dw;
  return sh >= 0 ? (m << sh) : 0;
}

// Shared memory: barriers, the ring, then the activation tile.
struct Ring {
  uint64_t* full;      // [NS]
  uint64_t* empty;     // [NS]
  uint8_t* stages;     // [NS][16][row_stride]
  uint8_t* act;        // [KG][MT][32]
  int* gB;             // [KG][MT]
  int* gA;             // [KG][MT]
  int* gC;             // [KG][MT]
  float* Sa;           // [MT]
  float* xs;           // [K]
  uint32_t* seg;       // [KG]
  uint32_t* qred;      // [40]
  long long* red;      // [2][kConsumers][32][4] partials of a tile (two tiles in turn)
};

__host__ __device__ inline size_t ring_layout(const RingCfg& rc, int MT, int K, bool fused,
                                              size_t* offs) {
  const size_t KG = K / 32;
  size_t off = 0;
  auto take = [&](int i, size_t bytes, size_t align) {
    off = (off + align - 1) & ~(align - 1);
    if (offs) offs[i] = off;
    off += bytes;
  };
  take(0, 8 * static_cast<size_t>(rc.ns), 16);
  take(1, 8 * static_cast<size_t>(rc.ns), 16);
  take(2, static_cast<size_t>(rc.ns) * 16 * rc.row_stride, 128);
  take(3, KG * MT * 32, 16);
  take(4, KG * MT * 4, 16);
  take(5, KG * MT * 4, 16);
  take(6, KG * MT * 4, 16);
  take(7, MT * 4, 16);
  take(8, fused ? static_cast<size_t>(K) * 4 : 0, 16);
  take(9, KG * 4, 16);
  take(10, 40 * 4, 16);
  take(11, 2 * static_cast<size_t>(kConsumers) * 32 * 4 * 8, 16);
  return off;
}

template <int MT>
__device__ __forceinline__ Ring carve(unsigned char* base, const RingCfg& rc, int K, bool fused) {
  size_t o[12];
  ring_layout(rc, MT, K, fused, o);
  Ring r;
  r.full = reinterpret_cast<uint64_t*>(base + o[0]);
  r.empty = reinterpret_cast<uint64_t*>(base + o[1]);
  r.stages = base + o[2];
  r.act = base + o[3];
  r.gB = reinterpret_cast<int*>(base + o[4]);
  r.gA = reinterpret_cast<int*>(base + o[5]);
  r.gC = reinterpret_cast<int*>(base + o[6]);
  r.Sa = reinterpret_cast<float*>(base + o[7]);
  r.xs = reinterpret_cast<float*>(base + o[8]);
  r.seg = reinterpret_cast<uint32_t*>(base + o[9]);
  r.qred = reinterpret_cast<uint32_t*>(base + o[10]);
  r.red = reinterpret_cast<long long*>(base + o[11]);
  return r;
}

template <int FMT, int MT>
__device__ __forceinline__ int act_index(int j, int i) {
  int e = i & 31;
  if constexpr (FMT == kFmtInt4) {
    const int r = e & 7;
    e = (e & ~7) | ((r & 1) ? 4 + (r >> 1) : (r >> 1));
  }
  return ((i >> 5) * MT + j) * 32 + e;
}

template <int FMT, int MT>
__device__ __forceinline__ void group_terms(const Ring& s, int j, int g, int da, int qsum) {
  const int sh = Fmt<FMT>::kW - da;
  s.gB[g * MT + j] = sh >= 0 ? (1 << sh) : 0;
  s.gA[g * MT + j] = sh;
  s.gC[g * MT + j] = 8 * qsum;
}

// The consumer warps fill the activation tile [m0, m0 + mt) (rows past mt are zeros).
template <int FMT, int MT>
__device__ void load_activations(const MMParams& p, const Ring& s, int m0, int mt,
                                 const ThreadGroup<kCThreads, 1>& grp) {
  const int K = p.K;
  const int KG = K >> 5;
  if (mt < MT) {
    for (int i = grp.tid; i < KG * MT * 8; i += kCThreads) {
      const int g = i / (MT * 8), rem = i % (MT * 8), j = rem / 8;
      if (j >= mt) reinterpret_cast<uint32_t*>(s.act)[i] = 0u;
      if (rem % 8 == 0 && j >= mt) {
        s.gB[g * MT + j] = 0;
        s.gA[g * MT + j] = -1;
        s.gC[g * MT + j] = 0;
      }
    }
    if (grp.tid < MT && grp.tid >= mt) s.Sa[grp.tid] = 0.0f;
  }
  if (p.x != nullptr) {
    for (int j = 0; j < mt; ++j) {
      stage_row(grp, p.x + static_cast<int64_t>(m0 + j) * p.ldx, s.xs, K);
      QactRowResult r = qact_row(grp, s.xs, K, 32, p.row_mode != 0, s.seg, s.qred,
                                 [&](int i, int qv, int d) {
                                   s.act[act_index<FMT, MT>(j, i)] =
                                       static_cast<uint8_t>(static_cast<int8_t>(qv));
                                   const int sum =
                                       (FMT == kFmtInt4) ? __reduce_add_sync(0xFFFFFFFFu, qv) : 0;
                                   if ((grp.tid & 31) == 0) group_terms<FMT, MT>(s, j, i >> 5, d, sum);
                                 });
      if (grp.tid == 0) s.Sa[j] = r.S;
    }
  } else {
    for (int j = 0; j < mt; ++j) {
      const int8_t* qr = p.q + static_cast<int64_t>(m0 + j) * p.ldq;
      const uint8_t* dr = p.da + static_cast<int64_t>(m0 + j) * p.ldd;
      for (int i = grp.tid; i < K; i += kCThreads) {
        const int qv = __ldcg(qr + i);
        s.act[act_index<FMT, MT>(j, i)] = static_cast<uint8_t>(static_cast<int8_t>(qv));
        const int sum = (FMT == kFmtInt4) ? __reduce_add_sync(0xFFFFFFFFu, qv) : 0;
        if ((grp.tid & 31) == 0) group_terms<FMT, MT>(s, j, i >> 5, __ldcg(dr + (i >> 5)), sum);
      }
      if (grp.tid == 0) s.Sa[j] = __ldcg(p.Sa + m0 + j);
    }
  }
  grp.sync();
}

// One group of a stage: acc (rows g, g+8 x activation rows 2t, 2t+1) += its exact contribution.
template <int FMT, int MT, bool PLAIN>
__device__ __forceinline__ void stage_group(const Ring& s, const uint8_t* stage, int row_stride,
                                            int Gl, int G, int lane, const uint8_t* sg,
                                            const uint8_t* sh, int k0, bool okg, bool okh,
                                            long long (&acc)[4]) {
  const int g = lane >> 2, t = lane & 3;
  uint32_t b0 = 0u, b1 = 0u;
  if (g < MT) {
    const uint2 bv = *reinterpret_cast<const uint2*>(s.act + (G * MT + g) * 32 + 8 * t);
    b0 = bv.x;
    b1 = bv.y;
  }
  const int cc0 = 2 * t < MT ? 2 * t : 0, cc1 = 2 * t + 1 < MT ? 2 * t + 1 : 0;
  const uint8_t* rg = stage + g * row_stride;
  const uint8_t* rh = rg + 8 * row_stride;
  uint32_t scg = 0u, sch = 0u;
  if constexpr (!PLAIN) {
    scg = okg ? load_scale<FMT>(sg, k0, G) : 0u;
    sch = okh ? load_scale<FMT>(sh, k0, G) : 0u;
  }
  if constexpr (FMT == kFmtInt8) {
    const uint2 wg = *reinterpret_cast<const uint2*>(rg + Gl * 32 + 8 * t);
    const uint2 wh = *reinterpret_cast<const uint2*>(rh + Gl * 32 + 8 * t);
    int d[4];
    imma(wg.x, wh.x, wg.y, wh.y, b0, b1, d);
    const int B0 = s.gB[G * MT + cc0], B1 = s.gB[G * MT + cc1];
    if constexpr (PLAIN) {
      acc[0] += static_cast<long long>(d[0]) * B0;
      acc[1] += static_cast<long long>(d[1]) * B1;
      acc[2] += static_cast<long long>(d[2]) * B0;
      acc[3] += static_cast<long long>(d[3]) * B1;
    } else {
      const int dwg = min(static_cast<int>(scg), 31), dwh = min(static_cast<int>(sch), 31);
      acc[0] += static_cast<long long>(d[0]) * (B0 >> dwg);
      acc[1] += static_cast<long long>(d[1]) * (B1 >> dwg);
      acc[2] += static_cast<long long>(d[2]) * (B0 >> dwh);
      acc[3] += static_cast<long long>(d[3]) * (B1 >> dwh);
    }
  } else {
    const uint32_t wg = *reinterpret_cast<const uint32_t*>(rg + Gl * 16 + 4 * t);
    const uint32_t wh = *reinterpret_cast<const uint32_t*>(rh + Gl * 16 + 4 * t);
    uint32_t glo, ghi, hlo, hhi;
    if constexpr (FMT == kFmtInt4) {
      int4_bytes(wg, glo, ghi);
      int4_bytes(wh, hlo, hhi);
    } else {
      fp4_bytes(wg, glo, ghi);
      fp4_bytes(wh, hlo, hhi);
    }
    if constexpr (FMT == kFmtInt4 || FMT == kFmtFp4) {
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
        const int dwg = static_cast<int>(scg & 0xFFu), dwh = static_cast<int>(sch & 0xFFu);
        const int mg = static_cast<int>((scg >> (8 + 6 * sub)) & 63u);
        const int mh = static_cast<int>((sch >> (8 + 6 * sub)) & 63u);
        acc[0] += static_cast<long long>(d[0]) * shifted(mg, A0, dwg);
        acc[1] += static_cast<long long>(d[1]) * shifted(mg, A1, dwg);
        acc[2] += static_cast<long long>(d[2]) * shifted(mh, A0, dwh);
        acc[3] += static_cast<long long>(d[3]) * shifted(mh, A1, dwh);
      }
    } else {   // nvfp4: two groups of 16 per sub-block (lanes t < 2 hold the first)
      const bool first = t < 2;
      int d0[4], d1[4];
      imma(first ? glo : 0u, first ? hlo : 0u, first ? ghi : 0u, first ? hhi : 0u, b0, b1, d0);
      imma(first ? 0u : glo, first ? 0u : hlo, first ? 0u : ghi, first ? 0u : hhi, b0, b1, d1);
      const int A0 = s.gA[G * MT + cc0], A1 = s.gA[G * MT + cc1];
      int mg0 = 1, mg1 = 1, mh0 = 1, mh1 = 1, dg0 = 0, dg1 = 0, dh0 = 0, dh1 = 0;
      if constexpr (!PLAIN) {
        auto e4 = [](uint32_t e, int& m, int& dw) {
          const int E = (e >> 3) & 15;
          m = E ? 8 + static_cast<int>(e & 7u) : static_cast<int>(e & 7u);
          dw = 15 - max(E, 1);
        };
        e4(scg & 0xFFu, mg0, dg0);
        e4((scg >> 8) & 0xFFu, mg1, dg1);
        e4(sch & 0xFFu, mh0, dh0);
        e4((sch >> 8) & 0xFFu, mh1, dh1);
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
}

template <int FMT, int MT, bool PLAIN>
__global__ void __launch_bounds__(kThreads, 1) mm_ring_kernel(const MMParams p, const RingCfg rc) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  using F = Fmt<FMT>;
  const int K = p.K;
  Ring s = carve<MT>(smem_raw, rc, K, p.x != nullptr);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (p.N + 15) / 16;
  const int my_tiles = static_cast<int>((ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x);
  const int nmt = (p.M + MT - 1) / MT;
  const int row_bytes = (FMT == kFmtInt8) ? K : (K >> 1);
  const int CB = rc.chunk_bytes;
  const int nch = (row_bytes + CB - 1) / CB;
  const uint32_t full0 = smem_addr(s.full), empty0 = smem_addr(s.empty);
  const uint32_t stage0 = smem_addr(s.stages);
  const uint32_t stage_bytes = 16u * static_cast<uint32_t>(rc.row_stride);

  if (threadIdx.x == 0) {
    for (int i = 0; i < rc.ns; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, kConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    // stages in order: m-tile, local tile, chunk
    uint32_t st = 0;
    for (int mi = 0; mi < nmt; ++mi) {
      for (int i = 0; i < my_tiles; ++i) {
        const int64_t tile = blockIdx.x + static_cast<int64_t>(i) * gridDim.x;
        const int64_t left = p.N - tile * 16;
        const int nrows = left < 16 ? static_cast<int>(left) : 16;
        for (int h = 0; h < nch; ++h, ++st) {
          const uint32_t bytes_h = static_cast<uint32_t>(min(CB, row_bytes - h * CB));
          const uint32_t slot = st % rc.ns;
          const uint32_t use = st / rc.ns;
          if (use > 0 && !mbar_wait(empty0 + 8 * slot, (use - 1) & 1, p.status)) return;
          if (lane == 0) mbar_expect_tx(full0 + 8 * slot, nrows * bytes_h);
          __syncwarp();
          if (lane < nrows)
            bulk_copy(stage0 + slot * stage_bytes + lane * rc.row_stride,
                      p.rows + (tile * 16 + lane) * p.rs + static_cast<int64_t>(h) * CB, bytes_h,
                      full0 + 8 * slot);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const ThreadGroup<kCThreads, 1> grp{static_cast<int>(threadIdx.x) - 32};
  const int c = warp - 1;
  const int g = lane >> 2, t = lane & 3;
  const bool unit = (p.flags & kMmUnit) != 0;
  // A consumer whose bounded wait runs out (the status word has it) computes nothing more but
  // keeps taking part in the consumers' named barriers, so no other consumer waits forever.
  bool ok = true;
  pdl_wait();   // the activations may come from the kernel launched before this one
  for (int mi = 0; mi < nmt; ++mi) {
    const int m0 = mi * MT;
    const int mt = min(MT, p.M - m0);
    if (mi > 0) grp.sync();   // every consumer is done with the previous activation tile
    load_activations<FMT, MT>(p, s, m0, mt, grp);
    if (mi == nmt - 1) pdl_launch();
    for (int i = 0; i < my_tiles; ++i) {
      const int64_t tile = blockIdx.x + static_cast<int64_t>(i) * gridDim.x;
      const int64_t r0 = tile * 16 + g, r1 = r0 + 8;
      const bool okg = r0 < p.N, okh = r1 < p.N;
      const uint8_t* sg = (PLAIN || !okg) ? nullptr : p.srows + r0 * p.srs;
      const uint8_t* sh = (PLAIN || !okh) ? nullptr : p.srows + r1 * p.srs;
      if constexpr (!PLAIN) {   // the rows' scale words are read group by group below
        if (okg) asm volatile("prefetch.global.L1 [%0];" ::"l"(sg));
        if (okh) asm volatile("prefetch.global.L1 [%0];" ::"l"(sh));
      }
      long long acc[4] = {0, 0, 0, 0};
      for (int h = 0; h < nch; ++h) {
        const uint32_t st = (static_cast<uint32_t>(mi) * my_tiles + i) * nch + h;
        const uint32_t slot = st % rc.ns;
        if (ok) ok = mbar_wait(full0 + 8 * slot, (st / rc.ns) & 1, p.status);
        if (!ok) continue;
        const uint8_t* stage = s.stages + slot * stage_bytes;
        const int gfirst = h * CB / F::kGroupBytes;
        const int gn = min(CB, row_bytes - h * CB) / F::kGroupBytes;
#pragma unroll 2
        for (int gl = c; gl < gn; gl += kConsumers)
          stage_group<FMT, MT, PLAIN>(s, stage, rc.row_stride, gl, gfirst + gl, lane, sg, sh, p.k0,
                                      okg, okh, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * slot);
      }
      // the four consumers' partials of this tile (buffer i % 2: the next tile's writes do not
      // touch the buffer being read, so one barrier per tile suffices)
      long long* red = s.red + static_cast<size_t>(i & 1) * kConsumers * 32 * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) red[(c * 32 + lane) * 4 + k] = acc[k];
      grp.sync();
      if (c == 0 && ok) {
#pragma unroll
        for (int o = 1; o < kConsumers; ++o)
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[k] += red[(o * 32 + lane) * 4 + k];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t row = k >= 2 ? r1 : r0;
          const int col = 2 * t + (k & 1);
          if (row < p.N && col < mt) {
            const float Sw =
                unit ? 1.0f : __ldg(reinterpret_cast<const float*>(p.srows + row * p.srs));
            float yv = mm_epilogue(acc[k], Sw, s.Sa[col], F::kW);
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
    }
  }
}

template <int FMT, int MT, bool PLAIN>
int launch_ring(const MMParams& p, const RingCfg& rc, cudaStream_t stream, bool pdl) {
  const size_t smem = ring_layout(rc, MT, p.K, p.x != nullptr, nullptr);
  auto kern = mm_ring_kernel<FMT, MT, PLAIN>;
  static size_t configured[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (configured[dev] < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = smem;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess)
    return kErrCuda;
  if (occ < 1) return kErrArg;
  const int64_t ntiles = (p.N + 15) / 16;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * occ;
  const int grid = static_cast<int>(ntiles < cap ? ntiles : cap);
  // two kernel parameters: a small launcher of its own
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {const_cast<MMParams*>(&p), const_cast<RingCfg*>(&rc)};
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kern), args) == cudaSuccess
             ? kOk
             : kErrCuda;
}

template <int FMT, int MT>
int ring_plain(const MMParams& p, const RingCfg& rc, cudaStream_t stream, bool pdl) {
  if (p.flags & (kMmUnit | kMmRsc)) return launch_ring<FMT, MT, true>(p, rc, stream, pdl);
  return launch_ring<FMT, MT, false>(p, rc, stream, pdl);
}

template <int FMT>
int ring_fmt(const MMParams& p, const RingCfg& rc, cudaStream_t stream, bool pdl) {
  if (p.M <= 1) return ring_plain<FMT, 1>(p, rc, stream, pdl);
  if (p.M <= 2) return ring_plain<FMT, 2>(p, rc, stream, pdl);
  if (p.M <= 4) return ring_plain<FMT, 4>(p, rc, stream, pdl);
  return ring_plain<FMT, 8>(p, rc, stream, pdl);
}

}  // namespace

// Ring geometry: row chunks of at most 2 KiB (int8) or 1 KiB (4-bit) per stage, rows padded
// for conflict-free fragment reads, as many stages as fit next to the activation tile (aiming
// at two CTAs per SM when the activation tile is small).
RingCfg ring_config(int fmt, int K, int M, bool fused) {
  RingCfg rc{};
  const int row_bytes = fmt == kFmtInt8 ? K : K / 2;
  const int cb_max = fmt == kFmtInt8 ? 2048 : 1024;
  rc.chunk_bytes = row_bytes < cb_max ? row_bytes : cb_max;
  rc.row_stride = rc.chunk_bytes + (fmt == kFmtInt8 ? 32 : 16);
  const int mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  rc.ns = 1;
  const size_t other = ring_layout(rc, mt, K, fused, nullptr) - 16 * static_cast<size_t>(rc.row_stride);
  const size_t budget = other < 24 * 1024 ? 104 * 1024 : 200 * 1024;
  const size_t stage = 16 * static_cast<size_t>(rc.row_stride);
  int ns = static_cast<int>((budget > other ? budget - other : 0) / (stage + 16));
  rc.ns = ns < 2 ? 2 : (ns > 12 ? 12 : ns);
  return rc;
}

size_t ring_smem_bytes(int fmt, int K, int M, bool fused) {
  const RingCfg rc = ring_config(fmt, K, M, fused);
  const int mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  return ring_layout(rc, mt, K, fused, nullptr);
}

int mm_ring_launch(const MMParams& p, cudaStream_t stream, bool pdl) {
  const RingCfg rc = ring_config(p.fmt, p.K, p.M, p.x != nullptr);
  switch (p.fmt) {
    case kFmtInt8: return ring_fmt<kFmtInt8>(p, rc, stream, pdl);
    case kFmtInt4: return ring_fmt<kFmtInt4>(p, rc, stream, pdl);
    case kFmtFp4: return ring_fmt<kFmtFp4>(p, rc, stream, pdl);
    case kFmtNvfp4: return ring_fmt<kFmtNvfp4>(p, rc, stream, pdl);
    default: return kErrFormat;
  }
}

}  // namespace otq
