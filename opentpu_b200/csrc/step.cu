// The decode step as ONE persistent launch: a chain of projections, one activation row, ordered
// by data instead of by kernel boundaries or grid barriers (the reference's qwen3_step,
// opentpu/llm/qwen3.py:1793, runs a layer's projections as QACT + MM programs -- MM:
// opentpu/isasim.py:749-910, QACT: :913-959, GATHER between row-sharded slices: :1413-1438).
// Two weight formats: int8 rows with a per-row fp32 scale (MM RSC, or UNIT), computed exactly
// through QACT + MM; and the 4-bit group-32 fp16-scale format (the reference's survey quantizer,
// opentpu/quant.py:225-227), weight-only on the fp32 row (`deq @ x`, fp32 sums).
//
// Data order. Every projection's output row is a row of tagged 8-byte words (fp32 value | 32-bit
// tag) in one buffer. The CTA that finishes rows of projection p stores their words with tag
// s * 1024 + p + 1 (s: steps completed) on this GPU and, with world > 1, into every other rank's
// copy over NVLink (the all-gather fused in). A projection that reads p's output reads those
// words until every tag has arrived; no fence, flag or barrier stands between projections.
//
// Weight streaming. One producer warp a CTA walks the CTA's items -- an item is one 8-row block
// of a projection and up to 8 chunks of its K (128 bytes of a row a chunk), ONE 3-D tensor copy
// of up to 8 KB with the 128-byte swizzle (plus, for 4-bit rows, a 2-D copy of the block's fp16
// group scales) -- in the order the CTA computes them, across projection boundaries, into a ring
// of shared-memory stages (full / empty mbarriers). Weights never depend on activations, so
// while the CTA waits for projection p's input the weights of the next projections arrive. (One
// tensor copy a 1 KB box, issued by the computing warps themselves, measured 0.3-0.5 us of issue
// stall a copy on a B200: eight times fewer, larger copies from a warp that does nothing else.)
//
// Work split. A projection's 8-row blocks go in balanced ranges to the CTAs (one CTA an SM, all
// resident: cooperative launch). Within a CTA either the 8 compute warps share each block's K
// chunks (short projections; the warps' row totals meet in shared memory) or each warp takes
// whole blocks (the LM head).
//
// Arithmetic, int8 rows: the class path of gemv.cu -- a group's multiplier 2^(16 - da) depends on
// the activation only, so A row c of an mma.sync m16n8k32 (s8) holds the bytes of the groups
// whose offset is c, and a block's groups accumulate exactly in int32; per block one int64
// scaling per class and a lane reduction. A row with a group of offset 16 (multiplier 1, no class
// row) takes the general path for that projection: each group's int32 result times its
// multiplier into int64. Epilogue (i2f(acc) * Sw) * (Sa * 2^-16), three flushed RNE products:
// bit-identical to otq_qmm. 4-bit rows: x is staged once per projection as x'[k] = x[k] *
// 2^(-4 (k mod 4)) with each group's sum of x, so a nibble masked in place under 2^23's
// exponent, less 2^23, times x' is (code + 8) * x; a group adds s * (sum - 8 sum x).
//
// The last projection (the LM head) also yields the greedy token: with one GPU each CTA folds
// its rows' (value, index) keys into one 64-bit atomicMax as it stores them; with several GPUs a
// final phase reads the whole tagged logit row. The CTA that finishes last converts the key into
// the index (first maximum, numpy's order: -0 = +0, NaN largest), clears the accumulator and
// advances s.
//
// Every wait is bounded: a tag wait after the configured number of polls (otq_set_wait_limit), a
// stage wait after kSpinLimit polls; either sets the status word and the launch runs to its end
// (its outputs are then not valid).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <memory>

#include "mm_common.cuh"
#include "otq_fp32.cuh"
#include "otq_internal.h"
#include "qact.cuh"

namespace otq {
namespace {

constexpr int kCW = 8;                       // compute warps
constexpr int kCT = kCW * 32;                // compute threads (named barrier 1)
constexpr int kTh = kCT + 32;                // + the producer warp
constexpr int kChunkB = 128;                 // bytes of a row a chunk
constexpr int kCB = 8;                       // chunks an item at most
constexpr int kCodeStage = 8 * kCB * kChunkB;    // 8 KB: 8 rows x 8 chunks
constexpr int kScaleStage = 8 * kCB * 16;        // 1 KB: 8 rows x 8 chunks x 8 fp16 scales
constexpr int kMaxProj = OTQ_STEP_MAX;
constexpr uint32_t kTagStride = 1024;
constexpr int kMaxWorld = 8;
constexpr int kMaxRedBlocks = 32;            // 8-row blocks a CTA adds up in one pass
constexpr int kFmtRsc = OTQ_STEP_RSC;
constexpr int kFmtG32 = OTQ_STEP_G32;

__device__ uint32_t g_step_wait_limit = 1u << 22;

struct SInfo {            // one projection, as the kernel reads it (shared memory)
  const uint8_t* srows;   // int8: scale rows, Sw the first fp32 word (null: UNIT)
  int srs;
  int N;                  // this rank's rows
  int K;
  int fmt;
  int split;              // 8: the warps share each block's chunks; 1: a warp owns blocks
  int in;                 // -1: the plain input x0; else the projection whose output is x
  int out;                // word offset of this projection's full output row
  int nfull;              // the full row's length (N * world)
  int kch;                // chunks a row
  int cb;                 // chunks an item (min(8, kch))
  int ngr;                // items a block (ceil(kch / cb))
  int pad[3];
};
static_assert(sizeof(SInfo) == 64, "SInfo is 64 bytes");

struct StepTable {
  int count, world, rank, ns, kmax, redb, maxrows, stage_bytes;
  const float* x0;
  unsigned long long* words;
  long long delta[kMaxWorld];
  int* counters;                 // [0] steps completed, [1] CTAs done
  unsigned long long* amax;      // the head's key accumulator (0 between steps)
  long long* token;
  int* status;
  SInfo info[kMaxProj];
  alignas(128) CUtensorMap map[kMaxProj];    // rows / codes: {128 B, N rows, chunks}
  CUtensorMap smap[kMaxProj];                // 4-bit scales: {K/16 B, N rows}
};

struct SSmem {
  SInfo* info;       // [count]
  uint8_t* act;      // [kmax] activation bytes
  uint8_t* cls;      // [kmax/32] a group's class (its offset), 255: none
  uint8_t* dg;       // [kmax/32] a group's offset
  float* xs;         // [kmax] the fp32 row (QACT staging; 4-bit: x')
  float* xsum;       // [kmax/32] 4-bit: each group's sum of x
  uint32_t* segm;    // [kmax/32]
  uint32_t* qred;    // [kCW + 8]
  long long* red;    // [redb][kCW][8] the warps' row totals (4-bit: floats)
  float* sws;        // [maxrows] Sw of this CTA's rows of the projection
  uint64_t* full;    // [ns]
  uint64_t* empty;   // [ns]
  uint8_t* ring;     // [ns][stage_bytes], 1024-byte aligned
};

__host__ __device__ inline size_t step_smem(int count, int kmax, int redb, int maxrows, int ns,
                                            int stage_bytes, size_t* o) {
  size_t off = 0;
  auto take = [&](int i, size_t bytes) {
    off = (off + 15) & ~size_t(15);
    if (o) o[i] = off;
    off += bytes;
  };
  take(0, static_cast<size_t>(count) * sizeof(SInfo));
  take(1, kmax);
  take(2, kmax / 32);
  take(3, kmax / 32);
  take(4, static_cast<size_t>(kmax) * 4);
  take(5, kmax / 32 * 4);
  take(6, kmax / 32 * 4);
  take(7, (kCW + 8) * 4);
  take(8, static_cast<size_t>(redb) * kCW * 8 * 8);
  take(9, static_cast<size_t>(maxrows) * 4);
  take(10, static_cast<size_t>(ns) * 8);
  take(11, static_cast<size_t>(ns) * 8);
  take(12, static_cast<size_t>(ns) * stage_bytes + 1024);
  return off;
}

__device__ __forceinline__ SSmem carve(unsigned char* base, const StepTable& T) {
  size_t o[13];
  step_smem(T.count, T.kmax, T.redb, T.maxrows, T.ns, T.stage_bytes, o);
  SSmem s;
  s.info = reinterpret_cast<SInfo*>(base + o[0]);
  s.act = base + o[1];
  s.cls = base + o[2];
  s.dg = base + o[3];
  s.xs = reinterpret_cast<float*>(base + o[4]);
  s.xsum = reinterpret_cast<float*>(base + o[5]);
  s.segm = reinterpret_cast<uint32_t*>(base + o[6]);
  s.qred = reinterpret_cast<uint32_t*>(base + o[7]);
  s.red = reinterpret_cast<long long*>(base + o[8]);
  s.sws = reinterpret_cast<float*>(base + o[9]);
  s.full = reinterpret_cast<uint64_t*>(base + o[10]);
  s.empty = reinterpret_cast<uint64_t*>(base + o[11]);
  const uint32_t r = smem_addr(base + o[12]);
  s.ring = base + o[12] + (((r + 1023u) & ~1023u) - r);
  return s;
}

__device__ __forceinline__ void cbar() {   // the compute warps meet (named barrier 1)
  asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory");
}

// This CTA's 8-row blocks [b0, b1) of a projection of N rows.
__device__ __forceinline__ void cta_blocks(int N, int& b0, int& b1) {
  const int nb = (N + 7) / 8;
  b0 = static_cast<int>(static_cast<long long>(nb) * blockIdx.x / gridDim.x);
  b1 = static_cast<int>(static_cast<long long>(nb) * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                       uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_n(uint32_t bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}

__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v, int world,
                                        int rank, const long long* delta) {
  if (world == 1) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
    return;
  }
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
  for (int r = 0; r < world; ++r)
    if (r != rank) {
      unsigned long long* q = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(p) + delta[r]);
      asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(q), "l"(v) : "memory");
    }
}

// numpy's argmax order as a 64-bit key: ord(value) << 32 | ~index (-0 = +0, NaN largest).
__device__ __forceinline__ unsigned long long amax_key(float v, uint32_t i) {
  uint32_t b = __float_as_uint(v);
  if ((b & 0x7FFFFFFFu) == 0u) b = 0u;
  const uint32_t o = (b & 0x7FFFFFFFu) > 0x7F800000u ? 0xFFFFFFFFu
                     : (b & 0x80000000u)             ? ~b
                                                     : (b | 0x80000000u);
  return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - i);
}

// Sum of the class path over lanes for one 8-row block (gemv.cu class_reduce<1>): the total of
// row 2t + (lane bit 4), owned by lanes with bits 2 and 3 clear.
__device__ __forceinline__ long long class_reduce8(long long v0, long long v1, int lane) {
  const bool b4 = (lane & 16) != 0;
  long long u = (b4 ? v1 : v0) + __shfl_xor_sync(0xFFFFFFFFu, b4 ? v0 : v1, 16);
  u += __shfl_xor_sync(0xFFFFFFFFu, u, 8);
  u += __shfl_xor_sync(0xFFFFFFFFu, u, 4);
  return u;
}

// The 4-bit input row: x' = x * 2^(-4 (k mod 4)) and the groups' sums, from plain fp32 x or from
// tagged words (read until their tags reach `expect`). The compute threads meet at the end.
__device__ void stage_x4(const float* x, const unsigned long long* xt, uint32_t expect, int K,
                         float* xs, float* xsum, int* status, uint32_t limit) {
  const int tid = threadIdx.x;
  for (int i = tid; i < K / 4; i += kCT) {   // K / 4 is a multiple of 32: whole warps
    float4 v;
    if (xt != nullptr) {
      unsigned long long w[4];
      ld_tagged2(xt + 4 * i, w[0], w[1]);
      ld_tagged2(xt + 4 * i + 2, w[2], w[3]);
      for (uint32_t spin = 0; behind(w[0], expect) || behind(w[1], expect) || behind(w[2], expect) ||
                              behind(w[3], expect);
           ++spin) {
        if (spin >= limit) {
          atomicOr(status, kStatusTimeout);
          break;
        }
        if (spin >= 16) __nanosleep(32);
        ld_tagged2(xt + 4 * i, w[0], w[1]);
        ld_tagged2(xt + 4 * i + 2, w[2], w[3]);
      }
      v = make_float4(__uint_as_float(static_cast<uint32_t>(w[0])), __uint_as_float(static_cast<uint32_t>(w[1])),
                      __uint_as_float(static_cast<uint32_t>(w[2])), __uint_as_float(static_cast<uint32_t>(w[3])));
    } else {
      v = ld_cg4(x + 4 * i);
    }
    *reinterpret_cast<float4*>(xs + 4 * i) =
        make_float4(v.x, v.y * 0.0625f, v.z * 0.00390625f, v.w * 0.000244140625f);
    float sum = (v.x + v.y) + (v.z + v.w);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
    if ((tid & 7) == 0) xsum[i >> 3] = sum;
  }
  cbar();
}

// Sum over the 16 elements of a group that one 64-bit piece of codes holds, against x' (nibble p
// of each 16-bit half masked in place under 2^23's exponent: 2^23 + u 16^p; less 2^23, times
// x'[k] = x[k] 16^-p: u x[k], u = code + 8).
__device__ __forceinline__ float dot16(uint32_t w0, uint32_t w1, const float* xq) {
  w0 ^= 0x88888888u;
  w1 ^= 0x88888888u;
  const float4 a = *reinterpret_cast<const float4*>(xq);
  const float4 b = *reinterpret_cast<const float4*>(xq + 4);
  const float4 c = *reinterpret_cast<const float4*>(xq + 8);
  const float4 d = *reinterpret_cast<const float4*>(xq + 12);
  constexpr float kB = 8388608.0f;
  float s = 0.0f;
  uint32_t h = w0;
  s = fmaf(__uint_as_float((h & 0xFu) | 0x4B000000u) - kB, a.x, s);
  s = fmaf(__uint_as_float((h & 0xF0u) | 0x4B000000u) - kB, a.y, s);
  s = fmaf(__uint_as_float((h & 0xF00u) | 0x4B000000u) - kB, a.z, s);
  s = fmaf(__uint_as_float((h & 0xF000u) | 0x4B000000u) - kB, a.w, s);
  h = w0 >> 16;
  s = fmaf(__uint_as_float((h & 0xFu) | 0x4B000000u) - kB, b.x, s);
  s = fmaf(__uint_as_float((h & 0xF0u) | 0x4B000000u) - kB, b.y, s);
  s = fmaf(__uint_as_float((h & 0xF00u) | 0x4B000000u) - kB, b.z, s);
  s = fmaf(__uint_as_float((h & 0xF000u) | 0x4B000000u) - kB, b.w, s);
  h = w1;
  s = fmaf(__uint_as_float((h & 0xFu) | 0x4B000000u) - kB, c.x, s);
  s = fmaf(__uint_as_float((h & 0xF0u) | 0x4B000000u) - kB, c.y, s);
  s = fmaf(__uint_as_float((h & 0xF00u) | 0x4B000000u) - kB, c.z, s);
  s = fmaf(__uint_as_float((h & 0xF000u) | 0x4B000000u) - kB, c.w, s);
  h = w1 >> 16;
  s = fmaf(__uint_as_float((h & 0xFu) | 0x4B000000u) - kB, d.x, s);
  s = fmaf(__uint_as_float((h & 0xF0u) | 0x4B000000u) - kB, d.y, s);
  s = fmaf(__uint_as_float((h & 0xF00u) | 0x4B000000u) - kB, d.z, s);
  s = fmaf(__uint_as_float((h & 0xF000u) | 0x4B000000u) - kB, d.w, s);
  return s;
}

__device__ __forceinline__ float half_to_float(uint16_t h) {
  float f;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
  return f;
}

__global__ void __launch_bounds__(kTh, 1) step_kernel(const StepTable* __restrict__ Tp) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ long long s_delta[kMaxWorld];
  __shared__ float s_Sa;
  __shared__ int s_flag;
  __shared__ unsigned int s_seq;
  const StepTable& T = *Tp;
  const SSmem s = carve(smem_raw, T);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NS = T.ns, SB = T.stage_bytes;
  const int count = T.count;

  for (int i = threadIdx.x; i < count * 16; i += kTh)
    reinterpret_cast<uint32_t*>(s.info)[i] = __ldg(reinterpret_cast<const uint32_t*>(T.info) + i);
  if (threadIdx.x < kMaxWorld) s_delta[threadIdx.x] = threadIdx.x < T.world ? T.delta[threadIdx.x] : 0;
  if (threadIdx.x == 0) {
    s_seq = *reinterpret_cast<volatile unsigned int*>(T.counters);
    for (int i = 0; i < NS; ++i) {
      mbar_init(smem_addr(s.full + i), 1);
      mbar_init(smem_addr(s.empty + i), kCW);
    }
    mbar_init_fence();
  }
  __syncthreads();
  const uint32_t ring_s = smem_addr(s.ring);

  if (warp == kCW) {
    // ---------------------------------------------------------------- the producer warp
    if (lane == 0) {
      int item = 0;
      for (int p = 0; p < count; ++p) {
        const SInfo& d = s.info[p];
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&T.map[p])) : "memory");
        int b0, b1;
        cta_blocks(d.N, b0, b1);
        const uint32_t bytes = 8u * d.cb * (kChunkB + (d.fmt == kFmtG32 ? 16u : 0u));
        for (int b = b0; b < b1; ++b)
          for (int cg = 0; cg < d.ngr; ++cg, ++item) {
            const int st = item % NS, use = item / NS;
            if (use > 0 && !mbar_wait(smem_addr(s.empty + st), static_cast<uint32_t>((use - 1) & 1), T.status))
              continue;   // a consumer never released the stage: this item is skipped (status set)
            const uint32_t fb = smem_addr(s.full + st);
            mbar_arrive_expect_tx(fb, bytes);
            tma_3d(ring_s + st * SB, &T.map[p], 0, b * 8, cg * kCB, fb);
            if (d.fmt == kFmtG32) tma_2d(ring_s + st * SB + kCodeStage, &T.smap[p], cg * kCB * 16, b * 8, fb);
          }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ the compute warps
  const int g = lane >> 2, t = lane & 3;
  const uint32_t base = s_seq * kTagStride;
  const uint32_t limit = g_step_wait_limit;
  const bool fused_amax = T.token != nullptr && T.world == 1;
  unsigned long long best = 0;   // this thread's largest head key (fused argmax)
  bool ok = true;
  int item_base = 0;             // the CTA's items before projection p

  for (int p = 0; p < count; ++p) {
    const SInfo& d = s.info[p];
    const int K = d.K, N = d.N;
    int b0, b1;
    cta_blocks(N, b0, b1);
    if (b0 == b1) continue;   // no rows here: this CTA neither reads the input nor computes
    const bool g32 = d.fmt == kFmtG32;
    const bool unit = d.srows == nullptr;
    // the row scales of this CTA's rows (they never depend on the input: loaded while it is
    // awaited; ordered before their use by the barriers below)
    const int row0 = b0 * 8, nrows = min(b1 * 8, N) - row0;
    if (!g32)
      for (int i = threadIdx.x; i < nrows; i += kCT)
        s.sws[i] = unit ? 1.0f : __ldg(reinterpret_cast<const float*>(d.srows + static_cast<long long>(row0 + i) * d.srs));
    // ---- the input row
    const bool tagged = d.in >= 0;
    const unsigned long long* xt = tagged ? T.words + s.info[d.in].out : nullptr;
    const uint32_t expect = base + static_cast<uint32_t>(d.in + 1);
    float Sa = 0.0f;
    bool cls_path = true;
    if (g32) {
      stage_x4(T.x0, xt, expect, K, s.xs, s.xsum, T.status, limit);
    } else {
      if (threadIdx.x == 0) s_flag = 0;
      qact_row4<kCT, 1>(
          T.x0, true, s.xs, K, false, s.segm, s.qred,
          [&](int i, int q0, int q1, int q2, int q3, int da) {
            const int G = i >> 3;
            if ((threadIdx.x & 7) == 0) {
              s.cls[G] = static_cast<uint8_t>(da < 16 ? da : 255);
              s.dg[G] = static_cast<uint8_t>(da);
              if (da == 16) s_flag = 1;
            }
            *reinterpret_cast<uint32_t*>(s.act + 4 * i) =
                (q0 & 0xFFu) | ((q1 & 0xFFu) << 8) | ((q2 & 0xFFu) << 16) | (static_cast<uint32_t>(q3 & 0xFF) << 24);
          },
          xt, expect, T.status, &s_Sa, limit);
      Sa = s_Sa;
      cls_path = s_flag == 0;
    }
    const uint32_t tag = base + static_cast<uint32_t>(p + 1);
    unsigned long long* const yw = T.words + d.out + static_cast<long long>(T.rank) * N;
    const bool last = p == count - 1;

    // one item's stage: wait for it, and release it to the producer
    auto item_wait = [&](int it) -> const uint8_t* {
      const int st = it % NS;
      if (!mbar_wait(smem_addr(s.full + st), static_cast<uint32_t>((it / NS) & 1), T.status)) ok = false;
      return s.ring + static_cast<size_t>(st) * SB;
    };
    auto item_release = [&](int it, uint32_t n) {
      __syncwarp();
      if (lane == 0) mbar_arrive_n(smem_addr(s.empty + it % NS), n);
    };
    // int8 chunk k (a 1 KB swizzled sub-stage) into the class / general accumulators
    auto chunk8 = [&](const uint8_t* st, int k, int (&D)[4], long long (&acc)[2]) {
      const uint8_t* row = st + g * kChunkB;
#pragma unroll
      for (int sg = 0; sg < 4; ++sg) {
        const int G = k * 4 + sg;
        const uint2 qv = *reinterpret_cast<const uint2*>(s.act + 32 * G + 8 * t);
        const int piece = (2 * sg + (t >> 1)) ^ g;
        const uint2 bv = *reinterpret_cast<const uint2*>(row + 16 * piece + 8 * (t & 1));
        if (cls_path) {
          const int c = s.cls[G];
          imma_acc(c == g ? qv.x : 0u, c == g + 8 ? qv.x : 0u, c == g ? qv.y : 0u,
                   c == g + 8 ? qv.y : 0u, bv.x, bv.y, D);
        } else {
          int dd[4] = {0, 0, 0, 0};
          imma_acc(g == 0 ? qv.x : 0u, 0u, g == 0 ? qv.y : 0u, 0u, bv.x, bv.y, dd);
          const int sh = 16 - static_cast<int>(s.dg[G]);
          const long long m = sh >= 0 ? (1ll << sh) : 0ll;
          acc[0] += static_cast<long long>(dd[0]) * m;
          acc[1] += static_cast<long long>(dd[1]) * m;
        }
      }
    };
    // 4-bit chunk k (codes sub-stage st; sc: this lane's two fp16 scales) for lane (row g,
    // quarter t: bytes 32t .. 32t + 31 of the row's chunk, groups 2t and 2t + 1)
    auto chunk4 = [&](const uint8_t* st, const uint8_t* sc, int k, float& acc) {
      const uint8_t* row = st + g * kChunkB;
      const uint4 c0 = *reinterpret_cast<const uint4*>(row + 16 * ((2 * t) ^ g));
      const uint4 c1 = *reinterpret_cast<const uint4*>(row + 16 * ((2 * t + 1) ^ g));
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(sc);
      const int G = k * 8 + 2 * t;
      const float* xq = s.xs + k * 256 + 64 * t;
      const float s0 = fmaf(-8.0f, s.xsum[G], dot16(c0.x, c0.y, xq) + dot16(c0.z, c0.w, xq + 16));
      const float s1 = fmaf(-8.0f, s.xsum[G + 1], dot16(c1.x, c1.y, xq + 32) + dot16(c1.z, c1.w, xq + 48));
      acc = fmaf(half_to_float(static_cast<uint16_t>(sw & 0xFFFFu)), s0, acc);
      acc = fmaf(half_to_float(static_cast<uint16_t>(sw >> 16)), s1, acc);
    };
    auto store_row = [&](int row, float y) {
      if (ok) st_word(yw + row, __float_as_uint(y) | (static_cast<unsigned long long>(tag) << 32), T.world, T.rank, s_delta);
      if (fused_amax && last) {
        const unsigned long long k = amax_key(y, static_cast<uint32_t>(T.rank * N + row));
        best = k > best ? k : best;
      }
    };

    if (d.split == 8) {
      // the warps share each block's chunks: warp w takes sub-stage w of every item
      for (int pass0 = b0; pass0 < b1; pass0 += kMaxRedBlocks) {
        const int pass1 = min(b1, pass0 + kMaxRedBlocks);
        for (int b = pass0; b < pass1; ++b) {
          int D[4] = {0, 0, 0, 0};
          long long acc[2] = {0, 0};
          float facc = 0.0f;
          for (int cg = 0; cg < d.ngr; ++cg) {
            const int it = item_base + (b - b0) * d.ngr + cg;
            const uint8_t* stg = item_wait(it);
            const int k = cg * kCB + warp;
            if (warp < d.cb && k < d.kch && ok) {
              if (g32) chunk4(stg + warp * 1024, stg + kCodeStage + g * (16 * d.cb) + warp * 16 + 4 * t, k, facc);
              else chunk8(stg + warp * 1024, k, D, acc);
            }
            item_release(it, 1);
          }
          long long* red = s.red + (static_cast<size_t>(b - pass0) * kCW + warp) * 8;
          if (g32) {
            facc += __shfl_xor_sync(0xFFFFFFFFu, facc, 1);
            facc += __shfl_xor_sync(0xFFFFFFFFu, facc, 2);
            if (t == 0) reinterpret_cast<float*>(red)[g] = facc;
          } else if (cls_path) {
            const long long mlo = 1ll << (16 - g), mhi = 1ll << (8 - g);
            const long long v0 = static_cast<long long>(D[0]) * mlo + static_cast<long long>(D[2]) * mhi;
            const long long v1 = static_cast<long long>(D[1]) * mlo + static_cast<long long>(D[3]) * mhi;
            const long long tot = class_reduce8(v0, v1, lane);
            if ((lane & 12) == 0) red[2 * t + ((lane >> 4) & 1)] = tot;
          } else if (g == 0) {
            red[2 * t] = acc[0];
            red[2 * t + 1] = acc[1];
          }
        }
        cbar();
        for (int i = threadIdx.x; i < (pass1 - pass0) * 8; i += kCT) {
          const int bl = i >> 3, r = i & 7;
          const int row = (pass0 + bl) * 8 + r;
          if (row >= N) continue;
          float y;
          if (g32) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) tot += reinterpret_cast<const float*>(s.red + (static_cast<size_t>(bl) * kCW + w) * 8)[r];
            y = tot;
          } else {
            long long tot = 0;
#pragma unroll
            for (int w = 0; w < kCW; ++w) tot += s.red[(static_cast<size_t>(bl) * kCW + w) * 8 + r];
            y = mm_epilogue(tot, s.sws[row - row0], Sa, 16);
          }
          store_row(row, y);
        }
        cbar();   // red is reused by the next pass
      }
    } else {
      // a warp owns whole blocks
      for (int b = b0 + warp; b < b1; b += kCW) {
        int D[4] = {0, 0, 0, 0};
        long long acc[2] = {0, 0};
        float facc = 0.0f;
        for (int cg = 0; cg < d.ngr; ++cg) {
          const int it = item_base + (b - b0) * d.ngr + cg;
          const uint8_t* stg = item_wait(it);
          if (ok) {
            for (int j = 0; j < d.cb; ++j) {
              const int k = cg * kCB + j;
              if (k >= d.kch) break;
              if (g32) chunk4(stg + j * 1024, stg + kCodeStage + g * (16 * d.cb) + j * 16 + 4 * t, k, facc);
              else chunk8(stg + j * 1024, k, D, acc);
            }
          }
          item_release(it, kCW);
        }
        if (g32) {
          facc += __shfl_xor_sync(0xFFFFFFFFu, facc, 1);
          facc += __shfl_xor_sync(0xFFFFFFFFu, facc, 2);
          if (t == 0 && b * 8 + g < N) store_row(b * 8 + g, facc);
        } else if (cls_path) {
          const long long mlo = 1ll << (16 - g), mhi = 1ll << (8 - g);
          const long long v0 = static_cast<long long>(D[0]) * mlo + static_cast<long long>(D[2]) * mhi;
          const long long v1 = static_cast<long long>(D[1]) * mlo + static_cast<long long>(D[3]) * mhi;
          const long long tot = class_reduce8(v0, v1, lane);
          const int row = b * 8 + 2 * t + ((lane >> 4) & 1);
          if ((lane & 12) == 0 && row < N) store_row(row, mm_epilogue(tot, s.sws[row - row0], Sa, 16));
        } else if (g == 0) {
          for (int h = 0; h < 2; ++h) {
            const int row = b * 8 + 2 * t + h;
            if (row < N) store_row(row, mm_epilogue(acc[h], s.sws[row - row0], Sa, 16));
          }
        }
      }
    }
    item_base += (b1 - b0) * d.ngr;
    cbar();   // act / cls / xs / sws are rewritten by the next projection
  }

  // ---- the greedy token
  if (T.token != nullptr) {
    if (!fused_amax) {
      // several GPUs: the whole tagged logit row, every rank's part, once it has arrived
      const SInfo& h = s.info[count - 1];
      const unsigned long long* row = T.words + h.out;
      const uint32_t want = base + static_cast<uint32_t>(count);
      for (int i = blockIdx.x * kCT + threadIdx.x; i < h.nfull; i += gridDim.x * kCT) {
        unsigned long long w = *reinterpret_cast<const volatile unsigned long long*>(row + i);
        for (uint32_t spin = 0; behind(w, want); ++spin) {
          if (spin >= limit) {
            atomicOr(T.status, kStatusTimeout);
            break;
          }
          if (spin >= 16) __nanosleep(32);
          w = *reinterpret_cast<const volatile unsigned long long*>(row + i);
        }
        const unsigned long long k = amax_key(__uint_as_float(static_cast<uint32_t>(w)), static_cast<uint32_t>(i));
        best = k > best ? k : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long v = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      best = v > best ? v : best;
    }
    unsigned long long* part = reinterpret_cast<unsigned long long*>(s.qred);
    if (lane == 0) part[warp] = best;
    cbar();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kCW; ++w) best = part[w] > best ? part[w] : best;
      atomicMax(T.amax, best);
    }
  }
  // ---- the last CTA to finish: the token, the accumulator cleared, the step counted
  cbar();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(T.counters + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      __threadfence();
      if (T.token != nullptr) {
        const unsigned long long k = atomicExch(T.amax, 0ull);
        *T.token = static_cast<long long>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
      }
      T.counters[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile int*>(T.counters) = static_cast<int>(s_seq + 1);
    }
  }
}

PFN_cuTensorMapEncodeTiled tensor_encoder() {
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return nullptr;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  return encode;
}

// The rows as {128 bytes, N rows, chunks}: a box is 8 rows x cb chunks, one 1 KB swizzled
// sub-stage a chunk.
bool encode_rows3(CUtensorMap* map, const uint8_t* rows, int64_t row_bytes, int64_t N, int64_t rs,
                  int cb) {
  PFN_cuTensorMapEncodeTiled enc = tensor_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kChunkB), static_cast<cuuint64_t>(N),
                              static_cast<cuuint64_t>(row_bytes / kChunkB)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(rs), static_cast<cuuint64_t>(kChunkB)};
  const cuuint32_t box[3] = {kChunkB, 8, static_cast<cuuint32_t>(cb)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(rows), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-bit scales as bytes {K/16, N rows}: a box is 8 rows x 16 cb bytes (the block's scales of cb
// chunks), unswizzled.
bool encode_scales(CUtensorMap* map, const uint8_t* sc, int64_t K, int64_t N, int64_t ss, int cb) {
  PFN_cuTensorMapEncodeTiled enc = tensor_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 16), static_cast<cuuint64_t>(N)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ss)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(16 * cb), 8};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(sc), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Layout {
  int kmax, redb, maxrows, stage_bytes, ns;
  size_t smem;
};

// The shared-memory layout of a step (computed alike at prepare and at launch).
int step_layout_of(const otq_step* st, int sms, Layout* L) {
  int kmax = 128, redb = 1, maxrows = 8;
  bool any4 = false;
  for (int i = 0; i < st->count; ++i) {
    const otq_step_proj& q = st->projs[i];
    const int nb = static_cast<int>((q.N + 7) / 8);
    const int per_cta = (nb + sms - 1) / sms;
    const bool owner = per_cta >= 2 * kCW;
    kmax = kmax > q.K ? kmax : static_cast<int>(q.K);
    if (!owner) redb = redb > per_cta ? redb : per_cta;
    maxrows = maxrows > per_cta * 8 ? maxrows : per_cta * 8;
    any4 = any4 || q.fmt == OTQ_STEP_G32;
  }
  L->kmax = kmax;
  L->redb = redb < kMaxRedBlocks ? redb : kMaxRedBlocks;
  L->maxrows = maxrows;
  L->stage_bytes = kCodeStage + (any4 ? kScaleStage : 0);
  const size_t budget = 227 * 1024 - 512;   // dynamic + the kernel's static shared memory
  const size_t fixed = step_smem(st->count, kmax, L->redb, maxrows, 0, L->stage_bytes, nullptr);
  if (fixed + 2 * (L->stage_bytes + 16) > budget) return kErrArg;
  int ns = static_cast<int>((budget - fixed) / (L->stage_bytes + 16));
  while (ns > 2 && step_smem(st->count, kmax, L->redb, maxrows, ns, L->stage_bytes, nullptr) > budget) --ns;
  if (ns < 2) return kErrArg;
  L->ns = ns;
  L->smem = step_smem(st->count, kmax, L->redb, maxrows, ns, L->stage_bytes, nullptr);
  return kOk;
}

}  // namespace

// Word offsets of every projection's output row in the step's buffer (16-byte aligned slots).
int step_layout(const otq_step_proj* pr, int count, int world, int64_t* offsets, int64_t* total) {
  if (pr == nullptr || count < 1 || count > kMaxProj || world < 1 || world > kMaxWorld || total == nullptr)
    return kErrArg;
  int64_t off = 0;
  for (int i = 0; i < count; ++i) {
    if (offsets) offsets[i] = off;
    off += ((pr[i].N * world + 1) / 2) * 2;
  }
  *total = off;
  return kOk;
}

int64_t step_table_bytes() { return static_cast<int64_t>(sizeof(StepTable)); }

int set_step_wait_limit(uint32_t polls) {
  const uint32_t v = polls == 0 ? (1u << 22) : polls;
  return cudaMemcpyToSymbol(g_step_wait_limit, &v, sizeof(v)) == cudaSuccess ? kOk : kErrCuda;
}

int step_prepare(const otq_step* st, void* table) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrCuda;
  const int sms = sm_count(dev);
  Layout L;
  if (step_layout_of(st, sms, &L) != kOk) return kErrArg;
  std::unique_ptr<StepTable> hold(new StepTable);
  StepTable& T = *hold;
  std::memset(&T, 0, sizeof(T));
  const int count = st->count;
  int64_t offs[kMaxProj], total = 0;
  if (step_layout(st->projs, count, st->world, offs, &total) != kOk) return kErrArg;
  if (total >= (int64_t{1} << 31)) return kErrArg;
  for (int i = 0; i < count; ++i) {
    const otq_step_proj& q = st->projs[i];
    SInfo& d = T.info[i];
    const bool g32 = q.fmt == OTQ_STEP_G32;
    const int64_t row_bytes = g32 ? q.K / 2 : q.K;
    d.kch = static_cast<int>(row_bytes / kChunkB);
    d.cb = d.kch < kCB ? d.kch : kCB;
    d.ngr = (d.kch + kCB - 1) / kCB;
    if (!encode_rows3(&T.map[i], q.rows, row_bytes, q.N, q.rs, d.cb)) return kErrCuda;
    if (g32 && !encode_scales(&T.smap[i], q.srows, q.K, q.N, q.srs, d.cb)) return kErrCuda;
    d.srows = g32 ? nullptr : q.srows;
    d.srs = static_cast<int>(q.srs);
    d.N = static_cast<int>(q.N);
    d.K = static_cast<int>(q.K);
    d.fmt = q.fmt;
    d.in = q.in;
    d.out = static_cast<int>(offs[i]);
    d.nfull = static_cast<int>(q.N * st->world);
    const int nb = static_cast<int>((q.N + 7) / 8);
    d.split = (nb + sms - 1) / sms >= 2 * kCW ? 1 : 8;
  }
  T.count = count;
  T.world = st->world;
  T.rank = st->rank;
  T.ns = L.ns;
  T.kmax = L.kmax;
  T.redb = L.redb;
  T.maxrows = L.maxrows;
  T.stage_bytes = L.stage_bytes;
  T.x0 = st->x0;
  T.words = reinterpret_cast<unsigned long long*>(st->out);
  for (int r = 0; r < kMaxWorld; ++r) T.delta[r] = r < st->world ? st->delta[r] : 0;
  T.counters = st->counters;
  T.amax = reinterpret_cast<unsigned long long*>(st->counters + 2);
  T.token = reinterpret_cast<long long*>(st->token);
  T.status = status_word();
  if (T.status == nullptr) return kErrCuda;
  return cudaMemcpy(table, &T, sizeof(T), cudaMemcpyHostToDevice) == cudaSuccess ? kOk : kErrCuda;
}

int step_launch(const otq_step* st, const void* table, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrCuda;
  const int sms = sm_count(dev);
  Layout L;
  if (step_layout_of(st, sms, &L) != kOk) return kErrArg;
  static size_t configured[kMaxDevices] = {0};
  if (configured[dev] < L.smem) {
    if (cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(L.smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = L.smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms), 1, 1);   // one CTA an SM, all resident
  cfg.blockDim = dim3(kTh, 1, 1);
  cfg.dynamicSmemBytes = L.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const StepTable* tp = static_cast<const StepTable*>(table);
  void* args[] = {&tp};
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(step_kernel), args) == cudaSuccess ? kOk
                                                                                               : kErrCuda;
}

}  // namespace otq
