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
// Weight streaming. One producer warp a CTA walks the CTA's items -- an item is one 16-row tile
// of a projection and up to 8 chunks of its K (128 bytes of a row a chunk), ONE 3-D tensor copy
// of up to 16 KB with the 128-byte swizzle (plus, for 4-bit rows, a 2-D copy of the tile's fp16
// group scales) -- in the order the CTA computes them, across projection boundaries, into a ring
// of shared-memory stages (full / empty mbarriers). Weights never depend on activations, so
// while the CTA waits for projection p's input the weights of the next projections arrive. (One
// tensor copy a 1 KB box, issued by the computing warps themselves, measured 0.3-0.5 us of issue
// stall a copy on a B200: far fewer, larger copies from a warp that does nothing else.)
//
// Work split. A projection's 16-row tiles go in balanced ranges to the CTAs (one CTA an SM, all
// resident: cooperative launch). Within a CTA either the 8 compute warps share each tile's K
// chunks (fewer than 8 tiles; the warps' row totals meet in shared memory) or each warp owns
// whole tiles, int8 two at a time (the LM head).
//
// Arithmetic, int8 rows: a group's multiplier 2^(16 - d) depends on the activation only (its
// QACT offset d). One mma.sync m16n8k32 (s8) a group and tile: A = the tile's 16 weight rows,
// B = the group's activation bytes in column (d mod 8) of accumulator set d / 8, zero in the
// other columns; each accumulator column is one offset class, exact in int32; a row's total is
// sum over columns of D * 2^(16 - class) in int64 after two lane shuffles. Offsets above 16
// drop out (the MM window). Epilogue (i2f(acc) * Sw) * (Sa * 2^-16), three flushed RNE
// products: bit-identical to otq_qmm. 4-bit rows: x is staged once per projection as x'[k] =
// x[k] * 2^(-4 (k mod 4)) with each group's sum of x, so a nibble masked in place under 2^23's
// exponent, less 2^23, times x' is (code + 8) * x; a group adds s * (sum - 8 sum x).
//
// Decoder stages: a projection's input may be the RMSNorm of the residual row (each CTA keeps
// the residual in shared memory and adds the named projection's output to it) or SwiGLU of an
// earlier output; the GateUp projection may write SwiGLU itself (OTQ_EPI_SWIGLU); an attention
// stage runs the new token's attention over the KV cache in chunks spread over the CTAs and
// combines them (attn_stage).
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
constexpr int kTR = 16;                      // rows a tile (the M of an mma.sync m16n8k32)
constexpr int kSub = kTR * kChunkB;          // 2 KB: a tile's chunk, one swizzled sub-stage
constexpr int kCodeStage = kCB * kSub;       // 16 KB: 16 rows x 8 chunks
constexpr int kScaleStage = kTR * kCB * 16;  // 2 KB: 16 rows x 8 chunks x 8 fp16 scales
constexpr int kMaxProj = OTQ_STEP_MAX;
constexpr uint32_t kTagStride = 1024;
constexpr int kMaxWorld = 8;
constexpr int kFmtG32 = OTQ_STEP_G32;
constexpr int kFmtAttn = OTQ_STEP_ATTN;
constexpr int kInDefault = OTQ_IN_DEFAULT;
constexpr int kInNorm = OTQ_IN_NORM;
constexpr int kInSwiglu = OTQ_IN_SWIGLU;
constexpr int kInAttn = OTQ_IN_ATTN;
constexpr int kEpiSwiglu = OTQ_EPI_SWIGLU;
constexpr int kHd = 128;                     // attention head dimension
constexpr int kMaxG = 4;                     // query heads a KV head
constexpr int kAttnChunk = 32;               // positions an attention item

__device__ uint32_t g_step_wait_limit = 1u << 22;

struct SInfo {            // one stage, as the kernel reads it (shared memory)
  const uint8_t* srows;   // int8: scale rows, Sw the first fp32 word (null: UNIT)
  const float* gamma;     // OTQ_IN_NORM: the norm's gains
  int srs;
  int N;                  // this rank's rows
  int K;
  int fmt;
  int split;              // unused
  int in;                 // -1: the plain input x0; else the projection whose output is x
  int out;                // word offset of this projection's full output row
  int nfull;              // the full row's length (N * world)
  int kch;                // chunks a row
  int cb;                 // chunks an item (min(8, kch))
  int ngr;                // items a block (ceil(kch / cb))
  int input;              // OTQ_IN_*
  int res;                // OTQ_IN_NORM: -2 (start from x0) or the projection added first
  int epi;                // OTQ_EPI_*
  int rep;                // world > 1 and every rank computes all rows (no NVLink stores)
  int pad[1];
};
static_assert(sizeof(SInfo) == 80, "SInfo is 80 bytes");

struct SAttn {            // an attention stage's operands
  const float* qg;        // q / k per-head norm gains (null: none)
  const float* kg;
  float* kc;              // [max_pos][n_kv][hd]
  float* vc;
  int nq, nkv, maxch, pad;
};

struct alignas(16) StepHead {   // the scalars and pointers of a step (the kernel keeps a copy in shared memory)
  int count, world, rank, ns, kmax, redb, maxrows, stage_bytes;
  const float* x0;
  unsigned long long* words;
  long long delta[kMaxWorld];
  int* counters;                 // [0] steps completed, [1] CTAs done
  unsigned long long* amax;      // the head's key accumulator (0 between steps)
  long long* token;
  int* status;
  float eps;
  int max_pos;
  const float* rope_cos;         // [max_pos][hd / 2]
  const float* rope_sin;
  int* pos;                      // this step's position (null: no attention)
  const float* embed;            // x0 = embed[*token_in] (null: x0)
  const long long* token_in;
  int hmax;                      // the residual row's length (0: none)
  int ascr;                      // floats of the attention combine's scratch
};
static_assert(sizeof(StepHead) % 16 == 0, "StepHead is copied in 16-byte words");

struct StepTable : StepHead {
  SInfo info[kMaxProj];
  SAttn attn[kMaxProj];
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
  long long* red;    // [kCW][16] the warps' row totals of a shared tile (4-bit: floats)
  float* sws;        // [maxrows] Sw of this CTA's rows of the projection
  float* xr;         // [hmax] the residual row (this CTA's copy)
  float* aq;         // [kMaxG][kHd] attention: the query heads, normed and rotated
  float* akv;        // [2][kHd] the new key (normed, rotated) and value
  float* asc;        // [kMaxG][kAttnChunk] scores, then their exponentials
  float* ascr;       // [ascr] the attention combine's (m, l) pairs and weights
  uint64_t* full;    // [ns]
  uint64_t* empty;   // [ns]
  uint8_t* ring;     // [ns][stage_bytes], 1024-byte aligned
};

// The shared-memory layout: every region at a fixed offset (sized for the largest step this
// kernel takes), so that the kernel addresses them as constants off one base; the ring of
// stages follows, 1024-byte aligned, as many stages as the rest of the 227 KB holds.
constexpr int kKcap = 8192;       // the longest input row (K)
constexpr int kHcap = 4096;       // the longest residual row (a norm's K)
constexpr int kRowsCap = 2048;    // a CTA's rows of one projection
constexpr int kNScap = 32;        // ring stages
constexpr int kAscrCap = 2048;    // floats of the attention combine's scratch (2 G maxch)
constexpr size_t al16(size_t x) { return (x + 15) & ~size_t(15); }
constexpr size_t kOffInfo = 0;
constexpr size_t kOffAct = al16(kOffInfo + kMaxProj * sizeof(SInfo));
constexpr size_t kOffCls = al16(kOffAct + kKcap);
constexpr size_t kOffDg = al16(kOffCls + kKcap / 32);
constexpr size_t kOffXs = al16(kOffDg + kKcap / 32);
constexpr size_t kOffXsum = al16(kOffXs + kKcap * 4);
constexpr size_t kOffSegm = al16(kOffXsum + kKcap / 32 * 4);
constexpr size_t kOffQred = al16(kOffSegm + kKcap / 32 * 4);
constexpr size_t kOffRed = al16(kOffQred + (kCW + 8) * 4);
constexpr size_t kOffSws = al16(kOffRed + static_cast<size_t>(kCW) * kTR * 8);
constexpr size_t kOffFull = al16(kOffSws + kRowsCap * 4);
constexpr size_t kOffEmpty = al16(kOffFull + kNScap * 8);
constexpr size_t kOffXr = al16(kOffEmpty + kNScap * 8);
constexpr size_t kOffAttn = al16(kOffXr + kHcap * 4);
constexpr size_t kOffAscr = al16(kOffAttn + (kMaxG * kHd + 2 * kHd + kMaxG * kAttnChunk) * 4);
constexpr size_t kOffRing = al16(kOffAscr + kAscrCap * 4);
static_assert(2 * kAttnChunk * kHd <= kKcap, "an attention chunk's keys and values fit the row staging");

extern __shared__ __align__(16) unsigned char smem_raw[];   // the step kernel's dynamic shared memory

__device__ __forceinline__ SSmem carve(unsigned char* base) {
  SSmem s;
  s.info = reinterpret_cast<SInfo*>(base + kOffInfo);
  s.act = base + kOffAct;
  s.cls = base + kOffCls;
  s.dg = base + kOffDg;
  s.xs = reinterpret_cast<float*>(base + kOffXs);
  s.xsum = reinterpret_cast<float*>(base + kOffXsum);
  s.segm = reinterpret_cast<uint32_t*>(base + kOffSegm);
  s.qred = reinterpret_cast<uint32_t*>(base + kOffQred);
  s.red = reinterpret_cast<long long*>(base + kOffRed);
  s.sws = reinterpret_cast<float*>(base + kOffSws);
  s.full = reinterpret_cast<uint64_t*>(base + kOffFull);
  s.empty = reinterpret_cast<uint64_t*>(base + kOffEmpty);
  s.xr = reinterpret_cast<float*>(base + kOffXr);
  s.aq = reinterpret_cast<float*>(base + kOffAttn);
  s.akv = s.aq + kMaxG * kHd;
  s.asc = s.akv + 2 * kHd;
  s.ascr = reinterpret_cast<float*>(base + kOffAscr);
  const uint32_t r = smem_addr(base + kOffRing);
  s.ring = base + kOffRing + (((r + 1023u) & ~1023u) - r);
  return s;
}

__device__ __forceinline__ void cbar() {   // the compute warps meet (named barrier 1)
  asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory");
}

// This CTA's 16-row tiles [b0, b1) of a projection of N rows.
__device__ __forceinline__ void cta_tiles(int N, int& b0, int& b1) {
  const int nb = (N + kTR - 1) / kTR;
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
// imma_acc when p != 0 (p the same in every lane: the mma is executed or skipped by the whole warp)
__device__ __forceinline__ void imma_acc_if(uint32_t p, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1, int (&d)[4]) {
  asm("{ .reg .pred q; setp.ne.b32 q, %10, 0;\n"
      "@q mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3}; }"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(p));
}
// 4 bytes global -> shared, asynchronously (completed by cp.async.wait_all)
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// 8 bytes of a ring stage (ordered after the stage's barrier wait: volatile)
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
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


// Four tagged words xt[0..3] (16-byte aligned) as floats, read until their tags reach `expect`
// (bounded: after `limit` polls the status word records a timeout and the values are used).
__device__ __forceinline__ float4 read_tagged4(const unsigned long long* xt, uint32_t expect,
                                               int* status, uint32_t limit) {
  unsigned long long w[4];
  ld_tagged2(xt, w[0], w[1]);
  ld_tagged2(xt + 2, w[2], w[3]);
  for (uint32_t spin = 0;
       behind(w[0], expect) || behind(w[1], expect) || behind(w[2], expect) || behind(w[3], expect);
       ++spin) {
    if (spin >= limit) {
      atomicOr(status, kStatusTimeout);
      break;
    }
    if (spin >= 64) __nanosleep(32);
    ld_tagged2(xt, w[0], w[1]);
    ld_tagged2(xt + 2, w[2], w[3]);
  }
  return make_float4(__uint_as_float(static_cast<uint32_t>(w[0])), __uint_as_float(static_cast<uint32_t>(w[1])),
                     __uint_as_float(static_cast<uint32_t>(w[2])), __uint_as_float(static_cast<uint32_t>(w[3])));
}

// The 4-bit input row as the operands of the group MMAs (the form of otq_linear_g32's tensor-pipe
// kernel): per 32-element group g, xi = rint(x * 2^e_g) with |xi| < 2^30 (e_g from the group's
// largest |x|), four signed base-256 limbs of xi in the MMA's K order at bytes [128 g, 128 g + 128)
// of xs (the group's own 32 floats, read by the same 8 lanes before they write), 2^-e_g in
// xsum[g], and the codes' +8 bias in corr[2 g + t] = 8 sum_k (l_2t + 256 l_2t+1). x comes from
// plain fp32 x, from tagged words (read until their tags reach `expect`), or (both null) from xs
// itself. The compute threads meet at the end.
__device__ void stage_limbs(const float* x, const unsigned long long* xt, uint32_t expect, int K,
                            float* xs, float* xsum, int* corr, int* status, uint32_t limit) {
  const int tid = threadIdx.x;
  uint8_t* const xl = reinterpret_cast<uint8_t*>(xs);
  for (int i = tid; i < K / 4; i += kCT) {   // K / 4 is a multiple of 32: whole warps, 8 lanes a group
    float4 v;
    if (xt != nullptr) {
      v = read_tagged4(xt + 4 * i, expect, status, limit);
    } else if (x == nullptr) {
      v = *reinterpret_cast<const float4*>(xs + 4 * i);
    } else {
      v = ld_cg4(x + 4 * i);
    }
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
    // e = 29 - exponent(m), at most 126: m 2^e in [2^29, 2^30)
    const int e = m > 0.0f ? min(126, 156 - static_cast<int>((__float_as_uint(m) >> 23) & 255u)) : 0;
    const float p2 = __int_as_float((127 + e) << 23);
    int r[4] = {__float2int_rn(__fmul_rn(v.x, p2)), __float2int_rn(__fmul_rn(v.y, p2)),
                __float2int_rn(__fmul_rn(v.z, p2)), __float2int_rn(__fmul_rn(v.w, p2))};
    int l[4][4];   // [limb][element]
#pragma unroll
    for (int el = 0; el < 4; ++el) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        l[j][el] = j < 3 ? ((r[el] + 128) & 255) - 128 : r[el];   // |r| <= 64 for the last
        r[el] = (r[el] - l[j][el]) >> 8;
      }
    }
    int c0 = 0, c1 = 0;
#pragma unroll
    for (int el = 0; el < 4; ++el) {
      c0 += l[0][el] + 256 * l[1][el];
      c1 += l[2][el] + 256 * l[3][el];
    }
    c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 1);
    c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 1);
    c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 2);
    c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 2);
    c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, 4);
    c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, 4);
    // elements 4q .. 4q + 3 of the group (q = i % 8): the even two at K slots b, b + 1 and the
    // odd two at 16 + b, 17 + b, b = 4 (q / 2) + 2 (q % 2) (slots 4t + i hold element 8t + 2i,
    // slots 16 + 4t + i element 8t + 2i + 1)
    const int gq = i >> 3, q = i & 7;
    uint8_t* const gl = xl + gq * 128 + 4 * (q >> 1) + 2 * (q & 1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      *reinterpret_cast<uint16_t*>(gl + j * 32) =
          static_cast<uint16_t>((l[j][0] & 0xFF) | ((l[j][2] & 0xFF) << 8));
      *reinterpret_cast<uint16_t*>(gl + j * 32 + 16) =
          static_cast<uint16_t>((l[j][1] & 0xFF) | ((l[j][3] & 0xFF) << 8));
    }
    if (q == 0) {
      xsum[gq] = __int_as_float((127 - e) << 23);
      corr[2 * gq] = 8 * c0;
      corr[2 * gq + 1] = 8 * c1;
    }
  }
  cbar();
}

__device__ __forceinline__ float half_to_float(uint16_t h) {
  float f;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
  return f;
}

// The compute threads' sum of one float each, in a fixed order (warp shuffles, then the warps'
// sums in warp order): the same bits in every CTA. scratch: kCW floats.
__device__ __forceinline__ float cta_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  cbar();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t += scratch[w];
  cbar();   // scratch is free again
  return t;
}

// OTQ_IN_NORM: the residual row xr (x0 when res == -2: the embedding row of *token_in, or x0;
// else xr + the output words of the projection at word offset `res_out`), then
// xs = (xr / sqrt(mean(xr^2) + eps)) * gamma (the reference's rmsnorm, qwen3.py:715-716).
__device__ void norm_prologue(const StepHead& T, const SSmem& s, const SInfo& d, int res_out,
                              uint32_t expect, uint32_t limit) {
  const int K = d.K;
  const float* x0 = T.embed != nullptr ? T.embed + (*T.token_in) * static_cast<long long>(K) : T.x0;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < K / 4; i += kCT) {
    float4 r;
    if (d.res == -2) {
      r = ld_cg4(x0 + 4 * i);
    } else {
      r = *reinterpret_cast<const float4*>(s.xr + 4 * i);
      const float4 y = read_tagged4(T.words + res_out + 4 * i, expect, T.status, limit);
      r = make_float4(r.x + y.x, r.y + y.y, r.z + y.z, r.w + y.w);
    }
    *reinterpret_cast<float4*>(s.xr + 4 * i) = r;
    ss += (r.x * r.x + r.y * r.y) + (r.z * r.z + r.w * r.w);
  }
  const float den = sqrtf(cta_sum(ss, reinterpret_cast<float*>(s.qred)) / static_cast<float>(K) + T.eps);
  for (int i = threadIdx.x; i < K / 4; i += kCT) {
    const float4 r = *reinterpret_cast<const float4*>(s.xr + 4 * i);
    const float4 g = __ldg(reinterpret_cast<const float4*>(d.gamma) + i);
    *reinterpret_cast<float4*>(s.xs + 4 * i) =
        make_float4((r.x / den) * g.x, (r.y / den) * g.y, (r.z / den) * g.z, (r.w / den) * g.w);
  }
  cbar();
}

// OTQ_IN_SWIGLU: xs = silu(y[0:K]) * y[K:2K] of the output words at `in_out`
// (the reference's (g / (1 + exp(-g))) * u, qwen3.py:741).
__device__ void swiglu_prologue(const StepHead& T, const SSmem& s, int K, int in_out, uint32_t expect,
                                uint32_t limit) {
  for (int i = threadIdx.x; i < K / 4; i += kCT) {
    const float4 g = read_tagged4(T.words + in_out + 4 * i, expect, T.status, limit);
    const float4 u = read_tagged4(T.words + in_out + K + 4 * i, expect, T.status, limit);
    *reinterpret_cast<float4*>(s.xs + 4 * i) =
        make_float4((g.x / (1.0f + expf(-g.x))) * u.x, (g.y / (1.0f + expf(-g.y))) * u.y,
                    (g.z / (1.0f + expf(-g.z))) * u.z, (g.w / (1.0f + expf(-g.w))) * u.w);
  }
  cbar();
}


// rmsnorm of one head (hd values in smem v, a warp) times gains gn (has_g false: none), then
// rotate-half RoPE with this position's tables (lane l holds cos / sin [4 (l & 15) ..])
// (qwen3.py:719-724, 335-346).
__device__ __forceinline__ void head_norm_rope(float* v, bool has_g, float4 gn, float4 c, float4 sv,
                                               float eps, int lane) {
  float4 x = *reinterpret_cast<const float4*>(v + 4 * lane);
  if (has_g) {
    float ss = (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float den = sqrtf(ss / static_cast<float>(kHd) + eps);
    x = make_float4((x.x / den) * gn.x, (x.y / den) * gn.y, (x.z / den) * gn.z, (x.w / den) * gn.w);
  }
  // lanes 0..15 hold elements 0..63 (v1), lanes 16..31 elements 64..127 (v2)
  const float4 other = make_float4(__shfl_xor_sync(0xFFFFFFFFu, x.x, 16), __shfl_xor_sync(0xFFFFFFFFu, x.y, 16),
                                   __shfl_xor_sync(0xFFFFFFFFu, x.z, 16), __shfl_xor_sync(0xFFFFFFFFu, x.w, 16));
  float4 r;
  if (lane < 16) {   // v1 * c - v2 * s
    r = make_float4(x.x * c.x - other.x * sv.x, x.y * c.y - other.y * sv.y, x.z * c.z - other.z * sv.z,
                    x.w * c.w - other.w * sv.w);
  } else {           // v2 * c + v1 * s
    r = make_float4(x.x * c.x + other.x * sv.x, x.y * c.y + other.y * sv.y, x.z * c.z + other.z * sv.z,
                    x.w * c.w + other.w * sv.w);
  }
  __syncwarp();
  *reinterpret_cast<float4*>(v + 4 * lane) = r;
  __syncwarp();
}

// The combine of the attention's nch chunks (flash-decoding), outputs [o0, o1) of the n_q hd
// (o = hq hd + dd, query head hq): with M the largest of query head hq's chunk maxima, chunk c
// weighs e_c = exp(m_c - M) / L, L = sum_c exp(m_c - M) l_c, and output o is sum_c e_c o_c, in
// chunk order. Written as tagged words at `out`: the O projection's input. The whole CTA; the
// chunks' words are awaited by their tags (bounded); every (output, chunk) word is one load of
// one thread, all of a pass in flight at once, and the products meet in shared memory.
__device__ void attn_combine(const StepHead& T, const SSmem& s, const SAttn& a, int nch, int part_out,
                             int out, uint32_t tag, uint32_t limit, bool ok, int o0, int o1) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hq0 = o0 / kHd, nh = (o1 - 1) / kHd - hq0 + 1;   // the query heads touched (<= kCW)
  float* wt = s.ascr;   // [nh][nch] the chunks' weights
  const long long stride = kHd + 2;
  if (warp < nh) {   // warp w, query head hq0 + w: lane c takes chunks c, c + 32, ...
    const unsigned long long* ph = T.words + part_out + static_cast<long long>(hq0 + warp) * a.maxch * stride;
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) {
      unsigned long long w0, w1;
      ld_tagged2(ph + c * stride, w0, w1);
      for (uint32_t spin = 0; behind(w0, tag) || behind(w1, tag); ++spin) {
        if (spin >= limit) {
          atomicOr(T.status, kStatusTimeout);
          break;
        }
        if (spin >= 64) __nanosleep(32);
        ld_tagged2(ph + c * stride, w0, w1);
      }
      const float m = __uint_as_float(static_cast<uint32_t>(w0));
      wt[warp * nch + c] = m;
      if (c < 32) s.asc[warp * kAttnChunk + c] = __uint_as_float(static_cast<uint32_t>(w1));   // l, first pass
      M = fmaxf(M, m);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    float L = 0.0f;
    for (int c = lane; c < nch; c += 32) {
      unsigned long long w0, w1;
      if (c >= 32) ld_tagged2(ph + c * stride, w0, w1);   // past the first pass: l again
      const float l = c < 32 ? s.asc[warp * kAttnChunk + c] : __uint_as_float(static_cast<uint32_t>(w1));
      const float e = expf(wt[warp * nch + c] - M);
      wt[warp * nch + c] = e;
      L += e * l;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, o);
    for (int c = lane; c < nch; c += 32) wt[warp * nch + c] = wt[warp * nch + c] / L;
  }
  cbar();
  const int no = o1 - o0;
  const int per = max(1, kKcap / no);   // chunks a pass (the products fit xs)
  float acc[2] = {0.0f, 0.0f};          // thread i's outputs o0 + i, o0 + i + kCT
  for (int c0 = 0; c0 < nch; c0 += per) {
    const int nc = min(per, nch - c0);
    for (int u = threadIdx.x; u < no * nc; u += kCT) {
      const int o = o0 + u / nc, c = c0 + u % nc;
      const int hq = o / kHd, dd = o % kHd;
      const unsigned long long* pw = T.words + part_out + (static_cast<long long>(hq) * a.maxch + c) * stride + 2 + dd;
      unsigned long long w = *reinterpret_cast<const volatile unsigned long long*>(pw);
      for (uint32_t spin = 0; behind(w, tag); ++spin) {
        if (spin >= limit) {
          atomicOr(T.status, kStatusTimeout);
          break;
        }
        if (spin >= 64) __nanosleep(32);
        w = *reinterpret_cast<const volatile unsigned long long*>(pw);
      }
      s.xs[u] = wt[(hq - hq0) * nch + c] * __uint_as_float(static_cast<uint32_t>(w));
    }
    cbar();
    for (int v = 0; v < 2; ++v) {
      const int oi = threadIdx.x + v * kCT;
      if (oi >= no) break;
      for (int c = 0; c < nc; ++c) acc[v] += s.xs[oi * nc + c];
    }
    cbar();   // xs is refilled by the next pass
  }
  for (int v = 0; v < 2; ++v) {
    const int oi = threadIdx.x + v * kCT;
    if (oi >= no || !ok) break;
    unsigned long long* dst = T.words + out + o0 + oi;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(dst), "l"(__float_as_uint(acc[v]) | (static_cast<unsigned long long>(tag) << 32)) : "memory");
  }
}

// An attention stage: items (chunk c of kAttnChunk positions, KV head h), chunk-major, dealt to
// the CTAs in order. Each reads its query heads, the new key and value (the QKV projection's
// words), normalises and rotates q and k, scores positions [32 c, min(32 c + 32, pos + 1))
// against the cache (the new token's key from shared memory), and stores per query head
// (m, l, o) as tagged words. The item of a head's last chunk also stores the new key and value
// into the caches. Then every CTA combines a slice of the outputs.
__device__ __noinline__ void attn_stage(const StepHead& T, const SAttn& a, int qkv_out, int out,
                                       int pos, uint32_t expect, uint32_t tag, uint32_t limit,
                                       bool ok) {
  const SSmem s = carve(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int part_out = out + a.nq * kHd;   // the partial results
  const int G = a.nq / a.nkv;
  const int nch = pos / kAttnChunk + 1;
  const float* cs = T.rope_cos + static_cast<long long>(pos) * (kHd / 2);
  const float* sn = T.rope_sin + static_cast<long long>(pos) * (kHd / 2);
  const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(kHd));
  for (int item = blockIdx.x; item < a.nkv * nch; item += gridDim.x) {
    const int c = item / a.nkv, h = item % a.nkv;
    const int j0 = c * kAttnChunk, j1 = min(j0 + kAttnChunk, pos + 1);
    // the chunk's cached keys and values (positions before pos) into shared memory, every copy
    // in flight at once: keys at xs[0 ..), values at xs[kAttnChunk * hd ..); warp w copies rows
    // w, w + 8, .., lane l their bytes 16 l .. 16 l + 15
    {
      const int nold = min(j1, pos) - j0;
      const uint32_t kv_s = smem_addr(s.xs) + 16u * static_cast<uint32_t>(lane);
      const long long rstride = static_cast<long long>(a.nkv) * kHd;
      const long long first = (static_cast<long long>(j0) * a.nkv + h) * kHd + 4 * lane;
      for (int r = warp; r < nold; r += kCW) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(kv_s + static_cast<uint32_t>(r) * (kHd * 4)),
                     "l"(a.kc + first + r * rstride) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(kv_s + static_cast<uint32_t>(kAttnChunk + r) * (kHd * 4)),
                     "l"(a.vc + first + r * rstride) : "memory");
      }
    }
    // the head norm's gains and this position's rotation, ahead of their use
    float4 gn = make_float4(1.0f, 1.0f, 1.0f, 1.0f), rc = gn, rs = gn;
    if (warp <= G) {
      const float* gp = warp < G ? a.qg : a.kg;
      if (gp != nullptr) gn = __ldg(reinterpret_cast<const float4*>(gp) + lane);
      rc = __ldg(reinterpret_cast<const float4*>(cs + 4 * (lane & 15)));
      rs = __ldg(reinterpret_cast<const float4*>(sn + 4 * (lane & 15)));
    }
    // the query heads h G .. h G + G - 1, the new key and value
    for (int i = threadIdx.x; i < (G + 2) * kHd / 4; i += kCT) {
      const int part = (4 * i) / kHd, e = (4 * i) % kHd;
      const long long w = part < G ? static_cast<long long>(h * G + part) * kHd + e
                                   : static_cast<long long>(a.nq + (part - G) * a.nkv + h) * kHd + e;
      const float4 v = read_tagged4(T.words + qkv_out + w, expect, T.status, limit);
      float* dst = part < G ? s.aq + part * kHd + e : s.akv + (part - G) * kHd + e;
      *reinterpret_cast<float4*>(dst) = v;
    }
    cbar();
    if (warp <= G)
      head_norm_rope(warp < G ? s.aq + warp * kHd : s.akv, (warp < G ? a.qg : a.kg) != nullptr, gn, rc, rs,
                     T.eps, lane);
    asm volatile("cp.async.wait_all;" ::: "memory");
    cbar();
    const float* sk = s.xs;
    const float* sv = s.xs + kAttnChunk * kHd;
    // scores: thread (g, j, quarter) takes 32 of position j's dims (float4 index skewed by lane:
    // conflict-free rows), the quarters meet by two shuffles
    for (int u = threadIdx.x; u < G * kAttnChunk * 4; u += kCT) {
      const int g = u / (kAttnChunk * 4), j = (u >> 2) % kAttnChunk, qt = u & 3;
      const bool valid = j0 + j < j1;
      const float* kr = (j0 + j == pos ? s.akv : sk + j * kHd) + 32 * qt;
      const float* qr = s.aq + g * kHd + 32 * qt;
      float d = 0.0f;
      if (valid) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int f = (e + lane) & 7;
          const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * f);
          const float4 q = *reinterpret_cast<const float4*>(qr + 4 * f);
          d += (q.x * kv.x + q.y * kv.y) + (q.z * kv.z + q.w * kv.w);
        }
      }
      d += __shfl_xor_sync(0xFFFFFFFFu, d, 1);
      d += __shfl_xor_sync(0xFFFFFFFFu, d, 2);
      if (qt == 0 && valid) s.asc[g * kAttnChunk + j] = d * inv_sqrt;
    }
    cbar();
    // per query head: the chunk's largest score and the sum of the exponentials (warp g)
    if (warp < G) {
      const int n = j1 - j0;
      float* sc = s.asc + warp * kAttnChunk;
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[j]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
      float l = 0.0f;
      for (int j = lane; j < n; j += 32) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
      if (lane == 0 && ok) {
        unsigned long long* o = T.words + part_out + (static_cast<long long>(h * G + warp) * a.maxch + c) * (kHd + 2);
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(o), "l"(__float_as_uint(m) | (static_cast<unsigned long long>(tag) << 32)) : "memory");
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(o + 1), "l"(__float_as_uint(l) | (static_cast<unsigned long long>(tag) << 32)) : "memory");
      }
    }
    cbar();
    // the unnormalised outputs: thread (g, dd), four partial sums over the positions
    for (int i = threadIdx.x; i < G * kHd; i += kCT) {
      const int g = i / kHd, dd = i % kHd;
      const float* p = s.asc + g * kAttnChunk;
      const int n = j1 - j0;
      float o4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
      for (int j = 0; j < n; ++j) {
        const float v = j0 + j == pos ? s.akv[kHd + dd] : sv[j * kHd + dd];
        o4[j & 3] += p[j] * v;
      }
      const float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
      if (ok) {
        unsigned long long* dst = T.words + part_out + (static_cast<long long>(h * G + g) * a.maxch + c) * (kHd + 2) + 2 + dd;
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(dst), "l"(__float_as_uint(o) | (static_cast<unsigned long long>(tag) << 32)) : "memory");
      }
    }
    if (c == nch - 1 && ok)   // the new key and value into the caches
      for (int i = threadIdx.x; i < 2 * kHd; i += kCT) {
        float* cache = i < kHd ? a.kc : a.vc;
        cache[(static_cast<long long>(pos) * a.nkv + h) * kHd + (i % kHd)] = s.akv[i];
      }
    cbar();   // xs / aq / akv / asc / ascr are rewritten by the next item
  }
  // the combine: every CTA, once its own items are done, takes a slice of the n_q hd outputs
  // (so a combine never waits on an item queued behind it on the same CTA)
  const int total = a.nq * kHd;
  const int P = (total + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int o0 = min(static_cast<int>(blockIdx.x) * P, total), o1 = min(o0 + P, total);
  if (o1 > o0) {
    attn_combine(T, s, a, nch, part_out, out, tag, limit, ok, o0, o1);
    cbar();   // xs / asc / ascr are rewritten by the next stage
  }
}

// kFeat: bit 0, the step has 4-bit projections; bit 1, decoder stages (norm / SwiGLU inputs, the
// SwiGLU epilogue, attention); bit 2, more than one GPU. A step without them runs an
// instantiation without their code, which measured ~11 % faster than the full kernel on the same
// projections.
constexpr int kFeatG32 = 1, kFeatDecoder = 2, kFeatMulti = 4;

template <int kFeat>
__global__ void __launch_bounds__(kTh, 1) step_kernel(const StepTable* __restrict__ Tp) {
  constexpr bool kG32 = (kFeat & kFeatG32) != 0, kDec = (kFeat & kFeatDecoder) != 0;
  // (the projection-only instantiations keep the several-GPU code: measured 2.7 % faster with it,
  // a register-allocation effect; the decoder ones measured faster without it)
  constexpr bool kMulti = (kFeat & kFeatMulti) != 0 || !kDec;
  __shared__ long long s_delta[kMaxWorld];
  __shared__ float s_Sa;
  __shared__ unsigned int s_seq;
  __shared__ int s_issued;   // items the producer has issued (or given up on)
  __shared__ int s_pos;      // this step's position (attention)
  // the table's scalars and pointers, read from shared memory from here on (the table itself is
  // read for the stages' descriptors and tensor maps)
  __shared__ __align__(16) StepHead sT;
  for (int i = threadIdx.x; i < static_cast<int>(sizeof(StepHead) / 16); i += kTh)
    reinterpret_cast<uint4*>(&sT)[i] = __ldg(reinterpret_cast<const uint4*>(Tp) + i);
  __syncthreads();
  const StepHead& T = sT;
  const SSmem s = carve(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NS = T.ns, SB = T.stage_bytes;
  const int count = T.count;

  for (int i = threadIdx.x; i < count * static_cast<int>(sizeof(SInfo) / 4); i += kTh)
    reinterpret_cast<uint32_t*>(s.info)[i] = __ldg(reinterpret_cast<const uint32_t*>(Tp->info) + i);
  if (threadIdx.x < kMaxWorld) s_delta[threadIdx.x] = threadIdx.x < T.world ? T.delta[threadIdx.x] : 0;
  if (threadIdx.x == 0) {
    s_issued = 0;
    s_seq = *reinterpret_cast<volatile unsigned int*>(T.counters);
    s_pos = T.pos != nullptr ? *reinterpret_cast<volatile int*>(T.pos) : 0;
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
        if (d.fmt == kFmtAttn) continue;   // no weights
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&Tp->map[p])) : "memory");
        int b0, b1;
        cta_tiles(d.N, b0, b1);
        const bool g4 = kG32 && d.fmt == kFmtG32;
        const uint32_t bytes = static_cast<uint32_t>(kTR) * d.cb * (kChunkB + (g4 ? 16u : 0u));
        for (int b = b0; b < b1; ++b)
          for (int cg = 0; cg < d.ngr; ++cg, ++item) {
            const int st = item % NS, use = item / NS;
            if (use == 0 || mbar_wait(smem_addr(s.empty + st), static_cast<uint32_t>((use - 1) & 1), T.status)) {
              const uint32_t fb = smem_addr(s.full + st);
              mbar_arrive_expect_tx(fb, bytes);
              tma_3d(ring_s + st * SB, &Tp->map[p], 0, b * kTR, cg * kCB, fb);
              if (g4) tma_2d(ring_s + st * SB + kCodeStage, &Tp->smap[p], cg * kCB * 16, b * kTR, fb);
            }   // else a consumer never released the stage: the item is given up (status set)
            // after the stage's previous use is released: a consumer may now wait on its parity
            *reinterpret_cast<volatile int*>(&s_issued) = item + 1;
          }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ the compute warps
  const int g = lane >> 2, t = lane & 3;
  // the split mode's per-lane offsets of its B fragments within a 1 KB swizzled sub-stage
  uint32_t boff[4];
#pragma unroll
  for (int sg = 0; sg < 4; ++sg) boff[sg] = g * kChunkB + 16 * ((2 * sg + (t >> 1)) ^ g) + 8 * (t & 1);
  const uint32_t full_s = smem_addr(s.full), empty_s = smem_addr(s.empty);
  const uint32_t mNS = 0xFFFFFFFFu / static_cast<uint32_t>(NS) + 1u;   // j / NS = umulhi(j, mNS), j < 2^16
  const uint32_t base = s_seq * kTagStride;
  const uint32_t limit = g_step_wait_limit;
  // the greedy token folded into the head's epilogue when its whole row is computed here
  const bool fused_amax = T.token != nullptr && (!kMulti || T.world == 1 || s.info[count - 1].rep);
  unsigned long long best = 0;   // this thread's largest head key (fused argmax)
  bool ok = true;
  int item_base = 0;             // the CTA's items before projection p

  for (int p = 0; p < count; ++p) {
    const SInfo& d = s.info[p];
    if (kDec && d.fmt == kFmtAttn) {   // the attention of this step's token (its items on some CTAs)
      attn_stage(T, Tp->attn[p], s.info[d.in].out, d.out, s_pos, base + static_cast<uint32_t>(d.in + 1),
                 base + static_cast<uint32_t>(p + 1), limit, ok);
      continue;
    }
    const int K = d.K, N = d.N;
    int b0, b1;
    cta_tiles(N, b0, b1);
    const bool norm = kDec && d.input == kInNorm;
    // no rows here: this CTA neither reads the input nor computes -- but every CTA keeps its
    // copy of the residual row, so a norm's input is read all the same
    if (b0 == b1 && !norm) continue;
    const bool g32 = kG32 && d.fmt == kFmtG32;
    const bool unit = d.srows == nullptr;
    // the row scales of this CTA's rows: they never depend on the input, so they are copied
    // asynchronously while it is awaited (complete, and visible to every thread, once the
    // quantization's last barrier has passed)
    const int row0 = b0 * kTR, nrows = min(b1 * kTR, N) - row0;
    if (!g32) {
      const uint32_t sws_s = smem_addr(s.sws);
      for (int i = threadIdx.x; i < nrows; i += kCT) {
        if (unit) s.sws[i] = 1.0f;
        else cp_async4(sws_s + 4u * static_cast<uint32_t>(i), d.srows + static_cast<long long>(row0 + i) * d.srs);
      }
    }
    // ---- the input row: x0, a projection's output words, or a decoder prologue into xs
    const float* xsrc = T.x0;
    const unsigned long long* xt = nullptr;
    uint32_t expect = 0;
    if (!kDec || d.input == kInDefault || d.input == kInAttn) {   // kInAttn: the attention's combined row
      if (d.in >= 0) {
        xt = T.words + s.info[d.in].out;
        expect = base + static_cast<uint32_t>(d.in + 1);
      }
    } else {
      if (norm) {
        norm_prologue(T, s, d, d.res >= 0 ? s.info[d.res].out : 0, base + static_cast<uint32_t>(d.res + 1), limit);
      } else if (d.input == kInSwiglu) {
        swiglu_prologue(T, s, K, s.info[d.in].out, base + static_cast<uint32_t>(d.in + 1), limit);
      }
      xsrc = nullptr;   // the row is in xs
      if (b0 == b1) continue;
    }
    float Sa = 0.0f;
    if (g32) {
      stage_limbs(xsrc, xt, expect, K, s.xs, s.xsum, reinterpret_cast<int*>(s.act), T.status, limit);
    } else {
      qact_row4<kCT, 1, true>(
          xsrc, true, s.xs, K, false, s.segm, s.qred,
          [&](int i, int q0, int q1, int q2, int q3, int da) {
            const int G = i >> 3;
            if ((threadIdx.x & 7) == 0) s.dg[G] = static_cast<uint8_t>(da);
            *reinterpret_cast<uint32_t*>(s.act + 4 * i) =
                (q0 & 0xFFu) | ((q1 & 0xFFu) << 8) | ((q2 & 0xFFu) << 16) | (static_cast<uint32_t>(q3 & 0xFF) << 24);
          },
          xt, expect, T.status, &s_Sa, limit);
      Sa = s_Sa;
    }
    const uint32_t tag = base + static_cast<uint32_t>(p + 1);
    // OTQ_EPI_SWIGLU: rows 16j .. 16j + 7 gate, 16j + 8 .. 16j + 15 up; output word 8j + r is
    // silu(gate) * up of tile rows r and r + 8 (the formula of the SwiGLU prologue)
    const bool swi = kDec && d.epi == kEpiSwiglu;
    const bool rep = kMulti && d.rep;   // every rank computes all rows: stores stay here
    const int rank_off = rep ? 0 : T.rank * (swi ? N / 2 : N);
    unsigned long long* const yw = T.words + d.out + rank_off;
    auto swiglu = [](float gv, float uv) { return (gv / (1.0f + expf(-gv))) * uv; };
    const bool last = p == count - 1;

    auto store_row = [&](int row, float y) {
      if (ok) st_word(yw + row, __float_as_uint(y) | (static_cast<unsigned long long>(tag) << 32), (kMulti && !rep) ? T.world : 1, T.rank, s_delta);
      if (fused_amax && last) {
        const unsigned long long k = amax_key(y, static_cast<uint32_t>(rank_off + row));
        best = k > best ? k : best;
      }
    };
    // ---- the MMA phase over this CTA's tiles [b0, b1): an item is a tile's cb chunks, one 2 KB
    // swizzled sub-stage (16 rows x 128 bytes) a chunk. The projection's it-th item is the CTA's
    // (item_base + it)-th: its stage and parity follow from the running count.
    const int nt = b1 - b0, ngr = d.ngr, cbn = d.cb, kch = d.kch;
    const uint32_t bslot = static_cast<uint32_t>(item_base % NS), bph = static_cast<uint32_t>(item_base / NS) & 1u;
    auto stage_of = [&](int it, uint32_t& par) -> uint32_t {
      const uint32_t j = bslot + static_cast<uint32_t>(it);
      const uint32_t q = __umulhi(j, mNS);
      par = bph ^ (q & 1u);
      return j - q * static_cast<uint32_t>(NS);
    };
    // A stage's full barrier is waited on by parity, which cannot tell its current use from the
    // one before: so first wait (bounded) until the producer has issued the item, i.e. until the
    // stage's previous use has been released (a warp may reach an item before the warps that
    // read the stage's previous item are done with it).
    auto wait_item = [&](int it, uint32_t sl, uint32_t par) {
      for (uint32_t i = 0; *reinterpret_cast<volatile int*>(&s_issued) <= item_base + it; ++i) {
        if (i >= kSpinLimit) {
          atomicOr(T.status, kStatusTimeout);
          ok = false;
          break;
        }
        if (i >= 16) __nanosleep(32);
      }
      const uint32_t fb = full_s + 8u * sl;
      if (!mbar_try_wait(fb, par) && !mbar_wait(fb, par, T.status)) ok = false;
    };
    // int8: the B fragment of group G is its activation bytes (k slots permuted alike in A and B:
    // bytes 8t .. 8t + 7 of the group in lane t) in column (offset & 7) of accumulator set
    // offset >> 3: the A fragment (the weights: rows g and g + 8 of the tile) is then multiplied
    // by 2^(16 - offset) per column, exactly in int32 per set. Offsets above 16 are dropped (the
    // product shifts out of the 16-bit window); offset 16 is set 2, column 0.
    // int8 chunk k of a tile (sub: its sub-stage) into the accumulators; set 0 alternates between
    // two accumulators for a shorter dependence chain
    auto mma_chunk = [&](uint32_t sub, int k, int (&Da)[4], int (&Db)[4], int (&D1)[4], int (&D2)[4]) {
      // every load of the chunk first (the four groups' offsets in one word), then the MMAs: all
      // into set 0 when every offset is below 8 (the usual case), else each group's mma
      // predicated on its set (no branch between the loads and the MMAs)
      const uint32_t c4 = *reinterpret_cast<const uint32_t*>(s.dg + 4 * k);
      uint2 qv[4], r0v[4], r1v[4];
#pragma unroll
      for (int sg = 0; sg < 4; ++sg) {
        qv[sg] = *reinterpret_cast<const uint2*>(s.act + 32 * (4 * k + sg) + 8 * t);
        r0v[sg] = lds64(sub + boff[sg]);
        r1v[sg] = lds64(sub + 1024u + boff[sg]);
      }
      if ((c4 & 0xF8F8F8F8u) == 0u) {
#pragma unroll
        for (int sg = 0; sg < 4; ++sg) {
          const bool on = static_cast<int>((c4 >> (8 * sg)) & 7u) == g;
          const uint32_t bv0 = on ? qv[sg].x : 0u, bv1 = on ? qv[sg].y : 0u;
          if (sg & 1) imma_acc(r0v[sg].x, r1v[sg].x, r0v[sg].y, r1v[sg].y, bv0, bv1, Db);
          else imma_acc(r0v[sg].x, r1v[sg].x, r0v[sg].y, r1v[sg].y, bv0, bv1, Da);
        }
      } else {
#pragma unroll
        for (int sg = 0; sg < 4; ++sg) {
          const uint32_t c = (c4 >> (8 * sg)) & 0xFFu;
          const bool on = static_cast<int>(c & 7u) == g;
          const uint32_t bv0 = on ? qv[sg].x : 0u, bv1 = on ? qv[sg].y : 0u;
          imma_acc_if(c < 8u, r0v[sg].x, r1v[sg].x, r0v[sg].y, r1v[sg].y, bv0, bv1, Da);
          imma_acc_if(c - 8u < 8u, r0v[sg].x, r1v[sg].x, r0v[sg].y, r1v[sg].y, bv0, bv1, D1);
          imma_acc_if(c == 16u, r0v[sg].x, r1v[sg].x, r0v[sg].y, r1v[sg].y, bv0, bv1, D2);
        }
      }
    };
    auto mma_chunk2 = [&](uint32_t subA, uint32_t subB, int k, int (&Da)[4], int (&Db)[4], int (&D1)[4], int (&D2)[4],
                          int (&Ea)[4], int (&Eb)[4], int (&E1)[4], int (&E2)[4]) {
      const uint32_t c4 = *reinterpret_cast<const uint32_t*>(s.dg + 4 * k);
      const bool low = (c4 & 0xF8F8F8F8u) == 0u;
#pragma unroll
      for (int h = 0; h < 2; ++h) {   // two groups' loads at a time
        uint2 qv[2], r0v[2], r1v[2], q0v[2], q1v[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int sg = 2 * h + u;
          qv[u] = *reinterpret_cast<const uint2*>(s.act + 32 * (4 * k + sg) + 8 * t);
          r0v[u] = lds64(subA + boff[sg]);
          r1v[u] = lds64(subA + 1024u + boff[sg]);
          q0v[u] = lds64(subB + boff[sg]);
          q1v[u] = lds64(subB + 1024u + boff[sg]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int sg = 2 * h + u;
          const uint32_t c = (c4 >> (8 * sg)) & 0xFFu;
          const bool on = static_cast<int>(c & 7u) == g;
          const uint32_t bv0 = on ? qv[u].x : 0u, bv1 = on ? qv[u].y : 0u;
          const uint2 r0 = r0v[u], r1 = r1v[u], q0 = q0v[u], q1 = q1v[u];
          if (low) {
            if (u) {
              imma_acc(r0.x, r1.x, r0.y, r1.y, bv0, bv1, Db);
              imma_acc(q0.x, q1.x, q0.y, q1.y, bv0, bv1, Eb);
            } else {
              imma_acc(r0.x, r1.x, r0.y, r1.y, bv0, bv1, Da);
              imma_acc(q0.x, q1.x, q0.y, q1.y, bv0, bv1, Ea);
            }
          } else {
            imma_acc_if(c < 8u, r0.x, r1.x, r0.y, r1.y, bv0, bv1, Da);
            imma_acc_if(c < 8u, q0.x, q1.x, q0.y, q1.y, bv0, bv1, Ea);
            imma_acc_if(c - 8u < 8u, r0.x, r1.x, r0.y, r1.y, bv0, bv1, D1);
            imma_acc_if(c - 8u < 8u, q0.x, q1.x, q0.y, q1.y, bv0, bv1, E1);
            imma_acc_if(c == 16u, r0.x, r1.x, r0.y, r1.y, bv0, bv1, D2);
            imma_acc_if(c == 16u, q0.x, q1.x, q0.y, q1.y, bv0, bv1, E2);
          }
        }
      }
    };

    // a tile's exact row totals: rows g (rg) and g + 8 (rg8), complete in lane t = 0 of the quad
    auto totals = [&](const int (&Da)[4], const int (&Db)[4], const int (&D1)[4], const int (&D2)[4],
                      long long& rg, long long& rg8) {
      const long long m0 = 1ll << (16 - 2 * t), m1 = 1ll << (15 - 2 * t);
      const long long n0 = 1ll << (8 - 2 * t), n1 = 1ll << (7 - 2 * t);
      rg = static_cast<long long>(Da[0] + Db[0]) * m0 + static_cast<long long>(Da[1] + Db[1]) * m1 +
           static_cast<long long>(D1[0]) * n0 + static_cast<long long>(D1[1]) * n1 + (t == 0 ? static_cast<long long>(D2[0]) : 0ll);
      rg8 = static_cast<long long>(Da[2] + Db[2]) * m0 + static_cast<long long>(Da[3] + Db[3]) * m1 +
            static_cast<long long>(D1[2]) * n0 + static_cast<long long>(D1[3]) * n1 + (t == 0 ? static_cast<long long>(D2[2]) : 0ll);
      rg += __shfl_xor_sync(0xFFFFFFFFu, rg, 1);
      rg8 += __shfl_xor_sync(0xFFFFFFFFu, rg8, 1);
      rg += __shfl_xor_sync(0xFFFFFFFFu, rg, 2);
      rg8 += __shfl_xor_sync(0xFFFFFFFFu, rg8, 2);
    };
    // 4-bit chunk k (8 groups) of the tile's rows g (into fg) and g + 8 (fg8): per group one
    // mma.sync m16n8k32 (codes + 8 as u8 x the limbs of xs) gives the 16 rows' four exact limb
    // sums; lane t < 2 adds s 2^-e (D_2t + 256 D_2t+1 - corr) 2^16t, so the quad's sum is the row's
    // sum_k w x for the group (stage_limbs). Code pieces: piece q of row r at (q ^ r % 8) 16.
    auto chunk4x2 = [&](uint32_t stg, int jj, int k, float& fg, float& fg8) {
      const uint8_t* const st = s.ring + (stg - ring_s) + jj * kSub;
      const uint8_t* const scb = s.ring + (stg - ring_s) + kCodeStage + g * (16 * cbn) + jj * 16;
      const uint16_t* const sc0p = reinterpret_cast<const uint16_t*>(scb);
      const uint16_t* const sc1p = reinterpret_cast<const uint16_t*>(scb + 8 * (16 * cbn));
      const uint8_t* const xl = reinterpret_cast<const uint8_t*>(s.xs) + k * 1024 + g * 32 + 4 * t;
      const int* const cr = reinterpret_cast<const int*>(s.act) + k * 16 + (t & 1);
      const float* const xf = s.xsum + k * 8;
      const float wt = t == 0 ? 1.0f : (t == 1 ? 65536.0f : 0.0f);
#pragma unroll 2
      for (int q = 0; q < 8; ++q) {
        const uint8_t* const ap = st + g * kChunkB + ((q ^ g) * 16) + 4 * t;
        const uint32_t wa = *reinterpret_cast<const uint32_t*>(ap);
        const uint32_t wb = *reinterpret_cast<const uint32_t*>(ap + 8 * kChunkB);
        uint32_t a0, a1, a2, a3;
        int4_bytes(wa, a0, a2);
        int4_bytes(wb, a1, a3);
        uint32_t b0 = 0u, b1 = 0u;   // columns 4-7 stay zero
        if (g < 4) {
          b0 = *reinterpret_cast<const uint32_t*>(xl + q * 128);
          b1 = *reinterpret_cast<const uint32_t*>(xl + q * 128 + 16);
        }
        int dd[4];
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};"
            : "=r"(dd[0]), "=r"(dd[1]), "=r"(dd[2]), "=r"(dd[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
        const int cq = cr[q * 2];
        const float fw = __fmul_rn(xf[q], wt);
        const float sc0 = half_to_float(sc0p[q]), sc1 = half_to_float(sc1p[q]);
        fg = fmaf(__fmul_rn(sc0, fw), static_cast<float>(dd[0] + 256 * dd[1] - cq), fg);
        fg8 = fmaf(__fmul_rn(sc1, fw), static_cast<float>(dd[2] + 256 * dd[3] - cq), fg8);
      }
    };
    auto quad_sum = [&](float& f) {
      f += __shfl_xor_sync(0xFFFFFFFFu, f, 1);
      f += __shfl_xor_sync(0xFFFFFFFFu, f, 2);
    };
    auto emit_rows = [&](int tile, long long rg, long long rg8, float fg, float fg8) {   // lane t = 0
      for (int h = 0; h < 2; ++h) {
        const int row = (b0 + tile) * kTR + g + 8 * h;
        if (row >= N) continue;
        store_row(row, g32 ? (h ? fg8 : fg) : mm_epilogue(h ? rg8 : rg, s.sws[row - row0], Sa, 16));
      }
    };

    if (nt < kCW) {
      // ---- few tiles: the S = 8 / TP warps of tile w % TP share its chunks (slice w / TP takes
      // chunks j = slice mod S of every item), and their row totals meet in shared memory
      const int TP = nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : 8;
      const int S = kCW / TP, tile = warp % TP, slice = warp / TP;
      if (tile < nt) {
        int Da[4] = {}, Db[4] = {}, D1[4] = {}, D2[4] = {};
        float fg = 0.0f, fg8 = 0.0f;
        for (int cg = 0; cg < ngr; ++cg) {
          const int it = tile * ngr + cg;
          uint32_t par;
          const uint32_t sl = stage_of(it, par);
          wait_item(it, sl, par);
          const uint32_t stg = ring_s + sl * static_cast<uint32_t>(SB);
          if (ok)
            for (int jj = slice; jj < cbn; jj += S) {
              const int k = cg * kCB + jj;
              if (k >= kch) break;
              if (g32) chunk4x2(stg, jj, k, fg, fg8);
              else mma_chunk(stg + static_cast<uint32_t>(jj * kSub), k, Da, Db, D1, D2);
            }
          __syncwarp();
          if (lane == 0) mbar_arrive_n(empty_s + 8u * sl, static_cast<uint32_t>(kCW / S));
        }
        long long* red = s.red + warp * kTR;
        if (g32) {
          quad_sum(fg);
          quad_sum(fg8);
          if (t == 0) {
            reinterpret_cast<float*>(red)[g] = fg;
            reinterpret_cast<float*>(red)[g + 8] = fg8;
          }
        } else {
          long long rg, rg8;
          totals(Da, Db, D1, D2, rg, rg8);
          if (t == 0) {
            red[g] = rg;
            red[g + 8] = rg8;
          }
        }
      }
      cbar();
      auto row_value = [&](int tl, int r) -> float {   // tile tl's row r: the slices' sum
        if (g32) {
          float f = 0.0f;
          for (int sl2 = 0; sl2 < S; ++sl2) f += reinterpret_cast<const float*>(s.red + (sl2 * TP + tl) * kTR)[r];
          return f;
        }
        long long tot = 0;
        for (int sl2 = 0; sl2 < S; ++sl2) tot += s.red[(sl2 * TP + tl) * kTR + r];
        return mm_epilogue(tot, s.sws[(b0 + tl) * kTR + r - row0], Sa, 16);
      };
      if (swi) {
        for (int i = threadIdx.x; i < nt * 8; i += kCT) {
          const int tl = i >> 3, r = i & 7;
          store_row((b0 + tl) * 8 + r, swiglu(row_value(tl, r), row_value(tl, r + 8)));
        }
      } else {
        for (int i = threadIdx.x; i < nt * kTR; i += kCT) {
          const int tl = i / kTR, r = i % kTR;
          const int row = (b0 + tl) * kTR + r;
          if (row >= N) continue;
          store_row(row, row_value(tl, r));
        }
      }
    } else if (!g32 && 2 * ngr < NS) {
      // ---- many tiles (int8): warp w owns tiles 2w, 2w + 1 of each round of 16, both at once (a
      // warp holds an item while it waits for one ngr further on: ngr < NS keeps that wait
      // satisfiable)
      for (int ta = 2 * warp; ta < nt; ta += 2 * kCW) {
        const int tb = ta + 1;
        const bool two = tb < nt;
        int Da[4] = {}, Db[4] = {}, D1[4] = {}, D2[4] = {};
        int Ea[4] = {}, Eb[4] = {}, E1[4] = {}, E2[4] = {};
        for (int cg = 0; cg < ngr; ++cg) {
          uint32_t pa, pb = 0;
          const uint32_t sa = stage_of(ta * ngr + cg, pa);
          const uint32_t sb = two ? stage_of(tb * ngr + cg, pb) : sa;
          wait_item(ta * ngr + cg, sa, pa);
          if (two) wait_item(tb * ngr + cg, sb, pb);
          const uint32_t stga = ring_s + sa * static_cast<uint32_t>(SB), stgb = ring_s + sb * static_cast<uint32_t>(SB);
          if (ok)
            for (int jj = 0; jj < cbn; ++jj) {
              const int k = cg * kCB + jj;
              if (k >= kch) break;
              if (two) {
                mma_chunk2(stga + static_cast<uint32_t>(jj * kSub), stgb + static_cast<uint32_t>(jj * kSub), k,
                           Da, Db, D1, D2, Ea, Eb, E1, E2);
              } else {
                mma_chunk(stga + static_cast<uint32_t>(jj * kSub), k, Da, Db, D1, D2);
              }
            }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_n(empty_s + 8u * sa, kCW);
            if (two) mbar_arrive_n(empty_s + 8u * sb, kCW);
          }
        }
        long long rg, rg8, qg, qg8;
        totals(Da, Db, D1, D2, rg, rg8);
        totals(Ea, Eb, E1, E2, qg, qg8);
        if (t == 0) {
          emit_rows(ta, rg, rg8, 0.0f, 0.0f);
          if (two) emit_rows(tb, qg, qg8, 0.0f, 0.0f);
        }
      }
    } else {
      // ---- many tiles, long rows: one tile at a time
      for (int ta = warp; ta < nt; ta += kCW) {
        int Da[4] = {}, Db[4] = {}, D1[4] = {}, D2[4] = {};
        float fa = 0.0f, fa8 = 0.0f;
        for (int cg = 0; cg < ngr; ++cg) {
          uint32_t pa;
          const uint32_t sa = stage_of(ta * ngr + cg, pa);
          wait_item(ta * ngr + cg, sa, pa);
          const uint32_t stga = ring_s + sa * static_cast<uint32_t>(SB);
          if (ok)
            for (int jj = 0; jj < cbn; ++jj) {
              const int k = cg * kCB + jj;
              if (k >= kch) break;
              if (g32) chunk4x2(stga, jj, k, fa, fa8);
              else mma_chunk(stga + static_cast<uint32_t>(jj * kSub), k, Da, Db, D1, D2);
            }
          __syncwarp();
          if (lane == 0) mbar_arrive_n(empty_s + 8u * sa, kCW);
        }
        long long rg = 0, rg8 = 0;
        if (g32) {
          quad_sum(fa);
          quad_sum(fa8);
        } else {
          totals(Da, Db, D1, D2, rg, rg8);
        }
        if (t == 0) emit_rows(ta, rg, rg8, fa, fa8);
      }
    }
    item_base += (b1 - b0) * d.ngr;
    cbar();   // act / cls / xs / sws are rewritten by the next projection
  }

  // ---- the greedy token
  if (T.token != nullptr) {
    if (kMulti && !fused_amax) {
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
      if (T.pos != nullptr) *T.pos = s_pos + 1;
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
  const cuuint32_t box[3] = {kChunkB, kTR, static_cast<cuuint32_t>(cb)};
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
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(16 * cb), kTR};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(sc), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Layout {
  int kmax, redb, maxrows, hmax, ascr, stage_bytes, ns;
  size_t smem;
};

// The shared-memory layout of a step (computed alike at prepare and at launch).
int step_layout_of(const otq_step* st, int sms, Layout* L) {
  int kmax = 128, redb = 1, maxrows = 8, hmax = 0, ascr = 0;
  bool any4 = false;
  for (int i = 0; i < st->count; ++i) {
    const otq_step_proj& q = st->projs[i];
    if (q.fmt == OTQ_STEP_ATTN) {
      const int maxch = (st->max_pos + kAttnChunk - 1) / kAttnChunk;
      const int G = q.n_kv > 0 ? q.n_q / q.n_kv : 0;
      ascr = ascr > 2 * G * maxch ? ascr : 2 * G * maxch;
      continue;
    }
    if (q.input == OTQ_IN_NORM) hmax = hmax > q.K ? hmax : static_cast<int>(q.K);
    const int nb = static_cast<int>((q.N + kTR - 1) / kTR);
    const int per_cta = (nb + sms - 1) / sms;
    // the SwiGLU epilogue is written where a CTA's warps share its tiles (fewer than 8 a CTA)
    if (q.epilogue == OTQ_EPI_SWIGLU && per_cta >= kCW) return kErrArg;
    kmax = kmax > q.K ? kmax : static_cast<int>(q.K);
    maxrows = maxrows > per_cta * kTR ? maxrows : per_cta * kTR;
    any4 = any4 || q.fmt == OTQ_STEP_G32;
  }
  // the fixed regions' capacities
  if (kmax > kKcap || hmax > kHcap || maxrows > kRowsCap || ascr > kAscrCap) return kErrArg;
  L->kmax = kmax;
  L->redb = redb;
  L->maxrows = maxrows;
  L->hmax = hmax;
  L->ascr = ascr;
  L->stage_bytes = kCodeStage + (any4 ? kScaleStage : 0);
  const size_t budget = 227 * 1024 - 512;   // dynamic + the kernel's static shared memory
  const size_t fixed = kOffRing + 1024;     // + the ring's alignment
  if (fixed + 4 * static_cast<size_t>(L->stage_bytes) > budget) return kErrArg;
  int ns = static_cast<int>((budget - fixed) / L->stage_bytes);
  ns = ns < kNScap ? ns : kNScap;
  L->ns = ns;
  L->smem = fixed + static_cast<size_t>(ns) * L->stage_bytes;
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
    // an attention stage's partial results stay on each rank (every rank computes them)
    const int64_t n = pr[i].fmt == OTQ_STEP_ATTN ? pr[i].N
                      : (pr[i].epilogue == OTQ_EPI_SWIGLU ? pr[i].N / 2 : pr[i].N) *
                            (pr[i].replicated ? 1 : world);
    off += ((n + 1) / 2) * 2;
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
    if (q.fmt == OTQ_STEP_ATTN) {
      d.fmt = q.fmt;
      d.in = q.in;
      d.N = static_cast<int>(q.N);
      d.out = static_cast<int>(offs[i]);
      SAttn& a = T.attn[i];
      a.qg = q.q_gain;
      a.kg = q.k_gain;
      a.kc = q.kcache;
      a.vc = q.vcache;
      a.nq = q.n_q;
      a.nkv = q.n_kv;
      a.maxch = (st->max_pos + kAttnChunk - 1) / kAttnChunk;
      continue;
    }
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
    d.input = q.input;
    d.res = q.res;
    d.gamma = q.gamma;
    d.out = static_cast<int>(offs[i]);
    d.epi = q.epilogue;
    d.rep = st->world > 1 && q.replicated ? 1 : 0;
    d.nfull = static_cast<int>((q.epilogue == OTQ_EPI_SWIGLU ? q.N / 2 : q.N) * (d.rep ? 1 : st->world));
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
  T.eps = st->eps;
  T.max_pos = st->max_pos;
  T.rope_cos = st->rope_cos;
  T.rope_sin = st->rope_sin;
  T.pos = st->pos;
  T.embed = st->embed;
  T.token_in = reinterpret_cast<const long long*>(st->token_in);
  T.hmax = L.hmax;
  T.ascr = L.ascr;
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
  int feat = st->embed != nullptr ? kFeatDecoder : 0;
  for (int i = 0; i < st->count; ++i) {
    const otq_step_proj& q = st->projs[i];
    if (q.fmt == OTQ_STEP_G32) feat |= kFeatG32;
    if (q.fmt == OTQ_STEP_ATTN || q.input != OTQ_IN_DEFAULT || q.epilogue != OTQ_EPI_NONE) feat |= kFeatDecoder;
  }
  if (st->world > 1) feat |= kFeatMulti;
  const void* const kernels[8] = {
      reinterpret_cast<const void*>(step_kernel<0>), reinterpret_cast<const void*>(step_kernel<1>),
      reinterpret_cast<const void*>(step_kernel<2>), reinterpret_cast<const void*>(step_kernel<3>),
      reinterpret_cast<const void*>(step_kernel<4>), reinterpret_cast<const void*>(step_kernel<5>),
      reinterpret_cast<const void*>(step_kernel<6>), reinterpret_cast<const void*>(step_kernel<7>)};
  const void* kernel = kernels[feat];
  static size_t configured[kMaxDevices][8] = {};
  if (configured[dev][feat] < L.smem) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(L.smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev][feat] = L.smem;
  }
  static int occupancy[kMaxDevices][8] = {};
  if (occupancy[dev][feat] == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kTh, L.smem) != cudaSuccess)
      return kErrCuda;
    if (occ < 1) return kErrArg;   // the step's shared memory does not fit an SM
    occupancy[dev][feat] = occ;
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
  return cudaLaunchKernelExC(&cfg, kernel, args) == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace otq
